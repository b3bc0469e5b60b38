"""``python -m d3d_b200.pruning {select,prune,train,choose}`` — one stage of
progressive pruning (reference: ``scripts/prune.sh``).

    select  --checkpoint DIR --output selection.json [--drop 1]
    prune   --selection selection.json --output DIR
    train   --parent DIR --child DIR --output DIR [--steps N]
    choose  --checkpoints DIR [DIR ...] --output best.json
"""
from __future__ import annotations

import argparse
import json
import random
from pathlib import Path

import torch

from ..checkpoint import load_model, save_model
from ..train.blocks import synthetic_examples
from ..train.optim import ShardedAdamW
from ..utils.io import write_json
from .modeling import examples_from_sequences
from .prune import prune_from_selection
from .recovery import recovery_step
from .select_checkpoint import choose
from .select_layer import select_layers, write_selection


def _eval_examples(cfg, n, block, seed):
    rng = random.Random(seed)
    vocab = min(cfg.vocab_size, 151643) - 2
    seqs = [[rng.randrange(vocab) for _ in range(96)] for _ in range(n)]
    return examples_from_sequences(seqs, block, 2, rng)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("stage", choices=["select", "prune", "train", "choose"])
    p.add_argument("--checkpoint")
    p.add_argument("--checkpoints", nargs="*")
    p.add_argument("--selection")
    p.add_argument("--parent")
    p.add_argument("--child")
    p.add_argument("--output", required=True)
    p.add_argument("--drop", type=int, default=1)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--samples", type=int, default=16)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--lr", type=float, default=1e-5)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = p.parse_args(argv)
    if a.stage == "select":
        m = load_model(a.checkpoint, device=a.device).eval()
        depth = m.cfg.num_hidden_layers
        res = select_layers(m, _eval_examples(m.cfg, a.samples, a.block_size, a.seed), a.block_size, a.drop)
        h = res["history"][0]
        write_selection(Path(a.output), a.checkpoint, depth, h["removed_compact_layer"],
                        [i for i in range(depth) if i != h["removed_compact_layer"]], m.cfg.mask_token_id, res)
        print(json.dumps({"removed": [x["removed_original_layer"] for x in res["history"]]}))
    elif a.stage == "prune":
        print(prune_from_selection(a.selection, a.output))
    elif a.stage == "train":
        parent = load_model(a.parent, device=a.device).eval()
        for q in parent.parameters():
            q.requires_grad_(False)
        child = load_model(a.child, device=a.device)
        prov = json.loads((Path(a.child) / "layer_prune.json").read_text())
        child.model.embed_tokens.weight.requires_grad_(False)
        opt = ShardedAdamW(child.parameters(), lr=a.lr)
        rng = random.Random(a.seed)
        vocab = min(child.cfg.vocab_size, 151643) - 2
        log = []
        for _ in range(a.steps):
            exs = synthetic_examples(2, 128, 0.25, vocab, rng)
            log.append(recovery_step(child, parent, prov["removed_compact_layer"],
                                     list(range(parent.cfg.num_hidden_layers)), exs, opt,
                                     block_size=a.block_size, anchors=8, rng=rng))
        save_model(child, a.output)
        (Path(a.output) / "layer_prune.json").write_text(json.dumps(prov, indent=2))
        write_json(str(Path(a.output) / "recovery_log.json"), log)
        print(json.dumps(log[-1]))
    else:
        m = load_model(a.checkpoints[0], device="cpu")
        res = choose(a.checkpoints, _eval_examples(m.cfg, a.samples, a.block_size, a.seed), a.block_size, a.device)
        write_json(a.output, res)
        print(json.dumps(res["best"]))


if __name__ == "__main__":
    main()
