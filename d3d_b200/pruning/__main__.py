"""``python -m d3d_b200.pruning {select,prune,train,choose}`` — one stage of
progressive pruning (reference: ``scripts/prune.sh``).

    select  --checkpoint DIR --output selection.json [--drop 1]
            (data-parallel under torch.distributed.run: one process per device)
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


class DataWindow:
    """Recovery data: a seeded permutation of a JSONL file's rows read as a
    sliding window from a cursor (no wrap-around: an exhausted window returns
    nothing), or fresh synthetic sequences (``pruning/data.py:52-98``)."""

    def __init__(self, path: str, seed: int, vocab: int, seq_len: int = 128):
        self.synthetic = path == "synthetic"
        self.vocab, self.seq_len = vocab, seq_len
        self.rng = random.Random(seed)
        if not self.synthetic:
            from ..train.data import JsonlIndex
            self.index = JsonlIndex(path)            # byte offsets; rows parsed when taken
            self.perm = list(range(len(self.index)))
            random.Random(seed).shuffle(self.perm)

    def take(self, start: int, n: int):
        if self.synthetic:
            return synthetic_examples(n, self.seq_len, 0.25, self.vocab, random.Random(self.rng.random() + start))
        from ..train.data import encode_row
        out = []
        for i in self.perm[start:start + n]:
            ex = encode_row(self.index.row(i))
            if ex is not None:
                out.append(ex)
        return out


def _agree(ok: bool, device) -> bool:
    """Every rank continues only if every rank has data for this step (MIN
    all-reduce before any collective of the step; ``pruning/train_recovery.py:157-190``)."""
    import torch.distributed as dist
    if not dist.is_initialized():
        return ok
    t = torch.tensor([1 if ok else 0], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def _eval_device(a):
    """Rank and device of an evaluation stage: under ``torch.distributed.run``
    one process per device (``LOCAL_RANK``), examples sharded across ranks."""
    import os
    from ..train.trainer import _init_dist
    device = torch.device(a.device)
    rank, _ = _init_dist(device.type)
    if device.type == "cuda":
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(device)
    return rank, device


def _recovery(a) -> list:
    """Recovery training of a pruned child against its parent: multi-rank
    under ``torch.distributed.run`` (sharded optimizer), agreed stop when any
    rank runs out of data, atomic step checkpoints carrying the next data
    cursor (``pruning/train_recovery.py:39-534``)."""
    import os
    from ..train.blocks import build_packed_block_batch
    from ..train.trainer import _init_dist
    device = torch.device(a.device)
    rank, world = _init_dist(device.type)
    if device.type == "cuda":
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(device)
    parent = load_model(a.parent, device=device).eval()
    for q in parent.parameters():
        q.requires_grad_(False)
    child = load_model(a.child, device=device)
    prov = json.loads((Path(a.child) / "layer_prune.json").read_text())
    child.model.embed_tokens.weight.requires_grad_(False)
    z3 = None
    if getattr(a, "fsdp", False):
        # the child's decoder layers as per-rank shards (the reference's FSDP2 student)
        from ..parallel.zero3 import Zero3Layers
        z3 = Zero3Layers(child.model.layers, lr=a.lr)
    opt = ShardedAdamW(child.parameters(), lr=a.lr)
    rng = random.Random(a.seed * 1000 + rank)
    window = DataWindow(a.data_path, a.seed, min(child.cfg.vocab_size, 151643) - 2)
    cursor = a.data_cursor
    out = Path(a.output)

    def save(dst: Path, log):
        extra = z3.full_state("model.layers.") if z3 is not None else None   # collective
        if rank == 0:
            save_model(child, dst, extra=extra)
            (dst / "layer_prune.json").write_text(json.dumps(prov, indent=2))
            write_json(str(dst / "recovery_log.json"), log)
            write_json(str(dst / "trainer_state.json"), {"next_data_cursor": cursor, "steps": len(log)})

    log = []
    for step in range(a.steps):
        exs = window.take(cursor + rank * a.batch_size, a.batch_size)
        ok = len(exs) > 0 and build_packed_block_batch(exs, block_size=a.block_size, mask_token_id=int(
            child.cfg.mask_token_id), max_anchors=8, rng=random.Random(0)) is not None
        if not _agree(ok, device):
            break
        cursor += world * a.batch_size
        rec = recovery_step(child, parent, prov["removed_compact_layer"], list(range(parent.cfg.num_hidden_layers)),
                            exs, opt, block_size=a.block_size, anchors=8, rng=rng, z3=z3)
        rec["next_data_cursor"] = cursor
        log.append(rec)
        if a.save_every and (step + 1) % a.save_every == 0:
            save(out.with_name(out.name + f".step{step + 1}"), log)
    save(out, log)
    if z3 is not None:
        z3.close()
    if log and rank == 0:
        print(json.dumps(log[-1]))
    return log


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
    p.add_argument("--data-path", default="synthetic", help="train: synthetic or JSONL of prompt_ids/response_ids")
    p.add_argument("--batch-size", type=int, default=2, help="train: sequences per rank per step")
    p.add_argument("--data-cursor", type=int, default=0, help="train: first row of the permuted data window")
    p.add_argument("--save-every", type=int, default=0, help="train: atomic step checkpoints")
    p.add_argument("--fsdp", action="store_true", help="train: shard the child's decoder layers over the ranks")
    a = p.parse_args(argv)
    if a.stage == "select":
        rank, device = _eval_device(a)
        m = load_model(a.checkpoint, device=device).eval()
        depth = m.cfg.num_hidden_layers
        res = select_layers(m, _eval_examples(m.cfg, a.samples, a.block_size, a.seed), a.block_size, a.drop)
        h = res["history"][0]
        if rank == 0:
            write_selection(Path(a.output), a.checkpoint, depth, h["removed_compact_layer"],
                            [i for i in range(depth) if i != h["removed_compact_layer"]], m.cfg.mask_token_id, res)
            print(json.dumps({"removed": [x["removed_original_layer"] for x in res["history"]]}))
    elif a.stage == "prune":
        print(prune_from_selection(a.selection, a.output))
    elif a.stage == "train":
        _recovery(a)
    else:
        rank, device = _eval_device(a)
        m = load_model(a.checkpoints[0], device="cpu")
        res = choose(a.checkpoints, _eval_examples(m.cfg, a.samples, a.block_size, a.seed), a.block_size, device)
        if rank == 0:
            write_json(a.output, res)
            print(json.dumps(res["best"]))


if __name__ == "__main__":
    main()
