"""Remote draft service adapter: a fake target loop that verifies the
service's proposals greedily must reproduce target-only AR decoding, with
branch reuse across steps; the same over the TCP transport."""
import random
import threading

import torch

from d3d_b200.adapters.sglang import DraftClient, DraftService, serve
from d3d_b200.config import tiny_drafter, tiny_target
from d3d_b200.engine.backends import TorchDraft, TorchTarget
from d3d_b200.engine.spec import ar_generate
from d3d_b200.engine.controlled import ControlledAcceptance
from d3d_b200.models.qwen3 import build_model


def _setup():
    t = build_model(tiny_target(), seed=0)
    d = build_model(tiny_drafter(cond=False), seed=1)
    rng = random.Random(4)
    prompts = [[rng.randrange(2, 1000) for _ in range(rng.randint(12, 30))] for _ in range(3)]
    ar = ar_generate(TorchTarget(t), prompts, 24, ignore_eos=True)["outputs"]
    return t, d, prompts, ar


def _target_next(t, seq):
    with torch.no_grad():
        return t.logits(t(torch.tensor([seq])))[0].argmax(-1).tolist()


def _drive(step, t, prompts, ar, n_new=24):
    outputs = {i: [ar[i][0]] for i in range(len(prompts))}   # first token from the target prefill
    rounds = 0
    while any(len(o) < n_new for o in outputs.values()):
        items = [{"rid": str(i), "prompt": prompts[i], "outputs": outputs[i]}
                 for i in outputs if len(outputs[i]) < n_new]
        props = step(items)
        rounds += 1
        for it in items:
            i = int(it["rid"])
            blk = props[it["rid"]]["tokens"]
            seq = prompts[i] + outputs[i][:-1] + blk
            post = _target_next(t, seq)[len(prompts[i]) + len(outputs[i]) - 1:]
            n = 1
            while n < len(blk) and blk[n] == post[n - 1]:
                n += 1
            outputs[i] += blk[1:n] + [post[n - 1]]
    return {i: o[:n_new] for i, o in outputs.items()}, rounds


def test_draft_service_matches_ar_with_branch_reuse():
    t, d, prompts, ar = _setup()
    svc = DraftService(TorchDraft(d), block_size=8, anchor_num=1)
    def step(items):
        out = svc.step(items)
        svc.speculate()
        return out["proposals"]

    outs, rounds = _drive(step, t, prompts, ar)
    for i in outs:
        assert outs[i] == ar[i]
    m = svc.metrics
    assert m["remote_hit_count"] + m["remote_miss_count"] >= rounds
    assert m["optional_forward_count"] == rounds


def test_draft_service_over_tcp():
    t, d, prompts, ar = _setup()
    svc = DraftService(TorchDraft(d), block_size=8, anchor_num=1)
    ready, bound = threading.Event(), []
    th = threading.Thread(target=serve, args=(svc, "127.0.0.1", 0, ready, bound), daemon=True)
    th.start()
    ready.wait(10)
    cli = DraftClient("127.0.0.1", bound[0])
    outs, _ = _drive(cli.step, t, prompts, ar)
    assert outs == {i: ar[i] for i in range(len(prompts))}
    assert cli.request({"cmd": "metrics"})["optional_forward_count"] > 0
    cli.close()
    th.join(10)
