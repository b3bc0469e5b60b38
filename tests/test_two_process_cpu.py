"""Draft process <-> target process over gloo on CPU (the tiny pair of the
baseline configuration): greedy speculative output must be token-identical
to target-only AR decoding, with the drafter conditioned on the target's
last-layer hidden state carried by the handoff; server-side failures must
surface as client errors and tear down cleanly."""
import os
import random
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts():
    rng = random.Random(0)
    return [[rng.randrange(2, 1000) for _ in range(rng.randint(16, 64))] for _ in range(4)]


class _FailingTarget:
    """Wraps a target backend and raises on the Nth verify (host-side fault injection)."""

    def __init__(self, inner, fail_at):
        self.inner, self.fail_at, self.n = inner, fail_at, 0
        self.hidden_size = inner.hidden_size

    def prefill(self, seqs):
        return self.inner.prefill(seqs)

    def verify(self, seqs, blocks, q=None):
        self.n += 1
        if self.n == self.fail_at:
            raise RuntimeError("injected target fault")
        return self.inner.verify(seqs, blocks, q)

    def release(self, s):
        self.inner.release(s)


def _worker(rank, port, out_path, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.backends import TorchDraft, TorchTarget
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.serving.remote import RemoteTarget, TargetServer
    try:
        if rank == 0:
            tgt = TorchTarget(build_model(tiny_target(), seed=0))
            if mode == "fault":
                tgt = _FailingTarget(tgt, fail_at=3)
            TargetServer(tgt, client_rank=1).serve()
        else:
            remote = RemoteTarget(0, hidden_size=128)
            drafter = TorchDraft(build_model(tiny_drafter(cond=True), seed=1))
            prompts = _prompts()
            cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=32, ignore_eos=True)
            if mode == "fault":
                try:
                    SpecDecoder(remote, drafter, cfg).generate(prompts)
                    result = "no error"
                except RuntimeError as e:
                    result = "error:" + ("injected target fault" in str(e)) * "injected"
                remote.close()
                torch.save({"result": result}, out_path)
            else:
                spec = SpecDecoder(remote, drafter, cfg).generate(prompts, concurrency=2)
                ar = ar_generate(remote, prompts, 32, ignore_eos=True)
                local_ar = ar_generate(TorchTarget(build_model(tiny_target(), seed=0)), prompts, 32,
                                       ignore_eos=True)
                remote.close()
                torch.save({"spec": [o.tokens for o in spec["outputs"]], "ar": ar["outputs"],
                            "local_ar": local_ar["outputs"],
                            "accepts": [o.accepts for o in spec["outputs"]]}, out_path)
    finally:
        dist.destroy_process_group()


def _run(mode):
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        mp.spawn(_worker, args=(_free_port(), out, mode), nprocs=2, join=True)
        return torch.load(out)


def test_tiny_pair_two_processes_token_identical():
    r = _run("ok")
    assert r["spec"] == r["ar"] == r["local_ar"]
    assert all(len(t) == 32 for t in r["spec"])
    assert all(sum(a) >= 31 for a in r["accepts"])


def test_target_fault_propagates_and_tears_down():
    r = _run("fault")
    assert r["result"] == "error:injected"
