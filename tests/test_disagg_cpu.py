"""Disaggregated decode protocol (target rank <-> drafter rank) over the
host link on CPU: the same messages and server loop as the NVLink mailbox
path, with gloo point-to-point transport.  Greedy speculative output must be
token-identical to target-only AR decoding, server-side failures must reach
the client as errors, and the server must keep serving afterwards."""
import os
import random
import socket
import tempfile

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
    rng = random.Random(1)
    return [[rng.randrange(2, 1000) for _ in range(rng.randint(16, 80))] for _ in range(3)]


class _FailOnce:
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
    from d3d_b200.engine.disagg import P2PTarget, P2PTargetServer
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.p2p import HostLink
    try:
        link = HostLink(1 - rank, slot_bytes=1 << 16)
        if rank == 0:
            tgt = TorchTarget(build_model(tiny_target(), seed=0))
            if mode == "fault":
                tgt = _FailOnce(tgt, fail_at=2)
            P2PTargetServer(tgt, link).serve()
        else:
            remote = P2PTarget(link, hidden_size=128)
            drafter = TorchDraft(build_model(tiny_drafter(cond=True), seed=1))
            cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=40, ignore_eos=True)
            prompts = _prompts()
            res = {}
            if mode == "fault":
                try:
                    SpecDecoder(remote, drafter, cfg).generate(prompts[:1])
                    res["first"] = "no error"
                except RuntimeError as e:
                    res["first"] = "injected" if "injected target fault" in str(e) else str(e)
                # the server survived the failure and still answers
                remote._pending = None
                res["after"] = ar_generate(remote, prompts[1:2], 8, ignore_eos=True)["outputs"]
                res["local"] = ar_generate(TorchTarget(build_model(tiny_target(), seed=0)), prompts[1:2], 8,
                                           ignore_eos=True)["outputs"]
            else:
                spec = SpecDecoder(remote, drafter, cfg).generate(prompts, concurrency=2)
                res["spec"] = [o.tokens for o in spec["outputs"]]
                res["accepts"] = [o.accepts for o in spec["outputs"]]
                res["ar"] = ar_generate(remote, prompts, 40, ignore_eos=True)["outputs"]
                res["local"] = ar_generate(TorchTarget(build_model(tiny_target(), seed=0)), prompts, 40,
                                           ignore_eos=True)["outputs"]
            remote.close()
            torch.save(res, out_path)
    finally:
        dist.destroy_process_group()


def _run(mode):
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        mp.spawn(_worker, args=(_free_port(), out, mode), nprocs=2, join=True)
        return torch.load(out)


def test_disaggregated_protocol_token_identical():
    r = _run("ok")
    assert r["spec"] == r["ar"] == r["local"]
    assert all(len(t) == 40 for t in r["spec"])
    assert all(sum(a) >= 39 for a in r["accepts"])


def test_disaggregated_fault_reported_and_server_survives():
    r = _run("fault")
    assert r["first"] == "injected"
    assert r["after"] == r["local"]


def _worker_group(rank, port, out_path):
    """Ranks 0 and 1 serve as the two ranks of a (simulated) tensor-parallel
    target -- rank 1 acknowledges only RELEASE -- and rank 2 drafts."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=3, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.backends import TorchDraft, TorchTarget
    from d3d_b200.engine.disagg import P2PTarget, P2PTargetServer
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.p2p import HostLink
    try:
        if rank < 2:
            tgt = TorchTarget(build_model(tiny_target(), seed=0))
            P2PTargetServer(tgt, HostLink(2, slot_bytes=1 << 16), replies="all" if rank == 0 else "ack").serve()
        else:
            remote = P2PTarget([HostLink(0, slot_bytes=1 << 16), HostLink(1, slot_bytes=1 << 16)], hidden_size=128)
            drafter = TorchDraft(build_model(tiny_drafter(cond=True), seed=1))
            cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=24, ignore_eos=True)
            prompts = _prompts()
            spec = SpecDecoder(remote, drafter, cfg).generate(prompts, concurrency=2)
            local = ar_generate(TorchTarget(build_model(tiny_target(), seed=0)), prompts, 24, ignore_eos=True)
            remote.close()
            torch.save({"spec": [o.tokens for o in spec["outputs"]], "local": local["outputs"]}, out_path)
    finally:
        dist.destroy_process_group()


def test_target_group_protocol_token_identical():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        mp.spawn(_worker_group, args=(_free_port(), out), nprocs=3, join=True)
        r = torch.load(out)
    assert r["spec"] == r["local"]
