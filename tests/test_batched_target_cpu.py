"""One target serving two drafter ranks (the multi-GPU layout's protocol) on
CPU over the host link: each round merges the drafters' requests into one
batched prefill / verify; every drafter's greedy speculative output must be
token-identical to target-only AR decoding of its own prompts, also when one
drafter finishes early and the other keeps decoding alone."""
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


def _prompts(d):
    rng = random.Random(10 + d)
    return [[rng.randrange(2, 1000) for _ in range(rng.randint(16, 60))] for _ in range(2 + d)]


def _worker(rank, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=3, timeout=datetime.timedelta(seconds=120))
    torch.manual_seed(0)
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.backends import TorchDraft, TorchTarget
    from d3d_b200.engine.disagg import BatchedTargetServer, P2PTarget
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.p2p import HostLink
    try:
        cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=32, ignore_eos=True)
        if rank == 0:
            srv = BatchedTargetServer(TorchTarget(build_model(tiny_target(), seed=0)),
                                      [HostLink(1, 1 << 16), HostLink(2, 1 << 16)])
            srv.serve()
            torch.save({"rounds": srv.rounds, "served": srv.served}, os.path.join(out_dir, "srv.pt"))
        else:
            d = rank - 1
            remote = P2PTarget(HostLink(0, 1 << 16), hidden_size=128)
            drafter = TorchDraft(build_model(tiny_drafter(cond=True), seed=1))
            prompts = _prompts(d)
            out = SpecDecoder(remote, drafter, cfg).generate(prompts)["outputs"]
            remote.close()
            ar = ar_generate(TorchTarget(build_model(tiny_target(), seed=0)), prompts, 32, ignore_eos=True)
            torch.save({"spec": [o.tokens for o in out], "ar": ar["outputs"]}, os.path.join(out_dir, f"d{d}.pt"))
    finally:
        dist.destroy_process_group()


def test_two_drafters_one_target_token_identical():
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_worker, args=(_free_port(), td), nprocs=3, join=True)
        for d in range(2):
            r = torch.load(os.path.join(td, f"d{d}.pt"))
            assert r["spec"] == r["ar"]
            assert all(len(t) == 32 for t in r["spec"])
        srv = torch.load(os.path.join(td, "srv.pt"))
        # merged rounds: fewer rounds than messages served
        assert srv["rounds"] < srv["served"]
