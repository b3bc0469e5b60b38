"""The multi-GPU serving layout on real GPUs: the target on T GPUs
(tensor-parallel when T = 2) serves D drafter GPUs, one request stream each,
through the batched server (merged verifies, per-drafter fused accept+send
replies over NVLink).  Every drafter's greedy output must be token-identical
to target-only AR decoding on the same target GPUs.  With 4+ GPUs: T = 2,
D = 2; with 3: T = 1, D = 2; with 2: T = 1, D = 1."""
import os
import random
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts(d):
    rng = random.Random(20 + d)
    return [[rng.randrange(2, 1000) for _ in range(rng.randint(16, 96))] for _ in range(2)]


def _worker(rank, world, T, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    import faulthandler
    faulthandler.dump_traceback_later(240, exit=True)   # a stuck worker reports where, then exits
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from d3d_b200.api import D3DEngine
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.disagg import BatchedTargetServer
    from d3d_b200.engine.fast import FastTarget
    from d3d_b200.engine.spec import DecodeConfig, ar_generate
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.p2p import Link
    from d3d_b200.parallel.tp import TPGroup, random_shard
    dev = torch.device("cuda", rank)
    D = world - T
    tp_group = dist.new_group(list(range(T)))
    pair = {(t, d): dist.new_group([t, T + d]) for t in range(T) for d in range(D)}
    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=40, ignore_eos=True)
    try:
        if rank < T:
            grp = TPGroup(rank, T, dev, group=tp_group, num_layers=tiny_target().num_hidden_layers) if T > 1 \
                else None
            w = random_shard(tiny_target(), T, rank, seed=0, device=dev) if T > 1 else \
                FastWeights.from_module(build_model(tiny_target(), seed=0), dev)
            links = [Link(1, 1 << 16, dev, group=pair[(rank, d)]) for d in range(D)]
            tgt = FastTarget(w, pages=512, max_seqs=8, max_context=512, device=dev, tp=grp)
            batch = [p for d in range(D) for p in _prompts(d)]
            ar = ar_generate(tgt, batch, 40, ignore_eos=True, concurrency=len(batch))["outputs"]
            box = [ar]
            dist.broadcast_object_list(box, src=0)
            srv = BatchedTargetServer(tgt, links, deadline_s=60, replies="all" if rank == 0 else "ack")
            srv.serve()
            if rank == 0:
                torch.save({"rounds": srv.rounds, "served": srv.served}, os.path.join(out_dir, "srv.pt"))
            for d, lk in enumerate(links):
                lk.close(pair[(rank, d)])
            if grp is not None:
                grp.close()
        else:
            me = rank - T
            # links first: the target ranks build theirs before the broadcast
            links = [Link(0, 1 << 16, dev, group=pair[(t, me)]) for t in range(T)]
            box = [None]
            dist.broadcast_object_list(box, src=0)
            ar = box[0][2 * me:2 * me + 2]
            dw = FastWeights.from_module(build_model(tiny_drafter(cond=True), seed=1), dev)
            eng = D3DEngine.from_remote_target(dw, links, 128, cfg, max_seqs=4, max_context=512, device=dev,
                                               deadline_s=60)
            res = eng.generate(_prompts(me), concurrency=1)
            eng.close()
            torch.save({"spec": [o.tokens for o in res["outputs"]], "ar": ar}, os.path.join(out_dir, f"d{me}.pt"))
            for t, lk in enumerate(links):
                lk.close(pair[(t, me)])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_batched_target_serves_drafter_gpus_token_identical():
    n = torch.cuda.device_count()
    world, T = (4, 2) if n >= 4 else ((3, 1) if n == 3 else (2, 1))
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, T, _free_port(), d), nprocs=world, join=True)
        for me in range(world - T):
            r = torch.load(os.path.join(d, f"d{me}.pt"))
            assert r["spec"] == r["ar"]
            assert all(len(t) == 40 for t in r["spec"])
        srv = torch.load(os.path.join(d, "srv.pt"))
        assert srv["served"] > 0
