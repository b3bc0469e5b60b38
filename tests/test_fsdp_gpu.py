"""Fused sharded AdamW on two GPUs: the reduce-scatter (peer loads), AdamW
and all-gather (peer stores) of ``FusedShardedAdamW`` give exactly the
parameters of the NCCL-based ``ShardedAdamW`` (two-rank sums are
order-free), and the ranks end with identical weights."""
import os
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


def _worker(rank, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from d3d_b200.config import tiny_drafter
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.fsdp import FusedShardedAdamW
    from d3d_b200.train.optim import ShardedAdamW
    dev = torch.device("cuda", rank)
    try:
        a = build_model(tiny_drafter(), seed=3, dtype=torch.bfloat16, device=dev)
        b = build_model(tiny_drafter(), seed=3, dtype=torch.bfloat16, device=dev)
        oa = ShardedAdamW(a.parameters(), lr=1e-3, weight_decay=0.01, align=4)
        ob = FusedShardedAdamW(b.parameters(), lr=1e-3, weight_decay=0.01)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        norms = []
        for step in range(3):
            for pa, pb in zip(a.parameters(), b.parameters()):
                gr = (torch.randn(pa.shape, generator=g, device=dev) * 0.1).to(pa.dtype)
                pa.grad, pb.grad = gr.clone(), gr.clone()
            na = oa.step(grad_clip=0.0)
            nb = ob.step(grad_clip=0.0)
            norms.append((na, nb))
        same = all(torch.equal(pa, pb) for pa, pb in zip(a.parameters(), b.parameters()))
        master_same = torch.equal(oa.master, ob.master)
        flat = torch.cat([p.detach().reshape(-1).float() for p in b.parameters()])
        other = [torch.empty_like(flat) for _ in range(2)]
        dist.all_gather(other, flat)
        ranks_agree = torch.equal(other[0], other[1])
        status = int(ob.status.item())
        ob.close()
        if rank == 0:
            torch.save({"same": same, "master_same": master_same, "ranks_agree": ranks_agree,
                        "status": status, "norms": norms}, out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_sharded_adamw_matches_nccl_path():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        mp.spawn(_worker, args=(_free_port(), out), nprocs=2, join=True)
        r = torch.load(out)
    assert r["status"] == 0
    assert r["master_same"] and r["same"] and r["ranks_agree"]
    for na, nb in r["norms"]:
        assert abs(na - nb) <= 1e-4 * max(1.0, na)
