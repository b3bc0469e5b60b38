"""Tensor-parallel target on two GPUs (one process each): the sharded
forward tracks the unsharded one, the exchange kernels report no timeout,
and greedy speculative decoding through the TP target is token-identical to
AR decoding through the same TP target.  The drafter is a CPU copy on each
rank, so both ranks issue identical verify calls (SPMD)."""
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


def _prompts():
    rng = random.Random(5)
    return [[rng.randrange(2, 1000) for _ in range(rng.randint(16, 80))] for _ in range(3)]


def _worker(rank, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.backends import SeqState, TorchDraft
    from d3d_b200.engine.fast import FastTarget
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.tp import TPGroup, shard_weights
    dev = torch.device("cuda", rank)
    try:
        cfg = tiny_target()
        full = FastWeights.from_module(build_model(cfg, seed=0), dev)
        grp = TPGroup(rank, 2, dev, num_layers=cfg.num_hidden_layers)
        tgt = FastTarget(shard_weights(full, 2, rank), pages=512, max_seqs=4, max_context=512, tp=grp)
        ref = FastTarget(full, pages=512, max_seqs=4, max_context=512)
        prompts = _prompts()
        seqs = [SeqState(index=i, prompt=p, prefix=len(p)) for i, p in enumerate(prompts)]
        a_tp, h_tp = tgt.prefill(seqs)
        seqs2 = [SeqState(index=i, prompt=p, prefix=len(p)) for i, p in enumerate(prompts)]
        a_ref, h_ref = ref.prefill(seqs2)
        for s in seqs:
            tgt.release(s)
        for s in seqs2:
            ref.release(s)
        herr = ((h_tp.float() - h_ref.float()).abs().max() / h_ref.float().abs().max()).item()
        ar = ar_generate(tgt, prompts, 40, ignore_eos=True)["outputs"]
        drafter = TorchDraft(build_model(tiny_drafter(), seed=1))
        dcfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=40, ignore_eos=True, use_cond=False)
        spec = SpecDecoder(tgt, drafter, dcfg).generate(prompts, concurrency=2)
        torch.cuda.synchronize()
        status = int(grp.status.item())
        res = {"herr": herr, "anchors_equal": bool(torch.equal(a_tp, a_ref)), "status": status,
               "spec": [o.tokens for o in spec["outputs"]], "ar": ar}
        grp.close()
        if rank == 0:
            torch.save(res, out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_target_matches_and_spec_is_token_identical():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        mp.spawn(_worker, args=(_free_port(), out), nprocs=2, join=True)
        r = torch.load(out)
    assert r["status"] == 0
    assert r["herr"] < 0.05, r["herr"]
    assert r["anchors_equal"]
    assert r["spec"] == r["ar"]
