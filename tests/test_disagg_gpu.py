"""Disaggregated decode across two GPUs over the NVLink mailboxes: the
target served on cuda:0, drafter + coordinator on cuda:1.  Greedy output
must be token-identical to target-only AR on the same kernels; a bounded
wait that nothing satisfies must return a timeout status (not hang), and the
mailbox stays usable afterwards."""
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
    rng = random.Random(2)
    return [[rng.randrange(2, 1000) for _ in range(rng.randint(16, 96))] for _ in range(3)]


def _worker(rank, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    import faulthandler
    faulthandler.dump_traceback_later(240, exit=True)   # a stuck worker reports where, then exits
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from d3d_b200.api import D3DEngine, open_pair_link, target_server
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.spec import DecodeConfig, ar_generate
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.models.qwen3 import build_model
    dev = torch.device("cuda", rank)
    try:
        link = open_pair_link(1 - rank, dev, slot_bytes=1 << 16)
        # a wait that nothing satisfies runs out and reports a timeout status
        st = torch.cuda.Stream(device=dev)
        timed_out = False
        try:
            link.inbox.wait(1 << 40, None, st, deadline_s=0.0)
        except TimeoutError:
            timed_out = True
        dist.barrier()
        prompts = _prompts()
        cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=48, ignore_eos=True)
        if rank == 0:
            tw = FastWeights.from_module(build_model(tiny_target(), seed=0), dev)
            srv = target_server(tw, link, max_seqs=4, max_context=512, device=dev, deadline_s=60)
            ar = ar_generate(srv.be, prompts, 48, ignore_eos=True)["outputs"]
            dist.broadcast_object_list([ar], src=0)
            srv.serve()
            dist.broadcast_object_list([timed_out], src=0)
        else:
            box = [None]
            dist.broadcast_object_list(box, src=0)
            ar = box[0]
            dw = FastWeights.from_module(build_model(tiny_drafter(cond=True), seed=1), dev)
            eng = D3DEngine.from_remote_target(dw, link, 128, cfg, max_seqs=4, max_context=512, device=dev,
                                               deadline_s=60)
            res = eng.generate(prompts, concurrency=2)
            eng.close()
            other = [None]
            dist.broadcast_object_list(other, src=0)
            torch.save({"spec": [o.tokens for o in res["outputs"]], "ar": ar,
                        "accepts": [o.accepts for o in res["outputs"]],
                        "timed_out": [other[0], timed_out]}, out_path)
        link.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_disaggregated_two_gpus_token_identical():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        mp.spawn(_worker, args=(_free_port(), out), nprocs=2, join=True)
        r = torch.load(out)
    assert r["timed_out"] == [True, True]
    assert r["spec"] == r["ar"]
    assert all(len(t) == 48 for t in r["spec"])
    assert all(sum(a) >= 47 for a in r["accepts"])
