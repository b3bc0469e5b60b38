"""Host-side fault injection on the disaggregated protocol (gloo, CPU): a
target rank that dies mid-stream and a reply that is dropped both surface
as errors on the drafter side within the process-group timeout -- no hang,
no GPU involved."""
import os
import random
import socket
import tempfile
import time

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


def _worker(rank, port, out_path, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=8))
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.backends import TorchDraft, TorchTarget
    from d3d_b200.engine.disagg import CMD_VERIFY, P2PTarget, P2PTargetServer
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.p2p import HostLink

    class Faulty(P2PTargetServer):
        verifies = 0

        def _verify(self, h):
            Faulty.verifies += 1
            if Faulty.verifies == 2:
                if mode == "die":
                    os._exit(0)            # the rank disappears without a word
                return                     # "drop": the reply is never sent
            super()._verify(h)

    link = HostLink(1 - rank, slot_bytes=1 << 16)
    if rank == 0:
        try:
            Faulty(TorchTarget(build_model(tiny_target(), seed=0)), link).serve()
        except Exception:
            pass                           # the peer gave up; this rank only has to end
        os._exit(0)
    t0 = time.monotonic()
    remote = P2PTarget(link, hidden_size=128)
    drafter = TorchDraft(build_model(tiny_drafter(cond=True), seed=1))
    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=24, ignore_eos=True)
    rng = random.Random(3)
    prompt = [[rng.randrange(2, 1000) for _ in range(20)]]
    try:
        SpecDecoder(remote, drafter, cfg).generate(prompt)
        res = "no error"
    except Exception as e:              # gloo reports the closed peer or the timeout
        res = "error:" + type(e).__name__
    torch.save({"result": res, "seconds": time.monotonic() - t0}, out_path)
    os._exit(0)


@pytest.mark.parametrize("mode", ["die", "drop"])
def test_target_failure_surfaces_without_hang(mode):
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        ctx = mp.start_processes(_worker, args=(_free_port(), out, mode), nprocs=2, join=False,
                                 start_method="spawn")
        deadline = time.monotonic() + 120
        while not ctx.join(timeout=5):
            assert time.monotonic() < deadline, "fault test did not finish"
        r = torch.load(out)
    assert r["result"].startswith("error:"), r
    assert r["seconds"] < 60
