"""A verifier process for the command-line drivers: the target runs in a
child process on its own device and serves verifies over a pair link, while
the calling process keeps the drafter and the coordinator (the reference's
``VerifierProcessClient`` of ``single/eval_async_packed.py``, with its
``--verifier-device`` / ``--draft-device`` and per-process CPU affinity).

On two GPUs the link is the NVLink mailbox pair (``api.open_pair_link``) and
both sides run the kernel backends; on CPU it is the ``gloo`` host link with
the PyTorch oracle backends.  The rendezvous is 127.0.0.1 on a free port.
"""
from __future__ import annotations

import datetime
import os
import socket
from typing import Optional

import torch
import torch.distributed as dist

from .common import load_fast_weights, load_module, model_config, pin_host_threads

SLOT_BYTES_CPU = 1 << 22


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _join_group(rank: int, port: int, timeout_s: float) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=timeout_s))


def _verifier_main(port: int, target: str, device: str, seed: int, max_seqs: int, max_context: int,
                   cpus: Optional[str], timeout_s: float, temperature: float, top_k: int, top_p: float) -> None:
    """Child process: serve verifies until the drafter side closes the link."""
    pin_host_threads(cpus)
    _join_group(0, port, timeout_s)
    link = None
    try:
        dev = torch.device(device)
        if dev.type == "cuda":
            from ..api import open_pair_link, target_server
            torch.cuda.set_device(dev)
            link = open_pair_link(1, dev)
            srv = target_server(load_fast_weights(target, dev, seed), link, max_seqs=max_seqs,
                                max_context=max_context, device=dev, deadline_s=timeout_s,
                                temperature=temperature, top_k=top_k, top_p=top_p)
        else:
            from ..engine.backends import TorchTarget
            from ..engine.disagg import P2PTargetServer
            from ..parallel.p2p import HostLink
            link = HostLink(1, SLOT_BYTES_CPU)
            srv = P2PTargetServer(TorchTarget(load_module(target, dev, seed).eval(), temperature, top_k, top_p),
                                  link, deadline_s=timeout_s)
        srv.serve()
    finally:
        if link is not None and hasattr(link, "close") and getattr(link, "supports_device_put", False):
            link.close()
        dist.destroy_process_group()


class VerifierProcess:
    """Start the target's process and build the drafter-side engine.

    ``engine`` is a :class:`~d3d_b200.api.D3DEngine` whose target is the
    child; :meth:`close` ends the child's serving loop and joins it."""

    def __init__(self, a, decode, max_seqs: int, max_context: int, timeout_s: float = 600.0):
        import torch.multiprocessing as mp
        from ..api import D3DEngine
        self.vdev = torch.device(a.verifier_device or a.device)
        self.ddev = torch.device(a.draft_device or a.device)
        if (self.vdev.type == "cuda") != (self.ddev.type == "cuda"):
            raise ValueError("the verifier and the drafter must both be on CUDA devices or both on the CPU")
        port = _free_port()
        ctx = mp.get_context("spawn")
        self.proc = ctx.Process(target=_verifier_main, daemon=True,
                                args=(port, a.target, str(self.vdev), a.seed, max_seqs, max_context,
                                      getattr(a, "verifier_cpu_affinity", None), timeout_s,
                                      decode.temperature, decode.target_top_k, decode.target_top_p))
        self.proc.start()
        self.link = None
        try:
            _join_group(1, port, timeout_s)
            hidden = model_config(a.target).hidden_size
            if self.ddev.type == "cuda":
                from ..api import open_pair_link
                torch.cuda.set_device(self.ddev)
                self.link = open_pair_link(0, self.ddev)
                dw = load_fast_weights(a.draft, self.ddev, a.seed, a.draft_layers, a.mask_token_id)
                self.engine = D3DEngine.from_remote_target(dw, self.link, hidden, decode, max_seqs=max_seqs,
                                                           max_context=max_context, device=self.ddev,
                                                           deadline_s=timeout_s)
            else:
                from ..engine.backends import TorchDraft
                from ..engine.disagg import P2PTarget
                from ..parallel.p2p import HostLink
                self.link = HostLink(0, SLOT_BYTES_CPU)
                d = load_module(a.draft, self.ddev, a.seed, a.draft_layers, a.mask_token_id).eval()
                self.engine = D3DEngine(P2PTarget(self.link, hidden, deadline_s=timeout_s,
                                                  want_hidden=decode.use_cond and bool(d.cfg.cond_hidden_size)),
                                        TorchDraft(d), decode)
        except BaseException:
            self._stop_child()
            raise

    def _stop_child(self, wait_s: float = 60.0) -> None:
        self.proc.join(wait_s)
        if self.proc.is_alive():
            self.proc.terminate()          # this child only, by its own handle
            self.proc.join(10)
        if dist.is_initialized():
            dist.destroy_process_group()

    def close(self) -> None:
        try:
            self.engine.close()
            if self.link is not None and getattr(self.link, "supports_device_put", False):
                self.link.close()
        finally:
            self._stop_child()
        if self.proc.exitcode not in (0, None):
            raise RuntimeError(f"verifier process exited with code {self.proc.exitcode}")
