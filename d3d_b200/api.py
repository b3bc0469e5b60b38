"""Public API: build a target + drafter pair and decode.

>>> eng = D3DEngine.from_pretrained("Qwen/Qwen3-8B-dir", "D3D-1.7B-dir")      # doctest: +SKIP
>>> out = eng.generate([[151644, 872, 198]], max_new_tokens=128)                 # doctest: +SKIP

``D3DEngine`` wraps the coordinator (:class:`~d3d_b200.engine.spec.SpecDecoder`)
with the kernel backends on CUDA and the PyTorch oracle backends on CPU.  The
same object also runs target-only AR decoding (:meth:`generate_ar`), the
baseline every speedup is measured against.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch

from .config import ModelConfig
from .engine.spec import DecodeConfig, SpecDecoder, ar_generate


class D3DEngine:
    def __init__(self, target, draft, decode: DecodeConfig):
        self.target = target
        self.draft = draft
        self.decode = decode
        self.decoder = SpecDecoder(target, draft, decode)

    # ------------------------------------------------------------ builders
    @classmethod
    def from_weights(cls, target_w, draft_w, decode: Optional[DecodeConfig] = None, *,
                     max_seqs: int = 16, max_context: int = 4096, target_pages: Optional[int] = None,
                     draft_pages: Optional[int] = None, page_size: int = 16, device="cuda",
                     use_graphs: bool = True, shared_stream: bool = True) -> "D3DEngine":
        """Kernel backends from :class:`~d3d_b200.models.fast.FastWeights`.

        ``shared_stream``: target and drafter enqueue on one CUDA stream (the
        verify then the packed draft, back to back).  Measured on B200 this is
        faster than two concurrent streams: both forwards are HBM-bound, and
        co-scheduling them slows each more than it overlaps them."""
        from .engine.fast import FastDraft, FastTarget
        from .engine.layout import paged_draft_branch_tokens

        decode = decode or DecodeConfig()
        packed_q = paged_draft_branch_tokens(decode.block_size, max(decode.anchor_num, 1))
        tp = target_pages or max_seqs * (max_context + 64 + page_size) // page_size + 8
        dp = draft_pages or max_seqs * (max_context + packed_q + page_size) // page_size + 8
        t = FastTarget(target_w, pages=tp, page_size=page_size, max_seqs=max_seqs,
                       max_context=max_context, use_graphs=use_graphs, device=device,
                       temperature=decode.temperature, top_k=decode.target_top_k,
                       top_p=decode.target_top_p)
        d = FastDraft(draft_w, pages=dp, page_size=page_size, max_seqs=max_seqs,
                      max_context=max_context, packed_q=packed_q, use_graphs=use_graphs,
                      device=device, stream=t.stream if shared_stream else None)
        return cls(t, d, decode)

    @classmethod
    def from_modules(cls, target_m, draft_m, decode: Optional[DecodeConfig] = None,
                     **kw) -> "D3DEngine":
        """Oracle backends on CPU, kernel backends when the modules are on CUDA."""
        dev = next(target_m.parameters()).device
        if dev.type == "cuda":
            from .models.fast import FastWeights
            return cls.from_weights(FastWeights.from_module(target_m, dev),
                                    FastWeights.from_module(draft_m, dev), decode, device=dev, **kw)
        from .engine.backends import TorchDraft, TorchTarget
        decode = decode or DecodeConfig()
        return cls(TorchTarget(target_m, decode.temperature, decode.target_top_k, decode.target_top_p), TorchDraft(draft_m), decode)

    @classmethod
    def from_pretrained(cls, target_path: str, draft_path: str,
                        decode: Optional[DecodeConfig] = None, device="cuda", **kw) -> "D3DEngine":
        from .checkpoint import load_model
        t = load_model(target_path, device="cpu")
        d = load_model(draft_path, device="cpu")
        if device != "cpu" and torch.cuda.is_available():
            from .models.fast import FastWeights
            return cls.from_weights(FastWeights.from_module(t, device),
                                    FastWeights.from_module(d, device), decode, device=device, **kw)
        return cls.from_modules(t, d, decode)

    @classmethod
    def from_remote_target(cls, draft_w, link, target_hidden_size: int,
                           decode: Optional[DecodeConfig] = None, *, max_seqs: int = 16,
                           max_context: int = 4096, draft_pages: Optional[int] = None,
                           page_size: int = 16, device="cuda", use_graphs: bool = True,
                           deadline_s: float = 600.0) -> "D3DEngine":
        """Drafter and coordinator on this GPU; the target is served by the
        peer at the other end of ``link`` (:func:`open_pair_link`,
        :func:`target_server`).  A reply that does not arrive within
        ``deadline_s`` raises ``TimeoutError``."""
        from .engine.disagg import P2PTarget
        from .engine.fast import FastDraft
        from .engine.layout import paged_draft_branch_tokens

        decode = decode or DecodeConfig()
        packed_q = paged_draft_branch_tokens(decode.block_size, max(decode.anchor_num, 1))
        dp = draft_pages or max_seqs * (max_context + packed_q + page_size) // page_size + 8
        d = FastDraft(draft_w, pages=dp, page_size=page_size, max_seqs=max_seqs,
                      max_context=max_context, packed_q=packed_q, use_graphs=use_graphs, device=device)
        t = P2PTarget(link, target_hidden_size, device, deadline_s=deadline_s,
                      want_hidden=decode.use_cond and draft_w.cond_proj is not None, draft_stream=d.stream)
        return cls(t, d, decode)

    def close(self) -> None:
        """Stop a remote target's serving loop (no-op for local targets)."""
        if hasattr(self.target, "close"):
            self.target.close()

    # ------------------------------------------------------------- decoding
    def generate(self, prompts: Sequence[Sequence[int]], *, max_new_tokens: Optional[int] = None,
                 concurrency: int = 1, controlled: Optional[Callable[[int], object]] = None,
                 max_new: Optional[Sequence[int]] = None) -> dict:
        """Speculative decoding.  ``max_new``: per-request output budgets;
        ``max_new_tokens``: one budget for every request of this call (the
        engine's default stays as configured)."""
        if isinstance(prompts, torch.Tensor):
            prompts = prompts.tolist()
        if max_new is None and max_new_tokens is not None:
            max_new = [int(max_new_tokens)] * len(prompts)
        return self.decoder.generate(prompts, concurrency=concurrency, controlled=controlled, max_new=max_new)

    def generate_ar(self, prompts: Sequence[Sequence[int]], *, max_new_tokens: Optional[int] = None,
                    concurrency: int = 1, max_new: Optional[Sequence[int]] = None) -> dict:
        n = max_new_tokens or self.decoder.cfg.max_new_tokens
        if isinstance(prompts, torch.Tensor):
            prompts = prompts.tolist()
        return ar_generate(self.target, prompts, n, eos=self.decoder.cfg.eos,
                           ignore_eos=self.decoder.cfg.ignore_eos, concurrency=concurrency, max_new=max_new)


def open_pair_link(peer: int, device, slot_bytes: Optional[int] = None, group=None):
    """Collective over ``group``: map NVLink mailboxes between this rank and
    ``peer`` (every rank of the group calls it, each with its own peer)."""
    from .engine.disagg import DEFAULT_SLOT_BYTES
    from .parallel.p2p import Link
    return Link(peer, slot_bytes or DEFAULT_SLOT_BYTES, torch.device(device), group)


def load_target_shard(path: str, tp: int, rank: int, device="cuda"):
    """One rank's :class:`~d3d_b200.models.fast.FastWeights` of a
    tensor-parallel target, read slice by slice from an HF checkpoint."""
    from .checkpoint import load_tp_shard
    from .models.fast import FastWeights
    from .parallel.tp import local_config
    cfg = ModelConfig.from_pretrained(path)
    w = FastWeights.from_state(local_config(cfg, tp), load_tp_shard(path, rank, tp, device=device), device)
    w.tp = (tp, rank, cfg)
    return w


def target_server(target_w, link, *, max_seqs: int = 16, max_context: int = 4096,
                  target_pages: Optional[int] = None, page_size: int = 16, device="cuda",
                  use_graphs: bool = True, deadline_s: float = 600.0, tp=None, replies: str = "all",
                  temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0):
    """The target side of a disaggregated pair: call ``.serve()`` on the result;
    it returns when the drafter side calls :meth:`D3DEngine.close`, and raises
    ``TimeoutError`` after ``deadline_s`` without a request.  For one rank of
    a tensor-parallel target pass its ``TPGroup`` as ``tp`` (and
    ``replies="ack"`` on every rank but 0).  ``temperature`` / ``top_k`` /
    ``top_p``: the target's sampling (sampled verifies carry the drafts'
    proposals in their requests)."""
    from .engine.disagg import P2PTargetServer
    from .engine.fast import FastTarget
    pages = target_pages or max_seqs * (max_context + 64 + page_size) // page_size + 8
    t = FastTarget(target_w, pages=pages, page_size=page_size, max_seqs=max_seqs,
                   max_context=max_context, use_graphs=use_graphs, device=device, tp=tp,
                   temperature=temperature, top_k=top_k, top_p=top_p)
    return P2PTargetServer(t, link, deadline_s=deadline_s, replies=replies)
