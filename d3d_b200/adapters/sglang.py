"""Thin adapter exposing the drafter as a remote draft service for an
SGLang-style target server (reference: ``d3d_sglang/service.py:22-219``,
``d3d_sglang/plugin.py``).

The service keeps one session per request id.  Each ``step`` receives, for
every live request, the prompt and the target's output tokens so far (the
last one is the anchor the target just produced).  If the outputs extend the
previous call's outputs, the newly committed tokens identify which
pre-drafted branch (commit length, anchor) became valid and that branch is
returned; otherwise (a new request, a rewritten history or a miss) the
drafter redrafts from the anchor.  After the reply is sent, ``speculate``
runs the packed all-outcome forward for every session, overlapping the
target's next verification — the decoupled loop of the reference's Hybrid
mode.

Transport: newline-delimited JSON over TCP (``serve``), commands
``step`` / ``metrics`` / ``close``.  The reference speaks ZeroMQ to its
vendored SGLang fork; neither ZeroMQ nor SGLang is part of this build, so
:func:`register` only reports that the SGLang plugin entry point needs
SGLang installed.
"""
from __future__ import annotations

import json
import socket
import socketserver
import threading
import time
from typing import Dict, List, Optional

from ..engine.backends import DraftBackend, SeqState
from ..engine.spec import DecodeConfig, SpecDecoder


class _NoTarget:
    def release(self, s):
        pass


class DraftService:
    def __init__(self, draft: DraftBackend, block_size: int = 16, anchor_num: int = 1,
                 attention_mask_mode: str = "causal", speculate: bool = True):
        self.d = draft
        self.cfg = DecodeConfig(block_size=block_size, anchor_num=anchor_num,
                                attention_mask_mode=attention_mask_mode, max_new_tokens=1 << 30,
                                use_cond=False)
        self.coord = SpecDecoder(_NoTarget(), draft, self.cfg)
        self.speculate_enabled = speculate
        self.sessions: Dict[str, dict] = {}
        self._next = 0
        self.metrics = {"required_forward_count": 0, "required_seconds": 0.0, "remote_hit_count": 0,
                        "remote_miss_count": 0, "optional_forward_count": 0, "optional_seconds": 0.0}

    def _new_seq(self, prefix: List[int]) -> SeqState:
        self._next += 1
        s = SeqState(index=self._next, prompt=list(prefix[:-1]), prefix=len(prefix) - 1)
        self.d.prefill([s], self.cfg.attention_mask_mode, self.cfg.block_size)
        s.anchor = int(prefix[-1])
        return s

    def _close(self, st: dict) -> None:
        self.d.release(st["seq"])

    def step(self, items: List[dict]) -> dict:
        live = {it["rid"] for it in items}
        for rid in list(self.sessions):
            if rid not in live:
                self._close(self.sessions.pop(rid))
        proposals = {}
        misses = []
        K = self.cfg.block_size
        for it in items:
            rid = it["rid"]
            prompt, outputs = list(it["prompt"]), list(it["outputs"])
            if not outputs:
                raise ValueError("missing target anchor")
            prev = self.sessions.get(rid)
            sel = None
            if prev is not None and prompt == prev["prompt"] and outputs[:len(prev["outputs"])] == prev["outputs"]:
                delta = outputs[len(prev["outputs"]):]
                s = prev["seq"]
                commit = len(delta)               # previous anchor + accepted drafts
                if commit >= 1:
                    key = (commit, None if commit == K else delta[-1])
                    oc = prev.get("outcomes")
                    sel = oc.get(key) if oc is not None else None
                    s.prefix += commit
                    s.anchor = int(outputs[-1])
                    self.d.trim(s, s.prefix)
            else:
                if prev is not None:
                    self._close(prev)
                s = self._new_seq(prompt + outputs)
            if sel is not None:
                blk, top, _ = sel
                blk = blk.clone()
                blk[0] = s.anchor
                s.current, s.top = blk, top
                self.metrics["remote_hit_count"] += 1
            else:
                misses.append(s)
                self.metrics["remote_miss_count"] += 1
            self.sessions[rid] = {"prompt": prompt, "outputs": outputs, "seq": s, "outcomes": None}
        if misses:
            t0 = time.perf_counter()
            self.coord.recover(misses)
            self.metrics["required_forward_count"] += 1
            self.metrics["required_seconds"] += time.perf_counter() - t0
        for it in items:
            s = self.sessions[it["rid"]]["seq"]
            proposals[it["rid"]] = {"tokens": [int(t) for t in s.current.tolist()]}
        return {"proposals": proposals}

    def speculate(self) -> None:
        if not self.speculate_enabled or not self.sessions:
            return
        t0 = time.perf_counter()
        states = list(self.sessions.values())
        preds = self.coord.predict([st["seq"] for st in states])
        for st in states:
            st["outcomes"] = preds.get(st["seq"].index)
        self.metrics["optional_forward_count"] += 1
        self.metrics["optional_seconds"] += time.perf_counter() - t0


# ------------------------------------------------------------------ transport
def serve(service: DraftService, host: str = "127.0.0.1", port: int = 0,
          ready: Optional[threading.Event] = None, bound: Optional[list] = None) -> None:
    """Serve newline-delimited JSON requests until a ``close`` command."""

    class Handler(socketserver.StreamRequestHandler):
        def handle(self):
            for line in self.rfile:
                req = json.loads(line)
                cmd = req.get("cmd")
                try:
                    if cmd == "step":
                        out = service.step(req["items"])
                    elif cmd == "metrics":
                        out = dict(service.metrics)
                    elif cmd == "close":
                        self.wfile.write(b'{"ok": true}\n')
                        threading.Thread(target=self.server.shutdown, daemon=True).start()
                        return
                    else:
                        raise ValueError(f"unknown command {cmd!r}")
                    self.wfile.write((json.dumps(out) + "\n").encode())
                    self.wfile.flush()
                    if cmd == "step":
                        service.speculate()         # overlaps the target's next verify
                except Exception as e:  # reported to the caller
                    self.wfile.write((json.dumps({"error": repr(e)}) + "\n").encode())
                    self.wfile.flush()

    with socketserver.TCPServer((host, port), Handler) as srv:
        if bound is not None:
            bound.append(srv.server_address[1])
        if ready is not None:
            ready.set()
        srv.serve_forever()


class DraftClient:
    def __init__(self, host: str, port: int, timeout: float = 60.0):
        self.sock = socket.create_connection((host, port), timeout=timeout)
        self.f = self.sock.makefile("rwb")

    def request(self, payload: dict) -> dict:
        self.f.write((json.dumps(payload) + "\n").encode())
        self.f.flush()
        line = self.f.readline()
        if not line:
            raise RuntimeError("draft service closed the connection")
        out = json.loads(line)
        if "error" in out:
            raise RuntimeError(f"draft service failed: {out['error']}")
        return out

    def step(self, items):
        return self.request({"cmd": "step", "items": items})["proposals"]

    def close(self):
        try:
            self.request({"cmd": "close"})
        finally:
            self.sock.close()


def register():
    """SGLang plugin entry point (``sglang.srt.plugins``)."""
    try:
        import sglang  # noqa: F401
    except ImportError as e:
        raise RuntimeError("the SGLang plugin needs SGLang installed; use DraftService/serve directly") from e
    raise RuntimeError("SGLang integration is provided as the DraftService protocol adapter only")
