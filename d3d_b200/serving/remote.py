"""Target service in another process, over ``torch.distributed`` messages.

The reference runs its target in a spawned process and ships Python lists
through a ``multiprocessing`` Pipe (``serving/target_process.py:9-139``,
``single/eval_async_packed.py:56-346``).  Here the two sides are ranks of a
process group (``gloo`` between CPU processes, or between the host sides of
two GPU processes).  The protocol, the server loop and the client backend
are those of :mod:`d3d_b200.engine.disagg` (PREFILL / VERIFY / RELEASE /
CLOSE, errors returned as tracebacks and re-raised by the client,
``serving/target_process.py:59-66``), carried by a
:class:`~d3d_b200.parallel.p2p.HostLink` instead of NVLink mailboxes.
Liveness relies on the process group's timeout: a peer that died or never
joined ends the next message with an error instead of hanging.
"""
from __future__ import annotations

from ..engine.disagg import P2PTarget, P2PTargetServer
from ..parallel.p2p import HostLink

HOST_SLOT_BYTES = 256 << 10   # one message: header + metadata + prompt tokens / verify result


class TargetServer(P2PTargetServer):
    """Serves a :class:`~d3d_b200.engine.backends.TargetBackend` to ``client_rank``."""

    def __init__(self, backend, client_rank: int, group=None, slot_bytes: int = HOST_SLOT_BYTES):
        super().__init__(backend, HostLink(client_rank, slot_bytes, group))


class RemoteTarget(P2PTarget):
    """Client side: a target backend whose target lives on ``server_rank``."""

    def __init__(self, server_rank: int, hidden_size: int, group=None, slot_bytes: int = HOST_SLOT_BYTES):
        super().__init__(HostLink(server_rank, slot_bytes, group), hidden_size)
