"""Counter of this framework's own kernel launches (host-side bookkeeping).

Eager launches add their count as they are issued; a CUDA-graph replay adds
the number of kernels that were captured into the graph.  ``bench.py``
reports the count of the timed region as ``gpu_launches``.
"""
_count = 0


def add(n: int) -> None:
    global _count
    _count += int(n)


def reset() -> None:
    global _count
    _count = 0


def count() -> int:
    return _count
