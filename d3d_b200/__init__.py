"""d3d_b200: asynchronous speculative decoding with block-diffusion drafters,
built for NVIDIA B200 (sm_100a).

Subpackages:

* :mod:`d3d_b200.models` — Qwen3 target / D3D drafter (PyTorch oracle) and the
  fast CUDA-kernel model;
* :mod:`d3d_b200.ops` — sm_100a kernels (tcgen05 GEMM, attention, norms,
  selection, acceptance, handoff, optimizer, fused loss) and their bindings;
* :mod:`d3d_b200.engine` — layouts, sampling/acceptance, the async decode
  coordinator and its backends;
* :mod:`d3d_b200.serving` — target service processes and the paged engine;
* :mod:`d3d_b200.parallel` — tensor parallelism, FSDP, peer-memory buffers;
* :mod:`d3d_b200.train` / :mod:`d3d_b200.pruning` — distillation and layer
  pruning;
* :mod:`d3d_b200.utils` — checkpoints, metrics, timing, runtime metadata.
"""
__version__ = "0.1.0"
