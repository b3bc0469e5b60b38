"""Command-line entry points (``python -m d3d_b200.cli.<name>``).

* ``single``  — single-request asynchronous decoding (``--verifier``/``--drafter``),
  the reference's ``single/eval_async_packed.py``;
* ``sync``    — synchronous multi-step denoising decode (``single/eval_sync.py``);
* ``serve``   — concurrent paged serving benchmark (``--target``/``--draft``,
  ``--pages``, ``--concurrency``), the reference's ``serving/bench.py``;
* ``train``   — drafter distillation (``train/train.py``);
* ``prune``   — layer selection / pruning / recovery (``pruning/*``).

Every model argument accepts a Hugging Face-layout checkpoint directory or a
preset name (``qwen3-8b``, ``qwen3-32b``, ``d3d-1.7b``, ``tiny-target`` ...),
which builds random-init weights from ``--seed``.
"""
