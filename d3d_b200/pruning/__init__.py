"""Progressive layer pruning of the drafter (reference: ``pruning/``):
:mod:`.modeling` (score single-layer removals), :mod:`.select_layer`,
:mod:`.prune` (physical checkpoint rewrite), :mod:`.recovery` (recovery
training) and :mod:`.select_checkpoint`; CLI ``python -m d3d_b200.pruning``."""
