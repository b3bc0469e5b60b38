"""Reference arm of bench.py (runs the unmodified reference from baseline/_ref)."""


def run(args, rank, world, local):
    return {"impl": "reference", "unavailable": "reference arm not wired yet"}
