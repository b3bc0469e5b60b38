"""Adapters to other serving stacks (off the decode hot path)."""
