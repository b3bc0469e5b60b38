"""Acceptance and throughput accounting (reference: ``common/metrics.py``,
``single/eval_sync.py:380-423``).

``accept_length`` is the number of tokens committed per verify, anchor
included; ``accepted_draft_tokens`` excludes the anchor.  Decode throughput
excludes prefill and the first (prefill-produced) token for single-request
runs, as in the reference.
"""
from __future__ import annotations

import statistics
from collections import Counter
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Sequence


@dataclass
class AcceptanceStep:
    accepted_draft_tokens: int
    accept_length: int
    emitted_count: int
    emitted_tokens: List[int] = field(default_factory=list)
    draft_tokens: List[int] = field(default_factory=list)
    target_tokens: List[int] = field(default_factory=list)
    stopped: bool = False
    mode: str = "draft"


def summarize_acceptance(steps: Sequence[AcceptanceStep], draft_tokens: int) -> Dict[str, Any]:
    hist_keys = [str(i) for i in range(1, int(draft_tokens) + 2)]
    if not steps:
        return {"num_verify_steps": 0, "avg_accepted_draft_tokens": 0.0, "avg_accept_length": 0.0,
                "avg_emitted_tokens": 0.0, "draft_accept_rate": 0.0, "reject_at_0_rate": 0.0,
                "all_draft_accepted_rate": 0.0, "no_draft_num_steps": 0,
                "avg_no_draft_verify_tokens": 0.0, "accept_length_histogram": {k: 0 for k in hist_keys}}
    drafted = [s for s in steps if s.draft_tokens]
    no_draft = [s for s in steps if s.mode == "no-draft"]
    total_draft = sum(len(s.draft_tokens) for s in steps)
    lengths = Counter(s.accept_length for s in steps)
    return {
        "num_verify_steps": len(steps),
        "avg_accepted_draft_tokens": statistics.fmean(s.accepted_draft_tokens for s in steps),
        "avg_accept_length": statistics.fmean(s.accept_length for s in steps),
        "avg_emitted_tokens": statistics.fmean(s.emitted_count for s in steps),
        "draft_accept_rate": sum(s.accepted_draft_tokens for s in steps) / total_draft if total_draft else 0.0,
        "reject_at_0_rate": (sum(s.accepted_draft_tokens == 0 for s in drafted) / len(drafted)
                             if drafted else 0.0),
        "all_draft_accepted_rate": (sum(s.accepted_draft_tokens == len(s.draft_tokens) for s in drafted)
                                    / len(drafted) if drafted else 0.0),
        "no_draft_num_steps": len(no_draft),
        "avg_no_draft_verify_tokens": statistics.fmean(s.emitted_count for s in no_draft) if no_draft else 0.0,
        "accept_length_histogram": {k: lengths.get(int(k), 0) for k in hist_keys},
    }


def steps_from_output(accepts: Sequence[int], block_size: int, tokens: Sequence[int]) -> List[AcceptanceStep]:
    """Acceptance steps of one request from its per-verify commit lengths."""
    out, off = [], 0
    for n in accepts:
        emitted = list(tokens[off:off + n])
        off += n
        out.append(AcceptanceStep(accepted_draft_tokens=max(int(n) - 1, 0), accept_length=int(n),
                                  emitted_count=len(emitted), emitted_tokens=emitted,
                                  draft_tokens=[0] * (block_size - 1)))
    return out


def summarize_timing(per_prompt: Sequence[Dict[str, Any]], *, elapsed_s: float) -> Dict[str, float]:
    out_tok = sum(int(x.get("output_tokens", 0)) for x in per_prompt)
    dec_tok = sum(int(x.get("decode_tokens", x.get("output_tokens", 0))) for x in per_prompt)
    dec_t = sum(float(x.get("decode_elapsed_s", 0.0)) for x in per_prompt)
    tps = [float(x.get("tokens_per_s", 0.0)) for x in per_prompt]
    tpot = [float(x.get("time_per_output_token", 0.0)) for x in per_prompt
            if int(x.get("decode_tokens", x.get("output_tokens", 0))) > 0]
    agg = dec_tok / dec_t if dec_t > 0 else 0.0
    return {"total_decode_elapsed_s": dec_t,
            "mean_tokens_per_s": statistics.fmean(tps) if tps else 0.0,
            "mean_prompt_decode_tps": statistics.fmean(tps) if tps else 0.0,
            "mean_time_per_output_token": statistics.fmean(tpot) if tpot else 0.0,
            "aggregate_decode_tokens_per_s": agg, "aggregate_decode_tps": agg,
            "elapsed_tokens_per_s": out_tok / elapsed_s if elapsed_s > 0 else 0.0}


def headline(d3d_tps: float, baseline_tps: float, accept_length: float, metric: str = "decode") -> Dict[str, Any]:
    d3d_tps, baseline_tps = float(d3d_tps or 0.0), float(baseline_tps or 0.0)
    return {"metric": metric, "d3d_tps": d3d_tps, "baseline_tps": baseline_tps,
            "speedup": d3d_tps / baseline_tps if baseline_tps > 0 else None,
            "accept_length": float(accept_length or 0.0)}


def percentile(values: Sequence[float], q: float) -> float:
    if not values:
        return 0.0
    xs = sorted(values)
    return float(xs[max(0, min(len(xs) - 1, int(round((len(xs) - 1) * q))))])


def compact_acceptance(per_sample: Sequence[float], flat: Sequence[int], block_size: int) -> Dict[str, Any]:
    hist = Counter(int(x) for x in flat)
    return {"num_samples": len(per_sample), "num_verify_steps": len(flat), "block_size": int(block_size),
            "mean_accept_per_sample": statistics.fmean(per_sample) if per_sample else 0.0,
            "mean_accept_per_verify": statistics.fmean(flat) if flat else 0.0,
            "median_accept_per_verify": statistics.median(flat) if flat else 0.0,
            "p90_accept_per_verify": percentile(flat, 0.90), "p95_accept_per_verify": percentile(flat, 0.95),
            "min_accept_per_verify": min(flat) if flat else 0, "max_accept_per_verify": max(flat) if flat else 0,
            "histogram": {str(k): hist.get(k, 0) for k in range(int(block_size) + 1)}}


def high_speed_runs(block_sizes: Sequence[int], accepts: Sequence[int], min_run: int = 3) -> Dict[str, Any]:
    """Blocks inside runs of >= min_run consecutive all-pass verifies
    (``single/eval_async_packed.py:_high_speed_continuous_stats``)."""
    total, blocks, regions, run = len(accepts), 0, 0, 0
    for bs, a in list(zip(block_sizes, accepts)) + [(1, 0)]:
        if int(a) == int(bs):
            run += 1
            continue
        if run >= min_run:
            regions += 1
            blocks += run
        run = 0
    return {"high_speed_min_consecutive_all_pass_blocks": min_run, "high_speed_continuous_blocks": blocks,
            "high_speed_total_blocks": total,
            "high_speed_continuous_block_rate": blocks / total if total else 0.0,
            "high_speed_continuous_regions": regions}


def source_stats(sources: Sequence[str], block_sizes: Sequence[int], accepts: Sequence[int]) -> Dict[str, Any]:
    grouped: Dict[str, List[tuple]] = {}
    for s, b, a in zip(sources, block_sizes, accepts):
        grouped.setdefault(s, []).append((int(b), int(a)))
    out = {}
    for s, rows in sorted(grouped.items()):
        allp = sum(1 for b, a in rows if a == b)
        out[s] = {"count": len(rows), "all_pass_count": allp, "all_pass_rate": allp / len(rows),
                  "mean_block_size": statistics.fmean(b for b, _ in rows),
                  "mean_accept_len": statistics.fmean(a for _, a in rows),
                  "accept_len_histogram": {str(k): v for k, v in sorted(Counter(a for _, a in rows).items())},
                  "reject_at_0_rate": sum(1 for _, a in rows if a <= 1) / len(rows)}
    return out


def step_dicts(steps: Sequence[AcceptanceStep]) -> List[Dict[str, Any]]:
    return [asdict(s) for s in steps]
