"""Acceptance and throughput accounting: hand-computed expectations for the
summaries the CLIs write (accept length includes the anchor, draft tokens
exclude it; histograms; all-pass runs; per-source statistics; timing
aggregates)."""
import pytest

from d3d_b200.utils.metrics import (AcceptanceStep, compact_acceptance, headline, high_speed_runs, percentile,
                                    source_stats, steps_from_output, summarize_acceptance, summarize_timing)


def test_acceptance_summary_by_hand():
    K = 4                                    # block: anchor + 3 drafts
    steps = steps_from_output([1, 4, 2, 4], K, list(range(11)))
    assert [s.accept_length for s in steps] == [1, 4, 2, 4]
    assert [s.accepted_draft_tokens for s in steps] == [0, 3, 1, 3]
    assert steps[1].emitted_tokens == [1, 2, 3, 4] and steps[3].emitted_tokens == [7, 8, 9, 10]
    s = summarize_acceptance(steps, K - 1)
    assert s["num_verify_steps"] == 4
    assert s["avg_accept_length"] == pytest.approx(11 / 4)
    assert s["avg_accepted_draft_tokens"] == pytest.approx(7 / 4)
    assert s["draft_accept_rate"] == pytest.approx(7 / 12)
    assert s["reject_at_0_rate"] == pytest.approx(1 / 4)
    assert s["all_draft_accepted_rate"] == pytest.approx(2 / 4)
    assert s["accept_length_histogram"] == {"1": 1, "2": 1, "3": 0, "4": 2}


def test_empty_and_no_draft_steps():
    e = summarize_acceptance([], 15)
    assert e["num_verify_steps"] == 0 and e["accept_length_histogram"]["16"] == 0
    steps = [AcceptanceStep(0, 1, 3, mode="no-draft"), AcceptanceStep(2, 3, 3, draft_tokens=[1, 2, 3])]
    s = summarize_acceptance(steps, 3)
    assert s["no_draft_num_steps"] == 1 and s["avg_no_draft_verify_tokens"] == 3
    assert s["reject_at_0_rate"] == 0.0 and s["draft_accept_rate"] == pytest.approx(2 / 3)


def test_runs_sources_and_percentiles():
    # all-pass runs of length >= 3: blocks 1-3 (one region), blocks 6-9 (another)
    acc = [16, 16, 16, 5, 16, 16, 16, 16, 16, 3]
    bs = [16] * 10
    r = high_speed_runs(bs, acc, 3)
    assert r["high_speed_continuous_blocks"] == 8 and r["high_speed_continuous_regions"] == 2
    assert r["high_speed_continuous_block_rate"] == pytest.approx(0.8)
    st = source_stats(["a", "b", "a", "b"], [16, 16, 16, 16], [16, 1, 8, 16])
    assert st["a"]["all_pass_count"] == 1 and st["a"]["mean_accept_len"] == 12
    assert st["b"]["reject_at_0_rate"] == 0.5
    assert percentile([5, 1, 3, 2, 4], 0.5) == 3 and percentile([], 0.9) == 0.0
    c = compact_acceptance([2.5, 3.0], [1, 4, 2, 4], 4)
    assert c["mean_accept_per_verify"] == pytest.approx(2.75) and c["histogram"]["4"] == 2


def test_timing_and_headline():
    per = [{"output_tokens": 10, "decode_tokens": 9, "decode_elapsed_s": 0.3, "tokens_per_s": 30.0,
            "time_per_output_token": 0.0333},
           {"output_tokens": 20, "decode_tokens": 19, "decode_elapsed_s": 0.7, "tokens_per_s": 27.1,
            "time_per_output_token": 0.0368}]
    t = summarize_timing(per, elapsed_s=2.0)
    assert t["aggregate_decode_tokens_per_s"] == pytest.approx(28 / 1.0)
    assert t["elapsed_tokens_per_s"] == pytest.approx(15.0)
    assert t["mean_tokens_per_s"] == pytest.approx(28.55)
    h = headline(300.0, 100.0, 4.5)
    assert h["speedup"] == pytest.approx(3.0) and h["accept_length"] == 4.5
    assert headline(300.0, 0.0, 1.0)["speedup"] is None
