"""Config and runtime plumbing: HF ``config.json`` round trips (drafter
fields, unknown keys kept), mask-token validation, paged-capacity checks,
model-path resolution, dtype names, run metadata and the host profiler."""
import json

import pytest

from d3d_b200.config import DEFAULT_MASK_TOKEN_ID, ModelConfig, tiny_drafter, tiny_target
from d3d_b200.utils.runtime import (check_paged_capacity, required_pages, resolve_dtype, resolve_model_path,
                                    runtime_metadata)
from d3d_b200.utils.timing import StepProfiler


def test_hf_config_roundtrip_and_drafter_fields(tmp_path):
    d = tiny_drafter()
    d.save(tmp_path / "d")
    raw = json.loads((tmp_path / "d" / "config.json").read_text())
    assert raw["architectures"] == ["Qwen3ForCausalLM"] and raw["d3d_draft"] is True
    back = ModelConfig.from_pretrained(tmp_path / "d")
    assert back.to_hf_dict() == d.to_hf_dict()
    # unknown upstream keys survive a round trip; rope_theta may sit in rope_parameters
    raw.pop("rope_theta")
    raw["rope_parameters"] = {"rope_theta": 123.0}
    raw["sliding_window"] = None
    c = ModelConfig.from_hf_dict(raw)
    assert c.rope_theta == 123.0 and "sliding_window" in c.to_hf_dict()
    t = tiny_target()
    assert "d3d_draft" not in t.to_hf_dict() and t.mask_token_id is None


def test_mask_token_validation(tmp_path):
    raw = tiny_drafter().to_hf_dict()
    mid = raw["mask_token_id"]
    assert ModelConfig.from_hf_dict(raw, mask_token_id=mid).mask_token_id == mid
    with pytest.raises(ValueError, match="conflicts"):
        ModelConfig.from_hf_dict(raw, mask_token_id=mid + 1)
    bad = dict(raw, mask_token_id=raw["vocab_size"] + 5)
    with pytest.raises(ValueError, match="outside"):
        ModelConfig.from_hf_dict(bad)
    no_id = {k: v for k, v in raw.items() if k != "mask_token_id"}
    if no_id["vocab_size"] > DEFAULT_MASK_TOKEN_ID:
        assert ModelConfig.from_hf_dict(no_id).mask_token_id == DEFAULT_MASK_TOKEN_ID
    else:
        with pytest.raises(ValueError):
            ModelConfig.from_hf_dict(no_id)
    with pytest.raises(ValueError, match="multiple"):
        ModelConfig.from_hf_dict(dict(raw, num_key_value_heads=3))


def test_paged_capacity_and_paths(tmp_path):
    assert required_pages([100, 30], 50, 2, 16, 16) == 2 * 11
    check_paged_capacity([100], 50, [1, 2], pages=200, page_size=16, block_size=4, anchor_num=1)
    with pytest.raises(ValueError, match="pages"):
        check_paged_capacity([100, 100], 400, [2], pages=20, page_size=16)
    with pytest.raises(ValueError, match="context limit"):
        check_paged_capacity([100], 20000, [1], pages=1 << 20, page_size=16)
    with pytest.raises(FileNotFoundError):
        resolve_model_path(str(tmp_path / "absent"))
    (tmp_path / "m").mkdir()
    with pytest.raises(FileNotFoundError, match="config.json"):
        resolve_model_path(str(tmp_path / "m"))
    tiny_target().save(tmp_path / "m")
    assert resolve_model_path(str(tmp_path / "m")).endswith("/m")
    import torch
    assert resolve_dtype("bf16") is torch.bfloat16 and resolve_dtype("fp32") is torch.float32
    with pytest.raises(ValueError):
        resolve_dtype("fp8")
    meta = runtime_metadata({"target": str(tmp_path / "m")})
    assert meta["checkpoints"]["target"]["model_type"] == "qwen3"
    assert any(k.endswith(".cu") for k in meta["source_sha256"])


def test_host_profiler_phases():
    prof = StepProfiler(True)
    for _ in range(3):
        with prof.phase("select"):
            pass
    with prof.phase("receive"):
        pass
    s = prof.summary()
    assert s["calls"] == {"select": 3, "receive": 1} and set(s["host_ms"]) == {"select", "receive"}
    assert s["device"] == {}
    off = StepProfiler(False)
    with off.phase("x"):
        pass
    assert off.summary()["calls"] == {} and off.dev_begin("v", None) is None


def test_cpu_lists_and_pinning():
    import os
    from d3d_b200.cli.common import parse_cpu_list, pin_host_threads
    assert parse_cpu_list("0-3,8, 10-11") == [0, 1, 2, 3, 8, 10, 11]
    assert parse_cpu_list(None) == [] and parse_cpu_list("") == []
    with pytest.raises(ValueError):
        parse_cpu_list("5-2")
    before = os.sched_getaffinity(0)
    try:
        one = str(min(before))
        assert pin_host_threads(one, None) == [int(one)]
        assert os.sched_getaffinity(0) == {int(one)}
        assert pin_host_threads(None, None) is None
    finally:
        os.sched_setaffinity(0, before)
