"""Checkpoint format: HF-layout safetensors round trips exactly (fp32 and
bf16, one file and sharded with an index), and the strict loader refuses
incomplete, padded, misshapen or dangling checkpoints with a clear error."""
import json

import pytest
import torch

from d3d_b200.checkpoint import INDEX, load_model, read_state, save_model, write_state
from d3d_b200.cli.common import model_config
from d3d_b200.models.qwen3 import build_model


def _tiny():
    return build_model(model_config("tiny-drafter"), seed=5, dtype=torch.float32, device="cpu")


def _same(a, b):
    sa, sb = a.state_dict(), b.state_dict()
    assert sa.keys() == sb.keys()
    return all(torch.equal(sa[k], sb[k]) for k in sa)


def test_roundtrip_exact_fp32_and_bf16(tmp_path):
    m = _tiny()
    save_model(m, tmp_path / "fp32")
    assert _same(m, load_model(tmp_path / "fp32"))
    mb = m.to(torch.bfloat16)
    save_model(mb, tmp_path / "bf16", dtype=torch.bfloat16)
    assert _same(mb, load_model(tmp_path / "bf16", dtype=torch.bfloat16))


def test_sharded_roundtrip_with_index(tmp_path):
    m = _tiny()
    save_model(m, tmp_path / "sh", max_shard_bytes=1 << 16)
    idx = json.loads((tmp_path / "sh" / INDEX).read_text())
    assert len(set(idx["weight_map"].values())) > 1
    assert _same(m, load_model(tmp_path / "sh"))
    # the replaced checkpoint keeps no stale files around
    save_model(m, tmp_path / "sh", max_shard_bytes=1 << 16)
    assert _same(m, load_model(tmp_path / "sh"))


def _write(tmp_path, name, state, cfg):
    d = tmp_path / name
    d.mkdir()
    write_state(state, d)
    cfg.save(d)
    return d


def test_strict_loader_negatives(tmp_path):
    m = _tiny()
    state = {k: v.clone() for k, v in m.state_dict().items()}
    cfg = m.cfg
    if cfg.tie_word_embeddings:
        state.pop("lm_head.weight", None)
    missing = dict(state)
    missing.pop("model.layers.0.mlp.down_proj.weight")
    with pytest.raises(ValueError, match="missing"):
        load_model(_write(tmp_path, "missing", missing, cfg))
    extra = dict(state)
    extra["model.layers.99.mlp.down_proj.weight"] = torch.zeros(2, 2)
    with pytest.raises(ValueError, match="unexpected"):
        load_model(_write(tmp_path, "extra", extra, cfg))
    bad = dict(state)
    bad["model.norm.weight"] = torch.zeros(cfg.hidden_size + 1)
    with pytest.raises(ValueError, match="shape"):
        load_model(_write(tmp_path, "shape", bad, cfg))
    d = tmp_path / "dangling"
    save_model(m, d, max_shard_bytes=1 << 16)
    victim = sorted(set(json.loads((d / INDEX).read_text())["weight_map"].values()))[0]
    (d / victim).unlink()
    with pytest.raises(FileNotFoundError, match="missing shard"):
        load_model(d)
    empty = tmp_path / "empty"
    empty.mkdir()
    cfg.save(empty)
    with pytest.raises(FileNotFoundError, match="no safetensors"):
        load_model(empty)
    with pytest.raises(KeyError):
        read_state(tmp_path / "missing", ["model.layers.0.mlp.down_proj.weight"])


def test_training_checkpoint_loads_for_inference(tmp_path):
    """A trainer checkpoint is an inference checkpoint: same names, and the
    loaded model gives the trained model's outputs."""
    m = _tiny()
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.01)
    save_model(m, tmp_path / "ck")
    r = load_model(tmp_path / "ck")
    ids = torch.randint(0, 1000, (1, 12))
    assert torch.equal(m(ids), r(ids))
