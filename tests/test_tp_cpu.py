"""Tensor-parallel weight sharding (host side): the shards reassemble into
the full weights and the per-rank shapes follow the column/row split."""
import pytest
import torch


def test_local_config_and_shards_reassemble():
    from d3d_b200 import ops
    from d3d_b200.config import tiny_target
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.tp import local_config, shard_weights
    cfg = tiny_target()
    lc = local_config(cfg, 2)
    assert (lc.num_attention_heads, lc.num_key_value_heads, lc.intermediate_size, lc.vocab_size) == \
        (cfg.num_attention_heads // 2, cfg.num_key_value_heads // 2, cfg.intermediate_size // 2, cfg.vocab_size // 2)
    with pytest.raises(ValueError):
        local_config(cfg, 3)
    full = FastWeights.from_module(build_model(cfg, seed=0), "cpu")
    sh = [shard_weights(full, 2, r) for r in range(2)]
    d, hq, hkv, I = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    L, L0, L1 = full.layers[0], sh[0].layers[0], sh[1].layers[0]
    qkv = L.qkv.unpack()
    qs, ks = hq * d, hkv * d
    q0, q1 = L0.qkv.unpack(), L1.qkv.unpack()
    lq = lc.num_attention_heads * d
    assert torch.equal(torch.cat([q0[:lq], q1[:lq]]), qkv[:qs])
    assert torch.equal(torch.cat([L0.o.unpack(), L1.o.unpack()], 1), L.o.unpack())
    assert torch.equal(torch.cat([L0.down.unpack(), L1.down.unpack()], 1), L.down.unpack())
    gu = torch.empty(2 * I, cfg.hidden_size, dtype=torch.bfloat16)
    gu[ops.gate_up_order(I)] = L.gate_up.unpack()
    il = lc.intermediate_size
    g0 = torch.empty(2 * il, cfg.hidden_size, dtype=torch.bfloat16)
    g0[ops.gate_up_order(il)] = L0.gate_up.unpack()
    assert torch.equal(g0[:il], gu[:il]) and torch.equal(g0[il:], gu[I:I + il])
    assert torch.equal(torch.cat([sh[0].lm_head.unpack(), sh[1].lm_head.unpack()]), full.lm_head.unpack())


def test_random_shard_shapes():
    """A directly drawn shard has the per-rank shapes and a full, replicated
    embedding identical on every rank."""
    from d3d_b200.config import tiny_target
    from d3d_b200.parallel.tp import local_config, random_shard
    cfg = tiny_target().replace(tie_word_embeddings=False)
    lc = local_config(cfg, 2)
    s0 = random_shard(cfg, 2, 0, seed=3, device="cpu")
    s1 = random_shard(cfg, 2, 1, seed=3, device="cpu")
    d = cfg.head_dim
    assert s0.layers[0].qkv.shape == ((lc.num_attention_heads + 2 * lc.num_key_value_heads) * d, cfg.hidden_size)
    assert s0.layers[0].o.shape == (cfg.hidden_size, lc.num_attention_heads * d)
    assert s0.layers[0].gate_up.shape == (2 * lc.intermediate_size, cfg.hidden_size)
    assert s0.layers[0].down.shape == (cfg.hidden_size, lc.intermediate_size)
    assert s0.lm_head.shape == (cfg.vocab_size // 2, cfg.hidden_size)
    assert s0.embed.shape == (cfg.vocab_size, cfg.hidden_size)
    assert torch.equal(s0.embed, s1.embed)
    assert not torch.equal(s0.layers[0].qkv.data, s1.layers[0].qkv.data)


def test_sliced_checkpoint_shards_equal_sharded_full_weights(tmp_path):
    """Reading one rank's slices from the safetensors checkpoint gives the
    same kernel weights as loading everything and sharding."""
    from d3d_b200.api import load_target_shard
    from d3d_b200.checkpoint import save_model
    from d3d_b200.config import tiny_target
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.models.qwen3 import build_model
    from d3d_b200.parallel.tp import shard_weights
    for tied in (False, True):
        cfg = tiny_target().replace(tie_word_embeddings=tied)
        m = build_model(cfg, seed=5)
        d = tmp_path / f"ck{int(tied)}"
        save_model(m, d)
        full = FastWeights.from_module(m, "cpu")
        for r in range(2):
            a = load_target_shard(str(d), 2, r, device="cpu")
            b = shard_weights(full, 2, r)
            for la, lb in zip(a.layers, b.layers):
                for name in ("qkv", "o", "gate_up", "down"):
                    assert torch.equal(getattr(la, name).data, getattr(lb, name).data), (tied, r, name)
            assert torch.equal(a.lm_head.data, b.lm_head.data)
            assert torch.equal(a.embed, b.embed)
