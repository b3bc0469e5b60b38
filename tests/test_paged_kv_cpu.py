"""Page allocator of the paged KV cache (host logic, runs on CPU): reserve
grows a sequence's table and mirrors it into the block table, trim returns
pages past a length, release frees everything, physical slots follow the
table, the scratch page is held outside every sequence, and nothing leaks."""
import pytest
import torch

from d3d_b200.config import tiny_target
from d3d_b200.models.fast import PagedKV


def test_reserve_trim_release_slots_and_scratch():
    kv = PagedKV(tiny_target(), num_pages=10, page_size=4, max_seqs=3, max_pages_per_seq=5, device="cpu")
    kv.reserve(7, 0, 9)                       # 3 pages
    kv.reserve(8, 1, 4)                       # 1 page
    assert len(kv.tables[7]) == 3 and len(kv.tables[8]) == 1 and len(kv.free) == 6
    assert kv.block_table[0, :3].tolist() == kv.tables[7]
    slots = kv.slots(7, 2, 5).tolist()        # logical positions 2..6 span pages 0 and 1
    t = kv.tables[7]
    assert slots == [t[0] * 4 + 2, t[0] * 4 + 3, t[1] * 4, t[1] * 4 + 1, t[1] * 4 + 2]
    kv.reserve(7, 0, 6)                       # already covered: nothing changes
    assert len(kv.tables[7]) == 3
    kv.trim(7, 0, 5)                          # keep ceil(5/4) = 2 pages
    assert len(kv.tables[7]) == 2 and len(kv.free) == 7
    s = kv.scratch_slot()
    assert s % 4 == 0 and kv.scratch_slot() == s and len(kv.free) == 6
    assert kv.leaked == 0
    with pytest.raises(RuntimeError, match="max_pages_per_seq"):
        kv.reserve(8, 1, 4 * 6)
    with pytest.raises(RuntimeError, match="out of KV pages"):
        kv.reserve(9, 2, 4 * 5)
        kv.reserve(10, 2, 4 * 5)
    for sid in list(kv.tables):
        kv.release(sid)
    assert kv.tables == {} and kv.leaked == 0 and len(kv.free) + len(kv.scratch) == kv.num_pages
    assert kv.k[0].shape == (10 * 4, tiny_target().num_key_value_heads, tiny_target().head_dim)
    assert kv.k[0].dtype == torch.bfloat16


def test_fast_weights_round_trip_to_module():
    """Kernel-layout weights back to a PyTorch module (tiles unpacked, gate|up
    rows re-ordered, folded norm scales divided out) equal the source within
    bf16 rounding."""
    import torch
    from d3d_b200.config import tiny_drafter
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.models.qwen3 import build_model
    m = build_model(tiny_drafter(cond=True), seed=3)
    with torch.no_grad():
        for L in m.model.layers:
            L.input_layernorm.weight.mul_(1.5)
            L.post_attention_layernorm.weight.add_(0.25)
    fw = FastWeights.from_module(m, "cpu")
    for fold in (False, True):
        if fold:
            fw.fold_norms()
        back = fw.to_module(dtype=torch.float32)
        sa, sb = m.state_dict(), back.state_dict()
        assert sa.keys() == sb.keys()
        for k in sa:
            scale = sa[k].float().abs().max().item() + 1e-9
            assert (sa[k].float() - sb[k].float()).abs().max().item() <= 1e-2 * scale, k
