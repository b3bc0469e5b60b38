"""The kernel-backed engine: greedy speculative output is token-identical to
AR decoding on the same kernels, and the kernel forward tracks the fp32 oracle."""
import random

import pytest
import torch

from d3d_b200.config import tiny_drafter, tiny_target
from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
from d3d_b200.models.qwen3 import build_model

pytestmark = pytest.mark.gpu


def _prompts(n=4, seed=0, lo=16, hi=64, vocab=1000):
    rng = random.Random(seed)
    return [[rng.randrange(2, vocab) for _ in range(rng.randint(lo, hi))] for _ in range(n)]


@pytest.fixture(scope="module")
def fast_pair():
    from d3d_b200.models.fast import FastWeights
    t = build_model(tiny_target(), seed=0)
    d = build_model(tiny_drafter(), seed=1)
    return t, d, FastWeights.from_module(t), FastWeights.from_module(d)


def _backends(tw, dw, graphs=True):
    from d3d_b200.engine.fast import FastDraft, FastTarget
    return (FastTarget(tw, pages=512, max_seqs=8, max_context=512, use_graphs=graphs),
            FastDraft(dw, pages=2048, max_seqs=8, max_context=512, packed_q=1024, use_graphs=graphs))


@pytest.mark.parametrize("mode,anchors,conc,graphs", [("causal", 1, 1, True), ("block_causal", 3, 2, True),
                                                      ("causal", 0, 4, False)])
def test_fast_spec_matches_fast_ar(fast_pair, mode, anchors, conc, graphs):
    _, _, tw, dw = fast_pair
    prompts = _prompts()
    t, d = _backends(tw, dw, graphs)
    ar = ar_generate(t, prompts, max_new_tokens=40, ignore_eos=True, concurrency=conc)
    cfg = DecodeConfig(block_size=8, anchor_num=anchors, attention_mask_mode=mode,
                       max_new_tokens=40, ignore_eos=True)
    res = SpecDecoder(t, d, cfg).generate(prompts, concurrency=conc)
    for o, ref in zip(res["outputs"], ar["outputs"]):
        assert o.tokens == ref
    assert len(t.kv.tables) == 0 and len(d.kv.tables) == 0
    # every page is free again, apart from the target's scratch page (placeholder KV stores)
    assert len(t.kv.free) + len(t.kv.scratch) == t.kv.num_pages and len(d.kv.free) == d.kv.num_pages
    assert t.kv.leaked == 0 and d.kv.leaked == 0


def test_fast_forward_tracks_oracle(fast_pair):
    from d3d_b200.engine.backends import SeqState
    t, _, tw, dw = fast_pair
    tgt, _ = _backends(tw, dw, graphs=False)
    prompts = _prompts(n=3, seed=4)
    seqs = [SeqState(index=i, prompt=p, prefix=len(p)) for i, p in enumerate(prompts)]
    anchors, hid = tgt.prefill(seqs)
    for i, p in enumerate(prompts):
        ids = torch.tensor([p])
        h = t(ids)[0, -1]
        ref_a = int(t.logits(h).argmax())
        rel = (hid[i].float().cpu() - h).norm() / h.norm()
        assert rel < 0.05, rel
        assert int(anchors[i]) == ref_a


@pytest.mark.parametrize("controlled", [False, True])
def test_pipelined_shared_stream_matches_ar(fast_pair, controlled):
    """Target and drafter on one stream: each verify is enqueued behind the
    drafter forward still in flight, its drafts gathered on the device (or
    rewritten on the host in controlled mode); output equals AR."""
    from d3d_b200.engine.controlled import ControlledAcceptance, rate_for_mean_accept
    from d3d_b200.engine.fast import FastDraft, FastTarget
    _, _, tw, dw = fast_pair
    t = FastTarget(tw, pages=512, max_seqs=8, max_context=512)
    d = FastDraft(dw, pages=2048, max_seqs=8, max_context=512, packed_q=1024, stream=t.stream)
    prompts = _prompts(n=3, seed=7)
    ar = ar_generate(t, prompts, max_new_tokens=48, ignore_eos=True)["outputs"]
    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=48, ignore_eos=True)
    dec = SpecDecoder(t, d, cfg)
    assert dec._pipelined()
    ctl = None
    if controlled:
        rate = rate_for_mean_accept(4.0, 8)
        ctl = lambda i: ControlledAcceptance(prompts[i] + ar[i], rate, 1024, stream=i, exclude=(1023,))
    res = dec.generate(prompts, concurrency=3, controlled=ctl)
    for o, ref in zip(res["outputs"], ar):
        assert o.tokens == ref
    if controlled:
        assert sum(sum(o.accepts) for o in res["outputs"]) / sum(len(o.accepts) for o in res["outputs"]) > 2.0


def test_sampled_kernel_path(fast_pair):
    """Sampled speculative decoding on the kernels: runs end to end with
    top-k (<= 4) proposals and target truncation, and at a temperature near
    zero reproduces greedy AR decoding token for token."""
    from d3d_b200.api import D3DEngine
    _, _, tw, dw = fast_pair
    prompts = _prompts(n=2, seed=11)
    greedy = D3DEngine.from_weights(tw, dw, DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=32,
                                                         ignore_eos=True), max_seqs=4, max_context=512)
    ar = greedy.generate_ar(prompts)["outputs"]
    cold = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=32, ignore_eos=True, temperature=2e-5,
                        top_k=2, target_top_k=2)
    eng = D3DEngine.from_weights(tw, dw, cold, max_seqs=4, max_context=512)
    out = eng.generate(prompts)["outputs"]
    assert [o.tokens for o in out] == ar
    warm = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=32, ignore_eos=True, temperature=0.8,
                        top_k=4, target_top_k=4, top_p=0.95, target_top_p=0.95)
    eng2 = D3DEngine.from_weights(tw, dw, warm, max_seqs=4, max_context=512)
    res = eng2.generate(prompts)
    for o in res["outputs"]:
        assert len(o.tokens) == 32 and all(0 <= t < 1024 for t in o.tokens)
    sar = eng2.generate_ar(prompts)["outputs"]
    assert all(len(t) == 32 for t in sar)


def test_full_vocab_sampled_verify_is_lossless():
    """Full-vocabulary sampled verification on the kernel path (target
    top_k = 0): with each draft sampled from the proposal q, the token
    emitted at the first drafted position (the draft if accepted, else the
    residual correction) follows the target distribution p exactly --
    checked against p with a chi-square bound over many draws."""
    import math
    import torch
    from d3d_b200.config import tiny_target
    from d3d_b200.engine.fast import FastTarget
    from d3d_b200.models.fast import FastWeights
    from d3d_b200.models.qwen3 import build_model
    dev = torch.device("cuda")
    tgt = FastTarget(FastWeights.from_module(build_model(tiny_target(), seed=0), dev), pages=64, max_seqs=2,
                     max_context=128, device=dev, temperature=1.0, top_k=0, seed=3)
    assert tgt.full_vocab
    K, V = 4, tgt.cfg.vocab_size
    b = tgt.runner.buffers(1, K, -1)
    a = tgt._abufs(1, K)
    g = torch.Generator(device=dev).manual_seed(0)
    logits = torch.randn(K, V, device=dev, generator=g) * 2.0
    b.logits.copy_(logits)
    p0 = torch.softmax(logits[0], -1)
    # proposal q over four ids (a plausible token and three others); each
    # trial's draft is sampled from q, as the drafter does
    support = [int(p0.argsort(descending=True)[3]), 11, 12, 13]
    qw = torch.tensor([0.6, 0.2, 0.1, 0.1])
    q_ids = torch.tensor([[support] * (K - 1)])
    q_p = qw.expand(1, K - 1, 4).clone()
    n = 20000
    drafts = torch.multinomial(qw, n, replacement=True, generator=torch.Generator().manual_seed(1))
    out = torch.empty(n, dtype=torch.long)
    ids = b.ids.view(1, K)
    for i in range(n):
        x1 = support[int(drafts[i])]
        ids.copy_(torch.tensor([[5, x1, 7, 9]]), non_blocking=True)
        tgt._sampled_accept(b, a, (q_ids, q_p))
        commit, corr = int(a["commit"][0]), int(a["corr"][0])
        out[i] = x1 if commit >= 2 else corr
    counts = torch.bincount(out, minlength=V).double()
    exp = p0.double().cpu() * n
    big = exp >= 20
    chi = (((counts[big] - exp[big]) ** 2) / exp[big]).sum().item()
    rest_o, rest_e = counts[~big].sum().item(), exp[~big].sum().item()
    chi += (rest_o - rest_e) ** 2 / max(rest_e, 1e-9)
    dof = int(big.sum()) + 1
    assert chi < dof + 6 * math.sqrt(2 * dof), (chi, dof)


def test_full_vocab_sampled_decoding_runs():
    import torch
    from d3d_b200.api import D3DEngine
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.spec import DecodeConfig
    from d3d_b200.models.qwen3 import build_model
    dev = torch.device("cuda")
    eng = D3DEngine.from_modules(build_model(tiny_target(), seed=0, device=dev),
                                 build_model(tiny_drafter(), seed=1, device=dev),
                                 DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=24, ignore_eos=True,
                                              temperature=0.8, top_k=4, target_top_k=0),
                                 max_seqs=2, max_context=256)
    assert eng.target.full_vocab
    out = eng.generate([[3, 4, 5, 6, 7, 8, 9, 10]])["outputs"][0]
    assert len(out.tokens) == 24 and all(0 <= t < tiny_target().vocab_size for t in out.tokens)
