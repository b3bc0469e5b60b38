"""CPU oracle tests of the async speculative decoder: greedy output must be
token-identical to target-only AR decoding (tiny pair, fp32)."""
import random

import pytest
import torch

from d3d_b200.config import tiny_drafter, tiny_target
from d3d_b200.engine.backends import TorchDraft, TorchTarget
from d3d_b200.engine.controlled import ControlledAcceptance, expected_commit, rate_for_mean_accept
from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
from d3d_b200.models.qwen3 import build_model


def _prompts(n=4, seed=0, lo=16, hi=64, vocab=1000):
    rng = random.Random(seed)
    return [[rng.randrange(2, vocab) for _ in range(rng.randint(lo, hi))] for _ in range(n)]


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    t = build_model(tiny_target(), seed=0)
    d = build_model(tiny_drafter(), seed=1)
    return t, d


@pytest.mark.parametrize("mode,anchors,conc", [("causal", 1, 1), ("block_causal", 3, 2),
                                               ("causal", 0, 4)])
def test_spec_matches_ar(pair, mode, anchors, conc):
    t, d = pair
    prompts = _prompts()
    ar = ar_generate(TorchTarget(t), prompts, max_new_tokens=32, ignore_eos=True)
    cfg = DecodeConfig(block_size=8, anchor_num=anchors, attention_mask_mode=mode,
                       max_new_tokens=32, ignore_eos=True)
    res = SpecDecoder(TorchTarget(t), TorchDraft(d), cfg).generate(prompts, concurrency=conc)
    for o, ref in zip(res["outputs"], ar["outputs"]):
        assert o.tokens == ref
        assert sum(o.accepts) >= len(o.tokens) - 1


def test_controlled_acceptance_matches_ar_and_rate(pair):
    t, d = pair
    prompts = _prompts(n=3, seed=3)
    ar = ar_generate(TorchTarget(t), prompts, max_new_tokens=48, ignore_eos=True)
    rate = rate_for_mean_accept(4.0, 8)
    assert abs(expected_commit(rate, 8) - 4.0) < 1e-6

    def ctl(i):
        return ControlledAcceptance(oracle=prompts[i] + ar["outputs"][i], rate=rate,
                                    vocab_size=1024, seed=7, stream=i, exclude=(1023,))

    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=48, ignore_eos=True)
    res = SpecDecoder(TorchTarget(t), TorchDraft(d), cfg).generate(prompts, controlled=ctl)
    for o, ref in zip(res["outputs"], ar["outputs"]):
        assert o.tokens == ref
    # every corrupted position is offered as the first alternative → anchors hit
    hits = sum(o.hits for o in res["outputs"])
    assert hits > 0
    assert res["mean_accept_length"] > 2.0


@pytest.mark.parametrize("proposal_top_k", [8, 0])
def test_sampling_runs(pair, proposal_top_k):
    """Sampled decoding with top-k proposals and with proposals from the
    drafter's full distribution (top-k 0, the reference's default)."""
    t, d = pair
    prompts = _prompts(n=2, seed=5)
    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=24, ignore_eos=True,
                       temperature=0.8, top_k=proposal_top_k)
    res = SpecDecoder(TorchTarget(t, temperature=0.8, top_k=0, seed=1), TorchDraft(d, seed=2),
                      cfg).generate(prompts)
    for o in res["outputs"]:
        assert len(o.tokens) == 24
        assert all(0 <= x < 1024 for x in o.tokens)


def test_gate_up_interleave_order():
    """The interleaved gate|up row order is a permutation that puts gate row
    64t+16w+j and its up row in lanes j and j+16 of warp w of tile t."""
    from d3d_b200 import ops
    i = 384
    order = ops.gate_up_order(i)
    assert sorted(order.tolist()) == list(range(2 * i))
    for t in range(2 * i // 128):
        for w in range(4):
            for j in range(16):
                r = 128 * t + 32 * w + j
                assert order[r] == 64 * t + 16 * w + j
                assert order[r + 16] == i + 64 * t + 16 * w + j
    g = torch.randn(i, 64).to(torch.bfloat16)
    u = torch.randn(i, 64).to(torch.bfloat16)
    pw = ops.pack_gate_up(g, u)
    full = torch.cat([g, u], 0)
    assert torch.equal(pw.unpack(), full[order])


class _SameStream:
    """Stands in for a CUDA stream shared by target and drafter."""


def _pipelined_pair():
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.backends import TorchDraft, TorchTarget
    from d3d_b200.models.qwen3 import build_model
    stream = _SameStream()

    class Target(TorchTarget):
        supports_gather = True

        def __init__(self, m):
            super().__init__(m)
            self.stream = stream
            self.gathers = 0
            self.pipelined = 0

        def submit_verify(self, seqs, blocks, q=None, gather=None):
            self.pipelined += gather is not None
            blocks = blocks.clone()
            for src, dst, rows in gather or ():
                blocks.view(-1)[torch.tensor(dst)] = src[torch.tensor(rows), 0]
                self.gathers += 1
            super().submit_verify(seqs, blocks, q)

    class Handle:
        def __init__(self, out):
            self.out, self.dev_top = out, out["dev_top"]

        def result(self):
            return self.out

    class Draft(TorchDraft):
        supports_async = True

        def __init__(self, m):
            super().__init__(m)
            self.stream = stream

        def forward(self, seqs, ids, positions, rows, *, store, topk, cond_rows=None, sample=None,
                    wait=True):
            out = super().forward(seqs, ids, positions, rows, store=store, topk=topk, cond_rows=cond_rows,
                                  sample=sample)
            b, q = out["greedy"].shape
            out["dev_top"] = (out["top"] if "top" in out else out["greedy"][..., None]).reshape(b * q, -1)
            return out if wait else Handle(out)

    return Target(build_model(tiny_target(), seed=0)), Draft(build_model(tiny_drafter(cond=True), seed=1))


@pytest.mark.parametrize("controlled", [False, True])
def test_pipelined_coordinator_matches_ar(controlled):
    """The pipelined step (next verify submitted before the draft is read,
    drafts gathered from the in-flight output or rewritten by the controlled
    injection) keeps greedy token identity."""
    from d3d_b200.engine.backends import TorchTarget
    from d3d_b200.engine.controlled import ControlledAcceptance, rate_for_mean_accept
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.config import tiny_target
    from d3d_b200.models.qwen3 import build_model
    tgt, drf = _pipelined_pair()
    rng = random.Random(9)
    prompts = [[rng.randrange(2, 1000) for _ in range(rng.randint(16, 48))] for _ in range(3)]
    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=40, ignore_eos=True)
    ref = ar_generate(TorchTarget(build_model(tiny_target(), seed=0)), prompts, 40, ignore_eos=True)["outputs"]
    ctl = None
    if controlled:
        rate = rate_for_mean_accept(4.0, 8)
        ctl = lambda i: ControlledAcceptance(prompts[i] + ref[i], rate, 1024, stream=i, exclude=(1023,))
    dec = SpecDecoder(tgt, drf, cfg)
    assert dec._pipelined()
    res = dec.generate(prompts, concurrency=3, controlled=ctl)
    assert [o.tokens for o in res["outputs"]] == ref
    if controlled:
        assert tgt.pipelined > 0


def test_device_rows_reproduce_selected_branch():
    """The rows ``_Outcomes.device_rows`` hands to the device gather hold the
    same drafts as the host-side branch (``_Outcomes.get``)."""
    from d3d_b200.engine.layout import branch_specs, packed_layout
    from d3d_b200.engine.spec import _Outcomes
    k = 8
    cur = torch.arange(100, 100 + k)
    top = torch.stack([cur, cur + 50], 1)
    lays = [packed_layout(cur + 3 * i, branch_specs((cur + 3 * i).tolist(), top.tolist(), 1), 40, k, 999, "causal")
            for i in range(2)]
    q = lays[0].q_len
    greedy = torch.randint(0, 1000, (2, q))
    out = {"greedy": greedy, "top": torch.stack([greedy, greedy + 1], -1),
           "dev_top": torch.stack([greedy, greedy + 1], -1).reshape(2 * q, 2)}
    for i, lay in enumerate(lays):
        oc = _Outcomes(lay, out, i, q)
        for key in lay.keys:
            blk = oc.get(key)[0]
            src, rows = oc.device_rows(key)
            assert torch.equal(src[torch.tensor(rows), 0], blk[1:])


def test_per_request_budgets_and_closed_loop_ar():
    """Per-request output budgets: speculative output matches closed-loop AR
    with the same budgets, and every request stops at its own budget."""
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.backends import TorchDraft, TorchTarget
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.models.qwen3 import build_model
    rng = random.Random(4)
    prompts = [[rng.randrange(2, 1000) for _ in range(rng.randint(12, 30))] for _ in range(4)]
    budgets = [5, 17, 9, 1]
    tgt = TorchTarget(build_model(tiny_target(), seed=0))
    drf = TorchDraft(build_model(tiny_drafter(cond=True), seed=1))
    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=32, ignore_eos=True)
    res = SpecDecoder(tgt, drf, cfg).generate(prompts, concurrency=2, max_new=budgets)
    ar = ar_generate(tgt, prompts, 32, ignore_eos=True, concurrency=3, max_new=budgets)["outputs"]
    assert [len(o.tokens) for o in res["outputs"]] == budgets
    assert [o.tokens for o in res["outputs"]] == ar


def test_serve_cli_tiny_pair(tmp_path):
    from d3d_b200.cli import serve
    rows = serve.main(["--target", "tiny-target", "--draft", "tiny-drafter", "--device", "cpu",
                       "--pages", "256", "--concurrency", "1,2", "--max-new-tokens-range", "6,14",
                       "--block-size", "8", "--max-samples", "3", "--prompt-min", "10", "--prompt-max", "20",
                       "--validate", "--ignore-eos", "--output-json", str(tmp_path / "s.json")])
    assert [r["concurrency"] for r in rows] == [1, 2]
    assert all(r["token_identical_to_ar"] for r in rows)


def test_serve_cli_datasets_repeats_and_fast_backup(tmp_path):
    """Several prompt sources in one run, repeated cells, and both fast-miss
    policies (shallow drafts with their own anchor count, and full-depth
    ``fast_legacy``) stay token-identical to AR."""
    import json
    from d3d_b200.cli import serve
    src = tmp_path / "p.jsonl"
    src.write_text("\n".join(json.dumps({"input_ids": list(range(5 + i, 17 + i))}) for i in range(3)))
    for backup, extra in (("fast", ["--fast-miss-anchors", "2"]), ("fast_legacy", [])):
        out = tmp_path / f"{backup}.json"
        rows = serve.main(["--target", "tiny-target", "--draft", "tiny-drafter", "--device", "cpu",
                           "--pages", "256", "--concurrency", "2", "--max-new-tokens", "12", "--block-size", "8",
                           "--anchor-num", "1", "--max-samples", "2", "--prompt-min", "10", "--prompt-max", "20",
                           "--datasets", "synthetic", str(src), "--repeats", "2", "--backup", backup, *extra,
                           "--validate", "--validate-draft", "--ignore-eos", "--output", str(out)])
        assert [(r["dataset"], r["repeat"]) for r in rows] == [("synthetic", 0), ("synthetic", 1),
                                                                (str(src), 0), (str(src), 1)]
        assert all(r["token_identical_to_ar"] for r in rows)
        d = json.loads(out.read_text())
        assert d["config"]["backup"] == backup and len(d["rows"]) == 4
        assert d["draft_validation"]["agreement"] == 1.0
    with pytest.raises(SystemExit):
        serve.main(["--target", "tiny-target", "--draft", "tiny-drafter", "--device", "cpu", "--repeats", "0"])


def test_single_cli_controlled_with_stage_timings(tmp_path):
    """The single-request CLI in controlled mode on the tiny pair (the
    corruption draws stay inside the model's vocabulary) with stage timings."""
    import json
    from d3d_b200.cli import single
    out = tmp_path / "single.json"
    single.main(["--verifier", "tiny-target", "--drafter", "tiny-drafter", "--device", "cpu",
                 "--max-new-tokens", "12", "--block-size", "8", "--anchor-num", "1", "--max-samples", "2",
                 "--prompt-min", "8", "--prompt-max", "16", "--baseline", "--controlled-accept-mean", "3",
                 "--collect-stage-timings", "--ignore-eos", "--warmup-new-tokens", "4",
                 "--output-json", str(out)])
    d = json.loads(out.read_text())
    assert d["summary"]["token_identical_to_ar"] is True
    assert "host_ms" in d["summary"]["stage_timings"]


def test_single_cli_verifier_process(tmp_path):
    """The single-request CLI with the target in its own process (the
    reference's verifier process; here the ``gloo`` host link on CPU): greedy
    output is token-identical to AR decoding through the same remote target,
    and a sampled run sends the drafts' sparse proposals in its requests."""
    import json
    from d3d_b200.cli import single
    base = ["--verifier", "tiny-target", "--drafter", "tiny-drafter", "--device", "cpu", "--verifier-process",
            "--max-new-tokens", "12", "--block-size", "8", "--anchor-num", "1", "--max-samples", "2",
            "--prompt-min", "8", "--prompt-max", "16", "--ignore-eos", "--warmup-new-tokens", "4"]
    out = tmp_path / "pair.json"
    summ = single.main(base + ["--drafter-tag", "tiny", "--verbose", "--output-json", str(out)])
    assert summ["layout"] == "verifier_process" and summ["token_identical_to_ar"] is True
    assert summ["async"]["verify_steps"] == sum(v["count"] for v in summ["async"]["sources"].values())
    d = json.loads(out.read_text())
    assert len(d["per_prompt"]) == 2 and all(len(x["tokens"]) == 12 for x in d["per_prompt"])
    sampled = ["--no-baseline", "--temperature", "0.8", "--proposal-top-k", "8", "--target-top-k", "20",
               "--sample-index", "1"]
    outs = []
    for extra in (["--verifier-process"], []):
        out = tmp_path / f"sampled{len(extra)}.json"
        args = [x for x in base if x != "--verifier-process"] + extra + sampled + ["--output-json", str(out)]
        summ = single.main(args)
        assert summ["token_identical_to_ar"] is None
        outs.append([x["tokens"] for x in json.loads(out.read_text())["per_prompt"]])
    # same seeds on both sides: the remote target draws exactly what a local one does
    assert outs[0] == outs[1] and len(outs[0]) == 1
    with pytest.raises(SystemExit):
        single.main(base + ["--denoising-steps", "2"])


def test_gemm_policies():
    """Token tiles and split-K choices: tiles cover the tokens within the MMA
    limits, and the target's split depends on the weight shape only."""
    from d3d_b200 import ops
    for m in (1, 15, 16, 17, 255, 256, 257, 272, 511, 512, 513, 1088, 4096):
        bt = ops.bt_for(m)
        assert bt % 16 == 0 and 16 <= bt <= 512
        if bt > 256:
            assert bt % 32 == 0
        tiles = -(-m // bt)
        assert tiles * bt >= m and (tiles - 1) * bt < m
    for n, k in ((6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288), (151936, 4096)):
        s = ops.splitk_for(n, k, mtiles=1, bt=16)
        assert 1 <= s <= 16 and (k // 64) // s >= 4 or s == 1
        assert s == ops.splitk_for(n, k, mtiles=1, bt=16)
    # the drafter cap keeps fp32 partials no larger than the weight
    s = ops.splitk_for(2048, 2048, mtiles=1, bt=288, m=272)
    assert s * 272 * 2048 * 4 <= 2048 * 2048 * 2 * 2


@pytest.mark.parametrize("miss_anchors", [0, 3])
def test_fast_backup_on_misses_keeps_token_identity(miss_anchors):
    """backup="fast": a miss verifies [anchor, random...] immediately (no
    redraft) and seeds the next step's branches off the critical path (a
    shallow packed forward: commit-1 outcomes only, ``fast_miss_anchors``
    anchors); greedy output still equals AR."""
    from d3d_b200.config import tiny_drafter, tiny_target
    from d3d_b200.engine.backends import TorchDraft, TorchTarget
    from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, ar_generate
    from d3d_b200.models.qwen3 import build_model
    rng = random.Random(12)
    prompts = [[rng.randrange(2, 1000) for _ in range(rng.randint(12, 30))] for _ in range(3)]
    tgt = TorchTarget(build_model(tiny_target(), seed=0))
    drf = TorchDraft(build_model(tiny_drafter(cond=True), seed=1))
    cfg = DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=40, ignore_eos=True, backup="fast",
                       fast_miss_anchors=miss_anchors)
    dec = SpecDecoder(tgt, drf, cfg)
    shapes = []
    orig = dec.d.forward

    def spy(group, ids, *a, **k):
        shapes.append(tuple(ids.shape))
        return orig(group, ids, *a, **k)
    dec.d.forward = spy
    res = dec.generate(prompts, concurrency=2)
    fan = miss_anchors or 1
    assert (1, 8 + fan * 8) in shapes or (2, 8 + fan * 8) in shapes    # a shallow packed forward ran
    ar = ar_generate(tgt, prompts, 40, ignore_eos=True)["outputs"]
    assert [o.tokens for o in res["outputs"]] == ar
    assert any("fast_backup" in o.sources for o in res["outputs"])
    with pytest.raises(ValueError):
        DecodeConfig(backup="fast", temperature=0.7, top_k=2).validate()


def test_full_support_proposals_are_lossless():
    """``pq_accept_sparse`` with proposals over the whole vocabulary (the
    support is every token): the first token it emits follows the target's
    distribution whatever the proposal, checked with a chi-square bound."""
    import math
    from d3d_b200.engine.sampling import pq_accept_sparse
    g = torch.Generator().manual_seed(3)
    V, K, B = 12, 3, 40000
    p = torch.softmax(torch.randn(K, V, generator=g) * 1.5, -1)
    q = torch.softmax(torch.randn(K - 1, V, generator=g) * 1.5, -1)
    drafts = torch.stack([torch.multinomial(q[i], B, replacement=True, generator=g) for i in range(K - 1)], 1)
    blocks = torch.cat([torch.full((B, 1), 5), drafts], 1)
    q_ids = torch.arange(V).expand(B, K - 1, V)
    q_probs = q.expand(B, K - 1, V)
    u = torch.rand(B, K - 1, generator=g)
    cu = torch.rand(B, generator=g)
    commit, corr = pq_accept_sparse(blocks, p.expand(B, K, V), q_ids, q_probs, u, cu)
    first = torch.where(commit >= 2, blocks[:, 1], corr)
    counts = torch.bincount(first, minlength=V).double()
    exp = p[0].double() * B
    chi = (((counts - exp) ** 2) / exp).sum().item()
    dof = V - 1
    assert chi < dof + 6 * math.sqrt(2 * dof), chi


def test_call_budget_does_not_change_the_engine_default(pair):
    """A per-call ``max_new_tokens`` (a short warm-up, say) leaves the
    engine's configured budget for later calls."""
    from d3d_b200.api import D3DEngine
    t, d = pair
    eng = D3DEngine.from_modules(t, d, DecodeConfig(block_size=8, anchor_num=1, max_new_tokens=20,
                                                    ignore_eos=True))
    prompts = _prompts(n=1, seed=9)
    assert len(eng.generate(prompts, max_new_tokens=5)["outputs"][0].tokens) == 5
    assert len(eng.generate(prompts)["outputs"][0].tokens) == 20


def test_draft_validation_against_oracle_module():
    """The engine's drafter agrees with its own oracle module exactly; a
    perturbed oracle is reported (recovery block or packed tokens differ)."""
    import copy
    from d3d_b200.engine.validation import validate_draft
    tgt = TorchTarget(build_model(tiny_target(), seed=0))
    dm = build_model(tiny_drafter(cond=True), seed=1)
    dec = SpecDecoder(tgt, TorchDraft(dm), DecodeConfig(block_size=8, anchor_num=2, max_new_tokens=16))
    prompt = list(range(30, 60))
    r = validate_draft(dec, copy.deepcopy(dm), prompt)
    assert r["recovery_equal"] and r["agreement"] == 1.0 and r["candidate_keys"] > 8
    bad = copy.deepcopy(dm)
    with torch.no_grad():
        for p in bad.model.layers[-1].parameters():
            p.add_(torch.randn_like(p) * 0.5)
    with pytest.raises(RuntimeError, match="differs materially"):
        validate_draft(dec, bad, prompt)


@pytest.mark.parametrize("counts", [None, (1, 3)])
def test_unanchored_outcomes_keep_token_identity(counts):
    """``anchor_num=0``: each commit length drafts one unanchored outcome whose
    first token is replaced by the target's correction on reuse
    (``single/eval_async_packed.py:1797-1803``); output equals AR and the
    outcomes are reused."""
    tgt = TorchTarget(build_model(tiny_target(), seed=0))
    drf = TorchDraft(build_model(tiny_drafter(cond=True), seed=1))
    rng = random.Random(3)
    prompts = [[rng.randrange(2, 1000) for _ in range(rng.randint(10, 30))] for _ in range(3)]
    cfg = DecodeConfig(block_size=8, anchor_num=0, max_new_tokens=24, ignore_eos=True,
                       packed_accepted_counts=counts)
    r = SpecDecoder(tgt, drf, cfg).generate(prompts, concurrency=2)
    assert [o.tokens for o in r["outputs"]] == ar_generate(tgt, prompts, 24, ignore_eos=True)["outputs"]
    assert sum(o.hits for o in r["outputs"]) > 0
