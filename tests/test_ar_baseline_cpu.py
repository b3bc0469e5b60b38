"""AR baseline accounting against a fake target that emits ``previous + 1``:
token counts, stop reasons, admission, batch sizes and the decode-only
boundary (the prefill's token excluded) of both AR paths."""
import torch

from d3d_b200.engine.backends import TargetBackend, VerifyResult
from d3d_b200.engine.spec import ar_decode_fixed, ar_generate


class _Fake(TargetBackend):
    hidden_size = 4

    def __init__(self):
        self.live, self.verifies, self.prefills = set(), 0, []
        self._pending = None

    def prefill(self, seqs):
        self.prefills.append(len(seqs))
        for s in seqs:
            self.live.add(s.index)
        return torch.tensor([100 + s.index * 1000 for s in seqs]), None

    def submit_verify(self, seqs, blocks, q=None):
        self._pending = blocks

    def receive(self):
        b, self._pending = self._pending, None
        self.verifies += 1
        nxt = b[:, -1] + 1
        return VerifyResult(torch.ones(b.shape[0], dtype=torch.long), nxt, nxt[:, None], None)

    def release(self, seq):
        self.live.discard(seq.index)


def test_ar_generate_accounting_and_eos():
    t = _Fake()
    prompts = [[1, 2, 3]] * 6
    r = ar_generate(t, prompts, 5, eos=(1103,), concurrency=4)
    assert r["outputs"][0] == [100, 101, 102, 103, 104]
    assert r["outputs"][1] == [1100, 1101, 1102, 1103]             # stops at (and keeps) the stop token
    assert r["finish_reasons"][:2] == ["length", "eos"]
    assert r["max_active"] == 4 and max(r["decode_batch_sizes"]) == 4 and not t.live
    assert r["output_tokens"] == sum(len(o) for o in r["outputs"])
    assert t.prefills[0] == 4 and sum(t.prefills) == 6            # prefill groups of at most 4
    assert len(r["decode_s"]) == 6 and all(d >= 0 for d in r["decode_s"])


def test_fixed_batch_decode_excludes_the_prefill_token():
    t = _Fake()
    r = ar_decode_fixed(t, [[1, 2]] * 3, 4, capture=True)
    assert r["tokens"] == 12 and t.verifies == 4 and not t.live
    assert r["outputs"][2] == [2100, 2101, 2102, 2103, 2104]
