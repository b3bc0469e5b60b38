"""The drafter-side device branch select (``select_send`` in
``ops/csrc/handoff.cu``) decides from the table the coordinator builds
(``SpecDecoder._arm_select``).  Restated here in Python exactly as the
kernel reads that table, it must send the next VERIFY exactly when the
host loop would continue every row on a drafted branch, and with the same
blocks -- for random outcomes, stop tokens, output budgets and controlled
acceptance."""
import random

import torch

from d3d_b200.engine.backends import SeqState
from d3d_b200.engine.controlled import ControlledAcceptance
from d3d_b200.engine.layout import branch_specs, packed_layout
from d3d_b200.engine.spec import DecodeConfig, SpecDecoder, _Outcomes

MASK = 999


class _FakeTarget:
    supports_select = True

    def __init__(self):
        self.calls = []

    def arm_select(self, B, K, nk, a0, n_eos, ctrl, top, tab):
        self.calls.append(dict(B=B, K=K, nk=nk, a0=a0, n_eos=n_eos, ctrl=ctrl, top=top, tab=list(tab)))
        return True


class _FakeDraft:
    mask_id = MASK


def _kernel(call, reply):
    """The select_send kernel's decision and request, from its table."""
    B, K, nk, a0, n_eos, ctrl, top, tab = (call[k] for k in ("B", "K", "nk", "a0", "n_eos", "ctrl", "top", "tab"))
    sid, prefix, n_limit = tab[:B], tab[B:2 * B], tab[2 * B:3 * B]
    keys = tab[3 * B:3 * B + B * nk * 2]
    key_rows = tab[3 * B + B * nk * 2:3 * B + B * nk * 3]
    eos = tab[3 * B + B * nk * 3:3 * B + B * nk * 3 + n_eos]
    ctl = tab[3 * B + B * nk * 3 + n_eos:]
    blocks = []
    for b in range(B):
        n, corr = reply[b]
        if n < 1 or n > K or n >= n_limit[b] or corr in eos:
            return None
        key = -1 if (n == K or a0) else corr
        j = -1
        for q in range(nk):
            if keys[(b * nk + q) * 2] == n and keys[(b * nk + q) * 2 + 1] == key:
                j = q
        if j < 0:
            return None
        blk = [corr]
        for i in range(1, K):
            if ctrl:
                blk.append(ctl[b * 2 * K + n + i - 1])
            else:
                blk.append(int(top[key_rows[b * nk + j] + i, 0]))
        blocks.append((sid[b], prefix[b] + n, blk))
    return blocks


def _host(dec, running, preds, block_t, reply):
    """What the host loop of ``SpecDecoder.generate`` does with the same outcome."""
    cfg, k = dec.cfg, dec.cfg.block_size
    out = []
    for i, s in enumerate(running):
        n, corr = reply[i]
        emitted = block_t[i, :n].tolist()[: s.budget - len(s.generated)]
        stop = False
        if not cfg.ignore_eos:
            for j, tok in enumerate(emitted):
                if tok in cfg.eos:
                    emitted = emitted[:j + 1]
                    stop = True
                    break
        if stop or len(s.generated) + len(emitted) >= s.budget:
            return None
        if not cfg.ignore_eos and corr in cfg.eos:
            return None
        key = (n, None if (n == k or cfg.anchor_num == 0) else corr)
        if not preds[s.index].has(key):
            return None
        blk = preds[s.index].get(key)[0].clone()
        blk[0] = corr
        if s.controlled is not None:
            s.controlled.override(blk, None, s.prefix + n)
        out.append((s.index, s.prefix + n, blk.tolist()))
    return out


def _case(rng, B, K, anchor_num, controlled, ignore_eos):
    eos = (7, 11)
    cfg = DecodeConfig(block_size=K, anchor_num=anchor_num, ignore_eos=ignore_eos, eos=eos)
    tgt = _FakeTarget()
    dec = SpecDecoder(tgt, _FakeDraft(), cfg)
    running, layouts = [], []
    for b in range(B):
        cur = torch.tensor([rng.randrange(0, 40) for _ in range(K)])
        # a drafter's top tokens are distinct; the block token may be among them
        top = torch.tensor([rng.sample(range(40), anchor_num + 1) for _ in range(K)])
        prefix = rng.randrange(20, 60)
        s = SeqState(index=100 + b, prompt=[1] * prefix, prefix=prefix, current=cur, top=top,
                     budget=rng.randrange(prefix // 4 + 2, 200))
        s.generated = [3] * rng.randrange(0, s.budget - 1)
        if controlled:
            s.controlled = ControlledAcceptance(oracle=[rng.randrange(0, 40) for _ in range(300)], rate=0.3,
                                                vocab_size=64, seed=5, stream=b)
        running.append(s)
        specs = branch_specs(cur.tolist(), top.tolist() if anchor_num else None, anchor_num)
        layouts.append(packed_layout(cur, specs, prefix, K, MASK, "causal"))
    q = layouts[0].q_len
    dev_top = torch.randint(0, 40, (B * q, anchor_num + 1))
    out = {"dev_top": dev_top, "greedy": dev_top[:, 0].view(B, q)}
    preds = {s.index: _Outcomes(lay, out, i, q) for i, (s, lay) in enumerate(zip(running, layouts))}
    block_t = torch.stack([s.current for s in running])
    assert dec._arm_select(running, preds, block_t)
    return dec, tgt.calls[-1], running, preds, block_t


def test_device_select_matches_host_loop():
    rng = random.Random(0)
    sent = held = 0
    for trial in range(300):
        B = rng.randrange(1, 4)
        K = rng.choice([4, 8, 16])
        anchor_num = rng.choice([0, 1, 2])
        dec, call, running, preds, block_t = _case(rng, B, K, anchor_num, controlled=trial % 3 == 0,
                                                   ignore_eos=trial % 5 == 0)
        for _ in range(6):
            reply = []
            for i, s in enumerate(running):
                n = rng.randrange(1, K + 1)
                keys = [kk for kk in preds[s.index].lay.keys if kk[0] == n and kk[1] is not None]
                if keys and rng.random() < 0.8:
                    corr = rng.choice(keys)[1]       # an outcome some branch drafted
                else:
                    corr = rng.choice([7, 11, rng.randrange(0, 80)])
                reply.append((n, corr))
            dev = _kernel(call, reply)
            host = _host(dec, running, preds, block_t, reply)
            assert dev == host, (trial, reply)
            sent += dev is not None
            held += dev is None
    assert sent > 50 and held > 50
