"""Auxiliary training objectives and hidden-trajectory distillation (CPU):
closed forms of the hard-negative CE and margin losses, the trajectory
selection and relation loss, and a trainer run with every option on."""
import math

import torch


def test_hard_negative_ce_and_margin_closed_forms():
    from d3d_b200.train.losses import ce_aux_per_token, hard_negative_ce_per_token, target_margin_per_token
    z = torch.tensor([[2.0, 1.0, 0.5, -1.0], [0.0, 3.0, 2.5, 1.0]])
    y = torch.tensor([0, 2])
    hn = hard_negative_ce_per_token(z, y, top_k=2, margin=0.0)
    want0 = math.log(1 + math.exp(1.0 - 2.0) + math.exp(0.5 - 2.0))
    want1 = math.log(1 + math.exp(3.0 - 2.5) + math.exp(1.0 - 2.5))
    assert torch.allclose(hn, torch.tensor([want0, want1]), atol=1e-6)
    # with every competitor included it equals plain CE
    full = hard_negative_ce_per_token(z, y, top_k=3)
    assert torch.allclose(full, torch.nn.functional.cross_entropy(z, y, reduction="none"), atol=1e-6)
    mg = target_margin_per_token(z, y, top_k=1, margin=1.0, smooth=False)
    assert torch.allclose(mg, torch.tensor([max(0.0, 1.0 - 2.0 + 1.0), max(0.0, 3.0 - 2.5 + 1.0)]))
    tot, ce, h2, m2 = ce_aux_per_token(z, y, ce_weight=1.0, hnce_weight=0.5, hnce_top_k=2, margin_weight=2.0,
                                       margin_top_k=1, margin_smooth=False)
    assert torch.allclose(tot, ce + 0.5 * h2 + 2.0 * m2)


def test_trajectory_selection_and_relation_loss():
    from d3d_b200.train import trajectory as T
    pred = torch.tensor([[[1, 2, 3], [1, 9, 3]]])
    tgt = torch.tensor([[[1, 2, 3], [1, 2, 3]]])
    valid = torch.ones_like(pred, dtype=torch.bool)
    acc = T.block_accept_lengths(pred, tgt, valid)
    assert acc.tolist() == [[3, 1]]
    sel = T.selection_mask(torch.tensor([[3, 3]]), acc, torch.tensor([[3, 3]]), torch.tensor([[True, True]]))
    assert sel.tolist() == [[True, True]]          # both full; teacher better
    h = torch.randn(1, 2, 4, 8)
    valid4 = torch.ones(1, 2, 4, dtype=torch.bool)
    loss, cnt = T.relational_loss(h, h * 3.0, valid4, sel)   # same directions -> same relations
    assert cnt == 2 and float(loss) < 1e-6
    loss2, _ = T.relational_loss(h, torch.randn(1, 2, 4, 16), valid4, sel)
    assert float(loss2) > 0
    assert float(T.distributed_block_mean(loss2, 4.0, 2)) == float(loss2) * 0.5


def test_trainer_with_aux_and_trajectory(tmp_path):
    from d3d_b200.train.args import parser as build_parser
    from d3d_b200.train.trainer import train
    args = build_parser().parse_args([
        "--draft-model", "tiny-drafter", "--target-model", "tiny-target", "--output-dir", str(tmp_path),
        "--max-steps", "2", "--batch-size", "2", "--seq-len", "64", "--device", "cpu", "--dtype", "fp32",
        "--hnce-weight", "0.5", "--margin-weight", "0.5", "--trajectory-weight", "1.0", "--ar-weight", "0.5",
        "--parallel-anchors-per-example", "4", "--vocab-chunk", "256"])
    out = train(args)
    assert len(out["log"]) == 2 and all(math.isfinite(r["loss"]) for r in out["log"])
