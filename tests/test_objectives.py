"""Self-distillation objectives and the micro-transformer block (CPU)."""

import math

import pytest
import torch
import torch.nn.functional as F

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.models.micro_transformer import MicroTransformerBlock
from burn_dragon_b200.train import objectives as O


def test_kl_kinds_and_js_bounds():
    g = torch.Generator().manual_seed(0)
    s, t = torch.randn(2, 3, 7, generator=g), torch.randn(2, 3, 7, generator=g)
    ls, lt = F.log_softmax(s, -1), F.log_softmax(t, -1)
    fwd = O.self_distillation_per_token(ls, lt, "forward")
    torch.testing.assert_close(fwd, F.kl_div(ls, lt, log_target=True, reduction="none").sum(-1))
    rev = O.self_distillation_per_token(ls, lt, "reverse")
    torch.testing.assert_close(rev, F.kl_div(lt, ls, log_target=True, reduction="none").sum(-1))
    js = O.self_distillation_per_token(ls, lt, "jensen_shannon")
    assert float(js.min()) >= 0 and float(js.max()) <= math.log(2) + 1e-6
    assert float(O.self_distillation_per_token(ls, ls, "jensen_shannon").abs().max()) < 1e-6
    mask = torch.tensor([[1, 0, 1], [0, 0, 0]])
    torch.testing.assert_close(O.masked_token_mean(fwd, mask), (fwd[0, 0] + fwd[0, 2]) / 2)


def test_clipped_policy_loss_and_advantage():
    new = torch.tensor([[0.0, -1.0]])
    old = torch.tensor([[-1.0, -1.0]])
    adv = torch.tensor([[1.0, -1.0]])
    # ratio e on the first token is clipped to 1.2 for a positive advantage
    loss = O.clipped_policy_loss(new, old, adv, clip=0.2)
    torch.testing.assert_close(loss, torch.tensor(-(1.2 * 1.0 + 1.0 * -1.0) / 2))
    a = O.sdpo_token_advantage(torch.tensor([[1.0, 3.0]]), torch.tensor([[0.0, 0.0]]), normalize=True)
    torch.testing.assert_close(a, torch.tensor([[-1.0, 1.0]]), atol=1e-5, rtol=0)
    assert float(O.clipped_policy_loss(new, old, adv, weight=0.0)) == 0.0


def test_window_objectives_and_ema_teacher():
    cfg = DragonConfig(n_layer=1, n_embd=16, n_head=2, mlp_internal_dim_multiplier=2, dropout=0.0,
                       rotary_embedding="rope", initialization="simple_normal", vocab_size=32)
    student = BDH(cfg, seed=0)
    teacher = O.EMATeacher(student, rate=0.5)
    x = torch.randint(0, 32, (2, 5))
    y = torch.randint(0, 32, (2, 5))
    for kind in ("sdft", "sdpo", "sdft_sdpo"):
        oc = O.ObjectiveConfig(type=kind)
        oc.validate()
        loss = O.window_objective_loss(student, teacher.model, x, y, oc)
        assert float(loss) < 1e-10  # teacher == student at start
    nt = O.window_objective_loss(student, teacher.model, x, y, O.ObjectiveConfig())
    torch.testing.assert_close(nt, student.loss(x, y))
    with torch.no_grad():
        student.encoder.add_(1.0)
    teacher.update(student)
    torch.testing.assert_close(teacher.model.encoder, student.encoder - 0.5)
    assert float(O.window_objective_loss(student, teacher.model, x, y, O.ObjectiveConfig(type="sdft"))) > 0
    with pytest.raises(ValueError):
        O.ObjectiveConfig(type="sdpo", sdpo=O.SdpoObjectiveConfig(alpha=2.0)).validate()


def test_micro_transformer_group_causal_mask():
    torch.manual_seed(0)
    blk = MicroTransformerBlock(16, 4, 2)
    x = torch.randn(1, 6, 16)
    full = blk(x)
    grp = blk(x, group_size=2)
    assert full.shape == grp.shape == (1, 6, 16)
    # with group size 2 the first group's outputs do not depend on later tokens
    x2 = x.clone()
    x2[:, 4:] += torch.randn(1, 2, 16)
    torch.testing.assert_close(blk(x2, group_size=2)[:, :4], grp[:, :4])
    assert not torch.allclose(blk(x2)[:, :4], full[:, :4])
