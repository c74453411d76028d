import pytest
import torch

from burn_dragon_b200.train.gdpo import gdpo_advantages, percentile_thresholds, percentile_thresholds_ref


def test_reference_rule():
    v = torch.tensor([[3.0, 1.0, 2.0, 4.0], [float("nan"), 1.0, float("inf"), -1.0]])
    out = percentile_thresholds_ref(v, 0.5)
    assert torch.allclose(out[0], torch.tensor(2.5))
    assert torch.allclose(out[1], torch.tensor(0.5))
    adv = gdpo_advantages(torch.tensor([[1.0, 2.0, 3.0, 4.0]]), 0.5)
    assert (adv[0, :2] == 0).all() and (adv[0, 2:] > 0).all()


@pytest.mark.gpu
@pytest.mark.parametrize("group", [1, 2, 3, 17, 256, 1000])
def test_percentile_kernel_matches_reference(group):
    torch.manual_seed(group)
    v = torch.randn(33, group, device="cuda")
    v[0, 0] = float("nan")
    for q in (0.0, 0.25, 0.9, 1.0):
        assert torch.allclose(percentile_thresholds(v, q).cpu(), percentile_thresholds_ref(v.cpu(), q), atol=1e-6)
