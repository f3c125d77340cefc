"""Fused GRPO / PPO loss kernel against the PyTorch composition of the same formulas (fp32)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ratio_level", ["sequence_mean", "token"])
@pytest.mark.parametrize("kl", ["logprob_diff", "logprob_diff_rows", "k3"])
def test_fused_loss_matches_reference(ratio_level, kl):
    from rl_project_b200.ops.rl_loss import clipped_kl_loss, clipped_kl_loss_reference

    torch.manual_seed(0)
    G, R = 16, 300
    mask = (torch.rand(G, R, device="cuda") < 0.8).float()
    mask[3] = 0  # an empty sequence
    old = -torch.rand(G, R, device="cuda") * 3 * mask
    ref = old + 0.3 * torch.randn(G, R, device="cuda") * mask
    new0 = old + 0.4 * torch.randn(G, R, device="cuda") * mask
    adv = torch.randn(G, device="cuda")
    outs = []
    for fn in (clipped_kl_loss, clipped_kl_loss_reference):
        new = new0.clone().requires_grad_(True)
        loss, pl, klv = fn(new * mask, old, ref, mask, adv, 0.2, 0.04, ratio_level, kl)
        (loss * 1.7).backward()
        outs.append((loss.detach(), pl.detach(), klv.detach(), new.grad))
    (l1, p1, k1, g1), (l2, p2, k2, g2) = outs
    torch.testing.assert_close(l1, l2, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(p1, p2, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(k1, k2, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(g1, g2, atol=1e-6, rtol=1e-4)
