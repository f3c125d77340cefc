"""The fused-loss reference path equals the composition GRPO / PPO used before the kernel."""
import pytest
import torch

from rl_project_b200.ops.rl_loss import clipped_kl_loss
from rl_project_b200.training.common.logprobs import kl_k3, kl_logprob_diff, masked_mean
from rl_project_b200.training.ppo import ppo_clipped_objective


@pytest.mark.parametrize("ratio_level", ["sequence_mean", "token"])
@pytest.mark.parametrize("kl", ["logprob_diff", "logprob_diff_rows", "k3"])
def test_reference_path_matches_composition(ratio_level, kl):
    torch.manual_seed(0)
    G, R = 6, 11
    mask = (torch.rand(G, R) < 0.7).float()
    old = -torch.rand(G, R) * mask
    ref = old + 0.2 * torch.randn(G, R) * mask
    new = (old + 0.3 * torch.randn(G, R)) * mask
    adv = torch.randn(G)
    loss, pl, klv = clipped_kl_loss(new, old, ref, mask, adv, 0.2, 0.04, ratio_level, kl)
    if ratio_level == "sequence_mean":
        want_pl = ppo_clipped_objective(torch.exp(masked_mean(new - old, mask)), adv, 0.2).mean()
    else:
        want_pl = masked_mean(ppo_clipped_objective(torch.exp(new - old), adv[:, None], 0.2), mask).mean()
    if kl == "k3":
        want_kl = kl_k3(ref, new, mask).mean()
    elif kl == "logprob_diff_rows":
        want_kl = kl_logprob_diff(ref, new, mask).mean()
    else:
        want_kl = kl_logprob_diff(ref, new, mask, clamp_min=None).mean().clamp(min=0)
    torch.testing.assert_close(pl, want_pl)
    torch.testing.assert_close(klv, want_kl)
    torch.testing.assert_close(loss, want_pl + 0.04 * want_kl)
