"""End-to-end gradient correctness of the bf16 sm_100a training path against the fp32 CPU path."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _spec(**kw):
    from rl_project_b200.core.config import model_spec_from_preset

    base = dict(n_layer=2, n_head=4, n_kv_head=2, n_embd=256, block_size=256, vocab_size=1024, d_ff=512,
                rope_theta=500000.0, dropout=0.0)
    base.update(kw)
    return model_spec_from_preset("bl_tiny", **base)


@pytest.mark.parametrize("masked", [False, True])
def test_gradients_match_fp32_cpu(masked):
    from rl_project_b200.models.transformer.model import TransformerLM

    torch.manual_seed(0)
    spec = _spec()
    cpu = TransformerLM(spec)
    gpu = TransformerLM(spec)
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.cuda().to(torch.bfloat16)
    x = torch.randint(0, spec.vocab_size, (4, 256))
    y = torch.roll(x, -1, 1)
    if masked:
        y[:, :64] = -1
    _, lc = cpu(x, y)
    lc.backward()
    _, lg = gpu(x.cuda(), y.cuda())
    lg.backward()
    assert abs(lc.item() - lg.item()) < 0.02 * lc.item()
    gp = dict(gpu.named_parameters())
    for n, p in cpu.named_parameters():
        a, b = p.grad.flatten().float(), gp[n].grad.flatten().float().cpu()
        cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
        rel = (b.norm() / a.norm()).item()
        assert cos > 0.99 and abs(rel - 1) < 0.05, (n, cos, rel)


def test_memorises_a_batch_like_fp32():
    """Same weights, same batch, same AdamW: the bf16 GPU path tracks the fp32 CPU loss curve."""
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.ops.optim import FusedAdamW

    torch.manual_seed(0)
    spec = _spec()
    cpu = TransformerLM(spec)
    gpu = TransformerLM(spec)
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.cuda().to(torch.bfloat16)
    x = torch.randint(0, spec.vocab_size, (4, 256))
    y = torch.roll(x, -1, 1)
    oc = torch.optim.AdamW(cpu.parameters(), lr=1e-3, betas=(0.9, 0.95), weight_decay=0.0)
    og = FusedAdamW(gpu.parameters(), lr=1e-3, betas=(0.9, 0.95), weight_decay=0.0)
    lcs, lgs = [], []
    for _ in range(12):
        oc.zero_grad()
        _, l1 = cpu(x, y)
        l1.backward()
        torch.nn.utils.clip_grad_norm_(cpu.parameters(), 1.0)
        oc.step()
        og.zero_grad()
        _, l2 = gpu(x.cuda(), y.cuda())
        l2.backward()
        og.clip_grad_norm(1.0)
        og.step()
        lcs.append(l1.item())
        lgs.append(l2.item())
    assert lcs[-1] < lcs[0] - 1.0
    assert abs(lgs[-1] - lcs[-1]) < 0.1 * lcs[0], (lcs, lgs)
