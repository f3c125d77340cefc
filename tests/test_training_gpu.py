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


def test_fp16_grad_scaler_trainer_matches_torch_loop(tmp_path):
    """fp16 on CUDA: fp32 parameters under autocast with a GradScaler; the fused AdamW's clip
    coefficient sees unscaled gradients, so the Trainer makes the same updates as torch's
    AdamW + GradScaler loop (a clip computed on scaled gradients shrinks them ~1e4x)."""
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.ops.optim import FusedAdamW
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    torch.manual_seed(0)
    spec = _spec()
    ref = TransformerLM(spec).cuda()
    ours = TransformerLM(spec).cuda()
    ours.load_state_dict(ref.state_dict())
    g = torch.Generator().manual_seed(1)
    batches = [torch.randint(0, spec.vocab_size, (4, 257), generator=g).cuda() for _ in range(4)]
    clip, lr = 0.05, 1e-3
    m = ExperimentManifest.from_dict({
        "name": "fp16", "algorithm": "pretrain", "model": spec.to_dict(), "output_dir": str(tmp_path),
        "trainer": {"device": "cuda", "precision": {"dtype": "float16"}, "max_steps": 4, "batch_size": 4,
                    "eval_every": 0, "log_every": 0, "checkpoint": {"save_every": 0},
                    "optimizer": {"learning_rate": lr, "grad_clip": clip, "weight_decay": 0.0},
                    "schedule": {"name": "constant", "warmup_steps": 0}}})
    ctx = RunContext.create(m, metrics_backend="none")
    alg = PretrainAlgorithm(ours, iter([(b[:, :-1], b[:, 1:]) for b in batches]), PretrainConfig(batch_size=4),
                            device=ctx.device)
    trainer = Trainer(ctx, alg)
    assert trainer.precision.scaler.is_enabled() and isinstance(trainer.optimizer, FusedAdamW)
    losses = [trainer.train_step().loss for _ in batches]

    opt = torch.optim.AdamW(ref.parameters(), lr=lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0)
    scaler = torch.amp.GradScaler("cuda")
    ref_losses = []
    for b in batches:
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.float16):
            _, loss = ref(b[:, :-1], b[:, 1:])
        scaler.scale(loss).backward()
        scaler.unscale_(opt)
        torch.nn.utils.clip_grad_norm_(ref.parameters(), clip)
        scaler.step(opt)
        scaler.update()
        ref_losses.append(loss.item())
    assert max(abs(a - b) for a, b in zip(losses, ref_losses)) < 1e-2 * ref_losses[0], (losses, ref_losses)
    for (n, a), b in zip(ref.named_parameters(), ours.parameters()):
        d = (a.detach() - b.detach()).abs().max().item()
        assert d < 3e-4, (n, d)  # 4 steps of lr 1e-3: a shrunken update would differ by ~4e-3
