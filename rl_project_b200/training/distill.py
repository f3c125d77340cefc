"""Knowledge distillation (the objective of ``src/forgeline/training/distill.py``):

    loss = alpha * T^2 * KL(softmax(t / T) || softmax(s / T))  (mean over rows)
         + (1 - alpha) * CE(s, labels)                          (mean over labelled rows, label -1 ignored)
         + feature_weight * mean over layers of MSE(P_l h_student_l, h_teacher_l)   (optional)

The logit terms are evaluated by ``distillation_loss`` as one custom autograd op that walks the rows in
chunks: per chunk it forms the fp32 log-softmaxes, the KL and CE row terms and, in the same pass, the
analytic gradient with respect to the student logits,

    d loss / d s = alpha * (T / N) * (softmax(s / T) - softmax(t / T)) + (1 - alpha) / N_lab * (softmax(s) - onehot),

which is stored in the student logits' own dtype.  No fp32 ``[N, V]`` tensor is ever alive beyond one
chunk (at vocab 128k an fp32 copy of the logits of a 4k-token batch is 2 GB), and backward is one
scale of the stored gradient.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, List, Mapping

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.training.common.trainer import PostTrainingAlgorithm

_CHUNK_ELEMS = 1 << 26  # fp32 elements per chunk of rows (256 MB)


class _DistillLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, s: torch.Tensor, t: torch.Tensor, labels: torch.Tensor, temperature: float, alpha: float):
        N, V = s.shape
        labelled = labels != -1
        n_lab = int(labelled.sum())
        grad = torch.empty_like(s) if s.requires_grad else None
        kl_sum = torch.zeros((), device=s.device, dtype=torch.float32)
        ce_sum = torch.zeros((), device=s.device, dtype=torch.float32)
        rows = max(1, _CHUNK_ELEMS // max(V, 1))
        for a in range(0, N, rows):
            b = min(N, a + rows)
            s32, t32 = s[a:b].float(), t[a:b].float()
            ls_T = torch.log_softmax(s32 / temperature, -1)
            lt_T = torch.log_softmax(t32 / temperature, -1)
            pt_T = lt_T.exp()
            kl_sum += (pt_T * (lt_T - ls_T)).sum()
            ls = torch.log_softmax(s32, -1)
            lab, ok = labels[a:b], labelled[a:b]
            picked = ls.gather(1, lab.clamp_min(0)[:, None])[:, 0]
            ce_sum += -(picked * ok).sum()
            if grad is not None:
                g = (ls_T.exp() - pt_T) * (alpha * temperature / N)
                if n_lab:
                    soft = ls.exp_()
                    soft.scatter_add_(1, lab.clamp_min(0)[:, None], -ok.float()[:, None])
                    g += soft * ok.float()[:, None] * ((1.0 - alpha) / n_lab)
                grad[a:b] = g.to(grad.dtype)
        ctx.save_for_backward(grad if grad is not None else torch.empty(0))
        kl = kl_sum / N * temperature ** 2
        ce = ce_sum / n_lab if n_lab else torch.full((), float("nan"), device=s.device)
        return alpha * kl + (1.0 - alpha) * ce

    @staticmethod
    def backward(ctx, g_out):
        (grad,) = ctx.saved_tensors
        return grad * g_out.to(grad.dtype), None, None, None, None


def distillation_loss(student_logits: torch.Tensor, teacher_logits: torch.Tensor, labels: torch.Tensor,
                      temperature: float = 4.0, alpha: float = 0.7) -> torch.Tensor:
    V = student_logits.shape[-1]
    return _DistillLoss.apply(student_logits.reshape(-1, V), teacher_logits.detach().reshape(-1, V),
                              labels.reshape(-1), float(temperature), float(alpha))


class FeatureDistiller(nn.Module):
    """Linear projections of the first ``n_layers`` student block outputs onto the teacher's width, scored by the
    mean over layers of their MSE against the teacher's block outputs."""

    def __init__(self, student_dim: int, teacher_dim: int, n_layers: int = 4):
        super().__init__()
        self.projectors = nn.ModuleList(nn.Linear(student_dim, teacher_dim, bias=False) for _ in range(n_layers))

    def forward(self, student_hiddens: List[torch.Tensor], teacher_hiddens: List[torch.Tensor]) -> torch.Tensor:
        pairs = list(zip(self.projectors, student_hiddens, teacher_hiddens))
        if not pairs:
            return torch.zeros(())
        terms = [F.mse_loss(proj(hs.to(proj.weight.dtype)).float(), ht.detach().float()) for proj, hs, ht in pairs]
        return torch.stack(terms).mean()


@dataclass
class DistillConfig:
    temperature: float = 4.0
    alpha: float = 0.7
    batch_size: int = 16
    feature_weight: float = 0.0
    eval_batches: int = 10
    seed: int = 0


def _block_outputs(model, x: torch.Tensor) -> List[torch.Tensor]:
    """Each transformer block's output hidden state for ``x`` (one forward)."""
    captured: List[torch.Tensor] = []
    handles = [blk.register_forward_hook(lambda _m, _i, out: captured.append(out[0] if isinstance(out, tuple) else out))
               for blk in model.transformer.h]
    try:
        model.full_logits(x)
    finally:
        for h in handles:
            h.remove()
    return captured


class DistillationAlgorithm(PostTrainingAlgorithm):
    name = "distill"

    def __init__(self, student, teacher, corpus, config: DistillConfig, val_corpus=None,
                 device: torch.device | str = "cpu"):
        if student.spec.vocab_size != teacher.spec.vocab_size:
            raise ValueError("student and teacher must share a vocabulary")
        teacher.eval().requires_grad_(False)
        self.student, self.teacher, self.cfg = student, teacher, config
        self.corpus, self.val_corpus = corpus, val_corpus
        self.device = torch.device(device)
        self.gen = torch.Generator().manual_seed(config.seed)
        self.feature = None
        if config.feature_weight > 0:
            self.feature = FeatureDistiller(student.spec.n_embd, teacher.spec.n_embd,
                                            min(student.spec.n_layer, teacher.spec.n_layer))

    def parameters(self) -> List[nn.Parameter]:
        extra = list(self.feature.parameters()) if self.feature is not None else []
        return list(self.student.parameters()) + extra

    def modules(self):
        return tuple(m for m in (self.student, self.feature) if m is not None)

    def frozen_modules(self):
        return (self.teacher,)

    def _draw(self, corpus):
        if hasattr(corpus, "sample_batch"):
            return corpus.sample_batch(self.cfg.batch_size, self.device, self.gen)
        x, y = next(corpus)
        return x.to(self.device), y.to(self.device)

    def collect(self, step: int):
        return self._draw(self.corpus)

    def _logit_loss(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            target = self.teacher.full_logits(x)
        return distillation_loss(self.student.full_logits(x), target, y, self.cfg.temperature, self.cfg.alpha)

    def loss(self, batch, micro_step: int, n_micro: int):
        x, y = batch
        loss = self._logit_loss(x, y)
        if self.feature is None:
            return loss, {}
        with torch.no_grad():
            teacher_h = _block_outputs(self.teacher, x)
        feat = self.feature(_block_outputs(self.student, x), teacher_h)
        return loss + self.cfg.feature_weight * feat, {"feature_loss": feat.detach()}

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        corpus = self.val_corpus or self.corpus
        if not hasattr(corpus, "sample_batch"):
            return {}
        vals = [float(self._logit_loss(*self._draw(corpus))) for _ in range(self.cfg.eval_batches)]
        return {"loss": sum(vals) / len(vals)}

    def state(self) -> Dict[str, Any]:
        return {"model": self.student.state_dict(), "teacher_spec": self.teacher.spec.to_dict()}

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.student.load_state_dict(state["model"])

    def model_spec(self) -> Dict[str, Any]:
        return self.student.spec.to_dict()
