"""Model inspection: weight statistics, layer summary, residual-stream flow and
attention patterns (the views of ``src/forgeline/evaluation/inspection.py:12-112``,
computed for this framework's modules)."""

from __future__ import annotations

import math
from typing import Any, Dict, List

import torch


def weight_statistics(model: torch.nn.Module, bins: int = 20) -> List[Dict[str, Any]]:
    """Per parameter: shape, size, mean, std, min, max, mean |w|, L2 norm and a ``bins``-bucket histogram.
    The scalar statistics of every parameter are computed on its device and fetched in one transfer; the
    histograms are built on the host."""
    named = list(model.named_parameters())
    if not named:
        return []
    rows = []
    for _, p in named:
        d = p.detach().float()
        std = d.std() if d.numel() > 1 else torch.zeros((), device=d.device)
        rows.append(torch.stack([d.mean(), std, d.min(), d.max(), d.abs().mean(), d.norm()]))
    same_device = len({r.device for r in rows}) == 1
    table = (torch.stack(rows).cpu() if same_device else torch.stack([r.cpu() for r in rows])).tolist()
    stats = []
    for (name, p), (mean, std, lo, hi, abs_mean, norm) in zip(named, table):
        counts = torch.histc(p.detach().float().flatten().cpu(), bins=bins, min=lo, max=hi if hi > lo else lo + 1e-12)
        stats.append({"name": name, "shape": list(p.shape), "numel": p.numel(), "mean": mean, "std": std, "min": lo,
                      "max": hi, "abs_mean": abs_mean, "norm": norm,
                      "histogram": {"counts": counts.tolist(), "edges": [lo + i * (hi - lo) / bins for i in range(bins + 1)]}})
    return stats


def layer_summary(spec) -> List[Dict[str, Any]]:
    layers: List[Dict[str, Any]] = [{"type": "embedding", "name": "token_embedding",
                                     "params": spec.vocab_size * spec.n_embd}]
    for i in range(spec.n_layer):
        if spec.use_mla:
            attn = "MLA"
        elif spec.use_nsa:
            attn = "NSA"
        else:
            attn = "GQA" if spec.n_kv_head < spec.n_head else "MHA"
        comps: List[Dict[str, Any]] = [{"type": "attention", "name": attn, "n_heads": spec.n_head,
                                        "n_kv_heads": spec.n_kv_head}]
        if spec.use_moe and i >= spec.n_dense_layers:
            comps.append({"type": "moe", "n_experts": spec.n_experts, "n_active": spec.n_experts_active,
                          "n_shared": spec.n_shared_experts})
        else:
            comps.append({"type": "ffn", "name": "SwiGLU" if spec.use_swiglu else "GELU"})
        layers.append({"type": "block", "layer_id": i, "components": comps})
    tied = getattr(spec, "tie_embeddings", True)
    layers.append({"type": "output", "name": "lm_head", "params": 0 if tied else spec.vocab_size * spec.n_embd,
                   "tied": tied})
    return layers


def _stats(name: str, t: torch.Tensor) -> Dict[str, float]:
    f = t.float()
    return {"name": name, "mean": float(f.mean()), "std": float(f.std()), "max_abs": float(f.abs().max()),
            "norm": float(f.norm())}


@torch.no_grad()
def activation_flow(model, ids: torch.Tensor) -> List[Dict[str, float]]:
    """Statistics of the residual stream after the embedding, each block and the final norm.

    The stream is walked block by block (the fused training forward keeps the
    last residual add pending inside the next block, so block outputs are not
    module outputs there)."""
    x = model._embed(ids)
    records = [_stats("embedding", x)]
    for i, blk in enumerate(model.transformer.h):
        x, _ = blk(x)
        records.append(_stats(f"block_{i}", x))
    records.append(_stats("final_norm", model.transformer.ln_f(x)))
    return records


@torch.no_grad()
def attention_patterns(model, ids: torch.Tensor, max_tokens: int = 48, per_head: bool = False) -> List[Dict[str, Any]]:
    """Head-averaged attention weights ``[T, T]`` and per-head entropy per layer for a ``[1, T]`` prompt.

    The weights are recomputed in fp32 from each grouped-query layer's own
    projections, rotary table, soft-cap and causal / sliding-window mask (the
    forward pass itself runs fused attention that never forms them).  MLA and
    NSA layers are reported as unsupported.
    """
    from rl_project_b200.models.attention.causal import CausalSelfAttention
    from rl_project_b200.ops.rope import apply_rope_reference

    ids = ids[:, -max_tokens:]
    blocks = list(model.transformer.h)
    captured: Dict[int, torch.Tensor] = {}
    handles = []
    for i, blk in enumerate(blocks):
        if isinstance(blk.attn, CausalSelfAttention):
            handles.append(blk.attn.register_forward_pre_hook(
                lambda m, args, i=i: captured.__setitem__(i, args[0].detach())))
    try:
        model(ids)
    finally:
        for h in handles:
            h.remove()
    out: List[Dict[str, Any]] = []
    for i, blk in enumerate(blocks):
        attn = blk.attn
        if i not in captured:
            out.append({"layer": i, "type": type(attn).__name__, "supported": False})
            continue
        x = captured[i].float()
        B, T, _ = x.shape
        H, Hkv, D = attn.n_head, attn.n_kv_head, attn.head_dim
        q = (x @ attn.q_proj.weight.float().t()).view(B, T, H, D).transpose(1, 2)
        k = (x @ attn.k_proj.weight.float().t()).view(B, T, Hkv, D).transpose(1, 2)
        if attn.use_rope:
            cos, sin = attn.rope.tables(T, x.device)
            q, k = apply_rope_reference(q, cos[:T], sin[:T]), apply_rope_reference(k, cos[:T], sin[:T])
        k = k.repeat_interleave(H // Hkv, dim=1)
        s = (q @ k.transpose(-2, -1)) / math.sqrt(D)
        if attn.attn_logit_cap > 0:
            s = torch.tanh(s / attn.attn_logit_cap) * attn.attn_logit_cap
        qi = torch.arange(T, device=x.device)[:, None]
        kj = torch.arange(T, device=x.device)[None, :]
        allowed = kj <= qi
        if attn.window_size > 0:
            allowed &= (qi - kj) < attn.window_size
        w = torch.softmax(s.masked_fill(~allowed, float("-inf")), dim=-1)[0]  # [H, T, T]
        entropy = -(w.clamp_min(1e-12).log() * w).sum(-1).mean(-1)
        rec = {"layer": i, "type": "GQA" if Hkv < H else "MHA", "supported": True, "window": attn.window_size,
               "weights": w.mean(0).tolist(), "head_entropy": entropy.tolist()}
        if per_head:
            rec["head_weights"] = w.tolist()
        out.append(rec)
    return out
