"""The decoder-only language model (``src/forgeline/models/transformer/model.py:18-215``).

Module tree and state-dict keys match the reference (``transformer.wte``,
``transformer.h.{i}.*``, ``transformer.ln_f``, ``lm_head``, ``wpe``,
``mtp_modules.{k}.*``), as do initialisation (N(0, 0.02), residual
projections scaled by ``1/sqrt(2L)``), tying and the loss (CE with
ignore index -1 + MoE aux + weighted mean MTP CE).

Differences by design: the loss never materialises fp32 logits (fused
LM-head log-softmax, ops/logprob.py) and ``forward`` returns logits only
when asked (``return_logits=True``) or when no targets are given; residual
adds are fused into the norms (``TransformerBlock.forward_fused``).
"""

from __future__ import annotations

import math
from typing import Any, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.utils.checkpoint

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.models.transformer.block import MTPModule, TransformerBlock
from rl_project_b200.models.transformer.norm import RMSNorm
from rl_project_b200.ops.embedding import embedding
from rl_project_b200.ops.linear import linear
from rl_project_b200.ops.logprob import linear_cross_entropy, linear_logprobs
from rl_project_b200.ops.norm import add_rms_norm, rms_norm


class TransformerLM(nn.Module):
    def __init__(self, spec: ModelSpec):
        super().__init__()
        self.spec = spec
        self.aux_losses: List[torch.Tensor] = []
        self.gradient_checkpointing = False
        self.transformer = nn.ModuleDict(dict(
            wte=nn.Embedding(spec.vocab_size, spec.n_embd),
            drop=nn.Dropout(spec.dropout),
            h=nn.ModuleList([TransformerBlock(i, spec) for i in range(spec.n_layer)]),
            ln_f=RMSNorm(spec.n_embd),
        ))
        self.wpe: Optional[nn.Embedding] = None
        if not spec.use_rope and not spec.use_mla:
            self.wpe = nn.Embedding(spec.block_size, spec.n_embd)
        self.lm_head = nn.Linear(spec.n_embd, spec.vocab_size, bias=False)
        if spec.tie_embeddings:
            self.transformer.wte.weight = self.lm_head.weight
        self.mtp_modules: Optional[nn.ModuleList] = None
        if spec.n_predict_tokens > 1:
            self.mtp_modules = nn.ModuleList([MTPModule(spec) for _ in range(spec.n_predict_tokens - 1)])
        self.apply(self._init_weights)
        resid_std = 0.02 / math.sqrt(2 * spec.n_layer)
        for name, p in self.named_parameters():
            if name.endswith(("c_proj.weight", "w2.weight", "wo.weight")):
                nn.init.normal_(p, 0.0, resid_std)
        self._last_hidden: Optional[torch.Tensor] = None

    # ------------------------------------------------------------ introspection
    @property
    def config(self) -> ModelSpec:
        return self.spec

    def num_parameters(self, non_embedding: bool = True) -> int:
        n = sum(p.numel() for p in self.parameters())
        if non_embedding and self.wpe is not None:
            n -= self.wpe.weight.numel()
        return n

    def num_active_parameters(self, non_embedding: bool = True) -> int:
        n = self.num_parameters(non_embedding)
        if self.spec.use_moe:
            for blk in self.transformer.h:
                if blk.use_moe:
                    per = sum(p.numel() for p in blk.ffn.experts[0].parameters())
                    n -= per * (self.spec.n_experts - self.spec.n_experts_active)
        return n

    def describe(self) -> str:
        s = self.spec
        parts = []
        if s.use_mla:
            parts.append(f"MLA(kv_rank={s.kv_lora_rank})")
        elif s.use_nsa:
            parts.append("NSA")
        elif s.n_kv_head < s.n_head:
            parts.append(f"GQA({s.n_head}Q/{s.n_kv_head}KV)")
        else:
            parts.append("MHA")
        if s.sliding_window > 0:
            parts.append(f"SlidingWindow({s.sliding_window},{'alternating' if s.alternating_layers else 'all'})")
        if s.attn_logit_cap > 0:
            parts.append(f"LogitCap({s.attn_logit_cap})")
        if s.rope_scaling_type != "none":
            parts.append(f"RoPE-{s.rope_scaling_type}({s.rope_scaling_factor}x)")
        if s.use_moe:
            parts.append(f"MoE({s.n_experts_active}/{s.n_experts}+{s.n_shared_experts}shared"
                         f"{',aux-free' if s.aux_loss_free else ''})")
        if s.n_predict_tokens > 1:
            parts.append(f"MTP({s.n_predict_tokens})")
        total = self.num_parameters() / 1e6
        head = (f"{total:.1f}M total / {self.num_active_parameters() / 1e6:.1f}M active" if s.use_moe
                else f"{total:.1f}M params")
        return head + " | " + " | ".join(parts)

    @staticmethod
    def _init_weights(m: nn.Module) -> None:
        if isinstance(m, nn.Linear):
            nn.init.normal_(m.weight, 0.0, 0.02)
            if m.bias is not None:
                nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, 0.0, 0.02)

    def enable_gradient_checkpointing(self) -> None:
        self.gradient_checkpointing = True

    def disable_gradient_checkpointing(self) -> None:
        self.gradient_checkpointing = False

    # ------------------------------------------------------------ forward
    def _embed(self, idx: torch.Tensor, offset: int = 0) -> torch.Tensor:
        x = embedding(idx, self.transformer.wte.weight)
        if self.wpe is not None:
            pos = torch.arange(offset, offset + idx.shape[1], device=idx.device)
            x = x + self.wpe(pos)
        return self.transformer.drop(x)

    def forward_hidden(self, idx: torch.Tensor) -> torch.Tensor:
        """Final normalised hidden states ``[B, T, n_embd]`` (collects MoE aux losses)."""
        T = idx.shape[1]
        if T > self.spec.block_size:
            raise ValueError(f"sequence length {T} exceeds block_size {self.spec.block_size}")
        x = self._embed(idx)
        self.aux_losses = []
        pending: Optional[torch.Tensor] = None
        ckpt = self.gradient_checkpointing and self.training
        for blk in self.transformer.h:
            if ckpt:
                x, pending = torch.utils.checkpoint.checkpoint(blk, x, pending=pending, fused=True,
                                                               use_reentrant=False)
            else:
                x, pending = blk(x, pending=pending, fused=True)
            if blk.use_moe and blk.ffn.aux_loss is not None:
                self.aux_losses.append(blk.ffn.aux_loss)
        ln_f = self.transformer.ln_f
        if pending is None:
            h = rms_norm(x, ln_f.weight, ln_f.eps)
        else:
            _, h = add_rms_norm(x, pending, ln_f.weight, ln_f.eps)
        self._last_hidden = h.detach()
        return h

    def head_weight(self) -> torch.Tensor:
        return self.lm_head.weight

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return linear(h, self.lm_head.weight)

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None, return_logits: bool = False):
        h = self.forward_hidden(idx)
        B, T = idx.shape
        if targets is None:
            return self.logits(h[:, -1:, :]), None
        loss = linear_cross_entropy(h.reshape(B * T, -1), self.lm_head.weight, targets.reshape(-1))
        if self.aux_losses:
            loss = loss + sum(self.aux_losses)
        if self.mtp_modules is not None and T > 1:
            total, n = 0.0, 0
            for d, mod in enumerate(self.mtp_modules):
                depth = d + 1
                if T - depth < 1:
                    break
                temb = embedding(idx[:, depth:], self.transformer.wte.weight)
                hm = mod(h[:, : T - depth], temb)
                tgt = targets[:, depth:][:, : T - depth].reshape(-1)
                total = total + linear_cross_entropy(hm.reshape(-1, hm.shape[-1]), self.lm_head.weight, tgt)
                n += 1
            if n:
                loss = loss + self.spec.mtp_loss_weight * (total / n)
        logits = self.logits(h) if return_logits else None
        return logits, loss

    def full_logits(self, idx: torch.Tensor) -> torch.Tensor:
        return self.logits(self.forward_hidden(idx))

    def token_logprobs(self, idx: torch.Tensor, targets: torch.Tensor, with_entropy: bool = False):
        """Per-position ``log p(targets | idx)`` ``[B, T]`` via the fused LM-head kernel."""
        h = self.forward_hidden(idx)
        B, T = idx.shape
        lp, extra = linear_logprobs(h.reshape(B * T, -1), self.lm_head.weight, targets.reshape(-1), with_entropy)
        lp = lp.view(B, T)
        if with_entropy:
            return lp, extra.view(B, T)
        return lp

    # ------------------------------------------------------------ incremental decoding
    @torch.no_grad()
    def prefill(self, idx: torch.Tensor, last_positions: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, List[Any]]:
        """Logits at the last position (or at ``last_positions[b]`` for right-padded rows) and the per-layer cache."""
        x = self._embed(idx)
        cache: List[Any] = []
        for blk in self.transformer.h:
            x, present = blk(x)
            cache.append(present)
        if last_positions is None:
            last = x[:, -1, :]
        else:
            last = x[torch.arange(x.shape[0], device=x.device), last_positions.to(x.device)]
        return self.logits(self.transformer.ln_f(last)), cache

    @torch.no_grad()
    def step(self, next_ids: torch.Tensor, cache: List[Any], position: int) -> Tuple[torch.Tensor, List[Any]]:
        x = self._embed(next_ids, offset=position)
        new_cache: List[Any] = []
        for i, blk in enumerate(self.transformer.h):
            x, present = blk(x, past_kv=cache[i])
            new_cache.append(present)
        h = self.transformer.ln_f(x)
        return self.logits(h[:, -1, :]), new_cache

    def supports_paged_decode(self) -> bool:
        """True when every layer is grouped-query attention (the paged KV kernels' layout)."""
        from rl_project_b200.models.attention.causal import CausalSelfAttention

        return all(type(b.attn) is CausalSelfAttention for b in self.transformer.h)

    def kv_layout(self) -> Tuple[int, int, int]:
        """``(n_layer, n_kv_head, head_dim)`` of this process's KV cache: the attention modules' own head
        counts, which tensor parallelism divides by the group size."""
        attn = self.transformer.h[0].attn
        return self.spec.n_layer, attn.n_kv_head, attn.head_dim

    @torch.no_grad()
    def decode_paged(self, tokens: torch.Tensor, cache: Any, meta: Any) -> torch.Tensor:
        """Logits ``[B, V]`` for one new token per sequence; K/V go into ``cache`` (a ``PagedKVCache``)."""
        x = embedding(tokens.view(-1, 1), self.transformer.wte.weight)
        if self.wpe is not None:
            x = x + self.wpe(meta.positions.long())
        for i, blk in enumerate(self.transformer.h):
            x = blk.forward_paged(x, cache.layer(i), meta)
        h = self.transformer.ln_f(x)
        return self.logits(h[:, 0])

    @torch.no_grad()
    def generate(self, idx: torch.Tensor, max_new_tokens: int, temperature: float = 1.0, top_k: Optional[int] = None,
                 top_p: Optional[float] = None, min_p: Optional[float] = None, repetition_penalty: float = 1.0,
                 use_cache: bool = True, stop_token_ids: Tuple[int, ...] = ()) -> torch.Tensor:
        from rl_project_b200.models.generation.sampling import generate_tokens

        return generate_tokens(self, idx, max_new_tokens, temperature=temperature, top_k=top_k, top_p=top_p,
                               min_p=min_p, repetition_penalty=repetition_penalty, use_cache=use_cache,
                               stop_token_ids=stop_token_ids)
