"""Fused multi-tensor AdamW with fp32 master weights (kernel: csrc/adamw.cu).

``FusedAdamW`` keeps bf16 parameters for compute and an fp32 master copy,
``exp_avg`` and ``exp_avg_sq`` in three flat fp32 buffers (one allocation
each).  One ``step`` is three launches regardless of the parameter count:
squared-norm partials, the norm/clip finish, and the update itself; the clip
coefficient never leaves the device.  Semantics match torch.optim.AdamW /
Adam as configured by ``src/forgeline/training/common/optim.py:11-30``.
"""

from __future__ import annotations

from typing import Dict, Iterable, List, Optional

import numpy as np
import torch

from rl_project_b200.ops._ext import native

# one AdamTensor of csrc/adamw.cu (packed, 56 bytes)
_DESC = np.dtype([("master", "<u8"), ("p16", "<u8"), ("grad", "<u8"), ("m", "<u8"), ("v", "<u8"), ("n", "<i8"),
                  ("wd", "<f4"), ("gb", "<i4")])


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params: Iterable, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, decoupled: bool = True, param16: Optional[dict] = None,
                 segments: Optional[dict] = None, process_group=None, post_step=None):
        """``param16``: fp32 parameter -> bf16 tensor rewritten by the update (sharded training).
        ``segments``: parameter -> [(start, end, weight_decay)] element ranges, each updated with its
        own decay (flat shards that mix matrices and vectors).  ``process_group``: the gradient norm
        is summed over it (sharded gradients).  ``post_step``: called after every update."""
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self.decoupled = decoupled
        self._param16 = dict(param16 or {})
        self._segments = dict(segments or {})
        self._group = process_group
        self._post_step = post_step
        self._flat: Dict[str, torch.Tensor] = {}
        self._desc_key = None
        self._desc = None
        self._host_desc = None
        self._entry_param = self._entry_goff = self._entry_grads = None
        self._grad_mask = None
        self._chunks = None
        self._nchunks = 0
        self._partial = None
        self.norm_coef: Optional[torch.Tensor] = None
        self._step = 0
        self._init_state()

    # ------------------------------------------------------------------ state
    def _params(self) -> List[torch.nn.Parameter]:
        return [p for g in self.param_groups for p in g["params"]]

    def _init_state(self) -> None:
        ps = self._params()
        if not ps:
            raise ValueError("no parameters")
        dev = ps[0].device
        if dev.type != "cuda":
            raise ValueError("FusedAdamW runs on CUDA parameters; use torch.optim.AdamW on CPU")
        total = sum(p.numel() for p in ps)
        for name in ("master", "exp_avg", "exp_avg_sq"):
            self._flat[name] = torch.zeros(total, dtype=torch.float32, device=dev)
        off = 0
        for p in ps:
            n = p.numel()
            st = self.state[p]
            st["master"] = self._flat["master"][off:off + n].view_as(p)
            st["master"].copy_(p.detach().float())
            st["exp_avg"] = self._flat["exp_avg"][off:off + n].view_as(p)
            st["exp_avg_sq"] = self._flat["exp_avg_sq"][off:off + n].view_as(p)
            off += n
        # per-parameter step counts (a parameter without a gradient in a step is not stepped), kept as one
        # array and written into the state only when it is serialised
        self._param_index = {id(p): i for i, p in enumerate(ps)}
        self._param_steps = np.zeros(len(ps), dtype=np.int64)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self._partial = torch.empty(sms * 8, dtype=torch.float32, device=dev)
        self.norm_coef = torch.zeros(2, dtype=torch.float32, device=dev)

    def _build_desc(self) -> None:
        """Device descriptors of every gradient-carrying tensor segment and the chunk list of the kernels.

        The layout (which segments, their master / moment / bf16 pointers, sizes, decays, the chunk list)
        only changes when the parameter set, a parameter's storage or a gradient dtype changes; it is then
        rebuilt, the chunk list generated with numpy.  Gradient tensors are usually new every step
        (``zero_grad(set_to_none=True)``): their pointers are patched into the host copy of the descriptors
        and the ~50 bytes per segment re-uploaded, nothing else."""
        ps = [p for g in self.param_groups for p in g["params"] if p.grad is not None]
        layout = tuple((id(p), p.data_ptr(), p.grad.dtype, p.grad.is_contiguous()) for p in ps) + tuple(
            a.data_ptr() for a in self._param16.values())
        if layout != self._desc_key:
            self._layout(ps)
            self._desc_key = layout
        gptr = np.fromiter((p.grad.data_ptr() for p in ps), dtype=np.uint64, count=len(ps))
        grads = gptr[self._entry_param] + self._entry_goff
        if self._entry_grads is None or not np.array_equal(grads, self._entry_grads):
            self._host_desc["grad"] = grads
            self._entry_grads = grads
            self._desc = torch.from_numpy(self._host_desc.view(np.uint8)).to(ps[0].device, non_blocking=False)

    def _layout(self, ps: List[torch.nn.Parameter]) -> None:
        C = native()
        chunk = C.adam_chunk_size()
        assert C.adam_tensor_desc_bytes() == _DESC.itemsize
        wd_of = {id(p): float(g["weight_decay"]) for g in self.param_groups for p in g["params"]}
        rows, owner, goff = [], [], []
        for k, p in enumerate(ps):
            st, g = self.state[p], p.grad
            if not g.is_contiguous():
                raise RuntimeError("FusedAdamW needs contiguous gradients")
            if p.dtype not in (torch.bfloat16, torch.float32):
                raise RuntimeError(f"unsupported parameter dtype {p.dtype}")
            if p.dtype == torch.float32:
                st["master"] = p.data  # fp32 parameters: the parameter itself is the master copy
            alias = self._param16.get(p)
            p16 = alias if alias is not None else (p if p.dtype == torch.bfloat16 else None)
            for (a, b, seg_wd) in self._segments.get(p, [(0, p.numel(), wd_of[id(p)])]):
                if b <= a:
                    continue
                rows.append((st["master"].data_ptr() + 4 * a, (p16.data_ptr() + 2 * a) if p16 is not None else 0, 0,
                             st["exp_avg"].data_ptr() + 4 * a, st["exp_avg_sq"].data_ptr() + 4 * a, b - a,
                             float(seg_wd), 1 if g.dtype == torch.bfloat16 else 0))
                owner.append(k)
                goff.append(g.element_size() * a)
        self._host_desc = np.array(rows, dtype=_DESC)
        self._entry_param = np.asarray(owner, dtype=np.int64)
        self._entry_goff = np.asarray(goff, dtype=np.uint64)
        self._entry_grads = None
        # chunk list: (segment, chunk within segment) for every chunk of every segment
        per = (self._host_desc["n"] + chunk - 1) // chunk
        seg = np.repeat(np.arange(len(rows), dtype=np.int32), per)
        first = np.repeat(np.cumsum(per) - per, per)
        pairs = np.stack([seg, (np.arange(seg.size) - first).astype(np.int32)], 1)
        dev = ps[0].device
        self._chunks = torch.from_numpy(np.ascontiguousarray(pairs)).reshape(-1).to(dev)
        self._nchunks = int(seg.size)
        self._grad_mask = np.zeros(len(self._param_index), dtype=bool)
        self._grad_mask[[self._param_index[id(p)] for p in ps]] = True

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def clip_grad_norm(self, max_norm: float, inv_scale: float = 1.0) -> torch.Tensor:
        """Compute the global grad norm on device and arm the clip coefficient for ``step``.

        Returns a 0-d device tensor with the (unscaled) norm; nothing is synchronised.
        """
        self._build_desc()
        if self._group is None or not torch.distributed.is_initialized() or \
                torch.distributed.get_world_size(self._group) == 1:
            native().grad_norm(self._desc, self._chunks, self._nchunks, self._partial, float(max_norm),
                               float(inv_scale), self.norm_coef, False)
        else:
            native().grad_norm(self._desc, self._chunks, self._nchunks, self._partial, float(max_norm),
                               float(inv_scale), self.norm_coef, True)
            torch.distributed.all_reduce(self.norm_coef[:1], group=self._group)
            native().grad_norm_finish(self.norm_coef, float(max_norm), float(inv_scale))
        self._armed = True
        return self.norm_coef[0]

    @torch.no_grad()
    def arm_clip(self, norm: torch.Tensor, max_norm: float) -> None:
        """Use a norm computed elsewhere (model-parallel reductions) for the next ``step``'s clip coefficient:
        ``min(1, max_norm / (norm + 1e-6))``, or 0 (skip the update) when the norm is not finite."""
        self.norm_coef[0] = norm
        coef = (max_norm / (norm + 1e-6)).clamp(max=1.0) if max_norm > 0 else torch.ones_like(norm)
        self.norm_coef[1] = torch.where(torch.isfinite(norm), coef, torch.zeros_like(coef))
        self._armed = True

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        self._build_desc()
        if self._nchunks == 0:
            return loss
        if not getattr(self, "_armed", False):
            self.norm_coef.fill_(1.0)
        self._armed = False
        self._step += 1
        g0 = self.param_groups[0]
        lrs = {float(g["lr"]) for g in self.param_groups}
        if len(lrs) != 1:
            raise RuntimeError("FusedAdamW expects one learning rate for all groups")
        b1, b2 = g0["betas"]
        self._param_steps += self._grad_mask
        native().adam_step(self._desc, self._chunks, self._nchunks, self.norm_coef, float(g0["lr"]), float(b1),
                           float(b2), float(g0["eps"]), self._step, self.decoupled)
        if self._post_step is not None:
            self._post_step()
        return loss

    def zero_grad(self, set_to_none: bool = True) -> None:
        super().zero_grad(set_to_none=set_to_none)

    # ------------------------------------------------------------------ (de)serialisation
    def state_dict(self):
        for p, n in zip(self._params(), self._param_steps):
            self.state[p]["step"] = torch.tensor(float(n))
        sd = super().state_dict()
        # detach views from the flat buffers so a checkpoint stores each tensor once
        for st in sd["state"].values():
            for k, v in list(st.items()):
                if isinstance(v, torch.Tensor):
                    st[k] = v.detach().clone()
        sd["fused_step"] = self._step
        return sd

    def load_state_dict(self, state_dict) -> None:
        ps = self._params()
        saved = state_dict.get("state", {})
        for i, p in enumerate(ps):
            src = saved.get(i, {})
            st = self.state[p]
            for k in ("exp_avg", "exp_avg_sq", "master"):
                if k in src:
                    st[k].copy_(src[k].to(st[k].device, torch.float32))
                elif k == "master":
                    st[k].copy_(p.detach().float())
            if "step" in src:
                self._param_steps[i] = int(float(src["step"]))
        for g, sg in zip(self.param_groups, state_dict.get("param_groups", [])):
            for k, v in sg.items():
                if k != "params":
                    g[k] = v
        self._step = int(state_dict.get("fused_step", max((int(s.get("step", 0)) for s in saved.values()),
                                                          default=0)))
        # re-derive the bf16 compute weights from the restored masters
        with torch.no_grad():
            for p in ps:
                if p.dtype != torch.float32:
                    p.copy_(self.state[p]["master"].to(p.dtype))
                if p in self._param16:
                    self._param16[p].copy_(self.state[p]["master"].to(self._param16[p].dtype))
        self._desc_key = None

    def master_params(self) -> Dict[torch.nn.Parameter, torch.Tensor]:
        return {p: self.state[p]["master"] for p in self._params()}
