"""Reference arm of bench.py: the UNMODIFIED reference (Forgeline) from ``baseline/_ref``.

Nothing from ``rl_project_b200`` is imported here.  The reference snapshot
lacks its ``forgeline.checkpoints`` package (its own .gitignore dropped it), so
the modules that import it at load time get an in-memory stand-in registered
in ``sys.modules``; no file of the installed reference is changed.

Workload = bench.py's (dense-1B SFT, seq 4096, 8 seqs/GPU, 25% prompt mask,
bf16).  The reference cannot express two of the config's fields, so they are
set from outside through its public classes:
  * d_ff 8192 (its SwiGLU width is derived, 5504 at d=2048): each block's
    ``ffn.w1/w2/w3`` are replaced by ``nn.Linear`` of width 8192 and
    initialised with the reference's own init rule;
  * RoPE theta 500000 (hard-coded 10000): each attention's ``rotary_emb`` is
    replaced by the reference's ``RotaryEmbedding(..., base=500000)``.
Step = reference ``FSDPStrategy`` (FULL_SHARD, bf16 MixedPrecision, size-based
auto-wrap) + ``build_optimizer`` (fused AdamW) + ``Precision`` autocast +
``TransformerLM.forward(idx, targets)`` (CE with ignore -1) + FSDP
``clip_grad_norm_`` + optimizer step, and the reference Trainer's per-step
loss read-back.
"""

from __future__ import annotations

import math
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def _install_checkpoint_stand_in() -> None:
    import torch

    pkg = types.ModuleType("forgeline.checkpoints")
    mgr = types.ModuleType("forgeline.checkpoints.manager")
    val = types.ModuleType("forgeline.checkpoints.validation")

    class CheckpointState:  # only constructed if a checkpoint is written (never in the benchmark)
        def __init__(self, model_state=None, **kw):
            self.model_state = model_state
            self.__dict__.update(kw)

    class CheckpointManager:
        def __init__(self, root, keep_last=3, async_save=False):
            self.root = root

        def save(self, *a, **k):
            raise RuntimeError("checkpointing is not part of the benchmark")

        def wait(self):
            pass

        def find_latest(self):
            return None

    def load_model_state(model, state, strict=True):
        state = {k.replace("_orig_mod.", ""): v for k, v in state.items()}
        return model.load_state_dict(state, strict=strict)

    mgr.CheckpointManager, mgr.CheckpointState, mgr.load_model_state = CheckpointManager, CheckpointState, load_model_state
    val.compare_state_shapes = lambda m, s: {"mismatched": {}}
    val.assert_compatible = lambda m, s: None
    val.finite_state = lambda s: all(torch.isfinite(v).all() for v in s.values() if torch.is_tensor(v))
    pkg.manager, pkg.validation = mgr, val
    pkg.CheckpointManager, pkg.CheckpointState, pkg.load_model_state = CheckpointManager, CheckpointState, load_model_state
    sys.modules["forgeline.checkpoints"] = pkg
    sys.modules["forgeline.checkpoints.manager"] = mgr
    sys.modules["forgeline.checkpoints.validation"] = val


def _unavailable(reason: str) -> dict:
    return {"impl": "reference", "unavailable": reason}


def run_reference(args, world, rank, local, *, time_device, time_wall, clock_sampler, metric, model_name):
    if not os.path.isdir(os.path.join(REF, "forgeline")):
        return _unavailable("reference not installed in baseline/_ref (pip install --target baseline/_ref failed)")
    sys.path.insert(0, REF)
    _install_checkpoint_stand_in()
    import torch
    import torch.nn as nn

    from forgeline.core.config import DistributedConfig, ModelSpec, OptimizerConfig, PrecisionConfig
    from forgeline.distributed.strategies import FSDPStrategy
    from forgeline.models.attention.rotary import RotaryEmbedding
    from forgeline.models.transformer.model import TransformerLM
    from forgeline.training.common.optim import build_optimizer
    from forgeline.training.common.precision import Precision

    seq, bpg = args.seq, args.batch_per_gpu
    spec = ModelSpec(block_size=seq, vocab_size=128256, n_layer=16, n_head=32, n_kv_head=8, n_embd=2048, dropout=0.0,
                     bias=False, use_rope=True, use_swiglu=True)
    strategy = FSDPStrategy(DistributedConfig(strategy="fsdp", backend="nccl"), dtype=torch.bfloat16)
    strategy.setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    torch.manual_seed(1234)
    model = TransformerLM(spec)
    d_ff = 8192
    for blk in model.transformer.h:
        ffn = blk.ffn
        ffn.w1 = nn.Linear(spec.n_embd, d_ff, bias=False)
        ffn.w3 = nn.Linear(spec.n_embd, d_ff, bias=False)
        ffn.w2 = nn.Linear(d_ff, spec.n_embd, bias=False)
        for lin in (ffn.w1, ffn.w3):
            TransformerLM._init_weights(lin)
        nn.init.normal_(ffn.w2.weight, mean=0.0, std=0.02 / math.sqrt(2 * spec.n_layer))
        blk.attn.rotary_emb = RotaryEmbedding(spec.n_embd // spec.n_head, max_seq_len=seq, base=500000.0)
    model = strategy.wrap_model(model.to(device))
    opt = build_optimizer(model.parameters(), OptimizerConfig(learning_rate=3e-4, weight_decay=0.1, grad_clip=1.0),
                          device)
    prec = Precision(PrecisionConfig(dtype="bfloat16"), device, torch.bfloat16)

    g = torch.Generator().manual_seed(1234 * 1_000_003 + rank)
    toks = torch.randint(0, spec.vocab_size, (bpg, seq + 1), generator=g)
    x_h, y_h = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    y_h[:, : seq // 4 - 1] = -1
    x_h, y_h = x_h.pin_memory(), y_h.pin_memory()
    x_d, y_d = x_h.to(device), y_h.to(device)
    state = {"x": x_d, "y": y_d, "host": False, "loss": None}

    def step():
        if state["host"]:
            x = x_h.to(device, non_blocking=True)
            y = y_h.to(device, non_blocking=True)
        else:
            x, y = state["x"], state["y"]
        opt.zero_grad(set_to_none=True)
        with prec.autocast():
            _, loss = model(x, y)
        if not torch.isfinite(loss):  # the reference Trainer's per-step check
            raise RuntimeError("non-finite loss")
        prec.backward(loss)
        prec.unscale(opt)
        strategy.clip_grad_norm(model, 1.0)
        prec.step(opt)
        state["loss"] = float(loss.detach())

    for _ in range(args.warmup):
        step()
    clk = clock_sampler(local)
    clk.start()
    ms = time_device(step, args.steps)
    clocks = clk.stop()
    tokens = seq * bpg * world
    e2e = None
    if not args.no_e2e:
        state["host"] = True
        step()
        k = args.e2e_steps or args.steps
        ms_e2e = time_wall(step, k)
        e2e = {"value": tokens / (ms_e2e / 1e3), "unit": "tokens/s", "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": x_h.numel() * 8 * 2, "d2h_bytes_per_step": 4,
               "api": "reference TransformerLM.forward + FSDPStrategy + build_optimizer"}
    strategy.teardown()
    return {"metric": metric, "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform token ids; random-init weights)",
            "config": {"model": model_name, "global_batch": bpg * world, "seq_len": seq,
                       "parallelism": f"fsdp{world}", "l2": "inputs larger than L2",
                       "patched_from_outside": ["ffn width 8192", "rope theta 500000"],
                       "final_loss": state["loss"]},
            "clocks": clocks, "e2e": e2e, "gpu_launches": 0, "impl": "reference"}
