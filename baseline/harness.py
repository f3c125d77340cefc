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
Step = the reference's strategy (N = 1: ``SingleProcessStrategy``, the model
unwrapped, as its Trainer runs one device; N > 1: ``FSDPStrategy`` with
FULL_SHARD, bf16 MixedPrecision, size-based auto-wrap) + ``build_optimizer``
(fused AdamW) + ``Precision`` autocast + ``TransformerLM.forward(idx, targets)``
(CE with ignore -1) + gradient-norm clip + optimizer step, and the reference
Trainer's per-step loss read-back.  Data: the same two-batch pool as
bench.py's own arm (same generator seed and draw order per rank), alternated.
At N = 1 a second number, ``compiled``, times the same step after the
reference's own ``compile_model`` path (``nn.Module.compile`` in place,
its Trainer's ``_compile_modules``), the configuration its published A40
run used.
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
    from forgeline.distributed.strategies import FSDPStrategy, SingleProcessStrategy
    from forgeline.models.attention.rotary import RotaryEmbedding
    from forgeline.models.transformer.model import TransformerLM
    from forgeline.training.common.optim import build_optimizer
    from forgeline.training.common.precision import Precision

    seq, bpg = args.seq, args.batch_per_gpu
    spec = ModelSpec(block_size=seq, vocab_size=128256, n_layer=16, n_head=32, n_kv_head=8, n_embd=2048, dropout=0.0,
                     bias=False, use_rope=True, use_swiglu=True)
    if world > 1:
        strategy = FSDPStrategy(DistributedConfig(strategy="fsdp", backend="nccl"), dtype=torch.bfloat16)
    else:
        strategy = SingleProcessStrategy(DistributedConfig(strategy="single"))
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

    # the two-batch pool of bench.py's own arm: same generator seed per rank, same draws in the same order
    g = torch.Generator().manual_seed(1234 * 1_000_003 + rank)
    pool = []
    for _ in range(2):
        toks = torch.randint(0, spec.vocab_size, (bpg, seq + 1), generator=g)
        x_h, y_h = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
        y_h[:, : seq // 4 - 1] = -1
        x_h, y_h = x_h.pin_memory(), y_h.pin_memory()
        pool.append((x_h, y_h, x_h.to(device), y_h.to(device)))
    state = {"i": 0, "host": False, "loss": None}

    def clip():
        if world > 1:
            strategy.clip_grad_norm(model, 1.0)
        else:
            torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)

    def step():
        x_h, y_h, x_d, y_d = pool[state["i"] % 2]
        state["i"] += 1
        if state["host"]:
            x = x_h.to(device, non_blocking=True)
            y = y_h.to(device, non_blocking=True)
        else:
            x, y = x_d, y_d
        opt.zero_grad(set_to_none=True)
        with prec.autocast():
            _, loss = model(x, y)
        if not torch.isfinite(loss):  # the reference Trainer's per-step check
            raise RuntimeError("non-finite loss")
        prec.backward(loss)
        prec.unscale(opt)
        clip()
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
               "h2d_bytes_per_step": pool[0][0].numel() * 8 * 2, "d2h_bytes_per_step": 4,
               "api": "reference TransformerLM.forward + " + type(strategy).__name__ + " + build_optimizer"}
    compiled = None
    if world == 1 and not os.environ.get("RLB_REF_NO_COMPILE"):
        # the reference Trainer's compile_model path: nn.Module.compile in place (default inductor backend)
        try:
            state["host"] = False
            model.compile()
            for _ in range(max(3, args.warmup)):  # the first calls compile
                step()
            ms_c = time_device(step, args.steps)
            compiled = {"value": tokens / (ms_c / 1e3), "ms_per_step": ms_c, "api": "nn.Module.compile (inductor)"}
        except Exception as e:  # noqa: BLE001 - recorded, the eager number stands
            compiled = {"error": f"{type(e).__name__}: {e}"[:300]}
    strategy.teardown()
    return {"metric": metric, "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform token ids; random-init weights)",
            "config": {"model": model_name, "global_batch": bpg * world, "seq_len": seq,
                       "parallelism": f"fsdp{world}" if world > 1 else "single", "l2": "inputs larger than L2",
                       "patched_from_outside": ["ffn width 8192", "rope theta 500000"],
                       "final_loss": state["loss"], "data_pool": "2 batches per rank, alternated (as bench.py)"},
            "clocks": clocks, "e2e": e2e, "compiled": compiled, "gpu_launches": 0, "impl": "reference"}


_PATCHES = {"mesh8b": ["ffn width 14336", "rope theta 500000", "untied lm_head"],
            "moe": ["dense ffn width 10944", "expert ffn width 1408", "shared expert ffn width 2816 (2 x 1408)"]}


def _build_reference_model(TransformerLM, spec, args, n_layer, seq, widen, RotaryEmbedding, nn):
    """The reference's TransformerLM with the config's widths set through its public modules."""
    model = TransformerLM(spec)
    if args.workload == "mesh8b":
        for blk in model.transformer.h:
            widen(blk.ffn, spec.n_embd, 14336, n_layer)
            blk.attn.rotary_emb = RotaryEmbedding(spec.n_embd // spec.n_head, max_seq_len=seq, base=500000.0)
        model.lm_head.weight = nn.Parameter(model.transformer.wte.weight.detach().clone())
        return model
    for blk in model.transformer.h:
        ffn = blk.ffn
        if hasattr(ffn, "experts"):
            for e in ffn.experts:
                widen(e, spec.n_embd, 1408, n_layer)
            if ffn.shared_experts is not None:  # one shared FFN of 2 x 1408 (the reference builds one)
                widen(ffn.shared_experts, spec.n_embd, 2 * 1408, n_layer)
        else:
            widen(ffn, spec.n_embd, 10944, n_layer)
    return model


def run_reference_workload(args, world, rank, local, *, time_device, clock_sampler, metric):
    """Reference arms of bench.py's ``--workload mesh8b`` and ``moe`` (config 4).

    The reference cannot run either layout (its TP breaks the attention reshape, its PP has no inter-stage
    backward, it has no expert parallelism), so, as planned for its baseline, each arm runs the reference's
    best runnable layout on the same GPUs: its ``TransformerLM`` under its own ``FSDPStrategy`` (FULL_SHARD,
    bf16 mixed precision) with every expert on every rank, its gradient checkpointing for the 8B model, its
    fused AdamW, the same global batch, sequence length and synthetic token distribution.  Widths the
    reference derives (dense / expert FFN), RoPE theta and the untied LM head of the 8B model are set from
    outside through its public modules and listed in ``patched_from_outside``.
    """
    if not os.path.isdir(os.path.join(REF, "forgeline")):
        return _unavailable("reference not installed in baseline/_ref (pip install --target baseline/_ref failed)")
    sys.path.insert(0, REF)
    _install_checkpoint_stand_in()
    import torch
    import torch.nn as nn

    from forgeline.core.config import DistributedConfig, ModelSpec, OptimizerConfig, PrecisionConfig
    from forgeline.distributed.strategies import FSDPStrategy, SingleProcessStrategy
    from forgeline.models.attention.rotary import RotaryEmbedding
    from forgeline.models.transformer.model import TransformerLM
    from forgeline.training.common.optim import build_optimizer
    from forgeline.training.common.precision import Precision

    def widen(ffn, dim, width, n_layer):
        ffn.w1 = nn.Linear(dim, width, bias=False)
        ffn.w3 = nn.Linear(dim, width, bias=False)
        ffn.w2 = nn.Linear(width, dim, bias=False)
        for lin in (ffn.w1, ffn.w3):
            TransformerLM._init_weights(lin)
        nn.init.normal_(ffn.w2.weight, mean=0.0, std=0.02 / math.sqrt(2 * n_layer))

    if args.workload == "mesh8b":
        seq = args.seq if args.seq != 4096 else 8192
        n_layer = args.layers or 32
        spec = ModelSpec(block_size=seq, vocab_size=128256, n_layer=n_layer, n_head=32, n_kv_head=8, n_embd=4096,
                         dropout=0.0, bias=False)
        gb = args.global_batch or 64
        ckpt = True
    else:
        seq = args.seq
        n_layer = args.layers or 27
        spec = ModelSpec(block_size=seq, vocab_size=102400, n_layer=n_layer, n_head=16, n_kv_head=16, n_embd=2048,
                         dropout=0.0, bias=False, use_mla=True, kv_lora_rank=512, q_lora_rank=0, qk_nope_head_dim=128,
                         qk_rope_head_dim=64, v_head_dim=128, use_moe=True, n_experts=64, n_experts_active=6,
                         n_shared_experts=2, n_dense_layers=1, score_func="sigmoid", aux_loss_free=True,
                         n_expert_groups=8, n_limited_groups=3, n_predict_tokens=2)
        gb = args.global_batch or 4 * world
        ckpt = bool(args.grad_ckpt)
    if gb % world:
        return _unavailable(f"global batch {gb} does not divide over {world} ranks")
    rows = gb // world
    strategy = (FSDPStrategy(DistributedConfig(strategy="fsdp", backend="nccl"), dtype=torch.bfloat16) if world > 1
                else SingleProcessStrategy(DistributedConfig(strategy="single")))
    strategy.setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    torch.manual_seed(1234)
    # built directly on the GPU (a default-device context; the reference code is unchanged): eight ranks each
    # materialising the 8B model in fp32 host memory first would need 256 GB of host RAM
    with torch.device(device):
        model = _build_reference_model(TransformerLM, spec, args, n_layer, seq, widen, RotaryEmbedding, nn)
    patched = _PATCHES[args.workload]
    if ckpt:
        model.enable_gradient_checkpointing()
    model = strategy.wrap_model(model.to(device))
    opt = build_optimizer(model.parameters(), OptimizerConfig(learning_rate=3e-4, weight_decay=0.1, grad_clip=1.0),
                          device)
    prec = Precision(PrecisionConfig(dtype="bfloat16"), device, torch.bfloat16)
    g = torch.Generator().manual_seed(1234 * 7919 + rank)
    pool = []
    for _ in range(2):
        toks = torch.randint(0, spec.vocab_size, (rows, seq + 1), generator=g)
        pool.append((toks[:, :-1].contiguous().to(device), toks[:, 1:].contiguous().to(device)))
    micro = 1 if args.workload == "mesh8b" else rows  # the 8B model: one sequence per micro-batch
    state = {"i": 0, "loss": None}

    def step():
        x, y = pool[state["i"] % 2]
        state["i"] += 1
        opt.zero_grad(set_to_none=True)
        total = torch.zeros((), device=device)
        for xs, ys in zip(x.split(micro), y.split(micro)):
            with prec.autocast():
                _, loss = model(xs, ys)
            prec.backward(loss * (xs.shape[0] / rows))
            total += loss.detach().float() * (xs.shape[0] / rows)  # read once, after timing
        prec.unscale(opt)
        if world > 1:
            strategy.clip_grad_norm(model, 1.0)
        else:
            torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        prec.step(opt)
        state["loss"] = total

    for _ in range(args.warmup):
        step()
    clk = clock_sampler(local)
    clk.start()
    ms = time_device(step, args.steps)
    clocks = clk.stop()
    strategy.teardown()
    return {"metric": metric, "value": seq * gb / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if args.workload == "mesh8b" else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform token ids; random-init weights)",
            "config": {"model": ("bl_dense_8b" if args.workload == "mesh8b" else "bl_mla_moe") +
                       (f" ({n_layer} layers)" if args.layers else ""), "global_batch": gb, "seq_len": seq,
                       "parallelism": f"fsdp{world}" if world > 1 else "single",
                       "reference_layout_note": "the config's TPxPP / EP layout is not runnable in the reference",
                       "gradient_checkpointing": ckpt, "patched_from_outside": patched,
                       "final_loss": float(state["loss"]), "workload": args.workload},
            "clocks": clocks, "e2e": None, "gpu_launches": 0, "impl": "reference"}
