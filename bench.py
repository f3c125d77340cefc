#!/usr/bin/env python
"""Headline benchmark: dense-1B SFT training tokens/s on N B200 GPUs.

Config (the dense-1B SFT headline): 16 layers, d_model 2048, 32 query / 8 KV heads,
head_dim 64, SwiGLU d_ff 8192, RMSNorm, RoPE theta 500000, vocab 128256, tied
embeddings; seq 4096, 8 sequences per GPU (weak scaling), first 25% of each
sequence prompt-masked; bf16; synthetic uniform token ids; random init.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

For N > 1 launch one rank per GPU with torch.distributed.run (127.0.0.1).
Two timed phases over the same Trainer.train_step (the public training API):
  * value: device time (CUDA events, barrier + synchronize on both sides,
    max over ranks) with the batch already resident on the device;
  * e2e:   wall time per step including the pinned-host -> device copy of the
    batch and the device -> host read of the loss, max over ranks.
Rank 0 prints ONE JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "train tokens/s (FSDP/TP/EP) + GRPO tokens/s at 1/2/4/8 B200 vs ref NCCL build"
MODEL_NAME = "dense-1B (16L d2048 32q/8kv hd64 ff8192 V128256 tied, RoPE 5e5)"
BASELINE_VALUE = None  # the reference published no number for this configuration


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--batch-per-gpu", type=int, default=8)
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--phase-steps", type=int, default=2,
                    help="untimed steps after the timed region with per-phase CUDA events (0: none)")
    ap.add_argument("--workload", choices=["sft1b", "mesh8b", "moe", "grpo"], default="sft1b",
                    help="sft1b: the headline (dense 1B SFT). mesh8b: dense-8B pretrain on a TP x PP x DP "
                         "mesh (1F1B). moe: MLA+MoE pretrain with expert parallelism. grpo: GRPO rollout+update, "
                         "FSDP learner + tensor-parallel rollout replicas on N GPUs (rl_project_b200.benchmarks.grpo; "
                         "its flags pass through).")
    ap.add_argument("--tp", type=int, default=2)
    ap.add_argument("--pp", type=int, default=2)
    ap.add_argument("--micro", type=int, default=8)
    ap.add_argument("--global-batch", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None, help="override the preset's layer count (smoke runs)")
    ap.add_argument("--grad-ckpt", action="store_true")
    ap.add_argument("--fused-comm", choices=["auto", "on", "off", "nccl_baseline"], default="auto",
                    help="FSDP gradient reduce-scatter: fused peer-memory kernel (auto/on) or NCCL")
    ap.add_argument("--fused-rs-ctas", type=int, default=32,
                    help="CTAs of each fused reduce-scatter that overlaps backward")
    ap.add_argument("--fused-multicast", choices=["off", "on", "symm"], default="off",
                    help="fused reduce-scatter transport: CUDA IPC peer loads (off) or NVLink multicast (on)")
    ap.add_argument("--gemm", choices=["tcgen05", "cublas", "tuned", "hybrid", "fwd_dgrad"], default="hybrid",
                    help="dense linear layers and LM head: hybrid (default: own 2-SM tcgen05 GEMM for the forward "
                         "products, SwiGLU fused into the FFN projection's epilogue, cuBLAS for the gradient products), "
                         "tcgen05 (own kernel for all), fwd_dgrad (own forward and input gradients), cublas, or tuned "
                         "(per shape the fastest, timed on the first call of each shape)")
    ap.add_argument("--attn", choices=["sdpa", "tcgen05"], default="sdpa",
                    help="training / prefill attention: torch SDPA (cuDNN / flash) or this library's tcgen05 kernels")
    ap.add_argument("--decode-graphs", choices=["on", "off"], default="on",
                    help="grpo workload: replay the paged decode step from CUDA graphs (single-GPU engines)")
    args, extra = ap.parse_known_args()
    args.extra = extra
    if extra and args.workload != "grpo":
        ap.error(f"unrecognised arguments: {' '.join(extra)}")
    return args


def apply_kernel_choices(args) -> dict:
    """Route attention / decode as the flags ask (before any model is built); returns the choices."""
    from rl_project_b200.ops import attention, gemm

    attention._ATTN = args.attn
    gemm._MODE = args.gemm
    os.environ["RLB_DECODE_GRAPHS"] = "1" if args.decode_graphs == "on" else "0"
    return {"attention": args.attn, "gemm": args.gemm, "decode_graphs": args.decode_graphs == "on"}


def gemm_choice_summary() -> dict:
    """In ``--gemm tuned`` mode: how many product shapes went to each kernel."""
    from rl_project_b200.ops import gemm

    picks = gemm.tuned_choices()
    if not picks:
        return {}
    counts: dict = {}
    for (a_mn, b_mn, _, M, N, K, _), choice in picks.items():
        layout = {(0, 0): "fwd", (0, 1): "dgrad", (1, 1): "wgrad"}.get((a_mn, b_mn), "other")
        counts.setdefault(layout, {}).setdefault(choice, 0)
        counts[layout][choice] += 1
    return {"gemm_tuned_picks": counts}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), float(parts[3]), float(parts[4]), parts[5:9]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [r for r in rows if r[3] >= 50] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[4]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(loaded), "reasons": reasons}


# --------------------------------------------------------------------------- helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float) -> float:
    import torch
    import torch.distributed as dist

    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def barrier():
    import torch
    import torch.distributed as dist

    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier(device_ids=[torch.cuda.current_device()])


def time_device(step, k: int) -> float:
    """ms per step: CUDA events on the launching stream, barrier+sync both sides, max over ranks."""
    import torch

    barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(k):
        step()
    b.record()
    torch.cuda.synchronize()
    barrier()
    return max_over_ranks(a.elapsed_time(b) / k)


def time_wall(step, k: int) -> float:
    import torch

    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(k):
        step()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier()
    return max_over_ranks((t1 - t0) * 1e3 / k)


def phase_breakdown(trainer, steps: int) -> dict:
    """Per-phase device time of a training step (ms, mean over `steps` untimed steps run after the timed region,
    max over ranks per phase): forward, backward (each with the collectives the strategy overlaps into them),
    grad_sync (the exposed tail of the gradient reduction), clip (global norm, incl. its all-reduce), optimizer,
    start (the device idle gap between steps).  Every rank takes the same all-reduces in the same order."""
    if steps <= 0:
        return {}
    trainer.phase_events = []
    for _ in range(steps):
        trainer.train_step()
    times = trainer.phase_times(trainer.phase_events)
    trainer.phase_events = None
    return {k: round(max_over_ranks(times.get(k, 0.0) / steps), 3)
            for k in ("forward", "backward", "grad_sync", "clip", "optimizer", "start")}


def emit(rank: int, payload: dict) -> None:
    if rank == 0:
        print(json.dumps(payload), flush=True)


# --------------------------------------------------------------------------- our framework
def run_ours(args, world, rank, local):
    import torch

    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.data.synthetic import SyntheticSFTSource
    from rl_project_b200.data.tokenizers import ByteTokenizer
    from rl_project_b200.models.policy import NativePolicy
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.ops._ext import launch_count, native
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.sft import SFTAlgorithm, SFTConfig

    native()  # the sm_100a library must be loaded
    strategy_name = "fsdp" if world > 1 else "single"
    manifest = ExperimentManifest.from_dict({
        "name": "bench-dense1b-sft", "algorithm": "sft", "model_preset": "bl_dense_1b",
        "model": {"block_size": args.seq},
        "trainer": {"batch_size": args.batch_per_gpu, "max_steps": 10**9, "eval_every": 0, "log_every": 0,
                    "seed": 1234, "precision": {"dtype": "bfloat16"},
                    "optimizer": {"learning_rate": 3e-4, "grad_clip": 1.0, "weight_decay": 0.1},
                    "schedule": {"name": "constant", "warmup_steps": 0},
                    "checkpoint": {"save_every": 0, "auto_resume": False}},
        "distributed": {"strategy": strategy_name, "timeout_s": 300, "fused_comm": args.fused_comm,
                        "fused_multicast": args.fused_multicast, "fused_rs_ctas": args.fused_rs_ctas},
        "output_dir": os.path.join(tempfile.gettempdir(), f"rlb_bench_{rank}"),
    })
    strategy = build_strategy(manifest.distributed)
    strategy.setup()
    torch.cuda.set_device(local)
    ctx = RunContext.create(manifest, metrics_backend="none", distributed=world > 1)
    spec = manifest.model
    torch.manual_seed(1234)
    with torch.device(ctx.device):
        model = TransformerLM(spec)
    policy = NativePolicy(model, ByteTokenizer())
    host_src = SyntheticSFTSource(spec.vocab_size, args.seq, args.batch_per_gpu, prompt_fraction=0.25, seed=1234,
                                  rank=rank, pin=True)

    class Resident:
        """The same batches, already on the device (device-timed phase)."""

        def __init__(self, src):
            self.batches = [b.to(ctx.device) for b in src._pool]
            self.i = 0

        def next_batch(self):
            b = self.batches[self.i % len(self.batches)]
            self.i += 1
            return b

    alg = SFTAlgorithm(policy, Resident(host_src), SFTConfig(batch_size=args.batch_per_gpu, max_length=args.seq + 1))
    trainer = Trainer(ctx, alg, strategy=strategy)
    n_params = sum(p.numel() for p in model.parameters())

    for _ in range(args.warmup):
        trainer.train_step()
    clocks = ClockSampler(local)
    clocks.start()
    l0 = launch_count()
    ms = time_device(trainer.train_step, args.steps)
    launches = launch_count() - l0  # every native launch of the K timed steps
    clk = clocks.stop()
    tokens_step = args.seq * args.batch_per_gpu * world
    value = tokens_step / (ms / 1e3)
    phases = phase_breakdown(trainer, args.phase_steps)

    e2e = None
    if not args.no_e2e:
        alg.dataset = host_src  # pinned host batches -> device every step, loss read back every step
        for _ in range(max(1, args.warmup // 2)):
            trainer.train_step()
        k = args.e2e_steps or args.steps
        ms_e2e = time_wall(trainer.train_step, k)
        h2d = host_src.bytes_per_batch()
        e2e = {"value": tokens_step / (ms_e2e / 1e3), "unit": "tokens/s", "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4 * (2 + 1), "api": "Trainer.train_step"}

    last = trainer.history[-1]
    flops_tok = 6 * n_params + 12 * spec.n_layer * spec.n_embd * args.seq // 2  # causal attention
    peak = _peak_tflops()
    payload = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None, "dtype": "bf16",
        "data": "synthetic (uniform token ids, seeded per rank; random-init weights)",
        "config": {"model": MODEL_NAME, "global_batch": args.batch_per_gpu * world, "seq_len": args.seq,
                   "parallelism": (f"fsdp{world}" if world > 1 else "single"), "prompt_mask": 0.25,
                   "params": n_params, "optimizer": "AdamW fp32 master, clip 1.0",
                   "l2": "inputs larger than L2 (activations >> 126 MB per step)",
                   "model_tflops_per_gpu": flops_tok * args.seq * args.batch_per_gpu / (ms / 1e3) / 1e12,
                   "mfu_vs_measured_bf16": (flops_tok * args.seq * args.batch_per_gpu / (ms / 1e3) / 1e12 / peak)
                   if peak else None,
                   "attention": args.attn, "gemm": args.gemm, **gemm_choice_summary(),
                   "final_loss": last.loss, "first_loss": trainer.history[0].loss,
                   "final_grad_norm": last.metrics.get("grad_norm"),
                   "grad_reduce": ("fused peer-memory reduce-scatter" + (" (NVLink multicast)"
                                   if getattr(strategy, "fused", None) is not None and strategy.fused.uses_multicast
                                   else "") if getattr(strategy, "fused", None) is not None
                                   else ("nccl reduce-scatter" if world > 1 else "none"))},
        "clocks": clk, "e2e": e2e, "gpu_launches": int(launches), "impl": "ours",
    }
    if phases:
        payload["config"]["phases_ms"] = phases
    emit(rank, payload)
    strategy.teardown()


def run_pretrain_workload(args, world, rank, local):
    """Configs 3 (mesh8b) and 4 (moe): synthetic pretraining through Trainer.train_step on a parallel layout."""
    import torch

    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.data.synthetic import SyntheticPretrainSource
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.ops._ext import launch_count, native
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    native()

    def tp_fused_used() -> bool:
        from rl_project_b200.parallel import tp_fused

        return any(r is not None and r.launches > 0 for r in tp_fused._REDUCERS.values())

    tp = 1
    if args.workload == "mesh8b":
        preset, seq = "bl_dense_8b", (args.seq if args.seq != 4096 else 8192)
        tp, pp = (args.tp, args.pp) if world > 1 else (1, 1)
        dp = world // (tp * pp)
        strategy = "single" if world == 1 else ("hybrid" if tp > 1 and pp > 1 else
                                                ("tensor_parallel" if tp > 1 else "pipeline_parallel"))
        gb = args.global_batch or 64
        dist_cfg = {"strategy": strategy, "tensor_parallel_size": tp, "pipeline_parallel_size": pp,
                    "timeout_s": 600, "fused_comm": args.fused_comm}
        layout = f"tp{tp}xpp{pp}xdp{dp}"
        micro = args.micro
    else:
        preset, seq = "bl_mla_moe", args.seq
        dp = world
        strategy = "expert_parallel" if world > 1 else "single"
        gb = args.global_batch or 4 * world
        dist_cfg = {"strategy": strategy, "expert_parallel_size": max(world, 1), "timeout_s": 600,
                    "fused_comm": args.fused_comm}
        layout = f"ep{world}" if world > 1 else "single"
        micro = 1
    rows = gb // dp
    model_over = {"block_size": seq}
    if args.layers:
        model_over["n_layer"] = args.layers
    manifest = ExperimentManifest.from_dict({
        "name": f"bench-{args.workload}", "algorithm": "pretrain", "model_preset": preset, "model": model_over,
        "trainer": {"batch_size": rows, "gradient_accumulation_steps": micro, "max_steps": 10 ** 9, "eval_every": 0,
                    "log_every": 0, "seed": 1234, "precision": {"dtype": "bfloat16"},
                    "gradient_checkpointing": bool(args.grad_ckpt),
                    "optimizer": {"learning_rate": 3e-4, "grad_clip": 1.0, "weight_decay": 0.1},
                    "schedule": {"name": "constant", "warmup_steps": 0},
                    "checkpoint": {"save_every": 0, "auto_resume": False}},
        "distributed": dist_cfg, "output_dir": os.path.join(tempfile.gettempdir(), f"rlb_bench_{rank}")})
    strat = build_strategy(manifest.distributed)
    strat.setup()
    torch.cuda.set_device(local)
    ctx = RunContext.create(manifest, metrics_backend="none", distributed=world > 1)
    spec = manifest.model
    torch.manual_seed(1234)
    with torch.device(ctx.device):
        model = TransformerLM(spec)
    n_params_full = sum(p.numel() for p in model.parameters())
    from rl_project_b200.parallel.mesh_strategies import data_parallel_rank

    src = SyntheticPretrainSource(spec.vocab_size, seq, rows, seed=1234, rank=data_parallel_rank())
    batches = [tuple(t.to(ctx.device) for t in next(iter(src))) for _ in range(2)]

    class Resident:
        def __init__(self):
            self.i = 0

        def __iter__(self):
            return self

        def __next__(self):
            self.i += 1
            return batches[self.i % 2]

    alg = PretrainAlgorithm(model, Resident(), PretrainConfig(batch_size=rows), device=ctx.device)
    trainer = Trainer(ctx, alg, strategy=strat)
    for _ in range(args.warmup):
        trainer.train_step()
    clocks = ClockSampler(local)
    clocks.start()
    l0 = launch_count()
    ms = time_device(trainer.train_step, args.steps)
    launches = launch_count() - l0  # every native launch of the K timed steps
    clk = clocks.stop()
    tokens = seq * gb
    payload = {"metric": METRIC, "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
               "scaling": "strong" if args.workload == "mesh8b" else "weak", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (uniform token ids; random-init weights)",
               "config": {"model": preset + (f" ({args.layers} layers)" if args.layers else ""), "global_batch": gb,
                          "seq_len": seq, "parallelism": layout, "micro_batches": micro,
                          "params_full_model": n_params_full, "workload": args.workload,
                          "l2": "inputs larger than L2", "first_loss": trainer.history[0].loss,
                          "final_loss": trainer.history[-1].loss,
                          "loss_terms": ("next-token CE + MTP CE x mtp_loss_weight (about 2 ln V at init)"
                                         if spec.n_predict_tokens > 1 else "next-token CE"),
                          "attention": args.attn, "gemm": args.gemm,
                          "tp_allreduce": (("fused tcgen05 GEMM epilogue over peer memory"
                                            if tp_fused_used() else "nccl") if args.workload == "mesh8b"
                                           and world > 1 and tp > 1 else None)},
               "clocks": clk, "e2e": None, "gpu_launches": int(launches), "impl": "ours"}
    emit(rank, payload)
    strat.teardown()


def _peak_tflops():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["bf16_tflops_sustained"])
    except Exception:
        return None


def main():
    args = parse_args()
    world, rank, local = dist_env()
    if os.environ.get("RLB_HANG_DUMP_S"):
        # diagnostics: every thread's Python stack goes to stderr after this many seconds (the run goes on)
        import faulthandler

        faulthandler.dump_traceback_later(float(os.environ["RLB_HANG_DUMP_S"]), repeat=False)
    if world != args.gpus:
        if rank == 0:
            print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        from baseline.harness import run_reference, run_reference_workload

        if args.workload in ("mesh8b", "moe"):
            payload = run_reference_workload(args, world, rank, local, time_device=time_device,
                                             clock_sampler=ClockSampler, metric=METRIC)
        elif args.workload == "grpo":
            payload = {"impl": "reference", "unavailable": "GRPO reference arm not built: the reference runs GRPO "
                       "only under DDP, whose 8B replica needs about 160 GB per GPU before activations (fp32 weights, "
                       "gradients, AdamW state and the fp32 frozen copy), and the FSDP fallback loop is not written"}
        else:
            payload = run_reference(args, world, rank, local, time_device=time_device, time_wall=time_wall,
                                    clock_sampler=ClockSampler, metric=METRIC, model_name=MODEL_NAME)
        emit(rank, payload)
        return
    apply_kernel_choices(args)
    if args.workload in ("mesh8b", "moe"):
        run_pretrain_workload(args, world, rank, local)
        return
    if args.workload == "grpo":
        from rl_project_b200.benchmarks import grpo

        # the GRPO flags (--preset, --prompts, --group, --max-new, --rollout-tp, ...) pass through
        grpo.run(["--steps", str(args.steps), "--warmup", str(args.warmup)] + list(args.extra))
        return
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
