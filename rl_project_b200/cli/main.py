"""``forgeline-b200`` command-line interface.

The command names and flags are those of the reference CLI (``src/forgeline/cli/main.py:21-586``), so scripts
written for it run unchanged: presets, validate, data, train, generate, evaluate, serve, export, registry,
rlaif, dashboard, allocation, synthesis-ppo.  The parser is generated from one table (``_command_table``) and
commands with sub-commands dispatch through handler tables.  Differences: ``train`` accepts every strategy
the trainer implements (single, ddp, fsdp, zero2, tensor / pipeline / expert parallel, hybrid) and ``serve``
runs the paged-KV engine.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

from rl_project_b200 import __version__
from rl_project_b200.core.errors import ForgelineError


def _print(obj: Any) -> None:
    print(obj if isinstance(obj, str) else json.dumps(obj, indent=2, default=str))


# ------------------------------------------------------------------ presets / validate / data
def cmd_presets(args: argparse.Namespace) -> int:
    from rl_project_b200.core.config import MODEL_PRESETS, model_spec_from_preset

    rows = []
    for name in MODEL_PRESETS:
        spec = model_spec_from_preset(name)
        row = {"preset": name, "layers": spec.n_layer, "heads": spec.n_head, "kv_heads": spec.n_kv_head,
               "dim": spec.n_embd, "context": spec.block_size, "moe": spec.use_moe, "mla": spec.use_mla,
               "sliding_window": spec.sliding_window}
        if args.count_params and spec.n_embd <= 1024:
            from rl_project_b200.models.transformer.model import TransformerLM

            with __import__("torch").device("meta"):
                model = TransformerLM(model_spec_from_preset(name, vocab_size=args.vocab_size))
            row["params_M"] = round(model.num_parameters() / 1e6, 1)
        rows.append(row)
    _print(rows)
    return 0


def cmd_validate(args: argparse.Namespace) -> int:
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.parallel.strategies import validate_distributed_config

    m = ExperimentManifest.load(args.manifest)
    topo = validate_distributed_config(m.distributed, world_size=args.world_size)
    _print({"ok": True, "name": m.name, "algorithm": m.algorithm, "model": m.model.to_dict(), "topology": topo})
    return 0


def _data_prepare(args):
    from rl_project_b200.data.preprocessing import prepare_text_corpus

    return prepare_text_corpus(args.input, args.output, tokenizer=args.tokenizer, val_fraction=args.val_fraction)


def _data_prepare_hf(args):
    from rl_project_b200.data.preprocessing import prepare_hf_corpus

    return prepare_hf_corpus(args.dataset, args.output, tokenizer_name=args.tokenizer, subset=args.subset,
                             max_tokens=args.max_tokens, shard_size=args.shard_size)


def _data_shard(args):
    from rl_project_b200.data.pretraining import detect_token_dtype
    from rl_project_b200.data.streaming import shard_token_file

    paths = shard_token_file(args.input, args.output, args.n_shards, dtype=detect_token_dtype(Path(args.input).parent))
    return [str(p) for p in paths]


def _data_gsm8k(args):
    from rl_project_b200.data.verifiable import build_gsm8k_tool_dataset

    return {"written": build_gsm8k_tool_dataset(args.output, split=args.split, limit=args.limit)}


def _data_validate(args):
    from rl_project_b200.data.records import SCHEMAS, ReadReport, read_jsonl

    report = ReadReport()
    rows = read_jsonl(args.input, SCHEMAS[args.kind], on_error="skip", report=report)
    return {"valid": len(rows), "skipped": report.skipped, "errors": report.errors[:20]}


_DATA = {"prepare": _data_prepare, "prepare-hf": _data_prepare_hf, "shard": _data_shard, "gsm8k": _data_gsm8k,
         "validate": _data_validate}


def cmd_data(args: argparse.Namespace) -> int:
    _print(_DATA[args.data_cmd](args))
    return 0


# ------------------------------------------------------------------ train
def apply_override(manifest, override: str) -> None:
    """``a.b.c=value`` dotted override; the value is parsed as YAML."""
    import yaml

    key, sep, raw = override.partition("=")
    if not sep:
        raise ForgelineError(f"override {override!r} must look like a.b.c=value")
    value = yaml.safe_load(raw)
    obj = manifest
    parts = key.split(".")
    for part in parts[:-1]:
        obj = obj[part] if isinstance(obj, dict) else getattr(obj, part)
    if isinstance(obj, dict):
        obj[parts[-1]] = value
    else:
        if not hasattr(obj, parts[-1]):
            raise ForgelineError(f"unknown manifest field {key!r}")
        setattr(obj, parts[-1], value)
    manifest.validate()


def _seed_per_rank(alg, strategy, manifest) -> None:
    """Model weights come from the base seed; sampling streams differ per data-parallel rank."""
    import random

    import torch

    from rl_project_b200.core.runtime import seed_everything

    if strategy.name == "single":
        return
    rank = strategy.rank()
    seed_everything(manifest.trainer.seed + rank)
    if hasattr(alg, "rng"):
        alg.rng = random.Random(manifest.trainer.seed + rank)
    if hasattr(alg, "gen"):
        alg.gen = torch.Generator().manual_seed(manifest.trainer.seed + rank)


def cmd_train(args: argparse.Namespace) -> int:
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.factory import build_algorithm

    manifest = ExperimentManifest.load(args.manifest)
    for ov in args.set or []:
        apply_override(manifest, ov)
    if args.max_steps is not None:
        manifest.trainer.max_steps = args.max_steps
    if args.output_dir:
        manifest.output_dir = args.output_dir
    manifest.with_runtime_environment()
    strategy = build_strategy(manifest.distributed)
    strategy.setup()
    ctx = RunContext.create(manifest, metrics_backend=args.metrics,
                            distributed=manifest.distributed.strategy != "single")
    if strategy.rank() == 0:
        manifest.save(Path(ctx.output_dir) / "manifest.yaml")
    alg = build_algorithm(manifest, ctx)
    _seed_per_rank(alg, strategy, manifest)
    trainer = Trainer(ctx, alg, strategy=strategy)
    if args.resume or manifest.trainer.checkpoint.resume_from:
        trainer.resume(args.resume or None)
    try:
        summary = trainer.fit()
    finally:
        if (manifest.orchestration or {}).get("type") == "ray":
            from rl_project_b200.orchestration.pools import shutdown_pools

            shutdown_pools()
        ctx.close()
        strategy.teardown()
    if strategy.rank() == 0:
        _print(summary)
    return 0


# ------------------------------------------------------------------ generate / evaluate / serve / export
def _load_policy(args: argparse.Namespace):
    from rl_project_b200.core.runtime import resolve_device
    from rl_project_b200.models.loading import load_policy_from_checkpoint

    return load_policy_from_checkpoint(args.checkpoint, resolve_device(args.device), data_dir=args.data_dir)


def cmd_generate(args: argparse.Namespace) -> int:
    from rl_project_b200.core.protocols import GenerationSettings
    from rl_project_b200.inference.generation import generate_text

    policy = _load_policy(args)
    settings = GenerationSettings(max_new_tokens=args.max_tokens, temperature=args.temperature,
                                  top_k=args.top_k or None, top_p=args.top_p, min_p=args.min_p,
                                  repetition_penalty=args.repetition_penalty, use_cache=not args.no_cache)
    spec_gen = None
    if args.draft_checkpoint:
        from rl_project_b200.models.generation.speculative import SpeculativeGenerator
        from rl_project_b200.models.loading import load_model_from_checkpoint

        draft, _, _ = load_model_from_checkpoint(args.draft_checkpoint, policy.device)
        spec_gen = SpeculativeGenerator(policy.model, draft, k=args.spec_k)

    def run(prompt: str, interactive: bool) -> None:
        text, stats = generate_text(policy.model, policy.tokenizer, prompt, settings, spec_generator=spec_gen)
        print(text)
        if interactive:
            print(f"[{stats['n_generated']} tokens, {stats['tokens_per_sec']:.1f} tok/s]")
        else:
            print(f"[{stats['n_generated']} tokens in {stats['elapsed_s']:.2f}s, {stats['tokens_per_sec']:.1f} tok/s]",
                  file=sys.stderr)

    if not args.interactive:
        run(args.prompt, False)
        return 0
    print("Interactive mode - type a prompt (empty line or 'quit' to exit).")
    while True:
        try:
            line = input("> ")
        except (EOFError, KeyboardInterrupt):
            break
        if not line or line.lower() in ("quit", "exit"):
            break
        run(line, True)
    return 0


def cmd_evaluate(args: argparse.Namespace) -> int:
    from rl_project_b200.evaluation.results import save_results
    from rl_project_b200.evaluation.suites import BenchmarkSuite, build_benchmark

    results = []
    policy = None
    if args.ray_workers:
        from rl_project_b200.orchestration.config import RayConfig
        from rl_project_b200.orchestration.pools import EvaluatorPool

        cfg = RayConfig(address=args.ray_address, cpus_per_worker=args.ray_cpus_per_worker,
                        backend=args.worker_backend)
        with EvaluatorPool(args.checkpoint, args.ray_workers, cfg, data_dir=args.data_dir) as evaluator:
            for name in args.suites:
                results.append(evaluator.run(name, max_new_tokens=args.max_tokens, n_shot=args.n_shot,
                                             max_tasks=args.max_tasks, offline=args.offline))
    else:
        policy = _load_policy(args)
        for name in args.suites:
            bench = build_benchmark(name, n_shot=args.n_shot, max_tasks=args.max_tasks, offline=args.offline)
            results.append(BenchmarkSuite(bench, max_new_tokens=args.max_tokens).run(policy))
    if args.heldout_data:
        from rl_project_b200.data.pretraining import MemmapCorpus
        from rl_project_b200.evaluation.quality import HeldOutLossSuite

        policy = policy or _load_policy(args)
        corpus = MemmapCorpus(args.heldout_data, "val", policy.spec.block_size)
        results.append(HeldOutLossSuite(corpus).run(policy.model))
    if args.output:
        save_results(results, args.output)
    _print([{"suite": r.suite, "metrics": r.metrics, "n": r.n_samples,
             "offline_samples": r.details.get("offline_samples")} for r in results])
    return 0


def cmd_export(args: argparse.Namespace) -> int:
    from rl_project_b200.models.loading import load_model_from_checkpoint
    from rl_project_b200.models.quantization.gguf import export_gguf

    model, spec, _ = load_model_from_checkpoint(args.checkpoint, "cpu")
    if args.merge_adapters:
        from rl_project_b200.models.adapters.lora import merge_lora

        merge_lora(model)
    _print(export_gguf(model.state_dict(), spec, args.output, quantize=args.quantize))
    return 0


def cmd_serve(args: argparse.Namespace) -> int:
    from rl_project_b200.inference.engine import InferenceEngine
    from rl_project_b200.observability.metrics import build_metrics_sink
    from rl_project_b200.serving import EngineBackend, Router, ServingServer

    policy = _load_policy(args)
    engine = InferenceEngine(policy.model, max_batch=args.max_batch, max_seq_len=args.max_seq_len)
    backend = EngineBackend(args.model_name, engine, policy.tokenizer)
    route_fn = None
    if args.routing:
        from rl_project_b200.deployment.rollout import RoutingPolicy

        route_fn = RoutingPolicy.load(args.routing).as_route_fn()
    router = Router({args.model_name: backend}, args.model_name, route_fn=route_fn,
                    metrics=build_metrics_sink(args.metrics, output_dir=args.output_dir, run_name="serve"))
    server = ServingServer(router, host=args.host, port=args.port)
    print(f"serving {args.model_name} on http://{args.host}:{server.port} "
          "(endpoints: /health /v1/models /v1/completions /v1/chat/completions /metrics)")
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        backend.close()
        server.stop()
    return 0


# ------------------------------------------------------------------ registry
def _registry_list(reg, args):
    return 0, [{"id": c.id, "key": c.key, "state": c.state.value, "algorithm": c.algorithm, "metrics": c.metrics,
                "promotion": c.promotion_status} for c in reg.list()]


def _registry_register(reg, args):
    from rl_project_b200.deployment import ModelCandidate

    metrics = json.loads(args.metrics) if args.metrics else {}
    if args.metrics_file:
        from rl_project_b200.evaluation.results import load_results, merge_metrics

        metrics.update(merge_metrics(load_results(args.metrics_file)))
    c = reg.register(ModelCandidate(name=args.name, version=args.version, algorithm=args.algorithm,
                                    checkpoint=args.checkpoint, metrics=metrics, tags=args.tags or []))
    return 0, {"registered": c.id, "key": c.key}


def _registry_promote(reg, args):
    """Move a candidate to ``--to``; a champion promotion with ``--gate`` must pass the gate against the incumbent
    (exit 2 when it does not), and a candidate below challenger is staged through challenger first."""
    from rl_project_b200.deployment import CandidateState, PromotionGate

    c = reg.get(args.id)
    target = CandidateState(args.to)
    champion = target == CandidateState.CHAMPION
    if champion and args.gate:
        from rl_project_b200.core.config import load_config

        incumbent = reg.champion(c.name)
        report = PromotionGate.from_config(load_config(args.gate)).evaluate(
            c.metrics, incumbent.metrics if incumbent else None)
        c.promotion_status, c.promotion_report = ("passed" if report.passed else "rejected"), report.to_dict()
        reg.update(c)
        if not report.passed:
            return 2, {"promoted": False, "report": report.to_dict()}
    if champion and c.state not in (CandidateState.CHALLENGER, CandidateState.CHAMPION):
        reg.transition(c.id, CandidateState.CHALLENGER, reason="staged before champion promotion")
    reg.transition(c.id, target, reason=args.reason)
    return 0, {"promoted": True, "id": c.id, "state": target.value}


def _registry_rollback(reg, args):
    from rl_project_b200.deployment import rollback

    return 0, {"champion": rollback(reg, args.name, reason=args.reason).key}


def _registry_disable(reg, args):
    from rl_project_b200.deployment import disable_candidate

    return 0, {"disabled": disable_candidate(reg, args.id, reason=args.reason).key}


_REGISTRY = {"list": _registry_list, "register": _registry_register, "promote": _registry_promote,
             "rollback": _registry_rollback, "disable": _registry_disable}


def cmd_registry(args: argparse.Namespace) -> int:
    from rl_project_b200.deployment import CandidateRegistry

    code, out = _REGISTRY[args.registry_cmd](CandidateRegistry(args.registry), args)
    _print(out)
    return code


# ------------------------------------------------------------------ rlaif / synthesis / dashboard / allocation
def cmd_rlaif(args: argparse.Namespace) -> int:
    from rl_project_b200.training import rlaif as R

    if args.rlaif_cmd == "pairwise":
        prompts = (R.SAMPLE_PROMPTS * 10)[: args.n_prompts]
        if args.checkpoint:
            policy = _load_policy(args)
            gen, judge = R.make_policy_generator(policy), R.make_policy_pairwise_judge(policy)
        else:
            gen, judge = R.rule_generator, R.rule_judge
        stats = R.run_pairwise_rlaif(prompts, gen, judge, n_candidates=args.candidates)
        _print(R.save_pairwise_output(stats, args.output))
        return 0
    prompts = (R.CONSTITUTIONAL_SAMPLE_PROMPTS * 10)[: args.n_prompts]
    model_fn = R.rule_based_constitutional_model
    if args.checkpoint:
        import torch

        from rl_project_b200.core.protocols import GenerationSettings

        policy = _load_policy(args)

        def model_fn(prompt: str) -> str:  # noqa: F811
            ids = torch.tensor(policy.encode(prompt)[-policy.spec.block_size // 2:], dtype=torch.long)
            out = policy.generate(ids.unsqueeze(0).to(policy.device),
                                  GenerationSettings(max_new_tokens=args.max_tokens, temperature=0.7))
            return policy.decode(out[0])

    examples = R.run_constitutional(prompts, model_fn, R.ConstitutionalConfig(n_principles_per_example=args.n_principles))
    _print(R.save_constitutional_output(examples, args.output))
    return 0


def cmd_synthesis(args: argparse.Namespace) -> int:
    from rl_project_b200.domains.synthesis import (TabularActorCritic, TabularPPOConfig, TabularPPOTrainer,
                                                   load_trajectories, rule_score)
    from rl_project_b200.evaluation.reward import RecordRewardSuite

    rows = load_trajectories(args.data)
    split = int(len(rows) * 0.8)
    trainer = TabularPPOTrainer(TabularActorCritic(), TabularPPOConfig(epochs=args.epochs, batch_size=args.batch_size,
                                                                      learning_rate=args.lr))
    metrics = trainer.train(rows[:split])
    held = RecordRewardSuite(rows[split:], rule_score).run()
    if args.output:
        Path(args.output).parent.mkdir(parents=True, exist_ok=True)
        Path(args.output).write_text(json.dumps({"training": dict(metrics), "heldout_record_reward": held.to_dict()},
                                                indent=2))
    _print({"final_train_reward": metrics["final_reward"], "heldout_record_reward_mean": held.metrics["mean"],
            "note": "heldout_record_reward scores dataset records (policy-independent)"})
    return 0


def cmd_dashboard(args: argparse.Namespace) -> int:
    from rl_project_b200.dashboard.data import DashboardSources, snapshot

    sources = DashboardSources(runs=list(args.runs), registry=args.registry, benchmarks=args.benchmarks)
    if args.export:
        path = Path(args.export)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(snapshot(sources), indent=1, default=str))
        print(f"wrote dashboard snapshot to {path}")
        return 0
    from rl_project_b200.dashboard.server import DashboardApp, DashboardServer

    server = DashboardServer(DashboardApp(sources), host=args.host, port=args.port)
    print(f"dashboard on {server.url} (runs: {', '.join(sources.runs)}; registry: {sources.registry}; "
          f"benchmarks: {sources.benchmarks})")
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        server.stop()
    return 0


def _alloc_policy(spec: str, env_cfg):
    """``dual`` / ``threshold`` build the baselines; anything else is a trained policy checkpoint."""
    from rl_project_b200.domains.allocation.policies import DualPacingPolicy, ThresholdPacingPolicy
    from rl_project_b200.domains.allocation.ppo import load_allocation_policy

    if spec == "dual":
        return DualPacingPolicy(env_cfg)
    if spec == "threshold":
        return ThresholdPacingPolicy(env_cfg, threshold=0.6)
    return load_allocation_policy(spec.split(":", 1)[-1])


def cmd_allocation(args: argparse.Namespace) -> int:
    from rl_project_b200.core.config import load_config
    from rl_project_b200.domains.allocation.env import AllocationEnvConfig
    from rl_project_b200.observability.events import Event
    from rl_project_b200.observability.metrics import build_metrics_sink

    if args.allocation_cmd == "benchmark":
        from rl_project_b200.domains.allocation.benchmark import BenchmarkConfig, run_benchmark

        cfg = BenchmarkConfig.from_dict(dict(load_config(args.config)))
        if args.output_dir:
            cfg.output_dir = args.output_dir
        run_benchmark(cfg)
        print(Path(cfg.output_dir, "summary.md").read_text())
        print(f"results: {Path(cfg.output_dir, 'results.json')}")
        return 0
    env_cfg = AllocationEnvConfig.from_dict(dict(load_config(args.env)) if args.env else {})
    sink = build_metrics_sink(args.metrics, output_dir=args.output_dir, run_name=f"allocation-{args.allocation_cmd}")
    if args.allocation_cmd == "ope":
        from rl_project_b200.domains.allocation.ope import OPEConfig, evaluate_target_policy
        from rl_project_b200.domains.allocation.rollout import read_episodes

        report = evaluate_target_policy(_alloc_policy(args.target, env_cfg), read_episodes(args.log), env_cfg,
                                        OPEConfig(max_weight=args.max_weight, n_bootstrap=args.bootstrap),
                                        target_name=args.target)
        d = report.to_dict()
        sink.event(Event.OPE_EVALUATED.value, {"target": args.target, "ess": d["diagnostics"]["ess"],
                                               **{k: v["value"] for k, v in d["estimates"].items()}})
        _print(d)
        return 3 if d["diagnostics"]["warnings"] else 0
    if args.allocation_cmd == "ab":
        from rl_project_b200.domains.allocation.experiment import ABConfig, run_ab_experiment

        res = run_ab_experiment(_alloc_policy(args.incumbent, env_cfg), _alloc_policy(args.challenger, env_cfg),
                                env_cfg, ABConfig(n_episodes=args.episodes, seed=args.seed,
                                                  challenger_percent=args.challenger_percent),
                                incumbent_name=args.incumbent, challenger_name=args.challenger)
        sink.event(Event.EXPERIMENT_AB.value, {"promote": res.promote, "p_value": res.p_value, **res.gate_metrics()})
        _print(res.to_dict())
        if args.gate_metrics:
            Path(args.gate_metrics).write_text(json.dumps(res.gate_metrics(), indent=2))
        return 0 if res.promote else 2
    if args.allocation_cmd == "shadow":
        from rl_project_b200.domains.allocation.experiment import shadow_evaluate
        from rl_project_b200.domains.allocation.rollout import seeds_for

        res = shadow_evaluate(_alloc_policy(args.incumbent, env_cfg), _alloc_policy(args.candidate, env_cfg), env_cfg,
                              seeds_for(args.seed, args.episodes))
        sink.event(Event.EXPERIMENT_SHADOW.value, {"divergence_rate": res.divergence_rate,
                                                   "candidate_replay_value": res.candidate_replay_value})
        _print(res.to_dict())
        return 0
    raise ForgelineError(f"unknown allocation command {args.allocation_cmd}")


# ------------------------------------------------------------------ parser
# The command line is data: every command is (help, handler, arguments), arguments are (flags, options), and a
# command with sub-commands carries {"dest": ..., name: (help, arguments)}.  ``build_parser`` walks the table.


def A(*flags: str, **options: Any):
    return flags, options


_POLICY_SOURCE = [A("--checkpoint", required=True),
                  A("--data-dir", default=None, help="directory with meta.pkl when the checkpoint lacks it"),
                  A("--device", default="auto")]

_GENERATE = _POLICY_SOURCE + [
    A("--prompt", default="\n"), A("--max-tokens", type=int, default=200), A("--temperature", type=float, default=0.8),
    A("--top-k", type=int, default=50), A("--top-p", type=float, default=None), A("--min-p", type=float, default=None),
    A("--repetition-penalty", type=float, default=1.0), A("--no-cache", action="store_true"),
    A("--interactive", action="store_true"), A("--draft-checkpoint", default=None), A("--spec-k", type=int, default=5)]

_EVALUATE = _POLICY_SOURCE + [
    A("--suites", nargs="+", default=["gsm8k"]), A("--n-shot", type=int, default=0),
    A("--max-tasks", type=int, default=0), A("--max-tokens", type=int, default=64),
    A("--offline", action="store_true", help="use built-in sample tasks (no download)"),
    A("--heldout-data", default=None), A("--output", default=None), A("--ray-workers", type=int, default=0),
    A("--ray-address", default=None), A("--ray-cpus-per-worker", type=float, default=1.0),
    A("--worker-backend", default="ray", choices=["ray", "threads"],
      help="where --ray-workers run: Ray actors or in-process threads")]

_SERVE = _POLICY_SOURCE + [
    A("--host", default="127.0.0.1"), A("--port", type=int, default=8000), A("--model-name", default="forgeline-model"),
    A("--max-batch", type=int, default=8), A("--max-seq-len", type=int, default=None),
    A("--routing", default=None, help="routing policy JSON"), A("--metrics", default="none"),
    A("--output-dir", default="runs/serve")]

_RLAIF_COMMON = [A("--output", required=True), A("--n-prompts", type=int, default=10), A("--checkpoint", default=None),
                 A("--data-dir", default=None), A("--device", default="auto"), A("--max-tokens", type=int, default=128)]

_ALLOC_COMMON = [A("--env", default=None), A("--metrics", default="none"), A("--output-dir", default="runs/allocation")]


def _command_table() -> Dict[str, Tuple[str, Any, Any]]:
    return {
        "presets": ("list model presets", cmd_presets,
                    [A("--count-params", action="store_true"), A("--vocab-size", type=int, default=65536)]),
        "validate": ("validate an experiment manifest without running it", cmd_validate,
                     [A("manifest"), A("--world-size", type=int, default=None)]),
        "data": ("dataset preparation and validation", cmd_data, {
            "dest": "data_cmd",
            "prepare": ("tokenize a text file into train.bin/val.bin", [
                A("--input", required=True), A("--output", required=True),
                A("--tokenizer", default="char", help="char | tiktoken[:enc] | hf:<name>"),
                A("--val-fraction", type=float, default=0.1)]),
            "prepare-hf": ("stream a HuggingFace dataset into shard files", [
                A("--dataset", required=True), A("--subset", default=None), A("--tokenizer", default="Qwen/Qwen2.5-0.5B"),
                A("--output", required=True), A("--max-tokens", type=int, default=100_000_000),
                A("--shard-size", type=int, default=10_000_000)]),
            "shard": ("split a .bin token file into shards", [
                A("--input", required=True), A("--output", required=True), A("--n-shards", type=int, default=16)]),
            "gsm8k": ("download GSM8K as verifiable tool-use tasks", [
                A("--output", required=True), A("--split", default="train"), A("--limit", type=int, default=None)]),
            "validate": ("validate a JSONL dataset against a schema", [
                A("--input", required=True),
                A("--kind", required=True, choices=["supervised", "preference", "verifiable", "process", "reward"])]),
        }),
        "train": ("run a training stage from a manifest", cmd_train, [
            A("manifest"), A("--set", action="append", help="dotted override, e.g. trainer.max_steps=10"),
            A("--max-steps", type=int, default=None), A("--output-dir", default=None), A("--resume", default=None),
            A("--metrics", default="local", help="local | none | wandb | tensorboard")]),
        "generate": ("", cmd_generate, _GENERATE),
        "evaluate": ("", cmd_evaluate, _EVALUATE),
        "serve": ("", cmd_serve, _SERVE),
        "export": ("export a checkpoint to GGUF", cmd_export, [
            A("--checkpoint", required=True), A("--output", required=True),
            A("--quantize", default="none", choices=["none", "q8_0", "q4_0"]), A("--merge-adapters", action="store_true")]),
        "registry": ("model candidate registry", cmd_registry, {
            "dest": "registry_cmd", "parent": [A("--registry", default="registry/candidates.json")],
            "list": ("", []),
            "register": ("", [A("--name", required=True), A("--version", required=True), A("--algorithm", required=True),
                              A("--checkpoint", required=True), A("--metrics", default=None, help="JSON object"),
                              A("--metrics-file", default=None, help="evaluation results JSON"), A("--tags", nargs="*")]),
            "promote": ("", [A("--id", required=True),
                             A("--to", required=True, choices=["shadow", "challenger", "champion", "retired"]),
                             A("--gate", default=None, help="promotion gate YAML"), A("--reason", default="")]),
            "rollback": ("", [A("--name", required=True), A("--reason", default="manual rollback")]),
            "disable": ("", [A("--id", required=True), A("--reason", default="disabled")]),
        }),
        "rlaif": ("AI-feedback data generation", cmd_rlaif, {
            "dest": "rlaif_cmd",
            "pairwise": ("", _RLAIF_COMMON + [A("--candidates", type=int, default=4)]),
            "constitutional": ("", _RLAIF_COMMON + [A("--n-principles", type=int, default=2)]),
        }),
        "dashboard": ("local read-only dashboard", cmd_dashboard, [
            A("--runs", nargs="+", default=["runs"]), A("--registry", default="registry/candidates.json"),
            A("--benchmarks", default="benchmarks"), A("--host", default="127.0.0.1"), A("--port", type=int, default=8765),
            A("--export", default=None, help="write a JSON snapshot instead of serving")]),
        "allocation": ("budgeted sequential-allocation benchmark, OPE, A/B, shadow", cmd_allocation, {
            "dest": "allocation_cmd",
            "benchmark": ("", [A("--config", required=True), A("--output-dir", default=None)]),
            "ope": ("", _ALLOC_COMMON + [A("--log", required=True), A("--target", required=True),
                                        A("--max-weight", type=float, default=20.0), A("--bootstrap", type=int, default=500)]),
            "ab": ("", _ALLOC_COMMON + [A("--incumbent", required=True), A("--challenger", required=True),
                                       A("--episodes", type=int, default=400), A("--seed", type=int, default=0),
                                       A("--challenger-percent", type=float, default=50.0),
                                       A("--gate-metrics", default=None)]),
            "shadow": ("", _ALLOC_COMMON + [A("--incumbent", required=True), A("--candidate", required=True),
                                           A("--episodes", type=int, default=100), A("--seed", type=int, default=0)]),
        }),
        "synthesis-ppo": ("tabular actor-critic PPO on synthesis trajectories", cmd_synthesis, [
            A("--data", required=True), A("--epochs", type=int, default=5), A("--batch-size", type=int, default=8),
            A("--lr", type=float, default=1e-4), A("--output", default=None)]),
    }


def _add_arguments(parser: argparse.ArgumentParser, args) -> None:
    for flags, options in args:
        parser.add_argument(*flags, **options)


def build_parser() -> argparse.ArgumentParser:
    root = argparse.ArgumentParser(prog="forgeline-b200", description="Post-training, distributed training, "
                                   "evaluation, inference and model life cycle for language models on B200.")
    root.add_argument("--version", action="version", version=f"forgeline-b200 {__version__}")
    commands = root.add_subparsers(dest="command", required=True)
    for name, (help_text, handler, body) in _command_table().items():
        cmd = commands.add_parser(name, help=help_text)
        cmd.set_defaults(func=handler)
        if isinstance(body, dict):
            _add_arguments(cmd, body.get("parent", []))
            subs = cmd.add_subparsers(dest=body["dest"], required=True)
            for sub_name, entry in body.items():
                if sub_name in ("dest", "parent"):
                    continue
                sub_help, sub_args = entry
                _add_arguments(subs.add_parser(sub_name, help=sub_help or None), sub_args)
        else:
            _add_arguments(cmd, body)
    return root


def main(argv: Optional[List[str]] = None) -> int:
    args = build_parser().parse_args(argv)
    try:
        return int(args.func(args) or 0)
    except ForgelineError as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 1


if __name__ == "__main__":
    sys.exit(main())
