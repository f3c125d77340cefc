"""Manifest -> tokenizer / model / policy / datasets / reward -> algorithm
(``src/forgeline/training/factory.py`` contract, same ``algorithm_params`` keys).

Extension: ``data.path`` values starting with ``synthetic`` select the seeded
synthetic sources used by the benchmark configurations:

* ``synthetic`` (pretraining / supervised): uniform token ids; ``data.extra``
  ``prompt_fraction`` sets the SFT prompt mask;
* ``synthetic:addition`` (supervised / verifiable): ``a+b=`` tasks;
* ``synthetic:random_prompts`` (GRPO/PPO/DAPO): uniform-id prompts with
  lengths ``data.extra.min_prompt``..``max_prompt``.
"""

from __future__ import annotations

import dataclasses
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch

from rl_project_b200.core.config import ExperimentManifest
from rl_project_b200.core.errors import ConfigError
from rl_project_b200.core.lifecycle import RunContext
from rl_project_b200.data.preference import PreferenceDataset
from rl_project_b200.data.pretraining import MemmapCorpus
from rl_project_b200.data.records import PreferenceRecord, SFTRecord, VerifiableTask, deterministic_split, read_jsonl
from rl_project_b200.data.supervised import SupervisedDataset
from rl_project_b200.data.tokenizers import (ByteTokenizer, CharTokenizer, load_tokenizer_metadata, resolve_tokenizer,
                                             tokenizer_from_metadata)
from rl_project_b200.data.verifiable import VerifiableTaskDataset, load_prompts
from rl_project_b200.models.loading import load_model_from_checkpoint
from rl_project_b200.models.policy import NativePolicy
from rl_project_b200.models.reward import SequenceRewardModel
from rl_project_b200.models.transformer.model import TransformerLM
from rl_project_b200.rollouts.engine import RolloutConfig
from rl_project_b200.rollouts.rewards import build_reward_provider
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm


def _kw(params: Dict[str, Any], cls):
    names = {f.name for f in dataclasses.fields(cls)}
    bad = sorted(set(params) - names)
    if bad:
        raise ConfigError(f"unknown {cls.__name__} keys: {bad}")
    return cls(**params)


def _synthetic(manifest: ExperimentManifest) -> bool:
    return str(manifest.data.path).startswith("synthetic")


def _attach_orchestration(algorithm, manifest, reward_cfg):
    orch = manifest.orchestration or {}
    if orch.get("type", "local") != "ray":
        return algorithm
    from rl_project_b200.orchestration.pools import attach_to_algorithm

    attach_to_algorithm(algorithm, orch, reward_cfg, seed=manifest.trainer.seed)
    return algorithm


def build_tokenizer(manifest: ExperimentManifest):
    if manifest.checkpoint_path:
        from rl_project_b200.checkpoints.manager import CheckpointManager

        meta = CheckpointManager.read_manifest(manifest.checkpoint_path).get("tokenizer_meta")
        if meta:
            return tokenizer_from_metadata(meta)
    spec = manifest.data.tokenizer
    if _synthetic(manifest):
        return ByteTokenizer() if spec in ("auto", "byte") or manifest.model.vocab_size == 256 else resolve_tokenizer(spec)
    data_dir = Path(manifest.data.path)
    try:
        return resolve_tokenizer(spec, data_dir if data_dir.exists() else None)
    except Exception:
        if spec in ("auto", "char"):
            return CharTokenizer.ascii()
        raise


def build_model(manifest: ExperimentManifest, ctx: RunContext, tokenizer=None) -> TransformerLM:
    if manifest.checkpoint_path:
        model, spec, _ = load_model_from_checkpoint(manifest.checkpoint_path, ctx.device)
        manifest.model = spec
        return model
    if tokenizer is not None and not _synthetic(manifest) and manifest.model.vocab_size != tokenizer.vocab_size:
        manifest.model.vocab_size = tokenizer.vocab_size
    with torch.device(ctx.device):
        model = TransformerLM(manifest.model)
    if manifest.trainer.gradient_checkpointing:
        model.enable_gradient_checkpointing()
    return model


def build_policy(manifest: ExperimentManifest, ctx: RunContext, value_head: bool = False):
    backend = manifest.backend or {}
    if backend.get("type") == "huggingface":
        from rl_project_b200.models.hf_policy import HFPolicy

        opts = {k: v for k, v in backend.items() if k not in ("type", "model_name", "adapter_path")}
        dt = opts.pop("torch_dtype", None)
        if isinstance(dt, str):
            opts["torch_dtype"] = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[dt]
        opts.setdefault("device_map", None if ctx.device.type == "cpu" else {"": ctx.device.index or 0})
        policy = HFPolicy(backend["model_name"], value_head=value_head, **opts)
        if backend.get("adapter_path"):
            policy.model.load_adapter(backend["adapter_path"], adapter_name="default", is_trainable=True)
        if manifest.checkpoint_path:
            from rl_project_b200.checkpoints.manager import CheckpointManager

            policy.load_checkpoint_state(CheckpointManager.load(manifest.checkpoint_path).model_state)
        return policy.to(ctx.device) if opts.get("device_map") is None else policy
    tok = build_tokenizer(manifest)
    model = build_model(manifest, ctx, tok)
    adapter = manifest.trainer.adapter if manifest.trainer.adapter.method != "none" else None
    return NativePolicy(model, tok, adapter=adapter, value_head=value_head).to(ctx.device)


def _trajectory_split(manifest):
    from rl_project_b200.domains.synthesis.tabular_ppo import load_trajectories

    rows = load_trajectories(manifest.data.path)
    cut = int(len(rows) * float(manifest.data.extra.get("train_fraction", 0.8)))
    return rows[:cut], rows[cut:]


def _tasks(manifest: ExperimentManifest) -> List[VerifiableTask]:
    path = str(manifest.data.path)
    if path == "synthetic:addition":
        from rl_project_b200.data.synthetic import addition_tasks

        n = int(manifest.data.extra.get("n_tasks", 256))
        return [VerifiableTask(prompt=t["prompt"], answer=t["answer"], task_type="exact")
                for t in addition_tasks(n, seed=manifest.data.seed)]
    p = Path(path)
    if p.is_file():
        return VerifiableTaskDataset.from_jsonl(p, on_error=manifest.data.extra.get("on_error", "raise"),
                                               limit=manifest.data.extra.get("limit")).tasks
    return VerifiableTaskDataset.builtin_arithmetic().tasks


def _rank() -> int:
    """Data rank: the data-parallel rank under a TP / PP mesh (all ranks of a replica see the same data)."""
    from rl_project_b200.parallel.mesh_strategies import data_parallel_rank

    return data_parallel_rank()


def build_algorithm(manifest: ExperimentManifest, ctx: RunContext) -> PostTrainingAlgorithm:
    alg = manifest.algorithm
    p = dict(manifest.algorithm_params)
    rp = p.pop("rollout", {}) or {}
    rollout = _kw(rp, RolloutConfig) if rp else None
    extra = manifest.data.extra
    if alg == "pretrain":
        from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

        cfg = _kw({"batch_size": manifest.trainer.batch_size, "eval_batches": manifest.trainer.eval_batches, **p},
                  PretrainConfig)
        if _synthetic(manifest):
            from rl_project_b200.data.synthetic import SyntheticPretrainSource

            model = build_model(manifest, ctx)
            src = SyntheticPretrainSource(manifest.model.vocab_size, manifest.model.block_size, cfg.batch_size,
                                          seed=manifest.data.seed, rank=_rank())
            return PretrainAlgorithm(model, src, cfg, None, device=ctx.device)
        meta_file = Path(manifest.data.path) / "meta.pkl"
        tok_meta = load_tokenizer_metadata(manifest.data.path) if meta_file.exists() else None
        if tok_meta:
            manifest.model.vocab_size = int(tok_meta["vocab_size"])
        model = build_model(manifest, ctx)
        train = MemmapCorpus(manifest.data.path, "train", manifest.model.block_size)
        val = (MemmapCorpus(manifest.data.path, "val", manifest.model.block_size)
               if (Path(manifest.data.path) / "val.bin").exists() else None)
        return PretrainAlgorithm(model, train, cfg, val, device=ctx.device, tokenizer_meta=tok_meta)
    if alg == "distill":
        from rl_project_b200.training.distill import DistillationAlgorithm, DistillConfig

        tpath = p.pop("teacher_checkpoint", None)
        if not tpath:
            raise ConfigError("distill needs algorithm_params.teacher_checkpoint")
        teacher, _, _ = load_model_from_checkpoint(tpath, ctx.device)
        manifest.model.vocab_size = teacher.spec.vocab_size
        student = build_model(manifest, ctx)
        corpus = MemmapCorpus(manifest.data.path, "train", manifest.model.block_size)
        return DistillationAlgorithm(student, teacher, corpus, _kw({"batch_size": manifest.trainer.batch_size, **p},
                                                                   DistillConfig), device=ctx.device)
    if alg == "sft":
        from rl_project_b200.training.sft import SFTAlgorithm, SFTConfig

        policy = build_policy(manifest, ctx)
        cfg = _kw({"batch_size": manifest.trainer.batch_size, "max_length": manifest.data.max_length, **p}, SFTConfig)
        if str(manifest.data.path) == "synthetic":
            from rl_project_b200.data.synthetic import SyntheticSFTSource

            src = SyntheticSFTSource(manifest.model.vocab_size, manifest.model.block_size, cfg.batch_size,
                                     prompt_fraction=float(extra.get("prompt_fraction", 0.25)),
                                     seed=manifest.data.seed, rank=_rank())
            return SFTAlgorithm(policy, src, cfg)
        if str(manifest.data.path) == "synthetic:addition":
            from rl_project_b200.data.synthetic import addition_tasks

            recs = [SFTRecord(t["prompt"], t["response"]) for t in
                    addition_tasks(int(extra.get("n_tasks", 512)), seed=manifest.data.seed)]
            train, val = deterministic_split(recs, manifest.data.val_fraction, manifest.data.seed)
        elif manifest.data.kind == "trajectories":
            from rl_project_b200.domains.synthesis import build_sft_records, filter_high_reward
            from rl_project_b200.domains.synthesis.tabular_ppo import load_trajectories

            train = build_sft_records(filter_high_reward(load_trajectories(manifest.data.path),
                                                         float(extra.get("reward_threshold", 0.8))))
            val = []
        else:
            recs = read_jsonl(manifest.data.path, SFTRecord, on_error=extra.get("on_error", "raise"))
            train, val = deterministic_split(recs, manifest.data.val_fraction, manifest.data.seed)
        return SFTAlgorithm(policy, SupervisedDataset(train, policy.tokenizer, cfg.max_length), cfg,
                            SupervisedDataset(val, policy.tokenizer, cfg.max_length) if val else None)
    if alg in ("dpo", "reward_model"):
        if manifest.data.kind == "trajectories":
            from rl_project_b200.domains.synthesis import build_preference_pairs
            from rl_project_b200.domains.synthesis.preferences import pairs_to_records

            rows, _ = _trajectory_split(manifest)
            train = pairs_to_records(build_preference_pairs(rows, int(extra.get("pairs_per_molecule", 20)),
                                                            seed=manifest.data.seed))
            val = []
        else:
            recs = read_jsonl(manifest.data.path, PreferenceRecord, on_error=extra.get("on_error", "raise"))
            train, val = deterministic_split(recs, manifest.data.val_fraction, manifest.data.seed)
        mp = extra.get("max_prompt_length", 384)
        mr = extra.get("max_response_length", manifest.data.max_length)
        if alg == "dpo":
            from rl_project_b200.training.dpo import DPOAlgorithm, DPOConfig

            policy = build_policy(manifest, ctx)
            return DPOAlgorithm(policy, PreferenceDataset(train, policy.tokenizer, mp, mr),
                                _kw({"batch_size": manifest.trainer.batch_size, **p}, DPOConfig),
                                PreferenceDataset(val, policy.tokenizer, mp, mr) if val else None)
        from rl_project_b200.training.reward_model import RewardModelAlgorithm, RewardModelConfig

        tok = build_tokenizer(manifest)
        manifest.model.vocab_size = tok.vocab_size
        rm = SequenceRewardModel(manifest.model, pooling=p.pop("pooling", "last")).to(ctx.device)
        if manifest.checkpoint_path:
            rm.backbone = load_model_from_checkpoint(manifest.checkpoint_path, ctx.device)[0]
        return RewardModelAlgorithm(rm, PreferenceDataset(train, tok, mp, mr),
                                    _kw({"batch_size": manifest.trainer.batch_size, **p}, RewardModelConfig),
                                    PreferenceDataset(val, tok, mp, mr) if val else None, tokenizer_meta=tok.metadata())
    if alg in ("ppo", "grpo", "dapo"):
        reward_cfg = manifest.reward or {"type": "rule", "name": "length", "target_length": 32}
        reward = build_reward_provider(reward_cfg)
        policy = build_policy(manifest, ctx, value_head=(alg == "ppo"))
        tasks: Optional[List[Dict[str, Any]]] = None
        if manifest.data.kind == "trajectories":
            from rl_project_b200.domains.synthesis import build_synthesis_prompt

            rows, _ = _trajectory_split(manifest)
            tasks = [dict(t, prompt=build_synthesis_prompt(t)) for t in rows]
        elif manifest.data.kind == "verifiable" and str(manifest.data.path) != "synthetic:random_prompts":
            tasks = [t.to_dict() for t in _tasks(manifest)]
        if str(manifest.data.path) == "synthetic:random_prompts":
            from rl_project_b200.data.synthetic import random_prompts

            # rollout replicas share one prompt pool (every rank draws the same prompts); otherwise per rank
            shared = rollout is not None and rollout.replica_tp > 0
            prompts = random_prompts(int(extra.get("n_prompts", 1024)), manifest.model.vocab_size,
                                     int(extra.get("min_prompt", 128)), int(extra.get("max_prompt", 512)),
                                     seed=manifest.data.seed + (0 if shared else _rank()))
        elif tasks:
            prompts = [torch.tensor(policy.encode(t["prompt"]), dtype=torch.long) for t in tasks]
        else:
            src = manifest.data.path if Path(manifest.data.path).is_file() else None
            prompts = [torch.tensor(ids, dtype=torch.long)
                       for ids in load_prompts(src, policy.tokenizer, manifest.data.max_length)]
        if alg == "ppo":
            from rl_project_b200.training.ppo import PPOAlgorithm, PPOConfig

            built = PPOAlgorithm(policy, prompts, reward, _kw(p, PPOConfig), rollout, tasks=tasks)
        elif alg == "grpo":
            from rl_project_b200.training.grpo import GRPOAlgorithm, GRPOConfig

            cfg = _kw(p, GRPOConfig)
            built = (GRPOAlgorithm(policy, tasks or [], reward, cfg) if cfg.agent
                     else GRPOAlgorithm(policy, prompts, reward, cfg, rollout, tasks=tasks))
        else:
            from rl_project_b200.training.dapo import DAPOAlgorithm, DAPOConfig

            built = DAPOAlgorithm(policy, prompts, reward, _kw(p, DAPOConfig), rollout, tasks=tasks)
        return _attach_orchestration(built, manifest, reward_cfg)
    if alg == "allocation_ppo":
        from rl_project_b200.domains.allocation.ppo import build_allocation_ppo

        return build_allocation_ppo(p, ctx.device)
    if alg == "rlvr":
        from rl_project_b200.training.dapo import DAPOConfig
        from rl_project_b200.training.grpo import GRPOConfig
        from rl_project_b200.training.rlvr import RLVRConfig, build_rlvr_algorithm

        policy = build_policy(manifest, ctx)
        grpo = _kw(p.pop("grpo", {}) or {}, GRPOConfig)
        dapo = _kw(p.pop("dapo", {}) or {}, DAPOConfig)
        return build_rlvr_algorithm(policy, _tasks(manifest), _kw({**p, "grpo": grpo, "dapo": dapo}, RLVRConfig), rollout)
    raise ConfigError(f"algorithm {alg!r} is not run through the step trainer; use the dedicated CLI command",
                      hint="rlaif/constitutional/star/hill_climb/tabular_ppo have their own commands.")
