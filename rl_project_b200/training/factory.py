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

from dataclasses import dataclass

import dataclasses
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

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


@dataclass
class _Job:
    """What every algorithm builder reads: the manifest, the run context, the algorithm parameters (the
    ``rollout`` block taken out and parsed) and the data section's extra keys."""

    manifest: ExperimentManifest
    ctx: RunContext
    params: Dict[str, Any]
    rollout: Optional[RolloutConfig]
    extra: Dict[str, Any]


def _build_pretrain(j: _Job) -> PostTrainingAlgorithm:
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    m, ctx = j.manifest, j.ctx
    cfg = _kw({"batch_size": m.trainer.batch_size, "eval_batches": m.trainer.eval_batches, **j.params}, PretrainConfig)
    if _synthetic(m):
        from rl_project_b200.data.synthetic import SyntheticPretrainSource

        model = build_model(m, ctx)
        src = SyntheticPretrainSource(m.model.vocab_size, m.model.block_size, cfg.batch_size, seed=m.data.seed,
                                      rank=_rank())
        return PretrainAlgorithm(model, src, cfg, None, device=ctx.device)
    root = Path(m.data.path)
    tok_meta = load_tokenizer_metadata(m.data.path) if (root / "meta.pkl").exists() else None
    if tok_meta:
        m.model.vocab_size = int(tok_meta["vocab_size"])
    model = build_model(m, ctx)
    train = MemmapCorpus(m.data.path, "train", m.model.block_size)
    val = MemmapCorpus(m.data.path, "val", m.model.block_size) if (root / "val.bin").exists() else None
    return PretrainAlgorithm(model, train, cfg, val, device=ctx.device, tokenizer_meta=tok_meta)


def _build_distill(j: _Job) -> PostTrainingAlgorithm:
    from rl_project_b200.training.distill import DistillationAlgorithm, DistillConfig

    m, p = j.manifest, j.params
    tpath = p.pop("teacher_checkpoint", None)
    if not tpath:
        raise ConfigError("distill needs algorithm_params.teacher_checkpoint")
    teacher, _, _ = load_model_from_checkpoint(tpath, j.ctx.device)
    m.model.vocab_size = teacher.spec.vocab_size
    student = build_model(m, j.ctx)
    corpus = MemmapCorpus(m.data.path, "train", m.model.block_size)
    return DistillationAlgorithm(student, teacher, corpus, _kw({"batch_size": m.trainer.batch_size, **p}, DistillConfig),
                                 device=j.ctx.device)


def _sft_records(j: _Job):
    """(train, val) SFT records of the data section: the addition tasks, synthesis trajectories or JSONL."""
    m, extra = j.manifest, j.extra
    if str(m.data.path) == "synthetic:addition":
        from rl_project_b200.data.synthetic import addition_tasks

        recs = [SFTRecord(t["prompt"], t["response"]) for t in
                addition_tasks(int(extra.get("n_tasks", 512)), seed=m.data.seed)]
        return deterministic_split(recs, m.data.val_fraction, m.data.seed)
    if m.data.kind == "trajectories":
        from rl_project_b200.domains.synthesis import build_sft_records, filter_high_reward
        from rl_project_b200.domains.synthesis.tabular_ppo import load_trajectories

        rows = filter_high_reward(load_trajectories(m.data.path), float(extra.get("reward_threshold", 0.8)))
        return build_sft_records(rows), []
    recs = read_jsonl(m.data.path, SFTRecord, on_error=extra.get("on_error", "raise"))
    return deterministic_split(recs, m.data.val_fraction, m.data.seed)


def _build_sft(j: _Job) -> PostTrainingAlgorithm:
    from rl_project_b200.training.sft import SFTAlgorithm, SFTConfig

    m = j.manifest
    policy = build_policy(m, j.ctx)
    cfg = _kw({"batch_size": m.trainer.batch_size, "max_length": m.data.max_length, **j.params}, SFTConfig)
    if str(m.data.path) == "synthetic":
        from rl_project_b200.data.synthetic import SyntheticSFTSource

        src = SyntheticSFTSource(m.model.vocab_size, m.model.block_size, cfg.batch_size,
                                 prompt_fraction=float(j.extra.get("prompt_fraction", 0.25)), seed=m.data.seed,
                                 rank=_rank())
        return SFTAlgorithm(policy, src, cfg)
    train, val = _sft_records(j)
    ds = lambda recs: SupervisedDataset(recs, policy.tokenizer, cfg.max_length)  # noqa: E731
    return SFTAlgorithm(policy, ds(train), cfg, ds(val) if val else None)


def _preference_records(j: _Job):
    m, extra = j.manifest, j.extra
    if m.data.kind == "trajectories":
        from rl_project_b200.domains.synthesis import build_preference_pairs
        from rl_project_b200.domains.synthesis.preferences import pairs_to_records

        rows, _ = _trajectory_split(m)
        return pairs_to_records(build_preference_pairs(rows, int(extra.get("pairs_per_molecule", 20)),
                                                       seed=m.data.seed)), []
    recs = read_jsonl(m.data.path, PreferenceRecord, on_error=extra.get("on_error", "raise"))
    return deterministic_split(recs, m.data.val_fraction, m.data.seed)


def _build_preference(j: _Job) -> PostTrainingAlgorithm:
    """DPO (a policy) or reward-model training (a sequence reward model) on preference pairs."""
    m, p = j.manifest, j.params
    train, val = _preference_records(j)
    mp = j.extra.get("max_prompt_length", 384)
    mr = j.extra.get("max_response_length", m.data.max_length)
    if m.algorithm == "dpo":
        from rl_project_b200.training.dpo import DPOAlgorithm, DPOConfig

        policy = build_policy(m, j.ctx)
        ds = lambda recs: PreferenceDataset(recs, policy.tokenizer, mp, mr)  # noqa: E731
        return DPOAlgorithm(policy, ds(train), _kw({"batch_size": m.trainer.batch_size, **p}, DPOConfig),
                            ds(val) if val else None)
    from rl_project_b200.training.reward_model import RewardModelAlgorithm, RewardModelConfig

    tok = build_tokenizer(m)
    m.model.vocab_size = tok.vocab_size
    rm = SequenceRewardModel(m.model, pooling=p.pop("pooling", "last")).to(j.ctx.device)
    if m.checkpoint_path:
        rm.backbone = load_model_from_checkpoint(m.checkpoint_path, j.ctx.device)[0]
    ds = lambda recs: PreferenceDataset(recs, tok, mp, mr)  # noqa: E731
    return RewardModelAlgorithm(rm, ds(train), _kw({"batch_size": m.trainer.batch_size, **p}, RewardModelConfig),
                                ds(val) if val else None, tokenizer_meta=tok.metadata())


def _rl_prompts(j: _Job, policy) -> Tuple[List[torch.Tensor], Optional[List[Dict[str, Any]]]]:
    """Prompt token tensors (and their task dicts, when the data has answers) for the online algorithms."""
    m, extra = j.manifest, j.extra
    tasks: Optional[List[Dict[str, Any]]] = None
    random_prompts_source = str(m.data.path) == "synthetic:random_prompts"
    if m.data.kind == "trajectories":
        from rl_project_b200.domains.synthesis import build_synthesis_prompt

        rows, _ = _trajectory_split(m)
        tasks = [dict(t, prompt=build_synthesis_prompt(t)) for t in rows]
    elif m.data.kind == "verifiable" and not random_prompts_source:
        tasks = [t.to_dict() for t in _tasks(m)]
    if random_prompts_source:
        from rl_project_b200.data.synthetic import random_prompts

        # rollout replicas share one prompt pool (every rank draws the same prompts); otherwise per rank
        shared = j.rollout is not None and j.rollout.replica_tp > 0
        prompts = random_prompts(int(extra.get("n_prompts", 1024)), m.model.vocab_size, int(extra.get("min_prompt", 128)),
                                 int(extra.get("max_prompt", 512)), seed=m.data.seed + (0 if shared else _rank()))
    elif tasks:
        prompts = [torch.tensor(policy.encode(t["prompt"]), dtype=torch.long) for t in tasks]
    else:
        src = m.data.path if Path(m.data.path).is_file() else None
        prompts = [torch.tensor(ids, dtype=torch.long) for ids in load_prompts(src, policy.tokenizer, m.data.max_length)]
    return prompts, tasks


def _build_online(j: _Job) -> PostTrainingAlgorithm:
    """PPO, GRPO (single-turn or agent) and DAPO."""
    m, p, alg = j.manifest, j.params, j.manifest.algorithm
    reward_cfg = m.reward or {"type": "rule", "name": "length", "target_length": 32}
    reward = build_reward_provider(reward_cfg)
    policy = build_policy(m, j.ctx, value_head=(alg == "ppo"))
    prompts, tasks = _rl_prompts(j, policy)
    if alg == "ppo":
        from rl_project_b200.training.ppo import PPOAlgorithm, PPOConfig

        built = PPOAlgorithm(policy, prompts, reward, _kw(p, PPOConfig), j.rollout, tasks=tasks)
    elif alg == "grpo":
        from rl_project_b200.training.grpo import GRPOAlgorithm, GRPOConfig

        cfg = _kw(p, GRPOConfig)
        built = (GRPOAlgorithm(policy, tasks or [], reward, cfg) if cfg.agent
                 else GRPOAlgorithm(policy, prompts, reward, cfg, j.rollout, tasks=tasks))
    else:
        from rl_project_b200.training.dapo import DAPOAlgorithm, DAPOConfig

        built = DAPOAlgorithm(policy, prompts, reward, _kw(p, DAPOConfig), j.rollout, tasks=tasks)
    return _attach_orchestration(built, m, reward_cfg)


def _build_allocation(j: _Job) -> PostTrainingAlgorithm:
    from rl_project_b200.domains.allocation.ppo import build_allocation_ppo

    return build_allocation_ppo(j.params, j.ctx.device)


def _build_rlvr(j: _Job) -> PostTrainingAlgorithm:
    from rl_project_b200.training.dapo import DAPOConfig
    from rl_project_b200.training.grpo import GRPOConfig
    from rl_project_b200.training.rlvr import RLVRConfig, build_rlvr_algorithm

    p = j.params
    policy = build_policy(j.manifest, j.ctx)
    grpo = _kw(p.pop("grpo", {}) or {}, GRPOConfig)
    dapo = _kw(p.pop("dapo", {}) or {}, DAPOConfig)
    return build_rlvr_algorithm(policy, _tasks(j.manifest), _kw({**p, "grpo": grpo, "dapo": dapo}, RLVRConfig),
                                j.rollout)


_BUILDERS = {"pretrain": _build_pretrain, "distill": _build_distill, "sft": _build_sft, "dpo": _build_preference,
             "reward_model": _build_preference, "ppo": _build_online, "grpo": _build_online, "dapo": _build_online,
             "allocation_ppo": _build_allocation, "rlvr": _build_rlvr}


def build_algorithm(manifest: ExperimentManifest, ctx: RunContext) -> PostTrainingAlgorithm:
    build = _BUILDERS.get(manifest.algorithm)
    if build is None:
        raise ConfigError(f"algorithm {manifest.algorithm!r} is not run through the step trainer; use the dedicated "
                          "CLI command",
                          hint="rlaif/constitutional/star/hill_climb/tabular_ppo have their own commands.")
    params = dict(manifest.algorithm_params)
    rp = params.pop("rollout", {}) or {}
    return build(_Job(manifest, ctx, params, _kw(rp, RolloutConfig) if rp else None, manifest.data.extra))
