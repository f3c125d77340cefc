"""Model spec, trainer config and the experiment manifest.

Schema parity: field names, defaults and validation rules follow the
reference manifest (``src/forgeline/core/config.py:33-424``) so an existing
YAML/TOML/JSON manifest loads unchanged.  Additive fields (all defaulting to
the reference behaviour):

* ``ModelSpec.d_ff``        -- dense SwiGLU hidden width (0 = ``64*ceil(8d/3/64)``)
* ``ModelSpec.moe_d_ff``    -- routed/shared expert hidden width (0 = ``d_ff`` rule)
* ``ModelSpec.rope_theta``  -- RoPE base (reference hard-codes 10000)
* ``ModelSpec.tie_embeddings`` -- reference always ties ``wte``/``lm_head``
* ``DistributedConfig.expert_parallel_size``, ``context_parallel_size``,
  ``reshard_after_forward``, ``fused_comm`` and the extra strategy names
  ``zero2`` / ``expert_parallel`` / ``hybrid``.
"""

from __future__ import annotations

import dataclasses
import json
import os
import platform
import sys
from dataclasses import dataclass, field, fields
from pathlib import Path
from typing import Any, Dict, List, Mapping

from rl_project_b200.core.errors import ConfigError, UnknownPresetError


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise ConfigError(msg)


# -----------------------------------------------------------------------------
# model
# -----------------------------------------------------------------------------


@dataclass
class ModelSpec:
    """Hyper-parameters of the decoder-only transformer family."""

    block_size: int = 256
    vocab_size: int = 65536
    n_layer: int = 6
    n_head: int = 6
    n_kv_head: int = 6
    n_embd: int = 384
    dropout: float = 0.1
    bias: bool = False
    use_rope: bool = True
    use_swiglu: bool = True
    # local attention
    sliding_window: int = 0
    alternating_layers: bool = False
    attn_logit_cap: float = 0.0
    # RoPE context extension
    rope_scaling_type: str = "none"
    rope_scaling_factor: float = 1.0
    # multi-head latent attention
    use_mla: bool = False
    kv_lora_rank: int = 512
    q_lora_rank: int = 0
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    # mixture of experts
    use_moe: bool = False
    n_experts: int = 8
    n_experts_active: int = 2
    n_shared_experts: int = 0
    n_dense_layers: int = 0
    score_func: str = "softmax"
    route_scale: float = 1.0
    aux_loss_free: bool = False
    bias_update_speed: float = 0.001
    moe_aux_loss_weight: float = 0.01
    n_expert_groups: int = 1
    n_limited_groups: int = 1
    # multi-token prediction
    n_predict_tokens: int = 1
    mtp_loss_weight: float = 1.0
    # native sparse attention
    use_nsa: bool = False
    nsa_block_size: int = 32
    nsa_top_k: int = 16
    nsa_window_size: int = 256
    # additive fields (defaults reproduce the reference)
    d_ff: int = 0
    moe_d_ff: int = 0
    rope_theta: float = 10000.0
    tie_embeddings: bool = True

    def __post_init__(self) -> None:
        self.validate()

    def validate(self) -> None:
        _check(self.block_size >= 1 and self.vocab_size >= 1, "block_size and vocab_size must be positive")
        _check(self.n_embd % self.n_head == 0, f"n_embd ({self.n_embd}) must be divisible by n_head ({self.n_head})")
        if not self.use_mla:
            _check(self.n_kv_head >= 1 and self.n_head % self.n_kv_head == 0,
                   f"n_head ({self.n_head}) must be divisible by n_kv_head ({self.n_kv_head})")
        _check(self.rope_scaling_type in ("none", "linear", "yarn"),
               f"rope_scaling_type must be none|linear|yarn, got {self.rope_scaling_type!r}")
        _check(self.score_func in ("softmax", "sigmoid"), f"score_func must be softmax|sigmoid, got {self.score_func!r}")
        if self.use_moe:
            _check(self.n_experts_active <= self.n_experts, "n_experts_active cannot exceed n_experts")
            _check(self.n_experts % self.n_expert_groups == 0, "n_experts must be divisible by n_expert_groups")
        _check(not (self.use_mla and self.use_nsa), "use_mla and use_nsa are mutually exclusive")
        _check(self.n_predict_tokens >= 1, "n_predict_tokens must be >= 1")
        _check(self.d_ff >= 0 and self.moe_d_ff >= 0, "d_ff / moe_d_ff must be >= 0 (0 = derived)")
        _check(self.rope_theta > 0, "rope_theta must be positive")

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def ffn_hidden(self) -> int:
        """Dense FFN width: explicit ``d_ff`` or the reference's derived width."""
        if self.d_ff:
            return self.d_ff
        if not self.use_swiglu:
            return 4 * self.n_embd
        raw = int(8 * self.n_embd / 3)
        return 64 * ((raw + 63) // 64)

    @property
    def expert_hidden(self) -> int:
        return self.moe_d_ff or self.ffn_hidden

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ModelSpec":
        names = {f.name for f in fields(cls)}
        extra = sorted(set(data) - names)
        if extra:
            raise ConfigError(f"Unknown ModelSpec keys: {extra}")
        return cls(**dict(data))


# Preset table.  The first nine names and their values are the reference's
# (``src/forgeline/core/config.py:133-159``) so manifests that name them keep
# their meaning; the ``bl_*`` presets are the benchmark configurations.
MODEL_PRESETS: Dict[str, Dict[str, Any]] = {
    "tiny": {"n_layer": 2, "n_head": 2, "n_kv_head": 2, "n_embd": 64, "block_size": 64, "dropout": 0.0},
    "small": {"n_layer": 6, "n_head": 6, "n_kv_head": 6, "n_embd": 384, "block_size": 256, "dropout": 0.1},
    "medium": {"n_layer": 12, "n_head": 12, "n_kv_head": 4, "n_embd": 768, "block_size": 512, "dropout": 0.1},
    "large": {"n_layer": 24, "n_head": 16, "n_kv_head": 4, "n_embd": 1024, "block_size": 2048, "dropout": 0.1},
    "xl": {"n_layer": 24, "n_head": 16, "n_kv_head": 8, "n_embd": 2048, "block_size": 4096, "dropout": 0.1},
    "moe_32l": {"n_layer": 32, "n_head": 32, "n_kv_head": 8, "n_embd": 4096, "block_size": 8192, "dropout": 0.1,
                "use_moe": True, "n_experts": 8, "n_experts_active": 2},
    "latent_moe_27l": {"n_layer": 27, "n_head": 16, "n_kv_head": 16, "n_embd": 2048, "block_size": 4096,
                       "dropout": 0.0, "bias": False, "use_mla": True, "kv_lora_rank": 512, "q_lora_rank": 1536,
                       "qk_nope_head_dim": 128, "qk_rope_head_dim": 64, "v_head_dim": 128, "use_moe": True,
                       "n_experts": 64, "n_experts_active": 6, "n_shared_experts": 2, "n_dense_layers": 1,
                       "score_func": "sigmoid", "route_scale": 1.0, "aux_loss_free": True,
                       "bias_update_speed": 0.001, "n_predict_tokens": 3},
    "sliding_window_32l": {"n_layer": 32, "n_head": 32, "n_kv_head": 8, "n_embd": 4096, "block_size": 8192,
                           "dropout": 0.0, "bias": False, "sliding_window": 4096},
    "alternating_28l": {"n_layer": 28, "n_head": 16, "n_kv_head": 4, "n_embd": 2304, "block_size": 8192,
                        "dropout": 0.0, "bias": False, "sliding_window": 4096, "alternating_layers": True,
                        "attn_logit_cap": 50.0},
    # benchmark configurations
    "bl_tiny": {"n_layer": 2, "n_head": 4, "n_kv_head": 2, "n_embd": 64, "block_size": 128, "dropout": 0.0,
                "vocab_size": 256, "d_ff": 176, "rope_theta": 10000.0},
    "bl_dense_1b": {"n_layer": 16, "n_head": 32, "n_kv_head": 8, "n_embd": 2048, "block_size": 4096, "dropout": 0.0,
                    "vocab_size": 128256, "d_ff": 8192, "rope_theta": 500000.0},
    "bl_dense_8b": {"n_layer": 32, "n_head": 32, "n_kv_head": 8, "n_embd": 4096, "block_size": 8192, "dropout": 0.0,
                    "vocab_size": 128256, "d_ff": 14336, "rope_theta": 500000.0, "tie_embeddings": False},
    "bl_mla_moe": {"n_layer": 27, "n_head": 16, "n_kv_head": 16, "n_embd": 2048, "block_size": 4096, "dropout": 0.0,
                   "vocab_size": 102400, "use_mla": True, "kv_lora_rank": 512, "q_lora_rank": 0,
                   "qk_nope_head_dim": 128, "qk_rope_head_dim": 64, "v_head_dim": 128, "use_moe": True,
                   "n_experts": 64, "n_experts_active": 6, "n_shared_experts": 2, "n_dense_layers": 1,
                   "score_func": "sigmoid", "aux_loss_free": True, "n_expert_groups": 8, "n_limited_groups": 3,
                   "d_ff": 10944, "moe_d_ff": 1408, "n_predict_tokens": 2},
}


def model_spec_from_preset(preset: str, **overrides: Any) -> ModelSpec:
    if preset not in MODEL_PRESETS:
        raise UnknownPresetError(f"Unknown model preset {preset!r}. Available: {sorted(MODEL_PRESETS)}")
    values = {**MODEL_PRESETS[preset], **overrides}
    return ModelSpec.from_dict(values)


# -----------------------------------------------------------------------------
# trainer
# -----------------------------------------------------------------------------


@dataclass
class OptimizerConfig:
    name: str = "adamw"
    learning_rate: float = 3e-4
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    eps: float = 1e-8
    grad_clip: float = 1.0
    decay_only_matrices: bool = True
    fused: str = "auto"

    def validate(self) -> None:
        _check(self.name in ("adamw", "adam"), f"optimizer name must be adamw|adam, got {self.name!r}")
        _check(self.learning_rate > 0, "learning_rate must be positive")
        _check(self.grad_clip >= 0, "grad_clip must be >= 0 (0 disables clipping)")
        _check(self.fused in ("auto", "always", "never"), "optimizer.fused must be auto|always|never")


@dataclass
class ScheduleConfig:
    name: str = "cosine"
    warmup_steps: int = 100
    decay_steps: int = 5000
    min_lr: float = 3e-5
    wsd_stable_fraction: float = 0.8

    def validate(self) -> None:
        _check(self.name in ("cosine", "wsd", "constant", "linear_decay"),
               f"schedule name must be cosine|wsd|constant|linear_decay, got {self.name!r}")
        _check(self.warmup_steps >= 0 and self.decay_steps >= 0, "warmup_steps and decay_steps must be >= 0")
        _check(0.0 <= self.wsd_stable_fraction <= 1.0, "wsd_stable_fraction must be in [0, 1]")


@dataclass
class PrecisionConfig:
    dtype: str = "auto"
    grad_scaler: str = "auto"

    def validate(self) -> None:
        _check(self.dtype in ("auto", "float32", "bfloat16", "float16"),
               f"precision dtype must be auto|float32|bfloat16|float16, got {self.dtype!r}")
        _check(self.grad_scaler in ("auto", "on", "off"), "grad_scaler must be auto|on|off")


@dataclass
class CheckpointConfig:
    directory: str = "checkpoints"
    save_every: int = 1000
    keep_last: int = 3
    async_save: bool = False
    resume_from: str = ""
    auto_resume: bool = True

    def validate(self) -> None:
        _check(self.save_every >= 0, "save_every must be >= 0")
        _check(self.keep_last >= 1, "keep_last must be >= 1")


@dataclass
class AdapterConfig:
    method: str = "none"
    rank: int = 16
    alpha: float = 32.0
    dropout: float = 0.0
    target_modules: List[str] = field(default_factory=list)
    merge_on_save: bool = False

    def validate(self) -> None:
        _check(self.method in ("none", "lora", "qlora"), f"adapter method must be none|lora|qlora, got {self.method!r}")
        _check(self.rank >= 1, "adapter rank must be >= 1")


@dataclass
class TrainerConfig:
    max_steps: int = 1000
    batch_size: int = 16
    gradient_accumulation_steps: int = 1
    eval_every: int = 200
    eval_batches: int = 20
    log_every: int = 10
    seed: int = 1337
    device: str = "auto"
    compile_model: bool = False
    compile_backend: str = "inductor"
    gradient_checkpointing: bool = False
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    schedule: ScheduleConfig = field(default_factory=ScheduleConfig)
    precision: PrecisionConfig = field(default_factory=PrecisionConfig)
    checkpoint: CheckpointConfig = field(default_factory=CheckpointConfig)
    adapter: AdapterConfig = field(default_factory=AdapterConfig)

    def validate(self) -> None:
        _check(self.max_steps >= 0, "max_steps must be >= 0")
        _check(self.batch_size >= 1 and self.gradient_accumulation_steps >= 1,
               "batch_size and gradient_accumulation_steps must be >= 1")
        for sub in (self.optimizer, self.schedule, self.precision, self.checkpoint, self.adapter):
            sub.validate()


# -----------------------------------------------------------------------------
# manifest
# -----------------------------------------------------------------------------

STRATEGIES = ("single", "ddp", "fsdp", "deepspeed", "tensor_parallel", "pipeline_parallel",
              "zero2", "expert_parallel", "hybrid")


@dataclass
class DistributedConfig:
    strategy: str = "single"
    backend: str = "auto"
    tensor_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    pipeline_micro_batches: int = 4
    fsdp_min_params_to_wrap: int = 100_000
    deepspeed_config: str = ""
    # additive
    expert_parallel_size: int = 1
    context_parallel_size: int = 1
    reshard_after_forward: bool = True
    fused_comm: str = "auto"  # auto | on | off | nccl_baseline
    fused_multicast: str = "off"  # off (CUDA IPC, peer loads) | on (NVLink multicast reduce) | symm
    fused_rs_ctas: int = 32  # CTAs of a fused reduce-scatter that overlaps backward compute
    heartbeat_interval_s: float = 1.0  # rank liveness beats through the job's store (0 disables)
    heartbeat_timeout_s: float = 60.0  # a peer silent this long fails the next step's health check
    timeout_s: float = 600.0

    def validate(self) -> None:
        _check(self.strategy in STRATEGIES, f"distributed strategy must be one of {STRATEGIES}, got {self.strategy!r}")
        _check(min(self.tensor_parallel_size, self.pipeline_parallel_size, self.expert_parallel_size,
                   self.context_parallel_size) >= 1, "parallel sizes must be >= 1")
        # reserved for a context-parallel attention path; sequences up to block_size fit one GPU today
        _check(self.context_parallel_size == 1,
               "context_parallel_size > 1 is not supported: sequences are not split across GPUs (keep it at 1)")
        _check(self.backend in ("auto", "nccl", "gloo"), "backend must be auto|nccl|gloo")
        _check(not (self.strategy == "deepspeed" and not self.deepspeed_config),
               "deepspeed strategy requires deepspeed_config path")
        _check(self.fused_comm in ("auto", "on", "off", "nccl_baseline"),
               "fused_comm must be auto|on|off|nccl_baseline")
        _check(self.fused_multicast in ("off", "on", "symm"), "fused_multicast must be off|on|symm")
        _check(self.fused_rs_ctas >= 1, "fused_rs_ctas must be >= 1")
        _check(self.pipeline_micro_batches >= 1, "pipeline_micro_batches must be >= 1")


DATA_KINDS = ("pretraining", "supervised", "preference", "reward", "verifiable", "process", "trajectories")


@dataclass
class DataConfig:
    kind: str = "pretraining"
    path: str = "data"
    tokenizer: str = "auto"
    val_fraction: float = 0.1
    max_length: int = 256
    seed: int = 1337
    extra: Dict[str, Any] = field(default_factory=dict)

    def validate(self) -> None:
        _check(self.kind in DATA_KINDS, f"data kind must be one of {DATA_KINDS}, got {self.kind!r}")
        _check(0.0 <= self.val_fraction < 1.0, "val_fraction must be in [0, 1)")


@dataclass
class ExperimentManifest:
    """The complete, serialisable record of one run."""

    name: str = "experiment"
    algorithm: str = "pretrain"
    model: ModelSpec = field(default_factory=ModelSpec)
    model_preset: str = ""
    checkpoint_path: str = ""
    trainer: TrainerConfig = field(default_factory=TrainerConfig)
    data: DataConfig = field(default_factory=DataConfig)
    distributed: DistributedConfig = field(default_factory=DistributedConfig)
    algorithm_params: Dict[str, Any] = field(default_factory=dict)
    backend: Dict[str, Any] = field(default_factory=dict)
    reward: Dict[str, Any] = field(default_factory=dict)
    orchestration: Dict[str, Any] = field(default_factory=dict)
    evaluation: List[str] = field(default_factory=list)
    output_dir: str = "runs/experiment"
    tags: List[str] = field(default_factory=list)
    runtime: Dict[str, Any] = field(default_factory=dict)

    KNOWN_ALGORITHMS = (
        "pretrain", "sft", "distill", "reward_model", "dpo", "ppo", "grpo", "dapo",
        "rlvr", "rlaif", "constitutional", "star", "hill_climb", "tabular_ppo", "allocation_ppo",
    )

    def validate(self) -> None:
        _check(self.algorithm in self.KNOWN_ALGORITHMS,
               f"Unknown algorithm {self.algorithm!r}; expected one of {self.KNOWN_ALGORITHMS}")
        btype = (self.backend or {}).get("type", "native")
        _check(btype in ("native", "huggingface"), "backend.type must be native|huggingface")
        _check(not (btype == "huggingface" and not self.backend.get("model_name")),
               "backend.type=huggingface requires backend.model_name")
        from rl_project_b200.orchestration.config import validate_orchestration

        validate_orchestration(self.orchestration)
        for part in (self.model, self.trainer, self.data, self.distributed):
            part.validate()

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ExperimentManifest":
        data = dict(data)
        known = {f.name for f in fields(cls)}
        extra = sorted(set(data) - known)
        if extra:
            raise ConfigError(f"Unknown manifest keys: {extra}")
        preset = data.get("model_preset") or ""
        model_part = dict(data.get("model") or {})
        model = model_spec_from_preset(preset, **model_part) if preset else ModelSpec.from_dict(model_part)
        out = cls(
            name=data.get("name", "experiment"),
            algorithm=data.get("algorithm", "pretrain"),
            model=model,
            model_preset=preset,
            checkpoint_path=data.get("checkpoint_path", "") or "",
            trainer=build_nested(TrainerConfig, data.get("trainer")),
            data=build_nested(DataConfig, data.get("data")),
            distributed=build_nested(DistributedConfig, data.get("distributed")),
            algorithm_params=dict(data.get("algorithm_params") or {}),
            backend=dict(data.get("backend") or {}),
            reward=dict(data.get("reward") or {}),
            orchestration=dict(data.get("orchestration") or {}),
            evaluation=list(data.get("evaluation") or []),
            output_dir=data.get("output_dir", "runs/experiment"),
            tags=list(data.get("tags") or []),
            runtime=dict(data.get("runtime") or {}),
        )
        out.validate()
        return out

    def with_runtime_environment(self) -> "ExperimentManifest":
        self.runtime = capture_runtime_environment()
        return self

    def save(self, path: str | os.PathLike) -> Path:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(dump_config(self.to_dict(), fmt=_format_of(path)))
        return path

    @classmethod
    def load(cls, path: str | os.PathLike) -> "ExperimentManifest":
        return cls.from_dict(load_config(path))


# -----------------------------------------------------------------------------
# helpers
# -----------------------------------------------------------------------------


def build_nested(cls, data: Mapping[str, Any] | None):
    """Instantiate dataclass ``cls`` from ``data`` recursively, rejecting unknown keys."""
    data = dict(data or {})
    by_name = {f.name: f for f in fields(cls)}
    extra = sorted(set(data) - set(by_name))
    if extra:
        raise ConfigError(f"Unknown {cls.__name__} keys: {extra}")
    kwargs: Dict[str, Any] = {}
    for key, value in data.items():
        f = by_name[key]
        if f.default_factory is not dataclasses.MISSING:  # type: ignore[misc]
            proto = f.default_factory()  # type: ignore[misc]
            if dataclasses.is_dataclass(proto) and isinstance(value, Mapping):
                value = build_nested(type(proto), value)
        kwargs[key] = value
    obj = cls(**kwargs)
    if hasattr(obj, "validate"):
        obj.validate()
    return obj


def _format_of(path: Path) -> str:
    ext = path.suffix.lower()
    table = {".yaml": "yaml", ".yml": "yaml", ".toml": "toml", ".json": "json"}
    if ext not in table:
        raise ConfigError(f"Unsupported config extension {ext!r}; use .yaml, .toml or .json")
    return table[ext]


def load_config(path: str | os.PathLike) -> Dict[str, Any]:
    path = Path(path)
    if not path.exists():
        raise ConfigError(f"Config file not found: {path}")
    fmt = _format_of(path)
    text = path.read_text()
    if fmt == "yaml":
        import yaml

        data = yaml.safe_load(text) or {}
    elif fmt == "toml":
        import tomllib

        data = tomllib.loads(text)
    else:
        data = json.loads(text)
    if not isinstance(data, Mapping):
        raise ConfigError(f"Config root must be a mapping: {path}")
    return dict(data)


def dump_config(data: Mapping[str, Any], fmt: str = "yaml") -> str:
    if fmt == "yaml":
        import yaml

        return yaml.safe_dump(dict(data), sort_keys=False)
    if fmt == "json":
        return json.dumps(dict(data), indent=2)
    if fmt == "toml":
        return _toml_table(dict(data), "")
    raise ConfigError(f"Unsupported dump format {fmt!r}")


def _toml_scalar(v: Any) -> str:
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, (int, float)):
        return repr(v)
    if v is None:
        return '""'
    if isinstance(v, (list, tuple)):
        return "[" + ", ".join(_toml_scalar(x) for x in v) + "]"
    s = str(v).replace("\\", "\\\\").replace('"', '\\"')
    return f'"{s}"'


def _toml_table(data: Mapping[str, Any], prefix: str) -> str:
    scalars = [f"{k} = {_toml_scalar(v)}" for k, v in data.items() if not isinstance(v, Mapping)]
    out = "\n".join(scalars)
    for k, v in data.items():
        if isinstance(v, Mapping):
            name = f"{prefix}.{k}" if prefix else k
            out += f"\n\n[{name}]\n" + _toml_table(v, name)
    return out.strip() + "\n"


def capture_runtime_environment() -> Dict[str, Any]:
    import torch

    env: Dict[str, Any] = {
        "python": platform.python_version(),
        "platform": platform.platform(),
        "torch": str(torch.__version__),
        "cuda_available": bool(torch.cuda.is_available()),
        "cuda_device_count": torch.cuda.device_count() if torch.cuda.is_available() else 0,
        "framework": "rl_project_b200",
    }
    if env["cuda_available"]:
        env["cuda_device_name"] = torch.cuda.get_device_name(0)
    return env
