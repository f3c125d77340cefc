"""GGUF (v3) export and header reading for the native model.

Follows the public GGUF/ggml file format: little-endian header (magic
``GGUF``, version, tensor count, metadata count), typed metadata, tensor infos
(name, dims innermost-first, ggml type, offset relative to the aligned data
section), 32-byte alignment.  Tensor encodings: F32, F16, Q8_0 (fp16 scale +
32 int8 per block) and Q4_0 (fp16 scale + 16 bytes; elements 0..15 in the low
nibbles, 16..31 in the high nibbles, stored as ``q + 8``).  Block quantisers are
vectorised over all blocks (no per-block Python loop).
Metadata keys match ``src/forgeline/models/quantization/gguf.py`` (architecture
"forgeline") so consumers of reference exports read ours.
"""

from __future__ import annotations

import struct
from pathlib import Path
from typing import Any, Dict, List, Mapping, Tuple

import numpy as np
import torch

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.core.errors import ExportError

GGUF_MAGIC = 0x46475547
GGUF_VERSION = 3
GGUF_ALIGNMENT = 32
T_U32, T_I32, T_F32, T_BOOL, T_STR, T_U64 = 4, 5, 6, 7, 8, 10
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8
FILE_TYPE = {GGML_F16: 1, GGML_Q8_0: 7, GGML_Q4_0: 2}
QUANT_FORMATS = ("none", "f16", "q8_0", "q4_0")

# reference-compatible aliases
GGUF_TYPE_UINT32, GGUF_TYPE_INT32, GGUF_TYPE_FLOAT32, GGUF_TYPE_BOOL, GGUF_TYPE_STRING, GGUF_TYPE_UINT64 = \
    T_U32, T_I32, T_F32, T_BOOL, T_STR, T_U64
GGML_TYPE_F32, GGML_TYPE_F16, GGML_TYPE_Q4_0, GGML_TYPE_Q8_0 = GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0


def _blocks(tensor: torch.Tensor) -> Tuple[np.ndarray, Tuple[int, ...], int]:
    arr = tensor.detach().float().cpu().numpy()
    flat = arr.reshape(-1)
    n = flat.size
    pad = (-n) % 32
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, np.float32)])
    return flat.reshape(-1, 32), arr.shape, n


def _pack(scales: np.ndarray, payload: np.ndarray) -> bytes:
    rec = np.empty(len(scales), dtype=[("d", "<f2"), ("q", payload.dtype, (payload.shape[1],))])
    rec["d"] = scales.astype(np.float16)
    rec["q"] = payload
    return rec.tobytes()


def quantize_q8_0(tensor: torch.Tensor) -> Tuple[bytes, Tuple[int, ...], int]:
    b, shape, n = _blocks(tensor)
    amax = np.abs(b).max(1)
    d = np.where(amax > 0, amax / 127.0, 1.0).astype(np.float32)
    q = np.clip(np.round(b / d[:, None]), -128, 127).astype(np.int8)
    return _pack(d, q), shape, n


def quantize_q4_0(tensor: torch.Tensor) -> Tuple[bytes, Tuple[int, ...], int]:
    b, shape, n = _blocks(tensor)
    amax = np.abs(b).max(1)
    d = np.where(amax > 0, amax / 7.0, 1.0).astype(np.float32)
    q = (np.clip(np.round(b / d[:, None]), -8, 7) + 8).astype(np.uint8)
    packed = (q[:, :16] | (q[:, 16:] << 4)).astype(np.uint8)
    return _pack(d, packed), shape, n


def _unpack(data: bytes, width: int, dtype) -> Tuple[np.ndarray, np.ndarray]:
    rec = np.frombuffer(data, dtype=[("d", "<f2"), ("q", dtype, (width,))])
    return rec["d"].astype(np.float32), rec["q"]


def dequantize_q8_0(data: bytes, n: int) -> np.ndarray:
    d, q = _unpack(data, 32, np.int8)
    return (q.astype(np.float32) * d[:, None]).reshape(-1)[:n]


def dequantize_q4_0(data: bytes, n: int) -> np.ndarray:
    d, p = _unpack(data, 16, np.uint8)
    lo = (p & 0x0F).astype(np.int8) - 8
    hi = (p >> 4).astype(np.int8) - 8
    return (np.concatenate([lo, hi], 1).astype(np.float32) * d[:, None]).reshape(-1)[:n]


def _str(f, s: str) -> None:
    b = s.encode("utf-8")
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


_FMT = {T_U32: "<I", T_I32: "<i", T_F32: "<f", T_BOOL: "<?", T_U64: "<Q"}


def _kv(f, key: str, vtype: int, value: Any) -> None:
    _str(f, key)
    f.write(struct.pack("<I", vtype))
    if vtype == T_STR:
        _str(f, str(value))
    elif vtype in _FMT:
        f.write(struct.pack(_FMT[vtype], value))
    else:
        raise ExportError(f"unsupported GGUF metadata type {vtype}")


def export_gguf(state_dict: Mapping[str, torch.Tensor], spec: ModelSpec, output_path: str | Path,
                quantize: str = "none", model_name: str = "forgeline") -> Dict[str, Any]:
    if quantize not in QUANT_FORMATS:
        raise ExportError(f"quantize must be one of {QUANT_FORMATS}, got {quantize!r}")
    out = Path(output_path)
    out.parent.mkdir(parents=True, exist_ok=True)
    infos: List[Dict[str, Any]] = []
    for name, p in state_dict.items():
        if "mtp_modules" in name:
            continue
        t = p.detach().cpu()
        if quantize in ("q8_0", "q4_0") and t.dim() >= 2:
            data, shape, n = (quantize_q8_0 if quantize == "q8_0" else quantize_q4_0)(t)
            ty = GGML_Q8_0 if quantize == "q8_0" else GGML_Q4_0
        elif t.dim() >= 2:
            data, shape, n, ty = t.half().numpy().tobytes(), tuple(t.shape), t.numel(), GGML_F16
        else:
            data, shape, n, ty = t.float().numpy().tobytes(), tuple(t.shape), t.numel(), GGML_F32
        infos.append({"name": name, "shape": list(shape), "type": ty, "data": data, "n_elem": n})
    off = 0
    for info in infos:
        info["offset"] = off
        off += len(info["data"]) + (-len(info["data"])) % GGUF_ALIGNMENT
    main = {"q8_0": GGML_Q8_0, "q4_0": GGML_Q4_0}.get(quantize, GGML_F16)
    meta = {
        "general.architecture": (T_STR, "forgeline"),
        "general.name": (T_STR, f"{model_name} {spec.n_layer}L"),
        "general.file_type": (T_U32, FILE_TYPE.get(main, 0)),
        "general.alignment": (T_U32, GGUF_ALIGNMENT),
        "forgeline.context_length": (T_U32, spec.block_size),
        "forgeline.embedding_length": (T_U32, spec.n_embd),
        "forgeline.block_count": (T_U32, spec.n_layer),
        "forgeline.head_count": (T_U32, spec.n_head),
        "forgeline.head_count_kv": (T_U32, spec.n_kv_head),
        "forgeline.vocab_size": (T_U32, spec.vocab_size),
        "forgeline.use_moe": (T_BOOL, spec.use_moe),
        "forgeline.use_mla": (T_BOOL, spec.use_mla),
        "forgeline.use_swiglu": (T_BOOL, spec.use_swiglu),
        "forgeline.use_rope": (T_BOOL, spec.use_rope),
        "forgeline.sliding_window": (T_U32, spec.sliding_window),
        "forgeline.feed_forward_length": (T_U32, spec.ffn_hidden),
        "forgeline.rope.freq_base": (T_F32, spec.rope_theta),
    }
    with out.open("wb") as f:
        f.write(struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(infos), len(meta)))
        for k, (vt, v) in meta.items():
            _kv(f, k, vt, v)
        for info in infos:
            _str(f, info["name"])
            f.write(struct.pack("<I", len(info["shape"])))
            for dim in reversed(info["shape"]):
                f.write(struct.pack("<Q", dim))
            f.write(struct.pack("<IQ", info["type"], info["offset"]))
        f.write(b"\x00" * ((-f.tell()) % GGUF_ALIGNMENT))
        start = f.tell()
        for info in infos:
            if f.tell() - start != info["offset"]:
                raise ExportError("GGUF offset bookkeeping error")
            f.write(info["data"])
            f.write(b"\x00" * ((-len(info["data"])) % GGUF_ALIGNMENT))
    size = out.stat().st_size
    fp32 = sum(int(p.numel()) * 4 for p in state_dict.values())
    return {"path": str(out), "bytes": size, "tensors": len(infos), "format": quantize, "fp32_bytes": fp32,
            "compression": size / max(fp32, 1)}


def read_gguf_header(path: str | Path) -> Dict[str, Any]:
    path = Path(path)
    with path.open("rb") as f:
        magic, version = struct.unpack("<II", f.read(8))
        if magic != GGUF_MAGIC:
            raise ExportError(f"{path} is not a GGUF file")
        n_t, n_kv = struct.unpack("<QQ", f.read(16))

        def rstr() -> str:
            (ln,) = struct.unpack("<Q", f.read(8))
            return f.read(ln).decode("utf-8")

        meta: Dict[str, Any] = {}
        for _ in range(n_kv):
            key = rstr()
            (vt,) = struct.unpack("<I", f.read(4))
            if vt == T_STR:
                meta[key] = rstr()
            elif vt in _FMT:
                fmt = _FMT[vt]
                meta[key] = struct.unpack(fmt, f.read(struct.calcsize(fmt)))[0]
            else:
                raise ExportError(f"unsupported GGUF metadata type {vt}")
        tensors = []
        for _ in range(n_t):
            name = rstr()
            (nd,) = struct.unpack("<I", f.read(4))
            dims = list(struct.unpack(f"<{nd}Q", f.read(8 * nd)))[::-1]
            ty, off = struct.unpack("<IQ", f.read(12))
            tensors.append({"name": name, "shape": dims, "type": ty, "offset": off})
        data_start = f.tell() + ((-f.tell()) % GGUF_ALIGNMENT)
    return {"version": version, "metadata": meta, "tensors": tensors, "data_start": data_start}


def read_gguf_tensor(path: str | Path, name: str) -> np.ndarray:
    hdr = read_gguf_header(path)
    info = next(t for t in hdr["tensors"] if t["name"] == name)
    n = int(np.prod(info["shape"])) if info["shape"] else 1
    nbytes = {GGML_F32: 4 * n, GGML_F16: 2 * n, GGML_Q8_0: ((n + 31) // 32) * 34,
              GGML_Q4_0: ((n + 31) // 32) * 18}[info["type"]]
    with Path(path).open("rb") as f:
        f.seek(hdr["data_start"] + info["offset"])
        raw = f.read(nbytes)
    if info["type"] == GGML_F32:
        arr = np.frombuffer(raw, np.float32)
    elif info["type"] == GGML_F16:
        arr = np.frombuffer(raw, np.float16).astype(np.float32)
    elif info["type"] == GGML_Q8_0:
        arr = dequantize_q8_0(raw, n)
    else:
        arr = dequantize_q4_0(raw, n)
    return arr.reshape(info["shape"])
