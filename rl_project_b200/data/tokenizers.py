"""Tokenizers: character (dependency-free), byte-level (vocab 256), tiktoken, HuggingFace.

Metadata is persisted as ``meta.pkl`` (same keys as
``src/forgeline/data/tokenizers.py:28-186`` so existing corpora and checkpoints
resolve the same vocabulary); ``resolve_tokenizer`` accepts
``auto | char | byte | tiktoken[:enc] | hf:<name>``.
"""

from __future__ import annotations

import pickle
from pathlib import Path
from typing import Any, Dict, List, Optional, Protocol, Sequence, runtime_checkable

from rl_project_b200.core.errors import OptionalDependencyError, TokenizerError


@runtime_checkable
class Tokenizer(Protocol):
    kind: str
    vocab_size: int

    def encode(self, text: str) -> List[int]: ...

    def decode(self, ids: Sequence[int]) -> str: ...

    def metadata(self) -> Dict[str, Any]: ...


class CharTokenizer:
    """One id per distinct character (sorted); unknown characters are dropped on encode."""

    kind = "char"

    def __init__(self, chars: Optional[Sequence[str]] = None):
        self.char_to_idx: Dict[str, int] = {}
        self.idx_to_char: Dict[int, str] = {}
        self.vocab_size = 0
        if chars is not None:
            self._vocab(chars)

    def _vocab(self, chars: Sequence[str]) -> None:
        ordered = sorted(set(chars))
        self.char_to_idx = {c: i for i, c in enumerate(ordered)}
        self.idx_to_char = {i: c for c, i in self.char_to_idx.items()}
        self.vocab_size = len(ordered)

    def fit(self, text: str) -> "CharTokenizer":
        self._vocab(list(text))
        return self

    @classmethod
    def ascii(cls) -> "CharTokenizer":
        return cls([chr(c) for c in range(32, 127)] + ["\n", "\t"])

    def encode(self, text: str) -> List[int]:
        table = self.char_to_idx
        return [table[c] for c in text if c in table]

    def decode(self, ids: Sequence[int]) -> str:
        return "".join(self.idx_to_char.get(int(i), "?") for i in ids)

    def metadata(self) -> Dict[str, Any]:
        return {"tokenizer_type": "char", "vocab_size": self.vocab_size, "char_to_idx": dict(self.char_to_idx),
                "idx_to_char": dict(self.idx_to_char)}

    @classmethod
    def from_metadata(cls, meta: Dict[str, Any]) -> "CharTokenizer":
        tok = cls()
        tok.char_to_idx = {str(k): int(v) for k, v in meta["char_to_idx"].items()}
        tok.idx_to_char = {int(k): str(v) for k, v in meta["idx_to_char"].items()}
        tok.vocab_size = int(meta["vocab_size"])
        return tok


class ByteTokenizer:
    """UTF-8 bytes as ids 0..255 (the tiny benchmark configuration's vocabulary)."""

    kind = "byte"
    vocab_size = 256

    def encode(self, text: str) -> List[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: Sequence[int]) -> str:
        return bytes(int(i) % 256 for i in ids).decode("utf-8", errors="replace")

    def metadata(self) -> Dict[str, Any]:
        return {"tokenizer_type": "byte", "vocab_size": 256}


class TiktokenTokenizer:
    kind = "tiktoken"

    def __init__(self, encoding_name: str = "cl100k_base"):
        try:
            import tiktoken
        except ImportError as exc:
            raise OptionalDependencyError("tiktoken is not installed", hint="pip install tiktoken") from exc
        self.encoding_name = encoding_name
        self.enc = tiktoken.get_encoding(encoding_name)
        self.vocab_size = self.enc.n_vocab

    def encode(self, text: str) -> List[int]:
        return self.enc.encode(text, allowed_special=set())

    def decode(self, ids: Sequence[int]) -> str:
        return self.enc.decode(list(ids))

    def metadata(self) -> Dict[str, Any]:
        return {"tokenizer_type": "tiktoken", "encoding_name": self.encoding_name, "vocab_size": self.vocab_size}


class HFTokenizer:
    kind = "huggingface"

    def __init__(self, name: str, padding_side: str = "left"):
        try:
            from transformers import AutoTokenizer
        except ImportError as exc:
            raise OptionalDependencyError("transformers is not installed", hint="pip install transformers") from exc
        self.name = name
        self.hf = AutoTokenizer.from_pretrained(name, trust_remote_code=True, padding_side=padding_side)
        if self.hf.pad_token is None:
            self.hf.pad_token = self.hf.eos_token
        self.vocab_size = int(self.hf.vocab_size)

    def encode(self, text: str) -> List[int]:
        return self.hf.encode(text, add_special_tokens=False)

    def decode(self, ids: Sequence[int]) -> str:
        return self.hf.decode(list(ids), skip_special_tokens=True)

    @property
    def eos_token_id(self) -> Optional[int]:
        return self.hf.eos_token_id

    def metadata(self) -> Dict[str, Any]:
        return {"tokenizer_type": "huggingface", "tokenizer_name": self.name, "vocab_size": self.vocab_size}


def save_tokenizer_metadata(tokenizer: Tokenizer, directory: str | Path) -> Path:
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    with (d / "meta.pkl").open("wb") as fh:
        pickle.dump(tokenizer.metadata(), fh)
    return d / "meta.pkl"


def load_tokenizer_metadata(directory: str | Path) -> Dict[str, Any]:
    p = Path(directory) / "meta.pkl"
    if not p.exists():
        raise TokenizerError(f"Tokenizer metadata not found at {p}", hint="Prepare the corpus first (`data prepare`).")
    with p.open("rb") as fh:
        meta = pickle.load(fh)
    if not isinstance(meta, dict) or "tokenizer_type" not in meta:
        raise TokenizerError(f"Malformed tokenizer metadata at {p}")
    return meta


def tokenizer_from_metadata(meta: Dict[str, Any]) -> Tokenizer:
    kind = meta.get("tokenizer_type", "char")
    if kind == "char":
        return CharTokenizer.from_metadata(meta)
    if kind == "byte":
        return ByteTokenizer()
    if kind == "tiktoken":
        return TiktokenTokenizer(meta.get("encoding_name", "cl100k_base"))
    if kind == "huggingface":
        return HFTokenizer(meta.get("tokenizer_name", ""))
    raise TokenizerError(f"Unknown tokenizer type {kind!r}")


def load_tokenizer(directory: str | Path) -> Tokenizer:
    return tokenizer_from_metadata(load_tokenizer_metadata(directory))


def resolve_tokenizer(spec: str, data_dir: Optional[str | Path] = None) -> Tokenizer:
    if spec == "auto":
        if data_dir is None:
            raise TokenizerError("tokenizer=auto requires a data directory containing meta.pkl")
        return load_tokenizer(data_dir)
    if spec == "char":
        if data_dir is not None and (Path(data_dir) / "meta.pkl").exists():
            return load_tokenizer(data_dir)
        return CharTokenizer.ascii()
    if spec == "byte":
        return ByteTokenizer()
    if spec.startswith("tiktoken"):
        return TiktokenTokenizer(spec.partition(":")[2] or "cl100k_base")
    if spec.startswith("hf:"):
        return HFTokenizer(spec[3:])
    raise TokenizerError(f"Unknown tokenizer spec {spec!r}; use auto|char|byte|tiktoken[:enc]|hf:<name>")


def token_dtype_for(vocab_size: int):
    import numpy as np

    return np.uint32 if vocab_size > 65535 else np.uint16
