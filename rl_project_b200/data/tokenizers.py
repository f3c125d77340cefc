"""Tokenizers: character (dependency-free), byte-level (vocab 256), tiktoken and HuggingFace.

Capabilities of ``src/forgeline/data/tokenizers.py``.  The on-disk contract is the reference's: a
``meta.pkl`` pickled dict keyed by ``tokenizer_type`` (``char`` with ``char_to_idx`` / ``idx_to_char``,
``tiktoken`` with ``encoding_name``, ``huggingface`` with ``tokenizer_name``, plus ``byte``) and
``vocab_size``, so prepared corpora and checkpoints resolve the same vocabulary.

The character tokenizer works on code-point arrays: the alphabet is held as one string plus its code
points sorted with their ids, ``encode`` maps a whole text with one ``searchsorted`` (characters outside the
alphabet are dropped) and ``decode`` indexes the alphabet.  Kinds are rebuilt from metadata through the
``_FROM_META`` table and specs (``auto | char | byte | tiktoken[:enc] | hf:<name>``) through ``_SPECS``.
"""

from __future__ import annotations

import pickle
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Protocol, Sequence, Tuple, runtime_checkable

import numpy as np

from rl_project_b200.core.errors import OptionalDependencyError, TokenizerError

META_FILE = "meta.pkl"


@runtime_checkable
class Tokenizer(Protocol):
    kind: str
    vocab_size: int

    def encode(self, text: str) -> List[int]: ...

    def decode(self, ids: Sequence[int]) -> str: ...

    def metadata(self) -> Dict[str, Any]: ...


def _code_points(text: str) -> np.ndarray:
    return np.frombuffer(text.encode("utf-32-le", errors="surrogatepass"), dtype=np.uint32)


class CharTokenizer:
    """One id per character of the alphabet (a fitted or given character set, ids in sorted order)."""

    kind = "char"

    def __init__(self, chars: Optional[Sequence[str]] = None):
        self._install("".join(sorted(set(chars or ()))))

    def _install(self, alphabet: str) -> None:
        """``alphabet[i]`` is the character of id ``i``."""
        self.alphabet = alphabet
        self.vocab_size = len(alphabet)
        points = _code_points(alphabet)
        order = np.argsort(points, kind="stable")
        self._sorted_points, self._sorted_ids = points[order], order.astype(np.int64)

    def fit(self, text: str) -> "CharTokenizer":
        self._install("".join(sorted(set(text))))
        return self

    @classmethod
    def ascii(cls) -> "CharTokenizer":
        """Printable ASCII plus newline and tab."""
        return cls([chr(c) for c in range(32, 127)] + ["\n", "\t"])

    @property
    def char_to_idx(self) -> Dict[str, int]:
        return {c: i for i, c in enumerate(self.alphabet)}

    @property
    def idx_to_char(self) -> Dict[int, str]:
        return dict(enumerate(self.alphabet))

    def encode(self, text: str) -> List[int]:
        if not self.vocab_size or not text:
            return []
        cp = _code_points(text)
        pos = np.searchsorted(self._sorted_points, cp)
        pos = np.minimum(pos, self.vocab_size - 1)
        hit = self._sorted_points[pos] == cp
        return self._sorted_ids[pos[hit]].tolist()

    def decode(self, ids: Sequence[int]) -> str:
        a, n = self.alphabet, self.vocab_size
        return "".join(a[i] if 0 <= i < n else "?" for i in map(int, ids))

    def metadata(self) -> Dict[str, Any]:
        return {"tokenizer_type": "char", "vocab_size": self.vocab_size, "char_to_idx": self.char_to_idx,
                "idx_to_char": self.idx_to_char}

    @classmethod
    def from_metadata(cls, meta: Dict[str, Any]) -> "CharTokenizer":
        by_id = sorted((int(i), str(c)) for i, c in meta["idx_to_char"].items())
        if [i for i, _ in by_id] != list(range(len(by_id))):
            raise TokenizerError("char tokenizer metadata: ids are not 0..n-1")
        tok = cls()
        tok._install("".join(c for _, c in by_id))
        return tok


class ByteTokenizer:
    """UTF-8 bytes as ids 0..255."""

    kind = "byte"
    vocab_size = 256

    def encode(self, text: str) -> List[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: Sequence[int]) -> str:
        return bytes(int(i) & 0xFF for i in ids).decode("utf-8", errors="replace")

    def metadata(self) -> Dict[str, Any]:
        return {"tokenizer_type": "byte", "vocab_size": 256}


def _optional(module: str, hint: str):
    import importlib

    try:
        return importlib.import_module(module)
    except ImportError as exc:
        raise OptionalDependencyError(f"{module} is not installed", hint=hint) from exc


class TiktokenTokenizer:
    kind = "tiktoken"

    def __init__(self, encoding_name: str = "cl100k_base"):
        self.encoding_name = encoding_name
        self.enc = _optional("tiktoken", "pip install tiktoken").get_encoding(encoding_name)
        self.vocab_size = self.enc.n_vocab

    def encode(self, text: str) -> List[int]:
        return self.enc.encode(text, allowed_special=set())  # special-token text is encoded as plain text

    def decode(self, ids: Sequence[int]) -> str:
        return self.enc.decode(list(ids))

    def metadata(self) -> Dict[str, Any]:
        return {"tokenizer_type": "tiktoken", "encoding_name": self.encoding_name, "vocab_size": self.vocab_size}


class HFTokenizer:
    kind = "huggingface"

    def __init__(self, name: str, padding_side: str = "left"):
        auto = _optional("transformers", "pip install transformers").AutoTokenizer
        self.name = name
        self.hf = auto.from_pretrained(name, trust_remote_code=True, padding_side=padding_side)
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


# ---------------------------------------------------------------- metadata files
def save_tokenizer_metadata(tokenizer: Tokenizer, directory: str | Path) -> Path:
    path = Path(directory) / META_FILE
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_bytes(pickle.dumps(tokenizer.metadata()))
    return path


def load_tokenizer_metadata(directory: str | Path) -> Dict[str, Any]:
    path = Path(directory) / META_FILE
    if not path.exists():
        raise TokenizerError(f"Tokenizer metadata not found at {path}", hint="Prepare the corpus first (`data prepare`).")
    meta = pickle.loads(path.read_bytes())
    if not isinstance(meta, dict) or "tokenizer_type" not in meta:
        raise TokenizerError(f"Malformed tokenizer metadata at {path}")
    return meta


_FROM_META: Dict[str, Callable[[Dict[str, Any]], Tokenizer]] = {
    "char": CharTokenizer.from_metadata,
    "byte": lambda meta: ByteTokenizer(),
    "tiktoken": lambda meta: TiktokenTokenizer(meta.get("encoding_name", "cl100k_base")),
    "huggingface": lambda meta: HFTokenizer(meta.get("tokenizer_name", "")),
}


def tokenizer_from_metadata(meta: Dict[str, Any]) -> Tokenizer:
    kind = meta.get("tokenizer_type", "char")
    build = _FROM_META.get(kind)
    if build is None:
        raise TokenizerError(f"Unknown tokenizer type {kind!r}")
    return build(meta)


def load_tokenizer(directory: str | Path) -> Tokenizer:
    return tokenizer_from_metadata(load_tokenizer_metadata(directory))


# ---------------------------------------------------------------- specs
def _auto(arg: str, data_dir: Optional[Path]) -> Tokenizer:
    if data_dir is None:
        raise TokenizerError("tokenizer=auto requires a data directory containing meta.pkl")
    return load_tokenizer(data_dir)


def _char(arg: str, data_dir: Optional[Path]) -> Tokenizer:
    if data_dir is not None and (data_dir / META_FILE).exists():
        return load_tokenizer(data_dir)  # the corpus's own fitted alphabet
    return CharTokenizer.ascii()


# spec head -> (takes an argument after ':', builder)
_SPECS: Dict[str, Tuple[bool, Callable[[str, Optional[Path]], Tokenizer]]] = {
    "auto": (False, _auto),
    "char": (False, _char),
    "byte": (False, lambda arg, d: ByteTokenizer()),
    "tiktoken": (True, lambda arg, d: TiktokenTokenizer(arg or "cl100k_base")),
    "hf": (True, lambda arg, d: HFTokenizer(arg)),
}


def resolve_tokenizer(spec: str, data_dir: Optional[str | Path] = None) -> Tokenizer:
    head, sep, arg = spec.partition(":")
    entry = _SPECS.get(head)
    if entry is None or (sep and not entry[0]) or (head == "hf" and not sep):
        raise TokenizerError(f"Unknown tokenizer spec {spec!r}; use auto|char|byte|tiktoken[:enc]|hf:<name>")
    return entry[1](arg, Path(data_dir) if data_dir is not None else None)


def token_dtype_for(vocab_size: int):
    """The narrowest unsigned id type that holds ``vocab_size`` ids (uint16 or uint32)."""
    return np.uint16 if vocab_size <= np.iinfo(np.uint16).max else np.uint32
