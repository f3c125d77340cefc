"""Corpus preparation: a text file (or a streamed HuggingFace dataset) to ``train.bin`` / ``val.bin`` token
files plus ``meta.pkl`` (capabilities of ``src/forgeline/data/preprocessing.py``; the file layout is the
reference's, so its prepared corpora load here and the other way round).

Character and byte tokenizers map text one character at a time, so a text file is read and encoded in
fixed-size chunks straight into one preallocated id array (memory: the ids plus one chunk of text; the
character alphabet is fitted in a first pass over the same chunks).  BPE tokenizers (tiktoken,
HuggingFace) see the whole text at once, since their merges may cross any chunk boundary.  The last
``val_fraction`` of the ids is the validation split.
"""

from __future__ import annotations

from pathlib import Path
from typing import Dict, Iterator, Optional

import numpy as np

from rl_project_b200.core.errors import DatasetError, OptionalDependencyError
from rl_project_b200.data.tokenizers import (ByteTokenizer, CharTokenizer, HFTokenizer, TiktokenTokenizer,
                                             save_tokenizer_metadata, token_dtype_for)

_CHUNK_CHARS = 1 << 24


def _chunks(path: Path) -> Iterator[str]:
    with path.open("r", encoding="utf-8") as fh:
        while True:
            piece = fh.read(_CHUNK_CHARS)
            if not piece:
                return
            yield piece


def _encode_per_char(path: Path, tok) -> np.ndarray:
    """Ids of the whole file, encoded chunk by chunk (exact for per-character tokenizers)."""
    parts = [np.asarray(tok.encode(c), dtype=token_dtype_for(tok.vocab_size)) for c in _chunks(path)]
    return np.concatenate(parts) if parts else np.zeros(0, dtype=token_dtype_for(tok.vocab_size))


def _tokenize_file(path: Path, name: str):
    if name == "char":
        alphabet = set()
        for c in _chunks(path):
            alphabet.update(c)
        tok = CharTokenizer(sorted(alphabet))
        return tok, _encode_per_char(path, tok)
    if name == "byte":
        tok = ByteTokenizer()
        return tok, _encode_per_char(path, tok)
    head, _, arg = name.partition(":")
    if head == "tiktoken":
        tok = TiktokenTokenizer(arg or "cl100k_base")
    elif head == "hf" and arg:
        tok = HFTokenizer(arg)
    else:
        raise DatasetError(f"Unknown tokenizer {name!r}; use char|byte|tiktoken[:enc]|hf:<name>")
    ids = tok.encode(path.read_text(encoding="utf-8"))
    return tok, np.asarray(ids, dtype=token_dtype_for(tok.vocab_size))


def prepare_text_corpus(input_file: str | Path, output_dir: str | Path, tokenizer: str = "char",
                        val_fraction: float = 0.1) -> Dict[str, object]:
    src = Path(input_file)
    if not src.exists():
        raise DatasetError(f"Input text file not found: {src}")
    tok, ids = _tokenize_file(src, tokenizer)
    n = int(ids.shape[0])
    if n < 10:
        raise DatasetError("corpus is too small after tokenization")
    cut = int(n * (1 - val_fraction))
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    ids[:cut].tofile(out / "train.bin")
    ids[cut:].tofile(out / "val.bin")
    save_tokenizer_metadata(tok, out)
    return {"tokens": n, "train_tokens": cut, "val_tokens": n - cut, "vocab_size": tok.vocab_size,
            "tokenizer": tok.kind, "output_dir": str(out)}


def prepare_hf_corpus(dataset_name: str, output_dir: str | Path, tokenizer_name: str = "Qwen/Qwen2.5-0.5B",
                      subset: Optional[str] = None, max_tokens: int = 100_000_000, shard_size: int = 10_000_000,
                      text_field: str = "text", split: str = "train") -> Dict[str, object]:
    """Stream a HuggingFace dataset's ``text_field`` into uint32 shard files (needs ``datasets``)."""
    from rl_project_b200.data.streaming import write_shards_from_documents

    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise OptionalDependencyError("datasets is not installed", hint="pip install datasets") from exc
    tok = HFTokenizer(tokenizer_name)
    args = (dataset_name, subset) if subset else (dataset_name,)
    rows = load_dataset(*args, split=split, streaming=True)
    res = write_shards_from_documents((r.get(text_field, "") for r in rows), tok, output_dir, max_tokens=max_tokens,
                                      shard_size=shard_size, dtype=np.uint32)
    save_tokenizer_metadata(tok, output_dir)
    return {**res, "dataset": dataset_name, "subset": subset, "tokenizer": tokenizer_name,
            "vocab_size": tok.vocab_size}
