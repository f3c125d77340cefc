"""Corpus preparation: text -> tokens -> ``train.bin`` / ``val.bin`` + ``meta.pkl``
(``src/forgeline/data/preprocessing.py``)."""

from __future__ import annotations

from pathlib import Path
from typing import Dict, Optional

import numpy as np

from rl_project_b200.core.errors import DatasetError, OptionalDependencyError
from rl_project_b200.data.tokenizers import (ByteTokenizer, CharTokenizer, HFTokenizer, TiktokenTokenizer,
                                             save_tokenizer_metadata, token_dtype_for)


def _tokenizer_for(name: str, text: str):
    if name == "char":
        return CharTokenizer().fit(text)
    if name == "byte":
        return ByteTokenizer()
    if name.startswith("tiktoken"):
        return TiktokenTokenizer(name.partition(":")[2] or "cl100k_base")
    if name.startswith("hf:"):
        return HFTokenizer(name[3:])
    raise DatasetError(f"Unknown tokenizer {name!r}; use char|byte|tiktoken[:enc]|hf:<name>")


def prepare_text_corpus(input_file: str | Path, output_dir: str | Path, tokenizer: str = "char",
                        val_fraction: float = 0.1) -> Dict[str, object]:
    src = Path(input_file)
    if not src.exists():
        raise DatasetError(f"Input text file not found: {src}")
    text = src.read_text(encoding="utf-8")
    tok = _tokenizer_for(tokenizer, text)
    ids = tok.encode(text)
    if len(ids) < 10:
        raise DatasetError("corpus is too small after tokenization")
    dt = token_dtype_for(tok.vocab_size)
    cut = int(len(ids) * (1 - val_fraction))
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    np.asarray(ids[:cut], dtype=dt).tofile(out / "train.bin")
    np.asarray(ids[cut:], dtype=dt).tofile(out / "val.bin")
    save_tokenizer_metadata(tok, out)
    return {"tokens": len(ids), "train_tokens": cut, "val_tokens": len(ids) - cut, "vocab_size": tok.vocab_size,
            "tokenizer": tok.kind, "output_dir": str(out)}


def prepare_hf_corpus(dataset_name: str, output_dir: str | Path, tokenizer_name: str = "Qwen/Qwen2.5-0.5B",
                      subset: Optional[str] = None, max_tokens: int = 100_000_000, shard_size: int = 10_000_000,
                      text_field: str = "text", split: str = "train") -> Dict[str, object]:
    from rl_project_b200.data.streaming import write_shards_from_documents

    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise OptionalDependencyError("datasets is not installed", hint="pip install datasets") from exc
    tok = HFTokenizer(tokenizer_name)
    ds = (load_dataset(dataset_name, subset, split=split, streaming=True) if subset
          else load_dataset(dataset_name, split=split, streaming=True))
    res = write_shards_from_documents((row.get(text_field, "") for row in ds), tok, output_dir, max_tokens=max_tokens,
                                      shard_size=shard_size, dtype=np.uint32)
    save_tokenizer_metadata(tok, output_dir)
    res.update({"dataset": dataset_name, "subset": subset, "tokenizer": tokenizer_name, "vocab_size": tok.vocab_size})
    return res
