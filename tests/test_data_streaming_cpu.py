"""Streaming data path: window packing, shard writing and merging, sharded windows, corpus preparation."""

from __future__ import annotations

import numpy as np
import torch

from rl_project_b200.data.collators import IGNORE_INDEX, collate_supervised, pad_sequences
from rl_project_b200.data.streaming import (ShardedTokenDataset, TokenPacker, pack_documents, shard_token_file,
                                            write_shards_from_documents)


class _Ids:
    """Tokeniser stub: whitespace-separated integers."""

    vocab_size = 1000

    def encode(self, text):
        return [int(t) for t in text.split()]


def test_packer_windows_overlap_by_one_token_across_documents():
    p = TokenPacker(3, capacity=4)  # forces compaction and growth
    got = []
    for doc in ([1, 2], [3, 4, 5, 6, 7], [8], list(range(9, 30))):
        p.push(doc)
        got += [(x.tolist(), y.tolist()) for x, y in p.windows()]
    flat = list(range(1, 30))
    want = [(flat[s:s + 3], flat[s + 1:s + 4]) for s in range(0, len(flat) - 3, 3)]
    assert got == want


def test_pack_documents_filters_and_stops_after_max_tokens():
    docs = ["1 2 3", "", "0 4 0 5", "6 7 8 9 10 11 12 13", "14 15"]
    wins = list(pack_documents(docs, _Ids(), 2, max_tokens=7, drop_token_zero=True))
    # the stream is 1..13 (zeros dropped); it stops after the document that passes 7 tokens
    assert [x.tolist() for x, _ in wins] == [[1, 2], [3, 4], [5, 6], [7, 8], [9, 10], [11, 12]]


def test_shard_writer_splits_long_documents_and_merges(tmp_path):
    docs = [" ".join(str(i) for i in range(1, 26)), "26 27 28", " ".join(str(i) for i in range(29, 41))]
    res = write_shards_from_documents(docs, _Ids(), tmp_path, max_tokens=10 ** 6, shard_size=7, dtype=np.uint32,
                                      min_chars=0)
    assert res["total_tokens"] == 40 and res["docs"] == 3 and res["num_shards"] == 6
    val = np.fromfile(tmp_path / "val.bin", dtype=np.uint32)
    train = np.fromfile(tmp_path / "train.bin", dtype=np.uint32)
    assert val.tolist() == list(range(1, 8)) and train.tolist() == list(range(8, 41))


def test_sharded_dataset_splits_shards_over_ranks(tmp_path):
    src = tmp_path / "all.bin"
    np.arange(400, dtype=np.uint16).tofile(src)
    paths = shard_token_file(src, tmp_path / "shards", 4)
    assert len(paths) == 4
    seen = []
    for rank in range(2):
        ds = ShardedTokenDataset(tmp_path / "shards", 16, shuffle=False, world_size=2, rank=rank)
        for x, y in ds:
            assert torch.equal(y[:-1], x[1:]) and int(y[-1]) == int(x[-1]) + 1
            seen.append(int(x[0]) // 100)
    assert sorted(set(seen)) == [0, 1, 2, 3]


def test_collators_pad_and_mask():
    ids, mask = pad_sequences([[5, 6], [], [7]], 0, "left")
    assert ids.tolist() == [[5, 6], [0, 0], [0, 7]] and mask.tolist() == [[1, 1], [0, 0], [0, 1]]
    b = collate_supervised([([1, 2, 3], [4, 5]), ([6], [7, 8])])
    assert b.input_ids.tolist() == [[1, 2, 3, 4], [6, 7, 8, 0]]
    I = IGNORE_INDEX
    assert b.targets.tolist() == [[I, I, 4, 5], [7, 8, I, I]]
    assert collate_supervised([([1, 2, 3], [4, 5])], mask_prompt=False).targets.tolist() == [[2, 3, 4, 5]]


def test_prepare_text_corpus_char_and_byte(tmp_path):
    from rl_project_b200.data.preprocessing import prepare_text_corpus
    from rl_project_b200.data.pretraining import MemmapCorpus
    from rl_project_b200.data.tokenizers import load_tokenizer

    text = "the quick brown fox jumps over the lazy dog\n" * 50
    (tmp_path / "in.txt").write_text(text)
    for kind in ("char", "byte"):
        out = tmp_path / kind
        info = prepare_text_corpus(tmp_path / "in.txt", out, tokenizer=kind, val_fraction=0.1)
        assert info["tokens"] == len(text) and info["train_tokens"] == int(len(text) * 0.9)
        tok = load_tokenizer(out)
        c = MemmapCorpus(out, "train", 32)
        x, y = c.sample_batch(3, generator=torch.Generator().manual_seed(0))
        assert all(tok.decode(row.tolist()) in text for row in x)
