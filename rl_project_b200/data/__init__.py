"""Data: tokenizers, record schemas, memmap / streaming corpora, collators, datasets, synthetic sources."""

from rl_project_b200.data.collators import (IGNORE_INDEX, SupervisedBatch, collate_lm, collate_preference,
                                            collate_supervised, pad_sequences)
from rl_project_b200.data.preference import PreferenceDataset
from rl_project_b200.data.pretraining import MemmapCorpus
from rl_project_b200.data.records import (PreferenceRecord, ProcessRecord, RewardRecord, SFTRecord, VerifiableTask,
                                          deterministic_split, read_jsonl, write_jsonl)
from rl_project_b200.data.supervised import SupervisedDataset
from rl_project_b200.data.tokenizers import (ByteTokenizer, CharTokenizer, resolve_tokenizer,
                                             save_tokenizer_metadata, tokenizer_from_metadata)
from rl_project_b200.data.verifiable import VerifiableTaskDataset, load_prompts
