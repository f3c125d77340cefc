import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "multi_gpu: needs >= 2 CUDA devices")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    has_gpu = torch.cuda.is_available()
    skip_gpu = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords and not has_gpu:
            item.add_marker(skip_gpu)
        if "multi_gpu" in item.keywords and (not has_gpu or torch.cuda.device_count() < 2):
            item.add_marker(pytest.mark.skip(reason="needs >= 2 CUDA devices"))


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    import random

    random.seed(0)
    yield


@pytest.fixture
def tiny_spec():
    from rl_project_b200.core.config import model_spec_from_preset

    return model_spec_from_preset("tiny", vocab_size=97)


@pytest.fixture
def char_tok():
    from rl_project_b200.data.tokenizers import CharTokenizer

    return CharTokenizer.ascii()


@pytest.fixture
def cspec(char_tok):
    from rl_project_b200.core.config import model_spec_from_preset

    return model_spec_from_preset("tiny", vocab_size=char_tok.vocab_size, block_size=64)


@pytest.fixture
def corpus_dir(tmp_path, char_tok):
    import numpy as np

    from rl_project_b200.data.tokenizers import save_tokenizer_metadata

    text = "a small corpus about foxes and dogs. 2 + 3 = 5\n" * 150
    ids = np.array(char_tok.encode(text), dtype=np.uint16)
    cut = int(len(ids) * 0.9)
    ids[:cut].tofile(tmp_path / "train.bin")
    ids[cut:].tofile(tmp_path / "val.bin")
    save_tokenizer_metadata(char_tok, tmp_path)
    return tmp_path


@pytest.fixture
def make_ctx(tmp_path, cspec):
    from rl_project_b200.core.config import CheckpointConfig, ExperimentManifest, OptimizerConfig, TrainerConfig
    from rl_project_b200.core.lifecycle import RunContext

    def make(algorithm: str, *, max_steps=3, batch_size=4, eval_every=2, save_every=2, lr=None, spec=None, run=None,
             **kw):
        opt = OptimizerConfig(learning_rate=lr) if lr else OptimizerConfig()
        m = ExperimentManifest(name=f"t-{algorithm}", algorithm=algorithm, model=spec or cspec,
                               output_dir=str(tmp_path / (run or algorithm)),
                               trainer=TrainerConfig(max_steps=max_steps, batch_size=batch_size, eval_every=eval_every,
                                                     log_every=1, device="cpu", optimizer=opt,
                                                     checkpoint=CheckpointConfig(save_every=save_every, directory="ckpt"),
                                                     **kw))
        return RunContext.create(m, metrics_backend="local")

    return make
