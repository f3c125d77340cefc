"""Adapters and quantisation (the reference's unit/test_adapters_quantization.py is the model): LoRA is the
identity at init and merges exactly, NF4 round trips within its grid, QLoRA trains only the adapter, GGUF
exports read back, block quantisers round trip."""
import numpy as np
import pytest
import torch

from rl_project_b200.core.config import model_spec_from_preset
from rl_project_b200.models.transformer.model import TransformerLM


def test_lora_identity_at_init_merge_and_state():
    from rl_project_b200.models.adapters.lora import (apply_lora, lora_state_dict, load_lora_state_dict, merge_lora,
                                                      set_lora_enabled, trainable_parameter_report)

    torch.manual_seed(0)
    m = TransformerLM(model_spec_from_preset("tiny", vocab_size=64)).eval()
    x = torch.randint(0, 64, (2, 16))
    base, _ = m(x)
    apply_lora(m, rank=4)
    same, _ = m(x)
    torch.testing.assert_close(same, base)  # B starts at zero
    rep = trainable_parameter_report(m)
    assert 0 < rep["trainable"] < rep["total"]
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("lora_B"):
                p.normal_(0, 0.05)
    adapted, _ = m(x)
    assert (adapted - base).abs().max() > 1e-4
    set_lora_enabled(m, False)
    torch.testing.assert_close(m(x)[0], base)
    set_lora_enabled(m, True)
    state = lora_state_dict(m)
    merged = merge_lora(m)
    torch.testing.assert_close(merged(x)[0], adapted, atol=1e-5, rtol=1e-5)
    m2 = TransformerLM(model_spec_from_preset("tiny", vocab_size=64)).eval()
    m2.load_state_dict(TransformerLM(model_spec_from_preset("tiny", vocab_size=64)).state_dict())
    apply_lora(m2, rank=4)
    assert load_lora_state_dict(m2, state) == len(state)


def test_nf4_roundtrip_and_qlora_trains_only_the_adapter():
    from rl_project_b200.models.adapters.qlora import apply_qlora
    from rl_project_b200.models.quantization.nf4 import dequantize_nf4, quantize_nf4

    torch.manual_seed(0)
    w = torch.randn(64, 128)
    packed, absmax, shape = quantize_nf4(w)
    back = dequantize_nf4(packed, absmax, shape)
    assert back.shape == w.shape
    assert (back - w).abs().max() <= absmax.max() * 0.2  # within half the widest NF4 level gap
    assert (back - w).pow(2).mean() < 0.02 * w.pow(2).mean()
    m = TransformerLM(model_spec_from_preset("tiny", vocab_size=64))
    apply_qlora(m, rank=4)
    trainable = [n for n, p in m.named_parameters() if p.requires_grad]
    assert trainable and all("lora_" in n for n in trainable if ".h." in n)
    x = torch.randint(0, 64, (2, 16))
    _, loss = m(x, x)
    loss.backward()
    assert all(p.grad is not None for n, p in m.named_parameters() if p.requires_grad and "lora_" in n)


@pytest.mark.parametrize("quant", ["none", "q8_0", "q4_0"])
def test_gguf_export_reads_back(tmp_path, quant):
    from rl_project_b200.models.quantization.gguf import export_gguf, read_gguf_header, read_gguf_tensor

    spec = model_spec_from_preset("tiny", vocab_size=64)
    m = TransformerLM(spec)
    sd = m.state_dict()
    out = tmp_path / f"m_{quant}.gguf"
    export_gguf(sd, spec, out, quantize=quant)
    hdr = read_gguf_header(out)
    assert hdr["version"] == 3 and hdr["tensors"]
    name = next(t["name"] for t in hdr["tensors"] if "wte" in t["name"])
    arr = read_gguf_tensor(out, name)
    ref = sd["transformer.wte.weight"].float().numpy()
    tol = {"none": 1e-3, "q8_0": 0.02, "q4_0": 0.3}[quant]  # "none" stores matrices as F16
    assert np.abs(arr.reshape(ref.shape) - ref).max() <= tol * max(1.0, np.abs(ref).max())


def test_block_quantizers_roundtrip():
    from rl_project_b200.models.quantization.gguf import (dequantize_q4_0, dequantize_q8_0, quantize_q4_0,
                                                          quantize_q8_0)

    torch.manual_seed(0)
    t = torch.randn(4, 64)
    d8, _, n = quantize_q8_0(t)
    d4, _, n4 = quantize_q4_0(t)
    r8, r4 = dequantize_q8_0(d8, n), dequantize_q4_0(d4, n4)
    amax = t.abs().max().item()
    assert np.abs(r8 - t.reshape(-1).numpy()).max() < amax / 100
    assert np.abs(r4 - t.reshape(-1).numpy()).max() < amax / 6
