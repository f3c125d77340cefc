"""Quantisation: NF4 (QLoRA base weights, dequantised on sm_100a) and GGUF export."""

from rl_project_b200.models.quantization.gguf import export_gguf, read_gguf_header, read_gguf_tensor
from rl_project_b200.models.quantization.nf4 import (NF4_BLOCK_SIZE, NF4_TABLE, NF4Linear, dequantize_nf4,
                                                     quantization_report, quantize_nf4)
