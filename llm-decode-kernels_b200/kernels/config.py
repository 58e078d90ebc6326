"""Constants of the decode path: the quantization group, the benchmark layer shapes, the models
of the benchmark configs, and the B200 roofline peaks.

The peaks come from `MEASURED_PEAKS.json` at the repository root when a measurement is present
(copy bandwidth and cuBLAS bf16 throughput measured on this pool's B200s); otherwise the fallback
figures below (an earlier measurement on the same pool) are used and reported as such.
"""

from __future__ import annotations

import json
from pathlib import Path

GROUP_SIZE = 128  # reference kernels/config.py:59

# (label, N, K): Qwen2.5-1.5B linears with qkv and gate_up fused (reference kernels/config.py:71-74
# has the first four), plus the lm_head the reference never benchmarked.
QWEN15_SHAPES = [
    ("qkv", 2048, 1536), ("o_proj", 1536, 1536), ("gate_up", 17920, 1536),
    ("down", 1536, 8960), ("lm_head", 151936, 1536),
]
QWEN7_SHAPES = [
    ("qkv", 4608, 3584), ("o_proj", 3584, 3584), ("gate_up", 37888, 3584),
    ("down", 3584, 18944), ("lm_head", 152064, 3584),
]

QWEN15 = dict(vocab_size=151936, hidden_size=1536, intermediate_size=8960, num_hidden_layers=28,
              num_attention_heads=12, num_key_value_heads=2, head_dim=128, tie_word_embeddings=True,
              rms_norm_eps=1e-6, rope_theta=1000000.0, max_position_embeddings=32768)
QWEN7 = dict(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
             num_attention_heads=28, num_key_value_heads=4, head_dim=128, tie_word_embeddings=False,
             rms_norm_eps=1e-6, rope_theta=1000000.0, max_position_embeddings=32768)

_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> dict:
    """{'hbm_gbs', 'bf16_tflops', 'bf16_tflops_sustained', 'source'}."""
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {**_FALLBACK, "source": "fallback"}
