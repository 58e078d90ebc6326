"""Pins the CPU oracle runner (used for the CPU baseline) to the reference's own runner: the
golden logits of the reference's w4_ref backend on the tiny random Qwen2."""

import numpy as np
import pytest
import torch

pytest.importorskip("transformers")

from oracle.runner import OracleRunner, weights_from_hf  # noqa: E402
from tests_golden_model import tiny_model, weights_digest  # noqa: E402


@pytest.mark.parametrize("name,quant_lm", [("w4_ref", False), ("w4_ref_lm", True)])
def test_oracle_runner_matches_reference_w4_ref(golden, name, quant_lm):
    g = golden("runner")
    model = tiny_model(torch.float16, "cpu")
    assert weights_digest(model) == str(g["runner_digest16"])
    cfg = model.config
    r = OracleRunner(weights_from_hf(model, quantized=True, quant_lm_head=quant_lm), cfg.num_attention_heads,
                     cfg.num_key_value_heads, cfg.hidden_size // cfg.num_attention_heads, cfg.rms_norm_eps,
                     cfg.rope_parameters["rope_theta"], max_len=32)
    ids = g["runner_ids"][0, :5]
    logits = np.stack([r.step(int(t), p).numpy() for p, t in enumerate(ids)])
    np.testing.assert_allclose(logits, g[f"runner_{name}_logits"][0].astype(np.float32), atol=5e-2, rtol=5e-2)


def test_oracle_runner_fp32_matches_hf():
    g_model = tiny_model(torch.float32, "cpu")
    cfg = g_model.config
    r = OracleRunner(weights_from_hf(g_model, quantized=False), cfg.num_attention_heads, cfg.num_key_value_heads,
                     cfg.hidden_size // cfg.num_attention_heads, cfg.rms_norm_eps, cfg.rope_parameters["rope_theta"],
                     max_len=32)
    ids = torch.randint(0, 512, (1, 7))
    with torch.no_grad():
        ref = g_model(ids).logits[0].numpy()
    logits = np.stack([r.step(int(t), p).numpy() for p, t in enumerate(ids[0])])
    np.testing.assert_allclose(logits, ref, atol=1e-3, rtol=1e-3)  # fp32, different op order
