"""The tiny random Qwen2 of the reference's tests/test_runner.py:15-23 (also used by the golden
fixture generator) and a digest of its weights."""

import hashlib

import torch


def tiny_model(dtype, device):
    import transformers

    cfg = transformers.Qwen2Config(
        vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
        tie_word_embeddings=True, rms_norm_eps=1e-6,
    )
    torch.manual_seed(0)
    return transformers.Qwen2ForCausalLM(cfg).to(device=device, dtype=dtype).eval()


def weights_digest(model) -> str:
    h = hashlib.sha256()
    for name, t in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(t.detach().float().cpu().numpy().tobytes())
    return h.hexdigest()
