"""The fused decode step (dk_step_run): one persistent kernel per greedy token.

Its reference is the same runner's per-op kernel path (QwenRunner.forward with T == 1, which the
tests in test_runner.py pin to the reference's numerics) on the same model and cache contents:
logits within the decode tolerance at every step, the greedy pick equal to the argmax of its own
fp16 logits (ties to the lowest index, like torch.argmax), KV-cache rows within fp16 rounding of the
per-op path's, `pos` advanced and the pick recorded in the history. Sizes cover batch 1, 2 and 4,
positions that cross the 128-position attention slices, and the benchmark model (Qwen2.5-1.5B
architecture), where the greedy streams are compared for 32 tokens from a 512-token prompt.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DECODE_TOL = 5e-2  # logits: the runner tests' tolerance (tests/test_runner.py of the reference: 5e-2)


def small_model(seed=0, layers=2):
    """A random Qwen2 whose sizes the fused step takes (hidden, intermediate and n_heads * 128
    multiples of 256, head_dim 128, vocab % 32 == 0)."""
    import transformers

    cfg = transformers.Qwen2Config(
        vocab_size=4096, hidden_size=512, intermediate_size=1280, num_hidden_layers=layers,
        num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=4096,
        tie_word_embeddings=True, rms_norm_eps=1e-6, rope_parameters={"rope_theta": 10000.0, "rope_type": "default"},
    )
    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = transformers.Qwen2ForCausalLM(cfg)
    return model.half().eval()


def _pair(model, batch, max_len):
    from kernels.e2e.model import QwenRunner, make_backend

    fused = QwenRunner(model, make_backend("ours"), max_len=max_len, batch=batch, fused_step=True)
    plain = QwenRunner(model, make_backend("ours"), max_len=max_len, batch=batch)
    assert fused.step_kernel() is not None and plain.step_kernel() is None
    return fused, plain


@pytest.mark.parametrize("batch,prompt,steps", [(1, 20, 6), (2, 125, 6), (4, 250, 8), (1, 1020, 6)])
def test_step_matches_per_op_path(batch, prompt, steps):
    from kernels import _lib

    model = small_model()
    fused, plain = _pair(model, batch, max_len=1152)
    g = torch.Generator().manual_seed(batch * 1000 + prompt)
    ids = torch.randint(0, 4096, (batch, prompt), generator=g).cuda()
    positions = torch.arange(prompt, device="cuda")
    fused.forward(ids, positions)
    plain.forward(ids, positions)
    tok = ids[:, -1:].clone()
    hist = torch.full((batch, fused.max_len), -1, dtype=torch.int64, device="cuda")
    logits = torch.empty(batch, 4096, dtype=torch.float16, device="cuda")
    for i in range(steps):
        p = prompt + i  # this step's token sits at position prompt + i
        t_in = tok.clone()
        pos = torch.tensor([p], device="cuda")
        ref = plain.forward(t_in, pos.clone())[:, -1].float()
        fused.step_kernel()(tok, pos, hist, logits)
        torch.cuda.synchronize()
        torch.testing.assert_close(logits.float(), ref, atol=DECODE_TOL, rtol=DECODE_TOL)
        pick = logits.argmax(-1)
        assert torch.equal(tok.view(-1), pick), (tok.view(-1), pick)
        assert int(pos.item()) == p + 1
        assert torch.equal(hist[:, p], pick)
        # the per-op path follows the fused path's tokens (teacher forcing): same cache contents
    for c_f, c_p in ((fused.k_cache, plain.k_cache), (fused.v_cache, plain.v_cache)):
        written = c_f[:, :, :, prompt: prompt + steps].float()
        torch.testing.assert_close(written, c_p[:, :, :, prompt: prompt + steps].float(), atol=2e-2, rtol=2e-2)
    assert _lib.device_error() == 0


def test_step_in_graph_decoder_matches_eager_steps():
    from kernels.e2e.run import GraphDecoder

    model = small_model(seed=1)
    fused, plain = _pair(model, 1, max_len=512)
    ids = torch.randint(0, 4096, (1, 100), generator=torch.Generator().manual_seed(5)).cuda()
    dec = GraphDecoder(fused)
    dec.capture(ids)
    toks, _ = dec.generate(ids, 40)  # crosses the 128-position slice boundary
    eager = GraphDecoder(fused)
    eager.prefill(ids)
    for _ in range(40):
        eager._step()
    assert toks[0] == eager.out[0, 99:140].tolist()
    # host-loop API through the same graph
    dec.prefill(ids)
    t = dec.tok.cpu()
    seq = []
    for _ in range(10):
        t = dec.step_host(t).clone()
        seq.append(int(t[0, 0]))
    assert seq == toks[0][1:11]


def test_step_rejects_unsupported_runners():
    from kernels import step
    from kernels.e2e.model import QwenRunner, make_backend

    model = small_model(seed=2)
    assert step.supported(QwenRunner(model, make_backend("ours"), max_len=256, batch=8, fused_step=True)) is not None
    assert step.supported(QwenRunner(model, make_backend("ours_lm"), max_len=256, fused_step=True)) is not None
    assert step.supported(QwenRunner(model, make_backend("ours"), max_len=200, fused_step=True)) is not None
    with pytest.raises(RuntimeError, match="unavailable"):
        step.DecodeStep(QwenRunner(model, make_backend("fp16"), max_len=256, fused_step=True))


def test_step_bad_position_writes_nothing():
    """pos outside [0, max_len): the step records DK_DEVERR_BAD_POSITION, writes no token, no cache
    row and no history entry, and leaves the plan usable."""
    from kernels import _lib

    model = small_model(seed=3, layers=1)
    fused, _ = _pair(model, 1, max_len=256)
    ids = torch.randint(0, 4096, (1, 10), generator=torch.Generator().manual_seed(1)).cuda()
    fused.forward(ids, torch.arange(10, device="cuda"))
    tok = torch.tensor([[7]], device="cuda")
    pos = torch.tensor([256], device="cuda")
    hist = torch.full((1, 256), -1, dtype=torch.int64, device="cuda")
    k_before = fused.k_cache.clone()
    fused.step_kernel()(tok, pos, hist)
    assert _lib.device_error() == 3  # DK_DEVERR_BAD_POSITION
    _lib.clear_device_error()
    assert int(tok.item()) == 7 and int(pos.item()) == 256 and bool((hist == -1).all())
    assert torch.equal(k_before, fused.k_cache)
    pos.fill_(10)  # the next step runs normally
    fused.step_kernel()(tok, pos, hist)
    assert _lib.device_error() == 0 and int(pos.item()) == 11 and int(hist[0, 10]) == int(tok.item())


@pytest.mark.slow
def test_step_greedy_stream_on_benchmark_model():
    """Qwen2.5-1.5B architecture (random init, seed 0), 512-token synthetic prompt: 32 greedy tokens
    of the fused step against the per-op kernel path and against the reference numerics (w4_ref:
    dequantize, cuBLAS fp16, SDPA). The logits stay within the decode tolerance; a divergence is
    only allowed where the reference's top two logits are within twice that tolerance (a near-tie)."""
    from kernels import config
    from kernels.e2e.model import QwenRunner, make_backend, random_qwen2
    from kernels.e2e.run import greedy_parity
    from kernels.step import StepLogits

    model = random_qwen2(config.QWEN15, dtype=torch.float16, device="cuda", seed=0)
    ids = torch.randint(0, config.QWEN15["vocab_size"], (1, 512), generator=torch.Generator().manual_seed(1)).cuda()

    fused = QwenRunner(model, make_backend("ours"), max_len=2048, fused_step=True)
    assert fused.step_kernel() is not None
    for ref_name in ("ours", "w4_ref"):
        ref = QwenRunner(model, make_backend(ref_name), max_len=2048)
        fused.k_cache.zero_()
        fused.v_cache.zero_()
        r = greedy_parity(StepLogits(fused), ref, ids, steps=32)
        tol = DECODE_TOL + DECODE_TOL * r["max_abs_ref_logit"]
        assert r["max_abs_logit_diff"] <= tol, (ref_name, r)
        if r["first_divergence"] < 32:
            assert r["ref_margin_at_divergence"] <= 2 * tol, (ref_name, r)
        del ref
        torch.cuda.empty_cache()
