"""The lm_head + greedy-pick kernel (dk_lm_head_greedy) and the embedding kernel (dk_embed_tokens).

The lm_head's reference is the reference runner's tail for T == 1 (kernels/e2e/model.py:248-253:
residual add + RMSNorm with the rounding of kernels/rmsnorm.py, then F.linear with the fp16 lm_head)
and its graph decoder's bookkeeping (kernels/e2e/run.py:69-74). Logits are compared with an fp32
matmul of the same normalized rows within fp16 rounding; the pick must be exactly the first maximum
of the kernel's own fp16 logits, and the reference's argmax wherever the reference's top two logits
are further apart than the tolerance. The embedding kernel must equal F.embedding bit for bit.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2  # fp16 logits of ~|10|: one fp16 ulp is 2**-7 there, plus fp32 summation order


def rmsnorm_fp16(x, res, w, eps):
    """kernels/rmsnorm.py:28-37: h = x + res (fp16), var in fp32, w * fp16(h / sqrt(var + eps))."""
    h = x + res if res is not None else x
    hf = h.float()
    inv = 1.0 / torch.sqrt(hf.pow(2).mean(-1, keepdim=True) + eps)
    return w * (hf * inv).half()


def case(M, V, H, seed, dev="cuda"):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, H, generator=g, device=dev).half()
    res = torch.randn(M, H, generator=g, device=dev).half()
    w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).half()
    W = (torch.randn(V, H, generator=g, device=dev) * 0.05).half()
    return x, res, w, W


def check_picks(picks, logits, ref_logits):
    """picks == first max of our logits; == the reference's argmax unless its top-2 is a near-tie."""
    assert torch.equal(picks.view(-1), logits.float().argmax(-1))
    top = ref_logits.topk(2, dim=-1).values
    clear = (top[:, 0] - top[:, 1]) > 2 * LOGIT_TOL
    assert torch.equal(picks.view(-1)[clear], ref_logits.argmax(-1)[clear])


@pytest.mark.parametrize("M,V,H", [(1, 151936, 1536), (2, 4099, 512), (3, 32000, 3584), (4, 1000, 1536),
                                   (8, 5003, 896), (1, 17, 64)])
def test_lm_head_greedy_matches_norm_then_matmul(M, V, H):
    from kernels import _lib, head

    x, res, w, W = case(M, V, H, seed=M * 7 + V)
    ws = head.workspace("cuda")
    tok = torch.full((M,), -1, dtype=torch.int64, device="cuda")
    logits = torch.empty(M, V, dtype=torch.float16, device="cuda")
    head.lm_head_greedy(x, res, w, 1e-6, W, tok, ws, logits=logits)
    torch.cuda.synchronize()
    ref = rmsnorm_fp16(x, res, w, 1e-6).float() @ W.float().t()
    torch.testing.assert_close(logits.float(), ref, atol=LOGIT_TOL, rtol=LOGIT_TOL)
    check_picks(tok, logits, ref)
    # a second call on the same workspace (its counter was left at zero) gives the same picks
    tok2 = torch.full((M,), -1, dtype=torch.int64, device="cuda")
    head.lm_head_greedy(x, res, w, 1e-6, W, tok2, ws)
    torch.cuda.synchronize()
    assert torch.equal(tok, tok2)
    assert _lib.device_error() == 0


def test_lm_head_greedy_without_norm_and_ties():
    """No residual, no norm: plain x @ W^T. Rows with equal logits pick the lowest index."""
    from kernels import head

    M, V, H = 2, 3000, 256
    x, _, _, W = case(M, V, H, seed=3)
    W[7] = 0.2  # rows 7 and 2500 are equal and, for positive inputs, the maxima of both rows
    W[2500] = 0.2
    x = x.abs()
    ws = head.workspace("cuda")
    tok = torch.empty(M, dtype=torch.int64, device="cuda")
    logits = torch.empty(M, V, dtype=torch.float16, device="cuda")
    head.lm_head_greedy(x, None, None, 1e-6, W, tok, ws, logits=logits)
    torch.cuda.synchronize()
    ref = x.float() @ W.float().t()
    torch.testing.assert_close(logits.float(), ref, atol=LOGIT_TOL, rtol=LOGIT_TOL)
    assert tok.tolist() == [7, 7]


def test_lm_head_greedy_bookkeeping():
    """history[:, pos] = picks, pos += 1; a position outside the history writes nothing there,
    leaves pos and records DK_DEVERR_BAD_POSITION."""
    from kernels import _lib, head

    M, V, H, L = 4, 2048, 512, 64
    x, res, w, W = case(M, V, H, seed=11)
    ws = head.workspace("cuda")
    tok = torch.zeros(M, 1, dtype=torch.int64, device="cuda")
    hist = torch.full((M, L), -1, dtype=torch.int64, device="cuda")
    pos = torch.tensor([5], device="cuda")
    head.lm_head_greedy(x, res, w, 1e-6, W, tok, ws, pos=pos, history=hist)
    torch.cuda.synchronize()
    ref = rmsnorm_fp16(x, res, w, 1e-6).float() @ W.float().t()
    assert int(pos.item()) == 6
    assert torch.equal(hist[:, 5], tok.view(-1))
    assert bool((hist[:, :5] == -1).all()) and bool((hist[:, 6:] == -1).all())
    top = ref.topk(2, dim=-1).values
    clear = (top[:, 0] - top[:, 1]) > 2 * LOGIT_TOL
    assert torch.equal(tok.view(-1)[clear], ref.argmax(-1)[clear])
    pos.fill_(L)
    head.lm_head_greedy(x, res, w, 1e-6, W, tok, ws, pos=pos, history=hist)
    assert _lib.device_error() == 3  # DK_DEVERR_BAD_POSITION
    _lib.clear_device_error()
    assert int(pos.item()) == L and int((hist != -1).sum()) == M
    pos.fill_(0)  # the workspace is still consistent: the next call works
    head.lm_head_greedy(x, res, w, 1e-6, W, tok, ws, pos=pos, history=hist)
    assert _lib.device_error() == 0 and int(pos.item()) == 1 and torch.equal(hist[:, 0], hist[:, 5])


def test_lm_head_greedy_rejects():
    from kernels import _lib, head

    x, res, w, W = case(1, 100, 64, seed=1)
    ws = head.workspace("cuda")
    tok = torch.empty(9, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        head.lm_head_greedy(torch.zeros(9, 64, dtype=torch.float16, device="cuda"), None, None, 1e-6, W, tok, ws)
    with pytest.raises(RuntimeError, match="workspace"):
        _lib.call("dk_lm_head_greedy", _lib.ptr(x), None, None, 1e-6, _lib.ptr(W), 100, 64, 1, _lib.ptr(tok), None,
                  None, 0, 0, None, _lib.ptr(ws), 16, _lib.stream_of(x))
    with pytest.raises(RuntimeError, match="aligned"):
        _lib.call("dk_lm_head_greedy", _lib.ptr(x[:, 1:]), None, None, 1e-6, _lib.ptr(W), 100, 64, 1, _lib.ptr(tok),
                  None, None, 0, 0, None, _lib.ptr(ws), ws.numel(), _lib.stream_of(x))


def test_embed_tokens_matches_embedding():
    from kernels import _lib, head

    E = torch.randn(5000, 1536, device="cuda").half()
    t = torch.randint(0, 5000, (4, 1), device="cuda")
    assert torch.equal(head.embed_tokens(t, E), F.embedding(t, E))
    bad = torch.tensor([[3], [5000]], device="cuda")
    out = head.embed_tokens(bad, E)
    assert _lib.device_error() == 6  # DK_DEVERR_BAD_TOKEN: row 0 instead
    _lib.clear_device_error()
    assert torch.equal(out[0, 0], E[3]) and torch.equal(out[1, 0], E[0])


def test_per_op_greedy_step_uses_the_kernels_and_matches_forward():
    """QwenRunner.greedy_step on the kernel backend (embedding kernel, the layers, the lm_head +
    greedy-pick kernel) against forward() + argmax (cuBLAS lm_head) for a few steps, eager and in the
    graph decoder."""
    from kernels.e2e.model import QwenRunner, make_backend
    from kernels.e2e.run import GraphDecoder, greedy_parity
    from kernels.head import KernelHeadLogits

    import transformers

    cfg = transformers.Qwen2Config(
        vocab_size=4096, hidden_size=512, intermediate_size=1280, num_hidden_layers=2, num_attention_heads=4,
        num_key_value_heads=2, head_dim=128, max_position_embeddings=4096, tie_word_embeddings=True,
        rms_norm_eps=1e-6, rope_parameters={"rope_theta": 10000.0, "rope_type": "default"})
    torch.manual_seed(4)
    with torch.device("cuda"):
        model = transformers.Qwen2ForCausalLM(cfg).half().eval()
    r = QwenRunner(model, make_backend("ours"), max_len=512)
    assert r._kernel_head() and r.step_kernel() is None
    ref = QwenRunner(model, make_backend("ours"), max_len=512)
    ids = torch.randint(0, 4096, (1, 40), generator=torch.Generator().manual_seed(2)).cuda()
    p = greedy_parity(KernelHeadLogits(r), ref, ids, steps=16)
    assert p["max_abs_logit_diff"] <= 5e-2, p
    dec = GraphDecoder(r)
    dec.capture(ids)
    toks, _ = dec.generate(ids, 16)
    if p["first_divergence"] == 16:
        assert toks[0][:16] == p["tokens"][:16]
