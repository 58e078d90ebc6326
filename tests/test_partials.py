"""Split-K partial sums handed from one decode GEMV to the next (dk_w4a16_matmul_partials,
dk_w4a16_rmsnorm_matmul_partials).

The pair must compute exactly what the reduced path computes - w4a16_matmul (whose cluster reduction
adds the same partial sums in the same order) followed by w4a16_rmsnorm_matmul - bit for bit, and
the partial sums must add up to the oracle's product within the matmul tolerance. The runner's
one-row decode step uses the pair between every down_proj and the next layer's norm + qkv, so its
logits must match the step without it bit for bit as well.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,H,I,with_bias", [(1, 1536, 8960, False), (2, 1536, 8960, True), (1, 512, 1280, False),
                                             (16, 896, 4864, True), (3, 2048, 11008, False)])
def test_partials_pair_equals_reduced_path(M, H, I, with_bias):
    from _util import MATMUL_TOL, to_cuda, w4_case, w4_ref
    from kernels.w4a16 import w4a16_matmul, w4a16_matmul_partials, w4a16_rmsnorm_matmul, w4a16_rmsnorm_matmul_partials

    # the producer: down-shaped [M, I] x [I, H]
    x, qw, s, z, b = w4_case(M, H, I, seed=M + H, bias=with_bias)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    bc = to_cuda(b)[0] if with_bias else None
    cfg = {"STATIC_WEIGHTS": True}
    parts = w4a16_matmul_partials(xc, qc, sc, zc, config=cfg)
    assert parts.dim() == 3 and parts.shape[1:] == (M, H) and 1 <= parts.shape[0] <= 8
    full = parts.sum(0) + (bc.float() if with_bias else 0)
    ref = w4_ref(x, qw, s, z, b if with_bias else None)
    torch.testing.assert_close(full.cpu(), torch.as_tensor(ref).float(), **MATMUL_TOL)
    # the reduced path on the same kernel (the decode GEMV; 9-16 rows with a long K would otherwise take
    # the tcgen05 small-M kernel) and with the norm inside the projection
    y_reduced = w4a16_matmul(xc, qc, sc, zc, bias=bc, config={**cfg, "DECODE_GEMV": True})
    # the consumer: residual + RMSNorm + a qkv-shaped projection [M, H] x [H, N]
    N = 2048
    _, qw2, s2, z2, b2 = w4_case(M, N, H, seed=7, bias=True)
    qc2, sc2, zc2, bc2 = to_cuda(qw2, s2, z2, b2)
    res = torch.randn(M, H, device="cuda").half()
    nw = (1 + 0.05 * torch.randn(H, device="cuda")).half()
    y1, r1 = w4a16_rmsnorm_matmul(y_reduced, nw, 1e-6, res, qc2, sc2, zc2, bias=bc2, config={**cfg, "FUSED_NORM": True})
    y2, r2 = w4a16_rmsnorm_matmul_partials(parts, bc, nw, 1e-6, res, qc2, sc2, zc2, bias=bc2, config=cfg)
    assert torch.equal(r1, r2.view(r1.shape))
    assert torch.equal(y1, y2.view(y1.shape))
    # SwiGLU form of the consumer
    _, qw3, s3, z3, _ = w4_case(M, 2 * 1280, H, seed=9)
    qc3, sc3, zc3 = to_cuda(qw3, s3, z3)
    g1, _ = w4a16_rmsnorm_matmul(y_reduced, nw, 1e-6, None, qc3, sc3, zc3, swiglu=True, config={**cfg, "FUSED_NORM": True})
    g2, _ = w4a16_rmsnorm_matmul_partials(parts, bc, nw, 1e-6, None, qc3, sc3, zc3, swiglu=True, config=cfg)
    assert torch.equal(g1, g2.view(g1.shape))
    from kernels import _lib

    assert _lib.device_error() == 0


def test_runner_step_with_partials_is_bit_identical():
    """The one-row decode step hands down_proj's partial sums to the next layer; turning that off
    (the reduced down_proj output instead) must not change a single logit bit."""
    import transformers
    from kernels.e2e.model import QwenRunner, make_backend

    cfg = transformers.Qwen2Config(
        vocab_size=4096, hidden_size=512, intermediate_size=1280, num_hidden_layers=3, num_attention_heads=4,
        num_key_value_heads=2, head_dim=128, max_position_embeddings=4096, tie_word_embeddings=True,
        rms_norm_eps=1e-6, rope_parameters={"rope_theta": 10000.0, "rope_type": "default"})
    torch.manual_seed(5)
    with torch.device("cuda"):
        model = transformers.Qwen2ForCausalLM(cfg).half().eval()
    ids = torch.randint(0, 4096, (1, 30), generator=torch.Generator().manual_seed(3)).cuda()
    outs = []
    for use in (True, False):
        be = make_backend("ours")
        if not use:
            class Reduced(type(be)):
                partials = False

            be.__class__ = Reduced
        r = QwenRunner(model, be, max_len=256)
        r.forward(ids, torch.arange(30, device="cuda"))
        tok = ids[:, -1:]
        step = []
        for i in range(4):
            logits = r.forward(tok, torch.tensor([30 + i], device="cuda"))
            step.append(logits.clone())
            tok = logits[:, -1].argmax(-1, keepdim=True)
        outs.append(torch.stack(step))
    assert torch.equal(outs[0], outs[1])
