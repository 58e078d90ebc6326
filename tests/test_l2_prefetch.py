"""The L2_PREFETCH config key (dk_matmul_config.l2_prefetch_*): a launch pulls byte ranges into L2
for a later launch. It is a hint, so every output must be bit-identical with and without it."""

import pytest
import torch

from _util import to_cuda, w4_case


def test_config_rejects_bad_prefetch_lists():
    from kernels import _lib
    from kernels.w4a16 import _config

    c = _config({"L2_PREFETCH": []})
    assert c.n_prefetch == 0
    with pytest.raises(ValueError, match="at most"):
        _config({"L2_PREFETCH": [torch.zeros(1)] * (_lib.MAX_L2_PREFETCH + 1)})
    with pytest.raises(RuntimeError, match="CUDA"):
        _config({"L2_PREFETCH": [torch.zeros(4)]})


def test_runner_prefetch_plan():
    """Projection j pulls projection j+2 of the decode chain (the first also pulls j+1)."""
    from kernels.e2e.model import Linear, QwenRunner

    chain = [Linear(qweight=torch.zeros(1) + i, scales=torch.zeros(1), zeros=torch.zeros(1)) for i in range(8)]

    class FakeLayer:
        def __init__(self, ps):
            self.qkv, self.o, self.gate_up, self.down = ps

    r = QwenRunner.__new__(QwenRunner)
    r.layers = [FakeLayer(chain[:4]), FakeLayer(chain[4:])]
    r._plan_l2_prefetch()
    assert [t.item() for t in chain[0].l2_next[::3]] == [2, 1]
    for j in range(1, 6):
        assert chain[j].l2_next[0] is chain[j + 2].qweight and len(chain[j].l2_next) == 3
    assert chain[6].l2_next is None and chain[7].l2_next is None


@pytest.mark.gpu
def test_prefetch_changes_no_result():
    from kernels.fp8 import quantize_fp8, w8a16_matmul
    from kernels.w4a16 import w4a16_matmul, w4a16_rmsnorm_matmul, w4a16_swiglu

    x, qw, s, z, b = w4_case(3, 1024, 1536, seed=3, bias=True)
    xc, qc, sc, zc, bc = to_cuda(x, qw, s, z, b)
    other = torch.randn(5_000_003, device="cuda")  # odd byte count: trimmed to 16-byte boundaries
    odd_view = other.view(torch.uint8)[3:1_000_000]  # unaligned start
    pf = [other, odd_view, qc, torch.empty(0, device="cuda")]
    for base in ({}, {"STATIC_WEIGHTS": True}, {"SPLIT_K": 4}):
        ref = w4a16_matmul(xc, qc, sc, zc, bias=bc, config=base or None)
        got = w4a16_matmul(xc, qc, sc, zc, bias=bc, config={**base, "L2_PREFETCH": pf})
        assert torch.equal(ref, got)
    ref = w4a16_swiglu(xc, qc, sc, zc)
    assert torch.equal(ref, w4a16_swiglu(xc, qc, sc, zc, config={"L2_PREFETCH": pf}))
    w = torch.ones(1536, device="cuda", dtype=torch.float16)
    r = torch.randn(3, 1536, device="cuda", dtype=torch.float16)
    y0, r0 = w4a16_rmsnorm_matmul(xc, w, 1e-6, r, qc, sc, zc, swiglu=True)
    y1, r1 = w4a16_rmsnorm_matmul(xc, w, 1e-6, r, qc, sc, zc, swiglu=True, config={"L2_PREFETCH": pf})
    assert torch.equal(y0, y1) and torch.equal(r0, r1)
    wq, ws = quantize_fp8(torch.randn(1024, 1536, device="cuda", dtype=torch.float16) * 0.02)
    ref = w8a16_matmul(xc, wq, ws)
    assert torch.equal(ref, w8a16_matmul(xc, wq, ws, config={"L2_PREFETCH": [other, wq]}))
    # M > 16 runs per 16-row block, the ranges go with the first block only
    x2 = torch.randn(40, 1536, device="cuda", dtype=torch.float16)
    assert torch.equal(w4a16_matmul(x2, qc, sc, zc), w4a16_matmul(x2, qc, sc, zc, config={"L2_PREFETCH": pf}))
    from kernels import _lib
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
