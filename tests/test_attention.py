"""Decode attention (kernels.attention.decode_attention, C-ABI dk_decode_attention) vs the oracle's
restatement of the runner's RoPE + cache append + SDPA for one token: RoPE'd k/v appended to the
cache bit-exactly, attention output within 2e-3 (fp32 softmax, different summation order)."""

import numpy as np
import pytest
import torch

from _util import bits16
from oracle import ref

pytestmark = pytest.mark.gpu


def _case(B, nq, nkv, max_len, pos, seed=0, hd=128, theta=1e6):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(B, (nq + 2 * nkv) * hd, generator=g).half().numpy()
    kc = torch.randn(B, nkv, max_len, hd, generator=g).half().numpy()
    vc = torch.randn(B, nkv, max_len, hd, generator=g).half().numpy()
    cos, sin = ref.rope_tables(pos, hd, theta)
    return qkv, kc, vc, cos, sin


@pytest.mark.parametrize("B,nq,nkv,max_len,pos,splits", [
    (1, 12, 2, 2048, 0, 0), (1, 12, 2, 2048, 511, 0), (1, 12, 2, 2048, 767, 0), (1, 12, 2, 2048, 2047, 0),
    (16, 12, 2, 1024, 300, 0), (1, 28, 4, 1024, 777, 0), (2, 8, 8, 64, 33, 3), (1, 4, 2, 96, 95, 1),
    (3, 12, 2, 512, 200, 8),
    # tensor-parallel shards of Qwen2.5-7B (28 query / 4 kv heads): 14/2 at 2 ranks, 7/1 at 4, 3/1 and 4/1 at 8
    (1, 14, 2, 2048, 1100, 0), (8, 7, 1, 2048, 1030, 0), (1, 3, 1, 2048, 1024, 0), (32, 4, 1, 2048, 1025, 0),
    (2, 5, 1, 128, 70, 0),
])
def test_decode_attention(B, nq, nkv, max_len, pos, splits):
    from kernels.attention import decode_attention

    qkv, kc, vc, cos, sin = _case(B, nq, nkv, max_len, pos)
    kc_t, vc_t = torch.from_numpy(kc.copy()).cuda(), torch.from_numpy(vc.copy()).cuda()
    out = decode_attention(torch.from_numpy(qkv).cuda().view(B, 1, -1), kc_t, vc_t,
                           torch.tensor([pos], device="cuda"), torch.from_numpy(cos).cuda().view(1, -1),
                           torch.from_numpy(sin).cuda().view(1, -1), nq, nkv, splits=splits)
    exp = ref.decode_attention_ref(qkv, kc, vc, pos, cos, sin, nq, nkv)
    assert np.array_equal(bits16(kc_t[:, :, pos]), bits16(kc[:, :, pos]))  # RoPE'd k, bit-exact
    assert np.array_equal(bits16(vc_t[:, :, pos]), bits16(vc[:, :, pos]))
    assert np.array_equal(bits16(kc_t), bits16(kc))  # nothing else in the cache changed
    np.testing.assert_allclose(out.view(B, -1).float().cpu().numpy(), exp, rtol=1e-2, atol=2e-3)


def test_bad_position_sets_device_error_and_writes_nothing():
    from kernels import _lib
    from kernels.attention import decode_attention

    qkv, kc, vc, cos, sin = _case(1, 12, 2, 64, 0)
    kc_t = torch.from_numpy(kc.copy()).cuda()
    _lib.clear_device_error()
    decode_attention(torch.from_numpy(qkv).cuda().view(1, 1, -1), kc_t, torch.from_numpy(vc).cuda(),
                     torch.tensor([64], device="cuda"), torch.from_numpy(cos).cuda().view(1, -1),
                     torch.from_numpy(sin).cuda().view(1, -1), 12, 2)
    assert _lib.device_error() == 3  # DK_DEVERR_BAD_POSITION
    _lib.clear_device_error()
    assert np.array_equal(bits16(kc_t), bits16(kc))


def test_rope_table_lookup_matches_per_position():
    """cos/sin passed as [positions, hd] tables: the kernel takes row `pos` - same result as
    passing that row."""
    from kernels.attention import decode_attention

    B, nq, nkv, max_len, pos = 1, 12, 2, 256, 100
    qkv, kc, vc, cos, sin = _case(B, nq, nkv, max_len, pos)
    tab_c = torch.zeros(max_len, 128, dtype=torch.float16)
    tab_s = torch.zeros(max_len, 128, dtype=torch.float16)
    tab_c[pos] = torch.from_numpy(cos)
    tab_s[pos] = torch.from_numpy(sin)
    args = (torch.from_numpy(qkv).cuda().view(B, 1, -1),)
    p = torch.tensor([pos], device="cuda")
    o1 = decode_attention(*args, torch.from_numpy(kc.copy()).cuda(), torch.from_numpy(vc.copy()).cuda(), p,
                          torch.from_numpy(cos).cuda().view(1, -1), torch.from_numpy(sin).cuda().view(1, -1), nq, nkv)
    o2 = decode_attention(*args, torch.from_numpy(kc.copy()).cuda(), torch.from_numpy(vc.copy()).cuda(), p,
                          tab_c.cuda(), tab_s.cuda(), nq, nkv)
    assert torch.equal(o1, o2)
