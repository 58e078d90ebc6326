"""Float references of the decode hot path, restated in numpy. TEST INFRASTRUCTURE ONLY.

Each function restates the reference's PyTorch code (file:line) with the same rounding steps:
numpy float16 arithmetic rounds every op to fp16 (computed through fp32, which is exact enough
that the double rounding is innocuous), exactly like torch's fp16 CPU ops.
"""

from __future__ import annotations

import numpy as np

from oracle import dequantize_fp8, dequantize_int4


def w4a16_ref(x, qweight, scales, zeros, group_size=128, bias=None) -> np.ndarray:
    """fp32 [M, N] = fp32(x) @ fp32(dequant(W)).T (+ fp32(bias)) (kernels/reference.py:39-45)."""
    w = dequantize_int4(qweight, scales, zeros, group_size).astype(np.float32)
    out = np.asarray(x, dtype=np.float16).astype(np.float32) @ w.T
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float16).astype(np.float32)
    return out


def w8a16_ref(x, wq, scale, bias=None) -> np.ndarray:
    """fp32 [M, N] = fp32(x) @ fp32(dequantize_fp8(wq, s)).T (+ bias) (tests/test_fp8.py:18-20,
    dequantization per kernels/fp8.py:33-35)."""
    w = dequantize_fp8(wq, scale).astype(np.float32)
    out = np.asarray(x, dtype=np.float16).astype(np.float32) @ w.T
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float16).astype(np.float32)
    return out


def rmsnorm_ref(x, weight, eps=1e-6, residual=None):
    """Qwen2RMSNorm with the optional fused residual add (kernels/reference.py:9-19).

    x = x + residual in fp16; var = mean(x^2) in fp32; out = w * fp16(x * rsqrt(var + eps)),
    the last product in fp16. Returns `out` or `(out, x + residual)`."""
    x = np.asarray(x, dtype=np.float16)
    if residual is not None:
        x = x + np.asarray(residual, dtype=np.float16)
    h = x.astype(np.float32)
    var = (h * h).mean(-1, keepdims=True, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    out = np.asarray(weight, dtype=np.float16) * (h * inv).astype(np.float16)
    return out if residual is None else (out, x)


def swiglu_ref(gate, up) -> np.ndarray:
    """fp16(silu(fp32(gate))) * up in fp16, like F.silu(gate) * up (kernels/reference.py:22-24)."""
    g = np.asarray(gate, dtype=np.float16).astype(np.float32)
    with np.errstate(over="ignore"):
        act = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float16)
    return act * np.asarray(up, dtype=np.float16)


def rope_ref(x, cos, sin):
    """x * cos + cat(-x2, x1) * sin in fp16, one rounding per op (kernels/e2e/model.py:212-214).
    x [..., hd] fp16; cos, sin [hd] fp16."""
    x = np.asarray(x, dtype=np.float16)
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return (x * cos) + (rot * sin)


def rope_tables(pos: int, head_dim: int, theta: float):
    """cos, sin fp16 [hd] for one position, as the runner computes them in fp32 and rounds
    (kernels/e2e/model.py:166, 222-224)."""
    inv = (1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))).astype(np.float32)
    f = np.float32(pos) * inv
    emb = np.concatenate([f, f]).astype(np.float32)
    return np.cos(emb).astype(np.float16), np.sin(emb).astype(np.float16)


def decode_attention_ref(qkv, k_cache, v_cache, pos, cos, sin, nq, nkv):
    """One new token per sequence: RoPE on q, k; append k, v at `pos`; softmax attention over
    positions 0..pos in fp32 (kernels/e2e/model.py:236-244 with T == 1).
    qkv [B, (nq+2nkv)*hd] fp16; caches [B, nkv, max_len, hd] fp16 (updated in place).
    Returns out [B, nq*hd] fp32."""
    B = qkv.shape[0]
    hd = k_cache.shape[-1]
    G = nq // nkv
    out = np.zeros((B, nq * hd), dtype=np.float32)
    for b in range(B):
        row = qkv[b]
        q = row[: nq * hd].reshape(nq, hd)
        k = row[nq * hd:(nq + nkv) * hd].reshape(nkv, hd)
        v = row[(nq + nkv) * hd:].reshape(nkv, hd)
        q = rope_ref(q, cos, sin)
        k = rope_ref(k, cos, sin)
        k_cache[b, :, pos] = k
        v_cache[b, :, pos] = v
        for hq in range(nq):
            hk = hq // G
            K = k_cache[b, hk, : pos + 1].astype(np.float32)
            V = v_cache[b, hk, : pos + 1].astype(np.float32)
            s = K @ q[hq].astype(np.float32) / np.float32(np.sqrt(hd))
            s = np.exp(s - s.max())
            out[b, hq * hd:(hq + 1) * hd] = (s / s.sum()) @ V
    return out
