"""Decode attention for one new token per sequence (the T == 1 case of the reference runner's
RoPE + KV-cache append + SDPA, kernels/e2e/model.py:236-244): one libdecodek kernel that reads only
the cached positions 0..pos instead of the whole max_len cache."""

from __future__ import annotations

import torch

from kernels import _lib


def decode_attention(qkv, k_cache, v_cache, pos, cos, sin, n_heads, n_kv, splits=0, static_cache=False):
    """qkv [B, 1, (nq + 2 nkv) * hd] fp16; k_cache, v_cache [B, nkv, max_len, hd] fp16 (updated
    in place at `pos`); pos int64 [1] (device); cos, sin [1, hd] fp16 for this position, or tables
    [positions, hd] from which the kernel takes row `pos`. Returns [B, 1, nq * hd].
    static_cache: the cache and `pos` were not written by the kernel just before this one (true
    inside a decode step), so the kernel fetches its cache slice before waiting for that kernel."""
    B, T, width = qkv.shape
    hd = k_cache.shape[-1]
    max_len = k_cache.shape[-2]
    _lib.require_extent(T == 1 and width == (n_heads + 2 * n_kv) * hd,
                        "decode_attention: qkv must be [B, 1, (n_heads + 2 n_kv) * head_dim]")
    _lib.require_extent(tuple(k_cache.shape) == (B, n_kv, max_len, hd) and v_cache.shape == k_cache.shape,
                        "decode_attention: k_cache and v_cache must be [B, n_kv, max_len, head_dim]")
    _lib.require_extent(pos.numel() >= 1, "decode_attention: pos holds the position")
    _lib.require_cuda("decode_attention", qkv, k_cache, v_cache, pos, cos, sin)
    _lib.require_dtype("decode_attention", torch.float16, qkv, k_cache, v_cache, cos, sin)
    _lib.require_dtype("decode_attention", torch.int64, pos)
    _lib.require_extent(k_cache.is_contiguous() and v_cache.is_contiguous(), "decode_attention: caches must be contiguous")
    qkv = qkv.contiguous()
    out = torch.empty((B, 1, n_heads * hd), dtype=qkv.dtype, device=qkv.device)
    cos, sin = cos.contiguous(), sin.contiguous()
    _lib.require_extent(cos.shape == sin.shape and cos.shape[-1] == hd, "decode_attention: cos and sin must be [.., head_dim]")
    if cos.shape[0] > 1 and cos.shape[0] < max_len:
        raise RuntimeError("decode_attention: a RoPE table needs at least max_len rows")
    stride = hd if cos.shape[0] > 1 else 0
    _lib.call("dk_decode_attention", _lib.ptr(qkv), _lib.ptr(k_cache), _lib.ptr(v_cache), _lib.ptr(pos),
              _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(out), B, n_heads, n_kv, hd, max_len, stride, splits,
              1 if static_cache else 0, _lib.stream_of(qkv))
    return out
