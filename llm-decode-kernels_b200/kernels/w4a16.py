"""W4A16 matmul: y = x @ dequant(W).T (+ bias), int4 weights, fp16 activations, fp32 accumulation.

Same entry point and weight format as the reference's kernels/w4a16.py:301-330. The Triton paths
(direct / split-K GEMM, GEMV, timed per-shape picker) are replaced by libdecodek's sm_100a kernel,
which chooses its column tile and cluster split-K from a static cost model - no timing runs inside
the first call, so the first call may happen under CUDA-graph capture.

`config` keeps the reference's Triton-style dict: `SPLIT_K` maps to the cluster split-K factor
(clamped to what K allows), `BLOCK_N` (32, 64, 128 or 256; other values mean automatic) to the
column tile of a CTA; other Triton tiling keys (BLOCK_M, BLOCK_K, GROUP_M, GEMV) have no meaning
here and are accepted and ignored. `FACTORED` keeps the reference's meaning: the decode kernel
computes s * sum(x * (q - z)) per group in fp32 by default (the reference's FACTORED numerics);
`FACTORED=False` (or `EXACT=True`) rounds every dequantized weight to fp16 first, exactly like the
reference's dequantize-then-matmul. Extra keys: `STATIC_WEIGHTS` (the weights are constant, so the
kernel may prefetch them before the previous kernel finishes), `GENERIC` (force the
any-alignment kernel, which always rounds like the reference) and `DECODE_GEMV` (run large M as
16-row launches of the decode kernel instead of the tensor-core GEMM).

Inputs of 128 rows or more (prefill) run the tcgen05 tensor-core GEMM and 16..127 rows (batched
decode) the tcgen05 small-M kernel; both dequantize with the reference's fp16 rounding. Above 16
rows the fused SwiGLU and RMSNorm variants run as that GEMM plus the separate norm / activation
kernels.
"""

from __future__ import annotations

import ctypes

import torch

from kernels import _lib

_choices: dict[tuple, dict] = {}  # (m_key, N, K, bias) -> config used (export/import_choices)
TC_MIN_ROWS = 128  # rows from which dk_w4a16_matmul runs the tensor-core GEMM
# rows above which the fused norm / SwiGLU entry points run as separate kernels around the tcgen05
# small-M GEMM (16 < M < 128) or the prefill GEMM instead of looping the fused decode GEMV per 16 rows
SPLIT_FUSED_ROWS = 16
# rows up to which w4a16_rmsnorm_matmul runs the norm inside the projection's kernel: every CTA of that
# kernel reduces all rows itself, which beats a separate RMSNorm launch (one CTA per row) only for one
# or two rows (B200, Qwen2.5-1.5B shapes: at 4 rows the two kernels are 1.0-1.8 us faster, at 16 rows
# 5.9-6.1 us); config {"FUSED_NORM": True} keeps the single kernel at any row count it supports
FUSED_NORM_ROWS = 2


def _check_weight_shapes(what, K, N, scales, zeros, group_size, bias):
    """The packed weight's scales / zeros are [K/group_size, N] and the bias [N]: the kernels read
    exactly those extents, so a smaller tensor would be read past its end."""
    g = K // group_size
    _lib.require_extent(tuple(scales.shape) == (g, N) and tuple(zeros.shape) == (g, N),
                        f"{what}: scales and zeros must be [{g}, {N}], got {tuple(scales.shape)} and "
                        f"{tuple(zeros.shape)}")
    _lib.require_extent(bias is None or tuple(bias.shape) == (N,), f"{what}: bias must be [{N}]")


def _config(config: dict | None) -> _lib.MatmulConfig:
    c = _lib.MatmulConfig()
    if not config:
        return c
    split = int(config.get("SPLIT_K", 0) or 0)
    if split > 8:
        raise RuntimeError(f"w4a16_matmul: SPLIT_K={split} exceeds the cluster limit of 8")
    c.split_k = max(split, 0)
    bn = int(config.get("BLOCK_N", 0) or 0)
    c.block_n = bn if bn in (32, 64, 128, 256) else 0
    exact = bool(config.get("EXACT")) or config.get("FACTORED") is False
    c.flags = (_lib.FLAG_STATIC_WEIGHTS if config.get("STATIC_WEIGHTS") else 0) | (
        _lib.FLAG_GENERIC if config.get("GENERIC") else 0) | (_lib.FLAG_EXACT_DEQUANT if exact else 0) | (
        _lib.FLAG_GEMV if config.get("DECODE_GEMV") else 0)
    # L2_PREFETCH: CUDA tensors (e.g. the weights of the launch after next) this launch pulls into L2
    pf = [t for t in (config.get("L2_PREFETCH") or ()) if t is not None and t.numel() > 0]
    if len(pf) > _lib.MAX_L2_PREFETCH:
        raise ValueError(f"L2_PREFETCH: at most {_lib.MAX_L2_PREFETCH} tensors, got {len(pf)}")
    for i, t in enumerate(pf):
        _lib.require_cuda("L2_PREFETCH", t)
        if not t.is_contiguous():
            raise ValueError("L2_PREFETCH: tensors must be contiguous")
        c.l2_prefetch_ptr[i] = t.data_ptr()
        c.l2_prefetch_bytes[i] = t.numel() * t.element_size()
    c.n_prefetch = len(pf)
    return c


def w4a16_matmul(x, qweight, scales, zeros, group_size=128, bias=None, config=None):
    """y = x @ dequant(W).T (+ bias). x: [..., K] fp16. Returns [..., N] in x's dtype."""
    K = x.shape[-1]
    N = qweight.shape[1]
    _lib.reference_assert(qweight.shape[0] * 8 == K and K % group_size == 0)
    _check_weight_shapes("w4a16_matmul", K, N, scales, zeros, group_size, bias)
    _lib.require_cuda("w4a16_matmul", x, qweight, scales, zeros, bias)
    _lib.require_dtype("w4a16_matmul", torch.float16, x, scales, zeros, bias)
    _lib.require_dtype("w4a16_matmul", torch.int32, qweight)
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    qweight, scales, zeros = qweight.contiguous(), scales.contiguous(), zeros.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    cfg = _config(config)
    _lib.call("dk_w4a16_matmul", _lib.ptr(x2), x2.stride(0), _lib.ptr(qweight), _lib.ptr(scales),
              _lib.ptr(zeros), _lib.ptr(bias), _lib.ptr(out), out.stride(0), M, N, K, group_size,
              ctypes.byref(cfg), _lib.stream_of(x))
    key = (min(1 << max(M - 1, 0).bit_length(), 4096), N, K, bias is not None)
    if key not in _choices:
        _choices[key] = {"SPLIT_K": cfg.split_k or "auto", "BLOCK_N": cfg.block_n or "auto"}
    return out.view(*x.shape[:-1], N)


def w4a16_swiglu(x, qweight, scales, zeros, group_size=128, bias=None, config=None):
    """silu(g) * u for [g, u] = x @ dequant(W).T (+ bias): the gate_up projection with SwiGLU
    fused into its epilogue (same roundings as w4a16_matmul followed by kernels.swiglu.swiglu_fused).
    W holds [gate; up] (2I output columns); returns [..., I]. Shapes the fused kernel does not cover
    (I % 32 != 0, other group sizes, unaligned operands) run the two kernels instead."""
    K = x.shape[-1]
    N = qweight.shape[1]
    _lib.reference_assert(qweight.shape[0] * 8 == K and K % group_size == 0)
    _lib.require_extent(N % 2 == 0, "w4a16_swiglu: the fused [gate; up] weight needs an even column count")
    _check_weight_shapes("w4a16_swiglu", K, N, scales, zeros, group_size, bias)
    I = N // 2
    _lib.require_cuda("w4a16_swiglu", x, qweight, scales, zeros, bias)
    _lib.require_dtype("w4a16_swiglu", torch.float16, x, scales, zeros, bias)
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    aligned = all(t.data_ptr() % 16 == 0 for t in (x2, qweight, scales, zeros)) and x2.stride(0) % 8 == 0
    cfg = _config(config)
    big = x2.shape[0] > SPLIT_FUSED_ROWS and not cfg.flags & _lib.FLAG_GEMV
    if I % 32 != 0 or group_size != 128 or not aligned or cfg.flags & _lib.FLAG_GENERIC or big:
        from kernels.swiglu import swiglu_fused

        return swiglu_fused(w4a16_matmul(x, qweight, scales, zeros, group_size, bias, config))
    qweight, scales, zeros = qweight.contiguous(), scales.contiguous(), zeros.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    M = x2.shape[0]
    out = torch.empty((M, I), dtype=x.dtype, device=x.device)
    _lib.call("dk_w4a16_swiglu", _lib.ptr(x2), x2.stride(0), _lib.ptr(qweight), _lib.ptr(scales),
              _lib.ptr(zeros), _lib.ptr(bias), _lib.ptr(out), out.stride(0), M, I, K, group_size,
              ctypes.byref(cfg), _lib.stream_of(x))
    return out.view(*x.shape[:-1], I)


def w4a16_rmsnorm_matmul(x, norm_weight, eps, residual, qweight, scales, zeros, group_size=128, bias=None,
                         swiglu=False, config=None):
    """Residual add + RMSNorm fused into the projection that consumes it.

    h = x + residual (fp16 add; h = x when residual is None); xn = rmsnorm(h, norm_weight, eps)
    (same roundings as kernels.rmsnorm.rmsnorm); returns (y, h_or_None) with y = xn @ dequant(W).T
    (+ bias), or silu(g) * u of that product when `swiglu` (W holds [gate; up]). One kernel on the
    fast path; shapes it does not cover run rmsnorm and the projection separately."""
    K = x.shape[-1]
    N = qweight.shape[1]
    _lib.reference_assert(qweight.shape[0] * 8 == K and K % group_size == 0)
    _check_weight_shapes("w4a16_rmsnorm_matmul", K, N, scales, zeros, group_size, bias)
    _lib.require_extent(norm_weight.numel() == K, f"w4a16_rmsnorm_matmul: norm_weight must have {K} elements")
    _lib.require_extent(residual is None or residual.shape == x.shape, "w4a16_rmsnorm_matmul: residual must match x")
    _lib.require_cuda("w4a16_rmsnorm_matmul", x, residual, norm_weight, qweight, scales, zeros, bias)
    _lib.require_dtype("w4a16_rmsnorm_matmul", torch.float16, x, residual, norm_weight, scales, zeros, bias)
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    r2 = None if residual is None else residual.reshape(-1, K)
    if r2 is not None and r2.stride(1) != 1:
        r2 = r2.contiguous()
    M = x2.shape[0]
    cfg = _config(config)
    I = N // 2
    tensors = [x2, qweight, scales, zeros, norm_weight] + ([r2] if r2 is not None else [])
    big = M > SPLIT_FUSED_ROWS and not cfg.flags & _lib.FLAG_GEMV
    if M > FUSED_NORM_ROWS and not (config or {}).get("FUSED_NORM"):
        big = True
    fast = (group_size == 128 and N % 8 == 0 and (not swiglu or I % 32 == 0) and not cfg.flags & _lib.FLAG_GENERIC
            and not big
            and all(t.data_ptr() % 16 == 0 for t in tensors) and x2.stride(0) % 8 == 0
            and (r2 is None or r2.stride(0) % 8 == 0) and norm_weight.is_contiguous())
    if not fast:
        from kernels.rmsnorm import rmsnorm

        normed = rmsnorm(x, norm_weight, eps, residual)
        h, res = (normed, None) if residual is None else normed
        fn = w4a16_swiglu if swiglu else w4a16_matmul
        return fn(h, qweight, scales, zeros, group_size, bias, config), res
    qweight, scales, zeros = qweight.contiguous(), scales.contiguous(), zeros.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    out = torch.empty((M, I if swiglu else N), dtype=x.dtype, device=x.device)
    res_out = None if r2 is None else torch.empty((M, K), dtype=x.dtype, device=x.device)
    _lib.call("dk_w4a16_rmsnorm_matmul", _lib.ptr(x2), x2.stride(0), _lib.ptr(r2), 0 if r2 is None else r2.stride(0),
              _lib.ptr(norm_weight), float(eps), _lib.ptr(res_out), 0 if res_out is None else res_out.stride(0),
              _lib.ptr(qweight), _lib.ptr(scales), _lib.ptr(zeros), _lib.ptr(bias), _lib.ptr(out), out.stride(0),
              M, N, K, group_size, 1 if swiglu else 0, ctypes.byref(cfg), _lib.stream_of(x))
    y = out.view(*x.shape[:-1], out.shape[-1])
    return y, None if res_out is None else res_out.view(x.shape)


def export_choices() -> dict:
    """Per-shape configs used so far (reference kernels/w4a16.py:333-335)."""
    return {",".join(map(str, k)): v for k, v in _choices.items()}


def import_choices(choices: dict) -> None:
    """Accepts the reference's format; the cost model makes the choice deterministic already
    (reference kernels/w4a16.py:338-342)."""
    for k, v in choices.items():
        m, n, kk, b = k.split(",")
        _choices[(int(m), int(n), int(kk), b == "True")] = v


def best_configs() -> dict:
    """Choices so far, for results JSON (reference kernels/w4a16.py:345-355)."""
    return {"decode_path": {str(k): v for k, v in _choices.items()}}


def w4a16_matmul_partials(x, qweight, scales, zeros, group_size=128, config=None) -> torch.Tensor:
    """x [.., K] @ dequant(W).T as fp32 split-K partial sums [S, M, N] (no bias; S is the split the
    library picks for this shape, 1 = the whole sum): the decode GEMV without its cluster reduction,
    for `w4a16_rmsnorm_matmul_partials` to add while it stages its input. 1..16 rows. No reference
    counterpart (the reference passes the complete fp16 output, kernels/e2e/model.py:247)."""
    K = x.shape[-1]
    N = qweight.shape[1]
    _lib.reference_assert(qweight.shape[0] * 8 == K and K % group_size == 0)
    _check_weight_shapes("w4a16_matmul_partials", K, N, scales, zeros, group_size, None)
    _lib.require_cuda("w4a16_matmul_partials", x, qweight, scales, zeros)
    _lib.require_dtype("w4a16_matmul_partials", torch.float16, x, scales, zeros)
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    _lib.require_extent(1 <= M <= 16, "w4a16_matmul_partials: 1..16 rows")
    buf = torch.empty(8 * M * N, dtype=torch.float32, device=x.device)
    n = ctypes.c_int32(0)
    _lib.call("dk_w4a16_matmul_partials", _lib.ptr(x2), x2.stride(0), _lib.ptr(qweight.contiguous()),
              _lib.ptr(scales.contiguous()), _lib.ptr(zeros.contiguous()), M, N, K, group_size, _lib.ptr(buf),
              buf.numel(), ctypes.byref(n), ctypes.byref(_config(config)), _lib.stream_of(x))
    return buf[: n.value * M * N].view(n.value, M, N)


def w4a16_rmsnorm_matmul_partials(parts, part_bias, norm_weight, eps, residual, qweight, scales, zeros,
                                  group_size=128, bias=None, swiglu=False, config=None):
    """`w4a16_rmsnorm_matmul` whose input is fp16(parts[0] + ... + parts[S-1] (+ part_bias)) - the
    previous projection's split-K partial sums [S, M, K] from `w4a16_matmul_partials`, added in slice
    order as that projection's own reduction would - in one kernel. Returns (y, h_or_None)."""
    S, M, K = parts.shape
    N = qweight.shape[1]
    _lib.reference_assert(qweight.shape[0] * 8 == K and K % group_size == 0)
    _check_weight_shapes("w4a16_rmsnorm_matmul_partials", K, N, scales, zeros, group_size, bias)
    _lib.require_extent(1 <= S <= 8 and 1 <= M <= 16 and parts.dtype == torch.float32 and parts.is_contiguous(),
                        "w4a16_rmsnorm_matmul_partials: parts must be contiguous fp32 [1..8, 1..16, K]")
    _lib.require_extent(part_bias is None or part_bias.numel() == K, "w4a16_rmsnorm_matmul_partials: part_bias [K]")
    _lib.require_extent(norm_weight.numel() == K, f"w4a16_rmsnorm_matmul_partials: norm_weight must have {K} elements")
    r2 = None if residual is None else residual.reshape(-1, K)
    _lib.require_extent(r2 is None or r2.shape[0] == M, "w4a16_rmsnorm_matmul_partials: residual must be [M, K]")
    _lib.require_cuda("w4a16_rmsnorm_matmul_partials", parts, part_bias, residual, norm_weight, qweight, scales, zeros,
                      bias)
    _lib.require_dtype("w4a16_rmsnorm_matmul_partials", torch.float16, residual, norm_weight, scales, zeros, bias,
                       part_bias)
    if r2 is not None and r2.stride(1) != 1:
        r2 = r2.contiguous()
    I = N // 2
    out = torch.empty((M, I if swiglu else N), dtype=torch.float16, device=parts.device)
    res_out = None if r2 is None else torch.empty((M, K), dtype=torch.float16, device=parts.device)
    _lib.call("dk_w4a16_rmsnorm_matmul_partials", _lib.ptr(parts), S, _lib.ptr(part_bias), _lib.ptr(r2),
              0 if r2 is None else r2.stride(0), _lib.ptr(norm_weight.contiguous()), float(eps), _lib.ptr(res_out),
              0 if res_out is None else res_out.stride(0), _lib.ptr(qweight.contiguous()), _lib.ptr(scales.contiguous()),
              _lib.ptr(zeros.contiguous()), _lib.ptr(None if bias is None else bias.contiguous()), _lib.ptr(out),
              out.stride(0), M, N, K, group_size, 1 if swiglu else 0, ctypes.byref(_config(config)),
              _lib.stream_of(parts))
    return out, res_out
