"""The two ends of a per-op greedy decode step as libdecodek kernels.

`lm_head_greedy` is the tail of the reference runner's T == 1 forward plus its graph decoder's
bookkeeping (kernels/e2e/model.py:248-253, kernels/e2e/run.py:69-74): final RMSNorm of the residual
stream, the fp16 lm_head (accumulated in fp32, logits rounded to fp16 as cuBLAS's fp16 GEMM does),
the greedy pick (first maximum, torch.argmax's rule), `out[:, pos] = pick`, `tok = pick` and
`pos += 1`, all in one kernel with everything on the device. `embed_tokens` is the embedding lookup
at the head of the forward (model.py:227).
"""

from __future__ import annotations

import ctypes

import torch

from kernels import _lib

MAX_ROWS = 8
# rows up to which the runner's per-op step ends in lm_head_greedy: its fp32 FMA form streams the
# lm_head at ~98% of HBM bandwidth for one row, but more rows make it compute-bound (cuBLAS then wins)
RUNNER_ROWS = 1


def workspace(device) -> torch.Tensor:
    """A zeroed workspace for `lm_head_greedy` (its arrival counter; calls that share one must be
    ordered on one stream)."""
    nbytes = ctypes.c_uint64(0)
    _lib.call("dk_lm_head_greedy_workspace_bytes", ctypes.byref(nbytes))
    return torch.zeros(int(nbytes.value), dtype=torch.uint8, device=device)


def lm_head_greedy(x: torch.Tensor, residual: torch.Tensor | None, norm_weight: torch.Tensor | None, eps: float,
                   lm_head: torch.Tensor, tokens: torch.Tensor, ws: torch.Tensor, pos: torch.Tensor | None = None,
                   history: torch.Tensor | None = None, logits: torch.Tensor | None = None) -> None:
    """x, residual [M, H] fp16 (residual may be None), norm_weight [H] or None, lm_head [V, H] fp16.
    Writes the greedy picks into tokens (int64, M elements); with history (int64 [M, >= 1], unit
    column stride) also history[:, pos] = picks and pos += 1 (pos int64 [1] on the device); logits
    (fp16 [M, V]) if given. Graph-capturable."""
    M, H = x.shape
    V = lm_head.shape[0]
    _lib.require_extent(1 <= M <= MAX_ROWS, f"lm_head_greedy: 1..{MAX_ROWS} rows")
    _lib.require_extent(lm_head.dim() == 2 and lm_head.shape[1] == H, "lm_head_greedy: lm_head must be [vocab, hidden]")
    _lib.require_extent(residual is None or tuple(residual.shape) == (M, H), "lm_head_greedy: residual must be [M, hidden]")
    _lib.require_extent(norm_weight is None or norm_weight.numel() == H, "lm_head_greedy: norm weight must hold hidden values")
    _lib.require_extent(tokens.numel() == M and tokens.dtype == torch.int64 and tokens.is_contiguous(),
                        "lm_head_greedy: tokens must be a contiguous int64 tensor of M elements")
    _lib.require_extent(logits is None or (tuple(logits.shape) == (M, V) and logits.is_contiguous()
                                           and logits.dtype == torch.float16),
                        "lm_head_greedy: logits must be a contiguous fp16 [M, vocab] tensor")
    ld = hlen = 0
    if history is not None:
        _lib.require_extent(pos is not None and pos.numel() >= 1 and pos.dtype == torch.int64,
                            "lm_head_greedy: history needs the int64 position tensor")
        _lib.require_extent(history.dim() == 2 and history.shape[0] == M and history.stride(1) == 1
                            and history.dtype == torch.int64, "lm_head_greedy: history must be int64 [M, len]")
        ld, hlen = history.stride(0), history.shape[1]
    _lib.require_cuda("lm_head_greedy", x, residual, norm_weight, lm_head, tokens, ws, pos, history, logits)
    _lib.require_dtype("lm_head_greedy", torch.float16, x, lm_head, *(t for t in (residual, norm_weight) if t is not None))
    x = x.contiguous()
    residual = residual.contiguous() if residual is not None else None
    _lib.call("dk_lm_head_greedy", _lib.ptr(x), _lib.ptr(residual), _lib.ptr(norm_weight), float(eps),
              _lib.ptr(lm_head.contiguous()), V, H, M, _lib.ptr(tokens), _lib.ptr(pos), _lib.ptr(history), ld, hlen,
              _lib.ptr(logits), _lib.ptr(ws), ws.numel(), _lib.stream_of(x))


def embed_tokens(tokens: torch.Tensor, embed: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """embed[tokens] for device int64 tokens of any shape: [*tokens.shape, hidden] fp16."""
    V, H = embed.shape
    _lib.require_extent(tokens.dtype == torch.int64, "embed_tokens: int64 token ids")
    _lib.require_cuda("embed_tokens", tokens, embed, out)
    _lib.require_dtype("embed_tokens", torch.float16, embed)
    t = tokens.contiguous()
    if out is None:
        out = torch.empty((*tokens.shape, H), dtype=embed.dtype, device=embed.device)
    _lib.require_extent(out.numel() == t.numel() * H and out.is_contiguous(), "embed_tokens: out must be [*tokens, hidden]")
    _lib.call("dk_embed_tokens", _lib.ptr(t), _lib.ptr(embed.contiguous()), V, H, t.numel(), _lib.ptr(out),
              _lib.stream_of(embed))
    return out


class KernelHeadLogits:
    """A runner-like view (`forward(tokens, pos)`, `greedy`) whose one-token forward is the per-op
    greedy step's own kernels - the embedding kernel, the runner's five kernels per layer and the
    lm_head + greedy-pick kernel - returning that kernel's fp16 logits, for parity checks
    (kernels.e2e.run.greedy_parity). Prompts go through the runner's own forward; `picks` holds the
    kernel's greedy picks of the last one-token forward."""

    def __init__(self, runner):
        if not runner._kernel_head():
            raise RuntimeError("the lm_head + greedy-pick kernel does not apply to this runner")
        self.r = runner
        B, V = runner.batch, runner.lm_head.shape[0]
        self.logits = torch.empty(B, V, dtype=torch.float16, device=runner.embed.device)
        self.picks = torch.empty(B, dtype=torch.int64, device=runner.embed.device)

    @torch.no_grad()
    def forward(self, tokens: torch.Tensor, pos: torch.Tensor, all_logits: bool = False):
        if tokens.shape[1] > 1:
            return self.r.forward(tokens, pos, all_logits)
        r = self.r
        B, H = tokens.shape[0], r.embed.shape[1]
        h, residual = r._decode_layers(embed_tokens(tokens, r.embed), pos)
        lm_head_greedy(h.reshape(B, H), residual.reshape(B, H), r.final_norm, r.eps, r.lm_head, self.picks,
                       r._head_ws, logits=self.logits)
        return self.logits.view(B, 1, -1)

    def greedy(self, logits):
        return self.r.greedy(logits)
