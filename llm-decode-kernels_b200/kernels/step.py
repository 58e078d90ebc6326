"""The fused decode step: one persistent libdecodek kernel per token (dk_step_run).

For the W4A16 runner at batch 1..4 this replaces the ~146 launches of a decode step (five per layer,
the final norm, the fp16 lm_head, argmax and the bookkeeping) with one cooperative launch: every SM's
producer warp streams that SM's share of each projection's weights into shared memory ahead of the
op that needs them, and the ops meet through arrival counters. The step is the reference runner's
T == 1 forward plus the greedy pick of its graph decoder (kernels/e2e/model.py:216-253,
kernels/e2e/run.py:69-74) with the numerics of the separate kernels.

The workspace (op table, tensor maps, counters, activations) is a torch uint8 tensor owned by the
`DecodeStep` object; the model's weights and KV caches are referenced, so the runner must outlive it.
"""

from __future__ import annotations

import ctypes

import torch

from kernels import _lib

MAX_ROWS = 4


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def supported(runner) -> str | None:
    """None if the fused step can run this runner, else why not."""
    be = runner.backend
    if getattr(be, "name", "") != "ours" or not getattr(be, "fused_decode", False):
        return f"backend {getattr(be, 'name', be)!r} (the fused step runs the W4A16 'ours' backend)"
    if runner.tp is not None:
        return "tensor parallel runner"
    if runner.batch > MAX_ROWS:
        return f"batch {runner.batch} > {MAX_ROWS}"
    if runner.head_q is not None:
        return "quantized lm_head"
    if runner.head_dim != 128 or runner.n_heads % runner.n_kv or runner.n_heads // runner.n_kv > 8:
        return "attention shape"
    H = runner.embed.shape[1]
    I = runner.layers[0].down.qweight.shape[0] * 8
    if H % 256 or I % 256 or (runner.n_heads * 128) % 256 or runner.embed.shape[0] % 32 or runner.max_len % 128:
        return "layer sizes"
    if runner.embed.dtype != torch.float16:
        return "dtype"
    return None


class DecodeStep:
    """One launch per greedy decode step of `runner` (a QwenRunner on the 'ours' backend)."""

    def __init__(self, runner):
        why = supported(runner)
        if why is not None:
            raise RuntimeError(f"fused decode step unavailable: {why}")
        self.runner = runner
        L0 = runner.layers[0]
        H = runner.embed.shape[1]
        I = L0.down.qweight.shape[0] * 8
        self._keep = []  # tensors whose pointers the plan holds

        def keep(t):
            if t is None:
                return None
            t = t.contiguous()
            self._keep.append(t)
            return _p(t)

        layers = (_lib.StepLayer * len(runner.layers))()
        for i, L in enumerate(runner.layers):
            y = layers[i]
            y.input_norm, y.post_norm = keep(L.ln1), keep(L.ln2)
            for name, lin in (("qkv", L.qkv), ("o", L.o), ("gate_up", L.gate_up), ("down", L.down)):
                setattr(y, f"{name}_qweight", keep(lin.qweight))
                setattr(y, f"{name}_scales", keep(lin.scales))
                setattr(y, f"{name}_zeros", keep(lin.zeros))
                setattr(y, f"{name}_bias", keep(lin.bias))
        self._layers = layers
        m = _lib.StepModel()
        m.n_layers = len(runner.layers)
        m.hidden = H
        m.n_heads = runner.n_heads
        m.n_kv = runner.n_kv
        m.head_dim = runner.head_dim
        m.intermediate = I
        m.vocab = runner.embed.shape[0]
        m.max_len = runner.max_len
        m.batch = runner.batch
        m.eps = float(runner.eps)
        m.embed = keep(runner.embed)
        m.final_norm = keep(runner.final_norm)
        m.lm_head = keep(runner.lm_head)
        m.rope_cos = keep(runner.rope_cos)
        m.rope_sin = keep(runner.rope_sin)
        for c in (runner.k_cache, runner.v_cache):
            if not c.is_contiguous():
                raise RuntimeError("fused decode step: the KV caches must be contiguous")
        m.k_cache = _p(runner.k_cache)
        m.v_cache = _p(runner.v_cache)
        m.layers = ctypes.cast(layers, ctypes.POINTER(_lib.StepLayer))
        self._model = m
        nbytes = ctypes.c_uint64(0)
        _lib.call("dk_step_workspace_bytes", ctypes.byref(m), ctypes.byref(nbytes))
        # 256-byte aligned workspace from the caching allocator (its blocks are 512-byte aligned)
        self.workspace = torch.zeros(int(nbytes.value), dtype=torch.uint8, device=runner.embed.device)
        plan = ctypes.c_void_p()
        _lib.call("dk_step_create", ctypes.byref(m), _p(self.workspace), nbytes.value, ctypes.byref(plan))
        self._plan = plan

    def __call__(self, tok: torch.Tensor, pos: torch.Tensor, hist: torch.Tensor | None = None,
                 logits: torch.Tensor | None = None) -> None:
        """tok int64 [B] or [B, 1] (in: this step's tokens; out: the greedy picks), pos int64 [1]
        (incremented), hist int64 [B, >= max_len] or None (hist[:, pos] = pick), logits fp16 [B, vocab]
        or None. Everything stays on the device (graph-capturable)."""
        r = self.runner
        B = r.batch
        if tok.numel() != B or tok.dtype != torch.int64 or not tok.is_contiguous():
            raise ValueError(f"fused decode step: tok must be a contiguous int64 tensor of {B} tokens")
        if pos.numel() < 1 or pos.dtype != torch.int64:
            raise ValueError("fused decode step: pos must be an int64 tensor holding the position")
        ld = 0
        if hist is not None:
            if hist.dtype != torch.int64 or hist.dim() != 2 or hist.shape[0] != B or hist.stride(1) != 1 \
                    or hist.shape[1] < r.max_len:
                raise ValueError(f"fused decode step: hist must be int64 [{B}, >= {r.max_len}] with unit stride")
            ld = hist.stride(0)
        if logits is not None and (logits.dtype != torch.float16 or tuple(logits.shape) != (B, r.embed.shape[0])
                                   or not logits.is_contiguous()):
            raise ValueError("fused decode step: logits must be a contiguous fp16 [batch, vocab] tensor")
        _lib.require_cuda("decode step", tok, pos, hist, logits)
        _lib.call("dk_step_run", self._plan, _p(tok), _p(pos), _p(hist), ld, _p(logits), _lib.stream_of(tok))

    KINDS = {1: "qkv", 2: "attention", 3: "o_proj", 4: "gate_up", 5: "down", 6: "lm_head"}

    def trace(self, tok: torch.Tensor, pos: torch.Tensor, hist: torch.Tensor | None = None) -> dict:
        """Run one step with dk_step_trace and summarize where its time goes (synchronizes; not for
        use under capture). Per op kind, averaged over its ops, in microseconds:
        `span` - from the previous op's last finished CTA to this op's last (the op's share of the step);
        for the median participating CTA: `input` - from the previous op's last CTA until this CTA had
        its input staged (polling the tagged words plus staging), `staging` - from having the op's
        descriptor to the input staged (includes waiting when the CTA was early), `products` - weights
        x input, `epilogue` - reduction and stores; `tail` - last CTA minus the median CTA (stragglers);
        `ring_wait_kcycles` - the most cycles any warp waited for its weights; `box_kcycles` - the median
        CTA's first consumer warp's cycles for its boxes; plus `step_us`."""
        nbytes = ctypes.c_uint64(0)
        _lib.call("dk_step_trace_bytes", self._plan, ctypes.byref(nbytes))
        buf = torch.zeros(int(nbytes.value) // 8, dtype=torch.int64, device=tok.device)
        n = ctypes.c_int32(0)
        _lib.call("dk_step_ops", self._plan, None, 0, ctypes.byref(n))
        kinds = (ctypes.c_int32 * n.value)()
        _lib.call("dk_step_ops", self._plan, kinds, n.value, ctypes.byref(n))
        ld = 0 if hist is None else hist.stride(0)
        _lib.call("dk_step_trace", self._plan, _p(tok), _p(pos), _p(hist), ld, None, _p(buf), _lib.stream_of(tok))
        torch.cuda.synchronize()
        t = buf.view(-1, n.value + 1, 12).cpu().double()
        t0 = t[:, n.value, 0].min()
        step_us = float((t[:, n.value, 1].max() - t0) / 1e3)
        rows = {}
        prev_last = t0
        keys = ("span", "input", "staging", "products", "epilogue", "tail", "ring_wait_kcycles", "box_kcycles", "ctas")
        for j in range(n.value):
            part = t[:, j, 1] > 0
            tj = t[part, j]
            done = tj[:, 4]
            last = done.max()
            med = float(done.median())
            r = rows.setdefault(self.KINDS.get(kinds[j], str(kinds[j])), dict.fromkeys(keys, 0.0) | {"n": 0})
            r["n"] += 1
            r["span"] += float(last - prev_last) / 1e3
            has_stage = tj[:, 2] > 0
            if bool(has_stage.any()):
                ts = tj[has_stage]
                r["input"] += float((ts[:, 2] - prev_last).median()) / 1e3
                r["staging"] += float((ts[:, 2] - ts[:, 1]).median()) / 1e3
                r["products"] += float((ts[:, 3] - ts[:, 2]).median()) / 1e3
                r["epilogue"] += float((ts[:, 4] - ts[:, 3]).median()) / 1e3
                if kinds[j] not in (2, 6):
                    r["box_kcycles"] += float(ts[:, 9].median()) / 1e3
            else:  # attention: from the previous op to the median CTA's end
                r["input"] += float(med - float(prev_last)) / 1e3
            r["tail"] += float(last - med) / 1e3
            r["ring_wait_kcycles"] += float(tj[:, 6].max()) / 1e3
            r["ctas"] += int(part.sum())
            prev_last = last
        for r in rows.values():
            for k in keys:
                r[k] = round(r[k] / r["n"], 3)
        return {"step_us": round(step_us, 2), "ops": rows}

    def close(self):
        if self._plan is not None and self._plan.value:
            _lib.call("dk_step_destroy", self._plan)
            self._plan = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StepLogits:
    """A runner-like view (`forward(tokens, pos)`, `greedy`) whose one-token forward is the fused
    step's logits, for parity checks (kernels.e2e.run.greedy_parity): prompts go through the runner's
    own forward; a single token runs the step kernel on copies of the token and position, so the
    caller's state is not advanced."""

    def __init__(self, runner):
        self.r = runner
        self.kernel = runner.step_kernel()
        if self.kernel is None:
            raise RuntimeError("fused decode step unavailable for this runner")
        self.logits = torch.empty(runner.batch, runner.embed.shape[0], dtype=torch.float16,
                                  device=runner.embed.device)

    def forward(self, tokens: torch.Tensor, pos: torch.Tensor, all_logits: bool = False):
        if tokens.shape[1] > 1:
            return self.r.forward(tokens, pos, all_logits)
        self.kernel(tokens.clone().contiguous(), pos.clone(), None, self.logits)
        return self.logits.view(self.r.batch, 1, -1)

    def greedy(self, logits):
        return self.r.greedy(logits)
