"""A Qwen2 decode runner on a Hugging Face model object, with swappable kernel backends.

Same structure and API as the reference's kernels/e2e/model.py: a static KV cache, RoPE, and the
fused qkv and gate/up projections, with the linear / norm / activation ops supplied by a backend.
The fp16 and w4_ref backends keep the reference's plain PyTorch numerics (the fp16 cuBLAS
baseline and the quality reference). The `ours*` backends run libdecodek's sm_100a kernels:
W4A16 (or FP8) linears with weight prefetch across kernels, fused residual+RMSNorm, SwiGLU fused
into the gate_up kernel's epilogue, and a decode-attention kernel that reads only the cached
positions (the reference's SDPA reads the whole `max_len` cache every step).

Kept in fp16 on every backend: embeddings, RoPE tables, the KV cache. lm_head (tied to the
embeddings) stays fp16 unless the backend name ends in `_lm`, which also quantizes a copy of it.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from kernels import config

# ------------------------------------------------------------------------------------- ops


@dataclass
class Linear:
    """One projection. fp16 holds `w`; quantized backends hold the packed tensors
    (reference kernels/e2e/model.py:25-33)."""

    w: torch.Tensor | None = None
    qweight: torch.Tensor | None = None
    scales: torch.Tensor | None = None
    zeros: torch.Tensor | None = None
    bias: torch.Tensor | None = None
    # kernel backends: tensors this projection's launch pulls into L2 for a later launch
    l2_next: tuple | None = None


class Backend:
    """fp16 eager PyTorch ops with Hugging Face Qwen2 numerics (reference model.py:36-52)."""

    name = "fp16"
    quantized = False
    fused_decode = False  # True: the runner uses attention_decode / gate_up_act hooks
    partials = False  # True: linear_partials / norm_linear_partials (split-K sums between launches)

    def linear(self, x, p: Linear):
        return F.linear(x, p.w, p.bias)

    def norm(self, x, w, eps, residual=None):
        from kernels.reference import rmsnorm_ref

        return rmsnorm_ref(x, w, eps, residual)

    def act(self, gate_up):
        i = gate_up.shape[-1] // 2
        return F.silu(gate_up[..., :i]) * gate_up[..., i:]

    def gate_up_act(self, x, p: Linear):
        return self.act(self.linear(x, p))

    def norm_linear(self, x, w, eps, residual, p: Linear):
        """(linear(norm(x [+ residual])), new residual or None) - fused by kernel backends."""
        if residual is None:
            return self.linear(self.norm(x, w, eps), p), None
        h, residual = self.norm(x, w, eps, residual=residual)
        return self.linear(h, p), residual

    def norm_gate_up_act(self, x, w, eps, residual, p: Linear):
        h, residual = self.norm(x, w, eps, residual=residual)
        return self.gate_up_act(h, p), residual


class W4RefBackend(Backend):
    """RTN 4-bit weights dequantized once to fp16, then cuBLAS (reference model.py:55-67): the
    same quality as the kernels, so quality changes come from quantization, not the kernels."""

    name = "w4_ref"
    quantized = True

    def linear(self, x, p: Linear):
        from kernels.reference import dequantize_ref

        if p.w is None:  # dequantize once, cache
            p.w = dequantize_ref(p.qweight, p.scales, p.zeros, config.GROUP_SIZE)
        return F.linear(x, p.w, p.bias)


class OursBackend(Backend):
    """libdecodek kernels: W4A16 linears, fused residual+RMSNorm, SwiGLU (reference model.py:70-97).

    `decode_kernel` keeps the reference's names ("triton" -> `ours`, "cuda" -> `ours_cuda`); both
    run the same sm_100a kernels here (`ours_cuda` goes through w4a16_decode_cuda for <= 16 rows,
    like the reference)."""

    quantized = True
    fused_decode = True
    # weights of a runner never change: let each kernel prefetch them before the previous ends
    LINEAR_CFG = {"STATIC_WEIGHTS": True}
    # the (norm +) gate_up + SwiGLU launch of up to 4 rows in 64-column tiles (gate and up chunk
    # pairs): in the decode step it then leaves room on the SMs for the down projection's CTAs to
    # start early and stream their weights (B200, Qwen2.5-1.5B, ms per step: batch 1 0.873 -> 0.827,
    # batch 2 0.945 -> 0.911, batch 4 1.162 -> 1.137; the cost model, which sees one launch at a
    # time, picks a tiling that fills every SM)
    GATE_UP_SMALL_M = {"BLOCK_N": 64}
    GATE_UP_SMALL_M_ROWS = 4

    def __init__(self, decode_kernel: str = "triton"):
        self.decode_kernel = decode_kernel
        self.name = "ours" if decode_kernel == "triton" else f"ours_{decode_kernel}"

    def cfg(self, p: Linear) -> dict:
        return self.LINEAR_CFG if p.l2_next is None else {**self.LINEAR_CFG, "L2_PREFETCH": p.l2_next}

    def linear(self, x, p: Linear):
        from kernels.w4a16 import w4a16_matmul

        rows = x.numel() // x.shape[-1]
        if self.decode_kernel == "cuda" and rows <= 16:
            from kernels.cuda.w4a16_cuda import w4a16_decode_cuda

            return w4a16_decode_cuda(x, p.qweight, p.scales, p.zeros, bias=p.bias)
        return w4a16_matmul(x, p.qweight, p.scales, p.zeros, bias=p.bias, config=self.cfg(p))

    def norm(self, x, w, eps, residual=None):
        from kernels.rmsnorm import rmsnorm

        return rmsnorm(x, w, eps, residual)

    def act(self, gate_up):
        from kernels.swiglu import swiglu_fused

        return swiglu_fused(gate_up)

    def gate_up_cfg(self, x, p: Linear) -> dict:
        cfg = self.cfg(p)
        return {**cfg, **self.GATE_UP_SMALL_M} if x.numel() <= self.GATE_UP_SMALL_M_ROWS * x.shape[-1] else cfg

    def gate_up_act(self, x, p: Linear):
        from kernels.w4a16 import w4a16_swiglu

        return w4a16_swiglu(x, p.qweight, p.scales, p.zeros, bias=p.bias, config=self.gate_up_cfg(x, p))

    def norm_linear(self, x, w, eps, residual, p: Linear):
        from kernels.w4a16 import w4a16_rmsnorm_matmul

        return w4a16_rmsnorm_matmul(x, w, eps, residual, p.qweight, p.scales, p.zeros, bias=p.bias,
                                    config=self.cfg(p))

    def norm_gate_up_act(self, x, w, eps, residual, p: Linear):
        from kernels.w4a16 import w4a16_rmsnorm_matmul

        return w4a16_rmsnorm_matmul(x, w, eps, residual, p.qweight, p.scales, p.zeros, bias=p.bias, swiglu=True,
                                    config=self.gate_up_cfg(x, p))

    # The down projection of a one-row decode step hands its split-K partial sums to the next layer's
    # norm + qkv launch, which adds them while staging its input (the same sums, one cluster
    # reduction fewer per layer).
    @property
    def partials(self) -> bool:
        return self.decode_kernel == "triton"

    def linear_partials(self, x, p: Linear):
        from kernels.w4a16 import w4a16_matmul_partials

        return w4a16_matmul_partials(x, p.qweight, p.scales, p.zeros, config=self.cfg(p))

    def norm_linear_partials(self, parts, part_bias, w, eps, residual, p: Linear):
        from kernels.w4a16 import w4a16_rmsnorm_matmul_partials

        return w4a16_rmsnorm_matmul_partials(parts, part_bias, w, eps, residual, p.qweight, p.scales, p.zeros,
                                             bias=p.bias, config=self.cfg(p))


class OursFP8Backend(OursBackend):
    """FP8 (e4m3) weight-only linears with the same fused norm/activation kernels
    (reference model.py:100-118)."""

    partials = False

    name = "ours_fp8"

    def __init__(self):
        super().__init__("triton")
        self.name = "ours_fp8"

    def quantize(self, w, b) -> Linear:
        from kernels.fp8 import quantize_fp8

        wq, s = quantize_fp8(w)
        return Linear(qweight=wq, scales=s, bias=b)

    def linear(self, x, p: Linear):
        from kernels.fp8 import w8a16_matmul

        return w8a16_matmul(x, p.qweight, p.scales, bias=p.bias, config=self.cfg(p))

    def gate_up_act(self, x, p: Linear):
        return self.act(self.linear(x, p))

    def norm_linear(self, x, w, eps, residual, p: Linear):
        return Backend.norm_linear(self, x, w, eps, residual, p)

    def norm_gate_up_act(self, x, w, eps, residual, p: Linear):
        return Backend.norm_gate_up_act(self, x, w, eps, residual, p)


_BACKENDS = {
    "fp16": Backend,
    "w4_ref": W4RefBackend,
    "ours": lambda: OursBackend("triton"),
    "ours_cuda": lambda: OursBackend("cuda"),
    "ours_fp8": OursFP8Backend,
}
_LM_SUFFIX = "_lm"


def make_backend(name: str) -> Backend:
    """A backend by the reference's names (kernels/e2e/model.py:121-136): one of `_BACKENDS`, or a
    quantized one with `_lm` appended to quantize lm_head as well (`fp16_lm` is a ValueError)."""
    base = name.removesuffix(_LM_SUFFIX)
    quant_head = base != name
    if base not in _BACKENDS:
        raise KeyError(name)
    backend = _BACKENDS[base]()
    if quant_head and not backend.quantized:
        raise ValueError(f"{name}: only quantized backends can quantize lm_head")
    backend.quant_lm_head = quant_head
    if quant_head:
        backend.name = name
    return backend


def _nbytes(*tensors) -> int:
    return sum(t.numel() * t.element_size() for t in tensors if t is not None)


# ------------------------------------------------------------------------------------- model
@dataclass
class Layer:
    """One decoder layer: its two RMSNorm weights and the four projections in launch order."""

    ln1: torch.Tensor
    ln2: torch.Tensor
    qkv: Linear
    o: Linear
    gate_up: Linear
    down: Linear

    def projections(self) -> tuple:
        return self.qkv, self.o, self.gate_up, self.down


class QwenRunner:
    """Qwen2 forward on a static KV cache (reference model.py:150-253): the T == 1 decode path runs
    the backend's fused kernels, longer inputs the reference's numerics (SDPA over the cache). A
    greedy step (`greedy_step`) on the kernel backends is the embedding kernel, five kernels per layer
    and one lm_head + greedy-pick kernel (batch 1, fp16 lm_head), or with fused_step=True the
    single decode-step kernel of the W4A16 runner at batch <= 4."""

    def __init__(self, hf_model, backend: Backend, max_len: int = 2048, batch: int = 1,
                 l2_prefetch: bool = False, tp=None, fused_step: bool = False):
        """tp: a kernels.tp.TensorParallel to hold only this rank's shards (column-sharded qkv,
        gate_up and lm_head; row-sharded o_proj and down, reduced over the group), or None.
        fused_step: run greedy_step as the single decode-step kernel where it supports the model."""
        cfg = hf_model.config
        self.backend = backend
        self.eps = cfg.rms_norm_eps
        self.n_heads = cfg.num_attention_heads
        self.n_kv = cfg.num_key_value_heads
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.n_heads
        self.max_len = max_len
        self.batch = batch
        self.fused_step = fused_step
        self._step_kernel = None
        self._head_ws = None  # workspace of the lm_head + greedy-pick kernel (made on first use)
        m = hf_model.model
        dev = m.embed_tokens.weight.device
        self.embed = m.embed_tokens.weight
        self.tp = tp
        hd = self.head_dim
        everything = (0, 1 << 62)
        if tp is not None:
            self.plan = tp.plan(cfg)
            self.n_heads, self.n_kv = self.plan.n_q, self.plan.n_kv
            qh, kvh, mlp, voc = self.plan.q_heads, self.plan.kv_heads, self.plan.mlp, self.plan.vocab
        else:
            self.plan = None
            qh = kvh = mlp = voc = everything
        self.vocab_start = voc[0] if tp is not None else 0
        q_rows, kv_rows = (qh[0] * hd, qh[1] * hd), (kvh[0] * hd, kvh[1] * hd)
        self.lm_head = hf_model.lm_head.weight[voc[0]:voc[1]]
        self.final_norm = m.norm.weight
        rope = getattr(cfg, "rope_parameters", None) or {}
        theta = rope.get("rope_theta", getattr(cfg, "rope_theta", 10000.0))
        self.inv_freq = 1.0 / (theta ** (torch.arange(0, hd, 2, device=dev, dtype=torch.float) / hd))

        def shard(mod, rows=everything, cols=everything):
            """(weight, bias) of a module cut to output rows / input columns (this rank's shard)."""
            w = mod.weight.data[rows[0]:rows[1], cols[0]:cols[1]]
            return w, None if mod.bias is None else mod.bias.data[rows[0]:rows[1]]

        def projection(*pieces) -> Linear:
            """Output rows of the pieces stacked (fused qkv, fused gate_up), then the backend's format."""
            w = torch.cat([pw for pw, _ in pieces]).contiguous()
            b = None if pieces[0][1] is None else torch.cat([pb for _, pb in pieces]).contiguous()
            if not backend.quantized:
                return Linear(w=w, bias=b)
            if hasattr(backend, "quantize"):  # formats other than int4 RTN (FP8)
                return backend.quantize(w, b)
            from kernels.quant import quantize_rtn

            qw, s, z = quantize_rtn(w, config.GROUP_SIZE)
            return Linear(qweight=qw, scales=s, zeros=z, bias=b)

        # Optional quantized copy of lm_head (the fp16 table stays for the embedding lookup).
        self.head_q = (projection(shard(hf_model.lm_head, rows=voc)) if getattr(backend, "quant_lm_head", False)
                       else None)
        self.layers = []
        for layer in m.layers:
            att, mlp_mod = layer.self_attn, layer.mlp
            self.layers.append(Layer(
                ln1=layer.input_layernorm.weight, ln2=layer.post_attention_layernorm.weight,
                qkv=projection(shard(att.q_proj, rows=q_rows), shard(att.k_proj, rows=kv_rows),
                               shard(att.v_proj, rows=kv_rows)),
                o=projection(shard(att.o_proj, cols=q_rows)),
                gate_up=projection(shard(mlp_mod.gate_proj, rows=mlp), shard(mlp_mod.up_proj, rows=mlp)),
                down=projection(shard(mlp_mod.down_proj, cols=mlp)),
            ))
        if tp is not None:
            tp.setup(cfg.hidden_size, dev)
        if backend.fused_decode and l2_prefetch:
            self._plan_l2_prefetch()
        # RoPE tables for the decode kernels, computed with the same ops as the T > 1 path uses per step
        if backend.fused_decode:
            self.rope_cos, self.rope_sin = self._rope_tables(torch.arange(max_len, device=dev), self.embed.dtype)
        self.k_cache, self.v_cache = self._new_caches(batch)

    def _new_caches(self, batch: int):
        shape = (len(self.layers), batch, self.n_kv, self.max_len, self.head_dim)
        dev, dt = self.embed.device, self.embed.dtype
        return torch.zeros(shape, device=dev, dtype=dt), torch.zeros(shape, device=dev, dtype=dt)

    def with_batch(self, batch: int) -> "QwenRunner":
        """A runner for another batch size that shares this one's weights (new, empty KV caches)."""
        import copy

        r = copy.copy(self)
        r.batch = batch
        r._step_kernel = None
        r.k_cache, r.v_cache = self._new_caches(batch)
        return r

    def _plan_l2_prefetch(self):
        """Each projection's launch pulls the weights of the projection two launches ahead in the
        decode chain (qkv, o, gate_up, down of layer 0, then layer 1, ...) into L2; the first one
        also pulls the next. A layer's weights (25 MB for Qwen2.5-1.5B) then arrive while the
        latency-bound launches before them run, and each GEMV reads L2 instead of HBM."""
        chain = [p for L in self.layers for p in (L.qkv, L.o, L.gate_up, L.down)]

        def tensors(p):
            return tuple(t for t in (p.qweight, p.scales, p.zeros) if t is not None)

        for j, p in enumerate(chain):
            ahead = chain[j + 2: j + 3] + (chain[1:2] if j == 0 else [])
            p.l2_next = tuple(t for q in ahead for t in tensors(q)) or None

    def weight_bytes(self) -> dict:
        """Bytes the swapped layers read per token vs the parts that stay fp16 (the reference's
        accounting, model.py:196-210): packed weights + scales + zeros + bias, or fp16 weights."""
        quantized = self.backend.quantized

        def size(p: Linear) -> int:
            return _nbytes(p.qweight, p.scales, p.zeros, p.bias) if quantized else _nbytes(p.w, p.bias)

        layers = sum(size(p) for L in self.layers for p in L.projections())
        return {"linear_layers": layers, "embed": _nbytes(self.embed),
                "lm_head_read": size(self.head_q) if self.head_q is not None else _nbytes(self.lm_head),
                "lm_head_quantized": self.head_q is not None,
                "lm_head_shared_with_embed": self.lm_head.data_ptr() == self.embed.data_ptr()}

    def _row_linear(self, x, p: Linear):
        """o_proj / down: the plain projection, or under tensor parallelism this rank's K-shard
        reduced over the group (fused NVLink allreduce or NCCL)."""
        if self.tp is None:
            return self.backend.linear(x, p)
        return self.tp.reduce_linear(self.backend, x, p)

    def greedy(self, logits: torch.Tensor) -> torch.Tensor:
        """Greedy next token [B] from forward()'s logits [B, T, V] (this rank's vocabulary shard
        under tensor parallelism: the argmax then spans all ranks)."""
        last = logits[:, -1]
        if self.tp is None:
            return last.argmax(-1)
        return self.tp.argmax(last, self.vocab_start)

    # ------------------------------------------------------------------ greedy decode step
    def step_kernel(self):
        """The fused decode-step kernel for this runner (built on first use; set-up synchronizes, so
        the first call must come before any graph capture), or None where it does not apply."""
        if not self.fused_step:
            return None
        if self._step_kernel is None:
            from kernels import step

            if step.supported(self) is not None:
                self.fused_step = False
                return None
            self._step_kernel = step.DecodeStep(self)
        return self._step_kernel

    def _kernel_head(self) -> bool:
        """Does the per-op greedy step end in the lm_head + greedy-pick kernel (kernel backend, one
        rank, fp16 lm_head, batch 1)? Makes its workspace on first use (before any capture)."""
        from kernels import head

        ok = (self.backend.fused_decode and self.tp is None and self.head_q is None and self.batch <= head.RUNNER_ROWS
              and self.embed.dtype == torch.float16 and self.lm_head.dtype == torch.float16
              and self.embed.shape[1] % 8 == 0)
        if ok and self._head_ws is None:
            self._head_ws = head.workspace(self.embed.device)
        return ok

    @torch.no_grad()
    def greedy_step(self, tok: torch.Tensor, pos: torch.Tensor, out: torch.Tensor) -> None:
        """One greedy decode step on device state (the reference's GraphDecoder._step,
        kernels/e2e/run.py:69-74): tok [B, 1] is fed at position pos [1]; the pick is stored in
        out[:, pos] and becomes tok; pos advances. Graph-capturable after a first eager call."""
        fused = self.step_kernel()
        if fused is not None:
            fused(tok, pos, out)
            return
        if self._kernel_head():
            from kernels import head

            B, H = tok.shape[0], self.embed.shape[1]
            x = head.embed_tokens(tok, self.embed)
            h, residual = self._decode_layers(x, pos)
            head.lm_head_greedy(h.reshape(B, H), residual.reshape(B, H), self.final_norm, self.eps, self.lm_head,
                                tok, self._head_ws, pos=pos, history=out)
            return
        pick = self.greedy(self.forward(tok, pos)).view(-1, 1)
        out.index_copy_(1, pos, pick)
        tok.copy_(pick)
        pos.add_(1)

    # ------------------------------------------------------------------ forward
    def _rope_tables(self, positions: torch.Tensor, dtype):
        """cos, sin [len(positions), head_dim] of the reference's RoPE (angles cat(freqs, freqs))."""
        ang = positions[:, None].float() * self.inv_freq[None, :]
        ang = torch.cat((ang, ang), dim=-1)
        return ang.cos().to(dtype).contiguous(), ang.sin().to(dtype).contiguous()

    def _rope(self, x, cos, sin):
        half = self.head_dim // 2
        return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin

    def _attention_sdpa(self, i, qkv, pos, cos, sin, mask, B, T):
        """RoPE, cache write and SDPA over the whole cache, as the reference does
        (reference model.py:236-244)."""
        nq, nkv, hd = self.n_heads, self.n_kv, self.head_dim
        q, k, v = qkv.split([nq * hd, nkv * hd, nkv * hd], dim=-1)
        heads = lambda t, n: t.view(B, T, n, hd).transpose(1, 2)  # noqa: E731
        q, k, v = self._rope(heads(q, nq), cos, sin), self._rope(heads(k, nkv), cos, sin), heads(v, nkv)
        self.k_cache[i].index_copy_(2, pos, k)
        self.v_cache[i].index_copy_(2, pos, v)
        attn = F.scaled_dot_product_attention(q, self.k_cache[i], self.v_cache[i], attn_mask=mask, enable_gqa=True)
        return attn.transpose(1, 2).reshape(B, T, nq * hd)

    def _decode_layers(self, x, pos):
        """T == 1 on the kernel backends: five kernels per layer (norm + qkv, attention, o_proj,
        norm + gate_up + SwiGLU, down). Returns (last MLP output, residual stream)."""
        from kernels.attention import decode_attention

        from kernels.w4a16 import FUSED_NORM_ROWS

        be, eps = self.backend, self.eps
        residual, h = None, x
        # one or two rows on one GPU: down_proj's split-K partial sums go to the next norm + qkv as they are
        split_sums = be.partials and self.tp is None and x.numel() // x.shape[-1] <= FUSED_NORM_ROWS
        parts = part_bias = None
        for i, L in enumerate(self.layers):
            if parts is not None:
                qkv, new_res = be.norm_linear_partials(parts, part_bias, L.ln1, eps, residual, L.qkv)
                qkv, new_res = qkv.view(*x.shape[:-1], -1), new_res.view(x.shape)
            else:
                qkv, new_res = be.norm_linear(h, L.ln1, eps, residual, L.qkv)
            residual = x if residual is None else new_res
            attn = decode_attention(qkv, self.k_cache[i], self.v_cache[i], pos, self.rope_cos, self.rope_sin,
                                    self.n_heads, self.n_kv, static_cache=True)
            act, residual = be.norm_gate_up_act(self._row_linear(attn, L.o), L.ln2, eps, residual, L.gate_up)
            if split_sums and i + 1 < len(self.layers):  # the last layer's output goes to the lm_head as fp16
                parts, part_bias = be.linear_partials(act, L.down), L.down.bias
            else:
                h, parts = self._row_linear(act, L.down), None
        return h, residual

    def _full_layers(self, x, pos, B, T):
        """Any T with the reference's per-op numerics (SDPA over the masked cache,
        reference model.py:216-247). Returns (last MLP output, residual stream)."""
        be, eps = self.backend, self.eps
        cos, sin = self._rope_tables(pos, x.dtype)
        mask = torch.arange(self.max_len, device=x.device)[None, :] <= pos[:, None]  # True = attend
        residual, h = x, None
        for i, L in enumerate(self.layers):
            if h is None:
                h = be.norm(x, L.ln1, eps)
            else:
                h, residual = be.norm(h, L.ln1, eps, residual=residual)
            attn = self._attention_sdpa(i, be.linear(h, L.qkv), pos, cos, sin, mask, B, T)
            h, residual = be.norm(self._row_linear(attn, L.o), L.ln2, eps, residual=residual)
            h = self._row_linear(be.gate_up_act(h, L.gate_up), L.down)
        return h, residual

    @torch.no_grad()
    def forward(self, tokens: torch.Tensor, pos: torch.Tensor, all_logits: bool = False):
        """tokens [B, T]; pos: int64 tensor [T] of absolute positions. Graph-capturable."""
        B, T = tokens.shape
        x = F.embedding(tokens, self.embed)
        if self.backend.fused_decode and T == 1:
            h, residual = self._decode_layers(x, pos)
        else:
            h, residual = self._full_layers(x, pos, B, T)
        h, _ = self.backend.norm(h, self.final_norm, self.eps, residual=residual)
        h = h if all_logits else h[:, -1:]
        return F.linear(h, self.lm_head) if self.head_q is None else self.backend.linear(h, self.head_q)


def random_qwen2(arch: dict, dtype=torch.float16, device="cuda", seed: int = 0):
    """A Hugging Face Qwen2ForCausalLM of the given architecture with seeded random weights
    (normal(0, 0.02) linears and embeddings, HF's own init), built directly on `device`. The
    benchmark configs use random-init weights: no checkpoint is downloaded."""
    import transformers

    arch = dict(arch)
    theta = arch.pop("rope_theta", 10000.0)
    cfg = transformers.Qwen2Config(**arch, rope_parameters={"rope_theta": theta, "rope_type": "default"})
    torch.manual_seed(seed)
    with torch.device(device):
        model = transformers.Qwen2ForCausalLM(cfg)
    return model.to(dtype=dtype).eval()
