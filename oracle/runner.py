"""CPU restatement of the reference's Qwen2 decode runner with dequantize-then-matmul linears.
TEST INFRASTRUCTURE AND CPU BASELINE ONLY (never the product path).

Follows kernels/e2e/model.py:216-253 (layer structure, fused residual+RMSNorm, fused qkv and
gate_up, RoPE, GQA attention over positions 0..pos, tied lm_head) with the linears of
kernels/reference.py:39-45 (`x.float() @ dequant(W).float().t()`): every weight is dequantized once
(oracle.torch_ref, bit-exact with the reference's dequantization) and kept in fp32; activations stay fp32 (the
reference's CPU path computes its matmuls in fp32). Used to time the reference's CPU path on the
benchmark model and, on the tiny model, pinned against the reference runner's golden logits.
"""

from __future__ import annotations

import math

import numpy as np
import torch

import oracle
from oracle import torch_ref


class OracleRunner:
    """weights: dict with `embed` [V, H], `final_norm` [H], optional `lm_head` [V, H] (tied if absent),
    and per layer `ln1`, `ln2`, `qkv`, `qkv_bias`, `o`, `gate_up`, `down` where each linear is either
    a dense fp16/fp32 [N, K] array or a tuple (qweight, scales, zeros) of the packed int4 format."""

    def __init__(self, weights: dict, n_heads: int, n_kv: int, head_dim: int, eps: float, theta: float,
                 max_len: int, threads: int | None = None):
        if threads:
            torch.set_num_threads(threads)
        self.nq, self.nkv, self.hd, self.eps, self.max_len = n_heads, n_kv, head_dim, eps, max_len

        def dense(w):
            if isinstance(w, tuple):  # torch restatement of the dequantization: same bits, all cores
                qw, s, z = (torch.as_tensor(np.asarray(a)) for a in w)
                return torch_ref.dequantize(qw, s, z, 128).float().contiguous()
            return torch.as_tensor(np.asarray(w, dtype=np.float32))

        f32 = lambda a: torch.as_tensor(np.asarray(a, dtype=np.float32))  # noqa: E731
        self.embed = f32(weights["embed"])
        self.lm_head = dense(weights["lm_head"]) if weights.get("lm_head") is not None else self.embed
        self.final_norm = f32(weights["final_norm"])
        self.layers = []
        for L in weights["layers"]:
            self.layers.append({
                "ln1": f32(L["ln1"]), "ln2": f32(L["ln2"]), "qkv": dense(L["qkv"]),
                "qkv_bias": None if L.get("qkv_bias") is None else f32(L["qkv_bias"]),
                "o": dense(L["o"]), "gate_up": dense(L["gate_up"]), "down": dense(L["down"]),
            })
        self.inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        n = len(self.layers)
        self.k = torch.zeros(n, n_kv, max_len, head_dim)
        self.v = torch.zeros(n, n_kv, max_len, head_dim)

    def _norm(self, x, w):
        return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps))

    def _rope(self, x, cos, sin):
        h = self.hd // 2
        return x * cos + torch.cat((-x[..., h:], x[..., :h]), dim=-1) * sin

    @torch.no_grad()
    def step(self, token: int, pos: int) -> torch.Tensor:
        """One decode token at position `pos`; returns fp32 logits [V]."""
        nq, nkv, hd = self.nq, self.nkv, self.hd
        x = self.embed[token]
        f = pos * self.inv_freq
        emb = torch.cat((f, f))
        cos, sin = emb.cos(), emb.sin()
        residual, h = x, None
        for i, L in enumerate(self.layers):
            if h is None:
                h = self._norm(x, L["ln1"])
            else:
                residual = residual + h
                h = self._norm(residual, L["ln1"])
            qkv = L["qkv"] @ h
            if L["qkv_bias"] is not None:
                qkv = qkv + L["qkv_bias"]
            q = self._rope(qkv[: nq * hd].view(nq, hd), cos, sin)
            k = self._rope(qkv[nq * hd:(nq + nkv) * hd].view(nkv, hd), cos, sin)
            v = qkv[(nq + nkv) * hd:].view(nkv, hd)
            self.k[i, :, pos] = k
            self.v[i, :, pos] = v
            K = self.k[i, :, : pos + 1].repeat_interleave(nq // nkv, 0)  # [nq, pos+1, hd]
            V = self.v[i, :, : pos + 1].repeat_interleave(nq // nkv, 0)
            s = torch.einsum("hd,hjd->hj", q, K) / math.sqrt(hd)
            attn = torch.einsum("hj,hjd->hd", torch.softmax(s, -1), V).reshape(-1)
            o = L["o"] @ attn
            residual = residual + o
            h = self._norm(residual, L["ln2"])
            gu = L["gate_up"] @ h
            I = gu.shape[0] // 2
            h = L["down"] @ (torch.nn.functional.silu(gu[:I]) * gu[I:])
        h = self._norm(residual + h, self.final_norm)
        return self.lm_head @ h


def weights_from_hf(model, quantized: bool = True, quant_lm_head: bool = False) -> dict:
    """Weights of a Hugging Face Qwen2 model in OracleRunner's format, int4-quantized by the oracle
    (fused qkv and gate_up as kernels/e2e/model.py:168-191)."""
    def npy(t):
        return t.detach().float().cpu().numpy()

    def lin(*mods):
        w = np.concatenate([mm.weight.detach().cpu().half().numpy() for mm in mods], 0)
        return oracle.quantize_rtn(w, 128) if quantized else w.astype(np.float32)

    m = model.model
    layers = []
    for layer in m.layers:
        a, mlp = layer.self_attn, layer.mlp
        bias = None if a.q_proj.bias is None else np.concatenate([npy(x.bias) for x in (a.q_proj, a.k_proj, a.v_proj)])
        layers.append({"ln1": npy(layer.input_layernorm.weight), "ln2": npy(layer.post_attention_layernorm.weight),
                       "qkv": lin(a.q_proj, a.k_proj, a.v_proj), "qkv_bias": bias, "o": lin(a.o_proj),
                       "gate_up": lin(mlp.gate_proj, mlp.up_proj), "down": lin(mlp.down_proj)})
    tied = model.lm_head.weight.data_ptr() == m.embed_tokens.weight.data_ptr()
    return {"embed": npy(m.embed_tokens.weight), "final_norm": npy(m.norm.weight), "layers": layers,
            "lm_head": lin(model.lm_head) if quant_lm_head else (None if tied else npy(model.lm_head.weight))}
