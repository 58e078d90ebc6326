"""Tensor parallelism for the decode path: shard plans, the NVLink communicator, and the row-sharded
W4A16 projection with its allreduce fused in.

No reference counterpart: the reference runs one GPU (README.md:249). The layout follows the usual
Megatron split of a Qwen2 layer, one process per GPU of one node:

* column-sharded (split N, no exchange): qkv by heads, gate_up (gate and up split separately and
  each rank's halves concatenated), lm_head by vocabulary rows;
* row-sharded (split K, one allreduce of [M, hidden]): o_proj (K = this rank's query heads) and
  down (K = this rank's MLP columns).

K splits land on 128-wide quantization groups, so a shard's packed weights, scales and zeros are
exactly the corresponding slices of the unsharded quantization (groups never straddle ranks).

`TPComm` owns one exchange buffer per rank, mapped into every peer with CUDA IPC;
`w4a16_matmul_allreduce` is one kernel (per 16 rows on the decode GEMV, up to 64 rows in one tcgen05
small-M launch) that computes this rank's partial sums, pushes
them into every rank's buffer over NVLink and adds the ranks' partials of its own columns in rank
order (every rank gets the same bits). `TensorParallel` is what the runner calls: the fused kernel,
or an NCCL allreduce after the plain kernel (`mode="nccl"`, the library baseline), and the
cross-rank greedy argmax over vocabulary shards.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from kernels import _lib

GROUP = 128


# ------------------------------------------------------------------------------------ shard plans
@dataclass(frozen=True)
class ShardPlan:
    """This rank's slices: [start, end) of query heads, kv heads, MLP columns and vocabulary rows."""

    rank: int
    world: int
    q_heads: tuple[int, int]
    kv_heads: tuple[int, int]
    mlp: tuple[int, int]
    vocab: tuple[int, int]

    @property
    def n_q(self) -> int:
        return self.q_heads[1] - self.q_heads[0]

    @property
    def n_kv(self) -> int:
        return self.kv_heads[1] - self.kv_heads[0]


def _even(n: int, parts: int, i: int) -> tuple[int, int]:
    """[start, end) of part i when n items are split into `parts` nearly equal contiguous parts."""
    return (i * n) // parts, ((i + 1) * n) // parts


def shard_plan(n_heads: int, n_kv: int, head_dim: int, intermediate: int, vocab: int, world: int, rank: int,
               group: int = GROUP) -> ShardPlan:
    """Head, MLP and vocabulary slices of `rank` out of `world`.

    kv heads: n_kv % world == 0 -> n_kv / world each with their query heads; world % n_kv == 0 ->
    each kv head is replicated on world / n_kv ranks, which split its query heads as evenly as
    possible (Qwen2.5-7B at 8 ranks: 7 query heads per kv head -> 3 and 4). MLP columns: split in
    whole quantization groups (18944 = 148 groups -> 19 or 18 groups per rank at 8). Vocabulary:
    split in multiples of 8 rows (the W4A16 kernel's column alignment)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n_heads % n_kv:
        raise ValueError("query heads must be a multiple of kv heads")
    G = n_heads // n_kv
    if n_kv % world == 0:
        kv0, kv1 = _even(n_kv, world, rank)
        q = (kv0 * G, kv1 * G)
    elif world % n_kv == 0:
        reps = world // n_kv
        if G < reps:
            raise ValueError(f"{G} query heads per kv head cannot be split over {reps} ranks")
        kv = rank // reps
        a, b = _even(G, reps, rank % reps)
        kv0, kv1 = kv, kv + 1
        q = (kv * G + a, kv * G + b)
    else:
        raise ValueError(f"{n_kv} kv heads cannot be sharded over {world} ranks")
    if (q[0] * head_dim) % group or (q[1] * head_dim) % group:
        raise ValueError("o_proj row shards must fall on quantization group boundaries")
    if intermediate % group:
        raise ValueError("intermediate size must be a multiple of the group size")
    g0, g1 = _even(intermediate // group, world, rank)
    if vocab % 8:
        raise ValueError("vocabulary must be a multiple of 8")
    v0, v1 = _even(vocab // 8, world, rank)
    return ShardPlan(rank, world, q, (kv0, kv1), (g0 * group, g1 * group), (v0 * 8, v1 * 8))


def plan_for(cfg, world: int, rank: int) -> ShardPlan:
    """shard_plan for a Hugging Face Qwen2 config."""
    hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    return shard_plan(cfg.num_attention_heads, cfg.num_key_value_heads, hd, cfg.intermediate_size,
                      cfg.vocab_size, world, rank)


# ----------------------------------------------------------------------------------- communicator
class TPComm:
    """The NVLink exchange buffers of one tensor-parallel group (set-up: allocates, maps, syncs).

    Every rank allocates one buffer (two slots of epoch-tagged partial sums of launches up to `max_m`
    rows x `max_n` columns per rank, behind a header holding the launch epoch and an arrival count),
    exports its CUDA IPC handle, gathers the others' over `group` and maps them. If set-up fails on
    this rank, what it allocated or mapped is released before the error propagates. With group None and no process group initialized, a single-rank communicator (world 1):
    the fused kernel then pushes to and waits on its own buffer only."""

    def __init__(self, max_n: int, max_m: int = 16, group=None, device=None):
        import torch.distributed as dist

        self.dist = dist.is_available() and dist.is_initialized()
        self.group = group
        self.rank = dist.get_rank(group) if self.dist else 0
        self.world = dist.get_world_size(group) if self.dist else 1
        self.max_m, self.max_n = int(max_m), int(max_n)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.handle = None
        self._own = None
        self._opened = []
        lib = _lib.lib()
        try:
            self._setup(lib, dist, group)
        except BaseException:
            self._release(lib)  # this rank's mappings and buffer; the peers fail at their next collective
            raise
        if self.world > 1:
            dist.barrier(group=group)

    def _setup(self, lib, dist, group) -> None:
        nbytes = ctypes.c_uint64(0)
        _lib.check(lib.dk_tp_buffer_bytes(self.world, self.max_m, self.max_n, ctypes.byref(nbytes)), "tp_buffer_bytes")
        handle = ctypes.create_string_buffer(64)
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.dk_tp_buffer_alloc(nbytes.value, ctypes.byref(own), handle), "tp_buffer_alloc")
        self._own = own
        handles = [bytes(handle.raw)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.raw), group=group)
        ptrs = (ctypes.c_void_p * self.world)()
        with torch.cuda.device(self.device):
            for q in range(self.world):
                if q == self.rank:
                    ptrs[q] = own.value
                    continue
                p = ctypes.c_void_p()
                _lib.check(lib.dk_tp_buffer_open(ctypes.create_string_buffer(handles[q], 64), ctypes.byref(p)),
                           "tp_buffer_open")
                self._opened.append(p)
                ptrs[q] = p.value
        comm = ctypes.c_void_p()
        _lib.check(lib.dk_tp_comm_create(ctypes.byref(comm), self.rank, self.world, ptrs, self.max_m, self.max_n),
                   "tp_comm_create")
        self.handle = comm

    def _release(self, lib) -> None:
        if self.handle is not None:
            lib.dk_tp_comm_destroy(self.handle)
            self.handle = None
        if self._opened or self._own is not None:
            with torch.cuda.device(self.device):
                for p in self._opened:
                    lib.dk_tp_buffer_close(p)
                if self._own is not None:
                    lib.dk_tp_buffer_free(self._own)
        self._opened = []
        self._own = None

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a barrier: no peer may still write)."""
        if self.handle is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            self.dist_barrier()
        self._release(_lib.lib())

    def dist_barrier(self) -> None:
        import torch.distributed as dist

        dist.barrier(group=self.group)


def w4a16_matmul_allreduce(x, qweight, scales, zeros, comm: TPComm, group_size=128, bias=None, config=None):
    """Row-sharded w4a16_matmul with the allreduce fused in: every rank passes its K-shard of x
    [..., K_r] and of the weight and gets y = fp16(sum over ranks of x_r @ dequant(W_r).T + bias),
    identical on every rank. All ranks must make the same calls in the same order."""
    from kernels.w4a16 import _check_weight_shapes, _config

    K = x.shape[-1]
    N = qweight.shape[1]
    _lib.reference_assert(qweight.shape[0] * 8 == K and K % group_size == 0)
    _check_weight_shapes("w4a16_matmul_allreduce", K, N, scales, zeros, group_size, bias)
    _lib.require_cuda("w4a16_matmul_allreduce", x, qweight, scales, zeros, bias)
    _lib.require_dtype("w4a16_matmul_allreduce", torch.float16, x, scales, zeros, bias)
    _lib.require_dtype("w4a16_matmul_allreduce", torch.int32, qweight)
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    qweight, scales, zeros = qweight.contiguous(), scales.contiguous(), zeros.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    cfg = _config(config)
    _lib.call("dk_w4a16_matmul_allreduce", _lib.ptr(x2), x2.stride(0), _lib.ptr(qweight), _lib.ptr(scales),
              _lib.ptr(zeros), _lib.ptr(bias), _lib.ptr(out), out.stride(0), M, N, K, group_size,
              ctypes.byref(cfg), comm.handle, _lib.stream_of(x))
    return out.view(*x.shape[:-1], N)


# --------------------------------------------------------------------------------- runner interface
class TensorParallel:
    """What a tensor-parallel runner needs from its group: the shard plan, the reduction of a
    row-sharded projection, and the greedy argmax over vocabulary shards.

    mode "fused": w4a16_matmul_allreduce (quantized kernel backends; up to 16 rows on the decode GEMV,
    17-32 rows on the tcgen05 small-M kernel, each with the allreduce in its epilogue).
    mode "nccl": the backend's own projection, then torch.distributed.all_reduce of the fp16 output
    (any backend, any device: the baseline and the CPU/gloo path)."""

    def __init__(self, group=None, mode: str = "fused"):
        import torch.distributed as dist

        if mode not in ("fused", "nccl"):
            raise ValueError(f"mode {mode!r}")
        self.dist = dist.is_available() and dist.is_initialized()
        self.group = group
        self.rank = dist.get_rank(group) if self.dist else 0
        self.world = dist.get_world_size(group) if self.dist else 1
        self.mode = mode
        self.comm: TPComm | None = None

    def plan(self, cfg) -> ShardPlan:
        return plan_for(cfg, self.world, self.rank)

    def setup(self, hidden: int, device) -> None:
        if self.mode == "fused" and self.comm is None:
            self.comm = TPComm(max_n=hidden, max_m=self.FUSED_MAX_ROWS, group=self.group, device=device)

    # rows up to which the projection carries its allreduce: the decode GEMV up to 16 rows, the tcgen05
    # small-M kernel (one pass over the weights) from 17 to 32; prefill-sized inputs use the GEMM plus
    # NCCL
    FUSED_MAX_ROWS = 32

    def reduce_linear(self, be, x, p):
        """sum over ranks of the row-sharded projection p of x (+ p.bias once)."""
        rows = x.numel() // x.shape[-1]
        if self.world == 1:  # nothing to reduce: the plain projection
            return be.linear(x, p)
        if (self.mode == "fused" and self.comm is not None and p.qweight is not None and p.zeros is not None
                and rows <= self.FUSED_MAX_ROWS):
            return w4a16_matmul_allreduce(x, p.qweight, p.scales, p.zeros, self.comm, bias=p.bias,
                                          config=getattr(be, "LINEAR_CFG", None))
        bias = p.bias
        if bias is not None and self.rank != 0:  # the bias is added once
            p = type(p)(**{**p.__dict__, "bias": None})
        y = be.linear(x, p)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(y, group=self.group)
        return y

    def argmax(self, logits: torch.Tensor, vocab_start: int) -> torch.Tensor:
        """Greedy token over the vocabulary shards: logits [B, V_r] of this rank (columns
        vocab_start..). Ties go to the lowest global index, as torch.argmax over the full row."""
        idx = logits.argmax(-1)
        val = logits.gather(-1, idx[..., None]).squeeze(-1).float()
        if self.world == 1:
            return idx + vocab_start
        import torch.distributed as dist

        mine = torch.stack([val, (idx + vocab_start).float()], -1)  # [B, 2]; ids < 2^24 are exact
        if mine.is_cuda:
            allv = torch.empty((self.world,) + tuple(mine.shape), dtype=mine.dtype, device=mine.device)
            dist.all_gather_into_tensor(allv, mine.contiguous(), group=self.group)
        else:
            parts = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(parts, mine.contiguous(), group=self.group)
            allv = torch.stack(parts)
        best = allv[..., 0].argmax(0)  # first maximal rank = lowest vocabulary index
        return allv[..., 1].gather(0, best[None]).squeeze(0).long()

    def close(self) -> None:
        if self.comm is not None:
            self.comm.close()
            self.comm = None
