"""Tensor parallelism: shard plans, the tensor-parallel runner, and the row-sharded W4A16 projection
with its allreduce fused in (no reference counterpart: the reference is single-GPU).

CPU (`not gpu`): the shard plans of the benchmark models at 1/2/4/8 ranks, and a world-2 gloo run of
the tensor-parallel runner (plain torch ops, NCCL-style allreduce through gloo) against the unsharded
runner. GPU: the fused kernel at world 1 against w4a16_matmul (bit-exact) on one GPU, and at world 2
(two processes, two GPUs) against the unsharded matmul; skipped with fewer GPUs.
"""

import os
import socket

import pytest
import torch

from kernels import config
from kernels.tp import shard_plan

transformers = pytest.importorskip("transformers")


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


# ------------------------------------------------------------------------------------ shard plans
@pytest.mark.parametrize("arch", ["QWEN7", "QWEN15"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plan_covers_model(arch, world):
    a = getattr(config, arch)
    nh, nkv, hd = a["num_attention_heads"], a["num_key_value_heads"], a["head_dim"]
    G = nh // nkv
    plans = [shard_plan(nh, nkv, hd, a["intermediate_size"], a["vocab_size"], world, r) for r in range(world)]
    # query heads: disjoint, in order, covering every head; each rank's heads use its kv heads
    assert plans[0].q_heads[0] == 0 and plans[-1].q_heads[1] == nh
    for p, q in zip(plans, plans[1:]):
        assert p.q_heads[1] == q.q_heads[0]
    for p in plans:
        assert p.n_q >= 1 and p.n_kv >= 1 and p.n_q % p.n_kv == 0
        assert all(p.kv_heads[0] <= h // G < p.kv_heads[1] for h in range(*p.q_heads))
        assert (p.q_heads[0] * hd) % 128 == 0 and (p.q_heads[1] * hd) % 128 == 0
    # MLP columns: whole 128-groups, covering; vocabulary rows: multiples of 8, covering
    for key, total in (("mlp", a["intermediate_size"]), ("vocab", a["vocab_size"])):
        spans = [getattr(p, key) for p in plans]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(x[1] == y[0] for x, y in zip(spans, spans[1:]))
        unit = 128 if key == "mlp" else 8
        assert all(s[0] % unit == 0 and s[1] % unit == 0 and s[1] > s[0] for s in spans)
        assert max(s[1] - s[0] for s in spans) - min(s[1] - s[0] for s in spans) <= unit


def test_shard_plan_qwen7b_tp8_uneven_heads():
    a = config.QWEN7
    sizes = [shard_plan(28, 4, 128, a["intermediate_size"], a["vocab_size"], 8, r).n_q for r in range(8)]
    assert sizes == [3, 4] * 4
    mlp = [shard_plan(28, 4, 128, a["intermediate_size"], a["vocab_size"], 8, r).mlp for r in range(8)]
    assert sorted({(hi - lo) // 128 for lo, hi in mlp}) == [18, 19]


def test_shard_plan_rejects_unshardable():
    with pytest.raises(ValueError):
        shard_plan(28, 4, 128, 18944, 152064, 3, 0)  # 4 kv heads over 3 ranks
    with pytest.raises(ValueError):
        shard_plan(4, 2, 32, 256, 512, 2, 0)  # o_proj shard of 64 columns splits a 128-group
    with pytest.raises(ValueError):
        shard_plan(2, 1, 128, 256, 512, 4, 0)  # 2 query heads over 4 ranks


# ------------------------------------------------------------------------- runner, world 2 on CPU
def tp_model(dtype, device):
    """A tiny Qwen2 whose shapes shard over 2 ranks on 128-wide quantization groups."""
    cfg = transformers.Qwen2Config(
        vocab_size=512, hidden_size=512, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
        num_key_value_heads=2, head_dim=128, max_position_embeddings=256, tie_word_embeddings=False,
        rms_norm_eps=1e-6)
    torch.manual_seed(0)
    return transformers.Qwen2ForCausalLM(cfg).to(device=device, dtype=dtype).eval()


def tp_model_7b_heads(dtype, device):
    """A tiny Qwen2 with Qwen2.5-7B's head layout (28 query / 4 kv heads of 128): at 8 ranks each kv
    head is replicated on 2 ranks, which take 3 and 4 of its 7 query heads."""
    cfg = transformers.Qwen2Config(
        vocab_size=1024, hidden_size=256, intermediate_size=2048, num_hidden_layers=2, num_attention_heads=28,
        num_key_value_heads=4, head_dim=128, max_position_embeddings=256, tie_word_embeddings=False,
        rms_norm_eps=1e-6)
    torch.manual_seed(0)
    return transformers.Qwen2ForCausalLM(cfg).to(device=device, dtype=dtype).eval()


def _runner_worker(rank, world, port, q, arch="tp"):
    import torch.distributed as dist

    from kernels.e2e.model import QwenRunner, make_backend
    from kernels.tp import TensorParallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = tp_model(torch.float32, "cpu") if arch == "tp" else tp_model_7b_heads(torch.float32, "cpu")
        ids = torch.randint(0, 512, (2, 10))  # within both models' vocabularies
        tp = TensorParallel(mode="nccl")
        shard = QwenRunner(model, make_backend("fp16"), max_len=32, batch=2, tp=tp)
        full = QwenRunner(model, make_backend("fp16"), max_len=32, batch=2)
        out, ref = [], []
        lo = shard.forward(ids[:, :8], torch.arange(8), all_logits=True)
        ro = full.forward(ids[:, :8], torch.arange(8), all_logits=True)
        parts = [torch.empty_like(lo) for _ in range(world)]
        dist.all_gather(parts, lo.contiguous())
        out.append(torch.cat(parts, -1))
        ref.append(ro)
        tok_s, tok_f = shard.greedy(lo), full.greedy(ro)
        for t in range(8, 10):  # decode steps on each runner's own greedy token
            lo = shard.forward(tok_s.view(2, 1), torch.tensor([t]))
            ro = full.forward(tok_f.view(2, 1), torch.tensor([t]))
            parts = [torch.empty_like(lo) for _ in range(world)]
            dist.all_gather(parts, lo.contiguous())
            out.append(torch.cat(parts, -1))
            ref.append(ro)
            tok_s, tok_f = shard.greedy(lo), full.greedy(ro)
            assert torch.equal(tok_s, tok_f)
        err = max((a - b).abs().max().item() for a, b in zip(out, ref))
        q.put((rank, err, shard.plan.n_q, shard.plan.n_kv))
    finally:
        dist.destroy_process_group()


def test_tp_runner_world2_gloo_matches_unsharded():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_runner_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    for rank, err, nq, nkv in res:
        assert (nq, nkv) == (2, 1)
        assert err < 1e-4, err


def test_tp_runner_world8_gloo_7b_head_layout():
    """8 ranks on CPU with the 7B head layout (uneven 3/4 query heads per rank, replicated kv heads,
    MLP and vocabulary shards of 2 groups / 128 rows): the same logits and greedy tokens as the
    unsharded runner."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_runner_worker, args=(r, 8, port, q, "7b")) for r in range(8)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(8))
    assert [(nq, nkv) for _, _, nq, nkv in res] == [(3, 1), (4, 1)] * 4
    for rank, err, nq, nkv in res:
        assert err < 1e-4, (rank, err)


# -------------------------------------------------------------------------- fused kernel on GPUs
def _quant_layer(N, K, seed):
    from kernels.quant import quantize_rtn

    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * 0.02).half().cuda()
    return quantize_rtn(w, 128)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,cfg", [
    (1, 1536, 1536, None), (1, 3584, 2432, None), (4, 3584, 512, None), (16, 2048, 1024, None),
    (20, 1536, 1536, None), (1, 1024, 8192, {"SPLIT_K": 4}), (3, 4096, 1024, {"BLOCK_N": 256}),
    (2, 1536, 2048, {"BLOCK_N": 64, "SPLIT_K": 2}),
])
def test_allreduce_world1_matches_matmul(M, N, K, cfg):
    """World 1: pushes to and waits on its own buffer; the result is w4a16_matmul's, bit for bit,
    on repeated calls (the epoch advances every launch) and with a bias."""
    from kernels.tp import TPComm, w4a16_matmul_allreduce
    from kernels.w4a16 import w4a16_matmul

    qw, s, z = _quant_layer(N, K, 1)
    x = torch.randn(M, K, device="cuda").half()
    b = (torch.randn(N, device="cuda") * 0.1).half()
    comm = TPComm(max_n=4096)
    try:
        # the fused kernel is the decode GEMV (16-row launches) with an allreduce epilogue: compare with
        # the same GEMV (above 16 rows w4a16_matmul would otherwise take the tcgen05 small-M kernel)
        ref = w4a16_matmul(x, qw, s, z, bias=b, config={**(cfg or {}), "DECODE_GEMV": True})
        for _ in range(3):
            y = w4a16_matmul_allreduce(x, qw, s, z, comm, bias=b, config=cfg)
            assert torch.equal(y, ref)
        torch.cuda.synchronize()
        from kernels import _lib

        assert _lib.device_error() == 0
    finally:
        comm.close()


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,with_bias", [(17, 1536, 1536, True), (24, 3584, 2432, False), (32, 1536, 9472, True),
                                             (32, 4096, 1024, False)])
def test_allreduce_world1_small_m_tcgen05(M, N, K, with_bias):
    """17..max_m rows run the tcgen05 small-M kernel with the allreduce epilogue in one launch: at world 1
    the result is that kernel's plain output (w4a16_matmul above 16 rows) bit for bit, on repeated
    calls (the epoch advances every launch) and under a CUDA graph."""
    from kernels.bench.harness import capture
    from kernels.tp import TPComm, w4a16_matmul_allreduce
    from kernels.w4a16 import w4a16_matmul

    qw, s, z = _quant_layer(N, K, 4)
    x = torch.randn(M, K, device="cuda").half()
    b = (torch.randn(N, device="cuda") * 0.1).half() if with_bias else None
    comm = TPComm(max_n=4096, max_m=32)
    try:
        ref = w4a16_matmul(x, qw, s, z, bias=b)
        for _ in range(3):
            assert torch.equal(w4a16_matmul_allreduce(x, qw, s, z, comm, bias=b), ref)
        out = {}

        def step():
            out["y"] = w4a16_matmul_allreduce(x, qw, s, z, comm, bias=b)

        step()
        torch.cuda.synchronize()
        graph, _ = capture(step)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out["y"], ref)
        del graph
        from kernels import _lib

        assert _lib.device_error() == 0
    finally:
        comm.close()


@pytest.mark.gpu
def test_allreduce_world1_in_cuda_graph():
    from kernels.bench.harness import capture
    from kernels.tp import TPComm, w4a16_matmul_allreduce
    from kernels.w4a16 import w4a16_matmul

    qw, s, z = _quant_layer(1536, 8960, 2)
    x = torch.randn(1, 8960, device="cuda").half()
    comm = TPComm(max_n=1536)
    try:
        ref = w4a16_matmul(x, qw, s, z)
        out = {}

        def step():
            out["y"] = w4a16_matmul_allreduce(x, qw, s, z, comm)

        step()
        torch.cuda.synchronize()
        graph, _ = capture(step)
        for _ in range(5):
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out["y"], ref)
        del graph
    finally:
        comm.close()


@pytest.mark.gpu
def test_allreduce_rejects_oversize():
    from kernels.tp import TPComm, w4a16_matmul_allreduce

    qw, s, z = _quant_layer(2048, 1024, 3)
    comm = TPComm(max_n=1024)
    try:
        with pytest.raises(RuntimeError, match="max_n"):
            w4a16_matmul_allreduce(torch.randn(1, 1024, device="cuda").half(), qw, s, z, comm)
    finally:
        comm.close()


def _fused_worker(rank, world, port, q):
    import torch.distributed as dist

    from kernels.tp import TPComm, w4a16_matmul_allreduce
    from kernels.w4a16 import w4a16_matmul

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = None
    try:
        comm = TPComm(max_n=4096, max_m=32)
        results = []
        # 17-32 rows: the tcgen05 small-M kernel with the allreduce epilogue, one launch
        for M, N, K in ((1, 3584, 2048), (4, 1536, 1024), (16, 2048, 2048), (1, 1024, 8192), (24, 1536, 2048),
                        (32, 3584, 4096)):
            qw, s, z = _quant_layer(N, K, 7)  # the same full layer on every rank
            g = torch.Generator().manual_seed(11)
            x = torch.randn(M, K, generator=g).half().cuda()
            b = (torch.randn(N, generator=g) * 0.1).half().cuda()
            ref = w4a16_matmul(x, qw, s, z, bias=b, config={"FACTORED": False})
            k0, k1 = rank * K // world, (rank + 1) * K // world
            xs = x[:, k0:k1].contiguous()
            y = None
            for _ in range(3):
                y = w4a16_matmul_allreduce(xs, qw[k0 // 8:k1 // 8].contiguous(), s[k0 // 128:k1 // 128].contiguous(),
                                           z[k0 // 128:k1 // 128].contiguous(), comm, bias=b)
            torch.cuda.synchronize()
            err = ((y.float() - ref.float()).abs() - (2e-3 + 2e-2 * ref.float().abs())).max().item()
            ys = [torch.empty_like(y.cpu()) for _ in range(world)]
            dist.all_gather(ys, y.cpu())
            same = all(torch.equal(ys[0], t) for t in ys)
            results.append((M, N, K, err, same))
        from kernels import _lib

        q.put((rank, results, _lib.device_error()))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_allreduce_wait_runs_out_when_the_peer_never_launches():
    """The fused allreduce's bounded wait, made to run out on ONE GPU with no second process: a
    world-2 communicator whose rank-1 buffer is a second local buffer that no kernel ever pushes
    into (a peer that never launches). With the bound set to 50 ms through the C ABI, every CTA
    gives up waiting for rank 1's partial sums, leaves its columns unwritten, records
    DK_DEVERR_TP_WAIT and returns; the context stays usable for the next launch."""
    import ctypes
    import time

    from _util import to_cuda, w4_case
    from kernels import _lib
    from kernels.tp import TPComm, w4a16_matmul_allreduce

    lib = _lib.lib()
    N, K = 1024, 512
    nbytes = ctypes.c_uint64(0)
    _lib.check(lib.dk_tp_buffer_bytes(2, 16, N, ctypes.byref(nbytes)), "tp_buffer_bytes")
    bufs = [ctypes.c_void_p(), ctypes.c_void_p()]
    for b in bufs:
        _lib.check(lib.dk_tp_buffer_alloc(nbytes.value, ctypes.byref(b), ctypes.create_string_buffer(64)), "alloc")
    comm = ctypes.c_void_p()
    try:
        ptrs = (ctypes.c_void_p * 2)(bufs[0].value, bufs[1].value)
        _lib.check(lib.dk_tp_comm_create(ctypes.byref(comm), 0, 2, ptrs, 16, N), "comm_create")
        assert lib.dk_tp_comm_set_wait(comm, 100) == -1  # below 1 ms: rejected
        _lib.check(lib.dk_tp_comm_set_wait(comm, 50_000_000), "comm_set_wait")

        class Comm:
            handle = comm

        x, qw, s, z = to_cuda(*w4_case(2, N, K, seed=11)[:4])
        _lib.clear_device_error()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        y = w4a16_matmul_allreduce(x, qw, s, z, Comm)
        err = _lib.device_error()  # synchronizes: the launch has returned
        elapsed = time.perf_counter() - t0
        assert err == 4, err  # DK_DEVERR_TP_WAIT
        assert elapsed < 5.0, elapsed
        del y  # its columns were left unwritten
        _lib.clear_device_error()
    finally:
        if comm.value:
            lib.dk_tp_comm_destroy(comm)
        for b in bufs:
            lib.dk_tp_buffer_free(b)
    # the context still runs kernels: a one-rank communicator gives the plain matmul's result
    one = TPComm(max_n=N)
    try:
        from kernels.w4a16 import w4a16_matmul

        torch.testing.assert_close(w4a16_matmul_allreduce(x, qw, s, z, one), w4a16_matmul(x, qw, s, z),
                                   rtol=0, atol=0)
    finally:
        one.close()
    assert _lib.device_error() == 0


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_allreduce_world2_matches_unsharded():
    """Two processes on two GPUs, each with half of K: both get the unsharded matmul (within the
    matmul tolerance rtol 2e-2 / atol 2e-3) and the same bits as each other."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for _ in range(2):
        rank, results, deverr = q.get(timeout=5)
        assert deverr == 0
        for M, N, K, err, same in results:
            assert err <= 0, (rank, M, N, K, err)
            assert same, (rank, M, N, K)


# ------------------------------------------------------------------------------ runner on GPUs
@pytest.mark.gpu
def test_tp_runner_world1_fused_is_the_plain_runner():
    """World 1: the tensor-parallel runner (a one-rank group reduces nothing: the plain projections)
    decodes the same tokens with the same logits as the unsharded runner, eagerly and under the CUDA
    graph. The fused kernel itself at world 1 is tested above, against the plain matmul."""
    from kernels.e2e.model import QwenRunner, make_backend
    from kernels.e2e.run import GraphDecoder
    from kernels.tp import TensorParallel

    model = tp_model(torch.float16, "cuda")
    ids = torch.randint(0, 512, (2, 20), generator=torch.Generator().manual_seed(5)).cuda()
    tp = TensorParallel(mode="fused")
    try:
        shard = QwenRunner(model, make_backend("ours_lm"), max_len=64, batch=2, tp=tp)
        plain = QwenRunner(model, make_backend("ours_lm"), max_len=64, batch=2)
        pos = torch.arange(20, device="cuda")
        assert torch.equal(shard.forward(ids, pos), plain.forward(ids, pos))
        toks = []
        for r in (shard, plain):
            dec = GraphDecoder(r)
            dec.capture(ids)
            toks.append(dec.generate(ids, 12)[0])
        assert toks[0] == toks[1]
        from kernels import _lib

        assert _lib.device_error() == 0
    finally:
        tp.close()


def _runner_gpu_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from kernels.e2e.model import QwenRunner, make_backend
    from kernels.e2e.run import GraphDecoder
    from kernels.tp import TensorParallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    tp = None
    try:
        model = tp_model(torch.float16, "cuda")
        ids = torch.randint(0, 512, (2, 20), generator=torch.Generator().manual_seed(5)).cuda()
        pos = torch.arange(20, device="cuda")
        plain = QwenRunner(model, make_backend("ours_lm"), max_len=64, batch=2)
        ref = plain.forward(ids, pos).float()
        tp = TensorParallel(mode="fused")
        shard = QwenRunner(model, make_backend("ours_lm"), max_len=64, batch=2, tp=tp)
        out = {}
        for mode in ("fused", "nccl"):
            tp.mode = mode
            lo = shard.forward(ids, pos)
            parts = [torch.empty_like(lo) for _ in range(world)]
            dist.all_gather(parts, lo.contiguous())
            full = torch.cat(parts, -1).float()
            dec = GraphDecoder(shard)
            dec.capture(ids)
            toks = dec.generate(ids, 12)[0]
            out[mode] = ((full - ref).abs().max().item(), bool(torch.equal(full.argmax(-1), ref.argmax(-1))), toks)
            del dec
        pdec = GraphDecoder(plain)
        pdec.capture(ids)
        out["plain_tokens"] = pdec.generate(ids, 12)[0]
        from kernels import _lib

        q.put((rank, out, _lib.device_error()))
    finally:
        if tp is not None:
            tp.close()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_runner_world2_matches_unsharded():
    """Two ranks on two GPUs (fused NVLink allreduce, then NCCL): logits of the sharded runner match
    the unsharded runner's and the greedy continuation under CUDA graphs is the same."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_runner_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for _ in range(2):
        rank, out, deverr = q.get(timeout=5)
        assert deverr == 0
        for mode in ("fused", "nccl"):
            err, same_argmax, toks = out[mode]
            assert err < 5e-2, (rank, mode, err)
            assert same_argmax, (rank, mode)
            assert toks == out["plain_tokens"], (rank, mode)


def _argmax_worker(rank, world, port, q):
    import torch.distributed as dist

    from kernels.tp import TensorParallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        V = 24  # 12 vocabulary rows per rank
        full = torch.tensor([
            [0.0] * V,                                  # all equal: index 0
            [1.0 if i in (5, 17) else 0.0 for i in range(V)],   # tie across ranks: 5
            [2.0 if i in (14, 19) else 0.0 for i in range(V)],  # tie inside rank 1: 14
            [float(i % 7) for i in range(V)],           # max 6 at 6 (rank 0), 13 and 20 (rank 1): 6
        ], dtype=torch.float16)
        lo = full[:, rank * 12:(rank + 1) * 12]
        got = TensorParallel(mode="nccl").argmax(lo, rank * 12)
        q.put((rank, got.tolist(), full.argmax(-1).tolist()))
    finally:
        dist.destroy_process_group()


def test_tp_argmax_ties_match_full_row():
    """The cross-rank greedy token equals torch.argmax over the whole row, ties included (lowest
    vocabulary index wins, within a rank and across ranks)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_argmax_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for _ in range(2):
        rank, got, want = q.get(timeout=5)
        assert got == want == [0, 5, 14, 6], (rank, got, want)


# --------------------------------------------------------------- communicator set-up failure (CPU)
class _FakeTpLib:
    """Stands in for libdecodek's TP set-up entry points: allocation succeeds, mapping the peer
    `fail_peer` fails; records what was allocated, mapped, closed and freed."""

    def __init__(self, fail_peer):
        self.fail_peer, self.log = fail_peer, []

    def dk_tp_buffer_bytes(self, world, max_m, max_n, out):
        out._obj.value = 256 + 2 * world * max_m * max_n * 8
        return 0

    def dk_tp_buffer_alloc(self, nbytes, out, handle):
        out._obj.value = 0x1000
        handle.raw = b"\x00" * 64
        self.log.append("alloc")
        return 0

    def dk_tp_buffer_open(self, handle, out):
        peer = handle.raw[0]
        if peer == self.fail_peer:
            return -3
        out._obj.value = 0x2000 + peer
        self.log.append(f"open{peer}")
        return 0

    def dk_tp_buffer_close(self, p):
        self.log.append(f"close{p.value - 0x2000}")
        return 0

    def dk_tp_buffer_free(self, p):
        self.log.append("free")
        return 0

    def dk_tp_comm_create(self, *a):
        self.log.append("create")
        return 0

    def dk_last_error(self):
        return b"cannot map the peer's buffer"


def test_tpcomm_setup_failure_releases_buffers(monkeypatch):
    """A rank whose mapping of a peer's exchange buffer fails closes the mappings made so far, frees
    its own buffer and raises (a fake library and a fake 4-rank group on the CPU)."""
    import contextlib

    import torch.distributed as dist

    from kernels import _lib
    from kernels.tp import TPComm

    fake = _FakeTpLib(fail_peer=3)
    monkeypatch.setattr(_lib, "lib", lambda: fake)
    monkeypatch.setattr(torch.cuda, "device", lambda d: contextlib.nullcontext())
    monkeypatch.setattr(dist, "is_initialized", lambda: True)
    monkeypatch.setattr(dist, "get_rank", lambda group=None: 0)
    monkeypatch.setattr(dist, "get_world_size", lambda group=None: 4)

    def gather(out, obj, group=None):  # rank q's handle starts with the byte q
        for q in range(len(out)):
            out[q] = bytes([q]) + obj[1:]

    monkeypatch.setattr(dist, "all_gather_object", gather)
    monkeypatch.setattr(dist, "barrier", lambda group=None: None)
    with pytest.raises(RuntimeError, match="tp_buffer_open: cannot map"):
        TPComm(max_n=64, device="cuda:0")
    assert fake.log == ["alloc", "open1", "open2", "close1", "close2", "free"]


# ------------------------------------------------ failure detection on the host (CPU, gloo ranks)
def _departing_rank_worker(rank, world, port, q):
    """Both ranks run one sharded decode step; rank 1 then leaves (between steps, nothing in flight)
    and rank 0 tries the next step. Its first collective must fail within the process group's
    timeout instead of waiting for good."""
    import datetime
    import time

    import torch.distributed as dist

    from kernels.e2e.model import QwenRunner, make_backend
    from kernels.tp import TensorParallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    model = tp_model(torch.float32, "cpu")
    ids = torch.randint(0, 512, (1, 6), generator=torch.Generator().manual_seed(1))
    shard = QwenRunner(model, make_backend("fp16"), max_len=16, batch=1, tp=TensorParallel(mode="nccl"))
    tok = shard.greedy(shard.forward(ids, torch.arange(6)))
    dist.barrier()
    if rank == 1:
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()  # the message is on the pipe before the process goes
        os._exit(0)  # leaves without a word: no destroy_process_group, no more collectives
    time.sleep(1.0)
    t0 = time.perf_counter()
    try:
        shard.forward(tok.view(1, 1), torch.tensor([6]))
        q.put((rank, "no error", time.perf_counter() - t0))
    except Exception as e:  # the collective reports the departed peer
        q.put((rank, type(e).__name__, time.perf_counter() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_departed_rank_is_detected_by_the_next_collective():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_departing_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict((r, (what, sec)) for r, what, sec in (q.get(timeout=5) for _ in range(2)))
    assert got[1][0] == "left"
    what, sec = got[0]
    assert what != "no error", "the surviving rank's collective did not notice the departed rank"
    assert sec < 60, f"detection took {sec:.1f} s"
