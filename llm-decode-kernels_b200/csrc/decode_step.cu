// One greedy decode step of a Qwen2 model as ONE persistent kernel (batch 1..4 rows).
//
// Replaces, for T == 1, the per-op launches of the runner's decode step (the reference's
// kernels/e2e/model.py:216-253 forward plus the greedy pick and bookkeeping of
// kernels/e2e/run.py:69-74): embedding lookup, per layer the fused residual + RMSNorm + qkv
// projection, RoPE + KV-cache append + attention over positions 0..pos, o_proj, the fused residual +
// RMSNorm + gate_up projection + SwiGLU, down_proj; then the final norm, the fp16 lm_head, the
// greedy argmax, the token feedback and the position bump.
//
// Why one kernel. At batch 1 every op is a few MB or less: launches are latency chains (kernel
// boundary, activation staging, the weight fetch, reduction, store), not bandwidth. The weights are
// static, so they do not have to wait for the activations that multiply them:
// * one CTA per SM (cooperative launch: all CTAs resident), 8 consumer warps and a producer warp
//   (whose warpgroup hands most of its registers to the consumers: setmaxnreg);
// * the producer warp walks the whole step's program and streams this CTA's share of every op's
//   weights (and of the KV cache rows before `pos`) into a shared-memory ring with TMA, gated only by
//   free ring slots - it runs ahead across op and layer boundaries, so an op's weights are usually
//   on chip before its input exists;
// * the consumer warps run the ops in order. Activations between ops are tagged words: each fp16
//   value travels with a 16-bit tag (each fp32 partial with a 32-bit tag) in one 4-byte (8-byte) store,
//   the tag naming the step and the op that wrote it (the low-latency protocol of NCCL, which this
//   library's fused allreduce also uses). A consumer polls the words it needs until their tags match:
//   no fence, no arrival counter and no flag between ops. It stages the input in shared memory (with
//   the fused residual add + RMSNorm where the model has one), multiplies it with the weights already
//   in the ring (mma.m16n8k16, fp32 accumulation, the int4 "magic number" unpack of the standalone
//   GEMV kernel), reduces across warps in a fixed order and stores its tagged output;
// * attention is split over (sequence, kv head, 128-position slice) items; each CTA combines its 8
//   warps' partials into one tagged partial per head, and the o_proj CTAs combine the slices while
//   they stage their input. The greedy argmax is combined by the last CTA to arrive on a counter.
// Every wait is bounded (2 s); a CTA that gives up records DK_DEVERR_STEP_WAIT and skips the rest of
// its work (the others then give up on its words in turn), but still arrives on the counters it uses,
// so they stay consistent for the next launch. No TMA multicast.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

struct dk_step_plan;

namespace dk {
namespace step {

constexpr int kCWarps = 8;                    // consumer warps
constexpr int kConsumers = kCWarps * 32;
constexpr int kThreads = kConsumers + 128;    // + one warpgroup: the producer warp and 3 idle warps
// Register split (setmaxnreg): the kernel is compiled for 168 registers a thread (384 threads, one CTA
// per SM: 64512 of the 65536), then the producer warpgroup gives registers back and the consumer
// warpgroups take them: 128 x 40 + 256 x 232 = 64512, the launch's whole allocation, so the consumers'
// increase is always satisfiable (dk_step_create checks the compiled count before any launch).
constexpr int kLaunchRegs = 168;
constexpr int kProducerRegs = 40;
constexpr int kConsumerRegs = 232;
static_assert(128 * kProducerRegs + kConsumers * kConsumerRegs <= kThreads * kLaunchRegs, "register split");
constexpr int kMaxRows = 4;                   // batch rows of one step
constexpr int kSlotW = 4096;                  // weight bytes of one ring slot (one TMA box)
constexpr int kSlotSZ = 256;                  // scale + zero bytes of one int4 ring slot
constexpr int kMaxChunks = 4;                 // int4 ops: 32-column chunks (or gate/up pairs) per CTA
constexpr int kHd = 128;                      // head_dim
constexpr int kAttnPos = 128;                 // cache positions per attention item (8 warps x 16)
constexpr int kMaxGroup = 8;                  // query heads per kv head
constexpr int kPartFloats = 2 + kHd;          // attention partial per head: max, sum, output[hd]
constexpr int kAttnBatch = 1;                 // attention slices whose partials one thread loads at once
constexpr int kMaxKSplit = 4;                 // K slices of a split-K projection (partials in fp32)
constexpr int kXsPad = 16;
constexpr int kTraceSlots = 12;  // per op: wait start, ready, staged, products, work done, arrival, ring wait, probes

enum OpKind : int { OP_QKV = 1, OP_ATTN = 2, OP_O = 3, OP_GATEUP = 4, OP_DOWN = 5, OP_HEAD = 6 };

// One op of the step program (device memory, written once at set-up, read-only while kernels run).
struct __align__(16) Op {
  int kind, layer;
  int cta0, ncta;   // participating CTAs: cta0 .. cta0 + ncta - 1 (mod grid); ATTN: first CTA of item 0
  int units;        // int4: 32-column chunks (gate_up: gate/up chunk pairs); HEAD: 32-row vocab chunks
  int stages;       // ring slots' worth of K per chunk: 256 K (int4) or 64 K (fp16 lm_head)
  int K, N;         // inner dim; output columns (gate_up: I, the SwiGLU width)
  int map;          // tensor-map index of the weights (int4: +1 scales, +2 zeros)
  int from_embed;   // QKV of layer 0: the input rows are embedding rows of the step's tokens
  int ksplit;       // > 1: each participant takes one (chunk, K slice) and writes fp32 partials to yp
  int xsplit;       // > 0: the input is fp16(sum of xsplit fp32 partials xp + xbias), not x
  int xop, rop;     // program index of the op that wrote the input / the residual (their tags)
  int cache_row0;   // ATTN: first row of this layer's cache in the 2-D cache maps
  int xattn;        // O: the input is the attention items' slice partials at xp (combined while staged)
  // activations are tagged words: fp16 value | 16-bit tag << 16 (LL16), fp32 bits | 32-bit tag << 32 (LL32)
  const unsigned long long* xp;  // [xsplit, M, K] LL32 partial sums of the previous projection; xattn: the
                                 // attention partials [M * nkv][max_len / 128][kMaxGroup][kPartFloats]
  const __half* xbias;  // [K] bias of that projection, or nullptr
  unsigned long long* yp;  // ksplit > 1: [ksplit, M, N] LL32 partial sums (no bias: the consumer adds it)
  const uint32_t* x;    // LL16 input [M, K] (not read when from_embed or xsplit)
  const uint32_t* res_in;  // LL16 residual added to x before the norm, or nullptr
  uint32_t* res_out;    // LL16: receives the new residual h = x (+ res_in) (one CTA writes it), or nullptr
  const __half* norm_w; // RMSNorm weight [K], or nullptr (no norm)
  const __half* bias;   // [N] (gate_up: [2I]) or nullptr
  uint32_t* y;          // LL16 output [M, N] (HEAD: unused, the logits pointer is per call)
};

// The fields of an op that decide who takes part and how many ring slots it uses: a copy of every
// op's lives in shared memory for the whole kernel (the full Op is fetched only by participants).
struct Ctl {
  int16_t kind, cta0, ncta, units, stages, ksplit, pad0, pad1;
};

struct Params {
  const Op* ops;
  int n_ops;
  const CUtensorMap* maps;
  int kmap, vmap;  // K / V cache maps: [layers * B * nkv * max_len rows, head_dim]
  int M, H, nq, nkv, max_len, vocab;
  int nslots;      // ring slots
  uint32_t nslots_rcp;  // ceil(2^32 / nslots): it / nslots == __umulhi(it, nslots_rcp) for it < 2^24
  int kmax;        // largest K of the int4 ops (staged rows, {C, X} table)
  int xs_pitch;    // bytes per staged input row
  int red_bytes;   // reduction scratch
  float eps, attn_scale;
  const __half* embed;
  const __half* rope_cos;  // [max_len, head_dim]
  const __half* rope_sin;
  __half* k_cache;         // [layers, B, nkv, max_len, head_dim]
  __half* v_cache;
  int64_t* tok;            // [M]: this step's tokens in, the greedy picks out
  int64_t* pos;            // [1]: this step's position in, + 1 out
  int64_t* hist;           // [M, hist_ld] or nullptr: hist[m][pos] = pick
  int64_t hist_ld;
  __half* logits;          // [M, vocab] or nullptr
  unsigned long long* trace;  // [grid][n_ops + 1][kTraceSlots] %globaltimer stamps, or nullptr (dk_step_trace)
  unsigned* epoch;         // launches so far (tags of this launch's words), advanced by the last CTA
  unsigned* exit_count;
  unsigned* head_count;
  unsigned long long* attn_part;  // LL32 [M * nkv * max_splits][group][kPartFloats]
  float* head_val;         // [grid][kMaxRows]
  int* head_idx;           // [grid][kMaxRows]
  int* err;
};

// ------------------------------------------------------------------------------ small helpers
// ------------------------------------------------------------------------------ tagged words
// The tag of op j of the launch with epoch e: never 0 (buffers start zeroed), and distinct for every
// op within 65535 (2^32 - 2) consecutive ops - a buffer is rewritten every step, so a word is never
// older than one step.
__device__ __forceinline__ uint32_t tag16(uint32_t epoch, int n_ops, int j) {
  return 1u + static_cast<uint32_t>((static_cast<uint64_t>(epoch) * n_ops + j) % 65535ull);
}
__device__ __forceinline__ uint32_t tag32(uint32_t epoch, int n_ops, int j) {
  return 1u + static_cast<uint32_t>((static_cast<uint64_t>(epoch) * n_ops + j) % 0xFFFFFFFEull);
}

// Tags of the op being run: of its input, its residual and its own outputs.
struct Tags {
  uint32_t x16, r16, o16, x32, o32;
};

__device__ __forceinline__ uint4 ldv_u32x4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void ldv_u64x2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool ll16_ok(const uint4& w, uint32_t tag) {
  return ((w.x >> 16) == tag) & ((w.y >> 16) == tag) & ((w.z >> 16) == tag) & ((w.w >> 16) == tag);
}
// the fp16 values of 8 LL16 words (two 4-word loads) as one 16-byte block of halves
__device__ __forceinline__ uint4 ll16_values(const uint4& a, const uint4& b) {
  return make_uint4(prmt(a.x, a.y, 0x5410), prmt(a.z, a.w, 0x5410), prmt(b.x, b.y, 0x5410), prmt(b.z, b.w, 0x5410));
}
// 8 halves (one 16-byte block) as 8 LL16 words: two 16-byte stores (each 4-byte word single-copy atomic)
__device__ __forceinline__ void ll16_store8(uint32_t* dst, const uint4& h, uint32_t tag) {
  const uint32_t t = tag << 16;
  const uint4 a = make_uint4(t | (h.x & 0xFFFFu), t | (h.x >> 16), t | (h.y & 0xFFFFu), t | (h.y >> 16));
  const uint4 b = make_uint4(t | (h.z & 0xFFFFu), t | (h.z >> 16), t | (h.w & 0xFFFFu), t | (h.w >> 16));
  reinterpret_cast<uint4*>(dst)[0] = a;
  reinterpret_cast<uint4*>(dst)[1] = b;
}
__device__ __forceinline__ uint32_t ll16_word(__half v, uint32_t tag) {
  return (tag << 16) | static_cast<uint32_t>(__half_as_ushort(v));
}
__device__ __forceinline__ unsigned long long ll32_word(float v, uint32_t tag) {
  return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}

// Bounded polling: again() after a failed check; false once this CTA gave up (then the caller stops).
struct Poller {
  volatile int* abort;
  int* err;
  uint64_t t0;
  int spins;
  __device__ Poller(volatile int* a, int* e) : abort(a), err(e), t0(0), spins(0) {}
  __device__ bool again() {
    if ((++spins & 31) == 0) {
      if (*abort) return false;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        record_device_error(err, DK_DEVERR_STEP_WAIT);
        *abort = 1;
        return false;
      }
    }
    return true;
  }
};

// 8 LL16 values at src once all 8 carry `tag` (first attempt's words in a, b); zeros on give-up.
__device__ __forceinline__ uint4 ll16_finish(const uint32_t* src, uint4 a, uint4 b, uint32_t tag, Poller& pl) {
  while (!(ll16_ok(a, tag) && ll16_ok(b, tag))) {
    if (!pl.again()) return make_uint4(0, 0, 0, 0);
    a = ldv_u32x4(src);
    b = ldv_u32x4(src + 4);
  }
  return ll16_values(a, b);
}
__device__ __forceinline__ uint4 ll16_load8(const uint32_t* src, uint32_t tag, Poller& pl) {
  return ll16_finish(src, ldv_u32x4(src), ldv_u32x4(src + 4), tag, pl);
}

// Release of this thread's (and, after a CTA barrier, the CTA's) earlier writes to the GPU before an
// arrival: acq_rel is enough for the acquire loads that pair with it (no total order needed).
__device__ __forceinline__ void fence_release_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// 16-byte word w of an op descriptor, global -> shared without stalling the issuing thread
__device__ __forceinline__ void cp_async16(Op* dst, int w, const Op* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(reinterpret_cast<uint4*>(dst) + w)),
               "l"(reinterpret_cast<const uint4*>(src) + w)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_group1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kConsumers) : "memory"); }

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}

// Participant index of this CTA in an op with participants cta0 .. cta0 + n - 1 (mod G), or -1.
__device__ __forceinline__ int participant(int cta, int cta0, int n, int G) {
  const int j = (cta - cta0 + G) % G;
  return j < n ? j : -1;
}

// Attention items of the step: M sequences x nkv heads x slices of kAttnPos positions.
__device__ __forceinline__ int attn_splits(int pos) { return pos / kAttnPos + 1; }

// This CTA's share of an int4 or head op: output chunks [c0, c1), and of each the K stages [st0, st1).
struct Work {
  int c0, c1, st0, st1;
};
template <class OpT>
__device__ __forceinline__ Work op_work(const OpT& op, int j) {
  Work w;
  if (op.ksplit > 1) {  // one (chunk, K slice) per participant
    const int c = j / op.ksplit, ks = j - c * op.ksplit;
    w.c0 = c;
    w.c1 = c + 1;
    w.st0 = ks * op.stages / op.ksplit;
    w.st1 = (ks + 1) * op.stages / op.ksplit;
  } else {
    w.c0 = static_cast<int>(static_cast<int64_t>(j) * op.units / op.ncta);
    w.c1 = static_cast<int>(static_cast<int64_t>(j + 1) * op.units / op.ncta);
    w.st0 = 0;
    w.st1 = op.stages;
  }
  return w;
}

// Ring slots one CTA uses for an op (the producer and every consumer warp walk the same sequence).
template <class OpT>
__device__ __forceinline__ int op_slots(const OpT& op, int cta, int G, int M, int nkv, int pos) {
  if (op.kind == OP_ATTN) {
    const int items = M * nkv * attn_splits(pos);
    const int j = (cta - op.cta0 + G) % G;
    const int mine = j < items ? (items - 1 - j) / G + 1 : 0;
    return mine * 16;
  }
  const int j = participant(cta, op.cta0, op.ncta, G);
  if (j < 0) return 0;
  const Work w = op_work(op, j);
  return (w.c1 - w.c0) * (w.st1 - w.st0) * (op.kind == OP_GATEUP ? 2 : 1);
}


// ------------------------------------------------------------------------------ shared memory
struct Smem {
  uint8_t* w;      // [nslots][kSlotW], 1024-byte aligned
  uint8_t* sz;     // [nslots][kSlotSZ]
  uint8_t* xs;     // staged input rows
  float* cx;       // int4 factored path: per (128-group, row) {C, X}, 8 rows per group
  float* red;      // reduction scratch
  uint64_t* full;
  uint64_t* empty;
};

// bytes: offsets from the 1024-aligned base
struct SmemLayout {
  int w, sz, xs, cx, red, bars, ctl, total;
};

__host__ __device__ inline SmemLayout smem_layout(int nslots, int M, int xs_pitch, int kmax, int red_bytes, int n_ops) {
  SmemLayout L;
  L.w = 0;
  L.sz = nslots * kSlotW;
  L.xs = L.sz + nslots * kSlotSZ;
  L.cx = L.xs + ((M * xs_pitch + 127) / 128) * 128;
  L.red = L.cx + (kmax / 128) * 8 * 8;
  L.bars = L.red + ((red_bytes + 127) / 128) * 128;
  L.ctl = L.bars + 2 * nslots * 8;
  L.total = L.ctl + n_ops * static_cast<int>(sizeof(Ctl));
  return L;
}

// ------------------------------------------------------------------------------ ring access
struct Ring {
  Smem s;
  int nslots;
  uint32_t rcp;
  volatile int* issued;  // slots the producer has armed (count); written by the producer only
  volatile int* abort;
  int* err;
  int seen;              // this thread's last read of *issued
  long long waited;      // tracing: clock cycles this thread spent in wait()
  bool timed;            // tracing on

  // Wait until slot sequence number `it` holds its data. First until the producer has armed it (so
  // the parity wait below cannot match a phase two rounds old), then the full barrier's phase.
  __device__ bool wait(int it) {
    if (it >= seen) {
      uint64_t t0 = 0;
      for (int spin = 0; (seen = *issued) <= it; ++spin) {
        if ((spin & 63) == 0) {  // the clock and the abort flag only now and then: they cost
          if (*abort) return false;
          const uint64_t now = globaltimer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > kWaitLimitNs) {
            record_device_error(err, DK_DEVERR_STEP_WAIT);
            *abort = 1;
            return false;
          }
        }
      }
      __threadfence_block();
    }
    const uint32_t round = __umulhi(static_cast<uint32_t>(it), rcp);
    const int slot = it - static_cast<int>(round) * nslots;
    if (!mbar_wait(&s.full[slot], round & 1, err, DK_DEVERR_STEP_WAIT)) {
      *abort = 1;
      return false;
    }
    return true;
  }
  __device__ int slot_of(int it) const {
    return it - static_cast<int>(__umulhi(static_cast<uint32_t>(it), rcp)) * nslots;
  }
  __device__ void release(int it) { mbar_arrive(&s.empty[slot_of(it)]); }
  // the same, agreed by the whole warp (the MMAs that follow need every lane)
  __device__ bool warp_wait(int it) {
    if (!timed) return __all_sync(0xffffffffu, wait(it));
    const long long c0 = clock64();
    const bool ok = __all_sync(0xffffffffu, wait(it));
    waited += clock64() - c0;
    return ok;
  }
};

// ------------------------------------------------------------------------------ int4 GEMV pieces
// One chunk-stage (32 columns x 256 K of packed int4) against the staged input, the factored
// numerics of the standalone decode GEMV (s * (sum(x' (1024 + q')) - C - z X) per 128-group, the
// reference's FACTORED path, kernels/w4a16.py:116-119): LOP3 with the 0x6400 exponent turns nibble
// pairs into fp16 1024 + q (low nibble) or 1024 + 16 q (high nibble, whose x was staged / 16), the
// MMA sums them against x (up to 8 batch rows as the B operand), and the per-(group, row) constants
// C = 1024 sum(x') and X = sum(x) remove the magic-number offset and the zero point once per group.
__device__ __forceinline__ void gemv_stage(uint32_t wbox, uint32_t szb, uint32_t xrow, uint32_t cxg, int xs_pitch,
                                           int M, int g, int t, float (&acc)[2][4]) {
  const uint32_t k1024 = 0x64006400u;
  const uint32_t w_even = wbox + (2 * t) * 128 + ((g ^ (2 * t)) << 4);
  const uint32_t w_odd = wbox + (2 * t + 1) * 128 + ((g ^ (2 * t + 1)) << 4);
  const uint32_t x_even = xrow + (2 * t) * 16 + g * xs_pitch, x_odd = xrow + (2 * t + 1) * 16 + g * xs_pitch;
  const bool have_row = g < M;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint2 s4 = lds64(szb + half * 64 + g * 8);
    const uint2 z4 = lds64(szb + 128 + half * 64 + g * 8);
    // one accumulator pair per sub-step: the 16 MMAs form 8 independent chains of 2 instead of 2 of 8
    float acs[4][2][4];
#pragma unroll
    for (int st4 = 0; st4 < 4; ++st4)
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int e = 0; e < 4; ++e) acs[st4][a][e] = 0.f;
#pragma unroll
    for (int st4 = 0; st4 < 4; ++st4) {
      const int st = half * 4 + st4;
      const uint4 wv = lds128(((st & 1) ? w_odd : w_even) + 1024 * (st >> 1));
      uint4 xv = make_uint4(0, 0, 0, 0);
      if (have_row) xv = lds128(((st & 1) ? x_odd : x_even) + 128 * (st >> 1));
      const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t W[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t w = words[c];
        const uint32_t w8 = w >> 8;
        W[c][0] = lop3_and_or(w, 0x000F000Fu, k1024);
        W[c][1] = lop3_and_or(w, 0x00F000F0u, k1024);
        W[c][2] = lop3_and_or(w8, 0x000F000Fu, k1024);
        W[c][3] = lop3_and_or(w8, 0x00F000F0u, k1024);
      }
      mma_16816(acs[st4][0], W[0][0], W[1][0], W[0][1], W[1][1], xv.x, xv.y);
      mma_16816(acs[st4][0], W[0][2], W[1][2], W[0][3], W[1][3], xv.z, xv.w);
      mma_16816(acs[st4][1], W[2][0], W[3][0], W[2][1], W[3][1], xv.x, xv.y);
      mma_16816(acs[st4][1], W[2][2], W[3][2], W[2][3], W[3][3], xv.z, xv.w);
    }
    float accg[2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int e = 0; e < 4; ++e) accg[a][e] = (acs[0][a][e] + acs[1][a][e]) + (acs[2][a][e] + acs[3][a][e]);
    const __half2 s01 = *reinterpret_cast<const __half2*>(&s4.x), s23 = *reinterpret_cast<const __half2*>(&s4.y);
    const __half2 z01 = *reinterpret_cast<const __half2*>(&z4.x), z23 = *reinterpret_cast<const __half2*>(&z4.y);
    const float sc[4] = {__low2float(s01), __high2float(s01), __low2float(s23), __high2float(s23)};
    const float zc[4] = {__low2float(z01), __high2float(z01), __low2float(z23), __high2float(z23)};
    // {C, X} of batch rows 2t and 2t + 1 (the D fragment's columns)
    const uint4 cxr = lds128(cxg + half * 64 + (2 * t) * 8);
    const float cx[2][2] = {{__uint_as_float(cxr.x), __uint_as_float(cxr.y)},
                            {__uint_as_float(cxr.z), __uint_as_float(cxr.w)}};
#pragma unroll
    for (int tile = 0; tile < 2; ++tile)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = 2 * tile + (e >> 1), r = e & 1;
        acc[tile][e] = fmaf(sc[col], accg[tile][e] - fmaf(zc[col], cx[r][1], cx[r][0]), acc[tile][e]);
      }
  }
}

// Block v (8 values) of input row m when the input is the sum of a split-K projection's fp32 partials:
// fp16(partial 0 + partial 1 + ... (+ bias)), partials added in slice order (deterministic), the same
// fp16 rounding the projection's own epilogue applies. Two partials' words are in flight at a time
// (partial q + 2 is requested once partial q is in): three partials cost two round trips to L2, not
// three, without holding every partial's 64-bit words in registers at once.
__device__ __forceinline__ uint4 split_input(const Op& op, int M, int K, int m, int v, uint32_t tag, Poller& pl) {
  const int nsplit = op.xsplit;
  const int64_t qstride = static_cast<int64_t>(M) * K;
  const unsigned long long* src = op.xp + static_cast<int64_t>(m) * K + 8 * v;
  unsigned long long w[2][8];
  auto request = [&](int q) {
#pragma unroll
    for (int i = 0; i < 4; ++i) ldv_u64x2(src + q * qstride + 2 * i, w[q & 1][2 * i], w[q & 1][2 * i + 1]);
  };
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  request(0);
  if (nsplit > 1) request(1);
#pragma unroll
  for (int q = 0; q < kMaxKSplit; ++q) {
    if (q >= nsplit) break;
    for (;;) {
      bool ok = true;
#pragma unroll
      for (int i = 0; i < 8; ++i) ok &= static_cast<uint32_t>(w[q & 1][i] >> 32) == tag;
      if (ok || !pl.again()) break;
      request(q);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __uint_as_float(static_cast<uint32_t>(w[q & 1][i]));
    if (q + 2 < nsplit) request(q + 2);
  }
  if (op.xbias != nullptr) {
    const uint4 bb = __ldg(reinterpret_cast<const uint4*>(op.xbias) + v);
    const __half* bh = reinterpret_cast<const __half*>(&bb);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __half2float(bh[i]);
  }
  uint4 out;
  __half2* oh = reinterpret_cast<__half2*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) oh[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
  return out;
}

// Block v (8 dims of one query head) of row b of the attention output, combined from the attention
// items' slice partials (per slice q: max score M_q, sum of weights L_q, unnormalized output O_q) in
// slice order, flash-decoding style: out = sum_q e^(M_q - M) O_q / sum_q e^(M_q - M) L_q with the
// running maximum M, rounded to fp16. The words of kAttnBatch slices are requested at once.
__device__ __forceinline__ uint4 attn_input(const Params& p, const Op& op, int b, int v, int S, uint32_t tag, Poller& pl) {
  const int G = p.nq / p.nkv;
  const int head = v >> 4, d0 = (v & 15) * 8;
  const int h = head / G, hh = head - h * G;
  const unsigned long long* parts =
      op.xp + (static_cast<int64_t>(b) * p.nkv + h) * (p.max_len / kAttnPos) * kMaxGroup * kPartFloats + hh * kPartFloats;
  float mx = -INFINITY, l = 0.f;
  float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int q0 = 0; q0 < S; q0 += kAttnBatch) {
    unsigned long long w[kAttnBatch][10];
    auto request = [&](int u) {
      const unsigned long long* src = parts + static_cast<int64_t>(q0 + u) * kMaxGroup * kPartFloats;
      ldv_u64x2(src, w[u][0], w[u][1]);
#pragma unroll
      for (int i = 0; i < 4; ++i) ldv_u64x2(src + 2 + d0 + 2 * i, w[u][2 + 2 * i], w[u][3 + 2 * i]);
    };
#pragma unroll
    for (int u = 0; u < kAttnBatch; ++u)
      if (q0 + u < S) request(u);
#pragma unroll
    for (int u = 0; u < kAttnBatch; ++u) {
      if (q0 + u >= S) break;
      for (;;) {
        bool ok = true;
#pragma unroll
        for (int i = 0; i < 10; ++i) ok &= static_cast<uint32_t>(w[u][i] >> 32) == tag;
        if (ok || !pl.again()) break;
        request(u);
      }
      const float mq = __uint_as_float(static_cast<uint32_t>(w[u][0]));
      const float lq = __uint_as_float(static_cast<uint32_t>(w[u][1]));
      if (lq > 0.f) {
        const float mn = fmaxf(mx, mq);
        const float a = __expf(mx - mn), c = __expf(mq - mn);  // a = 0 while nothing is summed (mx = -inf)
        l = fmaf(l, a, lq * c);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = fmaf(o[i], a, __uint_as_float(static_cast<uint32_t>(w[u][2 + i])) * c);
        mx = mn;
      }
    }
  }
  if (!(l > 0.f)) l = 1.f;  // only after a give-up (slice 0 always holds position 0)
  uint4 out;
  __half2* oh = reinterpret_cast<__half2*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) oh[i] = __floats2half2_rn(o[2 * i] / l, o[2 * i + 1] / l);
  return out;
}

// Stage block b (8 K values) of input row m: with a norm weight (wv != 0 words; sc = 1/rms) the
// RMSNorm output w * fp16(h * sc) first; then the (0,4,1,5,2,6,3,7) permutation, odd K / 16, and the
// {C, X} sums of the block's 128-group, reduced over the 16 lanes (a half-warp) that hold the group.
__device__ __forceinline__ void stage_block(const Params& p, const Smem& s, uint4 v, uint4 wv, float sc, int m, int b) {
  if (sc != 0.f) {
    __half2* vh = reinterpret_cast<__half2*>(&v);
    const __half2* wh = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(vh[j]);
      vh[j] = __hmul2_rn(wh[j], __floats2half2_rn(__fmul_rn(f.x, sc), __fmul_rn(f.y, sc)));
    }
  }
  uint4 o;
  o.x = prmt(v.x, v.z, 0x5410);
  o.y = prmt(v.x, v.z, 0x7632);
  o.z = prmt(v.y, v.w, 0x5410);
  o.w = prmt(v.y, v.w, 0x7632);
  o.y = hmul2_rn(o.y, 0x2C002C00u);
  o.w = hmul2_rn(o.w, 0x2C002C00u);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&o.x));
  const float2 bb = __half22float2(*reinterpret_cast<const __half2*>(&o.y));
  const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&o.z));
  const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&o.w));
  const float even = (a.x + a.y) + (c.x + c.y), odd = (bb.x + bb.y) + (d.x + d.y);
  float C = even + odd, X = fmaf(16.f, odd, even);
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) {
    C += __shfl_xor_sync(0xffffffffu, C, off);
    X += __shfl_xor_sync(0xffffffffu, X, off);
  }
  if ((threadIdx.x & 15) == 0) {
    float* dst = s.cx + 2 * ((b >> 4) * 8 + m);
    dst[0] = 1024.f * C;
    dst[1] = X;
  }
  *reinterpret_cast<uint4*>(s.xs + m * p.xs_pitch + b * 16) = o;
}

// Stage the op's input rows in shared memory for the int4 path: optional residual add + RMSNorm
// with the rounding of kernels/rmsnorm.py:28-37 (h = x + residual in fp16, var = sum(h^2)/K in fp32,
// out = w * fp16(h / sqrt(var + eps))), then each 8-value block permuted to (0,4,1,5,2,6,3,7) for the
// MMA fragments, odd K divided by 16 (exact) for the magic-number operands, and {C, X} per
// (128-group, row). `writer`: this CTA stores h as the new residual.
__device__ void stage_int4_input(const Params& p, const Op& op, const Tags& tg, const Smem& s, bool writer,
                                 float* inv_s, float (*part)[kCWarps], int st0, int st1, int pos, Poller& pl) {
  const int tid = threadIdx.x;
  const int K = op.K;
  const int nblk = K / 8;  // K % 256 == 0: a multiple of 32 blocks, so a warp's 32 items share a row
  const bool norm = op.norm_w != nullptr;  // (never with a K slice: norm ops are not split)
  auto embed_row = [&](int m) -> const __half* {
    int64_t t = __ldcg(reinterpret_cast<const long long*>(p.tok) + m);
    if (t < 0 || t >= p.vocab) {
      record_device_error(p.err, DK_DEVERR_BAD_TOKEN);
      t = 0;
    }
    return p.embed + t * static_cast<int64_t>(p.H);
  };
  auto load_h = [&](int m, int v) -> uint4 {  // 8 values of h = x (+ residual) at block v of row m
    // the residual's words are requested first, in flight together with the input's
    const uint32_t* rsrc = op.res_in != nullptr ? op.res_in + (static_cast<int64_t>(m) * K + 8 * v) : nullptr;
    uint4 ra = make_uint4(0, 0, 0, 0), rb = ra;
    if (rsrc != nullptr) {
      ra = ldv_u32x4(rsrc);
      rb = ldv_u32x4(rsrc + 4);
    }
    uint4 a;
    if (op.xsplit > 0)
      a = split_input(op, p.M, K, m, v, tg.x32, pl);
    else if (op.from_embed)
      a = __ldg(reinterpret_cast<const uint4*>(embed_row(m)) + v);
    else
      a = ll16_load8(op.x + (static_cast<int64_t>(m) * K + 8 * v), tg.x16, pl);
    if (rsrc != nullptr) {  // a + residual (fp16 add)
      const uint4 r = ll16_finish(rsrc, ra, rb, tg.r16, pl);
      __half2* ah = reinterpret_cast<__half2*>(&a);
      const __half2* rh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
      for (int j = 0; j < 4; ++j) ah[j] = __hadd2_rn(ah[j], rh[j]);
    }
    return a;
  };
  // One block of 8 values per thread and row (K <= 2048, every norm op of Qwen2.5-1.5B): one L2 read
  // of the row, held in registers from the sum of squares to the staging.
  if (norm && nblk <= kConsumers) {
    uint4 hv[kMaxRows];
    const bool mine = tid < nblk;
    for (int m = 0; m < p.M; ++m) {
      float acc = 0.f;
      if (mine) {
        hv[m] = load_h(m, tid);
        if (writer && op.res_out != nullptr) ll16_store8(op.res_out + (static_cast<int64_t>(m) * K + 8 * tid), hv[m], tg.o16);
        const __half2* ah = reinterpret_cast<const __half2*>(&hv[m]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(ah[j]);
          acc = fmaf(f.x, f.x, acc);
          acc = fmaf(f.y, f.y, acc);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if ((tid & 31) == 0) part[m][tid >> 5] = acc;
    }
    consumers_sync();
    if (tid < p.M) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) tot += part[tid][w];
      inv_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(K)), p.eps)));
    }
    consumers_sync();
    if (mine) {  // nblk % 32 == 0: whole warps, so the half-warp shuffles below see 16 blocks of a group
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(op.norm_w) + tid);
      for (int m = 0; m < p.M; ++m) stage_block(p, s, hv[m], wv, inv_s[m], m, tid);
    }
    consumers_sync();
    return;
  }
  if (norm) {
    for (int m = 0; m < p.M; ++m) {
      float acc = 0.f;
      for (int v = tid; v < nblk; v += kConsumers) {
        const uint4 a = load_h(m, v);
        if (writer && op.res_out != nullptr) ll16_store8(op.res_out + (static_cast<int64_t>(m) * K + 8 * v), a, tg.o16);
        const __half2* ah = reinterpret_cast<const __half2*>(&a);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(ah[j]);
          acc = fmaf(f.x, f.x, acc);
          acc = fmaf(f.y, f.y, acc);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if ((tid & 31) == 0) part[m][tid >> 5] = acc;
    }
    consumers_sync();
    if (tid < p.M) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) tot += part[tid][w];
      inv_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(K)), p.eps)));
    }
    consumers_sync();
  }
  // Only this CTA's K stages [st0, st1) are staged, at stage positions 0 .. st1 - st0. Block i of the
  // staged rows goes to thread i % kConsumers (sblk is a multiple of 32: warps are whole in every
  // round, as stage_block's half-warp sums need).
  const int sblk = (st1 - st0) * 32, b0 = st0 * 32;
  const int total = p.M * sblk;
  auto stage_one = [&](int i, uint4 v) {
    const int m = i / sblk, b = i % sblk;
    if (!norm && writer && op.res_out != nullptr)
      ll16_store8(op.res_out + (static_cast<int64_t>(m) * K + 8 * (b0 + b)), v, tg.o16);
    const uint4 wv = norm ? __ldg(reinterpret_cast<const uint4*>(op.norm_w) + b0 + b) : make_uint4(0, 0, 0, 0);
    stage_block(p, s, v, wv, norm ? inv_s[m] : 0.f, m, b);
  };
  if (op.xattn) {  // o_proj: the attention output, combined from the slice partials (no norm, no residual)
    const int S = attn_splits(pos);
    for (int i = tid; i < total; i += kConsumers) stage_one(i, attn_input(p, op, i / sblk, b0 + i % sblk, S, tg.x32, pl));
  } else if (op.xsplit == 0 && !op.from_embed && op.res_in == nullptr) {
    // a plain tagged input (down_proj's, a long row such as down's 8960 values): up to kBatch blocks
    // per thread with their first loads in flight at once, then checked and staged
    constexpr int kBatch = 4;
    for (int base0 = (tid & ~31); base0 < total; base0 += kBatch * kConsumers) {
      uint4 wa[kBatch], wb[kBatch];
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const int i = base0 + q * kConsumers + (tid & 31);
        if (i < total) {
          const uint32_t* src = op.x + (static_cast<int64_t>(i / sblk) * K + 8 * (b0 + i % sblk));
          wa[q] = ldv_u32x4(src);
          wb[q] = ldv_u32x4(src + 4);
        }
      }
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const int i = base0 + q * kConsumers + (tid & 31);
        if (base0 + q * kConsumers >= total) break;
        const uint4 v = ll16_finish(op.x + (static_cast<int64_t>(i / sblk) * K + 8 * (b0 + i % sblk)), wa[q], wb[q], tg.x16, pl);
        stage_one(i, v);
      }
    }
  } else {
    for (int i = tid; i < total; i += kConsumers) stage_one(i, load_h(i / sblk, b0 + i % sblk));
  }
  consumers_sync();
}

__device__ __forceinline__ __half swiglu_pick(float g, float u, const __half* bias, int n, int I) {
  if (bias != nullptr) {
    g += __half2float(__ldg(bias + n));
    u += __half2float(__ldg(bias + I + n));
  }
  const float gf = __half2float(__float2half_rn(g));
  const __half act = __float2half_rn(__fdiv_rn(gf, __fadd_rn(1.0f, expf(-gf))));
  return __hmul_rn(act, __float2half_rn(u));
}

// An int4 projection (QKV, O, GATEUP, DOWN) of this CTA's chunk range [c0, c1). Unit u of the range
// (chunk c0 + u / stages, stage u % stages) sits at ring slot base + u (gate_up: 2u and 2u + 1, the
// gate and the up box). Boxes are dealt to the consumer warps one by one (box b to warp b % kCWarps),
// so the warps' box counts differ by at most one; a warp keeps its sum in registers while its boxes
// stay in one chunk (and half) and parks it in red[chunk][warp][half] when that changes.
__device__ void run_int4(const Params& p, const Op& op, const Tags& tg, Ring& ring, int base, const Work& wk,
                         int ks, unsigned long long* stamp) {
  const int c0 = wk.c0, c1 = wk.c1, nst = wk.st1 - wk.st0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const bool pair = op.kind == OP_GATEUP;
  const int halves = pair ? 2 : 1;
  const int nunits = (c1 - c0) * nst;
  const int M = p.M;
  // red[chunk][warp][half][row][32]
  float* red = ring.s.red;
  auto cell = [&](int cl, int w, int h, int m) { return red + (((cl * kCWarps + w) * 2 + h) * kMaxRows + m) * 32; };
  for (int cl = 0; cl < c1 - c0; ++cl)
    for (int h = 0; h < halves; ++h)
      for (int m = 0; m < M; ++m) cell(cl, warp, h, m)[lane] = 0.f;
  float acc[2][4];
  int cur = -1, cur_h = 0;
  auto flush = [&]() {
    if (cur < 0) return;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int m = 2 * t + e;
      if (m < M) {
        float* dst = cell(cur, warp, cur_h, m) + 4 * g;
        dst[0] = acc[0][e];
        dst[1] = acc[0][2 + e];
        dst[2] = acc[1][e];
        dst[3] = acc[1][2 + e];
      }
    }
  };
  // the epilogue's bias values, fetched now so that their latency hides behind the products
  const int ncols = (c1 - c0) * 32;
  float bias_pre[2] = {0.f, 0.f};
  if (!pair && op.ksplit <= 1 && op.bias != nullptr)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int e = threadIdx.x + q * kConsumers;
      if (e < M * ncols) bias_pre[q] = __half2float(__ldg(op.bias + c0 * 32 + e % ncols));
    }
  const uint32_t w_base = smem_addr(ring.s.w), sz_base = smem_addr(ring.s.sz);
  const uint32_t xs_base = smem_addr(ring.s.xs), cx_base = smem_addr(ring.s.cx);
  // tracing (thread 0): clock cycles to the start of its second box and to the end of its last
  const long long clk0 = stamp ? clock64() : 0;
  for (int b = warp; b < nunits * halves; b += kCWarps) {
    if (stamp && b == warp + kCWarps) stamp[5] = static_cast<unsigned long long>(clock64() - clk0);
    const int u = pair ? b >> 1 : b, h = pair ? b & 1 : 0;
    const int cl = u / nst, st = u % nst;  // st: position in the staged K slice
    if (cl != cur || h != cur_h) {
      flush();
      cur = cl;
      cur_h = h;
#pragma unroll
      for (int a2 = 0; a2 < 2; ++a2)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[a2][e] = 0.f;
    }
    const uint32_t xrow = xs_base + st * 512, cxg = cx_base + st * 2 * 64;
    const int it = base + b;
    if (!ring.warp_wait(it)) break;
    const int slot = ring.slot_of(it);
    gemv_stage(w_base + slot * kSlotW, sz_base + slot * kSlotSZ, xrow, cxg, p.xs_pitch, M, g, t, acc);
    __syncwarp();
    if (lane == 0) ring.release(it);
    if (__any_sync(0xffffffffu, *ring.abort)) break;
  }
  if (stamp) stamp[6] = static_cast<unsigned long long>(clock64() - clk0);
  flush();
  consumers_sync();
  if (stamp) {
    stamp[0] = globaltimer_ns();
    stamp[7] = static_cast<unsigned long long>(clock64() - clk0);
  }
  if (*ring.abort) return;
  // fixed-order reduction over the warps, epilogue, store
  for (int e = threadIdx.x; e < M * ncols; e += kConsumers) {
    const int m = e / ncols, col = e % ncols;
    const int cl = col / 32, cc = col % 32;
    float v[2] = {0.f, 0.f};
    for (int h = 0; h < halves; ++h)
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) v[h] += cell(cl, w, h, m)[cc];
    const int n = c0 * 32 + col;
    if (op.ksplit > 1) {  // fp32 partial of this K slice; the consumer adds slices and bias
      op.yp[(static_cast<int64_t>(ks) * M + m) * op.N + n] = ll32_word(v[0], tg.o32);
    } else if (pair) {
      op.y[static_cast<int64_t>(m) * op.N + n] = ll16_word(swiglu_pick(v[0], v[1], op.bias, n, op.N), tg.o16);
    } else {
      float a = v[0];
      if (op.bias != nullptr)
        a += e < kConsumers ? bias_pre[0] : e < 2 * kConsumers ? bias_pre[1] : __half2float(__ldg(op.bias + n));
      op.y[static_cast<int64_t>(m) * op.N + n] = ll16_word(__float2half_rn(a), tg.o16);
    }
  }
}

// ------------------------------------------------------------------------------ attention
// RoPE of 4 consecutive dims and their partners half a head away with the reference's fp16 rounding
// per op (kernels/e2e/model.py:212-214: x * cos + cat(-x2, x1) * sin).
__device__ __forceinline__ void rope_quad(const uint32_t* src, const __half* cosr, const __half* sinr, int d,
                                          __half* dst, uint32_t tag, Poller& pl) {
  // 4 tagged values at d and their partners at d + 64
  uint4 wl = ldv_u32x4(src + d), wh = ldv_u32x4(src + d + kHd / 2);
  while (!(ll16_ok(wl, tag) && ll16_ok(wh, tag))) {
    if (!pl.again()) break;
    wl = ldv_u32x4(src + d);
    wh = ldv_u32x4(src + d + kHd / 2);
  }
  const uint2 lo = make_uint2(prmt(wl.x, wl.y, 0x5410), prmt(wl.z, wl.w, 0x5410));
  const uint2 hi = make_uint2(prmt(wh.x, wh.y, 0x5410), prmt(wh.z, wh.w, 0x5410));
  const uint2 cl = __ldg(reinterpret_cast<const uint2*>(cosr + d)), ch = __ldg(reinterpret_cast<const uint2*>(cosr + d + kHd / 2));
  const uint2 sl = __ldg(reinterpret_cast<const uint2*>(sinr + d)), sh = __ldg(reinterpret_cast<const uint2*>(sinr + d + kHd / 2));
  const __half* xl = reinterpret_cast<const __half*>(&lo);
  const __half* xh = reinterpret_cast<const __half*>(&hi);
  const __half* c_l = reinterpret_cast<const __half*>(&cl);
  const __half* c_h = reinterpret_cast<const __half*>(&ch);
  const __half* s_l = reinterpret_cast<const __half*>(&sl);
  const __half* s_h = reinterpret_cast<const __half*>(&sh);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    dst[d + i] = __hadd_rn(__hmul_rn(xl[i], c_l[i]), __hmul_rn(__hneg(xh[i]), s_l[i]));
    dst[d + kHd / 2 + i] = __hadd_rn(__hmul_rn(xh[i], c_h[i]), __hmul_rn(xl[i], s_h[i]));
  }
}

// Row r (0..15), dims d..d+7 of a 16-row x 128-dim cache block in a ring slot: two TMA boxes of 16 rows
// x 64 dims with the 128-byte swizzle (16-byte chunk index XOR row % 8).
__device__ __forceinline__ uint32_t kv_at(uint32_t slot, int r, int d) {
  const int seg = d >> 6, c16 = (d & 63) >> 3;
  return slot + seg * 2048 + r * 128 + (((c16 ^ r) & 7) << 4);
}

struct AttnSmem {
  __half q[kMaxGroup][kHd + 8];
  __half knew[kHd];
  __half vnew[kHd];
  __half vzero[8];
};

// One attention item: sequence b, kv head h, positions [s * 128, s * 128 + 128) cut at pos. Warp w
// runs flash decoding on block w (16 positions: K slot base + 2w, V slot base + 2w + 1): q.K^T on
// tensor cores (heads as MMA rows), softmax, P.V with P rounded to fp16 (as flash-style SDPA does on
// fp16 inputs). The 8 warps' (max, sum, output) are combined in shared memory into one partial per
// head; the last item of (b, h) to arrive combines every slice into the attention output.
__device__ void run_attention_item(const Params& p, const Op& op, const Tags& tg, Ring& ring, AttnSmem& as,
                                   int base, int item, int pos, int S, Poller& pl, unsigned long long* stamps) {
  // stamps (tracing, thread 0): [prologue done, blocks done, partial written]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.nq / p.nkv;
  const int s = item % S, bh = item / S;
  const int h = bh % p.nkv, b = bh / p.nkv;
  const int width = (p.nq + 2 * p.nkv) * kHd;
  const uint32_t* qrow = op.x + static_cast<int64_t>(b) * width;
  const __half* cosr = p.rope_cos + static_cast<int64_t>(pos) * kHd;
  const __half* sinr = p.rope_sin + static_cast<int64_t>(pos) * kHd;
  const bool owner = pos / kAttnPos == s;  // this slice holds position pos: append k, v
  const int64_t row_pos = static_cast<int64_t>(op.cache_row0) + (static_cast<int64_t>(b) * p.nkv + h) * p.max_len + pos;

  // ---- prologue: RoPE of this kv head's q heads and k; v as is
  constexpr int kQuads = kHd / 8;
  for (int e = tid; e < (G + 1) * kQuads + kHd / 8; e += kConsumers) {
    if (e < (G + 1) * kQuads) {
      const int hh = e / kQuads, d = 4 * (e % kQuads);
      const uint32_t* src = hh < G ? qrow + (h * G + hh) * kHd : qrow + (p.nq + h) * kHd;
      __half* dst = hh < G ? &as.q[hh][0] : as.knew;
      rope_quad(src, cosr, sinr, d, dst, tg.x16, pl);
      if (hh == G && owner) {
        *reinterpret_cast<uint2*>(p.k_cache + row_pos * kHd + d) = *reinterpret_cast<const uint2*>(as.knew + d);
        *reinterpret_cast<uint2*>(p.k_cache + row_pos * kHd + d + kHd / 2) =
            *reinterpret_cast<const uint2*>(as.knew + d + kHd / 2);
      }
    } else {
      const int v8 = 8 * (e - (G + 1) * kQuads);
      const uint4 v = ll16_load8(qrow + (p.nq + p.nkv + h) * kHd + v8, tg.x16, pl);
      *reinterpret_cast<uint4*>(as.vnew + v8) = v;
      if (owner) *reinterpret_cast<uint4*>(p.v_cache + row_pos * kHd + v8) = v;
    }
  }
  if (tid < 8) as.vzero[tid] = __float2half(0.f);
  consumers_sync();
  if (stamps) stamps[0] = globaltimer_ns();

  // ---- this warp's 16-position block
  const int p0 = s * kAttnPos + 16 * warp;
  float o[kHd / 8][4];
#pragma unroll
  for (int j = 0; j < kHd / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const int itk = base + 2 * warp, itv = itk + 1;
  bool ok = ring.warp_wait(itk);
  ok = ok && ring.warp_wait(itv);
  if (ok && p0 <= pos) {
    const uint32_t kt = smem_addr(ring.s.w) + ring.slot_of(itk) * kSlotW;
    const uint32_t vt = smem_addr(ring.s.w) + ring.slot_of(itv) * kSlotW;
    uint32_t qa[kHd / 16][2];
#pragma unroll
    for (int ks = 0; ks < kHd / 16; ++ks) {
      qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(&as.q[g][16 * ks + 2 * t]) : 0u;
      qa[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(&as.q[g][16 * ks + 8 + 2 * t]) : 0u;
    }
    const int mi = lane >> 3, rr = lane & 7;
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int krow = 8 * (mi >> 1) + rr;
    const bool k_new = p0 + krow == pos;
#pragma unroll
    for (int ks = 0; ks < kHd / 16; ++ks) {
      const int d0 = 16 * ks + 8 * (mi & 1);
      uint32_t kb[4];
      const uint32_t a = k_new ? smem_addr(as.knew + d0) : kv_at(kt, krow, d0);
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                   : "=r"(kb[0]), "=r"(kb[1]), "=r"(kb[2]), "=r"(kb[3])
                   : "r"(a));
      mma_16816(sc[0], qa[ks][0], 0u, qa[ks][1], 0u, kb[0], kb[1]);
      mma_16816(sc[1], qa[ks][0], 0u, qa[ks][1], 0u, kb[2], kb[3]);
    }
    float bm = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float v = p0 + 8 * nt + 2 * t + e <= pos ? sc[nt][e] * p.attn_scale : -INFINITY;
        sc[nt][e] = v;
        bm = fmaxf(bm, v);
      }
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
    m_run = bm;  // finite: position p0 <= pos is inside the block
    float pr[2][2];
    float ls = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        pr[nt][e] = __expf(sc[nt][e] - m_run);
        ls += pr[nt][e];
      }
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    l_run = ls;
    const uint32_t a0 = half2_bits(__float2half_rn(pr[0][0]), __float2half_rn(pr[0][1]));
    const uint32_t a2 = half2_bits(__float2half_rn(pr[1][0]), __float2half_rn(pr[1][1]));
    const int vrow = (mi & 1) * 8 + rr;
    const int vpos = p0 + vrow;
#pragma unroll
    for (int dp = 0; dp < kHd / 16; ++dp) {
      const int d0 = 16 * dp + (mi >> 1) * 8;
      const uint32_t a = vpos > pos ? smem_addr(as.vzero) : vpos == pos ? smem_addr(as.vnew + d0) : kv_at(vt, vrow, d0);
      uint32_t vb[4];
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                   : "=r"(vb[0]), "=r"(vb[1]), "=r"(vb[2]), "=r"(vb[3])
                   : "r"(a));
      mma_16816(o[2 * dp], a0, 0u, a2, 0u, vb[0], vb[1]);
      mma_16816(o[2 * dp + 1], a0, 0u, a2, 0u, vb[2], vb[3]);
    }
  }
  __syncwarp();
  if (lane == 0 && ok) {
    ring.release(itk);
    ring.release(itv);
  }
  // ---- combine the 8 warps' partials of every head in shared memory: red[w][head][2 + hd]
  float* red = ring.s.red;
  if (stamps) stamps[1] = globaltimer_ns();
  if (g < G) {
    float* mine = red + (warp * kMaxGroup + g) * kPartFloats;
    if (t == 0) {
      mine[0] = m_run;
      mine[1] = l_run;
    }
#pragma unroll
    for (int j = 0; j < kHd / 8; ++j) {
      mine[2 + 8 * j + 2 * t] = o[j][0];
      mine[2 + 8 * j + 2 * t + 1] = o[j][1];
    }
  }
  consumers_sync();
  // per head: the warps' weights exp(m_w - M) (0 for a warp without positions) and the slice's
  // (M, L = sum of weights x sums), once per (warp, head), then every output dim as one weighted sum
  float* wts = red + kCWarps * kMaxGroup * kPartFloats;  // [kCWarps][kMaxGroup], then M[8], L[8]
  if (tid < G) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCWarps; ++w) {
      const float* src = red + (w * kMaxGroup + tid) * kPartFloats;
      if (src[1] > 0.f) mx = fmaxf(mx, src[0]);
    }
    float lsum = 0.f;
#pragma unroll
    for (int w = 0; w < kCWarps; ++w) {
      const float* src = red + (w * kMaxGroup + tid) * kPartFloats;
      const float wt = src[1] > 0.f ? __expf(src[0] - mx) : 0.f;
      wts[w * kMaxGroup + tid] = wt;
      lsum = fmaf(wt, src[1], lsum);
    }
    wts[kCWarps * kMaxGroup + tid] = mx;
    wts[kCWarps * kMaxGroup + kMaxGroup + tid] = lsum;
  }
  consumers_sync();
  // this slice's partial as 32-bit-tagged words: per head [M, L, O[0..127]] (unnormalized O)
  unsigned long long* parts = p.attn_part + static_cast<int64_t>(bh) * (p.max_len / kAttnPos) * kMaxGroup * kPartFloats;
  unsigned long long* part = parts + static_cast<int64_t>(s) * kMaxGroup * kPartFloats;
  for (int e = tid; e < G * (kHd + 2); e += kConsumers) {
    const int hh = e / (kHd + 2), k = e % (kHd + 2);
    float v;
    if (k < 2) {
      v = wts[kCWarps * kMaxGroup + k * kMaxGroup + hh];
    } else {
      v = 0.f;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) v = fmaf(wts[w * kMaxGroup + hh], red[(w * kMaxGroup + hh) * kPartFloats + k], v);
    }
    part[hh * kPartFloats + k] = ll32_word(v, tg.o32);
  }
  if (stamps) stamps[2] = globaltimer_ns();
}

// ------------------------------------------------------------------------------ lm_head + argmax
// Stage the final hidden rows (residual add + final RMSNorm) in natural order for the fp16 head.
__device__ void stage_head_input(const Params& p, const Op& op, const Tags& tg, const Smem& s, float* inv_s,
                                 float (*part)[kCWarps], Poller& pl) {
  const int tid = threadIdx.x;
  const int K = op.K, nblk = K / 8;
  for (int m = 0; m < p.M; ++m) {
    float acc = 0.f;
    for (int v = tid; v < nblk; v += kConsumers) {
      uint4 a = op.xsplit > 0 ? split_input(op, p.M, K, m, v, tg.x32, pl)
                              : ll16_load8(op.x + (static_cast<int64_t>(m) * K + 8 * v), tg.x16, pl);
      const uint4 r = ll16_load8(op.res_in + (static_cast<int64_t>(m) * K + 8 * v), tg.r16, pl);
      __half2* ah = reinterpret_cast<__half2*>(&a);
      const __half2* rh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ah[j] = __hadd2_rn(ah[j], rh[j]);
        const float2 f = __half22float2(ah[j]);
        acc = fmaf(f.x, f.x, acc);
        acc = fmaf(f.y, f.y, acc);
      }
      *reinterpret_cast<uint4*>(s.xs + m * p.xs_pitch + v * 16) = a;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((tid & 31) == 0) part[m][tid >> 5] = acc;
  }
  consumers_sync();
  if (tid < p.M) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kCWarps; ++w) tot += part[tid][w];
    inv_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(K)), p.eps)));
  }
  consumers_sync();
  for (int e = tid; e < p.M * nblk; e += kConsumers) {
    const int m = e / nblk, v = e % nblk;
    uint4 a = *reinterpret_cast<const uint4*>(s.xs + m * p.xs_pitch + v * 16);
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(op.norm_w) + v);
    __half2* ah = reinterpret_cast<__half2*>(&a);
    const __half2* wh = reinterpret_cast<const __half2*>(&wv);
    const float sc = inv_s[m];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(ah[j]);
      ah[j] = __hmul2_rn(wh[j], __floats2half2_rn(__fmul_rn(f.x, sc), __fmul_rn(f.y, sc)));
    }
    *reinterpret_cast<uint4*>(s.xs + m * p.xs_pitch + v * 16) = a;
  }
  consumers_sync();
}

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// The fp16 lm_head over this CTA's vocab chunks [c0, c1) (32 rows each) with the greedy argmax.
// Warp w takes chunks c0 + 8r + w (round r) whole: K in 64-wide ring slots (TMA box of 32 rows x 64
// halves, 128-byte swizzle), A operand by ldmatrix, the staged rows as B; slot of (round r, stage k,
// warp w) = base_r + k * (chunks in round r) + w. Logits are rounded to fp16 like F.linear's output
// and compared in that precision; ties go to the lower index (torch.argmax's first maximum).
__device__ void run_head(const Params& p, const Op& op, Ring& ring, int base, int c0, int c1, float* best_v,
                         int* best_i) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int M = p.M;
  const int nch = c1 - c0;
  const uint32_t w_base = smem_addr(ring.s.w);
  float bv[2] = {-INFINITY, -INFINITY};
  int bi[2] = {0x7fffffff, 0x7fffffff};
  const int mi = lane >> 3, rr = lane & 7;
  int rbase = base;
  for (int r = 0; 8 * r < nch; ++r) {
    const int nr = min(8, nch - 8 * r);
    if (warp < nr) {
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      for (int k = 0; k < op.stages; ++k) {
        const int it = rbase + k * nr + warp;
        if (!ring.warp_wait(it)) break;
        const uint32_t slot = w_base + ring.slot_of(it) * kSlotW;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const int kk = k * 64 + ks * 16;
          uint32_t b0 = 0, b1 = 0;
          if (g < M) {
            b0 = *reinterpret_cast<const uint32_t*>(ring.s.xs + g * p.xs_pitch + (kk + 2 * t) * 2);
            b1 = *reinterpret_cast<const uint32_t*>(ring.s.xs + g * p.xs_pitch + (kk + 8 + 2 * t) * 2);
          }
#pragma unroll
          for (int tile = 0; tile < 2; ++tile) {
            const int row = tile * 16 + (mi & 1) * 8 + rr;
            const int c16 = 2 * ks + (mi >> 1);
            const uint32_t a = slot + row * 128 + (((c16 ^ row) & 7) << 4);
            uint32_t af[4];
            asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                         : "=r"(af[0]), "=r"(af[1]), "=r"(af[2]), "=r"(af[3])
                         : "r"(a));
            mma_16816(acc[tile], af[0], af[1], af[2], af[3], b0, b1);
          }
        }
        __syncwarp();
        if (lane == 0) ring.release(it);
      }
      // epilogue: rows tile*16 + g (+8) of chunk c, batch rows 2t, 2t + 1
      const int c = c0 + 8 * r + warp;
#pragma unroll
      for (int tile = 0; tile < 2; ++tile)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int m = 2 * t + (e & 1);
          const int vrow = c * 32 + tile * 16 + g + (e >> 1) * 8;
          if (m < M && vrow < p.vocab) {
            const __half lg = __float2half_rn(acc[tile][e]);
            if (p.logits != nullptr) p.logits[static_cast<int64_t>(m) * p.vocab + vrow] = lg;
            better(bv[e & 1], bi[e & 1], __half2float(lg), vrow);
          }
        }
    }
    rbase += nr * op.stages;
    if (__any_sync(0xffffffffu, *ring.abort)) break;
  }
  // best over the warp's lanes with the same t (same batch rows), then over warps in shared memory
#pragma unroll
  for (int e = 0; e < 2; ++e)
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv[e], off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi[e], off);
      better(bv[e], bi[e], ov, oi);
    }
  if (g == 0) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int m = 2 * t + e;
      if (m < kMaxRows) {
        best_v[warp * kMaxRows + m] = bv[e];
        best_i[warp * kMaxRows + m] = bi[e];
      }
    }
  }
}

// ------------------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const SmemLayout L = smem_layout(p.nslots, p.M, p.xs_pitch, p.kmax, p.red_bytes, p.n_ops);
  Smem s;
  s.w = base + L.w;
  s.sz = base + L.sz;
  s.xs = base + L.xs;
  s.cx = reinterpret_cast<float*>(base + L.cx);
  s.red = reinterpret_cast<float*>(base + L.red);
  s.full = reinterpret_cast<uint64_t*>(base + L.bars);
  s.empty = s.full + p.nslots;
  Ctl* ctl = reinterpret_cast<Ctl*>(base + L.ctl);
  __shared__ __align__(16) Op s_ops[2];  // the consumers' current op and the next one they take part in

  __shared__ int s_issued, s_abort, s_pos;
  __shared__ uint32_t s_epoch;
  __shared__ float s_inv[kMaxRows];
  __shared__ float s_part[kMaxRows][kCWarps];
  __shared__ float s_best_v[kCWarps * kMaxRows];
  __shared__ int s_best_i[kCWarps * kMaxRows];
  __shared__ int s_head_last, s_stop;
  __shared__ __align__(16) AttnSmem as;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  if (tid == 0) {
    for (int i = 0; i < p.nslots; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    fence_mbar_init();
    s_issued = 0;
    s_abort = 0;
    s_epoch = *reinterpret_cast<volatile const unsigned*>(p.epoch);
    int64_t pos = *reinterpret_cast<volatile const int64_t*>(p.pos);
    if (pos < 0 || pos >= p.max_len) {
      record_device_error(p.err, DK_DEVERR_BAD_POSITION);
      pos = -1;
    }
    s_pos = static_cast<int>(pos);
  }
  for (int j = threadIdx.x; j < p.n_ops; j += blockDim.x) {
    const Op& o = p.ops[j];
    Ctl c;
    c.kind = static_cast<int16_t>(o.kind);
    c.cta0 = static_cast<int16_t>(o.cta0);
    c.ncta = static_cast<int16_t>(o.ncta);
    c.units = static_cast<int16_t>(o.units);
    c.stages = static_cast<int16_t>(o.stages);
    c.ksplit = static_cast<int16_t>(o.ksplit);
    c.pad0 = c.pad1 = 0;
    ctl[j] = c;
  }
  __syncthreads();
  const int pos = s_pos;
  volatile int* abort = &s_abort;
  if (pos < 0) *abort = 1;  // every CTA decides the same: nothing is written, counters still move

  if (warp >= kCWarps) {  // the producer's warpgroup (warps 9-11 only wait for the exit)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
  }
  if (warp == kCWarps) {
    // ================================================================ producer warp
    // kPLanes lanes arm kPLanes consecutive slots in lockstep (each waits for its own slot's release,
    // arms it and issues its copies), then lane 0 publishes the batch: the per-slot mbarrier and copy
    // latencies overlap instead of adding up, one slot after another.
    constexpr int kPLanes = 8;
    if (lane < kPLanes) {
      int base = 0;       // slot number of the current op's first slot
      int armed_end = 0;  // slot numbers below this were (or were being) armed
      bool live = pos >= 0;
      for (int j = 0; j < p.n_ops && live; ++j) {
        const int n = op_slots(ctl[j], cta, G, p.M, p.nkv, pos);
        if (n == 0) continue;
        const Op& op = p.ops[j];
        // per-op constants of the slot -> copy mapping
        const int jj = (cta - op.cta0 + G) % G;
        int c0 = 0, nch = 0, S = 1, st0 = 0, nst = op.stages;
        if (op.kind == OP_ATTN) {
          S = attn_splits(pos);
        } else {
          const Work wk = op_work(op, jj);
          c0 = wk.c0;
          nch = wk.c1 - wk.c0;
          st0 = wk.st0;
          nst = wk.st1 - wk.st0;
        }
        const int halves = op.kind == OP_GATEUP ? 2 : 1;
        for (int j0 = 0; j0 < n && live; j0 += kPLanes) {
          const int jl = j0 + lane;
          bool ok = true;
          if (jl < n) {
            const int it = base + jl;
            const uint32_t round = __umulhi(static_cast<uint32_t>(it), p.nslots_rcp);
            const int slot = it - static_cast<int>(round) * p.nslots;
            if (round > 0) {  // wait for the release of the slot's previous round
              const uint32_t par = (round - 1) & 1;
              uint64_t t0 = 0;
              for (int spin = 0; !mbar_try_wait(&s.empty[slot], par); ++spin) {
                if ((spin & 15) == 0) {
                  if (*abort) {
                    ok = false;
                    break;
                  }
                  const uint64_t now = globaltimer_ns();
                  if (t0 == 0) {
                    t0 = now;
                  } else if (now - t0 > kWaitLimitNs) {
                    record_device_error(p.err, DK_DEVERR_STEP_WAIT);
                    *abort = 1;
                    ok = false;
                    break;
                  }
                }
              }
            }
            if (ok) {
              uint8_t* dst = s.w + slot * kSlotW;
              uint64_t* bar = &s.full[slot];
              if (op.kind == OP_ATTN) {
                const int i = jl >> 4, blk = (jl & 15) >> 1, kv = jl & 1;
                const int item = jj + i * G;
                const int sidx = item % S, bh = item / S;
                const int hh = bh % p.nkv, b = bh / p.nkv;
                const int row = op.cache_row0 + (b * p.nkv + hh) * p.max_len + sidx * kAttnPos + 16 * blk;
                const bool any = sidx * kAttnPos + 16 * blk <= pos;
                mbar_arrive_expect_tx(bar, any ? kSlotW : 0);
                if (any) {
                  const CUtensorMap* m = &p.maps[kv == 0 ? p.kmap : p.vmap];
                  tma_load_2d(dst, m, 0, row, bar);
                  tma_load_2d(dst + 2048, m, 64, row, bar);
                }
              } else if (op.kind == OP_HEAD) {
                const int per_round = 8 * op.stages;
                const int r = jl / per_round, rem = jl - r * per_round;
                const int nr = min(8, nch - 8 * r);
                const int k = rem / nr, w = rem - k * nr;
                mbar_arrive_expect_tx(bar, kSlotW);
                tma_load_2d(dst, &p.maps[op.map], k * 64, (c0 + 8 * r + w) * 32, bar);
              } else {
                const int u = jl / halves, h = jl - u * halves;
                const int c = c0 + u / nst, st = st0 + u % nst;
                const int col = c * 32 + h * op.N;
                const CUtensorMap* mq = &p.maps[op.map];
                uint8_t* sz = s.sz + slot * kSlotSZ;
                mbar_arrive_expect_tx(bar, kSlotW + kSlotSZ);
                tma_load_2d(dst, mq, col, st * 32, bar);
                tma_load_2d(sz, mq + 1, col, st * 2, bar);
                tma_load_2d(sz + 128, mq + 2, col, st * 2, bar);
              }
            }
          }
          __syncwarp(0xffu);
          armed_end = base + min(j0 + kPLanes, n);
          if (__any_sync(0xffu, !ok)) {
            live = false;
          } else if (lane == 0) {
            __threadfence_block();
            *reinterpret_cast<volatile int*>(&s_issued) = armed_end;
          }
        }
        base += n;
      }
      // copies still in flight must land before the shared memory goes away (only after a give-up:
      // otherwise every armed slot was consumed)
      if (lane == 0 && *abort) {
        const uint64_t t0 = globaltimer_ns();
        for (int i = max(0, armed_end - p.nslots); i < armed_end; ++i)
          while (!mbar_try_wait(&s.full[i % p.nslots], (i / p.nslots) & 1) && globaltimer_ns() - t0 < 500000000ull) {
          }
      }
    }
    __syncwarp();
  } else if (warp < kCWarps) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
    // ================================================================ consumer warps
    Ring ring;
    ring.s = s;
    ring.nslots = p.nslots;
    ring.rcp = p.nslots_rcp;
    ring.issued = &s_issued;
    ring.abort = abort;
    ring.err = p.err;
    ring.seen = 0;
    ring.waited = 0;
    ring.timed = p.trace != nullptr;
    __shared__ unsigned long long s_waited;
    Poller pl(abort, p.err);
    const uint32_t epoch = s_epoch;
    int base_it = 0;
    unsigned long long* trace = p.trace ? p.trace + static_cast<size_t>(cta) * (p.n_ops + 1) * kTraceSlots : nullptr;
    if (trace && tid == 0) trace[p.n_ops * kTraceSlots] = globaltimer_ns();
    // does this CTA take part in op j (attention: has it an item; others: is it a participant)
    auto takes_part = [&](int j) {
      const Ctl cj = ctl[j];
      return cj.kind == OP_ATTN ? (pos >= 0 && op_slots(cj, cta, G, p.M, p.nkv, pos) > 0)
                                : participant(cta, cj.cta0, cj.ncta, G) >= 0;
    };
    constexpr int kOpWords = static_cast<int>(sizeof(Op) / 16);
    static_assert(sizeof(Op) % 16 == 0 && kOpWords <= 32, "Op is copied in 16-byte words by one warp");
    int cur = 0;       // s_ops[cur] holds the op being run
    int fetched = -1;  // (warp 0) the op whose descriptor is in flight to s_ops[cur]
    for (int j = 0; j < p.n_ops; ++j) {
      const Ctl cj = ctl[j];
      const int nslots_op = pos >= 0 ? op_slots(cj, cta, G, p.M, p.nkv, pos) : 0;
      if (!takes_part(j)) continue;
      if (trace && tid == 0) trace[j * kTraceSlots] = globaltimer_ns();
      // The descriptors come from global memory asynchronously: op j's was requested while the
      // previous op ran (the first one now), the next op's is requested here into the other buffer,
      // whose readers passed the barrier that ended the previous op.
      if (warp == 0) {
        if (fetched != j && lane < kOpWords) cp_async16(&s_ops[cur], lane, p.ops + j);
        int jn = j + 1;
        while (jn < p.n_ops && !takes_part(jn)) ++jn;
        cp_async_commit();
        if (jn < p.n_ops && lane < kOpWords) cp_async16(&s_ops[cur ^ 1], lane, p.ops + jn);
        cp_async_commit();
        cp_async_wait_group1();  // op j's copy landed; op jn's stays in flight
        fetched = jn;
      }
      const Op& op = s_ops[cur];
      if (tid == 0) {
        s_stop = *abort;
        if (trace) trace[j * kTraceSlots + 1] = globaltimer_ns();
      }
      consumers_sync();
      // no wait here: the op's loads of its input poll the tagged words themselves
      Tags tg;
      tg.x16 = tag16(epoch, p.n_ops, op.xop);
      tg.r16 = tag16(epoch, p.n_ops, op.rop);
      tg.o16 = tag16(epoch, p.n_ops, j);
      tg.x32 = tag32(epoch, p.n_ops, op.xop);
      tg.o32 = tag32(epoch, p.n_ops, j);
      if (!s_stop) {  // one decision for the whole CTA: the branches below hold barriers
        if (op.kind == OP_ATTN) {
          const int S = attn_splits(pos);
          const int items = p.M * p.nkv * S;
          int b = base_it;
          for (int item = (cta - op.cta0 + G) % G; item < items; item += G) {
            run_attention_item(p, op, tg, ring, as, b, item, pos, S, pl,
                               trace && tid == 0 && b == base_it ? trace + j * kTraceSlots + 7 : nullptr);
            b += 16;
            if (tid == 0) s_stop = *abort;
            consumers_sync();
            if (s_stop) break;
          }
        } else {
          const int jj = participant(cta, op.cta0, op.ncta, G);
          const Work wk = op_work(op, jj);
          const int c0 = wk.c0, c1 = wk.c1;
          if (op.kind == OP_HEAD) {
            stage_head_input(p, op, tg, s, s_inv, s_part, pl);
            if (trace && tid == 0) trace[j * kTraceSlots + 2] = globaltimer_ns();
            run_head(p, op, ring, base_it, c0, c1, s_best_v, s_best_i);
            if (trace && tid == 0) trace[j * kTraceSlots + 3] = globaltimer_ns();
            consumers_sync();
            if (tid < p.M) {  // this CTA's best per row, then the grid's by the last to arrive
              float bv = -INFINITY;
              int bi = 0x7fffffff;
              for (int w = 0; w < kCWarps; ++w) better(bv, bi, s_best_v[w * kMaxRows + tid], s_best_i[w * kMaxRows + tid]);
              p.head_val[cta * kMaxRows + tid] = bv;
              p.head_idx[cta * kMaxRows + tid] = bi;
            }
            consumers_sync();
            if (tid == 0) {
              fence_release_gpu();
              const unsigned prev = atomicAdd(p.head_count, 1u);
              s_head_last = prev == static_cast<unsigned>(op.ncta - 1);
              if (s_head_last) {
                *p.head_count = 0;
                __threadfence();
              }
            }
            consumers_sync();
            if (s_head_last) {
              // every CTA's best of every row at once (one load per thread), then per row a warp
              // reduces them (max, ties to the lowest index: order-independent)
              float* rv = s.red;
              int* ri = reinterpret_cast<int*>(s.red) + G * kMaxRows;
              for (int e = tid; e < G * p.M; e += kConsumers) {
                const int q = e / p.M, m = e % p.M;
                rv[q * kMaxRows + m] = __ldcg(p.head_val + q * kMaxRows + m);
                ri[q * kMaxRows + m] = __ldcg(p.head_idx + q * kMaxRows + m);
              }
              consumers_sync();
              if (warp < p.M) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int q = lane; q < G; q += 32) better(bv, bi, rv[q * kMaxRows + warp], ri[q * kMaxRows + warp]);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                  const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                  const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                  better(bv, bi, ov, oi);
                }
                if (lane == 0) {
                  p.tok[warp] = bi;
                  if (p.hist != nullptr) p.hist[warp * p.hist_ld + pos] = bi;
                }
              }
            }
            consumers_sync();
            if (s_head_last && tid == 0) *p.pos = pos + 1;
          } else {
            stage_int4_input(p, op, tg, s, jj == 0, s_inv, s_part, wk.st0, wk.st1, pos, pl);
            if (trace && tid == 0) trace[j * kTraceSlots + 2] = globaltimer_ns();
            run_int4(p, op, tg, ring, base_it, wk, op.ksplit > 1 ? jj % op.ksplit : 0,
                     trace && tid == 0 ? trace + j * kTraceSlots + 3 : nullptr);
          }
        }
      }
      consumers_sync();
      if (trace) {  // the slowest warp's cycles spent waiting for ring slots in this op
        if (tid == 0) s_waited = 0;
        consumers_sync();
        if (lane == 0) atomicMax(&s_waited, static_cast<unsigned long long>(ring.waited));
        ring.waited = 0;
        consumers_sync();
      }
      if (tid == 0 && trace) {
        trace[j * kTraceSlots + 4] = globaltimer_ns();
        trace[j * kTraceSlots + 5] = trace[j * kTraceSlots + 4];  // no arrival: consumers poll the words
        trace[j * kTraceSlots + 6] = s_waited;
      }
      base_it += nslots_op;
      cur ^= 1;
    }
    if (warp == 0) cp_async_wait_all();  // no copy into shared memory outlives the kernel
  }

  // ---------------------------------------------------------------- exit: the last CTA resets the counters
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(p.exit_count, 1u);
    if (p.trace) p.trace[static_cast<size_t>(cta) * (p.n_ops + 1) * kTraceSlots + p.n_ops * kTraceSlots + 1] = globaltimer_ns();
    if (prev == static_cast<unsigned>(G - 1)) {  // every CTA has left: the next launch takes new tags
      *p.head_count = 0;
      *p.exit_count = 0;
      *p.epoch = s_epoch + 1;
      __threadfence();
    }
  }
}

}  // namespace step
}  // namespace dk

// ================================================================================== host side
using namespace dk;
using namespace dk::step;

struct dk_step_plan {
  Params params;
  int grid;
  size_t smem;
  int device;
  std::vector<int> kinds;  // op kind per op of the program (dk_step_ops)
};

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Offsets of the pieces of a step workspace (all from its 256-byte aligned start).
struct Workspace {
  size_t counters, ops, maps, qkv, o, act, down, down_part, res0, res1, attn_part, head_val, head_idx, total;
  int n_ops, n_maps, max_splits;
};

Workspace workspace_layout(const dk_step_model* m, int grid) {
  Workspace w;
  const int L = m->n_layers;
  w.n_ops = 5 * L + 1;
  w.n_maps = 12 * L + 1 + 2;
  w.max_splits = m->max_len / kAttnPos;
  const int64_t M = m->batch, H = m->hidden, nqkv = (m->n_heads + 2 * m->n_kv) * m->head_dim;
  size_t off = 0;
  w.counters = off;  // epoch, exit count, argmax count
  off = align_up(off + 4 * 4, 256);
  w.ops = off;
  off = align_up(off + sizeof(Op) * w.n_ops, 256);
  w.maps = off;
  off = align_up(off + sizeof(CUtensorMap) * w.n_maps, 256);
  // activations between ops: tagged words, 4 bytes per fp16 value, 8 per fp32 partial
  w.qkv = off;
  off = align_up(off + 4 * M * nqkv, 256);
  w.o = off;
  off = align_up(off + 4 * M * H, 256);
  w.act = off;
  off = align_up(off + 4 * M * m->intermediate, 256);
  w.down = off;
  off = align_up(off + 4 * M * H, 256);
  w.down_part = off;
  off = align_up(off + 8 * kMaxKSplit * M * H, 256);
  w.res0 = off;
  off = align_up(off + 4 * M * H, 256);
  w.res1 = off;
  off = align_up(off + 4 * M * H, 256);
  w.attn_part = off;
  off = align_up(off + 8 * static_cast<size_t>(M) * m->n_kv * w.max_splits * kMaxGroup * kPartFloats, 256);
  w.head_val = off;
  off = align_up(off + 4 * static_cast<size_t>(grid) * kMaxRows, 256);
  w.head_idx = off;
  off = align_up(off + 4 * static_cast<size_t>(grid) * kMaxRows, 256);
  w.total = off;
  return w;
}

int check_model(const dk_step_model* m) {
  if (m == nullptr || m->layers == nullptr) return set_error(DK_ERR_INVALID, "step: model description is NULL");
  if (m->n_layers <= 0 || m->batch <= 0 || m->hidden <= 0 || m->vocab <= 0 || m->max_len <= 0)
    return set_error(DK_ERR_INVALID, "step: sizes must be positive");
  if (m->batch > kMaxRows) return set_error(DK_ERR_UNSUPPORTED, "step: batch %d (at most %d rows)", m->batch, kMaxRows);
  if (m->head_dim != kHd) return set_error(DK_ERR_UNSUPPORTED, "step: head_dim %d (128 only)", m->head_dim);
  if (m->n_kv <= 0 || m->n_heads % m->n_kv != 0 || m->n_heads / m->n_kv > kMaxGroup)
    return set_error(DK_ERR_UNSUPPORTED, "step: %d query heads over %d kv heads", m->n_heads, m->n_kv);
  if (m->hidden % 256 || m->intermediate % 256 || (m->n_heads * kHd) % 256)
    return set_error(DK_ERR_UNSUPPORTED, "step: hidden, intermediate and n_heads * head_dim must be multiples of 256");
  if (m->vocab % 32 || m->max_len % kAttnPos)
    return set_error(DK_ERR_UNSUPPORTED, "step: vocab %% 32 == 0 and max_len %% 128 == 0 needed");
  if (static_cast<int64_t>(m->n_layers) * m->batch * m->n_kv * m->max_len >= (int64_t(1) << 31))
    return set_error(DK_ERR_INVALID, "step: the KV cache has too many rows");
  const void* ptrs[] = {m->embed, m->final_norm, m->lm_head, m->rope_cos, m->rope_sin, m->k_cache, m->v_cache};
  for (const void* q : ptrs)
    if (q == nullptr || !aligned16(q)) return set_error(DK_ERR_ALIGN, "step: model tensors must be non-NULL and 16-byte aligned");
  for (int l = 0; l < m->n_layers; ++l) {
    const dk_step_layer& y = m->layers[l];
    const void* lp[] = {y.input_norm, y.post_norm, y.qkv_qweight, y.qkv_scales, y.qkv_zeros, y.o_qweight, y.o_scales,
                        y.o_zeros, y.gate_up_qweight, y.gate_up_scales, y.gate_up_zeros, y.down_qweight,
                        y.down_scales, y.down_zeros};
    for (const void* q : lp)
      if (q == nullptr || !aligned16(q))
        return set_error(DK_ERR_ALIGN, "step: layer %d: weights must be non-NULL and 16-byte aligned", l);
  }
  return DK_OK;
}

// Shared memory: ring slots as many as fit next to the staged input, the {C, X} table and the
// reduction scratch.
bool plan_smem(const dk_step_model* m, int* nslots, int* xs_pitch, int* red_bytes, size_t* smem) {
  const int kmax = std::max(std::max(m->hidden, m->intermediate), m->n_heads * kHd);
  *xs_pitch = kmax * 2 + kXsPad;
  const int red_int4 = kMaxChunks * kCWarps * 2 * kMaxRows * 32 * 4;
  const int red_attn = (kCWarps * kMaxGroup * kPartFloats + kCWarps * kMaxGroup + 2 * kMaxGroup) * 4;
  *red_bytes = std::max(red_int4, red_attn);
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, decode_step_kernel) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  const int limit = device_info().max_smem_optin - static_cast<int>(fa.sharedSizeBytes);
  int n = 64;
  const int n_ops = 5 * m->n_layers + 1;
  while (n >= 16 && static_cast<int>(smem_layout(n, m->batch, *xs_pitch, kmax, *red_bytes, n_ops).total) + 1024 > limit) --n;
  if (n < 16) return false;
  *nslots = n;
  *smem = smem_layout(n, m->batch, *xs_pitch, kmax, *red_bytes, n_ops).total + 1024;
  return true;
}

}  // namespace

extern "C" int dk_step_workspace_bytes(const dk_step_model* m, uint64_t* bytes) {
  int rc = check_model(m);
  if (rc != DK_OK) return rc;
  if (bytes == nullptr) return set_error(DK_ERR_INVALID, "step: bytes is NULL");
  *bytes = workspace_layout(m, device_info().num_sms).total;
  return DK_OK;
}

extern "C" int dk_step_create(const dk_step_model* m, void* workspace, uint64_t bytes, dk_step_plan** out) {
  int rc = check_model(m);
  if (rc != DK_OK) return rc;
  if (out == nullptr || workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(DK_ERR_INVALID, "step: workspace must be non-NULL and 256-byte aligned");
  const DeviceInfo& dev = device_info();
  const int G = dev.num_sms;
  const Workspace w = workspace_layout(m, G);
  if (bytes < w.total) return set_error(DK_ERR_INVALID, "step: workspace of %llu bytes, %zu needed",
                                        (unsigned long long)bytes, w.total);
  int nslots = 0, xs_pitch = 0, red_bytes = 0;
  size_t smem = 0;
  if (!plan_smem(m, &nslots, &xs_pitch, &red_bytes, &smem))
    return set_error(DK_ERR_UNSUPPORTED, "step: the staged rows leave no room for the weight ring");
  const int kmax = std::max(std::max(m->hidden, m->intermediate), m->n_heads * kHd);

  char* ws = static_cast<char*>(workspace);
  const int L = m->n_layers, M = m->batch, H = m->hidden, I = m->intermediate;
  const int nqkv = (m->n_heads + 2 * m->n_kv) * kHd, nqd = m->n_heads * kHd;
  std::vector<CUtensorMap> maps(w.n_maps);
  std::vector<Op> ops;
  ops.reserve(w.n_ops);
  auto int4_maps = [&](int idx, const int32_t* q, const void* sc, const void* z, int64_t N, int64_t K) {
    return make_tensor_map_2d(&maps[idx], q, CU_TENSOR_MAP_DATA_TYPE_INT32, N, K / 8, N * 4, 32, 32,
                              CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_tensor_map_2d(&maps[idx + 1], sc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K / 128, N * 2, 32, 2,
                              CU_TENSOR_MAP_SWIZZLE_NONE) &&
           make_tensor_map_2d(&maps[idx + 2], z, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K / 128, N * 2, 32, 2,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
  };
  uint32_t* qkv = reinterpret_cast<uint32_t*>(ws + w.qkv);
  uint32_t* o = reinterpret_cast<uint32_t*>(ws + w.o);
  uint32_t* act = reinterpret_cast<uint32_t*>(ws + w.act);
  uint32_t* down = reinterpret_cast<uint32_t*>(ws + w.down);
  unsigned long long* down_part = reinterpret_cast<unsigned long long*>(ws + w.down_part);
  // down_proj in K slices over more CTAs: its 48-ish chunks alone would leave most SMs idle and give
  // each CTA the whole 8960-long K; the consumer (next qkv, or the lm_head) adds the fp32 partials
  int down_split = 1;
  while (down_split < kMaxKSplit && (H / 32) * (down_split + 1) <= G && (I / 256) / (down_split + 1) >= 2)
    ++down_split;
  uint32_t* res[2] = {reinterpret_cast<uint32_t*>(ws + w.res0), reinterpret_cast<uint32_t*>(ws + w.res1)};
  // Participants. An op spreads over as many CTAs as it has chunks (each CTA multiplies whole
  // chunks: no cross-CTA split-K), starting where the previous op's participants ended, so the
  // weights of consecutive ops are fetched by different SMs.
  int next_cta = 0;
  auto place = [&](Op& op) {
    op.ncta = std::min(op.units, G);
    op.cta0 = op.ncta == G ? 0 : next_cta % G;
    next_cta = (op.cta0 + op.ncta) % G;
  };
  int map = 0;
  int r_in = -1;  // residual buffer holding the current residual stream (-1: none yet)
  int r_op = -1;  // program index of the op that wrote it (the tag its words carry)
  int down_op = -1, qkv_op = -1, attn_op = -1, o_op = -1, gu_op = -1;
  for (int l = 0; l < L; ++l) {
    const dk_step_layer& y = m->layers[l];
    Op q = {};
    q.kind = OP_QKV;
    q.layer = l;
    q.units = nqkv / 32;
    q.stages = H / 256;
    q.K = H;
    q.N = nqkv;
    q.map = map;
    if (!int4_maps(map, y.qkv_qweight, y.qkv_scales, y.qkv_zeros, nqkv, H)) return DK_ERR_CUDA;
    map += 3;
    q.from_embed = l == 0;
    q.ksplit = 1;
    q.x = l == 0 ? nullptr : down;
    if (l > 0 && down_split > 1) {
      q.x = nullptr;
      q.xsplit = down_split;
      q.xp = down_part;
      q.xbias = static_cast<const __half*>(m->layers[l - 1].down_bias);
    }
    q.res_in = l == 0 ? nullptr : res[r_in];
    q.res_out = res[l == 0 ? 0 : 1 - r_in];
    q.norm_w = static_cast<const __half*>(y.input_norm);
    q.bias = static_cast<const __half*>(y.qkv_bias);
    q.y = qkv;
    q.xop = down_op;
    q.rop = r_op;
    place(q);
    qkv_op = static_cast<int>(ops.size());
    ops.push_back(q);
    r_in = l == 0 ? 0 : 1 - r_in;
    r_op = qkv_op;

    Op a = {};
    a.ksplit = 1;
    a.kind = OP_ATTN;
    a.layer = l;
    a.x = qkv;
    a.cta0 = next_cta;
    a.ncta = 0;
    a.cache_row0 = l * M * m->n_kv * m->max_len;
    a.xop = qkv_op;
    attn_op = static_cast<int>(ops.size());
    ops.push_back(a);
    next_cta = (next_cta + M * m->n_kv * 8) % G;

    Op op = {};
    op.ksplit = 1;
    op.kind = OP_O;
    op.layer = l;
    op.units = H / 32;
    op.stages = nqd / 256;
    op.K = nqd;
    op.N = H;
    op.map = map;
    if (!int4_maps(map, y.o_qweight, y.o_scales, y.o_zeros, H, nqd)) return DK_ERR_CUDA;
    map += 3;
    op.xattn = 1;
    op.xp = reinterpret_cast<const unsigned long long*>(ws + w.attn_part);
    op.bias = static_cast<const __half*>(y.o_bias);
    op.y = o;
    op.xop = attn_op;
    place(op);
    o_op = static_cast<int>(ops.size());
    ops.push_back(op);

    Op gu = {};
    gu.ksplit = 1;
    gu.kind = OP_GATEUP;
    gu.layer = l;
    gu.units = I / 32;
    gu.stages = H / 256;
    gu.K = H;
    gu.N = I;
    gu.map = map;
    if (!int4_maps(map, y.gate_up_qweight, y.gate_up_scales, y.gate_up_zeros, 2 * I, H)) return DK_ERR_CUDA;
    map += 3;
    gu.x = o;
    gu.res_in = res[r_in];
    gu.res_out = res[1 - r_in];
    gu.norm_w = static_cast<const __half*>(y.post_norm);
    gu.bias = static_cast<const __half*>(y.gate_up_bias);
    gu.y = act;
    gu.xop = o_op;
    gu.rop = r_op;
    place(gu);
    gu_op = static_cast<int>(ops.size());
    ops.push_back(gu);
    r_in = 1 - r_in;
    r_op = gu_op;

    Op dn = {};
    dn.kind = OP_DOWN;
    dn.layer = l;
    dn.units = H / 32;
    dn.stages = I / 256;
    dn.K = I;
    dn.N = H;
    dn.map = map;
    if (!int4_maps(map, y.down_qweight, y.down_scales, y.down_zeros, H, I)) return DK_ERR_CUDA;
    map += 3;
    dn.x = act;
    dn.bias = static_cast<const __half*>(y.down_bias);
    dn.y = down;
    dn.ksplit = down_split;
    dn.xop = gu_op;
    if (down_split > 1) {
      dn.yp = down_part;
      dn.units = H / 32;
      dn.ncta = dn.units * down_split;
      dn.cta0 = next_cta % G;
      next_cta = (dn.cta0 + dn.ncta) % G;
    } else {
      place(dn);
    }
    down_op = static_cast<int>(ops.size());
    ops.push_back(dn);
  }
  Op hd = {};
  hd.ksplit = 1;
  hd.kind = OP_HEAD;
  hd.layer = L;
  hd.units = m->vocab / 32;
  hd.stages = H / 64;
  hd.K = H;
  hd.N = m->vocab;
  hd.map = map;
  if (!make_tensor_map_2d(&maps[map], m->lm_head, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, H, m->vocab, H * 2, 64, 32,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return DK_ERR_CUDA;
  map += 1;
  hd.x = down;
  if (down_split > 1) {
    hd.x = nullptr;
    hd.xsplit = down_split;
    hd.xp = down_part;
    hd.xbias = static_cast<const __half*>(m->layers[L - 1].down_bias);
  }
  hd.res_in = res[r_in];
  hd.xop = down_op;
  hd.rop = r_op;
  hd.norm_w = static_cast<const __half*>(m->final_norm);
  hd.y = nullptr;  // the logits pointer is per call (dk_step_run)
  hd.ncta = G;
  hd.cta0 = 0;
  ops.push_back(hd);
  for (const Op& op : ops) {
    if (op.kind != OP_ATTN && op.kind != OP_HEAD && op.ksplit <= 1 && (op.units + op.ncta - 1) / op.ncta > kMaxChunks)
      return set_error(DK_ERR_UNSUPPORTED, "step: an op needs more than %d chunks per CTA", kMaxChunks);
    if (op.ksplit > 1 && (op.norm_w != nullptr || op.ncta > G || op.kind == OP_GATEUP))
      return set_error(DK_ERR_UNSUPPORTED, "step: internal: a split-K op with a norm, a pair epilogue or too many CTAs");
  }
  const uint64_t rows = static_cast<uint64_t>(L) * M * m->n_kv * m->max_len;
  const int kmap = map, vmap = map + 1;
  if (!make_tensor_map_2d(&maps[kmap], m->k_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kHd, rows, kHd * 2, 64, 16,
                          CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&maps[vmap], m->v_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kHd, rows, kHd * 2, 64, 16,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return DK_ERR_CUDA;

  // set-up copies (synchronous: before any capture)
  cudaError_t e = cudaMemset(ws + w.counters, 0, w.ops - w.counters);
  if (e == cudaSuccess) e = cudaMemcpy(ws + w.ops, ops.data(), sizeof(Op) * ops.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(ws + w.maps, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "step: set-up copies: %s", cudaGetErrorString(e));

  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    const int limit = opt_in_dynamic_smem(decode_step_kernel);
    if (limit < static_cast<int>(smem))
      return set_error(DK_ERR_UNSUPPORTED, "step: %zu bytes of shared memory do not fit", smem);
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_step_kernel, kThreads, smem) != cudaSuccess || occ < 1) {
    cudaGetLastError();
    return set_error(DK_ERR_UNSUPPORTED, "step: the kernel does not fit on an SM");
  }
  // the consumers' setmaxnreg.inc waits for registers the producer's warpgroup released: the launch
  // must hold at least the split's total, or that wait would never end
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, decode_step_kernel) != cudaSuccess ||
      fa.numRegs * kThreads < 128 * kProducerRegs + kConsumers * kConsumerRegs) {
    cudaGetLastError();
    return set_error(DK_ERR_UNSUPPORTED, "step: compiled with %d registers a thread, the register split needs %d",
                     fa.numRegs, kLaunchRegs);
  }

  dk_step_plan* plan = new dk_step_plan();
  Params& p = plan->params;
  p.ops = reinterpret_cast<const Op*>(ws + w.ops);
  p.n_ops = static_cast<int>(ops.size());
  p.maps = reinterpret_cast<const CUtensorMap*>(ws + w.maps);
  p.kmap = kmap;
  p.vmap = vmap;
  p.M = M;
  p.H = H;
  p.nq = m->n_heads;
  p.nkv = m->n_kv;
  p.max_len = m->max_len;
  p.vocab = m->vocab;
  p.nslots = nslots;
  p.nslots_rcp = static_cast<uint32_t>((0x100000000ull + nslots - 1) / nslots);
  p.kmax = kmax;
  p.xs_pitch = xs_pitch;
  p.red_bytes = red_bytes;
  p.eps = m->eps;
  p.attn_scale = 1.0f / sqrtf(static_cast<float>(kHd));
  p.embed = static_cast<const __half*>(m->embed);
  p.rope_cos = static_cast<const __half*>(m->rope_cos);
  p.rope_sin = static_cast<const __half*>(m->rope_sin);
  p.k_cache = static_cast<__half*>(m->k_cache);
  p.v_cache = static_cast<__half*>(m->v_cache);
  unsigned* ctr = reinterpret_cast<unsigned*>(ws + w.counters);
  p.epoch = ctr;
  p.exit_count = ctr + 1;
  p.head_count = ctr + 2;
  p.attn_part = reinterpret_cast<unsigned long long*>(ws + w.attn_part);
  p.head_val = reinterpret_cast<float*>(ws + w.head_val);
  p.head_idx = reinterpret_cast<int*>(ws + w.head_idx);
  p.err = dev.err_word;
  plan->grid = G;
  plan->smem = smem;
  for (const Op& op : ops) plan->kinds.push_back(op.kind);
  cudaGetDevice(&plan->device);
  *out = plan;
  return DK_OK;
}

namespace {
int step_launch(const dk_step_plan* plan, int64_t* tokens, int64_t* pos, int64_t* history, int64_t history_ld,
                void* logits, uint64_t* trace, dk_stream_t stream) {
  if (plan == nullptr || tokens == nullptr || pos == nullptr)
    return set_error(DK_ERR_INVALID, "step_run: plan, tokens and pos must be non-NULL");
  if (history != nullptr && history_ld < plan->params.max_len)
    return set_error(DK_ERR_INVALID, "step_run: history rows need at least max_len entries");
  Params p = plan->params;
  p.tok = tokens;
  p.pos = pos;
  p.hist = history;
  p.hist_ld = history_ld;
  p.logits = static_cast<__half*>(logits);
  p.trace = reinterpret_cast<unsigned long long*>(trace);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = plan->smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_step_kernel, p);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "step_run launch: %s", cudaGetErrorString(e));
  return DK_OK;
}
}  // namespace

extern "C" int dk_step_run(const dk_step_plan* plan, int64_t* tokens, int64_t* pos, int64_t* history,
                           int64_t history_ld, void* logits, dk_stream_t stream) {
  return step_launch(plan, tokens, pos, history, history_ld, logits, nullptr, stream);
}

extern "C" int dk_step_trace_bytes(const dk_step_plan* plan, uint64_t* bytes) {
  if (plan == nullptr || bytes == nullptr) return set_error(DK_ERR_INVALID, "step_trace_bytes: NULL argument");
  *bytes = static_cast<uint64_t>(plan->grid) * (plan->params.n_ops + 1) * kTraceSlots * 8;
  return DK_OK;
}

extern "C" int dk_step_trace(const dk_step_plan* plan, int64_t* tokens, int64_t* pos, int64_t* history,
                             int64_t history_ld, void* logits, uint64_t* trace, dk_stream_t stream) {
  if (trace == nullptr || (reinterpret_cast<uintptr_t>(trace) & 7))
    return set_error(DK_ERR_INVALID, "step_trace: trace must be a non-NULL, 8-byte aligned device buffer");
  return step_launch(plan, tokens, pos, history, history_ld, logits, trace, stream);
}

extern "C" int dk_step_ops(const dk_step_plan* plan, int32_t* kinds, int32_t capacity, int32_t* n_ops) {
  if (plan == nullptr || n_ops == nullptr) return set_error(DK_ERR_INVALID, "step_ops: NULL argument");
  *n_ops = plan->params.n_ops;
  if (kinds != nullptr) {
    for (int j = 0; j < plan->params.n_ops && j < capacity; ++j) kinds[j] = plan->kinds[j];
  }
  return DK_OK;
}

extern "C" int dk_step_destroy(dk_step_plan* plan) {
  delete plan;
  return DK_OK;
}
