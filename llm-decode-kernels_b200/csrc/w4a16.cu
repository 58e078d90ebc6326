// W4A16 matmul for decode (M <= 16 rows per launch): y = x @ dequant(W).T (+ bias).
//
// Replaces the reference's Triton GEMV/GEMM decode paths (kernels/w4a16.py:31-160) and its
// CUDA-core decode kernel (kernels/cuda/w4a16_decode.cu:29-121) with one sm_100a kernel.
//
// * Weight stream by TMA. The packed weights qweight[K/8, N] are read as 2-D boxes of 32 columns x
//   32 packed rows (4 KB, one "chunk-stage") with 128-byte swizzling; each box's scale and zero rows
//   come as two more 2-D boxes. A producer warp keeps a ring of `nbuf` stages full (one mbarrier per
//   stage counts the bytes); consumer warps release stages through a second mbarrier.
// * Persistent CTAs. Output columns are cut into 32-column chunks and every CTA takes a contiguous,
//   balanced run of chunks (ranges differ by at most one chunk), processed CW chunks at a time:
//   consumer warp w owns chunk w of the current tile for the whole K range, so no reduction between
//   warps is needed and a warp writes its outputs straight from registers.
// * Activations in shared memory. Each CTA copies its K slice of x once (after waiting for the
//   previous kernel), with the K order permuted to match the MMA fragments below.
// * Dequantization with the reference's rounding. A 32-bit word holds 8 K values of one column.
//   LOP3 with the 0x6400 exponent (the "magic number" int4 -> fp16 conversion of Kim et al., "Who
//   Says Elephants Can't Run?", and FasterTransformer) gives 1024+q in fp16; subtracting 1024+z is
//   exact and one fp16 multiply by s rounds once - the same value as the reference's
//   `(q.to(fp16) - z) * s` (kernels/reference.py:35, kernels/w4a16.py:84).
// * Dot products on tensor cores, fp32 accumulation. mma.m16n8k16 with the dequantized weights as
//   the 16-row A operand (MMA rows = output columns) and x as the B operand (MMA columns = batch
//   rows), so the multiply-adds cost the ALUs nothing and 1..16 batch rows cost the same per weight.
//   Within an MMA the K order is permuted (nibble pairs (0,4),(1,5),(2,6),(3,7) of a word, packed
//   rows 2t / 2t+1 of a swizzle group); x is staged with the same permutation, so every product
//   pairs the right x with the right weight.
// * Split-K without workspace or atomics. For layers with few columns the S K-slices of one tile
//   run as the S CTAs of a thread-block cluster; partial sums meet in distributed shared memory and
//   are added in rank order (deterministic). This replaces the reference's zero-fill + fp32 atomics
//   + cast kernels (kernels/w4a16.py:271-275, kernels/cuda/w4a16_decode.cu:161-180).
// * Programmatic dependent launch. With DK_FLAG_STATIC_WEIGHTS the producer starts streaming
//   weights before the previous kernel on the stream has finished; x is read only after
//   griddepcontrol.wait.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"

namespace dk {
namespace {

constexpr int kStageRows = 32;               // packed rows per stage (256 K values)
constexpr int kBoxBytes = kStageRows * 128;  // one 32-column x 32-row box of int32
constexpr int kGroupRows = 16;               // fast path: group_size 128
constexpr int kGroupsPerStage = kStageRows / kGroupRows;
constexpr int kSZBytes = kGroupsPerStage * 32 * 2;  // one scale (or zero) box per chunk-stage
constexpr int kChunkStageBytes = kBoxBytes + 2 * kSZBytes;
constexpr int kXsPad = 16;  // bytes added to each x row in shared memory (bank spread)

struct GemvParams {
  const __half* x;
  int64_t ldx;
  const __half* bias;
  __half* y;
  int64_t ldy;
  int M, N, K;
  int stages_total;  // ceil(K / 256)
  int split_stages;  // stages per cluster rank
  int chunks;        // ceil(N / 32)
  int nbuf;          // ring depth
  uint32_t nbuf_rcp; // ceil(2^32 / nbuf): it / nbuf == __umulhi(it, nbuf_rcp) for the small it used here
  int xs_pitch;      // bytes per staged x row
  int static_weights;
  int swiglu_i;      // > 0: fused SwiGLU over gate columns [0, I) and up columns [I, 2I); y is [M, I]
  // optional fused residual + RMSNorm of x before the matmul (norm_w == nullptr: x as given)
  const __half* norm_w;
  const __half* res;  // may be nullptr (norm without residual add)
  int64_t ldr;
  __half* res_out;    // receives x + res (written by one CTA) when res != nullptr
  int64_t ldro;
  float eps;
  int* err;
  L2Prefetch pf;  // ranges to pull into L2 for a later launch (a hint)
  // x given as the fp32 K-slice partial sums of the previous projection (xp != nullptr): x = fp16(
  // xp[0] + ... + xp[xparts - 1] (+ xbias)), each [M, K], added in slice order
  const float* xp;
  int xparts;
  const __half* xbias;
  // this launch's K-slice partial sums instead of y (yp != nullptr, no bias): yp[slice][M][N] fp32
  float* yp;
  TPArgs tp;      // tp.world > 0: row-sharded launch with the allreduce fused in (see tp_finish)
};

struct SmemLayout {
  int w_off, sz_off, xs_off, cx_off, red_off, bar_off, total;
};

constexpr int kWarps = 8;  // consumer warps per CTA (plus one producer warp)

// Offsets from the 1024-byte aligned base of dynamic shared memory.
__host__ __device__ inline SmemLayout smem_layout(int cw, int nbuf, int M, int xs_pitch, int /*split*/) {
  const int wpc = kWarps / cw;
  SmemLayout L;
  L.w_off = 0;
  L.sz_off = nbuf * cw * kBoxBytes;
  L.xs_off = L.sz_off + nbuf * cw * 2 * kSZBytes;
  // per (group, row) corrections of the factored path: {C, X} fp32 for 16 rows = 128 bytes a group
  L.cx_off = L.xs_off + ((M * xs_pitch + 15) / 16) * 16;
  L.red_off = L.cx_off + 2 * ((xs_pitch - kXsPad) / (kStageRows * 16)) * 128;
  // reduction scratch, always present: the fused-SwiGLU and split-K epilogues use it at any wpc
  L.bar_off = L.red_off + wpc * M * cw * 32 * 4;
  L.total = L.bar_off + 2 * nbuf * 8;
  return L;
}

// Fused SwiGLU epilogue with the reference's rounding: the gate_up matmul output is rounded to
// fp16 (kernels/w4a16.py:95), silu runs in fp32 on the fp16 gate and is rounded to fp16, and the
// product with the fp16 up value is an fp16 multiply (kernels/swiglu.py:26-28).
__device__ __forceinline__ __half swiglu_out(float g, float u, const __half* bias, int n, int I) {
  if (bias != nullptr) {
    g += __half2float(bias[n]);
    u += __half2float(bias[I + n]);
  }
  const float gf = __half2float(__float2half_rn(g));
  const __half act = __float2half_rn(__fdiv_rn(gf, __fadd_rn(1.0f, expf(-gf))));
  return __hmul_rn(act, __float2half_rn(u));
}

// One chunk-stage (32 columns x 32 packed rows) for one warp. EXACT: dequantize to fp16 exactly
// like the reference and accumulate into acc. Otherwise (factored, the reference's FACTORED
// numerics, kernels/w4a16.py:116-119): the MMA sums x*(q-z) per group with exact fp16 operands and
// the group's scale multiplies the fp32 group sum, which saves the fp16 multiply per weight.
template <int NT, bool EXACT>
__device__ __forceinline__ void consume_chunk_stage(const uint8_t* __restrict__ wbox, const uint8_t* __restrict__ szb,
                                                    const uint8_t* __restrict__ xrow, int xs_pitch, int M, int g,
                                                    int t, float (&acc)[2][NT][4]) {
  const uint32_t k1024 = 0x64006400u, nk64 = 0xD400D400u, sixteenth = 0x2C002C00u;
#pragma unroll
  for (int half = 0; half < kGroupsPerStage; ++half) {
    const uint2 s4 = *reinterpret_cast<const uint2*>(szb + half * 64 + g * 8);
    const uint2 z4 = *reinterpret_cast<const uint2*>(szb + kSZBytes + half * 64 + g * 8);
    const uint32_t zz[4] = {prmt(z4.x, 0, 0x1010), prmt(z4.x, 0, 0x3232), prmt(z4.y, 0, 0x1010),
                            prmt(z4.y, 0, 0x3232)};
    uint32_t zA[4], nzB[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      zA[c] = hfma2_rn(zz[c], 0x3C003C00u, k1024);  // z + 1024, exact
      nzB[c] = hsub2_rn(nk64, zz[c]);                // -64 - z, exact
    }
    uint32_t sc[4];
    float scf[4];
    float accg[2][NT][4];
    if constexpr (EXACT) {
      sc[0] = prmt(s4.x, 0, 0x1010);
      sc[1] = prmt(s4.x, 0, 0x3232);
      sc[2] = prmt(s4.y, 0, 0x1010);
      sc[3] = prmt(s4.y, 0, 0x3232);
    } else {
      const __half2 s01 = *reinterpret_cast<const __half2*>(&s4.x);
      const __half2 s23 = *reinterpret_cast<const __half2*>(&s4.y);
      scf[0] = __low2float(s01);
      scf[1] = __high2float(s01);
      scf[2] = __low2float(s23);
      scf[3] = __high2float(s23);
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
          for (int c = 0; c < 4; ++c) accg[a][b][c] = 0.f;
    }
#pragma unroll
    for (int st4 = 0; st4 < 4; ++st4) {
      const int st = half * 4 + st4;
      const int r = 8 * (st >> 1) + 2 * t + (st & 1);  // packed row within the stage
      const uint4 wv = *reinterpret_cast<const uint4*>(wbox + r * 128 + ((g ^ (r & 7)) << 4));
      uint32_t bx[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = nt * 8 + g;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (m < M) v = *reinterpret_cast<const uint4*>(xrow + m * xs_pitch + r * 16);
        bx[nt][0] = v.x;
        bx[nt][1] = v.y;
        bx[nt][2] = v.z;
        bx[nt][3] = v.w;
      }
      const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t W[4][4];  // [column][nibble pair]: (q - z) (factored) or (q - z) * s (exact)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t w = words[c];
        const uint32_t w8 = w >> 8;
        W[c][0] = hsub2_rn(lop3_and_or(w, 0x000F000Fu, k1024), zA[c]);                 // q0, q4
        W[c][1] = hfma2_rn(lop3_and_or(w, 0x00F000F0u, k1024), sixteenth, nzB[c]);     // q1, q5
        W[c][2] = hsub2_rn(lop3_and_or(w8, 0x000F000Fu, k1024), zA[c]);                // q2, q6
        W[c][3] = hfma2_rn(lop3_and_or(w8, 0x00F000F0u, k1024), sixteenth, nzB[c]);    // q3, q7
        if constexpr (EXACT) {
#pragma unroll
          for (int i = 0; i < 4; ++i) W[c][i] = hmul2_rn(W[c][i], sc[c]);
        }
      }
      float(&dst)[2][NT][4] = EXACT ? acc : accg;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        // tile 0: MMA rows g <- column 4g, g+8 <- 4g+1 ; tile 1: columns 4g+2, 4g+3
        mma_16816(dst[0][nt], W[0][0], W[1][0], W[0][1], W[1][1], bx[nt][0], bx[nt][1]);
        mma_16816(dst[0][nt], W[0][2], W[1][2], W[0][3], W[1][3], bx[nt][2], bx[nt][3]);
        mma_16816(dst[1][nt], W[2][0], W[3][0], W[2][1], W[3][1], bx[nt][0], bx[nt][1]);
        mma_16816(dst[1][nt], W[2][2], W[3][2], W[2][3], W[3][3], bx[nt][2], bx[nt][3]);
      }
    }
    if constexpr (!EXACT) {
#pragma unroll
      for (int tile = 0; tile < 2; ++tile)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[tile][nt][e] = fmaf(scf[2 * tile + (e >> 1)], accg[tile][nt][e], acc[tile][nt][e]);
    }
  }
}

// ------------------------------------------------------------------ fused allreduce (row sharding)
// A row-sharded launch computes this rank's partial sums of y. Instead of storing them, the
// epilogue pushes each one, tagged with the low 32 bits of the launch's epoch, into slot
// (epoch & 1), row `rank`, of every rank's exchange buffer over NVLink (one 8-byte {value, epoch}
// store per value, so a value is valid exactly when its tag matches: no fence, no flag). tp_finish
// then polls the cells of this CTA's own columns from every rank (each rank launches the same grid,
// so CTA i covers the same columns everywhere) and adds them in rank order. Two slots suffice: a rank
// starts launch e + 2 only after its launch e + 1 finished, and every CTA of that launch read all
// ranks' launch e + 1 values, which they wrote after their launch e had finished reading.
// Called by every thread of the CTA after its last push. Columns: [c_begin*32, min(c_end*32, N)) with
// split 1; with a cluster split S the elements e = m*ncols + col with e % S == cluster rank.
__device__ void tp_finish(const GemvParams& p, unsigned long long ep, bool ok, int c_begin, int c_end, int upt,
                          int S, int crank) {
  const TPArgs& tp = p.tp;
  const uint32_t tag = static_cast<uint32_t>(ep);
  __shared__ int s_give_up;
  if (threadIdx.x == 0) s_give_up = ok ? 0 : 1;
  __syncthreads();
  if (ok) {
    volatile int* give_up = &s_give_up;
    if (S == 1) {
      const int n_lo = c_begin * 32, n_hi = min(c_end * 32, p.N);
      const int nq = (n_hi - n_lo) / 4;  // N % 8 == 0 on this path
      for (int e = threadIdx.x; e < p.M * nq; e += blockDim.x) {
        const int m = e / nq, n = n_lo + 4 * (e % nq);
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
        bool good = true;
        for (int q = 0; q < tp.world && good; ++q) {
          float v[4];
          good = tp_poll4(tp_cell(tp, tp.rank, ep, q, m, n), tag, v, give_up, p.err, tp.wait_ns);
#pragma unroll
          for (int c = 0; c < 4; ++c) sum[c] += v[c];
        }
        if (!good) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (p.bias != nullptr) sum[c] += __half2float(p.bias[n + c]);
          p.y[m * p.ldy + n + c] = __float2half_rn(sum[c]);
        }
      }
    } else {
      const int ncols = min(upt, c_end - c_begin) * 32;
      for (int e = threadIdx.x; e < p.M * ncols; e += blockDim.x) {
        if (e % S != crank) continue;
        const int m = e / ncols, n = c_begin * 32 + e % ncols;
        if (n >= p.N) continue;
        float a = 0.f;
        bool good = true;
        for (int q = 0; q < tp.world && good; ++q) {
          float v = 0.f;
          good = tp_poll1(tp_cell(tp, tp.rank, ep, q, m, n), tag, v, give_up, p.err, tp.wait_ns);
          a += v;
        }
        if (!good) continue;
        if (p.bias != nullptr) a += __half2float(p.bias[n]);
        p.y[m * p.ldy + n] = __float2half_rn(a);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(tp.arrive, 1u) == gridDim.x * gridDim.y - 1) {
    // last CTA of the launch: the next launch on this communicator uses epoch ep + 1
    *tp.arrive = 0;
    *reinterpret_cast<volatile unsigned long long*>(tp.epoch) = ep;
  }
}

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

// The default (factored) path without a per-weight zero subtraction. A word's nibble pairs become
// fp16 by LOP3 with the 0x6400 exponent alone: 1024 + q for the low nibble of a byte (even K) and
// 1024 + 16 q for the high nibble (odd K), whose x values were staged divided by 16. The MMA then
// sums x'(1024 + q') = C + sum(x q) over a group, where C = 1024 * sum(x') is a per-(group, row)
// constant computed once per CTA from the staged x, and X = sum over the group of the x each weight
// is effectively multiplied by; the group's result is s * (mma - C - z * X), the reference's
// FACTORED numerics (kernels/w4a16.py:116-119) with the zero point applied once per group.
// Shared-memory operands come by 32-bit address: wbox (the chunk-stage's swizzled weight box), szb
// (its scale and zero boxes), xrow (this stage's staged x), cxg (the stage's two {C, X} groups).
template <int NT>
__device__ __forceinline__ void consume_chunk_stage_f(uint32_t wbox, uint32_t szb, uint32_t xrow, uint32_t cxg,
                                                      int xs_pitch, int M, int g, int t, float (&acc)[2][NT][4]) {
  const uint32_t k1024 = 0x64006400u;
  // a lane reads packed rows r = 8 * (st / 2) + 2t + (st % 2): two lane-dependent bases
  const uint32_t w_even = wbox + (2 * t) * 128 + ((g ^ (2 * t)) << 4);
  const uint32_t w_odd = wbox + (2 * t + 1) * 128 + ((g ^ (2 * t + 1)) << 4);
  const uint32_t x_even = xrow + (2 * t) * 16, x_odd = xrow + (2 * t + 1) * 16;
#pragma unroll
  for (int half = 0; half < kGroupsPerStage; ++half) {
    const uint2 s4 = lds64(szb + half * 64 + g * 8);
    const uint2 z4 = lds64(szb + kSZBytes + half * 64 + g * 8);
    float accg[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) accg[a][b][c] = 0.f;
#pragma unroll
    for (int st4 = 0; st4 < 4; ++st4) {
      const int st = half * 4 + st4;
      const uint4 wv = lds128(((st & 1) ? w_odd : w_even) + 1024 * (st >> 1));
      uint32_t bx[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = nt * 8 + g;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (m < M) v = lds128(((st & 1) ? x_odd : x_even) + 128 * (st >> 1) + m * xs_pitch);
        bx[nt][0] = v.x;
        bx[nt][1] = v.y;
        bx[nt][2] = v.z;
        bx[nt][3] = v.w;
      }
      const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t W[4][4];  // [column][nibble pair]
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t w = words[c];
        const uint32_t w8 = w >> 8;
        W[c][0] = lop3_and_or(w, 0x000F000Fu, k1024);   // 1024 + q0, 1024 + q4
        W[c][1] = lop3_and_or(w, 0x00F000F0u, k1024);   // 1024 + 16 q1, 1024 + 16 q5
        W[c][2] = lop3_and_or(w8, 0x000F000Fu, k1024);  // q2, q6
        W[c][3] = lop3_and_or(w8, 0x00F000F0u, k1024);  // q3, q7
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_16816(accg[0][nt], W[0][0], W[1][0], W[0][1], W[1][1], bx[nt][0], bx[nt][1]);
        mma_16816(accg[0][nt], W[0][2], W[1][2], W[0][3], W[1][3], bx[nt][2], bx[nt][3]);
        mma_16816(accg[1][nt], W[2][0], W[3][0], W[2][1], W[3][1], bx[nt][0], bx[nt][1]);
        mma_16816(accg[1][nt], W[2][2], W[3][2], W[2][3], W[3][3], bx[nt][2], bx[nt][3]);
      }
    }
    const __half2 s01 = *reinterpret_cast<const __half2*>(&s4.x), s23 = *reinterpret_cast<const __half2*>(&s4.y);
    const __half2 z01 = *reinterpret_cast<const __half2*>(&z4.x), z23 = *reinterpret_cast<const __half2*>(&z4.y);
    const float sc[4] = {__low2float(s01), __high2float(s01), __low2float(s23), __high2float(s23)};
    const float zc[4] = {__low2float(z01), __high2float(z01), __low2float(z23), __high2float(z23)};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      // {C, X} of rows nt*8 + 2t and nt*8 + 2t + 1 (the D fragment's two batch rows)
      const uint4 cxr = lds128(cxg + half * 128 + (nt * 8 + 2 * t) * 8);
      const float cx[2][2] = {{__uint_as_float(cxr.x), __uint_as_float(cxr.y)},
                              {__uint_as_float(cxr.z), __uint_as_float(cxr.w)}};
#pragma unroll
      for (int tile = 0; tile < 2; ++tile)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = 2 * tile + (e >> 1), r = e & 1;
          acc[tile][nt][e] = fmaf(sc[col], accg[tile][nt][e] - fmaf(zc[col], cx[r][1], cx[r][0]), acc[tile][nt][e]);
        }
    }
  }
}

// Stage x[:, K slice of this CTA] into shared memory, each 8-element block permuted to
// (0,4,1,5,2,6,3,7) for the MMA fragments. With `norm_w` the staged rows are the fused residual
// add + RMSNorm of the input, with the rounding of kernels/rmsnorm.py:28-37 (and the rmsnorm kernel
// of this library): h = x + residual (fp16 add), var = sum(h^2)/K in fp32, out = w * fp16(h / sqrt(
// var + eps)); every CTA reads the whole row for the sum of squares (per-warp partials added in a
// fixed order: deterministic), and `writer` (one CTA) stores h as the new residual stream.
// The norm weights of the blocks this thread stages in a one-row launch (blocks kb0 + tid and
// kb0 + tid + 256 of its K slice): constant, so they are loaded before the wait for the previous
// kernel and are in registers when the normalization needs them.
struct NormW {
  uint4 w[2];
};
__device__ __forceinline__ NormW norm_w_prefetch(const GemvParams& p, int s_begin) {
  constexpr int kThr = kWarps * 32;
  NormW r;
  r.w[0] = r.w[1] = make_uint4(0, 0, 0, 0);
  if (p.norm_w == nullptr || p.M != 1) return r;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int k = (s_begin * kStageRows + static_cast<int>(threadIdx.x) + j * kThr) * 8;
    if (k < p.K) r.w[j] = __ldg(reinterpret_cast<const uint4*>(p.norm_w + k));
  }
  return r;
}

// 8 values of x at row m, K offset k (k % 8 == 0): the activations, or the rounded sum of the
// previous projection's partial sums (the same additions in the same order as its cluster reduction).
__device__ __forceinline__ uint4 load_x8(const GemvParams& p, int m, int k) {
  if (p.xp == nullptr) return __ldcg(reinterpret_cast<const uint4*>(p.x + m * p.ldx + k));
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int q = 0; q < p.xparts; ++q) {
    const float4* src = reinterpret_cast<const float4*>(p.xp + (static_cast<int64_t>(q) * p.M + m) * p.K + k);
    const float4 u = __ldcg(src), w = __ldcg(src + 1);
    a[0] += u.x;
    a[1] += u.y;
    a[2] += u.z;
    a[3] += u.w;
    a[4] += w.x;
    a[5] += w.y;
    a[6] += w.z;
    a[7] += w.w;
  }
  if (p.xbias != nullptr) {
    const uint4 bb = __ldg(reinterpret_cast<const uint4*>(p.xbias + k));
    const __half* bh = reinterpret_cast<const __half*>(&bb);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] += __half2float(bh[i]);
  }
  uint4 out;
  __half2* oh = reinterpret_cast<__half2*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) oh[i] = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
  return out;
}

template <int kBatch>
__device__ __forceinline__ void stage_x(const GemvParams& p, uint8_t* xs, float* cx, int s_begin, int nst, bool writer,
                                        bool factored, const NormW& nwp) {
  constexpr int kThr = kWarps * 32;
  const int tid = threadIdx.x;
  const int kb0 = s_begin * kStageRows;  // first packed row (block of 8 K values)
  const int nblk = nst * kStageRows;
  __shared__ float inv[16];
  __shared__ float part[16][kWarps];
  const bool norm = p.norm_w != nullptr;
  // One row (M == 1, K <= 4096) and a slice that starts on a multiple of 256 blocks: the thread that
  // holds block kb0 + b in the sum-of-squares pass (v = tid + j * 256) is the one that stages block b,
  // so it keeps x + residual in registers instead of reading them from L2 a second time. The pass
  // order is unchanged, so every CTA of the launch computes the same 1/rms.
  const bool keep = norm && p.M == 1 && p.K / 8 <= 2 * kThr && kb0 % kThr == 0;
  uint4 keep0 = make_uint4(0, 0, 0, 0), keep1 = make_uint4(0, 0, 0, 0);
  if (norm) {
    const int nv = p.K / 8;
    for (int m = 0; m < p.M; ++m) {
      float acc = 0.f;
      for (int v = tid; v < nv; v += kThr) {
        uint4 a = load_x8(p, m, 8 * v);
        if (p.res != nullptr) {
          const uint4 r = __ldcg(reinterpret_cast<const uint4*>(p.res + m * p.ldr) + v);
          __half2* ah = reinterpret_cast<__half2*>(&a);
          const __half2* rh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
          for (int j = 0; j < 4; ++j) ah[j] = __hadd2_rn(ah[j], rh[j]);
          if (writer) reinterpret_cast<uint4*>(p.res_out + m * p.ldro)[v] = a;
        }
        if (keep) {
          if (v < kThr)
            keep0 = a;
          else
            keep1 = a;
        }
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
    asm volatile("bar.sync 1, %0;" ::"r"(kThr) : "memory");
    if (tid < p.M) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) tot += part[tid][w];
      inv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(p.K)), p.eps)));
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kThr) : "memory");
  }
  // One item = 8 K values of one row. nblk is a multiple of 32, so every warp iteration has 32 items
  // in range and the 16 lanes of a half-warp hold the 16 blocks of one 128-group: the factored path
  // reduces its {C, X} with shuffles in a fixed order (deterministic) - no second pass.
  // The loads of kBatch iterations are issued before any of them is stored (16 rows of a 1536-wide K
  // slice are 12 iterations per thread: one L2 round trip per kBatch iterations instead of one per
  // iteration). Item i still goes to the thread it went to one iteration at a time.
  const int items = p.M * nblk;
  for (int base0 = (tid & ~31); base0 < items; base0 += kBatch * kThr) {
    uint4 vb[kBatch], rb[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      vb[u] = rb[u] = make_uint4(0, 0, 0, 0);
      const int i = base0 + u * kThr + (tid & 31);
      if (base0 + u * kThr >= items) continue;  // warp-uniform: items is a multiple of 32
      const int m = i / nblk, b = i % nblk;
      const int k = (kb0 + b) * 8;
      if (k >= p.K) continue;
      if (keep)  // this thread read block kb0 + b (= tid + j * 256) in the pass above
        vb[u] = (kb0 + b) < kThr ? keep0 : keep1;
      else
        vb[u] = load_x8(p, m, k);
      if (norm && p.res != nullptr && !keep) rb[u] = __ldcg(reinterpret_cast<const uint4*>(p.res + m * p.ldr + k));
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int base = base0 + u * kThr;
      if (base >= items) break;  // warp-uniform
      const int i = base + (tid & 31);
      const int m = i / nblk, b = i % nblk;
      const int k = (kb0 + b) * 8;
      uint4 v = vb[u];
      if (k < p.K) {
        if (norm) {
          __half2* vh = reinterpret_cast<__half2*>(&v);
          if (p.res != nullptr && !keep) {
            const __half2* rh = reinterpret_cast<const __half2*>(&rb[u]);
#pragma unroll
            for (int j = 0; j < 4; ++j) vh[j] = __hadd2_rn(vh[j], rh[j]);
          }
          // one row: block b of the slice is this thread's block tid + j * kThr (prefetched above)
          const uint4 wv = (p.M == 1 && b < 2 * kThr) ? (b < kThr ? nwp.w[0] : nwp.w[1])
                                                      : __ldg(reinterpret_cast<const uint4*>(p.norm_w + k));
          const __half2* wh = reinterpret_cast<const __half2*>(&wv);
          const float s = inv[m];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(vh[j]);
            vh[j] = __hmul2_rn(wh[j], __floats2half2_rn(__fmul_rn(f.x, s), __fmul_rn(f.y, s)));
          }
        }
      }
      uint4 o;
      o.x = prmt(v.x, v.z, 0x5410);  // (x0, x4)
      o.y = prmt(v.x, v.z, 0x7632);  // (x1, x5)
      o.z = prmt(v.y, v.w, 0x5410);  // (x2, x6)
      o.w = prmt(v.y, v.w, 0x7632);  // (x3, x7)
      if (factored) {  // odd K meets 1024 + 16 q: stage x / 16 (exact, a power of two)
        o.y = hmul2_rn(o.y, 0x2C002C00u);
        o.w = hmul2_rn(o.w, 0x2C002C00u);
        // {C, X} of this 128-group and row: C = 1024 * sum of the staged values, X = the sum of the x
        // each weight is multiplied by (odd K: 16 * staged)
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
        if ((tid & 15) == 0) {
          float* dst = cx + 2 * ((b >> 4) * 16 + m);  // [group in slice][16 rows]{C, X}
          dst[0] = 1024.f * C;
          dst[1] = X;
        }
      }
      *reinterpret_cast<uint4*>(xs + m * p.xs_pitch + b * 16) = o;
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kThr) : "memory");
}

// CW chunks (32 columns each) per tile; kWarps / CW warps per chunk split the tile's stages
// round-robin and meet in shared memory at the end of the tile.
template <int NT, int CW, bool EXACT>
__global__ void __launch_bounds__((kWarps + 1) * 32, 3 - NT)  // M <= 8: two CTAs per SM
    w4a16_gemv_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap ms,
                      const __grid_constant__ CUtensorMap mz, const GemvParams p) {
  constexpr int WPC = kWarps / CW;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base, derived from smem_raw by pointer arithmetic so accesses stay shared-space
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int S = gridDim.y;
  const SmemLayout L = smem_layout(CW, p.nbuf, p.M, p.xs_pitch, S);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + p.nbuf;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = blockIdx.y;  // cluster dims (1, S, 1)
  __shared__ unsigned long long s_ep;  // fused allreduce: this launch's epoch
  const int s_begin = rank * p.split_stages;
  const int s_end = min(s_begin + p.split_stages, p.stages_total);
  const int nst = max(0, s_end - s_begin);
  // Work units: 32-column chunks, or (fused SwiGLU) pairs of a gate chunk and its up chunk. A tile
  // holds UPT units in CW box slots; with SwiGLU slot s is the gate (s < UPT) or up (s >= UPT)
  // chunk of unit tile + s % UPT.
  const bool swiglu = p.swiglu_i > 0;
  const int UPT = swiglu ? CW / 2 : CW;
  int c_begin, c_end;  // this CTA's unit range
  if (S == 1) {
    c_begin = static_cast<int>((static_cast<int64_t>(blockIdx.x) * p.chunks) / gridDim.x);
    c_end = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * p.chunks) / gridDim.x);
  } else {
    c_begin = blockIdx.x * UPT;
    c_end = min(c_begin + UPT, p.chunks);
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nbuf; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  bool ok = true;
  if (warp == kWarps) {
    // ---------------------------------------------------------------- producer warp
    if (p.pf.n) l2_prefetch_share(p.pf, blockIdx.x + gridDim.x * blockIdx.y, gridDim.x * gridDim.y, lane);
    if (!p.static_weights) pdl_wait();
    if (lane == 0) {
      prefetch_tensormap(&mq);
      prefetch_tensormap(&ms);
      prefetch_tensormap(&mz);
      int it = 0;
      for (int tile = c_begin; tile < c_end && ok; tile += UPT) {
        const int nch = min(UPT, c_end - tile);
        for (int s = s_begin; s < s_end; ++s, ++it) {
          const int round = static_cast<int>(__umulhi(static_cast<uint32_t>(it), p.nbuf_rcp));
          const int buf = it - round * p.nbuf;
          if (it >= p.nbuf && !mbar_wait(&empty[buf], (round - 1) & 1, p.err, DK_DEVERR_WAIT_EMPTY)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[buf], (swiglu ? 2 : 1) * nch * kChunkStageBytes);
          for (int c = 0; c < CW; ++c) {
            if (c % UPT >= nch) continue;
            const int col = (tile + c % UPT) * 32 + (c >= UPT ? p.swiglu_i : 0);
            tma_load_2d(smem + L.w_off + (buf * CW + c) * kBoxBytes, &mq, col, s * kStageRows, &full[buf]);
            uint8_t* sz = smem + L.sz_off + (buf * CW + c) * 2 * kSZBytes;
            tma_load_2d(sz, &ms, col, s * kGroupsPerStage, &full[buf]);
            tma_load_2d(sz + kSZBytes, &mz, col, s * kGroupsPerStage, &full[buf]);
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- consumer warps
    const NormW nwp = norm_w_prefetch(p, s_begin);
    if (p.bias != nullptr) {  // this CTA's bias columns into L2 while the previous kernel finishes
      const int n_lo = c_begin * 32, n_hi = min(c_end * 32, swiglu ? p.swiglu_i : p.N);
      for (int n = n_lo + 64 * static_cast<int>(threadIdx.x); n < n_hi; n += 64 * kWarps * 32) {
        prefetch_l2(p.bias + n);
        if (swiglu) prefetch_l2(p.bias + p.swiglu_i + n);
      }
    }
    pdl_wait();  // x (and the residual) come from the previous kernels
    if (p.tp.world > 0 && threadIdx.x == 0) s_ep = *reinterpret_cast<volatile unsigned long long*>(p.tp.epoch) + 1;
    stage_x<NT == 1 ? 1 : 4>(p, smem + L.xs_off, reinterpret_cast<float*>(smem + L.cx_off), s_begin, nst,
            blockIdx.x == 0 && blockIdx.y == 0, !EXACT, nwp);  // ends with a barrier
    const unsigned long long ep = s_ep;
    const int g = lane >> 2;  // MMA group: A rows g, g+8 ; B column g
    const int t = lane & 3;   // thread in group: K slots 2t.., 2t+8..
    const int slot = warp % CW;  // chunk of the tile this warp works on
    const int phase = warp / CW;  // which of the tile's stages (round-robin over WPC warps)
    float* red = reinterpret_cast<float*>(smem + L.red_off);
    int tile_idx = 0;
    for (int tile = c_begin; tile < c_end; tile += UPT, ++tile_idx) {
      const int nch = min(UPT, c_end - tile);
      const bool active = slot % UPT < nch;
      float acc[2][NT][4];
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

      for (int ls = phase; ls < nst && ok; ls += WPC) {
        const int it = tile_idx * nst + ls;
        const int round = static_cast<int>(__umulhi(static_cast<uint32_t>(it), p.nbuf_rcp));
        const int buf = it - round * p.nbuf;
        if (!mbar_wait(&full[buf], round & 1, p.err, DK_DEVERR_WAIT_FULL)) {
          ok = false;
          break;
        }
        if (active) {
          if constexpr (EXACT)
            consume_chunk_stage<NT, true>(smem + L.w_off + (buf * CW + slot) * kBoxBytes,
                                          smem + L.sz_off + (buf * CW + slot) * 2 * kSZBytes,
                                          smem + L.xs_off + ls * kStageRows * 16, p.xs_pitch, p.M, g, t, acc);
          else
            consume_chunk_stage_f<NT>(smem_addr(smem + L.w_off + (buf * CW + slot) * kBoxBytes),
                                      smem_addr(smem + L.sz_off + (buf * CW + slot) * 2 * kSZBytes),
                                      smem_addr(smem + L.xs_off + ls * kStageRows * 16),
                                      smem_addr(smem + L.cx_off + ls * kGroupsPerStage * 128), p.xs_pitch, p.M, g, t,
                                      acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
      }

      // ---------------------------------------------------------------- tile epilogue
      if (WPC == 1 && S == 1 && !swiglu && p.yp == nullptr) {
        if (active && ok) {
          const int n0 = (tile + slot) * 32 + 4 * g;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int m = nt * 8 + 2 * t + e;
              if (m >= p.M) continue;
              float v[4] = {acc[0][nt][e], acc[0][nt][2 + e], acc[1][nt][e], acc[1][nt][2 + e]};
              if (p.tp.world > 0) {  // N % 8 == 0: the 4 columns are all inside or all outside
                if (n0 < p.N) tp_push4(p.tp, ep, m, n0, make_float4(v[0], v[1], v[2], v[3]));
                continue;
              }
#pragma unroll
              for (int c = 0; c < 4; ++c)
                if (n0 + c < p.N) {
                  if (p.bias != nullptr) v[c] += __half2float(p.bias[n0 + c]);
                  p.y[m * p.ldy + n0 + c] = __float2half_rn(v[c]);
                }
            }
        }
      } else {
        // partial sums of the WPC warps of each chunk meet in shared memory: red[phase][m][col]
        if (active) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int m = nt * 8 + 2 * t + e;
              if (m >= p.M) continue;
              float* row = red + (phase * p.M + m) * CW * 32 + slot * 32 + 4 * g;
              row[0] = acc[0][nt][e];
              row[1] = acc[0][nt][2 + e];
              row[2] = acc[1][nt][e];
              row[3] = acc[1][nt][2 + e];
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kWarps * 32) : "memory");
        const int ncols = nch * 32;
        const int nhalves = swiglu ? 2 : 1;
        for (int e = threadIdx.x; e < p.M * ncols; e += kWarps * 32) {
          const int m = e / ncols, col = e % ncols;
          float v[2];
          for (int hh = 0; hh < nhalves; ++hh) {
            const int rc = hh * UPT * 32 + col;  // column of slot (gate or up) in red
            float a = red[m * CW * 32 + rc];
#pragma unroll
            for (int j = 1; j < WPC; ++j) a += red[(j * p.M + m) * CW * 32 + rc];
            v[hh] = a;
          }
          if (p.yp != nullptr) {  // this K slice's partial sums (no bias), read by the next kernel
            const int n = tile * 32 + col;
            if (n < p.N) p.yp[(static_cast<int64_t>(rank) * p.M + m) * p.N + n] = v[0];
          } else if (S == 1) {
            const int n = tile * 32 + col;
            if (!swiglu && n < p.N) {
              float a = v[0];
              if (p.tp.world > 0) {
                tp_push(p.tp, ep, m, n, a);
                continue;
              }
              if (p.bias != nullptr) a += __half2float(p.bias[n]);
              p.y[m * p.ldy + n] = __float2half_rn(a);
            } else if (swiglu && n < p.swiglu_i) {
              p.y[m * p.ldy + n] = swiglu_out(v[0], v[1], p.bias, n, p.swiglu_i);
            }
          } else {
            for (int hh = 0; hh < nhalves; ++hh)  // this rank's partial, read by the cluster below
              red[m * CW * 32 + hh * UPT * 32 + col] = v[hh];
          }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kWarps * 32) : "memory");
      }
    }
  }

  // ------------------------------------------------------------------ split-K reduction / exit
  if (__syncthreads_or(!ok)) {
    if (warp == kWarps && lane == 0) {
      // wait (bounded) for the copies still in flight before the shared memory goes away
      const uint64_t t0 = globaltimer_ns();
      for (int b = 0; b < p.nbuf; ++b)
        while (!mbar_try_wait(&full[b], 0) && !mbar_try_wait(&full[b], 1) &&
               globaltimer_ns() - t0 < 500000000ull) {
        }
    }
    if (S > 1 && p.yp == nullptr) {
      cluster_sync();
      cluster_sync();
    }
    if (p.tp.world > 0) tp_finish(p, s_ep, false, c_begin, c_end, UPT, S, rank);
    return;
  }
  if (S > 1 && p.yp == nullptr) {
    cluster_sync();
    const float* red = reinterpret_cast<const float*>(smem + L.red_off);
    const int ncols = min(UPT, c_end - c_begin) * 32;
    for (int e = threadIdx.x; e < p.M * ncols; e += blockDim.x) {
      if (e % S != rank) continue;
      const int m = e / ncols, col = e % ncols;
      const int n = c_begin * 32 + col;
      if (n >= (swiglu ? p.swiglu_i : p.N)) continue;
      float v[2] = {0.f, 0.f};
      for (int hh = 0; hh < (swiglu ? 2 : 1); ++hh) {
        const float* src = red + m * CW * 32 + hh * UPT * 32 + col;
        for (int q = 0; q < S; ++q) v[hh] += ld_shared_cluster_f32(map_shared_rank(src, q));
      }
      if (swiglu) {
        p.y[m * p.ldy + n] = swiglu_out(v[0], v[1], p.bias, n, p.swiglu_i);
      } else if (p.tp.world > 0) {
        tp_push(p.tp, s_ep, m, n, v[0]);
      } else {
        if (p.bias != nullptr) v[0] += __half2float(p.bias[n]);
        p.y[m * p.ldy + n] = __float2half_rn(v[0]);
      }
    }
    cluster_sync();  // keep this CTA's partial sums alive until every rank has read them
  }
  if (p.tp.world > 0) tp_finish(p, s_ep, true, c_begin, c_end, UPT, S, rank);
}

// Any-alignment fallback: one thread per (row, column), plain loads, the reference's fp16 weight
// rounding and an fp32 sum in K order (kernels/w4a16.py:134-152 without the tiling). Used for
// N % 8 != 0, group sizes other than 128, unaligned pointers or strides.
__global__ void w4a16_generic_kernel(const __half* __restrict__ x, int64_t ldx,
                                     const int32_t* __restrict__ qw, const __half* __restrict__ scales,
                                     const __half* __restrict__ zeros, const __half* __restrict__ bias,
                                     __half* __restrict__ y, int64_t ldy, int M, int N, int K, int group) {
  pdl_wait();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 8) {
    const uint32_t w = static_cast<uint32_t>(qw[static_cast<int64_t>(k0 / 8) * N + n]);
    const int g = k0 / group;
    const __half s = scales[static_cast<int64_t>(g) * N + n];
    const __half z = zeros[static_cast<int64_t>(g) * N + n];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __half q = __int2half_rn(static_cast<int>((w >> (4 * i)) & 0xF));
      const __half wv = __hmul_rn(__hsub_rn(q, z), s);
      acc = fmaf(__half2float(x[m * ldx + k0 + i]), __half2float(wv), acc);
    }
  }
  if (bias != nullptr) acc += __half2float(bias[n]);
  y[m * ldy + n] = __float2half_rn(acc);
}

using GemvKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const GemvParams);

// All compiled variants: [NT-1][log2(CW)][EXACT].
GemvKernel variant(int nt, int cw, bool exact) {
  static const GemvKernel table[2][4][2] = {
      {{w4a16_gemv_kernel<1, 1, false>, w4a16_gemv_kernel<1, 1, true>},
       {w4a16_gemv_kernel<1, 2, false>, w4a16_gemv_kernel<1, 2, true>},
       {w4a16_gemv_kernel<1, 4, false>, w4a16_gemv_kernel<1, 4, true>},
       {w4a16_gemv_kernel<1, 8, false>, w4a16_gemv_kernel<1, 8, true>}},
      {{w4a16_gemv_kernel<2, 1, false>, w4a16_gemv_kernel<2, 1, true>},
       {w4a16_gemv_kernel<2, 2, false>, w4a16_gemv_kernel<2, 2, true>},
       {w4a16_gemv_kernel<2, 4, false>, w4a16_gemv_kernel<2, 4, true>},
       {w4a16_gemv_kernel<2, 8, false>, w4a16_gemv_kernel<2, 8, true>}}};
  const int lg = cw == 1 ? 0 : cw == 2 ? 1 : cw == 4 ? 2 : 3;
  return table[nt - 1][lg][exact ? 1 : 0];
}

// Opt every variant in to the device's shared-memory limit (once per device).
void set_smem_attrs() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && !done[dev]) {
    for (int nt = 1; nt <= 2; ++nt)
      for (int cw = 1; cw <= 8; cw *= 2)
        for (int ex = 0; ex < 2; ++ex)
          opt_in_dynamic_smem(variant(nt, cw, ex));
    done[dev] = true;
  }
}

// Resident CTAs per SM of one variant at a given dynamic shared memory size (registers, threads
// and shared memory all counted by the runtime's occupancy calculator); memoized.
int occupancy(int nt, int cw, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, nt * 16 + cw, smem);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  set_smem_attrs();
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, variant(nt, cw, false), (kWarps + 1) * 32, smem) !=
      cudaSuccess) {
    cudaGetLastError();
    n = 1;
  }
  n = std::max(n, 1);
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

struct Choice {
  int cw, split, nbuf, nctas;
  size_t smem;  // dynamic bytes including the alignment slack
  double cost;
};

constexpr size_t kSmemBudget = 110 * 1024;  // two CTAs per SM fit
constexpr size_t kXsBudget = 64 * 1024;

int xs_pitch_for(int split_stages) { return split_stages * kStageRows * 16 + kXsPad; }

// Cost model (microseconds) for one launch: a fixed launch/fill latency, then the slowest of the
// busiest SM's HBM share, its instruction throughput, and one warp's serial chain of
// chunk-stages; plus the cluster and in-CTA reductions. `units` are 32-column chunks (or
// gate/up chunk pairs, bpu = 2 boxes per unit), `upt` units per tile.
double model_cost(const DeviceInfo& dev, int units, int bpu, int sps, int cw, int upt, int split, int nctas) {
  const int wpc = kWarps / cw;
  const double units_per_cta = std::ceil(static_cast<double>(units) / nctas);
  const double tiles_per_cta = std::ceil(units_per_cta / upt);
  const double ctas_per_sm = std::ceil(static_cast<double>(nctas) * split / dev.num_sms);
  const double cs_sm = ctas_per_sm * units_per_cta * bpu * sps;
  const double t_mem = cs_sm * kChunkStageBytes / (6.4e12 / dev.num_sms) * 1e6;
  const double t_issue = cs_sm / 10.0;
  const double t_chain = tiles_per_cta * std::ceil(static_cast<double>(sps) / wpc) * 0.5;
  return 2.0 + std::max(t_mem, std::max(t_issue, t_chain)) + (split > 1 ? 0.5 : 0.0) +
         (wpc > 1 ? 0.2 * tiles_per_cta : 0.0);
}

Choice choose_uncached(int M, int units, int K, bool swiglu, const dk_matmul_config* cfg) {
  const DeviceInfo& dev = device_info();
  const int stages_total = (K + 256 - 1) / 256;
  const int nt = M <= 8 ? 1 : 2;
  // M > 8 variants hold one CTA per SM (registers), so their ring may use the SM's whole shared memory
  const size_t budget = nt == 1 ? kSmemBudget : 2 * kSmemBudget;
  Choice best = {0, 0, 0, 0, 0, 1e300};
  // requested split: clamped to what K allows (every rank needs at least one 256-wide stage)
  int want_split = (cfg && cfg->split_k > 0) ? std::min(cfg->split_k, std::min(8, stages_total)) : 0;
  while (want_split > 1 && (want_split - 1) * ((stages_total + want_split - 1) / want_split) >= stages_total)
    --want_split;
  const int want_bn = (cfg && (cfg->block_n == 32 || cfg->block_n == 64 || cfg->block_n == 128 ||
                               cfg->block_n == 256)) ? cfg->block_n : 0;
  for (int cw = 8; cw >= 1; cw /= 2) {
    if (want_bn && want_bn != 32 * cw) continue;
    if (swiglu && cw < 2) continue;
    const int upt = swiglu ? cw / 2 : cw;
    for (int split = 1; split <= 8; ++split) {
      if (want_split && want_split != split) continue;
      if (split > stages_total) break;
      const int sps = (stages_total + split - 1) / split;
      if ((split - 1) * sps >= stages_total) continue;  // every rank gets at least one stage
      const int pitch = xs_pitch_for(sps);
      if (static_cast<size_t>(M) * pitch > kXsBudget) continue;
      const int tiles = (units + upt - 1) / upt;
      const int stages_per_cta = sps * (split > 1 ? 1 : (tiles + dev.num_sms - 1) / dev.num_sms);
      int nbuf = std::min(std::max(stages_per_cta, 2), 16);
      SmemLayout L = smem_layout(cw, nbuf, M, pitch, split);
      while (nbuf > 2 && static_cast<size_t>(L.total) + 1024 > budget) {
        --nbuf;
        L = smem_layout(cw, nbuf, M, pitch, split);
      }
      const size_t smem = static_cast<size_t>(L.total) + 1024;
      if (smem > static_cast<size_t>(dev.max_smem_optin)) continue;
      // Ring depth: a consumer warp's next stage is kWarps / cw stages after its previous one (and
      // its first stage of a tile at most that far after a stage the whole CTA has consumed), so
      // once buffers are reused the ring must hold at least that many stages; a shallower ring
      // would let a full-barrier parity wait pass on the buffer's previous phase. (Only very long
      // K slices with narrow tiles reach this: x's staging then leaves little shared memory.)
      if (nbuf < std::min(kWarps / cw, stages_per_cta)) continue;
      const int occ = occupancy(nt, cw, smem);
      const int nctas = split == 1 ? std::min(units, dev.num_sms * occ) : tiles;
      if (split > 1 && static_cast<long>(nctas) * split > static_cast<long>(dev.num_sms) * occ) continue;
      const double cost = model_cost(dev, units, swiglu ? 2 : 1, sps, cw, upt, split, nctas);
      if (cost < best.cost) best = {cw, split, nbuf, nctas, smem, cost};
    }
  }
  return best;
}

// Memoized per (device, M, units, K, mode, requested split, requested tile): the choice is a pure
// function of these, and computing it queries the occupancy calculator.
Choice choose(int M, int units, int K, bool swiglu, const dk_matmul_config* cfg) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int, int>, Choice> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, M, units, K, swiglu ? 1 : 0, cfg ? cfg->split_k : 0, cfg ? cfg->block_n : 0);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  Choice c = choose_uncached(M, units, K, swiglu, cfg);
  if (c.cw == 0 && cfg) {  // the requested split / tile does not fit: let the model choose
    dk_matmul_config auto_cfg = *cfg;
    auto_cfg.split_k = 0;
    auto_cfg.block_n = 0;
    c = choose_uncached(M, units, K, swiglu, &auto_cfg);
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = c;
  return c;
}

int launch_gemv(const CUtensorMap& mq, const CUtensorMap& ms, const CUtensorMap& mz, const GemvParams& p,
                const Choice& c, bool exact, cudaStream_t stream) {
  set_smem_attrs();
  const GemvKernel kernel = variant(p.M <= 8 ? 1 : 2, c.cw, exact);
  const dim3 grid(c.nctas, c.split, 1);
  const dim3 block((kWarps + 1) * 32, 1, 1);
  // split-K partials written to global memory need no cluster: the slices run as independent CTAs
  const dim3 cluster(1, p.yp != nullptr ? 1 : c.split, 1);
  cudaError_t e = launch(kernel, grid, block, c.smem, stream, pdl_enabled(), cluster, mq, ms, mz, p);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w4a16 gemv launch: %s", cudaGetErrorString(e));
  return DK_OK;
}

// Shared host path of dk_w4a16_matmul (swiglu_i == 0) and dk_w4a16_swiglu (swiglu_i == I, N == 2I).
struct NormArgs {
  const void* w = nullptr;  // RMSNorm weight [K]; nullptr = no fused norm
  const void* res = nullptr;
  int64_t ldr = 0;
  void* res_out = nullptr;
  int64_t ldro = 0;
  float eps = 1e-6f;
};

// Split-K partial sums between two launches (dk_w4a16_matmul_partials and its consumer
// dk_w4a16_rmsnorm_matmul_partials): one launch of at most 16 rows each.
struct PartialIO {
  const float* xp = nullptr;  // consumer: the previous projection's partial sums [xparts][M][K]
  int xparts = 0;
  const __half* xbias = nullptr;
  float* yp = nullptr;        // producer: this projection's partial sums [split][M][N]
  int64_t yp_capacity = 0;    // floats
  int* nparts = nullptr;      // producer: receives the split (the number of partial sums written)
};

int run_fast(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* zeros,
             const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group_size,
             const dk_matmul_config* cfg, int swiglu_i, const NormArgs& na, cudaStream_t st,
             const TPArgs* tp = nullptr, const PartialIO* pio = nullptr) {
  const int flags = cfg ? cfg->flags : 0;
  CUtensorMap mq, ms, mz;
  if (!make_tensor_map_2d(&mq, qweight, CU_TENSOR_MAP_DATA_TYPE_INT32, N, K / 8, N * 4, 32, kStageRows,
                          CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&ms, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K / group_size, N * 2, 32,
                          kGroupsPerStage, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tensor_map_2d(&mz, zeros, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K / group_size, N * 2, 32,
                          kGroupsPerStage, CU_TENSOR_MAP_SWIZZLE_NONE))
    return DK_ERR_CUDA;
  const DeviceInfo& dev = device_info();
  const int units = swiglu_i > 0 ? (swiglu_i + 31) / 32 : static_cast<int>((N + 31) / 32);
  const int64_t rows_per_launch = tp != nullptr ? std::min<int64_t>(16, tp->max_m) : 16;
  for (int64_t m0 = 0; m0 < M;) {
    int mc = static_cast<int>(std::min<int64_t>(rows_per_launch, M - m0));
    Choice c = choose(mc, units, static_cast<int>(K), swiglu_i > 0, cfg);
    // The staged x grows with the rows: when a long K slice leaves no tile for mc rows, launch fewer
    // rows at a time. (Not with the fused allreduce over several ranks: every rank must make the same
    // launches, and the ranks' K shards may differ. A one-rank launch meets nobody, and each launch
    // takes its own epoch, so it may halve like the plain path.)
    while ((tp == nullptr || tp->world == 1) && c.cw == 0 && mc > 1) {
      mc = (mc + 1) / 2;
      c = choose(mc, units, static_cast<int>(K), swiglu_i > 0, cfg);
    }
    if (c.cw == 0) return set_error(DK_ERR_UNSUPPORTED, "w4a16: no tile fits (M=%d, K=%lld)", mc, (long long)K);
    if (tp != nullptr && mc > tp->max_m)
      return set_error(DK_ERR_UNSUPPORTED, "w4a16_matmul_allreduce: %d rows exceed the communicator", mc);
    if (pio != nullptr && mc != M)
      return set_error(DK_ERR_UNSUPPORTED, "w4a16 partial sums: %lld rows do not fit one launch", (long long)M);
    if (pio != nullptr && pio->yp != nullptr) {
      if (static_cast<int64_t>(c.split) * M * N > pio->yp_capacity)
        return set_error(DK_ERR_INVALID, "w4a16_matmul_partials: %d partial sums of [%lld, %lld] exceed the buffer",
                         c.split, (long long)M, (long long)N);
      *pio->nparts = c.split;
    }
    GemvParams p;
    p.x = static_cast<const __half*>(x) + m0 * ldx;
    p.ldx = ldx;
    p.bias = static_cast<const __half*>(bias);
    p.y = static_cast<__half*>(y) + m0 * ldy;
    p.ldy = ldy;
    p.M = mc;
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.stages_total = static_cast<int>((K + 255) / 256);
    p.split_stages = (p.stages_total + c.split - 1) / c.split;
    p.chunks = units;
    p.nbuf = c.nbuf;
    p.nbuf_rcp = static_cast<uint32_t>((0x100000000ull + c.nbuf - 1) / c.nbuf);
    p.xs_pitch = xs_pitch_for(p.split_stages);
    p.static_weights = (flags & DK_FLAG_STATIC_WEIGHTS) ? 1 : 0;
    p.swiglu_i = swiglu_i;
    p.norm_w = static_cast<const __half*>(na.w);
    p.res = na.res ? static_cast<const __half*>(na.res) + m0 * na.ldr : nullptr;
    p.ldr = na.ldr;
    p.res_out = na.res_out ? static_cast<__half*>(na.res_out) + m0 * na.ldro : nullptr;
    p.ldro = na.ldro;
    p.eps = na.eps;
    p.err = dev.err_word;
    p.pf = l2_prefetch_from(m0 == 0 ? cfg : nullptr);
    p.xp = pio != nullptr ? pio->xp : nullptr;
    p.xparts = pio != nullptr ? pio->xparts : 0;
    p.xbias = pio != nullptr ? pio->xbias : nullptr;
    p.yp = pio != nullptr ? pio->yp : nullptr;
    if (tp != nullptr)
      p.tp = *tp;
    else
      std::memset(&p.tp, 0, sizeof(p.tp));
    const int rc = launch_gemv(mq, ms, mz, p, c, (flags & DK_FLAG_EXACT_DEQUANT) != 0, st);
    if (rc != DK_OK) return rc;
    m0 += mc;
  }
  return DK_OK;
}

int check_w4a16_args(const char* what, const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                     const void* zeros, const void* y, int64_t ldy, int64_t M, int64_t N, int64_t ycols,
                     int64_t K, int64_t group_size) {
  if (M < 0 || N < 0 || K < 0) return set_error(DK_ERR_INVALID, "%s: negative size", what);
  if (group_size <= 0 || group_size % 8 != 0 || K % group_size != 0)
    return set_error(DK_ERR_INVALID, "%s: need K %% group_size == 0 and group_size %% 8 == 0 (K=%lld, group_size=%lld)",
                     what, (long long)K, (long long)group_size);
  if (ldx < K || ldy < ycols) return set_error(DK_ERR_INVALID, "%s: row stride smaller than the row", what);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || (K / 8) * N > (int64_t(1) << 40))
    return set_error(DK_ERR_INVALID, "%s: size out of range", what);
  if (M > 0 && N > 0 && (!x || !qweight || !scales || !zeros || !y))
    return set_error(DK_ERR_INVALID, "%s: NULL pointer", what);
  return DK_OK;
}

bool fast_ok(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* zeros, int64_t N,
             int64_t K, int64_t group_size, int flags) {
  return !(flags & DK_FLAG_GENERIC) && N % 8 == 0 && group_size == 128 && K > 0 && aligned16(x) && ldx % 8 == 0 &&
         aligned16(qweight) && aligned16(scales) && aligned16(zeros);
}

}  // namespace
}  // namespace dk

namespace dk {
bool gemm_tc_ok(const void* x, int64_t ldx, const void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                int64_t group_size);
int launch_gemm_tc(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* zeros,
                   const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, cudaStream_t st);
void skinny_choice(int64_t rows, int64_t N, int64_t K, int* mb_out, int* split_out);
int launch_skinny_tc(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* zeros,
                     const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, bool static_weights,
                     cudaStream_t st,
                     const TPArgs* tp = nullptr);
}  // namespace dk

extern "C" int dk_w4a16_matmul(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                               const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M,
                               int64_t N, int64_t K, int64_t group_size, const dk_matmul_config* cfg,
                               dk_stream_t stream) {
  using namespace dk;
  int rc = check_w4a16_args("w4a16_matmul", x, ldx, qweight, scales, zeros, y, ldy, M, N, N, K, group_size);
  if (rc != DK_OK) return rc;
  if (M == 0 || N == 0) return DK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int flags = cfg ? cfg->flags : 0;
  if (!fast_ok(x, ldx, qweight, scales, zeros, N, K, group_size, flags)) {
    const dim3 grid(static_cast<unsigned>((N + 127) / 128), static_cast<unsigned>(M), 1);
    cudaError_t e = launch(w4a16_generic_kernel, grid, dim3(128, 1, 1), 0, st, pdl_enabled(), dim3(1, 1, 1),
                           static_cast<const __half*>(x), ldx, qweight, static_cast<const __half*>(scales),
                           static_cast<const __half*>(zeros), static_cast<const __half*>(bias),
                           static_cast<__half*>(y), ldy, static_cast<int>(M), static_cast<int>(N),
                           static_cast<int>(K), static_cast<int>(group_size));
    if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w4a16 generic launch: %s", cudaGetErrorString(e));
    return DK_OK;
  }
  if (!(flags & DK_FLAG_GEMV) && gemm_tc_ok(x, ldx, y, ldy, M, N, K, group_size))
    return launch_gemm_tc(x, ldx, qweight, scales, zeros, bias, y, ldy, M, N, K, st);
  // batched decode: tcgen05 swap-AB for 16 < M < 128; at 9-16 rows with K < 4096 the decode GEMV
  // measured faster (qkv, o_proj shapes), at K >= 4096 the tcgen05 kernel is much faster (down at 12
  // rows: 14 us against 22 us for the GEMV, which walks the long K with 16-row MMA tiles)
  if (!(flags & DK_FLAG_GEMV) && M > 8 && N >= 128 && (M > 16 || K >= 4096)) {
    int mb = 0, split = 0;
    skinny_choice(M, N, K, &mb, &split);
    if (mb != 0)
      return launch_skinny_tc(x, ldx, qweight, scales, zeros, bias, y, ldy, M, N, K,
                              (flags & DK_FLAG_STATIC_WEIGHTS) != 0, st);
  }
  return run_fast(x, ldx, qweight, scales, zeros, bias, y, ldy, M, N, K, group_size, cfg, 0, NormArgs(), st);
}

extern "C" int dk_w4a16_swiglu(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                               const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M,
                               int64_t I, int64_t K, int64_t group_size, const dk_matmul_config* cfg,
                               dk_stream_t stream) {
  using namespace dk;
  int rc = check_w4a16_args("w4a16_swiglu", x, ldx, qweight, scales, zeros, y, ldy, M, 2 * I, I, K, group_size);
  if (rc != DK_OK) return rc;
  if (M == 0 || I == 0) return DK_OK;
  const int flags = cfg ? cfg->flags : 0;
  if (I % 32 != 0 || !fast_ok(x, ldx, qweight, scales, zeros, 2 * I, K, group_size, flags))
    return set_error(DK_ERR_UNSUPPORTED,
                     "w4a16_swiglu: the fused kernel needs I %% 32 == 0, group_size 128 and 16-byte aligned operands");
  return run_fast(x, ldx, qweight, scales, zeros, bias, y, ldy, M, 2 * I, K, group_size, cfg, static_cast<int>(I),
                  NormArgs(), reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dk_w4a16_rmsnorm_matmul(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                                       const void* norm_weight, float eps, void* residual_out, int64_t ldro,
                                       const int32_t* qweight, const void* scales, const void* zeros,
                                       const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                                       int64_t group_size, int32_t swiglu, const dk_matmul_config* cfg,
                                       dk_stream_t stream) {
  using namespace dk;
  const int64_t ycols = swiglu ? N / 2 : N;
  int rc = check_w4a16_args("w4a16_rmsnorm_matmul", x, ldx, qweight, scales, zeros, y, ldy, M, N, ycols, K, group_size);
  if (rc != DK_OK) return rc;
  if (M == 0 || N == 0) return DK_OK;
  if (!norm_weight) return set_error(DK_ERR_INVALID, "w4a16_rmsnorm_matmul: norm_weight is NULL");
  if (residual && (!residual_out || ldr < K || ldro < K))
    return set_error(DK_ERR_INVALID, "w4a16_rmsnorm_matmul: residual needs residual_out and row strides >= K");
  const int flags = cfg ? cfg->flags : 0;
  const bool aligned = aligned16(norm_weight) && (!residual || (aligned16(residual) && aligned16(residual_out) &&
                                                                 ldr % 8 == 0 && ldro % 8 == 0));
  if (!aligned || K % 8 != 0 || (swiglu && (N % 2 != 0 || (N / 2) % 32 != 0)) ||
      !fast_ok(x, ldx, qweight, scales, zeros, N, K, group_size, flags))
    return set_error(DK_ERR_UNSUPPORTED,
                     "w4a16_rmsnorm_matmul: the fused kernel needs group_size 128, N %% 8 == 0 (I %% 32 == 0 with "
                     "swiglu) and 16-byte aligned operands and strides");
  NormArgs na;
  na.w = norm_weight;
  na.res = residual;
  na.ldr = ldr;
  na.res_out = residual_out;
  na.ldro = ldro;
  na.eps = eps;
  return run_fast(x, ldx, qweight, scales, zeros, bias, y, ldy, M, N, K, group_size, cfg,
                  swiglu ? static_cast<int>(N / 2) : 0, na, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dk_w4a16_matmul_partials(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                                        const void* zeros, int64_t M, int64_t N, int64_t K, int64_t group_size,
                                        float* partials, int64_t capacity, int32_t* nparts,
                                        const dk_matmul_config* cfg, dk_stream_t stream) {
  using namespace dk;
  int rc = check_w4a16_args("w4a16_matmul_partials", x, ldx, qweight, scales, zeros, partials, N, M, N, N, K,
                            group_size);
  if (rc != DK_OK) return rc;
  if (nparts == nullptr) return set_error(DK_ERR_INVALID, "w4a16_matmul_partials: nparts is NULL");
  if (M < 1 || M > 16) return set_error(DK_ERR_UNSUPPORTED, "w4a16_matmul_partials: 1..16 rows");
  const int flags = cfg ? cfg->flags : 0;
  if (!fast_ok(x, ldx, qweight, scales, zeros, N, K, group_size, flags) || !aligned16(partials))
    return set_error(DK_ERR_UNSUPPORTED,
                     "w4a16_matmul_partials: needs the fast path's conditions and a 16-byte aligned buffer");
  PartialIO pio;
  pio.yp = partials;
  pio.yp_capacity = capacity;
  pio.nparts = nparts;
  return run_fast(x, ldx, qweight, scales, zeros, nullptr, nullptr, N, M, N, K, group_size, cfg, 0, NormArgs(),
                  reinterpret_cast<cudaStream_t>(stream), nullptr, &pio);
}

extern "C" int dk_w4a16_rmsnorm_matmul_partials(const float* parts, int32_t nparts, const void* part_bias,
                                                const void* residual, int64_t ldr, const void* norm_weight, float eps,
                                                void* residual_out, int64_t ldro, const int32_t* qweight,
                                                const void* scales, const void* zeros, const void* bias, void* y,
                                                int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group_size,
                                                int32_t swiglu, const dk_matmul_config* cfg, dk_stream_t stream) {
  using namespace dk;
  const int64_t ycols = swiglu ? N / 2 : N;
  int rc = check_w4a16_args("w4a16_rmsnorm_matmul_partials", parts, K, qweight, scales, zeros, y, ldy, M, N, ycols, K,
                            group_size);
  if (rc != DK_OK) return rc;
  if (nparts < 1 || nparts > 8) return set_error(DK_ERR_INVALID, "w4a16_rmsnorm_matmul_partials: 1..8 partial sums");
  if (M < 1 || M > 16) return set_error(DK_ERR_UNSUPPORTED, "w4a16_rmsnorm_matmul_partials: 1..16 rows");
  if (!norm_weight) return set_error(DK_ERR_INVALID, "w4a16_rmsnorm_matmul_partials: norm_weight is NULL");
  if (residual && (!residual_out || ldr < K || ldro < K))
    return set_error(DK_ERR_INVALID, "w4a16_rmsnorm_matmul_partials: residual needs residual_out and row strides >= K");
  const int flags = cfg ? cfg->flags : 0;
  const bool aligned = aligned16(norm_weight) && (!part_bias || aligned16(part_bias)) &&
                       (!residual || (aligned16(residual) && aligned16(residual_out) && ldr % 8 == 0 && ldro % 8 == 0));
  if (!aligned || K % 8 != 0 || (swiglu && (N % 2 != 0 || (N / 2) % 32 != 0)) ||
      !fast_ok(parts, K, qweight, scales, zeros, N, K, group_size, flags))
    return set_error(DK_ERR_UNSUPPORTED,
                     "w4a16_rmsnorm_matmul_partials: needs group_size 128, N %% 8 == 0 (I %% 32 == 0 with swiglu) and "
                     "16-byte aligned operands and strides");
  NormArgs na;
  na.w = norm_weight;
  na.res = residual;
  na.ldr = ldr;
  na.res_out = residual_out;
  na.ldro = ldro;
  na.eps = eps;
  PartialIO pio;
  pio.xp = parts;
  pio.xparts = nparts;
  pio.xbias = static_cast<const __half*>(part_bias);
  return run_fast(parts, K, qweight, scales, zeros, bias, y, ldy, M, N, K, group_size, cfg,
                  swiglu ? static_cast<int>(N / 2) : 0, na, reinterpret_cast<cudaStream_t>(stream), nullptr, &pio);
}

namespace dk {
bool tp_args_from(const dk_tp_comm* c, TPArgs* a);
}

extern "C" int dk_w4a16_matmul_allreduce(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                                         const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M,
                                         int64_t N, int64_t K, int64_t group_size, const dk_matmul_config* cfg,
                                         const dk_tp_comm* comm, dk_stream_t stream) {
  using namespace dk;
  int rc = check_w4a16_args("w4a16_matmul_allreduce", x, ldx, qweight, scales, zeros, y, ldy, M, N, N, K, group_size);
  if (rc != DK_OK) return rc;
  TPArgs tp;
  if (!tp_args_from(comm, &tp)) return set_error(DK_ERR_INVALID, "w4a16_matmul_allreduce: comm is NULL");
  if (N > tp.max_n)
    return set_error(DK_ERR_INVALID, "w4a16_matmul_allreduce: N=%lld exceeds the communicator's max_n=%d",
                     (long long)N, tp.max_n);
  if (M == 0 || N == 0) return DK_OK;
  const int flags = cfg ? cfg->flags : 0;
  if (!fast_ok(x, ldx, qweight, scales, zeros, N, K, group_size, flags))
    return set_error(DK_ERR_UNSUPPORTED,
                     "w4a16_matmul_allreduce: needs group_size 128, N %% 8 == 0 and 16-byte aligned operands");
  // more than 16 rows (up to the communicator's max_m): the tcgen05 small-M kernel with the same
  // allreduce epilogue, all rows in one launch (one weight pass; the ranks' launches match because M
  // is the same on every rank and the kernel's row tile holds all of them)
  // (more rows than max_m, or DK_FLAG_GEMV: the decode GEMV in launches of up to min(16, max_m) rows)
  if (M > 16 && M <= tp.max_m && !(flags & DK_FLAG_GEMV)) {
    int mb = 0, split = 0;
    skinny_choice(M, N, K, &mb, &split);
    if (mb != 0 && M <= mb)
      return launch_skinny_tc(x, ldx, qweight, scales, zeros, bias, y, ldy, M, N, K,
                              (flags & DK_FLAG_STATIC_WEIGHTS) != 0, reinterpret_cast<cudaStream_t>(stream), &tp);
  }
  return run_fast(x, ldx, qweight, scales, zeros, bias, y, ldy, M, N, K, group_size, cfg, 0, NormArgs(),
                  reinterpret_cast<cudaStream_t>(stream), &tp);
}

// ---------------------------------------------------------------- allocation-free single-GPU variant
// dk_w4a16_matmul_reduce_static: the fused matmul + reduce launch of dk_w4a16_matmul_allreduce on one
// GPU (world 1), for callers that cannot allocate device memory themselves (see decodek.h). Its
// scratch - the header (launch epoch, CTA arrival count) and the tagged partial-sum cells - lives in
// the file-scope array below instead of a buffer from dk_tp_buffer_alloc.
namespace dk {
namespace {

constexpr int kStaticMaxM = 16;
constexpr int kStaticMaxN = 8192;
constexpr size_t kStaticScratchBytes = kTpHeaderBytes + 2ull * kStaticMaxM * kStaticMaxN * 8;  // 2 MiB + 256 B

// One copy per device that loads the library, held until the process exits. Host code must not use
// the name as an address: static_scratch_address() gets the device address.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device, looked up once per device (set-up done
// by the entry point's first call on that device). nullptr with dk_last_error set on failure.
void* static_scratch_address() {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    set_error(DK_ERR_CUDA, "w4a16_matmul_reduce_static: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error(DK_ERR_CUDA, "w4a16_matmul_reduce_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace
}  // namespace dk

extern "C" int dk_w4a16_matmul_reduce_static(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                                             const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M,
                                             int64_t N, int64_t K, int64_t group_size, const dk_matmul_config* cfg,
                                             dk_stream_t stream) {
  using namespace dk;
  int rc = check_w4a16_args("w4a16_matmul_reduce_static", x, ldx, qweight, scales, zeros, y, ldy, M, N, N, K,
                            group_size);
  if (rc != DK_OK) return rc;
  if (N > kStaticMaxN)
    return set_error(DK_ERR_INVALID,
                     "w4a16_matmul_reduce_static: N=%lld exceeds the static scratch limit of %d columns",
                     (long long)N, kStaticMaxN);
  if (M == 0 || N == 0) return DK_OK;
  const int flags = cfg ? cfg->flags : 0;
  if (!fast_ok(x, ldx, qweight, scales, zeros, N, K, group_size, flags))
    return set_error(DK_ERR_UNSUPPORTED,
                     "w4a16_matmul_reduce_static: needs group_size 128, N %% 8 == 0 and 16-byte aligned operands");
  char* base = static_cast<char*>(static_scratch_address());
  if (base == nullptr) return DK_ERR_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // No clearing: the array is zero when the library loads (epoch 0, no CTA arrived), and every launch
  // leaves the header consistent for the next one - each CTA arrives once, even one whose wait gave
  // up, and the last to arrive resets the count and stores the launch's epoch. So the epoch advances
  // across calls, and a cell left by an earlier call carries an older tag: a poll never accepts it.
  TPArgs tp;
  std::memset(&tp, 0, sizeof(tp));
  tp.cells[0] = reinterpret_cast<uint32_t*>(base + kTpHeaderBytes);
  tp.epoch = reinterpret_cast<unsigned long long*>(base);
  tp.arrive = reinterpret_cast<unsigned int*>(base + 8);
  tp.rank = 0;
  tp.world = 1;
  tp.max_m = kStaticMaxM;
  tp.max_n = kStaticMaxN;
  return run_fast(x, ldx, qweight, scales, zeros, bias, y, ldy, M, N, K, group_size, cfg, 0, NormArgs(), st, &tp);
}
