// W4A16 matmul for decode (M <= 16 rows per launch): y = x @ dequant(W).T (+ bias).
//
// Replaces the reference's Triton GEMV/GEMM decode paths (kernels/w4a16.py:31-160) and its
// CUDA-core decode kernel (kernels/cuda/w4a16_decode.cu:29-121) with one sm_100a kernel:
//
// * Weight stream. Each CTA owns BN = 32*CW output columns and a K slice. A producer warp copies
//   the CTA's packed weights into a ring of shared-memory stages with cp.async.bulk (one 1-D bulk
//   copy per packed row segment, completion counted in bytes on a per-stage mbarrier). A stage is
//   16 packed rows = 128 K values = one quantization group, plus that group's scale and zero rows.
//   When the weights are marked static the producer issues its copies before waiting for the
//   previous kernel (programmatic dependent launch), so the weight fetch of layer i+1 overlaps the
//   tail of layer i.
// * Dequantization with the reference's rounding. A 32-bit word holds 8 K values of one column.
//   LOP3 with the 0x6400 exponent ("magic number" int4->fp16 conversion of Kim et al., "Who Says
//   Elephants Can't Run", and FasterTransformer) turns nibble pairs into fp16 (1024+q); an fp16
//   subtract of (1024+z) gives q-z exactly and one fp16 multiply by s rounds once - the same value
//   as the reference's `(q.to(fp16) - z) * s` (kernels/reference.py:35, kernels/w4a16.py:84).
// * Dot products on tensor cores with fp32 accumulation. mma.m16n8k16 with the dequantized weights
//   as the 16-row A operand ("swap AB": MMA rows = output columns) and x as the 8-column B operand
//   (MMA columns = batch rows). The MMA does the multiply-add work the reference's GEMV does with
//   FFMA, so the per-weight ALU cost is only unpack + dequant and does not grow with M <= 16.
//   K order inside an MMA is permuted (nibble pairs (0,4),(1,5),(2,6),(3,7)); x fragments are
//   loaded with the same permutation, so the sum is unchanged.
// * Split-K without workspace or atomics. The S K-slices of one column tile run as the S CTAs of
//   a thread-block cluster; partial sums meet in distributed shared memory and are added in rank
//   order (deterministic), replacing the reference's zero-fill + fp32 atomics + cast kernels
//   (kernels/w4a16.py:271-275, kernels/cuda/w4a16_decode.cu:161-180).
//
// Shared-memory row pitch is BN*4 + 32 bytes: the 8 lanes of each quarter-warp read 4 rows x 2
// adjacent 16-byte pieces, and a pitch of 32 (mod 128) bytes puts them on 8 distinct bank groups.
#include <algorithm>
#include <cstdio>

#include "common.cuh"

namespace dk {
namespace {

constexpr int kStageRows = 16;  // packed rows per stage (128 K values)
constexpr int kRowPad = 32;     // bytes added to each shared-memory row

struct GemvParams {
  const __half* x;
  int64_t ldx;
  const int32_t* qw;
  const __half* scales;
  const __half* zeros;
  const __half* bias;
  __half* y;
  int64_t ldy;
  int M, N, K;
  int group_rows;      // group_size / 8 (multiple of kStageRows)
  int split_rows;      // packed rows per cluster rank (multiple of kStageRows)
  int nbuf;            // ring depth in stages
  int bar_off;         // byte offset of the mbarriers (after the ring and the reduction scratch)
  int static_weights;  // prefetch weights before waiting for the previous kernel
  int* err;
};

template <int CW>
struct GemvLayout {
  static constexpr int BN = 32 * CW;
  static constexpr int ROW_BYTES = BN * 4 + kRowPad;
  static constexpr int W_BYTES = kStageRows * ROW_BYTES;
  static constexpr int STAGE_BYTES = W_BYTES + 2 * BN * 2;  // weights, scales row, zeros row
};

// Shared memory: [ring of `nbuf` stages | reduction scratch] (the scratch reuses the ring once all
// copies have landed), then `nbuf` full and `nbuf` empty mbarriers at `bar_off`.
template <int NT, int CW, int NWC>
__global__ void __launch_bounds__((NWC + 1) * 32) w4a16_gemv_kernel(const GemvParams p) {
  using L = GemvLayout<CW>;
  constexpr int BN = L::BN;
  constexpr int MT = 8 * NT;
  constexpr int IPW = 4 * CW / NWC;  // (chunk, 4-row step) items per consumer warp per stage
  static_assert(NWC % CW == 0 && (4 * CW) % NWC == 0, "warp split");
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + p.nbuf;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int n_valid = min(BN, p.N - n0);
  const int rank = blockIdx.y;  // cluster dims (1, S, 1): rank == blockIdx.y
  const int S = gridDim.y;
  const int r0 = rank * p.split_rows;
  const int r1 = min(r0 + p.split_rows, p.K / 8);
  const int nstages = max(0, (r1 - r0) / kStageRows);

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nbuf; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NWC);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  bool ok = true;
  if (warp == NWC) {
    // ------------------------------------------------------------------ producer warp
    if (!p.static_weights) pdl_wait();
    const uint32_t w_bytes = static_cast<uint32_t>(n_valid) * 4;
    const uint32_t sz_bytes = static_cast<uint32_t>(n_valid) * 2;
    const uint32_t stage_tx = kStageRows * w_bytes + 2 * sz_bytes;
    for (int s = 0; s < nstages; ++s) {
      const int buf = s % p.nbuf;
      if (s >= p.nbuf && !mbar_wait(&empty[buf], ((s / p.nbuf) - 1) & 1, p.err, DK_DEVERR_WAIT_EMPTY)) {
        ok = false;
        break;
      }
      uint8_t* st = smem + buf * L::STAGE_BYTES;
      const int row0 = r0 + s * kStageRows;
      if (lane == 0) mbar_arrive_expect_tx(&full[buf], stage_tx);
      __syncwarp();
      if (lane < kStageRows) {
        bulk_g2s(st + lane * L::ROW_BYTES, p.qw + static_cast<int64_t>(row0 + lane) * p.N + n0,
                 w_bytes, &full[buf]);
      } else if (lane == kStageRows || lane == kStageRows + 1) {
        const int g = row0 / p.group_rows;
        const __half* src = (lane == kStageRows ? p.scales : p.zeros) + static_cast<int64_t>(g) * p.N + n0;
        bulk_g2s(st + L::W_BYTES + (lane - kStageRows) * BN * 2, src, sz_bytes, &full[buf]);
      }
    }
    if (p.static_weights) pdl_wait();
  } else {
    // ------------------------------------------------------------------ consumer warps
    pdl_wait();  // x (and, for non-static weights, W) come from earlier kernels
    const int g = lane >> 2;  // MMA group: A rows g, g+8 ; B column g
    const int t = lane & 3;   // MMA thread-in-group: K slots 2t.., 2t+8..
    const int chunk = warp % CW;
    const int step0 = warp / CW;
    constexpr int STEP_STRIDE = NWC / CW;
    float acc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

    for (int s = 0; s < nstages; ++s) {
      const int buf = s % p.nbuf;
      const int row0 = r0 + s * kStageRows;
      // x fragments for this stage (independent of the weights: issued before the wait)
      uint32_t bx[IPW][NT][4];
#pragma unroll
      for (int j = 0; j < IPW; ++j) {
        const int R = row0 + (step0 + j * STEP_STRIDE) * 4 + t;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m = nt * 8 + g;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (m < p.M) v = __ldcg(reinterpret_cast<const uint4*>(p.x + m * p.ldx + R * 8));  // L2, not L1
          bx[j][nt][0] = prmt(v.x, v.z, 0x5410);  // (x0, x4)
          bx[j][nt][1] = prmt(v.x, v.z, 0x7632);  // (x1, x5)
          bx[j][nt][2] = prmt(v.y, v.w, 0x5410);  // (x2, x6)
          bx[j][nt][3] = prmt(v.y, v.w, 0x7632);  // (x3, x7)
        }
      }
      if (!mbar_wait(&full[buf], (s / p.nbuf) & 1, p.err, DK_DEVERR_WAIT_FULL)) {
        ok = false;
        break;
      }
      const uint8_t* st = smem + buf * L::STAGE_BYTES;
      // per-column dequant constants for this group: zA = 1024+z, nzB = -(64+z), sc = s
      const uint2 s4 = *reinterpret_cast<const uint2*>(st + L::W_BYTES + (chunk * 32 + 4 * g) * 2);
      const uint2 z4 = *reinterpret_cast<const uint2*>(st + L::W_BYTES + BN * 2 + (chunk * 32 + 4 * g) * 2);
      uint32_t zA[4], nzB[4], sc[4];
      {
        const uint32_t k1024 = 0x64006400u, k64 = 0x54005400u;
        const uint32_t zz[4] = {prmt(z4.x, 0, 0x1010), prmt(z4.x, 0, 0x3232), prmt(z4.y, 0, 0x1010),
                                prmt(z4.y, 0, 0x3232)};
        const uint32_t ss[4] = {prmt(s4.x, 0, 0x1010), prmt(s4.x, 0, 0x3232), prmt(s4.y, 0, 0x1010),
                                prmt(s4.y, 0, 0x3232)};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          zA[c] = hsub2_rn(zz[c], hsub2_rn(0, k1024));  // z + 1024 (exact)
          nzB[c] = hsub2_rn(hsub2_rn(0, k64), zz[c]);    // -64 - z (exact)
          sc[c] = ss[c];
        }
      }
#pragma unroll
      for (int j = 0; j < IPW; ++j) {
        const int lr = (step0 + j * STEP_STRIDE) * 4 + t;
        const uint4 wv = *reinterpret_cast<const uint4*>(st + lr * L::ROW_BYTES + chunk * 128 + g * 16);
        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t W[4][4];  // [column][nibble pair]
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t w = words[c];
          const uint32_t w8 = w >> 8;
          const uint32_t p0 = lop3_and_or(w, 0x000F000Fu, 0x64006400u);   // 1024 + (q0, q4)
          const uint32_t p1 = lop3_and_or(w, 0x00F000F0u, 0x64006400u);   // 1024 + 16*(q1, q5)
          const uint32_t p2 = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);  // 1024 + (q2, q6)
          const uint32_t p3 = lop3_and_or(w8, 0x00F000F0u, 0x64006400u);  // 1024 + 16*(q3, q7)
          const uint32_t sixteenth = 0x2C002C00u;                         // (1/16, 1/16)
          W[c][0] = hmul2_rn(hsub2_rn(p0, zA[c]), sc[c]);
          W[c][1] = hmul2_rn(hfma2_rn(p1, sixteenth, nzB[c]), sc[c]);
          W[c][2] = hmul2_rn(hsub2_rn(p2, zA[c]), sc[c]);
          W[c][3] = hmul2_rn(hfma2_rn(p3, sixteenth, nzB[c]), sc[c]);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // tile 0: MMA rows g <- column 4g, g+8 <- column 4g+1 ; tile 1: columns 4g+2, 4g+3
          mma_16816(acc[0][nt], W[0][0], W[1][0], W[0][1], W[1][1], bx[j][nt][0], bx[j][nt][1]);
          mma_16816(acc[0][nt], W[0][2], W[1][2], W[0][3], W[1][3], bx[j][nt][2], bx[j][nt][3]);
          mma_16816(acc[1][nt], W[2][0], W[3][0], W[2][1], W[3][1], bx[j][nt][0], bx[j][nt][1]);
          mma_16816(acc[1][nt], W[2][2], W[3][2], W[2][3], W[3][3], bx[j][nt][2], bx[j][nt][3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[buf]);
    }

    // The reduction scratch overlays the ring: every consumer warp must be done reading it.
    asm volatile("bar.sync 1, %0;" ::"r"(NWC * 32) : "memory");
    if (ok) {
      float* red = reinterpret_cast<float*>(smem);
      const int kslot = step0;  // 0 .. NWC/CW-1
#pragma unroll
      for (int tile = 0; tile < 2; ++tile)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int m = nt * 8 + 2 * t + (e & 1);
            const int col = chunk * 32 + 4 * g + 2 * tile + (e >> 1);
            if (m < p.M) red[(kslot * MT + m) * BN + col] = acc[tile][nt][e];
          }
    }
  }

  // ------------------------------------------------------------------ reduction + epilogue
  // A consumer that timed out leaves the ring in an unknown state: the producer waits (bounded)
  // for the copies it issued, then every thread returns.
  if (__syncthreads_or(!ok)) {
    if (warp == NWC && lane == 0) {
      // outstanding copies of buffer b belong to the last stage issued into it
      const uint64_t t0 = globaltimer_ns();
      for (int b = 0; b < min(nstages, p.nbuf); ++b) {
        const int s_last = b + ((nstages - 1 - b) / p.nbuf) * p.nbuf;
        while (!mbar_try_wait(&full[b], (s_last / p.nbuf) & 1) && globaltimer_ns() - t0 < 500000000ull) {
        }
      }
    }
    if (gridDim.y > 1) {  // the other CTAs of the cluster still pass their two cluster barriers
      cluster_sync();
      cluster_sync();
    }
    return;
  }
  constexpr int KSLOTS = NWC / CW;
  float* red = reinterpret_cast<float*>(smem);
  const int M = min(p.M, MT);
  for (int e = threadIdx.x; e < M * BN; e += blockDim.x) {
    float v = red[e];
#pragma unroll
    for (int k = 1; k < KSLOTS; ++k) v += red[k * MT * BN + e];
    red[e] = v;
  }
  if (S > 1) {
    cluster_sync();
    for (int e = threadIdx.x; e < M * BN; e += blockDim.x) {
      if (e % S != rank) continue;
      const int m = e / BN, col = e % BN;
      if (col >= n_valid) continue;
      float v = 0.f;
      for (int q = 0; q < S; ++q) v += ld_shared_cluster_f32(map_shared_rank(red + e, q));
      if (p.bias != nullptr) v += __half2float(p.bias[n0 + col]);
      p.y[m * p.ldy + n0 + col] = __float2half_rn(v);
    }
    cluster_sync();  // keep this CTA's scratch alive until every rank has read it
  } else {
    __syncthreads();
    for (int e = threadIdx.x; e < M * BN; e += blockDim.x) {
      const int m = e / BN, col = e % BN;
      if (col >= n_valid) continue;
      float v = red[e];
      if (p.bias != nullptr) v += __half2float(p.bias[n0 + col]);
      p.y[m * p.ldy + n0 + col] = __float2half_rn(v);
    }
  }
}

// Any-alignment fallback: one thread per (row, column), plain loads, the reference's fp16 weight
// rounding and an fp32 sum in K order (kernels/w4a16.py:134-152 without the tiling). Used for
// N % 8 != 0, group sizes that are not a multiple of 128, unaligned pointers or strides.
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

struct Choice {
  int cw, split, nbuf;
  size_t smem;
};

// Byte offset of the mbarriers: after the ring and after the reduction scratch.
template <int CW>
size_t gemv_bar_off(int nbuf, int nwc, int mt) {
  using L = GemvLayout<CW>;
  const size_t ring = static_cast<size_t>(nbuf) * L::STAGE_BYTES;
  const size_t red = static_cast<size_t>(nwc / CW) * mt * L::BN * 4;
  return (std::max(ring, red) + 15) / 16 * 16;
}

size_t bar_off_for(int cw, int nbuf, int mt) {
  switch (cw) {
    case 1: return gemv_bar_off<1>(nbuf, 2, mt);
    case 2: return gemv_bar_off<2>(nbuf, 4, mt);
    default: return gemv_bar_off<4>(nbuf, 8, mt);
  }
}

size_t smem_for(int cw, int nbuf, int mt) { return bar_off_for(cw, nbuf, mt) + 2 * nbuf * sizeof(uint64_t); }

// Pick the column tile (BN = 32*cw) and cluster split-K for one launch. Cost model: the busiest
// SM's weight bytes at the HBM share of one SM, plus a per-stage latency term, plus a per-wave
// latency term. Requested values in cfg override the model.
Choice choose(int M, int N, int K, const dk_matmul_config* cfg) {
  const DeviceInfo& dev = device_info();
  const int rows = K / 8;
  const int total_stages = rows / kStageRows;
  const int mt = M <= 8 ? 8 : 16;
  const size_t smem_budget = 100 * 1024;  // two CTAs per SM, leaving room for the next kernel
  Choice best = {2, 1, 1, 0};
  double best_cost = 1e30;
  const int cws[3] = {1, 2, 4};
  for (int ci = 0; ci < 3; ++ci) {
    const int cw = cws[ci];
    if (cfg && cfg->block_n && cfg->block_n != 32 * cw) continue;
    const int bn = 32 * cw;
    const int tiles = (N + bn - 1) / bn;
    for (int split = 1; split <= 8; ++split) {
      if (cfg && cfg->split_k && cfg->split_k != split) continue;
      if (split > total_stages) break;
      const int stages = (total_stages + split - 1) / split;
      // each rank must own at least one stage
      if ((split - 1) * stages >= total_stages) continue;
      int nbuf = stages;
      while (nbuf > 2 && smem_for(cw, nbuf, mt) > smem_budget) --nbuf;
      const size_t smem = smem_for(cw, nbuf, mt);
      const int threads = (cw == 1 ? 3 : cw == 2 ? 5 : 9) * 32;
      int occ = std::min<int>(static_cast<int>(dev.smem_per_sm / (smem + 1024)), 2048 / threads);
      occ = std::max(occ, 1);
      const long ctas = static_cast<long>(tiles) * split;
      const long per_sm = (ctas + dev.num_sms - 1) / dev.num_sms;
      const double bytes_per_sm = static_cast<double>(per_sm) * stages * kStageRows * bn * 4.25;
      const double waves = static_cast<double>((ctas + static_cast<long>(dev.num_sms) * occ - 1) /
                                               (static_cast<long>(dev.num_sms) * occ));
      const double cost = bytes_per_sm / (6.4e12 / dev.num_sms) * 1e9  // ns of HBM time
                          + 40.0 * stages + 600.0 * waves + (split > 1 ? 300.0 : 0.0);
      if (cost < best_cost) {
        best_cost = cost;
        best = {cw, split, nbuf, smem};
      }
    }
  }
  return best;
}

template <int NT, int CW>
int launch_gemv(const GemvParams& p, const Choice& c, cudaStream_t stream) {
  constexpr int NWC = 2 * CW;
  auto kernel = w4a16_gemv_kernel<NT, CW, NWC>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         device_info().max_smem_optin);
    cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    attr_done[dev] = true;
  }
  const dim3 grid((p.N + 32 * CW - 1) / (32 * CW), c.split, 1);
  const dim3 block((NWC + 1) * 32, 1, 1);
  cudaError_t e = launch(kernel, grid, block, c.smem, stream, pdl_enabled(), dim3(1, c.split, 1), p);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w4a16 gemv launch: %s", cudaGetErrorString(e));
  return DK_OK;
}

}  // namespace
}  // namespace dk

extern "C" int dk_w4a16_matmul(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                               const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M,
                               int64_t N, int64_t K, int64_t group_size, const dk_matmul_config* cfg,
                               dk_stream_t stream) {
  using namespace dk;
  if (M < 0 || N < 0 || K < 0) return set_error(DK_ERR_INVALID, "w4a16_matmul: negative size");
  if (group_size <= 0 || group_size % 8 != 0 || K % group_size != 0)
    return set_error(DK_ERR_INVALID, "w4a16_matmul: need K %% group_size == 0 and group_size %% 8 == 0 (K=%lld, group_size=%lld)",
                     (long long)K, (long long)group_size);
  if (ldx < K || ldy < N) return set_error(DK_ERR_INVALID, "w4a16_matmul: row stride smaller than the row");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || (K / 8) * N > (int64_t(1) << 40))
    return set_error(DK_ERR_INVALID, "w4a16_matmul: size out of range");
  if (M == 0 || N == 0) return DK_OK;
  if (!x || !qweight || !scales || !zeros || !y) return set_error(DK_ERR_INVALID, "w4a16_matmul: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int flags = cfg ? cfg->flags : 0;
  const bool fast = !(flags & DK_FLAG_GENERIC) && N % 8 == 0 && group_size % 128 == 0 && K > 0 &&
                    aligned16(x) && ldx % 8 == 0 && aligned16(qweight) && aligned16(scales) && aligned16(zeros);
  if (!fast) {
    const dim3 grid(static_cast<unsigned>((N + 127) / 128), static_cast<unsigned>(M), 1);
    cudaError_t e = launch(w4a16_generic_kernel, grid, dim3(128, 1, 1), 0, st, pdl_enabled(), dim3(1, 1, 1),
                           static_cast<const __half*>(x), ldx, qweight, static_cast<const __half*>(scales),
                           static_cast<const __half*>(zeros), static_cast<const __half*>(bias),
                           static_cast<__half*>(y), ldy, static_cast<int>(M), static_cast<int>(N),
                           static_cast<int>(K), static_cast<int>(group_size));
    if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w4a16 generic launch: %s", cudaGetErrorString(e));
    return DK_OK;
  }
  const DeviceInfo& dev = device_info();
  for (int64_t m0 = 0; m0 < M; m0 += 16) {
    const int mc = static_cast<int>(std::min<int64_t>(16, M - m0));
    Choice c = choose(mc, static_cast<int>(N), static_cast<int>(K), cfg);
    if (c.smem > static_cast<size_t>(dev.max_smem_optin))
      return set_error(DK_ERR_UNSUPPORTED, "w4a16_matmul: tile needs %zu bytes of shared memory", c.smem);
    GemvParams p;
    p.x = static_cast<const __half*>(x) + m0 * ldx;
    p.ldx = ldx;
    p.qw = qweight;
    p.scales = static_cast<const __half*>(scales);
    p.zeros = static_cast<const __half*>(zeros);
    p.bias = static_cast<const __half*>(bias);
    p.y = static_cast<__half*>(y) + m0 * ldy;
    p.ldy = ldy;
    p.M = mc;
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.group_rows = static_cast<int>(group_size / 8);
    const int total_stages = static_cast<int>(K / 8) / kStageRows;
    p.split_rows = ((total_stages + c.split - 1) / c.split) * kStageRows;
    p.nbuf = c.nbuf;
    p.bar_off = static_cast<int>(bar_off_for(c.cw, c.nbuf, mc <= 8 ? 8 : 16));
    p.static_weights = (flags & DK_FLAG_STATIC_WEIGHTS) ? 1 : 0;
    p.err = dev.err_word;
    int rc;
    if (mc <= 8) {
      rc = c.cw == 1 ? launch_gemv<1, 1>(p, c, st) : c.cw == 2 ? launch_gemv<1, 2>(p, c, st) : launch_gemv<1, 4>(p, c, st);
    } else {
      rc = c.cw == 1 ? launch_gemv<2, 1>(p, c, st) : c.cw == 2 ? launch_gemv<2, 2>(p, c, st) : launch_gemv<2, 4>(p, c, st);
    }
    if (rc != DK_OK) return rc;
  }
  return DK_OK;
}
