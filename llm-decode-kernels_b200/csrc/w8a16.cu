// FP8 (e4m3) weight-only matmul for decode (M <= 16 rows per launch): y = (x @ fp16(Wq)) * s (+ b).
//
// Replaces the reference's Triton W8A16 paths (kernels/fp8.py:42-127): weights are e4m3 bytes
// wq[K, N] (N contiguous) with one fp16 scale per output column; the scale is constant along K, so
// it multiplies the fp32 sum once at the end (kernels/fp8.py:81-82, 120).
//
// Same design as the W4A16 decode kernel (w4a16.cu): a producer warp streams 2-D TMA boxes of
// 32 columns x 128 K rows (4 KB) through a ring of shared-memory stages; persistent CTAs take
// balanced runs of 32-column chunks; kWarps/CW warps per chunk split the K stages; x is staged
// once per CTA in shared memory; split-K across the CTAs of a cluster meets in distributed shared
// memory; dot products run on tensor cores (mma.m16n8k16, weights as the 16-row operand).
//
// Fragment mapping. In a 16-row K step, MMA thread t of group g reads the 4-byte words of rows
// t, t+4, t+8, t+12 at columns 4g..4g+3 (four rows t..t+3 of 32 bytes each are one 128-byte bank
// sweep, so the reads are conflict-free without swizzling). PRMT pairs the bytes of one column from
// rows (t, t+4) and (t+8, t+12); cvt.rn.f16x2.e4m3x2 turns each pair into exact fp16. x is staged
// with the matching K permutation.
#include <cuda_fp8.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"

namespace dk {
namespace {

constexpr int kRows = 128;                // K rows per stage
constexpr int kBox = 32 * kRows;          // bytes of one 32-column box
constexpr int kWarps8 = 8;
constexpr int kXsPad8 = 16;

struct W8Params {
  const __half* x;
  int64_t ldx;
  const __half* scale;
  const __half* bias;
  __half* y;
  int64_t ldy;
  int M, N, K;
  int stages_total, split_stages, chunks, nbuf, xs_pitch, static_weights;
  uint32_t nbuf_rcp;  // ceil(2^32 / nbuf): it / nbuf == __umulhi(it, nbuf_rcp) for it < 2^28
  int* err;
  L2Prefetch pf;  // ranges to pull into L2 for a later launch (a hint)
};

struct Layout8 {
  int w_off, xs_off, red_off, bar_off, total;
};

__host__ __device__ inline Layout8 layout8(int cw, int nbuf, int M, int xs_pitch, int /*split*/) {
  const int wpc = kWarps8 / cw;
  Layout8 L;
  L.w_off = 0;
  L.xs_off = nbuf * cw * kBox;
  L.red_off = L.xs_off + ((M * xs_pitch + 15) / 16) * 16;
  L.bar_off = L.red_off + wpc * M * cw * 32 * 4;  // the epilogue always reduces through it
  L.total = L.bar_off + 2 * nbuf * 8;
  return L;
}

__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t pair16) {
  uint32_t d;
  asm("{ .reg .b16 t; cvt.u16.u32 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(d) : "r"(pair16));
  return d;
}

template <int NT>
__device__ __forceinline__ void consume8(const uint8_t* __restrict__ box, const uint8_t* __restrict__ xrow,
                                         int xs_pitch, int M, int g, int t, float (&acc)[2][NT][4]) {
#pragma unroll
  for (int st = 0; st < kRows / 16; ++st) {
    const uint8_t* rb = box + (st * 16 + t) * 32 + g * 4;
    const uint32_t r0 = *reinterpret_cast<const uint32_t*>(rb);
    const uint32_t r1 = *reinterpret_cast<const uint32_t*>(rb + 4 * 32);
    const uint32_t r2 = *reinterpret_cast<const uint32_t*>(rb + 8 * 32);
    const uint32_t r3 = *reinterpret_cast<const uint32_t*>(rb + 12 * 32);
    const uint32_t p01a = prmt(r0, r1, 0x5140), p01b = prmt(r0, r1, 0x7362);  // cols 0,1 | 2,3
    const uint32_t p23a = prmt(r2, r3, 0x5140), p23b = prmt(r2, r3, 0x7362);
    const uint32_t a00 = e4m3x2_to_f16x2(p01a & 0xFFFF), a10 = e4m3x2_to_f16x2(p01a >> 16);
    const uint32_t a20 = e4m3x2_to_f16x2(p01b & 0xFFFF), a30 = e4m3x2_to_f16x2(p01b >> 16);
    const uint32_t a01 = e4m3x2_to_f16x2(p23a & 0xFFFF), a11 = e4m3x2_to_f16x2(p23a >> 16);
    const uint32_t a21 = e4m3x2_to_f16x2(p23b & 0xFFFF), a31 = e4m3x2_to_f16x2(p23b >> 16);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int m = nt * 8 + g;
      uint2 v = make_uint2(0, 0);
      if (m < M) v = *reinterpret_cast<const uint2*>(xrow + m * xs_pitch + st * 32 + t * 8);
      mma_16816(acc[0][nt], a00, a10, a01, a11, v.x, v.y);  // columns 4g, 4g+1
      mma_16816(acc[1][nt], a20, a30, a21, a31, v.x, v.y);  // columns 4g+2, 4g+3
    }
  }
}

template <int NT, int CW>
__global__ void __launch_bounds__((kWarps8 + 1) * 32, 3 - NT)
    w8a16_gemv_kernel(const __grid_constant__ CUtensorMap mw, const W8Params p) {
  constexpr int WPC = kWarps8 / CW;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the shared array (accesses stay shared-space)
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int S = gridDim.y;
  const Layout8 L = layout8(CW, p.nbuf, p.M, p.xs_pitch, S);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + p.nbuf;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = blockIdx.y;
  const int s_begin = rank * p.split_stages;
  const int s_end = min(s_begin + p.split_stages, p.stages_total);
  const int nst = max(0, s_end - s_begin);
  int c_begin, c_end;
  if (S == 1) {
    c_begin = static_cast<int>((static_cast<int64_t>(blockIdx.x) * p.chunks) / gridDim.x);
    c_end = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * p.chunks) / gridDim.x);
  } else {
    c_begin = blockIdx.x * CW;
    c_end = min(c_begin + CW, p.chunks);
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
  if (warp == kWarps8) {
    if (p.pf.n) l2_prefetch_share(p.pf, blockIdx.x + gridDim.x * blockIdx.y, gridDim.x * gridDim.y, lane);
    if (!p.static_weights) pdl_wait();
    if (lane == 0) {
      prefetch_tensormap(&mw);
      int it = 0;
      for (int tile = c_begin; tile < c_end && ok; tile += CW) {
        const int nch = min(CW, c_end - tile);
        for (int s = s_begin; s < s_end; ++s, ++it) {
          const int round = static_cast<int>(__umulhi(static_cast<uint32_t>(it), p.nbuf_rcp));
          const int buf = it - round * p.nbuf;
          if (it >= p.nbuf && !mbar_wait(&empty[buf], (round - 1) & 1, p.err, DK_DEVERR_WAIT_EMPTY)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[buf], nch * kBox);
          for (int c = 0; c < nch; ++c)
            tma_load_2d(smem + L.w_off + (buf * CW + c) * kBox, &mw, (tile + c) * 32, s * kRows, &full[buf]);
        }
      }
    }
    __syncwarp();
  } else {
    pdl_wait();
    {
      // x[:, K slice] -> shared memory; in each 16-element block lane t's 4 values come first:
      // (x_t, x_{t+4}, x_{t+8}, x_{t+12}) for t = 0..3
      // The M > 8 variant (24 iterations per thread for 16 rows of a 1536-wide K slice) issues the
      // loads of kB iterations before it stores any of them; item i goes to the same thread either way.
      const int k0 = s_begin * kRows;
      const int nblk = nst * (kRows / 16);
      constexpr int kB = NT == 1 ? 1 : 4;
      constexpr int kThr8 = kWarps8 * 32;
      const int items = p.M * nblk * 4;
      for (int i0 = threadIdx.x; i0 < items; i0 += kB * kThr8) {
        __half v[kB][4];
#pragma unroll
        for (int u = 0; u < kB; ++u) {
          const int i = i0 + u * kThr8;
          const int m = i / (nblk * 4), rem = i % (nblk * 4), b = rem / 4, t = rem % 4;
          const int k = k0 + b * 16 + t;
#pragma unroll
          for (int e = 0; e < 4; ++e)
            v[u][e] = (i < items && k + 4 * e < p.K) ? __ldcg(p.x + m * p.ldx + k + 4 * e) : __float2half(0.f);
        }
#pragma unroll
        for (int u = 0; u < kB; ++u) {
          const int i = i0 + u * kThr8;
          if (i >= items) break;
          const int m = i / (nblk * 4), rem = i % (nblk * 4), b = rem / 4, t = rem % 4;
          uint2 o;
          o.x = half2_bits(v[u][0], v[u][1]);
          o.y = half2_bits(v[u][2], v[u][3]);
          *reinterpret_cast<uint2*>(smem + L.xs_off + m * p.xs_pitch + b * 32 + t * 8) = o;
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kWarps8 * 32) : "memory");
    }
    const int g = lane >> 2, t = lane & 3;
    const int slot = warp % CW, phase = warp / CW;
    float* red = reinterpret_cast<float*>(smem + L.red_off);
    int tile_idx = 0;
    for (int tile = c_begin; tile < c_end; tile += CW, ++tile_idx) {
      const int nch = min(CW, c_end - tile);
      const bool active = slot < nch;
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
        if (active)
          consume8<NT>(smem + L.w_off + (buf * CW + slot) * kBox, smem + L.xs_off + ls * (kRows / 16) * 32,
                       p.xs_pitch, p.M, g, t, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
      }
      // partial sums -> red[phase][m][col]; combine, scale, bias
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
      asm volatile("bar.sync 1, %0;" ::"r"(kWarps8 * 32) : "memory");
      const int ncols = nch * 32;
      for (int e = threadIdx.x; e < p.M * ncols; e += kWarps8 * 32) {
        const int m = e / ncols, col = e % ncols;
        float v = red[m * CW * 32 + col];
#pragma unroll
        for (int j = 1; j < WPC; ++j) v += red[(j * p.M + m) * CW * 32 + col];
        const int n = tile * 32 + col;
        if (S == 1) {
          if (n < p.N) {
            v *= __half2float(p.scale[n]);
            if (p.bias != nullptr) v += __half2float(p.bias[n]);
            p.y[m * p.ldy + n] = __float2half_rn(v);
          }
        } else {
          red[m * CW * 32 + col] = v;
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kWarps8 * 32) : "memory");
    }
  }

  if (__syncthreads_or(!ok)) {
    if (warp == kWarps8 && lane == 0) {
      const uint64_t t0 = globaltimer_ns();
      for (int b = 0; b < p.nbuf; ++b)
        while (!mbar_try_wait(&full[b], 0) && !mbar_try_wait(&full[b], 1) && globaltimer_ns() - t0 < 500000000ull) {
        }
    }
    if (S > 1) {
      cluster_sync();
      cluster_sync();
    }
    return;
  }
  if (S > 1) {
    cluster_sync();
    const float* red = reinterpret_cast<const float*>(smem + L.red_off);
    const int ncols = min(CW, c_end - c_begin) * 32;
    for (int e = threadIdx.x; e < p.M * ncols; e += blockDim.x) {
      if (e % S != rank) continue;
      const int m = e / ncols, col = e % ncols;
      const int n = c_begin * 32 + col;
      if (n >= p.N) continue;
      const float* src = red + m * CW * 32 + col;
      float v = 0.f;
      for (int q = 0; q < S; ++q) v += ld_shared_cluster_f32(map_shared_rank(src, q));
      v *= __half2float(p.scale[n]);
      if (p.bias != nullptr) v += __half2float(p.bias[n]);
      p.y[m * p.ldy + n] = __float2half_rn(v);
    }
    cluster_sync();
  }
}

// Any-alignment fallback: one thread per (row, column), fp32 sum in K order, scale at the end
// (kernels/fp8.py:113-123 without the tiling).
__global__ void w8a16_generic_kernel(const __half* __restrict__ x, int64_t ldx, const uint8_t* __restrict__ wq,
                                     const __half* __restrict__ scale, const __half* __restrict__ bias,
                                     __half* __restrict__ y, int64_t ldy, int M, int N, int K) {
  pdl_wait();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) {
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(wq[static_cast<int64_t>(k) * N + n], __NV_E4M3);
    acc = fmaf(__half2float(x[m * ldx + k]), __half2float(__half(hr)), acc);
  }
  acc *= __half2float(scale[n]);
  if (bias != nullptr) acc += __half2float(bias[n]);
  y[m * ldy + n] = __float2half_rn(acc);
}

using W8Kernel = void (*)(const CUtensorMap, const W8Params);

W8Kernel variant8(int nt, int cw) {
  static const W8Kernel table[2][4] = {
      {w8a16_gemv_kernel<1, 1>, w8a16_gemv_kernel<1, 2>, w8a16_gemv_kernel<1, 4>, w8a16_gemv_kernel<1, 8>},
      {w8a16_gemv_kernel<2, 1>, w8a16_gemv_kernel<2, 2>, w8a16_gemv_kernel<2, 4>, w8a16_gemv_kernel<2, 8>}};
  const int lg = cw == 1 ? 0 : cw == 2 ? 1 : cw == 4 ? 2 : 3;
  return table[nt - 1][lg];
}

void set_attrs8() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && !done[dev]) {
    for (int nt = 1; nt <= 2; ++nt)
      for (int cw = 1; cw <= 8; cw *= 2)
        opt_in_dynamic_smem(variant8(nt, cw));
    done[dev] = true;
  }
}

struct Choice8 {
  int cw, split, nbuf, nctas;
  size_t smem;
  double cost;
};

int xs_pitch8(int sps) { return sps * (kRows / 16) * 32 + kXsPad8; }

Choice8 choose8_uncached(int M, int N, int K, const dk_matmul_config* cfg) {
  const DeviceInfo& dev = device_info();
  set_attrs8();
  const int stages_total = (K + kRows - 1) / kRows;
  const int chunks = (N + 31) / 32;
  const int nt = M <= 8 ? 1 : 2;
  Choice8 best = {0, 0, 0, 0, 0, 1e300};
  int want_split = (cfg && cfg->split_k > 0) ? std::min(cfg->split_k, std::min(8, stages_total)) : 0;
  while (want_split > 1 && (want_split - 1) * ((stages_total + want_split - 1) / want_split) >= stages_total)
    --want_split;
  const int want_bn = (cfg && (cfg->block_n == 32 || cfg->block_n == 64 || cfg->block_n == 128 ||
                               cfg->block_n == 256)) ? cfg->block_n : 0;
  for (int cw = 8; cw >= 1; cw /= 2) {
    if (want_bn && want_bn != 32 * cw) continue;
    const int wpc = kWarps8 / cw;
    for (int split = 1; split <= 8; ++split) {
      if (want_split && want_split != split) continue;
      if (split > stages_total) break;
      const int sps = (stages_total + split - 1) / split;
      if ((split - 1) * sps >= stages_total) continue;
      const int pitch = xs_pitch8(sps);
      if (static_cast<size_t>(M) * pitch > 64 * 1024) continue;
      const int tiles = (chunks + cw - 1) / cw;
      const int stages_per_cta = sps * (split > 1 ? 1 : (tiles + dev.num_sms - 1) / dev.num_sms);
      int nbuf = std::min(std::max(stages_per_cta, 2), 16);
      Layout8 L = layout8(cw, nbuf, M, pitch, split);
      while (nbuf > 2 && static_cast<size_t>(L.total) + 1024 > 110 * 1024) {
        --nbuf;
        L = layout8(cw, nbuf, M, pitch, split);
      }
      const size_t smem = static_cast<size_t>(L.total) + 1024;
      if (smem > static_cast<size_t>(dev.max_smem_optin)) continue;
      // ring depth >= warps per chunk once buffers are reused (the W4A16 GEMV's rule: a shallower
      // ring would let a full-barrier parity wait pass on the buffer's previous phase)
      if (nbuf < std::min(wpc, stages_per_cta)) continue;
      int occ = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, variant8(nt, cw), (kWarps8 + 1) * 32, smem) != cudaSuccess) {
        cudaGetLastError();
        occ = 1;
      }
      occ = std::max(occ, 1);
      const int nctas = split == 1 ? std::min(chunks, dev.num_sms * occ) : tiles;
      if (split > 1 && static_cast<long>(nctas) * split > static_cast<long>(dev.num_sms) * occ) continue;
      const double per_cta = std::ceil(static_cast<double>(chunks) / nctas);
      const double tiles_cta = std::ceil(per_cta / cw);
      const double ctas_sm = std::ceil(static_cast<double>(nctas) * split / dev.num_sms);
      const double cs_sm = ctas_sm * per_cta * sps;
      const double t_mem = cs_sm * kBox / (6.4e12 / dev.num_sms) * 1e6;
      const double t_issue = cs_sm / 16.0;
      const double t_chain = tiles_cta * std::ceil(static_cast<double>(sps) / wpc) * 0.35;
      const double cost = 2.0 + std::max(t_mem, std::max(t_issue, t_chain)) + (split > 1 ? 0.5 : 0.0) + 0.2 * tiles_cta;
      if (cost < best.cost) best = {cw, split, nbuf, nctas, smem, cost};
    }
  }
  return best;
}

Choice8 choose8(int M, int N, int K, const dk_matmul_config* cfg) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int>, Choice8> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, M, N, K, cfg ? cfg->split_k : 0, cfg ? cfg->block_n : 0);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  Choice8 c = choose8_uncached(M, N, K, cfg);
  if (c.cw == 0 && cfg) {
    dk_matmul_config a = *cfg;
    a.split_k = 0;
    a.block_n = 0;
    c = choose8_uncached(M, N, K, &a);
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = c;
  return c;
}

}  // namespace
}  // namespace dk

namespace dk {
bool gemm_tc_fp8_ok(const void* x, int64_t ldx, const void* wq, int64_t M, int64_t N, int64_t K);
int launch_gemm_tc_fp8(const void* x, int64_t ldx, const uint8_t* wq, const void* scale, const void* bias, void* y,
                       int64_t ldy, int64_t M, int64_t N, int64_t K, cudaStream_t st);
void skinny_choice(int64_t rows, int64_t N, int64_t K, int* mb_out, int* split_out);
int launch_skinny_tc_fp8(const void* x, int64_t ldx, const uint8_t* wq, const void* scale, const void* bias, void* y,
                         int64_t ldy, int64_t M, int64_t N, int64_t K, bool static_weights, cudaStream_t st);
}  // namespace dk

extern "C" int dk_w8a16_matmul(const void* x, int64_t ldx, const uint8_t* wq, const void* scale, const void* bias,
                               void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, const dk_matmul_config* cfg,
                               dk_stream_t stream) {
  using namespace dk;
  if (M < 0 || N < 0 || K < 0) return set_error(DK_ERR_INVALID, "w8a16_matmul: negative size");
  if (ldx < K || ldy < N) return set_error(DK_ERR_INVALID, "w8a16_matmul: row stride smaller than the row");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return set_error(DK_ERR_INVALID, "w8a16_matmul: size out of range");
  if (M == 0 || N == 0) return DK_OK;
  if (!x || !wq || !scale || !y) return set_error(DK_ERR_INVALID, "w8a16_matmul: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int flags = cfg ? cfg->flags : 0;
  const bool fast = !(flags & DK_FLAG_GENERIC) && N % 16 == 0 && K > 0 && aligned16(wq);
  if (!fast) {
    const dim3 grid(static_cast<unsigned>((N + 127) / 128), static_cast<unsigned>(M), 1);
    cudaError_t e = launch(w8a16_generic_kernel, grid, dim3(128), 0, st, pdl_enabled(), dim3(1, 1, 1),
                           static_cast<const __half*>(x), ldx, wq, static_cast<const __half*>(scale),
                           static_cast<const __half*>(bias), static_cast<__half*>(y), ldy, static_cast<int>(M),
                           static_cast<int>(N), static_cast<int>(K));
    if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w8a16 generic launch: %s", cudaGetErrorString(e));
    return DK_OK;
  }
  if (!(flags & DK_FLAG_GEMV) && gemm_tc_fp8_ok(x, ldx, wq, M, N, K))
    return launch_gemm_tc_fp8(x, ldx, wq, scale, bias, y, ldy, M, N, K, st);
  // batched decode (16..127 rows) on the tcgen05 small-M kernel, the same rule as the int4 path
  if (!(flags & DK_FLAG_GEMV) && M >= 16 && N >= 128 && N % 16 == 0 && K % 64 == 0 && aligned16(x) &&
      ldx % 8 == 0 && (M > 16 || K >= 4096)) {
    int mb = 0, split = 0;
    skinny_choice(M, N, K, &mb, &split);
    if (mb != 0)
      return launch_skinny_tc_fp8(x, ldx, wq, scale, bias, y, ldy, M, N, K, (flags & DK_FLAG_STATIC_WEIGHTS) != 0, st);
  }
  CUtensorMap mw;
  if (!make_tensor_map_2d(&mw, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, N, K, N, 32, kRows, CU_TENSOR_MAP_SWIZZLE_NONE))
    return DK_ERR_CUDA;
  const DeviceInfo& dev = device_info();
  for (int64_t m0 = 0; m0 < M;) {
    int mc = static_cast<int>(std::min<int64_t>(16, M - m0));
    Choice8 c = choose8(mc, static_cast<int>(N), static_cast<int>(K), cfg);
    while (c.cw == 0 && mc > 1) {  // a long K slice leaves no tile for mc staged rows: fewer rows per launch
      mc = (mc + 1) / 2;
      c = choose8(mc, static_cast<int>(N), static_cast<int>(K), cfg);
    }
    if (c.cw == 0) return set_error(DK_ERR_UNSUPPORTED, "w8a16_matmul: no tile fits (M=%d, K=%lld)", mc, (long long)K);
    W8Params p;
    p.x = static_cast<const __half*>(x) + m0 * ldx;
    p.ldx = ldx;
    p.scale = static_cast<const __half*>(scale);
    p.bias = static_cast<const __half*>(bias);
    p.y = static_cast<__half*>(y) + m0 * ldy;
    p.ldy = ldy;
    p.M = mc;
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.stages_total = static_cast<int>((K + kRows - 1) / kRows);
    p.split_stages = (p.stages_total + c.split - 1) / c.split;
    p.chunks = static_cast<int>((N + 31) / 32);
    p.nbuf = c.nbuf;
    p.nbuf_rcp = static_cast<uint32_t>((0x100000000ull + c.nbuf - 1) / c.nbuf);
    p.xs_pitch = xs_pitch8(p.split_stages);
    p.static_weights = (flags & DK_FLAG_STATIC_WEIGHTS) ? 1 : 0;
    p.err = dev.err_word;
    p.pf = l2_prefetch_from(m0 == 0 ? cfg : nullptr);
    const dim3 grid(c.nctas, c.split, 1);
    cudaError_t e = launch(variant8(mc <= 8 ? 1 : 2, c.cw), grid, dim3((kWarps8 + 1) * 32), c.smem, st, pdl_enabled(),
                           dim3(1, c.split, 1), mw, p);
    if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w8a16 gemv launch: %s", cudaGetErrorString(e));
    m0 += mc;
  }
  return DK_OK;
}
