// The end and the start of a per-op greedy decode step: the tied fp16 lm_head with the final RMSNorm
// and the greedy pick fused in, and the embedding gather of the step's tokens.
//
// Replaces, for T == 1, the tail of the reference's forward and the bookkeeping of its graph
// decoder (kernels/e2e/model.py:248-253: final norm, F.linear with the fp16 lm_head;
// kernels/e2e/run.py:69-74: argmax, out[:, pos] = pick, tok = pick, pos += 1) and the embedding
// lookup at the head of the forward (model.py:227), so a decode step launches only this library's
// kernels.
//
// lm_head: HBM-bound (vocab x hidden fp16 weights, 467 MB for Qwen2.5's 151936 x 1536, read once).
// Two CTAs per SM of 8 warps; each CTA owns a contiguous range of vocabulary rows and each warp
// 2 to 4 rows at a time, its lanes reading 16-byte vectors of those rows (a warp-wide 512-byte coalesced load
// per vector index) against the normalized input rows held in fp32 in shared memory. Dot products
// accumulate in fp32 and round to fp16 like the reference's cuBLAS fp16 GEMM output; the pick is the
// first maximum of those fp16 logits (torch.argmax's lowest-index tie rule). Every CTA leaves its best
// (value, index) per row in the workspace; the last CTA to arrive on the workspace counter combines
// them, writes the tokens, the history entry and the new position, and resets the counter.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace dk {
namespace {

constexpr int kHeadThreads = 256;
constexpr int kHeadWarps = kHeadThreads / 32;
constexpr int kHeadMaxRows = 8;
constexpr int kHeadCtasPerSm = 2;
// Vocabulary rows a warp reads at once and 16-byte vectors per lane and row in flight per round: at
// one input row 4 x 6 (4 x 96 bytes per lane, the whole 1536-wide row of Qwen2.5-1.5B per round; 98%
// of the measured copy bandwidth on B200), fewer for more input rows, whose fp32 sums need registers.
template <int MR>
struct HeadShape {
  static constexpr int rows = MR == 1 ? 4 : MR == 2 ? 4 : 2;
  static constexpr int unroll = MR == 1 ? 6 : 3;
};

// Workspace: [0, 256) the arrival counter; then per CTA and row its best fp16 logit (as float) and
// its index.
struct HeadWs {
  unsigned* counter;
  float* best_v;  // [grid][kHeadMaxRows]
  int* best_i;
};

__device__ __forceinline__ void head_better(float& bv, int& bi, float v, int i) {
  // larger value wins; equal values: lower index (NaN never wins here, as no comparison is true)
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

template <int MR>
__global__ void __launch_bounds__(kHeadThreads, kHeadCtasPerSm) head_greedy_kernel(
    const __half* __restrict__ x, const __half* __restrict__ res, const __half* __restrict__ norm_w, float eps,
    const __half* __restrict__ W, int V, int H, int M, int64_t* __restrict__ tokens, int64_t* __restrict__ pos,
    int64_t* __restrict__ hist, int64_t hist_ld, int64_t hist_len, __half* __restrict__ logits, HeadWs ws,
    int* err) {
  extern __shared__ __align__(16) float xs[];  // [MR][H] normalized input rows, fp32
  __shared__ float red[kHeadWarps][MR];
  __shared__ float s_inv[MR];
  __shared__ float s_bv[kHeadWarps][MR];
  __shared__ int s_bi[kHeadWarps][MR];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nv = H / 8;
  pdl_wait();
  pdl_trigger();

  // ---- the final RMSNorm of every row (kernels/rmsnorm.py:28-37 rounding): h = x + res in fp16,
  // var = sum(h^2) / H in fp32, out = w * fp16(h / sqrt(var + eps)); or x itself without a norm
  for (int m = 0; m < M; ++m) {
    float ss = 0.f;
    for (int v = tid; v < nv; v += kHeadThreads) {
      uint4 a = __ldcg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(m) * H) + v);
      if (res != nullptr) {
        const uint4 b = __ldcg(reinterpret_cast<const uint4*>(res + static_cast<int64_t>(m) * H) + v);
        __half2* ah = reinterpret_cast<__half2*>(&a);
        const __half2* bh = reinterpret_cast<const __half2*>(&b);
#pragma unroll
        for (int j = 0; j < 4; ++j) ah[j] = __hadd2_rn(ah[j], bh[j]);
      }
      const __half2* ah = reinterpret_cast<const __half2*>(&a);
      float* dst = xs + m * H + 8 * v;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(ah[j]);
        dst[2 * j] = f.x;
        dst[2 * j + 1] = f.y;
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp][m] = ss;
  }
  __syncthreads();
  if (tid < M) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kHeadWarps; ++w) tot += red[w][tid];
    s_inv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(H)), eps)));
  }
  __syncthreads();
  if (norm_w != nullptr) {
    for (int e = tid; e < M * H; e += kHeadThreads) {
      const int m = e / H, k = e - m * H;
      const __half nrm = __float2half_rn(__fmul_rn(xs[e], s_inv[m]));
      xs[e] = __half2float(__hmul_rn(norm_w[k], nrm));
    }
    __syncthreads();
  }

  // ---- this CTA's vocabulary rows [r0, r1), two rows per warp at a time
  const int G = gridDim.x;
  const int r0 = static_cast<int>(static_cast<int64_t>(V) * blockIdx.x / G);
  const int r1 = static_cast<int>(static_cast<int64_t>(V) * (blockIdx.x + 1) / G);
  float bv[MR];
  int bi[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    bv[m] = -INFINITY;
    bi[m] = 0x7fffffff;
  }
  for (int r = r0 + warp; r < r1; r += HeadShape<MR>::rows * kHeadWarps) {
    // rows r + i * kHeadWarps (i < HeadShape<MR>::rows) of this round; absent rows re-read row r
    const uint4* wr[HeadShape<MR>::rows];
    float acc[HeadShape<MR>::rows][MR];
#pragma unroll
    for (int i = 0; i < HeadShape<MR>::rows; ++i) {
      const int row = r + i * kHeadWarps;
      wr[i] = reinterpret_cast<const uint4*>(W + static_cast<int64_t>(row < r1 ? row : r) * H);
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[i][m] = 0.f;
    }
    for (int v0 = lane; v0 < nv; v0 += 32 * HeadShape<MR>::unroll) {
      uint4 q[HeadShape<MR>::rows][HeadShape<MR>::unroll];
#pragma unroll
      for (int u = 0; u < HeadShape<MR>::unroll; ++u)
#pragma unroll
        for (int i = 0; i < HeadShape<MR>::rows; ++i)
          if (v0 + 32 * u < nv) q[i][u] = __ldcs(wr[i] + v0 + 32 * u);  // streamed once: evict first
#pragma unroll
      for (int u = 0; u < HeadShape<MR>::unroll; ++u) {
        const int v = v0 + 32 * u;
        if (v >= nv) break;
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m >= M) break;
          const float4 x0 = *reinterpret_cast<const float4*>(xs + m * H + 8 * v);
          const float4 x1 = *reinterpret_cast<const float4*>(xs + m * H + 8 * v + 4);
#pragma unroll
          for (int i = 0; i < HeadShape<MR>::rows; ++i) {
            const __half2* hq = reinterpret_cast<const __half2*>(&q[i][u]);
            const float2 f0 = __half22float2(hq[0]), f1 = __half22float2(hq[1]);
            const float2 f2 = __half22float2(hq[2]), f3 = __half22float2(hq[3]);
            float a = acc[i][m];
            a = fmaf(f0.x, x0.x, a);
            a = fmaf(f0.y, x0.y, a);
            a = fmaf(f1.x, x0.z, a);
            a = fmaf(f1.y, x0.w, a);
            a = fmaf(f2.x, x1.x, a);
            a = fmaf(f2.y, x1.y, a);
            a = fmaf(f3.x, x1.z, a);
            a = fmaf(f3.y, x1.w, a);
            acc[i][m] = a;
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < HeadShape<MR>::rows; ++i) {
      const int row = r + i * kHeadWarps;
      if (row >= r1) break;
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        if (m >= M) break;
        float a = acc[i][m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        const __half l = __float2half_rn(a);
        head_better(bv[m], bi[m], __half2float(l), row);
        if (logits != nullptr && lane == m) logits[static_cast<int64_t>(m) * V + row] = l;
      }
    }
  }

  // ---- this CTA's best per row, then the grid's by the last CTA to arrive
  if (lane == 0)
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      s_bv[warp][m] = bv[m];
      s_bi[warp][m] = bi[m];
    }
  __syncthreads();
  if (tid < M) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int w = 0; w < kHeadWarps; ++w) head_better(v, i, s_bv[w][tid], s_bi[w][tid]);
    ws.best_v[blockIdx.x * kHeadMaxRows + tid] = v;
    ws.best_i[blockIdx.x * kHeadMaxRows + tid] = i;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();  // this CTA's bests before its arrival
    const unsigned prev = atomicAdd(ws.counter, 1u);
    s_last = prev == static_cast<unsigned>(G - 1);
    if (s_last) __threadfence();  // every other CTA's bests after their arrivals
  }
  __syncthreads();
  if (!s_last) return;
  if (tid == 0) {  // the history column: a position outside it writes no history and keeps *pos
    int ok = 1;
    if (hist != nullptr) {
      const int64_t p = *pos;
      ok = p >= 0 && p < hist_len;
      if (!ok) record_device_error(err, DK_DEVERR_BAD_POSITION);
    }
    s_last = ok ? 1 : 2;
  }
  __syncthreads();
  const bool pos_ok = s_last == 1;
  // one warp per row reduces the CTAs' bests (max, ties to the lowest index: order-independent)
  for (int m = warp; m < M; m += kHeadWarps) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int q = lane; q < G; q += 32) head_better(v, i, __ldcg(ws.best_v + q * kHeadMaxRows + m), __ldcg(ws.best_i + q * kHeadMaxRows + m));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      head_better(v, i, ov, oi);
    }
    if (lane == 0) {
      if (i == 0x7fffffff) i = 0;  // only if every logit was NaN
      tokens[m] = i;
      if (hist != nullptr && pos_ok) hist[m * hist_ld + *pos] = i;
    }
  }
  __syncthreads();
  if (tid == 0) {
    if (pos != nullptr && pos_ok) *pos += 1;
    *ws.counter = 0;  // ready for the next launch (launches on one workspace are stream-ordered)
  }
}

// out[m] = embed[tokens[m]] (a token outside [0, V) records DK_DEVERR_BAD_TOKEN and takes row 0)
__global__ void embed_rows_kernel(const int64_t* __restrict__ tokens, const __half* __restrict__ embed, int V,
                                  int H, __half* __restrict__ out, int* err) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.y;
  int64_t t = tokens[m];
  if (t < 0 || t >= V) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_device_error(err, DK_DEVERR_BAD_TOKEN);
    t = 0;
  }
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v < H / 8)
    reinterpret_cast<uint4*>(out + static_cast<int64_t>(m) * H)[v] =
        __ldg(reinterpret_cast<const uint4*>(embed + t * H) + v);
}

int head_grid() { return device_info().num_sms * kHeadCtasPerSm; }

template <int MR>
cudaError_t launch_head(size_t smem, cudaStream_t st, const __half* x, const __half* res, const __half* nw, float eps,
                        const __half* W, int V, int H, int M, int64_t* tokens, int64_t* pos, int64_t* hist,
                        int64_t hist_ld, int64_t hist_len, __half* logits, HeadWs ws) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {  // opt in to the largest dynamic size next to the static arrays
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, head_greedy_kernel<MR>);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(head_greedy_kernel<MR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               device_info().max_smem_optin - static_cast<int>(fa.sharedSizeBytes));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  return launch(head_greedy_kernel<MR>, dim3(head_grid()), dim3(kHeadThreads), smem, st, pdl_enabled(),
                dim3(1, 1, 1), x, res, nw, eps, W, V, H, M, tokens, pos, hist, hist_ld, hist_len, logits, ws,
                device_info().err_word);
}

}  // namespace
}  // namespace dk

using namespace dk;

extern "C" int dk_lm_head_greedy_workspace_bytes(uint64_t* bytes) {
  if (bytes == nullptr) return set_error(DK_ERR_INVALID, "lm_head_greedy: bytes is NULL");
  *bytes = 256 + static_cast<uint64_t>(head_grid()) * kHeadMaxRows * 8;
  return DK_OK;
}

extern "C" int dk_lm_head_greedy(const void* x, const void* residual, const void* norm_weight, float eps,
                                 const void* lm_head, int64_t vocab, int64_t hidden, int64_t M, int64_t* tokens,
                                 int64_t* pos, int64_t* history, int64_t history_ld, int64_t history_len,
                                 void* logits, void* workspace, uint64_t workspace_bytes, dk_stream_t stream) {
  if (M <= 0 || M > kHeadMaxRows) return set_error(DK_ERR_UNSUPPORTED, "lm_head_greedy: %lld rows (1..%d)", (long long)M, kHeadMaxRows);
  if (vocab <= 0 || hidden <= 0 || vocab > INT32_MAX / 2 || hidden > (1 << 16))
    return set_error(DK_ERR_INVALID, "lm_head_greedy: vocab %lld, hidden %lld out of range", (long long)vocab, (long long)hidden);
  if (hidden % 8) return set_error(DK_ERR_UNSUPPORTED, "lm_head_greedy: hidden %% 8 != 0");
  if (!x || !lm_head || !tokens || !workspace) return set_error(DK_ERR_INVALID, "lm_head_greedy: NULL pointer");
  if (history && (!pos || history_ld < history_len || history_len <= 0))
    return set_error(DK_ERR_INVALID, "lm_head_greedy: history needs pos and history_ld >= history_len > 0");
  if (!aligned16(x) || !aligned16(lm_head) || (residual && !aligned16(residual)) || (norm_weight && !aligned16(norm_weight)))
    return set_error(DK_ERR_ALIGN, "lm_head_greedy: x, residual, norm weight and lm_head must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(DK_ERR_ALIGN, "lm_head_greedy: workspace must be 256-byte aligned");
  uint64_t need = 0;
  dk_lm_head_greedy_workspace_bytes(&need);
  if (workspace_bytes < need)
    return set_error(DK_ERR_INVALID, "lm_head_greedy: workspace of %llu bytes, %llu needed", (unsigned long long)workspace_bytes,
                     (unsigned long long)need);
  const int mr = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  const size_t smem = static_cast<size_t>(mr) * hidden * 4;
  if (smem > static_cast<size_t>(device_info().max_smem_optin) - 2048)
    return set_error(DK_ERR_UNSUPPORTED, "lm_head_greedy: %lld rows of %lld values do not fit in shared memory", (long long)M,
                     (long long)hidden);
  char* w = static_cast<char*>(workspace);
  HeadWs ws;
  ws.counter = reinterpret_cast<unsigned*>(w);
  ws.best_v = reinterpret_cast<float*>(w + 256);
  ws.best_i = reinterpret_cast<int*>(w + 256 + static_cast<size_t>(head_grid()) * kHeadMaxRows * 4);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const auto* xr = static_cast<const __half*>(x);
  const auto* rr = static_cast<const __half*>(residual);
  const auto* nw = static_cast<const __half*>(norm_weight);
  const auto* W = static_cast<const __half*>(lm_head);
  auto* lg = static_cast<__half*>(logits);
  const int V = static_cast<int>(vocab), H = static_cast<int>(hidden), m = static_cast<int>(M);
  cudaError_t e;
  switch (mr) {
    case 1: e = launch_head<1>(smem, st, xr, rr, nw, eps, W, V, H, m, tokens, pos, history, history_ld, history_len, lg, ws); break;
    case 2: e = launch_head<2>(smem, st, xr, rr, nw, eps, W, V, H, m, tokens, pos, history, history_ld, history_len, lg, ws); break;
    case 4: e = launch_head<4>(smem, st, xr, rr, nw, eps, W, V, H, m, tokens, pos, history, history_ld, history_len, lg, ws); break;
    default: e = launch_head<8>(smem, st, xr, rr, nw, eps, W, V, H, m, tokens, pos, history, history_ld, history_len, lg, ws); break;
  }
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "lm_head_greedy launch: %s", cudaGetErrorString(e));
  return DK_OK;
}

extern "C" int dk_embed_tokens(const int64_t* tokens, const void* embed, int64_t vocab, int64_t hidden, int64_t M,
                               void* out, dk_stream_t stream) {
  if (M < 0 || vocab <= 0 || hidden <= 0 || M > 65535 || vocab > INT32_MAX || hidden > INT32_MAX)
    return set_error(DK_ERR_INVALID, "embed_tokens: size out of range");
  if (M == 0) return DK_OK;
  if (hidden % 8) return set_error(DK_ERR_UNSUPPORTED, "embed_tokens: hidden %% 8 != 0");
  if (!tokens || !embed || !out) return set_error(DK_ERR_INVALID, "embed_tokens: NULL pointer");
  if (!aligned16(embed) || !aligned16(out)) return set_error(DK_ERR_ALIGN, "embed_tokens: embed and out must be 16-byte aligned");
  const int threads = 128;
  const dim3 grid(static_cast<unsigned>((hidden / 8 + threads - 1) / threads), static_cast<unsigned>(M));
  const cudaError_t e = launch(embed_rows_kernel, grid, dim3(threads), 0, reinterpret_cast<cudaStream_t>(stream),
                               pdl_enabled(), dim3(1, 1, 1), tokens, static_cast<const __half*>(embed),
                               static_cast<int>(vocab), static_cast<int>(hidden), static_cast<__half*>(out),
                               device_info().err_word);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "embed_tokens launch: %s", cudaGetErrorString(e));
  return DK_OK;
}
