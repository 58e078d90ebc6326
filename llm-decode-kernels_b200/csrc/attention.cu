// Decode attention for one new token per sequence: RoPE on q and k, KV-cache append, and softmax
// attention over the cached positions 0..pos only.
//
// Replaces, for T == 1, the reference runner's per-layer sequence (kernels/e2e/model.py:236-244):
//   q, k = rope(q), rope(k)            x * cos + cat(-x2, x1) * sin, fp16 rounding after each op
//   k_cache[:, :, pos] = k ; v_cache[:, :, pos] = v
//   attn = SDPA(q, k_cache, v_cache, mask = keys <= pos, enable_gqa=True)
// The reference's SDPA reads all `max_len` cached positions every step and masks most of them; this
// kernel reads positions 0..pos. Scores, softmax and the weighted sum of V are fp32.
//
// Grid (n_kv, B, S) with the S CTAs of one (kv head, sequence) forming a thread-block cluster
// ("split-KV"): each CTA covers a contiguous slice of the positions, keeps its softmax partials
// (max, sum, unnormalized output) in shared memory, and the cluster combines them through
// distributed shared memory. The CTA whose slice holds `pos` takes the new token's k, v from
// registers and writes them to the cache; no other CTA reads position `pos`, so no ordering between
// CTAs is needed. `pos` is read on the device, so the launch can be captured in a CUDA graph once and
// replayed for every step.
#include <algorithm>
#include <cfloat>

#include "common.cuh"

namespace dk {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxGroup = 8;  // query heads per kv head
constexpr int kMaxSplit = 16;  // cluster of up to 16 CTAs (non-portable size, allowed on B200)

struct AttnParams {
  const __half* qkv;  // [B, (nq + 2 nkv) * hd]
  __half* k_cache;    // [B, nkv, max_len, hd]
  __half* v_cache;
  const int64_t* pos;  // [1]
  const __half* cos;   // [hd], or a table [positions, hd] when rope_stride > 0
  const __half* sin;
  int64_t rope_stride;  // > 0: cos/sin rows are selected by *pos
  __half* out;         // [B, nq * hd]
  int nq, nkv, max_len;
  int slice_max;     // positions per CTA at most, a multiple of 16 (sizes the shared-memory slices)
  int static_cache;  // see DK_ATTN_STATIC_CACHE
  float scale;
  int* err;
};

// RoPE for element d of one head, with the reference's fp16 rounding:
// x*cos + rot*sin, rot = -x[d+hd/2] (d < hd/2) or x[d-hd/2] (d >= hd/2).
template <int kHd>
__device__ __forceinline__ __half rope_elem(const __half* x, int d, const __half* cs, const __half* sn) {
  const __half rot = d < kHd / 2 ? __hneg(x[d + kHd / 2]) : x[d - kHd / 2];
  return __hadd_rn(__hmul_rn(x[d], cs[d]), __hmul_rn(rot, sn[d]));
}

// kHd / 32 consecutive fp16 values of a cache row for one lane, as fp32.
template <int E>
__device__ __forceinline__ void load_lane(const __half* row, int lane, float (&v)[E]) {
  if constexpr (E == 4) {
    const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(row) + lane);
    const __half* h = reinterpret_cast<const __half*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = __half2float(h[e]);
  } else if constexpr (E == 2) {
    const unsigned raw = __ldcg(reinterpret_cast<const unsigned*>(row) + lane);
    const __half* h = reinterpret_cast<const __half*>(&raw);
    v[0] = __half2float(h[0]);
    v[1] = __half2float(h[1]);
  } else {
    v[0] = __half2float(__ldcg(row + lane));
  }
}

template <int G, int kHd>
__global__ void __launch_bounds__(kThreads, 1) decode_attention_kernel(const AttnParams p) {
  static_assert(G <= 8, "query heads per kv head");
  __shared__ __align__(16) __half qs[8][kHd];  // rotated q, fp16 (rows G..7 zero: MMA padding)
  __shared__ __half knew[kHd], vnew[kHd];
  __shared__ float part_o[G][kHd];  // this CTA's unnormalized output
  __shared__ float part_m[G], part_l[G];
  // split-K combine, pushed by every rank of the cluster: softmax max / sum per head and the
  // unnormalized output of the dims this rank owns
  __shared__ float recv_ml[kMaxSplit][2][G];
  __shared__ float recv_o[G * (kHd + kMaxSplit)];
  __shared__ __align__(8) uint64_t bar;
  extern __shared__ __align__(128) uint8_t dsm[];  // Ks[slice][hd] | Vs[slice][hd] | scores[G][slice]

  const int h = blockIdx.x, b = blockIdx.y, rank = blockIdx.z, S = gridDim.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  // With a static cache the rows before `pos` and `pos` itself were written by kernels that
  // finished before the previous one started, so the slice can be fetched before waiting.
  if (!p.static_cache) pdl_wait();
  const int64_t pos64 = *p.pos;
  if (pos64 < 0 || pos64 >= p.max_len) {  // same decision in every CTA of the cluster
    if (p.static_cache) pdl_wait();
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
      record_device_error(p.err, DK_DEVERR_BAD_POSITION);
    return;
  }
  const int L = static_cast<int>(pos64) + 1;  // positions 0..pos
  const int slice = (L + S - 1) / S;
  const int j0 = min(rank * slice, L), j1 = min(j0 + slice, L);
  const int n = j1 - j0;
  const int pos = L - 1;
  const int64_t cache_base = (static_cast<int64_t>(b) * p.nkv + h) * p.max_len * kHd;
  __half* kc = p.k_cache + cache_base;
  __half* vc = p.v_cache + cache_base;
  __half* Ks = reinterpret_cast<__half*>(dsm);
  __half* Vs = Ks + static_cast<size_t>(p.slice_max) * kHd;
  float* scores = reinterpret_cast<float*>(Vs + static_cast<size_t>(p.slice_max) * kHd);
  if (tid == 0 && n > 0) {
    const uint32_t bytes = static_cast<uint32_t>(n) * kHd * 2;
    mbar_arrive_expect_tx(&bar, 2 * bytes);
    bulk_g2s(Ks, kc + static_cast<int64_t>(j0) * kHd, bytes, &bar);
    bulk_g2s(Vs, vc + static_cast<int64_t>(j0) * kHd, bytes, &bar);
  }
  if (p.static_cache) pdl_wait();  // qkv comes from the previous kernel

  const __half* cosr = p.cos + (p.rope_stride > 0 ? pos64 * p.rope_stride : 0);
  const __half* sinr = p.sin + (p.rope_stride > 0 ? pos64 * p.rope_stride : 0);
  const int row = (p.nq + 2 * p.nkv) * kHd;
  const __half* qrow = p.qkv + static_cast<int64_t>(b) * row;
  const __half* krow = qrow + p.nq * kHd + h * kHd;
  const __half* vrow = qrow + (p.nq + p.nkv) * kHd + h * kHd;
  for (int d = tid; d < kHd; d += kThreads) {
#pragma unroll
    for (int g = 0; g < 8; ++g)
      qs[g][d] = g < G ? rope_elem<kHd>(qrow + (h * G + g) * kHd, d, cosr, sinr) : __float2half(0.f);
    knew[d] = rope_elem<kHd>(krow, d, cosr, sinr);
    vnew[d] = vrow[d];
  }
  __syncthreads();
  const bool owner = pos >= j0 && pos < j1;
  if (owner) {  // append the new token to the cache
    for (int d = tid; d < kHd; d += kThreads) {
      kc[static_cast<int64_t>(pos) * kHd + d] = knew[d];
      vc[static_cast<int64_t>(pos) * kHd + d] = vnew[d];
    }
  }
  bool ok = true;
  if (n > 0) ok = mbar_wait(&bar, 0, p.err, DK_DEVERR_WAIT_FULL);
  if (__syncthreads_or(!ok)) {
    if (S > 1) cluster_sync();  // the one cluster barrier the other ranks pass as well
    return;
  }
  if (owner) {  // the slice copy holds the stale row at `pos`: replace it with the new k, v
    for (int d = tid; d < kHd; d += kThreads) {
      Ks[static_cast<size_t>(pos - j0) * kHd + d] = knew[d];
      Vs[static_cast<size_t>(pos - j0) * kHd + d] = vnew[d];
    }
  }
  __syncthreads();

  // scores[g][j] = (q_g . k_j) * scale on tensor cores: A = q (8 heads padded to 16 rows) x 16 dims,
  // B = K^T (16 dims x 8 positions), fp32 accumulation; warp w takes position tiles w, w+4, ...
  {
    const int g = lane >> 2, t = lane & 3;
    const int ntiles = (n + 7) / 8;
    for (int nt = warp; nt < ntiles; nt += kThreads / 32) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int prow = min(nt * 8 + g, max(n - 1, 0));  // clamp: padded columns read a valid row
      const __half* krow_s = Ks + static_cast<size_t>(prow) * kHd;
#pragma unroll
      for (int k0 = 0; k0 < kHd; k0 += 16) {
        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&qs[g][k0 + 2 * t]);
        const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&qs[g][k0 + 2 * t + 8]);
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow_s + k0 + 2 * t);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow_s + k0 + 2 * t + 8);
        mma_16816(acc, a0, 0u, a2, 0u, b0, b1);
      }
      if (g < G) {
        const int jj = nt * 8 + 2 * t;
        if (jj < n) scores[g * p.slice_max + jj] = acc[0] * p.scale;
        if (jj + 1 < n) scores[g * p.slice_max + jj + 1] = acc[1] * p.scale;
      }
    }
  }
  __syncthreads();
  // softmax partials per head (warp w handles heads w, w+4, ...)
  for (int g = warp; g < G; g += kThreads / 32) {
    float m = -FLT_MAX;
    for (int jj = lane; jj < n; jj += 32) m = fmaxf(m, scores[g * p.slice_max + jj]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int jj = lane; jj < n; jj += 32) {
      const float e = __expf(scores[g * p.slice_max + jj] - m);
      scores[g * p.slice_max + jj] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      part_m[g] = m;
      part_l[g] = l;
    }
  }
  __syncthreads();
  // unnormalized output O = P V on tensor cores: A = P (fp16, heads padded to 16 rows) x 16
  // positions, B = V (16 positions x 8 dims, ldmatrix.trans from the row-major slice); rows of the
  // last 16-position step beyond n are zero in both P and V.
  {
    const int kpad = (n + 15) / 16 * 16;
    for (int i = n * kHd + tid * 8; i < kpad * kHd; i += kThreads * 8)
      *reinterpret_cast<uint4*>(Vs + i) = make_uint4(0, 0, 0, 0);
    __syncthreads();
    const int g = lane >> 2, t = lane & 3;
    constexpr int kTiles = kHd / 8;  // 8-dim output tiles, two per ldmatrix.x4
    for (int tp = warp; tp < kTiles / 2; tp += kThreads / 32) {
      const int nb = tp * 16;
      float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
      for (int k0 = 0; k0 < kpad; k0 += 16) {
        uint32_t a0 = 0, a2 = 0;
        if (g < G) {
          const float* sr = scores + g * p.slice_max;
          const int j = k0 + 2 * t;
          const float p0 = j < n ? sr[j] : 0.f, p1 = j + 1 < n ? sr[j + 1] : 0.f;
          const float p8 = j + 8 < n ? sr[j + 8] : 0.f, p9 = j + 9 < n ? sr[j + 9] : 0.f;
          a0 = half2_bits(__float2half_rn(p0), __float2half_rn(p1));
          a2 = half2_bits(__float2half_rn(p8), __float2half_rn(p9));
        }
        // lane i addresses row (i % 8) of 8x8 tile (i / 8): tiles (k lo, d lo), (k hi, d lo),
        // (k lo, d hi), (k hi, d hi)
        const int tl = lane >> 3, r = lane & 7;
        const __half* src = Vs + static_cast<size_t>(k0 + (tl & 1) * 8 + r) * kHd + nb + (tl >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3)
                     : "r"(smem_addr(src)));
        mma_16816(acc0, a0, 0u, a2, 0u, b0, b1);
        mma_16816(acc1, a0, 0u, a2, 0u, b2, b3);
      }
      if (g < G) {
        part_o[g][nb + 2 * t] = acc0[0];
        part_o[g][nb + 2 * t + 1] = acc0[1];
        part_o[g][nb + 8 + 2 * t] = acc1[0];
        part_o[g][nb + 8 + 2 * t + 1] = acc1[1];
      }
    }
  }

  if (S == 1) {
    __syncthreads();
    for (int e = tid; e < G * kHd; e += kThreads) {
      const int g = e / kHd, d = e % kHd;
      p.out[static_cast<int64_t>(b) * p.nq * kHd + (h * G + g) * kHd + d] = __float2half_rn(part_o[g][d] / part_l[g]);
    }
    return;
  }
  // combine the S partials of the cluster: rank q owns dims [q*D, (q+1)*D); every rank pushes its
  // (max, sum) per head and its partial output of rank q's dims into rank q's shared memory
  // (remote stores, no round trips), one cluster barrier publishes them, and each rank combines
  // its own dims from local shared memory.
  __syncthreads();
  const int D = (kHd + S - 1) / S;
  for (int e = tid; e < S * G * D; e += kThreads) {
    const int q = e / (G * D), g = (e / D) % G, dd = e % D;
    const int d = q * D + dd;
    if (d < kHd) st_shared_cluster_f32(map_shared_rank(&recv_o[(rank * G + g) * D + dd], q), part_o[g][d]);
  }
  for (int e = tid; e < S * G; e += kThreads) {
    const int q = e / G, g = e % G;
    st_shared_cluster_f32(map_shared_rank(&recv_ml[rank][0][g], q), part_m[g]);
    st_shared_cluster_f32(map_shared_rank(&recv_ml[rank][1][g], q), part_l[g]);
  }
  cluster_sync();
  for (int e = tid; e < G * D; e += kThreads) {
    const int g = e / D, dd = e % D;
    const int d = rank * D + dd;
    if (d >= kHd) continue;
    float M = -FLT_MAX;
    for (int q = 0; q < S; ++q)
      if (recv_ml[q][1][g] > 0.f) M = fmaxf(M, recv_ml[q][0][g]);
    float num = 0.f, den = 0.f;
    for (int q = 0; q < S; ++q) {
      const float l = recv_ml[q][1][g];
      if (l <= 0.f) continue;
      const float w = __expf(recv_ml[q][0][g] - M);
      num = fmaf(w, recv_o[(q * G + g) * D + dd], num);
      den = fmaf(w, l, den);
    }
    p.out[static_cast<int64_t>(b) * p.nq * kHd + (h * G + g) * kHd + d] = __float2half_rn(num / den);
  }
}

}  // namespace
}  // namespace dk

using namespace dk;

extern "C" int dk_decode_attention(const void* qkv, void* k_cache, void* v_cache, const int64_t* pos,
                                   const void* cos, const void* sin, void* out, int64_t B, int64_t nq,
                                   int64_t nkv, int64_t head_dim, int64_t max_len, int64_t rope_stride,
                                   int32_t splits, int32_t flags, dk_stream_t stream) {
  if (B <= 0 || nq <= 0 || nkv <= 0 || max_len <= 0) return set_error(DK_ERR_INVALID, "decode_attention: bad sizes");
  if (head_dim != 32 && head_dim != 64 && head_dim != 128)
    return set_error(DK_ERR_UNSUPPORTED, "decode_attention: head_dim %lld (32, 64 or 128)", (long long)head_dim);
  if (nq % nkv != 0 || nq / nkv > kMaxGroup)
    return set_error(DK_ERR_UNSUPPORTED, "decode_attention: %lld query heads per kv head (max %d)",
                     (long long)(nq / nkv), kMaxGroup);
  if (B > 65535 || nkv > 65535) return set_error(DK_ERR_INVALID, "decode_attention: grid too large");
  if (!qkv || !k_cache || !v_cache || !pos || !cos || !sin || !out)
    return set_error(DK_ERR_INVALID, "decode_attention: NULL pointer");
  int S = splits > 0 ? splits : static_cast<int>(std::min<int64_t>(kMaxSplit, (max_len + 127) / 128));
  S = std::max(1, std::min(S, kMaxSplit));
  AttnParams p;
  p.qkv = static_cast<const __half*>(qkv);
  p.k_cache = static_cast<__half*>(k_cache);
  p.v_cache = static_cast<__half*>(v_cache);
  p.pos = pos;
  p.cos = static_cast<const __half*>(cos);
  p.sin = static_cast<const __half*>(sin);
  p.rope_stride = rope_stride;
  p.out = static_cast<__half*>(out);
  p.nq = static_cast<int>(nq);
  p.nkv = static_cast<int>(nkv);
  p.max_len = static_cast<int>(max_len);
  p.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
  p.err = device_info().err_word;
  const int G = static_cast<int>(nq / nkv);
  // rows per CTA slice, rounded up to the 16-position MMA step (the P V loop reads whole steps)
  const int slice_max = static_cast<int>(((max_len + S - 1) / S + 15) / 16 * 16);
  p.slice_max = slice_max;
  p.static_cache = (flags & DK_ATTN_STATIC_CACHE) ? 1 : 0;
  const size_t smem = 2 * static_cast<size_t>(slice_max) * head_dim * 2 + static_cast<size_t>(G) * slice_max * 4;
  if (smem > static_cast<size_t>(device_info().max_smem_optin) - 8 * 1024)
    return set_error(DK_ERR_UNSUPPORTED, "decode_attention: max_len %lld needs more shared memory per CTA than "
                     "the device has (use more splits)", (long long)max_len);
  const dim3 grid(static_cast<unsigned>(nkv), static_cast<unsigned>(B), static_cast<unsigned>(S));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
#define DK_ATTN(GG)                                                                                      \
  case GG: {                                                                                             \
    auto k = head_dim == 128 ? decode_attention_kernel<GG, 128>                                          \
             : head_dim == 64 ? decode_attention_kernel<GG, 64> : decode_attention_kernel<GG, 32>;       \
    cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);                             \
    if (opt_in_dynamic_smem(k) < static_cast<int>(smem))                                                   \
      return set_error(DK_ERR_UNSUPPORTED, "decode_attention: %zu bytes of shared memory do not fit", smem); \
    e = launch(k, grid, dim3(kThreads), smem, st, pdl_enabled(), dim3(1, 1, S), p);                       \
    break;                                                                                               \
  }
  switch (G) {
    DK_ATTN(1)
    DK_ATTN(2)
    DK_ATTN(4)
    DK_ATTN(6)
    DK_ATTN(7)
    DK_ATTN(8)
    default:
      return set_error(DK_ERR_UNSUPPORTED, "decode_attention: group size %d", G);
  }
#undef DK_ATTN
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "decode_attention launch: %s", cudaGetErrorString(e));
  return DK_OK;
}
