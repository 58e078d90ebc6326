// Decode attention for one new token per sequence: RoPE on q and k, KV-cache append, and softmax
// attention over the cached positions 0..pos only.
//
// Replaces, for T == 1, the reference runner's per-layer sequence (kernels/e2e/model.py:236-244):
//   q, k = rope(q), rope(k)            x * cos + cat(-x2, x1) * sin, fp16 rounding after each op
//   k_cache[:, :, pos] = k ; v_cache[:, :, pos] = v
//   attn = SDPA(q, k_cache, v_cache, mask = keys <= pos, enable_gqa=True)
// The reference's SDPA reads all `max_len` cached positions every step and masks most of them; this
// kernel reads positions 0..pos. Scores, softmax and the weighted sum of V are fp32 (P is rounded
// to fp16 for the tensor-core P.V product, as flash-style SDPA does on fp16 inputs).
//
// Layout of the work. Grid (n_kv, B, S): the S CTAs of one (kv head, sequence) form a thread-block
// cluster and split the positions 0..pos into contiguous slices ("split-KV"). In each CTA:
// * a producer warp streams the slice's K and V rows into a shared-memory ring of 64-position chunks
//   with 2-D TMA (128-byte swizzle, so the tensor-core operand reads below hit 32 different banks);
//   with a static cache it starts before waiting for the previous kernel;
// * four consumer warps each own one 16-position block of every chunk and run flash decoding on it:
//   q.K^T on tensor cores (heads as MMA rows, K rows by ldmatrix), an online softmax in registers,
//   and P.V on tensor cores with P taken straight from the score accumulators (no shared-memory
//   round trip) and V rows by ldmatrix.trans. The new token's k and v never go through the ring:
//   the lane that addresses cache row `pos` points ldmatrix at the freshly rotated row instead, and
//   rows past the slice end read a zero row, so no shared-memory patching or zero-filling is needed;
// * the four warps' (max, sum, unnormalized output) are combined into the CTA's partial in shared
//   memory. Rank q of the cluster owns output dims [q*D, (q+1)*D), D = head_dim / S; the CTA pushes
//   the slices of its partial straight into the owners' shared memory with st.async (completion
//   counted by the owner's mbarrier, so only the receiver waits), and each owner combines its dims
//   over the S partials (a half-warp per head).
// `pos` is read on the device, so the launch can be captured in a CUDA graph once and replayed for
// every step.
#include <algorithm>
#include <cfloat>

#include "common.cuh"

namespace dk {
namespace {

constexpr int kCWarps = 4;                    // consumer warps
constexpr int kThreads = (kCWarps + 1) * 32;  // + one TMA producer warp
constexpr int kChunk = 64;                    // cache positions per ring slot: one 16-row block per consumer warp
constexpr int kMaxRing = 4;
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
  __half* out;          // [B, nq * hd]
  int nq, nkv, max_len;
  int ring;          // chunk slots in shared memory
  int static_cache;  // see DK_ATTN_STATIC_CACHE
  float scale;
  int* err;
};

// One chunk of K (or V) in shared memory: kSegs TMA boxes of kChunk rows x kSegHalves dims, rows of
// 128 bytes with the 128-byte swizzle (64 bytes and the 64-byte swizzle when head_dim is 32).
template <int kHd>
struct Chunk {
  static constexpr int kSegHalves = kHd < 64 ? kHd : 64;
  static constexpr int kRowBytes = kSegHalves * 2;
  static constexpr int kSegs = kHd / kSegHalves;
  static constexpr int kSegBytes = kChunk * kRowBytes;
  static constexpr int kTensorBytes = kSegs * kSegBytes;
  static constexpr int kSlotBytes = 2 * kTensorBytes;  // K then V

  // The 16 bytes that hold dims d..d+7 (d % 8 == 0) of row r: the TMA swizzle XORs the 16-byte
  // chunk index with the row index (mod 8, or (row / 2) mod 4 for 64-byte rows).
  __device__ static const uint8_t* at(const uint8_t* t, int r, int d) {
    const int b = (d % kSegHalves) * 2;
    uint32_t off;
    if constexpr (kRowBytes == 128)
      off = r * 128 + ((((b >> 4) ^ r) & 7) << 4);
    else
      off = r * 64 + ((((b >> 4) ^ (r >> 1)) & 3) << 4);
    return t + (d / kSegHalves) * kSegBytes + off;
  }
};

// RoPE of 4 consecutive dims and their partners half a head away, with the reference's fp16
// rounding: lo' = lo*c_lo - hi*s_lo, hi' = hi*c_hi + lo*s_hi (rotate_half(x) = cat(-x2, x1)).
__device__ __forceinline__ void rope4(uint2 lo, uint2 hi, uint2 c_lo, uint2 c_hi, uint2 s_lo, uint2 s_hi,
                                      uint2& out_lo, uint2& out_hi) {
  const __half* xl = reinterpret_cast<const __half*>(&lo);
  const __half* xh = reinterpret_cast<const __half*>(&hi);
  const __half* cl = reinterpret_cast<const __half*>(&c_lo);
  const __half* ch = reinterpret_cast<const __half*>(&c_hi);
  const __half* sl = reinterpret_cast<const __half*>(&s_lo);
  const __half* sh = reinterpret_cast<const __half*>(&s_hi);
  __half* ol = reinterpret_cast<__half*>(&out_lo);
  __half* oh = reinterpret_cast<__half*>(&out_hi);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    ol[i] = __hadd_rn(__hmul_rn(xl[i], cl[i]), __hmul_rn(__hneg(xh[i]), sl[i]));
    oh[i] = __hadd_rn(__hmul_rn(xh[i], ch[i]), __hmul_rn(xl[i], sh[i]));
  }
}

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kCWarps * 32) : "memory");
}

template <int G, int kHd>
__global__ void __launch_bounds__(kThreads, 1)
    decode_attention_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv,
                            const AttnParams p) {
  static_assert(G <= kMaxGroup, "query heads per kv head");
  using CH = Chunk<kHd>;
  constexpr int kQuads = kHd / 8;  // RoPE: 4-dim groups in half a head
  constexpr int kTiles = kHd / 8;  // 8-dim output tiles
  __shared__ __align__(16) __half qs[G][kHd + 8];  // rotated q; +8 halves: conflict-free fragment reads
  __shared__ __align__(16) __half knew[kHd], vnew[kHd];
  __shared__ __align__(16) __half vzero[8];
  __shared__ __align__(16) float pre_o[kCWarps * G * kHd];    // this CTA's warps' outputs [warp][head][dim]
  __shared__ float pre_ml[kCWarps * G * 2];                   // [warp][head] {max, sum}
  __shared__ float pre_w[kCWarps * G];                        // [warp][head] weight in the CTA's partial
  __shared__ float cml[G * 2];                                // the CTA's partial per head {max, sum}
  __shared__ __align__(16) float recv_o[G * kHd];             // [rank][head][D] (S partials x D = hd)
  __shared__ __align__(16) float recv_ml[kMaxSplit * G * 2];  // [rank][head] {max, sum}
  __shared__ float wts[kMaxSplit * G];
  __shared__ float den[G];
  __shared__ __align__(8) uint64_t full[kMaxRing], empty[kMaxRing], recv;
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  uint8_t* ring = dsm_raw + ((1024u - (smem_addr(dsm_raw) & 1023u)) & 1023u);  // swizzle atoms: 1 KB aligned

  const int h = blockIdx.x, b = blockIdx.y, rank = blockIdx.z, S = gridDim.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nparts = S;  // one partial per cluster rank (its 4 warps combined first)
  const int D = kHd / S;  // output dims this rank combines (S is a power of two <= head_dim / 2)

  if (tid == 0) {
    for (int i = 0; i < p.ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCWarps);
    }
    mbar_init(&recv, 1);
    if (S > 1) mbar_arrive_expect_tx(&recv, static_cast<uint32_t>(nparts * G * (D + 2) * 4));
    fence_mbar_init();
  }
  if (tid < 8) vzero[tid] = __float2half(0.f);
  __syncthreads();
  if (S > 1) cluster_arrive_relaxed();  // (1) every CTA's mbarriers exist before anyone pushes
  pdl_trigger();

  // With a static cache the rows before `pos` and `pos` itself were written by kernels that
  // finished before the previous one started, so the slice can be fetched before waiting.
  if (!p.static_cache) pdl_wait();
  const int64_t pos64 = *p.pos;
  if (pos64 < 0 || pos64 >= p.max_len) {  // same decision in every CTA of the cluster
    if (p.static_cache) pdl_wait();
    if (tid == 0 && blockIdx.x == 0 && blockIdx.y == 0 && rank == 0)
      record_device_error(p.err, DK_DEVERR_BAD_POSITION);
    __syncwarp();
    if (S > 1) cluster_wait();
    return;
  }
  const int L = static_cast<int>(pos64) + 1;  // positions 0..pos
  const int slice = ((L + S - 1) / S + 15) / 16 * 16;
  const int j0 = min(rank * slice, L);
  const int n = min(j0 + slice, L) - j0;
  const int pos = L - 1;
  const int prel = pos - j0;  // row of the new token in this slice (valid when 0 <= prel < n)
  const int nchunks = (n + kChunk - 1) / kChunk;
  const int64_t cache_row0 = (static_cast<int64_t>(b) * p.nkv + h) * p.max_len + j0;

  bool ok = true;
  float o[kTiles][4];  // unnormalized output, 8-dim tiles (rows g: heads; rows g+8 unused)
  float m_run = -INFINITY, l_run = 0.f;
  const int g = lane >> 2, t = lane & 3;

  if (warp == kCWarps) {
    // ---------------------------------------------------------------- producer warp
    if (lane == 0 && nchunks > 0) {
      prefetch_tensormap(&mk);
      prefetch_tensormap(&mv);
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % p.ring;
        if (c >= p.ring && !mbar_wait(&empty[s], ((c / p.ring) - 1) & 1, p.err, DK_DEVERR_WAIT_EMPTY)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], CH::kSlotBytes);
        uint8_t* kt = ring + s * CH::kSlotBytes;
        const int y = static_cast<int>(cache_row0 + c * kChunk);  // rows < 2^31 (checked on the host)
#pragma unroll
        for (int sg = 0; sg < CH::kSegs; ++sg) {
          tma_load_2d(kt + sg * CH::kSegBytes, &mk, sg * CH::kSegHalves, y, &full[s]);
          tma_load_2d(kt + CH::kTensorBytes + sg * CH::kSegBytes, &mv, sg * CH::kSegHalves, y, &full[s]);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- consumer warps
    // q of this kv head's G query heads and the new k, v: RoPE with this thread's 4 dims (and
    // their partners); the tables are constant, so with a static cache their rows load before the
    // wait for the previous kernel.
    const int d = 4 * (tid % kQuads);
    const __half* cosr = p.cos + (p.rope_stride > 0 ? pos64 * p.rope_stride : 0);
    const __half* sinr = p.sin + (p.rope_stride > 0 ? pos64 * p.rope_stride : 0);
    const bool early_tables = p.static_cache && p.rope_stride > 0;
    uint2 c_lo, c_hi, s_lo, s_hi;
    if (early_tables) {
      c_lo = *reinterpret_cast<const uint2*>(cosr + d);
      c_hi = *reinterpret_cast<const uint2*>(cosr + d + kHd / 2);
      s_lo = *reinterpret_cast<const uint2*>(sinr + d);
      s_hi = *reinterpret_cast<const uint2*>(sinr + d + kHd / 2);
    }
    if (p.static_cache) pdl_wait();  // qkv comes from the previous kernel
    if (!early_tables) {
      c_lo = *reinterpret_cast<const uint2*>(cosr + d);
      c_hi = *reinterpret_cast<const uint2*>(cosr + d + kHd / 2);
      s_lo = *reinterpret_cast<const uint2*>(sinr + d);
      s_hi = *reinterpret_cast<const uint2*>(sinr + d + kHd / 2);
    }
    const bool owner = prel >= 0 && prel < n;
    const __half* qrow = p.qkv + static_cast<int64_t>(b) * (p.nq + 2 * p.nkv) * kHd;
    __half* kc = p.k_cache + (cache_row0 + prel) * kHd;  // row `pos` (used by the owner only)
    __half* vc = p.v_cache + (cache_row0 + prel) * kHd;
    constexpr int kRopeItems = (G + 1) * kQuads;
    for (int e = tid; e < kRopeItems + kHd / 8; e += kCWarps * 32) {
      if (e < kRopeItems) {  // e % kQuads == tid % kQuads: the table values above apply
        const int hh = e / kQuads;
        const __half* src = hh < G ? qrow + (h * G + hh) * kHd : qrow + (p.nq + h) * kHd;
        uint2 lo, hi;
        rope4(*reinterpret_cast<const uint2*>(src + d), *reinterpret_cast<const uint2*>(src + d + kHd / 2), c_lo,
              c_hi, s_lo, s_hi, lo, hi);
        __half* dst = hh < G ? &qs[hh][0] : knew;
        *reinterpret_cast<uint2*>(dst + d) = lo;
        *reinterpret_cast<uint2*>(dst + d + kHd / 2) = hi;
        if (hh == G && owner) {  // append k to the cache
          *reinterpret_cast<uint2*>(kc + d) = lo;
          *reinterpret_cast<uint2*>(kc + d + kHd / 2) = hi;
        }
      } else {
        const int v8 = 8 * (e - kRopeItems);
        const uint4 v = *reinterpret_cast<const uint4*>(qrow + (p.nq + p.nkv + h) * kHd + v8);
        *reinterpret_cast<uint4*>(vnew + v8) = v;
        if (owner) *reinterpret_cast<uint4*>(vc + v8) = v;
      }
    }
    consumers_sync();

    uint32_t qa[kHd / 16][2];  // q as the MMA A operand (rows: heads; rows >= G and g+8 are zero)
#pragma unroll
    for (int ks = 0; ks < kHd / 16; ++ks) {
      qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(&qs[g < G ? g : 0][16 * ks + 2 * t]) : 0u;
      qa[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(&qs[g < G ? g : 0][16 * ks + 8 + 2 * t]) : 0u;
    }
#pragma unroll
    for (int j = 0; j < kTiles; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: this lane addresses row rr of matrix mi
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % p.ring;
      if (ok && !mbar_wait(&full[s], (c / p.ring) & 1, p.err, DK_DEVERR_WAIT_FULL)) ok = false;
      ok = __all_sync(0xffffffffu, ok);  // the MMAs below need the whole warp
      const int rel0 = c * kChunk + 16 * warp;  // first position of this warp's block
      if (ok && rel0 < n) {
        const uint8_t* kt = ring + s * CH::kSlotBytes;
        const uint8_t* vt = kt + CH::kTensorBytes;
        // scores S[head][position] for positions rel0..rel0+15 (two 8-position MMA tiles)
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int krow = 16 * warp + 8 * (mi >> 1) + rr;  // matrices: (tile 0, k lo), (0, hi), (1, lo), (1, hi)
        const bool k_is_new = c * kChunk + krow == prel;
#pragma unroll
        for (int ks = 0; ks < kHd / 16; ++ks) {
          const int d0 = 16 * ks + 8 * (mi & 1);
          uint32_t kb[4];
          ldmatrix_x4(kb, k_is_new ? reinterpret_cast<const uint8_t*>(knew + d0) : CH::at(kt, krow, d0));
          mma_16816(sc[0], qa[ks][0], 0u, qa[ks][1], 0u, kb[0], kb[1]);
          mma_16816(sc[1], qa[ks][0], 0u, qa[ks][1], 0u, kb[2], kb[3]);
        }
        // online softmax (row g: the 4 lanes of a quad hold its 16 positions)
        float bm = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float v = rel0 + 8 * nt + 2 * t + e < n ? sc[nt][e] * p.scale : -INFINITY;
            sc[nt][e] = v;
            bm = fmaxf(bm, v);
          }
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
        const float m_new = fmaxf(m_run, bm);  // finite: position rel0 is inside the slice
        const float alpha = __expf(m_run - m_new);
        float pr[2][2];
        float ls = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            pr[nt][e] = __expf(sc[nt][e] - m_new);
            ls += pr[nt][e];
          }
        l_run = fmaf(l_run, alpha, ls);
        m_run = m_new;
#pragma unroll
        for (int j = 0; j < kTiles; ++j) {
          o[j][0] *= alpha;
          o[j][1] *= alpha;
        }
        // O += P V: P from the score accumulators (positions 2t.. of tile 0 and 8+2t.. of tile 1),
        // V by ldmatrix.trans; matrices: (k lo, d lo), (k hi, d lo), (k lo, d hi), (k hi, d hi)
        const uint32_t a0 = half2_bits(__float2half_rn(pr[0][0]), __float2half_rn(pr[0][1]));
        const uint32_t a2 = half2_bits(__float2half_rn(pr[1][0]), __float2half_rn(pr[1][1]));
        const int vrow = 16 * warp + (mi & 1) * 8 + rr;
        const int vrel = c * kChunk + vrow;
#pragma unroll
        for (int dp = 0; dp < kHd / 16; ++dp) {
          const int d0 = 16 * dp + (mi >> 1) * 8;
          const uint8_t* a = vrel >= n      ? reinterpret_cast<const uint8_t*>(vzero)
                             : vrel == prel ? reinterpret_cast<const uint8_t*>(vnew + d0)
                                            : CH::at(vt, vrow, d0);
          uint32_t vb[4];
          ldmatrix_x4_trans(vb, a);
          mma_16816(o[2 * dp], a0, 0u, a2, 0u, vb[0], vb[1]);
          mma_16816(o[2 * dp + 1], a0, 0u, a2, 0u, vb[2], vb[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  }

  // ------------------------------------------------------------------ this CTA's partial, pushed to the owners
  if (S > 1) cluster_wait();  // (1)
  if (warp < kCWarps) {
    // the 4 warps' (max, sum, unnormalized output) of every head combined in shared memory first, so
    // an owner adds S partials instead of 4 S
    if (g < G) {
#pragma unroll
      for (int j = 0; j < kTiles; ++j)
        *reinterpret_cast<float2*>(&pre_o[(warp * G + g) * kHd + 8 * j + 2 * t]) = make_float2(o[j][0], o[j][1]);
      if (t == 0) {
        pre_ml[(warp * G + g) * 2] = m_run;
        pre_ml[(warp * G + g) * 2 + 1] = l_run;
      }
    }
    consumers_sync();
    if (tid < G) {
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w)
        if (pre_ml[(w * G + tid) * 2 + 1] > 0.f) mx = fmaxf(mx, pre_ml[(w * G + tid) * 2]);
      float ls = 0.f;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) {
        const float l = pre_ml[(w * G + tid) * 2 + 1];
        const float wt = l > 0.f ? __expf(pre_ml[(w * G + tid) * 2] - mx) : 0.f;
        pre_w[w * G + tid] = wt;
        ls = fmaf(wt, l, ls);
      }
      cml[2 * tid] = mx;
      cml[2 * tid + 1] = ls;
    }
    consumers_sync();
    // output dims (two at a time) to the rank that owns them; (max, sum) of every head to every rank
    for (int e = tid; e < G * kHd / 2; e += kCWarps * 32) {
      const int gi = e / (kHd / 2), d = 2 * (e % (kHd / 2));
      float v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) {
        const float wt = pre_w[w * G + gi];
        const float2 ov = *reinterpret_cast<const float2*>(&pre_o[(w * G + gi) * kHd + d]);
        v0 = fmaf(wt, ov.x, v0);
        v1 = fmaf(wt, ov.y, v1);
      }
      const int q = d / D;
      float* dst = &recv_o[(rank * G + gi) * D + d % D];
      if (S > 1)
        st_async_v2_f32(map_shared_rank(dst, q), v0, v1, map_shared_rank(&recv, q));
      else
        *reinterpret_cast<float2*>(dst) = make_float2(v0, v1);
    }
    for (int e = tid; e < G * S; e += kCWarps * 32) {
      const int gi = e % G, q = e / G;
      float* dst = &recv_ml[(rank * G + gi) * 2];
      if (S > 1)
        st_async_v2_f32(map_shared_rank(dst, q), cml[2 * gi], cml[2 * gi + 1], map_shared_rank(&recv, q));
      else
        *reinterpret_cast<float2*>(dst) = make_float2(cml[2 * gi], cml[2 * gi + 1]);
    }
  }
  if (warp < kCWarps) {
    if (S > 1) {
      if (!mbar_wait(&recv, 0, p.err, DK_DEVERR_WAIT_FULL)) ok = false;
    } else {
      consumers_sync();
    }
  }
  __syncwarp();
  // (2) arrives once this CTA holds every partial sent to it; its wait before exit keeps each CTA
  // alive until all pushes in the cluster have landed
  if (S > 1) cluster_arrive_relaxed();

  // ------------------------------------------------------------------ combine this rank's dims
  if (warp < kCWarps) {
    // one half-warp per head (G <= 8 = 2 * kCWarps): the heads' maxima, weights and denominators at
    // once instead of two heads one after the other on one warp; every lane takes part in the
    // shuffles (they stay inside a half-warp), lanes of a half without a head only compute
    static_assert(G <= 2 * kCWarps, "a half-warp per head");
    const int gi = warp * 2 + (lane >> 4), hl = lane & 15;
    const bool head = gi < G;
    float mx = -INFINITY;
    if (head)
      for (int pp = hl; pp < nparts; pp += 16)
        if (recv_ml[(pp * G + gi) * 2 + 1] > 0.f) mx = fmaxf(mx, recv_ml[(pp * G + gi) * 2]);
#pragma unroll
    for (int x = 8; x > 0; x >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
    float ds = 0.f;
    if (head)
      for (int pp = hl; pp < nparts; pp += 16) {
        const float l = recv_ml[(pp * G + gi) * 2 + 1];
        const float w = l > 0.f ? __expf(recv_ml[(pp * G + gi) * 2] - mx) : 0.f;
        wts[pp * G + gi] = w;
        ds = fmaf(w, l, ds);
      }
#pragma unroll
    for (int x = 8; x > 0; x >>= 1) ds += __shfl_xor_sync(0xffffffffu, ds, x);
    if (head && hl == 0) den[gi] = ds;
    consumers_sync();
    __half* out = p.out + static_cast<int64_t>(b) * p.nq * kHd + h * G * kHd + rank * D;
    for (int e = tid; e < G * D; e += kCWarps * 32) {
      const int gi = e / D, dd = e % D;
      // 8 independent sums (partials pp = r mod 8), so the shared-memory loads of the up to 16
      // partials overlap instead of forming one chain of dependent multiply-adds
      float n[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int pp = 0; pp < nparts; pp += 8) {
#pragma unroll
        for (int r = 0; r < 8; ++r)
          if (pp + r < nparts) n[r] = fmaf(wts[(pp + r) * G + gi], recv_o[((pp + r) * G + gi) * D + dd], n[r]);
      }
      const float num = ((n[0] + n[1]) + (n[2] + n[3])) + ((n[4] + n[5]) + (n[6] + n[7]));
      out[gi * kHd + dd] = __float2half_rn(num / den[gi]);
    }
  }

  if (__syncthreads_or(!ok) && warp == kCWarps && lane == 0) {
    // a wait gave up: let copies still in flight land before the shared memory goes away (bounded)
    const uint64_t t0 = globaltimer_ns();
    for (int s = 0; s < min(p.ring, nchunks); ++s)
      while (!mbar_try_wait(&full[s], 0) && !mbar_try_wait(&full[s], 1) && globaltimer_ns() - t0 < 500000000ull) {
      }
  }
  __syncwarp();
  if (S > 1) cluster_wait();  // (2)
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
  if (B * nkv * max_len + kChunk >= (int64_t(1) << 31))
    return set_error(DK_ERR_INVALID, "decode_attention: B * n_kv * max_len must stay below 2^31 rows");
  if (!qkv || !k_cache || !v_cache || !pos || !cos || !sin || !out)
    return set_error(DK_ERR_INVALID, "decode_attention: NULL pointer");
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) ||
      (reinterpret_cast<uintptr_t>(cos) & 7) || (reinterpret_cast<uintptr_t>(sin) & 7) || (rope_stride & 3))
    return set_error(DK_ERR_ALIGN, "decode_attention: qkv, caches and out need 16-byte alignment, cos/sin 8 bytes");
  // S: a power of two (every rank combines an even number of output dims), at most 16. Automatic:
  // enough slices for one 128-position chunk pair each at max_len, but no more clusters than one wave
  // of CTAs (one per SM) once the (kv head, sequence) pairs alone fill the GPU - at batch 16 a 16-way
  // split ran 3.5 waves of CTAs.
  const int64_t per_wave = std::max<int64_t>(1, device_info().num_sms / (B * nkv));
  int want = splits > 0 ? splits
                        : static_cast<int>(std::min<int64_t>(std::min<int64_t>(kMaxSplit, (max_len + 127) / 128),
                                                             per_wave));
  want = std::max(1, std::min(want, kMaxSplit));
  int S = 1;
  while (S * 2 <= want) S *= 2;
  const int slice_max = static_cast<int>(((max_len + S - 1) / S + 15) / 16 * 16);
  const int ring = std::min(kMaxRing, (slice_max + kChunk - 1) / kChunk);

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
  p.ring = ring;
  p.static_cache = (flags & DK_ATTN_STATIC_CACHE) ? 1 : 0;
  p.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
  p.err = device_info().err_word;

  const uint64_t rows = static_cast<uint64_t>(B * nkv * max_len);
  const uint32_t box_inner = head_dim < 64 ? static_cast<uint32_t>(head_dim) : 64u;
  const CUtensorMapSwizzle sw = head_dim < 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap mk, mv;
  if (!make_tensor_map_2d(&mk, k_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, head_dim, rows, head_dim * 2, box_inner,
                          kChunk, sw) ||
      !make_tensor_map_2d(&mv, v_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, head_dim, rows, head_dim * 2, box_inner,
                          kChunk, sw))
    return DK_ERR_CUDA;

  const int G = static_cast<int>(nq / nkv);
  const size_t smem = 1024 + static_cast<size_t>(ring) * 2 * kChunk * head_dim * 2;
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
    e = launch(k, grid, dim3(kThreads), smem, st, pdl_enabled(), dim3(1, 1, S), mk, mv, p);               \
    break;                                                                                               \
  }
  switch (G) {
    DK_ATTN(1)
    DK_ATTN(2)
    DK_ATTN(3)
    DK_ATTN(4)
    DK_ATTN(5)
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
