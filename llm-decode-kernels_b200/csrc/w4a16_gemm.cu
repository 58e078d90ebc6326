// W4A16 (and W8A16) GEMM for prefill-sized inputs (M >= 128 rows) on the 5th-generation tensor cores:
// y[M, N] = x[M, K] @ dequant(W).T (+ bias), fp16 operands, fp32 accumulation in tensor memory.
// The e4m3 variant (kFp8) differs only in the weight tile and its conversion (see below) and applies
// the per-column scale to the fp32 accumulator in the epilogue.
//
// Replaces the reference's Triton tensor-core tile kernel for large M (kernels/w4a16.py:31-97,
// the `direct` path of w4a16_matmul) with tcgen05.mma. One CTA computes a 256 x BN tile of y (BN =
// 128, or 256 when the grid still has a tile per SM) as two 128-row accumulators that share each
// dequantized weight tile, so a weight is dequantized once per 256 rows of x:
// * warp 0 (one lane) streams, per 64-wide K step, the x tile [256 rows x 64] (two 128-row boxes)
//   with TMA into the 128-byte-swizzled K-major layout, and the packed weights of the tile (8 rows of
//   qweight x BN columns, int32) plus the step's scale and zero rows, into a 3- or 4-stage ring;
// * warps 2-9 dequantize: the 256 threads turn the BN columns' packed words (64 K values each) into
//   128-byte rows of the fp16 B tile, (q - z) * s with the reference's rounding (kernels/reference.py:35:
//   q - z is exact in fp16, one fp16 multiply by s), written straight into the swizzled K-major layout
//   that tcgen05 reads (16-byte chunk c of row t at c ^ (t % 8));
// * warp 1 allocates 2 x BN TMEM columns (the two 128 x BN fp32 accumulators) and one lane issues the
//   K = 16 tcgen05.mma of both halves per step, releasing each stage with tcgen05.commit;
// * warps 2-9 then read the accumulators back (tcgen05.ld, 32-lane quarters of TMEM), apply the e4m3
//   column scale, add the bias, round to fp16 and store.
// Nibble pairs become fp16 with the LOP3 "magic number" conversion (0x6400 exponent; Kim et al.,
// "Who Says Elephants Can't Run?"), after a PRMT that puts K values 2j and 2j+1 of a word into the
// low nibble of byte 0 and the high nibble of byte 2; one fp16x2 FMA with (1, 1/16) and
// (-(1024 + z), -(64 + z)) leaves (q_2j - z, q_2j+1 - z) exactly.
// Every mbarrier wait is bounded; a CTA whose wait gives up records a device error, waits (bounded)
// for its in-flight copies and MMAs, frees its TMEM and skips its stores.
#include <cstdio>
#include <mutex>

#include <cstring>

#include "common.cuh"
#include "tcgen05.cuh"

namespace dk {
namespace {

constexpr int kBM = 256, kBK = 64;  // CTA tile rows: two 128-row accumulators share one B tile
constexpr int kHalfRows = 128;                 // rows per tcgen05.mma (M = 128, cta_group::1)
constexpr int kThreads = 320;                  // warp 0 TMA, warp 1 TMEM + MMA, warps 2-9 dequant + epilogue
constexpr int kDeqThreads = 256;
constexpr int kAHalfBytes = kHalfRows * kBK * 2;  // 16 KB: one 128-row x 64 box of x
constexpr int kABytes = 2 * kAHalfBytes;

// Shared-memory layout per weight format and column tile BN (128 or 256): int4 (packed rows [8][BN]
// int32 + scale and zero rows; 4 stages at BN 128, 3 at 256) or e4m3 (the raw [64 K][128 N] byte
// tile, 3 stages). The TMEM accumulators take 2 * BN columns (512, all of TMEM, at BN 256).
template <bool kFp8, int BN>
struct Layout {
  static constexpr int kBBytes = BN * kBK * 2;  // dequantized weight tile
  static constexpr int kSZBytes = BN * 2;       // one scale (or zero) row (int4 format)
  static constexpr int kStages = (kFp8 || BN == 256) ? 3 : 4;
  static constexpr int kWBytes = kFp8 ? kBK * BN : (kBK / 8) * BN * 4;
  static constexpr uint32_t kWTx = kWBytes + (kFp8 ? 0 : 2 * kSZBytes);
  static constexpr int kOffB = kStages * kABytes;
  static constexpr int kOffW = kOffB + kStages * kBBytes;
  static constexpr int kOffS = kOffW + kStages * kWBytes;
  static constexpr int kOffZ = kOffS + kStages * kSZBytes;
  static constexpr int kOffBar = kOffZ + kStages * kSZBytes;
  static constexpr int kSmemBytes = kOffBar + (3 * kStages + 1) * 8 + 16 + 1024;  // + barriers, TMEM slot, alignment
};

struct GemmParams {
  __half* y;
  int64_t ldy;
  const __half* bias;
  const __half* scale;  // e4m3 format: per-column scale applied to the fp32 sum (kernels/fp8.py:81-82)
  int M, N, K;
  int ktiles;
  int* err;
};

// Convert the two e4m3 bytes of each 16-bit half of `v` to fp16 pairs (exact: every e4m3 value is an fp16).
__device__ __forceinline__ void e4m3x4_to_f16(uint32_t v, uint32_t& lo, uint32_t& hi) {
  asm("{\n.reg .b16 a, b;\nmov.b32 {a, b}, %2;\ncvt.rn.f16x2.e4m3x2 %0, a;\ncvt.rn.f16x2.e4m3x2 %1, b;\n}\n"
      : "=r"(lo), "=r"(hi)
      : "r"(v));
}

template <bool kFp8, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemm_tc_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mq,
                         const __grid_constant__ CUtensorMap ms, const __grid_constant__ CUtensorMap mz,
                         const GemmParams p) {
  using Lay = Layout<kFp8, BN>;
  constexpr int kStages = Lay::kStages;
  constexpr int kBN = BN, kBBytes = Lay::kBBytes, kSZBytes = Lay::kSZBytes, kTmemCols = 2 * BN;
  static_assert(!kFp8 || BN == 128, "the e4m3 tile is 128 columns");
  constexpr int kWBytes = Lay::kWBytes, kOffB = Lay::kOffB, kOffW = Lay::kOffW, kOffS = Lay::kOffS,
                kOffZ = Lay::kOffZ, kOffBar = Lay::kOffBar;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the shared array (accesses stay shared-space)
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kOffB;
  uint8_t* sW = smem + kOffW;
  uint8_t* sS = smem + kOffS;
  uint8_t* sZ = smem + kOffZ;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* deq = full + kStages;
  uint64_t* empty = deq + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const bool two = m0 + kHalfRows < p.M;  // second 128-row half has rows (uniform per CTA)
  const uint32_t stage_tx = Lay::kWTx + (two ? 2 : 1) * kAHalfBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&deq[s], kDeqThreads);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    s_fail = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // x comes from the previous kernel; y may alias memory it still reads

  bool ok = true;
  int issued = 0;  // producer: K steps whose copies were issued
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&mx);
      prefetch_tensormap(&mq);
      if (!kFp8) {
        prefetch_tensormap(&ms);
        prefetch_tensormap(&mz);
      }
      for (int kt = 0; kt < p.ktiles; ++kt) {
        const int s = kt % kStages;
        if (kt >= kStages && !mbar_wait(&empty[s], ((kt / kStages) - 1) & 1, p.err, DK_DEVERR_WAIT_EMPTY)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], stage_tx);
        tma_load_2d(sA + s * kABytes, &mx, kt * kBK, m0, &full[s]);
        if (two) tma_load_2d(sA + s * kABytes + kAHalfBytes, &mx, kt * kBK, m0 + kHalfRows, &full[s]);
        if (kFp8) {
          tma_load_2d(sW + s * kWBytes, &mq, n0, kt * kBK, &full[s]);  // e4m3 [64 K rows][128 N]
        } else {
          tma_load_2d(sW + s * kWBytes, &mq, n0, kt * (kBK / 8), &full[s]);
          tma_load_2d(sS + s * kSZBytes, &ms, n0, (kt * kBK) / 128, &full[s]);
          tma_load_2d(sZ + s * kSZBytes, &mz, n0, (kt * kBK) / 128, &full[s]);
        }
        issued = kt + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16_f32(kHalfRows, kBN);
      for (int kt = 0; kt < p.ktiles; ++kt) {
        const int s = kt % kStages;
        const uint32_t par = (kt / kStages) & 1;
        if (!mbar_wait(&full[s], par, p.err, DK_DEVERR_WAIT_FULL) ||
            !mbar_wait(&deq[s], par, p.err, DK_DEVERR_WAIT_FULL)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t a0 = smem_addr(sA + s * kABytes), b0 = smem_addr(sB + s * kBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t bdesc = tc::sdesc_k_sw128(b0 + 32 * kk);
          const uint32_t acc = (kt | kk) != 0 ? 1u : 0u;
          tc::mma_f16(tmem, tc::sdesc_k_sw128(a0 + 32 * kk), bdesc, idesc, acc);
          if (two) tc::mma_f16(tmem + kBN, tc::sdesc_k_sw128(a0 + kAHalfBytes + 32 * kk), bdesc, idesc, acc);
        }
        tc::commit(&empty[s]);  // the stage is free once these MMAs have read it
      }
      tc::commit(done);  // the accumulators are final once every MMA issued above has completed
    }
  } else if (kFp8) {
    // ------------------------------------------------------------ e4m3 -> fp16 (warps 2-9), transposing
    // Lane c owns columns 4c..4c+3; of the stage's 8 K-blocks (8 rows each) warp w takes block
    // (w + c / 2) % 8, so the 8 warps cover all 8 and the lanes of one store spread over the bank
    // groups. A K-block: 8 row words (4 columns each) -> PRMT pairs rows (2i, 2i+1) per column ->
    // cvt gives fp16 (k even, k odd) -> one 16-byte chunk per column.
    const int c = lane, w = warp - 2;
    const int kb = (w + (c >> 1)) & 7;
    for (int kt = 0; kt < p.ktiles; ++kt) {
      const int s = kt % kStages;
      if (!mbar_wait(&full[s], (kt / kStages) & 1, p.err, DK_DEVERR_WAIT_FULL)) {
        ok = false;
        break;
      }
      const uint32_t* raw = reinterpret_cast<const uint32_t*>(sW + s * kWBytes);  // row k: 32 words
      uint32_t r[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = raw[(kb * 8 + j) * (kBN / 4) + c];
      uint32_t h[4][4];  // [column][k pair]
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t lo, hi;
        e4m3x4_to_f16(prmt(r[2 * j], r[2 * j + 1], 0x5140u), lo, hi);  // columns 0, 1 of rows 2j, 2j+1
        h[0][j] = lo;
        h[1][j] = hi;
        e4m3x4_to_f16(prmt(r[2 * j], r[2 * j + 1], 0x7362u), lo, hi);  // columns 2, 3
        h[2][j] = lo;
        h[3][j] = hi;
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int n = 4 * c + cc;  // row n of the B tile, chunk kb
        *reinterpret_cast<uint4*>(sB + s * kBBytes + (n >> 3) * 1024 + (n & 7) * 128 + ((kb ^ (n & 7)) << 4)) =
            make_uint4(h[cc][0], h[cc][1], h[cc][2], h[cc][3]);
      }
      tc::fence_proxy_async_smem();
      mbar_arrive(&deq[s]);
    }
  } else {
    // ------------------------------------------------------------------ dequantization (warps 2-9)
    constexpr int kChunksPerThread = kBN / 32;  // 256 threads over BN columns x 8 packed rows
    const int t = threadIdx.x - 64;
    const int col = t & (kBN - 1);                   // output column n0 + col, row col of the B tile
    const int c0 = (t / kBN) * kChunksPerThread;     // this thread's packed rows (16-byte chunks)
    const uint32_t mul2 = 0x2C003C00u;  // (1.0, 1/16)
    for (int kt = 0; kt < p.ktiles; ++kt) {
      const int s = kt % kStages;
      if (!mbar_wait(&full[s], (kt / kStages) & 1, p.err, DK_DEVERR_WAIT_FULL)) {
        ok = false;
        break;
      }
      const uint32_t* w = reinterpret_cast<const uint32_t*>(sW + s * kWBytes);
      const __half sc = reinterpret_cast<const __half*>(sS + s * kSZBytes)[col];
      const __half zc = reinterpret_cast<const __half*>(sZ + s * kSZBytes)[col];
      const __half lo = __hneg(__hadd(__float2half_rn(1024.f), zc));  // -(1024 + z), exact
      const __half hi = __hneg(__hadd(__float2half_rn(64.f), zc));    // -(64 + z), exact
      const uint32_t add2 = half2_bits(lo, hi);
      const uint32_t sc2 = half2_bits(sc, sc);
      uint8_t* brow = sB + s * kBBytes + (col >> 3) * 1024 + (col & 7) * 128;
#pragma unroll
      for (int i = 0; i < kChunksPerThread; ++i) {  // packed row c = K 8c..8c+7 = 16-byte chunk c of row col
        const int c = c0 + i;
        const uint32_t word = w[c * kBN + col];
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t v = prmt(word, 0u, static_cast<uint32_t>(j | (4 << 4) | (j << 8) | (4 << 12)));
          const uint32_t u = lop3_and_or(v, 0x00F0000Fu, 0x64006400u);  // (1024 + q_2j, 1024 + 16 q_2j+1)
          h[j] = hmul2_rn(hfma2_rn(u, mul2, add2), sc2);                   // ((q - z) * s) for both
        }
        *reinterpret_cast<uint4*>(brow + ((c ^ (col & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
      }
      tc::fence_proxy_async_smem();  // these generic-proxy writes feed tcgen05.mma (async proxy)
      mbar_arrive(&deq[s]);
    }
  }

  if (!ok) atomicOr(&s_fail, 1);
  __syncthreads();
  const bool failed = s_fail != 0;
  if (failed && warp == 0 && lane == 0) {
    // wait (bounded) for the copies still in flight before the shared memory goes away
    const uint64_t t0 = globaltimer_ns();
    for (int it = issued > kStages ? issued - kStages : 0; it < issued; ++it)
      while (!mbar_try_wait(&full[it % kStages], (it / kStages) & 1) && globaltimer_ns() - t0 < 500000000ull) {
      }
  }

  // ------------------------------------------------------------------ epilogue (warps 2-9)
  if (warp >= 2) {
    const bool have = mbar_wait(done, 0, p.err, DK_DEVERR_WAIT_FULL) && !failed;
    __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the spin above
    tc::fence_after_sync();
    const int q = warp & 3;          // this warp's TMEM lane quarter (warp id mod 4)
    const int a = (warp - 2) >> 2;   // accumulator: rows 0-127 or 128-255 of the tile
    const int row = m0 + a * kHalfRows + 32 * q + lane;
    const bool used = a == 0 || two;
#pragma unroll 1
    for (int c0 = 0; c0 < kBN; c0 += 32) {
      float v[32];
      tc::tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + a * kBN + c0, v);
      const int n = n0 + c0;
      if (!have || !used || row >= p.M || n >= p.N) continue;
      if (kFp8) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < p.N) v[i] *= __half2float(p.scale[n + i]);
      }
      if (p.bias != nullptr) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n + i < p.N) v[i] += __half2float(p.bias[n + i]);
      }
      __half* dst = p.y + static_cast<int64_t>(row) * p.ldy + n;
      if (n + 32 <= p.N && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 o;
          o.x = half2_bits(__float2half_rn(v[i]), __float2half_rn(v[i + 1]));
          o.y = half2_bits(__float2half_rn(v[i + 2]), __float2half_rn(v[i + 3]));
          o.z = half2_bits(__float2half_rn(v[i + 4]), __float2half_rn(v[i + 5]));
          o.w = half2_bits(__float2half_rn(v[i + 6]), __float2half_rn(v[i + 7]));
          *reinterpret_cast<uint4*>(dst + i) = o;
        }
      } else {
        for (int i = 0; i < 32 && n + i < p.N; ++i) dst[i] = __float2half_rn(v[i]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool kFp8, int BN>
bool smem_ready() {
  static std::mutex mu;
  static bool done[64] = {};
  static bool okv[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && !done[dev]) {
    okv[dev] = opt_in_dynamic_smem(w4a16_gemm_tc_kernel<kFp8, BN>) >= Layout<kFp8, BN>::kSmemBytes;
    done[dev] = true;
  }
  return dev < 64 && okv[dev];
}

}  // namespace

// True when the tensor-core GEMM takes this shape: M >= 128 and N >= 128 (whole TMA boxes start
// inside the tensors), 16-byte aligned operands, x rows 16-byte aligned; group_size 128. Any y row
// stride works: the epilogue uses 16-byte stores only where the destination is aligned.
bool gemm_tc_ok(const void* x, int64_t ldx, const void* y, int64_t /*ldy*/, int64_t M, int64_t N, int64_t K,
                int64_t group_size) {
  return M >= kHalfRows && N >= 128 && N % 8 == 0 && K % 128 == 0 && group_size == 128 && aligned16(x) && ldx % 8 == 0 &&
         y != nullptr && M <= INT32_MAX && N <= INT32_MAX;
}

int launch_gemm_tc(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* zeros,
                   const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  // 256-column tiles halve the x re-reads per FLOP; take them when the grid still fills the GPU
  const int64_t tiles256 = ((N + 255) / 256) * ((M + kBM - 1) / kBM);
  const bool wide = N >= 256 && tiles256 >= device_info().num_sms;
  const int kBN = wide ? 256 : 128;
  const int kSmemBytes = wide ? Layout<false, 256>::kSmemBytes : Layout<false, 128>::kSmemBytes;
  if (!(wide ? smem_ready<false, 256>() : smem_ready<false, 128>()))
    return set_error(DK_ERR_UNSUPPORTED, "w4a16 gemm: %d bytes of shared memory do not fit", kSmemBytes);
  CUtensorMap mx, mq, ms, mz;
  if (!make_tensor_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, K, M, ldx * 2, kBK, kHalfRows,
                          CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&mq, qweight, CU_TENSOR_MAP_DATA_TYPE_INT32, N, K / 8, N * 4, kBN, kBK / 8,
                          CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tensor_map_2d(&ms, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K / 128, N * 2, kBN, 1,
                          CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tensor_map_2d(&mz, zeros, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K / 128, N * 2, kBN, 1,
                          CU_TENSOR_MAP_SWIZZLE_NONE))
    return DK_ERR_CUDA;
  GemmParams p;
  p.y = static_cast<__half*>(y);
  p.ldy = ldy;
  p.bias = static_cast<const __half*>(bias);
  p.scale = nullptr;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.ktiles = static_cast<int>(K / kBK);
  p.err = device_info().err_word;
  const dim3 grid(static_cast<unsigned>((N + kBN - 1) / kBN), static_cast<unsigned>((M + kBM - 1) / kBM), 1);
  cudaError_t e = launch(wide ? w4a16_gemm_tc_kernel<false, 256> : w4a16_gemm_tc_kernel<false, 128>, grid,
                         dim3(kThreads, 1, 1), kSmemBytes, st, pdl_enabled(), dim3(1, 1, 1), mx, mq, ms, mz, p);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w4a16 gemm launch: %s", cudaGetErrorString(e));
  return DK_OK;
}

// W8A16 (e4m3 weights [K, N], fp16 per-column scale) on the same tensor-core GEMM: kernels/fp8.py:42-127
// for large M. Same shape conditions as the int4 GEMM (M >= 128, N >= 128, N % 16 == 0 for the byte
// tile's 16-byte rows, K % 64 == 0, aligned operands).
bool gemm_tc_fp8_ok(const void* x, int64_t ldx, const void* wq, int64_t M, int64_t N, int64_t K) {
  return M >= kHalfRows && N >= 128 && N % 16 == 0 && K % kBK == 0 && K > 0 && aligned16(x) && ldx % 8 == 0 &&
         aligned16(wq) && M <= INT32_MAX && N <= INT32_MAX;
}

int launch_gemm_tc_fp8(const void* x, int64_t ldx, const uint8_t* wq, const void* scale, const void* bias, void* y,
                       int64_t ldy, int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  constexpr int kBN = 128;
  constexpr int kSmemBytes = Layout<true, 128>::kSmemBytes;
  if (!smem_ready<true, 128>())
    return set_error(DK_ERR_UNSUPPORTED, "w8a16 gemm: %d bytes of shared memory do not fit", kSmemBytes);
  CUtensorMap mx, mw;
  if (!make_tensor_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, K, M, ldx * 2, kBK, kHalfRows,
                          CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&mw, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, N, K, N, kBN, kBK, CU_TENSOR_MAP_SWIZZLE_NONE))
    return DK_ERR_CUDA;
  GemmParams p;
  p.y = static_cast<__half*>(y);
  p.ldy = ldy;
  p.bias = static_cast<const __half*>(bias);
  p.scale = static_cast<const __half*>(scale);
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.ktiles = static_cast<int>(K / kBK);
  p.err = device_info().err_word;
  const dim3 grid(static_cast<unsigned>((N + kBN - 1) / kBN), static_cast<unsigned>((M + kBM - 1) / kBM), 1);
  cudaError_t e = launch(w4a16_gemm_tc_kernel<true, 128>, grid, dim3(kThreads, 1, 1), kSmemBytes, st, pdl_enabled(),
                         dim3(1, 1, 1), mx, mw, mw, mw, p);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w8a16 gemm launch: %s", cudaGetErrorString(e));
  return DK_OK;
}

}  // namespace dk

// ------------------------------------------------------------------------------------------------
// Small-M W4A16 (and W8A16) on tcgen05 (16 <= M < 128 rows: batched decode), "swap AB": the MMA's M dimension is
// 128 output columns (the dequantized weight tile is the A operand) and its N dimension is the batch
// rows padded to MB = 16, 32 or 64 (x is the B operand), so the tensor core does no wasted work at small
// batch and the weights are read once for all rows. Replaces the reference's small-M tile kernel
// (kernels/w4a16.py:31-97 with BLOCK_M 16) and the M <= 16 CUDA decode kernel's batch loop
// (kernels/cuda/w4a16_decode.cu:29-121).
// * Split-K across a thread-block cluster of S CTAs (S <= 8) so that ~100-150 CTAs stream a layer's
//   weights; each CTA's partial [128 x MB] fp32 sums meet in distributed shared memory, added in rank
//   order (deterministic, no workspace).
// * x is staged once per CTA (its K slice, rows >= M zero) straight into the 128-byte-swizzled K-major
//   layout the B descriptor reads; the weights stream through a TMA ring and are dequantized by 8 warps
//   exactly like the prefill GEMM (the reference's fp16 rounding).
// * TMEM holds the [128 lanes x MB] accumulator; the epilogue reads it back by lane quarter.
// ------------------------------------------------------------------------------------------------
namespace dk {
namespace {

constexpr int kSkStages = 4;
constexpr int kSkBN = 128;                         // output columns per CTA (the MMA's M)
constexpr int kSkWBytes = (kBK / 8) * kSkBN * 4;   // 4 KB packed int4 weights per 64-K step
constexpr int kSkWSlot = kBK * kSkBN;              // ring slot: 8 KB (the e4m3 tile [64 K][128 N])
constexpr int kSkSZ = kSkBN * 2;                   // one scale (or zero) row
constexpr int kSkABytes = kSkBN * kBK * 2;         // 16 KB dequantized weight tile
constexpr int kSkXBudget = 96 * 1024;              // staged x slice per CTA
constexpr int kSkMaxSplit = 8;
// A split leaves every CTA at least this many 64-K steps (when a split is needed at all). Shallower
// splits were slower: qkv 2048 x 1536 at 32 rows took 23.9 us at S = 8 (3 steps per CTA, 16 clusters
// of 8) and 12.6 us at S = 4; batch-32 decode 12307 -> 13867 tok/s. The likely cause is that fewer
// 8-CTA clusters are resident at once than 148 / 8, so the last ones ran as a second wave (o_proj's
// 12 clusters of 8 were as fast as S = 4).
constexpr int kSkMinSteps = 6;
constexpr int kSkOffW = kSkStages * kSkABytes;
constexpr int kSkOffS = kSkOffW + kSkStages * kSkWSlot;
constexpr int kSkOffZ = kSkOffS + kSkStages * kSkSZ;
constexpr int kSkOffX = kSkOffZ + kSkStages * kSkSZ;  // 1024-aligned (all terms are multiples of 1024)

struct SkinnyParams {
  const __half* scale;  // e4m3 format: per-column scale applied to the fp32 sum (kernels/fp8.py:81-82)
  const __half* x;
  int64_t ldx;
  __half* y;
  int64_t ldy;
  const __half* bias;
  int M, N, K;
  int ktiles;  // K / 64
  int ks;      // 64-K steps per cluster rank
  int static_weights;
  int* err;
  TPArgs tp;  // tp.world > 0: a row-sharded launch with the allreduce fused in (skinny_tp_finish)
};

// The fused allreduce of a row-sharded small-M launch (dk_w4a16_matmul_allreduce above 16 rows): the
// epilogue pushed this rank's partial sums of the CTA's [M x 128] tile into every rank's cells (no
// bias); each CTA then polls the cells of its own column quads from every rank (with a cluster split
// S, the quads e with e % S == cluster rank), adds them in rank order plus the bias, and stores y.
// The last CTA to arrive advances the communicator's epoch. The same protocol and cells as the
// decode GEMV's fused allreduce (the ranks' grids may differ: cells are addressed by row and column).
__device__ void skinny_tp_finish(const SkinnyParams& p, unsigned long long ep, bool ok, int n0, int S, int crank) {
  const TPArgs& tp = p.tp;
  const uint32_t tag = static_cast<uint32_t>(ep);
  __shared__ int s_give_up;
  if (threadIdx.x == 0) s_give_up = ok ? 0 : 1;
  __syncthreads();
  if (ok) {
    volatile int* give_up = &s_give_up;
    // four adjacent columns at a time (N % 8 == 0): every rank's two 16-byte cell loads are issued
    // before the first is checked, so a quad costs one round trip, not one per rank and column
    const int nq = min(kSkBN, p.N - n0) / 4;
    for (int e = threadIdx.x; e < p.M * nq; e += blockDim.x) {
      if (e % S != crank) continue;
      const int m = e / nq, n = n0 + 4 * (e % nq);
      uint4 lo[DK_TP_MAX_WORLD], hi[DK_TP_MAX_WORLD];
#pragma unroll
      for (int q = 0; q < DK_TP_MAX_WORLD; ++q)
        if (q < tp.world) {
          const uint32_t* c = tp_cell(tp, tp.rank, ep, q, m, n);
          lo[q] = ld_volatile_v4(c);
          hi[q] = ld_volatile_v4(c + 4);
        }
      float sum[4] = {0.f, 0.f, 0.f, 0.f};
      bool good = true;
#pragma unroll
      for (int q = 0; q < DK_TP_MAX_WORLD; ++q) {
        if (q >= tp.world || !good) break;
        float v[4];
        if (lo[q].y == tag && lo[q].w == tag && hi[q].y == tag && hi[q].w == tag) {
          v[0] = __uint_as_float(lo[q].x);
          v[1] = __uint_as_float(lo[q].z);
          v[2] = __uint_as_float(hi[q].x);
          v[3] = __uint_as_float(hi[q].z);
        } else {
          good = tp_poll4(tp_cell(tp, tp.rank, ep, q, m, n), tag, v, give_up, p.err, tp.wait_ns);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) sum[c] += v[c];
      }
      if (!good) continue;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (p.bias != nullptr) sum[c] += __half2float(p.bias[n + c]);
        p.y[static_cast<int64_t>(m) * p.ldy + n + c] = __float2half_rn(sum[c]);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(tp.arrive, 1u) == gridDim.x * gridDim.y - 1) {
    *tp.arrive = 0;  // the next launch on this communicator uses epoch ep + 1
    *reinterpret_cast<volatile unsigned long long*>(tp.epoch) = ep;
  }
}

__host__ __device__ constexpr int skinny_smem_bytes(int MB, int ks) {
  return kSkOffX + ks * MB * 128 + (2 * kSkStages + 2) * 8 + 16 + 1024;
}

template <int MB, bool kFp8>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_skinny_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap ms,
                           const __grid_constant__ CUtensorMap mz, const SkinnyParams p) {
  constexpr int kXTile = MB * 128;                 // one 64-K x tile: MB rows of 128 bytes
  constexpr int kTmemCols = MB < 32 ? 32 : MB;     // allocation granularity is 32 columns
  constexpr int kHalf = MB / 2;                    // batch rows per epilogue warp
  static_assert(MB == 16 || MB == 32 || MB == 64, "batch tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sW = smem + kSkOffW;
  uint8_t* sS = smem + kSkOffS;
  uint8_t* sZ = smem + kSkOffZ;
  uint8_t* sX = smem + kSkOffX;
  uint64_t* full = reinterpret_cast<uint64_t*>(sX + p.ks * kXTile);
  uint64_t* deq = full + kSkStages;
  uint64_t* empty = deq + kSkStages;
  uint64_t* xready = empty + kSkStages;
  uint64_t* done = xready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ int s_fail;
  __shared__ unsigned long long s_ep;  // fused allreduce: this launch's epoch

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kSkBN;
  const int rank = blockIdx.y, S = gridDim.y;  // cluster dims (1, S, 1)
  const int kt0 = rank * p.ks;
  const int nk = max(0, min(p.ks, p.ktiles - kt0));  // >= 1 by the host's choice of S

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSkStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&deq[s], kDeqThreads);
      mbar_init(&empty[s], 1);
    }
    mbar_init(xready, kDeqThreads);
    mbar_init(done, 1);
    s_fail = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  bool ok = true;
  int issued = 0;
  if (warp == 0) {
    // ---------------------------------------------------------------- weight producer
    if (!p.static_weights) pdl_wait();
    if (lane == 0) {
      prefetch_tensormap(&mq);
      if (!kFp8) {
        prefetch_tensormap(&ms);
        prefetch_tensormap(&mz);
      }
      for (int i = 0; i < nk; ++i) {
        const int s = i % kSkStages;
        if (i >= kSkStages && !mbar_wait(&empty[s], ((i / kSkStages) - 1) & 1, p.err, DK_DEVERR_WAIT_EMPTY)) {
          ok = false;
          break;
        }
        const int kt = kt0 + i;
        if (kFp8) {
          mbar_arrive_expect_tx(&full[s], kSkWSlot);
          tma_load_2d(sW + s * kSkWSlot, &mq, n0, kt * kBK, &full[s]);  // e4m3 [64 K rows][128 N]
        } else {
          mbar_arrive_expect_tx(&full[s], kSkWBytes + 2 * kSkSZ);
          tma_load_2d(sW + s * kSkWSlot, &mq, n0, kt * (kBK / 8), &full[s]);
          tma_load_2d(sS + s * kSkSZ, &ms, n0, (kt * kBK) / 128, &full[s]);
          tma_load_2d(sZ + s * kSkSZ, &mz, n0, (kt * kBK) / 128, &full[s]);
        }
        issued = i + 1;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16_f32(kSkBN, MB);
      if (!mbar_wait(xready, 0, p.err, DK_DEVERR_WAIT_FULL)) ok = false;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % kSkStages;
        const uint32_t par = (i / kSkStages) & 1;
        if (!mbar_wait(&full[s], par, p.err, DK_DEVERR_WAIT_FULL) ||
            !mbar_wait(&deq[s], par, p.err, DK_DEVERR_WAIT_FULL)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t a0 = smem_addr(sA + s * kSkABytes), b0 = smem_addr(sX + i * kXTile);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          tc::mma_f16(tmem, tc::sdesc_k_sw128(a0 + 32 * kk), tc::sdesc_k_sw128(b0 + 32 * kk), idesc,
                      (i | kk) != 0 ? 1u : 0u);
        tc::commit(&empty[s]);
      }
      tc::commit(done);
    }
  } else {
    // ---------------------------------------------------------------- x staging, then dequantization
    const int t = threadIdx.x - 64;
    pdl_wait();  // x comes from the previous kernel
    // the epoch the previous launch on the communicator left (it finished before pdl_wait returned)
    if (p.tp.world > 0 && t == 0) s_ep = *reinterpret_cast<volatile unsigned long long*>(p.tp.epoch) + 1;
    {
      const int nchunks = nk * (kBK / 8);  // 16-byte chunks per staged row
      for (int idx = t; idx < MB * nchunks; idx += kDeqThreads) {
        const int m = idx / nchunks, kc = idx % nchunks;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (m < p.M) v = __ldcg(reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(m) * p.ldx +
                                                              (kt0 * kBK + kc * 8)));
        const int j = kc >> 3, c = kc & 7;
        *reinterpret_cast<uint4*>(sX + j * kXTile + (m >> 3) * 1024 + (m & 7) * 128 + ((c ^ (m & 7)) << 4)) = v;
      }
      tc::fence_proxy_async_smem();
      mbar_arrive(xready);
    }
    const int col = t & (kSkBN - 1);
    const int c0 = (t >> 7) * 4;  // this thread's half of the 8 packed rows
    const uint32_t mul2 = 0x2C003C00u;
    for (int i = 0; i < nk; ++i) {
      const int s = i % kSkStages;
      if (!mbar_wait(&full[s], (i / kSkStages) & 1, p.err, DK_DEVERR_WAIT_FULL)) {
        ok = false;
        break;
      }
      if constexpr (kFp8) {
        // e4m3 -> fp16, transposing: lane c owns columns 4c..4c+3, warp w the K-block (w + c / 2) % 8
        const int c = lane, kb = ((warp - 2) + (c >> 1)) & 7;
        const uint32_t* raw = reinterpret_cast<const uint32_t*>(sW + s * kSkWSlot);  // row k: 32 words
        uint32_t r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = raw[(kb * 8 + j) * (kSkBN / 4) + c];
        uint32_t h[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t lo, hi;
          e4m3x4_to_f16(prmt(r[2 * j], r[2 * j + 1], 0x5140u), lo, hi);
          h[0][j] = lo;
          h[1][j] = hi;
          e4m3x4_to_f16(prmt(r[2 * j], r[2 * j + 1], 0x7362u), lo, hi);
          h[2][j] = lo;
          h[3][j] = hi;
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int n = 4 * c + cc;
          *reinterpret_cast<uint4*>(sA + s * kSkABytes + (n >> 3) * 1024 + (n & 7) * 128 + ((kb ^ (n & 7)) << 4)) =
              make_uint4(h[cc][0], h[cc][1], h[cc][2], h[cc][3]);
        }
        tc::fence_proxy_async_smem();
        mbar_arrive(&deq[s]);
        continue;
      }
      const uint32_t* w = reinterpret_cast<const uint32_t*>(sW + s * kSkWSlot);
      const __half sc = reinterpret_cast<const __half*>(sS + s * kSkSZ)[col];
      const __half zc = reinterpret_cast<const __half*>(sZ + s * kSkSZ)[col];
      const uint32_t add2 = half2_bits(__hneg(__hadd(__float2half_rn(1024.f), zc)), __hneg(__hadd(__float2half_rn(64.f), zc)));
      const uint32_t sc2 = half2_bits(sc, sc);
      uint8_t* arow = sA + s * kSkABytes + (col >> 3) * 1024 + (col & 7) * 128;
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const int c = c0 + ii;
        const uint32_t word = w[c * kSkBN + col];
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t v = prmt(word, 0u, static_cast<uint32_t>(j | (4 << 4) | (j << 8) | (4 << 12)));
          const uint32_t u = lop3_and_or(v, 0x00F0000Fu, 0x64006400u);
          h[j] = hmul2_rn(hfma2_rn(u, mul2, add2), sc2);  // (q - z) * s with the reference's rounding
        }
        *reinterpret_cast<uint4*>(arow + ((c ^ (col & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
      }
      tc::fence_proxy_async_smem();
      mbar_arrive(&deq[s]);
    }
  }

  if (!ok) atomicOr(&s_fail, 1);
  __syncthreads();
  const bool failed = s_fail != 0;
  if (failed && warp == 0 && lane == 0) {
    const uint64_t t0 = globaltimer_ns();
    for (int it = issued > kSkStages ? issued - kSkStages : 0; it < issued; ++it)
      while (!mbar_try_wait(&full[it % kSkStages], (it / kSkStages) & 1) && globaltimer_ns() - t0 < 500000000ull) {
      }
  }

  // ------------------------------------------------------------------ epilogue (warps 2-9)
  // Lanes are output columns n0 + 32q + lane; warp pair h holds batch rows [h * MB/2, (h+1) * MB/2).
  float* red = reinterpret_cast<float*>(sA);  // [MB][128] partial sums; the A ring is idle once `done` fired
  bool have = false;
  if (warp >= 2) {
    have = mbar_wait(done, 0, p.err, DK_DEVERR_WAIT_FULL) && !failed;
    __syncwarp();
    tc::fence_after_sync();
    const int q = warp & 3, hrow = (warp - 2) >> 2;
    const int nl = 32 * q + lane, n = n0 + nl;
    float v[kHalf];
    const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * q) << 16) + hrow * kHalf;
    if constexpr (kHalf == 8) {
      tc::tmem_ld8(taddr, v);
    } else if constexpr (kHalf == 16) {
      tc::tmem_ld16(taddr, v);
    } else {
      tc::tmem_ld32(taddr, v);
    }
    if (have) {
#pragma unroll
      for (int j = 0; j < kHalf; ++j) {
        const int m = hrow * kHalf + j;
        if (kFp8 && n < p.N) v[j] *= __half2float(p.scale[n]);
        if (S == 1) {
          if (m < p.M && n < p.N) {
            if (p.tp.world > 0) {  // this rank's partial sum (the bias is added once, by the finish)
              tp_push(p.tp, s_ep, m, n, v[j]);
              continue;
            }
            float a = v[j];
            if (p.bias != nullptr) a += __half2float(p.bias[n]);
            p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2half_rn(a);
          }
        } else {
          red[m * kSkBN + nl] = v[j];
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
  if (S > 1) {
    // every rank's partials are in its shared memory; rank r sums elements e with e % S == r in rank order
    if (__syncthreads_or(!have && warp >= 2)) {
      cluster_sync();
      cluster_sync();
      if (p.tp.world > 0) skinny_tp_finish(p, s_ep, false, n0, S, rank);  // arrive all the same
      return;
    }
    cluster_sync();
    for (int e = threadIdx.x; e < MB * kSkBN; e += kThreads) {
      if (e % S != rank) continue;
      const int m = e / kSkBN, n = n0 + e % kSkBN;
      if (m >= p.M || n >= p.N) continue;
      float a = 0.f;
      for (int r = 0; r < S; ++r) a += ld_shared_cluster_f32(map_shared_rank(red + e, r));
      if (p.tp.world > 0) {
        tp_push(p.tp, s_ep, m, n, a);
        continue;
      }
      if (p.bias != nullptr) a += __half2float(p.bias[n]);
      p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2half_rn(a);
    }
    cluster_sync();  // keep the partial sums alive until every rank has read them
  }
  if (p.tp.world > 0) skinny_tp_finish(p, s_ep, !failed, n0, S, rank);
}

template <int MB, bool kFp8>
bool skinny_smem_ready(int bytes) {
  static std::mutex mu;
  static int limit[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (limit[dev] == 0) {
    limit[dev] = opt_in_dynamic_smem(w4a16_skinny_tc_kernel<MB, kFp8>);
    if (limit[dev] == 0) limit[dev] = -1;
  }
  return limit[dev] >= bytes;
}

}  // namespace

// The batch tile MB (16, 32 or 64) and cluster split S the small-M kernel uses for `rows` rows, or
// MB = 0 when it does not take the shape: N >= 128, K % 128 == 0, the staged x slice fits.
void skinny_choice(int64_t rows, int64_t N, int64_t K, int* mb_out, int* split_out) {
  *mb_out = 0;
  *split_out = 0;
  if (rows < 1 || N < kSkBN || K % kBK != 0 || K <= 0) return;
  const int ktiles = static_cast<int>(K / kBK);
  const int tiles_n = static_cast<int>((N + kSkBN - 1) / kSkBN);
  const int sms = device_info().num_sms;
  for (int mb : {64, 32, 16}) {
    if (mb > 16 && rows <= mb / 2) continue;  // the smallest tile that holds the rows
    int best = 0;
    for (int S = 1; S <= kSkMaxSplit && S <= ktiles; ++S) {
      const int ks = (ktiles + S - 1) / S;
      if ((S - 1) * ks >= ktiles) continue;             // every rank gets at least one K step
      if (ks * mb * 128 > kSkXBudget) continue;         // staged x slice
      if (best && tiles_n * S > sms) break;             // one wave of CTAs
      if (best && ks < kSkMinSteps) break;              // enough K steps per CTA
      best = S;
    }
    if (best) {
      *mb_out = mb;
      *split_out = best;
      return;
    }
  }
}

namespace {
template <bool kFp8>
int launch_skinny_core(const CUtensorMap& mq, const CUtensorMap& ms, const CUtensorMap& mz, const void* x, int64_t ldx,
                       const void* scale, const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                       bool static_weights, cudaStream_t st, const TPArgs* tp = nullptr) {
  for (int64_t m0 = 0; m0 < M;) {
    int mb = 0, S = 0;
    skinny_choice(M - m0, N, K, &mb, &S);
    if (mb == 0) return set_error(DK_ERR_UNSUPPORTED, "small-M tcgen05 gemm: no tile fits (N=%lld, K=%lld)",
                                  (long long)N, (long long)K);
    const int rows = static_cast<int>(std::min<int64_t>(mb, M - m0));
    if (tp != nullptr && rows > tp->max_m)
      return set_error(DK_ERR_UNSUPPORTED, "w4a16_matmul_allreduce: %d rows exceed the communicator", rows);
    SkinnyParams p;
    p.scale = static_cast<const __half*>(scale);
    p.x = static_cast<const __half*>(x) + m0 * ldx;
    p.ldx = ldx;
    p.y = static_cast<__half*>(y) + m0 * ldy;
    p.ldy = ldy;
    p.bias = static_cast<const __half*>(bias);
    p.M = rows;
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.ktiles = static_cast<int>(K / kBK);
    p.ks = (p.ktiles + S - 1) / S;
    p.static_weights = static_weights ? 1 : 0;
    p.err = device_info().err_word;
    if (tp != nullptr)
      p.tp = *tp;
    else
      std::memset(&p.tp, 0, sizeof(p.tp));
    const int smem = skinny_smem_bytes(mb, p.ks);
    const dim3 grid(static_cast<unsigned>((N + kSkBN - 1) / kSkBN), static_cast<unsigned>(S), 1);
    cudaError_t e = cudaSuccess;
    bool ready;
    if (mb == 16) {
      ready = skinny_smem_ready<16, kFp8>(smem);
      if (ready)
        e = launch(w4a16_skinny_tc_kernel<16, kFp8>, grid, dim3(kThreads), smem, st, pdl_enabled(), dim3(1, S, 1), mq,
                   ms, mz, p);
    } else if (mb == 32) {
      ready = skinny_smem_ready<32, kFp8>(smem);
      if (ready)
        e = launch(w4a16_skinny_tc_kernel<32, kFp8>, grid, dim3(kThreads), smem, st, pdl_enabled(), dim3(1, S, 1), mq,
                   ms, mz, p);
    } else {
      ready = skinny_smem_ready<64, kFp8>(smem);
      if (ready)
        e = launch(w4a16_skinny_tc_kernel<64, kFp8>, grid, dim3(kThreads), smem, st, pdl_enabled(), dim3(1, S, 1), mq,
                   ms, mz, p);
    }
    if (!ready) return set_error(DK_ERR_UNSUPPORTED, "small-M tcgen05 gemm: %d bytes of shared memory do not fit", smem);
    if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "small-M tcgen05 gemm launch: %s", cudaGetErrorString(e));
    m0 += rows;
  }
  return DK_OK;
}
}  // namespace

int launch_skinny_tc(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* zeros,
                     const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, bool static_weights,
                     cudaStream_t st, const TPArgs* tp) {
  CUtensorMap mq, ms, mz;
  if (!make_tensor_map_2d(&mq, qweight, CU_TENSOR_MAP_DATA_TYPE_INT32, N, K / 8, N * 4, kSkBN, kBK / 8,
                          CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tensor_map_2d(&ms, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K / 128, N * 2, kSkBN, 1,
                          CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tensor_map_2d(&mz, zeros, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, N, K / 128, N * 2, kSkBN, 1,
                          CU_TENSOR_MAP_SWIZZLE_NONE))
    return DK_ERR_CUDA;
  return launch_skinny_core<false>(mq, ms, mz, x, ldx, nullptr, bias, y, ldy, M, N, K, static_weights, st, tp);
}

// The e4m3 weight-only form (kernels/fp8.py:200-223 at 16..127 rows): wq [K, N] bytes, scale fp16 [N].
int launch_skinny_tc_fp8(const void* x, int64_t ldx, const uint8_t* wq, const void* scale, const void* bias, void* y,
                         int64_t ldy, int64_t M, int64_t N, int64_t K, bool static_weights, cudaStream_t st) {
  CUtensorMap mw;
  if (!make_tensor_map_2d(&mw, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, N, K, N, kSkBN, kBK, CU_TENSOR_MAP_SWIZZLE_NONE))
    return DK_ERR_CUDA;
  return launch_skinny_core<true>(mw, mw, mw, x, ldx, scale, bias, y, ldy, M, N, K, static_weights, st);
}

}  // namespace dk
