// W4A16 (and W8A16) GEMM for prefill-sized inputs (M >= 128 rows) on the 5th-generation tensor cores:
// y[M, N] = x[M, K] @ dequant(W).T (+ bias), fp16 operands, fp32 accumulation in tensor memory.
// The e4m3 variant (kFp8) differs only in the weight tile and its conversion (see below) and applies
// the per-column scale to the fp32 accumulator in the epilogue.
//
// Replaces the reference's Triton tensor-core tile kernel for large M (kernels/w4a16.py:31-97,
// the `direct` path of w4a16_matmul) with tcgen05.mma. One CTA computes a 128 x 128 tile of y:
// * warp 0 (one lane) streams, per 64-wide K step, the x tile [128 rows x 64] with TMA into the
//   128-byte-swizzled K-major layout, and the packed weights of the tile (8 rows of qweight x 128
//   columns, int32) plus the step's scale and zero rows, into a 4-stage ring;
// * warps 2-5 dequantize: thread t owns output column n0 + t and turns its 8 packed words (64 K
//   values) into one 128-byte row of the fp16 B tile, (q - z) * s with the reference's rounding
//   (kernels/reference.py:35: q - z is exact in fp16, one fp16 multiply by s), written straight
//   into the swizzled K-major layout that tcgen05 reads (16-byte chunk c of row t at c ^ (t % 8));
// * warp 1 allocates 128 TMEM columns (the 128 x 128 fp32 accumulator) and one lane issues four
//   K = 16 tcgen05.mma per step, releasing each stage with tcgen05.commit;
// * warps 2-5 then read the accumulator back (tcgen05.ld, one 32-lane quarter of TMEM per warp),
//   add the bias, round to fp16 and store.
// Nibble pairs become fp16 with the LOP3 "magic number" conversion (0x6400 exponent; Kim et al.,
// "Who Says Elephants Can't Run?"), after a PRMT that puts K values 2j and 2j+1 of a word into the
// low nibble of byte 0 and the high nibble of byte 2; one fp16x2 FMA with (1, 1/16) and
// (-(1024 + z), -(64 + z)) leaves (q_2j - z, q_2j+1 - z) exactly.
// Every mbarrier wait is bounded; a CTA whose wait gives up records a device error, waits (bounded)
// for its in-flight copies and MMAs, frees its TMEM and skips its stores.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace dk {
namespace {

constexpr int kBM = 256, kBN = 128, kBK = 64;  // CTA tile: two 128-row accumulators share one B tile
constexpr int kHalfRows = 128;                 // rows per tcgen05.mma (M = 128, cta_group::1)
constexpr int kThreads = 320;                  // warp 0 TMA, warp 1 TMEM + MMA, warps 2-9 dequant + epilogue
constexpr int kDeqThreads = 256;
constexpr int kTmemCols = 2 * kBN;             // two fp32 128 x 128 accumulators
constexpr int kAHalfBytes = kHalfRows * kBK * 2;  // 16 KB: one 128-row x 64 box of x
constexpr int kABytes = 2 * kAHalfBytes;
constexpr int kBBytes = kBN * kBK * 2;         // 16 KB dequantized weight tile
constexpr int kSZBytes = kBN * 2;              // one scale (or zero) row (int4 format)

// Shared-memory layout per weight format: int4 (packed rows [8][128] int32 + scale and zero rows, 4
// stages) or e4m3 (the raw [64 K][128 N] byte tile, 3 stages).
template <bool kFp8>
struct Layout {
  static constexpr int kStages = kFp8 ? 3 : 4;
  static constexpr int kWBytes = kFp8 ? kBK * kBN : (kBK / 8) * kBN * 4;  // 8 KB e4m3 / 4 KB int4
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

template <bool kFp8>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemm_tc_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mq,
                         const __grid_constant__ CUtensorMap ms, const __grid_constant__ CUtensorMap mz,
                         const GemmParams p) {
  using Lay = Layout<kFp8>;
  constexpr int kStages = Lay::kStages;
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
    const int t = threadIdx.x - 64;
    const int col = t & (kBN - 1);  // output column n0 + col, row col of the B tile
    const int c0 = (t >> 7) * 4;    // this thread's half of the 8 packed rows (16-byte chunks)
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
      for (int i = 0; i < 4; ++i) {  // packed row c = K values 8c..8c+7 = 16-byte chunk c of row col
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

template <bool kFp8>
bool smem_ready() {
  static std::mutex mu;
  static bool done[64] = {};
  static bool okv[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && !done[dev]) {
    okv[dev] = opt_in_dynamic_smem(w4a16_gemm_tc_kernel<kFp8>) >= Layout<kFp8>::kSmemBytes;
    done[dev] = true;
  }
  return dev < 64 && okv[dev];
}

}  // namespace

// True when the tensor-core GEMM takes this shape: M >= 128 and N >= 128 (whole TMA boxes start
// inside the tensors), 16-byte aligned operands, x rows 16-byte aligned; group_size 128.
bool gemm_tc_ok(const void* x, int64_t ldx, const void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                int64_t group_size) {
  return M >= kHalfRows && N >= kBN && N % 8 == 0 && K % 128 == 0 && group_size == 128 && aligned16(x) && ldx % 8 == 0 &&
         y != nullptr && M <= INT32_MAX && N <= INT32_MAX;
}

int launch_gemm_tc(const void* x, int64_t ldx, const int32_t* qweight, const void* scales, const void* zeros,
                   const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  constexpr int kSmemBytes = Layout<false>::kSmemBytes;
  if (!smem_ready<false>())
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
  cudaError_t e = launch(w4a16_gemm_tc_kernel<false>, grid, dim3(kThreads, 1, 1), kSmemBytes, st, pdl_enabled(),
                         dim3(1, 1, 1), mx, mq, ms, mz, p);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w4a16 gemm launch: %s", cudaGetErrorString(e));
  return DK_OK;
}

// W8A16 (e4m3 weights [K, N], fp16 per-column scale) on the same tensor-core GEMM: kernels/fp8.py:42-127
// for large M. Same shape conditions as the int4 GEMM (M >= 128, N >= 128, N % 16 == 0 for the byte
// tile's 16-byte rows, K % 64 == 0, aligned operands).
bool gemm_tc_fp8_ok(const void* x, int64_t ldx, const void* wq, int64_t M, int64_t N, int64_t K) {
  return M >= kHalfRows && N >= kBN && N % 16 == 0 && K % kBK == 0 && K > 0 && aligned16(x) && ldx % 8 == 0 &&
         aligned16(wq) && M <= INT32_MAX && N <= INT32_MAX;
}

int launch_gemm_tc_fp8(const void* x, int64_t ldx, const uint8_t* wq, const void* scale, const void* bias, void* y,
                       int64_t ldy, int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  constexpr int kSmemBytes = Layout<true>::kSmemBytes;
  if (!smem_ready<true>())
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
  cudaError_t e = launch(w4a16_gemm_tc_kernel<true>, grid, dim3(kThreads, 1, 1), kSmemBytes, st, pdl_enabled(),
                         dim3(1, 1, 1), mx, mw, mw, mw, p);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "w8a16 gemm launch: %s", cudaGetErrorString(e));
  return DK_OK;
}

}  // namespace dk
