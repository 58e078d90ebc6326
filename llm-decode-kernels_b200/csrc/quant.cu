// Weight-format kernels: int4 pack/unpack, RTN int4 quantization and dequantization, e4m3
// quantization and dequantization. All are bit-exact with the reference's torch code:
//   pack_int4 / unpack_int4  kernels/quant.py:20-35
//   quantize_rtn             kernels/quant.py:38-49
//   dequantize_ref           kernels/reference.py:27-36
//   quantize_fp8 / dequantize_fp8  kernels/fp8.py:25-35
// The fp32 math uses IEEE division and round-half-even (rintf) exactly like torch's CPU/GPU ops;
// clamps are written as compare-and-select like at::clamp, so a -0.0 zero point survives (the
// reference stores -0.0 when a group's minimum is +0.0).
#include <cuda_fp8.h>

#include "common.cuh"

namespace dk {
namespace {

__device__ __forceinline__ float clamp_like_torch(float x, float lo, float hi) {
  const float y = (x < lo) ? lo : x;
  return (y > hi) ? hi : y;
}

__global__ void pack_int4_kernel(const int32_t* __restrict__ q, int32_t* __restrict__ packed, int64_t R,
                                 int64_t N) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= R * N) return;
  const int64_t r = i / N, n = i % N;
  uint32_t acc = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) acc += static_cast<uint32_t>(q[(r * 8 + j) * N + n]) << (4 * j);
  packed[i] = static_cast<int32_t>(acc);
}

__global__ void unpack_int4_kernel(const int32_t* __restrict__ packed, int32_t* __restrict__ q, int64_t R,
                                   int64_t N) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= R * N) return;
  const int64_t r = i / N, n = i % N;
  const int32_t w = packed[i];
#pragma unroll
  for (int j = 0; j < 8; ++j) q[(r * 8 + j) * N + n] = (w >> (4 * j)) & 0xF;
}

// One warp per (group, column). Pass 1: min/max over the group; pass 2: quantize and pack.
__global__ void quantize_rtn_kernel(const __half* __restrict__ w, int64_t ldw, int32_t* __restrict__ qweight,
                                    __half* __restrict__ scales, __half* __restrict__ zeros, int64_t N,
                                    int64_t K, int G) {
  const int64_t wid = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t groups = K / G;
  if (wid >= groups * N) return;
  const int64_t n = wid / groups, g = wid % groups;
  const __half* row = w + n * ldw + g * G;
  float mn = INFINITY, mx = -INFINITY;
  for (int k = lane; k < G; k += 32) {
    const float v = __half2float(row[k]);
    mn = v < mn ? v : mn;
    mx = v > mx ? v : mx;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float a = __shfl_xor_sync(0xffffffffu, mn, o);
    const float b = __shfl_xor_sync(0xffffffffu, mx, o);
    mn = a < mn ? a : mn;
    mx = b > mx ? b : mx;
  }
  float scale = __fdiv_rn(mx - mn, 15.0f);
  scale = scale < 1e-6f ? 1e-6f : scale;
  const float zero = clamp_like_torch(rintf(__fdiv_rn(-mn, scale)), 0.0f, 15.0f);
  for (int k8 = lane * 8; k8 < G; k8 += 256) {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = __fadd_rn(__fdiv_rn(__half2float(row[k8 + i]), scale), zero);
      const float q = clamp_like_torch(rintf(v), 0.0f, 15.0f);
      word |= static_cast<uint32_t>(static_cast<int>(q)) << (4 * i);
    }
    qweight[((g * G + k8) / 8) * N + n] = static_cast<int32_t>(word);
  }
  if (lane == 0) {
    scales[g * N + n] = __float2half_rn(scale);
    zeros[g * N + n] = __float2half_rn(zero);
  }
}

// out[n, k] = (fp16(q) - z) * s, fp16 rounding after each op (both ops exact except the multiply).
__global__ void dequantize_int4_kernel(const int32_t* __restrict__ qweight, const __half* __restrict__ scales,
                                       const __half* __restrict__ zeros, __half* __restrict__ out, int64_t N,
                                       int64_t K, int G) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= N * K) return;
  const int64_t n = i / K, k = i % K;
  const int q = (qweight[(k / 8) * N + n] >> (4 * (k % 8))) & 0xF;
  const __half s = scales[(k / G) * N + n];
  const __half z = zeros[(k / G) * N + n];
  out[i] = __hmul_rn(__hsub_rn(__int2half_rn(q), z), s);
}

// One warp per output row n: absmax, scale = max(amax/448, 1e-12), wq[k, n] = e4m3(clamp(w/scale)).
__global__ void quantize_fp8_kernel(const __half* __restrict__ w, int64_t ldw, uint8_t* __restrict__ wq,
                                    __half* __restrict__ scale_out, int64_t N, int64_t K) {
  const int64_t n = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  const __half* row = w + n * ldw;
  float amax = 0.f;
  for (int64_t k = lane; k < K; k += 32) {
    const float v = fabsf(__half2float(row[k]));
    amax = v > amax ? v : amax;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float a = __shfl_xor_sync(0xffffffffu, amax, o);
    amax = a > amax ? a : amax;
  }
  float s = __fdiv_rn(amax, 448.0f);
  s = s < 1e-12f ? 1e-12f : s;
  for (int64_t k = lane; k < K; k += 32) {
    const float v = clamp_like_torch(__fdiv_rn(__half2float(row[k]), s), -448.0f, 448.0f);
    wq[k * N + n] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
  }
  if (lane == 0) scale_out[n] = __float2half_rn(s);
}

__global__ void dequantize_fp8_kernel(const uint8_t* __restrict__ wq, const __half* __restrict__ scale,
                                      __half* __restrict__ out, int64_t N, int64_t K) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= N * K) return;
  const int64_t n = i / K, k = i % K;
  const __half_raw hr = __nv_cvt_fp8_to_halfraw(wq[k * N + n], __NV_E4M3);
  const float v = __half2float(__half(hr));
  out[i] = __float2half_rn(__fmul_rn(v, __half2float(scale[n])));
}

inline unsigned blocks_for(int64_t threads, int per_block) {
  return static_cast<unsigned>((threads + per_block - 1) / per_block);
}

int finish(const char* what) { return check_launch(what); }

}  // namespace
}  // namespace dk

using namespace dk;

extern "C" int dk_pack_int4(const int32_t* q, int32_t* packed, int64_t K, int64_t N, dk_stream_t stream) {
  if (K < 0 || N < 0 || K % 8 != 0) return set_error(DK_ERR_INVALID, "pack_int4: K must be a multiple of 8");
  if (K == 0 || N == 0) return DK_OK;
  if (!q || !packed) return set_error(DK_ERR_INVALID, "pack_int4: NULL pointer");
  const int64_t n = (K / 8) * N;
  pack_int4_kernel<<<blocks_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(q, packed, K / 8, N);
  return finish("pack_int4");
}

extern "C" int dk_unpack_int4(const int32_t* packed, int32_t* q, int64_t K, int64_t N, dk_stream_t stream) {
  if (K < 0 || N < 0 || K % 8 != 0) return set_error(DK_ERR_INVALID, "unpack_int4: K must be a multiple of 8");
  if (K == 0 || N == 0) return DK_OK;
  if (!q || !packed) return set_error(DK_ERR_INVALID, "unpack_int4: NULL pointer");
  const int64_t n = (K / 8) * N;
  unpack_int4_kernel<<<blocks_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(packed, q, K / 8, N);
  return finish("unpack_int4");
}

extern "C" int dk_quantize_rtn(const void* w, int64_t ldw, int32_t* qweight, void* scales, void* zeros,
                               int64_t N, int64_t K, int64_t group_size, dk_stream_t stream) {
  if (N < 0 || K < 0) return set_error(DK_ERR_INVALID, "quantize_rtn: negative size");
  if (group_size <= 0 || group_size % 8 != 0 || K % group_size != 0)
    return set_error(DK_ERR_INVALID, "quantize_rtn: K=%lld must be a multiple of group_size=%lld (itself a multiple of 8)",
                     (long long)K, (long long)group_size);
  if (ldw < K) return set_error(DK_ERR_INVALID, "quantize_rtn: row stride smaller than K");
  if (K == 0 || N == 0) return DK_OK;
  if (!w || !qweight || !scales || !zeros) return set_error(DK_ERR_INVALID, "quantize_rtn: NULL pointer");
  const int64_t warps = (K / group_size) * N;
  quantize_rtn_kernel<<<blocks_for(warps * 32, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(w), ldw, qweight, static_cast<__half*>(scales), static_cast<__half*>(zeros), N,
      K, static_cast<int>(group_size));
  return finish("quantize_rtn");
}

extern "C" int dk_dequantize_int4(const int32_t* qweight, const void* scales, const void* zeros, void* w,
                                  int64_t N, int64_t K, int64_t group_size, dk_stream_t stream) {
  if (N < 0 || K < 0 || group_size <= 0 || K % group_size != 0 || K % 8 != 0)
    return set_error(DK_ERR_INVALID, "dequantize_int4: bad sizes");
  if (K == 0 || N == 0) return DK_OK;
  if (!w || !qweight || !scales || !zeros) return set_error(DK_ERR_INVALID, "dequantize_int4: NULL pointer");
  dequantize_int4_kernel<<<blocks_for(N * K, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      qweight, static_cast<const __half*>(scales), static_cast<const __half*>(zeros), static_cast<__half*>(w), N,
      K, static_cast<int>(group_size));
  return finish("dequantize_int4");
}

extern "C" int dk_quantize_fp8(const void* w, int64_t ldw, uint8_t* wq, void* scale, int64_t N, int64_t K,
                               dk_stream_t stream) {
  if (N < 0 || K < 0 || ldw < K) return set_error(DK_ERR_INVALID, "quantize_fp8: bad sizes");
  if (K == 0 || N == 0) return DK_OK;
  if (!w || !wq || !scale) return set_error(DK_ERR_INVALID, "quantize_fp8: NULL pointer");
  quantize_fp8_kernel<<<blocks_for(N * 32, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(w), ldw, wq, static_cast<__half*>(scale), N, K);
  return finish("quantize_fp8");
}

extern "C" int dk_dequantize_fp8(const uint8_t* wq, const void* scale, void* w, int64_t N, int64_t K,
                                 dk_stream_t stream) {
  if (N < 0 || K < 0) return set_error(DK_ERR_INVALID, "dequantize_fp8: bad sizes");
  if (K == 0 || N == 0) return DK_OK;
  if (!w || !wq || !scale) return set_error(DK_ERR_INVALID, "dequantize_fp8: NULL pointer");
  dequantize_fp8_kernel<<<blocks_for(N * K, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      wq, static_cast<const __half*>(scale), static_cast<__half*>(w), N, K);
  return finish("dequantize_fp8");
}
