// Fused RMSNorm (+ residual add) and fused SwiGLU: single-pass bandwidth kernels.
//
// RMSNorm restates kernels/rmsnorm.py:15-37 / kernels/reference.py:9-19:
//   h = x + residual            (fp16 add, stored as the new residual stream)
//   var = sum(h^2) / N          (fp32)
//   out = w * fp16(h * (1 / sqrt(var + eps)))   (last product in fp16)
// The reciprocal square root is computed as an IEEE sqrt followed by an IEEE division, which is
// how torch's CPU rsqrt computes it, so the normalized value rounds like the reference's.
//
// SwiGLU restates kernels/swiglu.py:14-28 / kernels/reference.py:22-24:
//   out = fp16(g / (1 + exp(-g))) * u   (silu in fp32, product in fp16)
//
// One CTA per row for RMSNorm (the row stays in registers between the reduction and the write),
// a 2-D grid of 16-byte vectors for SwiGLU. Both take programmatic dependent launch: they wait for
// the producing kernel before reading and release their dependents right away.
#include <algorithm>

#include "common.cuh"

namespace dk {
namespace {

constexpr int kNormThreads = 256;

template <int VPT>  // 8-half vectors per thread
__global__ void __launch_bounds__(kNormThreads) rmsnorm_vec_kernel(
    const __half* __restrict__ x, int64_t ldx, const __half* __restrict__ res, int64_t ldr,
    const __half* __restrict__ w, __half* __restrict__ out, int64_t ldo, __half* __restrict__ res_out,
    int64_t ldro, int N, float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int nv = N / 8;
  uint4 h[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    h[i] = make_uint4(0, 0, 0, 0);
    if (v < nv) {
      uint4 a = __ldcg(reinterpret_cast<const uint4*>(x + row * ldx) + v);
      if (res != nullptr) {
        const uint4 b = __ldcg(reinterpret_cast<const uint4*>(res + row * ldr) + v);
        __half2* ah = reinterpret_cast<__half2*>(&a);
        const __half2* bh = reinterpret_cast<const __half2*>(&b);
#pragma unroll
        for (int j = 0; j < 4; ++j) ah[j] = __hadd2_rn(ah[j], bh[j]);
        reinterpret_cast<uint4*>(res_out + row * ldro)[v] = a;
      }
      h[i] = a;
      const __half2* hh = reinterpret_cast<const __half2*>(&a);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(hh[j]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(N)), eps)));
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < nv) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + v);
      const __half2* hh = reinterpret_cast<const __half2*>(&h[i]);
      const __half2* wh = reinterpret_cast<const __half2*>(&wv);
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(hh[j]);
        const __half2 nrm = __floats2half2_rn(__fmul_rn(f.x, inv), __fmul_rn(f.y, inv));
        oh[j] = __hmul2_rn(wh[j], nrm);
      }
      reinterpret_cast<uint4*>(out + row * ldo)[v] = o;
    }
  }
}

// Any-alignment / any-N version (scalar loads, two passes over the row).
__global__ void __launch_bounds__(kNormThreads) rmsnorm_scalar_kernel(
    const __half* __restrict__ x, int64_t ldx, const __half* __restrict__ res, int64_t ldr,
    const __half* __restrict__ w, __half* __restrict__ out, int64_t ldo, __half* __restrict__ res_out,
    int64_t ldro, int N, float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  float ss = 0.f;
  for (int k = threadIdx.x; k < N; k += kNormThreads) {
    __half h = x[row * ldx + k];
    if (res != nullptr) {
      h = __hadd_rn(h, res[row * ldr + k]);
      res_out[row * ldro + k] = h;
    }
    const float f = __half2float(h);
    ss = fmaf(f, f, ss);
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(N)), eps)));
  for (int k = threadIdx.x; k < N; k += kNormThreads) {
    // res_out was written by this same thread above (same k mapping), so reading it back is safe
    const __half h = res != nullptr ? res_out[row * ldro + k] : x[row * ldx + k];
    const __half nrm = __float2half_rn(__fmul_rn(__half2float(h), inv));
    out[row * ldo + k] = __hmul_rn(w[k], nrm);
  }
}

__device__ __forceinline__ __half silu_f16(__half g) {
  const float f = __half2float(g);
  return __float2half_rn(__fdiv_rn(f, __fadd_rn(1.0f, expf(-f))));
}

__global__ void swiglu_vec_kernel(const __half* __restrict__ g, int64_t ldg, const __half* __restrict__ u,
                                  int64_t ldu, __half* __restrict__ out, int64_t ldo, int I) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= I / 8) return;
  const uint4 gv = __ldcg(reinterpret_cast<const uint4*>(g + row * ldg) + v);
  const uint4 uv = __ldcg(reinterpret_cast<const uint4*>(u + row * ldu) + v);
  const __half* gh = reinterpret_cast<const __half*>(&gv);
  const __half* uh = reinterpret_cast<const __half*>(&uv);
  uint4 o;
  __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
  for (int j = 0; j < 8; ++j) oh[j] = __hmul_rn(silu_f16(gh[j]), uh[j]);
  reinterpret_cast<uint4*>(out + row * ldo)[v] = o;
}

__global__ void swiglu_scalar_kernel(const __half* __restrict__ g, int64_t ldg, const __half* __restrict__ u,
                                     int64_t ldu, __half* __restrict__ out, int64_t ldo, int I) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.y;
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= I) return;
  out[row * ldo + k] = __hmul_rn(silu_f16(g[row * ldg + k]), u[row * ldu + k]);
}

}  // namespace
}  // namespace dk

using namespace dk;

extern "C" int dk_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, const void* weight,
                          void* out, int64_t ldo, void* residual_out, int64_t ldro, int64_t M, int64_t N,
                          float eps, dk_stream_t stream) {
  if (M < 0 || N < 0) return set_error(DK_ERR_INVALID, "rmsnorm: negative size");
  if (M > INT32_MAX || N > INT32_MAX) return set_error(DK_ERR_INVALID, "rmsnorm: size out of range");
  if (ldx < N || ldo < N || (residual && (ldr < N || ldro < N)))
    return set_error(DK_ERR_INVALID, "rmsnorm: row stride smaller than the row");
  if (M == 0 || N == 0) return DK_OK;
  if (!x || !weight || !out || (residual && !residual_out)) return set_error(DK_ERR_INVALID, "rmsnorm: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const __half* xr = static_cast<const __half*>(x);
  const __half* rr = static_cast<const __half*>(residual);
  const __half* wr = static_cast<const __half*>(weight);
  __half* o = static_cast<__half*>(out);
  __half* ro = static_cast<__half*>(residual_out);
  const bool vec = N % 8 == 0 && ldx % 8 == 0 && ldo % 8 == 0 && aligned16(x) && aligned16(weight) &&
                   aligned16(out) && (!residual || (ldr % 8 == 0 && ldro % 8 == 0 && aligned16(residual) &&
                                                   aligned16(residual_out)));
  const int vpt = static_cast<int>((N / 8 + kNormThreads - 1) / kNormThreads);
  cudaError_t e;
  const dim3 grid(static_cast<unsigned>(M)), block(kNormThreads);
  const bool pdl = pdl_enabled();
  const int n = static_cast<int>(N);
  if (vec && vpt <= 1) {
    e = launch(rmsnorm_vec_kernel<1>, grid, block, 0, st, pdl, dim3(1, 1, 1), xr, ldx, rr, ldr, wr, o, ldo, ro, ldro, n, eps);
  } else if (vec && vpt <= 2) {
    e = launch(rmsnorm_vec_kernel<2>, grid, block, 0, st, pdl, dim3(1, 1, 1), xr, ldx, rr, ldr, wr, o, ldo, ro, ldro, n, eps);
  } else if (vec && vpt <= 4) {
    e = launch(rmsnorm_vec_kernel<4>, grid, block, 0, st, pdl, dim3(1, 1, 1), xr, ldx, rr, ldr, wr, o, ldo, ro, ldro, n, eps);
  } else if (vec && vpt <= 8) {
    e = launch(rmsnorm_vec_kernel<8>, grid, block, 0, st, pdl, dim3(1, 1, 1), xr, ldx, rr, ldr, wr, o, ldo, ro, ldro, n, eps);
  } else {
    e = launch(rmsnorm_scalar_kernel, grid, block, 0, st, pdl, dim3(1, 1, 1), xr, ldx, rr, ldr, wr, o, ldo, ro, ldro, n, eps);
  }
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "rmsnorm launch: %s", cudaGetErrorString(e));
  return DK_OK;
}

extern "C" int dk_swiglu(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out, int64_t ldo,
                         int64_t M, int64_t I, dk_stream_t stream) {
  if (M < 0 || I < 0) return set_error(DK_ERR_INVALID, "swiglu: negative size");
  if (M > 65535 * 1024ll || I > INT32_MAX) return set_error(DK_ERR_INVALID, "swiglu: size out of range");
  if (ldg < I || ldu < I || ldo < I) return set_error(DK_ERR_INVALID, "swiglu: row stride smaller than the row");
  if (M == 0 || I == 0) return DK_OK;
  if (!gate || !up || !out) return set_error(DK_ERR_INVALID, "swiglu: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = I % 8 == 0 && ldg % 8 == 0 && ldu % 8 == 0 && ldo % 8 == 0 && aligned16(gate) &&
                   aligned16(up) && aligned16(out);
  const int threads = 128;
  cudaError_t e;
  const __half* g = static_cast<const __half*>(gate);
  const __half* u = static_cast<const __half*>(up);
  __half* o = static_cast<__half*>(out);
  for (int64_t m0 = 0; m0 < M; m0 += 65535) {
    const unsigned rows = static_cast<unsigned>(std::min<int64_t>(65535, M - m0));
    if (vec) {
      const dim3 grid(static_cast<unsigned>((I / 8 + threads - 1) / threads), rows);
      e = launch(swiglu_vec_kernel, grid, dim3(threads), 0, st, pdl_enabled(), dim3(1, 1, 1), g + m0 * ldg, ldg,
                 u + m0 * ldu, ldu, o + m0 * ldo, ldo, static_cast<int>(I));
    } else {
      const dim3 grid(static_cast<unsigned>((I + threads - 1) / threads), rows);
      e = launch(swiglu_scalar_kernel, grid, dim3(threads), 0, st, pdl_enabled(), dim3(1, 1, 1), g + m0 * ldg, ldg,
                 u + m0 * ldu, ldu, o + m0 * ldo, ldo, static_cast<int>(I));
    }
    if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "swiglu launch: %s", cudaGetErrorString(e));
  }
  return DK_OK;
}
