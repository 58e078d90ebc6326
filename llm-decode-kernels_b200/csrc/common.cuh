// Shared device/host helpers for the sm_100a decode kernels.
//
// Everything here is written for Blackwell (sm_100a): bulk async copies (cp.async.bulk) completing
// on shared-memory mbarriers, programmatic dependent launch (griddepcontrol), thread-block clusters
// with distributed shared memory, and warp-level tensor-core MMA. Every wait on an mbarrier is
// bounded: after ~2 s (measured on %globaltimer) the waiting thread records an error code in a
// device-global word that the host reads with dk_device_error(), and the kernel returns instead of
// hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "decodek.h"

namespace dk {

// ------------------------------------------------------------------------------------------ errors
// Device-side error word: one `__device__ int` per device, defined in abi.cu; kernels get its
// address as an argument (DeviceInfo::err_word). Codes: DK_DEVERR_* in decodek.h. The first
// error wins (atomicCAS from 0).
__device__ __forceinline__ void record_device_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// Host-side error reporting: thread-local message behind dk_last_error().
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);

// ----------------------------------------------------------------------------------------- timing
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate wait

// ------------------------------------------------------------------------------------- mbarriers
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Returns false (and records `code` in *err)
// if the phase did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_device_error(err, code);
      return false;
    }
  }
  return true;
}

// --------------------------------------------------------------------------------- bulk copies
// 1-D bulk async copy global -> shared (this CTA), completion counted on `bar` in bytes.
// Requirements (checked by the host before choosing this path): both addresses 16-byte aligned,
// size a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Same, with an L2 eviction-priority hint (policy from createpolicy).
__device__ __forceinline__ void bulk_g2s_hint(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
      "%2, [%3], %4;" ::"r"(smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tiled TMA load (no multicast) of box {x, y} of `map` into this CTA's shared memory.
// x is the innermost coordinate in elements; callers keep x * element size a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------- L2 prefetch of later launches' data
// Byte ranges (16-byte aligned start and size) that a launch asks L2 to fetch for a later launch.
struct L2Prefetch {
  const char* ptr[DK_MAX_L2_PREFETCH];
  uint64_t bytes[DK_MAX_L2_PREFETCH];
  int n;
};

// The ranges are cut into 32 KB pieces dealt round-robin to the threads (cta, lane) of one warp per
// CTA, consecutive pieces on different CTAs (so on different SMs). Fire and forget: nothing waits
// for the fetch, and L2 is the point of coherence, so a prefetch can never expose stale data.
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf, int cta, int nctas, int lane) {
  constexpr uint64_t kPiece = 32768;
  const uint64_t stride = static_cast<uint64_t>(nctas) * 32;
  const uint64_t me = static_cast<uint64_t>(lane) * nctas + cta;
  uint64_t base = 0;  // global index of this range's first piece
  for (int r = 0; r < pf.n; ++r) {
    const uint64_t pieces = (pf.bytes[r] + kPiece - 1) / kPiece;
    for (uint64_t j = (me + stride - base % stride) % stride; j < pieces; j += stride) {
      const uint64_t off = j * kPiece;
      const uint32_t len = static_cast<uint32_t>(pf.bytes[r] - off < kPiece ? pf.bytes[r] - off : kPiece);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(pf.ptr[r] + off), "r"(len) : "memory");
    }
    base += pieces;
  }
}

// Host: the config's ranges trimmed inward to 16-byte boundaries (empty ones dropped).
inline L2Prefetch l2_prefetch_from(const dk_matmul_config* cfg) {
  L2Prefetch pf{};
  const int n = cfg ? (cfg->n_prefetch < DK_MAX_L2_PREFETCH ? cfg->n_prefetch : DK_MAX_L2_PREFETCH) : 0;
  for (int i = 0; i < n; ++i) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(cfg->l2_prefetch_ptr[i]);
    if (!a) continue;
    const uintptr_t lo = (a + 15) & ~uintptr_t(15);
    const uintptr_t hi = (a + cfg->l2_prefetch_bytes[i]) & ~uintptr_t(15);
    if (hi <= lo) continue;
    pf.ptr[pf.n] = reinterpret_cast<const char*>(lo);
    pf.bytes[pf.n] = hi - lo;
    ++pf.n;
  }
  return pf;
}

// ------------------------------------------------------------------- tensor-parallel exchange
// One rank's exchange buffer (allocated by dk_tp_buffer_alloc, zeroed, mapped into every peer):
//   [0, 256)           header: launch epoch (u64), CTA arrival count (u32)
//   [256, ...)         cells[slot 0..1][src rank][max_m][max_n]: 8 bytes each, {fp32 partial sum bits,
//                      low 32 bits of the epoch of the launch that wrote it}
// A receiver polls a cell until its epoch word matches: value and epoch travel in one 8-byte store,
// so no fence or separate flag is needed (the "LL" idea of NCCL's low-latency protocol).
constexpr size_t kTpHeaderBytes = 256;

// What a fused-allreduce launch needs; world == 0 means a plain launch.
struct TPArgs {
  uint32_t* cells[DK_TP_MAX_WORLD];  // cell region of each rank's buffer (peer mappings)
  unsigned long long* epoch;         // this rank's header
  unsigned int* arrive;
  int rank, world, max_m, max_n;
  uint64_t wait_ns;  // bound of each wait for a peer's partial sums (0: kWaitLimitNs)
};

__device__ __forceinline__ void st_volatile_v4(uint32_t* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ void st_volatile_v2(uint32_t* p, uint32_t a, uint32_t b) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ uint4 ld_volatile_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint2 ld_volatile_v2(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

// ---- fused-allreduce cells (row-sharded projections; see the buffer layout above)
__device__ __forceinline__ uint32_t* tp_cell(const TPArgs& tp, int q, unsigned long long ep, int src, int m, int n) {
  return tp.cells[q] +
         2 * (((static_cast<size_t>(ep & 1) * tp.world + src) * tp.max_m + m) * static_cast<size_t>(tp.max_n) + n);
}

__device__ __forceinline__ void tp_push(const TPArgs& tp, unsigned long long ep, int m, int n, float v) {
  const uint32_t tag = static_cast<uint32_t>(ep);
  for (int q = 0; q < tp.world; ++q) st_volatile_v2(tp_cell(tp, q, ep, tp.rank, m, n), __float_as_uint(v), tag);
}

__device__ __forceinline__ void tp_push4(const TPArgs& tp, unsigned long long ep, int m, int n, float4 v) {
  const uint32_t tag = static_cast<uint32_t>(ep);
  for (int q = 0; q < tp.world; ++q) {
    uint32_t* c = tp_cell(tp, q, ep, tp.rank, m, n);  // n % 4 == 0: 32-byte aligned
    st_volatile_v4(c, __float_as_uint(v.x), tag, __float_as_uint(v.y), tag);
    st_volatile_v4(c + 4, __float_as_uint(v.z), tag, __float_as_uint(v.w), tag);
  }
}

// Bounded polling: false once the CTA gave up (another thread timed out) or this wait passed the
// limit (then it records the device error and makes the CTA give up).
__device__ __forceinline__ bool tp_keep_waiting(int it, uint64_t& t0, volatile int* give_up, int* err,
                                                uint64_t limit) {
  if (*give_up) return false;
  if (it == 0) {
    t0 = globaltimer_ns();
  } else if ((it & 63) == 0 && globaltimer_ns() - t0 > (limit ? limit : kWaitLimitNs)) {
    record_device_error(err, DK_DEVERR_TP_WAIT);
    *give_up = 1;
    return false;
  }
  return true;
}

// The four values of cells c[0..3] (32 bytes) once all four carry `tag`.
__device__ __forceinline__ bool tp_poll4(const uint32_t* c, uint32_t tag, float (&out)[4], volatile int* give_up,
                                         int* err, uint64_t limit) {
  uint64_t t0 = 0;
  for (int it = 0;; ++it) {
    const uint4 a = ld_volatile_v4(c), b = ld_volatile_v4(c + 4);
    if (a.y == tag && a.w == tag && b.y == tag && b.w == tag) {
      out[0] = __uint_as_float(a.x);
      out[1] = __uint_as_float(a.z);
      out[2] = __uint_as_float(b.x);
      out[3] = __uint_as_float(b.z);
      return true;
    }
    if (!tp_keep_waiting(it, t0, give_up, err, limit)) return false;
  }
}

__device__ __forceinline__ bool tp_poll1(const uint32_t* c, uint32_t tag, float& out, volatile int* give_up, int* err,
                                         uint64_t limit) {
  uint64_t t0 = 0;
  for (int it = 0;; ++it) {
    const uint2 a = ld_volatile_v2(c);
    if (a.y == tag) {
      out = __uint_as_float(a.x);
      return true;
    }
    if (!tp_keep_waiting(it, t0, give_up, err, limit)) return false;
  }
}


// Pull the 128-byte line holding p into L2 (a hint; no data returns to the thread).
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// ------------------------------------------------------------- programmatic dependent launch
// Wait until the preceding kernel on the stream (if it was launched as our PDL primary) has
// completed and its writes are visible. A no-op when there is no such kernel.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Allow the next kernel on the stream to be scheduled (it still waits in pdl_wait for our
// completion before touching our outputs).
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// -------------------------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Split cluster barrier: arrive early, wait late (every thread of every CTA in the cluster takes
// each arrive and each wait, in the same order).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Asynchronous 8-byte store into cluster CTA shared memory (addresses from map_shared_rank); the
// bytes count against the transaction count of the mbarrier at `remote_bar` in the same CTA.
__device__ __forceinline__ void st_async_v2_f32(uint32_t remote, float a, float b, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(remote),
               "f"(a), "f"(b), "r"(remote_bar)
               : "memory");
}

// Four 8x8 b16 matrices from shared memory; lane i gives the row address of row (i % 8) of matrix
// (i / 8). `trans` delivers each matrix transposed.
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(row)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(row)));
}

// Address of `p` (a shared-memory address of this CTA) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_shared_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ void st_shared_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// ----------------------------------------------------------------------------- fp16 helpers
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t d;
  // (a & mask) | orv
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}

__device__ __forceinline__ uint32_t hsub2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_rn(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t half2_bits(__half lo, __half hi) {
  return static_cast<uint32_t>(__half_as_ushort(lo)) |
         (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}

// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col).
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ----------------------------------------------------------------------------- host helpers
struct DeviceInfo {
  int num_sms;
  int max_smem_optin;  // bytes per block with opt-in
  int smem_per_sm;     // bytes per SM
  int cc_major, cc_minor;
  int* err_word;       // device address of this device's error word
};
const DeviceInfo& device_info();  // cached per device, thread-safe

// Launch with optional programmatic dependent launch and cluster dimensions.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, bool pdl, dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster.x;
    attrs[n].val.clusterDim.y = cluster.y;
    attrs[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Global PDL switch (dk_set_pdl); on by default.
bool pdl_enabled();

// 2-D tensor map for TMA: `inner` x `outer` elements, rows `row_bytes` apart, box
// `box_inner` x `box_outer`. Returns false (with dk_last_error set) if the driver rejects it.
bool make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner,
                        uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Opt a kernel in to the largest dynamic shared memory the device allows next to its static shared
// memory. Returns the dynamic limit in bytes (0 if the attribute could not be set).
template <typename F>
int opt_in_dynamic_smem(F* kernel) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, kernel) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const int limit = device_info().max_smem_optin - static_cast<int>(a.sharedSizeBytes);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, limit) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return limit;
}

}  // namespace dk
