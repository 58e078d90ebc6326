// Tensor-parallel set-up: exchange buffers shared between the processes of one node through CUDA
// IPC, and the host-side communicator that the fused row-sharded GEMV + allreduce launches read.
//
// No reference counterpart: the reference is single-GPU (README.md:249). The data path lives in
// w4a16.cu (the GEMV epilogue pushes fp32 partial sums, each tagged with the launch's epoch, into
// every rank's buffer and sums the ranks' partials of its own columns); this file only allocates,
// maps and describes the buffers. Every
// function here is set-up code: it may allocate, synchronize and call the driver, and must not be
// called inside a CUDA-graph capture.
#include <cstring>

#include "common.cuh"

struct dk_tp_comm {
  int rank, world;
  int64_t max_m, max_n;
  uint64_t wait_ns;
  void* bufs[DK_TP_MAX_WORLD];
};

namespace dk {

bool tp_args_from(const dk_tp_comm* c, TPArgs* a) {
  if (c == nullptr) return false;
  std::memset(a, 0, sizeof(*a));
  for (int q = 0; q < c->world; ++q)
    a->cells[q] = reinterpret_cast<uint32_t*>(static_cast<char*>(c->bufs[q]) + kTpHeaderBytes);
  char* own = static_cast<char*>(c->bufs[c->rank]);
  a->epoch = reinterpret_cast<unsigned long long*>(own);
  a->arrive = reinterpret_cast<unsigned int*>(own + 8);
  a->rank = c->rank;
  a->world = c->world;
  a->max_m = static_cast<int>(c->max_m);
  a->max_n = static_cast<int>(c->max_n);
  a->wait_ns = c->wait_ns;
  return true;
}

int64_t tp_comm_max_m(const dk_tp_comm* c) { return c->max_m; }
int64_t tp_comm_max_n(const dk_tp_comm* c) { return c->max_n; }

}  // namespace dk

extern "C" {

int dk_tp_buffer_bytes(int32_t world, int64_t max_m, int64_t max_n, uint64_t* bytes) {
  using namespace dk;
  if (bytes == nullptr) return set_error(DK_ERR_INVALID, "dk_tp_buffer_bytes: bytes is NULL");
  if (world < 1 || world > DK_TP_MAX_WORLD || max_m < 1 || max_m > 64 || max_n < 8 || max_n % 8 != 0 ||
      max_n > (int64_t(1) << 24))
    return set_error(DK_ERR_INVALID,
                     "dk_tp_buffer_bytes: need 1 <= world <= %d, 1 <= max_m <= 64, max_n a positive multiple of 8",
                     DK_TP_MAX_WORLD);
  *bytes = kTpHeaderBytes + 2ull * static_cast<uint64_t>(world) * max_m * max_n * 8;
  return DK_OK;
}

int dk_tp_buffer_alloc(uint64_t bytes, void** ptr, void* ipc_handle) {
  using namespace dk;
  if (ptr == nullptr || ipc_handle == nullptr || bytes < kTpHeaderBytes)
    return set_error(DK_ERR_INVALID, "dk_tp_buffer_alloc: NULL argument or buffer smaller than its header");
  static_assert(sizeof(cudaIpcMemHandle_t) == DK_TP_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "dk_tp_buffer_alloc: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(DK_ERR_CUDA, "dk_tp_buffer_alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return DK_OK;
}

int dk_tp_buffer_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return dk::set_error(DK_ERR_CUDA, "dk_tp_buffer_free: %s", cudaGetErrorString(e));
  return DK_OK;
}

int dk_tp_buffer_open(const void* ipc_handle, void** ptr) {
  using namespace dk;
  if (ptr == nullptr || ipc_handle == nullptr) return set_error(DK_ERR_INVALID, "dk_tp_buffer_open: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "dk_tp_buffer_open: %s", cudaGetErrorString(e));
  *ptr = p;
  return DK_OK;
}

int dk_tp_buffer_close(void* ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return dk::set_error(DK_ERR_CUDA, "dk_tp_buffer_close: %s", cudaGetErrorString(e));
  return DK_OK;
}

int dk_tp_comm_create(dk_tp_comm** comm, int32_t rank, int32_t world, void* const* bufs, int64_t max_m,
                      int64_t max_n) {
  using namespace dk;
  uint64_t bytes = 0;
  if (comm == nullptr || bufs == nullptr) return set_error(DK_ERR_INVALID, "dk_tp_comm_create: NULL argument");
  int rc = dk_tp_buffer_bytes(world, max_m, max_n, &bytes);
  if (rc != DK_OK) return rc;
  if (rank < 0 || rank >= world) return set_error(DK_ERR_INVALID, "dk_tp_comm_create: rank %d of %d", rank, world);
  for (int q = 0; q < world; ++q)
    if (bufs[q] == nullptr || !aligned16(bufs[q]))
      return set_error(DK_ERR_INVALID, "dk_tp_comm_create: buffer of rank %d is NULL or not 16-byte aligned", q);
  dk_tp_comm* c = new dk_tp_comm();
  c->rank = rank;
  c->world = world;
  c->max_m = max_m;
  c->max_n = max_n;
  c->wait_ns = kWaitLimitNs;
  for (int q = 0; q < world; ++q) c->bufs[q] = bufs[q];
  *comm = c;
  return DK_OK;
}

int dk_tp_comm_set_wait(dk_tp_comm* comm, uint64_t wait_ns) {
  using namespace dk;
  if (comm == nullptr) return set_error(DK_ERR_INVALID, "dk_tp_comm_set_wait: comm is NULL");
  if (wait_ns < 1000000ull || wait_ns > 10000000000ull)
    return set_error(DK_ERR_INVALID, "dk_tp_comm_set_wait: the bound must be 1 ms .. 10 s (got %llu ns)",
                     (unsigned long long)wait_ns);
  comm->wait_ns = wait_ns;
  return DK_OK;
}

int dk_tp_comm_destroy(dk_tp_comm* comm) {
  delete comm;
  return DK_OK;
}

}  // extern "C"
