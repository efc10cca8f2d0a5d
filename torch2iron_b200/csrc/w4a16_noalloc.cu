// t2b_w4a16_gemm_noalloc: the W4A16 GEMV/GEMM for callers that cannot
// allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: for instance a host
// runtime that owns the whole device heap through its own pool and forbids
// any outside allocation, or a latency-critical thread on which cudaMalloc /
// cudaFree could block or synchronize the device.  t2b_w4a16_gemm needs a
// caller-provided workspace when it splits K across CTAs; this entry point
// instead uses a fixed scratch array compiled into the library (a
// file-scope __device__ array of NOALLOC_SCRATCH_BYTES), so the caller passes
// only inputs and outputs.
//
// Consequences a caller must know:
//   * every GPU that loads the library holds the array until process exit;
//   * sizes whose workspace exceeds NOALLOC_SCRATCH_BYTES are rejected with
//     T2B_ERR_WORKSPACE before anything is enqueued;
//   * all calls share the one array, which keeps the last call's contents:
//     calls that can overlap on the GPU (different streams, no ordering)
//     race on it and must not be issued;
//   * the first call on a device resolves the array's device address
//     (cudaGetSymbolAddress, with that device current) and keeps it for the
//     life of the process; make that first call before any stream capture,
//     and do not use this entry point on a device after cudaDeviceReset
//     (the module, and with it the array's address, may change).
// No cudaMalloc, cudaFree or allocating library routine is called here.
#include <mutex>

#include "linear_common.cuh"

namespace t2b {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(8) << 20;

// The array's name is a host-side stand-in in host code; its device address
// comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_gemm_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
static void* g_scratch_dev_ptr[NOALLOC_MAX_DEVICES];
static std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (set up once per device).
static int scratch_on_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return T2B_ERR_LAUNCH;
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return T2B_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_dev_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_scratch) != cudaSuccess || p == nullptr) return T2B_ERR_LAUNCH;
    g_scratch_dev_ptr[dev] = p;
  }
  *out = g_scratch_dev_ptr[dev];
  return T2B_OK;
}

}  // namespace t2b

extern "C" T2B_API size_t t2b_w4a16_gemm_noalloc_max_workspace(void) { return t2b::NOALLOC_SCRATCH_BYTES; }

extern "C" T2B_API int t2b_w4a16_gemm_noalloc(const void* weight, const uint32_t* meta, int wfmt, const void* x,
                                              int x_dtype, void* y, int y_dtype, int M, int N, int K,
                                              int group_size, void* stream) {
  // every check first: a rejected call enqueues nothing
  t2b::LinearParams p;
  const int r = t2b::gemm_params(weight, meta, wfmt, x, x_dtype, y, y_dtype, M, N, K, group_size, &p);
  if (r != T2B_OK) return r;
  // scratch only for the path this call takes (the tcgen05 and large-M paths need none)
  size_t partial_bytes = 0, counter_bytes = 0;
  t2b::gemm_path_workspace(p, wfmt, &partial_bytes, &counter_bytes);
  if (partial_bytes + counter_bytes > t2b::NOALLOC_SCRATCH_BYTES) return T2B_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = t2b::scratch_on_current_device(&scratch);
  if (st != T2B_OK) return st;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (counter_bytes) {
    // split-K tile counters must start at zero (an earlier aborted call may have left them armed)
    if (cudaMemsetAsync(static_cast<char*>(scratch) + partial_bytes, 0, counter_bytes, s) != cudaSuccess)
      return T2B_ERR_LAUNCH;
  }
  return t2b::gemm_launch(p, wfmt, scratch, t2b::NOALLOC_SCRATCH_BYTES, s);
}
