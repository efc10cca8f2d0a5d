// Shared device helpers for the sm_100a W4A16 decode kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/t2b.h"

#define T2B_DEV __device__ __forceinline__

namespace t2b {

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).  A kernel launched with the
// programmatic-stream-serialization attribute may start while its predecessor
// is still running; it must not touch anything the predecessor writes (or
// reads) until grid_dep_wait() returns.  Weights are constant, so every
// kernel here prefetches them before the wait.
// ---------------------------------------------------------------------------
T2B_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
T2B_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Number formats
// ---------------------------------------------------------------------------
T2B_DEV float bf16_bits_to_f32(uint32_t lo16) { return __uint_as_float(lo16 << 16); }

// The fused layer's fp16 activations (norm inputs, SwiGLU output): a in the
// low half, b in the high half, round to nearest, saturating at +-65504
// instead of overflowing to infinity.
T2B_DEV uint32_t f16x2_sat(float a, float b) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}
T2B_DEV float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
T2B_DEV float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

enum XDtype { X_BF16 = T2B_DTYPE_BF16, X_F16 = T2B_DTYPE_F16, X_F32 = T2B_DTYPE_F32 };

T2B_DEV float load_act(const void* p, int dtype, size_t i) {
  if (dtype == X_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == X_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

T2B_DEV void store_act(void* p, int dtype, size_t i, float v) {
  if (dtype == X_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == X_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// ---------------------------------------------------------------------------
// Reductions
// ---------------------------------------------------------------------------
T2B_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
T2B_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Split-K ticket.  Every CTA that contributes a partial to output tile `t`
// stores it (plain global stores), then calls split_ticket(); exactly one CTA
// -- the last to arrive -- gets `true`, re-arms the counter to zero for the
// next launch and runs the epilogue.  Partials must then be read with
// ld.global.cg (L1 bypass) -- see ldcg().
// ---------------------------------------------------------------------------
T2B_DEV bool split_ticket(int* counter, int arrivals) {
  __shared__ int s_last;
  __threadfence();  // make this thread's partial stores visible device-wide
  __syncthreads();
  if (threadIdx.x == 0) {
    int prev = atomicAdd(counter, 1);
    s_last = (prev == arrivals - 1);
    if (s_last) atomicExch(counter, 0);
  }
  __syncthreads();
  bool last = s_last != 0;
  if (last) __threadfence();  // acquire side
  return last;
}

T2B_DEV float ldcg(const float* p) { return __ldcg(p); }

// Device status word of a launch on stream `st`: the word bound to that
// stream (t2b_bind_error_word), else the calling host thread's word
// (t2b_set_error_word).  Every launch passes it to its kernel, whose
// time-bounded waits record T2B_ERR_TIMEOUT there (atomicCAS from 0, so the
// first error sticks).  nullptr = not recorded.
int* error_word(cudaStream_t st);

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA 1-D) with bounded waits.
// ---------------------------------------------------------------------------
T2B_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

T2B_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
T2B_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
T2B_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

T2B_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
T2B_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

T2B_DEV bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

T2B_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Spin on an mbarrier phase for at most `limit_ns` of wall time (each
// try_wait already suspends for a hardware-chosen interval).  On timeout the
// error word (if any) gets T2B_ERR_TIMEOUT and false is returned; the caller
// must stop using the stage.
T2B_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t phase, int* err, uint64_t limit_ns = 500000000ull) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, phase)) return true;
    if (globaltimer_ns() - t0 > limit_ns) break;
  }
  if (err) atomicCAS(err, 0, T2B_ERR_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// src, dst 16-byte aligned; bytes a multiple of 16.
T2B_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled TMA load of one box at element coordinates (x, y); no multicast.
// x * element size must be a multiple of 16 bytes.
T2B_DEV void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load of one box at element coordinates (x, y, z) of the
// tensor map `tmap` (a __grid_constant__ kernel parameter); no multicast.
// x * element size must be a multiple of 16 bytes.
T2B_DEV void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace t2b

namespace t2b {
// ---------------------------------------------------------------------------
// Thread-block clusters / distributed shared memory
// ---------------------------------------------------------------------------
T2B_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA in the cluster must call this (hardware barrier).
T2B_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in cluster CTA `rank`.
T2B_DEV uint32_t map_peer(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Bulk copy of this CTA's shared memory into a cluster peer's, completing on
// the peer's mbarrier (dst and bar are shared::cluster addresses of the peer;
// 16-byte aligned, bytes a multiple of 16).  The source must stay allocated
// until the peer has seen the bytes arrive.
T2B_DEV void bulk_s2s_peer(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(bar)
               : "memory");
}
// The two halves of cluster_sync(), for work between arrival and waiting.
T2B_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
T2B_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
T2B_DEV float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
}  // namespace t2b

// ---------------------------------------------------------------------------
// Device phase tracing (compiled in only with -DT2B_TRACE; see
// `python -m torch2iron_b200.build --trace`).  Each CTA takes a record in
// arrival order and stamps %globaltimer at phase boundaries; the host reads
// the records back with t2b_trace_dump().  The product build has no trace
// code and no trace symbols.
// ---------------------------------------------------------------------------
#ifdef T2B_TRACE
namespace t2b {
struct TraceRec {
  unsigned long long t[12];
  int tag, bx, by, bz, nblocks, key, pad0, pad1;
};
constexpr int TRACE_CAP = 1 << 15;
// one buffer per translation unit (no relocatable device code); records carry
// global timestamps, so the host merges the per-unit dumps by time
static __device__ TraceRec g_trace[TRACE_CAP];
static __device__ unsigned int g_trace_n;
}  // namespace t2b
// Defines the unit's read-back entry point: copies up to max_records records
// (128 bytes each) to host `dst`, returns the count, resets if `reset`.
#define T2B_TRACE_DUMP_FN(fname)                                                                          \
  extern "C" __attribute__((visibility("default"))) int fname(void* dst, int max_records, int reset) {    \
    unsigned int n = 0;                                                                                   \
    if (cudaMemcpyFromSymbol(&n, t2b::g_trace_n, sizeof(n)) != cudaSuccess) return -1;                    \
    int m = (int)(n < (unsigned)t2b::TRACE_CAP ? n : (unsigned)t2b::TRACE_CAP);                           \
    if (m > max_records) m = max_records;                                                                 \
    if (m > 0 && cudaMemcpyFromSymbol(dst, t2b::g_trace, (size_t)m * sizeof(t2b::TraceRec)) != cudaSuccess) \
      return -1;                                                                                          \
    if (reset) {                                                                                          \
      unsigned int z = 0;                                                                                 \
      if (cudaMemcpyToSymbol(t2b::g_trace_n, &z, sizeof(z)) != cudaSuccess) return -1;                    \
    }                                                                                                     \
    return m;                                                                                             \
  }
#define T2B_TRACE_BEGIN(tagv, keyv)                                                              \
  __shared__ int t2b_trace_slot;                                                                 \
  if (threadIdx.x == 0) {                                                                        \
    const unsigned s_ = atomicAdd(&t2b::g_trace_n, 1u);                                          \
    t2b_trace_slot = (int)(s_ & (t2b::TRACE_CAP - 1));                                           \
    t2b::TraceRec& r_ = t2b::g_trace[t2b_trace_slot];                                            \
    r_.tag = (tagv);                                                                             \
    r_.bx = blockIdx.x;                                                                          \
    r_.by = blockIdx.y;                                                                          \
    r_.bz = blockIdx.z;                                                                          \
    r_.nblocks = gridDim.x * gridDim.y * gridDim.z;                                              \
    r_.key = (keyv);                                                                             \
    for (int i_ = 0; i_ < 12; ++i_) r_.t[i_] = 0;                                                \
    r_.t[0] = t2b::globaltimer_ns();                                                             \
  }
#define T2B_TRACE_MARK(phase) \
  if (threadIdx.x == 0) t2b::g_trace[t2b_trace_slot].t[(phase)] = t2b::globaltimer_ns();
// Stamp from whichever thread executes it (the caller picks one thread).
#define T2B_TRACE_STAMP(phase) t2b::g_trace[t2b_trace_slot].t[(phase)] = t2b::globaltimer_ns();
#else
#define T2B_TRACE_STAMP(phase)
#define T2B_TRACE_BEGIN(tagv, keyv)
#define T2B_TRACE_MARK(phase)
#define T2B_TRACE_DUMP_FN(fname)
#endif
