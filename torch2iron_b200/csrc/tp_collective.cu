// Tensor-parallel all-reduce of the row-parallel partials fused with the
// residual step, over peer memory.
//
// The o_proj and down projections of a tensor-parallel layer each leave a
// partial y_r [M][H] on every rank r; the layer continues with
//   x += sum_r y_r,  ssq[m] = sum_n x[m,n]^2,  xw = fp16(x * next_norm_w)
// (residual_add_rms_norm/kernel.cc:70-93 in split form, after the all-reduce
// that batch_decode_fused.py:485-498, 529-539 implies when the GEMM before it
// is split over devices).  Here one kernel does both: every rank signals
// that its partial is complete by storing the call's sequence number into a
// flag word in every peer's memory (release at system scope), waits (time
// bounded) until every peer has signalled the same call, then reads all
// partials straight from the peers' memory over NVLink and sums them in
// rank order -- the same order on every rank, so the replicated residual
// stream stays identical across ranks -- in fp32.
//
// Sequence numbers: each rank keeps a call counter in device memory; every
// CTA reads it at entry, and the last CTA to finish stores the next value,
// so a captured CUDA graph (constant kernel parameters) still signals a new
// number on every replay.  Flags only grow, so a wait is "flag >= call".
// Buffer reuse: a rank overwrites a partial buffer two calls later at the
// earliest (o_proj and down alternate between two buffers); by then every
// peer has signalled the call in between, which it does only after it
// finished reading this one.
#include "t2b_common.cuh"
#include "launch.cuh"

namespace t2b {

constexpr int TPAR_MAX_WORLD = 8;
constexpr int TPAR_THREADS = 512;   // one 8-element chunk per thread for H = 4096

struct TpArParams {
  const void* part[TPAR_MAX_WORLD];  // every rank's partial [M][H] (peer-mapped; this rank's at [rank])
  int* flags[TPAR_MAX_WORLD];        // every rank's flag words [world]: flags[q][r] = last call rank r signalled to q
  int* state;                        // this rank: [0] calls completed, [1] CTAs finished with the current call
  int rank, world, ybf16;
  float* x;
  float* ssq;
  const __nv_bfloat16* w;
  __half* xw;
  int M, H;
  int* err;
};

T2B_DEV int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

T2B_DEV void st_relaxed_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 16 bytes of a peer's partial, not cached on this GPU (the buffer is rewritten every other call)
T2B_DEV uint4 ld_peer16(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Eight partial values starting at element o from every rank, summed in rank
// order.  All ranks' loads are issued before the first add: each is an
// NVLink round trip, and issued one after another they would add up.
T2B_DEV void sum_partials8(const TpArParams& P, size_t o, float* a) {
  uint4 r[TPAR_MAX_WORLD][2];
  if (P.ybf16) {
#pragma unroll
    for (int q = 0; q < TPAR_MAX_WORLD; ++q)
      if (q < P.world) r[q][0] = ld_peer16(static_cast<const __nv_bfloat16*>(P.part[q]) + o);
#pragma unroll
    for (int q = 0; q < TPAR_MAX_WORLD; ++q) {
      if (q >= P.world) break;
      const uint32_t u[4] = {r[q][0].x, r[q][0].y, r[q][0].z, r[q][0].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        a[2 * j] += __uint_as_float(u[j] << 16);
        a[2 * j + 1] += __uint_as_float(u[j] & 0xffff0000u);
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < TPAR_MAX_WORLD; ++q)
      if (q < P.world) {
        const float* f = static_cast<const float*>(P.part[q]) + o;
        r[q][0] = ld_peer16(f);
        r[q][1] = ld_peer16(f + 4);
      }
#pragma unroll
    for (int q = 0; q < TPAR_MAX_WORLD; ++q) {
      if (q >= P.world) break;
      const uint32_t u[8] = {r[q][0].x, r[q][0].y, r[q][0].z, r[q][0].w, r[q][1].x, r[q][1].y, r[q][1].z, r[q][1].w};
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += __uint_as_float(u[j]);
    }
  }
}

// One CTA per row m.
__global__ void __launch_bounds__(TPAR_THREADS) tp_allreduce_residual_kernel(const __grid_constant__ TpArParams P) {
  grid_dep_wait();  // this rank's partial is complete (the GEMM before finished)
  grid_dep_launch();
  __shared__ int s_call, s_ok;
  __shared__ float part_sq[TPAR_THREADS / 32];
  const int m = blockIdx.x;
  const int call = *reinterpret_cast<volatile int*>(&P.state[0]) + 1;
  if (m == 0 && threadIdx.x < P.world) {
    // lane q signals rank q (this one included) that this rank's partial of `call`
    // is complete: a system-scope fence orders the partial before the flag, and the
    // stores to the peers go out in parallel, not one release after another
    __threadfence_system();
    st_relaxed_sys(P.flags[threadIdx.x] + P.rank, call);
  }
  if (threadIdx.x == 0) {
    s_call = call;
    bool ok = true;
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < P.world && ok; ++q)
      while (ld_acquire_sys(P.flags[P.rank] + q) < call) {
        if (globaltimer_ns() - t0 > 500000000ull) {  // 0.5 s: a peer never signalled
          if (P.err) atomicCAS(P.err, 0, T2B_ERR_TIMEOUT);
          ok = false;
          break;
        }
      }
    s_ok = ok;
  }
  __syncthreads();
  if (s_ok) {
    float sq = 0.f;
    for (int i = threadIdx.x * 8; i < P.H; i += TPAR_THREADS * 8) {
      const size_t o = (size_t)m * P.H + i;
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      sum_partials8(P, o, a);   // rank order on every rank
      float4* xp = reinterpret_cast<float4*>(P.x + o);
      const float4 x0 = xp[0], x1 = xp[1];
      const float v[8] = {x0.x + a[0], x0.y + a[1], x0.z + a[2], x0.w + a[3],
                          x1.x + a[4], x1.y + a[5], x1.z + a[6], x1.w + a[7]};
      xp[0] = make_float4(v[0], v[1], v[2], v[3]);
      xp[1] = make_float4(v[4], v[5], v[6], v[7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) sq += v[j] * v[j];
      if (P.xw) {
        const uint4 wr = *reinterpret_cast<const uint4*>(P.w + i);
        const uint32_t wu[4] = {wr.x, wr.y, wr.z, wr.w};
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          h[j] = f16x2_sat(v[2 * j] * __uint_as_float(wu[j] << 16), v[2 * j + 1] * __uint_as_float(wu[j] & 0xffff0000u));
        *reinterpret_cast<uint4*>(P.xw + o) = make_uint4(h[0], h[1], h[2], h[3]);
      }
    }
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) part_sq[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0 && P.ssq) {
      float t = 0.f;
      for (int k = 0; k < TPAR_THREADS / 32; ++k) t += part_sq[k];
      P.ssq[m] = t;
    }
  }
  // the last CTA of this call advances the call counter (every CTA read it at entry)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&P.state[1], 1) == (int)gridDim.x - 1) {
      P.state[1] = 0;
      __threadfence();
      atomicExch(&P.state[0], s_call);
    }
  }
}

}  // namespace t2b

using namespace t2b;

extern "C" T2B_API size_t t2b_tp_allreduce_state_bytes(void) { return 4 * sizeof(int32_t); }

extern "C" T2B_API int t2b_tp_allreduce_residual_norm_input(const void* const* partials, int y_dtype,
                                                             int32_t* const* flags, int32_t* state, int rank,
                                                             int world, float* x_resid, float* ssq_out,
                                                             const uint16_t* next_w, void* xw_out, int M, int H,
                                                             void* stream) {
  if (!partials || !flags || !state || !x_resid) return T2B_ERR_ARG;
  if (world < 1 || world > TPAR_MAX_WORLD || rank < 0 || rank >= world) return T2B_ERR_ARG;
  if (y_dtype != T2B_DTYPE_BF16 && y_dtype != T2B_DTYPE_F32) return T2B_ERR_ARG;
  if ((xw_out == nullptr) != (next_w == nullptr)) return T2B_ERR_ARG;
  if (M < 1 || M > 65535 || H < 8 || H % 8) return T2B_ERR_SHAPE;
  TpArParams P{};
  for (int q = 0; q < world; ++q) {
    if (!partials[q] || !flags[q]) return T2B_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(partials[q]) & 15) || (reinterpret_cast<uintptr_t>(flags[q]) & 3))
      return T2B_ERR_ALIGN;
    P.part[q] = partials[q];
    P.flags[q] = flags[q];
  }
  if ((reinterpret_cast<uintptr_t>(x_resid) | reinterpret_cast<uintptr_t>(next_w) |
       reinterpret_cast<uintptr_t>(xw_out)) & 15)
    return T2B_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(state) & 15) return T2B_ERR_ALIGN;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  P.state = state;
  P.rank = rank;
  P.world = world;
  P.ybf16 = y_dtype == T2B_DTYPE_BF16;
  P.x = x_resid;
  P.ssq = ssq_out;
  P.w = reinterpret_cast<const __nv_bfloat16*>(next_w);
  P.xw = reinterpret_cast<__half*>(xw_out);
  P.M = M;
  P.H = H;
  P.err = error_word(st);
  return launch_pdl(tp_allreduce_residual_kernel, dim3(M), dim3(TPAR_THREADS), 0, st, P);
}
