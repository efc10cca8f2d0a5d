// W4A16 group-128 GEMM on the 5th-generation tensor cores (tcgen05), for
// decode batches of 16..64 rows per CTA, with the same fused prologues /
// epilogues as the CUDA-core GEMV.
//
// Swap-AB formulation: D[128 weight rows, Bp batch rows] = W_tile[128, k] . X[Bp, k]^T
//   * MMA M = 128 (one T2B weight tile), N = Bp (batch padded to 16/32/64), K = 16.
//   * A (weights) lives in TENSOR MEMORY: producer warps unpack each nibble
//     pair straight into a bf16x2 register ((w >> 4j) & 0x000F000F | 0x4300_4300
//     = the exact bf16 values 128+q) and tcgen05.st it into TMEM -- no shared
//     memory round trip for the 4x-expanded weights.
//   * B (activations) is written once per CTA into shared memory in the
//     128-byte-swizzled K-major layout and read by the MMA through a UMMA
//     shared-memory descriptor.
//   * Scale and zero are applied per group AFTER the MMA: each group g gets
//     its own fp32 TMEM accumulator P_g = sum_k (128+q) x, and the drain
//     computes y += s_g * (P_g - (128+z_g) * sum_k x).  Products are exact,
//     the weights are never rounded, and the per-weight ALU cost is ~1 op.
//   * K order: a bf16x2 register holds nibbles (j, j+4) of a word, so within
//     every 8-k block the MMA sees k in the order 0,4,1,5,2,6,3,7; the X tile
//     is written in the same order, so the contraction is unchanged.
//   * Raw int4 blocks (8 KB + 512 B of meta per 128x128 tile-group) arrive by
//     1-D TMA bulk copies issued BEFORE the programmatic-dependent-launch
//     wait, so weight streaming overlaps the previous kernel's tail.
//
// Roles (256 threads): warps 0-3 own TMEM lane quarters 0-3 (weight rows
// 32w..32w+31): dequant producers, then accumulator drain.  Warp 4 allocates
// TMEM and one lane issues the MMAs.  All 8 warps build the X tile.  Every
// mbarrier wait is time-bounded; on timeout the CTA records T2B_ERR_TIMEOUT,
// frees its TMEM and exits.

#include "linear_common.cuh"
#include "launch.cuh"

namespace t2b {

// ---------------------------------------------------------------------------
// tcgen05 wrappers
// ---------------------------------------------------------------------------
T2B_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
T2B_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
T2B_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
T2B_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
T2B_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] . B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate)
T2B_DEV void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
T2B_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
T2B_DEV void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
T2B_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
T2B_DEV void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
T2B_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row core groups 1024 B apart.
T2B_DEV uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1u << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D fp32, A/B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__host__ __device__ constexpr uint32_t pow2_cols(uint32_t n) {
  uint32_t c = 32;
  while (c < n) c <<= 1;
  return c;
}

template <int BP, int S>
struct TcSmem {
  static constexpr int X_GROUP = BP * 256;                 // bf16 [2 atoms][BP][128 B]
  static constexpr int OFF_X = 0;
  static constexpr int OFF_RAW = OFF_X + S * X_GROUP;      // [S][8 KB]
  static constexpr int OFF_META = OFF_RAW + S * BLOCK_BYTES;
  static constexpr int OFF_TILE = OFF_META + S * TILE_N * 4;
  static constexpr int OFF_XSUM = OFF_TILE + BP * TILE_N * 4;
  static constexpr int OFF_SCR = OFF_XSUM + S * BP * 4;
  static constexpr int OFF_BAR = OFF_SCR + 8 * BP * 4;
  static constexpr int NBAR = S + 5;                         // raw_full[S], a_full[2], a_empty[2], acc_full
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int OFF_FLAG = OFF_TMEM + 8;
  static constexpr int BYTES = OFF_FLAG + 8 + 1024;          // + slack to 1024-align the base
  static constexpr uint32_t A_COL = 0;                       // 2 stages x 64 columns
  static constexpr uint32_t ACC_COL = 128;                   // S accumulators x BP columns
  static constexpr uint32_t TMEM_COLS = pow2_cols(128 + S * BP);
};

T2B_DEV uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int BP, int S, int PRO, int EPI>
__global__ void __launch_bounds__(256, 1) w4a16_tc_kernel(const LinearParams p) {
  using L = TcSmem<BP, S>;
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = sm + L::OFF_X;
  uint8_t* raw = sm + L::OFF_RAW;
  const uint32_t* rmeta = reinterpret_cast<const uint32_t*>(sm + L::OFF_META);
  float* tile_acc = reinterpret_cast<float*>(sm + L::OFF_TILE);
  float* xsum = reinterpret_cast<float*>(sm + L::OFF_XSUM);
  float* scratch = reinterpret_cast<float*>(sm + L::OFF_SCR);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* raw_full = bars;
  uint64_t* a_full = bars + S;
  uint64_t* a_empty = bars + S + 2;
  uint64_t* acc_full = bars + S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::OFF_TMEM);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::OFF_FLAG);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, mblk = blockIdx.z;
  const int g0 = split * S;
  const int m0 = mblk * BP;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) mbar_init(&raw_full[i], 1);
    mbar_init(&a_full[0], 4);
    mbar_init(&a_full[1], 4);
    mbar_init(&a_empty[0], 1);
    mbar_init(&a_empty[1], 1);
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // raw weight blocks of this CTA: constant data, fetched before the PDL wait
  if (threadIdx.x == 0) {
    for (int gl = 0; gl < S; ++gl) {
      mbar_arrive_expect_tx(&raw_full[gl], BLOCK_BYTES + TILE_N * 4);
      bulk_g2s(raw + gl * BLOCK_BYTES, p.qw + qw_block_offset(tile, g0 + gl, p.G), BLOCK_BYTES, &raw_full[gl]);
      bulk_g2s(sm + L::OFF_META + gl * TILE_N * 4, p.meta + meta_block_offset(tile, g0 + gl, p.G), TILE_N * 4,
               &raw_full[gl]);
    }
  }

  grid_dep_wait();
  grid_dep_launch();

  // TMEM is taken only after the wait: a dependent grid parked on its own
  // wait never holds columns this grid still needs.
  if (warp == 4) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }

  // ---- X tile: bf16, 128B-swizzled K-major, k permuted 0,4,1,5,2,6,3,7 ----
  if (PRO == PRO_RMSNORM) {
    for (int b = threadIdx.x; b < BP; b += 256) {
      const int m = m0 + b;
      scratch[b] = (m < p.M) ? rsqrtf(p.ssq[m] / (float)p.K + p.eps) : 0.f;
    }
    __syncthreads();
  }
  for (int t = threadIdx.x; t < S * BP * 16; t += 256) {
    const int c16 = t & 15, gb = t >> 4;
    const int gl = gb / BP, b = gb - gl * BP;
    const int m = m0 + b;
    const int k = (g0 + gl) * GROUP + c16 * 8;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.f;
    if (m < p.M) {
      if (PRO == PRO_RMSNORM) {
        const float* xr = reinterpret_cast<const float*>(p.x) + (size_t)m * p.x_ld + k;
        const float4 a0 = *reinterpret_cast<const float4*>(xr);
        const float4 a1 = *reinterpret_cast<const float4*>(xr + 4);
        const uint4 wn = *reinterpret_cast<const uint4*>(p.norm_w + k);
        const float xv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t ww[4] = {wn.x, wn.y, wn.z, wn.w};
        const float r = scratch[b];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float w = (e & 1) ? __uint_as_float(ww[e >> 1] & 0xffff0000u) : __uint_as_float(ww[e >> 1] << 16);
          v[e] = round_bf16((xv[e] * r) * w);   // model.py:179-181, A16
        }
      } else if (p.x_dtype == T2B_DTYPE_BF16) {
        const uint4 xb = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.x) +
                                                         (size_t)m * p.x_ld + k);
        const uint32_t ww[4] = {xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int e = 0; e < 8; ++e)
          v[e] = (e & 1) ? __uint_as_float(ww[e >> 1] & 0xffff0000u) : __uint_as_float(ww[e >> 1] << 16);
      } else {  // fp32 activations rounded to bf16
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = round_bf16(reinterpret_cast<const float*>(p.x)[(size_t)m * p.x_ld + k + e]);
      }
    }
    const uint4 packed = make_uint4(pack_bf16x2(v[0], v[4]), pack_bf16x2(v[1], v[5]), pack_bf16x2(v[2], v[6]),
                                    pack_bf16x2(v[3], v[7]));
    const int atom = c16 >> 3, cc = c16 & 7;
    *reinterpret_cast<uint4*>(xs + gl * L::X_GROUP + atom * (BP * 128) + b * 128 + ((cc ^ (b & 7)) << 4)) = packed;
    float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    s += __shfl_xor_sync(0xffffffffu, s, 8);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (c16 == 0) xsum[gl * BP + b] = s;
  }
  fence_proxy_async();  // generic-proxy smem writes -> visible to the tensor core
  maybe_clear_ssq(p, tile == 0 && split == 0 && mblk == 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  constexpr uint32_t IDESC = idesc_bf16(TILE_N, BP);

  if (warp < 4) {
    // ---- producers: row r's nibbles -> bf16x2 (128+q) -> TMEM lane r ----
    const int r = warp * 32 + lane;
    const uint32_t lane_base = tbase + ((uint32_t)(warp * 32) << 16);
    for (int gl = 0; gl < S; ++gl) {
      const int stage = gl & 1;
      bool ok = true;
      if (gl >= 2) ok = mbar_wait_bounded(&a_empty[stage], ((gl - 2) >> 1) & 1, p.err);
      if (ok) ok = mbar_wait_bounded(&raw_full[gl], 0, p.err);
      if (!ok) {
        *abort_flag = 1;
        break;
      }
#pragma unroll
      for (int pc = 0; pc < 4; ++pc) {
        const uint4 v = *reinterpret_cast<const uint4*>(raw + gl * BLOCK_BYTES + pc * 2048 + r * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t cols[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          cols[4 * j + 0] = (w[j] & 0x000F000Fu) | 0x43004300u;
          cols[4 * j + 1] = ((w[j] >> 4) & 0x000F000Fu) | 0x43004300u;
          cols[4 * j + 2] = ((w[j] >> 8) & 0x000F000Fu) | 0x43004300u;
          cols[4 * j + 3] = ((w[j] >> 12) & 0x000F000Fu) | 0x43004300u;
        }
        tmem_st16(lane_base + L::A_COL + stage * 64 + pc * 16, cols);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[stage]);
    }
  } else if (warp == 4 && lane == 0) {
    // ---- MMA issuer ----
    for (int gl = 0; gl < S; ++gl) {
      const int stage = gl & 1;
      if (!mbar_wait_bounded(&a_full[stage], (gl >> 1) & 1, p.err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t xg = smem_u32(xs + gl * L::X_GROUP);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t bdesc = sdesc_sw128(xg + (ks >> 2) * (BP * 128) + (ks & 3) * 32);
        mma_ts(tbase + L::ACC_COL + gl * BP, tbase + L::A_COL + stage * 64 + ks * 8, bdesc, IDESC, ks > 0);
      }
      mma_commit(&a_empty[stage]);
    }
    mma_commit(acc_full);
  }

  // ---- drain: y[b] = sum_g s_g * (P_g[b] - (128+z_g) * xsum_g[b]) ----
  if (warp < 4) {
    const int r = warp * 32 + lane;
    const uint32_t lane_base = tbase + ((uint32_t)(warp * 32) << 16);
    const bool ok = (*abort_flag == 0) && mbar_wait_bounded(acc_full, 0, p.err);
    if (!ok) *abort_flag = 1;
    tc_fence_after();
    float y[BP];
#pragma unroll
    for (int b = 0; b < BP; ++b) y[b] = 0.f;
    if (ok) {
#pragma unroll
      for (int gl = 0; gl < S; ++gl) {
        const uint32_t mw = rmeta[gl * TILE_N + r];
        const float s = __half2float(__ushort_as_half((unsigned short)(mw & 0xffffu)));
        const float zo = 128.f + (float)((mw >> 16) & 0x1fu);
#pragma unroll
        for (int cb = 0; cb < BP / 16; ++cb) {
          uint32_t v[16];
          tmem_ld16(lane_base + L::ACC_COL + gl * BP + cb * 16, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int b = cb * 16 + e;
            y[b] = fmaf(s, __uint_as_float(v[e]) - zo * xsum[gl * BP + b], y[b]);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < BP; ++b) tile_acc[b * TILE_N + r] = y[b];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tbase, L::TMEM_COLS);
  }
  if (*abort_flag) return;

  if (!splitk_fixup<BP>(p, tile_acc, tile, split, mblk, 256)) return;
  tile_epilogue<BP, EPI>(p, tile_acc, scratch, tile, m0);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int pick_bp(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : 64; }

// groups per CTA (1, 2 or 4): grow while the grid keeps >= 2 CTAs per SM,
// or while the split count would exceed 24 (workspace size).
static int pick_s(int N, int K, int mblocks) {
  const int G = K / GROUP;
  const long tiles = (long)(N / TILE_N) * mblocks;
  int s = 1;
  while (s < 4 && G % (2 * s) == 0 && (tiles * (G / (2 * s)) >= 2L * 148 || G / s > 24)) s *= 2;
  return s;
}

size_t tc_ws_bytes(int M, int N, int K) {
  const int BP = pick_bp(M);
  const int mblocks = (M + BP - 1) / BP;
  const int ksplit = (K / GROUP) / pick_s(N, K, mblocks);
  if (ksplit == 1) return 0;
  size_t part = ((size_t)mblocks * ksplit * BP * N * sizeof(float) + 255) & ~size_t(255);
  return part + (((size_t)mblocks * (N / TILE_N) * sizeof(int) + 255) & ~size_t(255));
}

template <int BP, int S, int PRO, int EPI>
static int tc_launch_t(LinearParams& p, dim3 grid, cudaStream_t st) {
  auto kern = w4a16_tc_kernel<BP, S, PRO, EPI>;
  const size_t smem = TcSmem<BP, S>::BYTES;
  if (allow_smem(kern, smem) != T2B_OK) return T2B_ERR_LAUNCH;
  return launch_pdl(kern, grid, dim3(256), smem, st, p);
}

template <int PRO, int EPI>
static int tc_dispatch(LinearParams& p, int BP, int S, dim3 grid, cudaStream_t st) {
#define T2B_TCASE(bp, s) \
  if (BP == bp && S == s) return tc_launch_t<bp, s, PRO, EPI>(p, grid, st);
  T2B_TCASE(16, 1) T2B_TCASE(16, 2) T2B_TCASE(16, 4) T2B_TCASE(32, 1) T2B_TCASE(32, 2) T2B_TCASE(32, 4)
  T2B_TCASE(64, 1) T2B_TCASE(64, 2) T2B_TCASE(64, 4)
#undef T2B_TCASE
  return T2B_ERR_ARG;
}

int tc_launch(LinearParams& p, int pro, int epi, void* ws, size_t ws_bytes, cudaStream_t st) {
  const int BP = pick_bp(p.M);
  const int mblocks = (p.M + BP - 1) / BP;
  const int S = pick_s(p.N, p.K, mblocks);
  p.kslice = S * GROUP;
  p.ksplit = p.K / p.kslice;
  if (ws_bytes < tc_ws_bytes(p.M, p.N, p.K) || (p.ksplit > 1 && ws == nullptr)) return T2B_ERR_WORKSPACE;
  if (p.x_dtype == T2B_DTYPE_F16 && pro == PRO_ACT) return T2B_ERR_ARG;
  size_t part = ((size_t)mblocks * p.ksplit * BP * p.N * sizeof(float) + 255) & ~size_t(255);
  p.ws_part = reinterpret_cast<float*>(ws);
  p.ws_cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + part);
  dim3 grid(p.N / TILE_N, p.ksplit, mblocks);
  if (pro == PRO_ACT && epi == EPI_STORE) return tc_dispatch<PRO_ACT, EPI_STORE>(p, BP, S, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_STORE) return tc_dispatch<PRO_RMSNORM, EPI_STORE>(p, BP, S, grid, st);
  if (pro == PRO_ACT && epi == EPI_RESIDUAL) return tc_dispatch<PRO_ACT, EPI_RESIDUAL>(p, BP, S, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_SWIGLU) return tc_dispatch<PRO_RMSNORM, EPI_SWIGLU>(p, BP, S, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_QKV) return tc_dispatch<PRO_RMSNORM, EPI_QKV>(p, BP, S, grid, st);
  return T2B_ERR_ARG;
}

}  // namespace t2b
