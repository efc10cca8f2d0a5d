// W4A16 group-128 GEMM for many activation rows (a prefill chunk: M = B x
// chunk tokens), on tcgen05, with the decode layer's fused epilogues.
//
// Work unit: one 128-row weight tile (n) x one block of BM = 128 activation
// rows (m), over all K.  Persistent CTAs (one per SM) walk the units with the
// weight tile fastest, so the CTAs running at once share an activation block.
// Per 128-k group of a unit:
//   * all 8 warps dequantise the tile's int4 rows straight from global memory
//     into a TMEM A stage (bf16 (q - z) * s pairs, the decode kernel's
//     arithmetic; warp w writes its TMEM lane quarter w % 4, pieces 2(w/4) and
//     2(w/4)+1), a ring of NA stages freed by tcgen05.commit;
//   * the activations arrive by TMA (two 64-k x BM-row boxes, 128-byte swizzle
//     = the UMMA K-major layout) into a ring of NX stages, issued NX-1 groups
//     ahead by thread 0, which also issues the 8 MMAs (M 128, N BM, K 16) of
//     each group into the fp32 TMEM accumulator (TS form: A from TMEM).
// The MMAs of one group overlap the dequantisation of the next.  At the end
// of a unit all warps drain the accumulator (times the RMSNorm row scale) into
// shared memory and run the fused epilogue of the decode path
// (linear_common.cuh) on the [BM][128] tile.  The weight tile is dequantised
// once per activation block (M/BM times in all), not once per 16-row batch
// tile as the decode kernel would.
// Every mbarrier wait is time-bounded; a CTA that gives up records
// T2B_ERR_TIMEOUT, stops issuing, waits (bounded) for its issued MMAs and
// frees its TMEM.

#include <algorithm>

#include "linear_common.cuh"
#include "launch.cuh"
#include "tmap.cuh"
#include "tcgen05.cuh"

namespace t2b {

constexpr int PF_BM = 128;        // activation rows per unit (MMA N)
constexpr int PF_NX = 3;          // activation stages
constexpr int PF_NA = 4;          // TMEM A stages (64 columns each)
constexpr int PF_GT = 256;        // threads
constexpr uint32_t PF_TMEM_COLS = 512;   // accumulator [0, BM) + A stages from column 128

struct PfLayout {
  static constexpr int X_STAGE = PF_BM * 256;                      // 2 atoms of [BM][128 B]
  static constexpr int OFF_TILE = PF_NX * X_STAGE;                 // fp32 [BM][128]
  static constexpr int OFF_SCR = OFF_TILE + PF_BM * TILE_N * 4;    // fp32 [2*BM] epilogue scratch
  static constexpr int OFF_RS = OFF_SCR + 2 * PF_BM * 4;           // fp32 [BM] row scales
  static constexpr int OFF_BAR = OFF_RS + PF_BM * 4;               // x_full[NX] free_x[NX] free_a[NA] acc_full done
  static constexpr int OFF_TMEM = OFF_BAR + (2 * PF_NX + PF_NA + 2) * 8;
  static constexpr int OFF_FLAG = OFF_TMEM + 8;
  static constexpr int BYTES = OFF_FLAG + 8 + 1024;                // + slack to 1024-align the base
};

template <int PRO, int EPI>
__global__ void __launch_bounds__(PF_GT, 1) w4a16_prefill_kernel(const __grid_constant__ LinearParams p) {
  using L = PfLayout;
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  float* tile_acc = reinterpret_cast<float*>(sm + L::OFF_TILE);
  float* scratch = reinterpret_cast<float*>(sm + L::OFF_SCR);
  float* rowscale = reinterpret_cast<float*>(sm + L::OFF_RS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* x_full = bars;                       // [NX]
  uint64_t* free_x = bars + PF_NX;               // [NX]
  uint64_t* free_a = bars + 2 * PF_NX;           // [NA]
  uint64_t* acc_full = bars + 2 * PF_NX + PF_NA;
  uint64_t* done = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::OFF_TMEM);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::OFF_FLAG);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;
  const int n_tiles = p.N / TILE_N;
  const int n_units = n_tiles * ((p.M + PF_BM - 1) / PF_BM);
  const int my_units = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int total = my_units * G;                // groups this CTA runs (global counter `it`)
  constexpr uint32_t IDESC = idesc_bf16(TILE_N, PF_BM);
  constexpr uint32_t A0 = PF_BM;                 // first A-stage column

  if (threadIdx.x == 0) {
    for (int i = 0; i < PF_NX; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&free_x[i], 1);
    }
    for (int i = 0; i < PF_NA; ++i) mbar_init(&free_a[i], 1);
    mbar_init(acc_full, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, PF_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  grid_dep_launch();   // this CTA holds its TMEM: dependents may start
  grid_dep_wait();     // activations, row sums and the residual come from earlier kernels
  maybe_clear_ssq(p, blockIdx.x == 0, threadIdx.x, PF_GT);

  // unit -> (weight tile, activation block), weight tile fastest
  auto unit_of = [&](int j) { return (int)blockIdx.x + j * (int)gridDim.x; };
  int x_issued = 0, x_waited = 0;   // thread 0: activation loads issued / consumed
  auto issue_x = [&](int it) {   // thread 0: TMA of group `it` of this CTA's sequence
    ++x_issued;
    const int s = it % PF_NX;
    const int u = unit_of(it / G), g = it % G;
    const int m0 = (u / n_tiles) * PF_BM;
    uint8_t* dst = sm + s * L::X_STAGE;
    mbar_arrive_expect_tx(&x_full[s], (uint32_t)L::X_STAGE);
    tma_load_2d(dst, &p.xmap, g * GROUP, m0, &x_full[s]);
    tma_load_2d(dst + PF_BM * 128, &p.xmap, g * GROUP + 64, m0, &x_full[s]);
  };
  if (threadIdx.x == 0)
    for (int it = 0; it < PF_NX - 1 && it < total; ++it) issue_x(it);

  const int q4 = warp & 3, hw = warp >> 2;      // TMEM lane quarter, piece pair / column half
  const int r = q4 * 32 + lane;                 // weight row of this thread (TMEM lane)
  const uint32_t lane_base = tbase + ((uint32_t)(q4 * 32) << 16);
  int it = 0;
  bool ok = true;
  for (int j = 0; j < my_units && ok; ++j) {
    const int u = unit_of(j);
    const int tile = u % n_tiles, m0 = (u / n_tiles) * PF_BM;
    if (PRO == PRO_RMSNORM && threadIdx.x < PF_BM) {
      const int m = m0 + threadIdx.x;
      rowscale[threadIdx.x] = (m < p.M) ? rsqrtf(p.ssq[m] / (float)p.K + p.eps) : 0.f;   // model.py:179-180
    }
    for (int g = 0; g < G; ++g, ++it) {
      // ---- this thread's raw nibbles and meta (independent of the pipeline) ----
      const uint8_t* blk = p.qw + qw_block_offset(tile, g, G);
      const uint4 v0 = __ldg(reinterpret_cast<const uint4*>(blk + (2 * hw) * 2048 + r * 16));
      const uint4 v1 = __ldg(reinterpret_cast<const uint4*>(blk + (2 * hw + 1) * 2048 + r * 16));
      const uint32_t mw = __ldg(p.meta + meta_block_offset(tile, g, G) + r);
      const int sa = it % PF_NA;
      bool w_ok = true;
      if (it >= PF_NA) w_ok = mbar_wait_bounded(&free_a[sa], ((it / PF_NA) - 1) & 1, p.err);
      if (__syncthreads_or(!w_ok)) {
        ok = false;
        break;
      }
      // ---- dequant into TMEM A stage sa: column c of the stage holds k 2c, 2c+1 ----
      const __nv_bfloat16 sb = __float2bfloat16_rn(__half2float(__ushort_as_half((unsigned short)(mw & 0xffffu))));
      const __nv_bfloat16 zb = __float2bfloat16_rn(128.f + (float)((mw >> 16) & 0x1fu));
      const __nv_bfloat162 s2 = __halves2bfloat162(sb, sb);
      const __nv_bfloat162 z2 = __halves2bfloat162(zb, zb);
      __syncwarp();   // tcgen05.st is warp-aligned: thread 0 may arrive late from the issue block
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 v = h ? v1 : v0;
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t cols[16];
#pragma unroll
        for (int jw = 0; jw < 4; ++jw)
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            // slot t holds k 2t, slot t+4 holds k 2t+1: the mask-or is the pair as 128+q
            const uint32_t biased = ((w[jw] >> (4 * t)) & 0x000F000Fu) | 0x43004300u;
            const __nv_bfloat162 q2 = *reinterpret_cast<const __nv_bfloat162*>(&biased);
            const __nv_bfloat162 d2 = __hmul2(__hsub2(q2, z2), s2);   // (q - z) exact, one rounding of * s
            cols[4 * jw + t] = *reinterpret_cast<const uint32_t*>(&d2);
          }
        tmem_st16(lane_base + A0 + (uint32_t)(sa * 64 + (2 * hw + h) * 16), cols);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncthreads();
      // ---- thread 0: this group's MMAs, then the activation TMA NX-1 groups ahead ----
      if (threadIdx.x == 0) {
        tc_fence_after();
        const int sx = it % PF_NX;
        bool t_ok = mbar_wait_bounded(&x_full[sx], (it / PF_NX) & 1, p.err);
        if (t_ok) ++x_waited;
        if (t_ok) {
          const uint32_t xa = smem_u32(sm + sx * L::X_STAGE);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t bdesc = sdesc_sw128(xa + (ks >> 2) * (PF_BM * 128) + (ks & 3) * 32);
            mma_ts(tbase, tbase + A0 + sa * 64 + ks * 8, bdesc, IDESC, (g > 0 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&free_a[sa]);
          mma_commit(&free_x[sx]);
          if (g == G - 1) mma_commit(acc_full);
          const int nx = it + PF_NX - 1;   // its stage was last read by group it-1
          if (nx < total) {
            if (nx >= PF_NX) t_ok = mbar_wait_bounded(&free_x[nx % PF_NX], ((nx / PF_NX) - 1) & 1, p.err);
            if (t_ok) issue_x(nx);
          }
        }
        if (!t_ok) *abort_flag = 1;
      }
    }
    if (!ok || __syncthreads_or(*abort_flag != 0)) {
      ok = false;
      break;
    }
    // ---- drain: accumulator column b (activation row m0+b) x lane r -> tile_acc[b][r] ----
    const bool a_ok = mbar_wait_bounded(acc_full, j & 1, p.err);
    if (__syncthreads_or(!a_ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    __syncwarp();
#pragma unroll 1
    for (int c0 = hw * (PF_BM / 2); c0 < (hw + 1) * (PF_BM / 2); c0 += 32) {
      uint32_t v[32];
      tmem_ld32(lane_base + (uint32_t)c0, v);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int b = c0 + e;
        float y = __uint_as_float(v[e]);
        if (PRO == PRO_RMSNORM) y *= rowscale[b];
        tile_acc[b * TILE_N + r] = y;
      }
    }
    tc_fence_before();
    __syncthreads();
    tile_epilogue<EPI>(p, tile_acc, scratch, tile, m0, PF_BM);
    __syncthreads();
  }
  if (!ok) *abort_flag = 1;
  // every MMA issued here has retired before TMEM is released, and (after an
  // abort) every activation load issued here has landed before the CTA exits
  if (threadIdx.x == 0) {
    mma_commit(done);
    mbar_wait_bounded(done, 0, p.err);
    for (int w = x_waited; w < x_issued; ++w) mbar_wait_bounded(&x_full[w % PF_NX], (w / PF_NX) & 1, p.err);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, PF_TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// Rows at or above this count take this kernel (env T2B_PREFILL_MIN_M overrides).
int prefill_min_m() {
  const char* e = getenv("T2B_PREFILL_MIN_M");
  if (e && *e) {
    const int v = atoi(e);
    if (v > 0) return v;
  }
  return 257;
}

template <int PRO, int EPI>
static int pf_launch_t(LinearParams& p, cudaStream_t st) {
  auto kern = w4a16_prefill_kernel<PRO, EPI>;
  const size_t smem = PfLayout::BYTES;
  if (allow_smem(kern, smem) != T2B_OK) return T2B_ERR_LAUNCH;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  const int units = (p.N / TILE_N) * ((p.M + PF_BM - 1) / PF_BM);
  const int grid = std::max(1, std::min(sms, units));
  return launch_pdl(kern, dim3(grid), dim3(PF_GT), smem, st, p);
}

int prefill_launch(LinearParams& p, int pro, int epi, cudaStream_t st) {
  if (p.x_dtype != T2B_DTYPE_BF16 || p.N % TILE_N || p.K % GROUP) return T2B_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(p.x) & 15) return T2B_ERR_ALIGN;
  if ((p.x_ld * 2) % 16) return T2B_ERR_ALIGN;
  cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)p.M};
  cuuint64_t strides[1] = {(cuuint64_t)p.x_ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)PF_BM};
  cuuint32_t estr[2] = {1, 1};
  const EncodeTiledFn encode = encode_tiled();
  if (encode == nullptr) return T2B_ERR_LAUNCH;
  if (encode(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p.x), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return T2B_ERR_ARG;
  p.kslice = p.K;
  p.ksplit = 1;
  if (pro == PRO_ACT && epi == EPI_STORE) return pf_launch_t<PRO_ACT, EPI_STORE>(p, st);
  if (pro == PRO_RMSNORM && epi == EPI_STORE) return pf_launch_t<PRO_RMSNORM, EPI_STORE>(p, st);
  if (pro == PRO_ACT && epi == EPI_RESIDUAL) return pf_launch_t<PRO_ACT, EPI_RESIDUAL>(p, st);
  if (pro == PRO_RMSNORM && epi == EPI_SWIGLU) return pf_launch_t<PRO_RMSNORM, EPI_SWIGLU>(p, st);
  if (pro == PRO_RMSNORM && epi == EPI_QKV) return pf_launch_t<PRO_RMSNORM, EPI_QKV>(p, st);
  return T2B_ERR_ARG;
}

}  // namespace t2b
