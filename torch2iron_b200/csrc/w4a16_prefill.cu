// W4A16 group-128 GEMM for many activation rows (a prefill chunk: M = B x
// chunk tokens), on tcgen05, with the decode layer's fused epilogues.
//
// Work unit: one 128-row weight tile (n) x one block of BM = 128 activation
// rows (m), over all K.  Persistent CTAs (one per SM) walk the units with the
// weight tile fastest, so the CTAs running at once share an activation block.
// Warp roles (608 threads), each a pipeline stage joined by mbarriers:
//   * warp 14, weights: one bulk copy per group of the tile's raw int4 block
//     (8 KB) and meta (512 B) into a ring of NR shared-memory stages
//     (constant data: this runs ahead of the dependency wait);
//   * warps 0-7, producers: warp w covers TMEM lane quarter w % 4 (weight
//     rows) and the 64-k half w / 4 of each group: it reads its rows' nibbles
//     and meta from the raw stage, dequantises to bf16 (q - z) * s pairs (the
//     decode kernel's arithmetic) and tcgen05.st's them into a ring of NA
//     TMEM A stages (two warps per scheduler hide the dequant latency);
//   * warp 12, TMA: the activations of each group (two 64-k x BM-row boxes,
//     128-byte swizzle = the UMMA K-major layout) into a ring of NX stages;
//   * warp 13, MMA: 8 tcgen05.mma (M 128, N BM, K 16, A from TMEM) per group
//     into one of two fp32 TMEM accumulators, freeing A and X stages by
//     tcgen05.commit;
//   * warps 8-11 and 15-18, epilogue: drain the other accumulator (times the
//     RMSNorm row scale) into shared memory -- each group of four warps half
//     of the tile's activation rows -- and run the decode path's fused
//     epilogue (linear_common.cuh) on the [BM][128] tile with all eight,
//     while the MMAs of the next unit run (the epilogue bounded this kernel
//     with four warps).
// A weight tile is dequantised once per activation block (M/BM times in all).
// Every mbarrier wait is time-bounded; a role that gives up records
// T2B_ERR_TIMEOUT and raises the CTA's abort flag, the others stop at their
// next wait; before TMEM is freed the MMA warp waits for its issued MMAs and
// the TMA and weight warps for their issued loads.

#include <algorithm>

#include "linear_common.cuh"
#include "launch.cuh"
#include "tmap.cuh"
#include "tcgen05.cuh"

namespace t2b {

constexpr int PF_BM = 128;               // activation rows per unit (MMA N)
constexpr int PF_NX = 3;                 // activation stages
constexpr int PF_NA = 4;                 // TMEM A stages (64 columns each)
constexpr int PF_NR = 4;                 // raw weight stages
constexpr int PF_RAW = BLOCK_BYTES + Q4NX_META_WORDS * 4;   // int4 block + meta of one (tile, group), either format
constexpr int PF_GT = 608;               // threads: 8 producer, 8 epilogue, TMA, MMA, weight warps
constexpr int PF_EPI = 256;              // epilogue threads: warps 8-11 and 15-18
constexpr uint32_t PF_TMEM_COLS = 512;   // accumulators [0, 2*BM), A stages from column 2*BM
constexpr uint32_t PF_A0 = 2 * PF_BM;

struct PfLayout {
  static constexpr int X_STAGE = PF_BM * 256;                      // 2 atoms of [BM][128 B]
  static constexpr int OFF_TILE = PF_NX * X_STAGE;                 // fp32 [BM][128]
  static constexpr int OFF_SCR = OFF_TILE + PF_BM * TILE_N * 4;    // fp32 [2*BM] epilogue scratch
  static constexpr int OFF_RS = OFF_SCR + 2 * PF_BM * 4;           // fp32 [BM] row scales
  static constexpr int OFF_RAW = OFF_RS + PF_BM * 4;               // [NR][8 KB int4 | 512 B (T2B) or 2 KB (Q4NX) meta]
  static constexpr int N_BARS = 2 * PF_NX + 2 * PF_NA + 2 * PF_NR + 4 + 1;
  static constexpr int OFF_BAR = OFF_RAW + PF_NR * PF_RAW;
  static constexpr int OFF_TMEM = OFF_BAR + N_BARS * 8;
  static constexpr int OFF_FLAG = OFF_TMEM + 8;
  static constexpr int BYTES = OFF_FLAG + 8 + 1024;                // + slack to 1024-align the base
};

// Trace build only (-DT2B_TRACE): SM cycles each role spends waiting, per CTA
// record (t[1] MMA on A stages, t[2] MMA on activations, t[3] MMA on a free
// accumulator, t[4] producers on raw weights, t[5] producers on a free A
// stage, t[6] epilogue on a finished accumulator, t[7] the CTA's whole run).
#ifdef T2B_TRACE
#define PF_CLK(v) const long long v = clock64()
#define PF_ADD(acc, t0) (acc) += clock64() - (t0)
#define PF_PUT(slot, v) t2b::g_trace[t2b_trace_slot].t[(slot)] = (unsigned long long)(v)
#else
#define PF_CLK(v)
#define PF_ADD(acc, t0)
#define PF_PUT(slot, v)
#endif

// Named barrier among the eight epilogue warps (id 1; 0 is __syncthreads).
T2B_DEV void epi_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Epilogues for a [BM][128] tile with many rows.  Same arithmetic as the
// decode path's (linear_common.cuh), but latency-batched: the decode
// epilogues take one batch row per warp pass and wait on its global loads
// (position, then its RoPE row; or its residual row) before the next, which
// for 128 rows costs tens of microseconds per tile.  Here a warp fetches the
// positions / sequences of 32 of its rows with one load per lane and issues
// the dependent loads of R rows before using any of them.
// ---------------------------------------------------------------------------
template <int HD, int R>
T2B_DEV void pf_qkv_epilogue(const LinearParams& p, const float* tile_acc, int tile, int m0, int MB, int t, int nt) {
  constexpr int HPT = TILE_N / HD;    // heads per tile
  constexpr int LPH = HD / 4;         // lanes per head
  const int warp = t >> 5, lane = t & 31, nwarps = nt >> 5;
  const int hl = lane / LPH, d0 = (lane % LPH) * 4;
  const int head = tile * HPT + hl;
  const int nq = p.n_heads, nkv = p.n_kv;
  const bool is_q = head < nq, is_v = head >= nq + nkv;
  const __nv_bfloat16* nw = is_v ? nullptr : (is_q ? p.qn_w : p.kn_w);
  const float4 w = nw ? unpack_bf16x4(*reinterpret_cast<const uint2*>(nw + d0)) : make_float4(1.f, 1.f, 1.f, 1.f);
  __nv_bfloat16* q_out = reinterpret_cast<__nv_bfloat16*>(p.y);
  const int rows = MB > warp ? (MB - warp + nwarps - 1) / nwarps : 0;   // this warp's rows: warp + k*nwarps
  for (int k0 = 0; k0 < rows; k0 += 32) {
    const int ml = m0 + warp + (k0 + lane) * nwarps;   // the row whose metadata this lane fetches
    int lpos = -1, lseq = -1;
    if (k0 + lane < rows && ml < p.M) {
      lpos = __ldg(p.pos + ml);
      lseq = p.row_seq ? __ldg(p.row_seq + ml) : ml;
    }
    const int kn = min(32, rows - k0);
    for (int k1 = 0; k1 < kn; k1 += R) {
      float4 x[R], cs[R];
      int pos[R], sq[R];
      bool live[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        pos[i] = __shfl_sync(0xffffffffu, lpos, (k1 + i) & 31);
        sq[i] = __shfl_sync(0xffffffffu, lseq, (k1 + i) & 31);
        const int b = warp + (k0 + k1 + i) * nwarps;
        live[i] = k1 + i < kn && m0 + b < p.M;   // warp-uniform
        x[i] = live[i] ? *reinterpret_cast<const float4*>(tile_acc + b * TILE_N + lane * 4)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const bool pos_ok = pos[i] >= 0 && pos[i] < p.max_ctx;
        cs[i] = (live[i] && !is_v) ? __ldg(reinterpret_cast<const float4*>(p.angles + (size_t)(pos_ok ? pos[i] : 0) * HD + d0))
                                   : make_float4(1.f, 0.f, 1.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < R; ++i) {
        if (!live[i]) continue;   // warp-uniform
        const int b = warp + (k0 + k1 + i) * nwarps, m = m0 + b;
        const float4 xv = x[i];
        float ss = xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w;
#pragma unroll
        for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const bool pos_ok = pos[i] >= 0 && pos[i] < p.max_ctx;
        const bool in_cache = pos_ok && (!p.row_seq || (sq[i] >= 0 && sq[i] < p.n_seq));
        const size_t cm = (size_t)sq[i];
        if (is_v) {  // value head: stored as projected (model.py:250,263)
          if (in_cache)
            *reinterpret_cast<uint2*>(&p.v_cache[((cm * nkv + (head - nq - nkv)) * p.max_ctx + pos[i]) * HD + d0]) =
                pack_bf16x4(xv.x, xv.y, xv.z, xv.w);
          continue;
        }
        if (!is_q && !in_cache) continue;
        const float rs = nw ? rsqrtf(ss / (float)HD + p.eps) : 1.f;   // model.py:179-180 on the head
        const float x0 = xv.x * rs * w.x, x1 = xv.y * rs * w.y, x2 = xv.z * rs * w.z, x3 = xv.w * rs * w.w;
        const float4 c = cs[i];   // interleaved RoPE (model.py:184-196)
        const uint2 o = pack_bf16x4(x0 * c.x - x1 * c.y, x1 * c.x + x0 * c.y, x2 * c.z - x3 * c.w, x3 * c.z + x2 * c.w);
        if (is_q)
          *reinterpret_cast<uint2*>(&q_out[(size_t)m * p.y_ld + head * HD + d0]) = o;
        else
          *reinterpret_cast<uint2*>(&p.k_cache[((cm * nkv + (head - nq)) * p.max_ctx + pos[i]) * HD + d0]) = o;
      }
    }
  }
}

// x += y; sum of squares for the next RMSNorm; fp16(x * w_next): R residual
// rows in flight per thread (a warp's 128 elements are one row of the tile).
template <int R>
T2B_DEV void pf_residual_epilogue(const LinearParams& p, const float* tile_acc, int tile, int m0, int MB, int t,
                                  int nt) {
  const int lane = t & 31, row0 = tile * TILE_N;
  const int lr = (t * 4) % TILE_N;   // the same tile column for every pass (a pass is nt*4 elements, a multiple of 128)
  const float4 wn = p.xw_out ? unpack_bf16x4(*reinterpret_cast<const uint2*>(p.next_w + row0 + lr))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int base = 0; base < MB * TILE_N; base += nt * 4 * R) {
    float4 rv[R];
    bool live[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int idx = base + i * nt * 4 + t * 4, m = m0 + idx / TILE_N;
      live[i] = idx < MB * TILE_N && m < p.M;   // warp-uniform
      rv[i] = live[i] ? *reinterpret_cast<const float4*>(p.resid + (size_t)m * p.y_ld + row0 + lr)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
      if (!live[i]) continue;
      const int idx = base + i * nt * 4 + t * 4, m = m0 + idx / TILE_N;
      const size_t o = (size_t)m * p.y_ld + row0 + lr;
      const float4 tv = *reinterpret_cast<const float4*>(tile_acc + idx);
      const float4 v = make_float4(rv[i].x + tv.x, rv[i].y + tv.y, rv[i].z + tv.z, rv[i].w + tv.w);
      *reinterpret_cast<float4*>(p.resid + o) = v;
      if (p.xw_out)
        *reinterpret_cast<uint2*>(p.xw_out + o) = pack_f16x4(v.x * wn.x, v.y * wn.y, v.z * wn.z, v.w * wn.w);
      const float sq = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      if (lane == 0) atomicAdd(p.ssq_out + m, sq);
    }
  }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(PF_GT, 1) w4a16_prefill_kernel(const __grid_constant__ LinearParams p) {
  using L = PfLayout;
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  float* tile_acc = reinterpret_cast<float*>(sm + L::OFF_TILE);
  float* scratch = reinterpret_cast<float*>(sm + L::OFF_SCR);
  float* rowscale = reinterpret_cast<float*>(sm + L::OFF_RS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* x_full = bars;                          // [NX]
  uint64_t* x_empty = bars + PF_NX;                 // [NX]
  uint64_t* a_full = bars + 2 * PF_NX;              // [NA]
  uint64_t* a_empty = a_full + PF_NA;               // [NA]
  uint64_t* w_full = a_empty + PF_NA;               // [NR]
  uint64_t* w_empty = w_full + PF_NR;               // [NR]
  uint64_t* acc_full = w_empty + PF_NR;             // [2]
  uint64_t* acc_empty = acc_full + 2;               // [2]
  uint64_t* done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::OFF_TMEM);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::OFF_FLAG);
  volatile int* epi_abort = abort_flag + 1;   // written only by the epilogue warps, read after their barrier

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;
  const int n_tiles = p.N / TILE_N;
  const int n_units = n_tiles * ((p.M + PF_BM - 1) / PF_BM);
  const int my_units = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int total = my_units * G;   // groups this CTA runs, in order (global counter `it`)
  auto unit_of = [&](int j) { return (int)blockIdx.x + j * (int)gridDim.x; };
  T2B_TRACE_BEGIN(30 + EPI, p.N);
  PF_CLK(t_start);

  if (threadIdx.x == 0) {
    for (int i = 0; i < PF_NX; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < PF_NA; ++i) {
      mbar_init(&a_full[i], 8);     // one arrival per producer warp
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < PF_NR; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 8);    // one arrival per producer warp
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);  // one arrival per epilogue warp
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    *epi_abort = 0;
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

  if (warp < 8) {
    // ---- producers: weight row r, pieces 2h and 2h+1 of each group -> TMEM A stage
    //      (column c = k 2c, 2c+1) ----
    const int q4 = warp & 3, h = warp >> 2;
    const int r = q4 * 32 + lane;
    const bool f16 = p.x_dtype == T2B_DTYPE_F16;
    const uint32_t lane_base = tbase + ((uint32_t)(q4 * 32) << 16);
    long long w_wait = 0, a_wait = 0;
    (void)w_wait;
    (void)a_wait;
    for (int it = 0; it < total; ++it) {
      const int sr = it % PF_NR, sa = it % PF_NA;
      PF_CLK(tw0);
      bool ok = *abort_flag == 0 && mbar_wait_bounded(&w_full[sr], (it / PF_NR) & 1, p.err);
      PF_ADD(w_wait, tw0);
      if (!__all_sync(0xffffffffu, ok)) {
        *abort_flag = 1;
        break;
      }
      const uint8_t* raw = sm + L::OFF_RAW + sr * PF_RAW;
      uint4 v[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) v[j] = *reinterpret_cast<const uint4*>(raw + (2 * h + j) * 2048 + r * 16);
      const uint32_t* rmeta = reinterpret_cast<const uint32_t*>(raw + BLOCK_BYTES);
      const uint32_t mw = rmeta[r];
      uint32_t mq[2] = {0u, 0u};                 // Q4NX: the words of pieces 2h, 2h+1
      if (p.q4nx) {
        mq[0] = rmeta[(2 * h) * TILE_N + r];
        mq[1] = rmeta[(2 * h + 1) * TILE_N + r];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&w_empty[sr]);   // this warp is done with the raw stage
      PF_CLK(ta0);
      if (it >= PF_NA) ok = mbar_wait_bounded(&a_empty[sa], ((it / PF_NA) - 1) & 1, p.err);
      PF_ADD(a_wait, ta0);
      if (!__all_sync(0xffffffffu, ok)) {   // the warp takes the same branch before tcgen05.st
        *abort_flag = 1;
        break;
      }
      uint32_t z2, s2;
      if (f16) t2b_meta_pairs<true>(mw, z2, s2);
      else t2b_meta_pairs<false>(mw, z2, s2);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int pc = 2 * h + j;
        uint32_t cols[16];
        // weights in the activations' 16-bit type (T2B: slot t holds k 2t, slot t+4 k 2t+1)
        if (p.q4nx) {
          if (f16) dequant_piece_q4nx<true>(v[j], bf16_lo_f32(mq[j]), bf16_hi_f32(mq[j]), cols);
          else dequant_piece_q4nx<false>(v[j], bf16_lo_f32(mq[j]), bf16_hi_f32(mq[j]), cols);
        } else {
          if (f16) dequant_piece_t2b<true>(v[j], z2, s2, cols);
          else dequant_piece_t2b<false>(v[j], z2, s2, cols);
        }
        tmem_st16(lane_base + PF_A0 + (uint32_t)(sa * 64 + pc * 16), cols);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[sa]);
    }
    if (threadIdx.x == 0) {
      PF_PUT(4, w_wait);
      PF_PUT(5, a_wait);
    }
  } else if (warp == 12) {
    // ---- TMA: the activations of every group, NX stages ahead of the MMAs ----
    grid_dep_wait();   // x comes from the preceding kernel
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < total; ++it) {
        const int s = it % PF_NX;
        if (it >= PF_NX && !mbar_wait_bounded(&x_empty[s], ((it / PF_NX) - 1) & 1, p.err)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int g = it % G, m0 = (unit_of(it / G) / n_tiles) * PF_BM;
        uint8_t* dst = sm + s * L::X_STAGE;
        mbar_arrive_expect_tx(&x_full[s], (uint32_t)L::X_STAGE);
        tma_load_2d(dst, &p.xmap, g * GROUP, m0, &x_full[s]);
        tma_load_2d(dst + PF_BM * 128, &p.xmap, g * GROUP + 64, m0, &x_full[s]);
        issued = it + 1;
      }
      // the last loads of each stage have landed before the CTA may exit
      for (int it = std::max(0, issued - PF_NX); it < issued; ++it)
        mbar_wait_bounded(&x_full[it % PF_NX], (it / PF_NX) & 1, p.err);
    }
  } else if (warp == 14) {
    // ---- raw weight blocks (constant: no dependency wait), NR stages ahead ----
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < total; ++it) {
        const int s = it % PF_NR;
        if (it >= PF_NR && !mbar_wait_bounded(&w_empty[s], ((it / PF_NR) - 1) & 1, p.err)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int tile = unit_of(it / G) % n_tiles, g = it % G;
        uint8_t* dst = sm + L::OFF_RAW + s * PF_RAW;
        const int mwords = p.q4nx ? Q4NX_META_WORDS : TILE_N;
        mbar_arrive_expect_tx(&w_full[s], (uint32_t)(BLOCK_BYTES + mwords * 4));
        bulk_g2s(dst, p.qw + qw_block_offset(tile, g, G), BLOCK_BYTES, &w_full[s]);
        bulk_g2s(dst + BLOCK_BYTES, p.meta + (p.q4nx ? meta_q4nx_offset(tile, g, G) : meta_block_offset(tile, g, G)),
                 (uint32_t)(mwords * 4), &w_full[s]);
        issued = it + 1;
      }
      for (int it = std::max(0, issued - PF_NR); it < issued; ++it)
        mbar_wait_bounded(&w_full[it % PF_NR], (it / PF_NR) & 1, p.err);
    }
  } else if (warp == 13) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t IDESC = p.x_dtype == T2B_DTYPE_F16 ? idesc_f16(TILE_N, PF_BM) : idesc_bf16(TILE_N, PF_BM);
      bool ok = true;
      long long wa = 0, wx = 0, we = 0;
      (void)wa;
      (void)wx;
      (void)we;
      for (int j = 0; j < my_units && ok; ++j) {
        const int buf = j & 1;
        PF_CLK(te0);
        if (j >= 2) ok = mbar_wait_bounded(&acc_empty[buf], ((j >> 1) - 1) & 1, p.err);
        PF_ADD(we, te0);
        tc_fence_after();
        for (int g = 0; g < G && ok; ++g) {
          const int it = j * G + g, sa = it % PF_NA, sx = it % PF_NX;
          PF_CLK(ta0);
          ok = *abort_flag == 0 && mbar_wait_bounded(&a_full[sa], (it / PF_NA) & 1, p.err);
          PF_ADD(wa, ta0);
          PF_CLK(tx0);
          ok = ok && mbar_wait_bounded(&x_full[sx], (it / PF_NX) & 1, p.err);
          PF_ADD(wx, tx0);
          if (!ok) break;
          tc_fence_after();
          const uint32_t xa = smem_u32(sm + sx * L::X_STAGE);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t bdesc = sdesc_sw128(xa + (ks >> 2) * (PF_BM * 128) + (ks & 3) * 32);
            mma_ts(tbase + (uint32_t)(buf * PF_BM), tbase + PF_A0 + sa * 64 + ks * 8, bdesc, IDESC,
                   (g > 0 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&a_empty[sa]);
          mma_commit(&x_empty[sx]);
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
      if (!ok) *abort_flag = 1;
      // every MMA issued here has retired before TMEM is released
      mma_commit(done);
      mbar_wait_bounded(done, 0, p.err);
      PF_PUT(1, wa);
      PF_PUT(2, wx);
      PF_PUT(3, we);
    }
  } else {
    // ---- epilogue warps 8-11 and 15-18: drain accumulator j&1 (group 0 takes the
    //      first 64 activation rows of the tile, group 1 the last 64), then the
    //      fused epilogue on the tile with all 256 threads ----
    const int grp = warp >= 15 ? 1 : 0;
    const int q4 = warp & 3;                            // TMEM lane quarter (a warp reaches lanes 32*(warp%4)..)
    const int t = grp * 128 + q4 * 32 + lane;           // 0..255
    const int r = q4 * 32 + lane;                       // weight row
    const uint32_t lane_base = tbase + ((uint32_t)(q4 * 32) << 16);
    grid_dep_wait();   // row sums, residual rows, positions come from earlier kernels
    maybe_clear_ssq(p, blockIdx.x == 0, t, PF_EPI);
    long long wf = 0;
    (void)wf;
    for (int j = 0; j < my_units; ++j) {
      const int buf = j & 1;
      const int u = unit_of(j);
      const int tile = u % n_tiles, m0 = (u / n_tiles) * PF_BM;
      if (PRO == PRO_RMSNORM && t < PF_BM) {
        const int m = m0 + t;
        rowscale[t] = (m < p.M) ? rsqrtf(p.ssq[m] / (float)p.K + p.eps) : 0.f;   // model.py:179-180
      }
      epi_sync();   // row scales written; the previous unit's epilogue is done with tile_acc
      PF_CLK(tf0);
      const bool ok = __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait_bounded(&acc_full[buf], (j >> 1) & 1, p.err));
      PF_ADD(wf, tf0);
      if (!ok && lane == 0) *epi_abort = 1;
      epi_sync();
      if (*epi_abort) {   // the same value in every epilogue warp: no warp is left at a named barrier
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c0 = grp * (PF_BM / 2); c0 < (grp + 1) * (PF_BM / 2); c0 += 32) {
        uint32_t v[32];
        tmem_ld32(lane_base + (uint32_t)(buf * PF_BM + c0), v);
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
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);   // the MMAs of unit j+2 may overwrite it
      epi_sync();                                    // the whole tile is in shared memory
      if (EPI == EPI_QKV) {
        if (p.head_dim == 128) pf_qkv_epilogue<128, 4>(p, tile_acc, tile, m0, PF_BM, t, PF_EPI);
        else pf_qkv_epilogue<64, 4>(p, tile_acc, tile, m0, PF_BM, t, PF_EPI);
      } else if (EPI == EPI_RESIDUAL) {
        pf_residual_epilogue<8>(p, tile_acc, tile, m0, PF_BM, t, PF_EPI);
      } else {
        tile_epilogue<EPI>(p, tile_acc, scratch, tile, m0, PF_BM, EpiCache{}, t, PF_EPI);
      }
    }
    if (t == 0) PF_PUT(6, wf);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, PF_TMEM_COLS);
  }
  if (threadIdx.x == 0) PF_PUT(7, clock64() - t_start);
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
  if ((p.x_dtype != T2B_DTYPE_BF16 && p.x_dtype != T2B_DTYPE_F16) || p.N % TILE_N || p.K % GROUP)
    return T2B_ERR_SHAPE;
  // bulk copies: weight blocks and meta 16-byte aligned; TMA base 16-byte aligned
  if ((reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.qw) | reinterpret_cast<uintptr_t>(p.meta)) & 15)
    return T2B_ERR_ALIGN;
  if ((p.x_ld * 2) % 16) return T2B_ERR_ALIGN;
  cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)p.M};
  cuuint64_t strides[1] = {(cuuint64_t)p.x_ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)PF_BM};
  cuuint32_t estr[2] = {1, 1};
  const EncodeTiledFn encode = encode_tiled();
  if (encode == nullptr) return T2B_ERR_LAUNCH;
  const CUtensorMapDataType dt =
      p.x_dtype == T2B_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (encode(&p.xmap, dt, 2, const_cast<void*>(p.x), dims, strides, box, estr,
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

T2B_TRACE_DUMP_FN(t2b_trace_dump_prefill)
