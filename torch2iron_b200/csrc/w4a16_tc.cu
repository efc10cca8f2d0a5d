// W4A16 group-128 GEMM on the 5th-generation tensor cores (tcgen05), for
// decode batches of 2..256 rows per CTA, with the same fused prologues /
// epilogues as the CUDA-core GEMV.
//
// Swap-AB formulation: D[128 weight rows, Bp batch rows] = W_tile[128, k] . X[Bp, k]^T
//   * MMA M = 128 (one T2B weight tile), N = Bp (batch padded to 16..256), K = 16.
//   * A (weights) lives in TENSOR MEMORY: producer warps turn each nibble
//     pair into bf16x2 (128+q) with one mask-or ((w >> 4t) & 0x000F000F |
//     0x4300_4300; the layout stores even-k nibbles first so the pair is
//     (k, k+1)), subtract (128+z) exactly and multiply by the group scale in
//     bf16x2 -- the bf16 dequant (q - z) * s of the reference's NPU kernels --
//     and tcgen05.st the result into TMEM: no shared-memory round trip for
//     the 4x-expanded weights.
//   * B (activations) arrives by one 2-D tiled TMA copy per 64-k atom, with
//     128-byte swizzle, straight into the UMMA K-major layout; rows past M
//     are zero-filled by the copy.
//   * One fp32 TMEM accumulator of Bp columns collects all groups.
//   * Everything that does not depend on the previous kernel runs BEFORE the
//     programmatic-dependent-launch wait: the raw int4 blocks (8 KB + 512 B
//     of meta per 128x128 tile-group) arrive by 1-D bulk copies, TMEM is
//     allocated, and the first A stages are dequantised; dependents are
//     released once the CTA holds its TMEM.
//   * The k-splits of a tile form a thread-block cluster; each CTA pushes the
//     rows a peer finishes into that peer's shared memory with one bulk
//     copy and finishes Bp/KS rows itself.
//
// Roles (256 threads): warps 0-3 own TMEM lane quarters 0-3 (weight rows
// 32w..32w+31) and produce A; warp 4 allocates TMEM, issues the activation
// TMA and (one lane) the MMAs; warps 5-7 compute the row scales and stage the
// epilogue inputs; all 8 warps drain TMEM.  Every mbarrier wait is
// time-bounded; on timeout the CTA records T2B_ERR_TIMEOUT, frees its TMEM,
// still passes its cluster barriers, and skips its epilogue.

#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "linear_common.cuh"
#include "launch.cuh"
#include "tmap.cuh"
#include "tcgen05.cuh"

namespace t2b {

// Shared-memory plan of one CTA (S groups, BP padded batch rows).
// Staged epilogue inputs: per-row data (angle rows or residual rows) of the
// rows this CTA finishes, then 256 bytes of row positions, then 1 KB of
// weights.  The per-row part is sized for those rows (at most 32 KB), so a
// CTA that finishes few rows keeps its shared memory small and leaves room on
// its SM for the neighbouring kernels' CTAs.
constexpr int EP_ROWS_MAX = 32 * 1024;
__host__ __device__ constexpr int tc_ep_rows_bytes(int BP, int KS) {
  return (BP / KS) * TILE_N * 4 < EP_ROWS_MAX ? (BP / KS) * TILE_N * 4 : EP_ROWS_MAX;
}

struct TcLayout {
  int x_group, off_raw, off_meta, off_tile, off_recv, off_scr, off_ep, ep_rows, off_bar, off_tmem, off_flag, bytes;
  // q4: Q4NX meta (512 words per group: [piece 4][row 128]) instead of 128
  __host__ __device__ TcLayout(int BP, int S, int KS, bool q4 = false) {
    x_group = BP * 256;                      // bf16 [2 atoms][BP][128 B] per group (TMA, 128B swizzle)
    off_raw = S * x_group;                   // [S][8 KB] raw int4 blocks
    off_meta = off_raw + S * BLOCK_BYTES;    // [S][128 or 512] meta words
    off_tile = off_meta + S * TILE_N * 4 * (q4 ? 4 : 1);   // fp32 [BP][128] partial tile
    off_recv = off_tile + BP * TILE_N * 4;   // fp32 [KS-1][BP/KS][128] peers' partials of this CTA's rows
    off_scr = off_recv + (BP - BP / KS) * TILE_N * 4;  // fp32 [8*BP] scratch (row scales, epilogue)
    off_ep = off_scr + 8 * BP * 4;           // epilogue inputs staged after the PDL wait
    ep_rows = tc_ep_rows_bytes(BP, KS);      // per-row part of the staged inputs
    off_bar = off_ep + ep_rows + 256 + 1024; // raw_full[S], a_full[NA], a_empty[NA], acc_full, x_full, recv_full
    off_tmem = off_bar + (S + 17) * 8;       // (NA <= 7)
    off_flag = off_tmem + 8;
    bytes = off_flag + 8 + 1024;             // + slack to 1024-align the base
  }
};


// Epilogue inputs that do not depend on this kernel's result, copied to
// shared memory right after the PDL wait so the tail after the reduction
// touches no global memory it must wait for: for EPI_QKV the rows'
// positions, their RoPE angle rows and the two QK-norm weights; for
// EPI_RESIDUAL the residual rows of this tile and the next-norm weights.
// Staged only when it fits the per-row capacity `cap` (TcLayout::ep_rows).
template <int EPI>
T2B_DEV bool epilogue_staged(const LinearParams& p, int rows, int cap) {
  if (EPI == EPI_QKV) return rows <= 64 && rows * p.head_dim * 4 <= cap;
  if (EPI == EPI_RESIDUAL) return rows * TILE_N * 4 <= cap;
  return false;
}

template <int EPI>
T2B_DEV void stage_epilogue_inputs(const LinearParams& p, uint8_t* ep, int cap, int tile, int m0, int rows, int t,
                                   int nt) {
  if (!epilogue_staged<EPI>(p, rows, cap)) return;
  if (EPI == EPI_QKV) {
    const int hd = p.head_dim;
    int* __restrict__ pos_s = reinterpret_cast<int*>(ep + cap);
    float* __restrict__ ang = reinterpret_cast<float*>(ep);
    __nv_bfloat16* __restrict__ qn = reinterpret_cast<__nv_bfloat16*>(ep + cap + 256);
    __nv_bfloat16* __restrict__ kn = qn + 256;
    // each thread takes whole 4-float chunks of an angle row: position and
    // angle loads of different chunks are independent and overlap
    for (int i = t; i < rows * hd / 4; i += nt) {
      const int b = (i * 4) / hd, d = i * 4 - b * hd, m = m0 + b;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < p.M) {
        const int ps = __ldg(p.pos + m);
        if (ps >= 0 && ps < p.max_ctx) v = __ldg(reinterpret_cast<const float4*>(p.angles + (size_t)ps * hd + d));
      }
      *reinterpret_cast<float4*>(ang + i * 4) = v;
    }
    for (int i = t; i < rows; i += nt) pos_s[i] = (m0 + i < p.M) ? __ldg(p.pos + m0 + i) : 0;
    if (p.qn_w)
      for (int i = t; i < hd; i += nt) {
        qn[i] = p.qn_w[i];
        kn[i] = p.kn_w[i];
      }
  } else if (EPI == EPI_RESIDUAL) {
    float* __restrict__ res = reinterpret_cast<float*>(ep);
    __nv_bfloat16* __restrict__ nw = reinterpret_cast<__nv_bfloat16*>(ep + cap + 256);
    for (int i = t; i < rows * TILE_N / 4; i += nt) {
      const int b = (i * 4) / TILE_N, c = i * 4 - b * TILE_N, m = m0 + b;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < p.M) v = *reinterpret_cast<const float4*>(p.resid + (size_t)m * p.y_ld + tile * TILE_N + c);
      *reinterpret_cast<float4*>(res + i * 4) = v;
    }
    if (p.next_w)
      for (int i = t; i < TILE_N; i += nt) nw[i] = p.next_w[tile * TILE_N + i];
  }
}

template <int EPI>
T2B_DEV EpiCache staged_epilogue_inputs(const LinearParams& p, uint8_t* ep, int cap, int rows) {
  EpiCache c{};
  if (!epilogue_staged<EPI>(p, rows, cap)) return c;
  if (EPI == EPI_QKV) {
    c.angles = reinterpret_cast<const float*>(ep);
    c.pos = reinterpret_cast<const int*>(ep + cap);
    if (p.qn_w) {
      c.qn = reinterpret_cast<const __nv_bfloat16*>(ep + cap + 256);
      c.kn = c.qn + 256;
    }
  } else if (EPI == EPI_RESIDUAL) {
    c.resid = reinterpret_cast<const float*>(ep);
    if (p.next_w) c.next_w = reinterpret_cast<const __nv_bfloat16*>(ep + cap + 256);
  }
  return c;
}

// TMEM columns (512 per SM): the fp32 accumulator at [0, BP), then NA
// 64-column A stages, one per group up to what fits; the first NA groups are
// dequantised before the PDL wait, later groups reuse the stages as a ring.
__host__ __device__ constexpr uint32_t tc_a0(int BP) { return BP <= 64 ? 64u : (uint32_t)BP; }
__host__ __device__ constexpr int tc_stages(int BP, int S) {
  return S < (int)((512u - tc_a0(BP)) / 64u) ? S : (int)((512u - tc_a0(BP)) / 64u);
}
__host__ __device__ constexpr uint32_t tc_tmem_cols(int BP, int S) {
  return pow2_cols(tc_a0(BP) + 64u * (uint32_t)tc_stages(BP, S));
}


// grid (N/128, KS, mblocks), cluster (1, KS, 1): the KS CTAs of a cluster are
// the k-splits of one 128-row tile (S groups each); each CTA finishes BP/KS
// rows.  After the drain, one thread pushes each peer's rows of the partial
// tile with one bulk shared->shared::cluster copy that completes on the
// peer's receive mbarrier (armed at start; a cluster barrier split around the
// PDL wait makes sure every peer initialised it first).  A final cluster
// barrier keeps every CTA alive until the copies into it have landed.
//
// Order: weight bulk copies, TMEM allocation and the dequantisation of all S
// groups into TMEM run BEFORE griddepcontrol.wait (weights are constant);
// dependents are released only once every CTA holds its TMEM, so a later
// grid's allocation can only wait for an earlier grid's columns, never the
// reverse.  After the wait: activation TMA, MMAs, row scales, drain, cluster
// sum, fused epilogue.
template <int BP, int PRO, int EPI>
__global__ void __launch_bounds__(256, 2) w4a16_tc_kernel(const __grid_constant__ LinearParams p) {
  const int S = p.kslice / GROUP;
  const int KS = p.ksplit;
  const bool q4 = p.q4nx != 0;
  const TcLayout L(BP, S, KS, q4);
  const int mwords = q4 ? Q4NX_META_WORDS : TILE_N;   // meta words per (tile, group)
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = sm;
  uint8_t* raw = sm + L.off_raw;
  const uint32_t* rmeta = reinterpret_cast<const uint32_t*>(sm + L.off_meta);
  float* tile_acc = reinterpret_cast<float*>(sm + L.off_tile);
  float* recv = reinterpret_cast<float*>(sm + L.off_recv);
  float* scratch = reinterpret_cast<float*>(sm + L.off_scr);
  float* rowscale = scratch + 4 * BP;  // [BP]; scratch[0..2*BP) is the epilogue's
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.off_bar);
  const int NA = tc_stages(BP, S);     // A stages in TMEM
  uint64_t* raw_full = bars;           // [S]
  uint64_t* a_full = bars + S;         // [NA]
  uint64_t* a_empty = bars + S + NA;   // [NA]
  uint64_t* acc_full = bars + S + 2 * NA;
  uint64_t* x_full = bars + S + 2 * NA + 1;
  uint64_t* recv_full = bars + S + 2 * NA + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L.off_tmem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L.off_flag);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, mblk = blockIdx.z;
  const int g0 = split * S;
  const int m0 = mblk * BP;
  const uint32_t rank = KS > 1 ? cluster_ctarank() : 0u;
  const int rows = BP / KS;  // rows this CTA finishes
  const int mrow0 = m0 + (int)rank * rows;
  const uint32_t tmem_cols = tc_tmem_cols(BP, S);
  const uint32_t a0 = tc_a0(BP);
  T2B_TRACE_BEGIN(1 + EPI, p.N);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) mbar_init(&raw_full[i], 1);
    for (int i = 0; i < NA; ++i) {
      mbar_init(&a_full[i], 4);
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(x_full, 1);
    mbar_init(recv_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (KS > 1) mbar_arrive_expect_tx(recv_full, (uint32_t)((BP - rows) * TILE_N * 4));
  }
  __syncthreads();
  if (KS > 1) cluster_arrive();  // this CTA's receive barrier is armed (wait: before the pushes)
  // raw weight blocks of this CTA: constant data, fetched before the PDL wait
  if (threadIdx.x == 0) {
    for (int gl = 0; gl < S; ++gl) {
      mbar_arrive_expect_tx(&raw_full[gl], (uint32_t)(BLOCK_BYTES + mwords * 4));
      bulk_g2s(raw + gl * BLOCK_BYTES, p.qw + qw_block_offset(tile, g0 + gl, p.G), BLOCK_BYTES, &raw_full[gl]);
      bulk_g2s(sm + L.off_meta + gl * mwords * 4,
               p.meta + (q4 ? meta_q4nx_offset(tile, g0 + gl, p.G) : meta_block_offset(tile, g0 + gl, p.G)),
               (uint32_t)(mwords * 4),
               &raw_full[gl]);
    }
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  grid_dep_launch();  // this CTA holds its TMEM: dependents may start
  T2B_TRACE_MARK(1);
  // weights are dequantised to the activations' 16-bit type (A and B of one MMA match)
  const bool f16 = p.x_dtype == T2B_DTYPE_F16;
  const uint32_t IDESC = f16 ? idesc_f16(TILE_N, BP) : idesc_bf16(TILE_N, BP);

  if (warp < 4) {
    // ---- producers: row r's nibbles -> bf16 (q - z) * s pairs -> TMEM lane r, A stage gl % NA ----
    const int r = warp * 32 + lane;
    const uint32_t lane_base = tbase + ((uint32_t)(warp * 32) << 16);
    for (int gl = 0; gl < S; ++gl) {
      const int stage = gl % NA;
      bool ok = true;
      if (gl >= NA) {
        // the stage frees when the MMAs of group gl - NA retire, which needs
        // this grid's activations: wait for the previous grid first
        if (gl == NA) grid_dep_wait();
        ok = mbar_wait_bounded(&a_empty[stage], (gl / NA - 1) & 1, p.err);
      }
      ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&raw_full[gl], 0, p.err));
      if (!ok) {  // the warp takes the same branch before tcgen05.st
        *abort_flag = 1;
        break;
      }
      if (q4) {  // Q4NX: a scale and zero point per 32-k piece, dequantised in fp32
#pragma unroll 1
        for (int pc = 0; pc < 4; ++pc) {
          const uint4 v = *reinterpret_cast<const uint4*>(raw + gl * BLOCK_BYTES + pc * 2048 + r * 16);
          const uint32_t mw = rmeta[gl * Q4NX_META_WORDS + pc * TILE_N + r];
          uint32_t cols[16];
          if (f16) dequant_piece_q4nx<true>(v, bf16_lo_f32(mw), bf16_hi_f32(mw), cols);
          else dequant_piece_q4nx<false>(v, bf16_lo_f32(mw), bf16_hi_f32(mw), cols);
          tmem_st16(lane_base + a0 + stage * 64 + pc * 16, cols);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[stage]);
        continue;
      }
      const uint32_t mw = rmeta[gl * TILE_N + r];
      uint32_t z2, s2;
      if (f16) t2b_meta_pairs<true>(mw, z2, s2);
      else t2b_meta_pairs<false>(mw, z2, s2);
#pragma unroll
      for (int pc = 0; pc < 4; ++pc) {
        const uint4 v = *reinterpret_cast<const uint4*>(raw + gl * BLOCK_BYTES + pc * 2048 + r * 16);
        uint32_t cols[16];
        // slot t holds k 2t, slot t+4 holds k 2t+1: the mask-or is the pair (2t, 2t+1), biased
        if (f16) dequant_piece_t2b<true>(v, z2, s2, cols);
        else dequant_piece_t2b<false>(v, z2, s2, cols);
        tmem_st16(lane_base + a0 + stage * 64 + pc * 16, cols);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[stage]);
    }
    T2B_TRACE_MARK(2);
    grid_dep_wait();
    T2B_TRACE_MARK(3);
  } else if (warp == 4) {
    grid_dep_wait();
    // ---- activations (one 64-k x BP-row TMA box per group and 64-k atom, swizzled
    // into the UMMA K-major layout; rows past M arrive as zeros), then the MMAs ----
    if (lane == 0) {
      mbar_arrive_expect_tx(x_full, (uint32_t)(S * L.x_group));
      for (int gl = 0; gl < S; ++gl)
        for (int atom = 0; atom < 2; ++atom)
          tma_load_2d(xs + gl * L.x_group + atom * (BP * 128), &p.xmap, (g0 + gl) * GROUP + atom * 64, m0, x_full);
      bool ok = mbar_wait_bounded(x_full, 0, p.err);
      T2B_TRACE_STAMP(8);   // activations in shared memory
      for (int gl = 0; ok && gl < S; ++gl) {
        const int stage = gl % NA;
        if (!mbar_wait_bounded(&a_full[stage], (gl / NA) & 1, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t xg = smem_u32(xs + gl * L.x_group);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t bdesc = sdesc_sw128(xg + (ks >> 2) * (BP * 128) + (ks & 3) * 32);
          mma_ts(tbase, tbase + a0 + stage * 64 + ks * 8, bdesc, IDESC, (gl > 0 || ks > 0) ? 1u : 0u);
        }
        if (gl + NA < S) mma_commit(&a_empty[stage]);
      }
      if (!ok) *abort_flag = 1;
      mma_commit(acc_full);
      T2B_TRACE_STAMP(9);   // every MMA issued
    }
    __syncwarp();
  } else {
    // ---- warps 5-7: ssq buffer hand-off, row scales, epilogue inputs ----
    grid_dep_wait();
    maybe_clear_ssq(p, tile == 0 && split == 0 && mblk == 0, threadIdx.x - 160, 96);
    if (PRO == PRO_RMSNORM)
      for (int b = threadIdx.x - 160; b < BP; b += 96) {
        const int m = m0 + b;
        rowscale[b] = (m < p.M) ? rsqrtf(p.ssq[m] / (float)p.K + p.eps) : 0.f;   // model.py:179-180
      }
    if (threadIdx.x == 160) T2B_TRACE_STAMP(10);   // row scales written
    stage_epilogue_inputs<EPI>(p, sm + L.off_ep, L.ep_rows, tile, mrow0, rows, threadIdx.x - 160, 96);
    if (threadIdx.x == 160) T2B_TRACE_STAMP(11);   // this thread's epilogue inputs staged
  }
  __syncthreads();  // row scales and staged inputs visible

  // ---- drain: D[r][b] (* row scale) -> the owning CTA's slot [rank][b - q*rows][r];
  // warps w and w+4 share TMEM lane quarter w%4 and split the BP columns ----
  {
    constexpr int HB = BP / 2;
    const int q4 = warp & 3, half = warp >> 2;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = tbase + ((uint32_t)(q4 * 32) << 16);
    const bool ok = __all_sync(0xffffffffu, (*abort_flag == 0) && mbar_wait_bounded(acc_full, 0, p.err));
    if (!ok) *abort_flag = 1;
    T2B_TRACE_MARK(4);
    tc_fence_after();
    constexpr int CB = HB < 32 ? HB : 32;  // columns per TMEM load round
#pragma unroll 1
    for (int c0 = 0; c0 < HB; c0 += CB) {
      uint32_t v[CB];
      if (ok) {
        if (CB >= 16) {
#pragma unroll
          for (int cb = 0; cb < CB / 16; ++cb)
            tmem_ld16(lane_base + half * HB + c0 + cb * 16, *reinterpret_cast<uint32_t(*)[16]>(&v[cb * 16]));
        } else {
          tmem_ld8(lane_base + half * HB + c0, *reinterpret_cast<uint32_t(*)[8]>(&v[0]));
        }
        tmem_ld_wait();
      }
#pragma unroll
      for (int e = 0; e < CB; ++e) {
        const int b = half * HB + c0 + e;
        float y = ok ? __uint_as_float(v[e]) : 0.f;
        if (PRO == PRO_RMSNORM) y *= rowscale[b];
        tile_acc[b * TILE_N + r] = y;
      }
    }
  }
  T2B_TRACE_MARK(5);
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tbase, tmem_cols);
  }

  // ---- cluster split-K: push each peer's rows, sum the rows pushed here ----
  // (every CTA passes both cluster barrier phases, aborted or not; an aborted
  // CTA still pushes so no peer waits out its receive barrier)
  if (KS > 1) {
    cluster_wait();
    if (threadIdx.x == 0) {
      fence_proxy_async();  // the drain's shared-memory stores, seen by the bulk copies
      for (int q = 0; q < KS; ++q) {
        if (q == (int)rank) continue;
        const int slot = (int)rank < q ? (int)rank : (int)rank - 1;  // this CTA's slot at rank q
        bulk_s2s_peer(map_peer(smem_u32(recv + slot * rows * TILE_N), (uint32_t)q), tile_acc + q * rows * TILE_N,
                      (uint32_t)(rows * TILE_N * 4), map_peer(smem_u32(recv_full), (uint32_t)q));
      }
    }
    const bool ok = __syncthreads_and(mbar_wait_bounded(recv_full, 0, p.err));
    if (!ok && threadIdx.x == 0) *abort_flag = 1;
    // sums go to receive slot 0: the other owners' rows of tile_acc may still
    // be read by this CTA's outgoing copies
    for (int i = threadIdx.x; i < rows * TILE_N / 4; i += 256) {
      float4 acc = reinterpret_cast<const float4*>(tile_acc + rank * rows * TILE_N)[i];
      for (int q = 0; q < KS - 1; ++q) {
        const float4 v = reinterpret_cast<const float4*>(recv + q * rows * TILE_N)[i];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      reinterpret_cast<float4*>(recv)[i] = acc;
    }
    __syncthreads();
  }
  const float* fin = KS > 1 ? recv : tile_acc;
  T2B_TRACE_MARK(6);
  if (!*abort_flag)
    tile_epilogue<EPI>(p, fin, scratch, tile, mrow0, rows,
                       staged_epilogue_inputs<EPI>(p, sm + L.off_ep, L.ep_rows, rows));
  __syncthreads();
  T2B_TRACE_MARK(7);
  // every peer has received this CTA's pushes (it waited for them before
  // arriving here), so this CTA's shared memory may be released
  if (KS > 1) cluster_sync();
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct TcPlan {
  int BP, KS, S, mblocks;
  size_t smem;
  bool ok;
};

// Groups per CTA S and cluster size KS = G/S (k-splits of a tile): the
// largest S <= 4 that keeps KS <= 8 and the grid at >= 64 CTAs (or as many
// as the shape allows).  Bp covers the batch up to 256 rows per CTA; shared
// memory bounds S * Bp.
// Largest batch tile (env T2B_TC_MAX_BP overrides, for experiments): a larger
// batch than this runs as several row blocks, each CTA dequantising its
// weight tile again (off the critical path, before the dependency wait).
// Env T2B_TC_PLAN="NxK:BP:S,..." (experiments) sets both for one shape.
static bool tc_shape_override(int N, int K, int* bp, int* s) {
  const char* e = getenv("T2B_TC_PLAN");
  if (!e || !*e) return false;
  int n = 0, k = 0, b = 0, g = 0, used = 0;
  while (sscanf(e, "%dx%d:%d:%d%n", &n, &k, &b, &g, &used) == 4) {
    if (n == N && k == K) {
      *bp = b;
      *s = g;
      return true;
    }
    e += used;
    if (*e != ',') break;
    ++e;
  }
  return false;
}

static int tc_max_bp(int N, int K) {
  int b = 0, g = 0;
  if (tc_shape_override(N, K, &b, &g) && (b == 16 || b == 32 || b == 64 || b == 128 || b == 256)) return b;
  const char* e = getenv("T2B_TC_MAX_BP");
  if (e && *e) {
    const int v = atoi(e);
    if (v == 16 || v == 32 || v == 64 || v == 128 || v == 256) return v;
  }
  return 256;
}

// Groups per CTA forced by env T2B_TC_S or T2B_TC_PLAN (experiments; 0: the
// planner's choice).  Taken only where the split is valid and fits.
static int tc_forced_s(int N, int K) {
  int b = 0, g = 0;
  if (tc_shape_override(N, K, &b, &g)) return g;
  const char* e = getenv("T2B_TC_S");
  return (e && *e) ? atoi(e) : 0;
}

// max_rows > 0: the plan for an epilogue with costly per-row work (the qkv
// epilogue: QK-norm, RoPE and the KV-cache write of every row), whose CTAs
// each finish at most max_rows batch rows where such a plan exists within
// about one wave: Bp <= 32 and the largest S >= 2 with Bp/KS <= max_rows.
// (Qwen3-0.6B qkv at 64 rows: Bp 32, 2 groups per CTA, clusters of 4 -- 8
// rows per CTA instead of 32 -- took 39 us off the 1.41 ms decode step.)
static TcPlan tc_plan(int M, int N, int K, bool q4 = false, int max_rows = 0) {
  TcPlan pl{};
  const int G = K / GROUP;
  const int tiles = N / TILE_N;
  const int max_bp = tc_max_bp(N, K);
  int bp = 16;
  while (bp < M && bp < max_bp) bp <<= 1;
  pl.BP = bp;
  pl.S = 0;
  auto fits = [&](int bp_, int s_) { return TcLayout(bp_, s_, G / s_, q4).bytes <= 210 * 1024; };
  // KS must divide BP: each CTA of a cluster finishes BP/KS rows, and its
  // receive barrier expects the (KS-1) * BP/KS rows its peers push.
  auto splits = [&](int bp_, int s_) { return G % s_ == 0 && G / s_ <= 8 && bp_ % (G / s_) == 0; };
  int ov_bp = 0, ov_s = 0;
  bool capped = false;
  if (max_rows > 0 && !tc_shape_override(N, K, &ov_bp, &ov_s)) {
    const int bpc = std::min(bp, 32);
    const long mbc = (M + bpc - 1) / bpc;
    for (int s_ : {4, 3, 2}) {
      if (!splits(bpc, s_) || !fits(bpc, s_) || bpc / (G / s_) > max_rows) continue;
      if ((long)tiles * (G / s_) * mbc > 2L * 148) continue;   // about one wave
      pl.BP = bpc;
      pl.S = s_;
      capped = true;
      break;
    }
  }
  for (int s_ : {4, 3, 2, 1}) {
    if (capped) break;
    if (!splits(bp, s_)) continue;
    if (!fits(bp, s_)) continue;
    const long ctas = (long)tiles * (G / s_) * ((M + bp - 1) / bp);
    if (ctas >= 64 || s_ == 1) {
      pl.S = s_;
      break;
    }
  }
  if (pl.S == 0) {  // long K: smallest S with KS <= 8 that fits, shrinking Bp if needed
    for (int s_ = (G + 7) / 8; s_ <= G && pl.S == 0; ++s_) {
      if (G % s_) continue;
      int b = bp;
      while (b > 16 && !fits(b, s_)) b >>= 1;
      if (fits(b, s_) && splits(b, s_)) {
        pl.S = s_;
        pl.BP = b;
      }
    }
  }
  pl.ok = pl.S > 0 && N % TILE_N == 0 && splits(pl.BP, pl.S);
  if (!pl.ok) return pl;
  // A grid of more than one wave (resident CTAs: shared memory and TMEM, at
  // most 2 per SM) takes more groups per CTA where they fit: fewer, longer CTAs.
  {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
    const int mb = (M + pl.BP - 1) / pl.BP;
    auto waves = [&](int s_) {
      const long bytes = TcLayout(pl.BP, s_, G / s_, q4).bytes;
      int per_sm = (int)((228L * 1024) / (bytes + 1024));
      per_sm = std::min(per_sm, (int)(512u / tc_tmem_cols(pl.BP, s_)));
      per_sm = std::max(1, std::min(per_sm, 2));
      const long ctas = (long)tiles * (G / s_) * mb;
      return (ctas + (long)sms * per_sm - 1) / ((long)sms * per_sm);
    };
    int best = pl.S;
    if (!capped && waves(best) > 1)
      for (int s_ = pl.S + 1; s_ <= G; ++s_) {
        if (!splits(pl.BP, s_) || !fits(pl.BP, s_)) continue;
        if (waves(s_) < waves(best)) best = s_;
      }
    pl.S = best;
  }
  {
    const int fs = tc_forced_s(N, K);
    if (fs > 0 && fs <= G && splits(pl.BP, fs) && fits(pl.BP, fs)) pl.S = fs;
  }
  pl.KS = G / pl.S;
  pl.mblocks = (M + pl.BP - 1) / pl.BP;
  pl.smem = (size_t)TcLayout(pl.BP, pl.S, pl.KS, q4).bytes;
  // A CTA holding more than half of the SM's 512 TMEM columns runs alone on
  // its SM (more than half of the shared memory requested): a second one
  // there would only sit in tcgen05.alloc until the first frees its columns.
  // (No wait cycle either way: a CTA frees its TMEM before the cluster
  // barrier, the only point where it waits for its peers.)
  if (tc_tmem_cols(pl.BP, pl.S) > 256 && pl.smem < 120 * 1024) pl.smem = 120 * 1024;
  return pl;
}

size_t tc_ws_bytes(int, int, int) { return 0; }  // split-K stays on chip (cluster DSMEM)

bool tc_supported(int M, int N, int K, bool q4) { return tc_plan(M, N, K, q4).ok; }

// CTAs of the tcgen05 decode grid for this shape (0 when the path cannot take it).
long tc_grid_ctas(int M, int N, int K, bool q4) {
  const TcPlan pl = tc_plan(M, N, K, q4);
  return pl.ok ? (long)(N / TILE_N) * pl.KS * pl.mblocks : 0;
}

bool tc_plan_info(int M, int N, int K, int* bp, int* s, int* ks, int max_rows) {
  const TcPlan pl = tc_plan(M, N, K, false, max_rows);
  *bp = pl.BP;
  *s = pl.S;
  *ks = pl.KS;
  return pl.ok;
}

template <int BP, int PRO, int EPI>
static int tc_launch_t(LinearParams& p, const TcPlan& pl, cudaStream_t st) {
  auto kern = w4a16_tc_kernel<BP, PRO, EPI>;
  if (allow_smem(kern, pl.smem) != T2B_OK) return T2B_ERR_LAUNCH;
  dim3 grid(p.N / TILE_N, pl.KS, pl.mblocks);
  return launch_pdl_cluster(kern, grid, dim3(256), pl.smem, st, pl.KS, p);
}

template <int PRO, int EPI>
static int tc_dispatch(LinearParams& p, const TcPlan& pl, cudaStream_t st) {
  if (pl.BP == 16) return tc_launch_t<16, PRO, EPI>(p, pl, st);
  if (pl.BP == 32) return tc_launch_t<32, PRO, EPI>(p, pl, st);
  if (pl.BP == 64) return tc_launch_t<64, PRO, EPI>(p, pl, st);
  if (pl.BP == 128) return tc_launch_t<128, PRO, EPI>(p, pl, st);
  if (pl.BP == 256) return tc_launch_t<256, PRO, EPI>(p, pl, st);
  return T2B_ERR_ARG;
}

// 2-D tiled tensor map over the bf16 activations [M][x_ld]: box 64 k x BP rows,
// 128-byte swizzle (the UMMA K-major canonical layout); out-of-range rows read 0.
static int make_x_map(LinearParams& p, int BP) {
  if (reinterpret_cast<uintptr_t>(p.x) & 15) return T2B_ERR_ALIGN;
  if ((p.x_ld * 2) % 16) return T2B_ERR_ALIGN;
  cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)p.M};
  cuuint64_t strides[1] = {(cuuint64_t)p.x_ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)BP};
  cuuint32_t estr[2] = {1, 1};
  const EncodeTiledFn encode = encode_tiled();
  if (encode == nullptr) return T2B_ERR_LAUNCH;
  const CUtensorMapDataType dt =
      p.x_dtype == T2B_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = encode(&p.xmap, dt, 2, const_cast<void*>(p.x), dims,
                                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? T2B_OK : T2B_ERR_ARG;
}

int tc_launch(LinearParams& p, int pro, int epi, void*, size_t, cudaStream_t st) {
  const TcPlan pl = tc_plan(p.M, p.N, p.K, p.q4nx != 0, epi == EPI_QKV ? QKV_MAX_ROWS_PER_CTA : 0);
  if (!pl.ok) return T2B_ERR_SHAPE;
  if (p.x_dtype != T2B_DTYPE_BF16 && p.x_dtype != T2B_DTYPE_F16) return T2B_ERR_ARG;
  const int mx = make_x_map(p, pl.BP);
  if (mx != T2B_OK) return mx;
  p.kslice = pl.S * GROUP;
  p.ksplit = pl.KS;
  if (pro == PRO_ACT && epi == EPI_STORE) return tc_dispatch<PRO_ACT, EPI_STORE>(p, pl, st);
  if (pro == PRO_RMSNORM && epi == EPI_STORE) return tc_dispatch<PRO_RMSNORM, EPI_STORE>(p, pl, st);
  if (pro == PRO_ACT && epi == EPI_RESIDUAL) return tc_dispatch<PRO_ACT, EPI_RESIDUAL>(p, pl, st);
  if (pro == PRO_RMSNORM && epi == EPI_SWIGLU) return tc_dispatch<PRO_RMSNORM, EPI_SWIGLU>(p, pl, st);
  if (pro == PRO_RMSNORM && epi == EPI_QKV) return tc_dispatch<PRO_RMSNORM, EPI_QKV>(p, pl, st);
  return T2B_ERR_ARG;
}

}  // namespace t2b

T2B_TRACE_DUMP_FN(t2b_trace_dump_tc)
