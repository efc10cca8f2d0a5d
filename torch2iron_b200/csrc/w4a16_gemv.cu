// W4A16 group-128 dequant-GEMV for small batches (M <= 8 rows per CTA) on
// CUDA cores, with the decode-layer prologues / epilogues fused in.
//
// Work decomposition (one CTA = 256 threads = 8 warps):
//   * output tile: 128 consecutive weight rows (= one QK head of 128, or a
//     64-row gate block + its 64-row up block), x one k-slice of CH*256.
//   * warp w owns rows 16w..16w+15 of the tile; lane l reads row
//     16w + 4i + (l>>3) (i = 0..3) at k offset (l&7)*32 of every 256-k chunk
//     -> each lane issues 4*CH independent 16-byte loads up front (all the
//     CTA's weight bytes are in flight at once), before the PDL wait.
//   * dequant per nibble: one PRMT builds the fp32 value 128+q, one FFMA
//     turns it into (q - zero) * scale exactly (19-bit products), then one
//     FFMA per batch row.
//   * the 8 lanes of a row reduce with 3 xor-shuffles.  k-slices (split-K)
//     of a tile form a thread-block cluster of up to 8 CTAs: every rank but
//     0 pushes its [MB][128] partial into rank 0's shared memory with one
//     bulk copy (completion on rank 0's mbarrier), and rank 0 sums and runs
//     the epilogue on the full 128-row tile.  More than 8 k-slices meet in a
//     fp32 workspace instead, where the last CTA of a tile (ticket counter)
//     runs the epilogue.
//   * the RMSNorm row scale rsqrt(ssq/K + eps) multiplies the finished dot
//     products (it is loaded alongside the activations, not before them).
//
// Algorithmic parity: W[n,k] = (q - zero) * scale exactly as
// src/models/fast_qwen3/fast_packed_format.py:158-160; fp32 accumulation as
// src/models/quantized_qwen3/model.py:133-146.

#include "linear_common.cuh"
#include "launch.cuh"

#include <stdlib.h>

namespace t2b {

constexpr int GV_THREADS = 256;

constexpr int GV_MAX_CLUSTER = 8;

// Shared memory: xs | tile_acc | scratch | recv [ksplit-1][MB][128] (cluster
// split-K only) | receive mbarrier.
template <int MB, int CH>
struct GemvSmem {
  static constexpr int XS_LD = CH * 288;  // 256 k per chunk, +4 floats pad per 32 (bank spread)
  static constexpr int XS_FLOATS = MB * XS_LD;
  static constexpr int TILE_FLOATS = MB * TILE_N;
  static constexpr size_t BYTES = sizeof(float) * (XS_FLOATS + TILE_FLOATS + 8 * MB);
  static size_t bytes(int ksplit, bool cluster) {
    return BYTES + (cluster ? sizeof(float) * (size_t)(ksplit - 1) * TILE_FLOATS + 16 : 0);
  }
};

// k-slices of one tile reduced inside a cluster (else through the workspace)
static inline bool gv_cluster(int ksplit) { return ksplit > 1 && ksplit <= GV_MAX_CLUSTER; }

T2B_DEV uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

T2B_DEV float nib_f(uint32_t v, int sel) { return __uint_as_float(__byte_perm(v, 0x43000000u, sel)); }

template <int MB, int CH, int PRO, int EPI, int WFMT>
__global__ void __launch_bounds__(GV_THREADS) w4a16_gemv_kernel(const LinearParams p) {
  using S = GemvSmem<MB, CH>;
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;
  float* tile_acc = smem + S::XS_FLOATS;
  float* scratch = tile_acc + S::TILE_FLOATS;   // [8*MB]
  float* recv = scratch + 8 * MB;               // cluster split-K: [ksplit-1][MB][128]
  const bool clus = p.ksplit > 1 && p.ksplit <= GV_MAX_CLUSTER;
  uint64_t* recv_full = reinterpret_cast<uint64_t*>(recv + (clus ? (p.ksplit - 1) * S::TILE_FLOATS : 0));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, mblk = blockIdx.z;
  const int row0 = tile * TILE_N;
  const int k0 = split * p.kslice;
  const int m0 = mblk * MB;
  T2B_TRACE_BEGIN(20 + EPI, p.N);

  // ---- 1. weight prefetch (independent of the previous kernel) ----------
  uint4 wv[CH][4];
  uint32_t mt[CH][4];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = warp * 16 + i * 4 + (lane >> 3);
      const int k = k0 + c * 256 + (lane & 7) * 32;
      if (WFMT == T2B_WFMT_T2B || WFMT == T2B_WFMT_Q4NX) {
        const int g = k >> 7, pc = (k & 127) >> 5;
        wv[c][i] = ldg_stream(p.qw + qw_block_offset(tile, g, p.G) + pc * 2048 + rr * 16);
        if (WFMT == T2B_WFMT_T2B)
          mt[c][i] = __ldg(p.meta + meta_block_offset(tile, g, p.G) + rr);
        else  // one Q4NX piece (32 k) per lane and chunk: its own scale and zero point
          mt[c][i] = __ldg(p.meta + meta_q4nx_offset(tile, g, p.G) + pc * TILE_N + rr);
      } else {  // qparam rows are K/2 + 2G bytes: only 4-byte aligned
        const uint8_t* rowp = p.qw + (size_t)(row0 + rr) * p.w_ld;
        const uint32_t* w4 = reinterpret_cast<const uint32_t*>(rowp + (k >> 1));
        wv[c][i] = make_uint4(__ldg(w4), __ldg(w4 + 1), __ldg(w4 + 2), __ldg(w4 + 3));
        mt[c][i] = __ldg(reinterpret_cast<const unsigned short*>(rowp + (p.K >> 1)) + (k >> 7));
      }
    }
  }

  // cluster split-K: rank 0's receive barrier, armed before any peer may push
  const uint32_t rank = clus ? cluster_ctarank() : 0u;
  if (clus) {
    if (threadIdx.x == 0) {
      mbar_init(recv_full, 1);
      fence_mbar_init();
      if (rank == 0) mbar_arrive_expect_tx(recv_full, (uint32_t)((p.ksplit - 1) * S::TILE_FLOATS * 4));
    }
    __syncthreads();
    cluster_arrive();
  }

  grid_dep_wait();
  grid_dep_launch();
  T2B_TRACE_MARK(1);

  // ---- 2. prologue: activations of this k-slice into shared fp32; the
  // RMSNorm row scale (model.py:179-181: x holds bf16(row * weight), the dot
  // product is then times rsqrt(mean(row^2)+eps)) loads alongside ----------
  if (PRO == PRO_RMSNORM && threadIdx.x < MB) {
    const int m = m0 + threadIdx.x;
    scratch[threadIdx.x] = (m < p.M) ? rsqrtf(p.ssq[m] / (float)p.K + p.eps) : 0.f;
  }
  for (int idx = threadIdx.x; idx < MB * CH * 256; idx += GV_THREADS) {
    const int b = idx / (CH * 256), kk = idx - b * (CH * 256);
    const int m = m0 + b;
    float v = 0.f;
    if (m < p.M) v = load_act(p.x, p.x_dtype, (size_t)m * p.x_ld + k0 + kk);
    xs[b * S::XS_LD + kk + (kk >> 5) * 4] = v;
  }
  maybe_clear_ssq(p, tile == 0 && split == 0 && mblk == 0, threadIdx.x, GV_THREADS);
  __syncthreads();
  T2B_TRACE_MARK(2);

  // ---- 3. dequant + FMA -------------------------------------------------
  float acc[4][MB];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int b = 0; b < MB; ++b) acc[i][b] = 0.f;

#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float sc[4], zc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (WFMT == T2B_WFMT_T2B) {
        sc[i] = __half2float(__ushort_as_half((unsigned short)(mt[c][i] & 0xffffu)));
        const float z = (float)((mt[c][i] >> 16) & 0x1fu);
        zc[i] = -(128.f + z) * sc[i];
      } else if (WFMT == T2B_WFMT_Q4NX) {
        sc[i] = bf16_lo_f32(mt[c][i]);
        zc[i] = bf16_hi_f32(mt[c][i]);       // the zero point itself (not folded)
      } else {
        sc[i] = bf16_bits_to_f32(mt[c][i] & 0xffffu);
        zc[i] = -(128.f + 8.f) * sc[i];
      }
    }
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
      const int kk = c * 256 + (lane & 7) * 32 + wd * 8;
      float wf[4][8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t w = wd == 0 ? wv[c][i].x : wd == 1 ? wv[c][i].y : wd == 2 ? wv[c][i].z : wv[c][i].w;
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        // (128+q)*s - (128+z)*s is exact in fp32: (q - z) * s
        if (WFMT == T2B_WFMT_Q4NX) {
          // (q - zero) * scale in fp32 as the reference (q4nx_layout.py:132-146):
          // nib_f - 128 is q exactly, then one rounded subtract and one multiply
#define T2B_Q4(sel, src) __fmul_rn(__fsub_rn(nib_f(src, sel) - 128.f, zc[i]), sc[i])
          wf[i][0] = T2B_Q4(0x7054, lo);
          wf[i][2] = T2B_Q4(0x7054, hi);
          wf[i][4] = T2B_Q4(0x7154, lo);
          wf[i][6] = T2B_Q4(0x7154, hi);
          wf[i][1] = T2B_Q4(0x7254, lo);
          wf[i][3] = T2B_Q4(0x7254, hi);
          wf[i][5] = T2B_Q4(0x7354, lo);
          wf[i][7] = T2B_Q4(0x7354, hi);
#undef T2B_Q4
        } else if (WFMT == T2B_WFMT_T2B) {  // nibble slots hold k 0,2,4,6,1,3,5,7
          wf[i][0] = fmaf(nib_f(lo, 0x7054), sc[i], zc[i]);
          wf[i][2] = fmaf(nib_f(hi, 0x7054), sc[i], zc[i]);
          wf[i][4] = fmaf(nib_f(lo, 0x7154), sc[i], zc[i]);
          wf[i][6] = fmaf(nib_f(hi, 0x7154), sc[i], zc[i]);
          wf[i][1] = fmaf(nib_f(lo, 0x7254), sc[i], zc[i]);
          wf[i][3] = fmaf(nib_f(hi, 0x7254), sc[i], zc[i]);
          wf[i][5] = fmaf(nib_f(lo, 0x7354), sc[i], zc[i]);
          wf[i][7] = fmaf(nib_f(hi, 0x7354), sc[i], zc[i]);
        } else {  // reference qparam: natural order, low nibble = even k
          wf[i][0] = fmaf(nib_f(lo, 0x7054), sc[i], zc[i]);
          wf[i][1] = fmaf(nib_f(hi, 0x7054), sc[i], zc[i]);
          wf[i][2] = fmaf(nib_f(lo, 0x7154), sc[i], zc[i]);
          wf[i][3] = fmaf(nib_f(hi, 0x7154), sc[i], zc[i]);
          wf[i][4] = fmaf(nib_f(lo, 0x7254), sc[i], zc[i]);
          wf[i][5] = fmaf(nib_f(hi, 0x7254), sc[i], zc[i]);
          wf[i][6] = fmaf(nib_f(lo, 0x7354), sc[i], zc[i]);
          wf[i][7] = fmaf(nib_f(hi, 0x7354), sc[i], zc[i]);
        }
      }
#pragma unroll
      for (int b = 0; b < MB; ++b) {
        const float4 xa = *reinterpret_cast<const float4*>(&xs[b * S::XS_LD + kk + (kk >> 5) * 4]);
        const float4 xb = *reinterpret_cast<const float4*>(&xs[b * S::XS_LD + kk + (kk >> 5) * 4 + 4]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float a = acc[i][b];
          a = fmaf(wf[i][0], xa.x, a);
          a = fmaf(wf[i][1], xa.y, a);
          a = fmaf(wf[i][2], xa.z, a);
          a = fmaf(wf[i][3], xa.w, a);
          a = fmaf(wf[i][4], xb.x, a);
          a = fmaf(wf[i][5], xb.y, a);
          a = fmaf(wf[i][6], xb.z, a);
          a = fmaf(wf[i][7], xb.w, a);
          acc[i][b] = a;
        }
      }
    }
  }

  // ---- 4. reduce the 8 lanes of each row into the tile ------------------
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int b = 0; b < MB; ++b) {
      float v = acc[i][b];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      if (PRO == PRO_RMSNORM) v *= scratch[b];
      if ((lane & 7) == 0) tile_acc[b * TILE_N + warp * 16 + i * 4 + (lane >> 3)] = v;
    }
  __syncthreads();

  // ---- 5. split-K + epilogue --------------------------------------------
  T2B_TRACE_MARK(3);
  if (clus) {
    cluster_wait();  // every rank's receive barrier is armed
    if (rank != 0) {
      if (threadIdx.x == 0) {
        fence_proxy_async();  // tile_acc's shared-memory stores, seen by the bulk copy
        bulk_s2s_peer(map_peer(smem_u32(recv + (rank - 1) * S::TILE_FLOATS), 0u), tile_acc,
                      (uint32_t)(S::TILE_FLOATS * 4), map_peer(smem_u32(recv_full), 0u));
      }
    } else {
      const bool ok = __syncthreads_and(mbar_wait_bounded(recv_full, 0, p.err));
      for (int idx = threadIdx.x; idx < S::TILE_FLOATS; idx += GV_THREADS) {
        float v = tile_acc[idx];
        for (int q = 0; q < p.ksplit - 1; ++q) v += recv[q * S::TILE_FLOATS + idx];
        tile_acc[idx] = v;
      }
      __syncthreads();
      T2B_TRACE_MARK(4);
      if (ok) tile_epilogue<EPI>(p, tile_acc, scratch, tile, m0, MB);
      __syncthreads();
      T2B_TRACE_MARK(5);
    }
    // rank 0 arrives after its pushes landed: the senders' shared memory may go
    cluster_sync();
    return;
  }
  if (!splitk_fixup<MB>(p, tile_acc, tile, split, mblk, GV_THREADS)) return;
  T2B_TRACE_MARK(4);
  tile_epilogue<EPI>(p, tile_acc, scratch, tile, m0, MB);
  __syncthreads();
  T2B_TRACE_MARK(5);
}

// ---------------------------------------------------------------------------
// Host-side launchers
// ---------------------------------------------------------------------------

static int pick_mb(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

// k-slice per CTA: the smallest of 256/512/1024 that keeps a tile's k-slices
// within one cluster (<= 8), else 256/512 with the grid at about 1-4 CTAs
// per SM (workspace split-K).
static int pick_kslice(int N, int K, int mblocks) {
  for (int ks : {256, 512, 1024})
    if (K % ks == 0 && K / ks <= GV_MAX_CLUSTER) return ks;
  const long tiles = (long)(N / TILE_N) * mblocks;
  if (K % 512 == 0 && tiles * (K / 256) > 4L * 148) return 512;
  return 256;
}

static size_t gemv_ws_bytes(int M, int N, int K) {
  const int MB = pick_mb(M);
  const int mblocks = (M + MB - 1) / MB;
  const int ksplit = K / pick_kslice(N, K, mblocks);
  if (ksplit == 1 || gv_cluster(ksplit)) return 0;
  size_t part = ((size_t)mblocks * ksplit * MB * N * sizeof(float) + 255) & ~size_t(255);
  return part + (((size_t)mblocks * (N / TILE_N) * sizeof(int) + 255) & ~size_t(255));
}

template <int MB, int CH, int PRO, int EPI, int WFMT>
static int gemv_launch_t(LinearParams& p, dim3 grid, cudaStream_t st) {
  auto kern = w4a16_gemv_kernel<MB, CH, PRO, EPI, WFMT>;
  const bool clus = gv_cluster(p.ksplit);
  const size_t smem = GemvSmem<MB, CH>::bytes(p.ksplit, clus);
  if (allow_smem(kern, smem) != T2B_OK) return T2B_ERR_LAUNCH;
  if (clus) return launch_pdl_cluster(kern, grid, dim3(GV_THREADS), smem, st, p.ksplit, p);
  return launch_pdl(kern, grid, dim3(GV_THREADS), smem, st, p);
}

template <int PRO, int EPI, int WFMT>
static int gemv_dispatch(LinearParams& p, int MB, int CH, dim3 grid, cudaStream_t st) {
#define T2B_CASE(mb, ch) \
  if (MB == mb && CH == ch) return gemv_launch_t<mb, ch, PRO, EPI, WFMT>(p, grid, st);
  T2B_CASE(1, 1) T2B_CASE(1, 2) T2B_CASE(1, 4) T2B_CASE(2, 1) T2B_CASE(2, 2) T2B_CASE(2, 4)
  T2B_CASE(4, 1) T2B_CASE(4, 2) T2B_CASE(4, 4) T2B_CASE(8, 1) T2B_CASE(8, 2) T2B_CASE(8, 4)
#undef T2B_CASE
  return T2B_ERR_ARG;
}

static int gemv_launch(LinearParams& p, int pro, int epi, int wfmt, void* ws, size_t ws_bytes, cudaStream_t st) {
  const int MB = pick_mb(p.M);
  const int mblocks = (p.M + MB - 1) / MB;
  p.kslice = pick_kslice(p.N, p.K, mblocks);
  p.ksplit = p.K / p.kslice;
  const bool need_ws = p.ksplit > 1 && !gv_cluster(p.ksplit);
  if (ws_bytes < gemv_ws_bytes(p.M, p.N, p.K) || (need_ws && ws == nullptr)) return T2B_ERR_WORKSPACE;
  size_t part = ((size_t)mblocks * p.ksplit * MB * p.N * sizeof(float) + 255) & ~size_t(255);
  p.ws_part = reinterpret_cast<float*>(ws);
  p.ws_cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + part);
  const int CH = p.kslice / 256;
  dim3 grid(p.N / TILE_N, p.ksplit, mblocks);
  if (wfmt == T2B_WFMT_QPARAM) {
    if (pro != PRO_ACT || epi != EPI_STORE) return T2B_ERR_ARG;
    return gemv_dispatch<PRO_ACT, EPI_STORE, T2B_WFMT_QPARAM>(p, MB, CH, grid, st);
  }
  if (wfmt == T2B_WFMT_Q4NX) {
    if (pro == PRO_ACT && epi == EPI_STORE) return gemv_dispatch<PRO_ACT, EPI_STORE, T2B_WFMT_Q4NX>(p, MB, CH, grid, st);
    if (pro == PRO_ACT && epi == EPI_RESIDUAL)
      return gemv_dispatch<PRO_ACT, EPI_RESIDUAL, T2B_WFMT_Q4NX>(p, MB, CH, grid, st);
    if (pro == PRO_RMSNORM && epi == EPI_SWIGLU)
      return gemv_dispatch<PRO_RMSNORM, EPI_SWIGLU, T2B_WFMT_Q4NX>(p, MB, CH, grid, st);
    if (pro == PRO_RMSNORM && epi == EPI_QKV)
      return gemv_dispatch<PRO_RMSNORM, EPI_QKV, T2B_WFMT_Q4NX>(p, MB, CH, grid, st);
    return T2B_ERR_ARG;
  }
  if (pro == PRO_ACT && epi == EPI_STORE) return gemv_dispatch<PRO_ACT, EPI_STORE, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_STORE)
    return gemv_dispatch<PRO_RMSNORM, EPI_STORE, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  if (pro == PRO_ACT && epi == EPI_RESIDUAL)
    return gemv_dispatch<PRO_ACT, EPI_RESIDUAL, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_SWIGLU)
    return gemv_dispatch<PRO_RMSNORM, EPI_SWIGLU, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_QKV)
    return gemv_dispatch<PRO_RMSNORM, EPI_QKV, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  return T2B_ERR_ARG;
}

// tcgen05 path (w4a16_tc.cu)
int tc_launch(LinearParams& p, int pro, int epi, void* ws, size_t ws_bytes, cudaStream_t st);
size_t tc_ws_bytes(int M, int N, int K);
bool tc_supported(int M, int N, int K, bool q4);
bool tc_plan_info(int M, int N, int K, int* bp, int* s, int* ks, int max_rows);
long tc_grid_ctas(int M, int N, int K, bool q4);

// Rows at or above this count take the tcgen05 path (env T2B_TC_MIN_M overrides).
static int tc_min_m() {
  const char* e = getenv("T2B_TC_MIN_M");
  if (e && *e) {
    const int v = atoi(e);
    if (v > 0) return v;
  }
  return 2;
}

// large-M path (w4a16_prefill.cu)
int prefill_min_m();
int prefill_launch(LinearParams& p, int pro, int epi, cudaStream_t st);

static bool tiled_wfmt(int wfmt) { return wfmt == T2B_WFMT_T2B || wfmt == T2B_WFMT_Q4NX; }
// 16-bit activations: the tensor-core paths dequantise the weights to the same type
static bool half_act(int x_dtype) { return x_dtype == T2B_DTYPE_BF16 || x_dtype == T2B_DTYPE_F16; }

static bool use_prefill(int M, int wfmt, int x_dtype) {
  return tiled_wfmt(wfmt) && half_act(x_dtype) && M >= prefill_min_m();
}

// A decode batch on a linear so wide that the tcgen05 decode grid runs more
// than two waves of CTAs (each CTA holds one weight tile's k-slice and runs
// once): the large-M kernel's persistent CTAs stream whole weight tiles
// instead (Qwen3-8B at 64 rows: gate/up 115 -> 51 us, down 118 -> 71 us; the
// tensor-parallel rank at TP2: gate/up 60 -> 29 us, down 43 -> 39 us).  Not
// for the qkv epilogue, whose fp32 q output the large-M kernel does not
// write.  Env T2B_WIDE_MIN_CTAS sets the threshold (experiments; a negative
// value turns the rule off).
static bool use_prefill_wide(int M, int N, int K, int wfmt, int x_dtype, int epi) {
  if (epi == EPI_QKV || M < 16 || !tiled_wfmt(wfmt) || !half_act(x_dtype)) return false;
  long min_ctas = 2L * 148;
  if (const char* e = getenv("T2B_WIDE_MIN_CTAS")) {
    if (*e) min_ctas = atol(e);
  }
  if (min_ctas < 0) return false;
  return tc_grid_ctas(M, N, K, wfmt == T2B_WFMT_Q4NX) > min_ctas;
}

static bool use_tc(int M, int N, int K, int wfmt, int x_dtype) {
  return tiled_wfmt(wfmt) && half_act(x_dtype) && M >= tc_min_m() &&
         tc_supported(M, N, K, wfmt == T2B_WFMT_Q4NX);
}

// Split of the CUDA-core path's workspace: fp32 partials, then the tile
// counters (which must be zero before a call).  Zero sizes when the call
// needs no workspace.
void linear_workspace_layout(int M, int N, int K, size_t* partial_bytes, size_t* counter_bytes) {
  *partial_bytes = 0;
  *counter_bytes = 0;
  if (M < 1 || N % TILE_N || K % 256 || gemv_ws_bytes(M, N, K) == 0) return;
  const int MB = pick_mb(M);
  const int mblocks = (M + MB - 1) / MB;
  const int ksplit = K / pick_kslice(N, K, mblocks);
  *partial_bytes = ((size_t)mblocks * ksplit * MB * N * sizeof(float) + 255) & ~size_t(255);
  *counter_bytes = (((size_t)mblocks * (N / TILE_N) * sizeof(int) + 255) & ~size_t(255));
}

size_t linear_workspace_bytes(int M, int N, int K) {
  // the path is chosen per call from M; size for the larger so either fits
  const size_t a = gemv_ws_bytes(M, N, K);
  const size_t b = tc_ws_bytes(M, N, K);
  return a > b ? a : b;
}

int linear_launch(LinearParams& p, int pro, int epi, int wfmt, void* ws, size_t ws_bytes, cudaStream_t st) {
  p.err = error_word(st);
  p.q4nx = wfmt == T2B_WFMT_Q4NX ? 1 : 0;
  if (p.M < 1 || p.N <= 0 || p.K <= 0) return T2B_ERR_SHAPE;
  if (p.N % TILE_N || p.K % 256) return T2B_ERR_SHAPE;
  p.G = p.K / GROUP;
  if (use_prefill(p.M, wfmt, p.x_dtype)) return prefill_launch(p, pro, epi, st);
  if (use_prefill_wide(p.M, p.N, p.K, wfmt, p.x_dtype, epi)) return prefill_launch(p, pro, epi, st);
  if (use_tc(p.M, p.N, p.K, wfmt, p.x_dtype)) return tc_launch(p, pro, epi, ws, ws_bytes, st);
  return gemv_launch(p, pro, epi, wfmt, ws, ws_bytes, st);
}

}  // namespace t2b

// ===========================================================================
// C ABI
// ===========================================================================
using namespace t2b;

static inline bool al(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
static inline cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

static LinearParams gemv_base(const void* weight, const uint32_t* meta, int w_ld, int M, int N, int K) {
  LinearParams p{};
  p.qw = reinterpret_cast<const uint8_t*>(weight);
  p.meta = meta;
  p.w_ld = w_ld;
  p.M = M;
  p.N = N;
  p.K = K;
  return p;
}

static int linear_plan(int M, int N, int K, int max_rows, int* path, int* rows_per_cta, int* groups_per_cta,
                       int* ksplit) {
  if (!path || !rows_per_cta || !groups_per_cta || !ksplit) return T2B_ERR_ARG;
  if (M < 1 || N <= 0 || K <= 0 || N % TILE_N || K % 256) return T2B_ERR_SHAPE;
  if (use_prefill(M, T2B_WFMT_T2B, T2B_DTYPE_BF16) ||   // one weight tile x 128 rows per work unit, all of K
      (max_rows == 0 && use_prefill_wide(M, N, K, T2B_WFMT_T2B, T2B_DTYPE_BF16, EPI_STORE))) {
    *path = 2;
    *rows_per_cta = 128;
    *groups_per_cta = K / GROUP;
    *ksplit = 1;
    return T2B_OK;
  }
  if (use_tc(M, N, K, T2B_WFMT_T2B, T2B_DTYPE_BF16)) {
    *path = 1;
    tc_plan_info(M, N, K, rows_per_cta, groups_per_cta, ksplit, max_rows);
    return T2B_OK;
  }
  *path = 0;
  *rows_per_cta = pick_mb(M);
  const int kslice = pick_kslice(N, K, (M + *rows_per_cta - 1) / *rows_per_cta);
  *groups_per_cta = kslice / GROUP;
  *ksplit = K / kslice;
  return T2B_OK;
}

extern "C" int t2b_linear_plan(int M, int N, int K, int* path, int* rows_per_cta, int* groups_per_cta,
                               int* ksplit) {
  return linear_plan(M, N, K, 0, path, rows_per_cta, groups_per_cta, ksplit);
}

extern "C" int t2b_linear_plan_qkv(int M, int N, int K, int* path, int* rows_per_cta, int* groups_per_cta,
                                   int* ksplit) {
  return linear_plan(M, N, K, QKV_MAX_ROWS_PER_CTA, path, rows_per_cta, groups_per_cta, ksplit);
}

extern "C" size_t t2b_w4a16_gemm_workspace_bytes(int M, int N, int K) {
  if (M < 1 || N < 1 || K < 256) return 0;
  return linear_workspace_bytes(M, N, K);
}

namespace t2b {

// Host-side checks of a plain W4A16 GEMM call; fills the launch parameters.
int gemm_params(const void* weight, const uint32_t* meta, int wfmt, const void* x, int x_dtype, void* y,
                int y_dtype, int M, int N, int K, int group_size, LinearParams* out) {
  if (group_size != (wfmt == T2B_WFMT_Q4NX ? 32 : 128)) return T2B_ERR_SHAPE;
  if (!weight || !x || !y) return T2B_ERR_ARG;
  if (x_dtype < 0 || x_dtype > 2 || y_dtype < 0 || y_dtype > 2) return T2B_ERR_ARG;
  if (M < 1 || N <= 0 || K <= 0 || N % TILE_N || K % 256) return T2B_ERR_SHAPE;
  int w_ld;
  if (tiled_wfmt(wfmt)) {
    if (!meta) return T2B_ERR_ARG;
    if (!al(weight, 16) || !al(meta, 4)) return T2B_ERR_ALIGN;
    w_ld = K / 2;
  } else if (wfmt == T2B_WFMT_QPARAM) {
    if (!al(weight, 4)) return T2B_ERR_ALIGN;
    w_ld = K / 2 + 2 * (K / 128);
  } else {
    return T2B_ERR_ARG;
  }
  LinearParams p = gemv_base(weight, meta, w_ld, M, N, K);
  p.x = x;
  p.x_dtype = x_dtype;
  p.x_ld = K;
  p.y = y;
  p.y_dtype = y_dtype;
  p.y_ld = N;
  *out = p;
  return T2B_OK;
}

// Workspace the path this call takes needs: 0 on the tcgen05 and large-M
// paths (their split-K stays on chip), the CUDA-core split-K partials and
// tile counters otherwise (zero when its k-slices meet in a cluster).
void gemm_path_workspace(const LinearParams& p, int wfmt, size_t* partial_bytes, size_t* counter_bytes) {
  *partial_bytes = 0;
  *counter_bytes = 0;
  if (use_prefill(p.M, wfmt, p.x_dtype) || use_tc(p.M, p.N, p.K, wfmt, p.x_dtype)) return;
  linear_workspace_layout(p.M, p.N, p.K, partial_bytes, counter_bytes);
}

int gemm_launch(LinearParams& p, int wfmt, void* ws, size_t ws_bytes, cudaStream_t st) {
  return linear_launch(p, PRO_ACT, EPI_STORE, wfmt, ws, ws_bytes, st);
}

}  // namespace t2b

extern "C" int t2b_w4a16_gemm(const void* weight, const uint32_t* meta, int wfmt, const void* x, int x_dtype,
                              void* y, int y_dtype, int M, int N, int K, int group_size, void* ws, size_t ws_bytes,
                              void* stream) {
  LinearParams p;
  const int r = gemm_params(weight, meta, wfmt, x, x_dtype, y, y_dtype, M, N, K, group_size, &p);
  if (r != T2B_OK) return r;
  return gemm_launch(p, wfmt, ws, ws_bytes, S_(stream));
}

extern "C" int t2b_w4a16_gemm_push(const void* weight, const uint32_t* meta, int wfmt, const void* x, int x_dtype,
                                   void* y, int y_dtype, void* const* y_peers, int n_peers, int M, int N, int K,
                                   int group_size, void* ws, size_t ws_bytes, void* stream) {
  LinearParams p;
  const int r = gemm_params(weight, meta, wfmt, x, x_dtype, y, y_dtype, M, N, K, group_size, &p);
  if (r != T2B_OK) return r;
  if (n_peers < 0 || n_peers > 7 || (n_peers > 0 && !y_peers)) return T2B_ERR_ARG;
  if (y_dtype != T2B_DTYPE_BF16 && y_dtype != T2B_DTYPE_F32) return T2B_ERR_ARG;
  if (!al(y, 16)) return T2B_ERR_ALIGN;
  for (int q = 0; q < n_peers; ++q) {
    if (!y_peers[q]) return T2B_ERR_ARG;
    if (!al(y_peers[q], 16)) return T2B_ERR_ALIGN;
    p.y_peer[q] = y_peers[q];
  }
  p.n_y_peer = n_peers;
  return gemm_launch(p, wfmt, ws, ws_bytes, S_(stream));
}

extern "C" size_t t2b_qkv_workspace_bytes(int M, int H, int n_heads, int n_kv, int head_dim) {
  if (M < 1 || H < 256 || n_kv < 1) return 0;
  return linear_workspace_bytes(M, (n_heads + 2 * n_kv) * head_dim, H);
}

static int qkv_impl(const uint8_t* qw, const uint32_t* meta, int wfmt, int q_dtype, const uint16_t* xw, const float* ssq,
                    float eps,
                    const uint16_t* q_norm_w, const uint16_t* k_norm_w, const float* angles, const int32_t* pos,
                    const int32_t* row_seq, int n_seq, void* q_out, uint16_t* k_cache, uint16_t* v_cache,
                    float* ssq_clear, int M, int H, int n_heads, int n_kv, int head_dim, int max_ctx, void* ws,
                    size_t ws_bytes, void* stream) {
  if (head_dim != 64 && head_dim != 128) return T2B_ERR_SHAPE;
  if (n_kv < 1 || n_heads % n_kv || max_ctx < 1) return T2B_ERR_SHAPE;
  if (!tiled_wfmt(wfmt)) return T2B_ERR_ARG;
  if (q_dtype != T2B_DTYPE_BF16 && q_dtype != T2B_DTYPE_F32) return T2B_ERR_ARG;
  // fp32 q comes from the decode kernels' epilogue (rows <= 256, the attention's limit)
  if (q_dtype == T2B_DTYPE_F32 && use_prefill(M, wfmt, T2B_DTYPE_F16)) return T2B_ERR_SHAPE;
  if (!qw || !meta || !xw || !ssq || !angles || !pos || !q_out || !k_cache || !v_cache) return T2B_ERR_ARG;
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return T2B_ERR_ARG;
  if (!al(qw, 16) || !al(xw, 16)) return T2B_ERR_ALIGN;
  // vectorised epilogue: float4 angle rows, 8-byte bf16 stores, 8-byte norm weights
  if (!al(q_out, 16) || !al(k_cache, 16) || !al(v_cache, 16) || !al(angles, 16)) return T2B_ERR_ALIGN;
  if ((q_norm_w && !al(q_norm_w, 8)) || (k_norm_w && !al(k_norm_w, 8))) return T2B_ERR_ALIGN;
  const int N = (n_heads + 2 * n_kv) * head_dim;
  LinearParams p = gemv_base(qw, meta, H / 2, M, N, H);
  p.x = xw;
  p.x_dtype = T2B_DTYPE_F16;   // the fused layer's activations are fp16
  p.x_ld = H;
  p.ssq = ssq;
  p.eps = eps;
  p.y = q_out;
  p.y_dtype = q_dtype;
  p.y_ld = n_heads * head_dim;
  p.ssq_clear = ssq_clear;
  p.qn_w = reinterpret_cast<const __nv_bfloat16*>(q_norm_w);
  p.kn_w = reinterpret_cast<const __nv_bfloat16*>(k_norm_w);
  p.angles = angles;
  p.pos = pos;
  p.row_seq = row_seq;
  p.n_seq = n_seq;
  p.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache);
  p.n_heads = n_heads;
  p.n_kv = n_kv;
  p.head_dim = head_dim;
  p.max_ctx = max_ctx;
  return linear_launch(p, PRO_RMSNORM, EPI_QKV, wfmt, ws, ws_bytes, S_(stream));
}

extern "C" int t2b_qkv_norm_rope_kvwrite(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* xw,
                                         const float* ssq, float eps, const uint16_t* q_norm_w,
                                         const uint16_t* k_norm_w, const float* angles, const int32_t* pos,
                                         void* q_out, int q_dtype, uint16_t* k_cache, uint16_t* v_cache,
                                         float* ssq_clear,
                                         int M, int H, int n_heads, int n_kv, int head_dim, int max_ctx, void* ws,
                                         size_t ws_bytes, void* stream) {
  return qkv_impl(qw, meta, wfmt, q_dtype, xw, ssq, eps, q_norm_w, k_norm_w, angles, pos, nullptr, M, q_out, k_cache,
                  v_cache,
                  ssq_clear, M, H, n_heads, n_kv, head_dim, max_ctx, ws, ws_bytes, stream);
}

extern "C" int t2b_qkv_norm_rope_kvwrite_seq(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* xw,
                                             const float* ssq, float eps, const uint16_t* q_norm_w,
                                             const uint16_t* k_norm_w, const float* angles, const int32_t* pos,
                                             const int32_t* row_seq, int n_seq, uint16_t* q_out,
                                             uint16_t* k_cache, uint16_t* v_cache, float* ssq_clear, int M, int H,
                                             int n_heads, int n_kv, int head_dim, int max_ctx, void* ws,
                                             size_t ws_bytes, void* stream) {
  if (!row_seq) return T2B_ERR_ARG;
  if (n_seq < 1) return T2B_ERR_SHAPE;
  return qkv_impl(qw, meta, wfmt, T2B_DTYPE_BF16, xw, ssq, eps, q_norm_w, k_norm_w, angles, pos, row_seq, n_seq, q_out,
                  k_cache, v_cache,
                  ssq_clear, M, H, n_heads, n_kv, head_dim, max_ctx, ws, ws_bytes, stream);
}

extern "C" size_t t2b_oproj_residual_workspace_bytes(int M, int H, int K) {
  if (M < 1 || H < 128 || K < 256) return 0;
  return linear_workspace_bytes(M, H, K);
}

extern "C" int t2b_oproj_residual(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* attn, float* x_resid,
                                  float* ssq_out, const uint16_t* next_norm_w, uint16_t* xw_out, int M, int H, int K,
                                  void* ws, size_t ws_bytes, void* stream) {
  if (!qw || !meta || !attn || !x_resid || !ssq_out || !tiled_wfmt(wfmt)) return T2B_ERR_ARG;
  if ((next_norm_w == nullptr) != (xw_out == nullptr)) return T2B_ERR_ARG;
  if (!al(qw, 16) || !al(attn, 16)) return T2B_ERR_ALIGN;
  // vectorised epilogue: float4 residual rows, 8-byte bf16 stores
  if (!al(x_resid, 16) || (xw_out && (!al(xw_out, 8) || !al(next_norm_w, 8)))) return T2B_ERR_ALIGN;
  LinearParams p = gemv_base(qw, meta, K / 2, M, H, K);
  p.x = attn;
  p.x_dtype = T2B_DTYPE_F16;   // the fused layer's activations are fp16
  p.x_ld = K;
  p.resid = x_resid;
  p.y_ld = H;
  p.ssq_out = ssq_out;
  p.next_w = reinterpret_cast<const __nv_bfloat16*>(next_norm_w);
  p.xw_out = reinterpret_cast<__half*>(xw_out);
  return linear_launch(p, PRO_ACT, EPI_RESIDUAL, wfmt, ws, ws_bytes, S_(stream));
}

extern "C" size_t t2b_upgate_swiglu_workspace_bytes(int M, int H, int I) {
  if (M < 1 || H < 256 || I < 64) return 0;
  return linear_workspace_bytes(M, 2 * I, H);
}

extern "C" int t2b_upgate_swiglu(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* xw, const float* ssq,
                                 float eps, uint16_t* h_out, float* ssq_clear, int M, int H, int I, void* ws,
                                 size_t ws_bytes, void* stream) {
  if (I % 64) return T2B_ERR_SHAPE;
  if (!qw || !meta || !xw || !ssq || !h_out || !tiled_wfmt(wfmt)) return T2B_ERR_ARG;
  if (!al(qw, 16) || !al(xw, 16) || !al(h_out, 8)) return T2B_ERR_ALIGN;
  LinearParams p = gemv_base(qw, meta, H / 2, M, 2 * I, H);
  p.x = xw;
  p.x_dtype = T2B_DTYPE_F16;   // the fused layer's activations are fp16
  p.x_ld = H;
  p.ssq = ssq;
  p.eps = eps;
  p.y = h_out;
  p.y_ld = I;
  p.ssq_clear = ssq_clear;
  return linear_launch(p, PRO_RMSNORM, EPI_SWIGLU, wfmt, ws, ws_bytes, S_(stream));
}

extern "C" size_t t2b_down_residual_workspace_bytes(int M, int H, int I) {
  if (M < 1 || H < 128 || I < 256) return 0;
  return linear_workspace_bytes(M, H, I);
}

extern "C" int t2b_down_residual(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* h, float* x_resid,
                                 float* ssq_out, const uint16_t* next_norm_w, uint16_t* xw_out, int M, int H, int I,
                                 void* ws, size_t ws_bytes, void* stream) {
  return t2b_oproj_residual(qw, meta, wfmt, h, x_resid, ssq_out, next_norm_w, xw_out, M, H, I, ws, ws_bytes, stream);
}

T2B_TRACE_DUMP_FN(t2b_trace_dump_gemv)
