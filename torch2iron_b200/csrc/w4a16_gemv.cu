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
//   * the 8 lanes of a row reduce with 3 xor-shuffles; k-slices (split-K)
//     meet in a fp32 workspace and the last CTA of a tile (ticket counter)
//     runs the epilogue on the full 128-row tile.
//
// Algorithmic parity: W[n,k] = (q - zero) * scale exactly as
// src/models/fast_qwen3/fast_packed_format.py:158-160; fp32 accumulation as
// src/models/quantized_qwen3/model.py:133-146.

#include "t2b_common.cuh"
#include "launch.cuh"

namespace t2b {

enum Prologue { PRO_ACT = 0, PRO_RMSNORM = 1 };
enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

constexpr int GV_THREADS = 256;
constexpr int GV_TILE = 128;

struct GemvParams {
  const uint8_t* qw;      // weight rows (T2B: [N][K/2]; QPARAM: [N][K/2+2G])
  const uint32_t* meta;   // T2B meta [N][G]
  int w_ld;               // bytes per weight row
  int N, K, G;
  const void* x;          // activations [M][x_ld]
  int x_dtype, x_ld;
  const float* ssq;       // PRO_RMSNORM: sum of squares per row
  const __nv_bfloat16* norm_w;
  float eps;
  int M, kslice, ksplit;
  float* ws_part;         // [mblocks][ksplit][MB][N]
  int* ws_cnt;            // [mblocks][N/128]
  void* y;                // EPI_STORE output / EPI_SWIGLU h / EPI_QKV q_out
  int y_dtype, y_ld;
  float* resid;           // EPI_RESIDUAL fp32 [M][y_ld]
  float* ssq_out;
  float* ssq_clear;
  const __nv_bfloat16* qn_w;
  const __nv_bfloat16* kn_w;
  const float* angles;
  const int* pos;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int n_heads, n_kv, head_dim, max_ctx;
};

template <int MB, int CH>
struct GemvSmem {
  static constexpr int XS_LD = CH * 288;  // 256 k per chunk, +4 floats pad per 32 (bank spread)
  static constexpr int XS_FLOATS = MB * XS_LD;
  static constexpr int TILE_FLOATS = MB * GV_TILE;
  static constexpr size_t BYTES = sizeof(float) * (XS_FLOATS + TILE_FLOATS + 2 * MB * 4);
};

T2B_DEV uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

T2B_DEV float nib_f(uint32_t v, int sel) { return __uint_as_float(__byte_perm(v, 0x43000000u, sel)); }

template <int MB, int CH, int PRO, int EPI, int WFMT>
__global__ void __launch_bounds__(GV_THREADS) w4a16_gemv_kernel(const GemvParams p) {
  using S = GemvSmem<MB, CH>;
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;
  float* tile_acc = smem + S::XS_FLOATS;
  float* scratch = tile_acc + S::TILE_FLOATS;   // [MB][4] rstd etc.

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, mblk = blockIdx.z;
  const int row0 = tile * GV_TILE;
  const int k0 = split * p.kslice;
  const int m0 = mblk * MB;

  // ---- 1. weight prefetch (independent of the previous kernel) ----------
  uint4 wv[CH][4];
  uint32_t mt[CH][4];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = row0 + warp * 16 + i * 4 + (lane >> 3);
      const int k = k0 + c * 256 + (lane & 7) * 32;
      const uint8_t* rowp = p.qw + (size_t)r * p.w_ld;
      if (WFMT == T2B_WFMT_T2B) {
        wv[c][i] = ldg_stream(rowp + (k >> 1));
      } else {  // qparam rows are K/2 + 2G bytes: only 4-byte aligned
        const uint32_t* w4 = reinterpret_cast<const uint32_t*>(rowp + (k >> 1));
        wv[c][i] = make_uint4(__ldg(w4), __ldg(w4 + 1), __ldg(w4 + 2), __ldg(w4 + 3));
      }
      if (WFMT == T2B_WFMT_T2B) {
        mt[c][i] = __ldg(p.meta + (size_t)r * p.G + (k >> 7));
      } else {
        mt[c][i] = __ldg(reinterpret_cast<const unsigned short*>(rowp + (p.K >> 1)) + (k >> 7));
      }
    }
  }

  grid_dep_wait();
  grid_dep_launch();

  // ---- 2. prologue: activations of this k-slice into shared fp32 --------
  if (PRO == PRO_RMSNORM) {
    if (threadIdx.x < MB) {
      const int m = m0 + threadIdx.x;
      scratch[threadIdx.x] = (m < p.M) ? rsqrtf(p.ssq[m] / (float)p.K + p.eps) : 0.f;
    }
    __syncthreads();
  }
  for (int idx = threadIdx.x; idx < MB * CH * 256; idx += GV_THREADS) {
    const int b = idx / (CH * 256), kk = idx - b * (CH * 256);
    const int m = m0 + b;
    float v = 0.f;
    if (m < p.M) {
      if (PRO == PRO_ACT) {
        v = load_act(p.x, p.x_dtype, (size_t)m * p.x_ld + k0 + kk);
      } else {
        // model.py:179-181: x * rsqrt(mean(x^2)+eps), then * weight; A16 -> bf16
        const float xv = reinterpret_cast<const float*>(p.x)[(size_t)m * p.x_ld + k0 + kk];
        v = round_bf16((xv * scratch[b]) * __bfloat162float(p.norm_w[k0 + kk]));
      }
    }
    xs[b * S::XS_LD + kk + (kk >> 5) * 4] = v;
  }
  if (p.ssq_clear != nullptr && tile == 0 && split == 0 && mblk == 0) {
    for (int i = threadIdx.x; i < p.M; i += GV_THREADS) p.ssq_clear[i] = 0.f;
  }
  __syncthreads();

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
        wf[i][0] = fmaf(nib_f(lo, 0x7054), sc[i], zc[i]);
        wf[i][1] = fmaf(nib_f(hi, 0x7054), sc[i], zc[i]);
        wf[i][2] = fmaf(nib_f(lo, 0x7154), sc[i], zc[i]);
        wf[i][3] = fmaf(nib_f(hi, 0x7154), sc[i], zc[i]);
        wf[i][4] = fmaf(nib_f(lo, 0x7254), sc[i], zc[i]);
        wf[i][5] = fmaf(nib_f(hi, 0x7254), sc[i], zc[i]);
        wf[i][6] = fmaf(nib_f(lo, 0x7354), sc[i], zc[i]);
        wf[i][7] = fmaf(nib_f(hi, 0x7354), sc[i], zc[i]);
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

  // ---- 4. reduce the 8 lanes of each row, publish the partial ------------
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int b = 0; b < MB; ++b) {
      float v = acc[i][b];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      acc[i][b] = v;
    }
  const int ntiles = p.N / GV_TILE;
  if (p.ksplit == 1) {
    if ((lane & 7) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int b = 0; b < MB; ++b) tile_acc[b * GV_TILE + warp * 16 + i * 4 + (lane >> 3)] = acc[i][b];
    }
    __syncthreads();
  } else {
    if ((lane & 7) == 0) {
      float* part = p.ws_part + ((size_t)(mblk * p.ksplit + split) * MB) * p.N;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int b = 0; b < MB; ++b) part[(size_t)b * p.N + row0 + warp * 16 + i * 4 + (lane >> 3)] = acc[i][b];
    }
    if (!split_ticket(p.ws_cnt + mblk * ntiles + tile, p.ksplit)) return;
    for (int idx = threadIdx.x; idx < MB * GV_TILE; idx += GV_THREADS) {
      const int b = idx / GV_TILE, lr = idx - b * GV_TILE;
      const float* base = p.ws_part + ((size_t)mblk * p.ksplit * MB + b) * p.N + row0 + lr;
      float s = 0.f;
      for (int sp = 0; sp < p.ksplit; ++sp) s += ldcg(base + (size_t)sp * MB * p.N);
      tile_acc[idx] = s;
    }
    __syncthreads();
  }

  // ---- 5. epilogues ------------------------------------------------------
  if (EPI == EPI_STORE) {
    for (int idx = threadIdx.x; idx < MB * GV_TILE; idx += GV_THREADS) {
      const int b = idx / GV_TILE, lr = idx - b * GV_TILE, m = m0 + b;
      if (m < p.M) store_act(p.y, p.y_dtype, (size_t)m * p.y_ld + row0 + lr, tile_acc[idx]);
    }
  } else if (EPI == EPI_RESIDUAL) {
    // 256 threads cover 2 batch rows x 128 tile rows per pass; each warp's
    // 32 elements belong to one batch row -> one atomic per warp per pass.
    for (int base = 0; base < MB * GV_TILE; base += GV_THREADS) {
      const int idx = base + threadIdx.x;
      const int b = idx / GV_TILE, lr = idx - b * GV_TILE, m = m0 + b;
      float sq = 0.f;
      if (idx < MB * GV_TILE && m < p.M) {
        float* xr = p.resid + (size_t)m * p.y_ld + row0 + lr;
        const float v = *xr + tile_acc[idx];
        *xr = v;
        sq = v * v;
      }
      sq = warp_sum(sq);
      if (lane == 0 && idx < MB * GV_TILE && m < p.M) atomicAdd(p.ssq_out + m, sq);
    }
  } else if (EPI == EPI_SWIGLU) {
    // tile = 64 gate rows then the matching 64 up rows (model.py:215-216)
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.y);
    for (int idx = threadIdx.x; idx < MB * 64; idx += GV_THREADS) {
      const int b = idx >> 6, t = idx & 63, m = m0 + b;
      if (m < p.M) {
        const float g = tile_acc[b * GV_TILE + t];
        const float u = tile_acc[b * GV_TILE + 64 + t];
        const float silu = g / (1.f + expf(-g));
        h[(size_t)m * p.y_ld + tile * 64 + t] = __float2bfloat16_rn(silu * u);
      }
    }
  } else {  // EPI_QKV
    const int hd = p.head_dim;
    const int hpt = GV_TILE / hd;  // heads per tile (1 or 2)
    const int nq = p.n_heads, nkv = p.n_kv;
    // per (b, head) inverse rms for q/k heads with QK-norm (model.py:252-253)
    for (int pair = warp; pair < MB * hpt; pair += GV_THREADS / 32) {
      const int b = pair / hpt, hl = pair - b * hpt;
      const int head = (row0 / hd) + hl;
      float ss = 0.f;
      for (int d = lane; d < hd; d += 32) {
        const float v = tile_acc[b * GV_TILE + hl * hd + d];
        ss += v * v;
      }
      ss = warp_sum(ss);
      if (lane == 0) {
        const bool normed = (head < nq && p.qn_w) || (head >= nq && head < nq + nkv && p.kn_w);
        scratch[MB * 4 + pair] = normed ? rsqrtf(ss / (float)hd + p.eps) : 1.f;
      }
    }
    __syncthreads();
    __nv_bfloat16* q_out = reinterpret_cast<__nv_bfloat16*>(p.y);
    for (int idx = threadIdx.x; idx < MB * GV_TILE; idx += GV_THREADS) {
      const int b = idx / GV_TILE, lr = idx - b * GV_TILE, m = m0 + b;
      if (m >= p.M) continue;
      const int hl = lr / hd, d = lr - hl * hd;
      const int head = (row0 / hd) + hl;
      const float* tv = tile_acc + b * GV_TILE + hl * hd;
      const int pos = p.pos[m];
      if (head >= nq + nkv) {  // value head: stored as projected (model.py:250,263)
        const int kvh = head - nq - nkv;
        p.v_cache[(((size_t)m * nkv + kvh) * p.max_ctx + pos) * hd + d] = __float2bfloat16_rn(tv[d]);
        continue;
      }
      const bool is_q = head < nq;
      const __nv_bfloat16* nw = is_q ? p.qn_w : p.kn_w;
      const float rs = scratch[MB * 4 + b * hpt + hl];
      const int d0 = d & ~1;
      float x0 = tv[d0], x1 = tv[d0 + 1];
      if (nw) {
        x0 = (x0 * rs) * __bfloat162float(nw[d0]);
        x1 = (x1 * rs) * __bfloat162float(nw[d0 + 1]);
      }
      // interleaved RoPE (model.py:184-196): out[2i] = x0 c - x1 s ; out[2i+1] = x1 c + x0 s
      const float c = p.angles[(size_t)pos * hd + d0];
      const float s = p.angles[(size_t)pos * hd + d0 + 1];
      const float o = (d & 1) ? (x1 * c + x0 * s) : (x0 * c - x1 * s);
      if (is_q) {
        q_out[(size_t)m * p.y_ld + head * hd + d] = __float2bfloat16_rn(o);
      } else {
        const int kvh = head - nq;
        p.k_cache[(((size_t)m * nkv + kvh) * p.max_ctx + pos) * hd + d] = __float2bfloat16_rn(o);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host-side launcher
// ---------------------------------------------------------------------------

static int pick_mb(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

// k-slice: 256 or 512 per CTA, chosen so the grid has about 1-4 CTAs per SM.
static int pick_kslice(int N, int K, int mblocks) {
  const long tiles = (long)(N / GV_TILE) * mblocks;
  if (K % 512 == 0 && tiles * (K / 256) > 4L * 148) return 512;
  return 256;
}

size_t gemv_workspace_bytes(int M, int N, int K) {
  const int MB = pick_mb(M);
  const int mblocks = (M + MB - 1) / MB;
  const int kslice = pick_kslice(N, K, mblocks);
  const int ksplit = K / kslice;
  if (ksplit == 1) return 0;
  size_t part = (size_t)mblocks * ksplit * MB * N * sizeof(float);
  part = (part + 255) & ~size_t(255);
  size_t cnt = (size_t)mblocks * (N / GV_TILE) * sizeof(int);
  return part + ((cnt + 255) & ~size_t(255));
}

template <int MB, int CH, int PRO, int EPI, int WFMT>
static int launch_t(GemvParams& p, dim3 grid, cudaStream_t st) {
  auto kern = w4a16_gemv_kernel<MB, CH, PRO, EPI, WFMT>;
  const size_t smem = GemvSmem<MB, CH>::BYTES;  // <= 23 KB for every instantiation
  return launch_pdl(kern, grid, dim3(GV_THREADS), smem, st, p);
}

template <int PRO, int EPI, int WFMT>
static int dispatch_mb(GemvParams& p, int MB, int CH, dim3 grid, cudaStream_t st) {
#define T2B_CASE(mb, ch) \
  if (MB == mb && CH == ch) return launch_t<mb, ch, PRO, EPI, WFMT>(p, grid, st);
  T2B_CASE(1, 1) T2B_CASE(1, 2) T2B_CASE(2, 1) T2B_CASE(2, 2)
  T2B_CASE(4, 1) T2B_CASE(4, 2) T2B_CASE(8, 1) T2B_CASE(8, 2)
#undef T2B_CASE
  return T2B_ERR_ARG;
}

// Fills the split / workspace fields of `p` and launches.
int gemv_launch(GemvParams& p, int pro, int epi, int wfmt, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (p.M < 1 || p.N <= 0 || p.K <= 0) return T2B_ERR_SHAPE;
  if (p.N % GV_TILE || p.K % 256) return T2B_ERR_SHAPE;
  const int MB = pick_mb(p.M);
  const int mblocks = (p.M + MB - 1) / MB;
  p.kslice = pick_kslice(p.N, p.K, mblocks);
  p.ksplit = p.K / p.kslice;
  p.G = p.K / 128;
  if (ws_bytes < gemv_workspace_bytes(p.M, p.N, p.K) || (p.ksplit > 1 && ws == nullptr)) return T2B_ERR_WORKSPACE;
  size_t part = (size_t)mblocks * p.ksplit * MB * p.N * sizeof(float);
  part = (part + 255) & ~size_t(255);
  p.ws_part = reinterpret_cast<float*>(ws);
  p.ws_cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + part);
  const int CH = p.kslice / 256;
  dim3 grid(p.N / GV_TILE, p.ksplit, mblocks);
  if (wfmt == T2B_WFMT_QPARAM) {
    if (pro != PRO_ACT || epi != EPI_STORE) return T2B_ERR_ARG;
    return dispatch_mb<PRO_ACT, EPI_STORE, T2B_WFMT_QPARAM>(p, MB, CH, grid, st);
  }
  if (pro == PRO_ACT && epi == EPI_STORE) return dispatch_mb<PRO_ACT, EPI_STORE, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_STORE)
    return dispatch_mb<PRO_RMSNORM, EPI_STORE, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  if (pro == PRO_ACT && epi == EPI_RESIDUAL)
    return dispatch_mb<PRO_ACT, EPI_RESIDUAL, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_SWIGLU)
    return dispatch_mb<PRO_RMSNORM, EPI_SWIGLU, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  if (pro == PRO_RMSNORM && epi == EPI_QKV) return dispatch_mb<PRO_RMSNORM, EPI_QKV, T2B_WFMT_T2B>(p, MB, CH, grid, st);
  return T2B_ERR_ARG;
}

}  // namespace t2b

// ===========================================================================
// C ABI
// ===========================================================================
using namespace t2b;

static inline bool al(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
static inline cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

static GemvParams gemv_base(const void* weight, const uint32_t* meta, int w_ld, int M, int N, int K) {
  GemvParams p{};
  p.qw = reinterpret_cast<const uint8_t*>(weight);
  p.meta = meta;
  p.w_ld = w_ld;
  p.M = M;
  p.N = N;
  p.K = K;
  return p;
}

extern "C" size_t t2b_w4a16_gemm_workspace_bytes(int M, int N, int K) {
  if (M < 1 || N < 1 || K < 256) return 0;
  return gemv_workspace_bytes(M, N, K);
}

extern "C" int t2b_w4a16_gemm(const void* weight, const uint32_t* meta, int wfmt, const void* x, int x_dtype,
                              void* y, int y_dtype, int M, int N, int K, int group_size, void* ws, size_t ws_bytes,
                              void* stream) {
  if (group_size != 128) return T2B_ERR_SHAPE;
  if (!weight || !x || !y) return T2B_ERR_ARG;
  if (x_dtype < 0 || x_dtype > 2 || y_dtype < 0 || y_dtype > 2) return T2B_ERR_ARG;
  int w_ld;
  if (wfmt == T2B_WFMT_T2B) {
    if (!meta) return T2B_ERR_ARG;
    if (!al(weight, 16) || !al(meta, 4)) return T2B_ERR_ALIGN;
    w_ld = K / 2;
  } else if (wfmt == T2B_WFMT_QPARAM) {
    if (!al(weight, 4)) return T2B_ERR_ALIGN;
    w_ld = K / 2 + 2 * (K / 128);
  } else {
    return T2B_ERR_ARG;
  }
  GemvParams p = gemv_base(weight, meta, w_ld, M, N, K);
  p.x = x;
  p.x_dtype = x_dtype;
  p.x_ld = K;
  p.y = y;
  p.y_dtype = y_dtype;
  p.y_ld = N;
  return gemv_launch(p, PRO_ACT, EPI_STORE, wfmt, ws, ws_bytes, S_(stream));
}

extern "C" size_t t2b_qkv_workspace_bytes(int M, int H, int n_heads, int n_kv, int head_dim) {
  if (M < 1 || H < 256 || n_kv < 1) return 0;
  return gemv_workspace_bytes(M, (n_heads + 2 * n_kv) * head_dim, H);
}

extern "C" int t2b_qkv_norm_rope_kvwrite(const uint8_t* qw, const uint32_t* meta, const float* x_resid,
                                         const float* ssq, const uint16_t* ln_w, float eps, const uint16_t* q_norm_w,
                                         const uint16_t* k_norm_w, const float* angles, const int32_t* pos,
                                         uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, float* ssq_clear,
                                         int M, int H, int n_heads, int n_kv, int head_dim, int max_ctx, void* ws,
                                         size_t ws_bytes, void* stream) {
  if (head_dim != 64 && head_dim != 128) return T2B_ERR_SHAPE;
  if (n_kv < 1 || n_heads % n_kv || max_ctx < 1) return T2B_ERR_SHAPE;
  if (!qw || !meta || !x_resid || !ssq || !ln_w || !angles || !pos || !q_out || !k_cache || !v_cache)
    return T2B_ERR_ARG;
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return T2B_ERR_ARG;
  if (!al(qw, 16)) return T2B_ERR_ALIGN;
  const int N = (n_heads + 2 * n_kv) * head_dim;
  GemvParams p = gemv_base(qw, meta, H / 2, M, N, H);
  p.x = x_resid;
  p.x_dtype = T2B_DTYPE_F32;
  p.x_ld = H;
  p.ssq = ssq;
  p.norm_w = reinterpret_cast<const __nv_bfloat16*>(ln_w);
  p.eps = eps;
  p.y = q_out;
  p.y_ld = n_heads * head_dim;
  p.ssq_clear = ssq_clear;
  p.qn_w = reinterpret_cast<const __nv_bfloat16*>(q_norm_w);
  p.kn_w = reinterpret_cast<const __nv_bfloat16*>(k_norm_w);
  p.angles = angles;
  p.pos = pos;
  p.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache);
  p.n_heads = n_heads;
  p.n_kv = n_kv;
  p.head_dim = head_dim;
  p.max_ctx = max_ctx;
  return gemv_launch(p, PRO_RMSNORM, EPI_QKV, T2B_WFMT_T2B, ws, ws_bytes, S_(stream));
}

extern "C" size_t t2b_oproj_residual_workspace_bytes(int M, int H, int K) {
  if (M < 1 || H < 128 || K < 256) return 0;
  return gemv_workspace_bytes(M, H, K);
}

extern "C" int t2b_oproj_residual(const uint8_t* qw, const uint32_t* meta, const uint16_t* attn, float* x_resid,
                                  float* ssq_out, int M, int H, int K, void* ws, size_t ws_bytes, void* stream) {
  if (!qw || !meta || !attn || !x_resid || !ssq_out) return T2B_ERR_ARG;
  if (!al(qw, 16)) return T2B_ERR_ALIGN;
  GemvParams p = gemv_base(qw, meta, K / 2, M, H, K);
  p.x = attn;
  p.x_dtype = T2B_DTYPE_BF16;
  p.x_ld = K;
  p.resid = x_resid;
  p.y_ld = H;
  p.ssq_out = ssq_out;
  return gemv_launch(p, PRO_ACT, EPI_RESIDUAL, T2B_WFMT_T2B, ws, ws_bytes, S_(stream));
}

extern "C" size_t t2b_upgate_swiglu_workspace_bytes(int M, int H, int I) {
  if (M < 1 || H < 256 || I < 64) return 0;
  return gemv_workspace_bytes(M, 2 * I, H);
}

extern "C" int t2b_upgate_swiglu(const uint8_t* qw, const uint32_t* meta, const float* x_resid, const float* ssq,
                                 const uint16_t* ln_w, float eps, uint16_t* h_out, float* ssq_clear, int M, int H,
                                 int I, void* ws, size_t ws_bytes, void* stream) {
  if (I % 64) return T2B_ERR_SHAPE;
  if (!qw || !meta || !x_resid || !ssq || !ln_w || !h_out) return T2B_ERR_ARG;
  if (!al(qw, 16)) return T2B_ERR_ALIGN;
  GemvParams p = gemv_base(qw, meta, H / 2, M, 2 * I, H);
  p.x = x_resid;
  p.x_dtype = T2B_DTYPE_F32;
  p.x_ld = H;
  p.ssq = ssq;
  p.norm_w = reinterpret_cast<const __nv_bfloat16*>(ln_w);
  p.eps = eps;
  p.y = h_out;
  p.y_ld = I;
  p.ssq_clear = ssq_clear;
  return gemv_launch(p, PRO_RMSNORM, EPI_SWIGLU, T2B_WFMT_T2B, ws, ws_bytes, S_(stream));
}

extern "C" size_t t2b_down_residual_workspace_bytes(int M, int H, int I) {
  if (M < 1 || H < 128 || I < 256) return 0;
  return gemv_workspace_bytes(M, H, I);
}

extern "C" int t2b_down_residual(const uint8_t* qw, const uint32_t* meta, const uint16_t* h, float* x_resid,
                                 float* ssq_out, int M, int H, int I, void* ws, size_t ws_bytes, void* stream) {
  return t2b_oproj_residual(qw, meta, h, x_resid, ssq_out, M, H, I, ws, ws_bytes, stream);
}
