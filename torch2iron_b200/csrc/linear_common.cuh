// Shared pieces of the W4A16 linear kernels (CUDA-core GEMV and tcgen05
// GEMM): parameters, the tiled T2B weight layout, the split-K fixup and the
// fused decode-layer epilogues.
//
// T2B weight layout (one [N, K] linear, group 128, N % 128 == 0):
//   qw   block (nt, g) = 128 rows x 128 k = 8192 bytes at ((nt*G + g) * 8192);
//        inside a block, piece p (k 32p..32p+31) of row r is 16 bytes at
//        p*2048 + r*16: four little-endian words; word j covers k0 = 32p+8j and
//        holds unsigned AutoGPTQ nibbles even-k first: nibble slot t = q[k0+2t]
//        for t < 4, q[k0+2(t-4)+1] for t >= 4.  So (w >> 4t) & 0x000F000F puts
//        the adjacent pair (k0+2t, k0+2t+1) in the two 16-bit halves.
//   meta block (nt, g) = 128 uint32 at ((nt*G + g) * 128): fp16 scale | zero << 16.
// One block is one contiguous 8 KB + 512 B pair, so a (128-row tile, group)
// stage is a single bulk copy, and a warp reading one piece of 32 rows reads
// 512 contiguous bytes.
#pragma once

#include <cuda.h>

#include "t2b_common.cuh"

namespace t2b {

enum Prologue { PRO_ACT = 0, PRO_RMSNORM = 1 };
enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

constexpr int TILE_N = 128;          // weight rows per output tile
constexpr int GROUP = 128;           // quantization group along K
constexpr int BLOCK_BYTES = TILE_N * GROUP / 2;

struct LinearParams {
  CUtensorMap xmap;       // tcgen05 path: 2-D tiled map of x (bf16 [M][K]), 64 x BP box, 128B swizzle
  const uint8_t* qw;      // T2B: tiled blocks; QPARAM: [N][K/2 + 2G] rows
  const uint32_t* meta;   // T2B meta blocks
  int w_ld;               // QPARAM bytes per row
  int N, K, G;
  const void* x;          // activations [M][x_ld]
  int x_dtype, x_ld;
  const float* ssq;       // PRO_RMSNORM: sum of squares of the un-normalised row
  float eps;              // PRO_RMSNORM: x is bf16(row * norm weight); y *= rsqrt(ssq/K + eps)
  int M, kslice, ksplit;  // kslice: k per CTA (multiple of 128)
  float* ws_part;         // [mblocks][ksplit][MB][N]
  int* ws_cnt;            // [mblocks][N/128]
  void* y;                // EPI_STORE output / EPI_SWIGLU h / EPI_QKV q_out
  int y_dtype, y_ld;
  float* resid;           // EPI_RESIDUAL fp32 [M][y_ld]
  float* ssq_out;
  const __nv_bfloat16* next_w;  // EPI_RESIDUAL: next RMSNorm weight [N] (nullable)
  __nv_bfloat16* xw_out;        // EPI_RESIDUAL: bf16(resid * next_w) [M][y_ld] (nullable)
  float* ssq_clear;
  const __nv_bfloat16* qn_w;
  const __nv_bfloat16* kn_w;
  const float* angles;
  const int* pos;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int n_heads, n_kv, head_dim, max_ctx;
  int* err;
};

T2B_DEV size_t qw_block_offset(int nt, int g, int G) { return ((size_t)nt * G + g) * BLOCK_BYTES; }
T2B_DEV size_t meta_block_offset(int nt, int g, int G) { return ((size_t)nt * G + g) * TILE_N; }

// ---------------------------------------------------------------------------
// Split-K: publish this CTA's [MB][128] partial (already in `tile_acc`) and,
// if it is the last of the tile's k-splits, leave the full sum in `tile_acc`.
// Returns false for CTAs that must exit.
// ---------------------------------------------------------------------------
template <int MB>
T2B_DEV bool splitk_fixup(const LinearParams& p, float* tile_acc, int tile, int split, int mblk, int nthreads) {
  if (p.ksplit == 1) return true;
  float* part = p.ws_part + ((size_t)(mblk * p.ksplit + split) * MB) * p.N + (size_t)tile * TILE_N;
  for (int idx = threadIdx.x; idx < MB * TILE_N; idx += nthreads) {
    const int b = idx / TILE_N, lr = idx - b * TILE_N;
    part[(size_t)b * p.N + lr] = tile_acc[idx];
  }
  if (!split_ticket(p.ws_cnt + mblk * (p.N / TILE_N) + tile, p.ksplit)) return false;
  for (int idx = threadIdx.x; idx < MB * TILE_N; idx += nthreads) {
    const int b = idx / TILE_N, lr = idx - b * TILE_N;
    const float* base = p.ws_part + ((size_t)mblk * p.ksplit * MB + b) * p.N + (size_t)tile * TILE_N + lr;
    float s = 0.f;
    for (int sp = 0; sp < p.ksplit; ++sp) s += ldcg(base + (size_t)sp * MB * p.N);
    tile_acc[idx] = s;
  }
  __syncthreads();
  return true;
}



// Epilogue inputs staged in shared memory ahead of time (any may be null:
// the epilogue then reads global memory).
struct EpiCache {
  const int* pos;              // [MB] positions of the epilogue rows
  const float* angles;         // [MB][head_dim] their RoPE rows
  const __nv_bfloat16* qn;     // [head_dim]
  const __nv_bfloat16* kn;     // [head_dim]
  const float* resid;          // [MB][128] residual tile rows
  const __nv_bfloat16* next_w; // [128] next-norm weight slice of this tile
};

// ---------------------------------------------------------------------------
// QKV epilogue (model.py:248-264): per 128-row tile = 128/HD heads of q, k or v
// for MB batch rows.  q/k heads: per-head RMSNorm (when weights are given),
// then interleaved RoPE on (x[2i], x[2i+1]) pairs; q goes to q_out, k/v to the
// cache at the row's position.  Work item = (row, dimension pair): float2
// reads, one bf16x2 store, no runtime division.
// ---------------------------------------------------------------------------
template <int HD>
T2B_DEV void qkv_epilogue(const LinearParams& p, const float* tile_acc, float* scratch, int tile, int m0, int MB,
                          const EpiCache& ec) {
  constexpr int NT = 256;
  constexpr int HPT = TILE_N / HD;  // heads per tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head0 = tile * HPT;
  const int nq = p.n_heads, nkv = p.n_kv;
  // per (row, head) inverse RMS over the head (model.py:179-180 on q/k heads)
  for (int pair = warp; pair < MB * HPT; pair += NT / 32) {
    const int b = pair / HPT, hl = pair - b * HPT;
    const int head = head0 + hl;
    float ss = 0.f;
#pragma unroll
    for (int d = lane; d < HD; d += 32) {
      const float v = tile_acc[b * TILE_N + hl * HD + d];
      ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) {
      const bool normed = (head < nq && p.qn_w) || (head >= nq && head < nq + nkv && p.kn_w);
      scratch[pair] = normed ? rsqrtf(ss / (float)HD + p.eps) : 1.f;
    }
  }
  __syncthreads();
  __nv_bfloat16* q_out = reinterpret_cast<__nv_bfloat16*>(p.y);
  const __nv_bfloat16* qn = ec.qn ? ec.qn : p.qn_w;
  const __nv_bfloat16* kn = ec.kn ? ec.kn : p.kn_w;
  for (int it = threadIdx.x; it < MB * (TILE_N / 2); it += NT) {
    const int b = it / (TILE_N / 2), pr = it - b * (TILE_N / 2);   // pr: pair index inside the tile
    const int m = m0 + b;
    if (m >= p.M) continue;
    const int hl = (2 * pr) / HD, d0 = 2 * pr - hl * HD;
    const int head = head0 + hl;
    const int pos = ec.pos ? ec.pos[b] : p.pos[m];
    const bool in_cache = pos >= 0 && pos < p.max_ctx;   // a bad position writes no cache entry
    const float2 xv = *reinterpret_cast<const float2*>(tile_acc + b * TILE_N + 2 * pr);
    if (head >= nq + nkv) {  // value head: stored as projected (model.py:250,263)
      if (in_cache)
        *reinterpret_cast<__nv_bfloat162*>(
            &p.v_cache[(((size_t)m * nkv + (head - nq - nkv)) * p.max_ctx + pos) * HD + d0]) =
            __floats2bfloat162_rn(xv.x, xv.y);
      continue;
    }
    const bool is_q = head < nq;
    if (!is_q && !in_cache) continue;
    const __nv_bfloat16* nw = is_q ? qn : kn;
    float x0 = xv.x, x1 = xv.y;
    if (nw) {
      const float rs = scratch[b * HPT + hl];
      const __nv_bfloat162 w2 = *reinterpret_cast<const __nv_bfloat162*>(nw + d0);
      x0 = (x0 * rs) * __low2float(w2);
      x1 = (x1 * rs) * __high2float(w2);
    }
    // interleaved RoPE (model.py:184-196): (x0, x1) -> (x0 c - x1 s, x1 c + x0 s)
    const float2 cs = *reinterpret_cast<const float2*>(
        ec.angles ? ec.angles + (size_t)b * HD + d0 : p.angles + (size_t)(in_cache ? pos : 0) * HD + d0);
    const __nv_bfloat162 o = __floats2bfloat162_rn(x0 * cs.x - x1 * cs.y, x1 * cs.x + x0 * cs.y);
    if (is_q)
      *reinterpret_cast<__nv_bfloat162*>(&q_out[(size_t)m * p.y_ld + head * HD + d0]) = o;
    else
      *reinterpret_cast<__nv_bfloat162*>(&p.k_cache[(((size_t)m * nkv + (head - nq)) * p.max_ctx + pos) * HD + d0]) =
          o;
  }
}

// ---------------------------------------------------------------------------
// Epilogues over a finished [MB][128] fp32 tile (rows tile*128.., batch rows
// m0..m0+MB-1).  `scratch` holds >= 2*MB floats.  256 threads.
// ---------------------------------------------------------------------------
template <int EPI>
T2B_DEV void tile_epilogue(const LinearParams& p, const float* tile_acc, float* scratch, int tile, int m0, int MB,
                           const EpiCache& ec = EpiCache{}) {
  constexpr int NT = 256;
  const int lane = threadIdx.x & 31;
  const int row0 = tile * TILE_N;
  if (EPI == EPI_STORE) {
    for (int idx = threadIdx.x; idx < MB * TILE_N; idx += NT) {
      const int b = idx / TILE_N, lr = idx - b * TILE_N, m = m0 + b;
      if (m < p.M) store_act(p.y, p.y_dtype, (size_t)m * p.y_ld + row0 + lr, tile_acc[idx]);
    }
  } else if (EPI == EPI_RESIDUAL) {
    // x += y ; sum of squares for the next RMSNorm ; bf16(x * w_next) for its GEMM.
    // Each warp's 32 elements share one batch row -> one atomic per warp per pass.
    for (int base = 0; base < MB * TILE_N; base += NT) {
      const int idx = base + threadIdx.x;
      const int b = idx / TILE_N, lr = idx - b * TILE_N, m = m0 + b;
      const bool live = idx < MB * TILE_N && m < p.M;
      float sq = 0.f;
      if (live) {
        const size_t o = (size_t)m * p.y_ld + row0 + lr;
        const float v = (ec.resid ? ec.resid[idx] : p.resid[o]) + tile_acc[idx];
        p.resid[o] = v;
        sq = v * v;
        if (p.xw_out) {
          const float w = __bfloat162float(ec.next_w ? ec.next_w[lr] : p.next_w[row0 + lr]);
          p.xw_out[o] = __float2bfloat16_rn(v * w);
        }
      }
      sq = warp_sum(sq);
      if (lane == 0 && live) atomicAdd(p.ssq_out + m, sq);
    }
  } else if (EPI == EPI_SWIGLU) {
    // tile = 64 gate rows then the matching 64 up rows (model.py:215-216)
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.y);
    for (int idx = threadIdx.x; idx < MB * 64; idx += NT) {
      const int b = idx >> 6, t = idx & 63, m = m0 + b;
      if (m < p.M) {
        const float g = tile_acc[b * TILE_N + t];
        const float u = tile_acc[b * TILE_N + 64 + t];
        const float silu = g / (1.f + expf(-g));
        h[(size_t)m * p.y_ld + tile * 64 + t] = __float2bfloat16_rn(silu * u);
      }
    }
  } else {  // EPI_QKV
    if (p.head_dim == 128) qkv_epilogue<128>(p, tile_acc, scratch, tile, m0, MB, ec);
    else qkv_epilogue<64>(p, tile_acc, scratch, tile, m0, MB, ec);
  }
}

// Clears p.ssq_clear (M floats) from one designated CTA, after the PDL wait.
// Threads t = 0..nt-1 of the designated CTA zero the next producer's ssq buffer.
T2B_DEV void maybe_clear_ssq(const LinearParams& p, bool designated, int t, int nt) {
  if (p.ssq_clear != nullptr && designated)
    for (int i = t; i < p.M; i += nt) p.ssq_clear[i] = 0.f;
}

// Host side: shared launch helpers (defined in w4a16_gemv.cu).
int linear_launch(LinearParams& p, int pro, int epi, int wfmt, void* ws, size_t ws_bytes, cudaStream_t st);
size_t linear_workspace_bytes(int M, int N, int K);
void linear_workspace_layout(int M, int N, int K, size_t* partial_bytes, size_t* counter_bytes);

}  // namespace t2b
