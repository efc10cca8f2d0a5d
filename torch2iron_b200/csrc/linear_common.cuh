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
// Batch rows each CTA of the tcgen05 path finishes under the qkv epilogue, at
// most (where a plan of about one wave allows it): its per-row work -- QK-norm,
// RoPE, the KV-cache write -- then stays short beside the contraction.
constexpr int QKV_MAX_ROWS_PER_CTA = 8;

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
  __half* xw_out;               // EPI_RESIDUAL: fp16(resid * next_w) [M][y_ld] (nullable)
  float* ssq_clear;
  const __nv_bfloat16* qn_w;
  const __nv_bfloat16* kn_w;
  const float* angles;
  const int* pos;
  const int* row_seq;     // EPI_QKV: cache sequence of each row (nullptr: row m writes sequence m)
  int n_seq;              // EPI_QKV with row_seq: sequences in the cache (others write nothing)
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int n_heads, n_kv, head_dim, max_ctx;
  int* err;
  int q4nx;               // 1: Q4NX meta (bf16 scale | bf16 zero per 32-k piece), 0: T2B (per 128-k group)
  // EPI_STORE: the same output also stored into these buffers (tensor-parallel
  // partials pushed into the peers' memory; same layout as y)
  void* y_peer[7];
  int n_y_peer;
};

T2B_DEV size_t qw_block_offset(int nt, int g, int G) { return ((size_t)nt * G + g) * BLOCK_BYTES; }
T2B_DEV size_t meta_block_offset(int nt, int g, int G) { return ((size_t)nt * G + g) * TILE_N; }
// Q4NX meta: 4 pieces x 128 rows per block, piece-major
constexpr int Q4NX_META_WORDS = 4 * TILE_N;
T2B_DEV size_t meta_q4nx_offset(int nt, int g, int G) { return ((size_t)nt * G + g) * Q4NX_META_WORDS; }
// One 16-byte piece of a T2B (group-128) weight as 16 bf16x2 / fp16x2 words:
// the mask-or builds the pair (k, k+1) as 128+q (bf16) or 1024+q (fp16)
// exactly, the subtraction of the equally biased zero point is exact, and
// the multiplication by the group scale rounds once.  z2 = biased zero, s2 =
// scale (bf16: the fp16 scale rounded; fp16: exact).
template <bool F16>
T2B_DEV void dequant_piece_t2b(const uint4 v, uint32_t z2, uint32_t s2, uint32_t cols[16]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t m = (w[j] >> (4 * t)) & 0x000F000Fu;
      if (F16) {
        const uint32_t b = m | 0x64006400u;
        const __half2 d = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&b), *reinterpret_cast<const __half2*>(&z2)),
                                  *reinterpret_cast<const __half2*>(&s2));
        cols[4 * j + t] = *reinterpret_cast<const uint32_t*>(&d);
      } else {
        const uint32_t b = m | 0x43004300u;
        const __nv_bfloat162 d = __hmul2(__hsub2(*reinterpret_cast<const __nv_bfloat162*>(&b),
                                                 *reinterpret_cast<const __nv_bfloat162*>(&z2)),
                                         *reinterpret_cast<const __nv_bfloat162*>(&s2));
        cols[4 * j + t] = *reinterpret_cast<const uint32_t*>(&d);
      }
    }
}

// (biased zero, scale) pairs of a T2B meta word for dequant_piece_t2b.
template <bool F16>
T2B_DEV void t2b_meta_pairs(uint32_t mw, uint32_t& z2, uint32_t& s2) {
  const unsigned short sh = (unsigned short)(mw & 0xffffu);
  const float z = (float)((mw >> 16) & 0x1fu);
  if (F16) {
    const __half zb = __float2half_rn(1024.f + z), sb = __ushort_as_half(sh);
    const __half2 z = __halves2half2(zb, zb), s = __halves2half2(sb, sb);
    z2 = *reinterpret_cast<const uint32_t*>(&z);
    s2 = *reinterpret_cast<const uint32_t*>(&s);
  } else {
    const __nv_bfloat16 zb = __float2bfloat16_rn(128.f + z), sb = __float2bfloat16_rn(__half2float(__ushort_as_half(sh)));
    const __nv_bfloat162 z = __halves2bfloat162(zb, zb), s = __halves2bfloat162(sb, sb);
    z2 = *reinterpret_cast<const uint32_t*>(&z);
    s2 = *reinterpret_cast<const uint32_t*>(&s);
  }
}

// Meta words of one (tile, group) block in either format.
T2B_DEV int meta_block_words(bool q4nx) { return q4nx ? Q4NX_META_WORDS : TILE_N; }

T2B_DEV float bf16_lo_f32(uint32_t w) { return __uint_as_float(w << 16); }
T2B_DEV float bf16_hi_f32(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// One 16-byte piece (32 k of one row, T2B nibble order) of a Q4NX weight as
// 16 bf16x2 or fp16x2 words (k pairs in order): (q - zero) * scale in fp32, as
// the reference computes it (q4nx_layout.py:132-146), rounded once.
// 0x43000000 | q << 16 is the fp32 value 128 + q.
template <bool F16>
T2B_DEV void dequant_piece_q4nx(const uint4 v, float s, float z, uint32_t cols[16]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t m = (w[j] >> (4 * t)) & 0x000F000Fu;
      const float q0 = __uint_as_float(0x43000000u | (m << 16)) - 128.f;
      const float q1 = __uint_as_float(0x43000000u | (m & 0xffff0000u)) - 128.f;
      const float d0 = __fmul_rn(__fsub_rn(q0, z), s), d1 = __fmul_rn(__fsub_rn(q1, z), s);
      if (F16) {
        const __half2 d = __floats2half2_rn(d0, d1);
        cols[4 * j + t] = *reinterpret_cast<const uint32_t*>(&d);
      } else {
        const __nv_bfloat162 d = __floats2bfloat162_rn(d0, d1);
        cols[4 * j + t] = *reinterpret_cast<const uint32_t*>(&d);
      }
    }
}

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
// cache at the row's position.  A warp owns one batch row of the tile per
// pass, lane = 4 consecutive dims (float4 in, 8-byte bf16 store out): a head
// is 32 lanes (HD 128) or 16 (HD 64), so its sum of squares is a warp
// reduction in the same pass.  q_out, the caches and the angle table are
// 16-byte aligned, the norm weights 8-byte (checked at the C ABI).
// ---------------------------------------------------------------------------
T2B_DEV uint2 pack_bf16x4(float a, float b, float c, float d) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}
T2B_DEV float4 unpack_bf16x4(uint2 v) {
  return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                     __uint_as_float(v.y & 0xffff0000u));
}
T2B_DEV uint2 pack_f16x4(float a, float b, float c, float d) { return make_uint2(f16x2_sat(a, b), f16x2_sat(c, d)); }

template <int HD>
T2B_DEV void qkv_epilogue(const LinearParams& p, const float* tile_acc, int tile, int m0, int MB, const EpiCache& ec,
                          int t, int nt) {
  constexpr int HPT = TILE_N / HD;    // heads per tile
  constexpr int LPH = HD / 4;         // lanes per head
  const int warp = t >> 5, lane = t & 31, nwarps = nt >> 5;
  const int hl = lane / LPH, d0 = (lane % LPH) * 4;
  const int head = tile * HPT + hl;
  const int nq = p.n_heads, nkv = p.n_kv;
  const bool is_q = head < nq, is_v = head >= nq + nkv;
  const __nv_bfloat16* nw = is_q ? (ec.qn ? ec.qn : p.qn_w) : (ec.kn ? ec.kn : p.kn_w);
  if (is_v) nw = nullptr;
  const float4 w = nw ? unpack_bf16x4(*reinterpret_cast<const uint2*>(nw + d0)) : make_float4(1.f, 1.f, 1.f, 1.f);
  __nv_bfloat16* q_out = reinterpret_cast<__nv_bfloat16*>(p.y);
  for (int b = warp; b < MB; b += nwarps) {
    const int m = m0 + b;
    if (m >= p.M) break;  // warp-uniform
    const float4 x = *reinterpret_cast<const float4*>(tile_acc + b * TILE_N + lane * 4);
    float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
#pragma unroll
    for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int pos = ec.pos ? ec.pos[b] : p.pos[m];
    const int sq = p.row_seq ? __ldg(p.row_seq + m) : m;   // cache sequence of row m
    // a bad position or sequence writes no cache entry
    const bool pos_ok = pos >= 0 && pos < p.max_ctx;
    const bool in_cache = pos_ok && (!p.row_seq || (sq >= 0 && sq < p.n_seq));
    const size_t cm = (size_t)sq;
    if (is_v) {  // value head: stored as projected (model.py:250,263)
      if (in_cache)
        *reinterpret_cast<uint2*>(&p.v_cache[((cm * nkv + (head - nq - nkv)) * p.max_ctx + pos) * HD + d0]) =
            pack_bf16x4(x.x, x.y, x.z, x.w);
      continue;
    }
    if (!is_q && !in_cache) continue;
    const float rs = nw ? rsqrtf(ss / (float)HD + p.eps) : 1.f;   // model.py:179-180 on the head
    const float x0 = x.x * rs * w.x, x1 = x.y * rs * w.y, x2 = x.z * rs * w.z, x3 = x.w * rs * w.w;
    // interleaved RoPE (model.py:184-196): (x0, x1) -> (x0 c - x1 s, x1 c + x0 s)
    const float4 cs = *reinterpret_cast<const float4*>(
        ec.angles ? ec.angles + (size_t)b * HD + d0 : p.angles + (size_t)(pos_ok ? pos : 0) * HD + d0);
    const uint2 o = pack_bf16x4(x0 * cs.x - x1 * cs.y, x1 * cs.x + x0 * cs.y, x2 * cs.z - x3 * cs.w,
                                x3 * cs.z + x2 * cs.w);
    if (is_q && p.y_dtype == T2B_DTYPE_F32)   // fp32 q for the attention's two-term score MMAs
      *reinterpret_cast<float4*>(static_cast<float*>(p.y) + (size_t)m * p.y_ld + head * HD + d0) =
          make_float4(x0 * cs.x - x1 * cs.y, x1 * cs.x + x0 * cs.y, x2 * cs.z - x3 * cs.w, x3 * cs.z + x2 * cs.w);
    else if (is_q)
      *reinterpret_cast<uint2*>(&q_out[(size_t)m * p.y_ld + head * HD + d0]) = o;
    else
      *reinterpret_cast<uint2*>(&p.k_cache[((cm * nkv + (head - nq)) * p.max_ctx + pos) * HD + d0]) = o;
  }
}

// ---------------------------------------------------------------------------
// Epilogues over a finished [MB][128] fp32 tile (rows tile*128.., batch rows
// m0..m0+MB-1).  `scratch` holds >= 2*MB floats.  256 threads; each thread
// takes 4 consecutive outputs (the residual stream and h are 16- / 8-byte
// aligned with row strides of multiples of 4, checked at the C ABI).
// ---------------------------------------------------------------------------
// Threads t = 0..nt-1 (whole warps; default: the CTA's 256 threads) share the work.
template <int EPI>
T2B_DEV void tile_epilogue(const LinearParams& p, const float* tile_acc, float* scratch, int tile, int m0, int MB,
                           const EpiCache& ec = EpiCache{}, int t = -1, int nt = 256) {
  if (t < 0) t = threadIdx.x;
  const int NT = nt;
  const int lane = t & 31;
  const int row0 = tile * TILE_N;
  if (EPI == EPI_STORE) {
    if (p.n_y_peer) {
      // tensor-parallel push: the tile into this rank's buffer and every peer's,
      // four outputs per store and the same bits everywhere (bf16 or fp32)
      for (int idx = t * 4; idx < MB * TILE_N; idx += NT * 4) {
        const int b = idx / TILE_N, lr = idx - b * TILE_N, m = m0 + b;
        if (m >= p.M) continue;
        const float4 v = *reinterpret_cast<const float4*>(tile_acc + idx);
        const size_t o = (size_t)m * p.y_ld + row0 + lr;
        if (p.y_dtype == T2B_DTYPE_F32) {
          *reinterpret_cast<float4*>(static_cast<float*>(p.y) + o) = v;
          for (int q = 0; q < p.n_y_peer; ++q) *reinterpret_cast<float4*>(static_cast<float*>(p.y_peer[q]) + o) = v;
        } else {
          const uint2 w = pack_bf16x4(v.x, v.y, v.z, v.w);
          *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.y) + o) = w;
          for (int q = 0; q < p.n_y_peer; ++q)
            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.y_peer[q]) + o) = w;
        }
      }
    } else {
      for (int idx = t; idx < MB * TILE_N; idx += NT) {
        const int b = idx / TILE_N, lr = idx - b * TILE_N, m = m0 + b;
        if (m < p.M) store_act(p.y, p.y_dtype, (size_t)m * p.y_ld + row0 + lr, tile_acc[idx]);
      }
    }
  } else if (EPI == EPI_RESIDUAL) {
    // x += y ; sum of squares for the next RMSNorm ; bf16(x * w_next) for its GEMM.
    // A warp's 128 elements are one batch row of the tile -> one atomic per warp per pass.
    for (int base = 0; base < MB * TILE_N; base += NT * 4) {
      const int idx = base + t * 4;
      const int b = idx / TILE_N, lr = idx - b * TILE_N, m = m0 + b;
      const bool live = idx < MB * TILE_N && m < p.M;
      float sq = 0.f;
      if (live) {
        const size_t o = (size_t)m * p.y_ld + row0 + lr;
        const float4 r = *reinterpret_cast<const float4*>(ec.resid ? ec.resid + idx : p.resid + o);
        const float4 t = *reinterpret_cast<const float4*>(tile_acc + idx);
        const float4 v = make_float4(r.x + t.x, r.y + t.y, r.z + t.z, r.w + t.w);
        *reinterpret_cast<float4*>(p.resid + o) = v;
        sq = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        if (p.xw_out) {
          const float4 w = unpack_bf16x4(
              *reinterpret_cast<const uint2*>(ec.next_w ? ec.next_w + lr : p.next_w + row0 + lr));
          *reinterpret_cast<uint2*>(p.xw_out + o) = pack_f16x4(v.x * w.x, v.y * w.y, v.z * w.z, v.w * w.w);
        }
      }
      sq = warp_sum(sq);
      if (lane == 0 && live) atomicAdd(p.ssq_out + m, sq);
    }
  } else if (EPI == EPI_SWIGLU) {
    // tile = 64 gate rows then the matching 64 up rows (model.py:215-216); h is fp16
    __half* h = reinterpret_cast<__half*>(p.y);
    for (int idx = t * 4; idx < MB * 64; idx += NT * 4) {
      const int b = idx >> 6, t = idx & 63, m = m0 + b;
      if (m < p.M) {
        const float4 g = *reinterpret_cast<const float4*>(tile_acc + b * TILE_N + t);
        const float4 u = *reinterpret_cast<const float4*>(tile_acc + b * TILE_N + 64 + t);
        *reinterpret_cast<uint2*>(&h[(size_t)m * p.y_ld + tile * 64 + t]) =
            pack_f16x4(g.x / (1.f + expf(-g.x)) * u.x, g.y / (1.f + expf(-g.y)) * u.y,
                       g.z / (1.f + expf(-g.z)) * u.z, g.w / (1.f + expf(-g.w)) * u.w);
      }
    }
  } else {  // EPI_QKV
    if (p.head_dim == 128) qkv_epilogue<128>(p, tile_acc, tile, m0, MB, ec, t, nt);
    else qkv_epilogue<64>(p, tile_acc, tile, m0, MB, ec, t, nt);
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
// Plain GEMM entry split into host checks and launch (w4a16_gemv.cu).
int gemm_params(const void* weight, const uint32_t* meta, int wfmt, const void* x, int x_dtype, void* y,
                int y_dtype, int M, int N, int K, int group_size, LinearParams* out);
void gemm_path_workspace(const LinearParams& p, int wfmt, size_t* partial_bytes, size_t* counter_bytes);
int gemm_launch(LinearParams& p, int wfmt, void* ws, size_t ws_bytes, cudaStream_t st);

}  // namespace t2b
