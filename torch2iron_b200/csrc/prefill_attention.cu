// Causal GQA attention for one prefill chunk over the bf16 KV cache.
//
// A chunk is C consecutive prompt tokens (absolute positions p0 .. p0+C-1) of
// each of B sequences; their K/V rows are already in the cache (written by
// the chunk's qkv kernel, earlier chunks by earlier calls).  Token i attends
// keys 0 .. p0+i of its own sequence, the causal rule the reference's chunked
// prefill applies per chunk (prefill_runtime.py:95-164,
// llama_chunked_prefill_attention/op.py:21-50) and the math of model.py:266-279.
//
// Work: one CTA = 64 query rows = 64/qpg tokens x the qpg q heads of one kv
// head g of one sequence b (so each K/V tile is read once for the whole GQA
// group), grid (ceil(C / (64/qpg)), n_kv, B).  Four warps, 16 query rows each.
//
// Data movement: Q and 64-key K/V tiles arrive by 16-byte cp.async into a
// double-buffered shared-memory ring; rows are stored with an XOR swizzle of
// their 16-byte chunks (chunk ^ (row & 7)) so the ldmatrix reads below hit 8
// distinct bank groups.  Keys past the CTA's last needed key are zero-filled.
//
// Math (mma.sync m16n8k16, bf16 operands, fp32 accumulation), flash-attention
// style per warp: S = Q K^T (16 rows x 64 keys), causal mask, online softmax
// in the log2 domain (running max and sum per row), P rounded to bf16 and
// reused in registers as the A operand of O += P V (V through ldmatrix.trans).
// No wait in this kernel spins on a flag: cp.async groups complete on their own.

#include <math.h>

#include "t2b_common.cuh"
#include "launch.cuh"
#include "mma_sync.cuh"

namespace t2b {

constexpr int PF_THREADS = 128;  // 4 warps x 16 query rows
constexpr int PF_ROWS = 64;      // query rows (token, head) per CTA
constexpr int PF_KEYS = 64;      // keys per tile

struct PrefillParams {
  const __nv_bfloat16* q;  // [B*C][n_heads*HD], row b*C + i
  const __nv_bfloat16* k;  // [B][n_kv][max_ctx][HD]
  const __nv_bfloat16* v;
  __nv_bfloat16* out;      // [B*C][n_heads*HD], bf16 or (out_f16) fp16
  int out_f16;
  int C, p0, n_heads, n_kv, qpg, max_ctx;
  float scale_log2;        // log2(e) / sqrt(HD)
};

template <int HD>
struct PfSmem {
  static constexpr int ROW_BYTES = HD * 2;
  static constexpr int TILE_BYTES = PF_KEYS * ROW_BYTES;
  static constexpr int Q_BYTES = PF_ROWS * ROW_BYTES;
  static constexpr int BYTES = Q_BYTES + 4 * TILE_BYTES;  // q | K0 V0 | K1 V1
};

// Byte offset of 16-byte chunk c of row r in a swizzled [rows][HD] bf16 array.
template <int HD>
T2B_DEV uint32_t sw_off(int r, int c) {
  return (uint32_t)(r * (HD * 2) + ((c ^ (r & 7)) << 4));
}

T2B_DEV void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
T2B_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
T2B_DEV void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(PF_THREADS) prefill_attention_kernel(const PrefillParams P) {
  using S = PfSmem<HD>;
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t s_q = smem_u32(sm);
  const uint32_t s_kv = s_q + S::Q_BYTES;  // stage st: K at s_kv + 2*st*TILE, V one TILE later
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qpg = P.qpg, T = PF_ROWS / qpg;  // tokens per CTA
  const int t0 = blockIdx.x * T, g = blockIdx.y, b = blockIdx.z;
  const int t_last = min(t0 + T, P.C) - 1;
  const int n_keys = P.p0 + t_last + 1;  // keys the CTA's last token attends
  const int n_tiles = (n_keys + PF_KEYS - 1) / PF_KEYS;
  const size_t q_ld = (size_t)P.n_heads * HD;
  const __nv_bfloat16* kb = P.k + ((size_t)b * P.n_kv + g) * P.max_ctx * HD;
  const __nv_bfloat16* vb = P.v + ((size_t)b * P.n_kv + g) * P.max_ctx * HD;

  grid_dep_wait();  // q and this chunk's K/V rows come from the preceding qkv kernel
  grid_dep_launch();

  // Q rows: r -> (token t0 + r / qpg, head g*qpg + r % qpg); rows past the chunk read zeros
  for (int i = threadIdx.x; i < PF_ROWS * CH; i += PF_THREADS) {
    const int r = i / CH, c = i - r * CH;
    const int tok = t0 + r / qpg;
    const bool ok = tok < P.C;
    const __nv_bfloat16* src =
        P.q + (size_t)(b * P.C + (ok ? tok : 0)) * q_ld + (size_t)(g * qpg + r % qpg) * HD + c * 8;
    cp_async16(s_q + sw_off<HD>(r, c), src, ok ? 16u : 0u);
  }
  auto load_tile = [&](int kt, int st) {
    const uint32_t dk = s_kv + (uint32_t)(st * 2 * S::TILE_BYTES), dv = dk + S::TILE_BYTES;
    for (int i = threadIdx.x; i < PF_KEYS * CH; i += PF_THREADS) {
      const int r = i / CH, c = i - r * CH;
      const int key = kt * PF_KEYS + r;
      const bool ok = key < n_keys;
      const size_t off = (size_t)(ok ? key : 0) * HD + c * 8;
      cp_async16(dk + sw_off<HD>(r, c), kb + off, ok ? 16u : 0u);
      cp_async16(dv + sw_off<HD>(r, c), vb + off, ok ? 16u : 0u);
    }
  };
  load_tile(0, 0);
  cp_async_commit();  // group: q + tile 0

  // this thread's two accumulator rows (C-fragment rows lane/4 and lane/4 + 8)
  const int ra = warp * 16 + (lane >> 2), rb = ra + 8;
  const int pos_a = P.p0 + t0 + ra / qpg, pos_b = P.p0 + t0 + rb / qpg;

  uint32_t qf[HD / 16][4];
  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

#pragma unroll 1
  for (int kt = 0; kt < n_tiles; ++kt) {
    if (kt + 1 < n_tiles) load_tile(kt + 1, (kt + 1) & 1);
    cp_async_commit();  // (empty on the last tile: the group count stays uniform)
    cp_async_wait_1();  // everything but the newest group has landed: tile kt (and q)
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks)
        ldsm_x4(qf[ks], s_q + sw_off<HD>(warp * 16 + (lane & 15), ks * 2 + (lane >> 4)));
    }
    const uint32_t sk = s_kv + (uint32_t)((kt & 1) * 2 * S::TILE_BYTES), sv = sk + S::TILE_BYTES;

    // ---- S = Q K^T: 8 n-tiles of 8 keys ----
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t kf[4];
        ldsm_x4(kf, sk + sw_off<HD>(np * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 2 + ((lane >> 3) & 1)));
        mma_bf16(s[2 * np], qf[ks], kf[0], kf[1]);
        mma_bf16(s[2 * np + 1], qf[ks], kf[2], kf[3]);
      }
    }

    // ---- causal mask + online softmax (log2 domain) ----
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k0 = kt * PF_KEYS + j * 8 + (lane & 3) * 2;
      s[j][0] = k0 <= pos_a ? s[j][0] * P.scale_log2 : -INFINITY;
      s[j][1] = k0 + 1 <= pos_a ? s[j][1] * P.scale_log2 : -INFINITY;
      s[j][2] = k0 <= pos_b ? s[j][2] * P.scale_log2 : -INFINITY;
      s[j][3] = k0 + 1 <= pos_b ? s[j][3] * P.scale_log2 : -INFINITY;
      mx_a = fmaxf(mx_a, fmaxf(s[j][0], s[j][1]));
      mx_b = fmaxf(mx_b, fmaxf(s[j][2], s[j][3]));
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    // key 0 is in every row's range, so the running max is finite from tile 0 on
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float ca = exp2f(m_a - mn_a), cb = exp2f(m_b - mn_b);
    m_a = mn_a;
    m_b = mn_b;
    uint32_t pf[4][4];  // P as the A operand: k-step j/2, registers (row a, row b) x (keys 0-7, 8-15)
    float ls_a = 0.f, ls_b = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float e0 = exp2f(s[j][0] - mn_a), e1 = exp2f(s[j][1] - mn_a);
      const float e2 = exp2f(s[j][2] - mn_b), e3 = exp2f(s[j][3] - mn_b);
      ls_a += e0 + e1;
      ls_b += e2 + e3;
      pf[j >> 1][(j & 1) * 2] = pack_bf16(e0, e1);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_bf16(e2, e3);
    }
    l_a = l_a * ca + ls_a;  // per-thread partial sums; the quad is summed at the end
    l_b = l_b * cb + ls_b;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      o[j][0] *= ca;
      o[j][1] *= ca;
      o[j][2] *= cb;
      o[j][3] *= cb;
    }

    // ---- O += P V ----
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t vf[4];
        ldsm_x4_t(vf, sv + sw_off<HD>(ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 2 + (lane >> 4)));
        mma_bf16(o[2 * dp], pf[ks], vf[0], vf[1]);
        mma_bf16(o[2 * dp + 1], pf[ks], vf[2], vf[3]);
      }
    }
    __syncthreads();  // the next iteration refills the other stage; this one is reused two tiles on
  }

  // ---- normalise and store ----
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float ia = 1.f / l_a, ib = 1.f / l_b;
  const int tok_a = t0 + ra / qpg, tok_b = t0 + rb / qpg;
  const int dc = (lane & 3) * 2;
  if (tok_a < P.C) {
    uint32_t* dst = reinterpret_cast<uint32_t*>(P.out + (size_t)(b * P.C + tok_a) * q_ld +
                                                (size_t)(g * qpg + ra % qpg) * HD + dc);
#pragma unroll
    for (int j = 0; j < HD / 8; ++j)
      dst[j * 4] = P.out_f16 ? f16x2_sat(o[j][0] * ia, o[j][1] * ia) : pack_bf16(o[j][0] * ia, o[j][1] * ia);
  }
  if (tok_b < P.C) {
    uint32_t* dst = reinterpret_cast<uint32_t*>(P.out + (size_t)(b * P.C + tok_b) * q_ld +
                                                (size_t)(g * qpg + rb % qpg) * HD + dc);
#pragma unroll
    for (int j = 0; j < HD / 8; ++j)
      dst[j * 4] = P.out_f16 ? f16x2_sat(o[j][2] * ib, o[j][3] * ib) : pack_bf16(o[j][2] * ib, o[j][3] * ib);
  }
}

}  // namespace t2b

using namespace t2b;

extern "C" int t2b_prefill_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                     uint16_t* out, int out_dtype, int B, int C, int p0, int n_heads, int n_kv,
                                     int head_dim, int max_ctx, void* stream) {
  if (!q || !k_cache || !v_cache || !out) return T2B_ERR_ARG;
  if (out_dtype != T2B_DTYPE_BF16 && out_dtype != T2B_DTYPE_F16) return T2B_ERR_ARG;
  if (head_dim != 64 && head_dim != 128) return T2B_ERR_SHAPE;
  if (B < 1 || B > 65535 || C < 1 || p0 < 0 || n_kv < 1 || n_kv > 65535 || n_heads % n_kv) return T2B_ERR_SHAPE;
  const int qpg = n_heads / n_kv;
  if (qpg > PF_ROWS || PF_ROWS % qpg) return T2B_ERR_SHAPE;
  if ((long long)p0 + C > max_ctx) return T2B_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return T2B_ERR_ALIGN;
  PrefillParams P{};
  P.q = reinterpret_cast<const __nv_bfloat16*>(q);
  P.k = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  P.v = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  P.out = reinterpret_cast<__nv_bfloat16*>(out);
  P.out_f16 = out_dtype == T2B_DTYPE_F16;
  P.C = C;
  P.p0 = p0;
  P.n_heads = n_heads;
  P.n_kv = n_kv;
  P.qpg = qpg;
  P.max_ctx = max_ctx;
  P.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  const int T = PF_ROWS / qpg;
  const dim3 grid((C + T - 1) / T, n_kv, B);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (head_dim == 128) {
    auto kern = prefill_attention_kernel<128>;
    if (allow_smem(kern, PfSmem<128>::BYTES) != T2B_OK) return T2B_ERR_LAUNCH;
    return launch_pdl(kern, grid, dim3(PF_THREADS), (size_t)PfSmem<128>::BYTES, st, P);
  }
  auto kern = prefill_attention_kernel<64>;
  if (allow_smem(kern, PfSmem<64>::BYTES) != T2B_OK) return T2B_ERR_LAUNCH;
  return launch_pdl(kern, grid, dim3(PF_THREADS), (size_t)PfSmem<64>::BYTES, st, P);
}
