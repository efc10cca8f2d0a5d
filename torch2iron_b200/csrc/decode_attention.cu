// GQA decode attention over a bf16 KV cache: persistent, tile-balanced,
// tensor-core tile math.
//
// Work: every (batch row m, kv head h) "unit" attends the qpg q heads of its
// GQA group (q[m, h*qpg .. +qpg], so each K/V byte is read once) over keys
// 0..pos[m], cut into 64-key tiles.  All tiles of all units form one list
// (row-major units); the grid (the CTAs resident at once) splits the list into
// equal contiguous ranges, so every CTA streams about the same number of KV
// bytes in a single wave whatever the context lengths.  A range boundary that
// falls inside a short unit moves to the nearer unit edge (short units are
// never cut, so short-context batches need no cross-CTA merge).  The
// after-kvwrite entry point builds the list and issues the loads of every
// tile older than a unit's newest key before the dependency wait.
//
// Data movement: K and V tiles arrive by 3-D TMA boxes (64 dims x 64 keys, or
// 64 dims x 16 keys for a tile that ends inside the context, so at most 15
// unused keys are read) in the 128-byte swizzled layout, which keeps the
// ldmatrix reads below free of bank conflicts.  The boxes land in a ring of
// shared-memory stages refilled ahead of use; completion is counted on
// mbarriers whose waits are time-bounded.
//
// Math (mma.sync m16n8k16, bf16 operands, fp32 accumulation), keys on the M
// side and the group's q heads on N (up to 8): warp w owns keys 16w..16w+15 of
// every tile and keeps its own online softmax for them (running max and sum
// per head, in the log2 domain; model.py:266-279, and the chunked update of
// llama_chunked_attention/kernel.cc:111-257):
//   S^T [16 keys x 8 heads]  = K_w . q^T                  HD/16 MMAs
//   P^T = 2^(S^T * log2(e)/sqrt(HD) - max), bf16, moved into the B-operand
//         layout in registers (movmatrix.trans)
//   O^T [HD x 8 heads]      += V_w^T . P^T                HD/16 MMAs
// At a unit's end the four warps' (o, max, sum) are combined in shared memory.
// A unit cut between CTAs leaves one normalised partial (o, max, sum) per CTA;
// after its last tile each CTA takes one ticket per cut unit, and the last
// CTA to arrive (ticket counter, re-armed) merges the unit's partials.
//
// The same kernel reads the reference's packet cache
// ([group][chunk][K 64*hd | V 64*hd | mask 64], decode_packet_cache.py:11-43):
// tile = chunk, and slots whose mask <= 0.5 are skipped
// (attention_reference.py:153-154).

#include <algorithm>
#include <cstdlib>
#include <math.h>

#include "t2b_common.cuh"
#include "launch.cuh"
#include "mma_sync.cuh"
#include "tmap.cuh"

namespace t2b {

constexpr int AT_THREADS = 128;
constexpr int AT_WARPS = AT_THREADS / 32;
constexpr int AT_TILE = 64;            // keys per ring stage
constexpr int AT_SUB = 16;             // keys per warp slice, and per box of a partial tile
constexpr int AT_MAX_CTAS_PER_SM = 4;  // workspace bound; the grid uses the measured occupancy
constexpr int AT_MAX_ROWS = 256;
constexpr int AT_MERGE_BATCH = 32;     // partial records weighed per pass of a cross-CTA merge

struct AttnParams {
  CUtensorMap kmap_full;  // box: 64 dims x 64 keys
  CUtensorMap vmap_full;
  CUtensorMap kmap_sub;   // box: 64 dims x 16 keys
  CUtensorMap vmap_sub;
  const void* q;               // [rows][n_heads*hd], bf16 or (q_f32) fp32
  int q_f32;
  const __nv_bfloat16* mask0;  // nullable (packet mode): mask of (unit u, tile j) at mask0 + u*mask_unit + j*mask_tile
  long long mask_unit, mask_tile;
  int tile_y, unit_z, tile_z;  // TMA coordinates of (unit u, tile j): y = j*tile_y, z = u*unit_z + j*tile_z
  const int* pos;              // nullable: keys = pos[m] + 1 (clamped to [1, n_keys]), else n_keys
  int n_keys;                  // packet mode: keys per unit; cache mode: max_ctx
  int rows;
  __nv_bfloat16* out;          // [rows][n_heads*hd], bf16 or (out_f16) fp16
  int out_f16;
  int n_heads, n_kv;
  float scale_log2;            // log2(e) / sqrt(hd)
  float* ws;                   // partial records [grid][2][qpg][hd + 2]
  int* cnt;                    // [rows][n_kv] tickets
  int* err;
  int kv_early;                // 1: pos and every tile but a unit's last may be read before the
                               // dependency wait (the preceding kernel writes only q and key pos[m])
};

template <int HD, int ST>
struct AtGeom {
  static constexpr int HALVES = HD / 64;                 // 128-byte swizzle spans per key row
  static constexpr int STAGES = ST;
  static constexpr int HALF_BYTES = AT_TILE * 128;       // 64 keys x 64 dims
  static constexpr int KV_BYTES = HALVES * HALF_BYTES;   // K (or V) of one tile
  static constexpr int STAGE_BYTES = 2 * KV_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
};

template <int HD, int QPG, int ST>
struct AttnAux {
  static constexpr int STAGES = ST;
  float qb[STAGES][QPG * HD];          // q heads of a unit (fp32, or bf16 in the first half), copied with the unit's first tile
  __nv_bfloat16 msk[STAGES][AT_TILE];
  float ow[AT_WARPS][QPG][HD];         // per-warp (o, max, sum) at a unit's end
  float mw[AT_WARPS][QPG];
  float lw[AT_WARPS][QPG];
  float wpart[AT_MERGE_BATCH][QPG];    // cross-CTA merge weights
  float mh[QPG], dh[QPG];
  int row_start[AT_MAX_ROWS + 1];      // first global tile index of row m (all its kv heads)
  int row_tiles[AT_MAX_ROWS];          // tiles per unit of row m
  int row_keys[AT_MAX_ROWS];           // keys attended by row m
  int flag;
  uint64_t bar[STAGES];
};

template <int HD, int QPG, int ST>
constexpr size_t attn_smem_bytes() {
  return 1024 + AtGeom<HD, ST>::RING_BYTES + sizeof(AttnAux<HD, QPG, ST>);
}

struct TileRef {
  int m, h, j, nt;  // unit (m, h), tile j of nt
};

// Keys attended by row m: pos[m] + 1, kept inside the cache whatever pos holds.
// (Read through L2: with kv_early it is read while the preceding kernel runs.)
T2B_DEV int keys_of_row_global(const AttnParams& P, int m) {
  if (!P.pos) return P.n_keys;
  const int k = __ldcg(P.pos + m) + 1;
  return k < 1 ? 1 : (k > P.n_keys ? P.n_keys : k);
}

// Two adjacent outputs (element i even): bf16, or fp16 for the fused layer's o_proj input.
T2B_DEV void store_out_pair(const AttnParams& P, size_t i, float a, float b) {
  if (P.out_f16) {
    *reinterpret_cast<uint32_t*>(reinterpret_cast<__half*>(P.out) + i) = f16x2_sat(a, b);
  } else {
    *reinterpret_cast<__nv_bfloat162*>(&P.out[i]) = __floats2bfloat162_rn(a, b);
  }
}

template <class Aux>
T2B_DEV TileRef locate(const Aux& S, int rows, int t) {
  int lo = 0, hi = rows - 1;  // last row with row_start <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (S.row_start[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  TileRef r;
  r.m = lo;
  r.nt = S.row_tiles[lo];
  const int off = t - S.row_start[lo];
  r.h = off / r.nt;
  r.j = off - r.h * r.nt;
  return r;
}

// Next tile of the list (call only while one remains).
template <class Aux>
T2B_DEV void next_tile(TileRef& r, const Aux& S, int n_kv) {
  if (++r.j < r.nt) return;
  r.j = 0;
  if (++r.h < n_kv) return;
  r.h = 0;
  ++r.m;
  r.nt = S.row_tiles[r.m];
}

// Even split of T tiles over NP CTAs, and the CTA holding tile t under it.
T2B_DEV int range_lo(long long c, long long T, long long NP) { return (int)(c * T / NP); }
T2B_DEV int cta_of_tile(long long t, long long T, long long NP) { return (int)(((t + 1) * NP + T - 1) / T - 1); }

// First tile of CTA c's range: the even split c*T/NP, moved to the nearer
// end of its unit when that unit is short (at most snap_max tiles), so a
// short unit is never cut between CTAs (a range may then be empty).  Only
// units longer than snap_max are cut, and only at even-split points, so the
// CTAs holding the first and last tile of such a unit are cta_of_tile() of
// those tiles.
template <class Aux>
T2B_DEV int range_start(const Aux& S, int rows, long long c, long long T, long long NP, int snap_max) {
  if (c <= 0) return 0;
  if (c >= NP) return (int)T;
  const int b = range_lo(c, T, NP);
  const TileRef r = locate(S, rows, b);
  if (r.j == 0 || r.nt > snap_max) return b;
  return 2 * r.j <= r.nt ? b - r.j : b - r.j + r.nt;
}

// A unit cut between CTAs c1..c2 (its tiles t0 .. t0+nt-1).
struct SplitUnit {
  int m, h, t0, c1, c2;
};

template <int HD, int QPG, int ST>
__global__ void __launch_bounds__(AT_THREADS) decode_attention_kernel(const __grid_constant__ AttnParams P) {
  using G = AtGeom<HD, ST>;
  using Aux = AttnAux<HD, QPG, ST>;
  constexpr int STAGES = G::STAGES;
  constexpr int NT16 = HD / 16;  // k-steps of K.q^T, and 16-dim m-tiles of O^T
  constexpr int REC = HD + 2;
  constexpr int NPAIR = QPG * HD / 2;
  constexpr int EPT = (NPAIR + AT_THREADS - 1) / AT_THREADS;
  static_assert(QPG >= 1 && QPG <= 8, "q heads per kv head: 1..8");
  extern __shared__ unsigned char smem_raw[];
  unsigned char* ring =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Aux& S = *reinterpret_cast<Aux*>(ring + G::RING_BYTES);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int c = blockIdx.x;
  T2B_TRACE_BEGIN(10, P.n_heads);

  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) mbar_init(&S.bar[i], 1);
    fence_mbar_init();
  }
  // With kv_early the tile list is built and the loads of tiles older than
  // the newest key are issued while the preceding kernel still runs.
  if (!P.kv_early) {
    grid_dep_wait();
    grid_dep_launch();
    T2B_TRACE_MARK(1);
  }

  // ---- tile list: tiles per unit of each row, exclusive prefix over rows ----
  const int rows = P.rows;
  for (int m = tid; m < rows; m += AT_THREADS) {
    const int nk = keys_of_row_global(P, m);
    S.row_keys[m] = nk;
    S.row_tiles[m] = (nk + AT_TILE - 1) / AT_TILE;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < rows; base += 32) {
      const int m = base + lane;
      const int v = (m < rows) ? S.row_tiles[m] * P.n_kv : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (m < rows) S.row_start[m] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) S.row_start[rows] = carry;
  }
  __syncthreads();
  const long long T = S.row_start[rows];
  const long long NP = T < (long long)gridDim.x ? T : (long long)gridDim.x;
  const int snap_max = max(STAGES, (int)((3 * T) / (5 * NP)));
  const int t_lo = c < NP ? range_start(S, rows, c, T, NP, snap_max) : 0;
  const int count = c < NP ? range_start(S, rows, c + 1, T, NP, snap_max) - t_lo : 0;
  if (count <= 0) {
    if (P.kv_early) grid_dep_launch();
    return;
  }

  // Tile `r` (the i-th of this CTA) goes to stage i % STAGES, with q on a
  // unit's first tile here: arm(), then load_kv() and load_q() (the last
  // tile of a unit holds the key the preceding kernel writes).
  auto tile_keys = [&](const TileRef& r) { return min(AT_TILE, S.row_keys[r.m] - r.j * AT_TILE); };
  auto with_q = [&](int i, const TileRef& r) { return (i == 0) || (r.j == 0); };
  auto arm = [&](int i, const TileRef& r) {
    const int nk = tile_keys(r);
    const bool full = nk == AT_TILE;
    const uint32_t kv = full ? (uint32_t)G::KV_BYTES : (uint32_t)(G::HALVES * ((nk + AT_SUB - 1) / AT_SUB) * AT_SUB * 128);
    const uint32_t qbytes = with_q(i, r) ? (uint32_t)(QPG * HD * (P.q_f32 ? 4 : 2)) : 0u;
    const uint32_t mbytes = P.mask0 ? (uint32_t)(AT_TILE * 2) : 0u;
    mbar_arrive_expect_tx(&S.bar[i % STAGES], 2u * kv + qbytes + mbytes);
  };
  auto load_kv = [&](int i, const TileRef& r) {
    const int nk = tile_keys(r);
    const int st = i % STAGES;
    const bool full = nk == AT_TILE;
    const int nbox = full ? 1 : (nk + AT_SUB - 1) / AT_SUB;
    const int u = r.m * P.n_kv + r.h;
    const int y0 = r.j * P.tile_y;
    const int z = u * P.unit_z + r.j * P.tile_z;
    unsigned char* kdst = ring + st * G::STAGE_BYTES;
    unsigned char* vdst = kdst + G::KV_BYTES;
    const void* km = full ? (const void*)&P.kmap_full : (const void*)&P.kmap_sub;
    const void* vm = full ? (const void*)&P.vmap_full : (const void*)&P.vmap_sub;
    for (int hf = 0; hf < G::HALVES; ++hf)
      for (int b = 0; b < nbox; ++b) {
        const int off = hf * G::HALF_BYTES + b * AT_SUB * 128;
        tma_load_3d(kdst + off, km, hf * 64, y0 + b * AT_SUB, z, &S.bar[st]);
        tma_load_3d(vdst + off, vm, hf * 64, y0 + b * AT_SUB, z, &S.bar[st]);
      }
    if (P.mask0)
      bulk_g2s(&S.msk[st][0], P.mask0 + u * P.mask_unit + r.j * P.mask_tile, (uint32_t)(AT_TILE * 2), &S.bar[st]);
  };
  auto load_q = [&](int i, const TileRef& r) {
    if (with_q(i, r))
      bulk_g2s(&S.qb[i % STAGES][0],
               static_cast<const unsigned char*>(P.q) +
                   ((size_t)r.m * P.n_heads * HD + (size_t)r.h * QPG * HD) * (P.q_f32 ? 4 : 2),
               (uint32_t)(QPG * HD * (P.q_f32 ? 4 : 2)), &S.bar[i % STAGES]);
  };
  TileRef cur = locate(S, rows, t_lo);  // consumer position
  TileRef pro = cur;                    // producer position (thread 0)
  int issued = 0;
  const int first = min(STAGES, count);
  if (P.kv_early) {
    if (tid == 0)
      for (int i = 0; i < first; ++i) {
        arm(i, pro);
        if (pro.j < pro.nt - 1) load_kv(i, pro);
        if (i + 1 < first) next_tile(pro, S, P.n_kv);
      }
    grid_dep_wait();
    grid_dep_launch();
    T2B_TRACE_MARK(1);
    pro = cur;
    if (tid == 0)
      for (int i = 0; i < first; ++i) {
        if (pro.j == pro.nt - 1) load_kv(i, pro);
        load_q(i, pro);
        if (i + 1 < count) next_tile(pro, S, P.n_kv);
      }
  } else if (tid == 0) {
    for (int i = 0; i < first; ++i) {
      arm(i, pro);
      load_kv(i, pro);
      load_q(i, pro);
      if (i + 1 < count) next_tile(pro, S, P.n_kv);
    }
  }
  issued = first;

  const int kb = AT_SUB * warp;  // this warp's first key in a tile
  const int h0 = 2 * t4, h1 = h0 + 1;
  float o[NT16][4];
  uint32_t qf[NT16][2];   // q^T fragments: bf16(q) ...
  uint32_t ql[NT16][2];   // ... and, for fp32 q, bf16(q - bf16(q)): the two terms carry 16 significant bits
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads h0, h1 (log2 domain)
  SplitUnit split[2];  // units of this range cut between CTAs: ticketed after the last tile
  int n_split = 0;

  for (int i = 0; i < count; ++i) {
    if (i > 0) next_tile(cur, S, P.n_kv);
    const TileRef r = cur;
    const bool unit_begin = (i == 0) || (r.j == 0);
    const bool unit_end = (i == count - 1) || (r.j == r.nt - 1);
    const int st = i % STAGES;
    // every thread takes the same outcome, so no thread is left at a barrier
    const bool ok = __syncthreads_and(mbar_wait_bounded(&S.bar[st], (i / STAGES) & 1, P.err));
    if (!ok) return;  // timeout recorded in P.err; no ticket is taken, so no CTA merges
    if (i == 0) T2B_TRACE_MARK(2);
    if (i == count - 1) T2B_TRACE_MARK(3);
    if (unit_begin) {  // new unit: B operand q^T (heads >= QPG are zero columns), fresh softmax state
      if (P.q_f32) {
        const float* qs = &S.qb[st][0];
#pragma unroll
        for (int ks = 0; ks < NT16; ++ks) {
          float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
          if (g < QPG) {
            a = *reinterpret_cast<const float2*>(qs + g * HD + ks * 16 + 2 * t4);
            b = *reinterpret_cast<const float2*>(qs + g * HD + ks * 16 + 2 * t4 + 8);
          }
          split_bf16(a.x, a.y, qf[ks][0], ql[ks][0]);
          split_bf16(b.x, b.y, qf[ks][1], ql[ks][1]);
        }
      } else {
        const __nv_bfloat16* qs = reinterpret_cast<const __nv_bfloat16*>(&S.qb[st][0]);
#pragma unroll
        for (int ks = 0; ks < NT16; ++ks) {
          qf[ks][0] = g < QPG ? *reinterpret_cast<const uint32_t*>(qs + g * HD + ks * 16 + 2 * t4) : 0u;
          qf[ks][1] = g < QPG ? *reinterpret_cast<const uint32_t*>(qs + g * HD + ks * 16 + 2 * t4 + 8) : 0u;
          ql[ks][0] = ql[ks][1] = 0u;
        }
      }
#pragma unroll
      for (int mt = 0; mt < NT16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }
    const int nk = min(AT_TILE, S.row_keys[r.m] - r.j * AT_TILE);
    if (kb < nk) {  // warp-uniform
      unsigned char* kst = ring + st * G::STAGE_BYTES;
      unsigned char* vst = kst + G::KV_BYTES;
      if (nk < kb + AT_SUB) {
        // keys past the context in this slice: their P is 0, but 0 * (stale
        // V) must not turn into NaN, so the rows are cleared
        const int nz = (kb + AT_SUB - nk) * G::HALVES * 8;
        for (int e = lane; e < nz; e += 32) {
          const int row = nk + e / (G::HALVES * 8), cc = e % (G::HALVES * 8);
          *reinterpret_cast<uint4*>(vst + (cc >> 3) * G::HALF_BYTES + row * 128 + (cc & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }
      // S^T = K_w . q^T, two accumulation chains
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
      const int krow = kb + (lane & 7) + ((lane >> 3) & 1) * 8;
      const uint32_t kaddr = smem_u32(kst) + krow * 128;
#pragma unroll
      for (int ks = 0; ks < NT16; ++ks) {
        const int ch = (ks & 3) * 2 + (lane >> 4);
        uint32_t a[4];
        ldsm_x4(a, kaddr + (ks >> 2) * G::HALF_BYTES + ((ch ^ (krow & 7)) << 4));
        if (P.q_f32) {   // the low terms of q in the second chain (warp-uniform branch)
          mma_bf16(sa, a, qf[ks][0], qf[ks][1]);
          mma_bf16(sb, a, ql[ks][0], ql[ks][1]);
        } else {
          mma_bf16((ks & 1) ? sb : sa, a, qf[ks][0], qf[ks][1]);
        }
      }
      // online softmax over this warp's 16 keys (rows g, g+8; heads h0, h1)
      const int k0 = kb + g, k1 = k0 + 8;
      bool live0 = k0 < nk, live1 = k1 < nk;
      if (P.mask0) {
        live0 = live0 && __bfloat162float(S.msk[st][k0]) > 0.5f;
        live1 = live1 && __bfloat162float(S.msk[st][k1]) > 0.5f;
      }
      const float x0 = live0 ? (sa[0] + sb[0]) * P.scale_log2 : -INFINITY;
      const float x1 = live0 ? (sa[1] + sb[1]) * P.scale_log2 : -INFINITY;
      const float x2 = live1 ? (sa[2] + sb[2]) * P.scale_log2 : -INFINITY;
      const float x3 = live1 ? (sa[3] + sb[3]) * P.scale_log2 : -INFINITY;
      float tm0 = fmaxf(x0, x2), tm1 = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, off));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, off));
      }
      const float n0 = fmaxf(m0, tm0), n1 = fmaxf(m1, tm1);
      const float c0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - n0);
      const float c1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - n1);
      const float p0 = live0 ? exp2f(x0 - n0) : 0.f;
      const float p1 = live0 ? exp2f(x1 - n1) : 0.f;
      const float p2 = live1 ? exp2f(x2 - n0) : 0.f;
      const float p3 = live1 ? exp2f(x3 - n1) : 0.f;
      m0 = n0;
      m1 = n1;
      l0 = l0 * c0 + p0 + p2;
      l1 = l1 * c1 + p1 + p3;
#pragma unroll
      for (int mt = 0; mt < NT16; ++mt) {
        o[mt][0] *= c0;
        o[mt][1] *= c1;
        o[mt][2] *= c0;
        o[mt][3] *= c1;
      }
      // P^T as the B operand, split into bf16(P) + bf16(P - bf16(P)) so the
      // probabilities enter O with 16 significant bits: transpose the 8x8
      // (key x head) blocks of both terms
      uint32_t ph0, pl0, ph1, pl1;
      split_bf16(p0, p1, ph0, pl0);
      split_bf16(p2, p3, ph1, pl1);
      const uint32_t b0 = movm_t(ph0), b1 = movm_t(ph1);
      const uint32_t bl0 = movm_t(pl0), bl1 = movm_t(pl1);
      // O^T += V_w^T . P^T
      const int vkey = kb + ((lane >> 4) << 3) + (lane & 7);
      const uint32_t vaddr = smem_u32(vst) + vkey * 128;
#pragma unroll
      for (int mt = 0; mt < NT16; ++mt) {
        const int dch = 2 * mt + ((lane >> 3) & 1);
        uint32_t a[4];
        ldsm_x4_t(a, vaddr + (dch >> 3) * G::HALF_BYTES + (((dch & 7) ^ (vkey & 7)) << 4));
        mma_bf16(o[mt], a, b0, b1);
        mma_bf16(o[mt], a, bl0, bl1);
      }
    }
    __syncthreads();  // stage consumed
    if (i == count - 1) T2B_TRACE_MARK(4);
    if (tid == 0 && issued < count) {
      fence_proxy_async();
      arm(issued, pro);
      load_kv(issued, pro);
      load_q(issued, pro);
      if (++issued < count) next_tile(pro, S, P.n_kv);
    }
    if (!unit_end) continue;

    // ---- unit (or this CTA's share of it) done: combine the four warps ----
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (g == 0) {
      if (h0 < QPG) {
        S.mw[warp][h0] = m0;
        S.lw[warp][h0] = l0;
      }
      if (h1 < QPG) {
        S.mw[warp][h1] = m1;
        S.lw[warp][h1] = l1;
      }
    }
#pragma unroll
    for (int mt = 0; mt < NT16; ++mt) {
      if (h0 < QPG) {
        S.ow[warp][h0][16 * mt + g] = o[mt][0];
        S.ow[warp][h0][16 * mt + g + 8] = o[mt][2];
      }
      if (h1 < QPG) {
        S.ow[warp][h1][16 * mt + g] = o[mt][1];
        S.ow[warp][h1][16 * mt + g + 8] = o[mt][3];
      }
    }
    __syncthreads();
    const size_t obase = (size_t)r.m * P.n_heads * HD + (size_t)r.h * QPG * HD;
    const int unit_t0 = S.row_start[r.m] + r.h * r.nt;  // global index of the unit's first tile
    bool whole = r.nt <= snap_max;
    int c1 = c, c2 = c;
    if (!whole) {
      c1 = cta_of_tile(unit_t0, T, NP);
      c2 = cta_of_tile(unit_t0 + r.nt - 1, T, NP);
      whole = c1 == c2;
    }
    // record slot: 0 for the unit this CTA's range starts in, 1 for a later one
    float* rec = P.ws + ((size_t)c * 2 + (t_lo >= unit_t0 ? 0 : 1)) * QPG * REC;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      const int e = tid + k * AT_THREADS;
      if (e < NPAIR) {
        const int hh = (2 * e) / HD, d = (2 * e) % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < AT_WARPS; ++w) M = fmaxf(M, S.mw[w][hh]);
        float den = 0.f, a0 = 0.f, a1 = 0.f;
        if (M != -INFINITY) {
#pragma unroll
          for (int w = 0; w < AT_WARPS; ++w) {
            const float mw = S.mw[w][hh];
            const float wt = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
            den += wt * S.lw[w][hh];
            a0 += wt * S.ow[w][hh][d];
            a1 += wt * S.ow[w][hh][d + 1];
          }
        }
        const float inv = den > 0.f ? 1.f / den : 0.f;
        if (whole) {
          store_out_pair(P, obase + hh * HD + d, a0 * inv, a1 * inv);
        } else {
          *reinterpret_cast<float2*>(&rec[hh * REC + d]) = make_float2(a0 * inv, a1 * inv);
          if (d == 0) *reinterpret_cast<float2*>(&rec[hh * REC + HD]) = make_float2(M, den);
        }
      }
    }
    if (i == count - 1) T2B_TRACE_MARK(5);
    if (!whole && n_split < 2) split[n_split++] = SplitUnit{r.m, r.h, unit_t0, c1, c2};
  }
  if (n_split == 0) {
    T2B_TRACE_MARK(6);
    return;
  }

  // ---- tickets for the cut units; the last CTA to arrive at a unit merges it ----
  __syncthreads();  // every record store of this CTA precedes thread 0's fence
  if (tid == 0) {
    __threadfence();
    int last = 0;
    for (int k = 0; k < n_split; ++k) {
      int* cnt = P.cnt + split[k].m * P.n_kv + split[k].h;
      const int prev = atomicAdd(cnt, 1);
      if (prev == split[k].c2 - split[k].c1) {
        atomicExch(cnt, 0);  // re-armed for the next launch
        last |= 1 << k;
      }
    }
    if (last) __threadfence();
    S.flag = last;
  }
  __syncthreads();
  const int last = S.flag;
  for (int k = 0; k < n_split; ++k) {
    if (!((last >> k) & 1)) continue;
    const SplitUnit su = split[k];
    const int n = su.c2 - su.c1 + 1;
    const int first_slot = range_start(S, rows, su.c1, T, NP, snap_max) >= su.t0 ? 0 : 1;
    auto part = [&](int p) -> const float* {
      return P.ws + ((size_t)(su.c1 + p) * 2 + (p == 0 ? first_slot : 0)) * QPG * REC;
    };
    for (int hh = warp; hh < QPG; hh += AT_WARPS) {  // per head: max and weighted sum over the parts
      float M = -INFINITY;
      for (int p = lane; p < n; p += 32) M = fmaxf(M, ldcg(part(p) + hh * REC + HD));
      M = warp_max(M);
      float den = 0.f;
      if (M != -INFINITY)
        for (int p = lane; p < n; p += 32) {
          const float mp = ldcg(part(p) + hh * REC + HD);
          if (mp != -INFINITY) den += exp2f(mp - M) * ldcg(part(p) + hh * REC + HD + 1);
        }
      den = warp_sum(den);
      if (lane == 0) {
        S.mh[hh] = M;
        S.dh[hh] = den;
      }
    }
    __syncthreads();
    float acc[EPT][2];
#pragma unroll
    for (int e = 0; e < EPT; ++e) acc[e][0] = acc[e][1] = 0.f;
    for (int b0 = 0; b0 < n; b0 += AT_MERGE_BATCH) {
      const int nb = min(AT_MERGE_BATCH, n - b0);
      for (int e = tid; e < nb * QPG; e += AT_THREADS) {
        const int p = e / QPG, hh = e - p * QPG;
        const float* rr = part(b0 + p) + hh * REC;
        const float mp = ldcg(rr + HD), M = S.mh[hh], den = S.dh[hh];
        S.wpart[p][hh] = (mp == -INFINITY || !(den > 0.f)) ? 0.f : exp2f(mp - M) * ldcg(rr + HD + 1) / den;
      }
      __syncthreads();
#pragma unroll
      for (int e2 = 0; e2 < EPT; ++e2) {
        const int e = tid + e2 * AT_THREADS;
        if (e < NPAIR) {
          const int hh = (2 * e) / HD, d = (2 * e) % HD;
#pragma unroll 4
          for (int p = 0; p < nb; ++p) {
            const float wt = S.wpart[p][hh];
            const float2 v = __ldcg(reinterpret_cast<const float2*>(part(b0 + p) + hh * REC + d));
            acc[e2][0] += wt * v.x;
            acc[e2][1] += wt * v.y;
          }
        }
      }
      __syncthreads();
    }
    const size_t obase = (size_t)su.m * P.n_heads * HD + (size_t)su.h * QPG * HD;
#pragma unroll
    for (int e2 = 0; e2 < EPT; ++e2) {
      const int e = tid + e2 * AT_THREADS;
      if (e < NPAIR) {
        const int hh = (2 * e) / HD, d = (2 * e) % HD;
        store_out_pair(P, obase + hh * HD + d, acc[e2][0], acc[e2][1]);
      }
    }
  }
  T2B_TRACE_MARK(6);
}

// ---------------------------------------------------------------------------

static long long max_tiles(int rows, int n_kv, int max_keys) {
  return (long long)rows * n_kv * ((max_keys + AT_TILE - 1) / AT_TILE);
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return n > 0 ? n : 148;
}

// Grid bound used to size the workspace (independent of the device).
static int grid_bound(int rows, int n_kv, int max_keys) {
  const long long g = std::min<long long>(max_tiles(rows, n_kv, max_keys), 160LL * AT_MAX_CTAS_PER_SM);
  return (int)(g < 1 ? 1 : g);
}

size_t attention_workspace_bytes(int rows, int n_heads, int n_kv, int head_dim, int max_keys) {
  const int qpg = n_heads / n_kv;
  const int g = grid_bound(rows, n_kv, max_keys);
  size_t part = (size_t)g * 2 * qpg * (head_dim + 2) * sizeof(float);
  part = (part + 255) & ~size_t(255);
  return part + (((size_t)rows * n_kv * sizeof(int) + 255) & ~size_t(255));
}

// Four tensor maps over a K and a V region viewed as [units][keys][hd] bf16
// (keys `key_stride` bytes apart, units `unit_stride` bytes apart), boxes of
// 64 dims x 64 keys and 64 dims x 16 keys, 128-byte swizzle; keys past
// `keys` read as zero.
static int make_kv_maps(AttnParams& P, const void* k, const void* v, int hd, long long keys, long long units,
                        long long key_stride, long long unit_stride) {
  const EncodeTiledFn encode = encode_tiled();
  if (encode == nullptr) return T2B_ERR_LAUNCH;
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) return T2B_ERR_ALIGN;
  if ((key_stride | unit_stride) & 15) return T2B_ERR_ALIGN;
  cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)keys, (cuuint64_t)units};
  cuuint64_t strides[2] = {(cuuint64_t)key_stride, (cuuint64_t)unit_stride};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap* maps[4] = {&P.kmap_full, &P.vmap_full, &P.kmap_sub, &P.vmap_sub};
  for (int i = 0; i < 4; ++i) {
    cuuint32_t box[3] = {64, (cuuint32_t)(i < 2 ? AT_TILE : AT_SUB), 1};
    CUresult r = encode(maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(i % 2 ? v : k), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return T2B_ERR_ARG;
  }
  return T2B_OK;
}

// One wave: as many CTAs as are resident at once (capped by the tile count
// and the workspace bound).
template <int HD, int QPG, int ST>
static int attn_launch_t(AttnParams& P, int max_grid, cudaStream_t st) {
  auto kern = decode_attention_kernel<HD, QPG, ST>;
  const size_t smem = attn_smem_bytes<HD, QPG, ST>();
  if (allow_smem(kern, smem) != T2B_OK) return T2B_ERR_LAUNCH;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, AT_THREADS, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  per_sm = std::min(per_sm, AT_MAX_CTAS_PER_SM);
  int grid = std::max(1, std::min(max_grid, sm_count() * per_sm));
  // env T2B_ATTN_GRID caps the grid (experiments: fewer CTAs, all resident
  // beside the preceding kernel's)
  if (const char* e = getenv("T2B_ATTN_GRID")) {
    const int cap = atoi(e);
    if (cap > 0) grid = std::min(grid, cap);
  }
  return launch_pdl(kern, dim3(grid), dim3(AT_THREADS), smem, st, P);
}

// Ring depth of the head_dim-128 kernel.  3 stages of 32 KB (2 CTAs per SM)
// while a CTA streams few tiles: at short contexts the loads issued before
// the dependency wait and whole units per CTA decide the time (Qwen3-0.6B,
// 64 rows, context 190: 16.7 us against 21.5 us with 2 stages).  2 stages
// (3 CTAs, 12 warps per SM) for long streams, where the tile math -- two
// score and two P.V MMAs per 16-key slice -- needs the extra warps to keep
// pace with the copies (Qwen3-8B, 64 rows, context 4096: 181 us against 334
// us, 5.9 TB/s).  max_keys (the cache length) stands in for the context.
static int attn_stages_hd128(int rows, int n_kv, int max_keys) {
  return max_tiles(rows, n_kv, max_keys) >= 12LL * 2 * sm_count() ? 2 : 3;
}

// max_keys: upper bound on keys per row (sizes the grid and the workspace).
int attention_launch(AttnParams& P, int rows, int head_dim, int max_keys, void* ws, size_t ws_bytes,
                     cudaStream_t st) {
  if (rows < 1 || rows > AT_MAX_ROWS || P.n_kv < 1 || P.n_heads % P.n_kv) return T2B_ERR_SHAPE;
  const int qpg = P.n_heads / P.n_kv;
  const size_t need = attention_workspace_bytes(rows, P.n_heads, P.n_kv, head_dim, max_keys);
  if (ws_bytes < need || !ws) return T2B_ERR_WORKSPACE;
  const int grid = grid_bound(rows, P.n_kv, max_keys);
  size_t part = (size_t)grid * 2 * qpg * (head_dim + 2) * sizeof(float);
  part = (part + 255) & ~size_t(255);
  P.ws = reinterpret_cast<float*>(ws);
  P.err = error_word(st);
  P.cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + part);
  P.rows = rows;
  P.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  const int st128 = attn_stages_hd128(rows, P.n_kv, max_keys);
#define T2B_ACASE(hd, qpg_, st_) \
  if (head_dim == hd && qpg == qpg_ && (hd == 64 || st128 == st_)) return attn_launch_t<hd, qpg_, st_>(P, grid, st);
  T2B_ACASE(128, 1, 3) T2B_ACASE(128, 2, 3) T2B_ACASE(128, 4, 3) T2B_ACASE(128, 8, 3)
  T2B_ACASE(128, 1, 2) T2B_ACASE(128, 2, 2) T2B_ACASE(128, 4, 2) T2B_ACASE(128, 8, 2)
  T2B_ACASE(64, 1, 4) T2B_ACASE(64, 2, 4) T2B_ACASE(64, 4, 4) T2B_ACASE(64, 8, 4)
#undef T2B_ACASE
  return T2B_ERR_SHAPE;
}

}  // namespace t2b

// ===========================================================================
// C ABI
// ===========================================================================
using namespace t2b;

extern "C" size_t t2b_decode_attention_workspace_bytes(int M, int n_heads, int n_kv, int head_dim, int max_ctx) {
  if (M < 1 || n_kv < 1 || max_ctx < 1) return 0;
  return attention_workspace_bytes(M, n_heads, n_kv, head_dim, max_ctx);
}

static int decode_attention_impl(const void* q, int q_dtype, const uint16_t* k_cache, const uint16_t* v_cache,
                                 const int32_t* pos, uint16_t* out, int out_dtype, int M, int n_heads, int n_kv,
                                 int head_dim, int max_ctx, void* ws, size_t ws_bytes, void* stream, int kv_early) {
  if (!q || !k_cache || !v_cache || !pos || !out) return T2B_ERR_ARG;
  if (out_dtype != T2B_DTYPE_BF16 && out_dtype != T2B_DTYPE_F16) return T2B_ERR_ARG;
  if (q_dtype != T2B_DTYPE_BF16 && q_dtype != T2B_DTYPE_F32) return T2B_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
       reinterpret_cast<uintptr_t>(q)) & 15)
    return T2B_ERR_ALIGN;
  if (max_ctx % 8 || (head_dim != 64 && head_dim != 128) || M < 1 || n_kv < 1) return T2B_ERR_SHAPE;
  AttnParams P{};
  const int mk = make_kv_maps(P, k_cache, v_cache, head_dim, max_ctx, (long long)M * n_kv, (long long)head_dim * 2,
                              (long long)max_ctx * head_dim * 2);
  if (mk != T2B_OK) return mk;
  P.q = q;
  P.q_f32 = q_dtype == T2B_DTYPE_F32;
  P.mask0 = nullptr;
  P.tile_y = AT_TILE;
  P.unit_z = 1;
  P.tile_z = 0;
  P.pos = pos;
  P.n_keys = max_ctx;
  P.out = reinterpret_cast<__nv_bfloat16*>(out);
  P.out_f16 = out_dtype == T2B_DTYPE_F16;
  P.n_heads = n_heads;
  P.n_kv = n_kv;
  P.kv_early = kv_early;
  return attention_launch(P, M, head_dim, max_ctx, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int t2b_decode_attention(const void* q, int q_dtype, const uint16_t* k_cache, const uint16_t* v_cache,
                                    const int32_t* pos, uint16_t* out, int out_dtype, int M, int n_heads, int n_kv,
                                    int head_dim, int max_ctx, void* ws, size_t ws_bytes, void* stream) {
  return decode_attention_impl(q, q_dtype, k_cache, v_cache, pos, out, out_dtype, M, n_heads, n_kv, head_dim,
                               max_ctx, ws, ws_bytes, stream, 0);
}

extern "C" int t2b_decode_attention_after_kvwrite(const void* q, int q_dtype, const uint16_t* k_cache,
                                                  const uint16_t* v_cache, const int32_t* pos, uint16_t* out,
                                                  int out_dtype, int M, int n_heads, int n_kv, int head_dim,
                                                  int max_ctx, void* ws, size_t ws_bytes, void* stream) {
  return decode_attention_impl(q, q_dtype, k_cache, v_cache, pos, out, out_dtype, M, n_heads, n_kv, head_dim,
                               max_ctx, ws, ws_bytes, stream, 1);
}

extern "C" int t2b_packet_attention(const uint16_t* q, const uint16_t* packet, uint16_t* out, int n_groups,
                                    int q_per_group, int head_dim, int packet_seq_len, int chunk, void* ws,
                                    size_t ws_bytes, void* stream) {
  if (!q || !packet || !out) return T2B_ERR_ARG;
  if (chunk != AT_TILE || packet_seq_len < chunk || packet_seq_len % chunk) return T2B_ERR_SHAPE;
  if (head_dim != 64 && head_dim != 128) return T2B_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(packet) | reinterpret_cast<uintptr_t>(q)) & 15) return T2B_ERR_ALIGN;
  const long long chunk_el = 2LL * chunk * head_dim + chunk;  // K, V, mask of one chunk
  const long long n_chunks = packet_seq_len / chunk;
  const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(packet);
  AttnParams P{};
  const int mk = make_kv_maps(P, base, base + (long long)chunk * head_dim, head_dim, chunk, n_groups * n_chunks,
                              (long long)head_dim * 2, chunk_el * 2);
  if (mk != T2B_OK) return mk;
  P.q = q;
  P.q_f32 = 0;
  P.mask0 = base + 2LL * chunk * head_dim;
  P.mask_unit = n_chunks * chunk_el;
  P.mask_tile = chunk_el;
  P.tile_y = 0;
  P.unit_z = (int)n_chunks;
  P.tile_z = 1;
  P.pos = nullptr;
  P.n_keys = packet_seq_len;
  P.out = reinterpret_cast<__nv_bfloat16*>(out);
  P.n_heads = n_groups * q_per_group;
  P.n_kv = n_groups;
  return attention_launch(P, 1, head_dim, packet_seq_len, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

T2B_TRACE_DUMP_FN(t2b_trace_dump_attn)
