// GQA decode attention over a bf16 KV cache, persistent and tile-balanced.
//
// Work: every (batch row m, kv head h) "unit" attends q[m, h*qpg .. +qpg]
// (all q heads of the GQA group in one pass, so each K/V byte is read once)
// over keys 0..pos[m], cut into 64-key tiles.  All tiles of all units form
// one list (row-major units); a fixed grid of ~3 CTAs per SM splits the list
// into equal contiguous ranges, so every SM streams the same number of KV
// bytes in a single wave whatever the context lengths.  Each CTA pulls its
// tiles through a shared-memory ring with 1-D TMA bulk copies (issued ahead,
// completion on mbarriers with time-bounded waits) and keeps an fp32 online
// softmax (running max / sum; model.py:266-279, and the chunked update of
// llama_chunked_attention/kernel.cc:111-257) for the unit it is in.  A unit
// cut between CTAs leaves one partial (o, max, sum) per CTA; the last CTA to
// finish it (ticket counter, re-armed) merges them.
//
// The same kernel reads the reference's packet cache
// ([group][chunk][K 64*hd | V 64*hd | mask 64], decode_packet_cache.py:11-43):
// tile = chunk, and slots whose mask <= 0.5 are skipped
// (attention_reference.py:153-154).

#include <algorithm>

#include "t2b_common.cuh"
#include "launch.cuh"

namespace t2b {

constexpr int AT_THREADS = 128;
constexpr int AT_TILE = 64;
constexpr int AT_STAGES = 2;
constexpr int AT_MAX_CTAS_PER_SM = 4;  // workspace bound; the grid uses the measured occupancy
constexpr int AT_MAX_ROWS = 256;

struct AttnParams {
  const __nv_bfloat16* q;    // [rows][n_heads*hd]
  const __nv_bfloat16* k0;   // key 0 of (row 0, kv head 0)
  const __nv_bfloat16* v0;
  const __nv_bfloat16* mask0;  // nullable (packet mode)
  long long stride_row;      // elements between batch rows
  long long stride_head;     // elements between kv heads
  long long tile_stride;     // elements between 64-key tiles
  const int* pos;            // nullable: keys = pos[m] + 1 (clamped to [1, n_keys]), else n_keys
  int n_keys;                // packet mode: keys per unit; cache mode: max_ctx
  int rows;
  __nv_bfloat16* out;        // [rows][n_heads*hd]
  int n_heads, n_kv;
  float scale;
  float* ws;                 // partial records [grid][2][qpg][hd + 2]
  int* cnt;                  // [rows][n_kv] tickets
  int* err;
};

template <int HD, int QPG>
struct AttnSmem {
  float q[QPG][HD];
  __nv_bfloat16 k[AT_STAGES][AT_TILE][HD];
  __nv_bfloat16 v[AT_STAGES][AT_TILE][HD];
  __nv_bfloat16 msk[AT_STAGES][AT_TILE];
  __nv_bfloat16 qb[AT_STAGES][QPG * HD];  // q heads of a unit, copied with the unit's first tile
  float p[QPG][AT_TILE];
  float corr[QPG];
  float mrun[QPG];
  float lrun[QPG];
  int row_start[AT_MAX_ROWS + 1];  // first global tile index of row m (all its kv heads)
  int row_tiles[AT_MAX_ROWS];      // tiles per unit of row m
  int row_keys[AT_MAX_ROWS];       // keys attended by row m
  uint64_t bar[AT_STAGES];
};

struct TileRef {
  int m, h, j, nt;  // unit (m, h), tile j of nt
};

// Keys attended by row m: pos[m] + 1, kept inside the cache whatever pos holds.
T2B_DEV int keys_of_row_global(const AttnParams& P, int m) {
  if (!P.pos) return P.n_keys;
  const int k = P.pos[m] + 1;
  return k < 1 ? 1 : (k > P.n_keys ? P.n_keys : k);
}

template <int HD, int QPG>
T2B_DEV TileRef locate(const AttnSmem<HD, QPG>& S, int rows, int t) {
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

// Contiguous split of T tiles over NP CTAs (NP <= T, so no range is empty).
T2B_DEV int range_lo(long long c, long long T, long long NP) { return (int)(c * T / NP); }
T2B_DEV int cta_of_tile(long long t, long long T, long long NP) { return (int)(((t + 1) * NP + T - 1) / T - 1); }

template <int HD, int QPG>
T2B_DEV int record_slot(const AttnSmem<HD, QPG>& S, int rows, long long T, long long NP, int cta, int m, int h) {
  const TileRef f = locate(S, rows, range_lo(cta, T, NP));
  return (f.m == m && f.h == h) ? 0 : 1;  // slot 0: the CTA's first unit, slot 1: its last
}

template <int HD, int QPG>
__global__ void __launch_bounds__(AT_THREADS) decode_attention_kernel(const AttnParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  AttnSmem<HD, QPG>& S = *reinterpret_cast<AttnSmem<HD, QPG>*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x;
  T2B_TRACE_BEGIN(10, P.n_heads);

  if (tid == 0) {
    for (int i = 0; i < AT_STAGES; ++i) mbar_init(&S.bar[i], 1);
    fence_mbar_init();
  }
  grid_dep_wait();
  grid_dep_launch();
  T2B_TRACE_MARK(1);

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
  const long long NP = T < (long long)gridDim.x ? T : (long long)gridDim.x;  // active CTAs
  if (c >= NP) return;
  const int t_lo = range_lo(c, T, NP), t_hi = range_lo(c + 1, T, NP);
  const int count = t_hi - t_lo;

  auto issue = [&](int i) {  // tile i of this CTA into stage i % AT_STAGES (+ q on a unit's first tile)
    const TileRef r = locate(S, rows, t_lo + i);
    const int nk = min(AT_TILE, S.row_keys[r.m] - r.j * AT_TILE);
    const uint32_t bytes = (uint32_t)nk * HD * 2;
    const int st = i % AT_STAGES;
    const long long base =
        (long long)r.m * P.stride_row + (long long)r.h * P.stride_head + (long long)r.j * P.tile_stride;
    const uint32_t mbytes = P.mask0 ? (uint32_t)AT_TILE * 2 : 0u;
    const bool with_q = (i == 0) || (r.j == 0);
    const uint32_t qbytes = with_q ? (uint32_t)(QPG * HD * 2) : 0u;
    mbar_arrive_expect_tx(&S.bar[st], 2 * bytes + mbytes + qbytes);
    bulk_g2s(&S.k[st][0][0], P.k0 + base, bytes, &S.bar[st]);
    bulk_g2s(&S.v[st][0][0], P.v0 + base, bytes, &S.bar[st]);
    if (P.mask0) bulk_g2s(&S.msk[st][0], P.mask0 + base, mbytes, &S.bar[st]);
    if (with_q) bulk_g2s(&S.qb[st][0], P.q + (size_t)r.m * P.n_heads * HD + (size_t)r.h * QPG * HD, qbytes, &S.bar[st]);
  };
  if (tid == 0)
    for (int i = 0; i < AT_STAGES && i < count; ++i) issue(i);

  constexpr int NPAIR = (QPG * HD / 2 + AT_THREADS - 1) / AT_THREADS;
  float o[NPAIR][2];
  constexpr int QH = QPG * HD;
  for (int i = 0; i < count; ++i) {
    const TileRef r = locate(S, rows, t_lo + i);
    const bool unit_begin = (i == 0) || (r.j == 0);
    const bool unit_end = (i == count - 1) || (r.j == r.nt - 1);
    const int st = i % AT_STAGES;
    // every thread takes the same outcome, so no thread is left at a barrier
    const bool ok = __syncthreads_and(mbar_wait_bounded(&S.bar[st], (i / AT_STAGES) & 1, P.err));
    if (!ok) break;  // timeout recorded in P.err
    if (i == 0) T2B_TRACE_MARK(2);
    if (unit_begin) {  // new unit: its q heads (arrived with this tile), fresh softmax state
      for (int e = tid; e < QH; e += AT_THREADS) S.q[e / HD][e % HD] = __bfloat162float(S.qb[st][e]);
      if (tid < QPG) {
        S.mrun[tid] = -INFINITY;
        S.lrun[tid] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < NPAIR; ++e) o[e][0] = o[e][1] = 0.f;
      __syncthreads();
    }
    const int nk = min(AT_TILE, S.row_keys[r.m] - r.j * AT_TILE);
    // scores: one (head, key) per thread-iteration; 16-byte K chunks rotated by
    // key index so the 8 lanes of a quarter-warp hit distinct banks
    for (int sidx = tid; sidx < QPG * AT_TILE; sidx += AT_THREADS) {
      const int hh = sidx / AT_TILE, j = sidx - hh * AT_TILE;
      float sc = -INFINITY;
      bool live = j < nk;
      if (live && P.mask0) live = __bfloat162float(S.msk[st][j]) > 0.5f;
      if (live) {
        float a = 0.f;
#pragma unroll
        for (int c0 = 0; c0 < HD / 8; ++c0) {
          const int cc = (c0 + j) & (HD / 8 - 1);
          const uint4 kv = *reinterpret_cast<const uint4*>(&S.k[st][j][cc * 8]);
          const float* qq = &S.q[hh][cc * 8];
          const uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            a = fmaf(qq[2 * e], __uint_as_float(w[e] << 16), a);
            a = fmaf(qq[2 * e + 1], __uint_as_float(w[e] & 0xffff0000u), a);
          }
        }
        sc = a * P.scale;
      }
      S.p[hh][j] = sc;
    }
    __syncthreads();
    // online softmax update, one warp per head
    for (int hh = warp; hh < QPG; hh += AT_THREADS / 32) {
      const float s0 = S.p[hh][lane], s1 = S.p[hh][lane + 32];
      const float tmax = warp_max(fmaxf(s0, s1));
      const float mold = S.mrun[hh];
      const float mnew = fmaxf(mold, tmax);
      float p0 = 0.f, p1 = 0.f, corr = 1.f;
      if (mnew != -INFINITY) {
        p0 = __expf(s0 - mnew);
        p1 = __expf(s1 - mnew);
        corr = (mold == -INFINITY) ? 0.f : __expf(mold - mnew);
      }
      S.p[hh][lane] = p0;
      S.p[hh][lane + 32] = p1;
      const float psum = warp_sum(p0 + p1);
      if (lane == 0) {
        S.lrun[hh] = S.lrun[hh] * corr + psum;
        S.mrun[hh] = mnew;
        S.corr[hh] = corr;
      }
    }
    __syncthreads();
    // o = o * corr + P . V
#pragma unroll
    for (int e = 0; e < NPAIR; ++e) {
      const int pr = tid + e * AT_THREADS;
      if (pr < QPG * HD / 2) {
        const int hh = pr / (HD / 2), d2 = pr - hh * (HD / 2);
        const float corr = S.corr[hh];
        float a0 = o[e][0] * corr, a1 = o[e][1] * corr;
        for (int j = 0; j < nk; ++j) {
          const float pj = S.p[hh][j];
          const uint32_t vv = *reinterpret_cast<const uint32_t*>(&S.v[st][j][2 * d2]);
          a0 = fmaf(pj, __uint_as_float(vv << 16), a0);
          a1 = fmaf(pj, __uint_as_float(vv & 0xffff0000u), a1);
        }
        o[e][0] = a0;
        o[e][1] = a1;
      }
    }
    __syncthreads();  // stage consumed; softmax state final for this tile
    if (tid == 0 && i + AT_STAGES < count) {
      fence_proxy_async();
      issue(i + AT_STAGES);
    }
    if (!unit_end) continue;

    // ---- unit (or this CTA's share of it) done ----
    const size_t obase = (size_t)r.m * P.n_heads * HD + (size_t)r.h * QPG * HD;
    const int unit_t0 = S.row_start[r.m] + r.h * r.nt;  // global index of the unit's first tile
    const int c1 = cta_of_tile(unit_t0, T, NP), c2 = cta_of_tile(unit_t0 + r.nt - 1, T, NP);
    if (c1 == c2) {  // the whole unit ran here
#pragma unroll
      for (int e = 0; e < NPAIR; ++e) {
        const int pr = tid + e * AT_THREADS;
        if (pr < QPG * HD / 2) {
          const int hh = pr / (HD / 2), d2 = pr - hh * (HD / 2);
          const float l = S.lrun[hh];
          const float inv = l > 0.f ? 1.f / l : 0.f;
          *reinterpret_cast<__nv_bfloat162*>(&P.out[obase + hh * HD + 2 * d2]) =
              __floats2bfloat162_rn(o[e][0] * inv, o[e][1] * inv);
        }
      }
      continue;
    }
    // partial: publish (o, max, sum); the unit's last CTA merges every part
    constexpr int REC = HD + 2;
    float* mine = P.ws + ((size_t)c * 2 + record_slot(S, rows, T, NP, c, r.m, r.h)) * QPG * REC;
#pragma unroll
    for (int e = 0; e < NPAIR; ++e) {
      const int pr = tid + e * AT_THREADS;
      if (pr < QPG * HD / 2) {
        const int hh = pr / (HD / 2), d2 = pr - hh * (HD / 2);
        mine[hh * REC + 2 * d2] = o[e][0];
        mine[hh * REC + 2 * d2 + 1] = o[e][1];
      }
    }
    if (tid < QPG) {
      mine[tid * REC + HD] = S.mrun[tid];
      mine[tid * REC + HD + 1] = S.lrun[tid];
    }
    if (!split_ticket(P.cnt + (size_t)r.m * P.n_kv + r.h, c2 - c1 + 1)) continue;
    for (int e = tid; e < QH; e += AT_THREADS) {
      const int hh = e / HD, d = e - hh * HD;
      float mx = -INFINITY;
      for (int cc = c1; cc <= c2; ++cc) {
        const int sl = record_slot(S, rows, T, NP, cc, r.m, r.h);
        mx = fmaxf(mx, ldcg(P.ws + ((size_t)cc * 2 + sl) * QPG * REC + hh * REC + HD));
      }
      float num = 0.f, den = 0.f;
      if (mx != -INFINITY) {
        for (int cc = c1; cc <= c2; ++cc) {
          const int sl = record_slot(S, rows, T, NP, cc, r.m, r.h);
          const float* rr = P.ws + ((size_t)cc * 2 + sl) * QPG * REC + hh * REC;
          const float ms = ldcg(rr + HD);
          if (ms == -INFINITY) continue;
          const float w = __expf(ms - mx);
          num += w * ldcg(rr + d);
          den += w * ldcg(rr + HD + 1);
        }
      }
      P.out[obase + hh * HD + d] = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
    }
    __syncthreads();
  }
  T2B_TRACE_MARK(3);
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

// One wave: as many CTAs as are resident at once (capped by the tile count
// and the workspace bound).
template <int HD, int QPG>
static int attn_launch_t(AttnParams& P, int max_grid, cudaStream_t st) {
  auto kern = decode_attention_kernel<HD, QPG>;
  const size_t smem = sizeof(AttnSmem<HD, QPG>);
  if (allow_smem(kern, smem) != T2B_OK) return T2B_ERR_LAUNCH;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, AT_THREADS, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  per_sm = std::min(per_sm, AT_MAX_CTAS_PER_SM);
  const int grid = std::max(1, std::min(max_grid, sm_count() * per_sm));
  return launch_pdl(kern, dim3(grid), dim3(AT_THREADS), smem, st, P);
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
  P.cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + part);
  P.rows = rows;
  P.scale = 1.f / sqrtf((float)head_dim);
#define T2B_ACASE(hd, qpg_)                                          \
  if (head_dim == hd && qpg == qpg_) return attn_launch_t<hd, qpg_>(P, grid, st);
  T2B_ACASE(128, 1) T2B_ACASE(128, 2) T2B_ACASE(128, 4) T2B_ACASE(128, 8)
  T2B_ACASE(64, 1) T2B_ACASE(64, 2) T2B_ACASE(64, 4) T2B_ACASE(64, 8)
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

extern "C" int t2b_decode_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                    const int32_t* pos, uint16_t* out, int M, int n_heads, int n_kv, int head_dim,
                                    int max_ctx, void* ws, size_t ws_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !pos || !out) return T2B_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) return T2B_ERR_ALIGN;
  if (max_ctx % 8) return T2B_ERR_SHAPE;  // keeps every 64-key tile 16-byte aligned
  AttnParams P{};
  P.q = reinterpret_cast<const __nv_bfloat16*>(q);
  P.k0 = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  P.v0 = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  P.stride_head = (long long)max_ctx * head_dim;
  P.stride_row = (long long)n_kv * P.stride_head;
  P.tile_stride = (long long)AT_TILE * head_dim;
  P.pos = pos;
  P.n_keys = max_ctx;
  P.out = reinterpret_cast<__nv_bfloat16*>(out);
  P.n_heads = n_heads;
  P.n_kv = n_kv;
  return attention_launch(P, M, head_dim, max_ctx, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int t2b_packet_attention(const uint16_t* q, const uint16_t* packet, uint16_t* out, int n_groups,
                                    int q_per_group, int head_dim, int packet_seq_len, int chunk, void* ws,
                                    size_t ws_bytes, void* stream) {
  if (!q || !packet || !out) return T2B_ERR_ARG;
  if (chunk != AT_TILE || packet_seq_len < chunk || packet_seq_len % chunk) return T2B_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(packet) & 15) return T2B_ERR_ALIGN;
  const long long chunk_el = 2LL * chunk * head_dim + chunk;
  AttnParams P{};
  P.q = reinterpret_cast<const __nv_bfloat16*>(q);
  P.k0 = reinterpret_cast<const __nv_bfloat16*>(packet);
  P.v0 = P.k0 + (long long)chunk * head_dim;
  P.mask0 = P.k0 + 2LL * chunk * head_dim;
  P.stride_head = (long long)(packet_seq_len / chunk) * chunk_el;
  P.stride_row = 0;
  P.tile_stride = chunk_el;
  P.pos = nullptr;
  P.n_keys = packet_seq_len;
  P.out = reinterpret_cast<__nv_bfloat16*>(out);
  P.n_heads = n_groups * q_per_group;
  P.n_kv = n_groups;
  return attention_launch(P, 1, head_dim, packet_seq_len, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

T2B_TRACE_DUMP_FN(t2b_trace_dump_attn)
