// Split-K (flash-decoding) GQA decode attention over a bf16 KV cache.
//
// One CTA = (kv head, batch row, key split).  All q heads of the GQA group
// (q_per_group of them) ride in the same CTA, so every K/V byte is read from
// HBM exactly once per step.  Keys stream through shared memory in 64-key
// tiles brought in by 1-D TMA bulk copies (cp.async.bulk) into a two-stage
// ring; completion is tracked by mbarriers with bounded waits.  Scores and
// the online softmax (running max / sum, fp32) follow
// src/models/quantized_qwen3/model.py:266-279 and the chunked update of
// src/torch2iron/operators/llama_chunked_attention/kernel.cc:111-257; splits
// meet in a fp32 workspace and the last CTA of a (row, kv head) merges them.
//
// The same kernel reads the reference's packet cache
// ([group][chunk][K 64*hd | V 64*hd | mask 64], decode_packet_cache.py:11-43):
// tile = chunk, and slots whose mask <= 0.5 are skipped
// (attention_reference.py:153-154).

#include "t2b_common.cuh"
#include "launch.cuh"

namespace t2b {

constexpr int AT_THREADS = 128;
constexpr int AT_TILE = 64;

struct AttnParams {
  const __nv_bfloat16* q;    // [rows][n_heads*hd]
  const __nv_bfloat16* k0;   // key 0 of (row 0, kv head 0)
  const __nv_bfloat16* v0;
  const __nv_bfloat16* mask0;  // nullable (packet mode)
  long long stride_row;      // elements between batch rows
  long long stride_head;     // elements between kv heads
  long long tile_stride;     // elements between 64-key tiles
  const int* pos;            // nullable: keys = pos[m] + 1, else n_keys
  int n_keys;
  __nv_bfloat16* out;        // [rows][n_heads*hd]
  int n_heads, n_kv;
  int nsplit;
  float scale;
  float* ws;                 // [rows][n_kv][nsplit][qpg][hd + 2]
  int* cnt;                  // [rows][n_kv]
  int* err;
};

template <int HD, int QPG>
struct AttnSmem {
  float q[QPG][HD];
  __nv_bfloat16 k[2][AT_TILE][HD];
  __nv_bfloat16 v[2][AT_TILE][HD];
  __nv_bfloat16 msk[2][AT_TILE];
  float p[QPG][AT_TILE];
  float corr[QPG];
  float mrun[QPG];
  float lrun[QPG];
  uint64_t bar[2];
};

template <int HD, int QPG>
__global__ void __launch_bounds__(AT_THREADS) decode_attention_kernel(const AttnParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  AttnSmem<HD, QPG>& S = *reinterpret_cast<AttnSmem<HD, QPG>*>(smem_raw);
  const int kvh = blockIdx.x, m = blockIdx.y, split = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  T2B_TRACE_BEGIN(10, P.n_heads);

  if (tid == 0) {
    mbar_init(&S.bar[0], 1);
    mbar_init(&S.bar[1], 1);
    fence_mbar_init();
  }
  grid_dep_wait();
  grid_dep_launch();
  T2B_TRACE_MARK(1);

  const int n_keys = P.pos ? P.pos[m] + 1 : P.n_keys;
  // key range of this split, in whole 64-key tiles
  const int tiles_total = (n_keys + AT_TILE - 1) / AT_TILE;
  const int tiles_per = (tiles_total + P.nsplit - 1) / P.nsplit;
  const int t_begin = split * tiles_per;
  const int t_end = min(tiles_total, t_begin + tiles_per);
  const int ntiles = max(0, t_end - t_begin);

  const __nv_bfloat16* kb = P.k0 + m * P.stride_row + kvh * P.stride_head;
  const __nv_bfloat16* vb = P.v0 + m * P.stride_row + kvh * P.stride_head;
  const __nv_bfloat16* mb = P.mask0 ? P.mask0 + m * P.stride_row + kvh * P.stride_head : nullptr;

  for (int i = tid; i < QPG * HD; i += AT_THREADS) {
    const int h = i / HD, d = i - h * HD;
    S.q[h][d] = __bfloat162float(P.q[(size_t)m * P.n_heads * HD + (kvh * QPG + h) * HD + d]);
  }
  if (tid < QPG) {
    S.mrun[tid] = -INFINITY;
    S.lrun[tid] = 0.f;
  }
  __syncthreads();

  auto issue = [&](int t, int buf) {
    const int key0 = (t_begin + t) * AT_TILE;
    const int nk = min(AT_TILE, n_keys - key0);
    const uint32_t bytes = (uint32_t)nk * HD * 2;
    const uint32_t mbytes = mb ? (uint32_t)AT_TILE * 2 : 0u;
    mbar_arrive_expect_tx(&S.bar[buf], 2 * bytes + mbytes);
    const long long off = (long long)(t_begin + t) * P.tile_stride;
    bulk_g2s(&S.k[buf][0][0], kb + off, bytes, &S.bar[buf]);
    bulk_g2s(&S.v[buf][0][0], vb + off, bytes, &S.bar[buf]);
    if (mb) bulk_g2s(&S.msk[buf][0], mb + off, mbytes, &S.bar[buf]);
  };
  if (tid == 0) {
    if (ntiles > 0) issue(0, 0);
    if (ntiles > 1) issue(1, 1);
  }

  // per-thread output slice: pairs of dims, QPG*HD/2 pairs over 128 threads
  constexpr int NPAIR = (QPG * HD / 2 + AT_THREADS - 1) / AT_THREADS;
  float o[NPAIR][2];
#pragma unroll
  for (int i = 0; i < NPAIR; ++i) o[i][0] = o[i][1] = 0.f;

  bool ok = true;
  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (!mbar_wait_bounded(&S.bar[buf], (t >> 1) & 1, P.err)) {
      ok = false;
      break;
    }
    if (t == 0) T2B_TRACE_MARK(2);
    const int key0 = (t_begin + t) * AT_TILE;
    const int nk = min(AT_TILE, n_keys - key0);
    // scores: one (head, key) per thread-iteration; 16-byte K chunks rotated by
    // key index so the 8 lanes of a quarter-warp hit distinct banks
    for (int sidx = tid; sidx < QPG * AT_TILE; sidx += AT_THREADS) {
      const int h = sidx / AT_TILE, j = sidx - h * AT_TILE;
      float s = -INFINITY;
      bool live = j < nk;
      if (live && mb) live = __bfloat162float(S.msk[buf][j]) > 0.5f;
      if (live) {
        float a = 0.f;
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
          const int cc = (c + j) & (HD / 8 - 1);
          const uint4 kv = *reinterpret_cast<const uint4*>(&S.k[buf][j][cc * 8]);
          const float* qq = &S.q[h][cc * 8];
          const uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            a = fmaf(qq[2 * e], __uint_as_float(w[e] << 16), a);
            a = fmaf(qq[2 * e + 1], __uint_as_float(w[e] & 0xffff0000u), a);
          }
        }
        s = a * P.scale;
      }
      S.p[h][j] = s;
    }
    __syncthreads();
    // online softmax update, one warp per head
    for (int h = warp; h < QPG; h += AT_THREADS / 32) {
      const float s0 = S.p[h][lane], s1 = S.p[h][lane + 32];
      const float tmax = warp_max(fmaxf(s0, s1));
      const float mold = S.mrun[h];
      const float mnew = fmaxf(mold, tmax);
      float p0 = 0.f, p1 = 0.f, corr = 1.f;
      if (mnew != -INFINITY) {
        p0 = __expf(s0 - mnew);
        p1 = __expf(s1 - mnew);
        corr = (mold == -INFINITY) ? 0.f : __expf(mold - mnew);
      }
      S.p[h][lane] = p0;
      S.p[h][lane + 32] = p1;
      const float psum = warp_sum(p0 + p1);
      if (lane == 0) {
        S.lrun[h] = S.lrun[h] * corr + psum;
        S.mrun[h] = mnew;
        S.corr[h] = corr;
      }
    }
    __syncthreads();
    // o = o * corr + P . V
#pragma unroll
    for (int i = 0; i < NPAIR; ++i) {
      const int pr = tid + i * AT_THREADS;
      if (pr < QPG * HD / 2) {
        const int h = pr / (HD / 2), d2 = pr - h * (HD / 2);
        const float corr = S.corr[h];
        float a0 = o[i][0] * corr, a1 = o[i][1] * corr;
        for (int j = 0; j < nk; ++j) {
          const float pj = S.p[h][j];
          const uint32_t vv = *reinterpret_cast<const uint32_t*>(&S.v[buf][j][2 * d2]);
          a0 = fmaf(pj, __uint_as_float(vv << 16), a0);
          a1 = fmaf(pj, __uint_as_float(vv & 0xffff0000u), a1);
        }
        o[i][0] = a0;
        o[i][1] = a1;
      }
    }
    __syncthreads();  // buffer `buf` fully consumed
    if (tid == 0 && t + 2 < ntiles) {
      fence_proxy_async();
      issue(t + 2, buf);
    }
  }
  T2B_TRACE_MARK(3);
  if (!ok) return;  // timeout already recorded in P.err

  const size_t obase = (size_t)m * P.n_heads * HD + (size_t)kvh * QPG * HD;
  if (P.nsplit == 1) {
#pragma unroll
    for (int i = 0; i < NPAIR; ++i) {
      const int pr = tid + i * AT_THREADS;
      if (pr < QPG * HD / 2) {
        const int h = pr / (HD / 2), d2 = pr - h * (HD / 2);
        const float l = S.lrun[h];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        *reinterpret_cast<__nv_bfloat162*>(&P.out[obase + h * HD + 2 * d2]) =
            __floats2bfloat162_rn(o[i][0] * inv, o[i][1] * inv);
      }
    }
    return;
  }
  // split-K: publish (o, m, l), last CTA of this (row, kv head) merges
  const int rec = HD + 2;
  float* wsb = P.ws + (((size_t)m * P.n_kv + kvh) * P.nsplit) * QPG * rec;
  float* mine = wsb + (size_t)split * QPG * rec;
#pragma unroll
  for (int i = 0; i < NPAIR; ++i) {
    const int pr = tid + i * AT_THREADS;
    if (pr < QPG * HD / 2) {
      const int h = pr / (HD / 2), d2 = pr - h * (HD / 2);
      mine[h * rec + 2 * d2] = o[i][0];
      mine[h * rec + 2 * d2 + 1] = o[i][1];
    }
  }
  if (tid < QPG) {
    mine[tid * rec + HD] = S.mrun[tid];
    mine[tid * rec + HD + 1] = S.lrun[tid];
  }
  if (!split_ticket(P.cnt + (size_t)m * P.n_kv + kvh, P.nsplit)) return;
  for (int i = tid; i < QPG * HD; i += AT_THREADS) {
    const int h = i / HD, d = i - h * HD;
    float mx = -INFINITY;
    for (int s = 0; s < P.nsplit; ++s) mx = fmaxf(mx, ldcg(wsb + (size_t)s * QPG * rec + h * rec + HD));
    float num = 0.f, den = 0.f;
    if (mx != -INFINITY) {
      for (int s = 0; s < P.nsplit; ++s) {
        const float* r = wsb + (size_t)s * QPG * rec + h * rec;
        const float ms = ldcg(r + HD);
        if (ms == -INFINITY) continue;
        const float w = __expf(ms - mx);
        num += w * ldcg(r + d);
        den += w * ldcg(r + HD + 1);
      }
    }
    P.out[obase + h * HD + d] = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
  }
}

// ---------------------------------------------------------------------------

static int pick_nsplit(int rows, int n_kv, int max_keys) {
  const int tiles = (max_keys + AT_TILE - 1) / AT_TILE;
  const int ctas = rows * n_kv;
  int ns = (2 * 148 + ctas - 1) / ctas;  // aim for ~2 CTAs per SM
  ns = max(1, min(ns, tiles));
  return ns;
}

size_t attention_workspace_bytes(int rows, int n_heads, int n_kv, int head_dim, int max_keys) {
  const int ns = pick_nsplit(rows, n_kv, max_keys);
  if (ns == 1) return 0;
  const int qpg = n_heads / n_kv;
  size_t part = (size_t)rows * n_kv * ns * qpg * (head_dim + 2) * sizeof(float);
  part = (part + 255) & ~size_t(255);
  return part + (((size_t)rows * n_kv * sizeof(int) + 255) & ~size_t(255));
}

template <int HD, int QPG>
static int attn_launch_t(AttnParams& P, int rows, cudaStream_t st) {
  auto kern = decode_attention_kernel<HD, QPG>;
  const size_t smem = sizeof(AttnSmem<HD, QPG>);
  if (allow_smem(kern, smem) != T2B_OK) return T2B_ERR_LAUNCH;
  return launch_pdl(kern, dim3(P.n_kv, rows, P.nsplit), dim3(AT_THREADS), smem, st, P);
}

// max_keys: upper bound on keys per row (for split selection / workspace).
int attention_launch(AttnParams& P, int rows, int head_dim, int max_keys, void* ws, size_t ws_bytes,
                     cudaStream_t st) {
  if (rows < 1 || P.n_kv < 1 || P.n_heads % P.n_kv) return T2B_ERR_SHAPE;
  const int qpg = P.n_heads / P.n_kv;
  P.nsplit = pick_nsplit(rows, P.n_kv, max_keys);
  const size_t need = attention_workspace_bytes(rows, P.n_heads, P.n_kv, head_dim, max_keys);
  if (ws_bytes < need || (need && !ws)) return T2B_ERR_WORKSPACE;
  if (need) {
    size_t part = (size_t)rows * P.n_kv * P.nsplit * qpg * (head_dim + 2) * sizeof(float);
    part = (part + 255) & ~size_t(255);
    P.ws = reinterpret_cast<float*>(ws);
    P.cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + part);
  }
  P.scale = 1.f / sqrtf((float)head_dim);
#define T2B_ACASE(hd, qpg_)                                          \
  if (head_dim == hd && qpg == qpg_) return attn_launch_t<hd, qpg_>(P, rows, st);
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
