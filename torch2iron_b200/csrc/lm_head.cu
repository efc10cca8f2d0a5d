// bf16 lm_head GEMM with the greedy argmax fused in:
//   logits[m, v] = xn[m, :] . E[v, :]        (model.py:409-420, 477)
//   token[m]     = argmax_v logits[m, v]     (the host argmax of qwen_npu.py:321)
//
// Swap-AB on tcgen05: D[128 vocab rows, BP batch rows] = E_tile . xn^T, both
// operands bf16 K-major in shared memory (2-D TMA boxes of 64 k with the
// 128-byte swizzle = the UMMA canonical layout), fp32 accumulator in TMEM.
// The table and the normalised rows share one 16-bit type: bf16, or fp16
// (the decode engines keep an fp16 copy of the head, exact for every table
// value in fp16 range, so xn enters with 11 significant bits instead of 8).
// Persistent CTAs (one per SM) walk the vocab tiles; the accumulator is
// double-buffered so the drain of one tile overlaps the MMAs of the next.
// Warp roles: 0-3 drain (thread = TMEM lane = vocab row), 4 TMA producer,
// 5 MMA issuer.  Every (logit, vocab index) becomes one 64-bit key
// (order-preserving value bits << 32 | ~index: the larger key is the larger
// logit, ties to the lower index as torch.argmax; NaN counts as -inf).  The
// drain reduces a 32-column slice of the accumulator with a register
// butterfly (transpose-reduce: 31 shuffle + max steps leave lane l with
// column l's max over the warp's 32 rows) and keeps a running max per lane
// across tiles; at the end each CTA folds its warps' keys into the rows'
// global keys with atomicMax, and the last CTA (ticket) writes the token ids
// (and maxima) and re-arms the keys.  Logits are written only when asked for.
// Every wait is time-bounded; a CTA that gives up still takes its ticket.

#include <algorithm>

#include "t2b_common.cuh"
#include "launch.cuh"
#include "tmap.cuh"
#include "tcgen05.cuh"

namespace t2b {

constexpr int LM_THREADS = 192;
constexpr int LM_ROWS = 128;   // vocab rows per tile (MMA M)
constexpr int LM_KB = 64;      // k per TMA box / pipeline stage
constexpr int LM_MAX_WORLD = 8;

struct LmParams {
  CUtensorMap emap;   // E [V][H] bf16, box 64 k x 128 rows
  CUtensorMap xmap;   // xn [M][H] bf16, box 64 k x BP rows (rows >= M read 0)
  int f16;            // table and xn are fp16 (else bf16)
  int M, H, V, n_tiles;
  int32_t* idx;       // [M]
  float* vals;        // [M] maxima (nullable)
  float* logits;      // [M][V] (nullable)
  unsigned long long* keys;  // [M], zero between calls
  int* cnt;           // ticket, zero between calls
  int* err;
  // tensor-parallel vocabulary slice (t2b_lm_head_argmax_tp): row v of this
  // table is vocabulary entry vocab_off + v, and the last CTA merges the
  // greedy pick over the ranks (tp_world > 0)
  int vocab_off;
  int tp_world, tp_rank;
  unsigned long long* gather[LM_MAX_WORLD];  // every rank's [world][M] key buffer (peer-mapped)
  int* flags[LM_MAX_WORLD];                  // every rank's [world] flag words (peer-mapped)
  int* tp_state;                             // this rank's call counter
};

template <int BP>
struct LmGeom {
  static constexpr int E_BYTES = LM_ROWS * LM_KB * 2;   // 16 KB
  static constexpr int X_BYTES = BP * LM_KB * 2;
  static constexpr int STAGE = E_BYTES + X_BYTES;
  static constexpr int STAGES = BP <= 64 ? 6 : (BP <= 128 ? 5 : 4);
  static constexpr int RING = STAGES * STAGE;
  static constexpr uint32_t TMEM_COLS = 2 * BP < 32 ? 32 : 2 * BP;   // two accumulators
  static constexpr int BEST = 4 * (BP < 32 ? 32 : BP) * 8;          // [4 warps][columns] keys
  static constexpr size_t SMEM = 1024 + RING + BEST + 8 * (2 * STAGES + 5) + 64;
};

T2B_DEV unsigned long long lm_key(float v, int i) {
  if (v != v) v = -INFINITY;
  const uint32_t u = __float_as_uint(v);
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)i);
}
T2B_DEV float lm_key_value(unsigned long long k) {
  const uint32_t ord = (uint32_t)(k >> 32);
  return __uint_as_float((ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord);
}
T2B_DEV unsigned long long shfl_xor_u64(unsigned long long x, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)x, m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(x >> 32), m);
  return ((unsigned long long)hi << 32) | lo;
}

template <int BP, bool TP>
__global__ void __launch_bounds__(LM_THREADS, 1) lm_head_argmax_kernel(const __grid_constant__ LmParams p) {
  using G = LmGeom<BP>;
  constexpr int STG = G::STAGES;
  const uint32_t IDESC = p.f16 ? idesc_f16(LM_ROWS, BP) : idesc_bf16(LM_ROWS, BP);
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  constexpr int NCOL = BP < 32 ? 32 : BP;                           // columns drained (padded to 32)
  unsigned long long* bkey = reinterpret_cast<unsigned long long*>(sm + G::RING);   // [4][NCOL]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + G::RING + G::BEST);
  uint64_t* full = bars;
  uint64_t* empty = bars + STG;
  uint64_t* acc_full = bars + 2 * STG;
  uint64_t* acc_empty = bars + 2 * STG + 2;
  uint64_t* mma_done = bars + 2 * STG + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STG + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  int* last_flag = const_cast<int*>(abort_flag) + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KC = p.H / LM_KB;
  if (tid == 0) {
    for (int i = 0; i < STG; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // the first ring fill of E (constant) goes out before the dependency wait
  const int my_chunks = ((p.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * KC;
  const int pre = my_chunks < STG ? my_chunks : STG;
  if (tid == 128) {
    for (int it = 0; it < pre; ++it) {
      mbar_arrive_expect_tx(&full[it], (uint32_t)G::STAGE);
      tma_load_2d(sm + it * G::STAGE, &p.emap, (it % KC) * LM_KB, (blockIdx.x + (it / KC) * gridDim.x) * LM_ROWS,
                  &full[it]);
    }
  }
  grid_dep_wait();
  grid_dep_launch();
  if (warp == 5) {
    tmem_alloc(tmem_slot, G::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 4) {
    // ---- TMA producer: (E box, xn box) per 64-k chunk into the stage ring ----
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < p.n_tiles && !*abort_flag; t += gridDim.x)
        for (int kc = 0; kc < KC; ++kc, ++it) {
          const int s = it % STG;
          if (it >= STG && !mbar_wait_bounded(&empty[s], ((it / STG) - 1) & 1, p.err)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* st = sm + s * G::STAGE;
          if (it >= pre) {
            mbar_arrive_expect_tx(&full[s], (uint32_t)G::STAGE);
            tma_load_2d(st, &p.emap, kc * LM_KB, t * LM_ROWS, &full[s]);
          }
          tma_load_2d(st + G::E_BYTES, &p.xmap, kc * LM_KB, 0, &full[s]);
        }
    }
  } else if (warp == 5) {
    // ---- MMA issuer: D[buf] = E_tile . xn^T over all k chunks ----
    if (lane == 0) {
      int it = 0, tl = 0;
      for (int t = blockIdx.x; t < p.n_tiles && !*abort_flag; t += gridDim.x, ++tl) {
        const int buf = tl & 1;
        if (tl >= 2 && !mbar_wait_bounded(&acc_empty[buf], ((tl >> 1) - 1) & 1, p.err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kc = 0; kc < KC; ++kc, ++it) {
          const int s = it % STG;
          if (!mbar_wait_bounded(&full[s], (it / STG) & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ea = smem_u32(sm + s * G::STAGE), xa = ea + G::E_BYTES;
#pragma unroll
          for (int ks = 0; ks < LM_KB / 16; ++ks)
            mma_ss(tbase + (uint32_t)(buf * BP), sdesc_sw128(ea + ks * 32), sdesc_sw128(xa + ks * 32), IDESC,
                   (kc > 0 || ks > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[buf]);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
      // every MMA issued here has retired before TMEM is released
      mma_commit(mma_done);
      if (!mbar_wait_bounded(mma_done, 0, p.err)) *abort_flag = 1;
    }
  } else {
    // ---- drain: per batch column, max key over this tile's 128 vocab rows ----
    const uint32_t lane_base = tbase + ((uint32_t)(warp * 32) << 16);
    unsigned long long run[NCOL / 32];   // lane l: running max of column 32r + l over this warp's rows
#pragma unroll
    for (int r = 0; r < NCOL / 32; ++r) run[r] = 0ull;
    int tl = 0;
    for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      const bool ok = __all_sync(0xffffffffu, (*abort_flag == 0) && mbar_wait_bounded(&acc_full[buf], (tl >> 1) & 1, p.err));
      if (!ok) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = t * LM_ROWS + warp * 32 + lane;
      const bool live = row < p.V;
#pragma unroll
      for (int r = 0; r < NCOL / 32; ++r) {
        uint32_t v[32];
        if (BP >= 32) {
          tmem_ld32(lane_base + (uint32_t)(buf * BP + r * 32), v);
        } else {
          tmem_ld16(lane_base + (uint32_t)(buf * BP), *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
        }
        tmem_ld_wait();
        unsigned long long c[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int col = r * 32 + e;
          const bool use = live && e < BP;
          const float val = __uint_as_float(v[e < BP ? e : 0]);
          if (p.logits && use && col < p.M) p.logits[(size_t)col * p.V + row] = val;
          c[e] = use ? lm_key(val, TP ? row + p.vocab_off : row) : 0ull;
        }
        // transpose-reduce: after the step with mask s, lane keeps the half of its
        // columns selected by its bit s, maxed with the partner's copy of that half
#pragma unroll
        for (int sh = 16; sh >= 1; sh >>= 1) {
          const bool upper = (lane & sh) != 0;
#pragma unroll
          for (int j = 0; j < sh; ++j) {
            const unsigned long long send = upper ? c[j] : c[j + sh];
            const unsigned long long keep = upper ? c[j + sh] : c[j];
            const unsigned long long recv = shfl_xor_u64(send, sh);
            c[j] = keep > recv ? keep : recv;
          }
        }
        if (c[0] > run[r]) run[r] = c[0];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
#pragma unroll
    for (int r = 0; r < NCOL / 32; ++r) bkey[warp * NCOL + r * 32 + lane] = run[r];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, G::TMEM_COLS);
  }
  // ---- fold the four warps, then this CTA's pick into each row's key ----
  if (!*abort_flag)
    for (int c = tid; c < p.M; c += LM_THREADS) {
      unsigned long long k = bkey[c];
      for (int w = 1; w < 4; ++w) k = bkey[w * NCOL + c] > k ? bkey[w * NCOL + c] : k;
      if (k) atomicMax(p.keys + c, k);
    }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int last = atomicAdd(p.cnt, 1) == (int)gridDim.x - 1;
    if (last) __threadfence();
    *last_flag = last;
  }
  __syncthreads();
  if (!*last_flag) return;
  if constexpr (TP) {
    // Tensor parallel: this rank's best key of every row goes to every rank's
    // gather buffer (slot [tp_rank][m]); after a system-scope fence one lane
    // per rank stores this call's number into that rank's flag word; then,
    // once every rank has signalled the call (time bounded), the largest key
    // over the ranks is the greedy pick of the whole vocabulary row (ties to
    // the lowest vocabulary index, as torch.argmax over the full row).
    volatile int* ok_flag = last_flag + 1;
    const int call = *reinterpret_cast<volatile int*>(p.tp_state) + 1;
    for (int m = tid; m < p.M; m += LM_THREADS) {
      const unsigned long long k = atomicExch(p.keys + m, 0ull);
      for (int q = 0; q < p.tp_world; ++q)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p.gather[q] + (size_t)p.tp_rank * p.M + m), "l"(k)
                     : "memory");
    }
    __syncthreads();
    if (tid < p.tp_world) {
      __threadfence_system();
      asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(p.flags[tid] + p.tp_rank), "r"(call) : "memory");
    }
    if (tid == 0) {
      bool ok = true;
      const uint64_t t0 = globaltimer_ns();
      for (int q = 0; q < p.tp_world && ok; ++q)
        for (;;) {
          int f;
          asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(f) : "l"(p.flags[p.tp_rank] + q) : "memory");
          if (f >= call) break;
          if (globaltimer_ns() - t0 > 500000000ull) {   // 0.5 s: a rank never signalled
            if (p.err) atomicCAS(p.err, 0, T2B_ERR_TIMEOUT);
            ok = false;
            break;
          }
        }
      *ok_flag = ok;
    }
    __syncthreads();
    if (*ok_flag)
      for (int m = tid; m < p.M; m += LM_THREADS) {
        unsigned long long best = 0ull;
        for (int q = 0; q < p.tp_world; ++q) {
          unsigned long long k;
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(k) : "l"(p.gather[p.tp_rank] + (size_t)q * p.M + m)
                       : "memory");
          best = k > best ? k : best;
        }
        p.idx[m] = best ? (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull)) : 0;
        if (p.vals) p.vals[m] = lm_key_value(best);
      }
    __syncthreads();
    if (tid == 0) {
      atomicExch(p.cnt, 0);
      *reinterpret_cast<volatile int*>(p.tp_state) = call;
    }
  } else {
    for (int m = tid; m < p.M; m += LM_THREADS) {
      const unsigned long long k = atomicExch(p.keys + m, 0ull);
      p.idx[m] = k ? (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
      if (p.vals) p.vals[m] = lm_key_value(k);
    }
    if (tid == 0) atomicExch(p.cnt, 0);
  }
}

// ---------------------------------------------------------------------------

static int lm_bp(int M) {
  int bp = 16;
  while (bp < M) bp <<= 1;
  return bp;
}

size_t lm_head_workspace_bytes(int M) { return (((size_t)M * 8 + 255) & ~size_t(255)) + 256; }

template <int BP, bool TP>
static int lm_launch_t(LmParams& p, cudaStream_t st) {
  auto kern = lm_head_argmax_kernel<BP, TP>;
  const size_t smem = LmGeom<BP>::SMEM;
  if (allow_smem(kern, smem) != T2B_OK) return T2B_ERR_LAUNCH;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  const int grid = std::max(1, std::min(sms, p.n_tiles));
  return launch_pdl(kern, dim3(grid), dim3(LM_THREADS), smem, st, p);
}

static int encode_2d(CUtensorMap* m, const void* base, int inner, int outer, int box_outer, bool f16) {
  const EncodeTiledFn encode = encode_tiled();
  if (encode == nullptr) return T2B_ERR_LAUNCH;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  cuuint32_t box[2] = {(cuuint32_t)LM_KB, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                      const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? T2B_OK : T2B_ERR_ARG;
}

struct LmTp {
  int vocab_off, world, rank;
  unsigned long long* const* gather;
  int* const* flags;
  int* state;
};

int lm_head_argmax(const uint16_t* xn, const uint16_t* lm, int dtype, int M, int H, int V, int32_t* idx,
                   float* vals, float* logits, void* ws, size_t ws_bytes, cudaStream_t st, const LmTp* tp = nullptr) {
  if (M < 1 || M > 256 || H < LM_KB || H % LM_KB || V < 1) return T2B_ERR_SHAPE;
  if (dtype != T2B_DTYPE_BF16 && dtype != T2B_DTYPE_F16) return T2B_ERR_ARG;
  if (ws_bytes < lm_head_workspace_bytes(M) || !ws) return T2B_ERR_WORKSPACE;
  LmParams p{};
  const int bp = lm_bp(M);
  p.f16 = dtype == T2B_DTYPE_F16;
  int r = encode_2d(&p.emap, lm, H, V, LM_ROWS, p.f16);
  if (r == T2B_OK) r = encode_2d(&p.xmap, xn, H, M, bp, p.f16);
  if (r != T2B_OK) return r;
  p.M = M;
  p.H = H;
  p.V = V;
  p.n_tiles = (V + LM_ROWS - 1) / LM_ROWS;
  p.idx = idx;
  p.vals = vals;
  p.logits = logits;
  p.keys = reinterpret_cast<unsigned long long*>(ws);
  p.cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + (((size_t)M * 8 + 255) & ~size_t(255)));
  p.err = error_word(st);
  if (tp) {
    p.vocab_off = tp->vocab_off;
    p.tp_world = tp->world;
    p.tp_rank = tp->rank;
    p.tp_state = tp->state;
    for (int q = 0; q < tp->world; ++q) {
      p.gather[q] = tp->gather[q];
      p.flags[q] = tp->flags[q];
    }
  }
  if (tp) {   // the tensor-parallel merge is its own instantiation: the one-GPU kernel is unchanged
    if (bp == 16) return lm_launch_t<16, true>(p, st);
    if (bp == 32) return lm_launch_t<32, true>(p, st);
    if (bp == 64) return lm_launch_t<64, true>(p, st);
    if (bp == 128) return lm_launch_t<128, true>(p, st);
    return lm_launch_t<256, true>(p, st);
  }
  if (bp == 16) return lm_launch_t<16, false>(p, st);
  if (bp == 32) return lm_launch_t<32, false>(p, st);
  if (bp == 64) return lm_launch_t<64, false>(p, st);
  if (bp == 128) return lm_launch_t<128, false>(p, st);
  return lm_launch_t<256, false>(p, st);
}

}  // namespace t2b

using namespace t2b;

extern "C" size_t t2b_lm_head_argmax_workspace_bytes(int M) {
  if (M < 1) return 0;
  return lm_head_workspace_bytes(M);
}

extern "C" int t2b_lm_head_argmax(const uint16_t* xn, const uint16_t* lm_head, int dtype, int M, int H, int V,
                                  int32_t* idx, float* max_logit, float* logits, void* ws, size_t ws_bytes,
                                  void* stream) {
  if (!xn || !lm_head || !idx) return T2B_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(xn) | reinterpret_cast<uintptr_t>(lm_head)) & 15) return T2B_ERR_ALIGN;
  return lm_head_argmax(xn, lm_head, dtype, M, H, V, idx, max_logit, logits, ws, ws_bytes,
                        reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int t2b_lm_head_argmax_tp(const uint16_t* xn, const uint16_t* lm_head_slice, int dtype, int M, int H,
                                     int V_local, int vocab_off, void* const* gather, int32_t* const* flags,
                                     int32_t* state, int rank, int world, int32_t* idx, void* ws, size_t ws_bytes,
                                     void* stream) {
  if (!xn || !lm_head_slice || !idx || !gather || !flags || !state) return T2B_ERR_ARG;
  if (world < 1 || world > LM_MAX_WORLD || rank < 0 || rank >= world || vocab_off < 0) return T2B_ERR_ARG;
  if ((long long)vocab_off + V_local > 0x7FFFFFFFLL) return T2B_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(xn) | reinterpret_cast<uintptr_t>(lm_head_slice)) & 15) return T2B_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(state) & 3) return T2B_ERR_ALIGN;
  for (int q = 0; q < world; ++q) {
    if (!gather[q] || !flags[q]) return T2B_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(gather[q]) & 7) || (reinterpret_cast<uintptr_t>(flags[q]) & 3))
      return T2B_ERR_ALIGN;
  }
  const LmTp tp{vocab_off, world, rank, reinterpret_cast<unsigned long long* const*>(gather), flags, state};
  return lm_head_argmax(xn, lm_head_slice, dtype, M, H, V_local, idx, nullptr, nullptr, ws, ws_bytes,
                        reinterpret_cast<cudaStream_t>(stream), &tp);
}
