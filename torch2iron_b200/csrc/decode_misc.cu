// Small kernels around the decode hot path: weight repack (load time),
// embedding gather, final RMSNorm, greedy argmax, and the standalone
// element-wise reference operators.

#include <mutex>
#include <vector>

#include "t2b_common.cuh"
#include "launch.cuh"

namespace t2b {

// ---------------------------------------------------------------------------
// AutoGPTQ-v1 -> T2B tiled layout (see linear_common.cuh).  Word j of piece p
// of row r in block (nt, g) holds the 8 nibbles of AutoGPTQ qweight word
// [g*16 + 4p + j, n] (q[n, k..k+7]) reordered even-k first: nibble slot t
// holds k+2t for t < 4 and k+2(t-4)+1 for t >= 4, so (w >> 4t) & 0x000F000F
// yields the adjacent pair (k+2t, k+2t+1).  Meta packs the fp16 scale with
// zero = stored + 1 (packed_format.py:103-106).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t even_odd_nibbles(uint32_t w) {
  uint32_t r = 0;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    r |= ((w >> (8 * t)) & 0xFu) << (4 * t);            // k = 2t
    r |= ((w >> (8 * t + 4)) & 0xFu) << (4 * (t + 4));  // k = 2t+1
  }
  return r;
}

__device__ __forceinline__ int mapped_row(int n, int dst_row0, int block_rows, int block_stride) {
  return dst_row0 + (n / block_rows) * block_stride + n % block_rows;
}

__global__ void repack_qweight_kernel(const int32_t* __restrict__ qweight, uint32_t* __restrict__ qw, int K8, int N,
                                      int G, int dst_row0, int block_rows, int block_stride) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)K8 * N) return;
  const int k8 = (int)(idx / N), n = (int)(idx - (long long)k8 * N);
  const int dst = mapped_row(n, dst_row0, block_rows, block_stride);
  const int nt = dst >> 7, r = dst & 127;
  const int g = k8 >> 4, pc = (k8 & 15) >> 2, j = k8 & 3;
  const size_t word = ((((size_t)nt * G + g) * 4 + pc) * 128 + r) * 4 + j;
  qw[word] = even_odd_nibbles((uint32_t)qweight[idx]);
}

__global__ void repack_meta_kernel(const int32_t* __restrict__ qzeros, const uint16_t* __restrict__ scales,
                                   uint32_t* __restrict__ meta, int G, int N, int dst_row0, int block_rows,
                                   int block_stride) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= G * N) return;
  const int g = idx / N, n = idx - g * N;
  const uint32_t zw = (uint32_t)qzeros[(size_t)g * (N / 8) + n / 8];
  const uint32_t z = ((zw >> (4 * (n % 8))) & 0xFu) + 1u;
  const int dst = mapped_row(n, dst_row0, block_rows, block_stride);
  meta[((size_t)(dst >> 7) * G + g) * 128 + (dst & 127)] = (uint32_t)scales[(size_t)g * N + n] | (z << 16);
}

int repack_autogptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales, int K, int N, int group,
                    uint8_t* qw, uint32_t* meta, int dst_row0, int block_rows, int block_stride, cudaStream_t st) {
  if (group != 128 || K % 128 || N % 8 || K <= 0 || N <= 0) return T2B_ERR_SHAPE;
  if (block_rows <= 0) return T2B_ERR_ARG;
  if (block_stride == 0) block_stride = block_rows;  // single block: rows map 1:1 (offset dst_row0)
  const int K8 = K / 8, G = K / 128;
  const long long words = (long long)K8 * N;
  repack_qweight_kernel<<<(unsigned)((words + 255) / 256), 256, 0, st>>>(
      qweight, reinterpret_cast<uint32_t*>(qw), K8, N, G, dst_row0, block_rows, block_stride);
  repack_meta_kernel<<<(G * N + 255) / 256, 256, 0, st>>>(qzeros, scales, meta, G, N, dst_row0, block_rows,
                                                          block_stride);
  return cudaGetLastError() == cudaSuccess ? T2B_OK : T2B_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------
// Embedding gather into the fp32 residual stream, with the row's sum of
// squares for the first RMSNorm (model.py:469 then :179).
// ---------------------------------------------------------------------------
__global__ void embed_rows_kernel(const __nv_bfloat16* __restrict__ table, const int* __restrict__ tokens,
                                  float* __restrict__ x, float* __restrict__ ssq,
                                  const __nv_bfloat16* __restrict__ norm_w, __half* __restrict__ xw, int H,
                                  int vocab, int* err) {
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x;
  int tok = tokens[m];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0 && err) atomicCAS(err, 0, T2B_ERR_ARG);
    tok = 0;
  }
  float s = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = __bfloat162float(table[(size_t)tok * H + i]);
    x[(size_t)m * H + i] = v;
    if (xw) xw[(size_t)m * H + i] = __float2half_rn(v * __bfloat162float(norm_w[i]));   // bf16 table * bf16 weight: in range
    s += v * v;
  }
  __shared__ float red[32];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) ssq[m] = v;
  }
}

// out: bf16, or fp16 (F16) for an fp16 head.
template <bool F16>
__global__ void rms_norm_rows_kernel(const float* __restrict__ x, const float* __restrict__ ssq,
                                     const __nv_bfloat16* __restrict__ w, float eps, void* __restrict__ out, int H) {
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x;
  const float r = rsqrtf(ssq[m] / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = (x[(size_t)m * H + i] * r) * __bfloat162float(w[i]);
    if (F16) static_cast<__half*>(out)[(size_t)m * H + i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(out)[(size_t)m * H + i] = __float2bfloat16_rn(v);
  }
}

// Residual add after a tensor-parallel all-reduce (the ResidualAddRMSNorm of
// residual_add_rms_norm/kernel.cc:70-93 in split form): x += y, then the row's
// sum of squares (written, not accumulated) and xw = bf16(x * w) -- the input
// the next linear normalises (model.py:179-181).  One CTA per row, float4.
// y: the all-reduced row-parallel partials, fp32 or bf16 (YBF16).
template <bool YBF16>
__global__ void __launch_bounds__(256) residual_norm_input_kernel(const void* __restrict__ yv, float* __restrict__ x,
                                                                  float* __restrict__ ssq,
                                                                  const __nv_bfloat16* __restrict__ w,
                                                                  __half* __restrict__ xw, int H) {
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x;
  float sq = 0.f;
  for (int i = threadIdx.x * 4; i < H; i += 256 * 4) {
    const size_t o = (size_t)m * H + i;
    const float4 a = *reinterpret_cast<const float4*>(x + o);
    float4 b;
    if (YBF16) {
      const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(yv) + o);
      b = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xffff0000u), __uint_as_float(r.y << 16),
                      __uint_as_float(r.y & 0xffff0000u));
    } else {
      b = *reinterpret_cast<const float4*>(static_cast<const float*>(yv) + o);
    }
    const float4 v = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    *reinterpret_cast<float4*>(x + o) = v;
    sq += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    if (xw) {
      const uint2 wr = *reinterpret_cast<const uint2*>(w + i);
      // fp16 next-norm input, saturating like the fused epilogues
      *reinterpret_cast<uint2*>(xw + o) =
          make_uint2(f16x2_sat(v.x * __uint_as_float(wr.x << 16), v.y * __uint_as_float(wr.x & 0xffff0000u)),
                     f16x2_sat(v.z * __uint_as_float(wr.y << 16), v.w * __uint_as_float(wr.y & 0xffff0000u)));
    }
  }
  sq = warp_sum(sq);
  __shared__ float part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += part[k];
    ssq[m] = t;
  }
}

// Status words: a per-stream binding table (t2b_bind_error_word) and a
// per-host-thread default (t2b_set_error_word).  The table is only touched at
// launch time on the host; a graph captured with a binding keeps the word
// pointer it was captured with.
struct ErrorBinding {
  cudaStream_t stream;
  int* word;
};
static std::mutex g_err_mu;
static std::vector<ErrorBinding> g_err_bindings;
static thread_local int* t_error_word = nullptr;

int* error_word(cudaStream_t st) {
  {
    std::lock_guard<std::mutex> lock(g_err_mu);
    for (const ErrorBinding& b : g_err_bindings)
      if (b.stream == st) return b.word;
  }
  return t_error_word;
}

// Exercises the bounded-wait path end to end without a fault: one thread arms
// an mbarrier for bytes no copy will deliver (nothing is issued, so nothing
// can land after the kernel ends), waits for at most limit_ns, and the
// timeout is recorded in `word` like any kernel's would be.
__global__ void selftest_bounded_wait_kernel(int* word, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  mbar_arrive_expect_tx(&bar, 16);
  mbar_wait_bounded(&bar, 0, word, limit_ns);
}

int residual_norm_input(const void* y, int y_dtype, float* x, float* ssq, const uint16_t* w, uint16_t* xw, int M,
                        int H, cudaStream_t st) {
  if (M < 1 || H < 4 || H % 4) return T2B_ERR_SHAPE;
  const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(w);
  __half* op = reinterpret_cast<__half*>(xw);
  if (y_dtype == T2B_DTYPE_BF16)
    return launch_pdl(residual_norm_input_kernel<true>, dim3(M), dim3(256), 0, st, y, x, ssq, wp, op, H);
  if (y_dtype == T2B_DTYPE_F32)
    return launch_pdl(residual_norm_input_kernel<false>, dim3(M), dim3(256), 0, st, y, x, ssq, wp, op, H);
  return T2B_ERR_ARG;
}

// ---------------------------------------------------------------------------
// Row argmax over a [M, V] logits matrix: grid (chunks, M); each CTA reduces
// an 8192-wide chunk (fp32 rows: 8 float4 loads per thread, all in flight)
// to (value, index), folds it into the row's 64-bit key with atomicMax, and
// the last CTA of the row (ticket) writes the index and re-arms both words.
// Key = order-preserving bits of the value << 32 | ~index, so ties resolve to
// the lowest index (torch.argmax); NaN entries are skipped.
// ---------------------------------------------------------------------------
constexpr int AM_THREADS = 256;
constexpr int AM_CHUNK = 8192;

T2B_DEV void argmax_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i) || (v != v && v2 == v2)) {
    v = v2;
    i = i2;
  }
}

T2B_DEV unsigned long long argmax_key(float v, int i) {
  const uint32_t u = __float_as_uint(v);
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)i);
}

template <bool F32X4>
__global__ void __launch_bounds__(AM_THREADS) argmax_rows_kernel(const void* __restrict__ logits, int dtype, int V,
                                                                 int ld, int* __restrict__ idx,
                                                                 unsigned long long* __restrict__ keys,
                                                                 int* __restrict__ cnt) {
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.y, c = blockIdx.x, nch = gridDim.x;
  const int v0 = c * AM_CHUNK, v1 = min(V, v0 + AM_CHUNK);
  float best = -INFINITY;
  int bi = 0x7fffffff;
  if (F32X4) {
    const float* row = reinterpret_cast<const float*>(logits) + (size_t)m * ld;
    float4 x[AM_CHUNK / (4 * AM_THREADS)];
#pragma unroll
    for (int u = 0; u < AM_CHUNK / (4 * AM_THREADS); ++u) {
      const int v = v0 + (u * AM_THREADS + (int)threadIdx.x) * 4;
      x[u] = v < v1 ? __ldg(reinterpret_cast<const float4*>(row + v)) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
#pragma unroll
    for (int u = 0; u < AM_CHUNK / (4 * AM_THREADS); ++u) {
      const int v = v0 + (u * AM_THREADS + (int)threadIdx.x) * 4;
      if (v < v1) {
        argmax_merge(best, bi, x[u].x, v);
        argmax_merge(best, bi, x[u].y, v + 1);
        argmax_merge(best, bi, x[u].z, v + 2);
        argmax_merge(best, bi, x[u].w, v + 3);
      }
    }
  } else {
    for (int v = v0 + threadIdx.x; v < v1; v += AM_THREADS)
      argmax_merge(best, bi, load_act(logits, dtype, (size_t)m * ld + v), v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(best, bi, v2, i2);
  }
  __shared__ float sv[AM_THREADS / 32];
  __shared__ int si[AM_THREADS / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 1; w < AM_THREADS / 32; ++w) argmax_merge(best, bi, sv[w], si[w]);
  if (nch == 1) {
    idx[m] = bi;
    return;
  }
  atomicMax(keys + m, argmax_key(best, bi));
  __threadfence();
  if (atomicAdd(cnt + m, 1) == nch - 1) {
    const unsigned long long k = atomicExch(keys + m, 0ull);
    idx[m] = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    atomicExch(cnt + m, 0);
  }
}

size_t argmax_workspace_bytes(int M, int V) {
  const int nch = (V + AM_CHUNK - 1) / AM_CHUNK;
  if (nch == 1) return 0;
  return (((size_t)M * 8 + 255) & ~size_t(255)) + (((size_t)M * 4 + 255) & ~size_t(255));
}

int argmax_rows(const void* logits, int dtype, int M, int V, int ld, int* idx, void* ws, size_t ws_bytes,
                cudaStream_t st) {
  if (M < 1 || V < 1 || ld < V) return T2B_ERR_SHAPE;
  const int nch = (V + AM_CHUNK - 1) / AM_CHUNK;
  const size_t need = argmax_workspace_bytes(M, V);
  if (ws_bytes < need || (need && !ws)) return T2B_ERR_WORKSPACE;
  unsigned long long* keys = nullptr;
  int* cnt = nullptr;
  if (need) {
    keys = reinterpret_cast<unsigned long long*>(ws);
    cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + (((size_t)M * 8 + 255) & ~size_t(255)));
  }
  const bool x4 = dtype == T2B_DTYPE_F32 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  if (x4)
    return launch_pdl(argmax_rows_kernel<true>, dim3(nch, M), dim3(AM_THREADS), 0, st, logits, dtype, V, ld, idx,
                      keys, cnt);
  return launch_pdl(argmax_rows_kernel<false>, dim3(nch, M), dim3(AM_THREADS), 0, st, logits, dtype, V, ld, idx, keys,
                    cnt);
}

int embed_rows(const uint16_t* table, const int* tokens, float* x, float* ssq, const uint16_t* norm_w, uint16_t* xw,
               int M, int H, int vocab, int* err, cudaStream_t st) {
  if (M < 1 || H < 1) return T2B_ERR_SHAPE;
  const __nv_bfloat16* t = reinterpret_cast<const __nv_bfloat16*>(table);
  const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(norm_w);
  __half* o = reinterpret_cast<__half*>(xw);
  return launch_pdl(embed_rows_kernel, dim3(M), dim3(256), 0, st, t, tokens, x, ssq, w, o, H, vocab, err);
}

int rms_norm_rows(const float* x, const float* ssq, const uint16_t* w, float eps, void* out, int out_dtype, int M,
                  int H, cudaStream_t st) {
  if (M < 1 || H < 1) return T2B_ERR_SHAPE;
  const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(w);
  if (out_dtype == T2B_DTYPE_F16)
    return launch_pdl(rms_norm_rows_kernel<true>, dim3(M), dim3(256), 0, st, x, ssq, wp, eps, out, H);
  if (out_dtype == T2B_DTYPE_BF16)
    return launch_pdl(rms_norm_rows_kernel<false>, dim3(M), dim3(256), 0, st, x, ssq, wp, eps, out, H);
  return T2B_ERR_ARG;
}

// ---------------------------------------------------------------------------
// Standalone reference operators (bf16 in / out).
// ---------------------------------------------------------------------------

// One warp per row: weighted RMSNorm over `cols`, then RoPE with the angle row
// r / (rows / angle_rows).  rope_mode 0 = interleaved pairs (model.py:184-196),
// 1 = two halves (rms_norm_rope/kernel.cc:39-67).  The normalised row is
// rounded to bf16 before the rotation, as the NPU operator stores it.
__global__ void rms_norm_rope_kernel(const __nv_bfloat16* __restrict__ in, const __nv_bfloat16* __restrict__ w,
                                     const __nv_bfloat16* __restrict__ ang, __nv_bfloat16* __restrict__ out, int rows,
                                     int cols, int rows_per_angle, float eps, int mode) {
  grid_dep_wait();
  grid_dep_launch();
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* x = in + (size_t)r * cols;
  float ss = 0.f;
  for (int d = lane; d < cols; d += 32) {
    const float v = __bfloat162float(x[d]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)cols + eps);
  const __nv_bfloat16* a = ang + (size_t)(r / rows_per_angle) * cols;
  const int half = cols / 2;
  for (int d = lane; d < cols; d += 32) {
    int pd;
    float c, s;
    if (mode == 0) {
      pd = d ^ 1;
      c = __bfloat162float(a[d & ~1]);
      s = __bfloat162float(a[(d & ~1) + 1]);
    } else {
      const int i = d < half ? d : d - half;
      pd = d < half ? d + half : d - half;
      c = __bfloat162float(a[2 * i]);
      s = __bfloat162float(a[2 * i + 1]);
    }
    const float xd = round_bf16((__bfloat162float(x[d]) * rs) * __bfloat162float(w[d]));
    const float xp = round_bf16((__bfloat162float(x[pd]) * rs) * __bfloat162float(w[pd]));
    const bool first = (mode == 0) ? ((d & 1) == 0) : (d < half);
    out[(size_t)r * cols + d] = __float2bfloat16_rn(first ? (xd * c - xp * s) : (xd * c + xp * s));
  }
}

// One CTA per tile_size row: x_out = x + update (bf16), norm_out = rmsnorm(x_out).
__global__ void residual_add_rms_norm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ u,
                                             const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ xo,
                                             __nv_bfloat16* __restrict__ no, int tile, float eps) {
  grid_dep_wait();
  grid_dep_launch();
  const size_t base = (size_t)blockIdx.x * tile;
  float ss = 0.f;
  for (int i = threadIdx.x; i < tile; i += blockDim.x) {
    const float v = round_bf16(__bfloat162float(x[base + i]) + __bfloat162float(u[base + i]));
    xo[base + i] = __float2bfloat16_rn(v);
    ss += v * v;
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rs = rsqrtf(red[0] / (float)tile + eps);
  for (int i = threadIdx.x; i < tile; i += blockDim.x) {
    const float v = round_bf16(__bfloat162float(x[base + i]) + __bfloat162float(u[base + i]));
    no[base + i] = __float2bfloat16_rn((v * rs) * __bfloat162float(w[i]));
  }
}

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
                                __nv_bfloat16* __restrict__ o, int n) {
  grid_dep_wait();
  grid_dep_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float g = __bfloat162float(a[i]);
  o[i] = __float2bfloat16_rn(g / (1.f + expf(-g)) * __bfloat162float(b[i]));
}

__global__ void copy_present_packet_kv_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                              __nv_bfloat16* pk, __nv_bfloat16* pv, __nv_bfloat16* packet, int groups,
                                              int hd, long long per_group, long long koff, long long voff,
                                              long long moff) {
  grid_dep_wait();
  grid_dep_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= groups * hd) return;
  const int g = i / hd, d = i - g * hd;
  const __nv_bfloat16 kv = k[i], vv = v[i];
  if (pk) pk[i] = kv;
  if (pv) pv[i] = vv;
  packet[g * per_group + koff + d] = kv;
  packet[g * per_group + voff + d] = vv;
  if (moff >= 0 && d == 0) packet[g * per_group + moff] = __float2bfloat16_rn(1.f);
}

int rms_norm_rope(const uint16_t* in, const uint16_t* w, const uint16_t* ang, uint16_t* out, int rows, int cols,
                  int angle_rows, float eps, int mode, cudaStream_t st) {
  if (rows < 1 || cols < 2 || cols % 2 || angle_rows < 1 || rows % angle_rows || (mode != 0 && mode != 1))
    return T2B_ERR_SHAPE;
  const int rpa = rows / angle_rows;
  auto c = [](const uint16_t* p) { return reinterpret_cast<const __nv_bfloat16*>(p); };
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
  const __nv_bfloat16* a0 = c(in);
  const __nv_bfloat16* a1 = c(w);
  const __nv_bfloat16* a2 = c(ang);
  return launch_pdl(rms_norm_rope_kernel, dim3((rows + 7) / 8), dim3(256), 0, st, a0, a1, a2, o, rows, cols, rpa, eps,
                    mode);
}

int residual_add_rms_norm(const uint16_t* x, const uint16_t* u, const uint16_t* w, uint16_t* xo, uint16_t* no,
                          int size, int tile, float eps, cudaStream_t st) {
  if (size < 1 || tile < 1 || size % tile) return T2B_ERR_SHAPE;
  auto c = [](const uint16_t* p) { return reinterpret_cast<const __nv_bfloat16*>(p); };
  auto m = [](uint16_t* p) { return reinterpret_cast<__nv_bfloat16*>(p); };
  const __nv_bfloat16 *a0 = c(x), *a1 = c(u), *a2 = c(w);
  __nv_bfloat16 *o0 = m(xo), *o1 = m(no);
  return launch_pdl(residual_add_rms_norm_kernel, dim3(size / tile), dim3(256), 0, st, a0, a1, a2, o0, o1, tile, eps);
}

int silu_mul(const uint16_t* a, const uint16_t* b, uint16_t* o, int n, cudaStream_t st) {
  if (n < 1) return T2B_ERR_SHAPE;
  const __nv_bfloat16* a0 = reinterpret_cast<const __nv_bfloat16*>(a);
  const __nv_bfloat16* a1 = reinterpret_cast<const __nv_bfloat16*>(b);
  __nv_bfloat16* o0 = reinterpret_cast<__nv_bfloat16*>(o);
  return launch_pdl(silu_mul_kernel, dim3((n + 255) / 256), dim3(256), 0, st, a0, a1, o0, n);
}

int copy_present_packet_kv(const uint16_t* k, const uint16_t* v, uint16_t* pk, uint16_t* pv, uint16_t* packet,
                           int groups, int hd, int per_group, int koff, int voff, int moff, cudaStream_t st) {
  if (groups < 1 || hd < 1 || per_group < 1) return T2B_ERR_SHAPE;
  const __nv_bfloat16* a0 = reinterpret_cast<const __nv_bfloat16*>(k);
  const __nv_bfloat16* a1 = reinterpret_cast<const __nv_bfloat16*>(v);
  __nv_bfloat16* o0 = reinterpret_cast<__nv_bfloat16*>(pk);
  __nv_bfloat16* o1 = reinterpret_cast<__nv_bfloat16*>(pv);
  __nv_bfloat16* o2 = reinterpret_cast<__nv_bfloat16*>(packet);
  long long pg = per_group, ko = koff, vo = voff, mo = moff;
  return launch_pdl(copy_present_packet_kv_kernel, dim3((groups * hd + 255) / 256), dim3(256), 0, st, a0, a1, o0, o1,
                    o2, groups, hd, pg, ko, vo, mo);
}

}  // namespace t2b

// ===========================================================================
// C ABI
// ===========================================================================
using namespace t2b;

static inline cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" int t2b_version(void) { return 1; }

extern "C" const char* t2b_status_string(int status) {
  switch (status) {
    case T2B_OK: return "ok";
    case T2B_ERR_SHAPE: return "unsupported or inconsistent shape";
    case T2B_ERR_ALIGN: return "pointer misaligned for the kernel's vector loads";
    case T2B_ERR_LAUNCH: return "CUDA launch failed";
    case T2B_ERR_TIMEOUT: return "device-side wait gave up (bounded spin expired)";
    case T2B_ERR_WORKSPACE: return "workspace missing or too small";
    case T2B_ERR_ARG: return "invalid argument";
    default: return "unknown status";
  }
}

extern "C" int t2b_workspace_init(void* ws, size_t bytes, void* stream) {
  if (!bytes) return T2B_OK;
  if (!ws) return T2B_ERR_ARG;
  return cudaMemsetAsync(ws, 0, bytes, S_(stream)) == cudaSuccess ? T2B_OK : T2B_ERR_LAUNCH;
}

extern "C" int t2b_repack_autogptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales_f16, int K,
                                   int N, int group_size, uint8_t* qw, uint32_t* meta, int dst_row0, int block_rows,
                                   int block_stride, void* stream) {
  if (!qweight || !qzeros || !scales_f16 || !qw || !meta) return T2B_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(qw) & 3) return T2B_ERR_ALIGN;
  return repack_autogptq(qweight, qzeros, scales_f16, K, N, group_size, qw, meta, dst_row0, block_rows, block_stride,
                         S_(stream));
}

extern "C" int t2b_embed_rows(const uint16_t* table, const int32_t* tokens, float* x_resid, float* ssq_out,
                              const uint16_t* norm_w, uint16_t* xw_out, int M, int H, int vocab, void* stream) {
  if (!table || !tokens || !x_resid || !ssq_out) return T2B_ERR_ARG;
  if ((norm_w == nullptr) != (xw_out == nullptr)) return T2B_ERR_ARG;
  return embed_rows(table, tokens, x_resid, ssq_out, norm_w, xw_out, M, H, vocab, nullptr, S_(stream));
}

extern "C" int t2b_rms_norm_rows(const float* x_resid, const float* ssq, const uint16_t* w, float eps, void* out,
                                 int out_dtype, int M, int H, void* stream) {
  if (!x_resid || !ssq || !w || !out) return T2B_ERR_ARG;
  return rms_norm_rows(x_resid, ssq, w, eps, out, out_dtype, M, H, S_(stream));
}

extern "C" int t2b_set_error_word(int32_t* word) {
  t_error_word = word;
  return T2B_OK;
}

extern "C" int t2b_bind_error_word(void* stream, int32_t* word) {
  const cudaStream_t st = S_(stream);
  std::lock_guard<std::mutex> lock(g_err_mu);
  for (size_t i = 0; i < g_err_bindings.size(); ++i) {
    if (g_err_bindings[i].stream != st) continue;
    if (word) {
      g_err_bindings[i].word = word;
    } else {
      g_err_bindings.erase(g_err_bindings.begin() + (long)i);
    }
    return T2B_OK;
  }
  if (word) g_err_bindings.push_back(ErrorBinding{st, word});
  return T2B_OK;
}

extern "C" int t2b_error_word_for_stream(void* stream, int32_t** word) {
  if (!word) return T2B_ERR_ARG;
  *word = error_word(S_(stream));
  return T2B_OK;
}

extern "C" int t2b_selftest_bounded_wait(int32_t* word, int limit_us, void* stream) {
  if (!word) word = error_word(S_(stream));   // the stream's (or thread's) status word
  if (!word || limit_us < 1 || limit_us > 1000000) return T2B_ERR_ARG;
  selftest_bounded_wait_kernel<<<1, 32, 0, S_(stream)>>>(word, 1000ull * (unsigned long long)limit_us);
  return cudaGetLastError() == cudaSuccess ? T2B_OK : T2B_ERR_LAUNCH;
}

extern "C" int t2b_residual_norm_input(const void* y, int y_dtype, float* x_resid, float* ssq_out,
                                       const uint16_t* next_norm_w, uint16_t* xw_out, int M, int H, void* stream) {
  if (!y || !x_resid || !ssq_out) return T2B_ERR_ARG;
  if ((next_norm_w == nullptr) != (xw_out == nullptr)) return T2B_ERR_ARG;
  if (y_dtype != T2B_DTYPE_BF16 && y_dtype != T2B_DTYPE_F32) return T2B_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(y) & (y_dtype == T2B_DTYPE_BF16 ? 7 : 15)) ||
      (reinterpret_cast<uintptr_t>(x_resid) & 15))
    return T2B_ERR_ALIGN;
  if (xw_out && ((reinterpret_cast<uintptr_t>(xw_out) | reinterpret_cast<uintptr_t>(next_norm_w)) & 7))
    return T2B_ERR_ALIGN;
  return residual_norm_input(y, y_dtype, x_resid, ssq_out, next_norm_w, xw_out, M, H, S_(stream));
}

extern "C" size_t t2b_argmax_workspace_bytes(int M, int V) {
  if (M < 1 || V < 1) return 0;
  return argmax_workspace_bytes(M, V);
}

extern "C" int t2b_argmax_rows(const void* logits, int dtype, int M, int V, int ld, int32_t* idx, void* ws,
                               size_t ws_bytes, void* stream) {
  if (!logits || !idx || dtype < 0 || dtype > 2) return T2B_ERR_ARG;
  return argmax_rows(logits, dtype, M, V, ld, idx, ws, ws_bytes, S_(stream));
}

extern "C" int t2b_rms_norm_rope(const uint16_t* in, const uint16_t* w, const uint16_t* angles, uint16_t* out,
                                 int rows, int cols, int angle_rows, float eps, int rope_mode, void* stream) {
  if (!in || !w || !angles || !out) return T2B_ERR_ARG;
  if (!(eps > 0.f)) return T2B_ERR_ARG;
  return rms_norm_rope(in, w, angles, out, rows, cols, angle_rows, eps, rope_mode, S_(stream));
}

extern "C" int t2b_residual_add_rms_norm(const uint16_t* x, const uint16_t* update, const uint16_t* w,
                                         uint16_t* x_out, uint16_t* norm_out, int size, int tile_size, float eps,
                                         void* stream) {
  if (!x || !update || !w || !x_out || !norm_out) return T2B_ERR_ARG;
  if (!(eps > 0.f)) return T2B_ERR_ARG;
  return residual_add_rms_norm(x, update, w, x_out, norm_out, size, tile_size, eps, S_(stream));
}

extern "C" int t2b_silu_mul(const uint16_t* a, const uint16_t* b, uint16_t* out, int size, void* stream) {
  if (!a || !b || !out) return T2B_ERR_ARG;
  return silu_mul(a, b, out, size, S_(stream));
}

extern "C" int t2b_copy_present_packet_kv(const uint16_t* k, const uint16_t* v, uint16_t* present_k,
                                          uint16_t* present_v, uint16_t* packet, int num_kv_groups, int head_dim,
                                          int packet_elements_per_group, int key_packet_offset,
                                          int value_packet_offset, int mask_offset, void* stream) {
  if (!k || !v || !packet) return T2B_ERR_ARG;
  return copy_present_packet_kv(k, v, present_k, present_v, packet, num_kv_groups, head_dim,
                                packet_elements_per_group, key_packet_offset, value_packet_offset, mask_offset,
                                S_(stream));
}
