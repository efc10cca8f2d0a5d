/*
 * libt2b -- B200 (sm_100a) W4A16 group-128 decode hot path of torch2iron.
 *
 * C ABI.  All tensor pointers are DEVICE pointers owned by the caller; every
 * call is asynchronous on the given stream (cudaStream_t passed as void*) and
 * returns a status code (T2B_OK = 0).  Shape / alignment errors are detected
 * on the host before anything is enqueued.
 *
 * Workspaces: kernels that split a reduction across CTAs take a caller-owned
 * workspace (size from the matching *_workspace_bytes query).  It must be
 * zero-filled once before first use (t2b_workspace_init); the kernels leave
 * its counters re-armed for the next call.  Calls that share one workspace
 * must be ordered on one stream.
 *
 * Ordering: kernels are launched with programmatic dependent launch.  Each
 * kernel may start reading its (constant) weights before the preceding kernel
 * in the stream has finished, so weights written by a kernel (e.g. a repack)
 * must be complete -- synchronize the stream -- before the first call that
 * reads them.
 *
 * Weight layout "T2B" (T2B_WFMT_T2B) for an [N, K] linear, group 128, built
 * by t2b_repack_autogptq (N % 128 == 0, K % 256 == 0):
 *   qw   N*K/2 bytes of 8 KB blocks, block (n/128, k/128) at ((n/128)*(K/128) + k/128) * 8192;
 *        inside it, the 16 bytes of row n%128 for k 32p..32p+31 sit at p*2048 + (n%128)*16,
 *        as 4 words of 8 unsigned nibbles (0..15) with the even k first: nibble
 *        slot t < 4 holds k 8j+2t, slot t >= 4 holds k 8j+2(t-4)+1 (word j)
 *   meta N*K/128 uint32 in 128-entry blocks in the same order: bits 0-15 fp16
 *        scale, bits 16-20 zero point (1..16)
 *   W[n,k] = (q[n,k] - zero[n,k/128]) * scale[n,k/128]
 * Weight layout "QPARAM" (T2B_WFMT_QPARAM) is the reference's runtime row
 * format (src/models/quantized_qwen3/packed_format.py:195-205): row n is
 * K/2 bytes of biased int4 (zero 8) followed by K/128 bf16 scales.
 * Weight layout "Q4NX" (T2B_WFMT_Q4NX) is the fast Qwen3 group-32 format
 * (src/models/fast_qwen3/q4nx_layout.py:30-38,132-174) in T2B blocks: qw as
 * above; meta N*K/32 uint32, block (n/128, k/128) at ((n/128)*(K/128) +
 * k/128) * 512 holding [piece p][row r] words: bits 0-15 bf16 scale, bits
 * 16-31 bf16 zero point of row r, k 32p..32p+31;
 *   W[n,k] = (q[n,k] - zero[n,k/32]) * scale[n,k/32]   (fp32 on the CUDA-core
 *   path, as the reference; rounded once to bf16 on the tcgen05 paths).
 * The fused layer operations take wfmt T2B or Q4NX.
 *
 * Activations of the fused decode layer: the inputs of its linears (the
 * split RMSNorm input xw, the attention output, the SwiGLU output h) are
 * fp16, and the tensor-core paths dequantise the weights to fp16 for them
 * (11-bit significands: 8x finer than bf16, which keeps a 28-layer decoder
 * within the decoder-logit tolerance of the fp32 reference); values beyond
 * fp16 range saturate at +-65504.  The KV cache is bf16, q leaves the qkv
 * operation in fp32 on the decode path (bf16 on the prefill path), the
 * residual stream is fp32.  t2b_w4a16_gemm follows its x_dtype (bf16 or fp16
 * weights).
 */
#ifndef T2B_H
#define T2B_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define T2B_API __attribute__((visibility("default")))
#else
#define T2B_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Status codes.  T2B_ERR_ALIGN: weights, activations, q/out, KV caches, RoPE
 * angles and the fp32 residual stream must be 16-byte aligned, bf16 norm
 * weights and bf16 outputs of the fused layer ops 8-byte aligned (any
 * cudaMalloc / torch allocation is).
 */
#define T2B_OK 0
#define T2B_ERR_SHAPE 1
#define T2B_ERR_ALIGN 2
#define T2B_ERR_LAUNCH 3
#define T2B_ERR_TIMEOUT 4
#define T2B_ERR_WORKSPACE 5
#define T2B_ERR_ARG 6

#define T2B_DTYPE_BF16 0
#define T2B_DTYPE_F16 1
#define T2B_DTYPE_F32 2

#define T2B_WFMT_T2B 0
#define T2B_WFMT_QPARAM 1
#define T2B_WFMT_Q4NX 2

/* Library / ABI version and a short human-readable message for a status. */
T2B_API int t2b_version(void);
T2B_API const char* t2b_status_string(int status);

/*
 * Device status words (int32, device memory, zeroed by the caller): a kernel
 * records T2B_ERR_TIMEOUT in its launch's word when one of its time-bounded
 * waits (0.5 s) gives up -- it then skips its output instead of hanging.
 * A launch on stream s uses the word bound to s by t2b_bind_error_word, else
 * the word the calling host thread set with t2b_set_error_word (NULL: no
 * record).  Bindings are per stream, defaults per host thread, so decoders
 * on different streams or threads keep separate words.  A CUDA graph keeps
 * the word its launches were captured with.  No counterpart in the reference
 * (its NPU runs are synchronous and report through XRT, fusion.py:718-726).
 */
T2B_API int t2b_set_error_word(int32_t* word);
/* Bind `word` to `stream` (NULL removes the binding; the thread default applies again). */
T2B_API int t2b_bind_error_word(void* stream, int32_t* word);
/* The word a launch on `stream` from this thread would record into (host only, no device work). */
T2B_API int t2b_error_word_for_stream(void* stream, int32_t** word);

/*
 * Self-test of that path: a kernel waits (at most limit_us) on a barrier no
 * copy completes and records T2B_ERR_TIMEOUT in `word` (NULL: the stream's
 * word as above); the stream stays usable.
 */
T2B_API int t2b_selftest_bounded_wait(int32_t* word, int limit_us, void* stream);

/* Zero a workspace (cudaMemsetAsync) before its first use. */
T2B_API int t2b_workspace_init(void* workspace, size_t bytes, void* stream);

/*
 * Repack AutoGPTQ-v1 tensors (qweight int32 [K/8,N], qzeros int32 [G,N/8],
 * scales fp16 [G,N]) into the T2B layout.  Source row n lands at destination
 * row  dst_row0 + (n / block_rows) * block_stride + n % block_rows, which
 * builds fused matrices ([q;k;v] rows, or gate/up interleaved in 64-row
 * blocks).  Plain copy: block_rows = N, block_stride = 0.
 * Replaces the offline unpack of packed_format.py:88-146 / the dequant of
 * fast_packed_format.py:132-161 (done once at load, never per token).
 */
T2B_API int t2b_repack_autogptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales_f16, int K, int N,
                        int group_size, uint8_t* qw, uint32_t* meta, int dst_row0, int block_rows,
                        int block_stride, void* stream);

/*
 * y[M,N] = x[M,K] . W^T  (fp32 accumulate of the exact dequantized weights).
 * x / y dtypes: T2B_DTYPE_*.  wfmt T2B (weight = qw, meta; group_size 128),
 * Q4NX (weight = qw, meta; group_size 32) or QPARAM (weight = qparam rows,
 * meta = NULL; group_size 128).  Any M >= 1; M <= 8 per CTA row-block.
 * Replaces W4A16GEMV (src/models/quantized_qwen3/operators/w4a16_gemv/op.py:22-126,
 * kernel.cc:29-133) and the W4A16GEMM family (w4a16_gemm/op.py:22-399).
 */
T2B_API size_t t2b_w4a16_gemm_workspace_bytes(int M, int N, int K);
/*
 * The same GEMM for a tensor-parallel row-parallel linear whose partial is
 * pushed where it is summed: y [M][N] (bf16 or fp32) is written to `y` and,
 * bit for bit, to each of n_peers (<= 7) buffers y_peers[q] of the same
 * layout -- other ranks' memory, peer-mapped -- from the GEMM's epilogue, so
 * the transfer over NVLink overlaps the other tiles' work.  y and the peers
 * 16-byte aligned.  No counterpart in the reference (its NPU path runs on one
 * device).
 */
T2B_API int t2b_w4a16_gemm_push(const void* weight, const uint32_t* meta, int wfmt, const void* x, int x_dtype,
                                void* y, int y_dtype, void* const* y_peers, int n_peers, int M, int N, int K,
                                int group_size, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The launch plan every W4A16 linear of shape [M,N,K] takes (host only, no
 * device work): path 0 = CUDA-core GEMV (rows_per_cta batch rows per CTA,
 * groups_per_cta k-groups of 128 per CTA), 1 = tcgen05 (rows_per_cta = the
 * padded batch tile Bp, groups_per_cta = S), 2 = the large-M tcgen05 kernel
 * of prefill chunks (128 rows x all K groups per work unit); ksplit = k-slices
 * of a 128-row tile (a thread-block cluster when <= 8).  On the tcgen05 path
 * ksplit divides rows_per_cta.  No counterpart in the reference (its tiling is fixed
 * at NPU compile time, w4a16_gemm/design.py); exported so callers and tests
 * can check a shape's decomposition without a GPU.
 */
T2B_API int t2b_linear_plan(int M, int N, int K, int* path, int* rows_per_cta, int* groups_per_cta, int* ksplit);
/* The plan the fused qkv operations (t2b_qkv_norm_rope_kvwrite[_seq]) take for the
 * same shape: on the tcgen05 path each CTA finishes at most 8 batch rows where a
 * grid of about one wave allows it, since the qkv epilogue's per-row work
 * (QK-norm, RoPE, KV write) would otherwise dominate the launch. */
T2B_API int t2b_linear_plan_qkv(int M, int N, int K, int* path, int* rows_per_cta, int* groups_per_cta,
                                int* ksplit);
T2B_API int t2b_w4a16_gemm(const void* weight, const uint32_t* meta, int wfmt, const void* x, int x_dtype, void* y,
                   int y_dtype, int M, int N, int K, int group_size, void* workspace, size_t workspace_bytes,
                   void* stream);

/*
 * t2b_w4a16_gemm without a workspace argument, for callers that cannot
 * allocate device memory (a host runtime that owns the device heap and
 * forbids outside allocations, or a latency-critical thread where
 * cudaMalloc/cudaFree could block).  No counterpart in the reference: it is
 * an addition of this library.  Scratch is a fixed array inside the library
 * (t2b_w4a16_gemm_noalloc_max_workspace() bytes, held on every GPU that loads
 * it).  The call sizes its need from the path it takes (the tcgen05 and
 * large-M paths need none; the CUDA-core split-K path needs its partials and
 * tile counters) and returns T2B_ERR_WORKSPACE for more; every check runs
 * before anything is enqueued.  All calls share that array: calls that may
 * overlap on the GPU race.  The first call on a device resolves the array's
 * address; issue it before any stream capture, and do not use this entry
 * point on a device after cudaDeviceReset.
 */
T2B_API size_t t2b_w4a16_gemm_noalloc_max_workspace(void);
T2B_API int t2b_w4a16_gemm_noalloc(const void* weight, const uint32_t* meta, int wfmt, const void* x, int x_dtype,
                                   void* y, int y_dtype, int M, int N, int K, int group_size, void* stream);

/*
 * Fused attention input block for one decoder layer, one new token per row:
 *   xn = RMSNorm(x) = (x * ln_w) * rsqrt(ssq/H + eps)  (model.py:172-181)
 *   [q;k;v] = xn . Wqkv^T                              (model.py:248-250)
 *   q,k = RMSNorm_head(q|k; q_norm_w|k_norm_w, eps)    (model.py:252-253; skipped if NULL)
 *   q,k = interleaved RoPE(angles[pos[m]])             (model.py:184-196)
 *   q_out[m] = q ; k_cache/v_cache[m][kv][pos[m]] = k, v   (model.py:256-264)
 * The RMSNorm input arrives split: xw fp16 [M,H] = fp16(x * ln_w) (written by
 * the producer of x: t2b_embed_rows / t2b_down_residual) and ssq fp32 [M] =
 * sum of x^2; the row scale is applied after the contraction.
 * angles fp32 [max_ctx, head_dim]; caches bf16 [M][n_kv][max_ctx][head_dim];
 * q_out [M][n_heads*head_dim] of q_dtype: T2B_DTYPE_F32 (the decode layer's
 * input of t2b_decode_attention*) or T2B_DTYPE_BF16; the _seq form writes
 * bf16 q (the prefill attention's input).  ssq_clear (may be NULL): fp32 [M] zeroed.
 * Replaces RMSNorm + W4A16KGroupGEMM(q) + W4A16PairedKGroupGEMM(k,v) +
 * 2x RMSNormRoPE + CopyPresentPacketKV (batch_decode_fused.py:426-474).
 */
T2B_API size_t t2b_qkv_workspace_bytes(int M, int H, int n_heads, int n_kv, int head_dim);
/* Same, with row m writing its K/V into cache sequence row_seq[m] of n_seq
 * (a prefill chunk: rows b*C + i of B sequences, pos[m] = p0 + i) instead of
 * sequence m; caches bf16 [n_seq][n_kv][max_ctx][head_dim].  A row whose
 * sequence is outside [0, n_seq) or position outside [0, max_ctx) writes no
 * cache entry. */
T2B_API int t2b_qkv_norm_rope_kvwrite_seq(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* xw,
                                          const float* ssq, float eps, const uint16_t* q_norm_w,
                                          const uint16_t* k_norm_w, const float* angles, const int32_t* pos,
                                          const int32_t* row_seq, int n_seq, uint16_t* q_out, uint16_t* k_cache,
                                          uint16_t* v_cache, float* ssq_clear, int M, int H, int n_heads, int n_kv,
                                          int head_dim, int max_ctx, void* workspace, size_t workspace_bytes,
                                          void* stream);
T2B_API int t2b_qkv_norm_rope_kvwrite(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* xw, const float* ssq,
                                      float eps, const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                      const float* angles, const int32_t* pos, void* q_out, int q_dtype,
                                      uint16_t* k_cache, uint16_t* v_cache, float* ssq_clear, int M, int H,
                                      int n_heads, int n_kv, int head_dim, int max_ctx, void* workspace,
                                      size_t workspace_bytes, void* stream);

/*
 * GQA decode attention, one query token per row, over the bf16 cache:
 *   out[m, h] = softmax(q[m,h] . K[m, h/qpg, 0..pos[m]]^T / sqrt(hd)) . V  (model.py:266-279)
 * q [M][n_heads*hd] of q_dtype (T2B_DTYPE_BF16, or T2B_DTYPE_F32: q enters
 * the score MMAs as two bf16 terms, 16 significant bits); caches bf16
 * [M][n_kv][max_ctx][hd]; out [M][n_heads*hd] of out_dtype (T2B_DTYPE_BF16,
 * or T2B_DTYPE_F16 for the fused layer's o_proj input).  The probabilities
 * enter the P.V MMAs as two bf16 terms as well.
 * Replaces LlamaChunkedAttention (src/torch2iron/operators/llama_chunked_attention/op.py:21-165).
 */
T2B_API size_t t2b_decode_attention_workspace_bytes(int M, int n_heads, int n_kv, int head_dim, int max_ctx);
T2B_API int t2b_decode_attention(const void* q, int q_dtype, const uint16_t* k_cache, const uint16_t* v_cache,
                         const int32_t* pos, uint16_t* out, int out_dtype, int M, int n_heads, int n_kv, int head_dim,
                         int max_ctx, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Same contract as t2b_decode_attention, for use directly after
 * t2b_qkv_norm_rope_kvwrite on the same stream (the fused decode layer,
 * batch_decode_fused.py:426-484): pos and every cache tile older than the
 * newest key are read while that kernel is still running, so the stream's
 * preceding kernel may write only q and cache key pos[m] of each row.
 */
T2B_API int t2b_decode_attention_after_kvwrite(const void* q, int q_dtype, const uint16_t* k_cache,
                                               const uint16_t* v_cache, const int32_t* pos, uint16_t* out,
                                               int out_dtype, int M, int n_heads, int n_kv, int head_dim, int max_ctx,
                                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * Causal GQA attention of a prefill chunk: C tokens (positions p0..p0+C-1) of
 * each of B sequences, whose K/V rows are already in the cache:
 *   out[b*C + i, h] = softmax(q[b*C + i, h] . K[b, h/qpg, 0..p0+i]^T / sqrt(hd)) . V
 * q bf16, out (out_dtype: bf16 or fp16) [B*C][n_heads*hd]; caches bf16 [B][n_kv][max_ctx][hd];
 * p0 + C <= max_ctx; 64 % (n_heads / n_kv) == 0.  No workspace.
 * Replaces LlamaChunkedPrefillAttention
 * (src/torch2iron/operators/llama_chunked_prefill_attention/op.py:21-197) as
 * driven by prefill_forward_pass (src/models/quantized_qwen3/prefill_runtime.py:95-164).
 */
T2B_API int t2b_prefill_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, uint16_t* out,
                                  int out_dtype, int B, int C, int p0, int n_heads, int n_kv, int head_dim,
                                  int max_ctx, void* stream);

/*
 * Attention over the reference's packet cache
 * [group][chunk][K chunk*hd | V chunk*hd | mask chunk] (bf16), skipping slots
 * whose mask <= 0.5, all packet_seq_len slots scanned.  q, out bf16 [G][qpg][hd].
 * Replaces LlamaChunkedAttention with its own packet argument
 * (llama_chunked_attention/op.py:156-165, attention_reference.py:110-171).
 */
T2B_API int t2b_packet_attention(const uint16_t* q, const uint16_t* packet, uint16_t* out, int n_groups, int q_per_group,
                         int head_dim, int packet_seq_len, int chunk, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * x_resid[M,H] += attn[M,K] . Wo^T ; ssq_out[m] += sum_n x_resid[m,n]^2 ;
 * xw_out = fp16(x_resid * next_norm_w) (both NULL to skip) -- the split
 * RMSNorm input of the following block.
 * ssq_out must be zero before the call (zeroed by the preceding block's ssq_clear).
 * Replaces W4A16KGroupGEMM(o) + ResidualAddRMSNorm (batch_decode_fused.py:485-498).
 */
T2B_API size_t t2b_oproj_residual_workspace_bytes(int M, int H, int K);
T2B_API int t2b_oproj_residual(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* attn, float* x_resid,
                               float* ssq_out, const uint16_t* next_norm_w, uint16_t* xw_out, int M, int H, int K,
                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * h[M,I] = silu(xn . Wg^T) * (xn . Wu^T), xn = RMSNorm(x) given as (xw, ssq)
 * like t2b_qkv_norm_rope_kvwrite.  qw/meta hold gate/up interleaved in
 * 64-row blocks (block b: gate rows 64b..64b+63, then up rows 64b..64b+63).
 * Replaces RMSNorm + W4A16PairedKGroupGEMM(gate,up) + SiLUMul
 * (batch_decode_fused.py:499-506, model.py:215-216).
 */
T2B_API size_t t2b_upgate_swiglu_workspace_bytes(int M, int H, int I);
T2B_API int t2b_upgate_swiglu(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* xw, const float* ssq,
                              float eps, uint16_t* h_out, float* ssq_clear, int M, int H, int I, void* workspace,
                              size_t workspace_bytes, void* stream);

/*
 * x_resid[M,H] += h[M,I] . Wd^T ; ssq_out / xw_out as for t2b_oproj_residual.
 * Replaces W4A16KGroupGEMM(down) + ResidualAddRMSNorm (batch_decode_fused.py:507-530).
 */
T2B_API size_t t2b_down_residual_workspace_bytes(int M, int H, int I);
T2B_API int t2b_down_residual(const uint8_t* qw, const uint32_t* meta, int wfmt, const uint16_t* h, float* x_resid,
                              float* ssq_out, const uint16_t* next_norm_w, uint16_t* xw_out, int M, int H, int I,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * x_resid[m] = float(table[tokens[m]]) ; ssq_out[m] = sum x_resid[m]^2 ;
 * xw_out = fp16(x_resid * norm_w) (both NULL to skip).
 * Replaces the host-side embedding of qwen_npu.py:180-185 (model.py:469).
 */
T2B_API int t2b_embed_rows(const uint16_t* table, const int32_t* tokens, float* x_resid, float* ssq_out,
                           const uint16_t* norm_w, uint16_t* xw_out, int M, int H, int vocab, void* stream);

/*
 * out[m] = RMSNorm(x_resid[m]; ssq, w, eps) -- the final norm (model.py:409,477) --
 * in out_dtype (T2B_DTYPE_BF16, or T2B_DTYPE_F16 for an fp16 lm_head).
 */
T2B_API int t2b_rms_norm_rows(const float* x_resid, const float* ssq, const uint16_t* w, float eps, void* out,
                              int out_dtype, int M, int H, void* stream);

/*
 * Greedy pick: idx[m] = argmax_v logits[m, v] (lowest index on ties), logits
 * dtype T2B_DTYPE_*, row stride ld.  Replaces the host argmax of
 * qwen_npu.py:321 / model.py:492.
 */
/*
 * Tensor-parallel residual step: after the all-reduce of the row-parallel
 * o_proj / down partials y [M][H] (y_dtype bf16 or fp32), x_resid += y, ssq_out[m] =
 * sum_n x_resid[m,n]^2 (overwritten) and xw_out = fp16(x_resid * next_norm_w)
 * (both NULL to skip).  Replaces ResidualAddRMSNorm
 * (src/torch2iron/operators/residual_add_rms_norm/kernel.cc:70-93) where the
 * GEMM before it is split over GPUs (batch_decode_fused.py:485-498, 529-539).
 */
T2B_API int t2b_residual_norm_input(const void* y, int y_dtype, float* x_resid, float* ssq_out,
                                    const uint16_t* next_norm_w, uint16_t* xw_out, int M, int H, void* stream);

/*
 * The same residual step fused with the tensor-parallel all-reduce it
 * follows, over peer memory (NVLink), in place of an NCCL all-reduce and
 * t2b_residual_norm_input.  partials[q] (q < world) is rank q's partial
 * buffer [M][H] (y_dtype bf16 or fp32) as this process maps it (a peer
 * pointer for q != rank); flags[q] is rank q's array of `world` int32 flag
 * words, zeroed before the first call; state is this rank's
 * t2b_tp_allreduce_state_bytes() of zeroed device memory.  Each rank signals
 * its partial complete in every peer's flag words, waits (at most 0.5 s,
 * then T2B_ERR_TIMEOUT in the stream's status word) for every peer's signal
 * of the same call, and sums the partials in rank order in fp32, so every
 * rank computes the same residual.  Every rank must make the same sequence
 * of calls; a partial buffer may be rewritten two calls later at the
 * earliest (alternate two buffers).  No counterpart in the reference (its NPU
 * path runs on one device).
 */
T2B_API size_t t2b_tp_allreduce_state_bytes(void);
T2B_API int t2b_tp_allreduce_residual_norm_input(const void* const* partials, int y_dtype, int32_t* const* flags,
                                                 int32_t* state, int rank, int world, float* x_resid,
                                                 float* ssq_out, const uint16_t* next_w, void* xw_out, int M, int H,
                                                 void* stream);

/*
 * Greedy lm_head: idx[m] = argmax_v (xn[m] . lm_head[v]) over V rows of a bf16
 * [V][H] table (tied embedding or untied head), fp32 accumulation; ties to
 * the lowest index (torch.argmax).  max_logit [M] (may be NULL) receives the
 * maximum, logits fp32 [M][V] (may be NULL) the full rows.  xn [M][H] and the
 * table share dtype: T2B_DTYPE_BF16, or T2B_DTYPE_F16 (the decode engines
 * hold an fp16 copy of the head: xn then keeps 11 significant bits instead
 * of 8); M <= 256, H % 64 == 0.  Workspace: t2b_lm_head_argmax_workspace_bytes(M),
 * zeroed once (re-armed by the kernel).  Replaces the lm_head DenseLinear +
 * host argmax (model.py:409-420, 477; qwen_npu.py:321).
 */
T2B_API size_t t2b_lm_head_argmax_workspace_bytes(int M);
T2B_API int t2b_lm_head_argmax(const uint16_t* xn, const uint16_t* lm_head, int dtype, int M, int H, int V,
                               int32_t* idx, float* max_logit, float* logits, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * The same greedy head on a tensor-parallel vocabulary slice (table rows are
 * vocabulary entries vocab_off .. vocab_off + V_local - 1), with the pick
 * merged over the ranks inside the kernel: its last CTA writes this rank's
 * best (logit, index) key of every row into every rank's gather buffer
 * (gather[q] is rank q's [world][M] uint64 buffer, peer-mapped), signals
 * through flags[q] (rank q's [world] int32 words, zeroed before the first
 * call) and, once every rank signalled the call (at most 0.5 s, then
 * T2B_ERR_TIMEOUT in the stream's status word), writes idx [M] = the
 * vocabulary index of the largest logit of the whole row (ties to the lowest
 * index).  state: this rank's call counter, one zeroed int32.  Every rank
 * makes the same sequence of calls.  Replaces a local argmax, two
 * all-gathers and a host-side merge; no counterpart in the reference (its
 * head runs on one device).
 */
T2B_API int t2b_lm_head_argmax_tp(const uint16_t* xn, const uint16_t* lm_head_slice, int dtype, int M, int H,
                                  int V_local, int vocab_off, void* const* gather, int32_t* const* flags,
                                  int32_t* state, int rank, int world, int32_t* idx, void* workspace,
                                  size_t workspace_bytes, void* stream);

T2B_API size_t t2b_argmax_workspace_bytes(int M, int V);
T2B_API int t2b_argmax_rows(const void* logits, int dtype, int M, int V, int ld, int32_t* idx, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * Standalone reference operators (same argument meaning as the NPU ops):
 *   RMSNormRoPE (src/torch2iron/operators/rms_norm_rope/op.py:19-90):
 *     out[r] = rope(rmsnorm(in[r]; w, eps), angles[r / (rows/angle_rows)]),
 *     rope_mode 0 = interleaved (model.py:184-196), 1 = two halves (kernel.cc:39-67).
 *   ResidualAddRMSNorm (residual_add_rms_norm/op.py:19-85):
 *     x_out = x + update ; norm_out = rmsnorm(x_out per tile_size row; w, eps)
 *   SiLUMul (silu_mul/op.py:20-80): out = silu(a) * b
 *   CopyPresentPacketKV (copy_present_packet_kv/op.py:19-80): present_k/v = k/v and
 *     packet[key/value offset + g*per_group + d] = k/v[g, d], mask slot set to 1.
 * All bf16.
 */
T2B_API int t2b_rms_norm_rope(const uint16_t* in, const uint16_t* w, const uint16_t* angles, uint16_t* out, int rows,
                      int cols, int angle_rows, float eps, int rope_mode, void* stream);
T2B_API int t2b_residual_add_rms_norm(const uint16_t* x, const uint16_t* update, const uint16_t* w, uint16_t* x_out,
                              uint16_t* norm_out, int size, int tile_size, float eps, void* stream);
T2B_API int t2b_silu_mul(const uint16_t* a, const uint16_t* b, uint16_t* out, int size, void* stream);
T2B_API int t2b_copy_present_packet_kv(const uint16_t* k, const uint16_t* v, uint16_t* present_k, uint16_t* present_v,
                               uint16_t* packet, int num_kv_groups, int head_dim, int packet_elements_per_group,
                               int key_packet_offset, int value_packet_offset, int mask_offset, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* T2B_H */
