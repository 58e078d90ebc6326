/*
 * decodek: the C ABI of the B200 (sm_100a) decode kernels.
 *
 * Every entry point takes plain device pointers, sizes in elements, row strides in elements and
 * a CUDA stream, and returns an int status (DK_OK = 0, negative on error, with the message in
 * dk_last_error()). Apart from the tensor-parallel set-up calls (dk_tp_buffer_*, which allocate and
 * synchronize once, before any capture), nothing allocates device memory, synchronizes or reads
 * device memory from the host, so every launch can be captured in a CUDA graph. Kernels are queued on `stream` and
 * report launch errors through the status; asynchronous device-side conditions (a bounded wait
 * that gave up) are recorded in a per-device error word read with dk_device_error().
 *
 * fp16 tensors are passed as `const void*` (IEEE binary16), e4m3 tensors as `uint8_t` bytes.
 * Layouts are the reference's (Charlie-Gzz/llm-decode-kernels):
 *   qweight  int32 [K/8, N], N contiguous; value i of a word is bits 4i..4i+3  (kernels/quant.py:4-8)
 *   scales, zeros  fp16 [K/group, N]                                           (kernels/quant.py:8)
 *   fp8 weight  e4m3 [K, N], N contiguous; scale fp16 [N]                        (kernels/fp8.py:3-6)
 */
#ifndef DECODEK_H_
#define DECODEK_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* dk_stream_t; /* same type as cudaStream_t */

#define DK_ABI_VERSION 6

/* status codes */
#define DK_OK 0
#define DK_ERR_INVALID (-1)     /* shape, size or argument outside the contract */
#define DK_ERR_ALIGN (-2)       /* pointer or stride alignment the kernel cannot handle */
#define DK_ERR_UNSUPPORTED (-3) /* valid request this build has no kernel for */
#define DK_ERR_CUDA (-4)        /* a CUDA runtime call failed (message has the CUDA error) */

/* device error codes (dk_device_error) */
#define DK_DEVERR_NONE 0
#define DK_DEVERR_WAIT_FULL 1  /* a consumer gave up waiting for a stage's copies */
#define DK_DEVERR_WAIT_EMPTY 2 /* the producer gave up waiting for a stage to be released */
#define DK_DEVERR_BAD_POSITION 3 /* decode attention / lm_head greedy: position outside the cache or history (no write done) */
#define DK_DEVERR_TP_WAIT 4      /* a fused-allreduce CTA gave up waiting for a peer's partial sums */
#define DK_DEVERR_STEP_WAIT 5    /* decode step: a CTA gave up waiting for another CTA or for its weight ring */
#define DK_DEVERR_BAD_TOKEN 6    /* decode step / embed tokens: a token id outside [0, vocab) (row 0 used instead) */

/* dk_matmul_config.flags */
#define DK_FLAG_STATIC_WEIGHTS 1 /* weights are not written by any kernel still in flight on the
                                    stream: the kernel may prefetch them before waiting for the
                                    previous kernel (programmatic dependent launch) */
#define DK_FLAG_GENERIC 2        /* force the simple (any alignment) kernel; for tests */
#define DK_FLAG_EXACT_DEQUANT 4  /* round every dequantized weight to fp16 exactly like the
                                    reference's dequantize-then-matmul ((q - z) * s in fp16) instead
                                    of the default factored form s * sum(x * (q - z)) in fp32 (the
                                    reference's FACTORED path, kernels/w4a16.py:116-119) */
#define DK_FLAG_GEMV 8           /* run M in launches of up to 16 rows of the decode GEMV even where
                                    the tensor-core GEMM would take the shape (M >= 128, N >= 128);
                                    for tests and comparisons */

#define DK_MAX_L2_PREFETCH 6

/* Optional per-call tuning; zero fields mean "choose automatically".
 * l2_prefetch: byte ranges of device memory (typically the weights of the launch after next) that
 * the launch asks the L2 cache to fetch while it runs (cp.async.bulk.prefetch.L2), so that the later
 * launch reads them from L2 instead of HBM. A hint only: it changes no result, and ranges are
 * trimmed inward to 16-byte boundaries. No reference counterpart (the reference's Triton launches
 * have no cross-launch prefetch). */
typedef struct dk_matmul_config {
  int32_t split_k;    /* K slices reduced inside a thread-block cluster (1..8; clamped to what K allows) */
  int32_t block_n;    /* output columns per CTA tile: 32, 64, 128 or 256 (other values: automatic) */
  int32_t flags;      /* DK_FLAG_* */
  int32_t n_prefetch; /* valid entries of l2_prefetch_ptr / l2_prefetch_bytes (0..DK_MAX_L2_PREFETCH) */
  const void* l2_prefetch_ptr[DK_MAX_L2_PREFETCH];
  uint64_t l2_prefetch_bytes[DK_MAX_L2_PREFETCH];
} dk_matmul_config;

/* ---- library ---------------------------------------------------------------------------- */
int dk_abi_version(void);
/* sizeof(dk_matmul_config) in this build, for FFI bindings that lay the struct out themselves. */
int dk_matmul_config_size(void);
/* Message of the last failing call on this host thread ("" if none). */
const char* dk_last_error(void);
/* Device error word of the current device (DK_DEVERR_*); reading it synchronizes the device.
 * No reference counterpart: the reference's kernels have no bounded waits. */
int dk_device_error(int32_t* code);
int dk_clear_device_error(void);
/* Programmatic dependent launch on (1, default) or off (0) for all later launches. */
int dk_set_pdl(int32_t enabled);

/* ---- int4 format: kernels/quant.py ------------------------------------------------------- */
/* pack_int4 (kernels/quant.py:20-28): q int32 [K, N] -> packed int32 [K/8, N]. K % 8 == 0. */
int dk_pack_int4(const int32_t* q, int32_t* packed, int64_t K, int64_t N, dk_stream_t stream);
/* unpack_int4 (kernels/quant.py:31-35): packed int32 [K/8, N] -> q int32 [K, N] in 0..15. */
int dk_unpack_int4(const int32_t* packed, int32_t* q, int64_t K, int64_t N, dk_stream_t stream);
/* quantize_rtn (kernels/quant.py:38-49): w fp16 [N, K] (row stride ldw) -> qweight, scales,
 * zeros. Bit-exact with the reference. K % group_size == 0, group_size % 8 == 0. */
int dk_quantize_rtn(const void* w, int64_t ldw, int32_t* qweight, void* scales, void* zeros,
                    int64_t N, int64_t K, int64_t group_size, dk_stream_t stream);
/* dequantize_ref (kernels/reference.py:27-36): -> fp16 [N, K], (fp16(q) - z) * s in fp16. */
int dk_dequantize_int4(const int32_t* qweight, const void* scales, const void* zeros, void* w,
                       int64_t N, int64_t K, int64_t group_size, dk_stream_t stream);

/* ---- W4A16 matmul: kernels/w4a16.py, kernels/cuda/w4a16_decode.cu ---------------------- */
/* w4a16_matmul (kernels/w4a16.py:301-330) and w4a16_decode (kernels/cuda/w4a16_decode.cu:136-181):
 * y[M, N] fp16 = x[M, K] fp16 @ dequant(W).T (+ bias[N]), fp32 accumulation.
 * x rows have stride ldx, y rows stride ldy (elements). bias may be NULL. cfg may be NULL.
 * Dispatch by rows (fast-path shapes: N % 8 == 0, group_size 128, 16-byte aligned operands):
 * up to 8 rows, or up to 16 with K < 4096: the decode GEMV, up to 16 rows per launch (fewer when a long
 * K slice leaves no tile for the staged rows); 9-16 rows with K >= 4096 and 17-127 rows, N >= 128: the
 * tcgen05 small-M kernel;
 * M >= 128 and N >= 128: the tcgen05 tensor-core GEMM (kernels/w4a16.py:31-97). The tcgen05 kernels
 * round every dequantized weight to fp16 like the reference's dequantize-then-matmul. DK_FLAG_GEMV
 * keeps any M on the decode GEMV. Other shapes run a one-thread-per-output kernel. */
int dk_w4a16_matmul(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                    const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M,
                    int64_t N, int64_t K, int64_t group_size, const dk_matmul_config* cfg,
                    dk_stream_t stream);

/* gate_up projection fused with SwiGLU (kernels/e2e/model.py:247 with kernels/swiglu.py:56-61):
 * qweight/scales/zeros hold the fused [gate; up] weight with 2I output columns; the output
 * y[M, I] = fp16(silu(fp16(g))) * fp16(u) for g, u = the gate and up halves of x @ dequant(W).T
 * (+ bias[2I]) - the same roundings as the two separate ops. Needs I % 32 == 0, group_size 128
 * and 16-byte aligned operands (DK_ERR_UNSUPPORTED otherwise: run the two ops instead). */
int dk_w4a16_swiglu(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                    const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M,
                    int64_t I, int64_t K, int64_t group_size, const dk_matmul_config* cfg,
                    dk_stream_t stream);

/* Fused residual add + RMSNorm + W4A16 projection (kernels/e2e/model.py:231-235 and 246-247 in one
 * kernel): h = x (+ residual, fp16 add, written to residual_out when residual != NULL);
 * xn = norm_weight * fp16(h * rsqrt(mean(h^2) + eps)) (the same roundings as dk_rmsnorm); then
 * y = xn @ dequant(W).T (+ bias), or with swiglu != 0 the gate_up + SwiGLU output of
 * dk_w4a16_swiglu (N = 2I columns of W, y is [M, I]). residual_out must not alias x or residual.
 * Needs the fast-path conditions of dk_w4a16_swiglu / dk_w4a16_matmul (DK_ERR_UNSUPPORTED
 * otherwise: run dk_rmsnorm then the projection). */
int dk_w4a16_rmsnorm_matmul(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                            const void* norm_weight, float eps, void* residual_out, int64_t ldro,
                            const int32_t* qweight, const void* scales, const void* zeros,
                            const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                            int64_t group_size, int32_t swiglu, const dk_matmul_config* cfg,
                            dk_stream_t stream);

/* A split-K projection handing its partial sums to the next projection, instead of reducing them
 * itself (the reference's decode step, kernels/e2e/model.py:247 then :231-235, passes the complete
 * fp16 down_proj output to the next layer's norm + qkv; no single-function counterpart):
 * dk_w4a16_matmul_partials writes x[M, K] @ dequant(W)^T as the fp32 partial sums of the launch's K
 * slices, partials[s][m][n] for s < *nparts (the split the library chose for this shape, set on the
 * host before the call returns; 1 = the whole sum), without bias; capacity is the buffer's size in
 * floats (8 * M * N always suffices). dk_w4a16_rmsnorm_matmul_partials is dk_w4a16_rmsnorm_matmul
 * with x = fp16(parts[0] + ... + parts[nparts - 1] (+ part_bias)), the additions in slice order, as
 * the projection's own reduction makes them: the pair computes the same values as dk_w4a16_matmul
 * followed by dk_w4a16_rmsnorm_matmul, in one dependency step fewer (no cluster reduction).
 * 1 <= M <= 16 rows in one launch, the fast path's conditions, 16-byte aligned buffers. */
int dk_w4a16_matmul_partials(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                             const void* zeros, int64_t M, int64_t N, int64_t K, int64_t group_size,
                             float* partials, int64_t capacity, int32_t* nparts,
                             const dk_matmul_config* cfg, dk_stream_t stream);
int dk_w4a16_rmsnorm_matmul_partials(const float* parts, int32_t nparts, const void* part_bias,
                                     const void* residual, int64_t ldr, const void* norm_weight, float eps,
                                     void* residual_out, int64_t ldro, const int32_t* qweight,
                                     const void* scales, const void* zeros, const void* bias, void* y,
                                     int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group_size,
                                     int32_t swiglu, const dk_matmul_config* cfg, dk_stream_t stream);

/* ---- FP8 e4m3 weight-only format: kernels/fp8.py ------------------------------------------ */
/* quantize_fp8 (kernels/fp8.py:25-30): w fp16 [N, K] (row stride ldw) -> wq e4m3 [K, N],
 * scale fp16 [N]; per-row absmax / 448 clamped >= 1e-12. Bit-exact with the reference. */
int dk_quantize_fp8(const void* w, int64_t ldw, uint8_t* wq, void* scale, int64_t N, int64_t K,
                    dk_stream_t stream);
/* dequantize_fp8 (kernels/fp8.py:33-35): -> fp16 [N, K] = fp16(fp32(wq) * fp32(scale)). */
int dk_dequantize_fp8(const uint8_t* wq, const void* scale, void* w, int64_t N, int64_t K,
                      dk_stream_t stream);

/* w8a16_matmul (kernels/fp8.py:200-223): y[M, N] fp16 = (x[M, K] @ fp16(wq)) * scale (+ bias),
 * wq e4m3 [K, N] (N contiguous), scale fp16 [N], fp32 accumulation, the scale applied to the
 * fp32 sum (kernels/fp8.py:81-82). cfg as for dk_w4a16_matmul (split_k, block_n, flags).
 * Dispatch by rows as for dk_w4a16_matmul: the decode GEMV (up to 16 rows per launch, fewer for long
 * K slices), the tcgen05 small-M kernel for 16-127 rows (N >= 128, K % 64 == 0; 16 rows only with
 * K >= 4096), the tcgen05 tensor-core GEMM for M >= 128 and N >= 128 (N % 16 == 0, K % 64 == 0,
 * aligned; kernels/fp8.py:42-127 for large M). DK_FLAG_GEMV keeps any M on the decode kernel. */
int dk_w8a16_matmul(const void* x, int64_t ldx, const uint8_t* wq, const void* scale, const void* bias,
                    void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, const dk_matmul_config* cfg,
                    dk_stream_t stream);

/* ---- fused RMSNorm (+ residual): kernels/rmsnorm.py ------------------------------------- */
/* rmsnorm (kernels/rmsnorm.py:44-68): out = w * fp16(h * rsqrt(mean(h^2) + eps)) with
 * h = x (+ residual, fp16 add, also written to residual_out). residual may be NULL (then
 * residual_out is unused). x, residual, out, residual_out are [M, N] with the given row strides. */
int dk_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, const void* weight,
               void* out, int64_t ldo, void* residual_out, int64_t ldro, int64_t M, int64_t N,
               float eps, dk_stream_t stream);

/* ---- fused SwiGLU: kernels/swiglu.py ----------------------------------------------------- */
/* swiglu / swiglu_fused (kernels/swiglu.py:49-61): out[M, I] = fp16(silu(gate)) * up.
 * For the fused [M, 2I] layout pass gate = gu, up = gu + I, ldg = ldu = 2I. */
int dk_swiglu(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out, int64_t ldo,
              int64_t M, int64_t I, dk_stream_t stream);

/* ---- decode attention: kernels/e2e/model.py:236-244 for one new token ---------------------- */
/* RoPE on q and k (x*cos + rotate_half(x)*sin, fp16 rounding per op), append k and v to the cache
 * at position *pos, and softmax(q k^T / sqrt(head_dim)) v over cache positions 0..*pos, with
 * grouped-query heads (nq / nkv query heads per kv head). qkv [B, (nq + 2 nkv) * head_dim] is the
 * fused projection output; caches [B, nkv, max_len, head_dim]; cos, sin [head_dim] for this
 * position; out [B, nq * head_dim]. `pos` is a device pointer (graph-capturable); a position outside
 * [0, max_len) writes nothing and sets DK_DEVERR_BAD_POSITION. splits: positions are cut into this
 * many slices combined inside a thread-block cluster (0 = automatic: max_len / 128, at most 16, and no
 * more than one wave of CTAs over B * nkv clusters; max 16). head_dim 32, 64 or 128. */
#define DK_ATTN_STATIC_CACHE 1 /* flags: the cache rows before *pos and *pos itself were not written
                                  by the kernel immediately before this one (true inside a decode
                                  step): the cache slice is fetched before waiting for that kernel */
/* rope_stride > 0: cos and sin are tables of at least max_len rows [positions, head_dim] (row stride
 * rope_stride elements) and the kernel uses row *pos; rope_stride == 0: they already hold this
 * position's [head_dim]. */
int dk_decode_attention(const void* qkv, void* k_cache, void* v_cache, const int64_t* pos,
                        const void* cos, const void* sin, void* out, int64_t B, int64_t nq,
                        int64_t nkv, int64_t head_dim, int64_t max_len, int64_t rope_stride,
                        int32_t splits, int32_t flags, dk_stream_t stream);

/* ---- lm_head + greedy pick of a decode step: kernels/e2e/model.py:248-253, run.py:69-74 ---- */
/* The tail of the reference's T == 1 forward and its graph decoder's greedy bookkeeping in one
 * kernel: the final RMSNorm (h = x + residual in fp16 with the rounding of kernels/rmsnorm.py:28-37;
 * residual and norm_weight may be NULL: no add, no norm), logits = fp16(h lm_head^T) accumulated in
 * fp32 (lm_head fp16 [vocab, hidden], tied to the embedding or not), and the greedy pick of every row
 * - the first maximum of its fp16 logits, torch.argmax's rule - stored to tokens[M] (device int64).
 * With history != NULL also history[m * history_ld + *pos] = pick, and with pos != NULL *pos += 1 (a
 * position outside [0, history_len) writes no history, leaves *pos and sets DK_DEVERR_BAD_POSITION);
 * logits [M, vocab] fp16 or NULL. 1 <= M <= 8, hidden % 8 == 0, 16-byte aligned x, residual, norm weight and
 * lm_head. The workspace (dk_lm_head_greedy_workspace_bytes, 256-byte aligned, zeroed once before the
 * first call) holds an arrival counter that each call leaves at zero, so calls sharing a workspace
 * must be ordered on one stream. */
int dk_lm_head_greedy_workspace_bytes(uint64_t* bytes);
int dk_lm_head_greedy(const void* x, const void* residual, const void* norm_weight, float eps,
                      const void* lm_head, int64_t vocab, int64_t hidden, int64_t M, int64_t* tokens,
                      int64_t* pos, int64_t* history, int64_t history_ld, int64_t history_len,
                      void* logits, void* workspace, uint64_t workspace_bytes, dk_stream_t stream);
/* The embedding lookup at the head of the forward (kernels/e2e/model.py:227, F.embedding):
 * out[m] = embed[tokens[m]] for device int64 tokens [M]; an id outside [0, vocab) takes row 0 and
 * sets DK_DEVERR_BAD_TOKEN. hidden % 8 == 0, 16-byte aligned embed and out. */
int dk_embed_tokens(const int64_t* tokens, const void* embed, int64_t vocab, int64_t hidden, int64_t M,
                    void* out, dk_stream_t stream);

/* ---- fused decode step: one persistent kernel per token ------------------------------------
 * One greedy decode step of a Qwen2 model with W4A16 linears and a tied or untied fp16 lm_head, for
 * 1..4 sequences: the reference runner's T == 1 forward (kernels/e2e/model.py:216-253: embedding,
 * per layer residual + RMSNorm, qkv with bias, RoPE, KV-cache append, GQA attention over positions
 * 0..pos, o_proj, residual + RMSNorm, gate_up, SwiGLU, down; final norm, lm_head) followed by the
 * greedy step of its graph decoder (kernels/e2e/run.py:69-74: argmax, token feedback, position
 * bump), as ONE cooperative kernel with one CTA per SM. Each CTA's producer warp streams its share
 * of every op's weights into shared memory ahead of the op's input (the weights are constant), and
 * the ops meet through tagged activation words in the workspace (each value carries the step and op
 * that wrote it; readers poll until the tags match). Numerics are those of the separate
 * kernels: dk_w4a16_rmsnorm_matmul / dk_w4a16_matmul (factored int4), dk_decode_attention,
 * dk_rmsnorm, and an fp16 lm_head with fp32 accumulation rounded to fp16 before the argmax (ties to
 * the lowest index, like torch.argmax). No reference counterpart as one kernel.
 * Limits: batch <= 4, head_dim 128, <= 8 query heads per kv head, hidden, intermediate and
 * n_heads * 128 multiples of 256, vocab % 32 == 0, max_len % 128 == 0, group size 128, 16-byte
 * aligned tensors (DK_ERR_UNSUPPORTED / DK_ERR_ALIGN otherwise: use the per-op entry points). */
typedef struct dk_step_layer {
  const void* input_norm; /* fp16 [hidden] */
  const void* post_norm;  /* fp16 [hidden] */
  const int32_t* qkv_qweight; /* [hidden/8, (n_heads + 2 n_kv) * head_dim]: q, k, v stacked */
  const void* qkv_scales;
  const void* qkv_zeros;
  const void* qkv_bias; /* fp16 [(n_heads + 2 n_kv) * head_dim] or NULL */
  const int32_t* o_qweight; /* [n_heads * head_dim / 8, hidden] */
  const void* o_scales;
  const void* o_zeros;
  const void* o_bias;
  const int32_t* gate_up_qweight; /* [hidden/8, 2 * intermediate]: gate then up */
  const void* gate_up_scales;
  const void* gate_up_zeros;
  const void* gate_up_bias;
  const int32_t* down_qweight; /* [intermediate/8, hidden] */
  const void* down_scales;
  const void* down_zeros;
  const void* down_bias;
} dk_step_layer;

typedef struct dk_step_model {
  int32_t n_layers, hidden, n_heads, n_kv, head_dim, intermediate, vocab, max_len, batch;
  float eps;
  const void* embed;      /* fp16 [vocab, hidden] */
  const void* final_norm; /* fp16 [hidden] */
  const void* lm_head;    /* fp16 [vocab, hidden]; may be `embed` (tied) */
  const void* rope_cos;   /* fp16 [max_len, head_dim]: cos(pos * inv_freq) of cat(freqs, freqs) */
  const void* rope_sin;
  void* k_cache;          /* fp16 [n_layers, batch, n_kv, max_len, head_dim] */
  void* v_cache;
  const dk_step_layer* layers; /* [n_layers] */
} dk_step_model;

typedef struct dk_step_plan dk_step_plan;

/* Bytes of the device workspace a plan needs (op table, tensor maps, arrival counters, the
 * activations between ops, attention and argmax partials). */
int dk_step_workspace_bytes(const dk_step_model* model, uint64_t* bytes);
/* Set-up only (synchronizes): build the step program for `model` in `workspace` (device memory of
 * at least dk_step_workspace_bytes, 256-byte aligned, owned by the caller and kept alive with the
 * plan). The model's tensors are referenced, not copied. */
int dk_step_create(const dk_step_model* model, void* workspace, uint64_t bytes, dk_step_plan** plan);
/* One decode step on `stream`: tokens int64 [batch] (this step's input tokens; overwritten with the
 * greedy picks), pos int64 [1] (their position; incremented), history int64 [batch, history_ld] or
 * NULL (history[b][pos] = pick), logits fp16 [batch, vocab] or NULL. All device pointers, read on the
 * device, so one captured launch replays for every step. Calls on one plan must not overlap. */
int dk_step_run(const dk_step_plan* plan, int64_t* tokens, int64_t* pos, int64_t* history, int64_t history_ld,
                void* logits, dk_stream_t stream);
int dk_step_destroy(dk_step_plan* plan);
/* Diagnostics. dk_step_trace runs dk_step_run and also records, per CTA and op of the program,
 * %globaltimer nanoseconds [wait start, input ready, input staged, products done, work done, arrival]
 * and clock cycles [most cycles a warp waited for its weights, one L2 load of the fresh input, the
 * release fence before the arrival, 0, 0, 0] (zero where the CTA has no part in the op; attention
 * records no staged / products stamps) and, in the slot after the last op, [kernel start, kernel end],
 * into `trace` (device memory of dk_step_trace_bytes, 8-byte aligned; [grid][n_ops + 1][12] uint64).
 * dk_step_ops gives the
 * program's op kinds (1 qkv, 2 attention, 3 o_proj, 4 gate_up + SwiGLU, 5 down, 6 lm_head + argmax). */
int dk_step_trace_bytes(const dk_step_plan* plan, uint64_t* bytes);
int dk_step_trace(const dk_step_plan* plan, int64_t* tokens, int64_t* pos, int64_t* history, int64_t history_ld,
                  void* logits, uint64_t* trace, dk_stream_t stream);
int dk_step_ops(const dk_step_plan* plan, int32_t* kinds, int32_t capacity, int32_t* n_ops);

/* ---- tensor parallelism: row-sharded W4A16 projection fused with its allreduce ------------
 * No reference counterpart: the reference runs on one GPU (README.md:249). These entry points serve
 * the tensor-parallel runner (column-sharded qkv/gate_up/lm_head, row-sharded o_proj/down), one
 * process per GPU of one node. Each rank owns one exchange buffer, allocated once at set-up and
 * mapped into every peer with CUDA IPC; a row-sharded projection then pushes its fp32 partial sums,
 * each tagged with the launch's epoch in the same 8-byte store, into every peer's buffer over NVLink
 * from the GEMV epilogue, and sums the ranks' partials of its own output columns in rank order once
 * their tags match, so the matmul and the allreduce are one kernel and every rank ends with the same
 * bits. No TMA multicast is used on peer memory. */
#define DK_TP_MAX_WORLD 8
#define DK_TP_IPC_HANDLE_BYTES 64 /* sizeof(cudaIpcMemHandle_t) */

typedef struct dk_tp_comm dk_tp_comm;

/* Bytes of one rank's exchange buffer for launches of up to max_m rows (max 64) and max_n columns. */
int dk_tp_buffer_bytes(int32_t world, int64_t max_m, int64_t max_n, uint64_t* bytes);
/* Set-up only (allocates and synchronizes): cudaMalloc `bytes` on the current device, zero them,
 * return the pointer and its IPC handle (DK_TP_IPC_HANDLE_BYTES bytes written to ipc_handle). */
int dk_tp_buffer_alloc(uint64_t bytes, void** ptr, void* ipc_handle);
int dk_tp_buffer_free(void* ptr);
/* Set-up only: map a peer process's buffer from its IPC handle (peer access over NVLink). */
int dk_tp_buffer_open(const void* ipc_handle, void** ptr);
int dk_tp_buffer_close(void* ptr);
/* A communicator over the exchange buffers of all ranks: bufs[rank] is this rank's own buffer
 * (dk_tp_buffer_alloc), bufs[q] the mapping of rank q's (dk_tp_buffer_open). Host object only;
 * destroying it frees and unmaps nothing. */
int dk_tp_comm_create(dk_tp_comm** comm, int32_t rank, int32_t world, void* const* bufs, int64_t max_m,
                      int64_t max_n);
int dk_tp_comm_destroy(dk_tp_comm* comm);
/* Bound of each wait of a fused-allreduce launch on this communicator for a peer's partial sums:
 * 1 ms .. 10 s (default 2 s). A CTA whose wait runs out leaves its columns of y unwritten, sets
 * DK_DEVERR_TP_WAIT and returns, so a rank that never launches cannot hang the others' kernels. */
int dk_tp_comm_set_wait(dk_tp_comm* comm, uint64_t wait_ns);

/* Row-sharded w4a16_matmul with the allreduce fused in:
 *   y[M, N] = fp16( sum over ranks r, in rank order, of x_r[M, K] @ dequant(W_r).T  + bias )
 * where each rank passes its own K-shard x_r and W_r (qweight [K/8, N], scales/zeros [K/128, N]) and
 * receives the full y. Every rank must make the same sequence of calls on one communicator with the
 * same M, N and K (the kernels of different ranks meet per CTA; a CTA that waits more than ~2 s for
 * a peer gives up, leaves its columns of y unwritten and sets DK_DEVERR_TP_WAIT). Needs the fast
 * path's conditions (group_size 128, N % 8 == 0, 16-byte aligned operands), N <= max_n. 17 .. max_m
 * rows (max_m <= 64) run as ONE launch of the tcgen05 small-M kernel (N >= 128; one pass over the
 * weights) with the same allreduce epilogue; otherwise the decode GEMV in launches of up to
 * min(16, max_m) rows. */
int dk_w4a16_matmul_allreduce(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                              const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M, int64_t N,
                              int64_t K, int64_t group_size, const dk_matmul_config* cfg,
                              const dk_tp_comm* comm, dk_stream_t stream);

/* ---- allocation-free variant ---------------------------------------------------------------
 * No counterpart in the reference. dk_w4a16_matmul_allreduce needs an exchange buffer from
 * dk_tp_buffer_alloc (cudaMalloc). Some callers cannot allocate device memory: a plugin loaded into a
 * serving process that owns the CUDA allocator and hands the plugin only its input and output
 * buffers, or a runtime that forbids raw cudaMalloc (it synchronizes the device and fragments a pool
 * it manages). For them this entry point runs the same fused matmul + reduce kernel on one GPU
 * (world 1: y = fp16(x @ dequant(W).T + bias), the result of dk_w4a16_matmul_allreduce with a
 * one-rank communicator) with its scratch - launch epoch, arrival count and the epoch-tagged
 * partial-sum cells - in a fixed array inside the library: 2 MiB + 256 bytes per GPU that loads the
 * library, held until the process exits. The caller passes inputs and outputs only. Limits: N <= 8192
 * (larger N returns DK_ERR_INVALID), M in launches of up to 16 rows, and the fast path's conditions
 * (group_size 128, N % 8 == 0, 16-byte aligned operands). It calls no cudaMalloc, cudaFree or
 * allocating library routine. Its first call on a device looks up the array's device address
 * (set-up): make that first call before any stream capture. Every call shares the one array, which
 * keeps what the last call left: the launch epoch in its header advances from call to call (the
 * array is zero when the library loads), so partial sums left in the cells by an earlier call carry
 * an older epoch tag and are never read as this call's. Calls that overlap on the GPU (other streams,
 * other host threads) race on the array. */
int dk_w4a16_matmul_reduce_static(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                                  const void* zeros, const void* bias, void* y, int64_t ldy, int64_t M, int64_t N,
                                  int64_t K, int64_t group_size, const dk_matmul_config* cfg, dk_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DECODEK_H_ */
