/*
 * rembed_gpu.h - C ABI of librembed_gpu.so, the B200 (sm_100a) encoder
 * forward pass for rembed.
 *
 * The library replaces the pure-Go kernel layer below rembed's
 * Model.ForwardWorkers / ForwardTokensWorkers (internal/model/bert.go:657-734)
 * for a whole batch of sequences at once.  rembed's host keeps Load, the
 * config derivation, the tokenizers and the Embed / EmbedTokens API; its
 * per-text forward fan-out (rembed.go:309-331) becomes one rg_forward call.
 *
 * Conventions follow the reference's own FFI (python/capi/main.go:9-13):
 *   - functions return 0 on success and -1 on failure;
 *   - on failure, if err != NULL, *err receives a malloc'd message that the
 *     caller releases with rg_free_string (RembedFreeString, main.go:150-155);
 *   - the caller owns every output buffer; host inputs are borrowed for the
 *     duration of the call only;
 *   - a context is safe for concurrent use (the reference Embedder is,
 *     rembed.go:37-41): calls on one context serialise internally.
 * Nothing here aborts the process, and there is no CPU fallback: a shape or
 * mode the CUDA path cannot run is an error.
 */
#ifndef REMBED_GPU_H
#define REMBED_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RG_ABI_VERSION 1

/* Architectures (model.Config.ModelType, config.go:17; dispatch bert.go:316-337). */
enum {
    RG_ARCH_BERT = 0, RG_ARCH_DISTILBERT = 1, RG_ARCH_ROBERTA = 2, RG_ARCH_MPNET = 3,
    RG_ARCH_MODERNBERT = 4, RG_ARCH_QWEN3 = 5, RG_ARCH_GEMMA3 = 6, RG_ARCH_NOMIC = 7
};
/* Pooling (Config.Pooling, bert.go:670-679). */
enum { RG_POOL_MEAN = 0, RG_POOL_CLS = 1, RG_POOL_LASTTOKEN = 2 };
/* Numeric modes.  RG_MODE_BF16: bf16 tensor-core GEMMs, fp32 accumulate,
 * fp32 residual stream (replaces the reference's fp32 path).  RG_MODE_F16:
 * the same with fp16 operands (8x finer rounding; weights must fit the fp16
 * range).  RG_MODE_INT8_W: weight-only int8, the PackB8 quantiser
 * (WithInt8, rembed.go:67-69): int8 weights in HBM, widened to fp16 inside
 * the GEMM mainloop, fp16 activations.  RG_MODE_INT8_FULL: int8 weights and
 * per-row int8 activations, the PackB8VNNI scheme (WithInt8Activations,
 * rembed.go:79-81).  RG_MODE_FP32: strict fp32 (the reference's own
 * arithmetic width): fp32 activations end to end, projections as 3xTF32
 * tensor-core GEMMs (tf32 hi/lo operand splits, fp32 accumulate), fp32
 * attention. */
enum { RG_MODE_BF16 = 0, RG_MODE_F16 = 1, RG_MODE_INT8_W = 2, RG_MODE_INT8_FULL = 3, RG_MODE_FP32 = 4 };
/* Host dtypes accepted by rg_upload_weight (safetensors.go:188-209). */
enum { RG_DTYPE_F32 = 0, RG_DTYPE_F16 = 1, RG_DTYPE_BF16 = 2 };
/* rg_forward output kinds: pooled (Embed) or per-token hidden states
 * (EmbedTokens, rembed.go:370-411). */
enum { RG_OUT_POOLED = 0, RG_OUT_TOKENS = 1 };

/* The Config fields the forward reads (model.Config, config.go:15-78).
 * Unused fields for an architecture are ignored; zero means "absent". */
typedef struct rg_model_desc {
    int arch;                     /* RG_ARCH_* */
    int hidden_size, num_hidden_layers, num_attention_heads, intermediate_size;
    int vocab_size, max_position_embeddings;
    float layer_norm_eps;         /* 0 -> 1e-12 (config.go:228-230) */
    int pooling;                  /* RG_POOL_* */
    int normalize;                /* L2-normalise the pooled vector */
    int pad_token_id, relative_attention_num_buckets;
    int head_dim, num_key_value_heads;
    double rope_theta, global_rope_theta, local_rope_theta;
    int global_attn_every_n_layers, local_attention;
    int sliding_window, sliding_window_pattern, query_pre_attn_scalar, dense_hidden;
} rg_model_desc;

typedef struct rg_ctx rg_ctx;

/* Create a context holding one weight replica per listed CUDA device
 * (data parallel across devices; sequences are sharded, never split).
 * Replaces model.Load's per-arch loader (bert.go:307-518) minus the
 * safetensors parsing, which stays with the caller.  mode is RG_MODE_*. */
int rg_init(const rg_model_desc *desc, const int *devices, int ndev, int mode,
            rg_ctx **out, char **err);

/* Hand one tensor to the context by its Hugging Face name, exactly as the
 * reference loader looks it up (bert.go:338-470; prefixes "bert.",
 * "roberta.", "mpnet.", "distilbert." accepted).  host is read during the
 * call only.  Shapes are checked against the descriptor. */
int rg_upload_weight(rg_ctx *ctx, const char *name, int dtype, const int64_t *shape, int ndim,
                     const void *host, char **err);

/* Once every tensor is uploaded: fuse Q|K|V (bert.go:479-485), quantise
 * with the reference's own quantisers for the int8 modes (newDense,
 * bert.go:263-278; PackB8 pack8.go:25-76, PackB8VNNI pack_vnni.go:28-77),
 * copy to every device.  A non-finite weight under an int8 mode is an
 * error (pack8.go:43-48). */
int rg_finalize(rg_ctx *ctx, char **err);

/* Forward a packed batch from HOST memory: ids [cu_seqlens[nseq]] token ids
 * (int64, as Model.Forward takes them), cu_seqlens [nseq+1] prefix offsets.
 * RG_OUT_POOLED writes host_out[nseq x out_dim]: pooled, Dense head (Gemma),
 * L2-normalised when the config says so, then truncated to out_dim and
 * re-normalised when out_dim < hidden (Matryoshka, rembed.go:441-448).
 * RG_OUT_TOKENS writes host_out[cu_seqlens[nseq] x hidden], the final hidden
 * states (out_dim must equal hidden).  Errors, checked before any launch:
 * empty sequence, sequence longer than the model maximum, token id outside
 * [0, vocab) (bert.go:742-747, 797-799). */
int rg_forward(rg_ctx *ctx, const int64_t *ids, const int32_t *cu_seqlens, int nseq, int out_kind,
               int out_dim, float *host_out, char **err);

/* The same forward, asynchronous: validates and stages the batch (ids and
 * cu_seqlens are copied before returning), enqueues it and returns a ticket
 * at once, so the caller can tokenise / pack the next batch while this one
 * runs.  host_out must stay valid until rg_collect(ticket), which waits for
 * the batch and writes host_out.  Two submissions may be outstanding per
 * context (two pinned staging slots per device); a third fails until the
 * oldest is collected.  Replaces nothing in the reference, whose Embed is
 * synchronous; it is the CPU-tokeniser / GPU overlap the reference host
 * needs to keep a GPU busy. */
int rg_submit(rg_ctx *ctx, const int64_t *ids, const int32_t *cu_seqlens, int nseq, int out_kind,
              int out_dim, float *host_out, int64_t *ticket, char **err);
int rg_collect(rg_ctx *ctx, int64_t ticket, char **err);

/* Forward a packed batch already resident on device `dev_index` (an index
 * into the rg_init device list): d_ids, d_cu_seqlens and d_out are device
 * pointers on that device; `stream` is a cudaStream_t (NULL = the context's
 * own stream for that device).  host_cu_seqlens is the same offsets in host
 * memory (used for validation and work partitioning, never for ids).  No
 * synchronisation on return: the result is ready when `stream` reaches this
 * point.  Ids are validated on the device; a bad id makes the call return
 * -1 at the next rg_forward_device / rg_sync on this device. */
int rg_forward_device(rg_ctx *ctx, int dev_index, const int64_t *d_ids, const int32_t *d_cu_seqlens,
                      const int32_t *host_cu_seqlens, int nseq, int out_kind, int out_dim, float *d_out,
                      void *stream, char **err);

/* Wait for all work on device `dev_index` and report any deferred error. */
int rg_sync(rg_ctx *ctx, int dev_index, char **err);

/* Output dimension before truncation (Config.HiddenSize). */
int rg_hidden(const rg_ctx *ctx);
/* Numeric mode actually running (replaces Model.Quantized /
 * QuantizedActivations, bert.go:531-644: there is never a silent fallback,
 * so this always equals the mode rg_init accepted). */
int rg_mode_active(const rg_ctx *ctx);
/* Number of kernel launches the last rg_forward / rg_forward_device issued
 * on device `dev_index` (for launch accounting in benchmarks). */
int rg_last_launches(const rg_ctx *ctx, int dev_index);

/* Kernel timing for measurement: when enabled, every launch of a forward on
 * device `dev_index` is bracketed by CUDA events on its stream.
 * rg_profile(enable=1) clears the counters; rg_profile_stats synchronises
 * the device and returns, for one kernel class (RG_KC_*), the summed device
 * milliseconds, launch count, algorithmic FLOPs and algorithmic bytes since
 * the last enable.  Off by default (no events recorded). */
enum { RG_KC_GEMM = 0, RG_KC_ATTENTION = 1, RG_KC_NORM = 2, RG_KC_POOL = 3, RG_KC_QUANT = 4, RG_KC_COUNT = 5 };
int rg_profile(rg_ctx *ctx, int dev_index, int enable);
int rg_profile_stats(rg_ctx *ctx, int dev_index, int kernel_class, double *ms, int *launches, double *flops,
                     double *bytes);

void rg_free(rg_ctx *ctx);
void rg_free_string(char *s);

/* Failure injection for tests of the error paths (never needed in
 * production; nothing is injected unless this is called).  Each injection
 * fires once:
 *   RG_INJECT_GEMM_WAIT (ctx may be NULL): the next rg_dense_bf16 launch
 *     withholds one of its pipeline's barrier arrivals and bounds every wait
 *     at `arg` cycles, so the wait runs out on the device; the kernel stops,
 *     drains what is in flight, frees its tensor memory and records the
 *     timeout, which the next rg_kernel_status reports;
 *   RG_INJECT_HOST_ALLOC: the next submission on ctx fails as if its pinned
 *     host staging could not be allocated;
 *   RG_INJECT_REPLICA: the next submission on ctx fails in the worker of
 *     replica `arg` (an index into rg_init's device list) after the replicas
 *     before it have started; their work is collected and the call returns
 *     the worker's error.
 * Returns 0, or -1 for an unknown injection or a bad argument. */
enum { RG_INJECT_GEMM_WAIT = 1, RG_INJECT_HOST_ALLOC = 2, RG_INJECT_REPLICA = 3 };
int rg_test_inject(rg_ctx *ctx, int what, long long arg, char **err);

/* ---- kernel-level entry points (parity tests, benchmarks) --------------
 * Device pointers on the current CUDA device; stream = cudaStream_t or NULL.
 *
 * rg_dense_bf16: y[M x N] = epilogue(x[M x K] . W[N x K]^T): the dense
 * projection of applyDense (bert.go:282-301) as one tcgen05 GEMM.
 * epilogue: 0 = +bias -> bf16 y; 1 = +bias, exact GELU -> bf16 y;
 * 2 = +bias +residual (fp32) -> fp32 y.  x, W bf16; bias fp32 or NULL.
 * K must be a multiple of 64, N of 128 (checked). */
int rg_dense_bf16(const void *x, const void *w, const float *bias, const float *residual, void *y,
                  int M, int N, int K, int epilogue, void *stream, char **err);

/* Every kernel-level call below is asynchronous.  A failure a kernel
 * detects on the device (a bounded pipeline wait that gave up, an fp16
 * output overflow) sets a bit in a status word of the device instead of
 * hanging or aborting; rg_kernel_status synchronises `stream`, reads and
 * clears the status words of the current device (the kernel-level calls'
 * and the no-allocation variant's) and returns -1 with a message if a
 * failure was recorded since the last check. */
int rg_kernel_status(void *stream, char **err);

/* rg_dense_residual_layernorm_bf16: the post-attention / post-FFN sublayer
 * of the BERT family (applyDense + Add + LayerNorm, bert.go:905-907 and
 * 916-918):  s = residual + (x . W^T + bias);  out32 = LayerNorm(s; gamma,
 * beta, eps) in fp32 and outb = bf16(out32).  x [M x K], W [N x K] bf16;
 * bias, gamma, beta [N] fp32; residual, out32 [M x N] fp32; outb [M x N]
 * bf16.  The fp32 sum s is scratch in a per-device buffer that the library
 * allocates on first use and grows as needed.  K % 64 == 0; N a multiple
 * of 128 up to 2048.  Asynchronous on `stream`. */
int rg_dense_residual_layernorm_bf16(const void *x, const void *w, const float *bias, const float *residual,
                                     const float *gamma, const float *beta, float eps, float *out32, void *outb,
                                     int M, int N, int K, void *stream, char **err);

/* rg_dense_residual_layernorm_bf16_noalloc: no counterpart in the reference.
 * The same sublayer as rg_dense_residual_layernorm_bf16, for callers that
 * cannot let a library call cudaMalloc: a host whose memory manager owns
 * every byte of device memory (an arena carved out of HBM up front, or an
 * allocator that must account for each buffer), or a latency-bound caller
 * that cannot afford the device synchronisation an allocation may bring.
 * It calls no allocator: its scratch is a fixed static device array of
 * RG_NOALLOC_SCRATCH_FLOATS floats (16 MiB) that the library image holds on
 * every GPU where the library is loaded, until process exit.
 * Limit: M * N <= RG_NOALLOC_SCRATCH_FLOATS (larger calls fail with an
 * error naming the limit).  The first call on each device looks up the
 * array's device address (in the device's primary context, the one the CUDA
 * runtime API uses); make that first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU race; order them
 * on one stream.  An in-kernel failure is reported by rg_kernel_status. */
#define RG_NOALLOC_SCRATCH_FLOATS ((size_t)4 * 1024 * 1024)
int rg_dense_residual_layernorm_bf16_noalloc(const void *x, const void *w, const float *bias,
                                             const float *residual, const float *gamma, const float *beta,
                                             float eps, float *out32, void *outb, int M, int N, int K,
                                             void *stream, char **err);

/* rg_attention: the attention core of encodeWorkers and of the per-arch
 * encoders (bert.go:853-902, modernbert.go:239-281, gemma3.go:303-354) and
 * flashAttnCausalHead (qwen3.go:307-390) over a packed batch, as one fused
 * kernel.  q [T x ldq], k [T x ldk], v [T x ldv]: token-major rows, query
 * head h at columns h*head_dim, key/value head h / (heads / kv_heads) (GQA).
 * cu_seqlens [nseq+1] are device offsets; host_cu the same offsets in host
 * memory (shapes only).  Query i attends to keys j of its own sequence with
 * rel_lo <= j - i <= rel_hi (causal: rel_hi = 0; window w: +-w; unbounded:
 * +-2^30), scores scaled by `scale`.  dtype RG_DTYPE_BF16 / RG_DTYPE_F16:
 * the tcgen05 kernel, out 16-bit [T x ldo]; RG_DTYPE_F32: the strict fp32
 * kernel, q/k/v/out fp32.  Head dims 32, 64, 128, 256. */
int rg_attention(const void *q, const void *k, const void *v, int ldq, int ldk, int ldv, const int32_t *cu_seqlens,
                 const int32_t *host_cu, int nseq, int heads, int kv_heads, int head_dim, float scale, int rel_lo,
                 int rel_hi, int dtype, void *out, int ldo, void *stream, char **err);

/* rg_quantize_rows_s8: the full-int8 mode's per-row activation quantiser,
 * QuantizeRowU8 (pack_vnni.go:85-117) with the +128 offset removed:
 * scale[r] = maxabs(x[r]) / 127 (1 for an all-zero row), q = clamp(
 * RoundToEven(x * (1 / scale)), -128, 127).  x bf16 [M x K], K % 8 == 0,
 * K <= 4096. */
int rg_quantize_rows_s8(const void *x, int M, int K, int8_t *q, float *row_scale, void *stream, char **err);

/* rg_dense_s8: the full-int8 projection, MatMulPackedVNNI + AddBias
 * (pack_vnni.go:124-176, bert.go:297-300) on tcgen05 kind::i8:
 * y[M x N] = f32(sum_k xq[m][k] * wq[n][k]) * row_scale[m] * col_scale[n]
 * (+ bias[n]), the integer sum exact (it equals the reference's
 * acc - 128 * colSum).  xq [M x K], wq [N x K] int8 (PackB8VNNI weights);
 * K % 128 == 0, N % 128 == 0; y fp32. */
int rg_dense_s8(const int8_t *xq, const float *row_scale, const int8_t *wq, const float *col_scale, const float *bias,
                float *y, int M, int N, int K, void *stream, char **err);

#ifdef __cplusplus
}
#endif
#endif
