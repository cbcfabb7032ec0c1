/*
 * oracle.h - CPU restatement of rembed's encoder forward pass.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA path and the timed CPU baseline ("port" kind) in bench.py.  Nothing
 * in the product (rembed_b200/, include/) links, loads or calls it.
 *
 * Every routine restates one reference routine (rostamlabs/rembed, Go) and
 * cites it by file:line.  Floating-point semantics follow the reference as
 * built with the default GOAMD64=v1: scalar float32 expressions are rounded
 * after every operation (no contraction, compiled with -ffp-contract=off),
 * while the assembly micro-kernels' fused multiply-adds are restated with
 * explicit fmaf() in the same accumulation order.
 */
#ifndef REMBED_ORACLE_H
#define REMBED_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- primitives (internal/tensor) ---------------------------------- */
float or_expf32(float x);        /* fastmath.go:26-55  */
float or_expnonpos(float x);     /* fastmath.go:93-109 */
float or_erff32(float x);        /* fastmath.go:71-83  */
void or_softmax(float *x, int m, int n);                                   /* tensor.go:391-428 */
void or_layernorm(float *x, const float *g, const float *b, int m, int n, float eps); /* tensor.go:433-452 */
void or_rmsnorm(float *x, const float *g, int m, int n, float eps);       /* tensor.go:459-471 */
void or_silu(float *x, int n);                                             /* tensor.go:477-481 */
void or_gelu_tanh(float *x, int n);                                        /* tensor.go:490-497 */
void or_gelu(float *x, int n);                                             /* tensor.go:508-538 */
void or_l2normalize(float *x, int n);                                      /* tensor.go:542-554 */
void or_add_bias(float *x, const float *bias, int m, int n);               /* tensor.go:373-380 */
void or_add(float *dst, const float *src, int n);                          /* tensor.go:383-387 */
int or_relpos_bucket(int rel, int num_buckets);                            /* bert.go:135-150 */

/* dst[m x n] = a[m x k] . bT[n x k]^T, k-ordered fused multiply-add from
 * zero per element: the gemm4x16/gemm6x16/gemm4x32 micro-kernels
 * (gemm_amd64.s:14-75, pack.go:123-210). */
void or_matmul_packed(float *dst, const float *a, const float *bT, int m, int k, int n);
/* MatMulSerial with the dot4 micro-kernel (tensor.go:284-330,
 * dot_amd64.s:13-80): 8-lane FMA partial sums, folded and reduced. */
void or_matmul_serial(float *dst, const float *a, const float *bT, int m, int k, int n);

/* PackB8 quantiser (pack8.go:25-76): q row-major [n x k]; returns 0 or -1
 * (non-finite weight, or n%16 != 0). */
int or_packb8(const float *bT, int k, int n, int8_t *q, float *scales);
/* MatMulPacked8 + gemm4x16i8 (pack8.go:80-126, gemm8_amd64.s:14-70). */
void or_matmul_packed8(float *dst, const float *a, const int8_t *q, const float *scales,
                       int m, int k, int n);
/* PackB8VNNI quantiser (pack_vnni.go:28-77); q row-major [n x k]. */
int or_packb8vnni(const float *bT, int k, int n, int8_t *q, int32_t *colsum, float *scales);
/* QuantizeRowU8 (pack_vnni.go:85-117): writes k bytes, zeroes [k, kpad). */
float or_quantize_row_u8(uint8_t *dst, const float *a, int k, int kpad);
/* MatMulPackedVNNI (pack_vnni.go:124-176): bit-exact integer accumulate. */
void or_matmul_vnni(float *dst, const float *a, const int8_t *q, const int32_t *colsum,
                    const float *scales, int m, int k, int n);

/* flashAttnCausalHead (qwen3.go:307-390): one head, q/k/v/out [seq x dh],
 * 64-row blocks with online softmax and future key blocks skipped.
 * Returns 0 or -1 (no scratch). */
int or_flash_attn_causal_head(const float *qH, const float *kH, const float *vH, float *out, int seq, int dh,
                              float scale);

/* ---- model ---------------------------------------------------------- */
enum { OR_ARCH_BERT = 0, OR_ARCH_DISTILBERT = 1, OR_ARCH_ROBERTA = 2, OR_ARCH_MPNET = 3,
       OR_ARCH_MODERNBERT = 4, OR_ARCH_QWEN3 = 5, OR_ARCH_GEMMA3 = 6, OR_ARCH_NOMIC = 7 };
enum { OR_POOL_MEAN = 0, OR_POOL_CLS = 1, OR_POOL_LAST = 2 };
enum { OR_QUANT_NONE = 0, OR_QUANT_WEIGHTS = 1, OR_QUANT_FULL = 2 };

/* The fields of model.Config (config.go:15-78) the forward reads. */
typedef struct {
    int arch;
    int hidden, layers, heads, inter, vocab, max_pos, type_vocab;
    float eps;
    int pooling, normalize;
    int pad_token_id, rel_buckets;
    int head_dim, kv_heads;
    double rope_theta, global_theta, local_theta;
    int global_every, local_attention;
    int sliding_window, sliding_pattern, query_pre_attn_scalar, dense_hidden;
} or_config;

typedef struct or_model or_model;

or_model *or_model_new(const or_config *cfg, int quant);
/* Borrow a float32 tensor by its Hugging Face name.  The caller keeps the
 * memory alive for the model's lifetime.  Returns 0, or -1 if the name is
 * unknown or the element count is wrong. */
int or_model_set(or_model *m, const char *name, const float *data, int64_t numel);
/* Quantise / fuse once all tensors are set (newDense, bert.go:263-278).
 * Returns 0, or -1 with a message in err (>= 256 bytes). */
int or_model_finalize(or_model *m, char *err);
void or_model_free(or_model *m);

/* One sequence (ForwardWorkers, bert.go:657-689): pooled[H] (pooled, head,
 * L2) and, if tokens != NULL, the final hidden states [seq x H]
 * (ForwardTokensWorkers, bert.go:715-734).  Returns 0 or -1 + err. */
int or_forward(or_model *m, const int64_t *ids, int seq, float *pooled, float *tokens, char *err);

/* Batch of packed sequences (Embed, rembed.go:287-332): one serial forward
 * per sequence across nthreads threads.  out_kind 0 = pooled, written as
 * out[nseq x dim] with the Matryoshka truncate (rembed.go:441-448) when dim <
 * H; out_kind 1 = per-token hidden states out[T x H].  Returns 0 or -1. */
int or_embed_batch(or_model *m, const int64_t *ids, const int32_t *cu_seqlens, int nseq,
                   int nthreads, int out_kind, int dim, float *out, char *err);

#ifdef __cplusplus
}
#endif
#endif
