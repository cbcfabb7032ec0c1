// kernels.cuh - the non-GEMM kernels of the encoder forward pass.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

namespace rg {

// Embedding rows (bert.go:795-814, qwen3.go:457-462, modernbert.go:204-211,
// gemma3.go:264-275, nomic.go:164-176): x = word[id] (+ pos[p + pos_off])
// (+ type0), times scale, then LayerNorm(g, b) when g is set; p is the
// token's index in its sequence.  Writes fp32 x32 and, if set, the 16-bit
// row xb (fp16 if f16, else bf16) and the int8 row (xq, xq_scale).  An id
// outside [0, vocab) raises kStatusBadToken and yields zeros (never an
// out-of-bounds read).
struct EmbedParams {
    const int64_t* ids;
    const int32_t* cu;
    int nseq, T, H, vocab, pos_off;
    const float *word, *pos, *type0;
    float scale;
    const float *g, *b;
    float eps;
    float* x32;
    uint16_t* xb;
    bool f16;
    int8_t* xq;
    float* xq_scale;
    int* status;
    float *xhi, *xlo;  // strict fp32: the normalised row as tf32-exact hi + fp32 remainder
    int32_t* pos_out;  // optional: each token's position in its sequence
};
cudaError_t launch_embed(const EmbedParams& p, cudaStream_t st);

// hi = x rounded to the nearest tf32 value (10 mantissa bits, ties to
// even), lo = x - hi (exact): the two operand parts of a 3xTF32 GEMM.
__host__ __device__ inline void tf32_split(float x, float& hi, float& lo) {
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(x);
#else
    uint32_t u;
    memcpy(&u, &x, 4);
#endif
    u = (u + 0xfffu + ((u >> 13) & 1u)) & 0xffffe000u;
#ifdef __CUDA_ARCH__
    hi = __uint_as_float(u);
#else
    memcpy(&hi, &u, 4);
#endif
    lo = x - hi;
}
// x [n] -> hi [n], lo [n] (hi may alias x); n % 4 == 0, 16-byte aligned.
cudaError_t launch_split_tf32(const float* x, size_t n, float* hi, float* lo, cudaStream_t st);

// Per-row LayerNorm statistics from the (mean, M2) of each row's nparts
// 32-column chunks (parts[i * T + row], as residual GEMM epilogues write
// them): stats[row] = (mean, 1 / sqrt(var + eps)).
// rms: RMSNorm statistics instead, stats[row] = (0, 1 / sqrt(mean(y^2) + eps))
// with sum(y^2) = sum(M2_i + 32 mean_i^2).
cudaError_t launch_merge_row_stats(const float2* parts, int nparts, int T, float eps, float2* stats, cudaStream_t st,
                                   bool rms = false);

// Row normalisation of in [T x H]: LayerNorm (g, b; b nullptr = zero) or
// RMSNorm (g); g nullptr = identity.  Outputs (each optional): out32 (may
// alias in), outb (16-bit: fp16 if f16, else bf16), outq + outqs (int8 row
// quantisation).
struct NormParams {
    const float* in;
    const float *g, *b;
    float eps;
    int T, H;
    float* out32;
    uint16_t* outb;
    bool f16;
    int8_t* outq;
    float* outqs;
    int* status;    // optional: kStatusF16Overflow if an fp16 output overflows
    float2* stats;  // optional: the row's (mean, rstd) (LayerNorm), for a consumer that
                    // rebuilds the fp32 output on load instead of reading out32
    float *outhi, *outlo;  // optional (strict fp32): the output as tf32 hi + fp32 remainder
    // optional: output row t normalises input row row_cu[t] (row_pick 1, a
    // sequence's first token) or row_cu[t + 1] - 1 (row_pick 2, its last),
    // clamped to [0, in_rows); T is then the number of sequences
    const int32_t* row_cu;
    int row_pick, in_rows;
};
cudaError_t launch_norm(const NormParams& p, bool rms, cudaStream_t st);
cudaError_t launch_ln(const float* y32, const float* g, const float* b, float eps, int T, int H, float* x32,
                      uint16_t* xb, bool f16, int8_t* xq, float* xq_scale, cudaStream_t st,
                      int* status = nullptr);
// x32 += RMSNorm(o32; g)  (Gemma's post-sublayer norms).
// x32 += RMSNorm(o32; g); with `next` (g, eps and the outputs of a NormParams)
// also the RMSNorm of the new x32 into next's outputs, as launch_norm would.
cudaError_t launch_add_rmsnorm(float* x32, const float* o32, const float* g, float eps, int T, int H, cudaStream_t st,
                               const NormParams* next = nullptr);

// QK-norm (optional) + RoPE (optional) in place on the q heads [0, nq) and
// k heads of the fused qkv buffer [T x ld] (q at column 0, k at nq*dh).
// cos/sin are [positions x dh/2] tables.  head_dim 64, 128 or 256.
struct QkRopeParams {
    uint16_t* qkv;  // 16-bit: fp16 if f16, else bf16
    bool f16;
    float* qkv32;   // strict fp32: the fp32 qkv buffer instead (qkv unused)
    int ld, T, nq, nkv;
    const float *q_norm, *k_norm;
    float eps;
    const float *cos, *sin;
    const int32_t* cu;
    int nseq;
    int* status;  // optional: kStatusF16Overflow
};
cudaError_t launch_qk_norm_rope(const QkRopeParams& p, int head_dim, cudaStream_t st);

// int8 -> fp16, exact (weight-only int8 at large batch: a layer's weights
// widened just before its first GEMM; the per-channel scale stays in the
// GEMM epilogue).  One launch over up to four (src, n, dst) widenings: n a
// multiple of 16, both pointers 16-byte aligned.
struct WidenJob {
    const int8_t* src;
    size_t n;
    uint16_t* dst;
};
cudaError_t launch_widen_s8_f16_multi(const WidenJob* jobs, int count, cudaStream_t st);

// Per-row symmetric int8 quantisation of a bf16 [T x K] matrix
// (QuantizeRowU8 with the +128 offset removed: q in [-128, 127]).
cudaError_t launch_quantize_rows(const __nv_bfloat16* x, int T, int K, int8_t* q, float* scale, cudaStream_t st);

// Varlen attention (bert.go:853-902, qwen3.go:307-390, modernbert.go:239-281,
// gemma3.go:303-354): per sequence and query head h (key/value head
// h / group), out = softmax(Q K^T * scale [+ bias(j - i)]) V over the keys j
// with rel_lo <= j - i <= rel_hi (causal: rel_hi = 0; symmetric window w:
// rel_lo = -w, rel_hi = w; unbounded: +-2^30).  Q, K, V, out are token-major
// 16-bit rows with strides ldq/ldk/ldv/ldo; head h's columns start at h*D.
// bias, if set, is [heads x (2*bias_off + 1)] indexed by j - i + bias_off
// (MPNet's bucketed relative-position bias, added after the scale).
struct AttnParams {
    const uint16_t *q, *k, *v;  // 16-bit: fp16 if f16, else bf16
    bool f16;
    int ldq, ldk, ldv;
    const int32_t* cu;
    int group;
    float scale, scale_log2;
    int rel_lo, rel_hi;
    const float* bias;
    int bias_off;
    uint16_t* out;
    int ldo;
    int T;         // rows of the packed buffers (tensor-map extent)
    int kv_heads;  // key/value heads (heads / group)
    int* status;   // device status word (bounded waits)
    int reverse;   // visit the sequences from the last to the first (L2 reuse of the rows written last)
};
// Head dims 32, 64, 128 and 256 (the tcgen05 kernel, attention_tc.cu).
cudaError_t launch_attention(const AttnParams& p, int nseq, int max_len, int heads, int head_dim, cudaStream_t st);
bool attention_tc_supported(int head_dim);
cudaError_t launch_attention_tc(const AttnParams& p, int T, int nseq, int max_len, int heads, int kv_heads,
                                int head_dim, int* status, cudaStream_t st);
// Strict fp32 attention (one warp per query row, fp32 FMA throughout):
// q/k/v are fp32 rows of the fp32 qkv buffer (strides ldq/ldk/ldv); the
// output is written as tf32 hi (out_hi) + fp32 remainder (out_lo), the A
// operand of the 3xTF32 projection that follows.
struct AttnF32Params {
    const float *q, *k, *v;
    int ldq, ldk, ldv;
    const int32_t* cu;
    int group;
    float scale;
    int rel_lo, rel_hi;
    const float* bias;
    int bias_off;
    float *out_hi, *out_lo;  // out_lo nullptr: out_hi receives the unsplit fp32 result
    int ldo;
};
cudaError_t launch_attention_f32(const AttnF32Params& p, int nseq, int max_len, int heads, int head_dim,
                                 cudaStream_t st);


// The status word the kernel-level C ABI entry points pass to their kernels
// (one per device, allocated on first use; read by rg_kernel_status).
cudaError_t kernel_status_word(int dev, int** out);

// Pooling + L2 + Matryoshka truncation (bert.go:657-703, rembed.go:441-448):
// out[nseq x dim].
cudaError_t launch_pool(const float* x32, const int32_t* cu, int nseq, int H, int pooling, int normalize, int dim,
                        float* out, cudaStream_t st);
// The same with the Dense head between pooling and L2 (gemma3.go:177-198):
// pooled -> W1 [D x H] -> W2 [H x D] -> L2 -> truncate, one launch (clusters
// of 8 CTAs share each stage through distributed shared memory).  H and D
// must be multiples of 8.  Without a head (w1 / w2 nullptr) the same kernel
// pools, normalises and truncates: the mean pooling of long sequences is
// then spread over eight CTAs per sequence group instead of one CTA per
// sequence.
cudaError_t launch_pool_head(const float* x32, const int32_t* cu, int nseq, int H, int D, int pooling,
                             const float* w1, const float* w2, int normalize, int dim, float* out, cudaStream_t st);

}  // namespace rg
