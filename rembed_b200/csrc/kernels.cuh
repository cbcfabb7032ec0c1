// kernels.cuh - the non-GEMM kernels of the encoder forward pass.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rg {

// Per-token embedding sum + LayerNorm (bert.go:795-814):
//   x = LN(word[id] + pos[p + pos_off] (+ type[0]))
// writes fp32 x32 and its bf16 copy xb; p is the token's index inside its
// sequence (cu_seqlens).  A token id outside [0, vocab) raises
// kStatusBadToken and writes zeros (never reads out of bounds).
cudaError_t launch_embed_ln(const int64_t* ids, const int32_t* cu, int nseq, int T, const float* word,
                            const float* pos, const float* type0, const float* g, const float* b, float eps,
                            int H, int vocab, int pos_off, float* x32, __nv_bfloat16* xb, int8_t* xq,
                            float* xq_scale, int* status, cudaStream_t st);

// LayerNorm of y32 rows (tensor.go:433-452) -> x32 (fp32) and xb (bf16);
// optionally also the per-row int8 quantisation of the fp32 result (xq,
// xq_scale) for the full-int8 mode (QuantizeRowU8, pack_vnni.go:85-117).
cudaError_t launch_ln(const float* y32, const float* g, const float* b, float eps, int T, int H, float* x32,
                      __nv_bfloat16* xb, int8_t* xq, float* xq_scale, cudaStream_t st);

// Per-row symmetric int8 quantisation of a bf16 [T x K] matrix
// (QuantizeRowU8 with the +128 offset removed: q in [-128, 127]).
cudaError_t launch_quantize_rows(const __nv_bfloat16* x, int T, int K, int8_t* q, float* scale, cudaStream_t st);

// Bidirectional varlen attention over the fused qkv buffer [T x 3H]
// (bert.go:853-902): per sequence and head, softmax(Q K^T * scale) V.
// Writes ctx [T x H] bf16.  head_dim 32 or 64.
cudaError_t launch_attention(const __nv_bfloat16* qkv, const int32_t* cu, int nseq, int max_len, int H,
                             int heads, int head_dim, float scale, __nv_bfloat16* ctx, cudaStream_t st);

// Pooling + L2 + Matryoshka truncation (bert.go:657-703, rembed.go:441-448):
// out[nseq x dim].
cudaError_t launch_pool(const float* x32, const int32_t* cu, int nseq, int H, int pooling, int normalize, int dim,
                        float* out, cudaStream_t st);

}  // namespace rg
