// gemm.cuh - the dense projection of rembed's applyDense
// (internal/model/bert.go:282-301) as one persistent tcgen05 GEMM with a
// fused epilogue:  out[M x N] = epi(A[M x K] . W[N x K]^T).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace rg {

enum Epilogue : int {
    kEpiBias = 0,       // + bias                      -> bf16
    kEpiBiasGelu = 1,   // + bias, exact (erf) GELU    -> bf16
    kEpiBiasRes = 2,    // + bias, + fp32 residual     -> fp32 (out may alias the residual)
    kEpiBiasF32 = 3,    // + bias                      -> fp32
    // Gated linear units over W rows interleaved in blocks of 32: block 2j
    // is the activated operand a, block 2j+1 the linear operand b of the
    // same 32 output columns; out[M x N/2] = act(a) * b -> bf16.
    kEpiGluSilu = 4,      // silu(a) * b   (qwen3.go:530-539, nomic.go:232-242)
    kEpiGluGeluErf = 5,   // gelu(a) * b   (modernbert.go:292-301)
    kEpiGluGeluTanh = 6,  // gelu_tanh(a) * b (gemma3.go:365-374)
    // + bias, + LayerNorm(fp32 residual) rebuilt on load from the row's
    // (mean, rstd) and the norm's gain/bias: (r - mean) * rstd * g + b, the
    // LayerNorm output of a post-norm stack that was never written out in
    // fp32 (bert.go:905-918)                                   -> fp32 (out may alias the residual)
    kEpiBiasResLN = 7,
    // + bias (or the folded norm), then per head of rope_dh columns the Q
    // heads (columns [0, rope_qd)) and K heads ([rope_qd, rope_qd +
    // rope_kvd)) rotated by the token's position (rotate-half RoPE,
    // modernbert.go:125-143, products rounded before the add); V heads pass
    // through                                                  -> bf16 / fp16
    kEpiRope = 8,
};
inline bool epi_is_glu(int epi) { return epi >= kEpiGluSilu && epi <= kEpiGluGeluTanh; }
inline bool epi_has_residual(int epi) { return epi == kEpiBiasRes || epi == kEpiBiasResLN; }

struct GemmArgs {
    int M, N, K;
    const float* bias;       // [N] or nullptr
    const float* col_scale;  // [N] or nullptr: int8 weight dequant scale
    const float* row_scale;  // [M] or nullptr: int8 activation dequant scale
    const float* residual;   // [M x N] fp32, kEpiBiasRes / kEpiBiasResLN
    const float2* ln_stats;  // [M] (mean, rstd), kEpiBiasResLN
    const float *ln_g, *ln_b;  // [N], kEpiBiasResLN
    void* out;               // [M x ld_out], 16-bit (bf16 / fp16 by kind) or fp32
    int ld_out;
    int* status;             // device status word
    // Norm folded into this GEMM (kEpiBias / kEpiBiasGelu, and the gated
    // epilogues for bias-free norms): A holds the unnormalised rows y and W
    // the weight times the norm's gain; with the row's (mean, rstd) from
    // fold_stats (mean 0 for an RMSNorm) the epilogue computes
    // rstd * acc + (bias[n] - rstd * mean * fold_c1[n]) (bias = W.beta + b;
    // the gated epilogues apply it to both halves without a bias).
    const float2* fold_stats;  // [M] (mean, rstd)
    const float* fold_c1;      // [N] column sums of the folded 16-bit weight
    // residual epilogues: also write the output as 16 bits (out16, row
    // stride ld16) and the (mean, M2) of each 32-column chunk of each row
    // (parts_out: [N / 32 x M], chunk-major)
    uint16_t* out16;
    int ld16;
    float2* parts_out;
    // optional with out16: the copy is round16(y[n] * copy_gain[n]) (a
    // folded LayerNorm whose gain cannot go into the consumer's weight: the
    // weight-only int8 mode keeps the reference's quantised weight)
    const float* copy_gain;
    // Failure injection for tests (zero in production): wait_limit > 0
    // bounds every mbarrier wait of the launch at that many cycles instead of
    // about a second, and inject_withhold makes the even CTA of every pair
    // withhold its arrival on the first k-block of its first tile, so the
    // MMA issuer's wait runs out and the launch ends with kStatusWaitTimeout.
    long long wait_limit;
    int inject_withhold;
    // Walk the row blocks from the last to the first (see the forward's
    // L2-aware ordering): the output is the same, only the order of tiles.
    int reverse_m;
    // kEpiRope: the RoPE tables laid out [rope_dh / 8][rope_npos][4] (entry
    // (p, d) at ((d / 4) * rope_npos + p) * 4 + d % 4: lanes on consecutive
    // positions read one contiguous run), each row's position in its
    // sequence, and the head layout of the Q|K|V output.
    const float *rope_cos, *rope_sin;
    const int32_t* positions;
    int rope_dh, rope_qd, rope_kvd, rope_npos;
    // kEpiRope, optional (Qwen3): an RMSNorm of each Q / K head over its dh
    // values (gains q_norm / k_norm, eps rope_eps) before the rotation
    const float *q_norm, *k_norm;
    float rope_eps;
};

// Operand element kind of the GEMM.
//   kBF16: bf16 A and W, bf16 output.
//   kS8:   int8 A (row scales) and int8 W (column scales), bf16 output.
//   kF16:  fp16 A and W, fp16 output.
//   kW8:   fp16 A, int8 W (column scales) widened to fp16 in shared memory
//          inside the mainloop, fp16 output.
//   kTF32x3: fp32 A and W as tf32-exact hi parts plus fp32 remainders,
//          kind::tf32 over K three times (A_hi W_hi + A_hi W_lo + A_lo W_hi),
//          fp32 output for every epilogue (the strict-fp32 mode).
enum class GemmKind : int { kBF16 = 0, kS8 = 1, kF16 = 2, kW8 = 3, kTF32x3 = 4 };

// Tensor maps one launch reads: A, W, the output and residual boxes, for
// kTF32x3 the remainder parts of A (a2) and W (b2), and the residual
// epilogues' 16-bit copy (out16).
struct GemmMaps {
    CUtensorMap a, b, out, res, a2, b2, out16;
};

// Encode a 2-D K-major tensor map over a row-major [rows x cols] matrix
// (cols contiguous) with a (128-byte x box_rows) box and 128-byte swizzle.
// elem_bytes: 4 (fp32), 2 (bf16 / fp16) or 1 (int8).  Returns false on failure.
bool make_kmajor_tmap(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols,
                      uint64_t row_stride_elems, uint32_t box_rows);
// Tensor map over an int8 weight [rows x cols] for GemmKind::kW8: boxes of
// 64 bytes of K x box_rows, unswizzled.
bool make_w8_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);

// Output tile width (128, 192 or 256 columns) for an M x N GEMM on num_sms
// SMs: the width dividing N with the least wave-quantised cost; 0 if none
// divides N.  head_dim > 0: only widths whose per-warp half (block_n / 2)
// holds whole heads of that many columns (kEpiRope).
int gemm_block_n(int M, int N, int num_sms, bool glu = false, int head_dim = 0);

// Rows of W one CTA loads per k-block: each CTA of the pair holds half of a
// tile's block_n columns.  The tensor map over W must use this box height.
inline int gemm_w_box_rows(int block_n) { return block_n / 2; }

// Launch the GEMM with tiles of 256 x block_n on CTA pairs.  tmA covers A
// [M x K] with box rows 128; tmB covers W [N x K] with box rows
// gemm_w_box_rows(block_n) (make_w8_tmap for kW8).  Requires K a multiple of
// 64 (128 for kS8) and N % block_n == 0.
cudaError_t gemm_launch(GemmKind kind, int epi, int block_n, const CUtensorMap& tmA, const CUtensorMap& tmB,
                        const GemmArgs& args, int num_sms, cudaStream_t stream);
// kTF32x3: tmA / tmB over the hi parts, tmA2 / tmB2 over the remainders
// (fp32 maps, box 32 elements x rows, 128-byte swizzle; K % 32 == 0).
cudaError_t gemm_launch_tf32x3(int epi, int block_n, const CUtensorMap& tmA, const CUtensorMap& tmA2,
                               const CUtensorMap& tmB, const CUtensorMap& tmB2, const GemmArgs& args, int num_sms,
                               cudaStream_t stream);

}  // namespace rg
