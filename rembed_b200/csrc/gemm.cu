// gemm.cu - host side of the tcgen05 GEMM: tensor maps, tile-width choice
// and the launch switch over operand kinds (kernel in gemm_impl.cuh, one
// translation unit per kind).
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm.cuh"

namespace rg {

template <int KIND>
cudaError_t dispatch_kind(int block_n, int epi, const GemmMaps& m, const GemmArgs& args, int num_sms,
                          cudaStream_t stream);

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

bool make_kmajor_tmap(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols,
                      uint64_t row_stride_elems, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
    if ((row_stride_elems * elem_bytes) % 16 != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_elems * elem_bytes};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem_bytes), box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUtensorMapDataType dt = elem_bytes == 4   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                             : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_w8_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols % 16 != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Output / residual maps: 32 x 32 boxes, rows of 128 bytes (fp32, 128-byte
// swizzle) or 64 bytes (16-bit, 64-byte swizzle), matching the kernel's
// staging-box layout (swz in gemm_impl.cuh).
static bool make_epilogue_tmap(CUtensorMap* map, const void* base, bool f32, bool f16, uint64_t rows,
                               uint64_t cols, uint64_t ld) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
    const uint64_t eb = f32 ? 4 : 2;
    if ((ld * eb) % 16 != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * eb};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : (f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
    CUresult r = fn(map, dt, 2,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int gemm_block_n(int M, int N, int num_sms, bool glu, int head_dim) {
    // Among the tile widths that divide N, the one with the fewest
    // (waves x per-tile cost), where a tile costs about BN + 32 columns of
    // work (the +32 models its fixed epilogue/pipeline overhead).
    const int m_tiles = (M + 255) / 256;
    const int pairs = num_sms / 2;
    int best = 0;
    long best_cost = 0;
    for (int bn : {256, 192, 128}) {
        // RoPE epilogue: whole heads in each half-warp's columns, or (head
        // dim 256) one head per tile
        const bool heads_fit = head_dim <= 0 || (bn / 2) % head_dim == 0 || (head_dim == 256 && bn == 256);
        if (N % bn != 0 || (glu && bn == 192) || !heads_fit) continue;
        const long tiles = static_cast<long>(m_tiles) * (N / bn);
        const long waves = (tiles + pairs - 1) / pairs;
        const long cost = waves * (bn + 32);
        if (best == 0 || cost < best_cost) {
            best = bn;
            best_cost = cost;
        }
    }
    return best;
}

static cudaError_t launch_impl(GemmKind kind, int epi, int block_n, GemmMaps& m, const GemmArgs& args, int num_sms,
                               cudaStream_t stream) {
    if (args.M <= 0) return cudaSuccess;
    const int kel = kind == GemmKind::kS8 ? 128 : (kind == GemmKind::kTF32x3 ? 32 : 64);
    if (args.K % kel != 0 || args.K <= 0 || block_n <= 0 || args.N % block_n != 0) return cudaErrorInvalidValue;
    const bool f32out = epi_has_residual(epi) || epi == kEpiBiasF32 || kind == GemmKind::kTF32x3;
    const bool f16out = kind == GemmKind::kF16 || kind == GemmKind::kW8;
    const bool glu = epi_is_glu(epi);
    // GLU tiles pair 32-column chunks inside each epilogue warp's columns.
    if (glu && (block_n == 192 || args.N % 64 != 0)) return cudaErrorInvalidValue;
    if (!make_epilogue_tmap(&m.out, args.out, f32out, f16out, args.M, glu ? args.N / 2 : args.N, args.ld_out))
        return cudaErrorInvalidValue;
    if (epi == kEpiBiasResLN && (!args.ln_stats || !args.ln_g || !args.ln_b)) return cudaErrorInvalidValue;
    // Folded LayerNorm and the chunk statistics / 16-bit copy of residual
    // outputs: the kinds with 16-bit activations only (kW8: fp16 activations,
    // int8 weights widened in shared memory).
    const bool k16 = kind == GemmKind::kBF16 || kind == GemmKind::kF16 || kind == GemmKind::kW8;
    // (a gated epilogue adds no bias: its folded norm must have none either)
    if (args.fold_stats &&
        (!k16 || !args.fold_c1 ||
         (epi_is_glu(epi) ? false : (!args.bias || (epi != kEpiBias && epi != kEpiBiasGelu && epi != kEpiRope)))))
        return cudaErrorInvalidValue;
    if (epi == kEpiRope &&
        (f32out || args.rope_dh <= 0 || args.rope_dh % 64 != 0 ||
         ((block_n / 2) % args.rope_dh != 0 && !(args.rope_dh == 256 && block_n == 256)) ||
         args.rope_qd % args.rope_dh != 0 || args.rope_kvd % args.rope_dh != 0 || args.rope_npos <= 0 ||
         (reinterpret_cast<uintptr_t>(args.rope_cos) & 15) != 0 || (reinterpret_cast<uintptr_t>(args.rope_sin) & 15) != 0 ||
         !args.rope_cos ||
         !args.rope_sin || !args.positions))
        return cudaErrorInvalidValue;
    if ((args.parts_out || args.out16) && (!k16 || !epi_has_residual(epi))) return cudaErrorInvalidValue;
    if (args.copy_gain && (!args.out16 || (reinterpret_cast<uintptr_t>(args.copy_gain) & 15) != 0))
        return cudaErrorInvalidValue;
    if (args.out16) {
        if (!make_epilogue_tmap(&m.out16, args.out16, false, kind == GemmKind::kF16 || kind == GemmKind::kW8, args.M,
                                args.N, args.ld16))
            return cudaErrorInvalidValue;
    } else {
        m.out16 = m.out;  // unused
    }
    if (epi_has_residual(epi)) {
        if (!args.residual || !make_epilogue_tmap(&m.res, args.residual, true, false, args.M, args.N, args.N))
            return cudaErrorInvalidValue;
    } else {
        m.res = m.out;  // unused
    }
    switch (kind) {
    case GemmKind::kBF16: return dispatch_kind<0>(block_n, epi, m, args, num_sms, stream);
    case GemmKind::kS8: return dispatch_kind<1>(block_n, epi, m, args, num_sms, stream);
    case GemmKind::kF16: return dispatch_kind<2>(block_n, epi, m, args, num_sms, stream);
    case GemmKind::kW8: return dispatch_kind<3>(block_n, epi, m, args, num_sms, stream);
    case GemmKind::kTF32x3: return dispatch_kind<4>(block_n, epi, m, args, num_sms, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemm_launch(GemmKind kind, int epi, int block_n, const CUtensorMap& tmA, const CUtensorMap& tmB,
                        const GemmArgs& args, int num_sms, cudaStream_t stream) {
    if (kind == GemmKind::kTF32x3) return cudaErrorInvalidValue;  // needs the remainder maps
    GemmMaps m;
    m.a = tmA;
    m.b = tmB;
    m.a2 = tmA;  // unused
    m.b2 = tmB;
    return launch_impl(kind, epi, block_n, m, args, num_sms, stream);
}

cudaError_t gemm_launch_tf32x3(int epi, int block_n, const CUtensorMap& tmA, const CUtensorMap& tmA2,
                               const CUtensorMap& tmB, const CUtensorMap& tmB2, const GemmArgs& args, int num_sms,
                               cudaStream_t stream) {
    GemmMaps m;
    m.a = tmA;
    m.b = tmB;
    m.a2 = tmA2;
    m.b2 = tmB2;
    return launch_impl(GemmKind::kTF32x3, epi, block_n, m, args, num_sms, stream);
}

}  // namespace rg
