// gemm.cu - persistent warp-specialised tcgen05 GEMM for sm_100a.
//
// One CTA per SM walks output tiles (128 x BN) in m-major order so that the
// CTAs in flight share the same A row-blocks through L2.  Roles:
//   warp 0     TMA producer: A and W k-blocks (128 bytes of K per row,
//              128-byte swizzle) into a STAGES-deep shared-memory ring;
//   warp 1     MMA issuer: one thread issues 4 tcgen05.mma per k-block into
//              one of two TMEM accumulators (2 x BN fp32/s32 columns);
//   warp 2     TMEM allocator;
//   warps 4-7  epilogue: tcgen05.ld 32 columns at a time, dequant scales,
//              bias, GELU or residual, global stores; releases the
//              accumulator so the next tile's MMAs overlap this epilogue.
// All waits are bounded (sm100.cuh); on a timeout every role stops, the
// producer drains its in-flight TMA loads, the issuer drains its MMAs, and
// TMEM is freed before the CTA exits with kStatusWaitTimeout raised.
#include <cuda_bf16.h>

#include "gemm.cuh"
#include "sm100.cuh"

namespace rg {

__device__ __forceinline__ float gelu_erf(float x) {
    // HF "gelu": 0.5 x (1 + erf(x / sqrt(2))), the function the reference's
    // geluScalar approximates (tensor.go:499-538).
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

template <int BN, int STAGES, bool S8, int EPI>
__global__ void __launch_bounds__(256, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int A_BYTES = 128 * 128;
    constexpr int B_BYTES = BN * 128;
    constexpr uint32_t TMEM_COLS = 2 * BN;
    constexpr int K_ELEMS = S8 ? 128 : 64;  // elements per 128-byte k-block
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (args.M + 127) / 128;
    const int n_tiles = args.N / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int kblocks = args.K / K_ELEMS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t issued_mask = 0, issued_parity = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int m_blk = tile / n_tiles, n_blk = tile % n_tiles;
            bool ok = true;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&empty[stage], phase ^ 1, args.status, abort_flag)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
                tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * K_ELEMS, m_blk * 128);
                tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * K_ELEMS, n_blk * BN);
                issued_mask |= 1u << stage;
                issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
        }
        // Every issued load has landed before the CTA may exit.
        for (int s = 0; s < STAGES; ++s)
            if (issued_mask & (1u << s)) mbar_drain(&full[s], (issued_parity >> s) & 1);
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = S8 ? idesc_s8(128, BN) : idesc_bf16(128, BN);
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool issued = false;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.status, abort_flag)) break;
            tc_fence_after();
            const uint32_t d = tmem_base + acc * BN;
            bool ok = true;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&full[stage], phase, args.status, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = sdesc_k128(smem_u32(sA + stage * A_BYTES));
                const uint64_t bd = sdesc_k128(smem_u32(sB + stage * B_BYTES));
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    // 32 bytes of K per instruction: +2 in 16-byte units.
                    if constexpr (S8)
                        umma_s8(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
                    else
                        umma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
                }
                issued = true;
                umma_commit(&empty[stage]);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
            umma_commit(&tfull[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (issued) {
            umma_commit(drain);
            mbar_drain(drain, 0);
        }
    } else if (warp >= 4) {
        // ---------------- epilogue ----------------
        const int quarter = warp - 4;  // TMEM lanes [32*quarter, 32*quarter+32)
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int m_blk = tile / n_tiles, n_blk = tile % n_tiles;
            if (!mbar_wait(&tfull[acc], acc_phase, args.status, abort_flag)) break;
            tc_fence_after();
            const int row = m_blk * 128 + quarter * 32 + lane;
            const bool live = row < args.M;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
            const float rs = (args.row_scale && live) ? args.row_scale[row] : 1.0f;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(taddr + c * 32, r);
                tmem_ld_wait();
                if (!live) continue;
                const int col0 = n_blk * BN + c * 32;
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if constexpr (S8)
                        v[i] = static_cast<float>(static_cast<int32_t>(r[i]));
                    else
                        v[i] = __uint_as_float(r[i]);
                }
                if (args.row_scale) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = v[i] * rs;
                }
                if (args.col_scale) {
                    const float4* cs = reinterpret_cast<const float4*>(args.col_scale + col0);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 s = __ldg(cs + i);
                        v[4 * i + 0] *= s.x;
                        v[4 * i + 1] *= s.y;
                        v[4 * i + 2] *= s.z;
                        v[4 * i + 3] *= s.w;
                    }
                }
                if (args.bias) {
                    const float4* bp = reinterpret_cast<const float4*>(args.bias + col0);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 b = __ldg(bp + i);
                        v[4 * i + 0] += b.x;
                        v[4 * i + 1] += b.y;
                        v[4 * i + 2] += b.z;
                        v[4 * i + 3] += b.w;
                    }
                }
                if constexpr (EPI == kEpiBiasGelu) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
                }
                if constexpr (EPI == kEpiBiasRes || EPI == kEpiBiasF32) {
                    float* o = reinterpret_cast<float*>(args.out) + static_cast<size_t>(row) * args.ld_out + col0;
                    if constexpr (EPI == kEpiBiasRes) {
                        const float4* rp = reinterpret_cast<const float4*>(args.residual +
                                                                           static_cast<size_t>(row) * args.N + col0);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 x = __ldg(rp + i);
                            v[4 * i + 0] = x.x + v[4 * i + 0];
                            v[4 * i + 1] = x.y + v[4 * i + 1];
                            v[4 * i + 2] = x.z + v[4 * i + 2];
                            v[4 * i + 3] = x.w + v[4 * i + 3];
                        }
                    }
                    float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
                    for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                } else {
                    __nv_bfloat16* o =
                        reinterpret_cast<__nv_bfloat16*>(args.out) + static_cast<size_t>(row) * args.ld_out + col0;
                    uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t w[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            __nv_bfloat162 p = __floats2bfloat162_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
                            w[j] = *reinterpret_cast<uint32_t*>(&p);
                        }
                        o4[i] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    }

    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Host side.

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
    CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, int STAGES, bool S8, int EPI>
static cudaError_t launch_one(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmArgs& args, int num_sms,
                              cudaStream_t stream) {
    constexpr int smem = STAGES * (128 * 128 + BN * 128) + 1024 + 256;
    auto kern = gemm_kernel<BN, STAGES, S8, EPI>;
    // The shared-memory opt-in is a per-device function attribute.
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 32) __atomic_fetch_or(&configured, 1u << dev, __ATOMIC_RELEASE);
    }
    const int tiles = ((args.M + 127) / 128) * (args.N / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    kern<<<grid, 256, smem, stream>>>(tmA, tmB, args);
    return cudaGetLastError();
}

template <int BN, int STAGES, bool S8>
static cudaError_t dispatch_epi(int epi, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmArgs& args,
                                int num_sms, cudaStream_t stream) {
    switch (epi) {
    case kEpiBias: return launch_one<BN, STAGES, S8, kEpiBias>(tmA, tmB, args, num_sms, stream);
    case kEpiBiasGelu: return launch_one<BN, STAGES, S8, kEpiBiasGelu>(tmA, tmB, args, num_sms, stream);
    case kEpiBiasRes: return launch_one<BN, STAGES, S8, kEpiBiasRes>(tmA, tmB, args, num_sms, stream);
    case kEpiBiasF32: return launch_one<BN, STAGES, S8, kEpiBiasF32>(tmA, tmB, args, num_sms, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemm_launch(GemmKind kind, int epi, const CUtensorMap& tmA, const CUtensorMap& tmB,
                        const GemmArgs& args, int num_sms, cudaStream_t stream) {
    if (args.M <= 0) return cudaSuccess;
    const int kel = kind == GemmKind::kS8 ? 128 : 64;
    if (args.N % 128 != 0 || args.K % kel != 0 || args.K <= 0) return cudaErrorInvalidValue;
    const int bn = gemm_block_n(args.N);
    if (kind == GemmKind::kBF16) {
        if (bn == 256) return dispatch_epi<256, 4, false>(epi, tmA, tmB, args, num_sms, stream);
        return dispatch_epi<128, 6, false>(epi, tmA, tmB, args, num_sms, stream);
    }
    if (bn == 256) return dispatch_epi<256, 4, true>(epi, tmA, tmB, args, num_sms, stream);
    return dispatch_epi<128, 6, true>(epi, tmA, tmB, args, num_sms, stream);
}

}  // namespace rg
