// kernels.cu - embedding + LayerNorm, residual LayerNorm, int8 row
// quantisation, varlen attention and pooling for the encoder forward pass.
//
// The row kernels (embed_ln, ln, quantize_rows) are HBM-bound: one warp per
// token row, float4 loads, two-pass statistics in registers, one write per
// output.  The attention kernel is a flash-style tiled kernel over the
// packed (cu_seqlens) batch: no FLOPs or bytes are spent on padding.
#include <cuda_bf16.h>
#include <stdint.h>

#include "kernels.cuh"
#include "sm100.cuh"

namespace rg {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Row i of a warp-per-row kernel holds H = 128*NV floats: lane owns the
// float4 chunks lane + 32*c, c < NV (coalesced 512-byte segments).
template <int NV>
__device__ __forceinline__ void ln_finish(float (&v)[NV][4], const float* g, const float* b, float eps, int H,
                                          float* x32_row, __nv_bfloat16* xb_row, int8_t* xq_row, float* xq_scale,
                                          int lane) {
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NV; ++c) s += (v[c][0] + v[c][1]) + (v[c][2] + v[c][3]);
    const float mean = warp_sum(s) / static_cast<float>(H);
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < NV; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float d = v[c][e] - mean;
            q += d * d;
        }
    const float var = warp_sum(q) / static_cast<float>(H);
    const float inv = 1.0f / sqrtf(var + eps);
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int j = (lane + 32 * c) * 4;
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g + j));
        const float4 bb = __ldg(reinterpret_cast<const float4*>(b + j));
        v[c][0] = (v[c][0] - mean) * inv * gg.x + bb.x;
        v[c][1] = (v[c][1] - mean) * inv * gg.y + bb.y;
        v[c][2] = (v[c][2] - mean) * inv * gg.z + bb.z;
        v[c][3] = (v[c][3] - mean) * inv * gg.w + bb.w;
        reinterpret_cast<float4*>(x32_row + j)[0] = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
        __nv_bfloat162 lo = __floats2bfloat162_rn(v[c][0], v[c][1]);
        __nv_bfloat162 hi = __floats2bfloat162_rn(v[c][2], v[c][3]);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        reinterpret_cast<uint2*>(xb_row + j)[0] = pk;
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[c][0]), fabsf(v[c][1])), fmaxf(fabsf(v[c][2]), fabsf(v[c][3]))));
    }
    if (xq_row) {
        // QuantizeRowU8 (pack_vnni.go:85-117) without the +128 offset:
        // float32 scale = maxAbs/127 (1 for a zero row), float32 reciprocal,
        // round-half-even, clamp to the int8 range.
        amax = warp_max(amax);
        float scale = amax / 127.0f;
        if (scale == 0.0f) scale = 1.0f;
        const float rinv = 1.0f / scale;
#pragma unroll
        for (int c = 0; c < NV; ++c) {
            const int j = (lane + 32 * c) * 4;
            char4 o;
            o.x = (signed char)max(-128, min(127, __float2int_rn(v[c][0] * rinv)));
            o.y = (signed char)max(-128, min(127, __float2int_rn(v[c][1] * rinv)));
            o.z = (signed char)max(-128, min(127, __float2int_rn(v[c][2] * rinv)));
            o.w = (signed char)max(-128, min(127, __float2int_rn(v[c][3] * rinv)));
            reinterpret_cast<char4*>(xq_row + j)[0] = o;
        }
        if (lane == 0) *xq_scale = scale;
    }
}

template <int NV>
__global__ void __launch_bounds__(256) embed_ln_kernel(const int64_t* __restrict__ ids, const int32_t* __restrict__ cu,
                                                      int nseq, int T, const float* __restrict__ word,
                                                      const float* __restrict__ pos, const float* __restrict__ type0,
                                                      const float* __restrict__ g, const float* __restrict__ b,
                                                      float eps, int H, int vocab, int pos_off, float* x32,
                                                      __nv_bfloat16* xb, int8_t* xq, float* xq_scale, int* status) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    // Sequence of token t: the last s with cu[s] <= t.
    int lo = 0, hi = nseq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(cu + mid) <= t) lo = mid;
        else hi = mid - 1;
    }
    const int p = t - __ldg(cu + lo) + pos_off;
    int64_t id = __ldg(ids + t);
    const bool bad = id < 0 || id >= vocab;
    if (bad) {
        if (lane == 0) atomicOr(status, kStatusBadToken);
        id = 0;
    }
    const float* w = word + id * H;
    const float* pr = pos + static_cast<int64_t>(p) * H;
    float v[NV][4];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int j = (lane + 32 * c) * 4;
        const float4 a = __ldg(reinterpret_cast<const float4*>(w + j));
        const float4 q = __ldg(reinterpret_cast<const float4*>(pr + j));
        // (word + pos) + type, the reference's summation order.
        v[c][0] = a.x + q.x;
        v[c][1] = a.y + q.y;
        v[c][2] = a.z + q.z;
        v[c][3] = a.w + q.w;
        if (type0) {
            const float4 ty = __ldg(reinterpret_cast<const float4*>(type0 + j));
            v[c][0] += ty.x;
            v[c][1] += ty.y;
            v[c][2] += ty.z;
            v[c][3] += ty.w;
        }
        if (bad) v[c][0] = v[c][1] = v[c][2] = v[c][3] = 0.f;
    }
    ln_finish<NV>(v, g, b, eps, H, x32 + static_cast<int64_t>(t) * H, xb + static_cast<int64_t>(t) * H,
                  xq ? xq + static_cast<int64_t>(t) * H : nullptr, xq_scale ? xq_scale + t : nullptr, lane);
}

template <int NV>
__global__ void __launch_bounds__(256) ln_kernel(const float* __restrict__ y32, const float* __restrict__ g,
                                                const float* __restrict__ b, float eps, int T, int H, float* x32,
                                                __nv_bfloat16* xb, int8_t* xq, float* xq_scale) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const float* y = y32 + static_cast<int64_t>(t) * H;
    float v[NV][4];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(y + (lane + 32 * c) * 4));
        v[c][0] = a.x;
        v[c][1] = a.y;
        v[c][2] = a.z;
        v[c][3] = a.w;
    }
    ln_finish<NV>(v, g, b, eps, H, x32 + static_cast<int64_t>(t) * H, xb + static_cast<int64_t>(t) * H,
                  xq ? xq + static_cast<int64_t>(t) * H : nullptr, xq_scale ? xq_scale + t : nullptr, lane);
}

#define RG_NV_DISPATCH(H, CALL)           \
    switch ((H) / 128) {                  \
    case 1: { constexpr int NV = 1; CALL; } break; \
    case 2: { constexpr int NV = 2; CALL; } break; \
    case 3: { constexpr int NV = 3; CALL; } break; \
    case 4: { constexpr int NV = 4; CALL; } break; \
    case 6: { constexpr int NV = 6; CALL; } break; \
    case 8: { constexpr int NV = 8; CALL; } break; \
    case 12: { constexpr int NV = 12; CALL; } break; \
    case 16: { constexpr int NV = 16; CALL; } break; \
    default: return cudaErrorInvalidValue; \
    }

cudaError_t launch_embed_ln(const int64_t* ids, const int32_t* cu, int nseq, int T, const float* word,
                            const float* pos, const float* type0, const float* g, const float* b, float eps,
                            int H, int vocab, int pos_off, float* x32, __nv_bfloat16* xb, int8_t* xq,
                            float* xq_scale, int* status, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % 128 != 0) return cudaErrorInvalidValue;
    const int grid = (T + 7) / 8;
    RG_NV_DISPATCH(H, (embed_ln_kernel<NV><<<grid, 256, 0, st>>>(ids, cu, nseq, T, word, pos, type0, g, b, eps, H,
                                                                vocab, pos_off, x32, xb, xq, xq_scale, status)));
    return cudaGetLastError();
}

cudaError_t launch_ln(const float* y32, const float* g, const float* b, float eps, int T, int H, float* x32,
                      __nv_bfloat16* xb, int8_t* xq, float* xq_scale, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % 128 != 0) return cudaErrorInvalidValue;
    const int grid = (T + 7) / 8;
    RG_NV_DISPATCH(H, (ln_kernel<NV><<<grid, 256, 0, st>>>(y32, g, b, eps, T, H, x32, xb, xq, xq_scale)));
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// int8 row quantisation of a bf16 matrix (full-int8 mode inputs that are not
// produced by a LayerNorm: the attention context and the GELU output).
__global__ void __launch_bounds__(256) quantize_rows_kernel(const __nv_bfloat16* __restrict__ x, int T, int K,
                                                           int8_t* q, float* scale) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const __nv_bfloat16* row = x + static_cast<int64_t>(t) * K;
    float amax = 0.f;
    for (int j = lane * 8; j < K; j += 256) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + j));
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(p[e]);
            amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
    amax = warp_max(amax);
    float s = amax / 127.0f;
    if (s == 0.0f) s = 1.0f;
    const float rinv = 1.0f / s;
    int8_t* qr = q + static_cast<int64_t>(t) * K;
    for (int j = lane * 8; j < K; j += 256) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + j));
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
        int8_t o[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(p[e]);
            o[2 * e] = (int8_t)max(-128, min(127, __float2int_rn(f.x * rinv)));
            o[2 * e + 1] = (int8_t)max(-128, min(127, __float2int_rn(f.y * rinv)));
        }
        *reinterpret_cast<uint2*>(qr + j) = *reinterpret_cast<uint2*>(o);
    }
    if (lane == 0) scale[t] = s;
}

cudaError_t launch_quantize_rows(const __nv_bfloat16* x, int T, int K, int8_t* q, float* scale, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (K % 8 != 0) return cudaErrorInvalidValue;
    quantize_rows_kernel<<<(T + 7) / 8, 256, 0, st>>>(x, T, K, q, scale);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Attention.  CTA = (64 query rows, head, sequence), 4 warps x 16 rows;
// key/value tiles of 64 rows; S = Q K^T and O += P V on bf16 mma.sync with
// fp32 accumulators; online softmax in the exp2 domain.  Rows of the
// shared tiles are padded by 16 bytes so ldmatrix is conflict-free.
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&p);
}

template <int D>
__device__ __forceinline__ void load_tile64(__nv_bfloat16* s, const __nv_bfloat16* g, int r0, int L, int ld) {
    constexpr int LDS = D + 8;
    constexpr int CPR = D / 8;  // 16-byte chunks per row
    for (int i = threadIdx.x; i < 64 * CPR; i += 128) {
        const int r = i / CPR, c = i % CPR;
        const int gr = r0 + r;
        const bool ok = gr < L;
        const __nv_bfloat16* src = g + static_cast<int64_t>(ok ? gr : 0) * ld + c * 8;
        cp_async16(s + r * LDS + c * 8, src, ok);
    }
}

template <int D>
__global__ void __launch_bounds__(128) attention_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                       const int32_t* __restrict__ cu, int H, float scale_log2,
                                                       __nv_bfloat16* __restrict__ ctx) {
    constexpr int LDS = D + 8;
    constexpr int KS = D / 16;   // k-steps over the head dim
    constexpr int DT = D / 8;    // n-tiles of the output
    __shared__ __align__(16) __nv_bfloat16 sQ[64 * LDS];
    __shared__ __align__(16) __nv_bfloat16 sK[64 * LDS];
    __shared__ __align__(16) __nv_bfloat16 sV[64 * LDS];

    const int s = blockIdx.z, h = blockIdx.y;
    const int s0 = __ldg(cu + s), L = __ldg(cu + s + 1) - s0;
    const int q0 = blockIdx.x * 64;
    if (q0 >= L) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ld = 3 * H;
    const __nv_bfloat16* Qg = qkv + static_cast<int64_t>(s0) * ld + h * D;
    const __nv_bfloat16* Kg = Qg + H;
    const __nv_bfloat16* Vg = Qg + 2 * H;

    load_tile64<D>(sQ, Qg, q0, L, ld);
    cp_async_commit_wait();
    __syncthreads();

    uint32_t qf[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = ks * 16 + (lane >> 4) * 8;
        ldsm_x4(qf[ks], sQ + r * LDS + c);
    }

    float o[DT][4];
#pragma unroll
    for (int i = 0; i < DT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;

    const int nkv = (L + 63) / 64;
    for (int kb = 0; kb < nkv; ++kb) {
        __syncthreads();  // previous tile fully consumed
        load_tile64<D>(sK, Kg, kb * 64, L, ld);
        load_tile64<D>(sV, Vg, kb * 64, L, ld);
        cp_async_commit_wait();
        __syncthreads();

        float sc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t b[4];
                const int r = 16 * j + (lane & 7) + (lane >> 4) * 8;
                const int c = ks * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x4(b, sK + r * LDS + c);
                mma_bf16_16816(sc[2 * j], qf[ks], b[0], b[1]);
                mma_bf16_16816(sc[2 * j + 1], qf[ks], b[2], b[3]);
            }
        }
        // scale into the exp2 domain, mask keys past the sequence end
        float tm0 = -1e30f, tm1 = -1e30f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int col = kb * 64 + nt * 8 + (lane & 3) * 2 + e;
                const bool ok = col < L;
                sc[nt][e] = ok ? sc[nt][e] * scale_log2 : -1e30f;
                sc[nt][2 + e] = ok ? sc[nt][2 + e] * scale_log2 : -1e30f;
                tm0 = fmaxf(tm0, sc[nt][e]);
                tm1 = fmaxf(tm1, sc[nt][2 + e]);
            }
        }
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 1));
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 2));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 1));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 2));
        const float nm0 = fmaxf(m0, tm0), nm1 = fmaxf(m1, tm1);
        const float c0 = exp2f(m0 - nm0), c1 = exp2f(m1 - nm1);
        m0 = nm0;
        m1 = nm1;
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int i = 0; i < DT; ++i) {
            o[i][0] *= c0;
            o[i][1] *= c0;
            o[i][2] *= c1;
            o[i][3] *= c1;
        }
        uint32_t pf[4][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const float p0 = exp2f(sc[nt][0] - m0), p1 = exp2f(sc[nt][1] - m0);
            const float p2 = exp2f(sc[nt][2] - m1), p3 = exp2f(sc[nt][3] - m1);
            l0 += p0 + p1;
            l1 += p2 + p3;
            pf[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(p0, p1);
            pf[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(p2, p3);
        }
        // O += P V over the 4 key sub-blocks of 16
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t a[4] = {pf[j][0], pf[j][1], pf[j][2], pf[j][3]};
#pragma unroll
            for (int i = 0; i < DT / 2; ++i) {
                uint32_t b[4];
                const int r = 16 * j + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int c = 16 * i + (lane >> 4) * 8;
                ldsm_x4_t(b, sV + r * LDS + c);
                mma_bf16_16816(o[2 * i], a, b[0], b[1]);
                mma_bf16_16816(o[2 * i + 1], a, b[2], b[3]);
            }
        }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
    const int r0 = q0 + warp * 16 + (lane >> 2);
    __nv_bfloat16* out = ctx + static_cast<int64_t>(s0) * H + h * D + (lane & 3) * 2;
#pragma unroll
    for (int i = 0; i < DT; ++i) {
        if (r0 < L)
            *reinterpret_cast<uint32_t*>(out + static_cast<int64_t>(r0) * H + i * 8) =
                pack_bf16(o[i][0] * i0, o[i][1] * i0);
        if (r0 + 8 < L)
            *reinterpret_cast<uint32_t*>(out + static_cast<int64_t>(r0 + 8) * H + i * 8) =
                pack_bf16(o[i][2] * i1, o[i][3] * i1);
    }
}

cudaError_t launch_attention(const __nv_bfloat16* qkv, const int32_t* cu, int nseq, int max_len, int H, int heads,
                             int head_dim, float scale, __nv_bfloat16* ctx, cudaStream_t st) {
    if (nseq <= 0) return cudaSuccess;
    const dim3 grid((max_len + 63) / 64, heads, nseq);
    const float sl2 = scale * 1.4426950408889634f;
    if (head_dim == 64)
        attention_kernel<64><<<grid, 128, 0, st>>>(qkv, cu, H, sl2, ctx);
    else if (head_dim == 32)
        attention_kernel<32><<<grid, 128, 0, st>>>(qkv, cu, H, sl2, ctx);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Pooling + L2 + truncate: one CTA per sequence.
__global__ void __launch_bounds__(256) pool_kernel(const float* __restrict__ x32, const int32_t* __restrict__ cu,
                                                  int H, int pooling, int normalize, int dim, float* __restrict__ out) {
    extern __shared__ float pooled[];  // [H]
    __shared__ double red[8];
    const int s = blockIdx.x;
    const int s0 = __ldg(cu + s), L = __ldg(cu + s + 1) - s0;
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
        float v;
        if (pooling == 1) {  // cls: first token
            v = x32[static_cast<int64_t>(s0) * H + j];
        } else if (pooling == 2) {  // lasttoken
            v = x32[static_cast<int64_t>(s0 + L - 1) * H + j];
        } else {  // mean, poolMean (bert.go:692-703): sequential sum, times 1/L
            float acc = 0.f;
            for (int i = 0; i < L; ++i) acc += x32[static_cast<int64_t>(s0 + i) * H + j];
            v = acc * (1.0f / static_cast<float>(L));
        }
        pooled[j] = v;
    }
    __syncthreads();
    auto block_sumsq = [&](int n) -> double {
        double a = 0.0;
        for (int j = threadIdx.x; j < n; j += blockDim.x) a += static_cast<double>(pooled[j]) * pooled[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
        __syncthreads();
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        __syncthreads();
        return t;
    };
    if (normalize) {  // L2Normalize (tensor.go:542-554): float64 sum, float32 scale
        const double ss = block_sumsq(H);
        if (ss != 0.0) {
            const float inv = static_cast<float>(1.0 / sqrt(ss));
            for (int j = threadIdx.x; j < H; j += blockDim.x) pooled[j] *= inv;
        }
        __syncthreads();
    }
    if (dim < H) {  // Matryoshka truncate: keep dim, re-normalise (rembed.go:441-448)
        const double ss = block_sumsq(dim);
        if (ss != 0.0) {
            const float inv = static_cast<float>(1.0 / sqrt(ss));
            for (int j = threadIdx.x; j < dim; j += blockDim.x) pooled[j] *= inv;
        }
        __syncthreads();
    }
    for (int j = threadIdx.x; j < dim; j += blockDim.x) out[static_cast<int64_t>(s) * dim + j] = pooled[j];
}

cudaError_t launch_pool(const float* x32, const int32_t* cu, int nseq, int H, int pooling, int normalize, int dim,
                        float* out, cudaStream_t st) {
    if (nseq <= 0) return cudaSuccess;
    pool_kernel<<<nseq, 256, H * sizeof(float), st>>>(x32, cu, H, pooling, normalize, dim, out);
    return cudaGetLastError();
}

}  // namespace rg
