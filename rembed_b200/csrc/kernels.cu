// kernels.cu - embedding + LayerNorm, residual LayerNorm, int8 row
// quantisation, varlen attention and pooling for the encoder forward pass.
//
// The row kernels (embed_ln, ln, quantize_rows) are HBM-bound: one warp per
// token row, float4 loads, two-pass statistics in registers, one write per
// output.  The attention kernel is a flash-style tiled kernel over the
// packed (cu_seqlens) batch: no FLOPs or bytes are spent on padding.
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>

#include "kernels.cuh"
#include "pdl.cuh"
#include "act16.cuh"
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
//
// Normalise the row in registers (LayerNorm, tensor.go:433-452: two-pass
// mean / biased variance; or RMSNorm, tensor.go:459-471: mean square) with
// gain g and bias b (LayerNorm only; nullptr = zero; g nullptr = identity),
// then write any of:
// fp32 row, bf16 row, int8 row + scale (QuantizeRowU8 without the +128
// offset, pack_vnni.go:85-117).
// Returns true (in every lane) if an fp16 output overflowed or was NaN.
template <int NV, bool RMS, bool F16>
__device__ __forceinline__ bool norm_finish(float (&v)[NV][4], const float* g, const float* b, float eps, int H,
                                            float* out32, uint16_t* outb, int8_t* outq, float* outqs, int lane,
                                            float2* stats = nullptr, float* outhi = nullptr,
                                            float* outlo = nullptr) {
    float mean = 0.f, inv = 1.f;
    if (!g) {
        // identity (ModernBERT's layer-0 attention norm): only the stores
    } else if constexpr (RMS) {
        float q = 0.f;
#pragma unroll
        for (int c = 0; c < NV; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) q += v[c][e] * v[c][e];
        inv = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(H) + eps);
    } else {
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < NV; ++c) s += (v[c][0] + v[c][1]) + (v[c][2] + v[c][3]);
        mean = warp_sum(s) / static_cast<float>(H);
        float q = 0.f;
#pragma unroll
        for (int c = 0; c < NV; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float d = v[c][e] - mean;
                q += d * d;
            }
        inv = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(H) + eps);
    }
    if (stats && lane == 0) *stats = make_float2(mean, inv);
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int j = (lane + 32 * c) * 4;
        const float4 gg = g ? __ldg(reinterpret_cast<const float4*>(g + j)) : make_float4(1.f, 1.f, 1.f, 1.f);
        float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
        if (!RMS && b) bb = __ldg(reinterpret_cast<const float4*>(b + j));
        if constexpr (RMS) {
            v[c][0] = v[c][0] * inv * gg.x;
            v[c][1] = v[c][1] * inv * gg.y;
            v[c][2] = v[c][2] * inv * gg.z;
            v[c][3] = v[c][3] * inv * gg.w;
        } else {
            v[c][0] = (v[c][0] - mean) * inv * gg.x + bb.x;
            v[c][1] = (v[c][1] - mean) * inv * gg.y + bb.y;
            v[c][2] = (v[c][2] - mean) * inv * gg.z + bb.z;
            v[c][3] = (v[c][3] - mean) * inv * gg.w + bb.w;
        }
        if (out32) reinterpret_cast<float4*>(out32 + j)[0] = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
        if (outb)
            reinterpret_cast<uint2*>(outb + j)[0] =
                make_uint2(pack2<F16>(v[c][0], v[c][1]), pack2<F16>(v[c][2], v[c][3]));
        if (outhi) {
            float4 h, l;
            tf32_split(v[c][0], h.x, l.x);
            tf32_split(v[c][1], h.y, l.y);
            tf32_split(v[c][2], h.z, l.z);
            tf32_split(v[c][3], h.w, l.w);
            reinterpret_cast<float4*>(outhi + j)[0] = h;
            reinterpret_cast<float4*>(outlo + j)[0] = l;
        }
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[c][0]), fabsf(v[c][1])), fmaxf(fabsf(v[c][2]), fabsf(v[c][3]))));
    }
    if (outq) {
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
            reinterpret_cast<char4*>(outq + j)[0] = o;
        }
        if (lane == 0) *outqs = scale;
    }
    if constexpr (F16) return outb && __any_sync(0xffffffffu, !(amax <= 65504.0f));
    return false;
}

template <int NV, bool F16>
__device__ __forceinline__ bool store_row(const float (&v)[NV][4], float* out32, uint16_t* outb, int lane) {
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int j = (lane + 32 * c) * 4;
        if (out32) reinterpret_cast<float4*>(out32 + j)[0] = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
        if (outb)
            reinterpret_cast<uint2*>(outb + j)[0] =
                make_uint2(pack2<F16>(v[c][0], v[c][1]), pack2<F16>(v[c][2], v[c][3]));
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[c][0]), fabsf(v[c][1])), fmaxf(fabsf(v[c][2]), fabsf(v[c][3]))));
    }
    if constexpr (F16) return outb && __any_sync(0xffffffffu, !(amax <= 65504.0f));
    return false;
}

__device__ __forceinline__ int seq_of_token(const int32_t* __restrict__ cu, int nseq, int t) {
    int lo = 0, hi = nseq - 1;  // the last s with cu[s] <= t
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(cu + mid) <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

template <int NV, bool F16>
__global__ void __launch_bounds__(256) embed_kernel(EmbedParams p) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= p.T) return;
    const int H = p.H;
    int64_t id = __ldg(p.ids + t);
    const bool bad = id < 0 || id >= p.vocab;
    if (bad) {
        if (lane == 0) atomicOr(p.status, kStatusBadToken);
        id = 0;
    }
    const float* w = p.word + id * H;
    const float* pr = nullptr;
    if (p.pos || p.pos_out) {
        const int s = seq_of_token(p.cu, p.nseq, t);
        const int posn = t - __ldg(p.cu + s);
        if (p.pos) pr = p.pos + static_cast<int64_t>(posn + p.pos_off) * H;
        if (p.pos_out && lane == 0) p.pos_out[t] = posn;
    }
    float v[NV][4];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int j = (lane + 32 * c) * 4;
        const float4 a = __ldg(reinterpret_cast<const float4*>(w + j));
        v[c][0] = a.x;
        v[c][1] = a.y;
        v[c][2] = a.z;
        v[c][3] = a.w;
        if (pr) {  // (word + pos) + type, the reference's summation order
            const float4 q = __ldg(reinterpret_cast<const float4*>(pr + j));
            v[c][0] += q.x;
            v[c][1] += q.y;
            v[c][2] += q.z;
            v[c][3] += q.w;
        }
        if (p.type0) {
            const float4 ty = __ldg(reinterpret_cast<const float4*>(p.type0 + j));
            v[c][0] += ty.x;
            v[c][1] += ty.y;
            v[c][2] += ty.z;
            v[c][3] += ty.w;
        }
        if (p.scale != 1.0f) {  // Gemma's sqrt(H) (gemma3.go:264-275)
            v[c][0] *= p.scale;
            v[c][1] *= p.scale;
            v[c][2] *= p.scale;
            v[c][3] *= p.scale;
        }
        if (bad) v[c][0] = v[c][1] = v[c][2] = v[c][3] = 0.f;
    }
    float* x32 = p.x32 + static_cast<int64_t>(t) * H;
    uint16_t* xb = p.xb ? p.xb + static_cast<int64_t>(t) * H : nullptr;
    bool overflow;
    if (p.g)
        overflow = norm_finish<NV, false, F16>(v, p.g, p.b, p.eps, H, x32, xb,
                                               p.xq ? p.xq + static_cast<int64_t>(t) * H : nullptr,
                                               p.xq_scale ? p.xq_scale + t : nullptr, lane, nullptr,
                                               p.xhi ? p.xhi + static_cast<int64_t>(t) * H : nullptr,
                                               p.xlo ? p.xlo + static_cast<int64_t>(t) * H : nullptr);
    else
        overflow = store_row<NV, F16>(v, x32, xb, lane);
    if (overflow && lane == 0) atomicOr(p.status, kStatusF16Overflow);
}

template <int NV, bool RMS, bool F16>
__global__ void __launch_bounds__(256) norm_kernel(NormParams p) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= p.T) return;
    const int64_t off = static_cast<int64_t>(t) * p.H;
    int64_t ioff = off;
    if (p.row_pick) {
        int row = p.row_pick == 1 ? __ldg(p.row_cu + t) : __ldg(p.row_cu + t + 1) - 1;
        row = min(max(row, 0), p.in_rows - 1);
        ioff = static_cast<int64_t>(row) * p.H;
    }
    float v[NV][4];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p.in + ioff + (lane + 32 * c) * 4));
        v[c][0] = a.x;
        v[c][1] = a.y;
        v[c][2] = a.z;
        v[c][3] = a.w;
    }
    const bool overflow = norm_finish<NV, RMS, F16>(v, p.g, p.b, p.eps, p.H, p.out32 ? p.out32 + off : nullptr,
                                                    p.outb ? p.outb + off : nullptr, p.outq ? p.outq + off : nullptr,
                                                    p.outqs ? p.outqs + t : nullptr, lane, p.stats ? p.stats + t : nullptr,
                                                    p.outhi ? p.outhi + off : nullptr, p.outlo ? p.outlo + off : nullptr);
    if (overflow && p.status && lane == 0) atomicOr(p.status, kStatusF16Overflow);
}

// x32 += RMSNorm(o32; g): Gemma's post-attention / post-FFN norm of the
// sublayer output before the residual add (gemma3.go:357-358, 376).  With
// NEXT the kernel also applies the norm that reads the new residual stream
// next (the pre-FFN norm, or the next layer's input norm: gemma3.go:359, 300)
// to the row it holds in registers and writes that norm's outputs (the next
// GEMM's A operand) as norm_kernel would from x32: the same values in the
// same order, so the same bits, without reading x32 again.
template <int NV, bool NEXT, bool F16>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(float* __restrict__ x32, const float* __restrict__ o32,
                                                         const float* __restrict__ g, float eps, int T, int H,
                                                         NormParams nx) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const int64_t off = static_cast<int64_t>(t) * H;
    float v[NV][4];
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(o32 + off + (lane + 32 * c) * 4));
        v[c][0] = a.x;
        v[c][1] = a.y;
        v[c][2] = a.z;
        v[c][3] = a.w;
        q += (a.x * a.x + a.y * a.y) + (a.z * a.z + a.w * a.w);
    }
    const float inv = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(H) + eps);
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int j = (lane + 32 * c) * 4;
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g + j));
        float4* xp = reinterpret_cast<float4*>(x32 + off + j);
        float4 x = *xp;
        x.x += v[c][0] * inv * gg.x;
        x.y += v[c][1] * inv * gg.y;
        x.z += v[c][2] * inv * gg.z;
        x.w += v[c][3] * inv * gg.w;
        *xp = x;
        v[c][0] = x.x;
        v[c][1] = x.y;
        v[c][2] = x.z;
        v[c][3] = x.w;
    }
    if constexpr (NEXT) {
        const bool overflow = norm_finish<NV, true, F16>(
            v, nx.g, nullptr, nx.eps, H, nullptr, nx.outb ? nx.outb + off : nullptr, nx.outq ? nx.outq + off : nullptr,
            nx.outqs ? nx.outqs + t : nullptr, lane, nullptr, nx.outhi ? nx.outhi + off : nullptr,
            nx.outlo ? nx.outlo + off : nullptr);
        if (overflow && nx.status && lane == 0) atomicOr(nx.status, kStatusF16Overflow);
    }
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

cudaError_t launch_embed(const EmbedParams& p, cudaStream_t st) {
    if (p.T <= 0) return cudaSuccess;
    if (p.H % 128 != 0) return cudaErrorInvalidValue;
    const int grid = (p.T + 7) / 8;
    if (p.f16) {
        RG_NV_DISPATCH(p.H, (launch_pdl(embed_kernel<NV, true>, dim3(grid), dim3(256), 0, st, p)));
    } else {
        RG_NV_DISPATCH(p.H, (launch_pdl(embed_kernel<NV, false>, dim3(grid), dim3(256), 0, st, p)));
    }
    return cudaGetLastError();
}

cudaError_t launch_norm(const NormParams& p, bool rms, cudaStream_t st) {
    if (p.T <= 0) return cudaSuccess;
    if (p.H % 128 != 0) return cudaErrorInvalidValue;
    const int grid = (p.T + 7) / 8;
    if (rms && p.f16) {
        RG_NV_DISPATCH(p.H, (launch_pdl(norm_kernel<NV, true, true>, dim3(grid), dim3(256), 0, st, p)));
    } else if (rms) {
        RG_NV_DISPATCH(p.H, (launch_pdl(norm_kernel<NV, true, false>, dim3(grid), dim3(256), 0, st, p)));
    } else if (p.f16) {
        RG_NV_DISPATCH(p.H, (launch_pdl(norm_kernel<NV, false, true>, dim3(grid), dim3(256), 0, st, p)));
    } else {
        RG_NV_DISPATCH(p.H, (launch_pdl(norm_kernel<NV, false, false>, dim3(grid), dim3(256), 0, st, p)));
    }
    return cudaGetLastError();
}

cudaError_t launch_ln(const float* y32, const float* g, const float* b, float eps, int T, int H, float* x32,
                      uint16_t* xb, bool f16, int8_t* xq, float* xq_scale, cudaStream_t st, int* status) {
    NormParams p{};
    p.f16 = f16;
    p.status = status;
    p.in = y32;
    p.g = g;
    p.b = b;
    p.eps = eps;
    p.T = T;
    p.H = H;
    p.out32 = x32;
    p.outb = xb;
    p.outq = xq;
    p.outqs = xq_scale;
    return launch_norm(p, false, st);
}

cudaError_t launch_add_rmsnorm(float* x32, const float* o32, const float* g, float eps, int T, int H, cudaStream_t st,
                               const NormParams* next) {
    if (T <= 0) return cudaSuccess;
    if (H % 128 != 0) return cudaErrorInvalidValue;
    const int grid = (T + 7) / 8;
    NormParams nx{};
    if (next) nx = *next;
    if (!next) {
        RG_NV_DISPATCH(H, (launch_pdl(add_rmsnorm_kernel<NV, false, false>, dim3(grid), dim3(256), 0, st, x32, o32, g,
                                      eps, T, H, nx)));
    } else if (next->f16) {
        RG_NV_DISPATCH(H, (launch_pdl(add_rmsnorm_kernel<NV, true, true>, dim3(grid), dim3(256), 0, st, x32, o32, g,
                                      eps, T, H, nx)));
    } else {
        RG_NV_DISPATCH(H, (launch_pdl(add_rmsnorm_kernel<NV, true, false>, dim3(grid), dim3(256), 0, st, x32, o32, g,
                                      eps, T, H, nx)));
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// QK-norm + RoPE in place on the q and k heads of the fused qkv buffer: one
// warp per token, over all its q and k heads.  A unit is 8 consecutive dims
// d in [8j, 8j + 8) of a head and their rotate-half partners d + dh/2: two
// 16-byte vectors (32 bytes for fp32).  A head has U = dh/16 units, held by
// U consecutive lanes (U divides 32), so the head's RMS (qwen3.go:485-508,
// gemma3.go:303-330) reduces with U-lane shuffles; then the rotation at the
// token's position in its sequence (modernbert.go:125-143: products rounded
// before the add/sub).
template <bool F16, bool F32>
__device__ __forceinline__ void load8(const void* base, int64_t off, float (&v)[8]) {
    if constexpr (F32) {
        const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
        const float4 a = q[0], b = q[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + off);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = unpack2<F16>(w[e]);
            v[2 * e] = f.x;
            v[2 * e + 1] = f.y;
        }
    }
}
template <bool F16, bool F32>
__device__ __forceinline__ float store8(void* base, int64_t off, const float (&v)[8]) {
    if constexpr (F32) {
        float4* q = reinterpret_cast<float4*>(static_cast<float*>(base) + off);
        q[0] = make_float4(v[0], v[1], v[2], v[3]);
        q[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + off) =
            make_uint4(pack2<F16>(v[0], v[1]), pack2<F16>(v[2], v[3]), pack2<F16>(v[4], v[5]),
                       pack2<F16>(v[6], v[7]));
    }
    float a = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) a = fmaxf(a, fabsf(v[e]));
    return a;
}

template <int DH, bool F16, bool F32>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(QkRopeParams p) {
    pdl_trigger();
    pdl_wait();
    constexpr int HALF = DH / 2, U = DH / 16;
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= p.T) return;
    void* base = F32 ? static_cast<void*>(p.qkv32) : static_cast<void*>(p.qkv);
    const int64_t row = static_cast<int64_t>(t) * p.ld;
    const float* cs = nullptr;
    const float* sn = nullptr;
    if (p.cos) {
        const int s = seq_of_token(p.cu, p.nseq, t);
        const int pos = t - __ldg(p.cu + s);
        cs = p.cos + static_cast<int64_t>(pos) * HALF;
        sn = p.sin + static_cast<int64_t>(pos) * HALF;
    }
    const int heads = p.nq + p.nkv;
    float amax = 0.f;
    for (int u0 = 0; u0 < heads * U; u0 += 32) {
        const int u = u0 + lane;
        const bool on = u < heads * U;  // lanes past the last head still join the shuffles
        const int h = on ? u / U : 0, j = u % U;
        const bool is_q = h < p.nq;
        const int64_t off = row + (is_q ? h * DH : p.nq * DH + (h - p.nq) * DH) + 8 * j;
        float x1[8], x2[8];
        if (on) {
            load8<F16, F32>(base, off, x1);
            load8<F16, F32>(base, off + HALF, x2);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) x1[e] = x2[e] = 0.f;
        }
        const float* g = is_q ? p.q_norm : p.k_norm;
        if (p.q_norm || p.k_norm) {
            float q = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) q += x1[e] * x1[e] + x2[e] * x2[e];
#pragma unroll
            for (int o = U / 2; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            if (on && g) {
                const float inv = 1.0f / sqrtf(q / static_cast<float>(DH) + p.eps);
                const float4* g1 = reinterpret_cast<const float4*>(g + 8 * j);
                const float4* g2 = reinterpret_cast<const float4*>(g + HALF + 8 * j);
                const float4 a0 = __ldg(g1), a1 = __ldg(g1 + 1), b0 = __ldg(g2), b1 = __ldg(g2 + 1);
                const float ga[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float gb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    x1[e] = x1[e] * inv * ga[e];
                    x2[e] = x2[e] * inv * gb[e];
                }
            }
        }
        if (!on) continue;
        if (cs) {
            const float4* c4 = reinterpret_cast<const float4*>(cs + 8 * j);
            const float4* s4 = reinterpret_cast<const float4*>(sn + 8 * j);
            const float4 c0 = __ldg(c4), c1 = __ldg(c4 + 1), s0 = __ldg(s4), s1 = __ldg(s4 + 1);
            const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float a = x1[e], b = x2[e];
                x1[e] = __fsub_rn(__fmul_rn(a, cc[e]), __fmul_rn(b, ss[e]));
                x2[e] = __fadd_rn(__fmul_rn(b, cc[e]), __fmul_rn(a, ss[e]));
            }
        }
        amax = fmaxf(amax, store8<F16, F32>(base, off, x1));
        amax = fmaxf(amax, store8<F16, F32>(base, off + HALF, x2));
    }
    if constexpr (F16)
        if (__any_sync(0xffffffffu, !(amax <= 65504.0f)) && lane == 0 && p.status)
            atomicOr(p.status, kStatusF16Overflow);
}

cudaError_t launch_qk_norm_rope(const QkRopeParams& p, int head_dim, cudaStream_t st) {
    if (p.T <= 0) return cudaSuccess;
    const int grid = (p.T + 7) / 8;
    switch (head_dim) {
#define RG_QKR(DH)                                                                                  \
    if (p.qkv32) launch_pdl(qk_norm_rope_kernel<DH, false, true>, dim3(grid), dim3(256), 0, st, p);    \
    else if (p.f16) launch_pdl(qk_norm_rope_kernel<DH, true, false>, dim3(grid), dim3(256), 0, st, p); \
    else launch_pdl(qk_norm_rope_kernel<DH, false, false>, dim3(grid), dim3(256), 0, st, p);
    case 32: RG_QKR(32) break;
    case 64: RG_QKR(64) break;
    case 128: RG_QKR(128) break;
    case 256: RG_QKR(256) break;
#undef RG_QKR
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// int8 -> fp16 widening, 16 weights per thread: (q + 128) placed in the low
// mantissa byte of 1024.0 is exactly 1024 + q + 128; subtracting 1152 leaves q.
// Several widenings (a layer's weights) in one launch: blocks are dealt over
// the jobs in proportion to their sizes (job j takes blocks [first[j],
// first[j + 1])).
struct WidenJobs {
    WidenJob job[4];
    int first[5];
};

__global__ void __launch_bounds__(256) widen_s8_f16_multi_kernel(WidenJobs js) {
    pdl_trigger();
    pdl_wait();
    int j = 0;
    while (j < 3 && static_cast<int>(blockIdx.x) >= js.first[j + 1]) ++j;
    const uint4* w = reinterpret_cast<const uint4*>(js.job[j].src);
    uint4* out = reinterpret_cast<uint4*>(js.job[j].dst);
    const size_t n16 = js.job[j].n / 16;
    const int nb = js.first[j + 1] - js.first[j];
    for (size_t i = (blockIdx.x - js.first[j]) * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n16;
         i += static_cast<size_t>(nb) * blockDim.x) {
        const uint4 u = __ldg(w + i);
        const uint32_t in[4] = {u.x, u.y, u.z, u.w};
        uint32_t o[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t b = in[k] ^ 0x80808080u;
            uint32_t lo, hi;
            asm("prmt.b32 %0, %1, %2, %3;" : "=r"(lo) : "r"(b), "r"(0x64646464u), "r"(0x4140u));
            asm("prmt.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(b), "r"(0x64646464u), "r"(0x4342u));
            asm("sub.f16x2 %0, %1, %2;" : "=r"(o[2 * k]) : "r"(lo), "r"(0x64806480u));
            asm("sub.f16x2 %0, %1, %2;" : "=r"(o[2 * k + 1]) : "r"(hi), "r"(0x64806480u));
        }
        out[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
        out[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

cudaError_t launch_widen_s8_f16_multi(const WidenJob* jobs, int count, cudaStream_t st) {
    if (count <= 0 || count > 4) return cudaErrorInvalidValue;
    WidenJobs js{};
    size_t total = 0;
    for (int j = 0; j < count; ++j) {
        const WidenJob& b = jobs[j];
        if (b.n == 0 || b.n % 16 != 0 || (reinterpret_cast<uintptr_t>(b.src) & 15) ||
            (reinterpret_cast<uintptr_t>(b.dst) & 15))
            return cudaErrorInvalidValue;
        js.job[j] = b;
        total += b.n / 16;
    }
    // about 4 blocks of 256 threads per SM in all, at least one per job
    const int budget = 148 * 4;
    js.first[0] = 0;
    for (int j = 0; j < 4; ++j) {
        int nb = 0;
        if (j < count) {
            const size_t n16 = js.job[j].n / 16;
            nb = static_cast<int>(std::max<size_t>(1, std::min<size_t>((n16 + 255) / 256, budget * n16 / total)));
        }
        js.first[j + 1] = js.first[j] + nb;
    }
    launch_pdl(widen_s8_f16_multi_kernel, dim3(js.first[4]), dim3(256), 0, st, js);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// int8 row quantisation of a bf16 matrix (full-int8 mode inputs that are not
// produced by a LayerNorm: the attention context and the FFN hidden state).
// One warp per row, single pass: the row (up to 16 vectors of 8 per lane,
// K <= 4096) stays in registers between the max and the quantisation.
template <int NV>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const __nv_bfloat16* __restrict__ x, int T, int K,
                                                           int8_t* q, float* scale) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const uint4* row = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * K);
    const int nvec = K / 8;  // 8-element vectors in the row
    uint4 u[NV];
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        u[c] = lane + 32 * c < nvec ? __ldg(row + lane + 32 * c) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w[4] = {u[c].x, u[c].y, u[c].z, u[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = unpack2<false>(w[e]);
            amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
    amax = warp_max(amax);
    float s = amax / 127.0f;
    if (s == 0.0f) s = 1.0f;
    const float rinv = 1.0f / s;
    uint2* qr = reinterpret_cast<uint2*>(q + static_cast<int64_t>(t) * K);
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const uint32_t w[4] = {u[c].x, u[c].y, u[c].z, u[c].w};
        int8_t o[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = unpack2<false>(w[e]);
            o[2 * e] = (int8_t)max(-128, min(127, __float2int_rn(f.x * rinv)));
            o[2 * e + 1] = (int8_t)max(-128, min(127, __float2int_rn(f.y * rinv)));
        }
        if (lane + 32 * c < nvec) qr[lane + 32 * c] = *reinterpret_cast<uint2*>(o);
    }
    if (lane == 0) scale[t] = s;
}

cudaError_t launch_quantize_rows(const __nv_bfloat16* x, int T, int K, int8_t* q, float* scale, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (K % 8 != 0 || K > 16 * 256) return cudaErrorInvalidValue;
    const int grid = (T + 7) / 8;
    switch ((K + 255) / 256) {
#define RG_QR(NV) \
    case NV: launch_pdl(quantize_rows_kernel<NV>, dim3(grid), dim3(256), 0, st, x, T, K, q, scale); break;
        RG_QR(1) RG_QR(2) RG_QR(3) RG_QR(4) RG_QR(5) RG_QR(6) RG_QR(7) RG_QR(8)
        RG_QR(9) RG_QR(10) RG_QR(11) RG_QR(12) RG_QR(13) RG_QR(14) RG_QR(15) RG_QR(16)
#undef RG_QR
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Attention: every supported head dim (32, 64, 128, 256) runs the tcgen05
// kernel (attention_tc.cu).
cudaError_t launch_attention(const AttnParams& p, int nseq, int max_len, int heads, int head_dim, cudaStream_t st) {
    if (!attention_tc_supported(head_dim) || !p.status) return cudaErrorInvalidValue;
    return launch_attention_tc(p, p.T, nseq, max_len, heads, p.kv_heads, head_dim, p.status, st);
}

// ---------------------------------------------------------------------------
// Row statistics of a folded LayerNorm: the chunks merged in a fixed order
// (Chan et al.'s update for equal-size parts): mean = sum of the chunk means
// / n, M2 = sum of (M2_i + 32 (mean_i - mean)^2), var = M2 / (32 n).  One
// thread per row; for each chunk a warp's 32 rows are 256 contiguous bytes.
// Rows of up to kMergeRegs chunks are loaded once into registers (every
// load in flight together); longer rows are read twice.
constexpr int kMergeRegs = 32;

__global__ void __launch_bounds__(64) merge_row_stats_kernel(const float2* __restrict__ parts, int nparts, int T,
                                                             float eps, float2* __restrict__ stats, bool rms) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= T) return;
    const float2* p = parts + row;
    float mean, m2 = 0.f;
    if (rms) {  // sum of squares about zero, the chunks in order
        float ss = 0.f;
        for (int i = 0; i < nparts; ++i) {
            const float2 q = p[static_cast<size_t>(i) * T];
            ss += fmaf(32.0f * q.x, q.x, q.y);
        }
        stats[row] = make_float2(0.f, 1.0f / sqrtf(ss / static_cast<float>(32 * nparts) + eps));
        return;
    }
    if (nparts <= kMergeRegs) {
        float2 q[kMergeRegs];
#pragma unroll
        for (int i = 0; i < kMergeRegs; ++i) q[i] = i < nparts ? p[static_cast<size_t>(i) * T] : make_float2(0.f, 0.f);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kMergeRegs; ++i) s += q[i].x;
        mean = s / static_cast<float>(nparts);
#pragma unroll
        for (int i = 0; i < kMergeRegs; ++i) {
            const float d = q[i].x - mean;
            if (i < nparts) m2 += fmaf(32.0f * d, d, q[i].y);
        }
    } else {
        float s = 0.f;
        for (int i = 0; i < nparts; ++i) s += p[static_cast<size_t>(i) * T].x;
        mean = s / static_cast<float>(nparts);
        for (int i = 0; i < nparts; ++i) {
            const float2 q = p[static_cast<size_t>(i) * T];
            const float d = q.x - mean;
            m2 += fmaf(32.0f * d, d, q.y);
        }
    }
    stats[row] = make_float2(mean, 1.0f / sqrtf(m2 / static_cast<float>(32 * nparts) + eps));
}

cudaError_t launch_merge_row_stats(const float2* parts, int nparts, int T, float eps, float2* stats, cudaStream_t st,
                                   bool rms) {
    if (T <= 0) return cudaSuccess;
    if (nparts <= 0 || !parts || !stats) return cudaErrorInvalidValue;
    launch_pdl(merge_row_stats_kernel, dim3((T + 63) / 64), dim3(64), 0, st, parts, nparts, T, eps, stats, rms);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// 3xTF32 operand split: hi = tf32(x) (nearest, ties to even), lo = x - hi.
__global__ void __launch_bounds__(256) split_tf32_kernel(const float4* __restrict__ x, size_t n4, float4* hi,
                                                        float4* lo) {
    pdl_trigger();
    pdl_wait();
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float4 v = x[i];
        float4 h, l;
        tf32_split(v.x, h.x, l.x);
        tf32_split(v.y, h.y, l.y);
        tf32_split(v.z, h.z, l.z);
        tf32_split(v.w, h.w, l.w);
        hi[i] = h;
        lo[i] = l;
    }
}

cudaError_t launch_split_tf32(const float* x, size_t n, float* hi, float* lo, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    if (n % 4 != 0) return cudaErrorInvalidValue;
    const size_t n4 = n / 4;
    const int grid = static_cast<int>(std::min<size_t>((n4 + 255) / 256, 148 * 16));
    launch_pdl(split_tf32_kernel, dim3(grid), dim3(256), 0, st, reinterpret_cast<const float4*>(x), n4,
               reinterpret_cast<float4*>(hi), reinterpret_cast<float4*>(lo));
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Strict fp32 attention.  CTA = 8 query rows of one (sequence, head), one
// warp per row.  Key/value blocks of 32 rows are staged in shared memory by
// the whole CTA (coalesced; K rows padded by one float so that lane j reading
// key j's row is bank-conflict-free).  Lane j computes q . k_j for its key,
// the warp keeps the running max / sum, and lane d accumulates output dims
// d, d + 32, ... over the block's probabilities (broadcast by shuffle).
// Strict fp32 attention, register-tiled on the FMA pipes: a CTA takes 64
// query rows of one (sequence, head) and walks 64-key blocks staged in
// shared memory.  Thread t = (row group rg = t / 16, column group cg =
// t % 16) holds the scores of rows 4 rg .. 4 rg + 3 against keys cg + 16 j
// (j < 4) and the output of the same rows at dims cg + 16 c (c < D / 16);
// the keys / dims strided by 16 keep the shared-memory reads of a warp on
// distinct banks.  Online softmax in the natural exp domain (expf), like the
// reference's fp32 path; a row's 64 scores of a block are reduced over its
// 16 threads by shuffles.
constexpr int kF32Rows = 64, kF32Keys = 64;

template <int D>
struct AttnF32Smem {
    static constexpr int QP = D + 1, KP = D + 1, VP = D, PP = kF32Keys + 1;
    static constexpr int FLOATS = kF32Rows * QP + kF32Keys * KP + kF32Keys * VP + kF32Rows * PP;
};

template <int D>
__global__ void __launch_bounds__(256) attention_f32_kernel(AttnF32Params p) {
    pdl_trigger();
    pdl_wait();
    using SM = AttnF32Smem<D>;
    constexpr int QP = SM::QP, KP = SM::KP, VP = SM::VP, PP = SM::PP;
    constexpr int NC = D / 16;  // output dims per thread and row
    extern __shared__ float fsm[];
    float* qs = fsm;                        // [64][D + 1]
    float* ks = qs + kF32Rows * QP;         // [64][D + 1]
    float* vs = ks + kF32Keys * KP;         // [64][D]
    float* ps = vs + kF32Keys * VP;         // [64][65]
    const int t = threadIdx.x, rg = t >> 4, cg = t & 15;
    const int s = blockIdx.z, h = blockIdx.y;
    const int s0 = __ldg(p.cu + s), L = __ldg(p.cu + s + 1) - s0;
    const int q0 = blockIdx.x * kF32Rows;
    if (q0 >= L) return;  // the whole CTA
    const int hk = h / p.group;
    const int nrow = min(kF32Rows, L - q0);
    for (int i = t; i < kF32Rows * D; i += 256) {
        const int r = i / D, d = i % D;
        qs[r * QP + d] = r < nrow ? p.q[static_cast<int64_t>(s0 + q0 + r) * p.ldq + h * D + d] : 0.f;
    }
    const float* K = p.k + static_cast<int64_t>(s0) * p.ldk + hk * D;
    const float* V = p.v + static_cast<int64_t>(s0) * p.ldv + hk * D;
    // keys any row of the tile may see
    const int clo = max(0, q0 + p.rel_lo), chi = min(L - 1, q0 + nrow - 1 + p.rel_hi);
    float m[4], l[4], o[4][NC];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < NC; ++c) o[i][c] = 0.f;
    }
    const float* bias_row = p.bias ? p.bias + static_cast<int64_t>(h) * (2 * p.bias_off + 1) : nullptr;
    for (int j0 = clo; j0 <= chi; j0 += kF32Keys) {
        __syncthreads();  // the previous block's K / V / P consumed (and, first time, Q written)
        const int nk = min(kF32Keys, chi - j0 + 1);
        for (int i = t; i < kF32Keys * D; i += 256) {
            const int r = i / D, d = i % D;
            const bool in = r < nk;
            ks[r * KP + d] = in ? __ldg(K + static_cast<int64_t>(j0 + r) * p.ldk + d) : 0.f;
            vs[r * VP + d] = in ? __ldg(V + static_cast<int64_t>(j0 + r) * p.ldv + d) : 0.f;
        }
        __syncthreads();
        // S = Q K^T for the thread's 4 rows x 4 keys
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; ++d) {
            float qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = qs[(4 * rg + i) * QP + d];
#pragma unroll
            for (int j = 0; j < 4; ++j) kv[j] = ks[(cg + 16 * j) * KP + d];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) sc[i][j] = fmaf(qv[i], kv[j], sc[i][j]);
        }
        // scale (+ relative bias), mask, online softmax per row
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int qi = q0 + 4 * rg + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kj = j0 + cg + 16 * j;
                const int rel = kj - qi;
                const bool valid = kj <= chi && rel >= p.rel_lo && rel <= p.rel_hi;
                float x = sc[i][j] * p.scale;
                if (bias_row) x += __ldg(bias_row + min(max(rel + p.bias_off, 0), 2 * p.bias_off));
                x = valid ? x : -INFINITY;
                sc[i][j] = x;
                mx = fmaxf(mx, x);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[i], mx);
            float alpha = 1.f, ls = 0.f;
            if (mn != -INFINITY) {  // the row has a key so far
                alpha = m[i] == -INFINITY ? 0.f : expf(m[i] - mn);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float e = sc[i][j] == -INFINITY ? 0.f : expf(sc[i][j] - mn);
                    sc[i][j] = e;
                    ls += e;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
            l[i] = l[i] * alpha + ls;
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < NC; ++c) o[i][c] *= alpha;
#pragma unroll
            for (int j = 0; j < 4; ++j) ps[(4 * rg + i) * PP + cg + 16 * j] = sc[i][j];
        }
        __syncthreads();  // P complete
        // O += P V for the thread's 4 rows x NC dims
#pragma unroll 4
        for (int k = 0; k < nk; ++k) {
            float pv[4], vv[NC];
#pragma unroll
            for (int i = 0; i < 4; ++i) pv[i] = ps[(4 * rg + i) * PP + k];
#pragma unroll
            for (int c = 0; c < NC; ++c) vv[c] = vs[k * VP + cg + 16 * c];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < NC; ++c) o[i][c] = fmaf(pv[i], vv[c], o[i][c]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 4 * rg + i;
        if (r >= nrow) continue;
        const float inv = l[i] > 0.f ? 1.0f / l[i] : 0.f;
        float* oh = p.out_hi + static_cast<int64_t>(s0 + q0 + r) * p.ldo + h * D;
        if (!p.out_lo) {  // the unsplit fp32 result (kernel-level entry point)
#pragma unroll
            for (int c = 0; c < NC; ++c) oh[cg + 16 * c] = o[i][c] * inv;
            continue;
        }
        float* ol = p.out_lo + static_cast<int64_t>(s0 + q0 + r) * p.ldo + h * D;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            float hi, lo;
            tf32_split(o[i][c] * inv, hi, lo);
            oh[cg + 16 * c] = hi;
            ol[cg + 16 * c] = lo;
        }
    }
}

template <int D>
static cudaError_t launch_attention_f32_d(const AttnF32Params& p, int nseq, int max_len, int heads,
                                          cudaStream_t st) {
    constexpr int smem = AttnF32Smem<D>::FLOATS * 4;
    static_assert(smem <= 232448, "shared memory budget");
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && (dev >= 32 || !(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << dev)))) {
        cudaError_t e = cudaFuncSetAttribute(attention_f32_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 32) __atomic_fetch_or(&configured, 1u << dev, __ATOMIC_RELEASE);
    }
    const dim3 grid((max_len + kF32Rows - 1) / kF32Rows, heads, nseq);
    launch_pdl(attention_f32_kernel<D>, dim3(grid), dim3(256), smem, st, p);
    return cudaGetLastError();
}

cudaError_t launch_attention_f32(const AttnF32Params& p, int nseq, int max_len, int heads, int head_dim,
                                 cudaStream_t st) {
    if (nseq <= 0) return cudaSuccess;
    switch (head_dim) {
    case 32: return launch_attention_f32_d<32>(p, nseq, max_len, heads, st);
    case 64: return launch_attention_f32_d<64>(p, nseq, max_len, heads, st);
    case 128: return launch_attention_f32_d<128>(p, nseq, max_len, heads, st);
    case 256: return launch_attention_f32_d<256>(p, nseq, max_len, heads, st);
    default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// Pooling + L2 + truncate: one CTA per sequence.
__global__ void __launch_bounds__(256) pool_kernel(const float* __restrict__ x32, const int32_t* __restrict__ cu,
                                                  int H, int pooling, int normalize, int dim, float* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float pooled[];  // [H]
    __shared__ double red[8];
    const int s = blockIdx.x;
    const int s0 = __ldg(cu + s), L = __ldg(cu + s + 1) - s0;
    if (pooling == 0) {
        // mean, poolMean (bert.go:692-703): each column summed in row order,
        // times 1/L; four columns per thread (16-byte loads) and eight rows'
        // loads issued before they are added (H % 4 == 0)
        const float invL = 1.0f / static_cast<float>(L);
        for (int j = 4 * threadIdx.x; j < H; j += 4 * blockDim.x) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            const float* col = x32 + static_cast<int64_t>(s0) * H + j;
            int i = 0;
            for (; i + 8 <= L; i += 8) {
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = __ldg(reinterpret_cast<const float4*>(col + static_cast<int64_t>(i + u) * H));
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    acc.x += v[u].x;
                    acc.y += v[u].y;
                    acc.z += v[u].z;
                    acc.w += v[u].w;
                }
            }
            for (; i < L; ++i) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(col + static_cast<int64_t>(i) * H));
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            pooled[j] = acc.x * invL;
            pooled[j + 1] = acc.y * invL;
            pooled[j + 2] = acc.z * invL;
            pooled[j + 3] = acc.w * invL;
        }
    } else {
        for (int j = threadIdx.x; j < H; j += blockDim.x)  // cls: first token; lasttoken: last
            pooled[j] = x32[static_cast<int64_t>(pooling == 1 ? s0 : s0 + L - 1) * H + j];
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
    if (H % 4 != 0) return cudaErrorInvalidValue;
    launch_pdl(pool_kernel, dim3(nseq), dim3(256), H * sizeof(float), st, x32, cu, H, pooling, normalize, dim, out);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Pooling, Dense head, L2 and Matryoshka truncation as one kernel
// (ForwardWorkers' pooling bert.go:670-703, the Gemma Dense head
// gemma3.go:177-198, L2Normalize tensor.go:542-554, truncate
// rembed.go:441-448).  A cluster of kHeadCtas CTAs serves kHeadSeqs
// sequences and splits every stage between its CTAs through distributed
// shared memory:
//   1. pool: CTA r sums rows [r L / 8, (r+1) L / 8) of each sequence
//      (mean) or takes its picked row (rank 0); the partial sums of all
//      CTAs are added in rank order and scaled by 1/L;
//   2. hid = pooled . W1^T: CTA r computes its D/8 hidden columns for the
//      group's sequences, one warp per column (lanes split K, coalesced
//      weight rows), and every CTA then gathers the whole hidden vector;
//   3. y = hid . W2^T: CTA r computes its H/8 output columns the same way;
//   4. L2 over H (float64 partial sums per CTA, added in rank order), then
//      for dim < H the first dim columns re-normalised the same way;
// each CTA writes its slice of the output.  The head weights stay fp32
// (never quantised, as in the reference) and are read once per cluster.
constexpr int kHeadCtas = 8, kHeadSeqs = 4, kHeadThreads = 256;

// Loads from another CTA's shared memory (distributed shared memory).
// Callers issue several of them before using the results, so that their
// latencies overlap.
__device__ __forceinline__ float ld_dsmem_f32(const float* local, uint32_t rank) {
    const uint32_t a = mapa_shared(smem_u32(local), rank);
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ double ld_dsmem_f64(const double* local, uint32_t rank) {
    const uint32_t a = mapa_shared(smem_u32(local), rank);
    double v;
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(a) : "memory");
    return v;
}

// Columns [col0, col0 + ncols) of out[g][col] = sum_k x[g][k] * w[col][k]
// for the group's kHeadSeqs rows of x (shared memory, row stride K): each
// warp takes four columns at a time, lanes split K (coalesced weight rows),
// and the k loop is unrolled so that sixteen weight loads are in flight per
// lane (the weights come from L2: one column at a time would wait for them
// one by one).
constexpr int kHeadColsPerWarp = 4;
__device__ __forceinline__ void head_columns(const float* __restrict__ w, const float* x, int K, int col0, int ncols,
                                             float* out, int out_stride, int warp, int lane) {
    for (int c = warp * kHeadColsPerWarp; c < ncols; c += (kHeadThreads / 32) * kHeadColsPerWarp) {
        const float* wr[kHeadColsPerWarp];
        bool on[kHeadColsPerWarp];
#pragma unroll
        for (int i = 0; i < kHeadColsPerWarp; ++i) {
            on[i] = c + i < ncols;
            wr[i] = w + static_cast<int64_t>(col0 + (on[i] ? c + i : c)) * K;
        }
        float acc[kHeadColsPerWarp][kHeadSeqs];
#pragma unroll
        for (int i = 0; i < kHeadColsPerWarp; ++i)
#pragma unroll
            for (int g = 0; g < kHeadSeqs; ++g) acc[i][g] = 0.f;
#pragma unroll 4
        for (int k = lane; k < K; k += 32) {
            float wv[kHeadColsPerWarp];
#pragma unroll
            for (int i = 0; i < kHeadColsPerWarp; ++i) wv[i] = __ldg(wr[i] + k);
#pragma unroll
            for (int g = 0; g < kHeadSeqs; ++g) {
                const float xv = x[g * K + k];
#pragma unroll
                for (int i = 0; i < kHeadColsPerWarp; ++i) acc[i][g] = fmaf(xv, wv[i], acc[i][g]);
            }
        }
#pragma unroll
        for (int i = 0; i < kHeadColsPerWarp; ++i)
#pragma unroll
            for (int g = 0; g < kHeadSeqs; ++g) {
                const float v = warp_sum(acc[i][g]);
                if (lane == 0 && on[i]) out[g * out_stride + col0 + c + i] = v;
            }
    }
}

__global__ void __cluster_dims__(kHeadCtas, 1, 1) __launch_bounds__(kHeadThreads)
    pool_head_kernel(const float* __restrict__ x32, const int32_t* __restrict__ cu, int nseq, int H, int D,
                     int pooling, const float* __restrict__ w1, const float* __restrict__ w2, int normalize, int dim,
                     float* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float hsm[];
    float* part = hsm;                        // [kHeadSeqs][H]: this CTA's pooling partial sums
    float* pooled = part + kHeadSeqs * H;     // [kHeadSeqs][H]
    float* hid = pooled + kHeadSeqs * H;      // [kHeadSeqs][D]: own slice written, others gathered
    float* y = hid + kHeadSeqs * D;           // [kHeadSeqs][H]: own slice of the head output
    __shared__ double ss[2][kHeadSeqs];       // this CTA's sums of squares (full row, first dim)
    __shared__ double red[kHeadThreads / 32][kHeadSeqs];
    __shared__ float scale[kHeadSeqs];
    const uint32_t rank = cluster_ctarank();
    const int grp = blockIdx.x / kHeadCtas;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

    // 1. pooling partial sums of this CTA's share of each sequence's rows
    for (int g = 0; g < kHeadSeqs; ++g) {
        const int s = grp * kHeadSeqs + g;
        int r0 = 0, r1 = 0;
        if (s < nseq) {
            const int s0 = __ldg(cu + s), L = __ldg(cu + s + 1) - s0;
            if (pooling == 0) {  // mean: rows split between the CTAs
                r0 = s0 + static_cast<int>((static_cast<int64_t>(L) * rank) / kHeadCtas);
                r1 = s0 + static_cast<int>((static_cast<int64_t>(L) * (rank + 1)) / kHeadCtas);
            } else if (rank == 0) {  // cls (first) / last token: one row
                r0 = pooling == 1 ? s0 : s0 + L - 1;
                r1 = r0 + 1;
            }
        }
        // four columns per thread (16-byte loads, a warp reads 512
        // contiguous bytes of a row) and sixteen rows' loads issued before
        // they are added, in row order
        for (int j = 4 * t; j < H; j += 4 * kHeadThreads) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            int i = r0;
            for (; i + 16 <= r1; i += 16) {
                float4 v[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) v[u] = __ldg(reinterpret_cast<const float4*>(x32 + static_cast<int64_t>(i + u) * H + j));
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    acc.x += v[u].x;
                    acc.y += v[u].y;
                    acc.z += v[u].z;
                    acc.w += v[u].w;
                }
            }
            for (; i < r1; ++i) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(x32 + static_cast<int64_t>(i) * H + j));
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            *reinterpret_cast<float4*>(part + g * H + j) = acc;
        }
    }
    cluster_sync();
    for (int g = 0; g < kHeadSeqs; ++g) {
        const int s = grp * kHeadSeqs + g;
        float invL = 1.0f;
        if (s < nseq && pooling == 0) invL = 1.0f / static_cast<float>(__ldg(cu + s + 1) - __ldg(cu + s));
        for (int j = t; j < H; j += kHeadThreads) {
            float pv[kHeadCtas];
#pragma unroll
            for (int q = 0; q < kHeadCtas; ++q) pv[q] = ld_dsmem_f32(part + g * H + j, q);
            float v = 0.f;
#pragma unroll
            for (int q = 0; q < kHeadCtas; ++q) v += pv[q];  // rank order
            pooled[g * H + j] = v * invL;
        }
    }
    __syncthreads();
    const int dper = D / kHeadCtas, hper = H / kHeadCtas;
    if (!w1) {
        // no Dense head: the output slice is the pooled vector's
        for (int i = t; i < kHeadSeqs * hper; i += kHeadThreads) {
            const int g = i / hper, c = static_cast<int>(rank) * hper + i % hper;
            y[g * H + c] = pooled[g * H + c];
        }
        __syncthreads();
    } else {
    // 2. this CTA's hidden columns, then the whole hidden vector
    head_columns(w1, pooled, H, static_cast<int>(rank) * dper, dper, hid, D, warp, lane);
    cluster_sync();
    for (int q = 0; q < kHeadCtas; ++q) {
        if (q == static_cast<int>(rank)) continue;
        for (int i0 = t; i0 < kHeadSeqs * dper; i0 += 4 * kHeadThreads) {
            float hv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kHeadThreads;
                hv[u] = i < kHeadSeqs * dper ? ld_dsmem_f32(hid + (i / dper) * D + q * dper + i % dper, q) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kHeadThreads;
                if (i < kHeadSeqs * dper) hid[(i / dper) * D + q * dper + i % dper] = hv[u];
            }
        }
    }
    __syncthreads();
    // 3. this CTA's output columns
    head_columns(w2, hid, D, static_cast<int>(rank) * hper, hper, y, H, warp, lane);
    __syncthreads();
    }
    // 4. L2 over H, then (dim < H) over the first dim columns
    const int c0 = static_cast<int>(rank) * hper;
    for (int pass = 0; pass < 2; ++pass) {
        const bool trunc = pass == 1;
        if (trunc && dim >= H) break;
        if (!trunc && !normalize) continue;
        const int lim = trunc ? dim : H;
        double a[kHeadSeqs];
#pragma unroll
        for (int g = 0; g < kHeadSeqs; ++g) a[g] = 0.0;
        for (int c = t; c < hper; c += kHeadThreads) {
            if (c0 + c >= lim) continue;
#pragma unroll
            for (int g = 0; g < kHeadSeqs; ++g) {
                const double v = y[g * H + c0 + c];
                a[g] += v * v;
            }
        }
#pragma unroll
        for (int g = 0; g < kHeadSeqs; ++g) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a[g] += __shfl_xor_sync(0xffffffffu, a[g], o);
            if (lane == 0) red[warp][g] = a[g];
        }
        __syncthreads();
        if (t < kHeadSeqs) {
            double v = 0.0;
            for (int w = 0; w < kHeadThreads / 32; ++w) v += red[w][t];
            ss[pass][t] = v;
        }
        cluster_sync();
        if (t < kHeadSeqs) {
            double sv[kHeadCtas];
#pragma unroll
            for (int q = 0; q < kHeadCtas; ++q) sv[q] = ld_dsmem_f64(&ss[pass][t], q);
            double v = 0.0;
#pragma unroll
            for (int q = 0; q < kHeadCtas; ++q) v += sv[q];  // rank order
            scale[t] = v != 0.0 ? static_cast<float>(1.0 / sqrt(v)) : 1.0f;
        }
        __syncthreads();
        for (int c = t; c < hper; c += kHeadThreads)
#pragma unroll
            for (int g = 0; g < kHeadSeqs; ++g) y[g * H + c0 + c] *= scale[g];
        __syncthreads();
    }
    for (int c = t; c < hper; c += kHeadThreads) {
        if (c0 + c >= dim) continue;
#pragma unroll
        for (int g = 0; g < kHeadSeqs; ++g) {
            const int s = grp * kHeadSeqs + g;
            if (s < nseq) out[static_cast<int64_t>(s) * dim + c0 + c] = y[g * H + c0 + c];
        }
    }
    // no CTA leaves while another may still read its shared memory
    cluster_sync();
}

cudaError_t launch_pool_head(const float* x32, const int32_t* cu, int nseq, int H, int D, int pooling,
                             const float* w1, const float* w2, int normalize, int dim, float* out, cudaStream_t st) {
    if (nseq <= 0) return cudaSuccess;
    if (!w1 || !w2) D = 0;  // pooling, L2 and truncation only
    if (H % kHeadCtas != 0 || H % 4 != 0 || D % kHeadCtas != 0 || dim < 1 || dim > H) return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * (3 * kHeadSeqs * static_cast<size_t>(H) + kHeadSeqs * static_cast<size_t>(D));
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(pool_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        if (dev < 32) __atomic_fetch_or(&configured, 1u << dev, __ATOMIC_RELEASE);
    }
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    const int groups = (nseq + kHeadSeqs - 1) / kHeadSeqs;
    launch_pdl(pool_head_kernel, dim3(groups * kHeadCtas), dim3(kHeadThreads), smem, st, x32, cu, nseq, H, D, pooling,
               w1, w2, normalize, dim, out);
    return cudaGetLastError();
}

}  // namespace rg
