// attention_tc.cu - varlen flash attention on the 5th-generation tensor
// cores (tcgen05) for head dims 32, 64, 128 and 256.
//
// CTA = 128 query rows of one (sequence, query head); key/value blocks of
// BKV rows.  Roles (192 threads):
//   warp 0     TMA producer: the Q tile once, then K blocks into a 2-deep
//              ring and V blocks into a 2-deep (head dim 64) or single
//              buffer, straight from the fused
//              token-major qkv buffer (128-byte swizzle);
//   warp 1     TMEM allocator and MMA issuer (one thread):
//                S  = Q K^T   (M 128, N BKV, K D; both operands K-major)
//                O += P V     (M 128, N D, K BKV; P K-major from shared
//                              memory, V MN-major as loaded);
//   warps 2-5  softmax, thread = query row = TMEM lane: read the S row
//              (64 keys),
//              mask (sequence end, window, causal), scale (+ relative
//              bias), online max / sum in the exp2 domain, rescale the O
//              row in TMEM when the running max moves, write P (16-bit,
//              swizzled K-major) for the next MMA; at the end O / l to the
//              output rows of the sequence.
// Rows of the packed buffer past the sequence's end are loaded like any
// other (they belong to the next sequence or are zero-filled past T) and are
// masked as keys and never stored as queries.  Every wait is bounded; on a
// timeout the roles stop, in-flight copies and MMAs are drained and TMEM is
// freed before the CTA exits with kStatusWaitTimeout raised.
#include <cuda.h>
#include <cuda_runtime.h>

#include "act16.cuh"
#include "kernels.cuh"
#include "pdl.cuh"
#include "sm100.cuh"

namespace rg {

template <int D>
struct AttnTc {
    static constexpr int BKV = 64;  // keys per block
    // 64-column (128-byte, one swizzle atom wide) blocks loaded per row; a
    // head of 32 loads one such block and the MMAs use its first 32 columns
    static constexpr int QB = D < 64 ? 1 : D / 64;
    static constexpr int Q_BYTES = 128 * QB * 128;
    static constexpr int KV_BYTES = BKV * QB * 128;
    static constexpr int P_BYTES = 128 * BKV * 2;
    static constexpr int VST = D <= 64 ? 2 : 1;  // V stages (larger heads fill the SM with one)
    static constexpr int SMEM = Q_BYTES + (2 + VST) * KV_BYTES + P_BYTES + 1024 + 256;
    // S at column 0 (BKV wide), O at column O_COL (D wide)
    static constexpr uint32_t O_COL = 64;
    static constexpr uint32_t TMEM_COLS = D <= 64 ? 128 : (D == 128 ? 256 : 512);
    static constexpr int THREADS = 192;
    // CTAs per SM (shared memory, TMEM, registers)
    static constexpr int MIN_BLOCKS = D <= 64 ? 3 : (D == 128 ? 2 : 1);
    // Which pairs of scores (bit j: pair index % 4 == j) take their
    // exponentials on the FMA pipe (ex2_fma) instead of the transcendental
    // unit, which also converts P to 16 bits.  Measured per head dim
    // (rg_attention, B200): at 128 one pair in four lifts Qwen3's causal
    // layers from 295 to 349 TFLOP/s (two in four: 285); at 64 (three CTAs
    // per SM, 96 registers) every share was slower (682 -> 642 TFLOP/s at one
    // in four on ModernBERT's global layers), and at 256 it made no
    // difference.
    static constexpr unsigned EXP_FMA_MASK = D == 128 ? 0x1u : 0x0u;
};

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// 2^x on the FMA pipe, for a share of the exponentials so that the
// transcendental unit (which also converts P to 16 bits) is not the only
// one computing them.  Range reduction with the round-to-nearest magic
// constant 1.5 * 2^23: t = x + M holds n = round(x) in its low mantissa bits,
// f = x - (t - M) in [-1/2, 1/2]; 2^f by a cubic fitted here to 2^f on
// [-1/2, 1/2] for least relative error (max 7.5e-5, below the 16-bit rounding
// of P that follows); 2^n enters by adding n to the exponent field, and
// since M's low nine bits are zero, n << 23 = t_bits << 23 (mod 2^32).  x is
// clamped at -125 so that the exponent stays normal (2^-125 is zero for P).
__device__ __forceinline__ float ex2_fma(float x) {
    x = fmaxf(x, -125.0f);
    const float M = 12582912.0f;
    const float t = x + M;
    const float f = x - (t - M);
    float p = fmaf(0.05517112836241722f, f, 0.24261008203029633f);
    p = fmaf(p, f, 0.6932609677314758f);
    p = fmaf(p, f, 0.9999281167984009f);
    return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}
// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float y;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
    return y;
}
// The softmax role of one 128-row query tile (4 warps, thread = query row =
// TMEM lane of the warp's quarter): for each of the nb key blocks from kb0 on,
// read the block's scores S from TMEM (tS), mask (sequence end, window,
// causal), scale (+ relative bias), online max / sum in the exp2 domain with
// lazy rescaling of the O row (tO), write P (16-bit, swizzled K-major) to sP
// for the next P.V MMA; at the end O / l to the output rows of the sequence.
// The barriers are the tile's: sfull (S ready), sfree (S read), pfull (P
// written), ofull (P.V done).  EMU: which pairs of every four take their
// exponentials on the FMA pipe.
template <int D, bool F16, bool BIAS, unsigned EMU>
__device__ __forceinline__ void attn_softmax_tile(const AttnParams& p, int h, int s0, int L, int q0, int kb0, int nb,
                                                  uint32_t tS, uint32_t tO, uint8_t* sP, uint64_t* sfull,
                                                  uint64_t* sfree, uint64_t* pfull, uint64_t* ofull, int* status,
                                                  volatile int* abort_flag, int quarter, int lane) {
    constexpr int BKV = 64;
    const int r = quarter * 32 + lane;  // row within the tile = TMEM lane
    const int qi = q0 + r;              // query index within the sequence
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
        const int kbase = (kb0 + i) * BKV;
        if (!mbar_wait(sfull, i & 1, status, abort_flag)) {
            ok = false;
            break;
        }
        tc_fence_after();
        uint32_t sr[BKV];
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c)
            tmem_ld32(tS + lane_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sfree);
        // Scores in the exp2 domain.  A block needs the per-key mask only
        // if it reaches past the sequence end or some (row, key) pair of
        // the tile falls outside the window [rel_lo, rel_hi]; otherwise
        // the scale folds into the exponent's FMA: with c = scale *
        // log2(e) > 0, max(c s) = c max(s) and exp2(c s - m) =
        // exp2(fma(s, c, -m)).  Uniform across the CTA.
        const bool fast = !BIAS && kbase + BKV <= L && kbase - (q0 + 127) >= p.rel_lo &&
                          kbase + BKV - 1 - q0 <= p.rel_hi;
        float mx;
        float cs = 1.0f;  // factor applied inside the exponent
        if (fast) {
            // 8 independent partial maxima (instruction-level
            // parallelism), each taking two scores per 3-input max
            float pm[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) pm[e] = __uint_as_float(sr[e]);
#pragma unroll
            for (int c = 8; c < BKV; c += 2)
                pm[(c >> 1) & 7] = max3f(pm[(c >> 1) & 7], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
            mx = max3f(max3f(pm[0], pm[1], pm[2]), max3f(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) *
                 p.scale_log2;
            cs = p.scale_log2;
        } else if constexpr (BIAS) {
            // the bias term: one table load per key; sr stays in
            // registers (the loop is unrolled) but the loads are issued
            // a few at a time
            mx = -INFINITY;
            const float* brow = p.bias + static_cast<int64_t>(h) * (2 * p.bias_off + 1);
#pragma unroll
            for (int c = 0; c < BKV; ++c) {
                const int kj = kbase + c;
                const int rel = kj - qi;
                const int bi = min(max(rel + p.bias_off, 0), 2 * p.bias_off);
                // scores * scale + bias[h][rel] (bert.go:876-889)
                float x = (__uint_as_float(sr[c]) * p.scale + __ldg(brow + bi)) * 1.4426950408889634f;
                const bool valid = kj < L && rel >= p.rel_lo && rel <= p.rel_hi;
                x = valid ? x : -INFINITY;
                sr[c] = __float_as_uint(x);
                mx = fmaxf(mx, x);
            }
        } else {
            mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < BKV; ++c) {
                const int kj = kbase + c;
                const int rel = kj - qi;
                float x = __uint_as_float(sr[c]);
                const bool valid = kj < L && rel >= p.rel_lo && rel <= p.rel_hi;
                x *= p.scale_log2;
                x = valid ? x : -INFINITY;
                sr[c] = __float_as_uint(x);
                mx = fmaxf(mx, x);
            }
        }
        // Lazy rescaling: the exponent keeps the max it used (m) until
        // the block max exceeds it by more than 2^8, so P <= 256 and O
        // needs rescaling (and the wait for the previous P V before it)
        // only then.  The final division by l cancels the stale max.
        const bool grow = mx > m + 8.0f;  // always true while m = -inf and the row has a key
        const float m_use0 = grow ? mx : m;
        const float m_use = m_use0 == -INFINITY ? 0.f : m_use0;  // a row with no key yet keeps p = 0
        const float xoff = -m_use;
        const float alpha = ex2f(m - m_use);  // m = -inf: 0 (O and l are still 0)
        // exponentials into packed 16-bit pairs (before waiting on the
        // previous P V, so they overlap it); the row sum in 4 partials
        uint32_t pk[BKV / 2];
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < BKV / 2; ++c) {
            const float xa = fmaf(__uint_as_float(sr[2 * c]), cs, xoff);
            const float xb = fmaf(__uint_as_float(sr[2 * c + 1]), cs, xoff);
            // EMU pairs of every four on the FMA pipe
            const bool fma_pipe = (EMU >> (c & 3)) & 1;
            const float a = fma_pipe ? ex2_fma(xa) : ex2f(xa);
            const float b = fma_pipe ? ex2_fma(xb) : ex2f(xb);
            ls[c & 3] += a + b;
            pk[c] = pack2<F16>(a, b);
        }
        // The previous P V is done: the P buffer is free and O holds
        // every earlier block.
        if (i > 0) {
            if (!mbar_wait(ofull, (i - 1) & 1, status, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
        }
        l = l * alpha + ((ls[0] + ls[1]) + (ls[2] + ls[3]));
#pragma unroll
        for (int q = 0; q < BKV / 8; ++q)
            *reinterpret_cast<uint4*>(sP + r * 128 + ((q ^ (r & 7)) << 4)) =
                make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        // rescale the O row when its max moved (warp-uniform: the TMEM
        // accesses are warp-wide; rows that did not move scale by 1)
        if (i > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(tO + lane_addr + c * 32, o);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                tmem_st32(tO + lane_addr + c * 32, o);
            }
            tmem_st_wait();
        }
        m = m_use0;
        fence_proxy_async_smem();  // P (generic writes) -> the MMA (async proxy)
        tc_fence_before();         // O rescale (tcgen05.st) -> the MMA
        __syncwarp();
        if (lane == 0) mbar_arrive(pfull);
    }
    if (ok && mbar_wait(ofull, (nb - 1) & 1, status, abort_flag)) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        uint16_t* out = p.out + static_cast<int64_t>(s0 + qi) * p.ldo + h * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + lane_addr + c * 32, o);
            tmem_ld_wait();
            if (qi < L) {
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    uint4 u;
                    u.x = pack2<F16>(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
                    u.y = pack2<F16>(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
                    u.z = pack2<F16>(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
                    u.w = pack2<F16>(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
                    *reinterpret_cast<uint4*>(out + c * 32 + v * 8) = u;
                }
            }
        }
    }
}

// PLAIN: no window, no bias (only the sequence end masks keys); BIAS: the
// MPNet relative-position bias (and any window); neither: a window / causal
// mask without bias.
template <int D, bool F16, bool PLAIN, bool BIAS>
__global__ void __launch_bounds__(192, AttnTc<D>::MIN_BLOCKS)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, AttnParams p, int* status) {
    using S = AttnTc<D>;
    constexpr int BKV = S::BKV, QB = S::QB;
    pdl_wait();  // the previous kernel's outputs are complete from here on
    const int s = p.reverse ? gridDim.z - 1 - blockIdx.z : blockIdx.z, h = blockIdx.y;
    const int s0 = __ldg(p.cu + s), L = __ldg(p.cu + s + 1) - s0;
    const int q0 = blockIdx.x * 128;
    if (q0 >= L) return;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + S::Q_BYTES;  // [2][KV_BYTES]
    uint8_t* sV = sK + 2 * S::KV_BYTES;  // [VST][KV_BYTES]
    uint8_t* sP = sV + S::VST * S::KV_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + S::P_BYTES);
    uint64_t* qbar = bars + 0;
    uint64_t* kfull = bars + 1;   // [2]
    uint64_t* kempty = bars + 3;  // [2]
    uint64_t* vfull = bars + 5;   // [2]
    uint64_t* vempty = bars + 7;  // [2]
    uint64_t* sfull = bars + 9;
    uint64_t* sfree = bars + 10;
    uint64_t* pfull = bars + 11;
    uint64_t* ofull = bars + 12;
    uint64_t* drain = bars + 13;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hk = h / p.group;
    // key blocks any row of this tile may see: j - i in [rel_lo, rel_hi]
    const int jmin = max(0, q0 + p.rel_lo);
    const int jmax = min(L - 1, q0 + 127 + p.rel_hi);
    const int kb0 = jmin / BKV, nb = jmax / BKV - kb0 + 1;

    if (threadIdx.x == 0) {
        mbar_init(qbar, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&kfull[i], 1);
            mbar_init(&kempty[i], 1);
            mbar_init(&vfull[i], 1);
            mbar_init(&vempty[i], 1);
        }
        mbar_init(sfull, 1);
        mbar_init(sfree, 4);  // one arrival per softmax warp
        mbar_init(pfull, 4);
        mbar_init(ofull, 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tO = tmem + S::O_COL;
    // The next kernel (a projection) may launch only from here on: its CTAs
    // allocate TMEM before they wait for this grid, so an allocation of this
    // CTA that came after theirs on a shared SM could wait for ever.
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t armed = 0, parity = 0;  // barriers with a load in flight, their phase parity
            auto arm = [&](int bit, uint32_t ph) {
                armed |= 1u << bit;
                parity = (parity & ~(1u << bit)) | (ph << bit);
            };
            mbar_arrive_expect_tx(qbar, S::Q_BYTES);
            for (int b = 0; b < QB; ++b)
                tma_load_2d(sQ + b * 16384, &tmQ, qbar, h * D + b * 64, s0 + q0);
            arm(0, 0);
            bool ok = true;
            for (int i = 0; i < nb && ok; ++i) {
                const int row = s0 + (kb0 + i) * BKV;
                const int st = i & 1;
                if (i >= 2 && !mbar_wait(&kempty[st], ((i >> 1) - 1) & 1, status, abort_flag)) break;
                mbar_arrive_expect_tx(&kfull[st], S::KV_BYTES);
                for (int b = 0; b < QB; ++b)
                    tma_load_2d(sK + st * S::KV_BYTES + b * BKV * 128, &tmK, &kfull[st], hk * D + b * 64, row);
                arm(1 + st, (i >> 1) & 1);
                const int vs = i % S::VST, vu = i / S::VST;  // V stage and its use count
                if (vu >= 1 && !mbar_wait(&vempty[vs], (vu - 1) & 1, status, abort_flag)) break;
                mbar_arrive_expect_tx(&vfull[vs], S::KV_BYTES);
                for (int b = 0; b < QB; ++b)
                    tma_load_2d(sV + vs * S::KV_BYTES + b * BKV * 128, &tmV, &vfull[vs], hk * D + b * 64, row);
                arm(3 + vs, vu & 1);
            }
            // every load issued has landed before the CTA may exit
            if (armed & 1) mbar_drain(qbar, parity & 1);
            for (int b = 0; b < 2; ++b) {
                if (armed & (2u << b)) mbar_drain(&kfull[b], (parity >> (1 + b)) & 1);
                if (armed & (8u << b)) mbar_drain(&vfull[b], (parity >> (3 + b)) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t fmt = F16 ? 0u : 1u;
            constexpr uint32_t idS = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BKV >> 3) << 17) |
                                     ((uint32_t)(128 >> 4) << 24);
            constexpr uint32_t idO = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) |
                                     ((uint32_t)(D >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
            bool issued = false;
            // S = Q K^T of block i into the (single) S buffer, once the
            // softmax warps have read the previous one
            auto issue_s = [&](int i) -> bool {
                const int st = i & 1;
                if (!mbar_wait(&kfull[st], (i >> 1) & 1, status, abort_flag)) return false;
                if (i > 0 && !mbar_wait(sfree, (i - 1) & 1, status, abort_flag)) return false;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint64_t a = sdesc_k128(smem_u32(sQ + (ks >> 2) * 16384 + (ks & 3) * 32));
                    const uint64_t b =
                        sdesc_k128(smem_u32(sK + st * S::KV_BYTES + (ks >> 2) * BKV * 128 + (ks & 3) * 32));
                    umma_bf16(tS, a, b, idS, ks > 0);
                }
                issued = true;
                umma_commit(sfull);
                umma_commit(&kempty[st]);
                return true;
            };
            if (mbar_wait(qbar, 0, status, abort_flag) && issue_s(0)) {
                for (int i = 0; i < nb; ++i) {
                    // the next block's S goes first: it runs while the softmax
                    // warps work on this block
                    if (i + 1 < nb && !issue_s(i + 1)) break;
                    const int vs = i % S::VST, vu = i / S::VST;
                    if (!mbar_wait(pfull, i & 1, status, abort_flag) ||
                        !mbar_wait(&vfull[vs], vu & 1, status, abort_flag))
                        break;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < BKV / 16; ++kk) {
                        const uint64_t a = sdesc_k128(smem_u32(sP + (kk >> 2) * 16384 + (kk & 3) * 32));
                        const uint64_t b = sdesc_mn128(smem_u32(sV + vs * S::KV_BYTES + kk * 2048), BKV * 128);
                        umma_bf16(tO, a, b, idO, (i | kk) != 0);
                    }
                    umma_commit(ofull);
                    umma_commit(&vempty[vs]);
                }
            }
            if (issued) {
                umma_commit(drain);
                mbar_drain(drain, 0);
            }
        }
    } else {
        // ---------------- softmax (warps 2-5), thread = query row ----------------
        attn_softmax_tile<D, F16, BIAS, S::EXP_FMA_MASK>(p, h, s0, L, q0, kb0, nb, tS, tO, sP, sfull, sfree, pfull,
                                                         ofull, status, abort_flag, warp & 3, lane);
    }

    // teardown: every MMA has completed (drained by the issuer) and every
    // TMEM access of the softmax warps is done before TMEM is freed
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Multi-tile variant for long sequences with head dim 128 and no relative
// bias: one CTA holds NT consecutive 128-row query tiles of one (sequence,
// head) and streams each key / value block once for all of them.  Roles
// (128 + 128 NT threads):
//   warp 0     TMA producer: the NT Q tiles, then the K / V blocks of the
//              union of the tiles' key ranges into KVS-deep rings;
//   warp 1     TMEM allocator; warps 1 .. NT the MMA issuers, one per tile
//              (S_t = Q_t K^T of the next block, then O_t += P_t V of this
//              one);
//   warps 4t+4 .. 4t+7   the softmax of tile t (attn_softmax_tile), each
//              tile with its own S and O in TMEM, P buffer and barriers.
// Against NT separate CTAs (two per SM at this head dim) this loads K and V
// once instead of NT times and gives the softmax warps 168 registers instead
// of 128.  Measured through rg_attention (bf16, B200): Qwen3's causal layers
// at 128 x U[32, 1024] tokens 348 -> 378 TFLOP/s.  At head dim 64 the same
// design (three tiles, 512 threads) stayed below three single-tile CTAs per
// SM (620 against 682 TFLOP/s on ModernBERT's global layers), and narrow
// windows gain nothing from shared K / V blocks, so those keep the
// single-tile kernel.  One issuing thread per tile because a thread issues
// a short chain of small (128 x 64 x 16) MMAs at about one per 110 cycles
// and the chain completes some 150 cycles after its last issue (measured);
// one thread serving every tile ran the tiles one after another at half the
// single-tile kernel's rate.
template <int D, int NT>
struct AttnMt {
    static constexpr int BKV = 64;
    static constexpr int QB = D / 64;
    static constexpr int Q_BYTES = 128 * QB * 128;
    static constexpr int KV_BYTES = BKV * QB * 128;
    static constexpr int P_BYTES = 128 * BKV * 2;
    static constexpr int KVS = 2;  // K and V ring depth (power of two; 4 measured no faster)
    static constexpr int SMEM = NT * Q_BYTES + 2 * KVS * KV_BYTES + NT * P_BYTES + 1024 + 512;
    static constexpr uint32_t O_COL = NT * BKV;  // S_t at t*BKV, O_t at O_COL + t*D
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int THREADS = 128 + 128 * NT;
    static_assert(NT * (BKV + D) <= 512, "TMEM");
    // every exponential on the transcendental unit (one pair in four on the
    // FMA pipe measured 361 against 378 TFLOP/s here)
    static constexpr unsigned EXP_FMA_MASK = 0x0u;
};

template <int D, bool F16, int NT>
__global__ void __launch_bounds__(AttnMt<D, NT>::THREADS, 1)
    attention_mt_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, AttnParams p, int* status) {
    using S = AttnMt<D, NT>;
    constexpr int BKV = S::BKV, QB = S::QB;
    pdl_wait();
    const int s = p.reverse ? gridDim.z - 1 - blockIdx.z : blockIdx.z, h = blockIdx.y;
    const int s0 = __ldg(p.cu + s), L = __ldg(p.cu + s + 1) - s0;
    const int q0 = blockIdx.x * 128 * NT;
    if (q0 >= L) return;
    const int nt = min(NT, (L - q0 + 127) / 128);  // tiles with rows in the sequence

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                       // [NT][Q_BYTES]
    constexpr int KVS = S::KVS, KSH = KVS == 4 ? 2 : (KVS == 2 ? 1 : 3);  // log2 KVS
    static_assert((1 << KSH) == KVS, "ring depth");
    uint8_t* sK = sQ + NT * S::Q_BYTES;       // [KVS][KV_BYTES]
    uint8_t* sV = sK + KVS * S::KV_BYTES;     // [KVS][KV_BYTES]
    uint8_t* sP = sV + KVS * S::KV_BYTES;     // [NT][P_BYTES]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + NT * S::P_BYTES);
    uint64_t* qbar = bars + 0;
    uint64_t* kfull = bars + 1;              // [KVS]
    uint64_t* kempty = kfull + KVS;          // [KVS]
    uint64_t* vfull = kempty + KVS;          // [KVS]
    uint64_t* vempty = vfull + KVS;          // [KVS]
    uint64_t* drain = vempty + KVS;          // [NT]: one per issuer
    uint64_t* tb = drain + NT;               // per tile t: sfull, sfree, pfull, ofull at tb + 4 t
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tb + 4 * NT);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hk = h / p.group;
    // each tile's key blocks (rows q0 + 128 t ...: j - i in [rel_lo, rel_hi])
    // and their union
    int kbt[NT], nbt[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const int qt = q0 + 128 * t;
        const int jmin = max(0, qt + p.rel_lo), jmax = min(L - 1, qt + 127 + p.rel_hi);
        kbt[t] = jmin / BKV;
        nbt[t] = t < nt ? jmax / BKV - kbt[t] + 1 : 0;
    }
    int kb0 = kbt[0], kb1 = kbt[0] + nbt[0];
#pragma unroll
    for (int t = 1; t < NT; ++t)
        if (t < nt) {
            kb0 = min(kb0, kbt[t]);
            kb1 = max(kb1, kbt[t] + nbt[t]);
        }
    const int nb = kb1 - kb0;

    if (threadIdx.x == 0) {
        mbar_init(qbar, 1);
        for (int i = 0; i < KVS; ++i) {
            mbar_init(&kfull[i], 1);
            mbar_init(&kempty[i], nt);  // one arrival per active tile's issuer
            mbar_init(&vfull[i], 1);
            mbar_init(&vempty[i], nt);
        }
        for (int t = 0; t < NT; ++t) {
            mbar_init(drain + t, 1);
            mbar_init(tb + 4 * t + 0, 1);  // sfull
            mbar_init(tb + 4 * t + 1, 4);  // sfree: one arrival per softmax warp
            mbar_init(tb + 4 * t + 2, 4);  // pfull
            mbar_init(tb + 4 * t + 3, 1);  // ofull
        }
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The next kernel (a projection) may launch only from here on: its CTAs
    // allocate TMEM before they wait for this grid, so an allocation of this
    // CTA that came after theirs on a shared SM could wait for ever.
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t armed = 0, parity = 0;  // barriers with a load in flight, their phase parity
            auto arm = [&](int bit, uint32_t ph) {
                armed |= 1u << bit;
                parity = (parity & ~(1u << bit)) | (ph << bit);
            };
            mbar_arrive_expect_tx(qbar, nt * S::Q_BYTES);
            for (int t = 0; t < nt; ++t)
                for (int b = 0; b < QB; ++b)
                    tma_load_2d(sQ + t * S::Q_BYTES + b * 16384, &tmQ, qbar, h * D + b * 64, s0 + q0 + 128 * t);
            arm(0, 0);
            for (int i = 0; i < nb; ++i) {
                const int row = s0 + (kb0 + i) * BKV;
                const int st = i & (KVS - 1);
                const uint32_t ph = (i >> KSH) & 1;
                if (i >= KVS && !mbar_wait(&kempty[st], ph ^ 1, status, abort_flag)) break;
                mbar_arrive_expect_tx(&kfull[st], S::KV_BYTES);
                for (int b = 0; b < QB; ++b)
                    tma_load_2d(sK + st * S::KV_BYTES + b * BKV * 128, &tmK, &kfull[st], hk * D + b * 64, row);
                arm(1 + st, ph);
                if (i >= KVS && !mbar_wait(&vempty[st], ph ^ 1, status, abort_flag)) break;
                mbar_arrive_expect_tx(&vfull[st], S::KV_BYTES);
                for (int b = 0; b < QB; ++b)
                    tma_load_2d(sV + st * S::KV_BYTES + b * BKV * 128, &tmV, &vfull[st], hk * D + b * 64, row);
                arm(1 + KVS + st, ph);
            }
            // every load issued has landed before the CTA may exit
            if (armed & 1) mbar_drain(qbar, parity & 1);
            for (int b = 0; b < KVS; ++b) {
                if (armed & (2u << b)) mbar_drain(&kfull[b], (parity >> (1 + b)) & 1);
                if (armed & (2u << (KVS + b))) mbar_drain(&vfull[b], (parity >> (1 + KVS + b)) & 1);
            }
        }
    } else if (warp <= NT) {
        // ---------------- MMA issuer of tile t = warp - 1 ----------------
        // One issuing thread per tile: a thread issues a short chain of
        // small MMAs at about one per 100 cycles and waits some 150 more for
        // it to complete, so one thread serving every tile would serialise
        // them.  Each issuer walks the union's blocks in order; a K / V
        // stage is released by one arrival per active tile (after the
        // tile's MMAs on it complete, or at once for a block outside the
        // tile's range once the block has landed, so that the arrival counts
        // toward that block's phase).
        const int t = warp - 1;
        if (lane == 0 && t < nt) {
            constexpr uint32_t fmt = F16 ? 0u : 1u;
            constexpr uint32_t idS = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BKV >> 3) << 17) |
                                     ((uint32_t)(128 >> 4) << 24);
            constexpr uint32_t idO = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) |
                                     ((uint32_t)(D >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
            int f = 0, e = 0;  // the tile's union blocks [f, e)
#pragma unroll
            for (int j = 0; j < NT; ++j)
                if (j == t) {
                    f = kbt[j] - kb0;
                    e = f + nbt[j];
                }
            const uint32_t tS = tmem + t * BKV, tO = tmem + S::O_COL + t * D;
            const uint8_t* q = sQ + t * S::Q_BYTES;
            const uint8_t* pp = sP + t * S::P_BYTES;
            uint64_t* sfull = tb + 4 * t + 0;
            uint64_t* sfree = tb + 4 * t + 1;
            uint64_t* pfull = tb + 4 * t + 2;
            uint64_t* ofull = tb + 4 * t + 3;
            bool issued = false;
            auto s_step = [&](int u) -> bool {
                const int st = u & (KVS - 1);
                if (!mbar_wait(&kfull[st], (u >> KSH) & 1, status, abort_flag)) return false;
                if (u < f || u >= e) {
                    mbar_arrive(&kempty[st]);
                    return true;
                }
                const int it = u - f;
                if (it > 0 && !mbar_wait(sfree, (it - 1) & 1, status, abort_flag)) return false;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint64_t a = sdesc_k128(smem_u32(q + (ks >> 2) * 16384 + (ks & 3) * 32));
                    const uint64_t b =
                        sdesc_k128(smem_u32(sK + st * S::KV_BYTES + (ks >> 2) * BKV * 128 + (ks & 3) * 32));
                    umma_bf16(tS, a, b, idS, ks > 0);
                }
                issued = true;
                umma_commit(sfull);
                umma_commit(&kempty[st]);
                return true;
            };
            auto pv_step = [&](int u) -> bool {
                const int st = u & (KVS - 1);
                if (u < f || u >= e) {
                    if (!mbar_wait(&vfull[st], (u >> KSH) & 1, status, abort_flag)) return false;
                    mbar_arrive(&vempty[st]);
                    return true;
                }
                const int it = u - f;
                if (!mbar_wait(pfull, it & 1, status, abort_flag) ||
                    !mbar_wait(&vfull[st], (u >> KSH) & 1, status, abort_flag))
                    return false;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < BKV / 16; ++kk) {
                    const uint64_t a = sdesc_k128(smem_u32(pp + (kk >> 2) * 16384 + (kk & 3) * 32));
                    const uint64_t b = sdesc_mn128(smem_u32(sV + st * S::KV_BYTES + kk * 2048), BKV * 128);
                    umma_bf16(tO, a, b, idO, (it | kk) != 0);
                }
                umma_commit(ofull);
                umma_commit(&vempty[st]);
                return true;
            };
            if (mbar_wait(qbar, 0, status, abort_flag) && s_step(0)) {
                for (int u = 0; u < nb; ++u) {
                    // the next block's S first: it runs while the softmax
                    // warps work on this block
                    if (u + 1 < nb && !s_step(u + 1)) break;
                    if (!pv_step(u)) break;
                }
            }
            if (issued) {
                umma_commit(drain + t);
                mbar_drain(drain + t, 0);
            }
        }
    } else if (warp >= 4) {
        // ---------------- softmax of tile t ----------------
        const int t = (warp - 4) >> 2;
        // the tile's key range, selected with constant indices so that kbt
        // and nbt stay in registers (a runtime index would put them in local
        // memory, read on every step of the issuer's loop)
        int my_kb = 0, my_nb = 0;
#pragma unroll
        for (int j = 0; j < NT; ++j)
            if (j == t) {
                my_kb = kbt[j];
                my_nb = nbt[j];
            }
        if (t < nt)
            attn_softmax_tile<D, F16, false, S::EXP_FMA_MASK>(
                p, h, s0, L, q0 + 128 * t, my_kb, my_nb, tmem + t * BKV, tmem + S::O_COL + t * D,
                sP + t * S::P_BYTES, tb + 4 * t + 0, tb + 4 * t + 1, tb + 4 * t + 2, tb + 4 * t + 3, status,
                abort_flag, warp & 3, lane);
    }

    // teardown: every MMA has completed (drained by the issuer) and every
    // TMEM access of the softmax warps is done before TMEM is freed
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn_attn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// [rows x cols] 16-bit matrix with row stride ld elements; boxes of 64
// columns (128 bytes, 128-byte swizzle) x box_rows.
static bool make_rows_tmap(CUtensorMap* map, const void* base, bool f16, uint64_t rows, uint64_t cols, uint64_t ld,
                           uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn_attn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 2) % 16 != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
              const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, bool F16, bool PLAIN, bool BIAS>
static cudaError_t launch_tc(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const AttnParams& p, int nseq, int max_len, int heads, int* status, cudaStream_t st) {
    constexpr int smem = AttnTc<D>::SMEM;
    auto kern = attention_tc_kernel<D, F16, PLAIN, BIAS>;
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 32) __atomic_fetch_or(&configured, 1u << dev, __ATOMIC_RELEASE);
    }
    const dim3 grid((max_len + 127) / 128, heads, nseq);
    launch_pdl(kern, grid, dim3(AttnTc<D>::THREADS), smem, st, tq, tk, tv, p, status);
    return cudaGetLastError();
}

template <int D, bool F16, int NT>
static cudaError_t launch_mt(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const AttnParams& p, int nseq, int max_len, int heads, int* status, cudaStream_t st) {
    using S = AttnMt<D, NT>;
    auto kern = attention_mt_kernel<D, F16, NT>;
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
        if (e != cudaSuccess) return e;
        if (dev < 32) __atomic_fetch_or(&configured, 1u << dev, __ATOMIC_RELEASE);
    }
    const dim3 grid((max_len + 128 * NT - 1) / (128 * NT), heads, nseq);
    launch_pdl(kern, grid, dim3(S::THREADS), S::SMEM, st, tq, tk, tv, p, status);
    return cudaGetLastError();
}

// The multi-tile kernel takes a head-dim-128 batch without bias whose
// sequences average at least kMtMinAvg tokens and whose window spans at
// least kMtMinSpan keys (causal and bidirectional layers; a narrow window
// leaves the tiles little K / V to share).
constexpr int kMtMinAvg = 384;
constexpr int kMtMinSpan = 1024;

bool attention_tc_supported(int head_dim) {
    return head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256;
}

cudaError_t launch_attention_tc(const AttnParams& p, int T, int nseq, int max_len, int heads, int kv_heads,
                                int head_dim, int* status, cudaStream_t st) {
    if (nseq <= 0 || T <= 0) return cudaSuccess;
    const int D = head_dim;
    if (!attention_tc_supported(D) || !status) return cudaErrorInvalidValue;
    const int bkv = 64;
    CUtensorMap tq, tk, tv;
    if (!make_rows_tmap(&tq, p.q, p.f16, T, static_cast<uint64_t>(heads) * D, p.ldq, 128) ||
        !make_rows_tmap(&tk, p.k, p.f16, T, static_cast<uint64_t>(kv_heads) * D, p.ldk, bkv) ||
        !make_rows_tmap(&tv, p.v, p.f16, T, static_cast<uint64_t>(kv_heads) * D, p.ldv, bkv))
        return cudaErrorInvalidValue;
    const bool plain = !p.bias && p.rel_lo <= -max_len && p.rel_hi >= max_len;
    if (D == 128 && !p.bias && T >= static_cast<int64_t>(kMtMinAvg) * nseq &&
        static_cast<int64_t>(p.rel_hi) - p.rel_lo >= kMtMinSpan) {
        if (p.f16) return launch_mt<128, true, 2>(tq, tk, tv, p, nseq, max_len, heads, status, st);
        return launch_mt<128, false, 2>(tq, tk, tv, p, nseq, max_len, heads, status, st);
    }
#define RG_TC_CASE(DD, FF)                                                                         \
    if (D == DD && p.f16 == FF) {                                                                  \
        if (p.bias) return launch_tc<DD, FF, false, true>(tq, tk, tv, p, nseq, max_len, heads, status, st); \
        if (plain) return launch_tc<DD, FF, true, false>(tq, tk, tv, p, nseq, max_len, heads, status, st);  \
        return launch_tc<DD, FF, false, false>(tq, tk, tv, p, nseq, max_len, heads, status, st);            \
    }
    RG_TC_CASE(32, false)
    RG_TC_CASE(32, true)
    RG_TC_CASE(64, false)
    RG_TC_CASE(64, true)
    RG_TC_CASE(128, false)
    RG_TC_CASE(128, true)
    RG_TC_CASE(256, false)
    RG_TC_CASE(256, true)
#undef RG_TC_CASE
    return cudaErrorInvalidValue;
}

}  // namespace rg
