// gemm_impl.cuh - persistent warp-specialised tcgen05 GEMM for sm_100a on CTA
// pairs (clusters of 2, tcgen05 cta_group::2).
//
// Each CTA pair walks output tiles of 256 x BN in m-major order (pairs in
// flight share A row-blocks through L2).  The pair MMA reads 128 rows of A
// and BN/2 rows of W from each CTA's shared memory and writes each CTA's
// 128 output rows into that CTA's TMEM, so per SM a k-block moves half the
// W bytes a single-CTA 128 x BN tile would.  Roles in every CTA:
//   warp 0      TMA producer: its CTA's A and W k-blocks (128 bytes of K per
//               row, 128-byte swizzle) into a STAGES-deep ring; both CTAs'
//               loads complete on the even CTA's barrier;
//   warp 1      (even CTA only) pair MMA issuer: 4 tcgen05.mma per k-block
//               into one of two TMEM accumulators, commits that free the
//               stage in both CTAs and publish finished accumulators;
//   warp 2      TMEM allocator (pair allocation);
//   warps 2-3   (kW8 only, after the allocation) converters: widen this
//               CTA's int8 W k-block to fp16 in the 128-byte-swizzled
//               layout the MMA reads, then arrive on the even CTA's barrier;
//   warps 4-11  epilogue: tcgen05.ld 32 columns at a time (thread = row),
//               dequant scales, bias, GELU or + residual (TMA-loaded) in
//               registers, the row into a swizzled staging box, one TMA
//               store per 32 x 32 box; then release the accumulator to the
//               even CTA so the next tile's MMAs overlap this epilogue.
// All waits are bounded (sm100.cuh); on a timeout every role stops, the
// loads and MMAs in flight are drained, and the pair's TMEM is freed before
// the CTAs exit with kStatusWaitTimeout raised.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "act16.cuh"
#include "gemm.cuh"
#include "pdl.cuh"
#include "sm100.cuh"

namespace rg {

// ---- packed fp32 pairs (sm_100 f32x2 ALU ops: two lanes of work per issue)
__device__ __forceinline__ uint64_t f2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2split(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// HF "gelu", 0.5 x (1 + erf(x / sqrt(2))), on a pair, with erf by
// Abramowitz & Stegun 7.1.28 (Hastings): erf(a) = 1 - (1 + a1 a + ... +
// a6 a^6)^-16, |error| <= 3e-7.  The reference's geluScalar (tensor.go:
// 499-538) uses A&S 7.1.26 (1.5e-7); the two differ by three orders of
// magnitude less than the 16-bit rounding of the output, and 7.1.28 needs
// one reciprocal and no exponential on the transcendental unit (7.1.26
// needs both).  The polynomial and the four squarings run on f32x2, with
// a = |x| / sqrt(2) folded into the coefficients (b_k = a_k / sqrt(2)^k):
// r = p(|x|)^-16, gelu(x) = x - x r / 2 for x >= 0 and x r / 2 for x < 0
// (max |error| 7e-7 over [-12, 12] in fp32).
__device__ __forceinline__ void gelu_as28x2(float& x0, float& x1) {
    const uint64_t xs = f2(x0, x1);
    const uint64_t ax = f2(fabsf(x0), fabsf(x1));
    uint64_t p = fma2(ax, f2(5.382975e-06f, 5.382975e-06f), f2(4.8890636e-05f, 4.8890636e-05f));
    p = fma2(p, ax, f2(3.8003575e-05f, 3.8003575e-05f));
    p = fma2(p, ax, f2(3.2776263e-03f, 3.2776263e-03f));
    p = fma2(p, ax, f2(2.1141006e-02f, 2.1141006e-02f));
    p = fma2(p, ax, f2(4.9867347e-02f, 4.9867347e-02f));
    p = fma2(p, ax, f2(1.0f, 1.0f));
    p = mul2(p, p);  // p^2
    p = mul2(p, p);  // p^4
    p = mul2(p, p);  // p^8
    p = mul2(p, p);  // p^16
    float q0, q1;
    f2split(p, q0, q1);
    const uint64_t r = f2(rcp_approx(q0), rcp_approx(q1));  // an overflowed p^16 (|x| > ~28) gives 0
    const uint64_t hr = mul2(mul2(xs, f2(0.5f, 0.5f)), r);  // x r / 2
    float h0, h1;
    f2split(hr, h0, h1);
    x0 = x0 >= 0.f ? x0 - h0 : h0;
    x1 = x1 >= 0.f ? x1 - h1 : h1;
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// x * sigmoid(z) on a pair as x / (1 + 2^(-z log2 e)) with the hardware
// exponential and reciprocal approximations (relative error about 1e-6,
// against the gated output's 16-bit rounding of 2^-9 or 2^-12).  z -> -inf
// gives 1/inf = 0.
__device__ __forceinline__ void x_sigmoid_x2(float& x0, float& x1, float z0, float z1) {
    float t0, t1;
    f2split(mul2(f2(z0, z1), f2(-1.4426950408889634f, -1.4426950408889634f)), t0, t1);
    float d0, d1;
    f2split(add2(f2(ex2_approx(t0), ex2_approx(t1)), f2(1.0f, 1.0f)), d0, d1);
    f2split(mul2(f2(x0, x1), f2(rcp_approx(d0), rcp_approx(d1))), x0, x1);
}
// SiLU x * sigmoid(x) (tensor.go:477-481 computes it through a float64 exp).
__device__ __forceinline__ void silu_x2(float& x0, float& x1) { x_sigmoid_x2(x0, x1, x0, x1); }
// tanh-approximation GELU (tensor.go:490-497; HF gelu_pytorch_tanh):
// 0.5 x (1 + tanh(u)) = x * sigmoid(2u), u = sqrt(2/pi) (x + 0.044715 x^3).
__device__ __forceinline__ void gelu_tanh_x2(float& x0, float& x1) {
    constexpr float c0 = 2.0f * 0.7978845608028654f, c1 = 2.0f * 0.7978845608028654f * 0.044715f;
    const uint64_t xs = f2(x0, x1);
    const uint64_t p = fma2(mul2(xs, xs), f2(c1, c1), f2(c0, c0));  // c0 + c1 x^2
    float z0, z1;
    f2split(mul2(p, xs), z0, z1);
    x_sigmoid_x2(x0, x1, z0, z1);
}

constexpr int kEpiWarps = 8;        // two epilogue warps per SM sub-partition
constexpr int kThreads = 128 + 32 * kEpiWarps;
constexpr int kChunk = 32;          // accumulator columns per TMEM load / TMA store box
constexpr int kStageBytes = 4096;   // one 32 x 32 fp32 (or 32 x 32 bf16, half used) staging box
constexpr int kY16Bytes = 2048;     // one 32 x 32 16-bit staging box

// Per-CTA shapes of the pair kernel: the tile is 256 x BN, each CTA of the
// pair holds 128 rows of A and BN/2 rows of W per 128-byte k-block.  With
// int8 weights widened in shared memory (W8), each stage also holds the
// int8 k-block as loaded (64 bytes x BN/2 rows).
// Residual epilogues of the 16-bit kinds (Y16) also stage the output's
// 16-bit copy: one 32 x 32 box per epilogue warp.
template <int BN, int KIND, int EPI>
struct GemmShape {
    static constexpr bool W8 = KIND == static_cast<int>(GemmKind::kW8);
    static constexpr bool Y16 = (EPI == kEpiBiasRes || EPI == kEpiBiasResLN) &&
                                (KIND == static_cast<int>(GemmKind::kBF16) || KIND == static_cast<int>(GemmKind::kF16) ||
                                 KIND == static_cast<int>(GemmKind::kW8));
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = (BN / 2) * 128;
    static constexpr int B8_BYTES = W8 ? (BN / 2) * 64 : 0;
    static constexpr int Y16_BYTES = Y16 ? kEpiWarps * kY16Bytes : 0;
    static constexpr int STAGES =
        W8 ? (BN == 128 ? 5 : (Y16 && BN == 256 ? 3 : 4)) : (BN == 128 ? 6 : (Y16 && BN == 256 ? 4 : 5));
    static constexpr uint32_t TMEM_COLS = BN == 128 ? 256 : 512;  // 2 accumulators, power of two
    // mainloop ring + two staging boxes per epilogue warp (+ the 16-bit
    // copy's box) + barriers
    static constexpr int SMEM =
        STAGES * (A_BYTES + B_BYTES + B8_BYTES) + kEpiWarps * 2 * kStageBytes + Y16_BYTES + 1024 + 512;
};

// Four int8 weights (bytes of x) to four exact fp16 values (lo: elements 0,
// 1; hi: 2, 3).  The IEEE magic-number method: q + 128 in [0, 255] placed in
// the low mantissa byte of 1024.0 (0x6400) is exactly 1024 + q + 128 as an
// fp16, and subtracting 1152.0 (0x6480) leaves q.
__device__ __forceinline__ void widen_s8x4_f16(uint32_t x, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = x ^ 0x80808080u;
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(a) : "r"(u), "r"(0x64646464u), "r"(0x4140u));
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(b) : "r"(u), "r"(0x64646464u), "r"(0x4342u));
    const uint32_t magic = 0x64806480u;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(magic));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(magic));
}

// Byte offset of 16-byte chunk c of row r in a staging box whose rows are
// row_bytes long, laid out as the TMA swizzle of the store/load map expects
// (128-byte swizzle for fp32 rows, 64-byte swizzle for bf16 rows): chunk bits
// [4,7) are XORed with bits [7,10) of the unswizzled offset.
__device__ __forceinline__ uint32_t swz(int r, int c, int row_bytes) {
    const uint32_t off = static_cast<uint32_t>(r * row_bytes + c * 16);
    const uint32_t mask = row_bytes == 128 ? 7u : 3u;
    return off ^ (((off >> 7) & mask) << 4);
}

template <int BN, int KIND, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmRes,
                const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                const __grid_constant__ CUtensorMap tmOut16, GemmArgs args) {
    constexpr bool S8 = KIND == static_cast<int>(GemmKind::kS8);
    constexpr bool W8 = KIND == static_cast<int>(GemmKind::kW8);
    constexpr bool F16 = KIND == static_cast<int>(GemmKind::kF16) || W8;  // fp16 operands and output
    // 3xTF32: fp32 operands split hi + lo, K walked three times
    // (A_hi W_hi, A_hi W_lo, A_lo W_hi), fp32 outputs
    constexpr bool X3 = KIND == static_cast<int>(GemmKind::kTF32x3);
    constexpr bool CSCALE = true;  // per-column dequant scales, whenever args.col_scale is set
    using S = GemmShape<BN, KIND, EPI>;
    constexpr int STAGES = S::STAGES;
    constexpr int A_BYTES = S::A_BYTES, B_BYTES = S::B_BYTES, B8_BYTES = S::B8_BYTES;
    constexpr int K_ELEMS = S8 ? 128 : (X3 ? 32 : 64);  // elements per 128-byte k-block of A
    constexpr int HALF = BN / 2;            // W rows per CTA; accumulator columns per epilogue warp
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;          // W k-blocks as the MMA reads them
    uint8_t* sB8 = sB + STAGES * B_BYTES;           // W8: int8 k-blocks as loaded
    uint8_t* stage_base = sB8 + STAGES * B8_BYTES;  // 1024-byte aligned
    uint8_t* y16_base = stage_base + kEpiWarps * 2 * kStageBytes;  // Y16: [kEpiWarps] 16-bit boxes
    uint64_t* full = reinterpret_cast<uint64_t*>(y16_base + S::Y16_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* resbar = tempty + 2;  // [kEpiWarps][2]: residual box landed
    uint64_t* drain = resbar + 2 * kEpiWarps;
    uint64_t* wfull = drain + 1;        // W8 [STAGES]: this CTA's int8 k-block landed
    uint64_t* cfull = wfull + STAGES;   // W8 [STAGES] (even CTA): both CTAs' k-blocks widened
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cfull + STAGES);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0: the CTA that issues the pair MMAs
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int m_tiles = (args.M + 255) / 256;
    const int n_tiles = args.N / BN;
    const int num_tiles = m_tiles * n_tiles;
    // Row block of a tile: m-major order, last row block first when
    // args.reverse_m (so that the rows the previous kernel wrote last, still
    // in L2, are read first).
    auto m_of = [&](int t) { return args.reverse_m ? m_tiles - 1 - t / n_tiles : t / n_tiles; };
    const int kb_real = args.K / K_ELEMS;
    const int kblocks = X3 ? 3 * kb_real : kb_real;
    const long long wlim = args.wait_limit > 0 ? args.wait_limit : kWaitLimitCycles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * kEpiWarps);  // one arrival per epilogue warp of both CTAs
        }
        for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&resbar[i], 1);
        mbar_init(drain, 1);
        if constexpr (W8) {
            for (int s = 0; s < STAGES; ++s) {
                mbar_init(&wfull[s], 1);
                mbar_init(&cfull[s], 4);  // the two converter warps of both CTAs
            }
        }
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (X3) {
            tma_prefetch_desc(&tmA2);
            tma_prefetch_desc(&tmB2);
        }
        tma_prefetch_desc(&tmOut);
        if (EPI == kEpiBiasRes || EPI == kEpiBiasResLN) tma_prefetch_desc(&tmRes);
        if (S::Y16 && args.out16) tma_prefetch_desc(&tmOut16);
    }
    if (warp == 2) {
        tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    pdl_trigger();
    pdl_wait();  // the previous kernel's outputs (A, residual, statistics) are complete from here on
    const uint32_t tmem_base = *tmem_slot;
    // shared::cluster addresses of the even CTA's full / tempty barriers.
    const uint32_t full_lead = mapa_shared(smem_u32(full), 0);
    const uint32_t tempty_lead = mapa_shared(smem_u32(tempty), 0);

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t issued_mask = 0, issued_parity = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs) {
            const int m_blk = m_of(tile), n_blk = tile % n_tiles;
            bool ok = true;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&empty[stage], phase ^ 1, args.status, abort_flag, wlim)) {
                    ok = false;
                    break;
                }
                // Both CTAs' loads complete on the even CTA's barrier, which
                // expects the bytes of both.
                const bool withhold = args.inject_withhold && tile == pair && kb == 0;
                if (rank == 0 && !withhold) mbar_arrive_expect_tx(&full[stage], 2 * (A_BYTES + (W8 ? 0 : B_BYTES)));
                // 3xTF32: segment 0 = (A_hi, W_hi), 1 = (A_hi, W_lo), 2 = (A_lo, W_hi)
                const int seg = X3 ? kb / kb_real : 0;
                const int kx = (X3 ? kb - seg * kb_real : kb) * K_ELEMS;
                tma_load_2d_pair(sA + stage * A_BYTES, seg == 2 ? &tmA2 : &tmA, full_lead + 8 * stage, kx,
                                 m_blk * 256 + rank * 128);
                if constexpr (W8) {
                    // the int8 k-block lands on this CTA's own barrier for its converters
                    mbar_arrive_expect_tx(&wfull[stage], B8_BYTES);
                    tma_load_2d(sB8 + stage * B8_BYTES, &tmB, &wfull[stage], kx, n_blk * BN + rank * HALF);
                } else {
                    tma_load_2d_pair(sB + stage * B_BYTES, seg == 1 ? &tmB2 : &tmB, full_lead + 8 * stage, kx,
                                     n_blk * BN + rank * HALF);
                }
                issued_mask |= 1u << stage;
                issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
        }
        // The even CTA sees every load of both CTAs land on its barriers;
        // each CTA sees its own int8 W loads land.
        for (int s = 0; s < STAGES; ++s) {
            if (!(issued_mask & (1u << s))) continue;
            if (rank == 0) mbar_drain(&full[s], (issued_parity >> s) & 1, wlim);
            if constexpr (W8) mbar_drain(&wfull[s], (issued_parity >> s) & 1, wlim);
        }
    } else if (W8 && (warp == 2 || warp == 3)) {
        // ---------------- int8 -> fp16 converters (kW8, both CTAs) ----------------
        // 16 weights (one 16-byte chunk of a 64-byte int8 row) per step:
        // row r, chunk q -> fp16 chunks 2q, 2q + 1 of the 128-byte row,
        // placed at chunk ^ (r & 7) as the 128-byte swizzle of a
        // 1024-byte-aligned tile requires.
        const int ct = (warp - 2) * 32 + lane;
        const uint32_t cfull_lead = mapa_shared(smem_u32(cfull), 0);
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&wfull[stage], phase, args.status, abort_flag, wlim)) {
                    ok = false;
                    break;
                }
                const uint8_t* src = sB8 + stage * B8_BYTES;
                uint8_t* dst = sB + stage * B_BYTES;
#pragma unroll 4
                for (int i = ct; i < HALF * 4; i += 64) {
                    const int r = i >> 2, q = i & 3;
                    const uint4 u = *reinterpret_cast<const uint4*>(src + i * 16);
                    uint4 lo, hi;
                    widen_s8x4_f16(u.x, lo.x, lo.y);
                    widen_s8x4_f16(u.y, lo.z, lo.w);
                    widen_s8x4_f16(u.z, hi.x, hi.y);
                    widen_s8x4_f16(u.w, hi.z, hi.w);
                    uint8_t* row = dst + r * 128;
                    *reinterpret_cast<uint4*>(row + (((2 * q) ^ (r & 7)) << 4)) = lo;
                    *reinterpret_cast<uint4*>(row + (((2 * q + 1) ^ (r & 7)) << 4)) = hi;
                }
                // generic-proxy writes -> visible to the MMA's async-proxy reads
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(cfull_lead + 8 * stage);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ---------------- pair MMA issuer (even CTA) ----------------
        constexpr uint32_t idesc =
            S8 ? idesc_s8(256, BN) : (F16 ? idesc_f16(256, BN) : (X3 ? idesc_tf32(256, BN) : idesc_bf16(256, BN)));
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool issued = false;
        for (int tile = pair; tile < num_tiles; tile += npairs) {
            if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.status, abort_flag, wlim)) break;
            tc_fence_after();
            const uint32_t d = tmem_base + acc * BN;
            bool ok = true;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&full[stage], phase, args.status, abort_flag, wlim) ||
                    (W8 && !mbar_wait(&cfull[stage], phase, args.status, abort_flag, wlim))) {
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
                        umma_s8_pair(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
                    else if constexpr (X3)
                        umma_tf32_pair(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
                    else
                        umma_bf16_pair(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
                }
                issued = true;
                // Free this stage in both CTAs once the MMAs have read it.
                umma_commit_pair_mc(smem_u32(&empty[stage]), 0x3);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
            umma_commit_pair_mc(smem_u32(&tfull[acc]), 0x3);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (issued) {
            umma_commit_pair(smem_u32(drain));
            mbar_drain(drain, 0, wlim);
        }
    } else if (warp >= 4) {
        // ---------------- epilogue (both CTAs, own 128 rows) ----------------
        // Warp (4 + 4h + q) owns TMEM lanes [32q, 32q + 32) (the lane quarter
        // its sub-partition may access) = 32 output rows, and accumulator
        // columns [h*HALF, (h+1)*HALF), processed 32 at a time: tcgen05.ld
        // (thread = row), dequant / bias / GELU / + residual in registers,
        // the row written into a swizzled staging box, one TMA store per box.
        // The fp32 residual box arrives by TMA one chunk ahead.
        constexpr bool RES = EPI == kEpiBiasRes || EPI == kEpiBiasResLN;
        constexpr bool F32OUT = RES || EPI == kEpiBiasF32 || X3;
        const int ew = warp - 4;
        const int quarter = warp & 3;
        const int half = ew >> 2;
        uint8_t* boxes = stage_base + ew * 2 * kStageBytes;
        uint64_t* rbar = resbar + 2 * ew;
        uint32_t rphase = 0;   // bit b: parity of the next completion of rbar[b]
        uint32_t rpending = 0; // bit b: a residual load into buffer b is in flight (lane 0's view)
        int k = 0;             // running chunk counter of this warp: buffer k & 1
        constexpr int CHUNKS = HALF / kChunk;
        // Issue the residual box of chunk c of tile t into buffer b (lane 0).
        auto load_residual = [&](int t, int c, int b) {
            if constexpr (RES) {
                if (t >= num_tiles) return;
                const int row0 = m_of(t) * 256 + static_cast<int>(rank) * 128 + quarter * 32;
                const int col0 = (t % n_tiles) * BN + half * HALF + c * kChunk;
                mbar_arrive_expect_tx(&rbar[b], kStageBytes);
                tma_load_2d(boxes + b * kStageBytes, &tmRes, &rbar[b], col0, row0);
                rpending |= 1u << b;
            }
        };
        if (lane == 0) load_residual(pair, 0, 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
            const int m_blk = m_of(tile), n_blk = tile % n_tiles;
            const int row0 = m_blk * 256 + static_cast<int>(rank) * 128 + quarter * 32;
            const int row = row0 + lane;
            // Per-row operands of the epilogue, fetched while the tile's MMAs run.
            float rs = 1.0f;
            if constexpr (S8) {
                if (args.row_scale && row < args.M) rs = args.row_scale[row];
            }
            float2 lnst = make_float2(0.f, 1.f);  // this row's (mean, rstd) for kEpiBiasResLN
            if constexpr (EPI == kEpiBiasResLN) {
                if (row < args.M) lnst = args.ln_stats[row];
            }
            // folded LayerNorm of the A rows: rstd and -rstd * mean
            float fr = 1.f, fnm = 0.f;
            if constexpr (EPI == kEpiBias || EPI == kEpiBiasGelu || EPI == kEpiRope ||
                          (EPI >= kEpiGluSilu && EPI <= kEpiGluGeluTanh)) {
                if (args.fold_stats && row < args.M) {
                    const float2 st = args.fold_stats[row];
                    fr = st.y;
                    fnm = -st.x * st.y;
                }
            }
            if (!mbar_wait(&tfull[acc], acc_phase, args.status, abort_flag, wlim)) break;
            tc_fence_after();
            const uint32_t taddr =
                tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN + half * HALF;
            constexpr bool GLU = EPI >= kEpiGluSilu && EPI <= kEpiGluGeluTanh;
            constexpr int STEP = GLU ? 2 : 1;  // accumulator chunks per output box
            if constexpr (EPI == kEpiRope) {
                // Heads of dh columns, whole inside this warp's HALF columns.
                // The projection values of 16 columns from col on: dequantised
                // (int8 kinds), then the folded norm or + bias, with the same
                // vector loads and packed arithmetic as kEpiBias.
                auto values16 = [&](const uint32_t (&r)[16], int col, float (&x)[16]) {
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        x[i] = S8 ? static_cast<float>(static_cast<int32_t>(r[i])) * rs : __uint_as_float(r[i]);
                    if (args.col_scale) {
                        const float4* cp = reinterpret_cast<const float4*>(args.col_scale + col);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float4 q = __ldg(cp + i);
                            x[4 * i] *= q.x;
                            x[4 * i + 1] *= q.y;
                            x[4 * i + 2] *= q.z;
                            x[4 * i + 3] *= q.w;
                        }
                    }
                    if (args.fold_stats) {  // rstd * acc + (bias - rstd * mean * c1)
                        const float4* c1 = reinterpret_cast<const float4*>(args.fold_c1 + col);
                        const float4* bp = reinterpret_cast<const float4*>(args.bias + col);
                        const uint64_t r2 = f2(fr, fr), nm2 = f2(fnm, fnm);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float4 q = __ldg(c1 + i), bb = __ldg(bp + i);
                            const uint64_t u0 = fma2(nm2, f2(q.x, q.y), f2(bb.x, bb.y));
                            const uint64_t u1 = fma2(nm2, f2(q.z, q.w), f2(bb.z, bb.w));
                            f2split(fma2(r2, f2(x[4 * i], x[4 * i + 1]), u0), x[4 * i], x[4 * i + 1]);
                            f2split(fma2(r2, f2(x[4 * i + 2], x[4 * i + 3]), u1), x[4 * i + 2], x[4 * i + 3]);
                        }
                    } else if (args.bias) {
                        const float4* bp = reinterpret_cast<const float4*>(args.bias + col);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float4 q = __ldg(bp + i);
                            f2split(add2(f2(x[4 * i], x[4 * i + 1]), f2(q.x, q.y)), x[4 * i], x[4 * i + 1]);
                            f2split(add2(f2(x[4 * i + 2], x[4 * i + 3]), f2(q.z, q.w)), x[4 * i + 2], x[4 * i + 3]);
                        }
                    }
                };
                const int dh = args.rope_dh, hd = dh / 2;
                // A head as wide as the tile (Gemma's 256) spans both
                // half-warps' columns: each half-warp then reads the whole
                // head (its RMS) and rotates half of its pairs, d in
                // [half hd/2, (half + 1) hd/2) with d + hd.
                const bool wide = dh > HALF;
                const uint32_t thead = wide ? taddr - half * HALF : taddr;
                const int colw = wide ? n_blk * BN : n_blk * BN + half * HALF;
                const int c_lo = wide ? half * (hd / 2) : 0, c_hi = wide ? c_lo + hd / 2 : hd;
                const int pos = (args.positions && row < args.M) ? __ldg(args.positions + row) : 0;
                // four 2 KB 16-bit boxes in the warp's staging area: column
                // pairs alternate between boxes {0, 1} and {2, 3} (k counts
                // this warp's pairs across tiles), so one pair's stores read
                // shared memory while the next is computed
                float amax = 0.f;
#pragma unroll 1
                for (int h0 = 0; h0 < (wide ? 1 : HALF); h0 += dh) {
                    const int gcol = colw + h0;  // first column of the head
                    const bool rot = gcol < args.rope_qd + args.rope_kvd;  // Q and K heads rotate
                    const float* g = !rot ? nullptr : (gcol < args.rope_qd ? args.q_norm : args.k_norm);
                    // the row's table entries: entry group g (dims 4g .. 4g + 3)
                    // of position pos at float4 g * npos + pos, so the
                    // warp's lanes (mostly consecutive positions) read one
                    // contiguous run; each 16-column step's are requested one
                    // step ahead
                    const int64_t npos = args.rope_npos;
                    const float4* cs = reinterpret_cast<const float4*>(args.rope_cos) + pos;
                    const float4* sn = reinterpret_cast<const float4*>(args.rope_sin) + pos;
                    float4 nc[4], ns[4];
                    if (rot) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            nc[i] = __ldg(cs + (c_lo / 4 + i) * npos);
                            ns[i] = __ldg(sn + (c_lo / 4 + i) * npos);
                        }
                    }
                    // QK-norm: the head's RMS over its dh values, read from
                    // TMEM in a first pass (the table entries above are
                    // already on their way)
                    float inv = 1.0f;
                    if (g) {
                        float ssq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
                        for (int c = 0; c < dh; c += 32) {
                            uint32_t ra[16], rb[16];
                            tmem_ld16(thead + h0 + c, ra);
                            tmem_ld16(thead + h0 + c + 16, rb);
                            tmem_ld_wait();
                            float xa[16], xb[16];
                            values16(ra, gcol + c, xa);
                            values16(rb, gcol + c + 16, xb);
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                ssq[i & 1] = fmaf(xa[i], xa[i], ssq[i & 1]);
                                ssq[2 + (i & 1)] = fmaf(xb[i], xb[i], ssq[2 + (i & 1)]);
                            }
                        }
                        inv = 1.0f / sqrtf(((ssq[0] + ssq[1]) + (ssq[2] + ssq[3])) / static_cast<float>(dh) +
                                           args.rope_eps);
                    }
                    // columns d (first half) and d + dh/2 (second half) of the
                    // head together, 32 at a time into a pair of staging boxes
#pragma unroll 1
                    for (int c = c_lo; c < c_hi; c += 32, ++k) {
                        uint8_t* box0 = boxes + (k & 1) * 2 * kY16Bytes;
                        uint8_t* box1 = box0 + kY16Bytes;
                        if (lane == 0) bulk_wait_read<1>();  // the pair two back has read these boxes
                        __syncwarp();
#pragma unroll 1
                        for (int sub = 0; sub < 32; sub += 16) {
                            const int d0 = c + sub;
                            uint32_t ra[16], rb[16];
                            tmem_ld16(thead + h0 + d0, ra);
                            tmem_ld16(thead + h0 + hd + d0, rb);
                            tmem_ld_wait();
                            float x1[16], x2[16];
                            values16(ra, gcol + d0, x1);
                            values16(rb, gcol + hd + d0, x2);
                            if (g) {  // x * rstd * gain (qwen3.go:485-508)
#pragma unroll
                                for (int i = 0; i < 16; i += 4) {
                                    const float4 ga = __ldg(reinterpret_cast<const float4*>(g + d0 + i));
                                    const float4 gb = __ldg(reinterpret_cast<const float4*>(g + hd + d0 + i));
                                    const float gaa[4] = {ga.x, ga.y, ga.z, ga.w}, gbb[4] = {gb.x, gb.y, gb.z, gb.w};
#pragma unroll
                                    for (int e = 0; e < 4; ++e) {
                                        x1[i + e] = x1[i + e] * inv * gaa[e];
                                        x2[i + e] = x2[i + e] * inv * gbb[e];
                                    }
                                }
                            }
                            if (rot) {
                                float4 c4v[4], s4v[4];
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    c4v[i] = nc[i];
                                    s4v[i] = ns[i];
                                }
                                if (d0 + 16 < c_hi) {  // the next step's entries
#pragma unroll
                                    for (int i = 0; i < 4; ++i) {
                                        nc[i] = __ldg(cs + ((d0 + 16) / 4 + i) * npos);
                                        ns[i] = __ldg(sn + ((d0 + 16) / 4 + i) * npos);
                                    }
                                }
#pragma unroll
                                for (int i = 0; i < 16; i += 4) {
                                    const float4 c4 = c4v[i / 4], s4 = s4v[i / 4];
                                    const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                                    for (int e = 0; e < 4; ++e) {
                                        const float a = x1[i + e], b = x2[i + e];
                                        x1[i + e] = __fsub_rn(__fmul_rn(a, cc[e]), __fmul_rn(b, ss[e]));
                                        x2[i + e] = __fadd_rn(__fmul_rn(b, cc[e]), __fmul_rn(a, ss[e]));
                                    }
                                }
                            }
                            if constexpr (F16) {
#pragma unroll
                                for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fmaxf(fabsf(x1[i]), fabsf(x2[i])));
                            }
#pragma unroll
                            for (int q = 0; q < 2; ++q) {
                                const int ci = sub / 8 + q;  // 16-byte chunk of the 64-byte box row
                                *reinterpret_cast<uint4*>(box0 + swz(lane, ci, 64)) =
                                    make_uint4(pack2<F16>(x1[8 * q], x1[8 * q + 1]), pack2<F16>(x1[8 * q + 2], x1[8 * q + 3]),
                                               pack2<F16>(x1[8 * q + 4], x1[8 * q + 5]),
                                               pack2<F16>(x1[8 * q + 6], x1[8 * q + 7]));
                                *reinterpret_cast<uint4*>(box1 + swz(lane, ci, 64)) =
                                    make_uint4(pack2<F16>(x2[8 * q], x2[8 * q + 1]), pack2<F16>(x2[8 * q + 2], x2[8 * q + 3]),
                                               pack2<F16>(x2[8 * q + 4], x2[8 * q + 5]),
                                               pack2<F16>(x2[8 * q + 6], x2[8 * q + 7]));
                            }
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tmOut, box0, gcol + c, row0);
                            tma_store_2d(&tmOut, box1, gcol + hd + c, row0);
                            bulk_commit();
                        }
                    }
                }
                // fp16 outputs fail loudly instead of turning into inf
                if (F16 && __any_sync(0xffffffffu, !(amax <= 65504.0f)) && lane == 0)
                    atomicOr(args.status, kStatusF16Overflow);
            }
#pragma unroll 1
            for (int c = 0; c < (EPI == kEpiRope ? 0 : CHUNKS); c += STEP, ++k) {
                const int b = k & 1;
                uint8_t* box = boxes + b * kStageBytes;
                const int col0 = n_blk * BN + half * HALF + c * kChunk;  // accumulator column
                const int ocol0 = GLU ? col0 / 2 : col0;                  // output column
                if (lane == 0) {
                    if constexpr (RES) {
                        // The other buffer's store (previous chunk) has read
                        // its box: it can take the next chunk's residual.
                        bulk_wait_read<0>();
                        if (c + STEP < CHUNKS)
                            load_residual(tile, c + STEP, b ^ 1);
                        else
                            load_residual(tile + npairs, 0, b ^ 1);
                    } else {
                        // This buffer's store (two chunks back) has read its box.
                        bulk_wait_read<1>();
                    }
                }
                __syncwarp();
                uint32_t r[32];
                tmem_ld32(taddr + c * kChunk, r);
                tmem_ld_wait();
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if constexpr (S8)
                        v[i] = static_cast<float>(static_cast<int32_t>(r[i])) * rs;
                    else
                        v[i] = __uint_as_float(r[i]);
                }
                if constexpr (GLU) {
                    // a = chunk c (activated), b = chunk c + 1 (linear)
                    uint32_t rb[32];
                    tmem_ld32(taddr + (c + 1) * kChunk, rb);
                    tmem_ld_wait();
                    float w[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        if constexpr (S8)
                            w[i] = static_cast<float>(static_cast<int32_t>(rb[i])) * rs;
                        else
                            w[i] = __uint_as_float(rb[i]);
                    }
                    if (args.fold_stats) {  // folded norm: rstd * acc - rstd * mean * c1 (bias-free)
                        const float4* c1a = reinterpret_cast<const float4*>(args.fold_c1 + col0);
                        const float4* c1b = reinterpret_cast<const float4*>(args.fold_c1 + col0 + kChunk);
                        const uint64_t r2 = f2(fr, fr), nm2 = f2(fnm, fnm);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 qa = __ldg(c1a + i), qb = __ldg(c1b + i);
                            f2split(fma2(r2, f2(v[4 * i], v[4 * i + 1]), mul2(nm2, f2(qa.x, qa.y))), v[4 * i],
                                    v[4 * i + 1]);
                            f2split(fma2(r2, f2(v[4 * i + 2], v[4 * i + 3]), mul2(nm2, f2(qa.z, qa.w))), v[4 * i + 2],
                                    v[4 * i + 3]);
                            f2split(fma2(r2, f2(w[4 * i], w[4 * i + 1]), mul2(nm2, f2(qb.x, qb.y))), w[4 * i],
                                    w[4 * i + 1]);
                            f2split(fma2(r2, f2(w[4 * i + 2], w[4 * i + 3]), mul2(nm2, f2(qb.z, qb.w))), w[4 * i + 2],
                                    w[4 * i + 3]);
                        }
                    }
                    if (CSCALE && args.col_scale) {
                        const float4* ca = reinterpret_cast<const float4*>(args.col_scale + col0);
                        const float4* cb = reinterpret_cast<const float4*>(args.col_scale + col0 + kChunk);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 qa = __ldg(ca + i), qb = __ldg(cb + i);
                            v[4 * i] *= qa.x;
                            v[4 * i + 1] *= qa.y;
                            v[4 * i + 2] *= qa.z;
                            v[4 * i + 3] *= qa.w;
                            w[4 * i] *= qb.x;
                            w[4 * i + 1] *= qb.y;
                            w[4 * i + 2] *= qb.z;
                            w[4 * i + 3] *= qb.w;
                        }
                    }
                    if constexpr (EPI == kEpiGluGeluErf) {
#pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            gelu_as28x2(v[i], v[i + 1]);
                            f2split(mul2(f2(v[i], v[i + 1]), f2(w[i], w[i + 1])), v[i], v[i + 1]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            if constexpr (EPI == kEpiGluSilu) silu_x2(v[i], v[i + 1]);
                            else gelu_tanh_x2(v[i], v[i + 1]);
                            f2split(mul2(f2(v[i], v[i + 1]), f2(w[i], w[i + 1])), v[i], v[i + 1]);
                        }
                    }
                }
                // (acc * row scale) * column scale + bias: the reference's
                // dequant-then-AddBias order (pack_vnni.go:155-173, bert.go:297-300)
                if (!GLU && CSCALE && args.col_scale) {
                    const float4* cs = reinterpret_cast<const float4*>(args.col_scale + col0);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 q = __ldg(cs + i);
                        v[4 * i] *= q.x;
                        v[4 * i + 1] *= q.y;
                        v[4 * i + 2] *= q.z;
                        v[4 * i + 3] *= q.w;
                    }
                }
                bool folded = false;
                if constexpr (EPI == kEpiBias || EPI == kEpiBiasGelu) {
                    if (args.fold_stats) {  // rstd * acc + (bias - rstd * mean * c1)
                        folded = true;
                        const float4* c1 = reinterpret_cast<const float4*>(args.fold_c1 + col0);
                        const float4* bp = reinterpret_cast<const float4*>(args.bias + col0);
                        const uint64_t r2 = f2(fr, fr), nm2 = f2(fnm, fnm);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 q = __ldg(c1 + i), bb = __ldg(bp + i);
                            const uint64_t u0 = fma2(nm2, f2(q.x, q.y), f2(bb.x, bb.y));
                            const uint64_t u1 = fma2(nm2, f2(q.z, q.w), f2(bb.z, bb.w));
                            f2split(fma2(r2, f2(v[4 * i], v[4 * i + 1]), u0), v[4 * i], v[4 * i + 1]);
                            f2split(fma2(r2, f2(v[4 * i + 2], v[4 * i + 3]), u1), v[4 * i + 2], v[4 * i + 3]);
                        }
                    }
                }
                if (!GLU && !folded && args.bias) {
                    const float4* bp = reinterpret_cast<const float4*>(args.bias + col0);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 q = __ldg(bp + i);
                        f2split(add2(f2(v[4 * i], v[4 * i + 1]), f2(q.x, q.y)), v[4 * i], v[4 * i + 1]);
                        f2split(add2(f2(v[4 * i + 2], v[4 * i + 3]), f2(q.z, q.w)), v[4 * i + 2], v[4 * i + 3]);
                    }
                }
                if constexpr (EPI == kEpiBiasGelu) {
#pragma unroll
                    for (int i = 0; i < 32; i += 2) gelu_as28x2(v[i], v[i + 1]);
                }
                if constexpr (RES) {
                    if (!mbar_wait(&rbar[b], (rphase >> b) & 1, args.status, abort_flag, wlim)) {
                        ok = false;
                        break;
                    }
                    rphase ^= 1u << b;
                    rpending &= ~(1u << b);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        float4 x = *reinterpret_cast<const float4*>(box + swz(lane, i, 128));
                        if constexpr (EPI == kEpiBiasResLN) {
                            // the LayerNorm kernel's own arithmetic: (x - mean) * rstd * g + b
                            const float4 g = __ldg(reinterpret_cast<const float4*>(args.ln_g + col0) + i);
                            const float4 bb = __ldg(reinterpret_cast<const float4*>(args.ln_b + col0) + i);
                            x.x = (x.x - lnst.x) * lnst.y * g.x + bb.x;
                            x.y = (x.y - lnst.x) * lnst.y * g.y + bb.y;
                            x.z = (x.z - lnst.x) * lnst.y * g.z + bb.z;
                            x.w = (x.w - lnst.x) * lnst.y * g.w + bb.w;
                        }
                        f2split(add2(f2(x.x, x.y), f2(v[4 * i], v[4 * i + 1])), v[4 * i], v[4 * i + 1]);
                        f2split(add2(f2(x.z, x.w), f2(v[4 * i + 2], v[4 * i + 3])), v[4 * i + 2], v[4 * i + 3]);
                    }
                    if (args.parts_out && row < args.M) {  // this chunk's (mean, M2)
                        float cs = 0.f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) cs += v[i];
                        const float cm = cs * (1.0f / 32.0f);
                        float c2 = 0.f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) c2 = fmaf(v[i] - cm, v[i] - cm, c2);
                        args.parts_out[static_cast<int64_t>(col0 / kChunk) * args.M + row] = make_float2(cm, c2);
                    }
                    if constexpr (S::Y16) {
                        // the 16-bit copy, staged for its own TMA store (the
                        // box is free: every earlier store has read its box);
                        // an fp16 copy fails loudly instead of turning into inf
                        if (args.out16) {
                            float y[32];
#pragma unroll
                            for (int i = 0; i < 32; ++i) y[i] = v[i];
                            if (args.copy_gain) {
                                const float4* gp = reinterpret_cast<const float4*>(args.copy_gain + col0);
#pragma unroll
                                for (int i = 0; i < 8; ++i) {
                                    const float4 q = __ldg(gp + i);
                                    f2split(mul2(f2(y[4 * i], y[4 * i + 1]), f2(q.x, q.y)), y[4 * i], y[4 * i + 1]);
                                    f2split(mul2(f2(y[4 * i + 2], y[4 * i + 3]), f2(q.z, q.w)), y[4 * i + 2],
                                            y[4 * i + 3]);
                                }
                            }
                            if constexpr (F16) {
                                float amax = 0.f;
#pragma unroll
                                for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(y[i]));
                                if (__any_sync(0xffffffffu, amax > 65504.0f) && lane == 0)
                                    atomicOr(args.status, kStatusF16Overflow);
                            }
                            uint8_t* y16 = y16_base + ew * kY16Bytes;
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                *reinterpret_cast<uint4*>(y16 + swz(lane, i, 64)) = make_uint4(
                                    pack2<F16>(y[8 * i], y[8 * i + 1]), pack2<F16>(y[8 * i + 2], y[8 * i + 3]),
                                    pack2<F16>(y[8 * i + 4], y[8 * i + 5]), pack2<F16>(y[8 * i + 6], y[8 * i + 7]));
                        }
                    }
                }
                if constexpr (F32OUT) {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *reinterpret_cast<float4*>(box + swz(lane, i, 128)) =
                            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                } else {
                    if constexpr (F16) {
                        // fp16 outputs fail loudly instead of turning into inf
                        // (fp32 accumulators cannot overflow to NaN here)
                        float amax = 0.f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
                        if (__any_sync(0xffffffffu, amax > 65504.0f) && lane == 0)
                            atomicOr(args.status, kStatusF16Overflow);
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t w[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) w[j] = pack2<F16>(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
                        *reinterpret_cast<uint4*>(box + swz(lane, i, 64)) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmOut, box, ocol0, row0);
                    if constexpr (S::Y16) {
                        if (args.out16) tma_store_2d(&tmOut16, y16_base + ew * kY16Bytes, col0, row0);
                    }
                    bulk_commit();
                }
            }
            if (!ok) break;
            // This warp is done with the accumulator: tell the even CTA.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_lead + 8 * acc);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        // Every store has read its staging box, and every residual box
        // requested has landed, before the CTA may exit.
        if (lane == 0) {
            bulk_wait_read<0>();
            for (int b = 0; b < 2; ++b)
                if (rpending & (1u << b)) mbar_drain(&rbar[b], (rphase >> b) & 1, wlim);
        }
        __syncwarp();
    }

    // Teardown: every MMA has completed (the issuer drained them) and every
    // TMEM read of both CTAs is done before the pair frees its TMEM.
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Launch: one instantiation per (tile width, operand kind, epilogue); each
// kind is compiled in its own translation unit (gemm_kind_*.cu).

template <int BN, int KIND, int EPI>
static cudaError_t launch_one(const GemmMaps& m, const GemmArgs& args, int num_sms, cudaStream_t stream) {
    constexpr int smem = GemmShape<BN, KIND, EPI>::SMEM;
    static_assert(smem <= 232448, "shared memory budget");
    auto kern = gemm_kernel<BN, KIND, EPI>;
    // The shared-memory opt-in is a per-device function attribute.
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 32) __atomic_fetch_or(&configured, 1u << dev, __ATOMIC_RELEASE);
    }
    // One CTA pair per tile slot: as many pairs as can be co-resident.
    static int max_pairs[32] = {};
    int pairs = dev < 32 ? __atomic_load_n(&max_pairs[dev], __ATOMIC_ACQUIRE) : 0;
    if (pairs == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = num_sms / 2;
        }
        pairs = n;
        if (dev < 32) __atomic_store_n(&max_pairs[dev], pairs, __ATOMIC_RELEASE);
    }
    const int tiles = ((args.M + 255) / 256) * (args.N / BN);
    const int grid = 2 * (tiles < pairs ? tiles : pairs);
    launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, m.a, m.b, m.out, m.res, m.a2, m.b2, m.out16, args);
    return cudaGetLastError();
}

template <int BN, int KIND>
static cudaError_t dispatch_epi(int epi, const GemmMaps& m, const GemmArgs& args, int num_sms, cudaStream_t stream) {
    switch (epi) {
    case kEpiBias: return launch_one<BN, KIND, kEpiBias>(m, args, num_sms, stream);
    case kEpiBiasGelu: return launch_one<BN, KIND, kEpiBiasGelu>(m, args, num_sms, stream);
    case kEpiBiasRes: return launch_one<BN, KIND, kEpiBiasRes>(m, args, num_sms, stream);
    case kEpiBiasF32: return launch_one<BN, KIND, kEpiBiasF32>(m, args, num_sms, stream);
    case kEpiGluSilu: return launch_one<BN, KIND, kEpiGluSilu>(m, args, num_sms, stream);
    case kEpiGluGeluErf: return launch_one<BN, KIND, kEpiGluGeluErf>(m, args, num_sms, stream);
    case kEpiGluGeluTanh: return launch_one<BN, KIND, kEpiGluGeluTanh>(m, args, num_sms, stream);
    case kEpiBiasResLN: return launch_one<BN, KIND, kEpiBiasResLN>(m, args, num_sms, stream);
    case kEpiRope:
        if constexpr (KIND == static_cast<int>(GemmKind::kTF32x3)) return cudaErrorInvalidValue;
        else return launch_one<BN, KIND, kEpiRope>(m, args, num_sms, stream);
    default: return cudaErrorInvalidValue;
    }
}

template <int KIND>
cudaError_t dispatch_kind(int block_n, int epi, const GemmMaps& m, const GemmArgs& args, int num_sms,
                          cudaStream_t stream) {
    switch (block_n) {
    case 256: return dispatch_epi<256, KIND>(epi, m, args, num_sms, stream);
    case 192: return dispatch_epi<192, KIND>(epi, m, args, num_sms, stream);
    case 128: return dispatch_epi<128, KIND>(epi, m, args, num_sms, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace rg
