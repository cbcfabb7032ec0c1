/*
 * oracle_prims.c - CPU restatement of rembed's internal/tensor kernels.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and CPU baseline; never part of
 * the product path).  Each function cites the reference routine it
 * restates.  Compiled with -ffp-contract=off so every float32 operation
 * rounds the way the reference's Go code (GOAMD64=v1) does; the fused
 * multiply-adds of the reference's assembly micro-kernels are written as
 * explicit fmaf() calls in the same order.
 */
#include "oracle.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define OR_HAVE_AVX2 1
#endif

/* fastmath.go:17-21 */
#define EXP_LOG2E 1.44269504088896341f
#define EXP_C1 0.693359375f
#define EXP_C2 -2.12194440e-4f

static inline float f32_from_bits(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Cephes polynomial core shared by expf32 / expNonPos: fastmath.go:38-45. */
static inline float exp_poly(float x) {
    float z = x * x;
    float y = 1.9875691500e-4f;
    y = y * x + 1.3981999507e-3f;
    y = y * x + 8.3334519073e-3f;
    y = y * x + 4.1665795894e-2f;
    y = y * x + 1.6666665459e-1f;
    y = y * x + 5.0000001201e-1f;
    return y * z + x + 1.0f;
}

/* expf32, fastmath.go:26-55 */
float or_expf32(float x) {
    if (x > 88.72f) return INFINITY;
    if (x < -87.33f) return 0.0f;
    float s = x < 0 ? -0.5f : 0.5f; /* sign05, fastmath.go:62-67 */
    float nf = (float)(int32_t)(x * EXP_LOG2E + s);
    x -= nf * EXP_C1;
    x -= nf * EXP_C2;
    float y = exp_poly(x);
    int32_t n = (int32_t)nf;
    if (n >= 128) return y * f32_from_bits((uint32_t)(127 + 127) << 23) * 2.0f;
    return y * f32_from_bits((uint32_t)(n + 127) << 23);
}

/* expNonPos, fastmath.go:93-109 */
float or_expnonpos(float x) {
    if (x < -87.33f) x = -87.33f;
    float nf = (float)(int32_t)(x * EXP_LOG2E - 0.5f);
    x -= nf * EXP_C1;
    x -= nf * EXP_C2;
    float y = exp_poly(x);
    return y * f32_from_bits((uint32_t)((int32_t)nf + 127) << 23);
}

/* A&S 7.1.26 polynomial, fastmath.go:76-77 / tensor.go:517-518 */
static inline float as_poly(float t) {
    return t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
}

/* erff32, fastmath.go:71-83 */
float or_erff32(float x) {
    int neg = x < 0;
    if (neg) x = -x;
    float t = 1.0f / (1.0f + 0.3275911f * x);
    float r = 1.0f - as_poly(t) * or_expf32(-x * x);
    return neg ? -r : r;
}

/* Softmax, tensor.go:391-428 (the exp is expNonPos written flat). */
void or_softmax(float *x, int m, int n) {
    for (int i = 0; i < m; i++) {
        float *row = x + (int64_t)i * n;
        float maxv = row[0];
        for (int j = 1; j < n; j++)
            if (row[j] > maxv) maxv = row[j];
        float sum = 0.0f;
        for (int j = 0; j < n; j++) {
            float e = or_expnonpos(row[j] - maxv);
            row[j] = e;
            sum += e;
        }
        float inv = 1.0f / sum;
        for (int j = 0; j < n; j++) row[j] *= inv;
    }
}

/* LayerNorm, tensor.go:433-452: two-pass float32 mean / biased variance,
 * inverse standard deviation through a float64 sqrt. */
void or_layernorm(float *x, const float *g, const float *b, int m, int n, float eps) {
    for (int i = 0; i < m; i++) {
        float *row = x + (int64_t)i * n;
        float mean = 0.0f;
        for (int j = 0; j < n; j++) mean += row[j];
        mean /= (float)n;
        float var = 0.0f;
        for (int j = 0; j < n; j++) {
            float d = row[j] - mean;
            var += d * d;
        }
        var /= (float)n;
        float inv = 1.0f / (float)sqrt((double)(var + eps));
        for (int j = 0; j < n; j++) row[j] = (row[j] - mean) * inv * g[j] + b[j];
    }
}

/* RMSNorm, tensor.go:459-471 */
void or_rmsnorm(float *x, const float *g, int m, int n, float eps) {
    for (int i = 0; i < m; i++) {
        float *row = x + (int64_t)i * n;
        float ss = 0.0f;
        for (int j = 0; j < n; j++) ss += row[j] * row[j];
        float inv = 1.0f / (float)sqrt((double)(ss / (float)n + eps));
        for (int j = 0; j < n; j++) row[j] = row[j] * inv * g[j];
    }
}

/* SiLU, tensor.go:477-481 (float64 exp) */
void or_silu(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] = x[i] / (float)(1.0 + exp(-(double)x[i]));
}

/* GELUTanh, tensor.go:490-497 (float64 tanh) */
void or_gelu_tanh(float *x, int n) {
    const double c = 0.7978845608028654;
    for (int i = 0; i < n; i++) {
        double v = (double)x[i];
        double inner = c * (v + 0.044715 * v * v * v);
        x[i] = (float)(0.5 * v * (1.0 + tanh(inner)));
    }
}

/* geluScalar, tensor.go:508-538: erf by A&S 7.1.26 with the flat Cephes
 * exp.  (On AVX2 hosts the reference runs geluAVX2 on 8-aligned spans,
 * gelu_amd64.s:37, which its own test pins to within 1e-6 of this.) */
void or_gelu(float *x, int n) {
    const float inv_sqrt2 = 0.7071067811865476f;
    for (int i = 0; i < n; i++) {
        float v = x[i];
        float a = v * inv_sqrt2;
        float sign = 1.0f;
        if (a < 0) {
            sign = -1.0f;
            a = -a;
        }
        float t = 1.0f / (1.0f + 0.3275911f * a);
        float poly = as_poly(t);
        float e = or_expnonpos(-a * a);
        float erf = sign * (1.0f - poly * e);
        x[i] = 0.5f * v * (1.0f + erf);
    }
}

/* L2Normalize, tensor.go:542-554 (float64 sum of squares) */
void or_l2normalize(float *x, int n) {
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += (double)x[i] * (double)x[i];
    if (sum == 0.0) return;
    float inv = (float)(1.0 / sqrt(sum));
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* AddBias, tensor.go:373-380 */
void or_add_bias(float *x, const float *bias, int m, int n) {
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) x[(int64_t)i * n + j] += bias[j];
}

/* Add, tensor.go:383-387 */
void or_add(float *dst, const float *src, int n) {
    for (int i = 0; i < n; i++) dst[i] += src[i];
}

/* relPosBucket, bert.go:126-150 (relMaxDistance = 128) */
int or_relpos_bucket(int rel, int num_buckets) {
    int n = -rel;
    int half = num_buckets / 2;
    int ret = 0;
    if (n < 0) {
        ret = half;
        n = -n;
    }
    int max_exact = half / 2;
    if (n < max_exact) return ret + n;
    int v = max_exact + (int)(log((double)n / (double)max_exact) / log(128.0 / (double)max_exact) *
                              (double)(half - max_exact));
    return ret + (v < half - 1 ? v : half - 1);
}

/* ---- dense GEMMs ----------------------------------------------------- */

/* Per output element: acc = fma(a[p], b[p], acc) for p = 0..k-1 from zero,
 * the order every packed micro-kernel uses (gemm_amd64.s:14-75,
 * gemm512_amd64.s:22).  16 columns at a time over a transposed B panel so
 * the compiler/AVX2 path vectorises across columns without reordering k. */
void or_matmul_packed(float *dst, const float *a, const float *bT, int m, int k, int n) {
    float *panel = (float *)malloc(sizeof(float) * 16 * (size_t)k);
    for (int j0 = 0; j0 < n; j0 += 16) {
        int nc = n - j0 < 16 ? n - j0 : 16;
        for (int p = 0; p < k; p++)
            for (int c = 0; c < 16; c++) panel[p * 16 + c] = c < nc ? bT[(int64_t)(j0 + c) * k + p] : 0.0f;
        for (int i0 = 0; i0 < m; i0 += 4) {
            int nr = m - i0 < 4 ? m - i0 : 4;
            float acc[4][16];
            memset(acc, 0, sizeof(acc));
#ifdef OR_HAVE_AVX2
            __m256 v[4][2];
            for (int r = 0; r < 4; r++) v[r][0] = v[r][1] = _mm256_setzero_ps();
            if (nr == 4) {
                const float *a0 = a + (int64_t)i0 * k;
                for (int p = 0; p < k; p++) {
                    __m256 b0 = _mm256_loadu_ps(panel + p * 16);
                    __m256 b1 = _mm256_loadu_ps(panel + p * 16 + 8);
                    for (int r = 0; r < 4; r++) {
                        __m256 av = _mm256_set1_ps(a0[(int64_t)r * k + p]);
                        v[r][0] = _mm256_fmadd_ps(av, b0, v[r][0]);
                        v[r][1] = _mm256_fmadd_ps(av, b1, v[r][1]);
                    }
                }
            } else {
                for (int p = 0; p < k; p++) {
                    __m256 b0 = _mm256_loadu_ps(panel + p * 16);
                    __m256 b1 = _mm256_loadu_ps(panel + p * 16 + 8);
                    for (int r = 0; r < nr; r++) {
                        __m256 av = _mm256_set1_ps(a[(int64_t)(i0 + r) * k + p]);
                        v[r][0] = _mm256_fmadd_ps(av, b0, v[r][0]);
                        v[r][1] = _mm256_fmadd_ps(av, b1, v[r][1]);
                    }
                }
            }
            for (int r = 0; r < 4; r++) {
                _mm256_storeu_ps(acc[r], v[r][0]);
                _mm256_storeu_ps(acc[r] + 8, v[r][1]);
            }
#else
            for (int r = 0; r < nr; r++) {
                const float *ar = a + (int64_t)(i0 + r) * k;
                for (int p = 0; p < k; p++)
                    for (int c = 0; c < 16; c++) acc[r][c] = fmaf(ar[p], panel[p * 16 + c], acc[r][c]);
            }
#endif
            for (int r = 0; r < nr; r++)
                for (int c = 0; c < nc; c++) dst[(int64_t)(i0 + r) * n + j0 + c] = acc[r][c];
        }
    }
    free(panel);
}

/* dot4 for one (a, b) pair: dot_amd64.s:13-80.  Eight lane accumulators
 * take k = l (mod 8) by FMA; lanes 4..7 fold into 0..3; the k%8 tail
 * accumulates into lane 0; two horizontal adds give (l0+l1)+(l2+l3). */
static inline float dot4_one(const float *a, const float *b, int k) {
    float l[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k8 = k & ~7;
    for (int p = 0; p < k8; p += 8)
        for (int i = 0; i < 8; i++) l[i] = fmaf(a[p + i], b[p + i], l[i]);
    float f0 = l[0] + l[4], f1 = l[1] + l[5], f2 = l[2] + l[6], f3 = l[3] + l[7];
    for (int p = k8; p < k; p++) f0 = fmaf(a[p], b[p], f0);
    return (f0 + f1) + (f2 + f3);
}

/* MatMulSerial -> matMulSIMDCols, tensor.go:284-330: dot4 for whole
 * groups of 4 columns, a plain sequential float32 sum for the n%4
 * remainder columns. */
void or_matmul_serial(float *dst, const float *a, const float *bT, int m, int k, int n) {
    int n4 = n & ~3;
    for (int i = 0; i < m; i++) {
        const float *ar = a + (int64_t)i * k;
        for (int j = 0; j < n4; j++) dst[(int64_t)i * n + j] = dot4_one(ar, bT + (int64_t)j * k, k);
        for (int j = n4; j < n; j++) {
            const float *br = bT + (int64_t)j * k;
            float s = 0.0f;
            for (int p = 0; p < k; p++) s += ar[p] * br[p];
            dst[(int64_t)i * n + j] = s;
        }
    }
}

static int finite_f32(float v) { return !(v != v || v > 3.40282346638528859811704183484516925440e+38f || v < -3.40282346638528859811704183484516925440e+38f); }

/* PackB8, pack8.go:25-76.  The scale is a float32 division; each weight is
 * divided in float64 and rounded half-to-even, clamped to +-127. */
int or_packb8(const float *bT, int k, int n, int8_t *q, float *scales) {
    if (n < 16 || n % 16 != 0 || k < 1) return -1;
    for (int j = 0; j < n; j++) {
        const float *row = bT + (int64_t)j * k;
        float maxabs = 0.0f;
        for (int p = 0; p < k; p++) {
            if (!finite_f32(row[p])) return -1;
            float a = fabsf(row[p]);
            if (a > maxabs) maxabs = a;
        }
        float scale = maxabs / 127.0f;
        if (scale == 0.0f) scale = 1.0f;
        scales[j] = scale;
        for (int p = 0; p < k; p++) {
            double qq = rint((double)row[p] / (double)scale);
            if (qq > 127) qq = 127;
            if (qq < -127) qq = -127;
            q[(int64_t)j * k + p] = (int8_t)qq;
        }
    }
    return 0;
}

/* MatMulPacked8 / gemm4x16i8, gemm8_amd64.s:14-70: k-ordered FMA of the
 * float32 activation with the int8 weight converted to float32, then one
 * multiply by the channel scale. */
void or_matmul_packed8(float *dst, const float *a, const int8_t *q, const float *scales,
                       int m, int k, int n) {
    float *panel = (float *)malloc(sizeof(float) * 16 * (size_t)k);
    for (int j0 = 0; j0 < n; j0 += 16) {
        int nc = n - j0 < 16 ? n - j0 : 16;
        for (int p = 0; p < k; p++)
            for (int c = 0; c < 16; c++) panel[p * 16 + c] = c < nc ? (float)q[(int64_t)(j0 + c) * k + p] : 0.0f;
        for (int i0 = 0; i0 < m; i0 += 4) {
            int nr = m - i0 < 4 ? m - i0 : 4;
            float acc[4][16];
            memset(acc, 0, sizeof(acc));
#ifdef OR_HAVE_AVX2
            __m256 v[4][2];
            for (int r = 0; r < 4; r++) v[r][0] = v[r][1] = _mm256_setzero_ps();
            for (int p = 0; p < k; p++) {
                __m256 b0 = _mm256_loadu_ps(panel + p * 16);
                __m256 b1 = _mm256_loadu_ps(panel + p * 16 + 8);
                for (int r = 0; r < nr; r++) {
                    __m256 av = _mm256_set1_ps(a[(int64_t)(i0 + r) * k + p]);
                    v[r][0] = _mm256_fmadd_ps(av, b0, v[r][0]);
                    v[r][1] = _mm256_fmadd_ps(av, b1, v[r][1]);
                }
            }
            for (int r = 0; r < 4; r++) {
                _mm256_storeu_ps(acc[r], v[r][0]);
                _mm256_storeu_ps(acc[r] + 8, v[r][1]);
            }
#else
            for (int r = 0; r < nr; r++) {
                const float *ar = a + (int64_t)(i0 + r) * k;
                for (int p = 0; p < k; p++)
                    for (int c = 0; c < 16; c++) acc[r][c] = fmaf(ar[p], panel[p * 16 + c], acc[r][c]);
            }
#endif
            for (int r = 0; r < nr; r++)
                for (int c = 0; c < nc; c++) dst[(int64_t)(i0 + r) * n + j0 + c] = acc[r][c] * scales[j0 + c];
        }
    }
    free(panel);
}

/* PackB8VNNI, pack_vnni.go:28-77.  Float64 scale; q = int8(RoundToEven(w /
 * scale)) without a clamp (|w|/scale <= 127 by construction); the stored
 * dequant scale is float32(scale); colSum = sum of q. */
int or_packb8vnni(const float *bT, int k, int n, int8_t *q, int32_t *colsum, float *scales) {
    if (n < 16 || n % 16 != 0 || k < 1) return -1;
    for (int c = 0; c < n; c++) {
        double maxabs = 0.0;
        for (int p = 0; p < k; p++) {
            double v = (double)bT[(int64_t)c * k + p];
            if (isnan(v) || isinf(v)) return -1;
            double a = fabs(v);
            if (a > maxabs) maxabs = a;
        }
        double scale = maxabs / 127.0;
        if (scale == 0.0) scale = 1.0;
        scales[c] = (float)scale;
        int32_t sum = 0;
        for (int p = 0; p < k; p++) {
            int8_t qq = (int8_t)(int32_t)rint((double)bT[(int64_t)c * k + p] / scale);
            sum += qq;
            q[(int64_t)c * k + p] = qq;
        }
        colsum[c] = sum;
    }
    return 0;
}

/* QuantizeRowU8, pack_vnni.go:85-117: float32 scale and reciprocal,
 * q = RoundToEven(float32(a*inv)) + 128 clamped to [0,255]. */
float or_quantize_row_u8(uint8_t *dst, const float *a, int k, int kpad) {
    float maxabs = 0.0f;
    for (int i = 0; i < k; i++) {
        float x = fabsf(a[i]);
        if (x > maxabs) maxabs = x;
    }
    float scale = maxabs / 127.0f;
    if (scale == 0.0f) scale = 1.0f;
    float inv = 1.0f / scale;
    for (int i = 0; i < k; i++) {
        float prod = a[i] * inv;
        int32_t qq = (int32_t)rint((double)prod) + 128;
        if (qq < 0) qq = 0;
        else if (qq > 255) qq = 255;
        dst[i] = (uint8_t)qq;
    }
    for (int i = k; i < kpad; i++) dst[i] = 0;
    return scale;
}

/* MatMulPackedVNNI, pack_vnni.go:124-176: u8 activations (+128 offset)
 * times s8 weights in int32, minus 128*colSum, then
 * float32(acc) * rowScale * colScale. */
void or_matmul_vnni(float *dst, const float *a, const int8_t *q, const int32_t *colsum,
                    const float *scales, int m, int k, int n) {
    uint8_t qa_stack[4096];
    uint8_t *qa = qa_stack;
    if (k > 4096) return; /* every supported width is <= 4096 */
    for (int r = 0; r < m; r++) {
        float rs = or_quantize_row_u8(qa, a + (int64_t)r * k, k, k);
        for (int c = 0; c < n; c++) {
            const int8_t *w = q + (int64_t)c * k;
            int32_t acc = 0;
            for (int p = 0; p < k; p++) acc += (int32_t)qa[p] * (int32_t)w[p];
            int32_t real = (int32_t)((uint32_t)acc - (uint32_t)(128 * colsum[c]));
            dst[(int64_t)r * n + c] = (float)real * rs * scales[c];
        }
    }
}
