// runtime.cu - librembed_gpu.so: the C ABI of include/rembed_gpu.h.
//
// Host side of the B200 forward pass: weight ingest by Hugging Face name
// (bert.go:338-518), Q|K|V fusion (bert.go:479-485), the reference's int8
// quantisers (pack8.go:25-76, pack_vnni.go:28-77), one replica per device,
// input validation (bert.go:742-747, 797-799), sequence sharding across
// devices, and the per-layer launch sequence of encodeWorkers
// (bert.go:839-919) over the packed batch.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "rembed_gpu.h"
#include "gemm.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

using act16 = uint16_t;  // 16-bit activation words: bf16 or fp16 by mode

namespace {

struct Error {
    std::string msg;
};

[[noreturn]] void fail(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    throw Error{buf};
}

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail("%s: %s", what, cudaGetErrorString(e));
}

void set_err(char** err, const std::string& m) {
    if (err) {
        *err = static_cast<char*>(malloc(m.size() + 1));
        if (*err) memcpy(*err, m.c_str(), m.size() + 1);
    }
}

struct HostTensor {
    std::vector<float> data;
    std::vector<int64_t> shape;
};

// One dense projection on a device: weights [N x K] (bf16 or int8),
// optional per-channel dequant scales, bias, and its TMA descriptor.
struct DevDense {
    int N = 0, K = 0;
    void* w = nullptr;
    float* scale = nullptr;
    float* bias = nullptr;
    CUtensorMap tmap[3];    // for tile widths 256, 192, 128 (only widths dividing N are valid)
    CUtensorMap tmap16[3];  // weight-only int8: the same shape over the replica's fp16 widening scratch
    void* w_lo = nullptr;   // strict fp32: the fp32 remainder of the tf32-rounded weight in w
    CUtensorMap tmap_lo[3];
    float* fold_c1 = nullptr;  // folded LayerNorm: column sums of the 16-bit w (w = W * gain)
    // weight-only int8 with a folded LayerNorm: w stays the quantised W, and
    // fold_c1 / fold_bias are s[n] * sum_k g[k] q[n][k] and bias[n] +
    // s[n] * sum_k b[k] q[n][k] (bias stays the unfolded one)
    float* fold_bias = nullptr;
    size_t w16_off = 0;  // weight-only int8: element offset of the widened copy in the layer scratch
};

// A GEMM's A operand: the tensor map of the buffer the MMA reads and, in the
// strict fp32 mode, of the fp32 remainder buffer (3xTF32).
struct OpMaps {
    CUtensorMap m, lo;
};

// Weight-only int8 GEMMs with at least this many rows widen the layer's
// int8 weight to fp16 first (about 3 bytes of traffic per weight, a few
// microseconds) and run the fp16 kernel: at this size the GEMM is
// tensor-bound and the in-mainloop converter warps would set its pace.
// Smaller GEMMs are weight-bandwidth-bound and keep the int8 weights
// end to end (GemmKind::kW8).
constexpr int kW8WidenRows = 4096;

int bn_index(int bn) { return bn == 256 ? 0 : (bn == 192 ? 1 : 2); }
constexpr int kBlockWidths[3] = {256, 192, 128};

// One layer on a device.  BERT family / nomic (post-norm): ln1/ln2 after
// the residual adds.  Qwen3 / ModernBERT / Gemma3 (pre-norm): attn_norm
// before QKV (nullptr: identity, ModernBERT layer 0), ffn_norm before the
// FFN, post_attn / post_ffn on the sublayer outputs (Gemma), q_norm /
// k_norm (QK-norm).  ffn1 is a GLU GEMM (rows interleaved by 32) where the
// architecture gates.
struct DevLayer {
    DevDense qkv, o, ffn1, ffn2;
    float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *post_attn = nullptr, *post_ffn = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
    bool global = true;
};

struct Replica {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
    float *word = nullptr, *pos = nullptr, *type0 = nullptr, *emb_g = nullptr, *emb_b = nullptr;
    float* rel_bias = nullptr;  // MPNet: [heads x (2*rel_bias_off + 1)] by j - i
    int rel_bias_off = 0;
    float emb_scale = 1.0f;     // Gemma: sqrt(H)
    float *final_norm = nullptr, *zero_beta = nullptr;
    float *cos_g = nullptr, *sin_g = nullptr, *cos_l = nullptr, *sin_l = nullptr;  // RoPE [positions x dh/2]
    // the same tables as [dh/8][positions][4] (the QKV epilogue's layout:
    // one 16-byte load per lane, lanes on consecutive positions contiguous)
    float *cos4_g = nullptr, *sin4_g = nullptr, *cos4_l = nullptr, *sin4_l = nullptr;
    int rope_npos = 0;
    float *dense1 = nullptr, *dense2 = nullptr;  // Gemma Dense head, fp32
    std::vector<DevLayer> layers;
    // workspace
    int cap_T = 0, cap_seq = 0, cap_out = 0;
    std::vector<void*> ws;
    float *x32 = nullptr, *y32 = nullptr;
    act16 *xb = nullptr, *qkv = nullptr, *ctx = nullptr, *ffh = nullptr;
    int8_t *xq = nullptr, *ctxq = nullptr, *ffhq = nullptr;
    float *xs = nullptr, *ctxs = nullptr, *ffhs = nullptr;
    float2* lnst = nullptr;  // post-norm: the last LayerNorm's per-row (mean, rstd)
    int32_t* pos32 = nullptr;  // [T]: each token's position in its sequence (RoPE in the QKV epilogue)
    // Folded norms (post-norm BERT family in the 16-bit modes; Qwen3 and
    // ModernBERT input norms in bf16): the residual GEMM writes its
    // output's 32-column chunk statistics (parts) and a 16-bit copy in xb, a
    // small kernel merges the chunks into lnst, and the next GEMM reads the
    // copy with the norm's gain folded into its weight.
    bool fold = false;
    bool fold_w8 = false;     // weight-only int8 folding (the gain through the activation copy)
    bool fold_rms = false;    // pre-norm stacks: the folded norms are RMSNorms (Qwen3)
    float2* parts = nullptr;  // [H / 32 x T]
    float* pick32 = nullptr;  // [sequences x H]: the final norm of each sequence's pooled row
    int32_t* iota = nullptr;                                            // [0, 1, ..., cap_seq]
    int64_t* d_ids = nullptr;
    int32_t* d_cu = nullptr;
    float* d_out = nullptr;
    int* d_status = nullptr;
    uint16_t* w16 = nullptr;  // weight-only int8: fp16 widening scratch (one layer's weights)
    size_t w16_elems = 0;
    // Pinned host staging, two slots so that one batch can be staged while
    // the previous one runs (rg_submit / rg_collect); the device buffers are
    // shared, the slots' work being ordered on the replica's stream.
    struct Staging {
        int64_t* ids = nullptr;
        int32_t* cu = nullptr;
        float* out = nullptr;
        int* status = nullptr;
        size_t cap_ids = 0, cap_cu = 0, cap_out = 0;
        cudaEvent_t done = nullptr;  // recorded after the slot's D2H copies
        bool busy = false;           // submitted, not yet collected
        float* user_out = nullptr;   // the caller's output buffer
        // where rg_collect copies the slot's result: (offset in user_out,
        // offset in out, floats), one entry per run of consecutive sequences
        std::vector<std::array<size_t, 3>> copies;
    };
    Staging stage[2];
    OpMaps tm_x, tm_ctx, tm_ffh;
    // strict fp32: GEMM operands as tf32 hi + fp32 remainder; qkv in fp32
    float *xh = nullptr, *xl = nullptr, *ctxh = nullptr, *ctxl = nullptr, *ffhh = nullptr, *ffhl = nullptr;
    float* qkv32 = nullptr;
    int tm_T = -1;
    int last_launches = 0;
    const int32_t* h_cu_view = nullptr;  // host copy of the current batch's offsets
    int rev_m = 0;  // the next GEMMs walk their row blocks last to first (L2-aware order)
    // kernel timing (rg_profile)
    bool prof = false;
    // CUDA graphs of whole forwards, one per batch shape and buffer set (see
    // GraphKey); ws_gen changes whenever a workspace or staging buffer is
    // reallocated, which retires every graph that captured the old ones.
    uint64_t ws_gen = 1;
    struct GraphKey {
        int T, nseq, max_len, out_kind, out_dim;
        const void *ids, *cu, *out;  // device inputs / output (nullptr: host path)
        uint64_t gen;
        bool operator==(const GraphKey& o) const {
            return T == o.T && nseq == o.nseq && max_len == o.max_len && out_kind == o.out_kind &&
                   out_dim == o.out_dim && ids == o.ids && cu == o.cu && out == o.out && gen == o.gen;
        }
    };
    std::vector<std::pair<GraphKey, cudaGraphExec_t>> graphs;
    std::vector<GraphKey> seen_once;  // shapes run once eagerly; captured on their second call
    int graph_launches = 0;           // kernel launches inside the cached graphs (last capture)
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_used = 0;
    struct Rec {
        int cls;
        size_t e0, e1;
        double flops, bytes;
    };
    std::vector<Rec> pending;
    double st_ms[RG_KC_COUNT] = {}, st_flops[RG_KC_COUNT] = {}, st_bytes[RG_KC_COUNT] = {};
    int st_n[RG_KC_COUNT] = {};
    std::mutex mu;
};

}  // namespace

struct rg_ctx {
    rg_model_desc d{};
    int mode = RG_MODE_BF16;
    std::vector<int> devices;
    std::map<std::string, HostTensor> host;
    std::vector<Replica*> reps;
    bool finalized = false;
    std::mutex mu;
    // host-batch submissions: ticket t uses staging slot t % 2 of every
    // replica; pending[slot] is the ticket in flight there, kSlotFree, or
    // kSlotCollecting while its results are being copied out
    std::mutex tmu;
    std::condition_variable tcv;  // a slot became free
    int64_t next_ticket = 0;
    int64_t pending[2] = {-1, -1};
    // failure injection for tests (rg_test_inject): the next submission's
    // host staging fails as an allocation failure would; replica
    // inject_replica fails its next shard submission
    bool inject_alloc = false;
    int inject_replica = -1;
};

constexpr int64_t kSlotFree = -1, kSlotCollecting = -2;

// rg_test_inject(RG_INJECT_GEMM_WAIT): the wait limit (cycles) of the next
// kernel-level rg_dense_bf16 launch, which withholds one pipeline arrival
// (0: none pending).
std::atomic<long long> g_inject_gemm_wait{0};

namespace {

int max_seq_len(const rg_model_desc& d) {
    int off = (d.arch == RG_ARCH_MPNET || d.arch == RG_ARCH_ROBERTA) ? d.pad_token_id + 1 : 0;
    return d.max_position_embeddings - off;
}
int pos_offset(const rg_model_desc& d) {
    return (d.arch == RG_ARCH_MPNET || d.arch == RG_ARCH_ROBERTA) ? d.pad_token_id + 1 : 0;
}

// Row widths the LayerNorm kernels are instantiated for (kernels.cu).
bool ln_width_ok(int n) {
    if (n <= 0 || n % 128 != 0) return false;
    switch (n / 128) {
    case 1: case 2: case 3: case 4: case 6: case 8: case 12: case 16: return true;
    default: return false;
    }
}

bool is_bert_family(int a) {
    return a == RG_ARCH_BERT || a == RG_ARCH_DISTILBERT || a == RG_ARCH_ROBERTA || a == RG_ARCH_MPNET;
}
// Pre-norm stacks: norm before each sublayer, residual added raw.
bool is_prenorm(int a) { return a == RG_ARCH_QWEN3 || a == RG_ARCH_MODERNBERT || a == RG_ARCH_GEMMA3; }
bool has_rope(int a) { return a == RG_ARCH_QWEN3 || a == RG_ARCH_MODERNBERT || a == RG_ARCH_GEMMA3 || a == RG_ARCH_NOMIC; }
bool is_glu(int a) { return a == RG_ARCH_QWEN3 || a == RG_ARCH_MODERNBERT || a == RG_ARCH_GEMMA3 || a == RG_ARCH_NOMIC; }

struct Dims {
    int H, I, nq, nkv, dh, qd, kvd, nqkv;
};
Dims dims(const rg_model_desc& d) {
    Dims m{};
    m.H = d.hidden_size;
    m.I = d.intermediate_size;
    m.nq = d.num_attention_heads;
    m.dh = d.head_dim > 0 ? d.head_dim : d.hidden_size / d.num_attention_heads;
    m.nkv = (d.arch == RG_ARCH_QWEN3 || d.arch == RG_ARCH_GEMMA3) ? d.num_key_value_heads : m.nq;
    m.qd = m.nq * m.dh;
    m.kvd = m.nkv * m.dh;
    m.nqkv = m.qd + 2 * m.kvd;
    return m;
}

// relPosBucket (bert.go:126-150): MPNet's bucket of a relative position
// (memory j - context i), HF's relative_position_bucket with max distance 128.
int rel_pos_bucket(int rel, int num_buckets) {
    int n = -rel;
    const int half = num_buckets / 2;
    int ret = 0;
    if (n < 0) {
        ret = half;
        n = -n;
    }
    const int max_exact = half / 2;
    if (n < max_exact) return ret + n;
    const int v = max_exact + static_cast<int>(std::log(static_cast<double>(n) / max_exact) /
                                               std::log(128.0 / max_exact) * static_cast<double>(half - max_exact));
    return ret + std::min(v, half - 1);
}

// bf16 round-to-nearest-even of a float (NaN kept quiet).
uint16_t to_bf16_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

// fp16 round-to-nearest-even of a float; false if it overflows the fp16
// range (|f| rounds above 65504) or is not finite.
bool to_f16_bits(float f, uint16_t* out) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return false;
    const int e = static_cast<int>(a >> 23) - 127;  // unbiased exponent
    if (e < -25) {                                  // below half the smallest subnormal
        *out = static_cast<uint16_t>(sign);
        return true;
    }
    uint32_t mant = (a & 0x7fffffu) | 0x800000u;  // 24-bit significand
    int shift;                                     // bits dropped from the 24-bit significand
    uint32_t base;                                 // exponent field of the result, pre-rounding
    if (e < -14) {  // subnormal result q * 2^-24 with q = mant * 2^(e + 1)
        shift = -e - 1;
        base = 0;
    } else {
        shift = 13;
        base = static_cast<uint32_t>(e + 15) << 10;
        mant &= 0x7fffffu;  // drop the implicit bit: it lives in the exponent field
    }
    uint32_t q = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (q & 1u))) ++q;  // carries into the exponent field as needed
    const uint32_t h = base + q;
    if (h >= 0x7c00u) return false;
    *out = static_cast<uint16_t>(sign | h);
    return true;
}

bool finite32(float v) { return std::isfinite(v); }

float bf16_bits_to_float(uint16_t h) {
    const uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float f16_bits_to_float(uint16_t h) {  // exact: every fp16 value is a float
    const int e = (h >> 10) & 0x1f, m = h & 0x3ff;
    const float v = e == 0 ? std::ldexp(static_cast<float>(m), -24) : std::ldexp(static_cast<float>(m | 0x400), e - 25);
    return (h & 0x8000) ? -v : v;
}

// PackB8 (pack8.go:25-76): float32 scale maxAbs/127, float64 division,
// round half to even, clamp +-127.
void quant_packb8(const float* w, int N, int K, int8_t* q, float* scales) {
    for (int j = 0; j < N; ++j) {
        const float* row = w + static_cast<size_t>(j) * K;
        float maxabs = 0.f;
        for (int p = 0; p < K; ++p) {
            if (!finite32(row[p])) fail("PackB8: channel %d has a non-finite weight", j);
            maxabs = std::max(maxabs, std::fabs(row[p]));
        }
        float s = maxabs / 127.0f;
        if (s == 0.f) s = 1.f;
        scales[j] = s;
        for (int p = 0; p < K; ++p) {
            double v = std::nearbyint(static_cast<double>(row[p]) / static_cast<double>(s));
            v = std::min(127.0, std::max(-127.0, v));
            q[static_cast<size_t>(j) * K + p] = static_cast<int8_t>(v);
        }
    }
}

// PackB8VNNI (pack_vnni.go:28-77): float64 scale, q = int8(RoundToEven(w/s)),
// stored dequant scale float32(s).
void quant_packb8vnni(const float* w, int N, int K, int8_t* q, float* scales) {
    for (int c = 0; c < N; ++c) {
        const float* row = w + static_cast<size_t>(c) * K;
        double maxabs = 0.0;
        for (int p = 0; p < K; ++p) {
            if (!finite32(row[p])) fail("PackB8VNNI: weight [%d,%d] is not finite", c, p);
            maxabs = std::max(maxabs, std::fabs(static_cast<double>(row[p])));
        }
        double s = maxabs / 127.0;
        if (s == 0.0) s = 1.0;
        scales[c] = static_cast<float>(s);
        for (int p = 0; p < K; ++p)
            q[static_cast<size_t>(c) * K + p] =
                static_cast<int8_t>(static_cast<int32_t>(std::nearbyint(static_cast<double>(row[p]) / s)));
    }
}

template <typename T>
T* dev_alloc(Replica& r, size_t count) {
    void* p = nullptr;
    check(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)), "cudaMalloc");
    r.allocs.push_back(p);
    return static_cast<T*>(p);
}

template <typename T>
T* dev_upload(Replica& r, const T* host, size_t count) {
    T* p = dev_alloc<T>(r, count);
    check(cudaMemcpy(p, host, count * sizeof(T), cudaMemcpyHostToDevice), "cudaMemcpy H2D");
    return p;
}

const HostTensor& get_tensor(rg_ctx* c, const std::string& name, std::initializer_list<int64_t> shape) {
    static const char* prefixes[] = {"", "bert.", "roberta.", "mpnet.", "distilbert.", "model."};
    for (const char* p : prefixes) {
        auto it = c->host.find(std::string(p) + name);
        if (it == c->host.end()) continue;
        const HostTensor& t = it->second;
        std::vector<int64_t> want(shape);
        if (t.shape != want) {
            std::string got, exp;
            for (auto v : t.shape) got += std::to_string(v) + ",";
            for (auto v : want) exp += std::to_string(v) + ",";
            fail("tensor %s has shape [%s], want [%s]", it->first.c_str(), got.c_str(), exp.c_str());
        }
        return t;
    }
    fail("missing tensor %s", name.c_str());
}

// Quantise/convert a [N x K] fp32 weight for `mode` and upload it.
DevDense make_dense(Replica& r, int mode, const float* w, const float* bias, int N, int K) {
    DevDense d;
    d.N = N;
    d.K = K;
    const size_t n = static_cast<size_t>(N) * K;
    if (mode == RG_MODE_BF16) {
        std::vector<uint16_t> h(n);
        for (size_t i = 0; i < n; ++i) h[i] = to_bf16_bits(w[i]);
        d.w = dev_upload(r, h.data(), n);
    } else if (mode == RG_MODE_FP32) {
        std::vector<float> hi(n), lo(n);
        for (size_t i = 0; i < n; ++i) {
            if (!finite32(w[i])) fail("weight [%zu, %zu] is not finite", i / K, i % K);
            rg::tf32_split(w[i], hi[i], lo[i]);
        }
        d.w = dev_upload(r, hi.data(), n);
        d.w_lo = dev_upload(r, lo.data(), n);
    } else if (mode == RG_MODE_F16) {
        std::vector<uint16_t> h(n);
        for (size_t i = 0; i < n; ++i)
            if (!to_f16_bits(w[i], &h[i]))
                fail("f16 mode: weight [%zu, %zu] = %g is outside the fp16 range", i / K, i % K,
                     static_cast<double>(w[i]));
        d.w = dev_upload(r, h.data(), n);
    } else {
        std::vector<int8_t> q(n);
        std::vector<float> s(N);
        if (mode == RG_MODE_INT8_FULL)
            quant_packb8vnni(w, N, K, q.data(), s.data());
        else
            quant_packb8(w, N, K, q.data(), s.data());
        d.w = dev_upload(r, q.data(), n);
        d.scale = dev_upload(r, s.data(), N);
    }
    const int eb = mode == RG_MODE_FP32 ? 4 : ((mode == RG_MODE_BF16 || mode == RG_MODE_F16) ? 2 : 1);
    for (int i = 0; i < 3; ++i) {
        if (N % kBlockWidths[i] != 0) continue;
        const uint32_t box_rows = rg::gemm_w_box_rows(kBlockWidths[i]);
        const bool ok = mode == RG_MODE_INT8_W ? rg::make_w8_tmap(&d.tmap[i], d.w, N, K, box_rows)
                                               : rg::make_kmajor_tmap(&d.tmap[i], d.w, eb, N, K, K, box_rows);
        if (!ok) fail("cuTensorMapEncodeTiled failed for a [%d x %d] weight", N, K);
        if (mode == RG_MODE_FP32 && !rg::make_kmajor_tmap(&d.tmap_lo[i], d.w_lo, 4, N, K, K, box_rows))
            fail("cuTensorMapEncodeTiled failed for a [%d x %d] weight remainder", N, K);
    }
    if (bias) d.bias = dev_upload(r, bias, N);
    return d;
}

// The weight W [N x K] of a GEMM whose input is LN(y) = (y - mean) * rstd *
// g + b, folded so the GEMM reads y itself: w = round16(W * g) by column,
// bias' = W.b + bias, and c1[n] = sum_k w[n][k] so the epilogue computes
// rstd * (y.w - mean * c1) + bias'.  In the fp16 mode it returns false
// (nothing uploaded) when some W * g falls outside the fp16 range.
bool fold_ok(int mode, const float* W, const float* g, int N, int K) {
    if (mode != RG_MODE_F16) return true;
    uint16_t h;
    for (int n = 0; n < N; ++n)
        for (int k = 0; k < K; ++k)
            if (!to_f16_bits(W[static_cast<size_t>(n) * K + k] * g[k], &h)) return false;
    return true;
}

DevDense make_dense_folded(Replica& r, int mode, const float* W, const float* bias, int N, int K, const float* g,
                           const float* b) {
    std::vector<float> wf(static_cast<size_t>(N) * K), bf(N), c1(N);
    for (int n = 0; n < N; ++n) {
        const float* row = W + static_cast<size_t>(n) * K;
        double wb = bias ? bias[n] : 0.0, cs = 0.0;
        for (int k = 0; k < K; ++k) {
            const float v = row[k] * g[k];
            wf[static_cast<size_t>(n) * K + k] = v;
            wb += static_cast<double>(row[k]) * b[k];
            uint16_t h;
            if (mode == RG_MODE_F16) {
                if (!to_f16_bits(v, &h)) fail("folded weight [%d, %d] outside the fp16 range", n, k);
                cs += f16_bits_to_float(h);
            } else {
                cs += bf16_bits_to_float(to_bf16_bits(v));
            }
        }
        bf[n] = static_cast<float>(wb);
        c1[n] = static_cast<float>(cs);
    }
    DevDense d = make_dense(r, mode, wf.data(), bf.data(), N, K);
    d.fold_c1 = dev_upload(r, c1.data(), N);
    return d;
}

// Weight-only int8 GEMM whose input is LN(y): the int8 weight is the
// reference's quantisation of W itself (q, per-column s; make_dense), and the
// gain reaches the product through the activation copy instead (the residual
// GEMM that writes y writes round16(y * g)), so the epilogue's fold terms are
// those of the dequantised weight q * s: c1[n] = s[n] * sum_k g[k] q[n][k],
// bias'[n] = bias[n] + s[n] * sum_k b[k] q[n][k] (double sums).
DevDense make_dense_w8_folded(Replica& r, const float* W, const float* bias, int N, int K, const float* g,
                              const float* b) {
    DevDense d = make_dense(r, RG_MODE_INT8_W, W, bias, N, K);
    std::vector<int8_t> q(static_cast<size_t>(N) * K);
    std::vector<float> s(N), c1(N), bf(N);
    quant_packb8(W, N, K, q.data(), s.data());
    for (int n = 0; n < N; ++n) {
        const int8_t* row = q.data() + static_cast<size_t>(n) * K;
        double cg = 0.0, cb = 0.0;
        for (int k = 0; k < K; ++k) {
            cg += static_cast<double>(g[k]) * row[k];
            cb += static_cast<double>(b[k]) * row[k];
        }
        c1[n] = static_cast<float>(s[n] * cg);
        bf[n] = static_cast<float>((bias ? bias[n] : 0.0) + s[n] * cb);
    }
    d.fold_c1 = dev_upload(r, c1.data(), N);
    d.fold_bias = dev_upload(r, bf.data(), N);
    return d;
}

void finalize_bert(rg_ctx* c, Replica& r) {
    const rg_model_desc& d = c->d;
    const int H = d.hidden_size, I = d.intermediate_size, V = d.vocab_size, P = d.max_position_embeddings;
    const bool distil = d.arch == RG_ARCH_DISTILBERT;
    const bool mpnet = d.arch == RG_ARCH_MPNET;
    check(cudaSetDevice(r.device), "cudaSetDevice");
    r.word = dev_upload(r, get_tensor(c, "embeddings.word_embeddings.weight", {V, H}).data.data(), (size_t)V * H);
    r.pos = dev_upload(r, get_tensor(c, "embeddings.position_embeddings.weight", {P, H}).data.data(), (size_t)P * H);
    r.emb_g = dev_upload(r, get_tensor(c, "embeddings.LayerNorm.weight", {H}).data.data(), H);
    r.emb_b = dev_upload(r, get_tensor(c, "embeddings.LayerNorm.bias", {H}).data.data(), H);
    if (mpnet) {
        // One shared bucketed bias table [buckets x heads] (bert.go:495-505),
        // expanded to [heads x (2*maxlen - 1)] by j - i (bert.go:820-830).
        const int nb = d.relative_attention_num_buckets, heads = d.num_attention_heads;
        const float* rb = get_tensor(c, "encoder.relative_attention_bias.weight", {nb, heads}).data.data();
        const int maxlen = max_seq_len(d);
        const int nd = 2 * maxlen - 1;
        std::vector<float> delta(static_cast<size_t>(heads) * nd);
        for (int dd = -(maxlen - 1); dd <= maxlen - 1; ++dd) {
            const int b = rel_pos_bucket(dd, nb);
            for (int h = 0; h < heads; ++h) delta[static_cast<size_t>(h) * nd + dd + maxlen - 1] = rb[b * heads + h];
        }
        r.rel_bias = dev_upload(r, delta.data(), delta.size());
        r.rel_bias_off = maxlen - 1;
    } else if (!distil) {
        // token_type_embeddings: any first dimension, row 0 used (bert.go:507-515)
        const HostTensor* tt = nullptr;
        for (const char* p : {"", "bert.", "roberta."}) {
            auto it = c->host.find(std::string(p) + "embeddings.token_type_embeddings.weight");
            if (it != c->host.end()) tt = &it->second;
        }
        if (!tt) fail("missing tensor embeddings.token_type_embeddings.weight");
        if (tt->shape.size() != 2 || tt->shape[1] != H || tt->shape[0] < 1)
            fail("token_type_embeddings has a bad shape");
        r.type0 = dev_upload(r, tt->data.data(), H);
    }
    r.layers.resize(d.num_hidden_layers);
    struct HostLayer {
        const float *qW, *qB, *kW, *kB, *vW, *vB, *oW, *oB, *f1W, *f1B, *f2W, *f2B, *g1, *b1, *g2, *b2;
    };
    std::vector<HostLayer> hl(d.num_hidden_layers);
    for (int li = 0; li < d.num_hidden_layers; ++li) {
        const std::string p = (distil ? "transformer.layer." : "encoder.layer.") + std::to_string(li) + ".";
        auto T = [&](const std::string& n, std::initializer_list<int64_t> s) -> const float* {
            return get_tensor(c, p + n, s).data.data();
        };
        HostLayer& w = hl[li];
        if (distil) {
            w.qW = T("attention.q_lin.weight", {H, H});
            w.qB = T("attention.q_lin.bias", {H});
            w.kW = T("attention.k_lin.weight", {H, H});
            w.kB = T("attention.k_lin.bias", {H});
            w.vW = T("attention.v_lin.weight", {H, H});
            w.vB = T("attention.v_lin.bias", {H});
            w.oW = T("attention.out_lin.weight", {H, H});
            w.oB = T("attention.out_lin.bias", {H});
            w.g1 = T("sa_layer_norm.weight", {H});
            w.b1 = T("sa_layer_norm.bias", {H});
            w.f1W = T("ffn.lin1.weight", {I, H});
            w.f1B = T("ffn.lin1.bias", {I});
            w.f2W = T("ffn.lin2.weight", {H, I});
            w.f2B = T("ffn.lin2.bias", {H});
            w.g2 = T("output_layer_norm.weight", {H});
            w.b2 = T("output_layer_norm.bias", {H});
        } else if (mpnet) {
            w.qW = T("attention.attn.q.weight", {H, H});
            w.qB = T("attention.attn.q.bias", {H});
            w.kW = T("attention.attn.k.weight", {H, H});
            w.kB = T("attention.attn.k.bias", {H});
            w.vW = T("attention.attn.v.weight", {H, H});
            w.vB = T("attention.attn.v.bias", {H});
            w.oW = T("attention.attn.o.weight", {H, H});
            w.oB = T("attention.attn.o.bias", {H});
            w.g1 = T("attention.LayerNorm.weight", {H});
            w.b1 = T("attention.LayerNorm.bias", {H});
            w.f1W = T("intermediate.dense.weight", {I, H});
            w.f1B = T("intermediate.dense.bias", {I});
            w.f2W = T("output.dense.weight", {H, I});
            w.f2B = T("output.dense.bias", {H});
            w.g2 = T("output.LayerNorm.weight", {H});
            w.b2 = T("output.LayerNorm.bias", {H});
        } else {
            w.qW = T("attention.self.query.weight", {H, H});
            w.qB = T("attention.self.query.bias", {H});
            w.kW = T("attention.self.key.weight", {H, H});
            w.kB = T("attention.self.key.bias", {H});
            w.vW = T("attention.self.value.weight", {H, H});
            w.vB = T("attention.self.value.bias", {H});
            w.oW = T("attention.output.dense.weight", {H, H});
            w.oB = T("attention.output.dense.bias", {H});
            w.g1 = T("attention.output.LayerNorm.weight", {H});
            w.b1 = T("attention.output.LayerNorm.bias", {H});
            w.f1W = T("intermediate.dense.weight", {I, H});
            w.f1B = T("intermediate.dense.bias", {I});
            w.f2W = T("output.dense.weight", {H, I});
            w.f2B = T("output.dense.bias", {H});
            w.g2 = T("output.LayerNorm.weight", {H});
            w.b2 = T("output.LayerNorm.bias", {H});
        }
    }
    // LayerNorm folding (16-bit modes, every folded weight in range; the
    // weight-only int8 mode, whose weights stay as quantised)
    r.fold_w8 = c->mode == RG_MODE_INT8_W && H % 32 == 0;
    r.fold = (c->mode == RG_MODE_BF16 || c->mode == RG_MODE_F16 || r.fold_w8) && H % 32 == 0;
    for (int li = 0; li < d.num_hidden_layers && r.fold; ++li) {
        const HostLayer& w = hl[li];
        r.fold = fold_ok(c->mode, w.f1W, w.g1, I, H);
        if (li > 0)
            for (const float* W : {w.qW, w.kW, w.vW}) r.fold = r.fold && fold_ok(c->mode, W, hl[li - 1].g2, H, H);
    }
    for (int li = 0; li < d.num_hidden_layers; ++li) {
        const HostLayer& w = hl[li];
        DevLayer& L = r.layers[li];
        L.ln1_g = dev_upload(r, w.g1, H);
        L.ln1_b = dev_upload(r, w.b1, H);
        L.ln2_g = dev_upload(r, w.g2, H);
        L.ln2_b = dev_upload(r, w.b2, H);
        // Q||K||V fused as [3H x H] rows (bert.go:479-485).
        std::vector<float> qkvW(static_cast<size_t>(3) * H * H), qkvB(3 * H);
        memcpy(qkvW.data(), w.qW, sizeof(float) * H * H);
        memcpy(qkvW.data() + (size_t)H * H, w.kW, sizeof(float) * H * H);
        memcpy(qkvW.data() + (size_t)2 * H * H, w.vW, sizeof(float) * H * H);
        memcpy(qkvB.data(), w.qB, sizeof(float) * H);
        memcpy(qkvB.data() + H, w.kB, sizeof(float) * H);
        memcpy(qkvB.data() + 2 * H, w.vB, sizeof(float) * H);
        // layer 0's QKV reads the embedding LayerNorm's output as is
        L.qkv = r.fold_w8 && li > 0
                    ? make_dense_w8_folded(r, qkvW.data(), qkvB.data(), 3 * H, H, hl[li - 1].g2, hl[li - 1].b2)
                : r.fold && li > 0
                    ? make_dense_folded(r, c->mode, qkvW.data(), qkvB.data(), 3 * H, H, hl[li - 1].g2, hl[li - 1].b2)
                    : make_dense(r, c->mode, qkvW.data(), qkvB.data(), 3 * H, H);
        L.o = make_dense(r, c->mode, w.oW, w.oB, H, H);
        L.ffn1 = r.fold_w8 ? make_dense_w8_folded(r, w.f1W, w.f1B, I, H, w.g1, w.b1)
                 : r.fold  ? make_dense_folded(r, c->mode, w.f1W, w.f1B, I, H, w.g1, w.b1)
                           : make_dense(r, c->mode, w.f1W, w.f1B, I, H);
        L.ffn2 = make_dense(r, c->mode, w.f2W, w.f2B, H, I);
    }
}

// GLU weight for the fused gate/up GEMM: rows interleaved in blocks of 32,
// block 2j = act[32j, 32j+32), block 2j+1 = lin[32j, 32j+32).
std::vector<float> interleave_glu(const float* act, const float* lin, int I, int K) {
    std::vector<float> w(static_cast<size_t>(2) * I * K);
    for (int b = 0; b < I / 32; ++b) {
        memcpy(&w[(static_cast<size_t>(2 * b) * 32) * K], act + static_cast<size_t>(b) * 32 * K, sizeof(float) * 32 * K);
        memcpy(&w[(static_cast<size_t>(2 * b + 1) * 32) * K], lin + static_cast<size_t>(b) * 32 * K,
               sizeof(float) * 32 * K);
    }
    return w;
}

std::vector<float> concat_rows(std::initializer_list<std::pair<const float*, size_t>> parts) {
    std::vector<float> w;
    for (const auto& p : parts) w.insert(w.end(), p.first, p.first + p.second);
    return w;
}

// ropeTable (modernbert.go:108-123): float64 inverse frequencies and trig,
// rounded to float32, for positions [0, npos).
void rope_tables(Replica& r, int npos, int dh, double theta, float** cosp, float** sinp, float** cos4p,
                 float** sin4p) {
    const int half = dh / 2;
    std::vector<float> cs(static_cast<size_t>(npos) * half), sn(static_cast<size_t>(npos) * half);
    for (int d = 0; d < half; ++d) {
        const double inv = std::pow(theta, -2.0 * d / dh);
        for (int p = 0; p < npos; ++p) {
            const double ang = static_cast<double>(p) * inv;
            cs[static_cast<size_t>(p) * half + d] = static_cast<float>(std::cos(ang));
            sn[static_cast<size_t>(p) * half + d] = static_cast<float>(std::sin(ang));
        }
    }
    *cosp = dev_upload(r, cs.data(), cs.size());
    *sinp = dev_upload(r, sn.data(), sn.size());
    r.rope_npos = npos;
    if (half % 4 == 0) {  // [half/4][npos][4]
        std::vector<float> c4(cs.size()), s4(sn.size());
        for (int p = 0; p < npos; ++p)
            for (int d = 0; d < half; ++d) {
                const size_t o = (static_cast<size_t>(d / 4) * npos + p) * 4 + d % 4;
                c4[o] = cs[static_cast<size_t>(p) * half + d];
                s4[o] = sn[static_cast<size_t>(p) * half + d];
            }
        *cos4p = dev_upload(r, c4.data(), c4.size());
        *sin4p = dev_upload(r, s4.data(), s4.size());
    }
}

std::vector<float> unit_offset(const float* v, int n) {  // gemma3.go:44-50
    std::vector<float> o(v, v + n);
    for (float& x : o) x += 1.0f;
    return o;
}

// Qwen3 (qwen3.go:114-183), Gemma3 (gemma3.go:57-170), ModernBERT
// (modernbert.go:33-106), nomic (nomic.go:22-111): weights by HF name.
void finalize_decoder(rg_ctx* c, Replica& r) {
    const rg_model_desc& d = c->d;
    const Dims m = dims(d);
    const int H = m.H, I = m.I, V = d.vocab_size, dh = m.dh;
    const int arch = d.arch;
    check(cudaSetDevice(r.device), "cudaSetDevice");
    auto G = [&](const std::string& n, std::initializer_list<int64_t> sh) -> const float* {
        return get_tensor(c, n, sh).data.data();
    };
    auto up = [&](const float* h, size_t n) { return dev_upload(r, h, n); };
    const int npos = d.max_position_embeddings;
    if (arch == RG_ARCH_QWEN3 || arch == RG_ARCH_GEMMA3) {
        r.word = up(G("embed_tokens.weight", {V, H}), static_cast<size_t>(V) * H);
        if (arch == RG_ARCH_QWEN3) {
            r.final_norm = up(G("norm.weight", {H}), H);
            rope_tables(r, npos, dh, d.rope_theta, &r.cos_g, &r.sin_g, &r.cos4_g, &r.sin4_g);
        } else {
            r.final_norm = up(unit_offset(G("norm.weight", {H}), H).data(), H);
            r.emb_scale = static_cast<float>(std::sqrt(static_cast<double>(H)));
            rope_tables(r, npos, dh, d.global_rope_theta, &r.cos_g, &r.sin_g, &r.cos4_g, &r.sin4_g);
            rope_tables(r, npos, dh, d.local_rope_theta, &r.cos_l, &r.sin_l, &r.cos4_l, &r.sin4_l);
            const int D = d.dense_hidden;
            r.dense1 = up(G("2_Dense.linear.weight", {D, H}), static_cast<size_t>(D) * H);
            r.dense2 = up(G("3_Dense.linear.weight", {H, D}), static_cast<size_t>(H) * D);
        }
    } else if (arch == RG_ARCH_MODERNBERT) {
        r.word = up(G("embeddings.tok_embeddings.weight", {V, H}), static_cast<size_t>(V) * H);
        r.emb_g = up(G("embeddings.norm.weight", {H}), H);
        r.final_norm = up(G("final_norm.weight", {H}), H);
        std::vector<float> z(H, 0.0f);
        r.zero_beta = up(z.data(), H);
        rope_tables(r, npos, dh, d.global_rope_theta, &r.cos_g, &r.sin_g, &r.cos4_g, &r.sin4_g);
        rope_tables(r, npos, dh, d.local_rope_theta, &r.cos_l, &r.sin_l, &r.cos4_l, &r.sin4_l);
    } else {  // nomic
        r.word = up(G("embeddings.word_embeddings.weight", {V, H}), static_cast<size_t>(V) * H);
        r.type0 = up(G("embeddings.token_type_embeddings.weight", {2, H}), H);
        r.emb_g = up(G("emb_ln.weight", {H}), H);
        r.emb_b = up(G("emb_ln.bias", {H}), H);
        rope_tables(r, npos, dh, d.rope_theta, &r.cos_g, &r.sin_g, &r.cos4_g, &r.sin4_g);
    }
    r.layers.resize(d.num_hidden_layers);
    // Pre-norm stacks whose input norms fold into the GEMMs (bf16 mode): the
    // residual GEMMs write a 16-bit copy of the stream and its chunk
    // statistics; QKV (layers 1...) and the gated FFN use gain-folded
    // weights.  Qwen3's RMSNorm (no mean) and ModernBERT's bias-free
    // LayerNorm; the first layer's first norm still runs as a kernel.
    r.fold = c->mode == RG_MODE_BF16 && (arch == RG_ARCH_QWEN3 || arch == RG_ARCH_MODERNBERT) && H % 32 == 0;
    r.fold_rms = r.fold && arch == RG_ARCH_QWEN3;
    const std::vector<float> zero_h(H, 0.f);
    auto dense = [&](const float* W, int N, int K, const float* gain) {
        return r.fold && gain ? make_dense_folded(r, c->mode, W, nullptr, N, K, gain, zero_h.data())
                              : make_dense(r, c->mode, W, nullptr, N, K);
    };
    for (int li = 0; li < d.num_hidden_layers; ++li) {
        DevLayer& L = r.layers[li];
        if (arch == RG_ARCH_QWEN3 || arch == RG_ARCH_GEMMA3) {
            const std::string p = "layers." + std::to_string(li) + ".";
            auto norm = [&](const std::string& n, int len) {
                const float* v = G(p + n, {len});
                return arch == RG_ARCH_GEMMA3 ? up(unit_offset(v, len).data(), len) : up(v, len);
            };
            L.attn_norm = norm("input_layernorm.weight", H);
            L.q_norm = norm("self_attn.q_norm.weight", dh);
            L.k_norm = norm("self_attn.k_norm.weight", dh);
            if (arch == RG_ARCH_QWEN3) {
                L.ffn_norm = norm("post_attention_layernorm.weight", H);
            } else {
                L.post_attn = norm("post_attention_layernorm.weight", H);
                L.ffn_norm = norm("pre_feedforward_layernorm.weight", H);
                L.post_ffn = norm("post_feedforward_layernorm.weight", H);
                L.global = (li + 1) % d.sliding_window_pattern == 0;  // gemma3.go:91
            }
            const size_t qn = static_cast<size_t>(m.qd) * H, kn = static_cast<size_t>(m.kvd) * H;
            std::vector<float> wqkv = concat_rows({{G(p + "self_attn.q_proj.weight", {m.qd, H}), qn},
                                                   {G(p + "self_attn.k_proj.weight", {m.kvd, H}), kn},
                                                   {G(p + "self_attn.v_proj.weight", {m.kvd, H}), kn}});
            // (Gemma never folds: r.fold is off for it)
            L.qkv = dense(wqkv.data(), m.nqkv, H, li > 0 ? G(p + "input_layernorm.weight", {H}) : nullptr);
            L.o = make_dense(r, c->mode, G(p + "self_attn.o_proj.weight", {H, m.qd}), nullptr, H, m.qd);
            std::vector<float> wgu = interleave_glu(G(p + "mlp.gate_proj.weight", {I, H}),
                                                    G(p + "mlp.up_proj.weight", {I, H}), I, H);
            L.ffn1 = dense(wgu.data(), 2 * I, H,
                           arch == RG_ARCH_QWEN3 ? G(p + "post_attention_layernorm.weight", {H}) : nullptr);
            L.ffn2 = make_dense(r, c->mode, G(p + "mlp.down_proj.weight", {H, I}), nullptr, H, I);
        } else if (arch == RG_ARCH_MODERNBERT) {
            const std::string p = "layers." + std::to_string(li) + ".";
            L.global = li % d.global_attn_every_n_layers == 0;  // modernbert.go:73
            if (li != 0) L.attn_norm = up(G(p + "attn_norm.weight", {H}), H);
            L.ffn_norm = up(G(p + "mlp_norm.weight", {H}), H);
            L.qkv = dense(G(p + "attn.Wqkv.weight", {3 * H, H}), 3 * H, H,
                          li != 0 ? G(p + "attn_norm.weight", {H}) : nullptr);
            L.o = make_dense(r, c->mode, G(p + "attn.Wo.weight", {H, H}), nullptr, H, H);
            const float* wi = G(p + "mlp.Wi.weight", {2 * I, H});  // value rows [0, I), gate rows [I, 2I)
            std::vector<float> wgu = interleave_glu(wi, wi + static_cast<size_t>(I) * H, I, H);
            L.ffn1 = dense(wgu.data(), 2 * I, H, G(p + "mlp_norm.weight", {H}));
            L.ffn2 = make_dense(r, c->mode, G(p + "mlp.Wo.weight", {H, I}), nullptr, H, I);
        } else {  // nomic
            const std::string p = "encoder.layers." + std::to_string(li) + ".";
            L.ln1_g = up(G(p + "norm1.weight", {H}), H);
            L.ln1_b = up(G(p + "norm1.bias", {H}), H);
            L.ln2_g = up(G(p + "norm2.weight", {H}), H);
            L.ln2_b = up(G(p + "norm2.bias", {H}), H);
            L.qkv = make_dense(r, c->mode, G(p + "attn.Wqkv.weight", {3 * H, H}), nullptr, 3 * H, H);
            L.o = make_dense(r, c->mode, G(p + "attn.out_proj.weight", {H, H}), nullptr, H, H);
            // fc11 * silu(fc12): the activated operand is fc12 (nomic.go:232-242)
            std::vector<float> wgu = interleave_glu(G(p + "mlp.fc12.weight", {I, H}), G(p + "mlp.fc11.weight", {I, H}),
                                                    I, H);
            L.ffn1 = make_dense(r, c->mode, wgu.data(), nullptr, 2 * I, H);
            L.ffn2 = make_dense(r, c->mode, G(p + "mlp.fc2.weight", {H, I}), nullptr, H, I);
        }
    }
}

// Weight-only int8: tensor maps of each weight's shape over the fp16
// widening scratch (made once the scratch has its final size).
void make_widen_maps(Replica& r) {
    // A layer's four weights side by side (the same offsets in every layer
    // of the same shapes); the scratch holds the largest layer.
    size_t need = 0;
    for (DevLayer& L : r.layers) {
        size_t off = 0;
        for (DevDense* d : {&L.qkv, &L.o, &L.ffn1, &L.ffn2}) {
            d->w16_off = off;
            off += (static_cast<size_t>(d->N) * d->K + 63) / 64 * 64;
        }
        need = std::max(need, off);
    }
    if (need > r.w16_elems) {
        if (r.w16) cudaFree(r.w16);
        r.w16 = nullptr;
        check(cudaMalloc(&r.w16, need * 2), "cudaMalloc");
        r.w16_elems = need;
    }
    for (DevLayer& L : r.layers)
        for (DevDense* d : {&L.qkv, &L.o, &L.ffn1, &L.ffn2})
            for (int i = 0; i < 3; ++i) {
                if (d->N % kBlockWidths[i] != 0) continue;
                if (!rg::make_kmajor_tmap(&d->tmap16[i], r.w16 + d->w16_off, 2, d->N, d->K, d->K,
                                          rg::gemm_w_box_rows(kBlockWidths[i])))
                    fail("cuTensorMapEncodeTiled failed for a [%d x %d] widened weight", d->N, d->K);
            }
}



void free_workspace(Replica& r) {
    for (void* p : r.ws) cudaFree(p);
    r.ws.clear();
    r.cap_T = r.cap_seq = r.cap_out = 0;
    r.tm_T = -1;
}

template <typename T>
T* ws_alloc(Replica& r, size_t count) {
    void* p = nullptr;
    check(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)), "cudaMalloc (workspace)");
    r.ws.push_back(p);
    return static_cast<T*>(p);
}

// Grow the device workspace to hold T tokens / nseq sequences / nout floats.
void ensure_workspace(rg_ctx* c, Replica& r, int T, int nseq, size_t nout) {
    const rg_model_desc& d = c->d;
    const Dims m = dims(d);
    const int H = m.H, I = m.I;
    if (T > r.cap_T || nseq > r.cap_seq || nout > static_cast<size_t>(r.cap_out)) {
        // Any stream (ours or a caller's) may still read the old buffers.
        check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        for (void* p : r.ws) cudaFree(p);
        r.ws.clear();
        const int capT = std::max(T, r.cap_T);
        const int capS = std::max(nseq, r.cap_seq);
        const size_t capO = std::max<size_t>(nout, r.cap_out);
        const size_t t = static_cast<size_t>((capT + 255) / 256 * 256);
        r.x32 = ws_alloc<float>(r, t * H);
        r.y32 = ws_alloc<float>(r, t * H);
        r.lnst = ws_alloc<float2>(r, t);
        r.pos32 = ws_alloc<int32_t>(r, t);
        if (r.fold) r.parts = ws_alloc<float2>(r, t * (H / 32));
        if (c->mode == RG_MODE_FP32) {
            r.xh = ws_alloc<float>(r, t * H);
            r.xl = ws_alloc<float>(r, t * H);
            r.qkv32 = ws_alloc<float>(r, t * m.nqkv);
            r.ctxh = ws_alloc<float>(r, t * m.qd);
            r.ctxl = ws_alloc<float>(r, t * m.qd);
            r.ffhh = ws_alloc<float>(r, t * I);
            r.ffhl = ws_alloc<float>(r, t * I);
        } else {
            r.xb = ws_alloc<act16>(r, t * H);
            r.qkv = ws_alloc<act16>(r, t * m.nqkv);
            r.ctx = ws_alloc<act16>(r, t * m.qd);
            r.ffh = ws_alloc<act16>(r, t * I);
        }
        r.pick32 = ws_alloc<float>(r, static_cast<size_t>(capS) * H);
        r.iota = ws_alloc<int32_t>(r, capS + 1);
        {
            std::vector<int32_t> io(capS + 1);
            for (int i = 0; i <= capS; ++i) io[i] = i;
            check(cudaMemcpy(r.iota, io.data(), sizeof(int32_t) * (capS + 1), cudaMemcpyHostToDevice), "cudaMemcpy");
        }
        if (c->mode == RG_MODE_INT8_FULL) {
            r.xq = ws_alloc<int8_t>(r, t * H);
            r.ctxq = ws_alloc<int8_t>(r, t * m.qd);
            r.ffhq = ws_alloc<int8_t>(r, t * I);
            r.xs = ws_alloc<float>(r, t);
            r.ctxs = ws_alloc<float>(r, t);
            r.ffhs = ws_alloc<float>(r, t);
        }
        r.d_ids = ws_alloc<int64_t>(r, t);
        r.d_cu = ws_alloc<int32_t>(r, capS + 1);
        r.d_out = ws_alloc<float>(r, capO);
        r.d_status = ws_alloc<int>(r, 1);
        r.cap_T = static_cast<int>(t);
        ++r.ws_gen;
        r.cap_seq = capS;
        r.cap_out = static_cast<int>(capO);
        r.tm_T = -1;
    }
    if (r.tm_T != T) {
        const bool s8 = c->mode == RG_MODE_INT8_FULL;
        const bool f32 = c->mode == RG_MODE_FP32;
        const int eb = s8 ? 1 : (f32 ? 4 : 2);
        const void* xa = s8 ? static_cast<const void*>(r.xq) : (f32 ? static_cast<const void*>(r.xh) : r.xb);
        const void* ca = s8 ? static_cast<const void*>(r.ctxq) : (f32 ? static_cast<const void*>(r.ctxh) : r.ctx);
        const void* fa = s8 ? static_cast<const void*>(r.ffhq) : (f32 ? static_cast<const void*>(r.ffhh) : r.ffh);
        if (!rg::make_kmajor_tmap(&r.tm_x.m, xa, eb, T, H, H, 128) ||
            !rg::make_kmajor_tmap(&r.tm_ctx.m, ca, eb, T, m.qd, m.qd, 128) ||
            !rg::make_kmajor_tmap(&r.tm_ffh.m, fa, eb, T, I, I, 128))
            fail("cuTensorMapEncodeTiled failed for the activation buffers");
        if (f32 && (!rg::make_kmajor_tmap(&r.tm_x.lo, r.xl, 4, T, H, H, 128) ||
                    !rg::make_kmajor_tmap(&r.tm_ctx.lo, r.ctxl, 4, T, m.qd, m.qd, 128) ||
                    !rg::make_kmajor_tmap(&r.tm_ffh.lo, r.ffhl, 4, T, I, I, 128)))
            fail("cuTensorMapEncodeTiled failed for the activation remainder buffers");
        r.tm_T = T;
    }
}

// Grow one staging slot (which is not in flight) to hold a batch.
void ensure_host_staging(Replica& r, Replica::Staging& s, size_t nids, size_t ncu, size_t nout) {
    if (nids > s.cap_ids || ncu > s.cap_cu || nout > s.cap_out || !s.status) ++r.ws_gen;
    if (nids > s.cap_ids) {
        if (s.ids) cudaFreeHost(s.ids);
        s.ids = nullptr;
        check(cudaMallocHost(&s.ids, nids * sizeof(int64_t)), "cudaMallocHost");
        s.cap_ids = nids;
    }
    if (ncu > s.cap_cu) {
        if (s.cu) cudaFreeHost(s.cu);
        s.cu = nullptr;
        check(cudaMallocHost(&s.cu, ncu * sizeof(int32_t)), "cudaMallocHost");
        s.cap_cu = ncu;
    }
    if (nout > s.cap_out) {
        if (s.out) cudaFreeHost(s.out);
        s.out = nullptr;
        check(cudaMallocHost(&s.out, nout * sizeof(float)), "cudaMallocHost");
        s.cap_out = nout;
    }
    if (!s.status) check(cudaMallocHost(&s.status, sizeof(int)), "cudaMallocHost");
    if (!s.done) check(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming), "cudaEventCreate");
}

void free_staging(Replica& r) {
    for (auto& s : r.stage) {
        if (s.ids) cudaFreeHost(s.ids);
        if (s.cu) cudaFreeHost(s.cu);
        if (s.out) cudaFreeHost(s.out);
        if (s.status) cudaFreeHost(s.status);
        if (s.done) cudaEventDestroy(s.done);
        s = Replica::Staging{};
    }
}

size_t prof_event(Replica& r, cudaStream_t st) {
    if (r.ev_used == r.ev_pool.size()) {
        cudaEvent_t e;
        check(cudaEventCreate(&e), "cudaEventCreate");
        r.ev_pool.push_back(e);
    }
    const size_t i = r.ev_used++;
    check(cudaEventRecord(r.ev_pool[i], st), "cudaEventRecord");
    return i;
}

// Brackets one launch with events when profiling is on.
struct ProfScope {
    Replica& r;
    cudaStream_t st;
    int cls;
    double flops, bytes;
    size_t e0 = 0;
    ProfScope(Replica& r_, cudaStream_t st_, int cls_, double f, double b) : r(r_), st(st_), cls(cls_), flops(f), bytes(b) {
        if (r.prof) e0 = prof_event(r, st);
    }
    ~ProfScope() {
        if (r.prof) {
            const size_t e1 = prof_event(r, st);
            r.pending.push_back({cls, e0, e1, flops, bytes});
        }
    }
};

void prof_collect(Replica& r) {
    if (r.pending.empty()) return;
    check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    for (const auto& p : r.pending) {
        float ms = 0.f;
        check(cudaEventElapsedTime(&ms, r.ev_pool[p.e0], r.ev_pool[p.e1]), "cudaEventElapsedTime");
        r.st_ms[p.cls] += ms;
        r.st_flops[p.cls] += p.flops;
        r.st_bytes[p.cls] += p.bytes;
        r.st_n[p.cls] += 1;
    }
    r.pending.clear();
    r.ev_used = 0;
}

// Folded-LayerNorm plumbing of one GEMM (post-norm stacks, 16-bit modes):
// fold_stats = the (mean, rstd) of the A rows whose LayerNorm is folded into
// the weight; out16 / parts_out = a residual output's 16-bit copy and chunk
// statistics.
struct LnFold {
    const float2* fold_stats = nullptr;
    act16* out16 = nullptr;
    float2* parts_out = nullptr;
    const float* copy_gain = nullptr;  // out16 = round16(y * copy_gain) (weight-only int8)
};

// RoPE applied by the QKV GEMM's epilogue (kEpiRope).
struct QkRope {
    const float *cos = nullptr, *sin = nullptr;
    const int32_t* positions = nullptr;
    int dh = 0, qd = 0, kvd = 0;
    int npos = 0;  // rows of the tables, laid out [dh/8][npos][4]
    const float *q_norm = nullptr, *k_norm = nullptr;  // optional QK-norm before the rotation
    float eps = 0.f;
};

// Weight-only int8 at >= kW8WidenRows rows: the layer's four int8 weights
// widened to fp16 into the scratch in one launch before its first GEMM.
void widen_layer(Replica& r, const DevLayer& L, cudaStream_t st, int& launches) {
    const DevDense* ds[4] = {&L.qkv, &L.o, &L.ffn1, &L.ffn2};
    rg::WidenJob jobs[4];
    double bytes = 0.0;
    for (int i = 0; i < 4; ++i) {
        jobs[i].src = static_cast<const int8_t*>(ds[i]->w);
        jobs[i].n = static_cast<size_t>(ds[i]->N) * ds[i]->K;
        jobs[i].dst = r.w16 + ds[i]->w16_off;
        bytes += 3.0 * jobs[i].n;
    }
    ProfScope pw(r, st, RG_KC_QUANT, 0.0, bytes);
    check(rg::launch_widen_s8_f16_multi(jobs, 4, st), "widen launch");
    ++launches;
}

void gemm(Replica& r, int mode, const OpMaps& tmA, const DevDense& w, int M, int epi, const float* row_scale,
          const float* residual, void* out, cudaStream_t st, int& launches, const float2* ln_stats = nullptr,
          const float* ln_g = nullptr, const float* ln_b = nullptr, const LnFold* lf = nullptr,
          const QkRope* qr = nullptr) {
    rg::GemmArgs a{};
    if (qr) {  // the bias epilogue with RoPE per head
        epi = rg::kEpiRope;
        a.rope_cos = qr->cos;
        a.rope_sin = qr->sin;
        a.rope_npos = qr->npos;
        a.q_norm = qr->q_norm;
        a.k_norm = qr->k_norm;
        a.rope_eps = qr->eps;
        a.positions = qr->positions;
        a.rope_dh = qr->dh;
        a.rope_qd = qr->qd;
        a.rope_kvd = qr->kvd;
    }
    a.ln_stats = ln_stats;
    a.ln_g = ln_g;
    a.ln_b = ln_b;
    double fold_bytes = 0.0;
    if (lf) {
        if (lf->fold_stats) {
            if (!w.fold_c1) fail("folded GEMM without folded weights");
            a.fold_stats = lf->fold_stats;
            a.fold_c1 = w.fold_c1;
            fold_bytes += 8.0 * M;
        }
        a.out16 = reinterpret_cast<uint16_t*>(lf->out16);
        a.copy_gain = lf->copy_gain;
        a.ld16 = w.N;
        a.parts_out = lf->parts_out;
        if (lf->out16) fold_bytes += 2.0 * M * w.N;
        if (lf->parts_out) fold_bytes += 8.0 * M * (w.N / 32);
    }
    a.M = M;
    a.N = w.N;
    a.K = w.K;
    a.bias = lf && lf->fold_stats && w.fold_bias ? w.fold_bias : w.bias;
    a.col_scale = w.scale;
    a.row_scale = row_scale;
    a.residual = residual;
    a.out = out;
    a.ld_out = rg::epi_is_glu(epi) ? w.N / 2 : w.N;
    a.status = r.d_status;
    a.reverse_m = r.rev_m;
    const rg::GemmKind kind = mode == RG_MODE_INT8_FULL ? rg::GemmKind::kS8
                              : mode == RG_MODE_F16     ? rg::GemmKind::kF16
                              : mode == RG_MODE_INT8_W  ? rg::GemmKind::kW8
                                                        : rg::GemmKind::kBF16;
    // Algorithmic bytes: A and W read once, output written once (+ fp32
    // residual read); FLOPs 2*M*N*K.
    const bool x3 = mode == RG_MODE_FP32;  // hi + lo fp32 operands, fp32 outputs
    const double eb = kind == rg::GemmKind::kS8 ? 1.0 : (x3 ? 8.0 : 2.0);
    const double ob = (rg::epi_has_residual(epi) || epi == rg::kEpiBiasF32 || x3) ? 4.0
                      : (rg::epi_is_glu(epi) ? 1.0 : 2.0);
    const double bytes = eb * (double(M) * w.K + double(w.N) * w.K) + ob * double(M) * w.N +
                         (rg::epi_has_residual(epi) ? 4.0 * double(M) * w.N : 0.0) + fold_bytes;
    const int bn = rg::gemm_block_n(M, w.N, r.num_sms, rg::epi_is_glu(epi), qr ? qr->dh : 0);
    if (bn == 0) fail("no GEMM tile width divides N=%d", w.N);
    if (kind == rg::GemmKind::kW8 && M >= kW8WidenRows) {
        // the layer's weights were widened by widen_layer before its first GEMM
        ProfScope ps(r, st, RG_KC_GEMM, 2.0 * M * w.N * w.K, bytes);
        check(rg::gemm_launch(rg::GemmKind::kF16, epi, bn, tmA.m, w.tmap16[bn_index(bn)], a, r.num_sms, st),
              "gemm launch");
        ++launches;
        return;
    }
    ProfScope ps(r, st, RG_KC_GEMM, 2.0 * M * w.N * w.K, bytes);
    if (mode == RG_MODE_FP32) {
        const int i = bn_index(bn);
        check(rg::gemm_launch_tf32x3(epi, bn, tmA.m, tmA.lo, w.tmap[i], w.tmap_lo[i], a, r.num_sms, st),
              "gemm launch");
    } else {
        check(rg::gemm_launch(kind, epi, bn, tmA.m, w.tmap[bn_index(bn)], a, r.num_sms, st), "gemm launch");
    }
    ++launches;
}

// Allowed key offsets j - i of a layer's attention (see AttnParams).
void layer_window(const rg_model_desc& d, const DevLayer& L, int* lo, int* hi) {
    *lo = -(1 << 30);
    *hi = 1 << 30;
    if (d.arch == RG_ARCH_QWEN3) {
        *hi = 0;  // causal (qwen3.go:319-390)
    } else if (d.arch == RG_ARCH_MODERNBERT && !L.global) {
        *lo = -(d.local_attention / 2);  // |i - j| <= LocalAttention/2 (modernbert.go:268-274)
        *hi = d.local_attention / 2;
    } else if (d.arch == RG_ARCH_GEMMA3 && !L.global) {
        *lo = -(d.sliding_window - 1);  // |i - j| < SlidingWindow (gemma3.go:339-346)
        *hi = d.sliding_window - 1;
    }
}

// Number of (i, j) pairs in [0, L)^2 with lo <= j - i <= hi (lo <= 0 <= hi),
// summed over the batch: sum over offsets d of (L - |d|).
double attn_pairs(const int32_t* cu, int nseq, int lo, int hi) {
    double n = 0.0;
    if (!cu) return n;
    for (int s = 0; s < nseq; ++s) {
        const double L = cu[s + 1] - cu[s];
        if (L <= 0) continue;
        const double a = std::min<double>(-static_cast<double>(lo), L - 1), b = std::min<double>(hi, L - 1);
        auto S = [&](double k) { return (k + 1) * L - k * (k + 1) / 2; };  // sum_{d=0..k} (L - d)
        n += S(a) + S(b) - L;
    }
    return n;
}

// The forward over a batch already on the device (ids, cu in r.d_ids /
// r.d_cu or the caller's buffers): encodeWorkers and its per-arch variants
// (bert.go:740-923, qwen3.go:395-548, modernbert.go:148-311,
// gemma3.go:206-384, nomic.go:113-250), then ForwardWorkers' pooling, Dense
// head and L2 (bert.go:657-703).
void forward_on_device(rg_ctx* c, Replica& r, const int64_t* d_ids, const int32_t* d_cu, int nseq, int T,
                       int max_len, int out_kind, int out_dim, float* d_out, cudaStream_t st) {
    const rg_model_desc& d = c->d;
    const Dims m = dims(d);
    const int H = m.H, I = m.I, dh = m.dh, arch = d.arch;
    const float eps = d.layer_norm_eps == 0.f ? 1e-12f : d.layer_norm_eps;
    const int mode = c->mode;
    const bool s8 = mode == RG_MODE_INT8_FULL;
    const bool f16 = mode == RG_MODE_F16 || mode == RG_MODE_INT8_W;  // fp16 activations, else bf16
    const bool f32 = mode == RG_MODE_FP32;  // strict: fp32 activations, hi/lo GEMM operands
    const bool pre = is_prenorm(arch);
    const bool fold_post = !pre && r.fold;  // post-norm stacks fold their inner LayerNorms (see below)
    int launches = 0;
    const double Td = T, Hd = H;

    // ---- embeddings
    {
        ProfScope ps(r, st, RG_KC_NORM, 8.0 * Td * Hd, Td * (8.0 + 4.0 * Hd * 2 + 6.0 * Hd));
        rg::EmbedParams e{};
        e.ids = d_ids;
        e.cu = d_cu;
        e.nseq = nseq;
        e.T = T;
        e.H = H;
        e.vocab = d.vocab_size;
        e.pos_off = pos_offset(d);
        e.word = r.word;
        e.pos = r.pos;
        e.type0 = r.type0;
        e.scale = r.emb_scale;
        e.g = r.emb_g;
        e.b = arch == RG_ARCH_MODERNBERT ? r.zero_beta : r.emb_b;
        e.eps = eps;
        e.x32 = r.x32;
        e.xb = (pre || f32) ? nullptr : r.xb;  // pre-norm stacks normalise before the first GEMM
        e.f16 = f16;
        e.xhi = (!pre && f32) ? r.xh : nullptr;
        e.xlo = (!pre && f32) ? r.xl : nullptr;
        e.xq = (!pre && s8) ? r.xq : nullptr;
        e.xq_scale = (!pre && s8) ? r.xs : nullptr;
        e.status = r.d_status;
        e.pos_out = has_rope(arch) ? r.pos32 : nullptr;
        check(rg::launch_embed(e, st), "embed launch");
        ++launches;
    }
    // Norm of x32 into the next GEMM's A operand (bf16, or int8 + scales).
    auto norm_into_a = [&](const float* g, const float* b, bool rms) {
        ProfScope ps(r, st, RG_KC_NORM, 8.0 * Td * Hd, Td * Hd * (4.0 + 2.0 + (s8 ? 1.0 : 0.0)));
        rg::NormParams p{};
        p.in = r.x32;
        p.g = g;
        p.b = b;
        p.eps = eps;
        p.T = T;
        p.H = H;
        p.outb = f32 ? nullptr : r.xb;
        p.outhi = f32 ? r.xh : nullptr;
        p.outlo = f32 ? r.xl : nullptr;
        p.f16 = f16;
        p.status = r.d_status;
        p.outq = s8 ? r.xq : nullptr;
        p.outqs = s8 ? r.xs : nullptr;
        check(rg::launch_norm(p, rms, st), "norm launch");  // g nullptr: identity
        ++launches;
    };
    // Post-norm stacks keep one fp32 buffer x32: a residual GEMM adds its
    // sublayer output in place, and the LayerNorm after it writes only the
    // next GEMM's A operand plus the row's (mean, rstd); the next residual
    // GEMM rebuilds LN(x32) on load (kEpiBiasResLN).  res_g / res_b are the
    // gain and bias of that pending LayerNorm (nullptr: x32 is the residual
    // as is, i.e. the embedding output).  The stack's last LayerNorm writes
    // x32 for pooling.
    //
    // With r.fold the inner LayerNorms run no normalisation kernel: the
    // residual GEMM also writes its output's 16-bit copy (xb) and 32-column
    // chunk statistics (r.parts), merge_row_stats turns those into lnst, the
    // consumer GEMM (QKV, FFN1) folds the norm into its weight and epilogue,
    // and the next residual GEMM rebuilds LN(x32) from lnst as before.
    const float *res_g = nullptr, *res_b = nullptr;
    bool folded = false;  // xb holds the unnormalised rows of the pending (folded) norm
    auto residual_gemm = [&](const OpMaps& tmA, const DevDense& w, const float* row_scale, bool fold_out,
                             const float* next_g = nullptr) {
        LnFold lf;
        lf.out16 = fold_out ? r.xb : nullptr;
        lf.parts_out = fold_out ? r.parts : nullptr;
        // weight-only int8: the next norm's gain goes into the copy
        lf.copy_gain = fold_out && r.fold_w8 ? next_g : nullptr;
        const LnFold* lfp = fold_out ? &lf : nullptr;
        if (res_g)
            gemm(r, mode, tmA, w, T, rg::kEpiBiasResLN, row_scale, r.x32, r.x32, st, launches, r.lnst, res_g, res_b,
                 lfp);
        else
            gemm(r, mode, tmA, w, T, rg::kEpiBiasRes, row_scale, r.x32, r.x32, st, launches, nullptr, nullptr,
                 nullptr, lfp);
    };
    // The folded form of post_norm (not the stack's last): the chunk
    // statistics merged into lnst; the norm (g, b) becomes the pending one.
    auto fold_norm = [&](const float* g, const float* b) {
        {
            ProfScope ps(r, st, RG_KC_NORM, 4.0 * Td * (H / 32), Td * (8.0 * (H / 32) + 8.0));
            check(rg::launch_merge_row_stats(r.parts, H / 32, T, eps, r.lnst, st), "merge_row_stats launch");
            ++launches;
        }
        res_g = g;
        res_b = b;
        folded = true;
    };
    // Pre-norm stacks: the residual GEMM adds in place on x32 and writes
    // the stream's 16-bit copy and chunk statistics; the merge gives the
    // next (folded) norm's per-row statistics.
    auto pre_residual_fold = [&](const OpMaps& tmA, const DevDense& w) {
        LnFold lf;
        lf.out16 = r.xb;
        lf.parts_out = r.parts;
        gemm(r, mode, tmA, w, T, rg::kEpiBiasRes, nullptr, r.x32, r.x32, st, launches, nullptr, nullptr, nullptr, &lf);
        ProfScope ps(r, st, RG_KC_NORM, 4.0 * Td * (H / 32), Td * (8.0 * (H / 32) + 8.0));
        check(rg::launch_merge_row_stats(r.parts, H / 32, T, eps, r.lnst, st, r.fold_rms), "merge_row_stats launch");
        ++launches;
        folded = true;
    };
    // A GEMM reading xb: LN(y) folded into it when the last norm was folded.
    auto input_gemm = [&](const DevDense& w, const OpMaps& tmA, int epi, void* out, const QkRope* qr = nullptr) {
        if (folded) {
            LnFold lf;
            lf.fold_stats = r.lnst;
            gemm(r, mode, tmA, w, T, epi, nullptr, nullptr, out, st, launches, nullptr, nullptr, nullptr, &lf, qr);
        } else {
            gemm(r, mode, tmA, w, T, epi, s8 ? r.xs : nullptr, nullptr, out, st, launches, nullptr, nullptr, nullptr,
                 nullptr, qr);
        }
    };
    // RoPE (and the QK-norm of Qwen3 and Gemma, as a first pass over each
    // head) in the QKV projection's epilogue where a tile holds whole heads
    // (head dims 64 and 128 in each half-warp's columns, 256 across the
    // tile; 16-bit outputs); the strict fp32 mode keeps the separate
    // kernel.
    const bool rope_in_gemm = has_rope(arch) && !f32 && dh % 64 == 0 &&
                              rg::gemm_block_n(T, m.nqkv, r.num_sms, false, dh) != 0;
    auto post_norm = [&](const float* g, const float* b, bool last) {
        ProfScope ps(r, st, RG_KC_NORM, 8.0 * Td * Hd, Td * Hd * (4.0 + 2.0 + (s8 ? 1.0 : 0.0) + (last ? 4.0 : 0.0)));
        rg::NormParams p{};
        p.in = r.x32;
        p.g = g;
        p.b = b;
        p.eps = eps;
        p.T = T;
        p.H = H;
        p.out32 = last ? r.x32 : nullptr;
        p.outb = f32 ? nullptr : r.xb;
        p.outhi = f32 ? r.xh : nullptr;
        p.outlo = f32 ? r.xl : nullptr;
        p.f16 = f16;
        p.outq = s8 ? r.xq : nullptr;
        p.outqs = s8 ? r.xs : nullptr;
        p.status = r.d_status;
        p.stats = last ? nullptr : r.lnst;
        check(rg::launch_norm(p, false, st), "ln launch");
        ++launches;
        res_g = last ? nullptr : g;
        res_b = last ? nullptr : b;
        folded = false;
    };
    // Pooled output with CLS / last-token pooling: only each sequence's
    // pooled row reaches the output, so the stack's final norm runs on
    // those rows alone (the same per-row arithmetic) into pick32.
    const bool pick = out_kind == RG_OUT_POOLED && (d.pooling == 1 || d.pooling == 2);
    auto picked_norm = [&](const float* g, const float* b, bool rms) {
        ProfScope ps(r, st, RG_KC_NORM, 8.0 * nseq * Hd, nseq * Hd * 8.0);
        rg::NormParams p{};
        p.in = r.x32;
        p.g = g;
        p.b = b;
        p.eps = eps;
        p.T = nseq;
        p.H = H;
        p.out32 = r.pick32;
        p.row_cu = d_cu;
        p.row_pick = d.pooling;
        p.in_rows = T;
        check(rg::launch_norm(p, rms, st), "final norm launch");
        ++launches;
    };
    auto quantize = [&](const act16* x, int K, int8_t* q, float* sc) {  // bf16 rows (full-int8 mode)
        ProfScope ps(r, st, RG_KC_QUANT, 0.0, Td * K * 3.0);
        check(rg::launch_quantize_rows(reinterpret_cast<const __nv_bfloat16*>(x), T, K, q, sc, st),
              "quantize launch");
        ++launches;
    };
    const float scale = static_cast<float>(
        1.0 / std::sqrt(static_cast<double>(arch == RG_ARCH_GEMMA3 ? d.query_pre_attn_scalar : dh)));
    const int glu_epi = arch == RG_ARCH_MODERNBERT ? rg::kEpiGluGeluErf
                        : arch == RG_ARCH_GEMMA3   ? rg::kEpiGluGeluTanh
                                                   : rg::kEpiGluSilu;

    // Gemma: each post-norm residual add also applies the norm that reads
    // the residual stream next (the pre-FFN norm; the next layer's input
    // norm), writing the next GEMM's A operand as norm_into_a would.
    const bool gemma = arch == RG_ARCH_GEMMA3;
    auto add_post_norm = [&](const float* post_g, const float* next_g) {
        const double out_b = next_g ? (f32 ? 8.0 : 2.0) + (s8 ? 1.0 : 0.0) : 0.0;
        ProfScope ps(r, st, RG_KC_NORM, 8.0 * Td * Hd * (next_g ? 2.0 : 1.0), Td * Hd * (12.0 + out_b));
        rg::NormParams nx{};
        if (next_g) {
            nx.g = next_g;
            nx.eps = eps;
            nx.outb = f32 ? nullptr : r.xb;
            nx.outhi = f32 ? r.xh : nullptr;
            nx.outlo = f32 ? r.xl : nullptr;
            nx.f16 = f16;
            nx.status = r.d_status;
            nx.outq = s8 ? r.xq : nullptr;
            nx.outqs = s8 ? r.xs : nullptr;
        }
        check(rg::launch_add_rmsnorm(r.x32, r.y32, post_g, eps, T, H, st, next_g ? &nx : nullptr),
              "add_rmsnorm launch");
        ++launches;
    };

    for (int li = 0; li < d.num_hidden_layers; ++li) {
        const DevLayer& L = r.layers[li];
        if (mode == RG_MODE_INT8_W && T >= kW8WidenRows) widen_layer(r, L, st, launches);
        // ---- attention sublayer
        // (a folded pre-norm stack enters layers 1... with the norm's
        // statistics already merged by the previous FFN's residual GEMM;
        // Gemma's layers 1... with the input norm applied by the previous
        // layer's last residual add)
        if (pre && !(r.fold && li > 0) && !(gemma && li > 0)) {
            norm_into_a(L.attn_norm, arch == RG_ARCH_MODERNBERT ? r.zero_beta : nullptr, arch != RG_ARCH_MODERNBERT);
            folded = false;
        }
        if (rope_in_gemm) {
            QkRope qr;
            qr.cos = L.global ? r.cos4_g : r.cos4_l;
            qr.sin = L.global ? r.sin4_g : r.sin4_l;
            qr.npos = r.rope_npos;
            qr.positions = r.pos32;
            qr.dh = dh;
            qr.qd = m.qd;
            qr.kvd = m.kvd;
            qr.q_norm = L.q_norm;
            qr.k_norm = L.k_norm;
            qr.eps = eps;
            input_gemm(L.qkv, r.tm_x, rg::kEpiBias, r.qkv, &qr);
        } else {
            input_gemm(L.qkv, r.tm_x, rg::kEpiBias, f32 ? static_cast<void*>(r.qkv32) : r.qkv);
        }
        if (has_rope(arch) && !rope_in_gemm) {
            ProfScope ps(r, st, RG_KC_NORM, 0.0, Td * (m.qd + m.kvd) * 4.0);
            rg::QkRopeParams q{};
            q.qkv = r.qkv;
            q.qkv32 = f32 ? r.qkv32 : nullptr;
            q.f16 = f16;
            q.status = r.d_status;
            q.ld = m.nqkv;
            q.T = T;
            q.nq = m.nq;
            q.nkv = m.nkv;
            q.q_norm = L.q_norm;
            q.k_norm = L.k_norm;
            q.eps = eps;
            q.cos = L.global ? r.cos_g : r.cos_l;
            q.sin = L.global ? r.sin_g : r.sin_l;
            q.cu = d_cu;
            q.nseq = nseq;
            check(rg::launch_qk_norm_rope(q, dh, st), "qk norm/rope launch");
            ++launches;
        }
        {
            int lo, hi;
            layer_window(d, L, &lo, &hi);
            const double pairs = attn_pairs(r.h_cu_view, nseq, lo, hi);
            ProfScope ps(r, st, RG_KC_ATTENTION, 4.0 * dh * pairs * m.nq,
                         2.0 * Td * (2.0 * m.qd + 2.0 * m.kvd));
            if (f32) {
                rg::AttnF32Params fp{};
                fp.q = r.qkv32;
                fp.k = r.qkv32 + m.qd;
                fp.v = r.qkv32 + m.qd + m.kvd;
                fp.ldq = fp.ldk = fp.ldv = m.nqkv;
                fp.cu = d_cu;
                fp.group = m.nq / m.nkv;
                fp.scale = scale;
                fp.rel_lo = lo;
                fp.rel_hi = hi;
                fp.bias = r.rel_bias;
                fp.bias_off = r.rel_bias_off;
                fp.out_hi = r.ctxh;
                fp.out_lo = r.ctxl;
                fp.ldo = m.qd;
                check(rg::launch_attention_f32(fp, nseq, max_len, m.nq, dh, st), "attention launch");
            } else {
                rg::AttnParams ap{};
                ap.q = r.qkv;
                ap.k = r.qkv + m.qd;
                ap.v = r.qkv + m.qd + m.kvd;
                ap.ldq = ap.ldk = ap.ldv = m.nqkv;
                ap.f16 = f16;
                ap.cu = d_cu;
                ap.group = m.nq / m.nkv;
                ap.scale = scale;
                ap.scale_log2 = scale * 1.4426950408889634f;
                ap.rel_lo = lo;
                ap.rel_hi = hi;
                ap.bias = r.rel_bias;
                ap.bias_off = r.rel_bias_off;
                ap.out = r.ctx;
                ap.ldo = m.qd;
                ap.T = T;
                ap.kv_heads = m.nkv;
                ap.status = r.d_status;
                // L2-aware order: the QKV GEMM wrote the last sequences'
                // rows last, so they are the ones still in the 126 MB L2
                ap.reverse = 1;
                check(rg::launch_attention(ap, nseq, max_len, m.nq, dh, st), "attention launch");
            }
            ++launches;
        }
        if (s8) quantize(r.ctx, m.qd, r.ctxq, r.ctxs);
        if (fold_post) {
            residual_gemm(r.tm_ctx, L.o, nullptr, true, L.ln1_g);
            fold_norm(L.ln1_g, L.ln1_b);
        } else if (!pre) {
            residual_gemm(r.tm_ctx, L.o, s8 ? r.ctxs : nullptr, false);
            post_norm(L.ln1_g, L.ln1_b, false);
        } else if (gemma) {
            gemm(r, mode, r.tm_ctx, L.o, T, rg::kEpiBiasF32, s8 ? r.ctxs : nullptr, nullptr, r.y32, st, launches);
            add_post_norm(L.post_attn, L.ffn_norm);
        } else if (r.fold) {  // residual in place + the folded FFN norm's statistics
            pre_residual_fold(r.tm_ctx, L.o);
        } else {  // residual added in place on x32
            gemm(r, mode, r.tm_ctx, L.o, T, rg::kEpiBiasRes, s8 ? r.ctxs : nullptr, r.x32, r.x32, st, launches);
        }
        // ---- FFN sublayer
        if (pre && !r.fold && !gemma)
            norm_into_a(L.ffn_norm, arch == RG_ARCH_MODERNBERT ? r.zero_beta : nullptr, arch != RG_ARCH_MODERNBERT);
        input_gemm(L.ffn1, r.tm_x, is_glu(arch) ? glu_epi : rg::kEpiBiasGelu,
                   f32 ? static_cast<void*>(r.ffhh) : r.ffh);
        if (f32) {  // the fp32 FFN hidden state -> tf32 hi (in place) + remainder
            ProfScope ps(r, st, RG_KC_QUANT, 0.0, Td * I * 12.0);
            check(rg::launch_split_tf32(r.ffhh, static_cast<size_t>(T) * I, r.ffhh, r.ffhl, st), "split launch");
            ++launches;
        }
        if (s8) quantize(r.ffh, I, r.ffhq, r.ffhs);
        const bool last = li == d.num_hidden_layers - 1;
        // FFN2 reads the FFN hidden state (4x the hidden width) that FFN1
        // just wrote in row-block order: last block first finds it in L2
        r.rev_m = 1;
        if (fold_post && !last) {
            residual_gemm(r.tm_ffh, L.ffn2, nullptr, true, L.ln2_g);
            fold_norm(L.ln2_g, L.ln2_b);
        } else if (!pre && last && pick) {
            residual_gemm(r.tm_ffh, L.ffn2, s8 ? r.ffhs : nullptr, false);
            picked_norm(L.ln2_g, L.ln2_b, false);
        } else if (!pre) {
            residual_gemm(r.tm_ffh, L.ffn2, s8 ? r.ffhs : nullptr, false);
            post_norm(L.ln2_g, L.ln2_b, last);
        } else if (gemma) {
            gemm(r, mode, r.tm_ffh, L.ffn2, T, rg::kEpiBiasF32, s8 ? r.ffhs : nullptr, nullptr, r.y32, st, launches);
            add_post_norm(L.post_ffn, last ? nullptr : r.layers[li + 1].attn_norm);
        } else {
            if (r.fold && !last)
                pre_residual_fold(r.tm_ffh, L.ffn2);
            else
                gemm(r, mode, r.tm_ffh, L.ffn2, T, rg::kEpiBiasRes, s8 ? r.ffhs : nullptr, r.x32, r.x32, st,
                     launches);
        }
        r.rev_m = 0;
    }
    if (r.final_norm && pick) {
        picked_norm(r.final_norm, arch == RG_ARCH_MODERNBERT ? r.zero_beta : nullptr, arch != RG_ARCH_MODERNBERT);
    } else if (r.final_norm) {  // qwen3.go:544, gemma3.go:380, modernbert.go:307
        ProfScope ps(r, st, RG_KC_NORM, 8.0 * Td * Hd, Td * Hd * 8.0);
        rg::NormParams p{};
        p.in = r.x32;
        p.g = r.final_norm;
        p.b = arch == RG_ARCH_MODERNBERT ? r.zero_beta : nullptr;
        p.eps = eps;
        p.T = T;
        p.H = H;
        p.out32 = r.x32;
        check(rg::launch_norm(p, arch != RG_ARCH_MODERNBERT, st), "final norm launch");
        ++launches;
    }
    if (out_kind == RG_OUT_POOLED) {
        const double rows = d.pooling == 0 ? Td : double(nseq);
        const double head_flops = r.dense1 ? 4.0 * double(nseq) * Hd * d.dense_hidden : 0.0;
        const double head_bytes = r.dense1 ? 8.0 * Hd * d.dense_hidden : 0.0;
        ProfScope ps(r, st, RG_KC_POOL, rows * Hd + head_flops, 4.0 * (rows * Hd + double(nseq) * out_dim) + head_bytes);
        // With the final norm applied to the pooled rows only (pick32), the
        // pool reads those rows as one-row sequences.
        const float* src = pick ? r.pick32 : r.x32;
        const int32_t* src_cu = pick ? r.iota : d_cu;
        const int pooling = pick ? 1 : d.pooling;
        if (r.dense1) {
            // pool, Dense head H -> D -> H (fp32), L2 and truncate in one
            // launch (gemma3.go:177-198)
            check(rg::launch_pool_head(src, src_cu, nseq, H, d.dense_hidden, pooling, r.dense1, r.dense2, d.normalize,
                                       out_dim, d_out, st),
                  "pool/head launch");
            ++launches;
        } else if (pooling == 0 && H % 8 == 0) {
            // mean pooling over whole sequences: rows spread over clusters
            check(rg::launch_pool_head(src, src_cu, nseq, H, 0, 0, nullptr, nullptr, d.normalize, out_dim, d_out, st),
                  "pool launch");
            ++launches;
        } else {
            check(rg::launch_pool(src, src_cu, nseq, H, pooling, d.normalize, out_dim, d_out, st), "pool launch");
            ++launches;
        }
    } else {
        check(cudaMemcpyAsync(d_out, r.x32, sizeof(float) * static_cast<size_t>(T) * H, cudaMemcpyDeviceToDevice,
                              st),
              "cudaMemcpyAsync D2D");
    }
    r.last_launches = launches;
}

std::string status_message(int s) {
    std::string m;
    if (s & rg::kStatusBadToken) m += "token id out of vocab range; ";
    if (s & rg::kStatusWaitTimeout) m += "a device pipeline wait timed out; ";
    if (s & rg::kStatusBadShape) m += "inconsistent shape on the device; ";
    if (s & rg::kStatusF16Overflow) m += "an activation overflowed the fp16 range (use the bf16 mode); ";
    if (m.empty()) m = "device error status " + std::to_string(s);
    return m;
}

// Validate a host batch exactly as encodeWorkers does, in sequence order
// (bert.go:742-747, 797-799); the first failing text is reported.
void validate_batch(const rg_model_desc& d, const int64_t* ids, const int32_t* cu, int nseq) {
    if (cu[0] != 0) fail("cu_seqlens[0] must be 0 (got %d)", cu[0]);
    const int maxlen = max_seq_len(d);
    for (int i = 0; i < nseq; ++i) {
        const int len = cu[i + 1] - cu[i];
        if (len < 0) fail("cu_seqlens must be non-decreasing (text %d)", i);
        if (len == 0) fail("rembed: text %d: empty token sequence", i);
        if (len > maxlen) fail("rembed: text %d: sequence length %d exceeds the model's maximum %d", i, len, maxlen);
        for (int t = cu[i]; t < cu[i + 1]; ++t)
            if (ids[t] < 0 || ids[t] >= d.vocab_size)
                fail("rembed: text %d: token id %lld out of vocab range %d", i, static_cast<long long>(ids[t]),
                     d.vocab_size);
    }
}

// Run sequences [s_lo, s_hi) of a host batch on replica r.
void drop_graphs(Replica& r) {
    for (auto& g : r.graphs) cudaGraphExecDestroy(g.second);
    r.graphs.clear();
    r.seen_once.clear();
}

// Run `enqueue` (the stream work of one forward) on st: eagerly the first
// time a key is seen, captured into a graph the second time, replayed from
// then on.  Profiling runs stay eager (their events time every launch).
template <typename F>
void run_graphed(Replica& r, cudaStream_t st, const Replica::GraphKey& key, F&& enqueue) {
    if (r.prof) {
        enqueue();
        return;
    }
    for (auto& g : r.graphs)
        if (g.first == key) {
            check(cudaGraphLaunch(g.second, st), "cudaGraphLaunch");
            r.last_launches = r.graph_launches;
            return;
        }
    // graphs of retired buffers go before a new one is made
    bool stale = false;
    for (auto& g : r.graphs) stale |= g.first.gen != key.gen;
    if (stale) drop_graphs(r);
    bool seen = false;
    for (auto& k : r.seen_once) seen |= k == key;
    if (!seen) {
        if (r.seen_once.size() >= 16) r.seen_once.erase(r.seen_once.begin());
        r.seen_once.push_back(key);
        enqueue();
        return;
    }
    if (r.graphs.size() >= 16) {
        cudaGraphExecDestroy(r.graphs.front().second);
        r.graphs.erase(r.graphs.begin());
    }
    check(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    try {
        enqueue();
    } catch (...) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(st, &g);  // leave the stream usable
        if (g) cudaGraphDestroy(g);
        throw;
    }
    cudaGraph_t g = nullptr;
    check(cudaStreamEndCapture(st, &g), "cudaStreamEndCapture");
    cudaGraphExec_t ge = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    check(e, "cudaGraphInstantiate");
    r.graphs.push_back({key, ge});
    r.graph_launches = r.last_launches;
    check(cudaGraphLaunch(ge, st), "cudaGraphLaunch");
}

// Stage the sequences `seqs` (ascending indices into a host batch) in
// staging slot `slot` of replica r, packed in that order, and enqueue pinned
// H2D -> forward -> D2H on its stream (a graph per repeated shape); each
// sequence's result is copied to its own place in host_out at collect time.
void submit_shard(rg_ctx* c, Replica& r, int slot, const int64_t* ids, const int32_t* cu, const std::vector<int>& seqs,
                  int out_kind, int out_dim, float* host_out) {
    std::lock_guard<std::mutex> lk(r.mu);
    check(cudaSetDevice(r.device), "cudaSetDevice");
    const int nseq = static_cast<int>(seqs.size());
    if (nseq <= 0) return;
    Replica::Staging& sg = r.stage[slot];
    if (sg.busy) fail("rembed: staging slot %d is still in flight (collect the oldest submission first)", slot);
    int T = 0;
    for (int s : seqs) T += cu[s + 1] - cu[s];
    const int H = c->d.hidden_size;
    const size_t nout = out_kind == RG_OUT_POOLED ? static_cast<size_t>(nseq) * out_dim : static_cast<size_t>(T) * H;
    ensure_workspace(c, r, T, nseq, nout);
    if (c->inject_alloc) {
        c->inject_alloc = false;
        fail("cudaMallocHost: out of memory (injected failure of the host staging allocation)");
    }
    ensure_host_staging(r, sg, T, nseq + 1, nout);
    // pack the sequences; runs of consecutive sequences copy in one piece
    const size_t row = out_kind == RG_OUT_POOLED ? static_cast<size_t>(out_dim) : static_cast<size_t>(H);
    sg.copies.clear();
    int max_len = 0, t = 0;
    sg.cu[0] = 0;
    for (int i = 0; i < nseq;) {
        int j = i + 1;
        while (j < nseq && seqs[j] == seqs[j - 1] + 1) ++j;
        const int a = seqs[i], b = seqs[j - 1] + 1;  // global sequences [a, b)
        const int n_tok = cu[b] - cu[a];
        memcpy(sg.ids + t, ids + cu[a], sizeof(int64_t) * n_tok);
        for (int k = i; k < j; ++k) {
            const int len = cu[seqs[k] + 1] - cu[seqs[k]];
            sg.cu[k + 1] = sg.cu[k] + len;
            max_len = std::max(max_len, len);
        }
        if (out_kind == RG_OUT_POOLED)
            sg.copies.push_back({static_cast<size_t>(a) * row, static_cast<size_t>(i) * row,
                                 static_cast<size_t>(j - i) * row});
        else
            sg.copies.push_back({static_cast<size_t>(cu[a]) * row, static_cast<size_t>(t) * row,
                                 static_cast<size_t>(n_tok) * row});
        t += n_tok;
        i = j;
    }
    cudaStream_t st = r.stream;
    r.h_cu_view = sg.cu;
    // pinned staging -> device, the forward, device -> pinned staging: one
    // graph per shape and slot once the shape repeats
    const Replica::GraphKey key{T, nseq, max_len, out_kind, out_dim, sg.ids, sg.cu, sg.out, r.ws_gen};
    run_graphed(r, st, key, [&] {
        check(cudaMemsetAsync(r.d_status, 0, sizeof(int), st), "cudaMemsetAsync");
        check(cudaMemcpyAsync(r.d_ids, sg.ids, sizeof(int64_t) * T, cudaMemcpyHostToDevice, st), "H2D ids");
        check(cudaMemcpyAsync(r.d_cu, sg.cu, sizeof(int32_t) * (nseq + 1), cudaMemcpyHostToDevice, st), "H2D cu");
        forward_on_device(c, r, r.d_ids, r.d_cu, nseq, T, max_len, out_kind, out_dim, r.d_out, st);
        check(cudaMemcpyAsync(sg.out, r.d_out, sizeof(float) * nout, cudaMemcpyDeviceToHost, st), "D2H out");
        check(cudaMemcpyAsync(sg.status, r.d_status, sizeof(int), cudaMemcpyDeviceToHost, st), "D2H status");
    });
    r.h_cu_view = nullptr;
    check(cudaEventRecord(sg.done, st), "cudaEventRecord");
    sg.busy = true;
    sg.user_out = host_out;
}

// Wait for replica r's slot and copy its result out (no-op if idle).
void collect_shard(Replica& r, int slot) {
    std::lock_guard<std::mutex> lk(r.mu);
    Replica::Staging& sg = r.stage[slot];
    if (!sg.busy) return;
    check(cudaSetDevice(r.device), "cudaSetDevice");
    sg.busy = false;
    check(cudaEventSynchronize(sg.done), "forward");
    if (*sg.status != 0) fail("rembed: %s", status_message(*sg.status).c_str());
    for (const auto& cp : sg.copies) memcpy(sg.user_out + cp[0], sg.out + cp[1], sizeof(float) * cp[2]);
}

// Estimated FLOPs of one sequence of length L through the whole stack: the
// dense projections of every layer (fused Q|K|V with grouped K/V heads, the
// output projection, a gated FFN at twice its intermediate width) and each
// layer's attention over the (query, key) pairs its mask allows (causal or
// windowed layers see fewer), plus the Gemma Dense head.
double seq_cost(const rg_model_desc& d, const std::vector<DevLayer>& layers, int L) {
    const Dims m = dims(d);
    const double H = m.H, I = m.I;
    const double lin = 2.0 * L * (H * m.nqkv + m.qd * H + H * I * (is_glu(d.arch) ? 2.0 : 1.0) + I * H);
    double cost = lin * d.num_hidden_layers;
    const int32_t one[2] = {0, L};
    for (const DevLayer& ly : layers) {
        int lo, hi;
        layer_window(d, ly, &lo, &hi);
        cost += 4.0 * m.dh * m.nq * attn_pairs(one, 1, lo, hi);
    }
    if (d.arch == RG_ARCH_GEMMA3) cost += 4.0 * H * d.dense_hidden;
    return cost;
}

// Sequences over replicas by the greedy longest-processing-time rule: in
// order of decreasing estimated cost (ties: lower index first), each to the
// replica with the smallest total so far (ties: lower replica).  Each
// replica's list is returned in ascending sequence order.  Every sequence's
// output is independent of which replica runs it and of its batch mates, so
// any assignment gives the same embeddings bit for bit.
std::vector<std::vector<int>> lpt_assign(const rg_model_desc& d, const std::vector<DevLayer>& layers,
                                         const int32_t* cu, int nseq, int nrep) {
    std::vector<std::vector<int>> out(nrep);
    if (nrep == 1) {
        out[0].resize(nseq);
        for (int i = 0; i < nseq; ++i) out[0][i] = i;
        return out;
    }
    std::vector<std::pair<double, int>> order(nseq);
    std::map<int, double> by_len;  // cost of each distinct length, computed once
    for (int i = 0; i < nseq; ++i) {
        const int L = cu[i + 1] - cu[i];
        auto it = by_len.find(L);
        if (it == by_len.end()) it = by_len.emplace(L, seq_cost(d, layers, L)).first;
        order[i] = {it->second, i};
    }
    std::stable_sort(order.begin(), order.end(),
                     [](const std::pair<double, int>& a, const std::pair<double, int>& b) { return a.first > b.first; });
    std::vector<double> load(nrep, 0.0);
    for (const auto& o : order) {
        const int k = static_cast<int>(std::min_element(load.begin(), load.end()) - load.begin());
        load[k] += o.first;
        out[k].push_back(o.second);
    }
    for (auto& v : out) std::sort(v.begin(), v.end());
    return out;
}

// Submit a validated host batch: split over the replicas (lpt_assign) and
// staged in slot ticket % 2 of each.
// wait_for_slot: the synchronous rg_forward waits for another thread to
// collect the slot it needs; rg_submit (whose caller may hold both
// outstanding tickets itself) reports the limit instead.
int64_t submit_batch(rg_ctx* c, const int64_t* ids, const int32_t* cu, int nseq, int out_kind, int out_dim,
                     float* host_out, bool wait_for_slot) {
    std::unique_lock<std::mutex> tl(c->tmu);
    while (c->pending[c->next_ticket & 1] != kSlotFree) {
        if (!wait_for_slot) {
            const int64_t p = c->pending[c->next_ticket & 1];
            if (p >= 0)
                fail("rembed: two submissions are outstanding; collect ticket %lld first", static_cast<long long>(p));
            fail("rembed: staging slot %d is still being collected", static_cast<int>(c->next_ticket & 1));
        }
        c->tcv.wait(tl);
    }
    const int64_t t = c->next_ticket;
    const int slot = static_cast<int>(t & 1);
    const int nrep = static_cast<int>(c->reps.size());
    const std::vector<std::vector<int>> parts = lpt_assign(c->d, c->reps[0]->layers, cu, nseq, nrep);
    int k = 0;
    try {
        for (; k < nrep; ++k) {
            if (c->inject_replica == k) {
                c->inject_replica = -1;
                fail("rembed: the worker of device %d failed (injected)", c->reps[k]->device);
            }
            submit_shard(c, *c->reps[k], slot, ids, cu, parts[k], out_kind, out_dim, host_out);
        }
    } catch (...) {
        for (int j = 0; j < k; ++j) {  // the shards already in flight finish before the slot is reused
            try {
                collect_shard(*c->reps[j], slot);
            } catch (...) {
            }
        }
        throw;
    }
    c->pending[slot] = t;
    c->next_ticket = t + 1;
    return t;
}

// Wait for a submitted batch and copy its results to the caller's buffer.
void collect_batch(rg_ctx* c, int64_t t) {
    const int slot = static_cast<int>(t & 1);
    {
        std::lock_guard<std::mutex> tl(c->tmu);
        if (t < 0 || c->pending[slot] != t) fail("rembed: ticket %lld is not outstanding", static_cast<long long>(t));
        c->pending[slot] = kSlotCollecting;  // no second collect; no submission into the slot yet
    }
    std::string first;
    for (Replica* r : c->reps) {
        try {
            collect_shard(*r, slot);
        } catch (const Error& e) {
            if (first.empty()) first = e.msg;
        }
    }
    {
        std::lock_guard<std::mutex> tl(c->tmu);
        c->pending[slot] = kSlotFree;  // the slot's staging buffers are idle again
    }
    c->tcv.notify_all();
    if (!first.empty()) fail("%s", first.c_str());
}

}  // namespace

// ===========================================================================
extern "C" {

int rg_init(const rg_model_desc* desc, const int* devices, int ndev, int mode, rg_ctx** out, char** err) {
    try {
        if (!desc || !out) fail("rg_init: null argument");
        *out = nullptr;
        const rg_model_desc& d = *desc;
        if (d.arch < RG_ARCH_BERT || d.arch > RG_ARCH_NOMIC) fail("rg_init: unknown architecture %d", d.arch);
        if (d.hidden_size <= 0 || d.num_hidden_layers <= 0 || d.num_attention_heads <= 0 ||
            d.intermediate_size <= 0 || d.vocab_size <= 0 || d.max_position_embeddings <= 0)
            fail("rg_init: missing or non-positive architecture fields");
        if (d.hidden_size % d.num_attention_heads != 0)
            fail("rg_init: hidden_size %d not divisible by num_attention_heads %d", d.hidden_size,
                 d.num_attention_heads);
        const Dims dm = dims(d);
        const int dh = dm.dh;
        if (dh != 32 && dh != 64 && dh != 128 && dh != 256)
            fail("rg_init: head dim %d unsupported (32, 64, 128 or 256)", dh);
        if (dm.nkv <= 0 || dm.nq % dm.nkv != 0)
            fail("rg_init: num_attention_heads %d not divisible by num_key_value_heads %d", dm.nq, dm.nkv);
        if (d.arch == RG_ARCH_MODERNBERT && (d.global_attn_every_n_layers < 1 || d.local_attention < 2))
            fail("rg_init: modernbert needs global_attn_every_n_layers >= 1 and local_attention >= 2");
        if (d.arch == RG_ARCH_GEMMA3 &&
            (d.sliding_window < 1 || d.sliding_window_pattern < 1 || d.query_pre_attn_scalar < 1 || d.dense_hidden < 1))
            fail("rg_init: gemma3 needs sliding_window, sliding_window_pattern, query_pre_attn_scalar, dense_hidden");
        if (d.arch == RG_ARCH_GEMMA3 && d.dense_hidden % 8 != 0)
            fail("rg_init: gemma3 dense_hidden must be a multiple of 8 (got %d)", d.dense_hidden);
        if (is_glu(d.arch) && (d.intermediate_size % 64 != 0))
            fail("rg_init: gated FFN needs intermediate_size %% 64 == 0 (got %d)", d.intermediate_size);
        if (dm.nqkv % 128 != 0 || dm.qd % 64 != 0)
            fail("rg_init: fused q/k/v width %d must be a multiple of 128", dm.nqkv);
        if (d.hidden_size % 128 != 0 || d.intermediate_size % 128 != 0)
            fail("rg_init: hidden_size and intermediate_size must be multiples of 128 (got %d, %d)", d.hidden_size,
                 d.intermediate_size);
        if (d.pooling < 0 || d.pooling > 2) fail("rg_init: bad pooling %d", d.pooling);
        if (d.arch == RG_ARCH_MPNET && d.relative_attention_num_buckets < 2)
            fail("rg_init: mpnet needs relative_attention_num_buckets >= 2");
        if (max_seq_len(d) <= 0) fail("rg_init: no usable positions (max_position_embeddings %d, offset %d)",
                                      d.max_position_embeddings, pos_offset(d));
        if (mode != RG_MODE_BF16 && mode != RG_MODE_F16 && mode != RG_MODE_INT8_W && mode != RG_MODE_INT8_FULL &&
            mode != RG_MODE_FP32)
            fail("rg_init: mode %d is not available in this build", mode);
        if (mode == RG_MODE_INT8_FULL && (d.hidden_size % 128 != 0 || d.intermediate_size % 128 != 0 ||
                                          dims(d).qd % 128 != 0))
            fail("rg_init: full-int8 needs K multiples of 128");
        if (mode == RG_MODE_INT8_FULL && (d.intermediate_size > 4096 || dims(d).qd > 4096))
            fail("rg_init: full-int8 row quantisation supports widths up to 4096 (got %d, %d)", dims(d).qd,
                 d.intermediate_size);
        int ndevs = 0;
        check(cudaGetDeviceCount(&ndevs), "cudaGetDeviceCount");
        std::vector<int> devs;
        if (!devices || ndev <= 0) devs.push_back(0);
        else devs.assign(devices, devices + ndev);
        for (int dv : devs)
            if (dv < 0 || dv >= ndevs) fail("rg_init: device %d out of range (%d visible)", dv, ndevs);
        rg_ctx* c = new rg_ctx();
        c->d = d;
        c->mode = mode;
        c->devices = devs;
        for (int dv : devs) {
            Replica* r = new Replica();
            r->device = dv;
            c->reps.push_back(r);
            try {
                check(cudaSetDevice(dv), "cudaSetDevice");
                cudaDeviceProp prop;
                check(cudaGetDeviceProperties(&prop, dv), "cudaGetDeviceProperties");
                if (prop.major != 10)
                    fail("rg_init: device %d is sm_%d%d; this library is built for sm_100a", dv, prop.major,
                         prop.minor);
                r->num_sms = prop.multiProcessorCount;
                check(cudaStreamCreateWithFlags(&r->stream, cudaStreamNonBlocking), "cudaStreamCreate");
            } catch (...) {
                rg_free(c);
                throw;
            }
        }
        *out = c;
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_upload_weight(rg_ctx* c, const char* name, int dtype, const int64_t* shape, int ndim, const void* host,
                     char** err) {
    try {
        if (!c || !name || !host || (!shape && ndim > 0)) fail("rg_upload_weight: null argument");
        std::lock_guard<std::mutex> lk(c->mu);
        if (c->finalized) fail("rg_upload_weight: context already finalized");
        HostTensor t;
        int64_t n = 1;
        for (int i = 0; i < ndim; ++i) {
            if (shape[i] < 0) fail("rg_upload_weight: negative dimension in %s", name);
            t.shape.push_back(shape[i]);
            n *= shape[i];
        }
        t.data.resize(n);
        if (dtype == RG_DTYPE_F32) {
            memcpy(t.data.data(), host, sizeof(float) * n);
        } else if (dtype == RG_DTYPE_BF16) {
            const uint16_t* s = static_cast<const uint16_t*>(host);
            for (int64_t i = 0; i < n; ++i) {
                uint32_t u = static_cast<uint32_t>(s[i]) << 16;
                memcpy(&t.data[i], &u, 4);
            }
        } else if (dtype == RG_DTYPE_F16) {
            const __half* s = static_cast<const __half*>(host);
            for (int64_t i = 0; i < n; ++i) t.data[i] = __half2float(s[i]);
        } else {
            fail("rg_upload_weight: unknown dtype %d for %s", dtype, name);
        }
        c->host[name] = std::move(t);
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_finalize(rg_ctx* c, char** err) {
    try {
        if (!c) fail("rg_finalize: null context");
        std::lock_guard<std::mutex> lk(c->mu);
        if (c->finalized) return 0;
        for (Replica* r : c->reps) {
            if (is_bert_family(c->d.arch))
                finalize_bert(c, *r);
            else
                finalize_decoder(c, *r);
            if (c->mode == RG_MODE_INT8_W) make_widen_maps(*r);
        }
        c->host.clear();
        c->finalized = true;
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_forward(rg_ctx* c, const int64_t* ids, const int32_t* cu, int nseq, int out_kind, int out_dim,
               float* host_out, char** err) {
    try {
        if (!c) fail("rembed: invalid context");
        if (!c->finalized) fail("rembed: weights not finalized");
        if (nseq < 0) fail("rembed: negative text count");
        if (nseq == 0) return 0;
        if (!ids || !cu || !host_out) fail("rembed: null buffer");
        const int H = c->d.hidden_size;
        if (out_kind == RG_OUT_POOLED) {
            if (out_dim < 1 || out_dim > H) fail("rembed: WithDim(%d) out of range [1, %d]", out_dim, H);
        } else if (out_kind == RG_OUT_TOKENS) {
            if (out_dim != H) fail("rembed: token output needs out_dim == hidden (%d)", H);
        } else {
            fail("rembed: bad out_kind %d", out_kind);
        }
        validate_batch(c->d, ids, cu, nseq);
        const int64_t t = submit_batch(c, ids, cu, nseq, out_kind, out_dim, host_out, true);
        collect_batch(c, t);
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_submit(rg_ctx* c, const int64_t* ids, const int32_t* cu, int nseq, int out_kind, int out_dim, float* host_out,
              int64_t* ticket, char** err) {
    try {
        if (!c) fail("rembed: invalid context");
        if (!c->finalized) fail("rembed: weights not finalized");
        if (!ticket) fail("rembed: null ticket");
        if (nseq <= 0) fail("rembed: empty batch");
        if (!ids || !cu || !host_out) fail("rembed: null buffer");
        const int H = c->d.hidden_size;
        if (out_kind == RG_OUT_POOLED) {
            if (out_dim < 1 || out_dim > H) fail("rembed: WithDim(%d) out of range [1, %d]", out_dim, H);
        } else if (out_kind == RG_OUT_TOKENS) {
            if (out_dim != H) fail("rembed: token output needs out_dim == hidden (%d)", H);
        } else {
            fail("rembed: bad out_kind %d", out_kind);
        }
        validate_batch(c->d, ids, cu, nseq);
        *ticket = submit_batch(c, ids, cu, nseq, out_kind, out_dim, host_out, false);
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_collect(rg_ctx* c, int64_t ticket, char** err) {
    try {
        if (!c) fail("rembed: invalid context");
        collect_batch(c, ticket);
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_forward_device(rg_ctx* c, int dev_index, const int64_t* d_ids, const int32_t* d_cu, const int32_t* h_cu,
                      int nseq, int out_kind, int out_dim, float* d_out, void* stream, char** err) {
    try {
        if (!c || dev_index < 0 || dev_index >= static_cast<int>(c->reps.size())) fail("rembed: invalid context");
        if (!c->finalized) fail("rembed: weights not finalized");
        if (nseq <= 0) return 0;
        Replica& r = *c->reps[dev_index];
        std::lock_guard<std::mutex> lk(r.mu);
        check(cudaSetDevice(r.device), "cudaSetDevice");
        const int H = c->d.hidden_size;
        if (out_kind == RG_OUT_POOLED && (out_dim < 1 || out_dim > H))
            fail("rembed: WithDim(%d) out of range [1, %d]", out_dim, H);
        if (out_kind == RG_OUT_TOKENS && out_dim != H) fail("rembed: token output needs out_dim == hidden");
        if (h_cu[0] != 0) fail("cu_seqlens[0] must be 0");
        int max_len = 0;
        const int maxlen_model = max_seq_len(c->d);
        for (int i = 0; i < nseq; ++i) {
            const int len = h_cu[i + 1] - h_cu[i];
            if (len <= 0) fail("rembed: text %d: empty token sequence", i);
            if (len > maxlen_model)
                fail("rembed: text %d: sequence length %d exceeds the model's maximum %d", i, len, maxlen_model);
            max_len = std::max(max_len, len);
        }
        const int T = h_cu[nseq];
        const size_t nout = out_kind == RG_OUT_POOLED ? static_cast<size_t>(nseq) * out_dim : static_cast<size_t>(T) * H;
        ensure_workspace(c, r, T, nseq, nout);
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : r.stream;
        r.h_cu_view = h_cu;
        const Replica::GraphKey key{T, nseq, max_len, out_kind, out_dim, d_ids, d_cu, d_out, r.ws_gen};
        run_graphed(r, st, key, [&] { forward_on_device(c, r, d_ids, d_cu, nseq, T, max_len, out_kind, out_dim, d_out, st); });
        r.h_cu_view = nullptr;
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_sync(rg_ctx* c, int dev_index, char** err) {
    try {
        if (!c || dev_index < 0 || dev_index >= static_cast<int>(c->reps.size())) fail("rembed: invalid context");
        Replica& r = *c->reps[dev_index];
        std::lock_guard<std::mutex> lk(r.mu);
        check(cudaSetDevice(r.device), "cudaSetDevice");
        check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        if (r.d_status) {
            int s = 0;
            check(cudaMemcpy(&s, r.d_status, sizeof(int), cudaMemcpyDeviceToHost), "D2H status");
            if (s != 0) {
                check(cudaMemset(r.d_status, 0, sizeof(int)), "cudaMemset");
                fail("rembed: %s", status_message(s).c_str());
            }
        }
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_profile(rg_ctx* c, int dev_index, int enable) {
    if (!c || dev_index < 0 || dev_index >= static_cast<int>(c->reps.size())) return -1;
    Replica& r = *c->reps[dev_index];
    std::lock_guard<std::mutex> lk(r.mu);
    cudaSetDevice(r.device);
    try {
        if (!r.pending.empty()) cudaDeviceSynchronize();
    } catch (...) {
    }
    r.pending.clear();
    r.ev_used = 0;
    for (int k = 0; k < RG_KC_COUNT; ++k) {
        r.st_ms[k] = r.st_flops[k] = r.st_bytes[k] = 0.0;
        r.st_n[k] = 0;
    }
    r.prof = enable != 0;
    return 0;
}

int rg_profile_stats(rg_ctx* c, int dev_index, int kc, double* ms, int* launches, double* flops, double* bytes) {
    if (!c || dev_index < 0 || dev_index >= static_cast<int>(c->reps.size()) || kc < 0 || kc >= RG_KC_COUNT)
        return -1;
    Replica& r = *c->reps[dev_index];
    std::lock_guard<std::mutex> lk(r.mu);
    try {
        cudaSetDevice(r.device);
        prof_collect(r);
    } catch (const Error&) {
        return -1;
    }
    if (ms) *ms = r.st_ms[kc];
    if (launches) *launches = r.st_n[kc];
    if (flops) *flops = r.st_flops[kc];
    if (bytes) *bytes = r.st_bytes[kc];
    return 0;
}

int rg_test_inject(rg_ctx* c, int what, long long arg, char** err) {
    try {
        if (what != RG_INJECT_GEMM_WAIT && what != RG_INJECT_HOST_ALLOC && what != RG_INJECT_REPLICA)
            fail("rg_test_inject: unknown injection %d", what);
        if (what == RG_INJECT_GEMM_WAIT) {
            if (arg <= 0) fail("rg_test_inject: the wait limit must be positive");
            g_inject_gemm_wait.store(arg);
            return 0;
        }
        if (!c) fail("rg_test_inject: null context");
        std::lock_guard<std::mutex> tl(c->tmu);
        if (what == RG_INJECT_HOST_ALLOC) {
            c->inject_alloc = true;
        } else if (what == RG_INJECT_REPLICA) {
            if (arg < 0 || arg >= static_cast<long long>(c->reps.size()))
                fail("rg_test_inject: replica %lld out of range", arg);
            c->inject_replica = static_cast<int>(arg);
        } else {
            fail("rg_test_inject: unknown injection %d", what);
        }
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_hidden(const rg_ctx* c) { return c ? c->d.hidden_size : 0; }
int rg_mode_active(const rg_ctx* c) { return c ? c->mode : -1; }
int rg_last_launches(const rg_ctx* c, int dev_index) {
    if (!c || dev_index < 0 || dev_index >= static_cast<int>(c->reps.size())) return -1;
    return c->reps[dev_index]->last_launches;
}

void rg_free(rg_ctx* c) {
    if (!c) return;
    for (Replica* r : c->reps) {
        cudaSetDevice(r->device);
        if (r->stream) cudaStreamSynchronize(r->stream);
        drop_graphs(*r);
        free_workspace(*r);
        for (cudaEvent_t e : r->ev_pool) cudaEventDestroy(e);
        for (void* p : r->allocs) cudaFree(p);
        if (r->w16) cudaFree(r->w16);
        free_staging(*r);
        if (r->stream) cudaStreamDestroy(r->stream);
        delete r;
    }
    delete c;
}

void rg_free_string(char* s) { free(s); }

int rg_dense_residual_layernorm_bf16(const void* x, const void* w, const float* bias, const float* residual,
                                     const float* gamma, const float* beta, float eps, float* out32, void* outb,
                                     int M, int N, int K, void* stream, char** err) {
    try {
        if (M <= 0) return 0;
        if (!x || !w || !residual || !gamma || !beta || !out32 || !outb)
            fail("rg_dense_residual_layernorm_bf16: null buffer");
        if (K % 64 != 0 || !ln_width_ok(N))
            fail("rg_dense_residual_layernorm_bf16: unsupported shape (K=%d must be a multiple of 64; N=%d must be "
                 "one of 128, 256, 384, 512, 768, 1024, 1536, 2048)", K, N);
        int dev = 0;
        check(cudaGetDevice(&dev), "cudaGetDevice");
        int sms = 148;
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        // Per-device scratch: the fp32 sum M x N.
        struct Scratch {
            float* base = nullptr;
            size_t floats = 0;
        };
        static std::mutex smu;
        static std::map<int, Scratch> scratch;
        const size_t need = static_cast<size_t>(M) * N;
        float* base = nullptr;
        {
            std::lock_guard<std::mutex> lk(smu);
            Scratch& sc = scratch[dev];
            if (sc.floats < need) {
                check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
                if (sc.base) check(cudaFree(sc.base), "cudaFree");
                sc.base = nullptr;
                sc.floats = 0;
                check(cudaMalloc(&sc.base, need * sizeof(float)), "cudaMalloc (sublayer scratch)");
                sc.floats = need;
            }
            base = sc.base;
        }
        // in-kernel failures accumulate in the device's kernel-level status
        // word until rg_kernel_status reads it
        int* status = nullptr;
        check(rg::kernel_status_word(dev, &status), "kernel status word");
        float* sum = base;
        CUtensorMap ta, tb;
        const int bn = rg::gemm_block_n(M, N, sms);
        if (!rg::make_kmajor_tmap(&ta, x, 2, M, K, K, 128) || !rg::make_kmajor_tmap(&tb, w, 2, N, K, K, rg::gemm_w_box_rows(bn)))
            fail("rg_dense_residual_layernorm_bf16: cuTensorMapEncodeTiled failed");
        rg::GemmArgs a{};
        a.M = M;
        a.N = N;
        a.K = K;
        a.bias = bias;
        a.residual = residual;
        a.out = sum;
        a.ld_out = N;
        a.status = status;
        check(rg::gemm_launch(rg::GemmKind::kBF16, rg::kEpiBiasRes, bn, ta, tb, a, sms, st), "gemm launch");
        check(rg::launch_ln(sum, gamma, beta, eps, M, N, out32, static_cast<act16*>(outb), false, nullptr, nullptr, st,
                            status),
              "ln launch");
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

int rg_dense_bf16(const void* x, const void* w, const float* bias, const float* residual, void* y, int M, int N,
                  int K, int epilogue, void* stream, char** err) {
    try {
        if (M <= 0) return 0;
        if (K % 64 != 0 || N % 128 != 0) fail("rg_dense_bf16: need K %% 64 == 0 and N %% 128 == 0 (K=%d N=%d)", K, N);
        if (epilogue < 0 || epilogue > 3) fail("rg_dense_bf16: bad epilogue %d", epilogue);
        if (epilogue == rg::kEpiBiasRes && !residual) fail("rg_dense_bf16: residual epilogue needs a residual");
        int dev = 0;
        check(cudaGetDevice(&dev), "cudaGetDevice");
        int sms = 148;
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
        CUtensorMap ta, tb;
        const int bn = rg::gemm_block_n(M, N, sms);
        if (!rg::make_kmajor_tmap(&ta, x, 2, M, K, K, 128) || !rg::make_kmajor_tmap(&tb, w, 2, N, K, K, rg::gemm_w_box_rows(bn)))
            fail("rg_dense_bf16: cuTensorMapEncodeTiled failed");
        int* status = nullptr;
        check(rg::kernel_status_word(dev, &status), "kernel status word");
        rg::GemmArgs a{};
        a.M = M;
        a.N = N;
        a.K = K;
        a.bias = bias;
        a.residual = residual;
        a.out = y;
        a.ld_out = N;
        a.status = status;
        const long long inj = g_inject_gemm_wait.exchange(0);
        if (inj > 0) {
            a.wait_limit = inj;
            a.inject_withhold = 1;
        }
        check(rg::gemm_launch(rg::GemmKind::kBF16, epilogue, bn, ta, tb, a, sms, static_cast<cudaStream_t>(stream)),
              "gemm launch");
        return 0;
    } catch (const Error& e) {
        set_err(err, e.msg);
        return -1;
    }
}

}  // extern "C"
