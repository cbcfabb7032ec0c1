// kernel_abi.cu - kernel-level C ABI entry points beyond the dense
// projections: varlen attention, the full-int8 row quantiser and integer
// GEMM, and the status check shared by every kernel-level call.
//
// These calls take device pointers on the current CUDA device and are
// asynchronous on the caller's stream.  A failure that a kernel detects on
// the device (a bounded pipeline wait that gave up, an fp16 overflow) is
// recorded in a status word of the device; rg_kernel_status reads it back.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "rembed_gpu.h"
#include "gemm.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace {

int set_err(char** err, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int set_err(char** err, const char* fmt, ...) {
    if (err) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        const size_t n = strlen(buf) + 1;
        *err = static_cast<char*>(malloc(n));
        if (*err) memcpy(*err, buf, n);
    }
    return -1;
}

std::string describe_status(int s) {
    std::string m;
    if (s & rg::kStatusWaitTimeout) m += "a device pipeline wait timed out; ";
    if (s & rg::kStatusBadShape) m += "inconsistent shape on the device; ";
    if (s & rg::kStatusF16Overflow) m += "an fp16 output overflowed; ";
    if (s & rg::kStatusBadToken) m += "token id out of vocab range; ";
    if (m.empty()) m = "device error status " + std::to_string(s);
    else m.resize(m.size() - 2);
    return m;
}

}  // namespace

namespace rg {

// One status word per device for the kernel-level entry points, allocated on
// first use and kept until exit.
cudaError_t kernel_status_word(int dev, int** out) {
    static std::mutex mu;
    static std::map<int, int*> words;
    std::lock_guard<std::mutex> lk(mu);
    auto it = words.find(dev);
    if (it != words.end()) {
        *out = it->second;
        return cudaSuccess;
    }
    int* w = nullptr;
    cudaError_t e = cudaMalloc(&w, sizeof(int));
    if (e != cudaSuccess) return e;
    e = cudaMemset(w, 0, sizeof(int));
    if (e != cudaSuccess) {
        cudaFree(w);
        return e;
    }
    words[dev] = w;
    *out = w;
    return cudaSuccess;
}

// noalloc.cu: read and clear the no-allocation entry point's status word.
cudaError_t noalloc_status_take(int* s);

}  // namespace rg

extern "C" {

int rg_kernel_status(void* stream, char** err) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_err(err, "cudaGetDevice: %s", cudaGetErrorString(e));
    e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return set_err(err, "rg_kernel_status: %s", cudaGetErrorString(e));
    int* word = nullptr;
    e = rg::kernel_status_word(dev, &word);
    if (e != cudaSuccess) return set_err(err, "rg_kernel_status: %s", cudaGetErrorString(e));
    int s = 0, s_noalloc = 0;
    e = cudaMemcpy(&s, word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && s != 0) e = cudaMemset(word, 0, sizeof(int));
    if (e == cudaSuccess) e = rg::noalloc_status_take(&s_noalloc);
    if (e != cudaSuccess) return set_err(err, "rg_kernel_status: %s", cudaGetErrorString(e));
    if (s | s_noalloc) return set_err(err, "kernel-level call failed on device %d: %s", dev,
                                      describe_status(s | s_noalloc).c_str());
    return 0;
}

int rg_attention(const void* q, const void* k, const void* v, int ldq, int ldk, int ldv, const int32_t* cu_seqlens,
                 const int32_t* host_cu, int nseq, int heads, int kv_heads, int head_dim, float scale, int rel_lo,
                 int rel_hi, int dtype, void* out, int ldo, void* stream, char** err) {
    if (nseq <= 0) return 0;
    if (!q || !k || !v || !cu_seqlens || !host_cu || !out) return set_err(err, "rg_attention: null buffer");
    if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256)
        return set_err(err, "rg_attention: head dim %d unsupported (32, 64, 128 or 256)", head_dim);
    if (heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0)
        return set_err(err, "rg_attention: heads %d not a multiple of kv_heads %d", heads, kv_heads);
    if (rel_lo > 0 || rel_hi < 0) return set_err(err, "rg_attention: the window [%d, %d] must contain 0", rel_lo, rel_hi);
    if (ldq < heads * head_dim || ldk < kv_heads * head_dim || ldv < kv_heads * head_dim || ldo < heads * head_dim)
        return set_err(err, "rg_attention: a row stride is narrower than its heads");
    if (host_cu[0] != 0) return set_err(err, "rg_attention: cu_seqlens[0] must be 0");
    int max_len = 0;
    for (int i = 0; i < nseq; ++i) {
        const int len = host_cu[i + 1] - host_cu[i];
        if (len <= 0) return set_err(err, "rg_attention: sequence %d is empty", i);
        max_len = std::max(max_len, len);
    }
    const int T = host_cu[nseq];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_err(err, "cudaGetDevice: %s", cudaGetErrorString(e));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == RG_DTYPE_F32) {
        rg::AttnF32Params p{};
        p.q = static_cast<const float*>(q);
        p.k = static_cast<const float*>(k);
        p.v = static_cast<const float*>(v);
        p.ldq = ldq;
        p.ldk = ldk;
        p.ldv = ldv;
        p.cu = cu_seqlens;
        p.group = heads / kv_heads;
        p.scale = scale;
        p.rel_lo = rel_lo;
        p.rel_hi = rel_hi;
        p.out_hi = static_cast<float*>(out);
        p.out_lo = nullptr;  // the unsplit fp32 result
        p.ldo = ldo;
        e = rg::launch_attention_f32(p, nseq, max_len, heads, head_dim, st);
    } else if (dtype == RG_DTYPE_BF16 || dtype == RG_DTYPE_F16) {
        int* status = nullptr;
        e = rg::kernel_status_word(dev, &status);
        if (e != cudaSuccess) return set_err(err, "rg_attention: status word: %s", cudaGetErrorString(e));
        rg::AttnParams p{};
        p.q = static_cast<const uint16_t*>(q);
        p.k = static_cast<const uint16_t*>(k);
        p.v = static_cast<const uint16_t*>(v);
        p.f16 = dtype == RG_DTYPE_F16;
        p.ldq = ldq;
        p.ldk = ldk;
        p.ldv = ldv;
        p.cu = cu_seqlens;
        p.group = heads / kv_heads;
        p.scale = scale;
        p.scale_log2 = scale * 1.4426950408889634f;
        p.rel_lo = rel_lo;
        p.rel_hi = rel_hi;
        p.out = static_cast<uint16_t*>(out);
        p.ldo = ldo;
        p.T = T;
        p.kv_heads = kv_heads;
        p.status = status;
        e = rg::launch_attention(p, nseq, max_len, heads, head_dim, st);
    } else {
        return set_err(err, "rg_attention: unknown dtype %d", dtype);
    }
    if (e != cudaSuccess) return set_err(err, "rg_attention: launch: %s", cudaGetErrorString(e));
    return 0;
}

int rg_quantize_rows_s8(const void* x, int M, int K, int8_t* q, float* row_scale, void* stream, char** err) {
    if (M <= 0) return 0;
    if (!x || !q || !row_scale) return set_err(err, "rg_quantize_rows_s8: null buffer");
    if (K <= 0 || K % 8 != 0 || K > 4096)
        return set_err(err, "rg_quantize_rows_s8: K=%d must be a multiple of 8 up to 4096", K);
    cudaError_t e = rg::launch_quantize_rows(static_cast<const __nv_bfloat16*>(x), M, K, q, row_scale,
                                             static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return set_err(err, "rg_quantize_rows_s8: launch: %s", cudaGetErrorString(e));
    return 0;
}

int rg_dense_s8(const int8_t* xq, const float* row_scale, const int8_t* wq, const float* col_scale, const float* bias,
                float* y, int M, int N, int K, void* stream, char** err) {
    if (M <= 0) return 0;
    if (!xq || !row_scale || !wq || !col_scale || !y) return set_err(err, "rg_dense_s8: null buffer");
    if (K % 128 != 0 || N % 128 != 0)
        return set_err(err, "rg_dense_s8: need K %% 128 == 0 and N %% 128 == 0 (K=%d N=%d)", K, N);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_err(err, "cudaGetDevice: %s", cudaGetErrorString(e));
    int sms = 148;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_err(err, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    int* status = nullptr;
    e = rg::kernel_status_word(dev, &status);
    if (e != cudaSuccess) return set_err(err, "rg_dense_s8: status word: %s", cudaGetErrorString(e));
    const int bn = rg::gemm_block_n(M, N, sms);
    CUtensorMap ta, tb;
    if (!rg::make_kmajor_tmap(&ta, xq, 1, M, K, K, 128) ||
        !rg::make_kmajor_tmap(&tb, wq, 1, N, K, K, rg::gemm_w_box_rows(bn)))
        return set_err(err, "rg_dense_s8: cuTensorMapEncodeTiled failed (16-byte aligned buffers needed)");
    rg::GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.row_scale = row_scale;
    a.col_scale = col_scale;
    a.out = y;
    a.ld_out = N;
    a.status = status;
    e = rg::gemm_launch(rg::GemmKind::kS8, rg::kEpiBiasF32, bn, ta, tb, a, sms, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return set_err(err, "rg_dense_s8: launch: %s", cudaGetErrorString(e));
    return 0;
}

}  // extern "C"
