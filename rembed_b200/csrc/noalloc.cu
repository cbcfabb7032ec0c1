// noalloc.cu - rg_dense_residual_layernorm_bf16_noalloc: the dense +
// residual + LayerNorm sublayer without any device allocation.
//
// Who needs it: callers that cannot call cudaMalloc.  A host whose memory
// manager owns every byte of device memory (a serving runtime that carves
// all of HBM into its own arena up front, or an allocator that must
// account for each buffer) cannot let a library allocate behind its back,
// and cudaMalloc may also synchronise the device, which a caller running a
// latency-bound pipeline must avoid.  rg_dense_residual_layernorm_bf16
// allocates its scratch on first use per device and grows it as needed;
// this variant never does.
//
// Where the scratch lives: g_noalloc_scratch, a file-scope static device
// array of RG_NOALLOC_SCRATCH_FLOATS floats plus a 256-byte header (one
// status word).  It is part of the library's device image, so every GPU on
// which the library's module is loaded holds these 16 MiB until the process
// exits.  In host code the array's name is only a host-side stand-in, not a
// device address; the host looks its device address up once per device
// (cudaGetSymbolAddress, with that device current) and passes that pointer
// to the kernels.
//
// Sharing: every call uses the same array and it keeps the last call's
// contents.  The fp32 sum region is fully overwritten by the GEMM before the
// LayerNorm reads it, so it needs no clearing.  The status word starts at
// zero when the module loads; a kernel that fails (a bounded pipeline wait
// that gave up) sets a bit in it, and rg_kernel_status reads and clears it
// (noalloc_status_take below, which copies through the symbol and so
// allocates nothing either).  Calls whose work overlaps on the GPU
// (different streams, or different host threads, on one device) race on the
// array: order them on one stream.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "rembed_gpu.h"
#include "gemm.cuh"
#include "kernels.cuh"

namespace {

constexpr size_t kHeaderFloats = 64;  // 256 bytes: the status word and padding
constexpr size_t kMaxDevices = 64;

// The scratch: [status word | pad to 256 B | fp32 sum, up to M*N floats].
__device__ __align__(256) static float g_noalloc_scratch[kHeaderFloats + RG_NOALLOC_SCRATCH_FLOATS];

std::mutex g_mu;
float* g_addr[kMaxDevices] = {};  // device address of g_noalloc_scratch, per device

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

bool ln_width_ok(int n) {
    if (n <= 0 || n % 128 != 0) return false;
    switch (n / 128) {
    case 1: case 2: case 3: case 4: case 6: case 8: case 12: case 16: return true;
    default: return false;
    }
}

}  // namespace

extern "C" int rg_dense_residual_layernorm_bf16_noalloc(const void* x, const void* w, const float* bias,
                                                        const float* residual, const float* gamma, const float* beta,
                                                        float eps, float* out32, void* outb, int M, int N, int K,
                                                        void* stream, char** err) {
    if (M <= 0) return 0;
    if (!x || !w || !residual || !gamma || !beta || !out32 || !outb)
        return set_err(err, "rg_dense_residual_layernorm_bf16_noalloc: null buffer");
    if (K % 64 != 0 || !ln_width_ok(N))
        return set_err(err,
                       "rg_dense_residual_layernorm_bf16_noalloc: unsupported shape (K=%d must be a multiple of 64; "
                       "N=%d must be one of 128, 256, 384, 512, 768, 1024, 1536, 2048)",
                       K, N);
    const size_t need = static_cast<size_t>(M) * static_cast<size_t>(N);
    if (need > RG_NOALLOC_SCRATCH_FLOATS)
        return set_err(err,
                       "rg_dense_residual_layernorm_bf16_noalloc: M*N = %d*%d = %zu floats exceeds the fixed scratch "
                       "of %zu floats (%zu MiB); split the rows into calls of at most %zu rows",
                       M, N, need, static_cast<size_t>(RG_NOALLOC_SCRATCH_FLOATS),
                       static_cast<size_t>(RG_NOALLOC_SCRATCH_FLOATS) * 4 / (1024 * 1024),
                       static_cast<size_t>(RG_NOALLOC_SCRATCH_FLOATS) / N);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_err(err, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || static_cast<size_t>(dev) >= kMaxDevices)
        return set_err(err, "rg_dense_residual_layernorm_bf16_noalloc: device %d out of range", dev);

    // Set-up, once per device, with that device current: the array's device
    // address.  This first call on a device must come before any stream
    // capture that includes this entry point.
    float* base;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_addr[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p)
                return set_err(err, "cudaGetSymbolAddress(g_noalloc_scratch) on device %d: %s", dev,
                               cudaGetErrorString(e));
            g_addr[dev] = static_cast<float*>(p);
        }
        base = g_addr[dev];
    }
    int sms = 148;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_err(err, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* status = reinterpret_cast<int*>(base);  // sticky until rg_kernel_status clears it
    float* sum = base + kHeaderFloats;

    CUtensorMap ta, tb;
    const int bn = rg::gemm_block_n(M, N, sms);
    if (!rg::make_kmajor_tmap(&ta, x, 2, M, K, K, 128) || !rg::make_kmajor_tmap(&tb, w, 2, N, K, K, rg::gemm_w_box_rows(bn)))
        return set_err(err, "rg_dense_residual_layernorm_bf16_noalloc: cuTensorMapEncodeTiled failed");
    rg::GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.residual = residual;
    a.out = sum;
    a.ld_out = N;
    a.status = status;
    e = rg::gemm_launch(rg::GemmKind::kBF16, rg::kEpiBiasRes, bn, ta, tb, a, sms, st);
    if (e != cudaSuccess) return set_err(err, "gemm launch: %s", cudaGetErrorString(e));
    e = rg::launch_ln(sum, gamma, beta, eps, M, N, out32, static_cast<uint16_t*>(outb), false, nullptr, nullptr, st,
                      status);
    if (e != cudaSuccess) return set_err(err, "ln launch: %s", cudaGetErrorString(e));
    return 0;
}

namespace rg {

// Read and clear the status word at the head of g_noalloc_scratch on the
// current device (synchronous copies through the symbol; no allocation).
cudaError_t noalloc_status_take(int* s) {
    *s = 0;
    cudaError_t e = cudaMemcpyFromSymbol(s, g_noalloc_scratch, sizeof(int), 0, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess || *s == 0) return e;
    const int zero = 0;
    return cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof(int), 0, cudaMemcpyHostToDevice);
}

}  // namespace rg
