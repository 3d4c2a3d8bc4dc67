// tz_noalloc.cu -- tz_linear_w8a8_noalloc: the W8A8 linear with its temporaries in a fixed,
// library-owned device array instead of the context's growable scratch arena.
//
// Who needs this: callers that must not allocate device memory while they run.  Examples are code
// that is being captured into a CUDA graph, where an allocation (or the device-wide synchronisation
// that growing the arena implies) breaks or serialises the capture; serving processes whose device
// memory is entirely reserved up front by another allocator, so a cudaMalloc can fail mid-request;
// and latency-critical threads that cannot afford the implicit device synchronisation of
// cudaMalloc / cudaFree.  tz_linear_w8a8 grows the context arena on demand (synchronise, free,
// allocate), which such callers cannot allow.
//
// The temporaries (the per-token int8 copy of x, its scales, and the widened weight scales) live in
// g_noalloc_scratch, a file-scope __device__ array of kNoallocBytes.  Every GPU that loads this
// library holds that array until the process exits.  All calls share it: two calls that overlap on
// the GPU (different streams, or different host threads on one device) race on it.  Its contents
// are whatever the last call left; nothing here needs it to start at zero, because every byte read
// is written first by the same call.
//
// The kernels run on the calling thread's current device, so that device must be the context's
// (the call is refused otherwise).  The array's device address is looked up once per device and
// kept for the life of the process: it assumes the device's primary context lives until exit (a
// cudaDeviceReset invalidates it).
#include <cuda_runtime.h>

#include <mutex>

#include "tz_internal.h"

namespace tz {
int launch_f16bits_to_f32(tz_ctx_t ctx, const uint16_t* x, float* y, long long n, cudaStream_t s);
int launch_quant_act(tz_ctx_t ctx, const float* x, int8_t* q, float* scale, long long rows, int cols, cudaStream_t s);
}  // namespace tz

namespace {

constexpr size_t kNoallocBytes = 8u << 20;  // 8 MiB per device
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};

size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// The device address of g_noalloc_scratch on `device`.  In host code the symbol itself is only a
// host-side stand-in, so the address is looked up once per device, with that device current.
int scratch_address(int device, void** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    TZ_CHECK(device >= 0 && device < kMaxDevices, TZ_EINVAL, "device %d", device);
    if (!g_addr[device]) {
        int prev = 0;
        TZ_CUDA(cudaGetDevice(&prev));
        cudaError_t e = cudaSetDevice(device);
        void* p = nullptr;
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        const cudaError_t r = cudaSetDevice(prev);
        if (e != cudaSuccess) return tz::cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        if (r != cudaSuccess) return tz::cuda_fail(r, "cudaSetDevice (restore)");
        g_addr[device] = p;
    }
    *out = g_addr[device];
    return TZ_OK;
}

}  // namespace

using namespace tz;

extern "C" int tz_linear_w8a8_noalloc(tz_ctx_t ctx, const float* x, const int8_t* wq, const uint16_t* scale_f16,
                                      const float* bias, float* y, int m, int k, int n, tz_stream_t stream) {
    TZ_CHECK(ctx && x && wq && scale_f16 && bias && y && m >= 0 && k > 0 && n > 0, TZ_EINVAL,
             "tz_linear_w8a8_noalloc: bad arguments");
    if (m == 0) return TZ_OK;
    TZ_CHECK(k % 16 == 0, TZ_EINVAL, "tz_linear_w8a8_noalloc: k must be a multiple of 16 (k=%d)", k);
    const size_t bq = round256(static_cast<size_t>(m) * static_cast<size_t>(k));
    const size_t bxs = round256(sizeof(float) * static_cast<size_t>(m));
    const size_t bs = round256(sizeof(float) * static_cast<size_t>(n));
    TZ_CHECK(bq + bxs + bs <= kNoallocBytes, TZ_EINVAL,
             "tz_linear_w8a8_noalloc: m=%d, k=%d, n=%d needs %zu bytes of scratch; the fixed scratch holds %zu "
             "(m*k + 4*m + 4*n, each rounded up to 256 bytes); split the rows or use tz_linear_w8a8",
             m, k, n, bq + bxs + bs, kNoallocBytes);
    int cur = -1;
    TZ_CUDA(cudaGetDevice(&cur));
    TZ_CHECK(cur == ctx->device, TZ_EINVAL,
             "tz_linear_w8a8_noalloc: the current device (%d) is not the context's (%d); make it current first", cur,
             ctx->device);
    void* base = nullptr;
    int rc = scratch_address(ctx->device, &base);
    if (rc) return rc;
    cudaStream_t s = pick_stream(ctx, stream);
    char* p = static_cast<char*>(base);
    int8_t* xq = reinterpret_cast<int8_t*>(p);
    float* xs = reinterpret_cast<float*>(p + bq);
    float* sc = reinterpret_cast<float*>(p + bq + bxs);
    if ((rc = launch_quant_act(ctx, x, xq, xs, m, k, s))) return rc;
    if ((rc = launch_f16bits_to_f32(ctx, scale_f16, sc, n, s))) return rc;
    GemmArgs g;
    g.kind = KIND_I8;
    g.a = xq; g.lda = k; g.b = wq; g.ldb = k; g.M = m; g.N = n; g.K = k;
    g.row_scale = xs; g.col_scale = sc; g.bias = bias; g.out = y; g.ldo = n; g.out_type = OUT_F32;
    return launch_gemm(ctx, g, s);
}
