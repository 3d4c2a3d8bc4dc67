// tz_runtime.cu -- context, errors, device memory, scratch arena and TMA descriptor encoding.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>

#include "tz_internal.h"
#include "tz_ptx.cuh"

namespace tz {

static thread_local char g_last_error[1024] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    const int code = (e == cudaErrorMemoryAllocation) ? TZ_ENOMEM : TZ_ECUDA;
    return fail(code, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

void clear_error() { g_last_error[0] = 0; }

cudaStream_t pick_stream(tz_ctx_t ctx, tz_stream_t s) {
    return s ? static_cast<cudaStream_t>(s) : ctx->stream;
}

int scratch_reserve(tz_ctx_t ctx, size_t bytes, void** out) {
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (ctx->scratch.bytes < bytes) {
        TZ_CUDA(cudaSetDevice(ctx->device));
        if (ctx->scratch.ptr) {
            TZ_CUDA(cudaDeviceSynchronize());
            TZ_CUDA(cudaFree(ctx->scratch.ptr));
            ctx->scratch.ptr = nullptr;
            ctx->scratch.bytes = 0;
        }
        size_t want = bytes + (bytes >> 2);
        want = (want + 0xFFFFF) & ~static_cast<size_t>(0xFFFFF);
        TZ_CUDA(cudaMalloc(&ctx->scratch.ptr, want));
        ctx->scratch.bytes = want;
    }
    *out = ctx->scratch.ptr;
    return TZ_OK;
}

int read_status(tz_ctx_t ctx, cudaStream_t s) {
    int h = 0;
    TZ_CUDA(cudaMemcpyAsync(&h, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, s));
    TZ_CUDA(cudaStreamSynchronize(s));
    if (h) {
        TZ_CUDA(cudaMemsetAsync(ctx->d_status, 0, sizeof(int), s));
        TZ_CUDA(cudaStreamSynchronize(s));
        if (h & TZ_DEV_TIMEOUT) return fail(TZ_ETIMEOUT, "a device-side wait expired (status 0x%x)", h);
        return fail(TZ_EINVAL, "a device-side bounds check fired (status 0x%x)", h);
    }
    return TZ_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_outer) {
    return encode_tmap_2d_swz(map, dtype, elem_bytes, base, inner, outer, row_stride_bytes, box_inner, box_outer,
                              CU_TENSOR_MAP_SWIZZLE_128B);
}

int encode_tmap_2d_swz(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                       uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                       uint32_t box_outer, CUtensorMapSwizzle swz) {
    auto enc = get_encode();
    TZ_CHECK(enc, TZ_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    TZ_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, TZ_EINVAL, "TMA base must be 16-byte aligned");
    TZ_CHECK(row_stride_bytes % 16 == 0, TZ_EINVAL, "TMA row stride must be a multiple of 16 bytes");
    const uint32_t inner_bytes = box_inner * static_cast<uint32_t>(elem_bytes);
    TZ_CHECK(inner_bytes % 16 == 0 && box_inner <= 256 && box_outer <= 256, TZ_EINVAL,
             "TMA box inner extent must be a multiple of 16 bytes (at most 256 x 256 elements)");
    if (swz != CU_TENSOR_MAP_SWIZZLE_NONE) {
        const uint32_t span = swz == CU_TENSOR_MAP_SWIZZLE_64B ? 64 : swz == CU_TENSOR_MAP_SWIZZLE_32B ? 32 : 128;
        TZ_CHECK(inner_bytes <= span, TZ_EINVAL, "TMA box too wide for its swizzle");
    }
    cuuint64_t dims[2] = {inner, outer < 1 ? 1 : outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TZ_CHECK(r == CUDA_SUCCESS, TZ_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return TZ_OK;
}

}  // namespace tz

using namespace tz;

namespace {
// The bounded-wait self-test: one thread waits on an mbarrier that nothing ever arrives on, through
// the same wait every kernel uses (mbar_wait: globaltimer-bounded, 1 s).  The wait expires, sets
// the timeout bit of the status word and returns; the kernel exits normally.
__global__ void selftest_wait_kernel(int* status) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        tzp::mbar_init(&bar, 1);
        tzp::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) tzp::mbar_wait(&bar, 0, status, nullptr);
    __syncthreads();
}
}  // namespace

extern "C" {

const char* tz_get_last_error(void) { return g_last_error; }

const char* tz_version(void) { return "tenzor_b200 0.1 (sm_100a; tcgen05 GEMM, mma.sync attention)"; }

int tz_cuda_create(int device, tz_ctx_t* out) {
    TZ_CHECK(out, TZ_EINVAL, "tz_cuda_create: out is NULL");
    *out = nullptr;
    int n = 0;
    TZ_CUDA(cudaGetDeviceCount(&n));
    TZ_CHECK(device >= 0 && device < n, TZ_EINVAL, "tz_cuda_create: device %d of %d", device, n);
    cudaDeviceProp p;
    TZ_CUDA(cudaGetDeviceProperties(&p, device));
    TZ_CHECK(p.major == 10 && p.minor == 0, TZ_EUNSUPPORTED,
             "tz_cuda_create: device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
             p.major, p.minor);
    TZ_CUDA(cudaSetDevice(device));
    auto* c = new tz_ctx_s();
    c->device = device;
    c->sm_count = p.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->d_status, 0, sizeof(int));
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "tz_cuda_create");
    }
    *out = c;
    return TZ_OK;
}

int tz_cuda_destroy(tz_ctx_t ctx) {
    if (!ctx) return TZ_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->scratch.ptr) cudaFree(ctx->scratch.ptr);
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return TZ_OK;
}

int tz_cuda_synchronize(tz_ctx_t ctx) {
    TZ_CHECK(ctx, TZ_EINVAL, "null context");
    TZ_CUDA(cudaSetDevice(ctx->device));
    TZ_CUDA(cudaDeviceSynchronize());
    return read_status(ctx, ctx->stream);
}

int tz_cuda_check_status(tz_ctx_t ctx) {
    TZ_CHECK(ctx, TZ_EINVAL, "null context");
    TZ_CUDA(cudaSetDevice(ctx->device));
    return read_status(ctx, ctx->stream);
}

int tz_cuda_sm_count(tz_ctx_t ctx) { return ctx ? ctx->sm_count : 0; }

int tz_cuda_set_sm_reserve(tz_ctx_t ctx, int n) {
    TZ_CHECK(ctx && n >= 0 && n < ctx->sm_count, TZ_EINVAL, "tz_cuda_set_sm_reserve: %d outside [0, SMs)", n);
    ctx->sm_reserve = n;
    return TZ_OK;
}

int tz_cuda_selftest_wait(tz_ctx_t ctx) {
    TZ_CHECK(ctx, TZ_EINVAL, "null context");
    TZ_CUDA(cudaSetDevice(ctx->device));
    selftest_wait_kernel<<<1, 32, 0, ctx->stream>>>(ctx->d_status);
    TZ_CUDA(cudaGetLastError());
    TZ_CUDA(cudaStreamSynchronize(ctx->stream));
    return read_status(ctx, ctx->stream);
}

int tz_alloc(tz_ctx_t ctx, size_t bytes, void** dptr) {
    TZ_CHECK(ctx && dptr, TZ_EINVAL, "tz_alloc: null argument");
    TZ_CUDA(cudaSetDevice(ctx->device));
    TZ_CUDA(cudaMalloc(dptr, bytes ? bytes : 16));
    return TZ_OK;
}

int tz_free(tz_ctx_t ctx, void* dptr) {
    TZ_CHECK(ctx, TZ_EINVAL, "tz_free: null context");
    if (!dptr) return TZ_OK;
    TZ_CUDA(cudaSetDevice(ctx->device));
    TZ_CUDA(cudaFree(dptr));
    return TZ_OK;
}

int tz_upload(tz_ctx_t ctx, void* dst, const void* src, size_t bytes) {
    TZ_CHECK(ctx && (bytes == 0 || (dst && src)), TZ_EINVAL, "tz_upload: null argument");
    TZ_CUDA(cudaSetDevice(ctx->device));
    TZ_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    TZ_CUDA(cudaStreamSynchronize(ctx->stream));
    return TZ_OK;
}

int tz_download(tz_ctx_t ctx, void* dst, const void* src, size_t bytes) {
    TZ_CHECK(ctx && (bytes == 0 || (dst && src)), TZ_EINVAL, "tz_download: null argument");
    TZ_CUDA(cudaSetDevice(ctx->device));
    TZ_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    TZ_CUDA(cudaStreamSynchronize(ctx->stream));
    return TZ_OK;
}

}  // extern "C"
