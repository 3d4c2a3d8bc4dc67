// tz_nd.cu -- N-dimensional tensor ops behind the `.eval()` executor (src/backend/cpu/executor.zig)
// and the ONNX op map (src/onnx/executor.zig): batched matmul with broadcast batch dimensions and
// strided operand views, single-axis reduce and softmax, transpose, cast, concat, and the
// f32-accurate (split-tf32) tcgen05 matmul used for their 2-D products.
//
// These are the general-shape forms of the path's ops.  The Arctic forward itself never calls them
// (its attention, LayerNorm and GEMMs are the fused kernels of tz_arctic / tz_attention / tz_gemm*).
// Every kernel is a grid-stride loop sized to a multiple of the SM count; the per-element index
// arithmetic is 64-bit.
#include <cuda_runtime.h>

#include <vector>

#include "tz_internal.h"
#include "tz_ptx.cuh"
#include "tz_rowops.cuh"

namespace tz {
namespace {

inline int grid_for(tz_ctx_t ctx, long long work, int threads) {
    long long blocks = (work + threads - 1) / threads;
    const long long cap = static_cast<long long>(ctx->sm_count) * 8;
    if (blocks > cap) blocks = cap;
    return static_cast<int>(blocks < 1 ? 1 : blocks);
}

// ---- batched matmul (CUDA cores, f32) -----------------------------------------------------------
// One CTA per 64 x 64 output tile of one batch (blockIdx.z strides over the batches); 256 threads,
// 4 x 4 outputs each; K in steps of 16 through shared memory.  Operands are read through their
// element strides, so transposed and head-interleaved views need no copy.  Each output is one
// sequential f32 fmaf chain over k (deterministic).
struct BmmArgs {
    int bnd;
    long long bshape[4];
    long long as[4], bs[4], cs[4];
    long long a_rs, a_cs, b_rs, b_cs, c_rs, c_cs;
    int m, k, n;
    long long nbatch;
};

__global__ void __launch_bounds__(256) bmm_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                  float* __restrict__ c, BmmArgs p) {
    __shared__ float As[16][64 + 4];  // [kk][row]
    __shared__ float Bs[16][64 + 4];  // [kk][col]
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
    for (long long bi = blockIdx.z; bi < p.nbatch; bi += gridDim.z) {
        long long rem = bi, ao = 0, bo = 0, co = 0;
        for (int d = p.bnd - 1; d >= 0; --d) {
            const long long q = rem / p.bshape[d];
            const long long x = rem - q * p.bshape[d];
            rem = q;
            ao += x * p.as[d];
            bo += x * p.bs[d];
            co += x * p.cs[d];
        }
        float acc[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[r][q] = 0.0f;
        for (int k0 = 0; k0 < p.k; k0 += 16) {
            for (int e = threadIdx.x; e < 1024; e += 256) {
                const int r = e >> 4, kk = e & 15;
                const int gi = i0 + r, gk = k0 + kk;
                As[kk][r] = (gi < p.m && gk < p.k) ? a[ao + gi * p.a_rs + gk * p.a_cs] : 0.0f;
            }
            for (int e = threadIdx.x; e < 1024; e += 256) {
                const int kk = e >> 6, q = e & 63;
                const int gk = k0 + kk, gj = j0 + q;
                Bs[kk][q] = (gk < p.k && gj < p.n) ? b[bo + gk * p.b_rs + gj * p.b_cs] : 0.0f;
            }
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) {
                float av[4], bv[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) av[r] = As[kk][ty * 4 + r];
#pragma unroll
                for (int q = 0; q < 4; ++q) bv[q] = Bs[kk][tx * 4 + q];
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[r][q] = fmaf(av[r], bv[q], acc[r][q]);
            }
            __syncthreads();
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int gi = i0 + ty * 4 + r;
            if (gi >= p.m) continue;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int gj = j0 + tx * 4 + q;
                if (gj < p.n) c[co + gi * p.c_rs + gj * p.c_cs] = acc[r][q];
            }
        }
    }
}

// ---- single-axis reduce / softmax ---------------------------------------------------------------
__device__ __forceinline__ double red_identity(int red) {
    return red == TZ_RED_PROD ? 1.0 : red == TZ_RED_MAX ? -INFINITY : red == TZ_RED_MIN ? INFINITY : 0.0;
}

// inner == 1: a warp per row of `len` contiguous values.
__global__ void reduce_rows_kernel(const float* __restrict__ x, long long outer, long long len, int red,
                                   float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    for (long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < outer; r += warps) {
        const float* xr = x + r * len;
        double acc = red_identity(red);
        for (long long i = lane; i < len; i += 32) acc = red_combine(red, acc, static_cast<double>(xr[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = red_combine(red, acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) out[r] = static_cast<float>(red == TZ_RED_MEAN ? acc / static_cast<double>(len) : acc);
    }
}

// inner > 1: a thread per (outer, inner) position, walking the axis (consecutive threads read
// consecutive inner positions: coalesced).
__global__ void reduce_cols_kernel(const float* __restrict__ x, long long outer, long long len, long long inner,
                                   int red, float* __restrict__ out) {
    const long long n = outer * inner;
    for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long o = t / inner, in = t - o * inner;
        const float* xp = x + o * len * inner + in;
        double acc = red_identity(red);
        for (long long i = 0; i < len; ++i) acc = red_combine(red, acc, static_cast<double>(xp[i * inner]));
        out[t] = static_cast<float>(red == TZ_RED_MEAN ? acc / static_cast<double>(len) : acc);
    }
}

// softmaxAxis general case (softmax.zig:185-216): per (outer, inner) position max, then
// y = exp(x - max) with their sum, then y *= 1 / sum.  Safe in place: the last pass reads only y.
__global__ void softmax_cols_kernel(const float* x, float* y, long long outer, long long len, long long inner) {
    const long long n = outer * inner;
    for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long o = t / inner, in = t - o * inner;
        const long long base = o * len * inner + in;
        float mx = -INFINITY;
        for (long long i = 0; i < len; ++i) mx = fmaxf(mx, x[base + i * inner]);
        float sum = 0.0f;
        for (long long i = 0; i < len; ++i) {
            const float e = expf(x[base + i * inner] - mx);
            y[base + i * inner] = e;
            sum += e;
        }
        const float inv = 1.0f / sum;
        for (long long i = 0; i < len; ++i) y[base + i * inner] *= inv;
    }
}

// ---- transpose ----------------------------------------------------------------------------------
struct PermArgs {
    int ndim;
    long long oshape[TZ_MAX_DIMS];   // output extents
    long long istride[TZ_MAX_DIMS];  // input element stride of the input dimension output d reads
};

template <typename E>
__global__ void permute_kernel(const E* __restrict__ x, E* __restrict__ y, PermArgs p, long long n) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        long long rem = i, off = 0;
        for (int d = p.ndim - 1; d >= 0; --d) {
            const long long q = rem / p.oshape[d];
            off += (rem - q * p.oshape[d]) * p.istride[d];
            rem = q;
        }
        y[i] = x[off];
    }
}

// ---- cast ---------------------------------------------------------------------------------------
template <typename S>
__device__ __forceinline__ double load_as_double(const void* x, long long i) {
    return static_cast<double>(static_cast<const S*>(x)[i]);
}

__device__ __forceinline__ double cast_load(const void* x, int dt, long long i) {
    switch (dt) {
        case TZ_DT_F32: return load_as_double<float>(x, i);
        case TZ_DT_F16: return static_cast<double>(__half2float(static_cast<const __half*>(x)[i]));
        case TZ_DT_I8: return load_as_double<int8_t>(x, i);
        case TZ_DT_I32: return load_as_double<int32_t>(x, i);
        case TZ_DT_I64: return load_as_double<long long>(x, i);
        default: return load_as_double<uint8_t>(x, i);  // TZ_DT_U8 (bool)
    }
}

__device__ __forceinline__ void cast_store(void* y, int dt, long long i, double v) {
    switch (dt) {
        case TZ_DT_F32: static_cast<float*>(y)[i] = static_cast<float>(v); break;
        case TZ_DT_F16: static_cast<__half*>(y)[i] = __float2half_rn(static_cast<float>(v)); break;
        case TZ_DT_I8: static_cast<int8_t*>(y)[i] = static_cast<int8_t>(static_cast<long long>(v)); break;
        case TZ_DT_I32: static_cast<int32_t*>(y)[i] = static_cast<int32_t>(static_cast<long long>(v)); break;
        case TZ_DT_I64: static_cast<long long*>(y)[i] = static_cast<long long>(v); break;
        default: static_cast<uint8_t*>(y)[i] = v != 0.0 ? 1 : 0; break;  // TZ_DT_U8 (bool)
    }
}

// Values round-trip through f64: exact for every f32, f16, 8/32-bit integer and for 64-bit
// integers up to 2^53 (the index and mask values ONNX graphs cast).
__global__ void cast_kernel(const void* x, int sdt, void* y, int ddt, long long n) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        cast_store(y, ddt, i, cast_load(x, sdt, i));
}

// ---- split-tf32 operands ------------------------------------------------------------------------
// dst row r (parts hi | lo [| hi]) from src element (r, k) at src[r * rs + k * cs]; k >= K is zero.
__global__ void split_tf32_kernel(const float* __restrict__ src, long long rs, long long cs, int rows, int K, int P,
                                  int parts, float* __restrict__ dst) {
    const long long n = static_cast<long long>(rows) * P;
    for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = t / P;
        const int k = static_cast<int>(t - r * P);
        const float x = k < K ? src[r * rs + k * cs] : 0.0f;
        const float hi = tzp::tf32_rna(x);
        const float lo = x - hi;  // exact: hi holds x's leading bits
        float* d = dst + r * static_cast<long long>(parts) * P;
        d[k] = hi;
        d[P + k] = lo;
        if (parts == 3) d[2 * P + k] = hi;
    }
}

bool is_dt(int d) {
    return d == TZ_DT_F32 || d == TZ_DT_F16 || d == TZ_DT_I8 || d == TZ_DT_I32 || d == TZ_DT_I64 || d == TZ_DT_U8;
}

}  // namespace
}  // namespace tz

using namespace tz;

extern "C" {

int tz_batched_matmul(tz_ctx_t ctx, const float* a, const float* b, float* c, const tz_bmm_layout* l,
                      tz_stream_t stream) {
    TZ_CHECK(ctx && a && b && c && l, TZ_EINVAL, "tz_batched_matmul: null argument");
    TZ_CHECK(l->batch_ndim >= 0 && l->batch_ndim <= 4 && l->m >= 0 && l->n >= 0 && l->k >= 0, TZ_EINVAL,
             "tz_batched_matmul: bad layout");
    BmmArgs p{};
    p.bnd = l->batch_ndim;
    p.nbatch = 1;
    for (int d = 0; d < p.bnd; ++d) {
        TZ_CHECK(l->batch_shape[d] >= 0, TZ_EINVAL, "tz_batched_matmul: negative batch extent");
        p.bshape[d] = l->batch_shape[d];
        p.as[d] = l->a_bstride[d];
        p.bs[d] = l->b_bstride[d];
        p.cs[d] = l->c_bstride[d];
        p.nbatch *= l->batch_shape[d];
    }
    p.a_rs = l->a_rs; p.a_cs = l->a_cs; p.b_rs = l->b_rs; p.b_cs = l->b_cs; p.c_rs = l->c_rs; p.c_cs = l->c_cs;
    p.m = l->m; p.k = l->k; p.n = l->n;
    if (p.nbatch == 0 || p.m == 0 || p.n == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const dim3 grid((p.n + 63) / 64, (p.m + 63) / 64,
                    static_cast<unsigned>(p.nbatch < 65535 ? p.nbatch : 65535));
    TZ_CHECK(grid.y <= 65535, TZ_EINVAL, "tz_batched_matmul: m = %d too large", p.m);
    bmm_kernel<<<grid, 256, 0, s>>>(a, b, c, p);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_matmul_f32x3(tz_ctx_t ctx, const float* a, const float* b, int trans_b, const float* bias, const int* ops,
                    int n_ops, float* c, int m, int k, int n, tz_stream_t stream) {
    TZ_CHECK(ctx && a && b && c && m >= 0 && k > 0 && n > 0 && n_ops >= 0 && n_ops <= 8 && (n_ops == 0 || ops), TZ_EINVAL,
             "tz_matmul_f32x3: bad arguments");
    for (int i = 0; i < n_ops; ++i)
        TZ_CHECK(ops[i] >= TZ_OP_ADD && ops[i] <= TZ_OP_LAST_UNARY, TZ_EINVAL, "tz_matmul_f32x3: bad op %d", ops[i]);
    if (m == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const int P = (k + 31) / 32 * 32;
    const size_t a_elems = static_cast<size_t>(m) * 2 * P, b_elems = static_cast<size_t>(n) * 3 * P;
    void* scratch = nullptr;
    int rc = scratch_reserve(ctx, sizeof(float) * (a_elems + b_elems) + 256, &scratch);
    if (rc) return rc;
    float* as = static_cast<float*>(scratch);
    float* bs = as + (a_elems + 63) / 64 * 64;  // 256-byte aligned
    split_tf32_kernel<<<grid_for(ctx, static_cast<long long>(m) * P, 256), 256, 0, s>>>(a, k, 1, m, k, P, 2, as);
    // b [n, k] (trans_b) or [k, n]: element (j, kk) of the [n, k] view
    split_tf32_kernel<<<grid_for(ctx, static_cast<long long>(n) * P, 256), 256, 0, s>>>(
        b, trans_b ? k : 1, trans_b ? 1 : n, n, k, P, 3, bs);
    TZ_CUDA(cudaGetLastError());
    GemmArgs g;
    g.kind = KIND_TF32;
    g.a3x = true;
    g.a = as; g.lda = 2 * P; g.b = bs; g.ldb = 3 * P; g.M = m; g.N = n; g.K = 3 * P;
    g.out = c; g.ldo = n; g.out_type = OUT_F32;
    const bool has_add = n_ops >= 1 && ops[0] == TZ_OP_ADD;
    const int act = n_ops == (has_add ? 2 : 1) ? ops[n_ops - 1] : 0;
    if (n_ops == 0 || (n_ops == 1 && has_add) || (n_ops <= 2 && (act == TZ_OP_GELU || act == TZ_OP_RELU))) {
        g.bias = has_add ? bias : nullptr;
        g.gelu = act == TZ_OP_GELU ? 2 : act == TZ_OP_RELU ? 3 : 0;
        return launch_gemm(ctx, g, s);
    }
    g.bias = bias;
    g.n_ops = n_ops;
    for (int i = 0; i < n_ops; ++i) g.ops[i] = ops[i];
    return launch_gemm(ctx, g, s);
}

int tz_reduce_axis(tz_ctx_t ctx, int reduce_op, const float* x, int64_t outer, int64_t len, int64_t inner, float* out,
                   tz_stream_t stream) {
    TZ_CHECK(ctx && x && out && outer >= 0 && len > 0 && inner > 0 && reduce_op >= TZ_RED_SUM && reduce_op <= TZ_RED_MIN,
             TZ_EINVAL, "tz_reduce_axis: bad arguments");
    if (outer == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    if (inner == 1)
        reduce_rows_kernel<<<grid_for(ctx, outer * 32, 256), 256, 0, s>>>(x, outer, len, reduce_op, out);
    else
        reduce_cols_kernel<<<grid_for(ctx, outer * inner, 256), 256, 0, s>>>(x, outer, len, inner, reduce_op, out);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_softmax_axis(tz_ctx_t ctx, const float* x, float* y, int64_t outer, int64_t len, int64_t inner, tz_stream_t stream) {
    TZ_CHECK(ctx && x && y && outer >= 0 && len > 0 && inner > 0, TZ_EINVAL, "tz_softmax_axis: bad arguments");
    if (outer == 0) return TZ_OK;
    if (inner == 1 && len <= 0x7fffffff) return tz_softmax_last_axis(ctx, x, nullptr, y, outer, static_cast<int>(len), stream);
    cudaStream_t s = pick_stream(ctx, stream);
    softmax_cols_kernel<<<grid_for(ctx, outer * inner, 256), 256, 0, s>>>(x, y, outer, len, inner);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_permute(tz_ctx_t ctx, const void* x, void* y, int elem_bytes, int ndim, const int64_t* shape, const int* perm,
               tz_stream_t stream) {
    TZ_CHECK(ctx && x && y && (ndim == 0 || (shape && perm)) && ndim >= 0 && ndim <= TZ_MAX_DIMS, TZ_EINVAL,
             "tz_permute: bad arguments");
    TZ_CHECK(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4 || elem_bytes == 8, TZ_EINVAL,
             "tz_permute: element size %d", elem_bytes);
    PermArgs p{};
    p.ndim = ndim;
    long long istr[TZ_MAX_DIMS];
    long long n = 1;
    for (int d = ndim - 1; d >= 0; --d) {
        TZ_CHECK(shape[d] >= 0, TZ_EINVAL, "tz_permute: negative extent");
        istr[d] = n;
        n *= shape[d];
    }
    unsigned seen = 0;
    for (int d = 0; d < ndim; ++d) {
        TZ_CHECK(perm[d] >= 0 && perm[d] < ndim && !(seen & (1u << perm[d])), TZ_EINVAL, "tz_permute: bad permutation");
        seen |= 1u << perm[d];
        p.oshape[d] = shape[perm[d]];
        p.istride[d] = istr[perm[d]];
    }
    if (n == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const int g = grid_for(ctx, n, 256);
    switch (elem_bytes) {
        case 1: permute_kernel<uint8_t><<<g, 256, 0, s>>>(static_cast<const uint8_t*>(x), static_cast<uint8_t*>(y), p, n); break;
        case 2: permute_kernel<uint16_t><<<g, 256, 0, s>>>(static_cast<const uint16_t*>(x), static_cast<uint16_t*>(y), p, n); break;
        case 4: permute_kernel<uint32_t><<<g, 256, 0, s>>>(static_cast<const uint32_t*>(x), static_cast<uint32_t*>(y), p, n); break;
        default: permute_kernel<unsigned long long><<<g, 256, 0, s>>>(static_cast<const unsigned long long*>(x),
                                                                     static_cast<unsigned long long*>(y), p, n); break;
    }
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_cast(tz_ctx_t ctx, const void* x, int src_dtype, void* y, int dst_dtype, int64_t n, tz_stream_t stream) {
    TZ_CHECK(ctx && (n == 0 || (x && y)) && n >= 0, TZ_EINVAL, "tz_cast: bad arguments");
    TZ_CHECK(is_dt(src_dtype) && is_dt(dst_dtype), TZ_EUNSUPPORTED, "tz_cast: dtype %d -> %d", src_dtype, dst_dtype);
    if (n == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    cast_kernel<<<grid_for(ctx, n, 256), 256, 0, s>>>(x, src_dtype, y, dst_dtype, n);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_concat(tz_ctx_t ctx, const void* const* inputs, const int64_t* axis_len, int n_inputs, int64_t outer, int64_t inner,
              int elem_bytes, void* out, tz_stream_t stream) {
    TZ_CHECK(ctx && inputs && axis_len && out && n_inputs > 0 && outer >= 0 && inner >= 0 && elem_bytes > 0, TZ_EINVAL,
             "tz_concat: bad arguments");
    int64_t total = 0;
    for (int i = 0; i < n_inputs; ++i) {
        TZ_CHECK(axis_len[i] >= 0 && (axis_len[i] == 0 || inputs[i]), TZ_EINVAL, "tz_concat: input %d", i);
        total += axis_len[i];
    }
    if (outer == 0 || inner == 0 || total == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const size_t dpitch = static_cast<size_t>(total) * inner * elem_bytes;
    size_t off = 0;
    for (int i = 0; i < n_inputs; ++i) {
        const size_t w = static_cast<size_t>(axis_len[i]) * inner * elem_bytes;
        if (w)
            TZ_CUDA(cudaMemcpy2DAsync(static_cast<char*>(out) + off, dpitch, inputs[i], w, w, static_cast<size_t>(outer),
                                      cudaMemcpyDeviceToDevice, s));
        off += w;
    }
    return TZ_OK;
}

}  // extern "C"
