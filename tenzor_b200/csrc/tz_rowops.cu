// tz_rowops.cu -- HBM-bound row and elementwise kernels: LayerNorm, softmax (additive mask and
// key-length mask), quantisers, converters, fused elementwise chains, fused reduce, row gather.
// Each is one pass over its data with 16-byte coalesced accesses: warp-per-row for the row ops
// (shuffle reductions, the row stays in registers between the passes), grid-stride float4 loops
// sized to a multiple of the SM count for the elementwise ops.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tz_internal.h"
#include "tz_ptx.cuh"
#include "tz_rowops.cuh"

namespace tz {
namespace {

// ---- LayerNorm (layernorm.zig:26-116) ----------------------------------------------------------
// Warp per R rows; VPL float4 per lane and row kept in registers (cols == VPL*128).  The R rows'
// loads are all issued before the first reduction, so a warp keeps R x 512 x VPL bytes in flight
// and the grid needs fewer waves.
template <int VPL, int R>
__global__ void ln_rows_reg_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                   const float* __restrict__ b, float* y, long long rows, int cols,
                                   float eps) {
    const long long row0 = ((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * R;
    const int lane = threadIdx.x & 31;
    if (row0 >= rows) return;
    float4 v[R][VPL];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float4* xr = reinterpret_cast<const float4*>(x + (row0 + r) * cols);
#pragma unroll
        for (int i = 0; i < VPL; ++i) v[r][i] = (row0 + r < rows) ? xr[lane + 32 * i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mean[R], inv_std[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) s += (v[r][i].x + v[r][i].y) + (v[r][i].z + v[r][i].w);
        mean[r] = warp_sum(s) / static_cast<float>(cols);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const float a = v[r][i].x - mean[r], bb = v[r][i].y - mean[r], c = v[r][i].z - mean[r], d = v[r][i].w - mean[r];
            q += (a * a + bb * bb) + (c * c + d * d);
        }
        inv_std[r] = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(cols) + eps);
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c4 = lane + 32 * i;
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g) + c4);
        const float4 bb = __ldg(reinterpret_cast<const float4*>(b) + c4);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (row0 + r >= rows) continue;
            float4 o;
            o.x = (v[r][i].x - mean[r]) * inv_std[r] * gg.x + bb.x;
            o.y = (v[r][i].y - mean[r]) * inv_std[r] * gg.y + bb.y;
            o.z = (v[r][i].z - mean[r]) * inv_std[r] * gg.z + bb.z;
            o.w = (v[r][i].w - mean[r]) * inv_std[r] * gg.w + bb.w;
            reinterpret_cast<float4*>(y + (row0 + r) * cols)[c4] = o;
        }
    }
}

// Any width: warp per row, three passes over the (L1/L2-resident) row.
__global__ void ln_rows_any_kernel(const float* x, const float* __restrict__ g,
                                   const float* __restrict__ b, float* y, long long rows, int cols,
                                   float eps) {
    const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * cols;
    float s = 0.f;
    for (int c = lane; c < cols; c += 32) s += xr[c];
    const float mean = warp_sum(s) / static_cast<float>(cols);
    float q = 0.f;
    for (int c = lane; c < cols; c += 32) {
        const float d = xr[c] - mean;
        q += d * d;
    }
    const float inv_std = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(cols) + eps);
    __syncwarp();
    float* yr = y + row * cols;
    for (int c = lane; c < cols; c += 32) yr[c] = (xr[c] - mean) * inv_std * g[c] + b[c];
}

// ---- softmax (softmax.zig:56-155) --------------------------------------------------------------
// Warp per row; additive mask (may be null); key_len (per group of rows_per_group rows) masks
// columns >= key_len with probability 0 (the -inf additive mask).
__global__ void softmax_rows_kernel(const float* x, const float* mask, const int* key_len,
                                    int rows_per_group, float* y, long long rows, int cols) {
    const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * cols;
    const float* mr = mask ? mask + row * cols : nullptr;
    const int valid = key_len ? min(max(key_len[row / rows_per_group], 0), cols) : cols;
    float* yr = y + row * cols;
    float mx = -INFINITY;
    for (int c = lane; c < valid; c += 32) mx = fmaxf(mx, mr ? xr[c] + mr[c] : xr[c]);
    mx = warp_max(mx);
    float s = 0.f;
    for (int c = lane; c < valid; c += 32) s += expf((mr ? xr[c] + mr[c] : xr[c]) - mx);
    s = warp_sum(s);
    const float inv = 1.0f / s;
    __syncwarp();
    for (int c = lane; c < cols; c += 32)
        yr[c] = (c < valid) ? expf((mr ? xr[c] + mr[c] : xr[c]) - mx) * inv : 0.0f;
}

// Fast path for cols == 128 (the Arctic attention shape at S=128): a row is one float4 per lane;
// a warp takes R rows and issues all their loads before the first reduction.  I32: every row index
// fits 31 bits, so the group of a row is a 32-bit division (the 64-bit one is a long call sequence
// on the key-length load's critical path).
template <int R, bool I32>
__global__ void softmax_rows128_kernel(const float* x, const float* mask, const int* key_len,
                                       int rows_per_group, float* y, long long rows) {
    const long long row0 = ((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * R;
    const int lane = threadIdx.x & 31;
    if (row0 >= rows) return;
    float4 v[R];
    int valid[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const long long row = row0 + r;
        const bool in = row < rows;
        v[r] = in ? reinterpret_cast<const float4*>(x + row * 128)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
        if (mask && in) {
            const float4 m = reinterpret_cast<const float4*>(mask + row * 128)[lane];
            v[r].x += m.x; v[r].y += m.y; v[r].z += m.z; v[r].w += m.w;
        }
        const long long grp = I32 ? static_cast<long long>(static_cast<unsigned>(row) / static_cast<unsigned>(rows_per_group))
                                  : row / rows_per_group;
        valid[r] = (key_len && in) ? min(max(key_len[grp], 0), 128) : 128;
    }
    const int c = lane * 4;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const long long row = row0 + r;
        if (c + 0 >= valid[r]) v[r].x = -INFINITY;
        if (c + 1 >= valid[r]) v[r].y = -INFINITY;
        if (c + 2 >= valid[r]) v[r].z = -INFINITY;
        if (c + 3 >= valid[r]) v[r].w = -INFINITY;
        const float mx = warp_max(fmaxf(fmaxf(v[r].x, v[r].y), fmaxf(v[r].z, v[r].w)));
        float4 e;
        e.x = (c + 0 < valid[r]) ? expf(v[r].x - mx) : 0.f;
        e.y = (c + 1 < valid[r]) ? expf(v[r].y - mx) : 0.f;
        e.z = (c + 2 < valid[r]) ? expf(v[r].z - mx) : 0.f;
        e.w = (c + 3 < valid[r]) ? expf(v[r].w - mx) : 0.f;
        const float inv = 1.0f / warp_sum((e.x + e.y) + (e.z + e.w));
        e.x *= inv; e.y *= inv; e.z *= inv; e.w *= inv;
        if (row < rows) reinterpret_cast<float4*>(y + row * 128)[lane] = e;
    }
}

// ---- quantisers ---------------------------------------------------------------------------------
// quantize_arctic_xs.zig:94-115 (f16 scale) when F16SCALE, else the per-token activation rule.
template <bool F16SCALE>
__global__ void quant_rows_kernel(const float* x, int8_t* q, void* scale, long long rows, int cols) {
    const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * cols;
    float m = 0.f;
    for (int c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(xr[c]));
    m = warp_max(m);
    float s = (m == 0.0f) ? 1.0f : __fdiv_rn(m, 127.0f);
    if constexpr (F16SCALE) {
        const __half h = __float2half_rn(s);
        if (lane == 0) reinterpret_cast<__half*>(scale)[row] = h;
        s = __half2float(h);
    } else {
        if (lane == 0) reinterpret_cast<float*>(scale)[row] = s;
    }
    const float inv = __fdiv_rn(1.0f, s);
    int8_t* qr = q + row * cols;
    if constexpr (F16SCALE) {  // weights: the f16-rounded scale can put |x / s| a little past 127
        for (int c = lane; c < cols; c += 32) qr[c] = quant1(xr[c], inv);
    } else {  // activations: quantised against their own |max| (the form the fused GEMM path uses)
        const uint64_t inv2 = tzp::f2_pack(inv, inv);
        for (int c = 2 * lane; c < cols; c += 64) {
            const float x1 = c + 1 < cols ? xr[c + 1] : 0.0f;
            const uint32_t b = quant2_own_max(xr[c], x1, inv2);
            qr[c] = static_cast<int8_t>(b & 0xFFu);
            if (c + 1 < cols) qr[c + 1] = static_cast<int8_t>((b >> 8) & 0xFFu);
        }
    }
}

// ---- converters ---------------------------------------------------------------------------------
__global__ void f32_to_f16_kernel(const float* x, __half* y, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = __float2half_rn(x[i]);
}
__global__ void i8_to_f16_kernel(const int8_t* x, __half* y, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = __int2half_rn(static_cast<int>(x[i]));
}
__global__ void f32_to_bf16_kernel(const float* x, __nv_bfloat16* y, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = __float2bfloat16_rn(x[i]);
}
__global__ void i8_to_bf16_kernel(const int8_t* x, __nv_bfloat16* y, long long n) {  // exact: |q| <= 127
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = __float2bfloat16_rn(static_cast<float>(x[i]));
}
__global__ void f16bits_to_f32_kernel(const uint16_t* x, float* y, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = __half2float(__ushort_as_half(x[i]));
}
__global__ void transpose_kernel(const float* x, float* y, int rows, int cols) {
    __shared__ float tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = by + j, c = bx + threadIdx.x;
        if (r < rows && c < cols) tile[j][threadIdx.x] = x[static_cast<long long>(r) * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = bx + j, c = by + threadIdx.x;  // y is [cols, rows]
        if (r < cols && c < rows) y[static_cast<long long>(r) * rows + c] = tile[threadIdx.x][j];
    }
}

// ---- elementwise chains -------------------------------------------------------------------------
// exp((a + b) * c), b broadcast along rows: the executor's three passes fused into one.
__global__ void ew_add_mul_exp_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                      const float4* __restrict__ c, float4* __restrict__ out,
                                      long long n4, int cols4) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float4 av = __ldcs(a + i);
        const float4 cv = __ldcs(c + i);
        const float4 bv = __ldg(b + (i % cols4));
        float4 o;
        o.x = expf((av.x + bv.x) * cv.x);
        o.y = expf((av.y + bv.y) * cv.y);
        o.z = expf((av.z + bv.z) * cv.z);
        o.w = expf((av.w + bv.w) * cv.w);
        __stcs(out + i, o);
    }
}
__global__ void ew_add_mul_exp_any_kernel(const float* a, const float* b, const float* c, float* out,
                                          long long n, int cols) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = expf((a[i] + b[i % cols]) * c[i]);
}

struct OpList {
    int n;
    int op[8];
};

__global__ void ew_unary_chain_kernel(const float* x, float* out, long long n, OpList ops) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        float v = x[i];
        for (int o = 0; o < ops.n; ++o) v = unary_op(ops.op[o], v);
        out[i] = v;
    }
}

// One pass over [rows, cols] evaluating a small register program per element.
struct EwProgram {
    int n_in;
    const float* in[4];
    long long rs[4], cs[4];
    int n_instr;
    int op[16], dst[16], a[16], b[16], c[16];
    int result;
    float consts[4];
};

// The program's instructions over one element whose inputs are in reg[0..3]; returns reg[result].
__device__ __forceinline__ float run_program(const EwProgram& p, float (&reg)[16]) {
#pragma unroll
    for (int k = 4; k < 12; ++k) reg[k] = 0.0f;
#pragma unroll
    for (int k = 12; k < 16; ++k) reg[k] = p.consts[k - 12];
    for (int t = 0; t < p.n_instr; ++t) {
        float va = 0.f, vb = 0.f, vc = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {  // register reads by unrolled select: no local memory
            va = (k == p.a[t]) ? reg[k] : va;
            vb = (k == p.b[t]) ? reg[k] : vb;
            vc = (k == p.c[t]) ? reg[k] : vc;
        }
        const float res = p.op[t] == TZ_EW_WHERE ? (va != 0.0f ? vb : vc) : binary_op(p.op[t], va, vb);
#pragma unroll
        for (int k = 4; k < 12; ++k) reg[k] = (k == p.dst[t]) ? res : reg[k];
    }
    float o = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) o = (k == p.result) ? reg[k] : o;
    return o;
}

__global__ void ew_program_kernel(EwProgram p, float* __restrict__ out, long long rows, int cols) {
    const long long n = rows * cols;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / cols, c = i - r * cols;
        float reg[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) reg[k] = k < p.n_in ? __ldg(p.in[k] + r * p.rs[k] + c * p.cs[k]) : 0.0f;
        out[i] = run_program(p, reg);
    }
}

// N-D broadcast form (executor.zig:152-197 evalBinaryBroadcast, any rank up to TZ_MAX_DIMS): the
// output is row-major [shape]; input k of output element idx is at sum_d idx[d] * stride[k][d]
// (stride 0 along a broadcast dimension).
struct NdLayout {
    int ndim;
    long long shape[TZ_MAX_DIMS];
    long long stride[4][TZ_MAX_DIMS];
};

__global__ void ew_program_nd_kernel(EwProgram p, NdLayout l, float* __restrict__ out, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        long long off[4] = {0, 0, 0, 0};
        long long rem = i;
        for (int d = l.ndim - 1; d >= 0; --d) {
            const long long q = rem / l.shape[d];
            const long long x = rem - q * l.shape[d];
            rem = q;
#pragma unroll
            for (int k = 0; k < 4; ++k) off[k] += x * l.stride[k][d];
        }
        float reg[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) reg[k] = k < p.n_in ? __ldg(p.in[k] + off[k]) : 0.0f;
        out[i] = run_program(p, reg);
    }
}

// Fused pre-ops + reduction.  Stage 1: per-block partials (f64 for sum/mean); stage 2: one block.
__global__ void reduce_stage1_kernel(const float* x, long long n, int red, OpList pre, double* part) {
    double acc = (red == TZ_RED_PROD) ? 1.0 : (red == TZ_RED_MAX) ? -INFINITY : (red == TZ_RED_MIN) ? INFINITY : 0.0;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        float v = x[i];
        for (int o = 0; o < pre.n; ++o) v = unary_op(pre.op[o], v);
        acc = red_combine(red, acc, static_cast<double>(v));
    }
    __shared__ double sh[32];
    acc = block_reduce(red, acc, sh);
    if (threadIdx.x == 0) part[blockIdx.x] = acc;
}
__global__ void reduce_stage2_kernel(const double* part, int nparts, long long n, int red, float* out) {
    double acc = (red == TZ_RED_PROD) ? 1.0 : (red == TZ_RED_MAX) ? -INFINITY : (red == TZ_RED_MIN) ? INFINITY : 0.0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) acc = red_combine(red, acc, part[i]);
    __shared__ double sh[32];
    acc = block_reduce(red, acc, sh);
    if (threadIdx.x == 0) {
        if (red == TZ_RED_MEAN && n > 0) acc /= static_cast<double>(n);
        *out = static_cast<float>(acc);
    }
}

// gather.zig:15-57 with the device status word in place of the safe-build bounds check.
__global__ void gather_rows_kernel(const float* table, long long table_rows, const uint32_t* ids,
                                   long long n_ids, int cols, float* out, int* status) {
    const long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n_ids) return;
    const uint32_t id = ids[r];
    const bool ok = id < table_rows;
    if (!ok && lane == 0) atomicOr(status, TZ_DEV_BOUNDS);
    const float* src = table + static_cast<long long>(ok ? id : 0) * cols;
    float* dst = out + r * cols;
    for (int c = lane; c < cols; c += 32) dst[c] = ok ? src[c] : 0.0f;
}

inline int ew_grid(tz_ctx_t ctx, long long work, int threads) {
    long long blocks = (work + threads - 1) / threads;
    const long long cap = static_cast<long long>(ctx->sm_count) * 8;
    if (blocks > cap) blocks = cap;
    return static_cast<int>(blocks < 1 ? 1 : blocks);
}

inline int warp_rows_grid(long long rows) { return static_cast<int>((rows * 32 + 255) / 256); }
inline int warp_rows_grid_r(long long rows, int r) { return warp_rows_grid((rows + r - 1) / r); }

}  // namespace

// ---- launchers shared with the model -----------------------------------------------------------
int launch_f32_to_f16(tz_ctx_t ctx, const float* x, void* y, long long n, cudaStream_t s) {
    f32_to_f16_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(x, static_cast<__half*>(y), n);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}
int launch_f32_to_bf16(tz_ctx_t ctx, const float* x, void* y, long long n, cudaStream_t s) {
    f32_to_bf16_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(x, static_cast<__nv_bfloat16*>(y), n);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}
int launch_i8_to_bf16(tz_ctx_t ctx, const int8_t* x, void* y, long long n, cudaStream_t s) {
    i8_to_bf16_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(x, static_cast<__nv_bfloat16*>(y), n);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}
int launch_i8_to_f16(tz_ctx_t ctx, const int8_t* x, void* y, long long n, cudaStream_t s) {
    i8_to_f16_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(x, static_cast<__half*>(y), n);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}
int launch_f16bits_to_f32(tz_ctx_t ctx, const uint16_t* x, float* y, long long n, cudaStream_t s) {
    f16bits_to_f32_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(x, y, n);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}
int launch_quant_act(tz_ctx_t ctx, const float* x, int8_t* q, float* scale, long long rows, int cols,
                     cudaStream_t s) {
    if (rows == 0) return TZ_OK;
    quant_rows_kernel<false><<<warp_rows_grid(rows), 256, 0, s>>>(x, q, scale, rows, cols);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

}  // namespace tz

using namespace tz;

extern "C" {

int tz_layernorm_last_dim(tz_ctx_t ctx, const float* x, const float* gamma, const float* beta,
                          float* y, int64_t rows, int cols, float eps, tz_stream_t stream) {
    TZ_CHECK(ctx && x && gamma && beta && y && rows >= 0 && cols > 0, TZ_EINVAL,
             "tz_layernorm_last_dim: bad arguments");
    if (rows == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const bool al = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(gamma) % 16 == 0 && reinterpret_cast<uintptr_t>(beta) % 16 == 0;
    const int g = warp_rows_grid(rows);
    if (al && cols == 384)
        ln_rows_reg_kernel<3, 2><<<warp_rows_grid_r(rows, 2), 256, 0, s>>>(x, gamma, beta, y, rows, cols, eps);
    else if (al && cols == 128)
        ln_rows_reg_kernel<1, 2><<<warp_rows_grid_r(rows, 2), 256, 0, s>>>(x, gamma, beta, y, rows, cols, eps);
    else if (al && cols == 256)
        ln_rows_reg_kernel<2, 2><<<warp_rows_grid_r(rows, 2), 256, 0, s>>>(x, gamma, beta, y, rows, cols, eps);
    else if (al && cols == 512)
        ln_rows_reg_kernel<4, 2><<<warp_rows_grid_r(rows, 2), 256, 0, s>>>(x, gamma, beta, y, rows, cols, eps);
    else if (al && cols == 768)
        ln_rows_reg_kernel<6, 1><<<warp_rows_grid_r(rows, 1), 256, 0, s>>>(x, gamma, beta, y, rows, cols, eps);
    else if (al && cols == 1024)
        ln_rows_reg_kernel<8, 1><<<warp_rows_grid_r(rows, 1), 256, 0, s>>>(x, gamma, beta, y, rows, cols, eps);
    else
        ln_rows_any_kernel<<<g, 256, 0, s>>>(x, gamma, beta, y, rows, cols, eps);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_softmax_last_axis(tz_ctx_t ctx, const float* x, const float* mask, float* y, int64_t rows,
                         int cols, tz_stream_t stream) {
    TZ_CHECK(ctx && x && y && rows >= 0 && cols >= 0, TZ_EINVAL, "tz_softmax_last_axis: bad arguments");
    if (rows == 0 || cols == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const bool al = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 &&
                    (!mask || reinterpret_cast<uintptr_t>(mask) % 16 == 0);
    if (cols == 128 && al)
        softmax_rows128_kernel<2, false><<<warp_rows_grid_r(rows, 2), 256, 0, s>>>(x, mask, nullptr, 1, y, rows);
    else
        softmax_rows_kernel<<<warp_rows_grid(rows), 256, 0, s>>>(x, mask, nullptr, 1, y, rows, cols);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_softmax_keylen(tz_ctx_t ctx, const float* x, const int32_t* key_len, float* y, int64_t groups,
                      int rows_per_group, int cols, tz_stream_t stream) {
    TZ_CHECK(ctx && x && y && key_len && groups >= 0 && rows_per_group > 0 && cols > 0, TZ_EINVAL,
             "tz_softmax_keylen: bad arguments");
    const long long rows = groups * static_cast<long long>(rows_per_group);
    if (rows == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const bool al = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
    if (cols == 128 && al)
        if (rows + 4 < (1ll << 31))
            softmax_rows128_kernel<2, true><<<warp_rows_grid_r(rows, 2), 256, 0, s>>>(x, nullptr, key_len, rows_per_group, y, rows);
        else
            softmax_rows128_kernel<4, false><<<warp_rows_grid_r(rows, 4), 256, 0, s>>>(x, nullptr, key_len, rows_per_group, y, rows);
    else
        softmax_rows_kernel<<<warp_rows_grid(rows), 256, 0, s>>>(x, nullptr, key_len, rows_per_group, y, rows, cols);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_quantize_weight_rows(tz_ctx_t ctx, const float* w, int8_t* q, uint16_t* scale_f16, int64_t rows,
                            int cols, tz_stream_t stream) {
    TZ_CHECK(ctx && w && q && scale_f16 && rows >= 0 && cols > 0, TZ_EINVAL,
             "tz_quantize_weight_rows: bad arguments");
    if (rows == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    quant_rows_kernel<true><<<warp_rows_grid(rows), 256, 0, s>>>(w, q, scale_f16, rows, cols);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_quantize_act_rows(tz_ctx_t ctx, const float* x, int8_t* q, float* scale, int64_t rows, int cols,
                         tz_stream_t stream) {
    TZ_CHECK(ctx && x && q && scale && rows >= 0 && cols > 0, TZ_EINVAL, "tz_quantize_act_rows: bad arguments");
    return launch_quant_act(ctx, x, q, scale, rows, cols, pick_stream(ctx, stream));
}

int tz_ew_add_mul_exp(tz_ctx_t ctx, const float* a, const float* b_row, const float* c, float* out,
                      int64_t rows, int cols, tz_stream_t stream) {
    TZ_CHECK(ctx && a && b_row && c && out && rows >= 0 && cols > 0, TZ_EINVAL, "tz_ew_add_mul_exp: bad arguments");
    const long long n = rows * static_cast<long long>(cols);
    if (n == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const bool al = cols % 4 == 0 && reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(c) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(out) % 16 == 0 && reinterpret_cast<uintptr_t>(b_row) % 16 == 0;
    if (al)
        ew_add_mul_exp_kernel<<<ew_grid(ctx, n / 4, 256), 256, 0, s>>>(
            reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b_row),
            reinterpret_cast<const float4*>(c), reinterpret_cast<float4*>(out), n / 4, cols / 4);
    else
        ew_add_mul_exp_any_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(a, b_row, c, out, n, cols);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

}  // extern "C"

namespace {
// Checks a tz_ew_program and converts it to the kernel's form.
int load_program(const tz_ew_program* prog, EwProgram* out, const char* who) {
    TZ_CHECK(prog->n_inputs >= 1 && prog->n_inputs <= TZ_EW_MAX_INPUTS && prog->n_instr >= 0 &&
                 prog->n_instr <= TZ_EW_MAX_INSTR && prog->result >= 0 && prog->result < 16,
             TZ_EINVAL, "%s: bad program shape", who);
    EwProgram& p = *out;
    p = EwProgram{};
    p.n_in = prog->n_inputs;
    for (int k = 0; k < p.n_in; ++k) {
        TZ_CHECK(prog->in[k], TZ_EINVAL, "%s: input %d is null", who, k);
        p.in[k] = prog->in[k];
        p.rs[k] = prog->row_stride[k];
        p.cs[k] = prog->col_stride[k];
    }
    p.n_instr = prog->n_instr;
    for (int t = 0; t < p.n_instr; ++t) {
        const tz_ew_instr& in = prog->instr[t];
        const bool unary = in.op >= TZ_OP_RELU && in.op <= TZ_OP_LAST_UNARY;
        const bool binary = in.op >= TZ_EW_ADD && in.op <= TZ_EW_GT;
        const bool ternary = in.op == TZ_EW_WHERE;
        TZ_CHECK((unary || binary || ternary) && in.dst >= 4 && in.dst < 12 && in.a >= 0 && in.a < 16 &&
                     (unary || (in.b >= 0 && in.b < 16)) && (!ternary || (in.c >= 0 && in.c < 16)),
                 TZ_EINVAL, "%s: bad instruction %d", who, t);
        p.op[t] = in.op;
        p.dst[t] = in.dst;
        p.a[t] = in.a;
        p.b[t] = unary ? 0 : in.b;
        p.c[t] = ternary ? in.c : 0;
    }
    p.result = prog->result;
    for (int k = 0; k < 4; ++k) p.consts[k] = prog->consts[k];
    return TZ_OK;
}
}  // namespace

extern "C" {

int tz_ew_program_run(tz_ctx_t ctx, const tz_ew_program* prog, float* out, int64_t rows, int cols,
                      tz_stream_t stream) {
    TZ_CHECK(ctx && prog && out && rows >= 0 && cols > 0, TZ_EINVAL, "tz_ew_program_run: bad arguments");
    EwProgram p;
    int rc = load_program(prog, &p, "tz_ew_program_run");
    if (rc) return rc;
    const long long n = rows * static_cast<long long>(cols);
    if (n == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    ew_program_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(p, out, rows, cols);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_ew_program_run_nd(tz_ctx_t ctx, const tz_ew_program* prog, const tz_nd_layout* layout, float* out,
                         tz_stream_t stream) {
    TZ_CHECK(ctx && prog && layout && out, TZ_EINVAL, "tz_ew_program_run_nd: null argument");
    TZ_CHECK(layout->ndim >= 0 && layout->ndim <= TZ_MAX_DIMS, TZ_EINVAL, "tz_ew_program_run_nd: rank %d", layout->ndim);
    EwProgram p;
    int rc = load_program(prog, &p, "tz_ew_program_run_nd");
    if (rc) return rc;
    NdLayout l{};
    l.ndim = layout->ndim;
    long long n = 1;
    for (int d = 0; d < l.ndim; ++d) {
        TZ_CHECK(layout->shape[d] >= 0, TZ_EINVAL, "tz_ew_program_run_nd: negative extent");
        l.shape[d] = layout->shape[d];
        n *= l.shape[d];
        for (int k = 0; k < 4; ++k) l.stride[k][d] = layout->stride[k][d];
    }
    if (n == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    ew_program_nd_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(p, l, out, n);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_ew_unary_chain(tz_ctx_t ctx, const float* x, float* out, int64_t n, const int* ops, int n_ops,
                      tz_stream_t stream) {
    TZ_CHECK(ctx && x && out && n >= 0 && n_ops >= 0 && n_ops <= 8 && (n_ops == 0 || ops), TZ_EINVAL,
             "tz_ew_unary_chain: bad arguments");
    if (n == 0) return TZ_OK;
    OpList l{};
    l.n = n_ops;
    for (int i = 0; i < n_ops; ++i) {
        TZ_CHECK(ops[i] >= TZ_OP_RELU && ops[i] <= TZ_OP_LAST_UNARY, TZ_EINVAL, "tz_ew_unary_chain: op %d is not unary", ops[i]);
        l.op[i] = ops[i];
    }
    cudaStream_t s = pick_stream(ctx, stream);
    ew_unary_chain_kernel<<<ew_grid(ctx, n, 256), 256, 0, s>>>(x, out, n, l);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_reduce(tz_ctx_t ctx, int reduce_op, const int* pre_ops, int n_pre, const float* x, int64_t n,
              float* out, tz_stream_t stream) {
    TZ_CHECK(ctx && out && (n == 0 || x) && n >= 0 && reduce_op >= 0 && reduce_op <= 4 && n_pre >= 0 && n_pre <= 8 &&
                 (n_pre == 0 || pre_ops),
             TZ_EINVAL, "tz_reduce: bad arguments");
    OpList l{};
    l.n = n_pre;
    for (int i = 0; i < n_pre; ++i) {
        TZ_CHECK(pre_ops[i] >= TZ_OP_RELU && pre_ops[i] <= TZ_OP_LAST_UNARY, TZ_EINVAL, "tz_reduce: op %d is not unary", pre_ops[i]);
        l.op[i] = pre_ops[i];
    }
    cudaStream_t s = pick_stream(ctx, stream);
    const int parts = ew_grid(ctx, n > 0 ? n : 1, 256);
    void* scratch = nullptr;
    int rc = scratch_reserve(ctx, sizeof(double) * parts, &scratch);
    if (rc) return rc;
    double* part = static_cast<double*>(scratch);
    reduce_stage1_kernel<<<parts, 256, 0, s>>>(x, n, reduce_op, l, part);
    reduce_stage2_kernel<<<1, 256, 0, s>>>(part, parts, n, reduce_op, out);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int tz_gather_rows(tz_ctx_t ctx, const float* table, int64_t table_rows, const uint32_t* ids, int64_t n_ids,
                   int cols, float* out, tz_stream_t stream) {
    TZ_CHECK(ctx && table && ids && out && n_ids >= 0 && cols > 0, TZ_EINVAL, "tz_gather_rows: bad arguments");
    if (n_ids == 0) return TZ_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    gather_rows_kernel<<<warp_rows_grid(n_ids), 256, 0, s>>>(table, table_rows, ids, n_ids, cols, out, ctx->d_status);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

}  // extern "C"

namespace tz {
int launch_transpose(const float* x, float* y, int rows, int cols, cudaStream_t s) {
    dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
    transpose_kernel<<<grid, block, 0, s>>>(x, y, rows, cols);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}
}  // namespace tz
