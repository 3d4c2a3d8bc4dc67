// tz_rowops.cuh -- device helpers shared by the row kernels and the model kernels.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "tz_ptx.cuh"

#include "../../include/tenzor_cuda.h"

namespace tz {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// q = clamp(round(x * inv), -127, 127), round half away from zero (Zig @round / C roundf), with
// q's two's-complement byte in the low 8 bits of the result.  Computed with adds on the FMA pipe
// instead of a round + float-to-int conversion pair (both on the narrow conversion pipe):
//   t = clamp(x * inv, -127, 127)             (clamping first is equivalent: round is monotonic and
//                                               +-127 are integers; NaN -> -127 as fmaxf drops it)
//   a = RD(|t| + 0.5)                          (rounding down keeps floor(a) = floor(|t| + 0.5))
//   f = RD(a + 2^23) - 2^23                    (floor: the sum's unit in the last place is 1)
//   bits(copysign(f, t) + 1.5 * 2^23)          (an integer in [2^23, 2^24): its low byte is the
//                                               two's-complement byte of copysign(f, t))
__device__ __forceinline__ uint32_t quant1_bits(float x, float inv) {
    const float t = fminf(fmaxf(__fmul_rn(x, inv), -127.0f), 127.0f);
    const float a = __fadd_rd(fabsf(t), 0.5f);
    const float f = __fsub_rn(__fadd_rd(a, 8388608.0f), 8388608.0f);
    return __float_as_uint(__fadd_rn(copysignf(f, t), 12582912.0f));
}

__device__ __forceinline__ int8_t quant1(float x, float inv) {
    return static_cast<int8_t>(quant1_bits(x, inv) & 0xFFu);
}

// quant1 of two values at once on packed f32x2 instructions, for a row quantised against its own
// |max| (|x| <= max, so |x * inv| exceeds 127 by at most one rounding and quant1's clamp cannot
// act: the same bytes as quant1 for every finite x; a NaN gives 0 where quant1 gives -127).  The
// two int8 results are returned in bytes 0 and 1.
__device__ __forceinline__ uint32_t quant2_own_max(float x0, float x1, uint64_t inv2) {
    const uint64_t half2 = 0x3F0000003F000000ull;   // (0.5, 0.5)
    const uint64_t two23 = 0x4B0000004B000000ull;   // (2^23, 2^23)
    const uint64_t magic = 0x4B4000004B400000ull;   // (1.5 * 2^23, 1.5 * 2^23)
    const uint64_t v = tzp::f2_mul(tzp::f2_pack(x0, x1), inv2);
    const uint64_t a = v & 0x7FFFFFFF7FFFFFFFull;
    const uint64_t f = tzp::f2_sub(tzp::f2_add_rd(tzp::f2_add_rd(a, half2), two23), two23);
    const uint64_t u = tzp::f2_add(f | (v & 0x8000000080000000ull), magic);
    return __byte_perm(static_cast<uint32_t>(u), static_cast<uint32_t>(u >> 32), 0x0040) & 0xFFFFu;
}

// Low bytes of four quant1_bits results packed little-endian into one word.
__device__ __forceinline__ uint32_t pack_q4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

// Unary op table of the reference fusion codegen (codegen.zig:228-244); TZ_OP_* codes.
__device__ __forceinline__ float unary_op(int op, float x) {
    switch (op) {
        case TZ_OP_RELU: return x > 0.0f ? x : 0.0f;
        case TZ_OP_GELU: {
            const float x3 = x * x * x;
            const float inner = 0.7978845608028654f * (x + 0.044715f * x3);
            return 0.5f * x * (1.0f + (2.0f * sigmoid_f(2.0f * inner) - 1.0f));
        }
        case TZ_OP_SIGMOID: return sigmoid_f(x);
        case TZ_OP_TANH: return 2.0f * sigmoid_f(2.0f * x) - 1.0f;
        case TZ_OP_EXP: return expf(x);
        case TZ_OP_NEG: return -x;
        case TZ_OP_ABS: return fabsf(x);
        case TZ_OP_SILU: return x * sigmoid_f(x);
        case TZ_OP_LOG: return logf(x);
        case TZ_OP_SQRT: return sqrtf(x);
        case TZ_OP_RSQRT: return 1.0f / sqrtf(x);
        case TZ_OP_SIN: return sinf(x);
        case TZ_OP_COS: return cosf(x);
        case TZ_OP_ERF: return erff(x);
        case TZ_OP_GELU_ERF: return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
        case TZ_OP_ERF_AS: {  // Abramowitz-Stegun 7.1.26, in the reference executor's operation order
            const float ax = fabsf(x);
            const float t = 1.0f / (1.0f + 0.3275911f * ax);
            const float y = 1.0f - (((((1.061405429f * t + -1.453152027f) * t) + 1.421413741f) * t + -0.284496736f) * t +
                                    0.254829592f) * t * expf(-ax * ax);
            return x < 0.0f ? -y : y;
        }
        case TZ_OP_GELU_TANH: return x * 0.5f * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
        default: return x;
    }
}

__device__ __forceinline__ float binary_op(int op, float a, float b) {
    switch (op) {
        case TZ_EW_ADD: return a + b;
        case TZ_EW_SUB: return a - b;
        case TZ_EW_MUL: return a * b;
        case TZ_EW_DIV: return a / b;
        case TZ_EW_MAX: return fmaxf(a, b);
        case TZ_EW_MIN: return fminf(a, b);
        case TZ_EW_POW: return powf(a, b);
        case TZ_EW_EQ: return a == b ? 1.0f : 0.0f;
        case TZ_EW_LT: return a < b ? 1.0f : 0.0f;
        case TZ_EW_GT: return a > b ? 1.0f : 0.0f;
        default: return unary_op(op, a);
    }
}

__device__ __forceinline__ double red_combine(int red, double a, double b) {
    switch (red) {
        case TZ_RED_PROD: return a * b;
        case TZ_RED_MAX: return a > b ? a : b;
        case TZ_RED_MIN: return a < b ? a : b;
        default: return a + b;
    }
}

__device__ __forceinline__ double block_reduce(int red, double v, double* sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = red_combine(red, v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) sh[w] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    if (w == 0) {
        double t = (lane < nw) ? sh[lane] : ((red == TZ_RED_PROD) ? 1.0 : (red == TZ_RED_MAX) ? -INFINITY : (red == TZ_RED_MIN) ? INFINITY : 0.0);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t = red_combine(red, t, __shfl_xor_sync(0xffffffffu, t, o));
        v = t;
    }
    return v;
}

}  // namespace tz
