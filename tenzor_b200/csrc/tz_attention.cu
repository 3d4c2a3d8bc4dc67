// tz_attention.cu -- fused masked multi-head self-attention for the Arctic encoder (d = 32, 12
// heads, variable-length packed sequences, no causal mask).
//
// Reference: selfAttention, arctic.zig:639-747 -- per head Q_h K_h^T, * 1/sqrt(32), row softmax
// (max, exp, sum, divide), P V_h.  The reference runs each sequence unpadded; here sequences are
// packed back to back (cu_seqlens) and each CTA only visits the keys of its own sequence, which is
// the masked-batch form with key mask = (position < length).
//
// CTA = (64-query tile, sequence), 4 warps x 16 query rows, loops over all 12 heads so that a
// whole 384-wide output row is produced in one CTA (the W8A8 path quantises it per token right
// here).  Per head: K_h, V_h for every key of the sequence are staged in shared memory by
// cp.async (double-buffered across heads, 16-byte chunks XOR-swizzled so ldmatrix is
// conflict-free); S = Q K^T and O = P V run on mma.sync m16n8k16 (f16 in, f32 accumulate) with an
// online softmax over 64-key blocks (exp2 with the 1/sqrt(32)*log2(e) scale folded in); scores
// never leave registers.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tz_internal.h"
#include "tz_ptx.cuh"
#include "tz_rowops.cuh"

namespace tz {
namespace {

constexpr int kHidden = 384, kQKV = 1152, kHeads = 12, kHd = 32;
constexpr int kQTile = 64;
constexpr int kOStride = 392;  // halves per staged output row (784 B: conflict-free fragment stores)

__device__ __forceinline__ uint32_t kv_off(int key, int chunk) {
    return static_cast<uint32_t>(key * 64 + ((chunk ^ ((key >> 1) & 3)) << 4));
}

// OUT_MODE 0: O f16 [T, 384];  OUT_MODE 1: O int8 [T, 384] + per-token scale [T] (W8A8 rule).
template <int OUT_MODE>
__global__ void __launch_bounds__(128)
    attention_kernel(const __half* __restrict__ qkv, const int* __restrict__ cu_seqlens, int lpad,
                     __half* __restrict__ out_h, int8_t* __restrict__ out_q,
                     float* __restrict__ out_s) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int b = blockIdx.y;
    const int seq0 = cu_seqlens[b];
    const int L = cu_seqlens[b + 1] - seq0;
    const int q0 = blockIdx.x * kQTile;
    if (q0 >= L) return;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kv_bytes = lpad * 64;                      // one K or V head tile
    uint8_t* kvbuf = sm;                                 // [2 buf][K | V]
    __half* ostage = reinterpret_cast<__half*>(sm + 4 * kv_bytes);
    const uint32_t kv_base = tzp::smem_u32(kvbuf);

    auto load_head = [&](int h, int buf) {
        uint8_t* kdst = kvbuf + buf * 2 * kv_bytes;
        uint8_t* vdst = kdst + kv_bytes;
        const int chunks = lpad * 4;
        for (int i = tid; i < chunks; i += 128) {
            const int key = i >> 2, c = i & 3;
            const bool ok = key < L;
            const __half* src = qkv + static_cast<long long>(seq0 + (ok ? key : 0)) * kQKV + kHidden + h * kHd + c * 8;
            tzp::cp_async16(kdst + kv_off(key, c), src, ok);
            tzp::cp_async16(vdst + kv_off(key, c), src + kHidden, ok);
        }
        tzp::cp_async_commit();
    };

    const float sl2 = 0.17677669529663687f * 1.4426950408889634f;  // 1/sqrt(32) * log2(e)
    const int r0 = warp * 16 + (lane >> 2);                        // row within the tile
    const int qrow0 = q0 + r0, qrow1 = qrow0 + 8;
    const int cq = 2 * (lane & 3);

    load_head(0, 0);
    for (int h = 0; h < kHeads; ++h) {
        const int buf = h & 1;
        if (h + 1 < kHeads) {
            load_head(h + 1, buf ^ 1);
            tzp::cp_async_wait<1>();
        } else {
            tzp::cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t kaddr = kv_base + buf * 2 * kv_bytes;
        const uint32_t vaddr = kaddr + kv_bytes;

        // Q fragments for this warp's 16 rows (rows past the sequence end read as zero).
        uint32_t qa[2][4];
        {
            const __half* q_r0 = qkv + static_cast<long long>(seq0 + (qrow0 < L ? qrow0 : 0)) * kQKV + h * kHd;
            const __half* q_r1 = qkv + static_cast<long long>(seq0 + (qrow1 < L ? qrow1 : 0)) * kQKV + h * kHd;
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
                const int d = 16 * ks + cq;
                qa[ks][0] = qrow0 < L ? *reinterpret_cast<const uint32_t*>(q_r0 + d) : 0u;
                qa[ks][1] = qrow1 < L ? *reinterpret_cast<const uint32_t*>(q_r1 + d) : 0u;
                qa[ks][2] = qrow0 < L ? *reinterpret_cast<const uint32_t*>(q_r0 + d + 8) : 0u;
                qa[ks][3] = qrow1 < L ? *reinterpret_cast<const uint32_t*>(q_r1 + d + 8) : 0u;
            }
        }
        float o[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

        for (int kb = 0; kb < L; kb += 64) {
            float s[8][4];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
                uint32_t bk[4];
                tzp::ldmatrix_x4(bk, kaddr + kv_off(kb + 8 * j + (lane & 7), lane >> 3));
                tzp::mma_f16_16816(s[j], qa[0], bk[0], bk[1]);
                tzp::mma_f16_16816(s[j], qa[1], bk[2], bk[3]);
            }
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int key = kb + 8 * j + cq;
                s[j][0] = key < L ? s[j][0] * sl2 : -INFINITY;
                s[j][1] = key + 1 < L ? s[j][1] * sl2 : -INFINITY;
                s[j][2] = key < L ? s[j][2] * sl2 : -INFINITY;
                s[j][3] = key + 1 < L ? s[j][3] * sl2 : -INFINITY;
                mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
                mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
            const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
            m0 = mn0;
            m1 = mn1;
            float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                s[j][0] = exp2f(s[j][0] - mn0);
                s[j][1] = exp2f(s[j][1] - mn0);
                s[j][2] = exp2f(s[j][2] - mn1);
                s[j][3] = exp2f(s[j][3] - mn1);
                ps0 += s[j][0] + s[j][1];
                ps1 += s[j][2] + s[j][3];
            }
            l0 = l0 * al0 + ps0;
            l1 = l1 * al1 + ps1;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                o[i][0] *= al0;
                o[i][1] *= al0;
                o[i][2] *= al1;
                o[i][3] *= al1;
            }
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                uint32_t a[4];
                a[0] = tzp::pack_half2(s[2 * ks][0], s[2 * ks][1]);
                a[1] = tzp::pack_half2(s[2 * ks][2], s[2 * ks][3]);
                a[2] = tzp::pack_half2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
                a[3] = tzp::pack_half2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
                for (int jd = 0; jd < 2; ++jd) {
                    uint32_t bv[4];
                    const int mi = lane >> 3;
                    tzp::ldmatrix_x4_trans(bv, vaddr + kv_off(kb + 16 * ks + (mi & 1) * 8 + (lane & 7), 2 * jd + (mi >> 1)));
                    tzp::mma_f16_16816(o[2 * jd], a, bv[0], bv[1]);
                    tzp::mma_f16_16816(o[2 * jd + 1], a, bv[2], bv[3]);
                }
            }
        }
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
#pragma unroll
        for (int jd = 0; jd < 4; ++jd) {
            const int col = h * kHd + 8 * jd + cq;
            *reinterpret_cast<uint32_t*>(ostage + r0 * kOStride + col) = tzp::pack_half2(o[jd][0] * inv0, o[jd][1] * inv0);
            *reinterpret_cast<uint32_t*>(ostage + (r0 + 8) * kOStride + col) = tzp::pack_half2(o[jd][2] * inv1, o[jd][3] * inv1);
        }
        __syncthreads();  // buffer `buf` is reloaded two heads later; ostage complete after the loop
    }

    if constexpr (OUT_MODE == 0) {
        for (int i = tid; i < kQTile * 48; i += 128) {
            const int r = i / 48, c = i % 48;
            if (q0 + r < L) {
                const uint4 v = *reinterpret_cast<const uint4*>(ostage + r * kOStride + c * 8);
                *reinterpret_cast<uint4*>(out_h + static_cast<long long>(seq0 + q0 + r) * kHidden + c * 8) = v;
            }
        }
    } else {
        for (int r = warp; r < kQTile; r += 4) {
            if (q0 + r >= L) break;
            const __half* src = ostage + r * kOStride;
            uint4 c0 = *reinterpret_cast<const uint4*>(src + lane * 8);
            uint4 c1 = make_uint4(0, 0, 0, 0);
            if (lane < 16) c1 = *reinterpret_cast<const uint4*>(src + 256 + lane * 8);
            const __half* h0 = reinterpret_cast<const __half*>(&c0);
            const __half* h1 = reinterpret_cast<const __half*>(&c1);
            float m = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) m = fmaxf(m, fmaxf(fabsf(__half2float(h0[i])), fabsf(__half2float(h1[i]))));
            m = warp_max(m);
            const float sc = (m == 0.0f) ? 1.0f : __fdiv_rn(m, 127.0f);
            const float inv = __fdiv_rn(1.0f, sc);
            const long long row = seq0 + q0 + r;
            uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                w0 |= (static_cast<uint32_t>(static_cast<uint8_t>(quant1(__half2float(h0[i]), inv)))) << (8 * i);
                w1 |= (static_cast<uint32_t>(static_cast<uint8_t>(quant1(__half2float(h0[i + 4]), inv)))) << (8 * i);
                w2 |= (static_cast<uint32_t>(static_cast<uint8_t>(quant1(__half2float(h1[i]), inv)))) << (8 * i);
                w3 |= (static_cast<uint32_t>(static_cast<uint8_t>(quant1(__half2float(h1[i + 4]), inv)))) << (8 * i);
            }
            *reinterpret_cast<uint2*>(out_q + row * kHidden + lane * 8) = make_uint2(w0, w1);
            if (lane < 16) *reinterpret_cast<uint2*>(out_q + row * kHidden + 256 + lane * 8) = make_uint2(w2, w3);
            if (lane == 0) out_s[row] = sc;
        }
    }
}

}  // namespace

size_t attention_smem_bytes(int max_len) {
    const int lpad = (max_len + 63) / 64 * 64;
    return static_cast<size_t>(4) * lpad * 64 + static_cast<size_t>(kQTile) * kOStride * 2;
}

// qkv f16 [T, 1152]; cu_seqlens device [B+1]; out f16 [T,384] (out_q == null) or int8 + scale.
int launch_attention(tz_ctx_t ctx, const void* qkv, const int* cu_seqlens, int batch, int max_len,
                     void* out_h, int8_t* out_q, float* out_s, cudaStream_t s) {
    TZ_CHECK(max_len >= 1 && max_len <= 512, TZ_EINVAL, "attention: max_len %d outside [1, 512]", max_len);
    if (batch == 0) return TZ_OK;
    const int lpad = (max_len + 63) / 64 * 64;
    const size_t smem = attention_smem_bytes(max_len);
    dim3 grid((max_len + kQTile - 1) / kQTile, batch);
    if (out_q) {
        static bool set = false;
        if (!set) {
            TZ_CUDA(cudaFuncSetAttribute(attention_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(attention_smem_bytes(512))));
            set = true;
        }
        attention_kernel<1><<<grid, 128, smem, s>>>(static_cast<const __half*>(qkv), cu_seqlens, lpad, nullptr, out_q, out_s);
    } else {
        static bool set = false;
        if (!set) {
            TZ_CUDA(cudaFuncSetAttribute(attention_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(attention_smem_bytes(512))));
            set = true;
        }
        attention_kernel<0><<<grid, 128, smem, s>>>(static_cast<const __half*>(qkv), cu_seqlens, lpad,
                                                    static_cast<__half*>(out_h), nullptr, nullptr);
    }
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

}  // namespace tz
