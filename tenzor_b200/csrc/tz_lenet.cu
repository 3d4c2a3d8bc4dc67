// tz_lenet.cu -- LeNet-5 batch inference on sm_100a (f32 CUDA-core arithmetic).
//
// Reference: LeNet.forward / forwardSequential, lenet.zig:262-321: conv1 6@5x5 -> ReLU -> 2x2
// maxpool -> conv2 16@5x5 -> ReLU -> 2x2 maxpool -> flatten (NHWC) -> FC 120 -> ReLU -> FC 84 ->
// ReLU -> FC 10, with conv2dForward (conv2d.zig:30-110), maxPool2dForward (maxpool.zig:25-78) and
// linearForward (lenet.zig:874-898).  Layouts as in the reference: images [N, 28, 28, 1], conv
// weights [out, kh, kw, in], FC weights [out, in].  Variant TZ_LENET_REF is lenet.zig itself
// (conv1 valid, 256 features, logits); TZ_LENET_PAD2 is the benchmark configuration (conv1 zero
// padding 2, 400 features, softmax over the logits).
//
// Three launches.  lenet_conv_kernel: a persistent CTA walks groups of G images; each group is staged
// in shared memory (zero border for the padding), conv1+ReLU+pool writes the pooled map (NHWC) to
// shared memory, conv2+ReLU+pool writes the flattened features to global memory, each split into a
// tf32 head and its f32 remainder (x = hi + lo exactly), row [hi | lo] of 2 KP floats (KP = the
// feature count rounded up to 32, zero padding).  A thread owns one
// pooled output position (all 6 channels for conv1; 8 of the 16 channels for conv2) and its four
// pre-pool conv outputs, so every input value read feeds 24 (conv1) or 32 (conv2) FMAs and the
// weights are warp-uniform shared-memory broadcasts.  The inner products run on packed f32x2 FMAs
// over output-channel pairs (each lane an IEEE fmaf).  FC1 (400 -> 120, 58% of the FC work) runs on
// the tensor cores as the split-tf32 GEMM of tz_gemm.cu (GemmArgs::a3x: hi*hi + hi*lo + lo*hi with
// f32 accumulation, the dropped lo*lo term about 2^-22 of each product) with bias + ReLU in its
// epilogue, writing h1 [n, 128] f32 (columns 120..127 zero).  lenet_fc_tail_kernel: 64-image tiles;
// FC2 and FC3 with the weights staged through shared memory in K chunks (transposed so a thread's
// 8 outputs are contiguous), 4 images x 8 outputs of register blocking per thread, ReLU fused,
// softmax per image at the end.  The convolutions are FMA-bound (0.83 MFLOP per image for the padded
// variant), not HBM-bound (3 KB in).
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>

#include "tz_internal.h"
#include "tz_ptx.cuh"

struct tz_lenet_s {
    tz_ctx_t ctx = nullptr;
    int device = 0;
    int variant = 0;
    float* d_w = nullptr;     // all weights, one allocation
    float* c1w = nullptr;     // [25][8]: conv1 weight by tap, channels padded to 8 (zeros)
    float* c1b = nullptr;     // [8]
    float* c2w = nullptr;     // [25][6][16]: conv2 weight by tap, input channel, output channel
    float* c2b = nullptr;     // [16]
    float* f1x = nullptr;     // FC1 for the split-tf32 GEMM: [128][3 KP] rows [hi | lo | hi], rows >= 120 zero
    float* f1b = nullptr;     // [128], zero past 120
    float *f2w = nullptr, *f2b = nullptr, *f3w = nullptr, *f3b = nullptr;
    float* d_feat = nullptr;  // [cap, 2 KP] split features between conv and FC1
    float* d_h1 = nullptr;    // [cap, 128] FC1 output
    int64_t cap = 0;
    float* d_io = nullptr;    // host-API staging: images [cap_io, 784] then logits [cap_io, 10]
    int64_t cap_io = 0;
    float* h_out = nullptr;           // pinned staging of the host-API probabilities [cap_io, 10]
    cudaStream_t s2 = nullptr;        // second stream of the host-API copy/compute pipeline
    cudaEvent_t ev = nullptr;         // its completion, joined into the context's stream
};

namespace tz {
namespace {

constexpr int kThreads = 256;

template <int PAD>
struct LenetShape {
    static constexpr int PW = 28 + 2 * PAD;      // staged (padded) image width
    static constexpr int C1 = PW - 4;            // conv1 output 24 / 28
    static constexpr int P1 = C1 / 2;            // pool1 12 / 14
    static constexpr int C2 = P1 - 4;            // conv2 output 8 / 10
    static constexpr int P2 = C2 / 2;            // pool2 4 / 5
    static constexpr int FEAT = P2 * P2 * 16;    // 256 / 400
    static constexpr int KP = (FEAT + 31) / 32 * 32;  // 256 / 416: one part of the split-tf32 K
    static constexpr int G = PAD ? 5 : 8;        // images per group: G * P2 * P2 * 2 <= 256 conv2 items
    static constexpr int SMEM_FLOATS = 25 * 8 + 8 + 25 * 6 * 16 + 16 + G * PW * PW + G * P1 * P1 * 6;
};

template <int PAD>
__global__ void __launch_bounds__(kThreads)
    lenet_conv_kernel(const float* __restrict__ images, int64_t n, const float* __restrict__ c1w,
                      const float* __restrict__ c1b, const float* __restrict__ c2w, const float* __restrict__ c2b,
                      float* __restrict__ feat) {
    using S = LenetShape<PAD>;
    extern __shared__ __align__(16) float sm[];
    float* s_w1 = sm;                        // [25][8]
    float* s_b1 = s_w1 + 25 * 8;             // [8]
    float* s_w2 = s_b1 + 8;                  // [25][6][16]
    float* s_b2 = s_w2 + 25 * 6 * 16;        // [16]
    float* s_img = s_b2 + 16;                // [G][PW][PW]
    float* s_p1 = s_img + S::G * S::PW * S::PW;  // [G][P1][P1][6]
    const int tid = threadIdx.x;
    for (int i = tid; i < 25 * 8 + 8; i += kThreads) s_w1[i] = i < 200 ? c1w[i] : c1b[i - 200];
    for (int i = tid; i < 25 * 6 * 16 + 16; i += kThreads) s_w2[i] = i < 2400 ? c2w[i] : c2b[i - 2400];
    for (int i = tid; i < S::G * S::PW * S::PW; i += kThreads) s_img[i] = 0.0f;  // the padding border stays 0
    __syncthreads();

    const int64_t groups = (n + S::G - 1) / S::G;
    for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
        const int64_t img0 = grp * S::G;
        const int gcount = static_cast<int>(n - img0 < S::G ? n - img0 : S::G);
        // ---- stage the group's images (float2: rows start 8-byte aligned at column PAD) ----
        for (int i = tid; i < gcount * 392; i += kThreads) {
            const int g = i / 392, r = i % 392, y = r / 14, x2 = r % 14;
            const float2 v = *reinterpret_cast<const float2*>(images + (img0 + g) * 784 + y * 28 + 2 * x2);
            *reinterpret_cast<float2*>(s_img + (g * S::PW + y + PAD) * S::PW + PAD + 2 * x2) = v;
        }
        __syncthreads();
        // ---- conv1 (6 channels) + ReLU + 2x2 max pool: one pooled position per item ----
        for (int item = tid; item < gcount * S::P1 * S::P1; item += kThreads) {
            const int g = item / (S::P1 * S::P1), r = item % (S::P1 * S::P1), py = r / S::P1, px = r % S::P1;
            const float* src = s_img + (g * S::PW + 2 * py) * S::PW + 2 * px;
            uint64_t acc[4][3];  // channel pairs (0,1) (2,3) (4,5) of the four pre-pool positions
#pragma unroll
            for (int p = 0; p < 4; ++p)
#pragma unroll
                for (int c = 0; c < 3; ++c) acc[p][c] = 0;
#pragma unroll 1
            for (int kh = 0; kh < 5; ++kh) {
                float row[2][6];  // input rows 2py + kh and 2py + kh + 1, columns 2px .. 2px + 5
#pragma unroll
                for (int a = 0; a < 2; ++a)
#pragma unroll
                    for (int b = 0; b < 6; b += 2) {
                        const float2 v = *reinterpret_cast<const float2*>(src + (kh + a) * S::PW + b);
                        row[a][b] = v.x;
                        row[a][b + 1] = v.y;
                    }
#pragma unroll
                for (int kw = 0; kw < 5; ++kw) {
                    const ulonglong2 wa = *reinterpret_cast<const ulonglong2*>(s_w1 + (kh * 5 + kw) * 8);
                    const uint64_t wb = *reinterpret_cast<const uint64_t*>(s_w1 + (kh * 5 + kw) * 8 + 4);
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const float x = row[p >> 1][(p & 1) + kw];
                        const uint64_t xx = tzp::f2_pack(x, x);
                        acc[p][0] = tzp::f2_fma(xx, wa.x, acc[p][0]);
                        acc[p][1] = tzp::f2_fma(xx, wa.y, acc[p][1]);
                        acc[p][2] = tzp::f2_fma(xx, wb, acc[p][2]);
                    }
                }
            }
            float* dst = s_p1 + ((g * S::P1 + py) * S::P1 + px) * 6;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                float m0 = 0.0f, m1 = 0.0f;  // max over ReLU outputs (all >= 0)
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const float2 a = tzp::f2_unpack(acc[p][c]);
                    m0 = fmaxf(m0, s_b1[2 * c] + a.x);
                    m1 = fmaxf(m1, s_b1[2 * c + 1] + a.y);
                }
                *reinterpret_cast<float2*>(dst + 2 * c) = make_float2(m0, m1);
            }
        }
        __syncthreads();
        // ---- conv2 (8 of 16 channels per item) + ReLU + 2x2 max pool -> features ----
        for (int item = tid; item < gcount * S::P2 * S::P2 * 2; item += kThreads) {
            const int half = item & 1, pos = item >> 1;
            const int g = pos / (S::P2 * S::P2), r = pos % (S::P2 * S::P2), py = r / S::P2, px = r % S::P2;
            const float* src = s_p1 + ((g * S::P1 + 2 * py) * S::P1 + 2 * px) * 6;
            uint64_t acc[4][4];  // output-channel pairs of the four pre-pool positions
#pragma unroll
            for (int p = 0; p < 4; ++p)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[p][c] = 0;
#pragma unroll 1
            for (int kh = 0; kh < 5; ++kh)
#pragma unroll 1
                for (int kw = 0; kw < 5; ++kw) {
                    float x[4][6];
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const float* q = src + (((p >> 1) + kh) * S::P1 + (p & 1) + kw) * 6;
#pragma unroll
                        for (int ic = 0; ic < 6; ic += 2) {
                            const float2 v = *reinterpret_cast<const float2*>(q + ic);
                            x[p][ic] = v.x;
                            x[p][ic + 1] = v.y;
                        }
                    }
                    const float* wt = s_w2 + (kh * 5 + kw) * 96 + half * 8;
#pragma unroll
                    for (int ic = 0; ic < 6; ++ic) {
                        const ulonglong2 wa = *reinterpret_cast<const ulonglong2*>(wt + ic * 16);
                        const ulonglong2 wb = *reinterpret_cast<const ulonglong2*>(wt + ic * 16 + 4);
#pragma unroll
                        for (int p = 0; p < 4; ++p) {
                            const uint64_t xx = tzp::f2_pack(x[p][ic], x[p][ic]);
                            acc[p][0] = tzp::f2_fma(xx, wa.x, acc[p][0]);
                            acc[p][1] = tzp::f2_fma(xx, wa.y, acc[p][1]);
                            acc[p][2] = tzp::f2_fma(xx, wb.x, acc[p][2]);
                            acc[p][3] = tzp::f2_fma(xx, wb.y, acc[p][3]);
                        }
                    }
                }
            float m[8];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float b0 = s_b2[half * 8 + 2 * c], b1 = s_b2[half * 8 + 2 * c + 1];
                float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const float2 a = tzp::f2_unpack(acc[p][c]);
                    m0 = fmaxf(m0, b0 + a.x);
                    m1 = fmaxf(m1, b1 + a.y);
                }
                m[2 * c] = m0;
                m[2 * c + 1] = m1;
            }
            float hi[8], lo[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                hi[c] = tzp::tf32_rna(m[c]);
                lo[c] = m[c] - hi[c];  // exact: hi and m share the exponent range, hi holds m's top bits
            }
            float* dst = feat + (img0 + g) * (2 * S::KP) + (py * S::P2 + px) * 16 + half * 8;
            *reinterpret_cast<float4*>(dst) = make_float4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<float4*>(dst + 4) = make_float4(hi[4], hi[5], hi[6], hi[7]);
            *reinterpret_cast<float4*>(dst + S::KP) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<float4*>(dst + S::KP + 4) = make_float4(lo[4], lo[5], lo[6], lo[7]);
        }
        __syncthreads();
    }
}

constexpr int kTile = 64;  // images per FC tile
constexpr int kKC = 40;    // K chunk of staged FC weights

// out[img][o] = act(b[o] + sum_k in[img][k] * W[o][k]) for the tile's 64 images.  Thread t: images
// (t % 16) + 16 i (i < 4, odd row strides keep the reads conflict-free), outputs 8 (t / 16) .. + 7.
template <int IN, int OUT, int LDI, int LDO, bool RELU>
__device__ __forceinline__ void fc_layer(const float* s_in, const float* __restrict__ w, const float* __restrict__ b,
                                         float* s_out, float* s_wc) {
    constexpr int OUTP = (OUT + 7) / 8 * 8;
    constexpr int LDW = OUTP + 4;
    const int tid = threadIdx.x;
    const int ig = tid & 15, og = tid >> 4;
    const bool active = og * 8 < OUT;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < IN; k0 += kKC) {
        __syncthreads();  // the previous chunk (or layer) is consumed
        for (int i = tid; i < OUTP * kKC; i += kThreads) {
            const int o = i / kKC, kk = i % kKC;
            s_wc[kk * LDW + o] = (o < OUT && k0 + kk < IN) ? w[o * IN + k0 + kk] : 0.0f;
        }
        __syncthreads();
        if (active) {
            const int kn = IN - k0 < kKC ? IN - k0 : kKC;
            for (int kk = 0; kk < kn; ++kk) {
                const float4 wa = *reinterpret_cast<const float4*>(s_wc + kk * LDW + og * 8);
                const float4 wb = *reinterpret_cast<const float4*>(s_wc + kk * LDW + og * 8 + 4);
                const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float x = s_in[(ig + 16 * i) * LDI + k0 + kk];
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(x, wv[j], acc[i][j]);
                }
            }
        }
    }
    __syncthreads();
    if (active) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int o = og * 8 + j;
            if (o < OUT) {
                const float bo = b[o];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float v = bo + acc[i][j];
                    s_out[(ig + 16 * i) * LDO + o] = RELU ? fmaxf(v, 0.0f) : v;
                }
            }
        }
    }
    __syncthreads();
}

template <bool SOFTMAX>
__global__ void __launch_bounds__(kThreads)
    lenet_fc_tail_kernel(const float* __restrict__ h1, int64_t n, const float* __restrict__ f2w,
                         const float* __restrict__ f2b, const float* __restrict__ f3w, const float* __restrict__ f3b,
                         float* __restrict__ out) {
    constexpr int L1 = 121, L2 = 85, L3 = 11;
    extern __shared__ __align__(16) float sm[];
    float* s_h1 = sm;                 // [64][L1]
    float* s_h2 = s_h1 + kTile * L1;  // [64][L2]
    float* s_wc = s_h2 + kTile * L2;  // [kKC][128 + 4]
    float* s_o = s_h1;                // [64][L3], reuses s_h1 after FC2
    const int tid = threadIdx.x;
    const int64_t tiles = (n + kTile - 1) / kTile;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int64_t base = t * kTile;
        const int cnt = static_cast<int>(n - base < kTile ? n - base : kTile);
        __syncthreads();
        for (int i = tid; i < kTile * 30; i += kThreads) {  // 120 columns as float4
            const int r = i / 30, k = (i % 30) * 4;
            const float4 v = r < cnt ? *reinterpret_cast<const float4*>(h1 + (base + r) * 128 + k)
                                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            float* d = s_h1 + r * L1 + k;
            d[0] = v.x;
            d[1] = v.y;
            d[2] = v.z;
            d[3] = v.w;
        }
        fc_layer<120, 84, L1, L2, true>(s_h1, f2w, f2b, s_h2, s_wc);
        fc_layer<84, 10, L2, L3, false>(s_h2, f3w, f3b, s_o, s_wc);
        if (tid < cnt) {
            float v[10];
#pragma unroll
            for (int j = 0; j < 10; ++j) v[j] = s_o[tid * L3 + j];
            if (SOFTMAX) {  // softmax.zig:20-47: max, exp(x - max), divide by the sum
                float m = v[0];
#pragma unroll
                for (int j = 1; j < 10; ++j) m = fmaxf(m, v[j]);
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < 10; ++j) {
                    v[j] = expf(v[j] - m);
                    s += v[j];
                }
#pragma unroll
                for (int j = 0; j < 10; ++j) v[j] = v[j] / s;
            }
            float* o = out + (base + tid) * 10;
#pragma unroll
            for (int j = 0; j < 10; ++j) o[j] = v[j];
        }
    }
}

// feat: [n, 2 KP] split features, h1: [n, 128] FC1 output; both slices of the model's scratch.
template <int PAD>
int launch_lenet(tz_lenet_s* m, const float* d_images, int64_t n, float* d_out, cudaStream_t s, float* feat,
                 float* h1) {
    using S = LenetShape<PAD>;
    const int conv_smem = S::SMEM_FLOATS * 4;
    const int fc_smem = (kTile * 121 + kTile * 85 + kKC * 132) * 4;
    static unsigned set = 0;
    const unsigned bit = 1u << (m->device & 31);
    if (!(set & bit)) {
        TZ_CUDA(cudaFuncSetAttribute(lenet_conv_kernel<PAD>, cudaFuncAttributeMaxDynamicSharedMemorySize, conv_smem));
        TZ_CUDA(cudaFuncSetAttribute(lenet_fc_tail_kernel<PAD != 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, fc_smem));
        set |= bit;
    }
    const int sms = m->ctx->sm_count;
    const int64_t groups = (n + S::G - 1) / S::G;
    // 24 CTAs per SM (3 resident): short per-CTA runs of groups balance the end of the grid, and
    // most CTAs stage the conv weights once for several groups (measured best of 3 .. 12k per SM)
    const int g1 = static_cast<int>(groups < 24LL * sms ? groups : 24LL * sms);
    lenet_conv_kernel<PAD><<<g1, kThreads, conv_smem, s>>>(d_images, n, m->c1w, m->c1b, m->c2w, m->c2b, feat);
    TZ_CUDA(cudaGetLastError());
    for (int64_t r = 0; r < n; r += INT32_MAX / 2) {  // the GEMM takes int M
        const int64_t rows = std::min<int64_t>(n - r, INT32_MAX / 2);
        GemmArgs g;
        g.kind = KIND_TF32;
        g.a3x = true;
        g.a = feat + 2 * S::KP * r;
        g.lda = 2 * S::KP;
        g.b = m->f1x;
        g.ldb = 3 * S::KP;
        g.M = static_cast<int>(rows);
        g.N = 128;
        g.K = 3 * S::KP;
        g.bias = m->f1b;
        g.gelu = 3;  // ReLU
        g.out = h1 + 128 * r;
        g.ldo = 128;
        g.out_type = OUT_F32;
        const int rc = launch_gemm(m->ctx, g, s);
        if (rc) return rc;
    }
    const int64_t tiles = (n + kTile - 1) / kTile;
    // 6 CTAs per SM (3 resident): fills every slot, shorter per-CTA runs of tiles (swept 2x .. all)
    const int g2 = static_cast<int>(tiles < 6LL * sms ? tiles : 6LL * sms);
    lenet_fc_tail_kernel<PAD != 0><<<g2, kThreads, fc_smem, s>>>(h1, n, m->f2w, m->f2b, m->f3w, m->f3b, d_out);
    TZ_CUDA(cudaGetLastError());
    return TZ_OK;
}

int lenet_kp(int variant) { return variant == TZ_LENET_PAD2 ? LenetShape<2>::KP : LenetShape<0>::KP; }

// Nearest tf32 value of a finite f32, ties away from zero (the rounding of cvt.rna.tf32.f32).
float tf32_rna_host(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x1000u) & 0xFFFFE000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

int lenet_reserve(tz_lenet_s* m, int64_t n) {
    if (n <= m->cap) return TZ_OK;
    TZ_CUDA(cudaSetDevice(m->device));
    TZ_CUDA(cudaDeviceSynchronize());
    if (m->d_feat) cudaFree(m->d_feat);
    if (m->d_h1) cudaFree(m->d_h1);
    m->d_feat = m->d_h1 = nullptr;
    m->cap = 0;
    const size_t row = 2 * static_cast<size_t>(lenet_kp(m->variant));
    if (cudaMalloc(reinterpret_cast<void**>(&m->d_feat), sizeof(float) * row * static_cast<size_t>(n)) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&m->d_h1), sizeof(float) * 128 * static_cast<size_t>(n)) != cudaSuccess)
        return fail(TZ_ENOMEM, "tz_lenet: feature scratch for %lld images", static_cast<long long>(n));
    // the padding columns of each [hi | lo] row are never written: zero them once
    TZ_CUDA(cudaMemset(m->d_feat, 0, sizeof(float) * row * static_cast<size_t>(n)));
    m->cap = n;
    return TZ_OK;
}

}  // namespace
}  // namespace tz

using namespace tz;

extern "C" {

int tz_lenet_load(tz_ctx_t ctx, const tz_lenet_weights* w, int variant, tz_lenet_t* out) {
    TZ_CHECK(ctx && w && out && (variant == TZ_LENET_REF || variant == TZ_LENET_PAD2), TZ_EINVAL,
             "tz_lenet_load: bad arguments");
    *out = nullptr;
    const float* req[] = {w->conv1_w, w->conv1_b, w->conv2_w, w->conv2_b, w->fc1_w,
                          w->fc1_b,   w->fc2_w,   w->fc2_b,   w->fc3_w,   w->fc3_b};
    for (const float* p : req) TZ_CHECK(p, TZ_EMISSING, "tz_lenet_load: a weight pointer is NULL");
    const int feat = variant == TZ_LENET_PAD2 ? 400 : 256;
    const int kp = lenet_kp(variant);
    // device layout: conv1 [25][8] + [8], conv2 [25][6][16] + [16], FC1 split [128][3 kp] + [128],
    // FC2 and FC3 as given
    const size_t n_c1 = 25 * 8 + 8, n_c2 = 25 * 96 + 16, n_f1 = 128 * 3 * static_cast<size_t>(kp) + 128,
                 n_f2 = 84 * 120 + 84, n_f3 = 10 * 84 + 10;
    const size_t total = n_c1 + n_c2 + n_f1 + n_f2 + n_f3;
    float* h = new float[total];
    std::memset(h, 0, sizeof(float) * total);
    for (int tap = 0; tap < 25; ++tap)
        for (int c = 0; c < 6; ++c) h[tap * 8 + c] = w->conv1_w[c * 25 + tap];  // [6,5,5,1] -> [tap][c]
    for (int c = 0; c < 6; ++c) h[200 + c] = w->conv1_b[c];
    float* c2 = h + n_c1;
    for (int oc = 0; oc < 16; ++oc)
        for (int tap = 0; tap < 25; ++tap)
            for (int ic = 0; ic < 6; ++ic) c2[tap * 96 + ic * 16 + oc] = w->conv2_w[(oc * 25 + tap) * 6 + ic];
    for (int oc = 0; oc < 16; ++oc) c2[2400 + oc] = w->conv2_b[oc];
    float* f = c2 + n_c2;
    for (int o = 0; o < 120; ++o)  // row o: [hi | lo | hi] of W1[o, :], each part kp wide
        for (int k = 0; k < feat; ++k) {
            const float x = w->fc1_w[o * feat + k], hi = tf32_rna_host(x);
            float* r = f + static_cast<size_t>(o) * 3 * kp;
            r[k] = hi;
            r[kp + k] = x - hi;
            r[2 * kp + k] = hi;
        }
    std::memcpy(f + 128 * 3 * static_cast<size_t>(kp), w->fc1_b, sizeof(float) * 120);
    f += n_f1;
    std::memcpy(f, w->fc2_w, sizeof(float) * 84 * 120);
    std::memcpy(f + 84 * 120, w->fc2_b, sizeof(float) * 84);
    f += n_f2;
    std::memcpy(f, w->fc3_w, sizeof(float) * 840);
    std::memcpy(f + 840, w->fc3_b, sizeof(float) * 10);

    tz_lenet_s* m = new tz_lenet_s;
    m->ctx = ctx;
    m->device = ctx->device;
    m->variant = variant;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&m->d_w), sizeof(float) * total);
    if (e == cudaSuccess) e = cudaMemcpy(m->d_w, h, sizeof(float) * total, cudaMemcpyHostToDevice);
    delete[] h;
    if (e != cudaSuccess) {
        if (m->d_w) cudaFree(m->d_w);
        delete m;
        return cuda_fail(e, "tz_lenet_load");
    }
    m->c1w = m->d_w;
    m->c1b = m->c1w + 200;
    m->c2w = m->d_w + n_c1;
    m->c2b = m->c2w + 2400;
    m->f1x = m->c2w + n_c2;
    m->f1b = m->f1x + 128 * 3 * static_cast<size_t>(kp);
    m->f2w = m->f1x + n_f1;
    m->f2b = m->f2w + 84 * 120;
    m->f3w = m->f2w + n_f2;
    m->f3b = m->f3w + 840;
    *out = m;
    return TZ_OK;
}

int tz_lenet_free(tz_lenet_t m) {
    if (!m) return TZ_OK;
    cudaSetDevice(m->device);
    cudaDeviceSynchronize();
    if (m->d_w) cudaFree(m->d_w);
    if (m->d_feat) cudaFree(m->d_feat);
    if (m->d_h1) cudaFree(m->d_h1);
    if (m->d_io) cudaFree(m->d_io);
    if (m->h_out) cudaFreeHost(m->h_out);
    if (m->s2) cudaStreamDestroy(m->s2);
    if (m->ev) cudaEventDestroy(m->ev);
    delete m;
    return TZ_OK;
}

int tz_lenet_reserve(tz_lenet_t m, int64_t n) {
    TZ_CHECK(m && n >= 0, TZ_EINVAL, "tz_lenet_reserve: bad arguments");
    return lenet_reserve(m, n);
}

int tz_lenet_forward_device(tz_lenet_t m, const float* images, int64_t n, float* out, tz_stream_t stream) {
    TZ_CHECK(m && images && out && n >= 0, TZ_EINVAL, "tz_lenet_forward_device: bad arguments");
    TZ_CHECK(reinterpret_cast<uintptr_t>(images) % 8 == 0, TZ_EINVAL, "tz_lenet_forward_device: images must be 8-byte aligned");
    if (n == 0) return TZ_OK;
    TZ_CUDA(cudaSetDevice(m->device));
    int rc = lenet_reserve(m, n);
    if (rc) return rc;
    cudaStream_t s = pick_stream(m->ctx, stream);
    return m->variant == TZ_LENET_PAD2 ? launch_lenet<2>(m, images, n, out, s, m->d_feat, m->d_h1)
                                       : launch_lenet<0>(m, images, n, out, s, m->d_feat, m->d_h1);
}

int tz_lenet_forward(tz_lenet_t m, const float* images, int64_t n, float* out) {
    TZ_CHECK(m && images && out && n >= 0, TZ_EINVAL, "tz_lenet_forward: bad arguments");
    if (n == 0) return TZ_OK;
    TZ_CUDA(cudaSetDevice(m->device));
    if (n > m->cap_io) {
        TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
        if (m->d_io) cudaFree(m->d_io);
        m->d_io = nullptr;
        m->cap_io = 0;
        if (m->h_out) cudaFreeHost(m->h_out);
        m->h_out = nullptr;
        if (cudaMalloc(reinterpret_cast<void**>(&m->d_io), sizeof(float) * 794 * static_cast<size_t>(n)) != cudaSuccess ||
            cudaMallocHost(reinterpret_cast<void**>(&m->h_out), sizeof(float) * 10 * static_cast<size_t>(n)) != cudaSuccess)
            return fail(TZ_ENOMEM, "tz_lenet_forward: staging for %lld images", static_cast<long long>(n));
        m->cap_io = n;
    }
    int rc = lenet_reserve(m, n);
    if (rc) return rc;
    if (!m->s2) {
        TZ_CUDA(cudaStreamCreateWithFlags(&m->s2, cudaStreamNonBlocking));
        TZ_CUDA(cudaEventCreateWithFlags(&m->ev, cudaEventDisableTiming));
    }
    // Copy/compute pipeline: chunks alternate between two streams, so the copy engine moves chunk
    // i + 1 (from pinned memory) while the SMs run chunk i.  Every chunk has its own slice of the
    // staging and of the feature scratch: no chunk waits for another's buffers.  Probabilities come
    // back through pinned staging (a copy into pageable memory would block the host between chunks).
    cudaStream_t st[2] = {m->ctx->stream, m->s2};
    const int64_t row = 2 * lenet_kp(m->variant);
    const int64_t chunk = n <= 8192 ? n : std::max<int64_t>(4096, ((n + 7) / 8 + kTile - 1) / kTile * kTile);
    TZ_CUDA(cudaEventRecord(m->ev, st[0]));  // s2 starts after the work already queued on the context's stream
    TZ_CUDA(cudaStreamWaitEvent(st[1], m->ev, 0));
    int k = 0;
    for (int64_t a = 0; a < n; a += chunk, k ^= 1) {
        const int64_t c = std::min(chunk, n - a);
        float* d_img = m->d_io + 784 * a;
        float* d_out = m->d_io + 784 * n + 10 * a;
        TZ_CUDA(cudaMemcpyAsync(d_img, images + 784 * a, sizeof(float) * 784 * c, cudaMemcpyHostToDevice, st[k]));
        float* feat = m->d_feat + row * a;
        float* h1 = m->d_h1 + 128 * a;
        rc = m->variant == TZ_LENET_PAD2 ? launch_lenet<2>(m, d_img, c, d_out, st[k], feat, h1)
                                         : launch_lenet<0>(m, d_img, c, d_out, st[k], feat, h1);
        if (rc) return rc;
        TZ_CUDA(cudaMemcpyAsync(m->h_out + 10 * a, d_out, sizeof(float) * 10 * c, cudaMemcpyDeviceToHost, st[k]));
    }
    TZ_CUDA(cudaEventRecord(m->ev, st[1]));
    TZ_CUDA(cudaStreamWaitEvent(st[0], m->ev, 0));
    TZ_CUDA(cudaStreamSynchronize(st[0]));
    memcpy(out, m->h_out, sizeof(float) * 10 * static_cast<size_t>(n));
    return TZ_OK;
}

}  // extern "C"
