// tz_attention.cu -- fused masked multi-head self-attention for the Arctic encoder (d = 32, 12
// heads, variable-length packed sequences, no causal mask).
//
// Reference: selfAttention, arctic.zig:639-747 -- per head Q_h K_h^T, * 1/sqrt(32), row softmax
// (max, exp, sum, divide), P V_h.  The reference runs each sequence unpadded; here sequences are
// packed back to back (cu_seqlens) and each CTA only visits the keys of its own sequence, which is
// the masked-batch form with key mask = (position < length).
//
// CTA = (query block, head, sequence): 4 warps x 16 query rows while the longest sequence has at most
// 128 keys, 8 warps beyond (attention_long_kernel).  The grid is (head, sequence,
// query block) with the last query block first: the block scheduler hands out the CTAs of long
// sequences' later queries (the ones that see every key, or exit at once for short sequences) before
// the first blocks of every sequence, so the lighter CTAs fill the tail of the wave.  K_h and V_h for every key of
// the sequence and the CTA's Q rows arrive in shared memory as 64- and 16-row TMA boxes (32 f16 columns,
// 64-byte swizzle: 16-byte chunk c of row r at c ^ ((r >> 1) & 3), so ldmatrix is conflict-free),
// issued by one thread (one mbarrier, or one per 64-key chunk for long sequences); V rows past the
// sequence's end are zeroed.  S = Q K^T and
// O = P V run on mma.sync m16n8k16 (f16 in, f32 accumulate) with an online softmax over 64-key
// blocks (exp2 with the 1/sqrt(32)*log2(e) scale folded in); scores never leave registers.  Full
// 64-key blocks run unmasked; the ragged last block runs at 16-key granularity with the key mask.  The
// f16 output goes straight to global memory; for the W8A8 path each row's |max| over the 12 heads
// is accumulated with atomicMax for the per-token requantisation that follows.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tz_internal.h"
#include "tz_ptx.cuh"
#include "tz_rowops.cuh"

namespace tz {
namespace {

constexpr int kHidden = 384, kQKV = 1152, kHeads = 12, kHd = 32;
constexpr int kShortQ = 64;  // queries per CTA of the short-sequence kernel

__device__ __forceinline__ uint32_t kv_off(int row, int chunk) {
    return static_cast<uint32_t>(row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4));
}

// One block of keys [kb, kb + 16*NCH) for the warp's 16 query rows: S = Q K^T on the tensor cores,
// the online-softmax update, then O += P V.  MASK = the block runs past the sequence's last key.
// Scores stay in raw units (m0/m1 are raw maxima); the 1/sqrt(32)*log2(e) scale and the max are
// applied by one FMA inside the exponent, which is exact in order: the scale is positive.
template <int NCH, bool MASK, bool BF>
__device__ __forceinline__ void attend_block(int kb, int L, uint32_t kaddr, uint32_t vaddr, const uint32_t (&qa)[2][4],
                                             float (&o)[4][4], float& m0, float& m1, float& l0, float& l1, int lane) {
    constexpr float sl2 = 0.17677669529663687f * 1.4426950408889634f;  // 1/sqrt(32) * log2(e)
    const int cq = 2 * (lane & 3);
    const int mi = lane >> 3;
    float s[2 * NCH][4];
#pragma unroll
    for (int j = 0; j < 2 * NCH; ++j) {
        s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
        uint32_t bk[4];
        tzp::ldmatrix_x4(bk, kaddr + kv_off(kb + 8 * j + (lane & 7), mi));
        tzp::mma16_16816<BF>(s[j], qa[0], bk[0], bk[1]);
        tzp::mma16_16816<BF>(s[j], qa[1], bk[2], bk[3]);
    }
    if (MASK) {
#pragma unroll
        for (int j = 0; j < 2 * NCH; ++j) {
            const int key = kb + 8 * j + cq;
            if (key >= L) s[j][0] = s[j][2] = -INFINITY;
            if (key + 1 >= L) s[j][1] = s[j][3] = -INFINITY;
        }
    }
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < 2 * NCH; ++j) {
        mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
        mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float al0 = tzp::ex2_approx((m0 - mx0) * sl2), al1 = tzp::ex2_approx((m1 - mx1) * sl2);
    const float nb0 = -mx0 * sl2, nb1 = -mx1 * sl2;
    m0 = mx0;
    m1 = mx1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 2 * NCH; ++j) {
        s[j][0] = tzp::ex2_approx(fmaf(s[j][0], sl2, nb0));
        s[j][1] = tzp::ex2_approx(fmaf(s[j][1], sl2, nb0));
        s[j][2] = tzp::ex2_approx(fmaf(s[j][2], sl2, nb1));
        s[j][3] = tzp::ex2_approx(fmaf(s[j][3], sl2, nb1));
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
    for (int kk = 0; kk < NCH; ++kk) {
        uint32_t a[4];
        a[0] = tzp::pack16x2<BF>(s[2 * kk][0], s[2 * kk][1]);
        a[1] = tzp::pack16x2<BF>(s[2 * kk][2], s[2 * kk][3]);
        a[2] = tzp::pack16x2<BF>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = tzp::pack16x2<BF>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int jd = 0; jd < 2; ++jd) {
            uint32_t bv[4];
            tzp::ldmatrix_x4_trans(bv, vaddr + kv_off(kb + 16 * kk + (mi & 1) * 8 + (lane & 7), 2 * jd + (mi >> 1)));
            tzp::mma16_16816<BF>(o[2 * jd], a, bv[0], bv[1]);
            tzp::mma16_16816<BF>(o[2 * jd + 1], a, bv[2], bv[3]);
        }
    }
}

// A chunk's bounded wait: one try_wait inline (the chunk has usually landed by the time a warp gets
// to it), the bounded spin out of line so that it costs the inner loop no registers.
__device__ __noinline__ bool chunk_wait_slow(uint64_t* bar, int* status) { return tzp::mbar_wait(bar, 0, status, nullptr); }
__device__ __forceinline__ bool chunk_wait(uint64_t* bar, int* status) {
    return tzp::mbar_try_wait(tzp::smem_u32(bar), 0) || chunk_wait_slow(bar, status);
}

// Sequences of up to 128 keys: CTA = (64-query block, head, sequence), 4 warps x 16 query rows; the
// whole K / V of the sequence and the Q rows complete one mbarrier.  80 registers: 6 CTAs (24 warps)
// per SM.
template <bool BF>
__global__ void __launch_bounds__(128)
    attention_short_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmQKV64,
                     const int* __restrict__ cu_seqlens, int lpad,
                     __half* __restrict__ out, unsigned* __restrict__ row_absmax, int* status) {
    extern __shared__ uint8_t sm_raw[];
    __shared__ uint64_t bar;
    uint8_t* sm = sm_raw + ((1024u - (tzp::smem_u32(sm_raw) & 1023u)) & 1023u);  // swizzle-atom aligned
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        tzp::mbar_init(&bar, 1);
        tzp::fence_mbar_init();
        tzp::tma_prefetch_desc(&tmQKV);
        tzp::tma_prefetch_desc(&tmQKV64);
    }
    // cu_seqlens is a forward input, written before the forward's first kernel: read it while the
    // previous kernel (QKV) may still run; Q/K/V are read only after griddepcontrol.wait.
    const int b = blockIdx.y;
    const int h = blockIdx.x;
    const int qb = static_cast<int>(gridDim.z - 1 - blockIdx.z);  // the last query block is dispatched first
    const int seq0 = cu_seqlens[b];
    const int L = cu_seqlens[b + 1] - seq0;
    __syncthreads();
    tzp::pdl_wait();
    const int q0 = qb * kShortQ;
    if (L > lpad || L < 0) {  // the caller's max_len was too small: refuse rather than overrun shared memory
        if (tid == 0 && qb == 0) atomicOr(status, TZ_DEV_BOUNDS);
        return;
    }
    if (q0 >= L) return;  // uniform over the CTA

    const int kv_bytes = lpad * 64;
    uint8_t* ks = sm;
    uint8_t* vs = sm + kv_bytes;
    uint8_t* qs = sm + 2 * kv_bytes;
    const int nk16 = (L + 15) >> 4;                                  // 16-key boxes of K and of V
    const int nq16 = ((L - q0 < kShortQ ? L - q0 : kShortQ) + 15) >> 4;  // 16-row boxes of Q
    if (tid == 0) {  // 64-row boxes where they fit, 16-row boxes for the rest (same shared layout)
        tzp::mbar_arrive_expect_tx(&bar, static_cast<uint32_t>((2 * nk16 + nq16) * 16 * 64));
        int i = 0;
        for (; i + 4 <= nk16; i += 4) {
            tzp::tma_load_2d(ks + i * 1024, &tmQKV64, kHidden + h * kHd, seq0 + 16 * i, &bar);
            tzp::tma_load_2d(vs + i * 1024, &tmQKV64, 2 * kHidden + h * kHd, seq0 + 16 * i, &bar);
        }
        for (; i < nk16; ++i) {
            tzp::tma_load_2d(ks + i * 1024, &tmQKV, kHidden + h * kHd, seq0 + 16 * i, &bar);
            tzp::tma_load_2d(vs + i * 1024, &tmQKV, 2 * kHidden + h * kHd, seq0 + 16 * i, &bar);
        }
        if (nq16 == 4) {
            tzp::tma_load_2d(qs, &tmQKV64, h * kHd, seq0 + q0, &bar);
        } else {
            for (int j = 0; j < nq16; ++j) tzp::tma_load_2d(qs + j * 1024, &tmQKV, h * kHd, seq0 + q0 + 16 * j, &bar);
        }
    }
    const bool landed = tzp::mbar_wait(&bar, 0, status, nullptr);
    // Keys in [L, 16 * nk16) are masked to -inf, but their V rows (the next sequence's tokens) still
    // enter P V with weight 0: zero them so a non-finite value there cannot leak in.
    if (landed && (L & 15)) {
        for (int i = tid; i < (16 * nk16 - L) * 4; i += 128) {
            const int key = L + (i >> 2);
            *reinterpret_cast<uint4*>(vs + kv_off(key, i & 3)) = make_uint4(0, 0, 0, 0);
        }
    }
    __syncthreads();
    tzp::pdl_trigger();
    if (!landed || q0 + warp * 16 >= L) return;  // no further block-wide synchronisation below

    const uint32_t kaddr = tzp::smem_u32(ks), vaddr = tzp::smem_u32(vs), qaddr = tzp::smem_u32(qs);
    const int cq = 2 * (lane & 3);
    const int mi = lane >> 3;

    uint32_t qa[2][4];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk)
        tzp::ldmatrix_x4(qa[kk], qaddr + kv_off(warp * 16 + (mi & 1) * 8 + (lane & 7), 2 * kk + (mi >> 1)));

    float o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    int kb = 0;
    for (; kb + 64 <= L; kb += 64) attend_block<4, false, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane);
    switch ((L - kb + 15) >> 4) {  // the ragged tail, in 16-key chunks
        case 1: attend_block<1, true, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane); break;
        case 2: attend_block<2, true, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane); break;
        case 3: attend_block<3, true, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane); break;
        case 4: attend_block<4, true, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane); break;
        default: break;
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
    const int r0 = q0 + warp * 16 + (lane >> 2), r1 = r0 + 8;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int jd = 0; jd < 4; ++jd) {
        const int col = h * kHd + 8 * jd + cq;
        const uint32_t p0 = tzp::pack16x2<BF>(o[jd][0] * inv0, o[jd][1] * inv0);
        const uint32_t p1 = tzp::pack16x2<BF>(o[jd][2] * inv1, o[jd][3] * inv1);
        if (r0 < L) *reinterpret_cast<uint32_t*>(out + static_cast<long long>(seq0 + r0) * kHidden + col) = p0;
        if (r1 < L) *reinterpret_cast<uint32_t*>(out + static_cast<long long>(seq0 + r1) * kHidden + col) = p1;
        if (row_absmax) {
            const __half2 h0 = *reinterpret_cast<const __half2*>(&p0);
            const __half2 h1 = *reinterpret_cast<const __half2*>(&p1);
            a0 = fmaxf(a0, fmaxf(fabsf(__low2float(h0)), fabsf(__high2float(h0))));
            a1 = fmaxf(a1, fmaxf(fabsf(__low2float(h1)), fabsf(__high2float(h1))));
        }
    }
    if (row_absmax) {
        a0 = fmaxf(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
        a0 = fmaxf(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
        a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
        a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
        if ((lane & 3) == 0) {
            if (r0 < L) atomicMax(row_absmax + seq0 + r0, __float_as_uint(a0));
            if (r1 < L) atomicMax(row_absmax + seq0 + r1, __float_as_uint(a1));
        }
    }
}


// Sequences beyond 128 keys: CTA = (128-query block, head, sequence), 8 warps x 16 query rows, so the
// staged K / V of a long sequence serve twice the queries and three CTAs (24 warps) fit an SM's
// shared memory at 512 keys.  K / V arrive in 64-key chunks, each completing its own mbarrier (chunk
// 0 also carries Q): the warps start on the first keys while the later chunks are still in flight.
constexpr int kMaxChunks = 8;  // 512 keys

template <int QW, bool BF>
__global__ void __launch_bounds__(32 * QW, 3)
    attention_long_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmQKV64,
                     const int* __restrict__ cu_seqlens, int lpad,
                     __half* __restrict__ out, unsigned* __restrict__ row_absmax, int* status) {
    constexpr int kQ = 16 * QW;
    extern __shared__ uint8_t sm_raw[];
    __shared__ uint64_t bar[kMaxChunks];
    __shared__ uint64_t vz;  // the V rows past the sequence's end are zeroed (tail chunk)
    uint8_t* sm = sm_raw + ((1024u - (tzp::smem_u32(sm_raw) & 1023u)) & 1023u);  // swizzle-atom aligned
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int c = 0; c < kMaxChunks; ++c) tzp::mbar_init(&bar[c], 1);
        tzp::mbar_init(&vz, 1);
        tzp::fence_mbar_init();
        tzp::tma_prefetch_desc(&tmQKV);
        tzp::tma_prefetch_desc(&tmQKV64);
    }
    // cu_seqlens is a forward input, written before the forward's first kernel: read it while the
    // previous kernel (QKV) may still run; Q/K/V are read only after griddepcontrol.wait.
    const int b = blockIdx.y;
    const int h = blockIdx.x;
    const int qb = static_cast<int>(gridDim.z - 1 - blockIdx.z);  // the last query block is dispatched first
    const int seq0 = cu_seqlens[b];
    const int L = cu_seqlens[b + 1] - seq0;
    __syncthreads();
    tzp::pdl_wait();
    const int q0 = qb * kQ;
    if (L > lpad || L < 0) {  // the caller's max_len was too small: refuse rather than overrun shared memory
        if (tid == 0 && qb == 0) atomicOr(status, TZ_DEV_BOUNDS);
        return;
    }
    if (q0 >= L) return;  // uniform over the CTA

    const int kv_bytes = lpad * 64;
    uint8_t* ks = sm;
    uint8_t* vs = sm + kv_bytes;
    uint8_t* qs = sm + 2 * kv_bytes;
    const int nk16 = (L + 15) >> 4;                            // 16-key boxes of K and of V
    const int nchunks = (nk16 + 3) >> 2;                       // 64-key chunks
    const int nq16 = ((L - q0 < kQ ? L - q0 : kQ) + 15) >> 4;  // 16-row boxes of Q
    // Long sequences (QW = 8) complete each 64-key chunk on its own barrier; short ones (at most two
    // chunks) complete everything on bar[0], which then stands for every chunk.
    constexpr bool kChunked = QW == 8;
    if (tid == 0) {
        if (!kChunked)
            tzp::mbar_arrive_expect_tx(&bar[0], static_cast<uint32_t>((2 * nk16 + nq16) * 16 * 64));
        // chunk c: K and V rows [64c, 64c + 64) -- one 64-row box each where the chunk is whole,
        // 16-row boxes for a partial last chunk (same shared layout); Q with chunk 0
        for (int c = 0; c < nchunks; ++c) {
            const int i0 = 4 * c, i1 = nk16 < i0 + 4 ? nk16 : i0 + 4;
            const int qbytes = c == 0 ? nq16 * 16 * 64 : 0;
            uint64_t* cb = kChunked ? &bar[c] : &bar[0];
            if (kChunked) tzp::mbar_arrive_expect_tx(cb, static_cast<uint32_t>(2 * (i1 - i0) * 16 * 64 + qbytes));
            if (c == 0) {
                if (nq16 == 4) {
                    tzp::tma_load_2d(qs, &tmQKV64, h * kHd, seq0 + q0, &bar[0]);
                } else if (nq16 == 8) {
                    tzp::tma_load_2d(qs, &tmQKV64, h * kHd, seq0 + q0, &bar[0]);
                    tzp::tma_load_2d(qs + 4096, &tmQKV64, h * kHd, seq0 + q0 + 64, &bar[0]);
                } else {
                    for (int j = 0; j < nq16; ++j) tzp::tma_load_2d(qs + j * 1024, &tmQKV, h * kHd, seq0 + q0 + 16 * j, &bar[0]);
                }
            }
            if (i1 - i0 == 4) {
                tzp::tma_load_2d(ks + i0 * 1024, &tmQKV64, kHidden + h * kHd, seq0 + 16 * i0, cb);
                tzp::tma_load_2d(vs + i0 * 1024, &tmQKV64, 2 * kHidden + h * kHd, seq0 + 16 * i0, cb);
            } else {
                for (int i = i0; i < i1; ++i) {
                    tzp::tma_load_2d(ks + i * 1024, &tmQKV, kHidden + h * kHd, seq0 + 16 * i, cb);
                    tzp::tma_load_2d(vs + i * 1024, &tmQKV, 2 * kHidden + h * kHd, seq0 + 16 * i, cb);
                }
            }
        }
    }
    // Keys in [L, 16 * nk16) are masked to -inf, but their V rows (the next sequence's tokens) still
    // enter P V with weight 0: they are zeroed once they have landed, so a non-finite value there
    // cannot leak in.  Short sequences: every thread waits for the whole staging and the CTA zeroes
    // them together.  Long ones: warp 0 zeroes them once the last chunk has landed and releases `vz`,
    // which only the ragged tail block waits for.
    if constexpr (!kChunked) {
        const bool landed = tzp::mbar_wait(&bar[0], 0, status, nullptr);
        if (landed && (L & 15)) {
            for (int i = tid; i < (16 * nk16 - L) * 4; i += 32 * QW) {
                const int key = L + (i >> 2);
                *reinterpret_cast<uint4*>(vs + kv_off(key, i & 3)) = make_uint4(0, 0, 0, 0);
            }
        }
        __syncthreads();
        tzp::pdl_trigger();
        if (!landed) return;
    } else {
        tzp::pdl_trigger();
        if (warp == 0) {
            bool ok = true;
            if (L & 15) {
                ok = tzp::mbar_wait(&bar[nchunks - 1], 0, status, nullptr);
                if (ok)
                    for (int i = lane; i < (16 * nk16 - L) * 4; i += 32) {
                        const int key = L + (i >> 2);
                        *reinterpret_cast<uint4*>(vs + kv_off(key, i & 3)) = make_uint4(0, 0, 0, 0);
                    }
                __syncwarp();
            }
            if (lane == 0) tzp::mbar_arrive(&vz);
            if (!ok) return;
        }
    }
    if (q0 + warp * 16 >= L) return;  // no block-wide synchronisation below

    const uint32_t kaddr = tzp::smem_u32(ks), vaddr = tzp::smem_u32(vs), qaddr = tzp::smem_u32(qs);
    const int cq = 2 * (lane & 3);
    const int mi = lane >> 3;

    if (kChunked && !chunk_wait(&bar[0], status)) return;
    uint32_t qa[2][4];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk)
        tzp::ldmatrix_x4(qa[kk], qaddr + kv_off(warp * 16 + (mi & 1) * 8 + (lane & 7), 2 * kk + (mi >> 1)));

    float o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    int kb = 0;
    for (; kb + 64 <= L; kb += 64) {
        if (kChunked && kb > 0 && !chunk_wait(&bar[kb >> 6], status)) return;
        attend_block<4, false, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane);
    }
    if (kb < L) {  // the ragged tail, in 16-key chunks: its chunk has landed and its V rows are zeroed
        if (kChunked && kb > 0 && !chunk_wait(&bar[kb >> 6], status)) return;
        if (kChunked && !chunk_wait(&vz, status)) return;
        switch ((L - kb + 15) >> 4) {
            case 1: attend_block<1, true, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane); break;
            case 2: attend_block<2, true, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane); break;
            case 3: attend_block<3, true, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane); break;
            case 4: attend_block<4, true, BF>(kb, L, kaddr, vaddr, qa, o, m0, m1, l0, l1, lane); break;
            default: break;
        }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
    const int r0 = q0 + warp * 16 + (lane >> 2), r1 = r0 + 8;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int jd = 0; jd < 4; ++jd) {
        const int col = h * kHd + 8 * jd + cq;
        const uint32_t p0 = tzp::pack16x2<BF>(o[jd][0] * inv0, o[jd][1] * inv0);
        const uint32_t p1 = tzp::pack16x2<BF>(o[jd][2] * inv1, o[jd][3] * inv1);
        if (r0 < L) *reinterpret_cast<uint32_t*>(out + static_cast<long long>(seq0 + r0) * kHidden + col) = p0;
        if (r1 < L) *reinterpret_cast<uint32_t*>(out + static_cast<long long>(seq0 + r1) * kHidden + col) = p1;
        if (row_absmax) {
            const __half2 h0 = *reinterpret_cast<const __half2*>(&p0);
            const __half2 h1 = *reinterpret_cast<const __half2*>(&p1);
            a0 = fmaxf(a0, fmaxf(fabsf(__low2float(h0)), fabsf(__high2float(h0))));
            a1 = fmaxf(a1, fmaxf(fabsf(__low2float(h1)), fabsf(__high2float(h1))));
        }
    }
    if (row_absmax) {
        a0 = fmaxf(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
        a0 = fmaxf(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
        a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
        a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
        if ((lane & 3) == 0) {
            if (r0 < L) atomicMax(row_absmax + seq0 + r0, __float_as_uint(a0));
            if (r1 < L) atomicMax(row_absmax + seq0 + r1, __float_as_uint(a1));
        }
    }
}

}  // namespace

// The long-sequence kernel serves batches whose longest sequence pads beyond 128 keys.
constexpr int kLongQW = 8;
bool attention_long(int lpad) { return lpad > 128; }

size_t attention_smem_bytes(int max_len) {
    const int lpad = (max_len + 63) / 64 * 64;
    const int qrows = attention_long(lpad) ? 16 * kLongQW : kShortQ;
    return static_cast<size_t>(2) * lpad * 64 + static_cast<size_t>(qrows) * 64 + 1024;  // + alignment
}

// qkv [T, 1152] f16 (or bf16 with `bf16`; 16-byte aligned); cu_seqlens device [B+1]; out [T, 384] of
// the same type; row_absmax (optional, f16 only) [T] float bits, accumulated with atomicMax (must start
// at zero).
int launch_attention(tz_ctx_t ctx, const void* qkv, int64_t total_tokens, const int* cu_seqlens, int batch, int max_len,
                     void* out, unsigned* row_absmax, cudaStream_t s, bool pdl, bool bf16) {
    TZ_CHECK(max_len >= 1 && max_len <= 512, TZ_EINVAL, "attention: max_len %d outside [1, 512]", max_len);
    TZ_CHECK(!(bf16 && row_absmax), TZ_EINVAL, "attention: the row |max| is taken on IEEE-half outputs");
    if (batch == 0) return TZ_OK;
    const int lpad = (max_len + 63) / 64 * 64;
    const bool lng = attention_long(lpad);
    const size_t smem = attention_smem_bytes(max_len);
    static unsigned set = 0;
    int dev = 0;
    TZ_CUDA(cudaGetDevice(&dev));
    if (!(set & (1u << (dev & 31)))) {
        const int ss = static_cast<int>(attention_smem_bytes(128)), sl = static_cast<int>(attention_smem_bytes(512));
        TZ_CUDA(cudaFuncSetAttribute(attention_short_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ss));
        TZ_CUDA(cudaFuncSetAttribute(attention_short_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ss));
        TZ_CUDA(cudaFuncSetAttribute(attention_long_kernel<kLongQW, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, sl));
        TZ_CUDA(cudaFuncSetAttribute(attention_long_kernel<kLongQW, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, sl));
        set |= 1u << (dev & 31);
    }
    // QKV [T, 1152]: 16- and 64-row x 32-column boxes, 64-byte swizzle; rows >= T read as 0
    const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap tm, tm64;
    int rc = encode_tmap_2d_swz(&tm, dt, 2, qkv, kQKV, static_cast<uint64_t>(total_tokens), kQKV * 2, kHd, 16,
                                CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    rc = encode_tmap_2d_swz(&tm64, dt, 2, qkv, kQKV, static_cast<uint64_t>(total_tokens), kQKV * 2, kHd, 64,
                            CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    __half* o = static_cast<__half*>(out);  // 16-bit container of either type
    // grid.y is the sequence: batches beyond 65535 sequences go in consecutive launches over slices of
    // cu_seqlens (its entries are absolute token offsets, so a slice needs no rebasing)
    const int qtile = lng ? 16 * kLongQW : kShortQ;
    for (int b0 = 0; b0 < batch; b0 += 65535) {
        const int nb = batch - b0 < 65535 ? batch - b0 : 65535;
        dim3 grid(kHeads, nb, (max_len + qtile - 1) / qtile);
        int rc;
        if (lng) {
            auto k = bf16 ? attention_long_kernel<kLongQW, true> : attention_long_kernel<kLongQW, false>;
            rc = launch_kernel(k, grid, dim3(32 * kLongQW), smem, s, pdl, tm, tm64, cu_seqlens + b0, lpad, o, row_absmax,
                               ctx->d_status);
        } else {
            auto k = bf16 ? attention_short_kernel<true> : attention_short_kernel<false>;
            rc = launch_kernel(k, grid, dim3(128), smem, s, pdl, tm, tm64, cu_seqlens + b0, lpad, o, row_absmax,
                               ctx->d_status);
        }
        if (rc) return rc;
    }
    return TZ_OK;
}

}  // namespace tz

extern "C" int tz_attention(tz_ctx_t ctx, const void* qkv, int64_t total_tokens, const int32_t* cu_seqlens, int batch,
                            int max_len, void* out, int bf16, tz_stream_t stream) {
    TZ_CHECK(ctx && qkv && cu_seqlens && out && total_tokens >= 0 && batch >= 0, TZ_EINVAL, "tz_attention: bad arguments");
    TZ_CHECK((reinterpret_cast<uintptr_t>(qkv) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0, TZ_EINVAL,
             "tz_attention: qkv and out must be 16-byte aligned");
    if (total_tokens == 0 || batch == 0) return TZ_OK;
    return tz::launch_attention(ctx, qkv, total_tokens, cu_seqlens, batch, max_len, out, nullptr,
                                tz::pick_stream(ctx, stream), false, bf16 != 0);
}
