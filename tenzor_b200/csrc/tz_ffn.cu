// tz_ffn.cu -- the W8A8 feed-forward block of an encoder layer as ONE persistent tcgen05 kernel:
//
//   H        = GELU(float(XQ[M, 384] * W1[1536, 384]^T) * (s_x * s_w1) + b1)     (f16 values)
//   HQ, s_h  = per-token int8 quantisation of H (s_h = max|H| / 127)
//   x_out    = LayerNorm(float(HQ * W2[384, 1536]^T) * (s_h * s_w2) + b2 + residual)
//   XQ', s_x'= per-token int8 quantisation of x_out                     (the next layer's operand)
//
// Reference: feedForward (arctic.zig:760-810) -- intermediate dense, GELU (arctic.zig:750-756),
// output dense, residual add, layerNormLastDim (layernorm.zig:26-116) -- in the W8A8 form whose
// GEMMs accumulate int8 x int8 in int32.  The arithmetic is the two-kernel path's (gemm_tc's GELU
// epilogue followed by gemm_ln with in-kernel A quantisation) operation for operation, so both
// paths give bit-identical results; what changes is that H never leaves the SM.
//
// Per 128-row tile (one tile per CTA at the configs[1] batch, 142 tiles on 148 SMs):
//   pass 1  FFN1 in twelve 128-column chunks; the epilogue warps form H and keep only each row's
//           max|H| (the per-token scale needs the whole row before any value can be quantised);
//   pass 2  FFN1 again, chunk by chunk: H is formed once more (the same instructions on the same
//           accumulators: the same values), quantised with the row's scale into a shared-memory
//           chunk, and FFN2 accumulates that chunk on the tensor core while the next FFN1 chunk
//           runs;
//   LN      FFN2's 384-column accumulator goes through gemm_ln's four epilogue passes (dequantise +
//           bias + residual, mean, variance, normalise + int8 output).
// The recomputed FFN1 costs 50% more MMAs than the two-kernel path, but removes H's round trip
// (T x 1536 f16 written and read back), FFN2's f16 operand loads and one launch per layer.
//
// Roles (64 + 16 x 32 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2..17
// epilogue (warp w reads TMEM lane quarter w % 4).  Shared memory: the tile's int8 operand XQ
// (3 K blocks, 48 KB, resident for both passes), a ring of seven 16 KB weight units (128 rows x
// 128 bytes: one K block of a W1 chunk or one 128-row block of a W2 chunk, in the MMA's order), two
// quantised H chunks (16 KB each), the per-column vectors.  TMEM (512 columns): FFN2's accumulator D2 at columns 0..383 and
// an FFN1 chunk accumulator at 384..511; pass 1, which has no D2 yet, uses all four 128-column
// blocks as chunk buffers.  Every wait is bounded (1 s) and reports through the status word.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tz_internal.h"
#include "tz_ptx.cuh"
#include "tz_rowops.cuh"

namespace tz {
namespace {

constexpr int kH = 384, kF = 1536, kNC = 128, kChunks = kF / kNC;
constexpr int kEpiWarps = 16, kThreads = 64 + 32 * kEpiWarps;
constexpr int kUnit = 128 * 128;  // one 128-row x 128-byte int8 box
constexpr int kRing = 7;
constexpr int kUnitsPass1 = kChunks * 3;              // W1 chunk j, K block kb
constexpr int kUnitsPerTile = kUnitsPass1 + kChunks * 6;  // + W1 chunk j and W2 chunk j (3 row blocks)
constexpr int kSliceL = kH / 4;  // LayerNorm columns per epilogue warp (96)
constexpr int kOutBox = 32 * kSliceL;  // one warp's int8 output block (32 rows x 96 bytes)

constexpr int OFF_XQ = 0;
constexpr int OFF_RING = OFF_XQ + 3 * kUnit;
constexpr int OFF_H = OFF_RING + kRing * kUnit;
constexpr int OFF_VEC = OFF_H + 2 * kUnit;           // b2, s2, gamma, beta [384] f32 each
constexpr int OFF_VEC1 = OFF_VEC + 4 * kH * 4;       // b1, s1 [1536] f32 each
constexpr int OFF_RED = OFF_VEC1 + 2 * kF * 4;       // row reductions [4 kinds][4 slices][128]
constexpr int OFF_BAR = OFF_RED + 4 * 4 * 128 * 4;
constexpr int SMEM = OFF_BAR + 512 + 1024;           // + barriers, alignment slack
static_assert(SMEM <= 227 * 1024, "shared memory");
static_assert(kEpiWarps * kOutBox <= 3 * kUnit, "the int8 output blocks are staged in the XQ region");

struct FfnParams {
    const float* s1;
    const float* b1;
    const float* s2;
    const float* b2;
    const float* gamma;
    const float* beta;
    float eps;
    float* x;       // residual stream, blocked (xblk), updated in place
    float* xs;      // per-token scales of XQ: read at the tile's start, rewritten with the output's
    int32_t* dbg_acc1;  // parity capture (or null): FFN1 accumulators [M, 1536]
    __half* dbg_h16;    // H as quantised [M, 1536]
    int8_t* dbg_hq;     // its int8 form [M, 1536]
    float* dbg_hs;      // its per-token scales [M]
    int32_t* dbg_acc2;  // FFN2 accumulators [M, 384]
};

// Chunk g of a tile's sequence is chunk (g + rot) % 12 of the FFN dimension, rot = tile % 12: the
// row max (pass 1) and the int32 FFN2 sum (pass 2) do not depend on the order, and rotating it per
// tile spreads the CTAs' simultaneous weight requests over different parts of W1 and W2 (the CTAs
// run in lock step, so without it every SM asks for the same 16 KB box at the same moment).
__device__ __forceinline__ int chunk_at(int g, int rot) {
    const int c = g + rot;
    return c < kChunks ? c : c - kChunks;
}

// The tile-local unit sequence, in the order the MMA warp consumes it (chunks in sequence order):
// pass 1 W1(0, 0..2) .. W1(11, 0..2); pass 2 W1(0, 0..2), then for g = 0..10: W1(g + 1, 0..2),
// W2(g, 0..2); W2(11, 0..2).  W1(g, kb): rows 128 c.. of W1, K columns 128 kb..; W2(g, nb): rows
// 128 nb.. of W2, K columns 128 c.. (c = chunk_at(g, rot)).
__device__ __forceinline__ void unit_of(int i, int rot, bool& w2, int& x, int& y) {
    int j, r;
    if (i < kUnitsPass1) {
        w2 = false;
        x = (i % 3) * 128;
        y = chunk_at(i / 3, rot) * 128;
        return;
    }
    i -= kUnitsPass1;
    if (i < 3) {
        w2 = false;
        x = i * 128;
        y = chunk_at(0, rot) * 128;
        return;
    }
    i -= 3;
    j = i / 6;
    r = i % 6;
    if (j < kChunks - 1 && r < 3) {  // W1(j + 1, r)
        w2 = false;
        x = r * 128;
        y = chunk_at(j + 1, rot) * 128;
    } else {  // W2(j, r - 3), or W2(11, r) for the last three
        w2 = true;
        const int nb = j < kChunks - 1 ? r - 3 : r;
        x = chunk_at(j, rot) * 128;
        y = nb * 128;
    }
}

__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t parity, int lane, int* status) {
    __syncwarp();
    if (lane == 0) tzp::mbar_arrive(bar);
    return tzp::mbar_wait(bar, parity, status, nullptr);
}

// One epilogue thread's 32 columns of an FFN1 chunk (b1c / s1c: their bias and scale in shared
// memory): dequantise (acc * (s_x * s_w1) + b1), GELU
// (arctic.zig:750-756 with the hardware tanh), round to f16 pairs -- gemm_tc's GELU epilogue
// instruction for instruction (packed f32x2 arithmetic, each operation one rounding).
__device__ __forceinline__ void ffn1_h16(const uint32_t (&acc)[32], const float* b1c, const float* s1c, uint64_t rs2,
                                         uint32_t (&h)[16]) {
    const uint64_t kG0 = tzp::f2_pack(0.7978845608f, 0.7978845608f);
    const uint64_t kG1 = tzp::f2_pack(0.7978845608f * 0.044715f, 0.7978845608f * 0.044715f);
    const uint64_t kHalf2 = tzp::f2_pack(0.5f, 0.5f);
#pragma unroll
    for (int q4 = 0; q4 < 8; ++q4) {
        const ulonglong2 bv = reinterpret_cast<const ulonglong2*>(b1c)[q4];
        const ulonglong2 sv = reinterpret_cast<const ulonglong2*>(s1c)[q4];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = 2 * q4 + u;
            uint64_t x = tzp::f2_pack(__int2float_rn(static_cast<int>(acc[2 * j])), __int2float_rn(static_cast<int>(acc[2 * j + 1])));
            x = tzp::f2_mul(x, tzp::f2_mul(rs2, u ? sv.y : sv.x));
            x = tzp::f2_add(x, u ? bv.y : bv.x);
            const uint64_t inner = tzp::f2_mul(x, tzp::f2_fma(tzp::f2_mul(x, x), kG1, kG0));
            const float2 in = tzp::f2_unpack(inner);
            const uint64_t th = tzp::f2_pack(tzp::tanh_approx(in.x), tzp::tanh_approx(in.y));
            const uint64_t hx = tzp::f2_mul(x, kHalf2);
            x = tzp::f2_fma(hx, th, hx);
            const float2 r = tzp::f2_unpack(x);
            h[j] = tzp::pack16x2<false>(r.x, r.y);
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1)
    ffn_w8a8_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmXo,
                    const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmW2, int M,
                    FfnParams p, int* status) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = tzp::smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* xq = smem + OFF_XQ;
    uint8_t* ring = smem + OFF_RING;
    uint8_t* hbuf = smem + OFF_H;
    float* sv_b = reinterpret_cast<float*>(smem + OFF_VEC);  // b2, s2, gamma, beta
    float* sv_s = sv_b + kH;
    float* sv_g = sv_s + kH;
    float* sv_be = sv_g + kH;
    float* sv_b1 = reinterpret_cast<float*>(smem + OFF_VEC1);  // b1, s1: every chunk's epilogue reads them
    float* sv_s1 = sv_b1 + kF;
    float* red_h = reinterpret_cast<float*>(smem + OFF_RED);  // [4 slices][128 rows] each
    float* red_sum = red_h + 4 * 128;
    float* red_ssq = red_sum + 4 * 128;
    float* red_max = red_ssq + 4 * 128;
    uint64_t* ufull = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* uempty = ufull + kRing;
    uint64_t* xfull = uempty + kRing;
    uint64_t* xempty = xfull + 1;
    uint64_t* tfull = xempty + 1;   // [4] FFN1 chunk buffers (TMEM columns 128 b)
    uint64_t* tempty = tfull + 4;   // [4]
    uint64_t* d2full = tempty + 4;
    uint64_t* d2empty = d2full + 1;
    uint64_t* hfull = d2empty + 1;  // [2]
    uint64_t* hempty = hfull + 2;   // [2]
    uint64_t* red_bar = hempty + 2; // [4]: row max of H, LayerNorm sum, ssq, output |max|
    uint64_t* drain = red_bar + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRing; ++s) {
            tzp::mbar_init(&ufull[s], 1);
            tzp::mbar_init(&uempty[s], 1);
        }
        tzp::mbar_init(xfull, 1);
        tzp::mbar_init(xempty, kEpiWarps);
        for (int b = 0; b < 4; ++b) {
            tzp::mbar_init(&tfull[b], 1);
            tzp::mbar_init(&tempty[b], kEpiWarps);
        }
        tzp::mbar_init(d2full, 1);
        tzp::mbar_init(d2empty, kEpiWarps);
        for (int b = 0; b < 2; ++b) {
            tzp::mbar_init(&hfull[b], 32 * kEpiWarps);
            tzp::mbar_init(&hempty[b], 1);
        }
        for (int i = 0; i < 4; ++i) tzp::mbar_init(&red_bar[i], kEpiWarps);
        tzp::mbar_init(drain, 1);
        *abort_flag = 0;
        tzp::fence_mbar_init();
        tzp::tma_prefetch_desc(&tmX);
        tzp::tma_prefetch_desc(&tmXo);
        tzp::tma_prefetch_desc(&tmW1);
        tzp::tma_prefetch_desc(&tmW2);
    }
    if (warp == 1) {
        tzp::tmem_alloc(tmem_slot, 512);
        tzp::tmem_relinquish();
    }
    if (warp >= 2) {  // per-column vectors are weights: read before waiting on the previous kernel
        for (int i = threadIdx.x - 64; i < kH; i += 32 * kEpiWarps) {
            sv_b[i] = p.b2[i];
            sv_s[i] = p.s2[i];
            sv_g[i] = p.gamma[i];
            sv_be[i] = p.beta[i];
        }
        for (int i = threadIdx.x - 64; i < kF / 4; i += 32 * kEpiWarps) {
            reinterpret_cast<float4*>(sv_b1)[i] = __ldg(reinterpret_cast<const float4*>(p.b1) + i);
            reinterpret_cast<float4*>(sv_s1)[i] = __ldg(reinterpret_cast<const float4*>(p.s1) + i);
        }
    }
    tzp::tc_fence_before();
    __syncthreads();
    tzp::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_tiles = (M + 127) / 128;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t u = 0;           // units issued so far (ring slot u % kRing, phase (u / kRing) & 1)
            uint32_t xload = 0;       // XQ loads issued
            bool ok = true;
            int rot = 0;
            auto issue = [&](int i) -> bool {
                const uint32_t slot = u % kRing;
                if (!tzp::mbar_wait(&uempty[slot], ((u / kRing) & 1u) ^ 1u, status, abort_flag)) return false;
                bool w2;
                int x, y;
                unit_of(i, rot, w2, x, y);
                tzp::mbar_arrive_expect_tx(&ufull[slot], kUnit);
                tzp::tma_load_2d(ring + slot * kUnit, w2 ? &tmW2 : &tmW1, x, y, &ufull[slot]);
                ++u;
                return true;
            };
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
                // The first ring-full of this tile's weight units: their slots were freed by the
                // previous tile's MMAs, which never wait on this tile's XQ.
                rot = tile % kChunks;
                int i = 0;
                for (; i < kRing && ok; ++i) ok = issue(i);
                if (!ok) break;
                if (it == 0) tzp::pdl_wait();  // XQ is the previous kernel's output
                if (!tzp::mbar_wait(xempty, (static_cast<uint32_t>(it) & 1u) ^ 1u, status, abort_flag)) break;
                tzp::mbar_arrive_expect_tx(xfull, 3 * kUnit);
                for (int kb = 0; kb < 3; ++kb) tzp::tma_load_2d(xq + kb * kUnit, &tmX, kb * 128, tile * 128, xfull);
                ++xload;
                for (; i < kUnitsPerTile && ok; ++i) ok = issue(i);
            }
            // nothing may land in shared memory after the CTA exits: wait for every load issued
            const uint32_t first = u > kRing ? u - kRing : 0u;
            for (uint32_t v = first; v < u; ++v) tzp::mbar_wait(&ufull[v % kRing], (v / kRing) & 1u, status, nullptr);
            if (xload) tzp::mbar_wait(xfull, (xload - 1) & 1u, status, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tzp::make_idesc(2u, 1u, 128, 128);  // s32 accumulate, signed int8, M = N = 128
            const uint64_t xd = tzp::sdesc_k128(tzp::smem_u32(xq));
            uint32_t u = 0;
            uint32_t tph = 0, hph = 0;  // bit b: phase parity of TMEM chunk buffer b / H buffer b
            bool ok = true;
            // A unit's four K steps (32 bytes each) into `d`, A from descriptor `ad`
            auto mma_unit = [&](uint32_t d, uint64_t ad, bool first) -> bool {
                const uint32_t slot = u % kRing;
                if (!tzp::mbar_wait(&ufull[slot], (u / kRing) & 1u, status, abort_flag)) return false;
                tzp::tc_fence_after();
                const uint64_t bd = tzp::sdesc_k128(tzp::smem_u32(ring + slot * kUnit));
#pragma unroll
                for (int k = 0; k < 4; ++k) tzp::umma<KIND_I8>(d, ad + 2u * k, bd + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
                tzp::umma_commit(&uempty[slot]);
                ++u;
                return true;
            };
            // FFN1 chunk into TMEM buffer b (columns 128 b): three K blocks of XQ
            auto ffn1 = [&](int b) -> bool {
                if (!tzp::mbar_wait(&tempty[b], ((tph >> b) & 1u) ^ 1u, status, abort_flag)) return false;
                tzp::tc_fence_after();
                for (int kb = 0; kb < 3; ++kb)
                    if (!mma_unit(tmem_base + 128u * b, xd + static_cast<uint64_t>((kb * kUnit) >> 4), kb == 0)) return false;
                tzp::umma_commit(&tfull[b]);
                tph ^= 1u << b;
                return true;
            };
            // FFN2 chunk g: H buffer g & 1 against W2's three 128-row blocks, into D2
            auto ffn2 = [&](int g) -> bool {
                const int hb = g & 1;
                if (!tzp::mbar_wait(&hfull[hb], (hph >> hb) & 1u, status, abort_flag)) return false;
                tzp::tc_fence_after();
                const uint64_t hd = tzp::sdesc_k128(tzp::smem_u32(hbuf + hb * kUnit));
                for (int nb = 0; nb < 3; ++nb)
                    if (!mma_unit(tmem_base + 128u * nb, hd, g == 0)) return false;
                tzp::umma_commit(&hempty[hb]);
                hph ^= 1u << hb;
                return true;
            };
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
                const uint32_t par = static_cast<uint32_t>(it) & 1u;
                if (!tzp::mbar_wait(xfull, par, status, abort_flag)) break;
                // the previous tile's D2 (TMEM columns 0..383) must be drained before pass 1 reuses them
                if (!tzp::mbar_wait(d2empty, par ^ 1u, status, abort_flag)) break;
                tzp::tc_fence_after();
                for (int j = 0; j < kChunks && ok; ++j) ok = ffn1(j & 3);  // pass 1
                if (!ok) break;
                // pass 2: D2 takes columns 0..383 once pass 1's last uses of them are drained
                for (int b = 0; b < 3 && ok; ++b) ok = tzp::mbar_wait(&tempty[b], ((tph >> b) & 1u) ^ 1u, status, abort_flag);
                if (!ok) break;
                tzp::tc_fence_after();
                ok = ffn1(3);
                for (int g = 0; g < kChunks - 1 && ok; ++g) {
                    ok = ffn1(3);
                    if (ok) ok = ffn2(g);
                }
                if (ok) ok = ffn2(kChunks - 1);
                if (!ok) break;
                tzp::umma_commit(d2full);
            }
            tzp::umma_commit(drain);
            tzp::mbar_wait(drain, 0, status, nullptr);
        }
    } else {
        tzp::pdl_wait();
        const int e = warp - 2;
        const int q = warp & 3;
        const int sl = e >> 2;
        const int rloc = q * 32 + lane;
        const uint32_t tlane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        uint32_t tph = 0, hph = 0;  // bit b: phase parity of TMEM chunk buffer b / H buffer b
        int it = 0;
        bool bad = false;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
            const uint32_t par = static_cast<uint32_t>(it) & 1u;
            const int row0 = tile * 128 + q * 32;
            const int row = row0 + lane;
            const bool ok = row < M;
            const int rot = tile % kChunks;
            const float xsv = ok ? p.xs[row] : 1.0f;
            const uint64_t rs2 = tzp::f2_pack(xsv, xsv);

            // ---- pass 1: each row's max |H| over the 1536 columns ----
            uint32_t amax2 = 0u;  // packed f16 pair; only the magnitudes matter (xorsign max)
            for (int j = 0; j < kChunks; ++j) {
                const int b = j & 3;
                if (!tzp::mbar_wait(&tfull[b], (tph >> b) & 1u, status, abort_flag)) {
                    bad = true;
                    break;
                }
                tph ^= 1u << b;
                tzp::tc_fence_after();
                uint32_t acc[32];
                tzp::tmem_ld32(tlane + 128u * b + 32u * sl, acc);
                tzp::tmem_ld_wait();
                tzp::tc_fence_before();
                __syncwarp();
                if (lane == 0) tzp::mbar_arrive(&tempty[b]);
                uint32_t h[16];
                const int c1 = chunk_at(j, rot) * kNC + 32 * sl;
                ffn1_h16(acc, sv_b1 + c1, sv_s1 + c1, rs2, h);
#pragma unroll
                for (int i = 0; i < 16; ++i) amax2 = tzp::hmax2_xorsign_abs(amax2, h[i]);
            }
            if (bad) break;
            red_h[sl * 128 + rloc] = fmaxf(fabsf(__low2float(*reinterpret_cast<const __half2*>(&amax2))),
                                           fabsf(__high2float(*reinterpret_cast<const __half2*>(&amax2))));
            if (!epi_sync(&red_bar[0], par, lane, status)) break;
            const float hm = fmaxf(fmaxf(red_h[rloc], red_h[128 + rloc]), fmaxf(red_h[256 + rloc], red_h[384 + rloc]));
            const float hsc = (hm == 0.0f) ? 1.0f : __fdiv_rn(hm, 127.0f);
            const uint64_t hinv2 = tzp::f2_pack(__fdiv_rn(1.0f, hsc), __fdiv_rn(1.0f, hsc));
            if (p.dbg_hs != nullptr && ok && sl == 0) p.dbg_hs[row] = hsc;
            // this warp's residual slice (32 rows x 96 columns, 12 KB contiguous) into L2 for the LayerNorm
            if (lane == 0) tzp::bulk_prefetch_l2(p.x + xblk(row0, sl * kSliceL), 32 * kSliceL * 4);

            // ---- pass 2: H again, quantised per token into the FFN2 operand chunks ----
            for (int j = 0; j < kChunks; ++j) {
                if (!tzp::mbar_wait(&tfull[3], (tph >> 3) & 1u, status, abort_flag)) {
                    bad = true;
                    break;
                }
                tph ^= 8u;
                tzp::tc_fence_after();
                uint32_t acc[32];
                tzp::tmem_ld32(tlane + 384u + 32u * sl, acc);
                tzp::tmem_ld_wait();
                tzp::tc_fence_before();
                __syncwarp();
                if (lane == 0) tzp::mbar_arrive(&tempty[3]);
                const int col = chunk_at(j, rot) * kNC + 32 * sl;
                if (p.dbg_acc1 != nullptr && ok) {
                    int4* d = reinterpret_cast<int4*>(p.dbg_acc1 + static_cast<long long>(row) * kF + col);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        d[i] = make_int4(static_cast<int>(acc[4 * i]), static_cast<int>(acc[4 * i + 1]),
                                         static_cast<int>(acc[4 * i + 2]), static_cast<int>(acc[4 * i + 3]));
                }
                uint32_t h[16];
                ffn1_h16(acc, sv_b1 + col, sv_s1 + col, rs2, h);
                uint32_t w[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&h[2 * i]));
                    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&h[2 * i + 1]));
                    w[i] = __byte_perm(quant2_own_max(f0.x, f0.y, hinv2), quant2_own_max(f1.x, f1.y, hinv2), 0x5410);
                }
                if (ok && p.dbg_h16 != nullptr) {
                    uint4* d = reinterpret_cast<uint4*>(p.dbg_h16 + static_cast<long long>(row) * kF + col);
#pragma unroll
                    for (int i = 0; i < 4; ++i) d[i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
                }
                if (ok && p.dbg_hq != nullptr) {
                    uint4* d = reinterpret_cast<uint4*>(p.dbg_hq + static_cast<long long>(row) * kF + col);
                    d[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    d[1] = make_uint4(w[4], w[5], w[6], w[7]);
                }
                const int hb = j & 1;
                int got = 1;  // FFN2 of chunk j - 2 has read this H buffer
                if (lane == 0) got = tzp::mbar_wait(&hempty[hb], ((hph >> hb) & 1u) ^ 1u, status, abort_flag) ? 1 : 0;
                got = __shfl_sync(0xffffffffu, got, 0);
                hph ^= 1u << hb;
                if (!got) {
                    bad = true;
                    break;
                }
                // row rloc of the SWIZZLE_128B chunk: 16-byte piece c at c ^ (rloc % 8); this thread's
                // 32 columns are pieces 2 sl and 2 sl + 1
                const uint32_t rowa = tzp::smem_u32(hbuf + hb * kUnit) + static_cast<uint32_t>(rloc * 128);
                tzp::st_shared_v4(rowa + (static_cast<uint32_t>((2 * sl) ^ (rloc & 7)) << 4), w[0], w[1], w[2], w[3]);
                tzp::st_shared_v4(rowa + (static_cast<uint32_t>((2 * sl + 1) ^ (rloc & 7)) << 4), w[4], w[5], w[6], w[7]);
                tzp::fence_proxy_async();
                tzp::mbar_arrive(&hfull[hb]);
            }
            if (bad) break;

            // ---- LayerNorm epilogue on D2 (gemm_ln's passes A..D) ----
            if (!tzp::mbar_wait(d2full, par, status, abort_flag)) break;
            tzp::tc_fence_after();
            const int c0 = sl * kSliceL;
            const uint32_t tbase = tlane + static_cast<uint32_t>(c0);
            if (p.dbg_acc2 != nullptr) {  // parity capture: the raw FFN2 accumulators, before pass A rewrites TMEM
#pragma unroll 1
                for (int c = 0; c < kSliceL / 16; ++c) {
                    uint32_t r[16];
                    tzp::tmem_ld16(tbase + 16 * c, r);
                    tzp::tmem_ld_wait();
                    if (ok) {
                        int4* d = reinterpret_cast<int4*>(p.dbg_acc2 + static_cast<long long>(row) * kH + c0 + 16 * c);
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            d[i] = make_int4(static_cast<int>(r[4 * i]), static_cast<int>(r[4 * i + 1]),
                                             static_cast<int>(r[4 * i + 2]), static_cast<int>(r[4 * i + 3]));
                    }
                }
            }
            // pass A: x = acc * (s_h * s_w2) + b2 + residual -> TMEM; row sum
            const uint64_t hs2 = tzp::f2_pack(hsc, hsc);
            uint64_t sum2 = 0;
            const float* resw = p.x + xblk(row0, c0) + lane * 4;
#pragma unroll
            for (int c = 0; c < kSliceL / 16; ++c) {
                uint32_t r[16];
                tzp::tmem_ld16(tbase + 16 * c, r);
                float4 cur[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) cur[i] = *reinterpret_cast<const float4*>(resw + c * 512 + i * 128);
                tzp::tmem_ld_wait();
                const int col = c0 + 16 * c;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    uint64_t x = tzp::f2_pack(__int2float_rn(static_cast<int>(r[2 * i])), __int2float_rn(static_cast<int>(r[2 * i + 1])));
                    const uint64_t cs2 = *reinterpret_cast<const uint64_t*>(sv_s + col + 2 * i);
                    x = tzp::f2_mul(x, tzp::f2_mul(hs2, cs2));
                    const uint64_t b2 = *reinterpret_cast<const uint64_t*>(sv_b + col + 2 * i);
                    const uint64_t res2 = reinterpret_cast<const uint64_t*>(cur)[i];
                    x = tzp::f2_add(tzp::f2_add(x, b2), res2);
                    sum2 = tzp::f2_add(sum2, x);
                    const float2 v = tzp::f2_unpack(x);
                    r[2 * i] = __float_as_uint(v.x);
                    r[2 * i + 1] = __float_as_uint(v.y);
                }
                tzp::tmem_st16(tbase + 16 * c, r);
            }
            tzp::tmem_st_wait();
            {
                const float2 sp = tzp::f2_unpack(sum2);
                red_sum[sl * 128 + rloc] = sp.x + sp.y;
            }
            if (!epi_sync(&red_bar[1], par, lane, status)) break;
            const float mean =
                ((red_sum[rloc] + red_sum[128 + rloc]) + (red_sum[256 + rloc] + red_sum[384 + rloc])) / static_cast<float>(kH);
            // pass B: sum of squared deviations
            const uint64_t mean2 = tzp::f2_pack(mean, mean);
            uint64_t ssq2 = 0;
#pragma unroll
            for (int c = 0; c < kSliceL / 16; ++c) {
                uint32_t r[16];
                tzp::tmem_ld16(tbase + 16 * c, r);
                tzp::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint64_t d = tzp::f2_sub(tzp::f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), mean2);
                    ssq2 = tzp::f2_fma(d, d, ssq2);
                }
            }
            {
                const float2 sp = tzp::f2_unpack(ssq2);
                red_ssq[sl * 128 + rloc] = sp.x + sp.y;
            }
            if (!epi_sync(&red_bar[2], par, lane, status)) break;
            const float var =
                ((red_ssq[rloc] + red_ssq[128 + rloc]) + (red_ssq[256 + rloc] + red_ssq[384 + rloc])) / static_cast<float>(kH);
            const float inv_std = 1.0f / sqrtf(var + p.eps);
            const uint64_t istd2 = tzp::f2_pack(inv_std, inv_std);
            // pass C: normalise, store x_out, y -> TMEM, |max|
            float amax = 0.f;
#pragma unroll
            for (int c = 0; c < kSliceL / 16; ++c) {
                uint32_t r[16];
                tzp::tmem_ld16(tbase + 16 * c, r);
                tzp::tmem_ld_wait();
                const int col = c0 + 16 * c;
                float y[16];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint64_t x = tzp::f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
                    const uint64_t g2 = *reinterpret_cast<const uint64_t*>(sv_g + col + 2 * i);
                    const uint64_t b2 = *reinterpret_cast<const uint64_t*>(sv_be + col + 2 * i);
                    const float2 v = tzp::f2_unpack(tzp::f2_fma(tzp::f2_mul(tzp::f2_sub(x, mean2), istd2), g2, b2));
                    y[2 * i] = v.x;
                    y[2 * i + 1] = v.y;
                }
                float* xo = p.x + xblk(row0, col) + lane * 4;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    *reinterpret_cast<float4*>(xo + i * 128) = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    amax = fmaxf(amax, fabsf(y[i]));
                    r[i] = __float_as_uint(y[i]);
                }
                tzp::tmem_st16(tbase + 16 * c, r);
            }
            // pass D: per-token int8 quantisation of the LayerNorm output (the next QKV operand)
            tzp::tmem_st_wait();
            red_max[sl * 128 + rloc] = amax;
            if (!epi_sync(&red_bar[3], par, lane, status)) break;
            const float m = fmaxf(fmaxf(red_max[rloc], red_max[128 + rloc]), fmaxf(red_max[256 + rloc], red_max[384 + rloc]));
            const float sc = (m == 0.0f) ? 1.0f : __fdiv_rn(m, 127.0f);
            const float inv = __fdiv_rn(1.0f, sc);
            const uint64_t inv2 = tzp::f2_pack(inv, inv);
            // this warp's 32 x 96 int8 block, row-major, staged in the XQ region (every MMA that read
            // XQ completed before d2full), then one TMA store
            uint8_t* obox = xq + e * kOutBox;
            uint8_t* qrow = obox + lane * kSliceL;
#pragma unroll
            for (int c = 0; c < kSliceL / 16; ++c) {
                uint32_t r[16];
                tzp::tmem_ld16(tbase + 16 * c, r);
                tzp::tmem_ld_wait();
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    w[i] = __byte_perm(quant2_own_max(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]), inv2),
                                       quant2_own_max(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]), inv2), 0x5410);
                *reinterpret_cast<uint4*>(qrow + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            // D2 fully read: the next tile's MMAs may take TMEM columns 0..383
            tzp::tc_fence_before();
            tzp::fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                tzp::mbar_arrive(d2empty);
                tzp::tma_store_2d(&tmXo, obox, c0, row0);
                tzp::bulk_commit();
                tzp::bulk_wait_read<0>();  // the block is read: the producer may load the next tile's XQ
                tzp::mbar_arrive(xempty);
            }
            if (ok && sl == 0) p.xs[row] = sc;
        }
        if (lane == 0) tzp::bulk_wait_all();
    }

    tzp::pdl_trigger();
    tzp::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tzp::tc_fence_after();
        tzp::tmem_dealloc(tmem_base, 512);
    }
}

}  // namespace

int launch_ffn_w8a8(tz_ctx_t ctx, const FfnArgs& a, cudaStream_t s) {
    TZ_CHECK(a.M >= 0, TZ_EINVAL, "ffn: bad shape");
    if (a.M == 0) return TZ_OK;
    TZ_CHECK(a.xq && a.xs && a.w1 && a.s1 && a.b1 && a.w2 && a.s2 && a.b2 && a.gamma && a.beta && a.x, TZ_EINVAL,
             "ffn: null operand");
    TZ_CHECK(reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && reinterpret_cast<uintptr_t>(a.xq) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(a.b1) % 16 == 0 && reinterpret_cast<uintptr_t>(a.s1) % 16 == 0,
             TZ_EINVAL, "ffn: operands must be 16-byte aligned");
    TZ_CHECK(reinterpret_cast<uintptr_t>(a.dbg_acc1) % 16 == 0 && reinterpret_cast<uintptr_t>(a.dbg_h16) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(a.dbg_hq) % 16 == 0 && reinterpret_cast<uintptr_t>(a.dbg_acc2) % 16 == 0,
             TZ_EINVAL, "ffn: capture buffers must be 16-byte aligned");
    static unsigned attr_set = 0;
    int dev = 0;
    TZ_CUDA(cudaGetDevice(&dev));
    if (!(attr_set & (1u << (dev & 31)))) {
        TZ_CUDA(cudaFuncSetAttribute(ffn_w8a8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        attr_set |= 1u << (dev & 31);
    }
    CUtensorMap tx, txo, tw1, tw2;
    const uint64_t M = static_cast<uint64_t>(a.M);
    int rc = encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.xq, kH, M, kH, 128, 128);
    if (!rc) rc = encode_tmap_2d_swz(&txo, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.xq, kH, M, kH, kSliceL, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!rc) rc = encode_tmap_2d(&tw1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w1, kH, kF, kH, 128, 128);
    if (!rc) rc = encode_tmap_2d(&tw2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w2, kF, kH, kF, 128, 128);
    if (rc) return rc;
    FfnParams p{a.s1, a.b1, a.s2, a.b2, a.gamma, a.beta, a.eps, a.x, a.xs,
                a.dbg_acc1, static_cast<__half*>(a.dbg_h16), a.dbg_hq, a.dbg_hs, a.dbg_acc2};
    const int tiles = (a.M + 127) / 128;
    const int sms = ctx->sm_count - ctx->sm_reserve;
    const int grid = tiles < sms ? tiles : sms;
    if (grid <= 0) return TZ_OK;
    return launch_kernel(ffn_w8a8_kernel, dim3(grid), dim3(kThreads), SMEM, s, a.pdl, tx, txo, tw1, tw2, a.M, p,
                         ctx->d_status);
}

}  // namespace tz
