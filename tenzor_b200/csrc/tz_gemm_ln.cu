// tz_gemm_ln.cu -- tcgen05 GEMM whose epilogue finishes a post-LN transformer sub-block:
//
//   x_out[M, 384] = LayerNorm( dequant(A[M, K] * W[384, K]^T) + bias + residual )
//   aux[M, 384]   = f16(x_out)                          (AUX = 0: the next GEMM's f16 operand)
//                 | int8(x_out) with per-row scale       (AUX = 1: the next GEMM's W8A8 operand)
//                 | bf16(x_out)                          (AUX = 2: the next GEMM's bf16 operand)
//
// Reference: selfAttention's output projection + residual + LayerNorm (arctic.zig:716-746) and
// feedForward's second projection + residual + LayerNorm (arctic.zig:779-807); layerNormLastDim
// numerics of layernorm.zig:26-116 (mean, then the mean of squared deviations, 1/sqrt(var+eps)).
//
// One CTA owns whole 128-row blocks (persistent over row blocks): the full 384-column accumulator
// lives in TMEM (two N=192 MMAs per K step).  64 + 16*32 threads: warp 0 TMA producer (A block and
// the two 192-row halves of W per 128-byte K block), warp 1 TMEM owner + MMA issuer, warps 2..17
// epilogue: warp w reads TMEM lane quarter (w % 4) and a 96-column slice.  Per row: pass A
// dequantises, adds bias and residual, writes x back into TMEM and sums; pass B sums squared
// deviations; pass C normalises and stores x_out (+ f16 aux, or y back to TMEM and |max|); pass D
// (AUX = 1) quantises.  The residual stream is in the blocked layout of xblk (tz_internal.h): a
// warp's 32 x 16 residual chunk is 2 KB contiguous, and its x_out chunk leaves as four coalesced
// 512-byte stores.  The four slices of a row combine their partial sums through shared memory at
// mbarriers (bounded waits, one phase per tile).  No separate LayerNorm launch and no round trip of
// the pre-LN activations.
//
// Two shared-memory layouts (Layout<AQ>):
//  * TMA-fed A (AQ = 0: the f16-operand modes): a 3-stage ring, so a K block's weight tile is
//    requested two MMA blocks ahead and its L2 latency hides under the MMAs; the residual chunks are
//    read with coalesced direct loads (the warp's 12 KB slice prefetched into L2 at the tile's start).
//  * A quantised in the kernel (AQ = 1, W8A8): the mainloop is paced by the quantising epilogue
//    warps, not the weight loads, so a 2-stage ring suffices and the freed 64 KB stage residual
//    chunks (1-D bulk copies, two in flight per warp, the first two during the mainloop) and the
//    int8 output blocks (one TMA store per warp).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tz_internal.h"
#include "tz_ptx.cuh"
#include "tz_rowops.cuh"

namespace tz {
namespace {

constexpr int kN = 384, kHalf = 192, kEpiWarps = 16, kThreads = 64 + 32 * kEpiWarps;
constexpr int kBox = 32 * 16 * 4;  // one 32-row x 16-column f32 chunk of the residual (2 KB, contiguous in xblk form)
constexpr int kSlice = kN / 4;  // 96 columns per epilogue warp

struct LnParams {
    const float* bias;
    const float* col_scale;
    const float* row_scale;
    const float* residual;
    const float* gamma;
    const float* beta;
    float eps;
    float* x_out;
    void* aux;
    float* aux_scale;
    const __half* a16;    // AQ: f16 A [M, K]
    long long lda16;
    unsigned* a_absmax;   // AQ: per-row |max| bits of A
    int32_t* dbg_acc;     // parity capture (or null): raw accumulators [M, 384]
    int8_t* dbg_aq;       // AQ parity capture (or null): the int8 A rows as quantised [M, K]
    float* dbg_as;        // AQ parity capture (or null): their per-token scales [M]
};

template <int KIND, int AQ>
struct LnCfg {
    static constexpr int ELEM = KIND == KIND_I8 ? 1 : (KIND == KIND_TF32 ? 4 : 2);
    static constexpr int BK = 128 / ELEM;
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = kN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr bool BOXES = AQ != 0;  // residual / int8 output staged in shared memory
    static constexpr int STAGES = BOXES ? 2 : 3;
    static constexpr int STAGING = BOXES ? kEpiWarps * 2 * kBox : 0;  // two residual/output boxes per epilogue warp
    static constexpr int RED_BYTES = 3 * 4 * 128 * 4 + 4 * kN * 4;  // row reductions + the 4 column vectors
    static constexpr int SMEM = STAGES * STAGE_BYTES + STAGING + RED_BYTES + 512 + 1024;  // + barriers, alignment
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert((kSlice / 16) % 2 == 0, "x_out chunks are stored in pairs");
    static_assert(32 * kSlice <= 2 * kBox, "the int8 LayerNorm output of one warp fits its two staging boxes");
};

// All epilogue warps meet here (one arrival per warp after its shared-memory writes); bounded wait on
// the barrier's phase `parity` (one phase per tile).  False when the wait expired.
__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t parity, int lane, int* status) {
    __syncwarp();
    if (lane == 0) tzp::mbar_arrive(bar);
    return tzp::mbar_wait(bar, parity, status, nullptr);
}

template <int KIND>
__device__ __forceinline__ float acc_to_f(uint32_t r) {
    if constexpr (KIND == KIND_I8)
        return __int2float_rn(static_cast<int>(r));
    else
        return __uint_as_float(r);
}

// AQ = 1: the A operand arrives as f16 rows with their |max| and the epilogue warps quantise it into
// the int8 stages (per-token W8A8 scale s = |max| / 127, or 1 for an all-zero row; q = clamp(round(x /
// s))) while the producer streams only W: no separate requantisation pass over A.  The epilogue
// warps are otherwise idle during the mainloop (one TMEM accumulator: the MMAs of the next tile wait
// for this tile's epilogue anyway).
template <int KIND, int AUX, int AQ>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmAux, int M, int K,
                   LnParams p, int* status) {
    using C = LnCfg<KIND, AQ>;
    constexpr int kStages = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = tzp::smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* staging = smem + kStages * C::STAGE_BYTES;                          // [16 warps][2 boxes]
    float* red_sum = reinterpret_cast<float*>(staging + C::STAGING);             // [4 slices][128 rows]
    float* red_ssq = red_sum + 4 * 128;
    float* red_max = red_ssq + 4 * 128;
    float* sv_bias = red_max + 4 * 128;  // [384] each: bias, column scale, gamma, beta (shared memory copies)
    float* sv_cs = sv_bias + kN;
    float* sv_g = sv_cs + kN;
    float* sv_b = sv_g + kN;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STAGING + C::RED_BYTES);
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;
    uint64_t* tempty = tfull + 1;
    uint64_t* drain = tempty + 1;
    uint64_t* red_bar = drain + 1;  // [3]: the epilogue warps' row reductions (sum, ssq, max)
    uint64_t* res_bar = red_bar + 3;  // [16 warps][2 boxes] (BOXES): residual tile arrivals
    uint64_t* afull = res_bar + 2 * kEpiWarps;  // [kStages] (AQ): A stage quantised by all epilogue threads
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(afull + kStages);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            tzp::mbar_init(&full[s], 1);
            tzp::mbar_init(&empty[s], 1);
        }
        tzp::mbar_init(tfull, 1);
        tzp::mbar_init(tempty, kEpiWarps);
        tzp::mbar_init(drain, 1);
        for (int i = 0; i < 3; ++i) tzp::mbar_init(&red_bar[i], kEpiWarps);
        if (C::BOXES)
            for (int i = 0; i < 2 * kEpiWarps; ++i) tzp::mbar_init(&res_bar[i], 1);
        for (int s = 0; s < kStages; ++s) tzp::mbar_init(&afull[s], 32 * kEpiWarps);
        *abort_flag = 0;
        tzp::fence_mbar_init();
        tzp::tma_prefetch_desc(&tmA);
        tzp::tma_prefetch_desc(&tmB);
        if (AUX == 1) tzp::tma_prefetch_desc(&tmAux);
    }
    if (warp == 1) {
        tzp::tmem_alloc(tmem_slot, 512);
        tzp::tmem_relinquish();
    }
    if (warp >= 2) {  // the per-column vectors are weights: read them before waiting on the previous kernel
        for (int i = threadIdx.x - 64; i < kN; i += 32 * kEpiWarps) {
            sv_bias[i] = p.bias[i];
            sv_cs[i] = p.col_scale ? p.col_scale[i] : 1.0f;
            sv_g[i] = p.gamma[i];
            sv_b[i] = p.beta[i];
        }
    }
    tzp::tc_fence_before();
    __syncthreads();
    tzp::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Programmatic launch: the producer requests the weight tiles of its first stages before it
    // waits for the previous grid (griddepcontrol.wait); the epilogue warps wait before they read
    // the activations, row scales or residual that grid wrote.  The MMA warp reads no global memory.

    const int num_tiles = (M + 127) / 128;
    const int kblocks = (K + C::BK - 1) / C::BK;
    constexpr uint32_t kExpect = AQ ? C::B_BYTES : C::STAGE_BYTES;

    if (warp == 0) {
        if (lane == 0) {
            int pre = 0;  // K blocks of the first tile whose B tiles are already requested
            if (static_cast<int>(blockIdx.x) < num_tiles) {
                pre = kblocks < kStages ? kblocks : kStages;
                for (int kb = 0; kb < pre; ++kb) {
                    uint8_t* sb = smem + kb * C::STAGE_BYTES + C::A_BYTES;
                    tzp::mbar_arrive_expect_tx(&full[kb], kExpect);
                    tzp::tma_load_2d(sb, &tmB, kb * C::BK, 0, &full[kb]);
                    tzp::tma_load_2d(sb + kHalf * 128, &tmB, kb * C::BK, kHalf, &full[kb]);
                }
            }
            tzp::pdl_wait();
            int stage = 0;
            uint32_t phase = 0, armed = 0, armed_par = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tzp::mbar_wait(&empty[stage], phase ^ 1u, status, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + stage * C::STAGE_BYTES;
                    const bool b_done = tile == static_cast<int>(blockIdx.x) && kb < pre;
                    if (!b_done) tzp::mbar_arrive_expect_tx(&full[stage], kExpect);
                    if constexpr (!AQ) tzp::tma_load_2d(sa, &tmA, kb * C::BK, tile * 128, &full[stage]);
                    if (!b_done) {
                        tzp::tma_load_2d(sa + C::A_BYTES, &tmB, kb * C::BK, 0, &full[stage]);
                        tzp::tma_load_2d(sa + C::A_BYTES + kHalf * 128, &tmB, kb * C::BK, kHalf, &full[stage]);
                    }
                    armed |= 1u << stage;
                    armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
            }
            for (int s = 0; s < kStages; ++s)
                if (armed & (1u << s)) tzp::mbar_wait(&full[s], (armed_par >> s) & 1u, status, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t c_fmt = KIND == KIND_I8 ? 2u : 1u;
            constexpr uint32_t ab_fmt = KIND == KIND_I8 ? 1u : (KIND == KIND_TF32 ? 2u : (KIND == KIND_BF16 ? 1u : 0u));
            constexpr uint32_t idesc = tzp::make_idesc(c_fmt, ab_fmt, 128, kHalf);
            int stage = 0;
            uint32_t phase = 0, tphase = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                if (!tzp::mbar_wait(tempty, tphase ^ 1u, status, abort_flag)) break;
                tzp::tc_fence_after();
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tzp::mbar_wait(&full[stage], phase, status, abort_flag) ||
                        (AQ && !tzp::mbar_wait(&afull[stage], phase, status, abort_flag))) {
                        ok = false;
                        break;
                    }
                    tzp::tc_fence_after();
                    uint8_t* sa = smem + stage * C::STAGE_BYTES;
                    const uint64_t ad = tzp::sdesc_k128(tzp::smem_u32(sa));
                    const uint64_t bd0 = tzp::sdesc_k128(tzp::smem_u32(sa + C::A_BYTES));
                    const uint64_t bd1 = tzp::sdesc_k128(tzp::smem_u32(sa + C::A_BYTES + kHalf * 128));
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t acc = (kb | k) != 0 ? 1u : 0u;
                        tzp::umma<KIND>(tmem_base, ad + 2u * k, bd0 + 2u * k, idesc, acc);
                        tzp::umma<KIND>(tmem_base + kHalf, ad + 2u * k, bd1 + 2u * k, idesc, acc);
                    }
                    tzp::umma_commit(&empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tzp::umma_commit(tfull);
                tphase ^= 1u;
            }
            tzp::umma_commit(drain);
            tzp::mbar_wait(drain, 0, status, nullptr);
        }
    } else {
        tzp::pdl_wait();
        const int e = warp - 2;
        const int q = warp & 3;
        const int slice = e >> 2;
        const int rloc = q * 32 + lane;
        const int c0 = slice * kSlice;
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c0);
        uint8_t* box[2] = {staging + e * 2 * kBox, staging + e * 2 * kBox + kBox};
        uint64_t* rbar = res_bar + 2 * e;
        uint32_t rph = 0;  // phase bit of rbar[0] (bit 0) and rbar[1] (bit 1)
        uint32_t tphase = 0;
        int cstage = 0;  // AQ: the A stages this thread quantises, in the MMA's order
        uint32_t cphase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int row0 = tile * 128 + q * 32;
            if constexpr (C::BOXES) {
                // residual boxes of chunks 0 and 1 (the boxes' previous TMA stores must have read them)
                if (lane == 0) {
                    tzp::bulk_wait_read<0>();
                    for (int b = 0; b < 2; ++b) {
                        tzp::mbar_arrive_expect_tx(&rbar[b], kBox);
                        tzp::bulk_load_1d(box[b], p.residual + xblk(row0, c0 + 16 * b), kBox, &rbar[b]);
                    }
                }
                __syncwarp();
            } else {
                // this warp's residual slice (32 rows x 96 columns, 12 KB contiguous) into L2 during the mainloop
                if (lane == 0) tzp::bulk_prefetch_l2(p.residual + xblk(row0, c0), 32 * kSlice * 4);
            }
            if constexpr (AQ) {
                // ---- quantise this tile's A rows into the int8 stages ----
                // Thread t: row t / 4 of the tile, 32 columns (64 bytes of f16) at (t % 4) * 32 of
                // each 128-column K block; writes two 16-byte chunks of the SWIZZLE_128B row
                // (chunk c of row r at c ^ (r % 8)).  The next K block's loads are in flight while
                // this one is converted.
                const int t = threadIdx.x - 64;
                const int crow = t >> 2, qq = t & 3;
                const int grow = tile * 128 + crow;
                const bool cok = grow < M;
                float inv = 1.0f;
                if (cok) {
                    const float mx = __uint_as_float(p.a_absmax[grow]);
                    const float sc = (mx == 0.0f) ? 1.0f : __fdiv_rn(mx, 127.0f);
                    inv = __fdiv_rn(1.0f, sc);
                }
                const uint64_t inv2 = tzp::f2_pack(inv, inv);  // rows carry their own |max|: quant2_own_max applies
                const uint4* src = reinterpret_cast<const uint4*>(p.a16 + static_cast<long long>(cok ? grow : 0) * p.lda16 + qq * 32);
                uint4 x[4], x1[4];  // K blocks kb and kb + 1 in flight
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    x[i] = cok ? __ldcs(src + i) : make_uint4(0, 0, 0, 0);
                    x1[i] = (cok && kblocks > 1) ? __ldcs(src + 16 + i) : make_uint4(0, 0, 0, 0);
                }
                bool cbad = false;
                for (int kb = 0; kb < kblocks; ++kb) {
                    uint4 nx[4];
                    if (kb + 2 < kblocks) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) nx[i] = cok ? __ldcs(src + (kb + 2) * 16 + i) : make_uint4(0, 0, 0, 0);
                    }
                    int got = 1;
                    if (lane == 0) got = tzp::mbar_wait(&empty[cstage], cphase ^ 1u, status, abort_flag) ? 1 : 0;
                    got = __shfl_sync(0xffffffffu, got, 0);
                    if (!got) {
                        cbad = true;
                        break;
                    }
                    uint32_t w[8];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const __half2* hp = reinterpret_cast<const __half2*>(&x[i]);
#pragma unroll
                        for (int j = 0; j < 2; ++j) {
                            const float2 f0 = __half22float2(hp[2 * j]);
                            const float2 f1 = __half22float2(hp[2 * j + 1]);
                            w[2 * i + j] = __byte_perm(quant2_own_max(f0.x, f0.y, inv2), quant2_own_max(f1.x, f1.y, inv2), 0x5410);
                        }
                    }
                    if (p.dbg_aq != nullptr && cok) {  // parity capture: this thread's 32 quantised columns
                        uint4* d = reinterpret_cast<uint4*>(p.dbg_aq + static_cast<long long>(grow) * K + kb * 128 + qq * 32);
                        d[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        d[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    }
                    const uint32_t rowa = tzp::smem_u32(smem + cstage * C::STAGE_BYTES) + static_cast<uint32_t>(crow * 128);
                    tzp::st_shared_v4(rowa + (static_cast<uint32_t>((2 * qq) ^ (crow & 7)) << 4), w[0], w[1], w[2], w[3]);
                    tzp::st_shared_v4(rowa + (static_cast<uint32_t>((2 * qq + 1) ^ (crow & 7)) << 4), w[4], w[5], w[6], w[7]);
                    tzp::fence_proxy_async();
                    tzp::mbar_arrive(&afull[cstage]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        x[i] = x1[i];
                        x1[i] = nx[i];
                    }
                    if (++cstage == kStages) {
                        cstage = 0;
                        cphase ^= 1u;
                    }
                }
                if (cbad) break;
            }
            if (!tzp::mbar_wait(tfull, tphase, status, abort_flag)) break;
            tzp::tc_fence_after();
            const int row = tile * 128 + rloc;
            const bool ok = row < M;
            float rs = (p.row_scale && ok) ? p.row_scale[row] : 1.0f;
            if constexpr (AQ) {
                if (ok) {
                    const float mx = __uint_as_float(p.a_absmax[row]);
                    rs = (mx == 0.0f) ? 1.0f : __fdiv_rn(mx, 127.0f);
                    if (p.dbg_as != nullptr && slice == 0) p.dbg_as[row] = rs;
                }
            }

            // ---- pass A: x = dequant(acc) + bias + residual -> TMEM; row sum ----
            if (p.dbg_acc != nullptr) {  // parity capture: the raw accumulators, before pass A rewrites TMEM
#pragma unroll 1
                for (int c = 0; c < kSlice / 16; ++c) {
                    uint32_t r[16];
                    tzp::tmem_ld16(tbase + 16 * c, r);
                    tzp::tmem_ld_wait();
                    if (ok) {
                        int4* d = reinterpret_cast<int4*>(p.dbg_acc + static_cast<long long>(row) * kN + c0 + 16 * c);
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            d[j] = make_int4(static_cast<int>(r[4 * j]), static_cast<int>(r[4 * j + 1]),
                                             static_cast<int>(r[4 * j + 2]), static_cast<int>(r[4 * j + 3]));
                    }
                }
            }
            const uint64_t rs2 = tzp::f2_pack(rs, rs);
            uint64_t sum2 = 0;  // (even columns, odd columns)
            bool bad = false;
            const float* resw = p.residual + xblk(row0, c0) + lane * 4;  // !BOXES: quad 0 of chunk 0, this row
#pragma unroll
            for (int c = 0; c < kSlice / 16; ++c) {
                const int b = c & 1;
                uint32_t r[16];
                tzp::tmem_ld16(tbase + 16 * c, r);
                float4 cur[4];  // this row's 16 residual values
                if constexpr (C::BOXES) {
                    if (!tzp::mbar_wait(&rbar[b], (rph >> b) & 1u, status, nullptr)) {
                        tzp::tmem_ld_wait();
                        bad = true;
                        break;
                    }
                    rph ^= 1u << b;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        cur[j] = *reinterpret_cast<const float4*>(box[b] + j * 512 + lane * 16);  // quad j, this row
                    __syncwarp();
                    if (lane == 0 && c + 2 < kSlice / 16) {  // refill this box with chunk c + 2
                        tzp::mbar_arrive_expect_tx(&rbar[b], kBox);
                        tzp::bulk_load_1d(box[b], p.residual + xblk(row0, c0 + 16 * (c + 2)), kBox, &rbar[b]);
                    }
                } else {
                    // quad j of the blocked chunk, lane = row: each quad one coalesced 512-byte load
#pragma unroll
                    for (int j = 0; j < 4; ++j) cur[j] = *reinterpret_cast<const float4*>(resw + c * 512 + j * 128);
                }
                tzp::tmem_ld_wait();
                const int col = c0 + 16 * c;
#pragma unroll
                for (int j = 0; j < 8; ++j) {  // column pairs on packed f32x2 arithmetic
                    uint64_t x = tzp::f2_pack(acc_to_f<KIND>(r[2 * j]), acc_to_f<KIND>(r[2 * j + 1]));
                    const uint64_t cs2 = *reinterpret_cast<const uint64_t*>(sv_cs + col + 2 * j);
                    if (AQ || p.row_scale)
                        x = tzp::f2_mul(x, tzp::f2_mul(rs2, cs2));
                    else if (p.col_scale)
                        x = tzp::f2_mul(x, cs2);
                    const uint64_t b2 = *reinterpret_cast<const uint64_t*>(sv_bias + col + 2 * j);
                    const uint64_t res2 = reinterpret_cast<const uint64_t*>(cur)[j];
                    x = tzp::f2_add(tzp::f2_add(x, b2), res2);
                    sum2 = tzp::f2_add(sum2, x);
                    const float2 v = tzp::f2_unpack(x);
                    r[2 * j] = __float_as_uint(v.x);
                    r[2 * j + 1] = __float_as_uint(v.y);
                }
                tzp::tmem_st16(tbase + 16 * c, r);
            }
            if (bad) break;
            tzp::tmem_st_wait();
            {
                const float2 sp = tzp::f2_unpack(sum2);
                red_sum[slice * 128 + rloc] = sp.x + sp.y;
            }
            if (!epi_sync(&red_bar[0], tphase, lane, status)) break;
            const float mean =
                ((red_sum[rloc] + red_sum[128 + rloc]) + (red_sum[256 + rloc] + red_sum[384 + rloc])) / static_cast<float>(kN);

            // ---- pass B: sum of squared deviations ----
            const uint64_t mean2 = tzp::f2_pack(mean, mean);
            uint64_t ssq2 = 0;
#pragma unroll
            for (int c = 0; c < kSlice / 16; ++c) {
                uint32_t r[16];
                tzp::tmem_ld16(tbase + 16 * c, r);
                tzp::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint64_t d = tzp::f2_sub(tzp::f2_pack(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), mean2);
                    ssq2 = tzp::f2_fma(d, d, ssq2);
                }
            }
            {
                const float2 sp = tzp::f2_unpack(ssq2);
                red_ssq[slice * 128 + rloc] = sp.x + sp.y;
            }
            if (!epi_sync(&red_bar[1], tphase, lane, status)) break;
            const float var =
                ((red_ssq[rloc] + red_ssq[128 + rloc]) + (red_ssq[256 + rloc] + red_ssq[384 + rloc])) / static_cast<float>(kN);
            const float inv_std = 1.0f / sqrtf(var + p.eps);
            const uint64_t istd2 = tzp::f2_pack(inv_std, inv_std);

            // ---- pass C: normalise, store x_out (+ f16 aux, or y -> TMEM and |max|) ----
            float amax = 0.f;
#pragma unroll
            for (int c = 0; c < kSlice / 16; ++c) {
                uint32_t r[16];
                tzp::tmem_ld16(tbase + 16 * c, r);
                tzp::tmem_ld_wait();
                const int col = c0 + 16 * c;
                float y[16];
#pragma unroll
                for (int j = 0; j < 8; ++j) {  // y = (x - mean) * inv_std * gamma + beta on column pairs
                    const uint64_t x = tzp::f2_pack(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                    const uint64_t g2 = *reinterpret_cast<const uint64_t*>(sv_g + col + 2 * j);
                    const uint64_t b2 = *reinterpret_cast<const uint64_t*>(sv_b + col + 2 * j);
                    const float2 v = tzp::f2_unpack(tzp::f2_fma(tzp::f2_mul(tzp::f2_sub(x, mean2), istd2), g2, b2));
                    y[2 * j] = v.x;
                    y[2 * j + 1] = v.y;
                }
                {  // x_out: four coalesced 512-byte stores (blocked layout; padding rows of the last tile too)
                    float* xq = p.x_out + xblk(row0, col) + lane * 4;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<float4*>(xq + j * 128) = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
                }
                if constexpr (AUX == 0 || AUX == 2) {
                    constexpr bool kBf = AUX == 2;
                    if (ok) {
                        uint16_t* a = static_cast<uint16_t*>(p.aux) + static_cast<long long>(row) * kN + col;
                        *reinterpret_cast<uint4*>(a) = make_uint4(tzp::pack16x2<kBf>(y[0], y[1]), tzp::pack16x2<kBf>(y[2], y[3]),
                                                                  tzp::pack16x2<kBf>(y[4], y[5]), tzp::pack16x2<kBf>(y[6], y[7]));
                        *reinterpret_cast<uint4*>(a + 8) = make_uint4(tzp::pack16x2<kBf>(y[8], y[9]), tzp::pack16x2<kBf>(y[10], y[11]),
                                                                      tzp::pack16x2<kBf>(y[12], y[13]), tzp::pack16x2<kBf>(y[14], y[15]));
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        amax = fmaxf(amax, fabsf(y[j]));
                        r[j] = __float_as_uint(y[j]);
                    }
                    tzp::tmem_st16(tbase + 16 * c, r);
                }
            }
            if constexpr (AUX == 1) {
                // ---- pass D: per-token int8 quantisation of the LayerNorm output ----
                tzp::tmem_st_wait();
                red_max[slice * 128 + rloc] = amax;
                if (!epi_sync(&red_bar[2], tphase, lane, status)) break;
                const float m = fmaxf(fmaxf(red_max[rloc], red_max[128 + rloc]), fmaxf(red_max[256 + rloc], red_max[384 + rloc]));
                const float sc = (m == 0.0f) ? 1.0f : __fdiv_rn(m, 127.0f);
                const float inv = __fdiv_rn(1.0f, sc);
                const uint64_t inv2 = tzp::f2_pack(inv, inv);
                // this warp's 32 x 96 int8 block, row-major (96-byte rows) in its staging boxes once the
                // x_out stores have read them, then one TMA store
                if (lane == 0) tzp::bulk_wait_read<0>();
                __syncwarp();
                uint8_t* qrow = box[0] + lane * kSlice;
#pragma unroll
                for (int c = 0; c < kSlice / 16; ++c) {
                    uint32_t r[16];
                    tzp::tmem_ld16(tbase + 16 * c, r);
                    tzp::tmem_ld_wait();
                    uint32_t w[4];  // rows quantised against their own |max|: the packed form applies
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        w[j] = __byte_perm(quant2_own_max(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), inv2),
                                           quant2_own_max(__uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]), inv2), 0x5410);
                    *reinterpret_cast<uint4*>(qrow + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
                }
                tzp::fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    tzp::tma_store_2d(&tmAux, box[0], c0, row0);
                    tzp::bulk_commit();
                }
                if (ok && slice == 0) p.aux_scale[row] = sc;
            }
            if constexpr (AQ) {
                if (ok && slice == 0) p.a_absmax[row] = 0u;  // every reader of this row's |max| is done
            }
            tzp::tc_fence_before();
            __syncwarp();
            if (lane == 0) tzp::mbar_arrive(tempty);
            tphase ^= 1u;
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

CUtensorMapDataType dtype_of(int kind) {
    return kind == KIND_I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                           : kind == KIND_TF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                               : kind == KIND_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

template <int KIND, int AUX, int AQ = 0>
int launch_ln_impl(tz_ctx_t ctx, const GemmLnArgs& g, cudaStream_t s) {
    using C = LnCfg<KIND, AQ>;
    static_assert(AUX != 1 || C::BOXES, "the int8 output is staged in the residual boxes");
    auto kern = gemm_ln_kernel<KIND, AUX, AQ>;
    static unsigned attr_set = 0;
    int dev = 0;
    TZ_CUDA(cudaGetDevice(&dev));
    if (!(attr_set & (1u << (dev & 31)))) {
        TZ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_set |= 1u << (dev & 31);
    }
    CUtensorMap ta, tb;
    int rc = TZ_OK;
    if (!AQ) {
        rc = encode_tmap_2d(&ta, dtype_of(KIND), C::ELEM, g.a, static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.M),
                            static_cast<uint64_t>(g.lda) * C::ELEM, C::BK, 128);
        if (rc) return rc;
    }
    rc = encode_tmap_2d(&tb, dtype_of(KIND), C::ELEM, g.b, static_cast<uint64_t>(g.K), kN,
                        static_cast<uint64_t>(g.ldb) * C::ELEM, C::BK, kHalf);
    if (rc) return rc;
    CUtensorMap tq = tb;  // AUX = 1: the int8 LayerNorm output [M, 384], one 96 x 32 box per epilogue warp
    if (AUX == 1) {
        rc = encode_tmap_2d_swz(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.aux, kN, static_cast<uint64_t>(g.M), kN, kSlice, 32,
                                CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    if (AQ) ta = tb;  // unused: A arrives through the epilogue warps
    LnParams p{g.bias, g.col_scale, g.row_scale, g.residual, g.gamma, g.beta, g.eps, g.x_out, g.aux, g.aux_scale,
               AQ ? static_cast<const __half*>(g.a) : nullptr, g.lda, g.a_absmax, g.dbg_acc, g.dbg_aq, g.dbg_as};
    const int tiles = (g.M + 127) / 128;
    const int sms = ctx->sm_count - ctx->sm_reserve;
    const int grid = tiles < sms ? tiles : sms;
    if (grid <= 0) return TZ_OK;
    return launch_kernel(kern, dim3(grid), dim3(kThreads), C::SMEM, s, g.pdl, ta, tb, tq, g.M, g.K, p, ctx->d_status);
}

}  // namespace

int launch_gemm_ln(tz_ctx_t ctx, const GemmLnArgs& g, cudaStream_t s) {
    TZ_CHECK(g.M >= 0 && g.K > 0, TZ_EINVAL, "gemm_ln: bad shape");
    if (g.M == 0) return TZ_OK;
    TZ_CHECK(g.a && g.b && g.bias && g.residual && g.gamma && g.beta && g.x_out && g.aux, TZ_EINVAL, "gemm_ln: null operand");
    TZ_CHECK(!g.row_scale || g.col_scale, TZ_EINVAL, "gemm_ln: row_scale needs col_scale");
    TZ_CHECK(g.aux_int8 == (g.aux_scale != nullptr), TZ_EINVAL, "gemm_ln: int8 aux needs its scale vector");
    TZ_CHECK(reinterpret_cast<uintptr_t>(g.residual) % 16 == 0 && reinterpret_cast<uintptr_t>(g.x_out) % 16 == 0, TZ_EINVAL,
             "gemm_ln: the blocked residual stream must be 16-byte aligned");
    TZ_CHECK(reinterpret_cast<uintptr_t>(g.dbg_acc) % 16 == 0 && reinterpret_cast<uintptr_t>(g.dbg_aq) % 16 == 0 &&
                 (!g.dbg_aq || g.a_absmax),
             TZ_EINVAL, "gemm_ln: capture buffers must be 16-byte aligned; A capture needs in-kernel quantisation");
    if (g.a_absmax) {
        TZ_CHECK(g.kind == KIND_I8 && g.aux_int8 && !g.row_scale && g.col_scale, TZ_EINVAL,
                 "gemm_ln: in-kernel A quantisation needs the int8 kind, int8 aux, column scales and no row scales");
        TZ_CHECK(g.K % 128 == 0 && g.lda % 8 == 0 && reinterpret_cast<uintptr_t>(g.a) % 16 == 0, TZ_EINVAL,
                 "gemm_ln: in-kernel A quantisation needs K %% 128 == 0 and 16-byte aligned f16 rows (K=%d)", g.K);
        return launch_ln_impl<KIND_I8, 1, 1>(ctx, g, s);
    }
    TZ_CHECK(!g.aux_int8, TZ_EUNSUPPORTED, "gemm_ln: the int8 LayerNorm output needs the in-kernel A quantisation");
    TZ_CHECK(g.aux_bf16 == (g.kind == KIND_BF16), TZ_EUNSUPPORTED, "gemm_ln: a bf16 aux goes with bf16 operands");
    if (g.kind == KIND_I8) return launch_ln_impl<KIND_I8, 0>(ctx, g, s);
    if (g.kind == KIND_F16) return launch_ln_impl<KIND_F16, 0>(ctx, g, s);
    if (g.kind == KIND_BF16) return launch_ln_impl<KIND_BF16, 2>(ctx, g, s);
    return fail(TZ_EUNSUPPORTED, "gemm_ln: kind %d", g.kind);
}

}  // namespace tz
