// tz_gemm.cu -- persistent warp-specialised tcgen05 GEMM for sm_100a with fused epilogues.
//
//   Y[M, N] = epilogue( A[M, K] * B[N, K]^T )        (both operands K-major, PyTorch [out,in] B)
//
// One CTA per SM (persistent, static round-robin over 128 x BN output tiles, tile index n-fastest
// so neighbouring CTAs share A rows in L2).  64 + 32*EPI_WARPS threads:
//   warp 0      TMA producer: 128-byte-wide K blocks of A (128 rows) and B (BN rows) into a
//               STAGES-deep shared-memory ring, SWIZZLE_128B, completion on `full[s]`;
//   warp 1      allocates TMEM (2 x BN fp32/int32 columns: double-buffered accumulators); lane 0
//               issues tcgen05.mma (M=128, N=BN, 32 bytes of K per instruction) and commits to
//               `empty[s]` (smem slot free) and `tfull[acc]` (accumulator ready);
//   warps 2..   epilogue: warp w reads TMEM lane quarter (w % 4) and one column slice, so each
//               thread owns one output row of that slice; 32 columns per tcgen05.ld; scale / bias /
//               GELU / residual / row-absmax fused in registers; each 32x32 chunk is staged in
//               swizzled shared memory and written by one TMA bulk-tensor store (double-buffered).
// The epilogue of tile t overlaps the MMAs of tile t+1 (second TMEM buffer).
//
// Replaces matmulTransposeB (reference matmul.zig:54-77), linearProjection (arctic.zig:599-635),
// matmulTransposeB_f32_i8_rowScale_bias (matmul_w8a32.zig:14-58) and FusedMatmulEpilogueKernel
// (codegen.zig:78-147).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tz_internal.h"
#include "tz_ptx.cuh"
#include "tz_rowops.cuh"

namespace tz {
namespace {

struct EpiParams {
    const float* bias;
    const float* col_scale;
    const float* row_scale;
    const float* residual;
    long long ldr;
    void* out;
    long long ldo;
    int out_type;
    int gelu;
    unsigned* row_absmax;
    int n_ops;
    uint64_t ops;  // op o in bits [5o, 5o+5) (packed: no dynamic indexing of kernel parameters)
    int vec_ok;  // 16-byte aligned rows for vector stores / residual loads
    int32_t* dbg_acc;  // parity capture: raw accumulators [M, N] (specialised epilogue), or null
};

// The fusion GELU (simd.zig:168-178: tanh(z) = 2 sigmoid(2z) - 1) for the fixed epilogue of the f32 /
// tf32 GEMMs: tanh(z) = 1 - 2 / (1 + exp(2z)) with the fast exponential (ex2.approx on a pre-scaled
// argument) and the approximate reciprocal (no slow path: an infinite or huge denominator gives 0,
// so tanh -> 1; exp underflowing to 0 gives -1).  A few 1e-7 relative from the expf /
// IEEE-division form, far inside the tf32 GEMM's own rounding.
__device__ __forceinline__ float gelu_sigmoid_fast(float x) {
    const float inner = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
    const float t = fmaf(-2.0f, __fdividef(1.0f, 1.0f + __expf(2.0f * inner)), 1.0f);
    const float hx = 0.5f * x;
    return fmaf(hx, t, hx);
}

// Unary op table of codegen.zig:228-244 (simd.zig scalar ops) for the generic epilogue chain: the
// shared table of the row kernels (tz_rowops.cuh).
__device__ __forceinline__ float apply_op(int op, float x) { return unary_op(op, x); }

template <int KIND>
struct KindTraits;
template <>
struct KindTraits<KIND_F16> {
    static constexpr int elem = 2;
    static constexpr uint32_t c_fmt = 1, ab_fmt = 0;
};
template <>
struct KindTraits<KIND_BF16> {
    static constexpr int elem = 2;
    static constexpr uint32_t c_fmt = 1, ab_fmt = 1;
};
template <>
struct KindTraits<KIND_TF32> {
    static constexpr int elem = 4;
    static constexpr uint32_t c_fmt = 1, ab_fmt = 2;
};
template <>
struct KindTraits<KIND_I8> {
    static constexpr int elem = 1;
    static constexpr uint32_t c_fmt = 2, ab_fmt = 1;
};

constexpr int CW = 16;  // epilogue chunk width (columns per tcgen05.ld / per TMA store box)

template <int KIND, int BN, int STAGES, int EPI_WARPS>
struct Cfg {
    static constexpr int BM = 128;
    static constexpr int ELEM = KindTraits<KIND>::elem;
    static constexpr int BK = 128 / ELEM;  // elements per 128-byte K block
    static constexpr int A_BYTES = BM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
    static constexpr int EPI_BUF = 32 * CW * 4;              // 32 rows x 16 columns x 4 bytes: one store box
    static constexpr int STAGING = EPI_WARPS * 2 * EPI_BUF;  // double-buffered per epilogue warp
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = STAGES * STAGE_BYTES + STAGING + BAR_BYTES + 1024;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int SLICES = EPI_WARPS / 4;             // warps sharing one TMEM lane quarter
    static constexpr int COLS_PER_WARP = BN / SLICES;
    // The specialised epilogue: two sets of a warp's f16 output boxes (tile t's stores drain while
    // tile t+1 is staged) + its column vectors.
    // (rounded to 256 bytes: every box starts on a whole 32-byte-swizzle atom)
    static constexpr int FAST_WARP_BYTES = (2 * (COLS_PER_WARP / CW) * (32 * CW * 2) + 2 * COLS_PER_WARP * 4 + 255) / 256 * 256;
    static constexpr int FAST_STAGING = EPI_WARPS * FAST_WARP_BYTES;
    static constexpr int SMEM_FAST = STAGES * STAGE_BYTES + FAST_STAGING + BAR_BYTES + 1024;
    static_assert(2 * BN <= 512, "two accumulators must fit in TMEM");
    static_assert(EPI_WARPS % 4 == 0 && COLS_PER_WARP % CW == 0, "epilogue split");
    static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "BN");
    static_assert((2 * STAGES + 5) * 8 + 8 <= BAR_BYTES, "barrier area");
    static_assert(SMEM <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ float gelu_fast(float x) {
    // arctic.zig:750-756 formula with the hardware tanh
    const float inner = 0.7978845608f * (x + 0.044715f * x * x * x);
    const float hx = 0.5f * x;
    return fmaf(hx, tzp::tanh_approx(inner), hx);
}

// Epilogue math for one CW-column chunk of one row (v[] in and out, fp32).
template <int KIND>
__device__ __forceinline__ void epilogue_math(const EpiParams& ep, float (&v)[CW], int row, bool row_ok, int col0,
                                              int N, float rs) {
    const bool full = (col0 + CW <= N);
    if (ep.n_ops >= 0) {
        // Generic chain (codegen.zig:101-145): TZ_OP_ADD adds bias[col], others are unary.
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            const int col = col0 + j;
            float x = v[j];
            if (col < N) {
                for (int o = 0; o < ep.n_ops; ++o) {
                    const int op = static_cast<int>((ep.ops >> (5 * o)) & 31u);
                    if (op == TZ_OP_ADD) {
                        if (ep.bias) x = x + __ldg(ep.bias + col);
                    } else {
                        x = apply_op(op, x);
                    }
                }
            }
            v[j] = x;
        }
        return;
    }
    if (full) {
        float4 res[CW / 4];
        if (ep.residual && row_ok) {  // issue the residual loads first: their latency overlaps the math
            const float* rp = ep.residual + static_cast<long long>(row) * ep.ldr + col0;
            if (ep.vec_ok) {
#pragma unroll
                for (int j = 0; j < CW / 4; ++j) res[j] = *reinterpret_cast<const float4*>(rp + 4 * j);
            } else {
#pragma unroll
                for (int j = 0; j < CW / 4; ++j) res[j] = make_float4(rp[4 * j], rp[4 * j + 1], rp[4 * j + 2], rp[4 * j + 3]);
            }
        }
#pragma unroll
        for (int j = 0; j < CW; j += 4) {
            const int col = col0 + j;
            if (ep.row_scale) {
                const float4 cs = __ldg(reinterpret_cast<const float4*>(ep.col_scale + col));
                v[j] = __fmul_rn(v[j], __fmul_rn(rs, cs.x));
                v[j + 1] = __fmul_rn(v[j + 1], __fmul_rn(rs, cs.y));
                v[j + 2] = __fmul_rn(v[j + 2], __fmul_rn(rs, cs.z));
                v[j + 3] = __fmul_rn(v[j + 3], __fmul_rn(rs, cs.w));
            } else if (ep.col_scale) {
                const float4 cs = __ldg(reinterpret_cast<const float4*>(ep.col_scale + col));
                v[j] = __fmul_rn(v[j], cs.x);
                v[j + 1] = __fmul_rn(v[j + 1], cs.y);
                v[j + 2] = __fmul_rn(v[j + 2], cs.z);
                v[j + 3] = __fmul_rn(v[j + 3], cs.w);
            }
            if (ep.bias) {
                const float4 b = __ldg(reinterpret_cast<const float4*>(ep.bias + col));
                v[j] = __fadd_rn(v[j], b.x);
                v[j + 1] = __fadd_rn(v[j + 1], b.y);
                v[j + 2] = __fadd_rn(v[j + 2], b.z);
                v[j + 3] = __fadd_rn(v[j + 3], b.w);
            }
        }
        if (ep.gelu == 1) {
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = gelu_fast(v[j]);
        } else if (ep.gelu == 2) {
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = gelu_sigmoid_fast(v[j]);
        } else if (ep.gelu == 3) {
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = v[j] > 0.0f ? v[j] : 0.0f;
        }
        if (ep.residual && row_ok) {
#pragma unroll
            for (int j = 0; j < CW / 4; ++j) {
                v[4 * j] = __fadd_rn(v[4 * j], res[j].x);
                v[4 * j + 1] = __fadd_rn(v[4 * j + 1], res[j].y);
                v[4 * j + 2] = __fadd_rn(v[4 * j + 2], res[j].z);
                v[4 * j + 3] = __fadd_rn(v[4 * j + 3], res[j].w);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            const int col = col0 + j;
            float x = v[j];
            if (col < N) {
                if (ep.row_scale)
                    x = __fmul_rn(x, __fmul_rn(rs, ep.col_scale[col]));
                else if (ep.col_scale)
                    x = __fmul_rn(x, ep.col_scale[col]);
                if (ep.bias) x = __fadd_rn(x, ep.bias[col]);
                if (ep.gelu == 1) x = gelu_fast(x);
                else if (ep.gelu == 2) x = gelu_sigmoid_fast(x);
                else if (ep.gelu == 3) x = x > 0.0f ? x : 0.0f;
                if (ep.residual && row_ok) x = __fadd_rn(x, ep.residual[static_cast<long long>(row) * ep.ldr + col]);
            }
            v[j] = x;
        }
    }
}

// Direct (non-TMA) stores of one chunk: used when the output is not 16-byte aligned per row.
__device__ __forceinline__ void store_direct(const EpiParams& ep, const float (&v)[CW], const uint32_t (&r)[CW], int row,
                                             int col0, int N, float& amax) {
#pragma unroll
    for (int j = 0; j < CW; ++j) {
        const int col = col0 + j;
        if (col < N) {
            const long long o = static_cast<long long>(row) * ep.ldo + col;
            if (ep.out_type == OUT_I32) {
                reinterpret_cast<int*>(ep.out)[o] = static_cast<int>(r[j]);
            } else if (ep.out_type == OUT_F16) {
                const __half h = __float2half_rn(v[j]);
                reinterpret_cast<__half*>(ep.out)[o] = h;
                amax = fmaxf(amax, fabsf(__half2float(h)));
            } else {
                reinterpret_cast<float*>(ep.out)[o] = v[j];
                amax = fmaxf(amax, fabsf(v[j]));
            }
        }
    }
}

// Swizzled staging of one 32 x 16 chunk for a TMA store (thread = row).  32-bit outputs: 64-byte
// rows, SWIZZLE_64B (16-byte unit c of row r at c ^ ((r >> 1) & 3)); f16 outputs: 32-byte rows,
// SWIZZLE_32B (unit c at c ^ ((r >> 2) & 1)).
__device__ __forceinline__ void stage_chunk(const EpiParams& ep, uint32_t buf, int lane, const float (&v)[CW],
                                            const uint32_t (&r)[CW], float& amax) {
    if (ep.out_type == OUT_F16) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const uint32_t a = buf + lane * 32 + ((c ^ ((lane >> 2) & 1)) << 4);
            tzp::st_shared_v4(a, tzp::pack_half2(v[8 * c], v[8 * c + 1]), tzp::pack_half2(v[8 * c + 2], v[8 * c + 3]),
                              tzp::pack_half2(v[8 * c + 4], v[8 * c + 5]), tzp::pack_half2(v[8 * c + 6], v[8 * c + 7]));
        }
        if (ep.row_absmax) {
#pragma unroll
            for (int j = 0; j < CW; ++j) amax = fmaxf(amax, fabsf(__half2float(__float2half_rn(v[j]))));
        }
    } else if (ep.out_type == OUT_I32) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t a = buf + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4);
            tzp::st_shared_v4(a, r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t a = buf + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4);
            tzp::st_shared_v4(a, __float_as_uint(v[4 * c]), __float_as_uint(v[4 * c + 1]), __float_as_uint(v[4 * c + 2]),
                              __float_as_uint(v[4 * c + 3]));
        }
        if (ep.row_absmax) {
#pragma unroll
            for (int j = 0; j < CW; ++j) amax = fmaxf(amax, fabsf(v[j]));
        }
    }
}

// Flags of the specialised epilogue (FAST & F_ON): f16 output through TMA, full column tiles, bias,
// no residual / op chain.  Everything else takes the general epilogue.
constexpr int F_ON = 1, F_GELU = 2, F_AMAX = 4, F_RSCALE = 8, F_CSCALE = 16;
// F_BMN (general epilogue, tf32 only): B arrives N-major, B[k, n] row-major as `A @ B` has it, and the
// MMA reads it through an MN-major descriptor: no transpose of B first.  Each stage's B tile is
// BN / 32 TMA boxes of 32 columns (128 bytes) x BK rows, BK * 128 bytes apart.  MN-major tf32
// operands take the 128-byte swizzle with 32-byte atoms (TMA's SWIZZLE_128B_ATOM_32B): 32-byte
// chunk c of 128-byte row r at c ^ (r % 4), 4-row K groups.
constexpr int F_BMN = 32;
// F_3X (general epilogue, tf32 only): the split-operand product of GemmArgs::a3x; the producer maps
// K block kb of the MMA's K = 3P onto A's [hi | lo] row as hi, hi, lo (P = K / 3).
constexpr int F_3X = 64;
// F_OBF (specialised epilogue): the 16-bit output is bf16 instead of IEEE half.
constexpr int F_OBF = 128;

// Shared-memory descriptor of such an MN-major tile: 128-byte rows along MN (32 tf32 elements),
// 4-row K groups 512 bytes apart (SBO), MN blocks of 32 elements `lbo` bytes apart (LBO), layout
// type SWIZZLE_128B_BASE32B (1).
__device__ __forceinline__ uint64_t sdesc_mn128_b32(uint32_t smem_addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(lbo >> 4) << 16;
    d |= static_cast<uint64_t>(512 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(1) << 61;
    return d;
}

template <int KIND, int BN, int STAGES, int EPI_WARPS, int FAST>
__global__ void __launch_bounds__(Cfg<KIND, BN, STAGES, EPI_WARPS>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmOut, int M, int N, int K, EpiParams ep, int use_tma_store,
                   int* status) {
    using C = Cfg<KIND, BN, STAGES, EPI_WARPS>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = tzp::smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* staging = smem + STAGES * C::STAGE_BYTES;
    constexpr bool kFastEpi = (FAST & F_ON) != 0;
    constexpr bool kBmn = (FAST & F_BMN) != 0;
    constexpr bool k3x = (FAST & F_3X) != 0;
    static_assert(!kBmn || (KIND == KIND_TF32 && !kFastEpi), "N-major B: tf32, general epilogue");
    static_assert(!k3x || (KIND == KIND_TF32 && !kFastEpi && !kBmn), "split tf32: tf32, general epilogue");
    static_assert((FAST & F_OBF) == 0 || (FAST & F_AMAX) == 0, "the row |max| is taken on IEEE-half outputs");
    const int part3 = K / 3;  // F_3X: elements of one part
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + (kFastEpi ? C::FAST_STAGING : C::STAGING));
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tzp::mbar_init(&full[s], 1);
            tzp::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            tzp::mbar_init(&tfull[a], 1);
            tzp::mbar_init(&tempty[a], EPI_WARPS);
        }
        tzp::mbar_init(drain, 1);
        *abort_flag = 0;
        tzp::fence_mbar_init();
        tzp::tma_prefetch_desc(&tmA);
        tzp::tma_prefetch_desc(&tmB);
        if (use_tma_store) tzp::tma_prefetch_desc(&tmOut);
    }
    if (warp == 1) {
        tzp::tmem_alloc(tmem_slot, C::TMEM_COLS);
        tzp::tmem_relinquish();
    }
    tzp::tc_fence_before();
    __syncthreads();
    tzp::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Programmatic launch: each role waits for the previous grid (griddepcontrol.wait) before it
    // touches that grid's output; the producer first requests the B (weight) tiles of its first
    // stages, which the model's previous kernel never writes.

    const int n_tiles = (N + BN - 1) / BN;
    const int m_tiles = (M + 127) / 128;
    const int num_tiles = m_tiles * n_tiles;
    const int kblocks = (K + C::BK - 1) / C::BK;
    // Tile schedule.  When the K blocks of a tile fill the stage ring exactly (kblocks == STAGES:
    // stage = K block for every tile) and there are at least as many CTAs as column blocks, each CTA
    // keeps one column block and walks row blocks: its weight (B) tiles are loaded once and stay in
    // the stages' B regions, and only A streams through the TMA path.  Otherwise tiles are dealt
    // round-robin over the linear (row block, column block) order.
    const bool fixed_n = kblocks == STAGES && n_tiles > 1 && static_cast<int>(gridDim.x) >= n_tiles;
    const int my_n = static_cast<int>(blockIdx.x) % n_tiles, my_r = static_cast<int>(blockIdx.x) / n_tiles;
    const int my_cn = (static_cast<int>(gridDim.x) - 1 - my_n) / n_tiles + 1;  // CTAs sharing my_n
    auto tile_of = [&](int i, int& m0, int& n0) -> bool {  // this CTA's i-th tile
        if (fixed_n) {
            const int m = my_r + i * my_cn;
            m0 = m * 128;
            n0 = my_n * BN;
            return m < m_tiles;
        }
        const int t = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
        m0 = (t / n_tiles) * 128;
        n0 = (t % n_tiles) * BN;
        return t < num_tiles;
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ----
            int pre = 0;  // K blocks of the first tile whose B tile is already requested
            int fm0 = 0, fn0 = 0;
            if (tile_of(0, fm0, fn0)) {
                pre = kblocks < STAGES ? kblocks : STAGES;
                for (int kb = 0; kb < pre; ++kb) {
                    tzp::mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
                    uint8_t* sb = smem + kb * C::STAGE_BYTES + C::A_BYTES;
                    const int nb = fn0;
                    if constexpr (kBmn) {
#pragma unroll
                        for (int j = 0; j < BN / 32; ++j) tzp::tma_load_2d(sb + j * C::BK * 128, &tmB, nb + 32 * j, kb * C::BK, &full[kb]);
                    } else {
                        tzp::tma_load_2d(sb, &tmB, kb * C::BK, nb, &full[kb]);
                    }
                }
            }
            tzp::pdl_wait();
            int stage = 0;
            uint32_t phase = 0, armed = 0, armed_par = 0;
            int m0 = 0, n0 = 0;
            for (int it = 0; tile_of(it, m0, n0); ++it) {
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tzp::mbar_wait(&empty[stage], phase ^ 1u, status, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + stage * C::STAGE_BYTES;
                    const bool armed_ab = it == 0 && kb < pre;  // armed for A + B before griddepcontrol.wait
                    const bool resident = fixed_n && it > 0;     // stage kb still holds this column block's B
                    const bool b_done = armed_ab || resident;
                    if (!armed_ab) tzp::mbar_arrive_expect_tx(&full[stage], resident ? C::A_BYTES : C::STAGE_BYTES);
                    int ax = kb * C::BK;
                    if constexpr (k3x) ax = ax < 2 * part3 ? ax % part3 : ax - part3;  // hi, hi, lo
                    tzp::tma_load_2d(sa, &tmA, ax, m0, &full[stage]);
                    if (!b_done) {
                        if constexpr (kBmn) {
#pragma unroll
                            for (int j = 0; j < BN / 32; ++j)
                                tzp::tma_load_2d(sa + C::A_BYTES + j * C::BK * 128, &tmB, n0 + 32 * j, kb * C::BK, &full[stage]);
                        } else {
                            tzp::tma_load_2d(sa + C::A_BYTES, &tmB, kb * C::BK, n0, &full[stage]);
                        }
                    }
                    armed |= 1u << stage;
                    armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
            }
            // Let every copy this thread issued land before the CTA can exit (bounded).
            for (int s = 0; s < STAGES; ++s)
                if (armed & (1u << s)) tzp::mbar_wait(&full[s], (armed_par >> s) & 1u, status, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            constexpr uint32_t idesc = tzp::make_idesc(KindTraits<KIND>::c_fmt, KindTraits<KIND>::ab_fmt, 128, BN) |
                                       (kBmn ? (1u << 16) : 0u);  // bit 16: B is MN-major
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            int m0 = 0, n0 = 0;
            for (int it = 0; tile_of(it, m0, n0); ++it) {
                if (!tzp::mbar_wait(&tempty[acc], acc_phase ^ 1u, status, abort_flag)) break;
                tzp::tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tzp::mbar_wait(&full[stage], phase, status, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tzp::tc_fence_after();
                    uint8_t* sa = smem + stage * C::STAGE_BYTES;
                    const uint64_t ad = tzp::sdesc_k128(tzp::smem_u32(sa));
                    const uint64_t bd = kBmn ? sdesc_mn128_b32(tzp::smem_u32(sa + C::A_BYTES), C::BK * 128)
                                             : tzp::sdesc_k128(tzp::smem_u32(sa + C::A_BYTES));
                    // 4 MMA K steps per 128-byte K block: A advances 32 bytes; B advances 32 bytes
                    // (K-major) or 8 rows, 1024 bytes (MN-major)
                    constexpr uint32_t kBstep = kBmn ? 1024u >> 4 : 2u;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        tzp::umma<KIND>(d, ad + 2u * k, bd + kBstep * k, idesc, (kb | k) != 0 ? 1u : 0u);
                    tzp::umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tzp::umma_commit(&tfull[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // Drain: every MMA this thread issued has completed before TMEM is released.
            tzp::umma_commit(drain);
            tzp::mbar_wait(drain, 0, status, nullptr);
        }
    } else if constexpr (kFastEpi) {
        tzp::pdl_wait();
        // ---- specialised epilogue: straight-line code per tile ----
        // Per tile, before the accumulator is ready: this row's scale and the slice's bias / column
        // scales (into this warp's staging area, read back as broadcasts).  Then the NCH chunks of
        // 16 columns: TMEM load of chunk c+1 in flight while chunk c is converted and staged; the
        // accumulator is released as soon as its last chunk is in registers; one proxy fence and NCH
        // TMA stores per tile, staged in one of two box sets so that they drain while the next tile
        // is staged (three operand stages leave room for the second set).  The arithmetic runs on packed f32x2 instructions (bit-identical to
        // the scalar forms) and |max| is taken on the packed f16 results.
        constexpr int CPW = C::COLS_PER_WARP;
        constexpr int NCH = CPW / CW;
        constexpr int BOX = 32 * CW * 2;  // one 32 x 16 f16 box
        const int e = warp - 2;
        const int q = warp & 3;
        const int slice = e >> 2;
        uint8_t* wst = staging + e * C::FAST_WARP_BYTES;  // [2 box sets][NCH boxes] + column vectors
        float* cvb = reinterpret_cast<float*>(wst + 2 * NCH * BOX);
        float* cvs = cvb + CPW;
        int pb = 0;  // box set of this tile
        const uint64_t kG0 = tzp::f2_pack(0.7978845608f, 0.7978845608f);
        const uint64_t kG1 = tzp::f2_pack(0.7978845608f * 0.044715f, 0.7978845608f * 0.044715f);
        const uint64_t kHalf = tzp::f2_pack(0.5f, 0.5f);
        int acc = 0;
        uint32_t acc_phase = 0;
        // The next tile's row scale and column vectors are fetched into registers while this tile
        // waits and is converted, so no tile starts on a global-memory round trip.
        constexpr int VPL = (CPW + 31) / 32;
        float nrs = 1.0f, nb[VPL], ns[VPL];
        auto fetch = [&](int i) {  // the CTA's i-th tile
            int fm0 = 0, fn0 = 0;
            if (!tile_of(i, fm0, fn0)) return;
            const int r = fm0 + q * 32 + lane;
            const int cb = fn0 + slice * CPW;
            if constexpr ((FAST & F_RSCALE) != 0) nrs = r < M ? __ldg(ep.row_scale + r) : 1.0f;
#pragma unroll
            for (int v = 0; v < VPL; ++v) {
                const int i = lane + 32 * v;
                if (i < CPW) {
                    nb[v] = __ldg(ep.bias + cb + i);
                    if constexpr ((FAST & (F_RSCALE | F_CSCALE)) != 0) ns[v] = __ldg(ep.col_scale + cb + i);
                }
            }
        };
        fetch(0);
        int m0 = 0, n0 = 0;
        for (int it = 0; tile_of(it, m0, n0); ++it) {
            const int row0 = m0 + q * 32;
            const int row = row0 + lane;
            const bool row_ok = row < M;
            const int cbase = n0 + slice * CPW;
            const float rs = nrs;
            const uint64_t rs2 = tzp::f2_pack(rs, rs);
            if (lane == 0) tzp::bulk_wait_read<1>();  // the stores of two tiles ago have read this box set
            uint8_t* wbox = wst + pb * NCH * BOX;
            const uint32_t wst_a = tzp::smem_u32(wbox);
#pragma unroll
            for (int v = 0; v < VPL; ++v) {  // the previous tile's reads of cvb / cvs are behind this warp
                const int i = lane + 32 * v;
                if (i < CPW) {
                    cvb[i] = nb[v];
                    if constexpr ((FAST & (F_RSCALE | F_CSCALE)) != 0) cvs[i] = ns[v];
                }
            }
            __syncwarp();
            fetch(it + 1);
            if (!tzp::mbar_wait(&tfull[acc], acc_phase, status, abort_flag)) break;
            tzp::tc_fence_after();
            const uint32_t tcol = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN + slice * CPW);
            uint32_t ra[CW], rb[CW];
            tzp::tmem_ld16(tcol, ra);
            tzp::tmem_ld_wait();
            uint32_t amax2 = 0u;  // packed f16 pair; only the magnitudes are meaningful (xorsign max)
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                uint32_t(&cur)[CW] = (c & 1) ? rb : ra;
                uint32_t(&nxt)[CW] = (c & 1) ? ra : rb;
                if (c + 1 < NCH) {
                    tzp::tmem_ld16(tcol + 16 * (c + 1), nxt);
                } else {  // every TMEM load of this tile has completed: release the accumulator
                    tzp::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tzp::mbar_arrive(&tempty[acc]);
                }
                if (ep.dbg_acc != nullptr && row_ok) {  // parity capture: the raw accumulators of this chunk
                    int4* d = reinterpret_cast<int4*>(ep.dbg_acc + static_cast<long long>(row) * N + cbase + 16 * c);
#pragma unroll
                    for (int j = 0; j < CW / 4; ++j)
                        d[j] = make_int4(static_cast<int>(cur[4 * j]), static_cast<int>(cur[4 * j + 1]),
                                         static_cast<int>(cur[4 * j + 2]), static_cast<int>(cur[4 * j + 3]));
                }
                // dequantise (+ bias, GELU) two columns per packed f32x2 instruction; the f16 pairs
                // feed both the staging and the row |max| (max |f16| is exact on the packed halves)
                uint32_t h[CW / 2];
                uint64_t bv[CW / 2], sv[CW / 2];  // this chunk's bias / column-scale pairs, 16-byte loads
#pragma unroll
                for (int q2 = 0; q2 < CW / 4; ++q2) {
                    const ulonglong2 tb = *reinterpret_cast<const ulonglong2*>(cvb + 16 * c + 4 * q2);
                    bv[2 * q2] = tb.x;
                    bv[2 * q2 + 1] = tb.y;
                    if constexpr ((FAST & (F_RSCALE | F_CSCALE)) != 0) {
                        const ulonglong2 ts = *reinterpret_cast<const ulonglong2*>(cvs + 16 * c + 4 * q2);
                        sv[2 * q2] = ts.x;
                        sv[2 * q2 + 1] = ts.y;
                    }
                }
#pragma unroll
                for (int j = 0; j < CW / 2; ++j) {
                    float lo, hi;
                    if constexpr (KIND == KIND_I8) {
                        lo = __int2float_rn(static_cast<int>(cur[2 * j]));
                        hi = __int2float_rn(static_cast<int>(cur[2 * j + 1]));
                    } else {
                        lo = __uint_as_float(cur[2 * j]);
                        hi = __uint_as_float(cur[2 * j + 1]);
                    }
                    uint64_t x = tzp::f2_pack(lo, hi);
                    const uint64_t b2 = bv[j];
                    if constexpr ((FAST & F_RSCALE) != 0)
                        x = tzp::f2_mul(x, tzp::f2_mul(rs2, sv[j]));
                    else if constexpr ((FAST & F_CSCALE) != 0)
                        x = tzp::f2_mul(x, sv[j]);
                    x = tzp::f2_add(x, b2);
                    if constexpr ((FAST & F_GELU) != 0) {
                        // GELU (arctic.zig:750-756, hardware tanh): 0.5 x (1 + tanh(x (k0 + k1 x^2))) with
                        // k0 = sqrt(2/pi), k1 = 0.044715 k0
                        const uint64_t inner = tzp::f2_mul(x, tzp::f2_fma(tzp::f2_mul(x, x), kG1, kG0));
                        const float2 in = tzp::f2_unpack(inner);
                        const uint64_t th = tzp::f2_pack(tzp::tanh_approx(in.x), tzp::tanh_approx(in.y));
                        const uint64_t hx = tzp::f2_mul(x, kHalf);
                        x = tzp::f2_fma(hx, th, hx);
                    }
                    const float2 r = tzp::f2_unpack(x);
                    h[j] = tzp::pack16x2<(FAST & F_OBF) != 0>(r.x, r.y);
                    if constexpr ((FAST & F_AMAX) != 0)
                        amax2 = tzp::hmax2_xorsign_abs(amax2, h[j]);
                }
                const uint32_t buf = wst_a + static_cast<uint32_t>(c * BOX);
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const uint32_t a = buf + lane * 32 + ((u ^ ((lane >> 2) & 1)) << 4);
                    tzp::st_shared_v4(a, h[4 * u], h[4 * u + 1], h[4 * u + 2], h[4 * u + 3]);
                }
                if (c + 1 < NCH) tzp::tmem_ld_wait();
            }
            tzp::fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
#pragma unroll
                for (int c = 0; c < NCH; ++c) tzp::tma_store_2d(&tmOut, wbox + c * BOX, cbase + 16 * c, row0);
                tzp::bulk_commit();
            }
            pb ^= 1;
            if constexpr ((FAST & F_AMAX) != 0) {
                if (row_ok)
                    atomicMax(ep.row_absmax + row, __float_as_uint(fmaxf(fabsf(__low2float(*reinterpret_cast<const __half2*>(&amax2))),
                                                                         fabsf(__high2float(*reinterpret_cast<const __half2*>(&amax2))))));
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) tzp::bulk_wait_all();
    } else {
        tzp::pdl_wait();
        // ---- epilogue warps: warp e reads TMEM lane quarter (warp % 4), column slice e / 4 ----
        const int e = warp - 2;
        const int q = warp & 3;
        const int slice = e >> 2;
        const uint32_t bufs = tzp::smem_u32(staging) + static_cast<uint32_t>(e * 2 * C::EPI_BUF);
        int acc = 0, nbuf = 0;
        uint32_t acc_phase = 0;
        int m0 = 0, n0 = 0;
        for (int it = 0; tile_of(it, m0, n0); ++it) {
            if (!tzp::mbar_wait(&tfull[acc], acc_phase, status, abort_flag)) break;
            tzp::tc_fence_after();
            const int row0 = m0 + q * 32;
            const int row = row0 + lane;
            const bool row_ok = row < M;
            const float rs = (ep.row_scale && row_ok) ? ep.row_scale[row] : 1.0f;
            float amax = 0.0f;
#pragma unroll 1
            for (int c = slice * C::COLS_PER_WARP; c < (slice + 1) * C::COLS_PER_WARP; c += CW) {
                uint32_t r[CW];
                tzp::tmem_ld16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN + c), r);
                tzp::tmem_ld_wait();
                const int col0 = n0 + c;
                if (col0 >= N) continue;  // warp-uniform
                float v[CW];
#pragma unroll
                for (int j = 0; j < CW; ++j) {
                    if constexpr (KIND == KIND_I8)
                        v[j] = __int2float_rn(static_cast<int>(r[j]));
                    else
                        v[j] = __uint_as_float(r[j]);
                }
                if (ep.out_type != OUT_I32) epilogue_math<KIND>(ep, v, row, row_ok, col0, N, rs);
                if (use_tma_store) {
                    const uint32_t buf = bufs + static_cast<uint32_t>(nbuf * C::EPI_BUF);
                    if (lane == 0) tzp::bulk_wait_read<1>();  // this buffer's previous store has read smem
                    __syncwarp();
                    stage_chunk(ep, buf, lane, v, r, amax);
                    tzp::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tzp::tma_store_2d(&tmOut, staging + e * 2 * C::EPI_BUF + nbuf * C::EPI_BUF, col0, row0);
                        tzp::bulk_commit();
                    }
                    nbuf ^= 1;
                } else if (row_ok) {
                    store_direct(ep, v, r, row, col0, N, amax);
                }
            }
            tzp::tc_fence_before();
            __syncwarp();
            if (lane == 0) tzp::mbar_arrive(&tempty[acc]);
            if (ep.row_absmax && row_ok) atomicMax(ep.row_absmax + row, __float_as_uint(amax));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (use_tma_store && lane == 0) tzp::bulk_wait_all();
    }

    tzp::pdl_trigger();
    tzp::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tzp::tc_fence_after();
        tzp::tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

CUtensorMapDataType tmap_dtype(int kind) {
    switch (kind) {
        case KIND_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        case KIND_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        case KIND_TF32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        default: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
    }
}

template <int KIND, int BN, int STAGES, int EPI_WARPS, int FAST = 0>
int launch_impl(tz_ctx_t ctx, const GemmArgs& g, cudaStream_t s) {
    using C = Cfg<KIND, BN, STAGES, EPI_WARPS>;
    auto kern = gemm_tc_kernel<KIND, BN, STAGES, EPI_WARPS, FAST>;
    constexpr int SMEM = (FAST & F_ON) != 0 ? C::SMEM_FAST : C::SMEM;
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static unsigned attr_set = 0;  // one bit per device
    int dev = 0;
    TZ_CUDA(cudaGetDevice(&dev));
    if (!(attr_set & (1u << (dev & 31)))) {
        TZ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        attr_set |= 1u << (dev & 31);
    }
    CUtensorMap ta, tb, to;
    const uint64_t a_rows = g.a_rows_alloc > 0 ? static_cast<uint64_t>(g.a_rows_alloc) : static_cast<uint64_t>(g.M);
    const uint64_t a_inner = (FAST & F_3X) != 0 ? static_cast<uint64_t>(2 * (g.K / 3)) : static_cast<uint64_t>(g.K);
    int rc = encode_tmap_2d(&ta, tmap_dtype(KIND), C::ELEM, g.a, a_inner, a_rows,
                            static_cast<uint64_t>(g.lda) * C::ELEM, C::BK, 128);
    if (rc) return rc;
    if constexpr ((FAST & F_BMN) != 0)  // B [K, N] row-major: 32-column x BK-row boxes
        rc = encode_tmap_2d_swz(&tb, tmap_dtype(KIND), C::ELEM, g.b, static_cast<uint64_t>(g.N),
                                static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.ldb) * C::ELEM, 32, C::BK,
                                CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    else
        rc = encode_tmap_2d(&tb, tmap_dtype(KIND), C::ELEM, g.b, static_cast<uint64_t>(g.K),
                            static_cast<uint64_t>(g.N), static_cast<uint64_t>(g.ldb) * C::ELEM, C::BK, BN);
    if (rc) return rc;
    EpiParams ep{};
    ep.bias = g.bias;
    ep.col_scale = g.col_scale;
    ep.row_scale = g.row_scale;
    ep.residual = g.residual;
    ep.ldr = g.ldr;
    ep.out = g.out;
    ep.ldo = g.ldo;
    ep.out_type = g.out_type;
    ep.gelu = g.gelu;
    ep.row_absmax = g.row_absmax;
    ep.n_ops = g.n_ops;
    ep.ops = 0;
    ep.dbg_acc = g.dbg_acc;
    for (int i = 0; i < 8; ++i) ep.ops |= (static_cast<uint64_t>(g.ops[i]) & 31u) << (5 * i);
    const int out_elem = (g.out_type == OUT_F16 || g.out_type == OUT_BF16) ? 2 : 4;
    const bool out_al = (reinterpret_cast<uintptr_t>(g.out) % 16 == 0) && ((g.ldo * out_elem) % 16 == 0);
    const bool res_al = !g.residual || ((reinterpret_cast<uintptr_t>(g.residual) % 16 == 0) && ((g.ldr * 4) % 16 == 0));
    const bool vec_al = (!g.bias || reinterpret_cast<uintptr_t>(g.bias) % 16 == 0) &&
                        (!g.col_scale || reinterpret_cast<uintptr_t>(g.col_scale) % 16 == 0);
    TZ_CHECK(vec_al, TZ_EINVAL, "gemm: bias/scale vectors must be 16-byte aligned");
    ep.vec_ok = (out_al && res_al) ? 1 : 0;
    int use_tma = (out_al && g.N % CW == 0) ? 1 : 0;
    if (use_tma) {
        const CUtensorMapDataType odt = g.out_type == OUT_F16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                        : g.out_type == OUT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : g.out_type == OUT_I32  ? CU_TENSOR_MAP_DATA_TYPE_INT32
                                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        const bool o16 = g.out_type == OUT_F16 || g.out_type == OUT_BF16;
        rc = encode_tmap_2d_swz(&to, odt, out_elem, g.out, static_cast<uint64_t>(g.N), static_cast<uint64_t>(g.M),
                                static_cast<uint64_t>(g.ldo) * out_elem, CW, 32,
                                o16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
    } else {
        to = tb;  // unused
    }
    if ((FAST & F_ON) != 0 && !use_tma) return fail(TZ_EINVAL, "gemm: specialised epilogue without TMA store");
    if (g.dbg_acc && ((FAST & F_ON) == 0 || reinterpret_cast<uintptr_t>(g.dbg_acc) % 16 != 0))
        return fail(TZ_EINVAL, "gemm: accumulator capture needs the specialised epilogue and a 16-byte aligned buffer");
    const int n_tiles = (g.N + BN - 1) / BN;
    const int tiles = ((g.M + 127) / 128) * n_tiles;
    const int sms = ctx->sm_count - ctx->sm_reserve;
    const int grid = tiles < sms ? tiles : sms;
    if (grid <= 0) return TZ_OK;
    return launch_kernel(kern, dim3(grid), dim3(C::THREADS), SMEM, s, g.pdl, ta, tb, to, g.M, g.N, g.K, ep, use_tma,
                         ctx->d_status);
}

}  // namespace

int launch_gemm(tz_ctx_t ctx, const GemmArgs& g, cudaStream_t s) {
    TZ_CHECK(g.M >= 0 && g.N > 0 && g.K > 0, TZ_EINVAL, "gemm: bad shape M=%d N=%d K=%d", g.M, g.N, g.K);
    if (g.M == 0) return TZ_OK;
    TZ_CHECK(g.a && g.b && g.out, TZ_EINVAL, "gemm: null operand");
    const int elem = g.kind == KIND_I8 ? 1 : g.kind == KIND_TF32 ? 4 : 2;
    TZ_CHECK((g.K * elem) % 16 == 0 && (g.lda * elem) % 16 == 0 && (g.ldb * elem) % 16 == 0, TZ_EINVAL,
             "gemm: K and leading dimensions must be multiples of 16 bytes (K=%d)", g.K);
    TZ_CHECK(reinterpret_cast<uintptr_t>(g.a) % 16 == 0 && reinterpret_cast<uintptr_t>(g.b) % 16 == 0,
             TZ_EINVAL, "gemm: operands must be 16-byte aligned");
    TZ_CHECK(!g.row_scale || g.col_scale, TZ_EINVAL, "gemm: row_scale needs col_scale");
    // The specialised epilogue: f16 output with 16-byte aligned rows, N a multiple of 192, bias,
    // optional row/column dequantisation scales, optional GELU (tanh form) and row |max|.
    const bool fast = (((g.kind == KIND_I8 || g.kind == KIND_F16) && g.out_type == OUT_F16) ||
                       (g.kind == KIND_BF16 && g.out_type == OUT_BF16 && !g.row_absmax)) &&
                      g.N % 192 == 0 && g.bias && !g.residual && g.n_ops < 0 && (g.gelu == 0 || g.gelu == 1) &&
                      reinterpret_cast<uintptr_t>(g.out) % 16 == 0 && (g.ldo * 2) % 16 == 0;
    TZ_CHECK(g.out_type != OUT_BF16 || fast, TZ_EUNSUPPORTED, "gemm: bf16 output only through the specialised epilogue");
    if (fast) {
        const int f = F_ON | (g.gelu == 1 ? F_GELU : 0) | (g.row_absmax ? F_AMAX : 0) |
                      (g.row_scale ? F_RSCALE : (g.col_scale ? F_CSCALE : 0)) | (g.out_type == OUT_BF16 ? F_OBF : 0);
#define TZ_FAST_CASE(K_, F_) \
    case F_: return launch_impl<K_, 192, 3, 16, F_>(ctx, g, s);
#define TZ_FAST_KIND(K_)                                                                                       \
    switch (f) {                                                                                               \
        TZ_FAST_CASE(K_, F_ON)                                                                                 \
        TZ_FAST_CASE(K_, F_ON | F_GELU)                                                                        \
        TZ_FAST_CASE(K_, F_ON | F_AMAX)                                                                        \
        TZ_FAST_CASE(K_, F_ON | F_GELU | F_AMAX)                                                               \
        TZ_FAST_CASE(K_, F_ON | F_CSCALE)                                                                      \
        TZ_FAST_CASE(K_, F_ON | F_CSCALE | F_GELU)                                                             \
        TZ_FAST_CASE(K_, F_ON | F_CSCALE | F_AMAX)                                                             \
        TZ_FAST_CASE(K_, F_ON | F_CSCALE | F_GELU | F_AMAX)                                                    \
        TZ_FAST_CASE(K_, F_ON | F_RSCALE)                                                                      \
        TZ_FAST_CASE(K_, F_ON | F_RSCALE | F_GELU)                                                             \
        TZ_FAST_CASE(K_, F_ON | F_RSCALE | F_AMAX)                                                             \
        TZ_FAST_CASE(K_, F_ON | F_RSCALE | F_GELU | F_AMAX)                                                    \
        default: break;                                                                                        \
    }
        if (g.kind == KIND_I8) {
            TZ_FAST_KIND(KIND_I8)
        } else if (g.kind == KIND_F16) {
            TZ_FAST_KIND(KIND_F16)
        } else {  // bf16 operands, bf16 output (no row |max|)
            switch (f) {
                TZ_FAST_CASE(KIND_BF16, F_ON | F_OBF)
                TZ_FAST_CASE(KIND_BF16, F_ON | F_GELU | F_OBF)
                TZ_FAST_CASE(KIND_BF16, F_ON | F_CSCALE | F_OBF)
                TZ_FAST_CASE(KIND_BF16, F_ON | F_CSCALE | F_GELU | F_OBF)
                default: break;
            }
        }
#undef TZ_FAST_KIND
#undef TZ_FAST_CASE
    }
    switch (g.kind) {
        // BN = 192 when it divides N (every Arctic projection: 384, 1152, 1536): 25% more output per
        // byte of A staged than BN = 128, and no partial tiles.
        case KIND_F16: return g.N % 192 == 0 ? launch_impl<KIND_F16, 192, 4, 16>(ctx, g, s) : launch_impl<KIND_F16, 128, 4, 16>(ctx, g, s);
        case KIND_BF16: return launch_impl<KIND_BF16, 128, 4, 16>(ctx, g, s);
        case KIND_TF32:
            if (g.a3x) {
                TZ_CHECK(!g.b_mn && g.K % 96 == 0, TZ_EINVAL, "gemm: split tf32 needs K = 3 parts of a multiple of 32");
                return g.N % 192 == 0 ? launch_impl<KIND_TF32, 192, 4, 16, F_3X>(ctx, g, s)
                                      : launch_impl<KIND_TF32, 128, 4, 16, F_3X>(ctx, g, s);
            }
            if (g.b_mn)
                return g.N % 192 == 0 ? launch_impl<KIND_TF32, 192, 4, 16, F_BMN>(ctx, g, s)
                                      : launch_impl<KIND_TF32, 128, 4, 16, F_BMN>(ctx, g, s);
            return g.N % 192 == 0 ? launch_impl<KIND_TF32, 192, 4, 16>(ctx, g, s) : launch_impl<KIND_TF32, 128, 4, 16>(ctx, g, s);
        case KIND_I8: return g.N % 192 == 0 ? launch_impl<KIND_I8, 192, 4, 16>(ctx, g, s) : launch_impl<KIND_I8, 128, 4, 16>(ctx, g, s);
        default: return fail(TZ_EINVAL, "gemm: unknown kind %d", g.kind);
    }
}

}  // namespace tz
