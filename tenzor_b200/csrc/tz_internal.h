// tz_internal.h -- host-side internals shared by the translation units of libtenzor_cuda.so.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/tenzor_cuda.h"

namespace tz {

// Thread-local last error (tz_get_last_error).
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
void clear_error();

#define TZ_CUDA(call)                                              \
    do {                                                           \
        cudaError_t _e = (call);                                   \
        if (_e != cudaSuccess) return ::tz::cuda_fail(_e, #call);  \
    } while (0)

#define TZ_CHECK(cond, code, ...)                                  \
    do {                                                           \
        if (!(cond)) return ::tz::fail((code), __VA_ARGS__);       \
    } while (0)

// A growable device scratch arena owned by a context (op-level calls that need temporaries).
struct Scratch {
    void* ptr = nullptr;
    size_t bytes = 0;
};

}  // namespace tz

struct tz_ctx_s {
    int device = 0;
    int sm_count = 0;
    int sm_reserve = 0;  // SMs the persistent GEMM grids leave free (for concurrent collective kernels)
    cudaStream_t stream = nullptr;
    int* d_status = nullptr;   // device status word (TZ_DEV_* bits)
    tz::Scratch scratch;       // op-level temporaries
    std::mutex mu;             // guards scratch growth
};

namespace tz {

cudaStream_t pick_stream(tz_ctx_t ctx, tz_stream_t s);
// Grows the context scratch to at least `bytes` (synchronising the context stream first).
int scratch_reserve(tz_ctx_t ctx, size_t bytes, void** out);
// Reads and clears the device status word; TZ_ETIMEOUT / TZ_EINVAL when a bit was set.
int read_status(tz_ctx_t ctx, cudaStream_t s);

// The tokenizer's encodeRaw (tz_tokenizer.cpp) for the document path of tz_arctic_embed_documents.
int tokenize_raw(tz_tokenizer_t tok, const char* text, int64_t len, std::vector<uint32_t>* ids);
uint32_t tokenizer_cls(tz_tokenizer_t tok);
uint32_t tokenizer_sep(tz_tokenizer_t tok);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_outer);
int encode_tmap_2d_swz(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                       uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                       uint32_t box_outer, CUtensorMapSwizzle swz);

// Kernel launch through cudaLaunchKernelEx; with `pdl` the launch may begin while the previous
// kernel in the stream is finishing (the kernel calls griddepcontrol.wait before reading inputs).
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                  Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx");
    return TZ_OK;
}

// ---- kernel launchers (defined in the .cu files) ---------------------------------------------
enum GemmKind { KIND_F16 = 0, KIND_BF16 = 1, KIND_TF32 = 2, KIND_I8 = 3 };
enum OutType { OUT_F32 = 0, OUT_F16 = 1, OUT_I32 = 2, OUT_BF16 = 3 };

struct GemmArgs {
    int kind = KIND_F16;
    const void* a = nullptr;  // [M, K] row-major, lda elements
    const void* b = nullptr;  // [N, K] row-major, ldb elements
    int64_t lda = 0, ldb = 0;
    int M = 0, N = 0, K = 0;
    int64_t a_rows_alloc = 0; // rows of A that are addressable (>= M); TMA bound
    // epilogue
    const float* bias = nullptr;       // [N]
    const float* col_scale = nullptr;  // [N]
    const float* row_scale = nullptr;  // [M]
    const float* residual = nullptr;   // [M, ldr] f32
    int64_t ldr = 0;
    void* out = nullptr;               // [M, ldo]
    int64_t ldo = 0;
    int out_type = OUT_F32;
    int gelu = 0;                      // after bias: 1 model GELU (hardware tanh), 2 codegen GELU
                                       // (tanh = 2 sigmoid(2x) - 1), 3 ReLU
    unsigned* row_absmax = nullptr;    // [M] atomicMax of |stored value| (float bits)
    int n_ops = -1;                    // >= 0: generic op chain instead of the fixed epilogue
    bool b_mn = false;                 // tf32 only: b is [K, N] row-major (ldb >= N), read N-major
    // tf32 only, f32-accurate products from three tf32 ones (x = hi + lo, hi = tf32(x)):
    // a rows hold [hi | lo] (K/3 each), b rows [hi | lo | hi], and the MMA walks K = 3 parts with A
    // reading hi, hi, lo: sum hi_a hi_b + hi_a lo_b + lo_a hi_b.  K/3 a multiple of 32.
    bool a3x = false;
    int ops[8] = {0};
    bool pdl = false;                  // programmatic dependent launch (inside the model forward)
    // Parity capture (int8 kind, specialised epilogue): when non-null the epilogue also stores the
    // raw int32 accumulators it reads from TMEM to dbg_acc [M, N] row-major.  A runtime pointer of
    // the same kernel instantiation: the forward's own code path writes the capture.
    int32_t* dbg_acc = nullptr;
};
int launch_gemm(tz_ctx_t ctx, const GemmArgs& g, cudaStream_t s);

// GEMM with N = 384 whose epilogue adds bias + residual and applies LayerNorm (tz_gemm_ln.cu).
// The model's residual stream X [rows, 384] f32 in blocked form: per group of 32 rows, 96 column
// quads, each quad 32 rows x 4 floats (512 contiguous bytes).  A warp that owns 32 rows (one per
// lane) reads or writes a 16-column chunk as four fully coalesced 512-byte accesses.  Buffers hold
// whole 128-row tiles (rows rounded up to a multiple of 128).
__host__ __device__ __forceinline__ long long xblk(long long row, int col) {
    return (((row >> 5) * 96 + (col >> 2)) << 7) + ((row & 31) << 2) + (col & 3);
}
inline long long xblk_rows(long long rows) { return (rows + 127) / 128 * 128; }

struct GemmLnArgs {
    int kind = KIND_F16;
    const void* a = nullptr;  // [M, K]
    const void* b = nullptr;  // [384, K]
    int64_t lda = 0, ldb = 0;
    int M = 0, K = 0;
    const float* bias = nullptr;       // [384]
    const float* col_scale = nullptr;  // [384]
    const float* row_scale = nullptr;  // [M]
    const float* residual = nullptr;   // [M, 384] f32, blocked (xblk), may alias x_out
    const float* gamma = nullptr;
    const float* beta = nullptr;
    float eps = 1e-12f;
    float* x_out = nullptr;            // [M, 384] f32, blocked (xblk)
    void* aux = nullptr;               // [M, 384] f16 or int8
    float* aux_scale = nullptr;        // [M] when aux is int8
    bool aux_int8 = false;
    bool aux_bf16 = false;             // a 16-bit aux is bf16 (else IEEE half)
    // W8A8 with the A operand quantised inside the kernel: `a` is then f16 [M, K] (row stride lda)
    // and a_absmax [M] holds each row's |max| (float bits, accumulated by the producer with
    // atomicMax); the kernel derives the per-token scale from it, quantises A into its int8 stages
    // and resets a_absmax[row] to 0 once the row is done.  kind must be KIND_I8, row_scale null.
    unsigned* a_absmax = nullptr;
    bool pdl = false;
    // Parity capture (same kernel instantiation, runtime pointers): dbg_acc [M, 384] receives the
    // raw accumulators (int32 for the int8 kind) read in the LayerNorm epilogue; with in-kernel A
    // quantisation dbg_aq [M, K] receives the int8 A rows as quantised into the MMA stages and
    // dbg_as [M] their per-token scales.
    int32_t* dbg_acc = nullptr;
    int8_t* dbg_aq = nullptr;
    float* dbg_as = nullptr;
};
int launch_gemm_ln(tz_ctx_t ctx, const GemmLnArgs& g, cudaStream_t s);

// The W8A8 feed-forward block in one kernel (tz_ffn.cu): FFN1 + GELU + per-token int8 + FFN2 +
// bias + residual + LayerNorm + the next layer's int8 operand, with the GELU output kept on chip.
struct FfnArgs {
    const int8_t* xq = nullptr;   // [M, 384] int8 operand; overwritten with the int8 LayerNorm output
    float* xs = nullptr;          // [M] its per-token scales; overwritten with the output's
    const int8_t* w1 = nullptr;   // [1536, 384]
    const float* s1 = nullptr;    // [1536] per-output-channel scales
    const float* b1 = nullptr;    // [1536]
    const int8_t* w2 = nullptr;   // [384, 1536]
    const float* s2 = nullptr;    // [384]
    const float* b2 = nullptr;    // [384]
    const float* gamma = nullptr;
    const float* beta = nullptr;
    float eps = 1e-12f;
    float* x = nullptr;           // [M, 384] f32 residual stream, blocked (xblk), updated in place
    int M = 0;
    bool pdl = false;
    // Parity capture (runtime pointers of the same kernel): FFN1 accumulators [M, 1536], the f16 GELU
    // output as quantised [M, 1536], its int8 form [M, 1536] and per-token scales [M], FFN2
    // accumulators [M, 384].
    int32_t* dbg_acc1 = nullptr;
    void* dbg_h16 = nullptr;
    int8_t* dbg_hq = nullptr;
    float* dbg_hs = nullptr;
    int32_t* dbg_acc2 = nullptr;
};
int launch_ffn_w8a8(tz_ctx_t ctx, const FfnArgs& a, cudaStream_t s);

}  // namespace tz
