/*
 * tenzor_cuda.h -- C ABI of libtenzor_cuda.so, the sm_100a (B200) backend for the Arctic-embed-xs
 * encoder hot path of tenzor.
 *
 * The reference (mattneel/tenzor) is Zig; its host code binds this header with `extern fn`
 * declarations of the same names and types.  Every entry point names the reference function it replaces
 * (path:line inside the reference project).  Conventions, mirroring the reference kernels:
 *   - caller-owned, contiguous, row-major buffers plus explicit dimensions;
 *   - Linear weights in PyTorch layout [out, in];
 *   - int8 weights carry one IEEE-half scale per output row (quantize_arctic_xs.zig:94-115);
 *   - every call returns a tz_status; tz_get_last_error() gives the message of the last failing
 *     call on the calling thread (the reference's error unions, arctic.zig:194-201, become codes).
 * Op-level entry points (tz_layernorm_last_dim ... tz_gather_rows) take DEVICE pointers and a
 * stream and are asynchronous; the model entry points take HOST pointers and are synchronous
 * unless noted.  There is no CPU fallback: without a usable sm_100 device every call fails with
 * TZ_ECUDA or TZ_EUNSUPPORTED.
 */
#ifndef TENZOR_CUDA_H
#define TENZOR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ------------------------------------------------------------------------------- */
typedef enum {
    TZ_OK = 0,
    TZ_EINVAL = 1,       /* bad argument (shape, null pointer, id out of range)              */
    TZ_ENOMEM = 2,       /* device allocation failed                                          */
    TZ_ECUDA = 3,        /* CUDA runtime/driver error                                         */
    TZ_ETIMEOUT = 4,     /* a bounded device-side wait expired; the kernel returned early     */
    TZ_EUNSUPPORTED = 5, /* not supported on this device / combination                        */
    TZ_EMISSING = 6      /* a required weight is missing (arctic.zig:194-196 MissingWeight)   */
} tz_status;

typedef struct tz_ctx_s* tz_ctx_t;     /* one device + one default stream + scratch arena */
typedef struct tz_model_s* tz_model_t; /* device-resident Arctic-embed-xs weights + workspace */
typedef struct tz_tokenizer_s* tz_tokenizer_t; /* WordPiece vocabulary (host) */
typedef void* tz_stream_t;             /* a cudaStream_t; NULL = the context's stream */

/* Message of the last failing call on this thread ("" if none).  SPEC.md:876 tz_get_last_error. */
const char* tz_get_last_error(void);
/* Library version string and build flags. */
const char* tz_version(void);

/* ---- context ------------------------------------------------------------------------------ */
/* Creates a context on CUDA device `device`.  Fails with TZ_EUNSUPPORTED unless the device is
 * compute capability 10.0 (B200).  Replaces the CPU ThreadPool.create of main.zig:787-789. */
int tz_cuda_create(int device, tz_ctx_t* out);
int tz_cuda_destroy(tz_ctx_t ctx);
int tz_cuda_synchronize(tz_ctx_t ctx);
/* Device status word: non-zero when a kernel's bounded wait expired (bit 0) or a kernel bounds
 * check fired (bit 1) since the last call.  Reading clears it. */
int tz_cuda_check_status(tz_ctx_t ctx);
int tz_cuda_sm_count(tz_ctx_t ctx);
/* Persistent GEMM grids of this context (the model's projections and the op-level GEMMs) use at most
 * SMs - n CTAs, so that n SMs stay free for kernels that run concurrently on another stream -- the
 * collective of a multi-GPU pipeline (e.g. NCCL limited to n CTAs with NCCL_MAX_CTAS), which would
 * otherwise hold SMs the one-CTA-per-SM grids wait for.  0 (the default) uses every SM. */
int tz_cuda_set_sm_reserve(tz_ctx_t ctx, int n);
/* Failure-detection self-test: runs a kernel whose bounded device wait (the one every kernel's
 * mbarrier waits use) can never be satisfied, so it expires after ~1 s and the kernel returns.
 * Returns TZ_ETIMEOUT (and clears the status word); the context stays usable. */
int tz_cuda_selftest_wait(tz_ctx_t ctx);

/* ---- device memory (SPEC.md:834-845 tz_tensor_from_data / copy_to_host) ------------------- */
int tz_alloc(tz_ctx_t ctx, size_t bytes, void** dptr);
int tz_free(tz_ctx_t ctx, void* dptr);
int tz_upload(tz_ctx_t ctx, void* dst_device, const void* src_host, size_t bytes);
int tz_download(tz_ctx_t ctx, void* dst_host, const void* src_device, size_t bytes);

/* ---- Arctic-embed-xs model ---------------------------------------------------------------- */
typedef enum {
    TZ_QUANT_F32 = 0,   /* f32 checkpoint; GEMMs on tcgen05 kind::f16 (f16 operands, f32 acc) */
    TZ_QUANT_W8A32 = 1, /* int8 checkpoint, f32 activations: the reference's int8 path        */
    TZ_QUANT_W8A8 = 2   /* int8 checkpoint, per-token int8 activations, int32 accumulators    */
} tz_quant_mode;

/* MatWeight (arctic.zig:47-58): either f32 [rows, cols] or int8 [rows, cols] + half scale [rows].
 * Exactly one of `f32` and `q8` is non-NULL. */
typedef struct {
    const float* f32;
    const int8_t* q8;
    const uint16_t* scale_f16;
} tz_mat_weight;

/* LayerWeights (arctic.zig:64-89). */
typedef struct {
    tz_mat_weight query, key, value, attn_output, intermediate, output;
    const float *query_bias, *key_bias, *value_bias, *attn_output_bias, *intermediate_bias,
        *output_bias;
    const float *attn_ln_gamma, *attn_ln_beta, *output_ln_gamma, *output_ln_beta;
} tz_arctic_layer;

/* ModelWeights (arctic.zig:92-110), config arctic.zig:29-42 (6 layers fixed). */
typedef struct {
    tz_mat_weight word_embeddings, position_embeddings, token_type_embeddings;
    const float *ln_gamma, *ln_beta;
    tz_arctic_layer layers[6];
} tz_arctic_weights;

/* Copies the host weights to the device in the layout the kernels want (QKV concatenated,
 * f16 or int8 operands, f32 scales).  TZ_QUANT_F32 needs f32 Linear weights.  The int8 modes take
 * q8 Linear weights (embedding tables may be either), or an all-f32 checkpoint, which is then
 * quantised on the device during the load exactly as quantize_arctic_xs.zig:22-115 would (every
 * Linear weight and the word / position tables; the 768-element type table stays f32).
 * Replaces ModelWeights.fromSafeTensors, arctic.zig:113-166 / getMatWeightAlloc 258-287. */
int tz_arctic_load(tz_ctx_t ctx, const tz_arctic_weights* w, int mode, tz_model_t* out);
/* GEMM operand precision of the f16-operand modes (TZ_QUANT_F32 and TZ_QUANT_W8A32): the 16-bit type
 * of every weight copy, GEMM operand and intermediate activation (QKV, attention and GELU outputs) of
 * the forward; accumulation, LayerNorm, softmax statistics and the residual stream stay f32.
 * TZ_PREC_BF16 trades three mantissa bits for f32's exponent range (checkpoints whose activations
 * exceed the f16 range).  W8A8 runs int8 GEMMs and takes only TZ_PREC_F16.  The op-level f32 GEMMs
 * offer the f32-accurate split-tf32 form (tz_matmul_f32x3); the model does not. */
typedef enum { TZ_PREC_F16 = 0, TZ_PREC_BF16 = 1 } tz_gemm_prec;
/* tz_arctic_load with an explicit GEMM precision (tz_arctic_load is prec = TZ_PREC_F16);
 * TZ_EUNSUPPORTED for a precision the mode does not run. */
int tz_arctic_load_ex(tz_ctx_t ctx, const tz_arctic_weights* w, int mode, int prec, tz_model_t* out);
/* Same, reading a safetensors checkpoint (f32, or I8 + '<name>.scale' F16 as written by
 * quantize_arctic_xs.zig), with or without the "bert." prefix.  safetensors.zig:275-295. */
int tz_arctic_load_safetensors(tz_ctx_t ctx, const char* path, int mode, tz_model_t* out);
int tz_arctic_free(tz_model_t model);
/* Reserves device workspace for up to max_batch sequences and max_tokens packed tokens
 * (InferenceContext.init, arctic.zig:424-460).  Forward calls grow it on demand otherwise. */
int tz_arctic_reserve(tz_model_t model, int max_batch, int64_t max_tokens);

/* Batch forward over ragged sequences (forwardBatchParallel, arctic.zig:959-1013, and forward,
 * arctic.zig:874-898): ids_packed holds the B sequences back to back, cu_seqlens[B+1] their
 * offsets (cu_seqlens[0] = 0, 1 <= length <= 512, ids < 30522).  Writes the L2-normalised CLS
 * embedding of each sequence to out[B, 384].  HOST pointers; synchronous. */
int tz_arctic_forward(tz_model_t model, const uint32_t* ids_packed, const int32_t* cu_seqlens,
                      int batch, float* out);
/* Padded batch: ids[B, S] row-major, lengths[B] (the masked-batch form; tokens at positions
 * >= length are ignored).  HOST pointers; synchronous. */
int tz_arctic_forward_padded(tz_model_t model, const uint32_t* ids, const int32_t* lengths,
                             int batch, int seq, float* out);
/* Device-resident variant: all pointers on the device, asynchronous on `stream`.  total_tokens =
 * cu_seqlens[B] and max_len >= every length must be passed by the caller (no host read-back); a
 * sequence longer than max_len is refused on the device (the bounds bit of the status word, so the
 * next tz_cuda_check_status returns TZ_EINVAL) and its embedding is not valid.  The
 * launch sequence is captured into a CUDA graph on first use and replayed while the buffers, the
 * shape and the stream repeat (the legacy default stream is never captured). */
int tz_arctic_forward_device(tz_model_t model, const uint32_t* d_ids_packed,
                             const int32_t* d_cu_seqlens, int batch, int64_t total_tokens,
                             int max_len, float* d_out, tz_stream_t stream);
/* Debug/parity hook: copies the device hidden state [T, 384] after stage `stage` (0 = after the
 * embeddings, l+1 = after layer l, 7 = layer 0's state after its attention block, i.e. the FFN1
 * input) of the LAST forward into host `out`.  Capture is switched on by a first call (which returns
 * TZ_EINVAL) and applies from the next forward. */
int tz_arctic_debug_hidden(tz_model_t model, int stage, float* out, int64_t total_tokens);
/* Switches the capture of the debug hooks on (from the next forward) or off (frees the capture
 * buffers; the forward returns to its captured CUDA graph). */
int tz_arctic_debug_capture(tz_model_t model, int on);
/* Debug/parity hooks (W8A8), written by the forward's own GEMM kernels for layer 0 during the LAST
 * forward (which: 0 = QKV, 1 = attention-output projection, 2 = FFN1, 3 = FFN2).  Capture is
 * switched on by a first call to any of them (which returns TZ_EINVAL) and applies from the next
 * forward; it adds stores to the same kernels and is meant for parity tests only.
 *   tz_arctic_debug_operand:    the int8 A operand [T, K] as the GEMM consumed it (K = 384, or 1536
 *                               for which = 3) and its per-token f32 scale [T]; for which = 1 and 3
 *                               these are the rows the gemm_ln kernel quantised into its MMA stages;
 *   tz_arctic_debug_accum:      the raw int32 accumulators [T, N] the epilogue read from TMEM
 *                               (N = 1152, 384, 1536, 384);
 *   tz_arctic_debug_gemm_input: (which = 1, 3) the f16 activation [T, K] (IEEE half bits) that the
 *                               kernel quantised per token. */
int tz_arctic_debug_operand(tz_model_t model, int which, int8_t* q_out, float* scale_out,
                            int64_t total_tokens);
int tz_arctic_debug_accum(tz_model_t model, int which, int32_t* acc_out, int64_t total_tokens);
int tz_arctic_debug_gemm_input(tz_model_t model, int which, uint16_t* x_out, int64_t total_tokens);

/* W8A8 feed-forward form.  fused = 0 (the default): the FFN1 GEMM writes the f16 GELU output to
 * device memory and the FFN2 kernel quantises it per token in its mainloop.  fused = 1: FFN1, GELU,
 * the per-token int8 quantisation of the GELU output, FFN2, bias, residual and LayerNorm run as one
 * kernel per layer and the GELU output never leaves the SM (FFN1 is computed twice per row tile:
 * once for each row's max |GELU|, which the per-token scale needs before any value can be
 * quantised, and once to quantise and feed FFN2); on B200 it is slower (the doubled GELU work is
 * bound by the special-function unit's tanh rate).  Both forms give bit-identical results; other
 * modes ignore the setting.  Replaces nothing in the reference: feedForward (arctic.zig:760-810) is
 * one function there. */
int tz_arctic_set_ffn_fusion(tz_model_t model, int fused);

/* Kernel timing of the forward: when enabled (enable = number of forwards to keep, 0 = off), CUDA
 * events are recorded on the launching stream between consecutive launches (inside a captured
 * graph too).  tz_arctic_profile_read returns, summed over the kept forwards since enabling, the
 * milliseconds and the launch count per kernel class:
 * 0 embedding+LN, 1 QKV GEMM, 2 attention, 3 attention-output GEMM + residual + LayerNorm,
 * 4 (unused: LayerNorm is fused into 3 and 7), 5 FFN1 GEMM,
 * 6 the fused W8A8 feed-forward block (FFN1 + GELU + FFN2 + residual + LayerNorm), 7 FFN2 GEMM +
 * residual + LayerNorm, 8 CLS pool + L2 (arrays of TZ_PROF_CLASSES). */
#define TZ_PROF_CLASSES 9
int tz_arctic_profile(tz_model_t model, int enable);
int tz_arctic_profile_read(tz_model_t model, float* ms, int* launches);

/* ---- op-level kernels (device pointers, async on `stream`) ------------------------------- */
/* Epilogue / unary op codes (OpTag subset of expr.zig:19-135 used by codegen.zig:228-244). */
typedef enum {
    TZ_OP_ADD = 1, /* bias add (matmul epilogue) */
    TZ_OP_RELU = 2,
    TZ_OP_GELU = 3, /* simd.zig gelu: tanh(x) = 2*sigmoid(2x)-1 */
    TZ_OP_SIGMOID = 4,
    TZ_OP_TANH = 5,
    TZ_OP_EXP = 6,
    TZ_OP_NEG = 7,
    TZ_OP_ABS = 8,
    TZ_OP_SILU = 9,
    TZ_OP_LOG = 10,
    TZ_OP_SQRT = 11,
    TZ_OP_RSQRT = 12,
    TZ_OP_SIN = 13,
    TZ_OP_COS = 14,
    TZ_OP_ERF = 15,       /* erf (the device erff)                                               */
    TZ_OP_GELU_ERF = 16,  /* the ONNX specification's Gelu: 0.5 x (1 + erf(x / sqrt 2))          */
    TZ_OP_ERF_AS = 17,    /* the reference ONNX executor's Erf (onnx/executor.zig:125-137): the
                             Abramowitz-Stegun 7.1.26 polynomial, |error| <= 1.5e-7               */
    TZ_OP_GELU_TANH = 18, /* the reference ONNX executor's Gelu (onnx/executor.zig:122):
                             0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))) with tanhf         */
    /* binary ops of an elementwise program (BinaryExpr, expr.zig:352-513) */
    TZ_EW_ADD = 20,
    TZ_EW_SUB = 21,
    TZ_EW_MUL = 22,
    TZ_EW_DIV = 23,
    TZ_EW_MAX = 24,
    TZ_EW_MIN = 25,
    TZ_EW_POW = 26,   /* powf(a, b) (onnx/executor.zig:3558 execPow)                             */
    TZ_EW_EQ = 27,    /* a == b ? 1 : 0 (execEqual 2656)                                         */
    TZ_EW_LT = 28,    /* a < b ? 1 : 0 (execCompare .less)                                       */
    TZ_EW_GT = 29,    /* a > b ? 1 : 0 (execCompare .greater)                                    */
    /* ternary op: reg[dst] = reg[a] != 0 ? reg[b] : reg[c] (execWhere 2733)                     */
    TZ_EW_WHERE = 30
} tz_op;
#define TZ_OP_LAST_UNARY TZ_OP_GELU_TANH

typedef enum { TZ_RED_SUM = 0, TZ_RED_MEAN = 1, TZ_RED_PROD = 2, TZ_RED_MAX = 3, TZ_RED_MIN = 4 } tz_reduce_op;

/* layerNormLastDim, layernorm.zig:26-116 (two-pass mean/variance).  x and y may alias. */
int tz_layernorm_last_dim(tz_ctx_t ctx, const float* x, const float* gamma, const float* beta,
                          float* y, int64_t rows, int cols, float eps, tz_stream_t stream);
/* softmaxLastAxis with optional additive mask [rows, cols] (softmax.zig:20-155); mask may be
 * NULL.  x and y may alias. */
int tz_softmax_last_axis(tz_ctx_t ctx, const float* x, const float* mask, float* y, int64_t rows,
                         int cols, tz_stream_t stream);
/* Attention-shaped masked softmax: x [groups, rows_per_group, cols]; in group g only the first
 * key_len[g] columns are valid (others get probability 0), the additive-mask form of
 * softmax.zig:423-440 with mask = -inf beyond the valid length. */
int tz_softmax_keylen(tz_ctx_t ctx, const float* x, const int32_t* key_len, float* y,
                      int64_t groups, int rows_per_group, int cols, tz_stream_t stream);
/* selfAttention, arctic.zig:639-747, over packed sequences (the kernel of the Arctic forward):
 * qkv [total_tokens, 1152] 16-bit, row t = Q | K | V of token t (12 heads of 32 columns each);
 * cu_seqlens device int32 [batch + 1], nondecreasing from 0 to total_tokens; out [total_tokens, 384]
 * of the same type: for each head, softmax(Q K^T / sqrt(32)) V over the keys of the token's own
 * sequence.  max_len (1..512) must bound every sequence length: a longer sequence is refused on the
 * device (tz_cuda_check_status then returns TZ_EINVAL).  bf16 = 1 reads and writes bfloat16, 0 IEEE
 * half.  qkv and out 16-byte aligned. */
int tz_attention(tz_ctx_t ctx, const void* qkv, int64_t total_tokens, const int32_t* cu_seqlens, int batch,
                 int max_len, void* out, int bf16, tz_stream_t stream);
/* linearProjection f32 arm, arctic.zig:599-620 (matmulTransposeB matmul.zig:54-77 + bias):
 * y[m,n] = x[m,k] w[n,k]^T (+ bias) [+ residual].  tcgen05 kind::tf32. */
int tz_linear_f32(tz_ctx_t ctx, const float* x, const float* w, const float* bias,
                  const float* residual, float* y, int m, int k, int n, tz_stream_t stream);
/* matmulTransposeB_f32_i8_rowScale_bias, matmul_w8a32.zig:14-58:
 * y = (x w_q^T) * f32(scale[j]) + bias[j].  Needs scratch from the context arena. */
int tz_linear_w8a32(tz_ctx_t ctx, const float* x, const int8_t* wq, const uint16_t* scale_f16,
                    const float* bias, float* y, int m, int k, int n, tz_stream_t stream);
/* W8A8 linear: per-token int8 quantisation of x, int8 x int8 -> int32 on tcgen05 kind::i8,
 * y = float(acc) * (sx[i] * f32(scale[j])) + bias[j].  No reference counterpart (the reference
 * int8 path is W8A32); scratch from the context arena. */
int tz_linear_w8a8(tz_ctx_t ctx, const float* x, const int8_t* wq, const uint16_t* scale_f16,
                   const float* bias, float* y, int m, int k, int n, tz_stream_t stream);
/* tz_linear_w8a8 for callers that cannot allocate device memory while they run (inside a CUDA
 * graph capture, under an allocator that has reserved all device memory, or on a thread that cannot
 * take the device-wide synchronisation of cudaMalloc / cudaFree).  This entry point has no
 * counterpart in the reference.  It allocates nothing: its temporaries live in an 8 MiB device array
 * that the library owns (every GPU that loads the library holds it until exit), so it needs
 * m*k + 4*m + 4*n bytes (each part rounded up to 256) <= 8 MiB and returns TZ_EINVAL otherwise.
 * The first call on a device looks the array's address up (cudaGetSymbolAddress); make that first
 * call before any stream capture.  All calls share the array: calls that overlap on the GPU race.
 * The context's device must be the calling thread's current device (TZ_EINVAL otherwise); the
 * array's address is kept per device for the life of the process, which assumes the device's
 * primary context is not reset (cudaDeviceReset) while the library is loaded.
 * Same arguments, result and stream semantics as tz_linear_w8a8. */
int tz_linear_w8a8_noalloc(tz_ctx_t ctx, const float* x, const int8_t* wq, const uint16_t* scale_f16,
                           const float* bias, float* y, int m, int k, int n, tz_stream_t stream);
/* Raw int8 GEMM: c[m,n] = a[m,k] w[n,k]^T in int32 (bit-exact accumulators).  k % 16 == 0. */
int tz_gemm_i8_i32(tz_ctx_t ctx, const int8_t* a, const int8_t* w, int32_t* c, int m, int k,
                   int n, tz_stream_t stream);
/* Per-row symmetric weight quantiser of quantize_arctic_xs.zig:94-115 (f16 scales). */
int tz_quantize_weight_rows(tz_ctx_t ctx, const float* w, int8_t* q, uint16_t* scale_f16,
                            int64_t rows, int cols, tz_stream_t stream);
/* Per-token activation quantiser used by the W8A8 path: s = max|x|/127 (1 if 0),
 * q = clamp(round(x * (1/s)), -127, 127). */
int tz_quantize_act_rows(tz_ctx_t ctx, const float* x, int8_t* q, float* scale, int64_t rows,
                         int cols, tz_stream_t stream);
/* FusedMatmulEpilogueKernel, codegen.zig:78-147: c = ops(a @ b) with b [k,n] (trans_b = 0) or
 * [n,k] (trans_b = 1); ops applied in order, TZ_OP_ADD adds bias[j].  n_ops <= 8.
 * tcgen05 kind::tf32; a trans_b = 0 operand is transposed through context scratch first. */
int tz_matmul_epilogue(tz_ctx_t ctx, const float* a, const float* b, int trans_b,
                       const float* bias, const int* ops, int n_ops, float* c, int m, int k, int n,
                       tz_stream_t stream);
/* Elementwise chain exp((a + b) * c), b broadcast along rows ([cols]); executor.zig:114-197
 * evaluation of UnaryExpr(exp, BinaryExpr(mul, BinaryExpr(add, a, b), c)) in one pass. */
int tz_ew_add_mul_exp(tz_ctx_t ctx, const float* a, const float* b_row, const float* c, float* out,
                      int64_t rows, int cols, tz_stream_t stream);
/* A fused elementwise expression over up to 4 broadcast inputs, evaluated in one pass (the launch
 * that an elementwise_chain FusionPlan, analyzer.zig:106-153, lowers to).  Input k is read at
 * in[k][r * row_stride[k] + c * col_stride[k]] for output element (r, c) of [rows, cols] (stride 0 =
 * broadcast, executor.zig:152-197).  Instruction i computes reg[dst] = op(reg[a], reg[b]); registers
 * 0..3 hold the inputs, 4..11 temporaries, 12..15 the constants consts[0..3]; unary ops
 * (TZ_OP_RELU..TZ_OP_LAST_UNARY) ignore b.  The output is reg[result]. */
#define TZ_EW_MAX_INPUTS 4
#define TZ_EW_MAX_INSTR 16
typedef struct {
    int op, dst, a, b, c; /* c: third operand of TZ_EW_WHERE, ignored otherwise */
} tz_ew_instr;
typedef struct {
    int n_inputs;
    const float* in[TZ_EW_MAX_INPUTS];
    int64_t row_stride[TZ_EW_MAX_INPUTS];
    int64_t col_stride[TZ_EW_MAX_INPUTS];
    int n_instr;
    tz_ew_instr instr[TZ_EW_MAX_INSTR];
    int result;
    float consts[4];
} tz_ew_program;
int tz_ew_program_run(tz_ctx_t ctx, const tz_ew_program* prog, float* out, int64_t rows, int cols,
                      tz_stream_t stream);
/* The same program over N-D broadcast operands (evalBinaryBroadcast, executor.zig:152-197, any rank
 * up to TZ_MAX_DIMS): out is row-major [shape]; input k of output element idx is read at
 * in[k][sum_d idx[d] * stride[k][d]] (element strides, 0 along a broadcast dimension).  The
 * program's row_stride / col_stride are not used. */
#define TZ_MAX_DIMS 6
typedef struct {
    int ndim;
    int64_t shape[TZ_MAX_DIMS];
    int64_t stride[TZ_EW_MAX_INPUTS][TZ_MAX_DIMS];
} tz_nd_layout;
int tz_ew_program_run_nd(tz_ctx_t ctx, const tz_ew_program* prog, const tz_nd_layout* layout, float* out,
                         tz_stream_t stream);
/* General fused elementwise chain (FusedElementwiseKernel, codegen.zig:15-74): out = ops(x). */
int tz_ew_unary_chain(tz_ctx_t ctx, const float* x, float* out, int64_t n, const int* ops,
                      int n_ops, tz_stream_t stream);
/* FusedReduceKernel, codegen.zig:151-205: *out (device) = reduce(pre_ops(x)). */
int tz_reduce(tz_ctx_t ctx, int reduce_op, const int* pre_ops, int n_pre, const float* x,
              int64_t n, float* out, tz_stream_t stream);
/* ---- N-D tensor ops of the `.eval()` executor and the ONNX op map ---------------------------
 * Device pointers, asynchronous on `stream`, f32 unless noted. */
/* Batched matmul with broadcast batch dimensions (evalBatchedMatmul, executor.zig:199-325, and
 * execMatMul, onnx/executor.zig:1490): for every batch index b (up to 4 dimensions, row-major
 * batch_shape), c[b][i, j] = sum_k a[b][i, k] * b[b][k, j], where operand element (i, k) of batch b
 * is at a + sum_d b[d] * a_bstride[d] + i * a_rs + k * a_cs (element strides; a zero batch stride
 * broadcasts; the matrix strides express transposed or head-interleaved views without a copy), and
 * the same for b and c.  Contiguous batches of large products go to the tcgen05 GEMM (tf32);
 * small or strided ones to an f32 CUDA-core kernel with f32 accumulation. */
typedef struct {
    int batch_ndim;
    int64_t batch_shape[4];
    int64_t a_bstride[4], b_bstride[4], c_bstride[4];
    int64_t a_rs, a_cs, b_rs, b_cs, c_rs, c_cs;
    int m, k, n;
} tz_bmm_layout;
int tz_batched_matmul(tz_ctx_t ctx, const float* a, const float* b, float* c, const tz_bmm_layout* layout,
                      tz_stream_t stream);
/* tz_matmul_epilogue with f32-accurate products: both operands are split into a tf32 head and its
 * f32 remainder in context scratch and the tcgen05 GEMM sums hi*hi + hi*lo + lo*hi with f32
 * accumulation (the dropped lo*lo term is about 2^-22 of each product).  Same arguments. */
int tz_matmul_f32x3(tz_ctx_t ctx, const float* a, const float* b, int trans_b, const float* bias,
                    const int* ops, int n_ops, float* c, int m, int k, int n, tz_stream_t stream);
/* reduceAxis (reduce.zig:52-95, executor.zig:327-361): x viewed as [outer, len, inner];
 * out[outer, inner] = reduce over len (sum / mean accumulate in f64; mean divides by len). */
int tz_reduce_axis(tz_ctx_t ctx, int reduce_op, const float* x, int64_t outer, int64_t len, int64_t inner,
                   float* out, tz_stream_t stream);
/* softmaxAxis (softmax.zig:157-220): x and y viewed as [outer, len, inner], softmax over len
 * (max-subtracted exp, then multiplied by 1 / sum).  x and y may alias. */
int tz_softmax_axis(tz_ctx_t ctx, const float* x, float* y, int64_t outer, int64_t len, int64_t inner,
                    tz_stream_t stream);
/* Transpose (onnx/executor.zig:2296-2390): y = x permuted, x row-major [shape[0..ndim)], y row-major
 * with y's dimension d = x's dimension perm[d]; elements of elem_bytes = 1, 2, 4 or 8. */
int tz_permute(tz_ctx_t ctx, const void* x, void* y, int elem_bytes, int ndim, const int64_t* shape,
               const int* perm, tz_stream_t stream);
/* Cast (onnx/executor.zig:2852): element conversion between the TZ_DT_* types f32, f16, i8, i32,
 * i64 and u8 (bool); float to integer truncates toward zero. */
int tz_cast(tz_ctx_t ctx, const void* x, int src_dtype, void* y, int dst_dtype, int64_t n, tz_stream_t stream);
/* Concat (onnx/executor.zig:2112-2225): inputs viewed as [outer, axis_len[i] * inner] row-major, out
 * [outer, sum(axis_len) * inner]; elements of elem_bytes. */
int tz_concat(tz_ctx_t ctx, const void* const* inputs, const int64_t* axis_len, int n_inputs, int64_t outer,
              int64_t inner, int elem_bytes, void* out, tz_stream_t stream);

/* gather, gather.zig:15-57: out[i,:] = table[ids[i],:]; ids out of range -> TZ_EINVAL via the
 * device status word (the row is zero-filled). */
int tz_gather_rows(tz_ctx_t ctx, const float* table, int64_t table_rows, const uint32_t* ids,
                   int64_t n_ids, int cols, float* out, tz_stream_t stream);

/* ---- LeNet-5 batch inference ------------------------------------------------------------------
 * Replaces LeNet.forward (lenet.zig:262-268 -> forwardSequential 270-321 / forwardParallel
 * 323-513): conv1 6@5x5 -> ReLU -> 2x2 maxpool -> conv2 16@5x5 -> ReLU -> 2x2 maxpool -> flatten
 * (NHWC) -> FC 120 -> ReLU -> FC 84 -> ReLU -> FC 10.  Images are [n, 28, 28, 1] f32 (NHWC); conv
 * weights [out, kh, kw, in] and FC weights [out, in] as LeNetWeights (lenet.zig:33-52).
 *   TZ_LENET_REF:  lenet.zig as written: conv1 valid (24x24), FC1 in = 256, out = logits [n, 10].
 *   TZ_LENET_PAD2: conv1 zero padding 2 (28x28), FC1 in = 400, out = softmax(logits) [n, 10]. */
typedef struct tz_lenet_s* tz_lenet_t;
enum { TZ_LENET_REF = 0, TZ_LENET_PAD2 = 1 };
typedef struct {
    const float *conv1_w, *conv1_b; /* [6,5,5,1], [6] */
    const float *conv2_w, *conv2_b; /* [16,5,5,6], [16] */
    const float *fc1_w, *fc1_b;     /* [120, 256 | 400], [120] */
    const float *fc2_w, *fc2_b;     /* [84,120], [84] */
    const float *fc3_w, *fc3_b;     /* [10,84], [10] */
} tz_lenet_weights;
/* Copies the host weights to the context's device (LeNet.init + initKaiming's caller-provided
 * weights).  TZ_EMISSING when a pointer is NULL. */
int tz_lenet_load(tz_ctx_t ctx, const tz_lenet_weights* w, int variant, tz_lenet_t* out);
int tz_lenet_free(tz_lenet_t model);
/* Pre-sizes the device scratch for n images (otherwise grown on demand, which synchronises). */
int tz_lenet_reserve(tz_lenet_t model, int64_t n);
/* Host images [n,784] -> host out [n,10]; synchronous (LeNet.forward's contract). */
int tz_lenet_forward(tz_lenet_t model, const float* images, int64_t n, float* out);
/* Device images (8-byte aligned) -> device out, asynchronous on `stream`. */
int tz_lenet_forward_device(tz_lenet_t model, const float* images, int64_t n, float* out,
                            tz_stream_t stream);

/* ---- .tenzor checkpoint files --------------------------------------------------------------
 * The reference's own format (src/io/tenzor_format.zig): 64-byte header, metadata JSON, 48-byte
 * index entries keyed by the FNV-1a hash of the tensor name, 4 KiB-aligned data.  The file is
 * memory-mapped read-only and tensor data is used in place (TenzorFile.open, 140-199). */
typedef struct tz_tenzor_s* tz_tenzor_t;
enum { /* DType, tenzor_format.zig:26-38 */
    TZ_DT_F32 = 0, TZ_DT_F16 = 1, TZ_DT_BF16 = 2, TZ_DT_F64 = 3, TZ_DT_I8 = 4, TZ_DT_I16 = 5,
    TZ_DT_I32 = 6, TZ_DT_I64 = 7, TZ_DT_U8 = 8, TZ_DT_U16 = 9, TZ_DT_U32 = 10, TZ_DT_U64 = 11
};
typedef struct { /* TensorEntry (tenzor_format.zig:84-104), data resolved into the mapping */
    uint64_t name_hash;
    int dtype, ndim;
    uint32_t shape[5];
    const void* data; /* valid until tz_tenzor_close */
    uint64_t bytes;
} tz_tenzor_entry;
/* hashName (tenzor_format.zig:107-114): FNV-1a 64 of the name's bytes. */
uint64_t tz_tenzor_hash_name(const char* name, size_t len);
/* TenzorFile.open / close.  TZ_EINVAL for a bad magic, version, or offsets outside the file. */
int tz_tenzor_open(const char* path, tz_tenzor_t* out);
int tz_tenzor_close(tz_tenzor_t file);
int64_t tz_tenzor_count(tz_tenzor_t file);
int tz_tenzor_entry_at(tz_tenzor_t file, int64_t index, tz_tenzor_entry* out);
/* getTensor (tenzor_format.zig:224-226); TZ_EMISSING when no entry has the name's hash. */
int tz_tenzor_find(tz_tenzor_t file, const char* name, tz_tenzor_entry* out);
/* The metadata JSON bytes (not NUL-terminated), valid until tz_tenzor_close. */
int tz_tenzor_metadata(tz_tenzor_t file, const char** json, uint64_t* len);
/* A LeNet training checkpoint (names conv1_weight .. fc3_bias, f32; main.zig:502-511, read back by
 * runEval 638-667) -> tz_lenet_load.  Every tensor is required (TZ_EMISSING otherwise). */
int tz_lenet_load_tenzor(tz_ctx_t ctx, const char* path, int variant, tz_lenet_t* out);
/* An Arctic checkpoint converted from safetensors (convertFromSafetensors, tenzor_format.zig:
 * 441-485: safetensors names and dtypes kept) -> tz_arctic_load, names resolved as in
 * tz_arctic_load_safetensors. */
int tz_arctic_load_tenzor(tz_ctx_t ctx, const char* path, int mode, tz_model_t* out);

/* ---- text -> device ids -> embeddings ------------------------------------------------------
 * The WordPiece tokenizer of src/io/tokenizer.zig (host code: string work) and the embed CLI's two
 * text paths of main.zig on the device.  Special ids are [UNK] 100, [CLS] 101, [SEP] 102
 * (tokenizer.zig:11-13) unless changed with tz_tokenizer_set_special. */
/* Tokenizer.init / deinit (tokenizer.zig:17-31). */
int tz_tokenizer_create(tz_tokenizer_t* out);
int tz_tokenizer_free(tz_tokenizer_t tok);
/* The public fields unk_id / cls_id / sep_id of Tokenizer (tokenizer.zig:11-13). */
int tz_tokenizer_set_special(tz_tokenizer_t tok, uint32_t unk_id, uint32_t cls_id, uint32_t sep_id);
/* Tokenizer.loadVocab / loadVocabFromBytes (tokenizer.zig:34-74): one token per line, id = line
 * index.  tz_tokenizer_put is vocab.put(token, id) (the reference's tests build vocabularies so). */
int tz_tokenizer_load_vocab(tz_tokenizer_t tok, const char* path);
int tz_tokenizer_load_vocab_bytes(tz_tokenizer_t tok, const char* data, int64_t len);
int tz_tokenizer_put(tz_tokenizer_t tok, const char* token, int64_t len, uint32_t id);
int tz_tokenizer_vocab_size(tz_tokenizer_t tok, int64_t* n);
/* Tokenizer.encode (tokenizer.zig:77-121): [CLS] ids [SEP] into out[cap] (cap >= 2); *n = count. */
int tz_tokenizer_encode(tz_tokenizer_t tok, const char* text, int64_t len, uint32_t* out, int64_t cap,
                        int64_t* n);
/* Tokenizer.encodeRaw (tokenizer.zig:123-200): ids without markers.  *n = the full count; out may
 * be NULL (size query); a non-NULL out with cap < *n fails with TZ_EINVAL. */
int tz_tokenizer_encode_raw(tz_tokenizer_t tok, const char* text, int64_t len, uint32_t* out, int64_t cap,
                            int64_t* n);
/* encode of every text into a max_len buffer (main.zig:939-950 uses [512]u32), packed as
 * (ids_packed, cu_seqlens[n_texts + 1]) for tz_arctic_forward; host threads for large batches. */
int tz_tokenizer_encode_batch(tz_tokenizer_t tok, const char* const* texts, const int64_t* lens, int n_texts,
                              int max_len, uint32_t* ids_packed, int32_t* cu_seqlens, int64_t cap_tokens);
/* Short texts (main.zig:934-980): encode each into 512 ids, forward the batch -> out[n_texts, 384]. */
int tz_arctic_embed_texts(tz_model_t model, tz_tokenizer_t tok, const char* const* texts, const int64_t* lens,
                          int n_texts, float* out);
/* Chunks a document of `tokens` raw ids takes (main.zig:806-809: 510-id chunks, 50 overlap; the
 * reference's count formula, whose last chunk can end before the document does, is kept). */
int64_t tz_doc_chunk_count(int64_t tokens);
/* Long documents (main.zig:796-925): encodeRaw, [CLS] chunk [SEP] per chunk, every chunk of every
 * document forwarded as one packed batch, then per document the mean of its chunk embeddings and
 * an L2 normalisation on the device -> out[n_docs, 384]. */
int tz_arctic_embed_documents(tz_model_t model, tz_tokenizer_t tok, const char* const* texts, const int64_t* lens,
                              int n_docs, float* out);

#ifdef __cplusplus
}
#endif
#endif /* TENZOR_CUDA_H */
