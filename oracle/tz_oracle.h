/*
 * tz_oracle.h -- CPU restatement of the reference (mattneel/tenzor, Zig) algorithms on the
 * Arctic-embed-xs encoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (tenzor_b200/, include/) links or calls this
 * library: it is the checker used by tests/, by __graft_entry__.smoke() and by bench.py's
 * cpu_baseline / --impl reference leg.
 *
 * Parity status: the reference cannot be built here (Zig toolchain absent; its BLAS dependency
 * "blazt" is not vendored).  The restatement is pinned against the reference's own unit-test
 * known answers (arctic.zig:1032-1057, softmax.zig:357-489, matmul.zig:985-1060,
 * layernorm.zig tests); end-to-end Arctic parity against HuggingFace is unpinned (the reference's
 * HF fixtures are not shipped).  The int8 W8A8 scheme is builder-defined (the reference only has
 * W8A32) and is therefore unpinned by construction.
 */
#ifndef TZ_ORACLE_H
#define TZ_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TZO_HIDDEN 384
#define TZO_LAYERS 6
#define TZO_HEADS 12
#define TZO_HEAD_DIM 32
#define TZO_FFN 1536
#define TZO_VOCAB 30522
#define TZO_MAX_POS 512
#define TZO_TYPES 2

/* forward modes */
#define TZO_MODE_F32 0   /* all-f32 forward, arctic.zig:874-898 */
#define TZO_MODE_W8A32 1 /* int8 weights, f32 activations, matmul_w8a32.zig:14-58 */
#define TZO_MODE_W8A8 2  /* builder-defined: per-token int8 activations, int32 accumulate; Q / K / V,
                          * the attention output and the GELU output held in f16 */

/* One transformer layer.  Matrices are PyTorch-layout [out, in] row-major.
 * f32 mode uses the *_w pointers; the int8 modes use *_q (int8) + *_s (IEEE half bits). */
typedef struct {
    const float *q_w, *k_w, *v_w, *o_w, *ffn1_w, *ffn2_w;
    const int8_t *q_q, *k_q, *v_q, *o_q, *ffn1_q, *ffn2_q;
    const uint16_t *q_s, *k_s, *v_s, *o_s, *ffn1_s, *ffn2_s;
    const float *q_b, *k_b, *v_b, *o_b, *ffn1_b, *ffn2_b;
    const float *ln1_g, *ln1_b, *ln2_g, *ln2_b;
} tzo_layer;

typedef struct {
    const float *word_w, *pos_w, *type_w; /* f32 tables */
    const int8_t *word_q, *pos_q;         /* int8 tables (quantize_arctic_xs.zig quantizes both) */
    const uint16_t *word_s, *pos_s;
    const float *emb_ln_g, *emb_ln_b;
    tzo_layer layers[TZO_LAYERS];
} tzo_arctic_weights;

/* ---- half-precision helpers (Zig @floatCast f32->f16 rounds to nearest even) ---- */
uint16_t tzo_f32_to_f16(float f);
float tzo_f16_to_f32(uint16_t h);
uint16_t tzo_f32_to_bf16(float f);
float tzo_bf16_to_f32(uint16_t h);

/* ---- element / row kernels ---- */
float tzo_gelu_model(float x); /* arctic.zig:750-756 */
float tzo_gelu_simd(float x);  /* simd.zig:297-303 scalar.gelu, tanh = 2*sigmoid(2x)-1 */
float tzo_unary(int op, float x);
void tzo_layernorm_rows(const float* x, const float* g, const float* b, float* y, int64_t rows,
                        int cols, float eps);
void tzo_softmax_rows(const float* x, const float* mask, float* y, int64_t rows, int cols);
void tzo_l2_normalize(float* v, int n);

/* ---- GEMMs ---- */
void tzo_sgemm_nt(const float* a, const float* b, float* c, int m, int k, int n);
void tzo_sgemm_nn(const float* a, const float* b, float* c, int m, int k, int n);
/* The attention core of selfAttention (arctic.zig:663-747) on packed sequences: qkv [T, 1152] rows
 * (Q | K | V, 12 heads of 32), cu_seqlens [batch + 1]; out [T, 384]. */
void tzo_attention_packed(const float* qkv, const int32_t* cu_seqlens, int batch, float* out);
void tzo_linear_f32(const float* x, const float* w, const float* bias, float* y, int m, int k,
                    int n);
void tzo_linear_w8a32(const float* x, const int8_t* wq, const uint16_t* s16, const float* bias,
                      float* y, int m, int k, int n);
void tzo_gemm_i8_i32(const int8_t* a, const int8_t* w, int32_t* c, int m, int k, int n);
void tzo_quantize_act_rows(const float* x, int8_t* q, float* s, int64_t rows, int cols);
void tzo_dequant_epilogue(const int32_t* acc, const float* a_s, const uint16_t* w_s16,
                          const float* bias, float* y, int m, int n);
void tzo_linear_w8a8(const float* x, const int8_t* wq, const uint16_t* s16, const float* bias,
                     float* y, int m, int k, int n);
void tzo_quantize_weight_rows(const float* w, int8_t* q, uint16_t* s16, int64_t rows, int cols);

/* ---- fusion patterns (codegen.zig) ---- */
void tzo_matmul_epilogue(const float* a, const float* b, int trans_b, const float* bias,
                         const int* ops, int n_ops, float* c, int m, int k, int n);
void tzo_ew_add_mul_exp(const float* a, const float* b_row, const float* c, float* out,
                        int64_t rows, int cols);
float tzo_reduce(int reduce_op, const int* pre_ops, int n_pre, const float* x, int64_t n);

/* ---- the model ---- */
/* ids_packed: concatenated token ids; cu_seqlens: B+1 prefix offsets; out: [B,384].
 * nthreads<=0 uses all cores (forwardBatchParallel semantics: one sequence per task). */
int tzo_arctic_forward(const tzo_arctic_weights* w, int mode, const uint32_t* ids_packed,
                       const int32_t* cu_seqlens, int B, float* out, int nthreads);
/* Layer dump for per-stage parity: writes the [T,384] hidden state after the embeddings
 * (stage 0) and after each layer (stage l+1) into dump[(stage)*T*384 ...] when dump != NULL. */
int tzo_arctic_forward_dump(const tzo_arctic_weights* w, int mode, const uint32_t* ids_packed,
                            const int32_t* cu_seqlens, int B, float* out, int nthreads,
                            float* dump);
const char* tzo_blas_status(void);

/* ---- LeNet-5 (lenet.zig), tz_oracle_lenet.c ---- */
#define TZO_LENET_REF 0  /* lenet.zig: conv1 valid, FC1 in 256, logits */
#define TZO_LENET_PAD2 1 /* benchmark variant: conv1 pad 2, FC1 in 400, softmax */
/* NHWC activations; conv weights [out, kh, kw, in]; FC weights [out, in]. */
typedef struct {
    const float *conv1_w, *conv1_b; /* [6,5,5,1], [6] */
    const float *conv2_w, *conv2_b; /* [16,5,5,6], [16] */
    const float *fc1_w, *fc1_b;     /* [120, 256 or 400], [120] */
    const float *fc2_w, *fc2_b;     /* [84,120], [84] */
    const float *fc3_w, *fc3_b;     /* [10,84], [10] */
} tzo_lenet_weights;
void tzo_lenet_forward_one(const tzo_lenet_weights* w, int variant, const float* img, float* out);
void tzo_lenet_forward(const tzo_lenet_weights* w, int variant, const float* images, int64_t n, float* out,
                       int nthreads);

#ifdef __cplusplus
}
#endif
#endif
