// tz_ops.cu -- op-level GEMM entry points of the C ABI (device pointers, async on a stream).
// Each routes to the tcgen05 GEMM of tz_gemm.cu with the matching fused epilogue; temporaries
// (f16 / int8 operand copies, scales, a transposed B) live in the context scratch arena.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tz_internal.h"

namespace tz {
int launch_f32_to_f16(tz_ctx_t ctx, const float* x, void* y, long long n, cudaStream_t s);
int launch_i8_to_f16(tz_ctx_t ctx, const int8_t* x, void* y, long long n, cudaStream_t s);
int launch_f16bits_to_f32(tz_ctx_t ctx, const uint16_t* x, float* y, long long n, cudaStream_t s);
int launch_quant_act(tz_ctx_t ctx, const float* x, int8_t* q, float* scale, long long rows, int cols, cudaStream_t s);
int launch_transpose(const float* x, float* y, int rows, int cols, cudaStream_t s);

static size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
}  // namespace tz

using namespace tz;

extern "C" {

int tz_linear_f32(tz_ctx_t ctx, const float* x, const float* w, const float* bias, const float* residual, float* y,
                  int m, int k, int n, tz_stream_t stream) {
    TZ_CHECK(ctx && x && w && y && m >= 0 && k > 0 && n > 0, TZ_EINVAL, "tz_linear_f32: bad arguments");
    GemmArgs g;
    g.kind = KIND_TF32;
    g.a = x; g.lda = k; g.b = w; g.ldb = k; g.M = m; g.N = n; g.K = k;
    g.bias = bias; g.residual = residual; g.ldr = n; g.out = y; g.ldo = n; g.out_type = OUT_F32;
    return launch_gemm(ctx, g, pick_stream(ctx, stream));
}

int tz_linear_w8a32(tz_ctx_t ctx, const float* x, const int8_t* wq, const uint16_t* scale_f16, const float* bias,
                    float* y, int m, int k, int n, tz_stream_t stream) {
    TZ_CHECK(ctx && x && wq && scale_f16 && bias && y && m >= 0 && k > 0 && n > 0, TZ_EINVAL,
             "tz_linear_w8a32: bad arguments");
    if (m == 0) return TZ_OK;
    TZ_CHECK(k % 8 == 0, TZ_EINVAL, "tz_linear_w8a32: k must be a multiple of 8 (k=%d)", k);
    cudaStream_t s = pick_stream(ctx, stream);
    const size_t bx = align256(sizeof(__half) * static_cast<size_t>(m) * k);
    const size_t bw = align256(sizeof(__half) * static_cast<size_t>(n) * k);
    const size_t bs = align256(sizeof(float) * n);
    void* base = nullptr;
    int rc = scratch_reserve(ctx, bx + bw + bs, &base);
    if (rc) return rc;
    char* p = static_cast<char*>(base);
    void* xh = p;
    void* wh = p + bx;
    float* sc = reinterpret_cast<float*>(p + bx + bw);
    if ((rc = launch_f32_to_f16(ctx, x, xh, static_cast<long long>(m) * k, s))) return rc;
    if ((rc = launch_i8_to_f16(ctx, wq, wh, static_cast<long long>(n) * k, s))) return rc;
    if ((rc = launch_f16bits_to_f32(ctx, scale_f16, sc, n, s))) return rc;
    GemmArgs g;
    g.kind = KIND_F16;
    g.a = xh; g.lda = k; g.b = wh; g.ldb = k; g.M = m; g.N = n; g.K = k;
    g.col_scale = sc; g.bias = bias; g.out = y; g.ldo = n; g.out_type = OUT_F32;
    return launch_gemm(ctx, g, s);
}

int tz_linear_w8a8(tz_ctx_t ctx, const float* x, const int8_t* wq, const uint16_t* scale_f16, const float* bias,
                   float* y, int m, int k, int n, tz_stream_t stream) {
    TZ_CHECK(ctx && x && wq && scale_f16 && bias && y && m >= 0 && k > 0 && n > 0, TZ_EINVAL,
             "tz_linear_w8a8: bad arguments");
    if (m == 0) return TZ_OK;
    TZ_CHECK(k % 16 == 0, TZ_EINVAL, "tz_linear_w8a8: k must be a multiple of 16 (k=%d)", k);
    cudaStream_t s = pick_stream(ctx, stream);
    const size_t bq = align256(static_cast<size_t>(m) * k);
    const size_t bxs = align256(sizeof(float) * m);
    const size_t bs = align256(sizeof(float) * n);
    void* base = nullptr;
    int rc = scratch_reserve(ctx, bq + bxs + bs, &base);
    if (rc) return rc;
    char* p = static_cast<char*>(base);
    int8_t* xq = reinterpret_cast<int8_t*>(p);
    float* xs = reinterpret_cast<float*>(p + bq);
    float* sc = reinterpret_cast<float*>(p + bq + bxs);
    if ((rc = launch_quant_act(ctx, x, xq, xs, m, k, s))) return rc;
    if ((rc = launch_f16bits_to_f32(ctx, scale_f16, sc, n, s))) return rc;
    GemmArgs g;
    g.kind = KIND_I8;
    g.a = xq; g.lda = k; g.b = wq; g.ldb = k; g.M = m; g.N = n; g.K = k;
    g.row_scale = xs; g.col_scale = sc; g.bias = bias; g.out = y; g.ldo = n; g.out_type = OUT_F32;
    return launch_gemm(ctx, g, s);
}

int tz_gemm_i8_i32(tz_ctx_t ctx, const int8_t* a, const int8_t* w, int32_t* c, int m, int k, int n, tz_stream_t stream) {
    TZ_CHECK(ctx && a && w && c && m >= 0 && k > 0 && n > 0, TZ_EINVAL, "tz_gemm_i8_i32: bad arguments");
    GemmArgs g;
    g.kind = KIND_I8;
    g.a = a; g.lda = k; g.b = w; g.ldb = k; g.M = m; g.N = n; g.K = k;
    g.out = c; g.ldo = n; g.out_type = OUT_I32;
    return launch_gemm(ctx, g, pick_stream(ctx, stream));
}

int tz_matmul_epilogue(tz_ctx_t ctx, const float* a, const float* b, int trans_b, const float* bias, const int* ops,
                       int n_ops, float* c, int m, int k, int n, tz_stream_t stream) {
    TZ_CHECK(ctx && a && b && c && m >= 0 && k > 0 && n > 0 && n_ops >= 0 && n_ops <= 8 && (n_ops == 0 || ops),
             TZ_EINVAL, "tz_matmul_epilogue: bad arguments");
    for (int i = 0; i < n_ops; ++i)
        TZ_CHECK(ops[i] >= TZ_OP_ADD && ops[i] <= TZ_OP_LAST_UNARY, TZ_EINVAL, "tz_matmul_epilogue: bad op %d", ops[i]);
    cudaStream_t s = pick_stream(ctx, stream);
    GemmArgs g;
    g.kind = KIND_TF32;
    g.a = a; g.lda = k; g.b = b; g.ldb = k; g.M = m; g.N = n; g.K = k;
    if (!trans_b) {
        if (n % 4 == 0) {  // B [k, n] read N-major by the MMA (16-byte rows for TMA)
            g.b_mn = true;
            g.ldb = n;
        } else {
            void* t = nullptr;
            int rc = scratch_reserve(ctx, sizeof(float) * static_cast<size_t>(k) * n, &t);
            if (rc) return rc;
            if ((rc = launch_transpose(b, static_cast<float*>(t), k, n, s))) return rc;  // [k,n] -> [n,k]
            g.b = static_cast<const float*>(t);
        }
    }
    g.out = c; g.ldo = n; g.out_type = OUT_F32;
    // Chains the fixed epilogue does natively (bias, then one activation) skip the op interpreter.
    const bool has_add = n_ops >= 1 && ops[0] == TZ_OP_ADD;
    const int act = n_ops == (has_add ? 2 : 1) ? ops[n_ops - 1] : 0;
    if (n_ops == 0 || (n_ops == 1 && has_add) || (n_ops <= 2 && (act == TZ_OP_GELU || act == TZ_OP_RELU))) {
        g.bias = has_add ? bias : nullptr;
        g.gelu = act == TZ_OP_GELU ? 2 : act == TZ_OP_RELU ? 3 : 0;
        return launch_gemm(ctx, g, s);
    }
    g.bias = bias;
    g.n_ops = n_ops;
    for (int i = 0; i < n_ops; ++i) g.ops[i] = ops[i];
    return launch_gemm(ctx, g, s);
}

}  // extern "C"
