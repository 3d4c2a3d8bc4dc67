/*
 * tz_oracle.c -- CPU restatement of the reference (mattneel/tenzor) Arctic-embed-xs forward and
 * the kernels it calls.  TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg as the checker; never linked into the product.
 *
 * Every function cites the reference file:line it restates (paths relative to the reference
 * project root).  Compiled with -ffp-contract=off so that a*b+c is two IEEE roundings, as in the
 * Zig source (Zig does not contract by default).
 *
 * Parity: pinned against the reference's unit-test known answers (see tests/test_oracle_kats.py);
 * the end-to-end HF fixtures of the reference are not shipped, so full-model parity against HF is
 * unpinned; the W8A8 scheme is builder-defined (unpinned by construction).
 */
#include "tz_oracle.h"

#include <dlfcn.h>
#include <stdio.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------------ */
/* half / bfloat16 conversions                                                                 */
/* ------------------------------------------------------------------------------------------ */

/* IEEE binary16 from binary32, round to nearest even (Zig @floatCast semantics). */
uint16_t tzo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ex = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (ex == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    int e = (int)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t half = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1u))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++; /* may carry into exponent: ok */
    return (uint16_t)h;
}

float tzo_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t x;
    if (ex == 0) {
        if (man == 0) {
            x = sign;
        } else {
            int e = -1;
            do {
                e++;
                man <<= 1;
            } while (!(man & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (ex == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((ex + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

uint16_t tzo_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7fffu + lsb;
    return (uint16_t)(x >> 16);
}

float tzo_bf16_to_f32(uint16_t h) {
    uint32_t x = (uint32_t)h << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------------------------------------ */
/* Optional CBLAS, loaded at run time like blas.zig:140-260 (env TENZOR_BLAS_LIB).              */
/* ------------------------------------------------------------------------------------------ */
static void* dlopen_with_siblings(const char* path, int depth);
static void* dlopen_with_siblings_global(const char* path, int depth) {
    void* h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
    if (h || depth > 6) return h;
    const char* err = dlerror();
    if (!err || !strstr(err, "cannot open shared object file")) return NULL;
    const char* colon = strchr(err, ':');
    char dep[256];
    size_t n = colon ? (size_t)(colon - err) : 0;
    if (n == 0 || n >= sizeof dep) return NULL;
    memcpy(dep, err, n);
    dep[n] = 0;
    char dir[800];
    if (strlen(path) >= sizeof dir) return NULL;
    memcpy(dir, path, strlen(path) + 1);
    char* slash = strrchr(dir, '/');
    if (!slash) return NULL;
    *slash = 0;
    char full[1200];
    snprintf(full, sizeof full, "%s/%s", dir, dep);
    if (!dlopen_with_siblings_global(full, depth + 1)) return NULL;
    return dlopen_with_siblings_global(path, depth + 1);
}

typedef void (*cblas_sgemm_fn)(int, int, int, int, int, int, float, const float*, int,
                               const float*, int, float, float*, int);
static cblas_sgemm_fn g_sgemm = NULL;
static int g_blas_tried = 0;
static char g_blas_status[512] = "not loaded";

/* dlopen that also resolves sibling dependencies of a bundled library (e.g. an OpenBLAS shipped with
 * its own libgfortran / libquadmath next to it and no RPATH): on "X: cannot open shared object
 * file", X is loaded from the library's directory with RTLD_GLOBAL and the open is retried. */
static void* dlopen_with_siblings(const char* path, int depth) {
    void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (h || depth > 6) return h;
    const char* err = dlerror();
    if (!err) return NULL;
    const char* colon = strchr(err, ':');
    if (!colon || !strstr(err, "cannot open shared object file")) return NULL;
    char dep[256];
    size_t n = (size_t)(colon - err);
    if (n == 0 || n >= sizeof dep) return NULL;
    memcpy(dep, err, n);
    dep[n] = 0;
    char dir[800];
    if (strlen(path) >= sizeof dir) return NULL;
    memcpy(dir, path, strlen(path) + 1);
    char* slash = strrchr(dir, '/');
    if (!slash) return NULL;
    *slash = 0;
    char full[1200];
    snprintf(full, sizeof full, "%s/%s", dir, dep);
    if (!dlopen_with_siblings_global(full, depth + 1)) return NULL;
    return dlopen_with_siblings(path, depth + 1);
}

static void blas_init(void) {
    if (g_blas_tried) return;
#pragma omp critical(tzo_blas)
    {
        if (!g_blas_tried) {
            /* TENZOR_BLAS_LIB first (blas.zig:199-204), else the library names of the reference's
             * Linux candidate list (blas.zig:206-220) through the dynamic loader's search path. */
            static const char* const kCandidates[] = {
                "libopenblas.so.0", "libopenblas.so", "libopenblas64_.so.0", "libopenblas64_.so",
                "libopenblas64.so.0", "libopenblas64.so", "libopenblasp.so.0", "libopenblasp.so",
                "libcblas.so.3", "libcblas.so", "libblas.so.3", "libblas.so", "libmkl_rt.so"};
            const char* env = getenv("TENZOR_BLAS_LIB");
            const int n_cand = (int)(sizeof kCandidates / sizeof kCandidates[0]);
            int tried_env = 0;
            for (int i = (env && *env) ? -1 : 0; i < n_cand && !g_sgemm; i++) {
                const char* path = i < 0 ? env : kCandidates[i];
                void* h = dlopen_with_siblings(path, 0);
                if (i < 0) tried_env = 1;
                if (!h) {
                    if (i < 0) snprintf(g_blas_status, sizeof g_blas_status, "dlopen failed: %s", path);
                    continue;
                }
                g_sgemm = (cblas_sgemm_fn)dlsym(h, "cblas_sgemm");
                if (!g_sgemm) continue;
                void (*set_threads)(int) = (void (*)(int))dlsym(h, "openblas_set_num_threads");
                if (set_threads) set_threads(1); /* parallelism is per sequence */
                snprintf(g_blas_status, sizeof g_blas_status, "%s", path);
            }
            if (!g_sgemm && !tried_env)
                snprintf(g_blas_status, sizeof g_blas_status, "no CBLAS found (restated loops)");
            __atomic_store_n(&g_blas_tried, 1, __ATOMIC_RELEASE);
        }
    }
}

const char* tzo_blas_status(void) {
    blas_init();
    return g_blas_status;
}

/* ------------------------------------------------------------------------------------------ */
/* GEMMs                                                                                       */
/* ------------------------------------------------------------------------------------------ */
#define CBLAS_MIN_SIZE 8 /* matmul.zig:19 */

/* C[m,n] = A[m,k] * B[n,k]^T.  matmulTransposeB, matmul.zig:54-77 (CBLAS when loadable and all
 * dims >= 8, else the pure loop of matmul.zig:80-104; partial sums in 16 lanes). */
void tzo_sgemm_nt(const float* a, const float* b, float* c, int m, int k, int n) {
    blas_init();
    if (g_sgemm && m >= CBLAS_MIN_SIZE && n >= CBLAS_MIN_SIZE && k >= CBLAS_MIN_SIZE) {
        g_sgemm(101, 111, 112, m, n, k, 1.0f, a, k, b, k, 0.0f, c, n);
        return;
    }
    for (int i = 0; i < m; i++) {
        const float* ar = a + (int64_t)i * k;
        for (int j = 0; j < n; j++) {
            const float* br = b + (int64_t)j * k;
            float lane[16] = {0};
            int kk = 0;
            for (; kk + 16 <= k; kk += 16)
                for (int l = 0; l < 16; l++) lane[l] += ar[kk + l] * br[kk + l];
            float s = 0.0f;
            for (int l = 0; l < 16; l++) s += lane[l];
            for (; kk < k; kk++) s += ar[kk] * br[kk];
            c[(int64_t)i * n + j] = s;
        }
    }
}

/* C[m,n] = A[m,k] * B[k,n].  matmulTiled, matmul.zig:107-165. */
void tzo_sgemm_nn(const float* a, const float* b, float* c, int m, int k, int n) {
    blas_init();
    if (g_sgemm && m >= CBLAS_MIN_SIZE && n >= CBLAS_MIN_SIZE && k >= CBLAS_MIN_SIZE) {
        g_sgemm(101, 111, 111, m, n, k, 1.0f, a, k, b, n, 0.0f, c, n);
        return;
    }
    memset(c, 0, sizeof(float) * (size_t)m * n);
    for (int i = 0; i < m; i++)
        for (int kk = 0; kk < k; kk++) {
            float av = a[(int64_t)i * k + kk];
            const float* br = b + (int64_t)kk * n;
            float* cr = c + (int64_t)i * n;
            for (int j = 0; j < n; j++) cr[j] += av * br[j];
        }
}

/* linearProjection f32 arm, arctic.zig:599-620: matmulTransposeB then a bias loop. */
void tzo_linear_f32(const float* x, const float* w, const float* bias, float* y, int m, int k,
                    int n) {
    tzo_sgemm_nt(x, w, y, m, k, n);
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) y[(int64_t)i * n + j] += bias[j];
}

/* matmulTransposeB_f32_i8_rowScale_bias, matmul_w8a32.zig:14-58: per (i,j) an f32 dot of the
 * activation row with the int8 weight row widened to f32, then sum*f32(scale[j]) + bias[j]. */
void tzo_linear_w8a32(const float* x, const int8_t* wq, const uint16_t* s16, const float* bias,
                      float* y, int m, int k, int n) {
    if (m == 0 || n == 0) return;
    for (int i = 0; i < m; i++) {
        const float* ar = x + (int64_t)i * k;
        for (int j = 0; j < n; j++) {
            const int8_t* wr = wq + (int64_t)j * k;
            float lane[16] = {0};
            int kk = 0;
            for (; kk + 16 <= k; kk += 16)
                for (int l = 0; l < 16; l++) lane[l] += ar[kk + l] * (float)wr[kk + l];
            float s = 0.0f;
            for (int l = 0; l < 16; l++) s += lane[l];
            for (; kk < k; kk++) s += ar[kk] * (float)wr[kk];
            y[(int64_t)i * n + j] = s * tzo_f16_to_f32(s16[j]) + bias[j];
        }
    }
}

/* Exact int8 x int8 -> int32 GEMM, C[m,n] = A[m,k] * W[n,k]^T. */
void tzo_gemm_i8_i32(const int8_t* a, const int8_t* w, int32_t* c, int m, int k, int n) {
    for (int i = 0; i < m; i++) {
        const int8_t* ar = a + (int64_t)i * k;
        for (int j = 0; j < n; j++) {
            const int8_t* wr = w + (int64_t)j * k;
            int32_t s = 0;
            for (int kk = 0; kk < k; kk++) s += (int32_t)ar[kk] * (int32_t)wr[kk];
            c[(int64_t)i * n + j] = s;
        }
    }
}

/* Builder-defined per-token symmetric activation quantisation (the reference has none; it mirrors
 * the weight rule of quantize_arctic_xs.zig:94-115 without the f16 rounding of the scale):
 *   amax = max|x_row|;  s = amax/127 (s = 1 when amax == 0);  q = clamp(round(x*(1/s)),-127,127)
 * round() is half-away-from-zero like Zig @round. */
void tzo_quantize_act_rows(const float* x, int8_t* q, float* s, int64_t rows, int cols) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * cols;
        float amax = 0.0f;
        for (int c = 0; c < cols; c++) {
            float a = fabsf(xr[c]);
            if (a > amax) amax = a;
        }
        float sc = (amax == 0.0f) ? 1.0f : amax / 127.0f;
        float inv = 1.0f / sc;
        s[r] = sc;
        for (int c = 0; c < cols; c++) {
            float qf = roundf(xr[c] * inv);
            int qi = (int)qf;
            if (qi > 127) qi = 127;
            if (qi < -127) qi = -127;
            q[r * cols + c] = (int8_t)qi;
        }
    }
}

/* W8A8 epilogue: y = float(acc) * (a_s[row] * f32(w_s[col])) + bias[col], each op one rounding. */
void tzo_dequant_epilogue(const int32_t* acc, const float* a_s, const uint16_t* w_s16,
                          const float* bias, float* y, int m, int n) {
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) {
            float sc = a_s[i] * tzo_f16_to_f32(w_s16[j]);
            float v = (float)acc[(int64_t)i * n + j] * sc;
            y[(int64_t)i * n + j] = v + bias[j];
        }
}

void tzo_linear_w8a8(const float* x, const int8_t* wq, const uint16_t* s16, const float* bias,
                     float* y, int m, int k, int n) {
    int8_t* xq = (int8_t*)malloc((size_t)m * k);
    float* xs = (float*)malloc(sizeof(float) * (size_t)(m > 0 ? m : 1));
    int32_t* acc = (int32_t*)malloc(sizeof(int32_t) * (size_t)m * n + 4);
    tzo_quantize_act_rows(x, xq, xs, m, k);
    tzo_gemm_i8_i32(xq, wq, acc, m, k, n);
    tzo_dequant_epilogue(acc, xs, s16, bias, y, m, n);
    free(xq);
    free(xs);
    free(acc);
}

/* quantize_arctic_xs.zig:94-115: per row max|w| -> s = max/127 (1 if 0) -> f16(s);
 * q = clamp(round(w * (1/f32(f16 s))), -127, 127). */
void tzo_quantize_weight_rows(const float* w, int8_t* q, uint16_t* s16, int64_t rows, int cols) {
    for (int64_t r = 0; r < rows; r++) {
        const float* wr = w + r * cols;
        float max_abs = 0.0f;
        for (int c = 0; c < cols; c++) {
            float a = fabsf(wr[c]);
            if (a > max_abs) max_abs = a;
        }
        float s = (max_abs == 0.0f) ? 1.0f : max_abs / 127.0f;
        uint16_t h = tzo_f32_to_f16(s);
        s16[r] = h;
        float inv = 1.0f / tzo_f16_to_f32(h);
        for (int c = 0; c < cols; c++) {
            float qf = roundf(wr[c] * inv);
            int qi = (int)qf;
            if (qi > 127) qi = 127;
            if (qi < -127) qi = -127;
            q[r * cols + c] = (int8_t)qi;
        }
    }
}

/* ------------------------------------------------------------------------------------------ */
/* Row kernels                                                                                 */
/* ------------------------------------------------------------------------------------------ */

/* layerNormLastDim, layernorm.zig:26-116: mean = sum/N; var = sum((x-mean)^2)/N;
 * inv_std = 1/sqrt(var+eps); y = (x-mean)*inv_std*gamma + beta.  In-place safe. */
void tzo_layernorm_rows(const float* x, const float* g, const float* b, float* y, int64_t rows,
                        int cols, float eps) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * cols;
        float* yr = y + r * cols;
        float sum = 0.0f;
        for (int c = 0; c < cols; c++) sum += xr[c];
        float mean = sum / (float)cols;
        float vs = 0.0f;
        for (int c = 0; c < cols; c++) {
            float d = xr[c] - mean;
            vs += d * d;
        }
        float var = vs / (float)cols;
        float inv_std = 1.0f / sqrtf(var + eps);
        for (int c = 0; c < cols; c++) yr[c] = (xr[c] - mean) * inv_std * g[c] + b[c];
    }
}

/* softmaxRow, softmax.zig:56-155: m = max(x+mask); e = exp(x+mask-m); y = e * (1/sum e).
 * mask is additive (e.g. -1e9 or -inf), NULL for none. */
void tzo_softmax_rows(const float* x, const float* mask, float* y, int64_t rows, int cols) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * cols;
        const float* mr = mask ? mask + r * cols : NULL;
        float* yr = y + r * cols;
        if (cols == 0) continue;
        float mx = -INFINITY;
        for (int c = 0; c < cols; c++) {
            float v = mr ? xr[c] + mr[c] : xr[c];
            if (v > mx) mx = v;
        }
        float sum = 0.0f;
        for (int c = 0; c < cols; c++) {
            float v = mr ? xr[c] + mr[c] : xr[c];
            float e = expf(v - mx);
            yr[c] = e;
            sum += e;
        }
        float inv = 1.0f / sum;
        for (int c = 0; c < cols; c++) yr[c] *= inv;
    }
}

/* l2Normalize, arctic.zig:851-863. */
void tzo_l2_normalize(float* v, int n) {
    float nsq = 0.0f;
    for (int i = 0; i < n; i++) nsq += v[i] * v[i];
    float norm = sqrtf(nsq);
    if (norm > 1e-12f)
        for (int i = 0; i < n; i++) v[i] /= norm;
}

/* gelu, arctic.zig:750-756 (std.math.tanh). */
float tzo_gelu_model(float x) {
    const float k0 = 0.7978845608f;
    const float k1 = 0.044715f;
    float inner = k0 * (x + k1 * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

static float sigmoid_ref(float x) { return 1.0f / (1.0f + expf(-x)); } /* simd.zig:252-254 */

/* scalar.gelu, simd.zig:297-303, with tanh = 2*sigmoid(2x)-1 (simd.zig:245-248). */
float tzo_gelu_simd(float x) {
    const float k0 = 0.7978845608028654f;
    const float k1 = 0.044715f;
    float x3 = x * x * x;
    float inner = k0 * (x + k1 * x3);
    float t = 2.0f * sigmoid_ref(2.0f * inner) - 1.0f;
    return 0.5f * x * (1.0f + t);
}

/* Unary op table of codegen.zig:228-244 / simd.zig scalar ops.  Op codes match
 * include/tenzor_cuda.h TZ_OP_*. */
float tzo_unary(int op, float x) {
    switch (op) {
        case 2: return x > 0.0f ? x : 0.0f;                   /* relu */
        case 3: return tzo_gelu_simd(x);                      /* gelu */
        case 4: return sigmoid_ref(x);                        /* sigmoid */
        case 5: return 2.0f * sigmoid_ref(2.0f * x) - 1.0f;   /* tanh */
        case 6: return expf(x);                               /* exp */
        case 7: return -x;                                    /* neg */
        case 8: return fabsf(x);                              /* abs */
        case 9: return x * sigmoid_ref(x);                    /* silu */
        case 10: return logf(x);                              /* log */
        case 11: return sqrtf(x);                             /* sqrt */
        case 12: return 1.0f / sqrtf(x);                      /* rsqrt */
        case 13: return sinf(x);                              /* sin */
        case 14: return cosf(x);                              /* cos */
        case 15: return erff(x);                              /* erf (ONNX Erf) */
        case 16: return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); /* ONNX Gelu */
        default: return x;
    }
}

/* FusedMatmulEpilogueKernel.apply, codegen.zig:78-147: matmulTiled (A@B, or A@B^T when trans_b)
 * then, per element, the epilogue ops in chain order; op 1 (add) adds bias[j]. */
void tzo_matmul_epilogue(const float* a, const float* b, int trans_b, const float* bias,
                         const int* ops, int n_ops, float* c, int m, int k, int n) {
    if (trans_b)
        tzo_sgemm_nt(a, b, c, m, k, n);
    else
        tzo_sgemm_nn(a, b, c, m, k, n);
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) {
            float v = c[(int64_t)i * n + j];
            for (int o = 0; o < n_ops; o++) {
                if (ops[o] == 1) {
                    if (bias) v += bias[j];
                } else {
                    v = tzo_unary(ops[o], v);
                }
            }
            c[(int64_t)i * n + j] = v;
        }
}

/* executor.evalInto of exp(mul(add(a, b), c)) with b broadcast along rows
 * (executor.zig:114-197 broadcast rule, elementwise.zig:13-66 op order). */
void tzo_ew_add_mul_exp(const float* a, const float* b_row, const float* c, float* out,
                        int64_t rows, int cols) {
    for (int64_t r = 0; r < rows; r++)
        for (int j = 0; j < cols; j++) {
            int64_t i = r * cols + j;
            float t = a[i] + b_row[j];
            t = t * c[i];
            out[i] = expf(t);
        }
}

/* FusedReduceKernel.apply, codegen.zig:151-205: reduce(pre_ops(x)); op codes TZ_RED_*:
 * 0 sum, 1 mean, 2 prod, 3 max, 4 min. */
float tzo_reduce(int reduce_op, const int* pre_ops, int n_pre, const float* x, int64_t n) {
    float acc;
    switch (reduce_op) {
        case 2: acc = 1.0f; break;
        case 3: acc = -INFINITY; break;
        case 4: acc = INFINITY; break;
        default: acc = 0.0f;
    }
    if (n == 0) return acc;
    double dacc = 0.0; /* sums in double: the oracle is the exact-ish reference value */
    for (int64_t i = 0; i < n; i++) {
        float v = x[i];
        for (int o = 0; o < n_pre; o++) v = tzo_unary(pre_ops[o], v);
        switch (reduce_op) {
            case 0:
            case 1: dacc += v; break;
            case 2: acc *= v; break;
            case 3: acc = v > acc ? v : acc; break;
            case 4: acc = v < acc ? v : acc; break;
        }
    }
    if (reduce_op == 0) acc = (float)dacc;
    if (reduce_op == 1) acc = (float)(dacc / (double)n);
    return acc;
}

/* ------------------------------------------------------------------------------------------ */
/* The model                                                                                   */
/* ------------------------------------------------------------------------------------------ */
#define H TZO_HIDDEN
#define F TZO_FFN
#define EPS 1e-12f /* arctic.zig:37 */

typedef struct {
    float *hidden, *qkv, *scores, *attn_out, *ffn, *tmp, *qh, *kh, *vh, *oh, *enc_in, *enc_out,
        *layer_in;
} scratch_t;

static void scratch_alloc(scratch_t* s, int L) {
    s->hidden = malloc(sizeof(float) * (size_t)L * H);
    s->qkv = malloc(sizeof(float) * (size_t)3 * L * H);
    s->scores = malloc(sizeof(float) * (size_t)L * L);
    s->attn_out = malloc(sizeof(float) * (size_t)L * H);
    s->ffn = malloc(sizeof(float) * (size_t)L * F);
    s->tmp = malloc(sizeof(float) * (size_t)L * H);
    s->qh = malloc(sizeof(float) * (size_t)L * 32);
    s->kh = malloc(sizeof(float) * (size_t)L * 32);
    s->vh = malloc(sizeof(float) * (size_t)L * 32);
    s->oh = malloc(sizeof(float) * (size_t)L * 32);
    s->enc_in = malloc(sizeof(float) * (size_t)L * H);
    s->enc_out = malloc(sizeof(float) * (size_t)L * H);
    s->layer_in = malloc(sizeof(float) * (size_t)L * H);
}

static void scratch_free(scratch_t* s) {
    free(s->hidden); free(s->qkv); free(s->scores); free(s->attn_out); free(s->ffn);
    free(s->tmp); free(s->qh); free(s->kh); free(s->vh); free(s->oh); free(s->enc_in);
    free(s->enc_out); free(s->layer_in);
}

/* linearProjection, arctic.zig:599-635, dispatching on the forward mode. */
static void linear(int mode, const float* x, const float* w, const int8_t* wq, const uint16_t* ws,
                   const float* b, float* y, int L, int k, int n) {
    if (mode == TZO_MODE_F32)
        tzo_linear_f32(x, w, b, y, L, k, n);
    else if (mode == TZO_MODE_W8A32)
        tzo_linear_w8a32(x, wq, ws, b, y, L, k, n);
    else
        tzo_linear_w8a8(x, wq, ws, b, y, L, k, n);
}

/* writeMatWeightRow / addMatWeightRow, arctic.zig:484-539. */
static void emb_row(float* dst, const float* wf, const int8_t* wq, const uint16_t* ws, int row,
                    int add) {
    if (wf) {
        const float* src = wf + (int64_t)row * H;
        for (int i = 0; i < H; i++) dst[i] = add ? dst[i] + src[i] : src[i];
    } else {
        const int8_t* src = wq + (int64_t)row * H;
        float s = tzo_f16_to_f32(ws[row]);
        for (int i = 0; i < H; i++) {
            float v = (float)src[i] * s;
            dst[i] = add ? dst[i] + v : v;
        }
    }
}

/* Rounds n values to IEEE half and back: the W8A8 scheme stores Q / K / V, the attention output and
 * the GELU output as f16 before they are used (and, for the latter two, quantised per token). */
static void round_f16(float* x, size_t n) {
    for (size_t i = 0; i < n; i++) x[i] = tzo_f16_to_f32(tzo_f32_to_f16(x[i]));
}

/* The per-head core of selfAttention, arctic.zig:663-747: for each head, scores = Q_h K_h^T / sqrt(32),
 * row softmax (max, exp, sum, divide), P V_h.  Q / K / V row t at q / k / v + t * ld. */
static void attend_heads(const float* q, const float* k, const float* v, size_t ld, float* attn_out,
                         scratch_t* s, int L) {
    const float scale = 1.0f / sqrtf(32.0f);
    for (int h = 0; h < TZO_HEADS; h++) {
        int off = h * 32;
        for (int t = 0; t < L; t++) {
            memcpy(s->qh + t * 32, q + (size_t)t * ld + off, 32 * sizeof(float));
            memcpy(s->kh + t * 32, k + (size_t)t * ld + off, 32 * sizeof(float));
            memcpy(s->vh + t * 32, v + (size_t)t * ld + off, 32 * sizeof(float));
        }
        tzo_sgemm_nt(s->qh, s->kh, s->scores, L, 32, L);
        for (int i = 0; i < L * L; i++) s->scores[i] *= scale;
        for (int qi = 0; qi < L; qi++) { /* arctic.zig:683-703: divide by the sum */
            float* row = s->scores + (size_t)qi * L;
            float mx = row[0];
            for (int j = 1; j < L; j++)
                if (row[j] > mx) mx = row[j];
            float sum = 0.0f;
            for (int j = 0; j < L; j++) {
                row[j] = expf(row[j] - mx);
                sum += row[j];
            }
            for (int j = 0; j < L; j++) row[j] /= sum;
        }
        tzo_sgemm_nn(s->scores, s->vh, s->oh, L, L, 32);
        for (int t = 0; t < L; t++)
            memcpy(attn_out + (size_t)t * H + off, s->oh + t * 32, 32 * sizeof(float));
    }
}

/* selfAttention, arctic.zig:639-747. */
static void self_attention(int mode, const tzo_layer* lw, float* out, const float* in,
                           scratch_t* s, int L) {
    float* q = s->qkv;
    float* k = s->qkv + (size_t)L * H;
    float* v = s->qkv + (size_t)2 * L * H;
    linear(mode, in, lw->q_w, lw->q_q, lw->q_s, lw->q_b, q, L, H, H);
    linear(mode, in, lw->k_w, lw->k_q, lw->k_s, lw->k_b, k, L, H, H);
    linear(mode, in, lw->v_w, lw->v_q, lw->v_s, lw->v_b, v, L, H, H);
    if (mode == TZO_MODE_W8A8) round_f16(s->qkv, (size_t)3 * L * H);
    attend_heads(q, k, v, H, s->attn_out, s, L);
    if (mode == TZO_MODE_W8A8) round_f16(s->attn_out, (size_t)L * H);
    linear(mode, s->attn_out, lw->o_w, lw->o_q, lw->o_s, lw->o_b, s->tmp, L, H, H);
    for (int i = 0; i < L * H; i++) out[i] = in[i] + s->tmp[i];
    tzo_layernorm_rows(out, lw->ln1_g, lw->ln1_b, out, L, H, EPS);
}

void tzo_attention_packed(const float* qkv, const int32_t* cu_seqlens, int batch, float* out) {
    for (int b = 0; b < batch; b++) {
        const int L = cu_seqlens[b + 1] - cu_seqlens[b];
        if (L <= 0) continue;
        scratch_t s;
        scratch_alloc(&s, L);
        const float* rows = qkv + (size_t)cu_seqlens[b] * 3 * H;
        attend_heads(rows, rows + H, rows + 2 * H, (size_t)3 * H, out + (size_t)cu_seqlens[b] * H, &s, L);
        scratch_free(&s);
    }
}

/* feedForward, arctic.zig:760-810. */
static void feed_forward(int mode, const tzo_layer* lw, float* out, const float* in, scratch_t* s,
                         int L) {
    linear(mode, in, lw->ffn1_w, lw->ffn1_q, lw->ffn1_s, lw->ffn1_b, s->ffn, L, H, F);
    for (int i = 0; i < L * F; i++) s->ffn[i] = tzo_gelu_model(s->ffn[i]);
    if (mode == TZO_MODE_W8A8) round_f16(s->ffn, (size_t)L * F);
    linear(mode, s->ffn, lw->ffn2_w, lw->ffn2_q, lw->ffn2_s, lw->ffn2_b, s->tmp, L, F, H);
    for (int i = 0; i < L * H; i++) out[i] = in[i] + s->tmp[i];
    tzo_layernorm_rows(out, lw->ln2_g, lw->ln2_b, out, L, H, EPS);
}

/* forward, arctic.zig:874-898 (embeddingsImpl 543-585, encoder 830-848). */
static void forward_one(const tzo_arctic_weights* w, int mode, const uint32_t* ids, int L,
                        float* out, scratch_t* s, float* dump, int64_t dump_stride,
                        int64_t dump_row0) {
    float* hs = s->enc_in;
    for (int p = 0; p < L; p++) {
        float* row = hs + (size_t)p * H;
        int imode = mode != TZO_MODE_F32;
        emb_row(row, imode ? NULL : w->word_w, w->word_q, w->word_s, (int)ids[p], 0);
        emb_row(row, imode ? NULL : w->pos_w, w->pos_q, w->pos_s, p, 1);
        emb_row(row, w->type_w, NULL, NULL, 0, 1); /* token type is always row 0: arctic.zig:557 */
    }
    tzo_layernorm_rows(hs, w->emb_ln_g, w->emb_ln_b, hs, L, H, EPS);
    if (dump) memcpy(dump + dump_row0 * H, hs, sizeof(float) * (size_t)L * H);
    float* eo = s->enc_out;
    for (int l = 0; l < TZO_LAYERS; l++) {
        const float* lin = hs;
        if (l > 0) {
            memcpy(s->layer_in, eo, sizeof(float) * (size_t)L * H);
            lin = s->layer_in;
        }
        self_attention(mode, &w->layers[l], s->hidden, lin, s, L);
        feed_forward(mode, &w->layers[l], eo, s->hidden, s, L);
        if (dump) memcpy(dump + (l + 1) * dump_stride + dump_row0 * H, eo,
                         sizeof(float) * (size_t)L * H);
    }
    memcpy(out, eo, sizeof(float) * H);
    tzo_l2_normalize(out, H);
}

int tzo_arctic_forward_dump(const tzo_arctic_weights* w, int mode, const uint32_t* ids_packed,
                            const int32_t* cu_seqlens, int B, float* out, int nthreads,
                            float* dump) {
    if (B <= 0) return 0;
    int maxL = 0;
    for (int b = 0; b < B; b++) {
        int L = cu_seqlens[b + 1] - cu_seqlens[b];
        if (L <= 0 || L > TZO_MAX_POS) return -1;
        if (L > maxL) maxL = L;
    }
    int64_t T = cu_seqlens[B];
    for (int64_t i = 0; i < T; i++)
        if (ids_packed[i] >= TZO_VOCAB) return -2;
    blas_init();
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
    nthreads = 1;
#endif
    /* forwardBatchParallel (arctic.zig:959-1013): one sequence per task, private scratch. */
#pragma omp parallel num_threads(nthreads)
    {
        scratch_t s;
        scratch_alloc(&s, maxL);
#pragma omp for schedule(dynamic, 1)
        for (int b = 0; b < B; b++) {
            int L = cu_seqlens[b + 1] - cu_seqlens[b];
            forward_one(w, mode, ids_packed + cu_seqlens[b], L, out + (size_t)b * H, &s, dump,
                        T * H, cu_seqlens[b]);
        }
        scratch_free(&s);
    }
    return 0;
}

int tzo_arctic_forward(const tzo_arctic_weights* w, int mode, const uint32_t* ids_packed,
                       const int32_t* cu_seqlens, int B, float* out, int nthreads) {
    return tzo_arctic_forward_dump(w, mode, ids_packed, cu_seqlens, B, out, nthreads, NULL);
}
