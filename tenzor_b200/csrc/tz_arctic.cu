// tz_arctic.cu -- Arctic-embed-xs forward on sm_100a: model kernels (embedding + LayerNorm, CLS
// pooling + L2 norm, long-document pooling) and the host orchestration behind tz_arctic_*.  Per layer: QKV GEMM (tz_gemm.cu) -> attention
// (tz_attention.cu) -> output projection + residual + LayerNorm (tz_gemm_ln.cu) -> FFN1 + GELU
// (tz_gemm.cu) -> FFN2 + residual + LayerNorm (tz_gemm_ln.cu).  In W8A8 the f16 attention and GELU
// outputs carry their row |max| and are quantised per token inside the consuming gemm_ln kernel.
//
// Reference call stack replaced (arctic.zig): forward 874-898 -> embeddingsImpl 543-585 ->
// encoder 830-848 -> transformerBlock 814-826 -> selfAttention 639-747 / feedForward 760-810 ->
// l2Normalize 851-863; forwardBatchParallel 959-1013 becomes one packed batch on the device.
//
// Data layout in HBM (T = packed tokens, row-major):
//   X    f32 [T,384]   residual stream (LayerNorm outputs)
//   XA   f16 [T,384]   GEMM operand copy of X (F32 / W8A32)   | int8 [T,384] + xs f32 [T] (W8A8)
//   QKV  f16 [T,1152]  Q | K | V, head h at columns h*32 of each third
//   OA   f16 [T,384]   attention output (F32 / W8A32); W8A8 writes it into H instead, with its
//                      row |max| in omax [T]
//   H    f16 [T,1536]  GELU(FFN1) (+ row |max| in hmax [T] for W8A8)
// W8A8 keeps no int8 copy of the attention or GELU outputs: the consuming gemm_ln quantises them.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "tz_internal.h"
#include "tz_ptx.cuh"
#include "tz_rowops.cuh"

namespace tz {
int launch_attention(tz_ctx_t ctx, const void* qkv, int64_t total_tokens, const int* cu_seqlens, int batch, int max_len,
                     void* out, unsigned* row_absmax, cudaStream_t s, bool pdl, bool bf16);
int launch_f32_to_f16(tz_ctx_t ctx, const float* x, void* y, long long n, cudaStream_t s);
int launch_i8_to_f16(tz_ctx_t ctx, const int8_t* x, void* y, long long n, cudaStream_t s);
int launch_f32_to_bf16(tz_ctx_t ctx, const float* x, void* y, long long n, cudaStream_t s);
int launch_i8_to_bf16(tz_ctx_t ctx, const int8_t* x, void* y, long long n, cudaStream_t s);
int launch_f16bits_to_f32(tz_ctx_t ctx, const uint16_t* x, float* y, long long n, cudaStream_t s);

namespace {

constexpr int kH = 384, kF = 1536, kV = 30522, kP = 512, kLayers = 6;
constexpr float kEps = 1e-12f;  // arctic.zig:37

// AUX: 0 = f16 copy, 1 = int8 + per-token scale, 2 = bf16 copy.
template <int AUX>
// LayerNorm of one row held as 12 values per lane (columns lane*4 + 128c .. +3); the f32 result
// goes to `xrow` (a 384-float shared-memory row whose 16-byte quads are XOR-swizzled by row % 8, so
// the column-quad reads of 8 consecutive rows hit distinct banks), the next GEMM's operand (f16, or
// int8 + scale) to global memory.
__device__ __forceinline__ void ln_finish_row(float (&v)[12], const float* __restrict__ g, const float* __restrict__ b,
                                              float* xrow, void* aux, float* aux_s, long long row, int lane) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 12; ++i) s += v[i];
    const float mean = warp_sum(s) / 384.0f;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 12; ++i) {
        const float d = v[i] - mean;
        q += d * d;
    }
    const float inv_std = 1.0f / sqrtf(warp_sum(q) / 384.0f + kEps);
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int col = c * 128 + lane * 4;
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g + col));
        const float4 bb = __ldg(reinterpret_cast<const float4*>(b + col));
        v[4 * c + 0] = (v[4 * c + 0] - mean) * inv_std * gg.x + bb.x;
        v[4 * c + 1] = (v[4 * c + 1] - mean) * inv_std * gg.y + bb.y;
        v[4 * c + 2] = (v[4 * c + 2] - mean) * inv_std * gg.z + bb.z;
        v[4 * c + 3] = (v[4 * c + 3] - mean) * inv_std * gg.w + bb.w;
        *reinterpret_cast<float4*>(xrow + (((col >> 2) ^ static_cast<int>(row & 7)) << 2)) =
            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[4 * c]), fabsf(v[4 * c + 1])), fmaxf(fabsf(v[4 * c + 2]), fabsf(v[4 * c + 3]))));
    }
    if constexpr (AUX == 0 || AUX == 2) {
        uint16_t* a = static_cast<uint16_t*>(aux) + row * kH;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const int col = c * 128 + lane * 4;
            uint2 pk;
            pk.x = tzp::pack16x2<AUX == 2>(v[4 * c], v[4 * c + 1]);
            pk.y = tzp::pack16x2<AUX == 2>(v[4 * c + 2], v[4 * c + 3]);
            *reinterpret_cast<uint2*>(a + col) = pk;
        }
    } else {
        amax = warp_max(amax);
        const float sc = (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 127.0f);
        const float inv = __fdiv_rn(1.0f, sc);
        int8_t* a = static_cast<int8_t*>(aux) + row * kH;
        const uint64_t inv2 = tzp::f2_pack(inv, inv);  // the row against its own |max|: the packed quantiser applies
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const int col = c * 128 + lane * 4;
            *reinterpret_cast<uint32_t*>(a + col) = __byte_perm(quant2_own_max(v[4 * c], v[4 * c + 1], inv2),
                                                                quant2_own_max(v[4 * c + 2], v[4 * c + 3], inv2), 0x5410);
        }
        if (lane == 0) aux_s[row] = sc;
    }
}

struct EmbTables {
    const float* word_f;
    const int8_t* word_q;
    const float* word_s;
    const float* pos_f;
    const int8_t* pos_q;
    const float* pos_s;
    const float* type_f;  // row 0 used (arctic.zig:557)
};

__device__ __forceinline__ void emb_load(float (&v)[12], const float* f, const int8_t* q, const float* s, int row,
                                         int lane, bool add) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int col = c * 128 + lane * 4;
        float4 t;
        if (f) {
            t = __ldg(reinterpret_cast<const float4*>(f + static_cast<long long>(row) * kH + col));
        } else {
            const char4 qq = __ldg(reinterpret_cast<const char4*>(q + static_cast<long long>(row) * kH + col));
            const float sc = __ldg(s + row);
            t = make_float4(__fmul_rn(static_cast<float>(qq.x), sc), __fmul_rn(static_cast<float>(qq.y), sc),
                            __fmul_rn(static_cast<float>(qq.z), sc), __fmul_rn(static_cast<float>(qq.w), sc));
        }
        if (add) {
            v[4 * c] += t.x;
            v[4 * c + 1] += t.y;
            v[4 * c + 2] += t.z;
            v[4 * c + 3] += t.w;
        } else {
            v[4 * c] = t.x;
            v[4 * c + 1] = t.y;
            v[4 * c + 2] = t.z;
            v[4 * c + 3] = t.w;
        }
    }
}

// embeddingsImpl, arctic.zig:543-585: word[id] + pos[p] + type[0], then LayerNorm.  CTA = one
// 32-row group of the packed tokens (8 warps x 4 tokens).  A token's position needs its sequence: a
// warp-cooperative search of cu_seqlens finds the group's first sequence (each round probes 32
// evenly spaced entries, so B <= 32^k sequences take k dependent loads), then one load of the next
// 32 sequence ends places every row (a ballot per row).  Each warp then requests the word /
// position / type rows of two tokens at a time before their LayerNorms.  The LayerNorm
// rows are assembled in shared memory and leave in the blocked layout of xblk as coalesced 512-byte
// stores; rows past the batch are written as zeros.  Ids >= vocab raise the bounds bit and embed
// row 0.
template <int AUX>
__global__ void __launch_bounds__(256, 4)
    embed_ln_kernel(const uint32_t* __restrict__ ids, const int* __restrict__ cu, int batch, long long total, EmbTables t,
                    const float* __restrict__ g, const float* __restrict__ b, float* __restrict__ xo, void* aux,
                    float* aux_s, int* status) {
    __shared__ __align__(16) float tile[32 * kH];
    tzp::pdl_wait();
    tzp::pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long g0 = static_cast<long long>(blockIdx.x) * 32;
    // the sequence s0 with cu[s0] <= g0 < cu[s0 + 1]: search [lo, hi) by 32-way probes (every warp
    // runs the same search; the probes hit L1 after the first warp)
    int lo = 0, hi = batch;
    while (hi - lo > 1) {
        const int step = (hi - lo + 31) >> 5;
        const int idx = lo + lane * step;
        const bool le = idx < hi && cu[idx] <= g0;  // cu ascending: the probes <= g0 form a prefix
        const unsigned m = __ballot_sync(0xffffffffu, le);
        const int k = 31 - __clz(m);                  // last probe <= g0 (probe 0 = cu[lo] always is)
        lo += k * step;
        hi = min(lo + step, hi);
    }
    // rows g0 .. g0+31 meet at most 32 sequences from s0: lane j holds the end of sequence s0 + j; a
    // row's sequence is s0 + the number of those ends at or before it
    const int sj = lo + lane;
    const int end_j = sj < batch ? cu[sj + 1] : 0x7fffffff;
    int tid[4], tpos[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const long long row = g0 + warp * 4 + i;
        const bool in = row < total;
        const int seq = lo + __popc(__ballot_sync(0xffffffffu, end_j <= row));
        const int start = (in && seq < batch) ? cu[seq] : 0;
        uint32_t id = in ? ids[row] : 0u;
        if (id >= static_cast<uint32_t>(kV)) {
            if (lane == 0) atomicOr(status, TZ_DEV_BOUNDS);
            id = 0;
        }
        const long long p = row - start;
        tid[i] = static_cast<int>(id);
        tpos[i] = p < kP ? static_cast<int>(p) : kP - 1;
    }
#pragma unroll
    for (int h = 0; h < 4; h += 2) {  // two tokens' gathers in flight together (registers: 4 CTAs per SM)
        float v[2][12];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            emb_load(v[i], t.word_f, t.word_q, t.word_s, tid[h + i], lane, false);
            emb_load(v[i], t.pos_f, t.pos_q, t.pos_s, tpos[h + i], lane, true);
            emb_load(v[i], t.type_f, nullptr, nullptr, 0, lane, true);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int r = warp * 4 + h + i;
            const long long row = g0 + r;
            float* xrow = tile + r * kH;
            if (row >= total) {
#pragma unroll
                for (int c = 0; c < 3; ++c) *reinterpret_cast<float4*>(xrow + c * 128 + lane * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
                ln_finish_row<AUX>(v[i], g, b, xrow, aux, aux_s, row, lane);
            }
        }
    }
    __syncthreads();
    // blocked write-out: quad q of the group is 32 rows x 16 bytes, contiguous; lane = row
    float* dst = xo + xblk(g0, 0);
    for (int q = warp; q < kH / 4; q += 8)
        *reinterpret_cast<float4*>(dst + q * 128 + lane * 4) = *reinterpret_cast<const float4*>(tile + lane * kH + ((q ^ (lane & 7)) << 2));
}

// CLS pooling + l2Normalize (arctic.zig:851-863, forward 894-897): warp per sequence.  `out` may be
// the device view of the caller's page-locked host buffer; with `status_dst` (the device view of a
// page-locked host word) thread 0 also hands the device status word to the host, since every
// kernel of the forward has completed by griddepcontrol.wait.
__global__ void pool_l2_kernel(const float* __restrict__ x, const int* __restrict__ cu, float* __restrict__ out,
                               int batch, const int* status_src, int* status_dst) {
    tzp::pdl_wait();
    tzp::pdl_trigger();
    if (status_dst && blockIdx.x == 0 && threadIdx.x == 0) *status_dst = *status_src;
    const int seq = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (seq >= batch) return;
    const long long row = cu[seq];  // the CLS token (position 0) of the sequence
    float v[12];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float4 t = *reinterpret_cast<const float4*>(x + xblk(row, c * 128 + lane * 4));
        v[4 * c] = t.x;
        v[4 * c + 1] = t.y;
        v[4 * c + 2] = t.z;
        v[4 * c + 3] = t.w;
        s += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
    }
    const float norm = sqrtf(warp_sum(s));
    float* o = out + static_cast<long long>(seq) * kH;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        float4 t = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        if (norm > 1e-12f) {
            t.x /= norm;
            t.y /= norm;
            t.z /= norm;
            t.w /= norm;
        }
        *reinterpret_cast<float4*>(o + c * 128 + lane * 4) = t;
    }
}

// Long-document pooling of the embed CLI (main.zig:909-925): per document the chunk embeddings are
// summed in chunk order, scaled by 1/n_chunks, then divided by their L2 norm when it is positive.
// CTA of 128 threads per document, three columns per thread; the squared norm is a block sum.
__global__ void doc_mean_l2_kernel(const float* __restrict__ emb, const int* __restrict__ doc_off, float* __restrict__ out) {
    __shared__ float part[4];
    const int d = blockIdx.x;
    const int c0 = doc_off[d], c1 = doc_off[d + 1];
    const float scale = 1.0f / static_cast<float>(c1 - c0);
    float v[3];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int j = threadIdx.x + 128 * k;
        float acc = 0.f;
        for (int c = c0; c < c1; ++c) acc = __fadd_rn(acc, emb[static_cast<long long>(c) * kH + j]);
        v[k] = __fmul_rn(acc, scale);
        ss = __fadd_rn(ss, __fmul_rn(v[k], v[k]));
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    const float norm = sqrtf((part[0] + part[1]) + (part[2] + part[3]));
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int j = threadIdx.x + 128 * k;
        out[static_cast<long long>(d) * kH + j] = norm > 0.f ? __fdiv_rn(v[k], norm) : v[k];
    }
}

}  // namespace
}  // namespace tz

using namespace tz;

// ------------------------------------------------------------------------------------------------
// Model object
// ------------------------------------------------------------------------------------------------
struct DevLayer {
    void* wqkv = nullptr;  // [1152,384] f16 or int8
    void* wo = nullptr;    // [384,384]
    void* w1 = nullptr;    // [1536,384]
    void* w2 = nullptr;    // [384,1536]
    float *bqkv = nullptr, *bo = nullptr, *b1 = nullptr, *b2 = nullptr;
    float *sqkv = nullptr, *so = nullptr, *s1 = nullptr, *s2 = nullptr;  // column scales (int8 modes)
    float *ln1g = nullptr, *ln1b = nullptr, *ln2g = nullptr, *ln2b = nullptr;
};

struct tz_model_s {
    tz_ctx_t ctx = nullptr;
    int device = 0;
    int mode = TZ_QUANT_F32;
    // TZ_PREC_BF16: the f16-operand modes (F32, W8A32) run every 16-bit tensor of the forward --
    // weight copies, GEMM operands, QKV, attention and GELU outputs -- in bf16 instead of IEEE half
    bool bf16 = false;
    // int8 mode from an f32 checkpoint: the weights quantize_arctic_xs.zig would quantise are
    // quantised on the device during the load (GPU row quantiser, same rounding)
    bool quantize_on_load = false;
    // load-time pinned staging: two chunks, so the host fills one while the other's DMA runs
    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t stage_ev[2] = {nullptr, nullptr};
    std::vector<void*> allocs;  // every device allocation owned by the model
    EmbTables emb{};
    float *emb_g = nullptr, *emb_b = nullptr;
    DevLayer layers[kLayers];
    // workspace
    int cap_batch = 0;
    int64_t cap_tokens = 0;
    std::vector<void*> ws;
    uint32_t* d_ids = nullptr;
    int* d_cu = nullptr;
    float *X = nullptr, *xs = nullptr, *out = nullptr;
    void *XA = nullptr, *QKV = nullptr, *OA = nullptr, *Hh = nullptr;
    unsigned* hmax = nullptr;
    unsigned* omax = nullptr;
    uint32_t* h_ids = nullptr;  // pinned staging (used when the caller's buffers are pageable)
    int* h_cu = nullptr;
    float* h_out = nullptr;
    int* h_status = nullptr;    // pinned slot: the device status word, read back with the output
    int* status_host_view = nullptr;  // set while a zero-copy host call is captured: h_status's device view
    // padded-input staging
    uint32_t* d_pad_ids = nullptr;
    int* d_pad_lens = nullptr;
    int64_t cap_pad = 0;
    // debug
    bool keep_stages = false;
    // [8, cap_tokens, 384] when keep_stages: 0 after the embeddings, l + 1 after layer l, 7 layer 0's
    // hidden state after its attention block (the FFN1 input)
    float* d_stages = nullptr;
    // W8A8 layer-0 GEMM captures, written by the forward's own kernels (which = 0 QKV, 1 O-proj,
    // 2 FFN1, 3 FFN2): the int8 A operand and its per-token scales as the GEMM consumed them, the
    // raw int32 accumulators, and (1, 3) the f16 activation the gemm_ln kernel quantised
    int8_t* d_opq[4] = {nullptr, nullptr, nullptr, nullptr};
    float* d_ops[4] = {nullptr, nullptr, nullptr, nullptr};
    int32_t* d_acc[4] = {nullptr, nullptr, nullptr, nullptr};
    __half* d_in16[4] = {nullptr, nullptr, nullptr, nullptr};
    int64_t last_T = 0;
    // kernel-class timing: events around every launch of the forward (recorded in graphs too)
    bool profile = false;
    std::vector<cudaEvent_t> ev;  // prof_slots x 65: one set of events per recorded forward
    int prof_slots = 0;
    int64_t prof_fwd = 0;         // forwards recorded since profiling was enabled
    int ev_base = 0;              // first event of the current forward's set
    int ev_n = 0;                 // events recorded by the last enqueue
    int ev_cls[64] = {0};         // class of launch i
    // graph cache for the host-pointer forward
    cudaGraphExec_t graph = nullptr;
    int g_batch = -1, g_maxlen = -1;
    int64_t g_tokens = -1;
    const void* g_io[3] = {nullptr, nullptr, nullptr};  // pinned ids / cu / out the graph copies (or none)
    bool use_graph = true;
    // W8A8: the feed-forward block as the FFN1 GEMM + FFN2 gemm_ln pair with the GELU output through
    // device memory (the default: faster on B200), or as one kernel with the GELU output kept on chip
    // (tz_ffn.cu; tz_arctic_set_ffn_fusion)
    bool ffn_fused = false;
    // graph cache for the device-pointer forward (keyed by buffers, shape and stream)
    cudaGraphExec_t dgraph = nullptr;
    const void* dkey[4] = {nullptr, nullptr, nullptr, nullptr};
    int64_t dkey_shape[3] = {-1, -1, -1};
};

namespace {

// K and N of the layer's four GEMMs (0 QKV, 1 attention output, 2 FFN1, 3 FFN2).
constexpr int gemm_k(int which) { return which == 3 ? kF : kH; }
constexpr int gemm_n(int which) { return which == 0 ? 3 * kH : (which == 2 ? kF : kH); }

int dalloc(tz_model_s* m, std::vector<void*>& list, size_t bytes, void** p) {
    TZ_CUDA(cudaMalloc(p, bytes ? bytes : 16));
    list.push_back(*p);
    return TZ_OK;
}

// Host -> device copy ordered on the context stream and complete on return.  (A plain cudaMemcpy
// from pageable memory may return before its DMA lands, and the conversion kernels that consume
// the copies run on the context's non-blocking stream, so the copy must be stream-ordered.)
// Copies of 4 MiB and more go through the model's two pinned staging chunks (memcpy into chunk k
// while chunk 1 - k is on the wire): the source may be pageable or a file mapping.
constexpr size_t kStageBytes = 8u << 20;
int h2d(tz_model_s* m, void* dst, const void* src, size_t bytes) {
    cudaStream_t s = m->ctx->stream;
    if (bytes < (4u << 20)) {
        TZ_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s));
        TZ_CUDA(cudaStreamSynchronize(s));
        return TZ_OK;
    }
    for (int k = 0; k < 2; ++k)
        if (!m->stage[k]) {
            TZ_CUDA(cudaMallocHost(&m->stage[k], kStageBytes));
            TZ_CUDA(cudaEventCreateWithFlags(&m->stage_ev[k], cudaEventDisableTiming));
        }
    const char* p = static_cast<const char*>(src);
    char* d = static_cast<char*>(dst);
    int k = 0;
    for (size_t off = 0; off < bytes; off += kStageBytes, k ^= 1) {
        const size_t n = bytes - off < kStageBytes ? bytes - off : kStageBytes;
        TZ_CUDA(cudaEventSynchronize(m->stage_ev[k]));  // chunk k's previous copy has left the buffer
        std::memcpy(m->stage[k], p + off, n);
        TZ_CUDA(cudaMemcpyAsync(d + off, m->stage[k], n, cudaMemcpyHostToDevice, s));
        TZ_CUDA(cudaEventRecord(m->stage_ev[k], s));
    }
    TZ_CUDA(cudaStreamSynchronize(s));
    return TZ_OK;
}

void release_staging(tz_model_s* m) {
    for (int k = 0; k < 2; ++k) {
        if (m->stage[k]) cudaFreeHost(m->stage[k]);
        if (m->stage_ev[k]) cudaEventDestroy(m->stage_ev[k]);
        m->stage[k] = nullptr;
        m->stage_ev[k] = nullptr;
    }
}

int upload_raw(tz_model_s* m, const void* src, size_t bytes, void** dst) {
    int rc = dalloc(m, m->allocs, bytes, dst);
    if (rc) return rc;
    return h2d(m, *dst, src, bytes);
}

int upload_f32(tz_model_s* m, const float* src, size_t n, float** dst, const char* what) {
    TZ_CHECK(src, TZ_EMISSING, "missing weight: %s", what);
    return upload_raw(m, src, n * sizeof(float), reinterpret_cast<void**>(dst));
}

// f32 host rows -> int8 rows + f16 scale bits on the device (quantize_arctic_xs.zig:94-115 rules,
// through the row quantiser of tz_quantize_weight_rows).
int quantize_upload(tz_model_s* m, const float* src, int64_t rows, int cols, int8_t* dq, uint16_t* ds) {
    void* tmp = nullptr;
    TZ_CUDA(cudaMalloc(&tmp, sizeof(float) * rows * cols));
    int rc = h2d(m, tmp, src, sizeof(float) * rows * cols);
    if (!rc) rc = tz_quantize_weight_rows(m->ctx, static_cast<const float*>(tmp), dq, ds, rows, cols, m->ctx->stream);
    cudaStreamSynchronize(m->ctx->stream);
    cudaFree(tmp);
    return rc;
}

// A Linear weight [rows, cols] into the device operand format of the mode, at row offset `row0` of
// a (possibly concatenated) destination with `total_rows` rows.
int upload_linear(tz_model_s* m, const tz_mat_weight& w, int rows, int cols, void* dst, int row0, float* scale_dst,
                  const char* what) {
    cudaStream_t s = m->ctx->stream;
    if (m->mode == TZ_QUANT_F32) {
        TZ_CHECK(w.f32, TZ_EINVAL, "%s: mode F32 needs f32 weights", what);
        void* tmp = nullptr;
        TZ_CUDA(cudaMalloc(&tmp, sizeof(float) * rows * cols));
        int rc = h2d(m, tmp, w.f32, sizeof(float) * rows * cols);
        if (!rc)
            rc = (m->bf16 ? launch_f32_to_bf16 : launch_f32_to_f16)(m->ctx, static_cast<float*>(tmp),
                                                                   static_cast<uint16_t*>(dst) + static_cast<long long>(row0) * cols,
                                                                   static_cast<long long>(rows) * cols, s);
        cudaStreamSynchronize(s);
        cudaFree(tmp);
        return rc;
    }
    const bool qload = m->quantize_on_load && !w.q8 && w.f32;
    TZ_CHECK(qload || (w.q8 && w.scale_f16), TZ_EINVAL, "%s: int8 modes need int8 weights with a half scale", what);
    void* tq = nullptr;
    void* ts = nullptr;
    TZ_CUDA(cudaMalloc(&tq, static_cast<size_t>(rows) * cols));
    TZ_CUDA(cudaMalloc(&ts, sizeof(uint16_t) * rows));
    int rc = qload ? quantize_upload(m, w.f32, rows, cols, static_cast<int8_t*>(tq), static_cast<uint16_t*>(ts))
                   : h2d(m, tq, w.q8, static_cast<size_t>(rows) * cols);
    if (!rc && !qload) rc = h2d(m, ts, w.scale_f16, sizeof(uint16_t) * rows);
    if (!rc)
        rc = launch_f16bits_to_f32(m->ctx, static_cast<uint16_t*>(ts), scale_dst + row0, rows, s);
    if (!rc) {
        if (m->mode == TZ_QUANT_W8A8)
            TZ_CUDA(cudaMemcpyAsync(static_cast<int8_t*>(dst) + static_cast<long long>(row0) * cols, tq,
                                    static_cast<size_t>(rows) * cols, cudaMemcpyDeviceToDevice, s));
        else  // W8A32: int8 values widened exactly to f16 (bf16); the scale is applied in the epilogue
            rc = (m->bf16 ? launch_i8_to_bf16 : launch_i8_to_f16)(m->ctx, static_cast<int8_t*>(tq),
                                                                 static_cast<uint16_t*>(dst) + static_cast<long long>(row0) * cols,
                                                                 static_cast<long long>(rows) * cols, s);
    }
    cudaStreamSynchronize(s);
    cudaFree(tq);
    cudaFree(ts);
    return rc;
}

int upload_table(tz_model_s* m, const tz_mat_weight& w, int rows, const float** f, const int8_t** q, const float** s,
                 const char* what) {
    *f = nullptr;
    *q = nullptr;
    *s = nullptr;
    // shouldQuantize (quantize_arctic_xs.zig:22-40): 2-D, >= 4096 elements (word and position tables)
    const bool qload = m->quantize_on_load && w.f32 && !w.q8 && static_cast<int64_t>(rows) * kH >= 4096;
    if (w.f32 && !qload) {
        float* d = nullptr;
        int rc = upload_f32(m, w.f32, static_cast<size_t>(rows) * kH, &d, what);
        *f = d;
        return rc;
    }
    TZ_CHECK(qload || (w.q8 && w.scale_f16), TZ_EMISSING, "missing weight: %s", what);
    void* dq = nullptr;
    int rc = dalloc(m, m->allocs, static_cast<size_t>(rows) * kH, &dq);
    if (rc) return rc;
    void* ts = nullptr;
    float* ds = nullptr;
    rc = dalloc(m, m->allocs, sizeof(float) * rows, reinterpret_cast<void**>(&ds));
    if (rc) return rc;
    TZ_CUDA(cudaMalloc(&ts, sizeof(uint16_t) * rows));
    rc = qload ? quantize_upload(m, w.f32, rows, kH, static_cast<int8_t*>(dq), static_cast<uint16_t*>(ts))
               : h2d(m, dq, w.q8, static_cast<size_t>(rows) * kH);
    if (!rc && !qload) rc = h2d(m, ts, w.scale_f16, sizeof(uint16_t) * rows);
    if (!rc) rc = launch_f16bits_to_f32(m->ctx, static_cast<uint16_t*>(ts), ds, rows, m->ctx->stream);
    cudaStreamSynchronize(m->ctx->stream);
    cudaFree(ts);
    *q = static_cast<int8_t*>(dq);
    *s = ds;
    return rc;
}

void drop_graphs(tz_model_s* m) {
    if (m->graph) {
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    m->g_io[0] = m->g_io[1] = m->g_io[2] = nullptr;
    if (m->dgraph) {
        cudaGraphExecDestroy(m->dgraph);
        m->dgraph = nullptr;
    }
    m->dkey[0] = m->dkey[1] = m->dkey[2] = m->dkey[3] = nullptr;
}

void free_workspace(tz_model_s* m) {
    drop_graphs(m);
    for (void* p : m->ws) cudaFree(p);
    m->ws.clear();
    if (m->h_ids) cudaFreeHost(m->h_ids);
    if (m->h_cu) cudaFreeHost(m->h_cu);
    if (m->h_out) cudaFreeHost(m->h_out);
    if (m->h_status) cudaFreeHost(m->h_status);
    m->h_ids = nullptr;
    m->h_cu = nullptr;
    m->h_out = nullptr;
    m->h_status = nullptr;
    m->cap_batch = 0;
    m->cap_tokens = 0;
    m->d_stages = nullptr;
    for (int i = 0; i < 4; ++i) {
        m->d_opq[i] = nullptr;
        m->d_ops[i] = nullptr;
        m->d_acc[i] = nullptr;
        m->d_in16[i] = nullptr;
    }
}

int reserve(tz_model_s* m, int batch, int64_t tokens) {
    if (batch <= m->cap_batch && tokens <= m->cap_tokens && (!m->keep_stages || m->d_stages)) return TZ_OK;
    TZ_CUDA(cudaSetDevice(m->ctx->device));
    TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
    const int nb = std::max(batch, m->cap_batch);
    const int64_t nt = std::max<int64_t>(tokens, m->cap_tokens);
    free_workspace(m);
    const size_t T = static_cast<size_t>(nt);
    int rc = 0;
    auto A = [&](size_t bytes, void** p) {
        if (!rc) rc = dalloc(m, m->ws, bytes, p);
    };
    A(sizeof(uint32_t) * T, reinterpret_cast<void**>(&m->d_ids));
    A(sizeof(int) * (nb + 1), reinterpret_cast<void**>(&m->d_cu));
    A(sizeof(float) * xblk_rows(static_cast<long long>(T)) * kH, reinterpret_cast<void**>(&m->X));  // blocked (xblk)
    A(sizeof(__half) * T * 3 * kH, &m->QKV);
    A(sizeof(float) * nb * kH, reinterpret_cast<void**>(&m->out));
    if (m->mode == TZ_QUANT_W8A8) {
        A(T * kH, &m->XA);
        A(sizeof(float) * T, reinterpret_cast<void**>(&m->xs));
        A(sizeof(unsigned) * T, reinterpret_cast<void**>(&m->hmax));
        A(sizeof(unsigned) * T, reinterpret_cast<void**>(&m->omax));
        A(sizeof(__half) * T * kF, &m->Hh);
    } else {
        A(sizeof(__half) * T * kH, &m->XA);
        A(sizeof(__half) * T * kH, &m->OA);
        A(sizeof(__half) * T * kF, &m->Hh);
    }
    if (m->keep_stages) {
        A(sizeof(float) * 8 * xblk_rows(static_cast<long long>(T)) * kH, reinterpret_cast<void**>(&m->d_stages));
        if (m->mode == TZ_QUANT_W8A8)
            for (int i = 0; i < 4; ++i) {
                A(T * gemm_k(i), reinterpret_cast<void**>(&m->d_opq[i]));
                A(sizeof(float) * T, reinterpret_cast<void**>(&m->d_ops[i]));
                A(sizeof(int32_t) * T * gemm_n(i), reinterpret_cast<void**>(&m->d_acc[i]));
                if (i & 1) A(sizeof(__half) * T * gemm_k(i), reinterpret_cast<void**>(&m->d_in16[i]));
            }
    }
    if (rc) {
        free_workspace(m);
        return rc;
    }
    if (m->hmax) TZ_CUDA(cudaMemset(m->hmax, 0, sizeof(unsigned) * T));
    if (m->omax) TZ_CUDA(cudaMemset(m->omax, 0, sizeof(unsigned) * T));
    TZ_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&m->h_ids), sizeof(uint32_t) * T, cudaHostAllocDefault));
    TZ_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&m->h_cu), sizeof(int) * (nb + 1), cudaHostAllocDefault));
    TZ_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&m->h_out), sizeof(float) * nb * kH, cudaHostAllocDefault));
    TZ_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&m->h_status), sizeof(int), cudaHostAllocDefault));
    m->cap_batch = nb;
    m->cap_tokens = nt;
    return TZ_OK;
}

enum ProfClass { P_EMBED = 0, P_QKV, P_ATTN, P_OPROJ, P_LN, P_FFN1, P_FFN, P_FFN2, P_POOL, P_NCLASS };

// Records the event that closes launch (ev_n - 1) and opens the next one.
int prof_mark(tz_model_s* m, int next_class, cudaStream_t s) {
    if (!m->profile) return TZ_OK;
    if (m->ev_n >= 65) return TZ_OK;
    // Inside a stream capture the record must become an external event node so that every graph
    // replay records it (a plain record only orders the captured work).
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    TZ_CUDA(cudaStreamIsCapturing(s, &cs));
    TZ_CUDA(cudaEventRecordWithFlags(m->ev[m->ev_base + m->ev_n], s,
                                     cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault));
    if (next_class >= 0 && m->ev_n < 64) m->ev_cls[m->ev_n] = next_class;
    ++m->ev_n;
    return TZ_OK;
}

// W8A8 parity hook: keeps a copy of a layer-0 GEMM operand (int8 rows + per-row scales).
int keep_operand(tz_model_s* m, int which, const void* q, const float* sc, int64_t T, int K, cudaStream_t s) {
    if (!m->keep_stages || m->mode != TZ_QUANT_W8A8 || !m->d_opq[which]) return TZ_OK;
    TZ_CUDA(cudaMemcpyAsync(m->d_opq[which], q, static_cast<size_t>(T) * K, cudaMemcpyDeviceToDevice, s));
    TZ_CUDA(cudaMemcpyAsync(m->d_ops[which], sc, sizeof(float) * T, cudaMemcpyDeviceToDevice, s));
    return TZ_OK;
}

// Enqueues the whole forward on `s`: device ids/cu already in place (d_ids/d_cu may be the
// caller's device buffers).
int enqueue_forward(tz_model_s* m, const uint32_t* d_ids, const int* d_cu, int B, int64_t T, int maxL, float* d_out,
                    cudaStream_t s) {
    tz_ctx_t ctx = m->ctx;
    const bool q8 = m->mode == TZ_QUANT_W8A8;
    const bool wscale = m->mode != TZ_QUANT_F32;
    const int M = static_cast<int>(T);
    int rc;
    m->ev_n = 0;
    if (m->profile) m->ev_base = static_cast<int>(m->prof_fwd % m->prof_slots) * 65;
    if ((rc = prof_mark(m, P_EMBED, s))) return rc;
    const bool pdl = !m->profile;  // events between launches would break the programmatic edges anyway
    if (q8)
        rc = launch_kernel(embed_ln_kernel<1>, dim3(static_cast<unsigned>((T + 31) / 32)), dim3(256), 0, s, pdl, d_ids, d_cu, B,
                           static_cast<long long>(T), m->emb, (const float*)m->emb_g,
                           (const float*)m->emb_b, m->X, m->XA, m->xs, ctx->d_status);
    else
        rc = launch_kernel(m->bf16 ? embed_ln_kernel<2> : embed_ln_kernel<0>, dim3(static_cast<unsigned>((T + 31) / 32)), dim3(256), 0,
                           s, pdl, d_ids, d_cu, B, static_cast<long long>(T), m->emb, (const float*)m->emb_g,
                           (const float*)m->emb_b, m->X, m->XA, (float*)nullptr, ctx->d_status);
    if (rc) return rc;
    if (m->keep_stages)
        TZ_CUDA(cudaMemcpyAsync(m->d_stages, m->X, sizeof(float) * xblk_rows(T) * kH, cudaMemcpyDeviceToDevice, s));
    for (int l = 0; l < kLayers; ++l) {
        const DevLayer& L = m->layers[l];
        GemmArgs g;
        g.pdl = pdl;
        g.kind = q8 ? KIND_I8 : (m->bf16 ? KIND_BF16 : KIND_F16);
        const int out16 = m->bf16 ? OUT_BF16 : OUT_F16;
        // QKV projection (3 linearProjection calls of selfAttention fused into one N=1152 GEMM)
        g.a = m->XA; g.lda = kH; g.b = L.wqkv; g.ldb = kH; g.M = M; g.N = 3 * kH; g.K = kH;
        g.bias = L.bqkv; g.col_scale = wscale ? L.sqkv : nullptr; g.row_scale = q8 ? m->xs : nullptr;
        g.out = m->QKV; g.ldo = 3 * kH; g.out_type = out16;
        const bool cap = q8 && l == 0 && m->keep_stages && m->d_acc[0];  // W8A8 layer-0 parity capture
        if (cap) g.dbg_acc = m->d_acc[0];
        if (l == 0 && (rc = keep_operand(m, 0, m->XA, m->xs, T, kH, s))) return rc;
        if ((rc = prof_mark(m, P_QKV, s))) return rc;
        if ((rc = launch_gemm(ctx, g, s))) return rc;
        if ((rc = prof_mark(m, P_ATTN, s))) return rc;
        // attention
        // W8A8: the f16 attention output (with each row's |max|) goes through the (still free) H
        // buffer; the output projection quantises it per token inside its own kernel.
        if ((rc = launch_attention(ctx, m->QKV, T, d_cu, B, maxL, q8 ? m->Hh : m->OA, q8 ? m->omax : nullptr, s, pdl, m->bf16)))
            return rc;
        if (cap)  // the f16 attention output the next kernel quantises in its mainloop
            TZ_CUDA(cudaMemcpyAsync(m->d_in16[1], m->Hh, sizeof(__half) * T * kH, cudaMemcpyDeviceToDevice, s));
        // output projection + bias + residual + LayerNorm in one kernel (arctic.zig:716-746)
        GemmLnArgs o;
        o.pdl = pdl;
        o.kind = g.kind;
        o.a = q8 ? m->Hh : m->OA; o.lda = kH; o.b = L.wo; o.ldb = kH; o.M = M; o.K = kH;
        o.bias = L.bo; o.col_scale = wscale ? L.so : nullptr; o.a_absmax = q8 ? m->omax : nullptr;
        o.residual = m->X; o.gamma = L.ln1g; o.beta = L.ln1b; o.eps = kEps;
        o.x_out = m->X; o.aux = m->XA; o.aux_scale = q8 ? m->xs : nullptr; o.aux_int8 = q8; o.aux_bf16 = m->bf16;
        if (cap) {
            o.dbg_acc = m->d_acc[1];
            o.dbg_aq = m->d_opq[1];
            o.dbg_as = m->d_ops[1];
        }
        if ((rc = prof_mark(m, P_OPROJ, s))) return rc;
        if ((rc = launch_gemm_ln(ctx, o, s))) return rc;
        if (l == 0 && m->keep_stages)  // layer 0's hidden state after the attention block
            TZ_CUDA(cudaMemcpyAsync(m->d_stages + static_cast<size_t>(7) * xblk_rows(m->cap_tokens) * kH, m->X,
                                    sizeof(float) * xblk_rows(T) * kH, cudaMemcpyDeviceToDevice, s));
        if (q8 && m->ffn_fused) {
            // the whole feed-forward block in one kernel (arctic.zig:760-810): FFN1 + GELU, the
            // per-token int8 form of the GELU output kept on chip, FFN2 + residual + LayerNorm and the
            // next layer's int8 operand
            FfnArgs fa;
            fa.pdl = pdl;
            fa.xq = static_cast<const int8_t*>(m->XA); fa.xs = m->xs; fa.M = M;
            fa.w1 = static_cast<const int8_t*>(L.w1); fa.s1 = L.s1; fa.b1 = L.b1;
            fa.w2 = static_cast<const int8_t*>(L.w2); fa.s2 = L.s2; fa.b2 = L.b2;
            fa.gamma = L.ln2g; fa.beta = L.ln2b; fa.eps = kEps; fa.x = m->X;
            if (cap) {
                fa.dbg_acc1 = m->d_acc[2];
                fa.dbg_h16 = m->d_in16[3];
                fa.dbg_hq = m->d_opq[3];
                fa.dbg_hs = m->d_ops[3];
                fa.dbg_acc2 = m->d_acc[3];
            }
            if (l == 0 && (rc = keep_operand(m, 2, m->XA, m->xs, T, kH, s))) return rc;
            if ((rc = prof_mark(m, P_FFN, s))) return rc;
            if ((rc = launch_ffn_w8a8(ctx, fa, s))) return rc;
        } else {
            // FFN1 + bias + GELU
            GemmArgs f1;
            f1.pdl = pdl;
            f1.kind = g.kind;
            f1.a = m->XA; f1.lda = kH; f1.b = L.w1; f1.ldb = kH; f1.M = M; f1.N = kF; f1.K = kH;
            f1.bias = L.b1; f1.col_scale = wscale ? L.s1 : nullptr; f1.row_scale = q8 ? m->xs : nullptr;
            f1.gelu = 1; f1.out = m->Hh; f1.ldo = kF; f1.out_type = out16; f1.row_absmax = q8 ? m->hmax : nullptr;
            if (cap) f1.dbg_acc = m->d_acc[2];
            if (l == 0 && (rc = keep_operand(m, 2, m->XA, m->xs, T, kH, s))) return rc;
            if ((rc = prof_mark(m, P_FFN1, s))) return rc;
            if ((rc = launch_gemm(ctx, f1, s))) return rc;
            if (cap)  // the f16 GELU output the next kernel quantises in its mainloop
                TZ_CUDA(cudaMemcpyAsync(m->d_in16[3], m->Hh, sizeof(__half) * T * kF, cudaMemcpyDeviceToDevice, s));
            // FFN2 + bias + residual + LayerNorm in one kernel (arctic.zig:779-807); W8A8 quantises the
            // f16 GELU output per token inside the kernel.
            GemmLnArgs f2;
            f2.pdl = pdl;
            f2.kind = g.kind;
            f2.a = m->Hh; f2.lda = kF; f2.b = L.w2; f2.ldb = kF; f2.M = M; f2.K = kF;
            f2.bias = L.b2; f2.col_scale = wscale ? L.s2 : nullptr; f2.a_absmax = q8 ? m->hmax : nullptr;
            f2.residual = m->X; f2.gamma = L.ln2g; f2.beta = L.ln2b; f2.eps = kEps;
            f2.x_out = m->X; f2.aux = m->XA; f2.aux_scale = q8 ? m->xs : nullptr; f2.aux_int8 = q8; f2.aux_bf16 = m->bf16;
            if (cap) {
                f2.dbg_acc = m->d_acc[3];
                f2.dbg_aq = m->d_opq[3];
                f2.dbg_as = m->d_ops[3];
            }
            if ((rc = prof_mark(m, P_FFN2, s))) return rc;
            if ((rc = launch_gemm_ln(ctx, f2, s))) return rc;
        }
        if (m->keep_stages)
            TZ_CUDA(cudaMemcpyAsync(m->d_stages + static_cast<size_t>(l + 1) * xblk_rows(m->cap_tokens) * kH, m->X,
                                    sizeof(float) * xblk_rows(T) * kH,
                                    cudaMemcpyDeviceToDevice, s));
    }
    if ((rc = prof_mark(m, P_POOL, s))) return rc;
    if ((rc = launch_kernel(pool_l2_kernel, dim3((B * 32 + 255) / 256), dim3(256), 0, s, pdl, (const float*)m->X, d_cu,
                            d_out, B, (const int*)m->ctx->d_status, m->status_host_view)))
        return rc;
    if ((rc = prof_mark(m, -1, s))) return rc;
    if (m->profile) ++m->prof_fwd;
    return TZ_OK;
}

int check_lengths(const int32_t* cu, int B, int64_t* T, int* maxL) {
    TZ_CHECK(cu[0] == 0, TZ_EINVAL, "cu_seqlens[0] must be 0");
    int mx = 0;
    for (int b = 0; b < B; ++b) {
        const int L = cu[b + 1] - cu[b];
        TZ_CHECK(L >= 1 && L <= kP, TZ_EINVAL, "sequence %d has length %d (must be 1..512)", b, L);
        mx = std::max(mx, L);
    }
    *T = cu[B];
    *maxL = mx;
    return TZ_OK;
}

// Host ids -> the model's device output rows (m->out), enqueued on the context's stream without
// a graph and without waiting; the caller reads m->out after synchronising.
int forward_to_device(tz_model_s* m, const uint32_t* ids, const int32_t* cu, int B) {
    int64_t T = 0;
    int maxL = 0;
    int rc = check_lengths(cu, B, &T, &maxL);
    if (rc) return rc;
    for (int64_t i = 0; i < T; ++i)
        TZ_CHECK(ids[i] < static_cast<uint32_t>(kV), TZ_EINVAL, "token id %u at %lld is >= vocab %d", ids[i],
                 static_cast<long long>(i), kV);
    if ((rc = reserve(m, B, T))) return rc;
    TZ_CUDA(cudaSetDevice(m->ctx->device));
    cudaStream_t s = m->ctx->stream;
    TZ_CUDA(cudaStreamSynchronize(s));  // the pinned staging may still feed an earlier forward
    memcpy(m->h_ids, ids, sizeof(uint32_t) * T);
    memcpy(m->h_cu, cu, sizeof(int) * (B + 1));
    TZ_CUDA(cudaMemcpyAsync(m->d_ids, m->h_ids, sizeof(uint32_t) * T, cudaMemcpyHostToDevice, s));
    TZ_CUDA(cudaMemcpyAsync(m->d_cu, m->h_cu, sizeof(int) * (B + 1), cudaMemcpyHostToDevice, s));
    m->last_T = T;
    return enqueue_forward(m, m->d_ids, m->d_cu, B, T, maxL, m->out, s);
}

bool host_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// The synchronous host-pointer forward.  The forward itself replays a CUDA graph (keyed by batch,
// tokens and longest sequence); the copies sit outside it, so page-locked caller buffers are read
// and written directly and only pageable ones go through the pinned staging.  The device status
// word comes back with the output: one synchronisation per call.
int forward_host(tz_model_s* m, const uint32_t* ids, const int32_t* cu, int B, float* out) {
    int64_t T = 0;
    int maxL = 0;
    int rc = check_lengths(cu, B, &T, &maxL);
    if (rc) return rc;
    if ((rc = reserve(m, B, T))) return rc;
    TZ_CUDA(cudaSetDevice(m->ctx->device));
    cudaStream_t s = m->ctx->stream;
    const bool ids_pin = host_pinned(ids), cu_pin = host_pinned(cu), out_pin = host_pinned(out);
    uint32_t bad = 0;  // ids >= vocab, checked in the same pass as the staging copy
    if (ids_pin) {
        for (int64_t i = 0; i < T; ++i) bad |= ids[i] >= static_cast<uint32_t>(kV) ? 1u : 0u;
    } else {
        for (int64_t i = 0; i < T; ++i) {
            const uint32_t v = ids[i];
            bad |= v >= static_cast<uint32_t>(kV) ? 1u : 0u;
            m->h_ids[i] = v;
        }
    }
    if (bad) {
        for (int64_t i = 0; i < T; ++i)
            TZ_CHECK(ids[i] < static_cast<uint32_t>(kV), TZ_EINVAL, "token id %u at %lld is >= vocab %d", ids[i],
                     static_cast<long long>(i), kV);
    }
    if (!cu_pin) memcpy(m->h_cu, cu, sizeof(int) * (B + 1));
    const bool graph_ok = m->use_graph && !m->keep_stages;
    // With every host buffer pinned, the copies are captured with the forward: one graph launch per
    // call (the graph is keyed by the buffers as well as the shape).
    const bool io_graph = graph_ok && ids_pin && cu_pin && out_pin;
    const void* io[3] = {io_graph ? static_cast<const void*>(ids) : nullptr, io_graph ? static_cast<const void*>(cu) : nullptr,
                         io_graph ? static_cast<const void*>(out) : nullptr};
    // Zero-copy output: when the caller's page-locked output buffer (and the model's status slot) have
    // device views, the pooling kernel writes the embeddings and the status word straight into host
    // memory -- no device-to-host copy nodes after the forward.  Otherwise the graph copies them.
    float* out_view = nullptr;
    int* status_view = nullptr;
    if (io_graph) {
        void* pv = nullptr;
        if (cudaHostGetDevicePointer(&pv, out, 0) == cudaSuccess) out_view = static_cast<float*>(pv);
        pv = nullptr;
        if (out_view && cudaHostGetDevicePointer(&pv, m->h_status, 0) == cudaSuccess) status_view = static_cast<int*>(pv);
        if (!status_view) out_view = nullptr;
        (void)cudaGetLastError();  // a buffer without a device view is not an error: the copies serve it
    }
    auto h2d_inputs = [&]() -> int {
        TZ_CUDA(cudaMemcpyAsync(m->d_ids, ids_pin ? ids : m->h_ids, sizeof(uint32_t) * T, cudaMemcpyHostToDevice, s));
        TZ_CUDA(cudaMemcpyAsync(m->d_cu, cu_pin ? cu : m->h_cu, sizeof(int) * (B + 1), cudaMemcpyHostToDevice, s));
        return TZ_OK;
    };
    auto d2h_outputs = [&]() -> int {
        TZ_CUDA(cudaMemcpyAsync(out_pin ? out : m->h_out, m->out, sizeof(float) * B * kH, cudaMemcpyDeviceToHost, s));
        TZ_CUDA(cudaMemcpyAsync(m->h_status, m->ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, s));
        return TZ_OK;
    };
    if (graph_ok && !(m->graph && m->g_batch == B && m->g_tokens == T && m->g_maxlen == maxL && m->g_io[0] == io[0] &&
                      m->g_io[1] == io[1] && m->g_io[2] == io[2])) {
        if (m->graph) {
            cudaGraphExecDestroy(m->graph);
            m->graph = nullptr;
        }
        cudaGraph_t gr = nullptr;
        TZ_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        int crc = io_graph ? h2d_inputs() : TZ_OK;
        m->status_host_view = status_view;
        if (!crc) crc = enqueue_forward(m, m->d_ids, m->d_cu, B, T, maxL, out_view ? out_view : m->out, s);
        m->status_host_view = nullptr;
        if (!crc && io_graph && !out_view) crc = d2h_outputs();
        const cudaError_t ee = cudaStreamEndCapture(s, &gr);
        if (crc) {
            if (gr) cudaGraphDestroy(gr);
            return crc;
        }
        if (ee != cudaSuccess) return cuda_fail(ee, "cudaStreamEndCapture");
        const cudaError_t ce = cudaGraphInstantiate(&m->graph, gr, 0);
        cudaGraphDestroy(gr);
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate");
        m->g_batch = B;
        m->g_tokens = T;
        m->g_maxlen = maxL;
        for (int i = 0; i < 3; ++i) m->g_io[i] = io[i];
    }
    if (!io_graph && (rc = h2d_inputs())) return rc;
    if (graph_ok) {
        TZ_CUDA(cudaGraphLaunch(m->graph, s));
    } else if ((rc = enqueue_forward(m, m->d_ids, m->d_cu, B, T, maxL, m->out, s))) {
        return rc;
    }
    if (!io_graph && (rc = d2h_outputs())) return rc;
    TZ_CUDA(cudaStreamSynchronize(s));
    if (*m->h_status) {
        if ((rc = read_status(m->ctx, s))) return rc;
    }
    if (!out_pin) memcpy(out, m->h_out, sizeof(float) * B * kH);
    m->last_T = T;
    return TZ_OK;
}

}  // namespace

extern "C" {

int tz_arctic_load(tz_ctx_t ctx, const tz_arctic_weights* w, int mode, tz_model_t* out) {
    return tz_arctic_load_ex(ctx, w, mode, TZ_PREC_F16, out);
}

int tz_arctic_load_ex(tz_ctx_t ctx, const tz_arctic_weights* w, int mode, int prec, tz_model_t* out) {
    TZ_CHECK(ctx && w && out, TZ_EINVAL, "tz_arctic_load: null argument");
    TZ_CHECK(mode >= TZ_QUANT_F32 && mode <= TZ_QUANT_W8A8, TZ_EINVAL, "tz_arctic_load: bad mode %d", mode);
    TZ_CHECK(prec == TZ_PREC_F16 || prec == TZ_PREC_BF16, TZ_EUNSUPPORTED,
             "tz_arctic_load: GEMM precision %d is not provided for the model (TZ_PREC_F16, TZ_PREC_BF16)", prec);
    TZ_CHECK(prec == TZ_PREC_F16 || mode != TZ_QUANT_W8A8, TZ_EUNSUPPORTED,
             "tz_arctic_load: W8A8 runs int8 GEMMs; the 16-bit precision applies to the F32 and W8A32 modes");
    *out = nullptr;
    TZ_CUDA(cudaSetDevice(ctx->device));
    auto m = std::make_unique<tz_model_s>();
    m->ctx = ctx;
    m->device = ctx->device;
    m->mode = mode;
    m->bf16 = prec == TZ_PREC_BF16;
    m->quantize_on_load = mode != TZ_QUANT_F32 && w->layers[0].query.f32 && !w->layers[0].query.q8;
    int rc = TZ_OK;
    auto fail_cleanup = [&](int code) {
        release_staging(m.get());
        for (void* p : m->allocs) cudaFree(p);
        m->allocs.clear();
        return code;
    };
#define TRY(x)                                      \
    do {                                            \
        if ((rc = (x))) return fail_cleanup(rc);    \
    } while (0)
    TRY(upload_table(m.get(), w->word_embeddings, kV, &m->emb.word_f, &m->emb.word_q, &m->emb.word_s, "embeddings.word_embeddings.weight"));
    TRY(upload_table(m.get(), w->position_embeddings, kP, &m->emb.pos_f, &m->emb.pos_q, &m->emb.pos_s, "embeddings.position_embeddings.weight"));
    {
        const float* tf = nullptr;
        const int8_t* tq = nullptr;
        const float* ts = nullptr;
        TRY(upload_table(m.get(), w->token_type_embeddings, 2, &tf, &tq, &ts, "embeddings.token_type_embeddings.weight"));
        TRY(tf ? TZ_OK : fail(TZ_EINVAL, "token_type_embeddings must be f32 (768 elements are never quantised)"));
        m->emb.type_f = tf;
    }
    TRY(upload_f32(m.get(), w->ln_gamma, kH, &m->emb_g, "embeddings.LayerNorm.weight"));
    TRY(upload_f32(m.get(), w->ln_beta, kH, &m->emb_b, "embeddings.LayerNorm.bias"));
    const size_t el = (mode == TZ_QUANT_W8A8) ? 1 : 2;
    for (int l = 0; l < kLayers; ++l) {
        const tz_arctic_layer& s = w->layers[l];
        DevLayer& d = m->layers[l];
        char nm[96];
        TRY(dalloc(m.get(), m->allocs, el * 3 * kH * kH, &d.wqkv));
        TRY(dalloc(m.get(), m->allocs, el * kH * kH, &d.wo));
        TRY(dalloc(m.get(), m->allocs, el * kF * kH, &d.w1));
        TRY(dalloc(m.get(), m->allocs, el * kH * kF, &d.w2));
        TRY(dalloc(m.get(), m->allocs, sizeof(float) * 3 * kH, reinterpret_cast<void**>(&d.sqkv)));
        TRY(dalloc(m.get(), m->allocs, sizeof(float) * kH, reinterpret_cast<void**>(&d.so)));
        TRY(dalloc(m.get(), m->allocs, sizeof(float) * kF, reinterpret_cast<void**>(&d.s1)));
        TRY(dalloc(m.get(), m->allocs, sizeof(float) * kH, reinterpret_cast<void**>(&d.s2)));
        snprintf(nm, sizeof nm, "encoder.layer.%d.attention.self.query.weight", l);
        TRY(upload_linear(m.get(), s.query, kH, kH, d.wqkv, 0, d.sqkv, nm));
        snprintf(nm, sizeof nm, "encoder.layer.%d.attention.self.key.weight", l);
        TRY(upload_linear(m.get(), s.key, kH, kH, d.wqkv, kH, d.sqkv, nm));
        snprintf(nm, sizeof nm, "encoder.layer.%d.attention.self.value.weight", l);
        TRY(upload_linear(m.get(), s.value, kH, kH, d.wqkv, 2 * kH, d.sqkv, nm));
        snprintf(nm, sizeof nm, "encoder.layer.%d.attention.output.dense.weight", l);
        TRY(upload_linear(m.get(), s.attn_output, kH, kH, d.wo, 0, d.so, nm));
        snprintf(nm, sizeof nm, "encoder.layer.%d.intermediate.dense.weight", l);
        TRY(upload_linear(m.get(), s.intermediate, kF, kH, d.w1, 0, d.s1, nm));
        snprintf(nm, sizeof nm, "encoder.layer.%d.output.dense.weight", l);
        TRY(upload_linear(m.get(), s.output, kH, kF, d.w2, 0, d.s2, nm));
        TRY(dalloc(m.get(), m->allocs, sizeof(float) * 3 * kH, reinterpret_cast<void**>(&d.bqkv)));
        TRY(s.query_bias && s.key_bias && s.value_bias ? TZ_OK : fail(TZ_EMISSING, "missing attention bias in layer %d", l));
        TRY(h2d(m.get(), d.bqkv, s.query_bias, sizeof(float) * kH));
        TRY(h2d(m.get(), d.bqkv + kH, s.key_bias, sizeof(float) * kH));
        TRY(h2d(m.get(), d.bqkv + 2 * kH, s.value_bias, sizeof(float) * kH));
        TRY(upload_f32(m.get(), s.attn_output_bias, kH, &d.bo, "attention.output.dense.bias"));
        TRY(upload_f32(m.get(), s.intermediate_bias, kF, &d.b1, "intermediate.dense.bias"));
        TRY(upload_f32(m.get(), s.output_bias, kH, &d.b2, "output.dense.bias"));
        TRY(upload_f32(m.get(), s.attn_ln_gamma, kH, &d.ln1g, "attention.output.LayerNorm.weight"));
        TRY(upload_f32(m.get(), s.attn_ln_beta, kH, &d.ln1b, "attention.output.LayerNorm.bias"));
        TRY(upload_f32(m.get(), s.output_ln_gamma, kH, &d.ln2g, "output.LayerNorm.weight"));
        TRY(upload_f32(m.get(), s.output_ln_beta, kH, &d.ln2b, "output.LayerNorm.bias"));
    }
#undef TRY
    TZ_CUDA(cudaDeviceSynchronize());
    release_staging(m.get());
    *out = m.release();
    return TZ_OK;
}

int tz_arctic_free(tz_model_t m) {
    if (!m) return TZ_OK;
    cudaSetDevice(m->device);  // the context may already be gone: touch only the model
    cudaDeviceSynchronize();
    free_workspace(m);
    for (void* p : m->allocs) cudaFree(p);
    for (auto& e : m->ev) cudaEventDestroy(e);
    delete m;
    return TZ_OK;
}

int tz_arctic_reserve(tz_model_t m, int max_batch, int64_t max_tokens) {
    TZ_CHECK(m && max_batch > 0 && max_tokens > 0, TZ_EINVAL, "tz_arctic_reserve: bad arguments");
    return reserve(m, max_batch, max_tokens);
}

int tz_arctic_forward(tz_model_t m, const uint32_t* ids, const int32_t* cu, int batch, float* out) {
    TZ_CHECK(m && batch >= 0 && (batch == 0 || (ids && cu && out)), TZ_EINVAL, "tz_arctic_forward: bad arguments");
    if (batch == 0) return TZ_OK;
    return forward_host(m, ids, cu, batch, out);
}

int tz_arctic_forward_padded(tz_model_t m, const uint32_t* ids, const int32_t* lengths, int batch, int seq, float* out) {
    TZ_CHECK(m && batch >= 0 && seq > 0 && (batch == 0 || (ids && lengths && out)), TZ_EINVAL,
             "tz_arctic_forward_padded: bad arguments");
    if (batch == 0) return TZ_OK;
    std::vector<int32_t> cu(batch + 1, 0);
    int64_t T = 0;
    for (int b = 0; b < batch; ++b) {
        TZ_CHECK(lengths[b] >= 1 && lengths[b] <= seq, TZ_EINVAL, "length %d of row %d outside [1, %d]", lengths[b], b, seq);
        cu[b + 1] = cu[b] + lengths[b];
    }
    T = cu[batch];
    std::vector<uint32_t> packed(static_cast<size_t>(T));
    for (int b = 0; b < batch; ++b) memcpy(&packed[cu[b]], ids + static_cast<int64_t>(b) * seq, sizeof(uint32_t) * lengths[b]);
    return forward_host(m, packed.data(), cu.data(), batch, out);
}

int tz_arctic_forward_device(tz_model_t m, const uint32_t* d_ids, const int32_t* d_cu, int batch, int64_t T, int max_len,
                             float* d_out, tz_stream_t stream) {
    TZ_CHECK(m && batch >= 0 && T >= 0 && max_len >= 1 && max_len <= kP, TZ_EINVAL, "tz_arctic_forward_device: bad arguments");
    if (batch == 0) return TZ_OK;
    TZ_CHECK(d_ids && d_cu && d_out, TZ_EINVAL, "tz_arctic_forward_device: null pointer");
    int rc = reserve(m, batch, T);
    if (rc) return rc;
    TZ_CUDA(cudaSetDevice(m->ctx->device));
    cudaStream_t s = pick_stream(m->ctx, stream);
    m->last_T = T;
    // The legacy / per-thread default streams cannot be captured: launch directly there.
    const bool capturable = m->use_graph && !m->keep_stages && s != cudaStreamLegacy && s != cudaStreamPerThread;
    if (!capturable) return enqueue_forward(m, d_ids, d_cu, batch, T, max_len, d_out, s);
    const bool hit = m->dgraph && m->dkey[0] == d_ids && m->dkey[1] == d_cu && m->dkey[2] == d_out &&
                     m->dkey[3] == static_cast<const void*>(s) && m->dkey_shape[0] == batch && m->dkey_shape[1] == T &&
                     m->dkey_shape[2] == max_len;
    if (!hit) {
        if (m->dgraph) {
            cudaGraphExecDestroy(m->dgraph);
            m->dgraph = nullptr;
        }
        cudaGraph_t gr = nullptr;
        TZ_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        const int crc = enqueue_forward(m, d_ids, d_cu, batch, T, max_len, d_out, s);
        const cudaError_t ee = cudaStreamEndCapture(s, &gr);
        if (crc) {
            if (gr) cudaGraphDestroy(gr);
            return crc;
        }
        if (ee != cudaSuccess) return cuda_fail(ee, "cudaStreamEndCapture");
        const cudaError_t ie = cudaGraphInstantiate(&m->dgraph, gr, 0);
        cudaGraphDestroy(gr);
        if (ie != cudaSuccess) return cuda_fail(ie, "cudaGraphInstantiate");
        m->dkey[0] = d_ids;
        m->dkey[1] = d_cu;
        m->dkey[2] = d_out;
        m->dkey[3] = s;
        m->dkey_shape[0] = batch;
        m->dkey_shape[1] = T;
        m->dkey_shape[2] = max_len;
    }
    TZ_CUDA(cudaGraphLaunch(m->dgraph, s));
    return TZ_OK;
}

int tz_arctic_debug_hidden(tz_model_t m, int stage, float* out, int64_t T) {
    TZ_CHECK(m && out && stage >= 0 && stage <= kLayers + 1, TZ_EINVAL, "tz_arctic_debug_hidden: bad arguments");
    if (!m->keep_stages) {
        m->keep_stages = true;  // takes effect from the next forward
        return fail(TZ_EINVAL, "stage capture was off; it is on from the next forward");
    }
    TZ_CHECK(m->d_stages && T == m->last_T, TZ_EINVAL, "no captured forward with %lld tokens", static_cast<long long>(T));
    // the device copy is in the blocked layout of xblk: download it whole and reorder into [T, 384]
    std::vector<float> blk(static_cast<size_t>(xblk_rows(T)) * kH);
    TZ_CUDA(cudaMemcpyAsync(blk.data(), m->d_stages + static_cast<size_t>(stage) * xblk_rows(m->cap_tokens) * kH,
                            sizeof(float) * blk.size(), cudaMemcpyDeviceToHost, m->ctx->stream));
    TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
    for (int64_t r = 0; r < T; ++r)
        for (int c = 0; c < kH; ++c) out[static_cast<size_t>(r) * kH + c] = blk[static_cast<size_t>(xblk(r, c))];
    return TZ_OK;
}

int tz_arctic_debug_capture(tz_model_t m, int on) {
    TZ_CHECK(m, TZ_EINVAL, "tz_arctic_debug_capture: null model");
    if (static_cast<bool>(on) == m->keep_stages) return TZ_OK;
    TZ_CUDA(cudaSetDevice(m->ctx->device));
    TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
    m->keep_stages = on != 0;
    if (!on) free_workspace(m);  // the next forward re-reserves without the capture buffers
    return TZ_OK;
}

int tz_arctic_set_ffn_fusion(tz_model_t m, int fused) {
    TZ_CHECK(m && (fused == 0 || fused == 1), TZ_EINVAL, "tz_arctic_set_ffn_fusion: bad arguments");
    if ((fused != 0) == m->ffn_fused) return TZ_OK;
    TZ_CUDA(cudaSetDevice(m->ctx->device));
    TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
    drop_graphs(m);  // the captured graphs hold the other launch sequence
    m->ffn_fused = fused != 0;
    return TZ_OK;
}

int tz_arctic_profile(tz_model_t m, int enable) {
    TZ_CHECK(m && enable >= 0, TZ_EINVAL, "tz_arctic_profile: bad arguments");
    TZ_CUDA(cudaSetDevice(m->ctx->device));
    TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
    if (enable && enable > m->prof_slots) {
        for (auto& e : m->ev) cudaEventDestroy(e);
        m->ev.assign(static_cast<size_t>(enable) * 65, nullptr);
        for (auto& e : m->ev) TZ_CUDA(cudaEventCreate(&e));
        m->prof_slots = enable;
    }
    drop_graphs(m);  // the captured graphs carry (or lack) the event nodes: recapture
    m->profile = enable != 0;
    m->prof_fwd = 0;
    m->ev_n = 0;
    return TZ_OK;
}

int tz_arctic_profile_read(tz_model_t m, float* ms, int* launches) {
    TZ_CHECK(m && ms && launches, TZ_EINVAL, "tz_arctic_profile_read: null argument");
    for (int c = 0; c < P_NCLASS; ++c) {
        ms[c] = 0.f;
        launches[c] = 0;
    }
    TZ_CHECK(m->profile && m->prof_fwd > 0 && m->ev_n >= 2, TZ_EINVAL, "no profiled forward recorded");
    TZ_CUDA(cudaSetDevice(m->ctx->device));
    const int sets = static_cast<int>(std::min<int64_t>(m->prof_fwd, m->prof_slots));
    for (int k = 0; k < sets; ++k) {
        const int b = k * 65;
        for (int i = 0; i + 1 < m->ev_n; ++i) {
            float t = 0.f;
            TZ_CUDA(cudaEventSynchronize(m->ev[b + i + 1]));
            TZ_CUDA(cudaEventElapsedTime(&t, m->ev[b + i], m->ev[b + i + 1]));
            const int c = m->ev_cls[i];
            ms[c] += t;
            launches[c] += 1;
        }
    }
    return TZ_OK;
}

int tz_arctic_debug_operand(tz_model_t m, int which, int8_t* q_out, float* scale_out, int64_t T) {
    TZ_CHECK(m && q_out && scale_out && which >= 0 && which < 4, TZ_EINVAL, "tz_arctic_debug_operand: bad arguments");
    TZ_CHECK(m->mode == TZ_QUANT_W8A8, TZ_EINVAL, "tz_arctic_debug_operand: W8A8 models only");
    if (!m->keep_stages) {
        m->keep_stages = true;
        return fail(TZ_EINVAL, "operand capture was off; it is on from the next forward");
    }
    TZ_CHECK(m->d_opq[which] && T == m->last_T, TZ_EINVAL, "no captured forward with %lld tokens", static_cast<long long>(T));
    const int K = gemm_k(which);
    TZ_CUDA(cudaMemcpyAsync(q_out, m->d_opq[which], static_cast<size_t>(T) * K, cudaMemcpyDeviceToHost, m->ctx->stream));
    TZ_CUDA(cudaMemcpyAsync(scale_out, m->d_ops[which], sizeof(float) * T, cudaMemcpyDeviceToHost, m->ctx->stream));
    TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
    return TZ_OK;
}

int tz_arctic_debug_accum(tz_model_t m, int which, int32_t* acc_out, int64_t T) {
    TZ_CHECK(m && acc_out && which >= 0 && which < 4, TZ_EINVAL, "tz_arctic_debug_accum: bad arguments");
    TZ_CHECK(m->mode == TZ_QUANT_W8A8, TZ_EINVAL, "tz_arctic_debug_accum: W8A8 models only");
    if (!m->keep_stages) {
        m->keep_stages = true;
        return fail(TZ_EINVAL, "accumulator capture was off; it is on from the next forward");
    }
    TZ_CHECK(m->d_acc[which] && T == m->last_T, TZ_EINVAL, "no captured forward with %lld tokens", static_cast<long long>(T));
    TZ_CUDA(cudaMemcpyAsync(acc_out, m->d_acc[which], sizeof(int32_t) * static_cast<size_t>(T) * gemm_n(which),
                            cudaMemcpyDeviceToHost, m->ctx->stream));
    TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
    return TZ_OK;
}

int tz_arctic_debug_gemm_input(tz_model_t m, int which, uint16_t* x_out, int64_t T) {
    TZ_CHECK(m && x_out && (which == 1 || which == 3), TZ_EINVAL, "tz_arctic_debug_gemm_input: which must be 1 or 3");
    TZ_CHECK(m->mode == TZ_QUANT_W8A8, TZ_EINVAL, "tz_arctic_debug_gemm_input: W8A8 models only");
    if (!m->keep_stages) {
        m->keep_stages = true;
        return fail(TZ_EINVAL, "input capture was off; it is on from the next forward");
    }
    TZ_CHECK(m->d_in16[which] && T == m->last_T, TZ_EINVAL, "no captured forward with %lld tokens", static_cast<long long>(T));
    TZ_CUDA(cudaMemcpyAsync(x_out, m->d_in16[which], sizeof(uint16_t) * static_cast<size_t>(T) * gemm_k(which),
                            cudaMemcpyDeviceToHost, m->ctx->stream));
    TZ_CUDA(cudaStreamSynchronize(m->ctx->stream));
    return TZ_OK;
}

int tz_arctic_embed_texts(tz_model_t m, tz_tokenizer_t tok, const char* const* texts, const int64_t* lens, int n,
                          float* out) {
    TZ_CHECK(m && tok && n >= 0 && (n == 0 || (texts && lens && out)), TZ_EINVAL, "tz_arctic_embed_texts: bad arguments");
    if (n == 0) return TZ_OK;
    std::vector<uint32_t> ids(static_cast<size_t>(n) * kP);
    std::vector<int32_t> cu(static_cast<size_t>(n) + 1);
    int rc = tz_tokenizer_encode_batch(tok, texts, lens, n, kP, ids.data(), cu.data(), static_cast<int64_t>(ids.size()));
    if (rc) return rc;
    return forward_host(m, ids.data(), cu.data(), n, out);
}

int64_t tz_doc_chunk_count(int64_t tokens) {
    constexpr int64_t kChunk = 510, kOverlap = 50;  // main.zig:784-785
    if (tokens <= kChunk) return 1;
    return 1 + (tokens - kChunk + kOverlap - 1) / (kChunk - kOverlap);
}

int tz_arctic_embed_documents(tz_model_t m, tz_tokenizer_t tok, const char* const* texts, const int64_t* lens, int n,
                              float* out) {
    TZ_CHECK(m && tok && n >= 0 && (n == 0 || (texts && lens && out)), TZ_EINVAL,
             "tz_arctic_embed_documents: bad arguments");
    if (n == 0) return TZ_OK;
    constexpr int64_t kChunk = 510, kStride = 510 - 50;
    const uint32_t cls = tokenizer_cls(tok), sep = tokenizer_sep(tok);
    std::vector<uint32_t> ids, raw;
    std::vector<int32_t> cu(1, 0);
    std::vector<int> doc_off(1, 0);
    for (int d = 0; d < n; ++d) {
        int rc = tokenize_raw(tok, texts[d], lens[d], &raw);
        if (rc) return rc;
        const int64_t T = static_cast<int64_t>(raw.size());
        const int64_t nc = tz_doc_chunk_count(T);
        for (int64_t c = 0; c < nc; ++c) {  // main.zig:869-878: [CLS] ids[start, min(start + 510, T)) [SEP]
            const int64_t a = c * kStride, b = std::min(a + kChunk, T);
            ids.push_back(cls);
            ids.insert(ids.end(), raw.begin() + a, raw.begin() + b);
            ids.push_back(sep);
            TZ_CHECK(ids.size() < (size_t(1) << 31), TZ_EINVAL, "tz_arctic_embed_documents: too many ids in one call");
            cu.push_back(static_cast<int32_t>(ids.size()));
        }
        doc_off.push_back(static_cast<int>(cu.size() - 1));
    }
    const int chunks = static_cast<int>(cu.size() - 1);
    int rc = forward_to_device(m, ids.data(), cu.data(), chunks);
    if (rc) return rc;
    cudaStream_t s = m->ctx->stream;
    int* d_off = nullptr;  // stream-ordered scratch for the document offsets and results
    float* d_doc = nullptr;
    TZ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&d_off), sizeof(int) * (n + 1), s));
    TZ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&d_doc), sizeof(float) * static_cast<size_t>(n) * kH, s));
    cudaError_t e = cudaMemcpyAsync(d_off, doc_off.data(), sizeof(int) * (n + 1), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        doc_mean_l2_kernel<<<n, 128, 0, s>>>(m->out, d_off, d_doc);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d_doc, sizeof(float) * static_cast<size_t>(n) * kH, cudaMemcpyDeviceToHost, s);
    cudaFreeAsync(d_off, s);
    cudaFreeAsync(d_doc, s);
    if (e != cudaSuccess) return cuda_fail(e, "tz_arctic_embed_documents");
    TZ_CUDA(cudaStreamSynchronize(s));
    return read_status(m->ctx, s);
}

}  // extern "C"
