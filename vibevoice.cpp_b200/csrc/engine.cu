// engine.cu -- host side of the B200 Qwen2 path and the exported C ABI.
//
// Mirrors the reference's layer interface (src/qwen2.hpp: Qwen2Hparams,
// Qwen2LayerWeights, ResidentKV) and the stack drivers that call it
// (run_qwen2_stack, src/vibevoice_tts.cpp:363-464; the ASR prefill/decode
// loops, src/vibevoice_asr.cpp:554-652,665-801), but keeps everything on the
// device: weights are uploaded once and repacked, the KV cache is an f16 paged
// pool, positions and the causal mask are computed by the kernels, and a step
// is a fixed sequence of launches on one stream.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cctype>
#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <type_traits>
#include <vector>

#include "../../include/vvq2_capi.h"
#include "common.cuh"
#include "kernels.h"

using namespace vvq2;

namespace {

constexpr int PART_SLOTS = 1024;   // (row, split) attention partial slots (>= GEMV_MAX_M x 64 splits)
constexpr int PREFILL_ROWS_DEFAULT = 16384;  // token rows per tensor-core chunk (VVQ2_PREFILL_ROWS overrides)

// cuTensorMapEncodeTiled from the driver, fetched through the runtime (no -lcuda)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// NCCL, resolved on first use (partitioned contexts only) instead of at
// load time: a process that loads this library before another user of NCCL
// (torch, for one) would otherwise bind its soname first and hand that user
// an older copy.  An NCCL already in the process is reused.
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*CommSplit)(ncclComm_t, int, int, ncclComm_t*, ncclConfig_t*);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
};

const NcclApi* nccl() {
    static NcclApi api;
    static const bool ok = [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
        if (!h) return false;
        bool all = true;
        auto sym = [&](auto& f, const char* name) {
            f = reinterpret_cast<std::remove_reference_t<decltype(f)>>(dlsym(h, name));
            all = all && f;
        };
        sym(api.GetUniqueId, "ncclGetUniqueId");
        sym(api.CommInitRank, "ncclCommInitRank");
        sym(api.CommSplit, "ncclCommSplit");
        sym(api.CommDestroy, "ncclCommDestroy");
        sym(api.AllGather, "ncclAllGather");
        sym(api.AllReduce, "ncclAllReduce");
        sym(api.GroupStart, "ncclGroupStart");
        sym(api.GroupEnd, "ncclGroupEnd");
        return all;
    }();
    return ok ? &api : nullptr;
}

// 2-D f16 activation matrix [rows][cols] (row-major) as a TMA map with a
// 64 x 128 box and the 128-byte swizzle the UMMA descriptors assume
bool make_act_map(CUtensorMap* m, const __half* base, int rows, int cols, int box_rows = 128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || cols % 64 || ((uintptr_t)base & 15) || box_rows < 8 || box_rows > 256) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One layer's K or V pool as a 2-D f16 [rows][hd] TMA map: 64-key x 64-column
// boxes, 128-byte swizzle (the prefill flash-attention operand layout).
bool kv_map_encode(CUtensorMap* m, const __half* base, int64_t rows, int hd) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || hd % 64 || ((uintptr_t)base & 15)) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
    const cuuint32_t box[2] = {64, 64};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Repacked Q8_0 rows ([cols quants][block scales, padded to 16 bytes]) as a
// byte map for the persistent GEMM's raw-weight TMA: box {box_x, box_rows},
// no swizzle; rows past the matrix read as zeros.
bool make_q8_map(CUtensorMap* m, const DevW& w, int box_x, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || w.type != W_Q8_0 || w.row_stride % 16 || ((uintptr_t)w.q & 15) || w.cols % 64) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)w.row_stride, (cuuint64_t)w.rows};
    const cuuint64_t strides[1] = {(cuuint64_t)w.row_stride};
    const cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w.q), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The four weight maps gemm_ws_launch (or, few_rows, gemm_tc_launch) takes
// for Q8_0 (w1 = w0 unless SwiGLU).
bool make_ws_weight_maps(CUtensorMap* wq, const GemmArgs& g, bool few_rows = false) {
    const int r = few_rows ? (g.epi == EPI_SWIGLU ? 64 : 128) : gemm_ws_weight_box_rows(g);
    const DevW& w1 = g.epi == EPI_SWIGLU ? g.w1 : g.w0;
    return make_q8_map(&wq[0], g.w0, 64, r) && make_q8_map(&wq[1], w1, 64, r) && make_q8_map(&wq[2], g.w0, 16, r) &&
           make_q8_map(&wq[3], w1, 16, r);
}

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CU(expr)                                                                        \
    do {                                                                                \
        cudaError_t e_ = (expr);                                                        \
        if (e_ != cudaSuccess)                                                          \
            return fail(VVQ2_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__, #expr,      \
                        cudaGetErrorString(e_));                                        \
    } while (0)

bool type_ok(int t) {
    return t == W_F32 || t == W_F16 || t == W_Q8_0 || t == W_Q5_K || t == W_Q6_K;
}

int block_elems(int t) { return t == W_Q8_0 ? 32 : (t == W_Q5_K || t == W_Q6_K) ? 256 : 1; }
int block_bytes(int t) {
    switch (t) {
        case W_F32: return 4;
        case W_F16: return 2;
        case W_Q8_0: return 34;
        case W_Q5_K: return 176;
        case W_Q6_K: return 210;
        default: return 0;
    }
}

bool is_device_ptr(const void* p) {
    if (!p) return false;
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

struct Owned {
    DevW w;
    std::vector<void*> allocs;
};

}  // namespace

namespace vvq2 {
bool make_kv_map(CUtensorMap* m, const __half* base, int64_t rows, int hd) { return kv_map_encode(m, base, rows, hd); }
}  // namespace vvq2

struct vvq2_ctx {
    vvq2_hparams hp{};
    int device = 0;
    // Multi-GPU partition of the attention (vvq2_partition): rank (g, s) holds
    // KV-head group g (its q heads' QKV rows and attention) and part s of every
    // sequence's keys; O-proj, FFN and lm_head are replicated.
    struct Part {
        int rank = 0, world = 1, seq_parts = 1, head_parts = 1, g = 0, s = 0;
        int nq = 0, nkv = 0;                // heads held locally
        int ffn = 0;                        // FFN intermediate features held locally (split over all ranks)
        ncclComm_t comm = nullptr, pair = nullptr, heads = nullptr;
        // decode-step exchanges over peer memory (peer.cu) instead of NCCL
        PeerArgs px;
        bool peer = false;
        std::vector<void*> ipc;             // other ranks' exchange buffers, opened here
        bool on() const { return world > 1; }
    } pt;
    __half *ATTl = nullptr, *ATTg = nullptr;   // local / gathered attention output (partitioned)
    float *LSEl = nullptr, *LSEg = nullptr;
    RowMeta* meta_rope = nullptr;              // true positions for the RoPE table (partitioned)
    float* Xp = nullptr;                       // partial down-projection rows before the all-reduce
    cudaStream_t stream = nullptr;
    float rope_ts = 0.f;
    struct Layer {
        bool set = false;
        DevW qkv, o, gate, up, down;
        float* attn_norm = nullptr;
        float* ffn_norm = nullptr;
        float* qkv_bias = nullptr;
    };
    std::vector<Layer> layers;
    float* out_norm = nullptr;
    DevW lm_head, tok_embd;
    // per-frame heads around the stack: speech connector and EOS classifier
    struct Head {
        DevW fc1, fc2;
        float *b1 = nullptr, *norm = nullptr, *b2 = nullptr;
        float *xin = nullptr, *mid = nullptr, *out = nullptr;   // [GEMV_MAX_M] rows of in / mid / out
    } conn, eos;
    std::vector<void*> allocs;
    // scratch for up to GEMV_MAX_M activation rows
    float *X = nullptr, *Q = nullptr, *ATT = nullptr, *FA = nullptr, *LOGITS = nullptr;
    // prefill (tensor-core) scratch for up to prefill_rows token rows
    int prefill_rows = PREFILL_ROWS_DEFAULT;
    __half *Xh = nullptr, *ATTh = nullptr, *Ah = nullptr;
    // chunks of more than ws_rows token rows use the persistent GEMM when its
    // tiles fill at least ws_min_tiles CTAs (0: one per SM)
    int ws_rows = 256, ws_min_tiles = 0;
    unsigned long long* tile_best = nullptr;   // many-row lm_head: best key per row and 128-column tile
    size_t tile_best_n = 0;
    float* kpart = nullptr;        // split-K partials of the tensor-core GEMMs
    size_t kpart_elems = 0;
    float2* rope_cs = nullptr;
    float *part = nullptr, *part_ml = nullptr;
    int* counters = nullptr;
    RowMeta* meta = nullptr;
    RowMeta* meta_host = nullptr;   // pinned
    unsigned long long* amax = nullptr;
    int32_t* tok = nullptr;
    int max_splits_cap = 64;
    int max_rows = GEMV_MAX_M;     // activation rows per GEMV launch (shared-memory bound)
    int* err = nullptr;            // device error word written by bounded waits
    std::vector<vvq2_kv*> kvs;   // caches created on this context (released with it)

    // persistent decode-step kernel state: per-KV device layer tables, the
    // flagged hand-over words (cleared to 0, a tag no launch uses), argmax keys
    // and end-of-step counter (zero between launches), launch epoch, abort flag
    uint64_t* mega_ll = nullptr;
    size_t mega_ll_n = 0;
    unsigned long long* mega_amax = nullptr;
    unsigned long long* mega_err_info = nullptr;   // [4] where a persistent step's first failing wait gave up
    unsigned int* mega_done = nullptr;
    unsigned int* epoch = nullptr;
    int* abort_flag = nullptr;
    unsigned long long* mega_trace = nullptr;   // VVQ2_MEGA_TRACE=1: phase timeline of the last step
    int mega_grid = 0;
    struct MegaTable {
        vvq2_kv* kv;
        MegaLayer* d_layers;
    };
    std::vector<MegaTable> mega_tables;

    // measurement: per-launch CUDA events (captured into decode graphs when on)
    struct Rec { int kind; int e0, e1; double bytes; };
    bool prof_on = false;
    std::vector<cudaEvent_t> events;
    double prof_ms[4] = {0, 0, 0, 0}, prof_bytes[4] = {0, 0, 0, 0};
    int64_t prof_n[4] = {0, 0, 0, 0};

    // decode-step CUDA graphs, keyed by (kv, sequence set, length bucket, profiling)
    struct Graph {
        vvq2_kv* kv;
        std::vector<int> seqs;
        int bucket;
        bool prof;
        cudaGraphExec_t exec;
        int kernels;
        std::vector<Rec> recs;
    };
    std::vector<Graph> graphs;
    // c->meta currently holds the next decode step of (meta_kv, meta_seqs)
    vvq2_kv* meta_kv = nullptr;
    std::vector<int> meta_seqs;

    template <class T>
    int alloc(T** p, size_t n) {
        void* q = nullptr;
        cudaError_t e = cudaMalloc(&q, n * sizeof(T) > 0 ? n * sizeof(T) : 16);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(VVQ2_ERR_OUT_OF_MEMORY, "cudaMalloc(%zu): %s", n * sizeof(T), cudaGetErrorString(e));
        }
        allocs.push_back(q);
        *p = static_cast<T*>(q);
        return 0;
    }
};

struct vvq2_kv {
    vvq2_ctx* ctx = nullptr;
    int n_seqs = 0, max_seq = 0, max_pages = 0;
    size_t layer_elems = 0;      // halves per layer per pool
    __half* k = nullptr;
    __half* v = nullptr;
    int* block_table = nullptr;
    std::vector<int> past;
    // Paged caches (vvq2_kv_init_paged): pool_pages pages per layer pool are
    // handed to sequences as they grow and returned when they shrink; every
    // unmapped block-table entry points at page null_page (one more page,
    // zero, never handed out), so a kernel reading past a sequence's pages
    // stays inside the pool.  bt mirrors the device block table.
    bool paged = false;
    int pool_pages = 0, null_page = 0;
    std::vector<int> bt, free_pages;
    KvLayer layer(int li) const {
        KvLayer L;
        L.k = k + (size_t)li * layer_elems;
        L.v = v + (size_t)li * layer_elems;
        L.block_table = block_table;
        L.max_pages = max_pages;
        L.n_kv = ctx->pt.nkv;
        L.hd = ctx->hp.head_dim;
        L.n_pages = (int)(layer_elems / ((size_t)L.n_kv * KV_PAGE * L.hd));
        return L;
    }
};

namespace {

// Host <-> device copy ordered on `st` and complete on return.  (A pageable
// cudaMemcpy may return before its DMA has landed, and the engine's
// non-blocking stream does not wait for the legacy stream.)
cudaError_t copy_on(void* dst, const void* src, size_t n, cudaStream_t st) {
    cudaError_t e = cudaMemcpyAsync(dst, src, n, cudaMemcpyDefault, st);
    return e == cudaSuccess ? cudaStreamSynchronize(st) : e;
}

// Host repack of one GGUF tensor into the device layout (DevW).
int upload_tensor(vvq2_ctx* c, const vvq2_tensor& t, DevW* out, int expect_ne0, int expect_ne1,
                  const char* name) {
    if (!t.data) return fail(VVQ2_ERR_INVALID_ARG, "%s: missing tensor", name);
    if (!type_ok(t.type)) return fail(VVQ2_ERR_NOT_IMPLEMENTED, "%s: ggml type %d not supported", name, t.type);
    if ((expect_ne0 > 0 && t.ne0 != expect_ne0) || (expect_ne1 > 0 && t.ne1 != expect_ne1))
        return fail(VVQ2_ERR_INVALID_ARG, "%s: shape [%lld, %lld], expected [%d, %d]", name,
                    (long long)t.ne0, (long long)t.ne1, expect_ne0, expect_ne1);
    const int be = block_elems(t.type), bb = block_bytes(t.type);
    if (t.ne0 % be) return fail(VVQ2_ERR_INVALID_ARG, "%s: ne0 %lld not a multiple of %d", name, (long long)t.ne0, be);
    const int64_t rows = t.ne1, cols = t.ne0, nb = cols / be;
    const uint8_t* src = static_cast<const uint8_t*>(t.data);
    DevW w;
    w.type = t.type;
    w.rows = (int)rows;
    w.cols = (int)cols;
    std::vector<uint8_t> q;
    std::vector<uint16_t> d;
    switch (t.type) {
        case W_Q8_0:
            // one row = [cols quants][nb f16 scales, padded to 16 bytes]: a run of
            // rows is one contiguous, 16-byte aligned range (one bulk copy).  Quants
            // are stored biased, q + 128 as an unsigned byte: the kernels turn a
            // byte b into the exact float 2^23 + b with one byte permute, so the
            // bias saves them an XOR per word
            w.row_stride = cols + (nb * 2 + 15) / 16 * 16;
            w.d_stride = w.row_stride / 2;
            q.assign((size_t)rows * w.row_stride, 0);
            for (int64_t r = 0; r < rows; ++r)
                for (int64_t b = 0; b < nb; ++b) {
                    const uint8_t* blk = src + ((size_t)r * nb + b) * 34;
                    memcpy(&q[(size_t)r * w.row_stride + cols + b * 2], blk, 2);
                    uint8_t* qd = &q[(size_t)r * w.row_stride + b * 32];
                    for (int i = 0; i < 32; ++i) qd[i] = (uint8_t)(blk[2 + i] ^ 0x80u);   // int8 q -> q + 128
                }
            break;
        case W_Q6_K:
            w.row_stride = nb * Q6K_PACKED;
            w.d_stride = nb;
            q.resize((size_t)rows * w.row_stride);
            d.resize((size_t)rows * nb);
            for (int64_t r = 0; r < rows; ++r)
                for (int64_t b = 0; b < nb; ++b) {
                    const uint8_t* blk = src + ((size_t)r * nb + b) * 210;
                    memcpy(&q[(size_t)r * w.row_stride + b * Q6K_PACKED], blk, Q6K_PACKED);
                    memcpy(&d[(size_t)r * nb + b], blk + 208, 2);
                }
            break;
        default:   // Q5_K blocks (176 B, 16-aligned), F32, F16: as-is
            w.row_stride = nb * bb;
            q.assign(src, src + (size_t)rows * w.row_stride);
            break;
    }
    uint8_t* dq = nullptr;
    if (int rc = c->alloc(&dq, q.size())) return rc;
    CU(copy_on(dq, q.data(), q.size(), c->stream));
    w.q = dq;
    if (t.type == W_Q8_0) w.d = reinterpret_cast<const __half*>(dq + cols);
    if (!d.empty()) {
        __half* dd = nullptr;
        if (int rc = c->alloc(&dd, d.size())) return rc;
        CU(copy_on(dd, d.data(), d.size() * 2, c->stream));
        w.d = dd;
    }
    *out = w;
    return 0;
}

// 1-D f32 vector (norm weights, biases) from any float type
int upload_vec(vvq2_ctx* c, const vvq2_tensor& t, int n, float** out, const char* name) {
    if (!t.data) return fail(VVQ2_ERR_INVALID_ARG, "%s: missing tensor", name);
    if (t.ne0 * std::max<int64_t>(t.ne1, 1) != n)
        return fail(VVQ2_ERR_INVALID_ARG, "%s: %lld elements, expected %d", name, (long long)(t.ne0 * t.ne1), n);
    std::vector<float> h(n);
    if (t.type == W_F32) memcpy(h.data(), t.data, (size_t)n * 4);
    else if (t.type == W_F16) {
        const __half* s = static_cast<const __half*>(t.data);
        for (int i = 0; i < n; ++i) h[i] = __half2float(s[i]);
    } else {
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "%s: vector type %d", name, t.type);
    }
    if (int rc = c->alloc(out, (size_t)n)) return rc;
    CU(copy_on(*out, h.data(), (size_t)n * 4, c->stream));
    return 0;
}

int check_ctx(vvq2_ctx* c) {
    if (!c) return fail(VVQ2_ERR_INVALID_ARG, "null context");
    CU(cudaSetDevice(c->device));
    return 0;
}

cudaStream_t pick_stream(vvq2_ctx* c, void* s) { return s ? static_cast<cudaStream_t>(s) : c->stream; }

// A kernel whose bounded wait gave up leaves a nonzero word; report and clear it.
int check_device_error(vvq2_ctx* c) {
    int e = 0;
    CU(cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        unsigned long long info[4] = {0, 0, 0, 0};
        if (c->mega_err_info) {
            cudaMemcpy(info, c->mega_err_info, sizeof(info), cudaMemcpyDeviceToHost);
            cudaMemsetAsync(c->mega_err_info, 0, sizeof(info), c->stream);
        }
        cudaMemsetAsync(c->err, 0, sizeof(int), c->stream);
        // a persistent step that gave up leaves words of its launch behind:
        // clear them (the next launch's tags differ, but a cleared buffer
        // leaves nothing to mistake) and its argmax / arrival bookkeeping
        if (c->mega_ll) cudaMemsetAsync(c->mega_ll, 0, c->mega_ll_n * sizeof(uint64_t), c->stream);
        if (c->mega_amax) cudaMemsetAsync(c->mega_amax, 0, 2 * sizeof(unsigned long long), c->stream);
        if (c->mega_done) cudaMemsetAsync(c->mega_done, 0, sizeof(unsigned int), c->stream);
        if (c->abort_flag) cudaMemsetAsync(c->abort_flag, 0, sizeof(int), c->stream);
        if (c->counters) cudaMemsetAsync(c->counters, 0, sizeof(int) * c->prefill_rows * c->hp.n_kv_heads, c->stream);
        cudaStreamSynchronize(c->stream);
        if (info[0])
            return fail(VVQ2_ERR_CUDA,
                        "a device-side wait timed out (code %d; persistent step: CTA %u, word %lld, tag %u, epoch %u, seen %016llx)",
                        e, (unsigned)(info[0] >> 32), (long long)info[1], (unsigned)info[2], (unsigned)(info[2] >> 32),
                        info[3]);
        return fail(VVQ2_ERR_CUDA, "a device-side wait timed out (code %d)", e);
    }
    return 0;
}

// Attention split: ~2 CTAs per SM overall, at most max_splits_cap splits per row.
void choose_split(const vvq2_ctx* c, int M, int max_lim, int* split, int* nsplit) {
    const int target = 296;
    const int per_row = std::max(1, target / std::max(1, M * c->hp.n_kv_heads));
    int s = (max_lim + per_row - 1) / per_row;
    s = (std::max(s, KV_PAGE) + KV_PAGE - 1) / KV_PAGE * KV_PAGE;   // whole pages per split
    while ((max_lim + s - 1) / s > c->max_splits_cap) s += KV_PAGE;
    *split = s;
    *nsplit = (max_lim + s - 1) / s;
}

// Algorithmic bytes of a weight matrix: its GGUF size (the padding of the
// device layout is not counted).
size_t weight_bytes(const DevW& w) {
    if (w.type < 0) return 0;
    return (size_t)w.rows * (size_t)(w.cols / block_elems(w.type)) * block_bytes(w.type);
}

// Records CUDA events around launches when profiling (kind 0 GEMV, 1 attention).
struct Recorder {
    vvq2_ctx* c;
    cudaStream_t st;
    std::vector<vvq2_ctx::Rec>* recs;
    int e0 = -1;
    // inside stream capture an event record must be an external node
    cudaError_t record(cudaEvent_t e) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) return cudaErrorInvalidValue;
        return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(e, st, cudaEventRecordExternal)
                                                   : cudaEventRecord(e, st);
    }
    cudaError_t begin() {
        if (!recs) return cudaSuccess;
        const int need = (int)recs->size() * 2 + 2;
        if ((int)c->events.size() < need) return cudaErrorInvalidValue;   // created before any capture
        e0 = (int)recs->size() * 2;
        return record(c->events[e0]);
    }
    cudaError_t end(int kind, double bytes) {
        if (!recs) return cudaSuccess;
        cudaError_t err = record(c->events[e0 + 1]);
        recs->push_back({kind, e0, e0 + 1, bytes});
        return err;
    }
};

// One pass over layers for M <= GEMV_MAX_M rows already in c->X with metadata
// in c->meta (device); attention uses `split` keys per CTA on an nsplit grid.
int run_layers_decode(vvq2_ctx* c, vvq2_kv* kv, int M, int split, int nsplit, int first, int n_layers,
                      cudaStream_t st, std::vector<vvq2_ctx::Rec>* recs, double attn_bytes_per_layer) {
    const vvq2_hparams& hp = c->hp;
    const int H = hp.hidden_size, nq = hp.n_heads, nkv = hp.n_kv_heads, hd = hp.head_dim;
    const int F = hp.intermediate_size;
    if (nsplit > c->max_splits_cap)
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "context of %d keys needs %d attention splits (max %d)",
                    nsplit * split, nsplit, c->max_splits_cap);
    Recorder R{c, st, recs};
    auto gemv = [&](const GemvArgs& g, double out_bytes) -> int {
        CU(R.begin());
        CU(gemv_launch(g, st));
        const double b = (double)weight_bytes(g.w0) + (g.epi == EPI_SWIGLU ? (double)weight_bytes(g.w1) : 0.0) +
                         4.0 * M * g.K + out_bytes;
        CU(R.end(0, b));
        return 0;
    };
    for (int li = first; li < first + n_layers; ++li) {
        const vvq2_ctx::Layer& L = c->layers[li];
        const KvLayer kvl = kv->layer(li);
        GemvArgs g;
        g.M = M;
        g.meta = c->meta;
        g.kv = kvl;
        g.n_q_heads = nq;
        g.n_kv_heads = nkv;
        g.hd = hd;
        g.rope_ts = c->rope_ts;
        g.eps = hp.rms_norm_eps;
        // 1. RMSNorm + QKV + bias + RoPE + KV append
        g.w0 = L.qkv;
        g.K = H;
        g.x = c->X;
        g.x_stride = H;
        g.norm_w = L.attn_norm;
        g.bias = L.qkv_bias;
        g.y = c->Q;
        g.y_stride = nq * hd;
        g.epi = EPI_QKV;
        if (int rc = gemv(g, 4.0 * M * nq * hd + 2.0 * M * 2 * nkv * hd)) return rc;
        // 2. attention
        AttnDecodeArgs ad;
        ad.q = c->Q;
        ad.out = c->ATT;
        ad.meta = c->meta;
        ad.kv = kvl;
        ad.M = M;
        ad.nq = nq;
        ad.nkv = nkv;
        ad.hd = hd;
        ad.split = split;
        ad.max_splits = nsplit;
        ad.scale = 1.0f / sqrtf((float)hd);
        ad.part = c->part;
        ad.part_ml = c->part_ml;
        ad.counters = c->counters;
        ad.err = c->err;
        CU(R.begin());
        CU(attn_decode_launch(ad, st));
        CU(R.end(1, attn_bytes_per_layer));
        // 3. O-proj + residual
        GemvArgs o = g;
        o.w0 = L.o;
        o.K = nq * hd;
        o.x = c->ATT;
        o.x_stride = nq * hd;
        o.norm_w = nullptr;
        o.bias = nullptr;
        o.y = c->X;
        o.y_stride = H;
        o.epi = EPI_RESID;
        if (int rc = gemv(o, 8.0 * M * H)) return rc;
        // 4. RMSNorm + gate/up + SwiGLU
        GemvArgs f = g;
        f.w0 = L.gate;
        f.w1 = L.up;
        f.K = H;
        f.x = c->X;
        f.x_stride = H;
        f.norm_w = L.ffn_norm;
        f.bias = nullptr;
        f.y = c->FA;
        f.y_stride = F;
        f.epi = EPI_SWIGLU;
        if (int rc = gemv(f, 4.0 * M * F)) return rc;
        // 5. down + residual
        GemvArgs d = g;
        d.w0 = L.down;
        d.K = F;
        d.x = c->FA;
        d.x_stride = F;
        d.norm_w = nullptr;
        d.bias = nullptr;
        d.y = c->X;
        d.y_stride = H;
        d.epi = EPI_RESID;
        if (int rc = gemv(d, 8.0 * M * H)) return rc;
    }
    return 0;
}

// One pass over layers for M (<= prefill_rows) rows in c->X with metadata in
// c->meta, on the tensor-core path: RMSNorm->f16, tcgen05 GEMMs with fused
// epilogues, and flash attention over each row's causal prefix.
int run_layers_prefill(vvq2_ctx* c, vvq2_kv* kv, int M, int n_seqs, int nt, int max_lim, int first, int n_layers,
                       cudaStream_t st, std::vector<vvq2_ctx::Rec>* recs, double attn_flops) {
    const vvq2_hparams& hp = c->hp;
    Recorder R{c, st, recs};
    // Chunks of more than ws_rows rows run the persistent GEMM (256 weight
    // rows x up to 256 tokens per tile) when its tiles fill the SMs; smaller
    // ones the few-row kernel, split along K when it has few tiles.  Both
    // dequantize the weight blocks in shared memory.
    // norm_w (residual GEMMs only): the RMSNorm -> f16 (c->Xh) that follows;
    // a split-K residual GEMM then folds its reduction into that norm (one
    // pass over the rows) and sets *normed
    auto gemm = [&](const GemmArgs& g, const CUtensorMap& map, const __half* act, const float* norm_w = nullptr,
                    bool* normed = nullptr) -> int {
        if (normed) *normed = false;
        const double n = g.epi == EPI_SWIGLU ? 2.0 * g.N : (double)g.N;
        const int nt = M > c->ws_rows ? gemm_ws_tile_rows(g, c->ws_min_tiles) : 0;
        if (nt) {
            CUtensorMap mt, wq[4];
            if (!make_act_map(&mt, act, M, g.K, nt)) return fail(VVQ2_ERR_CUDA, "activation tensor map");
            if (g.w0.type == W_Q8_0 && !make_ws_weight_maps(wq, g)) return fail(VVQ2_ERR_CUDA, "weight tensor map");
            CU(R.begin());
            CU(gemm_ws_launch(g, mt, wq, nt, st));
            CU(R.end(3, 2.0 * g.T * n * g.K));
            return 0;
        }
        // few output tiles (small N, few rows): split K over more CTAs, then an
        // in-order reduction applies the epilogue
        GemmArgs gg = g;
        const int tiles = (g.N + 127) / 128 * ((g.T + 255) / 256);
        if ((g.epi == EPI_QKV || g.epi == EPI_RESID) && tiles < 74) {
            const int ks = std::min(g.K / 64 / 2, std::max(1, 148 / tiles));
            if (ks > 1) {
                const size_t need = (size_t)ks * g.T * g.N;
                if (need > c->kpart_elems) {
                    if (int rc = c->alloc(&c->kpart, need)) return rc;
                    c->kpart_elems = need;
                }
                gg.kpart = c->kpart;
                gg.k_splits = ks;
            }
        }
        CUtensorMap wq[4];
        if (g.w0.type == W_Q8_0 && !make_ws_weight_maps(wq, g, true)) return fail(VVQ2_ERR_CUDA, "weight tensor map");
        CU(R.begin());
        CU(gemm_tc_launch(gg, map, wq, st));
        if (gg.kpart && gg.epi == EPI_RESID && norm_w && normed) {
            CU(splitk_resid_rmsnorm_f16_launch(gg.kpart, gg.k_splits, gg.bias, c->X, norm_w, M, g.N,
                                               hp.rms_norm_eps, c->Xh, st));
            *normed = true;
        } else if (gg.kpart) {
            CU(splitk_epilogue_launch(gg, st));
        }
        CU(R.end(3, 2.0 * g.T * n * g.K));
        return 0;
    };
    const int H = hp.hidden_size, hd = hp.head_dim;
    const int nq = c->pt.nq, nkv = c->pt.nkv;          // heads this rank holds (all, unpartitioned)
    const int F = c->pt.ffn, qw = hp.n_heads * hd, qw_l = nq * hd;   // F: this rank's FFN features
    const bool parted = c->pt.on();
    // one-token rows of one or two sequences (a partitioned decode step): the
    // linears are bandwidth-bound GEMVs, not 128-row tensor-core tiles
    const bool gv = nt == 1 && M <= 2 && M <= c->max_rows;
    GemvArgs gvb;
    gvb.M = M;
    gvb.meta = c->meta;
    gvb.rope_meta = parted ? c->meta_rope : nullptr;
    gvb.n_q_heads = nq;
    gvb.n_kv_heads = nkv;
    gvb.hd = hd;
    gvb.rope_ts = c->rope_ts;
    gvb.eps = hp.rms_norm_eps;
    auto gemv = [&](const GemvArgs& g) -> int {
        CU(R.begin());
        CU(gemv_launch(g, st));
        CU(R.end(0, (double)weight_bytes(g.w0) + (g.epi == EPI_SWIGLU ? (double)weight_bytes(g.w1) : 0.0)));
        return 0;
    };
    // RoPE from true positions (a later sequence part shifts meta.pos for its keys)
    CU(rope_table_launch(parted ? c->meta_rope : c->meta, M, hd, c->rope_ts, c->rope_cs, st));
    CUtensorMap mapX, mapA, mapF;
    if (!make_act_map(&mapX, c->Xh, M, H) || !make_act_map(&mapA, c->ATTh, M, qw) || !make_act_map(&mapF, c->Ah, M, F))
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "activation tensor map (dims %d/%d/%d must be multiples of 64)", H, qw, F);
    bool pre_normed = false;   // the next attention norm was done by the previous down projection
    for (int li = first; li < first + n_layers; ++li) {
        const vvq2_ctx::Layer& L = c->layers[li];
        const KvLayer kvl = kv->layer(li);
        GemmArgs g;
        g.T = M;
        g.meta = c->meta;
        g.kv = kvl;
        g.nq = nq;
        g.nkv = nkv;
        g.hd = hd;
        g.rope_cs = c->rope_cs;
        g.err = c->err;
        // 1. RMSNorm -> f16, QKV GEMM (+bias, RoPE, K/V append; Q f32)
        if (gv) {
            GemvArgs q = gvb;
            q.kv = kvl;
            q.w0 = L.qkv;
            q.K = H;
            q.x = c->X;
            q.x_stride = H;
            q.norm_w = L.attn_norm;
            q.bias = L.qkv_bias;
            q.y = c->Q;
            q.y_stride = qw_l;
            q.epi = EPI_QKV;
            if (int rc = gemv(q)) return rc;
        } else {
            if (!pre_normed) CU(rmsnorm_f16_launch(c->X, L.attn_norm, M, H, hp.rms_norm_eps, c->Xh, st));
            GemmArgs q = g;
            q.w0 = L.qkv;
            q.N = L.qkv.rows;
            q.K = H;
            q.epi = EPI_QKV;
            q.bias = L.qkv_bias;
            q.y = c->Q;
            q.y_stride = qw_l;
            if (int rc = gemm(q, mapX, c->Xh)) return rc;
        }
        __half* att_out = parted ? c->ATTl : (gv ? nullptr : c->ATTh);   // this rank's heads (gv: f32 c->ATT)
        float* att_lse = c->pt.seq_parts > 1 ? c->LSEl : nullptr;
        // 2. causal attention, f16 output: tcgen05 flash attention for prompt
        //    chunks (head_dim 64/128); rows of one token each (batched decode
        //    of many streams) and other head sizes use the split-K decode kernel
        if ((hd == 64 || hd == 128) && nt > 1) {
            const int64_t kv_rows = (int64_t)(kv->layer_elems / hd);   // every page of the pool
            CUtensorMap mk, mv;
            if (!make_kv_map(&mk, kvl.k, kv_rows, hd) || !make_kv_map(&mv, kvl.v, kv_rows, hd))
                return fail(VVQ2_ERR_CUDA, "kv tensor map");
            FaArgs fa;
            fa.q = c->Q;
            fa.out = att_out;
            fa.lse = att_lse;
            fa.meta = c->meta;
            fa.block_table = kvl.block_table;
            fa.max_pages = kvl.max_pages;
            fa.kv_rows = (int)kv_rows;
            fa.n_seqs = n_seqs;
            fa.nt = nt;
            fa.nq = nq;
            fa.nkv = nkv;
            fa.hd = hd;
            fa.scale = 1.0f / sqrtf((float)hd);
            fa.err = c->err;
            CU(R.begin());
            CU(fa_prefill_launch(fa, mk, mv, st));
            CU(R.end(2, attn_flops));
        } else {
        AttnDecodeArgs ad;
        ad.q = c->Q;
        ad.out_h = att_out;
        ad.out = att_out ? nullptr : c->ATT;
        ad.lse = att_lse;
        ad.meta = c->meta;
        ad.kv = kvl;
        ad.M = M;
        ad.nq = nq;
        ad.nkv = nkv;
        ad.hd = hd;
        if (nt == 1) {
            // partials [row][split] share the decode scratch: rows x splits <= its capacity
            // ~4 CTAs per SM over (row, KV head, split), whole pages per split
            const int want = std::max(1, (4 * 148 + M * nkv - 1) / (M * nkv));
            int split = (max_lim + want - 1) / want;
            split = (std::max(split, KV_PAGE) + KV_PAGE - 1) / KV_PAGE * KV_PAGE;
            int nsplit = (max_lim + split - 1) / split;
            while (nsplit > 1 && (M * nsplit > PART_SLOTS || nsplit > c->max_splits_cap)) {
                split += KV_PAGE;
                nsplit = (max_lim + split - 1) / split;
            }
            ad.split = split;
            ad.max_splits = nsplit;
        } else {
            ad.split = (max_lim + KV_PAGE - 1) / KV_PAGE * KV_PAGE;
            ad.max_splits = 1;
        }
        ad.scale = 1.0f / sqrtf((float)hd);
        ad.part = c->part;
        ad.part_ml = c->part_ml;
        ad.counters = c->counters;
        ad.err = c->err;
        CU(R.begin());
        CU(attn_decode_launch(ad, st));
        // f16 K and V read: 4 bytes per key and head dimension of each KV head
        CU(R.end(1, attn_flops * nkv / nq));
        }
        const bool px = parted && gv && c->pt.peer;   // decode-step exchanges over peer memory
        if (px) {
            // every rank's heads (both sequence parts merged) -> c->ATT, f32
            CU(peer_attn_gather_launch(c->pt.px, c->ATTl, att_lse, M, nq, hd, c->pt.seq_parts, c->ATT, st));
        } else if (parted) {
            // the two sequence parts of this head group: (O, LSE) all-gather, merge
            if (c->pt.seq_parts > 1) {
                if (nccl()->GroupStart() != ncclSuccess ||
                    nccl()->AllGather(c->ATTl, c->ATTg, (size_t)M * qw_l, ncclHalf, c->pt.pair, st) != ncclSuccess ||
                    nccl()->AllGather(c->LSEl, c->LSEg, (size_t)M * nq, ncclFloat, c->pt.pair, st) != ncclSuccess ||
                    nccl()->GroupEnd() != ncclSuccess)
                    return fail(VVQ2_ERR_CUDA, "NCCL all-gather of (O, LSE) failed");
                CU(lse_merge_launch(c->ATTg, c->LSEg, M, nq, hd, c->ATTl, st));
            }
            // head groups: all-gather the output rows, then [group][row][w] -> [row][all heads]
            if (c->pt.head_parts > 1) {
                if (nccl()->AllGather(c->ATTl, c->ATTg, (size_t)M * qw_l, ncclHalf, c->pt.heads, st) != ncclSuccess)
                    return fail(VVQ2_ERR_CUDA, "NCCL all-gather of attention rows failed");
                CU(gather_rows_launch(c->ATTg, M, c->pt.head_parts, qw_l, c->ATTh, st));
            } else {
                CU(cudaMemcpyAsync(c->ATTh, c->ATTl, sizeof(__half) * M * qw, cudaMemcpyDeviceToDevice, st));
            }
        }
        if (gv) {
            // 3-5 as GEMVs: O-proj + residual (replicated), RMSNorm + gate/up +
            // SwiGLU over this rank's features, down (partial sums when partitioned)
            if (parted && !px) CU(half_to_float_launch(c->ATTh, c->ATT, (int64_t)M * qw, st));
            GemvArgs o = gvb;
            o.w0 = L.o;
            o.K = qw;
            o.x = c->ATT;
            o.x_stride = qw;
            o.y = c->X;
            o.y_stride = H;
            o.epi = EPI_RESID;
            if (int rc = gemv(o)) return rc;
            GemvArgs f = gvb;
            f.w0 = L.gate;
            f.w1 = L.up;
            f.K = H;
            f.x = c->X;
            f.x_stride = H;
            f.norm_w = L.ffn_norm;
            f.y = c->FA;
            f.y_stride = F;
            f.epi = EPI_SWIGLU;
            if (int rc = gemv(f)) return rc;
            GemvArgs d = gvb;
            d.w0 = L.down;
            d.K = F;
            d.x = c->FA;
            d.x_stride = F;
            d.y = parted ? c->Xp : c->X;
            d.y_stride = H;
            d.epi = parted ? EPI_STORE : EPI_RESID;
            if (int rc = gemv(d)) return rc;
            if (px) {
                CU(peer_reduce_add_launch(c->pt.px, c->Xp, M * H, c->X, st));
            } else if (parted) {
                if (nccl()->AllReduce(c->Xp, c->Xp, (size_t)M * H, ncclFloat, ncclSum, c->pt.comm, st) != ncclSuccess)
                    return fail(VVQ2_ERR_CUDA, "NCCL all-reduce of the down projection failed");
                CU(add_rows_launch(c->X, c->Xp, (int64_t)M * H, st));
            }
            continue;
        }
        // 3. O-proj + residual (replicated on partitioned ranks)
        GemmArgs o = g;
        o.w0 = L.o;
        o.N = H;
        o.K = qw;
        o.epi = EPI_RESID;
        o.y = c->X;
        o.y_stride = H;
        bool o_normed = false;
        if (int rc = gemm(o, mapA, c->ATTh, L.ffn_norm, &o_normed)) return rc;
        // 4. RMSNorm -> f16, gate/up GEMM with SwiGLU epilogue (f16 out)
        if (!o_normed) CU(rmsnorm_f16_launch(c->X, L.ffn_norm, M, H, hp.rms_norm_eps, c->Xh, st));
        GemmArgs f = g;
        f.w0 = L.gate;
        f.w1 = L.up;
        f.N = F;
        f.K = H;
        f.epi = EPI_SWIGLU;
        f.yh = c->Ah;
        f.yh_stride = F;
        if (int rc = gemm(f, mapX, c->Xh)) return rc;
        // 5. down + residual (partitioned: partial sums over this rank's features,
        //    NCCL all-reduce, then the residual add)
        GemmArgs d = g;
        d.w0 = L.down;
        d.N = H;
        d.K = F;
        d.epi = parted ? EPI_STORE : EPI_RESID;
        d.y = parted ? c->Xp : c->X;
        d.y_stride = H;
        // unpartitioned and not the last layer here: the next layer's attention
        // norm can take the down projection's split-K reduction
        const bool fold = !parted && li + 1 < first + n_layers;
        if (int rc = gemm(d, mapF, c->Ah, fold ? c->layers[li + 1].attn_norm : nullptr, &pre_normed)) return rc;
        if (parted) {
            if (nccl()->AllReduce(c->Xp, c->Xp, (size_t)M * H, ncclFloat, ncclSum, c->pt.comm, st) != ncclSuccess)
                return fail(VVQ2_ERR_CUDA, "NCCL all-reduce of the down projection failed");
            CU(add_rows_launch(c->X, c->Xp, (int64_t)M * H, st));
        }
    }
    return 0;
}

// Whole decode step on the stream: embed(c->tok) -> layers -> output_norm ->
// lm_head -> argmax -> c->tok, then every row's metadata moves one position on.
int enqueue_decode(vvq2_ctx* c, vvq2_kv* kv, int M, int split, int nsplit, cudaStream_t st,
                   std::vector<vvq2_ctx::Rec>* recs, double attn_bytes) {
    const int H = c->hp.hidden_size;
    CU(embed_launch(c->tok_embd, c->tok, M, c->X, st));
    if (int rc = run_layers_decode(c, kv, M, split, nsplit, 0, c->hp.n_layers, st, recs, attn_bytes)) return rc;
    GemvArgs g;
    g.w0 = c->lm_head;
    g.M = M;
    g.K = H;
    g.x = c->X;
    g.x_stride = H;
    g.norm_w = c->out_norm;
    g.eps = c->hp.rms_norm_eps;
    g.y = nullptr;
    g.argmax = c->amax;
    g.epi = EPI_ARGMAX;
    CU(argmax_init_launch(c->amax, M, st));
    Recorder R{c, st, recs};
    CU(R.begin());
    CU(gemv_launch(g, st));
    CU(R.end(0, (double)weight_bytes(c->lm_head) + 4.0 * M * H));
    CU(argmax_final_launch(c->amax, M, c->tok, st));
    CU(advance_meta_launch(c->meta, M, st));
    return 0;
}

// Shared-memory and tile plan of the persistent decode step for M rows.
struct MegaPlan {
    bool ok = false;
    int nstage = 0, slot = 0, uni = 0, t_qkv = 1, t_o = 1, t_gu = 1, t_down = 1, t_lm = 1;
    size_t smem = 0;
};

MegaPlan mega_plan(const vvq2_ctx* c, int M) {
    MegaPlan p;
    const vvq2_hparams& hp = c->hp;
    const int grid = c->mega_grid, ncw = decode_mega_consumer_warps();
    if (grid <= 0 || M < 1 || M > 2 || c->layers.empty()) return p;
    const vvq2_ctx::Layer& L0 = c->layers[0];
    const int kmax = std::max({hp.hidden_size, hp.intermediate_size, hp.n_heads * hp.head_dim});
    p.uni = decode_mega_union_bytes(hp.head_dim, M, kmax, hp.hidden_size);
    const int lim = decode_mega_smem_limit() - decode_mega_table_bytes(hp.n_layers);
    // The ring has D slots per warp (D = 2 preferred): tile i of a CTA goes
    // to warp i % ncw, which streams it into one of its own slots.
    for (int k = decode_mega_max_stages() / ncw; k >= 1; --k) {
        const int nst = k * ncw;
        const int64_t slot_max = (int64_t)(lim - p.uni) / nst / 128 * 128;
        // rows per tile: a power of two that gives every consumer warp a tile
        // and fits a slot
        bool fits = true;
        auto pick = [&](const DevW& w, int cap, int mats) {
            const int rpc = (w.rows + grid - 1) / grid;
            int t = 1;
            while (t * 2 <= cap && t * 2 * ncw <= rpc && (int64_t)t * 2 * mats * w.row_stride <= slot_max) t *= 2;
            if ((int64_t)t * mats * w.row_stride > slot_max) fits = false;
            return t;
        };
        p.t_qkv = pick(L0.qkv, 4, 1);
        p.t_o = pick(L0.o, 4, 1);
        p.t_gu = pick(L0.gate, 2, 2);
        p.t_down = pick(L0.down, 4, 1);
        p.t_lm = pick(c->lm_head, 4, 1);
        if (!fits) continue;
        int64_t slot = std::max<int64_t>({p.t_qkv * L0.qkv.row_stride, p.t_o * L0.o.row_stride,
                                          2 * p.t_gu * L0.gate.row_stride, p.t_down * L0.down.row_stride,
                                          p.t_lm * c->lm_head.row_stride});
        slot = (slot + 127) / 128 * 128;
        p.slot = (int)slot;
        p.nstage = nst;
        p.smem = (size_t)p.uni + (size_t)p.nstage * p.slot + decode_mega_table_bytes(hp.n_layers);
        p.ok = true;
        return p;
    }
    return p;
}

// The persistent decode-step kernel covers Q8_0 models with head_dim 64/128,
// at most 8 q heads per KV head and up to 2 rows (the CFG pair);
// VVQ2_MEGA=0 forces the per-phase graph.
bool mega_eligible(const vvq2_ctx* c, int M) {
    const char* env = std::getenv("VVQ2_MEGA");
    if (env && env[0] == '0') return false;
    if (c->mega_grid <= 0 || M < 1 || M > 2) return false;
    if (c->hp.head_dim != 64 && c->hp.head_dim != 128) return false;
    if (c->hp.n_heads % c->hp.n_kv_heads || c->hp.n_heads / c->hp.n_kv_heads > 8) return false;
    if (c->lm_head.type != W_Q8_0 || c->tok_embd.type != W_Q8_0) return false;
    for (const auto& L : c->layers)
        if (L.qkv.type != W_Q8_0 || L.o.type != W_Q8_0 || L.gate.type != W_Q8_0 || L.up.type != W_Q8_0 ||
            L.down.type != W_Q8_0)
            return false;
    return mega_plan(c, M).ok;
}

// Attention split of the persistent step: every (row, KV head) gets up to
// (attention groups on the GPU) / (rows x KV heads) splits of whole pages.
void mega_split(const vvq2_ctx* c, int M, int max_lim, int* split, int* nsplit) {
    const int groups = decode_mega_att_groups() * c->mega_grid;
    const int per_row = std::max(1, std::min(64, groups / std::max(1, M * c->hp.n_kv_heads)));
    int s = (max_lim + per_row - 1) / per_row;
    s = (std::max(s, KV_PAGE) + KV_PAGE - 1) / KV_PAGE * KV_PAGE;
    while ((max_lim + s - 1) / s > 64) s += KV_PAGE;
    *split = s;
    *nsplit = (max_lim + s - 1) / s;
}

// A token row as this rank sees it.  `rope` gets the true position (RoPE
// table); the returned row has the cache index and key limits of the rank's
// sequence part: pos becomes the cache index of the part's last position <=
// pos (-1 if none), so the kernels' causal limit min(pos + 1, kvlen) counts
// exactly the part's keys at positions <= pos; kvlen the part's positions
// below kvlen; cidx < 0 when the other part stores the row.
RowMeta local_row(const vvq2_ctx* c, int seq, int pos, int cidx, int kvlen, RowMeta* rope) {
    RowMeta r{seq, pos, cidx, kvlen};
    if (rope) *rope = r;
    return c->pt.seq_parts < 2 ? r : zz_local_row(r, c->pt.s);
}

// Greedy decode step for more rows than the GEMV paths take (many streams at
// once): embedding, the stack on the tensor-core path (split-K decode
// attention over each row's ragged KV length), final RMSNorm, and the lm_head
// as a tcgen05 GEMM whose epilogue keeps each row's argmax.
int decode_step_batched(vvq2_ctx* c, vvq2_kv* kv, const int* seqs, int n_seqs, const int32_t* tokens_in,
                        int32_t* tokens_out, cudaStream_t st) {
    const vvq2_hparams& hp = c->hp;
    const int M = n_seqs, H = hp.hidden_size;
    if (M > c->prefill_rows) return fail(VVQ2_ERR_INVALID_ARG, "%d rows > %d per decode step", M, c->prefill_rows);
    int max_lim = 1;
    double attn_flops = 0.0;
    std::vector<RowMeta> rope(c->pt.on() ? M : 0);
    for (int s = 0; s < M; ++s) {
        const int past = kv->past[seqs[s]];
        const RowMeta r = local_row(c, seqs[s], past, past, past + 1, c->pt.on() ? &rope[s] : nullptr);
        c->meta_host[s] = r;
        max_lim = std::max(max_lim, std::min(r.pos + 1, r.kvlen));
        attn_flops += 4.0 * c->pt.nq * hp.head_dim * std::max(0, std::min(r.pos + 1, r.kvlen));
    }
    CU(cudaMemcpyAsync(c->meta, c->meta_host, sizeof(RowMeta) * M, cudaMemcpyHostToDevice, st));
    if (c->pt.on()) CU(copy_on(c->meta_rope, rope.data(), sizeof(RowMeta) * M, st));
    c->meta_kv = nullptr;   // c->meta no longer describes a graph-captured decode step
    CU(cudaMemcpyAsync(c->tok, tokens_in, sizeof(int32_t) * M, cudaMemcpyDefault, st));
    CU(embed_launch(c->tok_embd, c->tok, M, c->X, st));
    std::vector<vvq2_ctx::Rec> recs;
    if (c->prof_on && c->events.size() < 2 * (5 * (size_t)hp.n_layers + 4)) {
        for (size_t i = c->events.size(); i < 2 * (5 * (size_t)hp.n_layers + 4); ++i) {
            cudaEvent_t e;
            CU(cudaEventCreate(&e));
            c->events.push_back(e);
        }
    }
    if (int rc = run_layers_prefill(c, kv, M, M, 1, max_lim, 0, hp.n_layers, st, c->prof_on ? &recs : nullptr,
                                    attn_flops))
        return rc;
    CU(argmax_init_launch(c->amax, M, st));
    if (M <= 2 && M <= c->max_rows) {
        // one or two rows: output norm + lm_head + argmax as one streaming GEMV
        GemvArgs g;
        g.w0 = c->lm_head;
        g.M = M;
        g.K = H;
        g.x = c->X;
        g.x_stride = H;
        g.norm_w = c->out_norm;
        g.eps = hp.rms_norm_eps;
        g.argmax = c->amax;
        g.epi = EPI_ARGMAX;
        Recorder R{c, st, c->prof_on ? &recs : nullptr};
        CU(R.begin());
        CU(gemv_launch(g, st));
        CU(R.end(0, (double)weight_bytes(c->lm_head)));
    } else {
        CU(rmsnorm_f16_launch(c->X, c->out_norm, M, H, hp.rms_norm_eps, c->Xh, st));
        CUtensorMap mapX;
        if (!make_act_map(&mapX, c->Xh, M, H)) return fail(VVQ2_ERR_NOT_IMPLEMENTED, "hidden %d not a multiple of 64", H);
        // f16 operands: each row's candidate tiles (best approximate logit
        // within 1 % of the row's best) are rescored in f32 for the exact
        // argmax.  The f16 logits' error is ~2e-4 of the largest (f16
        // rounding of x and w, 2^-11 each, over K random-sign terms), so the
        // window is some 50 of those errors wide.
        const int ntiles = (c->lm_head.rows + 127) / 128;
        if ((size_t)M * ntiles > c->tile_best_n) {
            if (int rc = c->alloc(&c->tile_best, (size_t)M * ntiles)) return rc;
            c->tile_best_n = (size_t)M * ntiles;
        }
        GemmArgs g;
        g.w0 = c->lm_head;
        g.T = M;
        g.N = c->lm_head.rows;
        g.K = H;
        g.epi = EPI_ARGMAX;
        g.amax = c->amax;
        g.tile_best = c->tile_best;
        g.tile_stride = ntiles;
        g.err = c->err;
        Recorder R{c, st, c->prof_on ? &recs : nullptr};
        CU(R.begin());
        CUtensorMap wq[4];
        if (g.w0.type == W_Q8_0 && !make_ws_weight_maps(wq, g, true)) return fail(VVQ2_ERR_CUDA, "weight tensor map");
        CU(gemm_tc_launch(g, mapX, wq, st));
        CU(R.end(3, 2.0 * M * (double)g.N * H));
        CU(argmax_rescore_launch(c->X, c->out_norm, hp.rms_norm_eps, M, H, c->lm_head, c->tile_best, ntiles,
                                 0.01f, c->amax, c->err, st));
    }
    CU(argmax_final_launch(c->amax, M, c->tok, st));
    CU(cudaMemcpyAsync(tokens_out, c->tok, sizeof(int32_t) * M, cudaMemcpyDefault, st));
    CU(cudaStreamSynchronize(st));   // the meta staging buffer is reused by the next call
    if (int rc = check_device_error(c)) return rc;
    for (const auto& r : recs) {
        float ms = 0.f;
        CU(cudaEventElapsedTime(&ms, c->events[r.e0], c->events[r.e1]));
        c->prof_ms[r.kind] += ms;
        c->prof_bytes[r.kind] += r.bytes;
        c->prof_n[r.kind] += 1;
    }
    for (int s = 0; s < M; ++s) kv->past[seqs[s]] += 1;
    return 0;
}

// Device table of layer descriptors for (ctx, kv); built outside stream capture.
int ensure_mega_table(vvq2_ctx* c, vvq2_kv* kv, MegaLayer** out) {
    MegaLayer* dl = nullptr;
    for (const auto& t : c->mega_tables)
        if (t.kv == kv) dl = t.d_layers;
    if (!dl) {
        std::vector<MegaLayer> h(c->hp.n_layers);
        for (int li = 0; li < c->hp.n_layers; ++li) {
            const vvq2_ctx::Layer& L = c->layers[li];
            h[li].qkv = L.qkv;
            h[li].o = L.o;
            h[li].gate = L.gate;
            h[li].up = L.up;
            h[li].down = L.down;
            h[li].attn_norm = L.attn_norm;
            h[li].ffn_norm = L.ffn_norm;
            h[li].qkv_bias = L.qkv_bias;
            h[li].kv = kv->layer(li);
        }
        if (int rc = c->alloc(&dl, h.size())) return rc;
        CU(copy_on(dl, h.data(), sizeof(MegaLayer) * h.size(), c->stream));
        c->mega_tables.push_back({kv, dl});
    }
    const char* tr = std::getenv("VVQ2_MEGA_TRACE");
    if (tr && tr[0] == '1' && !c->mega_trace) {
        const size_t n = (size_t)mega_trace_slots(c->hp.n_layers) * c->mega_grid;
        if (int rc = c->alloc(&c->mega_trace, n)) return rc;
        CU(cudaMemsetAsync(c->mega_trace, 0, n * sizeof(unsigned long long), c->stream));
        CU(cudaStreamSynchronize(c->stream));
    }
    *out = dl;
    return 0;
}

int enqueue_decode_mega(vvq2_ctx* c, vvq2_kv* kv, int M, int max_lim, cudaStream_t st,
                        std::vector<vvq2_ctx::Rec>* recs, double step_bytes) {
    MegaLayer* dl = nullptr;
    for (const auto& t : c->mega_tables)
        if (t.kv == kv) dl = t.d_layers;
    if (!dl) return fail(VVQ2_ERR_GENERIC, "decode layer table missing");
    const MegaPlan p = mega_plan(c, M);
    if (!p.ok) return fail(VVQ2_ERR_GENERIC, "no shared-memory plan for the persistent step");
    const vvq2_hparams& hp = c->hp;
    MegaArgs a;
    a.layers = dl;
    a.n_layers = hp.n_layers;
    a.H = hp.hidden_size;
    a.F = hp.intermediate_size;
    a.nq = hp.n_heads;
    a.nkv = hp.n_kv_heads;
    a.hd = hp.head_dim;
    a.M = M;
    a.grid = c->mega_grid;
    a.lm_head = c->lm_head;
    a.tok_embd = c->tok_embd;
    a.out_norm = c->out_norm;
    a.qkv_rows = c->layers[0].qkv.rows;
    {
        uint64_t* w = c->mega_ll;
        a.xl = w;
        w += 2 * (size_t)hp.hidden_size;
        a.qkvl = w;
        w += 2 * (size_t)a.qkv_rows;
        a.attl = w;
        w += 2 * (size_t)hp.n_heads * hp.head_dim;
        a.fal = w;
        w += 2 * (size_t)hp.intermediate_size;
        a.pl = w;   // 2 * nq * MEGA_MAX_SPLITS * (hd + 2) words; every offset above is even (16-byte aligned)
    }
    a.meta = c->meta;
    a.tok = c->tok;
    a.amax = c->mega_amax;
    a.done = c->mega_done;
    a.epoch = c->epoch;
    a.abort = c->abort_flag;
    mega_split(c, M, max_lim, &a.split, &a.nsplit);
    a.eps = hp.rms_norm_eps;
    a.rope_ts = c->rope_ts;
    a.scale = 1.0f / sqrtf((float)hp.head_dim);
    a.err = c->err;
    a.err_info = c->mega_err_info;
    a.trace = c->mega_trace;
    a.nstage = p.nstage;
    a.slot_bytes = p.slot;
    a.union_bytes = p.uni;
    a.att_off = decode_mega_att_offset(M, hp.hidden_size);
    a.t_qkv = p.t_qkv;
    a.t_o = p.t_o;
    a.t_gu = p.t_gu;
    a.t_down = p.t_down;
    a.t_lm = p.t_lm;
    Recorder R{c, st, recs};
    CU(R.begin());
    CU(decode_mega_launch(a, p.smem, st));
    CU(R.end(0, step_bytes));
    return 0;
}

}  // namespace

// ======================================================================= C ABI

namespace {

// Upload one per-frame head: fc1 [mid][in] (+ b1), optional norm [mid], fc2
// [out][mid] (+ b2); scratch rows for GEMV_MAX_M frames.
int set_head(vvq2_ctx* c, vvq2_ctx::Head* h, const vvq2_tensor* fc1, const vvq2_tensor* b1, const vvq2_tensor* norm,
             const vvq2_tensor* fc2, const vvq2_tensor* b2, const char* name) {
    if (int rc = check_ctx(c)) return rc;
    if (!fc1 || !fc1->data || !fc2 || !fc2->data) return fail(VVQ2_ERR_INVALID_ARG, "%s: fc1 and fc2 required", name);
    const int in = (int)fc1->ne0, mid = (int)fc1->ne1, out = (int)fc2->ne1;
    if (fc2->ne0 != mid) return fail(VVQ2_ERR_INVALID_ARG, "%s: fc2 ne0 %lld != fc1 rows %d", name, (long long)fc2->ne0, mid);
    vvq2_ctx::Head n;
    if (int rc = upload_tensor(c, *fc1, &n.fc1, in, mid, name)) return rc;
    if (int rc = upload_tensor(c, *fc2, &n.fc2, mid, out, name)) return rc;
    if (b1 && b1->data)
        if (int rc = upload_vec(c, *b1, mid, &n.b1, name)) return rc;
    if (norm && norm->data)
        if (int rc = upload_vec(c, *norm, mid, &n.norm, name)) return rc;
    if (b2 && b2->data)
        if (int rc = upload_vec(c, *b2, out, &n.b2, name)) return rc;
    if (int rc = c->alloc(&n.xin, (size_t)GEMV_MAX_M * in)) return rc;
    if (int rc = c->alloc(&n.mid, (size_t)GEMV_MAX_M * mid)) return rc;
    if (int rc = c->alloc(&n.out, (size_t)GEMV_MAX_M * out)) return rc;
    *h = n;
    return 0;
}

// x [batch][in] -> fc1 (+b1) -> [relu] -> fc2 over [rms_norm * norm] (+b2) -> [sigmoid] -> y
int run_head(vvq2_ctx* c, const vvq2_ctx::Head& h, const float* x, int batch, float* y, bool relu_mid,
             bool sigmoid_out, void* stream, const char* name) {
    if (int rc = check_ctx(c)) return rc;
    if (h.fc1.type < 0) return fail(VVQ2_ERR_INVALID_ARG, "%s: weights not set", name);
    if (!x || !y || batch <= 0 || batch > GEMV_MAX_M)
        return fail(VVQ2_ERR_INVALID_ARG, "%s: batch %d (1..%d) or null buffers", name, batch, GEMV_MAX_M);
    cudaStream_t st = pick_stream(c, stream);
    const int in = h.fc1.cols, mid = h.fc1.rows, out = h.fc2.rows;
    CU(cudaMemcpyAsync(h.xin, x, sizeof(float) * batch * in, cudaMemcpyDefault, st));
    GemvArgs g;
    g.M = batch;
    g.w0 = h.fc1;
    g.K = in;
    g.x = h.xin;
    g.x_stride = in;
    g.bias = h.b1;
    g.y = h.mid;
    g.y_stride = mid;
    g.epi = EPI_STORE;
    if (gemv_launch(g, st) != cudaSuccess)
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "%s: fc1 [%d x %d] not supported by the GEMV", name, mid, in);
    if (relu_mid) CU(act_launch(h.mid, (int64_t)batch * mid, ACT_RELU, st));
    GemvArgs f = g;
    f.w0 = h.fc2;
    f.K = mid;
    f.x = h.mid;
    f.x_stride = mid;
    f.norm_w = h.norm;   // ggml_rms_norm(eps 1e-6) * norm, fused into the GEMV's staging
    f.eps = 1e-6f;
    f.bias = h.b2;
    f.y = h.out;
    f.y_stride = out;
    if (gemv_launch(f, st) != cudaSuccess)
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "%s: fc2 [%d x %d] not supported by the GEMV", name, out, mid);
    if (sigmoid_out) CU(act_launch(h.out, (int64_t)batch * out, ACT_SIGMOID, st));
    CU(cudaMemcpyAsync(y, h.out, sizeof(float) * batch * out, cudaMemcpyDefault, st));
    if (!is_device_ptr(y)) CU(cudaStreamSynchronize(st));
    return 0;
}

}  // namespace

extern "C" {

int vvq2_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int ok = 0;
    for (int i = 0; i < n; ++i) {
        cudaDeviceProp p{};
        if (cudaGetDeviceProperties(&p, i) == cudaSuccess && p.major == 10) ++ok;
    }
    return ok;
}

int vvq2_backend_selected(void) {
    const char* env = std::getenv("VIBEVOICE_BACKEND");
    if (!env) return 0;
    std::string s(env);
    for (auto& ch : s) ch = (char)std::tolower((unsigned char)ch);
    if (s != "b200" && s != "vvq2") return 0;
    return vvq2_device_count() > 0 ? 1 : 0;
}

const char* vvq2_version(void) { return "vvq2 0.1 (sm_100a)"; }
const char* vvq2_last_error(void) { return g_err.c_str(); }
int64_t vvq2_kernel_launches(void) { return (int64_t)launch_count(); }

int vvq2_init(const vvq2_hparams* hp, int device, vvq2_ctx** out) {
    if (!hp || !out) return fail(VVQ2_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    if (hp->hidden_size <= 0 || hp->n_heads <= 0 || hp->n_kv_heads <= 0 || hp->head_dim <= 0 ||
        hp->n_layers <= 0 || hp->n_heads % hp->n_kv_heads)
        return fail(VVQ2_ERR_INVALID_ARG, "bad hparams");
    if (hp->head_dim != 32 && hp->head_dim != 64 && hp->head_dim != 128)
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "head_dim %d (32, 64 and 128 supported)", hp->head_dim);
    if (hp->n_heads / hp->n_kv_heads > 8)
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "GQA group %d > 8", hp->n_heads / hp->n_kv_heads);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return fail(VVQ2_ERR_NO_DEVICE, "no CUDA device %d", device);
    }
    cudaDeviceProp p{};
    CU(cudaGetDeviceProperties(&p, device));
    if (p.major != 10) return fail(VVQ2_ERR_NO_DEVICE, "device %d is sm_%d%d, need sm_100", device, p.major, p.minor);
    CU(cudaSetDevice(device));
    CU(gemv_prepare());
    CU(decode_mega_prepare());
    CU(attn_decode_prepare());
    vvq2_ctx* c = new vvq2_ctx();
    c->hp = *hp;
    c->device = device;
    c->layers.resize(hp->n_layers);
    c->pt.nq = hp->n_heads;
    c->pt.nkv = hp->n_kv_heads;
    c->pt.ffn = hp->intermediate_size;
    c->rope_ts = powf(hp->rope_theta, -2.0f / (float)hp->head_dim);
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return fail(VVQ2_ERR_CUDA, "stream create failed");
    }
    const int M = GEMV_MAX_M;
    if (const char* pr = std::getenv("VVQ2_PREFILL_ROWS")) {
        const int v = atoi(pr);
        if (v >= 256 && v <= 65536) c->prefill_rows = v / 128 * 128;
    }
    if (const char* e = std::getenv("VVQ2_WS_ROWS")) c->ws_rows = std::max(0, atoi(e));
    if (const char* e = std::getenv("VVQ2_WS_MIN_TILES")) c->ws_min_tiles = std::max(1, atoi(e));
    const int P = c->prefill_rows;
    const int qw = hp->n_heads * hp->head_dim;
    const int F = std::max(hp->intermediate_size, 1);
    int rc = 0;
    if (cudaSuccess != gemm_tc_prepare() || cudaSuccess != gemm_ws_prepare())
        rc = fail(VVQ2_ERR_CUDA, "gemm prepare failed");
    if (!rc && cudaSuccess != fa_prefill_prepare()) rc = fail(VVQ2_ERR_CUDA, "flash attention prepare failed");
    if (!encode_fn()) rc = rc ? rc : fail(VVQ2_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    rc = rc ? rc : c->alloc(&c->X, (size_t)P * hp->hidden_size);
    rc = rc ? rc : c->alloc(&c->Q, (size_t)P * qw);
    rc = rc ? rc : c->alloc(&c->Xh, (size_t)P * std::max(hp->hidden_size, qw));
    rc = rc ? rc : c->alloc(&c->ATTh, (size_t)P * qw);
    rc = rc ? rc : c->alloc(&c->Ah, (size_t)P * F);
    rc = rc ? rc : c->alloc(&c->rope_cs, (size_t)P * hp->head_dim / 2);
    rc = rc ? rc : c->alloc(&c->ATT, (size_t)M * qw);
    rc = rc ? rc : c->alloc(&c->FA, (size_t)M * F);
    // attention partials: decode rows x splits, or batched-decode rows x splits (<= PART_SLOTS)
    rc = rc ? rc : c->alloc(&c->part, (size_t)PART_SLOTS * qw);
    rc = rc ? rc : c->alloc(&c->part_ml, (size_t)PART_SLOTS * hp->n_heads * 2);
    rc = rc ? rc : c->alloc(&c->counters, (size_t)P * hp->n_kv_heads);   // batched decode: one per (row, KV head)
    rc = rc ? rc : c->alloc(&c->meta, (size_t)P);
    rc = rc ? rc : c->alloc(&c->amax, (size_t)P);   // batched decode: one key / token per row
    rc = rc ? rc : c->alloc(&c->tok, (size_t)P);
    rc = rc ? rc : c->alloc(&c->err, (size_t)1);
    c->mega_ll_n = mega_ll_words(hp->hidden_size, (hp->n_heads + 2 * hp->n_kv_heads) * hp->head_dim, hp->n_heads,
                                 hp->head_dim, F);
    rc = rc ? rc : c->alloc(&c->mega_ll, c->mega_ll_n);
    rc = rc ? rc : c->alloc(&c->mega_amax, (size_t)2);
    rc = rc ? rc : c->alloc(&c->mega_err_info, (size_t)4);
    rc = rc ? rc : c->alloc(&c->mega_done, (size_t)1);
    rc = rc ? rc : c->alloc(&c->epoch, (size_t)1);
    rc = rc ? rc : c->alloc(&c->abort_flag, (size_t)1);
    c->mega_grid = decode_mega_grid();
    c->max_rows = std::min(GEMV_MAX_M, gemv_max_rows(std::max({hp->hidden_size, qw, F})));
    if (!rc && hp->vocab_size > 0) rc = c->alloc(&c->LOGITS, (size_t)M * hp->vocab_size);
    if (!rc && cudaMallocHost(&c->meta_host, sizeof(RowMeta) * P) != cudaSuccess)
        rc = fail(VVQ2_ERR_OUT_OF_MEMORY, "pinned alloc failed");
    if (!rc && (cudaMemset(c->counters, 0, sizeof(int) * P * hp->n_kv_heads) != cudaSuccess ||
                cudaMemset(c->err, 0, sizeof(int)) != cudaSuccess ||
                cudaMemset(c->mega_ll, 0, c->mega_ll_n * sizeof(uint64_t)) != cudaSuccess ||
                cudaMemset(c->mega_amax, 0, 2 * sizeof(unsigned long long)) != cudaSuccess ||
                cudaMemset(c->mega_err_info, 0, 4 * sizeof(unsigned long long)) != cudaSuccess ||
                cudaMemset(c->mega_done, 0, sizeof(unsigned int)) != cudaSuccess ||
                cudaMemset(c->epoch, 0, sizeof(unsigned int)) != cudaSuccess ||
                cudaMemset(c->abort_flag, 0, sizeof(int)) != cudaSuccess ||
                cudaDeviceSynchronize() != cudaSuccess))   // the engine stream does not wait for these
        rc = fail(VVQ2_ERR_CUDA, "memset failed");
    if (rc) {
        vvq2_free(c);
        return rc;
    }
    *out = c;
    return 0;
}

void vvq2_free(vvq2_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (auto& g : c->graphs) cudaGraphExecDestroy(g.exec);
    for (cudaEvent_t e : c->events) cudaEventDestroy(e);
    for (void* p : c->pt.ipc) cudaIpcCloseMemHandle(p);
    for (void* p : c->allocs) cudaFree(p);
    // caches outlive nothing: their device memory goes with the context and the
    // handles stay valid only for vvq2_kv_free
    for (vvq2_kv* kv : c->kvs) {
        if (kv->k) cudaFree(kv->k);
        if (kv->v) cudaFree(kv->v);
        if (kv->block_table) cudaFree(kv->block_table);
        kv->k = kv->v = nullptr;
        kv->block_table = nullptr;
        kv->ctx = nullptr;
    }
    if (c->meta_host) cudaFreeHost(c->meta_host);
    for (ncclComm_t m : {c->pt.heads, c->pt.pair, c->pt.comm})
        if (m) nccl()->CommDestroy(m);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

int vvq2_nccl_unique_id(void* out) {
    if (!out) return fail(VVQ2_ERR_INVALID_ARG, "null id buffer");
    static_assert(sizeof(ncclUniqueId) == VVQ2_NCCL_ID_BYTES, "NCCL unique id size");
    ncclUniqueId id;
    if (!nccl()) return fail(VVQ2_ERR_NOT_IMPLEMENTED, "libnccl.so.2 not found");
    if (nccl()->GetUniqueId(&id) != ncclSuccess) return fail(VVQ2_ERR_CUDA, "ncclGetUniqueId failed");
    memcpy(out, &id, sizeof id);
    return 0;
}

// Map every rank's exchange buffer into this process (CUDA IPC handles
// all-gathered over the NCCL communicator) for the decode-step exchanges.
// Returns 1 if the driver refuses (the context then keeps NCCL), a negative
// error code if CUDA or NCCL fails.
static int setup_peer(vvq2_ctx* c) {
    const vvq2_hparams& hp = c->hp;
    vvq2_ctx::Part& P = c->pt;
    if (P.world > PEER_MAX) return 1;
    // a decode step's rows: the partial down projection, or the attention block
    const int rows = 2;
    const int need = std::max(rows * hp.hidden_size * 4, peer_attn_block_bytes(rows, P.nq, hp.head_dim, P.seq_parts));
    PeerArgs& X = P.px;
    X.world = P.world;
    X.rank = P.rank;
    X.slot_bytes = (need + 255) / 256 * 256;
    X.err = c->err;
    uint8_t* buf = nullptr;
    if (int rc = c->alloc(&buf, peer_buffer_bytes(X.slot_bytes))) return rc;
    if (int rc = c->alloc(&X.epoch, 1)) return rc;
    char* hs = nullptr;   // [world][handle]
    if (int rc = c->alloc(&hs, (size_t)P.world * sizeof(cudaIpcMemHandle_t))) return rc;
    cudaIpcMemHandle_t h;
    CU(cudaMemsetAsync(buf, 0, peer_buffer_bytes(X.slot_bytes), c->stream));
    CU(cudaMemsetAsync(X.epoch, 0, sizeof(unsigned int), c->stream));
    if (cudaIpcGetMemHandle(&h, buf) != cudaSuccess) {
        cudaGetLastError();
        return 1;
    }
    CU(cudaMemcpyAsync(hs + (size_t)P.rank * sizeof h, &h, sizeof h, cudaMemcpyHostToDevice, c->stream));
    if (nccl()->AllGather(hs + (size_t)P.rank * sizeof h, hs, sizeof h, ncclChar, P.comm, c->stream) != ncclSuccess)
        return fail(VVQ2_ERR_CUDA, "NCCL all-gather of the exchange buffer handles failed");
    std::vector<cudaIpcMemHandle_t> all(P.world);
    CU(cudaMemcpyAsync(all.data(), hs, P.world * sizeof h, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    X.base[P.rank] = buf;
    for (int r = 0; r < P.world; ++r) {
        if (r == P.rank) continue;
        void* q = nullptr;
        if (cudaIpcOpenMemHandle(&q, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            return 1;
        }
        P.ipc.push_back(q);
        X.base[r] = static_cast<uint8_t*>(q);
    }
    // no rank's first exchange may reach a buffer before its owner cleared it:
    // every rank cleared its own before the all-gather above; one more
    // collective orders the mappings before any exchange
    if (nccl()->AllGather(hs + (size_t)P.rank * sizeof h, hs, sizeof h, ncclChar, P.comm, c->stream) != ncclSuccess)
        return fail(VVQ2_ERR_CUDA, "NCCL all-gather failed");
    CU(cudaStreamSynchronize(c->stream));
    return 0;
}

int vvq2_partition(vvq2_ctx* c, int rank, int world, int seq_parts, const void* nccl_id) {
    if (int rc = check_ctx(c)) return rc;
    const vvq2_hparams& hp = c->hp;
    if (world < 1 || rank < 0 || rank >= world || (seq_parts != 1 && seq_parts != 2) || world % seq_parts)
        return fail(VVQ2_ERR_INVALID_ARG, "bad partition rank %d / world %d / seq_parts %d", rank, world, seq_parts);
    const int hp_parts = world / seq_parts;
    if (hp.n_kv_heads % hp_parts) return fail(VVQ2_ERR_INVALID_ARG, "%d KV heads over %d head groups", hp.n_kv_heads, hp_parts);
    // 64-feature multiples per rank (GEMM K blocks, SwiGLU tiles); the weight
    // type's block alignment of the down columns is checked at vvq2_set_layer
    if (hp.intermediate_size % (world * 64))
        return fail(VVQ2_ERR_INVALID_ARG, "ffn %d not a multiple of %d (64 per rank)", hp.intermediate_size, world * 64);
    for (const auto& L : c->layers)
        if (L.set) return fail(VVQ2_ERR_INVALID_ARG, "vvq2_partition must precede vvq2_set_layer");
    if (!c->kvs.empty()) return fail(VVQ2_ERR_INVALID_ARG, "vvq2_partition must precede vvq2_kv_init");
    if (c->pt.on()) return fail(VVQ2_ERR_INVALID_ARG, "context already partitioned");
    if (world == 1) return 0;
    if (!nccl_id) return fail(VVQ2_ERR_INVALID_ARG, "null NCCL id");
    vvq2_ctx::Part P;
    P.rank = rank;
    P.world = world;
    P.seq_parts = seq_parts;
    P.head_parts = hp_parts;
    P.g = rank / seq_parts;
    P.s = rank % seq_parts;
    P.nq = hp.n_heads / hp_parts;
    P.nkv = hp.n_kv_heads / hp_parts;
    P.ffn = hp.intermediate_size / world;
    CU(cudaSetDevice(c->device));
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof id);
    if (!nccl()) return fail(VVQ2_ERR_NOT_IMPLEMENTED, "libnccl.so.2 not found");
    if (nccl()->CommInitRank(&P.comm, world, id, rank) != ncclSuccess) return fail(VVQ2_ERR_CUDA, "ncclCommInitRank failed");
    // the two ranks of a head group (sequence parts), and the ranks of one part across head groups
    if (seq_parts > 1 && nccl()->CommSplit(P.comm, P.g, P.s, &P.pair, nullptr) != ncclSuccess)
        return fail(VVQ2_ERR_CUDA, "ncclCommSplit (pair) failed");
    if (hp_parts > 1 && nccl()->CommSplit(P.comm, P.s, P.g, &P.heads, nullptr) != ncclSuccess)
        return fail(VVQ2_ERR_CUDA, "ncclCommSplit (heads) failed");
    c->pt = P;
    const size_t rows = (size_t)c->prefill_rows;
    const int qw = hp.n_heads * hp.head_dim;
    if (int rc = c->alloc(&c->ATTl, rows * qw)) return rc;
    if (int rc = c->alloc(&c->ATTg, 2 * rows * qw)) return rc;
    if (int rc = c->alloc(&c->LSEl, rows * hp.n_heads)) return rc;
    if (int rc = c->alloc(&c->LSEg, 2 * rows * hp.n_heads)) return rc;
    if (int rc = c->alloc(&c->meta_rope, rows)) return rc;
    if (int rc = c->alloc(&c->Xp, rows * hp.hidden_size)) return rc;
    const char* pe = std::getenv("VVQ2_PEER");
    if (!(pe && pe[0] == '0')) {
        const int rc = setup_peer(c);
        if (rc < 0) return rc;        // an error code: CUDA or NCCL failed
        c->pt.peer = rc == 0;
        if (rc == 1)                  // the driver refused the mapping: NCCL carries the exchanges
            fprintf(stderr, "vvq2: peer exchange buffers unavailable, decode exchanges use NCCL\n");
    }
    return 0;
}

int vvq2_set_layer(vvq2_ctx* c, int li, const vvq2_layer_weights* w) {
    if (int rc = check_ctx(c)) return rc;
    if (!w || li < 0 || li >= c->hp.n_layers) return fail(VVQ2_ERR_INVALID_ARG, "bad layer %d", li);
    const vvq2_hparams& hp = c->hp;
    const int H = hp.hidden_size, qw = hp.n_heads * hp.head_dim, kvw = hp.n_kv_heads * hp.head_dim;
    const int F = hp.intermediate_size;
    vvq2_ctx::Layer L;
    if (w->attn_q.type != w->attn_k.type || w->attn_q.type != w->attn_v.type)
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "attn_q/k/v types differ");
    // concatenated QKV rows [q; k; v] so one GEMV streams them
    {
        const int t = w->attn_q.type;
        if (!type_ok(t)) return fail(VVQ2_ERR_NOT_IMPLEMENTED, "attn_q type %d", t);
        const size_t rb = (size_t)(H / block_elems(t)) * block_bytes(t);
        if (H % block_elems(t)) return fail(VVQ2_ERR_INVALID_ARG, "hidden %d vs block %d", H, block_elems(t));
        for (const vvq2_tensor* tt : {&w->attn_q, &w->attn_k, &w->attn_v})
            if (!tt->data || tt->ne0 != H) return fail(VVQ2_ERR_INVALID_ARG, "attn q/k/v shape");
        if (w->attn_q.ne1 != qw || w->attn_k.ne1 != kvw || w->attn_v.ne1 != kvw)
            return fail(VVQ2_ERR_INVALID_ARG, "attn q/k/v rows");
        // a partitioned rank keeps the rows of its own heads: q heads
        // [g*nq_l, (g+1)*nq_l), k and v heads [g*nkv_l, (g+1)*nkv_l)
        const int hd = hp.head_dim;
        const int qw_l = c->pt.nq * hd, kvw_l = c->pt.nkv * hd;
        const size_t q0 = (size_t)c->pt.g * qw_l, k0 = (size_t)c->pt.g * kvw_l;
        std::vector<uint8_t> cat(rb * (qw_l + 2 * kvw_l));
        memcpy(cat.data(), static_cast<const uint8_t*>(w->attn_q.data) + rb * q0, rb * qw_l);
        memcpy(cat.data() + rb * qw_l, static_cast<const uint8_t*>(w->attn_k.data) + rb * k0, rb * kvw_l);
        memcpy(cat.data() + rb * (qw_l + kvw_l), static_cast<const uint8_t*>(w->attn_v.data) + rb * k0, rb * kvw_l);
        vvq2_tensor tc{cat.data(), t, H, qw_l + 2 * kvw_l};
        if (int rc = upload_tensor(c, tc, &L.qkv, H, qw_l + 2 * kvw_l, "attn_qkv")) return rc;
        std::vector<float> bias_full(qw + 2 * kvw, 0.0f);
        bool any = false;
        const vvq2_tensor* bs[3] = {&w->attn_q_bias, &w->attn_k_bias, &w->attn_v_bias};
        const int off[3] = {0, qw, qw + kvw}, n[3] = {qw, kvw, kvw};
        for (int i = 0; i < 3; ++i) {
            if (!bs[i]->data) continue;
            any = true;
            if (bs[i]->ne0 * std::max<int64_t>(bs[i]->ne1, 1) != n[i]) return fail(VVQ2_ERR_INVALID_ARG, "bias size");
            if (bs[i]->type == W_F32) memcpy(&bias_full[off[i]], bs[i]->data, (size_t)n[i] * 4);
            else if (bs[i]->type == W_F16)
                for (int j = 0; j < n[i]; ++j) bias_full[off[i] + j] = __half2float(static_cast<const __half*>(bs[i]->data)[j]);
            else return fail(VVQ2_ERR_NOT_IMPLEMENTED, "bias type");
        }
        std::vector<float> bias(qw_l + 2 * kvw_l);
        std::copy(bias_full.begin() + q0, bias_full.begin() + q0 + qw_l, bias.begin());
        std::copy(bias_full.begin() + qw + k0, bias_full.begin() + qw + k0 + kvw_l, bias.begin() + qw_l);
        std::copy(bias_full.begin() + qw + kvw + k0, bias_full.begin() + qw + kvw + k0 + kvw_l,
                  bias.begin() + qw_l + kvw_l);
        if (any) {
            if (int rc = c->alloc(&L.qkv_bias, bias.size())) return rc;
            CU(copy_on(L.qkv_bias, bias.data(), bias.size() * 4, c->stream));
        }
    }
    if (int rc = upload_tensor(c, w->attn_o, &L.o, qw, H, "attn_o")) return rc;
    if (c->pt.on()) {
        // FFN split over all ranks: gate/up rows and down columns [rank*F_l, (rank+1)*F_l)
        const int Fl = c->pt.ffn;
        const size_t f0 = (size_t)c->pt.rank * Fl;
        for (const vvq2_tensor* tt : {&w->ffn_gate, &w->ffn_up, &w->ffn_down})
            if (!tt->data || !type_ok(tt->type)) return fail(VVQ2_ERR_INVALID_ARG, "ffn tensor");
        if (w->ffn_gate.ne0 != H || w->ffn_gate.ne1 != F || w->ffn_up.ne0 != H || w->ffn_up.ne1 != F ||
            w->ffn_down.ne0 != F || w->ffn_down.ne1 != H)
            return fail(VVQ2_ERR_INVALID_ARG, "ffn shapes");
        const size_t rb_g = (size_t)(H / block_elems(w->ffn_gate.type)) * block_bytes(w->ffn_gate.type);
        const size_t rb_u = (size_t)(H / block_elems(w->ffn_up.type)) * block_bytes(w->ffn_up.type);
        vvq2_tensor tg{static_cast<const uint8_t*>(w->ffn_gate.data) + rb_g * f0, w->ffn_gate.type, H, Fl};
        vvq2_tensor tu{static_cast<const uint8_t*>(w->ffn_up.data) + rb_u * f0, w->ffn_up.type, H, Fl};
        if (int rc = upload_tensor(c, tg, &L.gate, H, Fl, "ffn_gate")) return rc;
        if (int rc = upload_tensor(c, tu, &L.up, H, Fl, "ffn_up")) return rc;
        const int dt = w->ffn_down.type, be = block_elems(dt), bb = block_bytes(dt);
        if (f0 % be || Fl % be) return fail(VVQ2_ERR_INVALID_ARG, "ffn slice not block aligned");
        const size_t rb_d = (size_t)(F / be) * bb, sl = (size_t)(Fl / be) * bb;
        std::vector<uint8_t> cols((size_t)H * sl);
        for (int r = 0; r < H; ++r)
            memcpy(cols.data() + (size_t)r * sl,
                   static_cast<const uint8_t*>(w->ffn_down.data) + (size_t)r * rb_d + f0 / be * bb, sl);
        vvq2_tensor td{cols.data(), dt, Fl, H};
        if (int rc = upload_tensor(c, td, &L.down, Fl, H, "ffn_down")) return rc;
    } else {
        if (int rc = upload_tensor(c, w->ffn_gate, &L.gate, H, F, "ffn_gate")) return rc;
        if (int rc = upload_tensor(c, w->ffn_up, &L.up, H, F, "ffn_up")) return rc;
        if (int rc = upload_tensor(c, w->ffn_down, &L.down, F, H, "ffn_down")) return rc;
    }
    if (L.gate.type != L.up.type) return fail(VVQ2_ERR_NOT_IMPLEMENTED, "ffn_gate/up types differ");
    if (int rc = upload_vec(c, w->attn_norm, H, &L.attn_norm, "attn_norm")) return rc;
    if (int rc = upload_vec(c, w->ffn_norm, H, &L.ffn_norm, "ffn_norm")) return rc;
    L.set = true;
    c->layers[li] = L;
    return 0;
}

int vvq2_set_output(vvq2_ctx* c, const vvq2_tensor* on, const vvq2_tensor* lm, const vvq2_tensor* te) {
    if (int rc = check_ctx(c)) return rc;
    const int H = c->hp.hidden_size;
    if (on && on->data)
        if (int rc = upload_vec(c, *on, H, &c->out_norm, "output_norm")) return rc;
    if (lm && lm->data) {
        if (c->hp.vocab_size <= 0 || lm->ne1 != c->hp.vocab_size)
            return fail(VVQ2_ERR_INVALID_ARG, "lm_head rows %lld vs vocab %d", (long long)lm->ne1, c->hp.vocab_size);
        if (int rc = upload_tensor(c, *lm, &c->lm_head, H, (int)lm->ne1, "lm_head")) return rc;
    }
    if (te && te->data) {
        if (lm && te->data == lm->data && te->type == lm->type) c->tok_embd = c->lm_head;   // tied
        else if (int rc = upload_tensor(c, *te, &c->tok_embd, H, (int)te->ne1, "tok_embd")) return rc;
    }
    return 0;
}

static int kv_create(vvq2_ctx* c, int n_seqs, int max_seq, int pool_pages, vvq2_kv** out) {
    if (int rc = check_ctx(c)) return rc;
    if (!out || n_seqs <= 0 || max_seq <= 0 || pool_pages < 0) return fail(VVQ2_ERR_INVALID_ARG, "bad kv size");
    *out = nullptr;
    vvq2_kv* kv = new vvq2_kv();
    kv->ctx = c;
    kv->n_seqs = n_seqs;
    kv->max_seq = max_seq;
    kv->max_pages = (max_seq + KV_PAGE - 1) / KV_PAGE;
    const size_t slots = (size_t)n_seqs * kv->max_pages;   // block-table entries
    kv->paged = pool_pages > 0;
    // identity: page s*max_pages + p of the pool is page p of sequence s
    const size_t pages = kv->paged ? (size_t)pool_pages + 1 : slots;
    kv->pool_pages = kv->paged ? pool_pages : (int)slots;
    kv->null_page = pool_pages;
    kv->layer_elems = pages * c->pt.nkv * KV_PAGE * c->hp.head_dim;   // this rank's KV heads
    const size_t bytes = kv->layer_elems * c->hp.n_layers * sizeof(__half);
    if (cudaMalloc(&kv->k, bytes) != cudaSuccess || cudaMalloc(&kv->v, bytes) != cudaSuccess ||
        cudaMalloc(&kv->block_table, slots * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        vvq2_kv_free(kv);
        return fail(VVQ2_ERR_OUT_OF_MEMORY, "kv cache of %zu bytes", 2 * bytes);
    }
    kv->bt.resize(slots);
    for (size_t i = 0; i < slots; ++i) kv->bt[i] = kv->paged ? kv->null_page : (int)i;
    if (kv->paged) {   // handed out lowest first
        kv->free_pages.resize(pool_pages);
        for (int i = 0; i < pool_pages; ++i) kv->free_pages[i] = pool_pages - 1 - i;
    }
    cudaError_t e = cudaMemsetAsync(kv->k, 0, bytes, c->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->v, 0, bytes, c->stream);
    if (e == cudaSuccess) e = copy_on(kv->block_table, kv->bt.data(), slots * sizeof(int), c->stream);
    if (e != cudaSuccess || cudaGetLastError() != cudaSuccess) {
        vvq2_kv_free(kv);
        return fail(VVQ2_ERR_CUDA, "kv init copy failed");
    }
    kv->past.assign(n_seqs, 0);
    c->kvs.push_back(kv);
    *out = kv;
    return 0;
}

int vvq2_kv_init(vvq2_ctx* c, int n_seqs, int max_seq, vvq2_kv** out) {
    return kv_create(c, n_seqs, max_seq, 0, out);
}

int vvq2_kv_init_paged(vvq2_ctx* c, int n_seqs, int max_seq, int pool_pages, vvq2_kv** out) {
    if (pool_pages <= 0) return fail(VVQ2_ERR_INVALID_ARG, "pool_pages must be positive");
    return kv_create(c, n_seqs, max_seq, pool_pages, out);
}

int vvq2_kv_free_pages(const vvq2_kv* kv) {
    if (!kv) return fail(VVQ2_ERR_INVALID_ARG, "null kv");
    return kv->paged ? (int)kv->free_pages.size() : 0;
}

// Positions of a sequence this rank stores among its first n (all of them
// unless a partitioned context splits sequences into parts).
static int kv_own(const vvq2_kv* kv, int n) {
    const vvq2_ctx* c = kv->ctx;
    return c->pt.seq_parts > 1 ? zz_count(c->pt.s, n) : n;
}

static int kv_push_row(vvq2_kv* kv, int seq, cudaStream_t st) {
    const size_t o = (size_t)seq * kv->max_pages;
    CU(cudaMemcpyAsync(kv->block_table + o, kv->bt.data() + o, kv->max_pages * sizeof(int), cudaMemcpyHostToDevice, st));
    return 0;
}

// Paged cache: give sequence seq pages for its first n positions.  Fails
// (nothing changed) when the pool has too few free pages.
int kv_reserve(vvq2_kv* kv, int seq, int n, cudaStream_t st) {
    if (!kv->paged) return 0;
    const int need = (kv_own(kv, std::min(n, kv->max_seq)) + KV_PAGE - 1) / KV_PAGE;
    int* row = kv->bt.data() + (size_t)seq * kv->max_pages;
    int missing = 0;
    for (int p = 0; p < need; ++p) missing += row[p] == kv->null_page;
    if (!missing) return 0;
    if (missing > (int)kv->free_pages.size())
        return fail(VVQ2_ERR_OUT_OF_MEMORY, "KV page pool exhausted: sequence %d needs %d more pages, %zu free of %d",
                    seq, missing, kv->free_pages.size(), kv->pool_pages);
    for (int p = 0; p < need; ++p)
        if (row[p] == kv->null_page) {
            row[p] = kv->free_pages.back();
            kv->free_pages.pop_back();
        }
    return kv_push_row(kv, seq, st);
}

// Paged cache: return the pages of sequence seq past its first n positions.
static int kv_release(vvq2_kv* kv, int seq, int n, cudaStream_t st) {
    if (!kv->paged) return 0;
    const int keep = (kv_own(kv, n) + KV_PAGE - 1) / KV_PAGE;
    int* row = kv->bt.data() + (size_t)seq * kv->max_pages;
    bool changed = false;
    for (int p = keep; p < kv->max_pages; ++p)
        if (row[p] != kv->null_page) {
            kv->free_pages.push_back(row[p]);
            row[p] = kv->null_page;
            changed = true;
        }
    return changed ? kv_push_row(kv, seq, st) : 0;
}

void vvq2_kv_free(vvq2_kv* kv) {
    if (!kv) return;
    if (kv->ctx) {
        vvq2_ctx* c = kv->ctx;
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
        for (auto& g : c->graphs)
            if (g.kv == kv) cudaGraphExecDestroy(g.exec);
        c->graphs.erase(std::remove_if(c->graphs.begin(), c->graphs.end(),
                                       [kv](const vvq2_ctx::Graph& g) { return g.kv == kv; }),
                        c->graphs.end());
        if (c->meta_kv == kv) c->meta_kv = nullptr;
        c->kvs.erase(std::remove(c->kvs.begin(), c->kvs.end(), kv), c->kvs.end());
        c->mega_tables.erase(std::remove_if(c->mega_tables.begin(), c->mega_tables.end(),
                                            [kv](const vvq2_ctx::MegaTable& t) { return t.kv == kv; }),
                             c->mega_tables.end());
    }
    if (kv->k) cudaFree(kv->k);
    if (kv->v) cudaFree(kv->v);
    if (kv->block_table) cudaFree(kv->block_table);
    delete kv;
}

int vvq2_kv_set_past_len(vvq2_kv* kv, int seq, int past) {
    if (!kv || !kv->ctx || seq < 0 || seq >= kv->n_seqs || past < 0 || past > kv->max_seq)
        return fail(VVQ2_ERR_INVALID_ARG, "bad seq/past_len");
    if (kv->paged) {   // a shorter sequence gives its later pages back; a longer one needs pages
        if (int rc = past < kv->past[seq] ? kv_release(kv, seq, past, kv->ctx->stream)
                                          : kv_reserve(kv, seq, past, kv->ctx->stream))
            return rc;
        CU(cudaStreamSynchronize(kv->ctx->stream));   // the table is current for work on any stream
    }
    kv->past[seq] = past;
    if (kv->ctx && kv->ctx->meta_kv == kv) kv->ctx->meta_kv = nullptr;
    return 0;
}

int vvq2_kv_past_len(const vvq2_kv* kv, int seq) {
    if (!kv || seq < 0 || seq >= kv->n_seqs) return fail(VVQ2_ERR_INVALID_ARG, "bad seq");
    return kv->past[seq];
}

static int kv_xfer(vvq2_kv* kv, int seq, int layer, float* k, float* v, const float* kc, const float* vc,
                   int n_pos, bool upload) {
    if (!kv || !kv->ctx) return fail(VVQ2_ERR_INVALID_ARG, "null or released kv");
    vvq2_ctx* c = kv->ctx;
    if (int rc = check_ctx(c)) return rc;
    if (seq < 0 || seq >= kv->n_seqs || layer < 0 || layer >= c->hp.n_layers || n_pos < 0 || n_pos > kv->max_seq)
        return fail(VVQ2_ERR_INVALID_ARG, "bad kv transfer");
    if (n_pos == 0) return 0;
    if (upload) {
        if (int rc = kv_reserve(kv, seq, n_pos, c->stream)) return rc;
    }
    std::vector<float> lk, lv;   // partitioned upload: this rank's heads and sequence part
    if (c->pt.on()) {
        if (!upload) return fail(VVQ2_ERR_NOT_IMPLEMENTED, "kv read on a partitioned context");
        const int W = c->hp.n_kv_heads * c->hp.head_dim, wl = c->pt.nkv * c->hp.head_dim, c0 = c->pt.g * wl;
        std::vector<float> hk((size_t)n_pos * W), hv((size_t)n_pos * W);
        if (is_device_ptr(kc) || is_device_ptr(vc)) CU(cudaDeviceSynchronize());
        CU(copy_on(hk.data(), kc, hk.size() * 4, c->stream));
        CU(copy_on(hv.data(), vc, hv.size() * 4, c->stream));
        // this rank's KV heads at the positions of its sequence part, in order
        const int own = c->pt.seq_parts > 1 ? zz_count(c->pt.s, n_pos) : n_pos;
        lk.resize((size_t)own * wl);
        lv.resize(lk.size());
        for (int p = 0, i = 0; p < n_pos; ++p) {
            if (c->pt.seq_parts > 1 && zz_part(p) != c->pt.s) continue;
            for (int j = 0; j < wl; ++j) {
                lk[(size_t)i * wl + j] = hk[(size_t)p * W + c0 + j];
                lv[(size_t)i * wl + j] = hv[(size_t)p * W + c0 + j];
            }
            ++i;
        }
        n_pos = own;
        kc = lk.data();
        vc = lv.data();
        if (n_pos == 0) return 0;
    }
    const size_t n = (size_t)n_pos * c->pt.nkv * c->hp.head_dim;
    float *dk = nullptr, *dv = nullptr;
    // device-resident k/v may still be being written on another stream
    if (upload && (is_device_ptr(kc) || is_device_ptr(vc))) CU(cudaDeviceSynchronize());
    CU(cudaMalloc(&dk, n * 4));
    if (cudaMalloc(&dv, n * 4) != cudaSuccess) {
        cudaFree(dk);
        return fail(VVQ2_ERR_OUT_OF_MEMORY, "kv staging");
    }
    cudaError_t e = cudaSuccess;
    if (upload) {
        e = cudaMemcpyAsync(dk, kc, n * 4, cudaMemcpyDefault, c->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(dv, vc, n * 4, cudaMemcpyDefault, c->stream);
        if (e == cudaSuccess) e = kv_upload_launch(kv->layer(layer), seq, dk, dv, n_pos, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    } else {
        e = kv_download_launch(kv->layer(layer), seq, dk, dv, n_pos, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        if (e == cudaSuccess) e = copy_on(k, dk, n * 4, c->stream);
        if (e == cudaSuccess) e = copy_on(v, dv, n * 4, c->stream);
    }
    cudaFree(dk);
    cudaFree(dv);
    if (e != cudaSuccess) return fail(VVQ2_ERR_CUDA, "kv transfer: %s", cudaGetErrorString(e));
    return 0;
}

int vvq2_kv_load_prefix(vvq2_kv* kv, int seq, int layer, const float* k, const float* v, int n_pos) {
    if (!k || !v) return fail(VVQ2_ERR_INVALID_ARG, "null k/v");
    return kv_xfer(kv, seq, layer, nullptr, nullptr, k, v, n_pos, true);
}

int vvq2_kv_read(vvq2_kv* kv, int seq, int layer, float* k, float* v, int n_pos) {
    if (!k || !v) return fail(VVQ2_ERR_INVALID_ARG, "null k/v");
    return kv_xfer(kv, seq, layer, k, v, nullptr, nullptr, n_pos, false);
}

int vvq2_forward(vvq2_ctx* c, vvq2_kv* kv, const int* seqs, int n_seqs, int n_tok, const float* x,
                 const int* pos_start, int first_layer, int n_layers, int flags, float* y, void* stream) {
    if (int rc = check_ctx(c)) return rc;
    if (!kv || kv->ctx != c || !seqs || !x || !pos_start || !y || n_seqs <= 0 || n_tok <= 0)
        return fail(VVQ2_ERR_INVALID_ARG, "bad forward arguments");
    if (first_layer < 0 || n_layers < 0 || first_layer + n_layers > c->hp.n_layers)
        return fail(VVQ2_ERR_INVALID_ARG, "layer range [%d, %d)", first_layer, first_layer + n_layers);
    for (int li = first_layer; li < first_layer + n_layers; ++li)
        if (!c->layers[li].set) return fail(VVQ2_ERR_INVALID_ARG, "layer %d has no weights", li);
    if ((flags & VVQ2_OUTPUT_NORM) && !c->out_norm) return fail(VVQ2_ERR_INVALID_ARG, "no output_norm set");
    std::vector<char> seen(kv->n_seqs, 0);
    for (int s = 0; s < n_seqs; ++s) {
        if (seqs[s] < 0 || seqs[s] >= kv->n_seqs || seen[seqs[s]])
            return fail(VVQ2_ERR_INVALID_ARG, "bad or repeated sequence id %d", seqs[s]);
        seen[seqs[s]] = 1;
        if (kv->past[seqs[s]] + n_tok > kv->max_seq)
            return fail(VVQ2_ERR_INVALID_ARG, "KV overflow: seq %d past %d + %d > max_seq %d", seqs[s],
                        kv->past[seqs[s]], n_tok, kv->max_seq);
        if (pos_start[s] < 0) return fail(VVQ2_ERR_INVALID_ARG, "negative position");
    }
    cudaStream_t st = pick_stream(c, stream);
    for (int s = 0; s < n_seqs; ++s)   // paged cache: pages for the positions this call writes
        if (int rc = kv_reserve(kv, seqs[s], kv->past[seqs[s]] + n_tok, st)) return rc;
    const int H = c->hp.hidden_size;
    const bool x_dev = is_device_ptr(x), y_dev = is_device_ptr(y);
    const bool last_only = (flags & VVQ2_LAST_ONLY) != 0;
    // Token chunks of at most GEMV_MAX_M rows over all sequences; each chunk
    // runs through every layer before the next (resident chunked prefill,
    // the ordering tests/test_qwen2_resident.cpp checks).
    // Few rows: decode GEMV path.  Otherwise tensor-core chunks of up to
    // prefill_rows rows.
    const bool tc_path = n_seqs * n_tok > c->max_rows || c->pt.on();   // partitioned: NCCL on the tensor-core path
    if (n_seqs > c->prefill_rows)
        return fail(VVQ2_ERR_NOT_IMPLEMENTED, "more than %d sequences per call", c->prefill_rows);
    const int tok_per_chunk = std::max(1, (tc_path ? c->prefill_rows : c->max_rows) / n_seqs);
    for (int t0 = 0; t0 < n_tok; t0 += tok_per_chunk) {
        const int nt = std::min(tok_per_chunk, n_tok - t0);
        const int M = n_seqs * nt;
        int max_lim = 1;
        std::vector<RowMeta> rope(c->pt.on() ? M : 0);
        for (int s = 0; s < n_seqs; ++s) {
            for (int t = 0; t < nt; ++t) {
                RowMeta& r = c->meta_host[s * nt + t];
                r = local_row(c, seqs[s], pos_start[s] + t0 + t, kv->past[seqs[s]] + t0 + t,
                              kv->past[seqs[s]] + t0 + nt, c->pt.on() ? &rope[s * nt + t] : nullptr);
                max_lim = std::max(max_lim, std::min(r.pos + 1, r.kvlen));
            }
        }
        CU(cudaMemcpyAsync(c->meta, c->meta_host, sizeof(RowMeta) * M, cudaMemcpyHostToDevice, st));
        if (c->pt.on()) CU(copy_on(c->meta_rope, rope.data(), sizeof(RowMeta) * M, st));
        for (int s = 0; s < n_seqs; ++s)
            CU(cudaMemcpyAsync(c->X + (size_t)s * nt * H, x + ((size_t)s * n_tok + t0) * H,
                               sizeof(float) * nt * H, x_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
        c->meta_kv = nullptr;   // c->meta no longer describes a decode step
        std::vector<vvq2_ctx::Rec> recs;
        if (tc_path && (M > c->max_rows || c->pt.on())) {
            // causal attention flops of one layer (this rank's heads and keys):
            // QK^T and PV, 2 flops per (head, dim, key)
            double attn_flops = 0.0;
            for (int r = 0; r < M; ++r)
                attn_flops += 4.0 * c->pt.nq * c->hp.head_dim *
                              std::max(0, std::min(c->meta_host[r].pos + 1, c->meta_host[r].kvlen));
            if (c->prof_on && c->events.size() < 2 * (5 * (size_t)n_layers + 2)) {
                for (size_t i = c->events.size(); i < 2 * (5 * (size_t)n_layers + 2); ++i) {
                    cudaEvent_t e;
                    CU(cudaEventCreate(&e));
                    c->events.push_back(e);
                }
            }
            if (int rc = run_layers_prefill(c, kv, M, n_seqs, nt, max_lim, first_layer, n_layers, st,
                                            c->prof_on ? &recs : nullptr, attn_flops))
                return rc;
        } else {
            int split = 0, nsplit = 0;
            choose_split(c, M, max_lim, &split, &nsplit);
            if (int rc = run_layers_decode(c, kv, M, split, nsplit, first_layer, n_layers, st, nullptr, 0.0)) return rc;
        }
        if (flags & VVQ2_OUTPUT_NORM) CU(rmsnorm_launch(c->X, c->out_norm, M, H, c->hp.rms_norm_eps, c->X, st));
        const cudaMemcpyKind k = y_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
        for (int s = 0; s < n_seqs; ++s) {
            if (last_only) {
                if (t0 + nt == n_tok)
                    CU(cudaMemcpyAsync(y + (size_t)s * H, c->X + ((size_t)s * nt + nt - 1) * H, sizeof(float) * H, k, st));
            } else {
                CU(cudaMemcpyAsync(y + ((size_t)s * n_tok + t0) * H, c->X + (size_t)s * nt * H,
                                   sizeof(float) * nt * H, k, st));
            }
        }
        // the meta staging buffer is reused by the next chunk
        CU(cudaStreamSynchronize(st));
        if (int rc = check_device_error(c)) return rc;
        for (const auto& r : recs) {
            float ms = 0.f;
            CU(cudaEventElapsedTime(&ms, c->events[r.e0], c->events[r.e1]));
            c->prof_ms[r.kind] += ms;
            c->prof_bytes[r.kind] += r.bytes;
            c->prof_n[r.kind] += 1;
        }
    }
    if (flags & VVQ2_ADVANCE)
        for (int s = 0; s < n_seqs; ++s) kv->past[seqs[s]] += n_tok;
    return 0;
}

int vvq2_lm_head(vvq2_ctx* c, int n, const float* h, float* logits, int32_t* argmax, void* stream) {
    if (int rc = check_ctx(c)) return rc;
    if (c->lm_head.type < 0) return fail(VVQ2_ERR_INVALID_ARG, "no lm_head set");
    if (n <= 0 || !h) return fail(VVQ2_ERR_INVALID_ARG, "bad lm_head arguments");
    cudaStream_t st = pick_stream(c, stream);
    const int H = c->hp.hidden_size, V = c->lm_head.rows;
    const bool h_dev = is_device_ptr(h);
    const int rows_per = gemv_max_rows(H);
    for (int i0 = 0; i0 < n; i0 += rows_per) {
        const int M = std::min(rows_per, n - i0);
        CU(cudaMemcpyAsync(c->X, h + (size_t)i0 * H, sizeof(float) * M * H,
                           h_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
        CU(argmax_init_launch(c->amax, M, st));
        GemvArgs g;
        g.w0 = c->lm_head;
        g.M = M;
        g.K = H;
        g.x = c->X;
        g.x_stride = H;
        g.y = logits ? c->LOGITS : nullptr;
        g.y_stride = V;
        g.argmax = c->amax;
        g.epi = EPI_ARGMAX;
        CU(gemv_launch(g, st));
        CU(argmax_final_launch(c->amax, M, c->tok, st));
        if (argmax)
            CU(cudaMemcpyAsync(argmax + i0, c->tok, sizeof(int32_t) * M,
                               is_device_ptr(argmax) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
        if (logits)
            CU(cudaMemcpyAsync(logits + (size_t)i0 * V, c->LOGITS, sizeof(float) * M * V,
                               is_device_ptr(logits) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
        CU(cudaStreamSynchronize(st));
    }
    return 0;
}

int vvq2_set_connector(vvq2_ctx* c, const vvq2_tensor* fc1_w, const vvq2_tensor* fc1_b, const vvq2_tensor* norm_w,
                       const vvq2_tensor* fc2_w, const vvq2_tensor* fc2_b) {
    if (fc1_w && c && fc2_w && fc2_w->ne1 != c->hp.hidden_size)
        return fail(VVQ2_ERR_INVALID_ARG, "connector output %lld != hidden %d", (long long)fc2_w->ne1, c->hp.hidden_size);
    return set_head(c, c ? &c->conn : nullptr, fc1_w, fc1_b, norm_w, fc2_w, fc2_b, "connector");
}

int vvq2_connector(vvq2_ctx* c, const float* x, int batch, float* y, void* stream) {
    return c ? run_head(c, c->conn, x, batch, y, false, false, stream, "connector") : check_ctx(c);
}

int vvq2_set_eos(vvq2_ctx* c, const vvq2_tensor* fc1_w, const vvq2_tensor* fc1_b, const vvq2_tensor* fc2_w,
                 const vvq2_tensor* fc2_b) {
    if (fc1_w && c && fc1_w->ne0 != c->hp.hidden_size)
        return fail(VVQ2_ERR_INVALID_ARG, "eos input %lld != hidden %d", (long long)fc1_w->ne0, c->hp.hidden_size);
    return set_head(c, c ? &c->eos : nullptr, fc1_w, fc1_b, nullptr, fc2_w, fc2_b, "eos");
}

int vvq2_eos(vvq2_ctx* c, const float* x, int batch, float* p, void* stream) {
    return c ? run_head(c, c->eos, x, batch, p, true, true, stream, "eos") : check_ctx(c);
}

int vvq2_embed(vvq2_ctx* c, int n, const int32_t* tokens, float* out, void* stream) {
    if (int rc = check_ctx(c)) return rc;
    if (c->tok_embd.type < 0) return fail(VVQ2_ERR_INVALID_ARG, "no tok_embd set");
    if (n <= 0 || !tokens || !out) return fail(VVQ2_ERR_INVALID_ARG, "bad embed arguments");
    for (int i = 0; i < n && !is_device_ptr(tokens); ++i)
        if (tokens[i] < 0 || tokens[i] >= c->tok_embd.rows) return fail(VVQ2_ERR_INVALID_ARG, "token id %d", tokens[i]);
    cudaStream_t st = pick_stream(c, stream);
    const int H = c->hp.hidden_size;
    int32_t* dt = nullptr;
    float* dout = nullptr;
    CU(cudaMalloc(&dt, sizeof(int32_t) * n));
    CU(cudaMalloc(&dout, sizeof(float) * n * H));
    cudaError_t e = cudaMemcpyAsync(dt, tokens, sizeof(int32_t) * n, cudaMemcpyDefault, st);
    if (e == cudaSuccess) e = embed_launch(c->tok_embd, dt, n, dout, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout, sizeof(float) * n * H, cudaMemcpyDefault, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFree(dt);
    cudaFree(dout);
    if (e != cudaSuccess) return fail(VVQ2_ERR_CUDA, "embed: %s", cudaGetErrorString(e));
    return 0;
}

// Decode step of a partitioned context for one or two rows, captured as one
// graph: embedding, the layers on the streaming-GEMV path with the
// peer-memory exchanges (no NCCL call inside), the lm_head GEMV + argmax,
// and the device-side advance of the true and the rank's own row tables.
int enqueue_decode_parted(vvq2_ctx* c, vvq2_kv* kv, int M, int bucket, cudaStream_t st) {
    const int H = c->hp.hidden_size;
    CU(embed_launch(c->tok_embd, c->tok, M, c->X, st));
    if (int rc = run_layers_prefill(c, kv, M, M, 1, bucket, 0, c->hp.n_layers, st, nullptr, 0.0)) return rc;
    GemvArgs g;
    g.w0 = c->lm_head;
    g.M = M;
    g.K = H;
    g.x = c->X;
    g.x_stride = H;
    g.norm_w = c->out_norm;
    g.eps = c->hp.rms_norm_eps;
    g.argmax = c->amax;
    g.epi = EPI_ARGMAX;
    CU(argmax_init_launch(c->amax, M, st));
    CU(gemv_launch(g, st));
    CU(argmax_final_launch(c->amax, M, c->tok, st));
    CU(advance_meta_part_launch(c->meta_rope, c->meta, M, c->pt.seq_parts, c->pt.s, st));
    return 0;
}

int vvq2_decode_step(vvq2_ctx* c, vvq2_kv* kv, const int* seqs, int n_seqs, const int32_t* tokens_in,
                     int32_t* tokens_out, void* stream) {
    if (int rc = check_ctx(c)) return rc;
    if (!kv || kv->ctx != c || !seqs || !tokens_in || !tokens_out || n_seqs <= 0)
        return fail(VVQ2_ERR_INVALID_ARG, "bad decode_step arguments");
    if (c->tok_embd.type < 0 || c->lm_head.type < 0 || !c->out_norm)
        return fail(VVQ2_ERR_INVALID_ARG, "decode_step needs output_norm, lm_head and tok_embd");
    for (int li = 0; li < c->hp.n_layers; ++li)
        if (!c->layers[li].set) return fail(VVQ2_ERR_INVALID_ARG, "layer %d has no weights", li);
    std::vector<char> seen(kv->n_seqs, 0);
    for (int s = 0; s < n_seqs; ++s) {
        if (seqs[s] < 0 || seqs[s] >= kv->n_seqs || seen[seqs[s]])
            return fail(VVQ2_ERR_INVALID_ARG, "bad or repeated sequence id");
        seen[seqs[s]] = 1;
        if (kv->past[seqs[s]] + 1 > kv->max_seq) return fail(VVQ2_ERR_INVALID_ARG, "KV overflow");
    }
    cudaStream_t st = pick_stream(c, stream);
    for (int s = 0; s < n_seqs; ++s)   // paged cache: a page for the position this step writes
        if (int rc = kv_reserve(kv, seqs[s], kv->past[seqs[s]] + 1, st)) return rc;
    // partitioned contexts: one or two rows with the peer-memory exchanges run
    // as a captured graph; otherwise the host-driven batched step (NCCL)
    const bool parted = c->pt.on() && c->pt.peer && n_seqs <= 2 && n_seqs <= c->max_rows;
    if (!parted && (n_seqs > c->max_rows || c->pt.on()))
        return decode_step_batched(c, kv, seqs, n_seqs, tokens_in, tokens_out, st);
    const int M = n_seqs;
    std::vector<int> sv(seqs, seqs + n_seqs);
    int max_lim = 1;
    double attn_bytes = 0.0;
    for (int s = 0; s < n_seqs; ++s) {
        max_lim = std::max(max_lim, kv->past[seqs[s]] + 1);
        attn_bytes += 4.0 * (kv->past[seqs[s]] + 1) * c->hp.n_kv_heads * c->hp.head_dim;   // f16 K and V
    }
    attn_bytes += 8.0 * M * c->hp.n_heads * c->hp.head_dim;
    // graphs are specialised per 512-position bucket of the longest row: the
    // attention grid covers the bucket and CTAs past a row's length exit
    const int bucket = (max_lim + 511) / 512 * 512;
    if (c->meta_kv != kv || c->meta_seqs != sv) {
        std::vector<RowMeta> rope(M);
        for (int s = 0; s < n_seqs; ++s) {
            const int past = kv->past[seqs[s]];
            c->meta_host[s] = local_row(c, seqs[s], past, past, past + 1, &rope[s]);
        }
        CU(cudaMemcpyAsync(c->meta, c->meta_host, sizeof(RowMeta) * M, cudaMemcpyHostToDevice, st));
        if (parted) CU(cudaMemcpyAsync(c->meta_rope, rope.data(), sizeof(RowMeta) * M, cudaMemcpyHostToDevice, st));
        c->meta_kv = kv;
        c->meta_seqs = sv;
    }
    vvq2_ctx::Graph* gr = nullptr;
    for (auto& g : c->graphs)
        if (g.kv == kv && g.seqs == sv && g.bucket == bucket && g.prof == c->prof_on) gr = &g;
    if (!gr) {
        int split = 0, nsplit = 0;
        choose_split(c, M, bucket, &split, &nsplit);
        vvq2_ctx::Graph g{kv, sv, bucket, c->prof_on, nullptr, 0, {}};
        const long long k0 = launch_count();
        cudaGraph_t graph = nullptr;
        if (!parted && mega_eligible(c, M)) {
            MegaLayer* dl = nullptr;
            if (int rc = ensure_mega_table(c, kv, &dl)) return rc;
        }
        CU(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc;
        if (parted) {
            rc = enqueue_decode_parted(c, kv, M, bucket, st);
        } else if (mega_eligible(c, M)) {
            double step_bytes = attn_bytes + (double)weight_bytes(c->lm_head);
            for (const auto& L : c->layers)
                step_bytes += (double)(weight_bytes(L.qkv) + weight_bytes(L.o) + weight_bytes(L.gate) +
                                       weight_bytes(L.up) + weight_bytes(L.down));
            step_bytes += (double)attn_bytes * (c->hp.n_layers - 1);   // attn_bytes covers one layer
            rc = enqueue_decode_mega(c, kv, M, bucket, st, c->prof_on ? &g.recs : nullptr, step_bytes);
        } else {
            rc = enqueue_decode(c, kv, M, split, nsplit, st, c->prof_on ? &g.recs : nullptr, attn_bytes);
        }
        cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        CU(e);
        e = cudaGraphInstantiate(&g.exec, graph, 0);
        cudaGraphDestroy(graph);
        CU(e);
        g.kernels = (int)(launch_count() - k0);
        c->graphs.push_back(std::move(g));
        gr = &c->graphs.back();
    }
    CU(cudaMemcpyAsync(c->tok, tokens_in, sizeof(int32_t) * M, cudaMemcpyDefault, st));
    CU(cudaGraphLaunch(gr->exec, st));
    note_launch(gr->kernels);
    CU(cudaMemcpyAsync(tokens_out, c->tok, sizeof(int32_t) * M, cudaMemcpyDefault, st));
    if (c->prof_on) {
        CU(cudaStreamSynchronize(st));
        for (const auto& r : gr->recs) {
            float ms = 0.f;
            CU(cudaEventElapsedTime(&ms, c->events[r.e0], c->events[r.e1]));
            c->prof_ms[r.kind] += ms;
            c->prof_bytes[r.kind] += r.bytes;
            c->prof_n[r.kind] += 1;
        }
    } else if (!is_device_ptr(tokens_out)) {
        CU(cudaStreamSynchronize(st));
        if (int rc = check_device_error(c)) return rc;
    }
    for (int s = 0; s < n_seqs; ++s) kv->past[seqs[s]] += 1;
    return 0;
}

int vvq2_profile(vvq2_ctx* c, int enable) {
    if (int rc = check_ctx(c)) return rc;
    c->prof_on = enable != 0;
    for (int k = 0; k < 4; ++k) c->prof_ms[k] = c->prof_bytes[k] = 0.0, c->prof_n[k] = 0;
    // events are created here, never during stream capture
    const size_t need = 2 * (6 * (size_t)c->hp.n_layers + 8);
    while (c->prof_on && c->events.size() < need) {
        cudaEvent_t e;
        CU(cudaEventCreate(&e));
        c->events.push_back(e);
    }
    return 0;
}

int vvq2_profile_read(vvq2_ctx* c, int kind, double* ms, double* bytes, int64_t* launches) {
    if (int rc = check_ctx(c)) return rc;
    if (kind < 0 || kind > 3) return fail(VVQ2_ERR_INVALID_ARG, "bad profile kind");
    if (ms) *ms = c->prof_ms[kind];
    if (bytes) *bytes = c->prof_bytes[kind];
    if (launches) *launches = c->prof_n[kind];
    return 0;
}

int vvq2_mega_trace(vvq2_ctx* c, uint64_t* out, int64_t cap, int* grid, int* slots) {
    if (int rc = check_ctx(c)) return rc;
    if (!c->mega_trace) return fail(VVQ2_ERR_INVALID_ARG, "no persistent-step trace (set VVQ2_MEGA_TRACE=1)");
    const int sl = mega_trace_slots(c->hp.n_layers);
    const int64_t n = (int64_t)sl * c->mega_grid;
    if (grid) *grid = c->mega_grid;
    if (slots) *slots = sl;
    if (!out) return 0;
    if (cap < n) return fail(VVQ2_ERR_INVALID_ARG, "trace buffer too small");
    CU(cudaDeviceSynchronize());
    CU(cudaMemcpy(out, c->mega_trace, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost));
    return 0;
}

int vvq2_dequantize(int type, const void* src, int64_t n, float* dst) {
    if (!src || !dst || n <= 0 || !type_ok(type) || n % block_elems(type))
        return fail(VVQ2_ERR_INVALID_ARG, "bad dequantize arguments");
    if (vvq2_device_count() == 0) return fail(VVQ2_ERR_NO_DEVICE, "no sm_100 device");
    // treat as one row of n elements; reuse the weight upload (repack) path
    vvq2_ctx tmp;
    vvq2_tensor t{src, type, n, 1};
    DevW w;
    int rc = upload_tensor(&tmp, t, &w, 0, 0, "dequantize");
    float* d = nullptr;
    if (!rc) rc = tmp.alloc(&d, (size_t)n);
    cudaError_t e = cudaSuccess;
    if (!rc) e = dequant_rows_launch(w, d, 0);
    if (!rc && e == cudaSuccess) e = cudaMemcpy(dst, d, sizeof(float) * n, cudaMemcpyDefault);
    for (void* p : tmp.allocs) cudaFree(p);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(VVQ2_ERR_CUDA, "dequantize: %s", cudaGetErrorString(e));
    return 0;
}

int vvq2_rope_neox(const float* x, int n_tok, int n_heads, int hd, const int32_t* pos, float theta, float* y) {
    if (!x || !pos || !y || n_tok <= 0 || n_heads <= 0 || hd <= 0 || hd % 2)
        return fail(VVQ2_ERR_INVALID_ARG, "bad rope arguments");
    if (vvq2_device_count() == 0) return fail(VVQ2_ERR_NO_DEVICE, "no sm_100 device");
    const size_t n = (size_t)n_tok * n_heads * hd;
    float *dx = nullptr, *dy = nullptr;
    int32_t* dp = nullptr;
    CU(cudaMalloc(&dx, n * 4));
    CU(cudaMalloc(&dy, n * 4));
    CU(cudaMalloc(&dp, (size_t)n_tok * 4));
    cudaError_t e = cudaMemcpy(dx, x, n * 4, cudaMemcpyDefault);
    if (e == cudaSuccess) e = cudaMemcpy(dp, pos, (size_t)n_tok * 4, cudaMemcpyDefault);
    if (e == cudaSuccess) e = rope_launch(dx, n_tok, n_heads, hd, dp, powf(theta, -2.0f / (float)hd), dy, 0);
    if (e == cudaSuccess) e = cudaMemcpy(y, dy, n * 4, cudaMemcpyDefault);
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(dp);
    if (e != cudaSuccess) return fail(VVQ2_ERR_CUDA, "rope: %s", cudaGetErrorString(e));
    return 0;
}

int vvq2_rms_norm(const float* x, const float* w, int rows, int n, float eps, float* y) {
    if (!x || !w || !y || rows <= 0 || n <= 0) return fail(VVQ2_ERR_INVALID_ARG, "bad rms_norm arguments");
    if (vvq2_device_count() == 0) return fail(VVQ2_ERR_NO_DEVICE, "no sm_100 device");
    const size_t nx = (size_t)rows * n;
    float *dx = nullptr, *dw = nullptr;
    CU(cudaMalloc(&dx, nx * 4));
    CU(cudaMalloc(&dw, (size_t)n * 4));
    cudaError_t e = cudaMemcpy(dx, x, nx * 4, cudaMemcpyDefault);
    if (e == cudaSuccess) e = cudaMemcpy(dw, w, (size_t)n * 4, cudaMemcpyDefault);
    if (e == cudaSuccess) e = rmsnorm_launch(dx, dw, rows, n, eps, dx, 0);
    if (e == cudaSuccess) e = cudaMemcpy(y, dx, nx * 4, cudaMemcpyDefault);
    cudaFree(dx);
    cudaFree(dw);
    if (e != cudaSuccess) return fail(VVQ2_ERR_CUDA, "rms_norm: %s", cudaGetErrorString(e));
    return 0;
}

int vvq2_debug_gemm(int type, const void* w, int n, int k, const float* x, int t, float* y) {
    if (!w || !x || !y || n <= 0 || k <= 0 || t <= 0 || k % 64) return fail(VVQ2_ERR_INVALID_ARG, "bad gemm args");
    if (vvq2_device_count() == 0) return fail(VVQ2_ERR_NO_DEVICE, "no sm_100 device");
    if (gemm_tc_prepare() != cudaSuccess || gemm_ws_prepare() != cudaSuccess)
        return fail(VVQ2_ERR_CUDA, "gemm prepare failed");
    vvq2_ctx tmp;
    vvq2_tensor tw{w, type, k, n};
    DevW dw;
    int rc = upload_tensor(&tmp, tw, &dw, 0, 0, "debug_gemm");
    float *dx = nullptr, *dy = nullptr;
    __half* dxh = nullptr;
    int* derr = nullptr;
    if (!rc) rc = tmp.alloc(&dx, (size_t)t * k);
    if (!rc) rc = tmp.alloc(&dxh, (size_t)t * k);
    if (!rc) rc = tmp.alloc(&dy, (size_t)t * n);
    if (!rc) rc = tmp.alloc(&derr, (size_t)1);
    cudaError_t e = cudaSuccess;
    if (!rc) {
        e = cudaMemcpy(dx, x, sizeof(float) * t * k, cudaMemcpyDefault);
        if (e == cudaSuccess) e = cudaMemset(derr, 0, sizeof(int));
        if (e == cudaSuccess) e = to_f16_launch(dx, (int64_t)t * k, dxh, 0);
        CUtensorMap map;
        if (e == cudaSuccess && !make_act_map(&map, dxh, t, k)) rc = fail(VVQ2_ERR_CUDA, "tensor map");
        if (!rc && e == cudaSuccess) {
            GemmArgs g;
            g.w0 = dw;
            g.T = t;
            g.N = n;
            g.K = k;
            g.epi = EPI_STORE;
            g.y = dy;
            g.y_stride = n;
            g.err = derr;
            // the prefill engine's kernel for chunks of more than 256 rows (here at
            // any tile count), else the few-row kernel
            const int nt = t > 256 ? gemm_ws_tile_rows(g, 1) : 0;
            CUtensorMap mt, wq[4];
            if (nt && !make_act_map(&mt, dxh, t, k, nt)) rc = fail(VVQ2_ERR_CUDA, "tensor map");
            if (!rc && dw.type == W_Q8_0 && !make_ws_weight_maps(wq, g, nt == 0)) rc = fail(VVQ2_ERR_CUDA, "tensor map");
            if (!rc) e = nt ? gemm_ws_launch(g, mt, wq, nt, 0) : gemm_tc_launch(g, map, wq, 0);
        }
        if (!rc && e == cudaSuccess) e = cudaDeviceSynchronize();
        int herr = 0;
        if (!rc && e == cudaSuccess) e = cudaMemcpy(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost);
        if (!rc && e == cudaSuccess && herr) rc = fail(VVQ2_ERR_CUDA, "gemm wait timed out (%d)", herr);
        if (!rc && e == cudaSuccess) e = cudaMemcpy(y, dy, sizeof(float) * t * n, cudaMemcpyDefault);
    }
    for (void* p : tmp.allocs) cudaFree(p);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(VVQ2_ERR_CUDA, "debug gemm: %s", cudaGetErrorString(e));
    return 0;
}

int vvq2_debug_gemv_mma(const void* w, int n, int k, const float* x, int m, float* y) {
    if (!w || !x || !y || n <= 0 || k <= 0 || k % 32 || m < 1 || m > 2)
        return fail(VVQ2_ERR_INVALID_ARG, "bad gemv args");
    if (vvq2_device_count() == 0) return fail(VVQ2_ERR_NO_DEVICE, "no sm_100 device");
    vvq2_ctx tmp;
    vvq2_tensor tw{w, W_Q8_0, k, n};
    DevW dw;
    int rc = upload_tensor(&tmp, tw, &dw, 0, 0, "debug_gemv_mma");
    float *dx = nullptr, *dy = nullptr;
    if (!rc) rc = tmp.alloc(&dx, (size_t)m * k);
    if (!rc) rc = tmp.alloc(&dy, (size_t)m * n);
    cudaError_t e = cudaSuccess;
    if (!rc) {
        e = cudaMemcpy(dx, x, sizeof(float) * m * k, cudaMemcpyDefault);
        if (e == cudaSuccess) e = debug_gemv_mma_launch(dw, dx, m, dy, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpy(y, dy, sizeof(float) * m * n, cudaMemcpyDefault);
    }
    for (void* p : tmp.allocs) cudaFree(p);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(VVQ2_ERR_CUDA, "debug gemv: %s", cudaGetErrorString(e));
    return 0;
}

}  // extern "C"
