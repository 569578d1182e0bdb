// attn_decode.cu -- split-K flash-decode over the f16 paged KV cache (sm_100a).
//
// Replaces ggml_flash_attn_ext (src/qwen2.cpp:327-335) for decode-sized query
// counts: softmax(Q K^T * 1/sqrt(hd) + causal mask) V with GQA (query head h
// reads KV head h / (nq/nkv), ggml's broadcast) and F32 accumulation
// (ggml_flash_attn_ext_set_prec(GGML_PREC_F32), src/qwen2.cpp:334).  The
// causal mask (key j masked iff j > pos, src/vibevoice_tts.cpp:432-441) is
// evaluated from the row's position; nothing is materialised.
//
// Grid (split, kv_head, row); a split is a whole number of 64-position pages.
// Each page's K and V slices ([64][hd] f16, contiguous in the paged pool) are
// staged into shared memory by the TMA bulk-copy engine (cp.async.bulk with an
// mbarrier), double-buffered so the next page streams in while this one is
// scored.  The whole GQA group (7 or 6 query heads) shares each K/V tile; Q is
// rounded to f16 as ggml does.  Online softmax runs across the pages of the
// split; the last CTA of a (row, kv_head) to finish -- a device-scope counter
// -- merges the splits' partial (O, max, sum) with the log-sum-exp rule.
//
// Every mbarrier wait is bounded: on timeout the kernel records an error code
// in args.err, stops, and returns (no trap, no endless spin).
#include "attn_dev.cuh"
#include "common.cuh"
#include "kernels.h"

namespace vvq2 {

namespace {

constexpr int AD_MAXG = ad::MAXG;
constexpr int TILE = ad::TILE;

struct CtaSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

template <int HD>
__global__ void __launch_bounds__(ad::THREADS) k_attn_decode(const AttnDecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ ad::Shared sh;
    __half* kt = reinterpret_cast<__half*>(smem);   // [2][TILE][HD]
    __half* vt = kt + 2 * TILE * HD;                // [2][TILE][HD]
    if (threadIdx.x == 0) ad::init_bars(sh);
    __syncthreads();
    uint32_t uses[2] = {0, 0};
    ad::item<HD>(a, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, kt, vt, sh, uses, CtaSync{});
}

// Log-sum-exp merge of many splits, one CTA per (query head, row): thread
// (split group sg, 4 columns d4) loads the partials of splits sg, sg + SG, ...
// all at once (one round of independent loads), then the CTA combines
//   O = sum_s e^{m_s - M} O_s / sum_s e^{m_s - M} l_s,   M = max_s m_s.
constexpr int MG_SG = 8;                          // split groups per head
constexpr int MG_PER = ad::MAX_MERGE / MG_SG;     // splits per thread
constexpr int MERGE_INLINE = 4;                   // up to this many splits the last CTA merges

template <int HD>
__global__ void __launch_bounds__(HD / 4 * MG_SG) k_attn_merge(const AttnDecodeArgs a) {
    constexpr int D4 = HD / 4;
    __shared__ float s_mx[MG_SG], s_den[MG_SG];
    __shared__ float4 s_num[MG_SG][D4];
    const int h = blockIdx.x, m = blockIdx.y;
    const int tid = threadIdx.x, d4 = tid % D4, sg = tid / D4;
    const RowMeta rm = a.meta[m];
    const int lim = min(rm.pos + 1, rm.kvlen);
    const int ns = lim > 0 ? (lim + a.split - 1) / a.split : 0;
    if (ns <= 1) return;   // no keys, or one split: the attention kernel wrote the output
    float4 p[MG_PER];
    float2 ml[MG_PER];
#pragma unroll
    for (int k = 0; k < MG_PER; ++k) {
        const int s = sg + k * MG_SG;
        if (s < ns) {
            const size_t r = ((size_t)m * a.max_splits + s) * a.nq + h;
            ml[k] = __ldcg(reinterpret_cast<const float2*>(a.part_ml) + r);
            p[k] = __ldcg(reinterpret_cast<const float4*>(a.part + r * HD) + d4);
        }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < MG_PER; ++k)
        if (sg + k * MG_SG < ns) mx = fmaxf(mx, ml[k].x);
    if (d4 == 0) s_mx[sg] = mx;
    __syncthreads();
    mx = s_mx[0];
#pragma unroll
    for (int i = 1; i < MG_SG; ++i) mx = fmaxf(mx, s_mx[i]);
    float den = 0.f;
    float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < MG_PER; ++k) {
        if (sg + k * MG_SG < ns) {
            const float w = expf(ml[k].x - mx);
            den = fmaf(w, ml[k].y, den);
            num.x = fmaf(w, p[k].x, num.x);
            num.y = fmaf(w, p[k].y, num.y);
            num.z = fmaf(w, p[k].z, num.z);
            num.w = fmaf(w, p[k].w, num.w);
        }
    }
    if (d4 == 0) s_den[sg] = den;
    s_num[sg][d4] = num;
    __syncthreads();
    if (sg != 0) return;
    float dt = 0.f;
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < MG_SG; ++i) {
        dt += s_den[i];
        t.x += s_num[i][d4].x;
        t.y += s_num[i][d4].y;
        t.z += s_num[i][d4].z;
        t.w += s_num[i][d4].w;
    }
    const float inv = 1.0f / dt;
    const size_t off = (size_t)m * a.nq * HD + (size_t)h * HD + d4 * 4;
    if (a.out_h) {
        reinterpret_cast<__half2*>(a.out_h + off)[0] = __floats2half2_rn(t.x * inv, t.y * inv);
        reinterpret_cast<__half2*>(a.out_h + off)[1] = __floats2half2_rn(t.z * inv, t.w * inv);
    } else {
        *reinterpret_cast<float4*>(a.out + off) = make_float4(t.x * inv, t.y * inv, t.z * inv, t.w * inv);
    }
    if (a.lse && d4 == 0) a.lse[(size_t)m * a.nq + h] = mx + logf(dt);
}

template <int HD>
cudaError_t launch_hd(const AttnDecodeArgs& a0, cudaStream_t st) {
    const size_t smem = ad::tile_smem_bytes(HD);   // attn_decode_prepare() opted in
    AttnDecodeArgs a = a0;
    a.defer_merge = a.max_splits > MERGE_INLINE;
    dim3 grid(a.max_splits, a.nkv, a.M);
    k_attn_decode<HD><<<grid, ad::THREADS, smem, st>>>(a);
    note_launch();
    if (a.defer_merge) {
        k_attn_merge<HD><<<dim3(a.nq, a.M), HD / 4 * MG_SG, 0, st>>>(a);
        note_launch();
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t attn_decode_prepare() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_attn_decode<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, ad::tile_smem_bytes(32))) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(k_attn_decode<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, ad::tile_smem_bytes(64))) != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_attn_decode<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, ad::tile_smem_bytes(128));
}

cudaError_t attn_decode_launch(const AttnDecodeArgs& a, cudaStream_t st) {
    if (a.nq % a.nkv || a.nq / a.nkv > AD_MAXG || a.split < TILE || a.split % TILE || a.max_splits > ad::MAX_MERGE)
        return cudaErrorInvalidValue;
    if (a.hd == 32) return launch_hd<32>(a, st);
    if (a.hd == 64) return launch_hd<64>(a, st);
    if (a.hd == 128) return launch_hd<128>(a, st);
    return cudaErrorInvalidValue;
}

// ===================================================================== no-alloc
// Decode attention for callers that cannot allocate device memory.
//
// Some hosts of this library run where cudaMalloc is not available to them:
// an engine that hands every byte of the GPU to its own memory pool up front,
// code running inside a CUDA-graph capture or a context owned by another
// framework, or a real-time audio thread that must not enter the driver's
// allocator.  They own the inputs (Q, the paged K/V, block table, row
// metadata) and the output, but not the kernel's scratch: the split-K partial
// O, the per-split max/sum, the per-(row, head) arrival counters and the
// error word.  That scratch lives here, in one fixed file-scope device array.
//
// Limits (checked, VVQ2_ERR_INVALID_ARG beyond them): up to NA_MAX_ROWS query
// rows, NA_MAX_SPLITS splits per row, n_heads * head_dim <= NA_MAX_QW,
// n_heads <= NA_MAX_HEADS, n_kv_heads <= NA_MAX_KV.  Size: about 2.1 MB per
// GPU, held by every GPU that loads the library until the process exits.
//
// The array is shared by every call: calls that overlap on the GPU (two
// streams, two threads) race on it and must be serialized by the caller.  Each
// call clears the counters and the error word it relies on before launching.
// The device address of the array is looked up once per device, on that
// device's first call (cudaGetSymbolAddress); make that first call before any
// stream capture.
namespace {

constexpr int NA_MAX_ROWS = 8;
constexpr int NA_MAX_SPLITS = 16;
constexpr int NA_MAX_QW = 4096;
constexpr int NA_MAX_HEADS = 64;
constexpr int NA_MAX_KV = 16;
constexpr size_t NA_PART = (size_t)NA_MAX_ROWS * NA_MAX_SPLITS * NA_MAX_QW * sizeof(float);
constexpr size_t NA_ML = (size_t)NA_MAX_ROWS * NA_MAX_SPLITS * NA_MAX_HEADS * 2 * sizeof(float);
constexpr size_t NA_COUNTERS = (size_t)NA_MAX_ROWS * NA_MAX_KV * sizeof(int);
constexpr size_t NA_BYTES = NA_PART + NA_ML + NA_COUNTERS + 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_BYTES];

constexpr int NA_MAX_DEVICES = 64;
unsigned char* g_noalloc_ptr[NA_MAX_DEVICES] = {};

}  // namespace

}  // namespace vvq2

extern "C" int vvq2_attention_decode_noalloc(const float* q, const void* k_pages, const void* v_pages,
                                             const int* block_table, int max_pages, const int* row_meta,
                                             int n_rows, int max_kv, int n_heads, int n_kv_heads,
                                             int head_dim, float* out, void* stream) {
    using namespace vvq2;
    if (!q || !k_pages || !v_pages || !block_table || !row_meta || !out || n_rows <= 0 || max_kv <= 0 ||
        max_pages <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
        return -2;   // VVQ2_ERR_INVALID_ARG
    if (n_rows > NA_MAX_ROWS || n_heads * head_dim > NA_MAX_QW || n_heads > NA_MAX_HEADS ||
        n_kv_heads > NA_MAX_KV || n_heads / n_kv_heads > AD_MAXG ||
        (head_dim != 32 && head_dim != 64 && head_dim != 128) || max_kv > max_pages * KV_PAGE)
        return -2;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NA_MAX_DEVICES) return -10;
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return -9;   // VVQ2_ERR_CUDA
        }
        if (attn_decode_prepare() != cudaSuccess) return -9;
        g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
    }
    unsigned char* base = g_noalloc_ptr[dev];
    // whole pages per split, at most NA_MAX_SPLITS splits over max_kv keys
    int split = (max_kv + NA_MAX_SPLITS - 1) / NA_MAX_SPLITS;
    split = (split + KV_PAGE - 1) / KV_PAGE * KV_PAGE;
    if (split < KV_PAGE) split = KV_PAGE;
    AttnDecodeArgs a;
    a.q = q;
    a.out = out;
    a.meta = reinterpret_cast<const RowMeta*>(row_meta);
    a.kv.k = static_cast<__half*>(const_cast<void*>(k_pages));
    a.kv.v = static_cast<__half*>(const_cast<void*>(v_pages));
    a.kv.block_table = block_table;
    a.kv.max_pages = max_pages;
    a.kv.n_kv = n_kv_heads;
    a.kv.hd = head_dim;
    a.M = n_rows;
    a.nq = n_heads;
    a.nkv = n_kv_heads;
    a.hd = head_dim;
    a.split = split;
    a.max_splits = (max_kv + split - 1) / split;
    a.scale = 1.0f / sqrtf((float)head_dim);
    a.part = reinterpret_cast<float*>(base);
    a.part_ml = reinterpret_cast<float*>(base + NA_PART);
    a.counters = reinterpret_cast<int*>(base + NA_PART + NA_ML);
    a.err = reinterpret_cast<int*>(base + NA_PART + NA_ML + NA_COUNTERS);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // counters and the error word must start at zero; partials are written before read
    if (cudaMemsetAsync(a.counters, 0, NA_COUNTERS + sizeof(int), st) != cudaSuccess) return -9;
    if (attn_decode_launch(a, st) != cudaSuccess) return -9;
    return 0;
}
