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
#include "common.cuh"
#include "kernels.h"

namespace vvq2 {

namespace {

constexpr int AD_THREADS = 128;
constexpr int AD_MAXG = 8;      // query heads per KV head (7 for 0.5B/7B, 6 for 1.5B)
constexpr int TILE = KV_PAGE;   // keys per staged tile (one page)
constexpr uint32_t WAIT_POLLS = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// bounded wait on an mbarrier phase; false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    for (uint32_t i = 0; i < WAIT_POLLS; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

template <int HD>
__global__ void __launch_bounds__(AD_THREADS) k_attn_decode(const AttnDecodeArgs a) {
    constexpr int NCH = HD / 8;                // 16-byte chunks per K row
    constexpr int TILE_BYTES = TILE * HD * 2;
    const int s = blockIdx.x, g = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.nq / a.nkv;
    const RowMeta rm = a.meta[m];
    const int lim = min(rm.pos + 1, rm.kvlen);
    const int nsplit = (lim + a.split - 1) / a.split;
    if (s >= nsplit) return;
    const int j0 = s * a.split, j1 = min(lim, j0 + a.split);
    const int ntiles = (j1 - j0 + TILE - 1) / TILE;

    extern __shared__ __align__(128) uint8_t smem[];
    __half* kt = reinterpret_cast<__half*>(smem);                   // [2][TILE][HD]
    __half* vt = kt + 2 * TILE * HD;                                // [2][TILE][HD]
    __shared__ __align__(16) float qs[AD_MAXG][HD];
    __shared__ float sc[AD_MAXG][TILE];
    __shared__ float red[AD_MAXG][2];
    __shared__ float run_max[AD_MAXG], run_sum[AD_MAXG], alpha[AD_MAXG];
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ int is_last, failed;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int t = tid; t < G * HD; t += AD_THREADS) {
        const int h = t / HD, d = t % HD;
        const float qv = a.q[(size_t)m * a.nq * HD + (size_t)(g * G + h) * HD + d];
        qs[h][d] = __half2float(__float2half_rn(qv));   // ggml FA converts Q to the K type
    }
    if (tid < AD_MAXG) {
        run_max[tid] = -INFINITY;
        run_sum[tid] = 0.f;
    }
    __syncthreads();

    auto page_src = [&](const __half* pool, int tile) {
        const int page = __ldg(a.kv.block_table + (size_t)rm.seq * a.kv.max_pages + (j0 + tile * TILE) / TILE);
        return pool + ((size_t)page * a.kv.n_kv + g) * TILE * HD;
    };
    auto issue = [&](int tile) {
        const int b = tile & 1;
        mbar_expect_tx(&bar[b], 2 * TILE_BYTES);
        bulk_g2s(kt + b * TILE * HD, page_src(a.kv.k, tile), TILE_BYTES, &bar[b]);
        bulk_g2s(vt + b * TILE * HD, page_src(a.kv.v, tile), TILE_BYTES, &bar[b]);
    };
    if (tid == 0) {
        issue(0);
        if (ntiles > 1) issue(1);
    }

    // P.V ownership: thread -> column pair dp and heads hs, hs + HSUB, ...
    constexpr int PAIRS = HD / 2;
    constexpr int HSUB = AD_THREADS / PAIRS;   // 8 (hd 32), 4 (hd 64), 2 (hd 128)
    constexpr int HPER = (AD_MAXG + HSUB - 1) / HSUB;
    const int dp = tid % PAIRS, hs = tid / PAIRS;
    float2 o[HPER];
#pragma unroll
    for (int k = 0; k < HPER; ++k) o[k] = make_float2(0.f, 0.f);

    // scores ownership: key kk = tid % TILE, heads hh, hh + 2, ...
    const int kk = tid % TILE, hh = tid / TILE;
    const int rot = (HD >= 64) ? (kk % NCH) : ((kk >> 1) % NCH);

    for (int t = 0; t < ntiles; ++t) {
        const int b = t & 1;
        if (!mbar_wait(&bar[b], (t >> 1) & 1)) {
            if (a.err) atomicExch(a.err, 1);
            failed = 1;
        }
        __syncthreads();
        if (failed) return;   // uniform: every thread saw the same flag after the barrier
        const __half* K = kt + b * TILE * HD;
        const __half* V = vt + b * TILE * HD;
        const int nk = min(TILE, j1 - (j0 + t * TILE));
        // ---- scores for this tile
        {
            float acc[AD_MAXG / 2];
#pragma unroll
            for (int i = 0; i < AD_MAXG / 2; ++i) acc[i] = 0.f;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const int ch = (c + rot) % NCH;
                const uint4 raw = reinterpret_cast<const uint4*>(K + kk * HD)[ch];
                const __half2* hp = reinterpret_cast<const __half2*>(&raw);
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(hp[e]);
                    kf[2 * e] = f.x;
                    kf[2 * e + 1] = f.y;
                }
#pragma unroll
                for (int i = 0; i < AD_MAXG / 2; ++i) {
                    const int h = hh + 2 * i;
                    if (h < G) {
                        const float4* qp = reinterpret_cast<const float4*>(&qs[h][ch * 8]);
                        const float4 q0 = qp[0], q1 = qp[1];
                        acc[i] = fmaf(q0.x, kf[0], acc[i]);
                        acc[i] = fmaf(q0.y, kf[1], acc[i]);
                        acc[i] = fmaf(q0.z, kf[2], acc[i]);
                        acc[i] = fmaf(q0.w, kf[3], acc[i]);
                        acc[i] = fmaf(q1.x, kf[4], acc[i]);
                        acc[i] = fmaf(q1.y, kf[5], acc[i]);
                        acc[i] = fmaf(q1.z, kf[6], acc[i]);
                        acc[i] = fmaf(q1.w, kf[7], acc[i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < AD_MAXG / 2; ++i) {
                const int h = hh + 2 * i;
                if (h < G) sc[h][kk] = kk < nk ? acc[i] * a.scale : -INFINITY;
            }
        }
        __syncthreads();
        // ---- per-head tile max and the running-max update (warp w < G owns head w... any order)
        if (warp < 4) {
            for (int h = warp; h < G; h += 4) {
                float mx = fmaxf(sc[h][lane], sc[h][lane + 32]);
                mx = warp_max(mx);
                if (lane == 0) {
                    const float mnew = fmaxf(run_max[h], mx);
                    alpha[h] = expf(run_max[h] - mnew);   // exp(-inf) = 0 on the first tile
                    run_max[h] = mnew;
                }
            }
        }
        __syncthreads();
        // ---- probabilities
        for (int i = tid; i < G * TILE; i += AD_THREADS) {
            const int h = i / TILE, k = i % TILE;
            sc[h][k] = expf(sc[h][k] - run_max[h]);   // masked keys: exp(-inf) = 0
        }
        __syncthreads();
        if (warp < 4) {
            for (int h = warp; h < G; h += 4) {
                const float sm = warp_sum(sc[h][lane] + sc[h][lane + 32]);
                if (lane == 0) run_sum[h] = run_sum[h] * alpha[h] + sm;
            }
        }
        // ---- O = O*alpha + P.V
#pragma unroll
        for (int k = 0; k < HPER; ++k) {
            const int h = hs + k * HSUB;
            if (h < G) {
                o[k].x *= alpha[h];
                o[k].y *= alpha[h];
            }
        }
        for (int j = 0; j < nk; ++j) {
            const float2 v = __half22float2(reinterpret_cast<const __half2*>(V + j * HD)[dp]);
#pragma unroll
            for (int k = 0; k < HPER; ++k) {
                const int h = hs + k * HSUB;
                if (h < G) {
                    const float p = sc[h][j];
                    o[k].x = fmaf(p, v.x, o[k].x);
                    o[k].y = fmaf(p, v.y, o[k].y);
                }
            }
        }
        __syncthreads();   // tile buffer b and sc are free again
        if (tid == 0 && t + 2 < ntiles) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(t + 2);
        }
    }

    if (nsplit == 1) {
#pragma unroll
        for (int k = 0; k < HPER; ++k) {
            const int h = hs + k * HSUB;
            if (h < G) {
                const float inv = 1.0f / run_sum[h];
                const size_t off = (size_t)m * a.nq * HD + (size_t)(g * G + h) * HD;
                if (a.out_h)
                    reinterpret_cast<__half2*>(a.out_h + off)[dp] = __floats2half2_rn(o[k].x * inv, o[k].y * inv);
                else
                    reinterpret_cast<float2*>(a.out + off)[dp] = make_float2(o[k].x * inv, o[k].y * inv);
            }
        }
        return;
    }
    // ---- partials, then the last CTA merges (log-sum-exp)
    const size_t pbase = ((size_t)m * a.max_splits + s) * a.nq;
#pragma unroll
    for (int k = 0; k < HPER; ++k) {
        const int h = hs + k * HSUB;
        if (h < G) reinterpret_cast<float2*>(a.part + (pbase + g * G + h) * HD)[dp] = o[k];
    }
    if (tid < G) {
        a.part_ml[(pbase + g * G + tid) * 2 + 0] = run_max[tid];
        a.part_ml[(pbase + g * G + tid) * 2 + 1] = run_sum[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int prev = atomicAdd(a.counters + m * a.nkv + g, 1);
        is_last = (prev == nsplit - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // merge: weights w_s = exp(m_s - max_s m_s) per head, staged in shared
    // memory with one parallel round of loads, then the partial O's summed
    // with independent (batched) loads
    __shared__ float wts[AD_MAXG][64];
    __shared__ float inv_den[AD_MAXG];
    float* ml_s = reinterpret_cast<float*>(kt);   // reuse the K stage: [G][nsplit][2]
    for (int i = tid; i < G * nsplit; i += AD_THREADS) {
        const int h = i / nsplit, ss = i % nsplit;
        const float2 v = __ldcg(reinterpret_cast<const float2*>(a.part_ml) +
                                ((size_t)m * a.max_splits + ss) * a.nq + g * G + h);
        ml_s[2 * i] = v.x;
        ml_s[2 * i + 1] = v.y;
    }
    __syncthreads();
    if (warp < 4) {
        for (int h = warp; h < G; h += 4) {
            float mx = -INFINITY;
            for (int ss = lane; ss < nsplit; ss += 32) mx = fmaxf(mx, ml_s[2 * (h * nsplit + ss)]);
            mx = warp_max(mx);
            float den = 0.f;
            for (int ss = lane; ss < nsplit; ss += 32) {
                const float w = expf(ml_s[2 * (h * nsplit + ss)] - mx);
                wts[h][ss] = w;
                den = fmaf(w, ml_s[2 * (h * nsplit + ss) + 1], den);
            }
            den = warp_sum(den);
            if (lane == 0) inv_den[h] = 1.0f / den;
        }
    }
    __syncthreads();
    for (int t = tid; t < G * PAIRS; t += AD_THREADS) {
        const int h = t / PAIRS, d2 = t % PAIRS;
        const int qh = g * G + h;
        float2 num = make_float2(0.f, 0.f);
#pragma unroll 8
        for (int ss = 0; ss < nsplit; ++ss) {
            const float2 p = __ldcg(reinterpret_cast<const float2*>(
                                        a.part + (((size_t)m * a.max_splits + ss) * a.nq + qh) * HD) + d2);
            num.x = fmaf(wts[h][ss], p.x, num.x);
            num.y = fmaf(wts[h][ss], p.y, num.y);
        }
        const size_t off = (size_t)m * a.nq * HD + (size_t)qh * HD;
        if (a.out_h)
            reinterpret_cast<__half2*>(a.out_h + off)[d2] = __floats2half2_rn(num.x * inv_den[h], num.y * inv_den[h]);
        else
            reinterpret_cast<float2*>(a.out + off)[d2] = make_float2(num.x * inv_den[h], num.y * inv_den[h]);
    }
    if (tid == 0) a.counters[m * a.nkv + g] = 0;   // ready for the next launch
}

template <int HD>
cudaError_t launch_hd(const AttnDecodeArgs& a, cudaStream_t st) {
    const size_t smem = (size_t)4 * TILE * HD * sizeof(__half);   // attn_decode_prepare() opted in
    dim3 grid(a.max_splits, a.nkv, a.M);
    k_attn_decode<HD><<<grid, AD_THREADS, smem, st>>>(a);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t attn_decode_prepare() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_attn_decode<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * TILE * 32 * 2)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(k_attn_decode<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * TILE * 64 * 2)) != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_attn_decode<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * TILE * 128 * 2);
}

cudaError_t attn_decode_launch(const AttnDecodeArgs& a, cudaStream_t st) {
    if (a.nq % a.nkv || a.nq / a.nkv > AD_MAXG || a.split < TILE || a.split % TILE) return cudaErrorInvalidValue;
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
