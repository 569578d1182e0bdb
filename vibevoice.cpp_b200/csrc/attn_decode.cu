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
// The whole GQA group (7 or 6 query heads) shares each K/V tile; Q is rounded
// to f16 as ggml does; online softmax runs across the pages of the split.
// Two kernels do the page math:
//  * k_attn_mma (head_dim 64/128, the engine's paths): pages arrive by TMA
//    tensor copies in the 128-byte swizzle, three in flight, and the dot
//    products run on mma.sync tensor cores (S = Q K^T, O^T += V^T P^T); the
//    splits' partial (O, max, sum) are merged afterwards by k_attn_merge with
//    the log-sum-exp rule, one CTA per (query head, row).
//  * k_attn_decode (head_dim 32, the allocation-free entry point): pages by
//    cp.async.bulk, double-buffered, CUDA-core math; the last CTA of a (row,
//    kv_head) to finish -- a device-scope counter -- merges the partials.
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
    asm volatile("griddepcontrol.launch_dependents;");   // see k_rmsnorm_f16
    const int h = blockIdx.x, m = blockIdx.y;
    const int tid = threadIdx.x, d4 = tid % D4, sg = tid / D4;
    const RowMeta rm = a.meta[m];
    const int lim = ad::key_limit(a, rm, false);   // the attention kernel flagged a clamped row
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

// ---------------------------------------------------------------------------
// Tensor-core decode attention (head_dim 64 / 128, pool with a TMA map).
//
// Same work item (split, KV head, row) and the same partial format as above,
// but the dot products run on mma.sync (m16n8k16, f16 in, f32 accumulate):
// warp w owns keys [16w, 16w + 16) of every 64-key page and keeps its own
// online softmax, so the page loop has no block barrier except the one that
// frees a stage for the next TMA copy.
//   S  = Q K^T     M = the GQA group's query heads (rows 8..15 zero), N = 8
//                  keys, K = head_dim; Q fragments live in registers.
//   O^T += V^T P^T M = 16 head-dim rows, N = the 8 query heads, K = the
//                  warp's 16 keys; P^T is exactly the S accumulator layout
//                  (rounded to f16), V^T comes from ldmatrix.trans.
// K/V pages arrive by TMA (64 x 64 boxes, 128-byte swizzle: 16-byte chunk c
// of key row r sits at chunk c ^ (r & 7)), AM_STAGES pages in flight.  At the end the
// four warps' (max, sum, O) combine through shared memory.
constexpr int AM_THREADS = 128;
constexpr int AM_STAGES = 3;          // pages of K and V in flight per CTA

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// shared address of the 16-byte chunk holding columns col .. col+7 (col % 8 == 0)
// of key row `row` in a swizzled [64][HD] tile
template <int HD>
__device__ __forceinline__ uint32_t swz(uint32_t tile, int row, int col) {
    return tile + (uint32_t)((col >> 6) * 8192 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4));
}

template <int HD>
__global__ void __launch_bounds__(AM_THREADS) k_attn_mma(const __grid_constant__ CUtensorMap mk,
                                                          const __grid_constant__ CUtensorMap mv,
                                                          const AttnDecodeArgs a) {
    constexpr int TILE_BYTES = TILE * HD * 2;   // K (or V) of one page
    constexpr int NB = HD / 64;                 // 64-column boxes per page
    constexpr int KS = HD / 16;                 // k-steps of S, m-tiles of O^T
    extern __shared__ __align__(1024) uint8_t dsm[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bar[AM_STAGES];
    __shared__ float cm[4][8], cl[4][8];
    const int s = blockIdx.x, g = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.nq / a.nkv;
    const RowMeta rm = a.meta[m];
    const int lim = ad::key_limit(a, rm, s == 0 && tid == 0);
    if (lim <= 0) {
        // no keys for this row here (another rank holds its part of the sequence)
        if (s == 0) {
            for (int t = tid; t < G * HD; t += AM_THREADS) {
                const size_t off = (size_t)m * a.nq * HD + (size_t)g * G * HD + t;
                if (a.out_h) a.out_h[off] = __float2half_rn(0.f);
                else a.out[off] = 0.f;
            }
            if (a.lse && tid < G) a.lse[(size_t)m * a.nq + g * G + tid] = -INFINITY;
        }
        return;
    }
    const int nsplit = (lim + a.split - 1) / a.split;
    if (s >= nsplit) return;
    const int j0 = s * a.split, j1 = min(lim, j0 + a.split);
    const int ntiles = (j1 - j0 + TILE - 1) / TILE;
    const uint32_t sbase = tc::smem_u32(sm);   // stage b: K at b * 2 * TILE_BYTES, V after it

    auto issue = [&](int t) {
        const int b = t % AM_STAGES;
        const int page = __ldg(a.kv.block_table + (size_t)rm.seq * a.kv.max_pages + (j0 + t * TILE) / TILE);
        const int y = (page * a.kv.n_kv + g) * TILE;
        uint8_t* kd = sm + b * 2 * TILE_BYTES;
        tc::mbar_arrive_expect_tx(&bar[b], 2 * TILE_BYTES);
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            tc::tma_load_2d(kd + nb * 8192, &mk, nb * 64, y, &bar[b]);
            tc::tma_load_2d(kd + TILE_BYTES + nb * 8192, &mv, nb * 64, y, &bar[b]);
        }
    };
    if (tid == 0) {
        for (int i = 0; i < AM_STAGES; ++i) tc::mbar_init(&bar[i], 1);
        tc::mbar_fence_init();
        issue(0);
        for (int i = 1; i < AM_STAGES && i < ntiles; ++i) issue(i);
    }

    // Q fragments (A of S): row r = lane / 4 is query head g * G + r (zero
    // beyond G), columns 16 kk + 2 (lane % 4) + {0, 1, 8, 9}; rounded to f16
    // as ggml's flash attention converts Q to the K type
    const int r = lane >> 2, q4 = lane & 3;
    uint32_t qa[KS][2];
    {
        const float* qp = a.q + (size_t)m * a.nq * HD + (size_t)(g * G + r) * HD;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            const int c = kk * 16 + 2 * q4;
            if (r < G) {
                const float2 x0 = __ldcg(reinterpret_cast<const float2*>(qp + c));
                const float2 x1 = __ldcg(reinterpret_cast<const float2*>(qp + c + 8));
                qa[kk][0] = pack_h2(x0.x, x0.y);
                qa[kk][1] = pack_h2(x1.x, x1.y);
            } else {
                qa[kk][0] = qa[kk][1] = 0u;
            }
        }
    }
    __syncthreads();   // barrier init visible

    float mrun = -INFINITY, lrun = 0.f;          // softmax state of head r over this warp's keys
    float oacc[KS][4];                            // O^T: rows = head dim, columns = heads 2 q4 + {0, 1}
#pragma unroll
    for (int i = 0; i < KS; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
    // ldmatrix lane roles: matrix i = lane / 8, row lane % 8
    const int li = lane >> 3, lr = lane & 7;
    const int krow = warp * 16 + (li >> 1) * 8 + lr;   // key row this lane addresses
    const int kcol = (li & 1) * 8;                      // + column offset of its matrix

    int t = 0;
    for (; t < ntiles; ++t) {
        const int b = t % AM_STAGES;
        const bool ok = tc::mbar_wait(&bar[b], (t / AM_STAGES) & 1);
        if (__syncthreads_or(!ok)) {   // uniform: every warp leaves the loop together
            if (tid == 0 && a.err) atomicExch(a.err, 1);
            break;
        }
        const uint32_t kt = sbase + b * 2 * TILE_BYTES, vt = kt + TILE_BYTES;
        const int nk = min(TILE, j1 - (j0 + t * TILE));
        if (nk < TILE) {
            // rows past the sequence end: P is 0 there, but 0 * V must not see a
            // non-finite stale value, so this warp zeroes its part of them
            uint8_t* vp = sm + b * 2 * TILE_BYTES + TILE_BYTES;
            for (int i = lane; i < 16 * (HD / 8); i += 32) {
                const int key = warp * 16 + i / (HD / 8), c = (i % (HD / 8)) * 8;
                if (key >= nk) *reinterpret_cast<uint4*>(vp + (swz<HD>(0u, key, c))) = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }
        // ---- S = Q K^T for keys warp*16 + [0, 16): two n-tiles of 8 keys
        float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            uint32_t b00, b01, b10, b11;
            ldsm_x4(swz<HD>(kt, krow, kk * 16 + kcol), b00, b01, b10, b11);
            const uint32_t af[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
            mma16816(sacc[0], af, b00, b01);
            mma16816(sacc[1], af, b10, b11);
        }
        // ---- online softmax of row r over these 16 keys (lanes 4r .. 4r+3)
        float sv[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = warp * 16 + nt * 8 + 2 * q4 + e;
                sv[nt * 2 + e] = key < nk ? sacc[nt][e] * a.scale : -INFINITY;
            }
        float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mnew = fmaxf(mrun, mx);
        const float mref = mnew == -INFINITY ? 0.f : mnew;   // nothing seen yet: p = 0, alpha = 0
        const float alpha = expf(mrun - mref);
        uint32_t pb[2];
        float ps = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const __half2 h = __floats2half2_rn(expf(sv[nt * 2] - mref), expf(sv[nt * 2 + 1] - mref));
            pb[nt] = *reinterpret_cast<const uint32_t*>(&h);
            const float2 f = __half22float2(h);   // the sum uses the rounded P the MMA sees
            ps += f.x + f.y;
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        lrun = fmaf(lrun, alpha, ps);
        mrun = mnew;
        // O^T columns of this lane are heads 2 q4 and 2 q4 + 1: their alphas
        const float al0 = __shfl_sync(0xffffffffu, alpha, 8 * q4);
        const float al1 = __shfl_sync(0xffffffffu, alpha, 8 * q4 + 4);
        // ---- O^T += V^T P^T (one k-step of 16 keys per m-tile of 16 head dims)
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
            uint32_t af[4];
            // matrices: (keys 0-7, dims 0-7), (keys 0-7, dims 8-15), (keys 8-15, dims 0-7), (keys 8-15, dims 8-15)
            // transposed they are A = V^T's (rows 0-7, k 0-7), (rows 8-15, k 0-7), (rows 0-7, k 8-15), (rows 8-15, k 8-15)
            ldsm_x4_t(swz<HD>(vt, krow, mt * 16 + kcol), af[0], af[1], af[2], af[3]);
            oacc[mt][0] *= al0;
            oacc[mt][1] *= al1;
            oacc[mt][2] *= al0;
            oacc[mt][3] *= al1;
            mma16816(oacc[mt], af, pb[0], pb[1]);
        }
        __syncthreads();   // every warp is done with stage b
        if (tid == 0 && t + AM_STAGES < ntiles) {
            tc::fence_proxy_async_smem();
            issue(t + AM_STAGES);
        }
    }
    if (t < ntiles) {
        // a wait gave up: wait (bounded) for the copies still in flight, then leave
        if (tid == 0)
            for (int tt = t; tt < min(ntiles, t + AM_STAGES); ++tt)
                tc::mbar_wait(&bar[tt % AM_STAGES], (tt / AM_STAGES) & 1);
        __syncthreads();
        return;
    }
    __syncthreads();
    // ---- combine the four warps: (max, sum) per head, O^T through shared memory (the stages are free)
    float* co = reinterpret_cast<float*>(sm);     // [4][8][HD]
    if (q4 == 0) {
        cm[warp][r] = mrun;
        cl[warp][r] = lrun;
    }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
        const int d = mt * 16 + r;
        co[(warp * 8 + 2 * q4) * HD + d] = oacc[mt][0];
        co[(warp * 8 + 2 * q4 + 1) * HD + d] = oacc[mt][1];
        co[(warp * 8 + 2 * q4) * HD + d + 8] = oacc[mt][2];
        co[(warp * 8 + 2 * q4 + 1) * HD + d + 8] = oacc[mt][3];
    }
    __syncthreads();
    const size_t pbase = ((size_t)m * a.max_splits + s) * a.nq;
    for (int i = tid; i < G * HD; i += AM_THREADS) {
        const int h = i / HD, d = i % HD;
        float M = cm[0][h];
#pragma unroll
        for (int w = 1; w < 4; ++w) M = fmaxf(M, cm[w][h]);
        float L = 0.f, o = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float e = cm[w][h] == -INFINITY ? 0.f : expf(cm[w][h] - M);
            L = fmaf(e, cl[w][h], L);
            o = fmaf(e, co[(w * 8 + h) * HD + d], o);
        }
        const int qh = g * G + h;
        if (nsplit == 1) {
            const size_t off = (size_t)m * a.nq * HD + (size_t)qh * HD + d;
            const float v = o / L;
            if (a.out_h) a.out_h[off] = __float2half_rn(v);
            else a.out[off] = v;
            if (a.lse && d == 0) a.lse[(size_t)m * a.nq + qh] = M + logf(L);
        } else {
            a.part[(pbase + qh) * HD + d] = o;
            if (d == 0) {
                a.part_ml[(pbase + qh) * 2 + 0] = M;
                a.part_ml[(pbase + qh) * 2 + 1] = L;
            }
        }
    }
}

template <int HD>
cudaError_t launch_hd(const AttnDecodeArgs& a0, cudaStream_t st) {
    const size_t smem = ad::tile_smem_bytes(HD);   // attn_decode_prepare() opted in
    AttnDecodeArgs a = a0;
    if constexpr (HD == 64 || HD == 128) {
        CUtensorMap mk, mv;
        const int64_t rows = (int64_t)a.kv.n_pages * a.kv.n_kv * TILE;
        if (a.kv.n_pages > 0 && make_kv_map(&mk, a.kv.k, rows, HD) && make_kv_map(&mv, a.kv.v, rows, HD)) {
            a.defer_merge = a.max_splits > 1;
            dim3 grid(a.max_splits, a.nkv, a.M);
            k_attn_mma<HD><<<grid, AM_THREADS, 2 * AM_STAGES * TILE * HD * 2 + 1024, st>>>(mk, mv, a);
            note_launch();
            if (a.defer_merge) {
                k_attn_merge<HD><<<dim3(a.nq, a.M), HD / 4 * MG_SG, 0, st>>>(a);
                note_launch();
            }
            return cudaGetLastError();
        }
    }
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
    if ((e = cudaFuncSetAttribute(k_attn_decode<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, ad::tile_smem_bytes(128))) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(k_attn_mma<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * AM_STAGES * TILE * 64 * 2 + 1024)) != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_attn_mma<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * AM_STAGES * TILE * 128 * 2 + 1024);
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
// call clears the counters and the error word it relies on before launching,
// and copies the error word out to the caller's `err_out` after the kernels,
// in stream order (a later call clears it again).  The array's device address
// and the kernel's shared-memory opt-in are looked up on every call, in the
// context current on the calling thread, so a call made in another
// framework's context never uses an address or attribute of a different
// context; neither lookup allocates.
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

template <int HD>
cudaError_t noalloc_opt_in() {
    return cudaFuncSetAttribute(k_attn_decode<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                ad::tile_smem_bytes(HD));
}

}  // namespace

}  // namespace vvq2

extern "C" int vvq2_attention_decode_noalloc(const float* q, const void* k_pages, const void* v_pages,
                                             const int* block_table, int max_pages, const int* row_meta,
                                             int n_rows, int max_kv, int n_heads, int n_kv_heads,
                                             int head_dim, float* out, int* err_out, void* stream) {
    using namespace vvq2;
    if (!q || !k_pages || !v_pages || !block_table || !row_meta || !out || n_rows <= 0 || max_kv <= 0 ||
        max_pages <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
        return -2;   // VVQ2_ERR_INVALID_ARG
    if (n_rows > NA_MAX_ROWS || n_heads * head_dim > NA_MAX_QW || n_heads > NA_MAX_HEADS ||
        n_kv_heads > NA_MAX_KV || n_heads / n_kv_heads > AD_MAXG ||
        (head_dim != 32 && head_dim != 64 && head_dim != 128) || max_kv > max_pages * KV_PAGE)
        return -2;
    // device address of the array in the calling thread's current context
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return -9;   // VVQ2_ERR_CUDA
    }
    const cudaError_t oe = head_dim == 32 ? noalloc_opt_in<32>() : head_dim == 64 ? noalloc_opt_in<64>()
                                                                                  : noalloc_opt_in<128>();
    if (oe != cudaSuccess) {
        cudaGetLastError();
        return -9;
    }
    unsigned char* base = static_cast<unsigned char*>(p);
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
    // the kernels' error word (0, 1 = a bounded wait gave up, 5 = a row longer
    // than max_kv or its block-table row) into the caller's memory, in stream order
    if (err_out && cudaMemcpyAsync(err_out, a.err, sizeof(int), cudaMemcpyDefault, st) != cudaSuccess) return -9;
    return 0;
}
