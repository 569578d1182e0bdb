// decode_mega.cu -- the whole greedy decode step of a Q8_0 Qwen2 stack as ONE
// persistent kernel (sm_100a), for 1 or 2 rows (one sequence or the CFG pair).
//
// A decode step of the 0.5B model is ~120 dependent phases (per layer:
// QKV -> attention -> O-proj -> gate/up -> down) over 0.9-9 MB matrices.  As
// separate launches every phase pays launch and prologue latency and starts
// its weight stream cold.  Here one CTA per SM walks the phase list,
// separated by grid-wide barriers, and the weight stream does not stop:
//
//  * weights: every warp owns D slots of a shared-memory ring (D = 1 or 2)
//    and streams its own share of the CTA's weight tiles: the CTA's
//    contiguous row slice of every matrix of the WHOLE step, cut into tiles
//    of T rows, goes round robin over the 16 warps (tile i -> warp i % 16).
//    Right after computing a tile a warp bulk-copies (cp.async.bulk; a run
//    of Q8_0 rows with their scales is one contiguous range) its next tile
//    into the freed slot.  Weights do not depend on activations, so a warp's
//    next tiles -- often of the next phase -- are in flight while it waits in
//    a grid barrier or runs attention, and no warp waits for another's slot.
//  * each warp stages nothing of its own: the CTA stages the phase's
//    activation rows (RMSNorm'd where the layer norms) from L2 into shared
//    memory, then each warp computes its tiles' T x M dot products over the
//    full K (exact dequantized int8 weights x f32 activations, packed FFMA2),
//    reduces them with one transposing butterfly and applies the epilogue
//    (bias, residual add, SwiGLU, running argmax) straight to global memory.
//  * attention: one item per (row, KV head, split of whole 64-key pages) on
//    128-thread groups.  The first page of each group's first item is
//    requested by TMA BEFORE the QKV -> attention barrier (past keys do not
//    depend on this step).  The item applies RoPE to this step's raw q/k,
//    patches the new key/value row into its tile, appends it to the paged
//    cache, and the last split to finish merges the partials (log-sum-exp).
//
// Every wait is bounded.  A wait that gives up records an error code, raises
// the global abort flag and this CTA's `fail` flag; all warps then skip the
// remaining work (control flow only changes at grid barriers, where it is
// uniform) and wait for their copies in flight before returning.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace vvq2 {

namespace {

constexpr int MT = 512;                 // threads per CTA
constexpr int NCW = 16;                 // warps (all compute and stream)
constexpr int NCT = NCW * 32;
constexpr int MAX_STAGES = 32;          // ring slots: NCW x D
constexpr int ATT_THREADS = 128;
constexpr int MAXG = 8;                 // q heads per KV head
constexpr int PAGE = KV_PAGE;           // keys per page / tile
constexpr int MAX_MERGE = 64;
constexpr uint32_t BAR_POLLS = 1u << 22;
constexpr uint32_t WAIT_POLLS = 1u << 24;

enum { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_LM = 4 };

template <int HD>
struct AttConst {
    static constexpr int NG = 2;                                 // attention groups per CTA
    static constexpr int TILE_BYTES = PAGE * HD * 2;             // one page of K (or V) of one head
    static constexpr int GROUP_BYTES = 2 * TILE_BYTES;           // K and V of one page
};

// per-group attention state (in the phase-shared dynamic region)
template <int HD>
struct __align__(16) AttSh {
    float qs[MAXG][HD];            // roped q, rounded to f16 (ggml FA converts Q to the K type)
    float sc[MAXG][PAGE];
    float run_max[MAXG], run_sum[MAXG], alpha[MAXG];
    __half kn[HD], vn[HD];         // this step's key (roped) and value row
    int is_last, failed;
};

struct Ctl {
    unsigned long long target;
    int aborted;                   // set only inside grid_sync: uniform control flow
    int fail;                      // set by any warp whose wait gave up: ends other waits early
    int nbar;
};

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void trace_mark(const MegaArgs& a, int slot) {
    if (a.trace) a.trace[(size_t)slot * gridDim.x + blockIdx.x] = gtimer();
}

__device__ __forceinline__ void cbar() { __syncthreads(); }

struct GroupSync {
    int id;
    __device__ __forceinline__ void operator()() const { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }
};

__device__ __forceinline__ bool try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(tc::smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait that also gives up once the CTA is failing.
__device__ __forceinline__ bool wait_or_fail(uint64_t* bar, uint32_t parity, const volatile int* fail) {
    for (uint32_t i = 0; i < WAIT_POLLS; ++i) {
        if (try_wait(bar, parity)) return true;
        if (*fail) return false;
    }
    return false;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            tc::smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
        : "memory");
}

__device__ void raise_fail(const MegaArgs& a, Ctl& ctl, int code) {
    atomicCAS(a.err, 0, code);
    atomicExch(a.abort, 1);
    *(volatile int*)&ctl.fail = 1;
}

// Grid barrier over the consumer threads of every CTA.  The arrival is one
// release reduction (orders this CTA's writes, observed through the CTA
// barrier, before it); the wait polls with acquire loads.
__device__ void grid_sync(const MegaArgs& a, Ctl& ctl) {
    cbar();
    if (threadIdx.x == 0) {
        trace_mark(a, 1 + 2 * ctl.nbar);
        ctl.target += gridDim.x;
        asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(a.bar_count), "l"(1ull) : "memory");
        uint32_t i = 0;
        while (true) {
            unsigned long long v;
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a.bar_count) : "memory");
            if (v >= ctl.target) break;
            if (*(volatile int*)a.abort) break;
            if (++i > BAR_POLLS) {
                atomicCAS(a.err, 0, 3);
                atomicExch(a.abort, 1);
                break;
            }
        }
        __threadfence();
        if (*(volatile int*)a.abort) {
            ctl.aborted = 1;
            *(volatile int*)&ctl.fail = 1;
        }
        trace_mark(a, 2 + 2 * ctl.nbar);
        ctl.nbar += 1;
    }
    cbar();
}

// ------------------------------------------------------------ tile schedule
struct Geo {
    const uint8_t* p0;     // first row of this CTA's slice (matrix 0)
    const uint8_t* p1;     // same rows of matrix 1 (up, next to gate) or null
    int64_t rs;            // bytes per row (quants + scales)
    int r0, n;             // slice rows
    int T;                 // rows per tile (per matrix)
    int K;
    int ntiles;
};

__device__ __forceinline__ Geo phase_geo(const MegaArgs& a, int li, int ph) {
    const DevW* w0;
    const DevW* w1 = nullptr;
    int T;
    if (ph == PH_LM) {
        w0 = &a.lm_head;
        T = a.t_lm;
    } else {
        const MegaLayer& L = a.layers[li];
        switch (ph) {
            case PH_QKV: w0 = &L.qkv; T = a.t_qkv; break;
            case PH_O: w0 = &L.o; T = a.t_o; break;
            case PH_GU: w0 = &L.gate; w1 = &L.up; T = a.t_gu; break;
            default: w0 = &L.down; T = a.t_down; break;
        }
    }
    Geo g;
    const int R = w0->rows;
    g.r0 = (int)((long long)R * blockIdx.x / gridDim.x);
    g.n = (int)((long long)R * (blockIdx.x + 1) / gridDim.x) - g.r0;
    g.rs = w0->row_stride;
    g.p0 = w0->q + (size_t)g.r0 * g.rs;
    g.p1 = w1 ? w1->q + (size_t)g.r0 * g.rs : nullptr;
    g.T = T;
    g.K = w0->cols;
    g.ntiles = (g.n + T - 1) / T;
    return g;
}

// ------------------------------------------------------------ weight ring
// Per-warp streaming state (identical in all lanes; lane 0 issues).
struct WarpRing {
    uint32_t used;         // tiles this warp has consumed
    uint32_t issued;       // tiles this warp has requested
    int ip, ij;            // next tile to request: phase-table index, tile in phase
};

__device__ __forceinline__ void ring_normalize(WarpRing& w, const Geo* tab, int nph) {
    while (w.ip < nph && w.ij >= tab[w.ip].ntiles) {
        w.ij -= tab[w.ip].ntiles;
        ++w.ip;
    }
}

// Request this warp's next tile into slot warp + NCW * (issued % D).
__device__ __forceinline__ void ring_issue(WarpRing& w, const Geo* tab, int nph, uint8_t* ring, uint64_t* full,
                                           int warp, int lane, int D, int slot_bytes) {
    if (w.ip >= nph) return;
    const Geo& e = tab[w.ip];
    const int slot = warp + NCW * (int)(w.issued % D);
    if (lane == 0) {
        const int r = w.ij * e.T;
        const uint32_t b0 = (uint32_t)(min(e.T, e.n - r) * e.rs);
        uint8_t* dst = ring + (size_t)slot * slot_bytes;
        tc::fence_proxy_async_smem();   // this warp's generic reads of the slot come first
        tc::mbar_arrive_expect_tx(&full[slot], e.p1 ? 2 * b0 : b0);
        bulk_g2s(dst, e.p0 + (size_t)r * e.rs, b0, &full[slot]);
        if (e.p1) bulk_g2s(dst + (size_t)e.T * e.rs, e.p1 + (size_t)r * e.rs, b0, &full[slot]);
    }
    w.issued += 1;
    w.ij += NCW;
    ring_normalize(w, tab, nph);
}

// ------------------------------------------------------------ activations
// act layout: float4 index ((m * 4 + g) * NC + c) holds elements
// 16c + 4g .. 16c + 4g + 3 of row m, so the lanes of a warp (consecutive
// chunks c) read consecutive 16-byte words.
//
// Where the phase RMSNorms its input, act = x * w (the norm weight) and the
// per-warp partial sums of squares go to red[m][warp]; the row scale
// 1/sqrt(mean(x^2) + eps) is applied to the dot products instead
// (W (x s o w) = s W (x o w)), so no second pass over act is needed.
template <int MB>
__device__ void stage(const float* x, const float* norm_w, int K, float* act, float* red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NC = K / 16, K4 = K / 4;
    float4* act4 = reinterpret_cast<float4*>(act);
    float ss[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) ss[m] = 0.f;
#pragma unroll 4
    for (int k4 = tid; k4 < K4; k4 += NCT) {
        const int c = k4 >> 2, g = k4 & 3;
        const float4 w = norm_w ? __ldg(reinterpret_cast<const float4*>(norm_w) + k4) : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            float4 v = __ldcg(reinterpret_cast<const float4*>(x + (size_t)m * K) + k4);
            if (norm_w) {
                ss[m] = fmaf(v.x, v.x, ss[m]);
                ss[m] = fmaf(v.y, v.y, ss[m]);
                ss[m] = fmaf(v.z, v.z, ss[m]);
                ss[m] = fmaf(v.w, v.w, ss[m]);
                v.x = __fmul_rn(v.x, w.x);
                v.y = __fmul_rn(v.y, w.y);
                v.z = __fmul_rn(v.z, w.z);
                v.w = __fmul_rn(v.w, w.w);
            }
            act4[(m * 4 + g) * NC + c] = v;
        }
    }
    if (norm_w) {
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) red[m * NCW + warp] = t;
        }
    }
    cbar();
}

// RMSNorm row scale from the staged partial sums (ggml_rms_norm: 1/sqrt(mean + eps)).
__device__ __forceinline__ float norm_scale(const float* red, int m, int K, float eps) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) t += red[m * NCW + w];
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), eps)));
}

// ------------------------------------------------------------ tile math
__device__ __forceinline__ uint32_t word(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

// NR rows (row stride rs bytes: Q8_0 quants, then f16 scales) of one tile
// times MB activation rows:
//   acc[t*MB+m] = sum_b d[t,b] * sum_{k in half-block} q[t,k] * x[m,k].
// The int8 quants become exact floats without I2F: the byte (q + 128) is
// placed in the mantissa of 2^23, then 2^23 + 128 is subtracted (exact).
template <int NR, int MB>
__device__ __forceinline__ void tile_dot(const uint8_t* tile, int rs, int K, const float4* act4, int lane,
                                         float (&acc)[NR * MB]) {
    const int NC = K / 16;
    const float2 one2 = make_float2(1.0f, 1.0f), magic2 = make_float2(-8388736.0f, -8388736.0f);
#pragma unroll
    for (int i = 0; i < NR * MB; ++i) acc[i] = 0.f;
    for (int c = lane; c < NC; c += 32) {
        float4 av[MB][4];
#pragma unroll
        for (int m = 0; m < MB; ++m)
#pragma unroll
            for (int g = 0; g < 4; ++g) av[m][g] = act4[(m * 4 + g) * NC + c];
#pragma unroll
        for (int t = 0; t < NR; ++t) {
            const uint8_t* rp = tile + (size_t)t * rs;
            const uint4 q = *reinterpret_cast<const uint4*>(rp + c * 16);
            const float d = __half2float(*reinterpret_cast<const __half*>(rp + K + (c >> 1) * 2));
            float2 s[MB];
#pragma unroll
            for (int m = 0; m < MB; ++m) s[m] = make_float2(0.f, 0.f);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const uint32_t w = word(q, g);   // the device layout stores q + 128 as unsigned bytes
                float2 f01 = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)),
                                         __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441)));
                float2 f23 = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)),
                                         __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443)));
                f01 = __ffma2_rn(f01, one2, magic2);
                f23 = __ffma2_rn(f23, one2, magic2);
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    s[m] = __ffma2_rn(f01, make_float2(av[m][g].x, av[m][g].y), s[m]);
                    s[m] = __ffma2_rn(f23, make_float2(av[m][g].z, av[m][g].w), s[m]);
                }
            }
#pragma unroll
            for (int m = 0; m < MB; ++m) acc[t * MB + m] = fmaf(d, s[m].x + s[m].y, acc[t * MB + m]);
        }
    }
}

template <int N>
struct Log2 {
    static constexpr int v = 1 + Log2<N / 2>::v;
};
template <>
struct Log2<1> {
    static constexpr int v = 0;
};

// Sum NV (a power of two) per-lane values over the warp; lane l returns the
// total of value index l >> (5 - log2 NV).
template <int NV>
__device__ __forceinline__ float warp_transpose_sum(float (&v)[NV], int lane) {
#pragma unroll
    for (int n = NV, o = 16; n > 1; n >>= 1, o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float keep = up ? v[i + n / 2] : v[i];
            const float send = up ? v[i] : v[i + n / 2];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
#pragma unroll
    for (int o = 16 >> Log2<NV>::v; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    return v[0];
}

// One tile of a GEMV phase: math + epilogue.  The epilogue's global
// operands (old residual, bias) are loaded before the math so their latency
// overlaps it.  For lm_head the writer lanes keep a running argmax key.
template <int PH, int T, int MB>
__device__ __forceinline__ void tile_epilogue(const MegaArgs& a, const MegaLayer* L, const uint8_t* tile,
                                              const Geo& g, int r, const float4* act4, int lane, float nsc,
                                              unsigned long long& kbest) {
    constexpr int NR = PH == PH_GU ? 2 * T : T;
    constexpr int NV = NR * MB;
    constexpr int SH = 5 - Log2<NV>::v;
    const int idx = lane >> SH;              // = t * MB + m
    const int t = idx / MB, m = idx % MB;
    const bool writer = (lane & ((1 << SH) - 1)) == 0;
    const int nr = min(T, g.n - r);
    const int row = g.r0 + r + t;
    const bool w_ok = writer && t < nr;
    float pre = 0.f;
    if constexpr (PH == PH_O || PH == PH_DOWN) {
        if (w_ok) pre = __ldcg(a.X + (size_t)m * a.H + row);
    } else if constexpr (PH == PH_QKV) {
        if (w_ok && L->qkv_bias) pre = L->qkv_bias[row];
    }
    float acc[NV];
    tile_dot<NR, MB>(tile, (int)g.rs, g.K, act4, lane, acc);
    float v = warp_transpose_sum<NV>(acc, lane);
    if constexpr (PH == PH_QKV || PH == PH_GU || PH == PH_LM) v = __fmul_rn(v, nsc);   // RMSNorm scale of row m
    if constexpr (PH == PH_GU) {
        const float u = __shfl_sync(0xffffffffu, v, (lane + ((T * MB) << SH)) & 31);
        if (w_ok) a.FA[(size_t)m * a.F + row] = __fmul_rn(silu_ref(v), u);   // ggml_swiglu_split: silu(g) * u
    } else if constexpr (PH == PH_QKV) {
        if (w_ok) a.QKV[(size_t)m * a.qkv_rows + row] = L->qkv_bias ? __fadd_rn(v, pre) : v;
    } else if constexpr (PH == PH_LM) {
        if (w_ok) {
            const unsigned long long k = argmax_key(v, row);
            kbest = k > kbest ? k : kbest;
        }
    } else {   // O-proj / down: residual add into X (ggml_add(x, o))
        if (w_ok) a.X[(size_t)m * a.H + row] = __fadd_rn(pre, v);
    }
}

template <int PH, int MB>
__device__ void gemv_tiles(const MegaArgs& a, int li, const Geo* tab, int nph, uint8_t* ring, uint64_t* full,
                           const float* act, const float* red, uint32_t& seq, WarpRing& wr, int D, Ctl& ctl,
                           unsigned long long* best) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const Geo& g = tab[PH == PH_LM ? 4 * a.n_layers : 4 * li + PH];
    const MegaLayer* L = PH == PH_LM ? nullptr : &a.layers[li];
    const float4* act4 = reinterpret_cast<const float4*>(act);
    const int j0 = (warp - (int)(seq % NCW) + NCW) % NCW;
    const volatile int* fl = &ctl.fail;
    unsigned long long kbest = 0ull;
    // this lane's row m is fixed by the lane and T; its RMSNorm scale where the phase norms
    float nsc = 1.f;
    if constexpr (PH == PH_QKV || PH == PH_GU || PH == PH_LM) {
        const int nv = (PH == PH_GU ? 2 : 1) * g.T * MB;
        const int sh = 5 - (nv == 1 ? 0 : nv == 2 ? 1 : nv == 4 ? 2 : nv == 8 ? 3 : 4);
        nsc = norm_scale(red, (lane >> sh) % MB, g.K, a.eps);
    }
    for (int j = j0; j < g.ntiles; j += NCW) {
        const int slot = warp + NCW * (int)(wr.used % D);
        if (!wait_or_fail(&full[slot], (wr.used / D) & 1, fl)) {
            if (lane == 0 && !*fl) raise_fail(a, ctl, 4);
            break;
        }
        const uint8_t* tile = ring + (size_t)slot * a.slot_bytes;
        const int r = j * g.T;
        switch (g.T) {
            case 1: tile_epilogue<PH, 1, MB>(a, L, tile, g, r, act4, lane, nsc, kbest); break;
            case 2: tile_epilogue<PH, 2, MB>(a, L, tile, g, r, act4, lane, nsc, kbest); break;
            default:
                if constexpr (PH != PH_GU) tile_epilogue<PH, 4, MB>(a, L, tile, g, r, act4, lane, nsc, kbest);
                break;
        }
        __syncwarp();
        wr.used += 1;
        ring_issue(wr, tab, nph, ring, full, warp, lane, D, a.slot_bytes);   // refill the slot just freed
    }
    if constexpr (PH == PH_LM) {
        // writer lanes hold one row's running best; the row index m is a function of the lane and T
        const int sh = 5 - (g.T == 1 ? 0 : g.T == 2 ? 1 : 2) - (MB == 2 ? 1 : 0);
        if (kbest) atomicMax(&best[(lane >> sh) % MB], kbest);
    }
    seq += g.ntiles;
}

// ------------------------------------------------------------ attention
struct AttItem {
    int m, g, s, nsplit, j0, j1, ntiles;
    int page0;             // physical page of the first tile
    RowMeta rm;
};

__device__ __forceinline__ bool att_item_geo(const MegaArgs& a, int it, AttItem& x) {
    x.s = it % a.nsplit;
    x.g = (it / a.nsplit) % a.nkv;
    x.m = it / (a.nsplit * a.nkv);
    x.rm = a.meta[x.m];
    const int lim = min(x.rm.pos + 1, x.rm.kvlen);
    x.nsplit = (lim + a.split - 1) / a.split;
    if (x.s >= x.nsplit) return false;
    x.j0 = x.s * a.split;
    x.j1 = min(lim, x.j0 + a.split);
    x.ntiles = (x.j1 - x.j0 + PAGE - 1) / PAGE;
    x.page0 = __ldg(a.layers[0].kv.block_table + (size_t)x.rm.seq * a.layers[0].kv.max_pages + x.j0 / PAGE);
    return true;
}

// K and V of page `tile` of the item into the group's single stage.
template <int HD>
__device__ __forceinline__ void att_issue(const KvLayer& kv, const AttItem& x, int tile, __half* kt, __half* vt,
                                          uint64_t* bar) {
    constexpr int TB = AttConst<HD>::TILE_BYTES;
    const int page =
        tile == 0 ? x.page0 : __ldg(kv.block_table + (size_t)x.rm.seq * kv.max_pages + (x.j0 + tile * PAGE) / PAGE);
    const size_t off = ((size_t)page * kv.n_kv + x.g) * PAGE * HD;
    tc::mbar_arrive_expect_tx(bar, 2 * TB);
    bulk_g2s(kt, kv.k + off, TB, bar);
    bulk_g2s(vt, kv.v + off, TB, bar);
}

// One attention item on a 128-thread group.  The first tile may already be
// in flight (`prefetched`).  Returns false after a timed-out wait.
template <int HD>
__device__ bool att_item(const MegaArgs& a, const KvLayer& kv, const AttItem& x, int tid, __half* kt, __half* vt,
                         AttSh<HD>& sh, const float2* cs_row, uint64_t* bar, uint32_t& uses, bool prefetched,
                         GroupSync sync, int* merge_n, int4* merges) {
    const int lane = tid & 31, warp = tid >> 5;
    const int G = a.nq / a.nkv;
    constexpr int half = HD / 2;
    const int m = x.m, g = x.g;
    const RowMeta& rm = x.rm;
    const int newj = rm.cidx;   // cache index of this step's key/value
    const bool has_new = newj >= x.j0 && newj < x.j1;

    if (tid == 0) sh.failed = 0;
    if (tid < MAXG) {
        sh.run_max[tid] = -INFINITY;
        sh.run_sum[tid] = 0.f;
    }
    sync();
    // this step's raw q (and new k, v) rows: all loads issued before any use
    const float* qkv = a.QKV + (size_t)m * a.qkv_rows;
    constexpr int QI = (MAXG * half + ATT_THREADS - 1) / ATT_THREADS;
    float qa[QI], qb[QI], ka = 0.f, kb = 0.f, vv = 0.f;
#pragma unroll
    for (int it = 0; it < QI; ++it) {
        const int t = tid + it * ATT_THREADS;
        if (t < G * half) {
            const float* q = qkv + (size_t)(g * G + t / half) * HD + t % half;
            qa[it] = __ldcg(q);
            qb[it] = __ldcg(q + half);
        }
    }
    if (has_new) {
        if (tid < half) {
            const float* k = qkv + (size_t)(a.nq + g) * HD + tid;
            ka = __ldcg(k);
            kb = __ldcg(k + half);
        }
        if (tid < HD) vv = __ldcg(qkv + (size_t)(a.nq + a.nkv + g) * HD + tid);
    }
#pragma unroll
    for (int it = 0; it < QI; ++it) {
        const int t = tid + it * ATT_THREADS;
        if (t < G * half) {
            const int h = t / half, i = t % half;
            const float2 cs = cs_row[i];
            const float y0 = __fsub_rn(__fmul_rn(qa[it], cs.x), __fmul_rn(qb[it], cs.y));
            const float y1 = __fadd_rn(__fmul_rn(qa[it], cs.y), __fmul_rn(qb[it], cs.x));
            sh.qs[h][i] = __half2float(__float2half_rn(y0));
            sh.qs[h][i + half] = __half2float(__float2half_rn(y1));
        }
    }
    if (has_new) {
        if (tid < half) {
            const float2 cs = cs_row[tid];
            sh.kn[tid] = __float2half_rn(__fsub_rn(__fmul_rn(ka, cs.x), __fmul_rn(kb, cs.y)));
            sh.kn[tid + half] = __float2half_rn(__fadd_rn(__fmul_rn(ka, cs.y), __fmul_rn(kb, cs.x)));
        }
        if (tid < HD) sh.vn[tid] = __float2half_rn(vv);
    }
    if (tid == 0 && !prefetched) {
        tc::fence_proxy_async_smem();
        att_issue<HD>(kv, x, 0, kt, vt, bar);
    }

    constexpr int NCH = HD / 8;
    constexpr int PAIRS = HD / 2;
    constexpr int HSUB = ATT_THREADS / PAIRS;
    constexpr int HPER = (MAXG + HSUB - 1) / HSUB;
    const int dp = tid % PAIRS, hs = tid / PAIRS;
    float2 o[HPER];
#pragma unroll
    for (int k = 0; k < HPER; ++k) o[k] = make_float2(0.f, 0.f);
    const int kk = tid % PAGE, hh = tid / PAGE;
    const int rot = kk % NCH;

    for (int t = 0; t < x.ntiles; ++t) {
        if (!tc::mbar_wait(bar, uses & 1)) {
            atomicCAS(a.err, 0, 1);
            sh.failed = 1;
        }
        uses += 1;
        sync();
        if (sh.failed) return false;   // uniform after the group barrier
        __half* K = kt;
        __half* V = vt;
        const int tj0 = x.j0 + t * PAGE;
        const int nk = min(PAGE, x.j1 - tj0);
        if (has_new && newj >= tj0 && newj < tj0 + PAGE) {
            // the page copy predates this step's row: patch it in
            for (int d = tid; d < HD; d += ATT_THREADS) {
                K[(newj - tj0) * HD + d] = sh.kn[d];
                V[(newj - tj0) * HD + d] = sh.vn[d];
            }
            sync();
        }
        {
            float acc[MAXG / 2];
#pragma unroll
            for (int i = 0; i < MAXG / 2; ++i) acc[i] = 0.f;
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
                for (int i = 0; i < MAXG / 2; ++i) {
                    const int h = hh + 2 * i;
                    if (h < G) {
                        const float4* qp = reinterpret_cast<const float4*>(&sh.qs[h][ch * 8]);
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
            for (int i = 0; i < MAXG / 2; ++i) {
                const int h = hh + 2 * i;
                if (h < G) sh.sc[h][kk] = kk < nk ? acc[i] * a.scale : -INFINITY;
            }
        }
        sync();
        for (int h = warp; h < G; h += 4) {
            float mx = fmaxf(sh.sc[h][lane], sh.sc[h][lane + 32]);
            mx = warp_max(mx);
            if (lane == 0) {
                const float mnew = fmaxf(sh.run_max[h], mx);
                sh.alpha[h] = expf(sh.run_max[h] - mnew);   // exp(-inf) = 0 on the first tile
                sh.run_max[h] = mnew;
            }
        }
        sync();
        for (int i = tid; i < G * PAGE; i += ATT_THREADS) {
            const int h = i / PAGE, k = i % PAGE;
            sh.sc[h][k] = expf(sh.sc[h][k] - sh.run_max[h]);   // masked keys: exp(-inf) = 0
        }
        sync();
        for (int h = warp; h < G; h += 4) {
            const float sm = warp_sum(sh.sc[h][lane] + sh.sc[h][lane + 32]);
            if (lane == 0) sh.run_sum[h] = sh.run_sum[h] * sh.alpha[h] + sm;
        }
#pragma unroll
        for (int k = 0; k < HPER; ++k) {
            const int h = hs + k * HSUB;
            if (h < G) {
                o[k].x *= sh.alpha[h];
                o[k].y *= sh.alpha[h];
            }
        }
        for (int j = 0; j < nk; ++j) {
            const float2 v = __half22float2(reinterpret_cast<const __half2*>(V + j * HD)[dp]);
#pragma unroll
            for (int k = 0; k < HPER; ++k) {
                const int h = hs + k * HSUB;
                if (h < G) {
                    const float p = sh.sc[h][j];
                    o[k].x = fmaf(p, v.x, o[k].x);
                    o[k].y = fmaf(p, v.y, o[k].y);
                }
            }
        }
        sync();   // the stage and sc are free again
        if (tid == 0 && t + 1 < x.ntiles) {
            tc::fence_proxy_async_smem();
            att_issue<HD>(kv, x, t + 1, kt, vt, bar);
        }
    }
    // append this step's K/V row to the paged cache (read by later steps)
    if (has_new) {
        const size_t off = kv_offset(kv, rm.seq, newj, g);
        for (int d = tid; d < HD; d += ATT_THREADS) {
            kv.k[off + d] = sh.kn[d];
            kv.v[off + d] = sh.vn[d];
        }
    }

    float* out = a.ATT + (size_t)m * a.nq * HD;
    if (x.nsplit == 1) {
#pragma unroll
        for (int k = 0; k < HPER; ++k) {
            const int h = hs + k * HSUB;
            if (h < G) {
                const float inv = 1.0f / sh.run_sum[h];
                reinterpret_cast<float2*>(out + (size_t)(g * G + h) * HD)[dp] = make_float2(o[k].x * inv, o[k].y * inv);
            }
        }
        sync();   // sh is reused by the next item
        return true;
    }
    // ---- partials, then the last arriving split merges (log-sum-exp)
    const size_t pbase = ((size_t)m * MAX_MERGE + x.s) * a.nq;
#pragma unroll
    for (int k = 0; k < HPER; ++k) {
        const int h = hs + k * HSUB;
        if (h < G) reinterpret_cast<float2*>(a.part + (pbase + g * G + h) * HD)[dp] = o[k];
    }
    if (tid < G) {
        a.part_ml[(pbase + g * G + tid) * 2 + 0] = sh.run_max[tid];
        a.part_ml[(pbase + g * G + tid) * 2 + 1] = sh.run_sum[tid];
    }
    sync();
    if (tid == 0) {
        // release the partials (written by the group, ordered by the group
        // barrier), count the split; the last one queues the merge for its CTA
        int prev;
        asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(a.counters + m * a.nkv + g)
                     : "memory");
        if (prev == x.nsplit - 1) {
            const int e = atomicAdd(merge_n, 1);
            merges[e] = make_int4(m, g, x.nsplit, 0);
        }
    }
    sync();
    return true;
}

// Log-sum-exp merge of the ns partials of (row m, KV head g) by the whole
// CTA (all partial loads in one round trip), then ATT[m][heads of g].
// `scr`: shared scratch of at least mega_merge_scratch bytes.
template <int HD>
__device__ void cta_merge(const MegaArgs& a, int m, int g, int ns, float* scr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.nq / a.nkv;
    constexpr int PAIRS = HD / 2;
    float* ml = scr;                                  // [G][ns][2]
    float* wts = ml + 2 * MAXG * MAX_MERGE;           // [G][ns]
    float* inv = wts + MAXG * MAX_MERGE;              // [G]
    float2* num = reinterpret_cast<float2*>(inv + 2 * MAXG);   // [Q][G * PAIRS]
    const float2* pml = reinterpret_cast<const float2*>(a.part_ml);
    for (int i = tid; i < G * ns; i += NCT) {
        const int h = i / ns, ss = i % ns;
        const float2 v = __ldcg(pml + ((size_t)m * MAX_MERGE + ss) * a.nq + g * G + h);
        ml[2 * i] = v.x;
        ml[2 * i + 1] = v.y;
    }
    cbar();
    for (int h = warp; h < G; h += NCW) {
        float mx = -INFINITY;
        for (int ss = lane; ss < ns; ss += 32) mx = fmaxf(mx, ml[2 * (h * ns + ss)]);
        mx = warp_max(mx);
        float den = 0.f;
        for (int ss = lane; ss < ns; ss += 32) {
            const float w = expf(ml[2 * (h * ns + ss)] - mx);
            wts[h * ns + ss] = w;
            den = fmaf(w, ml[2 * (h * ns + ss) + 1], den);
        }
        den = warp_sum(den);
        if (lane == 0) inv[h] = 1.0f / den;
    }
    cbar();
    const int np = G * PAIRS, Q = NCT / np;          // Q threads share one (head, column pair)
    if (tid < Q * np) {
        const int pidx = tid % np, qi = tid / np;
        const int h = pidx / PAIRS, d2 = pidx % PAIRS;
        const float2* src = reinterpret_cast<const float2*>(a.part + (size_t)(g * G + h) * HD) + d2;
        const size_t sstride = (size_t)a.nq * HD / 2;   // float2 per split
        float2 acc = make_float2(0.f, 0.f);
        for (int s0 = qi; s0 < ns; s0 += 8 * Q) {      // 8 independent loads in flight per batch
            float2 p[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (s0 + i * Q < ns) p[i] = __ldcg(src + ((size_t)m * MAX_MERGE + s0 + i * Q) * sstride);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (s0 + i * Q < ns) {
                    const float w = wts[h * ns + s0 + i * Q];
                    acc.x = fmaf(w, p[i].x, acc.x);
                    acc.y = fmaf(w, p[i].y, acc.y);
                }
        }
        num[qi * np + pidx] = acc;
    }
    cbar();
    float* out = a.ATT + (size_t)m * a.nq * HD;
    for (int pidx = tid; pidx < np; pidx += NCT) {
        float2 t = num[pidx];
        for (int qi = 1; qi < Q; ++qi) {
            t.x += num[qi * np + pidx].x;
            t.y += num[qi * np + pidx].y;
        }
        const int h = pidx / PAIRS, d2 = pidx % PAIRS;
        reinterpret_cast<float2*>(out + (size_t)(g * G + h) * HD)[d2] = make_float2(t.x * inv[h], t.y * inv[h]);
    }
    if (tid == 0) a.counters[m * a.nkv + g] = 0;   // ready for the next layer / launch
    cbar();
}

// ------------------------------------------------------------ kernel
template <int HD, int MB>
__global__ void __launch_bounds__(MT, 1) k_decode_mega(const MegaArgs a) {
    extern __shared__ __align__(1024) uint8_t dyn[];
    using AC = AttConst<HD>;
    __shared__ __align__(8) uint64_t full[MAX_STAGES];
    __shared__ __align__(8) uint64_t abar[AC::NG];
    __shared__ float red[2 * NCW];
    __shared__ unsigned long long best[2];
    __shared__ float2 rope_cs[2][64];              // RoPE (cos, sin) per row: positions are fixed for the launch
    __shared__ int merge_n;                        // attention merges this CTA owes in the current layer
    __shared__ int4 merges[16];                    // (m, g, nsplit)
    __shared__ Ctl ctl;
    const int tid = threadIdx.x, warp = tid >> 5;
    uint8_t* region = dyn;                         // activations | attention tiles + state
    uint8_t* ring = dyn + a.union_bytes;
    Geo* tab = reinterpret_cast<Geo*>(ring + (size_t)a.nstage * a.slot_bytes);   // [4 * n_layers + 1]
    const int nph = 4 * a.n_layers + 1;
    const int D = a.nstage / NCW;
    float* act = reinterpret_cast<float*>(region);

    if (tid == 0) {
        const unsigned long long per_launch = (unsigned long long)(5 * a.n_layers + 2) * gridDim.x;
        ctl.target = (unsigned long long)(*(volatile unsigned int*)a.epoch) * per_launch;
        ctl.aborted = 0;
        ctl.fail = 0;
        ctl.nbar = 0;
        trace_mark(a, 0);
        for (int i = 0; i < a.nstage; ++i) tc::mbar_init(&full[i], 1);
        for (int i = 0; i < AC::NG; ++i) tc::mbar_init(&abar[i], 1);
        tc::mbar_fence_init();
    }
    if (tid < 2) best[tid] = 0ull;
    if (blockIdx.x == 0 && tid < MB) a.amax[tid] = 0ull;
    // this CTA's tile geometry of every phase of the step
    for (int p = tid; p < nph; p += NCT)
        tab[p] = phase_geo(a, p == nph - 1 ? 0 : p / 4, p == nph - 1 ? PH_LM : p % 4);
    __syncthreads();

    // every warp requests its first D tiles (layer 0's weights land during the embedding)
    const int lane = tid & 31;
    WarpRing wr;
    wr.used = wr.issued = 0;
    wr.ip = 0;
    wr.ij = warp;
    ring_normalize(wr, tab, nph);
    for (int d = 0; d < D; ++d) ring_issue(wr, tab, nph, ring, full, warp, lane, D, a.slot_bytes);

    // ---- token embedding: X[m] = dequant(tok_embd[tok[m]])
    {
        const int H = a.H;
        const DevW& E = a.tok_embd;
        for (int t = blockIdx.x * NCT + tid; t < MB * H; t += gridDim.x * NCT) {
            const int m = t / H, k = t % H;
            const int r = a.tok[m];
            float v = 0.f;
            if (r >= 0 && r < E.rows) {
                const uint8_t* rp = E.q + (size_t)r * E.row_stride;
                const float d = __half2float(*reinterpret_cast<const __half*>(rp + H + (k / 32) * 2));
                v = __fmul_rn((float)((int)rp[k] - 128), d);   // quants stored as q + 128
            }
            a.X[t] = v;
        }
    }

    // RoPE table of each row's position (ggml CPU theta recurrence)
    for (int t = tid; t < MB * (HD / 2); t += NCT) {
        const int m = t / (HD / 2), i = t % (HD / 2);
        float th = (float)a.meta[m].pos;
        for (int k = 0; k < i; ++k) th = __fmul_rn(th, a.rope_ts);
        rope_cs[m][i] = make_float2(cosf(th), sinf(th));
    }

    uint32_t seq = 0;                    // ring tiles consumed so far
    uint32_t uses = 0;                   // completed phases of this group's attention barrier
    const int qw = a.nq * HD;
    const int grp = tid / ATT_THREADS, gtid = tid % ATT_THREADS;
    const int n_att = a.nsplit * a.nkv * MB;
    AttSh<HD>* ash = reinterpret_cast<AttSh<HD>*>(region + AC::NG * AC::GROUP_BYTES);
    __half* kt = reinterpret_cast<__half*>(region + (size_t)grp * AC::GROUP_BYTES);
    __half* vt = kt + PAGE * HD;
    // this group's first attention item: the same in every layer of the launch
    const int it0 = blockIdx.x + grp * gridDim.x;
    AttItem x0;
    const bool pre = grp < AC::NG && it0 < n_att && att_item_geo(a, it0, x0);   // uniform in the group

    for (int li = 0; li < a.n_layers; ++li) {
        const MegaLayer& L = a.layers[li];
        // 1. RMSNorm + QKV (+bias) -> raw q/k/v rows
        grid_sync(a, ctl);
        if (ctl.aborted) break;
        stage<MB>(a.X, L.attn_norm, a.H, act, red);
        gemv_tiles<PH_QKV, MB>(a, li, tab, nph, ring, full, act, red, seq, wr, D, ctl, best);
        // 2. attention: the first page of each group's first item is requested
        //    before the barrier (activations are dead: the region is free)
        cbar();
        if (tid == 0) merge_n = 0;
        if (pre && gtid == 0) {
            tc::fence_proxy_async_smem();
            att_issue<HD>(L.kv, x0, 0, kt, vt, &abar[grp]);
        }
        grid_sync(a, ctl);
        if (grp < AC::NG) {
            for (int it = it0; it < n_att; it += AC::NG * gridDim.x) {
                const bool first = it == it0;
                AttItem x;
                if (first && pre) x = x0;
                else if (!att_item_geo(a, it, x)) continue;
                // a prefetched item runs even when aborting, so its copies are waited for
                if (ctl.aborted && !(first && pre)) break;
                if (!att_item<HD>(a, L.kv, x, gtid, kt, vt, ash[grp], rope_cs[x.m], &abar[grp], uses,
                                  first && pre, GroupSync{1 + grp}, &merge_n, merges)) {
                    if (gtid == 0) raise_fail(a, ctl, 1);
                    break;
                }
            }
        }
        cbar();
        // splits that finished last merge with the whole CTA (the tiles are free now)
        for (int e = 0; e < merge_n && !ctl.aborted; ++e)
            cta_merge<HD>(a, merges[e].x, merges[e].y, merges[e].z, reinterpret_cast<float*>(region));
        if (ctl.aborted) break;
        // 3. O-proj + residual
        grid_sync(a, ctl);
        if (ctl.aborted) break;
        stage<MB>(a.ATT, nullptr, qw, act, red);
        gemv_tiles<PH_O, MB>(a, li, tab, nph, ring, full, act, red, seq, wr, D, ctl, best);
        // 4. RMSNorm + gate/up + SwiGLU
        grid_sync(a, ctl);
        if (ctl.aborted) break;
        stage<MB>(a.X, L.ffn_norm, a.H, act, red);
        gemv_tiles<PH_GU, MB>(a, li, tab, nph, ring, full, act, red, seq, wr, D, ctl, best);
        // 5. down + residual
        grid_sync(a, ctl);
        if (ctl.aborted) break;
        stage<MB>(a.FA, nullptr, a.F, act, red);
        gemv_tiles<PH_DOWN, MB>(a, li, tab, nph, ring, full, act, red, seq, wr, D, ctl, best);
    }
    // output norm + lm_head + argmax
    if (!ctl.aborted) {
        grid_sync(a, ctl);
        if (!ctl.aborted) {
            stage<MB>(a.X, a.out_norm, a.H, act, red);
            gemv_tiles<PH_LM, MB>(a, 0, tab, nph, ring, full, act, red, seq, wr, D, ctl, best);
            cbar();
            if (tid < MB && best[tid]) atomicMax(a.amax + tid, best[tid]);
            grid_sync(a, ctl);
        }
    }
    if (blockIdx.x == 0 && !ctl.aborted && tid < MB) {
        a.tok[tid] = argmax_key_index(a.amax[tid]);
        RowMeta r = a.meta[tid];
        r.pos += 1;
        r.cidx += 1;
        r.kvlen += 1;
        a.meta[tid] = r;
    }
    // copies still in flight (only after an abort): wait for them before exiting
    for (uint32_t k = wr.used; k < wr.issued; ++k)
        tc::mbar_wait(&full[warp + NCW * (int)(k % D)], (k / D) & 1, 1u << 20);
    if (tid == 0) {
        if (blockIdx.x == 0) {
            __threadfence();
            atomicAdd(a.epoch, 1u);
        }
        trace_mark(a, mega_trace_slots(a.n_layers) - 1);
    }
}

template <int HD, int MB>
cudaError_t set_smem(int bytes) {
    return cudaFuncSetAttribute(k_decode_mega<HD, MB>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <int HD>
size_t att_union_bytes() {
    return (size_t)AttConst<HD>::NG * (AttConst<HD>::GROUP_BYTES + sizeof(AttSh<HD>));
}

}  // namespace

int decode_mega_union_bytes(int hd, int M, int kmax) {
    const size_t act = (size_t)M * kmax * 4;
    const size_t att = hd == 64 ? att_union_bytes<64>() : att_union_bytes<128>();
    return (int)((std::max(act, att) + 1023) / 1024 * 1024);
}

int decode_mega_max_stages() { return MAX_STAGES; }

int decode_mega_consumer_warps() { return NCW; }

int decode_mega_att_groups() { return AttConst<64>::NG; }

int decode_mega_table_bytes(int n_layers) { return (int)((4 * n_layers + 1) * sizeof(Geo)); }

// dynamic shared memory available to the kernel: opt-in limit minus its static shared memory
int decode_mega_smem_limit() {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    size_t st = 0;
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, k_decode_mega<64, 2>) == cudaSuccess) st = std::max(st, fa.sharedSizeBytes);
    if (cudaFuncGetAttributes(&fa, k_decode_mega<128, 2>) == cudaSuccess) st = std::max(st, fa.sharedSizeBytes);
    return optin - (int)st;
}

cudaError_t decode_mega_prepare() {
    const int lim = decode_mega_smem_limit();
    cudaError_t e;
    if ((e = set_smem<64, 1>(lim)) != cudaSuccess) return e;
    if ((e = set_smem<64, 2>(lim)) != cudaSuccess) return e;
    if ((e = set_smem<128, 1>(lim)) != cudaSuccess) return e;
    return set_smem<128, 2>(lim);
}

int decode_mega_grid() {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_decode_mega<64, 2>, MT, decode_mega_smem_limit());
    return per >= 1 ? sms : 0;
}

cudaError_t decode_mega_launch(const MegaArgs& a, size_t smem, cudaStream_t st) {
    auto pow2_le4 = [](int t) { return t == 1 || t == 2 || t == 4; };
    const bool t_ok = a.t_gu == 1 || a.t_gu == 2;   // gate + up rows: at most 4 per tile
    if (a.M < 1 || a.M > 2 || a.nstage < NCW || a.nstage > MAX_STAGES || a.nstage % NCW || a.nsplit < 1 ||
        a.nsplit > MAX_MERGE ||
        !t_ok || !pow2_le4(a.t_qkv) || !pow2_le4(a.t_o) || !pow2_le4(a.t_down) || !pow2_le4(a.t_lm) ||
        a.slot_bytes % 16 || a.union_bytes % 1024)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.grid);
    cfg.blockDim = dim3(MT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs co-resident: the grid barriers rely on it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (a.hd == 64)
        e = a.M == 1 ? cudaLaunchKernelEx(&cfg, k_decode_mega<64, 1>, a) : cudaLaunchKernelEx(&cfg, k_decode_mega<64, 2>, a);
    else if (a.hd == 128)
        e = a.M == 1 ? cudaLaunchKernelEx(&cfg, k_decode_mega<128, 1>, a)
                     : cudaLaunchKernelEx(&cfg, k_decode_mega<128, 2>, a);
    else
        return cudaErrorInvalidValue;
    note_launch();
    return e;
}

}  // namespace vvq2
