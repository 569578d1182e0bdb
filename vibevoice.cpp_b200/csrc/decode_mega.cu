// decode_mega.cu -- the whole greedy decode step of a Q8_0 Qwen2 stack as ONE
// persistent kernel (sm_100a), for 1 or 2 rows (one sequence or the CFG pair).
//
// A decode step of the 0.5B model is ~140 dependent stages (per layer:
// QKV -> attention -> merge -> O-proj -> gate/up -> down) over 0.9-9 MB
// matrices.  One CTA per SM walks the stage list and the weight stream does
// not stop:
//
//  * weights: every warp owns D slots of a shared-memory ring (D = 1 or 2)
//    and streams its own share of the CTA's weight tiles: the CTA's
//    contiguous row slice of every matrix of the WHOLE step, cut into tiles
//    of T rows, goes round robin over the 16 warps (tile i -> warp i % 16).
//    Right after computing a tile a warp bulk-copies (cp.async.bulk; a run
//    of Q8_0 rows with their scales is one contiguous range) its next tile
//    into the freed slot.  Weights do not depend on activations, so a warp's
//    next tiles -- often of the next stage -- are in flight while it waits
//    for its inputs or runs attention.
//  * hand-over between stages: there is no grid barrier.  Every value one
//    stage hands to the next (hidden rows, raw q|k|v, attention partials,
//    attention output, SwiGLU output) is written as a FLAGGED WORD, one
//    64-bit store of (tag << 32 | f32 bits).  A 64-bit aligned store is
//    single-copy atomic, so a reader that sees the expected tag sees the
//    value with it; the consumer polls exactly the words it needs until all
//    carry the tag of the current launch and stage, which costs one L2 round
//    trip after the last producer instead of a barrier (release fence, atomic
//    round trip, poll) followed by a separate read.  Each buffer is reused by
//    every layer: every stage consumes ALL words of its predecessor's buffer
//    (or, for attention, all words of its KV head group), so a writer of
//    layer l + 1 is causally after every reader of layer l and no word is
//    overwritten while still unread.
//  * each warp stages nothing of its own: the CTA stages the stage's
//    activation rows (RMSNorm'd where the layer norms) into shared memory,
//    then each warp computes its tiles' T x M dot products over the full K
//    (exact dequantized int8 weights x f32 activations, packed FFMA2),
//    reduces them with one transposing butterfly and applies the epilogue
//    (bias, residual add, SwiGLU, running argmax).
//  * attention: one item per (row, KV head, split of whole 64-key pages) per
//    CTA, run by all 512 threads (four quarters share the page's keys and
//    the group's q heads).  The first page of a CTA's first item is
//    requested by TMA as soon as the shared memory it lands in is free (past
//    keys do not depend on this step), i.e. during the previous layer's
//    down-projection hand-over.  The item applies RoPE to this step's raw q/k, patches the new
//    key/value row into its tile, appends it to the paged cache and writes an
//    (O, max, sum) partial; one CTA per (row, q head) merges the partials
//    (log-sum-exp) into the attention output.
//  * the end of the step: each CTA folds its lm_head rows into a running
//    argmax key (atomicMax); the last CTA to arrive (an acquire-release
//    counter) writes the token ids, advances the row positions and the launch
//    epoch the tags derive from.
//
// Every wait is bounded.  A wait that gives up records an error code, raises
// the global abort flag and this CTA's `fail` flag; every other poll checks
// them, CTAs skip their remaining work at the next CTA-wide check (a
// __syncthreads_or, so control flow stays uniform), wait for their bulk copies
// in flight and still arrive at the end-of-step counter.  The host then clears
// the flagged buffers and the abort flag before reporting the error.
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
constexpr int MAXG = 8;                 // q heads per KV head
constexpr int PAGE = KV_PAGE;           // keys per page / tile
constexpr int MAX_MERGE = MEGA_MAX_SPLITS;
constexpr uint32_t WAIT_POLLS = 1u << 24;   // mbarrier try_waits
constexpr uint32_t LL_POLLS = 1u << 21;     // L2 polls of a flagged word (~0.5 us each)
// flagged float4 groups each thread keeps in flight while staging: the
// hidden-row and attention stages have fewer groups than threads; the
// SwiGLU stage (M x F words) takes SB_FA groups (fewer round trips).
// (Requests in flight hold registers, and at every other stage more of them
// spill the GEMV tile loop: the kernel sits at the 128-register limit.)
constexpr int SB_FA = 3;
constexpr int SB_MERGE = 1;             // word pairs per thread in flight while a merge gathers partials
// pause between unsuccessful poll rounds.  Every waiting thread of every CTA
// polls, but a poll round is already one L2 round trip per thread, and on
// the config-2 step no pause measured best (0.571 ms against 0.576 at 32 ns
// and 0.588 at 128 ns); a stage with little work between hand-overs (64
// copies of one layer with a 64-wide FFN) prefers 128 ns (17.6 against
// 19.0 us per layer)
constexpr unsigned POLL_PAUSE_NS = 0;

enum { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_LM = 4 };

constexpr int AQ = 4;                   // quarters of the CTA in an attention item (4 x 128 threads)
constexpr int AKEYS = PAGE / AQ;        // keys of a page per quarter

struct Ctl {
    int fail;                      // a wait of this CTA gave up or the step is aborting
};

// Tags of the flagged words of one launch: 8 per layer plus the embedding.
// Never 0 (the value buffers are cleared to), distinct for 2^32 - 1 stages.
struct Tags {
    unsigned long long base;
    __device__ __forceinline__ uint32_t at(unsigned long long k) const {
        return (uint32_t)((base + k) % 0xffffffffull) + 1u;
    }
    __device__ __forceinline__ uint32_t x_in(int l) const { return at(l == 0 ? 0 : 8ull * (l - 1) + 6); }
    __device__ __forceinline__ uint32_t qkv(int l) const { return at(8ull * l + 1); }
    __device__ __forceinline__ uint32_t part(int l) const { return at(8ull * l + 2); }
    __device__ __forceinline__ uint32_t att(int l) const { return at(8ull * l + 3); }
    __device__ __forceinline__ uint32_t x_o(int l) const { return at(8ull * l + 4); }
    __device__ __forceinline__ uint32_t fa(int l) const { return at(8ull * l + 5); }
};

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// (The warp reconverges before going on: a warp left diverged by a one-thread
// branch must not enter the out-of-line stage_ll, whose body assumes a
// converged warp and is followed by aligned CTA barriers.)
__device__ __forceinline__ void trace_mark(const MegaArgs& a, int slot) {
    if (a.trace) {
        const unsigned long long t = gtimer();
        if (threadIdx.x == 0) a.trace[(size_t)slot * gridDim.x + blockIdx.x] = t;
        __syncwarp();
    }
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

// The first failure of a launch also records where: code, CTA, an index
// (word offset for flagged-word waits, else 0), the expected tag and the last
// word seen.
__device__ void raise_fail(const MegaArgs& a, Ctl& ctl, int code, long long where = 0, uint32_t tag = 0,
                           uint64_t seen = 0) {
    if (atomicCAS(a.err, 0, code) == 0 && a.err_info) {
        a.err_info[0] = ((unsigned long long)blockIdx.x << 32) | (uint32_t)code;
        a.err_info[1] = (unsigned long long)where;
        a.err_info[2] = ((unsigned long long)*(volatile unsigned int*)a.epoch << 32) | tag;
        a.err_info[3] = seen;
    }
    atomicExch(a.abort, 1);
    *(volatile int*)&ctl.fail = 1;
}

// Uniform over the CTA (and a CTA barrier): true once any thread of the CTA
// failed or another CTA raised the abort flag.
// (A CTA learns of another CTA's failure when one of its polls sees the
// abort flag; no global read is spent here.)
__device__ __forceinline__ bool cta_failed(const MegaArgs&, Ctl& ctl) {
    return __syncthreads_or(*(volatile int*)&ctl.fail) != 0;
}

// ------------------------------------------------------------ flagged words
__device__ __forceinline__ uint64_t ll_word(float v, uint32_t tag) {
    return ((uint64_t)tag << 32) | __float_as_uint(v);
}
__device__ __forceinline__ bool ll_ok(uint64_t w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float((uint32_t)w); }

__device__ __forceinline__ void ll_put(uint64_t* p, float v, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(ll_word(v, tag)) : "memory");
}
// two flagged words at a 16-byte aligned address (each word is its own atomic unit)
__device__ __forceinline__ void ll_put2(uint64_t* p, float v0, float v1, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(ll_word(v0, tag)),
                 "l"(ll_word(v1, tag))
                 : "memory");
}
__device__ __forceinline__ uint64_t ll_get(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ void ll_get2(const uint64_t* p, uint64_t& w0, uint64_t& w1) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
}

// Called every 32nd unsuccessful poll round: give up once the CTA is failing,
// the step is aborting, or the poll budget is spent (then raise the failure).
__device__ __forceinline__ bool poll_give_up(const MegaArgs& a, Ctl& ctl, uint32_t it, int code,
                                             const uint64_t* p = nullptr, uint32_t tag = 0, uint64_t seen = 0) {
    if (*(volatile int*)&ctl.fail || *(volatile int*)a.abort) {
        *(volatile int*)&ctl.fail = 1;
        return true;
    }
    if (it > LL_POLLS) {
        raise_fail(a, ctl, code, p ? (long long)(p - a.xl) : 0, tag, seen);
        return true;
    }
    return false;
}

// One flagged word, bounded.  Returns 0 after giving up (the CTA is failing).
__device__ float ll_wait(const MegaArgs& a, Ctl& ctl, const uint64_t* p, uint32_t tag, int code) {
    for (uint32_t it = 1;; ++it) {
        const uint64_t w = ll_get(p);
        if (ll_ok(w, tag)) return ll_val(w);
        if ((it & 31) == 0 && poll_give_up(a, ctl, it, code, p, tag, w)) return 0.f;
        __nanosleep(POLL_PAUSE_NS);
    }
}

// ------------------------------------------------------------ activations
// act layout: float4 index ((m * 4 + g) * NC + c) holds elements
// 16c + 4g .. 16c + 4g + 3 of row m, so the lanes of a warp (consecutive
// chunks c) read consecutive 16-byte words.
//
// The rows come from flagged words src[m][K] with tag `tag`: every thread
// requests up to SB groups of 4 words at once and re-polls only the groups
// not yet tagged, so a stage costs about one L2 round trip after its last
// producer.  Where the stage RMSNorms its input, act = x * w (the norm
// weight) and the per-warp partial sums of squares go to red[m][warp] (in a
// fixed order, independent of arrival order); the row scale
// 1/sqrt(mean(x^2) + eps) is applied to the dot products instead
// (W (x s o w) = s W (x o w)), so no second pass over act is needed.
// The caller follows with cta_failed() (the CTA barrier that publishes act).
template <int MB, int SB = 1>
__device__ void stage_ll(const MegaArgs& a, Ctl& ctl, const uint64_t* src, int K, uint32_t tag, const float* norm_w,
                         float* act, float* red) {
    __syncwarp();   // entered by converged warps only (see trace_mark)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NC = K / 16, K4 = K / 4, NI = MB * K4;   // group i: words 4i..4i+3 = row i / K4, float4 i % K4
    float4* act4 = reinterpret_cast<float4*>(act);
    float ss0 = 0.f, ss1 = 0.f;
    bool bad = false;
    for (int b0 = tid; b0 < NI && !bad; b0 += SB * NCT) {
        uint64_t w[SB][4];
        uint32_t pend = 0;
#pragma unroll
        for (int j = 0; j < SB; ++j) {
            const int i = b0 + j * NCT;
            if (i < NI) {
                ll_get2(src + 4 * (size_t)i, w[j][0], w[j][1]);
                ll_get2(src + 4 * (size_t)i + 2, w[j][2], w[j][3]);
                pend |= 1u << j;
            }
        }
        // poll: re-request only the groups not yet tagged
        for (uint32_t it = 1;; ++it) {
#pragma unroll
            for (int j = 0; j < SB; ++j)
                if (ll_ok(w[j][0], tag) && ll_ok(w[j][1], tag) && ll_ok(w[j][2], tag) && ll_ok(w[j][3], tag))
                    pend &= ~(1u << j);
            if (!pend) break;
            if ((it & 31) == 0 && poll_give_up(a, ctl, it, 6)) {
                bad = true;
                break;
            }
            __nanosleep(POLL_PAUSE_NS);
#pragma unroll
            for (int j = 0; j < SB; ++j) {
                if ((pend >> j) & 1u) {
                    const uint64_t* p = src + 4 * (size_t)(b0 + j * NCT);
                    ll_get2(p, w[j][0], w[j][1]);
                    ll_get2(p + 2, w[j][2], w[j][3]);
                }
            }
        }
        // values, in group order (the sums of squares do not depend on arrival order)
#pragma unroll
        for (int j = 0; j < SB; ++j) {
            const int i = b0 + j * NCT;
            if (i < NI) {
                const int m = MB == 1 ? 0 : (i >= K4 ? 1 : 0);
                const int k4 = i - m * K4;
                float4 v = make_float4(ll_val(w[j][0]), ll_val(w[j][1]), ll_val(w[j][2]), ll_val(w[j][3]));
                if (norm_w) {
                    const float4 nw = __ldg(reinterpret_cast<const float4*>(norm_w) + k4);
                    float q = m == 0 ? ss0 : ss1;
                    q = fmaf(v.x, v.x, q);
                    q = fmaf(v.y, v.y, q);
                    q = fmaf(v.z, v.z, q);
                    q = fmaf(v.w, v.w, q);
                    if (m == 0) ss0 = q;
                    else ss1 = q;
                    v.x = __fmul_rn(v.x, nw.x);
                    v.y = __fmul_rn(v.y, nw.y);
                    v.z = __fmul_rn(v.z, nw.z);
                    v.w = __fmul_rn(v.w, nw.w);
                }
                act4[(m * 4 + (k4 & 3)) * NC + (k4 >> 2)] = v;
            }
        }
    }
    if (norm_w) {
        const float t0 = warp_sum(ss0);
        if (lane == 0) red[warp] = t0;
        if (MB > 1) {
            const float t1 = warp_sum(ss1);
            if (lane == 0) red[NCW + warp] = t1;
        }
    }
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

// Tags a GEMV stage writes with (out) and reads its residual with (res).
struct StageTags {
    uint32_t out, res;
};

// One tile of a GEMV stage: math + epilogue.  The epilogue's global
// operands (old residual, bias) are loaded before the math so their latency
// overlaps it.  For lm_head the writer lanes keep a running argmax key.
template <int PH, int T, int MB>
__device__ __forceinline__ void tile_epilogue(const MegaArgs& a, Ctl& ctl, const MegaLayer* L, const uint8_t* tile,
                                              const Geo& g, int r, const float4* act4, int lane, float nsc,
                                              StageTags tg, unsigned long long& kbest) {
    constexpr int NR = PH == PH_GU ? 2 * T : T;
    constexpr int NV = NR * MB;
    constexpr int SH = 5 - Log2<NV>::v;
    const int idx = lane >> SH;              // = t * MB + m
    const int t = idx / MB, m = idx % MB;
    const bool writer = (lane & ((1 << SH) - 1)) == 0;
    const int nr = min(T, g.n - r);
    const int row = g.r0 + r + t;
    const bool w_ok = writer && t < nr;
    uint64_t pre_w = 0;
    float pre = 0.f;
    if constexpr (PH == PH_O || PH == PH_DOWN) {
        // this CTA wrote these rows in the previous hand-over (the O and down
        // slices cover the same rows), or the embedding did: already tagged
        if (w_ok) pre_w = ll_get(a.xl + (size_t)m * a.H + row);
    } else if constexpr (PH == PH_QKV) {
        if (w_ok && L->qkv_bias) pre = L->qkv_bias[row];
    }
    float acc[NV];
    tile_dot<NR, MB>(tile, (int)g.rs, g.K, act4, lane, acc);
    float v = warp_transpose_sum<NV>(acc, lane);
    if constexpr (PH == PH_QKV || PH == PH_GU || PH == PH_LM) v = __fmul_rn(v, nsc);   // RMSNorm scale of row m
    if constexpr (PH == PH_GU) {
        const float u = __shfl_sync(0xffffffffu, v, (lane + ((T * MB) << SH)) & 31);
        if (w_ok) ll_put(a.fal + (size_t)m * a.F + row, __fmul_rn(silu_ref(v), u), tg.out);   // silu(g) * u
    } else if constexpr (PH == PH_QKV) {
        if (w_ok) ll_put(a.qkvl + (size_t)m * a.qkv_rows + row, L->qkv_bias ? __fadd_rn(v, pre) : v, tg.out);
    } else if constexpr (PH == PH_LM) {
        if (w_ok) {
            const unsigned long long k = argmax_key(v, row);
            kbest = k > kbest ? k : kbest;
        }
    } else {   // O-proj / down: residual add (ggml_add(x, o))
        if (w_ok) {
            pre = ll_ok(pre_w, tg.res) ? ll_val(pre_w) : ll_wait(a, ctl, a.xl + (size_t)m * a.H + row, tg.res, 7);
            ll_put(a.xl + (size_t)m * a.H + row, __fadd_rn(pre, v), tg.out);
        }
    }
}

template <int PH, int MB>
__device__ void gemv_tiles(const MegaArgs& a, Ctl& ctl, int li, const Geo* tab, int nph, uint8_t* ring,
                           uint64_t* full, const float* act, const float* red, uint32_t& seq, WarpRing& wr, int D,
                           StageTags tg, unsigned long long* best) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const Geo& g = tab[PH == PH_LM ? 4 * a.n_layers : 4 * li + PH];
    const MegaLayer* L = PH == PH_LM ? nullptr : &a.layers[li];
    const float4* act4 = reinterpret_cast<const float4*>(act);
    const int j0 = (warp - (int)(seq % NCW) + NCW) % NCW;
    const volatile int* fl = &ctl.fail;
    unsigned long long kbest = 0ull;
    // this lane's row m is fixed by the lane and T; its RMSNorm scale where the stage norms
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
            case 1: tile_epilogue<PH, 1, MB>(a, ctl, L, tile, g, r, act4, lane, nsc, tg, kbest); break;
            case 2: tile_epilogue<PH, 2, MB>(a, ctl, L, tile, g, r, act4, lane, nsc, tg, kbest); break;
            default:
                if constexpr (PH != PH_GU) tile_epilogue<PH, 4, MB>(a, ctl, L, tile, g, r, act4, lane, nsc, tg, kbest);
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

// Key splits of row m: whole pages of a.split keys over min(pos + 1, kvlen).
__device__ __forceinline__ int row_splits(const MegaArgs& a, const RowMeta& rm) {
    const int lim = min(rm.pos + 1, rm.kvlen);
    return (lim + a.split - 1) / a.split;
}

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

// K and V of the first page of item x into the stage the CTA's page counter
// selects (the same stage cta_att_item uses for it).
template <int HD>
__device__ __forceinline__ void att_prefetch(const KvLayer& kv, const AttItem& x, uint8_t* att, uint64_t* abar,
                                             uint32_t ptiles) {
    constexpr int TB = PAGE * HD * 2;
    const size_t off = ((size_t)x.page0 * kv.n_kv + x.g) * PAGE * HD;
    uint64_t* bar = &abar[ptiles & 1];
    __half* kd = reinterpret_cast<__half*>(att + (ptiles & 1) * 2 * TB);
    tc::fence_proxy_async_smem();
    tc::mbar_arrive_expect_tx(bar, 2 * TB);
    bulk_g2s(kd, kv.k + off, TB, bar);
    bulk_g2s(kd + PAGE * HD, kv.v + off, TB, bar);
}

// Flagged word of the partial (O, max, sum) buffer: [row][kv head][split][q head of the group][hd + 2].
template <int HD>
__device__ __forceinline__ uint64_t* part_ptr(const MegaArgs& a, int m, int g, int s, int h) {
    const int G = a.nq / a.nkv;
    return a.pl + ((((size_t)m * a.nkv + g) * MAX_MERGE + s) * G + h) * (HD + 2);
}

// Shared state of the CTA's attention item (in the attention part of the
// shared region, after the two K|V page stages).
template <int HD>
struct __align__(16) AttSh {
    float qs[MAXG][HD];                // roped q, rounded to f16 (ggml FA converts Q to the K type)
    float sc[AQ][MAXG][AKEYS];         // per quarter: probabilities of its keys of the page
    float alpha[AQ][MAXG];             // per quarter: rescale of O on a new running max
    float og[AQ][MAXG][HD];            // per quarter: unnormalized O at the end of the item
    float mg[AQ][MAXG], lg[AQ][MAXG];  // per quarter: running max and sum
    __half kn[HD], vn[HD];             // this step's key (roped) and value row
};

// One attention item (row m, KV head g, split s: pages [j0, j1) of keys) by
// the whole CTA.  The 16 warps form AQ = 4 quarters of 128 threads; quarter
// q owns keys 16q .. 16q + 15 of every page, with its own online softmax:
//  * scores: thread (key kk, head slot hh) computes one q.k dot product over
//    HD (K read in a per-key rotated 16-byte order: no bank conflicts); the
//    16 threads of a head are a half warp, so max and sum are shuffles;
//  * P.V: thread (column pair dp, head slot hs) accumulates its heads'
//    two columns over the quarter's 16 keys.
// The quarters' (O, max, sum) are then merged (log-sum-exp) into the item's
// partial, or -- when the row has a single split -- its output.
// Pages live in two K|V stages (page t of the launch's page counter p uses
// stage p & 1); the first page may have been requested already (`prefetched`).
// Returns false (uniform over the CTA) after a wait gave up; pages it
// requested are waited for before it returns.
template <int HD>
__device__ bool cta_att_item(const MegaArgs& a, Ctl& ctl, const KvLayer& kv, const AttItem& x, uint8_t* att,
                             const float2* cs_row, uint64_t* abar, uint32_t& ptiles, bool prefetched,
                             uint32_t tag_qkv, uint32_t tag_out) {
    constexpr int TB = PAGE * HD * 2;           // bytes of K (or V) of one page of one head
    constexpr int half = HD / 2;
    constexpr int NCH = HD / 8;                 // 16-byte chunks of a K row
    constexpr int PAIRS = HD / 2;
    constexpr int HSUB = 128 / PAIRS;           // head slots of P.V per quarter (4 at hd 64, 2 at hd 128)
    constexpr int HPER = MAXG / HSUB;           // heads per P.V thread
    AttSh<HD>& sh = *reinterpret_cast<AttSh<HD>*>(att + 4 * TB);
    const int tid = threadIdx.x;
    const int q = tid >> 7, gtid = tid & 127;   // quarter, thread in quarter
    const int G = a.nq / a.nkv;
    const int m = x.m, g = x.g;
    const RowMeta& rm = x.rm;
    const int newj = rm.cidx;                   // cache index of this step's key/value
    const bool has_new = newj >= x.j0 && newj < x.j1;
    const uint32_t base = ptiles;
    auto stage_k = [&](uint32_t t) { return reinterpret_cast<__half*>(att + ((base + t) & 1) * 2 * TB); };
    auto issue = [&](uint32_t t) {             // page t of the item into its stage (one thread)
        const int page = __ldg(kv.block_table + (size_t)rm.seq * kv.max_pages + (x.j0 + (int)t * PAGE) / PAGE);
        const size_t off = ((size_t)page * kv.n_kv + g) * PAGE * HD;
        uint64_t* bar = &abar[(base + t) & 1];
        __half* kd = stage_k(t);
        tc::fence_proxy_async_smem();
        tc::mbar_arrive_expect_tx(bar, 2 * TB);
        bulk_g2s(kd, kv.k + off, TB, bar);
        bulk_g2s(kd + PAGE * HD, kv.v + off, TB, bar);
    };
    if (tid == 0) {
        if (!prefetched) issue(0);
        if (x.ntiles > 1) issue(1);
    }
    uint32_t issued = min(x.ntiles, 2);       // pages requested (identical in every thread)

    // this step's raw q (and new k, v): flagged words of the QKV stage.  Task
    // list: the G * hd/2 rotation pairs of q, the hd/2 pairs of k, the hd
    // words of v; thread t takes tasks t, t + 512; all requested at once,
    // then re-polled until tagged.
    constexpr int NTASK = (MAXG * half + half + HD + MT - 1) / MT;
    const uint64_t* qkv = a.qkvl + (size_t)m * a.qkv_rows;
    const uint64_t ready = (uint64_t)tag_qkv << 32;   // a word that needs no poll
    const int nq_t = G * half, nk_t = has_new ? half : 0, nv_t = has_new ? HD : 0;
    const uint64_t* pw[NTASK][2];
    uint64_t w[NTASK][2];
#pragma unroll
    for (int k = 0; k < NTASK; ++k) {
        const int t = tid + k * MT;
        pw[k][0] = pw[k][1] = nullptr;
        if (t < nq_t) {
            pw[k][0] = qkv + (size_t)(g * G + t / half) * HD + t % half;   // (q_h[i], q_h[i + hd/2])
            pw[k][1] = pw[k][0] + half;
        } else if (t < nq_t + nk_t) {
            pw[k][0] = qkv + (size_t)(a.nq + g) * HD + (t - nq_t);         // (k[i], k[i + hd/2])
            pw[k][1] = pw[k][0] + half;
        } else if (t < nq_t + nk_t + nv_t) {
            pw[k][0] = qkv + (size_t)(a.nq + a.nkv + g) * HD + (t - nq_t - nk_t);   // v[i]
        }
        w[k][0] = pw[k][0] ? ll_get(pw[k][0]) : ready;
        w[k][1] = pw[k][1] ? ll_get(pw[k][1]) : ready;
    }
    bool bad = false;
    for (uint32_t it = 1;; ++it) {
        bool ok = true;
#pragma unroll
        for (int k = 0; k < NTASK; ++k) ok = ok && ll_ok(w[k][0], tag_qkv) && ll_ok(w[k][1], tag_qkv);
        if (ok) break;
        if ((it & 31) == 0 && poll_give_up(a, ctl, it, 8)) {
            bad = true;
            break;
        }
        __nanosleep(POLL_PAUSE_NS);
#pragma unroll
        for (int k = 0; k < NTASK; ++k) {
            if (!ll_ok(w[k][0], tag_qkv)) w[k][0] = ll_get(pw[k][0]);
            if (!ll_ok(w[k][1], tag_qkv)) w[k][1] = ll_get(pw[k][1]);
        }
    }
#pragma unroll
    for (int k = 0; k < NTASK; ++k) {
        const int t = tid + k * MT;
        const float va = ll_val(w[k][0]), vb = ll_val(w[k][1]);
        if (t < nq_t) {
            const int h = t / half, i = t % half;
            const float2 cs = cs_row[i];
            sh.qs[h][i] = __half2float(__float2half_rn(__fsub_rn(__fmul_rn(va, cs.x), __fmul_rn(vb, cs.y))));
            sh.qs[h][i + half] = __half2float(__float2half_rn(__fadd_rn(__fmul_rn(va, cs.y), __fmul_rn(vb, cs.x))));
        } else if (t < nq_t + nk_t) {
            const int i = t - nq_t;
            const float2 cs = cs_row[i];
            sh.kn[i] = __float2half_rn(__fsub_rn(__fmul_rn(va, cs.x), __fmul_rn(vb, cs.y)));
            sh.kn[i + half] = __float2half_rn(__fadd_rn(__fmul_rn(va, cs.y), __fmul_rn(vb, cs.x)));
        } else if (t < nq_t + nk_t + nv_t) {
            sh.vn[t - nq_t - nk_t] = __float2half_rn(va);
        }
    }

    // scores ownership: key kk of the quarter, head slot hh (a half warp per head)
    const int kk = gtid & (AKEYS - 1), hh = gtid >> 4;
    const int key = q * AKEYS + kk;
    const int rot = key % NCH;
    const bool hrow = hh < G;
    float rmax = -INFINITY, rsum = 0.f;         // running max / sum of head hh over this quarter's keys
    // P.V ownership: column pair dp, heads hs, hs + HSUB, ...
    const int dp = gtid % PAIRS, hs = gtid / PAIRS;
    float2 o[HPER];
#pragma unroll
    for (int k = 0; k < HPER; ++k) o[k] = make_float2(0.f, 0.f);
    GroupSync qsync{1 + q};

    for (uint32_t t = 0; t < (uint32_t)x.ntiles; ++t) {
        if (!tc::mbar_wait(&abar[(base + t) & 1], ((base + t) >> 1) & 1)) {
            if (!*(volatile int*)&ctl.fail) raise_fail(a, ctl, 1);
            bad = true;
        }
        __half* K = stage_k(t);
        __half* V = K + PAGE * HD;
        const int tj0 = x.j0 + (int)t * PAGE;
        const int nk = min(PAGE, x.j1 - tj0);
        if (has_new && newj >= tj0 && newj < tj0 + PAGE) {
            // the page copy predates this step's row: patch it in (after the stage wait)
            __syncthreads();
            for (int d = tid; d < HD; d += MT) {
                K[(newj - tj0) * HD + d] = sh.kn[d];
                V[(newj - tj0) * HD + d] = sh.vn[d];
            }
        }
        if (__syncthreads_or(bad ? 1 : 0)) break;   // also publishes qs / kn / vn / the patch
        // ---- scores of the quarter's keys, running max / sum per head
        float sres = -INFINITY;
        if (hrow) {
            float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const int ch = (c + rot) % NCH;
                const uint4 raw = reinterpret_cast<const uint4*>(K + key * HD)[ch];
                const __half2* hp = reinterpret_cast<const __half2*>(&raw);
                const float4* qp = reinterpret_cast<const float4*>(&sh.qs[hh][ch * 8]);
                const float4 q0 = qp[0], q1 = qp[1];
                const float2 k0 = __half22float2(hp[0]), k1 = __half22float2(hp[1]);
                const float2 k2 = __half22float2(hp[2]), k3 = __half22float2(hp[3]);
                acc0 = fmaf(q0.x, k0.x, acc0);
                acc1 = fmaf(q0.y, k0.y, acc1);
                acc0 = fmaf(q0.z, k1.x, acc0);
                acc1 = fmaf(q0.w, k1.y, acc1);
                acc0 = fmaf(q1.x, k2.x, acc0);
                acc1 = fmaf(q1.y, k2.y, acc1);
                acc0 = fmaf(q1.z, k3.x, acc0);
                acc1 = fmaf(q1.w, k3.y, acc1);
            }
            if (key < nk) sres = (acc0 + acc1) * a.scale;
        }
        float tmax = sres;
#pragma unroll
        for (int o2 = 8; o2 >= 1; o2 >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o2));
        const float mnew = fmaxf(rmax, tmax);
        // no key of this head seen yet in this quarter: nothing to rescale, p = 0
        const float al = mnew == -INFINITY ? 1.f : expf(rmax - mnew);
        const float p = sres == -INFINITY ? 0.f : expf(sres - mnew);
        float psum = p;
#pragma unroll
        for (int o2 = 8; o2 >= 1; o2 >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o2);
        rmax = mnew;
        rsum = rsum * al + psum;
        if (hrow) {
            sh.sc[q][hh][kk] = p;
            if (kk == 0) sh.alpha[q][hh] = al;
        }
        qsync();
        // ---- O = O * alpha + P.V over the quarter's keys
#pragma unroll
        for (int k = 0; k < HPER; ++k) {
            const int h = hs + k * HSUB;
            if (h < G) {
                const float al2 = sh.alpha[q][h];
                float2 acc = make_float2(o[k].x * al2, o[k].y * al2);
#pragma unroll
                for (int j = 0; j < AKEYS; ++j) {
                    if (q * AKEYS + j >= nk) break;   // keys past the row: the stale page entries may hold any bits
                    const float2 v = __half22float2(reinterpret_cast<const __half2*>(V + (q * AKEYS + j) * HD)[dp]);
                    const float pj = sh.sc[q][h][j];
                    acc.x = fmaf(pj, v.x, acc.x);
                    acc.y = fmaf(pj, v.y, acc.y);
                }
                o[k] = acc;
            }
        }
        __syncthreads();   // the stage and sc are free again
        if (tid == 0 && issued < (uint32_t)x.ntiles) issue(issued);
        issued = min((uint32_t)x.ntiles, issued + (t + 2 < (uint32_t)x.ntiles ? 1u : 0u));
    }
    ptiles = base + issued;
    if (bad) {
        // pages requested but not consumed: wait (bounded) before the stages are reused
        for (uint32_t t = 0; t < issued; ++t) tc::mbar_wait(&abar[(base + t) & 1], ((base + t) >> 1) & 1, 1u << 20);
        return false;
    }
    // ---- append this step's K/V row to the paged cache (read by later steps)
    if (has_new) {
        const size_t off = kv_offset(kv, rm.seq, newj, g);
        for (int d = tid; d < HD; d += MT) {
            kv.k[off + d] = sh.kn[d];
            kv.v[off + d] = sh.vn[d];
        }
    }
    // ---- merge the quarters
    if (hrow && kk == 0) {
        sh.mg[q][hh] = rmax;
        sh.lg[q][hh] = rsum;
    }
#pragma unroll
    for (int k = 0; k < HPER; ++k) {
        const int h = hs + k * HSUB;
        if (h < G) reinterpret_cast<float2*>(&sh.og[q][h][0])[dp] = o[k];
    }
    __syncthreads();
    const bool single = x.nsplit == 1;
    for (int i = tid; i < G * HD; i += MT) {
        const int h = i / HD, d = i % HD;
        float mx = sh.mg[0][h];
#pragma unroll
        for (int qq = 1; qq < AQ; ++qq) mx = fmaxf(mx, sh.mg[qq][h]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int qq = 0; qq < AQ; ++qq) {
            const float w = sh.mg[qq][h] == -INFINITY ? 0.f : expf(sh.mg[qq][h] - mx);
            num = fmaf(w, sh.og[qq][h][d], num);
            den = fmaf(w, sh.lg[qq][h], den);
        }
        if (single) {
            ll_put(a.attl + (size_t)m * a.nq * HD + (size_t)(g * G + h) * HD + d, num / den, tag_out);
        } else {
            uint64_t* pp = part_ptr<HD>(a, m, g, x.s, h);
            ll_put(pp + d, num, tag_out);
            if (d == 0) ll_put2(pp + HD, mx, den, tag_out);
        }
    }
    __syncthreads();   // sh and the stages are reused by the next item
    return true;
}

// Log-sum-exp merge of the ns partials of (row m, q head qh) by the whole CTA
// into the attention words of the head.  `scr`: shared scratch of
// ns * (HD + 2) + 2 * MAX_MERGE floats.  Returns false (uniform) after a
// poll gave up.
template <int HD>
__device__ bool cta_merge(const MegaArgs& a, Ctl& ctl, int m, int qh, int ns, uint32_t tag_part, uint32_t tag_out,
                          float* scr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.nq / a.nkv;
    const int g = qh / G, h = qh % G;
    constexpr int W2 = (HD + 2) / 2;                  // word pairs per split
    float* wts = scr + (size_t)MAX_MERGE * (HD + 2);  // [ns]
    float* inv = wts + MAX_MERGE;                     // [1]
    const size_t sstride = (size_t)G * (HD + 2);      // words between splits
    const uint64_t* src = part_ptr<HD>(a, m, g, 0, h);
    const int NP = ns * W2;
    bool bad = false;
    for (int b0 = 0; b0 < NP && !bad; b0 += SB_MERGE * NCT) {
        uint64_t w[SB_MERGE][2];
        uint32_t pend = 0;
#pragma unroll
        for (int j = 0; j < SB_MERGE; ++j) {
            const int p = b0 + j * NCT + tid;
            if (p < NP) {
                ll_get2(src + (p / W2) * sstride + 2 * (p % W2), w[j][0], w[j][1]);
                pend |= 1u << j;
            }
        }
        for (uint32_t it = 1; pend; ++it) {
#pragma unroll
            for (int j = 0; j < SB_MERGE; ++j) {
                if ((pend >> j) & 1u) {
                    const int p = b0 + j * NCT + tid;
                    if (ll_ok(w[j][0], tag_part) && ll_ok(w[j][1], tag_part)) {
                        pend &= ~(1u << j);
                        scr[(p / W2) * (HD + 2) + 2 * (p % W2)] = ll_val(w[j][0]);
                        scr[(p / W2) * (HD + 2) + 2 * (p % W2) + 1] = ll_val(w[j][1]);
                    } else {
                        ll_get2(src + (p / W2) * sstride + 2 * (p % W2), w[j][0], w[j][1]);
                    }
                }
            }
            if (pend && (it & 31) == 0 && poll_give_up(a, ctl, it, 9)) {
                bad = true;
                break;
            }
            if (pend) __nanosleep(POLL_PAUSE_NS);
        }
    }
    if (__syncthreads_or(bad ? 1 : 0)) return false;
    if (warp == 0) {
        float mx = -INFINITY;
        for (int s = lane; s < ns; s += 32) mx = fmaxf(mx, scr[s * (HD + 2) + HD]);
        mx = warp_max(mx);
        float den = 0.f;
        for (int s = lane; s < ns; s += 32) {
            const float w = expf(scr[s * (HD + 2) + HD] - mx);
            wts[s] = w;
            den = fmaf(w, scr[s * (HD + 2) + HD + 1], den);
        }
        den = warp_sum(den);
        if (lane == 0) inv[0] = 1.0f / den;
    }
    cbar();
    if (tid < HD) {
        float num = 0.f;
        for (int s = 0; s < ns; ++s) num = fmaf(wts[s], scr[s * (HD + 2) + tid], num);
        ll_put(a.attl + (size_t)m * a.nq * HD + (size_t)qh * HD + tid, num * inv[0], tag_out);
    }
    cbar();   // scr is reused by the next merge
    return true;
}

// ------------------------------------------------------------ kernel
template <int HD, int MB>
__global__ void __launch_bounds__(MT, 1) k_decode_mega(const MegaArgs a) {
    extern __shared__ __align__(1024) uint8_t dyn[];
    __shared__ __align__(8) uint64_t full[MAX_STAGES];
    __shared__ __align__(8) uint64_t abar[2];     // the two K|V page stages of the attention items
    __shared__ float red[2 * NCW];
    __shared__ unsigned long long best[2];
    __shared__ float2 rope_cs[2][64];              // RoPE (cos, sin) per row: positions are fixed for the launch
    __shared__ Ctl ctl;
    // state kept in shared memory rather than registers: the GEMV tile loop
    // needs every register, and values live across it would spill there
    __shared__ unsigned long long s_base;          // tag base of this launch
    __shared__ AttItem s_x0;                       // this CTA's first attention item
    __shared__ int s_pre;                          // ... exists
    __shared__ int s_pending;                      // ... its page is requested, not yet consumed
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint8_t* region = dyn;                         // activations / merge scratch | attention tiles + state
    uint8_t* ring = dyn + a.union_bytes;
    Geo* tab = reinterpret_cast<Geo*>(ring + (size_t)a.nstage * a.slot_bytes);   // [4 * n_layers + 1]
    const int nph = 4 * a.n_layers + 1;
    const int D = a.nstage / NCW;
    float* act = reinterpret_cast<float*>(region);
    if (tid == 0) {
        s_base = (unsigned long long)(*(volatile unsigned int*)a.epoch) * (8ull * a.n_layers + 8ull);
        ctl.fail = 0;
        for (int i = 0; i < a.nstage; ++i) tc::mbar_init(&full[i], 1);
        for (int i = 0; i < 2; ++i) tc::mbar_init(&abar[i], 1);
        tc::mbar_fence_init();
    }
    trace_mark(a, 0);
    if (tid < 2) best[tid] = 0ull;
    // this CTA's tile geometry of every stage of the step
    for (int p = tid; p < nph; p += NCT)
        tab[p] = phase_geo(a, p == nph - 1 ? 0 : p / 4, p == nph - 1 ? PH_LM : p % 4);
    __syncthreads();

    // every warp requests its first D tiles (layer 0's weights land during the embedding)
    WarpRing wr;
    wr.used = wr.issued = 0;
    wr.ip = 0;
    wr.ij = warp;
    ring_normalize(wr, tab, nph);
    for (int d = 0; d < D; ++d) ring_issue(wr, tab, nph, ring, full, warp, lane, D, a.slot_bytes);

    // attention: this CTA's first item is the same in every layer of the launch
    uint8_t* att = region + a.att_off;
    if (tid == 0) {
        AttItem x0;
        s_pre = (int)blockIdx.x < a.nsplit * a.nkv * MB && att_item_geo(a, blockIdx.x, x0);
        s_x0 = x0;
        s_pending = 0;
    }
    __syncthreads();
    uint32_t ptiles = 0;                 // K|V pages this CTA has requested in the launch
    // request the first item's page for layer li (the stages are free)
    auto prefetch = [&](int li) {
        if (tid == 0 && s_pre) {
            att_prefetch<HD>(a.layers[li].kv, s_x0, att, abar, ptiles);
            s_pending = 1;
        }
        __syncwarp();   // reconverge before stage_ll (see trace_mark)
    };
    prefetch(0);   // the attention region is free from the start

    // ---- token embedding: X[m] = dequant(tok_embd[tok[m]]) as flagged words
    {
        const int H = a.H;
        const DevW& E = a.tok_embd;
        const uint32_t t0 = Tags{s_base}.x_in(0);
        for (int t = blockIdx.x * NCT + tid; t < MB * H; t += gridDim.x * NCT) {
            const int m = t / H, k = t % H;
            const int r = a.tok[m];
            float v = 0.f;
            if (r >= 0 && r < E.rows) {
                const uint8_t* rp = E.q + (size_t)r * E.row_stride;
                const float d = __half2float(*reinterpret_cast<const __half*>(rp + H + (k / 32) * 2));
                v = __fmul_rn((float)((int)rp[k] - 128), d);   // quants stored as q + 128
            }
            ll_put(a.xl + t, v, t0);
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
    bool failed = false;
    for (int li = 0; li < a.n_layers; ++li) {
        const MegaLayer& L = a.layers[li];
        const int tb = 1 + 10 * li;
        const Tags tg{*(volatile unsigned long long*)&s_base};
        if (li > 0) {
            cbar();                      // the previous down tiles are done with act
            prefetch(li);
        }
        trace_mark(a, tb);
        // 1. RMSNorm + QKV (+bias) -> raw q|k|v words
        // (a CTA with no rows in a stage stages nothing: nothing downstream
        // waits for it, so the words it would read may already be renewed)
        if (tab[4 * li + PH_QKV].ntiles) stage_ll<MB>(a, ctl, a.xl, a.H, tg.x_in(li), L.attn_norm, act, red);
        if ((failed = cta_failed(a, ctl))) break;
        trace_mark(a, tb + 1);
        gemv_tiles<PH_QKV, MB>(a, ctl, li, tab, nph, ring, full, act, red, seq, wr, D, {tg.qkv(li), 0u}, best);
        trace_mark(a, tb + 2);
        // 2. attention items, one per CTA at a time (the attention region is not act)
        {
            const int pre = s_pre;
            for (int it = blockIdx.x; it < a.nsplit * a.nkv * MB && !failed; it += gridDim.x) {
                const bool first = it == (int)blockIdx.x;
                AttItem x;
                if (first && pre) x = s_x0;
                else if (!att_item_geo(a, it, x)) continue;
                const bool pf = first && pre;
                __syncthreads();   // every warp is done with its QKV tiles' shared reads of s_x0 / sh
                if (pf && tid == 0) s_pending = 0;
                failed = !cta_att_item<HD>(a, ctl, L.kv, x, att, rope_cs[x.m], abar, ptiles, pf, tg.qkv(li),
                                           x.nsplit == 1 ? tg.att(li) : tg.part(li));
            }
        }
        if ((failed = cta_failed(a, ctl))) break;
        trace_mark(a, tb + 3);
        // 3. merges: one (row, q head) per CTA from the top of the grid
        for (int u = gridDim.x - 1 - blockIdx.x; u < MB * a.nq && !failed; u += gridDim.x) {
            const int m = u / a.nq;
            const int ns = row_splits(a, a.meta[m]);
            if (ns > 1) failed = !cta_merge<HD>(a, ctl, m, u % a.nq, ns, tg.part(li), tg.att(li), act);
        }
        if (failed) break;
        trace_mark(a, tb + 4);
        // 4. O-proj + residual
        if (tab[4 * li + PH_O].ntiles) stage_ll<MB>(a, ctl, a.attl, a.nq * HD, tg.att(li), nullptr, act, red);
        if ((failed = cta_failed(a, ctl))) break;
        trace_mark(a, tb + 5);
        gemv_tiles<PH_O, MB>(a, ctl, li, tab, nph, ring, full, act, red, seq, wr, D, {tg.x_o(li), tg.x_in(li)},
                             best);
        // 5. RMSNorm + gate/up + SwiGLU
        cbar();
        trace_mark(a, tb + 6);
        if (tab[4 * li + PH_GU].ntiles) stage_ll<MB>(a, ctl, a.xl, a.H, tg.x_o(li), L.ffn_norm, act, red);
        if ((failed = cta_failed(a, ctl))) break;
        trace_mark(a, tb + 7);
        gemv_tiles<PH_GU, MB>(a, ctl, li, tab, nph, ring, full, act, red, seq, wr, D, {tg.fa(li), 0u}, best);
        // 6. down + residual
        cbar();
        trace_mark(a, tb + 8);
        if (tab[4 * li + PH_DOWN].ntiles) stage_ll<MB, SB_FA>(a, ctl, a.fal, a.F, tg.fa(li), nullptr, act, red);
        if ((failed = cta_failed(a, ctl))) break;
        trace_mark(a, tb + 9);
        gemv_tiles<PH_DOWN, MB>(a, ctl, li, tab, nph, ring, full, act, red, seq, wr, D,
                                {tg.x_in(li + 1), tg.x_o(li)}, best);
    }
    // output norm + lm_head + argmax
    if (!failed) {
        const Tags tg{*(volatile unsigned long long*)&s_base};
        cbar();
        trace_mark(a, 1 + 10 * a.n_layers);
        if (tab[4 * a.n_layers].ntiles) stage_ll<MB>(a, ctl, a.xl, a.H, tg.x_in(a.n_layers), a.out_norm, act, red);
        failed = cta_failed(a, ctl);
        if (!failed) {
            trace_mark(a, 2 + 10 * a.n_layers);
            gemv_tiles<PH_LM, MB>(a, ctl, 0, tab, nph, ring, full, act, red, seq, wr, D, {0u, 0u}, best);
            cbar();
            if (tid < MB && best[tid]) atomicMax(a.amax + tid, best[tid]);
        }
    }
    // copies still in flight (only after a failure): wait for them before exiting
    for (uint32_t k = wr.used; k < wr.issued; ++k)
        tc::mbar_wait(&full[warp + NCW * (int)(k % D)], (k / D) & 1, 1u << 20);
    if (tid == 0 && s_pending) tc::mbar_wait(&abar[ptiles & 1], (ptiles >> 1) & 1, 1u << 20);
    cbar();
    trace_mark(a, 3 + 10 * a.n_layers);
    if (tid == 0) {
        // arrival (releases this CTA's argmax keys); the last CTA ends the step
        unsigned int prev;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.done) : "memory");
        if (prev == gridDim.x - 1) {
            const bool ok = *(volatile int*)a.abort == 0;
            for (int m = 0; m < MB; ++m) {
                volatile unsigned long long* am = a.amax + m;
                if (ok) {
                    a.tok[m] = argmax_key_index(*am);
                    RowMeta r = a.meta[m];
                    r.pos += 1;
                    r.cidx += 1;
                    r.kvlen += 1;
                    a.meta[m] = r;
                }
                *am = 0ull;   // ready for the next launch
            }
            *(volatile unsigned int*)a.done = 0u;
            __threadfence();
            atomicAdd(a.epoch, 1u);
        }
        trace_mark(a, 4 + 10 * a.n_layers);
    }
}

template <int HD, int MB>
cudaError_t set_smem(int bytes) {
    return cudaFuncSetAttribute(k_decode_mega<HD, MB>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <int HD>
size_t att_region_bytes() {
    return (size_t)4 * PAGE * HD * 2 + sizeof(AttSh<HD>);   // two K|V page stages + item state
}

}  // namespace

// Shared region before the ring: the staged activation rows (up to M x kmax
// f32), the merge scratch, and -- past the rows the QKV stage stages, so a
// page prefetched during the previous layer survives that staging -- the
// attention groups' page tiles and state.
int decode_mega_att_offset(int M, int H) { return (M * H * 4 + 1023) / 1024 * 1024; }

int decode_mega_union_bytes(int hd, int M, int kmax, int H) {
    const size_t act = (size_t)M * kmax * 4;
    const size_t att = (size_t)decode_mega_att_offset(M, H) + (hd == 64 ? att_region_bytes<64>() : att_region_bytes<128>());
    const size_t merge = ((size_t)MAX_MERGE * (hd + 2) + 2 * MAX_MERGE) * 4;
    return (int)((std::max({act, att, merge}) + 1023) / 1024 * 1024);
}

int decode_mega_max_stages() { return MAX_STAGES; }

int decode_mega_consumer_warps() { return NCW; }

int decode_mega_att_groups() { return 1; }

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
        a.nsplit > MAX_MERGE || !t_ok || !pow2_le4(a.t_qkv) || !pow2_le4(a.t_o) || !pow2_le4(a.t_down) ||
        !pow2_le4(a.t_lm) || a.slot_bytes % 16 || a.union_bytes % 1024 || a.att_off % 1024 ||
        a.H % 16 || a.F % 16 || (a.nq * a.hd) % 16)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.grid);
    cfg.blockDim = dim3(MT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    // all CTAs co-resident: a CTA polls words that other CTAs of the same launch produce
    attr[0].id = cudaLaunchAttributeCooperative;
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
