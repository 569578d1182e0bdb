// decode_mega.cu -- the whole greedy decode step of a Q8_0 Qwen2 stack as ONE
// persistent kernel (sm_100a), for 1 or 2 rows (one sequence or the CFG pair).
//
// A decode step of the 0.5B model is ~120 dependent phases (per layer:
// QKV -> attention -> O-proj -> gate/up -> down) over 0.9-9 MB matrices.  As
// separate launches every phase pays launch and prologue latency and starts
// its weight stream cold.  Here one CTA per SM walks the phase list,
// separated by grid-wide barriers, and the weight stream does not stop:
//
//  * warp 15 of every CTA is a producer.  Its lane 0 walks the CTA's weight
//    tiles of the WHOLE step in consumption order (this CTA's contiguous row
//    slice of every matrix, cut into tiles of T rows) and bulk-copies them
//    (cp.async.bulk; a run of Q8_0 rows with their scales is one contiguous
//    range) into a ring of shared-memory slots, gated only by free slots.
//    Weights do not depend on activations, so while the consumers wait in a
//    grid barrier or run attention, the next phases' weights are landing.
//  * warps 0..14 consume: stage the phase's activation rows (RMSNorm'd where
//    the layer norms) from L2 into shared memory; then each warp takes whole
//    tiles (round robin), computes T x M dot products over the full K (exact
//    dequantized int8 weights x f32 activations, packed FFMA2), reduces them
//    with one transposing butterfly and applies the epilogue (bias, residual
//    add, SwiGLU, running argmax) straight to global memory.
//  * attention: one item per (row, KV head, split of whole 64-key pages) on
//    128-thread groups.  The first pages of each group's first item are
//    requested by TMA BEFORE the QKV -> attention barrier (past keys do not
//    depend on this step).  The item applies RoPE to this step's raw q/k,
//    patches the new key/value row into its tile, appends it to the paged
//    cache, and the last split to finish merges the partials (log-sum-exp).
//
// Every wait is bounded.  A wait that gives up records an error code, raises
// the global abort flag and this CTA's `fail` flag; all warps then skip the
// remaining work (control flow only changes at grid barriers, where it is
// uniform) and the producer waits for its copies in flight before returning.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace vvq2 {

namespace {

constexpr int MT = 512;                 // threads per CTA
constexpr int NCW = 15;                 // consumer warps
constexpr int NCT = NCW * 32;           // consumer threads
constexpr int PRODUCER = 15;            // producer warp
constexpr int BAR_CONS = 1;             // named barrier of the consumer threads (2.. = attention groups)
constexpr int MAX_STAGES = 32;
constexpr int ATT_THREADS = 128;
constexpr int MAXG = 8;                 // q heads per KV head
constexpr int PAGE = KV_PAGE;           // keys per page / tile
constexpr int MAX_MERGE = 64;
constexpr uint32_t BAR_POLLS = 1u << 22;
constexpr uint32_t WAIT_POLLS = 1u << 24;

enum { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_LM = 4 };

template <int HD>
struct AttConst {
    static constexpr int NG = HD >= 128 ? 2 : 3;                 // attention groups per CTA
    static constexpr int TILE_BYTES = PAGE * HD * 2;             // one page of K (or V) of one head
    static constexpr int GROUP_BYTES = 4 * TILE_BYTES;           // K, V x 2 stages
};

// per-group attention state (in the phase-shared dynamic region)
template <int HD>
struct __align__(16) AttSh {
    float qs[MAXG][HD];            // roped q, rounded to f16 (ggml FA converts Q to the K type)
    float sc[MAXG][PAGE];
    float run_max[MAXG], run_sum[MAXG], alpha[MAXG];
    float wts[MAXG][MAX_MERGE];
    float inv_den[MAXG];
    float2 cs[HD / 2];             // RoPE (cos, sin) of this row's position
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

__device__ __forceinline__ void cbar() { asm volatile("bar.sync %0, %1;" ::"n"(BAR_CONS), "n"(NCT) : "memory"); }

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

// Grid barrier over the consumer threads of every CTA.
__device__ void grid_sync(const MegaArgs& a, Ctl& ctl) {
    // generic global writes (K/V rows) are read by TMA in later steps
    asm volatile("fence.proxy.async.global;" ::: "memory");
    cbar();
    if (threadIdx.x == 0) {
        trace_mark(a, 1 + 2 * ctl.nbar);
        ctl.target += gridDim.x;
        __threadfence();
        atomicAdd(a.bar_count, 1ull);
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
            __nanosleep(20);
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
    return g;
}

// ------------------------------------------------------------ producer
__device__ void producer(const MegaArgs& a, uint8_t* ring, uint64_t* full, uint64_t* empty, Ctl& ctl) {
    const volatile int* fl = &ctl.fail;
    const int nst = a.nstage;
    uint32_t seq = 0;
    bool ok = true;
    for (int li = 0; li <= a.n_layers && ok; ++li) {
        const int nph = li == a.n_layers ? 1 : 4;
        for (int ph = 0; ph < nph && ok; ++ph) {
            const Geo g = phase_geo(a, li, li == a.n_layers ? PH_LM : ph);
            for (int r = 0; r < g.n; r += g.T) {
                const int slot = (int)(seq % nst);
                if (seq >= (uint32_t)nst && !wait_or_fail(&empty[slot], ((seq / nst) - 1) & 1, fl)) {
                    ok = false;
                    break;
                }
                const uint32_t b0 = (uint32_t)(min(g.T, g.n - r) * g.rs);
                uint8_t* dst = ring + (size_t)slot * a.slot_bytes;
                tc::fence_proxy_async_smem();   // consumers' generic reads of the slot are ordered before
                tc::mbar_arrive_expect_tx(&full[slot], g.p1 ? 2 * b0 : b0);
                bulk_g2s(dst, g.p0 + (size_t)r * g.rs, b0, &full[slot]);
                if (g.p1) bulk_g2s(dst + (size_t)g.T * g.rs, g.p1 + (size_t)r * g.rs, b0, &full[slot]);
                ++seq;
            }
        }
    }
    // drain: every issued copy has landed before the CTA exits.  (Slot i is
    // always consumed by warp i % NCW: a consumer never polls a slot's
    // barrier before the slot's previous tile has landed and been released.)
    const uint32_t lo = seq > (uint32_t)nst ? seq - nst : 0;
    for (uint32_t s = lo; s < seq; ++s) tc::mbar_wait(&full[s % nst], (s / nst) & 1, 1u << 20);
}

// ------------------------------------------------------------ activations
// act layout: float4 index ((m * 4 + g) * NC + c) holds elements
// 16c + 4g .. 16c + 4g + 3 of row m, so the lanes of a warp (consecutive
// chunks c) read consecutive 16-byte words.
template <int MB>
__device__ void stage(const MegaArgs& a, const float* x, const float* norm_w, int K, float* act, float* red,
                      float* scl) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NC = K / 16, K4 = K / 4;
    float4* act4 = reinterpret_cast<float4*>(act);
    float ss[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) ss[m] = 0.f;
    for (int k4 = tid; k4 < K4; k4 += NCT) {
        const int c = k4 >> 2, g = k4 & 3;
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(x + (size_t)m * K) + k4);
            ss[m] = fmaf(v.x, v.x, ss[m]);
            ss[m] = fmaf(v.y, v.y, ss[m]);
            ss[m] = fmaf(v.z, v.z, ss[m]);
            ss[m] = fmaf(v.w, v.w, ss[m]);
            act4[(m * 4 + g) * NC + c] = v;
        }
    }
    if (norm_w) {
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            const float w = warp_sum(ss[m]);
            if (lane == 0) red[m * NCW + warp] = w;
        }
        cbar();
        if (tid < MB) {
            float t = 0.f;
            for (int w = 0; w < NCW; ++w) t += red[tid * NCW + w];
            scl[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), a.eps)));
        }
        cbar();
        for (int k4 = tid; k4 < K4; k4 += NCT) {
            const int c = k4 >> 2, g = k4 & 3;
            const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w) + k4);
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                float4 t = act4[(m * 4 + g) * NC + c];
                const float s = scl[m];
                t.x = __fmul_rn(__fmul_rn(t.x, s), w.x);   // (x * scale) * w: ggml_rms_norm, then ggml_mul
                t.y = __fmul_rn(__fmul_rn(t.y, s), w.y);
                t.z = __fmul_rn(__fmul_rn(t.z, s), w.z);
                t.w = __fmul_rn(__fmul_rn(t.w, s), w.w);
                act4[(m * 4 + g) * NC + c] = t;
            }
        }
    }
    cbar();
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
                const uint32_t w = word(q, g) ^ 0x80808080u;   // q + 128 as unsigned bytes
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

// One tile of a GEMV phase: math + epilogue.
template <int PH, int T, int MB>
__device__ __forceinline__ void tile_epilogue(const MegaArgs& a, const MegaLayer* L, const uint8_t* tile,
                                              const Geo& g, int r, const float4* act4, int lane,
                                              unsigned long long* best) {
    constexpr int NR = PH == PH_GU ? 2 * T : T;
    constexpr int NV = NR * MB;
    constexpr int SH = 5 - Log2<NV>::v;
    float acc[NV];
    tile_dot<NR, MB>(tile, (int)g.rs, g.K, act4, lane, acc);
    float v = warp_transpose_sum<NV>(acc, lane);
    const int idx = lane >> SH;              // = t * MB + m
    const int t = idx / MB, m = idx % MB;
    const bool writer = (lane & ((1 << SH) - 1)) == 0;
    const int nr = min(T, g.n - r);
    if constexpr (PH == PH_GU) {
        const float u = __shfl_sync(0xffffffffu, v, (lane + ((T * MB) << SH)) & 31);
        if (writer && t < nr) a.FA[(size_t)m * a.F + g.r0 + r + t] = __fmul_rn(silu_ref(v), u);   // silu(g) * u
    } else if constexpr (PH == PH_QKV) {
        if (writer && t < nr) {
            const int row = g.r0 + r + t;
            if (L->qkv_bias) v = __fadd_rn(v, L->qkv_bias[row]);
            a.QKV[(size_t)m * a.qkv_rows + row] = v;
        }
    } else if constexpr (PH == PH_LM) {
        if (writer && t < nr) atomicMax(&best[m], argmax_key(v, g.r0 + r + t));
    } else {   // O-proj / down: residual add into X (ggml_add(x, o))
        if (writer && t < nr) {
            float* dst = a.X + (size_t)m * a.H + g.r0 + r + t;
            *dst = __fadd_rn(__ldcg(dst), v);
        }
    }
}

template <int PH, int MB>
__device__ void gemv_tiles(const MegaArgs& a, int li, const uint8_t* ring, uint64_t* full, uint64_t* empty,
                           const float* act, uint32_t& seq, Ctl& ctl, unsigned long long* best) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const Geo g = phase_geo(a, li, PH);
    const MegaLayer* L = PH == PH_LM ? nullptr : &a.layers[li];
    const int ntiles = (g.n + g.T - 1) / g.T;
    const float4* act4 = reinterpret_cast<const float4*>(act);
    const int j0 = (warp - (int)(seq % NCW) + NCW) % NCW;
    const volatile int* fl = &ctl.fail;
    for (int j = j0; j < ntiles; j += NCW) {
        const uint32_t s = seq + j;
        const int slot = (int)(s % a.nstage);
        if (!wait_or_fail(&full[slot], (s / a.nstage) & 1, fl)) {
            if (lane == 0 && !*fl) raise_fail(a, ctl, 4);
            break;
        }
        const uint8_t* tile = ring + (size_t)slot * a.slot_bytes;
        const int r = j * g.T;
        switch (g.T) {
            case 1: tile_epilogue<PH, 1, MB>(a, L, tile, g, r, act4, lane, best); break;
            case 2: tile_epilogue<PH, 2, MB>(a, L, tile, g, r, act4, lane, best); break;
            case 4: tile_epilogue<PH, 4, MB>(a, L, tile, g, r, act4, lane, best); break;
            default:
                if constexpr (PH != PH_GU) tile_epilogue<PH, 8, MB>(a, L, tile, g, r, act4, lane, best);
                break;
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[slot]);
    }
    seq += ntiles;
}

// ------------------------------------------------------------ attention
struct AttItem {
    int m, g, s, nsplit, j0, j1, ntiles;
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
    return true;
}

template <int HD>
__device__ __forceinline__ void att_issue(const KvLayer& kv, const AttItem& x, int tile, __half* kt, __half* vt,
                                          uint64_t* bar) {
    constexpr int TB = AttConst<HD>::TILE_BYTES;
    const int b = tile & 1;
    const int page = __ldg(kv.block_table + (size_t)x.rm.seq * kv.max_pages + (x.j0 + tile * PAGE) / PAGE);
    const size_t off = ((size_t)page * kv.n_kv + x.g) * PAGE * HD;
    tc::mbar_arrive_expect_tx(&bar[b], 2 * TB);
    bulk_g2s(kt + b * PAGE * HD, kv.k + off, TB, &bar[b]);
    bulk_g2s(vt + b * PAGE * HD, kv.v + off, TB, &bar[b]);
}

// One attention item on a 128-thread group.  The first two tiles may already
// be in flight (`prefetched`).  Returns false after a timed-out wait.
template <int HD>
__device__ bool att_item(const MegaArgs& a, const KvLayer& kv, const AttItem& x, int tid, __half* kt, __half* vt,
                         AttSh<HD>& sh, uint64_t* bar, uint32_t (&uses)[2], bool prefetched, GroupSync sync) {
    const int lane = tid & 31, warp = tid >> 5;
    const int G = a.nq / a.nkv;
    constexpr int half = HD / 2;
    const int m = x.m, g = x.g;
    const RowMeta& rm = x.rm;
    const int newj = rm.cidx;   // cache index of this step's key/value
    const bool has_new = newj >= x.j0 && newj < x.j1;

    if (tid == 0) sh.failed = 0;
    // RoPE table of this row's position (ggml CPU theta recurrence)
    for (int i = tid; i < half; i += ATT_THREADS) {
        float th = (float)rm.pos;
        for (int k = 0; k < i; ++k) th = __fmul_rn(th, a.rope_ts);
        sh.cs[i] = make_float2(cosf(th), sinf(th));
    }
    if (tid < MAXG) {
        sh.run_max[tid] = -INFINITY;
        sh.run_sum[tid] = 0.f;
    }
    sync();
    const float* qkv = a.QKV + (size_t)m * a.qkv_rows;
    for (int t = tid; t < G * half; t += ATT_THREADS) {
        const int h = t / half, i = t % half;
        const float* q = qkv + (size_t)(g * G + h) * HD;
        const float x0 = __ldcg(q + i), x1 = __ldcg(q + i + half);
        const float2 cs = sh.cs[i];
        const float y0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
        const float y1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
        sh.qs[h][i] = __half2float(__float2half_rn(y0));
        sh.qs[h][i + half] = __half2float(__float2half_rn(y1));
    }
    if (has_new) {
        const float* k = qkv + (size_t)(a.nq + g) * HD;
        const float* v = qkv + (size_t)(a.nq + a.nkv + g) * HD;
        for (int i = tid; i < half; i += ATT_THREADS) {
            const float x0 = __ldcg(k + i), x1 = __ldcg(k + i + half);
            const float2 cs = sh.cs[i];
            sh.kn[i] = __float2half_rn(__fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y)));
            sh.kn[i + half] = __float2half_rn(__fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x)));
        }
        for (int d = tid; d < HD; d += ATT_THREADS) sh.vn[d] = __float2half_rn(__ldcg(v + d));
    }
    if (tid == 0 && !prefetched) {
        tc::fence_proxy_async_smem();
        att_issue<HD>(kv, x, 0, kt, vt, bar);
        if (x.ntiles > 1) att_issue<HD>(kv, x, 1, kt, vt, bar);
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
        const int b = t & 1;
        if (!tc::mbar_wait(&bar[b], uses[b] & 1)) {
            atomicCAS(a.err, 0, 1);
            sh.failed = 1;
        }
        uses[b] += 1;
        sync();
        if (sh.failed) return false;   // uniform after the group barrier
        __half* K = kt + b * PAGE * HD;
        __half* V = vt + b * PAGE * HD;
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
        sync();   // tile buffer b and sc are free again
        if (tid == 0 && t + 2 < x.ntiles) {
            tc::fence_proxy_async_smem();
            att_issue<HD>(kv, x, t + 2, kt, vt, bar);
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
    __threadfence();
    sync();
    if (tid == 0) {
        const int prev = atomicAdd(a.counters + m * a.nkv + g, 1);
        sh.is_last = (prev == x.nsplit - 1);
    }
    sync();
    if (!sh.is_last) return true;
    __threadfence();
    const int ns = x.nsplit;
    float* ml = reinterpret_cast<float*>(kt);   // [G][ns][2]: the K stages are free now
    for (int i = tid; i < G * ns; i += ATT_THREADS) {
        const int h = i / ns, ss = i % ns;
        const float2 v = __ldcg(reinterpret_cast<const float2*>(a.part_ml) + ((size_t)m * MAX_MERGE + ss) * a.nq +
                                g * G + h);
        ml[2 * i] = v.x;
        ml[2 * i + 1] = v.y;
    }
    sync();
    for (int h = warp; h < G; h += 4) {
        float mx = -INFINITY;
        for (int ss = lane; ss < ns; ss += 32) mx = fmaxf(mx, ml[2 * (h * ns + ss)]);
        mx = warp_max(mx);
        float den = 0.f;
        for (int ss = lane; ss < ns; ss += 32) {
            const float w = expf(ml[2 * (h * ns + ss)] - mx);
            sh.wts[h][ss] = w;
            den = fmaf(w, ml[2 * (h * ns + ss) + 1], den);
        }
        den = warp_sum(den);
        if (lane == 0) sh.inv_den[h] = 1.0f / den;
    }
    sync();
    for (int t = tid; t < G * PAIRS; t += ATT_THREADS) {
        const int h = t / PAIRS, d2 = t % PAIRS;
        const int qh = g * G + h;
        float2 num = make_float2(0.f, 0.f);
#pragma unroll 8
        for (int ss = 0; ss < ns; ++ss) {
            const float2 p = __ldcg(reinterpret_cast<const float2*>(
                                        a.part + (((size_t)m * MAX_MERGE + ss) * a.nq + qh) * HD) + d2);
            num.x = fmaf(sh.wts[h][ss], p.x, num.x);
            num.y = fmaf(sh.wts[h][ss], p.y, num.y);
        }
        reinterpret_cast<float2*>(out + (size_t)qh * HD)[d2] =
            make_float2(num.x * sh.inv_den[h], num.y * sh.inv_den[h]);
    }
    if (tid == 0) a.counters[m * a.nkv + g] = 0;   // ready for the next layer / launch
    sync();
    return true;
}

// ------------------------------------------------------------ kernel
template <int HD, int MB>
__global__ void __launch_bounds__(MT, 1) k_decode_mega(const MegaArgs a) {
    extern __shared__ __align__(1024) uint8_t dyn[];
    using AC = AttConst<HD>;
    __shared__ __align__(8) uint64_t full[MAX_STAGES], empty[MAX_STAGES];
    __shared__ __align__(8) uint64_t abar[AC::NG][2];
    __shared__ float red[2 * NCW];
    __shared__ float scl[2];
    __shared__ unsigned long long best[2];
    __shared__ Ctl ctl;
    const int tid = threadIdx.x, warp = tid >> 5;
    uint8_t* region = dyn;                         // activations | attention tiles + state
    uint8_t* ring = dyn + a.union_bytes;
    float* act = reinterpret_cast<float*>(region);

    if (tid == 0) {
        const unsigned long long per_launch = (unsigned long long)(5 * a.n_layers + 2) * gridDim.x;
        ctl.target = (unsigned long long)(*(volatile unsigned int*)a.epoch) * per_launch;
        ctl.aborted = 0;
        ctl.fail = 0;
        ctl.nbar = 0;
        trace_mark(a, 0);
        for (int i = 0; i < a.nstage; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < AC::NG; ++i) {
            tc::mbar_init(&abar[i][0], 1);
            tc::mbar_init(&abar[i][1], 1);
        }
        tc::mbar_fence_init();
    }
    if (tid < 2) best[tid] = 0ull;
    if (blockIdx.x == 0 && tid < MB) a.amax[tid] = 0ull;
    __syncthreads();

    if (warp == PRODUCER) {
        if ((tid & 31) == 0) producer(a, ring, full, empty, ctl);
        return;
    }

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
                v = __fmul_rn((float)reinterpret_cast<const int8_t*>(rp)[k], d);
            }
            a.X[t] = v;
        }
    }

    uint32_t seq = 0;                    // ring tiles consumed so far
    uint32_t uses[2] = {0, 0};           // completed phases of this group's attention barriers
    const int qw = a.nq * HD;
    const int grp = tid / ATT_THREADS, gtid = tid % ATT_THREADS;
    const int n_att = a.nsplit * a.nkv * MB;
    AttSh<HD>* ash = reinterpret_cast<AttSh<HD>*>(region + AC::NG * AC::GROUP_BYTES);
    __half* kt = reinterpret_cast<__half*>(region + (size_t)grp * AC::GROUP_BYTES);
    __half* vt = kt + 2 * PAGE * HD;

    for (int li = 0; li < a.n_layers; ++li) {
        const MegaLayer& L = a.layers[li];
        // 1. RMSNorm + QKV (+bias) -> raw q/k/v rows
        grid_sync(a, ctl);
        if (ctl.aborted) break;
        stage<MB>(a, a.X, L.attn_norm, a.H, act, red, scl);
        gemv_tiles<PH_QKV, MB>(a, li, ring, full, empty, act, seq, ctl, best);
        // 2. attention: the first pages of each group's first item are requested
        //    before the barrier (activations are dead: the region is free)
        cbar();
        const int it0 = blockIdx.x + grp * gridDim.x;
        AttItem x0;
        const bool pre = grp < AC::NG && it0 < n_att && att_item_geo(a, it0, x0);   // uniform in the group
        if (pre && gtid == 0) {
            tc::fence_proxy_async_smem();
            att_issue<HD>(L.kv, x0, 0, kt, vt, abar[grp]);
            if (x0.ntiles > 1) att_issue<HD>(L.kv, x0, 1, kt, vt, abar[grp]);
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
                if (!att_item<HD>(a, L.kv, x, gtid, kt, vt, ash[grp], abar[grp], uses, first && pre,
                                  GroupSync{2 + grp})) {
                    if (gtid == 0) raise_fail(a, ctl, 1);
                    break;
                }
            }
        }
        if (ctl.aborted) break;
        // 3. O-proj + residual
        grid_sync(a, ctl);
        if (ctl.aborted) break;
        stage<MB>(a, a.ATT, nullptr, qw, act, red, scl);
        gemv_tiles<PH_O, MB>(a, li, ring, full, empty, act, seq, ctl, best);
        // 4. RMSNorm + gate/up + SwiGLU
        grid_sync(a, ctl);
        if (ctl.aborted) break;
        stage<MB>(a, a.X, L.ffn_norm, a.H, act, red, scl);
        gemv_tiles<PH_GU, MB>(a, li, ring, full, empty, act, seq, ctl, best);
        // 5. down + residual
        grid_sync(a, ctl);
        if (ctl.aborted) break;
        stage<MB>(a, a.FA, nullptr, a.F, act, red, scl);
        gemv_tiles<PH_DOWN, MB>(a, li, ring, full, empty, act, seq, ctl, best);
    }
    // output norm + lm_head + argmax
    if (!ctl.aborted) {
        grid_sync(a, ctl);
        if (!ctl.aborted) {
            stage<MB>(a, a.X, a.out_norm, a.H, act, red, scl);
            gemv_tiles<PH_LM, MB>(a, 0, ring, full, empty, act, seq, ctl, best);
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
    const bool t_ok = (a.t_gu == 1 || a.t_gu == 2 || a.t_gu == 4);
    auto pow2_le8 = [](int t) { return t == 1 || t == 2 || t == 4 || t == 8; };
    if (a.M < 1 || a.M > 2 || a.nstage < NCW || a.nstage > MAX_STAGES || a.nstage % NCW || a.nsplit < 1 ||
        a.nsplit > MAX_MERGE ||
        !t_ok || !pow2_le8(a.t_qkv) || !pow2_le8(a.t_o) || !pow2_le8(a.t_down) || !pow2_le8(a.t_lm) ||
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
