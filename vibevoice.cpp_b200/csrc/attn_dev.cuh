// attn_dev.cuh -- one split-K flash-decode work item (split, kv head, row) for a
// group of 128 threads; used by the standalone decode-attention kernel and by
// the persistent decode-step kernel.  See attn_decode.cu for the algorithm.
#pragma once

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace vvq2 {
namespace ad {

constexpr int THREADS = 128;    // threads per work item
constexpr int MAXG = 8;         // query heads per KV head (7 for 0.5B/7B, 6 for 1.5B)
constexpr int TILE = KV_PAGE;   // keys per staged tile (one page)
constexpr int MAX_MERGE = 64;   // splits merged by the last CTA

struct __align__(16) Shared {   // qs is read as float4; arrays of Shared stay aligned
    float qs[MAXG][128];
    float sc[MAXG][TILE];
    float run_max[MAXG], run_sum[MAXG], alpha[MAXG];
    float wts[MAXG][MAX_MERGE];
    float inv_den[MAXG];
    __align__(8) uint64_t bar[2];
    int is_last, failed;
};

// dynamic shared memory per group: K and V, two stages each
__host__ __device__ constexpr int tile_smem_bytes(int hd) { return 4 * TILE * hd * 2; }

// Error word value of a row whose key count exceeds what the launch covers.
constexpr int ERR_ROW_TOO_LONG = 5;

// Keys row `rm` attends: min(pos + 1, kv_len), clamped to what the launch
// covers -- max_splits * split keys (the grid) and max_pages * 64 (the
// block-table row).  A clamped row records ERR_ROW_TOO_LONG in a.err (when
// `flag`), so the caller learns that its output covers only the first keys;
// nothing is read past the block-table row or written past the split slots.
__device__ __forceinline__ int key_limit(const AttnDecodeArgs& a, const RowMeta& rm, bool flag) {
    int lim = min(rm.pos + 1, rm.kvlen);
    const int cap = min(a.max_splits * a.split, a.kv.max_pages * TILE);
    if (lim > cap) {
        if (flag && a.err) atomicCAS(a.err, 0, ERR_ROW_TOO_LONG);
        lim = cap;
    }
    return lim;
}

// Initialise the two stage barriers of a group (one thread, once).
__device__ __forceinline__ void init_bars(Shared& sh) {
    tc::mbar_init(&sh.bar[0], 1);
    tc::mbar_init(&sh.bar[1], 1);
    tc::mbar_fence_init();
}

// One work item.  `tid` in [0, 128); `sync` synchronises exactly the 128
// threads of the group; `uses` counts completed phases of each stage barrier
// across items (identical in every thread of the group).  Returns false if a
// bounded wait timed out (error recorded in a.err).
template <int HD, class Sync>
__device__ bool item(const AttnDecodeArgs& a, int s, int g, int m, int tid, __half* kt, __half* vt, Shared& sh,
                     uint32_t (&uses)[2], Sync sync) {
    constexpr int NCH = HD / 8;                // 16-byte chunks per K row
    constexpr int TILE_BYTES = TILE * HD * 2;
    const int lane = tid & 31, warp = tid >> 5;
    const int G = a.nq / a.nkv;
    const RowMeta rm = a.meta[m];
    const int lim = key_limit(a, rm, s == 0 && tid == 0);
    if (lim <= 0) {
        // no keys for this row here (another rank holds its part of the
        // sequence): zeros and LSE -inf, written once (split 0)
        if (s == 0) {
            for (int t = tid; t < G * HD; t += THREADS) {
                const size_t off = (size_t)m * a.nq * HD + (size_t)g * G * HD + t;
                if (a.out_h) a.out_h[off] = __float2half_rn(0.f);
                else a.out[off] = 0.f;
            }
            if (a.lse && tid < G) a.lse[(size_t)m * a.nq + g * G + tid] = -INFINITY;
        }
        return true;
    }
    const int nsplit = (lim + a.split - 1) / a.split;
    if (s >= nsplit) return true;
    const int j0 = s * a.split, j1 = min(lim, j0 + a.split);
    const int ntiles = (j1 - j0 + TILE - 1) / TILE;

    if (tid == 0) sh.failed = 0;
    for (int t = tid; t < G * HD; t += THREADS) {
        const int h = t / HD, d = t % HD;
        // L2 read: within the persistent decode kernel another CTA wrote Q
        const float qv = __ldcg(a.q + (size_t)m * a.nq * HD + (size_t)(g * G + h) * HD + d);
        sh.qs[h][d] = __half2float(__float2half_rn(qv));   // ggml FA converts Q to the K type
    }
    if (tid < MAXG) {
        sh.run_max[tid] = -INFINITY;
        sh.run_sum[tid] = 0.f;
    }
    sync();

    auto page_src = [&](const __half* pool, int tile) {
        const int page = __ldg(a.kv.block_table + (size_t)rm.seq * a.kv.max_pages + (j0 + tile * TILE) / TILE);
        return pool + ((size_t)page * a.kv.n_kv + g) * TILE * HD;
    };
    auto issue = [&](int tile) {
        const int b = tile & 1;
        tc::mbar_arrive_expect_tx(&sh.bar[b], 2 * TILE_BYTES);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                tc::smem_u32(kt + b * TILE * HD)),
            "l"(page_src(a.kv.k, tile)), "r"(TILE_BYTES), "r"(tc::smem_u32(&sh.bar[b]))
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                tc::smem_u32(vt + b * TILE * HD)),
            "l"(page_src(a.kv.v, tile)), "r"(TILE_BYTES), "r"(tc::smem_u32(&sh.bar[b]))
            : "memory");
    };
    if (tid == 0) {
        tc::fence_proxy_async_smem();   // previous item's generic reads of the stages are done
        issue(0);
        if (ntiles > 1) issue(1);
    }

    // P.V ownership: thread -> column pair dp and heads hs, hs + HSUB, ...
    constexpr int PAIRS = HD / 2;
    constexpr int HSUB = THREADS / PAIRS;   // 8 (hd 32), 4 (hd 64), 2 (hd 128)
    constexpr int HPER = (MAXG + HSUB - 1) / HSUB;
    const int dp = tid % PAIRS, hs = tid / PAIRS;
    float2 o[HPER];
#pragma unroll
    for (int k = 0; k < HPER; ++k) o[k] = make_float2(0.f, 0.f);

    // scores ownership: key kk = tid % TILE, heads hh, hh + 2, ...
    const int kk = tid % TILE, hh = tid / TILE;
    const int rot = (HD >= 64) ? (kk % NCH) : ((kk >> 1) % NCH);

    for (int t = 0; t < ntiles; ++t) {
        const int b = t & 1;
        if (!tc::mbar_wait(&sh.bar[b], uses[b] & 1)) {
            if (a.err) atomicExch(a.err, 1);
            sh.failed = 1;
        }
        uses[b] += 1;
        sync();
        if (sh.failed) return false;   // uniform after the barrier
        const __half* K = kt + b * TILE * HD;
        const __half* V = vt + b * TILE * HD;
        const int nk = min(TILE, j1 - (j0 + t * TILE));
        // ---- scores for this tile
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
        // ---- per-head tile max and the running-max update
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
        // ---- probabilities
        for (int i = tid; i < G * TILE; i += THREADS) {
            const int h = i / TILE, k = i % TILE;
            sh.sc[h][k] = expf(sh.sc[h][k] - sh.run_max[h]);   // masked keys: exp(-inf) = 0
        }
        sync();
        for (int h = warp; h < G; h += 4) {
            const float sm = warp_sum(sh.sc[h][lane] + sh.sc[h][lane + 32]);
            if (lane == 0) sh.run_sum[h] = sh.run_sum[h] * sh.alpha[h] + sm;
        }
        // ---- O = O*alpha + P.V
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
        if (tid == 0 && t + 2 < ntiles) {
            tc::fence_proxy_async_smem();
            issue(t + 2);
        }
    }

    if (nsplit == 1) {
        if (a.lse && tid < G) a.lse[(size_t)m * a.nq + g * G + tid] = sh.run_max[tid] + logf(sh.run_sum[tid]);
#pragma unroll
        for (int k = 0; k < HPER; ++k) {
            const int h = hs + k * HSUB;
            if (h < G) {
                const float inv = 1.0f / sh.run_sum[h];
                const size_t off = (size_t)m * a.nq * HD + (size_t)(g * G + h) * HD;
                if (a.out_h)
                    reinterpret_cast<__half2*>(a.out_h + off)[dp] = __floats2half2_rn(o[k].x * inv, o[k].y * inv);
                else
                    reinterpret_cast<float2*>(a.out + off)[dp] = make_float2(o[k].x * inv, o[k].y * inv);
            }
        }
        sync();   // sh is reused by the next item
        return true;
    }
    // ---- partials, then the last arriving item merges (log-sum-exp)
    const size_t pbase = ((size_t)m * a.max_splits + s) * a.nq;
#pragma unroll
    for (int k = 0; k < HPER; ++k) {
        const int h = hs + k * HSUB;
        if (h < G) reinterpret_cast<float2*>(a.part + (pbase + g * G + h) * HD)[dp] = o[k];
    }
    if (tid < G) {
        a.part_ml[(pbase + g * G + tid) * 2 + 0] = sh.run_max[tid];
        a.part_ml[(pbase + g * G + tid) * 2 + 1] = sh.run_sum[tid];
    }
    if (a.defer_merge) {   // many splits: k_attn_merge combines them after this launch
        sync();            // sh is reused by the next item
        return true;
    }
    __threadfence();
    sync();
    if (tid == 0) {
        const int prev = atomicAdd(a.counters + m * a.nkv + g, 1);
        sh.is_last = (prev == nsplit - 1);
    }
    sync();
    if (!sh.is_last) return true;
    __threadfence();
    // merge: weights w_s = exp(m_s - max_s m_s) per head, staged in shared
    // memory with one parallel round of loads, then the partial O's summed
    // with independent (batched) loads
    float* ml_s = reinterpret_cast<float*>(kt);   // reuse the K stage: [G][nsplit][2]
    for (int i = tid; i < G * nsplit; i += THREADS) {
        const int h = i / nsplit, ss = i % nsplit;
        const float2 v = __ldcg(reinterpret_cast<const float2*>(a.part_ml) +
                                ((size_t)m * a.max_splits + ss) * a.nq + g * G + h);
        ml_s[2 * i] = v.x;
        ml_s[2 * i + 1] = v.y;
    }
    sync();
    for (int h = warp; h < G; h += 4) {
        float mx = -INFINITY;
        for (int ss = lane; ss < nsplit; ss += 32) mx = fmaxf(mx, ml_s[2 * (h * nsplit + ss)]);
        mx = warp_max(mx);
        float den = 0.f;
        for (int ss = lane; ss < nsplit; ss += 32) {
            const float w = expf(ml_s[2 * (h * nsplit + ss)] - mx);
            sh.wts[h][ss] = w;
            den = fmaf(w, ml_s[2 * (h * nsplit + ss) + 1], den);
        }
        den = warp_sum(den);
        if (lane == 0) {
            sh.inv_den[h] = 1.0f / den;
            if (a.lse) a.lse[(size_t)m * a.nq + g * G + h] = mx + logf(den);
        }
    }
    sync();
    for (int t = tid; t < G * PAIRS; t += THREADS) {
        const int h = t / PAIRS, d2 = t % PAIRS;
        const int qh = g * G + h;
        float2 num = make_float2(0.f, 0.f);
#pragma unroll 8
        for (int ss = 0; ss < nsplit; ++ss) {
            const float2 p = __ldcg(reinterpret_cast<const float2*>(
                                        a.part + (((size_t)m * a.max_splits + ss) * a.nq + qh) * HD) + d2);
            num.x = fmaf(sh.wts[h][ss], p.x, num.x);
            num.y = fmaf(sh.wts[h][ss], p.y, num.y);
        }
        const size_t off = (size_t)m * a.nq * HD + (size_t)qh * HD;
        if (a.out_h)
            reinterpret_cast<__half2*>(a.out_h + off)[d2] = __floats2half2_rn(num.x * sh.inv_den[h], num.y * sh.inv_den[h]);
        else
            reinterpret_cast<float2*>(a.out + off)[d2] = make_float2(num.x * sh.inv_den[h], num.y * sh.inv_den[h]);
    }
    if (tid == 0) a.counters[m * a.nkv + g] = 0;   // ready for the next launch
    sync();   // sh and the K stage are reused by the next item
    return true;
}

}  // namespace ad
}  // namespace vvq2
