// attn_decode.cu -- split-K flash-decode over the f16 paged KV cache (sm_100a).
//
// Replaces ggml_flash_attn_ext (src/qwen2.cpp:327-335) for decode-sized query
// counts: softmax(Q K^T * 1/sqrt(hd) + causal mask) V with GQA (query head h
// reads KV head h / (nq/nkv), ggml's broadcast) and F32 accumulation
// (ggml_flash_attn_ext_set_prec(GGML_PREC_F32), src/qwen2.cpp:334).  The
// causal mask (key j masked iff j > pos, src/vibevoice_tts.cpp:432-441) is
// evaluated from the row's position; nothing is materialised.
//
// Grid (split, kv_head, row).  Each CTA scores one contiguous key range for
// the whole GQA group (Q is loaded once, rounded to f16 as ggml does), keeps
// an exact max/sum for its range, and writes an unnormalised partial O.  The
// last CTA of a (row, kv_head) to finish -- detected with a device-scope
// counter -- merges the partials with the log-sum-exp rule and writes the
// normalised output, so there is no second launch.
#include "common.cuh"
#include "kernels.h"

namespace vvq2 {

namespace {

constexpr int AD_THREADS = 128;
constexpr int AD_MAXG = 8;          // query heads per KV head (7 for 0.5B/7B, 6 for 1.5B)
constexpr int AD_MAX_SPLIT = 512;   // keys per CTA

template <int HD>
__global__ void __launch_bounds__(AD_THREADS) k_attn_decode(const AttnDecodeArgs a) {
    const int s = blockIdx.x, g = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.nq / a.nkv;
    const RowMeta rm = a.meta[m];
    const int lim = min(rm.pos + 1, rm.kvlen);
    const int nsplit = (lim + a.split - 1) / a.split;
    if (s >= nsplit) return;
    const int j0 = s * a.split, j1 = min(lim, j0 + a.split), nj = j1 - j0;

    __shared__ __align__(16) float qs[AD_MAXG][HD];
    __shared__ float sc[AD_MAXG][AD_MAX_SPLIT];
    __shared__ float red[AD_MAXG][AD_THREADS / 32];
    __shared__ float hmax[AD_MAXG], hsum[AD_MAXG];
    __shared__ int is_last;

    // Q of the group, rounded to f16 (ggml FA converts Q to the K type)
    for (int t = tid; t < G * HD; t += AD_THREADS) {
        const int h = t / HD, d = t % HD;
        const float qv = a.q[(size_t)m * a.nq * HD + (size_t)(g * G + h) * HD + d];
        qs[h][d] = __half2float(__float2half_rn(qv));
    }
    __syncthreads();

    // ---- scores: one key per thread per pass
    float lmax[AD_MAXG];
#pragma unroll
    for (int h = 0; h < AD_MAXG; ++h) lmax[h] = -INFINITY;
    for (int jj = tid; jj < nj; jj += AD_THREADS) {
        const int j = j0 + jj;
        const __half* kp = a.kv.k + kv_offset(a.kv, rm.seq, j, g);
        float acc[AD_MAXG];
#pragma unroll
        for (int h = 0; h < AD_MAXG; ++h) acc[h] = 0.0f;
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4*>(kp) + c);
            const __half2* hp = reinterpret_cast<const __half2*>(&raw);
            float kf[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(hp[e]);
                kf[2 * e] = f.x;
                kf[2 * e + 1] = f.y;
            }
#pragma unroll
            for (int h = 0; h < AD_MAXG; ++h) {
                if (h < G) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[h] = fmaf(qs[h][c * 8 + e], kf[e], acc[h]);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < AD_MAXG; ++h) {
            if (h < G) {
                const float v = acc[h] * a.scale;
                sc[h][jj] = v;
                lmax[h] = fmaxf(lmax[h], v);
            }
        }
    }
#pragma unroll
    for (int h = 0; h < AD_MAXG; ++h) {
        if (h < G) {
            const float w = warp_max(lmax[h]);
            if (lane == 0) red[h][warp] = w;
        }
    }
    __syncthreads();
    if (tid < G) {
        float mx = red[tid][0];
        for (int w = 1; w < AD_THREADS / 32; ++w) mx = fmaxf(mx, red[tid][w]);
        hmax[tid] = mx;
    }
    __syncthreads();
    float lsum[AD_MAXG];
#pragma unroll
    for (int h = 0; h < AD_MAXG; ++h) lsum[h] = 0.0f;
    for (int jj = tid; jj < nj; jj += AD_THREADS) {
#pragma unroll
        for (int h = 0; h < AD_MAXG; ++h) {
            if (h < G) {
                const float p = expf(sc[h][jj] - hmax[h]);
                sc[h][jj] = p;
                lsum[h] += p;
            }
        }
    }
#pragma unroll
    for (int h = 0; h < AD_MAXG; ++h) {
        if (h < G) {
            const float w = warp_sum(lsum[h]);
            if (lane == 0) red[h][warp] = w;
        }
    }
    __syncthreads();
    if (tid < G) {
        float sm = 0.0f;
        for (int w = 0; w < AD_THREADS / 32; ++w) sm += red[tid][w];
        hsum[tid] = sm;
    }
    // ---- P.V: thread owns a column pair and a subset of the group's heads
    constexpr int PAIRS = HD / 2;
    constexpr int HSUB = AD_THREADS / PAIRS;        // 4 (hd 64) or 2 (hd 128)
    constexpr int HPER = (AD_MAXG + HSUB - 1) / HSUB;
    const int dp = tid % PAIRS, hs = tid / PAIRS;
    float2 o[HPER];
#pragma unroll
    for (int k = 0; k < HPER; ++k) o[k] = make_float2(0.f, 0.f);
    __syncthreads();
    for (int jj = 0; jj < nj; ++jj) {
        const __half2 vv = *(reinterpret_cast<const __half2*>(a.kv.v + kv_offset(a.kv, rm.seq, j0 + jj, g)) + dp);
        const float2 v = __half22float2(vv);
#pragma unroll
        for (int k = 0; k < HPER; ++k) {
            const int h = hs + k * HSUB;
            if (h < G) {
                const float p = sc[h][jj];
                o[k].x = fmaf(p, v.x, o[k].x);
                o[k].y = fmaf(p, v.y, o[k].y);
            }
        }
    }
    if (nsplit == 1) {
#pragma unroll
        for (int k = 0; k < HPER; ++k) {
            const int h = hs + k * HSUB;
            if (h < G) {
                const float inv = 1.0f / hsum[h];
                float2* dst = reinterpret_cast<float2*>(a.out + (size_t)m * a.nq * HD + (size_t)(g * G + h) * HD) + dp;
                *dst = make_float2(o[k].x * inv, o[k].y * inv);
            }
        }
        return;
    }
    // ---- partials, then the last CTA merges (log-sum-exp)
    const size_t pbase = ((size_t)m * a.max_splits + s) * a.nq;
#pragma unroll
    for (int k = 0; k < HPER; ++k) {
        const int h = hs + k * HSUB;
        if (h < G) {
            float2* dst = reinterpret_cast<float2*>(a.part + (pbase + g * G + h) * HD) + dp;
            *dst = o[k];
        }
    }
    if (tid < G) {
        a.part_ml[(pbase + g * G + tid) * 2 + 0] = hmax[tid];
        a.part_ml[(pbase + g * G + tid) * 2 + 1] = hsum[tid];
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
    for (int t = tid; t < G * HD; t += AD_THREADS) {
        const int h = t / HD, d = t % HD;
        const int qh = g * G + h;
        float mx = -INFINITY;
        for (int ss = 0; ss < nsplit; ++ss)
            mx = fmaxf(mx, __ldcg(a.part_ml + (((size_t)m * a.max_splits + ss) * a.nq + qh) * 2));
        float num = 0.f, den = 0.f;
        for (int ss = 0; ss < nsplit; ++ss) {
            const size_t b = ((size_t)m * a.max_splits + ss) * a.nq + qh;
            const float w = expf(__ldcg(a.part_ml + b * 2) - mx);
            num = fmaf(w, __ldcg(a.part + b * HD + d), num);
            den = fmaf(w, __ldcg(a.part_ml + b * 2 + 1), den);
        }
        a.out[(size_t)m * a.nq * HD + (size_t)qh * HD + d] = num / den;
    }
    if (tid == 0) a.counters[m * a.nkv + g] = 0;   // ready for the next launch
}

}  // namespace

cudaError_t attn_decode_launch(const AttnDecodeArgs& a, cudaStream_t st) {
    if (a.nq % a.nkv || a.nq / a.nkv > AD_MAXG || a.split < 1 || a.split > AD_MAX_SPLIT)
        return cudaErrorInvalidValue;
    dim3 grid(a.max_splits, a.nkv, a.M);
    if (a.hd == 64) k_attn_decode<64><<<grid, AD_THREADS, 0, st>>>(a);
    else if (a.hd == 128) k_attn_decode<128><<<grid, AD_THREADS, 0, st>>>(a);
    else return cudaErrorInvalidValue;
    note_launch();
    return cudaGetLastError();
}

}  // namespace vvq2
