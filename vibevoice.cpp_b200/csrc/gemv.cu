// gemv.cu -- decode-time (<= 8 activation rows) fused dequant GEMV on sm_100a.
//
// One kernel family covers every linear of the Qwen2 layer at decode time
// (src/qwen2.cpp:19-26,274-276,349 and the FFN at :33-40), the lm_head
// (src/vibevoice_asr.cpp:285-311) and its greedy argmax (:702-706).
//
// Prologue (per CTA, from L2): optional RMSNorm (src/rms_norm.hpp:11-17) of
// the f32 activation rows, then quantization to the weight's ggml vec_dot
// type -- Q8_0 (per 32, f16 scale) for Q8_0 weights, Q8_K (per 256, f32 scale,
// int16 bsums) for Q5_K/Q6_K, f16 for F16 and f32 for F32 -- into shared
// memory.  This reproduces the integer dot products ggml's CPU backend runs
// (ggml_vec_dot_*_q8_*), so results differ from the reference only in float
// summation order.
//
// Main loop: each warp owns NR weight rows; lanes stride over 32-element
// blocks, reading 16-byte vectors of the repacked weights once from HBM and
// doing dp4a against the shared-memory activations for all M rows.
//
// Epilogues: QKV (+bias, NEOX RoPE on Q/K, Q to a buffer, K/V appended to the
// f16 paged cache), residual add, SwiGLU, plain store, and argmax.
#include "common.cuh"
#include "kernels.h"

namespace vvq2 {

namespace {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr size_t GEMV_SMEM_MAX = 200 * 1024;

// activation-quantization kind derived from the weight type
__host__ __device__ constexpr int act_kind(int wt) {
    return wt == W_Q8_0 ? 0 : (wt == W_Q5_K || wt == W_Q6_K) ? 1 : 2;  // 0 q8_0, 1 q8_K, 2 float
}

// shared-memory carve-up for M rows of K activations
struct ActSmem {
    int8_t* q;      // [M][K]
    float* d;       // [M][K/32] (q8_0) or [M][K/256] (q8_K)
    int16_t* bs;    // [M][K/16] (q8_K)
    float* f;       // [M][K] (float kind)
};

__host__ __device__ inline size_t act_smem_bytes(int wt, int M, int K) {
    const int kind = act_kind(wt);
    if (kind == 0) return (size_t)M * K + (size_t)M * (K / 32) * 4 + 64;
    if (kind == 1) return (size_t)M * K + (size_t)M * (K / 256) * 4 + (size_t)M * (K / 16) * 2 + 64;
    return (size_t)M * K * 4 + 64;
}

__device__ inline ActSmem carve(uint8_t* base, int wt, int M, int K) {
    ActSmem s{};
    const int kind = act_kind(wt);
    if (kind == 2) {
        s.f = reinterpret_cast<float*>(base);
        return s;
    }
    s.q = reinterpret_cast<int8_t*>(base);
    uint8_t* p = base + (size_t)M * K;
    s.d = reinterpret_cast<float*>(p);
    p += (size_t)M * (K / (kind == 0 ? 32 : 256)) * 4;
    s.bs = reinterpret_cast<int16_t*>(p);
    return s;
}

// Prologue: optional RMSNorm then quantization of M activation rows into smem.
template <int WT>
__device__ void load_activations(const GemvArgs& a, ActSmem s, float* red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = a.M, K = a.K;
    __shared__ float row_scale[GEMV_MAX_M];
    if (a.norm_w) {
        // ggml_compute_forward_rms_norm_f32: mean of squares, scale = 1/sqrtf(mean + eps)
        float ss[GEMV_MAX_M];
#pragma unroll
        for (int m = 0; m < GEMV_MAX_M; ++m) ss[m] = 0.0f;
        for (int k = tid; k < K; k += GEMV_THREADS) {
#pragma unroll
            for (int m = 0; m < GEMV_MAX_M; ++m)
                if (m < M) {
                    const float v = a.x[(size_t)m * a.x_stride + k];
                    ss[m] = __fadd_rn(ss[m], __fmul_rn(v, v));
                }
        }
#pragma unroll
        for (int m = 0; m < GEMV_MAX_M; ++m) {
            if (m < M) {
                const float w = warp_sum(ss[m]);
                if (lane == 0) red[m * GEMV_WARPS + warp] = w;
            }
        }
        __syncthreads();
        if (tid < M) {
            float t = 0.0f;
            for (int w = 0; w < GEMV_WARPS; ++w) t = __fadd_rn(t, red[tid * GEMV_WARPS + w]);
            const float mean = __fdiv_rn(t, (float)K);
            row_scale[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        }
        __syncthreads();
    }
    auto act = [&](int m, int k) -> float {
        const float v = a.x[(size_t)m * a.x_stride + k];
        if (!a.norm_w) return v;
        return __fmul_rn(__fmul_rn(v, row_scale[m]), a.norm_w[k]);   // (x*scale)*w
    };
    constexpr int kind = act_kind(WT);
    if constexpr (kind == 0) {
        // quantize_row_q8_0_ref: 8 lanes per 32-block, 4 elements each
        const int nb = K / 32;
        // warp-uniform trip count: every lane reaches the shuffles
        for (int t0 = warp * 4; t0 < M * nb; t0 += GEMV_WARPS * 4) {
            const int t = t0 + (lane >> 3);
            const bool on = t < M * nb;
            const int m = on ? t / nb : 0, b = on ? t % nb : 0, sub = lane & 7;
            float v[4], amax = 0.0f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                v[e] = on ? act(m, b * 32 + sub * 4 + e) : 0.0f;
                amax = fmaxf(amax, fabsf(v[e]));
            }
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o, 8));
            if (!on) continue;
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            char4 q;
            q.x = (signed char)roundf(__fmul_rn(v[0], id));
            q.y = (signed char)roundf(__fmul_rn(v[1], id));
            q.z = (signed char)roundf(__fmul_rn(v[2], id));
            q.w = (signed char)roundf(__fmul_rn(v[3], id));
            *reinterpret_cast<char4*>(s.q + (size_t)m * K + b * 32 + sub * 4) = q;
            if (sub == 0) s.d[m * nb + b] = __half2float(__float2half_rn(d));
        }
    } else if constexpr (kind == 1) {
        // quantize_row_q8_K_ref: one warp per 256-block, 8 elements per lane
        const int nb = K / 256;
        for (int t = warp; t < M * nb; t += GEMV_WARPS) {
            const int m = t / nb, b = t % nb;
            float v[8];
            float ax = 0.0f, mx = 0.0f;
            int ai = 0x7fffffff;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int k = b * 256 + lane * 8 + e;
                v[e] = act(m, k);
                const float av = fabsf(v[e]);
                if (av > ax) { ax = av; mx = v[e]; ai = k; }
            }
            // first index of the largest magnitude (strict > in ggml)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ax2 = __shfl_xor_sync(0xffffffffu, ax, o);
                const float mx2 = __shfl_xor_sync(0xffffffffu, mx, o);
                const int ai2 = __shfl_xor_sync(0xffffffffu, ai, o);
                if (ax2 > ax || (ax2 == ax && ai2 < ai)) { ax = ax2; mx = mx2; ai = ai2; }
            }
            int8_t* qd = s.q + (size_t)m * K + b * 256 + lane * 8;
            if (ax == 0.0f) {
#pragma unroll
                for (int e = 0; e < 8; ++e) qd[e] = 0;
                if (lane < 16) s.bs[m * (K / 16) + b * 16 + lane] = 0;
                if (lane == 0) s.d[m * nb + b] = 0.0f;
                continue;
            }
            const float iscale = __fdiv_rn(-127.0f, mx);
            int sum = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                int q = __float2int_rn(__fmul_rn(iscale, v[e]));
                q = q < 127 ? q : 127;
                qd[e] = (int8_t)q;
                sum += q;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            if ((lane & 1) == 0) s.bs[m * (K / 16) + b * 16 + lane / 2] = (int16_t)sum;
            if (lane == 0) s.d[m * nb + b] = __fdiv_rn(1.0f, iscale);
        }
    } else {
        for (int t = tid; t < M * K; t += GEMV_THREADS) {
            const int m = t / K, k = t % K;
            const float v = act(m, k);
            s.f[t] = (WT == W_F16) ? __half2float(__float2half_rn(v)) : v;
        }
    }
    __syncthreads();
}

__device__ __forceinline__ int dot8(const uint4& w0, const uint4& w1, const uint4& a0, const uint4& a1) {
    int s = 0;
    s = __dp4a((int)w0.x, (int)a0.x, s);
    s = __dp4a((int)w0.y, (int)a0.y, s);
    s = __dp4a((int)w0.z, (int)a0.z, s);
    s = __dp4a((int)w0.w, (int)a0.w, s);
    s = __dp4a((int)w1.x, (int)a1.x, s);
    s = __dp4a((int)w1.y, (int)a1.y, s);
    s = __dp4a((int)w1.z, (int)a1.z, s);
    s = __dp4a((int)w1.w, (int)a1.w, s);
    return s;
}

// Row r of a unit: which tensor and which row.
template <int EPI, int NR>
__device__ __forceinline__ void unit_rows(const GemvArgs& a, int u, int* row, int* which) {
    if constexpr (EPI == EPI_QKV) {
        const int half = a.hd / 2;
        const int h = u / half, i = u % half;
        row[0] = h * a.hd + i;
        row[1] = row[0] + half;
        which[0] = which[1] = 0;
    } else if constexpr (EPI == EPI_SWIGLU) {
        row[0] = u;
        row[1] = u;
        which[0] = 0;
        which[1] = 1;
    } else {
#pragma unroll
        for (int j = 0; j < NR; ++j) {
            row[j] = u * NR + j;
            which[j] = 0;
        }
    }
}

template <int WT, int NR, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float red[GEMV_MAX_M * GEMV_WARPS];
    __shared__ unsigned long long best[GEMV_MAX_M];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int M = a.M, K = a.K;
    ActSmem s = carve(smem, WT, M, K);
    if (EPI == EPI_ARGMAX && threadIdx.x < GEMV_MAX_M) best[threadIdx.x] = 0ull;
    load_activations<WT>(a, s, red);

    const int u = blockIdx.x * GEMV_WARPS + warp;
    float acc[NR][GEMV_MAX_M];
#pragma unroll
    for (int j = 0; j < NR; ++j)
#pragma unroll
        for (int m = 0; m < GEMV_MAX_M; ++m) acc[j][m] = 0.0f;

    int row[NR], which[NR];
    bool valid = u < a.n_units;
    if (valid) {
        unit_rows<EPI, NR>(a, u, row, which);
#pragma unroll
        for (int j = 0; j < NR; ++j)
            if (row[j] >= (which[j] ? a.w1.rows : a.w0.rows)) row[j] = -1;
    }
    if (valid) {
        if constexpr (WT == W_Q8_0) {
            const int nb = K / 32;
#pragma unroll 2
            for (int b = lane; b < nb; b += 32) {
                uint4 wq0[NR], wq1[NR];
                float wd[NR];
#pragma unroll
                for (int j = 0; j < NR; ++j) {
                    if (row[j] < 0) { wq0[j] = wq1[j] = make_uint4(0, 0, 0, 0); wd[j] = 0.0f; continue; }
                    const DevW& W = which[j] ? a.w1 : a.w0;
                    const uint4* p = reinterpret_cast<const uint4*>(W.q + (size_t)row[j] * W.row_stride + b * 32);
                    wq0[j] = __ldg(p);
                    wq1[j] = __ldg(p + 1);
                    wd[j] = __half2float(W.d[(size_t)row[j] * nb + b]);
                }
#pragma unroll
                for (int m = 0; m < GEMV_MAX_M; ++m) {
                    if (m >= M) break;
                    const uint4* ap = reinterpret_cast<const uint4*>(s.q + (size_t)m * K + b * 32);
                    const uint4 a0 = ap[0], a1 = ap[1];
                    const float da = s.d[m * nb + b];
#pragma unroll
                    for (int j = 0; j < NR; ++j) {
                        const int si = dot8(wq0[j], wq1[j], a0, a1);
                        acc[j][m] = __fadd_rn(acc[j][m], __fmul_rn((float)si, __fmul_rn(wd[j], da)));
                    }
                }
            }
        } else if constexpr (WT == W_Q5_K) {
            const int nsb = K / 256;
            // warp-uniform trip count; 8-lane groups are all-on or all-off
            for (int t0 = 0; t0 < nsb * 8; t0 += 32) {
                const int t = t0 + lane;
                const bool on = t < nsb * 8;
                const int sb = on ? t >> 3 : 0, sub = t & 7;
                uint32_t qw[NR][8];
                int sc[NR], mn[NR];
                float dd[NR], dm[NR];
#pragma unroll
                for (int j = 0; j < NR; ++j) {
                    const DevW& W = which[j] ? a.w1 : a.w0;
                    if (row[j] < 0 || !on) {
#pragma unroll
                        for (int w = 0; w < 8; ++w) qw[j][w] = 0;
                        sc[j] = mn[j] = 0; dd[j] = dm[j] = 0.0f;
                        continue;
                    }
                    const uint8_t* blk = W.q + (size_t)row[j] * W.row_stride + (size_t)sb * Q5K_BYTES;
                    const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(blk));        // d, dmin, scales[12]
                    const uint4* qh4 = reinterpret_cast<const uint4*>(blk + 16);
                    const uint4* qs4 = reinterpret_cast<const uint4*>(blk + 48 + 32 * (sub >> 1));
                    const uint4 h0 = __ldg(qh4), h1 = __ldg(qh4 + 1), s0 = __ldg(qs4), s1 = __ldg(qs4 + 1);
                    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                    const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                    const int shift = 4 * (sub & 1);
#pragma unroll
                    for (int w = 0; w < 8; ++w)
                        qw[j][w] = ((sw[w] >> shift) & 0x0F0F0F0Fu) | (((hw[w] >> sub) & 0x01010101u) << 4);
                    const uint8_t* scb = reinterpret_cast<const uint8_t*>(&hdr) + 4;
                    if (sub < 4) {
                        sc[j] = scb[sub] & 63;
                        mn[j] = scb[sub + 4] & 63;
                    } else {
                        sc[j] = (scb[sub + 4] & 0xF) | ((scb[sub - 4] >> 6) << 4);
                        mn[j] = (scb[sub + 4] >> 4) | ((scb[sub] >> 6) << 4);
                    }
                    const __half2 dh = *reinterpret_cast<const __half2*>(&hdr.x);
                    dd[j] = __low2float(dh);
                    dm[j] = __high2float(dh);
                }
#pragma unroll
                for (int m = 0; m < GEMV_MAX_M; ++m) {
                    if (m >= M) break;
                    const uint4* ap = reinterpret_cast<const uint4*>(s.q + (size_t)m * K + sb * 256 + sub * 32);
                    const uint4 a0 = ap[0], a1 = ap[1];   // sb = 0 when off: in bounds, result discarded
                    const float da = on ? s.d[m * nsb + sb] : 0.0f;
                    const int bsum = (int)s.bs[m * (K / 16) + sb * 16 + 2 * sub] +
                                     (int)s.bs[m * (K / 16) + sb * 16 + 2 * sub + 1];
#pragma unroll
                    for (int j = 0; j < NR; ++j) {
                        const uint4 w0 = make_uint4(qw[j][0], qw[j][1], qw[j][2], qw[j][3]);
                        const uint4 w1 = make_uint4(qw[j][4], qw[j][5], qw[j][6], qw[j][7]);
                        int is = sc[j] * dot8(w0, w1, a0, a1);
                        int ms = mn[j] * bsum;
                        // exact integer sums over the 8 sub-blocks of the super-block
#pragma unroll
                        for (int o = 1; o < 8; o <<= 1) {
                            is += __shfl_xor_sync(0xffffffffu, is, o, 8);
                            ms += __shfl_xor_sync(0xffffffffu, ms, o, 8);
                        }
                        if (sub == 0) {
                            const float d = __fmul_rn(dd[j], da), dmin = __fmul_rn(dm[j], da);
                            acc[j][m] = __fadd_rn(acc[j][m], __fmul_rn(d, (float)is));
                            acc[j][m] = __fsub_rn(acc[j][m], __fmul_rn(dmin, (float)ms));
                        }
                    }
                }
            }
        } else if constexpr (WT == W_Q6_K) {
            const int nsb = K / 256;
            for (int t0 = 0; t0 < nsb * 8; t0 += 32) {
                const int t = t0 + lane;
                const bool on = t < nsb * 8;
                const int sb = on ? t >> 3 : 0, L = t & 7, hf = L >> 2, kq = L & 3;
                uint32_t qw[NR][8];
                int sc0[NR], sc1[NR];
                float dd[NR];
#pragma unroll
                for (int j = 0; j < NR; ++j) {
                    const DevW& W = which[j] ? a.w1 : a.w0;
                    if (row[j] < 0 || !on) {
#pragma unroll
                        for (int w = 0; w < 8; ++w) qw[j][w] = 0x20202020u;
                        sc0[j] = sc1[j] = 0; dd[j] = 0.0f;
                        continue;
                    }
                    const uint8_t* blk = W.q + (size_t)row[j] * W.row_stride + (size_t)sb * Q6K_PACKED;
                    const uint4* ql4 = reinterpret_cast<const uint4*>(blk + hf * 64 + (kq & 1) * 32);
                    const uint4* qh4 = reinterpret_cast<const uint4*>(blk + 128 + hf * 32);
                    const uint4 l0 = __ldg(ql4), l1 = __ldg(ql4 + 1), h0 = __ldg(qh4), h1 = __ldg(qh4 + 1);
                    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
                    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                    const int ns = (kq >> 1) * 4;
#pragma unroll
                    for (int w = 0; w < 8; ++w)
                        qw[j][w] = ((lw[w] >> ns) & 0x0F0F0F0Fu) | (((hw[w] >> (2 * kq)) & 0x03030303u) << 4);
                    const int8_t* scl = reinterpret_cast<const int8_t*>(blk + 192);
                    sc0[j] = scl[2 * L];
                    sc1[j] = scl[2 * L + 1];
                    dd[j] = __half2float(W.d[(size_t)row[j] * nsb + sb]);
                }
#pragma unroll
                for (int m = 0; m < GEMV_MAX_M; ++m) {
                    if (m >= M) break;
                    const uint4* ap = reinterpret_cast<const uint4*>(s.q + (size_t)m * K + sb * 256 + L * 32);
                    const uint4 a0 = ap[0], a1 = ap[1];   // sb = 0 when off: in bounds, result discarded
                    const float da = on ? s.d[m * nsb + sb] : 0.0f;
#pragma unroll
                    for (int j = 0; j < NR; ++j) {
                        int d1 = 0, d2 = 0;
                        d1 = __dp4a((int)__vsub4(qw[j][0], 0x20202020u), (int)a0.x, d1);
                        d1 = __dp4a((int)__vsub4(qw[j][1], 0x20202020u), (int)a0.y, d1);
                        d1 = __dp4a((int)__vsub4(qw[j][2], 0x20202020u), (int)a0.z, d1);
                        d1 = __dp4a((int)__vsub4(qw[j][3], 0x20202020u), (int)a0.w, d1);
                        d2 = __dp4a((int)__vsub4(qw[j][4], 0x20202020u), (int)a1.x, d2);
                        d2 = __dp4a((int)__vsub4(qw[j][5], 0x20202020u), (int)a1.y, d2);
                        d2 = __dp4a((int)__vsub4(qw[j][6], 0x20202020u), (int)a1.z, d2);
                        d2 = __dp4a((int)__vsub4(qw[j][7], 0x20202020u), (int)a1.w, d2);
                        int is = sc0[j] * d1 + sc1[j] * d2;
#pragma unroll
                        for (int o = 1; o < 8; o <<= 1) is += __shfl_xor_sync(0xffffffffu, is, o, 8);
                        if (L == 0) acc[j][m] = __fadd_rn(acc[j][m], __fmul_rn(__fmul_rn(dd[j], da), (float)is));
                    }
                }
            }
        } else {
            // F32 / F16 weights: f32 (or f16-rounded) activations, f32 FMA
            for (int k = lane * 4; k < K; k += 128) {
                float wv[NR][4];
#pragma unroll
                for (int j = 0; j < NR; ++j) {
                    const DevW& W = which[j] ? a.w1 : a.w0;
                    if (row[j] < 0) { wv[j][0] = wv[j][1] = wv[j][2] = wv[j][3] = 0.0f; continue; }
                    if constexpr (WT == W_F32) {
                        const float4 f = __ldg(reinterpret_cast<const float4*>(W.q + (size_t)row[j] * W.row_stride) + k / 4);
                        wv[j][0] = f.x; wv[j][1] = f.y; wv[j][2] = f.z; wv[j][3] = f.w;
                    } else {
                        const uint2 h = __ldg(reinterpret_cast<const uint2*>(W.q + (size_t)row[j] * W.row_stride + k * 2));
                        const __half2 h0 = *reinterpret_cast<const __half2*>(&h.x);
                        const __half2 h1 = *reinterpret_cast<const __half2*>(&h.y);
                        wv[j][0] = __low2float(h0); wv[j][1] = __high2float(h0);
                        wv[j][2] = __low2float(h1); wv[j][3] = __high2float(h1);
                    }
                }
#pragma unroll
                for (int m = 0; m < GEMV_MAX_M; ++m) {
                    if (m >= M) break;
                    const float4 av = *reinterpret_cast<const float4*>(s.f + (size_t)m * K + k);
#pragma unroll
                    for (int j = 0; j < NR; ++j) {
                        acc[j][m] = fmaf(wv[j][0], av.x, acc[j][m]);
                        acc[j][m] = fmaf(wv[j][1], av.y, acc[j][m]);
                        acc[j][m] = fmaf(wv[j][2], av.z, acc[j][m]);
                        acc[j][m] = fmaf(wv[j][3], av.w, acc[j][m]);
                    }
                }
            }
        }
    }
    // lane reduction: every lane ends with every sum
#pragma unroll
    for (int j = 0; j < NR; ++j)
#pragma unroll
        for (int m = 0; m < GEMV_MAX_M; ++m)
            if (m < M) acc[j][m] = warp_sum(acc[j][m]);

    // ---------------------------------------------------------- epilogues
    if constexpr (EPI == EPI_QKV) {
        if (valid && lane < M) {
            const int m = lane;
            float v0 = 0.f, v1 = 0.f;
#pragma unroll
            for (int mm = 0; mm < GEMV_MAX_M; ++mm)
                if (mm == m) { v0 = acc[0][mm]; v1 = acc[1][mm]; }
            if (a.bias) {
                v0 = __fadd_rn(v0, a.bias[row[0]]);
                v1 = __fadd_rn(v1, a.bias[row[1]]);
            }
            const int h = row[0] / a.hd, i = row[0] % a.hd;
            const RowMeta rm = a.meta[m];
            if (h < a.n_q_heads + a.n_kv_heads) rope_pair(v0, v1, rm.pos, i, a.rope_ts);
            if (h < a.n_q_heads) {
                float* q = a.y + (size_t)m * a.y_stride + h * a.hd;
                q[i] = v0;
                q[i + a.hd / 2] = v1;
            } else {
                const bool is_k = h < a.n_q_heads + a.n_kv_heads;
                const int kvh = is_k ? h - a.n_q_heads : h - a.n_q_heads - a.n_kv_heads;
                __half* dst = (is_k ? a.kv.k : a.kv.v) + kv_offset(a.kv, rm.seq, rm.cidx, kvh);
                dst[i] = __float2half_rn(v0);
                dst[i + a.hd / 2] = __float2half_rn(v1);
            }
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
        if (valid && lane < M) {
            float g = 0.f, up = 0.f;
#pragma unroll
            for (int mm = 0; mm < GEMV_MAX_M; ++mm)
                if (mm == lane) { g = acc[0][mm]; up = acc[1][mm]; }
            a.y[(size_t)lane * a.y_stride + row[0]] = __fmul_rn(silu_ref(g), up);
        }
    } else if constexpr (EPI == EPI_RESID || EPI == EPI_STORE) {
        if (valid && lane < NR * M) {
            const int j = lane / M, m = lane % M;
            float v = 0.f;
            int r = -1;
#pragma unroll
            for (int jj = 0; jj < NR; ++jj)
#pragma unroll
                for (int mm = 0; mm < GEMV_MAX_M; ++mm)
                    if (jj == j && mm == m) { v = acc[jj][mm]; r = row[jj]; }
            if (r >= 0) {
                if (a.bias) v = __fadd_rn(v, a.bias[r]);
                float* dst = a.y + (size_t)m * a.y_stride + r;
                if (EPI == EPI_RESID) *dst = __fadd_rn(*dst, v);   // ggml_add(x, o)
                else *dst = v;
            }
        }
    } else if constexpr (EPI == EPI_ARGMAX) {
        if (valid && lane < M) {
            const int m = lane;
            unsigned long long k = 0ull;
#pragma unroll
            for (int j = 0; j < NR; ++j) {
                float v = 0.f;
#pragma unroll
                for (int mm = 0; mm < GEMV_MAX_M; ++mm)
                    if (mm == m) v = acc[j][mm];
                if (row[j] >= 0) {
                    if (a.y) a.y[(size_t)m * a.y_stride + row[j]] = v;
                    const unsigned long long kk = argmax_key(v, row[j]);
                    k = kk > k ? kk : k;
                }
            }
            atomicMax(&best[m], k);
        }
        __syncthreads();
        if (threadIdx.x < M) atomicMax(a.argmax + threadIdx.x, best[threadIdx.x]);
    }
}

template <int WT, int NR, int EPI>
cudaError_t launch_t(const GemvArgs& a, cudaStream_t st) {
    const size_t smem = act_smem_bytes(WT, a.M, a.K);
    if (smem > GEMV_SMEM_MAX) return cudaErrorInvalidValue;   // gemv_prepare() opted in up to this
    auto kern = k_gemv<WT, NR, EPI>;
    const int grid = (a.n_units + GEMV_WARPS - 1) / GEMV_WARPS;
    kern<<<grid, GEMV_THREADS, smem, st>>>(a);
    note_launch();
    return cudaGetLastError();
}

template <int EPI, int NR>
cudaError_t launch_wt(const GemvArgs& a, cudaStream_t st) {
    switch (a.w0.type) {
        case W_Q8_0: return launch_t<W_Q8_0, NR, EPI>(a, st);
        case W_Q5_K: return launch_t<W_Q5_K, NR, EPI>(a, st);
        case W_Q6_K: return launch_t<W_Q6_K, NR, EPI>(a, st);
        case W_F32: return launch_t<W_F32, NR, EPI>(a, st);
        case W_F16: return launch_t<W_F16, NR, EPI>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

template <int EPI, int NR>
cudaError_t prepare_wt() {
    const void* fns[] = {(const void*)k_gemv<W_Q8_0, NR, EPI>, (const void*)k_gemv<W_Q5_K, NR, EPI>,
                         (const void*)k_gemv<W_Q6_K, NR, EPI>, (const void*)k_gemv<W_F32, NR, EPI>,
                         (const void*)k_gemv<W_F16, NR, EPI>};
    for (const void* f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMV_SMEM_MAX);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

size_t gemv_smem_bytes(int wt, int M, int K) { return act_smem_bytes(wt, M, K); }

// Opt every instantiation in to large dynamic shared memory once per device,
// before any launch or stream capture.
cudaError_t gemv_prepare() {
    cudaError_t e;
    if ((e = prepare_wt<EPI_QKV, 2>()) != cudaSuccess) return e;
    if ((e = prepare_wt<EPI_SWIGLU, 2>()) != cudaSuccess) return e;
    if ((e = prepare_wt<EPI_RESID, 2>()) != cudaSuccess) return e;
    if ((e = prepare_wt<EPI_STORE, 4>()) != cudaSuccess) return e;
    return prepare_wt<EPI_ARGMAX, 4>();
}

cudaError_t gemv_launch(GemvArgs a, cudaStream_t st) {
    if (a.M < 1 || a.M > GEMV_MAX_M) return cudaErrorInvalidValue;
    if (a.w0.type == W_Q8_0 && a.K % 32) return cudaErrorInvalidValue;
    if ((a.w0.type == W_Q5_K || a.w0.type == W_Q6_K) && a.K % 256) return cudaErrorInvalidValue;
    if ((a.w0.type == W_F32 || a.w0.type == W_F16) && a.K % 4) return cudaErrorInvalidValue;
    switch (a.epi) {
        case EPI_QKV:
            a.n_units = a.w0.rows / 2;
            return launch_wt<EPI_QKV, 2>(a, st);
        case EPI_SWIGLU:
            a.n_units = a.w0.rows;
            return launch_wt<EPI_SWIGLU, 2>(a, st);
        case EPI_RESID:
            a.n_units = (a.w0.rows + 1) / 2;
            return launch_wt<EPI_RESID, 2>(a, st);
        case EPI_STORE:
            a.n_units = (a.w0.rows + 3) / 4;
            return launch_wt<EPI_STORE, 4>(a, st);
        case EPI_ARGMAX:
            a.n_units = (a.w0.rows + 3) / 4;
            return launch_wt<EPI_ARGMAX, 4>(a, st);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace vvq2
