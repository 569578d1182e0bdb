// gemv.cu -- decode-time (<= 8 activation rows) fused dequant GEMV on sm_100a.
//
// One kernel family covers every linear of the Qwen2 layer at decode time
// (src/qwen2.cpp:19-26,274-276,349 and the SwiGLU FFN at :33-40), the lm_head
// (src/vibevoice_asr.cpp:285-311) and its greedy argmax (:702-706).
//
// Numerics: weights are dequantized exactly as ggml's dequantize_row_* does
// (bit-identical f32 values), activations stay f32, products accumulate in f32
// (Blackwell packed FFMA2).  This is the
// "exact" restatement of ggml_mul_mat; ggml's CPU backend additionally rounds
// the activations to int8 blocks (its vec_dot_type), a step whose rounding
// flips cascade through RMSNorm, so it is reproduced only by the CPU oracle.
//
// Two kernels, both persistent grids (one wave of resident CTAs) that stage
// the M activation rows in shared memory first -- with the RMSNorm
// (src/rms_norm.hpp:11-17) when the linear follows one -- and read every
// weight byte from HBM once, 4-row units at a time, the activation chunk
// reused for the 4 rows:
//  * k_gemv_stream (1-2 rows, the decode of one sequence or a CFG pair; see
//    its own comment): register-pipelined weight loads, no block barrier in
//    the main loop, I2F-free dequantization;
//  * k_gemv (3-8 rows): warps split a unit's K, register ping-pong.
// Epilogues: QKV (+bias, NEOX RoPE on Q/K, Q to a buffer, K/V appended to the
// f16 paged cache), residual add, SwiGLU, store, and argmax.  Kernels are
// launched with programmatic dependent launch: weight loads start before
// griddepcontrol.wait, overlapping the previous kernel's tail.
#include <type_traits>

#include "common.cuh"
#include "gemv_dev.cuh"
#include "kernels.h"

namespace vvq2 {

namespace {

using gd::Chunk;
using gd::load_chunk;
using gd::expand4;
using gd::clear_chunk;

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int NR = 4;                        // weight rows per warp unit
constexpr size_t GEMV_SMEM_MAX = 200 * 1024;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// Row r of unit u: (tensor, row).  QKV: two NEOX pairs (i0, i0+1) of one head;
// SwiGLU: gate rows i0, i0+1 then up rows i0, i0+1; else 4 consecutive rows.
template <int EPI>
__device__ __forceinline__ void unit_rows(const GemvArgs& a, int u, int* row, int* which) {
    if constexpr (EPI == EPI_QKV) {
        const int half = a.hd / 2, per_head = half / 2;
        const int h = u / per_head, i0 = 2 * (u % per_head);
        row[0] = h * a.hd + i0;
        row[1] = row[0] + 1;
        row[2] = row[0] + half;
        row[3] = row[1] + half;
        which[0] = which[1] = which[2] = which[3] = 0;
    } else if constexpr (EPI == EPI_SWIGLU) {
        row[0] = row[2] = 2 * u;
        row[1] = row[3] = 2 * u + 1;
        which[0] = which[1] = 0;
        which[2] = which[3] = 1;
    } else {
#pragma unroll
        for (int j = 0; j < NR; ++j) {
            row[j] = u * NR + j;
            which[j] = 0;
        }
    }
}

// Stage M activation rows (optionally RMSNorm'd) as f32 in shared memory.
__device__ void stage_activations(const GemvArgs& a, float* act) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = a.M, K = a.K;
    __shared__ float red[GEMV_MAX_M * GEMV_WARPS];
    __shared__ float row_scale[GEMV_MAX_M];
    const int K4 = K / 4;
    if (a.norm_w) {
        // ggml_compute_forward_rms_norm_f32: scale = 1/sqrtf(mean(x^2) + eps)
        float ss[GEMV_MAX_M];
#pragma unroll
        for (int m = 0; m < GEMV_MAX_M; ++m) ss[m] = 0.f;
        for (int k = tid; k < K4; k += GEMV_THREADS) {
#pragma unroll
            for (int m = 0; m < GEMV_MAX_M; ++m) {
                if (m < M) {
                    const float4 v = reinterpret_cast<const float4*>(a.x + (size_t)m * a.x_stride)[k];
                    reinterpret_cast<float4*>(act + (size_t)m * K)[k] = v;
                    ss[m] = fmaf(v.x, v.x, ss[m]);
                    ss[m] = fmaf(v.y, v.y, ss[m]);
                    ss[m] = fmaf(v.z, v.z, ss[m]);
                    ss[m] = fmaf(v.w, v.w, ss[m]);
                }
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
            float t = 0.f;
            for (int w = 0; w < GEMV_WARPS; ++w) t += red[tid * GEMV_WARPS + w];
            const float mean = __fdiv_rn(t, (float)K);
            row_scale[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        }
        __syncthreads();
        for (int k = tid; k < K4; k += GEMV_THREADS) {
            const float4 w = reinterpret_cast<const float4*>(a.norm_w)[k];
#pragma unroll
            for (int m = 0; m < GEMV_MAX_M; ++m) {
                if (m < M) {
                    float4* p = reinterpret_cast<float4*>(act + (size_t)m * K) + k;
                    float4 v = *p;
                    const float s = row_scale[m];
                    v.x = __fmul_rn(__fmul_rn(v.x, s), w.x);   // (x*scale)*w
                    v.y = __fmul_rn(__fmul_rn(v.y, s), w.y);
                    v.z = __fmul_rn(__fmul_rn(v.z, s), w.z);
                    v.w = __fmul_rn(__fmul_rn(v.w, s), w.w);
                    *p = v;
                }
            }
        }
    } else {
        for (int k = tid; k < K4; k += GEMV_THREADS) {
#pragma unroll
            for (int m = 0; m < GEMV_MAX_M; ++m)
                if (m < M)
                    reinterpret_cast<float4*>(act + (size_t)m * K)[k] =
                        reinterpret_cast<const float4*>(a.x + (size_t)m * a.x_stride)[k];
        }
    }
    __syncthreads();
}

// Work decomposition.  A unit is NR weight rows; a unit is split across `wpu`
// warps (each takes every wpu-th 512-element "item" of the row: one 16-element
// chunk per lane), so 8 / wpu units form a CTA group.  CTAs loop over groups
// (persistent when there are more groups than resident CTAs).  Partial sums
// meet in shared memory; the unit's first warp runs the epilogue.
struct Work {
    int nchunk, niter, wpu, upc, sub, slot, n_it, n_groups;
};

__device__ __forceinline__ Work make_work(const GemvArgs& a, int warp) {
    Work w;
    w.nchunk = a.K / 16;
    w.niter = (w.nchunk + 31) / 32;
    w.wpu = a.wpu;
    w.upc = GEMV_WARPS / a.wpu;
    w.sub = warp % a.wpu;
    w.slot = warp / a.wpu;
    w.n_it = (w.niter - w.sub + w.wpu - 1) / w.wpu;   // >= 1 because wpu <= niter
    w.n_groups = (a.n_units + w.upc - 1) / w.upc;
    return w;
}

template <int WT, int EPI>
__device__ __forceinline__ void load_item(const GemvArgs& a, const Work& w, int group, int l, int lane,
                                          Chunk* dst) {
    const int u = group * w.upc + w.slot;
    const int c = (w.sub + l * w.wpu) * 32 + lane;
    int r[NR], wh[NR];
    unit_rows<EPI>(a, u < a.n_units ? u : 0, r, wh);
#pragma unroll
    for (int j = 0; j < NR; ++j) {
        const DevW& W = wh[j] ? a.w1 : a.w0;
        if (u < a.n_units && c < w.nchunk && r[j] < W.rows) load_chunk<WT>(W, r[j], c, dst[j]);
        else clear_chunk<WT>(dst[j]);
    }
}

template <int WT, int MB>
__device__ __forceinline__ void compute_item(const Chunk* ch, const float* act, int K, int M, int c,
                                             float2 (&acc2)[NR][MB]) {
    const int rot = (c >> 1) & 3;   // conflict-free float4 order within 8-lane phases
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int g = (t + rot) & 3;
        float w[NR][4];
#pragma unroll
        for (int j = 0; j < NR; ++j) expand4<WT>(ch[j], g, w[j]);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            if (m >= M) break;
            const float4 av = reinterpret_cast<const float4*>(act + (size_t)m * K + c * 16)[g];
            const float2 a01 = make_float2(av.x, av.y), a23 = make_float2(av.z, av.w);
#pragma unroll
            for (int j = 0; j < NR; ++j) {
                acc2[j][m] = __ffma2_rn(make_float2(w[j][0], w[j][1]), a01, acc2[j][m]);
                acc2[j][m] = __ffma2_rn(make_float2(w[j][2], w[j][3]), a23, acc2[j][m]);
            }
        }
    }
}

template <int WT, int EPI, int MB>
__global__ void __launch_bounds__(GEMV_THREADS, 2) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(16) float act[];
    __shared__ unsigned long long best[GEMV_MAX_M];
    __shared__ float part[GEMV_WARPS][NR * GEMV_MAX_M];
    __shared__ float rope_c[EPI == EPI_QKV ? GEMV_MAX_M : 1][EPI == EPI_QKV ? 64 : 1];
    __shared__ float rope_s[EPI == EPI_QKV ? GEMV_MAX_M : 1][EPI == EPI_QKV ? 64 : 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int M = a.M, K = a.K;
    const Work w = make_work(a, warp);
    const int my_groups = blockIdx.x < w.n_groups ? (w.n_groups - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const int n_items = my_groups * w.n_it;

    // weights do not depend on the previous kernel: issue the first item's
    // loads, then wait for the producer of the activations
    Chunk A[NR], B[NR];
    if (n_items > 0) load_item<WT, EPI>(a, w, blockIdx.x, 0, lane, A);
    pdl_launch();
    pdl_wait();
    if (EPI == EPI_ARGMAX && threadIdx.x < GEMV_MAX_M) best[threadIdx.x] = 0ull;
    if constexpr (EPI == EPI_QKV) {
        // NEOX cos/sin per (row, pair) with ggml's CPU theta recurrence, once per CTA
        const int half = a.hd / 2;
        for (int t = threadIdx.x; t < M * half; t += GEMV_THREADS) {
            const int m = t / half, i = t % half;
            float th = (float)(a.rope_meta ? a.rope_meta : a.meta)[m].pos;   // true position (partitioned ranks shift meta.pos)
            for (int k = 0; k < i; ++k) th = __fmul_rn(th, a.rope_ts);
            rope_c[m][i] = cosf(th);
            rope_s[m][i] = sinf(th);
        }
    }
    stage_activations(a, act);   // ends with __syncthreads

    float2 acc2[NR][MB];
#pragma unroll
    for (int j = 0; j < NR; ++j)
#pragma unroll
        for (int m = 0; m < MB; ++m) acc2[j][m] = make_float2(0.f, 0.f);

    int row[NR], which[NR];
    // one flattened item sequence per warp, ping-ponged between register sets
    // A and B so the next item's loads are in flight while one is computed
    auto finish = [&](int i) {
        // called after item i; if it closed a group: reduce, epilogue, reset
        if ((i % w.n_it) != w.n_it - 1) return;
        const int group = blockIdx.x + (i / w.n_it) * gridDim.x;
        const int u = group * w.upc + w.slot;
#pragma unroll
        for (int j = 0; j < NR; ++j)
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                const float v = (m < M) ? warp_sum(acc2[j][m].x + acc2[j][m].y) : 0.f;
                acc2[j][m] = make_float2(0.f, 0.f);
                if (lane == j * M + m && m < M) part[warp][lane] = v;
            }
        __syncthreads();
        if (w.sub == 0 && u < a.n_units) {
            unit_rows<EPI>(a, u, row, which);
            float v = 0.f;
            int jj = 0, mm = 0;
            if (lane < NR * M) {
                jj = lane / M;
                mm = lane % M;
                for (int s2 = 0; s2 < w.wpu; ++s2) v += part[warp + s2][lane];
            }
            if constexpr (EPI == EPI_QKV) {
                // lanes (j, m): NEOX partners j and j+2 sit in lanes L and L + 2M
                if (a.bias && lane < NR * M) v = __fadd_rn(v, a.bias[row[jj]]);
                const float partner = __shfl_down_sync(0xffffffffu, v, 2 * M);
                if (lane < 2 * M) {
                    const int r0 = row[jj];
                    const int h = r0 / a.hd, i2 = r0 % a.hd;
                    const RowMeta rm = a.meta[mm];
                    float x0 = v, x1 = partner;
                    if (h < a.n_q_heads + a.n_kv_heads) {
                        const float c = rope_c[mm][i2], s = rope_s[mm][i2];
                        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
                        const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
                        x0 = y0;
                        x1 = y1;
                    }
                    if (h < a.n_q_heads) {
                        float* q = a.y + (size_t)mm * a.y_stride + h * a.hd;
                        q[i2] = x0;
                        q[i2 + a.hd / 2] = x1;
                    } else if (rm.cidx >= 0) {   // cidx < 0: another rank stores this position
                        const bool is_k = h < a.n_q_heads + a.n_kv_heads;
                        const int kvh = is_k ? h - a.n_q_heads : h - a.n_q_heads - a.n_kv_heads;
                        __half* dst = (is_k ? a.kv.k : a.kv.v) + kv_offset(a.kv, rm.seq, rm.cidx, kvh);
                        dst[i2] = __float2half_rn(x0);
                        dst[i2 + a.hd / 2] = __float2half_rn(x1);
                    }
                }
            } else if constexpr (EPI == EPI_SWIGLU) {
                const float up = __shfl_down_sync(0xffffffffu, v, 2 * M);
                if (lane < 2 * M) a.y[(size_t)mm * a.y_stride + row[jj]] = __fmul_rn(silu_ref(v), up);
            } else if constexpr (EPI == EPI_RESID || EPI == EPI_STORE) {
                if (lane < NR * M && row[jj] < a.w0.rows) {
                    if (a.bias) v = __fadd_rn(v, a.bias[row[jj]]);
                    float* dst = a.y + (size_t)mm * a.y_stride + row[jj];
                    if (EPI == EPI_RESID) *dst = __fadd_rn(*dst, v);   // ggml_add(x, o)
                    else *dst = v;
                }
            } else if constexpr (EPI == EPI_ARGMAX) {
                unsigned long long k = 0ull;
                if (lane < NR * M && row[jj] < a.w0.rows) {
                    if (a.y) a.y[(size_t)mm * a.y_stride + row[jj]] = v;
                    k = argmax_key(v, row[jj]);
                }
                // max over the NR rows of each m (lanes m, m+M, m+2M, m+3M)
                for (int o = M; o < NR * M; o <<= 1) {
                    const unsigned long long k2 = __shfl_down_sync(0xffffffffu, k, o);
                    k = k2 > k ? k2 : k;
                }
                if (lane < M) atomicMax(&best[lane], k);
            }
        }
        __syncthreads();   // part[] is reused by the next group
    };
    auto item_chunk = [&](int i) { return (w.sub + (i % w.n_it) * w.wpu) * 32 + lane; };
    auto item_group = [&](int i) { return blockIdx.x + (i / w.n_it) * gridDim.x; };
    for (int i = 0; i < n_items; i += 2) {
        if (i + 1 < n_items) load_item<WT, EPI>(a, w, item_group(i + 1), (i + 1) % w.n_it, lane, B);
        {
            const int c = item_chunk(i);
            if (c < w.nchunk) compute_item<WT, MB>(A, act, K, M, c, acc2);
        }
        finish(i);
        if (i + 1 < n_items) {
            if (i + 2 < n_items) load_item<WT, EPI>(a, w, item_group(i + 2), (i + 2) % w.n_it, lane, A);
            const int c = item_chunk(i + 1);
            if (c < w.nchunk) compute_item<WT, MB>(B, act, K, M, c, acc2);
            finish(i + 1);
        }
    }
    if constexpr (EPI == EPI_ARGMAX) {
        __syncthreads();
        if (threadIdx.x < M && best[threadIdx.x]) atomicMax(a.argmax + threadIdx.x, best[threadIdx.x]);
    }
}

// ------------------------------------------------------------------------
// Streaming GEMV for one or two activation rows (a decode step of one
// sequence or of a CFG pair): the bandwidth-bound case.
//
// One CTA of 16 warps per SM.  CTA b owns a contiguous range of units (NR
// weight rows each, grouped by unit_rows), cut into (unit, item) pairs; an
// item is 512 consecutive K elements of the unit's rows, one 16-element chunk
// per lane.  Warp w takes pairs w, w + 16, w + 32, ... and keeps the weight
// loads of its next SP pairs in flight in registers -- the first ones are
// issued before the activations are even staged (programmatic dependent
// launch), and there is no block-wide barrier in the main loop, so every SM
// keeps ~SP x 2 KB per warp outstanding.  Q8_0/K-quant values become exact
// floats without I2F (the unsigned byte in the mantissa of 2^23, minus 2^23 +
// offset) and the block scale multiplies each 16-element partial sum.  Per
// pair the warp reduces its NR x MB sums with one transposing butterfly into
// shared memory; after one block barrier each row's per-item partials are
// summed in item order (deterministic), scaled by the row's RMSNorm factor
// (the staged activations are x * w; W (x s o w) = s W (x o w)), and the
// epilogue applied.
// K-quants use 32-weight lane tasks (gd::kq_*) with ~11-12 registers per row
// and 3 register stages: 256-thread CTAs (255 registers); everything else 512
template <int WT>
struct SKq {
    static constexpr bool v = WT == W_Q5_K || WT == W_Q6_K;
};
template <int WT>
struct SThreads {
    static constexpr int v = SKq<WT>::v ? 256 : 512;
};
constexpr size_t S_SMEM_MAX = 220 * 1024;

struct Q8Raw {
    uint4 q;        // 16 quants
    uint32_t d;     // f16 block scale bits
};

// one 32-weight K-quant lane task of one row, as loaded
struct KqRaw {
    uint4 lo, hi;   // low-bit run (Q6_K ql / Q5_K qs) and high-bit run (qh)
    uint4 aux;      // Q5_K: the block header (d, dmin, 12 scale bytes); Q6_K: x, y = the
                    // half's 8 int8 scales, z = f16 d bits
};

template <int WT>
using SChunk = typename std::conditional<WT == W_Q8_0, Q8Raw,
                                         typename std::conditional<SKq<WT>::v, KqRaw, Chunk>::type>::type;

// register stages of weight loads per warp (by type and activation rows)
template <int WT, int MB>
struct SPipe {
    static constexpr int P = WT == W_Q8_0 ? (MB == 1 ? 4 : 2) : WT == W_F32 ? 1 : SKq<WT>::v ? 3 : 2;
};

template <int WT>
__device__ __forceinline__ void s_load(const DevW& W, int row, int c, bool ok, SChunk<WT>& ch) {
    if constexpr (SKq<WT>::v) {
        // c is the lane task t: super-block t >> 3 (see gd::kq_*)
        if (ok) {
            const int sb = c >> 3;
            const uint8_t* b = W.q + (size_t)row * W.row_stride + (size_t)sb * (WT == W_Q6_K ? Q6K_PACKED : Q5K_BYTES);
            ch.lo = __ldg(reinterpret_cast<const uint4*>(b + gd::kq_lo_off<WT>(c)));
            ch.hi = __ldg(reinterpret_cast<const uint4*>(b + gd::kq_hi_off<WT>(c)));
            if constexpr (WT == W_Q6_K) {
                const uint2 sc = __ldg(reinterpret_cast<const uint2*>(b + 192 + ((c & 7) >> 2) * 8));
                ch.aux = make_uint4(sc.x, sc.y, __ldg(reinterpret_cast<const unsigned short*>(W.d) +
                                                      (size_t)row * W.d_stride + sb), 0u);
            } else {
                ch.aux = __ldg(reinterpret_cast<const uint4*>(b));
            }
        } else {
            ch.lo = ch.hi = ch.aux = make_uint4(0, 0, 0, 0);
        }
    } else if constexpr (WT == W_Q8_0) {
        if (ok) {
            const uint8_t* rp = W.q + (size_t)row * W.row_stride;
            ch.q = __ldg(reinterpret_cast<const uint4*>(rp) + c);
            ch.d = __ldg(reinterpret_cast<const unsigned short*>(W.d) + (size_t)row * W.d_stride + c / 2);
        } else {
            ch.q = make_uint4(0, 0, 0, 0);
            ch.d = 0;
        }
    } else {
        if (ok) load_chunk<WT>(W, row, c, ch);
        else clear_chunk<WT>(ch);
    }
}

// exact floats of the four unsigned bytes of w: 2^23 + byte (then an FFMA2 removes the offset)
__device__ __forceinline__ void magic4(uint32_t w, float2& f01, float2& f23) {
    f01 = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)),
                      __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441)));
    f23 = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)),
                      __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443)));
}

// Dot of one lane's 16-element chunk of one weight row with MB activation
// chunks (av[m][g] = elements 4g .. 4g+3 of row m).
template <int WT, int MB>
__device__ __forceinline__ void s_dot(const SChunk<WT>& ch, const float4 (&av)[MB][4], float (&out)[MB]) {
    const float2 one2 = make_float2(1.0f, 1.0f);
    float2 s[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) s[m] = make_float2(0.f, 0.f);
    if constexpr (WT == W_Q8_0 || WT == W_Q5_K || WT == W_Q6_K) {
        // Q8_0: stored as the unsigned byte q + 128; Q5_K: 0..31; Q6_K: q - 32 with q in 0..63
        constexpr float OFF = WT == W_Q8_0 ? -8388736.0f : WT == W_Q5_K ? -8388608.0f : -8388640.0f;
        const float2 off2 = make_float2(OFF, OFF);
        float2 as[MB], t[MB];
#pragma unroll
        for (int m = 0; m < MB; ++m) t[m] = make_float2(0.f, 0.f);
#pragma unroll
        for (int m = 0; m < MB; ++m) as[m] = make_float2(0.f, 0.f);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            uint32_t w;
            if constexpr (WT == W_Q8_0) {
                w = gd::word(ch.q, g);   // bytes are q + 128 (device layout)
            } else if constexpr (WT == W_Q5_K) {
                const int j = ch.shift;
                w = ((gd::word(ch.r0, g) >> (4 * (j & 1))) & 0x0F0F0F0Fu) |
                    (((gd::word(ch.r1, g) >> j) & 0x01010101u) << 4);
            } else {
                const int k = ch.shift;
                w = ((gd::word(ch.r0, g) >> (4 * (k >> 1))) & 0x0F0F0F0Fu) |
                    (((gd::word(ch.r1, g) >> (2 * k)) & 0x03030303u) << 4);
            }
            float2 f01, f23;
            magic4(w, f01, f23);
            f01 = __ffma2_rn(f01, one2, off2);
            f23 = __ffma2_rn(f23, one2, off2);
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                const float2 a01 = make_float2(av[m][g].x, av[m][g].y), a23 = make_float2(av[m][g].z, av[m][g].w);
                s[m] = __ffma2_rn(f01, a01, s[m]);    // two independent chains per row
                t[m] = __ffma2_rn(f23, a23, t[m]);
                if constexpr (WT == W_Q5_K) {
                    as[m] = __fadd2_rn(as[m], a01);
                    as[m] = __fadd2_rn(as[m], a23);
                }
            }
        }
        float d;
        if constexpr (WT == W_Q8_0) d = __half2float(__ushort_as_half((unsigned short)ch.d));
        else d = ch.scale;
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            out[m] = __fmul_rn(d, (s[m].x + s[m].y) + (t[m].x + t[m].y));
            // Q5_K: w = d1 q - m1, so w.a = d1 (q.a) - m1 (sum a)
            if constexpr (WT == W_Q5_K) out[m] = fmaf(-ch.mscale, as[m].x + as[m].y, out[m]);
        }
    } else {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            float w[4];
            expand4<WT>(ch, g, w);
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                s[m] = __ffma2_rn(make_float2(w[0], w[1]), make_float2(av[m][g].x, av[m][g].y), s[m]);
                s[m] = __ffma2_rn(make_float2(w[2], w[3]), make_float2(av[m][g].z, av[m][g].w), s[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < MB; ++m) out[m] = s[m].x + s[m].y;
    }
}

// byte k (runtime) of a 16-byte register quad
__device__ __forceinline__ uint32_t qbyte(const uint4& v, int k) { return (gd::word(v, k >> 2) >> (8 * (k & 3))) & 0xffu; }

// Dot of sub-chunk s (16 weights) of K-quant lane task t of one row with MB
// activation chunks; scales as ggml: Q6_K (d * sc) * (q - 32), Q5_K
// (d * sc) * q - dmin * m, factored out of the 16-weight sum.
template <int WT, int MB>
__device__ __forceinline__ void kq_dot(const KqRaw& ch, const float4 (&av)[MB][4], int t, int s, float (&out)[MB]) {
    const float2 one2 = make_float2(1.0f, 1.0f);
    constexpr float OFF = WT == W_Q5_K ? -8388608.0f : -8388640.0f;   // 2^23 (+ 32 for Q6_K)
    const float2 off2 = make_float2(OFF, OFF);
    float2 sa[MB], sb[MB], as[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) sa[m] = sb[m] = as[m] = make_float2(0.f, 0.f);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint32_t w = gd::kq_word<WT>(gd::word(ch.lo, g), gd::word(ch.hi, g), t, s);
        float2 f01, f23;
        magic4(w, f01, f23);
        f01 = __ffma2_rn(f01, one2, off2);
        f23 = __ffma2_rn(f23, one2, off2);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            const float2 a01 = make_float2(av[m][g].x, av[m][g].y), a23 = make_float2(av[m][g].z, av[m][g].w);
            sa[m] = __ffma2_rn(f01, a01, sa[m]);
            sb[m] = __ffma2_rn(f23, a23, sb[m]);
            if constexpr (WT == W_Q5_K) {
                as[m] = __fadd2_rn(as[m], a01);
                as[m] = __fadd2_rn(as[m], a23);
            }
        }
    }
    float scale, mscale = 0.f;
    if constexpr (WT == W_Q6_K) {
        const int k = gd::q6_scale_idx(t, s);
        const int sc = (int)(int8_t)(((k < 4 ? ch.aux.x : ch.aux.y) >> (8 * (k & 3))) & 0xffu);
        scale = __fmul_rn(__half2float(__ushort_as_half((unsigned short)ch.aux.z)), (float)sc);
    } else {
        const int j = ((t & 7) >> 1) * 2 + s;
        int sc, mn;
        if (j < 4) {
            sc = (int)(qbyte(ch.aux, 4 + j) & 63);
            mn = (int)(qbyte(ch.aux, 8 + j) & 63);
        } else {
            sc = (int)((qbyte(ch.aux, 8 + j) & 0xF) | ((qbyte(ch.aux, j) >> 6) << 4));
            mn = (int)((qbyte(ch.aux, 8 + j) >> 4) | ((qbyte(ch.aux, 4 + j) >> 6) << 4));
        }
        const __half2 dh = *reinterpret_cast<const __half2*>(&ch.aux.x);
        scale = __fmul_rn(__low2float(dh), (float)sc);     // d1 = d * sc
        mscale = __fmul_rn(__high2float(dh), (float)mn);   // m1 = dmin * m
    }
#pragma unroll
    for (int m = 0; m < MB; ++m) {
        out[m] = __fmul_rn(scale, (sa[m].x + sa[m].y) + (sb[m].x + sb[m].y));
        if constexpr (WT == W_Q5_K) out[m] = fmaf(-mscale, as[m].x + as[m].y, out[m]);
    }
}

template <int N>
struct SLog2 {
    static constexpr int v = 1 + SLog2<N / 2>::v;
};
template <>
struct SLog2<1> {
    static constexpr int v = 0;
};

// Sum NV (a power of two) per-lane values over the warp; lane l returns the
// total of value index l >> (5 - log2 NV).
template <int NV>
__device__ __forceinline__ float s_transpose_sum(float (&v)[NV], int lane) {
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
    for (int o = 16 >> SLog2<NV>::v; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    return v[0];
}

template <int WT, int EPI, int MB>
__global__ void __launch_bounds__(SThreads<WT>::v, 1) k_gemv_stream(const GemvArgs a) {
    constexpr int S_THREADS = SThreads<WT>::v;
    constexpr int S_WARPS = S_THREADS / 32;
    constexpr bool KQ = SKq<WT>::v;
    constexpr int P = SPipe<WT, MB>::P;
    constexpr int NV = NR * MB;
    constexpr int SH = 5 - SLog2<NV>::v;
    extern __shared__ __align__(16) float sm_act[];
    __shared__ float red[MB * S_WARPS];
    __shared__ unsigned long long best[MB];
    __shared__ float rope_c[EPI == EPI_QKV ? MB : 1][EPI == EPI_QKV ? 64 : 1];
    __shared__ float rope_s[EPI == EPI_QKV ? MB : 1][EPI == EPI_QKV ? 64 : 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // an item is 32 lane tasks: 16-weight chunks (NC per row) or, for the
    // K-quants, 32-weight lane tasks (NTK per row)
    const int K = a.K, NC = K / 16, NTK = K / 32, niter = ((KQ ? NTK : NC) + 31) / 32;
    const int U = a.n_units;
    const int u0 = (int)((long long)U * blockIdx.x / gridDim.x);
    const int nu = (int)((long long)U * (blockIdx.x + 1) / gridDim.x) - u0;
    float4* act4 = reinterpret_cast<float4*>(sm_act);            // [(m * 4 + g) * NC + c]
    float* part = sm_act + (size_t)MB * K;                        // [(ul * NR + j) * niter + it][MB]

    auto load_pair = [&](int ul, int it, SChunk<WT> (&dst)[NR]) {
        const int u = u0 + ul, c = it * 32 + lane;
        int r[NR], wh[NR];
        unit_rows<EPI>(a, u, r, wh);
#pragma unroll
        for (int j = 0; j < NR; ++j) {
            const DevW& W = wh[j] ? a.w1 : a.w0;
            s_load<WT>(W, r[j], c, c < (KQ ? NTK : NC) && r[j] < W.rows, dst[j]);
        }
    };

    // weights do not depend on the previous kernel: start the stream first
    SChunk<WT> buf[P][NR];
    // pairs as (unit, item): stage s of a round holds pair base + 16 s; a
    // round advances the base by 16 P pairs (no divisions in the loop)
    const int q16 = S_WARPS / niter, r16 = S_WARPS % niter;
    auto step16 = [&](int& ul, int& it) {
        ul += q16;
        it += r16;
        if (it >= niter) {
            it -= niter;
            ul += 1;
        }
    };
    int bul = warp / niter, bit = warp % niter;   // this round's base pair
    {
        int ul = bul, it = bit;
#pragma unroll
        for (int s = 0; s < P; ++s) {
            if (ul < nu) load_pair(ul, it, buf[s]);
            step16(ul, it);
        }
    }
    pdl_launch();
    pdl_wait();
    if (EPI == EPI_ARGMAX && tid < MB) best[tid] = 0ull;
    if constexpr (EPI == EPI_QKV) {
        // NEOX cos/sin per (row, pair) with ggml's CPU theta recurrence, once per CTA
        const int half = a.hd / 2;
        for (int t = tid; t < MB * half; t += S_THREADS) {
            const int m = t / half, i = t % half;
            float th = (float)(a.rope_meta ? a.rope_meta : a.meta)[m].pos;   // true position (partitioned ranks shift meta.pos)
            for (int k = 0; k < i; ++k) th = __fmul_rn(th, a.rope_ts);
            rope_c[m][i] = cosf(th);
            rope_s[m][i] = sinf(th);
        }
    }
    // stage x (times the norm weight where the linear follows an RMSNorm)
    {
        float ss[MB];
#pragma unroll
        for (int m = 0; m < MB; ++m) ss[m] = 0.f;
        const int K4 = K / 4;
        for (int k4 = tid; k4 < K4; k4 += S_THREADS) {
            const int c = k4 >> 2, g = k4 & 3;
            const float4 w = a.norm_w ? __ldg(reinterpret_cast<const float4*>(a.norm_w) + k4)
                                      : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                float4 v = __ldcg(reinterpret_cast<const float4*>(a.x + (size_t)m * a.x_stride) + k4);
                if (a.norm_w) {
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
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) red[m * S_WARPS + warp] = t;
        }
    }
    __syncthreads();

    // main loop: pair warp + (n + s) * 16 sits in register stage s
    while (bul < nu) {
        int ul = bul, it = bit;                 // pair of stage s
        int nul = bul, nit = bit;               // pair of stage s in the next round
#pragma unroll
        for (int s = 0; s < P; ++s) step16(nul, nit);
        bul = nul;
        bit = nit;
#pragma unroll
        for (int s = 0; s < P; ++s) {
            if (ul < nu) {
                const int c = it * 32 + lane;
                float acc[NV];
#pragma unroll
                for (int i = 0; i < NV; ++i) acc[i] = 0.f;
                if constexpr (KQ) {
                    if (c < NTK) {
                        // lane task c: two 16-weight chunks (its two groups)
#pragma unroll
                        for (int sc2 = 0; sc2 < 2; ++sc2) {
                            const int ch = (c >> 3) * 16 + gd::kq_chunk0<WT>(c) + sc2 * gd::kq_chunk_step<WT>();
                            float4 av[MB][4];
#pragma unroll
                            for (int m = 0; m < MB; ++m)
#pragma unroll
                                for (int g = 0; g < 4; ++g) av[m][g] = act4[(m * 4 + g) * NC + ch];
#pragma unroll
                            for (int j = 0; j < NR; ++j) {
                                float o[MB];
                                kq_dot<WT, MB>(buf[s][j], av, c, sc2, o);
#pragma unroll
                                for (int m = 0; m < MB; ++m) acc[j * MB + m] += o[m];
                            }
                        }
                    }
                } else if (c < NC) {
                    float4 av[MB][4];
#pragma unroll
                    for (int m = 0; m < MB; ++m)
#pragma unroll
                        for (int g = 0; g < 4; ++g) av[m][g] = act4[(m * 4 + g) * NC + c];
#pragma unroll
                    for (int j = 0; j < NR; ++j) {
                        float o[MB];
                        s_dot<WT, MB>(buf[s][j], av, o);
#pragma unroll
                        for (int m = 0; m < MB; ++m) acc[j * MB + m] = o[m];
                    }
                }
                // the stage is free: request its pair of the next round
                if (nul < nu) load_pair(nul, nit, buf[s]);
                const float v = s_transpose_sum<NV>(acc, lane);
                if ((lane & ((1 << SH) - 1)) == 0) {
                    const int idx = lane >> SH, j = idx / MB, m = idx % MB;
                    part[((size_t)(ul * NR + j) * niter + it) * MB + m] = v;
                }
            }
            step16(ul, it);
            step16(nul, nit);
        }
    }
    __syncthreads();

    // ---- epilogue: per-row sums in item order, RMSNorm scale, fused op
    float nsc[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) {
        nsc[m] = 1.f;
        if (a.norm_w) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < S_WARPS; ++w) t += red[m * S_WARPS + w];
            nsc[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), a.eps)));
        }
    }
    auto rowsum = [&](int ul, int j, int m) {
        const float* pp = part + (size_t)(ul * NR + j) * niter * MB + m;
        float v = 0.f;
        for (int it = 0; it < niter; ++it) v += pp[it * MB];
        return a.norm_w ? __fmul_rn(v, m == 0 ? nsc[0] : nsc[MB - 1]) : v;
    };
    if constexpr (EPI == EPI_QKV || EPI == EPI_SWIGLU) {
        // thread: (unit, pair jp in {0, 1}, row m); partners are unit rows jp and jp + 2
        for (int t = tid; t < nu * 2 * MB; t += S_THREADS) {
            const int m = t % MB, jp = (t / MB) & 1, ul = t / (2 * MB);
            const int u = u0 + ul;
            int row[NR], which[NR];
            unit_rows<EPI>(a, u, row, which);
            float v0 = rowsum(ul, jp, m), v1 = rowsum(ul, jp + 2, m);
            if constexpr (EPI == EPI_SWIGLU) {
                if (row[jp] < a.w0.rows) a.y[(size_t)m * a.y_stride + row[jp]] = __fmul_rn(silu_ref(v0), v1);
            } else {
                if (a.bias) {
                    v0 = __fadd_rn(v0, a.bias[row[jp]]);
                    v1 = __fadd_rn(v1, a.bias[row[jp + 2]]);
                }
                const int h = row[jp] / a.hd, i2 = row[jp] % a.hd;
                const RowMeta rm = a.meta[m];
                if (h < a.n_q_heads + a.n_kv_heads) {
                    const float cc = rope_c[m][i2], sn = rope_s[m][i2];
                    const float y0 = __fsub_rn(__fmul_rn(v0, cc), __fmul_rn(v1, sn));
                    const float y1 = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cc));
                    v0 = y0;
                    v1 = y1;
                }
                if (h < a.n_q_heads) {
                    float* q = a.y + (size_t)m * a.y_stride + h * a.hd;
                    q[i2] = v0;
                    q[i2 + a.hd / 2] = v1;
                } else if (rm.cidx >= 0) {   // cidx < 0: another rank stores this position
                    const bool is_k = h < a.n_q_heads + a.n_kv_heads;
                    const int kvh = is_k ? h - a.n_q_heads : h - a.n_q_heads - a.n_kv_heads;
                    __half* dst = (is_k ? a.kv.k : a.kv.v) + kv_offset(a.kv, rm.seq, rm.cidx, kvh);
                    dst[i2] = __float2half_rn(v0);
                    dst[i2 + a.hd / 2] = __float2half_rn(v1);
                }
            }
        }
    } else {
        for (int t = tid; t < nu * NR * MB; t += S_THREADS) {
            const int m = t % MB, j = (t / MB) % NR, ul = t / (NR * MB);
            const int row = (u0 + ul) * NR + j;
            if (row >= a.w0.rows) continue;
            float v = rowsum(ul, j, m);
            if constexpr (EPI == EPI_ARGMAX) {
                if (a.y) a.y[(size_t)m * a.y_stride + row] = v;
                atomicMax(&best[m], argmax_key(v, row));
            } else {
                if (a.bias) v = __fadd_rn(v, a.bias[row]);
                float* dst = a.y + (size_t)m * a.y_stride + row;
                if (EPI == EPI_RESID) *dst = __fadd_rn(*dst, v);   // ggml_add(x, o)
                else *dst = v;
            }
        }
        if constexpr (EPI == EPI_ARGMAX) {
            __syncthreads();
            if (tid < MB && best[tid]) atomicMax(a.argmax + tid, best[tid]);
        }
    }
}

size_t stream_smem(const GemvArgs& a, int grid) {
    const bool kq = a.w0.type == W_Q5_K || a.w0.type == W_Q6_K;   // 32-weight lane tasks
    const int niter = ((kq ? a.K / 32 : a.K / 16) + 31) / 32;
    const int nu_max = (a.n_units + grid - 1) / grid;
    return (size_t)a.M * a.K * sizeof(float) + (size_t)nu_max * NR * niter * a.M * sizeof(float);
}

template <int WT, int EPI>
cudaError_t launch_t(const GemvArgs& a, cudaStream_t st) {
    const size_t smem = (size_t)a.M * a.K * sizeof(float);
    if (smem > GEMV_SMEM_MAX) return cudaErrorInvalidValue;
    // persistent grid: one wave of resident CTAs at most
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    if (a.M <= 2) {
        // one or two rows: the streaming kernel, one CTA per SM
        const int grid = a.n_units < sms ? a.n_units : sms;
        const size_t ssm = stream_smem(a, grid);
        if (grid > 0 && ssm <= S_SMEM_MAX) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(grid);
            cfg.blockDim = dim3(SThreads<WT>::v);
            cfg.dynamicSmemBytes = ssm;
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            cudaError_t e = a.M == 1 ? cudaLaunchKernelEx(&cfg, k_gemv_stream<WT, EPI, 1>, a)
                                     : cudaLaunchKernelEx(&cfg, k_gemv_stream<WT, EPI, 2>, a);
            note_launch();
            return e;
        }
    }
    GemvArgs b = a;
    const int niter = (a.K / 16 + 31) / 32;
    b.wpu = 1;
    while (b.wpu * 2 <= GEMV_WARPS && b.wpu * 2 <= niter) b.wpu *= 2;   // warps per unit <= items per row
    const int upc = GEMV_WARPS / b.wpu;
    const int n_groups = (a.n_units + upc - 1) / upc;
    int per_sm = 1;
    if (a.M <= 2) cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_gemv<WT, EPI, 2>, GEMV_THREADS, smem);
    else cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_gemv<WT, EPI, GEMV_MAX_M>, GEMV_THREADS, smem);
    const int cap = sms * (per_sm > 0 ? per_sm : 1);
    const int grid = n_groups < cap ? n_groups : cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = a.M <= 2 ? cudaLaunchKernelEx(&cfg, k_gemv<WT, EPI, 2>, b)
                             : cudaLaunchKernelEx(&cfg, k_gemv<WT, EPI, GEMV_MAX_M>, b);
    note_launch();
    return e;
}

template <int EPI>
cudaError_t launch_wt(const GemvArgs& a, cudaStream_t st) {
    switch (a.w0.type) {
        case W_Q8_0: return launch_t<W_Q8_0, EPI>(a, st);
        case W_Q5_K: return launch_t<W_Q5_K, EPI>(a, st);
        case W_Q6_K: return launch_t<W_Q6_K, EPI>(a, st);
        case W_F32: return launch_t<W_F32, EPI>(a, st);
        case W_F16: return launch_t<W_F16, EPI>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

template <int EPI>
cudaError_t prepare_wt() {
    const void* fns[] = {(const void*)k_gemv<W_Q8_0, EPI, 2>, (const void*)k_gemv<W_Q5_K, EPI, 2>,
                         (const void*)k_gemv<W_Q6_K, EPI, 2>, (const void*)k_gemv<W_F32, EPI, 2>,
                         (const void*)k_gemv<W_F16, EPI, 2>,
                         (const void*)k_gemv<W_Q8_0, EPI, GEMV_MAX_M>, (const void*)k_gemv<W_Q5_K, EPI, GEMV_MAX_M>,
                         (const void*)k_gemv<W_Q6_K, EPI, GEMV_MAX_M>, (const void*)k_gemv<W_F32, EPI, GEMV_MAX_M>,
                         (const void*)k_gemv<W_F16, EPI, GEMV_MAX_M>};
    for (const void* f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMV_SMEM_MAX);
        if (e != cudaSuccess) return e;
    }
    const void* sfns[] = {(const void*)k_gemv_stream<W_Q8_0, EPI, 1>, (const void*)k_gemv_stream<W_Q8_0, EPI, 2>,
                          (const void*)k_gemv_stream<W_Q5_K, EPI, 1>, (const void*)k_gemv_stream<W_Q5_K, EPI, 2>,
                          (const void*)k_gemv_stream<W_Q6_K, EPI, 1>, (const void*)k_gemv_stream<W_Q6_K, EPI, 2>,
                          (const void*)k_gemv_stream<W_F32, EPI, 1>, (const void*)k_gemv_stream<W_F32, EPI, 2>,
                          (const void*)k_gemv_stream<W_F16, EPI, 1>, (const void*)k_gemv_stream<W_F16, EPI, 2>};
    for (const void* f : sfns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S_SMEM_MAX);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

size_t gemv_smem_bytes(int wt, int M, int K) {
    (void)wt;
    return (size_t)M * K * sizeof(float);
}

int gemv_max_rows(int K) {
    const int m = (int)(GEMV_SMEM_MAX / ((size_t)K * sizeof(float)));
    return m < GEMV_MAX_M ? m : GEMV_MAX_M;
}

// Opt every instantiation in to large dynamic shared memory once per device,
// before any launch or stream capture.
cudaError_t gemv_prepare() {
    cudaError_t e;
    if ((e = prepare_wt<EPI_QKV>()) != cudaSuccess) return e;
    if ((e = prepare_wt<EPI_SWIGLU>()) != cudaSuccess) return e;
    if ((e = prepare_wt<EPI_RESID>()) != cudaSuccess) return e;
    if ((e = prepare_wt<EPI_STORE>()) != cudaSuccess) return e;
    return prepare_wt<EPI_ARGMAX>();
}

cudaError_t gemv_launch(GemvArgs a, cudaStream_t st) {
    if (a.M < 1 || a.M > GEMV_MAX_M || a.K % 16) return cudaErrorInvalidValue;
    if (a.w0.type == W_Q8_0 && a.K % 32) return cudaErrorInvalidValue;
    if ((a.w0.type == W_Q5_K || a.w0.type == W_Q6_K) && a.K % 256) return cudaErrorInvalidValue;
    switch (a.epi) {
        case EPI_QKV:
            if (a.hd % 4) return cudaErrorInvalidValue;
            a.n_units = a.w0.rows / 4;
            return launch_wt<EPI_QKV>(a, st);
        case EPI_SWIGLU:
            if (a.w0.rows % 2) return cudaErrorInvalidValue;
            a.n_units = a.w0.rows / 2;
            return launch_wt<EPI_SWIGLU>(a, st);
        case EPI_RESID:
            a.n_units = (a.w0.rows + NR - 1) / NR;
            return launch_wt<EPI_RESID>(a, st);
        case EPI_STORE:
            a.n_units = (a.w0.rows + NR - 1) / NR;
            return launch_wt<EPI_STORE>(a, st);
        case EPI_ARGMAX:
            a.n_units = (a.w0.rows + NR - 1) / NR;
            return launch_wt<EPI_ARGMAX>(a, st);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace vvq2
