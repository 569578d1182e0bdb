// gemv_dev.cuh -- device helpers shared by the decode GEMV kernels: loading
// one 16-element chunk of a repacked weight row and expanding it to the exact
// dequantized f32 values (bit-identical with ggml's dequantize_row_*).
#pragma once

#include "common.cuh"

namespace vvq2 {
namespace gd {

// One 16-element chunk of one weight row, as loaded (raw bits + block scales).
struct Chunk {
    uint4 r0, r1, r2, r3;   // raw: Q8_0 q in r0; Q5_K qs/qh in r0/r1; Q6_K ql/qh in r0/r1;
                            // F16 in r0/r1; F32 in r0..r3
    float scale;            // Q8_0 d; Q5_K d*sc; Q6_K d*sc
    float mscale;           // Q5_K dmin*m
    int shift;              // Q5_K sub-block j; Q6_K quarter k
};

template <int WT>
__device__ __forceinline__ void load_chunk(const DevW& W, int row, int c, Chunk& ch) {
    const uint8_t* rp = W.q + (size_t)row * W.row_stride;
    if constexpr (WT == W_Q8_0) {
        ch.r0 = __ldg(reinterpret_cast<const uint4*>(rp) + c);
        ch.scale = __half2float(W.d[(size_t)row * W.d_stride + c / 2]);
    } else if constexpr (WT == W_Q5_K) {
        const int sb = c >> 4, e0 = (c & 15) * 16, j = e0 / 32, l0 = e0 & 31;
        const uint8_t* b = rp + (size_t)sb * Q5K_BYTES;
        const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(b));
        ch.r0 = __ldg(reinterpret_cast<const uint4*>(b + 48 + 32 * (j >> 1) + l0));
        ch.r1 = __ldg(reinterpret_cast<const uint4*>(b + 16 + l0));
        const uint8_t* scb = reinterpret_cast<const uint8_t*>(&hdr) + 4;
        int sc, m;
        if (j < 4) {
            sc = scb[j] & 63;
            m = scb[j + 4] & 63;
        } else {
            sc = (scb[j + 4] & 0xF) | ((scb[j - 4] >> 6) << 4);
            m = (scb[j + 4] >> 4) | ((scb[j] >> 6) << 4);
        }
        const __half2 dh = *reinterpret_cast<const __half2*>(&hdr.x);
        ch.scale = __fmul_rn(__low2float(dh), (float)sc);    // d1 = d*sc   (dequantize_row_q5_K)
        ch.mscale = __fmul_rn(__high2float(dh), (float)m);   // m1 = dmin*m
        ch.shift = j;
    } else if constexpr (WT == W_Q6_K) {
        const int sb = c >> 4, e0 = (c & 15) * 16;
        const int hf = e0 >> 7, r = e0 & 127, k = r >> 5, l0 = r & 31;
        const uint8_t* b = rp + (size_t)sb * Q6K_PACKED;
        ch.r0 = __ldg(reinterpret_cast<const uint4*>(b + hf * 64 + (k & 1) * 32 + l0));
        ch.r1 = __ldg(reinterpret_cast<const uint4*>(b + 128 + hf * 32 + l0));
        const int8_t sc = reinterpret_cast<const int8_t*>(b + 192)[hf * 8 + (l0 >> 4) + 2 * k];
        ch.scale = __fmul_rn(__half2float(W.d[(size_t)row * W.d_stride + sb]), (float)sc);  // d*sc
        ch.shift = k;
    } else if constexpr (WT == W_F16) {
        const uint4* p = reinterpret_cast<const uint4*>(rp) + 2 * c;
        ch.r0 = __ldg(p);
        ch.r1 = __ldg(p + 1);
    } else {
        const uint4* p = reinterpret_cast<const uint4*>(rp) + 4 * c;
        ch.r0 = __ldg(p);
        ch.r1 = __ldg(p + 1);
        ch.r2 = __ldg(p + 2);
        ch.r3 = __ldg(p + 3);
    }
}

__device__ __forceinline__ uint32_t word(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

// Dequantized weights g*4 .. g*4+3 of the chunk, bit-exact with ggml's
// dequantize_row_*: Q8_0 q*d; Q5_K d1*q - m1; Q6_K (d*sc)*(q-32); F16/F32 as is.
template <int WT>
__device__ __forceinline__ void expand4(const Chunk& ch, int g, float* w) {
    if constexpr (WT == W_Q8_0) {
        const uint32_t q = word(ch.r0, g);
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = __fmul_rn((float)((int)((q >> (8 * e)) & 0xff) - 128), ch.scale);   // q + 128 stored
    } else if constexpr (WT == W_Q5_K) {
        const int j = ch.shift;
        const uint32_t q = ((word(ch.r0, g) >> (4 * (j & 1))) & 0x0F0F0F0Fu) |
                           (((word(ch.r1, g) >> j) & 0x01010101u) << 4);
#pragma unroll
        for (int e = 0; e < 4; ++e)
            w[e] = __fsub_rn(__fmul_rn(ch.scale, (float)((q >> (8 * e)) & 0xff)), ch.mscale);
    } else if constexpr (WT == W_Q6_K) {
        const int k = ch.shift;
        const uint32_t q = ((word(ch.r0, g) >> (4 * (k >> 1))) & 0x0F0F0F0Fu) |
                           (((word(ch.r1, g) >> (2 * k)) & 0x03030303u) << 4);
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = __fmul_rn(ch.scale, (float)((int)((q >> (8 * e)) & 0xff) - 32));
    } else if constexpr (WT == W_F16) {
        const uint4& v = g < 2 ? ch.r0 : ch.r1;
        const uint32_t a = word(v, (g & 1) * 2), b = word(v, (g & 1) * 2 + 1);
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&a));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&b));
        w[0] = f0.x; w[1] = f0.y; w[2] = f1.x; w[3] = f1.y;
    } else {
        const uint4& v = g == 0 ? ch.r0 : g == 1 ? ch.r1 : g == 2 ? ch.r2 : ch.r3;
        w[0] = __uint_as_float(v.x); w[1] = __uint_as_float(v.y);
        w[2] = __uint_as_float(v.z); w[3] = __uint_as_float(v.w);
    }
}

// L2 prefetch of one weight row (128-byte lines spread over the warp)
template <int WT>
__device__ __forceinline__ void prefetch_row(const DevW& W, int row, int lane, int nchunk) {
    (void)nchunk;
    const uint8_t* rp = W.q + (size_t)row * W.row_stride;
    for (int64_t off = (int64_t)lane * 128; off < W.row_stride; off += 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(rp + off));
}

// zero only the fields the type uses, so unused ones stay dead in registers
template <int WT>
__device__ __forceinline__ void clear_chunk(Chunk& ch) {
    ch.r0 = make_uint4(0, 0, 0, 0);
    if constexpr (WT != W_Q8_0) ch.r1 = make_uint4(0, 0, 0, 0);
    if constexpr (WT == W_F32) ch.r2 = ch.r3 = make_uint4(0, 0, 0, 0);
    if constexpr (WT == W_Q8_0 || WT == W_Q5_K || WT == W_Q6_K) ch.scale = 0.f;
    if constexpr (WT == W_Q5_K) ch.mscale = 0.f;
    if constexpr (WT == W_Q5_K || WT == W_Q6_K) ch.shift = 0;
}

// ---------------------------------------------------------------------------
// K-quant lane tasks of 32 weights (the streaming GEMV's K-quant mapping).
// A lane task covers 16 consecutive positions l0 .. l0+15 of two 32-weight
// groups of one super-block that share their low-bit bytes, so one 16-byte
// run of low bits and one of high bits serve all 32 weights:
//   Q6_K task t (8 per super-block): half hf = (t & 7) >> 2, quarter pair
//     kk = ((t & 7) >> 1) & 1 (quarters kk and kk + 2: low / high nibbles of
//     ql[hf*64 + kk*32 + l], high bits 2k..2k+1 of qh[hf*32 + l]),
//     l0 = 16 * (t & 1); weights hf*128 + k*32 + l.
//   Q5_K task t: sub-block pair q = (t & 7) >> 1 (sub-blocks 2q and 2q + 1:
//     low / high nibbles of qs[32q + l], bit j of qh[l]), l0 = 16 * (t & 1);
//     weights j*32 + l.
// Sub-chunk s (0, 1) of a task is its first / second group; kq_word gives
// its four quants of 32-bit word g (positions l0 + 4g .. l0 + 4g + 3) as
// bytes: Q6_K q in 0..63 (value (q - 32) * d * sc), Q5_K q in 0..31 (value
// d * sc * q - dmin * m).  These are the bit layouts of ggml's
// dequantize_row_q6_K / dequantize_row_q5_K.

// first 16-weight chunk (of 16) of task t within its super-block, and the
// chunk distance to the task's second group
template <int WT>
__host__ __device__ __forceinline__ int kq_chunk0(int t) {
    const int sub = t & 7, l16 = sub & 1;
    if constexpr (WT == W_Q6_K) return (sub >> 2) * 8 + ((sub >> 1) & 1) * 2 + l16;
    else return (sub >> 1) * 4 + l16;
}
template <int WT>
__host__ __device__ __forceinline__ constexpr int kq_chunk_step() { return WT == W_Q6_K ? 4 : 2; }

// byte offsets (within the super-block) of the task's low-bit and high-bit runs
template <int WT>
__host__ __device__ __forceinline__ int kq_lo_off(int t) {
    const int sub = t & 7, l0 = (sub & 1) * 16;
    if constexpr (WT == W_Q6_K) return (sub >> 2) * 64 + ((sub >> 1) & 1) * 32 + l0;
    else return 48 + (sub >> 1) * 32 + l0;
}
template <int WT>
__host__ __device__ __forceinline__ int kq_hi_off(int t) {
    const int sub = t & 7, l0 = (sub & 1) * 16;
    if constexpr (WT == W_Q6_K) return 128 + (sub >> 2) * 32 + l0;
    else return 16 + l0;
}

// quants of sub-chunk s, word g: lo / hi are the task's low-bit / high-bit words g
template <int WT>
__host__ __device__ __forceinline__ uint32_t kq_word(uint32_t lo, uint32_t hi, int t, int s) {
    const int sub = t & 7;
    if constexpr (WT == W_Q6_K) {
        const int k = ((sub >> 1) & 1) + 2 * s;          // quarter
        return ((lo >> (4 * s)) & 0x0F0F0F0Fu) | (((hi >> (2 * k)) & 0x03030303u) << 4);
    } else {
        const int j = (sub >> 1) * 2 + s;                // sub-block
        return ((lo >> (4 * s)) & 0x0F0F0F0Fu) | (((hi >> j) & 0x01010101u) << 4);
    }
}

// Q6_K: index of the int8 scale of sub-chunk s within the half's 8 scales
__host__ __device__ __forceinline__ int q6_scale_idx(int t, int s) {
    const int sub = t & 7;
    return (sub & 1) + 2 * (((sub >> 1) & 1) + 2 * s);
}

// Q5_K: 6-bit scale and min of sub-block j from the 12 packed bytes (ggml's get_scale_min_k4)
__host__ __device__ __forceinline__ void q5_scale_min(const uint8_t* scb, int j, int& sc, int& m) {
    if (j < 4) {
        sc = scb[j] & 63;
        m = scb[j + 4] & 63;
    } else {
        sc = (scb[j + 4] & 0xF) | ((scb[j - 4] >> 6) << 4);
        m = (scb[j + 4] >> 4) | ((scb[j] >> 6) << 4);
    }
}

}  // namespace gd
}  // namespace vvq2
