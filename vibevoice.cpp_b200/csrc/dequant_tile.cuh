// dequant_tile.cuh -- weight producers of the tensor-core GEMMs: GGUF
// blocks (Q8_0 / Q5_K / Q6_K, or f16 / f32) to the f16 operand tile the UMMA
// descriptor reads, K-major with the 128-byte swizzle (row p of a tile is 128
// bytes = 64 K elements; its 16-byte chunk j sits at chunk j ^ (p & 7)).
// Values are ggml's dequantize_row_* results (exact in f32) rounded once to
// f16 (ggml-quants.c dequantize_row_q8_0 / _q5_K / _q6_K).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "dequant.cuh"

namespace vvq2 {
__device__ __forceinline__ void store_chunk(uint8_t* btile, int p, int j, uint4 v) {
    *reinterpret_cast<uint4*>(btile + p * 128 + ((j ^ (p & 7)) * 16)) = v;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t wsel(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

// Dequantize elements [k0, k0 + 64) of weight row `row` into 8 swizzled
// 16-byte chunks of row p of the B tile (exact ggml values, then f16 RNE).
template <int WT>
__device__ __forceinline__ void produce_row(const DevW& W, int row, int k0, uint8_t* btile, int p) {
    if (row < 0 || row >= W.rows) {
#pragma unroll
        for (int j = 0; j < 8; ++j) store_chunk(btile, p, j, make_uint4(0, 0, 0, 0));
        return;
    }
    const uint8_t* rp = W.q + (size_t)row * W.row_stride;
    if constexpr (WT == W_Q8_0) {
        const uint4* qp = reinterpret_cast<const uint4*>(rp + k0);
        uint4 q[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = __ldg(qp + i);
        const __half2 dd = *reinterpret_cast<const __half2*>(W.d + (size_t)row * W.d_stride + k0 / 32);
        const float d0 = __low2float(dd), d1 = __high2float(dd);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float d = j < 4 ? d0 : d1;
            const uint32_t w0 = wsel(q[j / 2], (j % 2) * 2), w1 = wsel(q[j / 2], (j % 2) * 2 + 1);
            uint4 o;
            o.x = pack_h2(__fmul_rn((float)((int)(w0 & 0xff) - 128), d), __fmul_rn((float)((int)((w0 >> 8) & 0xff) - 128), d));
            o.y = pack_h2(__fmul_rn((float)((int)((w0 >> 16) & 0xff) - 128), d), __fmul_rn((float)((int)(w0 >> 24) - 128), d));
            o.z = pack_h2(__fmul_rn((float)((int)(w1 & 0xff) - 128), d), __fmul_rn((float)((int)((w1 >> 8) & 0xff) - 128), d));
            o.w = pack_h2(__fmul_rn((float)((int)((w1 >> 16) & 0xff) - 128), d), __fmul_rn((float)((int)(w1 >> 24) - 128), d));
            store_chunk(btile, p, j, o);
        }
    } else if constexpr (WT == W_Q5_K) {
        const int sb = k0 / 256, qq = (k0 % 256) / 64;    // 64-element chunk qq of the super-block
        const uint8_t* b = rp + (size_t)sb * Q5K_BYTES;
        const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(b));
        uint4 qs[2], qh[2];
        qs[0] = __ldg(reinterpret_cast<const uint4*>(b + 48 + 32 * qq));
        qs[1] = __ldg(reinterpret_cast<const uint4*>(b + 48 + 32 * qq) + 1);
        qh[0] = __ldg(reinterpret_cast<const uint4*>(b + 16));
        qh[1] = __ldg(reinterpret_cast<const uint4*>(b + 16) + 1);
        const uint8_t* scb = reinterpret_cast<const uint8_t*>(&hdr) + 4;
        const __half2 dh = *reinterpret_cast<const __half2*>(&hdr.x);
        float d1[2], m1[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * qq + h;
            int s, m;
            if (j < 4) {
                s = scb[j] & 63;
                m = scb[j + 4] & 63;
            } else {
                s = (scb[j + 4] & 0xF) | ((scb[j - 4] >> 6) << 4);
                m = (scb[j + 4] >> 4) | ((scb[j] >> 6) << 4);
            }
            d1[h] = __fmul_rn(__low2float(dh), (float)s);
            m1[h] = __fmul_rn(__high2float(dh), (float)m);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int h = j / 4;                 // first or second 32 elements
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int l = (j % 4) * 8 + e;   // 0..31 within the sub-block
                const uint32_t qsw = wsel(qs[l / 16], (l % 16) / 4), qhw = wsel(qh[l / 16], (l % 16) / 4);
                const int qb = (qsw >> (8 * (l % 4))) & 0xff, hb = (qhw >> (8 * (l % 4))) & 0xff;
                const int q = ((qb >> (4 * h)) & 0xF) + (((hb >> (2 * qq + h)) & 1) ? 16 : 0);
                f[e] = __fsub_rn(__fmul_rn(d1[h], (float)q), m1[h]);
            }
            store_chunk(btile, p, j, make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]),
                                                pack_h2(f[6], f[7])));
        }
    } else if constexpr (WT == W_Q6_K) {
        const int sb = k0 / 256, qq = (k0 % 256) / 64, hf = qq >> 1, k0q = (qq & 1) * 2;
        const uint8_t* b = rp + (size_t)sb * Q6K_PACKED;
        uint4 ql[4], qh[2];
#pragma unroll
        for (int i = 0; i < 4; ++i) ql[i] = __ldg(reinterpret_cast<const uint4*>(b + hf * 64) + i);
        qh[0] = __ldg(reinterpret_cast<const uint4*>(b + 128 + hf * 32));
        qh[1] = __ldg(reinterpret_cast<const uint4*>(b + 128 + hf * 32) + 1);
        const int8_t* scl = reinterpret_cast<const int8_t*>(b + 192);
        const float dsb = __half2float(W.d[(size_t)row * W.d_stride + sb]);
        float ds[4];   // (k - k0q) * 2 + l/16
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) ds[kk * 2 + hh] = __fmul_rn(dsb, (float)scl[hf * 8 + hh + 2 * (k0q + kk)]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int kk = j / 4;                // quarter k = k0q + kk
            const int k = k0q + kk;
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int l = (j % 4) * 8 + e;   // 0..31
                const int qlbyte_idx = (k & 1) * 32 + l;   // within the 64 ql bytes of this half
                const uint32_t lw = wsel(ql[qlbyte_idx / 16], (qlbyte_idx % 16) / 4);
                const uint32_t hw = wsel(qh[l / 16], (l % 16) / 4);
                const int lb = (lw >> (8 * (qlbyte_idx % 4))) & 0xff, hb = (hw >> (8 * (l % 4))) & 0xff;
                const int q = (int)(((lb >> (4 * (k >> 1))) & 0xF) | (((hb >> (2 * k)) & 3) << 4)) - 32;
                f[e] = __fmul_rn(ds[kk * 2 + l / 16], (float)q);
            }
            store_chunk(btile, p, j, make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]),
                                                pack_h2(f[6], f[7])));
        }
    } else if constexpr (WT == W_F16) {
        const uint4* hp = reinterpret_cast<const uint4*>(rp + (size_t)k0 * 2);
#pragma unroll
        for (int j = 0; j < 8; ++j) store_chunk(btile, p, j, __ldg(hp + j));
    } else {
        const float4* fp = reinterpret_cast<const float4*>(rp + (size_t)k0 * 4);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 a = __ldg(fp + 2 * j), c = __ldg(fp + 2 * j + 1);
            store_chunk(btile, p, j, make_uint4(pack_h2(a.x, a.y), pack_h2(a.z, a.w), pack_h2(c.x, c.y),
                                                pack_h2(c.z, c.w)));
        }
    }
}

// Q8_0: 16 stored bytes (q + 128) of one block with its scale (f16 bits) to
// the two swizzled 16-byte chunks j0, j0 + 1 of a tile row (rowp: the row's
// 128 bytes, swz: its row index mod 8).  Exact f16 math: the byte in the
// mantissa of 1024, minus 1152, is q exactly; one f16 multiply by the block
// scale gives RN(q * d), the exact f32 product rounded to f16.
__device__ __forceinline__ void q8_0_chunk_pair(const uint4& v, unsigned short dbits, uint8_t* rowp, int swz, int j0) {
    const __half2 sc = __halves2half2(__ushort_as_half(dbits), __ushort_as_half(dbits));
    const __half2 off = __float2half2_rn(-1152.0f), one = __float2half2_rn(1.0f);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        uint32_t o[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t w = wsel(v, 2 * j + h);
            const uint32_t lo = __byte_perm(w, 0x64646464u, 0x5140);
            const uint32_t hi = __byte_perm(w, 0x64646464u, 0x7362);
            __half2 qlo = __hfma2(*reinterpret_cast<const __half2*>(&lo), one, off);
            __half2 qhi = __hfma2(*reinterpret_cast<const __half2*>(&hi), one, off);
            qlo = __hmul2(qlo, sc);
            qhi = __hmul2(qhi, sc);
            o[2 * h] = *reinterpret_cast<const uint32_t*>(&qlo);
            o[2 * h + 1] = *reinterpret_cast<const uint32_t*>(&qhi);
        }
        *reinterpret_cast<uint4*>(rowp + (((j0 + j) ^ swz) * 16)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

}  // namespace vvq2
