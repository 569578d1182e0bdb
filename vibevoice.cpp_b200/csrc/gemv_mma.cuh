// gemv_mma.cuh -- decode-size (1-2 rows) Q8_0 matrix-vector products on the
// tensor cores (mma.sync m16n8k32, u8 x s8 -> s32), with the exact dequantized
// weights and f32-grade activations.
//
// Weights: the device Q8_0 layout (quants stored biased, q + 128, as u8; f16
// block scale d).  Their exact value is q * d.
//
// Activations: each 32-element block of a row is written as three int8
// pieces with a power-of-two block scale s:
//     x = s * (a0 + a1 / 2^7 + a2 / 2^14 + r),  |r| <= 2^-15
// a0 = rint(x / s) with s the smallest power of two >= max|x| / 127 (so
// |a0| <= 127), a1 = rint(128 (x/s - a0)), a2 = rint(128 (128 (x/s - a0) - a1))
// (|a1|, |a2| <= 64).  Every step is exact in f32 (power-of-two scaling,
// subtraction of an integer from a value within 0.5 of it), so the only error
// is the final residual: 2^-15 s, i.e. about 2^-22 of the block's max |x| --
// the f32 rounding level.
//
// One MMA per 32-wide block multiplies 16 weight rows by the 8 columns
// (row m, piece p) = column 3m + p; the s32 sums are exact.  Per block the
// bias of the stored quants is removed with the integer correction
// 128 * sum_k a_p[k], and the block's contribution
//     d[row] * s[m] * 2^-7p * (sum - corr)
// is added in f32.  The three pieces of a row are added at the end.
//
// Fragment layout (m16n8k32, row.col): lane (g = lane/4, t = lane%4) holds
// A rows g and g+8 at k = 4t..4t+3 and 16+4t..16+4t+3, B column g at the same
// k.  Both operands are read at the SAME physical bytes 8t..8t+7 of the block
// (as the A pair and the B pair), which is the k-permutation k' = 4t+i <->
// 8t+i, 16+4t+i <-> 8t+4+i applied to both; the dot product is unchanged.
#pragma once

#include "common.cuh"

namespace vvq2 {
namespace gm {

constexpr int NP = 3;          // activation pieces

__device__ __forceinline__ void mma_u8s8(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %11, %12, %13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Power-of-two block scale for max|x| = amax: the smallest 2^e with
// amax / 2^e < 127.5 (so rint keeps |a0| <= 127); 1 for an all-zero block.
__device__ __forceinline__ float block_scale(float amax) {
    if (!(amax > 0.f)) return 1.f;
    const int e = ((__float_as_uint(amax) >> 23) & 0xff) - 127;   // amax in [2^e, 2^(e+1))
    float s = __uint_as_float((uint32_t)(e - 6 + 127) << 23);      // 2^(e-6): amax / s in [64, 128)
    if (amax / s >= 127.5f) s = s * 2.f;
    return s;
}

// Pieces of one element (x / s exact).
__device__ __forceinline__ void pieces(float x, float inv_s, int& a0, int& a1, int& a2) {
    const float u = x * inv_s;                 // exact: inv_s is a power of two
    const float f0 = rintf(u);
    const float r1 = (u - f0) * 128.f;         // exact
    const float f1 = rintf(r1);
    const float r2 = (r1 - f1) * 128.f;        // exact
    a0 = (int)f0;
    a1 = (int)f1;
    a2 = (int)rintf(r2);
}

// Shared-memory operand of one activation row set: pieces [m][p][K + AQ_PAD]
// int8 (natural k order), block scales s [m][K/32] f32, corrections
// [m][p][K/32] s32 (128 * sum of the block's piece values).
constexpr int AQ_PAD = 32;     // row padding of the piece rows (spreads B loads over the banks)

struct ActQ {
    int8_t* q;                 // [MB][NP][K + AQ_PAD]
    float* s;                  // [MB][K/32]
    int* corr;                 // [MB][NP][K/32]
    int K;
};

__host__ __device__ constexpr int actq_bytes(int MB, int K) {
    return MB * NP * (K + AQ_PAD) + MB * (K / 32) * 4 + MB * NP * (K / 32) * 4;
}

__device__ __forceinline__ ActQ actq_at(uint8_t* base, int MB, int K) {
    ActQ a;
    a.K = K;
    a.q = reinterpret_cast<int8_t*>(base);
    a.s = reinterpret_cast<float*>(base + MB * NP * (K + AQ_PAD));
    a.corr = reinterpret_cast<int*>(base + MB * NP * (K + AQ_PAD) + MB * (K / 32) * 4);
    return a;
}

// Quantize the 4 elements v of float4-group i (elements 4i..4i+3 of row m,
// k4 = i % (K/4)) into the pieces.  The 8 groups of a 32-element block must
// sit on 8 consecutive lanes of the warp (lane & ~7 = the block), all 32
// lanes participating; `valid` false lanes contribute nothing.
__device__ __forceinline__ void quantize_group(const ActQ& aq, int m, int k4, float4 v, bool valid) {
    float amax = valid ? fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))) : 0.f;
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    const float s = block_scale(amax);
    const float inv = 1.0f / s;                // exact (power of two)
    int p0[4], p1[4], p2[4];
    pieces(v.x, inv, p0[0], p1[0], p2[0]);
    pieces(v.y, inv, p0[1], p1[1], p2[1]);
    pieces(v.z, inv, p0[2], p1[2], p2[2]);
    pieces(v.w, inv, p0[3], p1[3], p2[3]);
    int c0 = p0[0] + p0[1] + p0[2] + p0[3];
    int c1 = p1[0] + p1[1] + p1[2] + p1[3];
    int c2 = p2[0] + p2[1] + p2[2] + p2[3];
#pragma unroll
    for (int o = 1; o <= 4; o <<= 1) {
        c0 += __shfl_xor_sync(0xffffffffu, c0, o);
        c1 += __shfl_xor_sync(0xffffffffu, c1, o);
        c2 += __shfl_xor_sync(0xffffffffu, c2, o);
    }
    if (!valid) return;
    const int K = aq.K, stride = K + AQ_PAD;
    auto pack = [](const int (&p)[4]) {
        return (uint32_t)(p[0] & 0xff) | ((uint32_t)(p[1] & 0xff) << 8) | ((uint32_t)(p[2] & 0xff) << 16) |
               ((uint32_t)(p[3] & 0xff) << 24);
    };
    int8_t* row = aq.q + (size_t)m * NP * stride;
    *reinterpret_cast<uint32_t*>(row + 0 * stride + 4 * k4) = pack(p0);
    *reinterpret_cast<uint32_t*>(row + 1 * stride + 4 * k4) = pack(p1);
    *reinterpret_cast<uint32_t*>(row + 2 * stride + 4 * k4) = pack(p2);
    if ((k4 & 7) == 0) {
        const int b = k4 >> 3, nb = K / 32;
        aq.s[m * nb + b] = s;
        aq.corr[(m * NP + 0) * nb + b] = 128 * c0;
        aq.corr[(m * NP + 1) * nb + b] = 128 * c1;
        aq.corr[(m * NP + 2) * nb + b] = 128 * c2;
    }
}

// Partial products of up to 16 weight rows (tile rows row0 .. row0 + 15, rows
// >= nrows skipped; row stride rs bytes, quants then f16 scales at byte K)
// over blocks [b0, b1), for MB activation rows.  acc[i], lane (g, t):
// i = 0/1 rows g, columns 2t/2t+1; i = 2/3 row g + 8.  Column 3m + p.
template <int MB>
__device__ __forceinline__ void tile_mma(const uint8_t* tile, int rs, int K, int row0, int nrows, int b0, int b1,
                                         const ActQ& aq, int lane, float (&acc)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const int ra = row0 + g, rb = row0 + g + 8;
    const bool va = g < nrows, vb = g + 8 < nrows;
    const int c0 = 2 * t, c1 = 2 * t + 1;                // this lane's columns
    const bool vc0 = c0 < NP * MB, vc1 = c1 < NP * MB;
    const int bcol = g < NP * MB ? g : 0;               // this lane's B column (zero past the last)
    const bool vbcol = g < NP * MB;
    const int nb = K / 32, stride = K + AQ_PAD;
    const int8_t* brow = aq.q + (size_t)(bcol / NP) * NP * stride + (bcol % NP) * stride;
    const uint8_t* rowa = tile + (size_t)ra * rs;
    const uint8_t* rowb = tile + (size_t)rb * rs;
    const __half* da = reinterpret_cast<const __half*>(rowa + K);
    const __half* db = reinterpret_cast<const __half*>(rowb + K);
    // per-column piece scale 2^-7p and the scale / correction row of column c
    const float ps0 = c0 % NP == 0 ? 1.f : c0 % NP == 1 ? 0.0078125f : 6.103515625e-05f;
    const float ps1 = c1 % NP == 0 ? 1.f : c1 % NP == 1 ? 0.0078125f : 6.103515625e-05f;
    const float* s0 = aq.s + (vc0 ? c0 / NP : 0) * nb;
    const float* s1 = aq.s + (vc1 ? c1 / NP : 0) * nb;
    const int* cr0 = aq.corr + (vc0 ? c0 : 0) * nb;
    const int* cr1 = aq.corr + (vc1 ? c1 : 0) * nb;
    for (int b = b0; b < b1; ++b) {
        uint32_t a[4] = {0u, 0u, 0u, 0u};
        if (va) {
            const uint2 w = *reinterpret_cast<const uint2*>(rowa + 32 * b + 8 * t);
            a[0] = w.x;
            a[2] = w.y;
        }
        if (vb) {
            const uint2 w = *reinterpret_cast<const uint2*>(rowb + 32 * b + 8 * t);
            a[1] = w.x;
            a[3] = w.y;
        }
        uint2 bb = make_uint2(0u, 0u);
        if (vbcol) bb = *reinterpret_cast<const uint2*>(brow + 32 * b + 8 * t);
        int c[4];
        mma_u8s8(a, bb.x, bb.y, c);
        const float wa = va ? __half2float(da[b]) : 0.f;
        const float wb = vb ? __half2float(db[b]) : 0.f;
        const float f0 = vc0 ? s0[b] * ps0 : 0.f, f1 = vc1 ? s1[b] * ps1 : 0.f;
        const int k0 = vc0 ? cr0[b] : 0, k1 = vc1 ? cr1[b] : 0;
        acc[0] = fmaf((float)(c[0] - k0), wa * f0, acc[0]);
        acc[1] = fmaf((float)(c[1] - k1), wa * f1, acc[1]);
        acc[2] = fmaf((float)(c[2] - k0), wb * f0, acc[2]);
        acc[3] = fmaf((float)(c[3] - k1), wb * f1, acc[3]);
    }
}

}  // namespace gm
}  // namespace vvq2
