// dequant.cuh -- element dequantization of the repacked device weight formats.
//
// Each routine reproduces ggml's dequantize_row_* arithmetic exactly (same
// operand order, no FMA contraction), so the f32 values are bit-identical to
// ggml's and to gguf-py's numpy dequantizers:
//   Q8_0 : y = q * d                                   (dequantize_row_q8_0)
//   Q5_K : y = (d*sc) * q - (dmin*m), q = nibble | hb<<4 (dequantize_row_q5_K)
//   Q6_K : y = (d*sc) * (q - 32), q = nibble | 2b<<4     (dequantize_row_q6_K)
#pragma once

#include "common.cuh"

namespace vvq2 {

__device__ __forceinline__ float deq_elem(const DevW& w, int row, int e) {
    switch (w.type) {
        case W_Q8_0: {
            const int q = (int)(w.q + (size_t)row * w.row_stride)[e] - 128;   // stored biased: q + 128
            const float d = __half2float(w.d[(size_t)row * w.d_stride + e / 32]);
            return __fmul_rn((float)q, d);
        }
        case W_Q5_K: {
            const uint8_t* b = w.q + (size_t)row * w.row_stride + (size_t)(e / 256) * Q5K_BYTES;
            const int r = e % 256, c = r / 64, l = r % 64;
            const int sub = 2 * c + (l >= 32), li = l % 32;
            const uint8_t* sc = b + 4;
            int s, m;
            if (sub < 4) {
                s = sc[sub] & 63;
                m = sc[sub + 4] & 63;
            } else {
                s = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4);
                m = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
            }
            const uint8_t qsb = b[48 + 32 * c + li], qhb = b[16 + li];
            const int q = ((qsb >> (4 * (sub & 1))) & 0xF) + (((qhb >> sub) & 1) ? 16 : 0);
            const __half2 dh = *reinterpret_cast<const __half2*>(b);
            const float d1 = __fmul_rn(__low2float(dh), (float)s);
            const float m1 = __fmul_rn(__high2float(dh), (float)m);
            return __fsub_rn(__fmul_rn(d1, (float)q), m1);
        }
        case W_Q6_K: {
            const int sb = e / 256;
            const uint8_t* b = w.q + (size_t)row * w.row_stride + (size_t)sb * Q6K_PACKED;
            const int r = e % 256, hf = r / 128, k = (r % 128) / 32, l = r % 32;
            const uint8_t qlb = b[hf * 64 + (k & 1) * 32 + l];
            const uint8_t qhb = b[128 + hf * 32 + l];
            const int q = (int)(((qlb >> (4 * (k >> 1))) & 0xF) | (((qhb >> (2 * k)) & 3) << 4)) - 32;
            const int8_t sc = reinterpret_cast<const int8_t*>(b + 192)[hf * 8 + l / 16 + 2 * k];
            const float d = __half2float(w.d[(size_t)row * w.d_stride + sb]);
            return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
        }
        case W_F16:
            return __half2float(reinterpret_cast<const __half*>(w.q + (size_t)row * w.row_stride)[e]);
        default:
            return reinterpret_cast<const float*>(w.q + (size_t)row * w.row_stride)[e];
    }
}

}  // namespace vvq2
