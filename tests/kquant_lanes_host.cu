// Host-side check of the streaming GEMV's K-quant lane mapping
// (vibevoice.cpp_b200/csrc/gemv_dev.cuh, kq_* helpers): reads one row of GGUF
// Q5_K / Q6_K blocks, decodes every weight through the lane tasks exactly as
// the kernel addresses them (task t -> chunk, byte runs, quant word, scale)
// and writes the dequantized row in element order.  Built and run by
// tests/test_kquant_lanes_cpu.py, which compares it with the oracle.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "gemv_dev.cuh"

using namespace vvq2;

static float h2f(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

template <int WT>
static void decode(const uint8_t* raw, int cols, float* out) {
    const int nb = cols / 256;
    const int bb = WT == W_Q6_K ? 210 : 176;
    for (int sb = 0; sb < nb; ++sb) {
        const uint8_t* b = raw + (size_t)sb * bb;   // GGUF block (Q6_K: ql|qh|scales|d, Q5_K: d|dmin|scales|qh|qs)
        for (int tt = 0; tt < 8; ++tt) {
            const int t = sb * 8 + tt;
            for (int s = 0; s < 2; ++s) {
                const int c = sb * 16 + gd::kq_chunk0<WT>(t) + s * gd::kq_chunk_step<WT>();
                float scale, mscale = 0.f;
                if constexpr (WT == W_Q6_K) {
                    const float d = h2f((uint16_t)(b[208] | (b[209] << 8)));
                    const int8_t sc = (int8_t)b[192 + ((t & 7) >> 2) * 8 + gd::q6_scale_idx(t, s)];
                    scale = d * (float)sc;
                } else {
                    const float d = h2f((uint16_t)(b[0] | (b[1] << 8))), dmin = h2f((uint16_t)(b[2] | (b[3] << 8)));
                    int sc, m;
                    gd::q5_scale_min(b + 4, ((t & 7) >> 1) * 2 + s, sc, m);
                    scale = d * (float)sc;
                    mscale = dmin * (float)m;
                }
                for (int g = 0; g < 4; ++g) {
                    uint32_t lo, hi;
                    memcpy(&lo, b + gd::kq_lo_off<WT>(t) + 4 * g, 4);
                    memcpy(&hi, b + gd::kq_hi_off<WT>(t) + 4 * g, 4);
                    const uint32_t w = gd::kq_word<WT>(lo, hi, t, s);
                    for (int e = 0; e < 4; ++e) {
                        const int q = (int)((w >> (8 * e)) & 0xff);
                        const int idx = c * 16 + 4 * g + e;
                        out[idx] = WT == W_Q6_K ? scale * (float)(q - 32) : scale * (float)q - mscale;
                    }
                }
            }
        }
    }
}

int main(int argc, char** argv) {
    if (argc != 5) return 2;
    const int qt = atoi(argv[1]), cols = atoi(argv[2]);
    const int bb = qt == W_Q6_K ? 210 : 176;
    std::vector<uint8_t> raw((size_t)cols / 256 * bb);
    FILE* f = fopen(argv[3], "rb");
    if (!f || fread(raw.data(), 1, raw.size(), f) != raw.size()) return 3;
    fclose(f);
    std::vector<float> out(cols, 0.f);
    if (qt == W_Q6_K) decode<W_Q6_K>(raw.data(), cols, out.data());
    else if (qt == W_Q5_K) decode<W_Q5_K>(raw.data(), cols, out.data());
    else return 4;
    f = fopen(argv[4], "wb");
    if (!f || fwrite(out.data(), 4, out.size(), f) != out.size()) return 5;
    fclose(f);
    return 0;
}
