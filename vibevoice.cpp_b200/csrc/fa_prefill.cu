// fa_prefill.cu -- causal flash attention for prefill chunks on the
// 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// softmax(Q K^T / sqrt(hd) + causal mask) V for a chunk of query rows
// against the f16 paged KV cache (the rows' own keys were appended by the QKV
// GEMM before this launch): ggml_flash_attn_ext with F32 precision,
// src/qwen2.cpp:327-335, causal mask src/vibevoice_tts.cpp:432-441.
//
// CTA = 128 query rows of one sequence x one q head (GQA: KV head h / G).
//   warp 0: TMA producer of 128-key K and V tiles (two 64-key pages each,
//           pages resolved through the block table, 128-byte swizzle)
//   warp 1: MMA issuer: S_j = Q K_j^T into one of two 128-column TMEM
//           buffers (Q read from TMEM); O += P_j V_j with P read from TMEM
//           and V from shared memory as an MN-major operand (no transpose)
//   warps 2-5: one query row per thread: Q staged as f16 into TMEM, then per
//           key tile the softmax from TMEM against a per-row reference max:
//           P = exp2((S - m_ref) log2e/sqrt(hd)) written as f16 over the
//           tile's own S columns.  O is only rescaled (TMEM load, scale,
//           store) when a row's max exceeds its reference by more than 2^8,
//           so P stays <= 256 and most tiles need no correction pass.
// Shared memory holds only K and V (3 stages); Q and P never touch it, which
// halves the shared-memory traffic of the two MMAs.  S_{j+1}, the loads of
// later tiles and P_{j-1} V_{j-1} overlap the softmax of tile j.  Every wait is bounded; a timeout records args.err and
// the CTA unwinds, still freeing its TMEM.
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace vvq2 {

namespace {

constexpr int FT = 192;        // threads
constexpr int BQ = 128;        // query rows per CTA
constexpr int BKV = 128;       // keys per tile
constexpr int BLK = 16384;     // one [128 rows][128 bytes] swizzled block
constexpr int PAGE_BYTES = KV_PAGE * 128;   // one 64-key box of 64 f16 columns
constexpr uint32_t TMEM_COLS = 512;         // S0 | S1 | O | Q
constexpr int NST = 3;                      // K/V stages

template <int HD>
struct FaCfg {
    static constexpr int NB = HD / 64;                    // 64-column blocks along hd
    static constexpr int K_OFF = 0;                       // NST stages
    static constexpr int V_OFF = K_OFF + NST * NB * BLK;  // NST stages
    static constexpr int SMEM = V_OFF + NST * NB * BLK + 1024;
    static constexpr uint32_t TILE_TX = NB * 2 * PAGE_BYTES;   // one K (or V) tile
    static constexpr uint32_t O_COL = 2 * BKV;            // output accumulator columns
    static constexpr uint32_t Q_COL = O_COL + HD;         // Q: HD/2 columns of f16 pairs
};

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// 2^x on the special-function unit (ex2.approx: ~2 ulp, -inf -> +0)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int HD>
__global__ void __launch_bounds__(FT, 1)
    k_fa_prefill(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv, const FaArgs a) {
    using C = FaCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t k_full[NST], k_empty[NST], v_full[NST], v_empty[NST], s_full[2], p_full, o_full[2];
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t mma_done;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int qtiles = (a.nt + BQ - 1) / BQ;
    const int s = blockIdx.x / qtiles;
    const int qt = qtiles - 1 - (int)(blockIdx.x % qtiles);   // longest (latest) tiles first
    const int h = blockIdx.y, G = a.nq / a.nkv, g = h / G;
    const int row0 = s * a.nt + qt * BQ, nrows = min(BQ, a.nt - qt * BQ);
    const RowMeta last = a.meta[row0 + nrows - 1];
    const int klim = min(last.pos + 1, last.kvlen);    // keys any row of the tile may see
    const int nkt = klim > 0 ? (klim + BKV - 1) / BKV : 0;   // 0: no keys here (another rank's part)

    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; ++i) {
            tc::mbar_init(&k_full[i], 1);
            tc::mbar_init(&k_empty[i], 1);
            tc::mbar_init(&v_full[i], 1);
            tc::mbar_init(&v_empty[i], 1);
        }
        tc::mbar_init(&s_full[0], 1);
        tc::mbar_init(&s_full[1], 1);
        tc::mbar_init(&p_full, 128);
        tc::mbar_init(&o_full[0], 1);
        tc::mbar_init(&o_full[1], 1);
        tc::mbar_init(&q_full, 128);
        tc::mbar_init(&mma_done, 1);
        abort_flag = 0;
        tc::mbar_fence_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&tmem_base, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = tmem_base;

    auto fail = [&]() {
        if (a.err) atomicExch(a.err, 5);
        atomicExch(&abort_flag, 1);
    };
    auto aborted = [&]() { return *(volatile int*)&abort_flag != 0; };

    if (warp == 0 && lane == 0) {
        // ---- TMA producer: K tile j after S_{j-NST} finished with its stage,
        //      V tile j after P V of tile j-NST
        auto load = [&](const CUtensorMap* map, uint8_t* stage, uint64_t* bar, int j) {
            tc::mbar_arrive_expect_tx(bar, C::TILE_TX);
            for (int ps = 0; ps < 2; ++ps) {
                const int lp = 2 * j + ps;   // logical page of the sequence
                // pages past the causal limit read rows beyond the pool: zero fill
                const int y = lp * KV_PAGE < klim
                                  ? (__ldg(a.block_table + (size_t)last.seq * a.max_pages + lp) * a.nkv + g) * KV_PAGE
                                  : a.kv_rows;
#pragma unroll
                for (int b = 0; b < C::NB; ++b) tc::tma_load_2d(stage + b * BLK + ps * PAGE_BYTES, map, b * 64, y, bar);
            }
        };
        int nk = 0, nv = 0;
        for (int j = 0; j < nkt; ++j) {
            const int st = j % NST;
            if (j >= NST && !tc::mbar_wait(&k_empty[st], ((j / NST) - 1) & 1)) { fail(); break; }
            if (aborted()) break;
            load(&mk, sm + C::K_OFF + st * C::NB * BLK, &k_full[st], j);
            ++nk;
            if (j >= NST && !tc::mbar_wait(&v_empty[st], ((j / NST) - 1) & 1)) { fail(); break; }
            if (aborted()) break;
            load(&mv, sm + C::V_OFF + st * C::NB * BLK, &v_full[st], j);
            ++nv;
        }
        // copies still in flight land before the CTA exits
        for (int j = max(0, nk - NST); j < nk; ++j) tc::mbar_wait(&k_full[j % NST], (j / NST) & 1, 1u << 20);
        for (int j = max(0, nv - NST); j < nv; ++j) tc::mbar_wait(&v_full[j % NST], (j / NST) & 1, 1u << 20);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idS = tc::idesc_f16(BQ, BKV);
        constexpr uint32_t idO = tc::idesc_f16_bmn(BQ, HD);
        bool ok = tc::mbar_wait(&q_full, 0);
        auto issue_s = [&](int j) -> bool {
            const int ks = j % NST;
            if (!tc::mbar_wait(&k_full[ks], (j / NST) & 1)) return false;
            if (aborted()) return false;
            tc::tc_fence_after();
            uint8_t* kt = sm + C::K_OFF + ks * C::NB * BLK;
#pragma unroll
            for (int k16 = 0; k16 < HD / 16; ++k16) {
                const int kb = k16 >> 2, w = k16 & 3;
                tc::mma_f16_ts(tmem + (j & 1) * BKV, tmem + C::Q_COL + k16 * 8, tc::desc_sw128(kt + kb * BLK) + 2 * w,
                               idS, k16 > 0);
            }
            tc::mma_commit(&k_empty[ks]);
            tc::mma_commit(&s_full[j & 1]);
            return true;
        };
        if (ok) {
            tc::tc_fence_after();
            ok = nkt == 0 || (issue_s(0) && (nkt < 2 || issue_s(1)));
        }
        for (int j = 0; ok && j < nkt; ++j) {
            const int vs = j % NST;
            if (!tc::mbar_wait(&p_full, j & 1) || !tc::mbar_wait(&v_full[vs], (j / NST) & 1) || aborted()) {
                ok = false;
                break;
            }
            tc::tc_fence_after();
            uint8_t* vt = sm + C::V_OFF + vs * C::NB * BLK;
#pragma unroll
            for (int k16 = 0; k16 < BKV / 16; ++k16) {
                // A = P (TMEM, over the tile's S columns), B = V (MN-major: hd contiguous per key)
                tc::mma_f16_ts(tmem + C::O_COL, tmem + (j & 1) * BKV + k16 * 8,
                               tc::desc_sw128_mn(vt + k16 * 16 * 128, BLK), idO, (j | k16) > 0);
            }
            tc::mma_commit(&v_empty[vs]);
            tc::mma_commit(&o_full[j & 1]);
            if (j + 2 < nkt && !issue_s(j + 2)) ok = false;
        }
        if (!ok) fail();
        tc::mma_commit(&mma_done);   // every MMA issued above has completed (also after an abort)
    } else if (warp >= 2) {
        // ---- softmax: thread owns query row rr (TMEM lane rr)
        const int quarter = warp & 3;
        const int rr = quarter * 32 + lane;
        const bool valid = rr < nrows;
        const int grow = row0 + rr;
        int kl = 0;
        if (valid) {
            const RowMeta rm = a.meta[grow];
            kl = min(rm.pos + 1, rm.kvlen);
        }
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        // Q row -> f16 pairs in this row's TMEM lane (the S MMA's A operand)
        {
            const float* qr = a.q + (size_t)grow * a.nq * HD + (size_t)h * HD;
#pragma unroll
            for (int cc = 0; cc < HD / 64; ++cc) {
                float qp[32];   // 32 columns = 64 elements, packed as f16 pairs
                uint32_t* qu = reinterpret_cast<uint32_t*>(qp);
#pragma unroll
                for (int e = 0; e < 64; e += 4) {
                    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (valid) x = __ldg(reinterpret_cast<const float4*>(qr + cc * 64 + e));
                    qu[e / 2] = pack_h2(x.x, x.y);
                    qu[e / 2 + 1] = pack_h2(x.z, x.w);
                }
                tc::tmem_st32(lane_base + C::Q_COL + cc * 32, qp);
            }
        }
        tc::tc_fence_before();
        tc::mbar_arrive(&q_full);

        const float c = a.scale * 1.4426950408889634f;   // scores to log2 units
        constexpr float RESCALE_LOG2 = 8.f;                 // P <= 2^8 between rescales
        float m_ref = -INFINITY, l = 0.f;
        const uint32_t to = lane_base + C::O_COL;           // this row's output accumulator
        int o_seen = 0;                                     // tiles whose P V is known complete
        bool ok = true;
        // Wait for P V of tiles < upto, in order.  o_full[t & 1] completes for
        // tiles t, t + 2, ...; P V of tile t + 2 needs this thread's p_full
        // arrival, so waiting in order before each arrival keeps parities exact.
        auto wait_o = [&](int upto) {
            while (ok && o_seen < upto) {
                ok = tc::mbar_wait(&o_full[o_seen & 1], (o_seen >> 1) & 1) && !aborted();
                ++o_seen;
            }
        };
        for (int j = 0; j < nkt; ++j) {
            const int st = j & 1;
            ok = ok && tc::mbar_wait(&s_full[st], (j >> 1) & 1) && !aborted();
            // tcgen05.ld/st are warp-collective: decide per warp
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc::tc_fence_after();
            const int k0 = j * BKV;
            // the whole S row of this tile in registers (4 loads in flight)
            uint32_t sr[BKV];
#pragma unroll
            for (int cc = 0; cc < BKV / 32; ++cc) tc::tmem_ld32_async(lane_base + st * BKV + cc * 32, sr + cc * 32);
            tc::tmem_wait_ld();
            float* sv = reinterpret_cast<float*>(sr);
            const bool edge = k0 + BKV > kl;   // causal limit inside (or before) this tile
            if (edge) {
#pragma unroll
                for (int e = 0; e < BKV; ++e)
                    if (k0 + e >= kl) sv[e] = -INFINITY;
            }
            float mx = -INFINITY;
#pragma unroll
            for (int e = 0; e < BKV; e += 4) mx = fmaxf(mx, fmaxf(fmaxf(sv[e], sv[e + 1]), fmaxf(sv[e + 2], sv[e + 3])));
            const bool need = mx != -INFINITY && (m_ref == -INFINITY || (mx - m_ref) * c > RESCALE_LOG2);
            if (__any_sync(0xffffffffu, need)) {
                const float alpha = need && m_ref != -INFINITY ? ex2((m_ref - mx) * c) : 1.f;
                if (j > 0) {
                    // O holds P V of tiles < j: let it complete, then rescale in TMEM
                    wait_o(j);
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) break;
                    tc::tc_fence_after();
#pragma unroll
                    for (int cc = 0; cc < HD / 32; ++cc) {
                        float v[32];
                        tc::tmem_ld32(to + cc * 32, v);
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] *= alpha;
                        tc::tmem_st32(to + cc * 32, v);
                    }
                }
                if (need) {
                    l *= alpha;
                    m_ref = mx;
                }
            }
            // arrivals stay within one tile of the o_full phases seen (parity tracking)
            wait_o(j - 1);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            // P = 2^(S c - m_ref c) (masked keys: 2^-inf = 0) as f16 pairs over
            // the first 64 of this tile's S columns (already read above)
            const float mc = m_ref == -INFINITY ? 0.f : m_ref * c;
            float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                float pp[32];
                uint32_t* pu = reinterpret_cast<uint32_t*>(pp);
#pragma unroll
                for (int e = 0; e < 64; e += 2) {
                    const float p0 = ex2(fmaf(sv[cc * 64 + e], c, -mc));
                    const float p1 = ex2(fmaf(sv[cc * 64 + e + 1], c, -mc));
                    if (e & 2) sum1 += p0 + p1;
                    else sum0 += p0 + p1;
                    pu[e / 2] = pack_h2(p0, p1);
                }
                tc::tmem_st32(lane_base + st * BKV + cc * 32, pp);
            }
            l += sum0 + sum1;
            tc::tc_fence_before();          // S reads, P stores and O rescale done before the MMA reuses them
            tc::mbar_arrive(&p_full);
        }
        wait_o(nkt);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
            fail();
        } else {
            tc::tc_fence_after();
            // a row without keys (l == 0) writes zeros and LSE -inf; its TMEM
            // accumulator may never have been written
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            if (valid && a.lse)   // log-sum-exp of the scaled scores, natural log
                a.lse[(size_t)grow * a.nq + h] = l > 0.f ? fmaf(m_ref, a.scale, logf(l)) : -INFINITY;
            __half* dst = a.out + (size_t)grow * a.nq * HD + (size_t)h * HD;
#pragma unroll
            for (int cc = 0; cc < HD / 32; ++cc) {
                float v[32];
                tc::tmem_ld32(to + cc * 32, v);
                if (l == 0.f) {
#pragma unroll
                    for (int d = 0; d < 32; ++d) v[d] = 0.f;
                }
                if (valid) {
#pragma unroll
                    for (int d = 0; d < 32; d += 8)
                        *reinterpret_cast<uint4*>(dst + cc * 32 + d) =
                            make_uint4(pack_h2(v[d] * inv, v[d + 1] * inv), pack_h2(v[d + 2] * inv, v[d + 3] * inv),
                                       pack_h2(v[d + 4] * inv, v[d + 5] * inv), pack_h2(v[d + 6] * inv, v[d + 7] * inv));
                }
            }
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        // no MMA may still be writing TMEM when it is released
        tc::mbar_wait(&mma_done, 0, 1u << 20);
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

cudaError_t fa_prefill_prepare() {
    cudaError_t e = cudaFuncSetAttribute(k_fa_prefill<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, FaCfg<64>::SMEM);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_fa_prefill<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, FaCfg<128>::SMEM);
}

cudaError_t fa_prefill_launch(const FaArgs& a, const CUtensorMap& mk, const CUtensorMap& mv, cudaStream_t st) {
    if (a.nt <= 0 || a.n_seqs <= 0) return cudaSuccess;
    if (a.nq % a.nkv || a.hd != 64 && a.hd != 128) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)(a.n_seqs * ((a.nt + BQ - 1) / BQ)), (unsigned)a.nq);
    if (a.hd == 64) k_fa_prefill<64><<<grid, FT, FaCfg<64>::SMEM, st>>>(mk, mv, a);
    else k_fa_prefill<128><<<grid, FT, FaCfg<128>::SMEM, st>>>(mk, mv, a);
    note_launch();
    return cudaGetLastError();
}

}  // namespace vvq2
