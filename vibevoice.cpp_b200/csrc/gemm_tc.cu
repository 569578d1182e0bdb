// gemm_tc.cu -- prefill-sized (> 8 rows) dequant GEMM on the 5th-generation
// tensor cores (tcgen05 + TMEM), sm_100a.
//
// Y[T, N] = X[T, K] . W[N, K]^T for every linear of the Qwen2 layer when a
// call carries more token rows than the decode GEMV handles
// (src/qwen2.cpp:19-26,274-276,349, the SwiGLU FFN at :33-40).  GGUF blocks
// cannot feed the tensor cores directly, so the weight operand is produced in
// shared memory by dequantizing warps: ggml's dequantize_row_* values (exact
// f32) rounded once to f16, written in the K-major 128-byte-swizzled layout
// the UMMA descriptor expects.  Activations arrive as f16 via TMA (same
// swizzle).  One thread issues tcgen05.mma (kind::f16, f32 accumulate) into
// two 128x128 TMEM accumulators, so each dequantized weight tile serves 256
// token rows.  Epilogue warps read TMEM with tcgen05.ld and apply the fused
// epilogue: QKV (+bias, NEOX RoPE, K/V into the f16 paged cache), residual
// add, SwiGLU (gate/up tiles interleaved), or a plain store.
//
// CTA: 6 warps.  warp 0: TMEM allocation + TMA producer (lane 0);
// warp 1: MMA issuer (lane 0); warps 2-5: weight producers, then epilogue.
//
// Chunks with enough rows to fill the SMs with 256 x 256 tiles run the
// persistent kernel of gemm_ws.cu instead; this one serves the few-row
// GEMMs (batched decode of many streams, short prompt chunks, split-K).
// Pipeline: stages of {A0, A1, B} 16 KB tiles (BK = 64), mbarriers
// full/empty; 4 stages, or 3 for Q8_0, whose raw bytes (each k-block's
// quants and its rows' block scales) arrive by TMA in an 8-deep ring that the
// producers read from shared memory, 512 contiguous bytes per warp load
// (other types: each producer thread decodes its row from global memory).
// Epilogues that write rows stage the accumulators through the drained
// pipeline buffers so that a warp stores whole rows.  The kernel is launched
// as a programmatic dependent: barrier setup, TMEM allocation and the first
// raw weight loads overlap the previous kernel; the TMA thread waits
// (griddepcontrol.wait) before loading anything that kernel wrote.  Every wait is bounded; a timeout sets args.err and unwinds without
// leaving TMEM allocated.
#include <algorithm>

#include "common.cuh"
#include "dequant_tile.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace vvq2 {

namespace {

constexpr int BM = 128;       // token rows per accumulator (two accumulators per CTA)
constexpr int BN = 128;       // output features per CTA
constexpr int BK = 64;        // K per stage (128 bytes of f16: one swizzle row)
constexpr int STAGES = 4;
constexpr int TILE_BYTES = BM * BK * 2;                 // 16 KB
constexpr int STAGE_BYTES = 3 * TILE_BYTES;             // A0, A1, B
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
// Q8_0: the raw weight bytes of a k-block (quants of the tile's 128 rows,
// then the rows' block scales of its group of 4 k-blocks) arrive by TMA into
// an R_STAGES-deep ring that runs ahead of the f16 stages; 3 f16 stages
// leave it room
constexpr int Q8_STAGES = 3, R_STAGES = 8;
constexpr int RQ_BYTES = BN * BK, R_STAGE = RQ_BYTES + BN * 16;
constexpr int Q8_SMEM_BYTES = Q8_STAGES * STAGE_BYTES + R_STAGES * R_STAGE + 1024;
__host__ __device__ constexpr int smem_bytes(int wt) { return wt == W_Q8_0 ? Q8_SMEM_BYTES : SMEM_BYTES; }
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 256;


template <int WT, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ0,
              const __grid_constant__ CUtensorMap tmQ1, const __grid_constant__ CUtensorMap tmS0,
              const __grid_constant__ CUtensorMap tmS1, const GemmArgs a) {
    constexpr int ST = WT == W_Q8_0 ? Q8_STAGES : STAGES;   // f16 pipeline stages
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[ST], empty[ST], done, r_full[R_STAGES], r_empty[R_STAGES];
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // a dependent GEMM may start its prologue and weight prefetch now (it waits
    // for this grid before reading anything this grid writes)
    asm volatile("griddepcontrol.launch_dependents;");
    const int n0 = blockIdx.x * BN, t0 = blockIdx.y * (2 * BM);
    const bool two = t0 + BM < a.T;
    // split-K: CTA z of gridDim.z takes k-blocks [kb0, kb0 + nk) and writes a
    // raw f32 partial (a.kpart); splitk_epilogue_launch sums them in order
    const int nk_all = a.K / BK;
    const int kb0 = (int)((long long)nk_all * blockIdx.z / gridDim.z);
    const int nk = (int)((long long)nk_all * (blockIdx.z + 1) / gridDim.z) - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            tc::mbar_init(&full[s], 1 + 128);
            tc::mbar_init(&empty[s], 1);
        }
        if (WT == W_Q8_0)
            for (int s = 0; s < R_STAGES; ++s) {
                tc::mbar_init(&r_full[s], 1);
                tc::mbar_init(&r_empty[s], 128);
            }
        tc::mbar_init(&done, 1);
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
        if (a.err) atomicExch(a.err, 2);
        atomicExch(&abort_flag, 1);
    };

    if (warp == 0 && lane == 0) {
        // ---- TMA producer: activation tiles A0 (rows t0..) and A1 (rows
        // t0+128..) and, for Q8_0, the raw weight ring (k-block j's quants and
        // its scale group), R_STAGES k-blocks ahead of the producers.
        // Launched as a programmatic dependent: everything before the wait
        // (barriers, TMEM, the first raw weight loads) overlapped the previous
        // kernel; its outputs (the activations A) are read only after it.
        uint8_t* const rawb = smem + ST * STAGE_BYTES;
        const int y = EPI == EPI_SWIGLU ? (int)blockIdx.x * 64 : n0;
        auto issue_raw = [&](int j) {   // j: local k-block
            uint8_t* rs = rawb + (j % R_STAGES) * R_STAGE;
            const int kx = (kb0 + j) * BK, xs = a.K + 16 * ((kb0 + j) >> 2);
            uint64_t* bar = &r_full[j % R_STAGES];
            tc::mbar_arrive_expect_tx(bar, R_STAGE);
            tc::tma_load_2d(rs, &tmQ0, kx, y, bar);
            tc::tma_load_2d(rs + RQ_BYTES, &tmS0, xs, y, bar);
            if (EPI == EPI_SWIGLU) {   // gate rows, then the same up rows
                tc::tma_load_2d(rs + 64 * BK, &tmQ1, kx, y, bar);
                tc::tma_load_2d(rs + RQ_BYTES + 64 * 16, &tmS1, xs, y, bar);
            }
        };
        if constexpr (WT == W_Q8_0)
            for (int j = 0; j < min(nk, R_STAGES); ++j) issue_raw(j);
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int i = 0; i < nk; ++i) {
            const int s = i % ST, kx = (kb0 + i) * BK;
            if (i >= ST && !tc::mbar_wait(&empty[s], ((i / ST) - 1) & 1)) { fail(); break; }
            if (*(volatile int*)&abort_flag) break;
            uint8_t* st = smem + s * STAGE_BYTES;
            tc::mbar_arrive_expect_tx(&full[s], (two ? 2 : 1) * TILE_BYTES);
            tc::tma_load_2d(st, &tmA, kx, t0, &full[s]);
            if (two) tc::tma_load_2d(st + TILE_BYTES, &tmA, kx, t0 + BM, &full[s]);
            if constexpr (WT == W_Q8_0) {
                // raw k-block i + R_STAGES into the slot the producers finish with k-block i
                const int j = i + R_STAGES;
                if (j < nk) {
                    if (!tc::mbar_wait(&r_empty[i % R_STAGES], (i / R_STAGES) & 1)) { fail(); break; }
                    issue_raw(j);
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = tc::idesc_f16(BM, BN);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {   // local k-block index
            const int s = kb % ST;
            if (!tc::mbar_wait(&full[s], (kb / ST) & 1)) { fail(); ok = false; break; }
            if (*(volatile int*)&abort_flag) { ok = false; break; }
            tc::tc_fence_after();
            uint8_t* st = smem + s * STAGE_BYTES;
            const uint64_t da0 = tc::desc_sw128(st), da1 = tc::desc_sw128(st + TILE_BYTES);
            const uint64_t db = tc::desc_sw128(st + 2 * TILE_BYTES);
#pragma unroll
            for (int k16 = 0; k16 < BK / 16; ++k16) {
                const uint32_t acc = (kb | k16) != 0;
                tc::mma_f16(tmem, da0 + 2 * k16, db + 2 * k16, idesc, acc);
                if (two) tc::mma_f16(tmem + BN, da1 + 2 * k16, db + 2 * k16, idesc, acc);
            }
            tc::mma_commit(&empty[s]);   // stage s free once these MMAs complete
        }
        tc::mma_commit(&done);          // all issued MMAs complete (also on the abort path)
        (void)ok;
    } else if (warp >= 2) {
        // ---- weight producers: thread p owns row p of the B tile
        const int p = threadIdx.x - 64;
        int wrow;
        const DevW* W;
        if (EPI == EPI_SWIGLU) {
            W = p < 64 ? &a.w0 : &a.w1;
            wrow = blockIdx.x * 64 + (p & 63);
        } else {
            W = &a.w0;
            wrow = n0 + p;
        }
        if constexpr (WT == W_Q8_0) {
            // Q8_0 from the raw ring: thread (w, l) converts 16-byte chunk
            // c = l % 4 of tile rows 8w + l/4 + 32i (i = 0..3): a warp reads 8
            // whole 64-byte rows, 512 contiguous bytes, per shared load
            const int w = p >> 5, l = p & 31, c = l & 3;
            const uint8_t* rawb = smem + ST * STAGE_BYTES;
            bool stop = false;
            for (int kb = 0; kb < nk && !stop; ++kb) {   // local k-block index
                const int s = kb % ST, rsl = kb % R_STAGES;
                if (!tc::mbar_wait(&r_full[rsl], (kb / R_STAGES) & 1) ||
                    (kb >= ST && !tc::mbar_wait(&empty[s], ((kb / ST) - 1) & 1))) {
                    fail();
                    break;
                }
                if (*(volatile int*)&abort_flag) break;
                const uint8_t* rs = rawb + rsl * R_STAGE;
                uint4 v[4];
                unsigned short d[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int rho = 8 * w + (l >> 2) + 32 * i;
                    v[i] = *reinterpret_cast<const uint4*>(rs + rho * BK + c * 16);
                    d[i] = *reinterpret_cast<const unsigned short*>(rs + RQ_BYTES + rho * 16 +
                                                                    ((kb0 + kb) & 3) * 4 + (c >> 1) * 2);
                }
                tc::mbar_arrive(&r_empty[rsl]);   // this thread's raw bytes are in registers
                uint8_t* bt = smem + s * STAGE_BYTES + 2 * TILE_BYTES;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int rho = 8 * w + (l >> 2) + 32 * i;
                    q8_0_chunk_pair(v[i], d[i], bt + rho * 128, rho & 7, 2 * c);
                }
                tc::fence_proxy_async_smem();
                tc::mbar_arrive(&full[s]);
            }
            (void)stop;
        } else {
            for (int kb = 0; kb < nk; ++kb) {   // local k-block index
                const int s = kb % ST;
                if (kb >= ST && !tc::mbar_wait(&empty[s], ((kb / ST) - 1) & 1)) { fail(); break; }
                if (*(volatile int*)&abort_flag) break;
                uint8_t* bt = smem + s * STAGE_BYTES + 2 * TILE_BYTES;
                produce_row<WT>(*W, wrow, (kb0 + kb) * BK, bt, p);
                tc::fence_proxy_async_smem();
                tc::mbar_arrive(&full[s]);
            }
        }
        (void)W;
        (void)wrow;
        // ---- epilogue: wait for the accumulators
        bool ok = tc::mbar_wait(&done, 0);
        if (!ok) fail();
        tc::tc_fence_after();
        const int quarter = warp & 3;    // TMEM lanes 32*quarter .. +31
        const int r = quarter * 32 + lane;
        // tcgen05.ld is warp-collective: decide per warp
        ok = __all_sync(0xffffffffu, ok && !*(volatile int*)&abort_flag);
        if (ok) {
            for (int acc = 0; acc < (two ? 2 : 1); ++acc) {
                const int t = t0 + acc * BM + r;
                const bool valid = t < a.T;
                const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + acc * BN;
                if (EPI == EPI_RESID || EPI == EPI_STORE || EPI == EPI_SWIGLU || (EPI == EPI_QKV && a.kpart)) {
                    // Staged through shared memory (the pipeline stages are free once
                    // every MMA completed) so that global rows are written whole by a
                    // warp: the warp's 32 rows x BN f32, 16-byte chunk j of row rr at
                    // chunk (j & ~7) | ((j ^ rr) & 7) (conflict-free both ways).
                    uint8_t* stg = smem + quarter * (32 * BN * 4);
                    for (int c = 0; c < BN; c += 32) {
                        float v[32];
                        tc::tmem_ld32(tbase + c, v);
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const int j = c / 4 + k, pj = (j & ~7) | ((j ^ lane) & 7);
                            *reinterpret_cast<float4*>(stg + lane * (BN * 4) + pj * 16) =
                                make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
                        }
                    }
                    __syncwarp();
#pragma unroll 4
                    for (int rr = 0; rr < 32; ++rr) {
                        const int tr = t0 + acc * BM + quarter * 32 + rr;
                        if (tr >= a.T) continue;   // uniform in the warp
                        if (EPI == EPI_SWIGLU) {
                            // columns 0-63 gate, 64-127 up of features i0 .. i0+63; lane: 2 features
                            const int i = blockIdx.x * 64 + 2 * lane;
                            const int jg = lane >> 1, ju = 16 + (lane >> 1);
                            const float4 g4 = *reinterpret_cast<const float4*>(
                                stg + rr * (BN * 4) + ((jg & ~7) | ((jg ^ rr) & 7)) * 16);
                            const float4 u4 = *reinterpret_cast<const float4*>(
                                stg + rr * (BN * 4) + ((ju & ~7) | ((ju ^ rr) & 7)) * 16);
                            const float g0 = (lane & 1) ? g4.z : g4.x, g1 = (lane & 1) ? g4.w : g4.y;
                            const float u0 = (lane & 1) ? u4.z : u4.x, u1 = (lane & 1) ? u4.w : u4.y;
                            __half* dst = a.yh + (size_t)tr * a.yh_stride + i;
                            if (i + 1 < a.N)
                                *reinterpret_cast<__half2*>(dst) =
                                    __floats2half2_rn(__fmul_rn(silu_f16out(g0), u0), __fmul_rn(silu_f16out(g1), u1));
                            else if (i < a.N)
                                *dst = __float2half_rn(__fmul_rn(silu_f16out(g0), u0));
                        } else {
                            const int pj = (lane & ~7) | ((lane ^ rr) & 7);
                            float4 x = *reinterpret_cast<const float4*>(stg + rr * (BN * 4) + pj * 16);
                            const int n = n0 + 4 * lane;
                            float xv[4] = {x.x, x.y, x.z, x.w};
                            if (a.kpart) {
                                // split-K partial [z][T][N], summed by splitk_epilogue_launch
                                float* dst = a.kpart + ((size_t)blockIdx.z * a.T + tr) * a.N + n;
                                if (n + 3 < a.N && (a.N & 3) == 0) *reinterpret_cast<float4*>(dst) = x;
                                else
                                    for (int e = 0; e < 4; ++e)
                                        if (n + e < a.N) dst[e] = xv[e];
                            } else {
                                float* dst = a.y + (size_t)tr * a.y_stride + n;
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    if (n + e < a.N) {
                                        float v = xv[e];
                                        if (a.bias) v = __fadd_rn(v, a.bias[n + e]);
                                        dst[e] = (EPI == EPI_RESID) ? __fadd_rn(dst[e], v) : v;
                                    }
                                }
                            }
                        }
                    }
                    __syncwarp();   // the region is reused by the next accumulator
                } else if (a.kpart && EPI != EPI_ARGMAX && EPI != EPI_SWIGLU) {
                    // split-K partial [z][T][N], summed by splitk_epilogue_launch
                    for (int c = 0; c < BN; c += 32) {
                        float v[32];
                        tc::tmem_ld32(tbase + c, v);
                        if (!valid) continue;
                        float* dst = a.kpart + ((size_t)blockIdx.z * a.T + t) * a.N + n0 + c;
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (n0 + c + e < a.N) dst[e] = v[e];
                    }
                } else if constexpr (EPI == EPI_ARGMAX) {
                    // lm_head: this row's best (logit, feature) over the tile, one atomic per row
                    unsigned long long best = 0ull;
                    for (int c = 0; c < BN; c += 32) {
                        float v[32];
                        tc::tmem_ld32(tbase + c, v);
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int n = n0 + c + e;
                            if (n < a.N) {
                                const unsigned long long k = argmax_key(v[e], n);
                                best = k > best ? k : best;
                            }
                        }
                    }
                    if (valid && best) atomicMax(a.amax + t, best);
                    if (valid && a.tile_best) a.tile_best[(size_t)t * a.tile_stride + blockIdx.x] = best;
                } else if constexpr (EPI == EPI_RESID || EPI == EPI_STORE) {
                    for (int c = 0; c < BN; c += 32) {
                        float v[32];
                        tc::tmem_ld32(tbase + c, v);
                        if (!valid) continue;
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int n = n0 + c + e;
                            if (n < a.N) {
                                float x = v[e];
                                if (a.bias) x = __fadd_rn(x, a.bias[n]);
                                float* dst = a.y + (size_t)t * a.y_stride + n;
                                *dst = (EPI == EPI_RESID) ? __fadd_rn(*dst, x) : x;
                            }
                        }
                    }
                } else if constexpr (EPI == EPI_SWIGLU) {
                    for (int c = 0; c < 64; c += 32) {
                        float g[32], u[32];
                        tc::tmem_ld32(tbase + c, g);
                        tc::tmem_ld32(tbase + 64 + c, u);
                        if (!valid) continue;
                        const int i0 = blockIdx.x * 64 + c;
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            if (i0 + e + 1 < a.N) {
                                *reinterpret_cast<__half2*>(a.yh + (size_t)t * a.yh_stride + i0 + e) =
                                    __floats2half2_rn(__fmul_rn(silu_f16out(g[e]), u[e]), __fmul_rn(silu_f16out(g[e + 1]), u[e + 1]));
                            } else if (i0 + e < a.N) {
                                a.yh[(size_t)t * a.yh_stride + i0 + e] = __float2half_rn(__fmul_rn(silu_f16out(g[e]), u[e]));
                            }
                        }
                    }
                } else if constexpr (EPI == EPI_QKV) {
                    const int hd = a.hd, half = hd / 2;
                    const RowMeta rm = valid ? a.meta[t] : RowMeta{0, 0, 0, 0};
                    for (int hb = 0; hb < BN; hb += hd) {          // heads within the tile
                        for (int i0 = 0; i0 < half; i0 += 32) {
                            float x0[32], x1[32];
                            int npair;
                            if (half >= 32) {
                                tc::tmem_ld32(tbase + hb + i0, x0);
                                tc::tmem_ld32(tbase + hb + half + i0, x1);
                                npair = 32;
                            } else {   // hd 32: one load holds both halves
                                float v[32];
                                tc::tmem_ld32(tbase + hb, v);
#pragma unroll
                                for (int e = 0; e < 16; ++e) {
                                    x0[e] = v[e];
                                    x1[e] = v[e + 16];
                                }
                                npair = 16;
                            }
                            const int f0 = n0 + hb;                // first feature of this head
                            if (!valid || f0 >= a.N) continue;
                            const int h = f0 / hd;
                            for (int e = 0; e < npair; ++e) {
                                const int i = i0 + e;
                                float v0 = x0[e], v1 = x1[e];
                                if (a.bias) {
                                    v0 = __fadd_rn(v0, a.bias[f0 + i]);
                                    v1 = __fadd_rn(v1, a.bias[f0 + i + half]);
                                }
                                if (h < a.nq + a.nkv) {
                                    const float2 cs = a.rope_cs[(size_t)t * half + i];
                                    const float y0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
                                    const float y1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
                                    v0 = y0;
                                    v1 = y1;
                                }
                                if (h < a.nq) {
                                    float* q = a.y + (size_t)t * a.y_stride + h * hd;
                                    q[i] = v0;
                                    q[i + half] = v1;
                                } else if (rm.cidx >= 0) {   // cidx < 0: another rank stores this position
                                    const bool is_k = h < a.nq + a.nkv;
                                    const int kvh = is_k ? h - a.nq : h - a.nq - a.nkv;
                                    __half* dst = (is_k ? a.kv.k : a.kv.v) + kv_offset(a.kv, rm.seq, rm.cidx, kvh);
                                    dst[i] = __float2half_rn(v0);
                                    dst[i + half] = __float2half_rn(v1);
                                }
                            }
                        }
                    }
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int EPI>
cudaError_t launch_epi(const GemmArgs& a, const CUtensorMap& tm, const CUtensorMap* wq, cudaStream_t st) {
    dim3 grid((EPI == EPI_SWIGLU ? (a.N + 63) / 64 : (a.N + BN - 1) / BN), (a.T + 2 * BM - 1) / (2 * BM),
              a.kpart ? a.k_splits : 1);
    // programmatic dependent launch: CTAs may start (prologue, weight
    // prefetch) while the previous kernel drains; see griddepcontrol.wait
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem_bytes(a.w0.type);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (a.w0.type) {
        case W_Q8_0: e = cudaLaunchKernelEx(&cfg, k_gemm_tc<W_Q8_0, EPI>, tm, wq[0], wq[1], wq[2], wq[3], a); break;
        case W_Q5_K: e = cudaLaunchKernelEx(&cfg, k_gemm_tc<W_Q5_K, EPI>, tm, tm, tm, tm, tm, a); break;
        case W_Q6_K: e = cudaLaunchKernelEx(&cfg, k_gemm_tc<W_Q6_K, EPI>, tm, tm, tm, tm, tm, a); break;
        case W_F16: e = cudaLaunchKernelEx(&cfg, k_gemm_tc<W_F16, EPI>, tm, tm, tm, tm, tm, a); break;
        case W_F32: e = cudaLaunchKernelEx(&cfg, k_gemm_tc<W_F32, EPI>, tm, tm, tm, tm, tm, a); break;
        default: return cudaErrorInvalidValue;
    }
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <int EPI>
cudaError_t prepare_epi() {
    const void* fns[] = {(const void*)k_gemm_tc<W_Q8_0, EPI>, (const void*)k_gemm_tc<W_Q5_K, EPI>,
                         (const void*)k_gemm_tc<W_Q6_K, EPI>, (const void*)k_gemm_tc<W_F16, EPI>,
                         (const void*)k_gemm_tc<W_F32, EPI>};
    const int types[] = {W_Q8_0, W_Q5_K, W_Q6_K, W_F16, W_F32};
    for (int i = 0; i < 5; ++i) {
        cudaError_t e = cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(types[i]));
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Sum the split-K partials in split order and apply the epilogue: one thread
// per (row, column) for RESID / STORE, per (row, rotation pair) for QKV.
__global__ void k_splitk_epilogue(const GemmArgs a) {
    const int64_t per_row = a.epi == EPI_QKV ? a.N / 2 : a.N;
    const int64_t total = (int64_t)a.T * per_row;
    const int ks = a.k_splits;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_row);
        auto sum = [&](int n) {
            // in split order; eight independent loads in flight at a time
            const float* kp = a.kpart + (size_t)t * a.N + n;
            const size_t zs = (size_t)a.T * a.N;
            float v = 0.f;
            int z = 0;
            for (; z + 8 <= ks; z += 8) {
                float p[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) p[i] = kp[(size_t)(z + i) * zs];
#pragma unroll
                for (int i = 0; i < 8; ++i) v += p[i];
            }
            for (; z < ks; ++z) v += kp[(size_t)z * zs];
            return v;
        };
        if (a.epi == EPI_QKV) {
            const int hd = a.hd, half = hd / 2;
            const int pr = (int)(i % per_row);
            const int h = pr / half, ii = pr % half, f0 = h * hd;
            float v0 = sum(f0 + ii), v1 = sum(f0 + ii + half);
            if (a.bias) {
                v0 = __fadd_rn(v0, a.bias[f0 + ii]);
                v1 = __fadd_rn(v1, a.bias[f0 + ii + half]);
            }
            if (h < a.nq + a.nkv) {
                const float2 cs = a.rope_cs[(size_t)t * half + ii];
                const float y0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
                const float y1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
                v0 = y0;
                v1 = y1;
            }
            if (h < a.nq) {
                float* q = a.y + (size_t)t * a.y_stride + f0;
                q[ii] = v0;
                q[ii + half] = v1;
            } else if (a.meta[t].cidx >= 0) {   // cidx < 0: another rank stores this position
                const RowMeta rm = a.meta[t];
                const bool is_k = h < a.nq + a.nkv;
                const int kvh = is_k ? h - a.nq : h - a.nq - a.nkv;
                __half* dst = (is_k ? a.kv.k : a.kv.v) + kv_offset(a.kv, rm.seq, rm.cidx, kvh);
                dst[ii] = __float2half_rn(v0);
                dst[ii + half] = __float2half_rn(v1);
            }
        } else {
            const int n = (int)(i % per_row);
            float v = sum(n);
            if (a.bias) v = __fadd_rn(v, a.bias[n]);
            float* dst = a.y + (size_t)t * a.y_stride + n;
            *dst = a.epi == EPI_RESID ? __fadd_rn(*dst, v) : v;
        }
    }
}

}  // namespace

cudaError_t splitk_epilogue_launch(const GemmArgs& a, cudaStream_t st) {
    if (!a.kpart || a.k_splits < 1) return cudaErrorInvalidValue;
    const int64_t total = (int64_t)a.T * (a.epi == EPI_QKV ? a.N / 2 : a.N);
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 8);
    k_splitk_epilogue<<<(unsigned)blocks, 256, 0, st>>>(a);
    note_launch();
    return cudaGetLastError();
}

cudaError_t gemm_tc_prepare() {
    cudaError_t e;
    if ((e = prepare_epi<EPI_QKV>()) != cudaSuccess) return e;
    if ((e = prepare_epi<EPI_RESID>()) != cudaSuccess) return e;
    if ((e = prepare_epi<EPI_SWIGLU>()) != cudaSuccess) return e;
    if ((e = prepare_epi<EPI_ARGMAX>()) != cudaSuccess) return e;
    return prepare_epi<EPI_STORE>();
}

cudaError_t gemm_tc_launch(const GemmArgs& a, const CUtensorMap& tmA, const CUtensorMap* wq, cudaStream_t st) {
    if (a.K % BK || a.T <= 0 || a.N <= 0) return cudaErrorInvalidValue;
    if (a.epi == EPI_QKV && (BN % a.hd || (a.hd != 32 && a.hd != 64 && a.hd != 128))) return cudaErrorInvalidValue;
    if (a.kpart && (a.k_splits < 1 || a.k_splits > a.K / BK || a.epi == EPI_SWIGLU || a.epi == EPI_ARGMAX))
        return cudaErrorInvalidValue;
    if (a.w0.type == W_Q8_0 && (!wq || a.w0.cols != a.K)) return cudaErrorInvalidValue;
    switch (a.epi) {
        case EPI_QKV: return launch_epi<EPI_QKV>(a, tmA, wq, st);
        case EPI_RESID: return launch_epi<EPI_RESID>(a, tmA, wq, st);
        case EPI_SWIGLU: return launch_epi<EPI_SWIGLU>(a, tmA, wq, st);
        case EPI_STORE: return launch_epi<EPI_STORE>(a, tmA, wq, st);
        case EPI_ARGMAX: return a.amax ? launch_epi<EPI_ARGMAX>(a, tmA, wq, st) : cudaErrorInvalidValue;
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace vvq2
