// gemm_ws.cu -- persistent prefill GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM) with the GGUF weight dequantization fused in, sm_100a.
//
// Y[T, N] = X[T, K] . W[N, K]^T for the Qwen2 layer's linears when a prompt
// chunk carries many token rows (src/qwen2.cpp:19-26,274-276,349; the SwiGLU
// FFN at :33-40).  ggml multiplies the quantized blocks directly; here the
// blocks are dequantized by producer warps into shared memory (ggml's exact
// dequantize_row_* values rounded once to f16), so no f16 copy of a weight
// matrix ever exists in HBM.
//
// Tile: 256 weight rows x nt token rows (nt = 128..256, chosen per launch so
// the tiles fill whole waves of the 148 SMs).  The weight rows are the MMA A
// operands (two 128-row halves), the tokens the shared B operand (f16 by
// TMA), so one token tile read from L2 serves 256 weight rows and one
// dequantized weight tile serves nt tokens.  Two TMEM accumulators of 128
// lanes x nt columns: lane = weight row (output feature), column = token.
// Epilogue warps read them with tcgen05.ld and store straight to global
// memory: for a fixed token the 32 lanes of a warp hold 32 consecutive
// features, so every store is one contiguous segment.
//
// Persistent: one CTA per SM walks the tile list (grouped raster: 16 token
// tiles at a time against every weight tile, so those token tiles stay in
// L2 while the weights stream once per group).  Three rings run ahead of
// the MMA, across tile boundaries: raw Q8_0 bytes (quants and block scales
// of 256 rows, by TMA), the dequantized f16 A tiles, the f16 token tiles.
// The producers read the raw ring from shared memory 512 contiguous bytes
// per warp instruction, so no weight byte passes the L1 load path.
//
// Accumulator layouts per epilogue:
//   RESID / STORE  acc0 = features n0..n0+127, acc1 = n0+128..n0+255
//   SWIGLU         acc0 = gate rows, acc1 = up rows of features f0..f0+127
//                  (a thread holds g and u of one feature: no exchange)
//   QKV            acc0 = first halves, acc1 = second halves (dims i and
//                  i + hd/2) of 256/hd heads, so the NEOX pair of a thread's
//                  lane sits in its own two accumulators
//
// CTA: 19 warps.  warp 0: TMEM allocation + token TMA (lane 0); warp 1: MMA
// issuer (lane 0); warp 2: raw-weight TMA (lane 0, Q8_0); warps 3-10:
// weight producers; warps 11-18: epilogue (two per TMEM lane quarter,
// alternating 32-column chunks).  Every wait is bounded; a timeout sets
// args.err and unwinds without leaving TMEM allocated.
#include <algorithm>

#include "common.cuh"
#include "dequant_tile.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace vvq2 {

namespace {

constexpr int WM = 128;                          // weight rows per accumulator (MMA M)
constexpr int BK = 64;                           // K per stage: 128 bytes of f16, one swizzle row
constexpr int MAX_NT = 256;                      // token rows per tile (MMA N)
constexpr int A_BYTES = WM * BK * 2;             // 16 KB per accumulator's weight tile
constexpr int A_STAGE = 2 * A_BYTES;             // both accumulators' A operands
constexpr int B_STAGE = MAX_NT * BK * 2;         // 32 KB token tile
constexpr int RQ_BYTES = 2 * WM * BK;            // raw Q8_0 quants of 256 rows x 64
constexpr int R_STAGE = RQ_BYTES + 2 * WM * 16;  // + 16 bytes of block scales per row (4 k-blocks)
constexpr int A_STAGES = 2, B_STAGES = 3, R_STAGES = 3;
constexpr int B_OFF = A_STAGES * A_STAGE, R_OFF = B_OFF + B_STAGES * B_STAGE;
constexpr int SMEM_BYTES = R_OFF + R_STAGES * R_STAGE + 1024;   // + alignment slack
constexpr int N_PROD = 8;                        // producer warps: 256 threads
constexpr int N_EPI = 8;                         // epilogue warps
constexpr int PROD0 = 3, EPI0 = PROD0 + N_PROD;  // first producer / epilogue warp
constexpr int THREADS = 32 * (EPI0 + N_EPI);
constexpr int TMEM_COLS = 512;                   // acc0 at column 0, acc1 at column 256
constexpr int TGROUP = 16;                       // token tiles per raster group

struct Sched {
    int wt, tt, nt, nk, n_tiles;
    __device__ __forceinline__ void tile(int id, int& wi, int& ti) const {
        const int g = id / (wt * TGROUP);
        const int within = id - g * wt * TGROUP;
        const int gg = min(TGROUP, tt - g * TGROUP);
        wi = within / gg;
        ti = g * TGROUP + within % gg;
    }
};

// Weight row behind A row p (0..255) of weight tile wi, and the matrix it
// comes from (rows past the matrix are zero-filled by the producers and
// never stored by the epilogue).
template <int EPI>
__device__ __forceinline__ int a_row(const GemmArgs& a, int wi, int p, const DevW*& W) {
    const int acc = p >> 7, r = p & 127;
    if constexpr (EPI == EPI_SWIGLU) {
        W = acc ? &a.w1 : &a.w0;
        return wi * WM + r;
    } else if constexpr (EPI == EPI_QKV) {
        W = &a.w0;
        const int half = a.hd >> 1;
        return wi * 2 * WM + (r / half) * a.hd + acc * half + r % half;
    } else {
        W = &a.w0;
        return wi * 2 * WM + p;
    }
}

// A row (0..255) fed by row rho of the tile's raw weight rows (the tile's
// 256 matrix rows in order; SwiGLU: 128 gate rows, then the same 128 up rows)
template <int EPI>
__device__ __forceinline__ int a_of_raw(const GemmArgs& a, int rho) {
    if constexpr (EPI == EPI_QKV) {
        const int half = a.hd >> 1, hh = rho / a.hd, rem = rho % a.hd;
        return (rem / half) * WM + hh * half + rem % half;
    } else {
        return rho;
    }
}

template <int WT, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_ws(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmQ0,
              const __grid_constant__ CUtensorMap tmQ1, const __grid_constant__ CUtensorMap tmS0,
              const __grid_constant__ CUtensorMap tmS1, const GemmArgs a, const Sched sc) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t a_full[A_STAGES], a_empty[A_STAGES], b_full[B_STAGES], b_empty[B_STAGES];
    __shared__ __align__(8) uint64_t r_full[R_STAGES], r_empty[R_STAGES], tfull, tempty, drain;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    asm volatile("griddepcontrol.launch_dependents;");

    if (threadIdx.x == 0) {
        for (int s = 0; s < A_STAGES; ++s) {
            tc::mbar_init(&a_full[s], 32 * N_PROD);
            tc::mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < B_STAGES; ++s) {
            tc::mbar_init(&b_full[s], 1);
            tc::mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < R_STAGES; ++s) {
            tc::mbar_init(&r_full[s], 1);
            tc::mbar_init(&r_empty[s], 32 * N_PROD);
        }
        tc::mbar_init(&tfull, 1);
        tc::mbar_init(&tempty, N_EPI);
        tc::mbar_init(&drain, 1);
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
    auto aborted = [&]() { return *(volatile int*)&abort_flag != 0; };
    const int nk = sc.nk;

    if (warp == 0) {
        if (lane == 0) {
            // ---- token TMA: the B operand of every k-block
            asm volatile("griddepcontrol.wait;" ::: "memory");
            uint32_t g = 0;
            const uint32_t bytes = (uint32_t)sc.nt * BK * 2;
            for (int id = blockIdx.x; id < sc.n_tiles && !aborted(); id += gridDim.x) {
                int wi, ti;
                sc.tile(id, wi, ti);
                const int t0 = ti * sc.nt;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % B_STAGES;
                    if (g >= B_STAGES && !tc::mbar_wait(&b_empty[s], ((g / B_STAGES) - 1) & 1)) { fail(); break; }
                    if (aborted()) break;
                    tc::mbar_arrive_expect_tx(&b_full[s], bytes);
                    tc::tma_load_2d(smem + B_OFF + s * B_STAGE, &tmX, kb * BK, t0, &b_full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: per stage 4 K-steps x 2 accumulators of 128 x nt
            const uint32_t idesc = tc::idesc_f16(WM, sc.nt);
            uint32_t g = 0;
            int it = 0;
            for (int id = blockIdx.x; id < sc.n_tiles; id += gridDim.x, ++it) {
                if (it > 0 && !tc::mbar_wait(&tempty, (it - 1) & 1)) { fail(); break; }
                if (aborted()) break;
                tc::tc_fence_after();
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int sa = g % A_STAGES, sb = g % B_STAGES;
                    if (!tc::mbar_wait(&a_full[sa], (g / A_STAGES) & 1) || !tc::mbar_wait(&b_full[sb], (g / B_STAGES) & 1)) {
                        fail();
                        ok = false;
                        break;
                    }
                    if (aborted()) { ok = false; break; }
                    tc::tc_fence_after();
                    uint8_t* sta = smem + sa * A_STAGE;
                    const uint64_t da0 = tc::desc_sw128(sta), da1 = tc::desc_sw128(sta + A_BYTES);
                    const uint64_t db = tc::desc_sw128(smem + B_OFF + sb * B_STAGE);
#pragma unroll
                    for (int k16 = 0; k16 < BK / 16; ++k16) {
                        const uint32_t acc = (kb | k16) != 0;
                        tc::mma_f16(tmem, da0 + 2 * k16, db + 2 * k16, idesc, acc);
                        tc::mma_f16(tmem + 256, da1 + 2 * k16, db + 2 * k16, idesc, acc);
                    }
                    tc::mma_commit(&a_empty[sa]);
                    tc::mma_commit(&b_empty[sb]);
                }
                if (!ok) break;
                tc::mma_commit(&tfull);
            }
            tc::mma_commit(&drain);   // every issued MMA complete (also after an abort)
            if (!tc::mbar_wait(&drain, 0)) fail();
        }
    } else if (warp == 2) {
        if (WT == W_Q8_0 && lane == 0) {
            // ---- raw-weight TMA: quants of the k-block and the block scales
            // of its group of 4 k-blocks (16 bytes per row, the row's scale
            // area starts at byte K of the row) for the tile's 256 rows
            uint32_t g = 0;
            const int rows_box = EPI == EPI_SWIGLU ? WM : 2 * WM;
            for (int id = blockIdx.x; id < sc.n_tiles && !aborted(); id += gridDim.x) {
                int wi, ti;
                sc.tile(id, wi, ti);
                const int y = wi * rows_box;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % R_STAGES;
                    if (g >= R_STAGES && !tc::mbar_wait(&r_empty[s], ((g / R_STAGES) - 1) & 1)) { fail(); break; }
                    if (aborted()) break;
                    uint8_t* rs = smem + R_OFF + s * R_STAGE;
                    const int xs = a.K + 16 * (kb >> 2);
                    tc::mbar_arrive_expect_tx(&r_full[s], R_STAGE);
                    tc::tma_load_2d(rs, &tmQ0, kb * BK, y, &r_full[s]);
                    tc::tma_load_2d(rs + RQ_BYTES, &tmS0, xs, y, &r_full[s]);
                    if (EPI == EPI_SWIGLU) {
                        tc::tma_load_2d(rs + WM * BK, &tmQ1, kb * BK, y, &r_full[s]);
                        tc::tma_load_2d(rs + RQ_BYTES + WM * 16, &tmS1, xs, y, &r_full[s]);
                    }
                }
            }
        }
    } else if (warp < EPI0) {
        // ---- weight producers
        const int t = threadIdx.x - 32 * PROD0;
        if constexpr (WT == W_Q8_0) {
            // thread (w, l) converts 16-byte chunk c = l % 4 of raw rows
            // 8w + l/4 + 64i (i = 0..3): a warp reads 8 whole 64-byte rows,
            // 512 contiguous bytes, per shared load
            const int w = t >> 5, l = t & 31, c = l & 3;
            int rho[4], aoff[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                rho[i] = 8 * w + (l >> 2) + 64 * i;
                const int p = a_of_raw<EPI>(a, rho[i]);
                aoff[i] = (p >> 7) * A_BYTES + (p & 127) * 128;
            }
            uint32_t g = 0;
            bool stop = false;
            for (int id = blockIdx.x; id < sc.n_tiles && !stop; id += gridDim.x) {
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int sr = g % R_STAGES, sa = g % A_STAGES;
                    if (!tc::mbar_wait(&r_full[sr], (g / R_STAGES) & 1) ||
                        (g >= A_STAGES && !tc::mbar_wait(&a_empty[sa], ((g / A_STAGES) - 1) & 1))) {
                        fail();
                        stop = true;
                        break;
                    }
                    if (aborted()) { stop = true; break; }
                    const uint8_t* rs = smem + R_OFF + sr * R_STAGE;
                    uint4 v[4];
                    unsigned short d[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        v[i] = *reinterpret_cast<const uint4*>(rs + rho[i] * BK + c * 16);
                        d[i] = *reinterpret_cast<const unsigned short*>(rs + RQ_BYTES + rho[i] * 16 + (kb & 3) * 4 +
                                                                        (c >> 1) * 2);
                    }
                    tc::mbar_arrive(&r_empty[sr]);   // this thread's raw bytes are in registers
                    uint8_t* st = smem + sa * A_STAGE;
#pragma unroll
                    for (int i = 0; i < 4; ++i) q8_0_chunk_pair(v[i], d[i], st + aoff[i], (aoff[i] >> 7) & 7, 2 * c);
                    tc::fence_proxy_async_smem();
                    tc::mbar_arrive(&a_full[sa]);
                }
            }
        } else {
            // other types: thread t produces A row t from global memory
            uint8_t* const aacc = smem + (t >> 7) * A_BYTES;
            const int r = t & 127;
            uint32_t g = 0;
            bool stop = false;
            for (int id = blockIdx.x; id < sc.n_tiles && !stop; id += gridDim.x) {
                int wi, ti;
                sc.tile(id, wi, ti);
                const DevW* W;
                const int row = a_row<EPI>(a, wi, t, W);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int sa = g % A_STAGES;
                    if (g >= A_STAGES && !tc::mbar_wait(&a_empty[sa], ((g / A_STAGES) - 1) & 1)) { fail(); stop = true; break; }
                    if (aborted()) { stop = true; break; }
                    produce_row<WT>(*W, row, kb * BK, aacc + sa * A_STAGE, r);
                    tc::fence_proxy_async_smem();
                    tc::mbar_arrive(&a_full[sa]);
                }
            }
        }
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32*(w%4)..+31 of both
        // accumulators, 32-column chunks e, e+2, e+4, ... (e = its set)
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int q = warp & 3, e = (warp - EPI0) >> 2;
        const int r = q * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        int it = 0;
        for (int id = blockIdx.x; id < sc.n_tiles; id += gridDim.x, ++it) {
            int wi, ti;
            sc.tile(id, wi, ti);
            const int t0 = ti * sc.nt;
            const int vt = min(sc.nt, a.T - t0);          // valid token columns
            const int nch = (vt + 31) >> 5;
            const int last = (nch - 1 - e) >= 0 ? e + ((nch - 1 - e) >> 1) * 2 : -1;
            // per-lane features and constants of this tile
            const DevW* W;
            const int f0 = a_row<EPI>(a, wi, r, W), f1 = a_row<EPI>(a, wi, r + 128, W);
            const bool ok0 = f0 < a.N, ok1 = f1 < a.N;
            const float b0 = (a.bias && ok0) ? a.bias[f0] : 0.f, b1 = (a.bias && ok1) ? a.bias[f1] : 0.f;
            if (!tc::mbar_wait(&tfull, it & 1)) { fail(); break; }
            if (aborted()) break;
            tc::tc_fence_after();
            auto release = [&]() {   // this warp's last TMEM read of the tile: the MMA may go on
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty);
            };
            if (last < 0) {   // no valid columns for this warp: release at once
                release();
                continue;
            }
            for (int c = e; c <= last; c += 2) {
                const int tb = t0 + c * 32;
                const int ne = min(32, a.T - tb);   // valid tokens in the chunk (warp-uniform)
                if constexpr (EPI == EPI_RESID || EPI == EPI_STORE) {
                    for (int acc = 0; acc < 2; ++acc) {
                        uint32_t u[32];
                        __syncwarp();
                        tc::tmem_ld32_async(lane_base + acc * 256 + c * 32, u);
                        tc::tmem_wait_ld();
                        if (acc == 1 && c == last) release();
                        const bool ok = acc ? ok1 : ok0;
                        const float b = acc ? b1 : b0;
                        if (ok) {
                            float* y = a.y + (size_t)tb * a.y_stride + (acc ? f1 : f0);
                            if constexpr (EPI == EPI_RESID) {
#pragma unroll
                                for (int h = 0; h < 32; h += 16) {   // 16 residual loads in flight
                                    float x[16];
#pragma unroll
                                    for (int j = 0; j < 16; ++j) x[j] = h + j < ne ? y[(size_t)(h + j) * a.y_stride] : 0.f;
#pragma unroll
                                    for (int j = 0; j < 16; ++j)
                                        if (h + j < ne)
                                            y[(size_t)(h + j) * a.y_stride] =
                                                __fadd_rn(x[j], __fadd_rn(__uint_as_float(u[h + j]), b));
                                }
                            } else {
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    if (j < ne) y[(size_t)j * a.y_stride] = __fadd_rn(__uint_as_float(u[j]), b);
                            }
                        }
                    }
                } else {
                    uint32_t u0[32], u1[32];
                    __syncwarp();
                    tc::tmem_ld32_async(lane_base + c * 32, u0);
                    tc::tmem_ld32_async(lane_base + 256 + c * 32, u1);
                    tc::tmem_wait_ld();
                    if (c == last) release();
                    if constexpr (EPI == EPI_SWIGLU) {
                        if (ok0) {
                            __half* yh = a.yh + (size_t)tb * a.yh_stride + f0;
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (j < ne)
                                    yh[(size_t)j * a.yh_stride] = __float2half_rn(
                                        __fmul_rn(silu_f16out(__uint_as_float(u0[j])), __uint_as_float(u1[j])));
                        }
                    } else {   // EPI_QKV
                        const int hd = a.hd, half = hd >> 1;
                        const int h = f0 / hd, i = f0 % hd;       // head; dim within the first half
                        const bool rot = h < a.nq + a.nkv;
                        const bool is_q = h < a.nq, is_k = !is_q && rot;
                        const int kvh = is_q ? 0 : (is_k ? h - a.nq : h - a.nq - a.nkv);
                        if (ok0) {
                            // 4 tokens at a time: their RoPE table loads go out
                            // before the stores
#pragma unroll
                            for (int j0 = 0; j0 < 32; j0 += 4) {
                                if (j0 >= ne) break;
                                float2 cs[4];
#pragma unroll
                                for (int jj = 0; jj < 4; ++jj)
                                    cs[jj] = (rot && j0 + jj < ne) ? __ldg(&a.rope_cs[(size_t)(tb + j0 + jj) * half + i])
                                                                   : make_float2(1.f, 0.f);
#pragma unroll
                                for (int jj = 0; jj < 4; ++jj) {
                                    const int j = j0 + jj;
                                    if (j >= ne) break;
                                    float v0 = __fadd_rn(__uint_as_float(u0[j]), b0);
                                    float v1 = __fadd_rn(__uint_as_float(u1[j]), b1);
                                    if (rot) {
                                        const float y0 = __fsub_rn(__fmul_rn(v0, cs[jj].x), __fmul_rn(v1, cs[jj].y));
                                        const float y1 = __fadd_rn(__fmul_rn(v0, cs[jj].y), __fmul_rn(v1, cs[jj].x));
                                        v0 = y0;
                                        v1 = y1;
                                    }
                                    if (is_q) {
                                        float* qd = a.y + (size_t)(tb + j) * a.y_stride + h * hd;
                                        qd[i] = v0;
                                        qd[i + half] = v1;
                                    } else {
                                        const RowMeta rm = a.meta[tb + j];
                                        if (rm.cidx >= 0) {   // cidx < 0: another rank stores this position
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
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

int sm_count() {
    static const int n = [] {
        int dev = 0, v = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

int weight_tiles(const GemmArgs& a) {
    return a.epi == EPI_SWIGLU ? (a.N + WM - 1) / WM : (a.N + 2 * WM - 1) / (2 * WM);
}

template <int EPI>
cudaError_t launch_ws(const GemmArgs& a, const CUtensorMap& tm, const CUtensorMap* wq, int nt, cudaStream_t st) {
    Sched sc;
    sc.wt = weight_tiles(a);
    sc.nt = nt;
    sc.tt = (a.T + nt - 1) / nt;
    sc.nk = a.K / BK;
    sc.n_tiles = sc.wt * sc.tt;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min(sc.n_tiles, sm_count()));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (a.w0.type) {
        case W_Q8_0: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_Q8_0, EPI>, tm, wq[0], wq[1], wq[2], wq[3], a, sc); break;
        case W_Q5_K: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_Q5_K, EPI>, tm, tm, tm, tm, tm, a, sc); break;
        case W_Q6_K: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_Q6_K, EPI>, tm, tm, tm, tm, tm, a, sc); break;
        case W_F16: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_F16, EPI>, tm, tm, tm, tm, tm, a, sc); break;
        case W_F32: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_F32, EPI>, tm, tm, tm, tm, tm, a, sc); break;
        default: return cudaErrorInvalidValue;
    }
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <int EPI>
cudaError_t prepare_ws() {
    const void* fns[] = {(const void*)k_gemm_ws<W_Q8_0, EPI>, (const void*)k_gemm_ws<W_Q5_K, EPI>,
                         (const void*)k_gemm_ws<W_Q6_K, EPI>, (const void*)k_gemm_ws<W_F16, EPI>,
                         (const void*)k_gemm_ws<W_F32, EPI>};
    for (const void* f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

// Token-tile height for a launch: the multiple of 32 in [128, 256] that
// minimises (waves of tiles over the SMs) x (tile height), the larger on a
// tie; 0 when the GEMM has fewer than min_tiles tiles (<= 0: the SM count)
// at every height (the few-row kernel with split-K serves those better).
int gemm_ws_tile_rows(const GemmArgs& a, int min_tiles) {
    const int wt = weight_tiles(a), sms = sm_count();
    if (min_tiles <= 0) min_tiles = sms;
    int best = 0;
    long long best_cost = 0;
    for (int nt = 256; nt >= 128; nt -= 32) {
        const long long tiles = (long long)wt * ((a.T + nt - 1) / nt);
        if (tiles < min_tiles) continue;
        const long long cost = (tiles + sms - 1) / sms * nt;
        if (!best || cost < best_cost) {
            best = nt;
            best_cost = cost;
        }
    }
    return best;
}

cudaError_t gemm_ws_prepare() {
    cudaError_t e;
    if ((e = prepare_ws<EPI_QKV>()) != cudaSuccess) return e;
    if ((e = prepare_ws<EPI_RESID>()) != cudaSuccess) return e;
    if ((e = prepare_ws<EPI_SWIGLU>()) != cudaSuccess) return e;
    return prepare_ws<EPI_STORE>();
}

int gemm_ws_weight_box_rows(const GemmArgs& a) { return a.epi == EPI_SWIGLU ? WM : 2 * WM; }

cudaError_t gemm_ws_launch(const GemmArgs& a, const CUtensorMap& tmX, const CUtensorMap* wq, int nt,
                           cudaStream_t st) {
    if (a.K % BK || a.T <= 0 || a.N <= 0 || nt < 128 || nt > MAX_NT || nt % 32) return cudaErrorInvalidValue;
    if (a.kpart || a.epi == EPI_ARGMAX) return cudaErrorInvalidValue;
    if (a.epi == EPI_QKV && ((2 * WM) % a.hd || (a.hd != 32 && a.hd != 64 && a.hd != 128)))
        return cudaErrorInvalidValue;
    if (a.epi == EPI_SWIGLU && (a.w1.type != a.w0.type || a.w1.rows != a.w0.rows)) return cudaErrorInvalidValue;
    if (a.w0.type == W_Q8_0 && (!wq || a.w0.cols != a.K)) return cudaErrorInvalidValue;
    switch (a.epi) {
        case EPI_QKV: return launch_ws<EPI_QKV>(a, tmX, wq, nt, st);
        case EPI_RESID: return launch_ws<EPI_RESID>(a, tmX, wq, nt, st);
        case EPI_SWIGLU: return launch_ws<EPI_SWIGLU>(a, tmX, wq, nt, st);
        case EPI_STORE: return launch_ws<EPI_STORE>(a, tmX, wq, nt, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace vvq2
