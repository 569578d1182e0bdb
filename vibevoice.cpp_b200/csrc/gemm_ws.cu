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
// L2 while the weights stream once per group).  The producers run ahead
// across tile boundaries, so the next tile's first stages are ready while
// the epilogue drains the accumulators.
//
// Accumulator layouts per epilogue:
//   RESID / STORE  acc0 = features n0..n0+127, acc1 = n0+128..n0+255
//   SWIGLU         acc0 = gate rows, acc1 = up rows of features f0..f0+127
//                  (a thread holds g and u of one feature: no exchange)
//   QKV            acc0 = first halves, acc1 = second halves (dims i and
//                  i + hd/2) of 256/hd heads, so the NEOX pair of a thread's
//                  lane sits in its own two accumulators
//
// CTA: 18 warps.  warp 0: TMEM allocation + TMA producer (lane 0); warp 1:
// MMA issuer (lane 0); warps 2-9: weight producers (one A row per thread);
// warps 10-17: epilogue (two per TMEM lane quarter, alternating 32-column
// chunks).  Every wait is bounded; a timeout sets args.err and unwinds
// without leaving TMEM allocated.
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
constexpr int B_BYTES = MAX_NT * BK * 2;         // 32 KB token tile
constexpr int STAGE_BYTES = 2 * A_BYTES + B_BYTES;
constexpr int STAGES = 3;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;   // + alignment slack
constexpr int N_PROD = 8;                        // producer warps: 256 threads, one A row each
constexpr int N_EPI = 8;                         // epilogue warps
constexpr int THREADS = 32 * (2 + N_PROD + N_EPI);
constexpr int TMEM_COLS = 512;                   // acc0 at column 0, acc1 at column 256
constexpr int TGROUP = 16;                       // token tiles per raster group
constexpr int PD = 3;                            // Q8_0 k-blocks fetched ahead of their conversion

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

template <int WT, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_ws(const __grid_constant__ CUtensorMap tmX, const GemmArgs a, const Sched sc) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], tfull, tempty, drain;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    asm volatile("griddepcontrol.launch_dependents;");

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full[s], 1 + 32 * N_PROD);
            tc::mbar_init(&empty[s], 1);
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
            // ---- TMA producer: the token tile of every stage
            asm volatile("griddepcontrol.wait;" ::: "memory");
            uint32_t kbg = 0;
            const uint32_t bytes = (uint32_t)sc.nt * BK * 2;
            for (int id = blockIdx.x; id < sc.n_tiles && !aborted(); id += gridDim.x) {
                int wi, ti;
                sc.tile(id, wi, ti);
                const int t0 = ti * sc.nt;
                for (int kb = 0; kb < nk; ++kb, ++kbg) {
                    const int s = kbg % STAGES;
                    if (kbg >= STAGES && !tc::mbar_wait(&empty[s], ((kbg / STAGES) - 1) & 1)) { fail(); break; }
                    if (aborted()) break;
                    tc::mbar_arrive_expect_tx(&full[s], bytes);
                    tc::tma_load_2d(smem + s * STAGE_BYTES + 2 * A_BYTES, &tmX, kb * BK, t0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: per stage 4 K-steps x 2 accumulators of 128 x nt
            const uint32_t idesc = tc::idesc_f16(WM, sc.nt);
            uint32_t kbg = 0;
            int it = 0;
            for (int id = blockIdx.x; id < sc.n_tiles; id += gridDim.x, ++it) {
                if (it > 0 && !tc::mbar_wait(&tempty, (it - 1) & 1)) { fail(); break; }
                if (aborted()) break;
                tc::tc_fence_after();
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++kbg) {
                    const int s = kbg % STAGES;
                    if (!tc::mbar_wait(&full[s], (kbg / STAGES) & 1)) { fail(); ok = false; break; }
                    if (aborted()) { ok = false; break; }
                    tc::tc_fence_after();
                    uint8_t* st = smem + s * STAGE_BYTES;
                    const uint64_t da0 = tc::desc_sw128(st), da1 = tc::desc_sw128(st + A_BYTES);
                    const uint64_t db = tc::desc_sw128(st + 2 * A_BYTES);
#pragma unroll
                    for (int k16 = 0; k16 < BK / 16; ++k16) {
                        const uint32_t acc = (kb | k16) != 0;
                        tc::mma_f16(tmem, da0 + 2 * k16, db + 2 * k16, idesc, acc);
                        tc::mma_f16(tmem + 256, da1 + 2 * k16, db + 2 * k16, idesc, acc);
                    }
                    tc::mma_commit(&empty[s]);
                }
                if (!ok) break;
                tc::mma_commit(&tfull);
            }
            tc::mma_commit(&drain);   // every issued MMA complete (also after an abort)
            if (!tc::mbar_wait(&drain, 0)) fail();
        }
    } else if (warp < 2 + N_PROD) {
        // ---- weight producers: thread p writes A row p (acc p / 128, lane p % 128)
        const int p = threadIdx.x - 64;
        uint8_t* const abase = smem + (p >> 7) * A_BYTES;
        const int r = p & 127;
        if constexpr (WT == W_Q8_0) {
            // raw blocks fetched PD k-blocks ahead, across tile boundaries
            int f_id = blockIdx.x, f_kb = 0;       // the next (tile, k-block) to fetch
            const uint8_t* f_rp = nullptr;
            const unsigned short* f_dp = nullptr;
            auto seek = [&]() {                     // row pointers of tile f_id
                f_rp = nullptr;
                if (f_id < sc.n_tiles) {
                    int wi, ti;
                    sc.tile(f_id, wi, ti);
                    const DevW* W;
                    const int row = a_row<EPI>(a, wi, p, W);
                    if (row < W->rows) {
                        f_rp = W->q + (size_t)row * W->row_stride;
                        f_dp = reinterpret_cast<const unsigned short*>(W->d) + (size_t)row * W->d_stride;
                    }
                }
            };
            auto fetch = [&](uint4 (&q)[4], uint32_t& d2) {
                if (f_rp) {
                    const int k0 = f_kb * BK;
#pragma unroll
                    for (int i = 0; i < 4; ++i) q[i] = __ldg(reinterpret_cast<const uint4*>(f_rp + k0) + i);
                    d2 = __ldg(reinterpret_cast<const unsigned int*>(f_dp + k0 / 32));
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) q[i] = make_uint4(0, 0, 0, 0);
                    d2 = 0u;
                }
                if (++f_kb == nk) {
                    f_kb = 0;
                    f_id += gridDim.x;
                    seek();
                }
            };
            seek();
            uint4 raw[PD][4];
            uint32_t dd[PD];
#pragma unroll
            for (int d = 0; d < PD; ++d) fetch(raw[d], dd[d]);
            const uint32_t total = (uint32_t)((sc.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * nk;
            bool stop = false;
            for (uint32_t kbg = 0; kbg < total && !stop; kbg += PD) {
#pragma unroll
                for (int d = 0; d < PD; ++d) {
                    const uint32_t g = kbg + d;
                    if (g >= total) break;
                    const int s = g % STAGES;
                    if (g >= STAGES && !tc::mbar_wait(&empty[s], ((g / STAGES) - 1) & 1)) { fail(); stop = true; break; }
                    if (aborted()) { stop = true; break; }
                    q8_0_tile_row(raw[d], dd[d], abase + s * STAGE_BYTES, r);
                    fetch(raw[d], dd[d]);
                    tc::fence_proxy_async_smem();
                    tc::mbar_arrive(&full[s]);
                }
            }
        } else {
            uint32_t kbg = 0;
            bool stop = false;
            for (int id = blockIdx.x; id < sc.n_tiles && !stop; id += gridDim.x) {
                int wi, ti;
                sc.tile(id, wi, ti);
                const DevW* W;
                const int row = a_row<EPI>(a, wi, p, W);
                for (int kb = 0; kb < nk; ++kb, ++kbg) {
                    const int s = kbg % STAGES;
                    if (kbg >= STAGES && !tc::mbar_wait(&empty[s], ((kbg / STAGES) - 1) & 1)) { fail(); stop = true; break; }
                    if (aborted()) { stop = true; break; }
                    produce_row<WT>(*W, row, kb * BK, abase + s * STAGE_BYTES, r);
                    tc::fence_proxy_async_smem();
                    tc::mbar_arrive(&full[s]);
                }
            }
        }
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32*(w%4)..+31 of both
        // accumulators, 32-column chunks e, e+2, e+4, ... (e = its set)
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int q = warp & 3, e = (warp - 2 - N_PROD) >> 2;
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
                                        __fmul_rn(silu_ref(__uint_as_float(u0[j])), __uint_as_float(u1[j])));
                        }
                    } else {   // EPI_QKV
                        const int hd = a.hd, half = hd >> 1;
                        const int h = f0 / hd, i = f0 % hd;       // head; dim within the first half
                        const bool rot = h < a.nq + a.nkv;
                        const bool is_q = h < a.nq, is_k = !is_q && rot;
                        const int kvh = is_q ? 0 : (is_k ? h - a.nq : h - a.nq - a.nkv);
                        if (ok0) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                if (j < ne) {
                                    const int t = tb + j;
                                    float v0 = __fadd_rn(__uint_as_float(u0[j]), b0);
                                    float v1 = __fadd_rn(__uint_as_float(u1[j]), b1);
                                    if (rot) {
                                        const float2 cs = a.rope_cs[(size_t)t * half + i];
                                        const float y0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
                                        const float y1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
                                        v0 = y0;
                                        v1 = y1;
                                    }
                                    if (is_q) {
                                        float* qd = a.y + (size_t)t * a.y_stride + h * hd;
                                        qd[i] = v0;
                                        qd[i + half] = v1;
                                    } else {
                                        const RowMeta rm = a.meta[t];
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
cudaError_t launch_ws(const GemmArgs& a, const CUtensorMap& tm, int nt, cudaStream_t st) {
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
        case W_Q8_0: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_Q8_0, EPI>, tm, a, sc); break;
        case W_Q5_K: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_Q5_K, EPI>, tm, a, sc); break;
        case W_Q6_K: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_Q6_K, EPI>, tm, a, sc); break;
        case W_F16: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_F16, EPI>, tm, a, sc); break;
        case W_F32: e = cudaLaunchKernelEx(&cfg, k_gemm_ws<W_F32, EPI>, tm, a, sc); break;
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

cudaError_t gemm_ws_launch(const GemmArgs& a, const CUtensorMap& tmX, int nt, cudaStream_t st) {
    if (a.K % BK || a.T <= 0 || a.N <= 0 || nt < 128 || nt > MAX_NT || nt % 32) return cudaErrorInvalidValue;
    if (a.kpart || a.epi == EPI_ARGMAX) return cudaErrorInvalidValue;
    if (a.epi == EPI_QKV && ((2 * WM) % a.hd || (a.hd != 32 && a.hd != 64 && a.hd != 128)))
        return cudaErrorInvalidValue;
    if (a.epi == EPI_SWIGLU && (a.w1.type != a.w0.type || a.w1.rows != a.w0.rows)) return cudaErrorInvalidValue;
    switch (a.epi) {
        case EPI_QKV: return launch_ws<EPI_QKV>(a, tmX, nt, st);
        case EPI_RESID: return launch_ws<EPI_RESID>(a, tmX, nt, st);
        case EPI_SWIGLU: return launch_ws<EPI_SWIGLU>(a, tmX, nt, st);
        case EPI_STORE: return launch_ws<EPI_STORE>(a, tmX, nt, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace vvq2
