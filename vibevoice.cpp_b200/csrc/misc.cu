// misc.cu -- small kernels around the hot path: dequantization (tests),
// standalone RoPE / RMSNorm (rope.hpp / rms_norm.hpp equivalents), token
// embedding rows, KV prefix upload/readback and argmax finalisation.
#include <atomic>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"

namespace vvq2 {

namespace {
std::atomic<long long> g_launches{0};
}

void note_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

namespace {

__global__ void k_dequant(DevW w, int64_t n, float* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = deq_elem(w, (int)(i / w.cols), (int)(i % w.cols));
}

// ggml_rope_ext NEOX on [n_tok][n_heads][hd]; one thread per rotation pair
__global__ void k_rope(const float* x, int n_tok, int n_heads, int hd, const int32_t* pos, float ts,
                       float* y) {
    const int half = hd / 2;
    const int64_t n = (int64_t)n_tok * n_heads * half;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(t % half);
        const int64_t th = t / half;          // token * n_heads + head
        const int tok = (int)(th / n_heads);
        float x0 = x[th * hd + i], x1 = x[th * hd + i + half];
        rope_pair(x0, x1, pos[tok], i, ts);
        y[th * hd + i] = x0;
        y[th * hd + i + half] = x1;
    }
}

// ggml_rms_norm + ggml_mul: one CTA per row
__global__ void k_rmsnorm(const float* x, const float* w, int n, float eps, float* y) {
    __shared__ float red[32];
    __shared__ float scale_s;
    const float* xr = x + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (int k = threadIdx.x; k < n; k += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xr[k], xr[k]));
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = __fadd_rn(t, red[i]);
        const float mean = __fdiv_rn(t, (float)n);
        scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    __syncthreads();
    const float sc = scale_s;
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        y[(size_t)blockIdx.x * n + k] = __fmul_rn(__fmul_rn(xr[k], sc), w[k]);
}

// RMSNorm rows to f16: one CTA per row
__global__ void k_rmsnorm_f16(const float* x, const float* w, int n, float eps, __half* y) {
    __shared__ float red[32];
    __shared__ float scale_s;
    // the next kernel (a GEMM launched as a programmatic dependent) may start its
    // prologue now; it reads y only after griddepcontrol.wait
    asm volatile("griddepcontrol.launch_dependents;");
    const float* xr = x + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (int k = threadIdx.x; k < n; k += blockDim.x) ss = fmaf(xr[k], xr[k], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
        scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)n), eps)));
    }
    __syncthreads();
    const float sc = scale_s;
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        y[(size_t)blockIdx.x * n + k] = __float2half_rn(__fmul_rn(__fmul_rn(xr[k], sc), w[k]));
}

// A residual projection split along K, finished together with the RMSNorm
// that reads its rows next: x[r][k] += (bias[k] +) sum over splits z, in
// order, of part[z][r][k] -- the split-K epilogue's sum -- then y[r] =
// f16(x[r] * rms_scale * w), the same arithmetic as k_rmsnorm_f16 on the
// updated row.  One launch and one pass over the rows instead of two.
__global__ void k_splitk_resid_rmsnorm_f16(const float* part, int ks, int64_t zs, const float* bias, float* x,
                                           const float* w, int n, float eps, __half* y) {
    __shared__ float red[32];
    __shared__ float scale_s;
    asm volatile("griddepcontrol.launch_dependents;");
    float* xr = x + (size_t)blockIdx.x * n;
    const float* pr = part + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        float v = 0.f;
        int z = 0;
        for (; z + 8 <= ks; z += 8) {
            float p[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) p[i] = pr[(size_t)(z + i) * zs + k];
#pragma unroll
            for (int i = 0; i < 8; ++i) v += p[i];
        }
        for (; z < ks; ++z) v += pr[(size_t)z * zs + k];
        if (bias) v = __fadd_rn(v, bias[k]);
        const float xv = __fadd_rn(xr[k], v);
        xr[k] = xv;
        ss = fmaf(xv, xv, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
        scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)n), eps)));
    }
    __syncthreads();
    const float sc = scale_s;
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        y[(size_t)blockIdx.x * n + k] = __float2half_rn(__fmul_rn(__fmul_rn(xr[k], sc), w[k]));
}

__global__ void k_rope_table(const RowMeta* meta, int rows, int half, float ts, float2* cs) {
    const int64_t n = (int64_t)rows * half;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(t / half), i = (int)(t % half);
        float th = (float)meta[r].pos;
        for (int k = 0; k < i; ++k) th = __fmul_rn(th, ts);
        cs[t] = make_float2(cosf(th), sinf(th));
    }
}

__global__ void k_to_f16(const float* x, int64_t n, __half* y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __float2half_rn(x[i]);
}

__global__ void k_embed(DevW t, const int32_t* tok, int n, float* out) {
    const int i = blockIdx.x;
    const int r = tok[i];
    if (r < 0 || r >= t.rows) {
        for (int k = threadIdx.x; k < t.cols; k += blockDim.x) out[(size_t)i * t.cols + k] = 0.f;
        return;
    }
    for (int k = threadIdx.x; k < t.cols; k += blockDim.x) out[(size_t)i * t.cols + k] = deq_elem(t, r, k);
}

__global__ void k_kv_upload(KvLayer kv, int seq, const float* k, const float* v, int n_pos) {
    const int w = kv.n_kv * kv.hd;
    const int64_t n = (int64_t)n_pos * w;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int p = (int)(t / w), r = (int)(t % w), h = r / kv.hd, d = r % kv.hd;
        const size_t off = kv_offset(kv, seq, p, h) + d;
        kv.k[off] = __float2half_rn(k[t]);
        kv.v[off] = __float2half_rn(v[t]);
    }
}

__global__ void k_kv_download(KvLayer kv, int seq, float* k, float* v, int n_pos) {
    const int w = kv.n_kv * kv.hd;
    const int64_t n = (int64_t)n_pos * w;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int p = (int)(t / w), r = (int)(t % w), h = r / kv.hd, d = r % kv.hd;
        const size_t off = kv_offset(kv, seq, p, h) + d;
        k[t] = __half2float(kv.k[off]);
        v[t] = __half2float(kv.v[off]);
    }
}

// decode graphs end by moving every row one position forward
__global__ void k_advance_meta(RowMeta* meta, int n) {
    if (threadIdx.x < n) {
        RowMeta r = meta[threadIdx.x];
        r.pos += 1;
        r.cidx += 1;
        r.kvlen += 1;
        meta[threadIdx.x] = r;
    }
}

// The next decode position of a partitioned context's rows: the true rows
// advance by one, this rank's rows are derived from them (its sequence part).
__global__ void k_advance_meta_part(RowMeta* meta_true, RowMeta* meta_local, int n, int seq_parts, int part) {
    if (threadIdx.x < n) {
        RowMeta r = meta_true[threadIdx.x];
        r.pos += 1;
        r.cidx += 1;
        r.kvlen += 1;
        meta_true[threadIdx.x] = r;
        meta_local[threadIdx.x] = seq_parts > 1 ? zz_local_row(r, part) : r;
    }
}

__global__ void k_argmax_init(unsigned long long* keys, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) keys[i] = 0ull;
}

__global__ void k_argmax_final(const unsigned long long* keys, int n, int32_t* out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = argmax_key_index(keys[i]);
}

// Float of an argmax key (inverse of argmax_key's order-preserving map).
__device__ __forceinline__ float argmax_key_value(unsigned long long k) {
    uint32_t u = (uint32_t)(k >> 32);
    u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
    return __uint_as_float(u);
}

constexpr int RS_THREADS = 256;
constexpr int RS_MAX_CAND = 256;   // candidate tiles rescored per row

// One CTA per row: x o w and the RMSNorm row scale into shared memory, the
// candidate tiles (best approximate key within margin of the row's best),
// then one warp per column computes the exact logit
//   (sum_k deq(W[n][k]) * (x[k] * w[k])) * 1/sqrt(mean(x^2) + eps)
// and the CTA keeps the first-maximum key.  More candidates than
// RS_MAX_CAND: the excess tiles keep their approximate keys and err gets 6.
__global__ void __launch_bounds__(RS_THREADS) k_argmax_rescore(const float* X, const float* norm_w, float eps,
                                                                int H, const DevW w,
                                                                const unsigned long long* tile_best, int ntiles,
                                                                float margin, unsigned long long* keys, int* err) {
    extern __shared__ float xs[];   // [H]
    __shared__ int cand[RS_MAX_CAND];
    __shared__ int ncand;
    __shared__ float red[RS_THREADS / 32];
    __shared__ unsigned long long best_w[RS_THREADS / 32];
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) ncand = 0;
    float ss = 0.f;
    for (int k = tid; k < H; k += RS_THREADS) {
        const float v = X[(size_t)t * H + k];
        ss = fmaf(v, v, ss);
        xs[k] = norm_w ? __fmul_rn(v, norm_w[k]) : v;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < RS_THREADS / 32; ++i) tot += red[i];
    const float nsc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
    const float M = argmax_key_value(keys[t]);
    const float thr = M - margin * fabsf(M);
    for (int j = tid; j < ntiles; j += RS_THREADS) {
        const unsigned long long kb = tile_best[(size_t)t * ntiles + j];
        if (kb && argmax_key_value(kb) >= thr) {
            const int e = atomicAdd(&ncand, 1);
            if (e < RS_MAX_CAND) cand[e] = j;
            else if (err) atomicCAS(err, 0, 6);
        }
    }
    __syncthreads();
    const int nc = min(ncand, RS_MAX_CAND);
    unsigned long long mine = 0ull;
    for (int c = warp; c < nc * 128; c += RS_THREADS / 32) {
        const int n = cand[c / 128] * 128 + (c % 128);
        if (n >= w.rows) continue;   // uniform in the warp
        float acc = 0.f;
        if (w.type == W_Q8_0) {
            // 16 stored bytes (q + 128) and their block scale per lane step;
            // q * d is exact in f32 (8 x 11 significant bits), as deq_elem's
            const uint8_t* rp = w.q + (size_t)n * w.row_stride;
            const __half* dp = w.d + (size_t)n * w.d_stride;
            for (int c = lane; c < H / 16; c += 32) {
                const uint4 q4 = __ldg(reinterpret_cast<const uint4*>(rp) + c);
                const float d = __half2float(dp[c >> 1]);
                const uint32_t wd[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int q = (int)((wd[i >> 2] >> (8 * (i & 3))) & 0xffu) - 128;
                    acc = fmaf(__fmul_rn((float)q, d), xs[c * 16 + i], acc);
                }
            }
        } else {
            for (int k = lane; k < H; k += 32) acc = fmaf(deq_elem(w, n, k), xs[k], acc);
        }
        acc = warp_sum(acc);
        const unsigned long long key = argmax_key(__fmul_rn(acc, nsc), n);
        mine = key > mine ? key : mine;
    }
    if (lane == 0) best_w[warp] = mine;
    __syncthreads();
    if (tid == 0) {
        unsigned long long b = 0ull;
        for (int i = 0; i < RS_THREADS / 32; ++i) b = best_w[i] > b ? best_w[i] : b;
        if (b) keys[t] = b;
    }
}

int grid_for(int64_t n, int threads) {
    const int64_t g = (n + threads - 1) / threads;
    return (int)(g < 148 * 16 ? (g < 1 ? 1 : g) : 148 * 16);
}

}  // namespace

cudaError_t dequant_rows_launch(const DevW& w, float* dst, cudaStream_t st) {
    const int64_t n = (int64_t)w.rows * w.cols;
    k_dequant<<<grid_for(n, 256), 256, 0, st>>>(w, n, dst);
    note_launch();
    return cudaGetLastError();
}

// Merge two attention results over disjoint key sets (log-sum-exp):
// o = (e^(l0-l) o0 + e^(l1-l) o1) / (e^(l0-l) + e^(l1-l)), l = max(l0, l1).
// o2: [2][rows][nh*hd] f16 (normalized parts), l2: [2][rows][nh] natural-log LSE.
__global__ void k_lse_merge(const __half* o2, const float* l2, int64_t rows, int nh, int hd, __half* out) {
    const int64_t n = rows * nh * hd;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t rh = i / hd;                        // row * nh + head
        const float l0 = l2[rh], l1 = l2[rows * nh + rh];
        const float mx = fmaxf(l0, l1);
        float v = 0.f;
        if (mx != -INFINITY) {
            const float w0 = expf(l0 - mx), w1 = expf(l1 - mx);
            v = (w0 * __half2float(o2[i]) + w1 * __half2float(o2[rows * nh * hd + i])) / (w0 + w1);
        }
        out[i] = __float2half_rn(v);
    }
}

// [parts][rows][w] -> [rows][parts * w] (all-gathered per-rank head blocks into rows)
__global__ void k_gather_rows(const __half* in, int64_t rows, int parts, int w, __half* out) {
    const int64_t n = rows * parts * w;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / ((int64_t)parts * w);
        const int c = (int)(i % ((int64_t)parts * w)), p = c / w, e = c % w;
        out[i] = in[((int64_t)p * rows + r) * w + e];
    }
}

// x += y (residual add of an all-reduced partial projection)
__global__ void k_add_rows(float* x, const float* y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], y[i]);
}

__global__ void k_half_to_float(const __half* x, float* y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __half2float(x[i]);
}

cudaError_t half_to_float_launch(const __half* x, float* y, int64_t n, cudaStream_t st) {
    k_half_to_float<<<grid_for(n, 256), 256, 0, st>>>(x, y, n);
    note_launch();
    return cudaGetLastError();
}

// ggml_relu and the classifier's sigmoid (src/vibevoice_tts.cpp:522,537)
__global__ void k_act(float* x, int64_t n, int act) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        x[i] = act == ACT_RELU ? fmaxf(v, 0.f) : __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
    }
}

cudaError_t act_launch(float* x, int64_t n, int act, cudaStream_t st) {
    k_act<<<grid_for(n, 256), 256, 0, st>>>(x, n, act);
    note_launch();
    return cudaGetLastError();
}

cudaError_t add_rows_launch(float* x, const float* y, int64_t n, cudaStream_t st) {
    k_add_rows<<<grid_for(n, 256), 256, 0, st>>>(x, y, n);
    note_launch();
    return cudaGetLastError();
}

cudaError_t lse_merge_launch(const __half* o2, const float* l2, int64_t rows, int nh, int hd, __half* out,
                             cudaStream_t st) {
    const int64_t n = rows * nh * hd;
    k_lse_merge<<<grid_for(n, 256), 256, 0, st>>>(o2, l2, rows, nh, hd, out);
    note_launch();
    return cudaGetLastError();
}

cudaError_t gather_rows_launch(const __half* in, int64_t rows, int parts, int w, __half* out, cudaStream_t st) {
    const int64_t n = rows * parts * w;
    k_gather_rows<<<grid_for(n, 256), 256, 0, st>>>(in, rows, parts, w, out);
    note_launch();
    return cudaGetLastError();
}

cudaError_t rope_launch(const float* x, int n_tok, int n_heads, int hd, const int32_t* pos, float ts,
                        float* y, cudaStream_t st) {
    const int64_t n = (int64_t)n_tok * n_heads * (hd / 2);
    k_rope<<<grid_for(n, 256), 256, 0, st>>>(x, n_tok, n_heads, hd, pos, ts, y);
    note_launch();
    return cudaGetLastError();
}

cudaError_t rmsnorm_launch(const float* x, const float* w, int rows, int n, float eps, float* y,
                           cudaStream_t st) {
    k_rmsnorm<<<rows, 256, 0, st>>>(x, w, n, eps, y);
    note_launch();
    return cudaGetLastError();
}

cudaError_t rmsnorm_f16_launch(const float* x, const float* w, int rows, int n, float eps, __half* y,
                               cudaStream_t st) {
    k_rmsnorm_f16<<<rows, 256, 0, st>>>(x, w, n, eps, y);
    note_launch();
    return cudaGetLastError();
}

cudaError_t splitk_resid_rmsnorm_f16_launch(const float* part, int ks, const float* bias, float* x, const float* w,
                                            int rows, int n, float eps, __half* y, cudaStream_t st) {
    k_splitk_resid_rmsnorm_f16<<<rows, 256, 0, st>>>(part, ks, (int64_t)rows * n, bias, x, w, n, eps, y);
    note_launch();
    return cudaGetLastError();
}

cudaError_t rope_table_launch(const RowMeta* meta, int rows, int hd, float ts, float2* cs, cudaStream_t st) {
    const int64_t n = (int64_t)rows * (hd / 2);
    k_rope_table<<<grid_for(n, 256), 256, 0, st>>>(meta, rows, hd / 2, ts, cs);
    note_launch();
    return cudaGetLastError();
}

cudaError_t to_f16_launch(const float* x, int64_t n, __half* y, cudaStream_t st) {
    k_to_f16<<<grid_for(n, 256), 256, 0, st>>>(x, n, y);
    note_launch();
    return cudaGetLastError();
}

cudaError_t embed_launch(const DevW& t, const int32_t* tok, int n, float* out, cudaStream_t st) {
    k_embed<<<n, 256, 0, st>>>(t, tok, n, out);
    note_launch();
    return cudaGetLastError();
}

cudaError_t kv_upload_launch(const KvLayer& kv, int seq, const float* k, const float* v, int n_pos,
                             cudaStream_t st) {
    const int64_t n = (int64_t)n_pos * kv.n_kv * kv.hd;
    if (n == 0) return cudaSuccess;
    k_kv_upload<<<grid_for(n, 256), 256, 0, st>>>(kv, seq, k, v, n_pos);
    note_launch();
    return cudaGetLastError();
}

cudaError_t kv_download_launch(const KvLayer& kv, int seq, float* k, float* v, int n_pos,
                               cudaStream_t st) {
    const int64_t n = (int64_t)n_pos * kv.n_kv * kv.hd;
    if (n == 0) return cudaSuccess;
    k_kv_download<<<grid_for(n, 256), 256, 0, st>>>(kv, seq, k, v, n_pos);
    note_launch();
    return cudaGetLastError();
}

cudaError_t advance_meta_part_launch(RowMeta* meta_true, RowMeta* meta_local, int n, int seq_parts, int part,
                                     cudaStream_t st) {
    k_advance_meta_part<<<1, 32, 0, st>>>(meta_true, meta_local, n, seq_parts, part);
    note_launch();
    return cudaGetLastError();
}

cudaError_t advance_meta_launch(RowMeta* meta, int n, cudaStream_t st) {
    k_advance_meta<<<1, 32, 0, st>>>(meta, n);
    note_launch();
    return cudaGetLastError();
}

cudaError_t argmax_init_launch(unsigned long long* keys, int n, cudaStream_t st) {
    k_argmax_init<<<(n + 127) / 128, 128, 0, st>>>(keys, n);
    note_launch();
    return cudaGetLastError();
}

cudaError_t argmax_rescore_launch(const float* X, const float* norm_w, float eps, int rows, int H, const DevW& w,
                                  const unsigned long long* tile_best, int ntiles, float margin,
                                  unsigned long long* keys, int* err, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_argmax_rescore<<<rows, RS_THREADS, (size_t)H * sizeof(float), st>>>(X, norm_w, eps, H, w, tile_best, ntiles,
                                                                          margin, keys, err);
    note_launch();
    return cudaGetLastError();
}

cudaError_t argmax_final_launch(const unsigned long long* keys, int n, int32_t* out, cudaStream_t st) {
    k_argmax_final<<<(n + 127) / 128, 128, 0, st>>>(keys, n, out);
    note_launch();
    return cudaGetLastError();
}

}  // namespace vvq2
