// common.cuh -- shared device types and helpers for the sm_100a Qwen2 path.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vvq2 {

// ggml_type ids of the weight formats on this path
enum WType : int { W_F32 = 0, W_F16 = 1, W_Q8_0 = 8, W_Q5_K = 13, W_Q6_K = 14 };

constexpr int QK8_0 = 32;
constexpr int QK_K = 256;
constexpr int KV_PAGE = 64;        // positions per KV page
constexpr int GEMV_MAX_M = 8;      // activation rows handled by the decode GEMV
constexpr int Q5K_BYTES = 176;     // GGUF block_q5_K, kept as-is on device
constexpr int Q6K_PACKED = 208;    // block_q6_K without its trailing d (ql|qh|scales)

// A weight matrix on the device, repacked for 16-byte aligned rows.
//   Q8_0 : q = int8 [rows][cols],            d = f16 [rows][cols/32]
//   Q5_K : q = block_q5_K [rows][cols/256],  d = unused
//   Q6_K : q = (ql|qh|scales) [rows][cols/256] x 208 B, d = f16 [rows][cols/256]
//   F32  : q = float [rows][cols]; F16 : q = half [rows][cols]
struct DevW {
    int type = -1;
    int rows = 0, cols = 0;
    const uint8_t* q = nullptr;
    const __half* d = nullptr;     // block scales: row r at d + r * d_stride
    int64_t row_stride = 0;        // bytes per row of q
    int64_t d_stride = 0;          // halves per row of d
};

// Per activation row (token of a sequence) metadata for the decode/prefill step.
struct RowMeta {
    int seq;    // KV sequence id
    int pos;    // absolute position (RoPE, causal limit: keys j <= pos).  A rank that
                // holds one sequence part sees the cache index of its last key at or
                // before the position here (zz_local_row) and gets RoPE from its own table
    int cidx;   // cache index the new K/V row is written to (< 0: another rank stores it)
    int kvlen;  // keys present after the step's writes (past_len + n_tok)
};

// f16 paged KV cache of one layer: pool[page][kv_head][KV_PAGE][head_dim]
struct KvLayer {
    __half* k = nullptr;
    __half* v = nullptr;
    const int* block_table = nullptr;   // [n_seqs][max_pages]
    int max_pages = 0;
    int n_kv = 0;
    int hd = 0;
    int n_pages = 0;                    // pages in the pool (0: unknown)
};

// Sequence parts of a partitioned context interleave whole pages: page p of
// every sequence belongs to part (0, 1, 1, 0)[p % 4], so each part holds
// half of every 256-position span and a causal prompt of any length (and any
// chunking) gives both parts the same attention work -- keys early in the
// sequence are seen by more queries, and each part holds as many early as
// late keys.  A part stores its positions in order: position p sits at cache
// index zz_count(part, p), the number of the part's positions below p.
__host__ __device__ inline int zz_part(int p) { return ((p / KV_PAGE) % 4 == 1 || (p / KV_PAGE) % 4 == 2) ? 1 : 0; }
__host__ __device__ inline int zz_count(int part, int n) {
    const int period = 4 * KV_PAGE, full = n / period, rem = n % period;
    int c = full * (period / 2);
    for (int j = 0; j < 4; ++j) {
        const int inpage = rem - j * KV_PAGE;
        if (zz_part(j * KV_PAGE) == part) c += inpage < 0 ? 0 : (inpage > KV_PAGE ? KV_PAGE : inpage);
    }
    return c;
}
// A row (true position, cache index, key count) as part `part` sees it: pos
// becomes the cache index of the part's last position <= pos (-1 if none),
// so the kernels' causal limit min(pos + 1, kvlen) counts exactly the part's
// keys at positions <= pos; kvlen the part's positions below kvlen; cidx < 0
// when the other part stores the row.
__host__ __device__ inline RowMeta zz_local_row(RowMeta r, int part) {
    RowMeta l = r;
    l.pos = zz_count(part, r.pos + 1) - 1;
    l.cidx = zz_part(r.cidx) == part ? zz_count(part, r.cidx) : -1;
    l.kvlen = zz_count(part, r.kvlen);
    return l;
}

__device__ __forceinline__ size_t kv_offset(const KvLayer& kv, int seq, int cidx, int kvh) {
    const int page = __ldg(kv.block_table + (size_t)seq * kv.max_pages + cidx / KV_PAGE);
    return (((size_t)page * kv.n_kv + kvh) * KV_PAGE + (cidx % KV_PAGE)) * (size_t)kv.hd;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ggml_silu_f32: x / (1 + expf(-x)), evaluated without contraction
__device__ __forceinline__ float silu_ref(float x) {
    return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

// The same function with the fast exponential and divide intrinsics (a few
// ulp of f32), for epilogues whose output is rounded to f16 at once (2^-11):
// the tensor-core GEMMs' SwiGLU.  Large -x: the divisor is inf and the
// result 0; large x: x.
__device__ __forceinline__ float silu_f16out(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// NEOX rotation of the pair (x0, x1) = (x[i], x[i + hd/2]) at position pos,
// with ggml's CPU theta cache: theta_0 = pos, theta_{k+1} = theta_k * ts
// (ggml_rope_cache_init), ts = powf(theta_base, -2/hd) computed on the host.
__device__ __forceinline__ void rope_pair(float& x0, float& x1, int pos, int i, float ts) {
    float th = (float)pos;
    for (int k = 0; k < i; ++k) th = __fmul_rn(th, ts);
    float s, c;
    s = sinf(th);
    c = cosf(th);
    const float a = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    const float b = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    x0 = a;
    x1 = b;
}

// Orderable packing of (logit, index) for a first-maximum argmax with one
// 64-bit atomicMax: larger logit wins, ties go to the smaller index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (uint32_t)(0x7fffffff - idx);
}

__device__ __forceinline__ int argmax_key_index(unsigned long long k) {
    return 0x7fffffff - (int)(uint32_t)(k & 0xffffffffu);
}

}  // namespace vvq2
