// kernels.h -- launch interfaces of the sm_100a kernels (host side).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace vvq2 {

void note_launch(int n = 1);   // counts this library's kernel launches

// ---------------------------------------------------------------- GEMV
enum GemvEpi : int {
    EPI_QKV = 0,     // +bias, RoPE Q/K, Q -> y[m][nq*hd], K/V -> paged cache
    EPI_RESID = 1,   // y[m][r] += W.x  (residual add, in place)
    EPI_SWIGLU = 2,  // y[m][i] = silu(W0.x)[i] * (W1.x)[i]
    EPI_STORE = 3,   // y[m][r] = W.x (+bias)
    EPI_ARGMAX = 4   // logits to y (optional) + first-max argmax key to argmax[m]
};

struct GemvArgs {
    DevW w0, w1;
    int M = 0, K = 0, n_units = 0;
    const float* x = nullptr;      // [M][x_stride] f32 activations
    int x_stride = 0;
    const float* norm_w = nullptr; // RMSNorm weight (f32 [K]) or null
    float eps = 0.f;
    int epi = 0;
    const float* bias = nullptr;
    float* y = nullptr;
    int y_stride = 0;
    const RowMeta* meta = nullptr;
    KvLayer kv;
    int n_q_heads = 0, n_kv_heads = 0, hd = 0;
    float rope_ts = 0.f;
    const RowMeta* rope_meta = nullptr;   // RoPE positions if not meta's (a later sequence part)
    unsigned long long* argmax = nullptr;
    int wpu = 1;                   // warps per unit (set by gemv_launch)
};

cudaError_t gemv_launch(GemvArgs a, cudaStream_t st);
size_t gemv_smem_bytes(int wt, int M, int K);
cudaError_t gemv_prepare();
int gemv_max_rows(int K);   // activation rows that fit the GEMV's shared memory

// ------------------------------------------------------ tcgen05 GEMM (prefill)
struct GemmArgs {
    DevW w0, w1;                   // weights; SwiGLU interleaves gate (w0) and up (w1) tiles
    int T = 0, N = 0, K = 0;       // token rows, output features, input dim
    int epi = 0;                   // EPI_QKV / EPI_RESID / EPI_SWIGLU / EPI_STORE
    const float* bias = nullptr;
    float* y = nullptr;            // f32 out: RESID/STORE [T][y_stride]; QKV: Q [T][nq*hd]
    int y_stride = 0;
    __half* yh = nullptr;          // f16 out: SwiGLU [T][yh_stride]
    int yh_stride = 0;
    const RowMeta* meta = nullptr; // per token row
    KvLayer kv;
    int nq = 0, nkv = 0, hd = 0;
    const float2* rope_cs = nullptr;   // [T][hd/2] (cos, sin)
    unsigned long long* amax = nullptr;   // ARGMAX: [T] running (logit, index) keys
    unsigned long long* tile_best = nullptr;   // ARGMAX, optional: [T][tile_stride] best key per 128-column tile
    int tile_stride = 0;
    float* kpart = nullptr;        // split-K: [k_splits][T][N] f32 partials (then splitk_epilogue_launch)
    int k_splits = 1;
    int* err = nullptr;
};
// tmA: f16 activations [T][K], box 64 x 128; weight tiles are dequantized in
// the kernel.  Q8_0 weights also take wq[4], the byte maps gemm_ws_launch
// takes, with box rows 128 (SwiGLU: 64).
cudaError_t gemm_tc_launch(const GemmArgs& a, const CUtensorMap& tmA, const CUtensorMap* wq, cudaStream_t st);
cudaError_t gemm_tc_prepare();
// sum split-K partials in order and apply a.epi (QKV / RESID / STORE)
cudaError_t splitk_epilogue_launch(const GemmArgs& a, cudaStream_t st);

// Persistent many-row GEMM with the weight dequantization fused (gemm_ws.cu):
// QKV / RESID / SWIGLU / STORE epilogues, no split-K.  tmX: f16 activations
// [T][K], box 64 x nt.  Q8_0 weights also take wq[4]: byte maps of the
// repacked rows of w0 and w1 (dims {row_stride, rows}, no swizzle), box
// {64, r} for the quants (wq[0], wq[1]) and {16, r} for the block scales
// (wq[2], wq[3]), r = gemm_ws_weight_box_rows.  gemm_ws_tile_rows picks nt
// for a launch (0: fewer than min_tiles tiles, <= 0 meaning one per SM; use
// gemm_tc_launch).
int gemm_ws_tile_rows(const GemmArgs& a, int min_tiles);
int gemm_ws_weight_box_rows(const GemmArgs& a);
cudaError_t gemm_ws_launch(const GemmArgs& a, const CUtensorMap& tmX, const CUtensorMap* wq, int nt,
                           cudaStream_t st);
cudaError_t gemm_ws_prepare();

// ------------------------------------------------------ peer exchanges (peer.cu)
// Every rank of a partitioned context owns one exchange buffer mapped into
// all ranks: [PEER_HDR bytes: flag (last epoch) per sender][2 parities]
// [PEER_MAX senders][slot_bytes].
constexpr int PEER_MAX = 8;
constexpr int PEER_HDR = 256;
struct PeerArgs {
    int world = 0, rank = 0;
    uint8_t* base[PEER_MAX] = {};        // rank r's buffer as mapped in this process
    int slot_bytes = 0;
    unsigned int* epoch = nullptr;       // exchanges so far (this rank's device counter)
    int* err = nullptr;                  // set to 6 when a wait for a peer runs out
};
inline size_t peer_buffer_bytes(int slot_bytes) { return PEER_HDR + 2 * (size_t)PEER_MAX * slot_bytes; }
// x[0..n) += sum over ranks of part[0..n) (n a multiple of 4)
cudaError_t peer_reduce_add_launch(const PeerArgs& p, const float* part, int n, float* x, cudaStream_t st);
// attention outputs o [M][nq_l*hd] f16 (+ lse [M][nq_l] with two sequence
// parts) of all ranks -> out [M][nq*hd] f32, parts merged by log-sum-exp
int peer_attn_block_bytes(int M, int nq_l, int hd, int seq_parts);
cudaError_t peer_attn_gather_launch(const PeerArgs& p, const __half* o, const float* lse, int M, int nq_l, int hd,
                                    int seq_parts, float* out, cudaStream_t st);

// ------------------------------------------------------ persistent decode step
struct MegaLayer {
    DevW qkv, o, gate, up, down;
    const float* attn_norm = nullptr;
    const float* ffn_norm = nullptr;
    const float* qkv_bias = nullptr;
    KvLayer kv;
};

constexpr int MEGA_MAX_SPLITS = 64;   // attention splits per (row, KV head) of the persistent step

// The persistent step hands values between its stages as flagged words:
// uint64 (tag << 32) | f32 bits, one 64-bit store each (see decode_mega.cu).
struct MegaArgs {
    const MegaLayer* layers = nullptr;   // device array
    int n_layers = 0, H = 0, F = 0, nq = 0, nkv = 0, hd = 0, M = 0, grid = 0;
    DevW lm_head, tok_embd;
    const float* out_norm = nullptr;
    uint64_t* xl = nullptr;              // [M][H] hidden rows
    uint64_t* qkvl = nullptr;            // [M][qkv_rows] raw q|k|v (+bias), before RoPE
    uint64_t* pl = nullptr;              // [M][nkv][MEGA_MAX_SPLITS][nq/nkv][hd + 2] partial O, max, sum
    uint64_t* attl = nullptr;            // [M][nq * hd] attention output
    uint64_t* fal = nullptr;             // [M][F] SwiGLU output
    int qkv_rows = 0;
    RowMeta* meta = nullptr;
    int32_t* tok = nullptr;
    unsigned long long* amax = nullptr;  // [2] running argmax keys, zero between launches
    unsigned int* done = nullptr;        // CTAs that finished the step, zero between launches
    unsigned int* epoch = nullptr;       // launches so far (the tags derive from it)
    int* abort = nullptr;
    int split = 0, nsplit = 0;
    float eps = 0.f, rope_ts = 0.f, scale = 0.f;
    int* err = nullptr;
    unsigned long long* err_info = nullptr;   // [4] where the first failing wait gave up
    // shared-memory plan: [union_bytes: activations | merge scratch, attention
    // at att_off][nstage x slot_bytes ring][stage table]
    int nstage = 0, slot_bytes = 0, union_bytes = 0, att_off = 0;
    int t_qkv = 1, t_o = 1, t_gu = 1, t_down = 1, t_lm = 1;   // weight rows per ring tile
    // optional timeline: [slot][grid] %globaltimer ns of thread 0 of every CTA;
    // slot 0 = start, per layer l slots 1 + 10l + {0: QKV stage begins, 1:
    // QKV input staged, 2: thread 0's QKV tiles done, 3: attention items
    // done (CTA), 4: merges done, 5: O input staged, 6: O tiles done (CTA),
    // 7: gate/up input staged, 8: gate/up tiles done (CTA), 9: down input
    // staged}, then lm_head stage begins, lm_head input staged, copies
    // drained, end
    unsigned long long* trace = nullptr;
};
__host__ __device__ constexpr int mega_trace_slots(int n_layers) { return 10 * n_layers + 5; }
// flagged words of the persistent step for up to 2 rows
__host__ __device__ constexpr size_t mega_ll_words(int H, int qkv_rows, int nq, int hd, int F) {
    return 2 * ((size_t)H + qkv_rows + (size_t)nq * hd + F + (size_t)nq * MEGA_MAX_SPLITS * (hd + 2));
}
cudaError_t decode_mega_prepare();
cudaError_t decode_mega_launch(const MegaArgs& a, size_t smem, cudaStream_t st);
int decode_mega_union_bytes(int hd, int M, int kmax, int H);
int decode_mega_att_offset(int M, int H);
int decode_mega_max_stages();
int decode_mega_consumer_warps();
int decode_mega_table_bytes(int n_layers);
int decode_mega_att_groups();
int decode_mega_smem_limit();
int decode_mega_grid();

// ------------------------------------------------------ decode attention
struct AttnDecodeArgs {
    const float* q = nullptr;      // [M][nq*hd] (roped)
    float* out = nullptr;          // [M][nq*hd]
    const RowMeta* meta = nullptr;
    KvLayer kv;
    int M = 0, nq = 0, nkv = 0, hd = 0;
    int split = 0;                 // keys per CTA
    int max_splits = 0;            // grid.x
    float scale = 0.f;
    float* part = nullptr;         // [M][max_splits][nq][hd] unnormalized partial O
    float* part_ml = nullptr;      // [M][max_splits][nq][2] (running max, sum)
    int* counters = nullptr;       // [M][nkv], zero between launches
    int* err = nullptr;            // set to nonzero if a bounded wait gave up
    __half* out_h = nullptr;       // if set, write f16 output here instead of `out`
    float* lse = nullptr;          // optional [M][nq]: log-sum-exp of the scaled scores (-inf: no keys)
    int defer_merge = 0;           // set by attn_decode_launch: partials only, a merge kernel follows
};
cudaError_t attn_decode_launch(const AttnDecodeArgs& a, cudaStream_t st);
// f16 paged pool [rows][hd] as a TMA map: 64 x 64 boxes, 128-byte swizzle (engine.cu)
bool make_kv_map(CUtensorMap* m, const __half* base, int64_t rows, int hd);
cudaError_t attn_decode_prepare();

// ------------------------------------------------------ prefill attention
struct FaArgs {
    const float* q = nullptr;            // [rows][nq*hd] roped Q, row = seq_slot * nt + t
    __half* out = nullptr;               // [rows][nq*hd]
    const RowMeta* meta = nullptr;
    const int* block_table = nullptr;    // [seq][max_pages]
    int max_pages = 0;
    int kv_rows = 0;                     // rows of the K/V tensor maps (pages * n_kv * 64)
    int n_seqs = 0, nt = 0;              // sequences in the chunk, rows per sequence
    int nq = 0, nkv = 0, hd = 0;
    float scale = 0.f;
    float* lse = nullptr;                // optional [rows][nq]: log-sum-exp of the scaled scores
    int* err = nullptr;
};
cudaError_t fa_prefill_prepare();
// mk / mv: the layer's K / V pool as 2-D f16 [kv_rows][hd], box 64 x 64, 128-byte swizzle
cudaError_t fa_prefill_launch(const FaArgs& a, const CUtensorMap& mk, const CUtensorMap& mv, cudaStream_t st);

// ------------------------------------------------------------- misc
long long launch_count();
// dequantize a repacked device weight matrix to f32 [rows][cols]
cudaError_t dequant_rows_launch(const DevW& w, float* dst, cudaStream_t st);
// log-sum-exp merge of two partial attention outputs over disjoint key sets:
// o2 [2][rows][nh*hd] f16, l2 [2][rows][nh] -> out [rows][nh*hd] f16
cudaError_t lse_merge_launch(const __half* o2, const float* l2, int64_t rows, int nh, int hd, __half* out,
                             cudaStream_t st);
// x += y over n floats
cudaError_t add_rows_launch(float* x, const float* y, int64_t n, cudaStream_t st);
cudaError_t half_to_float_launch(const __half* x, float* y, int64_t n, cudaStream_t st);
// in place: ACT_RELU max(x, 0); ACT_SIGMOID 1 / (1 + expf(-x))
enum { ACT_RELU = 0, ACT_SIGMOID = 1 };
cudaError_t act_launch(float* x, int64_t n, int act, cudaStream_t st);
// [parts][rows][w] -> [rows][parts*w]
cudaError_t gather_rows_launch(const __half* in, int64_t rows, int parts, int w, __half* out, cudaStream_t st);
cudaError_t rope_launch(const float* x, int n_tok, int n_heads, int hd, const int32_t* pos,
                        float ts, float* y, cudaStream_t st);
cudaError_t rmsnorm_launch(const float* x, const float* w, int rows, int n, float eps, float* y,
                           cudaStream_t st);
// RMSNorm to f16 (the tensor-core GEMM's activation operand)
// x[rows][n] += (bias +) the in-order sum of split-K partials part[ks][rows][n],
// then y = f16(RMSNorm(x) * w): a residual GEMM's split-K epilogue fused with
// the RMSNorm that follows it
cudaError_t splitk_resid_rmsnorm_f16_launch(const float* part, int ks, const float* bias, float* x, const float* w,
                                            int rows, int n, float eps, __half* y, cudaStream_t st);
cudaError_t rmsnorm_f16_launch(const float* x, const float* w, int rows, int n, float eps, __half* y,
                               cudaStream_t st);
// NEOX (cos, sin) per (row, pair) with ggml's CPU theta recurrence: [rows][hd/2]
cudaError_t rope_table_launch(const RowMeta* meta, int rows, int hd, float ts, float2* cs, cudaStream_t st);
// f32 -> f16 copy
cudaError_t to_f16_launch(const float* x, int64_t n, __half* y, cudaStream_t st);
// rows of a tok_embd table (any weight type) -> f32 [n][cols]
cudaError_t embed_launch(const DevW& t, const int32_t* tok, int n, float* out, cudaStream_t st);
// f32 [n_pos][n_kv][hd] -> f16 paged cache of one sequence / layer
cudaError_t kv_upload_launch(const KvLayer& kv, int seq, const float* k, const float* v,
                             int n_pos, cudaStream_t st);
cudaError_t kv_download_launch(const KvLayer& kv, int seq, float* k, float* v, int n_pos,
                               cudaStream_t st);
cudaError_t argmax_init_launch(unsigned long long* keys, int n, cudaStream_t st);
// test hook: y [M][rows] = x [M][cols] . W^T on the tensor-core decode GEMV
// math (gemv_mma.cuh), one CTA, M <= 2, Q8_0
cudaError_t debug_gemv_mma_launch(const DevW& w, const float* x, int M, float* y, cudaStream_t st);
// Exact argmax of rows whose lm_head ran on f16 operands: every 128-column
// tile whose best approximate logit lies within `margin` (relative to the
// row's approximate maximum) is rescored in f32 -- RMSNorm of X [rows][H]
// with norm_w, exactly dequantized weights -- and keys[] gets the exact key.
cudaError_t argmax_rescore_launch(const float* X, const float* norm_w, float eps, int rows, int H, const DevW& w,
                                  const unsigned long long* tile_best, int ntiles, float margin,
                                  unsigned long long* keys, int* err, cudaStream_t st);
cudaError_t advance_meta_launch(RowMeta* meta, int n, cudaStream_t st);
// partitioned rows: true rows + 1, this rank's rows derived from them
cudaError_t advance_meta_part_launch(RowMeta* meta_true, RowMeta* meta_local, int n, int seq_parts, int part,
                                     cudaStream_t st);
cudaError_t argmax_final_launch(const unsigned long long* keys, int n, int32_t* out,
                                cudaStream_t st);

}  // namespace vvq2
