/*
 * vvq2_capi.h -- flat C ABI of the B200 (sm_100a) Qwen2 attention hot path.
 *
 * This library replaces, for vibevoice.cpp's Qwen2 language model, the ggml
 * graph that src/qwen2.cpp builds per layer and that src/backend.cpp runs.
 * Signatures use plain pointers and sizes only (no ggml, no torch types) so a
 * purego / dlopen / ctypes caller binds them by name, in the style of
 * include/vibevoice_capi.h.
 *
 * Conventions (mirroring include/vibevoice.h:23-33 vv_status):
 *   - every int-returning entry point returns 0 on success or a negative
 *     status; vvq2_last_error() gives a message for the calling thread.
 *   - no callee-allocated host memory; outputs go to caller-owned buffers.
 *   - a context is bound to one CUDA device; it is thread-compatible, not
 *     thread-safe (one caller thread at a time per context).
 *   - activation / output pointers may be host or device memory; the library
 *     detects which (cudaPointerGetAttributes) and copies as needed.
 *   - `stream` is a cudaStream_t (NULL = the context's own stream).  Calls are
 *     synchronous with respect to host outputs: when a host pointer is written,
 *     the call returns after the data has landed.
 *   - there is no CPU fallback: without an sm_100 device every compute entry
 *     point fails with VVQ2_ERR_NO_DEVICE.
 */
#ifndef VVQ2_CAPI_H
#define VVQ2_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes: values shared with vv_status (include/vibevoice.h:23-33) */
enum {
    VVQ2_OK                  = 0,
    VVQ2_ERR_GENERIC         = -1,
    VVQ2_ERR_INVALID_ARG     = -2,   /* includes KV-cache overflow (the reference
                                        GGML_ASSERTs at src/qwen2.cpp:269)      */
    VVQ2_ERR_OUT_OF_MEMORY   = -5,
    VVQ2_ERR_NOT_IMPLEMENTED = -6,
    VVQ2_ERR_CUDA            = -9,
    VVQ2_ERR_NO_DEVICE       = -10
};

/* weight formats accepted: ggml_type ids */
enum {
    VVQ2_TYPE_F32  = 0,
    VVQ2_TYPE_F16  = 1,
    VVQ2_TYPE_Q8_0 = 8,
    VVQ2_TYPE_Q5_K = 13,
    VVQ2_TYPE_Q6_K = 14
};

/* vvq2_forward flags */
enum {
    VVQ2_ADVANCE     = 1 << 0,  /* grow each sequence's past_len by n_tok after the step
                                   (run_qwen2_stack does this, src/vibevoice_tts.cpp:459) */
    VVQ2_OUTPUT_NORM = 1 << 1,  /* apply output_norm (set by vvq2_set_output) at the end
                                   (src/vibevoice_tts.cpp:410-412)                        */
    VVQ2_LAST_ONLY   = 1 << 2   /* y holds only the last token of each sequence
                                   (out_hidden_last, src/vibevoice_tts.cpp:451-456)       */
};

/* Qwen2Hparams (src/qwen2.hpp:24-39) plus the stack-level sizes. */
typedef struct vvq2_hparams {
    int   hidden_size;
    int   n_heads;
    int   n_kv_heads;
    int   head_dim;
    int   intermediate_size;
    int   n_layers;
    int   vocab_size;        /* 0 when no lm_head is used */
    float rope_theta;        /* 1e6 for Qwen2 (src/rope.hpp:15) */
    float rms_norm_eps;      /* 1e-6 */
} vvq2_hparams;

/* One GGUF tensor as the model loader holds it (src/model_loader.cpp:21-110):
 * raw bytes of `type` blocks in HOST memory, ne0 = contiguous (input) dim,
 * ne1 = rows (output) dim.  1-D tensors (norms, biases) use ne1 = 1.
 * data == NULL marks an absent optional tensor (q/k/v biases). */
typedef struct vvq2_tensor {
    const void* data;
    int         type;
    int64_t     ne0;
    int64_t     ne1;
} vvq2_tensor;

/* Qwen2LayerWeights (src/qwen2.hpp:41-54), same field names. */
typedef struct vvq2_layer_weights {
    vvq2_tensor attn_norm, attn_q, attn_q_bias, attn_k, attn_k_bias, attn_v, attn_v_bias,
                attn_o, ffn_norm, ffn_gate, ffn_up, ffn_down;
} vvq2_layer_weights;

typedef struct vvq2_ctx vvq2_ctx;
typedef struct vvq2_kv  vvq2_kv;

/* ---- context / weights ------------------------------------------------ */

/* Creates a context on CUDA `device` (an sm_100 GPU).  Replaces the
 * process-wide backend() singleton for this path (src/backend.cpp:64-134). */
int  vvq2_init(const vvq2_hparams* hp, int device, vvq2_ctx** out);
void vvq2_free(vvq2_ctx* ctx);

/* Uploads one layer's weights (host GGUF blocks) to device memory, repacked
 * for coalesced 16-byte loads; dequantized values are unchanged.  Replaces
 * qwen2_load_layer (src/qwen2.cpp:44-75).  attn_q/k/v must share one type. */
int  vvq2_set_layer(vvq2_ctx* ctx, int layer, const vvq2_layer_weights* w);

/* Final norm, lm_head and token-embedding tables (any may be NULL).  A tied
 * model passes the same tensor as lm_head and tok_embd. */
int  vvq2_set_output(vvq2_ctx* ctx, const vvq2_tensor* output_norm,
                     const vvq2_tensor* lm_head, const vvq2_tensor* tok_embd);

/* ---- resident KV cache ------------------------------------------------ */

/* ResidentKV::init (src/qwen2.cpp:207-229) for n_seqs sequences (a CFG
 * cond/uncond pair is n_seqs = 2) of up to max_seq positions, every layer.
 * Storage is an f16 paged cache (64-position pages) on the context's device. */
int  vvq2_kv_init(vvq2_ctx* ctx, int n_seqs, int max_seq, vvq2_kv** out);
/* The same cache backed by a shared pool of pool_pages 64-position pages
 * (per layer) instead of n_seqs * ceil(max_seq / 64): a sequence takes pages
 * as its writes need them (vvq2_forward, vvq2_decode_step, load_prefix,
 * set_past_len to a longer length) and gives back the pages past a shorter
 * vvq2_kv_set_past_len.  A write that finds too few free pages fails with
 * VVQ2_ERR_OUT_OF_MEMORY and changes nothing.  This sizes memory by the
 * tokens actually held, as the reference's per-sequence ResidentKV
 * allocation does (src/qwen2.cpp:207-246), for many ragged streams. */
int  vvq2_kv_init_paged(vvq2_ctx* ctx, int n_seqs, int max_seq, int pool_pages, vvq2_kv** out);
/* Free pages of a paged cache (0 for an unpaged one). */
int  vvq2_kv_free_pages(const vvq2_kv* kv);
void vvq2_kv_free(vvq2_kv* kv);

/* Uploads a K/V prefix for one sequence and layer in the voice-GGUF layout
 * F32 [hd, n_kv, n_pos] (scripts/convert_voice_to_gguf.py:17-21; uploaded at
 * src/vibevoice_tts.cpp:735-749), converting to f16 (round to nearest even).
 * Positions [0, n_pos) are overwritten; past_len is not changed. */
int  vvq2_kv_load_prefix(vvq2_kv* kv, int seq, int layer, const float* k,
                         const float* v, int n_pos);
/* Reads positions [0, n_pos) back as f32 in the same layout (tests). */
int  vvq2_kv_read(vvq2_kv* kv, int seq, int layer, float* k, float* v, int n_pos);
int  vvq2_kv_set_past_len(vvq2_kv* kv, int seq, int past_len);
int  vvq2_kv_past_len(const vvq2_kv* kv, int seq);

/* ---- the hot path ----------------------------------------------------- */

/* Runs layers [first_layer, first_layer + n_layers) of the Qwen2 stack for
 * n_seqs sequences (`seqs`, distinct ids) with n_tok new tokens each.
 *   x : f32 [n_seqs][n_tok][hidden]   input hidden states (embeddings)
 *   pos_start[s] : absolute position of sequence s's first new token; RoPE and
 *       the causal mask (key j visible iff j <= pos) use pos_start[s] + t
 *   y : f32 [n_seqs][n_tok][hidden], or [n_seqs][hidden] with VVQ2_LAST_ONLY
 * New K/V rows land at each sequence's past_len (src/qwen2.cpp:289-306).
 * Per layer: RMSNorm -> QKV (+bias) -> NEOX RoPE -> f16 KV append -> GQA
 * flash attention -> O-proj + residual -> RMSNorm -> SwiGLU FFN + residual
 * (qwen2_layer_forward_resident, src/qwen2.cpp:250-359).  Replaces the
 * per-step graph of run_qwen2_stack (src/vibevoice_tts.cpp:363-464) and the
 * ASR prefill/decode loops (src/vibevoice_asr.cpp:554-652, :745-796).
 * Returns VVQ2_ERR_INVALID_ARG (and changes nothing) if any sequence would
 * overflow max_seq. */
int  vvq2_forward(vvq2_ctx* ctx, vvq2_kv* kv, const int* seqs, int n_seqs, int n_tok,
                  const float* x, const int* pos_start, int first_layer, int n_layers,
                  int flags, float* y, void* stream);

/* lm_head over n hidden rows (already output-normed): logits (optional,
 * f32 [n][vocab]) and first-maximum argmax ids (lm_head_logits_last and the
 * greedy pick, src/vibevoice_asr.cpp:285-311,702-706). */
int  vvq2_lm_head(vvq2_ctx* ctx, int n, const float* h, float* logits, int32_t* argmax,
                  void* stream);

/* ---- per-frame heads around the stack (src/vibevoice_tts.cpp:464-537) ----
 * SpeechConnector: y = fc2(rms_norm(fc1(x) + b1) * norm) + b2, eps 1e-6
 * (run_speech_connector): x f32 [batch][latent] -> y f32 [batch][hidden];
 * fc1 has ne0 = latent, ne1 = hidden; fc2 ne0 = ne1 = hidden; biases are
 * optional (data == NULL).  EOS classifier: p = sigmoid(fc2(relu(fc1(x) + b1))
 * + b2) (run_eos_classifier): x f32 [batch][hidden] -> p f32 [batch]; fc1 has
 * ne0 = hidden, ne1 = inner; fc2 ne0 = inner, ne1 = 1.  Weights in any type
 * the layers take (F32, F16, Q8_0, Q5_K, Q6_K); input dims must be multiples
 * of 16 (32 for Q8_0, 256 for K-quants); batch <= 8.  x, y and p may be host
 * or device pointers; with a host output the call returns when it is written. */
int  vvq2_set_connector(vvq2_ctx* ctx, const vvq2_tensor* fc1_w, const vvq2_tensor* fc1_b,
                        const vvq2_tensor* norm_w, const vvq2_tensor* fc2_w, const vvq2_tensor* fc2_b);
int  vvq2_connector(vvq2_ctx* ctx, const float* x, int batch, float* y, void* stream);
int  vvq2_set_eos(vvq2_ctx* ctx, const vvq2_tensor* fc1_w, const vvq2_tensor* fc1_b,
                  const vvq2_tensor* fc2_w, const vvq2_tensor* fc2_b);
int  vvq2_eos(vvq2_ctx* ctx, const float* x, int batch, float* p, void* stream);

/* Token-embedding rows (dequantized tok_embd rows), f32 [n][hidden]. */
int  vvq2_embed(vvq2_ctx* ctx, int n, const int32_t* tokens, float* out, void* stream);

/* One greedy decode step of the whole LM for n_seqs sequences (1 token each):
 * embed(tokens_in) -> all layers -> output_norm -> lm_head -> argmax ->
 * tokens_out; past_len advances by 1.  Equivalent to the ASR decode loop body
 * (src/vibevoice_asr.cpp:665-801) without penalties. */
int  vvq2_decode_step(vvq2_ctx* ctx, vvq2_kv* kv, const int* seqs, int n_seqs,
                      const int32_t* tokens_in, int32_t* tokens_out, void* stream);

/* ---- standalone pieces (rope.hpp / rms_norm.hpp equivalents, tests) --- */

/* Dequantizes n elements of GGUF `type` blocks with the same device routine
 * the GEMV/GEMM producers use (bit-exact with ggml dequantize_row_*). */
int  vvq2_dequantize(int type, const void* src, int64_t n, float* dst);
/* NEOX RoPE over x f32 [n_tok][n_heads][head_dim] at positions pos[n_tok]
 * (ggml_rope_ext, GGML_ROPE_TYPE_NEOX; src/rope.hpp:4-15). */
int  vvq2_rope_neox(const float* x, int n_tok, int n_heads, int head_dim, const int32_t* pos,
                    float theta, float* y);
/* y = x / sqrt(mean(x^2) + eps) * w over rows of n (src/rms_norm.hpp:11-17). */
int  vvq2_rms_norm(const float* x, const float* w, int rows, int n, float eps, float* y);

/* ---- backend selection (src/backend.cpp:64-127) ----------------------- */

/* 1 if VIBEVOICE_BACKEND selects this path ("b200" or "vvq2", case-insensitive)
 * and an sm_100 device is present, else 0.  backend.cpp calls this first. */
int  vvq2_backend_selected(void);
/* Number of sm_100 devices visible. */
int  vvq2_device_count(void);

const char* vvq2_version(void);
const char* vvq2_last_error(void);
/* Number of this library's kernels launched so far in this process (bench). */
int64_t vvq2_kernel_launches(void);

/* ---- test hook (no counterpart in the reference) ----------------------
 * y f32 [t][n] = x [t][k] . W[n][k]^T through the tensor-core (tcgen05) GEMM
 * used for prefill: x rounded to f16, W (host GGUF blocks of `type`)
 * dequantized exactly and rounded to f16, f32 accumulation.  k % 64 == 0. */
int  vvq2_debug_gemm(int type, const void* w, int n, int k, const float* x, int t, float* y);

/* ---- test hook (no counterpart in the reference) ----------------------
 * y f32 [m][n] = x [m][k] . W[n][k]^T for m <= 2 rows through the
 * tensor-core decode GEMV math of the persistent step (Q8_0 weights exact,
 * x split into three int8 pieces per 32-block, s32 block sums).  k % 32 == 0. */
int  vvq2_debug_gemv_mma(const void* w, int n, int k, const float* x, int m, float* y);

/* ---- allocation-free decode attention (no counterpart in the reference) --
 * For callers that cannot call cudaMalloc -- an engine whose pool owns all GPU
 * memory, code inside another framework's context or a graph capture, a
 * real-time thread that must not enter the allocator: the split-K decode
 * attention of this library with its scratch (partial O, per-split max/sum,
 * arrival counters, error word) in one fixed file-scope device array instead
 * of allocations.  The caller passes device pointers it owns:
 *   q          f32 [n_rows][n_heads*head_dim], RoPE already applied
 *   k_pages,
 *   v_pages    f16 pages [page][n_kv_heads][64][head_dim]
 *   block_table int32 [seq][max_pages] logical -> physical page
 *   row_meta   int32 [n_rows][4] = {seq, pos, (unused), kv_len}; keys j < kv_len
 *              with j <= pos are attended
 *   max_kv     an upper bound of every row's kv_len (sizes the split grid); a
 *              row with more keys than max_kv (or than its block-table row
 *              holds) is clamped to the first keys and sets error word 5
 *   out        f32 [n_rows][n_heads*head_dim]
 *   err_out    int the caller owns (device memory, or pinned / managed host
 *              memory), or NULL: receives the kernels' error word in stream
 *              order -- 0 ok, 1 a bounded wait gave up (out is not valid),
 *              5 a row was clamped.  A return of 0 only says the work was
 *              enqueued; read *err_out after the stream has finished.
 * Limits: n_rows <= 8, n_heads*head_dim <= 4096, n_heads <= 64, n_kv_heads
 * <= 16, head_dim 32/64/128, n_heads/n_kv_heads <= 8; beyond them it returns
 * VVQ2_ERR_INVALID_ARG.  The array (about 2.1 MB) stays allocated on every GPU
 * that loads the library until exit.  Calls share it: calls that overlap on
 * the GPU race and must be serialized by the caller.  Every call looks up the
 * array's device address (cudaGetSymbolAddress) in the calling thread's
 * current context; the first call in a context loads the library's module
 * there, so make it before any stream capture.  Allocates nothing. */
int  vvq2_attention_decode_noalloc(const float* q, const void* k_pages, const void* v_pages,
                                   const int* block_table, int max_pages, const int* row_meta,
                                   int n_rows, int max_kv, int n_heads, int n_kv_heads,
                                   int head_dim, float* out, int* err_out, void* stream);

/* ---- measurement (no counterpart in the reference, which has no profiler
 * hooks; used by bench.py for the roofline figures) ------------------------
 * While enabled, vvq2_decode_step brackets the persistent decode-step kernel
 * or every GEMV (kind 0) and attention (kind 1) launch, vvq2_forward on the
 * tensor-core path every flash-attention (kind 2) and GEMM (kind 3) launch,
 * and a decode step of many rows (tensor-core path) its split-K attention
 * (kind 1) and GEMM (kind 3) launches,
 * with CUDA events on the launching stream; per kind it accumulates device
 * time, algorithmic work (bytes for kinds 0/1, flops for kinds 2/3) and
 * launch counts.  Enabling resets the totals. */
int  vvq2_profile(vvq2_ctx* ctx, int enable);
int  vvq2_profile_read(vvq2_ctx* ctx, int kind, double* ms, double* bytes, int64_t* launches);

/* ---- multi-GPU partition of the attention (config 5: long-context ASR) ----
 * No reference counterpart (the reference runs one process on one device).
 * One context per GPU and process.  `world` = head_groups x seq_parts ranks;
 * rank r holds KV-head group r / seq_parts (the QKV rows and attention of its
 * q heads) and sequence part r % seq_parts of every sequence's keys (part 1
 * starts at a page-aligned split fixed by the sequence's first write: half
 * of it).  Each rank computes normalized attention output and its
 * log-sum-exp over its keys; the two parts of a head group merge (O, LSE)
 * through an NCCL all-gather, head groups all-gather the output rows, O-proj
 * runs replicated, the FFN is split over all ranks (gate/up rows, down
 * columns; intermediate_size / world must be a multiple of 64 and of the
 * down weight's block size) with an NCCL
 * all-reduce of the down projection, and final norm and lm_head run
 * replicated, so every rank returns the same hidden states and tokens.  Call after vvq2_init and before
 * vvq2_set_layer / vvq2_kv_init, on all ranks at once (NCCL init is
 * collective); every rank must then make the same calls with the same
 * inputs.  `nccl_id`: VVQ2_NCCL_ID_BYTES from vvq2_nccl_unique_id on one
 * rank, shared with the others by the host. */
#define VVQ2_NCCL_ID_BYTES 128
int  vvq2_nccl_unique_id(void* out);
int  vvq2_partition(vvq2_ctx* ctx, int rank, int world, int seq_parts, const void* nccl_id);

/* Phase timeline of the persistent decode-step kernel (no reference
 * counterpart).  With VVQ2_MEGA_TRACE=1 in the environment when a decode
 * graph is built, every CTA stamps %globaltimer (ns) at kernel start, at
 * arrival at / release from each grid barrier, and at the end of the last
 * step.  Layout [slots][grid]: slot 0 start, 1+2b arrive b, 2+2b release b,
 * slots-1 end.  `out` may be null to query grid and slots only. */
int  vvq2_mega_trace(vvq2_ctx* ctx, uint64_t* out, int64_t cap, int* grid, int* slots);

#ifdef __cplusplus
}
#endif
#endif /* VVQ2_CAPI_H */
