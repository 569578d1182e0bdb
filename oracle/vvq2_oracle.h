/*
 * vvq2_oracle.h -- CPU restatement of the vibevoice.cpp Qwen2 layer math.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the sm_100a
 * product path: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg may load it.  The product library
 * (libvvq2.so) never links, loads or calls anything in this directory.
 *
 * What it restates (reference paths are relative to the vibevoice.cpp tree):
 *   - layer order of qwen2_layer_forward_resident      src/qwen2.cpp:250-359
 *   - RMSNorm  y = x / sqrt(mean(x^2)+eps) * w        src/rms_norm.hpp:11-17
 *   - NEOX RoPE, theta 1e6                             src/rope.hpp:14-15,
 *                                                      src/qwen2.cpp:282-287
 *   - Q/K/V/O linear + optional bias                   src/qwen2.cpp:19-26,274-276,349
 *   - GQA flash attention, scale 1/sqrt(hd), causal    src/qwen2.cpp:324-335,
 *     mask j > pos -> -inf                             src/vibevoice_tts.cpp:432-441
 *   - SwiGLU FFN                                       src/qwen2.cpp:33-40,351-355
 *   - resident KV append at past_len                   src/qwen2.cpp:289-317
 *   - lm_head + first-max argmax                       src/vibevoice_asr.cpp:285-311,702-706
 * and, because the arithmetic lives in ggml (a git submodule that is empty in
 * the reference tree, pin unknown), the published ggml algorithms the graph
 * nodes above dispatch to on the CPU backend:
 *   dequantize_row_q8_0 / q5_K / q6_K, quantize_row_q8_0_ref,
 *   quantize_row_q8_K_ref, ggml_vec_dot_{q8_0_q8_0,q5_K_q8_K,q6_K_q8_K,f16,f32}
 *   (generic C versions), ggml_compute_forward_rms_norm_f32, the NEOX branch of
 *   ggml_compute_forward_rope_f32 with ggml_rope_cache_init's iterated theta,
 *   ggml_compute_forward_flash_attn_ext_f16_one_chunk (online softmax with an
 *   F16 V accumulator when V is F16), and ggml_vec_swiglu_f32.
 * Dequantisation is pinned bit-exactly against gguf-py's numpy dequantizers
 * (tests/golden/); RoPE against the reference's dump_rope_reference.py; the
 * f32 layer against the reference's dump_qwen2_reference.py (HF Qwen2 layer).
 */
#ifndef VVQ2_ORACLE_H
#define VVQ2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type ids for the weight formats on this path */
enum { VVO_F32 = 0, VVO_F16 = 1, VVO_Q8_0 = 8, VVO_Q5_K = 13, VVO_Q6_K = 14 };

/* numeric-mode flags */
enum {
    VVO_ACT_GGML   = 1 << 0, /* activations quantized to the weight's vec_dot_type
                                (Q8_0 / Q8_K / F16) and integer dots, as ggml CPU;
                                else exact f32 activations, double accumulation */
    VVO_KV_F16     = 1 << 1, /* K/V stored rounded to f16 (else f32)            */
    VVO_Q_F16      = 1 << 2, /* Q rounded to f16 before Q.K (ggml FA converts Q) */
    VVO_FA_F16ACC  = 1 << 3, /* ggml CPU FA: V accumulated in an f16 buffer      */
    VVO_ROPE_GGML  = 1 << 4, /* theta_i by iterated f32 product (ggml CPU cache)
                                else exact double pos*theta^(-2i/d)              */
    VVO_NO_FFN     = 1 << 5, /* attention half only (y = x + O(attn))            */
    VVO_SIMD       = 1 << 6  /* with VVO_ACT_GGML: Q8_0 x Q8_0 dots by the SIMD
                                integer kernel (AVX-512 VNNI when the CPU has
                                it, else AVX2), as ggml's x86 backend runs them:
                                same integer block sums, different float
                                summation order than the generic dot.  For the
                                timed CPU baseline; parity uses the generic one */
};

/* The SIMD instruction set VVO_SIMD uses on this CPU: "avx512vnni", "avx2"
 * or "generic" (no SIMD kernel available: the generic dot runs). */
const char* vvo_simd_isa(void);

typedef struct vvo_hparams {
    int   hidden, n_heads, n_kv_heads, head_dim, ffn, n_layers, vocab;
    float rope_theta, rms_eps;
} vvo_hparams;

/* A GGUF tensor exactly as the model loader hands it over: raw block bytes,
 * ggml type id, ne0 = contiguous (input) dim, ne1 = rows (output) dim. */
typedef struct vvo_tensor {
    const void* data;
    int         type;
    int64_t     ne0, ne1;
} vvo_tensor;

typedef struct vvo_layer {
    vvo_tensor attn_norm, attn_q, attn_q_bias, attn_k, attn_k_bias, attn_v,
               attn_v_bias, attn_o, ffn_norm, ffn_gate, ffn_up, ffn_down;
} vvo_layer;

/* ---- scalar helpers ---- */
uint16_t vvo_fp32_to_fp16(float f);
float    vvo_fp16_to_fp32(uint16_t h);
size_t   vvo_row_bytes(int type, int64_t n);   /* bytes of one row of n elements */
int      vvo_block_elems(int type);

/* ---- quantization formats ---- */
int vvo_dequantize(int type, const void* src, int64_t n, float* dst);
int vvo_quantize_q8_0(const float* src, int64_t n, void* dst);   /* ggml _ref */
int vvo_quantize_q8_K(const float* src, int64_t n, void* dst);   /* ggml _ref */
/* test-weight generators for the K-quants (own scale choice; parity is
 * defined on the produced bytes, not on ggml's scale search) */
int vvo_quantize_q5_K(const float* src, int64_t n, void* dst);
int vvo_quantize_q6_K(const float* src, int64_t n, void* dst);

/* y[r] = W[r,:] . x  for r in [0, rows)   (ggml_mul_mat of one activation row) */
int vvo_matvec(const vvo_tensor* w, const float* x, float* y, int flags);

/* ---- elementwise pieces ---- */
void vvo_rms_norm(const float* x, const float* w, int n, float eps, float* y);
void vvo_rope_neox(const float* x, int n_heads, int hd, int pos, float theta,
                   int flags, float* y);

/* ---- stateful model (mirrors ResidentKV + the stack drivers) ---- */
typedef struct vvo_model vvo_model;

vvo_model* vvo_model_new(const vvo_hparams* hp, int n_rows, int max_seq, int flags);
void       vvo_model_free(vvo_model* m);
int        vvo_model_set_layer(vvo_model* m, int layer, const vvo_layer* w);
int        vvo_model_set_output(vvo_model* m, const vvo_tensor* output_norm,
                                const vvo_tensor* lm_head, const vvo_tensor* tok_embd);
/* K/V prefix for one row/layer in the voice-GGUF layout [n_pos][n_kv][hd] f32 */
int        vvo_kv_load(vvo_model* m, int row, int layer, const float* k,
                       const float* v, int n_pos);
int        vvo_kv_read(const vvo_model* m, int row, int layer, float* k, float* v,
                       int n_pos);
int        vvo_set_past_len(vvo_model* m, int row, int past_len);
int        vvo_past_len(const vvo_model* m, int row);
/* Runs layers [first, first+n_layers) on n_sel rows (indices `rows`), n_tok
 * new tokens each, at absolute positions pos_start[r] + i.  x, y are
 * [n_sel][n_tok][hidden].  New K/V land at each row's past_len; if `advance`
 * the row's past_len grows by n_tok afterwards.  output_norm applied if asked. */
int        vvo_forward(vvo_model* m, int n_sel, const int* rows, int n_tok,
                       const float* x, const int* pos_start, int first_layer,
                       int n_layers, int apply_output_norm, int advance, float* y);
int        vvo_lm_head(vvo_model* m, int n, const float* h, float* logits, int* argmax);
int        vvo_embed(vvo_model* m, int n, const int* tok, float* out);

#ifdef __cplusplus
}
#endif
#endif
