/* Test infrastructure only: CPU restatement of the gten compute path of
 * iangitonga/nanochatllms.cpp (the "oracle"). Parity tests, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py use it as the checker; the product never links it.
 *
 * Every function restates one reference function and cites it (paths are relative to the
 * reference project root). Floating-point evaluation order, including the SIMD lane
 * structure of the reference's AVX build, is reproduced operation by operation, so results
 * are bit-identical with the reference build on the same inputs (pinned by tests against the
 * compiled reference and the committed golden vectors).
 *
 * dtype codes follow gten::Dtype (src/gten/gten_types.h:20-26):
 *   0 Int32, 1 Float16, 2 Float32, 3 Qint8, 4 Qint4.
 */
#ifndef GTEN_ORACLE_H
#define GTEN_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OR_I32 = 0, OR_F16 = 1, OR_F32 = 2, OR_Q8 = 3, OR_Q4 = 4 };

/* bytes of one row of `n` elements in dtype `dt` (block-aware, partial last Q8 block). */
long or_row_bytes(int dt, int n);

float or_fp16_to_fp32(uint16_t h);
uint16_t or_fp32_to_fp16(float f);

/* activation quantizer and row codecs */
void or_q8_quantize_row(const float* x, void* out, int n);
void or_read_row(const void* row, int dt, float* out, int n);
void or_write_row(const float* x, void* row, int dt, int n);

/* offline weight packer (the reference's Python q8_quantize/q4_quantize) */
void or_pack_q8(const float* w, int rows, int cols, void* out);
void or_pack_q4(const float* w, int rows, int cols, void* out);

/* dot products; order = 0 reference order, 1 per-block-sum order (fast tensor-core path) */
float or_vec_dot(const void* a, int adt, const void* b, int bdt, int n, int order);

/* ops (src/gten/ops.h) on contiguous row-major host buffers */
void or_matmul_2d(const void* x, int xdt, int n_ctx, int n_embd, const void* w, int wdt, int n_out,
                  void* out, int odt, int start_pos, int out_1d, int order);
void or_rms_norm(const void* x, int dt, int n_ctx, int n_embd, const uint16_t* w, void* out, int start_pos);
void or_rms_norm_3d(const void* x, int dt, int n_ctx, int n_heads, int d_head, const uint16_t* w, void* out,
                    int start_pos);
void or_layer_norm(const void* x, int dt, int n_ctx, int n_embd, const uint16_t* w, const uint16_t* b,
                   void* out, int start_pos);
void or_rotary_emb(const void* inp, void* out, int dt, int n_ctx, int n_embd, int d_head, float rope_pct,
                   int start_pos);
void or_silu(const void* x, void* out, int dt, int n_ctx, int n_embd, int start_pos);
void or_multiply(const void* a, const void* b, void* out, int dt, int n_ctx, int n_embd, int start_pos);
void or_add(const void* a, const void* b, void* out, int dt, int n_ctx, int n_embd, int start_pos);
void or_scale(void* x, int dt, int n_ctx, int n_embd, float s, int start_pos);
void or_bias_add_inplace(void* x, int dt, int n_ctx, int n_embd, const uint16_t* bias, int start_pos);
void or_token_embed(const void* w, int wdt, int n_vocab, int n_embd, const int32_t* tokens, int n_ctx,
                    void* out, int odt, int start_pos);
void or_qkv_attn(const void* q, const void* k, const void* v, int dt, int n_ctx, int n_head, int q_dim,
                 int kv_dim, void* qkv, int start_pos);
int or_argmax(const float* x, int n);

/* model wiring (src/tinyllama, src/zephyr, src/minicpm, src/openelm) */
typedef struct or_model or_model;
/* kind: 0 tinyllama, 1 zephyr, 2 minicpm, 3 openelm_sm, 4 openelm_md, 5 openelm_lg, 6 custom.
 * For kind 6 the layer dims come from `dims` = {n_vocab, n_embd, n_layers, n_heads, n_kv_heads,
 * n_ffn, family} with family 0 llama-like (RMSNorm), 1 zephyr-like, 2 minicpm-like. */
or_model* or_model_new(int kind, int wdt, int n_ctx, const int* dims);
void or_model_free(or_model* m);
/* parses a .gten byte image (header + records in the model's load order) */
int or_model_load(or_model* m, const void* image, long nbytes);
int or_model_n_vocab(const or_model* m);
int or_model_logits(or_model* m, const int32_t* tokens, int n_tokens, int start_pos, float* logits);
int or_model_greedy(or_model* m, const int32_t* prompt, int n_prompt, int n_gen, int32_t* out_tokens);

#ifdef __cplusplus
}
#endif
#endif
