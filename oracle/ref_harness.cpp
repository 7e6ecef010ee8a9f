// Test infrastructure only: a C-callable harness around the UNMODIFIED reference gten
// library (iangitonga/nanochatllms.cpp, src/gten/*.cpp and the four model files).
//
// This file is compiled together with the reference's own sources (read in place from the
// reference checkout, never copied) by oracle/build_ref.sh into oracle/_ref/libgtenref.so.
// It is used by the parity tests as the ground truth, and by bench.py's reference arm as the
// reference CPU baseline. Nothing in the product links or loads it.
//
// Dtype codes follow the reference enum `gten::Dtype` (src/gten/gten_types.h:20-26):
//   0 Int32, 1 Float16, 2 Float32, 3 Qint8, 4 Qint4.
#include <cstdint>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "gten/gten.h"
#include "tinyllama/tinyllama.h"
#include "zephyr/zephyr.h"
#include "minicpm/minicpm.h"
#include "openelm/openelm.h"

using namespace gten;

static Dtype dt(int c) {
    switch (c) {
        case 0: return kInt32;
        case 1: return kFloat16;
        case 2: return kFloat32;
        case 3: return kQint8;
        default: return kQint4;
    }
}

// Non-owning tensor view (reference ctor tensor.cpp:77-89).
static Tensor view(const void* p, std::vector<int> shape, int dtype) {
    return Tensor(p, shape, dt(dtype));
}

extern "C" {

// ---- quants.cpp ------------------------------------------------------------------------
void ref_q8_quantize_row(const float* inp, void* out, int rowsize) {
    ops::q8_quantize_row(inp, reinterpret_cast<Q8Block*>(out), rowsize);
}
void ref_q8_dequantize_row(const void* inp, float* out, int rowsize) {
    ops::q8_dequantize_row(reinterpret_cast<const Q8Block*>(inp), out, rowsize);
}
void ref_q4_dequantize_row(const void* inp, float* out, int rowsize) {
    ops::q4_dequantize_row(reinterpret_cast<const Q4Block*>(inp), out, rowsize);
}
uint16_t ref_fp32_to_fp16(float x) { return fp32_to_fp16(x); }
float ref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }

// ---- ops.h ---------------------------------------------------------------------------
// out_1d != 0 selects the 1-D fp32 output used by EmbeddingLinear (modules.cpp:111-122),
// i.e. the last row only with a stride-0 output.
void ref_matmul_2d(const void* x, int xdt, int n_ctx, int n_embd, const void* w, int wdt, int n_out,
                   void* out, int odt, int start_pos, int out_1d) {
    Tensor X = view(x, {n_ctx, n_embd}, xdt);
    Tensor W = view(w, {n_out, n_embd}, wdt);
    if (out_1d) {
        Tensor O = view(out, {n_out}, odt);
        O.set_strides({0});
        ops::matmul_2d(X, W, O, start_pos);
    } else {
        Tensor O = view(out, {n_ctx, n_out}, odt);
        ops::matmul_2d(X, W, O, start_pos);
    }
}

void ref_rms_norm(const void* x, int xdt, int n_ctx, int n_embd, const void* w, void* out, int start_pos) {
    Tensor X = view(x, {n_ctx, n_embd}, xdt);
    Tensor W = view(w, {n_embd}, 1);
    Tensor O = view(out, {n_ctx, n_embd}, xdt);
    ops::rms_norm(X, W, O, start_pos);
}

void ref_rms_norm_3d(const void* x, int xdt, int n_ctx, int n_heads, int d_head, const void* w, void* out,
                     int start_pos) {
    Tensor X = view(x, {n_ctx, n_heads, d_head}, xdt);
    Tensor W = view(w, {d_head}, 1);
    Tensor O = view(out, {n_ctx, n_heads * d_head}, xdt);
    ops::rms_norm(X, W, O, start_pos);
}

void ref_layer_norm(const void* x, int xdt, int n_ctx, int n_embd, const void* w, const void* b, void* out,
                    int start_pos) {
    Tensor X = view(x, {n_ctx, n_embd}, xdt);
    Tensor W = view(w, {n_embd}, 1);
    Tensor B = view(b, {n_embd}, 1);
    Tensor O = view(out, {n_ctx, n_embd}, xdt);
    ops::layer_norm(X, W, B, O, start_pos);
}

void ref_rotary_emb(void* inp, void* out, int dtype, int n_ctx, int n_embd, int d_head, float rope_pct,
                    int start_pos) {
    Tensor I = view(inp, {n_ctx, n_embd}, dtype);
    Tensor O = view(out, {n_ctx, n_embd}, dtype);
    ops::rotary_emb(I, O, d_head, rope_pct, start_pos);
}

void ref_silu(const void* x, void* out, int dtype, int n_ctx, int n_embd, int start_pos) {
    Tensor X = view(x, {n_ctx, n_embd}, dtype);
    Tensor O = view(out, {n_ctx, n_embd}, dtype);
    ops::silu(X, O, start_pos);
}

void ref_multiply(const void* a, const void* b, void* out, int dtype, int n_ctx, int n_embd, int start_pos) {
    Tensor A = view(a, {n_ctx, n_embd}, dtype);
    Tensor B = view(b, {n_ctx, n_embd}, dtype);
    Tensor O = view(out, {n_ctx, n_embd}, dtype);
    ops::multiply(A, B, O, start_pos);
}

void ref_add(const void* a, const void* b, void* out, int dtype, int n_ctx, int n_embd, int start_pos) {
    Tensor A = view(a, {n_ctx, n_embd}, dtype);
    Tensor B = view(b, {n_ctx, n_embd}, dtype);
    Tensor O = view(out, {n_ctx, n_embd}, dtype);
    ops::add(A, B, O, start_pos);
}

void ref_scale(void* x, int dtype, int n_ctx, int n_embd, float s, int start_pos) {
    Tensor X = view(x, {n_ctx, n_embd}, dtype);
    ops::scale(X, s, start_pos);
}

void ref_bias_add_inplace(void* x, int dtype, int n_ctx, int n_embd, const void* bias, int start_pos) {
    Tensor X = view(x, {n_ctx, n_embd}, dtype);
    Tensor B = view(bias, {n_embd}, 1);
    ops::bias_add_inplace(X, B, start_pos);
}

void ref_token_embed(const void* w, int wdt, int n_vocab, int n_embd, const int32_t* tokens, int n_ctx,
                     void* out, int odt, int start_pos) {
    Tensor W = view(w, {n_vocab, n_embd}, wdt);
    Tensor T = view(tokens, {n_ctx}, 0);
    Tensor O = view(out, {n_ctx, n_embd}, odt);
    ops::token_embed(W, T, O, start_pos);
}

// q: [n_ctx, n_head*d_head], k/v: [n_ctx, kv_dim]; qkv out: [n_ctx, n_head*d_head].
// The probability scratch is allocated here with the module's capacity
// (modules.cpp:273: Tensor({n_heads, max_ctx, max_ctx}, adtype)).
void ref_qkv_attn(const void* q, const void* k, const void* v, int dtype, int n_ctx, int n_head, int q_dim,
                  int kv_dim, int max_ctx, void* qkv, int start_pos) {
    Tensor Q = view(q, {n_ctx, q_dim}, dtype);
    Tensor K = view(k, {n_ctx, kv_dim}, dtype);
    Tensor V = view(v, {n_ctx, kv_dim}, dtype);
    Tensor QK({n_head, max_ctx, max_ctx}, dt(dtype));
    QK.resize({n_head, n_ctx, n_ctx});
    Tensor O = view(qkv, {n_ctx, q_dim}, dtype);
    ops::qkv_attn(Q, K, V, QK, O, max_ctx, start_pos);
}

// ---- models (abc.h:12-28) ------------------------------------------------------------
// kind: 0 tinyllama, 1 zephyr, 2 minicpm, 3 openelm_sm, 4 openelm_md, 5 openelm_lg
// wdtype: 1 fp16 (mFloat16), 3 q8 (mQint8), 4 q4 (mQint4)
void* ref_model_new(int kind, int wdtype, int n_ctx) {
    ModuleDtype md = wdtype == 1 ? mFloat16 : (wdtype == 3 ? mQint8 : mQint4);
    switch (kind) {
        case 0: return new TinyLLama(n_ctx, md);
        case 1: return new Zephyr(n_ctx, md);
        case 2: return new MiniCPM(n_ctx, md);
        case 3: return new OpenELM(n_ctx, md, openelm_sm_cfg);
        case 4: return new OpenELM(n_ctx, md, openelm_md_cfg);
        case 5: return new OpenELM(n_ctx, md, openelm_lg_cfg);
        default: return nullptr;
    }
}

void ref_model_free(void* m) { delete reinterpret_cast<Model*>(m); }

int ref_model_load(void* m, const char* path) {
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) return -1;
    reinterpret_cast<Model*>(m)->load_from_ckpt(f);
    return 0;
}

// One Model::logits call (the body of sampler.cpp:19-26). Writes n_vocab fp32 logits.
int ref_model_logits(void* m, const int32_t* tokens, int n_tokens, int start_pos, float* logits_out) {
    Tensor T(tokens, {n_tokens}, kInt32);
    Tensor L = reinterpret_cast<Model*>(m)->logits(T, start_pos);
    std::memcpy(logits_out, L.data_ptr<float>(), sizeof(float) * L.numel());
    return L.numel();
}

// Greedy decode as sampler.cpp:11-53 without the EOS break and without detokenization:
// prefill at start_pos 0, then one token per call at start_pos n-1, first-max argmax.
// Optionally records each step's top-2 margin (logit[best] - logit[second]).
int ref_model_greedy(void* m, const int32_t* prompt, int n_prompt, int n_gen, int32_t* out_tokens,
                     float* out_margins) {
    Model* model = reinterpret_cast<Model*>(m);
    std::vector<int32_t> tokens(prompt, prompt + n_prompt);
    tokens.reserve(n_prompt + n_gen);
    for (int i = 0; i < n_gen; i++) {
        Tensor input{tokens.data(), {(int)tokens.size()}, kInt32};
        const int start_pos = (i == 0) ? 0 : input.numel() - 1;
        Tensor logits = model->logits(input, start_pos);
        const int n = logits.numel();
        const float* d = logits.data_ptr<float>();
        float best = -std::numeric_limits<float>::infinity();
        int idx = 0;
        for (int j = 0; j < n; ++j) {
            if (d[j] > best) { best = d[j]; idx = j; }
        }
        if (out_margins) {
            float second = -std::numeric_limits<float>::infinity();
            for (int j = 0; j < n; ++j) {
                if (j != idx && d[j] > second) second = d[j];
            }
            out_margins[i] = best - second;
        }
        out_tokens[i] = idx;
        tokens.push_back(idx);
    }
    return 0;
}

}  // extern "C"
