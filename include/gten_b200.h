/* gten_b200 — C ABI of the B200 (sm_100a) implementation of the gten compute path of
 * iangitonga/nanochatllms.cpp.
 *
 * Drop-in boundary. Each entry point replaces one function of the reference's operator API
 * (namespace gten::ops, src/gten/ops.h) or of its model / sampler interface, keeps its argument
 * meaning and computes rows [start_pos, dimsize(0)) into a caller-owned, pre-sized output, with
 * the reference's numerics (results are bit-identical to the reference CPU build; see each
 * entry). Differences in error behaviour: where the reference's GTEN_ASSERT prints and calls
 * exit(1) (src/gten/log.h:6-23), these functions return a non-zero gtn_status and leave the
 * output untouched.
 *
 * Memory: tensor data pointers are CUDA device pointers unless an entry says "host".
 * Streams: `stream` is a cudaStream_t (NULL = the legacy default stream); calls are
 * asynchronous with respect to the host unless stated otherwise.
 * Threading: calls on distinct streams may run concurrently; a model handle is single-caller.
 */
#ifndef GTEN_B200_H
#define GTEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (0 = success). */
typedef enum {
    GTN_OK = 0,
    GTN_ERR_ARG = 1,     /* shape / dtype / range check failed (a GTEN_ASSERT in the reference) */
    GTN_ERR_CUDA = 2,    /* a CUDA runtime call or kernel launch failed */
    GTN_ERR_OOM = 3,     /* device or host allocation failed */
    GTN_ERR_FORMAT = 4,  /* malformed .gten checkpoint (bad magic, record size, truncation) */
    GTN_ERR_DEVICE = 5   /* a kernel reported a device-side error (e.g. a bounded wait expired) */
} gtn_status;

/* Element types; values equal the reference enum gten::Dtype (src/gten/gten_types.h:20-26). */
typedef enum { GTN_I32 = 0, GTN_F16 = 1, GTN_F32 = 2, GTN_Q8 = 3, GTN_Q4 = 4 } gtn_dtype;

/* Plain descriptor of a gten::Tensor (src/gten/tensor.h:17-137): data pointer, dtype, 1-3 dims,
 * element strides. Quantized tensors use the reference's block layout: rows of 32-element
 * blocks, Q8 block = fp16 delta + 32 int8 (34 bytes), Q4 block = fp16 delta + 16 bytes where
 * byte j holds element j (high nibble) and element j+16 (low nibble), both +7 biased
 * (src/gten/quants.h:11-30). Rows must be contiguous (stride(ndim-1) == 1). */
typedef struct gtn_tensor {
    void* data;
    int32_t dtype;
    int32_t ndim;
    int32_t shape[3];
    int32_t strides[3];
} gtn_tensor;

/* Human-readable text of the last error on the calling thread ("" if none). */
const char* gtn_last_error(void);

/* Number of CUDA kernels this library has launched in the process (a diagnostic counter). */
unsigned long long gtn_kernel_launches(void);

/* ---- gten::ops (src/gten/ops.h) ----------------------------------------------------------- */

/* ops.h:16 matmul_2d(x, w, out, start_pos): out[r,:] = x[r,:] . w^T for r in [start_pos, n_ctx),
 * dot products in the reference order (ops.cpp:292-523), rows written in out's dtype. A 1-D out
 * (EmbeddingLinear's fp32 logits, modules.cpp:111-122) requires n_ctx - start_pos == 1.
 * For a Q8 or fp16 `out` the fp32 dot products are staged in stream-ordered device scratch
 * (cudaMallocAsync / cudaFreeAsync on `stream`). */
int gtn_matmul_2d(const gtn_tensor* x, const gtn_tensor* w, gtn_tensor* out, int start_pos, void* stream);

/* No counterpart in the reference. gtn_matmul_2d for callers that may not allocate device memory
 * (a host that owns a fixed memory budget, code running inside an allocator or memory-pool
 * callback, paths that cannot risk an allocation's implicit synchronization): same arguments and
 * results, but a Q8 / fp16 `out` is staged in a fixed 8 MiB array inside the library instead of
 * cudaMallocAsync scratch, so (n_ctx - start_pos) * n_out may not exceed 2,097,152 (GTN_ERR_ARG
 * otherwise; fp32 outputs need no staging and have no limit). The array's device address is
 * looked up on the first call made on each device — make that call before any stream capture.
 * All calls share the array: calls that overlap on the GPU race on it. */
int gtn_matmul_2d_noalloc(const gtn_tensor* x, const gtn_tensor* w, gtn_tensor* out, int start_pos, void* stream);

/* ops.h:22 qkv_attn(q, k, v, qk, qkv, max_ctx, start_pos): causal attention with GQA, the
 * probability rows stored in the activation dtype as the reference does (ops.cpp:1017-1220).
 * `qk` is accepted for signature parity and may be NULL: the probabilities stay on chip. */
int gtn_qkv_attn(const gtn_tensor* q, const gtn_tensor* k, const gtn_tensor* v, gtn_tensor* qk, gtn_tensor* qkv,
                 int max_ctx, int start_pos, void* stream);

/* ops.h:24 rms_norm(inp, weight, out, start_pos): 2-D, or 3-D [n_ctx, heads, d_head] with a
 * d_head weight (ops.cpp:830-915). Weight fp16. */
int gtn_rms_norm(const gtn_tensor* inp, const gtn_tensor* weight, gtn_tensor* out, int start_pos, void* stream);

/* ops.h:14 layer_norm(inp, weight, bias, out, start_pos) (ops.cpp:669-730). Weight, bias fp16. */
int gtn_layer_norm(const gtn_tensor* inp, const gtn_tensor* weight, const gtn_tensor* bias, gtn_tensor* out,
                   int start_pos, void* stream);

/* ops.h:26 rotary_emb(inp, out, d_head, rope_pct, start_pos) (ops.cpp:775-827). inp may equal out. */
int gtn_rotary_emb(const gtn_tensor* inp, gtn_tensor* out, int d_head, float rope_pct, int start_pos, void* stream);

/* ops.h:30,32 silu / silu_inplace (ops.cpp:733-772). */
int gtn_silu(const gtn_tensor* inp, gtn_tensor* out, int start_pos, void* stream);
int gtn_silu_inplace(gtn_tensor* inp, int start_pos, void* stream);

/* ops.h:18,20 multiply / multiply_inplace (ops.cpp:918-970). */
int gtn_multiply(const gtn_tensor* inp0, const gtn_tensor* inp1, gtn_tensor* out, int start_pos, void* stream);
int gtn_multiply_inplace(gtn_tensor* inp0, const gtn_tensor* inp1, int start_pos, void* stream);

/* ops.h:10 add (ops.cpp:973-1014). */
int gtn_add(const gtn_tensor* inp0, const gtn_tensor* inp1, gtn_tensor* out, int start_pos, void* stream);

/* ops.h:28 scale(inp, scaler, start_pos), in place (ops.cpp:125-164). */
int gtn_scale(gtn_tensor* inp, float scaler, int start_pos, void* stream);

/* ops.h:12 bias_add_inplace(inp, bias, start_pos) (ops.cpp:639-666). Bias fp16. */
int gtn_bias_add_inplace(gtn_tensor* inp, const gtn_tensor* bias, int start_pos, void* stream);

/* ops.h:40 token_embed(weight, tokens, out, start_pos) (ops.cpp:526-576). Tokens int32 on device;
 * Q4 rows are requantized to Q8 as copy_row does. */
int gtn_token_embed(const gtn_tensor* weight, const gtn_tensor* tokens, gtn_tensor* out, int start_pos,
                    void* stream);

/* ---- quantization (src/gten/quants.cpp, src/<model>/<model>_to_gten.py) ------------------- */

/* Weight packer, bit-exact with the reference converters' q8_quantize / q4_quantize
 * (src/tinyllama/tinyllama_to_gten.py:24-91; identical copies in the other converters).
 * w: device fp32 [rows, cols], cols % 32 == 0, 16-byte aligned; out: rows*cols/32 blocks. */
int gtn_pack_q8(const float* w, int64_t rows, int64_t cols, void* out, void* stream);
int gtn_pack_q4(const float* w, int64_t rows, int64_t cols, void* out, void* stream);

/* Activation quantizer q8_quantize_row (quants.cpp:140-158) applied to `rows` rows of `cols`
 * fp32 values (partial last block allowed). out: rows * ceil(cols/32) Q8 blocks. */
int gtn_quantize_q8_rows(const float* x, int64_t rows, int64_t cols, void* out, void* stream);

/* ---- sampler (src/gten/sampler.cpp) ------------------------------------------------------ */

/* Greedy pick of sampler.cpp:30-41: index of the first maximum of n fp32 values. out_index:
 * device int32. */
int gtn_argmax(const float* logits, int n, int32_t* out_index, void* stream);

/* Seeded random number state for gtn_sample_topk: the Mersenne Twister MT19937 state of
 * std::mt19937(seed), kept on the current device. Replaces sampler.cpp:70-71, where the generator is
 * seeded from std::random_device (not reproducible). */
typedef struct gtn_rng gtn_rng;
int gtn_rng_create(uint32_t seed, gtn_rng** out);
int gtn_rng_free(gtn_rng* rng);

/* One top-k / temperature draw of topk_sample (sampler.cpp:63-128, the body of its loop after
 * model->logits): logits/temp in double, the top_k largest (partial_sort), exp and their sum in
 * double, the probabilities over the vocabulary, std::discrete_distribution (sum, normalize,
 * partial sums, lower_bound of one generate_canonical<double> draw of two 32-bit outputs).
 * top_k is clamped to 1000 and temp to 2.0 as the reference does; 1 <= top_k <= n, temp > 0.
 * logits: device fp32 [n]; out_index: device int32. Advances rng by two outputs (none when n = 1);
 * rng must live on the current device. Among logits
 * equal to the k-th largest, the lowest indices are taken (the reference's heap selection may take
 * others). */
int gtn_sample_topk(const float* logits, int n, float temp, int top_k, gtn_rng* rng, int32_t* out_index,
                    void* stream);

/* ---- models (src/gten/abc.h:12-28 Model; src/tinyllama, zephyr, minicpm, openelm) -------- */

typedef struct gtn_model gtn_model;

/* Model kinds (the reference's four families and OpenELM sizes, nanochat.cpp:186-229). */
enum {
    GTN_MODEL_TINYLLAMA = 0,
    GTN_MODEL_ZEPHYR = 1,
    GTN_MODEL_MINICPM = 2,
    GTN_MODEL_OPENELM_SM = 3,
    GTN_MODEL_OPENELM_MD = 4,
    GTN_MODEL_OPENELM_LG = 5,
    GTN_MODEL_CUSTOM = 6
};

/* Creates a model of `kind` with weight dtype `wdtype` (GTN_F16, GTN_Q8 or GTN_Q4; activations
 * are fp16 for GTN_F16 and Q8 otherwise, gten_types.h:40-42) on the current CUDA device, with
 * KV capacity for `max_ctx` tokens per sequence and `max_batch` independent sequences.
 * The reference's constructor is Model(n_ctx, dtype) (tinyllama.h:52 and siblings).
 * For GTN_MODEL_CUSTOM, dims = {n_vocab, n_embd, n_layers, n_heads, n_kv_heads, n_ffn, family}
 * with family 0 = TinyLlama-like, 1 = Zephyr-like, 2 = MiniCPM-like, 3 = OpenELM-like (QK-norm; the
 * same head and FFN widths in every layer); otherwise dims may be NULL. */
int gtn_model_create(int kind, int wdtype, int max_ctx, int max_batch, const int32_t* dims, gtn_model** out);
void gtn_model_free(gtn_model* m);
int gtn_model_n_vocab(const gtn_model* m);

/* load_from_ckpt (e.g. tinyllama.cpp:195-251; reader utils.cpp:29-61) from a complete .gten
 * image in host memory (magic, then records in the model's load order). The records go to HBM
 * through pinned staging buffers with asynchronous copies (host threads fill one buffer while
 * the copy engine drains the others). Synchronous. */
int gtn_model_load(gtn_model* m, const void* host_image, size_t nbytes);

/* load_from_ckpt from a .gten file path, as the reference opens it (utils.cpp:29-61): the file
 * is memory-mapped and loaded as gtn_model_load does. */
int gtn_model_load_file(gtn_model* m, const char* path);

/* Model::logits(tokens, start_pos) for sequence 0 (abc.h:25): tokens (host int32, n_tokens total,
 * rows [start_pos, n_tokens) are new) -> host fp32 logits of the last row. Synchronous. */
int gtn_model_logits(gtn_model* m, const int32_t* tokens, int n_tokens, int start_pos, float* logits);

/* greedy_sample (sampler.cpp:11-53) without tokenization and without the EOS stop: prefill the
 * prompt (host int32), then n_gen greedy steps; out_tokens (host) receives the n_gen ids.
 * Synchronous. */
int gtn_model_generate(gtn_model* m, const int32_t* prompt, int n_prompt, int n_gen, int32_t* out_tokens);

/* topk_sample (sampler.cpp:63-143) without tokenization and without the EOS stop: prefill the
 * prompt, then n_gen steps, each drawing its id as gtn_sample_topk does (same clamps and argument
 * rules) with the caller's seeded generator, which advances by two outputs per step. The draw runs
 * on the device inside the decode step. Synchronous; rng must live on the current device. */
int gtn_model_generate_topk(gtn_model* m, const int32_t* prompt, int n_prompt, int n_gen, float temp, int top_k,
                            gtn_rng* rng, int32_t* out_tokens);

/* greedy_sample for `batch` independent sequences (the reference has no batching: each sequence
 * gives exactly the ids it would give alone). prompts: host [batch][n_prompt]; out_tokens: host
 * [batch][n_gen]. batch <= max_batch; any model kind and weight dtype. Synchronous. */
int gtn_model_generate_batch(gtn_model* m, const int32_t* prompts, int batch, int n_prompt, int n_gen,
                             int32_t* out_tokens);

/* The same greedy loop with device-resident int32 prompt / output arrays, enqueued on the model's
 * stream without host synchronization (the ids never leave HBM). Token ids are range-checked on
 * the device; gtn_model_check reports violations. */
int gtn_model_generate_device(gtn_model* m, const int32_t* prompt, int n_prompt, int n_gen, int32_t* out_tokens);

/* Continuous batching over the model's max_batch slots (greedy; any model kind and weight dtype).
 * The reference decodes one sequence per greedy_sample call
 * (sampler.cpp:11-53); here sequences of any prompt length join and leave a running batch:
 *   gtn_slot_start   prefills a prompt (host int32) into a free slot, returns the slot and the
 *                    first greedy id; fails when every slot is busy;
 *   gtn_slots_step   one decode step of every busy slot (one captured CUDA graph over all slots;
 *                    idle slots are skipped on the device); ids (host, max_batch entries) receive
 *                    each busy slot's next id, -1 for idle slots; a slot whose last token sits at
 *                    position max_ctx - 1 must be finished first;
 *   gtn_slot_finish  frees a slot.
 * Every sequence gets exactly the ids it gets alone. While slots are busy, gtn_model_logits and
 * gtn_model_generate* refuse to run (they reuse the slots' rows). Synchronous. */
int gtn_slot_start(gtn_model* m, const int32_t* prompt, int n_prompt, int* slot, int32_t* first_id);
int gtn_slots_step(gtn_model* m, int32_t* ids);
int gtn_slot_finish(gtn_model* m, int slot);

/* The cudaStream_t the model enqueues its work on. */
void* gtn_model_stream(gtn_model* m);

/* Waits for the model's stream and returns GTN_ERR_DEVICE if a kernel flagged an error. */
int gtn_model_check(gtn_model* m);

/* ---- tokenizers (src/gten/abc.h:31-54 Tokenizer; src/gten/tokenizer.{h,cpp}) ---------------- */
/* Host code only (no CUDA calls). Ids and decoded bytes equal the reference's for every input;
 * a handle may be used from several threads at once (encode and decode do not modify it). */

typedef struct gtn_tokenizer gtn_tokenizer;

/* LLamaTokenizer(path, vocab_size, eos, prompt_prefix, prompt_suffix, tokens_prefix, tokens_suffix)
 * (tokenizer.h:27-31, tokenizer.cpp:30-65): the SentencePiece-BPE vocabulary file (int32
 * max_token_length, then vocab_size records of float32 score, int32 length, bytes). The prompt
 * strings are NUL-terminated (NULL = ""). GTN_ERR_FORMAT when the file holds fewer than vocab_size
 * records (the reference exits). */
int gtn_tokenizer_create_llama(const char* path, int vocab_size, int eos, const char* prompt_prefix,
                               const char* prompt_suffix, const int32_t* tokens_prefix, int n_prefix,
                               const int32_t* tokens_suffix, int n_suffix, gtn_tokenizer** out);

/* Gpt2Tokenizer(vocab_path, n_vocab, eos) (tokenizer.h:51, tokenizer.cpp:249-268): records of
 * uint32 length, bytes. As in the reference, ids past the file's last record repeat that record. */
int gtn_tokenizer_create_gpt2(const char* path, int n_vocab, int eos, gtn_tokenizer** out);

void gtn_tokenizer_free(gtn_tokenizer* t);
int gtn_tokenizer_vocab_size(const gtn_tokenizer* t);
int gtn_tokenizer_eos(const gtn_tokenizer* t);

/* Tokenizer::encode(prompt) (abc.h:53; tokenizer.cpp:103-241 and 278-331): len bytes of host text
 * -> ids (host int32). *n_ids receives the number of ids; when it exceeds cap nothing is copied and
 * GTN_ERR_ARG is returned (call again with a larger buffer). The caller's text is not modified (the
 * reference's LLamaTokenizer::encode rewrites its argument to prefix + prompt + suffix). */
int gtn_tokenizer_encode(const gtn_tokenizer* t, const char* text, size_t len, int32_t* ids, int cap, int* n_ids);

/* Tokenizer::decode(prev_token, token) (abc.h:52; tokenizer.cpp:77-93 and 272-275): *piece points
 * to *len bytes owned by the tokenizer (valid until gtn_tokenizer_free), the bytes of the C string
 * the reference returns. Ids outside [0, vocab_size) decode to "" (the reference reads out of bounds
 * for negative LLamaTokenizer ids). */
int gtn_tokenizer_decode(const gtn_tokenizer* t, int prev_token, int token, const char** piece, size_t* len);

#ifdef __cplusplus
}
#endif
#endif /* GTEN_B200_H */
