// Test infrastructure only. C entry points over the reference's own, unmodified tokenizers
// (src/gten/tokenizer.cpp, compiled from the reference checkout by build_ref.sh into
// oracle/_ref/libgtenref.so), so that tests and tests/golden/make_tokenizer_golden.py can drive
// LLamaTokenizer (tokenizer.h:27-45) and Gpt2Tokenizer (tokenizer.h:49-65) through ctypes.
// Nothing here is linked into the product library.
#include <cstring>
#include <string>
#include <vector>

#include "gten/tokenizer.h"

extern "C" {

void* tokref_llama(const char* path, int vocab_size, int eos, const char* prompt_prefix, const char* prompt_suffix,
                   const int* tokens_prefix, int n_prefix, const int* tokens_suffix, int n_suffix) {
    std::vector<int> tp(tokens_prefix, tokens_prefix + n_prefix), ts(tokens_suffix, tokens_suffix + n_suffix);
    return static_cast<gten::Tokenizer*>(
        new gten::LLamaTokenizer(path, vocab_size, eos, prompt_prefix, prompt_suffix, tp, ts));
}

void* tokref_gpt2(const char* path, int n_vocab, int eos) {
    return static_cast<gten::Tokenizer*>(new gten::Gpt2Tokenizer(path, n_vocab, eos));
}

// encode(prompt) of the given text bytes; returns the number of ids (copies at most cap of them).
int tokref_encode(void* t, const char* text, int len, int* out, int cap) {
    std::string s(text, (size_t)len);
    const std::vector<int> ids = static_cast<gten::Tokenizer*>(t)->encode(s);
    for (int i = 0; i < (int)ids.size() && i < cap; ++i) out[i] = ids[i];
    return (int)ids.size();
}

// decode(prev_token, token): the returned C string, copied (strlen bytes) into out; returns its length.
int tokref_decode(void* t, int prev, int token, char* out, int cap) {
    const char* p = static_cast<gten::Tokenizer*>(t)->decode(prev, token);
    const int n = (int)std::strlen(p);
    std::memcpy(out, p, (size_t)(n < cap ? n : cap));
    return n;
}

// The reference's Tokenizer base has no virtual destructor: delete through the concrete type
// (kind 0 = LLamaTokenizer, 1 = Gpt2Tokenizer).
void tokref_free(void* t, int kind) {
    if (kind == 0) delete static_cast<gten::LLamaTokenizer*>(static_cast<gten::Tokenizer*>(t));
    else delete static_cast<gten::Gpt2Tokenizer*>(static_cast<gten::Tokenizer*>(t));
}
}
