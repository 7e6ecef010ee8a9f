// Host tokenizers of the reference (src/gten/tokenizer.{h,cpp}), behind the C ABI:
//   LLamaTokenizer (tokenizer.cpp:30-245): llama2.c's SentencePiece-BPE encoder, used by TinyLlama,
//                   MiniCPM and OpenELM (nanochat.cpp:188-229);
//   Gpt2Tokenizer  (tokenizer.cpp:249-334): regex split + greedy longest match, used by Zephyr.
// Ids and decoded bytes equal the reference's for every input. The data structures are not the
// reference's: string -> id lookups are one hash probe instead of a binary search over a sorted
// copy of the vocabulary, the BPE merge loop keeps its candidate pairs in a max-heap (O(n log n)
// instead of rescanning every adjacent pair after every merge), the GPT-2 split is a hand-written
// scanner with the regex's leftmost-first semantics, and the longest-match search starts at the
// longest vocabulary entry instead of the whole word. Decoded pieces are precomputed at load.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <queue>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "gten_b200.h"

namespace gtn {
int fail(int code, const char* fmt, ...);
}

struct gtn_tokenizer {
    int kind = 0;  // 0 = SentencePiece-BPE (LLamaTokenizer), 1 = GPT-2 (Gpt2Tokenizer)
    int vocab_size = 0, eos = 0;
    std::string prompt_prefix, prompt_suffix;
    std::vector<int32_t> tokens_prefix, tokens_suffix;
    // kind 0: pieces as C strings (up to the first NUL, as strcmp / sprintf see them), scores,
    // the decoded piece after any token but 1 and after token 1 (BOS), the " " id
    std::vector<std::string> piece;
    std::vector<float> score;
    std::vector<std::string> dec, dec_bos;
    int space_id = -1;
    // kind 1: id -> string (full records), decoded as C strings
    std::vector<std::string> word;
    size_t max_len = 0;  // longest key in `ids`
    std::unordered_map<std::string, int> ids;
};

namespace {

using gtn::fail;

bool read_file(const char* path, std::string* out) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) out->append(buf, n);
    std::fclose(f);
    return true;
}

std::string c_string(const char* p, size_t n) { return std::string(p, strnlen(p, n)); }

// The byte a piece stands for when it scans as "<0x%02hhX>" (tokenizer.cpp:88-92), else -1.
int byte_piece(const std::string& s) {
    unsigned char v = 0;
    return std::sscanf(s.c_str(), "<0x%02hhX>", &v) == 1 ? (int)v : -1;
}

std::string decoded(const std::string& s) {
    const int b = byte_piece(s);
    return b < 0 ? s : std::string(b == 0 ? 0 : 1, (char)b);  // a C string: byte 0 reads as ""
}

// String -> id with the reference's resolution of equal strings: its lookup is bsearch over the
// vocabulary sorted by strcmp (equal strings in id order), so among equal strings it returns the
// one the binary search meets first.
void build_sp_index(gtn_tokenizer* t) {
    const int n = (int)t->piece.size();
    std::vector<int> order(n);
    for (int i = 0; i < n; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return t->piece[a] < t->piece[b]; });
    t->ids.reserve((size_t)n * 2);
    for (int k = 0; k < n;) {
        int e = k + 1;
        while (e < n && t->piece[order[e]] == t->piece[order[k]]) ++e;
        const std::string& key = t->piece[order[k]];
        int id = order[k];
        if (e - k > 1) {
            int lo = 0, hi = n;
            while (lo < hi) {
                const int mid = (lo + hi) / 2;
                const int c = key.compare(t->piece[order[mid]]);
                if (c < 0) hi = mid;
                else if (c > 0) lo = mid + 1;
                else { id = order[mid]; break; }
            }
        }
        t->ids.emplace(key, id);
        t->max_len = std::max(t->max_len, key.size());
        k = e;
    }
}

int sp_lookup(const gtn_tokenizer* t, const std::string& s) {
    if (s.size() > t->max_len) return -1;
    const auto it = t->ids.find(s);
    return it == t->ids.end() ? -1 : it->second;
}

// encode_internal (tokenizer.cpp:134-241) of a NUL-free byte string.
int sp_encode(const gtn_tokenizer* t, const std::string& text, std::vector<int32_t>* out) {
    std::vector<int32_t> tok;
    tok.reserve(text.size() + 1);
    if (!text.empty()) {
        if (t->space_id < 0) return fail(GTN_ERR_ARG, "tokenizer: the vocabulary has no \" \" piece");
        tok.push_back(t->space_id);
    }
    // one token per UTF-8 group (a byte and up to 3 continuation bytes), else its bytes + 3
    const size_t n = text.size();
    for (size_t i = 0; i < n;) {
        size_t j = i + 1;
        while (j < n && ((unsigned char)text[j] & 0xC0) == 0x80 && j - i < 4) ++j;
        const int id = sp_lookup(t, text.substr(i, j - i));
        if (id >= 0) {
            tok.push_back(id);
        } else {
            for (size_t k = i; k < j; ++k) {
                const int b = (unsigned char)text[k] + 3;
                if (b >= t->vocab_size) return fail(GTN_ERR_ARG, "tokenizer: byte id %d outside the vocabulary", b);
                tok.push_back(b);
            }
        }
        i = j;
    }
    // Merges: each round the reference takes the adjacent pair whose concatenation is a piece with
    // the highest score above -1e10, the leftmost among equal scores. Nodes keep their original
    // position, so "leftmost" is the smallest position; a heap entry is stale once either node
    // changed (version) or the pair is no longer adjacent.
    const int m = (int)tok.size();
    std::vector<int> nxt(m), prv(m), ver(m, 0);
    for (int i = 0; i < m; ++i) {
        nxt[i] = i + 1 < m ? i + 1 : -1;
        prv[i] = i - 1;
    }
    struct Cand {
        float score;
        int pos, right, id, vl, vr;
    };
    auto worse = [](const Cand& a, const Cand& b) {
        return a.score < b.score || (a.score == b.score && a.pos > b.pos);
    };
    std::priority_queue<Cand, std::vector<Cand>, decltype(worse)> heap(worse);
    std::string key;
    auto push = [&](int a) {
        if (a < 0 || nxt[a] < 0) return;
        const int b = nxt[a];
        key.assign(t->piece[tok[a]]);
        key.append(t->piece[tok[b]]);
        const int id = sp_lookup(t, key);
        if (id >= 0 && t->score[id] > -1e10f) heap.push({t->score[id], a, b, id, ver[a], ver[b]});
    };
    for (int i = 0; i + 1 < m; ++i) push(i);
    int alive = m;
    while (!heap.empty()) {
        const Cand c = heap.top();
        heap.pop();
        if (ver[c.pos] != c.vl || nxt[c.pos] != c.right || ver[c.right] != c.vr) continue;
        tok[c.pos] = c.id;
        ++ver[c.pos];
        ++ver[c.right];
        const int after = nxt[c.right];
        nxt[c.pos] = after;
        if (after >= 0) prv[after] = c.pos;
        --alive;
        push(prv[c.pos]);
        push(c.pos);
    }
    out->reserve(out->size() + alive);
    for (int i = m > 0 ? 0 : -1; i >= 0; i = nxt[i]) out->push_back(tok[i]);
    return GTN_OK;
}

// The split pattern of tokenizer.h:60,
//   's|'t|'re|'ve|'m|'ll|'d| ?[[:alpha:]]+| ?[[:digit:]]+| ?[^\s[:alpha:][:digit:]]+|\s+(?!\S)|\s+
// as std::regex (ECMAScript, leftmost-first alternation, "C" locale classes) matches it from the
// start of the remaining text. Every byte belongs to one class, so a match always starts there.
enum { C_SPACE, C_ALPHA, C_DIGIT, C_OTHER };
inline int byte_class(unsigned char c) {
    if (c == ' ' || (c >= '\t' && c <= '\r')) return C_SPACE;
    if ((c | 0x20) >= 'a' && (c | 0x20) <= 'z') return C_ALPHA;
    if (c >= '0' && c <= '9') return C_DIGIT;
    return C_OTHER;
}

size_t gpt2_word_end(const std::string& s, size_t p) {
    const size_t n = s.size();
    if (s[p] == '\'') {
        static const char* const kContractions[] = {"s", "t", "re", "ve", "m", "ll", "d"};
        for (const char* c : kContractions) {
            const size_t k = std::strlen(c);
            if (p + 1 + k <= n && s.compare(p + 1, k, c) == 0) return p + 1 + k;
        }
    }
    const int c0 = byte_class((unsigned char)s[p]);
    if (c0 != C_SPACE || (s[p] == ' ' && p + 1 < n && byte_class((unsigned char)s[p + 1]) != C_SPACE)) {
        // ' ?X+' for the class X of the first byte after an optional leading space
        const size_t q = c0 == C_SPACE ? p + 1 : p;
        const int want = byte_class((unsigned char)s[q]);
        size_t e = q;
        while (e < n && byte_class((unsigned char)s[e]) == want) ++e;
        return e;
    }
    // '\s+(?!\S)': the run minus its last byte when a non-space follows; '\s+' for a single byte
    size_t e = p;
    while (e < n && byte_class((unsigned char)s[e]) == C_SPACE) ++e;
    return (e == n || e - p == 1) ? e : e - 1;
}

int gpt2_encode(const gtn_tokenizer* t, const std::string& text, std::vector<int32_t>* out) {
    static const int32_t kPrefix[] = {27, 91, 882, 91, 29, 397};               // <|user|>\n
    static const int32_t kSuffix[] = {100257, 198, 27, 91, 78191, 91, 397};   // <|endoftext|>\n<|assistant|>\n
    out->insert(out->end(), std::begin(kPrefix), std::end(kPrefix));
    std::string sub;
    for (size_t p = 0; p < text.size();) {
        const size_t e = gpt2_word_end(text, p);
        // greedy longest match over [p, e) (tokenizer.cpp:300-328); after a match that does not end
        // the word, the reference's `j == i` branch also runs and emits the next byte on its own
        size_t i = p;
        while (i < e) {
            for (size_t j = std::min(e, i + t->max_len); j > i; --j) {
                sub.assign(text, i, j - i);
                const auto it = t->ids.find(sub);
                if (it != t->ids.end()) {
                    out->push_back(it->second);
                    i = j;
                    break;
                }
            }
            if (i == e) break;
            sub.assign(text, i, 1);
            const auto it = t->ids.find(sub);
            if (it != t->ids.end()) out->push_back(it->second);
            else std::fprintf(stderr, "encode: unknown token '%s'\n", sub.c_str());
            ++i;
        }
        p = e;
    }
    out->insert(out->end(), std::begin(kSuffix), std::end(kSuffix));
    return GTN_OK;
}

}  // namespace

extern "C" {

int gtn_tokenizer_create_llama(const char* path, int vocab_size, int eos, const char* prompt_prefix,
                               const char* prompt_suffix, const int32_t* tokens_prefix, int n_prefix,
                               const int32_t* tokens_suffix, int n_suffix, gtn_tokenizer** out) {
    if (!path || !out || vocab_size <= 0 || n_prefix < 0 || n_suffix < 0 || (n_prefix && !tokens_prefix) ||
        (n_suffix && !tokens_suffix))
        return fail(GTN_ERR_ARG, "tokenizer_create_llama: bad arguments");
    std::string data;
    if (!read_file(path, &data)) return fail(GTN_ERR_ARG, "tokenizer_create_llama: cannot open %s", path);
    auto* t = new gtn_tokenizer();
    t->kind = 0;
    t->vocab_size = vocab_size;
    t->eos = eos;
    t->prompt_prefix = prompt_prefix ? prompt_prefix : "";
    t->prompt_suffix = prompt_suffix ? prompt_suffix : "";
    t->tokens_prefix.assign(tokens_prefix, tokens_prefix + n_prefix);
    t->tokens_suffix.assign(tokens_suffix, tokens_suffix + n_suffix);
    // int32 max_token_length, then per token: float32 score, int32 length, bytes (tokenizer.cpp:46-64)
    size_t off = 4;
    t->piece.reserve(vocab_size);
    t->score.reserve(vocab_size);
    for (int i = 0; i < vocab_size; ++i) {
        float s;
        int32_t len;
        if (off + 8 > data.size()) break;
        std::memcpy(&s, data.data() + off, 4);
        std::memcpy(&len, data.data() + off + 4, 4);
        off += 8;
        if (len < 0 || off + (size_t)len > data.size()) break;
        t->piece.push_back(c_string(data.data() + off, (size_t)len));
        t->score.push_back(s);
        off += (size_t)len;
    }
    if ((int)t->piece.size() != vocab_size) {
        delete t;
        return fail(GTN_ERR_FORMAT, "tokenizer_create_llama: %s holds fewer than %d records", path, vocab_size);
    }
    build_sp_index(t);
    t->space_id = sp_lookup(t, " ");
    t->dec.resize(vocab_size);
    t->dec_bos.resize(vocab_size);
    for (int i = 0; i < vocab_size; ++i) {
        const std::string& p = t->piece[i];
        t->dec[i] = decoded(p);
        t->dec_bos[i] = (!p.empty() && p[0] == ' ') ? decoded(p.substr(1)) : t->dec[i];
    }
    *out = t;
    return GTN_OK;
}

int gtn_tokenizer_create_gpt2(const char* path, int n_vocab, int eos, gtn_tokenizer** out) {
    if (!path || !out || n_vocab <= 0) return fail(GTN_ERR_ARG, "tokenizer_create_gpt2: bad arguments");
    std::string data;
    if (!read_file(path, &data)) return fail(GTN_ERR_ARG, "tokenizer_create_gpt2: cannot open %s", path);
    auto* t = new gtn_tokenizer();
    t->kind = 1;
    t->vocab_size = n_vocab;
    t->eos = eos;
    // per token: uint32 length, bytes (tokenizer.cpp:255-267). The reference reads n_vocab records
    // whatever the file holds; past its end the reads fail and leave the last string in place, so
    // the remaining ids repeat the last record (Zephyr: 100,256 records for n_vocab 100,352).
    size_t off = 0;
    t->word.reserve(n_vocab);
    for (int i = 0; i < n_vocab; ++i) {
        if (off + 4 <= data.size()) {
            uint32_t len;
            std::memcpy(&len, data.data() + off, 4);
            if (off + 4 + (size_t)len > data.size()) {
                delete t;
                return fail(GTN_ERR_FORMAT, "tokenizer_create_gpt2: %s ends inside record %d", path, i);
            }
            t->word.emplace_back(data.data() + off + 4, (size_t)len);
            off += 4 + (size_t)len;
        } else if (!t->word.empty()) {
            t->word.push_back(t->word.back());
        } else {
            delete t;
            return fail(GTN_ERR_FORMAT, "tokenizer_create_gpt2: %s holds no records", path);
        }
    }
    t->ids.reserve((size_t)n_vocab * 2);
    for (int i = 0; i < n_vocab; ++i) {
        t->ids[t->word[i]] = i;  // equal strings: the last id wins (std::map assignment)
        t->max_len = std::max(t->max_len, t->word[i].size());
    }
    t->dec.resize(n_vocab);
    for (int i = 0; i < n_vocab; ++i) t->dec[i] = c_string(t->word[i].data(), t->word[i].size());
    *out = t;
    return GTN_OK;
}

void gtn_tokenizer_free(gtn_tokenizer* t) { delete t; }

int gtn_tokenizer_vocab_size(const gtn_tokenizer* t) { return t ? t->vocab_size : -1; }

int gtn_tokenizer_eos(const gtn_tokenizer* t) { return t ? t->eos : -1; }

int gtn_tokenizer_encode(const gtn_tokenizer* t, const char* text, size_t len, int32_t* ids, int cap, int* n_ids) {
    if (!t || (len && !text) || !n_ids || cap < 0 || (cap && !ids))
        return fail(GTN_ERR_ARG, "tokenizer_encode: bad arguments");
    std::vector<int32_t> out;
    int st;
    if (t->kind == 0) {
        // encode (tokenizer.cpp:103-132): the prompt between the prefix and suffix strings, read as a
        // C string, between the prefix and suffix ids
        std::string s = t->prompt_prefix;
        s.append(text ? text : "", len);
        s.append(t->prompt_suffix);
        s.resize(strnlen(s.c_str(), s.size()));
        out.assign(t->tokens_prefix.begin(), t->tokens_prefix.end());
        st = sp_encode(t, s, &out);
        out.insert(out.end(), t->tokens_suffix.begin(), t->tokens_suffix.end());
    } else {
        st = gpt2_encode(t, std::string(text ? text : "", len), &out);
    }
    if (st != GTN_OK) return st;
    *n_ids = (int)out.size();
    if ((int)out.size() > cap) return fail(GTN_ERR_ARG, "tokenizer_encode: %d ids do not fit in %d", (int)out.size(), cap);
    std::memcpy(ids, out.data(), out.size() * sizeof(int32_t));
    return GTN_OK;
}

int gtn_tokenizer_decode(const gtn_tokenizer* t, int prev_token, int token, const char** piece, size_t* len) {
    if (!t || !piece || !len) return fail(GTN_ERR_ARG, "tokenizer_decode: bad arguments");
    static const char kEmpty[] = "";
    if (token < 0 || token >= t->vocab_size) {
        // LLamaTokenizer: "" for ids >= vocab_size (tokenizer.cpp:78-80); Gpt2Tokenizer: "" for ids
        // it has no string for (std::map operator[]); negative ids are out of range here
        *piece = kEmpty;
        *len = 0;
        return GTN_OK;
    }
    const std::string& s = (t->kind == 0 && prev_token == 1) ? t->dec_bos[token] : t->dec[token];
    *piece = s.c_str();
    *len = s.size();
    return GTN_OK;
}
}
