// tokenizer.cpp -- WordPiece and SentencePiece Unigram tokenizers (see tokenizer.h).
#include "tokenizer.h"

#include <algorithm>
#include <cctype>
#include <cstdio>

#include "ceb_internal.h"
#include "gguf.h"

int ceb_tokenizer_family(bool type_key_present, int declared_type, const std::string& model_str, int64_t vocab_n) {
    if (type_key_present) return declared_type;
    if (model_str == "gpt2" || model_str == "bpe") return 1;
    if (model_str == "t5" || model_str == "unigram" || model_str == "spm" || model_str == "llama") return 2;
    if (model_str == "bert" || model_str == "wordpiece") return 0;
    return vocab_n > 100000 ? 2 : 0;
}

namespace {
int kv_int(const ceb_gguf& g, const char* key, int dflt) {
    int v;
    return g.get_u32(key, &v) ? v : dflt;
}
bool kv_bool(const ceb_gguf& g, const char* key, bool dflt) {
    const ceb_gguf_value* v = g.find(key);
    if (!v || v->type != 7) return dflt;  // GGUF_TYPE_BOOL
    return v->u != 0;
}
bool is_ascii_punct(unsigned char c) {
    return (c >= 33 && c <= 47) || (c >= 58 && c <= 64) || (c >= 91 && c <= 96) || (c >= 123 && c <= 126);
}

#include "spm_norm_table.inc"

// Next codepoint of a UTF-8 string at i (advanced); a byte that does not start a
// valid sequence is returned as itself (>= 0x80 values then pass through unchanged).
uint32_t utf8_next(const std::string& s, size_t& i, size_t* len) {
    const unsigned char c = (unsigned char)s[i];
    int n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
    if (n == 0 || i + n > s.size()) n = 1;
    uint32_t cp = n == 1 ? c : n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
    for (int k = 1; k < n; ++k) {
        const unsigned char d = (unsigned char)s[i + k];
        if ((d & 0xC0) != 0x80) {  // broken sequence: the lead byte alone
            n = 1;
            cp = 0xFFFFFFFFu;
            break;
        }
        cp = (cp << 6) | (d & 0x3F);
    }
    *len = (size_t)n;
    i += n;
    return cp;
}
}  // namespace

// SentencePiece nmt_nfkc normalisation one codepoint at a time (the table in
// spm_norm_table.inc), applied before the space -> U+2581 marking as the
// reference does for the embedding path (src/tokenizer_spm.cpp:57-70,
// src/crispembed.cpp:624).
std::string ceb_spm_normalize(const std::string& text) {
    std::string out;
    out.reserve(text.size());
    size_t i = 0;
    while (i < text.size()) {
        const unsigned char c = (unsigned char)text[i];
        if (c >= 0x20 && c < 0x7F) {  // printable ASCII is unchanged
            out += (char)c;
            ++i;
            continue;
        }
        const size_t at = i;
        size_t len = 0;
        const uint32_t cp = utf8_next(text, i, &len);
        int lo = 0, hi = kSpmNormN - 1, hit = -1;
        while (lo <= hi && cp != 0xFFFFFFFFu) {
            const int mid = (lo + hi) >> 1;
            if (kSpmNormCp[mid] == cp) {
                hit = mid;
                break;
            }
            if (kSpmNormCp[mid] < cp) lo = mid + 1;
            else hi = mid - 1;
        }
        if (hit < 0)
            out.append(text, at, len);
        else
            out.append(reinterpret_cast<const char*>(kSpmNormUtf8) + kSpmNormOff[hit],
                       kSpmNormOff[hit + 1] - kSpmNormOff[hit]);
    }
    return out;
}

int ceb_tokenizer::load(const ceb_gguf& g, int max_tok) {
    max_tokens = max_tok > 2 ? max_tok : 512;
    const ceb_gguf_value* toks = g.find("tokenizer.ggml.tokens");
    if (!toks || toks->arr_str.empty()) return ceb_set_error(1, "GGUF has no tokenizer.ggml.tokens");
    pieces = toks->arr_str;
    index.clear();
    index.reserve(pieces.size());
    for (size_t i = 0; i < pieces.size(); ++i) index[pieces[i]] = (int)i;  // a repeated piece maps to its last id
    int declared = 0;
    const bool has_type = g.get_u32("tokenizer.ggml.type", &declared);
    family = ceb_tokenizer_family(has_type, declared, g.get_str("tokenizer.ggml.model"), (int64_t)pieces.size());
    if (family == 2) {
        bos_id = kv_int(g, "tokenizer.ggml.bos_token_id", 0);
        eos_id = kv_int(g, "tokenizer.ggml.eos_token_id", 2);
        unk_id = kv_int(g, "tokenizer.ggml.unknown_token_id", 3);
        pad_id = kv_int(g, "tokenizer.ggml.padding_token_id", 1);
        add_bos = kv_bool(g, "tokenizer.ggml.add_bos_token", true);
        add_eos = kv_bool(g, "tokenizer.ggml.add_eos_token", true);
        scores.assign(pieces.size(), 0.0f);
        if (const ceb_gguf_value* sc = g.find("tokenizer.ggml.scores"))
            for (size_t i = 0; i < sc->arr_num.size() && i < scores.size(); ++i) scores[i] = (float)sc->arr_num[i];
        byte_piece.assign(256, -1);
        for (int b = 0; b < 256; ++b) {
            char hex[8];
            snprintf(hex, sizeof(hex), "<0x%02X>", b);
            auto it = index.find(hex);
            if (it != index.end()) byte_piece[b] = it->second;
        }
        build_trie();
    } else if (family == 0) {
        cls_id = kv_int(g, "tokenizer.ggml.cls_token_id", 101);
        sep_id = kv_int(g, "tokenizer.ggml.sep_token_id", 102);
        unk_id = kv_int(g, "tokenizer.ggml.unknown_token_id", 100);
        pad_id = kv_int(g, "tokenizer.ggml.padding_token_id", 0);
        lower = true;  // a single upper-case letter in the vocabulary marks a cased model
        for (const auto& t : pieces)
            if (t.size() == 1 && t[0] >= 'A' && t[0] <= 'Z') {
                lower = false;
                break;
            }
    }
    // every id the encoder can emit must name a piece: the ids index the token table
    const int n = (int)pieces.size();
    auto bad = [n](int id) { return id < 0 || id >= n; };
    const char* which = nullptr;
    int id = 0;
    if (family == 2) {
        if (add_bos && bad(bos_id)) which = "bos", id = bos_id;
        else if (add_eos && bad(eos_id)) which = "eos", id = eos_id;
        else if (bad(unk_id)) which = "unknown", id = unk_id;
    } else if (family == 0) {
        if (bad(cls_id)) which = "cls", id = cls_id;
        else if (bad(sep_id)) which = "sep", id = sep_id;
        else if (bad(unk_id)) which = "unknown", id = unk_id;
    }
    if (which) return ceb_set_error(1, "tokenizer: %s token id %d outside the vocabulary of %d pieces", which, id, n);
    return 0;
}

void ceb_tokenizer::build_trie() {
    trie_.assign(1, Node());
    for (size_t id = 0; id < pieces.size(); ++id) {
        const std::string& p = pieces[id];
        if (p.empty()) continue;
        int node = 0;
        for (unsigned char c : p) {
            int ch = trie_[node].child;
            while (ch >= 0 && trie_[ch].byte != c) ch = trie_[ch].sibling;
            if (ch < 0) {
                Node n;
                n.byte = c;
                n.sibling = trie_[node].child;
                trie_.push_back(n);
                ch = (int)trie_.size() - 1;
                trie_[node].child = ch;
            }
            node = ch;
        }
        trie_[node].id = (int)id;  // a repeated piece maps to its last id, as in the string index
    }
}

const std::string& ceb_tokenizer::token_str(int id) const {
    static const std::string empty;
    return (id >= 0 && id < (int)pieces.size()) ? pieces[id] : empty;
}

void ceb_tokenizer::wordpiece(const std::string& text, std::vector<int32_t>* ids) const {
    std::vector<std::string> words;
    std::string cur;
    for (unsigned char c : text) {
        if (std::isspace(c)) {
            if (!cur.empty()) words.push_back(cur), cur.clear();
        } else if (c < 128 && is_ascii_punct(c)) {
            if (!cur.empty()) words.push_back(cur), cur.clear();
            words.push_back(std::string(1, (char)c));
        } else {
            cur.push_back(lower && c < 128 ? (char)std::tolower(c) : (char)c);
        }
    }
    if (!cur.empty()) words.push_back(cur);
    ids->push_back(cls_id);
    const size_t limit = (size_t)max_tokens - 1;
    for (const auto& w : words) {
        if (ids->size() >= limit) break;
        if (w.size() > 100) {
            ids->push_back(unk_id);
            continue;
        }
        std::vector<int32_t> sub_ids;
        size_t start = 0;
        bool bad = false;
        while (start < w.size()) {
            size_t end = w.size();
            int found = -1;
            while (start < end) {
                std::string sub = w.substr(start, end - start);
                if (start > 0) sub = "##" + sub;
                auto it = index.find(sub);
                if (it != index.end()) {
                    found = it->second;
                    break;
                }
                --end;
            }
            if (found < 0) {
                bad = true;
                break;
            }
            sub_ids.push_back(found);
            start = end;
        }
        if (bad) {
            ids->push_back(unk_id);
        } else {
            for (int32_t p : sub_ids) {
                if (ids->size() >= limit) break;
                ids->push_back(p);
            }
        }
    }
    ids->push_back(sep_id);
}

// Viterbi over byte positions: best[e] = max over pieces p ending at e (starting at a
// reachable position s, e on a character boundary) of best[s] + score(p).  Starts are
// visited in increasing order and, per start, pieces by increasing length; a candidate
// replaces the current best only if strictly greater, so ties keep the earliest.
void ceb_tokenizer::unigram(const std::string& text, std::vector<int32_t>* out) const {
    const int n = (int)text.size();
    if (n == 0) return;
    const float kUnreached = -1e30f;
    std::vector<float> best(n + 1, kUnreached);
    std::vector<int> from(n + 1, -1), piece(n + 1, -1);
    best[0] = 0.0f;
    for (int s = 0; s < n; ++s) {
        if (best[s] <= -1e29f) continue;
        int node = 0;
        for (int e = s; e < n; ++e) {
            const unsigned char c = (unsigned char)text[e];
            int ch = trie_[node].child;
            while (ch >= 0 && trie_[ch].byte != c) ch = trie_[ch].sibling;
            if (ch < 0) break;
            node = ch;
            const int end = e + 1;
            if (trie_[node].id < 0) continue;
            if (end < n && ((unsigned char)text[end] & 0xC0) == 0x80) continue;  // not a character boundary
            const float cand = best[s] + scores[trie_[node].id];
            if (cand > best[end]) {
                best[end] = cand;
                from[end] = s;
                piece[end] = trie_[node].id;
            }
        }
        if (best[s + 1] <= -1e29f) {  // nothing reaches the next byte: byte fallback
            const int b = (unsigned char)text[s];
            const int id = byte_piece[b] >= 0 ? byte_piece[b] : unk_id;
            const float cand = best[s] - 100.0f;
            if (cand > best[s + 1]) {
                best[s + 1] = cand;
                from[s + 1] = s;
                piece[s + 1] = id;
            }
        }
    }
    std::vector<int32_t> rev;
    for (int pos = n; pos > 0;) {
        if (piece[pos] < 0) {
            --pos;
            continue;
        }
        rev.push_back(piece[pos]);
        pos = from[pos];
    }
    out->assign(rev.rbegin(), rev.rend());
}

int ceb_tokenizer::encode(const std::string& text, std::vector<int32_t>* ids) const {
    ids->clear();
    if (family == 0) {
        wordpiece(text, ids);
        return 0;
    }
    if (family != 2)
        return ceb_set_error(1, "tokenizer family %d (BPE) is not implemented by this build; "
                                "use crispembed_encode_ids_batch",
                             family);
    std::string marked;
    marked.reserve(text.size() * 3 + 3);
    for (char c : " " + (spm_normalize ? ceb_spm_normalize(text) : text)) {
        if (c == ' ')
            marked += "\xe2\x96\x81";  // U+2581
        else
            marked += c;
    }
    std::vector<int32_t> body;
    unigram(marked, &body);
    if (add_bos) ids->push_back(bos_id);
    const size_t cap = (size_t)max_tokens - (add_eos ? 1 : 0);
    for (int32_t id : body) {
        if (ids->size() >= cap) break;
        ids->push_back(id);
    }
    if (add_eos) ids->push_back(eos_id);
    return 0;
}
