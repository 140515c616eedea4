// tokenizer.h -- host-side tokenizers of the text ABI (crispembed_encode*).
//
// Families follow the reference's numbering of `tokenizer.ggml.type`
// (src/tokenizer.h:37-52): 0 WordPiece, 1 BPE, 2 SentencePiece Unigram.
//   WordPiece      BERT basic tokenizer (whitespace split, ASCII punctuation
//                  isolated, optional lower-casing) + greedy longest-match-first
//                  with "##" continuations, wrapped [CLS] ... [SEP]
//                  (src/crispembed.cpp:666-680 selects it).
//   SentencePiece  XLM-R style Unigram (src/tokenizer_spm.cpp): a leading space
//                  is prepended, every space becomes U+2581, and the segmentation
//                  maximising the sum of the pieces' scores is found by Viterbi
//                  over UTF-8 character boundaries; bytes no piece covers fall
//                  back to "<0xXX>" pieces (score -100) or <unk>; wrapped
//                  <s> ... </s> as tokenizer.ggml.add_bos_token / add_eos_token say.
//                  Before that, every codepoint goes through SentencePiece's
//                  nmt_nfkc charsmap (fullwidth forms, U+2026, U+3000, ligatures,
//                  control characters, ...), one codepoint at a time as the
//                  reference's embedding path does (ceb_spm_normalize).
// Not implemented: GPT-2 BPE (decoder-style models).
#pragma once

#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

class ceb_gguf;

// The reference's family decision: a numeric tokenizer.ggml.type is final; else
// the tokenizer.ggml.model string decides; else vocabularies above 100k tokens
// are SentencePiece.
int ceb_tokenizer_family(bool type_key_present, int declared_type, const std::string& model_str, int64_t vocab_n);

// SentencePiece nmt_nfkc normalisation, codepoint by codepoint (printable ASCII unchanged).
std::string ceb_spm_normalize(const std::string& text);

struct ceb_tokenizer {
    int family = 0;
    int max_tokens = 512;  // including the wrap tokens
    std::vector<std::string> pieces;
    std::unordered_map<std::string, int> index;
    // WordPiece
    int cls_id = 101, sep_id = 102, unk_id = 100, pad_id = 0;
    bool lower = true;
    // SentencePiece
    std::vector<float> scores;
    int bos_id = 0, eos_id = 2;
    bool add_bos = true, add_eos = true;
    bool spm_normalize = true;  // nmt_nfkc charsmap before segmentation (the reference's embedding path)
    std::vector<int32_t> byte_piece;  // id of "<0xXX>" per byte value, -1 when absent

    // Reads the tokenizer keys of an open GGUF; returns 0 or an error code (message via ceb_set_error).
    int load(const ceb_gguf& g, int max_tok);
    // Wrapped, truncated ids of `text`; returns 0 or an error code.
    int encode(const std::string& text, std::vector<int32_t>* ids) const;
    // Surface form of a piece ("" out of range).
    const std::string& token_str(int id) const;
    // crispembed_tokenizer_kind numbering: 1 WordPiece, 2 SentencePiece, 3 BPE.
    int kind() const { return family == 2 ? 2 : family == 1 ? 3 : 1; }

   private:
    struct Node {
        int child = -1, sibling = -1, id = -1;
        uint8_t byte = 0;
    };
    std::vector<Node> trie_;
    void build_trie();
    void wordpiece(const std::string& text, std::vector<int32_t>* ids) const;
    void unigram(const std::string& text, std::vector<int32_t>* out) const;
};
