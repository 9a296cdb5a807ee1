// tokenizer.h — vocabulary container with the reference's Tokenizer
// interface (include/tokenizer.h:7-30).  Tokenization is outside the decode
// path: encode() here is a plain greedy longest match over the vocabulary
// (with the SentencePiece "▁" space marker and <0xXX> byte fallback),
// not the reference's score-ordered merges.  Benchmarks feed token IDs.
#pragma once

#include <string>
#include <unordered_map>
#include <vector>

class Tokenizer {
public:
    Tokenizer();
    ~Tokenizer() = default;

    // Reads the reference's tokenizer.bin: u32 vocab_size, u32 max_len, then
    // per token f32 score, i32 length, bytes.
    bool load(const std::string& binary_path);
    void load_from_vocab(const std::vector<std::string>& vocab, const std::vector<float>& scores);

    std::vector<int> encode(const std::string& text, bool bos = true, bool eos = false) const;
    std::string decode(int token_id) const;
    std::string decode(const std::vector<int>& tokens) const;

    int vocab_size() const;
    int bos_id() const;
    int eos_id() const;

private:
    std::vector<std::string> id_to_token_;
    std::vector<float> id_to_score_;
    std::unordered_map<std::string, int> token_to_id_;
    int bos_id_;
    int eos_id_;
    int max_token_length_;
};
