// tokenizer.cpp — vocabulary container with the reference's Tokenizer
// interface.  Tokenization is outside the decode path (the benchmark and
// the tests feed token IDs); encode() is a greedy longest match.
#include "tokenizer.h"

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <fstream>

namespace {
const char kSpace[] = "\xe2\x96\x81";  // U+2581, SentencePiece's space marker
}

Tokenizer::Tokenizer() : bos_id_(1), eos_id_(2), max_token_length_(0) {}

bool Tokenizer::load(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) return false;
    uint32_t n = 0, max_len = 0;
    f.read(reinterpret_cast<char*>(&n), 4);
    f.read(reinterpret_cast<char*>(&max_len), 4);
    if (!f.good() || n == 0) return false;
    std::vector<std::string> vocab(n);
    std::vector<float> scores(n);
    for (uint32_t i = 0; i < n; ++i) {
        int32_t len = 0;
        f.read(reinterpret_cast<char*>(&scores[i]), 4);
        f.read(reinterpret_cast<char*>(&len), 4);
        if (!f.good() || len < 0) return false;
        vocab[i].resize(len);
        f.read(&vocab[i][0], len);
    }
    load_from_vocab(vocab, scores);
    max_token_length_ = (int)max_len;
    return f.good();
}

void Tokenizer::load_from_vocab(const std::vector<std::string>& vocab, const std::vector<float>& scores) {
    id_to_token_ = vocab;
    id_to_score_ = scores;
    token_to_id_.clear();
    max_token_length_ = 0;
    for (size_t i = 0; i < vocab.size(); ++i) {
        token_to_id_[vocab[i]] = (int)i;
        if ((int)vocab[i].size() > max_token_length_) max_token_length_ = (int)vocab[i].size();
    }
    auto b = token_to_id_.find("<s>");
    if (b != token_to_id_.end()) bos_id_ = b->second;
    auto e = token_to_id_.find("</s>");
    if (e != token_to_id_.end()) eos_id_ = e->second;
}

std::vector<int> Tokenizer::encode(const std::string& text, bool bos, bool eos) const {
    std::vector<int> out;
    if (bos) out.push_back(bos_id_);
    std::string s = kSpace;
    for (char c : text) {
        if (c == ' ')
            s += kSpace;
        else
            s += c;
    }
    size_t i = 0;
    while (i < s.size()) {
        int best = -1;
        size_t best_len = 0;
        const size_t lim = std::min(s.size() - i, (size_t)std::max(max_token_length_, 1));
        for (size_t len = lim; len >= 1; --len) {
            auto it = token_to_id_.find(s.substr(i, len));
            if (it != token_to_id_.end()) {
                best = it->second;
                best_len = len;
                break;
            }
        }
        if (best < 0) {  // byte fallback
            char buf[8];
            std::snprintf(buf, sizeof(buf), "<0x%02X>", (unsigned)(unsigned char)s[i]);
            auto it = token_to_id_.find(buf);
            out.push_back(it != token_to_id_.end() ? it->second : 0);
            best_len = 1;
        } else {
            out.push_back(best);
        }
        i += best_len;
    }
    if (eos) out.push_back(eos_id_);
    return out;
}

std::string Tokenizer::decode(int id) const {
    if (id < 0 || id >= (int)id_to_token_.size()) return "";
    if (id == bos_id_ || id == eos_id_) return "";
    const std::string& p = id_to_token_[id];
    if (p.size() == 6 && p.rfind("<0x", 0) == 0 && p[5] == '>') {
        return std::string(1, (char)std::stoi(p.substr(3, 2), nullptr, 16));
    }
    std::string r;
    for (size_t i = 0; i < p.size();) {
        if (p.compare(i, 3, kSpace) == 0) {
            r += ' ';
            i += 3;
        } else {
            r += p[i++];
        }
    }
    return r;
}

std::string Tokenizer::decode(const std::vector<int>& tokens) const {
    std::string r;
    for (int t : tokens) r += decode(t);
    if (!r.empty() && r[0] == ' ') r.erase(0, 1);
    return r;
}

int Tokenizer::vocab_size() const { return (int)id_to_token_.size(); }
int Tokenizer::bos_id() const { return bos_id_; }
int Tokenizer::eos_id() const { return eos_id_; }
