// tokenizer.hpp -- the Gemma 4 style BPE tokenizer carried by the GGUF file.
//
// Behaviour of Sources/GemmaEmbed/Tokenizer/Tokenizer.swift (llama.cpp's `gemma4` vocabulary):
// raw UTF-8 with U+2581 for spaces (Tokenizer.swift:205-210), runs of newlines and of other
// bytes encoded separately (211-218), a newline run that is itself a piece kept whole
// (236-240), otherwise UTF-8 characters merged by the lowest-ranked merge, leftmost first
// (241-270, min-heap 293-327), and `<0xXX>` byte fallback for symbols outside the vocabulary
// (271-281).  Special-token text is recognised only on request (170-188); decode drops
// control, unknown and unused tokens, reassembles byte tokens and turns U+2581 back into
// spaces (120-147).
//
// Strings are compared as bytes, as llama.cpp does.  (Swift's String keys also identify
// canonically equivalent spellings, e.g. a precomposed letter and its decomposed form; the
// two agree on every text whose characters and pieces are written the same way.)
#pragma once

#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

namespace ge {

class GgufFile;
struct GgufError;

// Open-addressing hash table from 64-bit keys to 64-bit values (linear probing, power-of-two
// capacity, never more than half full).  Keys must not be ~0, the empty marker.
class FlatMap64 {
public:
    void reset(size_t expected);
    // Inserts (key, value) unless the key is present; returns false when it was.
    bool insert(uint64_t key, uint64_t value);
    const uint64_t* find(uint64_t key) const {
        if (slots_.empty()) return nullptr;
        for (size_t i = hash(key) & mask_;; i = (i + 1) & mask_) {
            const Slot& s = slots_[i];
            if (s.key == key) return &s.value;
            if (s.key == kEmpty) return nullptr;
        }
    }
    size_t size() const { return size_; }

private:
    static constexpr uint64_t kEmpty = ~0ull;
    struct Slot {
        uint64_t key, value;
    };
    static size_t hash(uint64_t k) {
        k ^= k >> 33;
        k *= 0xff51afd7ed558ccdull;
        k ^= k >> 33;
        return size_t(k);
    }
    void grow();
    std::vector<Slot> slots_;
    size_t mask_ = 0, size_ = 0;
};

class Tokenizer {
public:
    enum TokenType : int32_t { kNormal = 1, kUnknown = 2, kControl = 3, kUserDefined = 4, kUnused = 5, kByte = 6 };

    // Tokenizer(gguf:) (Tokenizer.swift:40-56): returns 0 or a status code with `err` filled in.
    int build(const GgufFile& f, GgufError& err);
    // init(tokens:types:merges:...) (Tokenizer.swift:57-98).
    void build(std::vector<std::string> tokens, std::vector<int32_t> types, const std::vector<std::string>& merges,
               int32_t bos, int32_t eos, int32_t pad, int32_t unk, bool add_bos, bool add_eos);

    // encode(_:addSpecialTokens:parseSpecialTokens:) (Tokenizer.swift:105-117); appends to `out`.
    void encode(const uint8_t* text, size_t n, bool add_special, bool parse_special, std::vector<int32_t>& out) const;
    // decode(_:) (Tokenizer.swift:120-147): UTF-8 bytes, which may be an invalid sequence when
    // byte tokens split a character.
    void decode(const int32_t* ids, size_t n, std::string& out) const;

    const std::string* piece(int32_t id) const {
        return id >= 0 && size_t(id) < pieces_.size() ? &pieces_[size_t(id)] : nullptr;
    }
    bool is_control(int32_t id) const {
        return id >= 0 && size_t(id) < types_.size() && types_[size_t(id)] == kControl;
    }
    int32_t vocabulary_size() const { return int32_t(pieces_.size()); }

    int32_t bos_id = 2, eos_id = 1, pad_id = 0, unknown_id = -1;
    bool add_bos = true, add_eos = false;

private:
    struct Special {
        int32_t id;
        std::string text;
    };

    int32_t intern(const std::string& s);
    int32_t char_symbol(const uint8_t* p, int len) const;
    void encode_fragment(const uint8_t* p, size_t n, std::vector<int32_t>& out) const;
    void encode_word(const uint8_t* w, size_t n, bool all_newlines, std::vector<int32_t>& out) const;
    // The merge loop over one word; `whole` >= 0 makes the word a single symbol.
    void merge_word(const uint8_t* w, size_t n, int32_t whole, std::vector<int32_t>& out) const;

    std::vector<std::string> pieces_;
    std::vector<int32_t> types_;
    std::unordered_map<std::string, int32_t> piece_to_id_;  // first id of each piece
    // Every string a symbol can hold while merging -- vocabulary pieces, merge halves and merge
    // results -- gets a symbol id; merges are keyed by the two halves' symbol ids.
    std::unordered_map<std::string, int32_t> symbols_;
    std::vector<int32_t> symbol_token_;                // symbol id -> token id, or -1 (not a piece)
    int32_t byte_symbols_[256];  // one-byte character -> symbol id, or -1
    FlatMap64 char_symbols_;     // one UTF-8 character of 2..4 bytes -> symbol id
    FlatMap64 merges_;           // (left symbol << 32 | right symbol) -> (rank << 32 | result symbol)
    int32_t byte_to_id_[256];
    std::vector<Special> specials_;  // control, user-defined and unknown tokens, longest first
    bool split_words_ = true;         // no merge joins across a U+2581 that follows another character
    uint64_t instance_id_ = 0;        // distinguishes tokenizers in the per-thread word cache
};

}  // namespace ge
