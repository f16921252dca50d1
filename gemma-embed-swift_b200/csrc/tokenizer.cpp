// tokenizer.cpp -- encode and decode for the Gemma 4 style BPE tokenizer (tokenizer.hpp).
//
// The merge loop works on small integer symbol ids instead of strings: every string that a
// symbol can hold (a vocabulary piece, either half of a merge, a merge result) is interned
// once at build time, so a bigram lookup is one hash of two ids and the token id of a merged
// symbol is a table read.  A UTF-8 character that is no such string can take part in no merge
// and falls back to byte tokens, exactly as the string-keyed lookups of the reference decide.
#include "tokenizer.hpp"

#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <numeric>

#include "gemma_embed.h"
#include "gguf.hpp"

namespace ge {

namespace {

const uint8_t kSpace[3] = {0xE2, 0x96, 0x81};  // U+2581

// Byte length of the UTF-8 sequence a lead byte starts (Tokenizer.swift:284-290); a stray
// continuation or invalid byte counts as one.
inline int utf8_length(uint8_t lead) {
    if (lead < 0x80) return 1;
    if ((lead & 0xE0) == 0xC0) return 2;
    if ((lead & 0xF0) == 0xE0) return 3;
    if ((lead & 0xF8) == 0xF0) return 4;
    return 1;
}

inline uint64_t char_key(const uint8_t* p, int len) {
    uint64_t k = uint64_t(len) << 32;
    for (int i = 0; i < len; i++) k |= uint64_t(p[i]) << (8 * i);
    return k;
}

inline uint64_t pair_key(int32_t a, int32_t b) { return (uint64_t(uint32_t(a)) << 32) | uint32_t(b); }

// byteValue(ofPiece:) (Tokenizer.swift:160-163): "<0x" + two hex digits + ">", the form every
// byte-typed piece of a GGUF vocabulary has.
bool byte_value(const std::string& p, uint8_t& out) {
    if (p.size() != 6 || p.compare(0, 3, "<0x") != 0 || p[5] != '>') return false;
    int v = 0;
    for (int i = 3; i < 5; i++) {
        const char c = p[size_t(i)];
        int d;
        if (c >= '0' && c <= '9') d = c - '0';
        else if (c >= 'a' && c <= 'f') d = c - 'a' + 10;
        else if (c >= 'A' && c <= 'F') d = c - 'A' + 10;
        else return false;
        v = v * 16 + d;
    }
    out = uint8_t(v);
    return true;
}

struct Symbol {
    int32_t start, length, prev, next;
    int32_t sym;  // interned string id, -1 when the string is no piece or merge half
};

// A candidate merge.  `order` = rank << 32 | left index: the reference's min-heap order on
// (rank, left) (Tokenizer.swift:296-298) as one integer.
struct Bigram {
    uint64_t order;
    int32_t right, left_length, right_length, result;
};

inline bool heap_after(const Bigram& a, const Bigram& b) { return a.order > b.order; }

struct Scratch {
    std::vector<uint8_t> escaped;
    std::vector<Symbol> symbols;
    std::vector<Bigram> heap;
};

Scratch& scratch() {
    thread_local Scratch s;
    return s;
}

struct WordCache {
    uint64_t owner = 0;  // instance id of the tokenizer the entries belong to
    std::unordered_map<std::string, std::vector<int32_t>> map;
};

WordCache& word_cache() {
    thread_local WordCache c;
    return c;
}

constexpr size_t kWordCacheEntries = 1 << 16;

std::atomic<uint64_t> g_instances{0};

// True when the last character of `s` (split as a word is) is U+2581.
bool ends_with_space_char(const std::string& s) {
    size_t off = 0, last = 0, last_len = 0;
    while (off < s.size()) {
        const size_t len = std::min(s.size() - off, size_t(utf8_length(uint8_t(s[off]))));
        last = off;
        last_len = len;
        off += len;
    }
    return last_len == 3 && memcmp(s.data() + last, kSpace, 3) == 0;
}

}  // namespace

void FlatMap64::reset(size_t expected) {
    size_t cap = 16;
    while (cap < 2 * expected) cap <<= 1;
    slots_.assign(cap, Slot{kEmpty, 0});
    mask_ = cap - 1;
    size_ = 0;
}

void FlatMap64::grow() {
    std::vector<Slot> old;
    old.swap(slots_);
    reset(old.size());
    for (const Slot& s : old)
        if (s.key != kEmpty) insert(s.key, s.value);
}

bool FlatMap64::insert(uint64_t key, uint64_t value) {
    if (slots_.empty() || 2 * (size_ + 1) > slots_.size()) grow();
    for (size_t i = hash(key) & mask_;; i = (i + 1) & mask_) {
        Slot& s = slots_[i];
        if (s.key == key) return false;
        if (s.key == kEmpty) {
            s = Slot{key, value};
            size_++;
            return true;
        }
    }
}

int32_t Tokenizer::intern(const std::string& s) {
    auto it = symbols_.find(s);
    if (it != symbols_.end()) return it->second;
    const int32_t id = int32_t(symbol_token_.size());
    symbols_.emplace(s, id);
    auto p = piece_to_id_.find(s);
    symbol_token_.push_back(p == piece_to_id_.end() ? -1 : p->second);
    // A string no longer than the sequence its lead byte starts can be one character of a
    // word (a shorter one ends a word in mid-sequence).
    if (s.size() == 1) byte_symbols_[uint8_t(s[0])] = id;
    else if (!s.empty() && int(s.size()) <= utf8_length(uint8_t(s[0])))
        char_symbols_.insert(char_key(reinterpret_cast<const uint8_t*>(s.data()), int(s.size())), uint64_t(id));
    return id;
}

int32_t Tokenizer::char_symbol(const uint8_t* p, int len) const {
    if (len == 1) return byte_symbols_[p[0]];
    const uint64_t* v = char_symbols_.find(char_key(p, len));
    return v ? int32_t(*v) : -1;
}

void Tokenizer::build(std::vector<std::string> tokens, std::vector<int32_t> types, const std::vector<std::string>& merges,
                      int32_t bos, int32_t eos, int32_t pad, int32_t unk, bool add_bos_, bool add_eos_) {
    pieces_ = std::move(tokens);
    types_ = std::move(types);
    bos_id = bos;
    eos_id = eos;
    pad_id = pad;
    unknown_id = unk;
    add_bos = add_bos_;
    add_eos = add_eos_;
    piece_to_id_.clear();
    symbols_.clear();
    symbol_token_.clear();
    for (int32_t& b : byte_symbols_) b = -1;
    split_words_ = true;
    instance_id_ = ++g_instances;
    char_symbols_.reset(1024);
    merges_.reset(merges.size());
    specials_.clear();
    piece_to_id_.reserve(pieces_.size());
    for (size_t i = 0; i < pieces_.size(); i++) piece_to_id_.emplace(pieces_[i], int32_t(i));  // first id wins
    symbols_.reserve(pieces_.size() + merges.size());
    symbol_token_.reserve(pieces_.size() + merges.size());
    for (const std::string& p : pieces_) intern(p);
    // Merge rules "left right", split at the first space after the first byte; the first rank
    // of a repeated pair wins (Tokenizer.swift:75-81).
    std::string left, right;
    for (size_t r = 0; r < merges.size(); r++) {
        const std::string& m = merges[r];
        if (m.size() < 2) continue;
        const size_t split = m.find(' ', 1);
        if (split == std::string::npos) continue;
        left.assign(m, 0, split);
        right.assign(m, split + 1, std::string::npos);
        if (right.empty()) continue;  // an empty half never matches a symbol
        if (right.size() >= 3 && memcmp(right.data(), kSpace, 3) == 0 && !ends_with_space_char(left))
            split_words_ = false;  // this merge can join across a word start
        const int32_t a = intern(left), b = intern(right);
        const uint64_t key = pair_key(a, b);
        if (merges_.find(key)) continue;
        const int32_t res = intern(left + right);
        merges_.insert(key, (uint64_t(r) << 32) | uint32_t(res));
    }
    for (int b = 0; b < 256; b++) {
        char name[8];
        snprintf(name, sizeof name, "<0x%02X>", b);
        auto it = piece_to_id_.find(name);
        const bool ok = it != piece_to_id_.end() && size_t(it->second) < types_.size() && types_[size_t(it->second)] == kByte;
        byte_to_id_[b] = ok ? it->second : -1;
    }
    for (size_t i = 0; i < types_.size(); i++) {
        const int32_t t = types_[i];
        if (t == kControl || t == kUserDefined || t == kUnknown) specials_.push_back({int32_t(i), pieces_[i]});
    }
    std::stable_sort(specials_.begin(), specials_.end(),
                     [](const Special& a, const Special& b) { return a.text.size() > b.text.size(); });
}

int Tokenizer::build(const GgufFile& f, GgufError& err) {
    std::string model;
    if (!f.get_string("tokenizer.ggml.model", model) || model != "gemma4") {
        err = {GE_ERR_UNSUPPORTED_ARCHITECTURE,
               "unsupported architecture: tokenizer model " + (model.empty() ? std::string("missing") : model)};
        return err.code;
    }
    std::vector<std::string> tokens, merges;
    std::vector<int32_t> types;
    auto missing = [&](const char* key) {
        err = {GE_ERR_MISSING_METADATA, std::string("weight file lacks metadata key ") + key};
        return err.code;
    };
    if (!f.get_string_array("tokenizer.ggml.tokens", tokens)) return missing("tokenizer.ggml.tokens");
    if (!f.get_int_array("tokenizer.ggml.token_type", types)) return missing("tokenizer.ggml.token_type");
    if (!f.get_string_array("tokenizer.ggml.merges", merges)) return missing("tokenizer.ggml.merges");
    int64_t bos, eos, pad = 0, unk = -1;
    if (!f.get_int("tokenizer.ggml.bos_token_id", bos)) return missing("tokenizer.ggml.bos_token_id");
    if (!f.get_int("tokenizer.ggml.eos_token_id", eos)) return missing("tokenizer.ggml.eos_token_id");
    f.get_int("tokenizer.ggml.padding_token_id", pad);
    f.get_int("tokenizer.ggml.unknown_token_id", unk);
    if (types.size() != tokens.size()) {
        err = {GE_ERR_INVALID_GGUF, "invalid GGUF file: tokenizer.ggml.token_type has " + std::to_string(types.size()) +
                                        " entries for " + std::to_string(tokens.size()) + " tokens"};
        return err.code;
    }
    bool add_bos_ = true, add_eos_ = false;
    f.get_bool("tokenizer.ggml.add_bos_token", add_bos_);
    f.get_bool("tokenizer.ggml.add_eos_token", add_eos_);
    build(std::move(tokens), std::move(types), merges, int32_t(bos), int32_t(eos), int32_t(pad), int32_t(unk), add_bos_,
          add_eos_);
    return 0;
}

void Tokenizer::encode(const uint8_t* text, size_t n, bool add_special, bool parse_special,
                       std::vector<int32_t>& out) const {
    if (add_special && add_bos) out.push_back(bos_id);
    if (!parse_special) {
        encode_fragment(text, n, out);
    } else {
        // partition(_:parseSpecial:) (Tokenizer.swift:170-188): each special token in turn,
        // longest first, splits the remaining text fragments at its left-to-right matches.
        struct Frag {
            size_t begin, end;
            int32_t id;  // >= 0: a special token
        };
        std::vector<Frag> frags{{0, n, -1}}, next;
        for (const Special& sp : specials_) {
            if (sp.text.empty()) continue;
            next.clear();
            const size_t m = sp.text.size();
            for (const Frag& fr : frags) {
                if (fr.id >= 0) {
                    next.push_back(fr);
                    continue;
                }
                size_t start = fr.begin;
                while (fr.end - start >= m) {
                    const uint8_t* hit = std::search(text + start, text + fr.end, sp.text.begin(), sp.text.end(),
                                                     [](uint8_t a, char b) { return a == uint8_t(b); });
                    if (hit == text + fr.end) break;
                    const size_t at = size_t(hit - text);
                    if (at > start) next.push_back({start, at, -1});
                    next.push_back({0, 0, sp.id});
                    start = at + m;
                }
                if (start < fr.end) next.push_back({start, fr.end, -1});
            }
            frags.swap(next);
        }
        for (const Frag& fr : frags) {
            if (fr.id >= 0) out.push_back(fr.id);
            else encode_fragment(text + fr.begin, fr.end - fr.begin, out);
        }
    }
    if (add_special && add_eos) out.push_back(eos_id);
}

void Tokenizer::encode_fragment(const uint8_t* p, size_t n, std::vector<int32_t>& out) const {
    // Spaces become U+2581, then runs of newlines and runs of other bytes are encoded apart
    // (Tokenizer.swift:205-218).
    std::vector<uint8_t>& escaped = scratch().escaped;
    escaped.clear();
    for (size_t i = 0; i < n; i++) {
        if (p[i] == 0x20) escaped.insert(escaped.end(), kSpace, kSpace + 3);
        else escaped.push_back(p[i]);
    }
    size_t i = 0;
    while (i < escaped.size()) {
        const bool nl = escaped[i] == 0x0A;
        size_t j = i + 1;
        while (j < escaped.size() && (escaped[j] == 0x0A) == nl) j++;
        encode_word(escaped.data() + i, j - i, nl, out);
        i = j;
    }
}

void Tokenizer::encode_word(const uint8_t* w, size_t n, bool all_newlines, std::vector<int32_t>& out) const {
    if (all_newlines) {
        auto it = symbols_.find(std::string(reinterpret_cast<const char*>(w), n));
        const bool whole = it != symbols_.end() && symbol_token_[size_t(it->second)] >= 0;
        merge_word(w, n, whole ? it->second : -1, out);
        return;
    }
    if (!split_words_) {
        merge_word(w, n, -1, out);
        return;
    }
    // No merge joins a symbol ending in another character to one starting with U+2581, so
    // each U+2581 that follows another character starts a word that merges on its own; a
    // word's ids depend on its bytes alone and are kept in a per-thread cache.
    WordCache& cache = word_cache();
    if (cache.owner != instance_id_ || cache.map.size() > kWordCacheEntries) {
        cache.map.clear();
        cache.owner = instance_id_;
    }
    size_t begin = 0, off = 0;
    bool prev_space = false;
    auto flush = [&](size_t end) {
        if (end == begin) return;
        std::string key(reinterpret_cast<const char*>(w + begin), end - begin);
        auto it = cache.map.find(key);
        if (it == cache.map.end()) {
            std::vector<int32_t> ids;
            merge_word(w + begin, end - begin, -1, ids);
            it = cache.map.emplace(std::move(key), std::move(ids)).first;
        }
        out.insert(out.end(), it->second.begin(), it->second.end());
    };
    while (off < n) {
        const size_t len = std::min(n - off, size_t(utf8_length(w[off])));
        const bool space = len == 3 && w[off] == kSpace[0] && w[off + 1] == kSpace[1] && w[off + 2] == kSpace[2];
        if (space && !prev_space && off > begin) {
            flush(off);
            begin = off;
        }
        prev_space = space;
        off += len;
    }
    flush(n);
}

void Tokenizer::merge_word(const uint8_t* w, size_t n, int32_t whole, std::vector<int32_t>& out) const {
    Scratch& sc = scratch();
    std::vector<Symbol>& syms = sc.symbols;
    std::vector<Bigram>& heap = sc.heap;
    syms.clear();
    heap.clear();
    if (whole >= 0) {
        syms.push_back({0, int32_t(n), -1, -1, whole});
    } else {
        size_t off = 0;
        while (off < n) {
            const int len = int(std::min(n - off, size_t(utf8_length(w[off]))));
            const int32_t idx = int32_t(syms.size());
            syms.push_back({int32_t(off), len, idx - 1, off + size_t(len) == n ? -1 : idx + 1, char_symbol(w + off, len)});
            off += size_t(len);
        }
    }
    auto push = [&](int32_t l, int32_t r) {
        if (l < 0 || r < 0) return;
        const Symbol& a = syms[size_t(l)];
        const Symbol& b = syms[size_t(r)];
        if (a.sym < 0 || b.sym < 0) return;
        const uint64_t* m = merges_.find(pair_key(a.sym, b.sym));
        if (!m) return;
        heap.push_back({(*m & 0xFFFFFFFF00000000ull) | uint32_t(l), r, a.length, b.length, int32_t(uint32_t(*m))});
        std::push_heap(heap.begin(), heap.end(), heap_after);
    };
    for (size_t i = 1; i < syms.size(); i++) push(int32_t(i - 1), int32_t(i));
    while (!heap.empty()) {
        std::pop_heap(heap.begin(), heap.end(), heap_after);
        const Bigram bg = heap.back();
        heap.pop_back();
        const int32_t left = int32_t(uint32_t(bg.order));
        Symbol& l = syms[size_t(left)];
        Symbol& r = syms[size_t(bg.right)];
        if (l.length == 0 || r.length == 0 || l.length != bg.left_length || r.length != bg.right_length) continue;
        l.length += r.length;
        l.sym = bg.result;
        r.length = 0;
        l.next = r.next;
        if (r.next >= 0) syms[size_t(r.next)].prev = left;
        push(l.prev, left);
        push(left, l.next);
    }
    for (const Symbol& s : syms) {
        if (s.length == 0) continue;
        const int32_t tok = s.sym >= 0 ? symbol_token_[size_t(s.sym)] : -1;
        if (tok >= 0) {
            out.push_back(tok);
        } else {
            for (int32_t k = 0; k < s.length; k++) {
                const int32_t id = byte_to_id_[w[s.start + k]];
                if (id >= 0) out.push_back(id);
            }
        }
    }
}

void Tokenizer::decode(const int32_t* ids, size_t n, std::string& out) const {
    std::string bytes;
    for (size_t k = 0; k < n; k++) {
        const int32_t id = ids[k];
        if (id < 0 || size_t(id) >= pieces_.size()) continue;
        const int32_t t = size_t(id) < types_.size() ? types_[size_t(id)] : kNormal;
        if (t == kControl || t == kUnknown || t == kUnused) continue;
        const std::string& p = pieces_[size_t(id)];
        uint8_t b;
        if (t == kByte && byte_value(p, b)) bytes.push_back(char(b));
        else bytes += p;
    }
    out.clear();
    out.reserve(bytes.size());
    for (size_t i = 0; i < bytes.size();) {
        if (i + 2 < bytes.size() && uint8_t(bytes[i]) == kSpace[0] && uint8_t(bytes[i + 1]) == kSpace[1] &&
            uint8_t(bytes[i + 2]) == kSpace[2]) {
            out.push_back(' ');
            i += 3;
        } else {
            out.push_back(bytes[i]);
            i++;
        }
    }
}

}  // namespace ge
