// multimodal.cpp -- MultimodalSequence (Sources/GemmaEmbed/MultimodalEmbedding.swift:43-83).
#include "multimodal.hpp"

#include <algorithm>

namespace ge {

bool multimodal_sequence(const std::string& prefix, const std::vector<SeqPart>& in_parts,
                         const std::vector<EncoderSpan>& spans, int max_tokens, int32_t bos, int32_t eos,
                         const std::function<void(const std::string&, std::vector<int32_t>&)>& encode,
                         std::vector<int32_t>& ids, bool& truncated) {
    // The prefix joins the first text, or leads on its own before an image or clip.
    std::vector<SeqPart> parts = in_parts;
    if (!parts.empty() && parts[0].kind == kPartText) {
        parts[0].text = prefix + parts[0].text;
    } else {
        SeqPart p;
        p.kind = kPartText;
        p.text = prefix;
        parts.insert(parts.begin(), p);
    }
    // Encoded texts; nothing for the encoder parts.
    std::vector<std::vector<int32_t>> texts(parts.size());
    std::vector<bool> is_text(parts.size());
    size_t nspans = 0;
    for (size_t i = 0; i < parts.size(); i++) {
        is_text[i] = parts[i].kind == kPartText;
        if (is_text[i]) encode(parts[i].text, texts[i]);
        else nspans++;
    }
    if (nspans != spans.size()) return false;
    int64_t fixed = 2;
    for (const EncoderSpan& s : spans) fixed += s.rows + 2;
    if (fixed > max_tokens) return false;
    int64_t excess = fixed - max_tokens;
    for (size_t i = 0; i < parts.size(); i++)
        if (is_text[i]) excess += int64_t(texts[i].size());
    truncated = excess > 0;
    // Cut text from the end: the last text part first, from its end.
    for (size_t i = parts.size(); i-- > 0 && excess > 0;) {
        if (!is_text[i]) continue;
        const int64_t cut = std::min<int64_t>(excess, int64_t(texts[i].size()));
        texts[i].resize(texts[i].size() - size_t(cut));
        excess -= cut;
    }
    ids.clear();
    ids.push_back(bos);
    int32_t row = 0;
    size_t k = 0;
    for (size_t i = 0; i < parts.size(); i++) {
        if (is_text[i]) {
            ids.insert(ids.end(), texts[i].begin(), texts[i].end());
            continue;
        }
        const EncoderSpan& s = spans[k++];
        ids.push_back(s.begin);
        for (int r = 0; r < s.rows; r++) ids.push_back(-(row + r) - 1);
        ids.push_back(s.end);
        row += s.rows;
    }
    ids.push_back(eos);
    return true;
}

}  // namespace ge
