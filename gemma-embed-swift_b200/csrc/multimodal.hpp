// multimodal.hpp -- the text-tower sequence of an input that mixes text with image (and audio)
// spans (MultimodalSequence, Sources/GemmaEmbed/MultimodalEmbedding.swift:27-84).
#pragma once

#include <stdint.h>

#include <functional>
#include <string>
#include <vector>

namespace ge {

enum PartKind : int32_t { kPartText = 0, kPartImage = 1, kPartAudio = 2 };

struct SeqPart {
    int32_t kind = kPartText;
    std::string text;  // kPartText only
};

// An image's or a clip's rows inside the input and the tokens that frame them (EncoderSpan).
struct EncoderSpan {
    int rows = 0;
    int32_t begin = 0, end = 0;
};

// MultimodalSequence.init (MultimodalEmbedding.swift:43-83): `[bos] tok(prefix + first text)
// [begin] -1 ... -R [end] tok(text) ... [eos]`, where the k-th image or clip takes spans[k] and
// its rows are numbered -(r + 1) across the input's spans in order.  The prefix joins the first
// text, or leads on its own when the input opens with an image or clip.  Text is cut from the
// end (the last text part first) until the sequence fits `max_tokens`; returns false when the
// spans and their frames alone do not fit.  `encode` tokenizes without BOS/EOS.
bool multimodal_sequence(const std::string& prefix, const std::vector<SeqPart>& parts,
                         const std::vector<EncoderSpan>& spans, int max_tokens, int32_t bos, int32_t eos,
                         const std::function<void(const std::string&, std::vector<int32_t>&)>& encode,
                         std::vector<int32_t>& ids, bool& truncated);

}  // namespace ge
