// api.cpp -- the C ABI (include/gemma_embed.h): argument checks, the multi-GPU dispatcher and
// the host-side pieces of EmbeddingModel (Sources/GemmaEmbed/EmbeddingModel.swift):
// truncation, batch planning, packing and finish.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <memory>
#include <mutex>
#include <numeric>
#include <thread>

#include "audio_convert.hpp"
#include "gemma_embed.h"
#include "model.hpp"
#include "multimodal.hpp"
#include "wav.hpp"

namespace ge {
int load_model(ge_model* m, const char* path, const ge_load_opts* opts);
void free_model(ge_model* m);
}  // namespace ge

namespace ge {

// Sequences per device: longest first onto the least-loaded device, with a cost that counts
// attention's quadratic term, keeping each device's sequences in their original order.
std::vector<std::vector<int>> shard_sequences(const ge_seq* seqs, int nseq, int ndev) {
    std::vector<int> order(nseq);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return seqs[a].length > seqs[b].length; });
    std::vector<double> load(ndev, 0.0);
    std::vector<std::vector<int>> parts(ndev);
    for (int i : order) {
        const int dv = int(std::min_element(load.begin(), load.end()) - load.begin());
        const double n = seqs[i].length;
        load[dv] += n + n * n / 2048.0;
        parts[dv].push_back(i);
    }
    for (auto& p : parts) std::sort(p.begin(), p.end());
    return parts;
}

}  // namespace ge

namespace {

thread_local std::string t_last_error;

// Checks that `seqs` tile [0, ntok) in order with lengths 1..max_tokens, that every id is a
// token of the vocabulary (negative ids are the reference's vector rows, which only the image
// and audio towers produce) and that positions index the RoPE table.
int check_batch(ge_model* m, const int32_t* tokens, const int32_t* positions, int32_t ntok, const ge_seq* seqs,
                int32_t nseq) {
    const ge::Config& c = m->cfg;
    if (ntok < 0 || nseq < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: negative size");
    if ((ntok > 0 && !tokens) || (nseq > 0 && !seqs))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: NULL input array");
    uint64_t next = 0;
    for (int32_t s = 0; s < nseq; s++) {
        if (seqs[s].start != next)
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: sequence " + std::to_string(s) +
                                                                 " does not start where the previous one ends");
        if (seqs[s].length == 0 || seqs[s].length > uint32_t(c.max_tokens))
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS,
                                 "invalid options: sequence " + std::to_string(s) + " has " +
                                     std::to_string(seqs[s].length) + " tokens; allowed 1.." + std::to_string(c.max_tokens));
        next += seqs[s].length;
    }
    if (next != uint64_t(ntok))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: sequence lengths sum to " +
                                                            std::to_string(next) + ", not " + std::to_string(ntok));
    for (int32_t t = 0; t < ntok; t++) {
        if (tokens[t] < 0)
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS,
                                 "invalid options: vector rows (negative ids) need an image or audio encoder");
        if (tokens[t] >= c.vocab)
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: token id " + std::to_string(tokens[t]) +
                                                                " is outside the vocabulary of " + std::to_string(c.vocab));
        if (positions && (positions[t] < 0 || positions[t] >= c.max_tokens))
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: position " +
                                                                std::to_string(positions[t]) + " is out of range");
    }
    return GE_OK;
}

// Runs fn(dv) for each device share dv on the model's device workers (on the calling thread
// when the model has one device).
void run_per_device(ge_model* m, int n, const std::function<void(int)>& fn) {
    if (n <= 1 || !m->workers) {
        for (int i = 0; i < n; i++) fn(i);
        return;
    }
    m->workers->run(n, fn);
}

// The packed forward over every device of the model.  With fin_dims > 0 each device also runs
// EmbeddingModel.finish (the first fin_dims values, L2-normalised when fin_norm) and `out`
// receives [nseq][fin_dims] finished rows; otherwise [nseq][out_dim] pooled rows.
int forward_packed_locked(ge_model* m, const int32_t* tokens, const int32_t* positions, int32_t ntok, const ge_seq* seqs,
                          int32_t nseq, float* out, int fin_dims = 0, bool fin_norm = false) {
    const int ndev = int(m->devs.size());
    const int od = fin_dims > 0 ? fin_dims : m->cfg.out_dim;  // width of an output row
    if (ndev == 1 || nseq <= 1) {
        ge::ForwardArgs a;
        a.tokens = tokens;
        a.positions = positions;
        a.ntok = ntok;
        a.seqs = seqs;
        a.nseq = nseq;
        a.out = out;
        a.finish_dims = fin_dims;
        a.finish_normalise = fin_norm;
        return ge::run_forward(m, m->devs[0], a);
    }
    // Multi-GPU: each device packs its own share of the sequences, runs it on its own host
    // thread and stream, and its pooled rows go back to their original positions.
    auto parts = ge::shard_sequences(seqs, nseq, ndev);
    std::vector<int> rc(ndev, GE_OK);
    std::vector<std::string> msgs(ndev);
    run_per_device(m, ndev, [&](int dv) {
            const auto& idx = parts[size_t(dv)];
            if (idx.empty()) return;
            std::vector<int32_t> tk, ps;
            std::vector<ge_seq> sq;
            for (int i : idx) {
                sq.push_back({uint32_t(tk.size()), seqs[i].length});
                tk.insert(tk.end(), tokens + seqs[i].start, tokens + seqs[i].start + seqs[i].length);
                if (positions) ps.insert(ps.end(), positions + seqs[i].start, positions + seqs[i].start + seqs[i].length);
            }
            std::vector<float> o(idx.size() * size_t(od));
            ge::ForwardArgs a;
            a.tokens = tk.data();
            a.positions = positions ? ps.data() : nullptr;
            a.ntok = int(tk.size());
            a.seqs = sq.data();
            a.nseq = int(sq.size());
            a.out = o.data();
            a.finish_dims = fin_dims;
            a.finish_normalise = fin_norm;
            a.error = &msgs[dv];  // each device thread reports into its own string
            rc[dv] = ge::run_forward(m, m->devs[dv], a);
            if (rc[dv] == GE_OK)
                for (size_t j = 0; j < idx.size(); j++) memcpy(out + size_t(idx[j]) * od, o.data() + j * od, od * 4);
        });
    for (int dv = 0; dv < ndev; dv++)
        if (rc[dv] != GE_OK) return ge::set_error(m, rc[dv], msgs[dv]);
    return GE_OK;
}

// Option checks of EmbeddingModel.embed (EmbeddingModel.swift:147-153); fills `o` with the
// defaults overridden by `opts`.
int check_embed_opts(ge_model* m, const ge_embed_opts* opts, int32_t count, ge_embed_opts& o) {
    ge_embed_opts_default(&o);
    if (opts) o = *opts;
    const ge::Config& c = m->cfg;
    if (!(o.dimensions == 768 || o.dimensions == 512 || o.dimensions == 256 || o.dimensions == 128) ||
        o.dimensions > c.out_dim)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: dimensions must be one of [768, 512, 256, 128]");
    if (o.max_tokens < 2 || o.max_tokens > c.max_tokens)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS,
                             "invalid options: maxTokens must be between 2 and " + std::to_string(c.max_tokens));
    if (o.batch_size < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: batchSize must be at least 1");
    if (count < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: negative text count");
    return GE_OK;
}

// prepare's truncation (EmbeddingModel.swift:189-196): past max_tokens keep the first
// max_tokens - 1 ids and end with EOS.
void truncate_keeping_eos(ge_model* m, const ge_embed_opts& o, std::vector<int32_t>& ids, int32_t* token_counts,
                          int32_t* truncated, int32_t i) {
    const bool cut = int64_t(ids.size()) > o.max_tokens;
    if (cut) {
        ids.resize(size_t(o.max_tokens - 1));
        ids.push_back(m->cfg.eos_id);
    }
    if (token_counts) token_counts[i] = int32_t(ids.size());
    if (truncated) truncated[i] = cut ? 1 : 0;
}

// The batch loop of EmbeddingModel.embed (EmbeddingModel.swift:155-174): batches planned over
// the prepared lengths, one packed forward each, then finish into the caller's rows.
int embed_prepared(ge_model* m, const std::vector<std::vector<int32_t>>& prepared, const ge_embed_opts& o, float* out,
                   ge_progress_fn progress, void* user) {
    const int32_t count = int32_t(prepared.size());
    std::vector<int64_t> costs(static_cast<size_t>(count));
    for (int32_t i = 0; i < count; i++) costs[size_t(i)] = int64_t(prepared[size_t(i)].size());
    const int64_t budget = m->budget;
    std::vector<int32_t> ranges(2 * size_t(count));
    int32_t nr = 0;
    ge_batches(costs.data(), count, 1, o.batch_size, &budget, ranges.data(), &nr);
    int32_t done_texts = 0;
    int64_t done_tokens = 0;
    std::vector<int32_t> toks;
    std::vector<ge_seq> seqs;
    for (int32_t r = 0; r < nr; r++) {
        const int32_t b = ranges[2 * size_t(r)], e = ranges[2 * size_t(r) + 1];
        toks.clear();
        seqs.clear();
        for (int32_t i = b; i < e; i++) {
            seqs.push_back({uint32_t(toks.size()), uint32_t(prepared[size_t(i)].size())});
            toks.insert(toks.end(), prepared[size_t(i)].begin(), prepared[size_t(i)].end());
        }
        // finish (EmbeddingModel.swift:260-267) runs on the device, after the head: only the
        // rows' first o.dimensions values come back, finished, straight into the caller's rows.
        int rc;
        {
            std::lock_guard<std::mutex> g(m->mu);
            rc = check_batch(m, toks.data(), nullptr, int32_t(toks.size()), seqs.data(), int32_t(seqs.size()));
            if (rc == GE_OK)
                rc = forward_packed_locked(m, toks.data(), nullptr, int32_t(toks.size()), seqs.data(),
                                           int32_t(seqs.size()), out + size_t(b) * size_t(o.dimensions), o.dimensions,
                                           o.normalise != 0);
        }
        if (rc) return rc;
        done_texts += e - b;
        done_tokens += int64_t(toks.size());
        if (progress && progress(done_texts, count, done_tokens, user) != 0 && r + 1 < nr)
            return ge::set_error(m, GE_ERR_CANCELLED, "embedding was cancelled");
    }
    return GE_OK;
}

// The image forward of MetalForward.run(images:) (Metal/MetalForward.swift:211-219) on one
// device: the vision tower over the images, then the text tower over each image's
// [bos, <|image>, rows..., <image|>, eos] with the rows read from the tower's output.
// `pooled` receives n rows of the output width.
int images_on_device(ge_model* m, ge::Device& d, const ge::PreparedImage* const* ims, int n, float* pooled,
                     std::string* error, cudaStream_t stream = nullptr, const uint8_t* d_rgb = nullptr,
                     bool out_on_device = false) {
    ge::VisionArgs va;
    va.imgs = ims;
    va.n = n;
    va.d_rgb = d_rgb;
    va.stream = stream;
    va.error = error;
    int rc = ge::run_vision(m, d, va);
    if (rc) return rc;
    std::vector<int32_t> toks;
    std::vector<ge_seq> seqs;
    int32_t row = 0;
    for (int i = 0; i < n; i++) {
        seqs.push_back({uint32_t(toks.size()), uint32_t(ims[i]->tokens() + 4)});
        toks.push_back(m->cfg.bos_id);
        toks.push_back(m->image_begin);
        for (int t = 0; t < ims[i]->tokens(); t++) toks.push_back(-(row + t) - 1);
        toks.push_back(m->image_end);
        toks.push_back(m->cfg.eos_id);
        row += ims[i]->tokens();
    }
    ge::ForwardArgs a;
    a.tokens = toks.data();
    a.ntok = int(toks.size());
    a.seqs = seqs.data();
    a.nseq = int(seqs.size());
    a.out = pooled;
    a.out_on_device = out_on_device;
    a.stream = stream;
    a.error = error;
    a.vectors = d.vis.ws.vectors;
    a.vector_rows = row;
    return ge::run_forward(m, d, a);
}

// Prepares images on host threads (ImageEmbedding.prepare, ImageEmbedding.swift:75-103).
int prepare_images(ge_model* m, const ge_image* images, int32_t count, int max_image_tokens,
                   std::vector<ge::PreparedImage>& out) {
    for (int32_t i = 0; i < count; i++)
        if (!images[i].rgb || images[i].width <= 0 || images[i].height <= 0)
            return ge::set_error(m, GE_ERR_IMAGE_DECODING, "cannot decode image: image " + std::to_string(i) + " has no pixels");
    out.assign(size_t(count), ge::PreparedImage());
    std::atomic<int32_t> next{0};
    auto work = [&]() {
        for (int32_t i = next++; i < count; i = next++)
            ge::prepare_image(m->vcfg, images[i].rgb, images[i].width, images[i].height, max_image_tokens, out[size_t(i)]);
    };
    const int nt = int(std::min<int64_t>({int64_t(std::max(1u, std::thread::hardware_concurrency())), int64_t(count), 32}));
    std::vector<std::thread> th;
    for (int t = 1; t < nt; t++) th.emplace_back(work);
    work();
    for (auto& t : th) t.join();
    for (int32_t i = 0; i < count; i++) {
        const int rows = out[size_t(i)].tokens() + 4;
        if (rows > m->cfg.max_tokens)
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: image " + std::to_string(i) + " needs " +
                                                                std::to_string(rows) + " rows, the text model takes " +
                                                                std::to_string(m->cfg.max_tokens));
    }
    return GE_OK;
}

// The audio forward of MetalForward.run(audio:) on one device: the audio tower over the clips,
// then the text tower over each clip's [bos, <|audio>, rows..., <audio|>, eos] with the rows read
// from the tower's output.  `pooled` receives n rows of the output width.
int audios_on_device(ge_model* m, ge::Device& d, const ge::PreparedAudio* const* clips, int n, float* pooled,
                     std::string* error, cudaStream_t stream = nullptr, const float* d_pcm = nullptr,
                     bool out_on_device = false) {
    ge::AudioArgs aa;
    aa.clips = clips;
    aa.n = n;
    aa.d_pcm = d_pcm;
    aa.stream = stream;
    aa.error = error;
    int rc = ge::run_audio(m, d, aa);
    if (rc) return rc;
    std::vector<int32_t> toks;
    std::vector<ge_seq> seqs;
    int32_t row = 0;
    for (int i = 0; i < n; i++) {
        const int rows = clips[i]->tokens();
        seqs.push_back({uint32_t(toks.size()), uint32_t(rows + 4)});
        toks.push_back(m->cfg.bos_id);
        toks.push_back(m->audio_begin);
        for (int t = 0; t < rows; t++) toks.push_back(-(row + t) - 1);
        toks.push_back(m->audio_end);
        toks.push_back(m->cfg.eos_id);
        row += rows;
    }
    ge::ForwardArgs a;
    a.tokens = toks.data();
    a.ntok = int(toks.size());
    a.seqs = seqs.data();
    a.nseq = int(seqs.size());
    a.out = pooled;
    a.out_on_device = out_on_device;
    a.stream = stream;
    a.error = error;
    a.vectors = d.aud.ws.vectors;
    a.vector_rows = row;
    return ge::run_forward(m, d, a);
}

// AudioDecoder.decode's checks on its inputs (Audio/AudioDecoder.swift:28-38, 48-51): WAV bytes
// must be a RIFF/WAVE file (the library decodes no other container); samples need a positive
// channel count and rate and at least one sample.
std::string check_audio_input(const ge_audio& c) {
    if (c.wav) {
        if (!ge::is_wav(c.wav, c.wav_bytes))
            return "the bytes are not a WAV file; other containers (MP3, M4A, AIFF, CAF, FLAC) must be decoded to "
                   "samples by the caller";
        return std::string();
    }
    if (c.channels <= 0) return "channel count must be positive";
    if (c.sample_rate <= 0) return "sample rate must be positive";
    if (c.count < 0 || (c.count > 0 && !c.samples)) return "the samples are missing";
    if (c.count == 0) return "audio has no samples";
    return std::string();
}

// The 16 kHz mono samples of one clip (AudioDecoder.decode, Audio/AudioDecoder.swift:17-41): WAV
// bytes are decoded first; 16 kHz mono samples are used in place, anything else is converted
// (MiniaudioConverter).  An empty string, or the reason the clip cannot be decoded.
std::string decode_clip(const ge_audio& c, ge::PreparedAudio& p) {
    const float* samples = c.samples;
    int64_t frames = c.count;
    int channels = c.channels, rate = c.sample_rate;
    ge::DecodedWav w;
    if (c.wav) {
        std::string why;
        if (!ge::decode_wav(c.wav, c.wav_bytes, w, why)) return why;
        channels = w.channels;
        rate = w.sample_rate;
        frames = int64_t(w.samples.size()) / channels;
        samples = w.samples.data();
        if (frames == 0) return "audio has no samples";
    }
    if (rate == 16000 && channels == 1) {
        if (c.wav) {
            p.converted = std::move(w.samples);
            samples = p.converted.data();
        }
        p.samples = samples;
        p.count = frames;
    } else {
        ge::audio_to_mono_16k(samples, frames, channels, rate, p.converted);
        p.samples = p.converted.data();
        p.count = int64_t(p.converted.size());
    }
    return std::string();
}

// AudioEmbedding.prepare (AudioEmbedding.swift:78-101): every clip decoded (WAV bytes) and
// converted to 16 kHz mono (MiniaudioConverter) on host threads; then at least one frame, and at
// most max_rows rows with the 4 frame rows.  The first failing clip, in order, names the error.
int prepare_audios(ge_model* m, const ge_audio* clips, int32_t count, int max_rows, std::vector<ge::PreparedAudio>& out) {
    out.assign(size_t(count), ge::PreparedAudio());
    for (int32_t i = 0; i < count; i++) {
        const std::string why = check_audio_input(clips[i]);
        if (!why.empty())
            return ge::set_error(m, GE_ERR_AUDIO_DECODING, "cannot decode audio: audio " + std::to_string(i) + ": " + why);
    }
    {
        std::vector<std::string> errors(static_cast<size_t>(count));
        std::atomic<int32_t> next{0};
        auto work = [&]() {
            for (int32_t i = next++; i < count; i = next++) errors[size_t(i)] = decode_clip(clips[i], out[size_t(i)]);
        };
        const int nt = int(std::min<int64_t>({int64_t(std::max(1u, std::thread::hardware_concurrency())), int64_t(count), 16}));
        std::vector<std::thread> th;
        for (int t = 1; t < nt; t++) th.emplace_back(work);
        work();
        for (auto& t : th) t.join();
        for (int32_t i = 0; i < count; i++)
            if (!errors[size_t(i)].empty())
                return ge::set_error(m, GE_ERR_AUDIO_DECODING,
                                     "cannot decode audio: audio " + std::to_string(i) + ": " + errors[size_t(i)]);
    }
    for (int32_t i = 0; i < count; i++) {
        const ge::PreparedAudio& c = out[size_t(i)];
        const std::string name = "audio " + std::to_string(i);
        if (c.count < ge::kAudioMinimumSamples)
            return ge::set_error(m, GE_ERR_AUDIO_DECODING, "cannot decode audio: " + name + ": the clip has " +
                                                               std::to_string(c.count) +
                                                               " samples at 16 kHz; at least 2 are needed for one frame");
        // A final 30-second chunk of one sample has no frame; the reference stops on a
        // precondition there (AudioPreprocessor.swift:144), so such a clip is refused.
        if (c.count % ge::kAudioChunkSamples == 1)
            return ge::set_error(m, GE_ERR_AUDIO_DECODING, "cannot decode audio: " + name + ": its last 30-second chunk "
                                                               "has 1 sample; at least 2 are needed for one frame");
        const int64_t rows = ge::audio_token_count(c.count) + 4;
        if (rows > max_rows) {
            char buf[256];
            snprintf(buf, sizeof buf, "invalid options: %s is %.1f s and needs %lld rows; maxTokens allows %d (about %.1f s)",
                     name.c_str(), double(c.count) / 16000.0, (long long)rows, max_rows, double(max_rows - 4) * 0.04);
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, buf);
        }
    }
    return GE_OK;
}

// Writes the first min(size, cap) bytes of `s` and its full size (the buffer convention of the
// tokenizer entry points).
int copy_out(const std::string& s, char* text, int64_t cap, int64_t* len) {
    *len = int64_t(s.size());
    if (cap > 0) memcpy(text, s.data(), size_t(std::min<int64_t>(cap, *len)));
    return GE_OK;
}

}  // namespace

extern "C" {

void ge_load_opts_default(ge_load_opts* o) {
    if (!o) return;
    o->device_mask = 1;
    o->batch_token_budget = 8192;
    o->flags = 0;
    o->image_encoder_path = nullptr;
    o->image_patch_budget = 4096;
    o->audio_encoder_path = nullptr;
    o->audio_frame_budget = 96000;
}

void ge_embed_opts_default(ge_embed_opts* o) {
    if (!o) return;
    o->max_tokens = 2048;
    o->dimensions = 768;
    o->normalise = 1;
    o->batch_size = 0;
}

int ge_load(const char* path, const ge_load_opts* opts, ge_model** out) {
    if (!out) {
        t_last_error = "invalid options: output handle is NULL";
        return GE_ERR_INVALID_OPTIONS;
    }
    *out = nullptr;
    ge_model* m = new ge_model();
    ge_load_opts o;
    ge_load_opts_default(&o);
    if (opts) o = *opts;
    m->budget = std::max(64, o.batch_token_budget);
    m->flags = o.flags;
    m->patch_budget = o.image_patch_budget > 0 ? o.image_patch_budget : 4096;
    m->frame_budget = o.audio_frame_budget > 0 ? o.audio_frame_budget : 96000;
    int rc = ge::load_model(m, path, &o);
    if (rc == GE_OK && o.image_encoder_path) rc = ge::load_vision(m, o.image_encoder_path);
    if (rc == GE_OK && o.audio_encoder_path) rc = ge::load_audio(m, o.audio_encoder_path);
    if (rc == GE_OK) {
        // One forward over a short sequence initialises every kernel before the first request
        // (EmbeddingModel.swift:111-114).
        std::vector<int32_t> warm;
        if (m->tokenizer) {
            static const char kWarm[] = "warm up";
            m->tokenizer->t.encode(reinterpret_cast<const uint8_t*>(kWarm), sizeof kWarm - 1, true, false, warm);
        }
        if (warm.empty()) warm = {m->cfg.bos_id, 3, 4, m->cfg.eos_id};
        bool ids_ok = int(warm.size()) <= m->cfg.max_tokens;
        for (int32_t t : warm) ids_ok = ids_ok && t >= 0 && t < m->cfg.vocab;
        if (ids_ok) {
            ge_seq s{0, uint32_t(warm.size())};
            std::vector<float> v(size_t(m->cfg.out_dim));
            for (auto& d : m->devs) {
                ge::ForwardArgs a;
                a.tokens = warm.data();
                a.ntok = int32_t(warm.size());
                a.seqs = &s;
                a.nseq = 1;
                a.out = v.data();
                rc = ge::run_forward(m, d, a);
                if (rc) break;
            }
        }
    }
    if (rc != GE_OK) {
        t_last_error = m->last_error;
        ge::free_model(m);
        delete m;
        return rc;
    }
    *out = m;
    return GE_OK;
}

void ge_free(ge_model* m) {
    if (!m) return;
    {
        std::lock_guard<std::mutex> g(m->mu);
        ge::free_model(m);
    }
    delete m;
}

const char* ge_last_error(const ge_model* m) { return m ? m->last_error.c_str() : t_last_error.c_str(); }

int ge_info_get(const ge_model* m, ge_info* info) {
    if (!m || !info) return GE_ERR_INVALID_OPTIONS;
    const ge::Config& c = m->cfg;
    memset(info, 0, sizeof *info);
    snprintf(info->architecture, sizeof info->architecture, "%s", c.arch.c_str());
    snprintf(info->name, sizeof info->name, "%s", c.name.c_str());
    info->layer_count = c.layers;
    info->hidden_size = c.hidden;
    info->output_dimensions = c.out_dim;
    info->feed_forward_size = c.ff;
    info->per_layer_input_size = c.per_layer;
    info->head_count = c.heads;
    info->vocabulary_size = c.vocab;
    info->sliding_window = c.sliding_window;
    info->max_tokens = c.max_tokens;
    info->norm_epsilon = c.eps;
    snprintf(info->quantization, sizeof info->quantization, "%s", c.quant.c_str());
    info->file_size = m->file_size;
    info->device_count = int32_t(m->devs.size());
    info->eos_id = c.eos_id;
    info->bos_id = c.bos_id;
    if (!m->devs.empty()) snprintf(info->device_name, sizeof info->device_name, "%s", m->devs[0].name.c_str());
    info->kernel_launches = m->launches.load();
    info->host_to_device_bytes = m->h2d_bytes.load();
    info->device_to_host_bytes = m->d2h_bytes.load();
    info->graph_captures = m->graph_captures.load();
    if (m->has_vision) {
        info->image_layer_count = m->vcfg.layers;
        info->image_hidden_size = m->vcfg.hidden;
        info->image_patch_size = m->vcfg.patch;
        info->image_projection_dim = m->vcfg.projection_dim;
    }
    if (m->has_audio) {
        info->audio_layer_count = m->acfg.layers;
        info->audio_hidden_size = m->acfg.hidden;
        info->audio_head_count = m->acfg.heads;
        info->audio_feed_forward_size = m->acfg.ff;
        info->audio_mel_bins = m->acfg.mel_bins;
        info->audio_projection_dim = m->acfg.projection_dim;
    }
    return GE_OK;
}

int ge_profile(ge_model* m, const int32_t* tokens, int32_t ntok, const ge_seq* seqs, int32_t nseq, int32_t reps,
               ge_kernel_time* out, int32_t cap, int32_t* count) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    std::lock_guard<std::mutex> g(m->mu);
    if (reps < 1 || cap < 0 || (cap > 0 && !out) || !count)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: reps must be at least 1");
    int rc = check_batch(m, tokens, nullptr, ntok, seqs, nseq);
    if (rc) return rc;
    if (nseq == 0) {
        *count = 0;
        return GE_OK;
    }
    ge::ProfileSink sink;
    sink.reps = reps;
    std::vector<float> pooled(size_t(nseq) * m->cfg.out_dim);
    ge::ForwardArgs a;
    a.tokens = tokens;
    a.ntok = ntok;
    a.seqs = seqs;
    a.nseq = nseq;
    a.out = pooled.data();
    a.profile = &sink;
    rc = ge::run_forward(m, m->devs[0], a);
    if (rc) return rc;
    int32_t n = 0;
    for (auto& e : sink.entries) {
        if (n < cap) {
            ge_kernel_time& k = out[n];
            memset(&k, 0, sizeof k);
            snprintf(k.name, sizeof k.name, "%s", e.name.c_str());
            k.ms_per_launch = e.ms;
            k.flops_per_launch = e.flops;
            k.bytes_per_launch = e.bytes;
            k.launches_per_forward = e.occurrences;
        }
        n++;
    }
    *count = n < cap ? n : cap;
    return GE_OK;
}

int ge_forward_packed(ge_model* m, const int32_t* tokens, const int32_t* positions, int32_t ntok, const ge_seq* seqs,
                      int32_t nseq, float* pooled_out) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    std::lock_guard<std::mutex> g(m->mu);
    int rc = check_batch(m, tokens, positions, ntok, seqs, nseq);
    if (rc) return rc;
    if (nseq == 0) return GE_OK;
    if (!pooled_out) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: output array is NULL");
    return forward_packed_locked(m, tokens, positions, ntok, seqs, nseq, pooled_out);
}

int ge_forward_device(ge_model* m, int32_t device_ordinal, const int32_t* d_tokens, int32_t ntok, const ge_seq* seqs,
                      int32_t nseq, float* d_pooled, void* stream) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    std::lock_guard<std::mutex> g(m->mu);
    ge::Device* dev = nullptr;
    for (auto& d : m->devs)
        if (d.ordinal == device_ordinal) dev = &d;
    if (!dev) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: the model is not loaded on that device");
    if (ntok < 0 || nseq < 0 || (nseq > 0 && (!seqs || !d_tokens || !d_pooled)))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: bad sizes or NULL arrays");
    uint64_t next = 0;
    for (int32_t s = 0; s < nseq; s++) {
        if (seqs[s].start != next || seqs[s].length == 0 || seqs[s].length > uint32_t(m->cfg.max_tokens))
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: sequences must tile the batch in order");
        next += seqs[s].length;
    }
    if (next != uint64_t(ntok)) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: lengths do not sum to ntok");
    if (nseq == 0) return GE_OK;
    ge::ForwardArgs a;
    a.tokens = d_tokens;
    a.tokens_on_device = true;
    a.ntok = ntok;
    a.seqs = seqs;
    a.nseq = nseq;
    a.out = d_pooled;
    a.out_on_device = true;
    // NULL is the caller's legacy default stream, never the library's internal stream.
    a.stream = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
    return ge::run_forward(m, *dev, a);
}

int ge_forward_trace(ge_model* m, const int32_t* tokens, int32_t ntok, int32_t layer, float* hidden_out) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    std::lock_guard<std::mutex> g(m->mu);
    if (layer < -1 || layer >= m->cfg.layers || !hidden_out)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: layer out of range or NULL output");
    ge_seq s{0, uint32_t(ntok)};
    int rc = check_batch(m, tokens, nullptr, ntok, &s, 1);
    if (rc) return rc;
    ge::ForwardArgs a;
    a.tokens = tokens;
    a.ntok = ntok;
    a.seqs = &s;
    a.nseq = 1;
    a.trace_layer = layer;
    a.trace_out = hidden_out;
    return ge::run_forward(m, m->devs[0], a);
}

int ge_batches(const int64_t* costs, int32_t n, int32_t ncost, int32_t batch_size, const int64_t* budgets,
               int32_t* ranges_out, int32_t* count_out) {
    if (n < 0 || ncost < 1 || (n > 0 && (!costs || !ranges_out)) || !budgets || !count_out) return GE_ERR_INVALID_OPTIONS;
    // EmbeddingModel.batches (EmbeddingModel.swift:200-215).
    std::vector<int64_t> totals(size_t(ncost), 0);
    int32_t count = 0, start = 0;
    for (int32_t i = 0; i < n; i++) {
        bool full = false;
        if (batch_size > 0) {
            full = i - start >= batch_size;
        } else {
            for (int32_t c = 0; c < ncost; c++) full = full || totals[c] + costs[int64_t(i) * ncost + c] > budgets[c];
        }
        if (i > start && full) {
            ranges_out[2 * count] = start;
            ranges_out[2 * count + 1] = i;
            count++;
            start = i;
            std::fill(totals.begin(), totals.end(), 0);
        }
        for (int32_t c = 0; c < ncost; c++) totals[c] += costs[int64_t(i) * ncost + c];
    }
    if (start < n) {
        ranges_out[2 * count] = start;
        ranges_out[2 * count + 1] = n;
        count++;
    }
    *count_out = count;
    return GE_OK;
}

int ge_finish(const float* v, int32_t n, int32_t dims, int32_t normalise, float* out) {
    if (!v || !out || n < 0 || dims < 0) return GE_ERR_INVALID_OPTIONS;
    // EmbeddingModel.finish (EmbeddingModel.swift:260-267).
    const int32_t k = std::min(dims, n);
    for (int32_t i = 0; i < k; i++) out[i] = v[i];
    if (normalise) {
        float s = 0.f;
        for (int32_t i = 0; i < k; i++) s += out[i] * out[i];
        const float norm = sqrtf(s);
        if (norm > 0.f)
            for (int32_t i = 0; i < k; i++) out[i] /= norm;
    }
    return GE_OK;
}

int ge_embed_tokens(ge_model* m, const int32_t* const* texts, const int32_t* lengths, int32_t count,
                    const ge_embed_opts* opts, float* out, int32_t* token_counts, int32_t* truncated,
                    ge_progress_fn progress, void* user) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    ge_embed_opts o;
    int rc = check_embed_opts(m, opts, count, o);
    if (rc || count == 0) return rc;
    if (!texts || !lengths || !out) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: NULL array");
    std::vector<std::vector<int32_t>> prepared(static_cast<size_t>(count));
    for (int32_t i = 0; i < count; i++) {
        if (lengths[i] <= 0 || !texts[i])
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: text " + std::to_string(i) + " has no tokens");
        prepared[size_t(i)].assign(texts[i], texts[i] + lengths[i]);
        truncate_keeping_eos(m, o, prepared[size_t(i)], token_counts, truncated, i);
    }
    return embed_prepared(m, prepared, o, out, progress, user);
}

int ge_embed_texts(ge_model* m, const char* const* texts, const int64_t* lengths, int32_t count, const char* prefix,
                   const ge_embed_opts* opts, float* out, int32_t* token_counts, int32_t* truncated,
                   ge_progress_fn progress, void* user) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    ge_embed_opts o;
    int rc = check_embed_opts(m, opts, count, o);
    if (rc || count == 0) return rc;
    if (!texts || !lengths || !out) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: NULL array");
    if (!m->tokenizer)
        return ge::set_error(m, GE_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture: tokenizer model missing");
    for (int32_t i = 0; i < count; i++)
        if (lengths[i] < 0 || (lengths[i] > 0 && !texts[i]))
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: text " + std::to_string(i) + " is NULL");
    const ge::Tokenizer& tk = m->tokenizer->t;
    const std::string pre = prefix ? std::string(prefix) : std::string();
    std::vector<std::vector<int32_t>> prepared(static_cast<size_t>(count));
    // prepare (EmbeddingModel.swift:189-196) for every text, spread over host threads in
    // chunks; each text's ids depend on that text alone.
    int64_t bytes = 0;
    for (int32_t i = 0; i < count; i++) bytes += lengths[i] + int64_t(pre.size());
    const int hw = int(std::max(1u, std::thread::hardware_concurrency()));
    const int nthreads = int(std::min<int64_t>({int64_t(hw), int64_t(count), std::max<int64_t>(1, bytes / 16384), 64}));
    std::atomic<int32_t> next{0};
    constexpr int32_t kChunk = 8;
    auto work = [&]() {
        std::string joined;
        for (;;) {
            const int32_t b = next.fetch_add(kChunk);
            if (b >= count) break;
            for (int32_t i = b; i < std::min(count, b + kChunk); i++) {
                joined.assign(pre);
                joined.append(texts[i] ? texts[i] : "", size_t(lengths[i]));
                tk.encode(reinterpret_cast<const uint8_t*>(joined.data()), joined.size(), true, false, prepared[size_t(i)]);
            }
        }
    };
    if (nthreads <= 1) {
        work();
    } else {
        std::vector<std::thread> th;
        for (int t = 1; t < nthreads; t++) th.emplace_back(work);
        work();
        for (auto& t : th) t.join();
    }
    for (int32_t i = 0; i < count; i++) {
        if (prepared[size_t(i)].empty())  // no BOS/EOS in the metadata and an empty text
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: text " + std::to_string(i) + " has no tokens");
        truncate_keeping_eos(m, o, prepared[size_t(i)], token_counts, truncated, i);
    }
    return embed_prepared(m, prepared, o, out, progress, user);
}

void ge_image_opts_default(ge_image_opts* o) {
    if (!o) return;
    o->dimensions = 768;
    o->normalise = 1;
    o->max_image_tokens = 256;
    o->batch_size = 0;
}

int ge_embed_images(ge_model* m, const ge_image* images, int32_t count, const ge_image_opts* opts, float* out,
                    int32_t* token_counts, ge_progress_fn progress, void* user) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    ge_image_opts o;
    ge_image_opts_default(&o);
    if (opts) o = *opts;
    // forEachImageBatch's checks (ImageEmbedding.swift:55-64).
    if (!m->has_vision)
        return ge::set_error(m, GE_ERR_IMAGE_ENCODER_NOT_LOADED,
                             "no image encoder is loaded; pass the mmproj GGUF when loading the model");
    if (!(o.dimensions == 768 || o.dimensions == 512 || o.dimensions == 256 || o.dimensions == 128) ||
        o.dimensions > m->cfg.out_dim)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: dimensions must be one of [768, 512, 256, 128]");
    if (o.max_image_tokens < 1 || o.max_image_tokens > m->vcfg.native_max_image_tokens)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: maxImageTokens must be between 1 and " +
                                                            std::to_string(m->vcfg.native_max_image_tokens));
    if (o.batch_size < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: batchSize must be at least 1");
    if (count < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: negative image count");
    if (count == 0) return GE_OK;
    if (!images || !out) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: NULL array");
    std::vector<ge::PreparedImage> prepared;
    int rc = prepare_images(m, images, count, o.max_image_tokens, prepared);
    if (rc) return rc;
    std::vector<int64_t> costs(static_cast<size_t>(count));
    for (int32_t i = 0; i < count; i++) costs[size_t(i)] = prepared[size_t(i)].patches();
    const int64_t budget = m->patch_budget;
    std::vector<int32_t> ranges(2 * size_t(count));
    int32_t nr = 0;
    ge_batches(costs.data(), count, 1, o.batch_size, &budget, ranges.data(), &nr);
    std::lock_guard<std::mutex> g(m->mu);
    const int od = m->cfg.out_dim, ndev = int(m->devs.size());
    int32_t done = 0;
    int64_t done_tokens = 0;
    for (int32_t r = 0; r < nr; r++) {
        const int32_t b = ranges[2 * size_t(r)], e = ranges[2 * size_t(r) + 1];
        const int n = e - b;
        std::vector<float> pooled(size_t(n) * od);
        // Images of a batch spread over the devices, largest first onto the least-loaded one.
        std::vector<std::vector<int>> parts(size_t(std::max(1, std::min(ndev, n))));
        {
            std::vector<int> order(static_cast<size_t>(n));
            std::iota(order.begin(), order.end(), 0);
            std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return costs[size_t(b + x)] > costs[size_t(b + y)]; });
            std::vector<int64_t> load(parts.size(), 0);
            for (int i : order) {
                const size_t dv = size_t(std::min_element(load.begin(), load.end()) - load.begin());
                load[dv] += costs[size_t(b + i)];
                parts[dv].push_back(i);
            }
            for (auto& p : parts) std::sort(p.begin(), p.end());
        }
        std::vector<int> rcs(parts.size(), GE_OK);
        std::vector<std::string> msgs(parts.size());
        auto run_part = [&](size_t dv) {
            const auto& idx = parts[dv];
            if (idx.empty()) return;
            std::vector<const ge::PreparedImage*> ims;
            for (int i : idx) ims.push_back(&prepared[size_t(b + i)]);
            std::vector<float> po(idx.size() * size_t(od));
            rcs[dv] = images_on_device(m, m->devs[dv], ims.data(), int(ims.size()), po.data(), &msgs[dv]);
            if (rcs[dv] == GE_OK)
                for (size_t k = 0; k < idx.size(); k++)
                    memcpy(pooled.data() + size_t(idx[k]) * od, po.data() + k * od, size_t(od) * sizeof(float));
        };
        if (parts.size() == 1)
            run_part(0);
        else
            run_per_device(m, int(parts.size()), [&](int dv) { run_part(size_t(dv)); });
        for (size_t dv = 0; dv < parts.size(); dv++)
            if (rcs[dv] != GE_OK) return ge::set_error(m, rcs[dv], msgs[dv]);
        for (int32_t i = b; i < e; i++) {
            ge_finish(pooled.data() + size_t(i - b) * od, od, o.dimensions, o.normalise, out + size_t(i) * o.dimensions);
            const int rows = prepared[size_t(i)].tokens() + 4;  // EmbeddingModel.imageFrameRows
            if (token_counts) token_counts[i] = rows;
            done_tokens += rows;
        }
        done += n;
        if (progress && progress(done, count, done_tokens, user) != 0 && r + 1 < nr)
            return ge::set_error(m, GE_ERR_CANCELLED, "embedding was cancelled");
    }
    return GE_OK;
}

int32_t ge_image_tokens(const ge_model* m, int32_t width, int32_t height, int32_t max_image_tokens) {
    if (!m || !m->has_vision || width <= 0 || height <= 0 || max_image_tokens <= 0) return -1;
    const ge::VisionConfig& c = m->vcfg;
    const int a = c.alignment();
    int tw = 0, th = 0;
    ge::image_target_size(width, height, a, c.min_image_tokens * a * a, max_image_tokens * a * a, tw, th);
    return (tw / a) * (th / a);
}

int ge_image_vectors(ge_model* m, const ge_image* images, int32_t count, int32_t max_image_tokens, float* out,
                     int64_t cap_rows, int32_t* rows_per_image) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    if (!m->has_vision)
        return ge::set_error(m, GE_ERR_IMAGE_ENCODER_NOT_LOADED,
                             "no image encoder is loaded; pass the mmproj GGUF when loading the model");
    if (max_image_tokens < 1 || max_image_tokens > m->vcfg.native_max_image_tokens)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: maxImageTokens must be between 1 and " +
                                                            std::to_string(m->vcfg.native_max_image_tokens));
    if (count < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: negative image count");
    if (count == 0) return GE_OK;
    if (!images || !out) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: NULL array");
    std::vector<ge::PreparedImage> prepared;
    int rc = prepare_images(m, images, count, max_image_tokens, prepared);
    if (rc) return rc;
    int64_t rows = 0;
    for (auto& p : prepared) rows += p.tokens();
    if (rows > cap_rows)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: the images need " + std::to_string(rows) +
                                                            " rows, the output holds " + std::to_string(cap_rows));
    std::lock_guard<std::mutex> g(m->mu);
    ge::Device& d = m->devs[0];
    std::vector<const ge::PreparedImage*> ims;
    for (auto& p : prepared) ims.push_back(&p);
    ge::VisionArgs va;
    va.imgs = ims.data();
    va.n = count;
    rc = ge::run_vision(m, d, va);
    if (rc) return rc;
    const size_t bytes = size_t(rows) * m->vcfg.projection_dim * sizeof(float);
    cudaError_t e = cudaMemcpyAsync(out, d.vis.ws.vectors, bytes, cudaMemcpyDeviceToHost, d.stream);
    int h_err = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h_err, d.err, sizeof(int), cudaMemcpyDeviceToHost, d.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d.stream);
    if (e != cudaSuccess)
        return ge::set_error(m, GE_ERR_GPU_FAILURE, std::string("GPU execution failed: ") + cudaGetErrorString(e));
    if (h_err) {
        cudaMemset(d.err, 0, sizeof(int));
        return ge::set_error(m, h_err, "GPU execution failed: a device-side wait gave up (code " + std::to_string(h_err) + ")");
    }
    m->d2h_bytes += int64_t(bytes);
    for (int32_t i = 0; i < count && rows_per_image; i++) rows_per_image[i] = prepared[size_t(i)].tokens();
    return GE_OK;
}

int ge_image_forward_device(ge_model* m, int32_t device_ordinal, const uint8_t* d_rgb, const ge_image* images,
                            int32_t count, float* d_pooled, void* stream) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    if (!m->has_vision)
        return ge::set_error(m, GE_ERR_IMAGE_ENCODER_NOT_LOADED,
                             "no image encoder is loaded; pass the mmproj GGUF when loading the model");
    std::lock_guard<std::mutex> g(m->mu);
    ge::Device* dev = nullptr;
    for (auto& d : m->devs)
        if (d.ordinal == device_ordinal) dev = &d;
    if (!dev) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: the model is not loaded on that device");
    if (count < 0 || (count > 0 && (!d_rgb || !images || !d_pooled)))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: bad sizes or NULL arrays");
    if (count == 0) return GE_OK;
    const ge::VisionConfig& c = m->vcfg;
    std::vector<ge::PreparedImage> ims(static_cast<size_t>(count));
    std::vector<const ge::PreparedImage*> ptrs;
    for (int32_t i = 0; i < count; i++) {
        const int a = c.alignment();
        if (images[i].width <= 0 || images[i].height <= 0 || images[i].width % a || images[i].height % a)
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: image " + std::to_string(i) +
                                                                " is not at a tower size (sides multiples of " +
                                                                std::to_string(a) + ")");
        ge::PreparedImage& p = ims[size_t(i)];
        p.width = images[i].width;
        p.height = images[i].height;
        p.gx = p.width / c.patch;
        p.gy = p.height / c.patch;
        p.merge = c.merge;
        if (p.tokens() + 4 > m->cfg.max_tokens)
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: image " + std::to_string(i) + " needs " +
                                                                std::to_string(p.tokens() + 4) + " rows");
        ptrs.push_back(&p);
    }
    return images_on_device(m, *dev, ptrs.data(), count, d_pooled, nullptr,
                            stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy, d_rgb, true);
}

int ge_profile_images(ge_model* m, const ge_image* images, int32_t count, int32_t max_image_tokens, int32_t reps,
                      ge_kernel_time* out, int32_t cap, int32_t* n_out) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    if (!m->has_vision)
        return ge::set_error(m, GE_ERR_IMAGE_ENCODER_NOT_LOADED,
                             "no image encoder is loaded; pass the mmproj GGUF when loading the model");
    if (count <= 0 || !images || reps < 1 || !n_out || (cap > 0 && !out))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: images, reps or outputs");
    if (max_image_tokens < 1 || max_image_tokens > m->vcfg.native_max_image_tokens)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: maxImageTokens out of range");
    std::vector<ge::PreparedImage> prepared;
    int rc = prepare_images(m, images, count, max_image_tokens, prepared);
    if (rc) return rc;
    std::lock_guard<std::mutex> g(m->mu);
    ge::Device& d = m->devs[0];
    std::vector<const ge::PreparedImage*> ims;
    for (auto& p : prepared) ims.push_back(&p);
    std::vector<float> pooled(size_t(count) * m->cfg.out_dim);
    // One ordinary run uploads the pixels; the timed runs read them where they landed.
    if ((rc = images_on_device(m, d, ims.data(), count, pooled.data(), nullptr))) return rc;
    const uint8_t* d_rgb = d.vis.ws.rgb;
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    // The whole image forward (vision and text towers) and the vision tower alone, mean of reps.
    float whole = 0.f, tower = 0.f;
    for (int r = 0; r < reps && rc == GE_OK; r++) {
        cudaEventRecord(e0, d.stream);
        ge::VisionArgs va;
        va.imgs = ims.data();
        va.n = count;
        va.d_rgb = d_rgb;
        rc = ge::run_vision(m, d, va);
        cudaEventRecord(e1, d.stream);
        if (rc == GE_OK) rc = images_on_device(m, d, ims.data(), count, pooled.data(), nullptr, nullptr, d_rgb);
        cudaEventRecord(e2, d.stream);
        cudaEventSynchronize(e2);
        float t1 = 0.f, t2 = 0.f, t3 = 0.f;
        cudaEventElapsedTime(&t1, e0, e1);
        cudaEventElapsedTime(&t2, e1, e2);
        tower += t1;
        whole += t2;
        (void)t3;
    }
    ge::ProfileSink sink;
    sink.reps = reps;
    if (rc == GE_OK) {
        ge::VisionArgs va;
        va.imgs = ims.data();
        va.n = count;
        va.d_rgb = d_rgb;
        va.profile = &sink;
        rc = ge::run_vision(m, d, va);
        cudaStreamSynchronize(d.stream);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    if (rc) return rc;
    double patches = 0, tokens = 0;
    for (auto* p : ims) {
        patches += p->patches();
        tokens += p->tokens();
    }
    std::vector<ge_kernel_time> all;
    auto add = [&](const std::string& name, double ms, double flops, double bytes, int per) {
        ge_kernel_time k;
        memset(&k, 0, sizeof k);
        snprintf(k.name, sizeof k.name, "%s", name.c_str());
        k.ms_per_launch = ms;
        k.flops_per_launch = flops;
        k.bytes_per_launch = bytes;
        k.launches_per_forward = per;
        all.push_back(k);
    };
    add("image_forward", double(whole) / reps, 0, 0, 1);
    add("vision_tower", double(tower) / reps, 0, 0, 1);
    for (auto& e : sink.entries) add(e.name, e.ms, e.flops, e.bytes, e.occurrences);
    *n_out = int32_t(all.size());
    for (int32_t i = 0; i < std::min<int32_t>(cap, int32_t(all.size())); i++) out[i] = all[size_t(i)];
    return GE_OK;
}

void ge_audio_opts_default(ge_audio_opts* o) {
    if (!o) return;
    o->dimensions = 768;
    o->normalise = 1;
    o->max_tokens = 0;
    o->batch_size = 0;
}

int ge_audio_convert(const ge_audio* clip, float* out, int64_t cap, int64_t* count) {
    if (!clip || !count || cap < 0 || (cap > 0 && !out)) {
        t_last_error = "invalid options: NULL clip, count or output";
        return GE_ERR_INVALID_OPTIONS;
    }
    const std::string why = check_audio_input(*clip);
    if (!why.empty()) {
        t_last_error = "cannot decode audio: " + why;
        return GE_ERR_AUDIO_DECODING;
    }
    ge::PreparedAudio p;
    const std::string reason = decode_clip(*clip, p);
    if (!reason.empty()) {
        t_last_error = "cannot decode audio: " + reason;
        return GE_ERR_AUDIO_DECODING;
    }
    *count = p.count;
    if (cap > 0 && p.count > 0) memcpy(out, p.samples, size_t(std::min(cap, p.count)) * sizeof(float));
    return GE_OK;
}

int ge_audio_decode_wav(const uint8_t* bytes, int64_t length, float* out, int64_t cap, int64_t* frames,
                        int32_t* sample_rate, int32_t* channels) {
    if (!bytes || length < 0 || !frames || !sample_rate || !channels || cap < 0 || (cap > 0 && !out)) {
        t_last_error = "invalid options: NULL bytes or outputs";
        return GE_ERR_INVALID_OPTIONS;
    }
    ge::DecodedWav w;
    std::string why;
    if (!ge::decode_wav(bytes, length, w, why)) {
        t_last_error = "cannot decode audio: " + why;
        return GE_ERR_AUDIO_DECODING;
    }
    const int64_t n = int64_t(w.samples.size());
    *frames = n / w.channels;
    *sample_rate = w.sample_rate;
    *channels = w.channels;
    if (cap > 0 && n > 0) memcpy(out, w.samples.data(), size_t(std::min(cap, n)) * sizeof(float));
    return GE_OK;
}

int64_t ge_audio_tokens(int64_t samples) {
    return samples < ge::kAudioMinimumSamples ? 0 : ge::audio_token_count(samples);
}

int ge_embed_audios(ge_model* m, const ge_audio* clips, int32_t count, const ge_audio_opts* opts, float* out,
                    int32_t* token_counts, ge_progress_fn progress, void* user) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    ge_audio_opts o;
    ge_audio_opts_default(&o);
    if (opts) o = *opts;
    // forEachAudioBatch's checks (AudioEmbedding.swift:59-69).
    if (!m->has_audio)
        return ge::set_error(m, GE_ERR_AUDIO_ENCODER_NOT_LOADED,
                             "no audio encoder is loaded; pass the mmproj GGUF when loading the model");
    if (!(o.dimensions == 768 || o.dimensions == 512 || o.dimensions == 256 || o.dimensions == 128) ||
        o.dimensions > m->cfg.out_dim)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: dimensions must be one of [768, 512, 256, 128]");
    const int max_rows = o.max_tokens ? o.max_tokens : m->cfg.max_tokens;
    if (max_rows <= 4 || max_rows > m->cfg.max_tokens)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS,
                             "invalid options: maxTokens must be between 5 and " + std::to_string(m->cfg.max_tokens));
    if (o.batch_size < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: batchSize must be at least 1");
    if (count < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: negative clip count");
    if (count == 0) return GE_OK;
    if (!clips || !out) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: NULL array");
    std::vector<ge::PreparedAudio> prepared;
    int rc = prepare_audios(m, clips, count, max_rows, prepared);
    if (rc) return rc;
    std::vector<int64_t> costs(static_cast<size_t>(count));
    for (int32_t i = 0; i < count; i++) costs[size_t(i)] = prepared[size_t(i)].frames();
    const int64_t budget = m->frame_budget;
    std::vector<int32_t> ranges(2 * size_t(count));
    int32_t nr = 0;
    ge_batches(costs.data(), count, 1, o.batch_size, &budget, ranges.data(), &nr);
    std::lock_guard<std::mutex> g(m->mu);
    const int od = m->cfg.out_dim, ndev = int(m->devs.size());
    int32_t done = 0;
    int64_t done_tokens = 0;
    for (int32_t r = 0; r < nr; r++) {
        const int32_t b = ranges[2 * size_t(r)], e = ranges[2 * size_t(r) + 1];
        const int n = e - b;
        std::vector<float> pooled(size_t(n) * od);
        // Clips of a batch spread over the devices, longest first onto the least-loaded one.
        std::vector<std::vector<int>> parts(size_t(std::max(1, std::min(ndev, n))));
        {
            std::vector<int> order(static_cast<size_t>(n));
            std::iota(order.begin(), order.end(), 0);
            std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return costs[size_t(b + x)] > costs[size_t(b + y)]; });
            std::vector<int64_t> load(parts.size(), 0);
            for (int i : order) {
                const size_t dv = size_t(std::min_element(load.begin(), load.end()) - load.begin());
                load[dv] += costs[size_t(b + i)];
                parts[dv].push_back(i);
            }
            for (auto& p : parts) std::sort(p.begin(), p.end());
        }
        std::vector<int> rcs(parts.size(), GE_OK);
        std::vector<std::string> msgs(parts.size());
        auto run_part = [&](size_t dv) {
            const auto& idx = parts[dv];
            if (idx.empty()) return;
            std::vector<const ge::PreparedAudio*> cl;
            for (int i : idx) cl.push_back(&prepared[size_t(b + i)]);
            std::vector<float> po(idx.size() * size_t(od));
            rcs[dv] = audios_on_device(m, m->devs[dv], cl.data(), int(cl.size()), po.data(), &msgs[dv]);
            if (rcs[dv] == GE_OK)
                for (size_t k = 0; k < idx.size(); k++)
                    memcpy(pooled.data() + size_t(idx[k]) * od, po.data() + k * od, size_t(od) * sizeof(float));
        };
        if (parts.size() == 1)
            run_part(0);
        else
            run_per_device(m, int(parts.size()), [&](int dv) { run_part(size_t(dv)); });
        for (size_t dv = 0; dv < parts.size(); dv++)
            if (rcs[dv] != GE_OK) return ge::set_error(m, rcs[dv], msgs[dv]);
        for (int32_t i = b; i < e; i++) {
            ge_finish(pooled.data() + size_t(i - b) * od, od, o.dimensions, o.normalise, out + size_t(i) * o.dimensions);
            const int rows = prepared[size_t(i)].tokens() + 4;  // EmbeddingModel.audioFrameRows
            if (token_counts) token_counts[i] = rows;
            done_tokens += rows;
        }
        done += n;
        if (progress && progress(done, count, done_tokens, user) != 0 && r + 1 < nr)
            return ge::set_error(m, GE_ERR_CANCELLED, "embedding was cancelled");
    }
    return GE_OK;
}

int ge_audio_vectors(ge_model* m, const ge_audio* clips, int32_t count, float* out, int64_t cap_rows,
                     int32_t* rows_per_clip) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    if (!m->has_audio)
        return ge::set_error(m, GE_ERR_AUDIO_ENCODER_NOT_LOADED,
                             "no audio encoder is loaded; pass the mmproj GGUF when loading the model");
    if (count < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: negative clip count");
    if (count == 0) return GE_OK;
    if (!clips || !out) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: NULL array");
    std::vector<ge::PreparedAudio> prepared;
    int rc = prepare_audios(m, clips, count, INT32_MAX, prepared);
    if (rc) return rc;
    int64_t rows = 0;
    for (auto& p : prepared) rows += p.tokens();
    if (rows > cap_rows)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: the clips need " + std::to_string(rows) +
                                                            " rows, the output holds " + std::to_string(cap_rows));
    std::lock_guard<std::mutex> g(m->mu);
    ge::Device& d = m->devs[0];
    std::vector<const ge::PreparedAudio*> cl;
    for (auto& p : prepared) cl.push_back(&p);
    ge::AudioArgs aa;
    aa.clips = cl.data();
    aa.n = count;
    rc = ge::run_audio(m, d, aa);
    if (rc) return rc;
    const size_t bytes = size_t(rows) * m->acfg.projection_dim * sizeof(float);
    cudaError_t e = cudaMemcpyAsync(out, d.aud.ws.vectors, bytes, cudaMemcpyDeviceToHost, d.stream);
    int h_err = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h_err, d.err, sizeof(int), cudaMemcpyDeviceToHost, d.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d.stream);
    if (e != cudaSuccess)
        return ge::set_error(m, GE_ERR_GPU_FAILURE, std::string("GPU execution failed: ") + cudaGetErrorString(e));
    if (h_err) {
        cudaMemset(d.err, 0, sizeof(int));
        return ge::set_error(m, h_err, "GPU execution failed: a device-side wait gave up (code " + std::to_string(h_err) + ")");
    }
    m->d2h_bytes += int64_t(bytes);
    for (int32_t i = 0; i < count && rows_per_clip; i++) rows_per_clip[i] = prepared[size_t(i)].tokens();
    return GE_OK;
}

int ge_audio_forward_device(ge_model* m, int32_t device_ordinal, const float* d_pcm, const ge_audio* clips,
                            int32_t count, float* d_pooled, void* stream) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    if (!m->has_audio)
        return ge::set_error(m, GE_ERR_AUDIO_ENCODER_NOT_LOADED,
                             "no audio encoder is loaded; pass the mmproj GGUF when loading the model");
    std::lock_guard<std::mutex> g(m->mu);
    ge::Device* dev = nullptr;
    for (auto& d : m->devs)
        if (d.ordinal == device_ordinal) dev = &d;
    if (!dev) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: the model is not loaded on that device");
    if (count < 0 || (count > 0 && (!d_pcm || !clips || !d_pooled)))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: bad sizes or NULL arrays");
    if (count == 0) return GE_OK;
    std::vector<ge::PreparedAudio> cl(static_cast<size_t>(count));
    std::vector<const ge::PreparedAudio*> ptrs;
    int64_t off = 0;
    for (int32_t i = 0; i < count; i++) {
        if (clips[i].wav || clips[i].sample_rate != 16000 || clips[i].channels != 1 || clips[i].count < ge::kAudioMinimumSamples ||
            clips[i].count % ge::kAudioChunkSamples == 1)
            return ge::set_error(m, GE_ERR_AUDIO_DECODING, "cannot decode audio: clip " + std::to_string(i) +
                                                               " is not 16 kHz mono samples with at least 2 in every "
                                                               "30-second chunk");
        cl[size_t(i)].count = clips[i].count;
        cl[size_t(i)].device_offset = off;
        off += clips[i].count;
        if (cl[size_t(i)].tokens() + 4 > m->cfg.max_tokens)
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: clip " + std::to_string(i) + " needs " +
                                                                std::to_string(cl[size_t(i)].tokens() + 4) + " rows");
        ptrs.push_back(&cl[size_t(i)]);
    }
    return audios_on_device(m, *dev, ptrs.data(), count, d_pooled, nullptr,
                            stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy, d_pcm, true);
}

int ge_profile_audios(ge_model* m, const ge_audio* clips, int32_t count, int32_t reps, ge_kernel_time* out, int32_t cap,
                      int32_t* n_out) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    if (!m->has_audio)
        return ge::set_error(m, GE_ERR_AUDIO_ENCODER_NOT_LOADED,
                             "no audio encoder is loaded; pass the mmproj GGUF when loading the model");
    if (count <= 0 || !clips || reps < 1 || !n_out || (cap > 0 && !out))
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: clips, reps or outputs");
    std::vector<ge::PreparedAudio> prepared;
    int rc = prepare_audios(m, clips, count, m->cfg.max_tokens, prepared);
    if (rc) return rc;
    std::lock_guard<std::mutex> g(m->mu);
    ge::Device& d = m->devs[0];
    std::vector<const ge::PreparedAudio*> cl;
    for (auto& p : prepared) cl.push_back(&p);
    std::vector<float> pooled(size_t(count) * m->cfg.out_dim);
    // One ordinary run uploads the samples; the timed runs read them where they landed.
    if ((rc = audios_on_device(m, d, cl.data(), count, pooled.data(), nullptr))) return rc;
    std::vector<ge::PreparedAudio> dev_clips(prepared);
    std::vector<const ge::PreparedAudio*> dcl;
    int64_t off = 0;
    for (auto& p : dev_clips) {
        p.device_offset = off;
        off += p.count;
        dcl.push_back(&p);
    }
    const float* d_pcm = d.aud.ws.pcm;
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    float whole = 0.f, tower = 0.f;
    for (int r = 0; r < reps && rc == GE_OK; r++) {
        cudaEventRecord(e0, d.stream);
        ge::AudioArgs aa;
        aa.clips = dcl.data();
        aa.n = count;
        aa.d_pcm = d_pcm;
        rc = ge::run_audio(m, d, aa);
        cudaEventRecord(e1, d.stream);
        if (rc == GE_OK) rc = audios_on_device(m, d, dcl.data(), count, pooled.data(), nullptr, nullptr, d_pcm);
        cudaEventRecord(e2, d.stream);
        cudaEventSynchronize(e2);
        float t1 = 0.f, t2 = 0.f;
        cudaEventElapsedTime(&t1, e0, e1);
        cudaEventElapsedTime(&t2, e1, e2);
        tower += t1;
        whole += t2;
    }
    ge::ProfileSink sink;
    sink.reps = reps;
    if (rc == GE_OK) {
        ge::AudioArgs aa;
        aa.clips = dcl.data();
        aa.n = count;
        aa.d_pcm = d_pcm;
        aa.profile = &sink;
        rc = ge::run_audio(m, d, aa);
        cudaStreamSynchronize(d.stream);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    if (rc) return rc;
    std::vector<ge_kernel_time> all;
    auto add = [&](const std::string& name, double ms, double flops, double bytes, int per) {
        ge_kernel_time k;
        memset(&k, 0, sizeof k);
        snprintf(k.name, sizeof k.name, "%s", name.c_str());
        k.ms_per_launch = ms;
        k.flops_per_launch = flops;
        k.bytes_per_launch = bytes;
        k.launches_per_forward = per;
        all.push_back(k);
    };
    add("audio_forward", double(whole) / reps, 0, 0, 1);
    add("audio_tower", double(tower) / reps, 0, 0, 1);
    for (auto& e : sink.entries) add(e.name, e.ms, e.flops, e.bytes, e.occurrences);
    *n_out = int32_t(all.size());
    for (int32_t i = 0; i < std::min<int32_t>(cap, int32_t(all.size())); i++) out[i] = all[size_t(i)];
    return GE_OK;
}

void ge_multimodal_opts_default(ge_multimodal_opts* o) {
    if (!o) return;
    o->max_tokens = 2048;
    o->dimensions = 768;
    o->normalise = 1;
    o->max_image_tokens = 256;
    o->batch_size = 0;
}

int ge_embed_multimodal(ge_model* m, const ge_multimodal_input* inputs, int32_t count, const char* prefix,
                        const ge_multimodal_opts* opts, float* out, int32_t* token_counts, int32_t* truncated,
                        ge_progress_fn progress, void* user) {
    if (!m) return GE_ERR_INVALID_OPTIONS;
    ge_multimodal_opts o;
    ge_multimodal_opts_default(&o);
    if (opts) o = *opts;
    const ge::Config& c = m->cfg;
    // The option checks of embed(_ inputs:) (MultimodalEmbedding.swift:107-131).
    if (!(o.dimensions == 768 || o.dimensions == 512 || o.dimensions == 256 || o.dimensions == 128) ||
        o.dimensions > c.out_dim)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: dimensions must be one of [768, 512, 256, 128]");
    if (o.max_tokens < 2 || o.max_tokens > c.max_tokens)
        return ge::set_error(m, GE_ERR_INVALID_OPTIONS,
                             "invalid options: maxTokens must be between 2 and " + std::to_string(c.max_tokens));
    if (o.batch_size < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: batchSize must be at least 1");
    if (count < 0) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: negative input count");
    if (count > 0 && (!inputs || !out)) return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: NULL array");
    bool any_image = false, any_audio = false;
    for (int32_t i = 0; i < count; i++) {
        if (inputs[i].count < 0 || (inputs[i].count > 0 && !inputs[i].parts))
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: input " + std::to_string(i) + " has no parts array");
        for (int32_t k = 0; k < inputs[i].count; k++) {
            const ge_part& p = inputs[i].parts[k];
            if (p.kind == GE_PART_IMAGE) any_image = true;
            else if (p.kind == GE_PART_AUDIO) any_audio = true;
            else if (p.kind != GE_PART_TEXT || p.text_len < 0 || (p.text_len > 0 && !p.text))
                return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: input " + std::to_string(i) + ", part " +
                                                                    std::to_string(k) + " is malformed");
        }
    }
    if (m->has_vision) {
        if (o.max_image_tokens < 1 || o.max_image_tokens > m->vcfg.native_max_image_tokens)
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: maxImageTokens must be between 1 and " +
                                                                std::to_string(m->vcfg.native_max_image_tokens));
    } else if (any_image) {
        return ge::set_error(m, GE_ERR_IMAGE_ENCODER_NOT_LOADED,
                             "no image encoder is loaded; pass the mmproj GGUF when loading the model");
    }
    if (any_audio && !m->has_audio)
        return ge::set_error(m, GE_ERR_AUDIO_ENCODER_NOT_LOADED,
                             "no audio encoder is loaded; pass the mmproj GGUF as LoadOptions.audioEncoder when loading the model");
    if (count == 0) return GE_OK;
    if (!m->tokenizer)
        return ge::set_error(m, GE_ERR_UNSUPPORTED_ARCHITECTURE, "unsupported architecture: tokenizer model missing");
    // Images and clips of every input, in order, prepared on host threads.
    std::vector<ge_image> imgs;
    std::vector<ge_audio> auds;
    std::vector<int32_t> first_image(static_cast<size_t>(count) + 1, 0), first_clip(static_cast<size_t>(count) + 1, 0);
    for (int32_t i = 0; i < count; i++) {
        first_image[size_t(i)] = int32_t(imgs.size());
        first_clip[size_t(i)] = int32_t(auds.size());
        for (int32_t k = 0; k < inputs[i].count; k++) {
            if (inputs[i].parts[k].kind == GE_PART_IMAGE) imgs.push_back(inputs[i].parts[k].image);
            if (inputs[i].parts[k].kind == GE_PART_AUDIO) auds.push_back(inputs[i].parts[k].audio);
        }
    }
    first_image[size_t(count)] = int32_t(imgs.size());
    first_clip[size_t(count)] = int32_t(auds.size());
    std::vector<ge::PreparedImage> prepared;
    if (!imgs.empty()) {
        int rc = prepare_images(m, imgs.data(), int32_t(imgs.size()), o.max_image_tokens, prepared);
        if (rc) return rc;
    }
    std::vector<ge::PreparedAudio> clips;
    if (!auds.empty()) {
        int rc = prepare_audios(m, auds.data(), int32_t(auds.size()), INT32_MAX, clips);
        if (rc) return rc;
    }
    // One sequence per input (MultimodalSequence, MultimodalEmbedding.swift:43-83).
    const ge::Tokenizer& tk = m->tokenizer->t;
    auto encode = [&](const std::string& t, std::vector<int32_t>& ids) {
        ids.clear();
        tk.encode(reinterpret_cast<const uint8_t*>(t.data()), t.size(), false, false, ids);
    };
    const std::string pre = prefix ? std::string(prefix) : std::string();
    std::vector<std::vector<int32_t>> seqs(static_cast<size_t>(count));
    std::vector<int64_t> costs(3 * static_cast<size_t>(count));
    for (int32_t i = 0; i < count; i++) {
        std::vector<ge::SeqPart> parts;
        std::vector<ge::EncoderSpan> spans;
        int32_t img = first_image[size_t(i)], clip = first_clip[size_t(i)];
        int64_t patches = 0, frames = 0;
        for (int32_t k = 0; k < inputs[i].count; k++) {
            const ge_part& p = inputs[i].parts[k];
            ge::SeqPart sp;
            sp.kind = p.kind;
            if (p.kind == GE_PART_TEXT) {
                sp.text.assign(p.text ? p.text : "", size_t(p.text_len));
            } else if (p.kind == GE_PART_IMAGE) {
                const ge::PreparedImage& im = prepared[size_t(img++)];
                spans.push_back({im.tokens(), m->image_begin, m->image_end});
                patches += im.patches();
            } else {
                const ge::PreparedAudio& au = clips[size_t(clip++)];
                spans.push_back({au.tokens(), m->audio_begin, m->audio_end});
                frames += au.frames();
            }
            parts.push_back(std::move(sp));
        }
        bool cut = false;
        if (!ge::multimodal_sequence(pre, parts, spans, o.max_tokens, c.bos_id, c.eos_id, encode, seqs[size_t(i)], cut))
            return ge::set_error(m, GE_ERR_INVALID_OPTIONS, "invalid options: input " + std::to_string(i) +
                                                                ": its images and clips alone need more than maxTokens (" +
                                                                std::to_string(o.max_tokens) + ") rows");
        if (token_counts) token_counts[i] = int32_t(seqs[size_t(i)].size());
        if (truncated) truncated[i] = cut ? 1 : 0;
        costs[3 * size_t(i)] = int64_t(seqs[size_t(i)].size());
        costs[3 * size_t(i) + 1] = patches;
        costs[3 * size_t(i) + 2] = frames;
    }
    // The three budgets of MultimodalEmbedding.swift:143-145: tokens, image patches, audio frames.
    const int64_t budgets[3] = {m->budget, m->patch_budget, m->frame_budget};
    std::vector<int32_t> ranges(2 * static_cast<size_t>(count));
    int32_t nr = 0;
    ge_batches(costs.data(), count, 3, o.batch_size, budgets, ranges.data(), &nr);
    std::lock_guard<std::mutex> g(m->mu);
    ge::Device& d = m->devs[0];
    const int od = c.out_dim, hidden = c.hidden;
    int32_t done = 0;
    int64_t done_tokens = 0;
    for (int32_t r = 0; r < nr; r++) {
        const int32_t b = ranges[2 * size_t(r)], e = ranges[2 * size_t(r) + 1];
        // The towers over the batch's images and clips (MultimodalEmbedding.swift:173-192).
        std::vector<const ge::PreparedImage*> ims;
        for (int32_t i = first_image[size_t(b)]; i < first_image[size_t(e)]; i++) ims.push_back(&prepared[size_t(i)]);
        std::vector<const ge::PreparedAudio*> cls;
        for (int32_t i = first_clip[size_t(b)]; i < first_clip[size_t(e)]; i++) cls.push_back(&clips[size_t(i)]);
        if (!ims.empty()) {
            ge::VisionArgs va;
            va.imgs = ims.data();
            va.n = int(ims.size());
            const int rc = ge::run_vision(m, d, va);
            if (rc) return rc;
        }
        if (!cls.empty()) {
            ge::AudioArgs aa;
            aa.clips = cls.data();
            aa.n = int(cls.size());
            const int rc = ge::run_audio(m, d, aa);
            if (rc) return rc;
        }
        std::vector<int32_t> toks;
        std::vector<ge_seq> sq;
        int32_t row_base = 0;
        for (int32_t i = b; i < e; i++) {
            sq.push_back({uint32_t(toks.size()), uint32_t(seqs[size_t(i)].size())});
            int32_t rows = 0;
            for (int32_t id : seqs[size_t(i)]) {
                if (id < 0) {
                    toks.push_back(id - row_base);  // -(local + 1) -> -(row_base + local + 1)
                    rows++;
                } else {
                    toks.push_back(id);
                }
            }
            row_base += rows;
        }
        // With one kind of encoder the rows are already in sequence order in its output; with both,
        // each span's rows are copied into one buffer in the order the sequences number them.
        const float* vectors = nullptr;
        if (!ims.empty() && cls.empty()) vectors = d.vis.ws.vectors;
        if (ims.empty() && !cls.empty()) vectors = d.aud.ws.vectors;
        if (!ims.empty() && !cls.empty()) {
            const size_t need = size_t(std::max(row_base, 1)) * hidden;
            cudaError_t ce = cudaSetDevice(d.ordinal);
            if (ce == cudaSuccess && d.mm_vectors_cap < need) {
                if (d.mm_vectors) cudaFree(d.mm_vectors);
                d.mm_vectors = nullptr;
                d.mm_vectors_cap = 0;
                ce = cudaMalloc(&d.mm_vectors, need * sizeof(float));
                if (ce == cudaSuccess) d.mm_vectors_cap = need;
            }
            size_t dst = 0, img_row = 0, clip_row = 0;
            int32_t ii = first_image[size_t(b)], ci = first_clip[size_t(b)];
            for (int32_t i = b; i < e && ce == cudaSuccess; i++)
                for (int32_t k = 0; k < inputs[i].count && ce == cudaSuccess; k++) {
                    const int kind = inputs[i].parts[k].kind;
                    if (kind == GE_PART_TEXT) continue;
                    const bool is_img = kind == GE_PART_IMAGE;
                    const size_t n = is_img ? size_t(prepared[size_t(ii++)].tokens()) : size_t(clips[size_t(ci++)].tokens());
                    const float* src = is_img ? d.vis.ws.vectors + img_row * hidden : d.aud.ws.vectors + clip_row * hidden;
                    ce = cudaMemcpyAsync(d.mm_vectors + dst * hidden, src, n * hidden * sizeof(float),
                                         cudaMemcpyDeviceToDevice, d.stream);
                    (is_img ? img_row : clip_row) += n;
                    dst += n;
                }
            if (ce != cudaSuccess)
                return ge::set_error(m, ce == cudaErrorMemoryAllocation ? GE_ERR_OUT_OF_MEMORY : GE_ERR_GPU_FAILURE,
                                     std::string("GPU execution failed: mixed rows: ") + cudaGetErrorString(ce));
            vectors = d.mm_vectors;
        }
        std::vector<float> pooled(size_t(e - b) * od);
        ge::ForwardArgs a;
        a.tokens = toks.data();
        a.ntok = int(toks.size());
        a.seqs = sq.data();
        a.nseq = int(sq.size());
        a.out = pooled.data();
        a.vectors = vectors;
        a.vector_rows = row_base;
        const int rc = ge::run_forward(m, d, a);
        if (rc) return rc;
        for (int32_t i = b; i < e; i++)
            ge_finish(pooled.data() + size_t(i - b) * od, od, o.dimensions, o.normalise, out + size_t(i) * o.dimensions);
        done += e - b;
        done_tokens += int64_t(toks.size());
        if (progress && progress(done, count, done_tokens, user) != 0 && r + 1 < nr)
            return ge::set_error(m, GE_ERR_CANCELLED, "embedding was cancelled");
    }
    return GE_OK;
}

int ge_tokenizer_load(const char* path, ge_tokenizer** out) {
    if (!out) {
        t_last_error = "invalid options: output handle is NULL";
        return GE_ERR_INVALID_OPTIONS;
    }
    *out = nullptr;
    if (!path) {
        t_last_error = "invalid options: weight path is NULL";
        return GE_ERR_INVALID_OPTIONS;
    }
    ge::GgufFile f;
    ge::GgufError err;
    std::unique_ptr<ge_tokenizer> tk(new ge_tokenizer);
    if (f.open(path, err) || tk->t.build(f, err)) {
        t_last_error = err.message;
        return err.code;
    }
    *out = tk.release();
    return GE_OK;
}

void ge_tokenizer_free(ge_tokenizer* t) { delete t; }

const ge_tokenizer* ge_model_tokenizer(const ge_model* m) { return m ? m->tokenizer.get() : nullptr; }

int ge_tokenizer_get_info(const ge_tokenizer* t, ge_tokenizer_info* info) {
    if (!t || !info) return GE_ERR_INVALID_OPTIONS;
    info->bos_id = t->t.bos_id;
    info->eos_id = t->t.eos_id;
    info->pad_id = t->t.pad_id;
    info->unknown_id = t->t.unknown_id;
    info->vocabulary_size = t->t.vocabulary_size();
    info->add_bos = t->t.add_bos ? 1 : 0;
    info->add_eos = t->t.add_eos ? 1 : 0;
    return GE_OK;
}

int ge_tokenize(const ge_tokenizer* t, const char* text, int64_t len, uint32_t flags, int32_t* ids, int64_t cap,
                int64_t* count) {
    if (!t || !count || len < 0 || cap < 0 || (len > 0 && !text) || (cap > 0 && !ids)) {
        t_last_error = "invalid options: NULL argument or negative size";
        return GE_ERR_INVALID_OPTIONS;
    }
    thread_local std::vector<int32_t> v;
    v.clear();
    t->t.encode(reinterpret_cast<const uint8_t*>(text), size_t(len), (flags & GE_ENCODE_ADD_SPECIAL) != 0,
                (flags & GE_ENCODE_PARSE_SPECIAL) != 0, v);
    *count = int64_t(v.size());
    if (cap > 0) memcpy(ids, v.data(), size_t(std::min<int64_t>(cap, *count)) * sizeof(int32_t));
    return GE_OK;
}

int ge_detokenize(const ge_tokenizer* t, const int32_t* ids, int64_t n, char* text, int64_t cap, int64_t* len) {
    if (!t || !len || n < 0 || cap < 0 || (n > 0 && !ids) || (cap > 0 && !text)) {
        t_last_error = "invalid options: NULL argument or negative size";
        return GE_ERR_INVALID_OPTIONS;
    }
    std::string s;
    t->t.decode(ids, size_t(n), s);
    return copy_out(s, text, cap, len);
}

int ge_token_piece(const ge_tokenizer* t, int32_t id, char* text, int64_t cap, int64_t* len) {
    if (!t || !len || cap < 0 || (cap > 0 && !text)) {
        t_last_error = "invalid options: NULL argument or negative size";
        return GE_ERR_INVALID_OPTIONS;
    }
    const std::string* p = t->t.piece(id);
    if (!p) {
        t_last_error = "invalid options: token id " + std::to_string(id) + " is outside the vocabulary";
        *len = 0;
        return GE_ERR_INVALID_OPTIONS;
    }
    return copy_out(*p, text, cap, len);
}

int ge_token_is_control(const ge_tokenizer* t, int32_t id) { return t && t->t.is_control(id) ? 1 : 0; }

int ge_task_prefix(int32_t task, const char* arg, char* text, int64_t cap, int64_t* len) {
    if (!len || cap < 0 || (cap > 0 && !text)) {
        t_last_error = "invalid options: NULL argument or negative size";
        return GE_ERR_INVALID_OPTIONS;
    }
    std::string s;
    switch (task) {
    case GE_TASK_DOCUMENT: s = "title: " + std::string(arg ? arg : "none") + " | text: "; break;
    case GE_TASK_QUERY: s = "task: " + std::string(arg ? arg : "search result") + " | query: "; break;
    case GE_TASK_CLUSTERING: s = "task: clustering | query: "; break;
    case GE_TASK_CLASSIFICATION: s = "task: classification | query: "; break;
    case GE_TASK_SIMILARITY: s = "task: sentence similarity | query: "; break;
    case GE_TASK_NONE: break;
    default:
        t_last_error = "invalid options: unknown task " + std::to_string(task);
        return GE_ERR_INVALID_OPTIONS;
    }
    return copy_out(s, text, cap, len);
}

}  // extern "C"
