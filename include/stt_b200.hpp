/*
 * stt_b200.hpp — C++17 host interface over the C ABI of stt_b200.h, with the types and method
 * names of the stt-wasm crate that the library replaces, for C++ hosts and tests.
 *
 * Reference interface (paths inside the stt-web project) and the mirror here:
 *   SttConfig, SttConfig::default()      crates/stt-wasm/src/lib.rs:27-80    SttConfig (defaults on construction)
 *   SttModel, Q4ModelLoader::from_shards  crates/stt-wasm/src/model.rs:583-752,
 *     + load_deferred + finalize           gguf.rs:752-826, 658-692           SttModel::from_shards
 *   SttModel::create_cache -> LayerCaches model.rs:262-296, 728-738            SttModel::create_cache (n streams)
 *   SttModel::forward + argmax(2)         model.rs:631-664, stream.rs:104     LayerCaches::forward
 *   SttStream::new / feed_frame / flush /  stream.rs:53-81, 315-362           SttStream
 *     reset / reset_keep_buffers / set_last_text_token
 *   submit_frame_gpu + take_batch_pending  stream.rs:117-183                  LayerCaches::submit_frame,
 *     (async readback, web/bindings.rs:432-489)                                 PendingFrame::poll / wait
 *   Q4Tensor::from_q4_bytes, q4_matmul    gguf.rs:418-451, 517-578            Q4Tensor, q4_matmul
 *   SpmDecoder                            tokenizer.rs:7-38                   SpmDecoder
 *
 * Errors.  The reference returns anyhow errors at load and panics on bad shapes, token ids and
 * positions; here every failing call throws stt_web::Error, which carries the STT_E_* status and
 * the library's error text.  Ownership.  Handles are move-only RAII objects.  A LayerCaches must
 * not outlive the SttModel it was created from, nor an SttStream the LayerCaches it refers to.
 * Threading is that of the C ABI: calls on one model and its caches are serialised by the caller.
 */
#ifndef STT_B200_HPP
#define STT_B200_HPP

#include <cstdint>
#include <fstream>
#include <iterator>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

#include "stt_b200.h"

namespace stt_web {

class Error : public std::runtime_error {
public:
    Error(int code, const std::string& what) : std::runtime_error(what), code_(code) {}
    int code() const { return code_; }

private:
    int code_;
};

inline void check(int rc, const char* where) {
    if (rc != STT_OK) throw Error(rc, std::string(where) + ": " + stt_last_error());
}

/* SttConfig with SttConfig::default() values (lib.rs:60-80). */
struct SttConfig : stt_config {
    SttConfig() : stt_config() { stt_config_default(this); }
};

enum class KvDtype : int { Bf16 = STT_KV_BF16, F32 = STT_KV_F32 };

namespace detail {
struct ModelDel { void operator()(stt_model* m) const { stt_model_destroy(m); } };
struct StreamsDel { void operator()(stt_streams* s) const { stt_streams_destroy(s); } };
struct Q4Del { void operator()(stt_q4_tensor* t) const { stt_q4_tensor_destroy(t); } };
struct SpmDel { void operator()(stt_spm_decoder* d) const { stt_spm_decoder_destroy(d); } };
}  // namespace detail

/* N independent streams of one model: their KV rings and stream-loop state (LayerCaches,
 * model.rs:262-296, one per stream in the reference). */
class LayerCaches {
public:
    int size() const { return n_; }
    stt_streams* raw() const { return h_.get(); }

    /* SttModel::forward (model.rs:631-664) for one stream, then argmax (stream.rs:104): the
     * stream consumes one frame of audio tokens and the text token; returns the logits and
     * stores the greedy token in *argmax when given. */
    std::vector<float> forward(int stream_id, const std::vector<uint32_t>& audio, uint32_t text,
                               uint32_t* argmax = nullptr) {
        check_audio(audio.size(), 1);
        std::vector<float> logits((size_t)vocab_);
        uint32_t am = 0;
        const int32_t id = stream_id;
        check(stt_forward(h_.get(), &id, 1, audio.data(), &text, logits.data(), &am), "stt_forward");
        if (argmax) *argmax = am;
        return logits;
    }

    /* A submitted batched frame (the PendingFrames of take_batch_pending, stream.rs:146-183):
     * poll() gives its tokens once its step has completed (std::nullopt before), wait() blocks.
     * A token is -1 where the stream is inside the text delay.  Tokens are taken once. */
    class PendingFrame {
    public:
        std::optional<std::vector<int32_t>> poll() {
            std::vector<int32_t> t((size_t)n_);
            int ready = 0;
            check(stt_streams_poll_frame(h_, ticket_, t.data(), &ready), "stt_streams_poll_frame");
            if (!ready) return std::nullopt;
            return t;
        }
        std::vector<int32_t> wait() {
            std::vector<int32_t> t((size_t)n_);
            check(stt_streams_wait_frame(h_, ticket_, t.data()), "stt_streams_wait_frame");
            return t;
        }
        int64_t ticket() const { return ticket_; }

    private:
        friend class LayerCaches;
        PendingFrame(stt_streams* h, int64_t ticket, int n) : h_(h), ticket_(ticket), n_(n) {}
        stt_streams* h_;
        int64_t ticket_;
        int n_;
    };

    /* SttStream::submit_frame_gpu (stream.rs:117-138) for the streams `ids` at once: one frame of
     * audio per stream (ids.size() * codebooks tokens), the text token fed back on the device,
     * queued without waiting. */
    PendingFrame submit_frame(const std::vector<int32_t>& ids, const std::vector<uint32_t>& audio) {
        check_audio(audio.size(), ids.size());
        int64_t t = 0;
        check(stt_streams_submit_frame(h_.get(), ids.data(), (int)ids.size(), audio.data(), &t),
              "stt_streams_submit_frame");
        return PendingFrame(h_.get(), t, (int)ids.size());
    }

private:
    friend class SttModel;
    friend class SttStream;
    LayerCaches(stt_streams* h, int n, int codebooks, int vocab) : h_(h), n_(n), codebooks_(codebooks), vocab_(vocab) {}
    void check_audio(size_t got, size_t frames) const {
        if (got != frames * (size_t)codebooks_)
            throw Error(STT_E_INVALID_ARG, "audio: " + std::to_string(got) + " tokens for " + std::to_string(frames) +
                                               " frame(s) of " + std::to_string(codebooks_) + " codebooks");
    }
    std::unique_ptr<stt_streams, detail::StreamsDel> h_;
    int n_, codebooks_, vocab_;
};

/* The loaded transformer on one CUDA device (SttModel, model.rs:583-752). */
class SttModel {
public:
    /* Q4ModelLoader::from_shards + load_deferred + finalize (gguf.rs:752-826, 658-692). */
    static SttModel from_shards(const std::vector<std::vector<uint8_t>>& shards, int device = 0,
                                const SttConfig& config = SttConfig()) {
        std::vector<const uint8_t*> ptrs;
        std::vector<size_t> lens;
        for (const auto& s : shards) {
            ptrs.push_back(s.data());
            lens.push_back(s.size());
        }
        stt_model* h = nullptr;
        check(stt_model_load_gguf(ptrs.data(), lens.data(), (int)shards.size(), device, &config, &h),
              "stt_model_load_gguf");
        return SttModel(h, config);
    }

    /* SttModel::create_cache (model.rs:728-738), for n independent streams. */
    LayerCaches create_cache(int n_streams = 1, KvDtype kv = KvDtype::Bf16) const {
        stt_streams* s = nullptr;
        check(stt_streams_create(h_.get(), n_streams, (int)kv, &s), "stt_streams_create");
        const stt_model_info i = info();
        return LayerCaches(s, n_streams, i.num_codebooks, i.vocab_size);
    }

    stt_model_info info() const {
        stt_model_info i{};
        check(stt_model_get_info(h_.get(), &i), "stt_model_get_info");
        return i;
    }
    const SttConfig& config() const { return cfg_; }
    stt_model* raw() const { return h_.get(); }

private:
    SttModel(stt_model* h, const SttConfig& cfg) : h_(h), cfg_(cfg) {}
    std::unique_ptr<stt_model, detail::ModelDel> h_;
    SttConfig cfg_;
};

/* The delayed-streams loop of one stream (SttStream, stream.rs:19-363). */
class SttStream {
public:
    /* SttStream::new(config, cache) (stream.rs:53-64): stream `stream_id` of `caches`. */
    explicit SttStream(LayerCaches& caches, int stream_id = 0) : c_(&caches), id_(stream_id) {}

    /* SttStream::feed_frame (stream.rs:70-81): nullopt inside the text delay. */
    std::optional<uint32_t> feed_frame(const std::vector<uint32_t>& audio) {
        c_->check_audio(audio.size(), 1);
        int32_t tok = -1;
        check(stt_stream_feed_frame(c_->raw(), id_, audio.data(), &tok), "stt_stream_feed_frame");
        return tok >= 0 ? std::optional<uint32_t>((uint32_t)tok) : std::nullopt;
    }

    /* Consecutive feed_frame calls with the token fed back on the device (submit_frame_gpu,
     * stream.rs:117-138, with feed_frame's semantics): audio holds whole frames. */
    std::vector<std::optional<uint32_t>> feed_frames(const std::vector<uint32_t>& audio) {
        const size_t cb = (size_t)c_->codebooks_;
        const size_t frames = cb ? audio.size() / cb : 0;
        c_->check_audio(audio.size(), frames);
        std::vector<int32_t> tok(frames);
        check(stt_stream_feed_frames(c_->raw(), id_, (int)frames, audio.data(), tok.data()), "stt_stream_feed_frames");
        std::vector<std::optional<uint32_t>> out;
        out.reserve(frames);
        for (int32_t t : tok) out.push_back(t >= 0 ? std::optional<uint32_t>((uint32_t)t) : std::nullopt);
        return out;
    }

    /* SttStream::flush (stream.rs:315-338). */
    std::vector<uint32_t> flush() {
        std::vector<uint32_t> out(64);
        int n = 0;
        check(stt_stream_flush(c_->raw(), id_, out.data(), (int)out.size(), &n), "stt_stream_flush");
        out.resize((size_t)n);
        return out;
    }

    void reset() { check(stt_stream_reset(c_->raw(), id_, 0), "stt_stream_reset"); }
    void reset_keep_buffers() { check(stt_stream_reset(c_->raw(), id_, 1), "stt_stream_reset"); }
    void set_last_text_token(uint32_t token) {
        check(stt_stream_set_last_text_token(c_->raw(), id_, token), "stt_stream_set_last_text_token");
    }
    stt_stream_state state() const {
        stt_stream_state s{};
        check(stt_stream_get_state(c_->raw(), id_, &s), "stt_stream_get_state");
        return s;
    }

private:
    LayerCaches* c_;
    int id_;
};

/* One Q4_0 matrix in the device layout (Q4Tensor, gguf.rs:403-460). */
class Q4Tensor {
public:
    /* Q4Tensor::from_q4_bytes (gguf.rs:418-451): raw 18-byte blocks of an [n, k] matrix. */
    static Q4Tensor from_q4_bytes(const std::vector<uint8_t>& bytes, int n, int k, int device = 0) {
        stt_q4_tensor* t = nullptr;
        check(stt_q4_tensor_create(bytes.data(), bytes.size(), n, k, device, &t), "stt_q4_tensor_create");
        return Q4Tensor(t, n, k);
    }
    /* (nibble - 8) * scale for every weight, bit-exact with gguf.rs:616-633. */
    // Waits for the device; throws Error(STT_E_DEVICE_FLAG) if a device-side wait of a matmul on
    // this tensor ran out since the last check.
    void status() const { check(stt_q4_tensor_status(h_.get()), "stt_q4_tensor_status"); }
    std::vector<float> dequant() const {
        std::vector<float> out((size_t)n_ * (size_t)k_);
        check(stt_q4_tensor_dequant(h_.get(), out.data()), "stt_q4_tensor_dequant");
        return out;
    }
    int n() const { return n_; }
    int k() const { return k_; }
    stt_q4_tensor* raw() const { return h_.get(); }

private:
    Q4Tensor(stt_q4_tensor* t, int n, int k) : h_(t), n_(n), k_(k) {}
    std::unique_ptr<stt_q4_tensor, detail::Q4Del> h_;
    int n_, k_;
};

/* q4_matmul (gguf.rs:517-578): out[rows, n] = input[rows, k] x W^T. */
inline std::vector<float> q4_matmul(const std::vector<float>& input, int rows, const Q4Tensor& w) {
    if (rows < 0 || input.size() != (size_t)rows * (size_t)w.k())
        throw Error(STT_E_INVALID_ARG, "q4_matmul: input of " + std::to_string(input.size()) + " values is not " +
                                           std::to_string(rows) + " rows of " + std::to_string(w.k()));
    std::vector<float> out((size_t)rows * (size_t)w.n());
    check(stt_q4_matmul(w.raw(), input.data(), rows, out.data()), "stt_q4_matmul");
    return out;
}

/* SentencePiece detokeniser (SpmDecoder, tokenizer.rs:7-38); host only. */
class SpmDecoder {
public:
    static SpmDecoder from_bytes(const std::vector<uint8_t>& data) {
        stt_spm_decoder* d = nullptr;
        check(stt_spm_decoder_create(data.data(), data.size(), &d), "stt_spm_decoder_create");
        return SpmDecoder(d);
    }
    /* SpmDecoder::load on a native host (tokenizer.rs:23-26): reads the file. */
    static SpmDecoder load(const std::string& path) {
        std::ifstream f(path, std::ios::binary);
        if (!f) throw Error(STT_E_INVALID_ARG, "Failed to read " + path);
        return from_bytes(std::vector<uint8_t>(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>()));
    }
    std::string decode(const std::vector<uint32_t>& ids) const {
        size_t len = 0;
        check(stt_spm_decode(h_.get(), ids.data(), ids.size(), nullptr, 0, &len), "stt_spm_decode");
        std::string text(len + 1, '\0');
        check(stt_spm_decode(h_.get(), ids.data(), ids.size(), &text[0], text.size(), &len), "stt_spm_decode");
        text.resize(len);
        return text;
    }
    size_t vocab_len() const {
        int64_t n = 0;
        check(stt_spm_vocab_len(h_.get(), &n), "stt_spm_vocab_len");
        return (size_t)n;
    }

private:
    explicit SpmDecoder(stt_spm_decoder* d) : h_(d) {}
    std::unique_ptr<stt_spm_decoder, detail::SpmDel> h_;
};

}  // namespace stt_web

#endif  // STT_B200_HPP
