// Synthetic STT-1B checkpoint and input generator.
//
// The reference obtains its weights by downloading kyutai/stt-1b-en_fr and converting them with
// scripts/quantize.py.  Without the network, this file produces a checkpoint of the same
// architecture from a seed, in the same file format:
//   - every value is N(mean, std) drawn from Philox-4x32-10 (Salmon et al., SC'11) keyed by
//     (seed, tensor index), turned into normals by the Box-Muller transform in f64, rounded to
//     f32 and then to bf16 (round to nearest even);
//   - linear weights are Q4_0-quantised exactly as quantize_q4_0 does (scripts/quantize.py:65-116,
//     numpy 2 semantics: f32 absmax, f32 scale = absmax / 7, f32 division, round half to even,
//     clip to [-8, 7], f16 scale by round to nearest even, byte j = (q[j+16]+8) << 4 | (q[j]+8));
//   - norm alphas are written as F32 (quantize.py:223-246 keeps '.alpha' tensors F32);
//   - embedding tables are BF16 (GGML type 30), Q4_0 (as quantize.py writes them) or F32;
//   - tensors appear in sorted-name order with dims reversed and the data section aligned to 32
//     bytes, with no padding between tensors (quantize.py:149-199, 268).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <thread>
#include <vector>

#include "../../include/stt_synth.h"
#include "common.h"

namespace {
thread_local std::string g_synth_error;

int synth_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_synth_error = buf;
    return code;
}
}  // namespace

namespace stt {
namespace {

struct Philox {
    static inline void round(uint32_t c[4], const uint32_t k[2]) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        const uint32_t n0 = hi1 ^ c[1] ^ k[0];
        const uint32_t n2 = hi0 ^ c[3] ^ k[1];
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
    }
    // Philox-4x32-10 of counter `ctr` under key `key`.
    static inline void block(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
        uint32_t c[4] = {ctr[0], ctr[1], ctr[2], ctr[3]};
        uint32_t k[2] = {key[0], key[1]};
        for (int r = 0; r < 10; ++r) {
            round(c, k);
            k[0] += 0x9E3779B9u;
            k[1] += 0xBB67AE85u;
        }
        out[0] = c[0]; out[1] = c[1]; out[2] = c[2]; out[3] = c[3];
    }
};

// Four bf16-rounded N(mean, std) values for group `g` (elements 4g .. 4g+3) of tensor `tidx`.
static inline void normal4(uint64_t seed, uint32_t tidx, uint64_t g, float mean, float stdv,
                           float out[4]) {
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32) ^ tidx};
    const uint32_t ctr[4] = {(uint32_t)g, (uint32_t)(g >> 32), 0u, 0u};
    uint32_t r[4];
    Philox::block(ctr, key, r);
    const double inv32 = 1.0 / 4294967296.0;
    for (int p = 0; p < 2; ++p) {
        const double u1 = ((double)r[2 * p] + 1.0) * inv32;  // (0, 1]
        const double u2 = (double)r[2 * p + 1] * inv32;      // [0, 1)
        const double rad = std::sqrt(-2.0 * std::log(u1));
        const double th = 6.283185307179586476925286766559 * u2;
        const double z0 = rad * std::cos(th), z1 = rad * std::sin(th);
        const float v0 = (float)((double)mean + (double)stdv * z0);
        const float v1 = (float)((double)mean + (double)stdv * z1);
        out[2 * p] = bf16_bits_to_f32(f32_to_bf16_bits_rne(v0));
        out[2 * p + 1] = bf16_bits_to_f32(f32_to_bf16_bits_rne(v1));
    }
}

// Elements [e0, e1) of tensor `tidx` (e0 % 4 == 0).
static void normals(uint64_t seed, uint32_t tidx, uint64_t e0, uint64_t e1, float mean, float stdv,
                    float* dst) {
    float tmp[4];
    for (uint64_t e = e0; e < e1; e += 4) {
        normal4(seed, tidx, e >> 2, mean, stdv, tmp);
        const uint64_t n = std::min<uint64_t>(4, e1 - e);
        for (uint64_t i = 0; i < n; ++i) dst[e - e0 + i] = tmp[i];
    }
}

// quantize.py:91-114 for one block of 32 values.
static void quantize_block(const float* v, uint8_t* out) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(v[j]));
    const float scale = amax > 0.0f ? amax / 7.0f : 1.0f;
    const uint16_t h = f32_to_f16_bits_rne(scale);
    out[0] = (uint8_t)(h & 0xFF);
    out[1] = (uint8_t)(h >> 8);
    int q[32];
    for (int j = 0; j < 32; ++j) {
        float r = std::nearbyint(v[j] / scale);  // default rounding mode: half to even
        int qi = (int)r;
        q[j] = qi < -8 ? -8 : (qi > 7 ? 7 : qi);
    }
    for (int j = 0; j < 16; ++j)
        out[2 + j] = (uint8_t)((((q[j + 16] + 8) & 0x0F) << 4) | ((q[j] + 8) & 0x0F));
}

struct TensorSpec {
    std::string name;
    std::vector<uint64_t> shape;  // PyTorch order
    uint32_t ggml;
    uint32_t tidx;  // Philox key component
    float mean, stdv;
    uint64_t numel() const {
        uint64_t n = 1;
        for (auto d : shape) n *= d;
        return n;
    }
    uint64_t nbytes() const {
        const uint64_t n = numel();
        switch (ggml) {
            case GGML_F32: return n * 4;
            case GGML_F16:
            case GGML_BF16: return n * 2;
            default: return n / 32 * 18;
        }
    }
};

static void put_u32(std::vector<uint8_t>& b, uint32_t v) {
    for (int i = 0; i < 4; ++i) b.push_back((uint8_t)(v >> (8 * i)));
}
static void put_u64(std::vector<uint8_t>& b, uint64_t v) {
    for (int i = 0; i < 8; ++i) b.push_back((uint8_t)(v >> (8 * i)));
}
static void put_str(std::vector<uint8_t>& b, const std::string& s) {
    put_u64(b, s.size());
    b.insert(b.end(), s.begin(), s.end());
}
static void put_f32(std::vector<uint8_t>& b, float f) {
    uint32_t v;
    std::memcpy(&v, &f, 4);
    put_u32(b, v);
}

// Fills rows [r0, r1) of tensor `t` (shape [rows, cols] after flattening leading dims).
static void fill_rows(const TensorSpec& t, uint64_t seed, uint64_t cols, uint64_t r0, uint64_t r1,
                      uint8_t* data) {
    std::vector<float> vals((r1 - r0) * cols);
    normals(seed, t.tidx, r0 * cols, r1 * cols, t.mean, t.stdv, vals.data());
    switch (t.ggml) {
        case GGML_F32:
            std::memcpy(data + r0 * cols * 4, vals.data(), vals.size() * 4);
            break;
        case GGML_BF16: {
            uint16_t* o = reinterpret_cast<uint16_t*>(data) + r0 * cols;
            for (size_t i = 0; i < vals.size(); ++i) o[i] = f32_to_bf16_bits_rne(vals[i]);
            break;
        }
        case GGML_Q4_0: {
            uint8_t* o = data + r0 * cols / 32 * 18;
            for (size_t b = 0; b < vals.size() / 32; ++b) quantize_block(&vals[b * 32], o + b * 18);
            break;
        }
        default: break;
    }
}

}  // namespace
}  // namespace stt

using namespace stt;

extern "C" void stt_synth_default(stt_synth_params* p) {
    if (!p) return;
    std::memset(p, 0, sizeof(*p));
    p->seed = 0x5EED5EEDull;
    p->num_layers = 16;
    p->hidden_size = 2048;
    p->num_heads = 16;
    p->ffn_hidden = 8448;
    p->vocab_size = 8000;
    p->text_in_vocab_size = 8001;
    p->num_codebooks = 32;
    p->audio_vocab_size = 2049;
    p->embedding_dtype = GGML_BF16;
    p->weight_std = 0.02f;
    p->norm_mean = 1.0f;
    p->norm_std = 0.02f;
    p->n_threads = 0;
}

extern "C" int stt_synth_quantize_q4_0(const float* x, size_t n, uint8_t* out) {
    if (!x || !out || n % 32 != 0) return synth_error(STT_E_INVALID_ARG, "quantize: n %% 32 != 0 or NULL");
    for (size_t b = 0; b < n / 32; ++b) quantize_block(x + b * 32, out + b * 18);
    return STT_OK;
}

extern "C" int stt_synth_audio_tokens(uint64_t seed, int32_t stream, int32_t first_frame,
                                      int32_t n_frames, int32_t num_codebooks, uint32_t* out) {
    if (!out || n_frames < 0 || num_codebooks <= 0 || first_frame < 0)
        return synth_error(STT_E_INVALID_ARG, "audio_tokens: bad arguments");
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32) ^ 0x80000000u ^ (uint32_t)stream};
    for (int32_t f = 0; f < n_frames; ++f) {
        for (int32_t g = 0; g < (num_codebooks + 3) / 4; ++g) {
            const uint32_t ctr[4] = {(uint32_t)(first_frame + f), (uint32_t)g, 0xA0D10u, 0u};
            uint32_t r[4];
            Philox::block(ctr, key, r);
            for (int i = 0; i < 4 && 4 * g + i < num_codebooks; ++i)
                out[(size_t)f * num_codebooks + 4 * g + i] = r[i] & 2047u;
        }
    }
    return STT_OK;
}

extern "C" int stt_synth_gguf(const stt_synth_params* p_in, uint8_t** out_buf, size_t* out_len) {
    g_synth_error.clear();
    if (!out_buf || !out_len) return synth_error(STT_E_INVALID_ARG, "synth: NULL output");
    stt_synth_params p;
    if (p_in) p = *p_in; else stt_synth_default(&p);
    const uint64_t D = (uint64_t)p.hidden_size, F = (uint64_t)p.ffn_hidden;
    if (p.num_layers <= 0 || D == 0 || D % 32 || F % 32 || p.num_heads <= 0 || p.vocab_size <= 0 ||
        p.text_in_vocab_size <= 0 || p.num_codebooks <= 0 || p.audio_vocab_size <= 0)
        return synth_error(STT_E_INVALID_ARG, "synth: bad dimensions");
    const uint32_t edt = (uint32_t)p.embedding_dtype;
    if (edt != GGML_BF16 && edt != GGML_Q4_0 && edt != GGML_F32)
        return synth_error(STT_E_INVALID_ARG, "synth: embedding dtype must be 30, 2 or 0");

    std::vector<TensorSpec> ts;
    const float ws = p.weight_std;
    for (int i = 0; i < p.num_codebooks; ++i)
        ts.push_back({"emb." + std::to_string(i) + ".weight", {(uint64_t)p.audio_vocab_size, D}, edt,
                      (uint32_t)i, 0.0f, ws});
    ts.push_back({"text_emb.weight", {(uint64_t)p.text_in_vocab_size, D}, edt, 1000u, 0.0f, ws});
    ts.push_back({"text_linear.weight", {(uint64_t)p.vocab_size, D}, GGML_Q4_0, 1001u, 0.0f, ws});
    ts.push_back({"out_norm.alpha", {1, 1, D}, GGML_F32, 1002u, p.norm_mean, p.norm_std});
    for (int l = 0; l < p.num_layers; ++l) {
        const std::string pre = "transformer.layers." + std::to_string(l) + ".";
        const uint32_t b = 2000u + 16u * (uint32_t)l;
        ts.push_back({pre + "norm1.alpha", {1, 1, D}, GGML_F32, b + 0, p.norm_mean, p.norm_std});
        ts.push_back({pre + "self_attn.in_proj_weight", {3 * D, D}, GGML_Q4_0, b + 1, 0.0f, ws});
        ts.push_back({pre + "self_attn.out_proj.weight", {D, D}, GGML_Q4_0, b + 2, 0.0f, ws});
        ts.push_back({pre + "norm2.alpha", {1, 1, D}, GGML_F32, b + 3, p.norm_mean, p.norm_std});
        ts.push_back({pre + "gating.linear_in.weight", {2 * F, D}, GGML_Q4_0, b + 4, 0.0f, ws});
        ts.push_back({pre + "gating.linear_out.weight", {D, F}, GGML_Q4_0, b + 5, 0.0f, ws});
    }
    std::sort(ts.begin(), ts.end(), [](const TensorSpec& a, const TensorSpec& b) { return a.name < b.name; });

    // Header: magic, version 3, counts, metadata, tensor index (quantize.py:149-199).
    std::vector<uint8_t> hdr;
    put_u32(hdr, 0x46554747u);
    put_u32(hdr, 3u);
    put_u64(hdr, ts.size());
    struct KV { std::string k; int type; std::string s; uint32_t u; float f; };
    std::vector<KV> meta = {
        {"general.architecture", 8, "kyutai-stt", 0, 0.0f},
        {"general.name", 8, "stt-1b-synthetic", 0, 0.0f},
        {"stt.context_length", 4, "", 750u, 0.0f},
        {"stt.embedding_length", 4, "", (uint32_t)D, 0.0f},
        {"stt.block_count", 4, "", (uint32_t)p.num_layers, 0.0f},
        {"stt.feed_forward_length", 4, "", (uint32_t)F, 0.0f},
        {"stt.attention.head_count", 4, "", (uint32_t)p.num_heads, 0.0f},
        {"stt.vocab_size", 4, "", (uint32_t)p.vocab_size, 0.0f},
        {"stt.audio_vocab_size", 4, "", (uint32_t)p.audio_vocab_size, 0.0f},
        {"stt.rope.freq_base", 6, "", 0u, 100000.0f},
        {"stt.synthetic.seed", 8, std::to_string((unsigned long long)p.seed), 0u, 0.0f},
    };
    put_u64(hdr, meta.size());
    for (const auto& kv : meta) {
        put_str(hdr, kv.k);
        put_u32(hdr, (uint32_t)kv.type);
        if (kv.type == 8) put_str(hdr, kv.s);
        else if (kv.type == 4) put_u32(hdr, kv.u);
        else put_f32(hdr, kv.f);
    }
    uint64_t off = 0;
    std::vector<uint64_t> offs;
    for (const auto& t : ts) {
        put_str(hdr, t.name);
        put_u32(hdr, (uint32_t)t.shape.size());
        for (auto it = t.shape.rbegin(); it != t.shape.rend(); ++it) put_u64(hdr, *it);
        put_u32(hdr, t.ggml);
        put_u64(hdr, off);
        offs.push_back(off);
        off += t.nbytes();
    }
    while (hdr.size() % 32) hdr.push_back(0);
    const size_t total = hdr.size() + off;
    uint8_t* buf = (uint8_t*)std::malloc(total);
    if (!buf) return synth_error(STT_E_OOM, "synth: cannot allocate %zu bytes", total);
    std::memcpy(buf, hdr.data(), hdr.size());
    uint8_t* data = buf + hdr.size();

    // Work items: (tensor, row range) chunks of about 1 M values.
    struct Item { size_t t; uint64_t r0, r1, cols; };
    std::vector<Item> items;
    for (size_t i = 0; i < ts.size(); ++i) {
        const uint64_t cols = ts[i].shape.back();
        const uint64_t rows = ts[i].numel() / cols;
        const uint64_t step = std::max<uint64_t>(1, (1u << 20) / cols);
        for (uint64_t r = 0; r < rows; r += step) items.push_back({i, r, std::min(rows, r + step), cols});
    }
    int nth = p.n_threads > 0 ? p.n_threads : (int)std::max(1u, std::thread::hardware_concurrency());
    nth = std::min<int>(nth, (int)items.size());
    std::vector<std::thread> pool;
    std::atomic<size_t> next{0};
    for (int w = 0; w < nth; ++w) {
        pool.emplace_back([&]() {
            for (;;) {
                const size_t k = next.fetch_add(1);
                if (k >= items.size()) break;
                const Item& it = items[k];
                fill_rows(ts[it.t], p.seed, it.cols, it.r0, it.r1, data + offs[it.t]);
            }
        });
    }
    for (auto& th : pool) th.join();
    *out_buf = buf;
    *out_len = total;
    return STT_OK;
}

extern "C" void stt_synth_free(uint8_t* buf) { std::free(buf); }

extern "C" const char* stt_synth_last_error(void) { return g_synth_error.c_str(); }
