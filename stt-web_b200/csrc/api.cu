// C ABI of libsttb200: model loading, stream sets, decode steps and the isolated Q4 matmul.
// The entry points and the reference interfaces they replace are listed in include/stt_b200.h.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdarg>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.h"
#include "gguf.h"
#include "kernels.h"
#include "noalloc.h"
#include "tc_gemm.h"
#include "mega.h"

namespace stt {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}
// Resets the thread's error text and any stale, non-sticky CUDA runtime error left by a call whose
// failure was already handled (e.g. in a destructor), so it cannot surface in a later launch check.
void clear_error() {
    g_last_error.clear();
    (void)cudaGetLastError();
}

#define CUDA_TRY(expr)                                                                              \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            return set_error(STT_E_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_),    \
                             __FILE__, __LINE__);                                                   \
    } while (0)

#define TRY(expr)                  \
    do {                           \
        int rc_ = (expr);          \
        if (rc_ != STT_OK) return rc_; \
    } while (0)

// Allocation-failure injection for tests (stt_debug_fail_allocation): a countdown over the library's
// device and pinned-host allocations; the one that brings it to zero fails as if memory had run out.
std::atomic<int64_t> g_fail_after{-1};

bool injected_failure() {
    int64_t v = g_fail_after.load();
    while (v >= 0)
        if (g_fail_after.compare_exchange_weak(v, v - 1)) return v == 0;
    return false;
}
cudaError_t dev_alloc(void** p, size_t bytes) {
    if (injected_failure()) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMalloc(p, bytes);
}
cudaError_t host_alloc(void** p, size_t bytes) {
    if (injected_failure()) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaHostAlloc(p, bytes, cudaHostAllocDefault);
}

// An allocation: out of memory is STT_E_OOM, any other failure STT_E_CUDA.
#define ALLOC_TRY(expr)                                                                             \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess) {                                                                    \
            (void)cudaGetLastError();                                                               \
            return set_error(e_ == cudaErrorMemoryAllocation ? STT_E_OOM : STT_E_CUDA,              \
                             "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__,      \
                             __LINE__);                                                             \
        }                                                                                           \
    } while (0)

// Restores the calling thread's current device on scope exit.
struct DeviceScope {
    int prev = 0;
    bool ok = false;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
    }
    ~DeviceScope() {
        if (ok) cudaSetDevice(prev);
    }
};

// Device buffer that grows on demand.
struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
    int ensure(size_t bytes) {
        if (bytes <= cap) return STT_OK;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        ALLOC_TRY(dev_alloc(&p, bytes));
        cap = bytes;
        return STT_OK;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

// Pinned host buffer that grows on demand.
struct HostBuf {
    void* p = nullptr;
    size_t cap = 0;
    void release() {
        if (p) cudaFreeHost(p);
        p = nullptr;
        cap = 0;
    }
    int ensure(size_t bytes) {
        if (bytes <= cap) return STT_OK;
        if (p) cudaFreeHost(p);
        p = nullptr;
        cap = 0;
        ALLOC_TRY(host_alloc(&p, bytes));
        cap = bytes;
        return STT_OK;
    }
    ~HostBuf() {
        if (p) cudaFreeHost(p);
    }
};

// Parallel host copy of a byte range of a (possibly sharded) GGUF file: a few worker threads each
// copy one contiguous slice of every request.
class CopyPool {
public:
    explicit CopyPool(int n) {
        for (int i = 0; i < n; ++i) workers_.emplace_back([this, i, n] { loop(i, n); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
            ++gen_;
        }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }
    // Copies bytes [pos, pos + n) of the file to dst; returns false if they run past its end.
    bool read(const GgufFile& f, uint64_t pos, void* dst, uint64_t n) {
        std::unique_lock<std::mutex> lk(mu_);
        file_ = &f;
        pos_ = pos;
        dst_ = static_cast<uint8_t*>(dst);
        n_ = n;
        ok_ = true;
        pending_ = (int)workers_.size();
        ++gen_;
        cv_.notify_all();
        done_.wait(lk, [this] { return pending_ == 0; });
        return ok_;
    }

private:
    void loop(int id, int nw) {
        uint64_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [&] { return gen_ != seen; });
            seen = gen_;
            if (stop_) return;
            const GgufFile* f = file_;
            const uint64_t pos = pos_, n = n_;
            uint8_t* dst = dst_;
            lk.unlock();
            // slices on 4 KB boundaries: each worker touches whole pages of the destination
            const uint64_t pages = (n + 4095) / 4096;
            const uint64_t a = std::min(n, pages * id / nw * 4096), b = std::min(n, pages * (id + 1) / nw * 4096);
            const bool ok = b <= a || f->read_range(pos + a, dst + a, b - a);
            lk.lock();
            if (!ok) ok_ = false;
            if (--pending_ == 0) done_.notify_all();
        }
    }
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_, done_;
    uint64_t gen_ = 0;
    bool stop_ = false, ok_ = true;
    int pending_ = 0;
    const GgufFile* file_ = nullptr;
    uint64_t pos_ = 0, n_ = 0;
    uint8_t* dst_ = nullptr;
};

// Pipelined upload of a checkpoint: the host copies the next piece of the file into one of a few
// pinned staging buffers (several threads) while the copy engine moves the previous pieces to the
// device and the repack kernels split Q4_0 pieces into their planes, all on one stream.  A staging
// buffer is refilled once the event recorded after its last use has completed.
class Uploader {
public:
    static constexpr size_t kPiece = (size_t)16 << 20;       // bytes per staging buffer
    static constexpr size_t kQ4Piece = kPiece / 18 * 18;     // whole Q4_0 blocks per piece
    static constexpr int kStages = 3;

    Uploader() : pool_(std::max(1, std::min(8, (int)std::thread::hardware_concurrency()))) {}
    ~Uploader() {
        if (st_) cudaStreamSynchronize(st_);
        for (auto& e : ev_)
            if (e) cudaEventDestroy(e);
        if (pinned_) cudaFreeHost(pinned_);
        if (draw_) cudaFree(draw_);
        if (st_) cudaStreamDestroy(st_);
    }
    int init() {
        CUDA_TRY(cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking));
        ALLOC_TRY(host_alloc(&pinned_, kPiece * kStages));
        ALLOC_TRY(dev_alloc(&draw_, kPiece * kStages));
        for (auto& e : ev_) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        return STT_OK;
    }
    // File bytes [pos, pos + n) to device memory dst.
    int to_device(const GgufFile& f, uint64_t pos, uint64_t n, void* dst) {
        for (uint64_t o = 0; o < n; o += kPiece) {
            const uint64_t take = std::min<uint64_t>(kPiece, n - o);
            uint8_t* h;
            TRY(stage(f, pos + o, take, &h));
            CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(dst) + o, h, take, cudaMemcpyHostToDevice, st_));
            CUDA_TRY(cudaEventRecord(ev_[cur_], st_));
        }
        return STT_OK;
    }
    // A Q4_0 matrix of nblocks raw blocks at file offset pos, repacked into its planes; big_scale
    // (device) is set when a scale is too large for the tensor-core product.
    int q4(const GgufFile& f, uint64_t pos, int64_t nblocks, uint4* nib, uint16_t* scale, int* big_scale) {
        const int64_t per = (int64_t)(kQ4Piece / 18);
        for (int64_t b0 = 0; b0 < nblocks; b0 += per) {
            const int64_t nb = std::min<int64_t>(per, nblocks - b0);
            uint8_t* h;
            TRY(stage(f, pos + (uint64_t)b0 * 18, (uint64_t)nb * 18, &h));
            uint8_t* d = static_cast<uint8_t*>(draw_) + (size_t)cur_ * kPiece;
            CUDA_TRY(cudaMemcpyAsync(d, h, (size_t)nb * 18, cudaMemcpyHostToDevice, st_));
            CUDA_TRY(launch_repack_q4(d, nb, nib + b0, scale + b0, st_, big_scale));
            CUDA_TRY(cudaEventRecord(ev_[cur_], st_));
        }
        return STT_OK;
    }
    int finish() {
        CUDA_TRY(cudaStreamSynchronize(st_));
        return STT_OK;
    }
    cudaStream_t stream() const { return st_; }

private:
    // Next staging buffer, filled with file bytes [pos, pos + n) (n <= kPiece).
    int stage(const GgufFile& f, uint64_t pos, uint64_t n, uint8_t** out) {
        cur_ = next_;
        next_ = (next_ + 1) % kStages;
        if (used_[cur_]) CUDA_TRY(cudaEventSynchronize(ev_[cur_]));
        used_[cur_] = true;
        uint8_t* h = static_cast<uint8_t*>(pinned_) + (size_t)cur_ * kPiece;
        if (!pool_.read(f, pos, h, n))
            return set_error(STT_E_FORMAT, "tensor data (%llu bytes at %llu) runs past the end of the file",
                             (unsigned long long)n, (unsigned long long)pos);
        *out = h;
        return STT_OK;
    }
    CopyPool pool_;
    cudaStream_t st_ = nullptr;
    void* pinned_ = nullptr;
    void* draw_ = nullptr;
    cudaEvent_t ev_[kStages] = {};
    bool used_[kStages] = {};
    int next_ = 0, cur_ = 0;
};

}  // namespace stt

using namespace stt;

// ------------------------------------------------------------------------------------ model

struct stt_model {
    int device = 0;
    int num_sms = 148;
    stt_config cfg{};
    int32_t L = 0, D = 0, H = 0, HD = 0, F = 0, V = 0, TV = 0, AV = 0, NC = 0, ML = 0;
    int32_t emb_type = 0, emb_row_bytes = 0;
    void* d_mem = nullptr;  // weights, norms, embeddings, rope table
    size_t device_bytes = 0;
    uint64_t q4_bytes = 0;
    std::vector<LayerDev> h_layers;
    LayerDev* d_layers = nullptr;
    Q4Dev head{};
    const float* out_norm = nullptr;
    const float2* rope = nullptr;
    bool tc_ok = false;  // every layer product and the head fit the tensor-core path
    bool tc_gate_ok = false;  // and every linear_in can take the gate into its epilogue
    std::vector<TcWeight> tc_w;  // their TMA descriptors: 4 per layer (qkv, out, fin, fout), then the head
    std::vector<GemvMaps> gemv_maps;  // the GEMV's TMA descriptors, in the same order
    const uint8_t* emb_audio = nullptr;
    const uint8_t* emb_text = nullptr;
    float attn_scale = 0.0f;
};

extern "C" void stt_config_default(stt_config* c) {
    if (!c) return;
    c->num_layers = 16;
    c->hidden_size = 2048;
    c->num_heads = 16;
    c->num_kv_heads = 16;
    c->intermediate_size = 5632;
    c->vocab_size = 8000;
    c->text_in_vocab_size = 8001;
    c->num_codebooks = 32;
    c->audio_vocab_size = 2049;
    c->text_delay = 6;
    c->rope_theta = 100000.0;
    c->max_seq_len = 4096;
    c->sliding_window = 750;
    c->text_padding_id = 3;
    c->text_start_token = 8000;
}

extern "C" const char* stt_last_error(void) { return g_last_error.c_str(); }

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int require(const GgufFile& g, const std::string& name, const GgufTensor** out) {
    *out = g.find(name);
    if (!*out) return set_error(STT_E_FORMAT, "Tensor '%s' not found", name.c_str());
    return STT_OK;
}

// Q4Linear checks of load_q4_linear (gguf.rs:873-888) and Q4Tensor::from_q4_bytes (gguf.rs:418-432),
// plus the shape this build's kernels need.
int check_q4(const GgufTensor* t, uint64_t rows, uint64_t cols) {
    if (t->dtype != GGML_Q4_0)
        return set_error(STT_E_FORMAT, "Expected Q4_0 for '%s', got dtype %u", t->name.c_str(), t->dtype);
    if (t->dims.size() != 2)
        return set_error(STT_E_FORMAT, "'%s' must be 2-D, has %zu dims", t->name.c_str(), t->dims.size());
    const auto s = t->shape();
    if (t->numel % 32 != 0)
        return set_error(STT_E_FORMAT, "Q4_0 requires element count divisible by 32, got %llu",
                         (unsigned long long)t->numel);
    if (s[0] != rows || s[1] != cols)
        return set_error(STT_E_FORMAT, "'%s' has shape [%llu, %llu], expected [%llu, %llu]", t->name.c_str(),
                         (unsigned long long)s[0], (unsigned long long)s[1], (unsigned long long)rows,
                         (unsigned long long)cols);
    if (cols % 32 != 0 || cols > (uint64_t)kMaxGemvK)
        return set_error(STT_E_FORMAT, "'%s': in_features %llu unsupported (multiple of 32, at most %d)",
                         t->name.c_str(), (unsigned long long)cols, kMaxGemvK);
    return STT_OK;
}

// load_rms_norm (gguf.rs:890-925): F32 or F16 (converted with gguf.rs f16_to_f32), Q4_0 rejected.
int load_norm(const GgufFile& g, const GgufTensor* t, int32_t D, std::vector<float>& out) {
    if (t->dtype == GGML_Q4_0)
        return set_error(STT_E_FORMAT, "Cannot load Q4_0 tensor '%s' as norm weight", t->name.c_str());
    if (t->dtype != GGML_F32 && t->dtype != GGML_F16)
        return set_error(STT_E_FORMAT, "norm weight '%s' has unsupported dtype %u", t->name.c_str(), t->dtype);
    if (t->numel != (uint64_t)D)
        return set_error(STT_E_FORMAT, "norm weight '%s' has %llu elements, expected %d", t->name.c_str(),
                         (unsigned long long)t->numel, D);
    std::vector<uint8_t> scratch;
    const uint8_t* p = g.tensor_data(*t, scratch);
    if (!p) return STT_E_FORMAT;
    out.resize(D);
    for (int32_t i = 0; i < D; ++i) {
        if (t->dtype == GGML_F32) std::memcpy(&out[i], p + 4 * i, 4);
        else out[i] = f16_bits_to_f32_gguf((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8)));
    }
    return STT_OK;
}

}  // namespace

extern "C" int stt_model_load_gguf(const uint8_t* const* shards, const size_t* shard_lens, int n_shards,
                                   int device, const stt_config* cfg_in, stt_model** out) {
    clear_error();
    if (!out) return set_error(STT_E_INVALID_ARG, "out is NULL");
    *out = nullptr;
    stt_config cfg;
    if (cfg_in) cfg = *cfg_in; else stt_config_default(&cfg);
    if (cfg.num_layers <= 0 || cfg.num_layers > kMaxLayers || cfg.num_heads <= 0 || cfg.hidden_size <= 0 ||
        cfg.num_codebooks <= 0 || cfg.num_codebooks > kMaxCodebooks || cfg.sliding_window < 0 ||
        cfg.max_seq_len <= 0 || cfg.text_delay < 0)
        return set_error(STT_E_INVALID_ARG, "invalid stt_config");
    if (cfg.num_kv_heads != cfg.num_heads)
        return set_error(STT_E_INVALID_ARG, "num_kv_heads (%d) != num_heads (%d): only MHA is supported",
                         cfg.num_kv_heads, cfg.num_heads);
    GgufFile g;
    TRY(g.open(shards, shard_lens, n_shards));

    auto m = std::make_unique<stt_model>();
    m->device = device;
    m->cfg = cfg;
    m->L = cfg.num_layers;
    m->H = cfg.num_heads;
    m->NC = cfg.num_codebooks;
    m->ML = cfg.sliding_window + 1;  // model.rs:730

    // embeddings (gguf.rs:770-793): shape from the file, one dtype for all tables
    const GgufTensor* text_emb;
    TRY(require(g, "text_emb.weight", &text_emb));
    if (text_emb->dims.size() != 2) return set_error(STT_E_FORMAT, "text_emb.weight must be 2-D");
    m->TV = (int32_t)text_emb->shape()[0];
    m->D = (int32_t)text_emb->shape()[1];
    if (m->D != cfg.hidden_size)
        return set_error(STT_E_FORMAT, "text_emb.weight width %d != hidden_size %d", m->D, cfg.hidden_size);
    if (m->D % m->H != 0 || m->D / m->H != 128)
        return set_error(STT_E_FORMAT, "head_dim %d unsupported (this build needs 128)", m->D / m->H);
    m->HD = m->D / m->H;
    m->emb_type = (int32_t)text_emb->dtype;
    if (m->D % 32 != 0) return set_error(STT_E_FORMAT, "hidden size %d not a multiple of 32", m->D);
    switch (m->emb_type) {
        case GGML_Q4_0: m->emb_row_bytes = m->D / 32 * 18; break;
        case GGML_F32: m->emb_row_bytes = m->D * 4; break;
        default: m->emb_row_bytes = m->D * 2; break;
    }
    std::vector<const GgufTensor*> audio(m->NC);
    for (int i = 0; i < m->NC; ++i) {
        TRY(require(g, "emb." + std::to_string(i) + ".weight", &audio[i]));
        const auto s = audio[i]->shape();
        if (audio[i]->dims.size() != 2 || s[1] != (uint64_t)m->D || audio[i]->dtype != (uint32_t)m->emb_type)
            return set_error(STT_E_FORMAT, "emb.%d.weight: shape/dtype differs from text_emb.weight", i);
        if (i == 0) m->AV = (int32_t)s[0];
        else if (s[0] != (uint64_t)m->AV) return set_error(STT_E_FORMAT, "emb.%d.weight has %llu rows, emb.0 has %d", i, (unsigned long long)s[0], m->AV);
    }

    // layers
    struct LayerT { const GgufTensor *n1, *qkv, *out, *n2, *fin, *fout; };
    std::vector<LayerT> lt(m->L);
    for (int l = 0; l < m->L; ++l) {
        const std::string p = "transformer.layers." + std::to_string(l) + ".";
        TRY(require(g, p + "norm1.alpha", &lt[l].n1));
        TRY(require(g, p + "self_attn.in_proj_weight", &lt[l].qkv));
        TRY(require(g, p + "self_attn.out_proj.weight", &lt[l].out));
        TRY(require(g, p + "norm2.alpha", &lt[l].n2));
        TRY(require(g, p + "gating.linear_in.weight", &lt[l].fin));
        TRY(require(g, p + "gating.linear_out.weight", &lt[l].fout));
        if (l == 0) {
            if (lt[0].fin->dims.size() != 2 || lt[0].fin->shape()[0] % 2 != 0)
                return set_error(STT_E_FORMAT, "linear_in must have an even number of rows");
            m->F = (int32_t)(lt[0].fin->shape()[0] / 2);  // model.rs:519-520
        }
        TRY(check_q4(lt[l].qkv, 3ull * m->D, m->D));
        TRY(check_q4(lt[l].out, m->D, m->D));
        TRY(check_q4(lt[l].fin, 2ull * m->F, m->D));
        TRY(check_q4(lt[l].fout, m->D, m->F));
    }
    const GgufTensor *out_norm_t, *head_t;
    TRY(require(g, "out_norm.alpha", &out_norm_t));
    TRY(require(g, "text_linear.weight", &head_t));
    if (head_t->dims.size() != 2) return set_error(STT_E_FORMAT, "text_linear.weight must be 2-D");
    m->V = (int32_t)head_t->shape()[0];
    TRY(check_q4(head_t, m->V, m->D));
    if ((uint32_t)m->TV <= cfg.text_start_token || (uint32_t)m->TV <= cfg.text_padding_id)
        return set_error(STT_E_FORMAT, "text_emb rows (%d) do not cover start/padding tokens", m->TV);

    // norms (converted on the host)
    std::vector<float> norms((size_t)(2 * m->L + 1) * m->D);
    for (int l = 0; l < m->L; ++l) {
        std::vector<float> a, b;
        TRY(load_norm(g, lt[l].n1, m->D, a));
        TRY(load_norm(g, lt[l].n2, m->D, b));
        std::copy(a.begin(), a.end(), norms.begin() + (size_t)(2 * l) * m->D);
        std::copy(b.begin(), b.end(), norms.begin() + (size_t)(2 * l + 1) * m->D);
    }
    {
        std::vector<float> a;
        TRY(load_norm(g, out_norm_t, m->D, a));
        std::copy(a.begin(), a.end(), norms.begin() + (size_t)(2 * m->L) * m->D);
    }

    // RoPE table (RoPE::new, model.rs:34-59): f32 inverse frequencies, f32 angle, cos/sin.
    const int half = m->HD / 2;
    std::vector<float2> rope((size_t)cfg.max_seq_len * half);
    {
        std::vector<float> inv_freq(half);
        for (int i = 0; i < half; ++i)
            inv_freq[i] = 1.0f / std::pow((float)cfg.rope_theta, (float)(2 * i) / (float)m->HD);
        for (int p = 0; p < cfg.max_seq_len; ++p)
            for (int j = 0; j < half; ++j) {
                const float f = (float)p * inv_freq[j];
                rope[(size_t)p * half + j] = make_float2(std::cos(f), std::sin(f));
            }
    }
    m->attn_scale = std::pow((float)m->HD, -0.5f);  // model.rs:411

    // device memory plan
    std::vector<const GgufTensor*> q4s;
    for (int l = 0; l < m->L; ++l) {
        q4s.push_back(lt[l].qkv);
        q4s.push_back(lt[l].out);
        q4s.push_back(lt[l].fin);
        q4s.push_back(lt[l].fout);
    }
    q4s.push_back(head_t);
    size_t off = 0;
    std::vector<size_t> off_nib(q4s.size()), off_sc(q4s.size());
    for (size_t i = 0; i < q4s.size(); ++i) {
        const size_t nblk = q4s[i]->numel / 32;
        off_nib[i] = off;
        off = align_up(off + nblk * 16, 256);
        off_sc[i] = off;
        off = align_up(off + nblk * 2, 256);
        m->q4_bytes += q4s[i]->nbytes;
    }
    const size_t off_norms = off;
    off = align_up(off + norms.size() * sizeof(float), 256);
    const size_t off_rope = off;
    off = align_up(off + rope.size() * sizeof(float2), 256);
    const size_t audio_table = (size_t)m->AV * m->emb_row_bytes;
    const size_t off_emb = off;
    off = align_up(off + audio_table * m->NC, 256);
    const size_t off_text = off;
    off = align_up(off + (size_t)m->TV * m->emb_row_bytes, 256);
    const size_t off_layers = off;
    off = align_up(off + sizeof(LayerDev) * m->L, 256);
    const size_t off_flag = off;  // the loader's scale-range flag
    off = align_up(off + sizeof(int), 256);
    m->device_bytes = off;

    // Every tensor's bytes must lie inside the input (tensor_data, gguf.rs:298-310).
    {
        std::vector<const GgufTensor*> used(audio.begin(), audio.end());
        used.push_back(text_emb);
        used.push_back(out_norm_t);
        used.push_back(head_t);
        for (const auto& t : lt) {
            used.push_back(t.n1); used.push_back(t.qkv); used.push_back(t.out);
            used.push_back(t.n2); used.push_back(t.fin); used.push_back(t.fout);
        }
        for (const GgufTensor* t : used) {
            const uint64_t abs = g.data_offset() + t->offset;
            if (abs < g.data_offset() || abs > g.total_bytes() || t->nbytes > g.total_bytes() - abs)
                return set_error(STT_E_FORMAT, "tensor '%s' data (%llu bytes at %llu) runs past the end of the file (%llu bytes)",
                                 t->name.c_str(), (unsigned long long)t->nbytes, (unsigned long long)abs,
                                 (unsigned long long)g.total_bytes());
        }
    }

    // The file is fully validated above; only now touch the device.
    int ndev = 0;
    CUDA_TRY(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return set_error(STT_E_INVALID_ARG, "device %d out of range (%d devices)", device, ndev);
    DeviceScope ds(device);
    if (!ds.ok) return set_error(STT_E_CUDA, "cudaSetDevice(%d) failed", device);
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    m->num_sms = prop.multiProcessorCount;
    if (dev_alloc(&m->d_mem, off) != cudaSuccess) {
        cudaGetLastError();
        return set_error(STT_E_OOM, "cannot allocate %zu bytes on device %d", off, device);
    }
    uint8_t* base = static_cast<uint8_t*>(m->d_mem);
    struct Cleanup {
        stt_model* m;
        bool armed = true;
        ~Cleanup() {
            if (armed && m->d_mem) cudaFree(m->d_mem);
        }
    } cleanup{m.get()};

    // Upload: every Q4 matrix (repacked into its planes on the device, its scales checked there for
    // the tensor-core product's range), then the embedding tables as they are in the file; the
    // small host-built tables (norms, RoPE, layer table) go last.
    {
        Uploader up;
        TRY(up.init());
        int* big_scale = reinterpret_cast<int*>(base + off_flag);
        CUDA_TRY(cudaMemsetAsync(big_scale, 0, sizeof(int), up.stream()));
        std::vector<Q4Dev> qd(q4s.size());
        for (size_t i = 0; i < q4s.size(); ++i) {
            const auto s = q4s[i]->shape();
            qd[i].nib = reinterpret_cast<const uint4*>(base + off_nib[i]);
            qd[i].scale = reinterpret_cast<const uint16_t*>(base + off_sc[i]);
            qd[i].n = (int32_t)s[0];
            qd[i].k = (int32_t)s[1];
            TRY(up.q4(g, g.data_offset() + q4s[i]->offset, (int64_t)(q4s[i]->numel / 32), const_cast<uint4*>(qd[i].nib),
                      const_cast<uint16_t*>(qd[i].scale), big_scale));
        }
        for (int i = 0; i < m->NC; ++i)
            TRY(up.to_device(g, g.data_offset() + audio[i]->offset, audio_table, base + off_emb + audio_table * i));
        TRY(up.to_device(g, g.data_offset() + text_emb->offset, (size_t)m->TV * m->emb_row_bytes, base + off_text));
        int big = 0;
        CUDA_TRY(cudaMemcpyAsync(&big, big_scale, sizeof(int), cudaMemcpyDeviceToHost, up.stream()));
        TRY(up.finish());
        m->h_layers.resize(m->L);
        const float* dn = reinterpret_cast<const float*>(base + off_norms);
        for (int l = 0; l < m->L; ++l) {
            LayerDev& L = m->h_layers[l];
            L.qkv = qd[4 * l + 0];
            L.out = qd[4 * l + 1];
            L.fin = qd[4 * l + 2];
            L.fout = qd[4 * l + 3];
            L.norm1 = dn + (size_t)(2 * l) * m->D;
            L.norm2 = dn + (size_t)(2 * l + 1) * m->D;
        }
        m->head = qd.back();
        m->gemv_maps.resize(qd.size());
        for (size_t i = 0; i < qd.size(); ++i)
            if (gemv_make_maps(qd[i], &m->gemv_maps[i]) != cudaSuccess) m->gemv_maps[i].ok = false;
        m->tc_ok = big == 0;
        for (const Q4Dev& w : qd) m->tc_ok = m->tc_ok && tc_gemm_supported(w);
        if (m->tc_ok) {
            m->tc_w.resize(qd.size());
            for (size_t i = 0; i < qd.size(); ++i)
                if (tc_make_weight(qd[i], &m->tc_w[i]) != cudaSuccess) m->tc_ok = false;
            m->tc_gate_ok = m->tc_ok;
            for (int l = 0; l < m->L && m->tc_gate_ok; ++l)
                m->tc_gate_ok = tc_make_gate_maps(qd[4 * l + 2], &m->tc_w[4 * l + 2]) == cudaSuccess &&
                                m->tc_w[4 * l + 2].gate_ok;
        }
        m->out_norm = dn + (size_t)(2 * m->L) * m->D;
    }
    CUDA_TRY(cudaMemcpy(base + off_norms, norms.data(), norms.size() * sizeof(float), cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(base + off_rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(base + off_layers, m->h_layers.data(), sizeof(LayerDev) * m->L, cudaMemcpyHostToDevice));
    m->d_layers = reinterpret_cast<LayerDev*>(base + off_layers);
    m->rope = reinterpret_cast<const float2*>(base + off_rope);
    m->emb_audio = base + off_emb;
    m->emb_text = base + off_text;
    CUDA_TRY(configure_kernels());
    CUDA_TRY(configure_mega());
    CUDA_TRY(cudaDeviceSynchronize());
    cleanup.armed = false;
    *out = m.release();
    return STT_OK;
}

extern "C" int stt_model_destroy(stt_model* m) {
    if (!m) return STT_OK;
    {
        DeviceScope ds(m->device);
        if (m->d_mem) cudaFree(m->d_mem);
    }
    delete m;
    return STT_OK;
}

extern "C" int stt_model_get_info(const stt_model* m, stt_model_info* o) {
    if (!m || !o) return set_error(STT_E_INVALID_ARG, "NULL argument");
    o->num_layers = m->L;
    o->hidden_size = m->D;
    o->num_heads = m->H;
    o->head_dim = m->HD;
    o->ffn_hidden = m->F;
    o->vocab_size = m->V;
    o->text_in_vocab_size = m->TV;
    o->num_codebooks = m->NC;
    o->audio_vocab_size = m->AV;
    o->embedding_dtype = m->emb_type;
    o->device = m->device;
    o->q4_weight_bytes = m->q4_bytes;
    o->device_bytes = m->device_bytes;
    o->tensor_core_min_batch = m->tc_ok ? kTcMinBatch : 0;
    o->reserved = 0;
    return STT_OK;
}

// ------------------------------------------------------------------------------------ streams

struct stt_streams {
    stt_model* m = nullptr;
    int S = 0;
    int kv_f32 = 0;
    void* d_kv = nullptr;
    size_t kv_stream_bytes = 0;
    StreamState* d_state = nullptr;
    std::vector<StreamState> h_state;
    bool state_stale = false;
    // scratch, sized for S batch rows
    float *d_x = nullptr, *d_qkv = nullptr, *d_attn = nullptr, *d_hid = nullptr, *d_logits = nullptr, *d_part = nullptr;
    uint32_t* d_tickets = nullptr;
    __half* d_x16 = nullptr;    // f16 GEMM inputs of a batched step on the tensor cores
    __half* d_x16b = nullptr;   // linear_out's inputs when the gate is fused into linear_in
    float* d_tc_part = nullptr; // their K-slice partial sums
    int32_t* d_ids = nullptr;
    StepDesc* d_desc = nullptr;
    DevBuf in_audio, in_text, out_tokens, out_logits, mega_xa;
    HostBuf h_stage, h_tokens;
    void* d_scratch = nullptr;
    cudaStream_t stream = nullptr;
    std::map<int, cudaGraphExec_t> graphs;
    std::map<int, int> graph_kernels;  // kernel nodes of each captured step graph
    MegaState mega;
    // submitted batched frames whose tokens the caller has not taken yet (stt_streams_submit_frame)
    struct Pending {
        int64_t ticket = -1;
        int n = 0;
        bool taken = true;
        cudaEvent_t ev = nullptr;
    };
    std::vector<Pending> pend;
    HostBuf pend_in, pend_out;    // pinned: per slot the audio ids in, the tokens and step descriptor out
    DevBuf pend_audio, pend_tok;  // device: per slot the audio ids and the emitted tokens
    int64_t next_ticket = 0;
    int product_precision = STT_PRODUCTS_F16X3;  // batched tensor-core products
};

namespace {

constexpr int kTraceCap = 1024;

int nsplit_for(const stt_model* m, int n) {
    // about 4 CTAs per SM (measured best with the K/V staged through shared memory: one split per
    // head at 64 streams, 1.61 ms per step at positions 0..750 against 1.74 with two splits)
    const int want = (4 * m->num_sms + n * m->H - 1) / (n * m->H);
    return std::max(1, std::min(32, want));
}

StreamState fresh_state(const stt_model* m) {
    StreamState s{};
    s.last_text = m->cfg.text_start_token;
    s.prev0 = s.prev1 = 0xFFFFFFFFu;
    return s;
}

Ctx make_ctx(stt_streams* s, int n) {
    stt_model* m = s->m;
    Ctx c{};
    c.layers = m->d_layers;
    c.head = m->head;
    c.out_norm = m->out_norm;
    c.rope = m->rope;
    c.emb_audio = m->emb_audio;
    c.emb_text = m->emb_text;
    c.emb_type = m->emb_type;
    c.emb_row_bytes = m->emb_row_bytes;
    c.L = m->L; c.D = m->D; c.H = m->H; c.HD = m->HD; c.F = m->F; c.V = m->V; c.TV = m->TV; c.AV = m->AV;
    c.NC = m->NC; c.ML = m->ML; c.max_seq_len = m->cfg.max_seq_len;
    c.attn_scale = m->attn_scale;
    c.pad_id = m->cfg.text_padding_id;
    c.text_delay = m->cfg.text_delay;
    c.kv = s->d_kv;
    c.kv_f32 = s->kv_f32;
    c.kv_half_stride = (int64_t)m->H * m->ML * m->HD;
    c.kv_layer_stride = 2 * c.kv_half_stride;
    c.kv_stream_stride = (int64_t)m->L * c.kv_layer_stride;
    c.state = s->d_state;
    c.ids = s->d_ids;
    c.n = n;
    c.desc = s->d_desc;
    c.x = s->d_x; c.qkv = s->d_qkv; c.attn = s->d_attn; c.hid = s->d_hid; c.logits = s->d_logits;
    c.part = s->d_part;
    c.tickets = s->d_tickets;
    c.nsplit = nsplit_for(m, n);
    c.chunk = (m->ML + c.nsplit - 1) / c.nsplit;
    return c;
}

// Enqueues one decode step for batch size n on stream st.
int enqueue_step(stt_streams* s, int n, cudaStream_t st) {
    stt_model* m = s->m;
    const Ctx c = make_ctx(s, n);
    const int grid = 2 * m->num_sms;
    CUDA_TRY(launch_embed(c, st));
    // batches of kTcMinBatch streams or more: layer products on the tensor cores, each product's
    // epilogue writing the next one's f16 input tiles
    if (n >= kTcMinBatch && m->tc_ok && std::getenv("STT_DISABLE_TC") == nullptr) {
        Ctx ca = c;
        ca.x16 = s->d_x16;
        tc_batch_tiles(n, &ca.x16_nt, &ca.x16_rows_pad);
        float* part = s->d_tc_part;
        int* err = &s->d_desc->error;  // a GEMM timeout raises STT_E_DEVICE_FLAG like any step kernel
        int slices = 0;
        const bool x_lo = s->product_precision == STT_PRODUCTS_F16X3;
        // STT_UNFUSED_GATE (read when a batch size's graph is built) keeps linear_in and the gate
        // as two kernels, for the test that compares them
        const bool gate_fused = m->tc_gate_ok && std::getenv("STT_UNFUSED_GATE") == nullptr;
        CUDA_TRY(launch_tc_prep(s->d_x, m->h_layers[0].norm1, m->D, n, s->d_x16, st));
        for (int l = 0; l < m->L; ++l) {
            const LayerDev& L = m->h_layers[l];
            CUDA_TRY(launch_tc_product(m->tc_w[4 * l + 0], s->d_x16, n, part, err, m->num_sms, &slices, st, x_lo));
            GemvArgs a{};
            a.W = L.qkv; a.out = s->d_qkv; a.ldo = 3 * m->D; a.layer = l; a.n_units = 3 * m->D / 2;
            CUDA_TRY(launch_tc_epilogue(c, a, EPI_QKV, n, part, slices, st));
            CUDA_TRY(launch_attention(ca, l, st));
            CUDA_TRY(launch_tc_product(m->tc_w[4 * l + 1], s->d_x16, n, part, err, m->num_sms, &slices, st, x_lo));
            CUDA_TRY(launch_tc_resid_norm(s->d_x, part, slices, n, m->D, L.norm2, s->d_x16, st));
            if (gate_fused) {  // the gate in linear_in's epilogue, its output in the second input buffer
                CUDA_TRY(launch_tc_product_gate(m->tc_w[4 * l + 2], s->d_x16, n, s->d_x16b, err, st, x_lo));
                CUDA_TRY(launch_tc_product(m->tc_w[4 * l + 3], s->d_x16b, n, part, err, m->num_sms, &slices, st, x_lo));
            } else {
                CUDA_TRY(launch_tc_product(m->tc_w[4 * l + 2], s->d_x16, n, part, err, m->num_sms, &slices, st, x_lo));
                CUDA_TRY(launch_tc_gate(part, slices, n, m->F, s->d_x16, st));
                CUDA_TRY(launch_tc_product(m->tc_w[4 * l + 3], s->d_x16, n, part, err, m->num_sms, &slices, st, x_lo));
            }
            const float* next_norm = l + 1 < m->L ? m->h_layers[l + 1].norm1 : m->out_norm;
            CUDA_TRY(launch_tc_resid_norm(s->d_x, part, slices, n, m->D, next_norm, s->d_x16, st));
        }
        CUDA_TRY(launch_tc_product(m->tc_w[4 * m->L], s->d_x16, n, part, err, m->num_sms, &slices, st, x_lo));
        GemvArgs a{};
        a.W = m->head; a.out = s->d_logits; a.ldo = m->V; a.n_units = (m->V + 1) / 2;
        CUDA_TRY(launch_tc_epilogue(c, a, EPI_LOGITS, n, part, slices, st));
        CUDA_TRY(launch_finish(c, st));
        return STT_OK;
    }
    const GemvMaps* gm = m->gemv_maps.data();
    for (int l = 0; l < m->L; ++l) {
        const LayerDev& L = m->h_layers[l];
        GemvArgs a{};
        a.W = L.qkv; a.in = s->d_x; a.norm = L.norm1; a.out = s->d_qkv; a.ldo = 3 * m->D; a.layer = l;
        a.n_units = 3 * m->D / 2; a.maps = &gm[4 * l + 0];
        CUDA_TRY(launch_gemv(c, a, EPI_QKV, n, st));
        CUDA_TRY(launch_attention(c, l, st));
        a = GemvArgs{};
        a.W = L.out; a.in = s->d_attn; a.out = s->d_x; a.ldo = m->D; a.n_units = m->D / 2; a.maps = &gm[4 * l + 1];
        CUDA_TRY(launch_gemv(c, a, EPI_RESID, n, st));
        a = GemvArgs{};
        a.W = L.fin; a.in = s->d_x; a.norm = L.norm2; a.out = s->d_hid; a.ldo = m->F; a.n_units = m->F;
        a.half_n = m->F; a.maps = &gm[4 * l + 2];
        CUDA_TRY(launch_gemv(c, a, EPI_GATE, n, st));
        a = GemvArgs{};
        a.W = L.fout; a.in = s->d_hid; a.out = s->d_x; a.ldo = m->D; a.n_units = m->D / 2; a.maps = &gm[4 * l + 3];
        CUDA_TRY(launch_gemv(c, a, EPI_RESID, n, st));
    }
    GemvArgs a{};
    a.W = m->head; a.in = s->d_x; a.norm = m->out_norm; a.out = s->d_logits; a.ldo = m->V;
    a.n_units = (m->V + 1) / 2; a.maps = &gm[4 * m->L];
    CUDA_TRY(launch_gemv(c, a, EPI_LOGITS, n, st));
    CUDA_TRY(launch_finish(c, st));
    return STT_OK;
}

int graph_for(stt_streams* s, int n, cudaGraphExec_t* out) {
    auto it = s->graphs.find(n);
    if (it != s->graphs.end()) {
        *out = it->second;
        return STT_OK;
    }
    cudaGraph_t graph;
    CUDA_TRY(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(s, n, s->stream);
    cudaError_t e = cudaStreamEndCapture(s->stream, &graph);
    if (rc != STT_OK) {
        if (e == cudaSuccess) cudaGraphDestroy(graph);
        return rc;
    }
    CUDA_TRY(e);
    size_t nodes = 0;
    e = cudaGraphGetNodes(graph, nullptr, &nodes);
    if (e != cudaSuccess) {
        cudaGraphDestroy(graph);
        CUDA_TRY(e);
    }
    s->graph_kernels[n] = (int)nodes;
    cudaGraphExec_t exec;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    CUDA_TRY(e);
    s->graphs[n] = exec;
    *out = exec;
    return STT_OK;
}

// Brings the host copy of every stream state up to date.  Asynchronous calls may have queued
// steps on caller streams, so this waits for the whole device.
int refresh_state(stt_streams* s) {
    if (!s->state_stale) return STT_OK;
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(s->h_state.data(), s->d_state, sizeof(StreamState) * s->S, cudaMemcpyDeviceToHost));
    s->state_stale = false;
    return STT_OK;
}

int check_ids(stt_streams* s, const int32_t* ids, int n) {
    if (!ids || n <= 0 || n > s->S) return set_error(STT_E_INVALID_ARG, "need 1..%d stream ids, got %d", s->S, n);
    std::vector<uint8_t> seen(s->S, 0);
    for (int i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= s->S) return set_error(STT_E_INVALID_ARG, "stream id %d out of range [0, %d)", ids[i], s->S);
        if (seen[ids[i]]) return set_error(STT_E_INVALID_ARG, "stream id %d repeated in one call", ids[i]);
        seen[ids[i]] = 1;
    }
    return STT_OK;
}

// Host-side checks the reference makes by panicking: token ids index the embedding tables
// (gguf.rs:620-621) and positions index the RoPE table (model.rs:72-79).
int check_tokens(const stt_model* m, const uint32_t* audio, size_t n_audio, const uint32_t* text, size_t n_text) {
    for (size_t i = 0; i < n_audio; ++i)
        if (audio[i] >= (uint32_t)m->AV)
            return set_error(STT_E_INVALID_ARG, "audio token %u (index %zu) >= audio vocab %d", audio[i], i, m->AV);
    for (size_t i = 0; text && i < n_text; ++i)
        if (text[i] >= (uint32_t)m->TV)
            return set_error(STT_E_INVALID_ARG, "text token %u (index %zu) >= text vocab %d", text[i], i, m->TV);
    return STT_OK;
}

// Offsets advance by one per queued step, so the host copy of the offsets is always current
// even while other state fields are stale.
int check_positions(stt_streams* s, const int32_t* ids, int n, int steps) {
    for (int i = 0; i < n; ++i) {
        const StreamState& st = s->h_state[ids[i]];
        if ((int64_t)st.offset + steps > s->m->cfg.max_seq_len)
            return set_error(STT_E_STATE, "stream %d: position %d + %d steps exceeds max_seq_len %d", ids[i],
                             st.offset, steps, s->m->cfg.max_seq_len);
    }
    return STT_OK;
}

// Queues `steps` decode steps for the batch `ids` with device-resident inputs and outputs.
int run_steps(stt_streams* s, const int32_t* ids, int n, int steps, const uint32_t* d_audio, const uint32_t* d_text,
              int32_t* d_tokens, float* d_logits, int mode, cudaStream_t st) {
    stt_model* m = s->m;
    if (n > kMaxBatch) return set_error(STT_E_INVALID_ARG, "batch of %d streams exceeds %d", n, kMaxBatch);
    // Large (16 KB), so not on the stack; one per host thread, since threads may drive different
    // handles at the same time (one thread per GPU).  The launch copies it into the kernel's
    // parameters, so it is free again when launch_set_desc returns.
    static thread_local DescInit init;
    init.desc = StepDesc{d_audio, d_text, d_tokens, d_logits, 0, mode, 0, 0};
    init.n = n;
    std::memcpy(init.ids, ids, sizeof(int32_t) * n);
    const bool use_mega = n == 1 && mega_supported(m->L, m->D, m->F, m->HD, m->V, m->num_sms, m->ML, s->kv_f32);
    cudaGraphExec_t exec = nullptr;
    if (!use_mega) TRY(graph_for(s, n, &exec));
    CUDA_TRY(launch_set_desc(s->d_desc, s->d_ids, init, st));
    if (use_mega) {
        // single-stream steps go through the persistent step kernel
        if (s->mega.trace_frame >= 0) {
            CUDA_TRY(cudaMemsetAsync(s->mega.trace, 0, sizeof(unsigned long long) * s->mega.trace_cap, st));
            CUDA_TRY(cudaMemsetAsync(s->mega.trace_ctas, 0,
                                     sizeof(unsigned long long) * (size_t)m->num_sms * kTraceSlots, st));
        }
        if ((size_t)steps * m->D * 4 > s->mega_xa.cap) {
            // growing reallocates: work still queued on another stream may read the old buffer
            CUDA_TRY(cudaDeviceSynchronize());
            TRY(s->mega_xa.ensure((size_t)steps * m->D * 4));
        }
        s->mega.xa_all = static_cast<float*>(s->mega_xa.p);
        CUDA_TRY(launch_mega_steps(s->mega, make_ctx(s, 1), m->h_layers.data(), steps, st));
    } else {
        for (int t = 0; t < steps; ++t) CUDA_TRY(cudaGraphLaunch(exec, st));
    }
    for (int i = 0; i < n; ++i) s->h_state[ids[i]].offset += steps;
    s->state_stale = true;
    return STT_OK;
}

// Synchronous wrapper: host inputs in, host outputs out.
int run_host(stt_streams* s, const int32_t* ids, int n, int steps, const uint32_t* audio, const uint32_t* text,
             int32_t* tokens_out, float* logits_out, int mode) {
    stt_model* m = s->m;
    DeviceScope ds(m->device);
    TRY(check_ids(s, ids, n));
    const size_t n_audio = (size_t)steps * n * m->NC;
    TRY(check_tokens(m, audio, n_audio, text, (size_t)steps * n));
    TRY(check_positions(s, ids, n, steps));
    TRY(s->in_audio.ensure(n_audio * 4));
    TRY(s->out_tokens.ensure((size_t)steps * n * 4));
    if (text) TRY(s->in_text.ensure((size_t)steps * n * 4));
    if (logits_out) TRY(s->out_logits.ensure((size_t)steps * n * m->V * 4));
    // one pinned staging area for the inputs: audio then text
    const size_t in_bytes = n_audio * 4 + (text ? (size_t)steps * n * 4 : 0);
    HostBuf& hb = s->h_tokens;  // reused as the input stage before the outputs arrive
    TRY(hb.ensure(std::max(in_bytes, (size_t)steps * n * 4)));
    std::memcpy(hb.p, audio, n_audio * 4);
    if (text) std::memcpy(static_cast<uint8_t*>(hb.p) + n_audio * 4, text, (size_t)steps * n * 4);
    CUDA_TRY(cudaMemcpyAsync(s->in_audio.p, hb.p, n_audio * 4, cudaMemcpyHostToDevice, s->stream));
    if (text)
        CUDA_TRY(cudaMemcpyAsync(s->in_text.p, static_cast<uint8_t*>(hb.p) + n_audio * 4, (size_t)steps * n * 4,
                                 cudaMemcpyHostToDevice, s->stream));
    TRY(run_steps(s, ids, n, steps, static_cast<uint32_t*>(s->in_audio.p),
                  text ? static_cast<uint32_t*>(s->in_text.p) : nullptr, static_cast<int32_t*>(s->out_tokens.p),
                  logits_out ? static_cast<float*>(s->out_logits.p) : nullptr, mode, s->stream));
    // read-backs on the same stream into pinned memory, then one synchronisation: the tokens and the
    // step descriptor (its error word).  The host keeps the offsets itself (run_steps); the rest of
    // the stream state is read lazily (refresh_state) by the calls that need it.
    CUDA_TRY(cudaMemcpyAsync(hb.p, s->out_tokens.p, (size_t)steps * n * 4, cudaMemcpyDeviceToHost, s->stream));
    TRY(s->h_stage.ensure(sizeof(StepDesc)));
    StepDesc* desc_stage = static_cast<StepDesc*>(s->h_stage.p);
    CUDA_TRY(cudaMemcpyAsync(desc_stage, s->d_desc, sizeof(StepDesc), cudaMemcpyDeviceToHost, s->stream));
    if (logits_out)
        CUDA_TRY(cudaMemcpyAsync(logits_out, s->out_logits.p, (size_t)steps * n * m->V * 4, cudaMemcpyDeviceToHost,
                                 s->stream));
    CUDA_TRY(cudaStreamSynchronize(s->stream));
    if (tokens_out) std::memcpy(tokens_out, hb.p, (size_t)steps * n * 4);
    const StepDesc desc_back = *desc_stage;
    if (desc_back.error != 0)
        return set_error(desc_back.error == STT_E_INVALID_ARG ? STT_E_INVALID_ARG : STT_E_DEVICE_FLAG,
                         "a kernel raised error %d", desc_back.error);
    return STT_OK;
}

}  // namespace

extern "C" int stt_streams_create(stt_model* m, int n_streams, int kv_dtype, stt_streams** out) {
    clear_error();
    if (!m || !out || n_streams <= 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    if (kv_dtype != STT_KV_BF16 && kv_dtype != STT_KV_F32) return set_error(STT_E_INVALID_ARG, "kv_dtype must be 0 or 1");
    *out = nullptr;
    DeviceScope ds(m->device);
    auto s = std::make_unique<stt_streams>();
    s->m = m;
    s->S = n_streams;
    s->kv_f32 = kv_dtype == STT_KV_F32;
    const size_t elem = s->kv_f32 ? 4 : 2;
    s->kv_stream_bytes = (size_t)m->L * 2 * m->H * m->ML * m->HD * elem;
    int max_np = 0;
    for (int n = 1; n <= n_streams; ++n) max_np = std::max(max_np, n * nsplit_for(m, n));
    const size_t S = (size_t)n_streams;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = (off + bytes + 255) / 256 * 256; return o; };
    const size_t o_state = take(sizeof(StreamState) * S);
    const size_t o_x = take(S * m->D * 4), o_qkv = take(S * 3 * m->D * 4), o_attn = take(S * m->D * 4);
    const size_t o_hid = take(S * m->F * 4), o_logits = take(S * m->V * 4);
    // attention partials: the graph path uses n * nsplit_for(n) rows per head, the persistent
    // kernel one row per CTA (num_sms / H splits per head)
    const size_t part_rows = std::max<size_t>((size_t)max_np * m->H, (size_t)m->num_sms);
    const size_t o_part = take(part_rows * (m->HD + 4) * 4);
    const size_t o_tick = take((S * m->H + 1) * 4);
    const size_t o_desc = take(sizeof(StepDesc) + S * 4 + 64);
    const size_t o_mega = take(mega_scratch_bytes(m->num_sms, m->D, m->F, m->V, m->H, m->HD));
    const size_t o_trace = take(kTraceCap * sizeof(unsigned long long));
    // tensor-core products of batches kTcMinBatch .. S: tiled f16 inputs and K-slice partial sums
    size_t x16_bytes = 0, tc_part_bytes_max = 0;
    if (m->tc_ok)
        for (int rows = kTcMinBatch; rows <= n_streams; ++rows) {
            x16_bytes = std::max(x16_bytes, tc_x16_bytes(std::max(m->D, m->F), rows));
            for (const LayerDev& L : m->h_layers)
                for (const Q4Dev* w : {&L.qkv, &L.out, &L.fin, &L.fout})
                    tc_part_bytes_max = std::max(tc_part_bytes_max, tc_part_bytes(*w, rows, m->num_sms));
            tc_part_bytes_max = std::max(tc_part_bytes_max, tc_part_bytes(m->head, rows, m->num_sms));
        }
    const size_t o_x16 = take(x16_bytes);
    const size_t o_x16b = take(m->tc_gate_ok ? x16_bytes : 0);
    const size_t o_tc_part = take(tc_part_bytes_max);
    const size_t o_trace_ctas = take((size_t)m->num_sms * kTraceSlots * sizeof(unsigned long long));
    if (dev_alloc(&s->d_scratch, off) != cudaSuccess) {
        cudaGetLastError();
        return set_error(STT_E_OOM, "cannot allocate %zu bytes of step scratch", off);
    }
    if (dev_alloc(&s->d_kv, s->kv_stream_bytes * S) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(s->d_scratch);
        return set_error(STT_E_OOM, "cannot allocate the KV rings (%zu bytes)", s->kv_stream_bytes * S);
    }
    // from here on a failing call releases everything allocated so far; success hands the set out
    struct ReleaseOnError {
        std::unique_ptr<stt_streams>& set;
        ~ReleaseOnError() {
            if (set) stt_streams_destroy(set.release());
        }
    } release_on_error{s};
    uint8_t* b = static_cast<uint8_t*>(s->d_scratch);
    s->d_state = reinterpret_cast<StreamState*>(b + o_state);
    s->d_x = reinterpret_cast<float*>(b + o_x);
    s->d_qkv = reinterpret_cast<float*>(b + o_qkv);
    s->d_attn = reinterpret_cast<float*>(b + o_attn);
    s->d_hid = reinterpret_cast<float*>(b + o_hid);
    s->d_logits = reinterpret_cast<float*>(b + o_logits);
    s->d_part = reinterpret_cast<float*>(b + o_part);
    s->d_tickets = reinterpret_cast<uint32_t*>(b + o_tick);
    s->d_desc = reinterpret_cast<StepDesc*>(b + o_desc);
    s->d_ids = reinterpret_cast<int32_t*>(b + o_desc + sizeof(StepDesc));
    s->mega.scratch = b + o_mega;
    s->mega.scratch_bytes = mega_scratch_bytes(m->num_sms, m->D, m->F, m->V, m->H, m->HD);
    s->mega.trace = reinterpret_cast<unsigned long long*>(b + o_trace);
    s->mega.trace_cap = kTraceCap;
    s->d_x16 = reinterpret_cast<__half*>(b + o_x16);
    s->d_x16b = reinterpret_cast<__half*>(b + o_x16b);
    s->d_tc_part = reinterpret_cast<float*>(b + o_tc_part);
    s->mega.trace_ctas = reinterpret_cast<unsigned long long*>(b + o_trace_ctas);
    s->mega.trace_slots = kTraceSlots;
    CUDA_TRY(cudaMemset(s->d_scratch, 0, off));
    CUDA_TRY(cudaMemset(s->d_kv, 0, s->kv_stream_bytes * S));
    s->h_state.assign(S, fresh_state(m));
    CUDA_TRY(cudaMemcpy(s->d_state, s->h_state.data(), sizeof(StreamState) * S, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
    *out = s.release();
    return STT_OK;
}

extern "C" int stt_streams_destroy(stt_streams* s) {
    if (!s) return STT_OK;
    {
        DeviceScope ds(s->m->device);
        if (s->stream) cudaStreamSynchronize(s->stream);
        for (auto& p : s->pend)
            if (p.ev) cudaEventDestroy(p.ev);
        s->pend_in.release();
        s->pend_out.release();
        s->pend_audio.release();
        s->pend_tok.release();
        for (auto& kv : s->graphs) cudaGraphExecDestroy(kv.second);
        s->graphs.clear();
        if (s->stream) cudaStreamDestroy(s->stream);
        if (s->d_kv) cudaFree(s->d_kv);
        if (s->d_scratch) cudaFree(s->d_scratch);
        s->in_audio.release();
        s->in_text.release();
        s->out_tokens.release();
        s->out_logits.release();
        s->mega_xa.release();
        s->h_stage.release();
        s->h_tokens.release();
    }
    delete s;
    return STT_OK;
}

extern "C" int stt_forward(stt_streams* s, const int32_t* ids, int n, const uint32_t* audio, const uint32_t* text,
                           float* logits_out, uint32_t* argmax_out) {
    clear_error();
    if (!s || !audio || !text) return set_error(STT_E_INVALID_ARG, "NULL argument");
    std::vector<int32_t> tok(n > 0 ? n : 1);
    TRY(run_host(s, ids, n, 1, audio, text, tok.data(), logits_out, 0));
    if (argmax_out)
        for (int i = 0; i < n; ++i) argmax_out[i] = (uint32_t)tok[i];
    return STT_OK;
}

extern "C" int stt_stream_feed_frame(stt_streams* s, int stream_id, const uint32_t* audio, int32_t* token_out) {
    clear_error();
    if (!s || !audio || !token_out) return set_error(STT_E_INVALID_ARG, "NULL argument");
    const int32_t id = stream_id;
    return run_host(s, &id, 1, 1, audio, nullptr, token_out, nullptr, 1);
}

extern "C" int stt_streams_feed_frame(stt_streams* s, const int32_t* ids, int n, const uint32_t* audio,
                                      int32_t* tokens_out) {
    clear_error();
    if (!s || !audio || !tokens_out) return set_error(STT_E_INVALID_ARG, "NULL argument");
    return run_host(s, ids, n, 1, audio, nullptr, tokens_out, nullptr, 1);
}

extern "C" int stt_stream_feed_frames(stt_streams* s, int stream_id, int n_frames, const uint32_t* audio,
                                      int32_t* tokens_out) {
    clear_error();
    if (!s || !audio || !tokens_out || n_frames < 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    if (n_frames == 0) return STT_OK;
    const int32_t id = stream_id;
    return run_host(s, &id, 1, n_frames, audio, nullptr, tokens_out, nullptr, 1);
}

extern "C" int stt_stream_feed_frames_device(stt_streams* s, int stream_id, int n_frames, const uint32_t* d_audio,
                                             int32_t* d_tokens, void* cuda_stream) {
    clear_error();
    if (!s || !d_audio || !d_tokens || n_frames < 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    if (n_frames == 0) return STT_OK;
    DeviceScope ds(s->m->device);
    const int32_t id = stream_id;
    TRY(check_ids(s, &id, 1));
    TRY(check_positions(s, &id, 1, n_frames));
    TRY(run_steps(s, &id, 1, n_frames, d_audio, nullptr, d_tokens, nullptr, 1, static_cast<cudaStream_t>(cuda_stream)));
    s->state_stale = true;
    return STT_OK;
}

extern "C" int stt_streams_feed_frame_device(stt_streams* s, const int32_t* ids, int n, const uint32_t* d_audio,
                                             int32_t* d_tokens, void* cuda_stream) {
    clear_error();
    if (!s || !d_audio || !d_tokens) return set_error(STT_E_INVALID_ARG, "NULL argument");
    DeviceScope ds(s->m->device);
    TRY(check_ids(s, ids, n));
    TRY(check_positions(s, ids, n, 1));
    TRY(run_steps(s, ids, n, 1, d_audio, nullptr, d_tokens, nullptr, 1, static_cast<cudaStream_t>(cuda_stream)));
    s->state_stale = true;
    return STT_OK;
}

// ------------------------------------------------------------------------------------ submitted frames

namespace {
constexpr int kPendSlots = 64;  // submitted frames whose tokens may be outstanding at once

size_t pend_out_stride(const stt_streams* s) {
    return ((size_t)s->S * sizeof(int32_t) + sizeof(StepDesc) + 15) / 16 * 16;
}

int pend_setup(stt_streams* s) {
    if (!s->pend.empty()) return STT_OK;
    const size_t nc = (size_t)s->m->NC;
    TRY(s->pend_in.ensure((size_t)kPendSlots * s->S * nc * sizeof(uint32_t)));
    TRY(s->pend_out.ensure((size_t)kPendSlots * pend_out_stride(s)));
    TRY(s->pend_audio.ensure((size_t)kPendSlots * s->S * nc * sizeof(uint32_t)));
    TRY(s->pend_tok.ensure((size_t)kPendSlots * s->S * sizeof(int32_t)));
    std::vector<stt_streams::Pending> p(kPendSlots);
    for (auto& x : p) {
        if (cudaEventCreateWithFlags(&x.ev, cudaEventDisableTiming) != cudaSuccess) {
            for (auto& y : p)
                if (y.ev) cudaEventDestroy(y.ev);
            return set_error(STT_E_CUDA, "cudaEventCreate failed");
        }
    }
    s->pend = std::move(p);
    return STT_OK;
}

// The slot of `ticket` if it is a submitted frame whose tokens are still to be taken.
int pend_slot(stt_streams* s, int64_t ticket, int* slot) {
    if (ticket < 0 || ticket >= s->next_ticket || s->pend.empty())
        return set_error(STT_E_INVALID_ARG, "ticket %lld was not issued by this stream set", (long long)ticket);
    const int k = (int)(ticket % kPendSlots);
    if (s->pend[k].ticket != ticket || s->pend[k].taken)
        return set_error(STT_E_INVALID_ARG, "the tokens of ticket %lld were already taken", (long long)ticket);
    *slot = k;
    return STT_OK;
}

int pend_take(stt_streams* s, int k, int32_t* tokens_out) {
    stt_streams::Pending& p = s->pend[k];
    const uint8_t* o = static_cast<const uint8_t*>(s->pend_out.p) + (size_t)k * pend_out_stride(s);
    StepDesc desc;
    std::memcpy(&desc, o + (size_t)s->S * sizeof(int32_t), sizeof desc);
    if (tokens_out) std::memcpy(tokens_out, o, (size_t)p.n * sizeof(int32_t));
    p.taken = true;
    if (desc.error != 0)
        return set_error(desc.error == STT_E_INVALID_ARG ? STT_E_INVALID_ARG : STT_E_DEVICE_FLAG,
                         "a kernel raised error %d in submitted frame %lld", desc.error, (long long)p.ticket);
    return STT_OK;
}
}  // namespace

extern "C" int stt_streams_submit_frame(stt_streams* s, const int32_t* ids, int n, const uint32_t* audio,
                                        int64_t* ticket) {
    clear_error();
    if (!s || !audio || !ticket) return set_error(STT_E_INVALID_ARG, "NULL argument");
    stt_model* m = s->m;
    DeviceScope ds(m->device);
    TRY(check_ids(s, ids, n));
    const size_t nc = (size_t)m->NC;
    TRY(check_tokens(m, audio, (size_t)n * nc, nullptr, 0));
    TRY(check_positions(s, ids, n, 1));
    TRY(pend_setup(s));
    const int k = (int)(s->next_ticket % kPendSlots);
    stt_streams::Pending& p = s->pend[k];
    if (!p.taken)
        return set_error(STT_E_STATE, "%d submitted frames are outstanding; take the tokens of ticket %lld first",
                         kPendSlots, (long long)p.ticket);
    // the slot's previous copies have completed (its event passed when its tokens were taken)
    uint32_t* hin = static_cast<uint32_t*>(s->pend_in.p) + (size_t)k * s->S * nc;
    std::memcpy(hin, audio, (size_t)n * nc * sizeof(uint32_t));
    uint32_t* din = static_cast<uint32_t*>(s->pend_audio.p) + (size_t)k * s->S * nc;
    int32_t* dtok = static_cast<int32_t*>(s->pend_tok.p) + (size_t)k * s->S;
    uint8_t* hout = static_cast<uint8_t*>(s->pend_out.p) + (size_t)k * pend_out_stride(s);
    CUDA_TRY(cudaMemcpyAsync(din, hin, (size_t)n * nc * sizeof(uint32_t), cudaMemcpyHostToDevice, s->stream));
    TRY(run_steps(s, ids, n, 1, din, nullptr, dtok, nullptr, 1, s->stream));
    CUDA_TRY(cudaMemcpyAsync(hout, dtok, (size_t)n * sizeof(int32_t), cudaMemcpyDeviceToHost, s->stream));
    CUDA_TRY(cudaMemcpyAsync(hout + (size_t)s->S * sizeof(int32_t), s->d_desc, sizeof(StepDesc), cudaMemcpyDeviceToHost,
                             s->stream));
    CUDA_TRY(cudaEventRecord(p.ev, s->stream));
    p.ticket = s->next_ticket;
    p.n = n;
    p.taken = false;
    *ticket = s->next_ticket++;
    return STT_OK;
}

extern "C" int stt_streams_poll_frame(stt_streams* s, int64_t ticket, int32_t* tokens_out, int* ready) {
    clear_error();
    if (!s || !tokens_out || !ready) return set_error(STT_E_INVALID_ARG, "NULL argument");
    *ready = 0;
    DeviceScope ds(s->m->device);
    int k;
    TRY(pend_slot(s, ticket, &k));
    const cudaError_t e = cudaEventQuery(s->pend[k].ev);
    if (e == cudaErrorNotReady) {
        (void)cudaGetLastError();
        return STT_OK;
    }
    CUDA_TRY(e);
    *ready = 1;
    return pend_take(s, k, tokens_out);
}

extern "C" int stt_streams_wait_frame(stt_streams* s, int64_t ticket, int32_t* tokens_out) {
    clear_error();
    if (!s || !tokens_out) return set_error(STT_E_INVALID_ARG, "NULL argument");
    DeviceScope ds(s->m->device);
    int k;
    TRY(pend_slot(s, ticket, &k));
    CUDA_TRY(cudaEventSynchronize(s->pend[k].ev));
    return pend_take(s, k, tokens_out);
}

extern "C" int stt_stream_flush(stt_streams* s, int stream_id, uint32_t* tokens_out, int capacity, int* n_tokens) {
    clear_error();
    if (!s || !n_tokens || capacity < 0 || (capacity > 0 && !tokens_out)) return set_error(STT_E_INVALID_ARG, "bad arguments");
    *n_tokens = 0;
    const int steps = s->m->cfg.text_delay;
    if (steps == 0) return STT_OK;
    std::vector<uint32_t> zero((size_t)steps * s->m->NC, 0u);
    std::vector<int32_t> tok(steps);
    // text_delay frames of zero audio through feed_frame (stream.rs:329-335)
    TRY(stt_stream_feed_frames(s, stream_id, steps, zero.data(), tok.data()));
    for (int i = 0; i < steps; ++i)
        if (tok[i] >= 0 && *n_tokens < capacity) tokens_out[(*n_tokens)++] = (uint32_t)tok[i];
    return STT_OK;
}

extern "C" int stt_stream_reset(stt_streams* s, int stream_id, int keep_buffers) {
    clear_error();
    if (!s || stream_id < 0 || stream_id >= s->S) return set_error(STT_E_INVALID_ARG, "bad stream id");
    DeviceScope ds(s->m->device);
    TRY(refresh_state(s));
    s->h_state[stream_id] = fresh_state(s->m);
    CUDA_TRY(cudaMemcpy(s->d_state + stream_id, &s->h_state[stream_id], sizeof(StreamState),
                        cudaMemcpyHostToDevice));
    if (keep_buffers)
        CUDA_TRY(cudaMemsetAsync(static_cast<uint8_t*>(s->d_kv) + s->kv_stream_bytes * stream_id, 0,
                                 s->kv_stream_bytes, s->stream));
    CUDA_TRY(cudaStreamSynchronize(s->stream));
    return STT_OK;
}

extern "C" int stt_stream_reset_async(stt_streams* s, int stream_id, int keep_buffers, void* cuda_stream) {
    clear_error();
    if (!s || stream_id < 0 || stream_id >= s->S) return set_error(STT_E_INVALID_ARG, "bad stream id");
    DeviceScope ds(s->m->device);
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    const StreamState fresh = fresh_state(s->m);
    CUDA_TRY(launch_set_state(s->d_state + stream_id, fresh, st));
    if (keep_buffers)
        CUDA_TRY(cudaMemsetAsync(static_cast<uint8_t*>(s->d_kv) + s->kv_stream_bytes * stream_id, 0,
                                 s->kv_stream_bytes, st));
    // the offset mirror is exact; the other host fields are refreshed on the next synchronous call
    s->h_state[stream_id] = fresh;
    s->state_stale = true;
    return STT_OK;
}

extern "C" int stt_streams_set_product_precision(stt_streams* s, int precision) {
    clear_error();
    if (!s) return set_error(STT_E_INVALID_ARG, "NULL streams");
    if (precision != STT_PRODUCTS_F16X3 && precision != STT_PRODUCTS_F16X2)
        return set_error(STT_E_INVALID_ARG, "precision %d unknown", precision);
    if (precision == s->product_precision) return STT_OK;
    DeviceScope ds(s->m->device);
    CUDA_TRY(cudaStreamSynchronize(s->stream));
    for (auto& kv : s->graphs) cudaGraphExecDestroy(kv.second);  // recaptured with the new products
    s->graphs.clear();
    s->graph_kernels.clear();
    s->product_precision = precision;
    return STT_OK;
}

extern "C" int stt_stream_set_last_text_token(stt_streams* s, int stream_id, uint32_t token) {
    clear_error();
    if (!s || stream_id < 0 || stream_id >= s->S) return set_error(STT_E_INVALID_ARG, "bad stream id");
    if (token >= (uint32_t)s->m->TV) return set_error(STT_E_INVALID_ARG, "token %u >= text vocab %d", token, s->m->TV);
    DeviceScope ds(s->m->device);
    TRY(refresh_state(s));
    s->h_state[stream_id].last_text = token;
    CUDA_TRY(cudaMemcpy(s->d_state + stream_id, &s->h_state[stream_id], sizeof(StreamState),
                        cudaMemcpyHostToDevice));
    return STT_OK;
}

extern "C" int stt_stream_get_state(stt_streams* s, int stream_id, stt_stream_state* out) {
    clear_error();
    if (!s || !out || stream_id < 0 || stream_id >= s->S) return set_error(STT_E_INVALID_ARG, "bad arguments");
    DeviceScope ds(s->m->device);
    s->state_stale = true;
    TRY(refresh_state(s));
    const StreamState& st = s->h_state[stream_id];
    out->offset = st.offset;
    out->len = st.len;
    out->write_pos = st.write_pos;
    out->frame_count = st.frame_count;
    out->last_text_token = st.last_text;
    out->delay_prev[0] = st.prev0;
    out->delay_prev[1] = st.prev1;
    return STT_OK;
}

// ------------------------------------------------------------------------------------ Q4 matmul

struct stt_q4_tensor {
    int device = 0;
    int num_sms = 148;
    Q4Dev w{};
    void* mem = nullptr;
    int* d_err = nullptr;  // timeout flag of the tensor's kernels (inside mem)
    int stall_next = 0;    // test hook: the next integer-MMA GEMV launch waits for a stage never loaded
    bool tc_ok = false;    // shape and scales fit the tensor-core kernel
    TcWeight tc_w{};       // its TMA descriptors
    GemvMaps gemv_maps{};  // the GEMV's TMA descriptors
    mutable DevBuf tc_x16, tc_part;  // its scratch, grown on demand
};

extern "C" int stt_q4_tensor_create(const uint8_t* bytes, size_t n_bytes, int n, int k, int device, stt_q4_tensor** out) {
    clear_error();
    if (!bytes || !out || n <= 0 || k <= 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    *out = nullptr;
    const uint64_t numel = (uint64_t)n * (uint64_t)k;
    // Q4Tensor::from_q4_bytes (gguf.rs:418-432)
    if (numel % 32 != 0) return set_error(STT_E_FORMAT, "Q4_0 requires element count divisible by 32, got %llu", (unsigned long long)numel);
    const uint64_t nblk = numel / 32;
    if (n_bytes != nblk * 18)
        return set_error(STT_E_FORMAT, "Q4_0 byte count mismatch: expected %llu for %llu blocks, got %zu",
                         (unsigned long long)(nblk * 18), (unsigned long long)nblk, n_bytes);
    if (k % 32 != 0 || k > kMaxGemvK)
        return set_error(STT_E_INVALID_ARG, "in_features %d unsupported (multiple of 32, at most %d)", k, kMaxGemvK);
    DeviceScope ds(device);
    if (!ds.ok) return set_error(STT_E_INVALID_ARG, "cannot select device %d", device);
    auto t = std::make_unique<stt_q4_tensor>();
    t->device = device;
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    t->num_sms = prop.multiProcessorCount;
    const size_t nib_bytes = (nblk * 16 + 255) / 256 * 256;
    const size_t sc_bytes = (nblk * 2 + 255) / 256 * 256;
    if (dev_alloc(&t->mem, nib_bytes + sc_bytes + 256) != cudaSuccess) {
        cudaGetLastError();
        return set_error(STT_E_OOM, "cannot allocate Q4 tensor");
    }
    t->w.nib = static_cast<const uint4*>(t->mem);
    t->w.scale = reinterpret_cast<const uint16_t*>(static_cast<uint8_t*>(t->mem) + nib_bytes);
    t->w.n = n;
    t->w.k = k;
    t->d_err = reinterpret_cast<int*>(static_cast<uint8_t*>(t->mem) + nib_bytes + sc_bytes);
    t->tc_ok = tc_gemm_supported(t->w) && tc_gemm_scales_ok(bytes, (int64_t)nblk) &&
               tc_make_weight(t->w, &t->tc_w) == cudaSuccess;
    if (gemv_make_maps(t->w, &t->gemv_maps) != cudaSuccess) t->gemv_maps.ok = false;
    CUDA_TRY(cudaMemset(t->d_err, 0, sizeof(int)));
    DevBuf staging;
    TRY(staging.ensure(n_bytes));
    CUDA_TRY(cudaMemcpy(staging.p, bytes, n_bytes, cudaMemcpyHostToDevice));
    CUDA_TRY(launch_repack_q4(static_cast<const uint8_t*>(staging.p), (int64_t)nblk, const_cast<uint4*>(t->w.nib),
                              const_cast<uint16_t*>(t->w.scale), 0));
    CUDA_TRY(configure_kernels());
    CUDA_TRY(cudaDeviceSynchronize());
    *out = t.release();
    return STT_OK;
}

extern "C" int stt_q4_tensor_destroy(stt_q4_tensor* t) {
    if (!t) return STT_OK;
    {
        DeviceScope ds(t->device);
        if (t->mem) cudaFree(t->mem);
    }
    delete t;
    return STT_OK;
}

extern "C" int stt_q4_matmul_device(const stt_q4_tensor* t, const void* d_in, int in_dtype, int rows, float* d_out,
                                    void* cuda_stream) {
    if (!t || !d_in || !d_out || rows < 0 || in_dtype < 0 || in_dtype > 2)
        return set_error(STT_E_INVALID_ARG, "bad arguments");
    if (rows == 0) return STT_OK;
    DeviceScope ds(t->device);
    if (in_dtype == 2) {
        if (!tc_gemm_supported(t->w))
            return set_error(STT_E_INVALID_ARG, "f16 input needs in_features a multiple of 256, got %d", t->w.k);
        if (!t->tc_ok)
            return set_error(STT_E_INVALID_ARG, "f16 input needs Q4_0 scales of magnitude at most 4");
        if (reinterpret_cast<uintptr_t>(d_in) % 2 != 0)
            return set_error(STT_E_INVALID_ARG, "f16 input must be 2-byte aligned");
        TRY(t->tc_x16.ensure(tc_x16_bytes(t->w.k, rows)));
        TRY(t->tc_part.ensure(tc_part_bytes(t->w, rows, t->num_sms)));
        CUDA_TRY(launch_q4_tc_gemm(t->tc_w, t->w, static_cast<const __half*>(d_in), rows, d_out, t->w.n,
                                   static_cast<__half*>(t->tc_x16.p), static_cast<float*>(t->tc_part.p), t->d_err,
                                   t->num_sms, static_cast<cudaStream_t>(cuda_stream)));
        return STT_OK;
    }
    Ctx c{};
    GemvArgs a{};
    a.W = t->w;
    if (in_dtype == 0) a.in = static_cast<const float*>(d_in);
    else a.in_bf16 = static_cast<const __nv_bfloat16*>(d_in);
    a.out = d_out;
    a.ldo = t->w.n;
    a.n_units = (t->w.n + 1) / 2;
    a.err = t->d_err;
    a.maps = &t->gemv_maps;
    a.stall_test = t->stall_next;
    const_cast<stt_q4_tensor*>(t)->stall_next = 0;
    CUDA_TRY(launch_gemv(c, a, EPI_PLAIN, rows, static_cast<cudaStream_t>(cuda_stream)));
    return STT_OK;
}

// Split-K variant of stt_q4_matmul_device that requests no device memory: its partial sums and
// per-tile counters live in a fixed array of the library's device image (4 MiB of partials,
// 4096 tiles of 16 output rows).  For callers that cannot allocate during a call: a serving
// process that sizes all of its device memory up front and must not grow afterwards, and a
// latency-bound caller (one frame every 80 ms per stream) for which an allocation or a free,
// which can synchronise the whole device, would stall every stream queued on it.  The first call
// on a device looks up the array's address with that device current and keeps it; make that
// first call before capturing a stream.  Calls on one device share the array: they must be
// ordered (one stream, or explicit ordering between streams), or they race.
namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};
}  // namespace

extern "C" int stt_q4_matmul_device_noalloc(const stt_q4_tensor* t, const void* d_in, int in_dtype, int rows,
                                            int splits, float* d_out, void* cuda_stream) {
    clear_error();
    if (!t || !d_in || !d_out || rows < 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    if (in_dtype == 2)
        return set_error(STT_E_INVALID_ARG,
                         "in_dtype 2 (f16, the tensor-core product) is not available without allocation: "
                         "use in_dtype 0 (f32) or 1 (bf16)");
    if (in_dtype != 0 && in_dtype != 1) return set_error(STT_E_INVALID_ARG, "in_dtype %d unknown", in_dtype);
    const int NB = t->w.k / 32;
    if (splits < 1 || splits > kNoAllocMaxSplits || splits > NB)
        return set_error(STT_E_INVALID_ARG, "splits %d out of range [1, %d]", splits, std::min(kNoAllocMaxSplits, NB));
    const uintptr_t align = in_dtype == 0 ? 16 : 8;
    if (reinterpret_cast<uintptr_t>(d_in) % align != 0 || reinterpret_cast<uintptr_t>(d_out) % 4 != 0)
        return set_error(STT_E_INVALID_ARG, "input must be %d-byte aligned and output 4-byte aligned", (int)align);
    const int tiles = (t->w.n + kNoAllocTileRows - 1) / kNoAllocTileRows;
    if (tiles > kNoAllocTickets)
        return set_error(STT_E_INVALID_ARG, "%d output rows need %d tiles of %d; the fixed scratch has %d tile counters",
                         t->w.n, tiles, kNoAllocTileRows, kNoAllocTickets);
    const size_t need = (size_t)splits * (size_t)rows * (size_t)t->w.n * sizeof(float);
    if (need > kNoAllocPartialBytes)
        return set_error(STT_E_INVALID_ARG,
                         "%d splits x %d rows x %d outputs need %zu bytes of partial sums; the fixed scratch holds %zu "
                         "(use fewer splits or rows per call)",
                         splits, rows, t->w.n, need, kNoAllocPartialBytes);
    if (t->device < 0 || t->device >= kNoAllocMaxDevices)
        return set_error(STT_E_INVALID_ARG, "device %d out of range for the fixed scratch", t->device);
    if (rows == 0) return STT_OK;
    DeviceScope ds(t->device);
    if (!ds.ok) return set_error(STT_E_CUDA, "cudaSetDevice(%d) failed", t->device);
    void* scratch;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_addr[t->device]) {
            void* p = nullptr;
            const cudaError_t e = noalloc_scratch_address(&p);
            if (e != cudaSuccess || !p)
                return set_error(STT_E_CUDA, "cudaGetSymbolAddress(fixed scratch) failed on device %d: %s", t->device,
                                 cudaGetErrorString(e));
            g_noalloc_addr[t->device] = p;
        }
        scratch = g_noalloc_addr[t->device];
    }
    const float* in = in_dtype == 0 ? static_cast<const float*>(d_in) : nullptr;
    const __nv_bfloat16* in_bf16 = in_dtype == 1 ? static_cast<const __nv_bfloat16*>(d_in) : nullptr;
    CUDA_TRY(launch_q4_matmul_splitk(t->w, in, in_bf16, rows, d_out, splits, scratch,
                                     static_cast<cudaStream_t>(cuda_stream)));
    return STT_OK;
}

extern "C" int stt_q4_matmul(const stt_q4_tensor* t, const float* input, int rows, float* out) {
    clear_error();
    if (!t || !input || !out || rows < 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    if (rows == 0) return STT_OK;
    DeviceScope ds(t->device);
    DevBuf din, dout;
    TRY(din.ensure((size_t)rows * t->w.k * 4));
    TRY(dout.ensure((size_t)rows * t->w.n * 4));
    CUDA_TRY(cudaMemcpy(din.p, input, (size_t)rows * t->w.k * 4, cudaMemcpyHostToDevice));
    TRY(stt_q4_matmul_device(t, din.p, 0, rows, static_cast<float*>(dout.p), nullptr));
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(out, dout.p, (size_t)rows * t->w.n * 4, cudaMemcpyDeviceToHost));
    return stt_q4_tensor_status(t);
}

extern "C" int stt_q4_tensor_status(const stt_q4_tensor* t) {
    clear_error();
    if (!t) return set_error(STT_E_INVALID_ARG, "bad arguments");
    DeviceScope ds(t->device);
    CUDA_TRY(cudaDeviceSynchronize());
    int flag = 0;
    CUDA_TRY(cudaMemcpy(&flag, t->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (flag == 0) return STT_OK;
    CUDA_TRY(cudaMemset(t->d_err, 0, sizeof(int)));
    return set_error(STT_E_DEVICE_FLAG, "a device-side wait of a matmul on this tensor timed out; its output is invalid");
}

extern "C" int stt_debug_q4_arm_wait_timeout(stt_q4_tensor* t) {
    clear_error();
    if (!t) return set_error(STT_E_INVALID_ARG, "bad arguments");
    t->stall_next = 1;
    return STT_OK;
}

extern "C" int stt_q4_tensor_dequant(const stt_q4_tensor* t, float* out_host) {
    clear_error();
    if (!t || !out_host) return set_error(STT_E_INVALID_ARG, "bad arguments");
    DeviceScope ds(t->device);
    DevBuf d;
    const size_t bytes = (size_t)t->w.n * t->w.k * 4;
    TRY(d.ensure(bytes));
    CUDA_TRY(launch_dequant_q4(t->w, static_cast<float*>(d.p), nullptr));
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(out_host, d.p, bytes, cudaMemcpyDeviceToHost));
    return STT_OK;
}

// ------------------------------------------------------------------------------------ diagnostics

extern "C" int stt_debug_trace_frame(stt_streams* s, int frame) {
    clear_error();
    if (!s) return set_error(STT_E_INVALID_ARG, "NULL streams");
    s->mega.trace_frame = frame < 0 ? -1 : frame;
    return STT_OK;
}

extern "C" int stt_debug_get_trace(stt_streams* s, uint64_t* out, int cap, int* n) {
    clear_error();
    if (!s || !out || !n || cap < 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    DeviceScope ds(s->m->device);
    std::vector<unsigned long long> t(s->mega.trace_cap);
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(t.data(), s->mega.trace, sizeof(unsigned long long) * t.size(), cudaMemcpyDeviceToHost));
    // (tag, value) pairs up to the first pair whose value (a clock reading) is still zero
    int k = 0;
    while (k + 1 < (int)t.size() && t[k + 1] != 0) k += 2;
    *n = std::min(k, cap & ~1);
    for (int i = 0; i < *n; ++i) out[i] = t[i];
    return STT_OK;
}

extern "C" int stt_debug_get_trace_ctas(stt_streams* s, uint64_t* out, int cap, int* n_ctas, int* n_slots) {
    clear_error();
    if (!s || !out || !n_ctas || !n_slots || cap < 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    DeviceScope ds(s->m->device);
    const size_t total = (size_t)s->m->num_sms * kTraceSlots;
    if ((size_t)cap < total) return set_error(STT_E_INVALID_ARG, "capacity %d below %zu", cap, total);
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(out, s->mega.trace_ctas, sizeof(unsigned long long) * total, cudaMemcpyDeviceToHost));
    *n_ctas = s->m->num_sms;
    *n_slots = kTraceSlots;
    return STT_OK;
}

extern "C" int stt_debug_fail_allocation(int after) {
    clear_error();
    g_fail_after.store(after < 0 ? -1 : after);
    return STT_OK;
}

extern "C" int stt_debug_arm_wait_timeout(stt_streams* s) {
    clear_error();
    if (!s) return set_error(STT_E_INVALID_ARG, "NULL streams");
    s->mega.stall_next = 1;
    return STT_OK;
}

extern "C" int stt_debug_graph_kernels(stt_streams* s, int n, int* kernels) {
    clear_error();
    if (!s || !kernels || n <= 1 || n > s->S) return set_error(STT_E_INVALID_ARG, "bad arguments");
    DeviceScope ds(s->m->device);
    cudaGraphExec_t exec;
    TRY(graph_for(s, n, &exec));
    *kernels = s->graph_kernels[n];
    return STT_OK;
}

extern "C" int stt_debug_time_products(stt_streams* s, int n, int iters, double* us_out, double* flops_out) {
    clear_error();
    if (!s || !us_out || n < kTcMinBatch || n > s->S || iters <= 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    stt_model* m = s->m;
    if (!m->tc_ok) return set_error(STT_E_INVALID_ARG, "the model's products do not run on the tensor cores");
    DeviceScope ds(m->device);
    cudaEvent_t a, b;
    CUDA_TRY(cudaEventCreate(&a));
    if (cudaEventCreate(&b) != cudaSuccess) {
        cudaEventDestroy(a);
        return set_error(STT_E_CUDA, "cudaEventCreate failed");
    }
    int rc = STT_OK;
    const int which[5] = {0, 1, 2, 3, 4 * m->L};  // layer 0's four products, then the head
    for (int i = 0; i < 5 && rc == STT_OK; ++i) {
        const TcWeight& tw = m->tc_w[which[i]];
        int slices = 0;
        float ms = 0.0f;
        cudaError_t e = launch_tc_product(tw, s->d_x16, n, s->d_tc_part, &s->d_desc->error, m->num_sms, &slices,
                                          s->stream);
        if (e == cudaSuccess) e = cudaEventRecord(a, s->stream);
        for (int t = 0; t < iters && e == cudaSuccess; ++t)
            e = launch_tc_product(tw, s->d_x16, n, s->d_tc_part, &s->d_desc->error, m->num_sms, &slices, s->stream);
        if (e == cudaSuccess) e = cudaEventRecord(b, s->stream);
        if (e == cudaSuccess) e = cudaEventSynchronize(b);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
        if (e != cudaSuccess) {
            rc = set_error(STT_E_CUDA, "timing product %d: %s", i, cudaGetErrorString(e));
            break;
        }
        us_out[i] = (double)ms * 1000.0 / iters;
        if (flops_out) flops_out[i] = 2.0 * n * (double)tw.n * (double)tw.k;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return rc;
}

extern "C" int stt_debug_barrier_ns(int device, int iters, int mode, double* ns) {
    clear_error();
    if (!ns || iters <= 0) return set_error(STT_E_INVALID_ARG, "bad arguments");
    DeviceScope ds(device);
    if (!ds.ok) return set_error(STT_E_INVALID_ARG, "cannot select device %d", device);
    DevBuf b;
    TRY(b.ensure(256));
    float ms = 0.0f;
    CUDA_TRY(mega_barrier_probe(b.p, iters, mode, &ms));
    *ns = (double)ms * 1e6 / iters;
    return STT_OK;
}
