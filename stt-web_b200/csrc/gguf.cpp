#include "gguf.h"

#include <algorithm>
#include <functional>

namespace stt {

bool ggml_nbytes(uint32_t dtype, uint64_t numel, uint64_t* out) {
    switch (dtype) {
        case GGML_F32: *out = numel * 4; return true;
        case GGML_F16:
        case GGML_BF16: *out = numel * 2; return true;
        case GGML_Q4_0: *out = numel / 32 * 18; return true;
        default: return false;
    }
}

bool GgufFile::read(uint64_t pos, void* dst, uint64_t n) const {
    if (pos > total_ || n > total_ - pos) return false;
    uint8_t* d = static_cast<uint8_t*>(dst);
    // first shard whose end is beyond pos (ShardedCursor::shard_for_offset, gguf.rs:344-355)
    size_t s = std::upper_bound(end_.begin(), end_.end(), pos) - end_.begin();
    while (n > 0) {
        const uint64_t start = s == 0 ? 0 : end_[s - 1];
        const uint64_t local = pos - start;
        const uint64_t take = std::min<uint64_t>(n, end_[s] - pos);
        std::memcpy(d, ptr_[s] + local, take);
        d += take;
        pos += take;
        n -= take;
        ++s;
    }
    return true;
}

namespace {
// String::from_utf8 acceptance (gguf.rs:91-96): well-formed UTF-8, no surrogates or overlongs.
bool valid_utf8(const std::string& s) {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
    size_t i = 0, n = s.size();
    while (i < n) {
        unsigned c = p[i];
        size_t len;
        unsigned cp;
        if (c < 0x80) { ++i; continue; }
        else if ((c & 0xE0) == 0xC0) { len = 2; cp = c & 0x1F; }
        else if ((c & 0xF0) == 0xE0) { len = 3; cp = c & 0x0F; }
        else if ((c & 0xF8) == 0xF0) { len = 4; cp = c & 0x07; }
        else return false;
        if (i + len > n) return false;
        for (size_t k = 1; k < len; ++k) {
            if ((p[i + k] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (p[i + k] & 0x3F);
        }
        if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) ||
            cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))
            return false;
        i += len;
    }
    return true;
}
}  // namespace

int GgufFile::open(const uint8_t* const* shards, const size_t* lens, int n_shards) {
    if (!shards || !lens || n_shards <= 0) return set_error(STT_E_INVALID_ARG, "no GGUF shards given");
    ptr_.clear();
    end_.clear();
    tensors_.clear();
    total_ = 0;
    for (int i = 0; i < n_shards; ++i) {
        if (!shards[i] && lens[i]) return set_error(STT_E_INVALID_ARG, "GGUF shard %d is NULL", i);
        if (lens[i] == 0) continue;
        ptr_.push_back(shards[i]);
        total_ += lens[i];
        end_.push_back(total_);
    }
    uint64_t pos = 0;
    bool bad_utf8 = false;
    auto rd32 = [&](uint32_t* v) { bool ok = read(pos, v, 4); pos += 4; return ok; };
    auto rd64 = [&](uint64_t* v) { bool ok = read(pos, v, 8); pos += 8; return ok; };
    auto rdstr = [&](std::string* s) {
        uint64_t n;
        if (!rd64(&n)) return false;
        if (n > total_) return false;
        s->resize(n);
        if (n && !read(pos, &(*s)[0], n)) return false;
        pos += n;
        if (!valid_utf8(*s)) { bad_utf8 = true; return false; }
        return true;
    };

    uint32_t magic = 0;
    if (!rd32(&magic)) return set_error(STT_E_FORMAT, "Failed to read GGUF magic");
    if (magic != 0x46554747u)
        return set_error(STT_E_FORMAT, "Invalid GGUF magic: 0x%08X (expected 0x46554747)", magic);
    if (!rd32(&version_)) return set_error(STT_E_FORMAT, "Failed to read GGUF version");
    if (version_ != 2 && version_ != 3)
        return set_error(STT_E_FORMAT, "Unsupported GGUF version: %u (expected 2 or 3)", version_);
    uint64_t n_meta = 0;
    if (!rd64(&tensor_count_)) return set_error(STT_E_FORMAT, "Failed to read tensor count");
    if (!rd64(&n_meta)) return set_error(STT_E_FORMAT, "Failed to read metadata KV count");

    // skip_gguf_value (gguf.rs:98-122); arrays recurse with an explicit stack depth bound.
    std::function<bool(uint32_t, int)> skip = [&](uint32_t type, int depth) -> bool {
        static const uint8_t fixed[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (type > 12) {
            set_error(STT_E_FORMAT, "Unknown GGUF metadata value type: %u", type);
            return false;
        }
        if (type == 8) {
            std::string s;
            if (!rdstr(&s)) { set_error(STT_E_FORMAT, "truncated metadata string"); return false; }
            return true;
        }
        if (type == 9) {
            uint32_t et;
            uint64_t cnt;
            if (!rd32(&et) || !rd64(&cnt)) { set_error(STT_E_FORMAT, "truncated metadata array"); return false; }
            if (depth > 8) { set_error(STT_E_FORMAT, "metadata arrays nested too deeply"); return false; }
            if (et <= 12 && et != 8 && et != 9) {  // fixed-size elements: skip in one step
                const uint64_t sz = fixed[et];
                if (cnt > total_ / sz || pos + cnt * sz > total_) {
                    set_error(STT_E_FORMAT, "truncated metadata array");
                    return false;
                }
                pos += cnt * sz;
                return true;
            }
            for (uint64_t i = 0; i < cnt; ++i)
                if (!skip(et, depth + 1)) return false;
            return true;
        }
        pos += fixed[type];
        if (pos > total_) { set_error(STT_E_FORMAT, "truncated metadata value"); return false; }
        return true;
    };
    for (uint64_t i = 0; i < n_meta; ++i) {
        std::string key;
        uint32_t vt;
        if (!rdstr(&key))
            return set_error(STT_E_FORMAT, bad_utf8 ? "Invalid UTF-8 in GGUF string (metadata key %llu)"
                                                    : "Failed to read metadata key %llu", (unsigned long long)i);
        if (!rd32(&vt)) return set_error(STT_E_FORMAT, "Failed to read metadata value type %llu", (unsigned long long)i);
        if (!skip(vt, 0)) return STT_E_FORMAT;
    }
    for (uint64_t i = 0; i < tensor_count_; ++i) {
        GgufTensor t;
        uint32_t nd;
        if (!rdstr(&t.name))
            return set_error(STT_E_FORMAT, bad_utf8 ? "Invalid UTF-8 in GGUF string (tensor name %llu)"
                                                    : "Failed to read tensor name %llu", (unsigned long long)i);
        if (!rd32(&nd)) return set_error(STT_E_FORMAT, "Failed to read ndims for tensor %llu", (unsigned long long)i);
        if (nd > 8) return set_error(STT_E_FORMAT, "tensor %s has %u dims", t.name.c_str(), nd);
        t.numel = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            uint64_t v;
            if (!rd64(&v)) return set_error(STT_E_FORMAT, "Failed to read dim %u for tensor %llu", d, (unsigned long long)i);
            if (v != 0 && t.numel > UINT64_MAX / 16 / v)
                return set_error(STT_E_FORMAT, "tensor %s is too large", t.name.c_str());
            t.dims.push_back(v);
            t.numel *= v;
        }
        if (!rd32(&t.dtype)) return set_error(STT_E_FORMAT, "Failed to read dtype for tensor %llu", (unsigned long long)i);
        if (!ggml_nbytes(t.dtype, t.numel, &t.nbytes))
            return set_error(STT_E_FORMAT, "Unsupported GGML dtype code: %u", t.dtype);
        if (!rd64(&t.offset)) return set_error(STT_E_FORMAT, "Failed to read offset for tensor %llu", (unsigned long long)i);
        std::string key = t.name;
        tensors_[key] = std::move(t);
    }
    data_offset_ = (pos + 31) / 32 * 32;
    return STT_OK;
}

const GgufTensor* GgufFile::find(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

const uint8_t* GgufFile::tensor_data(const GgufTensor& t, std::vector<uint8_t>& scratch) const {
    const uint64_t abs = data_offset_ + t.offset;
    if (abs < data_offset_ || abs > total_ || t.nbytes > total_ - abs) {
        set_error(STT_E_FORMAT, "tensor '%s' data (%llu bytes at %llu) runs past the end of the file (%llu bytes)",
                  t.name.c_str(), (unsigned long long)t.nbytes, (unsigned long long)abs, (unsigned long long)total_);
        return nullptr;
    }
    if (t.nbytes == 0) return ptr_.empty() ? nullptr : ptr_[0];
    size_t s = std::upper_bound(end_.begin(), end_.end(), abs) - end_.begin();
    const uint64_t start = s == 0 ? 0 : end_[s - 1];
    if (abs + t.nbytes <= end_[s]) return ptr_[s] + (abs - start);
    scratch.resize(t.nbytes);
    read(abs, scratch.data(), t.nbytes);
    return scratch.data();
}

}  // namespace stt
