// SentencePiece detokeniser: the step after the decode path.  Token ids that the stream API
// emits become UTF-8 text with the rules of the reference's SpmDecoder
// (crates/stt-wasm/src/tokenizer.rs:7-192).  Host-only: it needs no device and is not part of
// the decode step's timing.
//
// The vocabulary is read from a SentencePiece `.model` protobuf: every field-1 entry (a
// SentencePiece message) of the ModelProto gives, in order, the piece of the next token id;
// inside it, the last field-1 string is the piece (tokenizer.rs:44-96).  Each piece is
// classified once at load: a byte-fallback piece "<0xHH>" keeps its byte value, every other
// piece its UTF-8 text, so decoding is a single pass over the ids.
#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "common.h"

namespace {

// A protobuf base-128 varint from buf[pos..], as tokenizer.rs:98-115 reads it: it stops at the
// first byte without the continuation bit or at the end of the buffer, and the shift of a group
// past the 64th bit wraps modulo 64 (the reference's release build).
uint64_t read_varint(const uint8_t* buf, size_t size, size_t pos, size_t* consumed) {
    uint64_t value = 0;
    unsigned shift = 0;
    size_t p = pos;
    while (p < size) {
        uint8_t b = buf[p++];
        value |= (uint64_t)(b & 0x7Fu) << (shift & 63u);
        shift += 7;
        if ((b & 0x80u) == 0) break;
    }
    *consumed = p - pos;
    return value;
}

// Position after a field of `wire_type` whose payload starts at `pos` (tokenizer.rs:117-136).
// Unknown wire types advance by one byte.  The result may lie past the end of the buffer,
// which ends the caller's loop.
size_t skip_field(const uint8_t* buf, size_t size, size_t pos, unsigned wire_type) {
    switch (wire_type) {
        case 0: {
            size_t p = pos;
            while (p < size && (buf[p] & 0x80u)) ++p;
            return p + 1;
        }
        case 1: return pos + 8;
        case 2: {
            size_t used;
            uint64_t len = read_varint(buf, size, pos, &used);
            size_t after = pos + used;
            return len > (uint64_t)(size - (after < size ? after : size)) ? size : after + (size_t)len;
        }
        case 5: return pos + 4;
        default: return pos + 1;
    }
}

// Appends bytes as UTF-8, replacing each maximal ill-formed subsequence by U+FFFD: Rust's
// String::from_utf8_lossy (tokenizer.rs:90), which follows the Unicode Standard's
// "substitution of maximal subparts" (chapter 3, U+FFFD substitution).
void append_utf8_lossy(std::string& out, const uint8_t* s, size_t n) {
    static const char kReplacement[] = "\xEF\xBF\xBD";
    size_t i = 0;
    while (i < n) {
        uint8_t b = s[i];
        if (b < 0x80) { out.push_back((char)b); ++i; continue; }
        size_t need;
        uint8_t lo = 0x80, hi = 0xBF;   // bounds of the second byte
        if (b >= 0xC2 && b <= 0xDF) need = 1;
        else if (b == 0xE0) { need = 2; lo = 0xA0; }
        else if (b >= 0xE1 && b <= 0xEC) need = 2;
        else if (b == 0xED) { need = 2; hi = 0x9F; }
        else if (b >= 0xEE && b <= 0xEF) need = 2;
        else if (b == 0xF0) { need = 3; lo = 0x90; }
        else if (b >= 0xF1 && b <= 0xF3) need = 3;
        else if (b == 0xF4) { need = 3; hi = 0x8F; }
        else { out.append(kReplacement, 3); ++i; continue; }   // 0x80-0xC1, 0xF5-0xFF
        size_t j = 1;
        bool ok = true;
        for (; j <= need; ++j) {
            if (i + j >= n) { ok = false; break; }
            uint8_t c = s[i + j];
            uint8_t l = (j == 1) ? lo : 0x80, h = (j == 1) ? hi : 0xBF;
            if (c < l || c > h) { ok = false; break; }
        }
        if (ok) { out.append((const char*)s + i, need + 1); i += need + 1; }
        else { out.append(kReplacement, 3); i += j; }   // the valid prefix (lead + j-1 bytes) is one subpart
    }
}

bool valid_utf8(const std::string& s) {
    std::string tmp;
    tmp.reserve(s.size());
    append_utf8_lossy(tmp, (const uint8_t*)s.data(), s.size());
    return tmp == s;   // no replacement was made: well-formed
}

int hex_digit(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
}

// Byte value of a byte-fallback piece, else -1 (tokenizer.rs:166-171): six bytes, "<0x" ... ">",
// and the two characters between parse as a base-16 u8 — Rust's u8::from_str_radix, which also
// takes a leading '+' before a single digit.
int byte_fallback_value(const std::string& p) {
    if (p.size() != 6 || p.compare(0, 3, "<0x") != 0 || p[5] != '>') return -1;
    if (p[3] == '+') return hex_digit(p[4]);
    int h = hex_digit(p[3]), l = hex_digit(p[4]);
    return (h < 0 || l < 0) ? -1 : h * 16 + l;
}

}  // namespace

struct stt_spm_decoder {
    std::vector<std::string> pieces;   // token id -> piece text (UTF-8, lossily decoded)
    std::vector<int16_t> byte_value;   // token id -> byte of a "<0xHH>" piece, or -1
};

namespace {

// The ModelProto walk of tokenizer.rs:44-72 and the SentencePiece message of :74-96.  A piece
// whose declared length runs past its buffer is a format error here (the reference's slice
// index panics there).
int parse_vocab(const uint8_t* data, size_t size, stt_spm_decoder* d) {
    size_t pos = 0;
    while (pos < size) {
        size_t used;
        uint64_t tag = read_varint(data, size, pos, &used);
        pos += used;
        unsigned field = (unsigned)(tag >> 3), wire = (unsigned)(tag & 7u);
        if (field == 1 && wire == 2) {
            uint64_t len = read_varint(data, size, pos, &used);
            pos += used;
            if (pos > size || len > (uint64_t)(size - pos))
                return stt::set_error(STT_E_FORMAT, "SentencePiece entry %zu: length %llu runs past the model (%zu bytes left)",
                                      d->pieces.size(), (unsigned long long)len, pos > size ? (size_t)0 : size - pos);
            const uint8_t* msg = data + pos;
            size_t msize = (size_t)len, mp = 0;
            std::string piece;
            while (mp < msize) {
                uint64_t t = read_varint(msg, msize, mp, &used);
                mp += used;
                unsigned f = (unsigned)(t >> 3), w = (unsigned)(t & 7u);
                if (f == 1 && w == 2) {
                    uint64_t plen = read_varint(msg, msize, mp, &used);
                    mp += used;
                    if (mp > msize || plen > (uint64_t)(msize - mp))
                        return stt::set_error(STT_E_FORMAT, "SentencePiece entry %zu: piece length %llu runs past its entry",
                                              d->pieces.size(), (unsigned long long)plen);
                    piece.clear();
                    append_utf8_lossy(piece, msg + mp, (size_t)plen);
                    mp += (size_t)plen;
                } else {
                    mp = skip_field(msg, msize, mp, w);
                }
            }
            d->pieces.push_back(piece);
            d->byte_value.push_back((int16_t)byte_fallback_value(piece));
            pos += (size_t)len;
        } else {
            pos = skip_field(data, size, pos, wire);
        }
    }
    return STT_OK;
}

// tokenizer.rs:150-192: skip ids 0 (end of stream) and 3 (padding) and ids past the vocabulary;
// collect consecutive byte-fallback bytes and emit them only if they form valid UTF-8 (an
// invalid run is dropped whole); join the pieces and turn U+2581 into a space.  No trimming:
// the leading space marks a word boundary for per-token streaming.
std::string decode_ids(const stt_spm_decoder* d, const uint32_t* ids, size_t n) {
    std::string text, bytes;
    auto flush = [&]() {
        if (!bytes.empty()) {
            if (valid_utf8(bytes)) text += bytes;
            bytes.clear();
        }
    };
    for (size_t i = 0; i < n; ++i) {
        uint32_t id = ids[i];
        if (id == 0 || id == 3 || id >= d->pieces.size()) continue;
        int bv = d->byte_value[id];
        if (bv >= 0) { bytes.push_back((char)bv); continue; }
        flush();
        text += d->pieces[id];
    }
    flush();
    std::string out;
    out.reserve(text.size());
    for (size_t i = 0; i < text.size(); ++i) {
        if (i + 2 < text.size() && (uint8_t)text[i] == 0xE2 && (uint8_t)text[i + 1] == 0x96 &&
            (uint8_t)text[i + 2] == 0x81) {
            out.push_back(' ');
            i += 2;
        } else {
            out.push_back(text[i]);
        }
    }
    return out;
}

int copy_out(const std::string& s, char* out, size_t cap, size_t* len, const char* what) {
    *len = s.size();
    if (!out) return STT_OK;   // size query
    if (cap < s.size() + 1)
        return stt::set_error(STT_E_INVALID_ARG, "%s: %zu bytes and a terminating NUL do not fit in %zu", what,
                              s.size(), cap);
    std::memcpy(out, s.data(), s.size());
    out[s.size()] = '\0';
    return STT_OK;
}

}  // namespace

extern "C" {

int stt_spm_decoder_create(const uint8_t* model_bytes, size_t n_bytes, stt_spm_decoder** out) {
    if (!out) return stt::set_error(STT_E_INVALID_ARG, "stt_spm_decoder_create: out is NULL");
    *out = nullptr;
    if (!model_bytes && n_bytes) return stt::set_error(STT_E_INVALID_ARG, "stt_spm_decoder_create: model bytes are NULL");
    stt_spm_decoder* d = new (std::nothrow) stt_spm_decoder();
    if (!d) return stt::set_error(STT_E_OOM, "stt_spm_decoder_create: out of host memory");
    int rc;
    try {
        rc = parse_vocab(model_bytes, n_bytes, d);
    } catch (const std::bad_alloc&) {
        rc = stt::set_error(STT_E_OOM, "stt_spm_decoder_create: out of host memory");
    }
    if (rc != STT_OK) { delete d; return rc; }
    *out = d;
    stt::clear_error();
    return STT_OK;
}

int stt_spm_decoder_destroy(stt_spm_decoder* dec) {
    delete dec;
    return STT_OK;
}

int stt_spm_vocab_len(const stt_spm_decoder* dec, int64_t* out) {
    if (!dec || !out) return stt::set_error(STT_E_INVALID_ARG, "stt_spm_vocab_len: NULL argument");
    *out = (int64_t)dec->pieces.size();
    return STT_OK;
}

int stt_spm_piece(const stt_spm_decoder* dec, int64_t id, char* out, size_t cap, size_t* len) {
    if (!dec || !len) return stt::set_error(STT_E_INVALID_ARG, "stt_spm_piece: NULL argument");
    if (id < 0 || (uint64_t)id >= dec->pieces.size())
        return stt::set_error(STT_E_INVALID_ARG, "stt_spm_piece: id %lld outside the vocabulary of %zu pieces",
                              (long long)id, dec->pieces.size());
    return copy_out(dec->pieces[(size_t)id], out, cap, len, "stt_spm_piece");
}

int stt_spm_decode(const stt_spm_decoder* dec, const uint32_t* ids, size_t n, char* out, size_t cap, size_t* len) {
    if (!dec || !len || (!ids && n)) return stt::set_error(STT_E_INVALID_ARG, "stt_spm_decode: NULL argument");
    try {
        return copy_out(decode_ids(dec, ids, n), out, cap, len, "stt_spm_decode");
    } catch (const std::bad_alloc&) {
        return stt::set_error(STT_E_OOM, "stt_spm_decode: out of host memory");
    }
}

}  // extern "C"
