/*
 * stt_oracle.c — CPU restatement of the stt-web STT-1B decode step.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library and the CPU baseline of bench.py.
 * Nothing in the library links or calls this file.
 *
 * What it restates (paths inside the stt-web project):
 *   crates/stt-wasm/src/gguf.rs      f16_to_f32 (:45-73), GGUF reader (:193-311),
 *                                    EmbeddingStore::embed_id_add_cpu (:616-633), loader (:763-925)
 *   crates/stt-wasm/src/wgsl/shader_naive.wgsl   Q4 matmul, per-output loop order (:30-98)
 *   crates/stt-wasm/src/model.rs     RoPE (:34-123), KVCache ring (:139-296), attention
 *                                    (:426-474), FFN (:517-524), block (:556-571), forward (:631-664)
 *   crates/stt-wasm/src/stream.rs    feed_frame / resolve_pending_as_token / flush / reset
 *   scripts/quantize.py              Q4_0 encoding (:65-116)
 * The Burn operators the reference calls (RmsNorm, softmax, silu, matmul, argmax, cos/sin) live
 * in the un-vendored burn 0.20 crate; they are restated from their textbook definitions:
 *   RmsNorm  y = (x / sqrt(mean(x^2) + eps)) * alpha     (eps 1e-8, gguf.rs:808, 838, 854)
 *   softmax  exp(s - max) / sum(exp(s - max))
 *   silu     x * (1 / (1 + exp(-x)))
 *   argmax   first index of the maximum
 * so parity is pinned at the Q4_0 format and matmul semantics and unpinned at those operators.
 *
 * Arithmetic is f32 with no contraction of a*b+c into fma (built with -ffp-contract=off).
 */
#include "stt_oracle.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static __thread char g_err[512];
static int set_err(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}
const char* orc_last_error(void) { return g_err; }

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
int orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_config_default(orc_config* c) {
    /* SttConfig::default (crates/stt-wasm/src/lib.rs:60-80) */
    c->num_layers = 16;
    c->num_heads = 16;
    c->num_codebooks = 32;
    c->text_delay = 6;
    c->max_seq_len = 4096;
    c->sliding_window = 750;
    c->rope_theta = 100000.0;
    c->text_padding_id = 3;
    c->text_start_token = 8000;
}

/* ------------------------------------------------------------------ scalar conversions */

static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* gguf.rs:45-73, line for line (including its subnormal exponent 127 - (15 + e - 1)). */
float orc_f16_to_f32_gguf(uint16_t bits) {
    uint32_t sign = (bits >> 15) & 1u, exponent = (bits >> 10) & 0x1Fu, mantissa = bits & 0x3FFu;
    if (exponent == 0) {
        if (mantissa == 0) return bits_f32(sign << 31);
        uint32_t e = 1, m = mantissa;
        while ((m & 0x400u) == 0) { m <<= 1; e += 1; }
        m &= 0x3FFu;
        uint32_t f32_exp = 127u - (15u + e - 1u);
        return bits_f32((sign << 31) | (f32_exp << 23) | (m << 13));
    } else if (exponent == 31) {
        return bits_f32((sign << 31) | (0xFFu << 23) | (mantissa << 13));
    }
    return bits_f32((sign << 31) | ((exponent - 15u + 127u) << 23) | (mantissa << 13));
}

/* IEEE binary16 -> binary32, as WGSL unpack2x16float (shader_naive.wgsl:20-23). */
float orc_f16_to_f32_ieee(uint16_t bits) {
    uint32_t sign = (bits >> 15) & 1u, exponent = (bits >> 10) & 0x1Fu, mantissa = bits & 0x3FFu;
    if (exponent == 0 && mantissa != 0) {
        float v = ldexpf((float)mantissa, -24);
        return sign ? -v : v;
    }
    return orc_f16_to_f32_gguf(bits);
}

static uint16_t f32_to_bf16_rne(float f) {
    uint32_t x = f32_bits(f);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}
static float round_bf16(float f) { return bits_f32((uint32_t)f32_to_bf16_rne(f) << 16); }

/* numpy.float16(x) for finite f32 x: round to nearest even, subnormals, overflow to inf. */
static uint16_t f32_to_f16_rne(float f) {
    uint32_t x = f32_bits(f), sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
    if (ax < 0x38800000u) {
        /* subnormal half: value / 2^-24 rounded half to even */
        double q = ldexp((double)fabsf(f), 24);
        double r = nearbyint(q);
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t e = (ax >> 23) - 112u, m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/* ------------------------------------------------------------------ Q4_0 */

/* scripts/quantize.py:88-114 (numpy 2 arithmetic: everything in float32). */
void orc_quantize_q4_0(const float* x, size_t n, uint8_t* out) {
    for (size_t b = 0; b < n / 32; ++b) {
        const float* block = x + b * 32;
        uint8_t* o = out + b * 18;
        float abs_max = 0.0f;
        for (int j = 0; j < 32; ++j) {
            float a = fabsf(block[j]);
            if (a > abs_max) abs_max = a;
        }
        float scale = abs_max > 0.0f ? abs_max / 7.0f : 1.0f;
        int q[32];
        for (int j = 0; j < 32; ++j) {
            int v = (int)nearbyintf(block[j] / scale);
            q[j] = v < -8 ? -8 : (v > 7 ? 7 : v);
        }
        uint16_t h = f32_to_f16_rne(scale);
        o[0] = (uint8_t)(h & 0xFF);
        o[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < 16; ++j) {
            int v_lo = (q[j] + 8) & 0x0F, v_hi = (q[j + 16] + 8) & 0x0F;
            o[2 + j] = (uint8_t)((v_hi << 4) | v_lo);
        }
    }
}

void orc_dequant_q4_0(const uint8_t* raw, int64_t rows, int64_t k, float* out) {
    const int64_t nb = k / 32;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t* blk = raw + (r * nb + b) * 18;
            float d = orc_f16_to_f32_ieee((uint16_t)(blk[0] | (blk[1] << 8)));
            float* o = out + r * k + b * 32;
            for (int j = 0; j < 16; ++j) {
                uint8_t byte = blk[2 + j];
                o[j] = ((float)(byte & 0x0F) - 8.0f) * d;
                o[j + 16] = ((float)((byte >> 4) & 0x0F) - 8.0f) * d;
            }
        }
}

/* gguf.rs:616-633 */
void orc_embed_id_add_q4(const uint8_t* table, int64_t dim, uint32_t id, float* out_buf) {
    const int64_t blocks_per_row = dim / 32, bytes_per_row = blocks_per_row * 18;
    const uint8_t* row_bytes = table + (int64_t)id * bytes_per_row;
    for (int64_t block = 0; block < blocks_per_row; ++block) {
        const int64_t bo = block * 18;
        float d = orc_f16_to_f32_gguf((uint16_t)(row_bytes[bo] | (row_bytes[bo + 1] << 8)));
        const int64_t base = block * 32;
        for (int j = 0; j < 16; ++j) {
            uint8_t byte = row_bytes[bo + 2 + j];
            out_buf[base + j] += ((float)(byte & 0x0F) - 8.0f) * d;
            out_buf[base + j + 16] += ((float)((byte >> 4) & 0x0F) - 8.0f) * d;
        }
    }
}

/* WGSL dot(vec4, vec4): ((a.x*b.x + a.y*b.y) + a.z*b.z) + a.w*b.w */
static inline float dot4(const float* a, const float* b) {
    float s = a[0] * b[0];
    s = s + a[1] * b[1];
    s = s + a[2] * b[2];
    s = s + a[3] * b[3];
    return s;
}

/* One output of shader_naive.wgsl:main — the block loop :51-95. */
static float q4_row_dot(const uint8_t* row, int64_t blocks_per_row, const float* input, uint32_t flags) {
    float acc = 0.0f;
    for (int64_t blk = 0; blk < blocks_per_row; ++blk) {
        const uint8_t* b = row + blk * 18;
        const float scale = orc_f16_to_f32_ieee((uint16_t)(b[0] | (b[1] << 8)));
        const int64_t k_base = blk * 32;
        for (int wi = 0; wi < 4; ++wi) {
            const uint8_t* p = b + 2 + wi * 4;
            float w_lo[4], w_hi[4], in_lo[4], in_hi[4];
            for (int i = 0; i < 4; ++i) {
                w_lo[i] = ((float)(p[i] & 0x0F) - 8.0f) * scale;
                w_hi[i] = ((float)((p[i] >> 4) & 0x0F) - 8.0f) * scale;
                in_lo[i] = input[k_base + wi * 4 + i];
                in_hi[i] = input[k_base + 16 + wi * 4 + i];
                if (flags & ORC_GEMM_BF16) {
                    w_lo[i] = round_bf16(w_lo[i]);
                    w_hi[i] = round_bf16(w_hi[i]);
                    in_lo[i] = round_bf16(in_lo[i]);
                    in_hi[i] = round_bf16(in_hi[i]);
                }
            }
            acc += dot4(w_lo, in_lo);
            acc += dot4(w_hi, in_hi);
        }
    }
    return acc;
}

void orc_q4_matmul(const uint8_t* w, int64_t n, int64_t k, const float* in, int64_t m, float* out,
                   uint32_t flags) {
    const int64_t nb = k / 32;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n * m; ++i) {
        const int64_t r = i / n, c = i % n;
        out[r * n + c] = q4_row_dot(w + c * nb * 18, nb, in + r * k, flags);
    }
}

/* ------------------------------------------------------------------ GGUF (gguf.rs:193-311) */

typedef struct {
    char name[128];
    int32_t ndims;
    uint64_t dims[8];
    uint32_t dtype;
    uint64_t offset, numel, nbytes;
} orc_tensor;

typedef struct {
    const uint8_t* buf;
    size_t len, pos;
    int ok;
} rdr;

static uint64_t rd(rdr* r, int n) {
    uint64_t v = 0;
    if (r->pos + (size_t)n > r->len) { r->ok = 0; return 0; }
    for (int i = 0; i < n; ++i) v |= (uint64_t)r->buf[r->pos + i] << (8 * i);
    r->pos += (size_t)n;
    return v;
}
static void rd_skip(rdr* r, uint64_t n) {
    if (n > r->len - r->pos) { r->ok = 0; return; }
    r->pos += n;
}
static int skip_value(rdr* r, uint32_t t, int depth) {
    static const int fixed[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (t > 12 || depth > 8) return 0;
    if (t == 8) { uint64_t n = rd(r, 8); rd_skip(r, n); return r->ok; }
    if (t == 9) {
        uint32_t et = (uint32_t)rd(r, 4);
        uint64_t cnt = rd(r, 8);
        for (uint64_t i = 0; i < cnt && r->ok; ++i)
            if (!skip_value(r, et, depth + 1)) return 0;
        return r->ok;
    }
    rd_skip(r, (uint64_t)fixed[t]);
    return r->ok;
}

static uint64_t dtype_bytes(uint32_t dt, uint64_t n) {
    switch (dt) {
        case 0: return n * 4;
        case 1: case 30: return n * 2;
        case 2: return n / 32 * 18;
        default: return (uint64_t)-1;
    }
}

/* ------------------------------------------------------------------ model */

typedef struct {
    float* norm1;
    float* norm2;
    const uint8_t *in_proj, *out_proj, *lin_in, *lin_out; /* raw Q4_0 rows */
} orc_layer;

struct orc_model {
    orc_config cfg;
    int32_t D, H, HD, F, V, TV, AV;
    uint32_t emb_dtype;
    const uint8_t* emb_audio[64];
    const uint8_t* emb_text;
    orc_layer* layers;
    float* out_norm;
    const uint8_t* head;
    float *rope_cos, *rope_sin; /* [max_seq_len][HD/2] */
    float attn_scale;
};

struct orc_stream {
    const orc_model* m;
    uint32_t flags;
    int32_t max_len;
    float *k, *v; /* [L][H][max_len][HD] */
    int32_t offset, len, write_pos;
    int32_t frame_count;
    uint32_t last_text_token;
    uint32_t delay_prev[2];
    /* scratch */
    float *x, *xn, *qkv, *attn, *tmp, *hid, *gate, *scores, *logits;
};

static const orc_tensor* find_t(const orc_tensor* ts, uint64_t n, const char* name) {
    const orc_tensor* hit = NULL;
    for (uint64_t i = 0; i < n; ++i)
        if (strcmp(ts[i].name, name) == 0) hit = &ts[i]; /* last entry wins, like the HashMap */
    return hit;
}

static float* load_norm(const uint8_t* data, const orc_tensor* t, int32_t D) {
    if (!t || (t->dtype != 0 && t->dtype != 1) || t->numel != (uint64_t)D) return NULL;
    float* a = (float*)malloc(sizeof(float) * D);
    for (int32_t i = 0; i < D; ++i) {
        if (t->dtype == 0) { uint32_t u; memcpy(&u, data + t->offset + 4 * i, 4); a[i] = bits_f32(u); }
        else a[i] = orc_f16_to_f32_gguf((uint16_t)(data[t->offset + 2 * i] | (data[t->offset + 2 * i + 1] << 8)));
    }
    return a;
}

int orc_model_load(const uint8_t* gguf, size_t len, const orc_config* cfg_in, orc_model** out) {
    orc_config cfg;
    if (cfg_in) cfg = *cfg_in; else orc_config_default(&cfg);
    rdr r = {gguf, len, 0, 1};
    if (rd(&r, 4) != 0x46554747u) return set_err(-2, "bad magic");
    uint32_t ver = (uint32_t)rd(&r, 4);
    if (ver != 2 && ver != 3) return set_err(-2, "bad version %u", ver);
    uint64_t nt = rd(&r, 8), nm = rd(&r, 8);
    for (uint64_t i = 0; i < nm && r.ok; ++i) {
        uint64_t kl = rd(&r, 8);
        rd_skip(&r, kl);
        uint32_t vt = (uint32_t)rd(&r, 4);
        if (!skip_value(&r, vt, 0)) return set_err(-2, "bad metadata");
    }
    if (!r.ok || nt > 100000) return set_err(-2, "truncated header");
    orc_tensor* ts = (orc_tensor*)calloc(nt ? nt : 1, sizeof(orc_tensor));
    for (uint64_t i = 0; i < nt && r.ok; ++i) {
        uint64_t nl = rd(&r, 8);
        if (nl >= sizeof ts[i].name || r.pos + nl > len) { free(ts); return set_err(-2, "bad name"); }
        memcpy(ts[i].name, gguf + r.pos, nl);
        r.pos += nl;
        ts[i].ndims = (int32_t)rd(&r, 4);
        if (ts[i].ndims > 8) { free(ts); return set_err(-2, "ndims"); }
        ts[i].numel = 1;
        for (int d = 0; d < ts[i].ndims; ++d) { ts[i].dims[d] = rd(&r, 8); ts[i].numel *= ts[i].dims[d]; }
        ts[i].dtype = (uint32_t)rd(&r, 4);
        ts[i].offset = rd(&r, 8);
        ts[i].nbytes = dtype_bytes(ts[i].dtype, ts[i].numel);
        if (ts[i].nbytes == (uint64_t)-1) { int rc = set_err(-2, "dtype %u", ts[i].dtype); free(ts); return rc; }
    }
    if (!r.ok) { free(ts); return set_err(-2, "truncated tensor index"); }
    const uint64_t data_off = (r.pos + 31) / 32 * 32;
    for (uint64_t i = 0; i < nt; ++i) {
        ts[i].offset += data_off; /* absolute from here on */
        if (ts[i].offset > len || ts[i].nbytes > len - ts[i].offset) {
            int rc = set_err(-2, "tensor %s truncated", ts[i].name);
            free(ts);
            return rc;
        }
    }

    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->cfg = cfg;
    char name[160];
    const orc_tensor* t = find_t(ts, nt, "text_linear.weight");
    if (!t || t->dtype != 2 || t->ndims != 2) { free(ts); free(m); return set_err(-2, "text_linear"); }
    m->D = (int32_t)t->dims[0];
    m->V = (int32_t)t->dims[1];
    m->head = gguf + t->offset;
    m->H = cfg.num_heads;
    m->HD = m->D / m->H;
    t = find_t(ts, nt, "text_emb.weight");
    if (!t) { free(ts); free(m); return set_err(-2, "text_emb"); }
    m->TV = (int32_t)t->dims[1];
    m->emb_dtype = t->dtype;
    m->emb_text = gguf + t->offset;
    for (int i = 0; i < cfg.num_codebooks; ++i) {
        snprintf(name, sizeof name, "emb.%d.weight", i);
        t = find_t(ts, nt, name);
        if (!t || t->dtype != m->emb_dtype) { free(ts); free(m); return set_err(-2, "%s", name); }
        m->AV = (int32_t)t->dims[1];
        m->emb_audio[i] = gguf + t->offset;
    }
    m->layers = (orc_layer*)calloc((size_t)cfg.num_layers, sizeof(orc_layer));
    for (int l = 0; l < cfg.num_layers; ++l) {
        orc_layer* L = &m->layers[l];
#define GETQ(field, suffix)                                                                 \
        snprintf(name, sizeof name, "transformer.layers.%d.%s", l, suffix);                 \
        t = find_t(ts, nt, name);                                                           \
        if (!t || t->dtype != 2) { free(ts); orc_model_free(m); return set_err(-2, "%s", name); } \
        L->field = gguf + t->offset;
        GETQ(in_proj, "self_attn.in_proj_weight")
        GETQ(out_proj, "self_attn.out_proj.weight")
        GETQ(lin_in, "gating.linear_in.weight")
        GETQ(lin_out, "gating.linear_out.weight")
        m->F = (int32_t)(t->dims[0]);
#undef GETQ
        snprintf(name, sizeof name, "transformer.layers.%d.norm1.alpha", l);
        L->norm1 = load_norm(gguf, find_t(ts, nt, name), m->D);
        snprintf(name, sizeof name, "transformer.layers.%d.norm2.alpha", l);
        L->norm2 = load_norm(gguf, find_t(ts, nt, name), m->D);
        if (!L->norm1 || !L->norm2) { free(ts); orc_model_free(m); return set_err(-2, "norm %d", l); }
    }
    m->out_norm = load_norm(gguf, find_t(ts, nt, "out_norm.alpha"), m->D);
    free(ts);
    if (!m->out_norm) { orc_model_free(m); return set_err(-2, "out_norm"); }

    /* RoPE::new (model.rs:34-59): f32 inverse frequencies, f32 angles, cos/sin. */
    const int half = m->HD / 2;
    m->rope_cos = (float*)malloc(sizeof(float) * (size_t)cfg.max_seq_len * half);
    m->rope_sin = (float*)malloc(sizeof(float) * (size_t)cfg.max_seq_len * half);
    float* inv_freq = (float*)malloc(sizeof(float) * half);
    for (int i = 0; i < half; ++i)
        inv_freq[i] = 1.0f / powf((float)cfg.rope_theta, (float)(2 * i) / (float)m->HD);
    for (int p = 0; p < cfg.max_seq_len; ++p)
        for (int j = 0; j < half; ++j) {
            float f = (float)p * inv_freq[j];
            m->rope_cos[(size_t)p * half + j] = cosf(f);
            m->rope_sin[(size_t)p * half + j] = sinf(f);
        }
    free(inv_freq);
    m->attn_scale = powf((float)m->HD, -0.5f); /* model.rs:411 */
    *out = m;
    return 0;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    if (m->layers) {
        for (int l = 0; l < m->cfg.num_layers; ++l) { free(m->layers[l].norm1); free(m->layers[l].norm2); }
        free(m->layers);
    }
    free(m->out_norm);
    free(m->rope_cos);
    free(m->rope_sin);
    free(m);
}

int orc_model_dims(const orc_model* m, int32_t* hidden, int32_t* ffn, int32_t* vocab, int32_t* text_vocab) {
    *hidden = m->D; *ffn = m->F; *vocab = m->V; *text_vocab = m->TV;
    return 0;
}

orc_stream* orc_stream_new(const orc_model* m, uint32_t flags) {
    orc_stream* s = (orc_stream*)calloc(1, sizeof(orc_stream));
    s->m = m;
    s->flags = flags;
    s->max_len = m->cfg.sliding_window + 1; /* model.rs:730 */
    const size_t kv = (size_t)m->cfg.num_layers * m->H * s->max_len * m->HD;
    s->k = (float*)calloc(kv, sizeof(float));
    s->v = (float*)calloc(kv, sizeof(float));
    s->x = (float*)calloc((size_t)m->D, 4);
    s->xn = (float*)calloc((size_t)m->D, 4);
    s->qkv = (float*)calloc((size_t)3 * m->D, 4);
    s->attn = (float*)calloc((size_t)m->D, 4);
    s->tmp = (float*)calloc((size_t)m->D, 4);
    s->hid = (float*)calloc((size_t)2 * m->F, 4);
    s->gate = (float*)calloc((size_t)m->F, 4);
    s->scores = (float*)calloc((size_t)s->max_len, 4);
    s->logits = (float*)calloc((size_t)m->V, 4);
    orc_stream_reset(s);
    return s;
}

void orc_stream_free(orc_stream* s) {
    if (!s) return;
    free(s->k); free(s->v); free(s->x); free(s->xn); free(s->qkv); free(s->attn); free(s->tmp);
    free(s->hid); free(s->gate); free(s->scores); free(s->logits);
    free(s);
}

/* SttStream::reset (stream.rs:341-349) with KVCache::reset (model.rs:233-239). */
void orc_stream_reset(orc_stream* s) {
    s->offset = 0;
    s->len = 0;
    s->write_pos = 0;
    s->frame_count = 0;
    s->last_text_token = s->m->cfg.text_start_token;
    s->delay_prev[0] = s->delay_prev[1] = 0xFFFFFFFFu;
}

void orc_stream_state(const orc_stream* s, int64_t out[7]) {
    out[0] = s->offset; out[1] = s->len; out[2] = s->write_pos; out[3] = s->frame_count;
    out[4] = s->last_text_token; out[5] = s->delay_prev[0]; out[6] = s->delay_prev[1];
}
void orc_stream_set_last_text_token(orc_stream* s, uint32_t token) { s->last_text_token = token; }

/* RmsNorm (burn::nn::RmsNorm via model.rs:365-373): (x / sqrt(mean(x^2) + eps)) * alpha. */
static void rmsnorm(const float* x, const float* alpha, int32_t n, float* y) {
    float ss = 0.0f;
    for (int32_t i = 0; i < n; ++i) ss += x[i] * x[i];
    const float rms = sqrtf(ss / (float)n + 1e-8f);
    for (int32_t i = 0; i < n; ++i) y[i] = (x[i] / rms) * alpha[i];
}

/* Embedding row of table `t` added to out (gguf.rs:616-633 for Q4_0; exact widening otherwise). */
static void embed_add(const orc_model* m, const uint8_t* t, uint32_t id, float* out) {
    const int32_t D = m->D;
    switch (m->emb_dtype) {
        case 2: orc_embed_id_add_q4(t, D, id, out); break;
        case 0: {
            const float* row = (const float*)(t + (size_t)id * D * 4);
            for (int32_t j = 0; j < D; ++j) out[j] += row[j];
            break;
        }
        case 30: {
            const uint16_t* row = (const uint16_t*)(t + (size_t)id * D * 2);
            for (int32_t j = 0; j < D; ++j) out[j] += bits_f32((uint32_t)row[j] << 16);
            break;
        }
        case 1: {
            const uint16_t* row = (const uint16_t*)(t + (size_t)id * D * 2);
            for (int32_t j = 0; j < D; ++j) out[j] += orc_f16_to_f32_ieee(row[j]);
            break;
        }
    }
}

/* RoPE::apply_rotation (model.rs:86-123) on one head vector at position `pos`. */
static void rope_rotate(const orc_model* m, float* x, int32_t pos) {
    const int half = m->HD / 2;
    const float* c = m->rope_cos + (size_t)pos * half;
    const float* s = m->rope_sin + (size_t)pos * half;
    for (int i = 0; i < half; ++i) {
        const float xr = x[2 * i], xi = x[2 * i + 1];
        x[2 * i] = xr * c[i] - xi * s[i];
        x[2 * i + 1] = xr * s[i] + xi * c[i];
    }
}

static float silu(float x) { return x * (1.0f / (1.0f + expf(-x))); }

/* Q4TransformerBlock::forward_with_cache (model.rs:556-571) with Q4Attention (model.rs:426-474)
 * and Q4FeedForward (model.rs:517-524) for one layer. */
static void block_forward(orc_stream* s, int l) {
    const orc_model* m = s->m;
    const orc_layer* L = &m->layers[l];
    const int32_t D = m->D, H = m->H, HD = m->HD, F = m->F, ML = s->max_len;
    const uint32_t gf = s->flags & ORC_GEMM_BF16;
    float* x = s->x;

    rmsnorm(x, L->norm1, D, s->xn);
    orc_q4_matmul(L->in_proj, 3 * D, D, s->xn, 1, s->qkv, gf);
    float *q = s->qkv, *k = s->qkv + D, *v = s->qkv + 2 * D;
    const int32_t offset = s->offset;
    for (int h = 0; h < H; ++h) {
        rope_rotate(m, q + h * HD, offset);
        rope_rotate(m, k + h * HD, offset);
    }
    /* KVCache::update (model.rs:176-222): write at write_pos, advance the ring. */
    const int32_t pos = s->write_pos;
    for (int h = 0; h < H; ++h) {
        float* kd = s->k + (((size_t)l * H + h) * ML + pos) * HD;
        float* vd = s->v + (((size_t)l * H + h) * ML + pos) * HD;
        for (int d = 0; d < HD; ++d) {
            kd[d] = (s->flags & ORC_KV_BF16) ? round_bf16(k[h * HD + d]) : k[h * HD + d];
            vd[d] = (s->flags & ORC_KV_BF16) ? round_bf16(v[h * HD + d]) : v[h * HD + d];
        }
    }
    const int32_t len = s->len + 1 < ML ? s->len + 1 : ML;
    /* scores = (q . k^T) * scale; softmax; attn . v   (model.rs:455-469; masks are no-ops at
     * q_len == 1, model.rs:309-311, 338-340) */
    for (int h = 0; h < H; ++h) {
        const float* qh = q + h * HD;
        const float* kb = s->k + ((size_t)l * H + h) * ML * HD;
        const float* vb = s->v + ((size_t)l * H + h) * ML * HD;
        float mx = -INFINITY;
        for (int32_t j = 0; j < len; ++j) {
            float dot = 0.0f;
            for (int d = 0; d < HD; ++d) dot += qh[d] * kb[(size_t)j * HD + d];
            s->scores[j] = dot * m->attn_scale;
            if (s->scores[j] > mx) mx = s->scores[j];
        }
        float sum = 0.0f;
        for (int32_t j = 0; j < len; ++j) { s->scores[j] = expf(s->scores[j] - mx); sum += s->scores[j]; }
        for (int32_t j = 0; j < len; ++j) s->scores[j] = s->scores[j] / sum;
        for (int d = 0; d < HD; ++d) {
            float acc = 0.0f;
            for (int32_t j = 0; j < len; ++j) acc += s->scores[j] * vb[(size_t)j * HD + d];
            s->attn[h * HD + d] = acc;
        }
    }
    orc_q4_matmul(L->out_proj, D, D, s->attn, 1, s->tmp, gf);
    for (int32_t i = 0; i < D; ++i) x[i] = s->tmp[i] + x[i];

    rmsnorm(x, L->norm2, D, s->xn);
    orc_q4_matmul(L->lin_in, 2 * F, D, s->xn, 1, s->hid, gf);
    for (int32_t i = 0; i < F; ++i) s->gate[i] = silu(s->hid[i]) * s->hid[F + i];
    orc_q4_matmul(L->lin_out, D, F, s->gate, 1, s->tmp, gf);
    for (int32_t i = 0; i < D; ++i) x[i] = s->tmp[i] + x[i];
}

int64_t orc_forward(orc_stream* s, const uint32_t* audio, uint32_t text, float* logits) {
    const orc_model* m = s->m;
    if (s->offset + 1 > m->cfg.max_seq_len)
        return set_err(-6, "position %d beyond the RoPE table (%d)", s->offset, m->cfg.max_seq_len);
    for (int i = 0; i < m->cfg.num_codebooks; ++i)
        if (audio[i] >= (uint32_t)m->AV) return set_err(-1, "audio token %u out of range", audio[i]);
    if (text >= (uint32_t)m->TV) return set_err(-1, "text token %u out of range", text);
    /* embedding sum on the CPU in codebook order, then the text row (model.rs:640-646) */
    memset(s->x, 0, sizeof(float) * (size_t)m->D);
    for (int i = 0; i < m->cfg.num_codebooks; ++i) embed_add(m, m->emb_audio[i], audio[i], s->x);
    embed_add(m, m->emb_text, text, s->x);
    for (int l = 0; l < m->cfg.num_layers; ++l) block_forward(s, l);
    s->write_pos = (s->write_pos + 1) % s->max_len;
    s->offset += 1;
    s->len = s->len + 1 < s->max_len ? s->len + 1 : s->max_len;
    rmsnorm(s->x, m->out_norm, m->D, s->xn);
    orc_q4_matmul(m->head, m->V, m->D, s->xn, 1, s->logits, s->flags & ORC_GEMM_BF16);
    if (logits) memcpy(logits, s->logits, sizeof(float) * (size_t)m->V);
    int64_t best = 0;
    for (int32_t i = 1; i < m->V; ++i)
        if (s->logits[i] > s->logits[best]) best = i;
    return best;
}

int64_t orc_feed_frame(orc_stream* s, const uint32_t* audio) {
    const orc_config* c = &s->m->cfg;
    /* submit_frame (stream.rs:90-107) */
    s->frame_count += 1;
    const int emits = s->frame_count >= c->text_delay;
    int64_t tok = orc_forward(s, audio, s->last_text_token, NULL);
    if (tok < 0) return tok - 100; /* keep errors below -1 */
    const uint32_t token = (uint32_t)tok;
    /* resolve_pending_as_token (stream.rs:231-266) */
    if (emits) {
        s->last_text_token = token;
        return token;
    }
    const uint32_t prev0 = s->delay_prev[0], prev1 = s->delay_prev[1];
    s->delay_prev[0] = prev1;
    s->delay_prev[1] = token;
    if (token != c->text_padding_id && token != 0 && token == prev0 && token != prev1)
        s->last_text_token = c->text_padding_id;
    else
        s->last_text_token = token;
    return -1;
}

int orc_flush(orc_stream* s, uint32_t* tokens, int capacity) {
    uint32_t zero[64] = {0};
    int n = 0;
    for (int i = 0; i < s->m->cfg.text_delay; ++i) {
        int64_t t = orc_feed_frame(s, zero);
        if (t < -1) return (int)t;
        if (t >= 0 && n < capacity) tokens[n++] = (uint32_t)t;
    }
    return n;
}
