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

/* Q4 matmul with the per-output summation order of shader_naive.wgsl:main (the block loop
 * :51-95): for each block, for each of its 4 words, acc += dot(lo vec4) then acc += dot(hi vec4),
 * with w = (nibble - 8) * scale in f32 (:64-81).  A weight row is dequantised once into `wrow`
 * (element j of a block holds the low nibble of byte j, element j + 16 the high one) and applied
 * to every input row, which gives the same values and the same order as a per-output loop. */
static void q4_row_dequant(const uint8_t* row, int64_t blocks_per_row, uint32_t flags, float* wrow) {
    for (int64_t blk = 0; blk < blocks_per_row; ++blk) {
        const uint8_t* b = row + blk * 18;
        const float scale = orc_f16_to_f32_ieee((uint16_t)(b[0] | (b[1] << 8)));
        float* w = wrow + blk * 32;
        for (int j = 0; j < 16; ++j) {
            w[j] = ((float)(b[2 + j] & 0x0F) - 8.0f) * scale;
            w[16 + j] = ((float)((b[2 + j] >> 4) & 0x0F) - 8.0f) * scale;
            if (flags & ORC_GEMM_BF16) {
                w[j] = round_bf16(w[j]);
                w[16 + j] = round_bf16(w[16 + j]);
            }
        }
    }
}

static float q4_row_dot(const float* wrow, int64_t blocks_per_row, const float* input) {
    float acc = 0.0f;
    for (int64_t blk = 0; blk < blocks_per_row; ++blk) {
        const int64_t kb = blk * 32;
        for (int wi = 0; wi < 4; ++wi) {
            acc += dot4(wrow + kb + wi * 4, input + kb + wi * 4);
            acc += dot4(wrow + kb + 16 + wi * 4, input + kb + 16 + wi * 4);
        }
    }
    return acc;
}

/* The same products for m input rows at once: the inputs are transposed to [k][m] so that the
 * loop over rows runs across SIMD lanes, while each row keeps its own accumulator and exactly the
 * operation order of q4_row_dot (dot4 products, then the two adds per word). */
static void q4_rows_dot(const float* wrow, int64_t blocks_per_row, const float* xt, int64_t m, float* acc,
                        float* s4) {
    for (int64_t r = 0; r < m; ++r) acc[r] = 0.0f;
    for (int64_t blk = 0; blk < blocks_per_row; ++blk) {
        const int64_t kb = blk * 32;
        for (int wi = 0; wi < 4; ++wi) {
            for (int half = 0; half < 2; ++half) {
                const int64_t k0 = kb + half * 16 + wi * 4;
                const float w0 = wrow[k0], w1 = wrow[k0 + 1], w2 = wrow[k0 + 2], w3 = wrow[k0 + 3];
                const float* x0 = xt + k0 * m;
                const float* x1 = x0 + m;
                const float* x2 = x1 + m;
                const float* x3 = x2 + m;
                for (int64_t r = 0; r < m; ++r) {
                    float t = w0 * x0[r];
                    t = t + w1 * x1[r];
                    t = t + w2 * x2[r];
                    t = t + w3 * x3[r];
                    s4[r] = t;
                }
                for (int64_t r = 0; r < m; ++r) acc[r] = acc[r] + s4[r];
            }
        }
    }
}

void orc_q4_matmul(const uint8_t* w, int64_t n, int64_t k, const float* in, int64_t m, float* out,
                   uint32_t flags) {
    const int64_t nb = k / 32;
    const float* x = in;
    float* xr = NULL;
    if (flags & ORC_GEMM_BF16) {
        xr = (float*)malloc(sizeof(float) * (size_t)(m * k));
        for (int64_t i = 0; i < m * k; ++i) xr[i] = round_bf16(in[i]);
        x = xr;
    }
    float* xt = NULL;
    if (m > 1) {
        xt = (float*)malloc(sizeof(float) * (size_t)(m * k));
        for (int64_t r = 0; r < m; ++r)
            for (int64_t j = 0; j < k; ++j) xt[j * m + r] = x[r * k + j];
    }
#pragma omp parallel
    {
        float* wrow = (float*)malloc(sizeof(float) * (size_t)k);
        float* acc = (float*)malloc(sizeof(float) * (size_t)(2 * m));
#pragma omp for schedule(static)
        for (int64_t c = 0; c < n; ++c) {
            q4_row_dequant(w + c * nb * 18, nb, flags, wrow);
            if (m == 1) {
                out[c] = q4_row_dot(wrow, nb, x);
            } else {
                q4_rows_dot(wrow, nb, xt, m, acc, acc + m);
                for (int64_t r = 0; r < m; ++r) out[r * n + c] = acc[r];
            }
        }
        free(acc);
        free(wrow);
    }
    free(xt);
    free(xr);
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
    orc_stream_reset(s);
    return s;
}

void orc_stream_free(orc_stream* s) {
    if (!s) return;
    free(s->k);
    free(s->v);
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
void orc_stream_set_delay_state(orc_stream* s, uint32_t last_text_token, uint32_t prev0, uint32_t prev1) {
    s->last_text_token = last_text_token;
    s->delay_prev[0] = prev0;
    s->delay_prev[1] = prev1;
}

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

/* Attention of head h of one stream at layer l (model.rs:426-474): RoPE on q and k at the
 * stream's position, the K/V ring write at write_pos (KVCache::update, model.rs:176-222), then
 * softmax(q . k^T * scale) . v over the len + 1 valid slots (masks are no-ops at q_len == 1,
 * model.rs:309-311, 338-340).  `scores` holds max_len floats. */
static void head_attention(orc_stream* s, int l, int h, float* qkv, float* out, float* scores) {
    const orc_model* m = s->m;
    const int32_t D = m->D, H = m->H, HD = m->HD, ML = s->max_len;
    float *q = qkv + h * HD, *k = qkv + D + h * HD, *v = qkv + 2 * D + h * HD;
    rope_rotate(m, q, s->offset);
    rope_rotate(m, k, s->offset);
    float* kd = s->k + (((size_t)l * H + h) * ML + s->write_pos) * HD;
    float* vd = s->v + (((size_t)l * H + h) * ML + s->write_pos) * HD;
    for (int d = 0; d < HD; ++d) {
        kd[d] = (s->flags & ORC_KV_BF16) ? round_bf16(k[d]) : k[d];
        vd[d] = (s->flags & ORC_KV_BF16) ? round_bf16(v[d]) : v[d];
    }
    const int32_t len = s->len + 1 < ML ? s->len + 1 : ML;
    const float* kb = s->k + ((size_t)l * H + h) * ML * HD;
    const float* vb = s->v + ((size_t)l * H + h) * ML * HD;
    float mx = -INFINITY;
    for (int32_t j = 0; j < len; ++j) {
        float dot = 0.0f;
        for (int d = 0; d < HD; ++d) dot += q[d] * kb[(size_t)j * HD + d];
        scores[j] = dot * m->attn_scale;
        if (scores[j] > mx) mx = scores[j];
    }
    float sum = 0.0f;
    for (int32_t j = 0; j < len; ++j) { scores[j] = expf(scores[j] - mx); sum += scores[j]; }
    for (int32_t j = 0; j < len; ++j) scores[j] = scores[j] / sum;
    for (int d = 0; d < HD; ++d) {
        float acc = 0.0f;
        for (int32_t j = 0; j < len; ++j) acc += scores[j] * vb[(size_t)j * HD + d];
        out[h * HD + d] = acc;
    }
}

/* Scratch of one batched step over n streams: the stacked rows of every stream. */
typedef struct {
    float *x, *xn, *qkv, *attn, *tmp, *hid, *gate, *logits;
} orc_batch;

static int batch_alloc(orc_batch* b, const orc_model* m, int n) {
    const size_t N = (size_t)n;
    b->x = (float*)calloc(N * m->D, 4);
    b->xn = (float*)calloc(N * m->D, 4);
    b->qkv = (float*)calloc(N * 3 * m->D, 4);
    b->attn = (float*)calloc(N * m->D, 4);
    b->tmp = (float*)calloc(N * m->D, 4);
    b->hid = (float*)calloc(N * 2 * m->F, 4);
    b->gate = (float*)calloc(N * m->F, 4);
    b->logits = (float*)calloc(N * m->V, 4);
    return b->x && b->xn && b->qkv && b->attn && b->tmp && b->hid && b->gate && b->logits;
}

static void batch_free(orc_batch* b) {
    free(b->x); free(b->xn); free(b->qkv); free(b->attn); free(b->tmp); free(b->hid); free(b->gate);
    free(b->logits);
}

/* Q4TransformerBlock::forward_with_cache (model.rs:556-571) with Q4Attention (model.rs:426-474)
 * and Q4FeedForward (model.rs:517-524) for one layer, over the stacked rows of n streams.  Each
 * stream's arithmetic is that of a lone stream: the matmuls give every row the per-output order
 * of orc_q4_matmul, and attention reads only the stream's own ring. */
static void block_forward(orc_stream* const* ss, int n, int l, orc_batch* b) {
    const orc_model* m = ss[0]->m;
    const orc_layer* L = &m->layers[l];
    const int32_t D = m->D, H = m->H, F = m->F;
    const uint32_t gf = ss[0]->flags & ORC_GEMM_BF16;

    for (int i = 0; i < n; ++i) rmsnorm(b->x + (size_t)i * D, L->norm1, D, b->xn + (size_t)i * D);
    orc_q4_matmul(L->in_proj, 3 * D, D, b->xn, n, b->qkv, gf);
#pragma omp parallel
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)ss[0]->max_len);
#pragma omp for schedule(dynamic)
        for (int t = 0; t < n * H; ++t) {
            const int i = t / H, h = t % H;
            head_attention(ss[i], l, h, b->qkv + (size_t)i * 3 * D, b->attn + (size_t)i * D, scores);
        }
        free(scores);
    }
    orc_q4_matmul(L->out_proj, D, D, b->attn, n, b->tmp, gf);
    for (size_t i = 0; i < (size_t)n * D; ++i) b->x[i] = b->tmp[i] + b->x[i];

    for (int i = 0; i < n; ++i) rmsnorm(b->x + (size_t)i * D, L->norm2, D, b->xn + (size_t)i * D);
    orc_q4_matmul(L->lin_in, 2 * F, D, b->xn, n, b->hid, gf);
    for (int i = 0; i < n; ++i) {
        const float* hd = b->hid + (size_t)i * 2 * F;
        float* g = b->gate + (size_t)i * F;
        for (int32_t j = 0; j < F; ++j) g[j] = silu(hd[j]) * hd[F + j];
    }
    orc_q4_matmul(L->lin_out, D, F, b->gate, n, b->tmp, gf);
    for (size_t i = 0; i < (size_t)n * D; ++i) b->x[i] = b->tmp[i] + b->x[i];
}

/* Checks the inputs of one batched step the way the reference would panic on them (nothing is
 * changed when a check fails). */
static int check_batch(orc_stream* const* ss, int n, const uint32_t* audio, const uint32_t* texts) {
    if (n <= 0 || !ss) return set_err(-1, "need at least one stream");
    const orc_model* m = ss[0]->m;
    for (int i = 0; i < n; ++i) {
        if (ss[i]->m != m || ss[i]->flags != ss[0]->flags) return set_err(-1, "streams of one batch share a model and flags");
        for (int j = 0; j < i; ++j)
            if (ss[j] == ss[i]) return set_err(-1, "stream repeated in one batch");
        if (ss[i]->offset + 1 > m->cfg.max_seq_len)
            return set_err(-6, "position %d beyond the RoPE table (%d)", ss[i]->offset, m->cfg.max_seq_len);
        for (int c = 0; c < m->cfg.num_codebooks; ++c)
            if (audio[(size_t)i * m->cfg.num_codebooks + c] >= (uint32_t)m->AV)
                return set_err(-1, "audio token %u out of range", audio[(size_t)i * m->cfg.num_codebooks + c]);
        if (texts[i] >= (uint32_t)m->TV) return set_err(-1, "text token %u out of range", texts[i]);
    }
    return 0;
}

static int64_t argmax_row(const float* lg, int32_t V) {
    int64_t best = 0;
    for (int32_t i = 1; i < V; ++i)
        if (lg[i] > lg[best]) best = i;
    return best;
}

int orc_forward_batch(orc_stream* const* ss, int n, const uint32_t* audio, const uint32_t* texts, float* logits,
                      int64_t* argmax) {
    const int rc = check_batch(ss, n, audio, texts);
    if (rc) return rc;
    const orc_model* m = ss[0]->m;
    const int32_t D = m->D, NC = m->cfg.num_codebooks;
    orc_batch b;
    if (!batch_alloc(&b, m, n)) { batch_free(&b); return set_err(-3, "out of memory"); }
    /* embedding sum on the CPU in codebook order, then the text row (model.rs:640-646) */
    for (int i = 0; i < n; ++i) {
        float* x = b.x + (size_t)i * D;
        for (int c = 0; c < NC; ++c) embed_add(m, m->emb_audio[c], audio[(size_t)i * NC + c], x);
        embed_add(m, m->emb_text, texts[i], x);
    }
    for (int l = 0; l < m->cfg.num_layers; ++l) block_forward(ss, n, l, &b);
    for (int i = 0; i < n; ++i) {
        orc_stream* s = ss[i];
        s->write_pos = (s->write_pos + 1) % s->max_len;
        s->offset += 1;
        s->len = s->len + 1 < s->max_len ? s->len + 1 : s->max_len;
        rmsnorm(b.x + (size_t)i * D, m->out_norm, D, b.xn + (size_t)i * D);
    }
    orc_q4_matmul(m->head, m->V, m->D, b.xn, n, b.logits, ss[0]->flags & ORC_GEMM_BF16);
    for (int i = 0; i < n; ++i) {
        const float* lg = b.logits + (size_t)i * m->V;
        if (logits) memcpy(logits + (size_t)i * m->V, lg, sizeof(float) * (size_t)m->V);
        argmax[i] = argmax_row(lg, m->V);
    }
    batch_free(&b);
    return 0;
}

int64_t orc_forward(orc_stream* s, const uint32_t* audio, uint32_t text, float* logits) {
    int64_t am = 0;
    const int rc = orc_forward_batch(&s, 1, audio, &text, logits, &am);
    return rc ? rc : am;
}

/* SttModel::forward_with_gpu_token (model.rs:675-722): the audio rows are summed on the CPU
 * (embed_id_add_cpu into a zero vector), the text row comes either from the f32 table that
 * dequant_embedding_to_gpu (gguf.rs:697-738) builds, selected by the previous argmax, or (no
 * argmax yet) from embed_id_add_cpu into a second zero vector; the two vectors are then added.
 * The rest of the step is SttModel::forward's. */
int64_t orc_forward_gpu_token(orc_stream* s, const uint32_t* audio, int has_argmax, uint32_t argmax,
                              uint32_t fallback_text, float* logits) {
    const orc_model* m = s->m;
    const uint32_t text = has_argmax ? argmax : fallback_text;
    const int rc = check_batch(&s, 1, audio, &text);
    if (rc) return rc;
    const int32_t D = m->D, NC = m->cfg.num_codebooks;
    orc_batch b;
    if (!batch_alloc(&b, m, 1)) { batch_free(&b); return set_err(-3, "out of memory"); }
    float* audio_sum = b.x;
    for (int c = 0; c < NC; ++c) embed_add(m, m->emb_audio[c], audio[c], audio_sum);
    float* text_in = (float*)calloc((size_t)D, 4);
    if (has_argmax && m->emb_dtype == 2) {
        /* dequant_embedding_to_gpu: data[j] = (nib - 8) * d, assigned (gguf.rs:725-732) */
        const uint8_t* row = m->emb_text + (size_t)argmax * (D / 32) * 18;
        for (int32_t blk = 0; blk < D / 32; ++blk) {
            const uint8_t* bo = row + blk * 18;
            const float d = orc_f16_to_f32_gguf((uint16_t)(bo[0] | (bo[1] << 8)));
            for (int j = 0; j < 16; ++j) {
                text_in[blk * 32 + j] = ((float)(bo[2 + j] & 0x0F) - 8.0f) * d;
                text_in[blk * 32 + j + 16] = ((float)((bo[2 + j] >> 4) & 0x0F) - 8.0f) * d;
            }
        }
    } else {
        embed_add(m, m->emb_text, text, text_in);
    }
    for (int32_t j = 0; j < D; ++j) audio_sum[j] = audio_sum[j] + text_in[j];
    free(text_in);
    for (int l = 0; l < m->cfg.num_layers; ++l) block_forward(&s, 1, l, &b);
    s->write_pos = (s->write_pos + 1) % s->max_len;
    s->offset += 1;
    s->len = s->len + 1 < s->max_len ? s->len + 1 : s->max_len;
    rmsnorm(b.x, m->out_norm, D, b.xn);
    orc_q4_matmul(m->head, m->V, m->D, b.xn, 1, b.logits, s->flags & ORC_GEMM_BF16);
    if (logits) memcpy(logits, b.logits, sizeof(float) * (size_t)m->V);
    const int64_t am = argmax_row(b.logits, m->V);
    batch_free(&b);
    return am;
}

/* SttStream::feed_frame (stream.rs:70-81) for n streams at once: submit_frame (stream.rs:90-107)
 * with each stream's last_text_token, one batched step, then resolve_pending_as_token
 * (stream.rs:231-266) per stream.  tokens[i] is the emitted token or -1 (None). */
int orc_feed_frame_batch(orc_stream* const* ss, int n, const uint32_t* audio, float* logits, int64_t* tokens) {
    if (n <= 0 || !ss) return set_err(-1, "need at least one stream");
    uint32_t* texts = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)n);
    int64_t* am = (int64_t*)malloc(sizeof(int64_t) * (size_t)n);
    for (int i = 0; i < n; ++i) texts[i] = ss[i]->last_text_token;
    const int rc = orc_forward_batch(ss, n, audio, texts, logits, am);
    if (rc == 0) {
        for (int i = 0; i < n; ++i) {
            orc_stream* s = ss[i];
            const orc_config* c = &s->m->cfg;
            s->frame_count += 1;
            const int emits = s->frame_count >= c->text_delay;
            const uint32_t token = (uint32_t)am[i];
            if (emits) {
                s->last_text_token = token;
                tokens[i] = token;
                continue;
            }
            const uint32_t prev0 = s->delay_prev[0], prev1 = s->delay_prev[1];
            s->delay_prev[0] = prev1;
            s->delay_prev[1] = token;
            if (token != c->text_padding_id && token != 0 && token == prev0 && token != prev1)
                s->last_text_token = c->text_padding_id;
            else
                s->last_text_token = token;
            tokens[i] = -1;
        }
    }
    free(texts);
    free(am);
    return rc;
}

int64_t orc_feed_frame(orc_stream* s, const uint32_t* audio) {
    int64_t tok = 0;
    const int rc = orc_feed_frame_batch(&s, 1, audio, NULL, &tok);
    if (rc) return rc - 100; /* keep errors below -1 */
    return tok;
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
