/*
 * stt_oracle.h — CPU restatement of the stt-web STT-1B decode step.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker that the CUDA library is compared against,
 * and the CPU baseline that bench.py times.  Only tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py load it; the library never links or calls it.
 */
#ifndef STT_ORACLE_H
#define STT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Precision modes.  0 = the reference's arithmetic: f32 activations, exact f32 dequantised
 * Q4_0 weights, f32 K/V (model.rs:185-192, Burn's default float).  The flags add the rounding
 * points of the B200 build so its results can be matched to summation-order noise. */
#define ORC_KV_BF16 1u    /* K and V rounded to bf16 (RNE) when written to the ring          */
#define ORC_GEMM_BF16 2u  /* each Q4 matmul rounds its input to bf16 and its weight          */
                          /* (nibble-8)*scale to bf16 before the f32 dot product             */

typedef struct orc_config {
    int32_t num_layers, num_heads, num_codebooks, text_delay, max_seq_len, sliding_window;
    double rope_theta;
    uint32_t text_padding_id, text_start_token;
} orc_config;

typedef struct orc_model orc_model;
typedef struct orc_stream orc_stream;

void orc_config_default(orc_config* c);

/* f16 -> f32 as gguf.rs:45-73 (subnormals map to half their value there). */
float orc_f16_to_f32_gguf(uint16_t bits);
/* f16 -> f32 as WGSL unpack2x16float (IEEE). */
float orc_f16_to_f32_ieee(uint16_t bits);

/* Q4_0 quantisation with the rules of scripts/quantize.py:65-116 (n % 32 == 0). */
void orc_quantize_q4_0(const float* x, size_t n, uint8_t* out);
/* Dequantise rows of raw 18-byte Q4_0 blocks: out[r*k+j] = (nib-8)*ieee_f16(scale). */
void orc_dequant_q4_0(const uint8_t* raw, int64_t rows, int64_t k, float* out);
/* EmbeddingStore::embed_id_add_cpu (gguf.rs:616-633): out[j] += row value, gguf f16 rule. */
void orc_embed_id_add_q4(const uint8_t* table, int64_t dim, uint32_t id, float* out);
/* q4_matmul (gguf.rs:517-578) with the summation order of shader_naive.wgsl:30-98:
 * out[r, n] = sum_k in[r, k] * W[n, k] for rows r < m.  flags: ORC_GEMM_BF16 or 0. */
void orc_q4_matmul(const uint8_t* w, int64_t n, int64_t k, const float* in, int64_t m,
                   float* out, uint32_t flags);

/* Loads a model from one contiguous GGUF buffer, which must outlive the model.  Returns 0 or
 * a negative code (message in orc_last_error()). */
int orc_model_load(const uint8_t* gguf, size_t len, const orc_config* cfg, orc_model** out);
void orc_model_free(orc_model* m);
int orc_model_dims(const orc_model* m, int32_t* hidden, int32_t* ffn, int32_t* vocab,
                   int32_t* text_vocab);

/* A stream = KV ring for every layer + the stream-loop state of stream.rs:20-41. */
orc_stream* orc_stream_new(const orc_model* m, uint32_t flags);
void orc_stream_free(orc_stream* s);
void orc_stream_reset(orc_stream* s);

/* SttModel::forward (model.rs:631-664): one step; logits (vocab floats) may be NULL; returns
 * the argmax (lowest index on ties) or a negative error. */
int64_t orc_forward(orc_stream* s, const uint32_t* audio, uint32_t text, float* logits);
/* orc_forward for n distinct streams of one model (same flags) in one step: audio holds
 * n * num_codebooks ids, texts n ids; logits (n * vocab) may be NULL; argmax receives n values.
 * Each stream gets exactly the values orc_forward would give it alone.  Returns 0 or a negative
 * error (then no stream has changed). */
int orc_forward_batch(orc_stream* const* ss, int n, const uint32_t* audio, const uint32_t* texts,
                      float* logits, int64_t* argmax);
/* SttModel::forward_with_gpu_token (model.rs:675-722): the audio sum, then the text row taken
 * from the dequantised f32 table by the previous argmax (has_argmax != 0) or built on the CPU
 * from fallback_text, added to it.  Returns the argmax or a negative error. */
int64_t orc_forward_gpu_token(orc_stream* s, const uint32_t* audio, int has_argmax, uint32_t argmax,
                              uint32_t fallback_text, float* logits);
/* SttStream::feed_frame (stream.rs:70-81, 90-107, 231-266).  Returns the emitted token,
 * -1 for None, or < -1 on error. */
int64_t orc_feed_frame(orc_stream* s, const uint32_t* audio);
/* feed_frame for n distinct streams in one batched step; logits (n * vocab) may be NULL;
 * tokens[i] receives the emitted token or -1.  Returns 0 or a negative error. */
int orc_feed_frame_batch(orc_stream* const* ss, int n, const uint32_t* audio, float* logits,
                         int64_t* tokens);
/* SttStream::flush (stream.rs:315-338); returns the number of tokens written. */
int orc_flush(orc_stream* s, uint32_t* tokens, int capacity);
/* State: offset, len, write_pos, frame_count, last_text_token, delay_prev0, delay_prev1. */
void orc_stream_state(const orc_stream* s, int64_t out[7]);
void orc_stream_set_last_text_token(orc_stream* s, uint32_t token);
/* Sets the next text token and the limit-cycle history (stream.rs:20-41) together, so that a
 * test can make the oracle continue from a state the device reached. */
void orc_stream_set_delay_state(orc_stream* s, uint32_t last_text_token, uint32_t prev0, uint32_t prev1);

/* Number of worker threads used by the matmuls (OpenMP); <= 0 leaves the default. */
void orc_set_threads(int n);
int orc_get_threads(void);
const char* orc_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
