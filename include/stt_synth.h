/*
 * stt_synth.h — seeded synthetic STT-1B checkpoints and audio-token streams.
 *
 * No counterpart in the reference, which downloads the real kyutai/stt-1b-en_fr checkpoint and
 * converts it with scripts/quantize.py.  This generator writes a checkpoint of the same
 * architecture and file format from a seed, so that the decode library, its tests, its
 * benchmark and the CPU restatement of the reference all read the same bytes without a network.
 *
 * It is a separate host-only library (libsttsynth.so, no CUDA): a program that only needs a
 * synthetic checkpoint (the CPU baseline, for one) does not load the decode library.
 *
 * Weights are drawn N(mean, std) from Philox-4x32-10 keyed by (seed, tensor index) with a
 * Box-Muller transform in f64, rounded to bf16, and Q4_0-quantised with the exact rules of
 * scripts/quantize.py:65-116; the file layout follows quantize.py:119-199.
 * Status codes are those of stt_b200.h (0 = OK, negative = error); the text of the last error
 * on the calling thread is available from stt_synth_last_error().
 */
#ifndef STT_SYNTH_H
#define STT_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct stt_synth_params {
    uint64_t seed;
    int32_t num_layers, hidden_size, num_heads, ffn_hidden;
    int32_t vocab_size, text_in_vocab_size, num_codebooks, audio_vocab_size;
    int32_t embedding_dtype;     /* 30 = BF16 (default), 2 = Q4_0, 0 = F32                  */
    float weight_std;            /* 0.02 */
    float norm_mean, norm_std;   /* 1.0, 0.02 (alphas rounded to bf16, stored F32)          */
    int32_t n_threads;           /* 0 = all host cores                                      */
} stt_synth_params;
void stt_synth_default(stt_synth_params* p);
/* Writes a whole GGUF v3 file into a buffer allocated by the library (*out_buf, *out_len);
 * release it with stt_synth_free. */
int stt_synth_gguf(const stt_synth_params* p, uint8_t** out_buf, size_t* out_len);
void stt_synth_free(uint8_t* buf);
/* Q4_0-quantises n floats (n % 32 == 0) with the rules of scripts/quantize.py:65-116. */
int stt_synth_quantize_q4_0(const float* x, size_t n, uint8_t* out);
/* Seeded uniform audio tokens in [0, 2048): out[f*num_codebooks + c] for frames
 * first_frame .. first_frame+n_frames-1 of stream `stream`. */
int stt_synth_audio_tokens(uint64_t seed, int32_t stream, int32_t first_frame, int32_t n_frames,
                           int32_t num_codebooks, uint32_t* out);
/* Text of the last error on the calling thread ("" if none). */
const char* stt_synth_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* STT_SYNTH_H */
