/*
 * stt_b200.h — C ABI of the B200-native (sm_100a) STT-1B decode step.
 *
 * This library replaces the GPU half of the stt-wasm crate of stt-web: the Q4 weight
 * store and loader (crates/stt-wasm/src/gguf.rs), the transformer step
 * (crates/stt-wasm/src/model.rs) and the delayed-streams step loop
 * (crates/stt-wasm/src/stream.rs).  Every entry point below names the reference
 * interface it replaces (path:line inside the stt-web project).
 *
 * Conventions
 *  - Every call returns an int status: STT_OK (0) or a negative STT_E_* code.  The text of
 *    the last error on the calling thread is available from stt_last_error().
 *  - No C++ exception crosses this boundary.  Host buffers are owned by the caller and are
 *    only read/written during the call.  Pointers documented as "device" must be CUDA device
 *    pointers on the model's device.
 *  - A model handle is bound to one CUDA device.  Calls on one handle (and on the stream
 *    sets created from it) are not thread-safe: the caller serialises them.  The multi-GPU
 *    pattern is one host thread per device, each with its own model.
 *  - Sizes are those of the loaded GGUF file; the defaults match kyutai/stt-1b-en_fr.
 */
#ifndef STT_B200_H
#define STT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (the reference reports anyhow::Result errors at load, gguf.rs:204-310,
 *      and panics on shape, launch and index errors, gguf.rs:521-529, 562-568, 620-621) ---- */
#define STT_OK 0
#define STT_E_INVALID_ARG (-1)  /* bad pointer, size, stream id or token id              */
#define STT_E_FORMAT (-2)       /* malformed or unsupported GGUF content                 */
#define STT_E_OOM (-3)          /* host or device allocation failed                      */
#define STT_E_CUDA (-4)         /* a CUDA runtime call failed                            */
#define STT_E_DEVICE_FLAG (-5)  /* a kernel raised its error word (bad index / timeout)  */
#define STT_E_STATE (-6)        /* call not valid in the current state (e.g. position    */
                                /* past max_seq_len, which panics in the reference)      */

/* Model hyper-parameters.  Mirrors SttConfig (crates/stt-wasm/src/lib.rs:27-58) field by
 * field; stt_config_default() gives the values of SttConfig::default() (lib.rs:60-80). */
typedef struct stt_config {
    int32_t num_layers;          /* 16 */
    int32_t hidden_size;         /* 2048 */
    int32_t num_heads;           /* 16 */
    int32_t num_kv_heads;        /* 16 (MHA) */
    int32_t intermediate_size;   /* 5632: unused, as in the reference; FFN width comes from
                                    the linear_in shape (model.rs:517-524) */
    int32_t vocab_size;          /* 8000: text_linear rows */
    int32_t text_in_vocab_size;  /* 8001: text_emb rows */
    int32_t num_codebooks;       /* 32 */
    int32_t audio_vocab_size;    /* 2049 */
    int32_t text_delay;          /* 6 */
    double rope_theta;           /* 100000.0 */
    int32_t max_seq_len;         /* 4096: RoPE table length; positions beyond it are an error */
    int32_t sliding_window;      /* 750: the KV ring holds sliding_window + 1 slots */
    uint32_t text_padding_id;    /* 3 */
    uint32_t text_start_token;   /* 8000 */
} stt_config;

/* Fills *cfg with SttConfig::default() (crates/stt-wasm/src/lib.rs:60-80). */
void stt_config_default(stt_config* cfg);

/* Storage type of the KV ring on the device. */
#define STT_KV_BF16 0   /* default: bf16 K and V (half the bytes of the reference's f32)    */
#define STT_KV_F32 1    /* f32 K and V, the reference's own precision (model.rs:185-192)    */

typedef struct stt_model stt_model;      /* loaded weights on one device                    */
typedef struct stt_streams stt_streams;  /* N independent streams: KV rings + step state    */
typedef struct stt_q4_tensor stt_q4_tensor; /* one Q4_0 matrix in the device layout         */

/* Read-only description of a loaded model. */
typedef struct stt_model_info {
    int32_t num_layers, hidden_size, num_heads, head_dim, ffn_hidden;
    int32_t vocab_size, text_in_vocab_size, num_codebooks, audio_vocab_size;
    int32_t embedding_dtype;     /* GGML dtype code of the embedding tables (0,1,2 or 30)  */
    int32_t device;
    uint64_t q4_weight_bytes;    /* Q4_0 bytes one decode step reads (all linear layers)   */
    uint64_t device_bytes;       /* total device memory held by the model                  */
    int32_t tensor_core_min_batch; /* batches of at least this many streams run their Q4
                                    * products on the tensor cores; 0 when the weights do not
                                    * fit that path (in_features not a multiple of 256, or a
                                    * Q4_0 scale of magnitude above 4) */
    int32_t reserved;
} stt_model_info;

/* ---------------------------------------------------------------------------------------
 * Loading — replaces Q4ModelLoader::from_shards (gguf.rs:752-755) + load_deferred
 * (gguf.rs:763-826) + Q4ModelParts::finalize (gguf.rs:658-692).
 * The GGUF bytes may be split over several shards (ShardedCursor, gguf.rs:321-397).
 * Tensor names, the dims-reversal rule (gguf.rs:83-85), the dtype checks (gguf.rs:880-882,
 * 906-916) and the 32-byte data alignment (gguf.rs:34, 273-274) follow the reference.
 * Embedding tables may be Q4_0 (the reference format, gguf.rs:616-633) or, as an
 * extension, F32 / F16 / BF16 (GGML type 30).  cfg == NULL means stt_config_default().
 * ------------------------------------------------------------------------------------- */
int stt_model_load_gguf(const uint8_t* const* shards, const size_t* shard_lens, int n_shards,
                        int device, const stt_config* cfg, stt_model** out);
int stt_model_destroy(stt_model* model);
int stt_model_get_info(const stt_model* model, stt_model_info* out);

/* ---------------------------------------------------------------------------------------
 * Streams — replaces SttModel::create_cache (model.rs:728-738) plus one SttStream::new
 * (stream.rs:53-64) per stream.  Each stream owns a ring of sliding_window + 1 K/V slots per
 * layer (model.rs:130-153) and the stream-loop state of stream.rs:20-41.
 * kv_dtype is STT_KV_BF16 or STT_KV_F32.
 * ------------------------------------------------------------------------------------- */
int stt_streams_create(stt_model* model, int n_streams, int kv_dtype, stt_streams** out);
int stt_streams_destroy(stt_streams* streams);

/* Raw decode step over a batch — replaces SttModel::forward (model.rs:631-664) followed by
 * logits.argmax(2) (stream.rs:104).  For each i < n, stream stream_ids[i] consumes
 * audio_tokens[i*num_codebooks .. +num_codebooks] and text_tokens[i]; its KV ring and
 * position advance by one.  Host buffers.  logits_out (n*vocab_size floats) and argmax_out
 * (n values, lowest index on ties) may each be NULL.  Stream ids in one call are distinct. */
int stt_forward(stt_streams* streams, const int32_t* stream_ids, int n,
                const uint32_t* audio_tokens, const uint32_t* text_tokens,
                float* logits_out, uint32_t* argmax_out);

/* One frame of the delayed-streams loop — replaces SttStream::feed_frame (stream.rs:70-81):
 * submit_frame (stream.rs:90-107) then resolve_pending_as_token (stream.rs:231-266),
 * including the delay gating and the limit-cycle breaker.  *token_out is the emitted token,
 * or -1 for the reference's None (a frame inside the text delay). */
int stt_stream_feed_frame(stt_streams* streams, int stream_id, const uint32_t* audio_tokens,
                          int32_t* token_out);

/* The same frame step for n streams at once (one batched decode step).  tokens_out[i] is the
 * token emitted by stream_ids[i] or -1. */
int stt_streams_feed_frame(stt_streams* streams, const int32_t* stream_ids, int n,
                           const uint32_t* audio_tokens, int32_t* tokens_out);

/* n_frames consecutive feed_frame calls on one stream, run back to back on the device with
 * the greedy token fed back on the device (the goal of submit_frame_gpu, stream.rs:117-138,
 * with the exact feed_frame semantics).  audio_tokens holds n_frames*num_codebooks ids;
 * tokens_out receives n_frames values (-1 = None).  Host buffers. */
int stt_stream_feed_frames(stt_streams* streams, int stream_id, int n_frames,
                           const uint32_t* audio_tokens, int32_t* tokens_out);

/* Device-pointer variant of stt_stream_feed_frames: d_audio and d_tokens are device buffers,
 * the work is queued on cuda_stream (a cudaStream_t, NULL = legacy default stream) and the
 * call returns without synchronising.  The stream's host-side mirror of its state is
 * refreshed by the next synchronous call on that stream. */
int stt_stream_feed_frames_device(stt_streams* streams, int stream_id, int n_frames,
                                  const uint32_t* d_audio, int32_t* d_tokens,
                                  void* cuda_stream);

/* Batched device-pointer frame step: stream_ids are host values, d_audio holds
 * n*num_codebooks ids and d_tokens n outputs, both on the device; queued on cuda_stream. */
int stt_streams_feed_frame_device(stt_streams* streams, const int32_t* stream_ids, int n,
                                  const uint32_t* d_audio, int32_t* d_tokens,
                                  void* cuda_stream);

/* Asynchronous batched frames — replaces SttStream::submit_frame_gpu (stream.rs:117-138) with
 * take_batch_pending / resolve_batch (stream.rs:146-183) as the WASM bindings drive them
 * (web/bindings.rs:432-489): frames are queued with the text token fed back on the device, and
 * their tokens are read back later, without stalling the submitting thread.
 *
 * stt_streams_submit_frame queues one feed_frame step (the delay gating and the limit-cycle rule
 * included) for the n streams stream_ids, with host audio (n*num_codebooks ids, copied before the
 * call returns), on the set's own CUDA stream, and returns without waiting; the step's emitted
 * tokens will land in pinned host memory behind an event.  *ticket identifies the frame.  At most
 * 64 submitted frames may be outstanding: a 65th submit without taking the oldest one's tokens
 * fails with STT_E_STATE.  Frames of one set run in submission order, and after any other call on
 * the set.
 * stt_streams_poll_frame takes the tokens of `ticket` if its step has completed (*ready = 1,
 * tokens_out[i] for stream_ids[i], -1 = None) and returns at once otherwise (*ready = 0).
 * stt_streams_wait_frame blocks until they are there.  Tokens are taken once per ticket, in any
 * order; a kernel error of that step is returned by the call that takes them. */
int stt_streams_submit_frame(stt_streams* streams, const int32_t* stream_ids, int n,
                             const uint32_t* audio_tokens, int64_t* ticket);
int stt_streams_poll_frame(stt_streams* streams, int64_t ticket, int32_t* tokens_out, int* ready);
int stt_streams_wait_frame(stt_streams* streams, int64_t ticket, int32_t* tokens_out);

/* Replaces SttStream::flush (stream.rs:315-338): text_delay frames of zero audio through
 * feed_frame, collecting the emitted tokens (at most text_delay).  *n_tokens receives the
 * count written to tokens_out (capacity entries available). */
int stt_stream_flush(stt_streams* streams, int stream_id, uint32_t* tokens_out, int capacity,
                     int* n_tokens);

/* Replaces SttStream::reset (stream.rs:341-349) when keep_buffers == 0 and
 * SttStream::reset_keep_buffers (stream.rs:354-362) otherwise.  Both zero the state; the
 * device ring is kept allocated in either case and zeroed when keep_buffers != 0. */
int stt_stream_reset(stt_streams* streams, int stream_id, int keep_buffers);

/* Asynchronous reset: the same state change as stt_stream_reset, queued on cuda_stream (NULL =
 * legacy default stream) behind work already queued there, without waiting for the device. */
int stt_stream_reset_async(stt_streams* streams, int stream_id, int keep_buffers, void* cuda_stream);

/* Precision of the layer products of batched steps on the tensor cores (batches of at least
 * tensor_core_min_batch streams; no counterpart in the reference, whose f32 shader has one).  Each
 * dequantised weight is split exactly into two f16 parts, w = w_hi + w_lo, and accumulated in f32:
 *   STT_PRODUCTS_F16X3 (default): the activation is split too, x = x_hi + x_lo, and three MMAs add
 *     w_hi.x_hi + w_hi.x_lo + w_lo.x_hi: about 22 significant bits per product, close to f32;
 *   STT_PRODUCTS_F16X2: the activation is rounded to f16 (11 bits) and two MMAs add
 *     w_hi.x + w_lo.x: a third less tensor work, about 2^-12 relative error per activation.
 * Applies to the set's later batched steps (their CUDA graphs are captured again). */
#define STT_PRODUCTS_F16X3 0
#define STT_PRODUCTS_F16X2 1
int stt_streams_set_product_precision(stt_streams* streams, int precision);

/* Replaces SttStream::set_last_text_token (stream.rs:190-192). */
int stt_stream_set_last_text_token(stt_streams* streams, int stream_id, uint32_t token);

/* Stream-loop state of one stream (stream.rs:20-41 and KVCache counters, model.rs:139-153). */
typedef struct stt_stream_state {
    int32_t offset;          /* absolute position (tokens seen), RoPE offset              */
    int32_t len;             /* valid ring entries, <= sliding_window + 1                 */
    int32_t write_pos;       /* next ring slot                                             */
    int32_t frame_count;     /* frames submitted since reset                               */
    uint32_t last_text_token;
    uint32_t delay_prev[2];  /* limit-cycle history, 0xFFFFFFFF = none (stream.rs:62)       */
} stt_stream_state;
int stt_stream_get_state(stt_streams* streams, int stream_id, stt_stream_state* out);

/* ---------------------------------------------------------------------------------------
 * Isolated Q4_0 matmul — replaces Q4Tensor::from_q4_bytes (gguf.rs:418-451) and
 * q4_matmul (gguf.rs:517-578, shader crates/stt-wasm/src/wgsl/shader_naive.wgsl:30-98).
 * ------------------------------------------------------------------------------------- */
/* Uploads raw Q4_0 bytes of an [n, k] matrix ((n*k/32)*18 bytes, k % 32 == 0) and repacks
 * them into the device layout. */
int stt_q4_tensor_create(const uint8_t* q4_bytes, size_t n_bytes, int n, int k, int device,
                         stt_q4_tensor** out);
int stt_q4_tensor_destroy(stt_q4_tensor* t);
/* out[rows, n] = input[rows, k] x W^T with f32 host buffers (rows = B*M of the reference). */
int stt_q4_matmul(const stt_q4_tensor* w, const float* input, int rows, float* out);
/* Device variant: d_input is f32 [rows, k] (in_dtype 0) or bf16 [rows, k] (in_dtype 1);
 * d_out is f32 [rows, n].  Queued on cuda_stream, no synchronisation.
 * in_dtype 2: f16 [rows, k] input (k a multiple of 256, Q4_0 scales of magnitude at most 4),
 * computed on the tensor cores with each dequantised weight split exactly into two f16 parts and
 * f32 accumulation (the batched-stream product).  Its scratch is kept with the tensor and grows
 * on demand: a call with more rows than any before it may allocate (and so synchronise). */
int stt_q4_matmul_device(const stt_q4_tensor* w, const void* d_input, int in_dtype, int rows,
                         float* d_out, void* cuda_stream);
/* No counterpart in the reference.  Split-K form of stt_q4_matmul_device for f32 (in_dtype 0) and
 * bf16 (in_dtype 1) input only, with `splits` (1..64 and at most k/32) added; in_dtype 2 (f16, the
 * tensor-core product, whose scratch grows with the rows) is rejected with STT_E_INVALID_ARG.  It
 * requests no device memory: partial sums and per-tile
 * counters live in a fixed 4 MiB + 16 KiB array of the library's device image, so
 * splits * rows * n * 4 must be at most 4 MiB and n at most 65536, else STT_E_INVALID_ARG.
 * The first call on a device looks up that array's address (make it before capturing a
 * stream).  Calls on one device share the array and must not overlap in time.  Queued on
 * cuda_stream, no synchronisation; d_input 16-byte aligned (f32) or 8-byte aligned (bf16). */
int stt_q4_matmul_device_noalloc(const stt_q4_tensor* w, const void* d_input, int in_dtype, int rows,
                                 int splits, float* d_out, void* cuda_stream);
/* No counterpart in the reference.  Waits for the device, then reports whether a device-side wait
 * of any matmul on this tensor since the last check ran out (STT_E_DEVICE_FLAG: that call's output
 * is invalid; the flag is cleared) or not (STT_OK).  stt_q4_matmul checks it itself. */
int stt_q4_tensor_status(const stt_q4_tensor* w);
/* Dequantises the whole matrix to f32 on the device and copies it to out_host (n*k floats):
 * out[r*k + j] = (nibble - 8) * f16_to_f32(scale), bit-exact with gguf.rs:616-633. */
int stt_q4_tensor_dequant(const stt_q4_tensor* w, float* out_host);

/* ---------------------------------------------------------------------------------------
 * SentencePiece detokeniser: the step after the decode path.  Replaces SpmDecoder
 * (crates/stt-wasm/src/tokenizer.rs:7-38), which turns the emitted text-token ids into text.
 * Host only: these calls touch no device.  A decoder is immutable after creation, so several
 * threads may decode with one decoder at the same time.
 * ------------------------------------------------------------------------------------- */
typedef struct stt_spm_decoder stt_spm_decoder;
/* SpmDecoder::from_bytes (tokenizer.rs:14-17, vocabulary walk :44-96): the pieces of a
 * SentencePiece `.model` protobuf, token id = entry order.  A piece whose declared length runs
 * past the buffer (a panic in the reference) is STT_E_FORMAT. */
int stt_spm_decoder_create(const uint8_t* model_bytes, size_t n_bytes, stt_spm_decoder** out);
int stt_spm_decoder_destroy(stt_spm_decoder* dec);
/* SpmDecoder::vocab_len (tokenizer.rs:35-37). */
int stt_spm_vocab_len(const stt_spm_decoder* dec, int64_t* out);
/* The piece of token `id` as the decoder holds it (UTF-8; invalid bytes of the file replaced
 * by U+FFFD as in tokenizer.rs:90).  Output convention of both calls below: *len receives the
 * text's byte length; with out == NULL nothing is written (a size query), else out must hold
 * *len + 1 bytes (the text and a NUL) or the call fails with STT_E_INVALID_ARG. */
int stt_spm_piece(const stt_spm_decoder* dec, int64_t id, char* out, size_t cap, size_t* len);
/* SpmDecoder::decode (tokenizer.rs:30-32, rules :150-192): ids 0 (end of stream) and 3
 * (padding) and ids past the vocabulary are skipped; runs of byte-fallback pieces "<0xHH>"
 * are emitted only when they form valid UTF-8; U+2581 becomes a space; nothing is trimmed. */
int stt_spm_decode(const stt_spm_decoder* dec, const uint32_t* ids, size_t n, char* out, size_t cap,
                   size_t* len);

/* ---------------------------------------------------------------------------------------
 * Diagnostics (no counterpart in the reference): timing probes of the persistent
 * single-stream step kernel, used by the benchmarks and profiles of this library.
 * ------------------------------------------------------------------------------------- */
/* Records (tag, SM clock cycles) pairs at the phase boundaries of frame `frame` of CTA 0, with
 * (0, %globaltimer ns) pairs at the frame's start and end, on later single-stream calls;
 * -1 disables. */
int stt_debug_trace_frame(stt_streams* streams, int frame);
/* Copies the timestamps of the last traced frame (at most cap); *n receives the count. */
int stt_debug_get_trace(stt_streams* streams, uint64_t* out, int cap, int* n);
/* Copies every CTA's %globaltimer stamps of the last traced frame: out[cta * n_slots + slot],
 * slot 0 the frame start, 1 + 16 l + i the i-th phase mark of layer l, 1 + 16 L + i the head's
 * marks and the argmax (0 = not reached by that CTA).  cap must hold num_sms * n_slots values. */
int stt_debug_get_trace_ctas(stt_streams* streams, uint64_t* out, int cap, int* n_ctas, int* n_slots);
/* Mean time of one grid barrier over `iters` back-to-back barriers on device `device`, in
 * nanoseconds: mode 0 is the persistent kernel's barrier (release add, acquire poll of the
 * counter), mode 1 a variant in which the last arriver publishes a flag that the others poll. */
int stt_debug_barrier_ns(int device, int iters, int mode, double* ns_per_barrier);

/* Allocation-failure injection for tests of the error paths: after `after` more successful
 * allocations of device or pinned host memory by this library (any thread, any device), the next
 * one fails as if memory had run out, so the call making it returns STT_E_OOM having released
 * whatever it had allocated; the countdown then stops.  after < 0 disarms it. */
int stt_debug_fail_allocation(int after);
/* Test of the persistent kernel's bounded waits.  Arms the next single-stream call on this set
 * (one launch only): in its first frame, the CTAs that compute the first layer's output projection
 * wait for an input epoch that no phase ever publishes.  That wait gives up after its limit (about
 * a second), the launch stops through the same abort path as a real timeout, and the call returns
 * STT_E_DEVICE_FLAG; the stream's state on the device is left as it was before the failed frame, so
 * stt_stream_reset (or the next call) continues normally.  Nothing faults or hangs. */
int stt_debug_arm_wait_timeout(stt_streams* streams);
/* Test of the integer-MMA GEMV's bounded waits.  Arms the next matmul call on this tensor that
 * takes that kernel (f32 or bf16 input, 2 to 8 rows per pass, k a multiple of 256; one launch
 * only): its first weight stage is never loaded, so the warps waiting for it give up after their
 * limit (4M polls, about 0.2 s measured on B200) and the kernel stops through the same path as a
 * real timeout, recording
 * STT_E_DEVICE_FLAG for stt_q4_tensor_status (stt_q4_matmul returns it).  Nothing faults or hangs. */
int stt_debug_q4_arm_wait_timeout(stt_q4_tensor* w);
/* Number of kernels one batched step of n streams (n >= 2) launches: the nodes of the CUDA
 * graph that the library captures for that batch size (captured on first use). */
int stt_debug_graph_kernels(stt_streams* streams, int n, int* kernels);
/* Mean device time of one launch of each of the five tensor-core products of a batched step of
 * n streams (tensor_core_min_batch <= n <= the set's size): layer 0's in_proj, out_proj,
 * linear_in and linear_out, then the text head, each timed over `iters` back-to-back launches
 * with CUDA events on the set's own stream.  us_out[5] receives microseconds per launch and
 * flops_out[5] (may be NULL) the useful work of one launch, 2 * n * rows * in_features.  The
 * products read the set's current input tiles and overwrite its partial-sum scratch, so call
 * this only between steps. */
int stt_debug_time_products(stt_streams* streams, int n, int iters, double* us_out, double* flops_out);

/* Text of the last error on the calling thread ("" if none). */
const char* stt_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* STT_B200_H */
