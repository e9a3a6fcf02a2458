/*
 * B200 strict speculative decoder: C ABI of the generate layer.
 *
 * This is the boundary the reference's generation layer would call instead of
 * its CPU path.  Each entry replaces one reference interface (paths relative
 * to the moss-transcribe.cpp project root):
 *
 *   mtb_model_load / mtb_model_free      ModelLoader::load (src/model_loader.cpp:21)
 *                                        + Qwen3Decoder::load weight part
 *                                        (src/qwen3_decoder.cpp:20-57)
 *   mtb_decoder_create / _free           Qwen3Decoder::load KV part
 *                                        (src/qwen3_decoder.cpp:59-85)
 *   mtb_decoder_run                      Qwen3Decoder::run / prefill / decode_one
 *                                        (src/qwen3_decoder.cpp:91-172)
 *   mtb_decoder_logits                   Qwen3Decoder::logits_from_hidden (:174-206)
 *   mtb_decoder_rewind / _past_len       CpuSpeculativeDecoder::rewind (src/cpu_speculative.cpp:22-24),
 *                                        Qwen3Decoder::past_len (src/qwen3_decoder.hpp:55)
 *   mtb_greedy_generate                  greedy_generate serial path (src/generate.cpp:235-326)
 *   mtb_spec_generate                    cpu_speculative_generate (src/cpu_speculative.cpp:68-147)
 *                                        with CpuSpeculativeHooks draft/committed
 *                                        (src/cpu_speculative.hpp:9-15)
 *   mtb_ngram_draft                      cpu_ngram_draft (src/cpu_speculative.cpp:27-38),
 *                                        evaluated by the device draft kernel
 *   mtb_greedy_choice                    cpu_greedy_choice (src/cpu_speculative.cpp:39-50),
 *                                        evaluated by the device choice kernel
 *   mtb_spec_step / _async, mtb_resume,  one verify step of the loop body
 *   mtb_spec_prime, mtb_spec_step_group_async, mtb_spec_run_group
 *                                        the same loop for several recordings at once
 *                                        (one launch per step; no reference counterpart:
 *                                        the reference decodes one recording at a time)
 *   mtb_snapshot_save / _restore         (src/cpu_speculative.cpp:100-137)
 *   mtb_audio_load / _encode / _free     AudioEncoder (src/audio_encoder.cpp:16-75): WhisperMel,
 *                                        WhisperEncoder, AudioAdaptor on the device
 *
 * Conventions: every function returns 0 on success or a negative code and
 * sets a per-object error string; no C++ exception crosses the boundary.  One
 * decoder is one CUDA device and one stream; decoders on different devices
 * may be driven from different host threads.  There is no CPU fallback: on a
 * host without a usable GPU, mtb_model_load fails with an error.
 */
#ifndef MTB_DECODER_H
#define MTB_DECODER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mtb_model mtb_model;
typedef struct mtb_decoder mtb_decoder;

/* KV cache element type; MTB_KV_DEFAULT reads MTB_KV_DTYPE ("f16" or "f32",
 * unset: f32, the reference's cache type, src/qwen3_decoder.cpp:67-75). */
enum { MTB_KV_DEFAULT = -1, MTB_KV_F32 = 0, MTB_KV_F16 = 1 };
enum { MTB_STOP_NONE = 0, MTB_STOP_EOS = 1, MTB_STOP_LIMIT = 2, MTB_STOP_ERROR = 3 };

/* Draft policy.  The reference policy is k_max 4, n-gram sizes 16..2
 * (src/cpu_speculative.cpp:29,104); penalty clamped to [1, 1.5] (:85-86).  A
 * NULL params pointer selects mtb_spec_params_from_env: that policy with the
 * penalty read from MTD_REPETITION_PENALTY, as the reference does, and k_max /
 * n_min / n_max overridable by MTB_SPEC_K / MTB_NGRAM_MIN / MTB_NGRAM_MAX. */
typedef struct mtb_spec_params {
    int32_t k_max;   /* proposals per step, 0..15 */
    int32_t n_min;   /* smallest n-gram size, >= 1 */
    int32_t n_max;   /* largest n-gram size */
    float penalty;   /* repetition penalty over the last 100 ids */
} mtb_spec_params;

/* Counters of the CPU_SPECULATIVE log line (src/cpu_speculative.cpp:140). */
typedef struct mtb_counters {
    int64_t target_calls, drafted_calls, proposed, accepted, target_input_tokens, rewinds;
    int32_t stop_reason; /* MTB_STOP_* */
    int32_t past_len;
} mtb_counters;

/* Mirrors CpuSpeculativeHooks::draft: write at most `budget` ids, return count. */
typedef int (*mtb_draft_fn)(void* user, const int32_t* ids, int n_ids, int budget, int32_t* out);
/* Mirrors CpuSpeculativeHooks::committed: after every commit. */
typedef void (*mtb_commit_fn)(void* user, const int32_t* ids, int n_ids, int past_len, int stopped);

int mtb_abi_version(void);
/* Whether moss_transcribe_capi_transcribe_pcm / _path can return a
 * transcript from this build: 0 (WAV decoding and the tokenizer are not part
 * of it; those calls return NULL with an error).  No counterpart in the
 * reference. */
int mtb_capi_can_transcribe(void);
/* The generate entries (mtb_spec_generate, mtb_spec_generate_ids,
 * mtb_greedy_generate) end by printing the reference's lines
 * (src/cpu_speculative.cpp:138-145) to stderr as "[mt I] <line>":
 * BENCH_GENERATION, CPU_PROFILE, CPU_SPECULATIVE and, with
 * MTD_TRACE_TOKENS=1 in the environment, BENCH_TOKEN_TRACE in chunks of 128
 * ids.  level 0 silences them, 1 (the default) prints them. */
void mtb_set_log_level(int level);
/* The same lines as text (no prefix, '\n' after each) for given results;
 * needs no GPU.  Returns the full length; out gets at most out_size - 1 bytes
 * and a terminating 0. */
int mtb_format_generation_log(const int32_t* ids, int n_ids, int eos, const mtb_counters* counters, int k_max,
                              double prefill_seconds, double decoder_seconds, int trace, char* out, int out_size);
/* The policy a NULL params pointer selects (see mtb_spec_params); needs no
 * GPU.  Unparsable or out-of-range variables are reported here (-1, with
 * mtb_global_error) rather than clamped. */
int mtb_spec_params_from_env(mtb_spec_params* out);
/* MTB_KV_F32 or MTB_KV_F16 as MTB_KV_DTYPE selects (unset: MTB_KV_F32), -1 for
 * an unknown value; needs no GPU. */
int mtb_kv_type_from_env(void);
/* 256-K slices per block the F16 GEMV uses for an n x k projection on the
 * device configured last (1, 2 or 4; -1 for an invalid shape), so tests can
 * check which block shapes a model's projections reach. */
int mtb_f16_slices_per_block(int n, int k);
/* Test hook (host-side fault injection): the n-th device allocation made by
 * this library from now on fails as if cudaMalloc had (n = 0: off).  The
 * failing call returns its error and leaves no allocation behind. */
void mtb_debug_fail_alloc(int n);
/* Bounds-check build (libmoss_transcribe_b200_bc.so, -DMTB_BOUNDS_CHECK):
 * the kernels check cache positions, page-table entries, the attention
 * partial buffers and step row counts, record the first violated check on the
 * device and skip or redirect that access (no trap).  _enabled: 1 in that
 * build, 0 otherwise.  _status: the recorded site on `device` (0 none, 1 a
 * cache position outside the decoder's pages, 2 a page-table entry outside
 * the pool, 3 attention chunks beyond the partial buffers, 4 a step beyond 16
 * rows), then cleared; always 0 in a normal build; -1 if the device cannot be
 * selected.  Restores the caller's current device. */
int mtb_bounds_check_enabled(void);
int mtb_bounds_check_status(int device);
/* Returns the error of the last failed call on this thread that had no object. */
const char* mtb_global_error(void);

/* ---- model: decoder weights resident on one device ---- */
int mtb_model_load(const char* gguf_path, int device, mtb_model** out);
void mtb_model_free(mtb_model* m);
const char* mtb_model_error(const mtb_model* m);
/* hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab, eos */
int mtb_model_dims(const mtb_model* m, int32_t* out8);
/* CTAs of the persistent verify-step kernel (one per SM), or 0 when verify
 * steps run as a graph of separate kernels (unsupported shape, repetition
 * penalty > 1, or MTB_NO_PERSISTENT set at load). */
int mtb_model_persistent_grid(const mtb_model* m);

/* ---- decoder: KV cache (paged, 64 positions per page) and step state ---- */
int mtb_decoder_create(mtb_model* m, int max_seq, int kv_type, int max_new, mtb_decoder** out);
void mtb_decoder_free(mtb_decoder* d);
const char* mtb_decoder_error(const mtb_decoder* d);
int mtb_decoder_past_len(const mtb_decoder* d);
int mtb_decoder_reset(mtb_decoder* d);
int mtb_decoder_rewind(mtb_decoder* d, int position);
/* Append T host rows [T][hidden] at past..past+T-1 (any T; chunks of 16),
 * writing the final-RMSNorm'd hidden rows to hidden_out [T][hidden] (may be NULL). */
int mtb_decoder_run(mtb_decoder* d, const float* embeds, int T, float* hidden_out);
/* Tied LM head on one host hidden row -> logits[vocab]. */
int mtb_decoder_logits(mtb_decoder* d, const float* hidden_row, float* logits);
/* KV rows of one layer (which 0 = K, 1 = V) as f32 [n_pos][n_kv][128]. */
int mtb_decoder_kv_read(mtb_decoder* d, int layer, int which, int pos0, int n_pos, float* out);
/* Synthetic fp16-valued KV at positions [0, n_pos) of every layer; sets past_len. */
int mtb_decoder_fill_synthetic_kv(mtb_decoder* d, int n_pos, uint32_t seed);

/* ---- generation ---- */
int mtb_greedy_generate(mtb_decoder* d, const float* fused, int seq, int max_new, int eos, float penalty,
                        int32_t* out_ids, int* n_out);
int mtb_spec_generate(mtb_decoder* d, const float* fused, int seq, int max_new, int eos,
                      const mtb_spec_params* params, int32_t* out_ids, int* n_out, mtb_counters* counters,
                      mtb_draft_fn draft, mtb_commit_fn commit, void* user);

/* fuse_embeds (src/generate.cpp:113-177) on the device: row p of out
 * [seq][hidden] (host) is the dequantised token_embd row of ids[p], except that
 * the k-th position holding audio_token_id takes audio row k (masked scatter).
 * Errors as the reference: an id outside [0, vocab), or more audio positions
 * than audio rows; fewer positions than rows is accepted. */
int mtb_fuse_embeds(mtb_decoder* d, const int32_t* ids, int seq, const float* audio, int n_audio, int audio_token_id,
                    float* out);
/* mtb_spec_generate from token ids + audio rows: the fused prompt is built on
 * the device (mtb_fuse_embeds) and prefilled from device memory, so it never
 * round-trips the host (generate.cpp:229-241 fuse_embeds + greedy_generate). */
int mtb_spec_generate_ids(mtb_decoder* d, const int32_t* ids, int seq, const float* audio, int n_audio,
                          int audio_token_id, int max_new, int eos, const mtb_spec_params* params, int32_t* out_ids,
                          int* n_out, mtb_counters* counters);

/* Continue from an existing cache: ids[0:n_ids] are the generated ids (the
 * last is the pending seed, not yet in the cache), past the cache length. */
int mtb_resume(mtb_decoder* d, const int32_t* ids, int n_ids, int past, int max_new, int eos,
               const mtb_spec_params* params);
/* One verify step.  draft == NULL -> on-device n-gram draft; otherwise the
 * n_draft host ids are the proposal.  Synchronous; new ids via mtb_read_ids. */
int mtb_spec_step(mtb_decoder* d, const int32_t* draft, int n_draft, mtb_counters* counters);
/* Same, asynchronous on the decoder's stream, proposal from DEVICE memory
 * (NULL -> on-device draft).  Nothing is copied to or from the host. */
int mtb_spec_step_async(mtb_decoder* d, const int32_t* draft_device, int n_draft);
/* Set the decode parameters and prefill the fused rows (the first id is
 * emitted), without decoding: the start of mtb_spec_generate
 * (src/cpu_speculative.cpp:68-99), for decoders stepped as a group.  Returns
 * once the prefill is queued on the decoder's stream (the rows have been
 * copied out of `fused`), so the members of a group prefill side by side; a
 * prefill that fails on the device is reported by the next call that reads
 * the decoder's state back (mtb_spec_run_group, mtb_read_ids, ...). */
int mtb_spec_prime(mtb_decoder* d, const float* fused, int seq, int max_new, int eos, const mtb_spec_params* params);
/* One verify step of n decoders (1..8) created from the same model, as ONE
 * persistent launch: each decoder drafts on the device; their rows (seed +
 * proposals, at most 16 together) are verified against their own KV caches;
 * each accepts and rolls back on its own.  Proposals beyond the 16 rows are
 * cut in group order (the accepted ids do not change: verification is strict
 * greedy; only the proposal counters do).  ds[0] needs the largest max_seq;
 * no repetition penalty.  Asynchronous: ordered after the work queued on every
 * member's stream and before the work queued on it later. */
int mtb_spec_step_group_async(mtb_decoder* const* ds, int n);
/* Group steps until every member has stopped (max_steps <= 0: no limit),
 * then synchronous; steps_out = steps launched.  New ids via mtb_read_ids. */
int mtb_spec_run_group(mtb_decoder* const* ds, int n, int max_steps, int* steps_out);
/* Device-side copy of the step state and ids (save) and back (restore),
 * asynchronous on the decoder's stream. */
int mtb_snapshot_save(mtb_decoder* d);
int mtb_snapshot_restore_async(mtb_decoder* d);
int mtb_read_ids(mtb_decoder* d, int32_t* out, int max_out, int* n_out, mtb_counters* counters);

/* ---- timing on the decoder's stream ---- */
int mtb_sync(mtb_decoder* d);
int mtb_event_record(mtb_decoder* d, int slot);          /* slot 0..15 */
int mtb_event_elapsed_ms(mtb_decoder* d, int a, int b, float* ms);
/* Kernel launches per verify step (counted when the step graph is built). */
int mtb_step_kernel_launches(mtb_decoder* d);
/* Timeline of the last persistent verify step (decoder created with
 * MTB_PROFILE=1 in the environment): out[2b], out[2b+1] = CTA 0's arrival and
 * release at grid barrier b, out[2*512], out[2*512+1] = kernel start and end,
 * out[2*512 + 2 + 4b + k] = sub-phase mark k of phase b (0 when unused),
 * out[6*512 + 2 + 512 c + b] = CTA c's arrival at barrier b,
 * out[6*512 + 2 + 256*512 + 16 (512 c + b) + k] = CTA c's sub-phase mark k of
 * phase b (c < 256, k < 16), all in ns of the
 * GPU global timer; the profile counterpart of the
 * reference's MTD_PROFILE phase timers (src/cpu_profile.cpp:23-68). */
int mtb_step_timeline(mtb_decoder* d, int64_t* out, int max_out, int* n_out);
/* Test read-back of the last persistent verify step's own outputs (decoder
 * created with MTB_STEP_CAPTURE=1 in the environment; for a group step, the
 * group's first decoder): the step's T rows (all streams, stream order) as
 * final-RMSNorm'd hidden rows hidden_out [T][hidden], each row's LM-head
 * maximum max_val[T] and its first index max_idx[T], and per stream
 * (rows, first row) in stream_rows[8][2].  Any output may be NULL. */
int mtb_step_capture(mtb_decoder* d, float* hidden_out, float* max_val, int32_t* max_idx, int32_t* stream_rows,
                     int* T_out);
/* Test hook: NaN into KV positions [pos0, pos0 + n_pos) of every layer (K and
 * V), to show that a step never reads a cache slot it has not written. */
int mtb_debug_poison_kv(mtb_decoder* d, int pos0, int n_pos);
/* Host<->device bytes this decoder has copied so far (both cumulative). */
int mtb_transfer_bytes(mtb_decoder* d, int64_t* h2d, int64_t* d2h);

/* ---- controller pieces, run by the same device kernels the loop uses ---- */
/* history: n host ids (n <= the decoder's max_new); out: up to `maximum` ids. */
int mtb_ngram_draft(mtb_decoder* d, const int32_t* history, int n, int maximum, int n_min, int n_max,
                    int32_t* out, int* n_out);
/* raw: n_raw host logits (n_raw <= vocab); history: n host ids. */
int mtb_greedy_choice(mtb_decoder* d, const float* raw, int n_raw, const int32_t* history, int n, float penalty,
                      int32_t* choice);

/* ---- LM head without device allocation ----
 * No counterpart in the reference (its LM head, Qwen3Decoder::logits_from_hidden,
 * allocates a ggml graph per call).  For callers that cannot allocate device
 * memory: serving processes that give all free device memory to their own pool
 * allocator at start-up and forbid later cudaMalloc, because a late cudaMalloc
 * can fail for lack of room and cudaMalloc/cudaFree synchronise the device.
 *
 * hidden_rows: DEVICE pointer to T final-normed hidden rows [T][hidden];
 * choices: DEVICE pointer to T int32, receives each row's first-max token id
 * (mtb_greedy_choice without penalty).  stream: a cudaStream_t, NULL for the
 * default stream; the call is asynchronous on it.  Limits: T in [1, 16],
 * hidden <= 4096; larger sizes return -2 with mtb_noalloc_error() set.
 * Intermediates live in one static device array of about 148 KB that every
 * device loading this library holds until exit; the first call on a device
 * looks its address up (call it once before any stream capture).  Calls share
 * that array: calls that overlap on the GPU race.  Nothing is allocated: no
 * cudaMalloc, cudaFree or allocating library routine is called.  The call runs
 * on the model's device and leaves the caller's current device as it found it. */
int mtb_lm_head_argmax_noalloc(const mtb_model* m, const float* hidden_rows, int T, int32_t* choices, void* stream);
const char* mtb_noalloc_error(void);

/* ---- Audio front end: 16 kHz samples -> the decoder's audio embedding rows ----
 * Replaces mt::AudioEncoder (src/audio_encoder.hpp:23-34, src/audio_encoder.cpp:16-75):
 * WhisperMel::compute (src/mel.cpp:153-224), WhisperEncoder::encode
 * (src/whisper_encoder.cpp:98-207) and AudioAdaptor::apply
 * (src/audio_adaptor.cpp:39-96), all on the device.  The GGUF is the one the
 * decoder loads (mtd.audio.*, mtd.feat.*, mel_filters, enc.*, adaptor.*);
 * the encoder and adaptor linear weights must be q8_0. */
typedef struct mtb_audio mtb_audio;
int mtb_audio_load(const char* gguf_path, int device, mtb_audio** out);
void mtb_audio_free(mtb_audio* a);
/* The object's last error, or the last load error of this thread for NULL. */
const char* mtb_audio_error(const mtb_audio* a);
/* dims[10]: hidden, d_model, n_layers, n_heads, ffn, n_mels, mel frames per
 * chunk, samples per chunk, encoder frames per chunk, merge size. */
int mtb_audio_dims(const mtb_audio* a, int32_t* dims);
/* Sum over 30 s chunks of token_len = (unpadded - 1) / (hop * 2 * merge) + 1:
 * the rows mtb_audio_encode returns for n_samples samples. */
int mtb_audio_tokens(const mtb_audio* a, int n_samples);
/* AudioEncoder::encode: host samples -> host rows out[n_tokens][hidden]
 * (max_tokens rows available).  Empty input and a too-small output are
 * errors, as in the reference. */
int mtb_audio_encode(mtb_audio* a, const float* samples16k, int n_samples, float* out, int max_tokens,
                     int* n_tokens);
/* Device time of the last mtb_audio_encode (host copies included), ms. */
float mtb_audio_last_ms(const mtb_audio* a);
/* Test read-back of one chunk: mel [n_mels][frames] (after the chunk
 * normalisation) and the encoder output [encoder frames][d_model] (after the
 * final LayerNorm, before the trim); n_samples <= samples per chunk (the rest
 * is zero-padded as in encode); either output may be NULL. */
int mtb_audio_debug_chunk(mtb_audio* a, const float* samples, int n_samples, float* mel_out, float* enc_out);

#ifdef __cplusplus
}
#endif
#endif
