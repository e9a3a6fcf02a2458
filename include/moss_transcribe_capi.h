/*
 * moss-transcribe C API, version 1, as exported by libmoss_transcribe_b200.so.
 *
 * Same symbols, signatures and ownership rules as the reference header
 * include/moss_transcribe_capi.h:14-60 (loaded with dlopen / cgo / purego):
 *   - the model is loaded once into an opaque context and reused;
 *   - returned strings are malloc'd UTF-8, released with
 *     moss_transcribe_capi_free_string;
 *   - errors are reported through moss_transcribe_capi_last_error;
 *   - no C++ exception crosses the boundary.
 *
 * This library holds the decoder hot path (strict speculative decoding on a
 * B200) and the audio front end before it (log mel, Whisper encoder, adaptor:
 * mtb_audio_encode in include/mtb_decoder.h).  WAV decoding and the tokenizer
 * (prompt ids, transcript text) are not part of it, so the transcribe entries
 * return NULL with a last-error that says so; callers that own a tokenizer
 * encode the audio with mtb_audio_encode and decode prompt ids + audio rows
 * with mtb_spec_generate_ids (or fused rows with mtb_spec_generate).
 */
#ifndef MOSS_TRANSCRIBE_CAPI_H
#define MOSS_TRANSCRIBE_CAPI_H

#ifdef __cplusplus
extern "C" {
#endif

/* replaces src/moss_transcribe_capi.cpp:48-50 (returns 1) */
int moss_transcribe_capi_abi_version(void);

typedef struct moss_transcribe_ctx moss_transcribe_ctx;

/* replaces src/moss_transcribe_capi.cpp:52-72: loads the GGUF decoder onto the
 * CUDA device named by MTB_DEVICE (default 0); NULL on failure. */
moss_transcribe_ctx* moss_transcribe_capi_load(const char* gguf_path);

/* replaces src/moss_transcribe_capi.cpp:74-76; NULL-safe. */
void moss_transcribe_capi_free(moss_transcribe_ctx* ctx);

/* replace src/moss_transcribe_capi.cpp:78-125: NULL + last error (the audio
 * front end is outside this library). */
char* moss_transcribe_capi_transcribe_path(moss_transcribe_ctx* ctx, const char* wav_path, int max_new);
char* moss_transcribe_capi_transcribe_pcm(moss_transcribe_ctx* ctx, const float* samples, int n_samples,
                                          int sample_rate, int max_new);

/* replaces src/moss_transcribe_capi.cpp:127-129; NULL-safe. */
void moss_transcribe_capi_free_string(char* s);

/* replaces src/moss_transcribe_capi.cpp:131-134: "" when ctx is NULL. */
const char* moss_transcribe_capi_last_error(moss_transcribe_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif
