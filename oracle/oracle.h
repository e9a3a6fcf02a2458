/*
 * CPU oracle for the strict speculative decode path of moss-transcribe.cpp.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is
 * compared against.  Only tests/, __graft_entry__.smoke() and the cpu_baseline
 * leg of bench.py may load it.  The product library never links it and has no
 * CPU fallback.
 *
 * What it restates (reference paths are relative to the moss-transcribe.cpp
 * project root):
 *   - src/cpu_speculative.cpp:27-38    n-gram draft (latest match, longest n first)
 *   - src/cpu_speculative.cpp:39-50    greedy choice (first max, recent-100 penalty)
 *   - src/cpu_speculative.cpp:68-147  strict speculative controller, counters,
 *                                      lazy per-row logits, logical rewind
 *   - src/generate.cpp:235-326         serial greedy generate
 *   - src/generate.cpp:33-66           q8_0 row dequant for the embedding lookup
 *   - src/qwen3_decoder.cpp:91-206     run(T): positions, causal mask, final norm,
 *                                      tied LM head
 *   - src/qwen3.cpp:62-218             one Qwen3 layer (norm, QKV, QK-norm, NEOX
 *                                      RoPE, KV store, GQA attention, O, SwiGLU)
 *   - src/cpu_context.cpp:13-33        P.V over the per-query valid length
 *   - src/cpu_softmax.cpp:26-36        scale, max, exp with a double sum, 1/sum
 *
 * The arithmetic of the ops above lives in ggml (commit eced84c, an
 * un-vendored submodule that is absent from the reference tree).  The oracle
 * restates ggml's published CPU algorithms:
 *   - q8_0 activation quantisation (x86 SIMD from_float): d = amax/127 stored as
 *     fp16 (round to nearest even), codes = round_half_even(x * (127/amax));
 *   - q8_0 weight quantisation (quantize_row_q8_0_ref, the algorithm of the
 *     gguf Python package the reference converter calls): codes =
 *     round_half_away(x * (1/d));
 *   - q8_0 x q8_0 dot: exact integer sum per 32-block scaled by
 *     fp32(d_w)*fp32(d_x) and accumulated in fp32;
 *   - rms_norm: sum of float squares accumulated in double, scale =
 *     1/sqrtf(mean + eps), y = (x*scale)*w;
 *   - NEOX rope: theta advanced by repeated float multiplication with
 *     powf(base, -2/n_dims), pairs (i, i + n_dims/2);
 *   - soft_max_ext: softmax(x*scale + causal mask), then P.V over the valid
 *     length.
 *
 * Evaluation order.  ggml's float summation order differs between its own
 * ISA paths (x86 lanes, ARM, the llamafile kernels), and a random-init q8_0
 * network amplifies any reordering: one ulp moves an activation code, which
 * the next layers carry on.  So this oracle fixes one documented order, and
 * the CUDA kernels evaluate exactly the same operations in the same order,
 * which makes the two bit-identical: q8_0 dots in 256-element slices (fmaf
 * per block, slices added in order); squares summed in the kernels' tree
 * (sum_squares_tree); softmax per 64-position chunk, merged with
 * exp(m_c - M); exp/sin/cos are this library's own (orc_expf, orc_sincosf:
 * Cody-Waite reduction and Taylor series in double).
 *
 * Parity status: the draft and greedy-choice functions are pinned by the 12
 * known-answer controls of tests/test_cpu_speculative.cpp and by vectors made
 * with the reference's own Python replay tool (cpu-lab/moss_ngram_audit.py);
 * the q8_0 weight bytes by the gguf package the reference converter calls.
 * The decoder's floating-point arithmetic is PARITY UNPINNED against ggml
 * itself: ggml is not on disk and the reference's golden GGUFs are not in the
 * tree, so the float ops above are restated from ggml's published algorithms
 * and have not been run against the reference binary.
 */
#ifndef MTB_ORACLE_H
#define MTB_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids used by the fixtures. */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8 };

typedef struct orc_model orc_model;
typedef struct orc_decoder orc_decoder;

typedef struct orc_counters {
    int64_t target_calls, drafted_calls, proposed, accepted, target_input_tokens, rewinds;
    int32_t stop_reason; /* 0 = error, 1 = eos, 2 = token_limit */
    int32_t pad;
} orc_counters;

/* A forced-proposal hook: mirrors CpuSpeculativeHooks::draft
 * (src/cpu_speculative.hpp:11).  Writes at most `budget` ids to `out` and
 * returns the count. */
typedef int (*orc_draft_fn)(void* user, const int32_t* ids, int n_ids, int budget, int32_t* out);
/* Mirrors CpuSpeculativeHooks::committed (src/cpu_speculative.hpp:14): called
 * after every commit with the decoder's logical length. */
typedef void (*orc_commit_fn)(void* user, const int32_t* ids, int n_ids, int past_len, int stopped);

/* ---- model ---- */
orc_model* orc_model_create(int hidden, int n_layers, int n_heads, int n_kv_heads, int head_dim,
                            int ffn, int vocab, float rms_eps, float rope_theta);
void orc_model_free(orc_model* m);
/* Attach a tensor by its GGUF name; the data is borrowed (the caller keeps it
 * alive).  type is ORC_F32 / ORC_F16 / ORC_Q8_0.  Returns 0 on success. */
int orc_model_set_tensor(orc_model* m, const char* name, const void* data, int type);
/* Returns 0 when every tensor the decoder needs is attached. */
int orc_model_check(const orc_model* m);

/* ---- decoder state (F32 KV, optionally rounded through fp16 on store) ---- */
orc_decoder* orc_decoder_create(const orc_model* m, int max_seq, int kv_fp16);
void orc_decoder_free(orc_decoder* d);
int orc_decoder_past_len(const orc_decoder* d);
void orc_decoder_reset(orc_decoder* d);
int orc_decoder_rewind(orc_decoder* d, int position);
/* run(T): append T embedding rows at positions past..past+T-1, write the final
 * RMSNorm'd hidden rows [T][hidden].  Returns 0 on success. */
int orc_decoder_run(orc_decoder* d, const float* embeds, int T, float* out_hidden);
/* Tied LM head on one hidden row -> logits[vocab]. */
void orc_decoder_logits(const orc_decoder* d, const float* hidden_row, float* logits);
/* KV access for tests: layer-major, [n_pos][n_kv_heads][head_dim] floats. */
int orc_decoder_kv_read(const orc_decoder* d, int layer, int which, int pos0, int n_pos, float* out);
int orc_decoder_kv_write(orc_decoder* d, int layer, int which, int pos0, int n_pos, const float* in);
/* Fill positions [0, n_pos) of every layer with the deterministic synthetic
 * values of orc_synthetic_kv_value and set past_len = n_pos. */
int orc_decoder_fill_synthetic_kv(orc_decoder* d, int n_pos, uint32_t seed);
/* The synthetic value for element (layer, which, pos, head, dim): an
 * Irwin-Hall(4) approximation of N(0,1) from a 32-bit integer hash, rounded
 * to fp16 and returned as float.  The CUDA library implements the same. */
float orc_synthetic_kv_value(uint32_t seed, int layer, int which, int pos, int head, int dim);

/* ---- embedding lookup (q8_0 row dequant) ---- */
int orc_embed_rows(const orc_model* m, const int32_t* ids, int n, float* out);

/* ---- controller ---- */
int orc_ngram_draft(const int32_t* history, int n, int maximum, int n_min, int n_max, int32_t* out);
int orc_greedy_choice(const float* raw, int vocab, const int32_t* history, int n, float penalty);
/* Strict speculative generate (src/cpu_speculative.cpp:68-147) with the draft
 * policy made explicit: at most k_max proposals, n-gram sizes n_max..n_min.
 * Returns the number of ids written (including a trailing EOS), -1 on error. */
int orc_spec_generate(orc_decoder* d, const float* fused, int seq, int max_new, int eos,
                      int k_max, int n_min, int n_max, float penalty,
                      int32_t* out_ids, orc_counters* counters,
                      orc_draft_fn draft, orc_commit_fn commit, void* user);
/* Serial greedy generate (src/generate.cpp:235-326). */
int orc_greedy_generate(orc_decoder* d, const float* fused, int seq, int max_new, int eos,
                        float penalty, int32_t* out_ids);

/* ---- q8_0 arithmetic ---- */
void orc_quantize_act_q8(const float* x, int64_t k, void* out_blocks);
void orc_quantize_ref_q8(const float* x, int64_t k, void* out_blocks);
void orc_mul_mat_q8(const void* w_blocks, int n_rows, int k, const float* x, int T, float* y);
/* The same for f16 weights [n_rows x k]: x rounded to fp16, exact products,
 * 32-element fmaf chains, blocks then 256-element slices added in order. */
void orc_mul_mat_f16(const void* w_half, int n_rows, int k, const float* x, int T, float* y);

/* TEST ONLY: the same decoder in the reference's own evaluation order (ggml's
 * x86 dot orders, whole-row softmax with the sum in double, P.V over the
 * valid length, libm expf/sinf/cosf), q8_0 models only.  Used to bound how far
 * this oracle's evaluation order sits from the reference's arithmetic. */
int orc_decoder_run_ref(orc_decoder* d, const float* embeds, int T, float* out_hidden);
void orc_decoder_logits_ref(const orc_decoder* d, const float* hidden_row, float* logits);
/* TEST ONLY: one attention row over K, V [valid][hd] in this oracle's order
 * (ref_order 0) or the reference's (1); one q8_0 x q8_0 dot of nb blocks in
 * either order. */
void orc_attention_row(int ref_order, const float* q, const float* k, const float* v, int valid, int hd, float* out);
float orc_dot_q8_blocks(int ref_order, const void* w, const void* x, int nb);
void orc_set_threads(int n);
/* The exp / sin / cos the oracle (and the CUDA kernels) evaluate. */
float orc_expf(float x);
/* erf by its Maclaurin series in double (the kernels' exact_erff). */
float orc_erff(float x);
void orc_sincosf(float x, float* s, float* c);

/* Audio front end (src/mel.cpp:153-224, src/whisper_encoder.cpp:98-207,
 * src/audio_adaptor.cpp:39-96, src/audio_encoder.cpp:16-75).  cfg: n_fft, hop,
 * n_mels, samples per chunk, mel frames per chunk, d_model, n_layers, n_heads,
 * ffn, merge, hidden.  Tensors are kept by pointer (the caller owns them):
 * F32 arrays, q8_0 rows for the encoder and adaptor linears.  The mel is in the
 * reference's own order; the encoder and adaptor in the CUDA kernels' order (in
 * the reference's order -- ggml's dot orders, sequential norms, whole-row
 * softmax, libm exp/erf -- with orc_audio_set_ref_order(a, 1)). */
typedef struct orc_audio orc_audio;
orc_audio* orc_audio_create(const int* cfg, float adaptor_eps);
void orc_audio_free(orc_audio* a);
void orc_audio_set_ref_order(orc_audio* a, int ref_order);
int orc_audio_set_tensor(orc_audio* a, const char* name, const void* data);
void orc_audio_mel(const orc_audio* a, const float* chunk, float* mel);
int orc_audio_encoder(const orc_audio* a, const float* mel, float* out);
int orc_audio_adaptor(const orc_audio* a, const float* enc, int frames, float* out);
int orc_audio_encode(const orc_audio* a, const float* samples, int n, float* out, int max_tokens);

#ifdef __cplusplus
}
#endif
#endif
