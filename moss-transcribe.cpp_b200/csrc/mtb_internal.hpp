// Internal types shared by the CUDA kernels and the host runtime.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace mtb {

constexpr int kHeadDim = 128;   // Qwen3 head_dim (src/model_loader.cpp:124)
constexpr int kTMax = 16;       // rows per verify step: seed + up to 15 proposals
constexpr int kQ8Block = 32;    // q8_0 block (34 bytes: fp16 d + 32 int8)
constexpr int kTileRows = 8;    // weight rows per tile (the mma N dimension)
constexpr int kTileK = 64;      // K per tile (two q8_0 blocks)
constexpr int kTileBytes = 544; // 512 code bytes + 16 fp16 scales = 16 q8_0 blocks
constexpr int kPage = 64;       // KV positions per page (= attention chunk)
constexpr int kMaxStreams = 8;  // decoders verified in one persistent launch (their rows share the 16)

enum KvType : int { KV_F32 = 0, KV_F16 = 1 };

enum StopReason : int { STOP_NONE = 0, STOP_EOS = 1, STOP_LIMIT = 2, STOP_ERROR = 3 };

// Device-resident generation state.  Every step kernel reads its dynamic
// sizes from here, so one captured launch sequence serves every step.
struct StepState {
    int past;        // logical KV length (Qwen3Decoder::past_len_)
    int n_ids;       // generated ids so far (including the pending seed)
    int max_new, eos, k_max, n_min, n_max, max_seq;
    float penalty;
    int stop;        // StopReason
    int seed;        // last emitted id, not yet in the cache
    int T;           // active rows this step (0 when stopped)
    int n_prop;      // proposals this step
    int before;      // past at step start
    int forced;      // 1: tokens[1..] were written by the host (draft hook)
    int error;
    int commit_n;    // ids at the last commit (before the next seed is emitted)
    int commit_stop; // stop status at that commit
    int tokens[kTMax];
    int choice[kTMax];
    long long target_calls, drafted_calls, proposed, accepted, target_input_tokens, rewinds;
};

struct LayerWeights {
    const uint8_t* qkv;    // tiles, rows: q (n_heads*128), k, v (n_kv*128 each)
    const uint8_t* o;      // tiles, rows: hidden, K = n_heads*128
    const uint8_t* gu;     // tiles, row groups interleaved gate/up
    const uint8_t* down;   // tiles, rows: hidden, K = ffn
    const float *attn_norm, *q_norm, *k_norm, *ffn_norm;
    // The same matrices as prefill weight steps (tcgen05 operand layout, prefill_tc.cu).
    const uint8_t *pf_qkv, *pf_o, *pf_gu, *pf_down;
    // F16 models instead: row-major fp16 [rows][K], q|k|v and gate|up rows concatenated.
    const uint16_t *h_qkv, *h_o, *h_gu, *h_down;
};

struct ModelDims {
    int hidden, n_layers, n_heads, n_kv, ffn, vocab;
    float eps, theta;
};

}  // namespace mtb
