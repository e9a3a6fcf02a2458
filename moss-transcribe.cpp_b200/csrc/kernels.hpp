// Launch wrappers for the sm_100a kernels of the verify step (kernels.cu).
#pragma once

#include "mtb_internal.hpp"

namespace mtb {

// Everything one verify step needs, as device pointers.  Dynamic sizes
// (rows, positions) are read by the kernels from `state`.
struct StepBuffers {
    StepState* state;
    int32_t* ids;           // generated ids [max_new]
    float* x;               // residual [kTMax][hidden]
    float* qkv;             // raw projections [kTMax][(n_heads + 2 n_kv) * 128]
    float* attn_out;        // combined attention [kTMax][n_heads * 128]
    float* gu;              // silu(gate) * up [kTMax][ffn]
    float* hid;             // final-normed hidden [kTMax][hidden]
    uint8_t* act_q;         // quantised activation in mma fragment order [K/32][512]
    float* act_d;           // its block scales [K/32][16]
    float* part_o;          // attention partials [n_kv][max_chunks][kTMax*group][128]
    float2* part_ml;        // (max, sum) per partial
    float2* lm_val;         // LM-head argmax partials (value, index-as-float bits)
    float* logits;          // [kTMax][vocab] (penalty path and tests), may be null
    uint16_t* act_h;        // F16 models: fp16 activation rows [kTMax][max(hidden, n_heads*128, ffn)]
    uint16_t* act_h2;       // F16 models: SwiGLU rows [kTMax][ffn] fp16 (the down projection's input)
    float* f16_part;        // F16 models: per-slice dot totals of split GEMVs (f16_part_floats)
    int* f16_cnt;           // F16 models: finished slice blocks per 32-output group (zero between launches)
    int max_chunks;
    int lm_blocks;          // LM-head partial blocks per row (q8_0: lm_head_blocks; F16: vocab / 32)
};

// Extra buffers of the persistent verify-step kernel.
struct MegaBuffers {
    uint8_t* act2_q;     // SwiGLU fragments (K = ffn)
    float* act2_d;
    float2* lm_val;      // [grid][16] LM-head partials
    unsigned* bar;       // zeroed before every launch, together with abort_flag and head_done
    int* abort_flag;
    unsigned* head_done; // [n_layers][kMaxStreams][n_kv] finished attention items per kv head
    unsigned* pair_done; // [n_layers][n_heads / 2] merged context blocks per pair of q heads
    unsigned* slice_done; // [n_layers][ffn / 256] finished gate/up blocks per 256-feature slice
    unsigned* m_max;     // [n_layers][n_kv][64] running chunk maxima per (kv head, partial row), ordered bits
    size_t zero_bytes;
    unsigned long long* timeline;  // optional, MTB_PROFILE=1 (layout: mtb_step_timeline)
    // Optional, MTB_STEP_CAPTURE=1 (test read-back of the persistent step's own
    // outputs, layout: mtb_step_capture): [16][hidden] final-normed rows, [16]
    // (LM-head maximum, its index as int bits), [kMaxStreams] (rows, first row)
    // as int bits, then the step's row count.
    float* capture = nullptr;
    // Bound on every grid-barrier wait, and a test hook: CTA 0 skips its
    // arrival at this barrier (-1: never), so the others' waits run out.
    unsigned long long wait_ns = 2000000000ull;
    int stall_barrier = -1;
};

constexpr int kMaxBarriers = 512;

// Floats of MegaBuffers::capture for a model of this hidden size.
inline size_t step_capture_floats(int hidden) { return size_t(kTMax) * hidden + 2 * kTMax + 2 * kMaxStreams + 1; }

// Buffers of a prefill pass (up to max_rows prompt rows through all layers at
// once, projections on tcgen05).
struct PrefillBuffers {
    float* x = nullptr;     // [max_rows][hidden] residual rows
    float* qkv = nullptr;   // [max_rows][(n_heads + 2 n_kv) * 128]
    float* attn = nullptr;  // [max_rows][n_heads * 128]
    float* gu = nullptr;    // [max_rows][ffn]
    float* hid = nullptr;   // [max_rows][hidden] final-normed rows
    uint8_t* xq = nullptr;  // activation steps of the widest K
    float* xd = nullptr;    // [max_rows][K / 32]
    float* part_o = nullptr;
    float2* part_ml = nullptr;
    size_t part_rows = 0;   // capacity of part_ml in (row block, kv head, chunk, query row) entries
    int max_rows = 0;
    int* status = nullptr;  // nonzero: a tcgen05 GEMM wait gave up
};

struct KvCache {
    void* base;              // pages of [n_layers][2][n_kv][kPage][128] elements
    const int32_t* pages;    // logical page -> physical page
    int type;                // KvType
    long long page_elems;    // elements per page
    int n_pages;             // pages in the pool (logical positions < n_pages * kPage)
};

// Bounds-check build (-DMTB_BOUNDS_CHECK): each compilation unit records the
// first violated index check here (the site code), skips or redirects the
// access, and its host reader returns and clears it.  0: nothing violated, or
// a normal build (the checks compile to nothing).
enum BcSite : unsigned {
    BC_NONE = 0,
    BC_KV_POSITION = 1,  // a cache position outside the decoder's pages
    BC_KV_PAGE = 2,      // a page-table entry outside the pool
    BC_PARTIALS = 3,     // attention chunks beyond the partial buffers
    BC_STEP_ROWS = 4,    // a step's rows beyond kTMax
};
unsigned bc_take_kernels();
unsigned bc_take_megakernel();
unsigned bc_take_prefill();

struct DeviceModel {
    ModelDims dims;
    LayerWeights* layers;    // host array of device pointers
    const uint8_t* embd;     // token_embd tiles (also the tied LM head)
    const uint8_t* pf_embd;  // token_embd as tcgen05 weight steps (LM head of the persistent step), or null
    const float* output_norm;
    float theta_scale;       // powf(rope_theta, -2/128), computed on the host
    bool f16;                // F16 weights: h_embd and LayerWeights::h_* instead of the q8_0 tiles
    const uint16_t* h_embd;  // F16 models: token_embd [vocab][hidden] fp16 (also the tied LM head)
};

// LM-head partial blocks per row of an F16 model (32 vocab rows per block).
constexpr int kF16Outs = 32;
// Largest projection K of an F16 model.
constexpr int kF16MaxK = 16384;
// Scratch of the F16 GEMVs for a model's shapes: floats of StepBuffers::f16_part
// and ints of StepBuffers::f16_cnt.
size_t f16_part_floats(const ModelDims& d);
int f16_groups_max(const ModelDims& d);

// q8_0 rows -> tiles (src: raw ggml blocks, n_rows x k).  Destination row group
// for source row group r is r * rg_stride + rg_offset.
// Row-major fp16 [n][k] (n a multiple of 32, k of 32) -> the tiled layout of
// the F16 GEMVs and embedding lookups.
void launch_repack_f16(const uint16_t* src, int n, int k, uint16_t* dst, cudaStream_t s);
void launch_repack_q8(const uint8_t* src, int n_rows, int k, uint8_t* dst, int rg_stride, int rg_offset,
                      cudaStream_t s);

// One full verify step for the rows in state->tokens (see decoder.cu).
// `mode`: 0 = draft on device, 1 = host-forced draft already in state,
//         2 = no draft (rows given by the host: prefill chunk or explicit run).
void launch_step(const DeviceModel& m, const KvCache& kv, const StepBuffers& b, int draft_mode,
                 bool want_logits, cudaStream_t s);

// Embedding rows from host-provided float rows instead of token ids
// (prefill and the run() test entry): copies `rows` into x.
// fuse_embeds on the device: token rows from the token_embd tiles, audio rows
// where slot[p] >= 0; out [seq][hidden] (device).
void launch_fuse_embeds(const DeviceModel& m, const int32_t* ids, const int32_t* slot, int seq, const float* audio,
                        float* out, cudaStream_t s);
// One prefill pass: P rows in p.x at positions before .. before + P - 1
// through every layer (tcgen05 projections); the final-normed rows into p.hid
// when want_hidden.  The KV cache receives the P positions.
void launch_prefill_pass(const DeviceModel& m, const KvCache& kv, const PrefillBuffers& p, int P, int before,
                         bool want_hidden, cudaStream_t s);
void launch_forward_rows(const DeviceModel& m, const KvCache& kv, const StepBuffers& b, bool lm_head,
                         bool want_logits, cudaStream_t s);

void launch_fill_synthetic_kv(const DeviceModel& m, const KvCache& kv, int n_pos, uint32_t seed, cudaStream_t s);
void launch_poison_kv(const DeviceModel& m, const KvCache& kv, int pos0, int n_pos, cudaStream_t s);
void launch_kv_gather(const DeviceModel& m, const KvCache& kv, int layer, int which, int pos0, int n_pos,
                      float* out, cudaStream_t s);
// LM head with its first max (b.lm_val) of one final-normed hidden row in
// device memory, as the step's only row (state T = 1).
void launch_lm_row(const DeviceModel& m, const StepBuffers& b, const float* hidden_row, cudaStream_t s);
void launch_logits_row(const DeviceModel& m, const StepBuffers& b, const float* hidden_row, cudaStream_t s);
void launch_prefill_seed(const StepBuffers& b, cudaStream_t s);

// Upper bound of lm_head_blocks(): four blocks per SM of a 148-SM B200 (the
// grid is tuned for that part; other SM counts only change the tuning).
constexpr int kLmHeadMaxBlocks = 148 * 4;
// Slices of 256 K per block of the F16 GEMV for an N x K projection (1, 2 or 4).
int f16_spb(int N, int K);
int lm_head_blocks(int vocab);

// Persistent verify step (megakernel.cu).
int megakernel_smem_bytes();
cudaError_t configure_megakernel(int device, int hidden, int* grid_out);
bool megakernel_supports(const ModelDims& d, int grid);
// TMA tensor map of a KV cache (an opaque CUtensorMap, kept by the decoder).
struct alignas(64) KvTensorMap {
    unsigned char bytes[128];
};
// The map the persistent kernel streams K/V chunk rows with: the cache pool
// (pool_elems elements from kv.base) as [rows][row bytes], swizzled boxes.
cudaError_t encode_kv_map(const KvCache& kv, long long pool_elems, KvTensorMap* out);

cudaError_t launch_step_persistent(const DeviceModel& m, const LayerWeights* layers_dev, const KvCache& kv,
                                   const KvTensorMap& map, const StepBuffers& b, const MegaBuffers& mb, int grid,
                                   cudaStream_t s);
// One persistent launch verifying n_streams decoders of the same model (one
// KV cache, step state and id array each; their drafted rows together at most
// kTMax, the proposals beyond that cut in stream order), with b's activation
// buffers and mb's counters.
cudaError_t launch_step_persistent_group(const DeviceModel& m, const LayerWeights* layers_dev, const KvCache* kvs,
                                         const KvTensorMap* maps, StepState* const* states, int32_t* const* ids,
                                         int n_streams, const StepBuffers& b, const MegaBuffers& mb, int grid,
                                         cudaStream_t s);
// The draft part of a step alone (0: on-device n-gram, 1: host-forced proposal).
void launch_draft(const StepBuffers& b, int draft_mode, cudaStream_t s);
// The device n-gram drafts of a group's members (one block each, the draft of
// launch_draft mode 0), and the group's "every member stopped" flag (1 or 0)
// into *flag: a group step's host work is two launches, not one per member.
struct DraftGroup {
    StepState* st[kMaxStreams];
    const int32_t* ids[kMaxStreams];
    int n;
};
void launch_draft_group(const DraftGroup& g, cudaStream_t s);
void launch_group_stopped(const DraftGroup& g, int* flag, cudaStream_t s);
cudaError_t configure_kernels();
void launch_draft_args(const int32_t* ids, int n, int maximum, int n_min, int n_max, int32_t* out, int* n_out,
                       cudaStream_t s);
void launch_choice_args(const float* logits, int n_raw, const int32_t* hist, int n_hist, float p, int* out,
                        cudaStream_t s);
void launch_rows_begin(const StepBuffers& b, int T, cudaStream_t s);
// LM head + first max of T host-independent device rows into `choices`, with
// every intermediate in caller-provided device scratch (no allocation).
void launch_lm_argmax_rows(const DeviceModel& m, StepState* state, const float* rows, int T, uint8_t* act_q,
                           float* act_d, float2* partials, int32_t* choices, cudaStream_t s);
void launch_set_forced(const StepBuffers& b, const int32_t* src, int n, int vocab, cudaStream_t s);
void launch_rows_end(const StepBuffers& b, cudaStream_t s);

}  // namespace mtb
