// Host runtime of the B200 strict speculative decoder (C ABI in
// include/mtb_decoder.h).
//
// Model: GGUF -> q8_0 tiles in HBM (ModelLoader::load + Qwen3Decoder::load,
// src/model_loader.cpp:21-114, src/qwen3_decoder.cpp:20-85).  Decoder: paged
// KV cache, device StepState, step buffers and the CUDA graphs of the verify
// step.  The generation loop (src/cpu_speculative.cpp:68-147) runs on the
// device: drafting, the verify forward, the LM-head first max, acceptance and
// rollback are kernels of one captured graph, and the host only watches the
// stop flag.  With draft/commit hooks the loop runs one step per host round
// trip so the hooks see every proposal and commit.
#include "../../include/mtb_decoder.h"
#include "gguf.hpp"
#include "kernels.hpp"
#include "prefill_tc.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <atomic>
#include <climits>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

using namespace mtb;

namespace {
thread_local std::string g_error;

constexpr int kAbiVersion = 1;
}  // namespace

struct mtb_model {
    int device = 0;
    DeviceModel dm{};
    std::vector<LayerWeights> layers;
    LayerWeights* layers_dev = nullptr;  // device copy for the persistent kernel
    int mega_grid = 0;                   // 0: the persistent kernel is not used
    std::vector<void*> allocs;
    std::string error;
    int eos = -1;
    ~mtb_model() {
        cudaSetDevice(device);
        for (void* p : allocs) cudaFree(p);
    }
};

struct mtb_decoder {
    mtb_model* model = nullptr;
    int device = 0;
    cudaStream_t stream = nullptr;
    int max_seq = 0, kv_type = 0, max_new = 0;
    KvCache kv{};
    KvTensorMap kv_map{};  // the cache for the persistent kernel's TMA tiles
    StepBuffers b{};
    MegaBuffers mb{};
    PrefillBuffers pf{};
    StepState* h_state = nullptr;  // pinned mirror
    float* h_rows = nullptr;       // pinned staging [kTMax][hidden]
    int32_t* h_ids = nullptr;      // pinned [max_new]
    int* h_flag = nullptr;         // pinned [2]
    int* h_pf_status = nullptr;    // pinned: a deferred prefill's status word (pf_status_pending)
    bool pf_status_pending = false;
    int* group_flag = nullptr;     // device [2]: a group run's "every member stopped", one per step parity
    StepState* snap_state = nullptr;
    int32_t* snap_ids = nullptr;
    int32_t* scratch_i = nullptr;  // [max_new + 16]
    int* scratch_n = nullptr;
    float* row_buf = nullptr;      // [hidden]
    // Device fuse_embeds buffers, allocated on first use: fused rows [max_seq][hidden],
    // ids + audio slots [2][max_seq], audio rows [max_seq][hidden].
    float* fused_dev = nullptr;
    int32_t* fuse_ids = nullptr;
    float* fuse_audio = nullptr;
    cudaGraphExec_t graphs[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};
    int launches = 0;
    long long h2d_bytes = 0, d2h_bytes = 0;  // host<->device bytes this decoder has issued
    cudaEvent_t ev[16] = {};
    cudaEvent_t group_ev = nullptr;  // orders a group step against this decoder's stream
    // The pinned step-state mirror equals the device state (no device work since
    // the last read-back or synchronised push): refresh() need not read it again.
    bool fresh = false;
    std::vector<void*> allocs;
    std::string error;
    ~mtb_decoder() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (auto& row : graphs)
            for (auto& g : row)
                if (g) cudaGraphExecDestroy(g);
        for (auto& e : ev)
            if (e) cudaEventDestroy(e);
        if (group_ev) cudaEventDestroy(group_ev);
        for (void* p : allocs) cudaFree(p);
        if (h_state) cudaFreeHost(h_state);
        if (h_rows) cudaFreeHost(h_rows);
        if (h_ids) cudaFreeHost(h_ids);
        if (h_flag) cudaFreeHost(h_flag);
        if (h_pf_status) cudaFreeHost(h_pf_status);
        if (stream) cudaStreamDestroy(stream);
    }
};

#define MTB_CK(obj, call)                                                                          \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) {                                                                   \
            (obj)->error = std::string(#call) + ": " + cudaGetErrorString(e_);                      \
            return -1;                                                                             \
        }                                                                                          \
    } while (0)

namespace {

// Allocation fault injection (mtb_debug_fail_alloc): counts down to the
// allocation that fails.
std::atomic<int> g_fail_alloc{0};

cudaError_t device_malloc(void** q, size_t bytes) {
    int n = g_fail_alloc.load();
    while (n > 0 && !g_fail_alloc.compare_exchange_weak(n, n - 1)) {
    }
    if (n == 1) return cudaErrorMemoryAllocation;
    return cudaMalloc(q, bytes);
}

template <class T>
int dalloc(std::vector<void*>& allocs, std::string& err, T** p, size_t bytes) {
    void* q = nullptr;
    const cudaError_t e = device_malloc(&q, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        err = "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e);
        return -1;
    }
    allocs.push_back(q);
    *p = static_cast<T*>(q);
    // Zeroed once so rows a step does not write (rows >= T of the activation
    // fragments, cache pages past the written positions) hold finite values.
    const cudaError_t z = cudaMemset(q, 0, bytes ? bytes : 16);
    if (z != cudaSuccess) {
        err = std::string("cudaMemset: ") + cudaGetErrorString(z);
        return -1;
    }
    return 0;
}

int fail(std::string& err, const std::string& msg) {
    err = msg;
    return -1;
}

// Upload one q8_0 matrix (ne = [k, n]) through `staging` and repack it into
// tiles at destination row groups r * stride + offset.
int upload_q8(mtb_model* m, const GgufFile& f, const std::string& name, int64_t k, int64_t n, uint8_t* staging,
              uint8_t* dst, int stride, int offset, uint8_t* pf_dst = nullptr, int pf_half = -1) {
    const GgufTensor* t = f.tensor(name);
    if (!t) return fail(m->error, "missing tensor " + name);
    if (t->type != GGML_Q8_0)
        return fail(m->error, name + ": only q8_0 decoder weights are supported (type " + std::to_string(t->type) + ")");
    if (t->ne.size() != 2 || t->ne[0] != k || t->ne[1] != n)
        return fail(m->error, name + ": unexpected shape");
    MTB_CK(m, cudaMemcpy(staging, t->data, t->nbytes, cudaMemcpyHostToDevice));
    launch_repack_q8(staging, int(n), int(k), dst, stride, offset, nullptr);
    if (pf_dst) pf_repack(staging, int(n), int(k), pf_half, pf_dst, nullptr);  // the prefill copy
    MTB_CK(m, cudaGetLastError());
    MTB_CK(m, cudaDeviceSynchronize());
    return 0;
}

// F16 rows [n][k] (ggml layout: k fastest) through `staging` into dst in the
// tiled layout of the F16 kernels (launch_repack_f16).
int upload_f16(mtb_model* m, const GgufFile& f, const std::string& name, int64_t k, int64_t n, uint16_t* staging,
               uint16_t* dst) {
    const GgufTensor* t = f.tensor(name);
    if (!t) return fail(m->error, "missing tensor " + name);
    if (t->type != GGML_F16) return fail(m->error, name + ": an F16 model needs F16 weights throughout");
    if (t->ne.size() != 2 || t->ne[0] != k || t->ne[1] != n) return fail(m->error, name + ": unexpected shape");
    if (n % 32 || k % 32) return fail(m->error, name + ": F16 matrices need multiples of 32 rows and columns");
    MTB_CK(m, cudaMemcpy(staging, t->data, size_t(k) * size_t(n) * 2, cudaMemcpyHostToDevice));
    launch_repack_f16(staging, int(n), int(k), dst, nullptr);
    MTB_CK(m, cudaGetLastError());
    MTB_CK(m, cudaDeviceSynchronize());
    return 0;
}

// ffn_gate and ffn_up [F][H] as one [2F][H] matrix, interleaved by 16 rows
// (gate rows 16 b .. 16 b + 15, then the same up rows), so each 32-row group
// of the F16 GEMV holds matching gate and up outputs (its SwiGLU epilogue).
int upload_f16_gate_up(mtb_model* m, const GgufFile& f, const std::string& gate, const std::string& up, int64_t k,
                       int64_t n, uint16_t* staging, uint16_t* dst) {
    const GgufTensor* tg = f.tensor(gate);
    const GgufTensor* tu = f.tensor(up);
    if (!tg || !tu) return fail(m->error, "missing tensor " + (tg ? up : gate));
    for (const GgufTensor* t : {tg, tu}) {
        if (t->type != GGML_F16) return fail(m->error, gate + ": an F16 model needs F16 weights throughout");
        if (t->ne.size() != 2 || t->ne[0] != k || t->ne[1] != n) return fail(m->error, gate + ": unexpected shape");
    }
    if (n % 16 || k % 32) return fail(m->error, gate + ": F16 matrices need multiples of 32 rows and columns");
    const size_t block = size_t(16) * size_t(k) * 2;  // 16 rows in bytes
    MTB_CK(m, cudaMemcpy2D(staging, 2 * block, tg->data, block, block, size_t(n / 16), cudaMemcpyHostToDevice));
    MTB_CK(m, cudaMemcpy2D(reinterpret_cast<char*>(staging) + block, 2 * block, tu->data, block, block, size_t(n / 16),
                           cudaMemcpyHostToDevice));
    launch_repack_f16(staging, int(2 * n), int(k), dst, nullptr);
    MTB_CK(m, cudaGetLastError());
    MTB_CK(m, cudaDeviceSynchronize());
    return 0;
}

int upload_f32(mtb_model* m, const GgufFile& f, const std::string& name, int64_t n, const float** out) {
    const GgufTensor* t = f.tensor(name);
    if (!t) return fail(m->error, "missing tensor " + name);
    if (t->type != GGML_F32 || t->ne.size() != 1 || t->ne[0] != n) return fail(m->error, name + ": expected F32 [" + std::to_string(n) + "]");
    float* p = nullptr;
    if (dalloc(m->allocs, m->error, &p, size_t(n) * 4)) return -1;
    MTB_CK(m, cudaMemcpy(p, t->data, size_t(n) * 4, cudaMemcpyHostToDevice));
    *out = p;
    return 0;
}

size_t tiles_bytes(int64_t n_rows, int64_t k) { return size_t(n_rows / kTileRows) * size_t(k / kTileK) * kTileBytes; }

int load_model(mtb_model* m, const char* path) {
    GgufFile f;
    if (!f.open(path)) return fail(m->error, f.error());
    ModelDims& d = m->dm.dims;
    d.hidden = int(f.get_u32("mtd.text.hidden", 1024));
    d.n_layers = int(f.get_u32("mtd.text.n_layers", 28));
    d.n_heads = int(f.get_u32("mtd.text.n_heads", 16));
    d.n_kv = int(f.get_u32("mtd.text.n_kv_heads", 8));
    d.ffn = int(f.get_u32("mtd.text.ffn", 3072));
    d.vocab = int(f.get_u32("mtd.text.vocab_size", 151936));
    d.eps = f.get_f32("mtd.text.rms_eps", 1e-6f);
    d.theta = f.get_f32("mtd.text.rope_theta", 1e6f);
    m->eos = int(f.get_u32("mtd.eos_token_id", 151645));
    const int head_dim = int(f.get_u32("mtd.text.head_dim", 128));
    if (head_dim != kHeadDim) return fail(m->error, "head_dim must be 128");
    // Every K of a projection is a whole number of 256-element slices.
    if (d.hidden <= 0 || d.hidden % 256 || d.hidden > 8192) return fail(m->error, "hidden must be a multiple of 256 (<= 8192)");
    if (d.ffn <= 0 || d.ffn % 256 || d.ffn > 16384) return fail(m->error, "ffn must be a multiple of 256 (<= 16384)");
    if ((d.n_heads * kHeadDim) % 256) return fail(m->error, "n_heads * 128 must be a multiple of 256");
    if (d.n_heads <= 0 || d.n_kv <= 0 || d.n_heads % d.n_kv || d.n_heads / d.n_kv > 4)
        return fail(m->error, "n_heads must be 1..4 times n_kv_heads");
    if (d.vocab <= 0 || d.vocab % kTileRows) return fail(m->error, "vocab must be a multiple of 8");
    if (d.n_layers <= 0) return fail(m->error, "n_layers must be positive");
    const int64_t H = d.hidden, F = d.ffn, qd = int64_t(d.n_heads) * kHeadDim, kd = int64_t(d.n_kv) * kHeadDim;
    const GgufTensor* te = f.tensor("token_embd.weight");
    if (!te) return fail(m->error, "missing token_embd.weight");
    if (te->type == GGML_F16) {
        // F16 weights: fp16 on the device in the F16 kernels'
        // tiled layout, the multi-kernel path with the F16 GEMV kernels; no
        // persistent kernel and no tcgen05 prefill (both are q8_0 designs).
        if (std::max(std::max(H, qd), F) > kF16MaxK) return fail(m->error, "F16 model: projection K too large");
        m->dm.f16 = true;
        const size_t staging_halves = std::max(size_t(d.vocab) * size_t(H), size_t(std::max(qd, 2 * F)) * size_t(H));
        uint16_t* stg = nullptr;
        std::vector<void*> tmp;
        if (dalloc(tmp, m->error, &stg, std::max(staging_halves, size_t(H) * size_t(F)) * 2)) return -1;
        struct Guard { std::vector<void*>& v; ~Guard() { for (void* p : v) cudaFree(p); } } guard{tmp};
        uint16_t* embd16 = nullptr;
        if (dalloc(m->allocs, m->error, &embd16, size_t(d.vocab) * size_t(H) * 2)) return -1;
        if (upload_f16(m, f, "token_embd.weight", H, d.vocab, stg, embd16)) return -1;
        m->dm.h_embd = embd16;
        if (upload_f32(m, f, "qwen3.output_norm.weight", H, &m->dm.output_norm)) return -1;
        m->layers.assign(size_t(d.n_layers), LayerWeights{});
        for (int l = 0; l < d.n_layers; ++l) {
            const std::string p = "qwen3.blk." + std::to_string(l) + ".";
            LayerWeights& w = m->layers[size_t(l)];
            uint16_t *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
            if (dalloc(m->allocs, m->error, &qkv, size_t(qd + 2 * kd) * size_t(H) * 2) ||
                dalloc(m->allocs, m->error, &o, size_t(H) * size_t(qd) * 2) ||
                dalloc(m->allocs, m->error, &gu, size_t(2 * F) * size_t(H) * 2) ||
                dalloc(m->allocs, m->error, &down, size_t(H) * size_t(F) * 2))
                return -1;
            if (upload_f16(m, f, p + "attn_q.weight", H, qd, stg, qkv) ||
                upload_f16(m, f, p + "attn_k.weight", H, kd, stg, qkv + size_t(qd) * size_t(H)) ||
                upload_f16(m, f, p + "attn_v.weight", H, kd, stg, qkv + size_t(qd + kd) * size_t(H)) ||
                upload_f16(m, f, p + "attn_o.weight", qd, H, stg, o) ||
                upload_f16_gate_up(m, f, p + "ffn_gate.weight", p + "ffn_up.weight", H, F, stg, gu) ||
                upload_f16(m, f, p + "ffn_down.weight", F, H, stg, down))
                return -1;
            w.h_qkv = qkv;
            w.h_o = o;
            w.h_gu = gu;
            w.h_down = down;
            if (upload_f32(m, f, p + "attn_norm.weight", H, &w.attn_norm) ||
                upload_f32(m, f, p + "attn_q_norm.weight", kHeadDim, &w.q_norm) ||
                upload_f32(m, f, p + "attn_k_norm.weight", kHeadDim, &w.k_norm) ||
                upload_f32(m, f, p + "ffn_norm.weight", H, &w.ffn_norm))
                return -1;
        }
        m->dm.layers = m->layers.data();
        m->dm.theta_scale = std::pow(d.theta, -2.0f / float(kHeadDim));
        MTB_CK(m, configure_kernels());
        m->mega_grid = 0;
        MTB_CK(m, cudaDeviceSynchronize());
        return 0;
    }
    size_t staging_bytes = te->nbytes;
    for (int l = 0; l < d.n_layers; ++l) {
        for (const char* nm : {"attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down"}) {
            const GgufTensor* t = f.tensor("qwen3.blk." + std::to_string(l) + "." + nm + ".weight");
            if (!t) return fail(m->error, "missing qwen3.blk." + std::to_string(l) + "." + nm + ".weight");
            staging_bytes = std::max<size_t>(staging_bytes, t->nbytes);
        }
    }
    uint8_t* staging = nullptr;
    std::vector<void*> tmp;
    if (dalloc(tmp, m->error, &staging, staging_bytes)) return -1;
    struct Guard { std::vector<void*>& v; ~Guard() { for (void* p : v) cudaFree(p); } } guard{tmp};

    uint8_t* embd = nullptr;
    if (dalloc(m->allocs, m->error, &embd, tiles_bytes(d.vocab, H))) return -1;
    // MTB_LM_TCGEN05=1: the persistent step's LM head on tcgen05 (128-row tiles
    // streamed through the ring).  Off by default: on B200 it measured slower
    // than the mma.sync LM phase (80 vs 62 us at T = 8), the 16-slot ring holding
    // one tile at a time.
    uint8_t* pf_embd = nullptr;
    if (std::getenv("MTB_LM_TCGEN05") && d.vocab % 128 == 0 &&
        dalloc(m->allocs, m->error, &pf_embd, pf_weight_bytes(d.vocab, int(H))))
        return -1;
    if (upload_q8(m, f, "token_embd.weight", H, d.vocab, staging, embd, 1, 0, pf_embd)) return -1;
    m->dm.embd = embd;
    m->dm.pf_embd = pf_embd;
    if (upload_f32(m, f, "qwen3.output_norm.weight", H, &m->dm.output_norm)) return -1;
    m->layers.resize(size_t(d.n_layers));
    for (int l = 0; l < d.n_layers; ++l) {
        const std::string p = "qwen3.blk." + std::to_string(l) + ".";
        LayerWeights& w = m->layers[size_t(l)];
        uint8_t *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
        uint8_t *pqkv = nullptr, *po = nullptr, *pgu = nullptr, *pdown = nullptr;
        if (dalloc(m->allocs, m->error, &qkv, tiles_bytes(qd + 2 * kd, H)) ||
            dalloc(m->allocs, m->error, &o, tiles_bytes(H, qd)) ||
            dalloc(m->allocs, m->error, &gu, tiles_bytes(2 * F, H)) ||
            dalloc(m->allocs, m->error, &down, tiles_bytes(H, F)) ||
            dalloc(m->allocs, m->error, &pqkv, pf_weight_bytes(int(qd + 2 * kd), int(H))) ||
            dalloc(m->allocs, m->error, &po, pf_weight_bytes(int(H), int(qd))) ||
            dalloc(m->allocs, m->error, &pgu, pf_weight_bytes(int(2 * F), int(H))) ||
            dalloc(m->allocs, m->error, &pdown, pf_weight_bytes(int(H), int(F))))
            return -1;
        // Prefill steps of q, k, v: whole 128-row tiles in that order.
        const size_t pf_rows_bytes = pf_weight_bytes(128, int(H));
        if (upload_q8(m, f, p + "attn_q.weight", H, qd, staging, qkv, 1, 0, pqkv) ||
            upload_q8(m, f, p + "attn_k.weight", H, kd, staging, qkv, 1, int(qd / kTileRows),
                      pqkv + size_t(qd / 128) * pf_rows_bytes) ||
            upload_q8(m, f, p + "attn_v.weight", H, kd, staging, qkv, 1, int((qd + kd) / kTileRows),
                      pqkv + size_t((qd + kd) / 128) * pf_rows_bytes) ||
            upload_q8(m, f, p + "attn_o.weight", qd, H, staging, o, 1, 0, po) ||
            upload_q8(m, f, p + "ffn_gate.weight", H, F, staging, gu, 2, 0, pgu, 0) ||
            upload_q8(m, f, p + "ffn_up.weight", H, F, staging, gu, 2, 1, pgu, 1) ||
            upload_q8(m, f, p + "ffn_down.weight", F, H, staging, down, 1, 0, pdown))
            return -1;
        w.qkv = qkv;
        w.o = o;
        w.gu = gu;
        w.down = down;
        w.pf_qkv = pqkv;
        w.pf_o = po;
        w.pf_gu = pgu;
        w.pf_down = pdown;
        if (upload_f32(m, f, p + "attn_norm.weight", H, &w.attn_norm) ||
            upload_f32(m, f, p + "attn_q_norm.weight", kHeadDim, &w.q_norm) ||
            upload_f32(m, f, p + "attn_k_norm.weight", kHeadDim, &w.k_norm) ||
            upload_f32(m, f, p + "ffn_norm.weight", H, &w.ffn_norm))
            return -1;
    }
    m->dm.layers = m->layers.data();
    if (dalloc(m->allocs, m->error, &m->layers_dev, sizeof(LayerWeights) * m->layers.size())) return -1;
    MTB_CK(m, cudaMemcpy(m->layers_dev, m->layers.data(), sizeof(LayerWeights) * m->layers.size(),
                         cudaMemcpyHostToDevice));
    // Same powf as the CPU path so the RoPE angles advance identically.
    m->dm.theta_scale = std::pow(d.theta, -2.0f / float(kHeadDim));
    MTB_CK(m, configure_kernels());
    if (!std::getenv("MTB_NO_PERSISTENT")) {
        int grid = 0;
        MTB_CK(m, configure_megakernel(m->device, d.hidden, &grid));
        m->mega_grid = megakernel_supports(d, grid) ? grid : 0;
    }
    MTB_CK(m, cudaDeviceSynchronize());
    return 0;
}

int refresh(mtb_decoder* d) {
    if (d->fresh && d->h_state->error == 0) return 0;
    d->d2h_bytes += sizeof(StepState);
    MTB_CK(d, cudaMemcpyAsync(d->h_state, d->b.state, sizeof(StepState), cudaMemcpyDeviceToHost, d->stream));
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    if (d->pf_status_pending) {
        d->pf_status_pending = false;
        if (*d->h_pf_status) return fail(d->error, "prefill projection gave up waiting (tcgen05 pipeline timeout)");
    }
    if (d->h_state->error) {
        d->error = d->h_state->error == 2   ? "verify step gave up waiting (persistent kernel timeout)"
                   : d->h_state->error == 3 ? "persistent kernel: shared-memory ring not 1024-byte aligned"
                                            : "device reported an out-of-range token id";
        return -1;
    }
    d->fresh = true;
    return 0;
}

int push_state(mtb_decoder* d) {
    d->h2d_bytes += sizeof(StepState);
    MTB_CK(d, cudaMemcpyAsync(d->b.state, d->h_state, sizeof(StepState), cudaMemcpyHostToDevice, d->stream));
    return 0;
}

cudaGraphExec_t step_graph(mtb_decoder* d, int mode, bool penalty) {
    cudaGraphExec_t& g = d->graphs[mode][penalty ? 1 : 0];
    if (g) return g;
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return nullptr;
    if (d->model->mega_grid > 0 && !penalty) {
        // Draft, then the whole verify step as one persistent kernel.
        launch_draft(d->b, mode, d->stream);
        launch_step_persistent(d->model->dm, d->model->layers_dev, d->kv, d->kv_map, d->b, d->mb, d->model->mega_grid,
                               d->stream);
    } else {
        launch_step(d->model->dm, d->kv, d->b, mode, penalty, d->stream);
    }
    if (cudaStreamEndCapture(d->stream, &graph) != cudaSuccess || !graph) return nullptr;
    // Kernel launches per step: the graph's kernel nodes (memset nodes excluded).
    size_t n = 0;
    cudaGraphGetNodes(graph, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    if (n) cudaGraphGetNodes(graph, nodes.data(), &n);
    int kernels = 0;
    for (size_t i = 0; i < n; ++i) {
        cudaGraphNodeType type;
        if (cudaGraphNodeGetType(nodes[i], &type) == cudaSuccess && type == cudaGraphNodeTypeKernel) ++kernels;
    }
    d->launches = kernels;
    if (cudaGraphInstantiate(&g, graph, 0) != cudaSuccess) g = nullptr;
    cudaGraphDestroy(graph);
    return g;
}

int run_step(mtb_decoder* d, int mode) {
    d->fresh = false;  // device work below changes the step state
    cudaGraphExec_t g = step_graph(d, mode, d->h_state->penalty > 1.f);
    if (!g) return fail(d->error, "could not build the verify-step graph: " + std::string(cudaGetErrorString(cudaGetLastError())));
    MTB_CK(d, cudaGraphLaunch(g, d->stream));
    return 0;
}

constexpr int kPrefillRows = 512;                  // rows per prefill pass at most
constexpr size_t kPrefillPartRows = size_t(1) << 19;  // attention partial entries (512 B each) per pass at most

// Rows of the next prefill pass: at most `remaining` and kPrefillRows, a
// multiple of 16, and few enough that the pass's attention partials fit.
int prefill_pass_rows(const mtb_decoder* d, int remaining, int before) {
    const ModelDims& dm = d->model->dm.dims;
    const int G = dm.n_heads / dm.n_kv;
    int P = std::min(remaining, d->pf.max_rows);
    if (P < remaining) P -= P % kTMax;  // a pass that leaves rows over ends on a row block
    while (P > kTMax) {
        const size_t need = size_t((P + kTMax - 1) / kTMax) * dm.n_kv * size_t((before + P + kPage - 1) / kPage) * (kTMax * G);
        if (need <= d->pf.part_rows) break;
        P -= kTMax;
    }
    return P;
}

// Rows [T][hidden] from the host at past..past+T-1.  More than kTMax rows: all
// in prefill passes (every layer over up to 512 rows at once, tcgen05
// projections), the LM head of the last row (when asked) from the last pass's
// final-normed rows.  At most kTMax rows: one step of the verify kernels.  The
// host's past (h_state) is current on entry.
int forward_host_rows(mtb_decoder* d, const float* rows, int T, float* hidden_out, bool lm_on_last,
                      bool rows_on_device = false, bool defer_status = false) {
    d->fresh = false;  // device work below changes the step state
    const int H = d->model->dm.dims.hidden;
    const cudaMemcpyKind in_kind = rows_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    int done = 0;
    if (d->pf.max_rows >= kTMax && T > kTMax) {
        const int past = d->h_state->past;
        while (done < T) {
            const int P = prefill_pass_rows(d, T - done, past + done);
            if (P < 1 || (P < kTMax && done + P < T)) return fail(d->error, "prefill pass does not fit its buffers");
            const bool last = done + P >= T;
            if (!rows_on_device) d->h2d_bytes += (long long)P * H * 4;
            MTB_CK(d, cudaMemcpyAsync(d->pf.x, rows + size_t(done) * H, size_t(P) * H * sizeof(float), in_kind,
                                      d->stream));
            launch_prefill_pass(d->model->dm, d->kv, d->pf, P, past + done,
                                hidden_out != nullptr || (lm_on_last && last), d->stream);
            launch_rows_begin(d->b, P, d->stream);
            launch_rows_end(d->b, d->stream);
            MTB_CK(d, cudaGetLastError());
            if (hidden_out) {
                d->d2h_bytes += (long long)P * H * 4;
                MTB_CK(d, cudaMemcpyAsync(hidden_out + size_t(done) * H, d->pf.hid, size_t(P) * H * sizeof(float),
                                          cudaMemcpyDeviceToHost, d->stream));
            }
            if (lm_on_last && last) launch_lm_row(d->model->dm, d->b, d->pf.hid + size_t(P - 1) * H, d->stream);
            done += P;
        }
        if (defer_status) {
            // Checked by the next refresh(): the caller does not wait here, so
            // several decoders' prefills can run side by side on their streams.
            MTB_CK(d, cudaMemcpyAsync(d->h_pf_status, d->pf.status, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
            d->pf_status_pending = true;
        } else {
            int status = 0;
            MTB_CK(d, cudaMemcpyAsync(&status, d->pf.status, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
            MTB_CK(d, cudaStreamSynchronize(d->stream));
            if (status) return fail(d->error, "prefill projection gave up waiting (tcgen05 pipeline timeout)");
            d->h_state->past = past + done;
        }
        // Deferred: the pinned state mirror is not written while its push may
        // still be pending; the device holds the new past (k_rows_end) and the
        // mirror is refreshed before any host use (fresh is false).
    }
    for (int r0 = done; r0 < T; r0 += kTMax) {
        const int n = std::min(kTMax, T - r0);
        if (rows_on_device) {
            MTB_CK(d, cudaMemcpyAsync(d->b.x, rows + size_t(r0) * H, size_t(n) * H * sizeof(float),
                                      cudaMemcpyDeviceToDevice, d->stream));
        } else {
            std::memcpy(d->h_rows, rows + size_t(r0) * H, size_t(n) * H * sizeof(float));
            MTB_CK(d, cudaMemcpyAsync(d->b.x, d->h_rows, size_t(n) * H * sizeof(float), cudaMemcpyHostToDevice, d->stream));
        }
        launch_rows_begin(d->b, n, d->stream);
        const bool last = r0 + n >= T;
        launch_forward_rows(d->model->dm, d->kv, d->b, lm_on_last && last, false, d->stream);
        launch_rows_end(d->b, d->stream);
        MTB_CK(d, cudaGetLastError());
        if (hidden_out) {
            MTB_CK(d, cudaMemcpyAsync(hidden_out + size_t(r0) * H, d->b.hid, size_t(n) * H * sizeof(float),
                                      cudaMemcpyDeviceToHost, d->stream));
        }
        MTB_CK(d, cudaStreamSynchronize(d->stream));  // h_rows is reused by the next chunk
    }
    return 0;
}

int g_log_level = 1;  // 0: silent, 1: the reference's INFO lines (the default)

// The reference's end-of-generation lines (src/cpu_speculative.cpp:138-145),
// without the "[mt I] " prefix its logger adds.  Embedding, logits, draft and
// rewind run inside the device step here, so their own times read 0; the
// decoder time is the whole step loop.
std::string generation_log(const int32_t* ids, int n, int eos, const mtb_counters& c, int k_max, double prefill_s,
                           double decoder_s, bool trace) {
    const char* stop = c.stop_reason == STOP_EOS ? "eos" : c.stop_reason == STOP_LIMIT ? "token_limit" : "error";
    char buf[512];
    std::string out;
    std::snprintf(buf, sizeof(buf), "BENCH_GENERATION tokens=%d stop=%s\n", n, stop);
    out += buf;
    std::snprintf(buf, sizeof(buf), "CPU_PROFILE prefill=%.6f embedding=%.6f decoder=%.6f logits=%.6f\n", prefill_s, 0.0,
                  decoder_s, 0.0);
    out += buf;
    std::snprintf(buf, sizeof(buf),
                  "CPU_SPECULATIVE targetCalls=%lld draftedCalls=%lld proposed=%lld accepted=%lld targetInputTokens=%lld "
                  "rewinds=%lld draftSeconds=%.9f rewindSeconds=%.9f maximumDraft=%d\n",
                  (long long)c.target_calls, (long long)c.drafted_calls, (long long)c.proposed, (long long)c.accepted,
                  (long long)c.target_input_tokens, (long long)c.rewinds, 0.0, 0.0, k_max);
    out += buf;
    if (trace) {
        for (int off = 0; off < n; off += 128) {
            std::snprintf(buf, sizeof(buf), "BENCH_TOKEN_TRACE eos=%d total=%d offset=%d ids=[", eos, n, off);
            out += buf;
            for (int i = off; i < std::min(n, off + 128); ++i) {
                if (i != off) out += ',';
                out += std::to_string(ids[i]);
            }
            out += "]\n";
        }
    }
    return out;
}

bool trace_tokens() {
    const char* t = std::getenv("MTD_TRACE_TOKENS");
    return t && !std::strcmp(t, "1");
}

void emit_generation_log(const int32_t* ids, int n, int eos, const mtb_counters& c, int k_max, double prefill_s,
                         double decoder_s) {
    if (g_log_level <= 0) return;
    const std::string lines = generation_log(ids, n, eos, c, k_max, prefill_s, decoder_s, trace_tokens());
    size_t a = 0;
    while (a < lines.size()) {
        const size_t b = lines.find('\n', a);
        std::fprintf(stderr, "[mt I] %s\n", lines.substr(a, b - a).c_str());
        a = b + 1;
    }
    std::fflush(stderr);
}

double wall_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

void fill_counters(const StepState& s, mtb_counters* c) {
    if (!c) return;
    c->target_calls = s.target_calls;
    c->drafted_calls = s.drafted_calls;
    c->proposed = s.proposed;
    c->accepted = s.accepted;
    c->target_input_tokens = s.target_input_tokens;
    c->rewinds = s.rewinds;
    c->stop_reason = s.stop;
    c->past_len = s.past;
}

// Without explicit parameters the reference policy applies: k 4, n-grams
// 16..2, and the repetition penalty from MTD_REPETITION_PENALTY (unset: 1),
// as src/cpu_speculative.cpp:85-86 and :104 read them.
float env_penalty() {
    const char* e = std::getenv("MTD_REPETITION_PENALTY");
    return e ? float(std::atof(e)) : 1.f;
}

// An integer environment variable: `dflt` when unset; false when it does not
// parse as a whole decimal integer.
bool env_int(const char* name, int dflt, int* out) {
    const char* e = std::getenv(name);
    if (!e || !*e) {
        *out = dflt;
        return true;
    }
    char* end = nullptr;
    const long v = std::strtol(e, &end, 10);
    if (*end != 0 || v < INT32_MIN || v > INT32_MAX) return false;
    *out = int(v);
    return true;
}

int params_from_env(mtb_spec_params* out, std::string& err) {
    int k, nmin, nmax;
    if (!env_int("MTB_SPEC_K", 4, &k) || !env_int("MTB_NGRAM_MIN", 2, &nmin) || !env_int("MTB_NGRAM_MAX", 16, &nmax))
        return fail(err, "MTB_SPEC_K / MTB_NGRAM_MIN / MTB_NGRAM_MAX must be integers");
    if (k < 0 || k > kTMax - 1) return fail(err, "MTB_SPEC_K must be in [0, 15]");
    if (nmin < 1 || nmax < nmin) return fail(err, "need 1 <= MTB_NGRAM_MIN <= MTB_NGRAM_MAX");
    out->k_max = k;
    out->n_min = nmin;
    out->n_max = nmax;
    out->penalty = env_penalty();
    return 0;
}

int kv_type_from_env() {
    const char* e = std::getenv("MTB_KV_DTYPE");
    if (!e || !*e || !std::strcmp(e, "f32")) return KV_F32;
    if (!std::strcmp(e, "f16")) return KV_F16;
    return -1;
}

int set_params(mtb_decoder* d, int max_new, int eos, const mtb_spec_params* p) {
    StepState& s = *d->h_state;
    if (max_new <= 0 || max_new > d->max_new) return fail(d->error, "max_new must be in [1, " + std::to_string(d->max_new) + "]");
    mtb_spec_params envp;
    if (!p) {
        if (params_from_env(&envp, d->error)) return -1;
        p = &envp;
    }
    const int k = p->k_max;
    if (k < 0 || k > kTMax - 1) return fail(d->error, "k_max must be in [0, 15]");
    const int nmin = p->n_min, nmax = p->n_max;
    if (nmin < 1 || nmax < nmin) return fail(d->error, "need 1 <= n_min <= n_max");
    float pen = p->penalty;
    if (!(pen == pen)) pen = 1.f;              // NaN (an unparsable variable reads as 0, clamped below)
    pen = std::max(1.f, std::min(1.5f, pen));  // src/cpu_speculative.cpp:86
    s.max_new = max_new;
    s.eos = eos;
    s.k_max = k;
    s.n_min = nmin;
    s.n_max = nmax;
    s.penalty = pen;
    s.max_seq = d->max_seq;
    return 0;
}

void clear_progress(StepState& s) {
    s.stop = STOP_NONE;
    s.error = 0;
    s.n_ids = 0;
    s.T = 0;
    s.n_prop = 0;
    s.forced = 0;
    s.target_calls = s.drafted_calls = s.proposed = s.accepted = s.target_input_tokens = s.rewinds = 0;
}

int prefill(mtb_decoder* d, const float* fused, int seq, bool on_device = false, bool defer_status = false) {
    d->fresh = false;  // device work below changes the step state
    if (!fused || seq <= 0) return fail(d->error, "empty prompt");
    if (seq + 1 > d->max_seq) return fail(d->error, "prompt exceeds max_seq");
    d->h_state->past = 0;
    clear_progress(*d->h_state);
    if (push_state(d)) return -1;
    if (forward_host_rows(d, fused, seq, nullptr, true, on_device, defer_status)) return -1;
    launch_prefill_seed(d->b, d->stream);
    MTB_CK(d, cudaGetLastError());
    return 0;
}

// fuse_embeds (src/generate.cpp:113-177) with the rows built on the device:
// ids are validated and the audio slots counted on the host (the k-th
// position holding audio_token_id takes audio row k), ids, slots and audio rows
// are uploaded, and k_fuse_embeds writes the fused rows into fused_dev.
int fuse_on_device(mtb_decoder* d, const int32_t* ids, int seq, const float* audio, int n_audio, int audio_token_id) {
    d->fresh = false;  // device work below changes the step state
    const ModelDims& dm = d->model->dm.dims;
    const int H = dm.hidden;
    if (!ids || seq <= 0) return fail(d->error, "fuse_embeds: empty input_ids");
    if (seq > d->max_seq) return fail(d->error, "fuse_embeds: input longer than max_seq");
    if (n_audio < 0 || n_audio > d->max_seq || (n_audio > 0 && !audio)) return fail(d->error, "fuse_embeds: invalid audio rows");
    std::vector<int32_t> slot(static_cast<size_t>(seq), -1);
    int k = 0;
    for (int p = 0; p < seq; ++p) {
        if (ids[p] < 0 || ids[p] >= dm.vocab)  // generate.cpp:140-146
            return fail(d->error, "fuse_embeds: input_ids[" + std::to_string(p) + "]=" + std::to_string(ids[p]) +
                                      " out of range [0," + std::to_string(dm.vocab) + ")");
        if (ids[p] != audio_token_id) continue;
        if (k >= n_audio)  // generate.cpp:163-167
            return fail(d->error, "fuse_embeds: more audio positions than audio rows (n_audio=" + std::to_string(n_audio) + ")");
        slot[size_t(p)] = k++;
    }
    // k < n_audio is allowed (the reference logs a warning and continues).
    auto& A = d->allocs;
    if (!d->fused_dev && (dalloc(A, d->error, &d->fused_dev, size_t(d->max_seq) * H * 4) ||
                          dalloc(A, d->error, &d->fuse_ids, size_t(d->max_seq) * 2 * 4) ||
                          dalloc(A, d->error, &d->fuse_audio, size_t(d->max_seq) * H * 4)))
        return -1;
    d->h2d_bytes += (long long)seq * 8 + (long long)n_audio * H * 4;
    MTB_CK(d, cudaMemcpyAsync(d->fuse_ids, ids, size_t(seq) * 4, cudaMemcpyHostToDevice, d->stream));
    MTB_CK(d, cudaMemcpyAsync(d->fuse_ids + d->max_seq, slot.data(), size_t(seq) * 4, cudaMemcpyHostToDevice, d->stream));
    if (n_audio > 0)
        MTB_CK(d, cudaMemcpyAsync(d->fuse_audio, audio, size_t(n_audio) * H * 4, cudaMemcpyHostToDevice, d->stream));
    launch_fuse_embeds(d->model->dm, d->fuse_ids, d->fuse_ids + d->max_seq, seq, d->fuse_audio, d->fused_dev, d->stream);
    MTB_CK(d, cudaGetLastError());
    MTB_CK(d, cudaStreamSynchronize(d->stream));  // `slot` is a host temporary
    return 0;
}

}  // namespace

// ================================================================= C ABI

extern "C" {

int mtb_abi_version(void) { return kAbiVersion; }

void mtb_set_log_level(int level) { g_log_level = level; }

int mtb_format_generation_log(const int32_t* ids, int n_ids, int eos, const mtb_counters* counters, int k_max,
                              double prefill_seconds, double decoder_seconds, int trace, char* out, int out_size) {
    if (!counters || n_ids < 0 || (n_ids > 0 && !ids)) return -1;
    const std::string s = generation_log(ids, n_ids, eos, *counters, k_max, prefill_seconds, decoder_seconds, trace != 0);
    if (out && out_size > 0) {
        const size_t m = std::min(s.size(), size_t(out_size - 1));
        std::memcpy(out, s.data(), m);
        out[m] = 0;
    }
    return int(s.size());
}

int mtb_capi_can_transcribe(void) { return 0; }

int mtb_spec_params_from_env(mtb_spec_params* out) {
    if (!out) { g_error = "null argument"; return -1; }
    return params_from_env(out, g_error);
}

int mtb_kv_type_from_env(void) { return kv_type_from_env(); }

int mtb_f16_slices_per_block(int n, int k) { return n > 0 && k > 0 && k % 256 == 0 ? f16_spb(n, k) : -1; }

int mtb_bounds_check_enabled(void) {
#ifdef MTB_BOUNDS_CHECK
    return 1;
#else
    return 0;
#endif
}

int mtb_bounds_check_status(int device) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess) return -1;
    unsigned site = bc_take_kernels();
    const unsigned m = bc_take_megakernel(), p = bc_take_prefill();
    if (!site) site = m;
    if (!site) site = p;
    cudaSetDevice(prev);
    return int(site);
}

void mtb_debug_fail_alloc(int n) { g_fail_alloc.store(n > 0 ? n : 0); }
const char* mtb_global_error(void) { return g_error.c_str(); }

int mtb_model_load(const char* path, int device, mtb_model** out) {
    if (!out || !path) { g_error = "null argument"; return -1; }
    *out = nullptr;
    try {
        int n_dev = 0;
        if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev <= 0) {
            g_error = "no CUDA device: this library has no CPU path";
            cudaGetLastError();
            return -2;
        }
        if (device < 0 || device >= n_dev) { g_error = "device index out of range"; return -2; }
        if (cudaSetDevice(device) != cudaSuccess) { g_error = "cudaSetDevice failed"; return -2; }
        cudaDeviceProp prop{};
        cudaGetDeviceProperties(&prop, device);
        if (prop.major != 10) {
            g_error = "this library is built for sm_100a (B200); device is sm_" + std::to_string(prop.major * 10 + prop.minor);
            return -2;
        }
        auto* m = new mtb_model();
        m->device = device;
        if (load_model(m, path)) {
            g_error = m->error;
            delete m;
            return -1;
        }
        *out = m;
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    } catch (...) {
        g_error = "unknown error";
        return -1;
    }
}

void mtb_model_free(mtb_model* m) { delete m; }
const char* mtb_model_error(const mtb_model* m) { return m ? m->error.c_str() : ""; }

// Device-side view of a loaded model for the other translation units (not
// part of the public ABI).
__attribute__((visibility("hidden"))) int mtb_model_device_view(const mtb_model* m, const void** view, int* device) {
    if (!m || !view || !device) return -1;
    *view = &m->dm;
    *device = m->device;
    return 0;
}

int mtb_model_persistent_grid(const mtb_model* m) { return m ? m->mega_grid : -1; }

int mtb_model_dims(const mtb_model* m, int32_t* o) {
    if (!m || !o) return -1;
    const ModelDims& d = m->dm.dims;
    o[0] = d.hidden; o[1] = d.n_layers; o[2] = d.n_heads; o[3] = d.n_kv; o[4] = kHeadDim; o[5] = d.ffn;
    o[6] = d.vocab; o[7] = m->eos;
    return 0;
}

int mtb_decoder_create(mtb_model* m, int max_seq, int kv_type, int max_new, mtb_decoder** out) {
    if (!m || !out) { g_error = "null argument"; return -1; }
    *out = nullptr;
    if (kv_type == MTB_KV_DEFAULT) {
        kv_type = kv_type_from_env();
        if (kv_type < 0) {
            g_error = "MTB_KV_DTYPE must be f16 or f32";
            return -1;
        }
    }
    if (max_seq <= 0 || max_new <= 0 || (kv_type != KV_F32 && kv_type != KV_F16)) {
        g_error = "invalid decoder arguments";
        return -1;
    }
    try {
        auto* d = new mtb_decoder();
        d->model = m;
        d->device = m->device;
        d->max_seq = max_seq;
        d->kv_type = kv_type;
        d->max_new = max_new;
        auto bail = [&](void) { g_error = d->error; delete d; return -1; };
        if (cudaSetDevice(d->device) != cudaSuccess) { d->error = "cudaSetDevice failed"; return bail(); }
        if (cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) != cudaSuccess) { d->error = "stream"; return bail(); }
        const ModelDims& dm = m->dm.dims;
        const int H = dm.hidden, F = dm.ffn, qd = dm.n_heads * kHeadDim, kd = dm.n_kv * kHeadDim;
        const int kmax = std::max(std::max(H, qd), F);
        const int n_pages = (max_seq + kPage - 1) / kPage;
        d->kv.type = kv_type;
        d->kv.page_elems = (long long)dm.n_layers * 2 * dm.n_kv * kPage * kHeadDim;
        const size_t esz = kv_type == KV_F16 ? 2 : 4;
        void* kvb = nullptr;
        int32_t* pages = nullptr;
        StepBuffers& b = d->b;
        b.max_chunks = n_pages;
        const bool f16 = m->dm.f16;
        b.lm_blocks = f16 ? (dm.vocab + kF16Outs - 1) / kF16Outs : lm_head_blocks(dm.vocab);
        auto& A = d->allocs;
        auto& E = d->error;
        uint8_t* zero_region = nullptr;
        const size_t head_bytes = size_t(dm.n_layers) * kMaxStreams * dm.n_kv * 4;
        const size_t pair_bytes = size_t(dm.n_layers) * (dm.n_heads / 2) * 4;
        const size_t slice_bytes = size_t(dm.n_layers) * (F / 256) * 4;
        const size_t mmax_bytes = size_t(dm.n_layers) * dm.n_kv * kTMax * 4 * 4;
        d->mb.zero_bytes = 16 + head_bytes + pair_bytes + slice_bytes + mmax_bytes;
        if (dalloc(A, E, &d->mb.act2_q, size_t(F / 32) * 512) || dalloc(A, E, &d->mb.act2_d, size_t(F / 32) * 16 * 4) ||
            dalloc(A, E, &d->mb.lm_val, size_t(std::max(m->mega_grid, 1)) * 16 * sizeof(float2)) ||
            dalloc(A, E, &zero_region, d->mb.zero_bytes))
            return bail();
        if (std::getenv("MTB_PROFILE") && dalloc(A, E, &d->mb.timeline, (6 * kMaxBarriers + 2 + 256 * kMaxBarriers * 17) * 8)) return bail();
        if (std::getenv("MTB_STEP_CAPTURE") && dalloc(A, E, &d->mb.capture, step_capture_floats(H) * 4)) return bail();
        d->mb.bar = reinterpret_cast<unsigned*>(zero_region);
        d->mb.abort_flag = reinterpret_cast<int*>(zero_region + 4);
        d->mb.head_done = reinterpret_cast<unsigned*>(zero_region + 16);
        d->mb.pair_done = reinterpret_cast<unsigned*>(zero_region + 16 + head_bytes);
        d->mb.slice_done = reinterpret_cast<unsigned*>(zero_region + 16 + head_bytes + pair_bytes);
        d->mb.m_max = reinterpret_cast<unsigned*>(zero_region + 16 + head_bytes + pair_bytes + slice_bytes);
        // Failure-path test hook (documented in tests/test_gpu_wait_timeout.py): a
        // barrier CTA 0 never arrives at, and a shorter wait bound.
        if (const char* sb = std::getenv("MTB_TEST_STALL_BARRIER")) d->mb.stall_barrier = std::atoi(sb);
        if (const char* wm = std::getenv("MTB_TEST_WAIT_MS")) d->mb.wait_ns = 1000000ull * std::max(1, std::atoi(wm));
        if (dalloc(A, E, &kvb, size_t(n_pages) * d->kv.page_elems * esz) || dalloc(A, E, &pages, size_t(n_pages) * 4) ||
            dalloc(A, E, &b.state, sizeof(StepState)) || dalloc(A, E, &b.ids, size_t(max_new) * 4) ||
            dalloc(A, E, &b.x, size_t(kTMax) * H * 4) || dalloc(A, E, &b.qkv, size_t(kTMax) * (qd + 2 * kd) * 4) ||
            dalloc(A, E, &b.attn_out, size_t(kTMax) * qd * 4) || dalloc(A, E, &b.gu, size_t(kTMax) * F * 4) ||
            dalloc(A, E, &b.hid, size_t(kTMax) * H * 4) || dalloc(A, E, &b.act_q, size_t(kmax / 32) * 512) ||
            dalloc(A, E, &b.act_d, size_t(kmax / 32) * 16 * 4) ||
            dalloc(A, E, &b.part_o, size_t(dm.n_kv) * n_pages * kTMax * 4 * kHeadDim * 4) ||
            dalloc(A, E, &b.part_ml, size_t(dm.n_kv) * n_pages * kTMax * 4 * sizeof(float2)) ||
            dalloc(A, E, &b.lm_val, size_t(b.lm_blocks) * 16 * sizeof(float2)) ||
            dalloc(A, E, &b.logits, size_t(kTMax) * dm.vocab * 4) || dalloc(A, E, &d->snap_state, sizeof(StepState)) ||
            dalloc(A, E, &d->snap_ids, size_t(max_new) * 4) || dalloc(A, E, &d->scratch_i, size_t(max_new + 16) * 4) ||
            dalloc(A, E, &d->group_flag, 2 * sizeof(int)) ||
            dalloc(A, E, &d->scratch_n, 64) || dalloc(A, E, &d->row_buf, size_t(H) * 4))
            return bail();
        if (f16 && (dalloc(A, E, &b.act_h, size_t(kTMax) * kmax * 2) || dalloc(A, E, &b.act_h2, size_t(kTMax) * F * 2) ||
                    dalloc(A, E, &b.f16_part, f16_part_floats(dm) * 4) ||
                    dalloc(A, E, &b.f16_cnt, size_t(f16_groups_max(dm)) * 4)))
            return bail();
        if (!f16) {
            // Prefill pass buffers: up to kPrefillRows rows per pass.
            PrefillBuffers& p = d->pf;
            const int G = dm.n_heads / dm.n_kv;
            p.max_rows = std::min(kPrefillRows, (max_seq + kTMax - 1) / kTMax * kTMax);
            const size_t P = size_t(p.max_rows);
            p.part_rows = std::min(kPrefillPartRows, size_t((P + kTMax - 1) / kTMax) * dm.n_kv * n_pages * kTMax * G);
            if (dalloc(A, E, &p.x, P * H * 4) || dalloc(A, E, &p.qkv, P * (qd + 2 * kd) * 4) ||
                dalloc(A, E, &p.attn, P * qd * 4) || dalloc(A, E, &p.gu, P * F * 4) || dalloc(A, E, &p.hid, P * H * 4) ||
                dalloc(A, E, &p.xq, pf_act_bytes(int(P), kmax)) || dalloc(A, E, &p.xd, P * (kmax / 32) * 4) ||
                dalloc(A, E, &p.part_o, p.part_rows * kHeadDim * 4) || dalloc(A, E, &p.part_ml, p.part_rows * sizeof(float2)) ||
                dalloc(A, E, &p.status, 16))
                return bail();
        }
        d->kv.base = kvb;
        d->kv.pages = pages;
        d->kv.n_pages = n_pages;
        std::vector<int32_t> ident(static_cast<size_t>(n_pages));
        for (int i = 0; i < n_pages; ++i) ident[size_t(i)] = i;
        if (cudaMemcpy(pages, ident.data(), ident.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemset(kvb, 0, size_t(n_pages) * d->kv.page_elems * esz) != cudaSuccess ||
            cudaMemset(b.state, 0, sizeof(StepState)) != cudaSuccess) {
            d->error = "device initialisation failed";
            return bail();
        }
        if (m->mega_grid > 0 && encode_kv_map(d->kv, (long long)n_pages * d->kv.page_elems, &d->kv_map) != cudaSuccess) {
            d->error = "could not encode the KV cache tensor map";
            return bail();
        }
        if (cudaMallocHost(&d->h_state, sizeof(StepState)) != cudaSuccess ||
            cudaMallocHost(&d->h_rows, size_t(kTMax) * H * 4) != cudaSuccess ||
            cudaMallocHost(&d->h_ids, size_t(max_new) * 4) != cudaSuccess ||
            cudaMallocHost(&d->h_flag, 2 * sizeof(int)) != cudaSuccess ||
            cudaMallocHost(&d->h_pf_status, sizeof(int)) != cudaSuccess) {
            d->error = "pinned host allocation failed";
            return bail();
        }
        std::memset(d->h_state, 0, sizeof(StepState));
        for (auto& e : d->ev)
            if (cudaEventCreate(&e) != cudaSuccess) { d->error = "event"; return bail(); }
        if (cudaEventCreateWithFlags(&d->group_ev, cudaEventDisableTiming) != cudaSuccess) {
            d->error = "event";
            return bail();
        }
        d->h_state->max_seq = max_seq;
        d->h_state->max_new = max_new;
        d->h_state->eos = m->eos;
        d->h_state->k_max = 4;
        d->h_state->n_min = 2;
        d->h_state->n_max = 16;
        d->h_state->penalty = 1.f;
        if (push_state(d) || cudaStreamSynchronize(d->stream) != cudaSuccess) return bail();
        *out = d;
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}

void mtb_decoder_free(mtb_decoder* d) { delete d; }
const char* mtb_decoder_error(const mtb_decoder* d) { return d ? d->error.c_str() : ""; }

int mtb_decoder_past_len(const mtb_decoder* dc) {
    auto* d = const_cast<mtb_decoder*>(dc);
    if (!d) return -1;
    cudaSetDevice(d->device);
    if (refresh(d)) return -1;
    return d->h_state->past;
}

int mtb_decoder_reset(mtb_decoder* d) {
    if (!d) return -1;
    d->fresh = false;
    cudaSetDevice(d->device);
    if (refresh(d)) return -1;
    d->h_state->past = 0;  // src/qwen3_decoder.cpp:87-89
    clear_progress(*d->h_state);
    if (push_state(d)) return -1;
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    return 0;
}

int mtb_decoder_rewind(mtb_decoder* d, int position) {
    if (!d) return -1;
    d->fresh = false;
    cudaSetDevice(d->device);
    if (refresh(d)) return -1;
    if (position < 0 || position > d->h_state->past) return fail(d->error, "invalid rewind");  // cpu_speculative.cpp:22-24
    d->h_state->past = position;
    if (push_state(d)) return -1;
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    return 0;
}

int mtb_decoder_run(mtb_decoder* d, const float* embeds, int T, float* hidden_out) {
    if (!d || !embeds || T <= 0) return -1;
    d->fresh = false;
    cudaSetDevice(d->device);
    if (refresh(d)) return -1;
    if (d->h_state->past + T > d->max_seq) return fail(d->error, "sequence exceeds max_seq");  // qwen3_decoder.cpp:102
    return forward_host_rows(d, embeds, T, hidden_out, false);
}

int mtb_decoder_logits(mtb_decoder* d, const float* hidden_row, float* logits) {
    if (!d || !hidden_row || !logits) return -1;
    d->fresh = false;
    cudaSetDevice(d->device);
    const ModelDims& dm = d->model->dm.dims;
    if (refresh(d)) return -1;
    d->fresh = false;
    const int saved_T = d->h_state->T;
    MTB_CK(d, cudaMemcpyAsync(d->row_buf, hidden_row, size_t(dm.hidden) * 4, cudaMemcpyHostToDevice, d->stream));
    const int one = 1;
    MTB_CK(d, cudaMemcpyAsync(&d->b.state->T, &one, sizeof(int), cudaMemcpyHostToDevice, d->stream));
    launch_logits_row(d->model->dm, d->b, d->row_buf, d->stream);
    MTB_CK(d, cudaGetLastError());
    MTB_CK(d, cudaMemcpyAsync(logits, d->b.logits, size_t(dm.vocab) * 4, cudaMemcpyDeviceToHost, d->stream));
    MTB_CK(d, cudaMemcpyAsync(&d->b.state->T, &saved_T, sizeof(int), cudaMemcpyHostToDevice, d->stream));
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    return 0;
}

int mtb_decoder_kv_read(mtb_decoder* d, int layer, int which, int pos0, int n_pos, float* out) {
    if (!d || !out) return -1;
    const ModelDims& dm = d->model->dm.dims;
    if (layer < 0 || layer >= dm.n_layers || which < 0 || which > 1 || pos0 < 0 || n_pos < 0 || pos0 + n_pos > d->max_seq)
        return fail(d->error, "kv range");
    cudaSetDevice(d->device);
    float* tmp = nullptr;
    const size_t bytes = size_t(n_pos) * dm.n_kv * kHeadDim * 4;
    MTB_CK(d, device_malloc(reinterpret_cast<void**>(&tmp), bytes ? bytes : 4));
    launch_kv_gather(d->model->dm, d->kv, layer, which, pos0, n_pos, tmp, d->stream);
    cudaError_t e = cudaMemcpyAsync(out, tmp, bytes, cudaMemcpyDeviceToHost, d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return fail(d->error, cudaGetErrorString(e));
    return 0;
}

int mtb_decoder_fill_synthetic_kv(mtb_decoder* d, int n_pos, uint32_t seed) {
    if (!d || n_pos < 0 || n_pos > d->max_seq) return -1;
    d->fresh = false;
    cudaSetDevice(d->device);
    launch_fill_synthetic_kv(d->model->dm, d->kv, n_pos, seed, d->stream);
    MTB_CK(d, cudaGetLastError());
    if (refresh(d)) return -1;
    d->h_state->past = n_pos;
    if (push_state(d)) return -1;
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    return 0;
}

int mtb_spec_generate(mtb_decoder* d, const float* fused, int seq, int max_new, int eos, const mtb_spec_params* params,
                      int32_t* out_ids, int* n_out, mtb_counters* counters, mtb_draft_fn draft, mtb_commit_fn commit,
                      void* user) {
    if (!d || !out_ids || !n_out) return -1;
    d->fresh = false;
    *n_out = 0;
    try {
        cudaSetDevice(d->device);
        if (refresh(d)) return -1;
        if (set_params(d, max_new, eos, params)) return -1;
        const double t0 = wall_s();
        if (prefill(d, fused, seq)) return -1;
        const double t1 = wall_s();
        StepState& s = *d->h_state;
        const int vocab = d->model->dm.dims.vocab;
        if (draft || commit) {
            // One step per host round trip: the hooks see every proposal and commit.
            std::vector<int32_t> prop(static_cast<size_t>(kTMax));
            for (;;) {
                if (refresh(d)) return -1;
                MTB_CK(d, cudaMemcpyAsync(d->h_ids, d->b.ids, size_t(s.n_ids) * 4, cudaMemcpyDeviceToHost, d->stream));
                MTB_CK(d, cudaStreamSynchronize(d->stream));
                if (s.stop != STOP_NONE) {
                    if (commit) commit(user, d->h_ids, s.n_ids, s.past, 1);
                    break;
                }
                int budget = std::min(s.k_max, s.max_new - s.n_ids);
                budget = std::max(0, std::min(budget, s.max_seq - s.past - 1));
                int mode = 0;
                if (draft) {
                    int np = draft(user, d->h_ids, s.n_ids, budget, prop.data());
                    np = std::max(0, std::min(np, budget));
                    for (int i = 0; i < np; ++i)
                        if (prop[size_t(i)] < 0 || prop[size_t(i)] >= vocab) return fail(d->error, "invalid draft token");
                    for (int i = 0; i < np; ++i) s.tokens[1 + i] = prop[size_t(i)];
                    s.n_prop = np;
                    if (push_state(d)) return -1;
                    mode = 1;
                }
                if (run_step(d, mode)) return -1;
                if (refresh(d)) return -1;
                // The commit point precedes the next seed (src/cpu_speculative.cpp:136 then :101).
                if (commit) {
                    MTB_CK(d, cudaMemcpyAsync(d->h_ids, d->b.ids, size_t(s.n_ids) * 4, cudaMemcpyDeviceToHost, d->stream));
                    MTB_CK(d, cudaStreamSynchronize(d->stream));
                    commit(user, d->h_ids, s.commit_n, s.past, s.commit_stop ? 1 : 0);
                }
                // Stopped on an accepted proposal: that commit was the last.  Stopped
                // on the seed emitted after the commit: the loop top commits once more.
                if (s.commit_stop) break;
            }
        } else {
            // Device-driven loop: the host only watches the stop flag, one step behind.
            int i = 0;
            for (;;) {
                if (run_step(d, 0)) return -1;
                MTB_CK(d, cudaMemcpyAsync(&d->h_flag[i & 1], &d->b.state->stop, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
                MTB_CK(d, cudaEventRecord(d->ev[i & 1], d->stream));
                if (i > 0) {
                    MTB_CK(d, cudaEventSynchronize(d->ev[(i - 1) & 1]));
                    if (d->h_flag[(i - 1) & 1] != STOP_NONE) break;
                }
                ++i;
            }
            if (refresh(d)) return -1;
        }
        MTB_CK(d, cudaMemcpyAsync(out_ids, d->b.ids, size_t(s.n_ids) * 4, cudaMemcpyDeviceToHost, d->stream));
        MTB_CK(d, cudaStreamSynchronize(d->stream));
        *n_out = s.n_ids;
        fill_counters(s, counters);
        mtb_counters c{};
        fill_counters(s, &c);
        emit_generation_log(out_ids, s.n_ids, s.eos, c, s.k_max, t1 - t0, wall_s() - t1);
        return 0;
    } catch (const std::exception& e) {
        d->error = e.what();
        return -1;
    }
}

int mtb_fuse_embeds(mtb_decoder* d, const int32_t* ids, int seq, const float* audio, int n_audio, int audio_token_id,
                    float* out) {
    if (!d || !out) return -1;
    d->fresh = false;
    try {
        cudaSetDevice(d->device);
        if (fuse_on_device(d, ids, seq, audio, n_audio, audio_token_id)) return -1;
        const size_t bytes = size_t(seq) * d->model->dm.dims.hidden * 4;
        d->d2h_bytes += (long long)bytes;
        MTB_CK(d, cudaMemcpyAsync(out, d->fused_dev, bytes, cudaMemcpyDeviceToHost, d->stream));
        MTB_CK(d, cudaStreamSynchronize(d->stream));
        return 0;
    } catch (const std::exception& e) {
        d->error = e.what();
        return -1;
    }
}

int mtb_spec_generate_ids(mtb_decoder* d, const int32_t* ids, int seq, const float* audio, int n_audio,
                          int audio_token_id, int max_new, int eos, const mtb_spec_params* params, int32_t* out_ids,
                          int* n_out, mtb_counters* counters) {
    if (!d || !out_ids || !n_out) return -1;
    d->fresh = false;
    *n_out = 0;
    try {
        cudaSetDevice(d->device);
        if (refresh(d)) return -1;
        if (set_params(d, max_new, eos, params)) return -1;
        const double t0 = wall_s();
        if (fuse_on_device(d, ids, seq, audio, n_audio, audio_token_id)) return -1;
        if (prefill(d, d->fused_dev, seq, true)) return -1;
        const double t1 = wall_s();
        StepState& s = *d->h_state;
        int i = 0;
        for (;;) {  // device-driven loop, as in mtb_spec_generate without hooks
            if (run_step(d, 0)) return -1;
            MTB_CK(d, cudaMemcpyAsync(&d->h_flag[i & 1], &d->b.state->stop, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
            MTB_CK(d, cudaEventRecord(d->ev[i & 1], d->stream));
            if (i > 0) {
                MTB_CK(d, cudaEventSynchronize(d->ev[(i - 1) & 1]));
                if (d->h_flag[(i - 1) & 1] != STOP_NONE) break;
            }
            ++i;
        }
        if (refresh(d)) return -1;
        MTB_CK(d, cudaMemcpyAsync(out_ids, d->b.ids, size_t(s.n_ids) * 4, cudaMemcpyDeviceToHost, d->stream));
        MTB_CK(d, cudaStreamSynchronize(d->stream));
        *n_out = s.n_ids;
        fill_counters(s, counters);
        mtb_counters c{};
        fill_counters(s, &c);
        emit_generation_log(out_ids, s.n_ids, s.eos, c, s.k_max, t1 - t0, wall_s() - t1);
        return 0;
    } catch (const std::exception& e) {
        d->error = e.what();
        return -1;
    }
}

int mtb_greedy_generate(mtb_decoder* d, const float* fused, int seq, int max_new, int eos, float penalty,
                        int32_t* out_ids, int* n_out) {
    const mtb_spec_params p{0, 2, 16, penalty};
    mtb_counters c{};
    return mtb_spec_generate(d, fused, seq, max_new, eos, &p, out_ids, n_out, &c, nullptr, nullptr, nullptr);
}

int mtb_resume(mtb_decoder* d, const int32_t* ids, int n_ids, int past, int max_new, int eos,
               const mtb_spec_params* params) {
    if (!d || !ids || n_ids <= 0) return -1;
    d->fresh = false;
    cudaSetDevice(d->device);
    if (refresh(d)) return -1;
    if (set_params(d, max_new, eos, params)) return -1;
    if (n_ids > max_new) return fail(d->error, "n_ids exceeds max_new");
    if (past < 0 || past + 1 > d->max_seq) return fail(d->error, "past out of range");
    const int vocab = d->model->dm.dims.vocab;
    for (int i = 0; i < n_ids; ++i)
        if (ids[i] < 0 || ids[i] >= vocab) return fail(d->error, "invalid token id");
    StepState& s = *d->h_state;
    clear_progress(s);
    s.past = past;
    s.n_ids = n_ids;
    s.seed = ids[n_ids - 1];
    std::memcpy(d->h_ids, ids, size_t(n_ids) * 4);
    d->h2d_bytes += size_t(n_ids) * 4;
    MTB_CK(d, cudaMemcpyAsync(d->b.ids, d->h_ids, size_t(n_ids) * 4, cudaMemcpyHostToDevice, d->stream));
    if (push_state(d)) return -1;
    // No synchronisation: the host copy of the state is what the device will
    // hold once the copies run (every later change of it is pushed again, in
    // stream order), so the next step needs no read-back.
    d->fresh = true;
    return 0;
}

int mtb_spec_step(mtb_decoder* d, const int32_t* draft, int n_draft, mtb_counters* counters) {
    if (!d) return -1;
    cudaSetDevice(d->device);
    if (refresh(d)) return -1;
    StepState& s = *d->h_state;
    int mode = 0;
    if (draft) {
        if (n_draft < 0 || n_draft > kTMax - 1) return fail(d->error, "n_draft must be in [0, 15]");
        const int vocab = d->model->dm.dims.vocab;
        for (int i = 0; i < n_draft; ++i) {
            if (draft[i] < 0 || draft[i] >= vocab) return fail(d->error, "invalid draft token");
            s.tokens[1 + i] = draft[i];
        }
        s.n_prop = n_draft;
        if (push_state(d)) return -1;
        mode = 1;
    }
    d->fresh = false;
    if (run_step(d, mode)) return -1;
    if (refresh(d)) return -1;
    fill_counters(s, counters);
    return 0;
}

int mtb_spec_step_async(mtb_decoder* d, const int32_t* draft_device, int n_draft) {
    if (!d) return -1;
    d->fresh = false;
    cudaSetDevice(d->device);
    int mode = 0;
    if (draft_device) {
        if (n_draft < 0 || n_draft > kTMax - 1) return fail(d->error, "n_draft must be in [0, 15]");
        launch_set_forced(d->b, draft_device, n_draft, d->model->dm.dims.vocab, d->stream);
        MTB_CK(d, cudaGetLastError());
        mode = 1;
    }
    cudaGraphExec_t g = step_graph(d, mode, d->h_state->penalty > 1.f);
    if (!g) return fail(d->error, "could not build the verify-step graph");
    MTB_CK(d, cudaGraphLaunch(g, d->stream));
    return 0;
}

int mtb_spec_prime(mtb_decoder* d, const float* fused, int seq, int max_new, int eos, const mtb_spec_params* params) {
    if (!d || !fused || seq <= 0) return -1;
    d->fresh = false;
    try {
        cudaSetDevice(d->device);
        if (refresh(d)) return -1;
        if (set_params(d, max_new, eos, params)) return -1;
        // No wait for the prefill: a group's members prime one after another
        // and their prefills overlap on their own streams.
        return prefill(d, fused, seq, false, true);
    } catch (const std::exception& e) {
        d->error = e.what();
        return -1;
    }
}

namespace {

// The group's requirements: 1..kMaxStreams distinct decoders of one model
// (the persistent kernel available, no repetition penalty), one KV type, and
// attention partial buffers of ds[0] that cover every member's cache.
int check_group(mtb_decoder* const* ds, int n) {
    if (!ds || n < 1 || n > kMaxStreams || !ds[0]) {
        g_error = "a group has 1 to " + std::to_string(kMaxStreams) + " decoders";
        return -1;
    }
    mtb_decoder* d0 = ds[0];
    if (d0->model->mega_grid <= 0) return fail(d0->error, "group steps need the persistent verify kernel");
    for (int i = 0; i < n; ++i) {
        mtb_decoder* di = ds[i];
        if (!di) return fail(d0->error, "null decoder in the group");
        for (int j = 0; j < i; ++j)
            if (ds[j] == di) return fail(d0->error, "a decoder appears twice in the group");
        if (di->model != d0->model) return fail(d0->error, "group decoders must share one model");
        if (di->kv_type != d0->kv_type) return fail(d0->error, "group decoders must share one KV type");
        if (di->b.max_chunks > d0->b.max_chunks)
            return fail(d0->error, "the first decoder of a group needs the largest max_seq");
        if (di->h_state->penalty > 1.f) return fail(d0->error, "group steps take no repetition penalty");
    }
    return 0;
}

// The group step on ds[0]'s stream, ordered after every member's queued work
// and before its later work.
int group_step(mtb_decoder* const* ds, int n) {
    mtb_decoder* d0 = ds[0];
    for (int i = 0; i < n; ++i) ds[i]->fresh = false;
    KvCache kvs[kMaxStreams];
    KvTensorMap maps[kMaxStreams];
    StepState* states[kMaxStreams];
    int32_t* ids[kMaxStreams];
    for (int i = 1; i < n; ++i) {
        MTB_CK(d0, cudaEventRecord(ds[i]->group_ev, ds[i]->stream));
        MTB_CK(d0, cudaStreamWaitEvent(d0->stream, ds[i]->group_ev, 0));
    }
    for (int i = 0; i < n; ++i) {
        launch_draft(ds[i]->b, 0, d0->stream);
        kvs[i] = ds[i]->kv;
        maps[i] = ds[i]->kv_map;
        states[i] = ds[i]->b.state;
        ids[i] = ds[i]->b.ids;
    }
    const mtb_model* m = d0->model;
    MTB_CK(d0, launch_step_persistent_group(m->dm, m->layers_dev, kvs, maps, states, ids, n, d0->b, d0->mb,
                                            m->mega_grid, d0->stream));
    MTB_CK(d0, cudaEventRecord(d0->group_ev, d0->stream));
    for (int i = 1; i < n; ++i) MTB_CK(d0, cudaStreamWaitEvent(ds[i]->stream, d0->group_ev, 0));
    return 0;
}

}  // namespace

int mtb_spec_step_group_async(mtb_decoder* const* ds, int n) {
    if (check_group(ds, n)) return -1;
    cudaSetDevice(ds[0]->device);
    return group_step(ds, n);
}

int mtb_spec_run_group(mtb_decoder* const* ds, int n, int max_steps, int* steps_out) {
    if (steps_out) *steps_out = 0;
    if (check_group(ds, n)) return -1;
    mtb_decoder* d0 = ds[0];
    cudaSetDevice(d0->device);
    // Device-driven loop on the first member's stream: the members' earlier
    // work is ordered before it once (events), then each step is two launches
    // (the members' drafts in one kernel, the verify step) and a one-int flag
    // copy; the host reads the flag one step behind.  The final
    // synchronisation orders the members' later work after the loop.
    for (int k = 1; k < n; ++k) {
        MTB_CK(d0, cudaEventRecord(ds[k]->group_ev, ds[k]->stream));
        MTB_CK(d0, cudaStreamWaitEvent(d0->stream, ds[k]->group_ev, 0));
    }
    DraftGroup g{};
    KvCache kvs[kMaxStreams];
    KvTensorMap maps[kMaxStreams];
    StepState* states[kMaxStreams];
    int32_t* idv[kMaxStreams];
    g.n = n;
    for (int k = 0; k < n; ++k) {
        g.st[k] = states[k] = ds[k]->b.state;
        g.ids[k] = idv[k] = ds[k]->b.ids;
        kvs[k] = ds[k]->kv;
        maps[k] = ds[k]->kv_map;
    }
    const mtb_model* m = d0->model;
    int i = 0;
    for (; max_steps <= 0 || i < max_steps; ++i) {
        for (int k = 0; k < n; ++k) ds[k]->fresh = false;
        launch_draft_group(g, d0->stream);
        MTB_CK(d0, launch_step_persistent_group(m->dm, m->layers_dev, kvs, maps, states, idv, n, d0->b, d0->mb,
                                                m->mega_grid, d0->stream));
        launch_group_stopped(g, d0->group_flag + (i & 1), d0->stream);
        MTB_CK(d0, cudaMemcpyAsync(&d0->h_flag[i & 1], d0->group_flag + (i & 1), sizeof(int), cudaMemcpyDeviceToHost,
                                   d0->stream));
        d0->d2h_bytes += sizeof(int);
        MTB_CK(d0, cudaEventRecord(d0->ev[i & 1], d0->stream));
        if (i > 0) {
            MTB_CK(d0, cudaEventSynchronize(d0->ev[(i - 1) & 1]));
            if (d0->h_flag[(i - 1) & 1]) { ++i; break; }
        }
    }
    MTB_CK(d0, cudaStreamSynchronize(d0->stream));
    if (steps_out) *steps_out = i;
    for (int k = 0; k < n; ++k)
        if (refresh(ds[k])) {
            if (k) d0->error = ds[k]->error;
            return -1;
        }
    return 0;
}

int mtb_snapshot_save(mtb_decoder* d) {
    if (!d) return -1;
    cudaSetDevice(d->device);
    MTB_CK(d, cudaMemcpyAsync(d->snap_state, d->b.state, sizeof(StepState), cudaMemcpyDeviceToDevice, d->stream));
    MTB_CK(d, cudaMemcpyAsync(d->snap_ids, d->b.ids, size_t(d->max_new) * 4, cudaMemcpyDeviceToDevice, d->stream));
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    return 0;
}

int mtb_snapshot_restore_async(mtb_decoder* d) {
    if (!d) return -1;
    d->fresh = false;
    cudaSetDevice(d->device);
    MTB_CK(d, cudaMemcpyAsync(d->b.state, d->snap_state, sizeof(StepState), cudaMemcpyDeviceToDevice, d->stream));
    MTB_CK(d, cudaMemcpyAsync(d->b.ids, d->snap_ids, size_t(d->max_new) * 4, cudaMemcpyDeviceToDevice, d->stream));
    return 0;
}

int mtb_read_ids(mtb_decoder* d, int32_t* out, int max_out, int* n_out, mtb_counters* counters) {
    if (!d) return -1;
    cudaSetDevice(d->device);
    if (refresh(d)) return -1;
    const int n = std::min(d->h_state->n_ids, std::max(0, max_out));
    if (out && n > 0) {
        d->d2h_bytes += size_t(n) * 4;
        MTB_CK(d, cudaMemcpyAsync(out, d->b.ids, size_t(n) * 4, cudaMemcpyDeviceToHost, d->stream));
        MTB_CK(d, cudaStreamSynchronize(d->stream));
    }
    if (n_out) *n_out = d->h_state->n_ids;
    fill_counters(*d->h_state, counters);
    return 0;
}

int mtb_sync(mtb_decoder* d) {
    if (!d) return -1;
    cudaSetDevice(d->device);
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    return 0;
}

int mtb_event_record(mtb_decoder* d, int slot) {
    if (!d || slot < 2 || slot > 15) return -1;  // slots 0-1 are used by the generate loop
    cudaSetDevice(d->device);
    MTB_CK(d, cudaEventRecord(d->ev[slot], d->stream));
    return 0;
}

int mtb_event_elapsed_ms(mtb_decoder* d, int a, int b, float* ms) {
    if (!d || !ms || a < 2 || a > 15 || b < 2 || b > 15) return -1;
    cudaSetDevice(d->device);
    MTB_CK(d, cudaEventSynchronize(d->ev[b]));
    MTB_CK(d, cudaEventElapsedTime(ms, d->ev[a], d->ev[b]));
    return 0;
}

int mtb_transfer_bytes(mtb_decoder* d, int64_t* h2d, int64_t* d2h) {
    if (!d) return -1;
    if (h2d) *h2d = d->h2d_bytes;
    if (d2h) *d2h = d->d2h_bytes;
    return 0;
}

int mtb_step_timeline(mtb_decoder* d, int64_t* out, int max_out, int* n_out) {
    if (!d || !out || !n_out) return -1;
    *n_out = 0;
    if (!d->mb.timeline) return fail(d->error, "set MTB_PROFILE=1 before creating the decoder");
    cudaSetDevice(d->device);
    const int n = std::min(max_out, 6 * kMaxBarriers + 2 + 256 * kMaxBarriers * 17);
    MTB_CK(d, cudaMemcpyAsync(out, d->mb.timeline, size_t(n) * 8, cudaMemcpyDeviceToHost, d->stream));
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    *n_out = n;
    return 0;
}

int mtb_step_capture(mtb_decoder* d, float* hidden_out, float* max_val, int32_t* max_idx, int32_t* stream_rows,
                     int* T_out) {
    if (!d || !T_out) return -1;
    *T_out = 0;
    if (!d->mb.capture) return fail(d->error, "set MTB_STEP_CAPTURE=1 before creating the decoder");
    cudaSetDevice(d->device);
    const int H = d->model->dm.dims.hidden;
    std::vector<float> cap(step_capture_floats(H));
    MTB_CK(d, cudaMemcpyAsync(cap.data(), d->mb.capture, cap.size() * 4, cudaMemcpyDeviceToHost, d->stream));
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    const float* mx = cap.data() + size_t(kTMax) * H;
    const int32_t* rows = reinterpret_cast<const int32_t*>(mx + 2 * kTMax);
    const int T = std::max(0, std::min(kTMax, rows[2 * kMaxStreams]));
    if (hidden_out) std::memcpy(hidden_out, cap.data(), size_t(T) * H * 4);
    for (int t = 0; t < T; ++t) {
        if (max_val) max_val[t] = mx[2 * t];
        if (max_idx) std::memcpy(&max_idx[t], &mx[2 * t + 1], 4);
    }
    if (stream_rows) std::memcpy(stream_rows, rows, 2 * kMaxStreams * 4);
    *T_out = T;
    return 0;
}

int mtb_debug_poison_kv(mtb_decoder* d, int pos0, int n_pos) {
    if (!d) return -1;
    if (pos0 < 0 || n_pos < 0 || pos0 + n_pos > d->max_seq) return fail(d->error, "poison range outside the cache");
    if (n_pos == 0) return 0;
    cudaSetDevice(d->device);
    launch_poison_kv(d->model->dm, d->kv, pos0, n_pos, d->stream);
    MTB_CK(d, cudaGetLastError());
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    return 0;
}

int mtb_step_kernel_launches(mtb_decoder* d) {
    if (!d) return -1;
    cudaSetDevice(d->device);
    if (!step_graph(d, 1, d->h_state->penalty > 1.f)) return -1;
    return d->launches;
}

int mtb_ngram_draft(mtb_decoder* d, const int32_t* history, int n, int maximum, int n_min, int n_max, int32_t* out,
                    int* n_out) {
    if (!d || !out || !n_out || n < 0 || n > d->max_new || (n > 0 && !history)) return -1;
    d->fresh = false;
    if (n_min < 1 || n_max < n_min) return fail(d->error, "need 1 <= n_min <= n_max");
    cudaSetDevice(d->device);
    if (n > 0) MTB_CK(d, cudaMemcpyAsync(d->scratch_i, history, size_t(n) * 4, cudaMemcpyHostToDevice, d->stream));
    int32_t* dev_out = d->scratch_i + n;  // the proposal never exceeds n ids; scratch holds max_new + 16
    if (maximum > 16 && n + std::min(maximum, n) > d->max_new + 16) return fail(d->error, "history too long");
    launch_draft_args(d->scratch_i, n, maximum, n_min, n_max, dev_out, d->scratch_n, d->stream);
    MTB_CK(d, cudaGetLastError());
    int cnt = 0;
    MTB_CK(d, cudaMemcpyAsync(&cnt, d->scratch_n, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    if (cnt > 0) {
        MTB_CK(d, cudaMemcpyAsync(out, dev_out, size_t(cnt) * 4, cudaMemcpyDeviceToHost, d->stream));
        MTB_CK(d, cudaStreamSynchronize(d->stream));
    }
    *n_out = cnt;
    return 0;
}

int mtb_greedy_choice(mtb_decoder* d, const float* raw, int n_raw, const int32_t* history, int n, float penalty,
                      int32_t* choice) {
    if (!d || !raw || !choice || n_raw <= 0 || n < 0 || n > d->max_new || (n > 0 && !history)) return -1;
    d->fresh = false;
    if (n_raw > d->model->dm.dims.vocab) return fail(d->error, "more logits than the vocabulary");
    cudaSetDevice(d->device);
    MTB_CK(d, cudaMemcpyAsync(d->b.logits, raw, size_t(n_raw) * 4, cudaMemcpyHostToDevice, d->stream));
    if (n > 0) MTB_CK(d, cudaMemcpyAsync(d->scratch_i, history, size_t(n) * 4, cudaMemcpyHostToDevice, d->stream));
    launch_choice_args(d->b.logits, n_raw, d->scratch_i, n, penalty, d->scratch_n, d->stream);
    MTB_CK(d, cudaGetLastError());
    int c = 0;
    MTB_CK(d, cudaMemcpyAsync(&c, d->scratch_n, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
    MTB_CK(d, cudaStreamSynchronize(d->stream));
    *choice = c;
    return 0;
}

}  // extern "C"
