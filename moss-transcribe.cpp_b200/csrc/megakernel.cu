// The verify step as one persistent kernel (one CTA per SM).
//
// Why: a verify step is 28 layers x ~10 dependent operations of a few
// microseconds each; as separate launches most of the step is launch gaps.
// Here every operation is a phase of one kernel, phases are separated by grid
// barriers, and one producer warp per CTA streams every weight tile the CTA
// will need (all layers, then the LM head) through a ring of shared-memory
// slots with cp.async.bulk (weights) and TMA tensor tiles (K/V) + mbarriers.
// Weights do not depend on the step's activations, so HBM keeps streaming
// while the consumer warps wait at barriers; the consumers find their tiles
// already in shared memory.  One launch may verify several decoders' rows
// together (a stream table: each stream its own KV cache, positions, draft
// and acceptance).
//
// Phases per layer (src/qwen3.cpp:62-218):
//   A  RMSNorm + q8_0 quantise (every CTA, into shared memory); QKV rows
//   B  attention per (stream, 64-position chunk, kv head): per-head RMSNorm + RoPE of
//      the head's q rows (and of k for the step's new positions, stored to
//      the KV cache with the new v rows by the item holding them), scores,
//      chunk softmax, P.V partials; the chunk's K/V rows streamed into the
//      ring by the producer like weights
//   C  chunk merge per (row, q head, 32-dim block) and q8_0 quantise of the
//      context
//   D  O projection + residual
//   E  RMSNorm + quantise; gate/up + SwiGLU per 32-feature block, quantised
//      for the down projection by the CTA that computed it
//   F  down projection + residual
// then the final RMSNorm, the LM head with a fused first max, and the
// acceptance / rollback of src/cpu_speculative.cpp:124-135 (CTA 0).
//
// Every operation evaluates the same arithmetic in the same order as the
// multi-kernel path (kernels.cu) and the CPU restatement, so the results are
// identical bit for bit.  All waits (grid barrier, mbarriers) are bounded by
// a time limit; on expiry the kernel records an error in the step state,
// raises an abort flag that every other wait watches, drains its own bulk
// copies and returns.
#include <cuda.h>

#include "device_common.cuh"

#include <algorithm>
#include <cstring>

namespace mtb {
namespace {

using namespace dev;

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kMegaThreads = kConsumers + 32;   // + the producer warp
constexpr int kSlotBytes = 16 * kTileBytes;      // 8704: 16 tiles = 4 slices of 256 K
constexpr int kRingSlots = 16;
constexpr int kRegionBytes = 64 * 1024;          // activation fragments / attention scratch
constexpr int kRopeBytes = kTMax * 64 * 2 * 4;   // cos/sin of the step's positions
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s bound on every wait
constexpr unsigned kSuspendHintNs = 20000;             // longest sleep in one mbarrier try_wait
constexpr int kTimelineStart = 2 * kMaxBarriers;       // kernel start / end slots
constexpr int kArrivalBase = 6 * kMaxBarriers + 2;     // [cta][barrier] arrivals after the marks
constexpr int kCtaMarkBase = kArrivalBase + 256 * kMaxBarriers;  // [cta][barrier][16] sub-phase marks
constexpr int kCtaMarks = 16;
// Timeline indices of the sub-phase marks of D (O) and F (down) of layer l,
// which have no grid barrier of their own: past every barrier index.
constexpr int kSubPhaseO = 320;
constexpr int kSubPhaseDown = 384;

// Shared memory, named at file scope so that every function's accesses
// compile to shared-window loads and stores (a pointer kept in memory, or a
// pointer parameter of a non-inlined function, would be a generic address).
// Dynamic: the ring (kRingSlots slots), the region (activation fragments,
// slice partials, attention scratch), the RoPE table, the ring's mbarriers.
extern __shared__ __align__(1024) uint8_t g_smem[];
__shared__ float2 g_cand[kConsumerWarps * kTMax];
__shared__ int g_flag;
__shared__ __align__(8) uint64_t g_lm_bars[4];  // tcgen05 LM head: half_full[2], half_free[2]
__shared__ uint32_t g_tmem;                      // TMEM base address of the tcgen05 LM head
__shared__ float g_qk_norm[2 * kHeadDim];        // the layer's q_norm and k_norm weights, staged by phase A for B

__device__ __forceinline__ uint8_t* s_ring() { return g_smem; }
__device__ __forceinline__ uint8_t* s_region() { return g_smem + (size_t)kRingSlots * kSlotBytes; }
__device__ __forceinline__ float* s_rope() { return reinterpret_cast<float*>(g_smem + (size_t)kRingSlots * kSlotBytes + kRegionBytes); }
__device__ __forceinline__ uint64_t* s_full() {
    return reinterpret_cast<uint64_t*>(g_smem + (size_t)kRingSlots * kSlotBytes + kRegionBytes + kRopeBytes);
}
__device__ __forceinline__ uint64_t* s_empty() { return s_full() + kRingSlots; }

struct MegaArgs {
    ModelDims d;
    const LayerWeights* layers;  // device array
    const uint8_t* embd;
    const uint8_t* lm_tiles;  // token_embd as tcgen05 weight steps: LM head on the tensor cores, or null
    const float* output_norm;
    float theta_scale;
    // Streams verified together (one decoder each: its KV cache, step state
    // and ids).  The step's rows are the streams' rows in stream order; a
    // single decoder is the one-stream case.
    int n_streams;
    KvCache st_kv[kMaxStreams];
    StepState* st_state[kMaxStreams];
    int32_t* st_ids[kMaxStreams];
    float* x;        // [16][H]
    float* qkv;      // [16][qd + 2 kd]
    float* gu;       // [16][F]
    uint8_t* act_q;  // context fragments (K = qd), then reused for K = F below
    float* act_d;
    uint8_t* act2_q; // SwiGLU fragments (K = F)
    float* act2_d;
    float* part_o;
    float2* part_ml;
    int max_chunks;
    float2* lm_val;  // [grid][16]
    unsigned* bar;   // grid barrier counter, zero at launch
    unsigned* head_done;  // [n_layers][kMaxStreams][n_kv] finished attention items per kv head, zero at launch
    unsigned* pair_done;  // [n_layers][n_heads / 2] merged (row, q head, block) tasks per pair of q heads, zero at launch
    unsigned* slice_done; // [n_layers][ffn / 256] finished gate/up blocks per 256-feature slice, zero at launch
    unsigned* m_max;      // [n_layers][n_kv][64] running max of the chunk maxima per (kv head, partial row), ordered bits, zero at launch
    int* abort_flag;
    unsigned long long wait_ns;  // bound on a grid-barrier wait
    int stall_barrier;           // test hook: CTA 0 does not arrive at this barrier (-1: off)
    unsigned long long* timeline;  // optional: CTA 0's [barrier][arrive, release] in ns
    float* capture;                // optional: the step's final-normed rows and LM-head maxima (test read-back)
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or the hint (ns) runs out, instead of spinning on the issue slots
// its warp scheduler shares with the consumer warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* b, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(b)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase; false on timeout or abort.
__device__ bool mbar_wait(uint64_t* b, unsigned parity, const int* abort_flag) {
    if (mbar_try_wait(b, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(b, parity)) return true;
        if (*reinterpret_cast<const volatile int*>(abort_flag)) return false;
        if (global_ns() - t0 > kWaitNs) return false;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(b)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(b))
        : "memory");
}


// Sub-phase mark k (0..3) of phase b in the optional timeline (CTA 0, thread 0).
__device__ __forceinline__ void mark(unsigned long long* timeline, int b, int k) {
    if (!timeline || threadIdx.x != 0 || b < 0 || b >= kMaxBarriers || blockIdx.x >= 256) return;
    const unsigned long long t = global_ns();
    if (blockIdx.x == 0 && k < 4) timeline[2 * kMaxBarriers + 2 + 4 * b + k] = t;
    if (k < kCtaMarks) timeline[kCtaMarkBase + ((size_t)blockIdx.x * kMaxBarriers + b) * kCtaMarks + k] = t;
}

// 2-D TMA tensor tile (box of the map) at coordinates (x, y) into shared
// memory, completing bytes on mbarrier b.  No multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(b))
        : "memory");
}

// ------------------------------------------------------------------ schedule

// Streamed phases in ring order: per layer A (QKV rows), B (the K/V rows of
// the attention items), D (O), E (gate/up pair), F (down); then G (LM head).
// Item i of a phase goes to CTA (i + rot) % grid, where rot is the number of
// items in all earlier streamed phases, so the work rotates over the CTAs from
// phase to phase.
enum WPhase { W_QKV = 0, W_ATTN = 1, W_O = 2, W_GU = 3, W_DOWN = 4, W_LM = 5 };
constexpr int kLayerPhases = 5;

// An attention item's K and V chunk rows in the ring: 64 rows each, 32 (fp16)
// or 16 (f32) rows per slot, so one item takes 4 (fp16) or 8 (f32) slots: K
// rows first, then V rows.  A slot holds its rows as 128-byte boxes (bytes
// [128 b, 128 b + 128) of every row, box after box), each written by one TMA
// tensor tile copy with the 128-byte swizzle: 16-byte chunk c of row p sits
// at chunk c ^ (p & 7) of the row's 128 bytes, so 16-byte reads of one chunk
// of 8 consecutive rows hit 8 different bank quads.  The boxes start at the
// slot's first 1024-byte boundary (the swizzle's alignment): slots are
// kSlotBytes = 8.5 KB apart in a 1024-aligned ring, so at +0 (even slots) or
// +512 (odd slots), and 8 KB of boxes fit either way.
template <bool F16>
struct KvSlots {
    static constexpr int kRowBytes = F16 ? 256 : 512;
    static constexpr int kRowsPerSlot = F16 ? 32 : 16;
    static constexpr int kSlotsPerHalf = kPage / kRowsPerSlot;
    static constexpr int kBoxBytes = kRowsPerSlot * 128;
    static constexpr int kBoxes = kRowBytes / 128;
};

// The K/V boxes of ring slot s.
__device__ __forceinline__ uint8_t* kv_slot_base(uint8_t* ring, int s) {
    return ring + (size_t)s * kSlotBytes + (s & 1) * 512;
}
// The same as a byte offset from the ring's start (1024-aligned).
__device__ __forceinline__ uint32_t kv_slot_off(int s) { return (uint32_t)s * kSlotBytes + (uint32_t)(s & 1) * 512u; }

struct PhaseInfo {
    int n_items;    // items in the phase
    int rot;        // rotation
    int bytes;      // streamed bytes per item
    int slots;      // ring slots per item
    int count;      // items of this CTA
    int first;      // first global item of this CTA
    long long slot0;  // first ring slot sequence number of this phase for this CTA
};

struct Schedule {
    int grid, cta;
    int qd, kd, H, F, V, L, nkv;
    bool kv_f16;
    // sizes per streamed phase kind, and n's quotient and remainder by the
    // grid (so a phase's item count and rotation need no division)
    int n[6], bytes[6], nq[6], nr[6], nslots[6];
    bool lm_tc;  // LM head items are 128-row tcgen05 weight tiles (else 8-row mma.sync tiles)
    int n_str;
    int item0[kMaxStreams + 1];  // first attention item of each stream (items: stream, chunk, kv head)
    __device__ void init(const ModelDims& d, int grid_, int cta_, bool kv_f16_, const int* chunks, int n_str_,
                         bool lm_tc_) {
        lm_tc = lm_tc_;
        n_str = n_str_;
        item0[0] = 0;
        for (int i = 0; i < n_str; ++i) item0[i + 1] = item0[i] + chunks[i] * d.n_kv;
        grid = grid_;
        cta = cta_;
        H = d.hidden;
        F = d.ffn;
        V = d.vocab;
        L = d.n_layers;
        nkv = d.n_kv;
        kv_f16 = kv_f16_;
        qd = d.n_heads * kHeadDim;
        kd = d.n_kv * kHeadDim;
        n[W_QKV] = (qd + 2 * kd) / kTileRows;
        bytes[W_QKV] = (H / kTileK) * kTileBytes;
        n[W_ATTN] = item0[n_str];  // (stream, chunk, kv head) items
        bytes[W_ATTN] = 2 * (kv_f16 ? KvSlots<true>::kSlotsPerHalf : KvSlots<false>::kSlotsPerHalf) * kSlotBytes;
        n[W_O] = H / kTileRows;
        bytes[W_O] = (qd / kTileK) * kTileBytes;
        n[W_GU] = F / 32;  // 32-feature blocks: four (gate, up) pairs of row groups
        bytes[W_GU] = 8 * (H / kTileK) * kTileBytes;
        n[W_DOWN] = H / kTileRows;
        bytes[W_DOWN] = (F / kTileK) * kTileBytes;
        n[W_LM] = lm_tc ? V / 128 : V / kTileRows;
        bytes[W_LM] = lm_tc ? (H / 64) * kSlotBytes : (H / kTileK) * kTileBytes;
        for (int k = 0; k < 6; ++k) {
            nq[k] = n[k] / grid;
            nr[k] = n[k] % grid;
            nslots[k] = (bytes[k] + kSlotBytes - 1) / kSlotBytes;
        }
    }
    __device__ int slots_of(int kind) const { return nslots[kind]; }
    // Attention item -> (stream, chunk, kv head).
    __device__ void attn_item_of(int item, int* str, int* chunk, int* h) const {
        int si = 0;
        while (si + 1 < n_str && item >= item0[si + 1]) ++si;
        *str = si;
        *chunk = (item - item0[si]) / nkv;
        *h = (item - item0[si]) % nkv;
    }
    // Items of phase `kind` for this CTA, with the phase rotated by `rot`
    // (0 <= rot < grid): the items first, first + grid, ... below n[kind].
    __device__ int count_of(int kind, int rot, int* first) const {
        int f = cta - rot;
        if (f < 0) f += grid;
        *first = f;
        return nq[kind] + (f < nr[kind] ? 1 : 0);
    }
    // The rotation of the phase after one of `kind` with rotation rot.
    __device__ int next_rot(int kind, int rot) const {
        int r = rot + nr[kind];
        return r >= grid ? r - grid : r;
    }
    // Running position in the phase sequence: both the producer and the
    // consumers advance it phase by phase (cursor[0] = the next phase's
    // rotation, cursor[1] = its first ring slot), so neither recomputes the prefix.
    __device__ PhaseInfo take(int kind, long long* rot_cursor, long long* slot_next) const {
        PhaseInfo pi{};
        pi.n_items = n[kind];
        pi.rot = int(*rot_cursor);
        pi.bytes = bytes[kind];
        pi.slots = nslots[kind];
        pi.count = count_of(kind, pi.rot, &pi.first);
        pi.slot0 = *slot_next;
        *rot_cursor = next_rot(kind, pi.rot);
        *slot_next += (long long)pi.count * pi.slots;
        return pi;
    }
    __device__ const uint8_t* item_src(const LayerWeights* lw, const uint8_t* embd, int kind, int layer, int item) const {
        if (kind == W_LM) return embd + (size_t)item * bytes[W_LM];  // embd: the LM-head source of this schedule
        const LayerWeights& w = lw[layer];
        switch (kind) {
            case W_QKV: return w.qkv + (size_t)item * bytes[W_QKV];
            case W_O: return w.o + (size_t)item * bytes[W_O];
            case W_GU: return w.gu + (size_t)item * bytes[W_GU];
            default: return w.down + (size_t)item * bytes[W_DOWN];
        }
    }
};

// 16-byte chunk c (0 .. kRowBytes / 16 - 1) of row r (0..63) of the K (which
// = 0) or V (which = 1) rows of the attention item whose slots start at
// sequence number q0.
template <bool F16>
__device__ __forceinline__ uint8_t* kv_chunk(uint8_t* ring, long long q0, int which, int r, int c) {
    using KS = KvSlots<F16>;
    const long long q = q0 + which * KS::kSlotsPerHalf + r / KS::kRowsPerSlot;
    const int p = r % KS::kRowsPerSlot;
    return kv_slot_base(ring, int(q % kRingSlots)) + (c >> 3) * KS::kBoxBytes + p * 128 + (((c & 7) ^ (p & 7)) << 4);
}

// ------------------------------------------------------------------ producer

// The LM-head phase's copies.  Item j (one slot: 8 vocabulary rows x the
// whole hidden K) sits in slot (q0 + j) mod kRingSlots and is consumed by
// consumer warp j mod kConsumerWarps, so each warp alternates between two
// slots.  Producer lane l < kConsumerWarps refills the slots of warp l: every
// round each lane probes its next slot without blocking and issues the copy
// as soon as that slot is free, so one slow warp holds back only its own
// refills (in ring order, every refill would wait for the slowest warp).
// Returns false on abort or when no lane made progress for kWaitNs; the
// lanes then drain their own copies still in flight (bounded by the same
// limit: a copy outstanding after it is left behind, the step having failed).
__device__ bool producer_lm(const MegaArgs& a, const Schedule& sch, uint8_t* ring, uint64_t* full, uint64_t* empty,
                            long long q0, int cnt, int first) {
    const int lane = threadIdx.x & 31;
    const bool mine = lane < kConsumerWarps;
    int j = lane;  // this lane's next item
    bool ok = true;
    unsigned long long last = global_ns();
    for (unsigned round = 0;; ++round) {
        int issued = 0;
        if (mine && j < cnt) {
            const long long q = q0 + j;
            const int s = int(q % kRingSlots);
            const long long use = q / kRingSlots;
            if (use == 0 || mbar_try_wait(&empty[s], unsigned((use - 1) & 1))) {
                const uint8_t* src = sch.item_src(a.layers, a.embd, W_LM, 0, first + j * sch.grid);
                const unsigned nbytes = unsigned(sch.bytes[W_LM]);  // one item: at most one slot
                mbar_expect_tx(&full[s], nbytes);
                bulk_g2s(ring + (size_t)s * kSlotBytes, src, nbytes, &full[s]);
                j += kConsumerWarps;
                issued = 1;
            }
        }
        const unsigned prog = __ballot_sync(0xffffffffu, issued);
        if (!__any_sync(0xffffffffu, mine && j < cnt)) break;
        if (prog) {
            last = global_ns();
        } else {
            if ((round & 63) == 63) {
                if (*reinterpret_cast<const volatile int*>(a.abort_flag) || global_ns() - last > kWaitNs) { ok = false; break; }
            }
            __nanosleep(64);
        }
    }
    if (!ok) {
        if (lane == 0) atomicExch(a.abort_flag, 1);
        if (mine)
            for (int k = 1; k <= 2; ++k) {
                const int jj = j - k * kConsumerWarps;
                if (jj < 0) break;
                const long long q = q0 + jj;
                const unsigned long long t0 = global_ns();
                while (!mbar_try_wait(&full[q % kRingSlots], unsigned((q / kRingSlots) & 1)) && global_ns() - t0 < kWaitNs) {
                }
            }
    }
    return ok;
}

// The producer warp: lane 0 waits for free slots, posts the expected bytes
// and issues the copies: a weight item slot is one bulk copy, an attention
// slot one TMA tile per 128-byte box of its rows (kv_maps[stream]: the
// stream's cache as [rows][row bytes], box [rows per slot][128], swizzled).
__device__ void producer(const MegaArgs& a, const CUtensorMap* kv_maps, const Schedule& sch, uint8_t* ring,
                         uint64_t* full, uint64_t* empty) {
    const int lane = threadIdx.x & 31;
    long long q = 0;  // ring slot sequence number
    const int n_phases = sch.L * kLayerPhases + 1;
    bool ok = true;
    bool lm_lanes = false;  // the LM phase ran in producer_lm (which drains its own copies)
    int rot = 0;  // rotation of the current phase (Schedule::take)
    const int rps = sch.kv_f16 ? KvSlots<true>::kRowsPerSlot : KvSlots<false>::kRowsPerSlot;
    const int n_box = sch.kv_f16 ? KvSlots<true>::kBoxes : KvSlots<false>::kBoxes;
    const int box_bytes = sch.kv_f16 ? KvSlots<true>::kBoxBytes : KvSlots<false>::kBoxBytes;
    for (int p = 0; p < n_phases && ok; ++p) {
        const int kind = p < sch.L * kLayerPhases ? p % kLayerPhases : W_LM;
        const int layer = p / kLayerPhases;
        int first = 0;
        const int cnt = sch.count_of(kind, rot, &first);
        const int slots = sch.slots_of(kind);
        if (kind == W_LM && !sch.lm_tc && slots == 1) {
            // The LM head is the last phase: its items (one slot each) are
            // refilled per consumer warp rather than in ring order.
            lm_lanes = true;
            ok = producer_lm(a, sch, ring, full, empty, q, cnt, first);
            break;
        }
        long long lane_row = 0;  // attention: cache row of item (j & ~31) + lane's K block
        for (int j = 0; j < cnt && ok; ++j) {
            const int item = first + j * sch.grid;
            if (kind == W_ATTN && (j & 31) == 0 && j + lane < cnt) {
                // The next 32 items' page-table lookups at once, one per lane
                // (one at a time they would serialise the copies behind them).
                int si, chunk, h;
                sch.attn_item_of(first + (j + lane) * sch.grid, &si, &chunk, &h);
                lane_row = kv_offset(a.st_kv[si], sch.nkv, layer, 0, h, chunk * kPage) / kHeadDim;
            }
            const long long item_row = __shfl_sync(0xffffffffu, lane_row, j & 31);
            for (int k = 0; k < slots; ++k, ++q) {
                const int s = int(q % kRingSlots);
                const long long use = q / kRingSlots;
                int good = 1;
                if (lane == 0 && use > 0 && !mbar_wait(&empty[s], unsigned((use - 1) & 1), a.abort_flag)) good = 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
                uint8_t* dst = ring + (size_t)s * kSlotBytes;
                if (kind == W_ATTN) {
                    if (lane == 0) {
                        // The slot's rps rows: contiguous rows of one (layer,
                        // K/V, head) block of the item's cache page.
                        const int half = slots / 2, which = k / half, r0 = (k % half) * rps;
                        int si, chunk, h;
                        sch.attn_item_of(item, &si, &chunk, &h);
                        const int y = int(item_row + (long long)which * sch.nkv * kPage + r0);
                        uint8_t* boxes = kv_slot_base(ring, s);
                        mbar_expect_tx(&full[s], unsigned(n_box * box_bytes));
                        for (int b = 0; b < n_box; ++b) tma_load_2d(boxes + b * box_bytes, &kv_maps[si], b * 128, y, &full[s]);
                    }
                } else if (lane == 0) {
                    const uint8_t* src = sch.item_src(a.layers, sch.lm_tc ? a.lm_tiles : a.embd, kind, layer, item);
                    const int off = k * kSlotBytes;
                    const int nbytes = min(kSlotBytes, sch.bytes[kind] - off);
                    mbar_expect_tx(&full[s], unsigned(nbytes));
                    bulk_g2s(dst, src + off, unsigned(nbytes), &full[s]);
                }
            }
        }
        rot = sch.next_rot(kind, rot);
    }
    if (!ok && lane == 0 && !lm_lanes) {
        atomicExch(a.abort_flag, 1);
        // Drain this CTA's copies still in flight before the CTA exits, each
        // wait bounded by kWaitNs (best effort: a copy still outstanding after
        // that is left behind; the step has already failed).
        for (long long r = q - 1; r >= 0 && r >= q - kRingSlots; --r) {
            const int s = int(r % kRingSlots);
            const unsigned long long t0 = global_ns();
            while (!mbar_try_wait(&full[s], unsigned((r / kRingSlots) & 1)) && global_ns() - t0 < kWaitNs) {
            }
        }
    }
}

// ------------------------------------------------------------------ consumer pieces

// Grid barrier over the consumer warps of every CTA (the counter only grows;
// barrier b completes at (b + 1) * grid arrivals).  Returns false on abort.
// A wait of the step gave up: every stream's state carries the error.
__device__ __forceinline__ void report_timeout(const MegaArgs& a) {
    for (int s = 0; s < a.n_streams; ++s) a.st_state[s]->error = 2;
}

__device__ bool grid_barrier(const MegaArgs& a, unsigned target, int b, int* s_flag) {
    consumer_sync();
    if (threadIdx.x == 0) {
        if (a.timeline && blockIdx.x == 0) a.timeline[2 * b] = global_ns();
        // Every CTA's arrival, for the skew between CTAs.
        if (a.timeline && b < kMaxBarriers) a.timeline[kArrivalBase + (size_t)blockIdx.x * kMaxBarriers + b] = global_ns();
        // Arrive with release semantics (the CTA's writes, ordered before by the
        // named barrier, become visible with it); poll with relaxed loads, then
        // one acquire load of the completed count orders everything after it
        // (an acquire on every poll would invalidate the L1 each time).
        if (!(b == a.stall_barrier && blockIdx.x == 0))
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
        const unsigned long long t0 = global_ns();
        int status = 0;
        for (unsigned it = 0;; ++it) {
            unsigned v;
            asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
            if (v >= target) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
                break;
            }
            if ((it & 255) == 255) {
                if (*reinterpret_cast<volatile int*>(a.abort_flag)) { status = 1; break; }
                if (global_ns() - t0 > a.wait_ns) {
                    atomicExch(a.abort_flag, 1);
                    report_timeout(a);
                    status = 1;
                    break;
                }
            }
        }
        if (a.timeline && blockIdx.x == 0) a.timeline[2 * b + 1] = global_ns();
        *s_flag = status;
    }
    consumer_sync();
    return *s_flag == 0;
}

// A consumer wait that gave up: flag the step and let every wait stop.  The
// warp then carries on to the next grid barrier (never returns alone: the
// consumer warps of a CTA meet at named barriers), where all warps exit.
__device__ void consumer_fail(const MegaArgs& a) {
    if ((threadIdx.x & 31) == 0) {
        atomicExch(a.abort_flag, 1);
        report_timeout(a);
    }
}

// Wait for ring slot q (consumer side), lane-0 poll, warp-wide result.
__device__ __forceinline__ bool slot_wait(uint64_t* full, long long q, const int* abort_flag) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(&full[q % kRingSlots], unsigned((q / kRingSlots) & 1), abort_flag);
    return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Wait for ring slots q0 .. q0 + n - 1 (n <= 32), one lane per slot.
__device__ __forceinline__ bool slots_wait(uint64_t* full, long long q0, int n, const int* abort_flag) {
    const int lane = threadIdx.x & 31;
    bool ok = true;
    if (lane < n) ok = mbar_wait(&full[(q0 + lane) % kRingSlots], unsigned(((q0 + lane) / kRingSlots) & 1), abort_flag);
    return __all_sync(0xffffffffu, ok) != 0;
}

// RMSNorm (the hidden-row tree of row_rms_scale) and q8_0 quantisation of
// rows [T][K] of global x into shared fragments (rows >= T are left as they
// are: every consumer discards the outputs of those rows), one warp per row:
// lane l owns block l of the row (elements 32 l .. 32 l + 31, K <= 1024), so
// the block's square sum, amax and scale need no other lane; one butterfly
// makes the row's total.  The 32 codes of a (row, block) are 8 words of the
// fragment; lanes write them in an order rotated by the lane so that a
// warp's stores spread over the banks.
// kUmma: the output is the tcgen05 operand layout instead (16 rows x K bytes
// as 64-K steps of 1024 bytes, core matrix (row group, 16-byte chunk) at
// (4 group + chunk) * 128, row at +16 row; scales f32 [16][K / 32]).
// This consumer thread's float4 of a row-norm weight vector (K = 256 NK),
// requested before the grid barrier that precedes the norm.
template <int NK>
__device__ __forceinline__ float4 norm_weights_prefetch(const float* wn) {
    constexpr int K = 256 * NK;
    return threadIdx.x < K / 4 ? __ldg(reinterpret_cast<const float4*>(wn) + threadIdx.x) : make_float4(0.f, 0.f, 0.f, 0.f);
}

template <int NK, bool kUmma = false>
__device__ __noinline__ void norm_quant_smem(const float* x, float4 wpre, float eps, int T,
                                            unsigned long long* timeline = nullptr, int pid = 0,
                                            float* normed_out = nullptr) {
    constexpr int K = 256 * NK;
    constexpr int NB = K / 32;  // blocks per row: one per lane at most
    static_assert(NB <= 32, "one block per lane");
    static_assert((size_t)K * 16 + NB * 64 + (size_t)(kConsumerWarps + 1) * NB * 36 * 4 <= (size_t)kRegionBytes,
                  "fragments, scales and the staging buffers fit the region");
    // Fragments at the region's start, scales after them (K / 32 blocks x 512
    // bytes, or the tcgen05 layout's K / 64 steps x 1024 bytes: the same size).
    uint8_t* act_q = s_region();
    float* act_d = reinterpret_cast<float*>(s_region() + (size_t)K * 16);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool has = lane < NB;
    // Rows and the norm weights come in with coalesced 16-byte loads and are
    // turned around through staging buffers after the fragments and scales in
    // the region (blocks 36 floats apart: the 16-byte writes of 8 lanes and the
    // block reads of 8 lanes each hit 32 distinct banks): one per warp for its
    // rows, one shared for the weights.
    float* stage_all = reinterpret_cast<float*>(s_region() + (size_t)K * 16 + (size_t)NB * 16 * 4);
    float* stage = stage_all + warp * NB * 36;
    float* wstage = stage_all + kConsumerWarps * NB * 36;
    // This warp's first row is requested before the weights' round trip.
    float4 f[NB / 4];
    if (warp < T) {
        const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)warp * K);
#pragma unroll
        for (int k = 0; k < NB / 4; ++k) f[k] = __ldcg(x4 + 32 * k + lane);
    }
    // The norm weights came in before the grid barrier (norm_weights_prefetch):
    // they do not depend on the step, and after a barrier their HBM round trip
    // would add to the rows' L2 round trip.
    static_assert(K / 4 <= kConsumers, "one float4 of norm weights per consumer thread");
    if (threadIdx.x < K / 4)
        *reinterpret_cast<float4*>(wstage + (threadIdx.x >> 3) * 36 + 4 * (threadIdx.x & 7)) = wpre;
    consumer_sync();
    float wv[32];
    if (has) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 f = *reinterpret_cast<const float4*>(wstage + lane * 36 + 4 * i);
            wv[4 * i] = f.x; wv[4 * i + 1] = f.y; wv[4 * i + 2] = f.z; wv[4 * i + 3] = f.w;
        }
    }
    for (int row = warp; row < T; row += kConsumerWarps) {
        float v[32];
        {
            if (row != warp) {
                const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)row * K);
#pragma unroll
                for (int k = 0; k < NB / 4; ++k) f[k] = __ldcg(x4 + 32 * k + lane);
            }
#pragma unroll
            for (int k = 0; k < NB / 4; ++k)
                *reinterpret_cast<float4*>(stage + (4 * k + (lane >> 3)) * 36 + 4 * (lane & 7)) = f[k];
            __syncwarp();
            if (has) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 g = *reinterpret_cast<const float4*>(stage + lane * 36 + 4 * i);
                    v[4 * i] = g.x; v[4 * i + 1] = g.y; v[4 * i + 2] = g.z; v[4 * i + 3] = g.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0.f;
            }
            __syncwarp();  // the buffer is reused by this warp's next row
        }
        if (row == warp) mark(timeline, pid, 4);
        const double tot = warp_sum_d(has ? block_sum_squares(v) : 0.0);
        const float scale = 1.0f / sqrtf((float)(tot / K) + eps);
        if (row == warp) mark(timeline, pid, 5);
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            v[i] = __fmul_rn(__fmul_rn(v[i], scale), wv[i]);
            am = fmaxf(am, fabsf(v[i]));
        }
        if (has) {
            if (normed_out) {
                float4* o4 = reinterpret_cast<float4*>(normed_out + (size_t)row * K + 32 * lane);
#pragma unroll
                for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
            const float d = am / 127.f;
            const float id = am != 0.0f ? 127.f / am : 0.0f;
            uint32_t word[8];  // codes 4 w .. 4 w + 3 of the block
#pragma unroll
            for (int wd = 0; wd < 8; ++wd) {
                uint32_t b[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) b[j] = q8_code_bits(__fmul_rn(v[4 * wd + j], id));
                word[wd] = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
            }
            const float dq = __half2float(__float2half_rn(d));
            // Words stored in an order rotated by the lane (spreads the warp's
            // stores over the banks): rotate the array by lane & 7 in three
            // conditional steps, then store rot[s8] as word (s8 + lane) & 7.
#pragma unroll
            for (int k = 1; k < 8; k <<= 1) {
                if (lane & k) {
                    uint32_t t[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) t[i] = word[(i + k) & 7];
#pragma unroll
                    for (int i = 0; i < 8; ++i) word[i] = t[i];
                }
            }
#pragma unroll
            for (int s8 = 0; s8 < 8; ++s8) {
                const int wd = (s8 + lane) & 7;
                const uint32_t val = word[s8];
                if constexpr (kUmma) {
                    const int e = 32 * lane + 4 * wd, kk = e % 64;
                    *reinterpret_cast<uint32_t*>(act_q + (e / 64) * 1024 + ((row / 8) * 4 + kk / 16) * 128 + (row % 8) * 16 +
                                                 kk % 16) = val;
                } else {
                    *reinterpret_cast<uint32_t*>(act_q + (size_t)lane * 512 + frag_offset(row, 4 * wd)) = val;
                }
            }
            if constexpr (kUmma)
                act_d[row * NB + lane] = dq;
            else
                act_d[lane * 16 + row] = dq;
        }
        if (row == warp) mark(timeline, pid, 6);
    }
    consumer_sync();
}

// Slice sl (blocks 8 sl .. 8 sl + 7) of the activation fragments [K/32][512]
// and scales [K/32][16] from global into the same places in shared memory,
// by one warp (8 x 16 bytes of fragments and 16 bytes of scales per lane).
__device__ __forceinline__ void load_act_slice(const uint8_t* gq, const float* gd, int sl, uint8_t* act_q, float* act_d) {
    const int lane = threadIdx.x & 31;
    const uint4* src = reinterpret_cast<const uint4*>(gq + (size_t)sl * 8 * 512);
    uint4* dst = reinterpret_cast<uint4*>(act_q + (size_t)sl * 8 * 512);
    uint4 r[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) r[u] = __ldcg(src + u * 32 + lane);
    const float4 dv = __ldcg(reinterpret_cast<const float4*>(gd + (size_t)sl * 8 * 16) + lane);
#pragma unroll
    for (int u = 0; u < 8; ++u) dst[u * 32 + lane] = r[u];
    reinterpret_cast<float4*>(act_d + (size_t)sl * 8 * 16)[lane] = dv;
    __syncwarp();
}

// One 256-K slice of one row group from shared memory: the slice partial of
// the 16 x 8 outputs this lane holds (one fmaf per block, in block order).
// kLow: the step has at most 8 rows, so the outputs of rows 8..15 (the .z/.w
// components) are not formed.
template <bool kLow>
__device__ __forceinline__ float4 slice_partial_regs(const uint4 (&wvs)[4], const uint2 (&svs)[4], const uint4* s_act,
                                                     const float* s_d, int kt0) {
    const int lane = threadIdx.x & 31, g = lane >> 2;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const uint4 wv = wvs[u];
        const uint2 sv = svs[u];
        const int kt = kt0 + u;
        int c0[4], c1[4];
        mma_s8(c0, s_act[(2 * kt) * 32 + lane], wv.x, wv.y);
        mma_s8(c1, s_act[(2 * kt + 1) * 32 + lane], wv.z, wv.w);
        const float x0g = s_d[(2 * kt) * 16 + g], x1g = s_d[(2 * kt + 1) * 16 + g];
        const float w00 = h2f_lo(sv.x), w01 = h2f_hi(sv.x), w10 = h2f_lo(sv.y), w11 = h2f_hi(sv.y);
        acc[0] = fmaf(small_int_to_float(c0[0]), w00 * x0g, acc[0]);
        acc[1] = fmaf(small_int_to_float(c0[1]), w01 * x0g, acc[1]);
        if (!kLow) {
            const float x0h = s_d[(2 * kt) * 16 + g + 8];
            acc[2] = fmaf(small_int_to_float(c0[2]), w00 * x0h, acc[2]);
            acc[3] = fmaf(small_int_to_float(c0[3]), w01 * x0h, acc[3]);
        }
        acc[0] = fmaf(small_int_to_float(c1[0]), w10 * x1g, acc[0]);
        acc[1] = fmaf(small_int_to_float(c1[1]), w11 * x1g, acc[1]);
        if (!kLow) {
            const float x1h = s_d[(2 * kt + 1) * 16 + g + 8];
            acc[2] = fmaf(small_int_to_float(c1[2]), w10 * x1h, acc[2]);
            acc[3] = fmaf(small_int_to_float(c1[3]), w11 * x1h, acc[3]);
        }
    }
    return make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// The same from shared memory (the slice's 4 tiles in a ring slot).
template <bool kLow>
__device__ __forceinline__ float4 slice_partial(const uint8_t* slice, const uint4* s_act, const float* s_d, int kt0) {
    const int lane = threadIdx.x & 31, t = lane & 3;
    uint4 wv[4];
    uint2 sv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        wv[u] = *reinterpret_cast<const uint4*>(slice + u * kTileBytes + lane * 16);
        sv[u] = *reinterpret_cast<const uint2*>(slice + u * kTileBytes + 512 + t * 8);
    }
    return slice_partial_regs<kLow>(wv, sv, s_act, s_d, kt0);
}

// One LM-head item (a row group's KT tiles, all in one ring slot): the lane's
// tile fragments are read into registers first and the slot is released
// before the arithmetic, so the producer refills it while this warp computes.
// Slices are added in order (0 + slice 0 + slice 1 + ...), as in item_rows.
template <int KT, bool kLow>
__device__ __forceinline__ float4 item_staged(const uint8_t* slot, uint64_t* empty_bar, const uint4* s_act, const float* s_d) {
    const int lane = threadIdx.x & 31, t = lane & 3;
    uint4 wv[KT];
    uint2 sv[KT];
#pragma unroll
    for (int u = 0; u < KT; ++u) {
        wv[u] = *reinterpret_cast<const uint4*>(slot + u * kTileBytes + lane * 16);
        sv[u] = *reinterpret_cast<const uint2*>(slot + u * kTileBytes + 512 + t * 8);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar);
    float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s4 = 0; s4 < KT / 4; ++s4) {
        const uint4 w4[4] = {wv[4 * s4], wv[4 * s4 + 1], wv[4 * s4 + 2], wv[4 * s4 + 3]};
        const uint2 v4[4] = {sv[4 * s4], sv[4 * s4 + 1], sv[4 * s4 + 2], sv[4 * s4 + 3]};
        const float4 p = slice_partial_regs<kLow>(w4, v4, s_act, s_d, 4 * s4);
        y.x = y.x + p.x; y.y = y.y + p.y; y.z = y.z + p.z; y.w = y.w + p.w;
    }
    return y;
}

// Outputs of row group `rg_local` (0 or 1 for a gate/up pair) of the item whose
// slots start at sequence number q0: 0 + slice 0 + slice 1 + ... in order.
// Waits for and releases the item's ring slots (all of them when `release`).
template <bool kLow>
__device__ __forceinline__ bool item_rows(const uint8_t* ring, uint64_t* full, uint64_t* empty, long long q0, int kt_n, int rg_local,
                          const uint4* s_act, const float* s_d, const int* abort_flag, float4* out) {
    const int S = kt_n / 4;
    float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < S; ++s) {
        const int off = (rg_local * kt_n + s * 4) * kTileBytes;
        const long long q = q0 + off / kSlotBytes;
        if ((off % kSlotBytes) == 0 || s == 0)
            if (!slot_wait(full, q, abort_flag)) return false;
        const float4 p = slice_partial<kLow>(ring + (size_t)(q % kRingSlots) * kSlotBytes + off % kSlotBytes, s_act, s_d, s * 4);
        y.x = y.x + p.x; y.y = y.y + p.y; y.z = y.z + p.z; y.w = y.w + p.w;
    }
    *out = y;
    return true;
}

// A weight phase of this CTA split into (item, row group, 256-K slice) units
// over the 8 consumer warps; each unit's partial goes to shared memory, then
// `epi(j, part)` runs once per item (item j's units start at part + j*U*32,
// row group r's slice s at (r*S + s)*32) and adds the slices in order.  The
// phase's ring slots are all released after the units (at most 8 per CTA).
// `pre(sl)` runs in the unit's warp before slice sl is used (it may wait for
// that slice's activations and bring them into shared memory); false aborts.
struct NoPrologue {
    __device__ bool operator()(int) const { return true; }
};

template <bool kLow, typename Epi, typename Pre = NoPrologue>
__device__ __forceinline__ bool weight_phase(const PhaseInfo& pi, int rgs, int kt_n, const uint8_t* ring,
                                             uint64_t* full, uint64_t* empty, const uint4* s_act, const float* s_d,
                                             float4* s_part, const int* abort_flag, Epi epi, Pre pre = Pre()) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = kt_n / 4, U = rgs * S;
    const int n_units = pi.count * U;
    bool ok = true;
    for (int u = warp; u < n_units; u += kConsumerWarps) {
        const int j = u / U, r = (u % U) / S, sl = u % S;
        const int off = (r * kt_n + sl * 4) * kTileBytes;
        const long long q = pi.slot0 + (long long)j * pi.slots + off / kSlotBytes;
        if (!pre(sl)) { ok = false; break; }
        if (!slot_wait(full, q, abort_flag)) { ok = false; break; }
        s_part[u * 32 + lane] = slice_partial<kLow>(ring + (size_t)(q % kRingSlots) * kSlotBytes + off % kSlotBytes, s_act, s_d, sl * 4);
    }
    consumer_sync();
    const int n_slots = pi.count * pi.slots;
    for (int k = threadIdx.x; k < n_slots; k += kConsumers) mbar_arrive(&empty[(pi.slot0 + k) % kRingSlots]);
    for (int j = warp; j < pi.count; j += kConsumerWarps) epi(j, s_part + (size_t)j * U * 32);
    return ok;
}

__device__ __forceinline__ float4 sum_slices(const float4* part, int S) {
    const int lane = threadIdx.x & 31;
    float4 y = make_float4(0.f, 0.f, 0.f, 0.f);  // 0 + slice 0 + slice 1 + ... as on the CPU
    for (int sl = 0; sl < S; ++sl) {
        const float4 p = part[sl * 32 + lane];
        y.x = y.x + p.x; y.y = y.y + p.y; y.z = y.z + p.z; y.w = y.w + p.w;
    }
    return y;
}

// Phase C for one (row t of the step, stream si, q head qh, 32-dim block k) by one warp, lane =
// dim 32 k + lane: merge of the chunk partials in chunk order (M = max m_c;
// w_c = exp(m_c - M); L = sum w_c l_c; o = sum w_c o_c / L, each sum one
// sequential fmaf chain), then that q8_0 block of the context row.  All of a
// batch's loads (32 chunks) are issued together, the next batch's while the
// current one is summed.
// Float <-> unsigned with the same order (0 is below every encoded value),
// for a running maximum by atomicMax.
__device__ __forceinline__ unsigned ordered_bits(float f) {
    const unsigned b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float from_ordered_bits(unsigned u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

// Wait (lane 0 polls with relaxed loads and ends with one acquire load, the
// warp follows) until the counter reaches `target`: its producers release-add
// after their results are stored, so the results are visible to the warp
// afterwards.  Bounded like a grid
// barrier; false on abort or timeout.
__device__ __forceinline__ bool wait_count(const MegaArgs& a, const unsigned* cnt, unsigned target) {
    int give_up = 0;
    if ((threadIdx.x & 31) == 0) {
        const unsigned long long t0 = global_ns();
        for (unsigned it = 0;; ++it) {
            unsigned v;
            asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
            if (v >= target) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
                break;
            }
            if ((it & 15) == 15) {
                if (*reinterpret_cast<const volatile int*>(a.abort_flag)) { give_up = 1; break; }
                if (global_ns() - t0 > a.wait_ns) {
                    atomicExch(a.abort_flag, 1);
                    report_timeout(a);
                    give_up = 1;
                    break;
                }
            }
        }
    }
    give_up = __shfl_sync(0xffffffffu, give_up, 0);
    __syncwarp();
    return give_up == 0;
}

__device__ __noinline__ bool combine_task(const MegaArgs& a, int l, int t, int si, int qh, int k, int n_chunks) {
    const int lane = threadIdx.x & 31;
    const int G = a.d.n_heads / a.d.n_kv, h = qh / G, qi = t * G + qh % G;
    // The head's chunk items are counted as they finish (release-add after
    // their partials).
    if (!wait_count(a, a.head_done + ((size_t)l * kMaxStreams + si) * a.d.n_kv + h, (unsigned)n_chunks)) return false;
    const size_t base = (size_t)h * a.max_chunks * (kTMax * 4) + qi;  // (h, chunk 0, qi)
    const float* po = a.part_o + base * kHeadDim + 32 * k + lane;
    const float2* pml = a.part_ml + base;
    constexpr size_t kStrideO = (size_t)kTMax * 4 * kHeadDim;         // one chunk further
    constexpr size_t kStrideM = (size_t)kTMax * 4;
    // M = the largest chunk maximum: kept by the attention items (atomicMax).
    const float M = from_ordered_bits(__ldcg(a.m_max + ((size_t)l * a.d.n_kv + h) * (kTMax * 4) + qi));
    // Chunks in batches of 32: each lane holds the batch's 32 values of its
    // dim and the (m, l) of chunk c0 + lane.  Two batches are requested ahead
    // of the one being summed (the sums are one sequential chain over the
    // chunks).  Chunks past the end read as weight 0 (m = -inf, l = 0, o = 0),
    // which adds nothing.
    auto load_batch = [&](int c0, float (&o)[32], float2& ml) {
#pragma unroll
        for (int u = 0; u < 32; ++u) o[u] = c0 + u < n_chunks ? __ldcg(po + (size_t)(c0 + u) * kStrideO) : 0.f;
        ml = c0 + lane < n_chunks ? __ldcg(pml + (size_t)(c0 + lane) * kStrideM) : make_float2(-INFINITY, 0.f);
    };
    float ov[32], o1[32];
    float2 ml0v, ml1v;
    load_batch(0, ov, ml0v);
    load_batch(32, o1, ml1v);
    float Ls = 0.f, acc = 0.f;
    for (int c0 = 0; c0 < n_chunks; c0 += 32) {
        float o2[32];
        float2 ml2v;
        load_batch(c0 + 64, o2, ml2v);
        const float wl = ml0v.x == -INFINITY ? 0.f : exact_expf(ml0v.x - M);
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            const float lc = __shfl_sync(0xffffffffu, ml0v.y, u);
            const float wgt = __shfl_sync(0xffffffffu, wl, u);
            Ls = fmaf(wgt, lc, Ls);
            acc = fmaf(wgt, ov[u], acc);
        }
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            ov[u] = o1[u];
            o1[u] = o2[u];
        }
        ml0v = ml1v;
        ml1v = ml2v;
    }
    const float o = acc / Ls;
    float am[1] = {warp_absmax(o)}, dq[1], iq[1];
    q8_scales<1>(am, dq, iq);
    const int blk = qh * 4 + k;
    a.act_q[(size_t)blk * 512 + frag_offset(t, lane)] = (uint8_t)q8_code_bits(__fmul_rn(o, iq[0]));
    if (lane == 0) a.act_d[blk * 16 + t] = __half2float(__float2half_rn(dq[0]));
    // The block is stored (every lane's byte, lane 0's scale): count it for
    // the O projection's 256-K slice of this pair of q heads.
    __syncwarp();
    if (lane == 0) {
        unsigned* cnt = a.pair_done + (size_t)l * (a.d.n_heads / 2) + qh / 2;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
    }
    return true;
}

// Per-head RMSNorm and NEOX RoPE of one q or k head row by one warp.  Lane
// `lane` holds elements lane + 32 q of the row (q = 0..3).  Sum of squares
// (the per-head tree shared with k_qk_norm_rope_store and the CPU
// restatement): each lane adds its four squares in q order in double, then
// one xor butterfly over the lanes.  The RoPE pairs (e, e + 64) are
// (lane, lane + 64) and (lane + 32, lane + 96); `rope` = the row's [64][cos, sin].
__device__ __forceinline__ double head_square_part(const float (&x)[4]) {
    double p = 0.0;
#pragma unroll
    for (int q = 0; q < 4; ++q) p += (double)(x[q] * x[q]);
    return p;
}

// The row's normalised, rotated elements from its butterfly total `tot`.
__device__ __forceinline__ void norm_rope_apply(const float (&x)[4], double tot, const float* __restrict__ wn, float eps,
                                                const float* rope, float (&o)[4]) {
    const int lane = threadIdx.x & 31;
    const float mean = (float)(tot * (1.0 / kHeadDim));  // exact: 128 is a power of two
    const float scale = 1.0f / sqrtf(mean + eps);
    float y[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) y[q] = __fmul_rn(__fmul_rn(x[q], scale), wn[32 * q + lane]);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int e = 32 * q + lane;
        const float cs = rope[e * 2], sn = rope[e * 2 + 1];
        o[q] = __fsub_rn(__fmul_rn(y[q], cs), __fmul_rn(y[q + 2], sn));
        o[q + 2] = __fadd_rn(__fmul_rn(y[q], sn), __fmul_rn(y[q + 2], cs));
    }
}

__device__ __forceinline__ void norm_rope_row(const float (&x)[4], const float* __restrict__ wn, float eps,
                                              const float* rope, float (&o)[4]) {
    norm_rope_apply(x, warp_sum_d(head_square_part(x)), wn, eps, rope, o);
}

// Attention of one (64-position chunk, kv head h) item (phase B) by `wpi`
// warps (the item's warp wl = 0..wpi-1, named barrier `bar` over them), its K
// and V rows already in ring slots q0.. (streamed by the producer).  The
// item's warp wl owns the query rows wl, wl + wpi, ... of the head's G query
// heads (row = t * G + j): lane `lane` holds positions lane and lane + 32, so
// each score is two sequential fmaf chains (even and odd dims, one __ffma2_rn
// per dim pair) added, the chunk softmax
// is the warp butterfly (max, then e = exp(s - m) and the pair/butterfly
// sum), and each P.V output (lane's dims 4 lane .. 4 lane + 3) is one
// sequential fmaf chain over the chunk's positions; the order of
// k_attn_chunk and the CPU restatement.
// Scratch of one warp group's item: query rows [rows][128] f32 + doubled exp
// weights [rows][64] float2, 1 KB per row.
constexpr int kAttnRowBytes = kHeadDim * 4 + kPage * 8;

__device__ __forceinline__ void item_sync(int bar, int nthr) {
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthr) : "memory");
}

// Scores, softmax and P.V of this warp's R rows (R a power of two; rows at or
// past `nq` are computed on spare query rows and not stored).
template <bool F16, int R>
__device__ __forceinline__ void attn_rows(const MegaArgs& a, const uint8_t* ring, long long q0, const float* sq,
                                          float2* sw, int wl, int wpi, int nq, int G, int p0, int n_pos, int before,
                                          size_t ml0, unsigned* mrow) {
    using KS = KvSlots<F16>;
    const int lane = threadIdx.x & 31;
    const float attn_scale = 1.0f / sqrtf((float)kHeadDim);
    // acc[rr][u] = {even-dim chain, odd-dim chain} of row rr, position lane + 32 u.
    float2 acc[R][2];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) acc[rr][0] = acc[rr][1] = make_float2(0.f, 0.f);
    {
        // K rows of positions lane and lane + 32 (row lane % rows-per-slot of
        // their slots; rows per slot divide 32, so both rows share the swizzle).
        const int s0 = int(q0 % kRingSlots), pr = lane % KS::kRowsPerSlot, xs = lane & 7;
        const uint8_t* ka_row = kv_slot_base(const_cast<uint8_t*>(ring), (s0 + lane / KS::kRowsPerSlot) % kRingSlots) + pr * 128;
        const uint8_t* kb_row =
            kv_slot_base(const_cast<uint8_t*>(ring), (s0 + (lane + 32) / KS::kRowsPerSlot) % kRingSlots) + pr * 128;
        constexpr int EB = F16 ? 8 : 4;  // dims per 16-byte read
#pragma unroll 2
        for (int eb = 0; eb < kHeadDim / EB; ++eb) {
            float2 ka[EB / 2], kb[EB / 2];
            const int off = (eb >> 3) * KS::kBoxBytes + (((eb & 7) ^ xs) << 4);
            const uint4 ua = *reinterpret_cast<const uint4*>(ka_row + off);
            const uint4 ub = *reinterpret_cast<const uint4*>(kb_row + off);
            if constexpr (F16) {
                const __half2* ha = reinterpret_cast<const __half2*>(&ua);
                const __half2* hb = reinterpret_cast<const __half2*>(&ub);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    ka[i] = __half22float2(ha[i]);
                    kb[i] = __half22float2(hb[i]);
                }
            } else {
                ka[0] = make_float2(__uint_as_float(ua.x), __uint_as_float(ua.y));
                ka[1] = make_float2(__uint_as_float(ua.z), __uint_as_float(ua.w));
                kb[0] = make_float2(__uint_as_float(ub.x), __uint_as_float(ub.y));
                kb[1] = make_float2(__uint_as_float(ub.z), __uint_as_float(ub.w));
            }
#pragma unroll
            for (int rr = 0; rr < R; ++rr) {
                const float* qrow = sq + (wl + wpi * rr) * kHeadDim + eb * EB;
                float2 qv[EB / 2];
#pragma unroll
                for (int i = 0; i < EB; i += 4) {
                    const float4 q4 = *reinterpret_cast<const float4*>(qrow + i);
                    qv[i / 2] = make_float2(q4.x, q4.y);
                    qv[i / 2 + 1] = make_float2(q4.z, q4.w);
                }
#pragma unroll
                for (int i = 0; i < EB / 2; ++i) {
                    acc[rr][0] = __ffma2_rn(qv[i], ka[i], acc[rr][0]);
                    acc[rr][1] = __ffma2_rn(qv[i], kb[i], acc[rr][1]);
                }
            }
        }
    }
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
        const int r = wl + wpi * rr, t = r / G;
        const bool ok0 = lane < n_pos && p0 + lane < before + t + 1;
        const bool ok1 = lane + 32 < n_pos && p0 + lane + 32 < before + t + 1;
        const float s0 = ok0 ? __fmul_rn(__fadd_rn(acc[rr][0].x, acc[rr][0].y), attn_scale) : -INFINITY;
        const float s1 = ok1 ? __fmul_rn(__fadd_rn(acc[rr][1].x, acc[rr][1].y), attn_scale) : -INFINITY;
        const float m = warp_max(fmaxf(s0, s1));
        const float x0 = exact_expf(s0 - m), x1 = exact_expf(s1 - m);
        const float e0 = s0 == -INFINITY ? 0.f : x0;
        const float e1 = s1 == -INFINITY ? 0.f : x1;
        const float lsum = warp_sum(e0 + e1);
        sw[(wl + wpi * rr) * kPage + lane] = make_float2(e0, e0);
        sw[(wl + wpi * rr) * kPage + lane + 32] = make_float2(e1, e1);
        if (lane == 0 && r < nq) {
            a.part_ml[ml0 + r] = make_float2(m, lsum);
            atomicMax(mrow + r, ordered_bits(m));  // the merge's M, without reading every chunk's m
        }
    }
    __syncwarp();
    // P.V: o[rr] = {dims 4 lane, 4 lane + 1}, {4 lane + 2, 4 lane + 3}; each
    // component one fmaf chain over the positions (two per __ffma2_rn).
    float2 o[R][2];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) o[rr][0] = o[rr][1] = make_float2(0.f, 0.f);
    auto load_v = [&](const uint8_t* row, float2& v01, float2& v23) {
        if constexpr (F16) {
            const uint2 hv = *reinterpret_cast<const uint2*>(row);
            v01 = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
            v23 = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
        } else {
            const float4 f = *reinterpret_cast<const float4*>(row);
            v01 = make_float2(f.x, f.y);
            v23 = make_float2(f.z, f.w);
        }
    };
    // Lane's 8 (fp16) or 16 (f32) bytes of V row p of a slot: chunk cv of
    // the row, at the swizzled position.
    const int cv = F16 ? lane >> 1 : lane, cc = cv & 7;
    const int v_lane = (cv >> 3) * KS::kBoxBytes + (F16 ? (lane & 1) * 8 : 0);
    const int s0v = int((q0 + KS::kSlotsPerHalf) % kRingSlots);
    for (int sidx = 0; sidx < KS::kSlotsPerHalf; ++sidx) {
        const int pb = sidx * KS::kRowsPerSlot;
        const int np = min(KS::kRowsPerSlot, n_pos - pb);
        if constexpr (F16) {
            if (np == KS::kRowsPerSlot) {
                // A full slot in blocks of 8 rows: row 8 m + k of the lane's
                // chunk cv sits at the lane's offset XOR k * 16, + (8 m + k) * 128.
                const uint32_t vA = kv_slot_off((s0v + sidx) % kRingSlots) + v_lane + ((uint32_t)cc << 4);
#pragma unroll 1
                for (int m = 0; m < KS::kRowsPerSlot / 8; ++m) {
                    const uint32_t vm = vA + m * 1024;
                    float2 v[8][2];
#pragma unroll
                    for (int k = 0; k < 8; ++k) load_v(ring + ((vm ^ (k << 4)) + k * 128), v[k][0], v[k][1]);
#pragma unroll
                    for (int rr = 0; rr < R; ++rr) {
                        const float4* w4 = reinterpret_cast<const float4*>(sw + (wl + wpi * rr) * kPage + pb + 8 * m);
#pragma unroll
                        for (int k2 = 0; k2 < 4; ++k2) {
                            const float4 w = w4[k2];
                            const float2 wa = make_float2(w.x, w.y), wb = make_float2(w.z, w.w);
                            o[rr][0] = __ffma2_rn(wa, v[2 * k2][0], o[rr][0]);
                            o[rr][1] = __ffma2_rn(wa, v[2 * k2][1], o[rr][1]);
                            o[rr][0] = __ffma2_rn(wb, v[2 * k2 + 1][0], o[rr][0]);
                            o[rr][1] = __ffma2_rn(wb, v[2 * k2 + 1][1], o[rr][1]);
                        }
                    }
                }
                continue;
            }
        }
        const uint8_t* vb = kv_slot_base(const_cast<uint8_t*>(ring), (s0v + sidx) % kRingSlots) + v_lane;
        auto v_at = [&](int p) -> const uint8_t* { return vb + p * 128 + ((cc ^ (p & 7)) << 4); };
        int pr = 0;
#pragma unroll 1
        for (; pr + 4 <= np; pr += 4) {
            float2 v[4][2];
#pragma unroll
            for (int i = 0; i < 4; ++i) load_v(v_at(pr + i), v[i][0], v[i][1]);
#pragma unroll
            for (int rr = 0; rr < R; ++rr) {
                const float4* wr = reinterpret_cast<const float4*>(sw + (wl + wpi * rr) * kPage + pb + pr);
                const float4 w01 = wr[0], w23 = wr[1];
                const float2 w[4] = {make_float2(w01.x, w01.y), make_float2(w01.z, w01.w),
                                     make_float2(w23.x, w23.y), make_float2(w23.z, w23.w)};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    o[rr][0] = __ffma2_rn(w[i], v[i][0], o[rr][0]);
                    o[rr][1] = __ffma2_rn(w[i], v[i][1], o[rr][1]);
                }
            }
        }
#pragma unroll 1
        for (; pr < np; ++pr) {
            float2 v01, v23;
            load_v(v_at(pr), v01, v23);
#pragma unroll
            for (int rr = 0; rr < R; ++rr) {
                const float2 w = sw[(wl + wpi * rr) * kPage + pb + pr];
                o[rr][0] = __ffma2_rn(w, v01, o[rr][0]);
                o[rr][1] = __ffma2_rn(w, v23, o[rr][1]);
            }
        }
    }
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
        const int r = wl + wpi * rr;
        if (r < nq)
            reinterpret_cast<float4*>(a.part_o + (ml0 + r) * kHeadDim)[lane] =
                make_float4(o[rr][0].x, o[rr][0].y, o[rr][1].x, o[rr][1].y);
    }
}

// The item with RP >= this warp's query rows (a power of two).  Returns false
// when a slot wait gave up.
// The item's stream has T rows from step row row0 on, after `before` cached
// positions, in cache `kv`.  Its partials are stored under step rows (row0 + t) * G + jh.
template <bool F16, int RP>
__device__ __noinline__ bool attn_body(const MegaArgs& a, size_t scratch_off, int rows_cap, int l, int chunk, int h,
                                       long long q0, int T, int before, int row0, const KvCache& kv, bool q_cached, int wl,
                                       int wpi, int bar, int mark_pid, int mark_k) {
    using KS = KvSlots<F16>;
    uint8_t* ring = s_ring();
    uint64_t* full = s_full();
    const float* rope = s_rope();
    const float* qk_norm = g_qk_norm;
    float* sq = reinterpret_cast<float*>(s_region() + scratch_off);
    float2* sw = reinterpret_cast<float2*>(s_region() + scratch_off + (size_t)rows_cap * kHeadDim * 4);
    const int nh = a.d.n_heads, nkv = a.d.n_kv, G = nh / nkv;
    const int lane = threadIdx.x & 31, nthr = wpi * 32;
    const int kv_len = before + T, NQ = T * G;
    const int p0 = chunk * kPage, n_pos = min(kPage, kv_len - p0);
    const int ldq = (nh + 2 * nkv) * kHeadDim;
    const int R = wl < NQ ? (NQ - 1 - wl) / wpi + 1 : 0;  // query rows of this warp
    // This warp's query rows: RMSNorm + RoPE of the raw projections (the
    // same rows in every chunk item of the head; cheaper than a phase), unless
    // the group's previous item had the same stream and head (q_cached: each
    // warp's rows are still in sq).  All rows' loads are issued first.
    if (!q_cached) {
        float x[RP][4];
#pragma unroll
        for (int rr = 0; rr < RP; ++rr) {
            const int r = wl + wpi * rr, t = row0 + r / G, jh = r % G;
            const float* src = a.qkv + (size_t)t * ldq + (size_t)(h * G + jh) * kHeadDim;
#pragma unroll
            for (int q = 0; q < 4; ++q) x[rr][q] = rr < R ? __ldcg(src + 32 * q + lane) : 0.f;
        }
        // The rows' butterflies interleaved (independent chains).
        double tot[RP];
#pragma unroll
        for (int rr = 0; rr < RP; ++rr) tot[rr] = head_square_part(x[rr]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int rr = 0; rr < RP; ++rr) tot[rr] += __shfl_xor_sync(0xffffffffu, tot[rr], o);
#pragma unroll
        for (int rr = 0; rr < RP; ++rr) {
            if (rr < R) {
                const int r = wl + wpi * rr, t = row0 + r / G;
                float o[4];
                norm_rope_apply(x[rr], tot[rr], qk_norm, a.d.eps, rope + t * 64 * 2, o);
#pragma unroll
                for (int q = 0; q < 4; ++q) sq[r * kHeadDim + 32 * q + lane] = o[q];
            }
        }
    }
    const bool ok = slots_wait(full, q0, 2 * KS::kSlotsPerHalf, a.abort_flag);
    if (wl == 0) mark(a.timeline, mark_pid, mark_k);
    // The step's own positions in this chunk: k (RMSNorm + RoPE) and v rows
    // from the raw projections into the ring rows and the KV cache (the
    // producer's copy of those rows predates them).  One row per warp.
    {
        const int r_lo = max(before - p0, 0), nr = max(n_pos - r_lo, 0);
        for (int i = wl; i < 2 * nr; i += wpi) {
            const int which = i / nr, r = r_lo + i % nr, t = row0 + p0 + r - before;
            const float* src = a.qkv + (size_t)t * ldq + (size_t)(nh + which * nkv + h) * kHeadDim;
            float x[4], o[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) x[q] = __ldcg(src + 32 * q + lane);
            if (which == 0) {
                norm_rope_row(x, qk_norm + kHeadDim, a.d.eps, rope + t * 64 * 2, o);
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) o[q] = x[q];
            }
            const long long off = kv_offset(kv, nkv, l, which, h, p0 + r);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                kv_store(kv, off + 32 * q + lane, o[q]);
                const int e = 32 * q + lane;  // element of the row
                if constexpr (F16)
                    *reinterpret_cast<__half*>(kv_chunk<true>(ring, q0, which, r, e >> 3) + (e & 7) * 2) =
                        __float2half_rn(o[q]);
                else
                    *reinterpret_cast<float*>(kv_chunk<false>(ring, q0, which, r, e >> 2) + (e & 3) * 4) = o[q];
            }
        }
        // Order these generic-proxy stores before the producer's next bulk copies into the slots.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    item_sync(bar, nthr);
    if (wl == 0) mark(a.timeline, mark_pid, mark_k + 1);
    const size_t ml0 = ((size_t)h * a.max_chunks + chunk) * (kTMax * 4) + (size_t)row0 * G;
    unsigned* mrow = a.m_max + ((size_t)l * nkv + h) * (kTMax * 4) + (size_t)row0 * G;
    if (R > 0) attn_rows<F16, RP>(a, ring, q0, sq, sw, wl, wpi, NQ, G, p0, n_pos, before, ml0, mrow);
    if (wl == 0) mark(a.timeline, mark_pid, mark_k + 2);
    return ok;
}

template <bool F16>
__device__ __forceinline__ bool attn_item(const MegaArgs& a, size_t scratch_off, int rows_cap, int l, int chunk, int h,
                                          long long q0, int T, int before, int row0, const KvCache& kv, bool q_cached,
                                          int wl, int wpi, int bar, int mark_pid, int mark_k) {
    const int NQ = T * (a.d.n_heads / a.d.n_kv);
    const int R = wl < NQ ? (NQ - 1 - wl) / wpi + 1 : 0;
#define MTB_ATTN_BODY(RP) \
    attn_body<F16, RP>(a, scratch_off, rows_cap, l, chunk, h, q0, T, before, row0, kv, q_cached, wl, wpi, bar, mark_pid, \
                       mark_k)
    if (R <= 1) return MTB_ATTN_BODY(1);
    if (R == 2) return MTB_ATTN_BODY(2);
    return MTB_ATTN_BODY(4);  // R <= 4: see KCtx::attn_wpi
#undef MTB_ATTN_BODY
}

// ------------------------------------------------------------------ the kernel

// Per-CTA context, built once in shared memory by thread 0: the phase
// functions below read their sizes and pointers from here instead of keeping
// them live in registers across the whole step.
struct KCtx {
    MegaArgs a;
    Schedule sch;
    int T;             // rows of the step, all streams
    // Per stream: rows, first step row, cached positions, attention chunks.
    int s_T[kMaxStreams], s_row0[kMaxStreams], s_before[kMaxStreams], s_chunks[kMaxStreams];
    int row_stream[kTMax];  // stream of each step row
    // Warps per attention item: 2 when every stream has <= 4 query rows per kv
    // head (fp16 KV), 8 above 16, else 4 -- so a warp never holds more than 4
    // query rows (more would raise the whole kernel's register pressure).
    int attn_wpi;
};

__shared__ KCtx g_ctx;

// Grid barrier at the end of a phase (barrier *nb, whose arrivals complete at
// *target); false when the step is being aborted.
__device__ __noinline__ bool end_phase(unsigned* target, int* nb) {
    const KCtx& c = g_ctx;
    *target += gridDim.x;
    return grid_barrier(c.a, *target, (*nb)++, &g_flag);
}

// RoPE angles of the step's positions (theta advanced by repeated float
// products, src/qwen3.cpp:109-118), shared by every layer; and the embedding
// rows of the step's tokens (q8_0 dequant from the token_embd tiles).
__device__ __noinline__ void phase_embed() {
    const KCtx& c = g_ctx;
    const MegaArgs& a = c.a;
    const int tid = threadIdx.x, H = a.d.hidden;
    for (int i = tid; i < kTMax * 64; i += kConsumers) {
        const int t = i / 64, k = i % 64;
        const int si = t < c.T ? c.row_stream[t] : 0;
        float theta = (float)(t < c.T ? c.s_before[si] + t - c.s_row0[si] : t);
        for (int j = 0; j < k; ++j) theta = __fmul_rn(theta, a.theta_scale);
        float sn, cs;
        exact_sincosf(theta, &sn, &cs);
        s_rope()[i * 2] = cs;
        s_rope()[i * 2 + 1] = sn;
    }
    const int kt_n = H / kTileK;
    for (int i = blockIdx.x * kConsumers + tid; i < kTMax * H; i += gridDim.x * kConsumers) {
        const int row = i / H, col = i % H;
        float v = 0.f;
        if (row < c.T) {
            const int si = c.row_stream[row];
            StepState* st = a.st_state[si];
            int id = st->tokens[row - c.s_row0[si]];
            if (id < 0 || id >= a.d.vocab) { st->error = 1; id = 0; }
            const int rg = id / kTileRows, g = id % kTileRows;
            const int kt = col / kTileK, blk = (col % kTileK) / 32, cc = col % 32;
            const uint8_t* tile = a.embd + ((size_t)rg * kt_n + kt) * kTileBytes;
            const int t4 = (cc & 15) >> 2, part = cc >> 4;
            const int8_t q = (int8_t)tile[(g * 4 + t4) * 16 + blk * 8 + part * 4 + (cc & 3)];
            const unsigned short hb =
                *reinterpret_cast<const unsigned short*>(tile + 512 + ((g >> 1) * 4 + blk * 2 + (g & 1)) * 2);
            v = (float)q * __half2float(__ushort_as_half(hb));
        }
        a.x[i] = v;
    }
    consumer_sync();
}

// Epilogue helper: lane (g, t) holds rows g, g + 8 x columns 2t, 2t + 1 of a row group.
template <typename F>
__device__ __forceinline__ void for_outputs(const float4& y, int T, F f) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const float yy[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int row = g + (k >> 1) * 8;
        if (row < T) f(row, 2 * t + (k & 1), yy[k]);
    }
}

// A: RMSNorm + quantise (every CTA), QKV rows -> qkv.
template <int NK, bool kLow>
__device__ __noinline__ bool phase_qkv(int l, long long* cur, int pid, float4 wpre) {
    const KCtx& c = g_ctx;
    const MegaArgs& a = c.a;
    const LayerWeights& w = a.layers[l];
    constexpr int K = 256 * NK;
    uint8_t* act_q = s_region();
    float* act_d = reinterpret_cast<float*>(act_q + (size_t)(K / 32) * 512);
    // The layer's q/k norm weights for phase B, loaded here where the latency
    // hides behind this phase's work (B would otherwise chase the layer's
    // pointers and then the weights before its first item could start).
    const float qkn = threadIdx.x < 2 * kHeadDim
                          ? __ldg((threadIdx.x < kHeadDim ? w.q_norm : w.k_norm) + (threadIdx.x % kHeadDim))
                          : 0.f;
    norm_quant_smem<NK>(a.x, wpre, a.d.eps, c.T, a.timeline, pid);
    if (threadIdx.x < 2 * kHeadDim) g_qk_norm[threadIdx.x] = qkn;
    mark(a.timeline, pid, 0);
    const PhaseInfo pi = c.sch.take(W_QKV, &cur[0], &cur[1]);
    float4* s_part = reinterpret_cast<float4*>(act_d + (K / 32) * 16);
    const int ldq = (a.d.n_heads + 2 * a.d.n_kv) * kHeadDim, T = c.T;
    return weight_phase<kLow>(pi, 1, K / kTileK, s_ring(), s_full(), s_empty(), reinterpret_cast<const uint4*>(act_q), act_d,
                        s_part, a.abort_flag, [&](int j, const float4* part) {
                            const int item = pi.first + j * gridDim.x;
                            for_outputs(sum_slices(part, K / kTileK / 4), T, [&](int row, int col, float v) {
                                a.qkv[(size_t)row * ldq + item * kTileRows + col] = v;
                            });
                        });
}

// B: attention items of this CTA in stream order, by independent groups of
// wpi warps (named barrier 2 + group): group g takes the CTA's items g,
// g + groups, ... and, as soon as an item is done, releases its ring slots and
// counts it for its head's merge.  Four groups of two warps when every stream
// has at most 4 query rows per kv head (four fp16 items fill the ring), one of
// eight above 16 rows, else two groups of four.
__device__ __noinline__ bool phase_attn(int l, long long* cur, int pid) {
    const KCtx& c = g_ctx;
    const MegaArgs& a = c.a;
    const PhaseInfo pi = c.sch.take(W_ATTN, &cur[0], &cur[1]);
    const int nkv = a.d.n_kv, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpi = c.attn_wpi, n_groups = kConsumerWarps / wpi, g = warp / wpi, wl = warp % wpi;
    const int rows_cap = wpi == 2 ? 4 : 32;
    const size_t scratch_off = (size_t)g * rows_cap * kAttnRowBytes;
    bool ok = true;
    int prev = -1;     // stream * n_kv + head of the group's previous item
    unsigned done = 0;  // the group's finished items of that (stream, head), not yet counted
    // Count finished items for their head's merge (release: cumulative over
    // the group's partial stores, ordered by the group's named barrier).  Once
    // per run of items of one (stream, head), not per item: each release waits
    // for the group's stores to complete.
    auto count_done = [&]() {
        if (done && wl == 0 && lane == 0) {
            unsigned* cnt = a.head_done + ((size_t)l * kMaxStreams + prev / nkv) * nkv + prev % nkv;
            asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(cnt), "r"(done) : "memory");
        }
        done = 0;
    };
    for (int j = g; j < pi.count; j += n_groups) {
        int si, chunk, h;
        c.sch.attn_item_of(pi.first + j * gridDim.x, &si, &chunk, &h);
        const bool q_cached = prev == si * nkv + h;
        if (!q_cached) count_done();
        prev = si * nkv + h;
        const long long q0 = pi.slot0 + (long long)j * pi.slots;
        const int mp = j == 0 ? pid : -1, mk = 0;  // marks: slots ready, rows patched, softmax, done
        const bool good = c.sch.kv_f16
                              ? attn_item<true>(a, scratch_off, rows_cap, l, chunk, h, q0, c.s_T[si],
                                                c.s_before[si], c.s_row0[si], a.st_kv[si], q_cached, wl, wpi, 2 + g,
                                                mp, mk)
                              : attn_item<false>(a, scratch_off, rows_cap, l, chunk, h, q0, c.s_T[si],
                                                 c.s_before[si], c.s_row0[si], a.st_kv[si], q_cached, wl, wpi, 2 + g,
                                                 mp, mk);
        ok = ok && good;
        // The group is done with the slots and its partials are stored: free
        // the slots; the item is counted with the run it belongs to.
        item_sync(2 + g, wpi * 32);
        if (wl == 0 && lane < pi.slots) mbar_arrive(&s_empty()[(q0 + lane) % kRingSlots]);
        ++done;
        mark(a.timeline, mp, mk + 3);
    }
    count_done();
    // Every group is done with its scratch in the region before phase D
    // (after the merges, with no grid barrier between) loads into it.
    consumer_sync();
    return ok;
}

// C: chunk merge + quantise, one (row, q head, block) per warp, warps
// numbered across CTAs; no grid barrier before it: each task waits for its
// head's attention items only (they finish at different times).
__device__ __noinline__ bool phase_combine(int l) {
    const KCtx& c = g_ctx;
    const int nh = c.a.d.n_heads, warp = threadIdx.x >> 5;
    const int n_tasks = c.T * nh * 4;
    bool ok = true;
    for (int it = blockIdx.x + gridDim.x * warp; it < n_tasks && ok; it += gridDim.x * kConsumerWarps) {
        const int t = it / (nh * 4), si = c.row_stream[t];
        ok = combine_task(c.a, l, t, si, (it / 4) % nh, it % 4, c.s_chunks[si]);
    }
    return ok;
}

// D: O projection + residual.  F: down projection + residual.  The residual
// values of the warp's first item are read before the weight work, so the
// epilogue does not wait for them.
template <bool kLow>
__device__ __noinline__ bool phase_proj_resid(int l, long long* cur, int pid, bool down) {
    const KCtx& c = g_ctx;
    const MegaArgs& a = c.a;
    const int K = down ? a.d.ffn : a.d.n_heads * kHeadDim, H = a.d.hidden, T = c.T;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    // No grid barrier before this phase: each unit waits for its own 256-K
    // slice of the input (O: the merged context of one pair of q heads, 8 T
    // merge tasks; down: the SwiGLU of 8 gate/up blocks) and brings that slice
    // into shared memory.  This CTA's warps are past their own uses of the
    // region by then: the attention phase ends with a CTA barrier (the merges
    // use no shared memory), and the gate/up phase's last barrier follows its
    // last shared-memory read.
    const PhaseInfo pi = c.sch.take(down ? W_DOWN : W_O, &cur[0], &cur[1]);
    float xr[4] = {0.f, 0.f, 0.f, 0.f};
    if (warp < pi.count) {
        const int item = pi.first + warp * gridDim.x;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int row = g + (k >> 1) * 8;
            if (row < T) xr[k] = __ldcg(a.x + (size_t)row * H + item * kTileRows + 2 * t + (k & 1));
        }
    }
    uint8_t* act_q = s_region();
    float* act_d = reinterpret_cast<float*>(act_q + (size_t)(K / 32) * 512);
    const uint8_t* gq = down ? a.act2_q : a.act_q;
    const float* gd = down ? a.act2_d : a.act_d;
    const unsigned* counts = down ? a.slice_done + (size_t)l * (a.d.ffn / 256) : a.pair_done + (size_t)l * (a.d.n_heads / 2);
    const unsigned need = down ? 8u : 8u * (unsigned)T;
    mark(a.timeline, pid, 0);
    float4* s_part = reinterpret_cast<float4*>(act_d + (K / 32) * 16);
    auto pre = [&](int sl) {
        if (!wait_count(a, counts + sl, need)) return false;
        load_act_slice(gq, gd, sl, act_q, act_d);
        return true;
    };
    return weight_phase<kLow>(pi, 1, K / kTileK, s_ring(), s_full(), s_empty(), reinterpret_cast<const uint4*>(act_q), act_d,
                        s_part, a.abort_flag, [&](int j, const float4* part) {
                            const int item = pi.first + j * gridDim.x;
                            const float4 y = sum_slices(part, K / kTileK / 4);
                            const float yy[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const int row = g + (k >> 1) * 8;
                                if (row < T) {
                                    float* o = a.x + (size_t)row * H + item * kTileRows + 2 * t + (k & 1);
                                    *o = (j == warp ? xr[k] : __ldcg(o)) + yy[k];
                                }
                            }
                        }, pre);
}

// E: RMSNorm + quantise; gate/up for one 32-feature block per item (four
// (gate, up) pairs of row groups, 8 ring slots), SwiGLU into shared memory
// (warp k: pair k), then the block's q8_0 quantisation for the down
// projection (one row per warp at a time) straight from shared memory.
template <int NK, bool kLow>
__device__ __noinline__ bool phase_gu(int l, long long* cur, int pid, float4 wpre) {
    const KCtx& c = g_ctx;
    const MegaArgs& a = c.a;
    constexpr int K = 256 * NK;
    constexpr int S = K / kTileK / 4;  // slices per row group
    const int T = c.T, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* act_q = s_region();
    float* act_d = reinterpret_cast<float*>(act_q + (size_t)(K / 32) * 512);
    const PhaseInfo pi = c.sch.take(W_GU, &cur[0], &cur[1]);
    // A CTA without gate/up blocks skips the RMSNorm: it must not read x here,
    // since the down projection (no grid barrier before it) may be updating x
    // by then; the CTAs with blocks have read x before any down item ends.
    if (pi.count == 0) return true;
    norm_quant_smem<NK>(a.x, wpre, a.d.eps, T, a.timeline, pid);
    mark(a.timeline, pid, 0);
    float4* s_part = reinterpret_cast<float4*>(act_d + (K / 32) * 16);
    float* s_gu = reinterpret_cast<float*>(s_part + (size_t)pi.count * 8 * S * 32);  // [16 rows][32 features]
    const bool ok = weight_phase<kLow>(pi, 8, K / kTileK, s_ring(), s_full(), s_empty(), reinterpret_cast<const uint4*>(act_q),
                                       act_d, s_part, a.abort_flag, [](int, const float4*) {});
    const int g = lane >> 2, t = lane & 3;
    for (int j = 0; j < pi.count; ++j) {
        const int blk = pi.first + j * gridDim.x;  // features 32 blk .. 32 blk + 31
        if (warp < 4) {
            const float4* part = s_part + (size_t)j * 8 * S * 32;
            const float4 gq = sum_slices(part + (2 * warp) * S * 32, S), uq = sum_slices(part + (2 * warp + 1) * S * 32, S);
            const float gg[4] = {gq.x, gq.y, gq.z, gq.w}, uu[4] = {uq.x, uq.y, uq.z, uq.w};
#pragma unroll
            for (int k = 0; k < (kLow ? 2 : 4); ++k) {
                const int row = g + (k >> 1) * 8;
                if (row < T) {
                    const float sl = gg[k] / (1.0f + exact_expf(-gg[k]));
                    s_gu[row * 32 + 8 * warp + 2 * t + (k & 1)] = sl * uu[k];
                }
            }
        }
        consumer_sync();
        for (int row = warp; row < T; row += kConsumerWarps) {
            const float v = s_gu[row * 32 + lane];
            float am[1] = {warp_absmax(v)}, dq[1], iq[1];
            q8_scales<1>(am, dq, iq);
            a.act2_q[(size_t)blk * 512 + frag_offset(row, lane)] = (uint8_t)q8_code_bits(__fmul_rn(v, iq[0]));
            if (lane == 0) a.act2_d[blk * 16 + row] = __half2float(__float2half_rn(dq[0]));
        }
        consumer_sync();
        // The block's rows are stored (ordered by the barrier): count it for its 256-feature slice.
        if (threadIdx.x == 0) {
            unsigned* cnt = a.slice_done + (size_t)l * (a.d.ffn / 256) + blk / 8;
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
        }
    }
    return ok;
}

// G: final RMSNorm + quantise; LM head with the fused first max -> lm_val[cta].
template <int NK, bool kLow>
__device__ __noinline__ bool phase_lm(long long* cur, int pid, float4 wpre) {
    const KCtx& c = g_ctx;
    const MegaArgs& a = c.a;
    constexpr int K = 256 * NK;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    uint8_t* act_q = s_region();
    float* act_d = reinterpret_cast<float*>(act_q + (size_t)(K / 32) * 512);
    norm_quant_smem<NK>(a.x, wpre, a.d.eps, c.T, a.timeline, pid, blockIdx.x == 0 ? a.capture : nullptr);
    mark(a.timeline, pid, 0);
    const PhaseInfo pi = c.sch.take(W_LM, &cur[0], &cur[1]);
    float best_v[2] = {-INFINITY, -INFINITY};
    int best_i[2] = {0x7fffffff, 0x7fffffff};
    bool ok = true;
    for (int j = warp; j < pi.count; j += kConsumerWarps) {
        const int item = pi.first + j * gridDim.x;
        const long long q0 = pi.slot0 + (long long)j * pi.slots;
        const int jw = j / kConsumerWarps;  // this warp's item count so far
        if (!slot_wait(s_full(), q0, a.abort_flag)) {
            ok = false;
            break;
        }
        if (warp == 0 && jw < 7) mark(a.timeline, pid, 1 + 2 * jw);
        static_assert((K / kTileK) * kTileBytes <= kSlotBytes, "an LM-head item fits one ring slot");
        const float4 y = item_staged<K / kTileK, kLow>(s_ring() + (size_t)(q0 % kRingSlots) * kSlotBytes,
                                                       &s_empty()[q0 % kRingSlots], reinterpret_cast<const uint4*>(act_q),
                                                       act_d);
        if (warp == 0 && jw < 7) mark(a.timeline, pid, 2 + 2 * jw);
        const float yy[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int col = item * kTileRows + 2 * t + (k & 1);
            const int slot = k >> 1;
            if (yy[k] > best_v[slot] || (yy[k] == best_v[slot] && col < best_i[slot])) {
                best_v[slot] = yy[k];
                best_i[slot] = col;
            }
        }
    }
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v[slot], o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i[slot], o);
            if (ov > best_v[slot] || (ov == best_v[slot] && oi < best_i[slot])) {
                best_v[slot] = ov;
                best_i[slot] = oi;
            }
        }
    }
    if (t == 0) {
        g_cand[warp * kTMax + g] = make_float2(best_v[0], __int_as_float(best_i[0]));
        g_cand[warp * kTMax + g + 8] = make_float2(best_v[1], __int_as_float(best_i[1]));
    }
    consumer_sync();
    if (tid < kTMax) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int r = 0; r < kConsumerWarps; ++r) {
            const float2 cc = g_cand[r * kTMax + tid];
            const int ci = __float_as_int(cc.y);
            if (cc.x > bv || (cc.x == bv && ci < bi)) { bv = cc.x; bi = ci; }
        }
        a.lm_val[blockIdx.x * kTMax + tid] = make_float2(bv, __int_as_float(bi));
    }
    return ok;
}

// G on the tensor cores: final RMSNorm + quantise into the tcgen05 operand
// layout; LM-head items are 128-row tiles streamed as 64-K ring slots (one
// tcgen05 weight step each).  Thread 0 issues one kind::i8 MMA (M 128, N 16,
// K 32) per q8_0 block into that block's 16 TMEM columns (all blocks of a tile
// in the 512 columns, two halves so the next tile overlaps the epilogue) and
// frees each ring slot with tcgen05.commit when its MMAs are done; warps 4-7
// (TMEM lane quarters 0-3: one vocab row per thread) read the block sums back,
// evaluate the library's slice-ordered fp32 epilogue per (row, token) and keep
// the first maximum per token.  Same values and the same first max as the
// mma.sync path.
__device__ __forceinline__ uint64_t lm_desc(uint32_t addr) {
    // K-major, no swizzle: 16-byte K chunks 128 bytes apart, 8-row groups 512 bytes apart, version 1.
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46);
}

template <int NK, bool kLow>
__device__ __noinline__ bool phase_lm_tc(long long* cur, int pid, float4 wpre) {
    const KCtx& c = g_ctx;
    const MegaArgs& a = c.a;
    constexpr int K = 256 * NK, NB = K / 32, STEPS = K / 64, HALF = STEPS / 2, TT = kLow ? 8 : kTMax;
    constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(16 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint8_t* act_q = s_region();                                          // [STEPS][1024]
    float* act_d = reinterpret_cast<float*>(s_region() + STEPS * 1024);   // [16][NB]
    norm_quant_smem<NK, true>(a.x, wpre, a.d.eps, c.T, nullptr, 0, blockIdx.x == 0 ? a.capture : nullptr);
    mark(a.timeline, pid, 0);
    const PhaseInfo pi = c.sch.take(W_LM, &cur[0], &cur[1]);
    uint64_t* half_full = g_lm_bars;
    uint64_t* half_free = g_lm_bars + 2;
    if (tid == 0) {
        mbar_init(&half_full[0], 1);
        mbar_init(&half_full[1], 1);
        mbar_init(&half_free[0], 4);
        mbar_init(&half_free[1], 4);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // The activation bytes were written by the generic proxy; the tensor core reads them through the async proxy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(&g_tmem)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    consumer_sync();
    mark(a.timeline, pid, 1);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = g_tmem;
    bool ok = true;
    float best_v[TT];
    int best_i[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) { best_v[t] = -INFINITY; best_i[t] = 0x7fffffff; }
    if (tid == 0) {
        for (int j = 0; j < pi.count && ok; ++j) {
            const long long q0 = pi.slot0 + (long long)j * pi.slots;
            for (int ks = 0; ks < STEPS && ok; ++ks) {
                const int h = ks / HALF;
                if (ks % HALF == 0 && j > 0 && !mbar_wait(&half_free[h], unsigned((j - 1) & 1), a.abort_flag)) { ok = false; break; }
                const long long q = q0 + ks;
                if (!mbar_wait(&s_full()[q % kRingSlots], unsigned((q / kRingSlots) & 1), a.abort_flag)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t wslot = smem_addr(s_ring() + (size_t)(q % kRingSlots) * kSlotBytes);
                const uint32_t xstep = smem_addr(act_q + ks * 1024);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const uint32_t d = tmem + (uint32_t)(((2 * ks + b) % NB) * 16);
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n"
                        ::"r"(d), "l"(lm_desc(wslot + b * 256)), "l"(lm_desc(xstep + b * 256)), "r"(kIdesc), "r"(0),
                          "r"(0), "r"(0), "r"(0), "r"(0)
                        : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                             ::"r"(smem_addr(&s_empty()[q % kRingSlots])) : "memory");
                if (ks % HALF == HALF - 1)
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                                 ::"r"(smem_addr(&half_full[h])) : "memory");
            }
        }
    } else if (warp >= 4) {
        const int q4 = warp & 3, r = 32 * q4 + lane;
        for (int j = 0; j < pi.count && ok; ++j) {
            const int item = pi.first + j * gridDim.x;
            const uint8_t* tile = a.lm_tiles + (size_t)item * STEPS * kSlotBytes;
            float y[TT], acc[TT];  // acc: the open 256-K slice (a slice may span both halves)
#pragma unroll
            for (int t = 0; t < TT; ++t) y[t] = acc[t] = 0.f;
            for (int h = 0; h < 2 && ok; ++h) {
                // This row's weight scales of the half (fp16 pairs per 64-K step), before the wait.
                uint32_t wsc[HALF];
#pragma unroll
                for (int u = 0; u < HALF; ++u)
                    wsc[u] = __ldg(reinterpret_cast<const uint32_t*>(tile + (size_t)(h * HALF + u) * kSlotBytes + 8192) + r);
                int wok = 1;
                if (lane == 0) wok = mbar_wait(&half_full[h], unsigned(j & 1), a.abort_flag) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, wok, 0)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                static_assert((2 * HALF) % 4 == 0, "blocks of a half in groups of 4");
#pragma unroll 1
                for (int b4 = 0; b4 < 2 * HALF; b4 += 4) {
                    // Four blocks' sums (4 x 16 columns) in one TMEM load.
                    uint32_t v[64];
                    const int kb0 = 2 * HALF * h + b4;
                    const uint32_t ta = tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)((kb0 % NB) * 16);
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,"
                        "%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
                        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
                          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
                          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]),
                          "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]),
                          "=r"(v[40]), "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]),
                          "=r"(v[48]), "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]),
                          "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
                        : "r"(ta));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int bb = b4 + u, kb = kb0 + u;
                        const float dw = (bb & 1) ? h2f_hi(wsc[bb / 2]) : h2f_lo(wsc[bb / 2]);
#pragma unroll
                        for (int t = 0; t < TT; ++t)
                            acc[t] = fmaf((float)(int)v[16 * u + t], __fmul_rn(dw, act_d[t * NB + kb]), acc[t]);
                        if (kb % 8 == 7) {  // a 256-K slice is complete: add it in order
#pragma unroll
                            for (int t = 0; t < TT; ++t) {
                                y[t] = __fadd_rn(y[t], acc[t]);
                                acc[t] = 0.f;
                            }
                        }
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&half_free[h]);
            }
            if (!ok) break;
            if (warp == 4 && j < 12 && lane == 0 && blockIdx.x < 256 && a.timeline)
                a.timeline[kCtaMarkBase + ((size_t)blockIdx.x * kMaxBarriers + pid) * kCtaMarks + 2 + j] = global_ns();
            const int col = item * 128 + r;
#pragma unroll
            for (int t = 0; t < TT; ++t)
                if (y[t] > best_v[t] || (y[t] == best_v[t] && col < best_i[t])) { best_v[t] = y[t]; best_i[t] = col; }
        }
        if (!ok) consumer_fail(a);
    }
    if (!ok && tid == 0) consumer_fail(a);
    // First max over the warp's rows for each token, then over the warps.
#pragma unroll
    for (int t = 0; t < TT; ++t) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v[t], o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i[t], o);
            if (ov > best_v[t] || (ov == best_v[t] && oi < best_i[t])) { best_v[t] = ov; best_i[t] = oi; }
        }
    }
    if (lane == 0)
#pragma unroll
        for (int t = 0; t < kTMax; ++t)
            g_cand[warp * kTMax + t] = t < TT ? make_float2(best_v[t < TT ? t : 0], __int_as_float(best_i[t < TT ? t : 0]))
                                              : make_float2(-INFINITY, __int_as_float(0x7fffffff));
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    consumer_sync();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    if (tid < kTMax) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < kConsumerWarps; ++w) {
            const float2 cc = g_cand[w * kTMax + tid];
            const int ci = __float_as_int(cc.y);
            if (cc.x > bv || (cc.x == bv && ci < bi)) { bv = cc.x; bi = ci; }
        }
        a.lm_val[blockIdx.x * kTMax + tid] = make_float2(bv, __int_as_float(bi));
    }
    return ok;
}

// H (CTA 0): first max over the CTA partials, acceptance and rollback.
__device__ __noinline__ void phase_accept() {
    const KCtx& c = g_ctx;
    const MegaArgs& a = c.a;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int row = warp; row < c.T; row += kConsumerWarps) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int b = lane; b < (int)gridDim.x; b += 32) {
            const float2 cc = __ldcg(&a.lm_val[b * kTMax + row]);
            const int ci = __float_as_int(cc.y);
            if (cc.x > bv || (cc.x == bv && ci < bi)) { bv = cc.x; bi = ci; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            const int si = c.row_stream[row];
            a.st_state[si]->choice[row - c.s_row0[si]] = bi == 0x7fffffff ? 0 : bi;
            if (a.capture) {
                float* cap = a.capture + (size_t)kTMax * a.d.hidden;
                cap[2 * row] = bv;
                cap[2 * row + 1] = __int_as_float(bi);
            }
        }
    }
    if (a.capture && threadIdx.x < kMaxStreams) {
        int* cap = reinterpret_cast<int*>(a.capture + (size_t)kTMax * a.d.hidden + 2 * kTMax);
        const bool on = (int)threadIdx.x < a.n_streams;
        cap[2 * threadIdx.x] = on ? c.s_T[threadIdx.x] : 0;
        cap[2 * threadIdx.x + 1] = on ? c.s_row0[threadIdx.x] : 0;
        if (threadIdx.x == 0) cap[2 * kMaxStreams] = c.T;
    }
    consumer_sync();
    // One thread per stream.  A stream whose proposals did not all fit the
    // step's rows verified the first s_T - 1 of them: its proposal count is cut to that.
    if (threadIdx.x < a.n_streams && c.s_T[threadIdx.x] > 0) {
        StepState* st = a.st_state[threadIdx.x];
        if (st->T != c.s_T[threadIdx.x]) {
            st->T = c.s_T[threadIdx.x];
            st->n_prop = st->T - 1;
        }
        accept_choices(st, a.st_ids[threadIdx.x]);
    }
    if (a.timeline && threadIdx.x == 0) {
        a.timeline[kTimelineStart + 1] = global_ns();
        a.timeline[kCtaMarkBase + (size_t)(kMaxBarriers - 1) * kCtaMarks + 1] = clock64();
    }
}

// The consumer warps' phase sequence; kLow: the step has at most 8 rows.
template <int kNK, bool kLow>
__device__ __noinline__ void run_phases() {
    const KCtx& c = g_ctx;
    unsigned target = 0;
    int nb = 0;                 // grid barriers passed (the timeline's phase index)
    long long cur[2] = {0, 0};  // schedule cursor (Schedule::take)
    const int L = c.a.d.n_layers;
    phase_embed();
    // Each row norm's weights are requested before the barrier in front of it.
    float4 wpre = norm_weights_prefetch<kNK>(c.a.layers[0].attn_norm);
    if (!end_phase(&target, &nb)) return;
    for (int l = 0; l < L; ++l) {
        if (!phase_qkv<kNK, kLow>(l, cur, nb, wpre)) consumer_fail(c.a);
        if (!end_phase(&target, &nb)) return;
        // B, C and D share one barrier interval (D waits per slice on C), as do E and F.
        if (!phase_attn(l, cur, nb)) consumer_fail(c.a);
        if (!phase_combine(l)) consumer_fail(c.a);
        if (!phase_proj_resid<kLow>(l, cur, kSubPhaseO + l, false)) consumer_fail(c.a);
        wpre = norm_weights_prefetch<kNK>(c.a.layers[l].ffn_norm);
        if (!end_phase(&target, &nb)) return;
        if (!phase_gu<kNK, kLow>(l, cur, nb, wpre)) consumer_fail(c.a);
        if (!phase_proj_resid<kLow>(l, cur, kSubPhaseDown + l, true)) consumer_fail(c.a);
        wpre = norm_weights_prefetch<kNK>(l + 1 < L ? c.a.layers[l + 1].attn_norm : c.a.output_norm);
        if (!end_phase(&target, &nb)) return;
    }
    if (c.a.lm_tiles ? !phase_lm_tc<kNK, kLow>(cur, nb, wpre)
                     : !phase_lm<kNK, kLow>(cur, nb, wpre))
        consumer_fail(c.a);
    if (!end_phase(&target, &nb)) return;
    if (blockIdx.x == 0) phase_accept();
}

// Tensor maps of the streams' KV caches (a kernel parameter: TMA reads them
// from parameter space).
struct KvMaps {
    CUtensorMap m[kMaxStreams];
};

template <int kNK>
__global__ void __launch_bounds__(kMegaThreads, 1)
    k_verify_persistent(MegaArgs args, const __grid_constant__ KvMaps kv_maps) {
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        KCtx& c = g_ctx;
        c.a = args;
        // The streams' rows: every active stream (T > 0) keeps its seed row;
        // the rows left over go to the proposals in stream order, so that
        // the step never exceeds kTMax rows (every CTA computes the same table).
        int active = 0;
        for (int si = 0; si < args.n_streams; ++si) active += args.st_state[si]->T > 0;
        int spare = kTMax - active, rows = 0;
        for (int si = 0; si < args.n_streams; ++si) {
            const StepState* st = args.st_state[si];
            int T = st->T;
            if (T > 0) {
                const int extra = min(T - 1, max(spare, 0));
                spare -= extra;
                T = 1 + extra;
            } else {
                T = 0;
            }
            if (rows + T > kTMax) T = 0;  // more active streams than rows: cannot happen with kMaxStreams <= kTMax
            // Checked build: a stream whose chunks exceed the partial buffers is left out.
            if (T > 0 && !bc_check((st->before + T + kPage - 1) / kPage <= args.max_chunks, BC_PARTIALS)) T = 0;
            c.s_T[si] = T;
            c.s_row0[si] = rows;
            c.s_before[si] = st->before;
            c.s_chunks[si] = T > 0 ? (st->before + T + kPage - 1) / kPage : 0;
            for (int t = 0; t < T; ++t) c.row_stream[rows + t] = si;
            rows += T;
        }
        c.T = rows;
        int max_nq = 0;
        for (int si = 0; si < args.n_streams; ++si) max_nq = max(max_nq, c.s_T[si] * (args.d.n_heads / args.d.n_kv));
        c.attn_wpi = max_nq <= 4 && args.st_kv[0].type == KV_F16 ? 2 : max_nq > 16 ? 8 : 4;
        c.sch.init(args.d, gridDim.x, blockIdx.x, args.st_kv[0].type == KV_F16, c.s_chunks, args.n_streams,
                   args.lm_tiles != nullptr);
        if (args.timeline && blockIdx.x == 0) {
            args.timeline[kTimelineStart] = global_ns();
            // SM cycles beside the timer (CTA 0, last barrier slot): the clock the step ran at.
            args.timeline[kCtaMarkBase + (size_t)(kMaxBarriers - 1) * kCtaMarks] = clock64();
        }
        for (int s = 0; s < kRingSlots; ++s) {
            mbar_init(&s_full()[s], 1);
            mbar_init(&s_empty()[s], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const KCtx& c = g_ctx;
    if (c.T <= 0) return;
    if (smem_addr(g_smem) & 1023) {  // the K/V boxes need a 1024-aligned ring
        if (threadIdx.x == 0 && blockIdx.x == 0) args.st_state[0]->error = 3;
        return;
    }
    if (warp == kConsumerWarps) {
        producer(c.a, kv_maps.m, c.sch, s_ring(), s_full(), s_empty());
        return;
    }
    if (c.T <= 8)
        run_phases<kNK, true>();
    else
        run_phases<kNK, false>();
}


}  // namespace

int megakernel_smem_bytes() {
    return kRingSlots * kSlotBytes + kRegionBytes + kRopeBytes + 2 * kRingSlots * 8;
}

template <int NK>
cudaError_t configure_one(int device, int* grid_out) {
    cudaError_t e = cudaFuncSetAttribute(k_verify_persistent<NK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         megakernel_smem_bytes());
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_verify_persistent<NK>, kMegaThreads,
                                                      megakernel_smem_bytes());
    if (e != cudaSuccess) return e;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    *grid_out = per_sm >= 1 ? sms : 0;
    return cudaSuccess;
}

cudaError_t configure_megakernel(int device, int hidden, int* grid_out) {
    switch (hidden) {
        case 256: return configure_one<1>(device, grid_out);
        case 512: return configure_one<2>(device, grid_out);
        case 1024: return configure_one<4>(device, grid_out);
        default: *grid_out = 0; return cudaSuccess;
    }
}

bool megakernel_supports(const ModelDims& d, int grid) {
    if (grid <= 0) return false;
    const bool hidden_ok = d.hidden == 256 || d.hidden == 512 || d.hidden == 1024;
    // Query rows are tiled in pairs (T * group must be even for every T).
    if (!hidden_ok || (d.n_heads / d.n_kv) % 2 != 0 || d.n_heads / d.n_kv * kTMax > 32) return false;
    if (d.ffn % 256 || (d.ffn / kTileRows) % 4) return false;  // down slices of 256 features = 8 gate/up blocks
    if (d.n_heads % 2) return false;                                // O slices of 256 = one pair of q heads
    const int qd = d.n_heads * kHeadDim;
    // Per weight phase: fragments + scales of its K plus 512 bytes per slice
    // unit of the CTA's items must fit the shared region.
    auto need = [&](int K, int items, int units_per_item) {
        return (size_t)(K / 32) * (512 + 64) + (size_t)((items + grid - 1) / grid) * units_per_item * 512;
    };
    const size_t worst = std::max(std::max(need(d.hidden, (qd + 2 * d.n_kv * kHeadDim) / kTileRows, d.hidden / 256),
                                           need(qd, d.hidden / kTileRows, qd / 256)),
                                  std::max(need(d.hidden, d.ffn / 32, 8 * d.hidden / 256) + 16 * 32 * 4,
                                           need(d.ffn, d.hidden / kTileRows, d.ffn / 256)));
    const size_t attn = (size_t)2 * 32 * kAttnRowBytes;  // two groups of up to 32 query rows
    return worst <= (size_t)kRegionBytes && attn <= (size_t)kRegionBytes;
}

static_assert(sizeof(KvTensorMap) == sizeof(CUtensorMap) && alignof(KvTensorMap) >= alignof(CUtensorMap),
              "KvTensorMap holds a CUtensorMap");

cudaError_t encode_kv_map(const KvCache& kv, long long pool_elems, KvTensorMap* out) {
    using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return e != cudaSuccess ? e : cudaErrorNotSupported;
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    const bool f16 = kv.type == KV_F16;
    const int row_bytes = f16 ? KvSlots<true>::kRowBytes : KvSlots<false>::kRowBytes;
    const int rps = f16 ? KvSlots<true>::kRowsPerSlot : KvSlots<false>::kRowsPerSlot;
    const long long rows = pool_elems / kHeadDim;
    if (rows >= (1ll << 31)) return cudaErrorInvalidValue;  // tile row coordinates are int32
    // The cache as bytes [rows][row_bytes]; a box is [rps rows][128 bytes].
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {128, (cuuint32_t)rps}, elem_strides[2] = {1, 1};
    CUtensorMap map;
    const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, kv.base, dims, strides, box, elem_strides,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    std::memcpy(out, &map, sizeof(map));
    return cudaSuccess;
}

cudaError_t launch_step_persistent_group(const DeviceModel& m, const LayerWeights* layers_dev, const KvCache* kvs,
                                         const KvTensorMap* maps, StepState* const* states, int32_t* const* ids,
                                         int n_streams, const StepBuffers& b, const MegaBuffers& mb, int grid,
                                         cudaStream_t s) {
    if (n_streams < 1 || n_streams > kMaxStreams) return cudaErrorInvalidValue;
    KvMaps km;
    std::memset(&km, 0, sizeof(km));
    for (int i = 0; i < n_streams; ++i) std::memcpy(&km.m[i], &maps[i], sizeof(CUtensorMap));
    MegaArgs a{};
    a.timeline = mb.timeline;
    a.capture = mb.capture;
    a.d = m.dims;
    a.layers = layers_dev;
    a.embd = m.embd;
    a.lm_tiles = m.pf_embd;
    a.output_norm = m.output_norm;
    a.theta_scale = m.theta_scale;
    a.n_streams = n_streams;
    for (int i = 0; i < n_streams; ++i) {
        a.st_kv[i] = kvs[i];
        a.st_state[i] = states[i];
        a.st_ids[i] = ids[i];
    }
    a.x = b.x;
    a.qkv = b.qkv;
    a.gu = b.gu;
    a.act_q = b.act_q;
    a.act_d = b.act_d;
    a.act2_q = mb.act2_q;
    a.act2_d = mb.act2_d;
    a.part_o = b.part_o;
    a.part_ml = b.part_ml;
    a.max_chunks = b.max_chunks;
    a.lm_val = mb.lm_val;
    a.bar = mb.bar;
    a.abort_flag = mb.abort_flag;
    a.head_done = mb.head_done;
    a.pair_done = mb.pair_done;
    a.m_max = mb.m_max;
    a.slice_done = mb.slice_done;
    a.wait_ns = mb.wait_ns;
    a.stall_barrier = mb.stall_barrier;
    cudaError_t e = cudaMemsetAsync(mb.bar, 0, mb.zero_bytes, s);  // barrier counter, abort flag, head counts
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMegaThreads);
    cfg.dynamicSmemBytes = megakernel_smem_bytes();
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident, or the launch fails
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (m.dims.hidden) {
        case 256: return cudaLaunchKernelEx(&cfg, k_verify_persistent<1>, a, km);
        case 512: return cudaLaunchKernelEx(&cfg, k_verify_persistent<2>, a, km);
        default: return cudaLaunchKernelEx(&cfg, k_verify_persistent<4>, a, km);
    }
}

cudaError_t launch_step_persistent(const DeviceModel& m, const LayerWeights* layers_dev, const KvCache& kv,
                                   const KvTensorMap& map, const StepBuffers& b, const MegaBuffers& mb, int grid,
                                   cudaStream_t s) {
    StepState* state = b.state;
    int32_t* ids = b.ids;
    return launch_step_persistent_group(m, layers_dev, &kv, &map, &state, &ids, 1, b, mb, grid, s);
}

MTB_BC_TAKE(bc_take_megakernel)

}  // namespace mtb
