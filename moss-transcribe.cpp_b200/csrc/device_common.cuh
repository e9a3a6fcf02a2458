// Device helpers shared by the verify-step kernels (kernels.cu) and the
// persistent verify-step kernel (megakernel.cu).
#pragma once

#include "mtb_internal.hpp"
#include "exact_math.cuh"
#include "kernels.hpp"

#include <cuda_fp16.h>

namespace mtb {
namespace dev {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    // D[16 tokens x 8 weight rows] = A[16 x 32] * B[32 x 8], int8 -> int32.
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ uint4 ld_stream_u4(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint2 ld_nc_u2(const uint8_t* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// (float)c for |c| < 2^22 (an int8 x int8 block sum of 32 or 64 products is
// at most 2^20): the int's bits added to those of 1.5 * 2^23, minus 1.5 * 2^23,
// on the FMA and integer pipes instead of the conversion unit.  Exact.
__device__ __forceinline__ float small_int_to_float(int c) {
    return __fsub_rn(__int_as_float(c + 0x4B400000), 12582912.0f);
}

__device__ __forceinline__ float h2f_lo(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xffffu))); }
__device__ __forceinline__ float h2f_hi(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The hidden-row RMSNorm sum of squares (the tree shared by every kernel and
// the CPU restatement).  Element squares s_i = (double)(x_i * x_i) (the float
// product, widened); each 32-element block summed pairwise over adjacent
// pairs, ((s0 + s1) + (s2 + s3)) + ...; lane l's partial the blocks l, l + 32,
// ... added in that order from 0; the lane partials combined by one xor
// butterfly.
__device__ __forceinline__ double block_sum_squares(const float (&v)[32]) {
    double u[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) u[i] = (double)(v[2 * i] * v[2 * i]) + (double)(v[2 * i + 1] * v[2 * i + 1]);
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) u[i] = u[2 * i] + u[2 * i + 1];
    return u[0];
}

// 1 / sqrt(mean(x^2) + eps) of a row of K (a multiple of 32, at most 32 x 64)
// elements by a block of nthreads >= K / 32 threads (all of them call it):
// thread b < K / 32 sums block b, warp 0 combines.  s_q holds K / 32 doubles.
__device__ __forceinline__ float row_rms_scale(const float* row, int K, float eps, double* s_q, float* s_scale) {
    const int nb = K / 32;
    if ((int)threadIdx.x < nb) {
        float v[32];
        const float4* r4 = reinterpret_cast<const float4*>(row + 32 * threadIdx.x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 f = r4[i];
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        s_q[threadIdx.x] = block_sum_squares(v);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        double p = 0.0;
        for (int b = threadIdx.x; b < nb; b += 32) p += s_q[b];
        p = warp_sum_d(p);
        if (threadIdx.x == 0) *s_scale = 1.0f / sqrtf((float)(p / K) + eps);
    }
    __syncthreads();
    return *s_scale;
}

// amax of |v| over the 32 lanes: non-negative floats order like their bit
// patterns, so one integer max reduction gives exactly fmaxf's result.
__device__ __forceinline__ float warp_absmax(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
}

// q8_0 scales of up to 32 blocks at once: amax[i] is uniform across the warp;
// lane i computes d = amax/127 and 1/d' = 127/amax of block i (correctly
// rounded divisions, one per lane instead of 2N in sequence), then block i's
// pair is broadcast back by shuffles.  Results equal the per-block formulas.
template <int N>
__device__ __forceinline__ void q8_scales(const float (&amax)[N], float (&d)[N], float (&inv)[N]) {
    static_assert(N <= 32, "one block per lane");
    const int lane = threadIdx.x & 31;
    float mine = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (lane == i) mine = amax[i];
    const float dl = mine / 127.f;
    const float il = mine != 0.0f ? 127.f / mine : 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        d[i] = __shfl_sync(0xffffffffu, dl, i);
        inv[i] = __shfl_sync(0xffffffffu, il, i);
    }
}

// Byte offset of activation element (row r in 0..15, column c in 0..31) inside
// one 512-byte block of the m16n8k32 A-fragment order: lane (g, t) holds
// {A[g][4t..], A[g+8][4t..], A[g][16+4t..], A[g+8][16+4t..]}.
__device__ __forceinline__ int frag_offset(int r, int c) {
    const int g = r & 7, hi = r >> 3, t4 = (c & 15) >> 2, part = c >> 4;
    return (g * 4 + t4) * 16 + (part * 2 + hi) * 4 + (c & 3);
}

// q8_0 quantisation of one 32-element block held one element per lane, as
// The q8_0 code of x (|x| <= 127, or NaN) as the low byte of the returned
// bits: adding 1.5 * 2^23 rounds x to the nearest integer, ties to even (the
// sum's unit in the last place is 1), and leaves it in two's complement in
// the low bits -- the same code as __float2int_rn, without the conversion
// unit.  NaN gives code 0, as the conversion does.
__device__ __forceinline__ uint32_t q8_code_bits(float x) {
    const uint32_t b = __float_as_uint(__fadd_rn(x, 12582912.0f));
    return x == x ? b : 0u;
}

// ggml's x86 from_float: d = amax/127 (stored fp16), code = rint(x * 127/amax).
__device__ __forceinline__ void quantize_block_lane(float v, int row, int blk, uint8_t* act_q, float* act_d) {
    const int lane = threadIdx.x & 31;
    const float amax = warp_absmax(v);
    const float d = amax / 127.f;
    const float id = amax != 0.0f ? 127.f / amax : 0.0f;
    act_q[(size_t)blk * 512 + frag_offset(row, lane)] = (uint8_t)q8_code_bits(__fmul_rn(v, id));
    if (lane == 0) act_d[blk * 16 + row] = __half2float(__float2half_rn(d));
}

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor in the
// stream still runs.  pdl_wait() returns once the predecessor has completed
// and its writes are visible (immediately for a normal launch), so a kernel
// reads or writes step data only after it; pdl_launch_dependents() lets the
// next such kernel start its own independent prologue (weight loads).  Every
// kernel of a programmatic chain calls pdl_wait() before touching step data.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Index checks of the bounds-check build: record the first violated site and
// tell the caller to skip (or redirect) the access.  In a normal build every
// check is `true` and compiles away.
#ifdef MTB_BOUNDS_CHECK
static __device__ unsigned g_bc_site;
__device__ __forceinline__ bool bc_check(bool ok, unsigned site) {
    if (!ok) atomicCAS(&g_bc_site, 0u, site);
    return ok;
}
#define MTB_BC_TAKE(fn)                                   \
    unsigned fn() {                                       \
        unsigned v = 0, z = 0;                            \
        cudaMemcpyFromSymbol(&v, g_bc_site, sizeof(v));   \
        cudaMemcpyToSymbol(g_bc_site, &z, sizeof(z));     \
        return v;                                         \
    }
#else
__device__ __forceinline__ bool bc_check(bool, unsigned) { return true; }
#define MTB_BC_TAKE(fn) \
    unsigned fn() { return 0; }
#endif

__device__ __forceinline__ long long kv_offset(const KvCache& kv, int n_kv, int layer, int which, int head, int pos) {
    // Checked build: an out-of-range position or page reads/writes element 0
    // of the pool instead (and the site is recorded).
    if (!bc_check(pos >= 0 && pos < kv.n_pages * kPage, BC_KV_POSITION)) return 0;
    const int page = kv.pages[pos / kPage];
    if (!bc_check(page >= 0 && page < kv.n_pages, BC_KV_PAGE)) return 0;
    return (long long)page * kv.page_elems +
           ((((long long)layer * 2 + which) * n_kv + head) * kPage + (pos % kPage)) * kHeadDim;
}

__device__ __forceinline__ float kv_load(const KvCache& kv, long long off) {
    return kv.type == KV_F16 ? __half2float(reinterpret_cast<const __half*>(kv.base)[off])
                             : reinterpret_cast<const float*>(kv.base)[off];
}

__device__ __forceinline__ void kv_store(const KvCache& kv, long long off, float v) {
    if (kv.type == KV_F16) reinterpret_cast<__half*>(kv.base)[off] = __float2half_rn(v);
    else reinterpret_cast<float*>(kv.base)[off] = v;
}


// Emit one id into the generated stream (src/cpu_speculative.cpp:90-98).
__device__ __forceinline__ void emit_id(StepState* st, int32_t* ids, int id) {
    ids[st->n_ids++] = id;
    if (id == st->eos) st->stop = STOP_EOS;
    else if (st->n_ids >= st->max_new) st->stop = STOP_LIMIT;
}

// Strict acceptance and logical rollback (src/cpu_speculative.cpp:124-136)
// given the per-row choices, then the next seed (the choice of the last kept
// row, :124-129).  One thread.
__device__ __forceinline__ void accept_choices(StepState* st, int32_t* ids) {
    const int np = st->n_prop;
    st->target_calls += 1;
    st->drafted_calls += np > 0;
    st->proposed += np;
    st->target_input_tokens += st->T;
    int keep = 1;
    for (int i = 0; i < np; ++i) {
        const int prop = st->tokens[1 + i];
        if (prop != st->choice[i]) break;
        st->accepted += 1;
        emit_id(st, ids, prop);
        if (st->stop) break;  // the terminating token is not kept in the cache
        ++keep;
    }
    const int position = st->before + keep;
    if (st->before + st->T != position) st->rewinds += 1;
    st->past = position;
    st->commit_n = st->n_ids;
    st->commit_stop = st->stop != STOP_NONE;
    if (!st->stop) {
        st->seed = st->choice[keep - 1];
        emit_id(st, ids, st->seed);
    }
}

}  // namespace dev
}  // namespace mtb
