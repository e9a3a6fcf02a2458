// sm_100a kernels of the strict speculative verify step.
//
// One verify step = draft -> embed -> 28 x (norm+quantise, QKV, QK-norm+RoPE+
// KV store, attention, O+residual, norm+quantise, gate/up+SwiGLU, quantise,
// down+residual) -> final norm -> LM head with fused first-max -> accept and
// rollback.  Every kernel reads the step's row count and positions from the
// device StepState, so the whole step is one fixed launch sequence that is
// captured once in a CUDA graph and replayed without host round trips.
//
// The layer arithmetic follows src/qwen3.cpp:62-218 of the reference; the
// q8_0 contract (activation quantised to q8_0 before every q8_0 dot, exact
// integer block sums, fp32 d_w*d_x scaling) follows ggml's CPU mul_mat as used
// by src/cpu_projection.cpp:16-37.
#include "device_common.cuh"
#include "prefill_tc.hpp"

#include <cuda_fp16.h>
#include <cfloat>
#include <cstdlib>
#include <cstdio>

namespace mtb {

// SMs of the device the kernels were last configured for (configure_kernels,
// at model load); the grid choices below are made for it.
static int g_sm_count = 148;

namespace {

using namespace dev;

// ------------------------------------------------------------------ repack

// Raw ggml q8_0 rows (34-byte blocks) -> 544-byte tiles of 8 rows x 64 k:
// lane (g, t) of a tile holds row g's bytes {4t, 16+4t} of both blocks, the
// B fragment of m16n8k32; the 16 fp16 scales follow as [t][block][row&1].
__global__ void k_repack_q8(const uint8_t* __restrict__ src, int n_rows, int k, uint8_t* __restrict__ dst,
                            int rg_stride, int rg_offset) {
    const int kt_n = k / kTileK;
    const long long tiles = (long long)(n_rows / kTileRows) * kt_n;
    const int blocks_per_row = k / kQ8Block;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tiles * 32; i += (long long)gridDim.x * blockDim.x) {
        const long long tile = i / 32;
        const int lane = int(i % 32);
        const int rg = int(tile / kt_n), kt = int(tile % kt_n);
        const int g = lane >> 2, t = lane & 3;
        const int row = rg * kTileRows + g;
        uint8_t* out = dst + ((long long)(rg * rg_stride + rg_offset) * kt_n + kt) * kTileBytes;
        uint8_t bytes[16];
        for (int blk = 0; blk < 2; ++blk) {
            const uint8_t* b = src + ((long long)row * blocks_per_row + kt * 2 + blk) * 34;
            for (int j = 0; j < 4; ++j) {
                bytes[blk * 8 + j] = b[2 + 4 * t + j];
                bytes[blk * 8 + 4 + j] = b[2 + 16 + 4 * t + j];
            }
        }
        for (int j = 0; j < 16; ++j) out[lane * 16 + j] = bytes[j];
        if (lane < 16) {  // scales: lane -> (t', blk, j) = (lane>>2, (lane>>1)&1, lane&1)
            const int tt = lane >> 2, blk = (lane >> 1) & 1, j = lane & 1;
            const int srow = rg * kTileRows + 2 * tt + j;
            const uint8_t* b = src + ((long long)srow * blocks_per_row + kt * 2 + blk) * 34;
            out[512 + lane * 2] = b[0];
            out[512 + lane * 2 + 1] = b[1];
        }
    }
}

// ------------------------------------------------------------------ GEMV

enum Epi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

struct GemvArgs {
    const uint8_t* w;     // tiles
    int n_rg;             // row groups of 8
    int kt_n;             // K / 64
    const uint8_t* act_q; // fragment-order activation, K/32 blocks of 512 bytes
    const float* act_d;   // [K/32][16]
    float* out;           // EPI_STORE / EPI_SWIGLU: [16][ld]; EPI_RESID: x [16][ld]
    int ld;               // output row stride (floats)
    const StepState* state;
    float2* lm_val;       // EPI_ARGMAX partials [gridDim.x][16]
    float* logits;        // EPI_ARGMAX: optional full logits [16][ld]
};

// Skinny q8_0 GEMM: y[t][n] = sum_blocks dw[n,b] * dx[t,b] * sum_32 qw * qx for
// up to 16 rows t.  Evaluation order (shared with the CPU restatement): per
// output, one fmaf per 32-block in ascending order inside each 256-element
// slice (4 tiles), then the slice partials added in ascending order.
// A CTA iteration covers RPB row groups; its RPB * S (row group, slice) items
// are spread over the 8 warps (the next item's tiles load while the current
// one computes), and warp r < RPB adds the slices of row group r.
constexpr int kSliceTiles = 4;

template <int EPI, int RPB>
__global__ void __launch_bounds__(kThreads) k_gemv(GemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int kb_n = a.kt_n * 2;
    const int S = a.kt_n / kSliceTiles;
    uint4* s_act = reinterpret_cast<uint4*>(smem);                       // [kb_n][32]
    float* s_d = reinterpret_cast<float*>(s_act + kb_n * 32);            // [kb_n][16]
    float4* s_part = reinterpret_cast<float4*>(s_d + kb_n * 16);         // [RPB][S][32]
    const int T = a.state->T;
    if (T <= 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    {
        const uint4* src = reinterpret_cast<const uint4*>(a.act_q);
        for (int i = threadIdx.x; i < kb_n * 32; i += kThreads) s_act[i] = src[i];
        for (int i = threadIdx.x; i < kb_n * 16; i += kThreads) s_d[i] = a.act_d[i];
    }
    __syncthreads();
    const int n_items = RPB * S;
    float best_v[2] = {-INFINITY, -INFINITY};
    int best_i[2] = {0x7fffffff, 0x7fffffff};

    for (int rg0 = blockIdx.x * RPB; rg0 < a.n_rg; rg0 += gridDim.x * RPB) {
        uint4 wv[kSliceTiles];
        uint2 sv[kSliceTiles];
        auto load = [&](int it, uint4 (&w)[kSliceTiles], uint2 (&sc)[kSliceTiles]) {
            const int rg = rg0 + it / S, sl = it % S;
            if (rg >= a.n_rg) return;
            const uint8_t* tile = a.w + ((size_t)rg * a.kt_n + (size_t)sl * kSliceTiles) * kTileBytes;
#pragma unroll
            for (int u = 0; u < kSliceTiles; ++u) {
                w[u] = ld_stream_u4(tile + (size_t)u * kTileBytes + lane * 16);
                sc[u] = ld_nc_u2(tile + (size_t)u * kTileBytes + 512 + t * 8);
            }
        };
        int it = warp;
        if (it < n_items) load(it, wv, sv);
        while (it < n_items) {
            const int next = it + kWarps;
            uint4 wn[kSliceTiles];
            uint2 sn[kSliceTiles];
            if (next < n_items) load(next, wn, sn);
            const int r = it / S, sl = it % S;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            if (rg0 + r < a.n_rg) {
#pragma unroll
                for (int u = 0; u < kSliceTiles; ++u) {
                    const int kt = sl * kSliceTiles + u;
                    int c0[4], c1[4];
                    mma_s8(c0, s_act[(2 * kt) * 32 + lane], wv[u].x, wv[u].y);
                    mma_s8(c1, s_act[(2 * kt + 1) * 32 + lane], wv[u].z, wv[u].w);
                    const float x0g = s_d[(2 * kt) * 16 + g], x0h = s_d[(2 * kt) * 16 + g + 8];
                    const float x1g = s_d[(2 * kt + 1) * 16 + g], x1h = s_d[(2 * kt + 1) * 16 + g + 8];
                    const float w00 = h2f_lo(sv[u].x), w01 = h2f_hi(sv[u].x);  // block 0, rows 2t, 2t+1
                    const float w10 = h2f_lo(sv[u].y), w11 = h2f_hi(sv[u].y);  // block 1
                    // d = dw * dx is exact (two fp16 values); one fmaf per block.
                    acc[0] = fmaf(small_int_to_float(c0[0]), w00 * x0g, acc[0]);
                    acc[1] = fmaf(small_int_to_float(c0[1]), w01 * x0g, acc[1]);
                    acc[2] = fmaf(small_int_to_float(c0[2]), w00 * x0h, acc[2]);
                    acc[3] = fmaf(small_int_to_float(c0[3]), w01 * x0h, acc[3]);
                    acc[0] = fmaf(small_int_to_float(c1[0]), w10 * x1g, acc[0]);
                    acc[1] = fmaf(small_int_to_float(c1[1]), w11 * x1g, acc[1]);
                    acc[2] = fmaf(small_int_to_float(c1[2]), w10 * x1h, acc[2]);
                    acc[3] = fmaf(small_int_to_float(c1[3]), w11 * x1h, acc[3]);
                }
            }
            s_part[(r * S + sl) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            if (next < n_items) {
#pragma unroll
                for (int u = 0; u < kSliceTiles; ++u) { wv[u] = wn[u]; sv[u] = sn[u]; }
            }
            it = next;
        }
        __syncthreads();
        if (warp < RPB) {
            const int r = warp, rg = rg0 + r;
            auto slice_sum = [&](int rr) {
                float4 y = make_float4(0.f, 0.f, 0.f, 0.f);  // 0 + p0 + p1 + ... as on the CPU
                for (int sl = 0; sl < S; ++sl) {
                    const float4 o = s_part[(rr * S + sl) * 32 + lane];
                    y.x = y.x + o.x; y.y = y.y + o.y; y.z = y.z + o.z; y.w = y.w + o.w;
                }
                return y;
            };
            if (EPI == EPI_SWIGLU) {
                // Row groups alternate gate (even) / up (odd).
                if (!(r & 1) && rg < a.n_rg) {
                    const float4 gq = slice_sum(r), uq = slice_sum(r + 1);
                    const float gg[4] = {gq.x, gq.y, gq.z, gq.w}, uu[4] = {uq.x, uq.y, uq.z, uq.w};
                    const int feat = (rg >> 1) * kTileRows + 2 * t;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int row = g + (j >> 1) * 8;
                        if (row < T) {
                            const float sl = gg[j] / (1.0f + exact_expf(-gg[j]));
                            a.out[(size_t)row * a.ld + feat + (j & 1)] = sl * uu[j];
                        }
                    }
                }
            } else if (rg < a.n_rg) {
                const float4 yq = slice_sum(r);
                const float y[4] = {yq.x, yq.y, yq.z, yq.w};
                const int n0 = rg * kTileRows + 2 * t;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int row = g + (j >> 1) * 8;
                    const int col = n0 + (j & 1);
                    if (row >= T) continue;
                    if (EPI == EPI_STORE) a.out[(size_t)row * a.ld + col] = y[j];
                    if (EPI == EPI_RESID) {
                        float* o = a.out + (size_t)row * a.ld + col;
                        *o = *o + y[j];
                    }
                    if (EPI == EPI_ARGMAX) {
                        if (a.logits) a.logits[(size_t)row * a.ld + col] = y[j];
                        const int slot = j >> 1;
                        if (y[j] > best_v[slot] || (y[j] == best_v[slot] && col < best_i[slot])) {
                            best_v[slot] = y[j];
                            best_i[slot] = col;
                        }
                    }
                }
            }
        }
        __syncthreads();
    }
    if (EPI == EPI_ARGMAX) {
        // (value, first index) over the 4 lanes of a row group, then over the
        // RPB warps, then this CTA's partial per row.
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
        float2* cand = reinterpret_cast<float2*>(s_part);  // [RPB][16]
        if (warp < RPB && t == 0) {
            cand[warp * 16 + g] = make_float2(best_v[0], __int_as_float(best_i[0]));
            cand[warp * 16 + g + 8] = make_float2(best_v[1], __int_as_float(best_i[1]));
        }
        __syncthreads();
        if (threadIdx.x < 16) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int rr = 0; rr < RPB; ++rr) {
                const float2 c = cand[rr * 16 + threadIdx.x];
                const int ci = __float_as_int(c.y);
                if (c.x > bv || (c.x == bv && ci < bi)) { bv = c.x; bi = ci; }
            }
            a.lm_val[blockIdx.x * 16 + threadIdx.x] = make_float2(bv, __int_as_float(bi));
        }
    }
}

template <int EPI, int RPB>
void gemv(const GemvArgs& a, int grid, cudaStream_t s) {
    const int kb_n = a.kt_n * 2;
    const int S = a.kt_n / kSliceTiles;
    const size_t smem = (size_t)kb_n * 32 * 16 + (size_t)kb_n * 16 * 4 + (size_t)RPB * S * 32 * 16;
    k_gemv<EPI, RPB><<<grid, kThreads, smem, s>>>(a);
}

// ------------------------------------------------------------ norms, quant

// RMSNorm (double sum of float squares in the hidden-row tree of
// row_rms_scale, 1/sqrtf(mean+eps), (x*s)*w) of each of the 16 rows,
// quantised to the fragment order; rows >= T become zero.
// Optionally stores the normed f32 rows (final norm -> hidden).
__global__ void __launch_bounds__(kThreads) k_rmsnorm_quant(const StepState* st, const float* __restrict__ x, int K,
                                                            const float* __restrict__ w, float eps,
                                                            uint8_t* act_q, float* act_d, float* normed) {
    const int row = blockIdx.x;
    const int T = st->T;
    if (T <= 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ double s_q[kThreads];
    __shared__ float s_scale;
    const bool live = row < T;
    // The hidden-row tree (row_rms_scale); the block is uniform in `live`.
    const float scale = live ? row_rms_scale(x + (size_t)row * K, K, eps, s_q, &s_scale) : 0.f;
    for (int blk = warp; blk < K / 32; blk += kWarps) {
        const int i = blk * 32 + lane;
        float v = 0.f;
        if (live) {
            v = __fmul_rn(__fmul_rn(x[(size_t)row * K + i], scale), w[i]);
            if (normed) normed[(size_t)row * K + i] = v;
        }
        quantize_block_lane(v, row, blk, act_q, act_d);
    }
}

// Plain quantisation of f32 rows [16][K] (rows >= T -> zero).
__global__ void __launch_bounds__(kThreads) k_quant_rows(const StepState* st, const float* __restrict__ x, int K,
                                                         uint8_t* act_q, float* act_d) {
    const int T = st->T;
    if (T <= 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = K / 32;
    for (int item = blockIdx.x * kWarps + warp; item < nb * kTMax; item += gridDim.x * kWarps) {
        const int row = item / nb, blk = item % nb;
        const float v = row < T ? x[(size_t)row * K + blk * 32 + lane] : 0.f;
        quantize_block_lane(v, row, blk, act_q, act_d);
    }
}

// Per-head RMSNorm + NEOX RoPE of q and k (src/qwen3.cpp:104-118), then the
// KV store of k and v at positions before+t (src/qwen3.cpp:123-140).
// grid (rows, n_heads + n_kv), block 128; T_arg < 0: T and before from the
// step state, else the prefill pass's rows at positions before_arg + t.
__global__ void __launch_bounds__(128) k_qk_norm_rope_store(const StepState* st, float* qkv, int n_heads, int n_kv,
                                                            const float* __restrict__ q_norm,
                                                            const float* __restrict__ k_norm, float eps,
                                                            float theta_scale, KvCache kv, int layer, int T_arg,
                                                            int before_arg) {
    pdl_wait();
    pdl_launch_dependents();
    const int T = T_arg < 0 ? st->T : T_arg;
    const int row = blockIdx.x, hh = blockIdx.y;
    if (row >= T) return;
    const int pos = (T_arg < 0 ? st->before : before_arg) + row;
    const int ld = (n_heads + 2 * n_kv) * kHeadDim;
    const bool is_q = hh < n_heads;
    float* src = qkv + (size_t)row * ld + (size_t)hh * kHeadDim;
    const float* w = is_q ? q_norm : k_norm;
    const int d = threadIdx.x;
    __shared__ float s_sq[kHeadDim];
    __shared__ double s_tot;
    __shared__ float s_y[kHeadDim];
    const float xv = src[d];
    // Sum of squares, the per-head tree: lane i of warp 0 adds the squares of
    // elements i, i + 32, i + 64, i + 96 in that order in double, then one xor
    // butterfly over the 32 lanes.
    s_sq[d] = xv * xv;
    __syncthreads();
    if (d < 32) {
        double p = 0.0;
#pragma unroll
        for (int q = 0; q < 4; ++q) p += (double)s_sq[d + 32 * q];
        p = warp_sum_d(p);
        if (d == 0) s_tot = p;
    }
    __syncthreads();
    const double tot = s_tot;
    const float mean = (float)(tot / kHeadDim);
    const float scale = 1.0f / sqrtf(mean + eps);
    s_y[d] = __fmul_rn(__fmul_rn(xv, scale), w[d]);
    __syncthreads();
    if (d < kHeadDim / 2) {
        float theta = (float)pos;
        for (int i = 0; i < d; ++i) theta = __fmul_rn(theta, theta_scale);
        float s, c;
        exact_sincosf(theta, &s, &c);
        const float x0 = s_y[d], x1 = s_y[d + kHeadDim / 2];
        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        if (is_q) {
            src[d] = y0;
            src[d + kHeadDim / 2] = y1;
        } else {
            const int head = hh - n_heads;
            const long long off = kv_offset(kv, n_kv, layer, 0, head, pos);
            kv_store(kv, off + d, y0);
            kv_store(kv, off + d + kHeadDim / 2, y1);
        }
    }
    if (!is_q) {
        const int head = hh - n_heads;
        const float vv = qkv[(size_t)row * ld + (size_t)(n_heads + n_kv + head) * kHeadDim + d];
        kv_store(kv, kv_offset(kv, n_kv, layer, 1, head, pos) + d, vv);
    }
}

// ------------------------------------------------------------ attention

// 16-byte chunks r[u] (chunk tid + 256 u of n16) of a chunk's contiguous K or
// V rows [n_pos][128] (fp16 or f32) -> f32 rows [64][129] in shared memory.
__device__ __forceinline__ void kv_rows_to_smem(const uint4 (&r)[8], int n16, bool f16, float* dst) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int i = threadIdx.x + u * kThreads;
        if (i >= n16) continue;
        if (f16) {
            const __half* hv = reinterpret_cast<const __half*>(&r[u]);
            const int e0 = i * 8, p = e0 / kHeadDim, d0 = e0 % kHeadDim;
#pragma unroll
            for (int e = 0; e < 8; ++e) dst[p * (kHeadDim + 1) + d0 + e] = __half2float(hv[e]);
        } else {
            const float* fv = reinterpret_cast<const float*>(&r[u]);
            const int e0 = i * 4, p = e0 / kHeadDim, d0 = e0 % kHeadDim;
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[p * (kHeadDim + 1) + d0 + e] = fv[e];
        }
    }
}

// Scores of k_attn_chunk: thread (position p, row group qg) forms rows qg,
// qg + 4, ... (at most NR of them) at p, so each K element loaded once feeds
// every row and the q rows are warp-uniform broadcast reads (16 bytes = two
// dim pairs).  Per row: the even-dim and odd-dim fmaf chains in dim order,
// then (even + odd) x scale; masked positions -inf.
template <int NR>
__device__ __forceinline__ void attn_scores(const float* sq, const float* sk, float* sp, int NQ, int G, int n_pos,
                                            int p0, int before, float scale) {
    static_assert(kThreads == 256 && kPage == 64 && kHeadDim == 128, "thread roles");
    const int p = threadIdx.x & (kPage - 1), qg = threadIdx.x >> 6;
    const int nr = (NQ - qg + 3) >> 2;
    float ae[NR], ao[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) ae[r] = ao[r] = 0.f;
    if (p < n_pos) {
        const float* ka = sk + p * (kHeadDim + 1);
#pragma unroll 2
        for (int d = 0; d < kHeadDim; d += 4) {
            const float k0 = ka[d], k1 = ka[d + 1], k2 = ka[d + 2], k3 = ka[d + 3];
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                if (r < nr) {
                    const float4 qq = *reinterpret_cast<const float4*>(sq + (qg + 4 * r) * kHeadDim + d);
                    ae[r] = fmaf(qq.x, k0, ae[r]);
                    ao[r] = fmaf(qq.y, k1, ao[r]);
                    ae[r] = fmaf(qq.z, k2, ae[r]);
                    ao[r] = fmaf(qq.w, k3, ao[r]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        if (r < nr) {
            const int q = qg + 4 * r, t = q / G;
            const bool live = p < n_pos && p0 + p < before + t + 1;
            sp[q * kPage + p] = live ? (ae[r] + ao[r]) * scale : -INFINITY;
        }
    }
}

// P.V of k_attn_chunk: thread (dim d, row group qg) accumulates rows qg,
// qg + 2, ... (at most NR): each V element loaded once feeds every row, four
// probabilities per 16-byte broadcast read; each row's chain runs over the
// positions in order.  po: this (kv head, chunk)'s partial rows [q][128].
template <int NR>
__device__ __forceinline__ void attn_pv(const float* sk, const float* sp, int NQ, int n_pos, float* po) {
    const int d = threadIdx.x & (kHeadDim - 1), qg = threadIdx.x >> 7;
    const int nr = (NQ - qg + 1) >> 1;
    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.f;
    const float* vd = sk + d;
    int p = 0;
    for (; p + 4 <= n_pos; p += 4) {
        const float v0 = vd[p * (kHeadDim + 1)], v1 = vd[(p + 1) * (kHeadDim + 1)];
        const float v2 = vd[(p + 2) * (kHeadDim + 1)], v3 = vd[(p + 3) * (kHeadDim + 1)];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if (r < nr) {
                const float4 pp = *reinterpret_cast<const float4*>(sp + (qg + 2 * r) * kPage + p);
                acc[r] = fmaf(pp.x, v0, acc[r]);
                acc[r] = fmaf(pp.y, v1, acc[r]);
                acc[r] = fmaf(pp.z, v2, acc[r]);
                acc[r] = fmaf(pp.w, v3, acc[r]);
            }
        }
    }
    for (; p < n_pos; ++p) {
        const float v0 = vd[p * (kHeadDim + 1)];
#pragma unroll
        for (int r = 0; r < NR; ++r)
            if (r < nr) acc[r] = fmaf(sp[(qg + 2 * r) * kPage + p], v0, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < NR; ++r)
        if (r < nr) po[(size_t)(qg + 2 * r) * kHeadDim + d] = acc[r];
}

// Split-KV causal GQA attention, one CTA per (64-position chunk, kv head):
// scores q.k * 1/sqrt(128) (q.k = even-dim fmaf chain + odd-dim fmaf chain), query row t sees positions < before + t + 1
// (src/qwen3_decoder.cpp:142-148), chunk-local max / exp-sum / P.V partials.
// T_arg < 0: the step's rows (state); else a prefill pass of T_arg rows at
// before_arg.., split into row blocks of 16 (blockIdx.z), each with its own
// partial buffers (qstride rows per (head, chunk)).
__global__ void __launch_bounds__(kThreads) k_attn_chunk(const StepState* st, const float* __restrict__ qkv, int n_heads,
                                                         int n_kv, KvCache kv, int layer, float* part_o,
                                                         float2* part_ml, int max_chunks, int T_arg, int before_arg,
                                                         int qstride) {
    pdl_wait();
    pdl_launch_dependents();
    const int rb = blockIdx.z;
    const int T_all = T_arg < 0 ? st->T : T_arg;
    const int T = min(kTMax, T_all - kTMax * rb);
    if (T <= 0) return;
    const int before = (T_arg < 0 ? st->before : before_arg) + kTMax * rb;
    const int kv_len = before + T;
    const int c = blockIdx.x, h = blockIdx.y;
    if (c * kPage >= kv_len) return;
    if (!bc_check((kv_len + kPage - 1) / kPage <= max_chunks, BC_PARTIALS)) return;
    const int G = n_heads / n_kv;
    const int NQ = T * G;
    const int ld = (n_heads + 2 * n_kv) * kHeadDim;
    qkv += (size_t)kTMax * rb * ld;
    part_o += (size_t)rb * n_kv * max_chunks * qstride * kHeadDim;
    part_ml += (size_t)rb * n_kv * max_chunks * qstride;
    extern __shared__ __align__(16) float sm[];
    float* sq = sm;                              // [NQ][128]
    float* sk = sq + kTMax * 4 * kHeadDim;       // [64][129]  (group <= 4)
    float* sp = sk + kPage * (kHeadDim + 1);     // [NQ][64]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int p0 = c * kPage;
    const int n_pos = min(kPage, kv_len - p0);
    // The chunk's K and V rows are contiguous in their page: all of both are
    // requested up front as 16-byte loads (V waits in registers until the
    // scores are done), so the block pays one memory round trip, not one per
    // loop trip.
    const bool f16 = kv.type == KV_F16;
    const int elem = f16 ? 2 : 4;
    const int n16 = n_pos * kHeadDim * elem / 16;
    const uint4* kg = reinterpret_cast<const uint4*>(static_cast<const char*>(kv.base) +
                                                     kv_offset(kv, n_kv, layer, 0, h, p0) * elem);
    const uint4* vg = reinterpret_cast<const uint4*>(static_cast<const char*>(kv.base) +
                                                     kv_offset(kv, n_kv, layer, 1, h, p0) * elem);
    uint4 kr[8], vr[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int i = tid + u * kThreads;
        if (i < n16) {
            kr[u] = kg[i];
            vr[u] = vg[i];
        }
    }
    for (int i = tid; i < NQ * kHeadDim / 4; i += kThreads) {
        const int q = i / (kHeadDim / 4), d = (i % (kHeadDim / 4)) * 4;
        const int t = q / G, j = q % G;
        *reinterpret_cast<float4*>(sq + q * kHeadDim + d) =
            *reinterpret_cast<const float4*>(qkv + (size_t)t * ld + (size_t)(h * G + j) * kHeadDim + d);
    }
    kv_rows_to_smem(kr, n16, f16, sk);
    __syncthreads();
    const float scale = 1.0f / sqrtf((float)kHeadDim);
    {
        const int ns = (NQ + 3) >> 2;  // rows per score thread (at most)
        if (ns <= 1) attn_scores<1>(sq, sk, sp, NQ, G, n_pos, p0, before, scale);
        else if (ns <= 2) attn_scores<2>(sq, sk, sp, NQ, G, n_pos, p0, before, scale);
        else if (ns <= 4) attn_scores<4>(sq, sk, sp, NQ, G, n_pos, p0, before, scale);
        else if (ns <= 8) attn_scores<8>(sq, sk, sp, NQ, G, n_pos, p0, before, scale);
        else attn_scores<16>(sq, sk, sp, NQ, G, n_pos, p0, before, scale);
    }
    __syncthreads();
    for (int q = warp; q < NQ; q += kWarps) {
        const float a0 = sp[q * kPage + lane], a1 = sp[q * kPage + lane + 32];
        const float m = warp_max(fmaxf(a0, a1));
        const float e0 = a0 == -INFINITY ? 0.f : exact_expf(a0 - m);
        const float e1 = a1 == -INFINITY ? 0.f : exact_expf(a1 - m);
        const float l = warp_sum(e0 + e1);
        sp[q * kPage + lane] = e0;
        sp[q * kPage + lane + 32] = e1;
        if (lane == 0) part_ml[((size_t)h * max_chunks + c) * qstride + q] = make_float2(m, l);
    }
    kv_rows_to_smem(vr, n16, f16, sk);  // the K rows are no longer read: the scores are in sp
    __syncthreads();
    float* po = part_o + ((size_t)h * max_chunks + c) * qstride * kHeadDim;
    const int npv = (NQ + 1) >> 1;  // rows per P.V thread (at most)
    if (npv <= 1) attn_pv<1>(sk, sp, NQ, n_pos, po);
    else if (npv <= 2) attn_pv<2>(sk, sp, NQ, n_pos, po);
    else if (npv <= 4) attn_pv<4>(sk, sp, NQ, n_pos, po);
    else if (npv <= 8) attn_pv<8>(sk, sp, NQ, n_pos, po);
    else if (npv <= 16) attn_pv<16>(sk, sp, NQ, n_pos, po);
    else attn_pv<32>(sk, sp, NQ, n_pos, po);
}

// Prefill attention, register-blocked: one (64-position chunk c, kv head h,
// 64-token tile) per block of 256 threads, the tile's 128 query rows (group 2)
// against the chunk's K/V rows.  Each thread forms an 8-row x 4-position score
// tile (rows 8 rg .. 8 rg + 7, positions pg + 16 i) and later an 8-row x 8-dim
// output tile (dims 2 dg + 32 i, + 1), so every shared-memory load feeds 4 to 8
// FMAs instead of one.  Each score and each output is the same chain in the
// same order as k_attn_chunk (even/odd dim chains, then their sum x scale; P.V
// one chain over the row block's positions), and the partials go to the same
// places (row blocks of 16 tokens), so k_attn_combine and the results are
// unchanged bit for bit.  The chunk softmax runs on the score registers: the
// 16 threads of a row group hold a row's 64 positions as k_attn_chunk's lanes
// pg and pg + 16 would (positions pg, pg + 32 and pg + 16, pg + 48), so the pair
// sums, the first butterfly level (within the thread) and the other four
// (xor 8, 4, 2, 1 across the 16 threads) add the same values in the same order.
// The exp weights then overwrite the q rows (done with), which keeps a block at
// ~100 KB of shared memory and two blocks per SM.  Row strides are padded for
// conflict-free 8-byte reads.
constexpr int kPfTok = 64;               // tokens per tile
constexpr int kPfRows = 2 * kPfTok;      // query rows per tile (group 2)
constexpr int kPfQS = kHeadDim + 2;      // q / K / V row stride (floats)
constexpr int kPfWS = kPage + 1;         // weight row stride (float2): rows of weights fit in the q rows
static_assert(kPfWS * 2 <= kPfQS, "weights reuse the q rows");
constexpr size_t kPfAttnSmem = (size_t)(kPfRows * kPfQS + kPage * kPfQS) * 4;

__global__ void __launch_bounds__(256, 2) k_pf_attn(const float* __restrict__ qkv, int n_heads, int n_kv, KvCache kv,
                                                   int layer, float* part_o, float2* part_ml, int max_chunks, int P,
                                                   int before, int qstride) {
    const int c = blockIdx.x, h = blockIdx.y, tile = blockIdx.z;
    const int t0 = tile * kPfTok;                     // first token of the tile (pass-relative)
    const int n_tok = min(kPfTok, P - t0);
    const int p0 = c * kPage;
    if (n_tok <= 0 || p0 > before + t0 + n_tok - 1) return;  // no row of the tile reaches this chunk
    const int G = 2, ld = (n_heads + 2 * n_kv) * kHeadDim;
    extern __shared__ __align__(16) float sm[];
    float* sq = sm;                                   // [128][130] query rows, then the exp weights
    float* skv = sq + kPfRows * kPfQS;                // [64][130] K, then V
    float2* sw = reinterpret_cast<float2*>(sq);       // [128][65] exp weights, doubled (over the q rows)
    const int tid = threadIdx.x;
    // Staging: every load of a batch is issued before the first store.
    // q rows: 4096 float4, 16 per thread in two batches.
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + 256 * (8 * b + u), r = i >> 5, d4 = i & 31, t = r / G, j = r % G;
            v[u] = t < n_tok ? __ldcg(reinterpret_cast<const float4*>(qkv + (size_t)(t0 + t) * ld +
                                                                      (size_t)(h * G + j) * kHeadDim) + d4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + 256 * (8 * b + u), r = i >> 5, d4 = i & 31;
            float* dst = sq + r * kPfQS + 4 * d4;
            *reinterpret_cast<float2*>(dst) = make_float2(v[u].x, v[u].y);
            *reinterpret_cast<float2*>(dst + 2) = make_float2(v[u].z, v[u].w);
        }
    }
    // K rows (64 x 128 contiguous elements): 16-byte loads, converted to f32.
    const long long koff = kv_offset(kv, n_kv, layer, 0, h, p0);
    const long long voff = kv_offset(kv, n_kv, layer, 1, h, p0);
    const bool f16 = kv.type == KV_F16;
    auto stage = [&](long long off) {
        constexpr int kU = kPage * kHeadDim * 4 / 16 / 256;  // 16-byte f32 units per thread (8); fp16 uses half
        const int nu = f16 ? kU / 2 : kU;
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(kv.base) + off * (f16 ? 2 : 4));
        uint4 reg[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (u < nu) reg[u] = __ldcg(src + tid + 256 * u);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (u >= nu) continue;
            const int e0 = (tid + 256 * u) * (f16 ? 8 : 4);  // first element of the unit
            float* dst = skv + (e0 / kHeadDim) * kPfQS + e0 % kHeadDim;
            if (f16) {
                const __half2* hh = reinterpret_cast<const __half2*>(&reg[u]);
#pragma unroll
                for (int q = 0; q < 4; ++q) *reinterpret_cast<float2*>(dst + 2 * q) = __half22float2(hh[q]);
            } else {
                *reinterpret_cast<float2*>(dst) = make_float2(__uint_as_float(reg[u].x), __uint_as_float(reg[u].y));
                *reinterpret_cast<float2*>(dst + 2) = make_float2(__uint_as_float(reg[u].z), __uint_as_float(reg[u].w));
            }
        }
    };
    stage(koff);
    __syncthreads();
    const int rg = tid >> 4, pg = tid & 15;
    float2 acc[8][4];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[r][i] = make_float2(0.f, 0.f);
    {
        const float* qb = sq + (rg * 8) * kPfQS;
        const float* kb = skv + pg * kPfQS;
#pragma unroll 2
        for (int d = 0; d < kHeadDim; d += 2) {
            float2 qv[8], kv4[4];
#pragma unroll
            for (int r = 0; r < 8; ++r) qv[r] = *reinterpret_cast<const float2*>(qb + r * kPfQS + d);
#pragma unroll
            for (int i = 0; i < 4; ++i) kv4[i] = *reinterpret_cast<const float2*>(kb + (16 * i) * kPfQS + d);
#pragma unroll
            for (int r = 0; r < 8; ++r)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[r][i] = __ffma2_rn(qv[r], kv4[i], acc[r][i]);
        }
    }
    __syncthreads();  // q and K rows are done with: the weights and V take their places
    stage(voff);
    {
        const float scale = 1.0f / sqrtf((float)kHeadDim);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int row = rg * 8 + r, t = row / G;  // tile-relative token
            float sc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int pp = pg + 16 * i;
                const bool ok = t < n_tok && p0 + pp <= before + t0 + t;
                sc[i] = ok ? __fmul_rn(__fadd_rn(acc[r][i].x, acc[r][i].y), scale) : -INFINITY;
            }
            float m = fmaxf(fmaxf(sc[0], sc[2]), fmaxf(sc[1], sc[3]));
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float e[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) e[i] = sc[i] == -INFINITY ? 0.f : exact_expf(sc[i] - m);
            // k_attn_chunk's lane pg holds positions pg, pg + 32; lane pg + 16 holds pg + 16, pg + 48.
            float l = (e[0] + e[2]) + (e[1] + e[3]);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
            for (int i = 0; i < 4; ++i) sw[row * kPfWS + pg + 16 * i] = make_float2(e[i], e[i]);
            const int sb = t / kTMax, rb = tile * (kPfTok / kTMax) + sb;
            const int kv_len = before + kTMax * rb + min(kTMax, P - kTMax * rb);
            if (pg == 0 && t < n_tok && p0 < kv_len)
                part_ml[((size_t)rb * n_kv + h) * max_chunks * qstride + (size_t)c * qstride + (t % kTMax) * G +
                        row % G] = make_float2(m, l);
        }
    }
    __syncthreads();
    // P.V: thread (rg, dg) = (tid / 16, tid % 16): rows 8 rg .. 8 rg + 7 (one row
    // block of 16 tokens), dims 2 dg + 32 i and + 1; positions up to the row
    // block's key count.
    {
        const int dg = pg;
        const int sb = (rg * 8 / G) / kTMax, rb = tile * (kPfTok / kTMax) + sb;
        const int T_rb = min(kTMax, P - kTMax * rb);
        if (T_rb > 0) {
            const int kv_len = before + kTMax * rb + T_rb;
            const int n_pos = min(kPage, kv_len - p0);
            float2 o[8][4];
#pragma unroll
            for (int r = 0; r < 8; ++r)
#pragma unroll
                for (int i = 0; i < 4; ++i) o[r][i] = make_float2(0.f, 0.f);
            const float* vb = skv + 2 * dg;
            const float2* wb = sw + (rg * 8) * kPfWS;
#pragma unroll 2
            for (int pp = 0; pp < n_pos; ++pp) {
                float2 v[4], w[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = *reinterpret_cast<const float2*>(vb + pp * kPfQS + 32 * i);
#pragma unroll
                for (int r = 0; r < 8; ++r) w[r] = wb[r * kPfWS + pp];
#pragma unroll
                for (int r = 0; r < 8; ++r)
#pragma unroll
                    for (int i = 0; i < 4; ++i) o[r][i] = __ffma2_rn(w[r], v[i], o[r][i]);
            }
            if (n_pos > 0) {
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const int row = rg * 8 + r, t = row / G;
                    if (t >= n_tok) continue;
                    float* dst = part_o + (((size_t)rb * n_kv + h) * max_chunks * qstride + (size_t)c * qstride +
                                           (t % kTMax) * G + row % G) * kHeadDim;
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        *reinterpret_cast<float2*>(dst + 2 * dg + 32 * i) = o[r][i];
                }
            }
        }
    }
}

// Merge the chunk partials of one (row, head): grid (rows, n_heads), block
// 128 (one output dim per thread); rows and partial buffers as in k_attn_chunk
// (row blocks of 16).  M = max over chunks; then, chunk by chunk in order,
// w = exp(m_c - M), L += w l_c, o += w o_c (one fmaf chain each, chunks with
// m_c = -inf skipped).  Chunks go in batches of 128: the batch's weights are
// formed in parallel (one chunk per thread) into shared memory and its
// partial loads are issued 16 at a time, so the chains wait on arithmetic,
// not on one load after another.  act_h (F16 models' step path, else null):
// the merged rows rounded to fp16 as well, rows >= T zero.
__global__ void __launch_bounds__(128) k_attn_combine(const StepState* st, int n_heads, int n_kv,
                                                      const float* part_o, const float2* part_ml, int max_chunks,
                                                      float* attn_out, int T_arg, int before_arg, int qstride,
                                                      __half* act_h) {
    pdl_wait();
    pdl_launch_dependents();
    const int T_all = T_arg < 0 ? st->T : T_arg;
    const int t_all = blockIdx.x, head = blockIdx.y;
    if (t_all >= T_all) {
        if (act_h) act_h[(size_t)t_all * n_heads * kHeadDim + (size_t)head * kHeadDim + threadIdx.x] = __float2half_rn(0.f);
        return;
    }
    const int rb = t_all / kTMax, t = t_all % kTMax;
    const int T = min(kTMax, T_all - kTMax * rb);
    const int G = n_heads / n_kv;
    const int h = head / G, q = t * G + head % G;
    const int kv_len = (T_arg < 0 ? st->before : before_arg) + kTMax * rb + T;
    const int n_chunks = (kv_len + kPage - 1) / kPage;
    part_o += (size_t)rb * n_kv * max_chunks * qstride * kHeadDim;
    part_ml += (size_t)rb * n_kv * max_chunks * qstride;
    const float2* ml = part_ml + (size_t)h * max_chunks * qstride + q;  // chunk c at ml[c * qstride]
    const float* po = part_o + ((size_t)h * max_chunks * qstride + q) * kHeadDim + threadIdx.x;
    const size_t so = (size_t)qstride * kHeadDim;                       // one chunk further in po
    __shared__ float s_red[4];
    __shared__ float2 s_wl[128];  // (w, l) of the batch's chunks; w < 0 marks a skipped chunk
    float M = -INFINITY;
    for (int c = threadIdx.x; c < n_chunks; c += 128) M = fmaxf(M, ml[(size_t)c * qstride].x);
    M = warp_max(M);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = M;
    __syncthreads();
    M = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
    float L = 0.f, o = 0.f;
    for (int c0 = 0; c0 < n_chunks; c0 += 128) {
        const int nb = min(128, n_chunks - c0);
        __syncthreads();  // the previous batch's weights are consumed
        if (threadIdx.x < nb) {
            const float2 v = ml[(size_t)(c0 + threadIdx.x) * qstride];
            s_wl[threadIdx.x] = v.x == -INFINITY ? make_float2(-1.f, 0.f) : make_float2(exact_expf(v.x - M), v.y);
        }
        __syncthreads();
        for (int u0 = 0; u0 < nb; u0 += 16) {
            float ov[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) ov[u] = u0 + u < nb ? __ldcg(po + (size_t)(c0 + u0 + u) * so) : 0.f;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                if (u0 + u < nb) {
                    const float2 wl = s_wl[u0 + u];
                    if (wl.x >= 0.f) {
                        L = fmaf(wl.x, wl.y, L);
                        o = fmaf(wl.x, ov[u], o);
                    }
                }
            }
        }
    }
    const float r = o / L;
    attn_out[(size_t)t_all * n_heads * kHeadDim + (size_t)head * kHeadDim + threadIdx.x] = r;
    if (act_h) act_h[(size_t)t_all * n_heads * kHeadDim + (size_t)head * kHeadDim + threadIdx.x] = __float2half_rn(r);
}

// ------------------------------------------------------------ embed, draft, accept

// q8_0 row dequant (d * q) of the step's tokens from the token_embd tiles
// (src/generate.cpp:33-66); rows >= T are zeroed.
__global__ void k_embed(StepState* st, const uint8_t* __restrict__ embd, int hidden, int vocab, float* x) {
    const int row = blockIdx.x;
    const int T = st->T;
    if (T <= 0) return;
    const int kt_n = hidden / kTileK;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float v = 0.f;
        if (row < T) {
            int id = st->tokens[row];
            if (id < 0 || id >= vocab) {  // ids are validated on the host; never read out of bounds
                if (i == 0) st->error = 1;
                id = 0;
            }
            const int rg = id / kTileRows, g = id % kTileRows;
            const int kt = i / kTileK, blk = (i % kTileK) / 32, cc = i % 32;
            const uint8_t* tile = embd + ((size_t)rg * kt_n + kt) * kTileBytes;
            const int t4 = (cc & 15) >> 2, part = cc >> 4;
            const int8_t q = (int8_t)tile[(g * 4 + t4) * 16 + blk * 8 + part * 4 + (cc & 3)];
            const unsigned short hb = *reinterpret_cast<const unsigned short*>(tile + 512 + ((g >> 1) * 4 + blk * 2 + (g & 1)) * 2);
            v = (float)q * __half2float(__ushort_as_half(hb));
        }
        x[(size_t)row * hidden + i] = v;
    }
}

// fuse_embeds on the device (src/generate.cpp:113-177): row p is the q8_0
// dequant (d * q) of token ids[p] from the token_embd tiles, or, where
// slot[p] >= 0 (the k-th audio placeholder, slots counted on the host), audio
// row slot[p].  grid (seq), block 256.
// F16 weights on the device, tiled for the GEMV's lane-per-output reads: the
// [n][k] matrix (n a multiple of 32) as tiles of 32 rows x 32 columns, tile
// (g, kb) at ((g * k/32) + kb) * 1024 halves, inside it column quarter u
// (8 columns) at u * 256, row o at o * 8, column e at e.  A warp reading one
// quarter of a tile for its 32 rows reads 512 contiguous bytes.
__host__ __device__ __forceinline__ size_t f16_tiled_index(size_t row, int col, int k) {
    return ((row >> 5) * (size_t)(k >> 5) + (size_t)(col >> 5)) * 1024 + (size_t)((col & 31) >> 3) * 256 +
           (row & 31) * 8 + (col & 7);
}

// Row-major [n][k] fp16 (src) -> tiled (dst); one thread per 8 columns.
__global__ void k_repack_f16(const uint4* __restrict__ src, int n, int k, __half* dst) {
    const size_t chunks = (size_t)n * (k >> 3);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < chunks; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / (k >> 3);
        const int col = (int)(i % (k >> 3)) * 8;
        *reinterpret_cast<uint4*>(dst + f16_tiled_index(row, col, k)) = src[i];
    }
}

__global__ void k_fuse_embeds_f16(const int32_t* __restrict__ ids, const int32_t* __restrict__ slot, int seq,
                                  const float* __restrict__ audio, const __half* __restrict__ embd, int hidden,
                                  float* out) {
    const int p = blockIdx.x;
    if (p >= seq) return;
    const int a = slot[p];
    for (int i = threadIdx.x; i < hidden; i += blockDim.x)
        out[(size_t)p * hidden + i] =
            a >= 0 ? audio[(size_t)a * hidden + i] : __half2float(embd[f16_tiled_index((size_t)ids[p], i, hidden)]);
}

__global__ void k_fuse_embeds(const int32_t* __restrict__ ids, const int32_t* __restrict__ slot, int seq,
                              const float* __restrict__ audio, const uint8_t* __restrict__ embd, int hidden,
                              float* out) {
    const int p = blockIdx.x;
    if (p >= seq) return;
    const int a = slot[p];
    const int kt_n = hidden / kTileK;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float v;
        if (a >= 0) {
            v = audio[(size_t)a * hidden + i];
        } else {
            const int id = ids[p];  // validated on the host
            const int rg = id / kTileRows, g = id % kTileRows;
            const int kt = i / kTileK, blk = (i % kTileK) / 32, cc = i % 32;
            const uint8_t* tile = embd + ((size_t)rg * kt_n + kt) * kTileBytes;
            const int t4 = (cc & 15) >> 2, part = cc >> 4;
            const int8_t q = (int8_t)tile[(g * 4 + t4) * 16 + blk * 8 + part * 4 + (cc & 3)];
            const unsigned short hb = *reinterpret_cast<const unsigned short*>(tile + 512 + ((g >> 1) * 4 + blk * 2 + (g & 1)) * 2);
            v = (float)q * __half2float(__ushort_as_half(hb));
        }
        out[(size_t)p * hidden + i] = v;
    }
}

// n-gram draft over the generated ids (src/cpu_speculative.cpp:27-38): the
// longest suffix size in [n_min, n_max] with an earlier occurrence, latest
// occurrence first.  For each end position e < n the common suffix length
// c(e) of ids[0:e] and ids[0:n] (capped at n_max) is computed; the answer is
// the largest c >= n_min, then the largest e with that c.  The proposal is
// ids[e : e + min(budget, n - e)].  Called by a whole CTA (blockDim % 32 == 0,
// <= 1024 threads); returns e (or -1) in every thread.
__device__ int draft_search(const int32_t* __restrict__ ids, int n, int budget, int n_min, int n_max) {
    __shared__ unsigned long long s_best[32];
    const int top = min(n_max, n - 1);
    unsigned long long best = 0;
    if (budget > 0 && n >= 2 && n >= n_min + 1 && top >= n_min) {
        for (int e = threadIdx.x + 1; e < n; e += blockDim.x) {
            int c = 0;
            while (c < top && c < e && ids[e - 1 - c] == ids[n - 1 - c]) ++c;
            if (c >= n_min) {
                const unsigned long long key = ((unsigned long long)c << 32) | (unsigned)e;
                best = key > best ? key : best;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
    __syncthreads();
    best = 0;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) best = s_best[i] > best ? s_best[i] : best;
    __syncthreads();
    return best ? (int)(best & 0xffffffffu) : -1;
}

__device__ __forceinline__ void draft_member(StepState* st, const int32_t* __restrict__ ids) {
    if (st->stop != STOP_NONE) {
        if (threadIdx.x == 0) st->T = 0;
        return;
    }
    const int n = st->n_ids;
    int budget = min(st->k_max, st->max_new - n);
    budget = max(min(budget, st->max_seq - st->past - 1), 0);
    const int e = draft_search(ids, n, budget, st->n_min, st->n_max);
    if (threadIdx.x == 0) {
        int np = 0;
        st->tokens[0] = st->seed;
        if (e >= 0) {
            np = min(budget, n - e);
            if (!bc_check(1 + np <= kTMax, BC_STEP_ROWS)) np = kTMax - 1;
            for (int i = 0; i < np; ++i) st->tokens[1 + i] = ids[e + i];
        }
        st->n_prop = np;
        st->T = 1 + np;
        st->before = st->past;
    }
}

__global__ void __launch_bounds__(256) k_draft(StepState* st, const int32_t* __restrict__ ids) { draft_member(st, ids); }

__global__ void __launch_bounds__(256) k_draft_group(DraftGroup g) { draft_member(g.st[blockIdx.x], g.ids[blockIdx.x]); }

__global__ void k_group_stopped(DraftGroup g, int* flag) {
    const int k = threadIdx.x;
    const bool stopped = k >= g.n || g.st[k]->stop != STOP_NONE;
    const unsigned all = __all_sync(0xffffffffu, stopped);
    if (k == 0) *flag = all ? 1 : 0;
}

// The same search on explicit arguments (mtb_ngram_draft).
__global__ void __launch_bounds__(256) k_draft_args(const int32_t* __restrict__ ids, int n, int maximum, int n_min,
                                                    int n_max, int32_t* out, int* n_out) {
    const int e = draft_search(ids, n, maximum, n_min, n_max);
    if (threadIdx.x == 0) {
        const int np = e >= 0 ? min(maximum, n - e) : 0;
        for (int i = 0; i < np; ++i) out[i] = ids[e + i];
        *n_out = np;
    }
}

// Host-forced proposal already in tokens[1..n_prop]: clamp to the budget.
__global__ void k_draft_forced(StepState* st) {
    if (st->stop != STOP_NONE) { st->T = 0; return; }
    int budget = min(st->k_max, st->max_new - st->n_ids);
    budget = max(min(budget, st->max_seq - st->past - 1), 0);
    st->n_prop = max(0, min(st->n_prop, budget));
    if (!bc_check(1 + st->n_prop <= kTMax, BC_STEP_ROWS)) st->n_prop = kTMax - 1;
    st->tokens[0] = st->seed;
    st->T = 1 + st->n_prop;
    st->before = st->past;
}

// First max over the CTA partials of the fused LM head, for rows < T.
__device__ void reduce_choices(StepState* st, const float2* lm_val, int lm_blocks) {
    const int T = st->T;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int row = warp; row < T; row += blockDim.x / 32) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int b = lane; b < lm_blocks; b += 32) {
            const float2 c = lm_val[b * 16 + row];
            const int ci = __float_as_int(c.y);
            if (c.x > bv || (c.x == bv && ci < bi)) { bv = c.x; bi = ci; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) st->choice[row] = bi == 0x7fffffff ? 0 : bi;
    }
}

// Strict acceptance and logical rollback (src/cpu_speculative.cpp:124-135),
// then the next seed (the choice of the last kept row, :119).
__global__ void k_accept(StepState* st, int32_t* ids, const float2* lm_val, int lm_blocks, int choices_ready) {
    if (st->T <= 0) return;
    if (!choices_ready) reduce_choices(st, lm_val, lm_blocks);
    __syncthreads();
    if (threadIdx.x != 0) return;
    accept_choices(st, ids);
}

// Seed after prefill: the choice of the last prefilled row, emitted.
__global__ void k_prefill_seed(StepState* st, int32_t* ids, const float2* lm_val, int lm_blocks, int choices_ready) {
    if (!choices_ready) reduce_choices(st, lm_val, lm_blocks);
    __syncthreads();
    if (threadIdx.x != 0) return;
    st->seed = st->choice[st->T - 1];
    emit_id(st, ids, st->seed);
}

// Penalised first max (src/cpu_speculative.cpp:39-50) of one logits row by a
// CTA of 1024 threads: the recent set is the last 100 of hist[0:n_hist] +
// extra[0:n_extra]; adjusted values x>0 ? x/p : x*p; the lowest index wins a
// tie (NaN entries never win).  `bits` is a dynamic shared bitmap of vocab bits.
__device__ int choice_block(const float* __restrict__ lr, int vocab, const int32_t* hist, int n_hist,
                            const int* extra, int n_extra, float p, unsigned int* bits) {
    const int words = (vocab + 31) / 32;
    for (int i = threadIdx.x; i < words; i += blockDim.x) bits[i] = 0;
    __syncthreads();
    const int len = n_hist + n_extra;
    if (p > 1.f)
        for (int i = max(0, len - 100) + threadIdx.x; i < len; i += blockDim.x) {
            const int id = i < n_hist ? hist[i] : extra[i - n_hist];
            if (id >= 0 && id < vocab) atomicOr(&bits[id >> 5], 1u << (id & 31));
        }
    __syncthreads();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        float v = lr[i];
        if ((bits[i >> 5] >> (i & 31)) & 1u) v = v > 0 ? v / p : v * p;
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
    __shared__ float s_v[32];
    __shared__ int s_i[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { s_v[threadIdx.x >> 5] = bv; s_i[threadIdx.x >> 5] = bi; }
    __syncthreads();
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) {
        const float ov = s_v[w];
        const int oi = s_i[w];
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    __syncthreads();
    // NaN never wins a strict '>' comparison; a NaN at index 0 keeps index 0.
    if (isnan(lr[0]) || bi == 0x7fffffff) return 0;
    return bi;
}

// Per verify row i: history = ids[0:n_ids] + proposals[0:i].  grid (kTMax).
__global__ void __launch_bounds__(1024) k_choice_penalty(StepState* st, const int32_t* ids, const float* logits,
                                                          int vocab) {
    extern __shared__ unsigned int bits[];
    const int T = st->T;
    const int row = blockIdx.x;
    if (row >= T) return;
    const int c = choice_block(logits + (size_t)row * vocab, vocab, ids, st->n_ids, st->tokens + 1, row,
                               st->penalty, bits);
    if (threadIdx.x == 0) st->choice[row] = c;
}

// mtb_greedy_choice on explicit arguments.
__global__ void __launch_bounds__(1024) k_choice_args(const float* logits, int n_raw, const int32_t* hist, int n_hist,
                                                      float p, int* out) {
    extern __shared__ unsigned int bits[];
    const int c = choice_block(logits, n_raw, hist, n_hist, nullptr, 0, p, bits);
    if (threadIdx.x == 0) *out = c;
}

// Proposal from device memory (asynchronous step API); ids are range-checked.
__global__ void k_set_forced(StepState* st, const int32_t* src, int n, int vocab) {
    for (int i = 0; i < n; ++i) {
        int id = src[i];
        if (id < 0 || id >= vocab) { st->error = 1; id = 0; }
        st->tokens[1 + i] = id;
    }
    st->n_prop = n;
}

// Step state for a standalone launch sequence: only T is read by the kernels.
__global__ void k_state_rows(StepState* st, int T) {
    StepState z = {};
    z.T = T;
    *st = z;
}

// First max of each row's LM-head partials, written to `out` (rows < T).
__global__ void k_reduce_choices_out(StepState* st, const float2* lm_val, int lm_blocks, int32_t* out) {
    reduce_choices(st, lm_val, lm_blocks);
    __syncthreads();
    if ((int)threadIdx.x < st->T) out[threadIdx.x] = st->choice[threadIdx.x];
}

// Host-supplied rows (prefill chunks, run()): positions before..before+T-1.
__global__ void k_rows_begin(StepState* st, int T) {
    st->before = st->past;
    st->T = T;
}
__global__ void k_rows_end(StepState* st) { st->past = st->before + st->T; }

// ------------------------------------------------------------ synthetic KV

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352du; x ^= x >> 15; x *= 0x846ca68bu; x ^= x >> 16;
    return x;
}

// Same values as the oracle's orc_synthetic_kv_value: Irwin-Hall(4) of a
// 32-bit hash, scaled to unit variance and rounded to fp16.
__device__ __forceinline__ float synthetic_kv_value(uint32_t seed, int layer, int which, int pos, int head, int dim) {
    uint32_t h = mix32(seed + 0x9E3779B9u * (uint32_t)(layer * 2 + which + 1));
    h = mix32(h ^ ((uint32_t)pos * 0x85EBCA6Bu));
    h = mix32(h ^ ((uint32_t)(head * 1024 + dim) * 0xC2B2AE35u));
    const uint32_t g = mix32(h ^ 0x68E31DA4u);
    const int s = (int)(h & 0xffffu) + (int)(h >> 16) + (int)(g & 0xffffu) + (int)(g >> 16) - 131070;
    return __half2float(__float2half_rn(__fmul_rn((float)s, 2.642912e-05f)));
}

__global__ void k_fill_synthetic_kv(KvCache kv, int n_layers, int n_kv, int n_pos, uint32_t seed) {
    const long long total = (long long)n_layers * 2 * n_kv * n_pos * kHeadDim;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int d = int(i % kHeadDim);
        long long r = i / kHeadDim;
        const int pos = int(r % n_pos); r /= n_pos;
        const int head = int(r % n_kv); r /= n_kv;
        const int which = int(r % 2);
        const int layer = int(r / 2);
        kv_store(kv, kv_offset(kv, n_kv, layer, which, head, pos) + d, synthetic_kv_value(seed, layer, which, pos, head, d));
    }
}

// Test hook: NaN into positions [pos0, pos0 + n_pos) of every layer, K and V,
// so that a step which read a cache slot it had not written would carry NaN.
__global__ void k_poison_kv(KvCache kv, int n_layers, int n_kv, int pos0, int n_pos) {
    const long long total = (long long)n_layers * 2 * n_kv * n_pos * kHeadDim;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int d = int(i % kHeadDim);
        long long r = i / kHeadDim;
        const int pos = pos0 + int(r % n_pos); r /= n_pos;
        const int head = int(r % n_kv); r /= n_kv;
        const int which = int(r % 2);
        const int layer = int(r / 2);
        kv_store(kv, kv_offset(kv, n_kv, layer, which, head, pos) + d, __int_as_float(0x7fc00000));
    }
}

__global__ void k_kv_gather(KvCache kv, int n_kv, int layer, int which, int pos0, int n_pos, float* out) {
    const long long total = (long long)n_pos * n_kv * kHeadDim;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int d = int(i % kHeadDim);
        const int head = int((i / kHeadDim) % n_kv);
        const int p = int(i / ((long long)kHeadDim * n_kv));
        out[i] = kv_load(kv, kv_offset(kv, n_kv, layer, which, head, pos0 + p) + d);
    }
}

}  // namespace

// ============================================================ launchers

void launch_repack_f16(const uint16_t* src, int n, int k, uint16_t* dst, cudaStream_t s) {
    k_repack_f16<<<g_sm_count * 8, 256, 0, s>>>(reinterpret_cast<const uint4*>(src), n, k, reinterpret_cast<__half*>(dst));
}

void launch_repack_q8(const uint8_t* src, int n_rows, int k, uint8_t* dst, int rg_stride, int rg_offset,
                      cudaStream_t s) {
    const long long work = (long long)(n_rows / kTileRows) * (k / kTileK) * 32;
    const int grid = (int)std::min<long long>((work + 255) / 256, 16LL * g_sm_count);
    k_repack_q8<<<grid, 256, 0, s>>>(src, n_rows, k, dst, rg_stride, rg_offset);
}

int lm_head_blocks(int vocab) {
    const int n_rg = vocab / kTileRows;
    return std::min(std::min(kLmHeadMaxBlocks, 4 * g_sm_count), (n_rg + 7) / 8);
}

static void configure_f16_kernels();

cudaError_t configure_kernels() {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    // Dynamic shared memory above 48 KB is opt-in per kernel (current device).
    cudaFuncSetAttribute(k_gemv<EPI_STORE, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k_gemv<EPI_RESID, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k_gemv<EPI_SWIGLU, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k_gemv<EPI_ARGMAX, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k_attn_chunk, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    cudaFuncSetAttribute(k_pf_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfAttnSmem);
    configure_f16_kernels();
    pf_configure();
    return cudaGetLastError();
}


// ------------------------------------------------------------ F16 weights
// Models with F16 weights (configs[2] of the benchmark) run the multi-kernel
// path with these kernels in place of the q8_0 ones.  ggml's mul_mat with an
// F16 src0 rounds the activations to fp16 and sums the exact fp16 x fp16
// products in f32; the order is the one shared with the CPU restatement
// (orc_mul_mat_f16): each 32-element block one fmaf chain from 0 in ascending
// order, the blocks of a 256-element slice added in ascending order, then the
// slices in ascending order.

// RMSNorm of rows < T (the tree of row_rms_scale) rounded to fp16 (rows >= T
// zero); `normed` (optional) gets the f32 rows.
__global__ void __launch_bounds__(kThreads) k_rmsnorm_f16(const StepState* st, const float* __restrict__ x, int K,
                                                         const float* __restrict__ w, float eps, __half* act,
                                                         float* normed) {
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.x;
    const int T = st->T;
    if (T <= 0) return;
    __shared__ double s_q[kThreads];
    __shared__ float s_scale;
    const bool live = row < T;
    // The hidden-row tree (row_rms_scale); the block is uniform in `live`.
    const float scale = live ? row_rms_scale(x + (size_t)row * K, K, eps, s_q, &s_scale) : 0.f;
    for (int i = threadIdx.x; i < K; i += kThreads) {
        float v = 0.f;
        if (live) {
            v = __fmul_rn(__fmul_rn(x[(size_t)row * K + i], scale), w[i]);
            if (normed) normed[(size_t)row * K + i] = v;
        }
        act[(size_t)row * K + i] = __float2half_rn(v);
    }
}

// Rows < T of f32 [16][K] rounded to fp16 (rows >= T zero).
__global__ void k_rows_f16(const StepState* st, const float* __restrict__ src, int K, __half* act) {
    const int T = st->T;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kTMax * K; i += gridDim.x * blockDim.x)
        act[i] = __float2half_rn(i / K < T ? src[i] : 0.f);
}

// Embedding rows of the step's tokens from fp16 token_embd (exact).
__global__ void k_embed_f16(StepState* st, const __half* __restrict__ embd, int hidden, int vocab, float* x) {
    const int row = blockIdx.x;
    const int T = st->T;
    if (T <= 0) return;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float v = 0.f;
        if (row < T) {
            int id = st->tokens[row];
            if (id < 0 || id >= vocab) {  // ids are validated on the host; never read out of bounds
                if (i == 0) st->error = 1;
                id = 0;
            }
            v = __half2float(embd[f16_tiled_index((size_t)id, i, hidden)]);
        }
        x[(size_t)row * hidden + i] = v;
    }
}

// y[t][o] = sum_k act[t][k] W[o][k], rows t < T.  One block of 256 threads
// takes 32 outputs (lane = output) and SPB (1, 2 or 4) consecutive
// 256-element slices of K; warp w takes the 32-element block w of each of those slices.  A lane
// loads its output's 32 weights of every block it takes up front (64 B per
// block, issued before the activations are staged so both latencies overlap),
// then runs each block's fmaf chain from 0 for the rows (1, 2, 4, 8 or 16 of
// them, the power of two at or above T; two rows per __ffma2_rn, each
// component its own chain) over the activations staged in shared memory as
// f32 [k][16] (broadcast reads).  The 8 block values of a
// slice meet in shared memory and thread (row, output) adds them in block
// order into the slice total.  With SPB equal to the slice count the block
// adds its slice totals in order and finishes; otherwise (split K: more blocks
// in flight for the narrow projections) each slice total goes to f16_part and
// the last block of the 32 outputs to finish (a counter per group, the
// fence-then-count pattern; no block waits for another) adds the totals of all
// slices in order.  Epilogues: store, residual add, SwiGLU into fp16 rows, or
// the first max over the 32 outputs per row (plus the logits when asked).
enum EpiF16 { F16_STORE = 0, F16_RESID = 1, F16_ARGMAX = 2, F16_SWIGLU = 3 };
constexpr int kF16MaxSpb = 4;  // slices per block when K is not split
constexpr int kF16Pad = 8;     // floats of padding after every 32 staged k (conflict-free staging)

__device__ __forceinline__ int f16_xs_idx(int k) { return k * kTMax + (k >> 5) * kF16Pad; }

template <int EPI>
__device__ __forceinline__ void f16_epilogue(float v, int t, int T, int o, int N, int g, float* out, int ld,
                                             float2* lm_val) {
    if (EPI == F16_ARGMAX) {
        float bv = (t < T && o < N) ? v : -INFINITY;
        int bi = (t < T && o < N) ? o : 0x7fffffff;
        if (out && t < T && o < N) out[(size_t)t * ld + o] = v;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if ((threadIdx.x & 31) == 0) lm_val[(size_t)g * kTMax + t] = make_float2(bv, __int_as_float(bi));
    } else if (EPI == F16_SWIGLU) {
        // Gate | up rows interleaved by 16 (upload): lanes 0-15 hold gate rows
        // 16 g .., lanes 16-31 the matching up rows.  out is the fp16 [16][ld]
        // activation of the down projection: silu(gate) * up (the q8_0
        // epilogue's expression), rows >= T zero.
        const float u = __shfl_down_sync(0xffffffffu, v, 16);
        const int i = g * 16 + (threadIdx.x & 31);
        if ((threadIdx.x & 31) < 16 && i < ld) {
            float r = 0.f;
            if (t < T) {
                const float sl = v / (1.0f + exact_expf(-v));
                r = sl * u;
            }
            reinterpret_cast<__half*>(out)[(size_t)t * ld + i] = __float2half_rn(r);
        }
    } else if (t < T && o < N) {
        if (EPI == F16_STORE) out[(size_t)t * ld + o] = v;
        else out[(size_t)t * ld + o] = out[(size_t)t * ld + o] + v;
    }
}

// Weights of block `warp` of each of the block's SPB slices for output o (W
// tiled; N is a multiple of 32, so every group's tiles exist).
template <int SPB>
__device__ __forceinline__ void f16_load_weights(const __half* __restrict__ W, int K, int g, int s0,
                                                 uint4 (&wr)[SPB][4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int si = 0; si < SPB; ++si) {
        // Tile (g, kb) of the tiled layout (f16_tiled_index): quarter u of
        // lane o's row is 16 bytes at u * 512 + o * 16, contiguous across lanes.
        const int kb = (s0 + si) * 8 + warp;
        const uint4* wp = reinterpret_cast<const uint4*>(W + ((size_t)g * (K >> 5) + kb) * 1024) + lane;
#pragma unroll
        for (int u = 0; u < 4; ++u) wr[si][u] = __ldg(wp + u * 32);
    }
}

template <int RB, int SPB, int EPI>
__device__ __forceinline__ void gemv_f16_body(int N, int K, int g, int s0, int nsb, int T, const uint4 (&wr)[SPB][4],
                                              const float* xs, float* bv, float* out, int ld, float2* lm_val,
                                              float* part, int* cnt) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int o = g * kF16Outs + lane;
    float tot[2] = {0.f, 0.f};  // rows warp, warp + 8 (this thread's share of the slice sums)
#pragma unroll
    for (int si = 0; si < SPB; ++si) {
        constexpr int NA = RB < 2 ? 1 : RB / 2;
        float2 acc[NA];
#pragma unroll
        for (int p = 0; p < NA; ++p) acc[p] = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float wj = __half2float(reinterpret_cast<const __half*>(wr[si])[j]);
            const float* xk = xs + f16_xs_idx(si * 256 + warp * 32 + j);
            if (RB == 1) {
                acc[0].x = fmaf(xk[0], wj, acc[0].x);
            } else if (RB == 2) {
                acc[0] = __ffma2_rn(*reinterpret_cast<const float2*>(xk), make_float2(wj, wj), acc[0]);
            } else {
                const float2 w2 = make_float2(wj, wj);
                const float4* xr = reinterpret_cast<const float4*>(xk);
#pragma unroll
                for (int q = 0; q < RB / 4; ++q) {
                    const float4 xv = xr[q];
                    acc[2 * q] = __ffma2_rn(make_float2(xv.x, xv.y), w2, acc[2 * q]);
                    acc[2 * q + 1] = __ffma2_rn(make_float2(xv.z, xv.w), w2, acc[2 * q + 1]);
                }
            }
        }
#pragma unroll
        for (int p = 0; p < NA; ++p) {
            bv[(warp * kTMax + 2 * p) * 32 + lane] = acc[p].x;
            if (RB > 1) bv[(warp * kTMax + 2 * p + 1) * 32 + lane] = acc[p].y;
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int t = warp + 8 * h;
            if (t < RB) {
                float a = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) a = a + bv[(i * kTMax + t) * 32 + lane];
                if (nsb == 1) tot[h] = tot[h] + a;
                else if (o < N) part[((size_t)(s0 + si) * kTMax + t) * N + o] = a;
            }
        }
        if (si + 1 < SPB) __syncthreads();
    }
    if (nsb > 1) {
        __shared__ int s_last;
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(&cnt[g], 1) == nsb - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        const int ns = K >> 8;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int t = warp + 8 * h;
            if (t < RB && o < N) {
                float a = 0.f;
                for (int s = 0; s < ns; ++s) a = a + __ldcg(&part[((size_t)s * kTMax + t) * N + o]);
                tot[h] = a;
            }
        }
        if (tid == 0) cnt[g] = 0;  // ready for the next launch
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) f16_epilogue<EPI>(tot[h], warp + 8 * h, T, o, N, g, out, ld, lm_val);
}

// grid: (N / 32) x (K / 256 / SPB) blocks, flattened; SPB (1, 2 or 4)
// divides the slice count.  SPB = 1 and 2 hold 16 and 32 weight registers (3
// blocks per SM), SPB = 4 holds 64 (2 blocks per SM).
template <int EPI, int SPB>
__global__ void __launch_bounds__(256, SPB == 4 ? 2 : 3)
    k_gemv_f16(const __half* __restrict__ W, int N, int K, const __half* __restrict__ act, const StepState* st,
               float* out, int ld, float2* lm_val, float* part, int* cnt) {
    extern __shared__ __align__(16) float sm_f16[];
    const int nsb = (K >> 8) / SPB;
    const int g = blockIdx.x / nsb, s0 = (blockIdx.x % nsb) * SPB;
    constexpr int kw = SPB * 256;
    // The weights do not depend on the step: they are requested before the
    // wait for the previous kernel (programmatic launch), so their HBM latency
    // overlaps that kernel's tail.
    uint4 wr[SPB][4];
    f16_load_weights<SPB>(W, K, g, s0, wr);
    pdl_wait();
    pdl_launch_dependents();
    const int T = st->T;
    if (T <= 0) return;
    float* xs = sm_f16;                                  // [kw][16] + padding
    float* bv = xs + kw * kTMax + (kw >> 5) * kF16Pad;  // [8 blocks][16 rows][32 outputs]
    const int RS = T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : T <= 8 ? 8 : kTMax;  // rows staged and computed
    // Stage rows < RS of act[:, s0*256 .. +kw) as f32: 8 halves per thread,
    // consecutive groups of RS threads in consecutive 32-k blocks.
    constexpr int nkb = kw >> 5;
    for (int i = threadIdx.x; i < RS * (kw >> 3); i += blockDim.x) {
        const int t = i % RS, q8 = i / RS;
        const int k0 = (q8 % nkb) * 32 + (q8 / nkb) * 8;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(act + (size_t)t * K + (size_t)s0 * 256 + k0));
        const __half* hv = reinterpret_cast<const __half*>(&v);
        float* dst = xs + f16_xs_idx(k0) + t;
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[e * kTMax] = __half2float(hv[e]);
    }
    __syncthreads();
    switch (RS) {
        case 1: gemv_f16_body<1, SPB, EPI>(N, K, g, s0, nsb, T, wr, xs, bv, out, ld, lm_val, part, cnt); break;
        case 2: gemv_f16_body<2, SPB, EPI>(N, K, g, s0, nsb, T, wr, xs, bv, out, ld, lm_val, part, cnt); break;
        case 4: gemv_f16_body<4, SPB, EPI>(N, K, g, s0, nsb, T, wr, xs, bv, out, ld, lm_val, part, cnt); break;
        case 8: gemv_f16_body<8, SPB, EPI>(N, K, g, s0, nsb, T, wr, xs, bv, out, ld, lm_val, part, cnt); break;
        default: gemv_f16_body<kTMax, SPB, EPI>(N, K, g, s0, nsb, T, wr, xs, bv, out, ld, lm_val, part, cnt);
    }
}

static size_t gemv_f16_smem(int spb) {
    const int kw = spb * 256;
    return ((size_t)kw * kTMax + (kw >> 5) * kF16Pad + 8 * kTMax * 32) * sizeof(float);
}

// Slices per block: the most of 4, 2, 1 (dividing K / 256) that still gives
// at least two blocks per SM; measured on the Qwen3-0.6B F16 step, more and
// shorter blocks beat fewer, longer ones until the grid fills the GPU twice.
int f16_spb(int N, int K) {
    const int ns = K >> 8, groups = (N + kF16Outs - 1) / kF16Outs;
    for (int spb : {kF16MaxSpb, 2})
        if (ns % spb == 0 && groups * (ns / spb) >= 2 * g_sm_count) return spb;
    return 1;
}

size_t f16_part_floats(const ModelDims& d) {
    const int H = d.hidden, F = d.ffn, qd = d.n_heads * kHeadDim, kd = d.n_kv * kHeadDim;
    const int shapes[5][2] = {{qd + 2 * kd, H}, {H, qd}, {2 * F, H}, {H, F}, {d.vocab, H}};
    size_t m = 0;
    for (const auto& sh : shapes)
        if (f16_spb(sh[0], sh[1]) < (sh[1] >> 8)) m = std::max(m, (size_t)(sh[1] >> 8) * kTMax * (size_t)sh[0]);
    return std::max<size_t>(m, 1);
}

int f16_groups_max(const ModelDims& d) {
    const int n = std::max(std::max(d.n_heads * kHeadDim + 2 * d.n_kv * kHeadDim, d.hidden), std::max(2 * d.ffn, d.vocab));
    return (n + kF16Outs - 1) / kF16Outs;
}

template <int SPB>
static void configure_f16_spb() {
    const int smem = (int)gemv_f16_smem(SPB);
    cudaFuncSetAttribute(k_gemv_f16<F16_STORE, SPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_gemv_f16<F16_RESID, SPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_gemv_f16<F16_ARGMAX, SPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_gemv_f16<F16_SWIGLU, SPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

static void configure_f16_kernels() {
    configure_f16_spb<1>();
    configure_f16_spb<2>();
    configure_f16_spb<kF16MaxSpb>();
}

// Launch with programmatic stream serialization (the F16 step's kernels, each
// of which calls pdl_wait() before touching step data): the next kernel's
// launch and weight loads overlap the current one's tail.  MTB_NO_PDL=1 at the
// first launch turns it off (ordinary stream order).
static bool pdl_enabled() {
    static const bool on = !std::getenv("MTB_NO_PDL");
    return on;
}

template <typename... KArgs, typename... Args>
static void launch_chain(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <int EPI>
static void gemv_f16(const uint16_t* W, int N, int K, const uint16_t* act, const StepBuffers& b, float* out, int ld,
                     float2* lm_val, cudaStream_t s) {
    const int spb = f16_spb(N, K);
    const int blocks = (N + kF16Outs - 1) / kF16Outs * ((K >> 8) / spb);
    const __half* w = reinterpret_cast<const __half*>(W);
    const __half* a = reinterpret_cast<const __half*>(act);
    const StepState* st = b.state;
    if (spb == kF16MaxSpb)
        launch_chain(k_gemv_f16<EPI, kF16MaxSpb>, blocks, 256, gemv_f16_smem(spb), s, w, N, K, a, st, out, ld, lm_val,
                     b.f16_part, b.f16_cnt);
    else if (spb == 2)
        launch_chain(k_gemv_f16<EPI, 2>, blocks, 256, gemv_f16_smem(2), s, w, N, K, a, st, out, ld, lm_val, b.f16_part,
                     b.f16_cnt);
    else
        launch_chain(k_gemv_f16<EPI, 1>, blocks, 256, gemv_f16_smem(1), s, w, N, K, a, st, out, ld, lm_val, b.f16_part,
                     b.f16_cnt);
}

// forward_layers for F16 weights: the same sequence with fp16 activations.
static void forward_layers_f16(const DeviceModel& m, const KvCache& kv, const StepBuffers& b, cudaStream_t s) {
    const ModelDims& d = m.dims;
    const int H = d.hidden, F = d.ffn;
    const int qd = d.n_heads * kHeadDim, kd = d.n_kv * kHeadDim;
    const size_t attn_smem = (size_t)(kTMax * 4 * kHeadDim + kPage * (kHeadDim + 1) + kTMax * 4 * kPage) * sizeof(float);
    __half* act = reinterpret_cast<__half*>(b.act_h);
    for (int l = 0; l < d.n_layers; ++l) {
        const LayerWeights& w = m.layers[l];
        launch_chain(k_rmsnorm_f16, kTMax, kThreads, 0, s, b.state, b.x, H, w.attn_norm, d.eps, act, (float*)nullptr);
        gemv_f16<F16_STORE>(w.h_qkv, qd + 2 * kd, H, b.act_h, b, b.qkv, qd + 2 * kd, nullptr, s);
        launch_chain(k_qk_norm_rope_store, dim3(kTMax, d.n_heads + d.n_kv), 128, 0, s, b.state, b.qkv, d.n_heads, d.n_kv,
                     w.q_norm, w.k_norm, d.eps, m.theta_scale, kv, l, -1, 0);
        launch_chain(k_attn_chunk, dim3(b.max_chunks, d.n_kv), kThreads, attn_smem, s, b.state, b.qkv, d.n_heads, d.n_kv,
                     kv, l, b.part_o, b.part_ml, b.max_chunks, -1, 0, kTMax * 4);
        launch_chain(k_attn_combine, dim3(kTMax, d.n_heads), 128, 0, s, b.state, d.n_heads, d.n_kv, b.part_o, b.part_ml,
                     b.max_chunks, b.attn_out, -1, 0, kTMax * 4, act);
        gemv_f16<F16_RESID>(w.h_o, H, qd, b.act_h, b, b.x, H, nullptr, s);
        launch_chain(k_rmsnorm_f16, kTMax, kThreads, 0, s, b.state, b.x, H, w.ffn_norm, d.eps, act, (float*)nullptr);
        // SwiGLU in the gate | up GEMV's epilogue, into act_h2 (act_h is its input).
        gemv_f16<F16_SWIGLU>(w.h_gu, 2 * F, H, b.act_h, b, reinterpret_cast<float*>(b.act_h2), F, nullptr, s);
        gemv_f16<F16_RESID>(w.h_down, H, F, b.act_h2, b, b.x, H, nullptr, s);
    }
    launch_chain(k_rmsnorm_f16, kTMax, kThreads, 0, s, b.state, b.x, H, m.output_norm, d.eps, act, b.hid);
}

static void lm_head_f16(const DeviceModel& m, const StepBuffers& b, bool want_logits, cudaStream_t s) {
    gemv_f16<F16_ARGMAX>(m.h_embd, m.dims.vocab, m.dims.hidden, b.act_h, b, want_logits ? b.logits : nullptr,
                         m.dims.vocab, b.lm_val, s);
}

// Layers, final norm and (optionally) the LM head for the rows in b.x.
static void forward_layers(const DeviceModel& m, const KvCache& kv, const StepBuffers& b, cudaStream_t s) {
    if (m.f16) {
        forward_layers_f16(m, kv, b, s);
        return;
    }
    const ModelDims& d = m.dims;
    const int H = d.hidden, F = d.ffn;
    const int qd = d.n_heads * kHeadDim, kd = d.n_kv * kHeadDim;
    const int G = d.n_heads / d.n_kv;
    const size_t attn_smem = (size_t)(kTMax * 4 * kHeadDim + kPage * (kHeadDim + 1) + kTMax * 4 * kPage) * sizeof(float);
    for (int l = 0; l < d.n_layers; ++l) {
        const LayerWeights& w = m.layers[l];
        k_rmsnorm_quant<<<kTMax, kThreads, 0, s>>>(b.state, b.x, H, w.attn_norm, d.eps, b.act_q, b.act_d, nullptr);
        {
            GemvArgs a{w.qkv, (qd + 2 * kd) / kTileRows, H / kTileK, b.act_q, b.act_d, b.qkv, qd + 2 * kd, b.state, nullptr, nullptr};
            gemv<EPI_STORE, 2>(a, (a.n_rg + 1) / 2, s);
        }
        k_qk_norm_rope_store<<<dim3(kTMax, d.n_heads + d.n_kv), 128, 0, s>>>(b.state, b.qkv, d.n_heads, d.n_kv, w.q_norm,
                                                                             w.k_norm, d.eps, m.theta_scale, kv, l, -1, 0);
        k_attn_chunk<<<dim3(b.max_chunks, d.n_kv), kThreads, attn_smem, s>>>(b.state, b.qkv, d.n_heads, d.n_kv, kv, l,
                                                                              b.part_o, b.part_ml, b.max_chunks, -1, 0,
                                                                              kTMax * 4);
        k_attn_combine<<<dim3(kTMax, d.n_heads), 128, 0, s>>>(b.state, d.n_heads, d.n_kv, b.part_o, b.part_ml,
                                                              b.max_chunks, b.attn_out, -1, 0, kTMax * 4, nullptr);
        k_quant_rows<<<(qd / 32 * kTMax + kWarps - 1) / kWarps, kThreads, 0, s>>>(b.state, b.attn_out, qd, b.act_q, b.act_d);
        {
            GemvArgs a{w.o, H / kTileRows, qd / kTileK, b.act_q, b.act_d, b.x, H, b.state, nullptr, nullptr};
            gemv<EPI_RESID, 1>(a, a.n_rg, s);
        }
        k_rmsnorm_quant<<<kTMax, kThreads, 0, s>>>(b.state, b.x, H, w.ffn_norm, d.eps, b.act_q, b.act_d, nullptr);
        {
            GemvArgs a{w.gu, 2 * F / kTileRows, H / kTileK, b.act_q, b.act_d, b.gu, F, b.state, nullptr, nullptr};
            gemv<EPI_SWIGLU, 2>(a, a.n_rg / 2, s);
        }
        k_quant_rows<<<(F / 32 * kTMax + kWarps - 1) / kWarps, kThreads, 0, s>>>(b.state, b.gu, F, b.act_q, b.act_d);
        {
            GemvArgs a{w.down, H / kTileRows, F / kTileK, b.act_q, b.act_d, b.x, H, b.state, nullptr, nullptr};
            gemv<EPI_RESID, 1>(a, a.n_rg, s);
        }
    }
    (void)G;
    k_rmsnorm_quant<<<kTMax, kThreads, 0, s>>>(b.state, b.x, H, m.output_norm, d.eps, b.act_q, b.act_d, b.hid);
}

// A prefill pass: the layer sequence of forward_layers over P rows at once,
// the projections on tcgen05 (prefill_tc.cu), attention as row blocks of 16
// through the same split-KV kernels (same arithmetic and order).
void launch_prefill_pass(const DeviceModel& m, const KvCache& kv, const PrefillBuffers& p, int P, int before,
                         bool want_hidden, cudaStream_t s) {
    const ModelDims& d = m.dims;
    const int H = d.hidden, F = d.ffn;
    const int qd = d.n_heads * kHeadDim, kd = d.n_kv * kHeadDim;
    const int G = d.n_heads / d.n_kv;
    const int n_rb = (P + kTMax - 1) / kTMax, max_chunks = (before + P + kPage - 1) / kPage, qstride = kTMax * G;
    const size_t attn_smem = (size_t)(kTMax * 4 * kHeadDim + kPage * (kHeadDim + 1) + kTMax * 4 * kPage) * sizeof(float);
    for (int l = 0; l < d.n_layers; ++l) {
        const LayerWeights& w = m.layers[l];
        pf_norm_quant(p.x, P, H, w.attn_norm, d.eps, p.xq, p.xd, nullptr, s);
        pf_gemm(w.pf_qkv, qd + 2 * kd, H, p.xq, p.xd, P, p.qkv, qd + 2 * kd, PF_EPI_STORE, p.status, s);
        k_qk_norm_rope_store<<<dim3(P, d.n_heads + d.n_kv), 128, 0, s>>>(nullptr, p.qkv, d.n_heads, d.n_kv, w.q_norm,
                                                                         w.k_norm, d.eps, m.theta_scale, kv, l, P, before);
        if (G == 2)
            k_pf_attn<<<dim3(max_chunks, d.n_kv, (P + kPfTok - 1) / kPfTok), 256, kPfAttnSmem, s>>>(
                p.qkv, d.n_heads, d.n_kv, kv, l, p.part_o, p.part_ml, max_chunks, P, before, qstride);
        else
            k_attn_chunk<<<dim3(max_chunks, d.n_kv, n_rb), kThreads, attn_smem, s>>>(
                nullptr, p.qkv, d.n_heads, d.n_kv, kv, l, p.part_o, p.part_ml, max_chunks, P, before, qstride);
        k_attn_combine<<<dim3(P, d.n_heads), 128, 0, s>>>(nullptr, d.n_heads, d.n_kv, p.part_o, p.part_ml, max_chunks,
                                                          p.attn, P, before, qstride, nullptr);
        pf_quant(p.attn, P, qd, p.xq, p.xd, s);
        pf_gemm(w.pf_o, H, qd, p.xq, p.xd, P, p.x, H, PF_EPI_RESID, p.status, s);
        pf_norm_quant(p.x, P, H, w.ffn_norm, d.eps, p.xq, p.xd, nullptr, s);
        pf_gemm(w.pf_gu, 2 * F, H, p.xq, p.xd, P, p.gu, F, PF_EPI_SWIGLU, p.status, s);
        pf_quant(p.gu, P, F, p.xq, p.xd, s);
        pf_gemm(w.pf_down, H, F, p.xq, p.xd, P, p.x, H, PF_EPI_RESID, p.status, s);
    }
    if (want_hidden) pf_norm_quant(p.x, P, H, m.output_norm, d.eps, p.xq, p.xd, p.hid, s);
}

static void lm_head(const DeviceModel& m, const StepBuffers& b, bool want_logits, cudaStream_t s) {
    if (m.f16) {
        lm_head_f16(m, b, want_logits, s);
        return;
    }
    GemvArgs a{m.embd, m.dims.vocab / kTileRows, m.dims.hidden / kTileK, b.act_q, b.act_d,
               nullptr, m.dims.vocab, b.state, b.lm_val, want_logits ? b.logits : nullptr};
    gemv<EPI_ARGMAX, 8>(a, b.lm_blocks, s);
}

void launch_step(const DeviceModel& m, const KvCache& kv, const StepBuffers& b, int draft_mode, bool want_logits,
                 cudaStream_t s) {
    if (draft_mode == 0) k_draft<<<1, 256, 0, s>>>(b.state, b.ids);
    else if (draft_mode == 1) k_draft_forced<<<1, 1, 0, s>>>(b.state);
    if (m.f16)
        k_embed_f16<<<kTMax, 256, 0, s>>>(b.state, reinterpret_cast<const __half*>(m.h_embd), m.dims.hidden,
                                          m.dims.vocab, b.x);
    else
        k_embed<<<kTMax, 256, 0, s>>>(b.state, m.embd, m.dims.hidden, m.dims.vocab, b.x);
    forward_layers(m, kv, b, s);
    const bool penalty_path = want_logits;
    lm_head(m, b, penalty_path, s);
    if (penalty_path) {
        const size_t bits = (size_t)((m.dims.vocab + 31) / 32) * 4;
        k_choice_penalty<<<kTMax, 1024, bits, s>>>(b.state, b.ids, b.logits, m.dims.vocab);
    }
    k_accept<<<1, 512, 0, s>>>(b.state, b.ids, b.lm_val, b.lm_blocks, penalty_path ? 1 : 0);
}

void launch_draft_group(const DraftGroup& g, cudaStream_t s) { k_draft_group<<<g.n, 256, 0, s>>>(g); }

void launch_group_stopped(const DraftGroup& g, int* flag, cudaStream_t s) { k_group_stopped<<<1, 32, 0, s>>>(g, flag); }

void launch_draft(const StepBuffers& b, int draft_mode, cudaStream_t s) {
    if (draft_mode == 0) k_draft<<<1, 256, 0, s>>>(b.state, b.ids);
    else if (draft_mode == 1) k_draft_forced<<<1, 1, 0, s>>>(b.state);
}

void launch_forward_rows(const DeviceModel& m, const KvCache& kv, const StepBuffers& b, bool lm, bool want_logits,
                         cudaStream_t s) {
    forward_layers(m, kv, b, s);
    if (lm) lm_head(m, b, want_logits, s);
}

void launch_draft_args(const int32_t* ids, int n, int maximum, int n_min, int n_max, int32_t* out, int* n_out,
                       cudaStream_t s) {
    k_draft_args<<<1, 256, 0, s>>>(ids, n, maximum, n_min, n_max, out, n_out);
}

void launch_choice_args(const float* logits, int n_raw, const int32_t* hist, int n_hist, float p, int* out,
                        cudaStream_t s) {
    k_choice_args<<<1, 1024, (size_t)((n_raw + 31) / 32) * 4, s>>>(logits, n_raw, hist, n_hist, p, out);
}

void launch_set_forced(const StepBuffers& b, const int32_t* src, int n, int vocab, cudaStream_t s) {
    k_set_forced<<<1, 1, 0, s>>>(b.state, src, n, vocab);
}

void launch_lm_argmax_rows(const DeviceModel& m, StepState* state, const float* rows, int T, uint8_t* act_q,
                           float* act_d, float2* partials, int32_t* choices, cudaStream_t s) {
    const int lm_blocks = lm_head_blocks(m.dims.vocab);
    k_state_rows<<<1, 1, 0, s>>>(state, T);
    k_quant_rows<<<(m.dims.hidden / 32 * kTMax + kWarps - 1) / kWarps, kThreads, 0, s>>>(state, rows, m.dims.hidden,
                                                                                        act_q, act_d);
    GemvArgs a{m.embd, m.dims.vocab / kTileRows, m.dims.hidden / kTileK, act_q, act_d,
               nullptr, m.dims.vocab, state, partials, nullptr};
    gemv<EPI_ARGMAX, 8>(a, lm_blocks, s);
    k_reduce_choices_out<<<1, 512, 0, s>>>(state, partials, lm_blocks, choices);
}

void launch_fuse_embeds(const DeviceModel& m, const int32_t* ids, const int32_t* slot, int seq, const float* audio,
                        float* out, cudaStream_t s) {
    if (m.f16)
        k_fuse_embeds_f16<<<seq, 256, 0, s>>>(ids, slot, seq, audio, reinterpret_cast<const __half*>(m.h_embd),
                                              m.dims.hidden, out);
    else
        k_fuse_embeds<<<seq, 256, 0, s>>>(ids, slot, seq, audio, m.embd, m.dims.hidden, out);
}

void launch_rows_begin(const StepBuffers& b, int T, cudaStream_t s) { k_rows_begin<<<1, 1, 0, s>>>(b.state, T); }
void launch_rows_end(const StepBuffers& b, cudaStream_t s) { k_rows_end<<<1, 1, 0, s>>>(b.state); }

void launch_prefill_seed(const StepBuffers& b, cudaStream_t s) {
    k_prefill_seed<<<1, 512, 0, s>>>(b.state, b.ids, b.lm_val, b.lm_blocks, 0);
}

void launch_lm_row(const DeviceModel& m, const StepBuffers& b, const float* hidden_row, cudaStream_t s) {
    // One final-normed row as the step's only row: quantised like the verify
    // path's last RMSNorm output, then the LM head with its first max (lm_val).
    k_rows_begin<<<1, 1, 0, s>>>(b.state, 1);
    if (m.f16) {
        k_rows_f16<<<64, 256, 0, s>>>(b.state, hidden_row, m.dims.hidden, reinterpret_cast<__half*>(b.act_h));
        lm_head(m, b, false, s);
        return;
    }
    k_quant_rows<<<(m.dims.hidden / 32 * kTMax + kWarps - 1) / kWarps, kThreads, 0, s>>>(b.state, hidden_row,
                                                                                        m.dims.hidden, b.act_q, b.act_d);
    lm_head(m, b, false, s);
}

void launch_logits_row(const DeviceModel& m, const StepBuffers& b, const float* hidden_row, cudaStream_t s) {
    // hidden_row is device memory holding one row; quantise it as row 0 (T is 1 in state).
    if (m.f16) {
        k_rows_f16<<<64, 256, 0, s>>>(b.state, hidden_row, m.dims.hidden, reinterpret_cast<__half*>(b.act_h));
        lm_head(m, b, true, s);
        return;
    }
    k_quant_rows<<<(m.dims.hidden / 32 * kTMax + kWarps - 1) / kWarps, kThreads, 0, s>>>(b.state, hidden_row,
                                                                                        m.dims.hidden, b.act_q, b.act_d);
    lm_head(m, b, true, s);
}

void launch_fill_synthetic_kv(const DeviceModel& m, const KvCache& kv, int n_pos, uint32_t seed, cudaStream_t s) {
    k_fill_synthetic_kv<<<g_sm_count * 8, 256, 0, s>>>(kv, m.dims.n_layers, m.dims.n_kv, n_pos, seed);
}

void launch_poison_kv(const DeviceModel& m, const KvCache& kv, int pos0, int n_pos, cudaStream_t s) {
    k_poison_kv<<<g_sm_count * 4, 256, 0, s>>>(kv, m.dims.n_layers, m.dims.n_kv, pos0, n_pos);
}

void launch_kv_gather(const DeviceModel& m, const KvCache& kv, int layer, int which, int pos0, int n_pos, float* out,
                      cudaStream_t s) {
    k_kv_gather<<<g_sm_count, 256, 0, s>>>(kv, m.dims.n_kv, layer, which, pos0, n_pos, out);
}

MTB_BC_TAKE(bc_take_kernels)

}  // namespace mtb
