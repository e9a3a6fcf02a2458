// Prefill projections on the 5th-generation tensor cores (tcgen05).
//
// A prefill runs T = 16 .. thousands of prompt rows through every projection
// at once, so the q8_0 contraction is GEMM-shaped: D[128 weight rows x 32
// tokens] per CTA, K streamed in 64-byte steps.  One `tcgen05.mma.kind::i8`
// per q8_0 block (K = 32) writes that block's exact int32 sums into its own 32
// TMEM columns (16 blocks = two 256-K slices in flight, all 512 columns); the
// epilogue warps read them back with `tcgen05.ld` and evaluate the same fp32
// order as every other path of this library: per output, one
// fmaf(isum, d_w * d_x, acc) per block in ascending order inside each 256-K
// slice, slices added in order from 0.  Integer block sums are exact, so the
// results equal the verify kernels' and the CPU restatement's bit for bit.
//
// Layouts (both operands K-major, no swizzle, 8-row x 16-byte core matrices):
//  * weights, per (128-row tile, 64-K step): 8192 code bytes, core matrix
//    (row group g, 16-byte chunk c) at (4 g + c) * 128, row r of it at +16 r;
//    then 512 bytes of fp16 scales [128 rows][2 blocks].  8704 bytes per step.
//  * activations, per (32-token tile, 64-K step): 2048 code bytes, the same
//    core-matrix order over 4 token groups; scales f32 [T][K / 32] apart.
// Warp roles (320 threads): warp 0 producer (cp.async.bulk into a 4-stage
// ring), warp 1 TMEM owner + MMA issuer, warps 2-9 epilogue in two warpgroups
// of 16 tokens each (warp w reads TMEM lanes 32 (w % 4) ..; pairs of tokens
// go through one __fmul2_rn and one __ffma2_rn, each half its own chain).
// Every wait is bounded; a timeout sets `status`.
#include "device_common.cuh"
#include "exact_math.cuh"
#include "prefill_tc.hpp"

namespace mtb {
namespace {

using namespace dev;

constexpr int kPfRows = 128;             // weight rows per tile (MMA M)
constexpr int kPfTok = 32;               // tokens per tile (MMA N)
constexpr int kPfStepW = kPfRows * 64;   // code bytes of one 64-K weight step
constexpr int kPfStepWB = kPfStepW + kPfRows * 2 * 2;  // + fp16 scales
constexpr int kPfStepX = kPfTok * 64;    // code bytes of one 64-K activation step
constexpr int kPfStages = 4;
constexpr int kPfThreads = 320;
constexpr int kPfHalfTok = kPfTok / 2;  // tokens per epilogue warpgroup
constexpr unsigned long long kPfWaitNs = 2000000000ull;
constexpr uint32_t kPfIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPfTok >> 3) << 17) |
                              ((uint32_t)(kPfRows >> 4) << 24);  // s32 <- s8 x s8, K-major, M 128, N 32

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long gns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) {
    // K-major, no swizzle: 16-byte K chunks 128 bytes apart (LBO), 8-row
    // groups 512 bytes apart (SBO), descriptor version 1.
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46);
}

__device__ __forceinline__ bool pf_wait(uint64_t* bar, unsigned parity, int* status) {
    const uint32_t a = su32(bar);
    unsigned long long t0 = 0;
    for (unsigned it = 0;; ++it) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok)
                     : "r"(a), "r"(parity), "r"(20000u)
                     : "memory");
        if (ok) return true;
        if (it == 0) t0 = gns();
        if (*reinterpret_cast<volatile int*>(status)) return false;
        if (gns() - t0 > kPfWaitNs) {
            atomicExch(status, 1);
            return false;
        }
    }
}

struct PfArgs {
    const uint8_t* w;   // weight steps [N / 128][K / 64][8704]
    const uint8_t* xq;  // activation steps [T_pad / 32][K / 64][2048]
    const float* xd;    // activation scales [T][K / 32]
    float* y;           // output rows [T][ldy]
    int T, K, ldy, epi;
    int* status;
    const float* bias;  // [n_rows] for the PF_EPI_BIAS* epilogues, else null
};

__global__ void __launch_bounds__(kPfThreads, 1) k_pf_gemm(PfArgs a) {
    extern __shared__ __align__(1024) uint8_t pf_smem[];
    uint8_t* stage_w = pf_smem;                                         // [stages][8704] (1024-aligned slots below)
    uint8_t* stage_x = pf_smem + kPfStages * 9216;                      // [stages][2048]
    float* s_dx = reinterpret_cast<float*>(stage_x + kPfStages * kPfStepX);  // [K / 32][32 tokens]
    __shared__ __align__(8) uint64_t full[kPfStages], empty[kPfStages], slice_full[2], slice_free[2];
    __shared__ uint32_t tmem_base;
    __shared__ float s_up[kPfTok][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tt = blockIdx.x, nt = blockIdx.y;
    const int n_steps = a.K / 64, n_slices = a.K / 256, nb = a.K / 32;
    const uint8_t* wt = a.w + (size_t)nt * n_steps * kPfStepWB;
    const uint8_t* xt = a.xq + (size_t)tt * n_steps * kPfStepX;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPfStages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&full[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&empty[s])) : "memory");
        }
        for (int s = 0; s < 2; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&slice_full[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 8;" ::"r"(su32(&slice_free[s])) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(su32(&tmem_base)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Activation scales of the tile's tokens (tokens past T read as 0).
    for (int i = threadIdx.x; i < kPfTok * nb; i += kPfThreads) {
        const int t = tt * kPfTok + i / nb, kb = i % nb;
        s_dx[kb * kPfTok + i / nb] = t < a.T ? a.xd[(size_t)t * nb + kb] : 0.f;
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        // Producer: one bulk copy for the weight step, one for the activation step.
        if (lane == 0) {
            for (int ks = 0; ks < n_steps; ++ks) {
                const int s = ks % kPfStages;
                if (ks >= kPfStages && !pf_wait(&empty[s], ((ks / kPfStages) - 1) & 1, a.status)) break;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[s])),
                             "r"((unsigned)(kPfStepWB + kPfStepX))
                             : "memory");
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                             ::"r"(su32(stage_w + s * 9216)), "l"(wt + (size_t)ks * kPfStepWB), "r"((unsigned)kPfStepWB),
                             "r"(su32(&full[s]))
                             : "memory");
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                             ::"r"(su32(stage_x + s * kPfStepX)), "l"(xt + (size_t)ks * kPfStepX), "r"((unsigned)kPfStepX),
                             "r"(su32(&full[s]))
                             : "memory");
            }
        }
    } else if (warp == 1) {
        // MMA issuer: block kb of the tile -> TMEM columns 32 (kb % 16).
        if (lane == 0) {
            for (int ks = 0; ks < n_steps; ++ks) {
                const int s = ks % kPfStages;
                const int sl = ks / 4;
                if (ks % 4 == 0 && sl >= 2 && !pf_wait(&slice_free[sl % 2], ((sl / 2) - 1) & 1, a.status)) break;
                if (!pf_wait(&full[s], (ks / kPfStages) & 1, a.status)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                for (int b = 0; b < 2; ++b) {
                    const int kb = 2 * ks + b;
                    const uint64_t da = umma_desc(su32(stage_w + s * 9216) + b * 256);
                    const uint64_t db = umma_desc(su32(stage_x + s * kPfStepX) + b * 256);
                    const uint32_t d = tmem + (uint32_t)((kb % 16) * kPfTok);
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n"
                        ::"r"(d), "l"(da), "l"(db), "r"(kPfIdesc), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
                        : "memory");
                }
                // The stage is free once these MMAs have read it.
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                             ::"r"(su32(&empty[s])) : "memory");
                if (ks % 4 == 3)
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                                 ::"r"(su32(&slice_full[sl % 2])) : "memory");
            }
        }
    } else {
        // Epilogue: thread = weight row r of the tile (TMEM lane r), tokens
        // 16 tg .. 16 tg + 15 of the tile.
        const int q = warp & 3, tg = (warp - 2) >> 2;
        const int r = 32 * q + lane;
        float2 y[kPfHalfTok / 2];
#pragma unroll
        for (int u = 0; u < kPfHalfTok / 2; ++u) y[u] = make_float2(0.f, 0.f);
        bool ok = true;
        for (int sl = 0; sl < n_slices && ok; ++sl) {
            // This row's 8 weight scales of the slice (fp16 pairs per 64-K step).
            float dw[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t v = __ldg(reinterpret_cast<const uint32_t*>(wt + (size_t)(4 * sl + j) * kPfStepWB + kPfStepW) + r);
                dw[2 * j] = h2f_lo(v);
                dw[2 * j + 1] = h2f_hi(v);
            }
            ok = pf_wait(&slice_full[sl % 2], (sl / 2) & 1, a.status);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float2 acc[kPfHalfTok / 2];
#pragma unroll
            for (int u = 0; u < kPfHalfTok / 2; ++u) acc[u] = make_float2(0.f, 0.f);
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const int kb = 8 * sl + b;
                uint32_t v[16];
                const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((kb % 16) * kPfTok + kPfHalfTok * tg);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15])
                    : "r"(ta));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const float2* dx = reinterpret_cast<const float2*>(s_dx + kb * kPfTok + kPfHalfTok * tg);
                const float2 dw2 = make_float2(dw[b], dw[b]);
#pragma unroll
                for (int u = 0; u < kPfHalfTok / 2; ++u) {
                    const float2 iv = make_float2(small_int_to_float((int)v[2 * u]), small_int_to_float((int)v[2 * u + 1]));
                    acc[u] = __ffma2_rn(iv, __fmul2_rn(dw2, dx[u]), acc[u]);
                }
            }
            // Columns of this slice may be reused by slice sl + 2.
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&slice_free[sl % 2])) : "memory");
#pragma unroll
            for (int u = 0; u < kPfHalfTok / 2; ++u) y[u] = __fadd2_rn(y[u], acc[u]);
        }
        float yt[kPfHalfTok];
#pragma unroll
        for (int u = 0; u < kPfHalfTok / 2; ++u) {
            yt[2 * u] = y[u].x;
            yt[2 * u + 1] = y[u].y;
        }
        const int n = nt * kPfRows + r;
        if (a.epi == PF_EPI_SWIGLU) {
            // Rows 0..63 of the tile are gate rows of features 64 nt + r,
            // rows 64..127 the up rows of the same features.  Every epilogue
            // warp meets the named barrier, whatever its wait results.
            if (ok && r >= 64)
#pragma unroll
                for (int t = 0; t < kPfHalfTok; ++t) s_up[kPfHalfTok * tg + t][r - 64] = yt[t];
            asm volatile("bar.sync 1, 256;" ::: "memory");
            if (ok && r < 64) {
#pragma unroll
                for (int t = 0; t < kPfHalfTok; ++t) {
                    const int tl = kPfHalfTok * tg + t, row = tt * kPfTok + tl;
                    if (row < a.T) {
                        const float g = yt[t];
                        const float sw = g / (1.0f + exact_expf(-g));
                        a.y[(size_t)row * a.ldy + nt * 64 + r] = sw * s_up[tl][r];
                    }
                }
            }
        } else if (ok && a.epi >= PF_EPI_BIAS) {
            // Linear layers with a bias (ggml_mul_mat then ggml_add): y = acc + b,
            // then GELU (erf form), SiLU, or the residual add res + (acc + b).
            const float b = a.bias[n];
#pragma unroll
            for (int t = 0; t < kPfHalfTok; ++t) {
                const int row = tt * kPfTok + kPfHalfTok * tg + t;
                if (row < a.T) {
                    float* o = a.y + (size_t)row * a.ldy + n;
                    const float v = __fadd_rn(yt[t], b);
                    if (a.epi == PF_EPI_BIAS_GELU)
                        *o = exact_gelu_erf(v);
                    else if (a.epi == PF_EPI_BIAS_SILU)
                        *o = __fdiv_rn(v, __fadd_rn(1.0f, exact_expf(-v)));
                    else if (a.epi == PF_EPI_BIAS_RESID)
                        *o = __fadd_rn(*o, v);
                    else
                        *o = v;
                }
            }
        } else if (ok) {
#pragma unroll
            for (int t = 0; t < kPfHalfTok; ++t) {
                const int row = tt * kPfTok + kPfHalfTok * tg + t;
                if (row < a.T) {
                    float* o = a.y + (size_t)row * a.ldy + n;
                    *o = a.epi == PF_EPI_RESID ? __fadd_rn(*o, yt[t]) : yt[t];
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

// q8_0 GGUF rows (34-byte blocks: fp16 d + 32 int8) -> prefill weight steps.
// half < 0: `n_src` rows fill whole 128-row tiles.  half 0 / 1: the gate / up
// rows of a gate/up pair: source row f goes to row 64 half + f % 64 of tile f / 64.
__global__ void k_pf_repack(const uint8_t* src, int n_src, int K, int half, uint8_t* dst) {
    const int n_steps = K / 64, blocks_per_row = K / 32;
    const long long total = (long long)n_src * n_steps;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int src_row = int(i % n_src), ks = int(i / n_src);
        const int nt = half < 0 ? src_row / kPfRows : src_row / 64;
        const int r = half < 0 ? src_row % kPfRows : 64 * half + src_row % 64;
        uint8_t* step = dst + ((size_t)nt * n_steps + ks) * kPfStepWB;
        for (int b = 0; b < 2; ++b) {
            const uint8_t* blk = src + ((size_t)src_row * blocks_per_row + 2 * ks + b) * 34;
            for (int k = 0; k < 32; ++k) {
                const int kk = 32 * b + k;
                step[((r / 8) * 4 + kk / 16) * 128 + (r % 8) * 16 + kk % 16] = blk[2 + k];
            }
            step[kPfStepW + r * 4 + b * 2] = blk[0];
            step[kPfStepW + r * 4 + b * 2 + 1] = blk[1];
        }
    }
}

// RMSNorm (the hidden-row tree of row_rms_scale) and q8_0 quantisation of
// T rows into activation steps + scales; one CTA per row.
__global__ void __launch_bounds__(256) k_pf_norm_quant(const float* __restrict__ x, int T, int K,
                                                      const float* __restrict__ w, float eps, uint8_t* xq, float* xd,
                                                      float* normed) {
    const int row = blockIdx.x;
    if (row >= T) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ double s_q[256];
    __shared__ float s_scale;
    const float scale = row_rms_scale(x + (size_t)row * K, K, eps, s_q, &s_scale);
    const int n_steps = K / 64, tt = row / kPfTok, tr = row % kPfTok;
    for (int blk = warp; blk < K / 32; blk += 8) {
        const int i = blk * 32 + lane;
        const float v = __fmul_rn(__fmul_rn(x[(size_t)row * K + i], scale), w[i]);
        if (normed) normed[(size_t)row * K + i] = v;
        const float am = warp_absmax(v);
        float amv[1] = {am}, dq[1], iq[1];
        q8_scales<1>(amv, dq, iq);
        const int kk = i % 64;
        xq[((size_t)tt * n_steps + i / 64) * kPfStepX + ((tr / 8) * 4 + kk / 16) * 128 + (tr % 8) * 16 + kk % 16] =
            (uint8_t)q8_code_bits(__fmul_rn(v, iq[0]));
        if (lane == 0) xd[(size_t)row * (K / 32) + blk] = __half2float(__float2half_rn(dq[0]));
    }
}

// Plain q8_0 quantisation of T rows [T][K] into activation steps + scales.
__global__ void __launch_bounds__(256) k_pf_quant(const float* __restrict__ x, int T, int K, uint8_t* xq, float* xd) {
    const int warp = (blockIdx.x * 256 + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nb = K / 32, n_steps = K / 64;
    if (warp >= T * nb) return;
    const int row = warp / nb, blk = warp % nb;
    const int i = blk * 32 + lane;
    const float v = x[(size_t)row * K + i];
    const float am = warp_absmax(v);
    float amv[1] = {am}, dq[1], iq[1];
    q8_scales<1>(amv, dq, iq);
    const int tt = row / kPfTok, tr = row % kPfTok, kk = i % 64;
    xq[((size_t)tt * n_steps + i / 64) * kPfStepX + ((tr / 8) * 4 + kk / 16) * 128 + (tr % 8) * 16 + kk % 16] =
        (uint8_t)q8_code_bits(__fmul_rn(v, iq[0]));
    if (lane == 0) xd[(size_t)row * nb + blk] = __half2float(__float2half_rn(dq[0]));
}

}  // namespace

size_t pf_weight_bytes(int n_rows, int K) { return (size_t)(n_rows / kPfRows) * (K / 64) * kPfStepWB; }
size_t pf_act_bytes(int T, int K) { return (size_t)((T + kPfTok - 1) / kPfTok) * (K / 64) * kPfStepX; }
int pf_smem_bytes(int K) { return kPfStages * 9216 + kPfStages * kPfStepX + kPfTok * (K / 32) * 4; }

cudaError_t pf_configure() {
    // Up to K = 3072 (the down projection); one CTA per SM (the tile owns all 512 TMEM columns).
    return cudaFuncSetAttribute(k_pf_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, 120 * 1024);
}

void pf_repack(const uint8_t* src_q8, int n_src, int K, int half, uint8_t* dst, cudaStream_t s) {
    k_pf_repack<<<148 * 4, 256, 0, s>>>(src_q8, n_src, K, half, dst);
}

void pf_norm_quant(const float* x, int T, int K, const float* w, float eps, uint8_t* xq, float* xd, float* normed,
                   cudaStream_t s) {
    k_pf_norm_quant<<<T, 256, 0, s>>>(x, T, K, w, eps, xq, xd, normed);
}

void pf_quant(const float* x, int T, int K, uint8_t* xq, float* xd, cudaStream_t s) {
    const int warps = T * (K / 32);
    k_pf_quant<<<(warps + 7) / 8, 256, 0, s>>>(x, T, K, xq, xd);
}

void pf_gemm(const uint8_t* w, int n_rows, int K, const uint8_t* xq, const float* xd, int T, float* y, int ldy, int epi,
             int* status, cudaStream_t s) {
    PfArgs a{w, xq, xd, y, T, K, ldy, epi, status, nullptr};
    // Dynamic shared memory >= 120 KB keeps one CTA per SM.
    k_pf_gemm<<<dim3((T + kPfTok - 1) / kPfTok, n_rows / kPfRows), kPfThreads, 120 * 1024, s>>>(a);
}

void pf_gemm_bias(const uint8_t* w, int n_rows, int K, const uint8_t* xq, const float* xd, int T, float* y, int ldy,
                  int epi, const float* bias, int* status, cudaStream_t s) {
    PfArgs a{w, xq, xd, y, T, K, ldy, epi, status, bias};
    k_pf_gemm<<<dim3((T + kPfTok - 1) / kPfTok, n_rows / kPfRows), kPfThreads, 120 * 1024, s>>>(a);
}

MTB_BC_TAKE(bc_take_prefill)

}  // namespace mtb
