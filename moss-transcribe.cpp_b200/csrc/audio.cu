// The audio front end on the device: Whisper log-mel, the Whisper encoder and
// the audio adaptor, from 16 kHz samples to the decoder's audio embedding rows
// (AudioEncoder::encode, src/audio_encoder.cpp:16-75; WhisperMel::compute,
// src/mel.cpp:153-214; WhisperEncoder::encode, src/whisper_encoder.cpp:98-207;
// AudioAdaptor::apply, src/audio_adaptor.cpp:39-96).
//
// Per 30 s chunk (zero-padded to feat_n_samples, as the reference pads it):
//  * k_mel_frames: one CTA per frame.  Reflect padding by index arithmetic,
//    the periodic-Hann window, the 201-bin real DFT in double with the
//    reference's float twiddle tables and its sequential sums, the power
//    spectrum, the mel projection in double and log10 (src/mel.cpp:177-209).
//    k_mel_finish: the chunk maximum, floor max - 8, (v + 4) / 4 (:216-223).
//  * k_conv_gelu: the two conv1d stem layers (kernel 3, half-kernel padding,
//    stride 1 then 2) as an implicit-im2col F32 GEMM with the bias, GELU (erf)
//    and, for conv2, the positional embedding in the epilogue.  The conv stem
//    stays F32 in the reference's GGUFs (scripts/convert_moss_transcribe_to_gguf.py:38-53).
//  * per layer: k_layer_norm (ggml_norm: mean and variance summed in double,
//    eps 1e-5) -> q8_0 activations -> the tcgen05 q8_0 GEMM of prefill_tc.cu for
//    Q|K|V (one weight matrix, K has no bias), k_enc_attn (bidirectional,
//    16 heads of 64, online softmax in f32), the O projection with bias and the
//    residual in its epilogue; LayerNorm, FFN-1 with bias + GELU, FFN-2 with
//    bias + residual.  Final LayerNorm written straight into the chunk's
//    slot of the concatenated encoder frames, trimmed to token_len * 4 rows.
//  * after the last chunk, the adaptor on the concatenation viewed as
//    [frames / 4][4 d]: fc1 + bias + SiLU, fc2 + bias, LayerNorm (eps from
//    mtd.adaptor_norm_eps).
// The encoder's linear weights must be q8_0 (the reference's q8_0 GGUFs); the
// activations are quantised to q8_0 before each of them, as ggml's mul_mat does.
// Layout in HBM: activations token-major [frames][channels]; the weights as the
// prefill GEMM's 128-row tiles; one scratch set per loaded model, sized for one
// chunk, plus the concatenation and adaptor buffers, grown on demand.
#include "../../include/mtb_decoder.h"
#include "device_common.cuh"
#include "gguf.hpp"
#include "prefill_tc.hpp"

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

using namespace mtb;
using namespace mtb::dev;

namespace {

thread_local std::string g_audio_error;

constexpr int kMelThreads = 256;
constexpr int kHd = 64;                   // Whisper head size (d_model / n_heads)
constexpr int kAttQ = 64, kAttK = 64;     // queries per CTA, keys per tile
constexpr int kAttPad = 68;               // shared-memory row stride (floats)
constexpr int kAttSmem = 4 * 64 * kAttPad * 4;
constexpr int kCvT = 64, kCvO = 64, kCvJ = 16;

// ------------------------------------------------------------------ log-mel

// One CTA per frame t: frame[i] = x[t * hop + i - n_fft / 2] (reflected at
// both ends, the edge sample excluded) * window[i]; for each bin b
// re = sum_i frame[i] cos_t[i][b], im = -sum_i frame[i] sin_t[i][b] in double,
// added in ascending i; power = re^2 + im^2; for each mel band m
// acc = sum_b fb[m][b] power[b] in ascending b; mel[m][t] = log10(max(acc, 1e-10)).
// frame_max[t] = the maximum of the frame's mel values.
__global__ void __launch_bounds__(kMelThreads) k_mel_frames(const float* __restrict__ x, int n, int n_fft, int hop,
                                                           const float* __restrict__ window,
                                                           const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t, int n_bins,
                                                           const float* __restrict__ fb, int n_mels, int n_frames,
                                                           float* __restrict__ mel, float* __restrict__ frame_max) {
    extern __shared__ double mel_power[];  // [n_bins], then the frame as floats [n_fft]
    float* frame = reinterpret_cast<float*>(mel_power + n_bins);
    __shared__ float s_max[kMelThreads / 32];
    const int t = blockIdx.x, pad = n_fft / 2;
    for (int i = threadIdx.x; i < n_fft; i += blockDim.x) {
        const int p = t * hop + i;
        const int src = p < pad ? pad - p : (p < pad + n ? p - pad : n - 2 - (p - pad - n));
        frame[i] = __fmul_rn(x[src], window[i]);
    }
    __syncthreads();
    for (int b = threadIdx.x; b < n_bins; b += blockDim.x) {
        double re = 0.0, im = 0.0;
        for (int i = 0; i < n_fft; ++i) {
            const double f = (double)frame[i];
            re = __dadd_rn(re, __dmul_rn(f, (double)cos_t[(size_t)i * n_bins + b]));
            im = __dsub_rn(im, __dmul_rn(f, (double)sin_t[(size_t)i * n_bins + b]));
        }
        mel_power[b] = __dadd_rn(__dmul_rn(re, re), __dmul_rn(im, im));
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int m = threadIdx.x; m < n_mels; m += blockDim.x) {
        const float* row = fb + (size_t)m * n_bins;
        double acc = 0.0;
        for (int b = 0; b < n_bins; ++b) acc = __dadd_rn(acc, __dmul_rn((double)row[b], mel_power[b]));
        const float v = (float)log10(fmax(acc, 1e-10));
        mel[(size_t)m * n_frames + t] = v;
        mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = s_max[0];
        for (int w = 1; w < kMelThreads / 32; ++w) v = fmaxf(v, s_max[w]);
        frame_max[t] = v;
    }
}

// v = (max(v, mx - 8) + 4) / 4 with mx the chunk's maximum (every CTA reduces
// the per-frame maxima itself: max is exact in any order).
__global__ void __launch_bounds__(256) k_mel_finish(float* __restrict__ mel, int count,
                                                   const float* __restrict__ frame_max, int n_frames) {
    __shared__ float s_max[8];
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n_frames; i += blockDim.x) mx = fmaxf(mx, frame_max[i]);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = s_max[0];
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s_max[w]);
    const float floor_v = __fsub_rn(mx, 8.0f);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        mel[i] = __fdiv_rn(__fadd_rn(fmaxf(mel[i], floor_v), 4.0f), 4.0f);
}

// ------------------------------------------------------------------ conv stem

// out[t][oc] = gelu(b[oc] + sum_j A[t][j] W[oc][j]) (+ pos[t][oc]) for the
// conv1d with kernel 3 and padding 1: j = ic * 3 + k, A[t][j] = x(ic, t s + k - 1)
// (zero outside [0, L)), x(ic, p) = x[p * sp + ic * sc].  W is the GGUF's
// [OC][IC][3] F32 kernel.  Each output is one fmaf chain over j from 0 in
// ascending order.  CTA: 64 frames x 64 channels, 4 x 4 outputs per thread.
__global__ void __launch_bounds__(256) k_conv_gelu(const float* __restrict__ x, int L, int IC, long long sp,
                                                  long long sc, int stride, const float* __restrict__ w,
                                                  const float* __restrict__ bias, const float* __restrict__ pos,
                                                  int OC, int OL, float* __restrict__ out) {
    __shared__ __align__(16) float As[kCvJ][kCvT];
    __shared__ __align__(16) float Ws[kCvJ][kCvO];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int t0 = blockIdx.x * kCvT, o0 = blockIdx.y * kCvO;
    const int J = IC * 3;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[i][k] = 0.f;
    for (int j0 = 0; j0 < J; j0 += kCvJ) {
        for (int e = threadIdx.x; e < kCvT * kCvJ; e += 256) {
            // Frames fastest when frames are contiguous in x, else channels.
            const int tl = sp == 1 ? e % kCvT : e / kCvJ, jj = sp == 1 ? e / kCvT : e % kCvJ;
            const int t = t0 + tl, j = j0 + jj, ic = j / 3, k = j % 3;
            const int p = t * stride + k - 1;
            As[jj][tl] = (t < OL && p >= 0 && p < L) ? x[(long long)p * sp + (long long)ic * sc] : 0.f;
        }
        for (int e = threadIdx.x; e < kCvO * kCvJ; e += 256) {
            const int ol = e / kCvJ, jj = e % kCvJ;
            Ws[jj][ol] = w[(size_t)(o0 + ol) * J + j0 + jj];
        }
        __syncthreads();
#pragma unroll
        for (int jj = 0; jj < kCvJ; ++jj) {
            const float4 a = *reinterpret_cast<const float4*>(&As[jj][ty * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&Ws[jj][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[i][k] = fmaf(av[i], bv[k], acc[i][k]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= OL) continue;
        float r[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int oc = o0 + tx * 4 + k;
            const float v = __fadd_rn(acc[i][k], bias[oc]);
            float g = exact_gelu_erf(v);
            if (pos) g = __fadd_rn(g, pos[(size_t)t * OC + oc]);
            r[k] = g;
        }
        *reinterpret_cast<float4*>(out + (size_t)t * OC + o0 + tx * 4) = make_float4(r[0], r[1], r[2], r[3]);
    }
}

// ------------------------------------------------------------------ LayerNorm

// ggml_norm + mul + add over rows of D: mean = sum x / D and the variance
// sum (x - mean)^2 / D, both sums in double (lane partials over i = lane,
// lane + 32, ..., then an xor butterfly); y = ((x - mean) * (1 / sqrtf(var + eps))) * w + b.
// One warp per row.
__global__ void __launch_bounds__(256) k_layer_norm(const float* __restrict__ x, long long ldx, int T, int D,
                                                   const float* __restrict__ w, const float* __restrict__ b,
                                                   float eps, float* __restrict__ y, long long ldy) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= T) return;
    const float* xr = x + (long long)row * ldx;
    float* yr = y + (long long)row * ldy;
    double s = 0.0;
    for (int i = lane; i < D; i += 32) s = __dadd_rn(s, (double)xr[i]);
    s = warp_sum_d(s);
    const float mean = (float)(s / D);
    double s2 = 0.0;
    for (int i = lane; i < D; i += 32) {
        const float v = __fsub_rn(xr[i], mean);
        s2 = __dadd_rn(s2, (double)__fmul_rn(v, v));
    }
    s2 = warp_sum_d(s2);
    const float var = (float)(s2 / D);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int i = lane; i < D; i += 32) {
        const float v = __fsub_rn(xr[i], mean);
        yr[i] = __fadd_rn(__fmul_rn(__fmul_rn(v, scale), w[i]), b[i]);
    }
}

// ------------------------------------------------------------------ attention

// Bidirectional attention of one head (size 64) over all T frames:
// out[t][64 h + i] = sum_j p_tj v_j[i] / sum_j p_tj, p_tj = exp(s_tj - max_j s_tj),
// s_tj = scale * (q_t . k_j), q/k/v read from the Q|K|V rows [T][3 d].
// CTA = 64 queries of head h, 256 threads as 16 x 16: thread (ty, tx) owns
// queries 4 ty .. 4 ty + 3 and, per 64-key tile, keys 4 tx .. 4 tx + 3 of the
// scores and dims 4 tx .. 4 tx + 3 of the output.  Online softmax over the key
// tiles (running maximum and sum per query, the output rescaled when the
// maximum grows); exp is exact_expf.
__global__ void __launch_bounds__(256, 3) k_enc_attn(const float* __restrict__ qkv, int T, int d, float scale,
                                                    float* __restrict__ out) {
    extern __shared__ __align__(16) float at_smem[];
    float* Qs = at_smem;                // [64 dims][kAttPad]: query fastest
    float* Ks = Qs + kHd * kAttPad;     // [64 dims][kAttPad]: key fastest
    float* Vs = Ks + kHd * kAttPad;     // [64 keys][kAttPad]: dim fastest
    float* Ps = Vs + kAttK * kAttPad;   // [64 keys][kAttPad]: query fastest
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int q0 = blockIdx.x * kAttQ, h = blockIdx.y;
    const long long ld = 3LL * d;
    const float* qb = qkv + h * kHd;
    const float* kb = qkv + d + h * kHd;
    const float* vb = qkv + 2 * d + h * kHd;
    for (int e = threadIdx.x; e < kAttQ * kHd; e += 256) {
        const int q = e / kHd, i = e % kHd;
        Qs[i * kAttPad + q] = q0 + q < T ? qb[(long long)(q0 + q) * ld + i] : 0.f;
    }
    float m[4], l[4], o[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        m[a] = -1e30f;
        l[a] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) o[a][c] = 0.f;
    }
    for (int k0 = 0; k0 < T; k0 += kAttK) {
        __syncthreads();  // the previous tile's K, V and P are consumed
        for (int e = threadIdx.x; e < kAttK * kHd; e += 256) {
            const int j = e / kHd, i = e % kHd;
            const bool valid = k0 + j < T;
            Ks[i * kAttPad + j] = valid ? kb[(long long)(k0 + j) * ld + i] : 0.f;
            Vs[j * kAttPad + i] = valid ? vb[(long long)(k0 + j) * ld + i] : 0.f;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) s[a][c] = 0.f;
#pragma unroll 8
        for (int i = 0; i < kHd; ++i) {
            const float4 qa = *reinterpret_cast<const float4*>(Qs + i * kAttPad + 4 * ty);
            const float4 kv = *reinterpret_cast<const float4*>(Ks + i * kAttPad + 4 * tx);
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) s[a][c] = fmaf(qv[a], kk[c], s[a][c]);
        }
        float alpha[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float tmax = -1e30f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                s[a][c] = k0 + 4 * tx + c < T ? __fmul_rn(s[a][c], scale) : -1e30f;
                tmax = fmaxf(tmax, s[a][c]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mn = fmaxf(m[a], tmax);
            alpha[a] = exact_expf(__fsub_rn(m[a], mn));
            m[a] = mn;
            float psum = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                s[a][c] = k0 + 4 * tx + c < T ? exact_expf(__fsub_rn(s[a][c], mn)) : 0.f;  // now p
                psum = __fadd_rn(psum, s[a][c]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) psum = __fadd_rn(psum, __shfl_xor_sync(0xffffffffu, psum, off));
            l[a] = __fadd_rn(__fmul_rn(l[a], alpha[a]), psum);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<float4*>(Ps + (4 * tx + c) * kAttPad + 4 * ty) = make_float4(s[0][c], s[1][c], s[2][c], s[3][c]);
        __syncthreads();
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) o[a][c] = __fmul_rn(o[a][c], alpha[a]);
#pragma unroll 8
        for (int j = 0; j < kAttK; ++j) {
            const float4 pa = *reinterpret_cast<const float4*>(Ps + j * kAttPad + 4 * ty);
            const float4 va = *reinterpret_cast<const float4*>(Vs + j * kAttPad + 4 * tx);
            const float pv[4] = {pa.x, pa.y, pa.z, pa.w}, vv[4] = {va.x, va.y, va.z, va.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) o[a][c] = fmaf(pv[a], vv[c], o[a][c]);
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int q = q0 + 4 * ty + a;
        if (q >= T) continue;
        const float inv = __fdiv_rn(1.0f, l[a]);
        *reinterpret_cast<float4*>(out + (long long)q * d + h * kHd + 4 * tx) =
            make_float4(__fmul_rn(o[a][0], inv), __fmul_rn(o[a][1], inv), __fmul_rn(o[a][2], inv),
                        __fmul_rn(o[a][3], inv));
    }
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

struct AudioLayer {
    const float *attn_ln_w, *attn_ln_b, *ffn_ln_w, *ffn_ln_b;
    const float *qkv_b, *o_b, *fc1_b, *fc2_b;  // qkv_b: q bias | zeros (K has none) | v bias
    const uint8_t *qkv, *o, *fc1, *fc2;        // prefill weight steps
};

struct mtb_audio {
    int device = 0;
    // Configuration (src/model_loader.cpp:131-153 keys).
    int n_fft = 400, hop = 160, n_mels = 80, n_bins = 201, n_samples = 480000, n_frames = 3000;
    int d = 1024, n_layers = 24, n_heads = 16, ffn = 4096, max_src_pos = 1500;
    int merge = 4, ad_in = 4096, hidden = 1024;
    float ad_eps = 1e-6f;
    int enc_T = 1500;  // encoder frames per chunk
    // Weights.
    float *window = nullptr, *cos_t = nullptr, *sin_t = nullptr, *fb = nullptr;
    float *conv1_w = nullptr, *conv1_b = nullptr, *conv2_w = nullptr, *conv2_b = nullptr, *pos = nullptr;
    float *ln_post_w = nullptr, *ln_post_b = nullptr;
    std::vector<AudioLayer> layers;
    const uint8_t *ad_fc1 = nullptr, *ad_fc2 = nullptr;
    float *ad_fc1_b = nullptr, *ad_fc2_b = nullptr, *ad_ln_w = nullptr, *ad_ln_b = nullptr;
    // Per-chunk scratch.
    float *samples = nullptr, *mel = nullptr, *frame_max = nullptr, *c1 = nullptr, *h = nullptr, *nrm = nullptr;
    float *qkv = nullptr, *att = nullptr, *f = nullptr;
    uint8_t* xq = nullptr;
    float* xd = nullptr;
    int* status = nullptr;
    // Concatenated encoder frames and adaptor buffers (grown on demand).
    float *enc_all = nullptr, *a1 = nullptr, *a2 = nullptr, *out = nullptr;
    uint8_t* axq = nullptr;
    float* axd = nullptr;
    int cap_frames = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    float last_ms = 0.f;
    std::vector<void*> allocs;
    std::vector<void*> grown;
    std::string error;
    ~mtb_audio() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : allocs) cudaFree(p);
        for (void* p : grown) cudaFree(p);
        for (auto& e : ev)
            if (e) cudaEventDestroy(e);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

#define AU_CK(call)                                                                \
    do {                                                                           \
        cudaError_t e_ = (call);                                                   \
        if (e_ != cudaSuccess) {                                                   \
            a->error = std::string(#call) + ": " + cudaGetErrorString(e_);         \
            return -1;                                                             \
        }                                                                          \
    } while (0)

template <class T>
int au_alloc(mtb_audio* a, T** p, size_t count) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T));
    if (e != cudaSuccess) {
        a->error = std::string("cudaMalloc: ") + cudaGetErrorString(e);
        return -1;
    }
    a->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return 0;
}

const GgufTensor* need(mtb_audio* a, const GgufFile& f, const std::string& name) {
    const GgufTensor* t = f.tensor(name);
    if (!t) a->error = "missing tensor '" + name + "'";
    return t;
}

// An F32 tensor of exactly `count` elements to the device.
int upload_f32(mtb_audio* a, const GgufFile& f, const std::string& name, size_t count, float** dst) {
    const GgufTensor* t = need(a, f, name);
    if (!t) return -1;
    if (t->type != GGML_F32 || t->nbytes != count * 4) {
        a->error = "tensor '" + name + "' must be F32 with " + std::to_string(count) + " elements";
        return -1;
    }
    if (au_alloc(a, dst, count)) return -1;
    AU_CK(cudaMemcpy(*dst, t->data, count * 4, cudaMemcpyHostToDevice));
    return 0;
}

// A q8_0 matrix of n rows x k (ggml ne = [k, n]) into prefill weight steps at
// dst (+ the steps of `row_offset` rows before it).
int upload_q8_steps(mtb_audio* a, const GgufFile& f, const std::string& name, int k, int n, uint8_t* staging,
                    uint8_t* dst, int row_offset) {
    const GgufTensor* t = need(a, f, name);
    if (!t) return -1;
    if (t->type != GGML_Q8_0 || t->ne.size() < 2 || t->ne[0] != k || t->ne[1] != n) {
        a->error = "tensor '" + name + "' must be q8_0 [" + std::to_string(n) + " x " + std::to_string(k) +
                   "] (the encoder's linear weights are supported as q8_0 only)";
        return -1;
    }
    AU_CK(cudaMemcpy(staging, t->data, t->nbytes, cudaMemcpyHostToDevice));
    pf_repack(staging, n, k, -1, dst + pf_weight_bytes(row_offset, k), nullptr);
    AU_CK(cudaGetLastError());
    AU_CK(cudaDeviceSynchronize());  // staging is reused by the next matrix
    return 0;
}

int load_audio(mtb_audio* a, const char* path) {
    GgufFile f;
    if (!f.open(path)) {
        a->error = f.error();
        return -1;
    }
    a->n_fft = int(f.get_u32("mtd.feat.n_fft", 400));
    a->hop = int(f.get_u32("mtd.feat.hop", 160));
    a->n_mels = int(f.get_u32("mtd.feat.feature_size", 80));
    a->n_samples = int(f.get_u32("mtd.feat.n_samples", 480000));
    a->n_frames = int(f.get_u32("mtd.feat.nb_max_frames", 3000));
    a->d = int(f.get_u32("mtd.audio.d_model", 1024));
    a->n_layers = int(f.get_u32("mtd.audio.n_layers", 24));
    a->n_heads = int(f.get_u32("mtd.audio.n_heads", 16));
    a->ffn = int(f.get_u32("mtd.audio.ffn", 4096));
    a->max_src_pos = int(f.get_u32("mtd.audio.max_src_pos", 1500));
    a->merge = int(f.get_u32("mtd.audio_merge_size", 4));
    a->ad_in = int(f.get_u32("mtd.adaptor_input_dim", 4096));
    a->ad_eps = f.get_f32("mtd.adaptor_norm_eps", 1e-6f);
    a->hidden = int(f.get_u32("mtd.text.hidden", 1024));
    a->n_bins = a->n_fft / 2 + 1;
    const int d = a->d;
    // The reference's conv stem (kernel 3, padding 1, strides 1 and 2) and the
    // shapes the device kernels tile.
    a->enc_T = (a->n_frames + 2 - 3) / 2 + 1;
    if (a->n_fft <= 0 || a->n_fft % 2 || a->hop <= 0 || a->n_mels <= 0 || a->n_frames <= 0 ||
        a->n_samples < a->n_fft || (long long)(a->n_frames - 1) * a->hop + a->n_fft > (long long)a->n_samples + a->n_fft ||
        a->n_heads <= 0 || d != a->n_heads * kHd || d % 256 || a->ffn % 256 || a->n_layers <= 0 ||
        a->merge <= 0 || a->ad_in != d * a->merge || a->ad_in % 256 || a->hidden % 256 || (3 * a->n_mels) % kCvJ ||
        a->enc_T > a->max_src_pos) {
        a->error = "unsupported audio configuration (needs head size 64, d_model/ffn/hidden multiples of 256, "
                   "adaptor input = d_model x merge, encoder frames <= max_src_pos)";
        return -1;
    }
    // Periodic Hann window and the real-DFT twiddle tables, formed exactly as
    // the reference forms them (src/mel.cpp:31-45), stored [i][bin].
    std::vector<float> win(a->n_fft), ct((size_t)a->n_fft * a->n_bins), st((size_t)a->n_fft * a->n_bins);
    for (int n = 0; n < a->n_fft; ++n) win[n] = 0.5f * (1.0f - std::cos(2.0 * M_PI * n / (double)a->n_fft));
    for (int k = 0; k < a->n_bins; ++k)
        for (int n = 0; n < a->n_fft; ++n) {
            const double ang = 2.0 * M_PI * (double)k * (double)n / (double)a->n_fft;
            ct[(size_t)n * a->n_bins + k] = (float)std::cos(ang);
            st[(size_t)n * a->n_bins + k] = (float)std::sin(ang);
        }
    if (au_alloc(a, &a->window, win.size()) || au_alloc(a, &a->cos_t, ct.size()) || au_alloc(a, &a->sin_t, st.size()))
        return -1;
    AU_CK(cudaMemcpy(a->window, win.data(), win.size() * 4, cudaMemcpyHostToDevice));
    AU_CK(cudaMemcpy(a->cos_t, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice));
    AU_CK(cudaMemcpy(a->sin_t, st.data(), st.size() * 4, cudaMemcpyHostToDevice));
    // Mel filters as [mel][bin], from either orientation (src/mel.cpp:50-66).
    {
        const GgufTensor* t = need(a, f, "mel_filters");
        if (!t) return -1;
        if (t->type != GGML_F32 || t->ne.size() < 2 ||
            !((t->ne[0] == a->n_bins && t->ne[1] == a->n_mels) || (t->ne[0] == a->n_mels && t->ne[1] == a->n_bins))) {
            a->error = "mel_filters must be F32 [n_mels x n_bins]";
            return -1;
        }
        std::vector<float> fbh((size_t)a->n_mels * a->n_bins);
        const float* raw = reinterpret_cast<const float*>(t->data);
        for (int m = 0; m < a->n_mels; ++m)
            for (int b = 0; b < a->n_bins; ++b)
                fbh[(size_t)m * a->n_bins + b] = t->ne[0] == a->n_bins ? raw[(size_t)m * a->n_bins + b]
                                                                      : raw[(size_t)b * a->n_mels + m];
        if (au_alloc(a, &a->fb, fbh.size())) return -1;
        AU_CK(cudaMemcpy(a->fb, fbh.data(), fbh.size() * 4, cudaMemcpyHostToDevice));
    }
    if (upload_f32(a, f, "enc.conv1.w", (size_t)d * a->n_mels * 3, &a->conv1_w) ||
        upload_f32(a, f, "enc.conv1.b", d, &a->conv1_b) ||
        upload_f32(a, f, "enc.conv2.w", (size_t)d * d * 3, &a->conv2_w) ||
        upload_f32(a, f, "enc.conv2.b", d, &a->conv2_b) ||
        upload_f32(a, f, "enc.ln_post.w", d, &a->ln_post_w) || upload_f32(a, f, "enc.ln_post.b", d, &a->ln_post_b))
        return -1;
    {
        // Positional embeddings: the first enc_T rows of [max_src_pos][d].
        const GgufTensor* t = need(a, f, "enc.pos_embd");
        if (!t) return -1;
        if (t->type != GGML_F32 || t->ne.size() < 2 || t->ne[0] != d || t->ne[1] < a->enc_T) {
            a->error = "enc.pos_embd must be F32 [>= encoder frames x d_model]";
            return -1;
        }
        if (au_alloc(a, &a->pos, (size_t)a->enc_T * d)) return -1;
        AU_CK(cudaMemcpy(a->pos, t->data, (size_t)a->enc_T * d * 4, cudaMemcpyHostToDevice));
    }
    size_t staging_bytes = 0;
    for (const char* nm : {"adaptor.fc1.w", "adaptor.fc2.w"})
        if (const GgufTensor* t = f.tensor(nm)) staging_bytes = std::max<size_t>(staging_bytes, t->nbytes);
    for (int l = 0; l < a->n_layers; ++l)
        for (const char* s : {"attn_q.w", "attn_k.w", "attn_v.w", "attn_out.w", "ffn_1.w", "ffn_2.w"})
            if (const GgufTensor* t = f.tensor("enc.blk." + std::to_string(l) + "." + s))
                staging_bytes = std::max<size_t>(staging_bytes, t->nbytes);
    uint8_t* staging = nullptr;
    if (au_alloc(a, &staging, staging_bytes)) return -1;
    a->layers.resize(a->n_layers);
    std::vector<float> qkv_b((size_t)3 * d);
    for (int l = 0; l < a->n_layers; ++l) {
        AudioLayer& L = a->layers[l];
        const std::string p = "enc.blk." + std::to_string(l) + ".";
        float *aw, *ab, *fw, *fbb, *ob, *b1, *b2;
        if (upload_f32(a, f, p + "attn_ln.w", d, &aw) || upload_f32(a, f, p + "attn_ln.b", d, &ab) ||
            upload_f32(a, f, p + "ffn_ln.w", d, &fw) || upload_f32(a, f, p + "ffn_ln.b", d, &fbb) ||
            upload_f32(a, f, p + "attn_out.b", d, &ob) || upload_f32(a, f, p + "ffn_1.b", a->ffn, &b1) ||
            upload_f32(a, f, p + "ffn_2.b", d, &b2))
            return -1;
        L.attn_ln_w = aw, L.attn_ln_b = ab, L.ffn_ln_w = fw, L.ffn_ln_b = fbb, L.o_b = ob, L.fc1_b = b1, L.fc2_b = b2;
        const GgufTensor* qb = need(a, f, p + "attn_q.b");
        const GgufTensor* vb = need(a, f, p + "attn_v.b");
        if (!qb || !vb) return -1;
        if (qb->type != GGML_F32 || vb->type != GGML_F32 || qb->nbytes != (size_t)d * 4 || vb->nbytes != (size_t)d * 4) {
            a->error = "attn_q.b / attn_v.b must be F32 [d_model]";
            return -1;
        }
        std::memcpy(qkv_b.data(), qb->data, (size_t)d * 4);
        std::fill(qkv_b.begin() + d, qkv_b.begin() + 2 * d, 0.0f);
        std::memcpy(qkv_b.data() + 2 * d, vb->data, (size_t)d * 4);
        float* qkvb = nullptr;
        if (au_alloc(a, &qkvb, qkv_b.size())) return -1;
        AU_CK(cudaMemcpy(qkvb, qkv_b.data(), qkv_b.size() * 4, cudaMemcpyHostToDevice));
        L.qkv_b = qkvb;
        uint8_t *wqkv, *wo, *w1, *w2;
        if (au_alloc(a, &wqkv, pf_weight_bytes(3 * d, d)) || au_alloc(a, &wo, pf_weight_bytes(d, d)) ||
            au_alloc(a, &w1, pf_weight_bytes(a->ffn, d)) || au_alloc(a, &w2, pf_weight_bytes(d, a->ffn)))
            return -1;
        if (upload_q8_steps(a, f, p + "attn_q.w", d, d, staging, wqkv, 0) ||
            upload_q8_steps(a, f, p + "attn_k.w", d, d, staging, wqkv, d) ||
            upload_q8_steps(a, f, p + "attn_v.w", d, d, staging, wqkv, 2 * d) ||
            upload_q8_steps(a, f, p + "attn_out.w", d, d, staging, wo, 0) ||
            upload_q8_steps(a, f, p + "ffn_1.w", d, a->ffn, staging, w1, 0) ||
            upload_q8_steps(a, f, p + "ffn_2.w", a->ffn, d, staging, w2, 0))
            return -1;
        L.qkv = wqkv, L.o = wo, L.fc1 = w1, L.fc2 = w2;
    }
    uint8_t *af1, *af2;
    if (au_alloc(a, &af1, pf_weight_bytes(a->hidden, a->ad_in)) || au_alloc(a, &af2, pf_weight_bytes(a->hidden, a->hidden)) ||
        upload_q8_steps(a, f, "adaptor.fc1.w", a->ad_in, a->hidden, staging, af1, 0) ||
        upload_q8_steps(a, f, "adaptor.fc2.w", a->hidden, a->hidden, staging, af2, 0) ||
        upload_f32(a, f, "adaptor.fc1.b", a->hidden, &a->ad_fc1_b) ||
        upload_f32(a, f, "adaptor.fc2.b", a->hidden, &a->ad_fc2_b) ||
        upload_f32(a, f, "adaptor.ln.w", a->hidden, &a->ad_ln_w) || upload_f32(a, f, "adaptor.ln.b", a->hidden, &a->ad_ln_b))
        return -1;
    a->ad_fc1 = af1, a->ad_fc2 = af2;
    // One chunk's scratch.
    const int T = a->enc_T, kmax = std::max(d, a->ffn);
    if (au_alloc(a, &a->samples, a->n_samples) || au_alloc(a, &a->mel, (size_t)a->n_mels * a->n_frames) ||
        au_alloc(a, &a->frame_max, a->n_frames) || au_alloc(a, &a->c1, (size_t)a->n_frames * d) ||
        au_alloc(a, &a->h, (size_t)T * d) || au_alloc(a, &a->nrm, (size_t)T * d) ||
        au_alloc(a, &a->qkv, (size_t)T * 3 * d) || au_alloc(a, &a->att, (size_t)T * d) ||
        au_alloc(a, &a->f, (size_t)T * a->ffn) || au_alloc(a, &a->xq, pf_act_bytes(T, kmax)) ||
        au_alloc(a, &a->xd, (size_t)T * (kmax / 32)) || au_alloc(a, &a->status, 1))
        return -1;
    AU_CK(cudaMemset(a->status, 0, sizeof(int)));
    AU_CK(pf_configure());
    AU_CK(cudaFuncSetAttribute(k_enc_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttSmem));
    const int mel_smem = a->n_bins * 8 + a->n_fft * 4;
    if (mel_smem > 48 * 1024) AU_CK(cudaFuncSetAttribute(k_mel_frames, cudaFuncAttributeMaxDynamicSharedMemorySize, mel_smem));
    AU_CK(cudaStreamCreateWithFlags(&a->stream, cudaStreamNonBlocking));
    AU_CK(cudaEventCreate(&a->ev[0]));
    AU_CK(cudaEventCreate(&a->ev[1]));
    AU_CK(cudaDeviceSynchronize());
    return 0;
}

// Grow the concatenation and adaptor buffers to `frames` encoder frames.
int ensure_frames(mtb_audio* a, int frames) {
    if (frames <= a->cap_frames) return 0;
    AU_CK(cudaStreamSynchronize(a->stream));
    for (void* p : a->grown) cudaFree(p);
    a->grown.clear();
    a->cap_frames = 0;
    const int N = frames / a->merge + 1;
    const int kmax = std::max(a->ad_in, a->hidden);
    void* p[6] = {};
    const size_t sizes[6] = {(size_t)frames * a->d * 4, (size_t)N * a->hidden * 4, (size_t)N * a->hidden * 4,
                             (size_t)N * a->hidden * 4, pf_act_bytes(N, kmax), (size_t)N * (kmax / 32) * 4};
    for (int i = 0; i < 6; ++i) {
        cudaError_t e = cudaMalloc(&p[i], sizes[i]);
        if (e != cudaSuccess) {
            for (int j = 0; j < i; ++j) cudaFree(p[j]);
            a->error = std::string("cudaMalloc: ") + cudaGetErrorString(e);
            return -1;
        }
        a->grown.push_back(p[i]);
    }
    a->enc_all = (float*)p[0], a->a1 = (float*)p[1], a->a2 = (float*)p[2], a->out = (float*)p[3];
    a->axq = (uint8_t*)p[4], a->axd = (float*)p[5];
    a->cap_frames = frames;
    return 0;
}

// Mel + encoder of one chunk (samples already in a->samples, padded).  The
// final LayerNorm writes the first `rows` frames to dst [rows][d].
void encode_chunk(mtb_audio* a, float* dst, int rows) {
    cudaStream_t s = a->stream;
    const int d = a->d, T = a->enc_T;
    k_mel_frames<<<a->n_frames, kMelThreads, a->n_bins * 8 + a->n_fft * 4, s>>>(
        a->samples, a->n_samples, a->n_fft, a->hop, a->window, a->cos_t, a->sin_t, a->n_bins, a->fb, a->n_mels,
        a->n_frames, a->mel, a->frame_max);
    const int count = a->n_mels * a->n_frames;
    k_mel_finish<<<std::min((count + 255) / 256, 1184), 256, 0, s>>>(a->mel, count, a->frame_max, a->n_frames);
    k_conv_gelu<<<dim3((a->n_frames + kCvT - 1) / kCvT, d / kCvO), 256, 0, s>>>(
        a->mel, a->n_frames, a->n_mels, 1, a->n_frames, 1, a->conv1_w, a->conv1_b, nullptr, d, a->n_frames, a->c1);
    k_conv_gelu<<<dim3((T + kCvT - 1) / kCvT, d / kCvO), 256, 0, s>>>(a->c1, a->n_frames, d, d, 1, 2, a->conv2_w,
                                                                      a->conv2_b, a->pos, d, T, a->h);
    const float scale = 1.0f / std::sqrt((float)kHd);
    const int ln_grid = (T + 7) / 8;
    for (int l = 0; l < a->n_layers; ++l) {
        const AudioLayer& L = a->layers[l];
        k_layer_norm<<<ln_grid, 256, 0, s>>>(a->h, d, T, d, L.attn_ln_w, L.attn_ln_b, 1e-5f, a->nrm, d);
        pf_quant(a->nrm, T, d, a->xq, a->xd, s);
        pf_gemm_bias(L.qkv, 3 * d, d, a->xq, a->xd, T, a->qkv, 3 * d, PF_EPI_BIAS, L.qkv_b, a->status, s);
        k_enc_attn<<<dim3((T + kAttQ - 1) / kAttQ, a->n_heads), 256, kAttSmem, s>>>(a->qkv, T, d, scale, a->att);
        pf_quant(a->att, T, d, a->xq, a->xd, s);
        pf_gemm_bias(L.o, d, d, a->xq, a->xd, T, a->h, d, PF_EPI_BIAS_RESID, L.o_b, a->status, s);
        k_layer_norm<<<ln_grid, 256, 0, s>>>(a->h, d, T, d, L.ffn_ln_w, L.ffn_ln_b, 1e-5f, a->nrm, d);
        pf_quant(a->nrm, T, d, a->xq, a->xd, s);
        pf_gemm_bias(L.fc1, a->ffn, d, a->xq, a->xd, T, a->f, a->ffn, PF_EPI_BIAS_GELU, L.fc1_b, a->status, s);
        pf_quant(a->f, T, a->ffn, a->xq, a->xd, s);
        pf_gemm_bias(L.fc2, d, a->ffn, a->xq, a->xd, T, a->h, d, PF_EPI_BIAS_RESID, L.fc2_b, a->status, s);
    }
    k_layer_norm<<<(rows + 7) / 8, 256, 0, s>>>(a->h, d, rows, d, a->ln_post_w, a->ln_post_b, 1e-5f, dst, d);
}

// Adaptor over `frames` concatenated encoder frames (a multiple of merge):
// rows [frames / merge][ad_in] -> a->out [N][hidden].
void run_adaptor(mtb_audio* a, int frames) {
    cudaStream_t s = a->stream;
    const int N = frames / a->merge;
    pf_quant(a->enc_all, N, a->ad_in, a->axq, a->axd, s);
    pf_gemm_bias(a->ad_fc1, a->hidden, a->ad_in, a->axq, a->axd, N, a->a1, a->hidden, PF_EPI_BIAS_SILU, a->ad_fc1_b,
                 a->status, s);
    pf_quant(a->a1, N, a->hidden, a->axq, a->axd, s);
    pf_gemm_bias(a->ad_fc2, a->hidden, a->hidden, a->axq, a->axd, N, a->a2, a->hidden, PF_EPI_BIAS, a->ad_fc2_b,
                 a->status, s);
    k_layer_norm<<<(N + 7) / 8, 256, 0, s>>>(a->a2, a->hidden, N, a->hidden, a->ad_ln_w, a->ad_ln_b, a->ad_eps, a->out,
                                             a->hidden);
}

// Sum of token_len over the 30 s chunks (src/audio_encoder.cpp:45-49).
long long tokens_for(const mtb_audio* a, long long n) {
    const long long stride = (long long)a->hop * 2 * a->merge;
    long long total = 0;
    for (long long off = 0; off < n; off += a->n_samples) {
        const long long unpadded = std::min<long long>(a->n_samples, n - off);
        total += (unpadded - 1) / stride + 1;
    }
    return total;
}

int check_status(mtb_audio* a) {
    int st = 0;
    AU_CK(cudaGetLastError());
    AU_CK(cudaMemcpyAsync(&st, a->status, sizeof(int), cudaMemcpyDeviceToHost, a->stream));
    AU_CK(cudaStreamSynchronize(a->stream));
    if (st) {
        a->error = "a tensor-core GEMM wait timed out";
        cudaMemsetAsync(a->status, 0, sizeof(int), a->stream);
        return -1;
    }
    return 0;
}

int upload_chunk(mtb_audio* a, const float* samples, long long n_left) {
    const long long unpadded = std::min<long long>(a->n_samples, n_left);
    AU_CK(cudaMemcpyAsync(a->samples, samples, (size_t)unpadded * 4, cudaMemcpyHostToDevice, a->stream));
    if (unpadded < a->n_samples)
        AU_CK(cudaMemsetAsync(a->samples + unpadded, 0, (size_t)(a->n_samples - unpadded) * 4, a->stream));
    return 0;
}

}  // namespace

extern "C" {

int mtb_audio_load(const char* gguf_path, int device, mtb_audio** out) {
    if (!out || !gguf_path) {
        g_audio_error = "null argument";
        return -1;
    }
    *out = nullptr;
    try {
        int n_dev = 0;
        if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev <= 0) {
            g_audio_error = "no CUDA device: this library has no CPU path";
            cudaGetLastError();
            return -2;
        }
        if (device < 0 || device >= n_dev) {
            g_audio_error = "device index out of range";
            return -2;
        }
        DeviceGuard guard(device);
        cudaDeviceProp prop{};
        cudaGetDeviceProperties(&prop, device);
        if (prop.major != 10) {
            g_audio_error = "this library is built for sm_100a (B200)";
            return -2;
        }
        auto* a = new mtb_audio();
        a->device = device;
        if (load_audio(a, gguf_path)) {
            g_audio_error = a->error;
            delete a;
            return -1;
        }
        *out = a;
        return 0;
    } catch (const std::exception& e) {
        g_audio_error = e.what();
        return -1;
    }
}

void mtb_audio_free(mtb_audio* a) {
    if (!a) return;
    DeviceGuard guard(a->device);
    delete a;
}

const char* mtb_audio_error(const mtb_audio* a) { return a ? a->error.c_str() : g_audio_error.c_str(); }

int mtb_audio_dims(const mtb_audio* a, int32_t* dims) {
    if (!a || !dims) return -1;
    const int32_t v[10] = {a->hidden, a->d, a->n_layers, a->n_heads, a->ffn, a->n_mels, a->n_frames, a->n_samples,
                           a->enc_T, a->merge};
    std::memcpy(dims, v, sizeof(v));
    return 0;
}

int mtb_audio_tokens(const mtb_audio* a, int n_samples) {
    if (!a || n_samples <= 0) return -1;
    const long long t = tokens_for(a, n_samples);
    return t > INT32_MAX ? -1 : int(t);
}

int mtb_audio_encode(mtb_audio* a, const float* samples16k, int n_samples, float* out, int max_tokens,
                     int* n_tokens) {
    if (!a) return -1;
    if (n_tokens) *n_tokens = 0;
    if (!samples16k || !out || !n_tokens) {
        a->error = "null argument";
        return -1;
    }
    if (n_samples <= 0) {
        a->error = "AudioEncoder: empty input samples";
        return -1;
    }
    try {
        DeviceGuard guard(a->device);
        const long long total = tokens_for(a, n_samples);
        if (total > max_tokens) {
            a->error = "output holds " + std::to_string(max_tokens) + " rows, the audio gives " + std::to_string(total);
            return -1;
        }
        const long long frames = total * a->merge;
        if (frames > INT32_MAX / 2) {
            a->error = "audio too long";
            return -1;
        }
        if (ensure_frames(a, int(frames))) return -1;
        const long long stride = (long long)a->hop * 2 * a->merge;
        AU_CK(cudaEventRecord(a->ev[0], a->stream));
        long long row = 0;
        for (long long off = 0; off < n_samples; off += a->n_samples) {
            const long long unpadded = std::min<long long>(a->n_samples, n_samples - off);
            const int token_len = int((unpadded - 1) / stride + 1);
            const int trim = token_len * a->merge;
            if (trim > a->enc_T) {
                a->error = "AudioEncoder: trim exceeds the encoder frames";
                return -1;
            }
            if (upload_chunk(a, samples16k + off, n_samples - off)) return -1;
            encode_chunk(a, a->enc_all + row * a->d, trim);
            row += trim;
        }
        run_adaptor(a, int(frames));
        AU_CK(cudaMemcpyAsync(out, a->out, (size_t)total * a->hidden * 4, cudaMemcpyDeviceToHost, a->stream));
        AU_CK(cudaEventRecord(a->ev[1], a->stream));
        if (check_status(a)) return -1;
        cudaEventElapsedTime(&a->last_ms, a->ev[0], a->ev[1]);
        *n_tokens = int(total);
        return 0;
    } catch (const std::exception& e) {
        a->error = e.what();
        return -1;
    }
}

float mtb_audio_last_ms(const mtb_audio* a) { return a ? a->last_ms : -1.f; }

int mtb_audio_debug_chunk(mtb_audio* a, const float* samples, int n_samples, float* mel_out, float* enc_out) {
    if (!a) return -1;
    if (!samples || n_samples <= 0 || n_samples > a->n_samples) {
        a->error = "debug_chunk takes 1 .. chunk samples";
        return -1;
    }
    try {
        DeviceGuard guard(a->device);
        if (ensure_frames(a, a->enc_T)) return -1;
        if (upload_chunk(a, samples, n_samples)) return -1;
        encode_chunk(a, a->enc_all, a->enc_T);
        if (mel_out)
            AU_CK(cudaMemcpyAsync(mel_out, a->mel, (size_t)a->n_mels * a->n_frames * 4, cudaMemcpyDeviceToHost,
                                  a->stream));
        if (enc_out)
            AU_CK(cudaMemcpyAsync(enc_out, a->enc_all, (size_t)a->enc_T * a->d * 4, cudaMemcpyDeviceToHost, a->stream));
        return check_status(a);
    } catch (const std::exception& e) {
        a->error = e.what();
        return -1;
    }
}

}  // extern "C"
