// Prefill projections on tcgen05 (prefill_tc.cu).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace mtb {

enum PfEpilogue {
    PF_EPI_STORE = 0,
    PF_EPI_RESID = 1,
    PF_EPI_SWIGLU = 2,
    // With a per-row bias (the Whisper encoder and the audio adaptor):
    PF_EPI_BIAS = 3,        // y = acc + b
    PF_EPI_BIAS_GELU = 4,   // y = gelu_erf(acc + b)
    PF_EPI_BIAS_SILU = 5,   // y = silu(acc + b)
    PF_EPI_BIAS_RESID = 6,  // y = y + (acc + b)
};

// Bytes of a matrix in prefill weight steps (n_rows a multiple of 128, K of 256).
size_t pf_weight_bytes(int n_rows, int K);
// Bytes of T activation rows in prefill activation steps (T padded to 32).
size_t pf_act_bytes(int T, int K);
cudaError_t pf_configure();
// GGUF q8_0 rows -> weight steps.  half < 0: n_src rows fill whole 128-row
// tiles (n_src a multiple of 128); half 0 / 1: gate / up rows of a gate/up
// pair, tile f / 64 rows 64 half + f % 64 (n_src a multiple of 64).
void pf_repack(const uint8_t* src_q8, int n_src, int K, int half, uint8_t* dst, cudaStream_t s);
// RMSNorm (optionally storing the normed rows) + q8_0 quantisation of T rows.
void pf_norm_quant(const float* x, int T, int K, const float* w, float eps, uint8_t* xq, float* xd, float* normed,
                   cudaStream_t s);
void pf_quant(const float* x, int T, int K, uint8_t* xq, float* xd, cudaStream_t s);
// y[T][ldy] (=, +=, or SwiGLU into 64-feature groups) from weight steps and activation steps.
void pf_gemm(const uint8_t* w, int n_rows, int K, const uint8_t* xq, const float* xd, int T, float* y, int ldy, int epi,
             int* status, cudaStream_t s);
// The same with a bias b[n_rows] and one of the PF_EPI_BIAS* epilogues.
void pf_gemm_bias(const uint8_t* w, int n_rows, int K, const uint8_t* xq, const float* xd, int T, float* y, int ldy,
                  int epi, const float* bias, int* status, cudaStream_t s);

}  // namespace mtb
