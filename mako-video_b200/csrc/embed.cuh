// The step's small kernels around the blocks: the fp32 time-embedding MLP, the AdaLN projections of every block
// (an HBM-bound multi-vector GEMV over bf16 weights) and the fp32 output heads.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace h3 {

enum class Act : int { none = 0, silu = 1 };

// out[u][n] = act(sum_k W[n][k] * x[u][k] + b[n]) for u < U (fp32 weights [N][K]); when out_silu_bf16 is given it
// also receives bf16(silu(out[u][n])) as a float (the AdaLN projections' input).
void gemv_f32(const float* W, const float* b, const float* x, int U, int N, int K, Act act, float* out, float* out_silu_bf16,
              cudaStream_t s);

// AdaLN projections: for each group g of G weight rows (bf16 [groups * G][K]),
// out[(g * U + u) * G + j] = sum_k W[g * G + j][k] * x[u][k] + b[g * G + j].
void adaln_gemv(const void* W_bf16, const float* b, const float* x, int U, int groups, int G, int K, float* out, cudaStream_t s);

// Pruned checkpoints' AdaLN projections (curve_mods): for each group g of G weight rows (fp32 [groups * G][K], K <= 16),
// out[(g * U + u) * G + j] = sum_k W[g * G + j][k] * c[u][k] + b[g * G + j], c the curve points [U][K].
void curve_mods(const float* W, const float* b, const float* c, int U, int groups, int G, int K, float* out, cudaStream_t s);

// out[r * ldo + j] = sum_k x[r][k] * W[j][k] + b[j]  (fp32; N <= 128, K a multiple of 32)
void heads_f32(const float* x, int64_t ldx, int rows, const float* W, const float* b, int N, int K, float* out, int64_t ldo,
               cudaStream_t s);

} // namespace h3
