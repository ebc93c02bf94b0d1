// Row kernels of the H3 step (HBM-bound): modulated RMS norm, gated residual add, SwiGLU, per-row int8
// quantisation, the standalone per-head q/k norm + rotary, and the small helpers around the step (fp32 -> bf16
// row packing, synthetic weight generation, weight quantisation).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace h3 {

enum class RowOut : int { bf16 = 0, f32 = 1, s8 = 2 };

// y[r] = RMSNorm(x[r]) (* w if given) * (1 + scale) + shift, the shift and scale picked by mod_idx[r] from
// mod[(idx * mod_slots + slot) * d]. RowOut::s8 also writes the row's int8 quantisation and its scale.
struct RmsModParams {
    const float* x = nullptr;
    int64_t ldx = 0;
    int rows = 0, d = 0;
    const float* w = nullptr; // norm weight [d] or null
    const float* mod = nullptr;
    const uint8_t* mod_idx = nullptr;
    int mod_slots = 6, shift_slot = 0, scale_slot = 1;
    float eps = 1e-6f;
    RowOut out_kind = RowOut::bf16;
    void* out = nullptr;
    int64_t ldo = 0;
    float* out_scale = nullptr; // s8 only
};
void rms_mod_rows(const RmsModParams& p, cudaStream_t s);

// x[r][c] += gate[mod_idx[r]][c] * y[r][c]   (y bf16)
void gate_add_rows(float* x, int64_t ldx, const void* y_bf16, int64_t ldy, int rows, int d, const float* mod,
                   const uint8_t* mod_idx, int gate_slot, cudaStream_t s);

// out[r][c] = silu(gv[r][c]) * gv[r][F + c]   (bf16 in and out; gv holds [gate; value] halves)
void swiglu_rows(const void* gv_bf16, int rows, int F, void* out_bf16, cudaStream_t s);

// Symmetric per-row int8: scale = max|x| / 127, q = rint(x * (127 / max|x|)) clamped to +-127 (0 for a zero row).
void quant_rows_i8(const void* x_bf16, int64_t ldx, int rows, int K, int8_t* q, float* scale, cudaStream_t s);
// The same for rows split into `chunks` column chunks stored one after another ([chunks][rows_stride][K / chunks]);
// q is written as dense [rows][K].
void quant_rows_i8_chunked(const void* x_bf16, int rows, int K, int chunks, int rows_stride, int8_t* q, float* scale, cudaStream_t s);

// The standalone heads_partial: per-head RMS norm (weights qn/kn) and rotary of q and k inside a
// [rows][3][heads][128] bf16 tensor, in place; v untouched.
void heads_partial(void* qkv_bf16, int rows, int heads, const float* qn_w, const float* kn_w, const float* rope, float eps,
                   cudaStream_t s);

// fp32 rows -> bf16 rows of width ld_out (zero padding past `cols`); output row r reads input row src_rows[r] when
// src_rows is given.
void pack_bf16_rows(const float* in, int rows, int cols, void* out_bf16, int ld_out, cudaStream_t s, const int32_t* src_rows = nullptr);

// The sampler's Euler move of n values in place (src/video/engine.cpp:705-711): x0 = x + (1 - t) v, then
// x = r x + (1 - r) x0 with r = sigma_next / sigma, every operation rounded on its own (no fused multiply-add).
void euler_rows(float* x, const float* v, size_t n, float t, float sigma, float sigma_next, cudaStream_t s);

// dst[r][c] = src[idx[r]][c] for c < cols (fp32).
void gather_rows_f32(const float* src, int64_t lds, const int32_t* idx, int rows, int cols, float* dst, int64_t ldd, cudaStream_t s);

// Synthetic parameters: value i of tensor `tensor_id` = mean + std * IH4(seed, tensor_id, i), IH4 the centred sum of
// four 16-bit uniforms from a splitmix64 hash (an Irwin-Hall approximation of a unit normal), computed with exact
// integer arithmetic and one fp32 rounding so that the CPU oracle regenerates identical bits.
void fill_synthetic(void* dst, int is_bf16, uint64_t n, uint64_t seed, uint32_t tensor_id, float mean, float stdev, cudaStream_t s);

// Per-output-row int8 quantisation of a bf16 weight [rows][K]: scale[r] = max|w_r| / 127.
void quant_weight_rows(const void* w_bf16, int rows, int K, int8_t* q, float* scale, cudaStream_t s);

// LoRA merge (W += s * B A): for i < out, j < in, W[row_map[i]][j] = bf16(base + s * sum_k B[i][k] A[k][j]) with B
// [out][r] and A [r][in] fp32, base the current bf16 weight, or q[row][j] * qscale[row] when q (int8 rows) is given.
void lora_merge(const float* B, const float* A, int out, int in, int r, float s, const int32_t* row_map, void* W_bf16, int64_t ldw,
                const int8_t* q, const float* qscale, cudaStream_t st);

// Permute fc1's rows from [gate (F); value (F)] to 128-row groups [gate g; value g] for the fused SwiGLU epilogue.
void interleave_gate_value(const void* w_bf16, int F, int K, void* out_bf16, cudaStream_t s);
void interleave_gate_value_f32(const float* b, int F, float* out, cudaStream_t s);

} // namespace h3
