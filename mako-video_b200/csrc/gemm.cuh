// Parameters of the tcgen05 projection GEMM and the epilogues fused into it.
//   D[M][N] = A[M][K] * B[N][K]^T   (A: activations, row-major, K contiguous; B: weights as stored, [out][in])
// A may be split into `a_chunks` column chunks stored one after another ([chunks][M][K / chunks]), which is how the
// attention output arrives after the sequence-parallel all-to-all.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace h3 {

enum class Epi : int {
    bf16 = 0,       // out (bf16) = acc + bias
    f32 = 1,        // out (f32)  = acc + bias
    qkv = 2,        // q/k: per-head RMS norm * weight, then rotary; v: + bias; bf16 into the head-split layout
    gate_resid = 3, // x (f32) += gate[row's modulation] * (acc + bias)
    swiglu = 4,     // out (bf16) = silu(gate + bg) * (value + bv); B's rows interleaved in 128-row gate/value groups
    s32 = 5,        // out (int32) = raw accumulator (int8 GEMM only)
};

struct GemmParams {
    int M = 0, N = 0, K = 0;
    int a_chunks = 1; // A split into this many consecutive column chunks of K / a_chunks
    int a_rows_stride = 0; // rows per chunk in A's storage (>= M); 0: M
    int lda = 0;      // A's row pitch in elements (one chunk's width when chunked); 0: K / a_chunks
    int ldb = 0;      // B's row pitch in elements; 0: K
    // epilogue
    void* out = nullptr;
    int64_t ldo = 0;
    const float* bias = nullptr;
    float* x = nullptr; // residual stream for gate_resid
    int64_t ldx = 0;
    const float* mod = nullptr;        // this block's modulation table [n_mod][6][dim]
    const uint8_t* mod_idx = nullptr;  // per row: which (level, modality) modulation it reads
    int gate_slot = 0;                 // 2: the attention gate, 5: the FFN gate
    int dim = 0;
    const float* rope = nullptr; // [M][48][2] (cos, sin) per row
    const float* qn_w = nullptr; // [128]
    const float* kn_w = nullptr; // [128]
    float eps = 1e-6f;
    int inner = 0;          // heads * 128
    int heads_per_rank = 0; // heads each rank attends (all heads with one rank)
    int rows_local = 0;     // rows of this rank (the qkv layout's per-destination block)
    // Sequence parallel with the exchange fused into the epilogue: rank r's receive buffer ([P x rows_local][3]
    // [heads_per_rank][128], this rank's rows at block my_rank), mapped into this process (null: use `out`).
    void* peer_out[8] = {};
    int my_rank = 0;
    const float* a_scale = nullptr; // int8: per-row activation scale
    const float* b_scale = nullptr; // int8: per-output-row weight scale
};

// bf16 x bf16 -> fp32 (tcgen05 kind::f16). A and B are device pointers; the epilogue arguments live in `p`.
void gemm_bf16(const void* A, const void* B, const GemmParams& p, Epi epi, cudaStream_t s);
// int8 x int8 -> int32 (tcgen05 kind::i8), dequantised by a_scale[row] * b_scale[col] before the epilogue.
void gemm_s8(const void* A, const void* B, const GemmParams& p, Epi epi, cudaStream_t s);

} // namespace h3
