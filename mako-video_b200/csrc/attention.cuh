// Flash attention for the H3 step on sm_100a tensor cores: bidirectional softmax(q k^T / sqrt(128)) v over
// 128-wide heads, dense (every key) or block-sparse over 4x4x4 latent cubes (Video Sparse Attention's training-free
// form as the reference runs it: a pass list per query tile of selected cubes plus every dense row).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#ifdef __CUDACC__
#define H3_HD __host__ __device__
#else
#define H3_HD
#endif

namespace h3 {

// The sparse attention's units: 64-row tiles, either a 4x4x4 cube of the generated video rows (latent frame, patch
// row, patch column; the grid padded to multiples of 4 with rows that are no token) or 64 consecutive dense rows
// (text, conditioning and audio rows, which precede the generated video rows). Units 0 .. cubes-1 are the cubes in
// (frame group, row group, column group) order; units cubes .. cubes+dense_units-1 the dense chunks.
struct CubeGrid {
    int dense_rows = 0; // D: rows before the generated video rows
    int frames = 0, ph = 0, pw = 0; // generated video rows as [frames][ph][pw]
    int nct = 0, ncy = 0, ncx = 0;  // cubes per axis (ceil of the grid / 4)
    H3_HD int cubes() const { return nct * ncy * ncx; }
    H3_HD int dense_units() const { return (dense_rows + 63) / 64; }
    H3_HD int units() const { return cubes() + dense_units(); }
};

struct AttnParams {
    // q, k, v: element (row, head, dim) at base + row * row_stride + head * 128 + dim (bf16), rows in model order
    const void* q = nullptr;
    const void* k = nullptr;
    const void* v = nullptr;
    int64_t row_stride = 0; // elements between consecutive rows of q, k and v
    int heads = 0;          // heads addressed by the q/k/v tensors
    int rows = 0;           // dense mode: query and key rows (keys at or past `rows` are masked)
    void* out = nullptr;    // o: (row, head, dim) at out + row * out_row_stride + head * 128 + dim
    int64_t out_row_stride = 0;
    // Sequence parallel with the exchange fused into the epilogue: row R's output goes straight to its owner
    // R / rows_per_rank, into that rank's [P][rows_per_rank][heads x 128] buffer (block my_rank), mapped into this
    // process (peer_out[0] null: write `out`).
    void* peer_out[8] = {};
    int rows_per_rank = 0, my_rank = 0;
    float scale = 0.08838834764831845f; // 1 / sqrt(128)

    // Sparse mode (blocks != null). Query tile t is the unit pair q_units[t]; for head h it visits
    // nblocks[h * q_tiles + t] key blocks blocks[(h * q_tiles + t) * max_blocks + j] = (unit a, unit b, keep, 0): keys
    // of unit a then unit b (b = -1: none), `keep` bit (2 * qh + kh) set when query half qh may see key unit kh.
    const int4* blocks = nullptr;
    const int32_t* nblocks = nullptr;
    const int2* q_units = nullptr;
    int q_tiles = 0;
    int max_blocks = 0;
    CubeGrid grid;
};

void attention(const AttnParams& p, cudaStream_t s);

} // namespace h3
