// Block-sparse attention's coarse pass: cube means of q and k per head, cube-pair scores, the per-query-cube top
// selection with forced local cubes, and the pass lists the sparse flash kernel walks.
//
// Arithmetic (fixed so that a CPU restatement reproduces every selected index bit for bit):
//   mean  m[c][d] = (sum over the cube's rows in (frame, row, column) order of float(x[row][d])) / count, fp32 adds
//   score s[i][j] = fmaf chain over d = 0..127 in order: acc = fmaf(mq[i][d], mk[j][d], acc), acc starting at 0
//   pick  per query cube i: the forced cubes (itself; with local 3 also the cubes one frame group before and after at
//         the same spatial position), then the highest scores among the rest until max(k, forced) are chosen;
//         equal scores go to the lower cube index; k = ceil(ratio * cubes) (at least 1, at most cubes).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "attention.cuh"

namespace h3 {

int sparse_k(float ratio, int cubes);
int sparse_forced(int local); // forced cubes at most (1 or 3; 0 when local is 0)

struct SparseBuffers {
    float* mq = nullptr;      // [heads][cubes][128]
    float* mk = nullptr;      // [heads][cubes][128]
    float* scores = nullptr;  // [heads][cubes][cubes]
    int32_t* sel = nullptr;   // [heads][cubes][kcap] ascending cube indices
    int32_t* nsel = nullptr;  // [heads][cubes]
    int kcap = 0;
    int4* blocks = nullptr;   // [heads][q_tiles][max_blocks]
    int32_t* nblocks = nullptr; // [heads][q_tiles]
    int4* q_rows = nullptr;   // [q_tiles]
    int q_tiles = 0, max_blocks = 0;
};

// Sizes for a grid: kcap, q_tiles and max_blocks.
void sparse_sizes(const CubeGrid& g, float ratio, int local, int& kcap, int& q_tiles, int& max_blocks);

// q, k: (row, head, dim) at base + row * row_stride + head * 128 + dim (bf16), packed row order (each cube's rows
// consecutive).
void cube_pool(const void* q, const void* k, int64_t row_stride, int heads, const CubeGrid& g, float* mq, float* mk, cudaStream_t s);
void cube_scores(const float* mq, const float* mk, int heads, int cubes, float* scores, cudaStream_t s);
void cube_topk(const float* scores, int heads, const CubeGrid& g, int k, int local, int32_t* sel, int32_t* nsel, int kcap,
               cudaStream_t s);
// Pass lists from the selections; q_rows is written too (the same for every head).
void build_passes(const int32_t* sel, const int32_t* nsel, int kcap, int heads, const CubeGrid& g, int4* blocks, int32_t* nblocks,
                  int4* q_rows, int q_tiles, int max_blocks, cudaStream_t s);

// The whole coarse pass and the sparse attention for `heads` heads.
void sparse_attention(const AttnParams& dense_args, const CubeGrid& g, float ratio, int local, const SparseBuffers& b, cudaStream_t s);

} // namespace h3
