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

// The sparse attention's units, 64-row key/query tiles: either a 4x4x4 cube of the generated video rows (latent
// frame, patch row, patch column; cubes at the grid's far edges are cut short) or 64 consecutive dense rows (text,
// conditioning and audio rows, which precede the generated video rows). Units 0 .. cubes-1 are the cubes in
// (frame group, row group, column group) order; units cubes .. cubes+dense_units-1 the dense chunks.
//
// Packed row order: the generated video rows are stored cube by cube, in unit order, each cube's rows in (frame, row,
// column) order with no padding, so that every cube is one run of consecutive rows. A cube of nf x ny x nx rows
// (each at most 4) starting at latent position (4 ct, 4 cy, 4 cx) begins at
//     dense_rows + 4 ct ph pw + nf (4 cy pw + ny 4 cx).
struct CubeGrid {
    int dense_rows = 0; // D: rows before the generated video rows
    int frames = 0, ph = 0, pw = 0; // generated video rows as [frames][ph][pw]
    int nct = 0, ncy = 0, ncx = 0;  // cubes per axis (ceil of the grid / 4)
    H3_HD int cubes() const { return nct * ncy * ncx; }
    H3_HD int dense_units() const { return (dense_rows + 63) / 64; }
    H3_HD int units() const { return cubes() + dense_units(); }
    H3_HD int video_rows() const { return frames * ph * pw; }
    H3_HD int rows() const { return dense_rows + video_rows(); }
    // First packed row and row count of unit u.
    H3_HD void unit_span(int u, int& first, int& n) const
    {
        if (u < cubes()) {
            const int cx = u % ncx, cy = (u / ncx) % ncy, ct = u / (ncx * ncy);
            const int nx = pw - 4 * cx < 4 ? pw - 4 * cx : 4, ny = ph - 4 * cy < 4 ? ph - 4 * cy : 4;
            const int nf = frames - 4 * ct < 4 ? frames - 4 * ct : 4;
            first = dense_rows + 4 * ct * ph * pw + nf * (4 * cy * pw + ny * 4 * cx);
            n = nf * ny * nx;
        } else {
            first = (u - cubes()) * 64;
            n = dense_rows - first < 64 ? dense_rows - first : 64;
        }
    }
    // Packed row of generated video row (f, y, x).
    H3_HD int video_pos(int f, int y, int x) const
    {
        const int ct = f >> 2, cy = y >> 2, cx = x >> 2;
        int first, n;
        unit_span((ct * ncy + cy) * ncx + cx, first, n);
        const int nx = pw - 4 * cx < 4 ? pw - 4 * cx : 4, ny = ph - 4 * cy < 4 ? ph - 4 * cy : 4;
        return first + ((f & 3) * ny + (y & 3)) * nx + (x & 3);
    }
};

struct AttnParams {
    // q, k, v: element (row, head, dim) at base + row * row_stride + head * head_dim + dim (bf16), rows in model order
    const void* q = nullptr;
    const void* k = nullptr;
    const void* v = nullptr;
    int64_t row_stride = 0; // elements between consecutive rows of q, k and v
    int heads = 0;          // heads addressed by the q/k/v tensors
    int rows = 0;           // query and key rows (sparse mode: grid.rows())
    int head_dim = 128;     // 128, or 64 (dense mode only; the video decoder's heads)
    // Dense mode: the rows as independent segments of seg_rows rows, one every seg_stride rows (0: one segment of
    // `rows`); queries see the keys of their own segment only.
    int seg_rows = 0;
    int64_t seg_stride = 0;
    void* out = nullptr;    // o: (row, head, dim) at out + row * out_row_stride + head * head_dim + dim
    int64_t out_row_stride = 0;
    // Sequence parallel with the exchange fused into the epilogue: row R's output goes straight to its owner
    // R / rows_per_rank, into that rank's [P][rows_per_rank][heads x 128] buffer (block my_rank), mapped into this
    // process (peer_out[0] null: write `out`).
    void* peer_out[8] = {};
    int rows_per_rank = 0, my_rank = 0;
    float scale = 0.08838834764831845f; // 1 / sqrt(head_dim)
    // Dense mode, launches of few waves: scratch for a key range split in two (null: never split). part_o
    // [2][rows][heads][128] fp32 receives each half's unnormalised output and part_ml [2][rows][heads][2] its row
    // maximum (log2 units) and sum; a combine kernel merges the halves into `out`. Sized by attention_split_bytes.
    float* part_o = nullptr;
    float* part_ml = nullptr;

    // Sparse mode (blocks != null; rows in the packed order above). Query tile t is two units (two cubes, or two
    // chunks of dense rows), q_rows[t] = (first row a, first row b or -1, rows of a, rows of b); each unit has its
    // own key list. For head h the tile takes nblocks[h * q_tiles + t] steps; step j has one entry per query unit,
    // blocks[(h * q_tiles + t) * max_blocks + 2 j + x] = (first row of key unit 0, of key unit 1 or -1, rows of unit 0
    // | rows of unit 1 << 8, 0): 64 keys from each first row, of which the unit's row count are its tokens (an entry
    // of -1s is padding). nblocks -1: both query units see every row (128-row blocks over all rows).
    const int4* blocks = nullptr;
    const int32_t* nblocks = nullptr;
    const int4* q_rows = nullptr;
    int q_tiles = 0;
    int max_blocks = 0;
    CubeGrid grid;
    // A bound on every score q.k scale log2(e) when one is known (q and k RMS-normed per head: qk_score_bound), at
    // most kMaxStaticBound. The softmax then takes it for the row maximum: no running maximum, no exchange of it between
    // a row's warps, no rescaling of O. 0: unknown (the online maximum).
    float static_max = 0.f;
};

// The largest score bound (log2 units) the attention takes in place of the row maximum. A row's largest P is
// 2^(s_max - bound) >= 2^(-2 bound) = 2^-80, so a key is flushed to zero (P below 2^-125) only when its score is more
// than 45 below the row's largest, where its weight is below 2^-45 of that one.
constexpr float kMaxStaticBound = 40.f;

// The score bound of q and k RMS-normed per head of head_dim dims with weights of largest magnitudes wq and wk (1 for
// an unweighted norm): |q| <= sqrt(head_dim) wq and |k| <= sqrt(head_dim) wk (the rotary embedding preserves norms),
// so q.k / sqrt(head_dim) <= sqrt(head_dim) wq wk; times log2(e), with room for the bf16 rounding of q and k. 0 when
// it is above kMaxStaticBound.
inline float qk_score_bound(float wq, float wk, int head_dim = 128)
{
    const float b = (head_dim == 64 ? 11.5416f : 16.3222f) * wq * wk * 1.02f + 0.05f; // sqrt(head_dim) log2(e)
    return b <= kMaxStaticBound ? b : 0.f;
}

// Launches the attention; returns the number of kernels launched.
int attention(const AttnParams& p, cudaStream_t s);

// Bytes of split scratch (part_o + part_ml) a dense launch of `rows` rows and `heads` heads uses, 0 when it runs in
// enough waves not to split (under six waves of CTAs on this device's SMs: the partial last wave costs more than
// writing and merging the two halves).
size_t attention_split_bytes(int rows, int heads);

} // namespace h3
