// The sparse attention's coarse pass (cube_pool, cube_scores, cube_topk) and its pass lists.
#include "common.hpp"
#include "ptx.cuh"
#include "sparse.cuh"

#include <algorithm>
#include <cmath>

namespace h3 {

int sparse_k(float ratio, int cubes)
{
    const int k = int(std::ceil(double(ratio) * cubes - 1e-6));
    return std::max(1, std::min(cubes, k));
}

int sparse_forced(int local) { return local <= 0 ? 0 : (local >= 3 ? 3 : 1); }

void sparse_sizes(const CubeGrid& g, float ratio, int local, int& kcap, int& q_tiles, int& max_blocks)
{
    kcap = std::max(sparse_k(ratio, g.cubes()), sparse_forced(local));
    kcap = std::min(kcap, g.cubes());
    q_tiles = (g.cubes() + 1) / 2 + (g.dense_units() + 1) / 2;
    max_blocks = 2 * ((kcap + g.dense_units() + 1) / 2); // two entries (one per cube of the tile) a step
}

namespace {

// One CTA per (cube, head), one thread per dim: the cube's rows are consecutive in the packed order.
__global__ void cube_pool_kernel(const __nv_bfloat16* q, const __nv_bfloat16* k, int64_t rs, CubeGrid g, float* mq, float* mk)
{
    const int c = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    int first, n;
    g.unit_span(c, first, n);
    float sq = 0.f, sk = 0.f;
    for (int r = 0; r < n; ++r) {
        const size_t row = size_t(first + r);
        sq = __fadd_rn(sq, __bfloat162float(q[row * rs + h * 128 + d]));
        sk = __fadd_rn(sk, __bfloat162float(k[row * rs + h * 128 + d]));
    }
    const size_t o = (size_t(h) * g.cubes() + c) * 128 + d;
    mq[o] = __fdiv_rn(sq, float(n));
    mk[o] = __fdiv_rn(sk, float(n));
}

// 64 x 64 scores per CTA, 4 x 4 per thread. The means are staged transposed ([d][cube]) so that a thread reads its
// four query means and four key means for one d as two 16-byte loads; each score is still one fmaf chain over
// d = 0..127 in order, as the selection's arithmetic fixes.
constexpr int CS_T = 64, CS_P = CS_T + 4;

__global__ void __launch_bounds__(256) cube_scores_kernel(const float* mq, const float* mk, int cubes, float* scores)
{
    extern __shared__ float cs_smem[];
    float* A = cs_smem;             // [128][CS_P]: query-cube means, transposed
    float* B = cs_smem + 128 * CS_P; // [128][CS_P]: key-cube means, transposed
    const int h = blockIdx.z, i0 = blockIdx.y * CS_T, j0 = blockIdx.x * CS_T;
    const float* qa = mq + size_t(h) * cubes * 128;
    const float* kb = mk + size_t(h) * cubes * 128;
    for (int e = threadIdx.x; e < CS_T * 128; e += 256) {
        const int r = e / 128, d = e % 128;
        A[d * CS_P + r] = i0 + r < cubes ? qa[size_t(i0 + r) * 128 + d] : 0.f;
        B[d * CS_P + r] = j0 + r < cubes ? kb[size_t(j0 + r) * 128 + d] : 0.f;
    }
    __syncthreads();
    const int ti = threadIdx.x / 16, tj = threadIdx.x % 16;
    float acc[4][4] = {};
#pragma unroll 4
    for (int d = 0; d < 128; ++d) {
        const float4 a = *reinterpret_cast<const float4*>(A + d * CS_P + ti * 4);
        const float4 b = *reinterpret_cast<const float4*>(B + d * CS_P + tj * 4);
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y)
                acc[x][y] = __fmaf_rn(av[x], bv[y], acc[x][y]);
    }
#pragma unroll
    for (int x = 0; x < 4; ++x) {
        const int i = i0 + ti * 4 + x;
        if (i >= cubes)
            continue;
#pragma unroll
        for (int y = 0; y < 4; ++y) {
            const int j = j0 + tj * 4 + y;
            if (j < cubes)
                scores[(size_t(h) * cubes + i) * cubes + j] = acc[x][y];
        }
    }
}

__device__ __forceinline__ uint32_t orderable(float f)
{
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Top-k cube selection, one warp per (query cube, head) row: the row's keys (scores made order-preserving as unsigned
// integers) in shared memory, then a radix select of 8 bits a pass over the keys that are not forced, the histogram
// built by lanes that agree on a digit adding once. The threshold key T is the remaining-th largest; selected are the
// forced cubes (the query cube itself, with local >= 3 also the same position one frame group before and after), every
// key above T, and the keys equal to T among the first `remaining` such by index; written in ascending index order,
// at most kcap of them. No CTA barrier: the warps of a CTA work on different rows.
constexpr int TK_ROWS = 8; // warps (rows) a CTA

__global__ void __launch_bounds__(TK_ROWS * 32) cube_topk_kernel(const float* scores, CubeGrid g, int k, int local, int32_t* sel,
                                                               int32_t* nsel, int kcap, int rows_per_cta)
{
    extern __shared__ uint32_t tk_smem[]; // per warp: keys [n], then the histogram [256]
    const int n = g.cubes();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int i = blockIdx.x * rows_per_cta + w, h = blockIdx.y;
    if (w >= rows_per_cta || i >= n)
        return;
    uint32_t* keys = tk_smem + size_t(w) * (n + 256);
    int* hist = reinterpret_cast<int*>(keys + n);
    const int per_plane = g.ncx * g.ncy;
    const int ct = i / per_plane; // the query cube's frame group
    auto forced = [&](int j) {
        if (local <= 0)
            return false;
        if (j == i)
            return true;
        return local >= 3 && ((ct > 0 && j == i - per_plane) || (ct + 1 < g.nct && j == i + per_plane));
    };
    const int n_forced = local <= 0 ? 0 : 1 + (local >= 3 ? int(ct > 0) + int(ct + 1 < g.nct) : 0);
    const float* row = scores + (size_t(h) * n + i) * n;
    for (int j = lane; j < n; j += 32)
        keys[j] = orderable(row[j]);
    __syncwarp();
    const int want = max(k, n_forced);
    const bool pick = want - n_forced > 0;
    int remaining = want - n_forced; // to pick among the non-forced cubes
    uint32_t prefix = 0, mask = 0;
    if (pick) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = lane; b < 256; b += 32)
                hist[b] = 0;
            __syncwarp();
            for (int j0 = 0; j0 < n; j0 += 32) {
                const int j = j0 + lane;
                const bool in = j < n && !forced(j) && (keys[j] & mask) == prefix;
                const int dg = in ? int((keys[j] >> shift) & 255) : -1;
                const unsigned same = __match_any_sync(0xffffffffu, dg);
                if (in && (__ffs(same) - 1) == lane)
                    atomicAdd(&hist[dg], __popc(same));
            }
            __syncwarp();
            // Lane l holds bins 255 - 8 l - t (t < 8), so the bins run from the highest digit down across the lanes;
            // the digit is the one whose bins from 255 down to it first hold at least `remaining` keys.
            int c[8], sum = 0;
#pragma unroll
            for (int t = 0; t < 8; ++t)
                c[t] = hist[255 - 8 * lane - t], sum += c[t];
            int incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o)
                    incl += v;
            }
            int above = incl - sum, digit = -1, acc = 0;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                if (digit < 0 && above < remaining && above + c[t] >= remaining)
                    digit = 255 - 8 * lane - t, acc = above;
                above += c[t];
            }
            const unsigned found = __ballot_sync(0xffffffffu, digit >= 0);
            if (!found) // fewer candidates than wanted (k above the cubes): keep what the passes so far select
                break;
            const int src = __ffs(found) - 1; // exactly one lane holds the digit (the counts are non-negative)
            digit = __shfl_sync(0xffffffffu, digit, src);
            acc = __shfl_sync(0xffffffffu, acc, src);
            remaining -= acc;
            prefix |= uint32_t(digit) << shift;
            mask |= 255u << shift;
            __syncwarp();
        }
    }
    int32_t* dst = sel + (size_t(h) * n + i) * kcap;
    const unsigned lt = (1u << lane) - 1u;
    int out = 0, ties_before = 0;
    for (int j0 = 0; j0 < n; j0 += 32) {
        const int j = j0 + lane;
        const bool valid = j < n;
        const bool f = valid && forced(j);
        const uint32_t key = valid ? keys[j] : 0u;
        const bool tie = valid && !f && pick && key == prefix;
        const unsigned tb = __ballot_sync(0xffffffffu, tie);
        const bool s = f || (valid && !f && pick && key > prefix) || (tie && ties_before + __popc(tb & lt) < remaining);
        ties_before += __popc(tb);
        const unsigned sb = __ballot_sync(0xffffffffu, s);
        const int pos = out + __popc(sb & lt);
        if (s && pos < kcap)
            dst[pos] = j;
        out += __popc(sb);
    }
    if (lane == 0)
        nsel[size_t(h) * n + i] = min(want, kcap);
}

// One thread per (head, video query tile): merge the two cubes' selections, append the dense units, pair them.
// (first row, rows) of unit u, or (-1, 0) for none.
__device__ __forceinline__ int2 span_of(int u, const CubeGrid& g)
{
    if (u < 0)
        return make_int2(-1, 0);
    int first, n;
    g.unit_span(u, first, n);
    return make_int2(first, n);
}

__global__ void build_passes_kernel(const int32_t* sel, const int32_t* nsel, int kcap, int heads, CubeGrid g, int4* blocks,
                                    int32_t* nblocks, int4* q_rows, int q_tiles, int max_blocks)
{
    const int nc = g.cubes(), nd = g.dense_units();
    const int vt = (nc + 1) / 2;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < q_tiles) {
        int2 a, b;
        if (idx < vt) {
            a = span_of(2 * idx, g), b = span_of(2 * idx + 1 < nc ? 2 * idx + 1 : -1, g);
        } else {
            const int t = idx - vt;
            a = span_of(nc + 2 * t, g), b = span_of(2 * t + 1 < nd ? nc + 2 * t + 1 : -1, g);
        }
        q_rows[idx] = make_int4(a.x, b.x, a.y, b.y);
    }
    if (idx >= heads * q_tiles)
        return;
    const int h = idx / q_tiles, t = idx % q_tiles;
    if (t >= vt) {
        nblocks[idx] = -1; // dense query rows attend every row
        return;
    }
    // Each cube of the tile gets its own list: its selected cubes (ascending) then every dense unit, two units a
    // step; the shorter list is padded with empty entries.
    const int max_steps = max_blocks / 2;
    int4* out = blocks + size_t(idx) * max_blocks;
    int steps = 0;
    for (int x = 0; x < 2; ++x) {
        const int c = 2 * t + x;
        const int32_t* L = c < nc ? sel + (size_t(h) * nc + c) * kcap : nullptr;
        const int n = c < nc ? nsel[size_t(h) * nc + c] : -nd; // a missing cube gets no units at all
        const int len = n + nd;
        const int st = (len + 1) / 2;
        steps = max(steps, st);
        for (int s2 = 0; s2 < min(st, max_steps); ++s2) {
            int2 sp[2];
            for (int k = 0; k < 2; ++k) {
                const int i = 2 * s2 + k;
                sp[k] = i < len ? span_of(i < n ? L[i] : nc + (i - n), g) : make_int2(-1, 0);
            }
            out[2 * s2 + x] = make_int4(sp[0].x, sp[1].x, sp[0].y | (sp[1].y << 8), 0);
        }
    }
    steps = min(steps, max_steps);
    for (int x = 0; x < 2; ++x) {
        const int c = 2 * t + x;
        const int len = (c < nc ? nsel[size_t(h) * nc + c] : -nd) + nd;
        for (int s2 = (len + 1) / 2; s2 < steps; ++s2)
            out[2 * s2 + x] = make_int4(-1, -1, 0, 0);
    }
    nblocks[idx] = steps;
}

} // namespace

void cube_pool(const void* q, const void* k, int64_t rs, int heads, const CubeGrid& g, float* mq, float* mk, cudaStream_t s)
{
    cube_pool_kernel<<<dim3(g.cubes(), heads), 128, 0, s>>>(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                                                            rs, g, mq, mk);
    H3_CUDA(cudaGetLastError());
}

void cube_scores(const float* mq, const float* mk, int heads, int cubes, float* scores, cudaStream_t s)
{
    const dim3 grid((cubes + CS_T - 1) / CS_T, (cubes + CS_T - 1) / CS_T, heads);
    const size_t smem = size_t(2) * 128 * CS_P * sizeof(float);
    static std::atomic<uint64_t> opt_in;
    smem_opt_in(cube_scores_kernel, int(smem), opt_in);
    cube_scores_kernel<<<grid, 256, smem, s>>>(mq, mk, cubes, scores);
    H3_CUDA(cudaGetLastError());
}

void cube_topk(const float* scores, int heads, const CubeGrid& g, int k, int local, int32_t* sel, int32_t* nsel, int kcap, cudaStream_t s)
{
    const int n = g.cubes();
    const size_t per_row = (size_t(n) + 256) * 4; // a warp's keys and histogram
    if (per_row > 160 * 1024)
        throw CudaError("cube_topk: too many cubes");
    const int rows = int(std::min<size_t>(TK_ROWS, (160 * 1024) / per_row));
    static std::atomic<uint64_t> opt_in;
    smem_opt_in(cube_topk_kernel, 160 * 1024, opt_in);
    cube_topk_kernel<<<dim3((n + rows - 1) / rows, heads), TK_ROWS * 32, rows * per_row, s>>>(scores, g, k, local, sel, nsel, kcap, rows);
    H3_CUDA(cudaGetLastError());
}

void build_passes(const int32_t* sel, const int32_t* nsel, int kcap, int heads, const CubeGrid& g, int4* blocks, int32_t* nblocks,
                  int4* q_rows, int q_tiles, int max_blocks, cudaStream_t s)
{
    const int n = std::max(heads * q_tiles, q_tiles);
    build_passes_kernel<<<(n + 127) / 128, 128, 0, s>>>(sel, nsel, kcap, heads, g, blocks, nblocks, q_rows, q_tiles, max_blocks);
    H3_CUDA(cudaGetLastError());
}

void sparse_attention(const AttnParams& a, const CubeGrid& g, float ratio, int local, const SparseBuffers& b, cudaStream_t s)
{
    cube_pool(a.q, a.k, a.row_stride, a.heads, g, b.mq, b.mk, s);
    cube_scores(b.mq, b.mk, a.heads, g.cubes(), b.scores, s);
    cube_topk(b.scores, a.heads, g, sparse_k(ratio, g.cubes()), local, b.sel, b.nsel, b.kcap, s);
    build_passes(b.sel, b.nsel, b.kcap, a.heads, g, b.blocks, b.nblocks, b.q_rows, b.q_tiles, b.max_blocks, s);
    AttnParams p = a;
    p.rows = g.rows();
    p.blocks = b.blocks;
    p.nblocks = b.nblocks;
    p.q_rows = b.q_rows;
    p.q_tiles = b.q_tiles;
    p.max_blocks = b.max_blocks;
    p.grid = g;
    attention(p, s);
}

} // namespace h3
