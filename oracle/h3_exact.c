/* Exact CPU restatement of the sparse attention's coarse pass -- TEST INFRASTRUCTURE ONLY (tests/ use it to check
 * that the library selects identical cube indices; the library never links it).
 *
 * Follows the reference's description of Video Sparse Attention's training-free form (docs/architecture.md:118-133:
 * "pools each cube's queries and keys to their mean, scores every cube pair per head and keeps the top `ratio` share
 * of cubes per query cube"; "--sparse-local puts the query cube itself (and with 3 the cubes a frame group before and
 * after it) into the selection ahead of the scores") and docs/performance.md:158-198. The kernels themselves
 * (cube_pool, cube_scores, cube_topk in mako-common) are absent from the reference mount, so parity is unpinned;
 * the arithmetic order below is the one the library documents, which makes the comparison bit-exact:
 *   mean  = (sum over the cube's valid rows in cube order of float(x)) / count, sequential fp32 adds
 *   score = fmaf chain over the 128 dims in order
 *   pick  = forced cubes, then highest scores (ties to the lower index) until max(k, forced).
 * Build: gcc -O2 -ffp-contract=off -fopenmp -shared -fPIC -o oracle/libh3_exact.so oracle/h3_exact.c -lm (done by
 * __graft_entry__.build()). */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float bf16_to_f32(uint16_t b)
{
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* q, k: bf16 bits, element (row, head, dim) at row * row_stride + head * 128 + dim. mq, mk: [heads][cubes][128]. */
void h3x_cube_pool(const uint16_t* q, const uint16_t* k, int64_t row_stride, int heads, int dense_rows, int frames, int ph, int pw,
                   float* mq, float* mk)
{
    const int nct = (frames + 3) / 4, ncy = (ph + 3) / 4, ncx = (pw + 3) / 4, nc = nct * ncy * ncx;
    for (int h = 0; h < heads; ++h)
        for (int c = 0; c < nc; ++c) {
            const int cx = c % ncx, cy = (c / ncx) % ncy, ct = c / (ncx * ncy);
            for (int d = 0; d < 128; ++d) {
                float sq = 0.f, sk = 0.f;
                int n = 0;
                for (int kr = 0; kr < 64; ++kr) {
                    const int x = 4 * cx + (kr & 3), y = 4 * cy + ((kr >> 2) & 3), f = 4 * ct + (kr >> 4);
                    if (x >= pw || y >= ph || f >= frames)
                        continue;
                    const int64_t row = (int64_t)dense_rows + ((int64_t)f * ph + y) * pw + x;
                    sq = sq + bf16_to_f32(q[row * row_stride + h * 128 + d]);
                    sk = sk + bf16_to_f32(k[row * row_stride + h * 128 + d]);
                    ++n;
                }
                mq[((int64_t)h * nc + c) * 128 + d] = sq / (float)n;
                mk[((int64_t)h * nc + c) * 128 + d] = sk / (float)n;
            }
        }
}

void h3x_cube_scores(const float* mq, const float* mk, int heads, int cubes, float* scores)
{
    /* every score is its own fmaf chain, so splitting the heads over threads changes no result */
#pragma omp parallel for schedule(static)
    for (int h = 0; h < heads; ++h)
        for (int i = 0; i < cubes; ++i)
            for (int j = 0; j < cubes; ++j) {
                const float* a = mq + ((int64_t)h * cubes + i) * 128;
                const float* b = mk + ((int64_t)h * cubes + j) * 128;
                float acc = 0.f;
                for (int d = 0; d < 128; ++d)
                    acc = fmaf(a[d], b[d], acc);
                scores[((int64_t)h * cubes + i) * cubes + j] = acc;
            }
}

typedef struct {
    float s;
    int j;
} cand;

static int by_score_then_index(const void* a, const void* b)
{
    const cand* x = (const cand*)a;
    const cand* y = (const cand*)b;
    if (x->s > y->s)
        return -1;
    if (x->s < y->s)
        return 1;
    return x->j - y->j;
}

static int cmp_int(const void* a, const void* b) { return *(const int*)a - *(const int*)b; }

/* sel [heads][cubes][kcap] ascending, nsel [heads][cubes]. k: cubes to keep per query cube (forced ones count). */
void h3x_cube_topk(const float* scores, int heads, int frames, int ph, int pw, int k, int local, int32_t* sel, int32_t* nsel, int kcap)
{
    const int nct = (frames + 3) / 4, ncy = (ph + 3) / 4, ncx = (pw + 3) / 4, nc = nct * ncy * ncx, plane = ncx * ncy;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < heads; ++h) {
        cand* cs = (cand*)malloc(sizeof(cand) * (size_t)nc);
        int* out = (int*)malloc(sizeof(int) * (size_t)nc);
        for (int i = 0; i < nc; ++i) {
            const int ct = i / plane;
            int nout = 0, ncand = 0;
            for (int j = 0; j < nc; ++j) {
                int forced = 0;
                if (local > 0 && j == i)
                    forced = 1;
                if (local >= 3 && ((ct > 0 && j == i - plane) || (ct + 1 < nct && j == i + plane)))
                    forced = 1;
                if (forced)
                    out[nout++] = j;
                else {
                    cs[ncand].s = scores[((int64_t)h * nc + i) * nc + j];
                    cs[ncand].j = j;
                    ++ncand;
                }
            }
            int want = k > nout ? k : nout;
            qsort(cs, (size_t)ncand, sizeof(cand), by_score_then_index);
            for (int t = 0; nout < want && t < ncand; ++t)
                out[nout++] = cs[t].j;
            qsort(out, (size_t)nout, sizeof(int), cmp_int);
            const int n = nout < kcap ? nout : kcap;
            for (int t = 0; t < n; ++t)
                sel[((int64_t)h * nc + i) * kcap + t] = out[t];
            nsel[(int64_t)h * nc + i] = n;
        }
        free(cs);
        free(out);
    }
}

/* The synthetic weights of oracle/h3_oracle.py:synthetic, as a loop (the numpy form is the definition; a CPU test
 * pins the two together): value i = mean + k * s(i), s(i) = the sum of the four 16-bit fields of
 * splitmix64(key + i) minus 131070, one fp32 multiply and one fp32 add (-ffp-contract=off keeps them apart), then
 * optional bf16 rounding to nearest even. k = stdev / sqrt((65536^2 - 1) / 3), computed by the caller. */
static uint64_t splitmix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

void h3x_synthetic(float* out, int64_t n, uint64_t key, float mean, float k, int bf16)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t h = splitmix64(key + (uint64_t)i);
        const int64_t s = (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) + (int64_t)((h >> 32) & 0xFFFF) + (int64_t)(h >> 48) - 131070;
        float v = mean + k * (float)s;
        if (bf16) {
            uint32_t u;
            memcpy(&u, &v, 4);
            u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
            memcpy(&v, &u, 4);
        }
        out[i] = v;
    }
}
