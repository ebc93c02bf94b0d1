// Flash attention on sm_100a: tcgen05.mma with the scores S and the output O accumulated in TMEM, P (bf16) written
// back into TMEM and read from there by the PV MMA, K/V tiles streamed by TMA, online softmax in the exp2 domain
// with O rescaled only when a row's running maximum grows by more than 2^8 (the exponentials use the stale maximum
// meanwhile, exact after the final division).
//   attn2_kernel  dense: two 128-row query tiles per CTA share each K/V tile; the tensor core alternates between the
//                 tiles so one tile's MMAs overlap the other tile's softmax.
//   attn3_kernel  sparse: one query tile of two units (cubes) per CTA, each unit with its own key list, as two
//                 M = 64 MMAs into the two lane halves of TMEM; two S buffers, so S(j+1) is computed while the softmax
//                 works on S(j).
// Every tile is four 64x64 TMA boxes (two 64-row units x two 64-dim halves) of consecutive rows: in the packed row
// order each 4x4x4 latent cube is one run of rows, so a sparse unit is the same plain box as a dense one (the rows
// past a cut-short cube's count belong to the next unit and are masked).
#include "attention.cuh"
#include "common.hpp"
#include "ptx.cuh"

#include <cmath>

namespace h3 {

namespace {

constexpr int HALF = 16384; // 128 rows x 64 dims bf16
constexpr int TILE = 32768; // 128 rows x 128 dims
constexpr float kRescaleThreshold = 8.0f; // log2 units

struct Maps {
    CUtensorMap q, k, v; // (dim, head, row), box 64 x 1 x 64
};

// Issue the TMA loads of the 64 rows from `row` into rows [64 * half, 64 * half + 64) of a 128-row tile (every 64-dim
// half of a head of HD dims). Rows past the tensor read as zeros.
template <int HD = 128>
__device__ __forceinline__ void load_rows(uint8_t* tile, int half, int row, int head, const CUtensorMap* map, uint64_t* bar)
{
#pragma unroll
    for (int hh = 0; hh < HD / 64; ++hh)
        tma_load_3d(tile + hh * HALF + half * 8192, map, bar, hh * 64, head, row);
}

// Where query row `row`'s output (head `head`, dims from `d0`) goes: this rank's buffer, or straight to the row's
// owner when the sequence-parallel exchange is fused into the epilogue (the stores are performed when the kernel
// completes; the barrier that follows it on the stream orders them before any reader). Null for padding rows.
template <int HD = 128>
__device__ __forceinline__ __nv_bfloat16* out_ptr(const AttnParams& p, int row, int head, int d0)
{
    if (row < 0)
        return nullptr;
    if (!p.peer_out[0])
        return reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(row) * p.out_row_stride + head * HD + d0;
    const int owner = row / p.rows_per_rank, local = row - owner * p.rows_per_rank;
    return reinterpret_cast<__nv_bfloat16*>(p.peer_out[owner]) +
           (size_t(p.my_rank) * p.rows_per_rank + local) * (size_t(p.heads) * HD) + head * HD + d0;
}

// Key block j of a query unit that sees every row: rows [128 j, 128 j + 128) as two 64-row key units, in the pass
// list entry format (first row of key unit 0, of key unit 1 or -1, rows of unit 0 | rows of unit 1 << 8, 0).
__device__ __forceinline__ int4 every_row_block(int j, int rows)
{
    const int na = min(max(rows - 128 * j, 0), 64), nb = min(max(rows - 128 * j - 64, 0), 64);
    return make_int4(128 * j, nb > 0 ? 128 * j + 64 : -1, na | (nb << 8), 0);
}

// ------------------------------------------------------------------------------------------------------------
// Dense attention, two query tiles per CTA (256 query rows of one head) sharing every K/V tile. Heads of HD = 128 or
// 64 dims. The rows may form several independent segments (seg_rows rows every seg_stride rows, e.g. the tiles of
// a decoder batch): each CTA then takes query rows and keys of one segment only.
//   warp 0      TMA: Q0 and Q1 once, then K_j and V_j (2-stage ring each)
//   warp 1      MMA, in the order S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) | ...: while one tile's softmax runs
//               the tensor core works on the other tile
//   warps 2..5  softmax of tile 0, warps 6..9 softmax of tile 1 (thread = query row)
// TMEM (512 columns): S0 | S1 | O0 | O1 (128 columns each for S, HD for O). P_t (bf16, two per column) is written back
// over the first 64
// columns of S_t and the PV MMA reads it from TMEM (A operand in TMEM), so P never touches shared memory. The
// tensor core executes one thread's MMAs in issue order, so S_t(j+1) overwrites P_t(j) only after PV_t(j) read it;
// and s_full_t(j) tracks every earlier MMA, so once S_t(j) is complete, PV_t(j-1) is too and the softmax may write
// P_t(j) and rescale O_t.
// Warps sharing a query row in the softmax: with the online maximum one (two measured no faster: they must agree on the
// row maximum every step); with a known score bound two, each over its 64-key half, exchanging only the row sums at
// the end.
constexpr int A2_SPLIT = 1, A2_SPLIT_BOUNDED = 2;
constexpr int A2_KST = 3, A2_VST = 2; // K is freed once both S MMAs read it, V after both PV MMAs
template <int HD, int SPLIT, bool STATIC>
struct A2Smem {
    static constexpr int TL = 128 * HD * 2; // a 128-row tile of one head
    static constexpr int OFF_Q = 0;         // Q0, Q1
    static constexpr int OFF_K = 2 * TL;
    static constexpr int OFF_V = OFF_K + A2_KST * TL;
    static constexpr int OFF_BAR = OFF_V + A2_VST * TL;
    // row maxima and sums exchanged between a row's warps (with a score bound only the sums, through the tile's Q
    // buffer once its last score MMA is done)
    static constexpr int OFF_RED = OFF_BAR + 256;
    static constexpr int TOTAL = OFF_RED + (SPLIT > 1 && !STATIC ? 2 * 3 * SPLIT * 128 * 4 : 0) + 1024;
};

template <int SPLIT, int HD, bool STATIC>
__global__ void __launch_bounds__(64 + 256 * SPLIT, 1) attn2_kernel(const __grid_constant__ Maps maps, const AttnParams p)
{
    using SM = A2Smem<HD, SPLIT, STATIC>;
    constexpr int TL = SM::TL, A2_OFF_Q = SM::OFF_Q, A2_OFF_K = SM::OFF_K, A2_OFF_V = SM::OFF_V, A2_OFF_BAR = SM::OFF_BAR,
                  A2_OFF_RED = SM::OFF_RED;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + A2_OFF_BAR);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;          // [A2_KST]
    uint64_t* k_empty = k_full + A2_KST;  // [A2_KST]
    uint64_t* v_full = k_empty + A2_KST;  // [A2_VST]
    uint64_t* v_empty = v_full + A2_VST;  // [A2_VST]
    uint64_t* s_full = v_empty + A2_VST;  // [2] per tile
    uint64_t* p_full = s_full + 2;        // [2] per tile
    uint64_t* pv_done = p_full + 2;       // [2] per tile
    uint64_t* drain = pv_done + 2;
    uint64_t* xchg = drain + 1;           // [2] per tile: the row-maximum / row-sum exchange between a row's warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xchg + 2);

    const int warp = warp_id();
    const int head = blockIdx.y;
    // the segment of this CTA's query rows and keys: rows [seg0, seg0 + seg_rows)
    const int seg_rows = p.seg_rows > 0 ? p.seg_rows : p.rows;
    const int pairs_per_seg = (seg_rows + 255) / 256;
    const int seg = blockIdx.x / pairs_per_seg, pair = blockIdx.x - seg * pairs_per_seg;
    const int seg0 = int(seg * (p.seg_rows > 0 ? p.seg_stride : 0));
    // keys: 128-row blocks [kv0, kv0 + nkv) of the segment, all of them or this CTA's part of a split launch (gridDim.z)
    const int nkv_all = (seg_rows + 127) / 128, per = (nkv_all + gridDim.z - 1) / gridDim.z;
    const int kv0 = blockIdx.z * per;
    const int nkv = min(nkv_all, kv0 + per) - kv0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < A2_KST; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < A2_VST; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4 * SPLIT);
            mbar_init(&pv_done[i], 1);
            mbar_init(&xchg[i], 4 * SPLIT);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && elect_one_lane()) {
        // ------------------------------------------------------------------------------------------ TMA
        mbar_arrive_expect_tx(q_full, 2 * TL);
        for (int u = 0; u < 4; ++u)
            load_rows<HD>(smem + A2_OFF_Q + (u >> 1) * TL, u & 1, seg0 + (4 * pair + u) * 64, head, &maps.q, q_full);
        // K runs ahead of V by up to the depth of its ring
        int jk = 0, jv = 0;
        while (jv < nkv) {
            if (jk < nkv && jk < jv + A2_KST) {
                const int s = jk % A2_KST;
                if (!mbar_wait(&k_empty[s], ((jk / A2_KST) & 1) ^ 1))
                    break;
                mbar_arrive_expect_tx(&k_full[s], TL);
                load_rows<HD>(smem + A2_OFF_K + s * TL, 0, seg0 + 128 * (kv0 + jk), head, &maps.k, &k_full[s]);
                load_rows<HD>(smem + A2_OFF_K + s * TL, 1, seg0 + 128 * (kv0 + jk) + 64, head, &maps.k, &k_full[s]);
                ++jk;
            } else {
                const int s = jv % A2_VST;
                if (!mbar_wait(&v_empty[s], ((jv / A2_VST) & 1) ^ 1))
                    break;
                mbar_arrive_expect_tx(&v_full[s], TL);
                load_rows<HD>(smem + A2_OFF_V + s * TL, 0, seg0 + 128 * (kv0 + jv), head, &maps.v, &v_full[s]);
                load_rows<HD>(smem + A2_OFF_V + s * TL, 1, seg0 + 128 * (kv0 + jv) + 64, head, &maps.v, &v_full[s]);
                ++jv;
            }
        }
    } else if (warp == 1 && elect_one_lane()) {
        // ------------------------------------------------------------------------------------------ MMA
        const uint32_t id_s = idesc_bf16(128, 128);
        const uint32_t id_pv = idesc_bf16(128, HD, false, true);
        // TMEM column of P's K = 16 slice kk: with a score bound each 64-key slice's P (32 columns) lies over the first
        // half of that slice's own scores, else P fills the first 64 columns
        auto p_col2 = [](int kk) { return uint32_t(kk * 8 + (STATIC && SPLIT > 1 && kk >= 4 ? 32 : 0)); };
        auto issue_s = [&](int t, int j) {
            const int ks = j % A2_KST;
            const uint32_t sq = smem_u32(smem + A2_OFF_Q + t * TL);
            const uint32_t sk = smem_u32(smem + A2_OFF_K + ks * TL);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
                const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
                mma_bf16_ss(tmem + t * 128, sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), id_s, kk > 0);
            }
            mma_commit(&s_full[t]);
            if (t == 1)
                mma_commit(&k_empty[ks]); // both tiles' S MMAs have read K_j
        };
        auto issue_pv = [&](int t, int j) {
            const int vs = j % A2_VST;
            const uint32_t sv = smem_u32(smem + A2_OFF_V + vs * TL);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                mma_bf16_ts(tmem + 256 + t * HD, tmem + t * 128 + p_col2(kk), sdesc_sw128(sv + kk * 2048, HALF, 1024), id_pv,
                            (j | kk) != 0);
            mma_commit(&pv_done[t]);
            if (t == 1)
                mma_commit(&v_empty[vs]); // both tiles' PV MMAs have read V_j
        };
        bool ok = mbar_wait(q_full, 0) && mbar_wait(&k_full[0], 0);
        if (ok) {
            tc_fence_after();
            issue_s(0, 0);
            issue_s(1, 0);
        }
        for (int j = 0; j < nkv && ok; ++j) {
            if (!(ok = mbar_wait(&v_full[j % A2_VST], (j / A2_VST) & 1) && mbar_wait(&p_full[0], j & 1)))
                break;
            tc_fence_after();
            issue_pv(0, j);
            const bool more = j + 1 < nkv;
            if (more) {
                if (!(ok = mbar_wait(&k_full[(j + 1) % A2_KST], ((j + 1) / A2_KST) & 1)))
                    break;
                tc_fence_after();
                issue_s(0, j + 1);
            }
            if (!(ok = mbar_wait(&p_full[1], j & 1)))
                break;
            tc_fence_after();
            issue_pv(1, j);
            if (more)
                issue_s(1, j + 1);
        }
        mma_commit(drain);
        mbar_wait(drain, 0);
    } else if (warp >= 2) {
        // -------------------------------------------------------------------------------------- softmax
        // SPLIT warps share each row: the warps of (tile t, slice hc) handle keys [hc NC, hc NC + NC) of their rows
        // and agree on the row maximum through shared memory.
        constexpr int NC = 128 / SPLIT; // keys of a step this slice handles
        constexpr int OC = HD / SPLIT;  // output columns this slice rescales and stores
        const int t = (warp - 2) / (4 * SPLIT);
        const int hc = ((warp - 2) % (4 * SPLIT)) / 4;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane_id();
        const uint32_t lane_base = uint32_t(quarter * 32) << 16;
        const uint32_t tS = tmem + lane_base + t * 128;
        const uint32_t tO = tmem + lane_base + 256 + t * HD + hc * OC;
        float* red = reinterpret_cast<float*>(smem + A2_OFF_RED) + t * (3 * SPLIT * 128); // [3 slots][SPLIT][128 rows]
        const float sl2 = p.scale * 1.4426950408889634f;
        // STATIC: every score is at most p.static_max (log2 units), which then serves as the row maximum throughout
        float m = STATIC ? p.static_max : -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            if (!(ok = mbar_wait(&s_full[t], j & 1)))
                break;
            tc_fence_after();
            float s[NC];
            {
                uint32_t r[NC / 32][32];
#pragma unroll
                for (int c = 0; c < NC / 32; ++c)
                    tmem_ld32(tS + hc * NC + c * 32, r[c]);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < NC / 32; ++c)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        s[c * 32 + i] = __uint_as_float(r[c][i]);
            }
            const int left = seg_rows - (kv0 + j) * 128 - hc * NC;
            if (left < NC) {
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    if (c >= left)
                        s[c] = -INFINITY;
            }
            // Row maximum over 8 independent chains of three-input maxima (a single chain would serialise the
            // latencies); the exponent arguments and the row sum as packed fp32 pairs.
            float mx = -INFINITY;
            if constexpr (!STATIC) {
                float mp[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    mp[i] = fmaxf(s[2 * i], s[2 * i + 1]);
#pragma unroll
                for (int c = 16; c < NC; c += 16)
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        mp[i] = max3f(mp[i], s[c + 2 * i], s[c + 2 * i + 1]);
                mx = max3f(max3f(mp[0], mp[1], mp[2]), max3f(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
            }
            if constexpr (SPLIT > 1 && !STATIC) {
                // Every slice has loaded its scores once this exchange completes, so P may then overwrite them.
                float* slot = red + (j & 1) * SPLIT * 128;
                slot[hc * 128 + row] = mx;
                __syncwarp();
                if (elect_one_lane())
                    mbar_arrive(&xchg[t]);
                if (!(ok = mbar_wait(&xchg[t], j & 1)))
                    break;
#pragma unroll
                for (int o = 0; o < SPLIT; ++o)
                    if (o != hc)
                        mx = fmaxf(mx, slot[o * 128 + row]);
            }
            const float m_cand = mx * sl2;
            const bool need = !STATIC && m_cand > m + kRescaleThreshold;
            const float m_use = need ? m_cand : m;
            const float alpha = need ? ex2_approx(m - m_use) : 1.f;
            const float msub = m_use == -INFINITY ? 0.f : m_use;
            const float2 scale2 = make_float2(sl2, sl2), neg2 = make_float2(-msub, -msub);
            float2 sp[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            uint32_t pk[NC / 2];
#pragma unroll
            for (int c = 0; c < NC / 2; ++c) {
                const float2 x = fma2(make_float2(s[2 * c], s[2 * c + 1]), scale2, neg2);
                // with the bound, one exponent pair in eight on the FMA pipes relieves the MUFU (one in four or more
                // measured slower: the softmax's own issue then lengthens)
                const float2 e = STATIC && (c & 7) == 7 ? ex2_fma2(x) : make_float2(ex2_approx(x.x), ex2_approx(x.y));
                sp[c & 3] = add2(sp[c & 3], e);
                pk[c] = pack_bf16x2(e.x, e.y);
            }
            const float2 s01 = add2(add2(sp[0], sp[1]), add2(sp[2], sp[3]));
            const float rs = s01.x + s01.y;
            if (!STATIC && j > 0 && __any_sync(0xffffffffu, need)) {
                // O_t holds PV_t(0..j-1), complete (S_t(j) was issued after PV_t(j-1)); each slice rescales its columns
#pragma unroll 1
                for (int c = 0; c < OC / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(tO + c * 32, o);
                }
            }
            l = l * alpha + rs; // this slice's share of the row sum
            m = m_use;
#pragma unroll
            for (int c = 0; c < NC / 64; ++c)
                tmem_st32(tS + (STATIC ? hc * NC : hc * (NC / 2)) + c * 32, *reinterpret_cast<uint32_t(*)[32]>(pk + c * 32));
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (elect_one_lane())
                mbar_arrive(&p_full[t]);
        }
        if constexpr (SPLIT > 1) {
            if (ok) {
                // S_t(nkv - 1) is done, so no MMA reads Q_t any more
                float* slot = STATIC ? reinterpret_cast<float*>(smem + A2_OFF_Q + t * TL) : red + 2 * SPLIT * 128;
                slot[hc * 128 + row] = l;
                __syncwarp();
                if (elect_one_lane())
                    mbar_arrive(&xchg[t]);
                ok = mbar_wait(&xchg[t], STATIC ? 0 : nkv & 1);
                l = 0.f;
#pragma unroll
                for (int o = 0; o < SPLIT; ++o)
                    l += slot[o * 128 + row];
            }
        }
        const bool done = ok && mbar_wait(&pv_done[t], (nkv - 1) & 1);
        if (done && gridDim.z > 1) {
            // a split launch: this part's unnormalised output, row maximum and sum, for the combine kernel
            tc_fence_after();
            const int out_row = pair * 256 + t * 128 + row;
            const size_t item = (size_t(blockIdx.z) * p.rows + out_row) * p.heads + head;
#pragma unroll 1
            for (int c = 0; c < OC / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(tO + c * 32, o);
                tmem_wait_ld();
                if (out_row < p.rows) {
                    float4* d4 = reinterpret_cast<float4*>(p.part_o + item * 128 + hc * OC + c * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        d4[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]), __uint_as_float(o[4 * i + 2]),
                                            __uint_as_float(o[4 * i + 3]));
                }
            }
            if (out_row < p.rows && hc == 0)
                *reinterpret_cast<float2*>(p.part_ml + item * 2) = make_float2(m, l);
        } else if (done) {
            tc_fence_after();
            const int in_seg = pair * 256 + t * 128 + row;
            const int out_row = seg0 + in_seg;
            const float inv = l > 0.f ? 1.f / l : 0.f;
            __nv_bfloat16* dst = in_seg < seg_rows && out_row < p.rows ? out_ptr<HD>(p, out_row, head, hc * OC) : nullptr;
#pragma unroll 1
            for (int c = 0; c < OC / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(tO + c * 32, o);
                tmem_wait_ld();
                if (dst) {
                    uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        d4[i] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                                           pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                                           pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                                           pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------------------------
// Sparse attention: one CTA per query tile of two units (two cubes, or two chunks of dense rows), each unit with its
// own key list, so no unit computes scores against keys only the other one selected. The tensor core runs M = 64
// MMAs: unit a's 64 query rows land in TMEM lanes 0-15 of every 32-lane subpartition, unit b's in lanes 16-31 (the
// lane offset of the MMA's TMEM address), so the two units' S and O share columns and every softmax warp holds 16 rows
// of each. Per step j: S_a(j) = Q_a K_a(j)^T and S_b(j) = Q_b K_b(j)^T (128 keys each), then P_x(j) V_x(j) into O_x.
//   warp 0      TMA: Q once; per step K_a, K_b into a 3-slot ring (freed as soon as their S MMAs are done) and V_a,
//               V_b into a 2-slot ring
//   warp 1      MMA: S(0), S(1) up front; then per step PV_a(j), PV_b(j) (A = P from TMEM) and S(j+2) into the S
//               buffer step j leaves, so S(j+1) is ready when the softmax finishes step j
//   warps 2..9  softmax: two warps per 32-lane quarter, each over one 64-key half of the step (hc = 0, 1), agreeing on
//               the row maximum through shared memory (unless a bound on the scores stands in for it); each half's P
//               (bf16) written back over the first 32 of its own 64 score columns
// TMEM: S buffer 0 | S buffer 1 | O (128 columns each). S(j+2) overwrites P(j) only after PV(j) read it (one thread
// issues both, and the tensor core runs them in order). The softmax of step j may rescale O only once PV(j-1) is
// done (it waits for that only when a rescale is needed).
// A tile of dense rows (text, conditioning, audio) sees every key, the same for both of its units: it runs as one
// M = 128 tile (unit a in lanes 0-63, unit b in 64-127, the tensor core's full rate) over 128-key blocks loaded
// once, the ring holding one item per step instead of one per unit.
constexpr int A3_KST = 3, A3_VST = 2;
constexpr int NT3 = 64 + 256;
constexpr int A3_OFF_Q = 0;
constexpr int A3_OFF_K = TILE;
constexpr int A3_OFF_V = A3_OFF_K + A3_KST * TILE;
constexpr int A3_OFF_BAR = A3_OFF_V + A3_VST * TILE;
constexpr int A3_OFF_RED = A3_OFF_BAR + 256;
constexpr int A3_SMEM = A3_OFF_RED + 3 * 2 * 128 * 4 + 1024;
constexpr uint32_t LANE16 = 16u << 16; // TMEM address of lane 16: unit b's half of each subpartition

// TMEM column (from an S buffer's first) of P's K = 16 slice kk: each 64-key half's P (bf16 pairs, 32 columns) is
// written over the first half of that half's own scores, so neither slice overwrites scores the other has yet to load.
__device__ __forceinline__ uint32_t p_col(int kk) { return uint32_t(kk * 8 + (kk >= 4 ? 32 : 0)); }

template <bool STATIC>
__global__ void __launch_bounds__(NT3, 1) attn3_kernel(const __grid_constant__ Maps maps, const AttnParams p)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + A3_OFF_BAR);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;                   // [A3_KST]
    uint64_t* k_empty = k_full + A3_KST;           // [A3_KST]
    uint64_t* v_full = k_empty + A3_KST;           // [A3_VST]
    uint64_t* v_empty = v_full + A3_VST;           // [A3_VST]
    uint64_t* s_full = v_empty + A3_VST;           // [2] per S buffer
    // p_full per S buffer too: the softmax may finish steps j and j + 1 before the MMA warp waits for P(j), and a
    // single barrier would then be two phases ahead of that wait; step j + 2 needs S(j + 2), issued after PV(j).
    uint64_t* p_full = s_full + 2;                 // [2] per S buffer
    uint64_t* pv_done = p_full + 2;
    uint64_t* xchg = pv_done + 1;
    uint64_t* drain = xchg + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = warp_id();
    // Launches are 1-D and longest first: the dense-row query tiles (which see every key, several times a video
    // tile's work) of every head, then each head's video tiles together (they share the head's keys in L2).
    int tile, head;
    {
        const int vt = (p.grid.cubes() + 1) / 2, dt = p.q_tiles - vt;
        const int id = blockIdx.x;
        if (id < p.heads * dt)
            head = id % p.heads, tile = vt + id / p.heads;
        else
            head = (id - p.heads * dt) / vt, tile = (id - p.heads * dt) % vt;
    }
    int nkv = p.nblocks[head * p.q_tiles + tile];
    const bool every = nkv < 0; // a dense-row tile: one M = 128 tile over every key
    if (every)
        nkv = (p.rows + 127) / 128;
    const int4 qr = p.q_rows[tile]; // (first row of unit a, of unit b or -1, rows of a, rows of b)
    const int4* entries = p.blocks + (size_t(head) * p.q_tiles + tile) * p.max_blocks;
    // step j's keys for query unit x
    auto entry = [&](int j, int x) -> int4 { return every ? every_row_block(j, p.rows) : entries[2 * j + x]; };

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < A3_KST; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < A3_VST; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(&p_full[0], 8);
        mbar_init(&p_full[1], 8);
        mbar_init(pv_done, 1);
        mbar_init(xchg, 8);
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t T_O = 256;

    if (nkv > 0 && warp == 0 && elect_one_lane()) {
        // ------------------------------------------------------------------------------------------ TMA
        // Q: unit a's rows into rows 0-63 of the tile, unit b's into rows 64-127 (unit a's again if there is no b)
        mbar_arrive_expect_tx(q_full, TILE);
        load_rows(smem + A3_OFF_Q, 0, qr.x, head, &maps.q, q_full);
        load_rows(smem + A3_OFF_Q, 1, qr.y < 0 ? qr.x : qr.y, head, &maps.q, q_full);
        // Ring items i = 2 j + x (step j, query unit x), or i = j for a dense-row tile: K runs ahead of V by up to the
        // depth of its ring. A padding entry (no key unit) loads row 0: the keys are masked.
        const int items = every ? nkv : 2 * nkv;
        int ik = 0, iv = 0;
        bool ok = true;
        while (ok && iv < items) {
            const bool k_turn = ik < items && ik < iv + A3_KST;
            const int i = k_turn ? ik : iv;
            const int4 e = every ? every_row_block(i, p.rows) : entry(i >> 1, i & 1);
            const int r0 = e.x < 0 ? 0 : e.x, r1 = e.y < 0 ? r0 : e.y;
            if (k_turn) {
                const int s = ik % A3_KST;
                if (!(ok = mbar_wait(&k_empty[s], ((ik / A3_KST) & 1) ^ 1)))
                    break;
                mbar_arrive_expect_tx(&k_full[s], TILE);
                load_rows(smem + A3_OFF_K + s * TILE, 0, r0, head, &maps.k, &k_full[s]);
                load_rows(smem + A3_OFF_K + s * TILE, 1, r1, head, &maps.k, &k_full[s]);
                ++ik;
            } else {
                const int s = iv % A3_VST;
                if (!(ok = mbar_wait(&v_empty[s], ((iv / A3_VST) & 1) ^ 1)))
                    break;
                mbar_arrive_expect_tx(&v_full[s], TILE);
                load_rows(smem + A3_OFF_V + s * TILE, 0, r0, head, &maps.v, &v_full[s]);
                load_rows(smem + A3_OFF_V + s * TILE, 1, r1, head, &maps.v, &v_full[s]);
                ++iv;
            }
        }
    } else if (nkv > 0 && warp == 1 && elect_one_lane()) {
        // ------------------------------------------------------------------------------------------ MMA
        const uint32_t id_s = idesc_bf16(64, 128), id_s128 = idesc_bf16(128, 128);
        const uint32_t id_pv = idesc_bf16(64, 128, false, true), id_pv128 = idesc_bf16(128, 128, false, true);
        const uint32_t sq = smem_u32(smem + A3_OFF_Q);
        // S(j) for both query units (unit x: query rows at 8192 x within each dim half, lanes at 16 x), or for the
        // whole 128-row tile of a dense-row tile
        auto issue_s = [&](int j) -> bool {
            if (every) {
                const int s = j % A3_KST;
                if (!mbar_wait(&k_full[s], (j / A3_KST) & 1))
                    return false;
                tc_fence_after();
                const uint32_t sk = smem_u32(smem + A3_OFF_K + s * TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
                    mma_bf16_ss(tmem + (j & 1) * 128, sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), id_s128, kk > 0);
                }
                mma_commit(&k_empty[s]);
                mma_commit(&s_full[j & 1]);
                return true;
            }
            for (int x = 0; x < 2; ++x) {
                const int i = 2 * j + x, s = i % A3_KST;
                if (!mbar_wait(&k_full[s], (i / A3_KST) & 1))
                    return false;
                tc_fence_after();
                const uint32_t sk = smem_u32(smem + A3_OFF_K + s * TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
                    mma_bf16_ss(tmem + (j & 1) * 128 + (x ? LANE16 : 0u), sdesc_sw128(sq + x * 8192 + off, 16, 1024),
                                sdesc_sw128(sk + off, 16, 1024), id_s, kk > 0);
                }
                mma_commit(&k_empty[s]);
            }
            mma_commit(&s_full[j & 1]);
            return true;
        };
        bool ok = mbar_wait(q_full, 0);
        for (int j = 0; j < 2 && j < nkv && ok; ++j)
            ok = issue_s(j);
        for (int j = 0; j < nkv && ok; ++j) {
            if (!(ok = mbar_wait(&p_full[j & 1], (j >> 1) & 1)))
                break;
            if (every) {
                const int sv = j % A3_VST;
                if (!(ok = mbar_wait(&v_full[sv], (j / A3_VST) & 1)))
                    break;
                tc_fence_after();
                const uint32_t vb = smem_u32(smem + A3_OFF_V + sv * TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_bf16_ts(tmem + T_O, tmem + (j & 1) * 128 + p_col(kk), sdesc_sw128(vb + kk * 2048, HALF, 1024), id_pv128, (j | kk) != 0);
                mma_commit(&v_empty[sv]);
            }
            for (int x = 0; x < 2 && ok && !every; ++x) {
                const int i = 2 * j + x, sv = i % A3_VST;
                if (!(ok = mbar_wait(&v_full[sv], (i / A3_VST) & 1)))
                    break;
                tc_fence_after();
                const uint32_t vb = smem_u32(smem + A3_OFF_V + sv * TILE);
                const uint32_t lane = x ? LANE16 : 0u;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_bf16_ts(tmem + T_O + lane, tmem + (j & 1) * 128 + lane + p_col(kk), sdesc_sw128(vb + kk * 2048, HALF, 1024), id_pv,
                                (j | kk) != 0);
                mma_commit(&v_empty[sv]);
            }
            if (!ok)
                break;
            mma_commit(pv_done);
            if (j + 2 < nkv)
                ok = issue_s(j + 2);
        }
        mma_commit(drain);
        mbar_wait(drain, 0);
    } else if (nkv > 0 && warp >= 2) {
        // -------------------------------------------------------------------------------------- softmax
        const int hc = (warp - 2) >> 2; // 64-key half of the step this warp handles
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane_id(); // TMEM lane
        // query unit of this lane's row and the row's index inside it (M = 64 layout: 16 lanes of each quarter per
        // unit; M = 128 layout of a dense-row tile: lane = row of the tile)
        const int x = every ? quarter >> 1 : (lane_id() >> 4) & 1;
        const int m = every ? (quarter & 1) * 32 + lane_id() : quarter * 16 + (lane_id() & 15);
        const uint32_t lane_base = uint32_t(quarter * 32) << 16;
        const uint32_t tO = tmem + lane_base + T_O + hc * 64;
        float* red = reinterpret_cast<float*>(smem + A3_OFF_RED); // [3 slots][2 slices][128 rows]
        const float sl2 = p.scale * 1.4426950408889634f;
        // STATIC: every score is at most p.static_max (log2 units), the row maximum throughout, so the two slices of a
        // row exchange nothing per step and O is never rescaled
        float m_run = STATIC ? p.static_max : -INFINITY, l = 0.f;
        bool ok = true;
        int4 e_next = entry(0, x);
        for (int j = 0; j < nkv; ++j) {
            const uint32_t tS = tmem + lane_base + (j & 1) * 128;
            // The keys of this slice the row may see: the first n rows of its unit's key unit hc
            const int4 e = e_next;
            if (j + 1 < nkv)
                e_next = entry(j + 1, x);
            const int first = hc ? e.y : e.x;
            const int n = first < 0 ? 0 : min((e.z >> (8 * hc)) & 0xff, 64);
            // the whole warp may skip the exponentials only when neither unit's rows see a key here
            const bool warp_dead = __all_sync(0xffffffffu, n == 0);
            if (!(ok = mbar_wait(&s_full[j & 1], (j >> 1) & 1)))
                break;
            tc_fence_after();
            float s[64];
            float mx = -INFINITY;
            if (!warp_dead) {
                {
                    uint32_t r[2][32];
                    tmem_ld32(tS + hc * 64, r[0]);
                    tmem_ld32(tS + hc * 64 + 32, r[1]);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 2; ++c)
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            s[c * 32 + i] = __uint_as_float(r[c][i]);
                }
                if (n < 64) {
#pragma unroll
                    for (int c = 0; c < 64; ++c)
                        if (c >= n)
                            s[c] = -INFINITY;
                }
                if constexpr (!STATIC) {
                    float mp[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        mp[i] = fmaxf(s[2 * i], s[2 * i + 1]);
#pragma unroll
                    for (int c = 16; c < 64; c += 16)
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            mp[i] = max3f(mp[i], s[c + 2 * i], s[c + 2 * i + 1]);
                    mx = max3f(max3f(mp[0], mp[1], mp[2]), max3f(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
                }
            }
            if constexpr (!STATIC) {
                // the row maximum over both slices
                float* slot = red + (j & 1) * 256;
                slot[hc * 128 + row] = mx;
                __syncwarp();
                if (elect_one_lane())
                    mbar_arrive(xchg);
                if (!(ok = mbar_wait(xchg, j & 1)))
                    break;
                mx = fmaxf(mx, slot[(hc ^ 1) * 128 + row]);
            }
            const float m_cand = mx * sl2;
            const bool need = !STATIC && m_cand > m_run + kRescaleThreshold;
            const float m_use = need ? m_cand : m_run;
            const float alpha = need ? ex2_approx(m_run - m_use) : 1.f;
            const float msub = m_use == -INFINITY ? 0.f : m_use;
            const float2 scale2 = make_float2(sl2, sl2), neg2 = make_float2(-msub, -msub);
            uint32_t pk[32];
            float rs = 0.f;
            if (!warp_dead) {
                float2 sp[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float2 xx = fma2(make_float2(s[2 * c], s[2 * c + 1]), scale2, neg2);
                    const float2 ev = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
                    sp[c & 3] = add2(sp[c & 3], ev);
                    pk[c] = pack_bf16x2(ev.x, ev.y);
                }
                const float2 s01 = add2(add2(sp[0], sp[1]), add2(sp[2], sp[3]));
                rs = s01.x + s01.y;
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c)
                    pk[c] = 0u;
            }
            if (!STATIC && j > 0 && __any_sync(0xffffffffu, need)) {
                // O holds PV(0..j-2) for sure; wait for PV(j-1) before scaling it
                if (!(ok = mbar_wait(pv_done, (j - 1) & 1)))
                    break;
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    uint32_t o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(tO + c * 32, o);
                }
            }
            l = l * alpha + rs;
            m_run = m_use;
            tmem_st32(tS + hc * 64, pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (elect_one_lane())
                mbar_arrive(&p_full[j & 1]);
        }
        if (ok) {
            float* slot = red + 2 * 256;
            slot[hc * 128 + row] = l;
            __syncwarp();
            if (elect_one_lane())
                mbar_arrive(xchg);
            ok = mbar_wait(xchg, STATIC ? 0 : nkv & 1);
            l = slot[row] + slot[128 + row];
        }
        // The last two PVs may both be pending here (S(j) completing implies only PV(j - 2) did), which a parity wait
        // on pv_done cannot tell apart; drain completes once, after every MMA of the CTA.
        if (ok && mbar_wait(drain, 0)) {
            tc_fence_after();
            const int first = x ? qr.y : qr.x, nq = x ? qr.w : qr.z;
            const int out_row = first >= 0 && m < nq ? first + m : -1;
            const float inv = l > 0.f ? 1.f / l : 0.f;
            __nv_bfloat16* dst = out_ptr(p, out_row, head, hc * 64);
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                uint32_t o[32];
                tmem_ld32(tO + c * 32, o);
                tmem_wait_ld();
                if (dst) {
                    uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        d4[i] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                                           pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                                           pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                                           pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Merges the two halves of a split dense launch: per (row, head) one warp, four dims a lane; the halves' outputs
// weighted by 2^(m_s - max(m_0, m_1)), divided by the weighted sum, bf16 into the output (this rank's or its owner's).
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnParams p)
{
    const size_t item = size_t(blockIdx.x) * 8 + warp_id();
    if (item >= size_t(p.rows) * p.heads)
        return;
    const int row = int(item / p.heads), head = int(item % p.heads);
    const size_t i1 = size_t(p.rows) * p.heads + item;
    const float2 a = *reinterpret_cast<const float2*>(p.part_ml + item * 2);
    const float2 b = *reinterpret_cast<const float2*>(p.part_ml + i1 * 2);
    const float mx = fmaxf(a.x, b.x);
    const float wa = mx == -INFINITY ? 0.f : ex2_approx(a.x - mx), wb = mx == -INFINITY ? 0.f : ex2_approx(b.x - mx);
    const float sum = wa * a.y + wb * b.y;
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    const float4 oa = *reinterpret_cast<const float4*>(p.part_o + item * 128 + lane_id() * 4);
    const float4 ob = *reinterpret_cast<const float4*>(p.part_o + i1 * 128 + lane_id() * 4);
    __nv_bfloat16* dst = out_ptr(p, row, head, lane_id() * 4);
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2((oa.x * wa + ob.x * wb) * inv, (oa.y * wa + ob.y * wb) * inv),
                                                pack_bf16x2((oa.z * wa + ob.z * wb) * inv, (oa.w * wa + ob.w * wb) * inv));
}

// A dense launch of this many rows and heads splits its keys in two when its CTAs fill fewer than six waves.
bool split_dense(int rows, int heads)
{
    const long long ctas = (long long)((rows + 255) / 256) * heads;
    return (rows + 127) / 128 >= 4 && ctas < 6LL * num_sms();
}

CUtensorMap rows_map(const void* base, int heads, int rows, int64_t row_stride, int head_dim = 128)
{
    const uint64_t dims[3] = {uint64_t(head_dim), uint64_t(heads), uint64_t(rows > 0 ? rows : 1)};
    const uint64_t str[2] = {uint64_t(head_dim) * 2, uint64_t(row_stride) * 2};
    const uint32_t box[3] = {64, 1, 64};
    return make_tmap(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, str, box);
}

} // namespace

size_t attention_split_bytes(int rows, int heads)
{
    if (rows <= 0 || heads <= 0 || !split_dense(rows, heads))
        return 0;
    return size_t(2) * rows * heads * (128 + 2) * sizeof(float);
}

int attention(const AttnParams& p, cudaStream_t s)
{
    if (p.heads <= 0 || !p.q || !p.k || !p.v || !p.out || (p.row_stride * 2) % 16 || (p.out_row_stride * 2) % 16)
        throw CudaError("attention: bad arguments");
    const bool sparse = p.blocks != nullptr;
    if (sparse && (p.grid.cubes() <= 0 || !p.nblocks || !p.q_rows || p.q_tiles <= 0 || p.rows != p.grid.rows()))
        throw CudaError("attention: bad sparse arguments");
    if (p.head_dim != 128 && (p.head_dim != 64 || sparse || p.peer_out[0] || p.part_o))
        throw CudaError("attention: heads of 64 dims are for dense attention on one rank only");
    if (p.seg_rows < 0 || (p.seg_rows > 0 && (sparse || p.part_o || p.seg_stride < p.seg_rows || p.rows % p.seg_stride)))
        throw CudaError("attention: segments must tile the rows (rows a multiple of seg_stride >= seg_rows; dense, unsplit)");
    if (p.rows <= 0)
        return 0;
    Maps maps;
    maps.q = rows_map(p.q, p.heads, p.rows, p.row_stride, p.head_dim);
    maps.k = rows_map(p.k, p.heads, p.rows, p.row_stride, p.head_dim);
    maps.v = rows_map(p.v, p.heads, p.rows, p.row_stride, p.head_dim);
    static std::atomic<uint64_t> opt_in[6];
    if (sparse) {
        // Query tiles have their own key lists, so one tile per CTA with double-buffered scores.
        if (p.static_max > 0.f && p.static_max <= kMaxStaticBound) {
            smem_opt_in(attn3_kernel<true>, A3_SMEM, opt_in[5]);
            attn3_kernel<true><<<p.q_tiles * p.heads, NT3, A3_SMEM, s>>>(maps, p);
        } else {
            smem_opt_in(attn3_kernel<false>, A3_SMEM, opt_in[1]);
            attn3_kernel<false><<<p.q_tiles * p.heads, NT3, A3_SMEM, s>>>(maps, p);
        }
        H3_CUDA(cudaGetLastError());
        return 1;
    }
    // Dense: two query tiles per CTA share every K/V tile (half the shared-memory traffic per FLOP).
    const int segs = p.seg_rows > 0 ? p.rows / int(p.seg_stride) : 1;
    const int pairs = ((p.seg_rows > 0 ? p.seg_rows : p.rows) + 255) / 256;
    const bool bounded = p.static_max > 0.f && p.static_max <= kMaxStaticBound;
    constexpr int SB = A2_SPLIT_BOUNDED, NTB = 64 + 256 * SB, NTO = 64 + 256 * A2_SPLIT;
    if (p.head_dim == 64) {
        const dim3 grid(pairs * segs, p.heads, 1);
        if (bounded) {
            using SM = A2Smem<64, SB, true>;
            smem_opt_in(attn2_kernel<SB, 64, true>, SM::TOTAL, opt_in[4]);
            attn2_kernel<SB, 64, true><<<grid, NTB, SM::TOTAL, s>>>(maps, p);
        } else {
            using SM = A2Smem<64, A2_SPLIT, false>;
            smem_opt_in(attn2_kernel<A2_SPLIT, 64, false>, SM::TOTAL, opt_in[2]);
            attn2_kernel<A2_SPLIT, 64, false><<<grid, NTO, SM::TOTAL, s>>>(maps, p);
        }
        H3_CUDA(cudaGetLastError());
        return 1;
    }
    // A launch of few waves (several ranks leave each a few heads) loses much of its last wave; splitting every CTA's
    // keys in two, given scratch for the halves, doubles the CTAs, and a combine kernel merges them.
    const int parts = segs == 1 && p.part_o && p.part_ml && split_dense(p.rows, p.heads) ? 2 : 1;
    const dim3 grid(pairs * segs, p.heads, parts);
    if (bounded) {
        using SM = A2Smem<128, SB, true>;
        smem_opt_in(attn2_kernel<SB, 128, true>, SM::TOTAL, opt_in[3]);
        attn2_kernel<SB, 128, true><<<grid, NTB, SM::TOTAL, s>>>(maps, p);
    } else {
        using SM = A2Smem<128, A2_SPLIT, false>;
        smem_opt_in(attn2_kernel<A2_SPLIT, 128, false>, SM::TOTAL, opt_in[0]);
        attn2_kernel<A2_SPLIT, 128, false><<<grid, NTO, SM::TOTAL, s>>>(maps, p);
    }
    H3_CUDA(cudaGetLastError());
    if (parts == 1)
        return 1;
    const size_t items = size_t(p.rows) * p.heads;
    attn_combine_kernel<<<unsigned((items + 7) / 8), 256, 0, s>>>(p);
    H3_CUDA(cudaGetLastError());
    return 2;
}

} // namespace h3
