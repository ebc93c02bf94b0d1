// The H3 step's projection GEMMs (q/k/v, out, fc1, fc2, the patch and text projections) on sm_100a tensor cores.
//
// One persistent kernel per GEMM, one CTA per SM, three warp roles:
//   warp 0      TMA producer: A and B tiles (128-byte swizzled) into a STAGES-deep shared-memory ring
//   warp 1      MMA issuer:   tcgen05.mma (M=128, N=BN, K=16 bf16 / 32 int8) into one of two TMEM accumulators
//   warps 2..5  epilogue:     tcgen05.ld of the finished accumulator, the fused epilogue, stores to HBM
// The two TMEM accumulators let the epilogue of tile i overlap the main loop of tile i+1. Tiles are visited in
// groups of GROUP_M row tiles so the A and B panels a wave of CTAs touches stay in L2.
//
// The epilogues replace the reference's separate row kernels (rms_mod_rows follows elsewhere):
//   qkv         heads_partial: per-head RMS norm of q and k and the 3-axis rotary, written in the head-split layout
//               the attention (and the sequence-parallel all-to-all) reads
//   gate_resid  gate_add_rows: x += gate * (y + bias)
//   swiglu      swiglu_rows: silu(gate) * value of fc1's [gate; value] halves
#include "common.hpp"
#include "gemm.cuh"
#include "ptx.cuh"

#include <algorithm>

namespace h3 {

namespace {

constexpr int BM = 128;
constexpr int KBYTES = 128;       // bytes of K per stage and row: 64 bf16 or 128 int8
constexpr int STAGES = 4;
constexpr int GROUP_M = 16;
constexpr int NUM_THREADS = 192;  // 6 warps

template <int BN, Epi EPI>
struct Smem {
    static constexpr int A_BYTES = BM * KBYTES;
    static constexpr int B_BYTES = BN * KBYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // the q/k/v and SwiGLU epilogues stage one 128 x 128 bf16 tile (two 128-byte-swizzled halves) for TMA stores
    static constexpr int STAGING = (EPI == Epi::qkv || EPI == Epi::swiglu) ? BM * 256 : 0;
    static constexpr int TOTAL = STAGES * STAGE_BYTES + STAGING + 1024 /* alignment slack */ + 256 /* barriers */;
};

// Destination tensor maps of the TMA-store epilogues. q/k/v: one per rank that owns heads, (dim, q/k/v x head slot,
// row) over that rank's block of this rank's rows, in its receive buffer (fused exchange) or in this rank's send
// layout. SwiGLU: m[0] is the output [M][ldo] (box 64 columns x 128 rows).
struct OutMaps {
    CUtensorMap m[8];
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); } // the 4 epilogue warps

__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* smem_src, int32_t c0, int32_t c1, int32_t c2)
{
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tmap)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int32_t c0, int32_t c1)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(tmap)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& tm, int& tn)
{
    const int group_size = GROUP_M * tiles_n;
    const int g = tile / group_size;
    const int first_m = g * GROUP_M;
    const int gm = min(tiles_m - first_m, GROUP_M);
    const int in_group = tile - g * group_size;
    tm = first_m + in_group % gm;
    tn = in_group / gm;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v)
{
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        d[i] = make_uint4(pack_bf16x2(v[8 * i + 0], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                          pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
}

// Loads `NCHUNK` 32-column chunks of this thread's accumulator row (starting at column `col0`) as floats, dequantising
// int32 with the row and column scales when IS_I8.
template <bool IS_I8, int NCHUNK>
__device__ __forceinline__ void load_acc(uint32_t taddr, int col0, float* v, float a_scale, const float* b_scale_cols)
{
    uint32_t r[NCHUNK][32];
#pragma unroll
    for (int c = 0; c < NCHUNK; ++c)
        tmem_ld32(taddr + col0 + c * 32, r[c]);
    tmem_wait_ld();
#pragma unroll
    for (int c = 0; c < NCHUNK; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if constexpr (IS_I8)
                v[c * 32 + i] = float(int32_t(r[c][i])) * (a_scale * b_scale_cols[c * 32 + i]);
            else
                v[c * 32 + i] = __uint_as_float(r[c][i]);
        }
}

template <int BN, Epi EPI, bool IS_I8>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, uint32_t tacc, int m0, int n0, uint8_t* stage, const OutMaps* om)
{
    const int quarter = warp_id() & 3;
    const int row = quarter * 32 + lane_id();
    const int gm = m0 + row;
    const bool valid = gm < p.M;
    const uint32_t taddr = tacc + (uint32_t(quarter * 32) << 16);
    const float a_scale = (IS_I8 && valid) ? p.a_scale[gm] : 1.0f;
    const float* bsc = IS_I8 ? p.b_scale + n0 : nullptr;

    if constexpr (EPI == Epi::qkv) {
        // BN = 256 covers two heads; the q/k/v section never changes inside a tile (inner % 256 == 0). Every epilogue
        // thread takes part in each head (the staging barriers), rows past M included (their stores are clipped).
        const int sec = n0 / p.inner;
        const int grow = valid ? gm : p.M - 1; // rows past M read a valid row's rotary entry
#pragma unroll 1
        for (int hh = 0; hh < BN / 128; ++hh) {
            float v[128];
            load_acc<IS_I8, 4>(taddr, hh * 128, v, a_scale, IS_I8 ? bsc + hh * 128 : nullptr);
            const int col = n0 + hh * 128;
            if (p.bias) {
                const float4* b4 = reinterpret_cast<const float4*>(p.bias + col);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float4 b = __ldg(b4 + i);
                    v[4 * i] += b.x, v[4 * i + 1] += b.y, v[4 * i + 2] += b.z, v[4 * i + 3] += b.w;
                }
            }
            if (sec < 2) {
                float ss = 0.f;
#pragma unroll
                for (int i = 0; i < 128; ++i)
                    ss += v[i] * v[i];
                const float rinv = rsqrtf(ss * (1.0f / 128.0f) + p.eps);
                const float* w = sec == 0 ? p.qn_w : p.kn_w;
#pragma unroll
                for (int i = 0; i < 128; ++i)
                    v[i] = v[i] * rinv * __ldg(w + i);
                const float2* cs = reinterpret_cast<const float2*>(p.rope) + size_t(grow) * 48;
#pragma unroll
                for (int j = 0; j < 48; ++j) {
                    const float2 t = __ldg(cs + j);
                    const float a = v[j], b = v[j + 48];
                    v[j] = a * t.x - b * t.y;
                    v[j + 48] = b * t.x + a * t.y;
                }
            }
            const int head = (col % p.inner) / 128;
            const int rank = head / p.heads_per_rank, hl = head % p.heads_per_rank;
            // Stage the head tile in shared memory (once the previous head's store has read it) and let TMA store it
            // into the head group's owner: its receive buffer over NVLink (fused exchange) or this rank's send layout.
            if (threadIdx.x == 64)
                bulk_wait_read0();
            epi_bar();
#pragma unroll
            for (int c8 = 0; c8 < 16; ++c8) {
                const int half = c8 >> 3, c = c8 & 7;
                const uint4 w = make_uint4(pack_bf16x2(v[c8 * 8 + 0], v[c8 * 8 + 1]), pack_bf16x2(v[c8 * 8 + 2], v[c8 * 8 + 3]),
                                           pack_bf16x2(v[c8 * 8 + 4], v[c8 * 8 + 5]), pack_bf16x2(v[c8 * 8 + 6], v[c8 * 8 + 7]));
                *reinterpret_cast<uint4*>(stage + half * (BM * 128) + row * 128 + ((c ^ (row & 7)) << 4)) = w;
            }
            fence_proxy_async_smem();
            epi_bar();
            if (threadIdx.x == 64) {
                const int slot = sec * p.heads_per_rank + hl;
                tma_store_3d(&om->m[rank], stage, 0, slot, m0);
                tma_store_3d(&om->m[rank], stage + BM * 128, 64, slot, m0);
                bulk_commit();
            }
        }
    } else if constexpr (EPI == Epi::swiglu) {
        // Gate columns [0,128) and value columns [128,256) of the tile pair up: 128 outputs per row, staged as two
        // 128-byte-swizzled halves of 64 columns and written by two TMA stores (rows past M are clipped by the store,
        // so every thread takes part in the staging).
        if (threadIdx.x == 64)
            bulk_wait_read0(); // the previous tile's stores have read the staging buffer
        epi_bar();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            float g[32], u[32];
            load_acc<IS_I8, 1>(taddr, c * 32, g, a_scale, IS_I8 ? bsc + c * 32 : nullptr);
            load_acc<IS_I8, 1>(taddr, 128 + c * 32, u, a_scale, IS_I8 ? bsc + 128 + c * 32 : nullptr);
            if (p.bias) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    g[i] += __ldg(p.bias + n0 + c * 32 + i);
                    u[i] += __ldg(p.bias + n0 + 128 + c * 32 + i);
                }
            }
#pragma unroll
            for (int i = 0; i < 32; ++i)
                g[i] = silu(g[i]) * u[i];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int chunk = (c & 1) * 4 + q;
                const uint4 w = make_uint4(pack_bf16x2(g[8 * q + 0], g[8 * q + 1]), pack_bf16x2(g[8 * q + 2], g[8 * q + 3]),
                                           pack_bf16x2(g[8 * q + 4], g[8 * q + 5]), pack_bf16x2(g[8 * q + 6], g[8 * q + 7]));
                *reinterpret_cast<uint4*>(stage + (c >> 1) * (BM * 128) + row * 128 + ((chunk ^ (row & 7)) << 4)) = w;
            }
        }
        fence_proxy_async_smem();
        epi_bar();
        if (threadIdx.x == 64) {
            tma_store_2d(&om->m[0], stage, n0 / 2, m0);
            tma_store_2d(&om->m[0], stage + BM * 128, n0 / 2 + 64, m0);
            bulk_commit();
        }
    } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            const int col = n0 + c * 32;
            if constexpr (EPI == Epi::s32) {
                uint32_t r[32];
                tmem_ld32(taddr + c * 32, r);
                tmem_wait_ld();
                if (!valid)
                    continue;
                uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<int32_t*>(p.out) + size_t(gm) * p.ldo + col);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    d[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
            } else {
                float v[32];
                load_acc<IS_I8, 1>(taddr, c * 32, v, a_scale, IS_I8 ? bsc + c * 32 : nullptr);
                if (!valid)
                    continue;
                if (p.bias) {
                    const float4* b4 = reinterpret_cast<const float4*>(p.bias + col);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 b = __ldg(b4 + i);
                        v[4 * i] += b.x, v[4 * i + 1] += b.y, v[4 * i + 2] += b.z, v[4 * i + 3] += b.w;
                    }
                }
                if constexpr (EPI == Epi::bf16) {
                    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(gm) * p.ldo + col, v);
                } else if constexpr (EPI == Epi::f32) {
                    float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + size_t(gm) * p.ldo + col);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                } else if constexpr (EPI == Epi::gate_resid) {
                    const float4* g4 = reinterpret_cast<const float4*>(
                        p.mod + (size_t(p.mod_idx[gm]) * 6 + p.gate_slot) * p.dim + col);
                    float4* x4 = reinterpret_cast<float4*>(p.x + size_t(gm) * p.ldx + col);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 g = __ldg(g4 + i);
                        float4 x = x4[i];
                        x.x += g.x * v[4 * i], x.y += g.y * v[4 * i + 1], x.z += g.z * v[4 * i + 2], x.w += g.w * v[4 * i + 3];
                        x4[i] = x;
                    }
                }
            }
        }
    }
}

template <int BN, Epi EPI, bool IS_I8>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmParams p,
                const __grid_constant__ OutMaps om)
{
    using SM = Smem<BN, EPI>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
    uint8_t* stage = smem + STAGES * SM::STAGE_BYTES; // q/k/v epilogue staging (1024-aligned)
    uint64_t* bars = reinterpret_cast<uint64_t*>(stage + SM::STAGING);
    uint64_t* full = bars;                 // [STAGES]
    uint64_t* empty = bars + STAGES;       // [STAGES]
    uint64_t* tfull = bars + 2 * STAGES;   // [2]
    uint64_t* tempty = bars + 2 * STAGES + 2; // [2]
    uint64_t* drain = bars + 2 * STAGES + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);

    const int warp = warp_id();
    const int tiles_m = (p.M + BM - 1) / BM;
    const int tiles_n = p.N / BN;
    const int num_tiles = tiles_m * tiles_n;
    const int kb_per_chunk = (p.K / p.a_chunks + KBYTES / (IS_I8 ? 1 : 2) - 1) / (KBYTES / (IS_I8 ? 1 : 2));
    const int num_kb = kb_per_chunk * p.a_chunks;
    constexpr int KELEMS = KBYTES / (IS_I8 ? 1 : 2);

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 4);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0 && elect_one_lane()) {
        // ---------------------------------------------------------------------------------------- producer
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            int tm, tn;
            tile_coords(tile, tiles_m, tiles_n, tm, tn);
            for (int kb = 0; kb < num_kb; ++kb, ++it) {
                const int s = it % STAGES;
                if (!(ok = mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1)))
                    break;
                uint8_t* sa = smem + s * SM::STAGE_BYTES;
                uint8_t* sb = sa + SM::A_BYTES;
                mbar_arrive_expect_tx(&full[s], SM::STAGE_BYTES);
                // A's chunk and column inside it; B's column is the same k in the unsplit K.
                const int chunk = kb / kb_per_chunk, kin = (kb % kb_per_chunk) * KELEMS;
                tma_load_3d(sa, &tmA, &full[s], kin, tm * BM, chunk);
                tma_load_2d(sb, &tmB, &full[s], chunk * (p.K / p.a_chunks) + kin, tn * BN);
            }
        }
        // Wait for the loads still in flight to land before the CTA can exit.
        if (ok)
            for (uint32_t j = it >= STAGES ? it - STAGES : 0; j < it; ++j)
                mbar_wait(&empty[j % STAGES], (j / STAGES) & 1);
    } else if (warp == 1 && elect_one_lane()) {
        // ------------------------------------------------------------------------------------- MMA issuer
        const uint32_t idesc = IS_I8 ? idesc_s8(BM, BN) : idesc_bf16(BM, BN);
        uint32_t it = 0, t_local = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t_local) {
            const int acc = t_local & 1;
            if (!(ok = mbar_wait(&tempty[acc], ((t_local >> 1) & 1) ^ 1)))
                break;
            tc_fence_after();
            const uint32_t d = tmem_base + acc * BN;
            for (int kb = 0; kb < num_kb; ++kb, ++it) {
                const int s = it % STAGES;
                if (!(ok = mbar_wait(&full[s], (it / STAGES) & 1)))
                    break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * SM::STAGE_BYTES);
                const uint32_t sb = sa + SM::A_BYTES;
#pragma unroll
                for (int k = 0; k < KBYTES / 32; ++k) {
                    const uint64_t ad = sdesc_sw128(sa + k * 32, 16, 1024);
                    const uint64_t bd = sdesc_sw128(sb + k * 32, 16, 1024);
                    if constexpr (IS_I8)
                        mma_i8_ss(d, ad, bd, idesc, (kb | k) != 0);
                    else
                        mma_bf16_ss(d, ad, bd, idesc, (kb | k) != 0);
                }
                mma_commit(&empty[s]);
            }
            if (ok)
                mma_commit(&tfull[acc]);
        }
        // Every MMA this thread issued has completed once `drain` flips.
        mma_commit(drain);
        mbar_wait(drain, 0);
    } else if (warp >= 2) {
        // ---------------------------------------------------------------------------------------- epilogue
        uint32_t t_local = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t_local) {
            const int acc = t_local & 1;
            if (!mbar_wait(&tfull[acc], (t_local >> 1) & 1))
                break;
            tc_fence_after();
            int tm, tn;
            tile_coords(tile, tiles_m, tiles_n, tm, tn);
            epilogue_tile<BN, EPI, IS_I8>(p, tmem_base + acc * BN, tm * BM, tn * BN, stage, &om);
            tc_fence_before();
            __syncwarp();
            if (elect_one_lane())
                mbar_arrive(&tempty[acc]);
        }
        if ((EPI == Epi::qkv || EPI == Epi::swiglu) && threadIdx.x == 64)
            bulk_wait0(); // the staged tiles' TMA stores are complete
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * BN);
    }
}

template <int BN, Epi EPI, bool IS_I8>
void launch(const void* A, const void* B, const GemmParams& p, cudaStream_t s)
{
    const int kelems = IS_I8 ? 128 : 64;
    const CUtensorMapDataType dt = IS_I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t esz = IS_I8 ? 1 : 2;
    const uint64_t kc = uint64_t(p.K / p.a_chunks);
    const uint64_t lda = p.lda ? uint64_t(p.lda) : kc;
    const uint64_t arows = p.a_rows_stride ? uint64_t(p.a_rows_stride) : uint64_t(p.M);
    const uint64_t ldb = p.ldb ? uint64_t(p.ldb) : uint64_t(p.K);
    const uint64_t adims[3] = {kc, uint64_t(p.M), uint64_t(p.a_chunks)};
    const uint64_t astr[2] = {lda * esz, arows * lda * esz};
    const uint32_t abox[3] = {uint32_t(kelems), 128, 1};
    const CUtensorMap ta = make_tmap(dt, 3, A, adims, astr, abox);
    const uint64_t bdims[2] = {uint64_t(p.K), uint64_t(p.N)};
    const uint64_t bstr[1] = {ldb * esz};
    const uint32_t bbox[2] = {uint32_t(kelems), uint32_t(BN)};
    const CUtensorMap tb = make_tmap(dt, 2, B, bdims, bstr, bbox);
    static std::atomic<uint64_t> opt_in;
    const int smem = Smem<BN, EPI>::TOTAL;
    smem_opt_in(gemm_kernel<BN, EPI, IS_I8>, smem, opt_in);
    const int tiles = ((p.M + BM - 1) / BM) * (p.N / BN);
    const int grid = std::min(tiles, num_sms());
    OutMaps om{};
    if constexpr (EPI == Epi::qkv) {
        // rank r's block of this rank's rows: in r's receive buffer (fused exchange) or in this rank's send layout
        const int P = p.inner / 128 / p.heads_per_rank;
        const uint64_t slots = 3 * uint64_t(p.heads_per_rank);
        const uint64_t odims[3] = {128, slots, uint64_t(p.rows_local)};
        const uint64_t ostr[2] = {256, slots * 256};
        const uint32_t obox[3] = {64, 1, 128};
        for (int r = 0; r < P; ++r) {
            const size_t block = size_t(p.peer_out[r] ? p.my_rank : r) * p.rows_local * slots * 128;
            const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(p.peer_out[r] ? p.peer_out[r] : p.out) + block;
            om.m[r] = make_tmap(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, odims, ostr, obox);
        }
    }
    if constexpr (EPI == Epi::swiglu) {
        const uint64_t odims[2] = {uint64_t(p.N / 2), uint64_t(p.M)};
        const uint64_t ostr[1] = {uint64_t(p.ldo) * 2};
        const uint32_t obox[2] = {64, 128};
        om.m[0] = make_tmap(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.out, odims, ostr, obox);
    }
    gemm_kernel<BN, EPI, IS_I8><<<grid, NUM_THREADS, smem, s>>>(ta, tb, p, om);
    H3_CUDA(cudaGetLastError());
}

void check_shape(const GemmParams& p, Epi epi, int bn, bool i8)
{
    const int kelems = i8 ? 128 : 64;
    if (p.M <= 0 || p.N <= 0 || p.K <= 0)
        throw std::runtime_error("gemm: empty shape");
    if (p.N % bn)
        throw std::runtime_error("gemm: N must be a multiple of " + std::to_string(bn));
    if (p.K % p.a_chunks || (p.a_chunks > 1 && (p.K / p.a_chunks) % kelems))
        throw std::runtime_error("gemm: chunked A needs chunk widths that are multiples of the K tile");
    if ((p.K * (i8 ? 1 : 2)) % 16)
        throw std::runtime_error("gemm: K rows must be 16-byte multiples");
    if (epi == Epi::qkv && (p.inner % 256 || !p.rope || !p.qn_w || !p.kn_w || p.heads_per_rank <= 0 ||
                            (p.inner / 128) % p.heads_per_rank || p.inner / 128 / p.heads_per_rank > 8 || p.rows_local < p.M))
        throw std::runtime_error("gemm: qkv epilogue arguments");
    if (epi == Epi::qkv)
        for (int r = 0; r < p.inner / 128 / p.heads_per_rank; ++r)
            if (!p.peer_out[r] && !p.out)
                throw std::runtime_error("gemm: qkv epilogue needs an output for every head group");
    if (epi == Epi::gate_resid && (!p.x || !p.mod || !p.mod_idx))
        throw std::runtime_error("gemm: gate_resid epilogue arguments");
    if (epi == Epi::s32 && !i8)
        throw std::runtime_error("gemm: s32 output is for the int8 GEMM");
    if (i8 && (!p.a_scale || !p.b_scale) && epi != Epi::s32)
        throw std::runtime_error("gemm: int8 needs row and column scales");
}

} // namespace

void gemm_bf16(const void* A, const void* B, const GemmParams& p, Epi epi, cudaStream_t s)
{
    check_shape(p, epi, 256, false);
    switch (epi) {
    case Epi::bf16: return launch<256, Epi::bf16, false>(A, B, p, s);
    case Epi::f32: return launch<256, Epi::f32, false>(A, B, p, s);
    case Epi::qkv: return launch<256, Epi::qkv, false>(A, B, p, s);
    case Epi::gate_resid: return launch<256, Epi::gate_resid, false>(A, B, p, s);
    case Epi::swiglu: return launch<256, Epi::swiglu, false>(A, B, p, s);
    default: throw std::runtime_error("gemm_bf16: unsupported epilogue");
    }
}

void gemm_s8(const void* A, const void* B, const GemmParams& p, Epi epi, cudaStream_t s)
{
    check_shape(p, epi, 256, true);
    switch (epi) {
    case Epi::s32: return launch<256, Epi::s32, true>(A, B, p, s);
    case Epi::bf16: return launch<256, Epi::bf16, true>(A, B, p, s);
    case Epi::qkv: return launch<256, Epi::qkv, true>(A, B, p, s);
    case Epi::gate_resid: return launch<256, Epi::gate_resid, true>(A, B, p, s);
    case Epi::swiglu: return launch<256, Epi::swiglu, true>(A, B, p, s);
    default: throw std::runtime_error("gemm_s8: unsupported epilogue");
    }
}

} // namespace h3
