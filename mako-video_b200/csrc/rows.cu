// Row kernels (HBM-bound): 128-bit loads and stores, one CTA (or warp) per row, warp-shuffle reductions.
#include "common.hpp"
#include "ptx.cuh"
#include "rows.cuh"

#include <algorithm>
#include <cmath>

namespace h3 {

namespace {

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* red)
{
    v = warp_max(v);
    if (lane_id() == 0)
        red[warp_id()] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i)
        t = fmaxf(t, red[i]);
    __syncthreads();
    return t;
}


// y = RMSNorm(x) * w * (1 + scale[r]) + shift[r] per row, bf16, fp32 or int8 (+ row scale) out.
// A persistent kernel: CTA b owns a contiguous range of rows and walks it in batches of nb rows through a ring of
// nbufs shared-memory buffers filled by bulk copies (as many as fit in ~200 KB: the following batches stream in while
// one is worked on; the bytes in flight per SM set the bandwidth). The
// columns are split across the CTA's eight warps: each lane keeps w (1 + scale) and shift of its columns in registers,
// reloading them only when a row's modulation index changes (the boundaries of the packed row order's segments), so
// a row is read from HBM once and from shared memory twice (sum of squares, then the output), and the modulation
// vectors are not re-read per row. A row's sum of squares (and, for int8, its maximum) is combined from the warps'
// partials through shared memory in a fixed order.
// Shared memory: nbufs mbarriers, the partials [RM_BATCH][RM_WARPS] (sum) and [RM_BATCH][RM_WARPS] (max), then at
// byte RM_ROWS_OFF the row buffers [nbufs][nb][d] fp32. Batches hold as many rows as two buffers fit (each batch costs
// two CTA barriers, so narrow rows take bigger batches).
constexpr int RM_WARPS = 8, RM_BATCH = 16, RM_MAXBUFS = 6, RM_MAXJ = 8; // RM_MAXJ float4 per lane: rows up to 8192 wide
constexpr int RM_ROWS_OFF = 64 + 2 * RM_BATCH * RM_WARPS * 4;           // after the barriers and the partials
constexpr size_t kRmsRowSmem = 204800;                                  // row buffers: 2 x 5 rows of 5120 floats

__global__ void __launch_bounds__(RM_WARPS * 32, 1) rms_mod_kernel(const RmsModParams p, int nb, int nbufs, int rows_per_cta)
{
    extern __shared__ __align__(128) uint8_t rm_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(rm_smem); // [nbufs]
    float* part = reinterpret_cast<float*>(rm_smem + 64);
    float* pmax = part + RM_BATCH * RM_WARPS;
    float* rows = reinterpret_cast<float*>(rm_smem + RM_ROWS_OFF);
    const int w = warp_id(), lane = lane_id();
    const int n4 = p.d >> 2, nw4 = (n4 + RM_WARPS - 1) / RM_WARPS;
    const int r0 = blockIdx.x * rows_per_cta, r1 = min(p.rows, r0 + rows_per_cta);
    if (r0 >= r1)
        return;
    const int batches = (r1 - r0 + nb - 1) / nb;
    const uint32_t row_bytes = uint32_t(p.d) * 4;
    auto issue = [&](int b) { // one thread: the bulk copies of batch b into buffer b % nbufs
        const int first = r0 + b * nb, n = min(nb, r1 - first);
        float* dst = rows + size_t(b % nbufs) * nb * p.d;
        mbar_arrive_expect_tx(&full[b % nbufs], uint32_t(n) * row_bytes);
        for (int i = 0; i < n; ++i)
            bulk_load(dst + size_t(i) * p.d, p.x + size_t(first + i) * p.ldx, row_bytes, &full[b % nbufs]);
    };
    if (threadIdx.x == 0) {
        for (int k = 0; k < nbufs; ++k)
            mbar_init(&full[k], 1);
        fence_barrier_init();
        for (int k = 0; k < nbufs && k < batches; ++k)
            issue(k);
    }
    __syncthreads();
    // this lane's columns: float4 index col(j) = w nw4 + lane + 32 j, where lane + 32 j < nw4 and col(j) < n4
    auto col = [&](int j) { return w * nw4 + lane + 32 * j; };
    auto valid = [&](int j) { return lane + 32 * j < nw4 && col(j) < n4; };
    float4 wa[RM_MAXJ], sh[RM_MAXJ];
    int m_cur = -1;
    auto load_mod = [&](int m) {
        const float4* sh4 = reinterpret_cast<const float4*>(p.mod + (size_t(m) * p.mod_slots + p.shift_slot) * p.d);
        const float4* sc4 = reinterpret_cast<const float4*>(p.mod + (size_t(m) * p.mod_slots + p.scale_slot) * p.d);
        const float4* w4 = reinterpret_cast<const float4*>(p.w);
#pragma unroll
        for (int j = 0; j < RM_MAXJ; ++j) {
            if (!valid(j))
                continue;
            const float4 sc = __ldg(sc4 + col(j));
            const float4 wt = p.w ? __ldg(w4 + col(j)) : make_float4(1.f, 1.f, 1.f, 1.f);
            wa[j] = make_float4(wt.x * (1.f + sc.x), wt.y * (1.f + sc.y), wt.z * (1.f + sc.z), wt.w * (1.f + sc.w));
            sh[j] = __ldg(sh4 + col(j));
        }
        m_cur = m;
    };
    auto r16 = [](float a) { return __bfloat162float(__float2bfloat16_rn(a)); };
    bool ok = true;
    int b = 0;
    for (; b < batches; ++b) {
        const int first = r0 + b * nb, n = min(nb, r1 - first);
        const float* buf = rows + size_t(b % nbufs) * nb * p.d;
        if (!(ok = mbar_wait(&full[b % nbufs], (b / nbufs) & 1)))
            break;
        for (int i = 0; i < n; ++i) {
            const float4* x4 = reinterpret_cast<const float4*>(buf + size_t(i) * p.d);
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < RM_MAXJ; ++j)
                if (valid(j)) {
                    const float4 v = x4[col(j)];
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
            ss = warp_sum(ss);
            if (lane == 0)
                part[i * RM_WARPS + w] = ss;
        }
        __syncthreads();
        float amax_local[RM_BATCH];
        for (int i = 0; i < n; ++i) {
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < RM_WARPS; ++k)
                ss += part[i * RM_WARPS + k];
            const float rinv = rsqrtf(ss / float(p.d) + p.eps);
            const int r = first + i;
            const int m = p.mod_idx ? p.mod_idx[r] : 0;
            if (m != m_cur)
                load_mod(m);
            const float4* x4 = reinterpret_cast<const float4*>(buf + size_t(i) * p.d);
            float am = 0.f;
#pragma unroll
            for (int j = 0; j < RM_MAXJ; ++j) {
                if (!valid(j))
                    continue;
                const float4 v = x4[col(j)];
                const float4 y = make_float4(v.x * rinv * wa[j].x + sh[j].x, v.y * rinv * wa[j].y + sh[j].y,
                                             v.z * rinv * wa[j].z + sh[j].z, v.w * rinv * wa[j].w + sh[j].w);
                if (p.out_kind == RowOut::bf16) {
                    reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(r) * p.ldo)[col(j)] =
                        make_uint2(pack_bf16x2(y.x, y.y), pack_bf16x2(y.z, y.w));
                } else if (p.out_kind == RowOut::f32) {
                    reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + size_t(r) * p.ldo)[col(j)] = y;
                } else {
                    am = fmaxf(am, fmaxf(fmaxf(fabsf(r16(y.x)), fabsf(r16(y.y))), fmaxf(fabsf(r16(y.z)), fabsf(r16(y.w)))));
                }
            }
            amax_local[i] = am;
        }
        if (p.out_kind == RowOut::s8) {
            // the GEMM input is the bf16 rounding of y (as in the bf16 path), quantised per row by its maximum
            for (int i = 0; i < n; ++i) {
                const float am = warp_max(amax_local[i]);
                if (lane == 0)
                    pmax[i * RM_WARPS + w] = am;
            }
            __syncthreads();
            for (int i = 0; i < n; ++i) {
                float amax = 0.f, ss = 0.f;
#pragma unroll
                for (int k = 0; k < RM_WARPS; ++k)
                    amax = fmaxf(amax, pmax[i * RM_WARPS + k]), ss += part[i * RM_WARPS + k];
                const float rinv = rsqrtf(ss / float(p.d) + p.eps);
                const int r = first + i;
                const int m = p.mod_idx ? p.mod_idx[r] : 0;
                if (m != m_cur)
                    load_mod(m);
                const float inv = amax > 0.f ? 127.0f / amax : 0.f;
                if (threadIdx.x == 0)
                    p.out_scale[r] = amax / 127.0f;
                auto q = [&](float y) { return static_cast<signed char>(fminf(fmaxf(rintf(r16(y) * inv), -127.f), 127.f)); };
                const float4* x4 = reinterpret_cast<const float4*>(buf + size_t(i) * p.d);
                char4* o = reinterpret_cast<char4*>(reinterpret_cast<int8_t*>(p.out) + size_t(r) * p.ldo);
#pragma unroll
                for (int j = 0; j < RM_MAXJ; ++j) {
                    if (!valid(j))
                        continue;
                    const float4 v = x4[col(j)];
                    o[col(j)] = make_char4(q(v.x * rinv * wa[j].x + sh[j].x), q(v.y * rinv * wa[j].y + sh[j].y),
                                           q(v.z * rinv * wa[j].z + sh[j].z), q(v.w * rinv * wa[j].w + sh[j].w));
                }
            }
        }
        // every read of the buffer is done: refill it with batch b + nbufs
        fence_proxy_async_smem();
        __syncthreads();
        if (threadIdx.x == 0 && b + nbufs < batches)
            issue(b + nbufs);
    }
    if (!ok && threadIdx.x == 0) {
        // a wait ran out: let the copies still in flight land before the CTA's shared memory is released
        for (int k = b; k < min(b + nbufs, batches); ++k)
            mbar_wait(&full[k % nbufs], (k / nbufs) & 1, 100000000ll);
    }
}

__global__ void gate_add_kernel(float* x, int64_t ldx, const __nv_bfloat16* y, int64_t ldy, int rows, int d, const float* mod,
                                const uint8_t* mod_idx, int gate_slot)
{
    const int n8 = d / 8;
    const size_t total = size_t(rows) * n8;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int r = int(i / n8), c = int(i % n8) * 8;
        const uint4 yv = *reinterpret_cast<const uint4*>(y + size_t(r) * ldy + c);
        const float* g = mod + (size_t(mod_idx[r]) * 6 + gate_slot) * d + c;
        float4* xp = reinterpret_cast<float4*>(x + size_t(r) * ldx + c);
        const __nv_bfloat162* yb = reinterpret_cast<const __nv_bfloat162*>(&yv);
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(g)), g1 = __ldg(reinterpret_cast<const float4*>(g) + 1);
        float4 x0 = xp[0], x1 = xp[1];
        const float2 y0 = __bfloat1622float2(yb[0]), y1 = __bfloat1622float2(yb[1]), y2 = __bfloat1622float2(yb[2]),
                     y3 = __bfloat1622float2(yb[3]);
        x0.x += g0.x * y0.x, x0.y += g0.y * y0.y, x0.z += g0.z * y1.x, x0.w += g0.w * y1.y;
        x1.x += g1.x * y2.x, x1.y += g1.y * y2.y, x1.z += g1.z * y3.x, x1.w += g1.w * y3.y;
        xp[0] = x0, xp[1] = x1;
    }
}

__global__ void swiglu_kernel(const __nv_bfloat16* gv, int rows, int F, __nv_bfloat16* out)
{
    const int n8 = F / 8;
    const size_t total = size_t(rows) * n8;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int r = int(i / n8), c = int(i % n8) * 8;
        const uint4 g = *reinterpret_cast<const uint4*>(gv + size_t(r) * 2 * F + c);
        const uint4 u = *reinterpret_cast<const uint4*>(gv + size_t(r) * 2 * F + F + c);
        const __nv_bfloat162* gb = reinterpret_cast<const __nv_bfloat162*>(&g);
        const __nv_bfloat162* ub = reinterpret_cast<const __nv_bfloat162*>(&u);
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 a = __bfloat1622float2(gb[k]), b = __bfloat1622float2(ub[k]);
            o[k] = pack_bf16x2(a.x / (1.f + __expf(-a.x)) * b.x, a.y / (1.f + __expf(-a.y)) * b.y);
        }
        *reinterpret_cast<uint4*>(out + size_t(r) * F + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// One CTA (256 threads) per row; two passes over the row (the second from L1/L2). The row may be split into column
// chunks of Kc elements stored one after another (element k at x + (k / Kc) * chunk_stride + r * ldx + k % Kc), the
// layout the out projection's input has after the sequence-parallel exchange.
__global__ void __launch_bounds__(256) quant_rows_kernel(const __nv_bfloat16* x, int64_t ldx, int K, int Kc, int64_t chunk_stride,
                                                         int8_t* q, float* scale)
{
    __shared__ float red[8];
    const int r = blockIdx.x;
    auto at = [&](int c) { return x + (c / Kc) * chunk_stride + size_t(r) * ldx + (c % Kc); };
    float amax = 0.f;
    for (int c = threadIdx.x * 8; c < K; c += 256 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(at(c));
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(b[k]);
            amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
    amax = block_max<256>(amax, red);
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
    if (threadIdx.x == 0)
        scale[r] = amax / 127.0f;
    for (int c = threadIdx.x * 8; c < K; c += 256 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(at(c));
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
        signed char o[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(b[k]);
            o[2 * k] = static_cast<signed char>(fminf(fmaxf(rintf(f.x * inv), -127.f), 127.f));
            o[2 * k + 1] = static_cast<signed char>(fminf(fmaxf(rintf(f.y * inv), -127.f), 127.f));
        }
        *reinterpret_cast<uint2*>(q + size_t(r) * K + c) = *reinterpret_cast<uint2*>(o);
    }
}

// One warp per (row, head, q-or-k): 128 values, 4 per lane.
__global__ void heads_partial_kernel(__nv_bfloat16* qkv, int rows, int heads, const float* qn_w, const float* kn_w,
                                     const float* rope, float eps)
{
    const size_t wid = (blockIdx.x * size_t(blockDim.x) + threadIdx.x) / 32;
    const int lane = lane_id();
    if (wid >= size_t(rows) * heads * 2)
        return;
    const int sec = int(wid % 2);
    const int h = int((wid / 2) % heads);
    const int r = int(wid / (2 * size_t(heads)));
    __nv_bfloat16* p = qkv + (size_t(r) * 3 + sec) * heads * 128 + h * 128;
    // lane l holds dims l, l + 32, l + 64, l + 96: dims d and d + 48 pair up across lanes, so stage through shuffles.
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        v[k] = __bfloat162float(p[lane + 32 * k]);
    float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
    const float rinv = rsqrtf(ss * (1.f / 128.f) + eps);
    const float* w = sec == 0 ? qn_w : kn_w;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        v[k] = v[k] * rinv * w[lane + 32 * k];
    __shared__ float buf[8][128];
    float* b = buf[(threadIdx.x / 32) & 7];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        b[lane + 32 * k] = v[k];
    __syncwarp();
    const float2* cs = reinterpret_cast<const float2*>(rope) + size_t(r) * 48;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int dd = lane + 32 * k;
        float o = b[dd];
        if (dd < 48) {
            const float2 t = cs[dd];
            o = b[dd] * t.x - b[dd + 48] * t.y;
        } else if (dd < 96) {
            const float2 t = cs[dd - 48];
            o = b[dd] * t.x + b[dd - 48] * t.y;
        }
        p[dd] = __float2bfloat16_rn(o);
    }
}

__global__ void pack_bf16_kernel(const float* in, int rows, int cols, __nv_bfloat16* out, int ld_out, const int32_t* src_rows)
{
    const size_t total = size_t(rows) * ld_out;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int r = int(i / ld_out), c = int(i % ld_out);
        const size_t sr = src_rows ? size_t(src_rows[r]) : size_t(r);
        out[i] = __float2bfloat16_rn(c < cols ? in[sr * cols + c] : 0.f);
    }
}

__global__ void euler_kernel(float* x, const float* v, size_t n, float st, float ratio, float keep)
{
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        const float xi = x[i];
        const float x0 = __fadd_rn(xi, __fmul_rn(st, v[i]));
        x[i] = __fadd_rn(__fmul_rn(ratio, xi), __fmul_rn(keep, x0));
    }
}

// 64 x 64 outputs per CTA, 4 x 4 per thread; B and A staged through shared memory 32 of the rank at a time.
__global__ void __launch_bounds__(256) lora_merge_kernel(const float* B, const float* A, int out, int in, int r, float s,
                                                         const int32_t* row_map, __nv_bfloat16* W, int64_t ldw, const int8_t* q,
                                                         const float* qscale)
{
    __shared__ float Bs[32][64 + 1]; // [k][i]
    __shared__ float As[32][64 + 4]; // [k][j]
    const int i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
    const int ti = threadIdx.x / 16, tj = threadIdx.x % 16;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < r; k0 += 32) {
        for (int e = threadIdx.x; e < 32 * 64; e += 256) {
            const int k = e / 64, x = e % 64;
            Bs[k][x] = (i0 + x < out && k0 + k < r) ? B[size_t(i0 + x) * r + k0 + k] : 0.f;
            As[k][x] = (j0 + x < in && k0 + k < r) ? A[size_t(k0 + k) * in + j0 + x] : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; ++k)
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    acc[a][b] = fmaf(Bs[k][ti * 4 + a], As[k][tj * 4 + b], acc[a][b]);
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int i = i0 + ti * 4 + a;
        if (i >= out)
            continue;
        const size_t wr = size_t(row_map[i]);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int j = j0 + tj * 4 + b;
            if (j >= in)
                continue;
            const float base = q ? float(q[wr * ldw + j]) * qscale[wr] : __bfloat162float(W[wr * ldw + j]);
            W[wr * ldw + j] = __float2bfloat16_rn(base + s * acc[a][b]);
        }
    }
}

__global__ void gather_rows_kernel(const float* src, int64_t lds, const int32_t* idx, int rows, int cols, float* dst, int64_t ldd)
{
    const size_t total = size_t(rows) * cols;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int r = int(i / cols), c = int(i % cols);
        dst[size_t(r) * ldd + c] = src[size_t(idx[r]) * lds + c];
    }
}

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__global__ void fill_kernel(void* dst, int is_bf16, uint64_t n, uint64_t key, float mean, float k)
{
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t h = splitmix64(key + i);
        const int32_t s = int32_t(h & 0xFFFF) + int32_t((h >> 16) & 0xFFFF) + int32_t((h >> 32) & 0xFFFF) + int32_t(h >> 48) - 131070;
        const float v = __fadd_rn(mean, __fmul_rn(k, float(s)));
        if (is_bf16)
            reinterpret_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
        else
            reinterpret_cast<float*>(dst)[i] = v;
    }
}

__global__ void __launch_bounds__(256) quant_weight_kernel(const __nv_bfloat16* w, int K, int8_t* q, float* scale)
{
    __shared__ float red[8];
    const int r = blockIdx.x;
    const __nv_bfloat16* wr = w + size_t(r) * K;
    float amax = 0.f;
    for (int c = threadIdx.x; c < K; c += 256)
        amax = fmaxf(amax, fabsf(__bfloat162float(wr[c])));
    amax = block_max<256>(amax, red);
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
    if (threadIdx.x == 0)
        scale[r] = amax / 127.0f;
    for (int c = threadIdx.x; c < K; c += 256)
        q[size_t(r) * K + c] = static_cast<signed char>(fminf(fmaxf(rintf(__bfloat162float(wr[c]) * inv), -127.f), 127.f));
}

__global__ void interleave_kernel(const __nv_bfloat16* w, int F, int K, __nv_bfloat16* out)
{
    // output row o: group g = o / 256, j = o % 256; j < 128: gate row g*128 + j, else value row F + g*128 + j - 128
    const int o = blockIdx.x;
    const int g = o / 256, j = o % 256;
    const int src = j < 128 ? g * 128 + j : F + g * 128 + (j - 128);
    const uint4* s = reinterpret_cast<const uint4*>(w + size_t(src) * K);
    uint4* d = reinterpret_cast<uint4*>(out + size_t(o) * K);
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x)
        d[c] = s[c];
}

__global__ void interleave_f32_kernel(const float* b, int F, float* out)
{
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= 2 * F)
        return;
    const int g = o / 256, j = o % 256;
    out[o] = b[j < 128 ? g * 128 + j : F + g * 128 + (j - 128)];
}

int grid_for(size_t work, int threads)
{
    const size_t g = (work + threads - 1) / threads;
    return int(std::min<size_t>(g, size_t(num_sms()) * 16));
}

} // namespace

void rms_mod_rows(const RmsModParams& p, cudaStream_t s)
{
    const size_t row_bytes = size_t(p.d) * 4;
    if (p.d <= 0 || p.d % 4 || p.d > RM_WARPS * 32 * RM_MAXJ * 4 || !p.x || !p.mod || !p.out ||
        (p.out_kind == RowOut::s8 && !p.out_scale))
        throw CudaError("rms_mod_rows: bad arguments");
    // 16-byte aligned rows for the bulk copies and the vector loads and stores
    if (reinterpret_cast<uintptr_t>(p.x) % 16 || p.ldx % 4 || reinterpret_cast<uintptr_t>(p.out) % 16 || p.ldo % 4 ||
        (p.w && reinterpret_cast<uintptr_t>(p.w) % 16) || reinterpret_cast<uintptr_t>(p.mod) % 16)
        throw CudaError("rms_mod_rows: rows and vectors must start on 16-byte boundaries");
    if (p.rows == 0)
        return;
    // batches of up to RM_BATCH rows, as many buffers as fit (at least two)
    const int nb = int(std::max<size_t>(1, std::min<size_t>(RM_BATCH, kRmsRowSmem / (2 * row_bytes))));
    const int nbufs = int(std::min<size_t>(RM_MAXBUFS, kRmsRowSmem / (nb * row_bytes)));
    const int per = std::max(1, (p.rows + num_sms() - 1) / num_sms());
    const int grid = (p.rows + per - 1) / per;
    const int smem = RM_ROWS_OFF + int(nbufs * nb * row_bytes);
    static std::atomic<uint64_t> opt_in;
    smem_opt_in(rms_mod_kernel, RM_ROWS_OFF + int(kRmsRowSmem), opt_in);
    rms_mod_kernel<<<grid, RM_WARPS * 32, smem, s>>>(p, nb, nbufs, per);
    H3_CUDA(cudaGetLastError());
}

void gate_add_rows(float* x, int64_t ldx, const void* y, int64_t ldy, int rows, int d, const float* mod, const uint8_t* mod_idx,
                   int gate_slot, cudaStream_t s)
{
    if (d % 8)
        throw CudaError("gate_add_rows: d must be a multiple of 8");
    if (!rows)
        return;
    gate_add_kernel<<<grid_for(size_t(rows) * d / 8, 256), 256, 0, s>>>(x, ldx, static_cast<const __nv_bfloat16*>(y), ldy, rows, d,
                                                                          mod, mod_idx, gate_slot);
    H3_CUDA(cudaGetLastError());
}

void swiglu_rows(const void* gv, int rows, int F, void* out, cudaStream_t s)
{
    if (F % 8)
        throw CudaError("swiglu_rows: F must be a multiple of 8");
    if (!rows)
        return;
    swiglu_kernel<<<grid_for(size_t(rows) * F / 8, 256), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gv), rows, F,
                                                                        static_cast<__nv_bfloat16*>(out));
    H3_CUDA(cudaGetLastError());
}

void quant_rows_i8(const void* x, int64_t ldx, int rows, int K, int8_t* q, float* scale, cudaStream_t s)
{
    if (K % 8)
        throw CudaError("quant_rows_i8: K must be a multiple of 8");
    if (!rows)
        return;
    quant_rows_kernel<<<rows, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, K, K, 0, q, scale);
    H3_CUDA(cudaGetLastError());
}

void quant_rows_i8_chunked(const void* x, int rows, int K, int chunks, int rows_stride, int8_t* q, float* scale, cudaStream_t s)
{
    const int Kc = K / chunks;
    if (K % chunks || Kc % 8 || rows_stride < rows)
        throw CudaError("quant_rows_i8_chunked: chunk widths must be multiples of 8");
    if (!rows)
        return;
    quant_rows_kernel<<<rows, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), Kc, K, Kc, int64_t(rows_stride) * Kc, q, scale);
    H3_CUDA(cudaGetLastError());
}

void heads_partial(void* qkv, int rows, int heads, const float* qn_w, const float* kn_w, const float* rope, float eps, cudaStream_t s)
{
    if (!rows)
        return;
    const size_t warps = size_t(rows) * heads * 2;
    heads_partial_kernel<<<unsigned((warps * 32 + 255) / 256), 256, 0, s>>>(static_cast<__nv_bfloat16*>(qkv), rows, heads, qn_w, kn_w,
                                                                             rope, eps);
    H3_CUDA(cudaGetLastError());
}

void pack_bf16_rows(const float* in, int rows, int cols, void* out, int ld_out, cudaStream_t s, const int32_t* src_rows)
{
    if (!rows)
        return;
    pack_bf16_kernel<<<grid_for(size_t(rows) * ld_out, 256), 256, 0, s>>>(in, rows, cols, static_cast<__nv_bfloat16*>(out), ld_out,
                                                                           src_rows);
    H3_CUDA(cudaGetLastError());
}

void euler_rows(float* x, const float* v, size_t n, float t, float sigma, float sigma_next, cudaStream_t s)
{
    if (!n)
        return;
    const float st = 1.0f - t, ratio = sigma_next / sigma, keep = 1.0f - ratio;
    euler_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, v, n, st, ratio, keep);
    H3_CUDA(cudaGetLastError());
}

void lora_merge(const float* B, const float* A, int out, int in, int r, float s, const int32_t* row_map, void* W, int64_t ldw,
                const int8_t* q, const float* qscale, cudaStream_t st)
{
    if (out <= 0 || in <= 0 || r <= 0)
        return;
    const dim3 grid((in + 63) / 64, (out + 63) / 64);
    lora_merge_kernel<<<grid, 256, 0, st>>>(B, A, out, in, r, s, row_map, static_cast<__nv_bfloat16*>(W), ldw, q, qscale);
    H3_CUDA(cudaGetLastError());
}

void gather_rows_f32(const float* src, int64_t lds, const int32_t* idx, int rows, int cols, float* dst, int64_t ldd, cudaStream_t s)
{
    if (!rows)
        return;
    gather_rows_kernel<<<grid_for(size_t(rows) * cols, 256), 256, 0, s>>>(src, lds, idx, rows, cols, dst, ldd);
    H3_CUDA(cudaGetLastError());
}

void fill_synthetic(void* dst, int is_bf16, uint64_t n, uint64_t seed, uint32_t tensor_id, float mean, float stdev, cudaStream_t s)
{
    if (!n)
        return;
    const double norm = 1.0 / std::sqrt((65536.0 * 65536.0 - 1.0) / 3.0);
    const float k = float(double(stdev) * norm);
    const uint64_t key = splitmix64(seed * 0x632BE59BD9B4E019ull + tensor_id);
    fill_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, is_bf16, n, key, mean, k);
    H3_CUDA(cudaGetLastError());
}

void quant_weight_rows(const void* w, int rows, int K, int8_t* q, float* scale, cudaStream_t s)
{
    if (!rows)
        return;
    quant_weight_kernel<<<rows, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), K, q, scale);
    H3_CUDA(cudaGetLastError());
}

void interleave_gate_value(const void* w, int F, int K, void* out, cudaStream_t s)
{
    if (F % 128 || K % 8)
        throw CudaError("interleave_gate_value: F must be a multiple of 128 and K of 8");
    interleave_kernel<<<2 * F, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(w), F, K, static_cast<__nv_bfloat16*>(out));
    H3_CUDA(cudaGetLastError());
}

void interleave_gate_value_f32(const float* b, int F, float* out, cudaStream_t s)
{
    interleave_f32_kernel<<<(2 * F + 255) / 256, 256, 0, s>>>(b, F, out);
    H3_CUDA(cudaGetLastError());
}

} // namespace h3
