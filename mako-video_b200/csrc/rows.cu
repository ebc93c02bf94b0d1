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

constexpr size_t kRmsStreamSmem = 172032; // row slots of the streaming kernel: 4 warps x 2 rows of 5376 floats

// y = RMSNorm(x) * w * (1 + scale[r]) + shift[r] per row, bf16, fp32 or int8 (+ row scale) out. A persistent kernel
// that streams rows through shared memory: each warp owns two row slots
// and keeps the next row's bulk copy in flight while it works on the current one (eight rows of HBM reads in flight
// per SM with four warps), reads the row twice from shared memory (sum of squares, then the output) and the shift,
// scale and weight vectors through L1 (consecutive rows share them). Rows r = (CTA x warps + warp) + i x grid x warps.
// Shared memory: [warps][2] mbarriers (256 bytes), then [warps][2][d] fp32 row slots.
__global__ void __launch_bounds__(256) rms_mod_stream_kernel(const RmsModParams p)
{
    extern __shared__ __align__(128) uint8_t rm_smem[];
    const int nw = blockDim.x >> 5, w = warp_id(), lane = lane_id();
    const uint32_t row_bytes = uint32_t(p.d) * 4;
    uint64_t* bar = reinterpret_cast<uint64_t*>(rm_smem) + 2 * w;
    float* buf = reinterpret_cast<float*>(rm_smem + 256) + size_t(2 * w) * p.d;
    const int stride = gridDim.x * nw;
    const int first = blockIdx.x * nw + w;
    if (lane == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
        for (int k = 0; k < 2; ++k) {
            const int r = first + k * stride;
            if (r < p.rows) {
                mbar_arrive_expect_tx(&bar[k], row_bytes);
                bulk_load(buf + size_t(k) * p.d, p.x + size_t(r) * p.ldx, row_bytes, &bar[k]);
            }
        }
    }
    __syncwarp();
    const int n4 = p.d >> 2;
    int it = 0;
    bool ok = true;
    for (int r = first; r < p.rows; r += stride, ++it) {
        const int slot = it & 1;
        float4* x4 = reinterpret_cast<float4*>(buf + size_t(slot) * p.d);
        if (!(ok = mbar_wait(&bar[slot], (it >> 1) & 1)))
            break;
        float ss0 = 0.f, ss1 = 0.f;
        int c = lane;
        for (; c + 32 < n4; c += 64) {
            const float4 a = x4[c], b = x4[c + 32];
            ss0 += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
            ss1 += b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
        }
        if (c < n4) {
            const float4 a = x4[c];
            ss0 += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
        }
        const float rinv = rsqrtf(warp_sum(ss0 + ss1) / float(p.d) + p.eps);
        const int m = p.mod_idx ? p.mod_idx[r] : 0;
        const float4* sh4 = reinterpret_cast<const float4*>(p.mod + (size_t(m) * p.mod_slots + p.shift_slot) * p.d);
        const float4* sc4 = reinterpret_cast<const float4*>(p.mod + (size_t(m) * p.mod_slots + p.scale_slot) * p.d);
        const float4* w4 = reinterpret_cast<const float4*>(p.w);
        auto y_of = [&](int c) {
            const float4 v = x4[c], sh = __ldg(sh4 + c), sc = __ldg(sc4 + c);
            const float4 wt = p.w ? __ldg(w4 + c) : make_float4(1.f, 1.f, 1.f, 1.f);
            return make_float4(v.x * rinv * wt.x * (1.f + sc.x) + sh.x, v.y * rinv * wt.y * (1.f + sc.y) + sh.y,
                               v.z * rinv * wt.z * (1.f + sc.z) + sh.z, v.w * rinv * wt.w * (1.f + sc.w) + sh.w);
        };
        if (p.out_kind == RowOut::bf16) {
            uint2* o = reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(r) * p.ldo);
#pragma unroll 4
            for (int c = lane; c < n4; c += 32) {
                const float4 y = y_of(c);
                o[c] = make_uint2(pack_bf16x2(y.x, y.y), pack_bf16x2(y.z, y.w));
            }
        } else if (p.out_kind == RowOut::f32) {
            float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + size_t(r) * p.ldo);
#pragma unroll 4
            for (int c = lane; c < n4; c += 32)
                o[c] = y_of(c);
        } else {
            // the GEMM input is the bf16 rounding of y (as in the bf16 path), quantised per row: y's bf16 values go
            // back into the slot, then a third pass quantises them by the row's maximum
            auto r16 = [](float a) { return __bfloat162float(__float2bfloat16_rn(a)); };
            float amax = 0.f;
#pragma unroll 4
            for (int c = lane; c < n4; c += 32) {
                float4 y = y_of(c);
                y = make_float4(r16(y.x), r16(y.y), r16(y.z), r16(y.w));
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w))));
                x4[c] = y;
            }
            amax = warp_max(amax);
            const float inv = amax > 0.f ? 127.0f / amax : 0.f;
            if (lane == 0)
                p.out_scale[r] = amax / 127.0f;
            __syncwarp();
            auto q = [&](float b) { return static_cast<signed char>(fminf(fmaxf(rintf(b * inv), -127.f), 127.f)); };
            char4* o = reinterpret_cast<char4*>(reinterpret_cast<int8_t*>(p.out) + size_t(r) * p.ldo);
            for (int c = lane; c < n4; c += 32) {
                const float4 y = x4[c];
                o[c] = make_char4(q(y.x), q(y.y), q(y.z), q(y.w));
            }
        }
        // the slot's reads (and the int8 pass's writes) come before the next bulk copy into it
        fence_proxy_async_smem();
        __syncwarp();
        const int next = r + 2 * stride;
        if (lane == 0 && next < p.rows) {
            mbar_arrive_expect_tx(&bar[slot], row_bytes);
            bulk_load(buf + size_t(slot) * p.d, p.x + size_t(next) * p.ldx, row_bytes, &bar[slot]);
        }
    }
    if (!ok && lane == 0) {
        // a wait ran out: let this warp's copies still in flight land before the CTA's shared memory is released
        for (int k = 1; k < 3; ++k) {
            const int r = first + (it + k - 1) * stride;
            if (r < p.rows)
                mbar_wait(&bar[(it + k - 1) & 1], ((it + k - 1) >> 1) & 1, 100000000ll);
        }
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
    const size_t slot_bytes = size_t(p.d) * 4;
    const int nw = int(std::min<size_t>(4, kRmsStreamSmem / (2 * std::max<size_t>(slot_bytes, 16))));
    if (p.d <= 0 || p.d % 4 || nw < 1 || !p.x || !p.mod || !p.out || (p.out_kind == RowOut::s8 && !p.out_scale))
        throw CudaError("rms_mod_rows: bad arguments");
    // 16-byte aligned rows for the bulk copies and the vector loads and stores
    if (reinterpret_cast<uintptr_t>(p.x) % 16 || p.ldx % 4 || reinterpret_cast<uintptr_t>(p.out) % 16 || p.ldo % 4 ||
        (p.w && reinterpret_cast<uintptr_t>(p.w) % 16) || reinterpret_cast<uintptr_t>(p.mod) % 16)
        throw CudaError("rms_mod_rows: rows and vectors must start on 16-byte boundaries");
    if (p.rows == 0)
        return;
    const int smem = 256 + int(nw * 2 * slot_bytes);
    static std::atomic<uint64_t> opt_in;
    smem_opt_in(rms_mod_stream_kernel, 256 + int(kRmsStreamSmem), opt_in);
    const int grid = int(std::min<int64_t>(num_sms(), (int64_t(p.rows) + nw - 1) / nw));
    rms_mod_stream_kernel<<<grid, nw * 32, smem, s>>>(p);
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
