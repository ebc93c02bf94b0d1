// Row kernels (HBM-bound): 128-bit loads and stores, one CTA (or warp) per row, warp-shuffle reductions.
#include "common.hpp"
#include "ptx.cuh"
#include "rows.cuh"

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

// Block-wide sum for a CTA of NT threads (NT a multiple of 32); every thread gets the total.
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red)
{
    v = warp_sum(v);
    if (lane_id() == 0)
        red[warp_id()] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i)
        t += red[i];
    __syncthreads();
    return t;
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

constexpr int RMS_NT = 128;
constexpr int RMS_VPT = 16; // float4 per thread: rows up to 128 * 16 * 4 = 8192 wide

// One CTA per row; the row is held in registers between the reduction and the output pass.
__global__ void __launch_bounds__(RMS_NT) rms_mod_kernel(const RmsModParams p)
{
    __shared__ float red[RMS_NT / 32];
    const int r = blockIdx.x;
    const int n4 = p.d / 4;
    const float4* x4 = reinterpret_cast<const float4*>(p.x + size_t(r) * p.ldx);
    float4 v[RMS_VPT];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < RMS_VPT; ++i) {
        const int c = threadIdx.x + i * RMS_NT;
        if (c < n4) {
            v[i] = x4[c];
            ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        }
    }
    ss = block_sum<RMS_NT>(ss, red);
    const float rinv = rsqrtf(ss / float(p.d) + p.eps);
    const int m = p.mod_idx ? p.mod_idx[r] : 0;
    const float4* sh4 = reinterpret_cast<const float4*>(p.mod + (size_t(m) * p.mod_slots + p.shift_slot) * p.d);
    const float4* sc4 = reinterpret_cast<const float4*>(p.mod + (size_t(m) * p.mod_slots + p.scale_slot) * p.d);
    const float4* w4 = reinterpret_cast<const float4*>(p.w);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < RMS_VPT; ++i) {
        const int c = threadIdx.x + i * RMS_NT;
        if (c < n4) {
            const float4 sh = __ldg(sh4 + c), sc = __ldg(sc4 + c);
            float4 w = make_float4(1.f, 1.f, 1.f, 1.f);
            if (p.w)
                w = __ldg(w4 + c);
            v[i].x = v[i].x * rinv * w.x * (1.f + sc.x) + sh.x;
            v[i].y = v[i].y * rinv * w.y * (1.f + sc.y) + sh.y;
            v[i].z = v[i].z * rinv * w.z * (1.f + sc.z) + sh.z;
            v[i].w = v[i].w * rinv * w.w * (1.f + sc.w) + sh.w;
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        }
    }
    if (p.out_kind == RowOut::bf16) {
        uint2* o = reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(r) * p.ldo);
#pragma unroll
        for (int i = 0; i < RMS_VPT; ++i) {
            const int c = threadIdx.x + i * RMS_NT;
            if (c < n4)
                o[c] = make_uint2(pack_bf16x2(v[i].x, v[i].y), pack_bf16x2(v[i].z, v[i].w));
        }
    } else if (p.out_kind == RowOut::f32) {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + size_t(r) * p.ldo);
#pragma unroll
        for (int i = 0; i < RMS_VPT; ++i) {
            const int c = threadIdx.x + i * RMS_NT;
            if (c < n4)
                o[c] = v[i];
        }
    } else {
        // The GEMM input is the bf16 rounding of y (as in the bf16 path), quantised per row.
        amax = block_max<RMS_NT>(amax, red);
        const float inv = amax > 0.f ? 127.0f / __bfloat162float(__float2bfloat16_rn(amax)) : 0.f;
        if (threadIdx.x == 0)
            p.out_scale[r] = __bfloat162float(__float2bfloat16_rn(amax)) / 127.0f;
        char4* o = reinterpret_cast<char4*>(reinterpret_cast<int8_t*>(p.out) + size_t(r) * p.ldo);
        auto q = [&](float a) {
            const float b = __bfloat162float(__float2bfloat16_rn(a));
            return static_cast<signed char>(fminf(fmaxf(rintf(b * inv), -127.f), 127.f));
        };
#pragma unroll
        for (int i = 0; i < RMS_VPT; ++i) {
            const int c = threadIdx.x + i * RMS_NT;
            if (c < n4)
                o[c] = make_char4(q(v[i].x), q(v[i].y), q(v[i].z), q(v[i].w));
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
    if (p.d % 4 || p.d > RMS_NT * RMS_VPT * 4 || !p.mod || !p.out || (p.out_kind == RowOut::s8 && !p.out_scale))
        throw CudaError("rms_mod_rows: bad arguments");
    if (p.rows == 0)
        return;
    rms_mod_kernel<<<p.rows, RMS_NT, 0, s>>>(p);
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
