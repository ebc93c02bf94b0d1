// Time-embedding MLP, AdaLN projections (full and pruned-curve) and the fp32 heads.
#include "common.hpp"
#include "embed.cuh"
#include "ptx.cuh"

#include <algorithm>

namespace h3 {

namespace {

__device__ __forceinline__ float silu(float v) { return v / (1.0f + __expf(-v)); }

constexpr int MAXU = 4;

// One warp per output row n; the U input vectors in shared memory.
__global__ void gemv_f32_kernel(const float* W, const float* b, const float* x, int U, int N, int K, int act, float* out,
                                float* out2)
{
    extern __shared__ float xs[];
    for (int i = threadIdx.x; i < U * K; i += blockDim.x)
        xs[i] = x[i];
    __syncthreads();
    const int warps = blockDim.x / 32;
    for (int n = blockIdx.x * warps + warp_id(); n < N; n += gridDim.x * warps) {
        float acc[MAXU] = {0.f, 0.f, 0.f, 0.f};
        const float* w = W + size_t(n) * K;
        for (int k = lane_id(); k < K; k += 32) {
            const float wv = __ldg(w + k);
#pragma unroll
            for (int u = 0; u < MAXU; ++u)
                if (u < U)
                    acc[u] += wv * xs[u * K + k];
        }
#pragma unroll
        for (int u = 0; u < MAXU; ++u) {
            float v = acc[u];
#pragma unroll
            for (int o = 16; o; o >>= 1)
                v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane_id() == 0 && u < U) {
                v += b ? b[n] : 0.f;
                if (act == int(Act::silu))
                    v = silu(v);
                out[size_t(u) * N + n] = v;
                if (out2)
                    out2[size_t(u) * N + n] = __bfloat162float(__float2bfloat16_rn(silu(v)));
            }
        }
    }
}

// Pruned checkpoints: one thread per projection row (K fp32 weights, a 32-byte row at K = 8, so a warp reads 1 KB of
// consecutive rows), all U curve points from shared memory; an fmaf chain over k from the bias.
constexpr int CM_MAXK = 16;

__global__ void __launch_bounds__(256) curve_mods_kernel(const float* W, const float* b, const float* c, int U, size_t rows, int G, int K,
                                                         float* out)
{
    __shared__ float cs[MAXU * CM_MAXK];
    for (int i = threadIdx.x; i < U * K; i += blockDim.x)
        cs[i] = c[i];
    __syncthreads();
    for (size_t r = size_t(blockIdx.x) * blockDim.x + threadIdx.x; r < rows; r += size_t(gridDim.x) * blockDim.x) {
        float w[CM_MAXK];
#pragma unroll
        for (int k = 0; k < CM_MAXK; ++k)
            w[k] = k < K ? __ldg(W + r * K + k) : 0.f;
        const float bias = __ldg(b + r);
        const size_t g = r / G, j = r - g * G;
#pragma unroll
        for (int u = 0; u < MAXU; ++u) {
            if (u >= U)
                break;
            float acc = bias;
#pragma unroll
            for (int k = 0; k < CM_MAXK; ++k)
                if (k < K)
                    acc = fmaf(w[k], cs[u * K + k], acc);
            out[(g * U + u) * G + j] = acc;
        }
    }
}

// One warp per weight row; each lane streams 16-byte chunks of the row (8 bf16) past L1, ADALN_UNROLL loads in
// flight before their products are summed (the kernel is HBM bound: it needs many bytes in flight per SM).
constexpr int ADALN_UNROLL = 4;

__device__ __forceinline__ uint4 ld_stream(const uint4* p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__global__ void __launch_bounds__(256) adaln_kernel(const __nv_bfloat16* W, const float* b, const float* x, int U, int groups, int G,
                                                    int K, float* out)
{
    extern __shared__ float xs[];
    for (int i = threadIdx.x; i < U * K; i += blockDim.x)
        xs[i] = x[i];
    __syncthreads();
    const size_t rows = size_t(groups) * G;
    const int k8 = K / 8;
    for (size_t r = size_t(blockIdx.x) * 8 + warp_id(); r < rows; r += size_t(gridDim.x) * 8) {
        const uint4* w = reinterpret_cast<const uint4*>(W + r * K);
        float acc[MAXU] = {0.f, 0.f, 0.f, 0.f};
        for (int c0 = lane_id(); c0 < k8; c0 += 32 * ADALN_UNROLL) {
            uint4 v[ADALN_UNROLL];
#pragma unroll
            for (int q = 0; q < ADALN_UNROLL; ++q)
                v[q] = c0 + 32 * q < k8 ? ld_stream(w + c0 + 32 * q) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int q = 0; q < ADALN_UNROLL; ++q) {
                const int c = c0 + 32 * q;
                if (c >= k8)
                    break;
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[q]);
                float f[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 t = __bfloat1622float2(h[i]);
                    f[2 * i] = t.x, f[2 * i + 1] = t.y;
                }
#pragma unroll
                for (int u = 0; u < MAXU; ++u)
                    if (u < U) {
                        const float4* xv = reinterpret_cast<const float4*>(xs + u * K + c * 8);
                        const float4 a = xv[0], bb = xv[1];
                        acc[u] += f[0] * a.x + f[1] * a.y + f[2] * a.z + f[3] * a.w + f[4] * bb.x + f[5] * bb.y + f[6] * bb.z + f[7] * bb.w;
                    }
            }
        }
        const size_t g = r / G, j = r % G;
#pragma unroll
        for (int u = 0; u < MAXU; ++u) {
            float v = acc[u];
#pragma unroll
            for (int o = 16; o; o >>= 1)
                v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane_id() == 0 && u < U)
                out[(g * U + u) * G + j] = v + b[r];
        }
    }
}

constexpr int HB_M = 64, HB_N = 32, HB_K = 32;

__global__ void __launch_bounds__(256) heads_kernel(const float* x, int64_t ldx, int rows, const float* W, const float* b, int N, int K,
                                                    float* out, int64_t ldo)
{
    __shared__ float As[HB_K][HB_M + 4];
    __shared__ float Bs[HB_K][HB_N + 4];
    const int m0 = blockIdx.x * HB_M, n0 = blockIdx.y * HB_N;
    const int tx = threadIdx.x % 8, ty = threadIdx.x / 8;
    float acc[2][4] = {};
    for (int k0 = 0; k0 < K; k0 += HB_K) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int e = threadIdx.x + i * 256; // 512 float4 = 64 rows x 8
            const int r = e / 8, c = (e % 8) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m0 + r < rows)
                v = *reinterpret_cast<const float4*>(x + size_t(m0 + r) * ldx + k0 + c);
            As[c][r] = v.x, As[c + 1][r] = v.y, As[c + 2][r] = v.z, As[c + 3][r] = v.w;
        }
        {
            const int r = threadIdx.x / 8, c = (threadIdx.x % 8) * 4; // 32 cols x 8 float4
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (n0 + r < N)
                v = *reinterpret_cast<const float4*>(W + size_t(n0 + r) * K + k0 + c);
            Bs[c][r] = v.x, Bs[c + 1][r] = v.y, Bs[c + 2][r] = v.z, Bs[c + 3][r] = v.w;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < HB_K; ++k) {
            const float a0 = As[k][ty * 2], a1 = As[k][ty * 2 + 1];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float bv = Bs[k][tx * 4 + j];
                acc[0][j] += a0 * bv;
                acc[1][j] += a1 * bv;
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int r = m0 + ty * 2 + i;
        if (r >= rows)
            continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < N)
                out[size_t(r) * ldo + n] = acc[i][j] + b[n];
        }
    }
}

} // namespace

void gemv_f32(const float* W, const float* b, const float* x, int U, int N, int K, Act act, float* out, float* out2, cudaStream_t s)
{
    if (U < 1 || U > MAXU)
        throw CudaError("gemv_f32: 1 to 4 vectors");
    const size_t smem = size_t(U) * K * sizeof(float);
    static std::atomic<uint64_t> opt_in;
    smem_opt_in(gemv_f32_kernel, 200 * 1024, opt_in);
    const int grid = std::min((N + 7) / 8, num_sms() * 4);
    gemv_f32_kernel<<<grid, 256, smem, s>>>(W, b, x, U, N, K, int(act), out, out2);
    H3_CUDA(cudaGetLastError());
}

void adaln_gemv(const void* W, const float* b, const float* x, int U, int groups, int G, int K, float* out, cudaStream_t s)
{
    if (U < 1 || U > MAXU || K % 8)
        throw CudaError("adaln_gemv: 1 to 4 vectors and K a multiple of 8");
    const size_t smem = size_t(U) * K * sizeof(float);
    static std::atomic<uint64_t> opt_in;
    smem_opt_in(adaln_kernel, 200 * 1024, opt_in);
    const size_t rows = size_t(groups) * G;
    const int grid = int(std::min<size_t>((rows + 7) / 8, size_t(num_sms()) * 8));
    adaln_kernel<<<grid, 256, smem, s>>>(static_cast<const __nv_bfloat16*>(W), b, x, U, groups, G, K, out);
    H3_CUDA(cudaGetLastError());
}

void curve_mods(const float* W, const float* b, const float* c, int U, int groups, int G, int K, float* out, cudaStream_t s)
{
    if (U < 1 || U > MAXU || K < 1 || K > CM_MAXK)
        throw CudaError("curve_mods: 1 to 4 curve points of at most 16 coordinates");
    const size_t rows = size_t(groups) * G;
    if (!rows)
        return;
    const int grid = int(std::min<size_t>((rows + 255) / 256, size_t(num_sms()) * 8));
    curve_mods_kernel<<<grid, 256, 0, s>>>(W, b, c, U, rows, G, K, out);
    H3_CUDA(cudaGetLastError());
}

void heads_f32(const float* x, int64_t ldx, int rows, const float* W, const float* b, int N, int K, float* out, int64_t ldo, cudaStream_t s)
{
    if (K % HB_K || N > 128)
        throw CudaError("heads_f32: K must be a multiple of 32");
    if (!rows)
        return;
    const dim3 grid((rows + HB_M - 1) / HB_M, (N + HB_N - 1) / HB_N);
    heads_kernel<<<grid, 256, 0, s>>>(x, ldx, rows, W, b, N, K, out, ldo);
    H3_CUDA(cudaGetLastError());
}

} // namespace h3
