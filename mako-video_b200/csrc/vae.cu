// Kernels of the video VAE decoder; see vae.cuh. All HBM-bound row and pixel work (the decoder's blocks run on the
// step's tcgen05 GEMM and attention kernels).
#include "common.hpp"
#include "ptx.cuh"
#include "vae.cuh"

#include <cuda_bf16.h>

#include <algorithm>

namespace h3 {

namespace {

constexpr int kPatch = 16, kPatchT = 4;
constexpr int kMaxC = 32; // latent channels at most

int blocks_for(size_t n, int threads) { return int(std::min<size_t>((n + threads - 1) / threads, size_t(1) << 30)); }

// One thread per voxel token.
__global__ void vae_inputs_kernel(const float* in, int C, VaeTiles t, const float* mean, const float* stdv, const float* wpq,
                                  const float* bpq, __nv_bfloat16* out, int kin)
{
    const size_t per_tile = size_t(t.frames) * t.th * t.tw;
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= per_tile * t.tiles())
        return;
    const int tile = int(i / per_tile);
    const int v = int(i - size_t(tile) * per_tile);
    const int f = v / (t.th * t.tw), y = (v / t.tw) % t.th, x = v % t.tw;
    const int gy = t.y0[tile / t.tiles_x] + y, gx = t.x0[tile % t.tiles_x] + x;
    const float* src = in + ((size_t(f) * t.h + gy) * t.w + gx) * C;
    float z[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c)
        z[c] = c < C ? src[c] * stdv[c] + mean[c] : 0.f;
    __nv_bfloat16* dst = out + (size_t(tile) * t.T + t.R + v) * kin;
    for (int o = 0; o < kin; ++o) {
        float acc = 0.f;
        if (o < C) {
            acc = bpq[o];
#pragma unroll
            for (int c = 0; c < kMaxC; ++c)
                if (c < C)
                    acc = fmaf(wpq[o * C + c], z[c], acc);
        }
        dst[o] = __float2bfloat16_rn(acc);
    }
}

__global__ void vae_special_rows_kernel(float* x, int d, VaeTiles t, const float* registers)
{
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; // (tile, special row, column)
    const size_t n = size_t(t.tiles()) * t.R * d;
    if (i >= n)
        return;
    const int c = int(i % d);
    const int r = int((i / d) % t.R);
    const int tile = int(i / (size_t(d) * t.R));
    x[(size_t(tile) * t.T + r) * d + c] = r < t.R - 1 ? registers[size_t(r) * d + c] : 0.f;
}

// One thread per (row, head, q or k): the 64 values in registers.
__global__ void vae_heads_kernel(__nv_bfloat16* qkv, int rows, int heads, int T, const float* rope, float eps)
{
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(rows) * heads * 2)
        return;
    const int part = int(i & 1);
    const int head = int((i >> 1) % heads);
    const size_t row = (i >> 1) / heads;
    uint4* p = reinterpret_cast<uint4*>(qkv + (row * 3 + part) * size_t(heads) * 64 + size_t(head) * 64);
    float v[64];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint4 u = p[k];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[e]);
            v[8 * k + 2 * e] = __bfloat162float(b.x);
            v[8 * k + 2 * e + 1] = __bfloat162float(b.y);
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int d = 0; d < 64; ++d)
        ss = fmaf(v[d], v[d], ss);
    const float r = rsqrtf(ss / 64.f + eps);
#pragma unroll
    for (int d = 0; d < 64; ++d)
        v[d] *= r;
    const float* cs = rope + size_t(row % T) * 48;
#pragma unroll
    for (int j = 0; j < 24; ++j) {
        const float c = cs[2 * j], sn = cs[2 * j + 1];
        const float a = v[j], b = v[j + 24];
        v[j] = a * c - b * sn;
        v[j + 24] = b * c + a * sn;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k)
        p[k] = make_uint4(pack_bf16x2(v[8 * k], v[8 * k + 1]), pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                          pack_bf16x2(v[8 * k + 4], v[8 * k + 5]), pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
}

// One warp per row, the row in registers (d <= 4096).
constexpr int LN_MAXV = 32; // float4 per lane

__global__ void __launch_bounds__(256) layer_norm_kernel(const float* x, int rows, int d, const float* w, const float* b, float eps,
                                                         __nv_bfloat16* out)
{
    const int row = blockIdx.x * 8 + warp_id();
    if (row >= rows)
        return;
    const int n4 = d / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x + size_t(row) * d);
    float4 v[LN_MAXV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
        const int c = lane_id() + 32 * i;
        if (c < n4) {
            v[i] = x4[c];
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
        s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / float(d);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
        const int c = lane_id() + 32 * i;
        if (c < n4) {
            const float a = v[i].x - mean, bb = v[i].y - mean, cc = v[i].z - mean, dd = v[i].w - mean;
            q += (a * a + bb * bb) + (cc * cc + dd * dd);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
        q += __shfl_xor_sync(0xffffffffu, q, o);
    const float r = rsqrtf(q / float(d) + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    uint2* o2 = reinterpret_cast<uint2*>(out + size_t(row) * d);
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
        const int c = lane_id() + 32 * i;
        if (c < n4) {
            const float4 ww = __ldg(w4 + c), bb = __ldg(b4 + c);
            o2[c] = make_uint2(pack_bf16x2((v[i].x - mean) * r * ww.x + bb.x, (v[i].y - mean) * r * ww.y + bb.y),
                               pack_bf16x2((v[i].z - mean) * r * ww.z + bb.z, (v[i].w - mean) * r * ww.w + bb.w));
        }
    }
}

// The tiles covering latent coordinate g on one axis, in order. Tiles placed as vae_tile_starts places them cover a
// coordinate at most three times (on axes a little longer than a tile the overlaps exceed half a tile); kMaxCover
// leaves room.
constexpr int kMaxCover = 4;
__device__ __forceinline__ int covering(const int* o, int n, int size, int g, int (&idx)[kMaxCover])
{
    int k = 0;
    for (int i = 0; i < n && k < kMaxCover; ++i)
        if (g >= o[i] && g < o[i] + size)
            idx[k++] = i;
    return k;
}

// One thread per canvas pixel (frame, row, column), its three channels.
__global__ void vae_pixels_kernel(const float* pix, VaeTiles t, float* canvas)
{
    const int H = t.h * kPatch, W = t.w * kPatch, F = t.frames * kPatchT;
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(F) * H * W)
        return;
    const int X = int(i % W), Y = int((i / W) % H), fr = int(i / (size_t(W) * H));
    const int f = fr / kPatchT, ft = fr % kPatchT;
    int iy[kMaxCover], ix[kMaxCover];
    const int ny = covering(t.y0, t.tiles_y, t.th, Y / kPatch, iy);
    const int nx = covering(t.x0, t.tiles_x, t.tw, X / kPatch, ix);
    float acc[3] = {0.f, 0.f, 0.f};
    bool first = true;
    for (int a = 0; a < ny; ++a)
        for (int b = 0; b < nx; ++b) {
            const int ty = iy[a], tx = ix[b];
            const int ly = Y - t.y0[ty] * kPatch, lx = X - t.x0[tx] * kPatch; // pixel inside the tile
            const int vy = ly / kPatch, py = ly % kPatch, vx = lx / kPatch, px = lx % kPatch;
            const size_t row = size_t(ty * t.tiles_x + tx) * t.T + t.R + (size_t(f) * t.th + vy) * t.tw + vx;
            const float* src = pix + row * (3 * kPatchT * kPatch * kPatch);
            // fade-in over the overlap with the tile above / to the left (in pixels)
            const int oy = ty > 0 ? (t.y0[ty - 1] + t.th - t.y0[ty]) * kPatch : 0;
            const int ox = tx > 0 ? (t.x0[tx - 1] + t.tw - t.x0[tx]) * kPatch : 0;
            const float wy = ly < oy ? float(ly) / float(oy) : 1.f;
            const float wx = lx < ox ? float(lx) / float(ox) : 1.f;
            const float wt = wy * wx;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const float val = src[((c * kPatchT + ft) * kPatch + py) * kPatch + px];
                acc[c] = first ? val : acc[c] * (1.f - wt) + val * wt;
            }
            first = false;
        }
    float* dst = canvas + i * 3;
    dst[0] = acc[0], dst[1] = acc[1], dst[2] = acc[2];
}

__global__ void vae_emit_kernel(const float* canvas, int pre, int n, const float* prev, int fade, int H, int W, float* out)
{
    const size_t frame = size_t(H) * W * 3;
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= frame * n)
        return;
    const int k = int(i / frame);
    const size_t e = i - size_t(k) * frame;
    float v = canvas[size_t(pre + k) * frame + e];
    if (prev && k < fade) {
        const float wb = float(k) / float(fade), wa = 1.0f - wb;
        v = prev[size_t(k) * frame + e] * wa + v * wb;
    }
    // ImageNet statistics of the RGB channels
    const int c = int(e % 3);
    const float mean = c == 0 ? 0.485f : (c == 1 ? 0.456f : 0.406f);
    const float sd = c == 0 ? 0.229f : (c == 1 ? 0.224f : 0.225f);
    out[i] = fminf(fmaxf(v * sd + mean, 0.0f), 1.0f);
}

} // namespace

void vae_inputs(const float* in, int C, const VaeTiles& t, const float* mean, const float* stdv, const float* wpq, const float* bpq,
                void* out, int kin, cudaStream_t s)
{
    if (C <= 0 || C > kMaxC || kin < C)
        throw CudaError("vae_inputs: latent channels");
    const size_t n = size_t(t.frames) * t.th * t.tw * t.tiles();
    if (!n)
        return;
    vae_inputs_kernel<<<blocks_for(n, 128), 128, 0, s>>>(in, C, t, mean, stdv, wpq, bpq, static_cast<__nv_bfloat16*>(out), kin);
    H3_CUDA(cudaGetLastError());
}

void vae_special_rows(float* x, int d, const VaeTiles& t, const float* registers, cudaStream_t s)
{
    const size_t n = size_t(t.tiles()) * t.R * d;
    if (!n)
        return;
    vae_special_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, d, t, registers);
    H3_CUDA(cudaGetLastError());
}

void vae_heads(void* qkv, int rows, int heads, int T, const float* rope, float eps, cudaStream_t s)
{
    const size_t n = size_t(rows) * heads * 2;
    if (!n)
        return;
    vae_heads_kernel<<<blocks_for(n, 128), 128, 0, s>>>(static_cast<__nv_bfloat16*>(qkv), rows, heads, T, rope, eps);
    H3_CUDA(cudaGetLastError());
}

void layer_norm_rows(const float* x, int rows, int d, const float* w, const float* b, float eps, void* out, cudaStream_t s)
{
    if (d % 4 || d > 32 * 4 * LN_MAXV)
        throw CudaError("layer_norm_rows: width");
    if (!rows)
        return;
    layer_norm_kernel<<<(rows + 7) / 8, 256, 0, s>>>(x, rows, d, w, b, eps, static_cast<__nv_bfloat16*>(out));
    H3_CUDA(cudaGetLastError());
}

void vae_pixels(const float* pix, const VaeTiles& t, float* canvas, cudaStream_t s)
{
    const size_t n = size_t(t.frames) * kPatchT * t.h * kPatch * t.w * kPatch;
    if (!n)
        return;
    vae_pixels_kernel<<<blocks_for(n, 256), 256, 0, s>>>(pix, t, canvas);
    H3_CUDA(cudaGetLastError());
}

void vae_emit(const float* canvas, int pre, int n, const float* prev, int fade, int H, int W, float* out, cudaStream_t s)
{
    const size_t m = size_t(H) * W * 3 * n;
    if (!m)
        return;
    vae_emit_kernel<<<blocks_for(m, 256), 256, 0, s>>>(canvas, pre, n, prev, fade, H, W, out);
    H3_CUDA(cudaGetLastError());
}

} // namespace h3
