// Kernels of the video VAE decoder (MiniMax-H3's ViT decoder, docs/architecture.md:80-92 of the reference): the
// per-tile token inputs, the q/k norms and rotary of its 64-dim heads, its final layer norm, the pixels of a clip
// assembled from overlapping tiles, and the frames a clip emits (cross-fade with the previous clip, ImageNet
// de-normalisation, clamp). The transformer blocks themselves run on the step's GEMM, RMS-norm and attention kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#ifdef __CUDACC__
#define H3_VAE_HD __host__ __device__
#else
#define H3_VAE_HD
#endif

namespace h3 {

// Spatial tiling of a clip: tiles_y x tiles_x tiles of th x tw latents, tile (ty, tx) at latent (y0[ty], x0[tx]);
// every tile has T = frames x th x tw + R tokens (R = registers + the zero token), rows [tile T, tile T + T) of the
// batch, the voxel tokens after the R special ones in (frame, row, column) order.
struct VaeTiles {
    int frames = 0, h = 0, w = 0;   // the clip's latent grid
    int th = 0, tw = 0;             // latents a tile covers on each axis
    int tiles_y = 0, tiles_x = 0;
    int R = 0, T = 0;               // special tokens a tile, tokens a tile
    const int* y0 = nullptr;        // [tiles_y] (device)
    const int* x0 = nullptr;        // [tiles_x] (device)
    H3_VAE_HD int tiles() const { return tiles_y * tiles_x; }
};

// in: normalized latents [frames][h][w][C] (fp32). For every voxel token: z = in * std + mean per channel, then the
// 1x1 post-quant convolution z' = Wpq z + bpq (C x C), written as bf16 [rows][kin] (channels >= C left zero; special
// rows untouched).
void vae_inputs(const float* in, int C, const VaeTiles& t, const float* mean, const float* stdv, const float* wpq, const float* bpq,
                void* out_bf16, int kin, cudaStream_t s);

// x [tiles T][d] fp32: each tile's rows 0 .. R-2 get the register vectors [R-1][d], row R-1 zeros.
void vae_special_rows(float* x, int d, const VaeTiles& t, const float* registers, cudaStream_t s);

// qkv [rows][3][heads][64] bf16 in place: q and k RMS-normed per head (no weight), then rotated: dims j and j + 24
// by angle j (j < 24) of the row's token (rope [T][24][2] cos, sin; token = row mod T); dims 48..63 pass.
void vae_heads(void* qkv, int rows, int heads, int T, const float* rope, float eps, cudaStream_t s);

// y = (x - mean) / sqrt(var + eps) * w + b per row, bf16 out.
void layer_norm_rows(const float* x, int rows, int d, const float* w, const float* b, float eps, void* out_bf16, cudaStream_t s);

// The clip's canvas [frames * 4][16 h][16 w][3] (ImageNet-normalized RGB) from the projection output
// pix [tiles T][3 * 4 * 16 * 16] (per voxel token: channel, frame, pixel row, pixel column): every pixel takes the
// tiles covering it in raster order, each tile fading in linearly over its overlap with the tile above and the tile
// to the left (weight 0 at the overlap's first pixel).
void vae_pixels(const float* pix, const VaeTiles& t, float* canvas, cudaStream_t s);

// The frames a clip emits (video_vae.cpp:34-44 of the reference): canvas frames [pre, pre + n) to out[n][H][W][3] in
// [0, 1]; the first `fade` of them fade in from prev[fade][H][W][3] (weight (f - pre) / fade) when prev is given.
void vae_emit(const float* canvas, int pre, int n, const float* prev, int fade, int H, int W, float* out, cudaStream_t s);

} // namespace h3
