// The video VAE decoder of MiniMax-H3 (the reference's models::H3Vae as video::VideoVae drives it,
// src/video/video_vae.cpp:17-50 and docs/architecture.md:80-92), on the step's sm_100a kernels:
//   latents of a clip (7 latent frames, normalized) -> per-channel de-normalisation, the 1x1 post-quant convolution
//   -> 256-pixel tiles (16 x 16 latents) overlapping by at least 64 pixels, every tile's voxels one token each
//   (24 -> 2048, padded to 64 inputs for the GEMM) plus 4 register tokens and a zero token at the origin
//   -> 36 blocks: RMS norm with weight, q/k/v with biases, q/k RMS-normed per head without weights, 48 of 64 values
//      rotated by three axes of 8 frequencies of base 100 (coordinates on [-1, 1) times 2 pi), attention within the
//      tile, x += scale1 * out; RMS norm, SwiGLU 8192, x += scale2 * ffn
//   -> layer norm, the patch projection 2048 -> 3 x 4 x 16 x 16 -> each token's four 16 x 16 RGB frames, tiles faded
//      into each other over their overlaps -> the clip's 28 ImageNet-normalized frames.
// All the clip's tiles run as one batch of rows (attention segmented per tile). The video loop (decode) emits 17
// frames a clip, the first 5 cross-faded with the previous clip's last 5, de-normalized and clamped.
#pragma once
#include "devbuf.hpp"
#include "vae.cuh"

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

namespace h3 {

struct VaeConfig {
    int dim = 2048, heads = 32, ffn = 8192, blocks = 36;
    int channels = 24;  // latent channels
    int registers = 4;
    int clip = 7;       // latent frames a clip decodes
    int tile = 16;      // latents a tile spans (256 pixels)
    int overlap = 4;    // latents two tiles overlap at least (64 pixels)
    float eps = 1e-6f;
    static constexpr int kin = 64;       // token inputs, the channels padded for the GEMM's 64-wide K tile
    static constexpr int head_dim = 64;
    static constexpr int patch = 16, patch_t = 4;
    int pix() const { return 3 * patch_t * patch * patch; }
};

// Tile starts along an axis of n latents: one tile of n when n <= tile; else the fewest tiles of `tile` latents
// overlapping by at least `overlap`, the slack spread over the overlaps in whole latents (the first gaps one more).
std::vector<int> vae_tile_starts(int n, int tile, int overlap);

// The rotary table of one tile's tokens [T][24][2] (cos, sin): specials at the origin, voxel (f, y, x) of a
// frames x th x tw tile at coordinates -1 + 2 i / n on each axis, times 2 pi, times 100^(-k / 8) (k < 8).
std::vector<float> vae_rope_table(int frames, int th, int tw, int specials);

class VideoDecoder {
public:
    // Synthetic weights from `seed` (fill_synthetic, the oracle regenerates them) on `device`.
    VideoDecoder(const VaeConfig& c, uint64_t seed, int device);
    ~VideoDecoder();
    VideoDecoder(const VideoDecoder&) = delete;
    VideoDecoder& operator=(const VideoDecoder&) = delete;

    const VaeConfig& config() const { return c_; }
    cudaStream_t stream() const { return stream_; }

    // H3Vae's decode of one clip: latents [clip][h][w][channels] (normalized) -> canvas [4 clip][16 h][16 w][3]
    // (ImageNet-normalized). Host or device pointers (device_io).
    void decode_clip(const float* latents, int h, int w, float* canvas, bool device_io);
    // VideoVae::decode: latents [frames][h][w][channels], frames = 5 n + 2, to the 17 n + 5 frames in [0, 1], each
    // handed to `sink` (index, [16 h][16 w][3] host floats) in order.
    void decode(const float* latents, int frames, int h, int w, const std::function<void(int, const float*)>& sink);
    int last_launches() const { return launches_; }

private:
    struct Block {
        DevBuf norm1, qkv_w, qkv_b, out_w, out_b, norm2, fc1_w, fc1_b, fc2_w, fc2_b, mods; // mods [6][d]: scale1 at 2, scale2 at 5
    };
    VaeConfig c_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    int launches_ = 0;
    DevBuf mean_, std_, pq_w_, pq_b_, emb_w_, emb_b_, registers_, ln_w_, ln_b_, proj_w_, proj_b_, zero_mod_, ones_;
    std::vector<Block> blocks_;
    // activations, grown to the largest clip seen
    DevBuf lat_, inp_, x_, h_, qkv_, o_, ffn_, canvas_, rope_, starts_, midx_, overlap_, frames_out_;
    std::vector<float> host_frames_;
    int rope_key_[3] = {-1, -1, -1};
    void run_clip(const float* d_latents, int h, int w); // into canvas_
};

} // namespace h3
