// Drop-in for jhanssen/mako-video's src/video/video_vae.hpp: the class mako::video::VideoVae that the engine uses to
// turn the transformer's latents into frames (src/video/engine.cpp:157-162, 196-199), with the members its call sites
// need, implemented over the C ABI of libh3b200.so (include/h3_c.h, h3vae_*). Header-only; link with -lh3b200.
// Failures throw std::runtime_error, as the reference does. The decoder's weights: "synthetic:SEED" (random-init);
// the reference's video_vae directory is refused with a message (its tensor names are in the absent mako-common).
#pragma once

#include "../h3_c.h"

#include <cstdint>
#include <functional>
#include <span>
#include <stdexcept>
#include <string>

namespace mako::video {

class VideoVae {
public:
    // src/video/video_vae.hpp:20, and the latent / patch sizes of models::H3Vae
    static constexpr uint32_t kPatchT = 4, kClipLatents = 5, kClipOverlap = 2, kPrePad = 3, kFrameOverlap = 5;
    static constexpr uint32_t kLatent = 24, kPatch = 16;
    // A decoded frame: its index and its pixels [16 h][16 w][3] in [0, 1] (video_vae.hpp:21-22).
    using FrameSink = std::function<void(uint32_t index, std::span<const float> rgb)>;

    // VideoVae(dir, ctx, telemetry) (video_vae.hpp:19); `cfg` selects the shape (MiniMax-H3's by default).
    template <class Context, class Telemetry>
    VideoVae(const std::string& dir, Context&, Telemetry, h3vae_config cfg = h3_minimax_vae(), int32_t device = 0)
    {
        if (dir.rfind("synthetic:", 0) != 0)
            throw std::runtime_error(dir + ": the video VAE decoder loads synthetic weights only (\"synthetic:SEED\")");
        if (h3vae_create(&cfg, dir.c_str(), device, &m_) != H3_OK)
            throw std::runtime_error(h3_last_error());
    }
    template <class Context>
    VideoVae(const std::string& dir, Context& ctx) : VideoVae(dir, ctx, 0)
    {
    }
    ~VideoVae() { h3vae_destroy(m_); }
    VideoVae(const VideoVae&) = delete;
    VideoVae& operator=(const VideoVae&) = delete;

    // The transformer's normalized latents as voxels [frames][h][w][24] (frames = 5 n + 2) to the video's 17 n + 5
    // frames, delivered in order (video_vae.hpp:23-25).
    void decode(std::span<const float> latents, uint32_t frames, uint32_t h, uint32_t w, const FrameSink& sink)
    {
        if (latents.size() != uint64_t(frames) * h * w * kLatent)
            throw std::runtime_error("video VAE: voxels [5 n + 2][h][w][24]");
        struct Ctx {
            const FrameSink* sink;
        } c{&sink};
        auto fn = [](void* user, uint32_t index, const float* rgb, uint64_t count) {
            (*static_cast<Ctx*>(user)->sink)(index, std::span<const float>(rgb, count));
        };
        if (h3vae_decode(m_, latents.data(), frames, h, w, fn, &c) != H3_OK)
            throw std::runtime_error(h3_last_error());
    }
    static uint32_t pixel_frames(uint32_t latent_frames) { return (latent_frames - 2) / kClipLatents * 17 + 5; }

    static h3vae_config h3_minimax_vae() { return h3vae_config{2048, 32, 8192, 36, 24, 4, 7, 16, 4, 1e-6f}; }

private:
    h3vae_model* m_ = nullptr;
};

} // namespace mako::video
