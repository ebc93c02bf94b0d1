// Drop-in for mako-common's models/h3.hpp: the class mako::models::H3 that jhanssen/mako-video's sampler uses
// (src/video/engine.hpp:22 `using H3 = models::H3;`), with the member signatures its call sites need
// (src/video/engine.cpp:105-117, 666-676, 700, 714; tests/h3_ref_test.cpp:194, 215-224, 484-502), implemented over
// the C ABI of libh3b200.so (include/h3_c.h). Header-only; link with -lh3b200. Failures throw std::runtime_error, as
// the reference does.
#pragma once

#include "../h3_c.h"

#include <cstdint>
#include <functional>
#include <optional>
#include <span>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

namespace mako::models {

class H3 {
public:
    // Widths of the rows the step reads and writes (H3::kText, kVideoPatch, kAudioChannels).
    static constexpr uint32_t kText = 5120, kVideoPatch = 96, kAudioChannels = 32;
    static constexpr uint8_t kVideoTag = 0, kTextTag = 1, kAudioTag = 2;
    // MiniMax-H3's shape (docs/architecture.md:23-27, 47-67).
    static constexpr uint32_t kDim = 5376, kTimeDim = 2688;

    enum Int8 : uint32_t { qkv = 1, out = 2, fc1 = 4, fc2 = 8 };

    struct Layout {
        // A reference block (ref2va): a picture (frames 1), a video (frames, h, w and its soundtrack's audio latents)
        // or a soundtrack (audio latents) (src/video/engine.cpp:604-616; tests/h3_ref_test.cpp:475-479).
        struct Reference {
            enum class Kind : int32_t { image = H3_REF_IMAGE, video = H3_REF_VIDEO, audio = H3_REF_AUDIO };
            Kind kind = Kind::image;
            uint32_t frames = 0, h = 0, w = 0, audio = 0;
        };
        uint32_t text = 0, frames = 0, h = 0, w = 0, audio = 0, cond_frames = 0;
        std::vector<uint8_t> cond_last; // per keyframe: anchored at the last generated frame
        std::vector<Reference> refs;    // reference blocks in reading order
        std::vector<uint8_t> text_tags; // per text row: 1 text, 0 video (a vision block's rows)
        uint32_t patch_rows() const { return (h / 2) * (w / 2); }
        uint32_t cond_rows() const
        {
            uint32_t n = cond_frames * patch_rows();
            for (const Reference& r : refs)
                if (r.kind != Reference::Kind::audio)
                    n += (r.kind == Reference::Kind::image ? 1 : r.frames) * (r.h / 2) * (r.w / 2);
            return n;
        }
        uint32_t cond_audio_rows() const
        {
            uint32_t n = 0;
            for (const Reference& r : refs)
                if (r.kind != Reference::Kind::image)
                    n += 2 * r.audio;
            return n;
        }
        uint32_t video_rows() const { return cond_rows() + frames * patch_rows(); }
        uint32_t audio_rows() const { return cond_audio_rows() + 2 * audio; }
        uint32_t rows() const { return text + video_rows() + audio_rows(); }
        // The C view; `refs_c` holds the reference blocks it points at.
        h3_layout c(std::vector<h3_layout_ref>& refs_c) const
        {
            refs_c.clear();
            for (const Reference& r : refs)
                refs_c.push_back(h3_layout_ref{int32_t(r.kind), r.frames, r.h, r.w, r.audio});
            return h3_layout{text, frames, h, w, audio, cond_frames, cond_last.empty() ? nullptr : cond_last.data(),
                             text_tags.empty() ? nullptr : text_tags.data(), refs_c.empty() ? nullptr : refs_c.data(),
                             uint32_t(refs_c.size())};
        }
    };

    struct Rows {
        std::vector<double> pos; // [S][3]: t, h, w
        std::vector<uint8_t> tags, roles;
    };

    struct Velocities {
        std::vector<float> video, audio;
    };

    using ProbeFn = std::function<void(const std::string& name, int layer, const float* data, size_t n)>;

    // H3(path, ctx, telemetry, int8) (src/video/engine.cpp:109-110). `path` is a checkpoint (a safetensors file or a
    // directory of them, see h3_create) or "synthetic:SEED" (random-init weights). The context and telemetry
    // arguments of mako-common's runtime are accepted and unused: the GPU is the current CUDA device.
    template <class Context, class Telemetry>
    H3(const std::string& path, Context&, Telemetry, uint32_t int8, h3_config cfg = h3_mini_h3(), const h3_world* world = nullptr,
       int device = 0)
    {
        check(h3_create(&cfg, path.c_str(), int8, 0.0f, 1, world, device, &m_));
    }
    explicit H3(const std::string& path, uint32_t int8 = 0, h3_config cfg = h3_mini_h3(), const h3_world* world = nullptr, int device = 0)
    {
        check(h3_create(&cfg, path.c_str(), int8, 0.0f, 1, world, device, &m_));
    }
    ~H3() { h3_destroy(m_); }
    H3(const H3&) = delete;
    H3& operator=(const H3&) = delete;

    // MiniMax-H3's shape.
    static h3_config h3_mini_h3() { return h3_config{kDim, 56, 14336, 50, kTimeDim, kText, kVideoPatch, kAudioChannels, 1e-6f, 2, 0}; }

    // Writes the weights to a safetensors file a later H3(path, ...) reads back (h3_save_weights; bf16 models).
    void save_weights(const std::string& path) { check(h3_save_weights(m_, path.c_str())); }

    // set_sparse(ratio, local) (src/video/engine.cpp:112).
    void set_sparse(float ratio, uint32_t local) { check(h3_set_sparse(m_, ratio, local)); }
    // add_lora(path, scale, strict) (src/video/engine.cpp:114): merges a Diffusers-named LoRA file into the weights.
    void add_lora(const std::string& path, float scale, bool strict) { check(h3_add_lora(m_, path.c_str(), scale, strict ? 1 : 0, nullptr, nullptr)); }

    // begin(text [T][5120], layout) (src/video/engine.cpp:700).
    void begin(std::span<const float> text, const Layout& l)
    {
        std::vector<h3_layout_ref> refs;
        const h3_layout c = l.c(refs);
        check(h3_begin(m_, text.data(), uint32_t(text.size() / kText), &c));
        layout_ = l;
    }

    // step(video [V][96], audio [A][32], t_video, t_audio) (src/video/engine.cpp:714).
    Velocities step(std::span<const float> video, std::span<const float> audio, float t_video, float t_audio)
    {
        Velocities v;
        v.video.resize(video.size());
        v.audio.resize(audio.size());
        check(h3_step(m_, video.data(), video.size() / kVideoPatch, audio.data(), audio.size() / kAudioChannels, t_video, t_audio,
                      v.video.data(), v.audio.data()));
        return v;
    }

    // Engine::denoise's step loop on the GPU (src/video/engine.cpp:701-719): the sample (conditioning rows, then
    // noise) in, the final sample out; sigmas from Engine::sigmas for video and audio. No counterpart member in the
    // reference's H3, whose caller runs this loop on the host around step(). `progress(step, steps)` returning
    // false stops the loop after that step. Returns the steps run.
    uint32_t denoise(std::span<float> video, std::span<float> audio, std::span<const float> sigma_video, std::span<const float> sigma_audio,
                     std::function<bool(uint32_t, uint32_t)> progress = {})
    {
        if (sigma_video.size() != sigma_audio.size())
            throw std::runtime_error("H3::denoise: the video and audio schedules differ in length");
        struct Ctx {
            std::function<bool(uint32_t, uint32_t)>* fn;
        } ctx{&progress};
        auto thunk = [](void* user, uint32_t i, uint32_t n) -> int { return (*static_cast<Ctx*>(user)->fn)(i, n) ? 0 : 1; };
        uint32_t ran = 0;
        check(h3_denoise(m_, video.data(), video.size() / kVideoPatch, audio.data(), audio.size() / kAudioChannels, sigma_video.data(),
                         sigma_audio.data(), uint32_t(sigma_video.size()), progress ? +thunk : nullptr, &ctx, &ran));
        return ran;
    }

    // Engine::sigmas(steps, shift) (src/video/engine.cpp:71-88).
    static std::vector<float> sigmas(uint32_t steps, float shift)
    {
        std::vector<float> out(steps < 2 ? 2 : steps);
        uint32_t n = 0;
        check(h3_sigmas(steps, shift, out.data(), &n));
        out.resize(n);
        return out;
    }

    // set_probe (tests/h3_ref_test.cpp:215-217): txt (from begin: the text after the token refiner), temb (not for a
    // pruned checkpoint), mod0, x0, block (layer), norm_out.
    void set_probe(ProbeFn fn)
    {
        probe_ = std::move(fn);
        check(h3_set_probe(m_, probe_ ? &H3::probe_thunk : nullptr, this));
    }

    // H3::rows(layout) (tests/h3_ref_test.cpp:484-502).
    static Rows rows(const Layout& l)
    {
        std::vector<h3_layout_ref> refs;
        const h3_layout c = l.c(refs);
        const uint64_t S = h3_layout_rows(&c);
        Rows r;
        r.pos.resize(S * 3);
        r.tags.resize(S);
        r.roles.resize(S);
        check(h3_rows(&c, r.pos.data(), r.tags.data(), r.roles.data()));
        return r;
    }

    // Checkpoints (no counterpart in the reference; host only). check_weights: "" when the checkpoint at `path` fits
    // the shape, else its first problem. convert_weights: the checkpoint at `src` rewritten at `dst` in this library's
    // layout through `renames` lines ("this_name source_name", "qkv_layout interleaved"); see h3_convert_weights.
    static std::string check_weights(const std::string& path, h3_config cfg = h3_mini_h3())
    {
        char msg[4096] = {};
        return h3_check_weights(&cfg, path.c_str(), msg, sizeof msg) == H3_OK ? std::string() : std::string(msg);
    }
    static void convert_weights(const std::string& src, const std::string& dst, const std::string& renames = {},
                                h3_config cfg = h3_mini_h3())
    {
        check(h3_convert_weights(&cfg, src.c_str(), dst.c_str(), renames.c_str()));
    }

    // parse_int8 (tools/mako_video.cpp:108-114).
    static std::optional<uint32_t> parse_int8(std::string_view s)
    {
        uint32_t m = 0;
        if (h3_parse_int8(std::string(s).c_str(), &m) != H3_OK)
            return std::nullopt;
        return m;
    }

private:
    h3_model* m_ = nullptr;
    Layout layout_;
    ProbeFn probe_;

    static void check(int rc)
    {
        if (rc != H3_OK)
            throw std::runtime_error(h3_last_error());
    }
    static void probe_thunk(void* user, const char* name, int32_t layer, const float* data, uint64_t n)
    {
        static_cast<H3*>(user)->probe_(name, layer, data, n);
    }
};

} // namespace mako::models
