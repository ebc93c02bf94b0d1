// The C ABI of the video VAE decoder (h3vae_*, include/h3_c.h) and the kernel-level entry points its parity tests
// call (h3k_attention_segments, h3k_vae_heads, h3k_layer_norm).
#include "h3_c.h"

#include "attention.cuh"
#include "common.hpp"
#include "vae.hpp"

#include <cmath>
#include <cstring>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>

struct h3vae_model {
    std::unique_ptr<h3::VideoDecoder> m;
    int device = 0;
};

namespace h3 {
int run_guarded(const std::function<void()>& f); // capi.cpp: the status codes and message of every entry point
} // namespace h3

namespace {

h3::VaeConfig to_vae_config(const h3vae_config* c)
{
    if (!c)
        throw std::invalid_argument("h3vae: null config");
    h3::VaeConfig v;
    v.dim = int(c->dim), v.heads = int(c->heads), v.ffn = int(c->ffn), v.blocks = int(c->blocks), v.channels = int(c->channels);
    v.registers = int(c->registers), v.clip = int(c->clip), v.tile = int(c->tile), v.overlap = int(c->overlap);
    v.eps = c->eps > 0.f ? c->eps : 1e-6f;
    return v;
}

h3::VideoDecoder& model_of(h3vae_model* m)
{
    if (!m || !m->m)
        throw std::invalid_argument("h3vae: null model");
    H3_CUDA(cudaSetDevice(m->device));
    return *m->m;
}

void device_only(const char* what, std::initializer_list<const void*> ptrs)
{
    for (const void* p : ptrs)
        if (!h3::device_accessible(p))
            throw std::invalid_argument(std::string(what) + ": a pointer argument is host memory the GPU cannot access");
}

} // namespace

extern "C" {

int h3vae_create(const h3vae_config* cfg, const char* weights, int32_t device, h3vae_model** out)
{
    return h3::run_guarded([&] {
        if (!out || !weights)
            throw std::invalid_argument("h3vae_create: null argument");
        *out = nullptr;
        const h3::VaeConfig c = to_vae_config(cfg);
        const std::string src(weights);
        if (src.rfind("synthetic:", 0) != 0)
            throw std::invalid_argument("h3vae_create: weights \"synthetic:SEED\" (the decoder's checkpoint names are not in the "
                                        "reference tree)");
        const uint64_t seed = std::stoull(src.substr(10));
        auto m = std::make_unique<h3vae_model>();
        m->device = device;
        m->m = std::make_unique<h3::VideoDecoder>(c, seed, device);
        *out = m.release();
    });
}

int h3vae_decode_clip(h3vae_model* m, const float* latents, uint32_t h, uint32_t w, float* canvas)
{
    return h3::run_guarded([&] { model_of(m).decode_clip(latents, int(h), int(w), canvas, false); });
}

int h3vae_decode_clip_device(h3vae_model* m, const float* latents, uint32_t h, uint32_t w, float* canvas)
{
    return h3::run_guarded([&] {
        h3::VideoDecoder& d = model_of(m);
        device_only("h3vae_decode_clip_device", {latents, canvas});
        d.decode_clip(latents, int(h), int(w), canvas, true);
    });
}

int h3vae_decode(h3vae_model* m, const float* latents, uint32_t frames, uint32_t h, uint32_t w, h3vae_frame_fn sink, void* user)
{
    return h3::run_guarded([&] {
        h3::VideoDecoder& d = model_of(m);
        if (!sink)
            throw std::invalid_argument("h3vae_decode: null sink");
        const uint64_t count = uint64_t(h) * 16 * w * 16 * 3;
        d.decode(latents, int(frames), int(h), int(w), [&](int index, const float* rgb) { sink(user, uint32_t(index), rgb, count); });
    });
}

int h3vae_tile_starts(uint32_t n, uint32_t tile, uint32_t overlap, uint32_t* starts, uint32_t cap, uint32_t* count)
{
    return h3::run_guarded([&] {
        const std::vector<int> s = h3::vae_tile_starts(int(n), int(tile), int(overlap));
        if (count)
            *count = uint32_t(s.size());
        for (size_t i = 0; i < s.size() && starts && i < cap; ++i)
            starts[i] = uint32_t(s[i]);
    });
}

int h3vae_rope_table(uint32_t frames, uint32_t th, uint32_t tw, uint32_t specials, float* out)
{
    return h3::run_guarded([&] {
        if (!out)
            throw std::invalid_argument("h3vae_rope_table: null output");
        const std::vector<float> t = h3::vae_rope_table(int(frames), int(th), int(tw), int(specials));
        std::memcpy(out, t.data(), t.size() * 4);
    });
}

int32_t h3vae_last_launches(h3vae_model* m) { return m && m->m ? m->m->last_launches() : 0; }

void* h3vae_stream(h3vae_model* m) { return m && m->m ? static_cast<void*>(m->m->stream()) : nullptr; }

void h3vae_destroy(h3vae_model* m)
{
    if (!m)
        return;
    if (m->m)
        cudaSetDevice(m->device);
    delete m;
}

int h3k_attention_segments(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, int32_t head_dim, int32_t rows,
                           int32_t seg_rows, int32_t seg_stride, void* out, int64_t out_row_stride, void* stream)
{
    return h3::run_guarded([&] {
        if (!q || !k || !v || !out)
            throw std::invalid_argument("h3k_attention_segments: null argument");
        device_only("h3k_attention_segments", {q, k, v, out});
        h3::AttnParams p;
        p.q = q, p.k = k, p.v = v, p.row_stride = row_stride, p.heads = heads, p.rows = rows, p.head_dim = head_dim;
        p.seg_rows = seg_rows, p.seg_stride = seg_stride, p.out = out, p.out_row_stride = out_row_stride;
        p.scale = 1.0f / std::sqrt(float(head_dim));
        h3::attention(p, static_cast<cudaStream_t>(stream));
    });
}

int h3k_vae_heads(void* qkv, int32_t rows, int32_t heads, int32_t T, const float* rope, float eps, void* stream)
{
    return h3::run_guarded([&] {
        device_only("h3k_vae_heads", {qkv, rope});
        h3::vae_heads(qkv, rows, heads, T, rope, eps, static_cast<cudaStream_t>(stream));
    });
}

int h3k_layer_norm(const float* x, int32_t rows, int32_t d, const float* w, const float* b, float eps, void* out, void* stream)
{
    return h3::run_guarded([&] {
        device_only("h3k_layer_norm", {x, w, b, out});
        h3::layer_norm_rows(x, rows, d, w, b, eps, out, static_cast<cudaStream_t>(stream));
    });
}

} // extern "C"
