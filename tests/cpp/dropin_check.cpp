// Compiles the drop-in header the way the reference's sampler would use it (mako::models::H3) and exercises its
// host-side members, which need no GPU: parse_int8, rows, and the refusal of a missing checkpoint.
#include "models/h3.hpp"
#include "video/video_vae.hpp"

#include <cstddef>
#include <cstdio>

namespace mako::mtl {
struct Context {};
} // namespace mako::mtl
namespace mako::gpu {
enum class Telemetry { off };
} // namespace mako::gpu

int main()
{
    using mako::models::H3;
    int failures = 0;
    auto check = [&](bool ok, const char* what) {
        std::printf("  %-4s %s\n", ok ? "ok" : "FAIL", what);
        failures += !ok;
    };
    check(H3::parse_int8("all") == 15u && H3::parse_int8("qkv,fc2") == 9u && !H3::parse_int8("bogus"), "parse_int8");
    H3::Layout l;
    l.text = 4, l.frames = 2, l.h = 4, l.w = 6, l.audio = 3;
    const H3::Rows r = H3::rows(l);
    check(r.tags.size() == l.rows() && r.pos.size() == 3 * l.rows(), "rows: one entry per row");
    check(r.tags[0] == H3::kTextTag && r.tags[4] == H3::kAudioTag && r.tags.back() == H3::kVideoTag, "rows: tags by segment");
    // A ref2va layout written the way tests/h3_ref_test.cpp:475-480 writes it.
    using LR = H3::Layout::Reference;
    H3::Layout ref{.text = 7, .frames = 6, .h = 8, .w = 12, .audio = 9};
    ref.refs = {LR{.kind = LR::Kind::image, .frames = 1, .h = 6, .w = 10}, LR{.kind = LR::Kind::audio, .audio = 5},
                LR{.kind = LR::Kind::video, .frames = 3, .h = 4, .w = 6, .audio = 11}};
    check(ref.cond_rows() == 15 + 18 && ref.cond_audio_rows() == 32 && ref.rows() == 7 + 33 + 6 * 24 + 32 + 18,
          "ref2va layout: row counts");
    const H3::Rows rr = H3::rows(ref);
    check(rr.tags.size() == ref.rows() && rr.roles[7] == 1 && rr.roles[7 + 15] == 2 && rr.pos[3 * 7] == 7.0 &&
              rr.pos[3 * (7 + 15)] == 8.0,
          "ref2va layout: rows (picture at the text's length, the soundtrack after it)");
    const std::vector<float> sv = H3::sigmas(3, 12.0f);
    check(sv.size() == 3 && sv[0] == 1.0f && sv[2] == 0.0f, "sigmas (tests/geometry_test.cpp:32-36)");
    bool threw = false;
    try {
        mako::mtl::Context ctx;
        H3 h("/models/minimax-h3/FL2VA/transformer", ctx, mako::gpu::Telemetry::off, 0);
    } catch (const std::runtime_error& e) {
        threw = std::string(e.what()).find("cannot open") != std::string::npos;
    }
    check(threw, "a missing checkpoint is refused with a message");
    check(H3::check_weights("/models/minimax-h3/FL2VA/transformer").find("cannot open") != std::string::npos,
          "check_weights reports a missing checkpoint");
    // The video decoder's drop-in: the engine's call shapes compile; a real model directory is refused with a message.
    check(mako::video::VideoVae::pixel_frames(37) == 124 && mako::video::VideoVae::pixel_frames(7) == 22, "VideoVae::pixel_frames");
    bool vae_threw = false;
    try {
        mako::mtl::Context ctx;
        mako::video::VideoVae vae("/models/minimax-h3/video_vae", ctx, mako::gpu::Telemetry::off);
    } catch (const std::runtime_error& e) {
        vae_threw = std::string(e.what()).find("synthetic") != std::string::npos;
    }
    check(vae_threw, "VideoVae refuses a checkpoint directory with a message");
    // The C ABI's struct layouts, for the bindings' own declarations to be checked against (tests/test_cpp_dropin.py).
    std::printf("abi h3_config %zu %zu %zu\n", sizeof(h3_config), offsetof(h3_config, refiner_blocks), offsetof(h3_config, curve_dims));
    std::printf("abi h3_layout %zu %zu %zu\n", sizeof(h3_layout), offsetof(h3_layout, refs), offsetof(h3_layout, n_refs));
    std::printf("abi h3_layout_ref %zu\n", sizeof(h3_layout_ref));
    std::printf("abi h3_world %zu %zu\n", sizeof(h3_world), offsetof(h3_world, nccl_id));
    std::printf("abi h3k_gemm_args %zu %zu\n", sizeof(h3k_gemm_args), offsetof(h3k_gemm_args, b_scale));
    std::printf("abi h3k_cube_grid %zu\n", sizeof(h3k_cube_grid));
    std::printf("abi h3vae_config %zu %zu\n", sizeof(h3vae_config), offsetof(h3vae_config, eps));
    return failures ? 1 : 0;
}
