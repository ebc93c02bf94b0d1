// Compiles the drop-in header the way the reference's sampler would use it (mako::models::H3) and exercises its
// host-side members, which need no GPU: parse_int8, rows, and the refusal of a checkpoint path.
#include "models/h3.hpp"

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
    bool threw = false;
    try {
        mako::mtl::Context ctx;
        H3 h("/models/minimax-h3/FL2VA/transformer", ctx, mako::gpu::Telemetry::off, 0);
    } catch (const std::runtime_error& e) {
        threw = std::string(e.what()).find("synthetic") != std::string::npos;
    }
    check(threw, "a checkpoint path is refused with a message");
    return failures ? 1 : 0;
}
