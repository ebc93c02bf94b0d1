// The H3 step's host runtime: weights, per-layout tables, the step's kernel sequence and, with more than one rank,
// the Ulysses all-to-alls over NCCL (sequence split outside attention, head split inside it).
#include "model.hpp"

#include "common.hpp"
#include "devbuf.hpp"
#include "embed.cuh"
#include "gemm.cuh"
#include "rows.cuh"
#include "safetensors.hpp"

#include <nccl.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <map>
#include <sstream>
#include <stdexcept>

namespace h3 {

// ------------------------------------------------------------------------------------------------ layout rows
namespace {

// NVTX range over a scope (the step, each block, each denoising step): what a profiler's timeline groups the
// launches by, free when no tool is attached.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    explicit NvtxRange(const std::string& name) { nvtxRangePushA(name.c_str()); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

// Time position of generated latent frame f, in audio-latent units (40 a second): the frames before it at 24 fps,
// the video VAE packing 17 frames into 5 latents as (1, 4, 4, 4, 4).
double video_time(int f)
{
    static const int within[5] = {0, 1, 5, 9, 13};
    const int frames_before = 17 * (f / 5) + within[f % 5];
    return 5.0 / 3.0 * frames_before;
}

} // namespace

// Positions follow docs/architecture.md:35-45 (text, keyframes, audio, video) and :203-215 (reference blocks): the
// media rows share one time clock that starts at the text's length; a picture sits at one slot and advances the
// clock by one, a soundtrack one slot a latent, a video's soundtrack and frames start together and advance the clock
// by the longer of the two spans (its frames spaced as the generated video's); the generated audio and video rows
// start where the clock ends. The spatial axes are each block's own latent grid centred on the unit square; audio
// rows sit at the two ends of the width axis of the grid they belong to (a video's own, else the generated one's).
Rows layout_rows(const Layout& l)
{
    Rows r;
    const int S = l.rows();
    r.pos.assign(size_t(S) * 3, 0.0);
    r.tags.assign(S, 0);
    r.roles.assign(S, 0);
    struct Grid {
        int ph, pw;
        double norm;
        double hpos(int y) const { return (y + 0.5 - ph / 2.0) / norm * 32.0; }
        double wpos(int x) const { return (x + 0.5 - pw / 2.0) / norm * 32.0; }
    };
    auto grid_of = [](int h, int w) { return Grid{h / 2, w / 2, std::sqrt(double(h / 2) * (w / 2))}; };
    const Grid gen = grid_of(l.h, l.w);
    int row = 0;
    auto put = [&](double t, double y, double x, uint8_t tag, uint8_t role) {
        r.pos[3 * row] = t, r.pos[3 * row + 1] = y, r.pos[3 * row + 2] = x;
        r.tags[row] = tag, r.roles[row] = role;
        ++row;
    };
    auto frame_rows = [&](const Grid& g, double t, uint8_t role) {
        for (int y = 0; y < g.ph; ++y)
            for (int x = 0; x < g.pw; ++x)
                put(t, g.hpos(y), g.wpos(x), 0, role);
    };
    auto audio_rows = [&](const Grid& g, double t, int n, uint8_t role) {
        for (int c = 0; c < 2; ++c)
            for (int a = 0; a < n; ++a)
                put(t + a, 0.0, g.wpos(c == 0 ? 0 : g.pw - 1), 2, role);
    };
    for (int i = 0; i < l.text; ++i)
        put(i, 0.0, 0.0, l.text_tags.empty() ? 1 : l.text_tags[i], 0);
    double clock = l.text;
    for (int k = 0; k < l.cond_frames; ++k) {
        const bool last = k < int(l.cond_last.size()) && l.cond_last[k];
        frame_rows(gen, clock + video_time(last ? std::max(l.frames - 1, 0) : 0), 1);
    }
    for (const LayoutRef& ref : l.refs) {
        if (ref.kind == LayoutRef::kImage) {
            frame_rows(grid_of(ref.h, ref.w), clock, 1);
            clock += 1.0;
        } else if (ref.kind == LayoutRef::kAudio) {
            audio_rows(gen, clock, ref.audio, 2);
            clock += ref.audio;
        } else {
            const Grid g = grid_of(ref.h, ref.w);
            audio_rows(g, clock, ref.audio, 2);
            for (int f = 0; f < ref.frames; ++f)
                frame_rows(g, clock + video_time(f), 1);
            clock += std::max(double(ref.audio), video_time(ref.frames));
        }
    }
    audio_rows(gen, clock, l.audio, 3);
    for (int f = 0; f < l.frames; ++f)
        frame_rows(gen, clock + video_time(f), 4);
    return r;
}

std::vector<Segment> layout_segments(const Layout& l)
{
    const Rows r = layout_rows(l);
    std::vector<Segment> out;
    int in_video = 0, in_audio = 0;
    const int S = int(r.roles.size());
    for (int i = 0; i < S;) {
        int j = i;
        while (j < S && r.roles[j] == r.roles[i])
            ++j;
        const int role = r.roles[i];
        Segment sg{i, j - i, role, -1};
        if (role == 1 || role == 4)
            sg.input_row = in_video, in_video += j - i;
        else if (role == 2 || role == 3)
            sg.input_row = in_audio, in_audio += j - i;
        out.push_back(sg);
        i = j;
    }
    return out;
}

void rope_inv_freq(float out[16])
{
    // In float throughout, as torch evaluates 1 / 10000 ** (arange(0, 32, 2, float32) / 32).
    for (int i = 0; i < 16; ++i) {
        const float e = float(2 * i) / 32.0f;
        out[i] = 1.0f / powf(10000.0f, e);
    }
}

std::vector<float> rope_table(const Rows& r)
{
    float f[16];
    rope_inv_freq(f);
    const size_t S = r.tags.size();
    std::vector<float> t(S * 96);
    for (size_t i = 0; i < S; ++i)
        for (int a = 0; a < 3; ++a)
            for (int k = 0; k < 16; ++k) {
                const float ang = float(r.pos[3 * i + a]) * f[k];
                t[i * 96 + (a * 16 + k) * 2] = float(std::cos(double(ang)));
                t[i * 96 + (a * 16 + k) * 2 + 1] = float(std::sin(double(ang)));
            }
    return t;
}

bool parse_int8(const std::string& s, uint32_t& mask)
{
    if (s == "none" || s.empty()) {
        mask = 0;
        return true;
    }
    if (s == "all") {
        mask = kInt8Qkv | kInt8Out | kInt8Fc1 | kInt8Fc2;
        return true;
    }
    uint32_t m = 0;
    std::stringstream ss(s);
    std::string item;
    while (std::getline(ss, item, ',')) {
        if (item == "qkv")
            m |= kInt8Qkv;
        else if (item == "out")
            m |= kInt8Out;
        else if (item == "fc1")
            m |= kInt8Fc1;
        else if (item == "fc2")
            m |= kInt8Fc2;
        else
            return false;
    }
    mask = m;
    return true;
}

namespace {

// Synthetic tensor ids (fixed: the CPU oracle regenerates the same values from them).
enum : uint32_t {
    kTInW = 1, kTInB, kTOutW, kTOutB, kVpW, kVpB, kApW, kApB, kCondW, kCondB, kFadaW, kFadaB, kHvW, kHvB, kHaW, kHaB,
    kRefinerNorm = 17, kCurveTable = 18,
    kBlockBase = 100, kBlockStride = 20,
    kRefinerBase = 60, // token refiner block r (r < 2) at kRefinerBase + kBlockStride * r, without the AdaLN ids
};
enum : uint32_t { kAdaW = 0, kAdaB, kNorm1, kQkvW, kQkvB, kQn, kKn, kOutW, kOutB, kNorm2, kFc1W, kFc1B, kFc2W, kFc2B };

constexpr float kStd = 0.02f;
constexpr float kCurveStd = 4.0f; // synthetic adaln_t_table values: modulations of the same size as the full model's

} // namespace

struct Model::Impl {
    // weights
    DevBuf t_in_w, t_in_b, t_out_w, t_out_b;
    DevBuf vp_w, vp_b, ap_w, ap_b, cond_w, cond_b;
    DevBuf ada_w, ada_b;   // all blocks: [L][18 d][t_dim] bf16 ([L][18 d][8] f32 for a pruned checkpoint), [L][18 d] f32
    DevBuf fada_w, fada_b; // [2 d][t_dim] bf16 ([2 d][8] f32 pruned), [2 d]
    std::vector<float> curve_table; // pruned checkpoint: adaln_t_table [1025][8] (host copy; read per step)
    DevBuf hv_w, hv_b, ha_w, ha_b;
    struct Block {
        DevBuf norm1, qkv_w, qkv_b, qn, kn, out_w, out_b, norm2, fc1_w, fc1_b, fc2_w, fc2_b;
        DevBuf qkv_q, qkv_s, out_q, out_s, fc1_q, fc1_s, fc2_q, fc2_s; // int8 rows and scales
        // bound on the block's attention scores (log2 units) from its q/k norm weights, 0 when above the attention's
        // limit for one (set at load; LoRA leaves the norm weights as they are)
        float qk_bound = 0.f;
    };
    std::vector<Block> blocks;
    std::vector<Block> refiner; // token refiner blocks (bf16 only; no AdaLN)
    DevBuf refiner_norm;        // [d] weight of the refiner's final RMS norm
    // per layout
    DevBuf x_text;     // [T][d] f32
    DevBuf rope;       // [S_local][48][2]
    DevBuf mod_idx;    // [S_local] u8: level * 3 + tag
    DevBuf lvl_idx;    // [S_local] u8: level
    // The step keeps the generated video rows in the packed (cube-major) order; these map between it and the
    // layout's (frame, row, column) order: video_src[i] = layout index of packed video row i, video_dst the inverse.
    CubeGrid grid;
    std::vector<int32_t> h_video_src;
    DevBuf video_src, video_dst, out_video_rows;
    DevBuf den_video, den_audio, vel_video, vel_audio; // the denoising loop's sample and velocities
    // Pinned staging of a step's small host tables (row levels, time embeddings), reused once the previous step's
    // copies have run (upload_done), so consecutive steps queue without draining the stream.
    uint8_t* pinned = nullptr;
    size_t pinned_bytes = 0;
    cudaEvent_t upload_done = nullptr;
    // per global row; lvl_kind: 0 video/text level, 1 audio, 2 conditioning video (0.999), 3 reference audio (1)
    std::vector<uint8_t> h_tags, h_roles, h_lvl_kind;
    std::vector<Segment> segs;
    // per step
    DevBuf emb, th, temb, tsilu, mods, fmods;
    DevBuf x, h, hq, hs, qkv, qkv_recv, o, o_recv, act;
    DevBuf in_video, in_audio, pk_video, pk_audio, rows_out, rows_all;
    SparseBuffers sp;
    DevBuf sp_mq, sp_mk, sp_scores, sp_sel, sp_nsel, sp_blocks, sp_nblocks, sp_qrows;
    DevBuf attn_part; // dense attention split scratch: [2][S][H/P][128] fp32 outputs, then [2][S][H/P][2] (max, sum)
    size_t attn_split_bytes = 0;
    ncclComm_t comm = nullptr;
    std::vector<cudaEvent_t> ev;
    // Sequence parallel with the exchange fused into the kernels: every rank's qkv_recv and o_recv mapped here.
    bool fused = true;
    void* peer_qkv[8] = {};
    void* peer_o[8] = {};
    std::vector<void*> opened; // peers' buffers mapped by cudaIpcOpenMemHandle (closed on re-map and exit)
    void* mapped_qkv = nullptr;
    void* mapped_o = nullptr;
    DevBuf barrier_word, ipc_stage;
    void close_peers()
    {
        for (void* p : opened)
            cudaIpcCloseMemHandle(p);
        opened.clear();
        mapped_qkv = mapped_o = nullptr;
    }
};

#define H3_NCCL(x)                                                                                                       \
    do {                                                                                                                 \
        const ncclResult_t r_ = (x);                                                                                     \
        if (r_ != ncclSuccess)                                                                                           \
            throw CudaError(std::string("NCCL: ") + #x + ": " + ncclGetErrorString(r_));                                  \
    } while (0)

// ------------------------------------------------------------------------------------------------ weights

std::vector<WeightSpec> weight_specs(const Config& c)
{
    const int64_t d = c.dim, inner = c.inner(), F = c.ffn, td = c.time_dim;
    const bool pruned = c.curve > 0;
    const int64_t ka = pruned ? c.curve : td; // the AdaLN projections' input width
    std::vector<WeightSpec> w;
    auto add = [&](std::string name, std::vector<int64_t> shape, bool bf16, uint32_t id, float mean, float stdev, int owner = 0,
                   int index = -1) {
        WeightSpec sp;
        sp.name = std::move(name), sp.shape = std::move(shape), sp.bf16 = bf16, sp.id = id, sp.mean = mean, sp.stdev = stdev;
        sp.owner = owner, sp.index = index;
        w.push_back(std::move(sp));
    };
    // model-level weights: the names the reference's own files and prose use where they give one (time_embedder.*,
    // blocks.N.adaln_proj.linear.*, adaln_t_table: tools/check_pruned_curve.py:43-56; condition_proj, video_patch_proj,
    // audio_patch_proj, proj_out: docs/architecture.md:26-31,115), this build's names elsewhere
    if (!pruned) {
        add("time_embedder.proj_in.weight", {d, 256}, false, kTInW, 0.f, kStd);
        add("time_embedder.proj_in.bias", {d}, false, kTInB, 0.f, kStd);
        add("time_embedder.proj_out.weight", {td, d}, false, kTOutW, 0.f, kStd);
        add("time_embedder.proj_out.bias", {td}, false, kTOutB, 0.f, kStd);
    } else {
        add("adaln_t_table", {1025, int64_t(c.curve)}, false, kCurveTable, 0.f, kCurveStd);
    }
    add("video_patch_proj.weight", {d, int64_t(c.video_patch)}, true, kVpW, 0.f, kStd);
    add("video_patch_proj.bias", {d}, false, kVpB, 0.f, kStd);
    add("audio_patch_proj.weight", {d, int64_t(c.audio_channels)}, true, kApW, 0.f, kStd);
    add("audio_patch_proj.bias", {d}, false, kApB, 0.f, kStd);
    add("condition_proj.weight", {d, int64_t(c.text_dim)}, true, kCondW, 0.f, kStd);
    add("condition_proj.bias", {d}, false, kCondB, 0.f, kStd);
    add("norm_out.adaln_proj.weight", {2 * d, ka}, !pruned, kFadaW, 0.f, kStd);
    add("norm_out.adaln_proj.bias", {2 * d}, false, kFadaB, 0.f, kStd);
    add("proj_out.weight", {int64_t(c.video_patch), d}, false, kHvW, 0.f, kStd);
    add("proj_out.bias", {int64_t(c.video_patch)}, false, kHvB, 0.f, kStd);
    add("audio_proj_out.weight", {int64_t(c.audio_channels), d}, false, kHaW, 0.f, kStd);
    add("audio_proj_out.bias", {int64_t(c.audio_channels)}, false, kHaB, 0.f, kStd);
    auto block = [&](int owner, int index, uint32_t base) {
        const std::string p = (owner == 1 ? "blocks." : "token_refiner.blocks.") + std::to_string(index) + ".";
        if (owner == 1) {
            add(p + "adaln_proj.linear.weight", {18 * d, ka}, !pruned, base + kAdaW, 0.f, kStd, owner, index);
            add(p + "adaln_proj.linear.bias", {18 * d}, false, base + kAdaB, 0.f, kStd, owner, index);
        }
        add(p + "norm1.weight", {d}, false, base + kNorm1, 1.f, kStd, owner, index);
        add(p + "attn.qkv.weight", {3 * inner, d}, true, base + kQkvW, 0.f, kStd, owner, index);
        add(p + "attn.qkv.bias", {3 * inner}, false, base + kQkvB, 0.f, kStd, owner, index);
        add(p + "attn.norm_q.weight", {128}, false, base + kQn, 1.f, kStd, owner, index);
        add(p + "attn.norm_k.weight", {128}, false, base + kKn, 1.f, kStd, owner, index);
        add(p + "attn.to_out.weight", {d, inner}, true, base + kOutW, 0.f, kStd, owner, index);
        add(p + "attn.to_out.bias", {d}, false, base + kOutB, 0.f, kStd, owner, index);
        add(p + "norm2.weight", {d}, false, base + kNorm2, 1.f, kStd, owner, index);
        add(p + "ff.fc1.weight", {2 * F, d}, true, base + kFc1W, 0.f, kStd, owner, index);
        add(p + "ff.fc1.bias", {2 * F}, false, base + kFc1B, 0.f, kStd, owner, index);
        add(p + "ff.fc2.weight", {d, F}, true, base + kFc2W, 0.f, kStd, owner, index);
        add(p + "ff.fc2.bias", {d}, false, base + kFc2B, 0.f, kStd, owner, index);
    };
    for (int l = 0; l < c.blocks; ++l)
        block(1, l, kBlockBase + kBlockStride * l);
    for (int r = 0; r < c.refiner; ++r)
        block(2, r, kRefinerBase + kBlockStride * r);
    if (c.refiner > 0)
        add("token_refiner.norm.weight", {d}, false, kRefinerNorm, 1.f, kStd);
    return w;
}

void SyntheticWeights::get(const WeightSpec& spec, void* dst, cudaStream_t s)
{
    fill_synthetic(dst, spec.bf16, spec.count(), seed_, spec.id, spec.mean, spec.stdev, s);
}

struct CheckpointWeights::Files {
    std::vector<std::unique_ptr<SafeTensors>> files;
    std::vector<bool> interleaved;       // per file: metadata qkv_layout = interleaved
    std::vector<bool> tagged;            // per file: the metadata has a qkv_layout entry
    std::vector<std::string> paths;
    std::map<std::string, size_t> where; // tensor name -> file
    std::map<std::string, std::string> renames;
    // the checkpoint's name of a weight
    const std::string& source(const std::string& name) const
    {
        const auto it = renames.find(name);
        return it == renames.end() ? name : it->second;
    }
};

CheckpointWeights::CheckpointWeights(const std::string& path, std::map<std::string, std::string> renames, bool interleaved)
    : f_(new Files)
{
    f_->renames = std::move(renames);
    std::vector<std::string> paths;
    std::error_code ec;
    if (std::filesystem::is_directory(path, ec)) {
        for (const auto& e : std::filesystem::directory_iterator(path, ec))
            if (e.is_regular_file(ec) && e.path().extension() == ".safetensors")
                paths.push_back(e.path().string());
        std::sort(paths.begin(), paths.end());
        if (paths.empty())
            throw std::invalid_argument("checkpoint: no .safetensors file in " + path);
    } else {
        paths.push_back(path);
    }
    for (const std::string& p : paths) {
        std::unique_ptr<SafeTensors> st;
        try {
            st = std::make_unique<SafeTensors>(p);
        } catch (const std::runtime_error& e) {
            throw std::invalid_argument(std::string("checkpoint: ") + e.what());
        }
        const auto it = st->metadata().find("qkv_layout");
        f_->interleaved.push_back(interleaved || (it != st->metadata().end() && it->second == "interleaved"));
        f_->tagged.push_back(it != st->metadata().end());
        f_->paths.push_back(p);
        for (const auto& [name, t] : st->tensors())
            if (!f_->where.emplace(name, f_->files.size()).second)
                throw std::invalid_argument("checkpoint: tensor " + name + " appears in two files");
        f_->files.push_back(std::move(st));
    }
}

CheckpointWeights::~CheckpointWeights() = default;

std::string CheckpointWeights::check(const Config& c) const
{
    for (const WeightSpec& sp : weight_specs(c)) {
        const std::string& src = f_->source(sp.name);
        const auto it = f_->where.find(src);
        if (it == f_->where.end())
            return "no tensor " + src + (src == sp.name ? "" : " (for " + sp.name + ")");
        const SafeTensor& t = f_->files[it->second]->tensors().at(src);
        if (t.shape != sp.shape) {
            std::string got, want;
            for (int64_t v : t.shape)
                got += (got.empty() ? "" : "x") + std::to_string(v);
            for (int64_t v : sp.shape)
                want += (want.empty() ? "" : "x") + std::to_string(v);
            return sp.name + " is " + got + ", this model needs " + want;
        }
        if (t.dtype != "BF16" && t.dtype != "F16" && t.dtype != "F32")
            return sp.name + " has dtype " + t.dtype + " (BF16, F16 or F32 expected)";
    }
    return "";
}

static bool is_qkv(const std::string& name)
{
    return (name.size() > 15 && name.compare(name.size() - 15, 15, "attn.qkv.weight") == 0) ||
           (name.size() > 13 && name.compare(name.size() - 13, 13, "attn.qkv.bias") == 0);
}

std::string CheckpointWeights::untagged_qkv_file(const Config& c) const
{
    for (const WeightSpec& sp : weight_specs(c)) {
        if (!is_qkv(sp.name))
            continue;
        const auto it = f_->where.find(f_->source(sp.name));
        if (it != f_->where.end() && !f_->tagged[it->second])
            return f_->paths[it->second];
    }
    return "";
}

void CheckpointWeights::get(const WeightSpec& spec, void* dst, cudaStream_t s)
{
    const std::vector<unsigned char> h = host(spec);
    H3_CUDA(cudaMemcpyAsync(dst, h.data(), h.size(), cudaMemcpyHostToDevice, s));
    H3_CUDA(cudaStreamSynchronize(s)); // the host copy goes out of scope
}

std::vector<unsigned char> CheckpointWeights::host(const WeightSpec& spec) const
{
    const std::string& src = f_->source(spec.name);
    const auto it = f_->where.find(src);
    if (it == f_->where.end())
        throw std::invalid_argument("checkpoint: no tensor " + src);
    const SafeTensors& st = *f_->files[it->second];
    if (st.tensors().at(src).shape != spec.shape)
        throw std::invalid_argument("checkpoint: " + src + " has another shape than this model's " + spec.name);
    const size_t esz = spec.bf16 ? 2 : 4;
    std::vector<unsigned char> host(spec.count() * esz);
    if (spec.bf16) {
        const std::vector<uint16_t> v = st.read_bf16(src);
        std::memcpy(host.data(), v.data(), host.size());
    } else {
        const std::vector<float> v = st.read_f32(src);
        std::memcpy(host.data(), v.data(), host.size());
    }
    if (is_qkv(spec.name) && f_->interleaved[it->second]) {
        // [q_h; k_h; v_h] for every head h -> [q (all heads); k; v]
        const int64_t rows = spec.shape[0], cols = spec.shape.size() > 1 ? spec.shape[1] : 1, inner = rows / 3;
        const size_t row_bytes = size_t(cols) * esz;
        std::vector<unsigned char> stacked(host.size());
        for (int64_t h = 0; h < inner / 128; ++h)
            for (int p = 0; p < 3; ++p)
                for (int r = 0; r < 128; ++r)
                    std::memcpy(&stacked[size_t(p * inner + h * 128 + r) * row_bytes], &host[size_t(h * 384 + p * 128 + r) * row_bytes], row_bytes);
        host.swap(stacked);
    }
    return host;
}

void convert_checkpoint(const Config& c, const std::string& src, const std::string& dst, std::map<std::string, std::string> renames,
                        bool interleaved, bool layout_given)
{
    const CheckpointWeights ck(src, std::move(renames), interleaved);
    const std::string problem = ck.check(c);
    if (!problem.empty())
        throw std::invalid_argument("convert: " + src + ": " + problem);
    if (!layout_given) {
        const std::string untagged = ck.untagged_qkv_file(c);
        if (!untagged.empty())
            throw std::invalid_argument("convert: " + untagged + " holds q/k/v tensors but its metadata has no qkv_layout: add a "
                                        "\"qkv_layout interleaved\" or \"qkv_layout stacked\" line (the reference's shards keep "
                                        "each head's q, k, v rows together)");
    }
    const std::vector<WeightSpec> specs = weight_specs(c);
    std::vector<SafeTensorOut> outs;
    for (const WeightSpec& sp : specs) {
        SafeTensorOut o;
        o.name = sp.name, o.dtype = sp.bf16 ? "BF16" : "F32", o.shape = sp.shape, o.bytes = sp.count() * (sp.bf16 ? 2 : 4);
        outs.push_back(std::move(o));
    }
    write_safetensors(dst, outs, {{"format", "pt"}, {"qkv_layout", "stacked"}, {"writer", "libh3b200"}},
                      [&](size_t i, std::vector<unsigned char>& buf) { buf = ck.host(specs[i]); });
}

Model::Model(const Config& c, uint64_t seed, uint32_t int8_mask, const World& world)
    : d_(new Impl), c_(c), world_(world), int8_(int8_mask)
{
    SyntheticWeights src(seed);
    init(src);
}

Model::Model(const Config& c, WeightSource& src, uint32_t int8_mask, const World& world)
    : d_(new Impl), c_(c), world_(world), int8_(int8_mask)
{
    init(src);
}

// Where a weight lives on the device and how its logical layout maps onto the stored one.
struct Model::Target {
    enum Mode { plain, audio_padded, fc1_rows, fc1_bias, curve } mode = plain;
    DevBuf* buf = nullptr;
    size_t offset = 0; // bytes into buf (plain: the AdaLN projections of all blocks share one buffer)
};

Model::Target Model::locate(const WeightSpec& sp)
{
    const int d = c_.dim;
    const size_t ka = c_.curve ? size_t(c_.curve) : size_t(c_.time_dim);
    Target t;
    if (sp.owner == 0) {
        switch (sp.id) {
        case kTInW: t.buf = &d_->t_in_w; break;
        case kTInB: t.buf = &d_->t_in_b; break;
        case kTOutW: t.buf = &d_->t_out_w; break;
        case kTOutB: t.buf = &d_->t_out_b; break;
        case kCurveTable: t.mode = Target::curve; break;
        case kVpW: t.buf = &d_->vp_w; break;
        case kVpB: t.buf = &d_->vp_b; break;
        case kApW: t.buf = &d_->ap_w, t.mode = Target::audio_padded; break;
        case kApB: t.buf = &d_->ap_b; break;
        case kCondW: t.buf = &d_->cond_w; break;
        case kCondB: t.buf = &d_->cond_b; break;
        case kFadaW: t.buf = &d_->fada_w; break;
        case kFadaB: t.buf = &d_->fada_b; break;
        case kHvW: t.buf = &d_->hv_w; break;
        case kHvB: t.buf = &d_->hv_b; break;
        case kHaW: t.buf = &d_->ha_w; break;
        case kHaB: t.buf = &d_->ha_b; break;
        case kRefinerNorm: t.buf = &d_->refiner_norm; break;
        default: throw CudaError("weights: unknown tensor " + sp.name);
        }
        return t;
    }
    Impl::Block& B = sp.owner == 1 ? d_->blocks.at(sp.index) : d_->refiner.at(sp.index);
    const uint32_t local = sp.id - (sp.owner == 1 ? kBlockBase : kRefinerBase) - kBlockStride * uint32_t(sp.index);
    switch (local) {
    case kAdaW: t.buf = &d_->ada_w, t.offset = size_t(sp.index) * 18 * d * ka * (c_.curve ? 4 : 2); break;
    case kAdaB: t.buf = &d_->ada_b, t.offset = size_t(sp.index) * 18 * d * 4; break;
    case kNorm1: t.buf = &B.norm1; break;
    case kQkvW: t.buf = &B.qkv_w; break;
    case kQkvB: t.buf = &B.qkv_b; break;
    case kQn: t.buf = &B.qn; break;
    case kKn: t.buf = &B.kn; break;
    case kOutW: t.buf = &B.out_w; break;
    case kOutB: t.buf = &B.out_b; break;
    case kNorm2: t.buf = &B.norm2; break;
    case kFc1W: t.buf = &B.fc1_w, t.mode = Target::fc1_rows; break;
    case kFc1B: t.buf = &B.fc1_b, t.mode = Target::fc1_bias; break;
    case kFc2W: t.buf = &B.fc2_w; break;
    case kFc2B: t.buf = &B.fc2_b; break;
    default: throw CudaError("weights: unknown tensor " + sp.name);
    }
    return t;
}

void Model::init(WeightSource& src)
{
    const Config& c = c_;
    const World& world = world_;
    if (c.dim % 256 || c.inner() % 256 || c.ffn % 128 || (2 * c.ffn) % 256 || c.time_dim % 8 || c.text_dim % 8 || c.dim > 8192)
        throw CudaError("config: dim and heads*128 multiples of 256, ffn of 128, time_dim and text_dim of 8, dim <= 8192");
    if (world.size < 1 || world.rank < 0 || world.rank >= world.size || c.heads % world.size)
        throw CudaError("world: heads must divide evenly over the ranks");
    if (c.curve != 0 && c.curve != 8)
        throw CudaError("config: curve_dims is 0 or 8");
    if (c.refiner < 0 || c.refiner > 2)
        throw CudaError("config: at most 2 token refiner blocks");
    H3_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    if (world.size > 1) {
        if (world.size > 8)
            throw CudaError("world: at most 8 ranks (one NVSwitch box)");
        ncclUniqueId id;
        static_assert(sizeof(id) == 128, "ncclUniqueId size");
        std::memcpy(&id, world.nccl_id, 128);
        H3_NCCL(ncclCommInitRank(&d_->comm, world.size, id, world.rank));
        const char* ex = std::getenv("H3_EXCHANGE");
        d_->fused = !(ex && std::string(ex) == "nccl");
    }
    const int d = c.dim, L = c.blocks, inner = c.inner(), F = c.ffn;
    const size_t ka = c.curve ? size_t(c.curve) : size_t(c.time_dim);
    cudaStream_t s = stream_;
    d_->blocks.resize(L);
    d_->refiner.resize(c.refiner);
    // the AdaLN projections of every block in one tensor (one GEMV reads them all): block l at offset l * 18 d ka
    d_->ada_w.ensure(size_t(L) * 18 * d * ka * (c.curve ? 4 : 2));
    d_->ada_b.ensure(size_t(L) * 18 * d * 4);
    d_->ap_w.ensure(size_t(d) * 64 * 2); // zeroed: padded to 64 inputs, the first 32 columns set below
    for (const WeightSpec& sp : weight_specs(c)) {
        const Target t = locate(sp);
        const size_t bytes = sp.count() * (sp.bf16 ? 2 : 4);
        switch (t.mode) {
        case Target::plain:
            if (t.buf != &d_->ada_w && t.buf != &d_->ada_b)
                t.buf->ensure(bytes);
            src.get(sp, t.buf->as<uint8_t>() + t.offset, s);
            break;
        case Target::audio_padded: {
            DevBuf tmp;
            tmp.ensure(bytes);
            src.get(sp, tmp.p, s);
            H3_CUDA(cudaMemcpy2DAsync(t.buf->p, 64 * 2, tmp.p, size_t(c.audio_channels) * 2, size_t(c.audio_channels) * 2, d,
                                      cudaMemcpyDeviceToDevice, s));
            H3_CUDA(cudaStreamSynchronize(s));
            break;
        }
        case Target::fc1_rows:
        case Target::fc1_bias: {
            // stored as [gate; value]; regrouped into 128-row [gate g; value g] pairs for the fused SwiGLU epilogue
            DevBuf tmp;
            tmp.ensure(bytes);
            src.get(sp, tmp.p, s);
            t.buf->ensure(bytes);
            if (t.mode == Target::fc1_rows)
                interleave_gate_value(tmp.p, F, d, t.buf->p, s);
            else
                interleave_gate_value_f32(tmp.as<float>(), F, t.buf->as<float>(), s);
            H3_CUDA(cudaStreamSynchronize(s));
            break;
        }
        case Target::curve: {
            // adaln_t_table: kept on the host for the per-step lookup
            DevBuf tab;
            tab.ensure(bytes);
            src.get(sp, tab.p, s);
            d_->curve_table.resize(sp.count());
            H3_CUDA(cudaMemcpyAsync(d_->curve_table.data(), tab.p, bytes, cudaMemcpyDeviceToHost, s));
            H3_CUDA(cudaStreamSynchronize(s));
            break;
        }
        }
    }
    // int8 at load: the chosen projections' rows quantised per row; their bf16 rows released
    for (Impl::Block& b : d_->blocks) {
        auto quant = [&](DevBuf& w, DevBuf& q, DevBuf& sc, int rows, int K) {
            q.ensure(size_t(rows) * K);
            sc.ensure(size_t(rows) * 4);
            quant_weight_rows(w.p, rows, K, q.as<int8_t>(), sc.as<float>(), s);
            H3_CUDA(cudaStreamSynchronize(s));
            w.release();
        };
        if (int8_ & kInt8Qkv)
            quant(b.qkv_w, b.qkv_q, b.qkv_s, 3 * inner, d);
        if (int8_ & kInt8Out)
            quant(b.out_w, b.out_q, b.out_s, d, inner);
        if (int8_ & kInt8Fc1)
            quant(b.fc1_w, b.fc1_q, b.fc1_s, 2 * F, d);
        if (int8_ & kInt8Fc2)
            quant(b.fc2_w, b.fc2_q, b.fc2_s, d, F);
    }
    H3_CUDA(cudaStreamSynchronize(s));
    if (take_device_error(s))
        throw CudaError("device error during weight set-up");
    // Every block's score bound: q and k are RMS-normed per head with these weights, so |q.k| / sqrt(128) is at most
    // sqrt(128) max|w_q| max|w_k|. H3_ATTN_ONLINE=1 keeps the online row maximum instead (for comparison).
    const char* online = std::getenv("H3_ATTN_ONLINE");
    const bool bounded = !(online && std::string(online) == "1");
    std::vector<float> wq(128), wk(128);
    std::vector<Impl::Block*> all;
    for (auto& b : d_->blocks)
        all.push_back(&b);
    for (auto& b : d_->refiner)
        all.push_back(&b);
    for (Impl::Block* bp : all) {
        Impl::Block& b = *bp;
        H3_CUDA(cudaMemcpy(wq.data(), b.qn.p, 128 * sizeof(float), cudaMemcpyDeviceToHost));
        H3_CUDA(cudaMemcpy(wk.data(), b.kn.p, 128 * sizeof(float), cudaMemcpyDeviceToHost));
        float mq = 0.f, mk = 0.f;
        for (int i = 0; i < 128; ++i)
            mq = std::max(mq, std::fabs(wq[i])), mk = std::max(mk, std::fabs(wk[i]));
        b.qk_bound = bounded && std::isfinite(mq) && std::isfinite(mk) ? qk_score_bound(mq, mk) : 0.f;
    }
}

void Model::save(const std::string& path)
{
    if (int8_)
        throw std::invalid_argument("save: an int8 model no longer holds the bf16 rows of its quantised projections; save a bf16 model");
    const std::vector<WeightSpec> specs = weight_specs(c_);
    std::vector<SafeTensorOut> outs;
    for (const WeightSpec& sp : specs) {
        SafeTensorOut o;
        o.name = sp.name, o.dtype = sp.bf16 ? "BF16" : "F32", o.shape = sp.shape, o.bytes = sp.count() * (sp.bf16 ? 2 : 4);
        outs.push_back(std::move(o));
    }
    cudaStream_t s = stream_;
    const int d = c_.dim, F = c_.ffn;
    const std::map<std::string, std::string> meta = {{"format", "pt"}, {"qkv_layout", "stacked"}, {"writer", "libh3b200"}};
    write_safetensors(path, outs, meta, [&](size_t i, std::vector<unsigned char>& buf) {
        const WeightSpec& sp = specs[i];
        const Target t = locate(sp);
        switch (t.mode) {
        case Target::plain:
            H3_CUDA(cudaMemcpyAsync(buf.data(), t.buf->as<uint8_t>() + t.offset, buf.size(), cudaMemcpyDeviceToHost, s));
            break;
        case Target::audio_padded:
            H3_CUDA(cudaMemcpy2DAsync(buf.data(), size_t(c_.audio_channels) * 2, t.buf->p, 64 * 2, size_t(c_.audio_channels) * 2, d,
                                      cudaMemcpyDeviceToHost, s));
            break;
        case Target::fc1_rows:
        case Target::fc1_bias: {
            // back from the 128-row [gate g; value g] pairs to [gate; value]
            std::vector<unsigned char> stored(buf.size());
            H3_CUDA(cudaMemcpyAsync(stored.data(), t.buf->p, stored.size(), cudaMemcpyDeviceToHost, s));
            H3_CUDA(cudaStreamSynchronize(s));
            const size_t row = t.mode == Target::fc1_rows ? size_t(d) * 2 : 4;
            for (int i = 0; i < 2 * F; ++i) {
                const int r = i < F ? (i / 128) * 256 + i % 128 : ((i - F) / 128) * 256 + 128 + (i - F) % 128;
                std::memcpy(&buf[size_t(i) * row], &stored[size_t(r) * row], row);
            }
            break;
        }
        case Target::curve:
            std::memcpy(buf.data(), d_->curve_table.data(), buf.size());
            break;
        }
        H3_CUDA(cudaStreamSynchronize(s));
    });
}

Model::~Model()
{
    if (d_)
        d_->close_peers();
    if (d_ && d_->comm)
        ncclCommDestroy(d_->comm);
    if (d_)
        for (cudaEvent_t e : d_->ev)
            cudaEventDestroy(e);
    if (d_ && d_->upload_done)
        cudaEventDestroy(d_->upload_done);
    if (d_ && d_->pinned)
        cudaFreeHost(d_->pinned);
    d_.reset();
    if (stream_)
        cudaStreamDestroy(stream_);
}

void Model::set_sparse(float ratio, int local)
{
    if (!(ratio >= 0.f) || ratio > 1.f)
        throw CudaError("sparse ratio must be within [0, 1]");
    if (local != 0 && local != 1 && local != 3)
        throw CudaError("sparse-local must be 0, 1 or 3");
    sparse_ratio_ = ratio;
    sparse_local_ = local;
    if (begun_) {
        // the layout is known: size the selection and pass-list buffers for the new ratio now (the reference sets
        // the ratio before begin, engine.cpp:112; a caller may also change it between steps)
        size_sparse();
        H3_CUDA(cudaStreamSynchronize(stream_));
    }
}

// The sparse attention's buffers for this layout's cube grid and the current ratio (kept, and only grown, while the
// ratio is zero or the grid has no cubes).
void Model::size_sparse()
{
    const CubeGrid& g = d_->grid;
    if (!(sparse_ratio_ > 0.f) || g.cubes() <= 0)
        return;
    const int Hp = c_.heads / world_.size;
    SparseBuffers& b = d_->sp;
    sparse_sizes(g, sparse_ratio_, sparse_local_, b.kcap, b.q_tiles, b.max_blocks);
    const size_t nc = g.cubes();
    d_->sp_mq.ensure(size_t(Hp) * nc * 128 * 4);
    d_->sp_mk.ensure(size_t(Hp) * nc * 128 * 4);
    d_->sp_scores.ensure(size_t(Hp) * nc * nc * 4);
    d_->sp_sel.ensure(size_t(Hp) * nc * b.kcap * 4);
    d_->sp_nsel.ensure(size_t(Hp) * nc * 4);
    d_->sp_blocks.ensure(size_t(Hp) * b.q_tiles * b.max_blocks * 16);
    d_->sp_nblocks.ensure(size_t(Hp) * b.q_tiles * 4);
    d_->sp_qrows.ensure(size_t(b.q_tiles) * 16);
    b.mq = d_->sp_mq.as<float>(), b.mk = d_->sp_mk.as<float>(), b.scores = d_->sp_scores.as<float>();
    b.sel = d_->sp_sel.as<int32_t>(), b.nsel = d_->sp_nsel.as<int32_t>();
    b.blocks = d_->sp_blocks.as<int4>(), b.nblocks = d_->sp_nblocks.as<int32_t>(), b.q_rows = d_->sp_qrows.as<int4>();
}

void Model::alloc_activations()
{
    const int d = c_.dim, inner = c_.inner(), F = c_.ffn, P = world_.size, Hp = c_.heads / P;
    const size_t M = size_t(S_local_);
    const size_t Spad = M * P;
    d_->x.ensure(M * d * 4);
    d_->h.ensure(M * d * 2);
    const size_t qkv_elems = std::max(M * 3 * inner, M * F);
    // also holds the final norm's fp32 rows
    d_->qkv.ensure(std::max(qkv_elems * 2, M * d * 4));
    if (P > 1) {
        d_->qkv_recv.ensure(Spad * 3 * Hp * 128 * 2);
        d_->o_recv.ensure(M * inner * 2);
    }
    d_->o.ensure(Spad * Hp * 128 * 2);
    if (int8_) {
        d_->hq.ensure(M * std::max({d, F, inner}));
        d_->hs.ensure(M * 4);
    }
    d_->rows_out.ensure(M * 128 * 4);
    d_->rows_all.ensure(Spad * 128 * 4);
    // scratch for the dense attention's key-split halves (only layouts whose attention launch fills few waves)
    d_->attn_split_bytes = attention_split_bytes(S_, Hp);
    if (d_->attn_split_bytes)
        d_->attn_part.ensure(d_->attn_split_bytes);
    if (P > 1 && d_->fused)
        map_peers();
}

void Model::map_peers()
{
    Impl& d = *d_;
    if (d.mapped_qkv == d.qkv_recv.p && d.mapped_o == d.o_recv.p)
        return;
    d.close_peers();
    const int P = world_.size, me = world_.rank;
    cudaIpcMemHandle_t mine[2];
    H3_CUDA(cudaIpcGetMemHandle(&mine[0], d.qkv_recv.p));
    H3_CUDA(cudaIpcGetMemHandle(&mine[1], d.o_recv.p));
    static_assert(sizeof(mine) == 128, "two 64-byte IPC handles");
    d.ipc_stage.ensure(size_t(P) * 128);
    d.barrier_word.ensure(16);
    uint8_t* stage = d.ipc_stage.as<uint8_t>();
    H3_CUDA(cudaMemcpyAsync(stage + size_t(me) * 128, mine, 128, cudaMemcpyHostToDevice, stream_));
    H3_NCCL(ncclAllGather(stage + size_t(me) * 128, stage, 128, ncclUint8, d.comm, stream_));
    std::vector<cudaIpcMemHandle_t> all(2 * size_t(P));
    H3_CUDA(cudaMemcpyAsync(all.data(), stage, size_t(P) * 128, cudaMemcpyDeviceToHost, stream_));
    H3_CUDA(cudaStreamSynchronize(stream_));
    for (int r = 0; r < P; ++r) {
        if (r == me) {
            d.peer_qkv[r] = d.qkv_recv.p;
            d.peer_o[r] = d.o_recv.p;
            continue;
        }
        void* q = nullptr;
        void* o = nullptr;
        H3_CUDA(cudaIpcOpenMemHandle(&q, all[2 * r], cudaIpcMemLazyEnablePeerAccess));
        d.opened.push_back(q);
        H3_CUDA(cudaIpcOpenMemHandle(&o, all[2 * r + 1], cudaIpcMemLazyEnablePeerAccess));
        d.opened.push_back(o);
        d.peer_qkv[r] = q;
        d.peer_o[r] = o;
    }
    d.mapped_qkv = d.qkv_recv.p;
    d.mapped_o = d.o_recv.p;
}

void Model::begin(const float* text, int T, const Layout& l)
{
    if (T != l.text)
        throw CudaError("begin: the text rows do not match the layout");
    if (l.h % 2 || l.w % 2 || l.frames < 0 || l.audio < 0 || l.cond_frames < 0)
        throw CudaError("begin: the latent grid must have even sides");
    if (!l.text_tags.empty() && int(l.text_tags.size()) != T)
        throw CudaError("begin: one text tag per text row");
    if (l.cond_frames > 0 && !l.refs.empty())
        throw CudaError("begin: a layout holds keyframes or reference blocks, not both");
    for (const LayoutRef& ref : l.refs)
        if (ref.kind < LayoutRef::kImage || ref.kind > LayoutRef::kAudio || ref.frames < 0 || ref.audio < 0 || ref.h % 2 || ref.w % 2 ||
            (ref.kind == LayoutRef::kImage && ref.frames != 1) || (ref.kind != LayoutRef::kAudio && (ref.h <= 0 || ref.w <= 0)))
            throw CudaError("begin: bad reference block (a picture is one latent frame; pictures and videos need even sides)");
    layout_ = l;
    S_ = l.rows();
    if (S_ <= 0)
        throw CudaError("begin: empty sequence");
    const int P = world_.size;
    S_local_ = (S_ + P - 1) / P;
    row0_ = world_.rank * S_local_;
    alloc_activations();
    cudaStream_t s = stream_;
    const int d = c_.dim;
    // text rows: condition_proj (text_dim -> d) of the bf16-rounded embeddings
    d_->x_text.ensure(size_t(std::max(T, 1)) * d * 4);
    if (T > 0) {
        DevBuf tin, tpk;
        tin.ensure(size_t(T) * c_.text_dim * 4);
        tpk.ensure(size_t(T) * c_.text_dim * 2);
        H3_CUDA(cudaMemcpyAsync(tin.p, text, size_t(T) * c_.text_dim * 4, cudaMemcpyDefault, s));
        pack_bf16_rows(tin.as<float>(), T, c_.text_dim, tpk.p, c_.text_dim, s);
        GemmParams g;
        g.M = T, g.N = d, g.K = c_.text_dim;
        g.out = d_->x_text.p, g.ldo = d, g.bias = d_->cond_b.as<float>();
        gemm_bf16(tpk.p, d_->cond_w.p, g, Epi::f32, s);
        refine_text(T);
        H3_CUDA(cudaStreamSynchronize(s));
        emit_probe("txt", -1, d_->x_text.as<float>(), size_t(T) * d);
    }
    // the packed row order: generated video rows cube by cube
    CubeGrid& g = d_->grid;
    g = CubeGrid();
    g.dense_rows = l.dense_rows();
    g.frames = l.frames, g.ph = l.h / 2, g.pw = l.w / 2;
    g.nct = (g.frames + 3) / 4, g.ncy = (g.ph + 3) / 4, g.ncx = (g.pw + 3) / 4;
    const int Vg = g.video_rows();
    std::vector<int32_t>& src = d_->h_video_src;
    src.assign(Vg, 0);
    std::vector<int32_t> dst(Vg);
    for (int f = 0, n = 0; f < g.frames; ++f)
        for (int y = 0; y < g.ph; ++y)
            for (int x = 0; x < g.pw; ++x, ++n) {
                const int i = g.video_pos(f, y, x) - g.dense_rows;
                src[i] = n, dst[n] = i;
            }
    d_->video_src.ensure(size_t(std::max(Vg, 1)) * 4);
    d_->video_dst.ensure(size_t(std::max(Vg, 1)) * 4);
    d_->out_video_rows.ensure(size_t(std::max(Vg, 1)) * c_.video_patch * 4);
    if (Vg) {
        H3_CUDA(cudaMemcpyAsync(d_->video_src.p, src.data(), size_t(Vg) * 4, cudaMemcpyHostToDevice, s));
        H3_CUDA(cudaMemcpyAsync(d_->video_dst.p, dst.data(), size_t(Vg) * 4, cudaMemcpyHostToDevice, s));
    }
    // row tables for this rank's rows, in the packed order
    Rows r = layout_rows(l);
    {
        const Rows nat = r;
        const size_t D = size_t(g.dense_rows);
        for (int i = 0; i < Vg; ++i) {
            const size_t to = D + i, from = D + src[i];
            r.tags[to] = nat.tags[from], r.roles[to] = nat.roles[from];
            for (int a = 0; a < 3; ++a)
                r.pos[3 * to + a] = nat.pos[3 * from + a];
        }
    }
    d_->h_tags = r.tags;
    d_->h_roles = r.roles;
    d_->h_lvl_kind.assign(S_, 0);
    for (int i = 0; i < S_; ++i)
        d_->h_lvl_kind[i] = r.roles[i] == 3 ? 1 : (r.roles[i] == 1 ? 2 : (r.roles[i] == 2 ? 3 : 0));
    d_->segs = layout_segments(l);
    const std::vector<float> rope = rope_table(r);
    std::vector<float> local(size_t(S_local_) * 96, 0.f);
    for (int i = 0; i < S_local_ && row0_ + i < S_; ++i)
        std::memcpy(&local[size_t(i) * 96], &rope[size_t(row0_ + i) * 96], 96 * 4);
    d_->rope.ensure(local.size() * 4);
    H3_CUDA(cudaMemcpyAsync(d_->rope.p, local.data(), local.size() * 4, cudaMemcpyHostToDevice, s));
    d_->mod_idx.ensure(S_local_);
    d_->lvl_idx.ensure(S_local_);
    size_sparse();
    H3_CUDA(cudaStreamSynchronize(s));
    begun_ = true;
}

// The token refiner over the text rows x_text (docs/architecture.md:25-27: "a two-block token refiner (plain pre-norm
// blocks, no rotary positions), then its final RMS norm"). Each block is the step's block with its modulation
// replaced by a constant table (shift 0, scale 0, gate 1: plain RMS norms and plain residual adds) and the rotary
// table by the identity (cos 1, sin 0), so it runs on the step's own kernels: the modulated norm, the q/k/v GEMM with
// the per-head q/k norms in its epilogue, dense attention over the T text rows (all heads, on every rank: the text is
// replicated), the out and fc2 GEMMs with the residual add in their epilogues and fc1 with the fused SwiGLU. The final
// norm is x = RMSNorm(x) * refiner_norm. Always bf16 (the int8 mask is for the step's projections).
void Model::refine_text(int T)
{
    const int R = int(d_->refiner.size());
    if (R == 0 || T <= 0)
        return;
    cudaStream_t s = stream_;
    const int d = c_.dim, inner = c_.inner(), F = c_.ffn, H = c_.heads;
    DevBuf h, qkv, o, rope, mod, midx, xn;
    h.ensure(size_t(T) * d * 2);
    qkv.ensure(size_t(T) * std::max(3 * inner, F) * 2);
    o.ensure(size_t(T) * inner * 2);
    midx.ensure(size_t(T)); // zeros: every row reads modulation 0
    xn.ensure(size_t(T) * d * 4);
    {
        std::vector<float> id(size_t(T) * 96);
        for (size_t i = 0; i < id.size(); i += 2)
            id[i] = 1.f, id[i + 1] = 0.f;
        rope.ensure(id.size() * 4);
        H3_CUDA(cudaMemcpyAsync(rope.p, id.data(), id.size() * 4, cudaMemcpyHostToDevice, s));
        std::vector<float> m(size_t(6) * d, 0.f); // shift, scale, gate of attention, then of the FFN
        std::fill(m.begin() + size_t(2) * d, m.begin() + size_t(3) * d, 1.f);
        std::fill(m.begin() + size_t(5) * d, m.end(), 1.f);
        mod.ensure(m.size() * 4);
        H3_CUDA(cudaMemcpyAsync(mod.p, m.data(), m.size() * 4, cudaMemcpyHostToDevice, s));
        H3_CUDA(cudaStreamSynchronize(s)); // the host vectors go out of scope
    }
    float* x = d_->x_text.as<float>();
    const uint8_t* mi = midx.as<uint8_t>();
    for (int r = 0; r < R; ++r) {
        const Impl::Block& B = d_->refiner[r];
        RmsModParams rp;
        rp.x = x, rp.ldx = d, rp.rows = T, rp.d = d, rp.w = B.norm1.as<float>(), rp.mod = mod.as<float>(), rp.mod_idx = mi;
        rp.mod_slots = 6, rp.shift_slot = 0, rp.scale_slot = 1, rp.eps = c_.eps, rp.out_kind = RowOut::bf16, rp.out = h.p, rp.ldo = d;
        rms_mod_rows(rp, s);
        GemmParams gq;
        gq.M = T, gq.N = 3 * inner, gq.K = d;
        gq.out = qkv.p, gq.bias = B.qkv_b.as<float>(), gq.rope = rope.as<float>(), gq.qn_w = B.qn.as<float>(), gq.kn_w = B.kn.as<float>();
        gq.eps = c_.eps, gq.inner = inner, gq.heads_per_rank = H, gq.rows_local = T;
        gemm_bf16(h.p, B.qkv_w.p, gq, Epi::qkv, s);
        const __nv_bfloat16* q = qkv.as<__nv_bfloat16>();
        AttnParams ap;
        ap.q = q, ap.k = q + H * 128, ap.v = q + 2 * H * 128, ap.row_stride = 3 * H * 128, ap.heads = H, ap.rows = T;
        ap.out = o.p, ap.out_row_stride = inner, ap.static_max = B.qk_bound;
        attention(ap, s);
        GemmParams go;
        go.M = T, go.N = d, go.K = inner;
        go.x = x, go.ldx = d, go.bias = B.out_b.as<float>(), go.mod = mod.as<float>(), go.mod_idx = mi, go.gate_slot = 2, go.dim = d;
        gemm_bf16(o.p, B.out_w.p, go, Epi::gate_resid, s);
        rp.w = B.norm2.as<float>(), rp.shift_slot = 3, rp.scale_slot = 4;
        rms_mod_rows(rp, s);
        GemmParams g1;
        g1.M = T, g1.N = 2 * F, g1.K = d, g1.out = qkv.p, g1.ldo = F, g1.bias = B.fc1_b.as<float>();
        gemm_bf16(h.p, B.fc1_w.p, g1, Epi::swiglu, s);
        GemmParams g2;
        g2.M = T, g2.N = d, g2.K = F;
        g2.x = x, g2.ldx = d, g2.bias = B.fc2_b.as<float>(), g2.mod = mod.as<float>(), g2.mod_idx = mi, g2.gate_slot = 5, g2.dim = d;
        gemm_bf16(qkv.p, B.fc2_w.p, g2, Epi::gate_resid, s);
    }
    RmsModParams fp;
    fp.x = x, fp.ldx = d, fp.rows = T, fp.d = d, fp.w = d_->refiner_norm.as<float>(), fp.mod = mod.as<float>(), fp.mod_idx = mi;
    fp.mod_slots = 6, fp.shift_slot = 0, fp.scale_slot = 1, fp.eps = c_.eps, fp.out_kind = RowOut::f32, fp.out = xn.p, fp.ldo = d;
    rms_mod_rows(fp, s);
    H3_CUDA(cudaMemcpyAsync(x, xn.p, size_t(T) * d * 4, cudaMemcpyDeviceToDevice, s));
    H3_CUDA(cudaStreamSynchronize(s)); // the temporaries are freed on return
}

void Model::emit_probe(const char* name, int layer, const float* dev, size_t n, bool rows)
{
    if (!probe_)
        return;
    std::vector<float> h(n);
    H3_CUDA(cudaMemcpyAsync(h.data(), dev, n * 4, cudaMemcpyDeviceToHost, stream_));
    H3_CUDA(cudaStreamSynchronize(stream_));
    if (rows && S_ > 0 && !d_->h_video_src.empty()) {
        const size_t w = n / size_t(S_), D = size_t(d_->grid.dense_rows);
        std::vector<float> packed(h.begin() + D * w, h.end());
        for (size_t i = 0; i < d_->h_video_src.size(); ++i)
            std::memcpy(&h[(D + d_->h_video_src[i]) * w], &packed[i * w], w * 4);
    }
    probe_(name, layer, h.data(), n);
}

void Model::step(const float* video, const float* audio, float t_video, float t_audio, float* out_video, float* out_audio, bool device_io)
{
    if (!begun_)
        throw CudaError("step before begin");
    NvtxRange step_range("h3.step");
    cudaStream_t s = stream_;
    const Layout& l = layout_;
    const int d = c_.dim, inner = c_.inner(), F = c_.ffn, td = c_.time_dim, L = c_.blocks;
    const int P = world_.size, Hp = c_.heads / P;
    const int T = l.text, C = l.cond_rows(), CA = l.cond_audio_rows(), A = l.audio_rows(), V = l.video_rows(), D = l.dense_rows();
    const int M = S_local_;
    launches_ = 0;
    stage_ms_.clear();

    // ---- noise levels: the video / text level, the audio level, the conditioning video level (max(t_video, 0.999)),
    // the reference audio level (1, clean)
    const float t_cond = std::max(t_video, 0.999f);
    std::vector<float> levels;
    auto level_of = [&](float t) {
        for (size_t i = 0; i < levels.size(); ++i)
            if (levels[i] == t)
                return int(i);
        levels.push_back(t);
        return int(levels.size() - 1);
    };
    const int lv_video = level_of(t_video);
    const int lv_audio = A - CA > 0 ? level_of(t_audio) : lv_video;
    const int lv_cond = C > 0 ? level_of(t_cond) : lv_video;
    const int lv_ref_audio = CA > 0 ? level_of(1.0f) : lv_video;
    const int U = int(levels.size());
    {
        // staged in pinned memory: [M] mod_idx, [M] lvl_idx, then [U][256] f32 embeddings at a 16-byte offset
        const size_t emb_off = (size_t(2) * M + 15) & ~size_t(15);
        const size_t need = emb_off + size_t(U) * 256 * 4;
        if (!d_->upload_done)
            H3_CUDA(cudaEventCreateWithFlags(&d_->upload_done, cudaEventDisableTiming));
        else
            H3_CUDA(cudaEventSynchronize(d_->upload_done)); // the previous step's copies have read the staging
        if (need > d_->pinned_bytes) {
            if (d_->pinned)
                H3_CUDA(cudaFreeHost(d_->pinned));
            d_->pinned = nullptr;
            H3_CUDA(cudaMallocHost(reinterpret_cast<void**>(&d_->pinned), need));
            d_->pinned_bytes = need;
        }
        uint8_t* midx = d_->pinned;
        uint8_t* lidx = d_->pinned + M;
        float* emb = reinterpret_cast<float*>(d_->pinned + emb_off);
        std::memset(midx, 0, size_t(2) * M);
        for (int i = 0; i < M && row0_ + i < S_; ++i) {
            const int g = row0_ + i;
            const int kind = d_->h_lvl_kind[g];
            const int lv = kind == 1 ? lv_audio : (kind == 2 ? lv_cond : (kind == 3 ? lv_ref_audio : lv_video));
            lidx[i] = uint8_t(lv);
            midx[i] = uint8_t(lv * 3 + d_->h_tags[g]);
        }
        H3_CUDA(cudaMemcpyAsync(d_->mod_idx.p, midx, M, cudaMemcpyHostToDevice, s));
        H3_CUDA(cudaMemcpyAsync(d_->lvl_idx.p, lidx, M, cudaMemcpyHostToDevice, s));
        if (c_.curve) {
            // pruned checkpoint: the curve adaln_t_table [1025][8] read at t * 1024 with linear interpolation
            // (tools/check_pruned_curve.py:66-70, the hypothesis the reference implements), [U][8]; in double, rounded
            // to float at the end (a float position would move the weight by an ulp of t * 1024, ~3e-5 near 341)
            const int K8 = c_.curve;
            const float* tab = d_->curve_table.data();
            for (int u = 0; u < U; ++u) {
                const double pos = std::min(std::max(double(levels[u]) * 1024.0, 0.0), 1024.0);
                const int i0 = std::min(int(std::floor(pos)), 1023);
                const double w = pos - double(i0);
                for (int k = 0; k < K8; ++k)
                    emb[u * K8 + k] = float((1.0 - w) * double(tab[i0 * K8 + k]) + w * double(tab[(i0 + 1) * K8 + k]));
            }
        } else {
            // sinusoidal embeddings [U][256]: cos half first, freq_i = exp(-ln(10000) * i / 128)
            for (int u = 0; u < U; ++u)
                for (int i = 0; i < 128; ++i) {
                    const float fr = float(std::exp(-std::log(10000.0) * i / 128.0));
                    const float a = levels[u] * fr;
                    emb[u * 256 + i] = float(std::cos(double(a)));
                    emb[u * 256 + 128 + i] = float(std::sin(double(a)));
                }
        }
        const size_t emb_bytes = size_t(U) * (c_.curve ? c_.curve : 256) * 4;
        d_->emb.ensure(emb_bytes);
        H3_CUDA(cudaMemcpyAsync(d_->emb.p, emb, emb_bytes, cudaMemcpyHostToDevice, s));
        H3_CUDA(cudaEventRecord(d_->upload_done, s));
    }

    // Timing: an event after each kernel class (from a pool reused across steps); stage i is the time between
    // events i - 1 and i, named by what ran in between ("h2d" and "d2h": the host copies of a step with host I/O).
    size_t ev_used = 0;
    auto mark = [&](const char* name) {
        if (!timing_)
            return;
        if (ev_used == d_->ev.size()) {
            cudaEvent_t e;
            H3_CUDA(cudaEventCreate(&e));
            d_->ev.push_back(e);
        }
        H3_CUDA(cudaEventRecord(d_->ev[ev_used++], s));
        stage_ms_.push_back({name, 0.f});
    };
    mark("start");

    // ---- inputs
    const float* dv = video;
    const float* da = audio;
    if (!device_io) {
        d_->in_video.ensure(size_t(std::max(V, 1)) * c_.video_patch * 4);
        d_->in_audio.ensure(size_t(std::max(A, 1)) * c_.audio_channels * 4);
        if (V)
            H3_CUDA(cudaMemcpyAsync(d_->in_video.p, video, size_t(V) * c_.video_patch * 4, cudaMemcpyHostToDevice, s));
        if (A)
            H3_CUDA(cudaMemcpyAsync(d_->in_audio.p, audio, size_t(A) * c_.audio_channels * 4, cudaMemcpyHostToDevice, s));
        dv = d_->in_video.as<float>();
        da = d_->in_audio.as<float>();
        mark("h2d");
    }

    // ---- time embedding and modulation
    d_->th.ensure(size_t(U) * d * 4);
    d_->temb.ensure(size_t(U) * td * 4);
    d_->tsilu.ensure(size_t(U) * td * 4);
    // With several ranks each computes the AdaLN projections of its share of the blocks (the weights stream from HBM
    // once per step in all) and an all-gather hands every rank all of them.
    const int nb = (L + P - 1) / P;
    const size_t block_mods = size_t(U) * 18 * d;
    d_->mods.ensure(size_t(nb) * P * block_mods * 4);
    d_->fmods.ensure(size_t(U) * 2 * d * 4);
    if (c_.curve) {
        // pruned checkpoint (curve_mods): every block's [18 d][8] projection of the curve point, fp32, no SiLU; tiny,
        // so every rank computes all blocks
        curve_mods(d_->ada_w.as<float>(), d_->ada_b.as<float>(), d_->emb.as<float>(), U, L, 18 * d, c_.curve, d_->mods.as<float>(), s);
        curve_mods(d_->fada_w.as<float>(), d_->fada_b.as<float>(), d_->emb.as<float>(), U, 1, 2 * d, c_.curve, d_->fmods.as<float>(), s);
        launches_ += 2;
    } else {
    gemv_f32(d_->t_in_w.as<float>(), d_->t_in_b.as<float>(), d_->emb.as<float>(), U, d, 256, Act::silu, d_->th.as<float>(), nullptr, s);
    gemv_f32(d_->t_out_w.as<float>(), d_->t_out_b.as<float>(), d_->th.as<float>(), U, td, d, Act::none, d_->temb.as<float>(),
             d_->tsilu.as<float>(), s);
    {
        const int b0 = std::min(L, world_.rank * nb), b1 = std::min(L, b0 + nb);
        float* mine = d_->mods.as<float>() + size_t(world_.rank) * nb * block_mods;
        if (b1 > b0)
            adaln_gemv(static_cast<const __nv_bfloat16*>(d_->ada_w.p) + size_t(b0) * 18 * d * td, d_->ada_b.as<float>() + size_t(b0) * 18 * d,
                       d_->tsilu.as<float>(), U, b1 - b0, 18 * d, td, mine, s);
        if (P > 1)
            H3_NCCL(ncclAllGather(mine, d_->mods.p, size_t(nb) * block_mods, ncclFloat32, d_->comm, s));
    }
    adaln_gemv(d_->fada_w.p, d_->fada_b.as<float>(), d_->tsilu.as<float>(), U, 1, 2 * d, td, d_->fmods.as<float>(), s);
    launches_ += 4;
    }
    mark("adaln");
    if (!c_.curve)
        emit_probe("temb", -1, d_->temb.as<float>(), size_t(U) * td);
    emit_probe("mod0", -1, d_->mods.as<float>(), size_t(U) * 18 * d);

    // ---- packed input x0 for this rank's rows [row0, row0 + M)
    float* x = d_->x.as<float>();
    H3_CUDA(cudaMemsetAsync(x, 0, size_t(M) * d * 4, s));
    const int r0 = row0_, r1 = std::min(S_, row0_ + M);
    auto overlap = [&](int a, int b, int& lo, int& hi) {
        lo = std::max(a, r0), hi = std::min(b, r1);
        return lo < hi;
    };
    int lo, hi;
    if (overlap(0, T, lo, hi))
        H3_CUDA(cudaMemcpyAsync(x + size_t(lo - r0) * d, d_->x_text.as<float>() + size_t(lo) * d, size_t(hi - lo) * d * 4,
                                cudaMemcpyDeviceToDevice, s));
    d_->pk_video.ensure(size_t(std::max(V, 1)) * c_.video_patch * 2);
    d_->pk_audio.ensure(size_t(std::max(A, 1)) * 64 * 2);
    if (C) {
        pack_bf16_rows(dv, C, c_.video_patch, d_->pk_video.p, c_.video_patch, s);
        ++launches_;
    }
    if (V - C) {
        // generated video rows gathered into the packed order
        pack_bf16_rows(dv + size_t(C) * c_.video_patch, V - C, c_.video_patch,
                       static_cast<__nv_bfloat16*>(d_->pk_video.p) + size_t(C) * c_.video_patch, c_.video_patch, s,
                       d_->video_src.as<int32_t>());
        ++launches_;
    }
    if (A) {
        pack_bf16_rows(da, A, c_.audio_channels, d_->pk_audio.p, 64, s);
        ++launches_;
    }
    auto proj = [&](const void* pk, int ld, int first_in, int model_row0, int n, const DevBuf& w, const DevBuf& b, int K) {
        int a, bnd;
        if (!overlap(model_row0, model_row0 + n, a, bnd))
            return;
        GemmParams g;
        g.M = bnd - a, g.N = d, g.K = K, g.lda = ld;
        g.out = x + size_t(a - r0) * d, g.ldo = d, g.bias = b.as<float>();
        const void* A0 = static_cast<const uint8_t*>(pk) + size_t(first_in + (a - model_row0)) * ld * 2;
        gemm_bf16(A0, w.p, g, Epi::f32, s);
        ++launches_;
    };
    for (const Segment& sg : d_->segs) {
        if (sg.role == 1 || sg.role == 4) // conditioning and generated video rows (the generated ones packed)
            proj(d_->pk_video.p, c_.video_patch, sg.input_row, sg.row0, sg.rows, d_->vp_w, d_->vp_b, c_.video_patch);
        else if (sg.role == 2 || sg.role == 3) // reference and generated audio rows
            proj(d_->pk_audio.p, 64, sg.input_row, sg.row0, sg.rows, d_->ap_w, d_->ap_b, 64);
    }
    mark("input");
    if (P == 1)
        emit_probe("x0", -1, x, size_t(S_) * d, true);

    // ---- blocks
    const bool sparse = sparse_ratio_ > 0.f && d_->sp.blocks != nullptr;
    const CubeGrid& grid = d_->grid;
    const uint8_t* midx = d_->mod_idx.as<uint8_t>();
    __nv_bfloat16* qkv = d_->qkv.as<__nv_bfloat16>();
    // With several ranks the Ulysses exchanges are fused into the q/k/v GEMM's and the attention's epilogues
    // (stores into the peers' receive buffers); a 4-byte all-reduce then serves as the barrier after each.
    const bool fused = P > 1 && d_->fused;
    auto barrier = [&]() {
        H3_NCCL(ncclAllReduce(d_->barrier_word.p, d_->barrier_word.p, 1, ncclInt32, ncclSum, d_->comm, s));
    };
    for (int bl = 0; bl < L; ++bl) {
        NvtxRange block_range("h3.block " + std::to_string(bl));
        Impl::Block& B = d_->blocks[bl];
        const float* mod = d_->mods.as<float>() + size_t(bl) * U * 18 * d;
        // attention half
        RmsModParams rp;
        rp.x = x, rp.ldx = d, rp.rows = M, rp.d = d, rp.w = B.norm1.as<float>(), rp.mod = mod, rp.mod_idx = midx;
        rp.mod_slots = 6, rp.shift_slot = 0, rp.scale_slot = 1, rp.eps = c_.eps;
        GemmParams gq;
        gq.M = M, gq.N = 3 * inner, gq.K = d;
        gq.out = qkv, gq.bias = B.qkv_b.as<float>(), gq.rope = d_->rope.as<float>(), gq.qn_w = B.qn.as<float>(),
        gq.kn_w = B.kn.as<float>(), gq.eps = c_.eps, gq.inner = inner, gq.heads_per_rank = Hp, gq.rows_local = M;
        if (fused) {
            // the epilogue stores each head group's rows straight into its owner's receive buffer over NVLink
            for (int r = 0; r < P; ++r)
                gq.peer_out[r] = d_->peer_qkv[r];
            gq.my_rank = world_.rank;
        }
        if (int8_ & kInt8Qkv) {
            rp.out_kind = RowOut::s8, rp.out = d_->hq.p, rp.ldo = d, rp.out_scale = d_->hs.as<float>();
            rms_mod_rows(rp, s);
            mark("norm");
            gq.a_scale = d_->hs.as<float>(), gq.b_scale = B.qkv_s.as<float>();
            gemm_s8(d_->hq.p, B.qkv_q.p, gq, Epi::qkv, s);
        } else {
            rp.out_kind = RowOut::bf16, rp.out = d_->h.p, rp.ldo = d;
            rms_mod_rows(rp, s);
            mark("norm");
            gemm_bf16(d_->h.p, B.qkv_w.p, gq, Epi::qkv, s);
        }
        launches_ += 2;
        mark("qkv");
        const __nv_bfloat16* qsrc = qkv;
        if (fused) {
            barrier(); // every rank's rows have landed in every receive buffer
            qsrc = d_->qkv_recv.as<__nv_bfloat16>();
            mark("a2a");
        } else if (P > 1) {
            const size_t chunk = size_t(M) * 3 * Hp * 128;
            H3_NCCL(ncclGroupStart());
            for (int r = 0; r < P; ++r) {
                H3_NCCL(ncclSend(qkv + r * chunk, chunk, ncclBfloat16, r, d_->comm, s));
                H3_NCCL(ncclRecv(d_->qkv_recv.as<__nv_bfloat16>() + r * chunk, chunk, ncclBfloat16, r, d_->comm, s));
            }
            H3_NCCL(ncclGroupEnd());
            qsrc = d_->qkv_recv.as<__nv_bfloat16>();
            mark("a2a");
        }
        AttnParams ap;
        ap.q = qsrc, ap.k = qsrc + Hp * 128, ap.v = qsrc + 2 * Hp * 128;
        ap.row_stride = 3 * Hp * 128, ap.heads = Hp, ap.rows = S_;
        ap.out = d_->o.p, ap.out_row_stride = Hp * 128;
        if (fused) {
            // the epilogue stores each row's output straight to the rank that owns the row
            for (int r = 0; r < P; ++r)
                ap.peer_out[r] = d_->peer_o[r];
            ap.rows_per_rank = M, ap.my_rank = world_.rank;
        }
        if (sparse) {
            // coarse pass (cube_pool, cube_scores, cube_topk, pass lists), then the sparse flash kernel
            const SparseBuffers& b = d_->sp;
            cube_pool(ap.q, ap.k, ap.row_stride, Hp, grid, b.mq, b.mk, s);
            cube_scores(b.mq, b.mk, Hp, grid.cubes(), b.scores, s);
            cube_topk(b.scores, Hp, grid, sparse_k(sparse_ratio_, grid.cubes()), sparse_local_, b.sel, b.nsel, b.kcap, s);
            build_passes(b.sel, b.nsel, b.kcap, Hp, grid, b.blocks, b.nblocks, b.q_rows, b.q_tiles, b.max_blocks, s);
            mark("select");
            ap.blocks = b.blocks, ap.nblocks = b.nblocks, ap.q_rows = b.q_rows, ap.q_tiles = b.q_tiles;
            ap.max_blocks = b.max_blocks, ap.grid = grid;
            ap.static_max = B.qk_bound;
            launches_ += 4 + attention(ap, s);
        } else {
            if (d_->attn_split_bytes) {
                ap.part_o = d_->attn_part.as<float>();
                ap.part_ml = ap.part_o + size_t(2) * S_ * Hp * 128;
            }
            ap.static_max = B.qk_bound;
            launches_ += attention(ap, s);
        }
        mark("attn");
        const void* oin = d_->o.p;
        GemmParams go;
        go.M = M, go.N = d, go.K = inner;
        if (fused) {
            barrier(); // every rank's head outputs for this rank's rows have landed
            oin = d_->o_recv.p;
            go.a_chunks = P, go.lda = Hp * 128, go.a_rows_stride = M;
            mark("a2a");
        } else if (P > 1) {
            const size_t chunk = size_t(M) * Hp * 128;
            H3_NCCL(ncclGroupStart());
            for (int r = 0; r < P; ++r) {
                H3_NCCL(ncclSend(d_->o.as<__nv_bfloat16>() + r * chunk, chunk, ncclBfloat16, r, d_->comm, s));
                H3_NCCL(ncclRecv(d_->o_recv.as<__nv_bfloat16>() + r * chunk, chunk, ncclBfloat16, r, d_->comm, s));
            }
            H3_NCCL(ncclGroupEnd());
            oin = d_->o_recv.p;
            go.a_chunks = P, go.lda = Hp * 128, go.a_rows_stride = M;
            mark("a2a");
        }
        go.x = x, go.ldx = d, go.bias = B.out_b.as<float>(), go.mod = mod, go.mod_idx = midx, go.gate_slot = 2, go.dim = d;
        if (int8_ & kInt8Out) {
            // quantised per row (across the chunks of every rank's heads), written as dense int8 rows
            quant_rows_i8_chunked(oin, M, inner, go.a_chunks, M, d_->hq.as<int8_t>(), d_->hs.as<float>(), s);
            go.a_chunks = 1, go.lda = 0, go.a_rows_stride = 0;
            go.a_scale = d_->hs.as<float>(), go.b_scale = B.out_s.as<float>();
            gemm_s8(d_->hq.p, B.out_q.p, go, Epi::gate_resid, s);
            launches_ += 2;
        } else {
            gemm_bf16(oin, B.out_w.p, go, Epi::gate_resid, s);
            launches_ += 1;
        }
        mark("out");
        // FFN half
        rp.w = B.norm2.as<float>(), rp.shift_slot = 3, rp.scale_slot = 4;
        GemmParams g1;
        g1.M = M, g1.N = 2 * F, g1.K = d, g1.out = qkv, g1.ldo = F, g1.bias = B.fc1_b.as<float>();
        if (int8_ & kInt8Fc1) {
            rp.out_kind = RowOut::s8, rp.out = d_->hq.p, rp.ldo = d, rp.out_scale = d_->hs.as<float>();
            rms_mod_rows(rp, s);
            mark("norm");
            g1.a_scale = d_->hs.as<float>(), g1.b_scale = B.fc1_s.as<float>();
            gemm_s8(d_->hq.p, B.fc1_q.p, g1, Epi::swiglu, s);
        } else {
            rp.out_kind = RowOut::bf16, rp.out = d_->h.p, rp.ldo = d;
            rms_mod_rows(rp, s);
            mark("norm");
            gemm_bf16(d_->h.p, B.fc1_w.p, g1, Epi::swiglu, s);
        }
        launches_ += 2;
        mark("fc1");
        GemmParams g2;
        g2.M = M, g2.N = d, g2.K = F;
        g2.x = x, g2.ldx = d, g2.bias = B.fc2_b.as<float>(), g2.mod = mod, g2.mod_idx = midx, g2.gate_slot = 5, g2.dim = d;
        if (int8_ & kInt8Fc2) {
            quant_rows_i8(qkv, F, M, F, d_->hq.as<int8_t>(), d_->hs.as<float>(), s);
            mark("quant");
            g2.a_scale = d_->hs.as<float>(), g2.b_scale = B.fc2_s.as<float>();
            gemm_s8(d_->hq.p, B.fc2_q.p, g2, Epi::gate_resid, s);
            launches_ += 2;
        } else {
            gemm_bf16(qkv, B.fc2_w.p, g2, Epi::gate_resid, s);
            launches_ += 1;
        }
        mark("fc2");
        if (probe_ && P == 1)
            emit_probe("block", bl, x, size_t(S_) * d, true);
    }

    // ---- final norm (per level shift and scale, no weight) and the heads
    float* xn = reinterpret_cast<float*>(d_->qkv.p);
    RmsModParams fp;
    fp.x = x, fp.ldx = d, fp.rows = M, fp.d = d, fp.w = nullptr, fp.mod = d_->fmods.as<float>(), fp.mod_idx = d_->lvl_idx.as<uint8_t>();
    fp.mod_slots = 2, fp.shift_slot = 0, fp.scale_slot = 1, fp.eps = c_.eps, fp.out_kind = RowOut::f32, fp.out = xn, fp.ldo = d;
    rms_mod_rows(fp, s);
    ++launches_;
    if (P == 1)
        emit_probe("norm_out", -1, xn, size_t(S_) * d, true);
    float* ro = d_->rows_out.as<float>();
    // rows_out: 128 floats a row (a video row's 96 values or an audio row's 32)
    auto head = [&](int first, int n, const DevBuf& w, const DevBuf& b, int N) {
        int a, bnd;
        if (!overlap(first, first + n, a, bnd))
            return;
        heads_f32(xn + size_t(a - r0) * d, d, bnd - a, w.as<float>(), b.as<float>(), N, d, ro + size_t(a - r0) * 128, 128, s);
        ++launches_;
    };
    for (const Segment& sg : d_->segs) {
        if (sg.role == 1 || sg.role == 4)
            head(sg.row0, sg.rows, d_->hv_w, d_->hv_b, c_.video_patch);
        else if (sg.role == 2 || sg.role == 3)
            head(sg.row0, sg.rows, d_->ha_w, d_->ha_b, c_.audio_channels);
    }
    const float* all = ro;
    if (P > 1) {
        H3_NCCL(ncclAllGather(ro, d_->rows_all.p, size_t(M) * 128, ncclFloat32, d_->comm, s));
        all = d_->rows_all.as<float>();
    }
    mark("final");
    // ---- outputs: video rows (conditioning rows first, then generated) and audio rows (reference rows first), in
    // the inputs' row order
    const cudaMemcpyKind kind = device_io ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
    for (const Segment& sg : d_->segs) {
        if (sg.role == 1)
            H3_CUDA(cudaMemcpy2DAsync(out_video + size_t(sg.input_row) * c_.video_patch, c_.video_patch * 4, all + size_t(sg.row0) * 128,
                                      128 * 4, c_.video_patch * 4, sg.rows, kind, s));
        else if (sg.role == 2 || sg.role == 3)
            H3_CUDA(cudaMemcpy2DAsync(out_audio + size_t(sg.input_row) * c_.audio_channels, c_.audio_channels * 4,
                                      all + size_t(sg.row0) * 128, 128 * 4, c_.audio_channels * 4, sg.rows, kind, s));
    }
    if (V - C) {
        // back to the layout's row order
        float* vo = device_io ? out_video + size_t(C) * c_.video_patch : d_->out_video_rows.as<float>();
        gather_rows_f32(all + size_t(D) * 128, 128, d_->video_dst.as<int32_t>(), V - C, c_.video_patch, vo, c_.video_patch, s);
        ++launches_;
        if (!device_io)
            H3_CUDA(cudaMemcpyAsync(out_video + size_t(C) * c_.video_patch, vo, size_t(V - C) * c_.video_patch * 4,
                                    cudaMemcpyDeviceToHost, s));
    }
    mark(device_io ? "output" : "d2h");
    if (timing_) {
        H3_CUDA(cudaStreamSynchronize(s));
        for (size_t i = 1; i < ev_used; ++i)
            H3_CUDA(cudaEventElapsedTime(&stage_ms_[i].second, d_->ev[i - 1], d_->ev[i]));
    }
    if (!device_io) {
        H3_CUDA(cudaStreamSynchronize(s));
        if (const uint32_t e = take_device_error(s))
            throw CudaError("device error " + std::to_string(e) + " during the step (a bounded wait ran out)");
    }
}

int Model::denoise(float* video, float* audio, const float* sigma_video, const float* sigma_audio, int points,
                   const std::function<bool(int, int)>& progress)
{
    if (!begun_)
        throw CudaError("denoise before begin");
    if (points < 2 || !sigma_video || !sigma_audio)
        throw CudaError("denoise: at least 2 schedule points for video and audio");
    for (int i = 0; i + 1 < points; ++i)
        if (!(sigma_video[i] > 0.f) || !(sigma_audio[i] > 0.f))
            throw CudaError("denoise: every schedule point but the last must be positive");
    const Layout& l = layout_;
    const size_t V = size_t(l.video_rows()), A = size_t(l.audio_rows()), C = size_t(l.cond_rows()), CA = size_t(l.cond_audio_rows());
    const size_t vn = V * c_.video_patch, an = A * c_.audio_channels;
    cudaStream_t s = stream_;
    d_->den_video.ensure(std::max<size_t>(vn, 1) * 4);
    d_->den_audio.ensure(std::max<size_t>(an, 1) * 4);
    d_->vel_video.ensure(std::max<size_t>(vn, 1) * 4);
    d_->vel_audio.ensure(std::max<size_t>(an, 1) * 4);
    float* xv = d_->den_video.as<float>();
    float* xa = d_->den_audio.as<float>();
    if (vn)
        H3_CUDA(cudaMemcpyAsync(xv, video, vn * 4, cudaMemcpyHostToDevice, s));
    if (an)
        H3_CUDA(cudaMemcpyAsync(xa, audio, an * 4, cudaMemcpyHostToDevice, s));
    const int steps = points - 1;
    int done = 0;
    for (int i = 0; i < steps; ++i) {
        NvtxRange denoise_range("h3.denoise " + std::to_string(i));
        const float tv = 1.0f - sigma_video[i], ta = 1.0f - sigma_audio[i];
        step(xv, xa, tv, ta, d_->vel_video.as<float>(), d_->vel_audio.as<float>(), true);
        euler_rows(xv + C * c_.video_patch, d_->vel_video.as<float>() + C * c_.video_patch, (V - C) * c_.video_patch, tv,
                   sigma_video[i], sigma_video[i + 1], s);
        euler_rows(xa + CA * c_.audio_channels, d_->vel_audio.as<float>() + CA * c_.audio_channels, (A - CA) * c_.audio_channels,
                   ta, sigma_audio[i], sigma_audio[i + 1], s);
        launches_ += 2;
        ++done;
        if (progress) {
            H3_CUDA(cudaStreamSynchronize(s));
            if (const uint32_t e = take_device_error(s))
                throw CudaError("device error " + std::to_string(e) + " during the denoising loop (a bounded wait ran out)");
            if (!progress(i + 1, steps))
                break;
        }
    }
    if (vn)
        H3_CUDA(cudaMemcpyAsync(video, xv, vn * 4, cudaMemcpyDeviceToHost, s));
    if (an)
        H3_CUDA(cudaMemcpyAsync(audio, xa, an * 4, cudaMemcpyDeviceToHost, s));
    H3_CUDA(cudaStreamSynchronize(s));
    if (const uint32_t e = take_device_error(s))
        throw CudaError("device error " + std::to_string(e) + " during the denoising loop (a bounded wait ran out)");
    return done;
}

std::vector<float> sigmas(int steps, float shift)
{
    if (steps < 2)
        throw CudaError("sigmas: at least 2 schedule points");
    if (!(shift > 0.f))
        throw CudaError("sigmas: the shift must be positive");
    // torch.linspace(1, 0, steps) in float: the first half counts up from 1, the second half down from 0 (so the
    // last point is exactly 0); then sigma -> shift * sigma / (1 + (shift - 1) * sigma), consecutive repeats dropped.
    const float delta = -1.0f / float(steps - 1);
    std::vector<float> out;
    for (int i = 0; i < steps; ++i) {
        const float lin = i < steps / 2 ? 1.0f + float(i) * delta : -(float(steps - 1 - i) * delta);
        const float num = shift * lin;
        const float den = 1.0f + (shift - 1.0f) * lin;
        const float v = num / den;
        if (out.empty() || out.back() != v)
            out.push_back(v);
    }
    return out;
}

Model::LoraResult Model::add_lora(const std::string& path, float scale, bool strict)
{
    const SafeTensors st(path);
    const int d = c_.dim, inner = c_.inner(), F = c_.ffn, td = c_.time_dim, L = c_.blocks;
    cudaStream_t s = stream_;
    LoraResult res;
    auto strip = [](std::string n) {
        for (const char* pre : {"base_model.model.", "diffusion_model.", "transformer."})
            if (n.rfind(pre, 0) == 0)
                n = n.substr(std::strlen(pre));
        return n;
    };
    auto ends_with = [](const std::string& a, const std::string& b) {
        return a.size() >= b.size() && a.compare(a.size() - b.size(), b.size(), b) == 0;
    };
    float file_alpha = 0.f;
    if (const auto it = st.metadata().find("alpha"); it != st.metadata().end())
        file_alpha = std::stof(it->second);
    enum Kind { kQ, kK, kV, kOut, kFc1, kFc2, kAda, kNone };
    struct Item {
        std::string a, b, prefix;
        Kind kind;
        int block, r, in, out;
        float sc;
    };
    // every adapter is checked (name, shapes) before any weight changes
    std::vector<Item> plan;
    for (const auto& [name, t] : st.tensors()) {
        std::string a_suffix;
        for (const char* suf : {".lora_A.weight", ".lora_down.weight"})
            if (ends_with(name, suf))
                a_suffix = suf;
        if (a_suffix.empty())
            continue;
        const std::string prefix = name.substr(0, name.size() - a_suffix.size());
        const std::string b_name = prefix + (a_suffix == ".lora_A.weight" ? ".lora_B.weight" : ".lora_up.weight");
        const std::string target = strip(prefix);
        if (!st.tensors().count(b_name))
            throw CudaError("add_lora: " + name + " has no matching " + b_name);
        // transformer_blocks.N.<module>
        int block = -1;
        std::string module;
        if (target.rfind("transformer_blocks.", 0) == 0) {
            const size_t dot = target.find('.', 19);
            if (dot != std::string::npos) {
                block = std::atoi(target.substr(19, dot - 19).c_str());
                module = target.substr(dot + 1);
            }
        }
        Kind kind = kNone;
        if (module == "attn.to_q") kind = kQ;
        else if (module == "attn.to_k") kind = kK;
        else if (module == "attn.to_v") kind = kV;
        else if (module == "attn.to_out.0") kind = kOut;
        else if (module == "ff.net.0.proj") kind = kFc1;
        else if (module == "ff.net.2") kind = kFc2;
        else if (module == "adaln_proj.linear") kind = kAda;
        if (kind == kNone || block < 0 || block >= L || (kind == kAda && c_.curve)) {
            // Known but not merged: the token refiner's targets, and the AdaLN projections of a pruned checkpoint
            // (its [18 d][8] projections of the curve are not the full model's [18 d][time_dim] ones the adapter is for).
            const bool known = target.rfind("token_refiner", 0) == 0 || (kind == kAda && c_.curve && block >= 0 && block < L);
            if (strict && !known)
                throw CudaError("add_lora: no H3 weight is named " + target);
            ++res.skipped;
            continue;
        }
        const SafeTensor& ta = t;
        const SafeTensor& tb = st.tensors().at(b_name);
        if (ta.shape.size() != 2 || tb.shape.size() != 2 || ta.shape[0] != tb.shape[1])
            throw CudaError("add_lora: " + prefix + ": lora_A [r][in] and lora_B [out][r] shapes disagree");
        const int r = int(ta.shape[0]), in = int(ta.shape[1]), out = int(tb.shape[0]);
        const int want_in = kind == kOut ? inner : kind == kFc2 ? F : kind == kAda ? td : d;
        const int want_out = kind <= kV ? inner : kind == kFc1 ? 2 * F : kind == kAda ? 18 * d : d;
        if (in != want_in || out != want_out || r <= 0)
            throw CudaError("add_lora: " + prefix + " is " + std::to_string(out) + " x " + std::to_string(in) + ", the weight " +
                            std::to_string(want_out) + " x " + std::to_string(want_in));
        float alpha = float(r);
        if (const auto it = st.tensors().find(prefix + ".alpha"); it != st.tensors().end())
            alpha = st.read_f32(prefix + ".alpha").at(0);
        else if (file_alpha > 0.f)
            alpha = file_alpha;
        plan.push_back(Item{name, b_name, prefix, kind, block, r, in, out, scale * alpha / float(r)});
    }
    for (const Item& it : plan) {
        const Kind kind = it.kind;
        const int block = it.block, r = it.r, in = it.in, out = it.out;
        // the adapter's row i lands on stored row map[i] of the target matrix
        std::vector<int32_t> map(out);
        for (int i = 0; i < out; ++i) {
            int row = i;
            if (kind == kK)
                row = inner + i;
            else if (kind == kV)
                row = 2 * inner + i;
            else if (kind == kFc1) {
                const int logical = i < F ? F + i : i - F; // Diffusers [value; gate] -> [gate; value]
                row = logical < F ? (logical / 128) * 256 + logical % 128 : ((logical - F) / 128) * 256 + 128 + (logical - F) % 128;
            } else if (kind == kAda) {
                const int c = (i / d) / 3, md = (i / d) % 3, j = i % d; // Diffusers (chunk, modality) -> (modality, chunk)
                row = block * 18 * d + (md * 6 + c) * d + j;
            }
            map[i] = row;
        }
        const std::vector<float> A = st.read_f32(it.a), Bm = st.read_f32(it.b);
        DevBuf dA, dB, dmap;
        dA.ensure(A.size() * 4), dB.ensure(Bm.size() * 4), dmap.ensure(map.size() * 4);
        H3_CUDA(cudaMemcpyAsync(dA.p, A.data(), A.size() * 4, cudaMemcpyHostToDevice, s));
        H3_CUDA(cudaMemcpyAsync(dB.p, Bm.data(), Bm.size() * 4, cudaMemcpyHostToDevice, s));
        H3_CUDA(cudaMemcpyAsync(dmap.p, map.data(), map.size() * 4, cudaMemcpyHostToDevice, s));
        Impl::Block& B = d_->blocks[block];
        DevBuf* w = nullptr;
        DevBuf *q = nullptr, *qs = nullptr;
        int rows_total = 0;
        bool i8 = false;
        switch (kind) {
        case kQ: case kK: case kV: w = &B.qkv_w, q = &B.qkv_q, qs = &B.qkv_s, rows_total = 3 * inner, i8 = int8_ & kInt8Qkv; break;
        case kOut: w = &B.out_w, q = &B.out_q, qs = &B.out_s, rows_total = d, i8 = int8_ & kInt8Out; break;
        case kFc1: w = &B.fc1_w, q = &B.fc1_q, qs = &B.fc1_s, rows_total = 2 * F, i8 = int8_ & kInt8Fc1; break;
        case kFc2: w = &B.fc2_w, q = &B.fc2_q, qs = &B.fc2_s, rows_total = d, i8 = int8_ & kInt8Fc2; break;
        default: w = &d_->ada_w; break;
        }
        if (!i8) {
            lora_merge(dB.as<float>(), dA.as<float>(), out, in, r, it.sc, dmap.as<int32_t>(), w->p, in, nullptr, nullptr, s);
        } else {
            // int8 rows: dequantised, merged into a bf16 copy, requantised per row (the rows the adapter covers)
            DevBuf tmp;
            tmp.ensure(size_t(rows_total) * in * 2);
            lora_merge(dB.as<float>(), dA.as<float>(), out, in, r, it.sc, dmap.as<int32_t>(), tmp.p, in, q->as<int8_t>(), qs->as<float>(), s);
            const int first = kind == kK ? inner : kind == kV ? 2 * inner : 0;
            quant_weight_rows(static_cast<__nv_bfloat16*>(tmp.p) + size_t(first) * in, out, in, q->as<int8_t>() + size_t(first) * in,
                              qs->as<float>() + first, s);
            H3_CUDA(cudaStreamSynchronize(s));
        }
        H3_CUDA(cudaStreamSynchronize(s)); // the host copies and temporaries go out of scope
        ++res.merged;
        res.rank = r;
    }
    return res;
}

} // namespace h3
