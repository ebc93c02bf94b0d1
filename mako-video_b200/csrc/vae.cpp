// The video VAE decoder on the step's kernels; see vae.hpp.
#include "vae.hpp"

#include "attention.cuh"
#include "common.hpp"
#include "gemm.cuh"
#include "rows.cuh"

#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <stdexcept>

namespace h3 {

namespace {

// Synthetic tensor ids of the decoder (fixed: the CPU oracle regenerates the same values from them).
enum : uint32_t {
    kVMean = 5001, kVStd, kVPqW, kVPqB, kVEmbW, kVEmbB, kVReg, kVLnW, kVLnB, kVProjW, kVProjB,
    kVBlockBase = 5100, kVBlockStride = 20,
};
enum : uint32_t { kVNorm1, kVQkvW, kVQkvB, kVOutW, kVOutB, kVScale1, kVNorm2, kVFc1W, kVFc1B, kVFc2W, kVFc2B, kVScale2 };

constexpr float kStd = 0.02f;

} // namespace

std::vector<int> vae_tile_starts(int n, int tile, int overlap)
{
    if (n <= 0 || tile <= 0 || overlap < 0 || overlap >= tile)
        throw std::invalid_argument("vae tiles: bad sizes");
    if (n <= tile)
        return {0};
    const int k = (n - overlap + (tile - overlap) - 1) / (tile - overlap);
    const int slack = k * tile - n, gaps = k - 1;
    std::vector<int> s(k, 0);
    for (int g = 0; g < gaps; ++g)
        s[g + 1] = s[g] + tile - (slack / gaps + (g < slack % gaps ? 1 : 0));
    return s;
}

std::vector<float> vae_rope_table(int frames, int th, int tw, int specials)
{
    const int T = frames * th * tw + specials;
    std::vector<float> t(size_t(T) * 48, 0.f);
    double inv[8];
    for (int k = 0; k < 8; ++k)
        inv[k] = 1.0 / std::pow(100.0, double(2 * k) / 16.0);
    const double two_pi = 6.283185307179586;
    for (int r = 0; r < T; ++r) {
        double coord[3] = {0.0, 0.0, 0.0}; // the special tokens sit at the origin
        if (r >= specials) {
            const int v = r - specials, f = v / (th * tw), y = (v / tw) % th, x = v % tw;
            coord[0] = -1.0 + 2.0 * f / frames, coord[1] = -1.0 + 2.0 * y / th, coord[2] = -1.0 + 2.0 * x / tw;
        }
        for (int a = 0; a < 3; ++a)
            for (int k = 0; k < 8; ++k) {
                const float ang = float(coord[a] * two_pi) * float(inv[k]);
                t[(size_t(r) * 24 + a * 8 + k) * 2] = float(std::cos(double(ang)));
                t[(size_t(r) * 24 + a * 8 + k) * 2 + 1] = float(std::sin(double(ang)));
            }
    }
    return t;
}

VideoDecoder::VideoDecoder(const VaeConfig& c, uint64_t seed, int device) : c_(c), device_(device)
{
    if (c.dim <= 0 || c.dim % 256 || c.heads * VaeConfig::head_dim != c.dim || c.ffn % 256 || c.blocks <= 0 || c.channels <= 0 ||
        c.channels > 32 || c.registers < 0 || c.clip <= 0 || c.tile <= 0 || c.overlap < 0 || c.overlap * 2 > c.tile)
        throw std::invalid_argument("vae config: dim a multiple of 256 = heads x 64, ffn a multiple of 256, 1-32 channels, "
                                    "overlap at most half a tile");
    H3_CUDA(cudaSetDevice(device));
    H3_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    const int d = c.dim, F = c.ffn, C = c.channels, kin = VaeConfig::kin;
    cudaStream_t s = stream_;
    auto fill = [&](DevBuf& b, size_t n, bool bf16, uint32_t id, float mean, float sd) {
        b.ensure(n * (bf16 ? 2 : 4));
        fill_synthetic(b.p, bf16 ? 1 : 0, n, seed, id, mean, sd, s);
    };
    fill(mean_, C, false, kVMean, 0.f, 0.1f);
    fill(std_, C, false, kVStd, 1.f, 0.1f);
    fill(pq_w_, size_t(C) * C, false, kVPqW, 0.f, 0.2f);
    fill(pq_b_, C, false, kVPqB, 0.f, kStd);
    {
        // [d][C] bf16, placed in [d][kin] with the padding columns zero
        DevBuf tmp;
        fill(tmp, size_t(d) * C, true, kVEmbW, 0.f, 0.2f);
        emb_w_.ensure(size_t(d) * kin * 2);
        H3_CUDA(cudaMemcpy2DAsync(emb_w_.p, kin * 2, tmp.p, size_t(C) * 2, size_t(C) * 2, d, cudaMemcpyDeviceToDevice, s));
        H3_CUDA(cudaStreamSynchronize(s));
    }
    fill(emb_b_, d, false, kVEmbB, 0.f, kStd);
    fill(registers_, size_t(std::max(c.registers, 1)) * d, false, kVReg, 0.f, 1.f);
    fill(ln_w_, d, false, kVLnW, 1.f, kStd);
    fill(ln_b_, d, false, kVLnB, 0.f, kStd);
    fill(proj_w_, size_t(c.pix()) * d, true, kVProjW, 0.f, kStd);
    fill(proj_b_, c.pix(), false, kVProjB, 0.f, kStd);
    blocks_.resize(c.blocks);
    for (int l = 0; l < c.blocks; ++l) {
        Block& B = blocks_[l];
        const uint32_t base = kVBlockBase + kVBlockStride * uint32_t(l);
        fill(B.norm1, d, false, base + kVNorm1, 1.f, kStd);
        fill(B.qkv_w, size_t(3) * d * d, true, base + kVQkvW, 0.f, kStd);
        fill(B.qkv_b, size_t(3) * d, false, base + kVQkvB, 0.f, kStd);
        fill(B.out_w, size_t(d) * d, true, base + kVOutW, 0.f, kStd);
        fill(B.out_b, d, false, base + kVOutB, 0.f, kStd);
        fill(B.norm2, d, false, base + kVNorm2, 1.f, kStd);
        {
            // stored [gate; value]; regrouped into 128-row [gate g; value g] pairs for the fused SwiGLU epilogue
            DevBuf tw, tb;
            fill(tw, size_t(2) * F * d, true, base + kVFc1W, 0.f, kStd);
            fill(tb, size_t(2) * F, false, base + kVFc1B, 0.f, kStd);
            B.fc1_w.ensure(size_t(2) * F * d * 2);
            B.fc1_b.ensure(size_t(2) * F * 4);
            interleave_gate_value(tw.p, F, d, B.fc1_w.p, s);
            interleave_gate_value_f32(tb.as<float>(), F, B.fc1_b.as<float>(), s);
            H3_CUDA(cudaStreamSynchronize(s));
        }
        fill(B.fc2_w, size_t(d) * F, true, base + kVFc2W, 0.f, kStd);
        fill(B.fc2_b, d, false, base + kVFc2B, 0.f, kStd);
        // modulation table [6][d] of the step's row kernels: shift and scale 0 (plain weighted RMS norms), the
        // residual scales as the gates of slots 2 and 5
        B.mods.ensure(size_t(6) * d * 4);
        fill_synthetic(B.mods.as<float>() + size_t(2) * d, 0, d, seed, base + kVScale1, 0.1f, kStd, s);
        fill_synthetic(B.mods.as<float>() + size_t(5) * d, 0, d, seed, base + kVScale2, 0.1f, kStd, s);
    }
    H3_CUDA(cudaStreamSynchronize(s));
}

VideoDecoder::~VideoDecoder()
{
    if (stream_) {
        cudaSetDevice(device_);
        cudaStreamSynchronize(stream_);
        cudaStreamDestroy(stream_);
    }
}

void VideoDecoder::run_clip(const float* lat, int h, int w)
{
    const int d = c_.dim, F = c_.ffn, C = c_.channels, kin = VaeConfig::kin, H = c_.heads;
    cudaStream_t s = stream_;
    launches_ = 0;
    const std::vector<int> ys = vae_tile_starts(h, c_.tile, c_.overlap), xs = vae_tile_starts(w, c_.tile, c_.overlap);
    VaeTiles t;
    t.frames = c_.clip, t.h = h, t.w = w;
    t.th = std::min(c_.tile, h), t.tw = std::min(c_.tile, w);
    t.tiles_y = int(ys.size()), t.tiles_x = int(xs.size());
    t.R = c_.registers + 1;
    t.T = c_.clip * t.th * t.tw + t.R;
    const int M = t.tiles() * t.T;
    std::vector<int> st(ys);
    st.insert(st.end(), xs.begin(), xs.end());
    starts_.ensure(st.size() * 4);
    H3_CUDA(cudaMemcpyAsync(starts_.p, st.data(), st.size() * 4, cudaMemcpyHostToDevice, s));
    t.y0 = starts_.as<int>(), t.x0 = starts_.as<int>() + ys.size();
    if (rope_key_[0] != c_.clip || rope_key_[1] != t.th || rope_key_[2] != t.tw) {
        const std::vector<float> r = vae_rope_table(c_.clip, t.th, t.tw, t.R);
        rope_.release();
        rope_.ensure(r.size() * 4);
        H3_CUDA(cudaMemcpyAsync(rope_.p, r.data(), r.size() * 4, cudaMemcpyHostToDevice, s));
        H3_CUDA(cudaStreamSynchronize(s)); // the host table goes out of scope
        rope_key_[0] = c_.clip, rope_key_[1] = t.th, rope_key_[2] = t.tw;
    }
    inp_.ensure(size_t(M) * kin * 2);
    x_.ensure(size_t(M) * d * 4);
    h_.ensure(size_t(M) * d * 2);
    qkv_.ensure(std::max(size_t(M) * 3 * d * 2, size_t(M) * c_.pix() * 4));
    o_.ensure(size_t(M) * d * 2);
    ffn_.ensure(size_t(M) * F * 2);
    midx_.ensure(size_t(M));
    canvas_.ensure(size_t(c_.clip) * VaeConfig::patch_t * h * VaeConfig::patch * w * VaeConfig::patch * 3 * 4);

    // tokens: the voxels' inputs, their embedding, the register and zero tokens
    H3_CUDA(cudaMemsetAsync(inp_.p, 0, size_t(M) * kin * 2, s));
    vae_inputs(lat, C, t, mean_.as<float>(), std_.as<float>(), pq_w_.as<float>(), pq_b_.as<float>(), inp_.p, kin, s);
    GemmParams ge;
    ge.M = M, ge.N = d, ge.K = kin, ge.out = x_.p, ge.ldo = d, ge.bias = emb_b_.as<float>();
    gemm_bf16(inp_.p, emb_w_.p, ge, Epi::f32, s);
    vae_special_rows(x_.as<float>(), d, t, registers_.as<float>(), s);
    launches_ += 3;

    for (const Block& B : blocks_) {
        RmsModParams rp;
        rp.x = x_.as<float>(), rp.ldx = d, rp.rows = M, rp.d = d, rp.w = B.norm1.as<float>(), rp.mod = B.mods.as<float>();
        rp.mod_idx = nullptr, rp.mod_slots = 6, rp.shift_slot = 0, rp.scale_slot = 1, rp.eps = c_.eps;
        rp.out_kind = RowOut::bf16, rp.out = h_.p, rp.ldo = d;
        rms_mod_rows(rp, s);
        GemmParams gq;
        gq.M = M, gq.N = 3 * d, gq.K = d, gq.out = qkv_.p, gq.ldo = 3 * d, gq.bias = B.qkv_b.as<float>();
        gemm_bf16(h_.p, B.qkv_w.p, gq, Epi::bf16, s);
        vae_heads(qkv_.p, M, H, t.T, rope_.as<float>(), c_.eps, s);
        AttnParams ap;
        const __nv_bfloat16* q = qkv_.as<__nv_bfloat16>();
        ap.q = q, ap.k = q + d, ap.v = q + 2 * d, ap.row_stride = 3 * d, ap.heads = H, ap.rows = M, ap.head_dim = VaeConfig::head_dim;
        ap.seg_rows = t.T, ap.seg_stride = t.T, ap.out = o_.p, ap.out_row_stride = d, ap.scale = 0.125f;
        ap.static_max = qk_score_bound(1.f, 1.f, VaeConfig::head_dim); // q and k RMS-normed without weights
        launches_ += attention(ap, s);
        GemmParams go;
        go.M = M, go.N = d, go.K = d, go.x = x_.as<float>(), go.ldx = d, go.bias = B.out_b.as<float>(), go.mod = B.mods.as<float>();
        go.mod_idx = midx_.as<uint8_t>(), go.gate_slot = 2, go.dim = d;
        gemm_bf16(o_.p, B.out_w.p, go, Epi::gate_resid, s);
        rp.w = B.norm2.as<float>(), rp.shift_slot = 3, rp.scale_slot = 4;
        rms_mod_rows(rp, s);
        GemmParams g1;
        g1.M = M, g1.N = 2 * F, g1.K = d, g1.out = ffn_.p, g1.ldo = F, g1.bias = B.fc1_b.as<float>();
        gemm_bf16(h_.p, B.fc1_w.p, g1, Epi::swiglu, s);
        GemmParams g2;
        g2.M = M, g2.N = d, g2.K = F, g2.x = x_.as<float>(), g2.ldx = d, g2.bias = B.fc2_b.as<float>(), g2.mod = B.mods.as<float>();
        g2.mod_idx = midx_.as<uint8_t>(), g2.gate_slot = 5, g2.dim = d;
        gemm_bf16(ffn_.p, B.fc2_w.p, g2, Epi::gate_resid, s);
        launches_ += 7;
    }
    // layer norm, the patch projection, the tiles' pixels into the clip's canvas
    layer_norm_rows(x_.as<float>(), M, d, ln_w_.as<float>(), ln_b_.as<float>(), c_.eps, h_.p, s);
    GemmParams gp;
    gp.M = M, gp.N = c_.pix(), gp.K = d, gp.out = qkv_.p, gp.ldo = c_.pix(), gp.bias = proj_b_.as<float>();
    gemm_bf16(h_.p, proj_w_.p, gp, Epi::f32, s);
    vae_pixels(qkv_.as<float>(), t, canvas_.as<float>(), s);
    launches_ += 3;
}

void VideoDecoder::decode_clip(const float* latents, int h, int w, float* canvas, bool device_io)
{
    if (!latents || !canvas || h <= 0 || w <= 0)
        throw std::invalid_argument("vae decode_clip: null pointer or empty grid");
    H3_CUDA(cudaSetDevice(device_));
    const size_t in_bytes = size_t(c_.clip) * h * w * c_.channels * 4;
    const size_t out_bytes = size_t(c_.clip) * VaeConfig::patch_t * h * VaeConfig::patch * w * VaeConfig::patch * 3 * 4;
    const float* lat = latents;
    if (!device_io) {
        lat_.ensure(in_bytes);
        H3_CUDA(cudaMemcpyAsync(lat_.p, latents, in_bytes, cudaMemcpyHostToDevice, stream_));
        lat = lat_.as<float>();
    }
    run_clip(lat, h, w);
    H3_CUDA(cudaMemcpyAsync(canvas, canvas_.p, out_bytes, device_io ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, stream_));
    H3_CUDA(cudaStreamSynchronize(stream_));
    if (const uint32_t e = take_device_error(stream_))
        throw CudaError("device error " + std::to_string(e) + " during the decode (a bounded wait ran out)");
}

void VideoDecoder::decode(const float* latents, int frames, int h, int w, const std::function<void(int, const float*)>& sink)
{
    // video_vae.cpp:17-50: clips of 7 latent frames, 5 apart; 17 frames a clip after 3 of padding, the first 5 faded
    // in from the previous clip's last 5; the last clip's 5 after the loop
    constexpr int kClipLatents = 5, kPrePad = 3, kFade = 5;
    if (!latents || frames < c_.clip || (frames - 2) % kClipLatents || c_.clip != kClipLatents + 2 || h <= 0 || w <= 0)
        throw std::invalid_argument("vae decode: voxels [5 n + 2][h][w][channels] with clips of 7 latent frames");
    H3_CUDA(cudaSetDevice(device_));
    const int Hp = h * VaeConfig::patch, Wp = w * VaeConfig::patch;
    const size_t frame = size_t(Hp) * Wp * 3, voxels = size_t(h) * w * c_.channels;
    const int chunks = (frames - 2) / kClipLatents, per_clip = kClipLatents * VaeConfig::patch_t - kPrePad;
    const int pf = c_.clip * VaeConfig::patch_t;
    lat_.ensure(size_t(c_.clip) * voxels * 4);
    overlap_.ensure(size_t(kFade) * frame * 4);
    frames_out_.ensure(size_t(per_clip) * frame * 4);
    host_frames_.resize(size_t(per_clip) * frame);
    int emitted = 0;
    auto deliver = [&](int n) {
        H3_CUDA(cudaMemcpyAsync(host_frames_.data(), frames_out_.p, size_t(n) * frame * 4, cudaMemcpyDeviceToHost, stream_));
        H3_CUDA(cudaStreamSynchronize(stream_));
        if (const uint32_t e = take_device_error(stream_))
            throw CudaError("device error " + std::to_string(e) + " during the decode (a bounded wait ran out)");
        for (int k = 0; k < n; ++k)
            sink(emitted++, host_frames_.data() + size_t(k) * frame);
    };
    for (int ci = 0; ci < chunks; ++ci) {
        H3_CUDA(cudaMemcpyAsync(lat_.p, latents + size_t(ci) * kClipLatents * voxels, size_t(c_.clip) * voxels * 4, cudaMemcpyHostToDevice,
                                stream_));
        run_clip(lat_.as<float>(), h, w);
        vae_emit(canvas_.as<float>(), kPrePad, per_clip, ci > 0 ? overlap_.as<float>() : nullptr, kFade, Hp, Wp, frames_out_.as<float>(),
                 stream_);
        H3_CUDA(cudaMemcpyAsync(overlap_.p, canvas_.as<float>() + size_t(kClipLatents * VaeConfig::patch_t + kPrePad) * frame,
                                size_t(pf - kClipLatents * VaeConfig::patch_t - kPrePad) * frame * 4, cudaMemcpyDeviceToDevice, stream_));
        deliver(per_clip);
    }
    vae_emit(overlap_.as<float>(), 0, kFade, nullptr, kFade, Hp, Wp, frames_out_.as<float>(), stream_);
    deliver(kFade);
}

} // namespace h3
