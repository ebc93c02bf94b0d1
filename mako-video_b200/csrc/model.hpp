// The H3 transformer step on one B200 (or one rank of a sequence-parallel group): weights resident in HBM, the
// packed sequence's layout, and the step that turns the noisy video and audio rows into their velocities.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "attention.cuh"
#include "sparse.cuh"

namespace h3 {

struct Config {
    int dim = 5120, heads = 40, ffn = 13824, blocks = 48, time_dim = 2560;
    int text_dim = 5120, video_patch = 96, audio_channels = 32;
    float eps = 1e-6f;
    int refiner = 2; // token refiner blocks over the text rows (begin); 0 skips the refiner
    int curve = 0;   // 0: full time embedder + AdaLN; 8: pruned checkpoint (adaln_t_table curve, [18 d][8] projections)
    int inner() const { return heads * 128; }
};

// The packed sequence [text | conditioning video | audio | generated video] of one request
// (mirrors the reference's H3::Layout; references are not supported).
// A reference block of a ref2va layout (H3::Layout::Reference, src/video/engine.cpp:604-616): a picture (one latent
// frame of h x w latents), a video (`frames` latent frames of h x w, with `audio` soundtrack latents or none) or a
// soundtrack alone (`audio` latents).
struct LayoutRef {
    enum Kind : int { kImage = 0, kVideo = 1, kAudio = 2 };
    int kind = kImage;
    int frames = 0, h = 0, w = 0, audio = 0;
    int visual_rows() const { return kind == kAudio ? 0 : (kind == kImage ? 1 : frames) * (h / 2) * (w / 2); }
    int audio_rows() const { return kind == kImage ? 0 : 2 * audio; }
};

// The packed sequence [text | keyframe rows or reference blocks | audio | generated video].
struct Layout {
    int text = 0;              // text rows T
    int frames = 0, h = 0, w = 0; // generated video: latent frames and latent height / width (2x2 patches a row)
    int audio = 0;             // audio latents per channel (rows = 2 * audio: left channel then right)
    int cond_frames = 0;       // keyframe latent frames (each h/2 * w/2 rows at t = 0.999), ahead of the audio rows
    std::vector<uint8_t> cond_last; // per keyframe: anchored at the last generated frame (else the first)
    std::vector<uint8_t> text_tags; // per text row: modality tag (1 text, 0 video); empty: all text
    std::vector<LayoutRef> refs;    // reference blocks in reading order (ref2va)
    int patch_rows() const { return (h / 2) * (w / 2); }
    // conditioning video rows: keyframes and the references' pictures and videos (the first rows of the video input)
    int cond_rows() const
    {
        int n = cond_frames * patch_rows();
        for (const LayoutRef& r : refs)
            n += r.visual_rows();
        return n;
    }
    // conditioning audio rows: the references' soundtracks (the first rows of the audio input)
    int cond_audio_rows() const
    {
        int n = 0;
        for (const LayoutRef& r : refs)
            n += r.audio_rows();
        return n;
    }
    int video_rows() const { return cond_rows() + frames * patch_rows(); } // conditioning + generated
    int audio_rows() const { return cond_audio_rows() + 2 * audio; }
    int rows() const { return text + video_rows() + audio_rows(); }
    int dense_rows() const { return rows() - frames * patch_rows(); } // every row before the generated video
};

// Per-row metadata of a layout (the reference's H3::rows): rotary positions (t, h, w) in double, modality tag
// (0 video, 1 text, 2 audio) and role (0 text, 1 reference video, 2 reference audio, 3 audio, 4 video).
struct Rows {
    std::vector<double> pos; // [S][3]
    std::vector<uint8_t> tags, roles;
};
Rows layout_rows(const Layout& l);

// Runs of rows with one role, in sequence order, and where each run's rows come from in the step's inputs: video
// roles (1, 4) from the video rows, audio roles (2, 3) from the audio rows, in order (input_row -1 for text).
struct Segment {
    int row0 = 0, rows = 0, role = 0, input_row = -1;
};
std::vector<Segment> layout_segments(const Layout& l);

// The sampler's noise schedule (Engine::sigmas, src/video/engine.cpp:71-88): `steps` points from 1 to 0 spaced as
// torch.linspace computes them in float, shifted by s x / (1 + (s - 1) x), consecutive repeats dropped.
std::vector<float> sigmas(int steps, float shift);

// The rotary frequencies: 16 per axis, base 10000 (1 / 10000^(2i/32) in float).
void rope_inv_freq(float out[16]);
// Per-row (cos, sin) of the 48 rotary angles (16 per axis, angle = float(pos) * inv_freq in float).
std::vector<float> rope_table(const Rows& r);

struct World {
    int rank = 0, size = 1;
    uint8_t nccl_id[128] = {};
};

using Probe = std::function<void(const std::string& name, int layer, const float* data, size_t n)>;

enum Int8Mask : uint32_t { kInt8Qkv = 1, kInt8Out = 2, kInt8Fc1 = 4, kInt8Fc2 = 8 };
// "none", "all" or a comma list of qkv, out, fc1, fc2; false when the text is not one of these.
bool parse_int8(const std::string& s, uint32_t& mask);

// One named weight of the model in its logical layout (as a checkpoint stores it): fc1 [gate; value] rows, q/k/v
// stacked q, k, v, the audio projection 32 inputs wide. Its name in a checkpoint, shape, element type, and the tensor
// id and distribution of the synthetic generator.
struct WeightSpec {
    std::string name;
    std::vector<int64_t> shape;
    bool bf16 = false;
    uint32_t id = 0;
    float mean = 0.f, stdev = 0.02f;
    int owner = 0;  // 0 the model, 1 a block, 2 a token refiner block
    int index = -1; // the block or refiner block
    uint64_t count() const
    {
        uint64_t n = 1;
        for (int64_t v : shape)
            n *= uint64_t(v);
        return n;
    }
};

// Every weight of a model of this shape, in the order they are set up and saved.
std::vector<WeightSpec> weight_specs(const Config& c);

// Writes a checkpoint for a model of shape c in this build's layout (its names, stacked q/k/v, the model's element
// types) from the checkpoint at `src` read through `renames` / `interleaved` as CheckpointWeights reads it. Host only.
// layout_given: the caller stated the source's q/k/v layout; without it a source file that holds q/k/v tensors but
// no qkv_layout metadata is refused (the shapes cannot tell interleaved from stacked rows).
void convert_checkpoint(const Config& c, const std::string& src, const std::string& dst, std::map<std::string, std::string> renames,
                        bool interleaved, bool layout_given);

// Where a model's weights come from: spec's values, in its logical layout and element type, written to device memory.
class WeightSource {
public:
    virtual ~WeightSource() = default;
    virtual void get(const WeightSpec& spec, void* dst, cudaStream_t s) = 0;
};

// Random-init weights: value i of a tensor = mean + stdev * a hash of (seed, tensor id, i) (fill_synthetic).
class SyntheticWeights : public WeightSource {
public:
    explicit SyntheticWeights(uint64_t seed) : seed_(seed) {}
    void get(const WeightSpec& spec, void* dst, cudaStream_t s) override;

private:
    uint64_t seed_;
};

// A checkpoint: one safetensors file, or a directory of them. Tensors are found by the names weight_specs gives,
// checked against the expected shape, and converted to the weight's element type (BF16, F16 or F32 sources). A file
// whose metadata says qkv_layout = interleaved stores each head's q, k and v rows together ([q_h; k_h; v_h] for head
// h), as the reference's shards do (docs/architecture.md:62-63); they are stacked q, k, v at load (its upload_qkv).
class CheckpointWeights : public WeightSource {
public:
    // renames: this build's name -> the checkpoint's, for checkpoints that name tensors otherwise (a name not in the
    // map is looked up as it is); interleaved: treat every file's q/k/v as interleaved, whatever its metadata says.
    explicit CheckpointWeights(const std::string& path, std::map<std::string, std::string> renames = {}, bool interleaved = false);
    ~CheckpointWeights() override;
    void get(const WeightSpec& spec, void* dst, cudaStream_t s) override;
    // spec's values in its logical layout and element type, in host memory (what get uploads).
    std::vector<unsigned char> host(const WeightSpec& spec) const;
    // The first problem a model of shape c would meet loading this checkpoint ("" if none): a missing tensor or a
    // shape that disagrees. Host only.
    std::string check(const Config& c) const;
    // A file holding one of c's q/k/v tensors whose metadata does not say its qkv_layout ("" if none).
    std::string untagged_qkv_file(const Config& c) const;

private:
    struct Files;
    std::unique_ptr<Files> f_;
};

class Model {
public:
    // Weights from `src` (synthetic or a checkpoint); the int8_mask's projections are quantised per row at load.
    Model(const Config& c, WeightSource& src, uint32_t int8_mask, const World& world);
    // Synthetic weights from `seed` (every value a hash of seed, tensor and index; see fill_synthetic).
    Model(const Config& c, uint64_t seed, uint32_t int8_mask, const World& world);
    ~Model();
    Model(const Model&) = delete;
    Model& operator=(const Model&) = delete;

    void set_sparse(float ratio, int local);
    void set_probe(Probe p) { probe_ = std::move(p); }
    // Caches the text rows (condition_proj of the text embeddings [T][text_dim], then the token refiner) and the
    // layout's row tables.
    void begin(const float* text, int T, const Layout& l);
    // One forward: video [V][96] and audio [A][32] rows (host or device memory) to velocities of the same shapes.
    // With `device_io` the pointers are device pointers and the step stays on `stream` (no host synchronisation
    // beyond the error check).
    void step(const float* video, const float* audio, float t_video, float t_audio, float* out_video, float* out_audio,
              bool device_io = false);
    // The denoising loop on the device (Engine::denoise's step loop): `points` schedule points give points - 1
    // steps; step i runs the forward at t = 1 - sigma[i] and moves the generated rows (video rows past the
    // conditioning rows, audio rows past the reference soundtracks) by Euler to sigma[i + 1]. video [V][96] and
    // audio [A][32] are host memory, read at the start and overwritten with the final sample; the conditioning rows
    // are unchanged. `progress(i + 1, steps)` runs on the host after each step's work has finished; a false return
    // stops the loop there (the sample so far is still written back). Returns the steps run.
    int denoise(float* video, float* audio, const float* sigma_video, const float* sigma_audio, int points,
                const std::function<bool(int, int)>& progress);

    // LoRA merge at load (H3::add_lora, src/video/engine.cpp:114; docs/architecture.md:108-116): a safetensors file
    // of Diffusers-named adapters (transformer_blocks.N.attn.to_q / to_k / to_v / to_out.0, ff.net.0.proj, ff.net.2,
    // adaln_proj.linear; X.lora_A.weight [r][in], X.lora_B.weight [out][r]; alpha from X.alpha or the file's
    // "alpha" metadata, else r) merged as W += scale * alpha / r * B A into the bf16 matrices, or into the int8 rows
    // by requantizing them. Diffusers orders fc1 [value; gate] (this build [gate; value]) and the AdaLN rows
    // (chunk, modality) (this build (modality, chunk)); the adapter's rows are permuted to match. The token refiner's
    // targets (its Diffusers module names are not documented in the reference) are skipped and counted; with
    // `strict`, any other unknown name is an error.
    struct LoraResult {
        int merged = 0, skipped = 0, rank = 0;
    };
    LoraResult add_lora(const std::string& path, float scale, bool strict);

    // Writes every weight to a safetensors file under the names of weight_specs, in the logical layout (metadata
    // qkv_layout = stacked), such that a model created from it is this one. bf16 models only (the int8 rows replace
    // the bf16 ones).
    void save(const std::string& path);

    const Config& config() const { return c_; }
    const Layout& layout() const { return layout_; }
    int rows() const { return S_; }
    cudaStream_t stream() const { return stream_; }
    // Kernel launches of the last step (this library's kernels, counted at launch).
    int last_launches() const { return launches_; }
    // Device timings (ms) of the last step by stage when timing is on.
    void set_timing(bool on) { timing_ = on; }
    const std::vector<std::pair<std::string, float>>& last_timing() const { return stage_ms_; }

private:
    struct Impl;
    std::unique_ptr<Impl> d_;
    Config c_;
    Layout layout_;
    World world_;
    int S_ = 0, S_local_ = 0, row0_ = 0;
    uint32_t int8_ = 0;
    float sparse_ratio_ = 0;
    int sparse_local_ = 1;
    Probe probe_;
    cudaStream_t stream_ = nullptr;
    int launches_ = 0;
    bool timing_ = false;
    std::vector<std::pair<std::string, float>> stage_ms_;
    bool begun_ = false;
    void alloc_activations();
    void size_sparse(); // the sparse attention's buffers for the layout's grid and the current ratio
    void refine_text(int T); // the token refiner over x_text (begin)
    void init(WeightSource& src); // the constructors' body: checks, stream, communicator, weights
    struct Target;
    Target locate(const WeightSpec& sp); // where a weight lives on the device
    void map_peers(); // the ranks' receive buffers, mapped into every rank (sequence-parallel, fused exchange)
    // Copies a device tensor to the host and hands it to the probe; with `rows` set it is [S][n / S] in the packed row
    // order and is handed over in the layout's row order.
    void emit_probe(const char* name, int layer, const float* dev, size_t n, bool rows = false);
};

} // namespace h3
