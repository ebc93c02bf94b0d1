// The C ABI (include/h3_c.h): status codes and a per-thread error message around the C++ runtime.
#include "h3_c.h"

#include "common.hpp"
#include "embed.cuh"
#include "gemm.cuh"
#include "model.hpp"
#include "rows.cuh"
#include "safetensors.hpp"
#include "sparse.cuh"

#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <functional>
#include <initializer_list>
#include <map>
#include <memory>
#include <sstream>
#include <string>

struct h3_model {
    std::unique_ptr<h3::Model> m;
    int device = 0;
    h3_probe_fn probe = nullptr;
    void* probe_user = nullptr;
};

namespace {

thread_local std::string g_error;

struct ArgError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct StateError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct DeviceError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

template <class F>
int guarded(F&& f)
{
    try {
        f();
        g_error.clear();
        return H3_OK;
    } catch (const ArgError& e) {
        g_error = e.what();
        return H3_ERR_ARG;
    } catch (const StateError& e) {
        g_error = e.what();
        return H3_ERR_STATE;
    } catch (const DeviceError& e) {
        g_error = e.what();
        return H3_ERR_DEVICE;
    } catch (const std::invalid_argument& e) {
        g_error = e.what();
        return H3_ERR_ARG;
    } catch (const h3::CudaError& e) {
        g_error = e.what();
        const std::string w = e.what();
        if (w.find("device error") != std::string::npos)
            return H3_ERR_DEVICE;
        if (w.find("config") == 0 || w.find("world") == 0 || w.find("begin:") == 0 || w.find("gemm:") == 0 || w.find("add_lora:") == 0 ||
            w.find("sparse") != std::string::npos || w.find("attention:") == 0)
            return H3_ERR_ARG;
        return H3_ERR_CUDA;
    } catch (const std::exception& e) {
        g_error = e.what();
        return H3_ERR_CUDA;
    }
}

// The h3k_* kernel entry points take device-accessible memory only (device, managed, or mapped pinned host memory):
// a plain host pointer passed by mistake is refused here rather than faulting inside a kernel. Null is let through
// (each call checks its own required arguments).
void device_ptrs(const char* fn, std::initializer_list<const void*> ptrs)
{
    for (const void* p : ptrs)
        if (!h3::device_accessible(p))
            throw ArgError(std::string(fn) + ": a pointer argument is host memory the GPU cannot access");
}

h3::Layout to_layout(const h3_layout* l)
{
    if (!l)
        throw ArgError("layout: null");
    h3::Layout o;
    o.text = int(l->text), o.frames = int(l->frames), o.h = int(l->h), o.w = int(l->w), o.audio = int(l->audio);
    o.cond_frames = int(l->cond_frames);
    if (l->cond_last)
        o.cond_last.assign(l->cond_last, l->cond_last + l->cond_frames);
    if (l->text_tags)
        o.text_tags.assign(l->text_tags, l->text_tags + l->text);
    if (l->n_refs && !l->refs)
        throw ArgError("layout: n_refs without refs");
    for (uint32_t i = 0; i < l->n_refs; ++i) {
        const h3_layout_ref& r = l->refs[i];
        if (r.kind < H3_REF_IMAGE || r.kind > H3_REF_AUDIO)
            throw ArgError("layout: reference kind 0 picture, 1 video, 2 soundtrack");
        h3::LayoutRef x;
        x.kind = r.kind, x.frames = int(r.frames), x.h = int(r.h), x.w = int(r.w), x.audio = int(r.audio);
        if (x.kind == h3::LayoutRef::kImage)
            x.frames = 1, x.audio = 0;
        if (x.kind == h3::LayoutRef::kAudio)
            x.frames = x.h = x.w = 0;
        if (x.kind != h3::LayoutRef::kAudio && (x.h <= 0 || x.w <= 0 || x.h % 2 || x.w % 2 || x.frames <= 0))
            throw ArgError("layout: a reference picture or video needs frames and even latent sides");
        o.refs.push_back(x);
    }
    if (o.cond_frames > 0 && !o.refs.empty())
        throw ArgError("layout: keyframes or reference blocks, not both");
    if (o.h % 2 || o.w % 2)
        throw ArgError("layout: the latent height and width must be even");
    return o;
}

h3::Config to_config(const h3_config* cfg)
{
    h3::Config c;
    c.dim = int(cfg->dim), c.heads = int(cfg->heads), c.ffn = int(cfg->ffn), c.blocks = int(cfg->blocks);
    c.time_dim = int(cfg->time_dim), c.text_dim = int(cfg->text_dim), c.video_patch = int(cfg->video_patch);
    c.audio_channels = int(cfg->audio_channels), c.eps = cfg->eps, c.refiner = int(cfg->refiner_blocks);
    if (c.video_patch != 96 || c.audio_channels != 32)
        throw ArgError("h3_create: video_patch must be 96 and audio_channels 32");
    if (cfg->refiner_blocks > 2)
        throw ArgError("h3_create: at most 2 token refiner blocks (MiniMax-H3 has 2)");
    if (cfg->curve_dims != 0 && cfg->curve_dims != 8)
        throw ArgError("h3_create: curve_dims is 0 (full model) or 8 (pruned checkpoint)");
    c.curve = int(cfg->curve_dims);
    return c;
}

h3::CubeGrid to_grid(const h3k_cube_grid* g)
{
    if (!g || g->frames <= 0 || g->ph <= 0 || g->pw <= 0 || g->dense_rows < 0)
        throw ArgError("cube grid: bad sizes");
    h3::CubeGrid c;
    c.dense_rows = g->dense_rows, c.frames = g->frames, c.ph = g->ph, c.pw = g->pw;
    c.nct = (c.frames + 3) / 4, c.ncy = (c.ph + 3) / 4, c.ncx = (c.pw + 3) / 4;
    return c;
}

cudaStream_t st(void* s) { return static_cast<cudaStream_t>(s); }

void check_model(h3_model* m)
{
    if (!m || !m->m)
        throw ArgError("null model");
    H3_CUDA(cudaSetDevice(m->device));
}

// Scratch owned for the duration of one kernel-level call.
struct Scratch {
    std::vector<void*> ptrs;
    void* get(size_t bytes)
    {
        void* p = nullptr;
        H3_CUDA(cudaMalloc(&p, bytes ? bytes : 16));
        ptrs.push_back(p);
        return p;
    }
    ~Scratch()
    {
        for (void* p : ptrs)
            cudaFree(p);
    }
};

} // namespace

namespace h3 {
// For entry points defined in other translation units (noalloc.cu): runs f with the status mapping and error message
// every other entry point uses.
int run_guarded(const std::function<void()>& f) { return guarded(f); }
} // namespace h3

extern "C" {

const char* h3_last_error(void) { return g_error.c_str(); }

int h3_nccl_unique_id(uint8_t out[128])
{
    return guarded([&] {
        ncclUniqueId id;
        if (ncclGetUniqueId(&id) != ncclSuccess)
            throw h3::CudaError("ncclGetUniqueId failed");
        std::memcpy(out, &id, 128);
    });
}

int h3_parse_int8(const char* text, uint32_t* mask)
{
    return guarded([&] {
        uint32_t m = 0;
        if (!text || !mask || !h3::parse_int8(text, m))
            throw ArgError("int8: none, all, or a comma list of qkv, out, fc1, fc2");
        *mask = m;
    });
}

int h3_create(const h3_config* cfg, const char* weights, uint32_t int8_mask, float sparse_ratio, uint32_t sparse_local,
              const h3_world* world, int32_t device, h3_model** out)
{
    return guarded([&] {
        if (!cfg || !out || !weights)
            throw ArgError("h3_create: null argument");
        *out = nullptr;
        const std::string w = weights;
        if (int8_mask & ~15u)
            throw ArgError("h3_create: int8 mask bits are 1 qkv, 2 out, 4 fc1, 8 fc2");
        const h3::Config c = to_config(cfg);
        // the weights: synthetic, or a checkpoint whose names and shapes are checked before any device work
        std::unique_ptr<h3::WeightSource> src;
        if (w.rfind("synthetic:", 0) == 0) {
            src = std::make_unique<h3::SyntheticWeights>(std::stoull(w.substr(10)));
        } else {
            auto ck = std::make_unique<h3::CheckpointWeights>(w);
            const std::string problem = ck->check(c);
            if (!problem.empty())
                throw ArgError("h3_create: " + w + ": " + problem);
            src = std::move(ck);
        }
        h3::World wd;
        if (world) {
            wd.rank = world->rank, wd.size = world->size;
            std::memcpy(wd.nccl_id, world->nccl_id, 128);
        }
        H3_CUDA(cudaSetDevice(device));
        auto m = std::make_unique<h3_model>();
        m->device = device;
        m->m = std::make_unique<h3::Model>(c, *src, int8_mask, wd);
        m->m->set_sparse(sparse_ratio, int(sparse_local));
        *out = m.release();
    });
}

int h3_set_sparse(h3_model* m, float ratio, uint32_t local)
{
    return guarded([&] {
        check_model(m);
        m->m->set_sparse(ratio, int(local));
    });
}

int h3_begin(h3_model* m, const float* text, uint32_t text_rows, const h3_layout* layout)
{
    return guarded([&] {
        check_model(m);
        if (text_rows && !text)
            throw ArgError("h3_begin: null text");
        m->m->begin(text, int(text_rows), to_layout(layout));
    });
}

static void check_io(h3_model* m, uint64_t video_rows, uint64_t audio_rows)
{
    const h3::Layout& l = m->m->layout();
    if (video_rows != uint64_t(l.video_rows()) || audio_rows != uint64_t(l.audio_rows()))
        throw ArgError("h3_step: " + std::to_string(l.video_rows()) + " video rows and " + std::to_string(l.audio_rows()) +
                       " audio rows expected");
}

int h3_step(h3_model* m, const float* video, uint64_t video_rows, const float* audio, uint64_t audio_rows, float t_video, float t_audio,
            float* out_video, float* out_audio)
{
    return guarded([&] {
        check_model(m);
        if (m->m->rows() == 0)
            throw StateError("h3_step before h3_begin");
        check_io(m, video_rows, audio_rows);
        m->m->step(video, audio, t_video, t_audio, out_video, out_audio, false);
    });
}

int h3_step_device(h3_model* m, const float* video, uint64_t video_rows, const float* audio, uint64_t audio_rows, float t_video,
                   float t_audio, float* out_video, float* out_audio)
{
    return guarded([&] {
        check_model(m);
        if (m->m->rows() == 0)
            throw StateError("h3_step_device before h3_begin");
        check_io(m, video_rows, audio_rows);
        m->m->step(video, audio, t_video, t_audio, out_video, out_audio, true);
    });
}

int h3_add_lora(h3_model* m, const char* path, float scale, int32_t strict, uint32_t* merged, uint32_t* skipped)
{
    return guarded([&] {
        check_model(m);
        if (!path)
            throw ArgError("h3_add_lora: null path");
        h3::Model::LoraResult r;
        try {
            r = m->m->add_lora(path, scale, strict != 0);
        } catch (const h3::CudaError&) {
            throw;
        } catch (const std::runtime_error& e) { // the file's own problems (safetensors reader)
            throw ArgError(e.what());
        }
        if (merged)
            *merged = uint32_t(r.merged);
        if (skipped)
            *skipped = uint32_t(r.skipped);
    });
}

int h3_weight_specs(const h3_config* cfg, char* out, uint64_t cap, uint32_t* count)
{
    return guarded([&] {
        if (!cfg)
            throw ArgError("h3_weight_specs: null config");
        const std::vector<h3::WeightSpec> specs = h3::weight_specs(to_config(cfg));
        std::string text;
        for (const h3::WeightSpec& sp : specs) {
            text += sp.name + (sp.bf16 ? " BF16 " : " F32 ");
            for (size_t k = 0; k < sp.shape.size(); ++k)
                text += (k ? "x" : "") + std::to_string(sp.shape[k]);
            text += "\n";
        }
        if (out && cap) {
            const size_t n = std::min<size_t>(text.size(), cap - 1);
            std::memcpy(out, text.data(), n);
            out[n] = '\0';
        }
        if (count)
            *count = uint32_t(specs.size());
    });
}

int h3_convert_weights(const h3_config* cfg, const char* src, const char* dst, const char* renames)
{
    return guarded([&] {
        if (!cfg || !src || !dst)
            throw ArgError("h3_convert_weights: null argument");
        std::map<std::string, std::string> table;
        bool interleaved = false, layout_given = false;
        if (renames) {
            std::istringstream in(renames);
            std::string line;
            while (std::getline(in, line)) {
                std::istringstream ls(line);
                std::string a, b, extra;
                if (!(ls >> a) || a[0] == '#')
                    continue;
                if (!(ls >> b) || (ls >> extra))
                    throw ArgError("h3_convert_weights: a rename line is \"this_name source_name\", not \"" + line + "\"");
                if (a == "qkv_layout") {
                    if (b != "interleaved" && b != "stacked")
                        throw ArgError("h3_convert_weights: qkv_layout is interleaved or stacked");
                    interleaved = b == "interleaved";
                    layout_given = true;
                    continue;
                }
                table[a] = b;
            }
        }
        h3::convert_checkpoint(to_config(cfg), src, dst, std::move(table), interleaved, layout_given);
    });
}

int h3_save_weights(h3_model* m, const char* path)
{
    return guarded([&] {
        check_model(m);
        if (!path)
            throw ArgError("h3_save_weights: null path");
        m->m->save(path);
    });
}

int h3_check_weights(const h3_config* cfg, const char* path, char* message, uint64_t cap)
{
    return guarded([&] {
        if (!cfg || !path)
            throw ArgError("h3_check_weights: null argument");
        std::string problem;
        try {
            problem = h3::CheckpointWeights(path).check(to_config(cfg));
        } catch (const std::exception& e) {
            problem = e.what(); // a file that cannot be read is the problem to report
        }
        if (message && cap) {
            const size_t n = std::min<size_t>(problem.size(), cap - 1);
            std::memcpy(message, problem.data(), n);
            message[n] = '\0';
        }
        if (!problem.empty())
            throw ArgError("h3_check_weights: " + std::string(path) + ": " + problem);
    });
}

int h3_lora_inspect(const char* path, char* names, uint64_t cap, uint32_t* count, uint32_t* rank, float* alpha)
{
    return guarded([&] {
        if (!path)
            throw ArgError("h3_lora_inspect: null path");
        std::unique_ptr<h3::SafeTensors> st;
        try {
            st = std::make_unique<h3::SafeTensors>(path);
        } catch (const std::runtime_error& e) {
            throw ArgError(e.what());
        }
        std::string list;
        uint32_t n = 0, r = 0;
        for (const auto& [name, t] : st->tensors()) {
            for (const char* suf : {".lora_A.weight", ".lora_down.weight"}) {
                const std::string sfx(suf);
                if (name.size() < sfx.size() || name.compare(name.size() - sfx.size(), sfx.size(), sfx) != 0)
                    continue;
                std::string target = name.substr(0, name.size() - sfx.size());
                for (const char* pre : {"base_model.model.", "diffusion_model.", "transformer."})
                    if (target.rfind(pre, 0) == 0)
                        target = target.substr(std::strlen(pre));
                list += (n ? "\n" : "") + target;
                if (!n && !t.shape.empty())
                    r = uint32_t(t.shape[0]);
                ++n;
            }
        }
        if (names && cap) {
            const size_t k = std::min<size_t>(list.size(), size_t(cap - 1));
            std::memcpy(names, list.data(), k);
            names[k] = 0;
        }
        if (count)
            *count = n;
        if (rank)
            *rank = r;
        if (alpha) {
            const auto it = st->metadata().find("alpha");
            *alpha = it == st->metadata().end() ? 0.f : std::stof(it->second);
        }
    });
}

int h3_sigmas(uint32_t steps, float shift, float* out, uint32_t* points)
{
    return guarded([&] {
        if (!out || !points)
            throw ArgError("h3_sigmas: null output");
        if (steps < 2 || !(shift > 0.f))
            throw ArgError("h3_sigmas: at least 2 points and a positive shift");
        const std::vector<float> v = h3::sigmas(int(steps), shift);
        std::memcpy(out, v.data(), v.size() * 4);
        *points = uint32_t(v.size());
    });
}

int h3_denoise(h3_model* m, float* video, uint64_t video_rows, float* audio, uint64_t audio_rows, const float* sigma_video,
               const float* sigma_audio, uint32_t points, h3_progress_fn progress, void* user, uint32_t* steps_run)
{
    return guarded([&] {
        check_model(m);
        if (m->m->rows() == 0)
            throw StateError("h3_denoise before h3_begin");
        check_io(m, video_rows, audio_rows);
        if ((video_rows && !video) || (audio_rows && !audio) || !sigma_video || !sigma_audio)
            throw ArgError("h3_denoise: null argument");
        if (points < 2)
            throw ArgError("h3_denoise: at least 2 schedule points");
        for (uint32_t i = 0; i + 1 < points; ++i)
            if (!(sigma_video[i] > 0.f) || !(sigma_audio[i] > 0.f))
                throw ArgError("h3_denoise: every schedule point but the last must be positive");
        std::function<bool(int, int)> cb;
        if (progress)
            cb = [&](int i, int n) { return progress(user, uint32_t(i), uint32_t(n)) == 0; };
        const int n = m->m->denoise(video, audio, sigma_video, sigma_audio, int(points), cb);
        if (steps_run)
            *steps_run = uint32_t(n);
    });
}

int h3_synchronize(h3_model* m)
{
    return guarded([&] {
        check_model(m);
        H3_CUDA(cudaStreamSynchronize(m->m->stream()));
        if (const uint32_t e = h3::take_device_error(m->m->stream()))
            throw DeviceError("device error " + std::to_string(e) + ": a kernel's bounded wait ran out");
    });
}

void* h3_stream(h3_model* m) { return m && m->m ? static_cast<void*>(m->m->stream()) : nullptr; }

int h3_set_probe(h3_model* m, h3_probe_fn fn, void* user)
{
    return guarded([&] {
        check_model(m);
        m->probe = fn;
        m->probe_user = user;
        if (!fn) {
            m->m->set_probe(nullptr);
            return;
        }
        m->m->set_probe([m](const std::string& name, int layer, const float* data, size_t n) {
            m->probe(m->probe_user, name.c_str(), layer, data, n);
        });
    });
}

uint64_t h3_layout_rows(const h3_layout* layout)
{
    if (!layout)
        return 0;
    const h3::Layout l = to_layout(layout);
    return uint64_t(l.rows());
}

int h3_rows(const h3_layout* layout, double* pos, uint8_t* tags, uint8_t* roles)
{
    return guarded([&] {
        const h3::Rows r = h3::layout_rows(to_layout(layout));
        if (pos)
            std::memcpy(pos, r.pos.data(), r.pos.size() * sizeof(double));
        if (tags)
            std::memcpy(tags, r.tags.data(), r.tags.size());
        if (roles)
            std::memcpy(roles, r.roles.data(), r.roles.size());
    });
}

int h3_rope_table(const h3_layout* layout, float* out)
{
    return guarded([&] {
        if (!out)
            throw ArgError("h3_rope_table: null output");
        const std::vector<float> t = h3::rope_table(h3::layout_rows(to_layout(layout)));
        std::memcpy(out, t.data(), t.size() * sizeof(float));
    });
}

int32_t h3_last_launches(h3_model* m) { return m && m->m ? m->m->last_launches() : 0; }

int h3_set_timing(h3_model* m, int32_t on)
{
    return guarded([&] {
        check_model(m);
        m->m->set_timing(on != 0);
    });
}

int32_t h3_last_timing(h3_model* m, float* ms, char* names, int32_t names_cap, int32_t cap)
{
    if (!m || !m->m)
        return 0;
    const auto& t = m->m->last_timing();
    int32_t n = 0, off = 0;
    for (size_t i = 1; i < t.size() && n < cap; ++i, ++n) {
        if (ms)
            ms[n] = t[i].second;
        if (names) {
            const std::string& s = t[i].first;
            if (off + int32_t(s.size()) + 1 > names_cap)
                break;
            std::memcpy(names + off, s.c_str(), s.size() + 1);
            off += int32_t(s.size()) + 1;
        }
    }
    return n;
}

void h3_destroy(h3_model* m)
{
    if (!m)
        return;
    cudaSetDevice(m->device);
    delete m;
}

// ------------------------------------------------------------------------------------------------ kernels
int h3k_gemm(const void* A, const void* B, const h3k_gemm_args* a, int32_t epilogue, int32_t int8, void* stream)
{
    return guarded([&] {
        if (!A || !B || !a)
            throw ArgError("h3k_gemm: null argument");
        device_ptrs("h3k_gemm", {A, B, a->out, a->bias, a->x, a->mod, a->mod_idx, a->rope, a->qn_w, a->kn_w, a->a_scale, a->b_scale});
        if (epilogue < 0 || epilogue > 5)
            throw ArgError("h3k_gemm: unknown epilogue");
        h3::GemmParams p;
        p.M = a->M, p.N = a->N, p.K = a->K, p.a_chunks = a->a_chunks > 0 ? a->a_chunks : 1, p.a_rows_stride = a->a_rows_stride;
        p.lda = a->lda, p.ldb = a->ldb, p.out = a->out, p.ldo = a->ldo, p.bias = a->bias, p.x = a->x, p.ldx = a->ldx;
        p.mod = a->mod, p.mod_idx = a->mod_idx, p.gate_slot = a->gate_slot, p.dim = a->dim, p.rope = a->rope;
        p.qn_w = a->qn_w, p.kn_w = a->kn_w, p.eps = a->eps, p.inner = a->inner, p.heads_per_rank = a->heads_per_rank;
        p.rows_local = a->rows_local, p.a_scale = a->a_scale, p.b_scale = a->b_scale;
        if (!p.out && epilogue != H3K_EPI_GATE_RESID)
            throw ArgError("h3k_gemm: null output");
        if (int8)
            h3::gemm_s8(A, B, p, h3::Epi(epilogue), st(stream));
        else
            h3::gemm_bf16(A, B, p, h3::Epi(epilogue), st(stream));
    });
}

int h3k_rms_mod(const float* x, int64_t ldx, int32_t rows, int32_t d, const float* w, const float* mod, const uint8_t* mod_idx,
                int32_t mod_slots, int32_t shift_slot, int32_t scale_slot, float eps, int32_t out_kind, void* out, int64_t ldo,
                float* out_scale, void* stream)
{
    return guarded([&] {
        if (out_kind < 0 || out_kind > 2)
            throw ArgError("h3k_rms_mod: out_kind 0 bf16, 1 f32, 2 int8");
        device_ptrs("h3k_rms_mod", {x, w, mod, mod_idx, out, out_scale});
        h3::RmsModParams p;
        p.x = x, p.ldx = ldx, p.rows = rows, p.d = d, p.w = w, p.mod = mod, p.mod_idx = mod_idx, p.mod_slots = mod_slots;
        p.shift_slot = shift_slot, p.scale_slot = scale_slot, p.eps = eps, p.out_kind = h3::RowOut(out_kind), p.out = out, p.ldo = ldo;
        p.out_scale = out_scale;
        h3::rms_mod_rows(p, st(stream));
    });
}

int h3k_gate_add(float* x, int64_t ldx, const void* y, int64_t ldy, int32_t rows, int32_t d, const float* mod, const uint8_t* mod_idx,
                 int32_t gate_slot, void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_gate_add", {x, y, mod, mod_idx});
        h3::gate_add_rows(x, ldx, y, ldy, rows, d, mod, mod_idx, gate_slot, st(stream));
    });
}

int h3k_swiglu(const void* gv, int32_t rows, int32_t F, void* out, void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_swiglu", {gv, out});
        h3::swiglu_rows(gv, rows, F, out, st(stream));
    });
}

int h3k_quant_rows_i8(const void* x, int64_t ldx, int32_t rows, int32_t K, int8_t* q, float* scale, void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_quant_rows_i8", {x, q, scale});
        h3::quant_rows_i8(x, ldx, rows, K, q, scale, st(stream));
    });
}

int h3k_quant_weight(const void* w, int32_t rows, int32_t K, int8_t* q, float* scale, void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_quant_weight", {w, q, scale});
        h3::quant_weight_rows(w, rows, K, q, scale, st(stream));
    });
}

int h3k_heads_partial(void* qkv, int32_t rows, int32_t heads, const float* qn_w, const float* kn_w, const float* rope, float eps,
                      void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_heads_partial", {qkv, qn_w, kn_w, rope});
        h3::heads_partial(qkv, rows, heads, qn_w, kn_w, rope, eps, st(stream));
    });
}

int h3k_attention(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, int32_t rows, void* out,
                  int64_t out_row_stride, void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_attention", {q, k, v, out});
        h3::AttnParams p;
        p.q = q, p.k = k, p.v = v, p.row_stride = row_stride, p.heads = heads, p.rows = rows, p.out = out;
        p.out_row_stride = out_row_stride;
        h3::attention(p, st(stream));
    });
}

int h3k_attention_bounded(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, int32_t rows,
                          float score_bound, void* out, int64_t out_row_stride, void* stream)
{
    return guarded([&] {
        if (!(score_bound >= 0.f && score_bound <= h3::kMaxStaticBound))
            throw ArgError("h3k_attention_bounded: the score bound must be in [0, 40]");
        device_ptrs("h3k_attention_bounded", {q, k, v, out});
        h3::AttnParams p;
        p.q = q, p.k = k, p.v = v, p.row_stride = row_stride, p.heads = heads, p.rows = rows, p.out = out;
        p.out_row_stride = out_row_stride, p.static_max = score_bound;
        h3::attention(p, st(stream));
    });
}

int h3k_sparse_sizes(const h3k_cube_grid* g, float ratio, int32_t local, int32_t* cubes, int32_t* kcap, int32_t* q_tiles,
                     int32_t* max_blocks)
{
    return guarded([&] {
        const h3::CubeGrid c = to_grid(g);
        int kc, qt, mb;
        h3::sparse_sizes(c, ratio, local, kc, qt, mb);
        if (cubes)
            *cubes = c.cubes();
        if (kcap)
            *kcap = kc;
        if (q_tiles)
            *q_tiles = qt;
        if (max_blocks)
            *max_blocks = mb;
    });
}

int h3k_sparse_select(const void* q, const void* k, int64_t row_stride, int32_t heads, const h3k_cube_grid* g, float ratio, int32_t local,
                      float* mq, float* mk, float* scores, int32_t* sel, int32_t* nsel, void* stream)
{
    return guarded([&] {
        const h3::CubeGrid c = to_grid(g);
        if (!q || !k || !sel || !nsel)
            throw ArgError("h3k_sparse_select: null argument");
        device_ptrs("h3k_sparse_select", {q, k, mq, mk, scores, sel, nsel});
        int kc, qt, mb;
        h3::sparse_sizes(c, ratio, local, kc, qt, mb);
        Scratch sc;
        const size_t nc = c.cubes();
        if (!mq)
            mq = static_cast<float*>(sc.get(size_t(heads) * nc * 128 * 4));
        if (!mk)
            mk = static_cast<float*>(sc.get(size_t(heads) * nc * 128 * 4));
        if (!scores)
            scores = static_cast<float*>(sc.get(size_t(heads) * nc * nc * 4));
        h3::cube_pool(q, k, row_stride, heads, c, mq, mk, st(stream));
        h3::cube_scores(mq, mk, heads, c.cubes(), scores, st(stream));
        h3::cube_topk(scores, heads, c, h3::sparse_k(ratio, c.cubes()), local, sel, nsel, kc, st(stream));
        H3_CUDA(cudaStreamSynchronize(st(stream)));
    });
}

int h3k_video_order(const h3k_cube_grid* g, int32_t* src)
{
    return guarded([&] {
        const h3::CubeGrid c = to_grid(g);
        if (!src)
            throw ArgError("h3k_video_order: null output");
        for (int f = 0, n = 0; f < c.frames; ++f)
            for (int y = 0; y < c.ph; ++y)
                for (int x = 0; x < c.pw; ++x, ++n)
                    src[c.video_pos(f, y, x) - c.dense_rows] = n;
    });
}

int h3k_cube_topk(const float* scores, int32_t heads, const h3k_cube_grid* g, float ratio, int32_t local, int32_t* sel, int32_t* nsel,
                  void* stream)
{
    return guarded([&] {
        const h3::CubeGrid c = to_grid(g);
        if (!scores || !sel || !nsel)
            throw ArgError("h3k_cube_topk: null argument");
        device_ptrs("h3k_cube_topk", {scores, sel, nsel});
        int kc, qt, mb;
        h3::sparse_sizes(c, ratio, local, kc, qt, mb);
        h3::cube_topk(scores, heads, c, h3::sparse_k(ratio, c.cubes()), local, sel, nsel, kc, st(stream));
    });
}

namespace {
int sparse_attention_call(const char* name, const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads,
                          const h3k_cube_grid* g, float ratio, int32_t local, float score_bound, void* out, int64_t out_row_stride,
                          void* stream)
{
    return guarded([&] {
        const h3::CubeGrid c = to_grid(g);
        if (!q || !k || !v || !out)
            throw ArgError(std::string(name) + ": null argument");
        if (!(score_bound >= 0.f && score_bound <= h3::kMaxStaticBound))
            throw ArgError(std::string(name) + ": the score bound must be in [0, 40]");
        device_ptrs(name, {q, k, v, out});
        h3::SparseBuffers b;
        h3::sparse_sizes(c, ratio, local, b.kcap, b.q_tiles, b.max_blocks);
        Scratch sc;
        const size_t nc = c.cubes();
        b.mq = static_cast<float*>(sc.get(size_t(heads) * nc * 128 * 4));
        b.mk = static_cast<float*>(sc.get(size_t(heads) * nc * 128 * 4));
        b.scores = static_cast<float*>(sc.get(size_t(heads) * nc * nc * 4));
        b.sel = static_cast<int32_t*>(sc.get(size_t(heads) * nc * b.kcap * 4));
        b.nsel = static_cast<int32_t*>(sc.get(size_t(heads) * nc * 4));
        b.blocks = static_cast<int4*>(sc.get(size_t(heads) * b.q_tiles * b.max_blocks * 16));
        b.nblocks = static_cast<int32_t*>(sc.get(size_t(heads) * b.q_tiles * 4));
        b.q_rows = static_cast<int4*>(sc.get(size_t(b.q_tiles) * 16));
        h3::AttnParams p;
        p.q = q, p.k = k, p.v = v, p.row_stride = row_stride, p.heads = heads, p.rows = c.dense_rows + c.frames * c.ph * c.pw;
        p.out = out, p.out_row_stride = out_row_stride;
        p.static_max = score_bound;
        h3::sparse_attention(p, c, ratio, local, b, st(stream));
        H3_CUDA(cudaStreamSynchronize(st(stream)));
    });
}
} // namespace

int h3k_sparse_attention(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, const h3k_cube_grid* g, float ratio,
                         int32_t local, void* out, int64_t out_row_stride, void* stream)
{
    return sparse_attention_call("h3k_sparse_attention", q, k, v, row_stride, heads, g, ratio, local, 0.f, out, out_row_stride, stream);
}

int h3k_sparse_attention_bounded(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, const h3k_cube_grid* g,
                                 float ratio, int32_t local, float score_bound, void* out, int64_t out_row_stride, void* stream)
{
    return sparse_attention_call("h3k_sparse_attention_bounded", q, k, v, row_stride, heads, g, ratio, local, score_bound, out,
                                 out_row_stride, stream);
}

int h3k_fill_synthetic(void* dst, int32_t is_bf16, uint64_t n, uint64_t seed, uint32_t tensor_id, float mean, float stdev, void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_fill_synthetic", {dst});
        h3::fill_synthetic(dst, is_bf16, n, seed, tensor_id, mean, stdev, st(stream));
    });
}

int h3k_gemv_f32(const float* W, const float* b, const float* x, int32_t U, int32_t N, int32_t K, int32_t act, float* out, float* out2,
                 void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_gemv_f32", {W, b, x, out, out2});
        h3::gemv_f32(W, b, x, U, N, K, h3::Act(act), out, out2, st(stream));
    });
}

int h3k_adaln(const void* W, const float* b, const float* x, int32_t U, int32_t groups, int32_t G, int32_t K, float* out, void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_adaln", {W, b, x, out});
        h3::adaln_gemv(W, b, x, U, groups, G, K, out, st(stream));
    });
}

int h3k_heads(const float* x, int64_t ldx, int32_t rows, const float* W, const float* b, int32_t N, int32_t K, float* out, int64_t ldo,
              void* stream)
{
    return guarded([&] {
        device_ptrs("h3k_heads", {x, W, b, out});
        h3::heads_f32(x, ldx, rows, W, b, N, K, out, ldo, st(stream));
    });
}

int h3k_wait_selftest(uint64_t budget_cycles, void* stream)
{
    return guarded([&] {
        h3::wait_selftest((long long)budget_cycles, st(stream));
        H3_CUDA(cudaStreamSynchronize(st(stream)));
        const uint32_t e = h3::take_device_error(st(stream));
        if (e)
            throw DeviceError("device error " + std::to_string(e) + ": the self-test's bounded wait ran out, as it must");
        throw StateError("h3k_wait_selftest: the wait did not give up");
    });
}

int h3k_check(void* stream)
{
    return guarded([&] {
        H3_CUDA(cudaStreamSynchronize(st(stream)));
        if (const uint32_t e = h3::take_device_error(st(stream)))
            throw DeviceError("device error " + std::to_string(e) + ": a kernel's bounded wait ran out");
    });
}

} // extern "C"
