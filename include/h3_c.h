/* C ABI of the B200 implementation of the MiniMax-H3 transformer step (libh3b200.so).
 *
 * Drop-in for the transformer the reference's sampler calls once per schedule point: the C++ class
 * mako::models::H3 (aliased video::H3, src/video/engine.hpp:22 of jhanssen/mako-video). Each entry point below names
 * the reference call it replaces. Plain pointers and sizes only; every call returns H3_OK or an error code, and
 * h3_last_error() gives the message of the last failure on the calling thread (the reference throws
 * std::runtime_error at the same places; include/models/h3.hpp re-throws).
 *
 * One process per GPU. With more than one rank the step is sequence-parallel (Ulysses): every rank passes the same
 * inputs, holds the same weights, computes a contiguous share of the rows outside attention and all rows for
 * heads / ranks heads inside it, and returns the full outputs. */
#ifndef H3_C_H
#define H3_C_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3_OK 0
#define H3_ERR_ARG 1    /* bad argument or shape */
#define H3_ERR_CUDA 2   /* a CUDA or NCCL call failed */
#define H3_ERR_STATE 3  /* call out of order (step before begin) */
#define H3_ERR_DEVICE 4 /* a kernel reported a device-side failure (a bounded wait ran out) */

typedef struct h3_model h3_model;

/* Model shape. MiniMax-H3: dim 5376, heads 56, ffn 14336, blocks 50, time_dim 2688 (docs/architecture.md:23-27,
 * 47-67); the benchmark's synthetic 768p stack: 5120, 40, 13824, 48, 2560. Heads are 128 wide. */
typedef struct h3_config {
    uint32_t dim, heads, ffn, blocks, time_dim;
    uint32_t text_dim;       /* the text encoder's width (5120, H3::kText) */
    uint32_t video_patch;    /* 96 (H3::kVideoPatch: a 2x2 patch of 24 channels) */
    uint32_t audio_channels; /* 32 (H3::kAudioChannels) */
    float eps;               /* RMS norm epsilon */
    uint32_t refiner_blocks; /* token refiner blocks run over the text rows in h3_begin (MiniMax-H3: 2; 0: none, at most
                              * 2). Plain pre-norm blocks of the step's widths without modulation or rotary positions,
                              * then a weighted RMS norm (docs/architecture.md:25-27). */
    uint32_t curve_dims;     /* 0: the full model (time embedder, SiLU, [18 dim][time_dim] AdaLN projections). 8: a pruned
                              * checkpoint (docs/architecture.md:57-60): no time embedder; a level t reads the curve
                              * adaln_t_table [1025][8] at t * 1024 with linear interpolation, and every block's AdaLN
                              * projection is [18 dim][8] (the final layer's [2 dim][8]) applied in fp32 without SiLU
                              * (curve_mods; tools/check_pruned_curve.py:43-70). */
} h3_config;

/* A reference block of a ref2va layout (H3::Layout::Reference, src/video/engine.cpp:604-616;
 * tests/h3_ref_test.cpp:475-479): a picture (frames 1, h x w latents), a video (frames latent frames of h x w, audio
 * soundtrack latents or 0) or a soundtrack (audio latents). Its visual rows are held at t = 0.999, its audio rows at
 * t = 1 (docs/architecture.md:38-42, 203-215). */
enum { H3_REF_IMAGE = 0, H3_REF_VIDEO = 1, H3_REF_AUDIO = 2 };
typedef struct h3_layout_ref {
    int32_t kind;
    uint32_t frames, h, w, audio;
} h3_layout_ref;

/* The packed sequence [text | keyframe rows or reference blocks | audio | generated video] (H3::Layout,
 * src/video/engine.cpp:666-676; tests/h3_ref_test.cpp:194, 476-481). The video input/output rows are the conditioning
 * rows (keyframes, or the references' pictures and videos in reading order) then the generated rows; the audio rows
 * are the references' soundtracks (reading order) then the generated audio. */
typedef struct h3_layout {
    uint32_t text;        /* text rows T */
    uint32_t frames;      /* generated latent frames */
    uint32_t h, w;        /* latent height and width (a row is a 2x2 patch: (h / 2) * (w / 2) rows a frame) */
    uint32_t audio;       /* audio latents per channel (2 * audio rows) */
    uint32_t cond_frames; /* keyframe latent frames (rows held at t = 0.999) */
    const uint8_t* cond_last; /* [cond_frames]: keyframe anchored at the last generated frame (NULL: all first) */
    const uint8_t* text_tags; /* [text]: modality tag per text row, 1 text or 0 video (NULL: all text) */
    const h3_layout_ref* refs; /* [n_refs] reference blocks in reading order (NULL when n_refs is 0) */
    uint32_t n_refs;
} h3_layout;

typedef struct h3_world {
    int32_t rank, size;      /* this process's rank and the number of ranks (one GPU each) */
    uint8_t nccl_id[128];    /* from h3_nccl_unique_id on rank 0, passed to every rank */
} h3_world;

/* Probe callback (H3::set_probe, tests/h3_ref_test.cpp:215-217): name is one of txt (the text rows after the token
 * refiner, from h3_begin; tests/h3_ref_test.cpp:219), temb (not for a pruned checkpoint, which has no time embedder),
 * mod0, x0, block, norm_out; layer is the block for "block" and -1 otherwise; data is host memory valid during the call. Single-rank only. */
typedef void (*h3_probe_fn)(void* user, const char* name, int32_t layer, const float* data, uint64_t n);

/* The message of the last failed call on this thread ("" if none). */
const char* h3_last_error(void);

/* An NCCL unique id for a multi-rank group (rank 0 makes it, every rank passes it in h3_world). */
int h3_nccl_unique_id(uint8_t out[128]);

/* H3::H3(path, ctx, telemetry, int8) and Engine::transformer (src/video/engine.cpp:105-117).
 * weights: "synthetic:SEED" for random-init weights (every value a hash of SEED, tensor and index), or a checkpoint:
 * a safetensors file or a directory of them holding every tensor h3_check_weights lists, under this build's names
 * (the reference's own where its files or prose give them: time_embedder.*, blocks.N.adaln_proj.linear.*,
 * adaln_t_table, condition_proj, video_patch_proj, audio_patch_proj, proj_out), in the logical layout: fc1
 * [gate; value], q/k/v stacked q, k, v (or, with file metadata qkv_layout = interleaved, each head's q, k and v rows
 * together, stacked at load as the reference's upload_qkv does, docs/architecture.md:62-63). BF16, F16 and F32
 * tensors are converted to the model's element types. A missing tensor or a shape that disagrees returns H3_ERR_ARG
 * before any device work. int8_mask: bits 1 qkv, 2 out, 4 fc1, 8 fc2 (H3::Int8), quantised per row at load.
 * sparse_ratio / sparse_local as h3_set_sparse. world: NULL for one rank. device: the CUDA device. */
int h3_create(const h3_config* cfg, const char* weights, uint32_t int8_mask, float sparse_ratio, uint32_t sparse_local,
              const h3_world* world, int32_t device, h3_model** out);

/* H3::set_sparse(ratio, local) (src/video/engine.cpp:112): ratio 0 dense attention, else the share of video cubes
 * each cube attends; local 0, 1 (itself) or 3 (itself and its temporal neighbours). Takes effect at h3_begin. */
int h3_set_sparse(h3_model* m, float ratio, uint32_t local);

/* H3::parse_int8 (tools/mako_video.cpp:108-114): "none", "all" or a comma list of qkv, out, fc1, fc2. */
int h3_parse_int8(const char* text, uint32_t* mask);

/* H3::begin(text, layout) (src/video/engine.cpp:700; tests/h3_ref_test.cpp:218): text is [T][text_dim] fp32 host
 * memory; caches the text rows and the layout's tables for the steps that follow. */
int h3_begin(h3_model* m, const float* text, uint32_t text_rows, const h3_layout* layout);

/* H3::step(video, audio, t_video, t_audio) (src/video/engine.cpp:714; tests/h3_ref_test.cpp:224): video [V][96]
 * (keyframe rows first) and audio [A][32] fp32 host memory in; their velocities out (host memory, same shapes). */
int h3_step(h3_model* m, const float* video, uint64_t video_rows, const float* audio, uint64_t audio_rows, float t_video,
            float t_audio, float* out_video, float* out_audio);

/* The same with device pointers; the step is queued on the model's stream (h3_stream) and not waited for. */
int h3_step_device(h3_model* m, const float* video, uint64_t video_rows, const float* audio, uint64_t audio_rows, float t_video,
                   float t_audio, float* out_video, float* out_audio);

/* Waits for the model's stream and reports a device-side failure of the queued work as H3_ERR_DEVICE. */
int h3_synchronize(h3_model* m);

/* H3::add_lora(path, scale, strict) (src/video/engine.cpp:114; docs/architecture.md:108-116): merges a safetensors
 * file of Diffusers-named LoRA adapters into the weights, W += scale * alpha / rank * B A (bf16 matrices; int8
 * matrices are requantised per row). Targets: transformer_blocks.N.attn.to_q/to_k/to_v/to_out.0, ff.net.0.proj
 * (Diffusers' [value; gate] rows rotated to [gate; value]), ff.net.2, adaln_proj.linear (rows re-laid out from
 * (chunk, modality) to (modality, chunk)). Token-refiner targets are skipped; with strict, any other unknown name
 * fails. merged / skipped (may be NULL) get the counts. */
int h3_add_lora(h3_model* m, const char* path, float scale, int32_t strict, uint32_t* merged, uint32_t* skipped);

/* Reads a LoRA file's adapter list without a model (host only): `names` gets the adapter target names (prefixes
 * stripped), '\n'-separated, NUL-terminated, truncated to cap bytes; *count the adapters, *rank the first one's
 * rank, *alpha the file's "alpha" metadata (0 when absent). Any pointer may be NULL. No counterpart in the reference. */
int h3_lora_inspect(const char* path, char* names, uint64_t cap, uint32_t* count, uint32_t* rank, float* alpha);

/* Every tensor a checkpoint for this model shape holds, one line each: "name dtype shape" (dtype BF16 or F32, the
 * element type the model keeps; shape as d0xd1), in set-up order; NUL-terminated, truncated to cap bytes; *count the
 * tensors. For converters from other layouts. Host only. No counterpart in the reference. */
int h3_weight_specs(const h3_config* cfg, char* out, uint64_t cap, uint32_t* count);

/* Rewrites the checkpoint at src (a safetensors file or a directory of them) as a file at dst in the layout h3_create
 * reads, for a model of shape cfg: every tensor under this library's name, the model's element type, q/k/v stacked.
 * renames (may be NULL): lines "this_name source_name" for tensors the source names otherwise, '#' lines ignored,
 * and "qkv_layout interleaved" (or "qkv_layout stacked") for a source whose metadata does not say how it keeps each
 * head's q, k and v rows (the reference's shards keep them together, docs/architecture.md:62-63): the shapes cannot
 * tell the two apart, so a source file with q/k/v tensors and no qkv_layout metadata is refused (H3_ERR_ARG) unless
 * that line is given. The source is checked first (a missing tensor or a shape that disagrees: H3_ERR_ARG). Host only. No counterpart in the reference: the path from its FL2VA files (whose
 * block-internal tensor names are not in the reference tree) to this library. */
int h3_convert_weights(const h3_config* cfg, const char* src, const char* dst, const char* renames);

/* Writes the model's weights to a safetensors file in the layout h3_create reads (qkv_layout = stacked), so that a
 * model created from the file computes what this one does. bf16 models only (an int8 model holds no bf16 rows of its
 * quantised projections: H3_ERR_ARG). The file holding the weights is the reference's model directory's role
 * (src/video/engine.cpp:105-117); the writer itself has no counterpart in the reference. */
int h3_save_weights(h3_model* m, const char* path);

/* Checks a checkpoint (file or directory) against a model shape without touching a GPU: H3_OK when every tensor
 * h3_create needs is there with its shape, else H3_ERR_ARG with the first problem (a missing tensor, a shape that
 * disagrees) in message (NUL-terminated, truncated to cap bytes; may be NULL) and h3_last_error(). Host only. No
 * counterpart in the reference. */
int h3_check_weights(const h3_config* cfg, const char* path, char* message, uint64_t cap);

/* Engine::sigmas(steps, shift) (src/video/engine.cpp:71-88): the schedule from 1 to 0, torch.linspace's float
 * spacing, shifted by s x / (1 + (s - 1) x), consecutive repeats dropped. Writes up to `steps` points to out and
 * their count to *points. Host only. */
int h3_sigmas(uint32_t steps, float shift, float* out, uint32_t* points);

/* Progress of h3_denoise: called on the host after step `step` (1-based) of `steps` has finished on the GPU; a
 * nonzero return stops the loop after that step (the reference's cooperative cancellation,
 * src/video/engine.cpp:717-718, tools/video_server.cpp:499-501). */
typedef int (*h3_progress_fn)(void* user, uint32_t step, uint32_t steps);

/* Engine::denoise's step loop (src/video/engine.cpp:701-719) on the GPU: for i < points - 1, the forward at
 * t_video = 1 - sigma_video[i], t_audio = 1 - sigma_audio[i], then the Euler move of the generated rows to
 * sigma[i + 1] (x0 = x + (1 - t) v; x = r x + (1 - r) x0, r = sigma[i + 1] / sigma[i]); the conditioning rows stay.
 * video [V][96] and audio [A][32] are host memory holding the start sample (conditioning rows, then noise) and get
 * the final sample. The sample stays on the device between steps: no host copies per step. progress may be NULL.
 * *steps_run (may be NULL) gets the steps taken. */
int h3_denoise(h3_model* m, float* video, uint64_t video_rows, float* audio, uint64_t audio_rows, const float* sigma_video,
               const float* sigma_audio, uint32_t points, h3_progress_fn progress, void* user, uint32_t* steps_run);

/* The model's CUDA stream (a cudaStream_t). */
void* h3_stream(h3_model* m);

int h3_set_probe(h3_model* m, h3_probe_fn fn, void* user);

/* H3::rows(layout) (tests/h3_ref_test.cpp:484-502): per row the rotary position (t, h, w) [S][3] in double, the
 * modality tag (0 video, 1 text, 2 audio) and the role (0 text, 1 keyframe video, 3 audio, 4 video). Any output
 * may be NULL. h3_layout_rows gives S. */
uint64_t h3_layout_rows(const h3_layout* layout);
int h3_rows(const h3_layout* layout, double* pos, uint8_t* tags, uint8_t* roles);

/* The rotary table the step uses for a layout: [S][48][2] (cos, sin) of angle = float(pos_axis) * inv_freq (16
 * frequencies per axis t, h, w of base 10000; docs/architecture.md:35-40, tools/dump_h3_ref.py:140-141). */
int h3_rope_table(const h3_layout* layout, float* out);

/* This library's kernel launches in the last step. */
int32_t h3_last_launches(h3_model* m);

/* Device milliseconds of the last step's stages (start..adaln, ..input, ..block 0 parts, ..blocks, ..heads) when
 * timing is on; returns the number of stages written (at most `cap`), names as a '\0'-separated list. */
int h3_set_timing(h3_model* m, int32_t on);
int32_t h3_last_timing(h3_model* m, float* ms, char* names, int32_t names_cap, int32_t cap);

void h3_destroy(h3_model* m);

/* ------------------------------------------------------------------------------------------------------------
 * Kernel-level entry points: the reference's GPU kernels (mako-common, named in docs/architecture.md:52,64,124-127
 * and docs/performance.md:39-45,120-126), each as one sm_100a kernel on device pointers. `stream` is a
 * cudaStream_t (NULL: the legacy default stream). They do not synchronize; h3k_check does. */

/* Gemm::encode / gemm_i8 with a fused epilogue. D[M][N] = A[M][K] B[N][K]^T; A and B row-major with K contiguous. */
#define H3K_EPI_BF16 0       /* out bf16 [M][ldo] = acc + bias */
#define H3K_EPI_F32 1        /* out f32 = acc + bias */
#define H3K_EPI_QKV 2        /* heads_partial fused: q/k per-head RMS norm + rotary, v + bias; [rows][3][heads][128] */
#define H3K_EPI_GATE_RESID 3 /* gate_add_rows fused: x += gate[mod_idx[r]] * (acc + bias) */
#define H3K_EPI_SWIGLU 4     /* swiglu_rows fused: out = silu(gate) * value; B rows in 128-row [gate; value] groups */
#define H3K_EPI_S32 5        /* int8 only: out int32 = the raw integer dot products */
typedef struct h3k_gemm_args {
    int32_t M, N, K;
    int32_t a_chunks, a_rows_stride, lda, ldb; /* A split into a_chunks column chunks ([chunk][rows][K/chunks]) */
    void* out;
    int64_t ldo;
    const float* bias;
    float* x;
    int64_t ldx;
    const float* mod;       /* [n_mod][6][dim] */
    const uint8_t* mod_idx; /* [M] */
    int32_t gate_slot, dim;
    const float* rope; /* [M][48][2] */
    const float* qn_w;
    const float* kn_w;
    float eps;
    int32_t inner, heads_per_rank, rows_local;
    const float* a_scale; /* int8: per row of A */
    const float* b_scale; /* int8: per row of B */
} h3k_gemm_args;
int h3k_gemm(const void* A, const void* B, const h3k_gemm_args* args, int32_t epilogue, int32_t int8, void* stream);

/* rms_mod_rows: y = RMSNorm(x) (* w) * (1 + scale) + shift per row; out_kind 0 bf16, 1 f32, 2 int8 + row scale. */
int h3k_rms_mod(const float* x, int64_t ldx, int32_t rows, int32_t d, const float* w, const float* mod, const uint8_t* mod_idx,
                int32_t mod_slots, int32_t shift_slot, int32_t scale_slot, float eps, int32_t out_kind, void* out, int64_t ldo,
                float* out_scale, void* stream);
/* gate_add_rows: x += gate * y (y bf16). */
int h3k_gate_add(float* x, int64_t ldx, const void* y, int64_t ldy, int32_t rows, int32_t d, const float* mod, const uint8_t* mod_idx,
                 int32_t gate_slot, void* stream);
/* swiglu_rows: out [rows][F] = silu(gv[:, :F]) * gv[:, F:] (bf16). */
int h3k_swiglu(const void* gv, int32_t rows, int32_t F, void* out, void* stream);
/* quant_rows_i8: per-row symmetric int8 (scale = max|x| / 127). */
int h3k_quant_rows_i8(const void* x, int64_t ldx, int32_t rows, int32_t K, int8_t* q, float* scale, void* stream);
/* Per-output-row int8 quantisation of a weight (what the int8 load does). */
int h3k_quant_weight(const void* w, int32_t rows, int32_t K, int8_t* q, float* scale, void* stream);
/* heads_partial (standalone): per-head q/k RMS norm + rotary in a [rows][3][heads][128] bf16 tensor, in place. */
int h3k_heads_partial(void* qkv, int32_t rows, int32_t heads, const float* qn_w, const float* kn_w, const float* rope, float eps,
                      void* stream);
/* flash_attn_coop_128_32: dense bidirectional attention over `rows` rows and `heads` heads of 128. */
int h3k_attention(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, int32_t rows, void* out,
                  int64_t out_row_stride, void* stream);
/* The same given a bound on every score, q.k / sqrt(128) * log2(e) <= score_bound (at most 40; see
 * h3k_sparse_attention_bounded): the softmax takes it for the row maximum. 0 means unknown (as h3k_attention). It
 * stands for the same reference kernel (flash_attn_coop_128_32). */
int h3k_attention_bounded(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, int32_t rows,
                          float score_bound, void* out, int64_t out_row_stride, void* stream);

/* The sparse attention's cube grid: dense_rows rows (text, keyframe, audio) then frames x ph x pw generated video
 * rows (a row is a 2x2 patch), cut into 4x4x4 cubes (cubes at the far edges cut short). The h3k_sparse_* calls take
 * q, k, v and write out in the packed row order: the dense rows, then the generated video rows cube by cube (cubes
 * in (frame group, row group, column group) order, each cube's rows in (frame, row, column) order), which is the
 * order the step keeps its rows in. (The reference's sparse kernels gather a cube's rows through a row map instead,
 * h3.hpp Cubes per its arch.md:121-124; the packed order makes every cube one run of rows.) */
typedef struct h3k_cube_grid {
    int32_t dense_rows, frames, ph, pw;
} h3k_cube_grid;
/* The packed order of the generated video rows: src[i] = (f * ph + y) * pw + x of packed video row i (the row
 * dense_rows + i), for i < frames * ph * pw. No counterpart in the reference. */
int h3k_video_order(const h3k_cube_grid* g, int32_t* src);
/* Sizes for a grid: cubes, kcap (selected cubes per query cube at most), q_tiles, max_blocks. */
int h3k_sparse_sizes(const h3k_cube_grid* g, float ratio, int32_t local, int32_t* cubes, int32_t* kcap, int32_t* q_tiles,
                     int32_t* max_blocks);
/* cube_pool + cube_scores + cube_topk: mq, mk [heads][cubes][128] f32, scores [heads][cubes][cubes] f32 (any may be
 * NULL for internal scratch), sel [heads][cubes][kcap] ascending cube indices, nsel [heads][cubes]. */
int h3k_sparse_select(const void* q, const void* k, int64_t row_stride, int32_t heads, const h3k_cube_grid* g, float ratio,
                      int32_t local, float* mq, float* mk, float* scores, int32_t* sel, int32_t* nsel, void* stream);
/* cube_topk alone, on given scores [heads][cubes][cubes]. */
int h3k_cube_topk(const float* scores, int32_t heads, const h3k_cube_grid* g, float ratio, int32_t local, int32_t* sel, int32_t* nsel,
                  void* stream);
/* The whole sparse attention (selection, pass lists, flash_attn_sparse_128); scratch is allocated per call. */
int h3k_sparse_attention(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, const h3k_cube_grid* g,
                         float ratio, int32_t local, void* out, int64_t out_row_stride, void* stream);

/* The same sparse attention given a bound on every score: q.k / sqrt(128) * log2(e) <= score_bound for all rows and
 * heads (at most 40; q and k RMS-normed per head with weights of magnitude at most wq and wk give 16.3222 wq wk, as
 * the step uses). The softmax then takes the bound for the row maximum: no running maximum, no exchange of it between
 * a row's warps, no rescaling. 0 means unknown (as h3k_sparse_attention). A bound below the true maximum gives wrong
 * results, not an error. Same scratch and synchronisation as h3k_sparse_attention; it stands for the same reference
 * kernel (flash_attn_sparse_128). */
int h3k_sparse_attention_bounded(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads,
                                 const h3k_cube_grid* g, float ratio, int32_t local, float score_bound, void* out,
                                 int64_t out_row_stride, void* stream);

/* The same sparse attention without any device allocation (no counterpart in the reference, whose Metal runtime
 * owns its buffers). For callers that cannot call cudaMalloc around an attention call: a serving stack that has
 * reserved nearly all device memory for its own pool, or one whose other streams must not stall on the device-wide
 * synchronisation of cudaMalloc / cudaFree. The scratch is a fixed 16 MiB array inside the library, held by every GPU
 * that loads it until the process exits; a grid and head count that need more return H3_ERR_ARG with the sizes.
 * Every call shares that array: calls whose work overlaps on the GPU race. The first call in each CUDA context (the
 * device's primary context, normally) looks up the array's device address; make it before any stream capture. A
 * context torn down and re-created (cudaDeviceReset) is recognised by its id and looked up afresh. Queued on
 * `stream`, not waited for (h3k_check). */
int h3k_sparse_attention_noalloc(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads,
                                 const h3k_cube_grid* g, float ratio, int32_t local, void* out, int64_t out_row_stride, void* stream);

/* Synthetic parameters as the model makes them (value = mean + std * IH4(seed, tensor_id, i)). */
int h3k_fill_synthetic(void* dst, int32_t is_bf16, uint64_t n, uint64_t seed, uint32_t tensor_id, float mean, float stdev, void* stream);

/* Time-embedding MLP layer (fp32): out[u][n] = act(W[n] . x[u] + b[n]), act 0 none / 1 silu; out2 (optional) gets
 * bf16(silu(out)). AdaLN projections: out[(g * U + u) * G + j] = W[g * G + j] . x[u] + b (W bf16). Heads (fp32). */
int h3k_gemv_f32(const float* W, const float* b, const float* x, int32_t U, int32_t N, int32_t K, int32_t act, float* out, float* out2,
                 void* stream);
int h3k_adaln(const void* W, const float* b, const float* x, int32_t U, int32_t groups, int32_t G, int32_t K, float* out, void* stream);
int h3k_heads(const float* x, int64_t ldx, int32_t rows, const float* W, const float* b, int32_t N, int32_t K, float* out, int64_t ldo,
              void* stream);

/* Failure-detection self-test (no counterpart in the reference): a kernel waits on an mbarrier that nothing arrives
 * on; the wait gives up after about budget_cycles SM clocks (at most 4e9), records its error and the kernel ends.
 * Returns H3_ERR_DEVICE with the device error, as a step whose pipeline wait ran out does; the context stays usable
 * and the error word is cleared. */
int h3k_wait_selftest(uint64_t budget_cycles, void* stream);
/* Waits for `stream` and reports a device-side failure (bounded wait ran out) as H3_ERR_DEVICE. */
int h3k_check(void* stream);

/* ------------------------------------------------------------------------------------------ video VAE decoder
 * MiniMax-H3's ViT video decoder (models::H3Vae, driven clip by clip by video::VideoVae, src/video/video_vae.hpp:16-27,
 * video_vae.cpp:17-50; architecture in docs/architecture.md:80-92). Latents are voxels [frames][h][w][channels], the
 * transformer's normalized latents; frames come out [16 h][16 w][3] RGB. */
typedef struct h3vae_config {
    uint32_t dim;       /* 2048 */
    uint32_t heads;     /* 32 (of 64 dims) */
    uint32_t ffn;       /* SwiGLU hidden, 8192 */
    uint32_t blocks;    /* 36 */
    uint32_t channels;  /* latent channels, 24 */
    uint32_t registers; /* register tokens, 4 */
    uint32_t clip;      /* latent frames a clip decodes, 7 */
    uint32_t tile;      /* latents a tile spans, 16 (256 pixels) */
    uint32_t overlap;   /* latents tiles overlap at least, 4 (64 pixels) */
    float eps;          /* norms' epsilon (0: 1e-6) */
} h3vae_config;

typedef struct h3vae_model h3vae_model;
/* A decoded frame: its index in the video and its pixels [16 h][16 w][3] in [0, 1] (count floats, host memory valid
 * during the call) -- VideoVae::FrameSink (video_vae.hpp:22). */
typedef void (*h3vae_frame_fn)(void* user, uint32_t index, const float* rgb, uint64_t count);

/* VideoVae(dir, ctx, telemetry) (video_vae.cpp:9-15): weights "synthetic:SEED" (random-init, the decoder's checkpoint
 * tensor names being in the absent mako-common sources). On `device`. */
int h3vae_create(const h3vae_config* cfg, const char* weights, int32_t device, h3vae_model** out);
/* VideoVae::decode(latents, frames, h, w, sink) (video_vae.cpp:17-50): frames = 5 n + 2; clips of 7 latent frames 5
 * apart, each 28 pixel frames of which 17 are emitted after 3 of padding, the first 5 cross-faded linearly from the
 * previous clip's last 5; ImageNet-normalized RGB reverted and clamped to [0, 1]; 17 n + 5 frames in order. */
int h3vae_decode(h3vae_model* m, const float* latents, uint32_t frames, uint32_t h, uint32_t w, h3vae_frame_fn sink, void* user);
/* H3Vae's decode of one clip (video_vae.cpp:33, decode_normalized): latents [clip][h][w][channels] (host) ->
 * canvas [4 clip][16 h][16 w][3] ImageNet-normalized RGB (host). The _device form takes and fills device memory. */
int h3vae_decode_clip(h3vae_model* m, const float* latents, uint32_t h, uint32_t w, float* canvas);
int h3vae_decode_clip_device(h3vae_model* m, const float* latents, uint32_t h, uint32_t w, float* canvas);
/* The tile layout along an axis of n latents (host; no counterpart in the reference's public interface). */
int h3vae_tile_starts(uint32_t n, uint32_t tile, uint32_t overlap, uint32_t* starts, uint32_t cap, uint32_t* count);
/* The rotary table of a tile's tokens [T][24][2] (cos, sin), T = frames th tw + specials (host). */
int h3vae_rope_table(uint32_t frames, uint32_t th, uint32_t tw, uint32_t specials, float* out);
int32_t h3vae_last_launches(h3vae_model* m);
void* h3vae_stream(h3vae_model* m);
void h3vae_destroy(h3vae_model* m);

/* Kernel level, for the decoder's parity tests: dense attention with heads of head_dim (64 or 128) over independent
 * segments (seg_rows rows every seg_stride rows; rows a multiple of seg_stride); the decoder's q/k norm and rotary on
 * qkv [rows][3][heads][64] in place (rope [T][24][2], token = row mod T); a layer norm to bf16. */
int h3k_attention_segments(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads, int32_t head_dim, int32_t rows,
                           int32_t seg_rows, int32_t seg_stride, void* out, int64_t out_row_stride, void* stream);
int h3k_vae_heads(void* qkv, int32_t rows, int32_t heads, int32_t T, const float* rope, float eps, void* stream);
int h3k_layer_norm(const float* x, int32_t rows, int32_t d, const float* w, const float* b, float eps, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* H3_C_H */
