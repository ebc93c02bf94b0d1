"""CPU oracle of the MiniMax-H3 transformer step -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only as the checker or
the timed CPU baseline. The product (libh3b200.so) never calls it.

PARITY STATUS: partially pinned. The reference's step lives in the mako-common submodule, which is empty in the
reference mount, and its Python reference (diffusers' MiniMaxH3Transformer3DModel, "diffusers from git", no pinned
version, README.md:198-199) is not installed. So this is a restatement of the step from the reference's prose and
harness, not a run of its code:
  * pinned against the reference's own code: the time embedding and AdaLN projection formula
    (tools/check_pruned_curve.py:58-67, executed from the reference file to make tests/golden/time_adaln.npz), the
    rotary frequencies (tools/dump_h3_ref.py:140-141, likewise), the probe comparison metric
    (tests/h3_ref_test.cpp:67-90) and its tolerances (tests/h3_ref_test.cpp:219-249);
  * unpinned (restated from docs/architecture.md:35-70,112-133 and docs/performance.md:120-126, no golden vectors
    exist): the block internals, the rotary position grid, the sparse selection's exact rules.

Semantics (each a choice where the reference's prose leaves it open):
  * fp32 compute with bf16-stored weights (tools/dump_h3_ref.py:150-166: BF16 weights upcast per module);
    silu(temb) rounded to bf16 before the AdaLN projections (dump_h3_ref.py:150-151; architecture.md:50);
    the text embeddings enter in bf16 (dump_h3_ref.py:183-184);
  * time embedding: 256 sinusoids, cos half first, freq_i = exp(-ln(1e4) i / 128), argument t in [0, 1]
    (check_pruned_curve.py:58-64) -> Linear 256->d -> SiLU -> Linear d->time_dim (architecture.md:49-51);
  * AdaLN per block: [U][3 modalities][6][d], the six (shift, scale, gate) of attention then of the FFN;
    the final layer [U][2][d] (shift, scale) per level (architecture.md:50-53,66);
  * block (architecture.md:61-65): y = RMSNorm(x) * w * (1 + scale) + shift; q/k/v; per-head RMS norm of q and
    k with 128-wide weights; rotary on 96 of 128 dims (first 48 paired with the second 48; 16 frequencies per
    axis t, h, w; base 10000); softmax attention; x += gate * out(o); the same for the SwiGLU FFN with fc1
    stored [gate; value] (architecture.md:112-114);
  * final: RMSNorm (no weight) * (1 + scale) + shift per row's level, fp32 heads d->96 (video rows) and
    d->32 (audio rows) (architecture.md:66-67).
"""
import math
import re

import numpy as np
import torch

M64 = (1 << 64) - 1

# ------------------------------------------------------------------------------------------ synthetic values


def _splitmix64_np(x):
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return x ^ (x >> np.uint64(31))


def _splitmix64_int(x):
    x = (x + 0x9E3779B97F4A7C15) & M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M64
    return x ^ (x >> 31)


def bf16_round(a):
    """Round fp32 to bf16 (nearest even), returned as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def synthetic(n, seed, tensor_id, mean=0.0, stdev=0.02, bf16=False):
    """Value i = mean + stdev * IH4(seed, tensor_id, i): the centred sum of four 16-bit fields of a splitmix64 hash
    (an Irwin-Hall approximation of a unit normal), one fp32 multiply and one fp32 add, then optional bf16
    rounding. Bit-identical to the library's fill_synthetic. Large tensors go through the same arithmetic written as
    a C loop (oracle/h3_exact.c: h3x_synthetic; pinned to synthetic_np by a CPU test): the numpy form takes minutes
    for a 5120-wide model's weights."""
    if n >= (1 << 20):
        from oracle import exact
        key = _splitmix64_int((seed * 0x632BE59BD9B4E019 + tensor_id) & M64)
        norm = 1.0 / math.sqrt((65536.0 * 65536.0 - 1.0) / 3.0)
        return exact.synthetic(n, key, np.float32(mean), np.float32(float(np.float32(stdev)) * norm), bf16)
    return synthetic_np(n, seed, tensor_id, mean, stdev, bf16)


def synthetic_np(n, seed, tensor_id, mean=0.0, stdev=0.02, bf16=False):
    """The numpy definition of `synthetic`."""
    key = _splitmix64_int((seed * 0x632BE59BD9B4E019 + tensor_id) & M64)
    with np.errstate(over="ignore"):
        h = _splitmix64_np(np.uint64(key) + np.arange(n, dtype=np.uint64))
    s = ((h & np.uint64(0xFFFF)).astype(np.int64) + ((h >> np.uint64(16)) & np.uint64(0xFFFF)).astype(np.int64) +
         ((h >> np.uint64(32)) & np.uint64(0xFFFF)).astype(np.int64) + (h >> np.uint64(48)).astype(np.int64) - 131070)
    norm = 1.0 / math.sqrt((65536.0 * 65536.0 - 1.0) / 3.0)
    k = np.float32(float(np.float32(stdev)) * norm)
    v = np.float32(mean) + k * s.astype(np.float32)
    return bf16_round(v) if bf16 else v.astype(np.float32)


# tensor ids, as the library assigns them
T_IN_W, T_IN_B, T_OUT_W, T_OUT_B, VP_W, VP_B, AP_W, AP_B, COND_W, COND_B, FADA_W, FADA_B, HV_W, HV_B, HA_W, HA_B = range(1, 17)
REFINER_NORM = 17
CURVE_TABLE = 18  # pruned checkpoints: adaln_t_table [1025][curve]
CURVE_STD = 4.0
BLOCK_BASE, BLOCK_STRIDE = 100, 20
REFINER_BASE = 60  # token refiner block r at REFINER_BASE + BLOCK_STRIDE * r (r < 2), the block sub-ids without ADA_*
ADA_W, ADA_B, NORM1, QKV_W, QKV_B, QN, KN, OUT_W, OUT_B, NORM2, FC1_W, FC1_B, FC2_W, FC2_B = range(14)


def make_weights(cfg, seed, blocks=None):
    """The model's synthetic weights as fp32 torch tensors (bf16-valued where the model stores bf16)."""
    d, H, F, td, tx = cfg["dim"], cfg["heads"], cfg["ffn"], cfg["time_dim"], cfg.get("text_dim", 5120)
    inner = H * 128
    L = cfg["blocks"] if blocks is None else blocks
    t = lambda n, tid, shape, mean=0.0, bf16=False: torch.from_numpy(synthetic(n, seed, tid, mean, 0.02, bf16).reshape(shape))
    K8 = cfg.get("curve", 0)  # pruned checkpoint: the AdaLN projections read an 8-point curve instead of silu(temb)
    ka = K8 if K8 else td
    w = {
        "vp_w": t(d * 96, VP_W, (d, 96), bf16=True), "vp_b": t(d, VP_B, (d,)),
        "ap_w": t(d * 32, AP_W, (d, 32), bf16=True), "ap_b": t(d, AP_B, (d,)),
        "cond_w": t(d * tx, COND_W, (d, tx), bf16=True), "cond_b": t(d, COND_B, (d,)),
        "fada_w": t(2 * d * ka, FADA_W, (2 * d, ka), bf16=not K8), "fada_b": t(2 * d, FADA_B, (2 * d,)),
        "hv_w": t(96 * d, HV_W, (96, d)), "hv_b": t(96, HV_B, (96,)),
        "ha_w": t(32 * d, HA_W, (32, d)), "ha_b": t(32, HA_B, (32,)),
        "blocks": [],
    }
    if K8:
        w["curve_table"] = torch.from_numpy(synthetic(1025 * K8, seed, CURVE_TABLE, 0.0, CURVE_STD).reshape(1025, K8))
    else:
        w.update({"t_in_w": t(d * 256, T_IN_W, (d, 256)), "t_in_b": t(d, T_IN_B, (d,)),
                  "t_out_w": t(td * d, T_OUT_W, (td, d)), "t_out_b": t(td, T_OUT_B, (td,))})
    def block(b):
        return {
            "norm1": t(d, b + NORM1, (d,), mean=1.0),
            "qkv_w": t(3 * inner * d, b + QKV_W, (3 * inner, d), bf16=True), "qkv_b": t(3 * inner, b + QKV_B, (3 * inner,)),
            "qn": t(128, b + QN, (128,), mean=1.0), "kn": t(128, b + KN, (128,), mean=1.0),
            "out_w": t(d * inner, b + OUT_W, (d, inner), bf16=True), "out_b": t(d, b + OUT_B, (d,)),
            "norm2": t(d, b + NORM2, (d,), mean=1.0),
            "fc1_w": t(2 * F * d, b + FC1_W, (2 * F, d), bf16=True), "fc1_b": t(2 * F, b + FC1_B, (2 * F,)),
            "fc2_w": t(d * F, b + FC2_W, (d, F), bf16=True), "fc2_b": t(d, b + FC2_B, (d,)),
        }

    for l in range(L):
        b = BLOCK_BASE + BLOCK_STRIDE * l
        w["blocks"].append(dict(block(b), ada_w=t(18 * d * ka, b + ADA_W, (18 * d, ka), bf16=not K8),
                                ada_b=t(18 * d, b + ADA_B, (18 * d,))))
    w["refiner"] = [block(REFINER_BASE + BLOCK_STRIDE * r) for r in range(cfg.get("refiner", 0))]
    if w["refiner"]:
        w["refiner_norm"] = t(d, REFINER_NORM, (d,), mean=1.0)
    return w


# ------------------------------------------------------------------------------------------------- layout


def video_time(f):
    """Latent frame f's time position in audio-latent units (40 a second): 5/3 x the video frames before it, the VAE
    packing 17 frames into 5 latents as (1, 4, 4, 4, 4) (architecture.md:35-40)."""
    within = (0, 1, 5, 9, 13)
    return 5.0 / 3.0 * (17 * (f // 5) + within[f % 5])


def layout_rows(L):
    """H3::rows restated: positions [S][3] f64, tags, roles for [text | keyframe rows or reference blocks | audio (left
    then right) | generated video] (architecture.md:35-45 for the target's rows; :203-215 for the reference blocks:
    one clock from the text's length, a picture one slot, a soundtrack one slot a latent at the ends of its block's
    width axis, a video's soundtrack and frames from one origin with the clock advanced by the longer span; the
    generated rows from where the clock ends). Roles: 0 text, 1 conditioning video, 2 reference audio, 3 audio,
    4 video. Reference blocks: L["refs"] = [dict(kind="image"|"video"|"audio", frames, h, w, audio)]."""
    T, Fr, h, w, A, CF = L["text"], L["frames"], L["h"], L["w"], L.get("audio", 0), L.get("cond_frames", 0)

    def axes(hh, ww):
        ph_, pw_ = hh // 2, ww // 2
        nrm = math.sqrt(ph_ * pw_)
        return (ph_, pw_, lambda y: (y + 0.5 - ph_ / 2.0) / nrm * 32.0, lambda x: (x + 0.5 - pw_ / 2.0) / nrm * 32.0)

    ph, pw, hp, wp = axes(h, w)
    pos, tags, roles = [], [], []
    tt = L.get("text_tags")
    for i in range(T):
        pos.append((float(i), 0.0, 0.0)); tags.append(1 if tt is None else int(tt[i])); roles.append(0)

    def frame(t, grid, role):
        gph, gpw, ghp, gwp = grid
        for y in range(gph):
            for x in range(gpw):
                pos.append((t, ghp(y), gwp(x))); tags.append(0); roles.append(role)

    def sound(t0, n, grid, role):
        gwp, gpw = grid[3], grid[1]
        for c in range(2):
            for a in range(n):
                pos.append((float(t0 + a), 0.0, gwp(0 if c == 0 else gpw - 1))); tags.append(2); roles.append(role)

    clock = float(T)
    cl = L.get("cond_last") or []
    for k in range(CF):
        frame(clock + video_time(max(Fr - 1, 0) if (k < len(cl) and cl[k]) else 0), (ph, pw, hp, wp), 1)
    for r in L.get("refs") or []:
        if r["kind"] == "image":
            frame(clock, axes(r["h"], r["w"]), 1)
            clock += 1.0
        elif r["kind"] == "audio":
            sound(clock, r["audio"], (ph, pw, hp, wp), 2)
            clock += r["audio"]
        else:
            g = axes(r["h"], r["w"])
            sound(clock, r.get("audio", 0), g, 2)
            for f in range(r["frames"]):
                frame(clock + video_time(f), g, 1)
            clock += max(float(r.get("audio", 0)), video_time(r["frames"]))
    sound(clock, A, (ph, pw, hp, wp), 3)
    for f in range(Fr):
        frame(clock + video_time(f), (ph, pw, hp, wp), 4)
    return np.array(pos, np.float64).reshape(-1, 3), np.array(tags, np.uint8), np.array(roles, np.uint8)


def rope_inv_freq():
    """16 frequencies per axis of base 10000 (dump_h3_ref.py:140-141: 1 / 10000^(arange(0, 32, 2) / 32))."""
    return np.array([np.float32(1.0 / 10000.0 ** (np.float32(2 * i) / np.float32(32.0))) for i in range(16)], np.float32)


def rope_table(pos):
    """[S][48][2] (cos, sin): angle = float(pos_axis) * inv_freq in fp32, cos/sin of that angle."""
    f = rope_inv_freq()
    ang = (pos.astype(np.float32)[:, :, None] * f[None, None, :]).reshape(pos.shape[0], 48)
    a = ang.astype(np.float64)
    return np.stack([np.cos(a), np.sin(a)], -1).astype(np.float32)


# ------------------------------------------------------------------------------------------------ the step


def time_embedding(levels, w):
    """temb [U][time_dim] and bf16(silu(temb)) (check_pruned_curve.py:58-64; architecture.md:49-51)."""
    emb = np.zeros((len(levels), 256), np.float32)
    for u, t in enumerate(levels):
        for i in range(128):
            fr = np.float32(math.exp(-math.log(10000.0) * i / 128.0))
            a = np.float32(t) * fr
            emb[u, i] = np.float32(math.cos(float(a)))
            emb[u, 128 + i] = np.float32(math.sin(float(a)))
    e = torch.from_numpy(emb)
    h = torch.nn.functional.silu(e @ w["t_in_w"].T + w["t_in_b"])
    temb = h @ w["t_out_w"].T + w["t_out_b"]
    s = torch.from_numpy(bf16_round(torch.nn.functional.silu(temb).numpy()))
    return temb, s


def curve_points(levels, table):
    """Pruned checkpoints (architecture.md:57-60): the 8-point curve c(t) read from adaln_t_table [1025][8] at
    t * 1024 with linear interpolation, clamped to the table (tools/check_pruned_curve.py:66-70, `c_of`, the t * 1024
    hypothesis the reference implements); in double from the float level and table, rounded to float at the end, as
    the library does it. [U][8]."""
    tab = np.asarray(table, np.float32).astype(np.float64)
    out = np.zeros((len(levels), tab.shape[1]), np.float32)
    for u, t in enumerate(levels):
        pos = min(max(float(np.float32(t)) * 1024.0, 0.0), 1024.0)
        i0 = min(int(math.floor(pos)), 1023)
        wt = pos - i0
        out[u] = ((1.0 - wt) * tab[i0] + wt * tab[i0 + 1]).astype(np.float32)
    return torch.from_numpy(out)


def rms(x, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def rope(x, cs):
    """x [S][H][128]; cs [S][48][2]: dims j and j + 48 (j < 48) rotate by angle j; dims 96..127 pass."""
    c = cs[:, None, :, 0]
    s = cs[:, None, :, 1]
    a, b, rest = x[..., :48], x[..., 48:96], x[..., 96:]
    return torch.cat([a * c - b * s, b * c + a * s, rest], -1)


def attention(q, k, v, allowed=None):
    """softmax(q k^T / sqrt(128)) v per head; q, k, v [S][H][128]; allowed [H][S][S] bool or None."""
    qh, kh, vh = q.permute(1, 0, 2), k.permute(1, 0, 2), v.permute(1, 0, 2)
    out = torch.empty_like(qh)
    S = q.shape[0]
    chunk = max(1, min(S, (1 << 26) // max(S, 1)))
    for h in range(qh.shape[0]):
        for i in range(0, S, chunk):
            s = (qh[h, i:i + chunk] @ kh[h].T) / math.sqrt(128.0)
            if allowed is not None:
                s = s.masked_fill(~allowed[h, i:i + chunk], float("-inf"))
            out[h, i:i + chunk] = torch.softmax(s, -1) @ vh[h]
    return out.permute(1, 0, 2)


def quant_rows(x):
    """Symmetric per-row int8 of fp32 values (already bf16-valued): scale = max|x| / 127,
    q = rint(x * (127 / max|x|)) clamped to +-127 (perf.md:122-125; quant_rows_i8)."""
    x = np.ascontiguousarray(x, np.float32)
    amax = np.abs(x).max(-1).astype(np.float32)
    inv = np.where(amax > 0, np.float32(127.0) / np.where(amax > 0, amax, np.float32(1)), np.float32(0)).astype(np.float32)
    q = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    return q, (amax / np.float32(127.0)).astype(np.float32)


def int8_linear(x_bf16vals, w, b):
    """The reference's int8 dequant path: per-row int8 of the activations and of the weight's rows, int32 (exact
    here in int64) dot products, times the row and column scales, plus the bias."""
    qa, sa = quant_rows(x_bf16vals.numpy())
    qw, sw = quant_rows(w.numpy())
    acc = qa.astype(np.int64) @ qw.astype(np.int64).T
    y = acc.astype(np.float32) * (sa[:, None] * sw[None, :])
    return torch.from_numpy(y) + b


def bf(t):
    return torch.from_numpy(bf16_round(t.numpy()))


def refine(cfg, w, x, R, eps):
    """The token refiner over the text rows after condition_proj (architecture.md:25-27: "a two-block token refiner
    (plain pre-norm blocks, no rotary positions), then its final RMS norm"): per block x += attn(norm1(x)),
    x += swiglu_ffn(norm2(x)), with the step's widths, per-head q/k RMS norms, no modulation (no gates) and no rotary
    positions; then x = RMSNorm(x) * refiner_norm. The block internals beyond that sentence are this build's choice
    (the refiner's code is not in the reference tree)."""
    if not w.get("refiner"):
        return x
    H, F = cfg["heads"], cfg["ffn"]
    T = x.shape[0]
    for B in w["refiner"]:
        h = rms(x, eps) * B["norm1"]
        qkv = (R(h) @ B["qkv_w"].T + B["qkv_b"]).reshape(T, 3, H, 128)
        q = R(rms(qkv[:, 0], eps) * B["qn"])
        k = R(rms(qkv[:, 1], eps) * B["kn"])
        v = R(qkv[:, 2])
        o = attention(q, k, v).reshape(T, H * 128)
        x = x + (R(o) @ B["out_w"].T + B["out_b"])
        h = rms(x, eps) * B["norm2"]
        gv = R(h) @ B["fc1_w"].T + B["fc1_b"]
        a = torch.nn.functional.silu(gv[:, :F]) * gv[:, F:]
        x = x + (R(a) @ B["fc2_w"].T + B["fc2_b"])
    return rms(x, eps) * w["refiner_norm"]


def step(cfg, w, L, text, video, audio, t_video, t_audio, allowed_fn=None, int8=0, probes=None, eps=1e-6,
         round_activations=False):
    """One forward: velocities for every video row [V][96] (conditioning rows first) and audio row [A][32] (reference
    soundtrack rows first), in the inputs' row order.
    allowed_fn(block, q, k) -> [H][S][S] bool restricts attention (sparse); int8 a mask (1 qkv, 2 out, 4 fc1, 8 fc2)
    switching those projections to the int8 dequant path; probes(name, layer, array) sees txt (the text rows after the
    token refiner), temb, mod0, x0, block l and norm_out. round_activations rounds every GEMM and attention input to bf16 as the GPU path does."""
    d, H, F = cfg["dim"], cfg["heads"], cfg["ffn"]
    T = L["text"]
    pos, tags, roles = layout_rows(L)
    S = len(roles)
    video_rows = np.nonzero((roles == 1) | (roles == 4))[0]  # the video input's rows in sequence order
    audio_rows = np.nonzero((roles == 2) | (roles == 3))[0]  # the audio input's rows in sequence order
    V, A = len(video_rows), len(audio_rows)
    C = int((roles == 1).sum())
    CA = int((roles == 2).sum())
    cs = torch.from_numpy(rope_table(pos))
    R = (lambda t: bf(t)) if round_activations else (lambda t: t)
    # levels: video/text, audio, conditioning video (max(t_video, 0.999)), reference audio (1), in order of first
    # appearance (architecture.md:38-42)
    levels = []

    def lv(t):
        if t not in levels:
            levels.append(t)
        return levels.index(t)

    t_cond = max(np.float32(t_video), np.float32(0.999))
    lv_v = lv(np.float32(t_video))
    lv_a = lv(np.float32(t_audio)) if A - CA else lv_v
    lv_c = lv(t_cond) if C else lv_v
    lv_r = lv(np.float32(1.0)) if CA else lv_v
    lvl = np.array([lv_a if r == 3 else (lv_c if r == 1 else (lv_r if r == 2 else lv_v)) for r in roles], np.int64)
    midx = torch.from_numpy(lvl * 3 + tags.astype(np.int64))
    U = len(levels)
    if "curve_table" in w:
        s = curve_points(levels, w["curve_table"])  # no time embedder: the projections read the curve, no SiLU
    else:
        temb, s = time_embedding(levels, w)
        if probes:
            probes("temb", -1, temb.numpy())
    # packed input
    x = torch.zeros(S, d)
    if T:
        xt = refine(cfg, w, bf(torch.from_numpy(np.asarray(text, np.float32))) @ w["cond_w"].T + w["cond_b"], R, eps)
        x[:T] = xt
        if probes:
            probes("txt", -1, xt.numpy().copy())
    vin = torch.from_numpy(np.asarray(video, np.float32).reshape(V, 96))
    ain = torch.from_numpy(np.asarray(audio, np.float32).reshape(A, 32))
    vi, ai = torch.from_numpy(video_rows), torch.from_numpy(audio_rows)
    if V:
        x[vi] = R(vin) @ w["vp_w"].T + w["vp_b"]
    if A:
        x[ai] = R(ain) @ w["ap_w"].T + w["ap_b"]
    if probes:
        probes("x0", -1, x.numpy().copy())

    def lin(a, W, B, use_int8):
        if use_int8:
            return int8_linear(bf(a), W, B)
        return R(a) @ W.T + B

    for l, B in enumerate(w["blocks"]):
        mod = (s @ B["ada_w"].T + B["ada_b"]).reshape(U * 3, 6, d)
        if probes and l == 0:
            probes("mod0", -1, mod.reshape(U, 18 * d).numpy().copy())
        m = mod[midx]  # [S][6][d]
        h = rms(x, eps) * B["norm1"] * (1 + m[:, 1]) + m[:, 0]
        qkv = lin(h, B["qkv_w"], B["qkv_b"], int8 & 1).reshape(S, 3, H, 128)
        q = rope(rms(qkv[:, 0], eps) * B["qn"], cs)
        k = rope(rms(qkv[:, 1], eps) * B["kn"], cs)
        v = qkv[:, 2]
        q, k, v = R(q), R(k), R(v)
        allowed = allowed_fn(l, q, k) if allowed_fn else None
        o = attention(q, k, v, allowed).reshape(S, H * 128)
        x = x + m[:, 2] * lin(o, B["out_w"], B["out_b"], int8 & 2)
        h = rms(x, eps) * B["norm2"] * (1 + m[:, 4]) + m[:, 3]
        gv = lin(h, B["fc1_w"], B["fc1_b"], int8 & 4)
        a = torch.nn.functional.silu(gv[:, :F]) * gv[:, F:]
        x = x + m[:, 5] * lin(a, B["fc2_w"], B["fc2_b"], int8 & 8)
        if probes:
            probes("block", l, x.numpy().copy())
    fm = (s @ w["fada_w"].T + w["fada_b"]).reshape(U, 2, d)[torch.from_numpy(lvl)]
    xn = rms(x, eps) * (1 + fm[:, 1]) + fm[:, 0]
    if probes:
        probes("norm_out", -1, xn.numpy().copy())
    out_v = xn[vi] @ w["hv_w"].T + w["hv_b"]
    out_a = xn[ai] @ w["ha_w"].T + w["ha_b"]
    return out_v.numpy(), out_a.numpy()


# ---------------------------------------------------------------------------------------------- LoRA merge


def apply_lora(cfg, w, adapters, scale, alpha=None):
    """TransformerRuntime::add_lora restated (architecture.md:108-116): for each Diffusers-named adapter
    {target: (A [r][in], B [out][r])}, W += scale * alpha / r * B A in fp32, the sum rounded to bf16. The q/k/v
    targets are the stacked thirds of qkv_w; ff.net.0.proj is [value; gate] in Diffusers and [gate; value] here (rows
    rotated by half); adaln_proj.linear's rows go from (chunk, modality) to (modality, chunk) (h3_ref_test.cpp:229-241).
    Targets that are not block matrices are skipped. Returns the number merged."""
    d, inner, F = cfg["dim"], cfg["heads"] * 128, cfg["ffn"]
    merged = 0
    for tgt, (A, B) in adapters.items():
        m = re.match(r"transformer_blocks\.(\d+)\.(.+)$", tgt)
        if not m:
            continue
        blk, mod = int(m.group(1)), m.group(2)
        A, B = torch.as_tensor(A, dtype=torch.float32), torch.as_tensor(B, dtype=torch.float32)
        r = A.shape[0]
        s = scale * (alpha if alpha else r) / r
        delta = s * (B @ A)
        out = delta.shape[0]
        if mod in ("attn.to_q", "attn.to_k", "attn.to_v"):
            key, rows = "qkv_w", torch.arange(out) + {"attn.to_q": 0, "attn.to_k": inner, "attn.to_v": 2 * inner}[mod]
        elif mod == "attn.to_out.0":
            key, rows = "out_w", torch.arange(out)
        elif mod == "ff.net.0.proj":
            key, rows = "fc1_w", (torch.arange(out) + F) % (2 * F)
        elif mod == "ff.net.2":
            key, rows = "fc2_w", torch.arange(out)
        elif mod == "adaln_proj.linear":
            i = torch.arange(out)
            c, md, j = (i // d) // 3, (i // d) % 3, i % d
            key, rows = "ada_w", (md * 6 + c) * d + j
        else:
            continue
        W = w["blocks"][blk][key]
        W[rows] = bf(W[rows] + delta)
        merged += 1
    return merged


# ---------------------------------------------------------------------------------------------- the sampler


def sigmas(steps, shift):
    """Engine::sigmas restated (src/video/engine.cpp:71-88): torch.linspace(1, 0, steps) in float32 (first half from
    the start, second half from the end), shifted by s x / (1 + (s - 1) x) in float32, consecutive repeats dropped."""
    f = np.float32
    step = (f(0.0) - f(1.0)) / f(steps - 1)
    out = []
    for i in range(steps):
        base = f(1.0) + f(i) * step if i < steps // 2 else f(0.0) - f(steps - 1 - i) * step
        v = f(shift) * base / (f(1.0) + (f(shift) - f(1.0)) * base)
        if not out or out[-1] != v:
            out.append(v)
    return np.array(out, np.float32)


def euler(x, v, t, sigma, sigma_next):
    """The sampler's Euler move (src/video/engine.cpp:705-711) in float32, each operation rounded on its own."""
    f = np.float32
    st, ratio = f(1.0) - f(t), f(sigma_next) / f(sigma)
    x = np.asarray(x, np.float32)
    x0 = x + st * np.asarray(v, np.float32)
    return ratio * x + (f(1.0) - ratio) * x0


# -------------------------------------------------------------------------------------- comparison metric


def diff(got, want, width):
    """tests/h3_ref_test.cpp:67-90: relative RMS error over everything and the lowest cosine of a row of `width`."""
    g = np.asarray(got, np.float64).reshape(-1, width)
    r = np.asarray(want, np.float64).reshape(-1, width)
    rel = math.sqrt(((g - r) ** 2).sum() / max((r ** 2).sum(), 1e-300))
    gw = (g * r).sum(1)
    gg = (g * g).sum(1)
    ww = (r * r).sum(1)
    ok = (gg > 0) & (ww > 0)
    cos = np.where(ok, gw / np.sqrt(np.where(ok, gg * ww, 1.0)), 1.0)
    return rel, float(cos.min()) if cos.size else 1.0
