"""ctypes binding of libh3b200.so (include/h3_c.h) for the tests and the benchmark.

The library is the product; this module only loads it and converts arguments. There is no fallback: if the shared
library is missing, `lib()` raises. Device memory for the kernel-level calls is whatever the caller passes (the
tests use torch tensors' data pointers); the model-level calls take host arrays (numpy) or device pointers.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "lib", "libh3b200.so")

H3_OK, H3_ERR_ARG, H3_ERR_CUDA, H3_ERR_STATE, H3_ERR_DEVICE = 0, 1, 2, 3, 4
EPI_BF16, EPI_F32, EPI_QKV, EPI_GATE_RESID, EPI_SWIGLU, EPI_S32 = range(6)
INT8_QKV, INT8_OUT, INT8_FC1, INT8_FC2 = 1, 2, 4, 8

# Model shapes (h3_config): the benchmark's synthetic stacks and the real MiniMax-H3.
CONFIGS = {
    # one tiny block
    "c1": dict(dim=1024, heads=8, ffn=2816, blocks=1, time_dim=512, text_dim=5120, refiner=2),
    # the 768p stack
    "c2": dict(dim=5120, heads=40, ffn=13824, blocks=48, time_dim=2560, text_dim=5120, refiner=2),
    # MiniMax-H3 itself (docs/architecture.md:23-27, 47-67 of the reference)
    "h3": dict(dim=5376, heads=56, ffn=14336, blocks=50, time_dim=2688, text_dim=5120, refiner=2),
}

# Layouts (h3_layout): latent h / w are twice the patch grid.
LAYOUTS = {
    # 512 video rows (4 frames x 8 x 16 patches) + 64 text rows
    "c1": dict(text=64, frames=4, h=16, w=32, audio=0, cond_frames=0),
    # 768p: 32 latent frames x 24 x 42 patches + 512 text rows + 256 audio rows (2 x 128 latents)
    "c2": dict(text=512, frames=32, h=48, w=84, audio=128, cond_frames=0),
    # long clip: 92 frames + one keyframe (1008 rows at t = 0.999) + 512 text + 640 audio rows
    "c5": dict(text=512, frames=92, h=48, w=84, audio=320, cond_frames=1),
    # MiniMax-H3's own 1344 x 768 x 124 frames: 37 latent frames of 24 x 42 patches, 512 text rows, 2 x 207 audio rows
    # (docs/architecture.md:28-33; tests/geometry_test.cpp:24-26 of the reference)
    "h3": dict(text=512, frames=37, h=48, w=84, audio=207, cond_frames=0),
}


class H3Error(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"h3 error {code}: {msg}")
        self.code = code


class h3_config(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_uint32), ("heads", ctypes.c_uint32), ("ffn", ctypes.c_uint32), ("blocks", ctypes.c_uint32),
                ("time_dim", ctypes.c_uint32), ("text_dim", ctypes.c_uint32), ("video_patch", ctypes.c_uint32),
                ("audio_channels", ctypes.c_uint32), ("eps", ctypes.c_float), ("refiner_blocks", ctypes.c_uint32),
                ("curve_dims", ctypes.c_uint32)]


class h3_layout_ref(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("frames", ctypes.c_uint32), ("h", ctypes.c_uint32), ("w", ctypes.c_uint32),
                ("audio", ctypes.c_uint32)]


REF_KINDS = {"image": 0, "video": 1, "audio": 2}


class h3_layout(ctypes.Structure):
    _fields_ = [("text", ctypes.c_uint32), ("frames", ctypes.c_uint32), ("h", ctypes.c_uint32), ("w", ctypes.c_uint32),
                ("audio", ctypes.c_uint32), ("cond_frames", ctypes.c_uint32), ("cond_last", ctypes.c_void_p),
                ("text_tags", ctypes.c_void_p), ("refs", ctypes.POINTER(h3_layout_ref)), ("n_refs", ctypes.c_uint32)]


class h3_world(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("size", ctypes.c_int32), ("nccl_id", ctypes.c_uint8 * 128)]


class h3k_gemm_args(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int32), ("N", ctypes.c_int32), ("K", ctypes.c_int32), ("a_chunks", ctypes.c_int32),
                ("a_rows_stride", ctypes.c_int32), ("lda", ctypes.c_int32), ("ldb", ctypes.c_int32), ("out", ctypes.c_void_p),
                ("ldo", ctypes.c_int64), ("bias", ctypes.c_void_p), ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
                ("mod", ctypes.c_void_p), ("mod_idx", ctypes.c_void_p), ("gate_slot", ctypes.c_int32), ("dim", ctypes.c_int32),
                ("rope", ctypes.c_void_p), ("qn_w", ctypes.c_void_p), ("kn_w", ctypes.c_void_p), ("eps", ctypes.c_float),
                ("inner", ctypes.c_int32), ("heads_per_rank", ctypes.c_int32), ("rows_local", ctypes.c_int32),
                ("a_scale", ctypes.c_void_p), ("b_scale", ctypes.c_void_p)]


class h3k_cube_grid(ctypes.Structure):
    _fields_ = [("dense_rows", ctypes.c_int32), ("frames", ctypes.c_int32), ("ph", ctypes.c_int32), ("pw", ctypes.c_int32)]


class h3vae_config(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_uint32), ("heads", ctypes.c_uint32), ("ffn", ctypes.c_uint32), ("blocks", ctypes.c_uint32),
                ("channels", ctypes.c_uint32), ("registers", ctypes.c_uint32), ("clip", ctypes.c_uint32), ("tile", ctypes.c_uint32),
                ("overlap", ctypes.c_uint32), ("eps", ctypes.c_float)]


# The video VAE decoder's shapes: MiniMax-H3's (docs/architecture.md:80-92 of the reference) and a small one for tests.
VAE_CONFIGS = {
    "h3": dict(dim=2048, heads=32, ffn=8192, blocks=36, channels=24, registers=4, clip=7, tile=16, overlap=4),
    "small": dict(dim=256, heads=4, ffn=512, blocks=2, channels=24, registers=4, clip=7, tile=16, overlap=4),
}

PROGRESS_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32)
FRAME_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_float), ctypes.c_uint64)
PROBE_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_float), ctypes.c_uint64)

# Every exported symbol and its signature (restype, argtypes). Tests check the library exports each of them.
_P, _I32, _U32, _I64, _U64, _F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float
SIGNATURES = {
    "h3_last_error": (ctypes.c_char_p, []),
    "h3_nccl_unique_id": (ctypes.c_int, [_P]),
    "h3_create": (ctypes.c_int, [ctypes.POINTER(h3_config), ctypes.c_char_p, _U32, _F, _U32, ctypes.POINTER(h3_world), _I32, _P]),
    "h3_set_sparse": (ctypes.c_int, [_P, _F, _U32]),
    "h3_parse_int8": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32)]),
    "h3_begin": (ctypes.c_int, [_P, _P, _U32, ctypes.POINTER(h3_layout)]),
    "h3_step": (ctypes.c_int, [_P, _P, _U64, _P, _U64, _F, _F, _P, _P]),
    "h3_step_device": (ctypes.c_int, [_P, _P, _U64, _P, _U64, _F, _F, _P, _P]),
    "h3_synchronize": (ctypes.c_int, [_P]),
    "h3_sigmas": (ctypes.c_int, [_U32, _F, _P, _P]),
    "h3_add_lora": (ctypes.c_int, [_P, ctypes.c_char_p, _F, _I32, _P, _P]),
    "h3_lora_inspect": (ctypes.c_int, [ctypes.c_char_p, _P, _U64, _P, _P, _P]),
    "h3_weight_specs": (ctypes.c_int, [ctypes.POINTER(h3_config), _P, _U64, _P]),
    "h3_save_weights": (ctypes.c_int, [_P, ctypes.c_char_p]),
    "h3_convert_weights": (ctypes.c_int, [ctypes.POINTER(h3_config), ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p]),
    "h3_check_weights": (ctypes.c_int, [ctypes.POINTER(h3_config), ctypes.c_char_p, _P, _U64]),
    "h3k_wait_selftest": (ctypes.c_int, [_U64, _P]),
    "h3_denoise": (ctypes.c_int, [_P, _P, _U64, _P, _U64, _P, _P, _U32, PROGRESS_FN, _P, _P]),
    "h3_stream": (_P, [_P]),
    "h3_set_probe": (ctypes.c_int, [_P, PROBE_FN, _P]),
    "h3_layout_rows": (_U64, [ctypes.POINTER(h3_layout)]),
    "h3_rows": (ctypes.c_int, [ctypes.POINTER(h3_layout), _P, _P, _P]),
    "h3_rope_table": (ctypes.c_int, [ctypes.POINTER(h3_layout), _P]),
    "h3_last_launches": (_I32, [_P]),
    "h3_set_timing": (ctypes.c_int, [_P, _I32]),
    "h3_last_timing": (_I32, [_P, _P, _P, _I32, _I32]),
    "h3_destroy": (None, [_P]),
    "h3k_gemm": (ctypes.c_int, [_P, _P, ctypes.POINTER(h3k_gemm_args), _I32, _I32, _P]),
    "h3k_rms_mod": (ctypes.c_int, [_P, _I64, _I32, _I32, _P, _P, _P, _I32, _I32, _I32, _F, _I32, _P, _I64, _P, _P]),
    "h3k_gate_add": (ctypes.c_int, [_P, _I64, _P, _I64, _I32, _I32, _P, _P, _I32, _P]),
    "h3k_swiglu": (ctypes.c_int, [_P, _I32, _I32, _P, _P]),
    "h3k_quant_rows_i8": (ctypes.c_int, [_P, _I64, _I32, _I32, _P, _P, _P]),
    "h3k_quant_weight": (ctypes.c_int, [_P, _I32, _I32, _P, _P, _P]),
    "h3k_heads_partial": (ctypes.c_int, [_P, _I32, _I32, _P, _P, _P, _F, _P]),
    "h3k_attention": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _P, _I64, _P]),
    "h3k_attention_bounded": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _F, _P, _I64, _P]),
    "h3k_sparse_sizes": (ctypes.c_int, [ctypes.POINTER(h3k_cube_grid), _F, _I32, _P, _P, _P, _P]),
    "h3k_sparse_select": (ctypes.c_int, [_P, _P, _I64, _I32, ctypes.POINTER(h3k_cube_grid), _F, _I32, _P, _P, _P, _P, _P, _P]),
    "h3k_cube_topk": (ctypes.c_int, [_P, _I32, ctypes.POINTER(h3k_cube_grid), _F, _I32, _P, _P, _P]),
    "h3k_video_order": (ctypes.c_int, [ctypes.POINTER(h3k_cube_grid), _P]),
    "h3k_sparse_attention": (ctypes.c_int, [_P, _P, _P, _I64, _I32, ctypes.POINTER(h3k_cube_grid), _F, _I32, _P, _I64, _P]),
    "h3k_sparse_attention_bounded": (ctypes.c_int, [_P, _P, _P, _I64, _I32, ctypes.POINTER(h3k_cube_grid), _F, _I32, _F, _P, _I64, _P]),
    "h3k_sparse_attention_noalloc": (ctypes.c_int, [_P, _P, _P, _I64, _I32, ctypes.POINTER(h3k_cube_grid), _F, _I32, _P, _I64, _P]),
    "h3k_fill_synthetic": (ctypes.c_int, [_P, _I32, _U64, _U64, _U32, _F, _F, _P]),
    "h3k_gemv_f32": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I32, _I32, _P, _P, _P]),
    "h3k_adaln": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I32, _I32, _P, _P]),
    "h3k_heads": (ctypes.c_int, [_P, _I64, _I32, _P, _P, _I32, _I32, _P, _I64, _P]),
    "h3k_check": (ctypes.c_int, [_P]),
    "h3vae_create": (ctypes.c_int, [ctypes.POINTER(h3vae_config), ctypes.c_char_p, _I32, _P]),
    "h3vae_decode": (ctypes.c_int, [_P, _P, _U32, _U32, _U32, FRAME_FN, _P]),
    "h3vae_decode_clip": (ctypes.c_int, [_P, _P, _U32, _U32, _P]),
    "h3vae_decode_clip_device": (ctypes.c_int, [_P, _P, _U32, _U32, _P]),
    "h3vae_tile_starts": (ctypes.c_int, [_U32, _U32, _U32, _P, _U32, _P]),
    "h3vae_rope_table": (ctypes.c_int, [_U32, _U32, _U32, _U32, _P]),
    "h3vae_last_launches": (_I32, [_P]),
    "h3vae_stream": (_P, [_P]),
    "h3vae_destroy": (None, [_P]),
    "h3k_attention_segments": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _P, _I64, _P]),
    "h3k_vae_heads": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _F, _P]),
    "h3k_layer_norm": (ctypes.c_int, [_P, _I32, _I32, _P, _P, _F, _P, _P]),
}

_lib = None


def lib():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with python mako-video_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc):
    if rc != H3_OK:
        raise H3Error(rc, lib().h3_last_error().decode())
    return rc


def make_config(name_or_dict, eps=1e-6):
    c = CONFIGS[name_or_dict] if isinstance(name_or_dict, str) else name_or_dict
    return h3_config(c["dim"], c["heads"], c["ffn"], c["blocks"], c["time_dim"], c.get("text_dim", 5120), 96, 32, eps,
                     c.get("refiner", 0), c.get("curve", 0))


class Layout:
    """An h3_layout plus the arrays it points at (kept alive with it). refs: reference blocks in reading order, each
    a dict(kind="image"|"video"|"audio", frames=, h=, w=, audio=)."""

    def __init__(self, text, frames, h, w, audio=0, cond_frames=0, cond_last=None, text_tags=None, refs=None):
        self.refs = [dict(kind=r["kind"], frames=1 if r["kind"] == "image" else r.get("frames", 0),
                          h=r.get("h", 0) if r["kind"] != "audio" else 0, w=r.get("w", 0) if r["kind"] != "audio" else 0,
                          audio=r.get("audio", 0) if r["kind"] != "image" else 0) for r in (refs or [])]
        self.d = dict(text=text, frames=frames, h=h, w=w, audio=audio, cond_frames=cond_frames, refs=self.refs)
        self._cl = None if cond_last is None else np.ascontiguousarray(cond_last, dtype=np.uint8)
        self._tt = None if text_tags is None else np.ascontiguousarray(text_tags, dtype=np.uint8)
        self._refs = (h3_layout_ref * max(len(self.refs), 1))(
            *[h3_layout_ref(REF_KINDS[r["kind"]], r["frames"], r["h"], r["w"], r["audio"]) for r in self.refs])
        self.c = h3_layout(text, frames, h, w, audio, cond_frames,
                           None if self._cl is None else self._cl.ctypes.data,
                           None if self._tt is None else self._tt.ctypes.data,
                           self._refs if self.refs else None, len(self.refs))

    @property
    def patch_rows(self):
        return (self.d["h"] // 2) * (self.d["w"] // 2)

    @property
    def cond_rows(self):
        n = self.d["cond_frames"] * self.patch_rows
        for r in self.refs:
            if r["kind"] != "audio":
                n += r["frames"] * (r["h"] // 2) * (r["w"] // 2)
        return n

    @property
    def cond_audio_rows(self):
        return sum(2 * r["audio"] for r in self.refs if r["kind"] != "image")

    @property
    def video_rows(self):
        return self.cond_rows + self.d["frames"] * self.patch_rows

    @property
    def audio_rows(self):
        return self.cond_audio_rows + 2 * self.d["audio"]

    @property
    def rows(self):
        return self.d["text"] + self.video_rows + self.audio_rows

    @property
    def dense_rows(self):
        return self.rows - self.d["frames"] * self.patch_rows

    @classmethod
    def named(cls, name):
        return cls(**LAYOUTS[name])


def rows(layout):
    """h3_rows: positions [S][3] f64, tags [S], roles [S]."""
    S = int(lib().h3_layout_rows(ctypes.byref(layout.c)))
    pos = np.zeros((S, 3), np.float64)
    tags = np.zeros(S, np.uint8)
    roles = np.zeros(S, np.uint8)
    check(lib().h3_rows(ctypes.byref(layout.c), pos.ctypes.data, tags.ctypes.data, roles.ctypes.data))
    return pos, tags, roles


def rope_table(layout):
    """h3_rope_table: [S][48][2] (cos, sin) per row."""
    S = int(lib().h3_layout_rows(ctypes.byref(layout.c)))
    out = np.zeros((S, 48, 2), np.float32)
    check(lib().h3_rope_table(ctypes.byref(layout.c), out.ctypes.data))
    return out


def lora_inspect(path):
    """h3_lora_inspect: (target names, rank, alpha metadata or 0)."""
    buf = ctypes.create_string_buffer(1 << 20)
    n, r, a = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_float()
    check(lib().h3_lora_inspect(str(path).encode(), buf, len(buf), ctypes.byref(n), ctypes.byref(r), ctypes.byref(a)))
    names = buf.value.decode().split("\n") if n.value else []
    return names, r.value, a.value


def sigmas(steps, shift):
    """h3_sigmas: the sampler's schedule (Engine::sigmas)."""
    out = np.zeros(max(steps, 2), np.float32)
    n = ctypes.c_uint32()
    check(lib().h3_sigmas(steps, shift, out.ctypes.data, ctypes.byref(n)))
    return out[:n.value].copy()


def packed_order(dense_rows, frames, ph, pw):
    """Row permutation of the packed order the h3k_sparse_* calls and the step use: packed row i holds layout row
    order[i] (the dense rows keep their places; the generated video rows go cube by cube)."""
    g = h3k_cube_grid(dense_rows, frames, ph, pw)
    src = np.zeros(frames * ph * pw, np.int32)
    check(lib().h3k_video_order(ctypes.byref(g), src.ctypes.data))
    return np.concatenate([np.arange(dense_rows, dtype=np.int64), dense_rows + src.astype(np.int64)])


def nccl_unique_id():
    buf = (ctypes.c_uint8 * 128)()
    check(lib().h3_nccl_unique_id(buf))
    return bytes(buf)


class Model:
    """The transformer (h3_create / h3_begin / h3_step)."""

    def __init__(self, config="c1", seed=0, int8_mask=0, sparse_ratio=0.0, sparse_local=1, rank=0, world=1, nccl_id=None,
                 device=0, eps=1e-6, weights=None):
        """weights: a checkpoint path (safetensors file or directory); None for synthetic weights from `seed`."""
        self.cfg = make_config(config, eps)
        w = None
        if world > 1:
            w = h3_world(rank, world)
            ctypes.memmove(w.nccl_id, nccl_id, 128)
        self.h = ctypes.c_void_p()
        src = str(weights).encode() if weights is not None else f"synthetic:{seed}".encode()
        check(lib().h3_create(ctypes.byref(self.cfg), src, int8_mask, sparse_ratio, sparse_local,
                              None if w is None else ctypes.byref(w), device, ctypes.byref(self.h)))
        self._probe_cb = None
        self.layout = None

    def close(self):
        if self.h:
            lib().h3_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def save_weights(self, path):
        """h3_save_weights: every weight to a safetensors file that h3_create reads back."""
        check(lib().h3_save_weights(self.h, str(path).encode()))

    def add_lora(self, path, scale=1.0, strict=True):
        """h3_add_lora: returns (merged, skipped) adapter counts."""
        merged, skipped = ctypes.c_uint32(), ctypes.c_uint32()
        check(lib().h3_add_lora(self.h, str(path).encode(), scale, 1 if strict else 0, ctypes.byref(merged), ctypes.byref(skipped)))
        return merged.value, skipped.value

    def set_sparse(self, ratio, local=1):
        check(lib().h3_set_sparse(self.h, ratio, local))

    def begin(self, text, layout):
        text = np.ascontiguousarray(text, dtype=np.float32)
        self.layout = layout
        check(lib().h3_begin(self.h, text.ctypes.data, layout.d["text"], ctypes.byref(layout.c)))

    def step(self, video, audio, t_video, t_audio):
        video = np.ascontiguousarray(video, dtype=np.float32)
        audio = np.ascontiguousarray(audio, dtype=np.float32)
        ov = np.empty_like(video)
        oa = np.empty_like(audio)
        check(lib().h3_step(self.h, video.ctypes.data, video.shape[0], audio.ctypes.data if audio.size else None, audio.shape[0],
                            t_video, t_audio, ov.ctypes.data, oa.ctypes.data if oa.size else None))
        return ov, oa

    def step_device(self, video_ptr, video_rows, audio_ptr, audio_rows, t_video, t_audio, out_video_ptr, out_audio_ptr):
        check(lib().h3_step_device(self.h, video_ptr, video_rows, audio_ptr, audio_rows, t_video, t_audio, out_video_ptr,
                                   out_audio_ptr))

    def synchronize(self):
        check(lib().h3_synchronize(self.h))

    def denoise(self, video, audio, sigma_video, sigma_audio, progress=None):
        """h3_denoise: the whole step loop on the GPU. Returns (video, audio, steps run); progress(step, steps) -> bool
        (False stops after that step)."""
        video = np.array(video, dtype=np.float32, order="C", copy=True)
        audio = np.array(audio, dtype=np.float32, order="C", copy=True)
        sv = np.ascontiguousarray(sigma_video, dtype=np.float32)
        sa = np.ascontiguousarray(sigma_audio, dtype=np.float32)
        assert sv.shape == sa.shape
        cb = None
        if progress is not None:
            cb = PROGRESS_FN(lambda user, i, n: 0 if progress(int(i), int(n)) else 1)
        ran = ctypes.c_uint32()
        check(lib().h3_denoise(self.h, video.ctypes.data, video.shape[0], audio.ctypes.data if audio.size else None, audio.shape[0],
                               sv.ctypes.data, sa.ctypes.data, sv.size, cb if cb is not None else PROGRESS_FN(), None,
                               ctypes.byref(ran)))
        return video, audio, ran.value

    @property
    def stream(self):
        return lib().h3_stream(self.h)

    def last_launches(self):
        return int(lib().h3_last_launches(self.h))

    def set_timing(self, on):
        check(lib().h3_set_timing(self.h, 1 if on else 0))

    def last_timing(self):
        """[(stage, ms)] of the last step with timing on: an entry per kernel class per block."""
        cap = 8192
        ms = (ctypes.c_float * cap)()
        names = ctypes.create_string_buffer(cap * 16)
        n = lib().h3_last_timing(self.h, ms, names, cap * 16, cap)
        labels = names.raw.split(b"\0")[:n]
        return [(labels[i].decode(), ms[i]) for i in range(n)]

    def timing_by_class(self):
        """{stage: (total ms, count)} of the last step with timing on."""
        out = {}
        for name, t in self.last_timing():
            tot, cnt = out.get(name, (0.0, 0))
            out[name] = (tot + t, cnt + 1)
        return out

    def set_probe(self, fn):
        """fn(name, layer, numpy array) for each probe of the following steps (None to stop)."""
        if fn is None:
            self._probe_cb = None
            check(lib().h3_set_probe(self.h, PROBE_FN(), None))
            return

        def cb(user, name, layer, data, n):
            fn(name.decode(), layer, np.ctypeslib.as_array(data, shape=(n,)).copy())

        self._probe_cb = PROBE_FN(cb)
        check(lib().h3_set_probe(self.h, self._probe_cb, None))


def weight_specs(config, eps=1e-6):
    """h3_weight_specs: [(name, dtype, shape)] of every tensor a checkpoint for this shape holds (host only)."""
    cfg = make_config(config, eps)
    n = ctypes.c_uint32()
    check(lib().h3_weight_specs(ctypes.byref(cfg), None, 0, ctypes.byref(n)))
    buf = ctypes.create_string_buffer(1 << 22)
    check(lib().h3_weight_specs(ctypes.byref(cfg), buf, len(buf), ctypes.byref(n)))
    out = []
    for line in buf.value.decode().splitlines():
        name, dtype, shape = line.split()
        out.append((name, dtype, tuple(int(v) for v in shape.split("x"))))
    assert len(out) == n.value
    return out


def check_weights(config, path, eps=1e-6):
    """h3_check_weights: "" when the checkpoint fits the shape, else its first problem (host only)."""
    cfg = make_config(config, eps)
    msg = ctypes.create_string_buffer(4096)
    rc = lib().h3_check_weights(ctypes.byref(cfg), str(path).encode(), msg, len(msg))
    return "" if rc == H3_OK else (msg.value.decode() or lib().h3_last_error().decode())


def convert_weights(config, src, dst, renames=None, interleaved=False, eps=1e-6):
    """h3_convert_weights: src (file or directory) rewritten at dst in this library's layout; renames {this library's
    name: the source's}; interleaved: the source keeps each head's q, k, v rows together (host only)."""
    cfg = make_config(config, eps)
    lines = [f"{a} {b}" for a, b in (renames or {}).items()]
    if interleaved:
        lines.append("qkv_layout interleaved")
    check(lib().h3_convert_weights(ctypes.byref(cfg), str(src).encode(), str(dst).encode(), "\n".join(lines).encode()))


def vae_tile_starts(n, tile=16, overlap=4):
    """h3vae_tile_starts: the tile layout along an axis of n latents."""
    buf = (ctypes.c_uint32 * 256)()
    cnt = ctypes.c_uint32()
    check(lib().h3vae_tile_starts(n, tile, overlap, buf, 256, ctypes.byref(cnt)))
    return [buf[i] for i in range(cnt.value)]


def vae_rope_table(frames, th, tw, specials):
    T = frames * th * tw + specials
    out = np.zeros((T, 24, 2), np.float32)
    check(lib().h3vae_rope_table(frames, th, tw, specials, out.ctypes.data))
    return out


class VideoDecoder:
    """The video VAE decoder (h3vae_create / h3vae_decode / h3vae_decode_clip)."""

    def __init__(self, config="small", seed=0, device=0, eps=1e-6):
        c = VAE_CONFIGS[config] if isinstance(config, str) else config
        self.cfg = dict(c)
        self.c = h3vae_config(c["dim"], c["heads"], c["ffn"], c["blocks"], c["channels"], c["registers"], c["clip"], c["tile"],
                              c["overlap"], eps)
        self.h = ctypes.c_void_p()
        check(lib().h3vae_create(ctypes.byref(self.c), f"synthetic:{seed}".encode(), device, ctypes.byref(self.h)))

    def close(self):
        if self.h:
            lib().h3vae_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def decode_clip(self, latents):
        """latents [clip][h][w][channels] -> canvas [4 clip][16 h][16 w][3] (ImageNet-normalized)."""
        lat = np.ascontiguousarray(latents, dtype=np.float32)
        clip, h, w, _ = lat.shape
        out = np.zeros((clip * 4, h * 16, w * 16, 3), np.float32)
        check(lib().h3vae_decode_clip(self.h, lat.ctypes.data, h, w, out.ctypes.data))
        return out

    def decode_clip_device(self, lat_ptr, h, w, out_ptr):
        check(lib().h3vae_decode_clip_device(self.h, lat_ptr, h, w, out_ptr))

    def decode(self, latents, sink=None):
        """latents [5 n + 2][h][w][channels] -> the 17 n + 5 frames [16 h][16 w][3] in [0, 1] (a list, or each handed to
        sink(index, frame))."""
        lat = np.ascontiguousarray(latents, dtype=np.float32)
        frames, h, w, _ = lat.shape
        got = []

        def cb(user, index, rgb, count):
            a = np.ctypeslib.as_array(rgb, shape=(count,)).reshape(h * 16, w * 16, 3)
            if sink is None:
                got.append(a.copy())
            else:
                sink(int(index), a)

        fn = FRAME_FN(cb)
        check(lib().h3vae_decode(self.h, lat.ctypes.data, frames, h, w, fn, None))
        return got

    @property
    def stream(self):
        return lib().h3vae_stream(self.h)

    def last_launches(self):
        return int(lib().h3vae_last_launches(self.h))
