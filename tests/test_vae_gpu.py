"""The video VAE decoder (MiniMax-H3's ViT decoder, docs/architecture.md:80-92 and src/video/video_vae.cpp:17-50 of
the reference) through the C ABI against the CPU oracle (oracle/vae_oracle.py) on the same synthetic weights and
latents: its kernels one by one (attention with 64-dim heads over independent tiles, the q/k norm and rotary, the
layer norm), one clip's canvas, and the clip-by-clip loop with its cross-fades. Tolerances: rel L2 <= 1e-2 and lowest
row cosine >= 0.999 for bf16 results; attention kernels as the step's (1e-2)."""
import ctypes
import math

import numpy as np
import pytest
import torch

import h3b200 as H
from oracle import h3_oracle as O, vae_oracle as V

pytestmark = pytest.mark.gpu


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def sync():
    H.check(H.lib().h3k_check(stream()))


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("hd,seg_rows,segs,heads", [(64, 1797, 3, 2), (64, 300, 4, 3), (64, 130, 1, 2), (128, 700, 3, 2)])
def test_attention_over_segments(cuda, hd, seg_rows, segs, heads):
    """Each segment's queries see only that segment's keys (the decoder's tiles in one batch), 64- or 128-dim heads;
    ragged segment lengths (not multiples of 128) so tiles straddle segment ends."""
    S = seg_rows * segs
    g = torch.Generator().manual_seed(hd + seg_rows)
    qkv = (torch.randn(S, 3, heads, hd, generator=g) * 1.3).bfloat16()
    t = qkv.to(cuda)
    out = torch.zeros(S, heads, hd, device=cuda, dtype=torch.bfloat16)
    H.check(H.lib().h3k_attention_segments(ptr(t[:, 0]), ptr(t[:, 1]), ptr(t[:, 2]), 3 * heads * hd, heads, hd, S, seg_rows, seg_rows,
                                           ptr(out), heads * hd, stream()))
    sync()
    got = out.float().cpu()
    for s in range(segs):
        r = slice(s * seg_rows, (s + 1) * seg_rows)
        q, k, v = qkv[r, 0].float(), qkv[r, 1].float(), qkv[r, 2].float()
        want = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd), -1)
        want = torch.einsum("hqk,khd->qhd", want, v)
        assert rel(got[r], want) < 1e-2, s
        assert O.diff(got[r].numpy(), want.numpy(), hd)[1] > 0.999


def test_vae_heads_norm_and_rotary(cuda):
    rows, heads, frames, th, tw, R = 2 * (7 * 4 * 5 + 5), 3, 7, 4, 5, 5
    T = frames * th * tw + R
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(rows, 3, heads, 64, generator=g).bfloat16()
    rope = torch.from_numpy(V.rope_table(frames, th, tw, R))
    t = qkv.to(cuda)
    rc = rope.to(cuda)
    H.check(H.lib().h3k_vae_heads(ptr(t), rows, heads, T, ptr(rc), 1e-6, stream()))
    sync()
    cs = rope[torch.arange(rows) % T]
    for part in (0, 1):
        want = V.heads(qkv[:, part].float(), cs, 1e-6)
        assert rel(t[:, part].float(), want) < 5e-3
    assert torch.equal(t[:, 2].cpu(), qkv[:, 2])


def test_layer_norm_rows(cuda):
    rows, d = 777, 2048
    x = torch.randn(rows, d, device=cuda) * 3 + 1
    w = 1 + 0.1 * torch.randn(d, device=cuda)
    b = 0.1 * torch.randn(d, device=cuda)
    out = torch.zeros(rows, d, device=cuda, dtype=torch.bfloat16)
    H.check(H.lib().h3k_layer_norm(ptr(x), rows, d, ptr(w), ptr(b), 1e-6, ptr(out), stream()))
    sync()
    want = torch.nn.functional.layer_norm(x.cpu(), (d,), w.cpu(), b.cpu(), 1e-6)
    assert rel(out.float(), want) < 4e-3


def _latents(frames, h, w, seed):
    return O.synthetic(frames * h * w * 24, seed, 77, 0.0, 1.0).reshape(frames, h, w, 24)


@pytest.mark.parametrize("h,w", [(16, 24), (9, 16), (20, 20)])
def test_decode_clip_matches_oracle(cuda, h, w):
    """One clip (7 latent frames) through the whole decoder: tiles (one, two with an 8-latent overlap, 2 x 2 with a
    corner where four tiles meet), tokens, two blocks, layer norm, projection, the tiles faded into one canvas."""
    cfg = H.VAE_CONFIGS["small"]
    lat = _latents(7, h, w, 1)
    m = H.VideoDecoder(cfg, seed=2)
    got = m.decode_clip(lat)
    m.close()
    want = V.decode_clip(cfg, V.make_weights(cfg, 2), lat)
    r, cos = O.diff(got, want, 3 * 16)
    assert r < 1e-2 and cos > 0.999, (r, cos)


def test_decode_video_clip_loop_matches_oracle(cuda):
    """VideoVae::decode: 12 latent frames = two clips -> 39 frames in [0, 1]; the second clip's first 5 frames fade in
    from the first clip's last 5, the last clip's 5 come out at the end."""
    cfg = H.VAE_CONFIGS["small"]
    lat = _latents(12, 16, 16, 4)
    m = H.VideoDecoder(cfg, seed=5)
    seen = []
    frames = m.decode(lat)
    m.decode(lat, sink=lambda i, a: seen.append(i))
    m.close()
    assert len(frames) == 17 * 2 + 5 and seen == list(range(39))
    want = V.decode(cfg, V.make_weights(cfg, 5), lat)
    got, ref = np.stack(frames), np.stack(want)
    assert got.min() >= 0.0 and got.max() <= 1.0
    r, cos = O.diff(got, ref, 3 * 16)
    assert r < 1e-2 and cos > 0.999, (r, cos)


def test_decode_refuses_bad_shapes(cuda):
    m = H.VideoDecoder("small", seed=0)
    with pytest.raises(H.H3Error) as e:
        m.decode(_latents(8, 16, 16, 0))  # not 5 n + 2 latent frames
    assert e.value.code == H.H3_ERR_ARG
    m.close()
