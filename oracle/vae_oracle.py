"""CPU oracle of MiniMax-H3's video VAE decoder -- TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU-baseline leg import this module, as the checker or the timed CPU baseline; the product
(libh3b200.so) never calls it.

PARITY STATUS: unpinned. The decoder (models::H3Vae) lives in the reference's empty mako-common submodule and no
reference tensors of it exist, so this restates the reference's description of it (docs/architecture.md:80-92) and
its clip loop (src/video/video_vae.cpp:17-50), not its code. Choices where the prose leaves the details open (each
also the library's):
  * tiles: along an axis of n latents one tile of n when n <= 16, else the fewest 16-latent tiles overlapping by at
    least 4, the slack spread over the overlaps in whole latents, the first gaps taking one more;
  * tokens of a tile: 4 register tokens, then a zero token, then the voxels in (frame, row, column) order; the
    voxel's input is the post-quant 1x1 convolution of its de-normalized latent (z * std + mean), embedded 24 -> d;
  * rotary: the special tokens at the origin; voxel coordinates -1 + 2 i / n on each axis (frames, rows, columns of
    the tile), times 2 pi, times 100^(-2 k / 16) for k < 8; dims j and j + 24 rotate by angle j (axis-major), 48..63
    pass; q and k RMS-normed per head (no weight) before the rotary;
  * block: x += scale1 * (attn(RMSNorm(x) w1) W_o + b_o); x += scale2 * (SwiGLU(RMSNorm(x) w2)); attention within
    the tile, 1/sqrt(64); fc1 stored [gate; value];
  * pixels: layer norm, projection to 3 x 4 x 16 x 16 (channel, frame, row, column) per voxel; tiles in raster order,
    each faded in linearly over its overlap with the tile above and the tile to the left (weight 0 at the overlap's
    first pixel, the product of the two where both apply);
  * frames: ImageNet statistics (0.485, 0.456, 0.406) / (0.229, 0.224, 0.225).
"""
import math

import numpy as np
import torch

from oracle import h3_oracle as O

# synthetic tensor ids, as the library assigns them
V_MEAN, V_STD, V_PQW, V_PQB, V_EMBW, V_EMBB, V_REG, V_LNW, V_LNB, V_PROJW, V_PROJB = range(5001, 5012)
V_BLOCK_BASE, V_BLOCK_STRIDE = 5100, 20
NORM1, QKVW, QKVB, OUTW, OUTB, SCALE1, NORM2, FC1W, FC1B, FC2W, FC2B, SCALE2 = range(12)
PIXEL_MEAN = np.array([0.485, 0.456, 0.406], np.float32)
PIXEL_STD = np.array([0.229, 0.224, 0.225], np.float32)
PATCH, PATCH_T = 16, 4


def make_weights(cfg, seed):
    d, F, C, R = cfg["dim"], cfg["ffn"], cfg["channels"], cfg["registers"]
    t = lambda n, tid, shape, mean=0.0, sd=0.02, bf16=False: torch.from_numpy(O.synthetic(n, seed, tid, mean, sd, bf16).reshape(shape))
    w = {"mean": t(C, V_MEAN, (C,), 0.0, 0.1), "std": t(C, V_STD, (C,), 1.0, 0.1),
         "pq_w": t(C * C, V_PQW, (C, C), 0.0, 0.2), "pq_b": t(C, V_PQB, (C,)),
         "emb_w": t(d * C, V_EMBW, (d, C), 0.0, 0.2, True), "emb_b": t(d, V_EMBB, (d,)),
         "registers": t(max(R, 1) * d, V_REG, (max(R, 1), d), 0.0, 1.0),
         "ln_w": t(d, V_LNW, (d,), 1.0), "ln_b": t(d, V_LNB, (d,)),
         "proj_w": t(3 * PATCH_T * PATCH * PATCH * d, V_PROJW, (3 * PATCH_T * PATCH * PATCH, d), bf16=True),
         "proj_b": t(3 * PATCH_T * PATCH * PATCH, V_PROJB, (3 * PATCH_T * PATCH * PATCH,)), "blocks": []}
    for l in range(cfg["blocks"]):
        b = V_BLOCK_BASE + V_BLOCK_STRIDE * l
        w["blocks"].append({
            "norm1": t(d, b + NORM1, (d,), 1.0), "qkv_w": t(3 * d * d, b + QKVW, (3 * d, d), bf16=True), "qkv_b": t(3 * d, b + QKVB, (3 * d,)),
            "out_w": t(d * d, b + OUTW, (d, d), bf16=True), "out_b": t(d, b + OUTB, (d,)), "scale1": t(d, b + SCALE1, (d,), 0.1),
            "norm2": t(d, b + NORM2, (d,), 1.0), "fc1_w": t(2 * F * d, b + FC1W, (2 * F, d), bf16=True), "fc1_b": t(2 * F, b + FC1B, (2 * F,)),
            "fc2_w": t(d * F, b + FC2W, (d, F), bf16=True), "fc2_b": t(d, b + FC2B, (d,)), "scale2": t(d, b + SCALE2, (d,), 0.1)})
    return w


def tile_starts(n, tile=16, overlap=4):
    if n <= tile:
        return [0]
    k = -(-(n - overlap) // (tile - overlap))
    slack, gaps = k * tile - n, k - 1
    s = [0]
    for g in range(gaps):
        s.append(s[-1] + tile - (slack // gaps + (1 if g < slack % gaps else 0)))
    return s


def rope_table(frames, th, tw, specials):
    """[T][24][2] (cos, sin), computed as the library's host code does (angle in fp32 from double coordinates)."""
    T = frames * th * tw + specials
    inv = [np.float32(1.0 / 100.0 ** (2 * k / 16.0)) for k in range(8)]
    out = np.zeros((T, 24, 2), np.float32)
    for r in range(T):
        coord = (0.0, 0.0, 0.0)
        if r >= specials:
            v = r - specials
            f, y, x = v // (th * tw), (v // tw) % th, v % tw
            coord = (-1.0 + 2.0 * f / frames, -1.0 + 2.0 * y / th, -1.0 + 2.0 * x / tw)
        for a in range(3):
            for k in range(8):
                ang = np.float32(np.float32(coord[a] * 2 * math.pi) * inv[k])
                out[r, a * 8 + k] = (np.float32(math.cos(float(ang))), np.float32(math.sin(float(ang))))
    return out


def rms(x, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def heads(x, cs, eps):
    """x [T][H][64]: RMS norm per head, then dims j, j + 24 rotated by angle j (j < 24)."""
    x = rms(x, eps)
    c, s = cs[:, None, :, 0], cs[:, None, :, 1]
    a, b, rest = x[..., :24], x[..., 24:48], x[..., 48:]
    return torch.cat([a * c - b * s, b * c + a * s, rest], -1)


def decode_clip(cfg, w, lat, eps=1e-6):
    """lat [clip][h][w][C] normalized latents -> canvas [4 clip][16 h][16 w][3] (ImageNet-normalized)."""
    clip, h, wd, C = lat.shape
    d, H, F, R = cfg["dim"], cfg["heads"], cfg["ffn"], cfg["registers"] + 1
    ys, xs = tile_starts(h), tile_starts(wd)
    th, tw = min(16, h), min(16, wd)
    T = clip * th * tw + R
    cs = torch.from_numpy(rope_table(clip, th, tw, R))
    lat = torch.from_numpy(np.ascontiguousarray(lat, np.float32))
    canvas = torch.zeros(clip * PATCH_T, h * PATCH, wd * PATCH, 3)
    covered = torch.zeros(clip * PATCH_T, h * PATCH, wd * PATCH, dtype=torch.bool)
    for ty, y0 in enumerate(ys):
        for tx, x0 in enumerate(xs):
            z = lat[:, y0:y0 + th, x0:x0 + tw, :].reshape(-1, C) * w["std"] + w["mean"]
            z = z @ w["pq_w"].T + w["pq_b"]
            x = torch.zeros(T, d)
            x[:R - 1] = w["registers"][:R - 1]
            x[R:] = z @ w["emb_w"].T + w["emb_b"]
            for B in w["blocks"]:
                hh = rms(x, eps) * B["norm1"]
                qkv = (hh @ B["qkv_w"].T + B["qkv_b"]).reshape(T, 3, H, 64)
                q, k, v = heads(qkv[:, 0], cs, eps), heads(qkv[:, 1], cs, eps), qkv[:, 2]
                o = _attention64(q, k, v).reshape(T, d)
                x = x + B["scale1"] * (o @ B["out_w"].T + B["out_b"])
                hh = rms(x, eps) * B["norm2"]
                gv = hh @ B["fc1_w"].T + B["fc1_b"]
                x = x + B["scale2"] * ((torch.nn.functional.silu(gv[:, :F]) * gv[:, F:]) @ B["fc2_w"].T + B["fc2_b"])
            xn = torch.nn.functional.layer_norm(x, (d,), w["ln_w"], w["ln_b"], eps)
            pix = (xn[R:] @ w["proj_w"].T + w["proj_b"]).reshape(clip, th, tw, 3, PATCH_T, PATCH, PATCH)
            # [clip][th][tw][c][ft][py][px] -> [clip * 4][th * 16][tw * 16][3]
            img = pix.permute(0, 4, 1, 5, 2, 6, 3).reshape(clip * PATCH_T, th * PATCH, tw * PATCH, 3)
            oy = (ys[ty - 1] + th - y0) * PATCH if ty > 0 else 0
            ox = (xs[tx - 1] + tw - x0) * PATCH if tx > 0 else 0
            wy = torch.ones(th * PATCH)
            wx = torch.ones(tw * PATCH)
            if oy:
                wy[:oy] = torch.arange(oy, dtype=torch.float32) / oy
            if ox:
                wx[:ox] = torch.arange(ox, dtype=torch.float32) / ox
            wt = (wy[:, None] * wx[None, :])[None, :, :, None]
            Y, X = slice(y0 * PATCH, (y0 + th) * PATCH), slice(x0 * PATCH, (x0 + tw) * PATCH)
            prev = canvas[:, Y, X]
            cov = covered[:, Y, X][..., None]
            canvas[:, Y, X] = torch.where(cov, prev * (1 - wt) + img * wt, img)
            covered[:, Y, X] = True
    return canvas.numpy()


def _attention64(q, k, v):
    """softmax(q k^T / 8) v per head; q, k, v [T][H][64]."""
    qh, kh, vh = q.permute(1, 0, 2), k.permute(1, 0, 2), v.permute(1, 0, 2)
    p = torch.softmax(qh @ kh.transpose(1, 2) / 8.0, -1)
    return (p @ vh).permute(1, 0, 2)


def emit(frames_normalized):
    return np.clip(frames_normalized * PIXEL_STD + PIXEL_MEAN, 0.0, 1.0).astype(np.float32)


def decode(cfg, w, lat):
    """video_vae.cpp:17-50 restated: lat [5 n + 2][h][w][C] -> the 17 n + 5 frames in [0, 1]."""
    frames = lat.shape[0]
    chunks = (frames - 2) // 5
    out, overlap = [], None
    for ci in range(chunks):
        canvas = decode_clip(cfg, w, lat[ci * 5:ci * 5 + 7])
        for fr in range(3, 20):
            cur = canvas[fr]
            if ci > 0 and fr - 3 < 5:
                wb = np.float32((fr - 3) / 5.0)
                cur = overlap[fr - 3] * (np.float32(1.0) - wb) + cur * wb
            out.append(emit(cur))
        overlap = canvas[23:28].copy()
    for fr in range(5):
        out.append(emit(overlap[fr]))
    return out
