"""CPU tests: the oracle against the reference's golden vectors, the oracle's exact sparse selection against a
brute-force restatement, the library's host-side functions (layout rows, rotary table, int8 mask parsing, sparse
sizes) against the oracle, and that the library exports every symbol include/h3_c.h declares. No GPU is used."""
import ctypes
import json
import math
import os
import re

import numpy as np
import pytest
import torch

import h3b200
from oracle import exact, h3_oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")


# ------------------------------------------------------------------------------------ oracle vs golden vectors

def test_time_embedding_and_adaln_match_reference_formula():
    """tools/check_pruned_curve.py:58-67 (executed from the reference file) vs the oracle's time MLP + AdaLN."""
    g = np.load(os.path.join(GOLDEN, "time_adaln.npz"))
    w = {"t_in_w": torch.from_numpy(g["p_in_w"]).float(), "t_in_b": torch.from_numpy(g["p_in_b"]).float(),
         "t_out_w": torch.from_numpy(g["p_out_w"]).float(), "t_out_b": torch.from_numpy(g["p_out_b"]).float()}
    temb, s = O.time_embedding([float(t) for t in g["t"]], w)
    rel = np.linalg.norm(temb.numpy() - g["temb"]) / np.linalg.norm(g["temb"])
    assert rel < 1e-5, rel
    # AdaLN: the reference's mods_full has no bf16 rounding of silu(temb); the oracle applies it (dump_h3_ref.py:150)
    silu = torch.nn.functional.silu(temb)
    mods = silu @ torch.from_numpy(g["Wf"]).float().T + torch.from_numpy(g["bf"]).float()
    rel = np.linalg.norm(mods.numpy() - g["mods"]) / np.linalg.norm(g["mods"])
    assert rel < 1e-5, rel
    mods_r = s @ torch.from_numpy(g["Wf"]).float().T + torch.from_numpy(g["bf"]).float()
    rel_r = np.linalg.norm(mods_r.numpy() - g["mods"]) / np.linalg.norm(g["mods"])
    assert rel_r < 1e-2, rel_r  # bf16 rounding of the projection input only


def test_rope_frequencies_match_reference_expression():
    """tools/dump_h3_ref.py:140-141 evaluated from the reference file, bit for bit."""
    want = np.load(os.path.join(GOLDEN, "rope_freq.npy"))
    assert want.shape == (16,)
    np.testing.assert_array_equal(O.rope_inv_freq(), want)


def test_geometry_known_answers_are_consistent():
    """tests/geometry_test.cpp:22-27: the latent-frame and audio-latent counts the layouts are built from."""
    g = json.load(open(os.path.join(GOLDEN, "geometry.json")))
    for f, lf in g["latent_frames"]:
        assert (f - 5) // 17 * 5 + 2 == lf
    for f, a in g["audio_latents"]:
        assert round(f / 24 * 40) == a


def test_synthetic_values_are_deterministic_and_normal_like():
    a = O.synthetic(200000, 0, 7, 0.0, 0.02)
    b = O.synthetic(200000, 0, 7, 0.0, 0.02)
    np.testing.assert_array_equal(a, b)
    assert abs(a.mean()) < 2e-4 and abs(a.std() - 0.02) < 2e-4
    c = O.synthetic(1000, 1, 7)
    assert not np.array_equal(a[:1000], c)
    bf = O.synthetic(1000, 0, 7, bf16=True)
    assert (bf.view(np.uint32) & 0xFFFF).max() == 0


@pytest.mark.parametrize("seed,tid,mean,stdev,bf16", [(0, 7, 0.0, 0.02, False), (3, 104, 1.0, 0.02, False),
                                                      (5, 123, 0.0, 0.02, True), (11, 2, 0.0, 1.0, False), (0, 18, 0.0, 4.0, True)])
def test_synthetic_c_loop_equals_the_numpy_definition(seed, tid, mean, stdev, bf16):
    """Large tensors use the C loop form of the generator; it must give the numpy definition's bits."""
    n = (1 << 20) + 37
    np.testing.assert_array_equal(O.synthetic(n, seed, tid, mean, stdev, bf16).view(np.uint32),
                                  O.synthetic_np(n, seed, tid, mean, stdev, bf16).view(np.uint32))


def test_bf16_round_half_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e-39], np.float32)  # exact halves at bf16 spacing 2^-7
    r = O.bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == 1.015625 and r[3] == -2.5


def test_diff_metric_matches_reference_definition():
    got = np.array([[1.0, 0.0], [0.0, 2.0]])
    want = np.array([[1.0, 0.0], [0.0, 1.0]])
    rel, cos = O.diff(got, want, 2)
    assert abs(rel - math.sqrt(1 / 2)) < 1e-12 and abs(cos - 1.0) < 1e-12


# --------------------------------------------------------------------------- exact sparse selection (oracle)

def brute_topk(scores, frames, ph, pw, ratio, local):
    nct, ncy, ncx = (frames + 3) // 4, (ph + 3) // 4, (pw + 3) // 4
    nc = nct * ncy * ncx
    k = exact.sparse_k(ratio, nc)
    out = []
    for h in range(scores.shape[0]):
        rows = []
        for i in range(nc):
            ct = i // (ncx * ncy)
            forced = set()
            if local > 0:
                forced.add(i)
            if local >= 3:
                if ct > 0:
                    forced.add(i - ncx * ncy)
                if ct + 1 < nct:
                    forced.add(i + ncx * ncy)
            rest = sorted((j for j in range(nc) if j not in forced), key=lambda j: (-scores[h, i, j], j))
            want = max(k, len(forced))
            rows.append(sorted(list(forced) + rest[:want - len(forced)]))
        out.append(rows)
    return out


@pytest.mark.parametrize("ratio,local", [(0.1, 1), (0.25, 3), (0.5, 0), (1.0, 0), (0.01, 3)])
def test_exact_topk_matches_brute_force_with_ties(ratio, local):
    rng = np.random.default_rng(3)
    frames, ph, pw = 9, 6, 10
    nc = 3 * 2 * 3
    # quantised scores: many exact ties, which go to the lower cube index
    scores = (rng.integers(-4, 5, size=(2, nc, nc)) * 0.25).astype(np.float32)
    sel, nsel = exact.cube_topk(scores, frames, ph, pw, ratio, local)
    want = brute_topk(scores, frames, ph, pw, ratio, local)
    for h in range(2):
        for i in range(nc):
            assert list(sel[h, i, :nsel[h, i]]) == want[h][i]


def test_exact_pool_means_over_valid_rows_only():
    frames, ph, pw, D, H = 5, 6, 7, 11, 2
    S = D + frames * ph * pw
    rng = np.random.default_rng(0)
    q = O.bf16_round(rng.standard_normal((S, H, 128)).astype(np.float32))
    k = O.bf16_round(rng.standard_normal((S, H, 128)).astype(np.float32))
    bits = lambda a: (a.view(np.uint32) >> 16).astype(np.uint16).reshape(-1)
    mq, mk = exact.cube_pool(bits(q), bits(k), H * 128, H, D, frames, ph, pw)
    vid = q[D:].reshape(frames, ph, pw, H, 128)
    # cube (1, 1, 1): frames 4.., rows 4..5, cols 4..6 (padding beyond the grid)
    ncx, ncy = 2, 2
    c = (1 * ncy + 1) * ncx + 1
    ref = vid[4:8, 4:8, 4:8].reshape(-1, H, 128).astype(np.float64).mean(0)
    assert np.allclose(mq[:, c], ref.T.T, atol=1e-5)
    scores = exact.cube_scores(mq, mk)
    assert np.allclose(scores[0, 3, 5], float(np.dot(mq[0, 3].astype(np.float64), mk[0, 5])), rtol=1e-5)


# -------------------------------------------------------------------------------- library host-side functions

def test_library_exports_every_declared_symbol():
    header = open(os.path.join(REPO, "include", "h3_c.h")).read()
    declared = set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(h3k?_\w+)\(", header, re.M))
    declared -= {"h3_c"}
    L = h3b200.lib()
    for name in sorted(declared):
        assert hasattr(L, name), name
    assert declared <= set(h3b200.SIGNATURES), sorted(declared - set(h3b200.SIGNATURES))


@pytest.mark.parametrize("name", ["c1", "c2", "c5", "h3"])
def test_layout_rows_match_oracle(name):
    lay = h3b200.Layout.named(name)
    pos, tags, roles = h3b200.rows(lay)
    p2, t2, r2 = O.layout_rows(dict(h3b200.LAYOUTS[name]))
    np.testing.assert_array_equal(pos, p2)
    np.testing.assert_array_equal(tags, t2)
    np.testing.assert_array_equal(roles, r2)
    assert pos.shape[0] == lay.rows


def test_layout_with_keyframes_and_tags():
    tags = np.array([1, 1, 0, 0, 1], np.uint8)
    lay = h3b200.Layout(text=5, frames=6, h=8, w=12, audio=3, cond_frames=2, cond_last=[0, 1], text_tags=tags)
    pos, t, r = h3b200.rows(lay)
    d = dict(text=5, frames=6, h=8, w=12, audio=3, cond_frames=2, cond_last=[0, 1], text_tags=list(tags))
    p2, t2, r2 = O.layout_rows(d)
    np.testing.assert_array_equal(pos, p2)
    np.testing.assert_array_equal(t, t2)
    np.testing.assert_array_equal(r, r2)
    assert list(r[:5]) == [0] * 5 and (r[5:5 + 2 * 24] == 1).all()


REF_LAYOUT = dict(text=7, frames=6, h=8, w=12, audio=9, refs=[
    dict(kind="image", frames=1, h=6, w=10), dict(kind="audio", audio=5),
    dict(kind="video", frames=3, h=4, w=6, audio=11), dict(kind="video", frames=7, h=4, w=4, audio=2)])


def test_layout_with_reference_blocks():
    """Reference blocks (ref2va): row counts as the reference's Layout reports them, and H3::rows against the
    oracle's own restatement of architecture.md:203-215 (one clock for every block, the generated rows after)."""
    lay = h3b200.Layout(**REF_LAYOUT)
    pos, t, r = h3b200.rows(lay)
    p2, t2, r2 = O.layout_rows(REF_LAYOUT)
    np.testing.assert_array_equal(pos, p2)
    np.testing.assert_array_equal(t, t2)
    np.testing.assert_array_equal(r, r2)
    # counts: pictures and videos are conditioning video rows, soundtracks conditioning audio rows
    assert lay.cond_rows == 3 * 5 + 3 * 2 * 3 + 7 * 2 * 2 == (r == 1).sum()
    assert lay.cond_audio_rows == 2 * (5 + 11 + 2) == (r == 2).sum()
    assert pos.shape[0] == lay.rows == int(h3b200.lib().h3_layout_rows(ctypes.byref(lay.c)))
    # the clock: picture at 7, soundtrack at 8..12, the first video's rows from 13 (soundtrack 11 latents, frames
    # spanning 5/3 x 9 = 15), the second video from 28 (soundtrack 2, frames 5/3 x 22), the generated rows after
    assert (pos[r == 1][:15, 0] == 7).all()
    assert pos[7 + 15, 0] == 8 and pos[7 + 15 + 4, 0] == 12
    first_video_audio = pos[(r == 2)][10:, 0]
    assert first_video_audio[0] == 13
    gen_audio = pos[r == 3][:, 0]
    assert gen_audio[0] == 28 + 5.0 / 3.0 * 22
    assert (t[r == 2] == 2).all() and (t[r == 1] == 0).all()


def test_layout_refuses_keyframes_with_reference_blocks():
    lay = h3b200.Layout(text=2, frames=2, h=4, w=4, cond_frames=1, refs=[dict(kind="audio", audio=3)])
    n = np.zeros((64, 3))
    rc = h3b200.lib().h3_rows(ctypes.byref(lay.c), n.ctypes.data, None, None)
    assert rc == h3b200.H3_ERR_ARG


def test_sigmas_match_reference_known_answers():
    """tests/geometry_test.cpp:32-45 of the reference: 3 points shifted by 12 and 3, and 50 strictly decreasing
    points ending at 0; plus the whole schedule against the oracle's restatement for several sizes and shifts."""
    v, a = h3b200.sigmas(3, 12.0), h3b200.sigmas(3, 3.0)
    assert len(v) == 3 and v[0] == 1.0 and v[2] == 0.0 and abs(v[1] - 12.0 * 0.5 / (1.0 + 11.0 * 0.5)) < 1e-7
    assert len(a) == 3 and abs(a[1] - 0.75) < 1e-7
    s50 = h3b200.sigmas(50, 12.0)
    assert len(s50) == 50 and (np.diff(s50) < 0).all() and s50[-1] == 0.0
    for steps in (2, 3, 9, 10, 50, 51):
        for shift in (1.0, 3.0, 5.5, 12.0):
            np.testing.assert_array_equal(h3b200.sigmas(steps, shift), O.sigmas(steps, shift))


def test_lora_inspect_reads_names_rank_and_alpha(tmp_path):
    """The safetensors reader behind H3::add_lora: adapter names (file prefixes stripped), rank, the "alpha" metadata."""
    from tests import safetensors_util as ST
    rng = np.random.default_rng(0)
    t = {}
    for name in ("transformer.transformer_blocks.0.attn.to_q", "transformer.transformer_blocks.3.ff.net.2",
                 "transformer.token_refiner.blocks.0.attn.to_k"):
        t[name + ".lora_A.weight"] = rng.standard_normal((16, 64))
        t[name + ".lora_B.weight"] = rng.standard_normal((32, 16))
    path = tmp_path / "adapter.safetensors"
    ST.write(path, t, metadata={"alpha": 8})
    names, rank, alpha = h3b200.lora_inspect(path)
    assert sorted(names) == ["token_refiner.blocks.0.attn.to_k", "transformer_blocks.0.attn.to_q", "transformer_blocks.3.ff.net.2"]
    assert rank == 16 and alpha == 8.0


@pytest.mark.parametrize("damage", ["truncated", "garbage", "outside"])
def test_lora_inspect_refuses_malformed_files(tmp_path, damage):
    from tests import safetensors_util as ST
    path = tmp_path / "bad.safetensors"
    ST.write(path, {"a.lora_A.weight": np.ones((2, 4)), "a.lora_B.weight": np.ones((4, 2))})
    raw = path.read_bytes()
    if damage == "truncated":
        raw = raw[:20]
    elif damage == "garbage":
        raw = raw[:8] + b"{not json" + raw[17:]
    else:
        raw = raw[:-8]  # the last tensor's bytes run past the end of the file
    path.write_bytes(raw)
    rc = h3b200.lib().h3_lora_inspect(str(path).encode(), None, 0, None, None, None)
    assert rc == h3b200.H3_ERR_ARG
    assert h3b200.lib().h3_last_error()


def test_rope_table_matches_oracle():
    lay = h3b200.Layout.named("c1")
    got = h3b200.rope_table(lay)
    pos, _, _ = O.layout_rows(dict(h3b200.LAYOUTS["c1"]))
    np.testing.assert_array_equal(got, O.rope_table(pos))


def test_parse_int8():
    L = h3b200.lib()
    m = ctypes.c_uint32()
    for text, want in [("none", 0), ("all", 15), ("qkv", 1), ("out,fc2", 10), ("fc1,qkv", 5)]:
        assert L.h3_parse_int8(text.encode(), ctypes.byref(m)) == 0 and m.value == want
    assert L.h3_parse_int8(b"qkv,bogus", ctypes.byref(m)) == h3b200.H3_ERR_ARG
    assert b"comma list" in L.h3_last_error()


def test_sparse_sizes_for_768p():
    g = h3b200.h3k_cube_grid(768, 32, 24, 42)
    cubes, kcap, qt, mb = (ctypes.c_int32() for _ in range(4))
    h3b200.check(h3b200.lib().h3k_sparse_sizes(ctypes.byref(g), 0.1, 1, ctypes.byref(cubes), ctypes.byref(kcap),
                                                ctypes.byref(qt), ctypes.byref(mb)))
    assert cubes.value == 8 * 6 * 11 == 528  # the grid padded to multiples of 4 (architecture.md:122-124)
    assert kcap.value == 53                  # ceil(0.1 * 528)
    assert qt.value == 264 + 6               # cube pairs + dense-unit pairs
    assert exact.sparse_k(0.1, 528) == 53


@pytest.mark.parametrize("dims", [(768, 32, 24, 42), (5, 6, 7, 10), (0, 3, 2, 5), (64, 4, 4, 4)])
def test_packed_order_puts_each_cube_in_one_run(dims):
    """h3k_video_order: a permutation that lists the generated video rows cube by cube (cubes in (frame group, row
    group, column group) order, rows inside a cube in (frame, row, column) order), dense rows first and unmoved."""
    D, F, ph, pw = dims
    order = h3b200.packed_order(D, F, ph, pw)
    want = list(range(D))
    for ct in range(0, F, 4):
        for cy in range(0, ph, 4):
            for cx in range(0, pw, 4):
                for f in range(ct, min(ct + 4, F)):
                    for y in range(cy, min(cy + 4, ph)):
                        for x in range(cx, min(cx + 4, pw)):
                            want.append(D + (f * ph + y) * pw + x)
    assert order.tolist() == want


def test_create_refuses_a_missing_checkpoint_without_touching_the_gpu():
    L = h3b200.lib()
    cfg = h3b200.make_config("c1")
    h = ctypes.c_void_p()
    rc = L.h3_create(ctypes.byref(cfg), b"/models/minimax-h3/FL2VA/transformer", 0, 0.0, 1, None, 0, ctypes.byref(h))
    assert rc == h3b200.H3_ERR_ARG and not h.value
    assert b"cannot open" in L.h3_last_error()


def test_weight_specs_and_checkpoint_checks(tmp_path):
    """The tensors a checkpoint holds (h3_weight_specs), and h3_check_weights on a file with all of them, on a
    directory of two shards, and with one missing, one of the wrong shape or one in a second shard twice."""
    from tests import safetensors_util as ST

    cfg = dict(dim=256, heads=2, ffn=512, blocks=2, time_dim=128, text_dim=256, refiner=1)
    specs = h3b200.weight_specs(cfg)
    shape = {n: s for n, _, s in specs}
    dtypes = {n: d for n, d, _ in specs}
    assert specs[0][0] == "time_embedder.proj_in.weight"
    assert shape["blocks.0.attn.qkv.weight"] == (768, 256) and dtypes["blocks.0.attn.qkv.weight"] == "BF16"
    assert shape["blocks.1.ff.fc1.weight"] == (1024, 256) and shape["blocks.1.adaln_proj.linear.weight"] == (18 * 256, 128)
    assert "token_refiner.blocks.0.attn.to_out.weight" in shape and "token_refiner.norm.weight" in shape
    assert "token_refiner.blocks.0.adaln_proj.linear.weight" not in shape
    tensors = {n: np.zeros(s, np.float32) for n, s in shape.items()}
    ST.write(tmp_path / "all.safetensors", tensors, dtype=dtypes)
    assert h3b200.check_weights(cfg, tmp_path / "all.safetensors") == ""
    names = list(tensors)
    shards = tmp_path / "shards"
    shards.mkdir()
    ST.write(shards / "a.safetensors", {n: tensors[n] for n in names[:20]}, dtype="F32")
    ST.write(shards / "b.safetensors", {n: tensors[n] for n in names[20:]}, dtype="BF16")
    assert h3b200.check_weights(cfg, shards) == ""
    ST.write(tmp_path / "missing.safetensors", {n: a for n, a in tensors.items() if n != "blocks.1.attn.norm_k.weight"})
    assert h3b200.check_weights(cfg, tmp_path / "missing.safetensors") == "no tensor blocks.1.attn.norm_k.weight"
    bad = dict(tensors, **{"proj_out.weight": np.zeros((95, 256), np.float32)})
    ST.write(tmp_path / "bad.safetensors", bad)
    assert h3b200.check_weights(cfg, tmp_path / "bad.safetensors") == "proj_out.weight is 95x256, this model needs 96x256"
    ST.write(shards / "c.safetensors", {names[0]: tensors[names[0]]})
    assert "two files" in h3b200.check_weights(cfg, shards)
    pruned = h3b200.weight_specs(dict(cfg, curve=8))
    pn = {n: s for n, _, s in pruned}
    assert pn["adaln_t_table"] == (1025, 8) and "time_embedder.proj_in.weight" not in pn
    assert pn["blocks.0.adaln_proj.linear.weight"] == (18 * 256, 8)


def test_oracle_token_refiner_ends_in_its_weighted_rms_norm():
    """The oracle's token refiner (architecture.md:25-27): refiner blocks change the text rows, and the output is
    RMSNorm(x) * refiner_norm, so every row divided by the weight has unit RMS; without refiner blocks the rows pass
    unchanged."""
    import torch

    cfg = dict(dim=256, heads=2, ffn=512, blocks=0, time_dim=128, text_dim=256, refiner=2)
    w = O.make_weights(cfg, 5)
    assert len(w["refiner"]) == 2 and w["refiner_norm"].shape == (256,)
    x = torch.from_numpy(O.synthetic(7 * 256, 5, 9, 0.0, 1.0).reshape(7, 256))
    y = O.refine(cfg, w, x, lambda t: t, 1e-6)
    r = (y / w["refiner_norm"]).pow(2).mean(-1).sqrt()
    np.testing.assert_allclose(r.numpy(), 1.0, rtol=1e-4)
    assert not torch.allclose(y, O.rms(x, 1e-6) * w["refiner_norm"], atol=1e-3)  # the blocks did something
    w0 = O.make_weights(dict(cfg, refiner=0), 5)
    assert O.refine(cfg, w0, x, lambda t: t, 1e-6) is x


def test_oracle_curve_lookup_matches_reference_c_of():
    """Pruned checkpoints: the oracle's curve lookup (fp32) against tools/check_pruned_curve.py's own `c_of` (run on a
    seeded table by tests/golden/make_golden.py) at t * 1024 and past both ends of the table."""
    g = np.load(os.path.join(GOLDEN, "curve.npz"))
    got = O.curve_points([float(t) for t in g["t"]], g["table"]).numpy()
    np.testing.assert_allclose(got, g["c"], rtol=2e-6, atol=2e-6)
    out = O.curve_points([float(p) / 1024.0 for p in g["outside_pos"]], g["table"]).numpy()
    np.testing.assert_allclose(out, g["outside"], rtol=2e-6, atol=2e-6)


def test_oracle_pruned_checkpoint_has_no_time_embedder():
    """A pruned checkpoint's weights: adaln_t_table [1025][8], [18 d][8] and [2 d][8] fp32 projections, no time MLP; block
    0's modulation is the curve point projected without SiLU."""
    import torch

    cfg = dict(dim=256, heads=2, ffn=512, blocks=2, time_dim=128, text_dim=256, curve=8)
    w = O.make_weights(cfg, 2)
    assert "t_in_w" not in w and w["curve_table"].shape == (1025, 8)
    assert w["blocks"][0]["ada_w"].shape == (18 * 256, 8) and w["fada_w"].shape == (512, 8)
    seen = {}
    L = dict(text=3, frames=1, h=4, w=4, audio=0)
    text = np.zeros((3, 256), np.float32)
    video = O.synthetic(4 * 96, 1, 2, 0.0, 1.0).reshape(4, 96)
    O.step(cfg, w, L, text, video, np.zeros((0, 32), np.float32), 0.6, 0.6, probes=lambda n, l, a: seen.__setitem__(n, a))
    assert "temb" not in seen
    c = O.curve_points([0.6], w["curve_table"])
    want = (c @ w["blocks"][0]["ada_w"].T + w["blocks"][0]["ada_b"]).numpy()
    np.testing.assert_allclose(seen["mod0"], want, rtol=1e-6, atol=1e-6)


def test_convert_renames_and_stacks_a_foreign_checkpoint(tmp_path):
    """h3_convert_weights: a checkpoint that names two tensors otherwise, keeps each head's q, k and v rows together
    and stores everything as F32 becomes one that h3_create reads: this library's names, q/k/v stacked, bf16 matrices
    rounded to nearest even, fp32 vectors as they were."""
    from tests import safetensors_util as ST

    cfg = dict(dim=256, heads=2, ffn=512, blocks=1, time_dim=128, text_dim=256, refiner=1)
    specs = h3b200.weight_specs(cfg)
    rng = np.random.default_rng(0)
    ours = {n: rng.standard_normal(s).astype(np.float32) for n, _, s in specs}
    renames = {"blocks.0.attn.qkv.weight": "model.layers.0.attention.wqkv.weight", "blocks.0.norm1.weight": "model.layers.0.ln1.weight"}
    src = {}
    for n, a in ours.items():
        if n.endswith("attn.qkv.weight") or n.endswith("attn.qkv.bias"):
            parts = a.reshape((3, 2, 128) + a.shape[1:])
            a = np.ascontiguousarray(parts.transpose((1, 0, 2) + tuple(range(3, parts.ndim)))).reshape(a.shape)
        src[renames.get(n, n)] = a
    ST.write(tmp_path / "src.safetensors", src, dtype="F32")
    assert h3b200.check_weights(cfg, tmp_path / "src.safetensors") == "no tensor blocks.0.norm1.weight"
    h3b200.convert_weights(cfg, tmp_path / "src.safetensors", tmp_path / "dst.safetensors", renames=renames, interleaved=True)
    assert h3b200.check_weights(cfg, tmp_path / "dst.safetensors") == ""
    got, dtypes, meta = ST.read(tmp_path / "dst.safetensors")
    assert meta["qkv_layout"] == "stacked" and set(got) == set(ours)
    for n, d, _ in specs:
        want = ST.bf16_values(ours[n]).numpy() if d == "BF16" else ours[n]
        assert dtypes[n] == d
        np.testing.assert_array_equal(got[n], want)
    with pytest.raises(h3b200.H3Error):
        h3b200.convert_weights(cfg, tmp_path / "src.safetensors", tmp_path / "x.safetensors")  # the renames are needed


def test_convert_refuses_an_untagged_qkv_layout_unless_stated(tmp_path):
    """A source without qkv_layout metadata could hold q/k/v rows per head (the reference's shards) or stacked; the
    shapes are the same, so h3_convert_weights refuses to guess: it needs a "qkv_layout interleaved|stacked" line."""
    from tests import safetensors_util as ST

    cfg = dict(dim=256, heads=2, ffn=512, blocks=1, time_dim=128, text_dim=256, refiner=0)
    rng = np.random.default_rng(1)
    src = {n: rng.standard_normal(s).astype(np.float32) for n, _, s in h3b200.weight_specs(cfg)}
    ST.write(tmp_path / "untagged.safetensors", src, dtype="F32")
    with pytest.raises(h3b200.H3Error) as e:
        h3b200.convert_weights(cfg, tmp_path / "untagged.safetensors", tmp_path / "out.safetensors")
    assert e.value.code == h3b200.H3_ERR_ARG and "qkv_layout" in str(e.value)
    cfgc = h3b200.make_config(cfg)
    lib = h3b200.lib()
    assert lib.h3_convert_weights(ctypes.byref(cfgc), str(tmp_path / "untagged.safetensors").encode(),
                                  str(tmp_path / "out.safetensors").encode(), b"qkv_layout stacked") == h3b200.H3_OK
    got, _, meta = ST.read(tmp_path / "out.safetensors")
    assert meta["qkv_layout"] == "stacked"
    np.testing.assert_array_equal(got["blocks.0.attn.qkv.bias"], src["blocks.0.attn.qkv.bias"])
    h3b200.convert_weights(cfg, tmp_path / "untagged.safetensors", tmp_path / "out2.safetensors", interleaved=True)
    got2, _, _ = ST.read(tmp_path / "out2.safetensors")
    assert not np.array_equal(got2["blocks.0.attn.qkv.bias"], src["blocks.0.attn.qkv.bias"])


def test_h3_shape_holds_the_reference_parameter_counts():
    """MiniMax-H3's shape in this build (dim 5376, 56 heads of 128, SwiGLU 14336, 50 blocks, time 2688, the two-block
    token refiner) holds the sizes the reference documents: 20 B parameters without the AdaLN projections and 33 B with
    (docs/architecture.md:11-12); the AdaLN projections 26 GB of the 66, and 47 GB once q/k/v, out, fc1 and fc2 are
    int8 rows (docs/architecture.md:53-56)."""
    specs = h3b200.weight_specs("h3")
    count = lambda pick: sum(math.prod(s) for n, _, s in specs if pick(n))
    total, adaln = count(lambda n: True), count(lambda n: "adaln_proj" in n)
    assert round(total / 1e9) == 33 and round((total - adaln) / 1e9) == 20
    nbytes = sum(math.prod(s) * (2 if d == "BF16" else 4) for _, d, s in specs)
    assert round(nbytes / 1e9) == 66 and round(2 * adaln / 1e9) == 26
    projections = count(lambda n: n.startswith("blocks.") and any(k in n for k in ("attn.qkv.weight", "attn.to_out.weight",
                                                                                  "ff.fc1.weight", "ff.fc2.weight")))
    assert round((nbytes - projections) / 1e9) == 47  # int8 rows: one byte instead of two


def test_h3_tensor_shapes_and_768p_rows_match_the_reference_prose():
    """Shapes the reference states for MiniMax-H3: AdaLN 2688 -> 96768 = 3 x 6 x 5376 and the final layer's 2688 ->
    2 x 5376 (docs/architecture.md:49-53), q/k/v 5376 -> 21504 and out 7168 -> 5376, fc1 28672 rows [gate; value], fc2
    from 14336 (docs/architecture.md:61-65; docs/performance.md:41-43), condition_proj 5120 -> 5376, the patch
    projections 96 and 32 -> 5376 (docs/architecture.md:25-31), a pruned checkpoint's [96768][8] and [10752][8]
    projections (docs/architecture.md:57-60); and the 768p x 124-frame layout's 37 x 24 x 42 = 37296 video rows and
    414 audio rows (docs/architecture.md:31-33; tests/geometry_test.cpp:24-26)."""
    shape = {n: s for n, _, s in h3b200.weight_specs("h3")}
    assert shape["blocks.0.adaln_proj.linear.weight"] == (96768, 2688)
    assert shape["norm_out.adaln_proj.weight"] == (10752, 2688)
    assert shape["blocks.49.attn.qkv.weight"] == (21504, 5376) and shape["blocks.49.attn.to_out.weight"] == (5376, 7168)
    assert shape["blocks.0.ff.fc1.weight"] == (28672, 5376) and shape["blocks.0.ff.fc2.weight"] == (5376, 14336)
    assert shape["condition_proj.weight"] == (5376, 5120)
    assert shape["video_patch_proj.weight"] == (5376, 96) and shape["audio_patch_proj.weight"] == (5376, 32)
    assert "blocks.50.norm1.weight" not in shape
    pruned = {n: s for n, _, s in h3b200.weight_specs(dict(h3b200.CONFIGS["h3"], curve=8))}
    assert pruned["blocks.0.adaln_proj.linear.weight"] == (96768, 8) and pruned["norm_out.adaln_proj.weight"] == (10752, 8)
    lay = h3b200.Layout(text=300, frames=37, h=48, w=84, audio=207, cond_frames=0)
    assert lay.video_rows == 37296 and lay.audio_rows == 414
    assert h3b200.lib().h3_layout_rows(ctypes.byref(lay.c)) == 300 + 414 + 37296


# ------------------------------------------------------------------------------------------- video VAE decoder

@pytest.mark.parametrize("n", [1, 7, 16, 17, 20, 24, 29, 48, 84, 135, 240])
def test_vae_tile_layout_matches_oracle(n):
    """Tiles of 16 latents overlapping by at least 4 (64 pixels), the slack spread over the overlaps: the library's
    layout equals the oracle's, covers the axis exactly, and 768p decodes as 4 x 7 tiles a clip
    (docs/architecture.md:91-92)."""
    from oracle import vae_oracle as V
    got = h3b200.vae_tile_starts(n)
    assert got == V.tile_starts(n)
    size = min(16, n)
    assert got[0] == 0 and got[-1] + size == n
    for a, b in zip(got, got[1:]):
        assert 4 <= a + 16 - b < 16
    if n == 48:
        assert len(got) == 4
    if n == 84:
        assert len(got) == 7


def test_vae_rope_table_matches_oracle():
    from oracle import vae_oracle as V
    for frames, th, tw in ((7, 16, 16), (7, 9, 16), (3, 5, 4)):
        np.testing.assert_array_equal(h3b200.vae_rope_table(frames, th, tw, 5), V.rope_table(frames, th, tw, 5))
