"""The whole step through the C ABI (h3_create / h3_begin / h3_step) against the CPU oracle on the same synthetic
weights and inputs, probe by probe as the reference's harness compares the Diffusers tensors
(tests/h3_ref_test.cpp:214-250): the text after the token refiner, time embedding, block-0 modulation, packed input,
blocks, final norm, velocities."""
import numpy as np
import pytest

import h3b200 as H
from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu

# tests/h3_ref_test.cpp:219, 228-249
TOL = {"txt": 5e-3, "temb": 1e-4, "mod0": 5e-3, "x0": 5e-3, "block": 1e-2, "norm_out": 6e-2}
# north star: bf16 path vs the fp32 oracle
VEL_REL, VEL_COS = 1e-2, 0.999


def inputs(layout, cfg, seed=11):
    lay = H.Layout(**layout)
    text = O.synthetic(layout["text"] * cfg["text_dim"], seed, 1, 0.0, 1.0).reshape(layout["text"], cfg["text_dim"])
    video = O.synthetic(lay.video_rows * 96, seed, 2, 0.0, 1.0).reshape(lay.video_rows, 96)
    audio = O.synthetic(lay.audio_rows * 32, seed, 3, 0.0, 1.0).reshape(lay.audio_rows, 32)
    return lay, text, video, audio


def run_both(cfg, layout, t_video, t_audio, int8=0, sparse=0.0, local=1, seed=0):
    lay, text, video, audio = inputs(layout, cfg)
    m = H.Model(cfg, seed=seed, int8_mask=int8, sparse_ratio=sparse, sparse_local=local)
    got = {}
    m.set_probe(lambda name, layer, a: got.__setitem__(name if layer < 0 else f"{name}{layer}", a))
    m.begin(text, lay)
    gv, ga = m.step(video, audio, t_video, t_audio)
    launches = m.last_launches()
    m.close()
    w = O.make_weights(cfg, seed)
    want = {}
    ov, oa = O.step(cfg, w, layout, text, video, audio, t_video, t_audio, int8=int8,
                    probes=lambda n, l, a: want.__setitem__(n if l < 0 else f"{n}{l}", a))
    return got, want, (gv, ga), (ov, oa), launches


def check_probes(got, want, d, blocks, tol_scale=1.0):
    assert set(got) == set(want), (sorted(got), sorted(want))
    for name, tol in TOL.items():
        if name == "temb" and "temb" not in want:  # a pruned checkpoint has no time embedder
            continue
        keys = [f"block{l}" for l in range(blocks)] if name == "block" else [name]
        for k in keys:
            width = d if k != "temb" else want[k].size // max(1, want[k].shape[0] if want[k].ndim > 1 else 1)
            g = got[k].reshape(want[k].shape)
            rel, cos = O.diff(g, want[k], want[k].shape[-1] if want[k].ndim > 1 else want[k].size)
            assert rel < tol * tol_scale, (k, rel, cos)


def test_step_c1_matches_oracle(cuda):
    """one d=1024 block, 8 heads, SwiGLU 2816, 512 video + 64 text rows, t = 0.5."""
    cfg = H.CONFIGS["c1"]
    got, want, (gv, ga), (ov, oa), launches = run_both(cfg, H.LAYOUTS["c1"], 0.5, 0.5)
    check_probes(got, want, cfg["dim"], cfg["blocks"])
    rel, cos = O.diff(gv, ov, 96)
    assert rel < VEL_REL and cos > VEL_COS, (rel, cos)
    assert launches > 5


MINI = dict(dim=512, heads=4, ffn=1280, blocks=3, time_dim=256, text_dim=512, refiner=2)
MINI_LAYOUT = dict(text=40, frames=6, h=12, w=14, audio=24, cond_frames=1, cond_last=[1])


def test_step_with_audio_keyframes_and_three_levels(cuda):
    """Three noise levels in one forward (video/text, audio, keyframe rows at 0.999), three modalities."""
    got, want, (gv, ga), (ov, oa), _ = run_both(MINI, MINI_LAYOUT, 0.7, 0.4)
    check_probes(got, want, MINI["dim"], MINI["blocks"])
    for g, o, wdt in ((gv, ov, 96), (ga, oa, 32)):
        rel, cos = O.diff(g, o, wdt)
        assert rel < VEL_REL and cos > VEL_COS, (rel, cos)


def test_step_pruned_checkpoint_matches_oracle(cuda):
    """A pruned checkpoint (docs/architecture.md:57-60): no time embedder; each noise level's curve point read from
    adaln_t_table at t * 1024 with linear interpolation, the [18 d][8] projections applied in fp32 without SiLU
    (curve_mods); three levels in one forward."""
    cfg = dict(MINI, curve=8)
    got, want, (gv, ga), (ov, oa), launches = run_both(cfg, MINI_LAYOUT, 0.7, 0.4)
    assert "temb" not in got
    check_probes(got, want, cfg["dim"], cfg["blocks"])
    for g, o, wdt in ((gv, ov, 96), (ga, oa, 32)):
        rel, cos = O.diff(g, o, wdt)
        assert rel < VEL_REL and cos > VEL_COS, (rel, cos)


REF_LAYOUT = dict(text=24, frames=6, h=12, w=14, audio=16, refs=[
    dict(kind="image", frames=1, h=10, w=8), dict(kind="audio", audio=9),
    dict(kind="video", frames=3, h=6, w=8, audio=13)])


@pytest.mark.parametrize("sparse", [0.0, 0.5])
def test_step_with_reference_blocks_and_four_levels(cuda, sparse):
    """ref2va: a picture, a soundtrack and a video with its soundtrack ahead of the generated rows; four noise levels
    (video/text, audio, reference pictures and videos at 0.999, reference soundtracks at 1) in one forward. The
    sparse case keeps every reference row among the dense rows every video query sees."""
    if sparse:
        lay, text, video, audio = inputs(REF_LAYOUT, MINI)
        m = H.Model(MINI, seed=0, sparse_ratio=1.0, sparse_local=1)
        m.begin(text, lay)
        sv, sa = m.step(video, audio, 0.7, 0.4)
        m.close()
        _, _, (gv, ga), _, _ = run_both(MINI, REF_LAYOUT, 0.7, 0.4)
        for g, o, wdt in ((sv, gv, 96), (sa, ga, 32)):
            rel, cos = O.diff(g, o, wdt)
            assert rel < 1e-2 and cos > 0.9999, (rel, cos)  # every cube selected = dense
        return
    got, want, (gv, ga), (ov, oa), _ = run_both(MINI, REF_LAYOUT, 0.7, 0.4)
    assert want["temb"].shape[0] == 4
    check_probes(got, want, MINI["dim"], MINI["blocks"])
    for g, o, wdt in ((gv, ov, 96), (ga, oa, 32)):
        rel, cos = O.diff(g, o, wdt)
        assert rel < VEL_REL and cos > VEL_COS, (rel, cos)


def test_step_sparse_every_cube_equals_dense(cuda):
    """--sparse 1.0 --sparse-local 0: every cube selected, so the sparse path must give the dense model's velocities
    (the reference's h3_dit_sparse_all, tests/CMakeLists.txt:9-12)."""
    lay = dict(text=40, frames=9, h=12, w=18, audio=16)
    _, _, (gv, ga), (ov, oa), _ = run_both(MINI, lay, 0.6, 0.6, sparse=1.0, local=0)
    rel, cos = O.diff(gv, ov, 96)
    assert rel < VEL_REL and cos > VEL_COS, (rel, cos)


def test_step_int8_all_matches_int8_oracle(cuda):
    """--int8 all: the W8A8 path against the oracle's int8 dequant path (the integer products are exact; the
    activations' int8 roundings can differ where fp32 paths differ by an ulp, hence a tolerance)."""
    _, _, (gv, ga), (ov, oa), _ = run_both(MINI, MINI_LAYOUT, 0.7, 0.4, int8=15)
    rel, cos = O.diff(gv, ov, 96)
    assert rel < 2e-2 and cos > 0.998, (rel, cos)


def test_step_is_deterministic_and_reuses_begin(cuda):
    lay, text, video, audio = inputs(MINI_LAYOUT, MINI)
    m = H.Model(MINI, seed=4)
    m.begin(text, lay)
    a = m.step(video, audio, 0.7, 0.4)
    b = m.step(video, audio, 0.7, 0.4)
    c = m.step(video, audio, 0.2, 0.1)
    m.close()
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert not np.array_equal(a[0], c[0])


def test_set_sparse_after_begin_takes_effect(cuda):
    """H3::set_sparse between begin and step (or between steps) switches the attention: the same bits as a model
    created with that ratio, and back to the dense model's bits at ratio 0."""
    lay, text, video, audio = inputs(MINI_LAYOUT, MINI)

    def run(create_ratio, then=None):
        m = H.Model(MINI, seed=4, sparse_ratio=create_ratio, sparse_local=1)
        m.begin(text, lay)
        outs = [m.step(video, audio, 0.7, 0.4)]
        for r in then or ():
            m.set_sparse(r, 1)
            outs.append(m.step(video, audio, 0.7, 0.4))
        m.close()
        return outs

    dense, sparse = run(0.0)[0], run(0.3)[0]
    assert not np.array_equal(dense[0], sparse[0])
    switched = run(0.0, then=[0.3, 0.0])
    for got, want in zip(switched, (dense, sparse, dense)):
        np.testing.assert_array_equal(got[0], want[0])
        np.testing.assert_array_equal(got[1], want[1])


def test_step_errors(cuda):
    m = H.Model(MINI, seed=4)
    lay, text, video, audio = inputs(MINI_LAYOUT, MINI)
    with pytest.raises(H.H3Error) as e:
        m.step(video, audio, 0.5, 0.5)
    assert e.value.code in (H.H3_ERR_STATE, H.H3_ERR_ARG, H.H3_ERR_CUDA)
    m.begin(text, lay)
    with pytest.raises(H.H3Error) as e:
        m.step(video[:-1], audio, 0.5, 0.5)
    assert e.value.code == H.H3_ERR_ARG
    m.close()


def _host_loop(m, video, audio, sv, sa, steps, C, CA):
    video, audio = video.copy(), audio.copy()
    for i in range(steps):
        tv, ta = 1.0 - sv[i], 1.0 - sa[i]
        vv, va = m.step(video, audio, np.float32(tv), np.float32(ta))
        video[C:] = O.euler(video[C:], vv[C:], np.float32(tv), sv[i], sv[i + 1])
        audio[CA:] = O.euler(audio[CA:], va[CA:], np.float32(ta), sa[i], sa[i + 1])
    return video, audio


@pytest.mark.parametrize("layout", ["keyframes", "refs"])
def test_denoise_on_device_equals_step_by_step_host_loop(cuda, layout):
    """h3_denoise (the sample kept on the GPU, Euler there) against h3_step plus the host Euler of the reference's
    sampler (src/video/engine.cpp:705-716) over three steps: identical bits; the conditioning rows unchanged."""
    L = MINI_LAYOUT if layout == "keyframes" else REF_LAYOUT
    lay, text, video, audio = inputs(L, MINI)
    sv, sa = H.sigmas(4, 5.0), H.sigmas(4, 3.0)
    m = H.Model(MINI, seed=2)
    m.begin(text, lay)
    gv, ga, ran = m.denoise(video, audio, sv, sa)
    assert ran == 3
    hv, ha = _host_loop(m, video, audio, sv, sa, 3, lay.cond_rows, lay.cond_audio_rows)
    m.close()
    np.testing.assert_array_equal(gv, hv)
    np.testing.assert_array_equal(ga, ha)
    np.testing.assert_array_equal(gv[:lay.cond_rows], video[:lay.cond_rows])
    np.testing.assert_array_equal(ga[:lay.cond_audio_rows], audio[:lay.cond_audio_rows])
    assert not np.array_equal(gv[lay.cond_rows:], video[lay.cond_rows:])


def test_denoise_progress_reports_and_cancels(cuda):
    lay, text, video, audio = inputs(MINI_LAYOUT, MINI)
    sv = H.sigmas(6, 5.0)
    m = H.Model(MINI, seed=2)
    m.begin(text, lay)
    seen = []

    def progress(i, n):
        seen.append((i, n))
        return i < 2

    gv, ga, ran = m.denoise(video, audio, sv, sv, progress)
    assert ran == 2 and seen == [(1, 5), (2, 5)]
    hv, ha = _host_loop(m, video, audio, sv, sv, 2, lay.cond_rows, lay.cond_audio_rows)
    m.close()
    np.testing.assert_array_equal(gv, hv)
    np.testing.assert_array_equal(ga, ha)


EDGE = dict(dim=256, heads=2, ffn=512, blocks=2, time_dim=128, text_dim=256, refiner=1)


@pytest.mark.parametrize("layout", [
    dict(text=1, frames=1, h=2, w=2, audio=0),                                              # two rows in all
    dict(text=3, frames=5, h=6, w=10, audio=3),                                             # cubes cut short on every axis
    dict(text=130, frames=9, h=10, w=2, audio=65, cond_frames=2, cond_last=[0, 1]),          # odd sizes, keyframes
    dict(text=5, frames=2, h=4, w=4, audio=0, refs=[dict(kind="audio", audio=7)]),           # a lone reference soundtrack
])
def test_step_edge_layouts(cuda, layout):
    """Small and ragged layouts (row counts that fill no tile, one-row cubes, cubes cut short in frames, rows and
    columns, odd audio and text counts, keyframes at both ends, a lone reference soundtrack): dense against the
    oracle; sparse with every cube selected against dense; sparse at 0.3 with local 3 finite and repeatable."""
    lay, text, video, audio = inputs(layout, EDGE)

    def run(sparse, local=1):
        m = H.Model(EDGE, seed=4, sparse_ratio=sparse, sparse_local=local)
        m.begin(text, lay)
        out = m.step(video, audio, 0.6, 0.3)
        m.close()
        return out

    dv, da = run(0.0)
    ov, oa = O.step(EDGE, O.make_weights(EDGE, 4), layout, text, video, audio, 0.6, 0.3)
    for g, o, wdt in ((dv, ov, 96), (da, oa, 32)):
        if o.size:
            rel, cos = O.diff(g, o, wdt)
            assert rel < VEL_REL and cos > VEL_COS, (rel, cos)
    sv, sa = run(1.0)
    for g, o, wdt in ((sv, dv, 96), (sa, da, 32)):
        if o.size:
            rel, cos = O.diff(g, o, wdt)
            assert rel < 1e-2 and cos > 0.9999, (rel, cos)
    p1, p2 = run(0.3, 3), run(0.3, 3)
    for a, b in zip(p1, p2):
        assert np.isfinite(a).all()
        np.testing.assert_array_equal(a, b)


def _lora_file(path, cfg, rank=16, seed=3, extra=()):
    """A Diffusers-named LoRA over several kinds of target (two q/k/v thirds, the out projection, fc1 with its
    [value; gate] rows, fc2, an AdaLN projection) plus a token-refiner target this build skips."""
    from tests import safetensors_util as ST
    d, inner, F, td = cfg["dim"], cfg["heads"] * 128, cfg["ffn"], cfg["time_dim"]
    shapes = {"transformer_blocks.0.attn.to_q": (inner, d), "transformer_blocks.0.attn.to_v": (inner, d),
              "transformer_blocks.0.attn.to_out.0": (d, inner), "transformer_blocks.1.ff.net.0.proj": (2 * F, d),
              "transformer_blocks.1.ff.net.2": (d, F), "transformer_blocks.2.adaln_proj.linear": (18 * d, td),
              "token_refiner.blocks.0.attn.to_q": (d, d)}
    shapes.update(dict(extra))
    rng = np.random.default_rng(seed)
    tensors, adapters = {}, {}
    for name, (out, inn) in shapes.items():
        # large enough that every merged matrix moves the output well past the parity tolerance
        A = rng.standard_normal((rank, inn)) * 0.15
        B = rng.standard_normal((out, rank)) * 0.15
        tensors["transformer." + name + ".lora_A.weight"] = A
        tensors["transformer." + name + ".lora_B.weight"] = B
        adapters[name] = (ST.bf16_values(A), ST.bf16_values(B))  # the values the BF16 file holds
    ST.write(path, tensors, metadata={"alpha": 8})
    return adapters


def test_add_lora_merges_like_the_oracle(cuda, tmp_path):
    """H3::add_lora on a BF16 LoRA file: the merged step against the oracle with the same adapters merged in its own
    layout; and far from the unmerged model, so every mapped target took effect."""
    path = tmp_path / "turbo.safetensors"
    adapters = _lora_file(path, MINI)
    lay, text, video, audio = inputs(MINI_LAYOUT, MINI)
    m = H.Model(MINI, seed=0)
    merged, skipped = m.add_lora(path, scale=0.7)
    assert (merged, skipped) == (6, 1)
    m.begin(text, lay)
    gv, ga = m.step(video, audio, 0.7, 0.4)
    m.close()
    w = O.make_weights(MINI, 0)
    ov0, _ = O.step(MINI, w, MINI_LAYOUT, text, video, audio, 0.7, 0.4)
    assert O.apply_lora(MINI, w, adapters, 0.7, alpha=8.0) == 6
    ov, oa = O.step(MINI, w, MINI_LAYOUT, text, video, audio, 0.7, 0.4)
    for g, o, wdt in ((gv, ov, 96), (ga, oa, 32)):
        rel, cos = O.diff(g, o, wdt)
        assert rel < VEL_REL and cos > VEL_COS, (rel, cos)
    assert O.diff(ov0, ov, 96)[0] > 2 * VEL_REL  # the merge moves the model past the tolerance


LORA_TARGETS = ["transformer_blocks.0.attn.to_q", "transformer_blocks.0.attn.to_v", "transformer_blocks.0.attn.to_out.0",
                "transformer_blocks.1.ff.net.0.proj", "transformer_blocks.1.ff.net.2", "transformer_blocks.2.adaln_proj.linear"]


@pytest.mark.parametrize("target", LORA_TARGETS)
def test_add_lora_each_target_moves_the_step_like_the_oracle(cuda, tmp_path, target):
    """One adapter at a time: the change it makes to the velocities on the GPU against the change the oracle's own
    merge makes (the bf16 noise of the two GPU runs largely cancels in the difference, so a row mapped to the wrong
    place would show as an unrelated change)."""
    from tests import safetensors_util as ST
    path = tmp_path / "one.safetensors"
    adapters = _lora_file(path, MINI)
    ST.write(path, {"transformer." + target + ".lora_A.weight": adapters[target][0].numpy(),
                    "transformer." + target + ".lora_B.weight": adapters[target][1].numpy()}, metadata={"alpha": 8})
    lay, text, video, audio = inputs(MINI_LAYOUT, MINI)
    outs = []
    for merge in (False, True):
        m = H.Model(MINI, seed=0)
        if merge:
            assert m.add_lora(path, scale=2.0) == (1, 0)
        m.begin(text, lay)
        outs.append(m.step(video, audio, 0.7, 0.4)[0])
        m.close()
    w = O.make_weights(MINI, 0)
    o0, _ = O.step(MINI, w, MINI_LAYOUT, text, video, audio, 0.7, 0.4)
    O.apply_lora(MINI, w, {target: adapters[target]}, 2.0, alpha=8.0)
    o1, _ = O.step(MINI, w, MINI_LAYOUT, text, video, audio, 0.7, 0.4)
    d_gpu, d_ref = outs[1] - outs[0], o1 - o0
    rel = np.linalg.norm(d_gpu - d_ref) / np.linalg.norm(d_ref)
    assert np.linalg.norm(d_ref) > 1e-3 * np.linalg.norm(o0)
    assert rel < 0.2, rel


def test_add_lora_int8_and_strict(cuda, tmp_path):
    """int8 weights take the adapters by requantising their rows (close to the bf16 merge); strict refuses names that
    match no H3 weight; a file with a bad shape is refused."""
    path = tmp_path / "turbo.safetensors"
    adapters = _lora_file(path, MINI)
    lay, text, video, audio = inputs(MINI_LAYOUT, MINI)
    m = H.Model(MINI, seed=0, int8_mask=H.INT8_QKV | H.INT8_OUT | H.INT8_FC1 | H.INT8_FC2)
    assert m.add_lora(path, scale=0.7) == (6, 1)
    m.begin(text, lay)
    gv, _ = m.step(video, audio, 0.7, 0.4)
    m.close()
    w = O.make_weights(MINI, 0)
    O.apply_lora(MINI, w, adapters, 0.7, alpha=8.0)
    ov, _ = O.step(MINI, w, MINI_LAYOUT, text, video, audio, 0.7, 0.4, int8=15)
    rel, cos = O.diff(gv, ov, 96)
    assert rel < 3e-2 and cos > 0.995, (rel, cos)
    bad = tmp_path / "unknown.safetensors"
    _lora_file(bad, MINI, extra=[("transformer_blocks.0.attn.to_z", (512, 512))])
    m = H.Model(MINI, seed=0)
    with pytest.raises(H.H3Error):
        m.add_lora(bad, strict=True)
    assert m.add_lora(bad, strict=False) == (6, 2)
    wrong = tmp_path / "wrong.safetensors"
    _lora_file(wrong, MINI, extra=[("transformer_blocks.0.ff.net.2", (512, 999))])
    with pytest.raises(H.H3Error):
        m.add_lora(wrong)
    m.close()
