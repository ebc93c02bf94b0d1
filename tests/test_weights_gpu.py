"""Checkpoints through the C ABI: a model's weights written by h3_save_weights load back (h3_create with the path) to
the same step, from one file or a directory of shards; a file in the reference's interleaved q/k/v layout
(docs/architecture.md:62-63) is stacked at load; int8 quantisation at load; pruned checkpoints."""
import numpy as np
import pytest

import h3b200 as H
from tests import safetensors_util as ST
from tests.test_step_gpu import MINI, MINI_LAYOUT, inputs

pytestmark = pytest.mark.gpu


def _step(model, cfg=MINI):
    lay, text, video, audio = inputs(MINI_LAYOUT, cfg)
    model.begin(text, lay)
    out = model.step(video, audio, 0.7, 0.4)
    model.close()
    return out


def _same(a, b):
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def _save(cfg, path, seed=3):
    m = H.Model(cfg, seed=seed)
    m.save_weights(path)
    m.close()


def test_saved_weights_load_back_to_the_same_step(cuda, tmp_path):
    p = tmp_path / "h3.safetensors"
    _save(MINI, p)
    assert H.check_weights(MINI, p) == ""
    _same(_step(H.Model(MINI, weights=p)), _step(H.Model(MINI, seed=3)))
    # the same tensors as a directory of two shards
    t, dt, meta = ST.read(p)
    names = list(t)
    d = tmp_path / "shards"
    d.mkdir()
    ST.write(d / "model-00001.safetensors", {n: t[n] for n in names[::2]}, meta, {n: dt[n] for n in names[::2]})
    ST.write(d / "model-00002.safetensors", {n: t[n] for n in names[1::2]}, meta, {n: dt[n] for n in names[1::2]})
    _same(_step(H.Model(MINI, weights=d)), _step(H.Model(MINI, seed=3)))


def test_interleaved_qkv_checkpoint_is_stacked_at_load(cuda, tmp_path):
    """Each head's q, k and v rows together ([q_h; k_h; v_h]), metadata qkv_layout = interleaved: the loader stacks
    them q, k, v (the reference's upload_qkv) and the step is the stacked checkpoint's."""
    p = tmp_path / "stacked.safetensors"
    _save(MINI, p)
    t, dt, meta = ST.read(p)
    heads = MINI["heads"]
    for name in list(t):
        if name.endswith("attn.qkv.weight") or name.endswith("attn.qkv.bias"):
            a = t[name]
            parts = a.reshape((3, heads, 128) + a.shape[1:])
            t[name] = np.ascontiguousarray(parts.transpose((1, 0, 2) + tuple(range(3, parts.ndim)))).reshape(a.shape)
    q = tmp_path / "interleaved.safetensors"
    ST.write(q, t, dict(meta, qkv_layout="interleaved"), dt)
    _same(_step(H.Model(MINI, weights=q)), _step(H.Model(MINI, weights=p)))


def test_int8_quantised_at_load(cuda, tmp_path):
    p = tmp_path / "h3.safetensors"
    _save(MINI, p)
    _same(_step(H.Model(MINI, weights=p, int8_mask=15)), _step(H.Model(MINI, seed=3, int8_mask=15)))


def test_pruned_checkpoint_round_trip(cuda, tmp_path):
    cfg = dict(MINI, curve=8)
    p = tmp_path / "pruned.safetensors"
    _save(cfg, p)
    _same(_step(H.Model(cfg, weights=p), cfg), _step(H.Model(cfg, seed=3), cfg))


def test_an_int8_model_does_not_save(cuda, tmp_path):
    m = H.Model(MINI, seed=3, int8_mask=H.INT8_QKV)
    with pytest.raises(H.H3Error) as e:
        m.save_weights(tmp_path / "x.safetensors")
    m.close()
    assert e.value.code == H.H3_ERR_ARG


def test_a_checkpoint_of_another_shape_is_refused_before_device_work(cuda, tmp_path):
    p = tmp_path / "h3.safetensors"
    _save(MINI, p)
    other = dict(MINI, ffn=1536)
    assert "ff.fc1.weight is 2560x512, this model needs 3072x512" in H.check_weights(other, p)
    with pytest.raises(H.H3Error) as e:
        H.Model(other, weights=p)
    assert e.value.code == H.H3_ERR_ARG
