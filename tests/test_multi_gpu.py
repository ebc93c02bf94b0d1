"""Sequence-parallel (Ulysses) step on 2 GPUs, one process per GPU over NCCL: every rank must return the velocities the
single-GPU step returns (the same kernels see the same rows and keys; only the rows' placement differs). Skipped
with fewer than two GPUs."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CFG = dict(dim=512, heads=4, ffn=1280, blocks=2, time_dim=256, text_dim=512, refiner=2)
LAYOUT = dict(text=40, frames=6, h=12, w=14, audio=24, cond_frames=1, cond_last=[1])


# 640 rows: five 128-key blocks, so the dense attention's few CTAs split their keys in two (combine kernel)
LAYOUT_SPLIT = dict(text=64, frames=8, h=16, w=16, audio=32)


def _inputs(layout=None):
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "mako-video_b200"))
    import h3b200 as H
    layout = layout or LAYOUT
    lay = H.Layout(**layout)
    rng = np.random.default_rng(5)
    text = rng.standard_normal((layout["text"], CFG["text_dim"]), dtype=np.float32)
    video = rng.standard_normal((lay.video_rows, 96), dtype=np.float32)
    audio = rng.standard_normal((lay.audio_rows, 32), dtype=np.float32)
    return H, lay, text, video, audio


def _rank(rank, world, nccl_id, sparse, q, exchange="fused", int8_mask=0, cfg=None, layout=None):
    os.environ["H3_EXCHANGE"] = exchange
    H, lay, text, video, audio = _inputs(layout)
    torch.cuda.set_device(rank)
    m = H.Model(cfg or CFG, seed=1, rank=rank, world=world, nccl_id=nccl_id, device=rank, sparse_ratio=sparse, sparse_local=1,
                int8_mask=int8_mask)
    m.begin(text, lay)
    v, a = m.step(video, audio, 0.7, 0.4)
    v2, a2 = m.step(video, audio, 0.3, 0.2)
    m.close()
    q.put((rank, v, a, v2, a2))


def _compare_two_ranks_with_one(sparse, exchange, int8_mask=0, cfg=None, layout=None):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    H, *_ = _inputs()
    nccl_id = H.nccl_unique_id()
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, nccl_id, sparse, q, exchange, int8_mask, cfg, layout)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=300)
        res[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    one = ctx.Process(target=_rank, args=(0, 1, None, sparse, q, exchange, int8_mask, cfg, layout))
    one.start()
    ref = q.get(timeout=300)[1:]
    one.join(timeout=120)
    for rank in (0, 1):
        for got, want in zip(res[rank], ref):
            rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
            assert rel < 1e-5, (rank, rel)


@pytest.mark.parametrize("exchange", ["fused", "nccl"])
@pytest.mark.parametrize("sparse", [0.0, 0.5])
def test_two_rank_step_matches_one_rank(cuda, sparse, exchange):
    """exchange: fused = the epilogues store into the peers' buffers over NVLink; nccl = NCCL all-to-alls."""
    _compare_two_ranks_with_one(sparse, exchange)


@pytest.mark.parametrize("exchange", ["fused", "nccl"])
def test_two_rank_int8_step_matches_one_rank(cuda, exchange):
    """W8A8 on every projection: the out projection's input arrives in per-rank column chunks and is quantised per
    row across them, so the int8 rows (and the step) equal the single-rank ones."""
    H, *_ = _inputs()
    _compare_two_ranks_with_one(0.0, exchange, int8_mask=H.INT8_QKV | H.INT8_OUT | H.INT8_FC1 | H.INT8_FC2)


@pytest.mark.parametrize("exchange", ["fused", "nccl"])
def test_two_rank_split_key_attention_matches_one_rank(cuda, exchange):
    """A layout whose dense attention launch is a few CTAs: the keys of every CTA are split in two and a combine
    kernel merges the halves, storing each row into its owner's buffer (fused) or the local one (nccl)."""
    _compare_two_ranks_with_one(0.0, exchange, layout=LAYOUT_SPLIT)


def test_two_rank_pruned_checkpoint_step_matches_one_rank(cuda):
    """A pruned checkpoint: every rank projects the curve point for all blocks itself (no AdaLN all-gather)."""
    _compare_two_ranks_with_one(0.0, "fused", cfg=dict(CFG, curve=8))


def _two_devices_one_process(q):
    H, lay, text, video, audio = _inputs()
    out = []
    for dev in (0, 1):
        m = H.Model(dict(CFG, blocks=1), seed=1, device=dev, sparse_ratio=0.5, sparse_local=1)
        m.begin(text, lay)
        out.append(m.step(video, audio, 0.7, 0.4))
        m.close()
    q.put(out)


def test_models_on_two_devices_in_one_process(cuda):
    """One process driving two GPUs (a model on each, one after the other): every kernel's per-device set-up (the
    dynamic shared-memory opt-in) must happen on each device, and both give the same velocities."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_two_devices_one_process, args=(q,))
    p.start()
    (v0, a0), (v1, a1) = q.get(timeout=300)
    p.join(timeout=120)
    assert p.exitcode == 0
    np.testing.assert_array_equal(v0, v1)
    np.testing.assert_array_equal(a0, a1)
