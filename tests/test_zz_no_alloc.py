"""h3k_sparse_attention_noalloc: the sparse attention for callers that cannot call cudaMalloc (a serving stack whose
device memory is already reserved by its own pool, or one that cannot afford the device-wide synchronisation of
cudaMalloc / cudaFree). It must give what the allocating entry point gives, on consecutive calls that share its
fixed scratch, and refuse work that does not fit that scratch. Both entry points run the same kernels on the same
inputs, so their outputs must be identical bit for bit. Collected last (file name), so a run that stops at the first
failure has run every other test; it also passes alone in a fresh process."""
import ctypes

import pytest
import torch

import h3b200 as H

pytestmark = pytest.mark.gpu

def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _case(cuda, seed):
    dense, frames, ph, pw, heads = 70, 5, 6, 7, 2
    S = dense + frames * ph * pw
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(S, 3, heads, 128, generator=g)
    base = torch.randn(frames * ph * pw, heads, 128, generator=g)
    qkv[dense:, 0] += 2 * base
    qkv[dense:, 1] += 2 * base.roll(5, 0)
    return qkv.bfloat16().to(cuda), H.h3k_cube_grid(dense, frames, ph, pw)


def _run(fn, qkv, grid, ratio, local):
    S, _, heads, _ = qkv.shape
    out = torch.zeros(S, heads, 128, device=qkv.device, dtype=torch.bfloat16)
    H.check(fn(_ptr(qkv[:, 0]), _ptr(qkv[:, 1]), _ptr(qkv[:, 2]), 3 * heads * 128, heads, ctypes.byref(grid), ratio, local, _ptr(out),
               heads * 128, _stream()))
    H.check(H.lib().h3k_check(_stream()))
    return out


def test_noalloc_matches_the_allocating_entry_point_on_two_calls(cuda):
    qkv, grid = _case(cuda, 3)
    L = H.lib()
    for ratio, local in ((0.1, 1), (0.4, 3)):  # two calls in a row on the shared scratch, different selections
        want = _run(L.h3k_sparse_attention, qkv, grid, ratio, local)
        got = _run(L.h3k_sparse_attention_noalloc, qkv, grid, ratio, local)
        assert torch.equal(got, want), (ratio, local, float((got.double() - want.double()).abs().max()))


def test_noalloc_refuses_grids_beyond_its_scratch(cuda):
    tiny = torch.zeros(4, 3, 40, 128, device=cuda, dtype=torch.bfloat16)
    grid = H.h3k_cube_grid(768, 32, 24, 42)  # 528 cubes x 40 heads: the scores alone are 44.6 MB
    rc = H.lib().h3k_sparse_attention_noalloc(_ptr(tiny), _ptr(tiny), _ptr(tiny), 3 * 40 * 128, 40, ctypes.byref(grid), 0.1, 1,
                                              _ptr(tiny), 40 * 128, _stream())
    assert rc == H.H3_ERR_ARG
    msg = H.lib().h3_last_error().decode()
    assert "scratch" in msg and "bytes" in msg
