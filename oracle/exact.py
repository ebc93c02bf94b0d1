"""ctypes access to oracle/h3_exact.c (the exact CPU restatement of the sparse coarse pass) -- TEST INFRASTRUCTURE
ONLY: tests/ use it as the checker of the library's cube selection."""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "h3_exact.c")
LIB = os.path.join(HERE, "libh3_exact.so")


def build(force=False):
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fopenmp", "-shared", "-fPIC", "-o", LIB, SRC, "-lm"], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        P, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.h3x_cube_pool.argtypes = [P, P, I64, I, I, I, I, I, P, P]
        L.h3x_cube_scores.argtypes = [P, P, I, I, P]
        L.h3x_cube_topk.argtypes = [P, I, I, I, I, I, I, P, P, I]
        L.h3x_synthetic.argtypes = [P, I64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float, I]
        _lib = L
    return _lib


def synthetic(n, key, mean, k, bf16):
    """h3x_synthetic: the loop form of oracle/h3_oracle.py:synthetic (key and k as that function derives them)."""
    out = np.empty(n, np.float32)
    lib().h3x_synthetic(out.ctypes.data, n, key, float(mean), float(k), 1 if bf16 else 0)
    return out


def grid_cubes(frames, ph, pw):
    return ((frames + 3) // 4) * ((ph + 3) // 4) * ((pw + 3) // 4)


def cube_pool(q_bits, k_bits, row_stride, heads, dense_rows, frames, ph, pw):
    """q_bits, k_bits: uint16 arrays of bf16 bits (flat, element (row, head, dim) at row*row_stride + head*128 + dim)."""
    nc = grid_cubes(frames, ph, pw)
    mq = np.zeros((heads, nc, 128), np.float32)
    mk = np.zeros((heads, nc, 128), np.float32)
    q_bits = np.ascontiguousarray(q_bits, np.uint16)
    k_bits = np.ascontiguousarray(k_bits, np.uint16)
    lib().h3x_cube_pool(q_bits.ctypes.data, k_bits.ctypes.data, row_stride, heads, dense_rows, frames, ph, pw, mq.ctypes.data,
                        mk.ctypes.data)
    return mq, mk


def cube_scores(mq, mk):
    heads, nc, _ = mq.shape
    s = np.zeros((heads, nc, nc), np.float32)
    mq = np.ascontiguousarray(mq, np.float32)
    mk = np.ascontiguousarray(mk, np.float32)
    lib().h3x_cube_scores(mq.ctypes.data, mk.ctypes.data, heads, nc, s.ctypes.data)
    return s


def sparse_k(ratio, cubes):
    """k = ceil(ratio * cubes) (1e-6 slack against float noise), at least 1 and at most the cubes."""
    import math
    return max(1, min(cubes, int(math.ceil(float(np.float32(ratio)) * cubes - 1e-6))))


def cube_topk(scores, frames, ph, pw, ratio, local):
    heads, nc, _ = scores.shape
    k = sparse_k(ratio, nc)
    forced = 0 if local <= 0 else (3 if local >= 3 else 1)
    kcap = min(max(k, forced), nc)
    sel = np.full((heads, nc, kcap), -1, np.int32)
    nsel = np.zeros((heads, nc), np.int32)
    scores = np.ascontiguousarray(scores, np.float32)
    lib().h3x_cube_topk(scores.ctypes.data, heads, frames, ph, pw, k, local, sel.ctypes.data, nsel.ctypes.data, kcap)
    return sel, nsel
