"""The C++ drop-in headers (include/models/h3.hpp, include/video/video_vae.hpp) compile against the reference's usage and its host-side members
work through libh3b200.so (no GPU needed)."""
import ctypes
import os
import subprocess

import h3b200

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_dropin_header_compiles_and_runs(tmp_path):
    lib = h3b200.LIB_PATH
    exe = tmp_path / "dropin_check"
    subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-I", os.path.join(REPO, "include"),
                    os.path.join(REPO, "tests", "cpp", "dropin_check.cpp"), "-o", str(exe), lib,
                    "-Wl,-rpath," + os.path.dirname(lib)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout
    # the ctypes declarations of the Python binding match the header's struct layouts
    abi = {line.split()[1]: [int(v) for v in line.split()[2:]] for line in r.stdout.splitlines() if line.startswith("abi ")}
    H = h3b200
    want = {
        "h3_config": [ctypes.sizeof(H.h3_config), H.h3_config.refiner_blocks.offset, H.h3_config.curve_dims.offset],
        "h3_layout": [ctypes.sizeof(H.h3_layout), H.h3_layout.refs.offset, H.h3_layout.n_refs.offset],
        "h3_layout_ref": [ctypes.sizeof(H.h3_layout_ref)],
        "h3_world": [ctypes.sizeof(H.h3_world), H.h3_world.nccl_id.offset],
        "h3k_gemm_args": [ctypes.sizeof(H.h3k_gemm_args), H.h3k_gemm_args.b_scale.offset],
        "h3k_cube_grid": [ctypes.sizeof(H.h3k_cube_grid)],
        "h3vae_config": [ctypes.sizeof(H.h3vae_config), H.h3vae_config.eps.offset],
    }
    assert abi == want, (abi, want)
