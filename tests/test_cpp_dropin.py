"""The C++ drop-in header (include/models/h3.hpp) compiles against the reference's usage and its host-side members
work through libh3b200.so (no GPU needed)."""
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
