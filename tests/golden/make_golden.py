"""Generates the golden fixtures in this directory from the reference's own code (run here, where the reference is
mounted; the fixtures travel, the reference does not):

  time_adaln.npz  the time embedding and the AdaLN projection exactly as tools/check_pruned_curve.py:58-67 computes
                  them (its functions `temb` and `mods_full`, taken from the file's syntax tree and executed in float64
                  on seeded small weights)
  rope_freq.npy   the rotary frequencies exactly as tools/dump_h3_ref.py:140-141 builds them (the expression taken from
                  the file's syntax tree and evaluated with torch on the CPU)
  curve.npz       a pruned checkpoint's curve lookup exactly as tools/check_pruned_curve.py:66-70 does it (its function
                  `c_of`, taken from the file's syntax tree and executed in float64 on a seeded [1025][8] table, at the
                  t * 1024 positions the reference implements, and past both ends)
  geometry.json   the known answers of tests/geometry_test.cpp:22-43 (read as text)

    python tests/golden/make_golden.py [/path/to/reference]
"""
import ast
import json
import math
import os
import re
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def functions_from(path, names):
    tree = ast.parse(open(path).read())
    out = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    if len(out) != len(names):
        raise RuntimeError(f"{path}: functions {names} not found")
    return ast.Module(body=out, type_ignores=[])


def time_adaln(ref):
    path = os.path.join(ref, "tools", "check_pruned_curve.py")
    mod = functions_from(path, ["temb", "mods_full"])
    g = torch.Generator().manual_seed(1234)
    dm, td, R = 64, 32, 48  # small stand-ins for 5376 / 2688 / 96768
    ns = {"torch": torch, "math": math}
    w = {
        "p_in_w": torch.randn(dm, 256, generator=g, dtype=torch.float64) * 0.05,
        "p_in_b": torch.randn(dm, generator=g, dtype=torch.float64) * 0.05,
        "p_out_w": torch.randn(td, dm, generator=g, dtype=torch.float64) * 0.05,
        "p_out_b": torch.randn(td, generator=g, dtype=torch.float64) * 0.05,
        "Wf": torch.randn(R, td, generator=g, dtype=torch.float64) * 0.05,
        "bf": torch.randn(R, generator=g, dtype=torch.float64) * 0.05,
    }
    ns.update(w)
    exec(compile(mod, path, "exec"), ns)
    ts = [0.0, 0.0769230769, 0.25, 0.5, 0.7, 0.9, 0.999, 1.0]
    temb = np.stack([ns["temb"](t).numpy() for t in ts])
    mods = np.stack([ns["mods_full"](t).numpy() for t in ts])
    np.savez(os.path.join(HERE, "time_adaln.npz"), t=np.array(ts), temb=temb, mods=mods,
             **{k: v.numpy() for k, v in w.items()})


def curve(ref):
    path = os.path.join(ref, "tools", "check_pruned_curve.py")
    mod = functions_from(path, ["c_of"])
    g = torch.Generator().manual_seed(4321)
    table = torch.randn(1025, 8, generator=g, dtype=torch.float64) * 4.0
    ns = {"torch": torch, "math": math, "table": table}
    exec(compile(mod, path, "exec"), ns)
    # the levels as the step receives them (float), so the comparison measures the lookup and not the rounding of t
    ts = [float(np.float32(t)) for t in (0.0, 1e-4, 0.0769230769, 0.25, 0.3333333, 0.5, 0.7, 0.9, 0.999, 0.99999, 1.0)]
    c = np.stack([ns["c_of"](t * 1024).numpy() for t in ts])
    outside = np.stack([ns["c_of"](p).numpy() for p in (-3.5, 1030.25)])
    np.savez(os.path.join(HERE, "curve.npz"), table=table.numpy(), t=np.array(ts), c=c, outside_pos=np.array([-3.5, 1030.25]),
             outside=outside)


def rope_freq(ref):
    path = os.path.join(ref, "tools", "dump_h3_ref.py")
    tree = ast.parse(open(path).read())
    expr = None
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and ast.unparse(node.targets[0]) == "dit.rope.inv_freq" and isinstance(node.value, ast.IfExp):
            expr = node.value.orelse
    if expr is None:
        raise RuntimeError("dump_h3_ref.py: the inv_freq expression was not found")
    f = eval(compile(ast.Expression(expr), path, "eval"), {"torch": torch, "dev": torch.device("cpu")})
    np.save(os.path.join(HERE, "rope_freq.npy"), f.numpy().astype(np.float32))


def geometry(ref):
    src = open(os.path.join(ref, "tests", "geometry_test.cpp")).read()
    kat = {
        "align_frames": [[int(a), int(b)] for a, b in re.findall(r"align_frames\((\d+)\) == (\d+)", src)],
        "latent_frames": [[int(a), int(b)] for a, b in re.findall(r"latent_frames\((\d+)\) == (\d+)", src)],
        "audio_latents": [[int(a), int(b)] for a, b in re.findall(r"audio_latents\((\d+)\) == (\d+)", src)],
    }
    json.dump(kat, open(os.path.join(HERE, "geometry.json"), "w"), indent=1)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MAKO_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py REFERENCE_CHECKOUT (or set MAKO_REFERENCE): the mako-video source tree to read")
    time_adaln(ref)
    rope_freq(ref)
    geometry(ref)
    curve(ref)
    print("golden fixtures written to", HERE)
