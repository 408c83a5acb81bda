"""Generates the golden fixtures in this directory by running the REFERENCE's own Python code.

Run only where the reference sources are present; give their root as the argument or in
$B2_REFERENCE_ROOT:

    python tests/golden/make_golden.py <reference-root>

The reference package cannot be imported as a whole here (``import torch_vulkan`` dlopens its Vulkan
extension, torch_vulkan/__init__.py:18-29), so this script parses the reference files with ``ast`` and
executes, unchanged, only the functions that run on the CPU:

* ``dequant_int8`` of torch_vulkan/__init__.py:193-205 (its pure-PyTorch branch is the reference's
  CPU implementation of the dequant), driven by ``make`` of tests/test_dequant_int8.py:24-30 over the
  13 shapes x 3 dtypes of tests/test_dequant_int8.py:36-48 and the extreme-value case of 51-55;
* the seeded input generators ``rnd`` of tests/test_mm.py:26-28, tests/test_fused_attention.py:43-45,
  tests/test_rows.py:24-26 and tests/test_ops_ew.py:27-29, and the CPU reference computations the
  reference tests compare against (``reference`` of tests/test_fused_attention.py:54-60, ``ref_ln`` of
  tests/test_rows.py:79-81).

Outputs: dequant_int8.json (sha256 of inputs/outputs for every case), dequant_small.npz (full arrays of
the small cases) and ops_small.npz (inputs and reference outputs of small mm/sdpa/softmax/LN/ternary
cases). Nothing here is needed at test time except these files.
"""

from __future__ import annotations

import ast
import hashlib
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("B2_REFERENCE_ROOT", "")
if not REF or not os.path.isdir(REF):
    sys.exit("make_golden.py: pass the reference source root as the argument or set B2_REFERENCE_ROOT")


def load_functions(path, names, extra_globals=None):
    """Executes the named top-level function definitions of a reference file and returns them."""
    with open(os.path.join(REF, path), encoding="utf-8") as f:
        tree = ast.parse(f.read())
    mod = ast.Module(body=[n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names], type_ignores=[])
    ns = {"torch": torch, "F": F}
    ns.update(extra_globals or {})
    exec(compile(mod, path, "exec"), ns)
    missing = [n for n in names if n not in ns]
    if missing:
        raise RuntimeError(f"{path}: functions not found: {missing}")
    return [ns[n] for n in names]


def sha(t: torch.Tensor) -> str:
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def np_of(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()  # bf16 bit patterns
    return t.numpy()


DEQ_SHAPES = [(1, 64), (1, 36), (3, 100), (5, 4608), (2, 63), (7, 65), (4, 1), (1, 1), (320, 2880), (1280, 5120),
              (2048, 8192), (640, 1280), (33, 130)]
DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def main():
    if not os.path.isdir(REF):
        sys.exit(f"reference sources not found at {REF}")
    (ref_dequant,) = load_functions("torch_vulkan/__init__.py", ["dequant_int8"])
    (make,) = load_functions("tests/test_dequant_int8.py", ["make"])

    cases, small = [], {}
    for rows, cols in DEQ_SHAPES:
        q, scale = make(rows, cols, seed=rows * 1000 + cols)
        for dn, dt in DTYPES.items():
            out = ref_dequant(q, scale, dt)  # CPU input -> the reference's pure-PyTorch branch
            cases.append({"rows": rows, "cols": cols, "seed": rows * 1000 + cols, "dtype": dn, "q_sha": sha(q),
                          "scale_sha": sha(scale), "out_sha": sha(out)})
            if rows * cols <= 8192:
                key = f"{rows}x{cols}_{dn}"
                small[key + "_q"] = np_of(q)
                small[key + "_scale"] = np_of(scale)
                small[key + "_out"] = np_of(out)
    # extremes and a zero scale (tests/test_dequant_int8.py:51-55)
    q = torch.tensor([[-128, -127, 0, 1, 127] * 13], dtype=torch.int8)
    scale = torch.tensor([[0.5, 0.0]], dtype=torch.bfloat16)
    for dn, dt in DTYPES.items():
        out = ref_dequant(q, scale, dt)
        small[f"extreme_{dn}_q"] = np_of(q)
        small[f"extreme_{dn}_scale"] = np_of(scale)
        small[f"extreme_{dn}_out"] = np_of(out)
    with open(os.path.join(HERE, "dequant_int8.json"), "w") as f:
        json.dump({"source": "torch_vulkan/__init__.py:193-205 via tests/test_dequant_int8.py:24-48",
                   "torch": torch.__version__, "cases": cases}, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "dequant_small.npz"), **small)

    # ---- small op cases through the reference tests' generators and CPU references ----------------
    ops = {}
    (rnd_mm,) = load_functions("tests/test_mm.py", ["rnd"])
    for m, k, n in [(7, 5, 3), (65, 17, 63), (33, 100, 40)]:
        for dn in ("float32", "bfloat16"):
            a, b = rnd_mm((m, k), DTYPES[dn], 1), rnd_mm((k, n), DTYPES[dn], 2)
            key = f"mm_{m}x{k}x{n}_{dn}"
            ops[key + "_a"], ops[key + "_b"] = np_of(a), np_of(b)
            ops[key + "_ref"] = (a.double() @ b.double()).numpy()  # tests/test_mm.py:59

    rnd_attn, reference = load_functions("tests/test_fused_attention.py", ["rnd", "reference"])
    for shape in [(1, 2, 40, 50, 64), (1, 2, 17, 5, 20), (1, 1, 48, 48, 36)]:
        B, H, Sq, Sk, D = shape
        for dn in ("float32", "bfloat16"):
            dt = DTYPES[dn]
            q, k, v, g = rnd_attn((B, H, Sq, D), dt, 1), rnd_attn((B, H, Sk, D), dt, 2), rnd_attn((B, H, Sk, D), dt, 3), rnd_attn((B, H, Sq, D), dt, 4)
            o, dq, dk, dv = reference(q, k, v, g)  # CPU fp32 MATH backend fwd + bwd
            key = "sdpa_" + "x".join(map(str, shape)) + "_" + dn
            for nm, t in (("q", q), ("k", k), ("v", v), ("g", g)):
                ops[f"{key}_{nm}"] = np_of(t)
            for nm, t in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
                ops[f"{key}_{nm}_ref"] = t.numpy()

    rnd_rows, ref_ln = load_functions("tests/test_rows.py", ["rnd", "ref_ln"])
    for shape, dim in [((7, 33), -1), ((3, 5, 4), 1), ((4, 5000), -1)]:
        x = rnd_rows(shape, torch.float32, scale=3.0)
        key = "softmax_" + "x".join(map(str, shape)) + f"_d{dim}"
        ops[key + "_x"] = np_of(x)
        ops[key + "_ref"] = torch.softmax(x.double(), dim).numpy()  # tests/test_rows.py:46-51
    for rows, D in [(3, 7), (5, 256), (2, 2048)]:
        x = rnd_rows((rows, D), torch.float32, scale=2.0)
        w, b = rnd_rows((D,), torch.float32, 1), rnd_rows((D,), torch.float32, 2)
        key = f"ln_{rows}x{D}"
        ops[key + "_x"], ops[key + "_w"], ops[key + "_b"] = np_of(x), np_of(w), np_of(b)
        ops[key + "_ref"] = ref_ln(x, (D,), w, b).numpy()  # eps 1e-5 default of ref_ln

    (rnd_ew,) = load_functions("tests/test_ops_ew.py", ["rnd"])
    a, b, c = rnd_ew((6, 9), torch.float32, seed=1), rnd_ew((6, 9), torch.float32, seed=2), rnd_ew((6, 9), torch.float32, 0.5, 3.0, seed=3)
    ops["ew_a"], ops["ew_b"], ops["ew_c"] = np_of(a), np_of(b), np_of(c)
    ops["ew_addcmul_ref"] = torch.addcmul(a, b, c, value=0.3).numpy()  # tests/test_ops_ew.py:295
    ops["ew_addcdiv_ref"] = torch.addcdiv(a, b, c, value=-0.7).numpy()
    ops["ew_lerp_ref"] = torch.lerp(a, b, 0.1).numpy()
    np.savez_compressed(os.path.join(HERE, "ops_small.npz"), **ops)
    print("wrote", len(cases), "dequant cases,", len(small), "small dequant arrays,", len(ops), "op arrays")


if __name__ == "__main__":
    main()
