"""Pins the CPU oracle to the reference: its outputs must match the golden fixtures produced by the
reference's own Python code (tests/golden/make_golden.py), bit-exactly for int8 dequant and rounding."""

import ctypes
import hashlib
import json
import os
import subprocess

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import from_np, make_int8, rnd_mm, rnd_normal, rnd_range, rnd_unit

GOLD = os.path.join(os.path.dirname(__file__), "golden")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def sha(t):
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


@pytest.fixture(scope="module")
def gold_dequant():
    with open(os.path.join(GOLD, "dequant_int8.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def small():
    return np.load(os.path.join(GOLD, "dequant_small.npz"))


@pytest.fixture(scope="module")
def ops():
    return np.load(os.path.join(GOLD, "ops_small.npz"))


def test_generators_reproduce_reference_inputs(gold_dequant):
    """make_int8 regenerates exactly the reference's int8 test inputs (sha256 of q and scale)."""
    for c in gold_dequant["cases"]:
        q, s = make_int8(c["rows"], c["cols"], c["seed"])
        assert sha(q) == c["q_sha"] and sha(s) == c["scale_sha"], c


def test_oracle_dequant_matches_reference_bitwise(gold_dequant):
    """Every case of tests/test_dequant_int8.py:36-48 (13 shapes x 3 dtypes), compared by sha256."""
    for c in gold_dequant["cases"]:
        q, s = make_int8(c["rows"], c["cols"], c["seed"])
        out = oracle.dequant_int8(q, s, DT[c["dtype"]])
        assert sha(out) == c["out_sha"], c


def test_oracle_dequant_small_arrays_and_extremes(small):
    keys = sorted({k.rsplit("_", 1)[0] for k in small.files})
    assert any(k.startswith("extreme") for k in keys)
    for k in keys:
        dn = k.split("_")[-1]
        dt = DT[dn]
        q = torch.from_numpy(small[k + "_q"])
        s = from_np(small[k + "_scale"], torch.bfloat16)
        want = from_np(small[k + "_out"], dt)
        got = oracle.dequant_int8(q, s, dt)
        assert torch.equal(got.view(torch.int16) if dt != torch.float32 else got,
                           want.view(torch.int16) if dt != torch.float32 else want), k


def _liboracle():
    so = os.path.join(ROOT, "oracle", "liboracle.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)
    lib = ctypes.CDLL(so)
    lib.oracle_f2bf_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    lib.oracle_f2h_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    lib.oracle_dequant_int8.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_int]
    return lib


def _special_floats(n=1 << 18, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32) * np.float32(10.0) ** rng.integers(-8, 8, n).astype(np.float32)
    bits = rng.integers(0, 2**32, n // 4, dtype=np.uint64).astype(np.uint32).view(np.float32)
    specials = np.array([0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0, 6e-8, 3e-8, 1e-45, 3.3895314e38,
                         1.0 + 2**-8, 1.0 + 2**-9, 1.0 + 3 * 2**-9], dtype=np.float32)
    out = np.concatenate([x, bits, specials])
    return out[~np.isnan(out)]


def test_c_rounding_matches_torch_conversion():
    """The C restatement of the shaders' f2bf/f2h (types.glsl:18-50) equals torch's RNE conversion
    over random, random-bit and special values (NaN excluded: payloads differ by design)."""
    lib = _liboracle()
    x = _special_floats()
    bf = np.empty(x.size, np.uint16)
    hf = np.empty(x.size, np.uint16)
    lib.oracle_f2bf_array(x.ctypes.data, bf.ctypes.data, x.size)
    lib.oracle_f2h_array(x.ctypes.data, hf.ctypes.data, x.size)
    t = torch.from_numpy(x)
    np.testing.assert_array_equal(bf, t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
    np.testing.assert_array_equal(hf, t.to(torch.float16).view(torch.int16).numpy().view(np.uint16))
    np.testing.assert_array_equal(bf, oracle.f32_to_bf16_bits(x))


def test_c_dequant_matches_python_oracle():
    lib = _liboracle()
    for rows, cols in [(7, 65), (33, 130), (5, 4608)]:
        q, s = make_int8(rows, cols, rows * 1000 + cols)
        for kind, dt in ((0, torch.float32), (1, torch.bfloat16), (2, torch.float16)):
            out = np.empty(rows * cols, np.float32 if kind == 0 else np.uint16)
            lib.oracle_dequant_int8(q.numpy().ctypes.data, s.view(torch.int16).numpy().ctypes.data, out.ctypes.data,
                                    rows, cols, kind)
            want = oracle.dequant_int8(q, s, dt).reshape(-1)
            want = want.numpy() if kind == 0 else want.view(torch.int16).numpy().view(np.uint16)
            np.testing.assert_array_equal(out, want)


def test_oracle_gemm_matches_reference_tests(ops):
    for m, k, n in [(7, 5, 3), (65, 17, 63), (33, 100, 40)]:
        for dn in ("float32", "bfloat16"):
            key = f"mm_{m}x{k}x{n}_{dn}"
            a, b = from_np(ops[key + "_a"], DT[dn]), from_np(ops[key + "_b"], DT[dn])
            assert torch.equal(a, rnd_mm((m, k), DT[dn], 1)) and torch.equal(b, rnd_mm((k, n), DT[dn], 2))
            np.testing.assert_allclose(oracle.mm(a, b).numpy(), ops[key + "_ref"], rtol=0, atol=1e-12)


def test_oracle_sdpa_matches_reference_cpu_math(ops):
    """float64 oracle vs the reference test's CPU fp32 MATH fwd+bwd (tests/test_fused_attention.py:54-60)."""
    for shape in [(1, 2, 40, 50, 64), (1, 2, 17, 5, 20), (1, 1, 48, 48, 36)]:
        B, H, Sq, Sk, D = shape
        for dn in ("float32", "bfloat16"):
            key = "sdpa_" + "x".join(map(str, shape)) + "_" + dn
            q, k, v, g = (from_np(ops[f"{key}_{n}"], DT[dn]) for n in "qkvg")
            assert torch.equal(q, rnd_unit((B, H, Sq, D), DT[dn], 1))
            o, _ = oracle.sdpa_fwd(q, k, v)
            dq, dk, dv = oracle.sdpa_bwd(q, k, v, g)
            for name, got in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
                ref = torch.from_numpy(ops[f"{key}_{name}_ref"]).double()
                err = ((got - ref).norm() / (ref.norm() + 1e-12)).item()
                assert err < 2e-6, (key, name, err)


def test_oracle_rows_and_ternaries_match_reference(ops):
    for shape, dim in [((7, 33), -1), ((3, 5, 4), 1), ((4, 5000), -1)]:
        key = "softmax_" + "x".join(map(str, shape)) + f"_d{dim}"
        x = torch.from_numpy(ops[key + "_x"])
        assert torch.equal(x, rnd_normal(shape, torch.float32, scale=3.0))
        np.testing.assert_allclose(oracle.softmax(x, dim).numpy(), ops[key + "_ref"], rtol=1e-12, atol=1e-15)
    for rows, D in [(3, 7), (5, 256), (2, 2048)]:
        key = f"ln_{rows}x{D}"
        x, w, b = (torch.from_numpy(ops[key + s]) for s in ("_x", "_w", "_b"))
        y, mean, rstd = oracle.layer_norm(x, (D,), w, b)
        np.testing.assert_allclose(y.numpy(), ops[key + "_ref"], rtol=1e-9, atol=1e-9)
    a, b, c = (torch.from_numpy(ops["ew_" + s]) for s in "abc")
    assert torch.equal(c, rnd_range((6, 9), torch.float32, 0.5, 3.0, seed=3))
    np.testing.assert_allclose(oracle.addcmul(a, b, c, 0.3).numpy(), ops["ew_addcmul_ref"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(oracle.addcdiv(a, b, c, -0.7).numpy(), ops["ew_addcdiv_ref"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(oracle.lerp(a, b, 0.1).numpy(), ops["ew_lerp_ref"], rtol=1e-6, atol=1e-6)


def test_oracle_planted_mistake_is_caught():
    """A wrong oracle (scale applied per 32 columns instead of 64) must fail the golden check."""
    q, s = make_int8(7, 130, 7130)
    bad = (q.float() * s.float().repeat_interleave(32, 1)[:, :130].repeat(1, 2)[:, :130]).to(torch.bfloat16)
    with open(os.path.join(GOLD, "dequant_int8.json")) as f:
        case = next(c for c in json.load(f)["cases"] if c["rows"] == 7 and c["cols"] == 65)
    q65, s65 = make_int8(7, 65, 7065)
    bad65 = (q65.float() * s65.float()[:, :1]).to(torch.bfloat16)  # ignores the second 64-block
    assert sha(bad65) != case["out_sha"]
    assert not torch.equal(bad, oracle.dequant_int8(q, s, torch.bfloat16))
