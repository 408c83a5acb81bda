"""The C-ABI library loads and exports every function include/b2rt.h declares (no GPU needed)."""

import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "torch_vulkan_b200", "libb2rt.so")
HDR = os.path.join(ROOT, "include", "b2rt.h")


def declared_functions():
    src = open(HDR).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(b2\w*)\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if not n.startswith("B2")))


def test_header_declares_the_expected_families():
    names = declared_functions()
    for must in ("b2rt_init", "b2rt_last_error", "b2rt_alloc", "b2rt_free", "b2_malloc", "b2_free", "b2_gemm",
                 "b2_int8_gemm", "b2_dequant_int8", "b2_attn_fwd", "b2_attn_bwd", "b2_softmax_fwd", "b2_softmax_bwd",
                 "b2_layernorm_fwd", "b2_layernorm_bwd", "b2_ew_ternary", "b2_adamw_step", "b2_mse_loss_fwd",
                 "b2_mse_loss_bwd"):
        assert must in names, must


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_non_compute_calls_work_without_gpu():
    lib = ctypes.CDLL(LIB)
    lib.b2rt_stat.restype = ctypes.c_uint64
    assert lib.b2rt_stat(99) == 0
    lib.b2rt_count_op(b"unit::probe")
    n = lib.b2rt_op_counts(None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    lib.b2rt_op_counts(buf, n + 1)
    assert "unit::probe\t" in buf.value.decode()
    lib.b2rt_reset_op_counts()
    assert lib.b2rt_op_counts(None, 0) == 0


def test_kernel_entry_points_reject_bad_arguments_on_the_host():
    """Argument validation happens before any device work; with no GPU the calls must still return
    an error code (never crash)."""
    lib = ctypes.CDLL(LIB)
    assert lib.b2_gemm(None, None) < 0
    assert lib.b2_dequant_int8(None, None) < 0
    assert lib.b2_attn_fwd(None, None) < 0
    n = lib.b2rt_last_error(None, 0)
    assert n > 0
