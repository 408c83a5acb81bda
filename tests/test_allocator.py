"""Slab allocator policy, tested host-only through the C ABI with the malloc-backed test backend.

Spec: the reference runtime's own tests vkrt/tests/basic.rs:14-182 (round trip with offsets,
out-of-range / unknown / double free rejected, above-maximum allocation fails, 20 000 small blocks in
< 20 slabs, coalescing, dedicated slabs released on free, empty_cache), plus the emulated memory limit
(vkrt/src/lib.rs:748-761, tests/test_memory_api.py:18-31). Each test runs in a fresh subprocess so the
process-wide allocator starts empty."""

import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PRELUDE = textwrap.dedent(
    f"""
    import ctypes
    lib = ctypes.CDLL({os.path.join(ROOT, 'torch_vulkan_b200', 'libb2rt.so')!r})
    u64 = ctypes.c_uint64
    for n in ("b2rt_alloc", "b2rt_live_bytes", "b2rt_peak_live_bytes", "b2rt_reserved_bytes", "b2rt_max_alloc"):
        getattr(lib, n).restype = u64
    lib.b2rt_alloc.argtypes = [u64]
    lib.b2rt_free.argtypes = [u64]
    lib.b2rt_upload.argtypes = [u64, ctypes.c_void_p, u64]
    lib.b2rt_download.argtypes = [ctypes.c_void_p, u64, u64]
    lib.b2rt_copy_d2d.argtypes = [u64, u64, u64]
    lib.b2rt_set_memory_limit.argtypes = [u64]
    lib.b2rt_slab_count.restype = ctypes.c_size_t
    lib.b2rt_live_blocks.restype = ctypes.c_size_t
    lib.b2rt_empty_cache.restype = ctypes.c_size_t
    assert lib.b2rt_debug_host_backend(1) == 0
    """
)


def run(body):
    r = subprocess.run([sys.executable, "-c", PRELUDE + textwrap.dedent(body)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr


def test_roundtrip_with_offsets_and_d2d():
    run("""
    import array
    n = 1000
    src = array.array('f', [i * 0.5 for i in range(n)])
    a, b = lib.b2rt_alloc(n * 4), lib.b2rt_alloc(n * 4)
    assert a and b and a % 512 == 0 and b % 512 == 0
    assert lib.b2rt_upload(a, src.buffer_info()[0], n * 4) == 0
    assert lib.b2rt_copy_d2d(b, a, n * 4) == 0
    out = array.array('f', [0.0] * n)
    assert lib.b2rt_download(out.buffer_info()[0], b, n * 4) == 0
    assert out == src
    part = array.array('f', [0.0] * 100)
    assert lib.b2rt_download(part.buffer_info()[0], b + 400, 400) == 0
    assert list(part) == list(src[100:200])
    assert lib.b2rt_free(a) == 0 and lib.b2rt_free(b) == 0
    """)


def test_out_of_range_unknown_and_double_free_are_rejected():
    run("""
    buf = ctypes.create_string_buffer(128)
    a = lib.b2rt_alloc(64)
    assert lib.b2rt_download(buf, a, 128) < 0       # past the requested size
    assert lib.b2rt_download(buf, 0x1234, 4) < 0    # unknown address
    assert lib.b2rt_free(0x1234) < 0
    assert lib.b2rt_free(a) == 0
    assert lib.b2rt_free(a) < 0                     # double free
    """)


def test_allocation_above_device_maximum_fails():
    run("""
    limit = lib.b2rt_max_alloc()
    assert limit > 0
    assert lib.b2rt_alloc(limit + 1) == 0
    assert lib.b2rt_alloc(0) == 0
    """)


def test_many_small_allocations_share_few_slabs():
    run("""
    before = lib.b2rt_slab_count()
    addrs = [lib.b2rt_alloc(1000 + (i % 7) * 100) for i in range(20000)]
    assert all(addrs)
    assert lib.b2rt_slab_count() - before < 20, lib.b2rt_slab_count()
    assert len(set(addrs)) == len(addrs)
    assert lib.b2rt_live_blocks() == 20000
    for a in addrs:
        assert lib.b2rt_free(a) == 0
    assert lib.b2rt_live_bytes() == 0
    """)


def test_freed_neighbours_coalesce_and_data_is_isolated():
    run("""
    a, b, c = lib.b2rt_alloc(4096), lib.b2rt_alloc(4096), lib.b2rt_alloc(4096)
    da, dc = ctypes.create_string_buffer(b'\\xaa' * 4096, 4096), ctypes.create_string_buffer(b'\\xcc' * 4096, 4096)
    lib.b2rt_upload(a, da, 4096); lib.b2rt_upload(c, dc, 4096)
    lib.b2rt_free(b)
    big = lib.b2rt_alloc(8192)
    lib.b2rt_upload(big, ctypes.create_string_buffer(b'\\x55' * 8192, 8192), 8192)
    ra, rc = ctypes.create_string_buffer(4096), ctypes.create_string_buffer(4096)
    lib.b2rt_download(ra, a, 4096); lib.b2rt_download(rc, c, 4096)
    assert ra.raw == da.raw and rc.raw == dc.raw
    for p in (a, c, big):
        assert lib.b2rt_free(p) == 0
    # the whole slab is one free range again: the first fit starts at the slab base
    all_ = lib.b2rt_alloc(3 * 4096 + 8192)
    assert all_ == a, (hex(all_), hex(a))
    lib.b2rt_free(all_)
    """)


def test_dedicated_slabs_release_and_empty_cache():
    run("""
    big = lib.b2rt_alloc(300 << 20)
    assert big
    reserved = lib.b2rt_reserved_bytes()
    assert reserved >= 300 << 20
    assert lib.b2rt_free(big) == 0
    assert lib.b2rt_reserved_bytes() < reserved
    small = lib.b2rt_alloc(1024)
    lib.b2rt_free(small)
    assert lib.b2rt_empty_cache() >= 1
    assert lib.b2rt_slab_count() == 0
    """)


def test_memory_limit_is_enforced_and_peak_tracked():
    run("""
    lib.b2rt_set_memory_limit(64 << 20)
    lib.b2rt_reset_peak_live_bytes()
    x = lib.b2rt_alloc(4096)
    assert x and lib.b2rt_peak_live_bytes() >= 4096
    assert lib.b2rt_reserved_bytes() <= 64 << 20      # head-room slab, not a full 512 MiB one
    assert lib.b2rt_alloc(256 << 20) == 0             # over the limit
    y = lib.b2rt_alloc(32 << 20)                      # still fits under it
    assert y
    lib.b2rt_free(x); lib.b2rt_free(y)
    lib.b2rt_set_memory_limit(0)
    assert lib.b2rt_alloc(256 << 20) != 0
    """)


def test_retry_after_returning_idle_slabs():
    run("""
    lib.b2rt_set_memory_limit(600 << 20)
    a = lib.b2rt_alloc(1 << 20)          # creates a 512 MiB shared slab
    lib.b2rt_free(a)                     # slab idle but reserved
    big = lib.b2rt_alloc(300 << 20)      # dedicated: 512 + 300 > 600 -> returns the idle slab, retries
    assert big, "allocation should succeed after empty_cache retry"
    assert lib.b2rt_slab_count() == 1
    """)
