"""torch_vulkan_b200 — B200-native hot path of torch-vulkan, as a drop-in for CUDA tensors.

Importing this package loads two native libraries built for sm_100a (see ``_build.py``):

* ``libb2rt.so`` — the C ABI (``include/b2rt.h``): slab allocator, stream/launch layer, stats, and
  every kernel (tcgen05 GEMM and int8-dequant GEMM, fused attention, softmax/LayerNorm row kernels,
  optimizer ternaries);
* ``_b2ops.so`` — the ATen shim that registers ``mm/bmm/addmm/baddbmm``, the SDPA
  ``_fused_attention_overrideable`` pair, ``_softmax``/``_safe_softmax``/``_softmax_backward_data``,
  ``native_layer_norm[_backward]`` and ``addcmul(_)/addcdiv(_)/lerp(_).Scalar`` for the CUDA key.

The public functions mirror the reference package ``torch_vulkan/__init__.py`` (memory API 58-111,
stats 155-213, ``dequant_int8`` 193-205, ``set_fused_attention`` 84-87, ``set_coop_enabled`` 253-266)
with CUDA devices in place of the "vk" device. There is no CPU fallback: if the native libraries are
missing the import fails.
"""

from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libb2rt.so")
_OPS_PATH = os.path.join(_HERE, "_b2ops.so")


def _load():
    missing = [p for p in (_LIB_PATH, _OPS_PATH) if not os.path.exists(p)]
    if missing:
        raise ImportError(
            "torch_vulkan_b200: native libraries not built (missing: %s); run "
            "`python -c 'import __graft_entry__ as g; g.build()'` or `python torch_vulkan_b200/_build.py`"
            % ", ".join(os.path.basename(m) for m in missing)
        )
    lib = ctypes.CDLL(_LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    torch.ops.load_library(_OPS_PATH)
    return lib


_lib = _load()
_u64 = ctypes.c_uint64
_lib.b2rt_live_bytes.restype = _u64
_lib.b2rt_peak_live_bytes.restype = _u64
_lib.b2rt_reserved_bytes.restype = _u64
_lib.b2rt_max_alloc.restype = _u64
_lib.b2rt_stat.restype = _u64
_lib.b2rt_stat.argtypes = [ctypes.c_uint32]
_lib.b2rt_set_memory_limit.argtypes = [_u64]
_lib.b2rt_alloc.restype = _u64
_lib.b2rt_alloc.argtypes = [_u64]
_lib.b2rt_free.argtypes = [_u64]
_lib.b2rt_empty_cache.restype = ctypes.c_size_t
_lib.b2rt_live_blocks.restype = ctypes.c_size_t
_lib.b2rt_slab_count.restype = ctypes.c_size_t
_lib.b2rt_op_counts.restype = ctypes.c_size_t
_lib.b2rt_profile_dump.restype = ctypes.c_size_t
_lib.b2rt_last_error.restype = ctypes.c_size_t
_lib.b2rt_device_name.restype = ctypes.c_size_t
_lib.b2rt_validation_errors.restype = ctypes.c_size_t
_lib.b2rt_coop_caps.restype = ctypes.c_uint32

_STAT_NAMES = ["launches", "launch_ns", "upload_bytes", "download_bytes", "allocs", "frees", "sync_ns",
               "cross_stream_waits"]


def _text(fn) -> str:
    n = fn(None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    fn(buf, n + 1)
    return buf.value.decode()


def last_error() -> str:
    return _text(_lib.b2rt_last_error)


# ---- enable / disable the operator overrides ---------------------------------------------------

def enable(on: bool = True) -> None:
    """Register (or remove) the hot-path kernels for CUDA tensors. Removing restores PyTorch's own CUDA
    kernels, which makes A/B comparisons possible in one process."""
    torch.ops.b2.set_enabled(bool(on))


def is_enabled() -> bool:
    return bool(torch.ops.b2.is_enabled())


# ---- device API (torch_vulkan/__init__.py:34-56) -----------------------------------------------

def is_available() -> bool:
    return torch.cuda.is_available()


def device_count() -> int:
    return torch.cuda.device_count()


def current_device() -> int:
    return torch.cuda.current_device()


def synchronize(device=None) -> None:
    torch.cuda.synchronize(device)


def device_name() -> str:
    return _text(_lib.b2rt_device_name)


# ---- memory API (torch_vulkan/__init__.py:58-111) ----------------------------------------------
# These report the slab allocator of libb2rt (used by b2rt_alloc and, after use_slab_allocator(),
# by every CUDA tensor).

def live_bytes() -> int:
    return int(_lib.b2rt_live_bytes())


def memory_info() -> dict:
    out = (_u64 * 3)()
    rc = _lib.b2rt_memory_info(out)
    if rc != 0:
        raise RuntimeError("memory_info: " + last_error())
    return {"budget": int(out[0]), "usage": int(out[1]), "heap": int(out[2])}


def peak_live_bytes() -> int:
    return int(_lib.b2rt_peak_live_bytes())


def reset_peak_live_bytes() -> None:
    _lib.b2rt_reset_peak_live_bytes()


def set_memory_limit(megabytes: int) -> None:
    """Cap the slab allocator's reserved bytes (MiB, 0 = none) to emulate a smaller GPU."""
    _lib.b2rt_set_memory_limit(int(megabytes) << 20)


def empty_cache() -> None:
    _lib.b2rt_empty_cache()


def reserved_bytes() -> int:
    return int(_lib.b2rt_reserved_bytes())


def live_blocks() -> int:
    return int(_lib.b2rt_live_blocks())


def slab_count() -> int:
    return int(_lib.b2rt_slab_count())


_slab_installed = False


def use_slab_allocator() -> None:
    """Route every CUDA tensor allocation through the slab allocator (b2_malloc / b2_free), the
    counterpart of the reference's c10::Allocator over vkrt (csrc/shim.cpp:154-171). Must run before
    the first CUDA allocation of the process."""
    global _slab_installed
    if _slab_installed:
        return
    alloc = torch.cuda.memory.CUDAPluggableAllocator(_LIB_PATH, "b2_malloc", "b2_free")
    torch.cuda.memory.change_current_allocator(alloc)
    _slab_installed = True


# ---- stats (torch_vulkan/__init__.py:155-213) --------------------------------------------------

def stats() -> dict:
    return {name: int(_lib.b2rt_stat(i)) for i, name in enumerate(_STAT_NAMES)}


def _counts() -> dict:
    out = {}
    for line in _text(_lib.b2rt_op_counts).splitlines():
        if line:
            k, v = line.rsplit("\t", 1)
            out[k] = int(v)
    return out


def kernel_counts() -> dict:
    """Operator name -> number of calls served by this library's kernels."""
    return {k: v for k, v in _counts().items() if not k.startswith("fallback:")}


def fallback_counts() -> dict:
    """Operator name -> number of calls that took PyTorch's stock CUDA path (uncovered dtypes)."""
    return {k[len("fallback:"):]: v for k, v in _counts().items() if k.startswith("fallback:")}


def reset_fallback_counts() -> None:
    _lib.b2rt_reset_op_counts()


reset_counts = reset_fallback_counts


def validation_errors() -> int:
    """Device-side error word (bounded waits that expired); 0 when every kernel completed normally.
    The counterpart of the reference's Vulkan validation-error counter."""
    return int(_lib.b2rt_device_error(0))


def profile_enable(on: bool = True) -> None:
    _lib.b2rt_profile_enable(1 if on else 0)


def gpu_sleep(ns: int, stream=None) -> None:
    """Occupy the (current) CUDA stream for `ns` nanoseconds (<= 1 s); work enqueued behind it then runs
    back to back without host launch gaps."""
    s = stream if stream is not None else torch.cuda.current_stream()
    rc = _lib.b2rt_gpu_sleep(ctypes.c_uint64(int(ns)), ctypes.c_void_p(s.cuda_stream))
    if rc != 0:
        raise RuntimeError("gpu_sleep: " + last_error())


def profile() -> str:
    """'name\\tms\\tcount' lines of per-kernel GPU time (after profile_enable or B2RT_PROFILE=1)."""
    return _text(_lib.b2rt_profile_dump)


# ---- kernel switches (torch_vulkan/__init__.py:84-87, 253-266) -----------------------------------

def set_fused_attention(mode: str) -> None:
    """Fused attention policy: "auto" (default), "on" or "off" (env B2_FUSED_ATTN=0/1)."""
    torch.ops.b2.set_fused_attention({"off": 0, "on": 1, "auto": 2}[mode])


_force = 0


def set_coop_enabled(on: bool) -> None:
    """True (default): bf16/f16 GEMMs use the tcgen05 tensor-core kernel; False: the strided SIMT
    kernel (the reference's coop/tiled switch, used to A/B kernels)."""
    global _force
    _force = (_force & ~1) | (0 if on else 1)
    torch.ops.b2.set_force_simt(_force)


def set_tc_attention_enabled(on: bool) -> None:
    """True (default): eligible attention uses the tcgen05 kernels; False: the SIMT kernels."""
    global _force
    _force = (_force & ~2) | (0 if on else 2)
    torch.ops.b2.set_force_simt(_force)


def coop_caps() -> int:
    """bit0 = f16, bit1 = bf16 tensor-core GEMM available (a tcgen05-capable sm_100a device is current)."""
    return int(_lib.b2rt_coop_caps()) if torch.cuda.is_available() else 0


def gemm_path(a: torch.Tensor, b: torch.Tensor) -> str:
    """Which kernel serves mm(a, b): "tcgen05", "skinny" (one output dimension <= 64, mma.sync with the
    K loop split across warps) or "simt"."""
    return {1: "tcgen05", 2: "skinny"}.get(int(torch.ops.b2.gemm_path(a, b)), "simt")


# ---- int8 weight-only quantisation ---------------------------------------------------------------

def dequant_int8(q: torch.Tensor, scale: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """out[r, c] = float(q[r, c]) * float(scale) rounded to out_dtype (round-to-nearest-even).

    scale is bf16 [rows, ceil(cols/64)] (one scale per 64-column block, the reference layout of
    torch_vulkan/__init__.py:193-205) or fp32 [rows] (per output row). CUDA tensors only."""
    if not q.is_cuda:
        raise RuntimeError("dequant_int8: q must be a CUDA tensor (this package has no CPU path)")
    return torch.ops.b2.dequant_int8(q, scale, out_dtype)


class _Int8Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, q, scale, bias):
        ctx.save_for_backward(q, scale)
        ctx.has_bias = bias is not None
        return torch.ops.b2.int8_linear_fwd(x, q, scale, bias)

    @staticmethod
    def backward(ctx, gy):
        q, scale = ctx.saved_tensors
        gx = torch.ops.b2.int8_linear_dx(gy.contiguous(), q, scale) if ctx.needs_input_grad[0] else None
        gb = gy.reshape(-1, gy.shape[-1]).sum(0) if (ctx.has_bias and ctx.needs_input_grad[3]) else None
        return gx, None, None, gb


def int8_linear(x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None = None):
    """y = x @ (q * scale)^T + bias with the dequantisation fused into the tcgen05 GEMM mainloop.
    Differentiable in x (and bias); q/scale are frozen. x bf16 [..., K], q int8 [N, K]."""
    return _Int8Linear.apply(x, q, scale, bias)


class _Int8LoRA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, q, scale, bias, a, b):
        x2 = x.reshape(-1, x.shape[-1])
        h = torch.mm(x2, a.t())  # the rank-r down-projection
        y = torch.ops.b2.int8_lora_fwd(x2, q, scale, bias, h, b)  # base + bias + h b^T in one GEMM
        ctx.save_for_backward(x2, q, scale, a, b, h)
        ctx.x_shape = x.shape
        ctx.has_bias = bias is not None
        return y.view(*x.shape[:-1], q.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, q, scale, a, b, h = ctx.saved_tensors
        gy2 = gy.reshape(-1, gy.shape[-1]).contiguous()
        dh = torch.mm(gy2, b)  # [rows, r]
        gx = None
        if ctx.needs_input_grad[0]:  # dy @ W~ + dh @ A in one GEMM
            gx = torch.ops.b2.int8_lora_dx(gy2, q, scale, dh, a).view(ctx.x_shape)
        ga = torch.mm(dh.t(), x2) if ctx.needs_input_grad[4] else None
        gb = torch.mm(gy2.t(), h) if ctx.needs_input_grad[5] else None
        gbias = gy2.sum(0) if (ctx.has_bias and ctx.needs_input_grad[3]) else None
        return gx, None, None, gbias, ga, gb


def int8_lora_linear(x, q, scale, bias, a, b):
    """y = x @ (q * scale)^T + bias + (x @ a^T) @ b^T — a frozen int8 linear with its LoRA side path, where
    a [r, K] is the down-projection and b [N, r] the up-projection already multiplied by alpha / r (r a
    multiple of 8, at most 64; stacked modules pass their concatenated down-projections and block-diagonal
    up-projections). The up-projection is one more 64-wide reduction block of the int8 GEMM, and in the
    backward dX = dY @ W~ + (dY @ b) @ a is one GEMM too. Differentiable in x, a, b (and bias)."""
    return _Int8LoRA.apply(x, q, scale, bias, a, b)


class _MseLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, t):
        ctx.save_for_backward(x, t)
        return torch.ops.b2.mse_loss_fwd(x, t)

    @staticmethod
    def backward(ctx, g):
        x, t = ctx.saved_tensors
        gx = torch.ops.b2.mse_loss_bwd(g, x, t) if ctx.needs_input_grad[0] else None
        gt = (-torch.ops.b2.mse_loss_bwd(g, x, t)) if ctx.needs_input_grad[1] else None
        return gx, gt


def mse_loss(x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
    """F.mse_loss(x.float(), t.float()) (mean reduction, fp32 result) computed from x and t in their own
    16-bit dtype: two launches forward, one backward, no fp32 copies, a fixed summation order. The
    gradient is returned in x's dtype."""
    return _MseLoss.apply(x, t)


class _Int8GeluMLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, q1, s1, b1, q2, s2, b2):
        act, h = torch.ops.b2.int8_linear_gelu_fwd(x, q1, s1, b1)  # one GEMM: h and gelu(h)
        y = torch.ops.b2.int8_linear_fwd(act, q2, s2, b2)
        ctx.save_for_backward(q1, s1, q2, s2, h)
        ctx.bias_grad = (b1 is not None and ctx.needs_input_grad[3], b2 is not None and ctx.needs_input_grad[6])
        return y

    @staticmethod
    def backward(ctx, gy):
        q1, s1, q2, s2, h = ctx.saved_tensors
        gy = gy.contiguous()
        dh = torch.ops.b2.int8_linear_dx_gelu(gy, q2, s2, h)  # one GEMM: (gy @ W2) * gelu'(h)
        gx = torch.ops.b2.int8_linear_dx(dh, q1, s1) if ctx.needs_input_grad[0] else None
        gb1 = dh.reshape(-1, dh.shape[-1]).sum(0) if ctx.bias_grad[0] else None
        gb2 = gy.reshape(-1, gy.shape[-1]).sum(0) if ctx.bias_grad[1] else None
        return gx, None, None, gb1, None, None, gb2


def int8_mlp(x, q1, s1, b1, q2, s2, b2):
    """fc2(gelu_tanh(fc1(x))) over frozen int8 weights (the DiT block's MLP), with the GELU fused into
    the GEMM epilogues: fc1's epilogue writes the pre-activation h and gelu(h), and in the backward fc2's
    dX epilogue multiplies by gelu'(h). No separate GELU kernels and no extra pass over the
    [tokens, mlp] activation. Differentiable in x (and the biases)."""
    return _Int8GeluMLP.apply(x, q1, s1, b1, q2, s2, b2)


if os.environ.get("B2_DISABLE", "0") in ("", "0"):
    enable(True)

if os.environ.get("B2_MEM_LIMIT_MB"):
    set_memory_limit(int(os.environ["B2_MEM_LIMIT_MB"]))
