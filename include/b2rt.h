/*
 * b2rt.h — C ABI of the B200 hot-path library (libb2rt.so).
 *
 * This header is the drop-in boundary that replaces torch-vulkan's Rust runtime ABI
 * (csrc/vkrt.h:6-32) and the per-kernel push-constant structs its ATen shim fills
 * (csrc/ops_mm.cpp:19-29 MmPush, csrc/ops_quant.cpp:17-21 Dq8Push, csrc/ops_attn.cpp:24-41
 * AttnPush/CoopPush, csrc/ops_rows.cpp:37-42 SoftmaxPush and :103-109 LnPush,
 * csrc/ops_ew.cpp:22-28 EwPush).
 *
 * Conventions (same as vkrt):
 *   - functions returning int: 0 = success, negative = error; the message is kept per thread
 *     and read with b2rt_last_error();
 *   - getters returning sizes/counts return 0 on error;
 *   - device memory is addressed by plain 64-bit device addresses (uint64_t) or void*;
 *   - every launch takes the CUDA stream (cudaStream_t passed as void*) it is ordered on;
 *     nothing in this library synchronises the host except b2rt_synchronize/b2rt_download
 *     and the allocator's dedicated-slab release (as vkrt's free of a dedicated slab, lib.rs:770-777).
 *   - the kernel entry points never allocate tensors: outputs and any workspace are passed in.
 *
 * There are no torch types in any signature; the ATen shim (torch_vulkan_b200/csrc/shim) and
 * ctypes/cffi callers bind these symbols directly.
 */
#ifndef B2RT_H_
#define B2RT_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default) /* exported even when the library builds with -fvisibility=hidden */
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* b2_stream_t; /* a cudaStream_t; NULL = the legacy default stream */

/* Element types. 0..2 follow the reference's shader KIND numbering (vkrt/shaders/types.glsl:1). */
enum b2_dtype {
  B2_F32 = 0,
  B2_BF16 = 1,
  B2_F16 = 2,
  B2_F64 = 3,
  B2_I8 = 4,
};

/* Error codes. */
enum b2_status {
  B2_OK = 0,
  B2_ERR_ARG = -1,       /* invalid argument / unsupported shape or stride */
  B2_ERR_CUDA = -2,      /* a CUDA runtime call failed */
  B2_ERR_OOM = -3,       /* allocation failed (device or emulated limit) */
  B2_ERR_UNKNOWN_PTR = -4,
  B2_ERR_DEVICE = -5,    /* a bounded device-side wait expired; see b2rt_device_error */
};

/* ------------------------------------------------------------------------------------------ */
/* Runtime: init, errors, device info (vkrt.h:8-10)                                            */
/* ------------------------------------------------------------------------------------------ */

/* Replaces vkrt_init (vkrt/src/lib.rs:980-994): selects the current CUDA device, reads its
 * properties (SM count, shared memory) and resolves the driver entry points the TMA kernels need. */
int b2rt_init(void);
/* Replaces vkrt_last_error (lib.rs:1001-1016). Copies the calling thread's last error message
 * (NUL-terminated, truncated to cap) and returns its full length. */
size_t b2rt_last_error(char* buf, size_t cap);
/* Replaces vkrt_device_name (lib.rs:1018-1030). */
size_t b2rt_device_name(char* buf, size_t cap);
/* Number of SMs of the current device (0 before init / without a GPU). */
int b2rt_sm_count(void);
/* Device-side error word written by kernels whose bounded waits expired (0 = none).
 * reset != 0 clears it. Synchronises the device. */
int b2rt_device_error(int reset);
/* Replaces vkrt_validation_errors (vkrt.h:28, lib.rs:1183-1186): the number of launches this
 * library's runtime refused, plus 1 when the device error word is set. It does not synchronise the
 * device: the word is read by a copy on a private stream, so a kernel still in flight may set it
 * after the read (b2rt_device_error waits for everything). */
size_t b2rt_validation_errors(void);
/* Replaces vkrt_coop_caps (vkrt.h:31, lib.rs:1242-1244): bit 0 = f16 and bit 1 = bf16 tensor-core
 * GEMM available (a tcgen05-capable sm_100a device is current); 0 without one. */
uint32_t b2rt_coop_caps(void);

/* ------------------------------------------------------------------------------------------ */
/* Memory: slab sub-allocator (replaces vkrt/src/lib.rs:646-810 and the c10 allocator at       */
/* csrc/shim.cpp:154-171). 512 MiB slabs, 512 B alignment, requests >= 256 MiB get a           */
/* dedicated slab, best fit with coalescing, one retry after returning idle slabs.              */
/* ------------------------------------------------------------------------------------------ */

uint64_t b2rt_max_alloc(void);                      /* vkrt_max_alloc (lib.rs:1032-1036) */
/* vkrt_memory_info (lib.rs:1038-1055): out[0]=budget, out[1]=usage, out[2]=heap size (bytes). */
int32_t b2rt_memory_info(uint64_t* out);
uint64_t b2rt_live_bytes(void);                     /* vkrt_live_bytes (lib.rs:1057-1061) */
uint64_t b2rt_peak_live_bytes(void);                /* vkrt_peak_live_bytes (lib.rs:1063-1067) */
void b2rt_reset_peak_live_bytes(void);              /* vkrt_reset_peak_live_bytes (lib.rs:1069-1073) */
void b2rt_set_memory_limit(uint64_t bytes);         /* vkrt_set_memory_limit (lib.rs:1079-1091); 0 = none */
uint64_t b2rt_alloc(uint64_t size);                 /* vkrt_alloc (lib.rs:1095-1099); 0 on failure */
int b2rt_free(uint64_t addr);                       /* vkrt_free (lib.rs:1101-1107) */
int b2rt_upload(uint64_t dst, const void* src, uint64_t n);   /* vkrt_upload (lib.rs:1126-1138) */
int b2rt_download(void* dst, uint64_t src, uint64_t n);       /* vkrt_download (lib.rs:1140-1149) */
int b2rt_copy_d2d(uint64_t dst, uint64_t src, uint64_t n);    /* vkrt_copy_d2d (lib.rs:1151-1158) */
int b2rt_synchronize(void);                         /* vkrt_synchronize (lib.rs:1177-1179) */
size_t b2rt_empty_cache(void);                      /* vkrt_empty_cache (lib.rs:1189-1193) */
uint64_t b2rt_reserved_bytes(void);                 /* vkrt_reserved_bytes (lib.rs:1195-1199) */
size_t b2rt_live_blocks(void);                      /* vkrt_live_blocks (lib.rs:1201-1205) */
size_t b2rt_slab_count(void);                       /* vkrt_slab_count (lib.rs:1207-1211) */
/* Test hook with no reference counterpart in behaviour: route slab creation to host malloc
 * so the allocator policy can be unit-tested on a machine without a GPU (the reference tests
 * the same policy on a real device, vkrt/tests/basic.rs:14-182). Only valid while no slab exists. */
int b2rt_debug_host_backend(int on);

/* torch.cuda.memory.CUDAPluggableAllocator entry points (same slab allocator, stream-aware:
 * a block freed on stream S is reused on another stream only after that stream waits on S).
 * Each device ordinal has its own slabs: b2_malloc/b2_free use `device`; the b2rt_* memory calls
 * above act on the calling thread's current device, except b2rt_free, b2rt_upload, b2rt_download
 * and b2rt_copy_d2d, which find the device that owns the address. The memory limit applies to
 * every device separately. */
void* b2_malloc(ptrdiff_t size, int device, b2_stream_t stream);
void b2_free(void* ptr, ptrdiff_t size, int device, b2_stream_t stream);

/* ------------------------------------------------------------------------------------------ */
/* Stats and profiling (vkrt_stat lib.rs:1213-1220, vkrt_profile_dump lib.rs:1222-1238,         */
/* kernel counters csrc/shim.cpp:52-67)                                                        */
/* ------------------------------------------------------------------------------------------ */

enum b2_stat_id {
  B2_STAT_LAUNCHES = 0,      /* kernels launched by this library */
  B2_STAT_LAUNCH_NS = 1,     /* host time spent in launch calls */
  B2_STAT_UPLOAD_BYTES = 2,
  B2_STAT_DOWNLOAD_BYTES = 3,
  B2_STAT_ALLOCS = 4,
  B2_STAT_FREES = 5,
  B2_STAT_SYNC_NS = 6,       /* host time blocked in b2rt_synchronize / downloads */
  B2_STAT_CROSS_STREAM_WAITS = 7,
  B2_STAT_COUNT = 8
};
uint64_t b2rt_stat(uint32_t i);
/* Count one call of an ATen-level operator name (the shim calls this, like count_kernel). */
void b2rt_count_op(const char* name);
/* "name\tcount\n" lines for every operator counted so far. Returns the full length. */
size_t b2rt_op_counts(char* buf, size_t cap);
void b2rt_reset_op_counts(void);
/* Per-kernel GPU time (enabled with B2RT_PROFILE=1 or b2rt_profile_enable(1)): each launch is
 * bracketed by CUDA events on its stream (no forced sync); the dump resolves them.
 * Format "name\tms\tcount\n", sorted by time. */
void b2rt_profile_enable(int on);
size_t b2rt_profile_dump(char* buf, size_t cap);
/* Occupies `stream` for `ns` nanoseconds (<= 1 s) with a one-thread spin on the global timer, so a
 * host can enqueue work behind it and have the GPU run that work back to back (measurement aid;
 * no counterpart in the reference). */
int b2rt_gpu_sleep(uint64_t ns, b2_stream_t stream);

/* ------------------------------------------------------------------------------------------ */
/* Kernel entry points                                                                         */
/* ------------------------------------------------------------------------------------------ */

/* C[b] = alpha * A[b] @ B[b] + beta * bias[b]  (bias broadcast through its strides; a stride of
 * 0 broadcasts). Replaces the MmPush dispatch of try_gemm (csrc/ops_mm.cpp:61-175; kernels
 * vkrt/shaders/mm.comp.in:90-155 and mm_coop.comp.in:96-209). A, B, bias and C share dtype
 * (F32, BF16, F16 or F64); accumulation is fp32 (fp64 for F64). All strides are in elements and
 * non-negative. C is written with its own strides. bf16/f16 with TMA-compatible layouts run on the
 * tcgen05 tensor-core kernel; everything else on the strided SIMT kernel. */
typedef struct b2_gemm_args {
  const void* a;
  const void* b;
  void* c;
  const void* bias; /* NULL or has_bias == 0: no bias */
  int64_t M, N, K, batch;
  int64_t a_sb, a_sm, a_sk;
  int64_t b_sb, b_sk, b_sn;
  int64_t c_sb, c_sm, c_sn;
  int64_t bias_sb, bias_sm, bias_sn;
  float alpha, beta;
  int32_t dtype;    /* enum b2_dtype */
  int32_t has_bias;
  int32_t force_simt; /* 1: always use the SIMT kernel (A/B switch, like set_coop_enabled) */
  int32_t pad_;
  /* Optional scratch for split-K (GEMMs with few output tiles and a long K): at least
   * b2_gemm_workspace_bytes(args) bytes, 16-byte aligned. NULL or too small: no split. */
  void* workspace;
  int64_t workspace_bytes;
} b2_gemm_args;
int b2_gemm(const b2_gemm_args* args, b2_stream_t stream);
/* Scratch bytes b2_gemm would use for these arguments (0: none). */
uint64_t b2_gemm_workspace_bytes(const b2_gemm_args* args);
/* Which kernel b2_gemm would pick for these arguments: 0 = SIMT, 1 = tcgen05, 2 = skinny (bf16/f16 with one
 * output dimension <= 64 and a multiple of 8 and K >= 256: mma.sync with the reduction split across the
 * warps of a CTA, one launch and no workspace). */
int b2_gemm_path(const b2_gemm_args* args);

/* Weight-only int8 dequant. Replaces dequant_int8_vk (csrc/ops_quant.cpp:34-59, kernel
 * vkrt/shaders/dq8.comp.in:39-62): out[r,c] = round_to(out_dtype)(float(q[r,c]) * scale(r,c))
 * with one fp32 multiply and one round-to-nearest-even, bit-exact with
 * torch_vulkan/__init__.py:203-205.
 *   scale_layout 0: scale is bf16 [rows, ceil(cols/64)], scale(r,c) = scale[r, c/64]   (reference)
 *   scale_layout 1: scale is fp32 [rows],                 scale(r,c) = scale[r]        (per-row)
 * q is [rows, cols] with row stride q_ld (elements), out is contiguous [rows, cols]. */
typedef struct b2_dequant_args {
  const int8_t* q;
  const void* scale;
  void* out;
  int64_t rows, cols, q_ld;
  int32_t scale_layout;
  int32_t out_dtype; /* F32, BF16 or F16 */
} b2_dequant_args;
int b2_dequant_int8(const b2_dequant_args* args, b2_stream_t stream);

/* Fused int8-weight linear (new; the reference dequantises then calls addmm,
 * tests/test_dequant_int8.py:1-2). The dequantised weight W~[n,k] = bf16(float(q[n,k]) * s(n,k))
 * is produced in shared memory inside the GEMM mainloop, bit-identical to b2_dequant_int8, and
 * never written to HBM.
 *   transpose_w == 0 (forward):  out[M,N] = x[M,K] @ W~^T + bias[N]           (q is [N,K])
 *   transpose_w == 1 (backward): out[M,K] = x[M,N] @ W~      (dX = dY @ W~)   (q is [N,K])
 * x, bias and out are BF16 (row-major, leading dims x_ld/out_ld); scale as b2_dequant_args. */
typedef struct b2_int8_gemm_args {
  const void* x;
  const int8_t* q;
  const void* scale;
  const void* bias; /* NULL: none (forward only) */
  void* out;
  int64_t M;     /* rows of x */
  int64_t N;     /* rows of q (output features) */
  int64_t K;     /* cols of q (input features) */
  int64_t x_ld, out_ld;
  int32_t scale_layout;
  int32_t transpose_w;
  /* optional fp32 scratch of b2_int8_gemm_workspace_bytes() bytes (16-byte aligned) that lets GEMMs
   * with too few output tiles for the GPU split their reduction (partials summed, plus the bias, by a
   * second kernel); NULL or too small: no split */
  void* workspace;
  int64_t workspace_bytes;
  /* Fused activation epilogue of the DiT MLP (new; the reference runs GELU as its own elementwise
   * kernels, csrc/ops_ew.cpp:321-326 and :352). aux is bf16 [M, out_cols] with row stride aux_ld.
   *   0: none.
   *   1 (forward form): out = h = x @ W~^T + bias and aux = gelu_tanh(h) of the bf16-rounded h.
   *   2 (transposed form): out = bf16(dY @ W~) * gelu_tanh'(aux), aux = the forward's h.
   * GELU is the tanh approximation (F.gelu(approximate="tanh")). No split-K with an epilogue. */
  int32_t epilogue;
  int32_t pad_;
  void* aux;
  int64_t aux_ld;
  /* LoRA side path added by the same GEMM as one extra 64-wide reduction block (new; the reference
   * runs it as separate linears, tests/anima_on_vk.py:43-48). lora_r (8..64, a multiple of 8) = 0: none.
   *   forward form:    out += lora_h[M, r] @ lora_b[N, r]^T  (lora_h = x @ A^T, lora_b = B * alpha / r)
   *   transposed form: out += lora_h[M, r] @ lora_b[r, K]    (lora_h = dY @ B * alpha / r, lora_b = A)
   * bf16, rows 16-byte aligned with leading dims lora_h_ld / lora_b_ld (multiples of 8). No split-K. */
  const void* lora_h;
  const void* lora_b;
  int64_t lora_h_ld, lora_b_ld;
  int32_t lora_r;
  int32_t pad2_;
} b2_int8_gemm_args;
int b2_int8_gemm(const b2_int8_gemm_args* args, b2_stream_t stream);
uint64_t b2_int8_gemm_workspace_bytes(const b2_int8_gemm_args* args);

/* Fused scaled-dot-product attention (no mask, no dropout, not causal), D <= 128.
 * Replaces k_sdpa_fwd / k_sdpa_bwd (csrc/ops_attn.cpp:166-295; kernels attn.comp.in and
 * attn_coop.comp.in). Tensors are [B,H,S,D] addressed through (batch, head, seq) strides in
 * elements with unit stride along D. lse and delta are fp32 [B,H,Sq] contiguous.
 * Forward:  O = softmax(scale * Q K^T) V, lse = rowmax + log(rowsum)  (natural log).
 * Backward: delta = rowsum(O * dO); dQ, dK, dV as FlashAttention-2.
 * workspace: fp32 scratch of b2_attn_bwd_workspace_bytes() bytes (dQ accumulator), or NULL
 * for the kernels that need none. */
typedef struct b2_attn_args {
  const void* q;
  const void* k;
  const void* v;
  void* o;          /* forward output / backward input */
  float* lse;
  const void* d_o;  /* backward: upstream gradient */
  void* dq;
  void* dk;
  void* dv;
  float* delta;     /* backward scratch/output [B,H,Sq] fp32 */
  void* workspace;
  int64_t B, H, Sq, Sk, D;
  int64_t q_s[3], k_s[3], v_s[3], o_s[3], do_s[3], dq_s[3], dk_s[3], dv_s[3];
  float scale;
  int32_t dtype;    /* F32, BF16 or F16 (all of q/k/v/o/dO/dQ/dK/dV) */
  int32_t force_simt;
  int32_t pad_;
} b2_attn_args;
int b2_attn_fwd(const b2_attn_args* args, b2_stream_t stream);
int b2_attn_bwd(const b2_attn_args* args, b2_stream_t stream);
uint64_t b2_attn_bwd_workspace_bytes(const b2_attn_args* args);
/* 0 = SIMT path, 1 = tcgen05 path. */
int b2_attn_path(const b2_attn_args* args);

/* Row softmax over the middle axis of a contiguous [outer, R, inner] view.
 * Replaces try_softmax / k_softmax_backward (csrc/ops_rows.cpp:59-100; softmax.comp.in:20-51).
 * fwd:  y = exp(x - max) / sum      (safe != 0: rows that are all -inf give 0, _safe_softmax)
 * bwd:  dx = y * (g - sum(g * y))
 * in_dtype is the dtype of x (fwd) or of y and g (bwd); out_dtype that of y (fwd) / dx (bwd). */
typedef struct b2_softmax_args {
  const void* x;   /* fwd input */
  const void* y;   /* fwd output / bwd input */
  const void* g;   /* bwd upstream gradient */
  void* out;       /* fwd: y, bwd: dx */
  int64_t outer, R, inner;
  int32_t in_dtype, out_dtype;
  int32_t safe;
  int32_t pad_;
} b2_softmax_args;
int b2_softmax_fwd(const b2_softmax_args* args, b2_stream_t stream);
int b2_softmax_bwd(const b2_softmax_args* args, b2_stream_t stream);

/* LayerNorm over the last D elements of a contiguous [rows, D] tensor.
 * Replaces k_native_layer_norm[_backward] (csrc/ops_rows.cpp:117-181; ln.comp.in:25-84).
 * fwd:  y = (x - mean) * rstd * w + b;  mean/rstd fp32 [rows]
 * bwd:  dx = rstd * (gw - mean(gw) - xhat * mean(gw * xhat)), gw = g * w;
 *       dw = sum_rows g * xhat, db = sum_rows g (written when the pointers are non-NULL).
 * workspace: fp32 scratch of b2_layernorm_bwd_workspace_bytes() bytes when dw or db is wanted. */
typedef struct b2_layernorm_args {
  const void* x;
  const void* w;   /* NULL: no affine weight */
  const void* b;   /* NULL: no bias */
  void* y;         /* fwd output */
  float* mean;
  float* rstd;
  const void* g;   /* bwd upstream gradient */
  void* dx;        /* bwd outputs (NULL = not wanted) */
  void* dw;
  void* db;
  void* workspace;
  int64_t rows, D;
  float eps;
  int32_t dtype;   /* of x, y, g, dx, w, b, dw, db */
} b2_layernorm_args;
int b2_layernorm_fwd(const b2_layernorm_args* args, b2_stream_t stream);
int b2_layernorm_bwd(const b2_layernorm_args* args, b2_stream_t stream);
uint64_t b2_layernorm_bwd_workspace_bytes(const b2_layernorm_args* args);
/* LayerNorm backward that allocates nothing (no counterpart in the reference). For callers that
 * cannot allocate device memory mid-step: a host framework that owns all VRAM through its own
 * allocator or a fixed budget, or an FFI caller that only holds the tensors. Same arguments and
 * results as b2_layernorm_bwd except that args->workspace is ignored: the dw/db partial sums go to a
 * 2 MiB scratch array compiled into the library (kept by every GPU that loads it until exit), so
 * D <= 262144 when dw or db is requested; larger D is rejected with B2_ERR_ARG. The first call on a
 * device looks up that array's device address (cudaGetSymbolAddress), so make it before any CUDA
 * graph capture. The address is cached per device for the life of the process and is not valid after
 * cudaDeviceReset (or anything else that destroys the device's primary context): do not call this entry
 * point after such a reset. Every call reuses the same array: calls that can overlap on the GPU (different
 * streams, no ordering between them) race; calls ordered on one stream are safe. Nothing in the
 * array needs to start at zero (every partial is written before it is read). */
int b2_layernorm_bwd_noalloc(const b2_layernorm_args* args, b2_stream_t stream);

/* Optimizer ternaries (csrc/ops_ew.cpp:405-455, expressions tools/gen_shaders.py:83-92):
 *   op 0 addcmul: out = x + value * t1 * t2
 *   op 1 addcdiv: out = x + value * t1 / t2
 *   op 2 lerp:    out = x + value * (t1 - x)   (evaluated as torch does: for value >= 0.5 as
 *                 t1 - (t1 - x) * (1 - value))
 * Broadcasting through strides: every operand is addressed as [ndim] sizes with its own strides
 * (elements, 0 = broadcast), ndim <= 8. fp32 math, one rounding to dtype. out may alias x. */
#define B2_EW_MAX_DIMS 8
typedef struct b2_ew_args {
  void* out;
  const void* x;
  const void* t1;
  const void* t2; /* unused for lerp */
  int64_t sizes[B2_EW_MAX_DIMS];
  int64_t out_s[B2_EW_MAX_DIMS], x_s[B2_EW_MAX_DIMS], t1_s[B2_EW_MAX_DIMS], t2_s[B2_EW_MAX_DIMS];
  int32_t ndim;
  int32_t op;
  int32_t dtype;
  float value;
} b2_ew_args;
int b2_ew_ternary(const b2_ew_args* args, b2_stream_t stream);

/* Multi-tensor AdamW step (the addcmul_/addcdiv_/lerp_ sequence of torch.optim.AdamW with
 * foreach=False, csrc/ops_ew.cpp:432-451 call stack E), applied to n contiguous parameter
 * tensors in one launch. param/grad/exp_avg/exp_avg_sq are arrays of n device pointers. */
typedef struct b2_adamw_args {
  void* const* param;
  const void* const* grad;
  void* const* exp_avg;
  void* const* exp_avg_sq;
  const int64_t* numel;
  int32_t n;
  int32_t dtype;       /* of param/grad/exp_avg/exp_avg_sq: F32 or BF16 */
  float lr, beta1, beta2, eps, weight_decay;
  float bias_correction1, bias_correction2; /* 1 - beta^t */
} b2_adamw_args;
int b2_adamw_step(const b2_adamw_args* args, b2_stream_t stream);

/* Mean squared error between two contiguous tensors of n elements (the training loss of the DiT LoRA step,
 * F.mse_loss(x.float(), t.float()); replaces the fp32 mse_loss the reference's autocast policy routes to,
 * csrc/shim.cpp:414, as its training tests call it, tests/test_ops_ew.py:333), computed from the 16-bit (or fp32) inputs with fp32 arithmetic and a
 * fixed summation order (deterministic):
 *   forward:  *loss = sum((x - t)^2) / n  (fp32), in two launches; `partial` is scratch of
 *             b2_mse_loss_workspace_bytes(n) bytes
 *   backward: grad_x = 2 (x - t) * (*grad_loss) / n, rounded to the dtype of x, in one launch
 * grad_loss and loss are device pointers to fp32 scalars (n = 0 gives a NaN loss, the mean over nothing). dtype: F32, BF16 or F16
 * (x, t, grad_x). */
typedef struct b2_mse_args {
  const void* x;
  const void* t;
  float* loss;
  void* grad_x;
  const float* grad_loss;
  float* partial;
  int64_t n;
  int32_t dtype;
  int32_t pad_;
} b2_mse_args;
int b2_mse_loss_fwd(const b2_mse_args* args, b2_stream_t stream);
int b2_mse_loss_bwd(const b2_mse_args* args, b2_stream_t stream);
uint64_t b2_mse_loss_workspace_bytes(int64_t n);

#ifdef __cplusplus
}
#endif

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif /* B2RT_H_ */
