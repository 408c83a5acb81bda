// Runtime part of libb2rt.so: init, errors, stats, operator counters and per-kernel profiling.
//
// Replaces the Rust runtime's C ABI (vkrt/src/lib.rs:974-1244): last-error string, device name,
// STATS counters (lib.rs:127-132) and the VKRT_PROFILE per-kernel timing (lib.rs:133-138, 942-951).
// Differences by design: CUDA launches are already asynchronous and stream ordered, so there is
// no command-buffer batching to manage (lib.rs:543-643); profiling records CUDA events around each
// launch instead of flushing and waiting after every dispatch.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "b2_internal.h"

namespace b2 {

namespace {
thread_local std::string t_last_error;

std::atomic<uint64_t> g_stats[B2_STAT_COUNT];

std::mutex g_ops_mu;
std::map<std::string, uint64_t> g_op_counts;

std::atomic<int> g_profile{-1};  // -1 = not yet read from the environment
struct ProfRecord {
  const char* name;
  cudaEvent_t a, b;
};
std::mutex g_prof_mu;
std::vector<ProfRecord> g_prof_pending;
std::map<std::string, std::pair<double, uint64_t>> g_prof_done;  // name -> (ms, count)

std::once_flag g_init_once;
DeviceInfo g_dev;
int g_init_rc = 0;
std::string g_init_err;

__device__ int d_error_word;

bool profiling() {
  int p = g_profile.load(std::memory_order_relaxed);
  if (p < 0) {
    const char* e = getenv("B2RT_PROFILE");
    p = (e && e[0] && e[0] != '0') ? 1 : 0;
    g_profile.store(p);
  }
  return p == 1;
}

uint64_t now_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

void resolve_profile_locked() {
  std::vector<ProfRecord> keep;
  for (auto& r : g_prof_pending) {
    if (cudaEventQuery(r.b) == cudaSuccess) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, r.a, r.b);
      auto& slot = g_prof_done[r.name];
      slot.first += ms;
      slot.second += 1;
      cudaEventDestroy(r.a);
      cudaEventDestroy(r.b);
    } else {
      keep.push_back(r);
    }
  }
  (void)cudaGetLastError();  // a not-ready query is not an error
  g_prof_pending.swap(keep);
}
}  // namespace

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int fail_cuda(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  (void)cudaGetLastError();
  return fail(B2_ERR_CUDA, m);
}

const DeviceInfo& device_info() {
  std::call_once(g_init_once, [] {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    int n = 0;
    if (e == cudaSuccess) e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
      g_init_rc = B2_ERR_CUDA;
      g_init_err = std::string("b2rt: no CUDA device (") + cudaGetErrorString(e) + ")";
      (void)cudaGetLastError();
      return;
    }
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, dev);
    g_dev.device = dev;
    g_dev.sm_count = p.multiProcessorCount;
    g_dev.smem_optin = (int)p.sharedMemPerBlockOptin;
    g_dev.cc_major = p.major;
    g_dev.cc_minor = p.minor;
    g_dev.tcgen05 = (p.major == 10 && p.minor == 0);
    g_dev.coop_launch = p.cooperativeLaunch != 0;
  });
  return g_dev;
}

int ensure_init() {
  const DeviceInfo& d = device_info();
  if (d.device < 0) return fail(g_init_rc ? g_init_rc : B2_ERR_CUDA, g_init_err);
  return 0;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("B2_NO_PDL");
    return !(e && *e && *e != '0');
  }();
  return on;
}

LaunchScope::LaunchScope(const char* kernel_name, cudaStream_t s) : name(kernel_name), stream(s) {
  g_stats[B2_STAT_LAUNCHES].fetch_add(1, std::memory_order_relaxed);
  if (profiling()) {
    cudaEventCreate(&ev0);
    cudaEventRecord(ev0, stream);
  }
}

LaunchScope::~LaunchScope() {
  if (ev0) {
    cudaEvent_t ev1;
    cudaEventCreate(&ev1);
    cudaEventRecord(ev1, stream);
    std::lock_guard<std::mutex> g(g_prof_mu);
    g_prof_pending.push_back({name, ev0, ev1});
    if (g_prof_pending.size() > 4096) resolve_profile_locked();
  }
}

std::atomic<uint64_t> g_launch_errors{0};  // launches the runtime refused (b2rt_validation_errors)

int after_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_launch_errors.fetch_add(1, std::memory_order_relaxed);
    return fail_cuda(e, what);
  }
  return 0;
}

int* device_error_ptr() {
  void* p = nullptr;
  cudaGetSymbolAddress(&p, d_error_word);
  return (int*)p;
}

void stat_add(int id, uint64_t v) { g_stats[id].fetch_add(v, std::memory_order_relaxed); }

namespace {
// Spins one thread for `ns` nanoseconds of %globaltimer (bounded by construction).
__global__ void gpu_sleep_kernel(uint64_t ns) {
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  do {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  } while (t - t0 < ns);
}
}  // namespace

}  // namespace b2

using namespace b2;

extern "C" {

int b2rt_init(void) { return ensure_init(); }

size_t b2rt_last_error(char* buf, size_t cap) {
  const std::string& s = t_last_error;
  if (buf && cap) {
    size_t n = std::min(cap - 1, s.size());
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return s.size();
}

size_t b2rt_device_name(char* buf, size_t cap) {
  if (ensure_init()) return 0;
  cudaDeviceProp p;
  cudaGetDeviceProperties(&p, device_info().device);
  size_t len = strlen(p.name);
  if (buf && cap) {
    size_t n = std::min(cap - 1, len);
    memcpy(buf, p.name, n);
    buf[n] = 0;
  }
  return len;
}

int b2rt_sm_count(void) { return device_info().sm_count; }

int b2rt_device_error(int reset) {
  if (ensure_init()) return 0;
  int v = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, d_error_word, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(d_error_word, &z, sizeof(int));
  }
  (void)cudaGetLastError();
  return v;
}

size_t b2rt_validation_errors(void) {
  size_t n = (size_t)g_launch_errors.load(std::memory_order_relaxed);
  if (ensure_init()) return n;
  // read the device error word on a private non-blocking stream: waits for that copy only, not for
  // the work in flight on other streams (a kernel still running may set it later)
  static cudaStream_t s = [] {
    cudaStream_t t = nullptr;
    if (cudaStreamCreateWithFlags(&t, cudaStreamNonBlocking) != cudaSuccess) (void)cudaGetLastError();
    return t;
  }();
  static int* host_word = [] {
    int* h = nullptr;
    if (cudaMallocHost(&h, sizeof(int)) != cudaSuccess) (void)cudaGetLastError();
    return h;
  }();
  if (!s || !host_word) return n;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (cudaMemcpyFromSymbolAsync(host_word, d_error_word, sizeof(int), 0, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
      cudaStreamSynchronize(s) == cudaSuccess)
    n += *host_word != 0 ? 1 : 0;
  (void)cudaGetLastError();
  return n;
}

uint32_t b2rt_coop_caps(void) {
  if (ensure_init()) return 0;
  return device_info().tcgen05 ? 3u : 0u;
}

uint64_t b2rt_stat(uint32_t i) { return i < B2_STAT_COUNT ? g_stats[i].load() : 0; }

void b2rt_count_op(const char* name) {
  std::lock_guard<std::mutex> g(g_ops_mu);
  g_op_counts[name] += 1;
}

size_t b2rt_op_counts(char* buf, size_t cap) {
  std::string s;
  {
    std::lock_guard<std::mutex> g(g_ops_mu);
    for (auto& kv : g_op_counts) s += kv.first + "\t" + std::to_string(kv.second) + "\n";
  }
  if (buf && cap) {
    size_t n = std::min(cap - 1, s.size());
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return s.size();
}

void b2rt_reset_op_counts(void) {
  std::lock_guard<std::mutex> g(g_ops_mu);
  g_op_counts.clear();
}

void b2rt_profile_enable(int on) { g_profile.store(on ? 1 : 0); }

size_t b2rt_profile_dump(char* buf, size_t cap) {
  std::string s;
  {
    std::lock_guard<std::mutex> g(g_prof_mu);
    for (auto& r : g_prof_pending) cudaEventSynchronize(r.b);
    resolve_profile_locked();
    std::vector<std::pair<std::string, std::pair<double, uint64_t>>> rows(g_prof_done.begin(), g_prof_done.end());
    std::sort(rows.begin(), rows.end(), [](auto& a, auto& b) { return a.second.first > b.second.first; });
    char line[512];
    for (auto& r : rows) {
      snprintf(line, sizeof(line), "%s\t%.6f\t%llu\n", r.first.c_str(), r.second.first,
               (unsigned long long)r.second.second);
      s += line;
    }
  }
  if (buf && cap) {
    size_t n = std::min(cap - 1, s.size());
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return s.size();
}

int b2rt_gpu_sleep(uint64_t ns, b2_stream_t stream) {
  if (int rc = ensure_init()) return rc;
  if (ns > 1000000000ull) return fail(B2_ERR_ARG, "gpu_sleep: at most 1 s");
  gpu_sleep_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(ns);
  return after_launch("b2rt_gpu_sleep");
}

int b2rt_synchronize(void) {
  if (ensure_init()) return B2_ERR_CUDA;
  uint64_t t0 = now_ns();
  cudaError_t e = cudaDeviceSynchronize();
  g_stats[B2_STAT_SYNC_NS].fetch_add(now_ns() - t0);
  return check_cuda(e, "b2rt_synchronize");
}

}  // extern "C"
