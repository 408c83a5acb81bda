// Slab sub-allocator of libb2rt.so.
//
// Policy (same as the reference runtime, vkrt/src/lib.rs:31-46 constants, 646-810 logic):
//   * device memory is taken from the driver in slabs of 512 MiB; requests are rounded up to 512 B;
//   * a request >= 256 MiB gets a dedicated slab that goes back to the driver when freed;
//   * best-fit carve among the free ranges of all shared slabs; freed ranges coalesce with their
//     neighbours; empty_cache() returns idle slabs;
//   * an emulated memory limit (set_memory_limit) caps the reserved bytes; when the limit leaves
//     less than a slab but the request fits, a smaller slab is made from the remaining head-room;
//   * when a slab cannot be created, idle slabs are returned and the creation retried once;
//   * downloads/uploads are bounds-checked against the live block that contains them.
// B200-specific differences:
//   * best fit is an O(log n) lookup in a size-ordered index instead of a scan under one lock;
//   * stream awareness for the PyTorch pluggable-allocator entry points: a free range remembers the
//     streams that freed into it; a carve for stream T makes T wait (cudaStreamWaitEvent, no host
//     sync) on each other stream S recorded there, so a block is never reused across streams before
//     the work that used it is ordered ahead;
//   * one allocator per device ordinal (the reference runtime drives a single Vulkan device): slabs,
//     free ranges and statistics never mix devices. b2_malloc/b2_free use their device argument; the
//     b2rt_* calls without one use the calling thread's current CUDA device, and b2rt_free and the
//     copy calls find the device that owns the address.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <tuple>
#include <vector>

#include "b2_internal.h"

namespace b2 {
namespace {

constexpr uint64_t kAlign = 512;
constexpr uint64_t kSlabBytes = 512ull << 20;
constexpr uint64_t kDedicatedMin = 256ull << 20;

struct FreeRange {
  uint64_t len = 0;
  std::vector<cudaStream_t> streams;  // streams whose frees made up this range
};

struct Slab {
  uint64_t size = 0;
  bool dedicated = false;
  uint64_t used = 0;
};

struct Block {
  uint64_t size = 0;  // rounded
  uint64_t req = 0;   // requested
  cudaStream_t stream = nullptr;
};

void merge_streams(std::vector<cudaStream_t>& into, const std::vector<cudaStream_t>& from) {
  for (auto s : from)
    if (std::find(into.begin(), into.end(), s) == into.end()) into.push_back(s);
}

// Makes `dev` current for the lifetime of the guard (no-op when it already is).
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) {
      (void)cudaGetLastError();
      return;
    }
    if (cur != dev && cudaSetDevice(dev) == cudaSuccess) prev = cur;
    (void)cudaGetLastError();
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

class Allocator {
 public:
  explicit Allocator(int dev) : device(dev) {}
  const int device;  // CUDA ordinal whose memory this allocator hands out
  std::mutex mu;
  bool host_backend = false;
  uint64_t mem_limit = 0;
  uint64_t live = 0, peak = 0;
  std::map<uint64_t, Slab> slabs;             // base -> slab
  std::map<uint64_t, FreeRange> free_ranges;  // absolute address -> range (shared slabs only)
  std::set<std::pair<uint64_t, uint64_t>> by_size;  // (len, addr)
  std::map<uint64_t, Block> blocks;           // address -> live block
  std::vector<cudaEvent_t> event_pool;

  uint64_t reserved() const {
    uint64_t r = 0;
    for (auto& kv : slabs) r += kv.second.size;
    return r;
  }

  uint64_t device_total = 0;  // cached total device memory (the largest single allocation)

  uint64_t max_alloc() {
    if (host_backend) return 1ull << 40;
    if (device_total) return device_total;
    if (ensure_init()) return 0;
    DeviceGuard dg(device);
    size_t fr = 0, tot = 0;
    if (cudaMemGetInfo(&fr, &tot) != cudaSuccess) {
      (void)cudaGetLastError();
      return 0;
    }
    device_total = tot;
    return tot;
  }

  // -- raw slab memory ------------------------------------------------------------------------
  int raw_alloc(uint64_t size, uint64_t* base) {
    if (host_backend) {
      void* p = nullptr;
      if (posix_memalign(&p, 4096, size) != 0 || !p) return fail(B2_ERR_OOM, "host backend: out of memory");
      *base = (uint64_t)p;
      return 0;
    }
    if (int rc = ensure_init()) return rc;
    DeviceGuard dg(device);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, size);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(B2_ERR_OOM, std::string("cudaMalloc(") + std::to_string(size) + ") failed: " + cudaGetErrorString(e));
    }
    *base = (uint64_t)p;
    return 0;
  }
  void raw_free(uint64_t base) {
    if (host_backend) {
      free((void*)base);
      return;
    }
    DeviceGuard dg(device);
    cudaFree((void*)base);  // waits for work in flight, like vkrt's flush(true) before destroy
    (void)cudaGetLastError();
  }

  // -- free-range index ----------------------------------------------------------------------
  void add_range(uint64_t addr, FreeRange r) {
    by_size.insert({r.len, addr});
    free_ranges.emplace(addr, std::move(r));
  }
  void drop_range(std::map<uint64_t, FreeRange>::iterator it) {
    by_size.erase({it->second.len, it->first});
    free_ranges.erase(it);
  }

  std::map<uint64_t, Slab>::iterator slab_of(uint64_t addr) {
    auto it = slabs.upper_bound(addr);
    if (it == slabs.begin()) return slabs.end();
    --it;
    if (addr >= it->first + it->second.size) return slabs.end();
    return it;
  }

  int new_slab_checked(uint64_t size, bool dedicated, uint64_t* base) {
    if (mem_limit > 0) {
      uint64_t r = reserved();
      if (r + size > mem_limit)
        return fail(B2_ERR_OOM, "memory limit of " + std::to_string(mem_limit >> 20) + " MiB exceeded (reserved " +
                                    std::to_string(r >> 20) + " MiB + request " + std::to_string(size >> 20) + " MiB)");
    }
    if (int rc = raw_alloc(size, base)) return rc;
    Slab s;
    s.size = size;
    s.dedicated = dedicated;
    slabs.emplace(*base, s);
    if (!dedicated) add_range(*base, FreeRange{size, {}});
    return 0;
  }

  int new_slab_with_retry(uint64_t size, bool dedicated, uint64_t* base) {
    int rc = new_slab_checked(size, dedicated, base);
    if (rc == 0) return 0;
    if (empty_cache_locked() == 0) return rc;
    rc = new_slab_checked(size, dedicated, base);
    if (rc) fail(rc, "slab allocation failed after returning idle slabs (live " + std::to_string(live) + " bytes)");
    return rc;
  }

  // Orders `stream` after every other stream that freed into the range being reused.
  void order_after(const std::vector<cudaStream_t>& from, cudaStream_t stream) {
    if (host_backend) return;
    DeviceGuard dg(device);  // events belong to this allocator's device, like its streams
    for (cudaStream_t s : from) {
      if (s == stream) continue;
      cudaEvent_t ev;
      if (event_pool.empty()) {
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
          (void)cudaGetLastError();
          cudaDeviceSynchronize();
          return;
        }
      } else {
        ev = event_pool.back();
        event_pool.pop_back();
      }
      if (cudaEventRecord(ev, s) != cudaSuccess || cudaStreamWaitEvent(stream, ev, 0) != cudaSuccess) {
        (void)cudaGetLastError();
        DeviceGuard dg(device);
        cudaDeviceSynchronize();  // the freeing stream is gone: fall back to a full barrier
      }
      event_pool.push_back(ev);  // safe to re-record: the wait captured the recorded state
      stat_add(B2_STAT_CROSS_STREAM_WAITS, 1);
    }
  }

  bool carve(uint64_t rounded, cudaStream_t stream, uint64_t* out) {
    auto it = by_size.lower_bound({rounded, 0});
    if (it == by_size.end()) return false;
    uint64_t addr = it->second;
    auto fr = free_ranges.find(addr);
    FreeRange r = fr->second;
    drop_range(fr);
    order_after(r.streams, stream);
    if (r.len > rounded) add_range(addr + rounded, FreeRange{r.len - rounded, r.streams});
    auto sl = slab_of(addr);
    sl->second.used += rounded;
    *out = addr;
    return true;
  }

  int alloc(uint64_t size, cudaStream_t stream, uint64_t* out) {
    if (size == 0) return fail(B2_ERR_ARG, "zero-size allocation");
    uint64_t rounded = (size + kAlign - 1) / kAlign * kAlign;
    uint64_t mx = max_alloc();
    if (rounded > mx)
      return fail(B2_ERR_OOM, "allocation of " + std::to_string(size) + " bytes exceeds the device maximum " + std::to_string(mx));
    uint64_t addr = 0;
    if (rounded >= kDedicatedMin) {
      if (int rc = new_slab_with_retry(rounded, true, &addr)) return rc;
      slabs[addr].used = rounded;
    } else if (!carve(rounded, stream, &addr)) {
      uint64_t slab_bytes = kSlabBytes;
      if (mem_limit > 0) {
        uint64_t r = reserved();
        uint64_t head = mem_limit > r ? mem_limit - r : 0;
        head -= head % 256;
        if (head >= rounded) slab_bytes = std::min(slab_bytes, head);
      }
      uint64_t base;
      if (int rc = new_slab_with_retry(slab_bytes, false, &base)) return rc;
      if (!carve(rounded, stream, &addr)) return fail(B2_ERR_OOM, "allocation failed right after creating a slab");
    }
    blocks[addr] = Block{rounded, size, stream};
    live += rounded;
    peak = std::max(peak, live);
    stat_add(B2_STAT_ALLOCS, 1);
    *out = addr;
    return 0;
  }

  int release(uint64_t addr, cudaStream_t stream, bool use_stream) {
    auto bi = blocks.find(addr);
    if (bi == blocks.end()) return fail(B2_ERR_UNKNOWN_PTR, "free of unknown address");
    Block blk = bi->second;
    blocks.erase(bi);
    auto sl = slab_of(addr);
    if (sl == slabs.end()) return fail(B2_ERR_UNKNOWN_PTR, "free: slab not found");
    sl->second.used -= blk.size;
    live -= blk.size;
    stat_add(B2_STAT_FREES, 1);
    if (sl->second.dedicated) {
      uint64_t base = sl->first;
      slabs.erase(sl);
      raw_free(base);
      return 0;
    }
    FreeRange r{blk.size, {use_stream ? stream : blk.stream}};
    uint64_t start = addr;
    // coalesce with the previous range if it ends here (and is in the same slab)
    auto nx = free_ranges.lower_bound(addr);
    if (nx != free_ranges.begin()) {
      auto pv = std::prev(nx);
      if (pv->first + pv->second.len == addr && pv->first >= sl->first) {
        start = pv->first;
        r.len += pv->second.len;
        merge_streams(r.streams, pv->second.streams);
        drop_range(pv);
      }
    }
    nx = free_ranges.find(addr + blk.size);
    if (nx != free_ranges.end() && addr + blk.size < sl->first + sl->second.size) {
      r.len += nx->second.len;
      merge_streams(r.streams, nx->second.streams);
      drop_range(nx);
    }
    add_range(start, std::move(r));
    return 0;
  }

  size_t empty_cache_locked() {
    if (!host_backend && !slabs.empty()) {
      DeviceGuard dg(device);
      cudaDeviceSynchronize();
      (void)cudaGetLastError();
    }
    std::vector<uint64_t> idle;
    for (auto& kv : slabs)
      if (kv.second.used == 0) idle.push_back(kv.first);
    for (uint64_t b : idle) {
      auto fr = free_ranges.find(b);
      if (fr != free_ranges.end()) drop_range(fr);
      slabs.erase(b);
      raw_free(b);
    }
    return idle.size();
  }

  // true when addr lies inside one of this allocator's live blocks (sets no error)
  bool resolve_quiet(uint64_t addr) const {
    auto it = blocks.upper_bound(addr);
    if (it == blocks.begin()) return false;
    --it;
    return addr >= it->first && addr < it->first + it->second.size;
  }

  // [addr, addr+n) must lie inside one live block's requested size.
  int resolve(uint64_t addr, uint64_t n) {
    auto it = blocks.upper_bound(addr);
    if (it == blocks.begin()) return fail(B2_ERR_UNKNOWN_PTR, "unknown device address");
    --it;
    if (addr < it->first || addr + n > it->first + it->second.req)
      return fail(B2_ERR_ARG, "out-of-range access: " + std::to_string(n) + " bytes at offset " +
                                  std::to_string(addr - it->first) + " of a " + std::to_string(it->second.req) +
                                  "-byte block");
    return 0;
  }
};

constexpr int kMaxDevices = 64;
std::mutex g_devices_mu;
Allocator* g_alloc[kMaxDevices];  // never destroyed: frees may arrive during exit
bool g_host_backend = false;      // test hook: every allocator carves host memory (device 0 only)
uint64_t g_mem_limit = 0;         // emulated per-device limit on reserved bytes (0 = none)

Allocator* A(int dev) {
  if (dev < 0 || dev >= kMaxDevices) {
    fail(B2_ERR_ARG, "allocator: device ordinal " + std::to_string(dev) + " out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> g(g_devices_mu);
  if (!g_alloc[dev]) {
    g_alloc[dev] = new Allocator(dev);
    g_alloc[dev]->host_backend = g_host_backend;
    g_alloc[dev]->mem_limit = g_mem_limit;
  }
  return g_alloc[dev];
}

int current_device() {
  if (g_host_backend) return 0;
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) {
    (void)cudaGetLastError();
    d = 0;
  }
  return d;
}

// The allocator of the calling thread's current device (always valid: ordinals are < kMaxDevices).
Allocator& A() {
  Allocator* a = A(current_device());
  return a ? *a : *A(0);
}

// The allocator holding a live block at `addr` (the current device's first), or nullptr.
Allocator* owner_of(uint64_t addr) {
  Allocator& cur = A();
  {
    std::lock_guard<std::mutex> g(cur.mu);
    if (cur.resolve_quiet(addr)) return &cur;
  }
  for (int d = 0; d < kMaxDevices; ++d) {
    Allocator* a = nullptr;
    {
      std::lock_guard<std::mutex> g(g_devices_mu);
      a = g_alloc[d];
    }
    if (!a || a == &cur) continue;
    std::lock_guard<std::mutex> g(a->mu);
    if (a->resolve_quiet(addr)) return a;
  }
  return nullptr;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

uint64_t b2rt_max_alloc(void) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  return a.max_alloc();
}

int32_t b2rt_memory_info(uint64_t* out) {
  if (!out) return fail(B2_ERR_ARG, "memory_info: null output");
  Allocator& a = A();
  if (a.host_backend) {
    std::lock_guard<std::mutex> g(a.mu);
    out[0] = 1ull << 40;
    out[1] = a.reserved();
    out[2] = 1ull << 40;
    return 0;
  }
  if (int rc = ensure_init()) return rc;
  size_t fr = 0, tot = 0;
  if (int rc = check_cuda(cudaMemGetInfo(&fr, &tot), "cudaMemGetInfo")) return rc;
  out[0] = tot;       // budget: the whole device is usable by this process
  out[1] = tot - fr;  // usage as the driver sees it (all processes)
  out[2] = tot;       // heap size
  return 0;
}

uint64_t b2rt_live_bytes(void) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  return a.live;
}
uint64_t b2rt_peak_live_bytes(void) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  return a.peak;
}
void b2rt_reset_peak_live_bytes(void) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  a.peak = a.live;
}
// The limit applies to each device's reserved bytes (every device, including ones not used yet).
void b2rt_set_memory_limit(uint64_t bytes) {
  {
    std::lock_guard<std::mutex> g(g_devices_mu);
    g_mem_limit = bytes;
  }
  for (int d = 0; d < kMaxDevices; ++d) {
    Allocator* a = nullptr;
    {
      std::lock_guard<std::mutex> g(g_devices_mu);
      a = g_alloc[d];
    }
    if (!a) continue;
    std::lock_guard<std::mutex> g(a->mu);
    a->mem_limit = bytes;
  }
}

uint64_t b2rt_alloc(uint64_t size) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  uint64_t addr = 0;
  return a.alloc(size, nullptr, &addr) == 0 ? addr : 0;
}

int b2rt_free(uint64_t addr) {
  Allocator* a = owner_of(addr);
  if (!a) return fail(B2_ERR_UNKNOWN_PTR, "free of unknown address");
  std::lock_guard<std::mutex> g(a->mu);
  return a->release(addr, nullptr, false);
}

int b2rt_upload(uint64_t dst, const void* src, uint64_t n) {
  Allocator* a = owner_of(dst);
  if (!a) return fail(B2_ERR_UNKNOWN_PTR, "unknown device address");
  {
    std::lock_guard<std::mutex> g(a->mu);
    if (int rc = a->resolve(dst, n)) return rc;
  }
  stat_add(B2_STAT_UPLOAD_BYTES, n);
  if (a->host_backend) {
    memcpy((void*)dst, src, n);
    return 0;
  }
  return check_cuda(cudaMemcpy((void*)dst, src, n, cudaMemcpyHostToDevice), "b2rt_upload");
}

int b2rt_download(void* dst, uint64_t src, uint64_t n) {
  Allocator* a = owner_of(src);
  if (!a) return fail(B2_ERR_UNKNOWN_PTR, "unknown device address");
  {
    std::lock_guard<std::mutex> g(a->mu);
    if (int rc = a->resolve(src, n)) return rc;
  }
  stat_add(B2_STAT_DOWNLOAD_BYTES, n);
  if (a->host_backend) {
    memcpy(dst, (const void*)src, n);
    return 0;
  }
  return check_cuda(cudaMemcpy(dst, (const void*)src, n, cudaMemcpyDeviceToHost), "b2rt_download");
}

int b2rt_copy_d2d(uint64_t dst, uint64_t src, uint64_t n) {
  Allocator* ad = owner_of(dst);
  Allocator* as = owner_of(src);
  if (!ad || !as) return fail(B2_ERR_UNKNOWN_PTR, "unknown device address");
  {
    std::lock_guard<std::mutex> g(ad->mu);
    if (int rc = ad->resolve(dst, n)) return rc;
  }
  {
    std::lock_guard<std::mutex> g(as->mu);
    if (int rc = as->resolve(src, n)) return rc;
  }
  if (ad->host_backend) {
    memmove((void*)dst, (const void*)src, n);
    return 0;
  }
  return check_cuda(cudaMemcpyAsync((void*)dst, (const void*)src, n, cudaMemcpyDeviceToDevice, nullptr),
                    "b2rt_copy_d2d");
}

size_t b2rt_empty_cache(void) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  return a.empty_cache_locked();
}

uint64_t b2rt_reserved_bytes(void) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  return a.reserved();
}

size_t b2rt_live_blocks(void) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  return a.blocks.size();
}

size_t b2rt_slab_count(void) {
  Allocator& a = A();
  std::lock_guard<std::mutex> g(a.mu);
  return a.slabs.size();
}

int b2rt_debug_host_backend(int on) {
  std::lock_guard<std::mutex> g(g_devices_mu);
  for (int d = 0; d < kMaxDevices; ++d)
    if (g_alloc[d] && !g_alloc[d]->slabs.empty()) return fail(B2_ERR_ARG, "debug_host_backend: slabs already exist");
  g_host_backend = on != 0;
  for (int d = 0; d < kMaxDevices; ++d)
    if (g_alloc[d]) g_alloc[d]->host_backend = g_host_backend;
  return 0;
}

void* b2_malloc(ptrdiff_t size, int device, b2_stream_t stream) {
  if (size <= 0) return nullptr;
  Allocator* a = A(g_host_backend ? 0 : device);
  if (!a) return nullptr;
  std::lock_guard<std::mutex> g(a->mu);
  uint64_t addr = 0;
  if (a->alloc((uint64_t)size, (cudaStream_t)stream, &addr)) return nullptr;
  return (void*)addr;
}

void b2_free(void* ptr, ptrdiff_t size, int device, b2_stream_t stream) {
  (void)size;
  if (!ptr) return;
  Allocator* a = A(g_host_backend ? 0 : device);
  if (!a) return;
  std::lock_guard<std::mutex> g(a->mu);
  a->release((uint64_t)ptr, (cudaStream_t)stream, true);
}

}  // extern "C"
