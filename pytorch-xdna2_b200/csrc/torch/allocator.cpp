// Stream-ordered HBM caching allocator behind `xdna` storage.
//
// Replaces the reference's XRT buffer-object cache (XdnaBoCache, XdnaAllocator,
// torch_xdna_device.cpp:205-296, 658-716): host-visible BOs with coherency
// states become plain device memory, and the size-binned free list becomes a
// per-(device, stream) best-fit cache.  A block freed on the stream that
// allocated it is reusable on that stream at once (stream order makes it
// safe); a block also used on other streams (record_stream) waits for events
// recorded on those streams before it returns to the cache.  The cache budget
// is XDNA_BO_CACHE_MB (0 or unset: unlimited); on an out-of-memory the cache is
// released and the allocation retried once.
//
// CUDA graph capture (xdna_train.graphs): while a stream captures, its
// allocations come from a private pool of that capture (device memory
// allocated under the relaxed capture mode on a miss); a pool block freed
// during or after the capture returns to its pool only, because replays of
// the graph write it; blocks of the ordinary cache freed during a capture are
// held back until the capture ends; no event is queried while a capture runs.
// Releasing the pool (the graph is gone) hands its blocks to the ordinary
// cache.
#include <c10/cuda/CUDAFunctions.h>

#include <cstdlib>
#include <unordered_map>
#include <vector>

#include "xdna.h"

namespace xdna {
namespace {

struct Block {
  void* ptr = nullptr;
  size_t size = 0;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::vector<cudaStream_t> used_on;  // other streams that touched the block
  int pool = 0;                       // graph pool id, 0: the ordinary cache
};

struct GraphPool {
  int device = 0;
  std::multimap<size_t, Block*> free;
  int64_t live = 0;
  size_t bytes = 0;
  bool released = false;
};

struct PendingFree {
  Block* block;
  std::vector<cudaEvent_t> events;
};

size_t round_size(size_t n) {
  if (n < (1u << 20)) return ((n + 511) / 512) * 512;       // 512 B granules below 1 MiB
  return ((n + (2u << 20) - 1) / (2u << 20)) * (2u << 20);   // 2 MiB granules above
}

class Cache {
 public:
  void* malloc(size_t n, int dev, cudaStream_t st) {
    const size_t sz = round_size(n);
    std::lock_guard<std::mutex> lk(mu_);
    if (capturing_ > 0) {
      auto cp = capture_pool_.find(st);
      if (cp != capture_pool_.end()) return pool_malloc(cp->second, sz, n, dev, st);
    } else {
      poll_pending();
    }
    auto& fl = free_[key(dev, st)];
    auto it = fl.lower_bound(sz);
    // best fit, but do not hand out a block more than twice the request
    if (it != fl.end() && it->first <= 2 * sz + (4u << 20)) {
      Block* b = it->second;
      fl.erase(it);
      cached_bytes_ -= b->size;
      live_[b->ptr] = b;
      allocated_bytes_ += b->size;
      peak_allocated_ = std::max(peak_allocated_, allocated_bytes_);
      ++cache_hits_;
      ++num_allocs_;
      return b->ptr;
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, sz);
    if (e != cudaSuccess && capturing_ == 0) {  // cudaFree synchronizes: not while capturing
      (void)cudaGetLastError();
      release_cached_locked();
      e = cudaMalloc(&p, sz);
      if (e != cudaSuccess) {
        (void)cudaGetLastError();
        TORCH_CHECK_WITH(OutOfMemoryError, false, "xdna: out of device memory allocating ", n,
                         " bytes on xdna:", dev, " (", allocated_bytes_, " bytes in use)");
      }
    }
    Block* b = new Block{p, sz, dev, st, {}};
    live_[p] = b;
    reserved_bytes_ += sz;
    allocated_bytes_ += sz;
    peak_allocated_ = std::max(peak_allocated_, allocated_bytes_);
    peak_reserved_ = std::max(peak_reserved_, reserved_bytes_);
    ++num_allocs_;
    ++device_mallocs_;
    return p;
  }

  void free(void* p) {
    if (!p) return;
    on_release(p);
    std::lock_guard<std::mutex> lk(mu_);
    auto it = live_.find(p);
    if (it == live_.end()) return;
    Block* b = it->second;
    live_.erase(it);
    allocated_bytes_ -= b->size;
    ++num_frees_;
    if (b->pool != 0) {  // graph memory: back to its pool (replays write it)
      GraphPool& gp = pools_[b->pool];
      --gp.live;
      b->used_on.clear();
      if (!gp.released) {
        gp.free.emplace(b->size, b);
        return;
      }
      gp.bytes -= b->size;
      if (gp.live == 0) pools_.erase(b->pool);
      b->pool = 0;
      to_cache(b);
      return;
    }
    if (capturing_ > 0) {  // ordinary memory freed while a capture runs
      b->used_on.clear();
      held_.push_back(b);
      return;
    }
    if (b->used_on.empty()) {
      to_cache(b);
      return;
    }
    PendingFree pf{b, {}};
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != b->device) cudaSetDevice(b->device);
    for (cudaStream_t s : b->used_on) {
      cudaEvent_t ev;
      if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess) {
        cudaEventRecord(ev, s);
        pf.events.push_back(ev);
      }
    }
    if (prev != b->device) cudaSetDevice(prev);
    b->used_on.clear();
    pending_.push_back(std::move(pf));
  }

  int capture_begin(int dev, cudaStream_t st, int share) {
    std::lock_guard<std::mutex> lk(mu_);
    int pid = share;
    if (pid == 0 || !pools_.count(pid) || pools_[pid].released) {
      pid = next_pool_++;
      pools_[pid].device = dev;
    }
    capture_pool_[st] = pid;
    ++capturing_;
    return pid;
  }

  void capture_end(cudaStream_t st) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!capture_pool_.erase(st)) return;
    if (--capturing_ == 0) {
      for (Block* b : held_) to_cache(b);
      held_.clear();
    }
  }

  void release_pool(int pid) {
    std::lock_guard<std::mutex> lk(mu_);
    auto it = pools_.find(pid);
    if (it == pools_.end() || it->second.released) return;
    for (const auto& kv : capture_pool_)
      if (kv.second == pid) return;  // still capturing into it
    GraphPool& gp = it->second;
    gp.released = true;
    for (auto& e : gp.free) {
      gp.bytes -= e.second->size;
      e.second->pool = 0;
      to_cache(e.second);
    }
    gp.free.clear();
    if (gp.live == 0) pools_.erase(it);
  }

  void record(void* p, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(mu_);
    auto it = live_.find(p);
    if (it == live_.end()) return;
    Block* b = it->second;
    if (s == b->stream) return;
    for (cudaStream_t u : b->used_on)
      if (u == s) return;
    b->used_on.push_back(s);
  }

  void empty() {
    std::lock_guard<std::mutex> lk(mu_);
    if (capturing_ > 0) return;  // it synchronizes: not while a capture runs
    // wait for cross-stream frees, then return everything cached
    for (auto& pf : pending_) {
      for (cudaEvent_t ev : pf.events) {
        cudaEventSynchronize(ev);
        cudaEventDestroy(ev);
      }
      to_cache(pf.block);
    }
    pending_.clear();
    release_cached_locked();
  }

  std::map<std::string, int64_t> stats() {
    std::lock_guard<std::mutex> lk(mu_);
    return {{"allocated_bytes", int64_t(allocated_bytes_)},
            {"peak_allocated_bytes", int64_t(peak_allocated_)},
            {"reserved_bytes", int64_t(reserved_bytes_)},
            {"peak_reserved_bytes", int64_t(peak_reserved_)},
            {"cached_bytes", int64_t(cached_bytes_)},
            {"num_allocs", int64_t(num_allocs_)},
            {"num_frees", int64_t(num_frees_)},
            {"cache_hits", int64_t(cache_hits_)},
            {"device_mallocs", int64_t(device_mallocs_)},
            {"pending_cross_stream_frees", int64_t(pending_.size())},
            {"live_blocks", int64_t(live_.size())},
            {"graph_pools", int64_t(pools_.size())},
            {"graph_pool_bytes", int64_t(pool_bytes())}};
  }

 private:
  void* pool_malloc(int pid, size_t sz, size_t n, int dev, cudaStream_t st) {
    GraphPool& gp = pools_[pid];
    auto it = gp.free.lower_bound(sz);
    if (it != gp.free.end() && it->first <= 2 * sz + (4u << 20)) {
      Block* b = it->second;
      gp.free.erase(it);
      ++gp.live;
      live_[b->ptr] = b;
      allocated_bytes_ += b->size;
      peak_allocated_ = std::max(peak_allocated_, allocated_bytes_);
      ++cache_hits_;
      ++num_allocs_;
      return b->ptr;
    }
    // device memory while capturing: allowed under the relaxed capture mode
    void* p = nullptr;
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    cudaError_t e = cudaMalloc(&p, sz);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      TORCH_CHECK_WITH(OutOfMemoryError, false, "xdna: out of device memory allocating ", n,
                       " bytes for a CUDA graph capture on xdna:", dev);
    }
    Block* b = new Block{p, sz, dev, st, {}, pid};
    ++gp.live;
    gp.bytes += sz;
    live_[p] = b;
    reserved_bytes_ += sz;
    allocated_bytes_ += sz;
    peak_allocated_ = std::max(peak_allocated_, allocated_bytes_);
    peak_reserved_ = std::max(peak_reserved_, reserved_bytes_);
    ++num_allocs_;
    ++device_mallocs_;
    return p;
  }

  size_t pool_bytes() const {
    size_t t = 0;
    for (const auto& kv : pools_) t += kv.second.bytes;
    return t;
  }

  static uint64_t key(int dev, cudaStream_t s) {
    return (uint64_t(reinterpret_cast<uintptr_t>(s)) << 8) ^ uint64_t(dev);
  }

  void to_cache(Block* b) {
    free_[key(b->device, b->stream)].emplace(b->size, b);
    cached_bytes_ += b->size;
    const size_t budget = budget_bytes();
    if (budget && cached_bytes_ > budget) release_cached_locked();
  }

  void poll_pending() {
    for (size_t i = 0; i < pending_.size();) {
      bool done = true;
      for (cudaEvent_t ev : pending_[i].events)
        if (cudaEventQuery(ev) != cudaSuccess) {
          done = false;
          break;
        }
      if (done) {
        (void)cudaGetLastError();
        for (cudaEvent_t ev : pending_[i].events) cudaEventDestroy(ev);
        to_cache(pending_[i].block);
        pending_[i] = std::move(pending_.back());
        pending_.pop_back();
      } else {
        (void)cudaGetLastError();
        ++i;
      }
    }
  }

  void release_cached_locked() {
    // cudaFree synchronizes the device, so every use of a cached block on any
    // stream has finished before its memory goes back to the driver.
    for (auto& kv : free_) {
      for (auto& e : kv.second) {
        cudaFree(e.second->ptr);
        reserved_bytes_ -= e.second->size;
        delete e.second;
      }
      kv.second.clear();
    }
    cached_bytes_ = 0;
  }

  static size_t budget_bytes() {
    static const size_t b = [] {
      const char* s = std::getenv("XDNA_BO_CACHE_MB");
      return s ? size_t(std::strtoull(s, nullptr, 10)) << 20 : size_t(0);
    }();
    return b;
  }

  std::mutex mu_;
  std::unordered_map<uint64_t, std::multimap<size_t, Block*>> free_;
  std::unordered_map<void*, Block*> live_;
  std::vector<PendingFree> pending_;
  std::unordered_map<int, GraphPool> pools_;
  std::unordered_map<cudaStream_t, int> capture_pool_;  // capturing stream -> pool id
  std::vector<Block*> held_;                            // ordinary blocks freed during a capture
  int capturing_ = 0, next_pool_ = 1;
  size_t allocated_bytes_ = 0, reserved_bytes_ = 0, cached_bytes_ = 0;
  size_t peak_allocated_ = 0, peak_reserved_ = 0;
  int64_t num_allocs_ = 0, num_frees_ = 0, cache_hits_ = 0, device_mallocs_ = 0;
};

Cache& cache() {
  static Cache* c = new Cache();  // leaked on purpose: frees may run during exit
  return *c;
}

void raw_delete(void* p) { cache().free(p); }

struct XdnaAllocator final : c10::Allocator {
  c10::DataPtr allocate(size_t n) override {
    int dev = 0;
    XDNA_CUDA(cudaGetDevice(&dev));
    void* p = nullptr;
    if (n) p = cache().malloc(n, dev, stream(c10::DeviceIndex(dev)));
    return {p, p, &raw_delete, c10::Device(kXdna, c10::DeviceIndex(dev))};
  }
  c10::DeleterFnPtr raw_deleter() const override { return &raw_delete; }
  void copy_data(void* dst, const void* src, std::size_t count) const override {
    int dev = 0;
    XDNA_CUDA(cudaGetDevice(&dev));
    XDNA_CUDA(cudaMemcpyAsync(dst, src, count, cudaMemcpyDeviceToDevice, stream(c10::DeviceIndex(dev))));
  }
};

XdnaAllocator g_allocator;

}  // namespace

c10::Allocator* allocator() { return &g_allocator; }

void record_stream(const c10::DataPtr& ptr, cudaStream_t s) {
  if (ptr.get_deleter() == &raw_delete) cache().record(ptr.get(), s);
}

void empty_cache() { cache().empty(); }

int graph_capture_begin(int device, cudaStream_t stream, int share_pool) {
  return cache().capture_begin(device, stream, share_pool);
}
void graph_capture_end(cudaStream_t stream) { cache().capture_end(stream); }
void graph_pool_release(int pool) { cache().release_pool(pool); }

std::map<std::string, int64_t> allocator_stats() { return cache().stats(); }

REGISTER_ALLOCATOR(c10::DeviceType::PrivateUse1, &g_allocator);

}  // namespace xdna
