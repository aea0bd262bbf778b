// Native device runtime: a stream-ordered caching allocator and a stream pool.
//
// Reference counterparts: PredictiveCoding.Device/Allocators/CudaAllocator.cs:19-104 (one
// cudaMalloc / cudaFree per DeviceTensor, byte accounting) and Streams/CudaStreamManager.cs:17-83
// (a lazily created per-device stream list).  The B200 design keeps freed blocks in per-device
// size-binned free lists instead of returning them to the driver (cudaMalloc/cudaFree synchronise
// the device), rounds requests to 512 B below 1 MiB and to 2 MiB above, and makes reuse
// stream-safe: a block freed while work on another stream may still read it carries an event and
// is handed out again only after that event has completed.  Everything here is host code.
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace {

constexpr size_t kSmallLimit = 1u << 20;   // 1 MiB
constexpr size_t kSmallRound = 512;
constexpr size_t kLargeRound = 2u << 20;   // 2 MiB

size_t round_size(size_t n) {
  if (n == 0) n = 1;
  if (n < kSmallLimit) return (n + kSmallRound - 1) / kSmallRound * kSmallRound;
  return (n + kLargeRound - 1) / kLargeRound * kLargeRound;
}

struct Block {
  void* ptr = nullptr;
  size_t size = 0;
  int device = 0;
  cudaStream_t stream = nullptr;    // allocating stream
  std::vector<cudaEvent_t> pending; // one per foreign stream that used the block, recorded at free
};

struct DeviceStats {
  long long allocated = 0, reserved = 0, peak = 0, n_alloc = 0, n_hit = 0, n_driver = 0;
};

class CachingAllocator {
 public:
  static CachingAllocator& get() {
    static CachingAllocator a;
    return a;
  }

  // returns 0 and the pointer, or a negative code
  int alloc(int device, size_t bytes, cudaStream_t stream, void** out) {
    std::lock_guard<std::mutex> g(mu_);
    const size_t sz = round_size(bytes);
    auto& pool = free_[device];
    // best fit among blocks of the same stream; small blocks may be at most 2x, large at most +4 MiB
    const size_t limit = sz < kSmallLimit ? 2 * sz : sz + 2 * kLargeRound;
    for (auto it = pool.lower_bound(sz); it != pool.end() && it->first <= limit; ++it) {
      Block* b = it->second;
      if (b->stream != stream) continue;
      if (!b->pending.empty()) {
        bool ready = true;
        for (cudaEvent_t ev : b->pending) {
          if (cudaEventQuery(ev) != cudaSuccess) {
            ready = false;
            break;
          }
        }
        if (!ready) {
          cudaGetLastError();   // clear cudaErrorNotReady
          continue;
        }
        for (cudaEvent_t ev : b->pending) cudaEventDestroy(ev);
        b->pending.clear();
      }
      pool.erase(it);
      live_[b->ptr] = b;
      auto& st = stats_[device];
      st.allocated += b->size;
      st.peak = st.allocated > st.peak ? st.allocated : st.peak;
      st.n_alloc++;
      st.n_hit++;
      *out = b->ptr;
      return 0;
    }
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, sz);
    if (e != cudaSuccess) {
      cudaGetLastError();
      release_cached_locked(device);   // retry once after giving the cache back
      e = cudaMalloc(&p, sz);
    }
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return -4;
    }
    Block* b = new Block{p, sz, device, stream, {}};
    live_[p] = b;
    auto& st = stats_[device];
    st.reserved += sz;
    st.allocated += sz;
    st.peak = st.allocated > st.peak ? st.allocated : st.peak;
    st.n_alloc++;
    st.n_driver++;
    *out = p;
    return 0;
  }

  // record that `stream` (other than the allocating one) used the block
  int record_stream(void* ptr, cudaStream_t stream) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = live_.find(ptr);
    if (it == live_.end()) return -2;
    used_on_[ptr].push_back(stream);
    return 0;
  }

  int free(void* ptr) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = live_.find(ptr);
    if (it == live_.end()) return -2;
    Block* b = it->second;
    live_.erase(it);
    auto u = used_on_.find(ptr);
    if (u != used_on_.end()) {
      // the block may be reused once every foreign stream has passed this point
      for (cudaStream_t s : u->second) {
        if (s == b->stream) continue;
        cudaEvent_t ev;
        cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        cudaEventRecord(ev, s);
        b->pending.push_back(ev);
      }
      used_on_.erase(u);
    }
    stats_[b->device].allocated -= b->size;
    free_[b->device].emplace(b->size, b);
    return 0;
  }

  void release_cached(int device) {
    std::lock_guard<std::mutex> g(mu_);
    release_cached_locked(device);
  }

  DeviceStats stats(int device) {
    std::lock_guard<std::mutex> g(mu_);
    return stats_[device];
  }

  void reset_peak(int device) {
    std::lock_guard<std::mutex> g(mu_);
    stats_[device].peak = stats_[device].allocated;
  }

 private:
  void release_cached_locked(int device) {
    auto& pool = free_[device];
    for (auto it = pool.begin(); it != pool.end();) {
      Block* b = it->second;
      for (cudaEvent_t ev : b->pending) {
        cudaEventSynchronize(ev);
        cudaEventDestroy(ev);
      }
      cudaFree(b->ptr);
      stats_[device].reserved -= b->size;
      delete b;
      it = pool.erase(it);
    }
  }

  std::mutex mu_;
  std::unordered_map<int, std::multimap<size_t, Block*>> free_;
  std::unordered_map<void*, Block*> live_;
  std::unordered_map<void*, std::vector<cudaStream_t>> used_on_;
  std::unordered_map<int, DeviceStats> stats_;
};

class StreamPool {
 public:
  static StreamPool& get() {
    static StreamPool p;
    return p;
  }
  // n streams per (device, priority) created on first use; returns the i-th (mod n)
  int stream(int device, int index, int high_priority, int n, cudaStream_t* out) {
    std::lock_guard<std::mutex> g(mu_);
    auto key = std::make_pair(device, high_priority);
    auto& v = pools_[key];
    if (v.empty()) {
      int prev = -1;
      cudaGetDevice(&prev);
      if (prev != device) cudaSetDevice(device);
      int lo = 0, hi = 0;
      cudaDeviceGetStreamPriorityRange(&lo, &hi);
      for (int i = 0; i < n; ++i) {
        cudaStream_t s;
        if (cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, high_priority ? hi : lo) != cudaSuccess) {
          if (prev != device) cudaSetDevice(prev);
          return -3;
        }
        v.push_back(s);
      }
      if (prev != device) cudaSetDevice(prev);
    }
    *out = v[static_cast<size_t>(index) % v.size()];
    return 0;
  }
  int count(int device, int high_priority) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = pools_.find(std::make_pair(device, high_priority));
    return it == pools_.end() ? 0 : static_cast<int>(it->second.size());
  }

 private:
  std::mutex mu_;
  std::map<std::pair<int, int>, std::vector<cudaStream_t>> pools_;
};

}  // namespace

int pcb_alloc(int device, size_t bytes, void* stream, void** out) {
  return CachingAllocator::get().alloc(device, bytes, reinterpret_cast<cudaStream_t>(stream), out);
}
int pcb_free(void* ptr) { return CachingAllocator::get().free(ptr); }
int pcb_record_stream(void* ptr, void* stream) {
  return CachingAllocator::get().record_stream(ptr, reinterpret_cast<cudaStream_t>(stream));
}
void pcb_release_cached(int device) { CachingAllocator::get().release_cached(device); }
void pcb_alloc_stats(int device, long long* out6) {
  DeviceStats s = CachingAllocator::get().stats(device);
  out6[0] = s.allocated;
  out6[1] = s.reserved;
  out6[2] = s.peak;
  out6[3] = s.n_alloc;
  out6[4] = s.n_hit;
  out6[5] = s.n_driver;
}
void pcb_alloc_reset_peak(int device) { CachingAllocator::get().reset_peak(device); }
int pcb_stream(int device, int index, int high_priority, int n, void** out) {
  cudaStream_t s = nullptr;
  int rc = StreamPool::get().stream(device, index, high_priority, n, &s);
  *out = s;
  return rc;
}
int pcb_stream_count(int device, int high_priority) { return StreamPool::get().count(device, high_priority); }
