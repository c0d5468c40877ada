#include "C3/CudaRuntime.h"

#include <algorithm>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <vector>

#include "c3cu.h"

namespace ct {
namespace c3 {
namespace cuda {

namespace {
thread_local cudaStream_t t_stream = nullptr;

void configurePool(int dev) {
  static std::mutex mu;
  static std::vector<bool> done;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(done.size()) <= dev) done.resize(dev + 1, false);
  if (done[dev]) return;
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  }
  done[dev] = true;
}
}  // namespace

cudaStream_t currentStream() { return t_stream; }
void setCurrentStream(cudaStream_t s) { t_stream = s; }

bool deviceAvailable() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

void* allocDevice(size_t bytes) {
  if (bytes == 0) bytes = 256;
  int dev = 0;
  checkCuda(cudaGetDevice(&dev), "allocDevice: cudaGetDevice");
  configurePool(dev);
  void* p = nullptr;
  checkCuda(cudaMallocAsync(&p, bytes, t_stream), "allocDevice: cudaMallocAsync");
  return p;
}

void freeDevice(void* p, cudaStream_t stream) {
  if (p) cudaFreeAsync(p, stream);
}

namespace {

// A fixed pool of host threads for the staging copies (created on first use, joined at exit).
class CopyPool {
 public:
  static CopyPool& instance() {
    static CopyPool p;
    return p;
  }

  // memcpy of `n` bytes split over the pool's threads (and the calling thread); returns when done.
  void copy(void* dst, const void* src, size_t n) {
    const size_t parts = std::min<size_t>(workers_.size() + 1, std::max<size_t>(1, n >> 20));
    if (parts <= 1) {
      std::memcpy(dst, src, n);
      return;
    }
    const size_t per = (n + parts - 1) / parts;
    {
      std::lock_guard<std::mutex> lk(mu_);
      for (size_t i = 1; i < parts; ++i) {
        const size_t o = i * per;
        if (o >= n) break;
        const size_t len = std::min(per, n - o);
        ++pending_;
        jobs_.push_back([=] { std::memcpy(static_cast<char*>(dst) + o, static_cast<const char*>(src) + o, len); });
      }
    }
    cv_.notify_all();
    std::memcpy(dst, src, std::min(per, n));
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return pending_ == 0; });
  }

 private:
  CopyPool() {
    const unsigned hc = std::thread::hardware_concurrency();
    const unsigned n = std::max(1u, std::min(8u, hc > 1 ? hc / 2 : 1u));
    for (unsigned i = 0; i + 1 < n; ++i) workers_.emplace_back([this] { run(); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  void run() {
    for (;;) {
      std::function<void()> job;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || !jobs_.empty(); });
        if (stop_ && jobs_.empty()) return;
        job = std::move(jobs_.back());
        jobs_.pop_back();
      }
      job();
      {
        std::lock_guard<std::mutex> lk(mu_);
        --pending_;
      }
      done_cv_.notify_all();
    }
  }
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::vector<std::function<void()>> jobs_;
  std::vector<std::thread> workers_;
  size_t pending_ = 0;
  bool stop_ = false;
};

// Pinned staging buffers, each with the event of the last DMA that used it. One set per device:
// an event can only be recorded on a stream of the device it was created on.
struct Staging {
  static constexpr size_t kChunk = 8u << 20;
  static constexpr int kBuffers = 3;
  std::mutex mu;
  void* buf[kBuffers] = {};
  cudaEvent_t ev[kBuffers] = {};
  bool ready = false;

  // The set of the current device (the device of the copy's stream and device buffer).
  static Staging& forCurrentDevice() {
    static std::mutex mu_all;
    static std::vector<std::unique_ptr<Staging>> per_device;
    int dev = 0;
    checkCuda(cudaGetDevice(&dev), "staging: cudaGetDevice");
    std::lock_guard<std::mutex> lk(mu_all);
    if (static_cast<int>(per_device.size()) <= dev) per_device.resize(dev + 1);
    if (!per_device[dev]) per_device[dev] = std::make_unique<Staging>();
    return *per_device[dev];
  }
  void init() {  // under mu
    if (ready) return;
    for (int i = 0; i < kBuffers; ++i) {
      checkCuda(cudaMallocHost(&buf[i], kChunk), "staging: cudaMallocHost");
      checkCuda(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming), "staging: cudaEventCreate");
    }
    ready = true;
  }
};

constexpr size_t kStageThreshold = 4u << 20;

}  // namespace

void copyToDevice(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  if (bytes < kStageThreshold) {
    checkCuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream), "copyToDevice");
    return;
  }
  Staging& st = Staging::forCurrentDevice();
  std::lock_guard<std::mutex> lk(st.mu);
  st.init();
  size_t o = 0;
  for (int i = 0; o < bytes; ++i, o += Staging::kChunk) {
    const int b = i % Staging::kBuffers;
    const size_t len = std::min(Staging::kChunk, bytes - o);
    checkCuda(cudaEventSynchronize(st.ev[b]), "copyToDevice: staging buffer free");
    CopyPool::instance().copy(st.buf[b], static_cast<const char*>(src) + o, len);
    checkCuda(cudaMemcpyAsync(static_cast<char*>(dst) + o, st.buf[b], len, cudaMemcpyHostToDevice, stream),
              "copyToDevice: chunk");
    checkCuda(cudaEventRecord(st.ev[b], stream), "copyToDevice: event");
  }
}

void copyToHost(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  if (bytes < kStageThreshold) {
    checkCuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, stream), "copyToHost");
    checkCuda(cudaStreamSynchronize(stream), "copyToHost: synchronize");
    return;
  }
  Staging& st = Staging::forCurrentDevice();
  std::lock_guard<std::mutex> lk(st.mu);
  st.init();
  const size_t n = (bytes + Staging::kChunk - 1) / Staging::kChunk;
  auto drain = [&](size_t i) {  // chunk i has landed in its staging buffer: copy it out
    const int b = static_cast<int>(i % Staging::kBuffers);
    const size_t o = i * Staging::kChunk, len = std::min(Staging::kChunk, bytes - o);
    checkCuda(cudaEventSynchronize(st.ev[b]), "copyToHost: chunk landed");
    CopyPool::instance().copy(static_cast<char*>(dst) + o, st.buf[b], len);
  };
  for (size_t i = 0; i < n; ++i) {
    const int b = static_cast<int>(i % Staging::kBuffers);
    if (i >= static_cast<size_t>(Staging::kBuffers)) drain(i - Staging::kBuffers);  // frees buffer b
    checkCuda(cudaEventSynchronize(st.ev[b]), "copyToHost: staging buffer free");
    const size_t o = i * Staging::kChunk, len = std::min(Staging::kChunk, bytes - o);
    checkCuda(cudaMemcpyAsync(st.buf[b], static_cast<const char*>(src) + o, len, cudaMemcpyDeviceToHost, stream),
              "copyToHost: chunk");
    checkCuda(cudaEventRecord(st.ev[b], stream), "copyToHost: event");
  }
  for (size_t i = n > static_cast<size_t>(Staging::kBuffers) ? n - Staging::kBuffers : 0; i < n; ++i) drain(i);
}

void checkAbi(int rc, const char* what) {
  if (rc != C3CU_OK) throw std::runtime_error(std::string(what) + ": " + c3cu_last_error());
}

void checkCuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace cuda
}  // namespace c3
}  // namespace ct
