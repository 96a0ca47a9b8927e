// host_io.cpp — host<->device staging for the host-pointer entry points.
//
// A pageable host buffer handed to cudaMemcpyAsync moves through the
// driver's own bounce buffer at a fraction of the link rate. Large inputs
// instead go through two context-owned pinned stages: worker threads copy
// chunk i+1 into one stage while the DMA engine drains chunk i from the
// other. Page-locked host buffers are copied directly. The copy is complete from the caller's point of view (the source
// may be reused) when h2d_staged returns; the device side is ordered on the
// context stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "mvr_internal.h"

namespace mvr {

// Fixed worker pool; run(n, f) executes f(0) .. f(n-1) on the workers and
// the calling thread and returns when all are done.
class HostPool {
 public:
  explicit HostPool(int workers) {
    for (int i = 0; i < workers; ++i) th_.emplace_back([this] { loop(); });
  }
  ~HostPool() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
  }
  int size() const { return (int)th_.size() + 1; }
  void run(int n, const std::function<void(int)>& f) {
    {
      std::lock_guard<std::mutex> lk(m_);
      job_ = &f;
      n_ = n;
      next_ = 0;
      done_ = 0;
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> lk(m_);
    done_cv_.wait(lk, [&] { return done_ == n_; });
    job_ = nullptr;
  }

 private:
  void work() {
    for (;;) {
      int i;
      const std::function<void(int)>* f;
      {
        std::lock_guard<std::mutex> lk(m_);
        if (!job_ || next_ >= n_) return;
        i = next_++;
        f = job_;
      }
      (*f)(i);
      std::lock_guard<std::mutex> lk(m_);
      if (++done_ == n_) done_cv_.notify_all();
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(m_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
      }
      work();
    }
  }
  std::vector<std::thread> th_;
  std::mutex m_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int)>* job_ = nullptr;
  int n_ = 0, next_ = 0, done_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

namespace {
// Page-locked (pinned or registered) host memory goes to the DMA engine
// directly; only pageable memory needs the stages.
bool is_pinned(const void* h) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, h) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

constexpr size_t kStageBytes = 32u << 20;
constexpr size_t kStagedMin = 8u << 20;  // smaller copies go straight to the driver
constexpr size_t kPiece = 2u << 20;

int ensure_io(Ctx* c) {
  if (!c->io_pool) {
    const unsigned hc = std::max(1u, std::thread::hardware_concurrency());
    c->io_pool = new HostPool((int)std::min(hc, 8u) - 1);
  }
  for (int s = 0; s < 2; ++s) {
    if (!c->stage[s]) MVR_CUDA(c, cudaMallocHost(&c->stage[s], kStageBytes));
    if (!c->stage_ev[s]) MVR_CUDA(c, cudaEventCreateWithFlags(&c->stage_ev[s], cudaEventDisableTiming));
  }
  return MVR_OK;
}
}  // namespace

bool host_is_pinned(const void* h) { return is_pinned(h); }

int h2d_staged(Ctx* c, void* d, const void* h, size_t bytes) {
  if (bytes == 0) return MVR_OK;
  if (bytes < kStagedMin || is_pinned(h)) {
    MVR_CUDA(c, cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, c->stream));
    return MVR_OK;
  }
  MVR_TRY(ensure_io(c));
  const auto* src = static_cast<const unsigned char*>(h);
  auto* dst = static_cast<unsigned char*>(d);
  size_t off = 0;
  for (int i = 0; off < bytes; ++i) {
    const int s = i & 1;
    const size_t len = std::min(kStageBytes, bytes - off);
    MVR_CUDA(c, cudaEventSynchronize(c->stage_ev[s]));  // the DMA that last read stage s is done
    unsigned char* stage = static_cast<unsigned char*>(c->stage[s]);
    const int pieces = (int)((len + kPiece - 1) / kPiece);
    c->io_pool->run(pieces, [&](int p) {
      const size_t o = (size_t)p * kPiece;
      std::memcpy(stage + o, src + off + o, std::min(kPiece, len - o));
    });
    MVR_CUDA(c, cudaMemcpyAsync(dst + off, stage, len, cudaMemcpyHostToDevice, c->stream));
    MVR_CUDA(c, cudaEventRecord(c->stage_ev[s], c->stream));
    off += len;
  }
  return MVR_OK;
}

int d2h_staged(Ctx* c, void* h, const void* d, size_t bytes) {
  if (bytes == 0) return MVR_OK;
  if (bytes < kStagedMin || is_pinned(h)) {
    MVR_CUDA(c, cudaMemcpyAsync(h, d, bytes, cudaMemcpyDeviceToHost, c->stream));
    MVR_CUDA(c, cudaStreamSynchronize(c->stream));
    return MVR_OK;
  }
  MVR_TRY(ensure_io(c));
  auto* out = static_cast<unsigned char*>(h);
  const auto* src = static_cast<const unsigned char*>(d);
  // DMA chunk i+1 into one stage while the workers drain chunk i from the other
  const size_t n = (bytes + kStageBytes - 1) / kStageBytes;
  auto issue = [&](size_t i) -> int {
    const int s = (int)(i & 1);
    const size_t o = i * kStageBytes, len = std::min(kStageBytes, bytes - o);
    MVR_CUDA(c, cudaMemcpyAsync(c->stage[s], src + o, len, cudaMemcpyDeviceToHost, c->stream));
    MVR_CUDA(c, cudaEventRecord(c->stage_ev[s], c->stream));
    return MVR_OK;
  };
  MVR_TRY(issue(0));
  for (size_t i = 0; i < n; ++i) {
    const int s = (int)(i & 1);
    MVR_CUDA(c, cudaEventSynchronize(c->stage_ev[s]));
    if (i + 1 < n) MVR_TRY(issue(i + 1));
    const size_t o = i * kStageBytes, len = std::min(kStageBytes, bytes - o);
    const unsigned char* stage = static_cast<const unsigned char*>(c->stage[s]);
    const int pieces = (int)((len + kPiece - 1) / kPiece);
    c->io_pool->run(pieces, [&](int p) {
      const size_t q = (size_t)p * kPiece;
      std::memcpy(out + o + q, stage + q, std::min(kPiece, len - q));
    });
  }
  return MVR_OK;
}

void destroy_host_io(Ctx* c) {
  delete c->io_pool;
  c->io_pool = nullptr;
  for (int s = 0; s < 2; ++s) {
    if (c->stage_ev[s]) cudaEventSynchronize(c->stage_ev[s]);
    if (c->stage[s]) cudaFreeHost(c->stage[s]);
    if (c->stage_ev[s]) cudaEventDestroy(c->stage_ev[s]);
    c->stage[s] = nullptr;
    c->stage_ev[s] = nullptr;
  }
}

}  // namespace mvr
