// loader.cpp — native batch loader: worker threads fill a ring of (pinned) host buffers
// with token windows ahead of the training step, so batch assembly never sits on the
// step's critical path.
//
// Sources:
//   random  uniform tokens from a counter-based generator: token (b, t) of step s for
//           rank r is a pure function of (seed, s, r, b, t) (SplitMix64 finaliser over a
//           Weyl sequence), so batches do not depend on thread scheduling
//   file    windows of T + 1 tokens of a memory-mapped token file — uint8 (bytes) or
//           little-endian uint16 (a BPE vocabulary) — split train / valid at `ratio`,
//           window starts drawn from the same counter-based generator
//   stream  consecutive chunks of `batch` independent streams (stateful TBPTT): stream b
//           of the split is the contiguous range [b * len, (b + 1) * len); chunk k covers
//           positions [k * chunk, k * chunk + chunk + 1) and wraps to 0 at the end
//
// The data-loading role of the reference's Rust loaders (random and streaming loaders
// with prefetch workers, burn_dragon_language/src/dataset/scheduler.rs); the windows and
// RNG stream are this framework's own.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <torch/extension.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// 64-bit draw number `i` of stream (seed, step, rank)
inline uint64_t draw(uint64_t seed, uint64_t step, uint64_t rank, uint64_t i) {
  const uint64_t key = mix64(seed * 0x9e3779b97f4a7c15ull ^ mix64(step + 0x632be59bd9b4e019ull) ^
                             mix64(rank + 0x8cb92ba72f3d8dd7ull));
  return mix64(key + i * 0x9e3779b97f4a7c15ull);
}

class Loader {
 public:
  Loader(const std::string& mode, const std::string& path, int64_t batch, int64_t block, int64_t vocab,
         int64_t seed, int64_t rank, int64_t world, double ratio, bool valid_split, int64_t chunk,
         std::vector<at::Tensor> buffers, int64_t workers, int64_t start_step, int64_t elem_bytes)
      : esize_(elem_bytes), mode_(mode), batch_(batch), block_(block), vocab_(vocab), seed_(seed), rank_(rank), world_(world),
        chunk_(chunk), bufs_(std::move(buffers)), next_issue_(start_step), next_take_(start_step) {
    if (mode_ != "random" && mode_ != "file" && mode_ != "stream") throw std::invalid_argument("unknown mode " + mode_);
    if (esize_ != 1 && esize_ != 2) throw std::invalid_argument("token files hold 1- or 2-byte tokens");
    if (batch_ <= 0 || block_ <= 0 || bufs_.empty()) throw std::invalid_argument("batch, block > 0 and >= 1 buffer");
    for (auto& b : bufs_) {
      TORCH_CHECK(b.scalar_type() == at::kLong && b.is_contiguous() && !b.is_cuda(), "buffers: contiguous int64 host");
      TORCH_CHECK(b.numel() >= batch_ * (block_ + 1), "buffer too small for [batch, block + 1]");
    }
    if (mode_ != "random") open_file(path, ratio, valid_split);
    slot_step_.assign(bufs_.size(), -1);
    ready_.assign(bufs_.size(), false);
    for (size_t i = 0; i < bufs_.size(); ++i) free_.push_back((int)i);
    const int n = (int)std::max<int64_t>(1, workers);
    for (int i = 0; i < n; ++i) threads_.emplace_back([this] { work(); });
  }

  ~Loader() { close(); }

  void close() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    cv_work_.notify_all();
    cv_ready_.notify_all();
    for (auto& t : threads_)
      if (t.joinable()) t.join();
    threads_.clear();
    if (map_) {
      munmap(map_, map_len_);
      map_ = nullptr;
    }
  }

  // Blocks until the batch of the next step is ready; returns (buffer index, step).
  std::vector<int64_t> take() {
    std::unique_lock<std::mutex> lk(mu_);
    const int64_t want = next_take_;
    cv_ready_.wait(lk, [&] { return stop_ || find_ready(want) >= 0 || !error_.empty(); });
    if (!error_.empty()) throw std::runtime_error(error_);
    if (stop_) throw std::runtime_error("loader closed");
    const int slot = find_ready(want);
    ready_[slot] = false;
    ++next_take_;
    return {slot, want};
  }

  // The caller is done with a buffer (after its host-to-device copy has been ordered).
  void release(int64_t slot) {
    {
      std::lock_guard<std::mutex> g(mu_);
      slot_step_[slot] = -1;
      free_.push_back((int)slot);
    }
    cv_work_.notify_one();
  }

  int64_t split_len() const { return (int64_t)split_len_; }

 private:
  void open_file(const std::string& path, double ratio, bool valid_split) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("cannot open " + path);
    struct stat st;
    fstat(fd, &st);
    map_len_ = (size_t)st.st_size;
    map_ = map_len_ ? mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    ::close(fd);
    if (map_ == MAP_FAILED) throw std::runtime_error("mmap failed for " + path);
    const size_t n = map_len_ / (size_t)esize_;  // tokens in the file
    const size_t cut = (size_t)((double)n * ratio);
    base_ = static_cast<const uint8_t*>(map_) + (valid_split ? cut : 0) * (size_t)esize_;
    split_len_ = valid_split ? n - cut : cut;
    if (mode_ == "file" && split_len_ <= (size_t)block_ + 1) throw std::runtime_error("split shorter than a window");
    if (mode_ == "stream") {
      stream_len_ = split_len_ / (size_t)batch_;
      if (chunk_ <= 0 || stream_len_ < (size_t)chunk_ + 1) throw std::runtime_error("streams shorter than a chunk");
    }
  }

  // token i of the split
  inline int64_t tok(size_t i) const {
    if (esize_ == 1) return base_[i];
    return (int64_t)base_[2 * i] | ((int64_t)base_[2 * i + 1] << 8);
  }

  int find_ready(int64_t step) const {
    for (size_t i = 0; i < ready_.size(); ++i)
      if (ready_[i] && slot_step_[i] == step) return (int)i;
    return -1;
  }

  void fill(int64_t step, int64_t* out) {
    const int64_t W = block_ + 1;
    if (mode_ == "random") {
      for (int64_t b = 0; b < batch_; ++b)
        for (int64_t t = 0; t < W; ++t)
          out[b * W + t] = (int64_t)(draw(seed_, (uint64_t)step, (uint64_t)rank_, (uint64_t)(b * W + t)) %
                                     (uint64_t)vocab_);
    } else if (mode_ == "file") {
      const uint64_t span = split_len_ - (size_t)W;
      for (int64_t b = 0; b < batch_; ++b) {
        const uint64_t s = draw(seed_, (uint64_t)step, (uint64_t)(rank_ + world_ * 7919), (uint64_t)b) % span;
        for (int64_t t = 0; t < W; ++t) out[b * W + t] = tok(s + (size_t)t);
      }
    } else {  // stream
      const int64_t per = (int64_t)((stream_len_ - 1) / (size_t)chunk_);  // whole chunks per stream
      const int64_t k = step % per;
      for (int64_t b = 0; b < batch_; ++b) {
        const size_t s0 = (size_t)b * stream_len_ + (size_t)(k * chunk_);
        for (int64_t t = 0; t < W; ++t) out[b * W + t] = tok(s0 + (size_t)t);
      }
    }
  }

  void work() {
    for (;;) {
      int slot;
      int64_t step;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_work_.wait(lk, [&] { return stop_ || !free_.empty(); });
        if (stop_) return;
        slot = free_.front();
        free_.pop_front();
        step = next_issue_++;
        slot_step_[slot] = step;
      }
      try {
        fill(step, bufs_[slot].data_ptr<int64_t>());
      } catch (const std::exception& e) {
        std::lock_guard<std::mutex> g(mu_);
        error_ = e.what();
      }
      {
        std::lock_guard<std::mutex> g(mu_);
        ready_[slot] = true;
      }
      cv_ready_.notify_all();
    }
  }

  int64_t esize_;
  std::string mode_;
  int64_t batch_, block_, vocab_, seed_, rank_, world_, chunk_;
  std::vector<at::Tensor> bufs_;
  void* map_ = nullptr;
  size_t map_len_ = 0, split_len_ = 0, stream_len_ = 0;
  const uint8_t* base_ = nullptr;
  std::mutex mu_;
  std::condition_variable cv_work_, cv_ready_;
  std::deque<int> free_;
  std::vector<int64_t> slot_step_;
  std::vector<bool> ready_;
  int64_t next_issue_, next_take_;
  bool stop_ = false;
  std::string error_;
  std::vector<std::thread> threads_;
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  pybind11::class_<Loader>(m, "Loader")
      .def(pybind11::init<const std::string&, const std::string&, int64_t, int64_t, int64_t, int64_t, int64_t,
                          int64_t, double, bool, int64_t, std::vector<at::Tensor>, int64_t, int64_t, int64_t>())
      .def("take", &Loader::take, pybind11::call_guard<pybind11::gil_scoped_release>())
      .def("release", &Loader::release)
      .def("split_len", &Loader::split_len)
      .def("close", &Loader::close, pybind11::call_guard<pybind11::gil_scoped_release>());
  m.def("draw", [](int64_t seed, int64_t step, int64_t rank, int64_t i) {
    return (int64_t)(draw((uint64_t)seed, (uint64_t)step, (uint64_t)rank, (uint64_t)i) >> 1);
  });
}
