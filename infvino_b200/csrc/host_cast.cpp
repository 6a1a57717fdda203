// Host fp32 -> fp16 truncating cast and the worker pool it runs on.
#include "host_cast.h"

#include <immintrin.h>
#include <sched.h>

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace ivb {

namespace {

// One value; the branch-free form the vector paths follow lane by lane.
inline uint16_t trunc1(uint32_t x) {
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int32_t e = (int32_t)((x >> 23) & 0xffu) - 112;
  const uint32_t normal = sign | ((uint32_t)e << 10) | ((x >> 13) & 0x3ffu);
  const uint32_t h = e <= 0 ? sign : e >= 31 ? (sign | 0x7c00u) : normal;
  return (uint16_t)h;
}

void span_scalar(const float *in, uint16_t *out, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    uint32_t x;
    std::memcpy(&x, in + i, 4);
    out[i] = trunc1(x);
  }
}

// Eight values per 256-bit register: the same integer steps, the two
// selects as blends, and two registers packed to sixteen halves (the pack
// works per 128-bit lane, so a cross-lane permute restores the order).
__attribute__((target("avx2"))) __m256i trunc8(__m256i x) {
  const __m256i sign = _mm256_and_si256(_mm256_srli_epi32(x, 16), _mm256_set1_epi32(0x8000));
  const __m256i e = _mm256_sub_epi32(_mm256_and_si256(_mm256_srli_epi32(x, 23), _mm256_set1_epi32(0xff)),
                                     _mm256_set1_epi32(112));
  const __m256i normal = _mm256_or_si256(
      _mm256_or_si256(sign, _mm256_slli_epi32(e, 10)),
      _mm256_and_si256(_mm256_srli_epi32(x, 13), _mm256_set1_epi32(0x3ff)));
  const __m256i under = _mm256_cmpgt_epi32(_mm256_set1_epi32(1), e);  // e <= 0
  const __m256i over = _mm256_cmpgt_epi32(e, _mm256_set1_epi32(30));  // e >= 31
  __m256i h = _mm256_blendv_epi8(normal, sign, under);
  return _mm256_blendv_epi8(h, _mm256_or_si256(sign, _mm256_set1_epi32(0x7c00)), over);
}

__attribute__((target("avx2"))) void span_avx2(const float *in, uint16_t *out, size_t n) {
  // Streaming (non-temporal) stores from the first 32-byte boundary on: the
  // fp16 output is read next by the copy engine, not by this core, and a
  // streaming store skips the read-for-ownership of each destination line,
  // which takes a third of the host memory traffic off the cast.
  size_t i = 0;
  const size_t head = std::min(n, (size_t)(((32u - (reinterpret_cast<uintptr_t>(out) & 31u)) & 31u) / 2u));
  span_scalar(in, out, head);
  i = head;
  const bool aligned = (reinterpret_cast<uintptr_t>(out + i) & 31u) == 0;
  for (; i + 16 <= n; i += 16) {
    const __m256i a = trunc8(_mm256_loadu_si256(reinterpret_cast<const __m256i *>(in + i)));
    const __m256i b = trunc8(_mm256_loadu_si256(reinterpret_cast<const __m256i *>(in + i + 8)));
    const __m256i p = _mm256_permute4x64_epi64(_mm256_packus_epi32(a, b), 0xd8);  // 0, 2, 1, 3
    if (aligned)
      _mm256_stream_si256(reinterpret_cast<__m256i *>(out + i), p);
    else
      _mm256_storeu_si256(reinterpret_cast<__m256i *>(out + i), p);
  }
  _mm_sfence();  // the streamed lines reach memory before the copy that reads them is queued
  span_scalar(in + i, out + i, n - i);
}

unsigned process_cpus() {
  cpu_set_t set;
  CPU_ZERO(&set);
  if (sched_getaffinity(0, sizeof(set), &set) == 0) return (unsigned)CPU_COUNT(&set);
  return std::thread::hardware_concurrency();
}

bool have_avx2() {
  static const bool yes = __builtin_cpu_supports("avx2") != 0;
  return yes;
}

// Worker threads that wait for one job at a time: a job is a function over
// [0, n) cut into `parts` ranges, taken by index until none is left.
class Pool {
 public:
  Pool() {
    // sized from the CPUs this process may run on (its affinity mask, which a
    // multi-GPU launcher may have narrowed to the cores near the rank's GPU),
    // not from the machine's core count: ranks sharing a host must not
    // oversubscribe it
    const unsigned cpus = std::max(1u, process_cpus());
    const unsigned workers = std::min(cpus, 16u) - 1;  // the caller works too
    for (unsigned t = 0; t < workers; ++t) th_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto &t : th_) t.join();
  }
  size_t threads() const { return th_.size() + 1; }

  void run(size_t n, size_t parts, const std::function<void(size_t, size_t)> &f) {
    std::lock_guard<std::mutex> job(job_mu_);  // one job at a time
    {
      std::lock_guard<std::mutex> lk(mu_);
      fn_ = &f;
      n_ = n;
      parts_ = parts;
      next_ = 0;
      left_ = parts;
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [this] { return left_ == 0; });
    fn_ = nullptr;
  }

 private:
  void work() {  // take ranges of the current job until none is left
    while (true) {
      size_t k;
      const std::function<void(size_t, size_t)> *f;
      {
        std::lock_guard<std::mutex> lk(mu_);
        if (fn_ == nullptr || next_ >= parts_) return;
        k = next_++;
        f = fn_;
      }
      const size_t b = n_ * k / parts_, e = n_ * (k + 1) / parts_;
      (*f)(b, e);
      std::lock_guard<std::mutex> lk(mu_);
      if (--left_ == 0) done_cv_.notify_all();
    }
  }
  void loop() {
    uint64_t seen = 0;
    while (true) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
      }
      work();
    }
  }

  std::vector<std::thread> th_;
  std::mutex mu_, job_mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(size_t, size_t)> *fn_ = nullptr;
  size_t n_ = 0, parts_ = 0, next_ = 0, left_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

Pool &pool() {
  static Pool p;
  return p;
}

}  // namespace

void f32_to_f16_trunc_span(const float *in, uint16_t *out, size_t n) {
  if (have_avx2())
    span_avx2(in, out, n);
  else
    span_scalar(in, out, n);
}

void host_parallel_for(size_t n, size_t grain, const std::function<void(size_t, size_t)> &f) {
  if (n == 0) return;
  const size_t parts = std::max<size_t>(1, std::min<size_t>(pool().threads(), n / std::max<size_t>(grain, 1)));
  if (parts == 1) {
    f(0, n);
    return;
  }
  pool().run(n, parts, f);
}

void f32_to_f16_trunc_host(const float *in, uint16_t *out, size_t n) {
  host_parallel_for(n, 1 << 16, [&](size_t b, size_t e) { f32_to_f16_trunc_span(in + b, out + b, e - b); });
}

}  // namespace ivb
