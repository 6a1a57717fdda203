// Host-side fp32 -> fp16 cast with the reference's truncation rule
// (include/infvino/Half.hpp:14-24: the mantissa is truncated, exponents that
// underflow give a signed zero, ones that overflow give a signed infinity),
// vectorised and spread over a process-wide pool of worker threads.
// `ClBackend::infer` on host buffers casts its f32 input here, so that the
// PCIe copy carries fp16 (half the bytes of the f32 input).
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>

namespace ivb {

// out[i] = truncating fp16 bits of in[i], for i in [0, n), on this thread.
void f32_to_f16_trunc_span(const float *in, uint16_t *out, size_t n);

// The same over all worker threads (the caller's thread takes a share too).
void f32_to_f16_trunc_host(const float *in, uint16_t *out, size_t n);

// Runs f(begin, end) over [0, n) split into at most one range per worker
// thread (plus the caller), each at least `grain` long; returns when every
// range is done.  Calls from several threads take turns.
void host_parallel_for(size_t n, size_t grain, const std::function<void(size_t, size_t)> &f);

}  // namespace ivb
