// C-linkage shim over the reference's fp16 conversion routines
// (include/infvino/Half.hpp:14-49, src/Half.cpp:93-107), compiled together with
// the reference's own src/Half.cpp into oracle/_ref/ so that tests can check the
// oracle's conversions against the reference itself.  Test infrastructure only.
#include <cstddef>
#include <cstdint>

#include "infvino/Half.hpp"

extern "C" {
uint16_t ref_f32_to_f16(float f) { return infvino::f32_to_f16(f); }
float ref_f16_to_f32(uint16_t h) { return infvino::f16_to_f32(h); }
void ref_f32_to_f16_bulk(const float *in, uint16_t *out, size_t n) { infvino::f32_to_f16_bulk(in, out, n); }
void ref_f16_to_f32_bulk(const uint16_t *in, float *out, size_t n) { infvino::f16_to_f32_bulk(in, out, n); }
// scalar paths over buffers (no float return through the C ABI, which would
// quiet signalling NaNs)
void ref_f32_to_f16_scalar_n(const float *in, uint16_t *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = infvino::f32_to_f16(in[i]);
}
void ref_f16_to_f32_scalar_n(const uint16_t *in, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = infvino::f16_to_f32(in[i]);
}
}
