// Shared device helpers for the sm_100a kernels: fp16 epilogue math, mbarriers,
// TMA (cp.async.bulk.tensor, no multicast), tcgen05 (TMEM alloc / MMA / commit /
// load) and a bounded wait that reports a timeout instead of spinning forever.
#pragma once

#include <atomic>
#include <utility>

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace ivb {

// ------------------------------------------------------------------ activations
// Canonical conv / gemm codes: 1=SiLU 2=ReLU 3=HardSwish 4=HardSigmoid 5=Sigmoid.
// `kind` selects the reference kernel family whose exact f32 expression is used:
//   0 = conv3x3_ov (only 1 and 3 act, kernels/conv_ov.cl:121-131)
//   1 = gemm / gemv (1..5, kernels/gemm.cl:137-153, kernels/conv1x1.cl:52-68)
//   2 = depthwise_f16 (1..4, HardSwish written f*(clamp/6), conv_general.cl:71-83)
enum ActKind : int { kActConv3x3 = 0, kActGemm = 1, kActDepthwise = 2 };

__device__ __forceinline__ float act_f32(float f, int act, int kind) {
  switch (act) {
    case 1:
      return f / (1.0f + expf(-f));
    case 2:
      return (kind == kActConv3x3) ? f : fmaxf(f, 0.0f);
    case 3:
      if (kind == kActDepthwise) return f * (fminf(fmaxf(f + 3.0f, 0.0f), 6.0f) / 6.0f);
      return f * fminf(fmaxf(f + 3.0f, 0.0f), 6.0f) / 6.0f;
    case 4:
      return (kind == kActConv3x3) ? f : fminf(fmaxf(f + 3.0f, 0.0f), 6.0f) / 6.0f;
    case 5:
      return (kind == kActConv3x3 || kind == kActDepthwise) ? f : 1.0f / (1.0f + expf(-f));
    default:
      return f;
  }
}

// Epilogue rounding points of the reference: v = half(half(acc) + bias);
// v = half(act(float(v))); v = half(v + res).  f32 arithmetic on two halves
// followed by one rounding equals the correctly rounded half operation.
__device__ __forceinline__ __half epilogue(float acc, float bias, int act, int kind) {
  const float v = __half2float(__float2half_rn(acc)) + bias;
  const float a = act_f32(__half2float(__float2half_rn(v)), act, kind);
  return __float2half_rn(a);
}

// ------------------------------------------------------------------ programmatic dependent launch
// Kernels are launched with programmatic stream serialization, so a grid can
// start while the previous one finishes.  Each kernel therefore waits for the
// grids before it (griddepcontrol.wait) before it touches global memory, and
// then lets the next grid launch: its CTAs take SMs as ours retire and run
// their own on-chip prologue in the meantime.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_and_release() {
  pdl_wait();
  pdl_release();
}

// Host side: whether launches on this thread carry the attribute (the engine
// turns it off for IVC_FLAG_NO_PDL), and the launcher every kernel goes through.
extern thread_local bool g_launch_pdl;
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_launch_pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// A kernel's dynamic shared-memory ceiling is a per-device attribute: it is set
// on the current device once, and `done` (one flag per device ordinal, shared
// by the threads of the process) remembers which devices have it.  Two threads
// may both set it the first time; setting it twice is harmless.  A failed call
// returns its error and clears the runtime's last error, so a later launch
// check does not report it.
constexpr int kAttrMaxDevices = 64;
template <typename... KArgs>
inline cudaError_t ensure_dynamic_smem(void (*kernel)(KArgs...), int bytes, std::atomic<bool> (&done)[kAttrMaxDevices]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool tracked = dev >= 0 && dev < kAttrMaxDevices;
  if (tracked && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return e;
  }
  if (tracked) done[dev].store(true, std::memory_order_release);
  return cudaSuccess;
}

// The shared-memory carveout (percent of the unified L1 / shared storage) a
// kernel prefers, set once per device like the dynamic ceiling above: kernels
// whose occupancy is bound by static shared memory ask for the largest.
template <typename... KArgs>
inline cudaError_t ensure_smem_carveout(void (*kernel)(KArgs...), int percent,
                                        std::atomic<bool> (&done)[kAttrMaxDevices]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool tracked = dev >= 0 && dev < kAttrMaxDevices;
  if (tracked && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, percent);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return e;
  }
  if (tracked) done[dev].store(true, std::memory_order_release);
  return cudaSuccess;
}

// ------------------------------------------------------------------ resolved activations
// The (act code, kernel family) pair resolved on the host to one function, so
// epilogues are compiled per function with no per-element dispatch.
enum ActFn : int {
  kFnNone = 0,
  kFnSilu = 1,
  kFnRelu = 2,
  kFnHswishA = 3,   // f * clamp(f + 3, 0, 6) / 6          (conv3x3_ov, gemm)
  kFnHsigmoid = 4,  // clamp(f + 3, 0, 6) / 6
  kFnSigmoid = 5,   // 1 / (1 + exp(-f))
  kFnHswishB = 6,   // f * (clamp(f + 3, 0, 6) / 6)        (depthwise_f16)
};

__host__ __device__ inline int resolve_act(int act, int kind) {
  if (act == 1) return kFnSilu;
  if (kind == kActConv3x3) return act == 3 ? kFnHswishA : kFnNone;
  if (act == 2) return kFnRelu;
  if (act == 3) return kind == kActDepthwise ? kFnHswishB : kFnHswishA;
  if (act == 4) return kFnHsigmoid;
  if (act == 5) return kind == kActDepthwise ? kFnNone : kFnSigmoid;
  return kFnNone;
}

// Reference-expression value of a resolved activation (accurate expf, IEEE division).
template <int FN>
__device__ __forceinline__ float act_exact(float f) {
  if (FN == kFnSilu) return f / (1.0f + expf(-f));
  if (FN == kFnRelu) return fmaxf(f, 0.0f);
  if (FN == kFnHswishA) return f * fminf(fmaxf(f + 3.0f, 0.0f), 6.0f) / 6.0f;
  if (FN == kFnHsigmoid) return fminf(fmaxf(f + 3.0f, 0.0f), 6.0f) / 6.0f;
  if (FN == kFnSigmoid) return 1.0f / (1.0f + expf(-f));
  if (FN == kFnHswishB) return f * (fminf(fmaxf(f + 3.0f, 0.0f), 6.0f) / 6.0f);
  return f;
}

// SiLU through the MUFU exp2 and reciprocal.  Relative error below 2^-19
// wherever the result is a normal fp16 value (f > -12.2, so |t| < 18; the
// rounding of -f*log2(e) dominates); below that the result lies in the fp16
// subnormal range, where the same relative error is far below the spacing.
__device__ __forceinline__ float silu_fast(float f) {
  const float t = -f * 1.4426950408889634f;
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
  const float d = 1.0f + e;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return f * r;
}

// Reference epilogue for 8 consecutive output channels of one pixel:
// half(half(acc) + bias) -> act (f32) -> half.  The half additions are packed
// f16x2 operations (correctly rounded, like the reference's half arithmetic).
// SiLU uses the MUFU exp2/reciprocal form (relative error below 2^-19, so the
// fp16 result is the correctly rounded one or its neighbour, like the
// reference's own relaxed-math exp); the other activations use the reference
// expression.
template <int FN>
__device__ __forceinline__ uint4 epilogue8(const uint32_t (&acc)[8], uint4 bias8) {
  const __half2 *hb = reinterpret_cast<const __half2 *>(&bias8);
  uint4 out;
  __half2 *ho = reinterpret_cast<__half2 *>(&out);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __half2 h = __hadd2(__floats2half2_rn(__uint_as_float(acc[2 * k]), __uint_as_float(acc[2 * k + 1])), hb[k]);
    const float2 f = __half22float2(h);
    const float y0 = FN == kFnSilu ? silu_fast(f.x) : act_exact<FN>(f.x);
    const float y1 = FN == kFnSilu ? silu_fast(f.y) : act_exact<FN>(f.y);
    ho[k] = __floats2half2_rn(y0, y1);
  }
  return out;
}

// One lane of the (converged) warp is elected; the others get false.  Roles
// that issue tcgen05 / TMA work run their loops on the whole warp and issue
// from the elected lane, so loop values stay warp-uniform (a loop run by one
// divergent lane issues small MMAs at about half the rate).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .pred P;\n elect.sync _|P, 0xffffffff;\n selp.u32 %0, 1, 0, P;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

// ------------------------------------------------------------------ smem/mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or `ns` nanoseconds pass, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait without a suspend hint: a short poll for waits expected to end
// within microseconds (one waiter per CTA; the others wait at a barrier).
__device__ __forceinline__ bool mbar_wait_poll(uint32_t bar, uint32_t parity, long long limit_cycles) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > limit_cycles) return false;
  return true;
}

// Error codes a kernel writes to its status word (first error wins).
enum KernelStatus : int {
  kStatusOk = 0,
  kStatusTimeoutFull = 1,
  kStatusTimeoutEmpty = 2,
  kStatusTimeoutAcc = 3,
  kStatusTimeoutAccEmpty = 4,
  kStatusTimeoutDrain = 5,
  kStatusBadConfig = 6,
  kStatusTimeoutProbe = 7,  // the test probe's wait (a barrier nothing arrives on) ran out
};

// Default limit of a conv kernel's working waits, in SM clocks (about 2 s).
constexpr long long kConvWaitLimitDefault = 4000000000LL;

// Bounded wait: gives up after ~`limit_cycles` SM clocks, records `code` in the
// global status word and raises the CTA-wide abort flag so the other roles stop.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                                  int *status, int code,
                                                  long long limit_cycles = 4000000000LL) {
  // The thread sleeps inside try_wait (woken when the phase completes) rather
  // than spinning, so idle roles do not take issue slots from working warps.
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > limit_cycles) {
      *abort_flag = 1;
      if (status) atomicCAS(status, 0, code);
      return false;
    }
  }
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const void *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void *map, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 in, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all prior tcgen05.mma of this thread have completed.
// Same MMA with the descriptors passed as (low, high) words: the low word holds
// the start address (>> 4) and the leading byte offset, so an operand offset is
// one 32-bit add on the low word (the start field never carries: shared memory
// addresses stay below 2^18).
__device__ __forceinline__ void umma_f16_lh(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                            uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
      "mov.b64 ad, {%1, %2};\n\t"
      "mov.b64 bd, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 32 bit, 8 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major operand with a swizzled canonical
// layout: rows of `row_bytes` (= swizzle span 32/64/128 B), 8-row groups
// `8*row_bytes` apart (stride byte offset); version field 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t saddr, uint32_t row_bytes) {
  uint32_t layout;
  switch (row_bytes) {
    case 128: layout = 2; break;  // SWIZZLE_128B
    case 64: layout = 4; break;   // SWIZZLE_64B
    default: layout = 6; break;   // SWIZZLE_32B
  }
  const uint64_t start = (saddr & 0x3FFFFu) >> 4;
  const uint64_t lbo = 1;                         // ignored for swizzled K-major
  const uint64_t sbo = (8u * row_bytes) >> 4;     // 8-row group stride
  return start | (lbo << 16) | (sbo << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Same layout with an explicit 8-row group stride and a start anywhere on a
// 16-byte boundary of the operand (the 3x3 halo tile: a tap is a start offset
// of whole rows).  `base_off` is the descriptor's matrix base offset field; the
// MMA applies the swizzle to absolute shared-memory address bits, as TMA does
// when it writes the tile, so shifted starts keep base_off = 0 (checked by the
// conv3x3 parity tests: a phase-derived base offset gives wrong results).
__device__ __forceinline__ uint64_t smem_desc_kmajor_at(uint32_t saddr, uint32_t row_bytes, uint32_t sbo_bytes,
                                                       uint32_t base_off) {
  uint32_t layout;
  switch (row_bytes) {
    case 128: layout = 2; break;
    case 64: layout = 4; break;
    default: layout = 6; break;
  }
  const uint64_t start = (saddr & 0x3FFFFu) >> 4;
  const uint64_t sbo = sbo_bytes >> 4;
  return start | (1ull << 16) | (sbo << 32) | (1ull << 46) | ((uint64_t)(base_off & 7u) << 49) |
         ((uint64_t)layout << 61);
}

// Instruction descriptor, kind::f16: D f32, A/B f16, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4)                       // D format f32
         | (0u << 7) | (0u << 10)        // A, B f16
         | (0u << 15) | (0u << 16)       // K-major A and B
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

}  // namespace ivb
