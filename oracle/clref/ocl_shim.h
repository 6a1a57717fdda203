// Minimal OpenCL-C -> C++ shim so that the reference's portable kernel sources
// (kernels/ops.cl, kernels/conv_general.cl, kernels/gemm.cl with SG=0) compile
// with g++ and run on the CPU.  TEST INFRASTRUCTURE ONLY: the resulting library
// (oracle/_ref/libclref.so) produces golden vectors that pin the oracle; the
// product never links it.
//
// Semantics: `half` is _Float16 compiled with -fexcess-precision=16, so every
// half operation is rounded to half as in OpenCL C; work-items run on host
// threads (harness.cpp), `__local` arrays become function statics shared by
// the threads of the one work-group in flight, barrier() is a thread barrier.
#pragma once
#include <cmath>
#include <cstddef>
#include <cstdint>

typedef _Float16 half;
typedef half half2 __attribute__((vector_size(4)));
typedef half half4 __attribute__((vector_size(8)));
typedef half half8 __attribute__((vector_size(16)));
typedef half half16 __attribute__((vector_size(32)));
typedef float float2 __attribute__((vector_size(8)));
typedef float float4 __attribute__((vector_size(16)));
typedef float float8 __attribute__((vector_size(32)));
typedef unsigned int uint;
typedef unsigned short ushort;
typedef unsigned char uchar;

#define __kernel extern "C"
#define __global
#define __local static
#define __constant const
#define __private
#define restrict __restrict__
#define CLK_LOCAL_MEM_FENCE 1
#define CLK_GLOBAL_MEM_FENCE 2

extern "C" {
size_t get_global_id(uint d);
size_t get_local_id(uint d);
size_t get_group_id(uint d);
size_t get_global_size(uint d);
size_t get_local_size(uint d);
size_t get_num_groups(uint d);
void barrier(int flags);
}

// OpenCL built-ins used by the compiled sources
static inline half mad(half a, half b, half c) { return (half)((float)a * (float)b + (float)c); }
static inline float mad(float a, float b, float c) { return a * b + c; }
static inline float clamp(float x, float lo, float hi) { return std::fmin(std::fmax(x, lo), hi); }

// ---- additions for kernels/gemm.cl and kernels/conv_ov.cl (compiled after the
// source pre-pass clref/prepass.sed, which turns `(half2)(a, b)` literals into
// brace initialisers, `.s0` / `.s1` into subscripts, work-group arrays into
// IVB_GROUP_ARRAY statics and drops `__local` from pointer declarations and casts)
#define IVB_GROUP_ARRAY static __attribute__((aligned(64)))
typedef ushort ushort2 __attribute__((vector_size(4)));

static inline half2 mad(half2 a, half2 b, half2 c) {
  half2 r;
  r[0] = mad(a[0], b[0], c[0]);
  r[1] = mad(a[1], b[1], c[1]);
  return r;
}
static inline half2 as_half2(ushort2 u) {
  half2 h;
  __builtin_memcpy(&h, &u, sizeof(h));
  return h;
}
// Sub-groups (harness.cpp): the work-items of a work-group form sub-groups of
// clref_set_sub_group_size() consecutive linear local ids; a broadcast is an
// exchange through a group-shared slot between two barriers.
uint get_sub_group_local_id();
uint get_sub_group_id();
half sub_group_broadcast(half v, uint lane);
ushort2 intel_sub_group_block_read_us2(const ushort *p);
