// Load-time compilation of the fused planar tail (TailProgram) into one
// straight-line CUDA kernel: NVRTC (loaded at run time) turns generated CUDA C
// into an sm_100a cubin, the driver API loads and launches it.  The generated
// code performs the same operations with the same fp16 rounding points as the
// interpreting kernel (tail_vm_k), which remains the path when NVRTC or the
// driver entry points are unavailable.
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "kernels/ops.cuh"

namespace ivb {

// Shape facts the generated code bakes in (known once tensors are laid out).
struct TailJitLayout {
  long long A = 0;                       // anchors per row
  long long out_img = 0;                 // output image stride (elements)
  long long leaf_img[kTailMaxLeaves] = {};  // leaf image strides (0: shared initializer)
  long long leaf_row[kTailMaxLeaves] = {};  // leaf row strides
  int V = 1;                             // anchors per thread (1, 2 or 4)
};

// The kernel's work split: the program's independent op chains in groups,
// each group a range of blocks with its own anchors per thread.
constexpr int kTailJitLightGroups = 4;
constexpr int kTailJitMaxGroups = 32;
struct TailJitGroup {
  std::vector<int> chains;
  int V = 1;
};
std::vector<TailJitGroup> tail_jit_groups(const TailProgram &prog, const TailJitLayout &lay);

// CUDA C source of the kernel `ivb_tail` for `prog`.
std::string tail_jit_source(const TailProgram &prog, const TailJitLayout &lay);

class TailJit {
 public:
  TailJit() = default;
  TailJit(const TailJit &) = delete;
  TailJit &operator=(const TailJit &) = delete;
  ~TailJit();
  // Compiles and (with `load`) loads the kernel on the current device; false
  // (with the reason) when NVRTC, the driver entry points or the compile fail.
  bool build(const TailProgram &prog, const TailJitLayout &lay, bool load, std::string *err);
  bool ready() const { return fn_ != nullptr; }
  // Runs the kernel over `batch` images with the program's current pointers.
  cudaError_t launch(const TailProgram &prog, int batch, bool pdl, cudaStream_t st) const;

 private:
  void *module_ = nullptr;
  void *fn_ = nullptr;
  TailJitLayout lay_{};
  int n_leaves_ = 0;
  std::vector<int> group_v_;  // anchors per thread of each group
};


}  // namespace ivb
