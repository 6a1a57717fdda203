// Host-visible declarations of the bandwidth-bound kernels (ops.cu).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <vector>

namespace ivb {

// A 4-D activation view: element (b, c, y, x) lives at ptr[b*sb + c*sc + y*sy + x*sx].
// NHWC: sc = 1, sx = Cs, sy = W*Cs, sb = H*W*Cs.  Planar NCHW: sx = 1, sy = W,
// sc = H*W, sb = C*H*W.  A stride of 0 broadcasts that dimension.
struct View4 {
  __half *ptr;
  int C, H, W;
  long long sb, sc, sy, sx;
};

constexpr int kMaxRank = 8;

struct BcastArgs {          // rank-generic broadcast binary op (planar operands)
  int rank;
  long long dims[kMaxRank];  // output dims, dims[0] = batch
  long long as[kMaxRank], bs[kMaxRank];
};

cudaError_t launch_ew_binary_flat(const __half *a, const __half *b, __half *y, long long n, int op, int b_scalar,
                                  long long per_img, int batch, long long a_bstride, long long b_bstride,
                                  cudaStream_t st);
cudaError_t launch_ew_binary_v4(View4 a, View4 b, View4 y, int batch, int op, cudaStream_t st);
cudaError_t launch_ew_binary_bcast(const __half *a, const __half *b, __half *y, const BcastArgs &args, int op,
                                   cudaStream_t st);
cudaError_t launch_ew_unary_flat(const __half *x, __half *y, long long n, int op, cudaStream_t st);
cudaError_t launch_ew_unary_v4(View4 x, View4 y, int batch, int op, cudaStream_t st);
cudaError_t launch_copy_v4(View4 x, View4 y, int batch, cudaStream_t st);
cudaError_t launch_slice_axis(const __half *x, __half *y, long long outer, int axdim, long long inner, int start,
                              int len, cudaStream_t st);
struct ConcatSrc {
  const __half *ptr;
  int c;           // extent along the concat axis
  int shared;      // 1: initializer (same data for every image)
};
cudaError_t launch_concat_planar(const ConcatSrc *src, int nsrc, __half *y, long long outer, long long per_img_outer,
                                 long long inner, cudaStream_t st);
cudaError_t launch_maxpool_v4(View4 x, View4 y, int batch, int K, int S, int P, cudaStream_t st);
cudaError_t launch_resize_nn_v4(View4 x, View4 y, int batch, int S, cudaStream_t st);
// `levels` (<= 3) chained KxK stride-1 pools: ys[l] = pool(level l-1), level -1
// being x (the SPPF chain), fused in one kernel when the plane fits shared memory.
cudaError_t launch_maxpool_chain_v4(View4 x, const View4 *ys, int levels, int batch, int K, int P,
                                    cudaStream_t st);
cudaError_t launch_softmax_axis(const __half *x, __half *y, long long outer, int axdim, long long inner,
                                cudaStream_t st);
cudaError_t launch_permute_0213(const __half *x, __half *y, int batch, int D1, int D2, long long I, int mode,
                                cudaStream_t st);
cudaError_t launch_gap_v4(View4 x, __half *y, int batch, cudaStream_t st);
cudaError_t launch_bmm(const __half *A, const __half *B, __half *Y, int batch, int B1, int M, int K, int N,
                       long long a_bstride, long long b_bstride, cudaStream_t st);
// ta / tb: A stored as [K][M], B as [N][K] (a folded transposing permute)
cudaError_t launch_bmm_t(const __half *A, const __half *B, __half *Y, int batch, int B1, int M, int K, int N,
                         long long a_bstride, long long b_bstride, int ta, int tb, cudaStream_t st);
cudaError_t launch_bias_add(const __half *x, const __half *b, __half *y, long long per_img, int HW, int batch,
                            cudaStream_t st);

// Depthwise KxK (groups == C), reference depthwise_f16 epilogue.
cudaError_t launch_depthwise_v4(View4 x, const __half *w, const __half *bias, View4 y, int batch, int K, int S,
                                int P, int act, cudaStream_t st);
// Direct CUDA-core convolution over views (any K/S/P/G).  epi: 0 = conv_general
// (fp32 accumulator starting at bias, activation on f32, codes 2=HardSwish
// 3=ReLU), 1 = gemm-family rounding, 2 = conv3x3 rounding.
cudaError_t launch_conv_direct_v4(View4 x, const __half *w, const __half *bias, const __half *res_ptr, View4 res,
                                  View4 y, int batch, int Cout, int K, int S, int P, int G, int act, int epi,
                                  cudaStream_t st);
// Stem: 3x3 conv with Cin <= 4 (tiny K), conv3x3 rounding, NHWC or planar output.
// `blob` (from stem_params, host memory: Cin 3 -> Cout 16 weights packed as
// K-major rows) selects the tensor-core kernel (stride 1 or 2, pad 1; `status`
// receives a bounded-wait timeout); without it the generic CUDA-core kernel
// reads `w` / `bias` on the device.
bool stem_params(int cin, int cout, const uint16_t *w_host, const uint16_t *b_host, std::vector<float> *blob);
cudaError_t launch_stem3x3_v4(View4 x, const __half *w, const __half *bias, const float *blob, View4 y, int batch,
                              int Cout, int S, int P, int act, int *status, cudaStream_t st);
// 1x1 conv over planar [Cin][N] rows with few outputs (Cin <= 64, Cout <= 8),
// gemm-family rounding, fp32 accumulation over ci in order.
// ---- fused planar tail: a region of slice / concat / elementwise / reshape
// nodes (plus the DFL chain) whose tensors all keep the anchor axis (A) as the
// innermost dimension, compiled at load time into a straight-line program per
// anchor column.  Every op's result is rounded to fp16 like the node it
// replaces.  Operands are slots (earlier results, in shared memory
// [slot][thread]), rows of leaf tensors read directly, or immediates; an op may
// also write its result to a row of the output.
constexpr int kTailMaxOps = 400;
constexpr int kTailMaxLeaves = 8;
constexpr int kTailMaxDfl = 2;
constexpr int kTailMaxSlots = 40;
constexpr int kTailMaxComp = 64;  // independent op chains (one per blockIdx.y)
enum TailOpCode : int {
  kTailBin = 0,   // half(binop(a, b, arg))
  kTailUn = 1,    // half(unop(a, arg))
  kTailDfl = 2,   // DFL of leaf a.idx, rows a.row .. +15, table arg
  kTailCopy = 3,  // a
};
enum TailOperandKind : int { kTailSlot = 0, kTailLeafRow = 1, kTailImm = 2 };
struct TailOperand {
  int kind, idx, row;  // slot: idx; leaf row: leaf idx, row; immediate: float bits in idx
};
struct TailOp {
  int code, dst, store_row, arg;  // dst: slot or -1; store_row: output row or -1
  TailOperand a, b;
};
struct TailLeaf {
  const __half *ptr;
  long long img_stride, row_stride;
};
struct TailDfl {
  float w[16];
  float bias;
  int act;
};
struct TailProgram {
  int n_ops = 0, n_slots = 0, n_leaves = 0, n_dfl = 0;
  int n_comp = 0;
  int comp_begin[kTailMaxComp + 1];  // ops of chain c: [comp_begin[c], comp_begin[c + 1])
  long long A = 0, out_img = 0;
  __half *out = nullptr;
  TailLeaf leaves[kTailMaxLeaves];
  TailDfl dfl[kTailMaxDfl];
  TailOp ops[kTailMaxOps];
};
cudaError_t launch_tail_program(const TailProgram &prog, int batch, cudaStream_t st);

// permute_0213 (mode 0) -> softmax over D2 bins -> 1x1 conv D2 -> Cout, fused
// (the YOLO DFL head).  Supported for D2 == 16 and Cout <= 8.
// Pose decode + greedy NMS over a batch of channel-major fp16 pose outputs
// [5 + nk * kdims, A] (pose_nms.cu); one CTA per image.  pose_nms_k writes each
// image's keep list; the host orders and cuts it like the reference, and
// pose_gather_k writes the chosen detections' rows.
constexpr int kPoseNmsThreads = 1024;
constexpr int kPoseNmsMaxAnchors = 16384;  // P: the sort runs over a power of two >= A, in shared memory
struct PoseNmsArgs {
  const void *out;         // image 0 of the output: fp16, or its exact f32 copy (out_f32)
  int out_f32;
  long long img_stride;    // elements
  int A;                   // anchors
  int P;                   // power of two >= A (sort length)
  int nk, kdims;           // keypoints, values per keypoint
  float conf, iou;
  const float *letterbox;  // [batch][scale, pad_left, pad_top] or null (scale 1, no padding)
  float4 *boxes;           // scratch [batch][P] (used when the boxes do not fit in shared memory)
  int boxes_in_smem;       // 1: boxes in shared memory (pose_nms_smem_bytes(P, A, true) <= kPoseNmsSmemMax)
  int *kept;               // scratch [batch][P] (used when the kept list does not fit in shared memory)
  int kept_idx_smem;       // 1: kept list in shared memory
  int *counts;             // [batch]: kept candidates
  int2 *pairs;             // [batch][P]: the keep list in keep order, (anchor, score as f32 bits)
};
struct PoseGatherArgs {
  const void *out;         // as PoseNmsArgs
  int out_f32;
  long long img_stride;
  int A, nk, kdims, max_det;
  const float *letterbox;  // as PoseNmsArgs
  const int *counts;       // [batch]: detections chosen per image (<= max_det)
  const int *anchors;      // [batch][max_det]: their anchors, in output order
  float *dets;             // [batch][max_det][6 + 2 * nk]: anchor, score, x, y, w, h, then (x, y) per keypoint
};
constexpr int kPoseNmsSmemMax = 225 * 1024;  // dynamic; the kernel's static shared memory (~1 KB) fits beside it
inline size_t pose_nms_smem_bytes(int P, int A, bool boxes_in_smem, int kept_in_smem) {
  return (size_t)P * 4 + (boxes_in_smem ? (size_t)A * 16 : 0) + (size_t)kept_in_smem * 4;  // keys, boxes, kept list
}
cudaError_t launch_pose_nms(const PoseNmsArgs &args, int batch, cudaStream_t st);
cudaError_t launch_pose_gather(const PoseGatherArgs &args, int batch, cudaStream_t st);

// Letterbox preprocessing of 8-bit BGR frames into the planar fp16 network
// input (preprocess.cu; the reference's Preprocessor::operator() + the
// truncating cast of ClBackend::infer).  The coordinate tables come from the
// host (OpenCV's INTER_LINEAR rules): xtab[dx] = {byte offset of tap 0, of
// tap 1, weight 0, weight 1}, ytab[dy] = {row 0, row 1, weight 0, weight 1},
// weights in 11-bit fixed point.
struct LetterboxArgs {
  const uint8_t *src;          // image 0 of the frames (HWC BGR)
  long long img_stride;        // bytes between frames
  long long row_stride;        // bytes between rows
  const int4 *xtab, *ytab;     // [rw], [rh]
  void *dst;                   // image 0 of the network input (fp16, [3][in_h][in_w])
  long long dst_img_stride;    // elements between images
  int in_h, in_w;              // the canvas (network input) size
  int rw, rh, pad_left, pad_top;  // the resized image inside the canvas
  int to_rgb, normalize, has_mean_std;
  float mean[3], std[3];
  int vec_store;               // destination rows 8-byte aligned (in_w % 4 == 0, aligned base)
};
cudaError_t launch_letterbox_bgr(const LetterboxArgs &args, int batch, cudaStream_t st);

bool dfl_fused_supported(int D2, int Cout);
cudaError_t launch_dfl_fused(const __half *x, const __half *w, const __half *bias, __half *y, int batch, int D1, int D2,
                             long long I, int Cout, int act, cudaStream_t st);
cudaError_t launch_conv1x1_planar(const __half *x, const __half *w, const __half *bias, __half *y, int batch,
                                  long long N, int Cin, int Cout, int act, cudaStream_t st);
// Reference host conversion on the device: f32 -> f16 by mantissa truncation.
cudaError_t launch_f32_to_f16_trunc(const float *x, __half *y, long long n, cudaStream_t st);
cudaError_t launch_f16_to_f32(const __half *x, float *y, long long n, cudaStream_t st);

}  // namespace ivb
