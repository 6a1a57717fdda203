// Pose decode + greedy NMS on the device: the reference's PoseDecoder::decode
// (src/Decoders.cpp:127-179) with nmsPerClass (:33-65, one class) and nms /
// iou (src/Nms.cpp:10-55), one CTA per image over the [5 + nk * kdims, A]
// channel-major fp16 output.
//
// pose_nms_k, per image:
//   1. candidates: anchors whose score is not below `conf` (`score < conf`
//      skips, as in the reference);
//   2. the candidates in descending score, ties by anchor index (the
//      reference's stable sort): a 30-bit key per anchor (the fp16 score's
//      order inverted, then the anchor) bitonic-sorted in shared memory;
//   3. each candidate's box (x, y, w, h) in image coordinates through the
//      letterbox (rectToImage), in shared memory when keys, boxes and flags
//      fit there (A <= 9,800 or so), else in global scratch;
//   4. greedy suppression in that order (IoU above `iou` removes a later
//      candidate) over every candidate: a candidate is tested against the
//      boxes kept so far, 64 candidates at a time;
//   5. the keep list (anchor, score) in keep order.
// The reference then re-sorts the keep list by score with std::sort, which is
// not stable, and cuts it at max_det; the host does that step with the same
// std::sort on the same sequence (Engine::decode_pose), and pose_gather_k
// writes the chosen detections' rows.
// All float arithmetic is the reference's, operation by operation, with
// round-to-nearest intrinsics so that nothing is contracted into an FMA.
#include <cuda_fp16.h>

#include "common.cuh"
#include "ops.cuh"

namespace ivb {

namespace {

// One output value as f32: the fp16 output tensor, or its exact f32 copy that
// ClBackend::infer's chunked paths leave for the whole batch.
struct PoseOut {
  const void *p;
  int f32;
  __device__ __forceinline__ float operator[](long long i) const {
    return f32 ? static_cast<const float *>(p)[i] : __half2float(static_cast<const __half *>(p)[i]);
  }
  __device__ __forceinline__ PoseOut image(long long b, long long stride) const {
    PoseOut r = *this;
    r.p = f32 ? (const void *)(static_cast<const float *>(p) + b * stride)
              : (const void *)(static_cast<const __half *>(p) + b * stride);
    return r;
  }
};

__device__ __forceinline__ float4 pose_box(const PoseOut &o, long long A, int a, float scale, float pl, float pt) {
  const float cx = o[a], cy = o[A + a];
  const float w = o[2 * A + a], h = o[3 * A + a];
  const float x = __fdiv_rn(__fsub_rn(cx, pl), scale), y = __fdiv_rn(__fsub_rn(cy, pt), scale);
  const float ws = __fdiv_rn(w, scale), hs = __fdiv_rn(h, scale);
  return make_float4(__fsub_rn(x, __fdiv_rn(ws, 2.0f)), __fsub_rn(y, __fdiv_rn(hs, 2.0f)), ws, hs);
}

__device__ __forceinline__ float box_iou(float4 a, float4 b) {
  const float x1 = fmaxf(a.x, b.x), y1 = fmaxf(a.y, b.y);
  const float x2 = fminf(__fadd_rn(a.x, a.z), __fadd_rn(b.x, b.z));
  const float y2 = fminf(__fadd_rn(a.y, a.w), __fadd_rn(b.y, b.w));
  const float inter = __fmul_rn(fmaxf(0.0f, __fsub_rn(x2, x1)), fmaxf(0.0f, __fsub_rn(y2, y1)));
  const float area_a = __fmul_rn(fmaxf(0.0f, a.z), fmaxf(0.0f, a.w));
  const float area_b = __fmul_rn(fmaxf(0.0f, b.z), fmaxf(0.0f, b.w));
  const float uni = __fsub_rn(__fadd_rn(area_a, area_b), inter);
  return uni > 1e-9f ? __fdiv_rn(inter, uni) : 0.0f;
}

__global__ void __launch_bounds__(kPoseNmsThreads) pose_nms_k(PoseNmsArgs p) {
  pdl_wait_and_release();
  extern __shared__ uint32_t nms_sm[];
  // shared memory: P sort keys, then the boxes (A, when they fit), then the
  // kept candidates' indices (up to A, when they fit)
  uint32_t *key = nms_sm;
  float4 *bx = p.boxes_in_smem ? reinterpret_cast<float4 *>(nms_sm + p.P) : p.boxes + (long long)blockIdx.x * p.P;
  int *kept_sm = reinterpret_cast<int *>(reinterpret_cast<unsigned char *>(nms_sm + p.P) +
                                         (p.boxes_in_smem ? (size_t)p.A * sizeof(float4) : 0));
  __shared__ int n_cand;
  const int b = blockIdx.x, tid = threadIdx.x;
  const long long A = p.A;
  const PoseOut o = PoseOut{p.out, p.out_f32}.image(b, p.img_stride);
  const float scale = p.letterbox ? p.letterbox[3 * b] : 1.0f;
  const float pl = p.letterbox ? p.letterbox[3 * b + 1] : 0.0f, pt = p.letterbox ? p.letterbox[3 * b + 2] : 0.0f;
  if (tid == 0) n_cand = 0;
  __syncthreads();
  // 1. keys: the fp16 score mapped to an unsigned order (+0 and -0 alike),
  // inverted so that ascending keys run in descending score, then the anchor
  for (int a = tid; a < p.P; a += blockDim.x) {
    uint32_t k = 0xffffffffu;
    if (a < p.A) {
      const float fs = o[4 * A + a];
      if (!(fs < p.conf)) {
        // every output value is an fp16 value, so the score is exact in fp16
        uint32_t u = __half_as_ushort(__float2half_rn(fs));
        if ((u & 0x7fffu) == 0) u = 0;
        const uint32_t ord = (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u);
        k = ((0xffffu - ord) << 14) | (uint32_t)a;
        atomicAdd(&n_cand, 1);
      }
    }
    key[a] = k;
  }
  __syncthreads();
  // 2. bitonic sort, ascending (P is a power of two)
  for (int size = 2; size <= p.P; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = tid; t < p.P / 2; t += blockDim.x) {
        // lo = 2 * stride * (t / stride) + t % stride, stride a power of two
        const int lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
        const uint32_t x = key[lo], y = key[hi];
        if ((x > y) == ((lo & size) == 0)) {
          key[lo] = y;
          key[hi] = x;
        }
      }
      __syncthreads();
    }
  const int n = n_cand;
  // 3. boxes of the candidates in sorted order
  for (int i = tid; i < n; i += blockDim.x) bx[i] = pose_box(o, A, (int)(key[i] & 0x3fffu), scale, pl, pt);
  __syncthreads();
  // 4. greedy suppression.  A candidate is kept when no earlier kept box
  // overlaps it above `iou` (the reference's loop, which removes every later
  // candidate a kept box overlaps, decides the same).  Candidates go in groups
  // of 64, lane l holding group candidates l and l + 32: warp w tests kept
  // boxes w, w + 32, ... against the group, and group rows w and w + 32 (one
  // candidate against the later ones in the group); thread 0 then walks the
  // group in order with 64-bit masks.  Two barriers per group.
  __shared__ unsigned long long sup_mask, row_mask[64];
  __shared__ int n_kept;
  const int warp = tid >> 5, lane = tid & 31;
  int *kept_idx = p.kept_idx_smem ? kept_sm : p.kept + (long long)b * p.P;
  if (tid == 0) {
    n_kept = 0;
    sup_mask = 0ull;
  }
  __syncthreads();
  for (int base = 0; base < n; base += 64) {
    const int nk_now = n_kept;
    const int c0 = base + lane, c1 = base + 32 + lane;
    const bool v0 = c0 < n, v1 = c1 < n;
    const float4 b0 = v0 ? bx[c0] : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 b1 = v1 ? bx[c1] : make_float4(0.f, 0.f, 0.f, 0.f);
    bool h0 = false, h1 = false;
    for (int k = warp; k < nk_now && (v0 || v1); k += 32) {
      const float4 bk = bx[kept_idx[k]];
      h0 = h0 || (v0 && box_iou(bk, b0) > p.iou);
      h1 = h1 || (v1 && box_iou(bk, b1) > p.iou);
    }
    const unsigned long long sup = (unsigned long long)__ballot_sync(0xffffffffu, h0) |
                                   ((unsigned long long)__ballot_sync(0xffffffffu, h1) << 32);
    unsigned long long rows[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {  // group row r = warp + 32 q against group columns lane, lane + 32
      const int r = warp + 32 * q;
      const bool rv = base + r < n;
      const float4 br = rv ? bx[base + r] : make_float4(0.f, 0.f, 0.f, 0.f);
      const bool o0 = rv && v0 && lane > r && box_iou(br, b0) > p.iou;
      const bool o1 = rv && v1 && 32 + lane > r && box_iou(br, b1) > p.iou;
      rows[q] = (unsigned long long)__ballot_sync(0xffffffffu, o0) |
                ((unsigned long long)__ballot_sync(0xffffffffu, o1) << 32);
    }
    if (lane == 0) {
      if (sup) atomicOr(&sup_mask, sup);
      row_mask[warp] = rows[0];
      row_mask[warp + 32] = rows[1];
    }
    __syncthreads();
    if (tid == 0) {
      unsigned long long m = sup_mask;
      int nk = n_kept;
      for (int j = 0; j < 64 && base + j < n; ++j)
        if (!((m >> j) & 1ull)) {
          kept_idx[nk++] = base + j;
          m |= row_mask[j];
        }
      n_kept = nk;
      sup_mask = 0ull;  // for the next group (its ORs come after the next barrier)
    }
    __syncthreads();
  }
  // 5. the keep list in keep order: anchor and score (the score as the f32
  // value the reference's Detection holds)
  const int kept = n_kept;
  int2 *pairs = p.pairs + (long long)b * p.P;
  for (int k = tid; k < kept; k += blockDim.x) {
    const int a = (int)(key[kept_idx[k]] & 0x3fffu);
    pairs[k] = make_int2(a, __float_as_int(o[4 * A + a]));
  }
  if (tid == 0) p.counts[b] = kept;
}

// The rows of the detections the host chose (std::sort of the keep list by
// score, cut at max_det): anchor, score, box through the letterbox, keypoints.
__global__ void __launch_bounds__(256) pose_gather_k(PoseGatherArgs p) {
  pdl_wait_and_release();
  const int b = blockIdx.x;
  const long long A = p.A;
  const PoseOut o = PoseOut{p.out, p.out_f32}.image(b, p.img_stride);
  const float scale = p.letterbox ? p.letterbox[3 * b] : 1.0f;
  const float pl = p.letterbox ? p.letterbox[3 * b + 1] : 0.0f, pt = p.letterbox ? p.letterbox[3 * b + 2] : 0.0f;
  const int S = 6 + 2 * p.nk, count = p.counts[b];
  const int *anchors = p.anchors + (long long)b * p.max_det;
  float *dets = p.dets + (long long)b * p.max_det * S;
  for (long long e = threadIdx.x; e < (long long)count * S; e += blockDim.x) {
    const int k = (int)(e / S), f = (int)(e - (long long)k * S);
    const int a = anchors[k];
    float v;
    if (f == 0) v = (float)a;
    else if (f == 1) v = o[4 * A + a];
    else if (f < 6) {
      const float4 bi = pose_box(o, A, a, scale, pl, pt);
      v = f == 2 ? bi.x : f == 3 ? bi.y : f == 4 ? bi.z : bi.w;
    } else {
      const int kk = (f - 6) >> 1, xy = (f - 6) & 1;
      v = __fdiv_rn(__fsub_rn(o[(5 + (long long)kk * p.kdims + xy) * A + a], xy ? pt : pl), scale);
    }
    dets[e] = v;
  }
}

}  // namespace

cudaError_t launch_pose_nms(const PoseNmsArgs &args, int batch, cudaStream_t st) {
  if (args.P < 4 || args.P > kPoseNmsMaxAnchors || (args.P & (args.P - 1)) || args.A > args.P || args.A < 1 ||
      batch < 1)
    return cudaErrorInvalidValue;
  const size_t smem = pose_nms_smem_bytes(args.P, args.A, args.boxes_in_smem != 0, args.kept_idx_smem ? args.A : 0);
  if (smem > (size_t)kPoseNmsSmemMax) return cudaErrorInvalidValue;
  static std::atomic<bool> attr_set[kAttrMaxDevices];
  const cudaError_t e = ensure_dynamic_smem(pose_nms_k, kPoseNmsSmemMax, attr_set);
  if (e != cudaSuccess) return e;
  launch_kernel(pose_nms_k, dim3((unsigned)batch), dim3(kPoseNmsThreads), smem, st, args);
  return cudaGetLastError();
}

cudaError_t launch_pose_gather(const PoseGatherArgs &args, int batch, cudaStream_t st) {
  if (args.A < 1 || args.max_det < 1 || batch < 1) return cudaErrorInvalidValue;
  launch_kernel(pose_gather_k, dim3((unsigned)batch), dim3(256), 0, st, args);
  return cudaGetLastError();
}

}  // namespace ivb
