// Device image preprocessing: the reference's Preprocessor::operator()
// (src/Preprocess.cpp:13-77) and the truncating f32 -> f16 cast of
// ClBackend::infer (include/infvino/Half.hpp:14-24), fused into one pass that
// writes the network's planar fp16 input.
//
// Per output pixel of the in_h x in_w canvas: inside the letterboxed image,
// the bilinear sample of the 8-bit BGR frame with OpenCV's INTER_LINEAR
// arithmetic for 8-bit images (11-bit fixed-point weights from the host's
// coordinate tables, int32 horizontal taps, then the vectorised vertical
// step ((b0 * (h0 >> 4)) >> 16) + ((b1 * (h1 >> 4)) >> 16) + 2) >> 2);
// outside it the border value 114; then blobFromImage's float(u8) * float(1/255)
// (optional), (v - mean) / std per channel (optional), channel order RGB or
// BGR, and the reference's truncating cast to fp16.  HBM-bound: every output
// value is written once with 8-byte stores (four pixels per thread per plane),
// the frame is read through L1/L2.
#include <cuda_fp16.h>

#include "common.cuh"
#include "ops.cuh"

namespace ivb {

namespace {

// include/infvino/Half.hpp:14-24: mantissa truncation, exp <= 0 -> +-0, exp >= 31 -> +-inf
__device__ __forceinline__ uint16_t f32_to_f16_trunc_bits(float f) {
  const uint32_t x = __float_as_uint(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int e = (int)((x >> 23) & 0xffu) - 112;
  if (e <= 0) return (uint16_t)sign;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | ((uint32_t)e << 10) | ((x >> 13) & 0x3ffu));
}

__device__ __forceinline__ int resize_tap(const uint8_t *r0, const uint8_t *r1, int4 xt, int b0, int b1, int c) {
  const int h0 = (int)r0[xt.x + c] * xt.z + (int)r0[xt.y + c] * xt.w;
  const int h1 = (int)r1[xt.x + c] * xt.z + (int)r1[xt.y + c] * xt.w;
  const int v = (((b0 * (h0 >> 4)) >> 16) + ((b1 * (h1 >> 4)) >> 16) + 2) >> 2;
  return v < 0 ? 0 : v > 255 ? 255 : v;
}

__global__ void __launch_bounds__(256) letterbox_bgr_k(LetterboxArgs p) {
  pdl_wait_and_release();
  const int b = blockIdx.z;
  const int oy = blockIdx.y * blockDim.y + threadIdx.y;
  const int ox0 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (oy >= p.in_h || ox0 >= p.in_w) return;
  const uint8_t *img = p.src + (long long)b * p.img_stride;
  const int dy = oy - p.pad_top;
  const bool row_in = dy >= 0 && dy < p.rh;
  int4 yt = make_int4(0, 0, 0, 0);
  if (row_in) yt = p.ytab[dy];
  const uint8_t *r0 = img + (long long)yt.x * p.row_stride, *r1 = img + (long long)yt.y * p.row_stride;
  uint16_t out[3][4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int ox = ox0 + k, dx = ox - p.pad_left;
    int bgr[3] = {114, 114, 114};
    if (row_in && ox < p.in_w && dx >= 0 && dx < p.rw) {
      const int4 xt = p.xtab[dx];  // byte offsets of the two taps, their weights
#pragma unroll
      for (int c = 0; c < 3; ++c) bgr[c] = resize_tap(r0, r1, xt, yt.z, yt.w, c);
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float v = (float)bgr[p.to_rgb ? 2 - c : c];
      if (p.normalize) v = __fmul_rn(v, 1.0f / 255.0f);
      if (p.has_mean_std) v = __fdiv_rn(__fsub_rn(v, p.mean[c]), p.std[c]);
      out[c][k] = f32_to_f16_trunc_bits(v);
    }
  }
  const long long plane = (long long)p.in_h * p.in_w;
  uint16_t *dst = reinterpret_cast<uint16_t *>(p.dst) + (long long)b * p.dst_img_stride + (long long)oy * p.in_w + ox0;
  if (p.vec_store && ox0 + 4 <= p.in_w) {
#pragma unroll
    for (int c = 0; c < 3; ++c)
      *reinterpret_cast<uint2 *>(dst + c * plane) =
          make_uint2((uint32_t)out[c][0] | ((uint32_t)out[c][1] << 16), (uint32_t)out[c][2] | ((uint32_t)out[c][3] << 16));
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (ox0 + k < p.in_w)
#pragma unroll
        for (int c = 0; c < 3; ++c) dst[c * plane + k] = out[c][k];
  }
}

}  // namespace

cudaError_t launch_letterbox_bgr(const LetterboxArgs &args, int batch, cudaStream_t st) {
  if (batch < 1 || args.in_h < 1 || args.in_w < 1 || args.rw < 1 || args.rh < 1 || args.rw > args.in_w ||
      args.rh > args.in_h || args.pad_left < 0 || args.pad_top < 0 || args.pad_left + args.rw > args.in_w ||
      args.pad_top + args.rh > args.in_h)
    return cudaErrorInvalidValue;
  const dim3 block(64, 4);
  const dim3 grid((unsigned)((args.in_w + 4 * 64 - 1) / (4 * 64)), (unsigned)((args.in_h + 3) / 4), (unsigned)batch);
  launch_kernel(letterbox_bgr_k, grid, block, 0, st, args);
  return cudaGetLastError();
}

}  // namespace ivb
