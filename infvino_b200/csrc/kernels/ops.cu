// Bandwidth-bound kernels of the plan executor (CUDA cores, no tensor cores):
// elementwise / broadcast, layout copies, concat, slice, maxpool, nearest
// resize, softmax, permute, global average pool, batched matmul, depthwise and
// direct convolutions, the Cin<=4 stem, and the f32<->f16 conversions.
//
// Arithmetic follows the reference kernels (kernels/ops.cl, kernels/conv_general.cl):
// inputs are widened to f32, the op is evaluated in f32 and rounded once to fp16.
// 4-D operands are strided views so one kernel serves NHWC and planar tensors.
#include <algorithm>
#include <vector>
#include <cstring>

#include "common.cuh"
#include "ops.cuh"
#include "../tma.h"

namespace ivb {

thread_local bool g_launch_pdl = true;

namespace {

constexpr int kThreads = 256;

inline int grid_for(long long n, int threads = kThreads) {
  long long g = (n + threads - 1) / threads;
  if (g > 148LL * 64) g = 148LL * 64;  // grid-stride loops beyond this
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

__device__ __forceinline__ float binop(float a, float b, int op) {
  if (op == 0) return a + b;
  if (op == 1) return a - b;
  if (op == 2) return a * b;
  return a / b;
}

// ew_unary codes (kernels/ops.cl:49-62): 0=sigmoid 1=silu 2=relu 3=hswish 4=hsigmoid
__device__ __forceinline__ float unop(float v, int op) {
  if (op == 0) return 1.0f / (1.0f + expf(-v));
  if (op == 1) return v / (1.0f + expf(-v));
  if (op == 2) return fmaxf(v, 0.0f);
  if (op == 3) return v * fminf(fmaxf(v + 3.0f, 0.0f), 6.0f) / 6.0f;
  if (op == 4) return fminf(fmaxf(v + 3.0f, 0.0f), 6.0f) / 6.0f;
  return v;
}

// decompose a linear index over (b, c, y, x) in the iteration order that makes
// the OUTPUT view coalesced: channel-fastest for NHWC, x-fastest otherwise.
struct Idx4 {
  long long b;
  int c, y, x;
};
__device__ __forceinline__ Idx4 idx4(long long i, const View4 &o, bool cfast) {
  Idx4 r;
  if (cfast) {
    r.c = (int)(i % o.C);
    long long t = i / o.C;
    r.x = (int)(t % o.W);
    t /= o.W;
    r.y = (int)(t % o.H);
    r.b = t / o.H;
  } else {
    r.x = (int)(i % o.W);
    long long t = i / o.W;
    r.y = (int)(t % o.H);
    t /= o.H;
    r.c = (int)(t % o.C);
    r.b = t / o.C;
  }
  return r;
}
__device__ __forceinline__ long long at(const View4 &v, const Idx4 &i) {
  return i.b * v.sb + (long long)i.c * v.sc + (long long)i.y * v.sy + (long long)i.x * v.sx;
}

// ------------------------------------------------------------------ elementwise
__global__ void ew_binary_flat_k(const __half *__restrict__ a, const __half *__restrict__ b, __half *__restrict__ y,
                                 long long n, int op, int b_scalar, long long per_img, long long a_bs,
                                 long long b_bs) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long img = i / per_img, r = i - img * per_img;
    const float av = __half2float(a[img * a_bs + r]);
    const float bv = __half2float(b_scalar ? b[img * b_bs] : b[img * b_bs + r]);
    y[i] = __float2half_rn(binop(av, bv, op));
  }
}

__global__ void ew_binary_v4_k(View4 a, View4 b, View4 y, long long n, int op, bool cfast) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const Idx4 ix = idx4(i, y, cfast);
    const float av = __half2float(a.ptr[at(a, ix)]);
    const float bv = __half2float(b.ptr[at(b, ix)]);
    y.ptr[at(y, ix)] = __float2half_rn(binop(av, bv, op));
  }
}

__global__ void ew_binary_bcast_k(const __half *__restrict__ a, const __half *__restrict__ b, __half *__restrict__ y,
                                  BcastArgs g, long long n, int op) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long rem = i, ai = 0, bi = 0;
    for (int r = g.rank - 1; r >= 0; --r) {
      const long long coord = rem % g.dims[r];
      rem /= g.dims[r];
      ai += coord * g.as[r];
      bi += coord * g.bs[r];
    }
    y[i] = __float2half_rn(binop(__half2float(a[ai]), __half2float(b[bi]), op));
  }
}

__global__ void ew_unary_flat_k(const __half *__restrict__ x, __half *__restrict__ y, long long n, int op) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(unop(__half2float(x[i]), op));
}

__global__ void ew_unary_v4_k(View4 x, View4 y, long long n, int op, bool cfast) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const Idx4 ix = idx4(i, y, cfast);
    y.ptr[at(y, ix)] = __float2half_rn(unop(__half2float(x.ptr[at(x, ix)]), op));
  }
}

__global__ void copy_v4_k(View4 x, View4 y, long long n, bool cfast) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const Idx4 ix = idx4(i, y, cfast);
    y.ptr[at(y, ix)] = x.ptr[at(x, ix)];
  }
}

// ------------------------------------------------------------------ layout ops
__global__ void slice_axis_k(const __half *__restrict__ x, __half *__restrict__ y, long long outer, int axdim,
                             long long inner, int start, int len) {
  pdl_wait_and_release();
  const long long n = outer * len * inner;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long o = i / ((long long)len * inner), rem = i - o * ((long long)len * inner);
    y[i] = x[(o * axdim + start) * inner + rem];
  }
}

struct ConcatArgs {
  ConcatSrc s[4];
  int nsrc;
  int sum;
};

__global__ void maxpool_v4_k(View4 x, View4 y, long long n, int K, int S, int P, bool cfast) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const Idx4 o = idx4(i, y, cfast);
    float m = -3.4e38f;
    for (int kh = 0; kh < K; ++kh) {
      const int yy = o.y * S - P + kh;
      if (yy < 0 || yy >= x.H) continue;
      for (int kw = 0; kw < K; ++kw) {
        const int xx = o.x * S - P + kw;
        if (xx < 0 || xx >= x.W) continue;
        m = fmaxf(m, __half2float(x.ptr[o.b * x.sb + (long long)o.c * x.sc + (long long)yy * x.sy + (long long)xx * x.sx]));
      }
    }
    y.ptr[at(y, o)] = __float2half_rn(m);
  }
}

__global__ void resize_nn_v4_k(View4 x, View4 y, long long n, int S, bool cfast) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const Idx4 o = idx4(i, y, cfast);
    y.ptr[at(y, o)] = x.ptr[o.b * x.sb + (long long)o.c * x.sc + (long long)(o.y / S) * x.sy + (long long)(o.x / S) * x.sx];
  }
}

// serial softmax over the axis, one thread per (outer, inner) column (ops.cl:181-196)
__global__ void softmax_axis_k(const __half *__restrict__ x, __half *__restrict__ y, long long outer, int axdim,
                               long long inner) {
  pdl_wait_and_release();
  const long long n = outer * inner;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long o = i / inner, r = i - o * inner;
    const __half *xp = x + o * axdim * inner + r;
    __half *yp = y + o * axdim * inner + r;
    float m = -3.4e38f;
    for (int a = 0; a < axdim; ++a) m = fmaxf(m, __half2float(xp[(long long)a * inner]));
    float s = 0.0f;
    for (int a = 0; a < axdim; ++a) s += expf(__half2float(xp[(long long)a * inner]) - m);
    for (int a = 0; a < axdim; ++a)
      yp[(long long)a * inner] = __float2half_rn(expf(__half2float(xp[(long long)a * inner]) - m) / s);
  }
}

// Softmax over the last axis (inner == 1), one warp per row, with softmax_axis_k's
// arithmetic: the max (order-free), expf(x - max) per element, their sum added
// in axis order by one lane, then each value over the sum, rounded once.
constexpr int kSoftmaxRowMax = 1024;
__global__ void __launch_bounds__(256) softmax_rows_k(const __half *__restrict__ x, __half *__restrict__ y,
                                                      long long rows, int axdim) {
  pdl_wait_and_release();
  __shared__ float e_sh[8][kSoftmaxRowMax];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float *e = e_sh[warp];
  for (long long r = (long long)blockIdx.x * 8 + warp; r < rows; r += (long long)gridDim.x * 8) {
    const __half *xr = x + r * axdim;
    __half *yr = y + r * axdim;
    float m = -3.4e38f;
    for (int a = lane; a < axdim; a += 32) m = fmaxf(m, __half2float(xr[a]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    for (int a = lane; a < axdim; a += 32) e[a] = expf(__half2float(xr[a]) - m);
    __syncwarp();
    float s = 0.0f;
    if (lane == 0) {
      int a = 0;
      for (; a + 8 <= axdim; a += 8) {  // loads ahead of the dependent adds
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = e[a + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) s += v[u];
      }
      for (; a < axdim; ++a) s += e[a];
    }
    s = __shfl_sync(0xffffffffu, s, 0);
    for (int a = lane; a < axdim; a += 32) yr[a] = __float2half_rn(e[a] / s);
    __syncwarp();  // e is rewritten by the next row
  }
}

__global__ void permute_0213_k(const __half *__restrict__ x, __half *__restrict__ y, long long n, int D1, int D2,
                               long long I, int mode) {
  pdl_wait_and_release();
  const long long per = (long long)D1 * D2 * I;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long img = i / per, j = i - img * per;
    const long long d1 = j / ((long long)D2 * I), rem = j - d1 * ((long long)D2 * I);
    const long long d2 = rem / I, r = rem - d2 * I;
    const long long o = (mode == 0) ? ((d2 * D1 + d1) * I + r) : ((d1 * I + r) * D2 + d2);
    y[img * per + o] = x[i];
  }
}

// global average pool: grid (batch, ceil(C/32)); 32 channels x 8 pixel lanes
__global__ void gap_v4_k(View4 x, __half *__restrict__ y) {
  pdl_wait_and_release();
  __shared__ float part[8][33];
  const int cl = threadIdx.x & 31, pl = threadIdx.x >> 5;
  const long long b = blockIdx.x;
  const int c = blockIdx.y * 32 + cl;
  const int HW = x.H * x.W;
  float acc = 0.0f;
  if (c < x.C) {
    for (int p = pl; p < HW; p += 8) {
      const int yy = p / x.W, xx = p - yy * x.W;
      acc += __half2float(x.ptr[b * x.sb + (long long)c * x.sc + (long long)yy * x.sy + (long long)xx * x.sx]);
    }
  }
  part[pl][cl] = acc;
  __syncthreads();
  if (pl == 0 && c < x.C) {
    float s = 0.0f;
    for (int k = 0; k < 8; ++k) s += part[k][cl];
    y[b * x.C + c] = __float2half_rn(s / (float)HW);
  }
}

// Global average pool of a channels-last tensor in the reference's summation
// order (kernels/ops.cl gap_r, GAP_WGS = 128): lane l of 128 sums pixels l,
// l + 128, ... in sequence, then a tree adds lane l + off into lane l for off =
// 64, 32, ..., 1, and the sum is divided by H*W.  One block of 128 threads per
// (image, 8-channel group); each lane keeps the 8 channels' sums.
__global__ void __launch_bounds__(128) gap_nhwc8_k(View4 x, __half *__restrict__ y, int nq) {
  pdl_wait_and_release();
  __shared__ float part[64][8];
  const int l = threadIdx.x;
  const int b = blockIdx.x / nq, q = blockIdx.x - b * nq;
  const int W = x.W, HW = x.H * x.W;
  const __half *base = x.ptr + (long long)b * x.sb + q * 8;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
  int p = l;
  // four loads in flight, added in pixel order
  for (; p + 3 * 128 < HW; p += 4 * 128) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int pp = p + u * 128, yy = pp / W, xx = pp - yy * W;
      v[u] = __ldg(reinterpret_cast<const uint4 *>(base + (long long)yy * x.sy + (long long)xx * x.sx));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const __half *h = reinterpret_cast<const __half *>(&v[u]);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += __half2float(h[e]);
    }
  }
  for (; p < HW; p += 128) {
    const int yy = p / W, xx = p - yy * W;
    const uint4 v = __ldg(reinterpret_cast<const uint4 *>(base + (long long)yy * x.sy + (long long)xx * x.sx));
    const __half *h = reinterpret_cast<const __half *>(&v);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += __half2float(h[e]);
  }
  // tree: off = 64 (lanes 64..127 into 0..63), off = 32 (through shared memory),
  // then 16 .. 1 inside warp 0
  if (l >= 64) {
#pragma unroll
    for (int e = 0; e < 8; ++e) part[l - 64][e] = acc[e];
  }
  __syncthreads();
  if (l < 64) {
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += part[l][e];
  }
  __syncthreads();
  if (l >= 32 && l < 64) {
#pragma unroll
    for (int e = 0; e < 8; ++e) part[l - 32][e] = acc[e];
  }
  __syncthreads();
  if (l < 32) {
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += part[l][e];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += __shfl_down_sync(0xffffffffu, acc[e], off);
    }
    if (l == 0) {
      __align__(16) __half o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(acc[e] / (float)HW);
      *reinterpret_cast<uint4 *>(y + (long long)b * x.C + q * 8) = *reinterpret_cast<const uint4 *>(o);
    }
  }
}

// Batched matmul Y[z] = A[z] B[z] on the CUDA cores in 64 x 64 output tiles
// (4 x 4 per thread), K in 32-wide slices staged in shared memory as f32, two
// slice buffers: the next slice's global loads (one 16-byte load per operand
// per thread, eight halves) are in flight while the current slice computes.
// Every output accumulates its K products in order with one fused
// multiply-add each, as bmm_k does, so the two kernels agree bit for bit.
// TA / TB: the operand is stored transposed (A as [K][M], B as [N][K]), which
// lets a transposing permute that only feeds this product be folded into it.
// `vec`: both operands' rows and batch offsets are 16-byte aligned, so full
// eight-half chunks are read with one load (edge chunks element by element).
// At most 64 registers, so four blocks share an SM: YOLO11's v·attnᵀ launch
// (896 blocks) then runs in two waves instead of three.
constexpr int kBmmT = 64, kBmmKT = 32, kBmmPad = 68;  // rows of 68 floats: aligned float4 reads
// One operand's slice: 64 rows (m or n) x 32 k as eight-half chunks, one per
// thread.  K-contiguous storage ([rows][K]): thread t takes row t % 64 and k
// chunk (t / 64) * 8 (stores across consecutive rows, no bank conflicts);
// row-contiguous storage ([K][rows]): k = t / 8, rows (t % 8) * 8 .. +7.
template <bool KCONTIG>
__device__ __forceinline__ void bmm_load_slice(const __half *__restrict__ base, int rows, int K, int r0, int k0,
                                               bool vec, float (&v)[8]) {
  const int t = threadIdx.x;
  const int r = KCONTIG ? r0 + (t & 63) : r0 + (t & 7) * 8;
  const int k = KCONTIG ? k0 + (t >> 6) * 8 : k0 + (t >> 3);
  if (KCONTIG) {  // eight k of one row
    if (r < rows && vec && k + 8 <= K) {
      const uint4 u = __ldg(reinterpret_cast<const uint4 *>(base + (long long)r * K + k));
      const __half *h = reinterpret_cast<const __half *>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __half2float(h[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (r < rows && k + j < K) ? __half2float(base[(long long)r * K + k + j]) : 0.0f;
    }
  } else {  // eight rows of one k
    if (k < K && vec && r + 8 <= rows) {
      const uint4 u = __ldg(reinterpret_cast<const uint4 *>(base + (long long)k * rows + r));
      const __half *h = reinterpret_cast<const __half *>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __half2float(h[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (k < K && r + j < rows) ? __half2float(base[(long long)k * rows + r + j]) : 0.0f;
    }
  }
}
template <bool KCONTIG>
__device__ __forceinline__ void bmm_store_slice(float (*S)[kBmmPad], const float (&v)[8]) {
  const int t = threadIdx.x;
  if (KCONTIG) {
    const int r = t & 63, k = (t >> 6) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) S[k + j][r] = v[j];
  } else {
    const int k = t >> 3, r = (t & 7) * 8;
    *reinterpret_cast<float4 *>(&S[k][r]) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4 *>(&S[k][r + 4]) = make_float4(v[4], v[5], v[6], v[7]);
  }
}

template <bool TA, bool TB>
__global__ void __launch_bounds__(256, 4) bmm_tiled_k(const __half *__restrict__ A, const __half *__restrict__ B,
                                                   __half *__restrict__ Y, int B1, int M, int K, int N, long long a_bs,
                                                   long long b_bs, int tiles_m, int tiles_n, int vec) {
  pdl_wait_and_release();
  __shared__ __align__(16) float As[2][kBmmKT][kBmmPad];  // As[k][m]
  __shared__ __align__(16) float Bs[2][kBmmKT][kBmmPad];  // Bs[k][n]
  const int tile = blockIdx.x % (tiles_m * tiles_n);
  const long long z = blockIdx.x / (tiles_m * tiles_n);  // b0 * B1 + b1
  const long long b0 = z / B1, b1 = z - b0 * B1;
  const int m0 = (tile / tiles_n) * kBmmT, n0 = (tile % tiles_n) * kBmmT;
  const __half *Az = A + b0 * a_bs + b1 * (long long)M * K;
  const __half *Bz = B + b0 * b_bs + b1 * (long long)K * N;
  __half *Yz = Y + z * (long long)M * N;
  const bool vc = vec != 0;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // outputs m0 + 4 ty + i, n0 + 4 tx + j
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  // A non-transposed is [M][K] (K-contiguous); B transposed is [N][K] (K-contiguous)
  float va[8], vb[8];
  bmm_load_slice<!TA>(Az, M, K, m0, 0, vc, va);
  bmm_load_slice<TB>(Bz, N, K, n0, 0, vc, vb);
  bmm_store_slice<!TA>(As[0], va);
  bmm_store_slice<TB>(Bs[0], vb);
  __syncthreads();
  int cur = 0;
  for (int k0 = 0; k0 < K; k0 += kBmmKT) {
    const bool more = k0 + kBmmKT < K;
    if (more) {  // the next slice's loads fly while this one computes
      bmm_load_slice<!TA>(Az, M, K, m0, k0 + kBmmKT, vc, va);
      bmm_load_slice<TB>(Bz, N, K, n0, k0 + kBmmKT, vc, vb);
    }
    const int kl = min(kBmmKT, K - k0);
    for (int kk = 0; kk < kl; ++kk) {
      const float4 av = *reinterpret_cast<const float4 *>(&As[cur][kk][4 * ty]);
      const float4 bv = *reinterpret_cast<const float4 *>(&Bs[cur][kk][4 * tx]);
      const float a[4] = {av.x, av.y, av.z, av.w}, b[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
    }
    if (more) {  // the other buffer was last read before the previous barrier
      bmm_store_slice<!TA>(As[cur ^ 1], va);
      bmm_store_slice<TB>(Bs[cur ^ 1], vb);
    }
    __syncthreads();
    cur ^= 1;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + 4 * ty + i;
    if (gm >= M) continue;
    const int gn = n0 + 4 * tx;
    __half *yr = Yz + (long long)gm * N;
    if (vc && (N & 3) == 0 && gn + 4 <= N) {  // four consecutive outputs, 8 bytes
      const __half2 lo = __floats2half2_rn(acc[i][0], acc[i][1]), hi = __floats2half2_rn(acc[i][2], acc[i][3]);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t *>(&lo);
      u.y = *reinterpret_cast<const uint32_t *>(&hi);
      *reinterpret_cast<uint2 *>(yr + gn) = u;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (gn + j < N) yr[gn + j] = __float2half_rn(acc[i][j]);
    }
  }
}

__global__ void bmm_k(const __half *__restrict__ A, const __half *__restrict__ B, __half *__restrict__ Y, long long n,
                      int B1, int M, int K, int N, long long a_bs, long long b_bs) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int nn = (int)(i % N);
    long long t = i / N;
    const int m = (int)(t % M);
    t /= M;
    const int b1 = (int)(t % B1);
    const long long b0 = t / B1;
    const __half *ap = A + b0 * a_bs + ((long long)b1 * M + m) * K;
    const __half *bp = B + b0 * b_bs + (long long)b1 * K * N + nn;
    float acc = 0.0f;
    for (int k = 0; k < K; ++k) acc += __half2float(ap[k]) * __half2float(bp[(long long)k * N]);
    Y[i] = __float2half_rn(acc);
  }
}

__global__ void bias_add_k(const __half *__restrict__ x, const __half *__restrict__ b, __half *__restrict__ y,
                           long long n, long long per_img, int HW) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i % per_img;
    y[i] = __float2half_rn(__half2float(x[i]) + __half2float(b[r / HW]));
  }
}

// ------------------------------------------------------------------ convolutions
// depthwise, weights repacked [K*K][C]; fp32 accumulation in (ky, kx) order,
// then half(half(acc) + bias) -> act (depthwise_f16 expressions).
__global__ void depthwise_v4_k(View4 x, const __half *__restrict__ w, const __half *__restrict__ bias, View4 y,
                               long long n, int K, int S, int P, int act, bool cfast) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const Idx4 o = idx4(i, y, cfast);
    float acc = 0.0f;
    for (int ky = 0; ky < K; ++ky) {
      const int iy = o.y * S - P + ky;
      if (iy < 0 || iy >= x.H) continue;
      for (int kx = 0; kx < K; ++kx) {
        const int ix = o.x * S - P + kx;
        if (ix < 0 || ix >= x.W) continue;
        acc += __half2float(x.ptr[o.b * x.sb + (long long)o.c * x.sc + (long long)iy * x.sy + (long long)ix * x.sx]) *
               __half2float(w[(ky * K + kx) * y.C + o.c]);
      }
    }
    const float bv = bias ? __half2float(bias[o.c]) : 0.0f;
    y.ptr[at(y, o)] = epilogue(acc, bv, act, kActDepthwise);
  }
}

// NHWC fast path: 8 channels per thread with 16-byte loads/stores.
__global__ void depthwise_nhwc8_k(View4 x, const __half *__restrict__ w, const __half *__restrict__ bias, View4 y,
                                  long long n8, int K, int S, int P, int act) {
  pdl_wait_and_release();
  const int C8 = y.C / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const int c8 = (int)(i % C8);
    long long t = i / C8;
    const int ox = (int)(t % y.W);
    t /= y.W;
    const int oy = (int)(t % y.H);
    const long long b = t / y.H;
    const int c = c8 * 8;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    for (int ky = 0; ky < K; ++ky) {
      const int iy = oy * S - P + ky;
      if (iy < 0 || iy >= x.H) continue;
      for (int kx = 0; kx < K; ++kx) {
        const int ix = ox * S - P + kx;
        if (ix < 0 || ix >= x.W) continue;
        const uint4 xv = *reinterpret_cast<const uint4 *>(x.ptr + b * x.sb + (long long)iy * x.sy + (long long)ix * x.sx + c);
        const uint4 wv = *reinterpret_cast<const uint4 *>(w + (ky * K + kx) * y.C + c);
        const __half *xh = reinterpret_cast<const __half *>(&xv);
        const __half *wh = reinterpret_cast<const __half *>(&wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += __half2float(xh[j]) * __half2float(wh[j]);
      }
    }
    __align__(16) __half out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = epilogue(acc[j], bias ? __half2float(bias[c + j]) : 0.0f, act, kActDepthwise);
    *reinterpret_cast<uint4 *>(y.ptr + b * y.sb + (long long)oy * y.sy + (long long)ox * y.sx + c) =
        *reinterpret_cast<const uint4 *>(out);
  }
}

// Depthwise in row blocks: blockIdx.y is one output row of one image (b * Ho
// + oy, grid-strided beyond the grid), threads run over that row's (ox,
// channel) positions, so every index comes from 32-bit arithmetic and the
// divisions by the row's channel count are multiply-highs.  The activation is
// a template parameter (the depthwise_f16 expressions, resolved on the host).
// Same fp32 accumulation order (ky, kx) and epilogue as above.
struct DwDiv {
  uint32_t m, s;  // q = (n * m) >> (31 + s), exact for n < 2^31
};
__device__ __forceinline__ uint32_t dw_div(uint32_t n, DwDiv d) { return (uint32_t)(((uint64_t)n * d.m) >> (31u + d.s)); }
inline DwDiv dw_make_div(uint32_t dv) {  // host: the multiplier and shift of division by dv >= 1
  DwDiv d{0u, 0u};
  uint32_t sh = 0;
  while ((1ull << sh) < dv) ++sh;
  d.s = sh;
  d.m = (uint32_t)(((1ull << (31 + sh)) / dv) + 1ull);
  return d;
}

// ew_binary_flat_k eight elements at a time: 16-byte loads and stores, the
// image of a chunk from a 32-bit multiply-high division (per_img and the
// batch offsets are multiples of 8, so a chunk never straddles two images);
// each element is the same f32 operation rounded once.
__global__ void ew_binary_flat8_k(const __half *__restrict__ a, const __half *__restrict__ b, __half *__restrict__ y,
                                  long long n8, int op, int b_scalar, uint32_t per8, long long a_bs, long long b_bs,
                                  DwDiv d_per8) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const uint32_t img = dw_div((uint32_t)i, d_per8), r = ((uint32_t)i - img * per8) * 8u;
    const uint4 au = *reinterpret_cast<const uint4 *>(a + (long long)img * a_bs + r);
    uint4 bu;
    if (b_scalar) {
      const __half s = b[(long long)img * b_bs];
      const __half2 s2 = __halves2half2(s, s);
      bu.x = bu.y = bu.z = bu.w = *reinterpret_cast<const uint32_t *>(&s2);
    } else {
      bu = *reinterpret_cast<const uint4 *>(b + (long long)img * b_bs + r);
    }
    const __half *ah = reinterpret_cast<const __half *>(&au), *bh = reinterpret_cast<const __half *>(&bu);
    uint4 ou;
    __half *oh = reinterpret_cast<__half *>(&ou);
#pragma unroll
    for (int j = 0; j < 8; ++j) oh[j] = __float2half_rn(binop(__half2float(ah[j]), __half2float(bh[j]), op));
    *reinterpret_cast<uint4 *>(y + i * 8) = ou;
  }
}

// SiLU in the MUFU form the tensor-core epilogue uses (relative error below
// 2^-19: the fp16 result is the correctly rounded one or its neighbour), the
// other activations in the reference expression.
template <int FN>
__device__ __forceinline__ __half dw_epilogue(float acc, float bias) {
  const float v = __half2float(__float2half_rn(__half2float(__float2half_rn(acc)) + bias));
  return __float2half_rn(FN == kFnSilu ? silu_fast(v) : act_exact<FN>(v));
}

template <int FN>
__global__ void __launch_bounds__(256) depthwise_nhwc8_rows_k(View4 x, const __half *__restrict__ w,
                                                             const __half *__restrict__ bias, View4 y, int rows,
                                                             int K, int S, int P, DwDiv dc8) {
  pdl_wait_and_release();
  const int C8 = y.C / 8, per_row = y.W * C8;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const int b = r / y.H, oy = r - b * y.H;
    const __half *xb = x.ptr + (long long)b * x.sb;
    __half *yrow = y.ptr + (long long)b * y.sb + (long long)oy * y.sy;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < per_row; t += gridDim.x * blockDim.x) {
      const int ox = (int)dw_div((uint32_t)t, dc8), c = (t - ox * C8) * 8;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
      for (int ky = 0; ky < K; ++ky) {
        const int iy = oy * S - P + ky;
        if (iy < 0 || iy >= x.H) continue;
        const __half *xr = xb + (long long)iy * x.sy + c;
        for (int kx = 0; kx < K; ++kx) {
          const int ix = ox * S - P + kx;
          if (ix < 0 || ix >= x.W) continue;
          const uint4 xv = __ldg(reinterpret_cast<const uint4 *>(xr + (long long)ix * x.sx));
          const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(w + (ky * K + kx) * y.C + c));
          const __half *xh = reinterpret_cast<const __half *>(&xv);
          const __half *wh = reinterpret_cast<const __half *>(&wv);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += __half2float(xh[j]) * __half2float(wh[j]);
        }
      }
      __align__(16) __half out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = dw_epilogue<FN>(acc[j], bias ? __half2float(__ldg(bias + c + j)) : 0.0f);
      *reinterpret_cast<uint4 *>(yrow + (long long)ox * y.sx + c) = *reinterpret_cast<const uint4 *>(out);
    }
  }
}

// Depthwise K x K (3 or 5), stride S (1 or 2), channels-last, in strips: a
// thread computes kDwNhwcStrip neighbouring output pixels of one 8-channel
// group, so each weight vector is loaded once for them and each input vector
// once per kernel row for all the outputs that use it (two outputs keep the
// registers at 80, three blocks per SM, which measured faster than four
// outputs at two blocks per SM).  Same fp32 accumulation
// order (ky, kx), same skipped padding taps and epilogue as above, so the
// results are identical.  Threads run over (output row, strip, channel
// group) with the channel group fastest (consecutive threads, consecutive
// 16-byte vectors).
constexpr int kDwNhwcStrip = 2;  // outputs per thread of the channels-last strip kernel
template <int FN, int K, int S>
__global__ void __launch_bounds__(256) depthwise_nhwc8_strip_k(View4 x, const __half *__restrict__ w,
                                                              const __half *__restrict__ bias, View4 y,
                                                              long long items, int P, int C8, int strips,
                                                              DwDiv d_item, DwDiv d_c8, DwDiv d_ho) {
  pdl_wait_and_release();
  constexpr int NO = kDwNhwcStrip, NX = (NO - 1) * S + K;  // input columns the NO outputs read
  const int per_row = strips * C8;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < items;
       idx += (long long)gridDim.x * blockDim.x) {
    const uint32_t r = dw_div((uint32_t)idx, d_item);          // output row b * Ho + oy
    const uint32_t it = (uint32_t)idx - r * (uint32_t)per_row;  // strip * C8 + channel group
    const uint32_t sx = dw_div(it, d_c8);
    const int c = (int)(it - sx * (uint32_t)C8) * 8;
    const uint32_t b = dw_div(r, d_ho);
    const int oy = (int)(r - b * (uint32_t)y.H), ox0 = (int)sx * NO;
    const __half *xb = x.ptr + (long long)b * x.sb + c;
    float acc[NO][8];
#pragma unroll
    for (int o = 0; o < NO; ++o)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[o][j] = 0.0f;
#pragma unroll
    for (int ky = 0; ky < K; ++ky) {
      const int iy = oy * S - P + ky;
      if (iy < 0 || iy >= x.H) continue;
      const __half *xr = xb + (long long)iy * x.sy;
      uint4 xv[NX];
      bool ok[NX];
#pragma unroll
      for (int q = 0; q < NX; ++q) {
        const int ix = ox0 * S - P + q;
        ok[q] = ix >= 0 && ix < x.W;
        xv[q] = ok[q] ? __ldg(reinterpret_cast<const uint4 *>(xr + (long long)ix * x.sx)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int kx = 0; kx < K; ++kx) {
        const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(w + (ky * K + kx) * y.C + c));
        const __half *wh = reinterpret_cast<const __half *>(&wv);
#pragma unroll
        for (int o = 0; o < NO; ++o) {
          const int q = o * S + kx;
          if (!ok[q]) continue;
          const __half *xh = reinterpret_cast<const __half *>(&xv[q]);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[o][j] += __half2float(xh[j]) * __half2float(wh[j]);
        }
      }
    }
    __align__(16) float bv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) bv[j] = bias ? __half2float(__ldg(bias + c + j)) : 0.0f;
    __half *yrow = y.ptr + (long long)b * y.sb + (long long)oy * y.sy + c;
#pragma unroll
    for (int o = 0; o < NO; ++o) {
      if (ox0 + o >= y.W) break;
      __align__(16) __half out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = dw_epilogue<FN>(acc[o][j], bv[j]);
      *reinterpret_cast<uint4 *>(yrow + (long long)(ox0 + o) * y.sx) = *reinterpret_cast<const uint4 *>(out);
    }
  }
}

// Planar depthwise, one output per thread over (plane, oy, ox) flattened, so
// small planes still fill whole blocks; same arithmetic as the kernels above.
template <int FN>
__global__ void __launch_bounds__(256) depthwise_planar_flat_k(View4 x, const __half *__restrict__ w,
                                                              const __half *__restrict__ bias, View4 y,
                                                              long long n, int K, int S, int P, DwDiv d_hw,
                                                              DwDiv d_wo, DwDiv d_c) {
  pdl_wait_and_release();
  const uint32_t hw = (uint32_t)(y.H * y.W);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const uint32_t plane = dw_div((uint32_t)i, d_hw), p = (uint32_t)i - plane * hw;
    const uint32_t b = dw_div(plane, d_c), c = plane - b * (uint32_t)y.C;
    const uint32_t oy = dw_div(p, d_wo), ox = p - oy * (uint32_t)y.W;
    const __half *xp = x.ptr + (long long)b * x.sb + (long long)c * x.sc;
    float acc = 0.0f;
    for (int ky = 0; ky < K; ++ky) {
      const int iy = (int)oy * S - P + ky;
      if (iy < 0 || iy >= x.H) continue;
      const __half *xr = xp + (long long)iy * x.sy;
      for (int kx = 0; kx < K; ++kx) {
        const int ix = (int)ox * S - P + kx;
        if (ix < 0 || ix >= x.W) continue;
        acc += __half2float(xr[(long long)ix * x.sx]) * __half2float(__ldg(w + (ky * K + kx) * y.C + c));
      }
    }
    y.ptr[(long long)b * y.sb + (long long)c * y.sc + (long long)oy * y.sy + (long long)ox * y.sx] =
        dw_epilogue<FN>(acc, bias ? __half2float(bias[c]) : 0.0f);
  }
}

// Planar depthwise over small planes (H * W <= 512, e.g. the 20 x 20 maps of
// YOLO11's attention): a block stages 16 whole input planes in shared memory
// with coalesced loads, and 16 threads per plane, each holding the plane's
// K*K weights in registers, compute its outputs from shared memory.  Same
// arithmetic as the kernels above (taps in (ky, kx) order, out-of-image taps
// skipped, one fused multiply-add each).
constexpr int kDwPlanesPerBlock = 16, kDwPlaneMax = 512;
template <int FN, int K, int S>
__global__ void __launch_bounds__(256) depthwise_planar_plane_k(View4 x, const __half *__restrict__ w,
                                                               const __half *__restrict__ bias, View4 y, int planes,
                                                               int P, int dense, DwDiv d_hw, DwDiv d_w, DwDiv d_wo,
                                                               DwDiv d_c) {
  pdl_wait_and_release();
  __shared__ __align__(16) __half xs[kDwPlanesPerBlock * kDwPlaneMax];
  const int H = x.H, W = x.W, HW = H * W, Ho = y.H, Wo = y.W, HWo = Ho * Wo, C = y.C;
  const int p0 = blockIdx.x * kDwPlanesPerBlock;
  const int np = min(kDwPlanesPerBlock, planes - p0);
  if (dense) {
    // the block's planes are one contiguous, 16-byte aligned run of np * HW
    // halves (planes packed, C a multiple of 16): 16-byte loads, all issued
    // before the first store; plane q lands at q * HW
    const uint32_t b0 = dw_div((uint32_t)p0, d_c), c0 = (uint32_t)p0 - b0 * (uint32_t)C;
    const uint4 *src = reinterpret_cast<const uint4 *>(x.ptr + (long long)b0 * x.sb + (long long)c0 * x.sc);
    uint4 *dst = reinterpret_cast<uint4 *>(xs);
    const int n16 = np * HW / 8;
    constexpr int kLd = 4;
    for (int e0 = threadIdx.x; e0 < n16; e0 += kLd * (int)blockDim.x) {
      uint4 v[kLd];
#pragma unroll
      for (int j = 0; j < kLd; ++j)
        if (e0 + j * (int)blockDim.x < n16) v[j] = __ldg(src + e0 + j * (int)blockDim.x);
#pragma unroll
      for (int j = 0; j < kLd; ++j)
        if (e0 + j * (int)blockDim.x < n16) dst[e0 + j * (int)blockDim.x] = v[j];
    }
  } else {
    constexpr int kLd = 8;  // loads in flight per thread before their stores
    for (int e0 = threadIdx.x; e0 < np * HW; e0 += kLd * (int)blockDim.x) {
      __half v[kLd];
#pragma unroll
      for (int j = 0; j < kLd; ++j) {
        const int e = e0 + j * (int)blockDim.x;
        if (e >= np * HW) break;
        const uint32_t q = dw_div((uint32_t)e, d_hw), r = (uint32_t)e - q * (uint32_t)HW;
        const uint32_t yy = dw_div(r, d_w), xx = r - yy * (uint32_t)W;
        const uint32_t pl = (uint32_t)p0 + q, b = dw_div(pl, d_c), c = pl - b * (uint32_t)C;
        v[j] = x.ptr[(long long)b * x.sb + (long long)c * x.sc + (long long)yy * x.sy + (long long)xx * x.sx];
      }
#pragma unroll
      for (int j = 0; j < kLd; ++j) {
        const int e = e0 + j * (int)blockDim.x;
        if (e >= np * HW) break;
        xs[e] = v[j];  // plane q at q * HW
      }
    }
  }
  __syncthreads();
  const int q = threadIdx.x >> 4, sub = threadIdx.x & 15;  // plane of this thread, its place among 16
  if (q >= np) return;
  const uint32_t pl = (uint32_t)(p0 + q), b = dw_div(pl, d_c), c = pl - b * (uint32_t)C;
  float wv[K * K];
#pragma unroll
  for (int t = 0; t < K * K; ++t) wv[t] = __half2float(__ldg(w + t * C + (int)c));
  const float bv = bias ? __half2float(bias[c]) : 0.0f;
  const __half *xp = xs + q * HW;
  __half *yp = y.ptr + (long long)b * y.sb + (long long)c * y.sc;
  for (int r = sub; r < HWo; r += 16) {
    const int oy = (int)dw_div((uint32_t)r, d_wo), ox = r - oy * Wo;
    float acc = 0.0f;
#pragma unroll
    for (int ky = 0; ky < K; ++ky) {
      const int iy = oy * S - P + ky;
      if (iy < 0 || iy >= H) continue;
#pragma unroll
      for (int kx = 0; kx < K; ++kx) {
        const int ix = ox * S - P + kx;
        if (ix < 0 || ix >= W) continue;
        acc += __half2float(xp[iy * W + ix]) * wv[ky * K + kx];
      }
    }
    yp[(long long)oy * y.sy + (long long)ox * y.sx] = dw_epilogue<FN>(acc, bv);
  }
}

// Planar depthwise, four neighbouring outputs of one row per thread: each
// input row segment is loaded once for the four, the K*K weights once per
// thread.  Same arithmetic as the kernels above: taps in (ky, kx) order, one
// fused multiply-add each; an out-of-image tap reads 0, which leaves the sum
// unchanged (it never holds -0), so it equals skipping the tap.
template <int FN, int K, int S>
__global__ void __launch_bounds__(256) depthwise_planar_strip_k(View4 x, const __half *__restrict__ w,
                                                               const __half *__restrict__ bias, View4 y,
                                                               long long items, int P, int strips, DwDiv d_strips,
                                                               DwDiv d_ho, DwDiv d_c) {
  pdl_wait_and_release();
  constexpr int IW = 3 * S + K;  // input columns under four outputs
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (long long)gridDim.x * blockDim.x) {
    const uint32_t row = dw_div((uint32_t)i, d_strips), sx = (uint32_t)i - row * (uint32_t)strips;
    const uint32_t plane = dw_div(row, d_ho), oy = row - plane * (uint32_t)y.H;
    const uint32_t b = dw_div(plane, d_c), c = plane - b * (uint32_t)y.C;
    const int ox0 = (int)sx * 4, ix0 = ox0 * S - P;
    const __half *xp = x.ptr + (long long)b * x.sb + (long long)c * x.sc;
    float wv[K * K];
#pragma unroll
    for (int t = 0; t < K * K; ++t) wv[t] = __half2float(__ldg(w + t * y.C + c));
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ky = 0; ky < K; ++ky) {
      const int iy = (int)oy * S - P + ky;
      const bool row_ok = iy >= 0 && iy < x.H;
      const __half *xr = xp + (long long)(row_ok ? iy : 0) * x.sy;
      float v[IW];
#pragma unroll
      for (int j = 0; j < IW; ++j) {
        const int ix = ix0 + j;
        v[j] = (row_ok && ix >= 0 && ix < x.W) ? __half2float(xr[(long long)ix * x.sx]) : 0.0f;
      }
#pragma unroll
      for (int kx = 0; kx < K; ++kx) {
#pragma unroll
        for (int o = 0; o < 4; ++o) acc[o] += v[o * S + kx] * wv[ky * K + kx];
      }
    }
    const float bv = bias ? __half2float(bias[c]) : 0.0f;
    __half *yr = y.ptr + (long long)b * y.sb + (long long)c * y.sc + (long long)oy * y.sy;
#pragma unroll
    for (int o = 0; o < 4; ++o)
      if (ox0 + o < y.W) yr[(long long)(ox0 + o) * y.sx] = dw_epilogue<FN>(acc[o], bv);
  }
}

// Planar depthwise in plane rows: blockIdx.y is one (image, channel, output
// row), threads run over the row's output columns (coalesced stores).
template <int FN>
__global__ void __launch_bounds__(256) depthwise_planar_rows_k(View4 x, const __half *__restrict__ w,
                                                              const __half *__restrict__ bias, View4 y, int rows,
                                                              int K, int S, int P) {
  pdl_wait_and_release();
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const int oy = r % y.H, bc = r / y.H, c = bc % y.C, b = bc / y.C;
    const __half *xp = x.ptr + (long long)b * x.sb + (long long)c * x.sc;
    __half *yr = y.ptr + (long long)b * y.sb + (long long)c * y.sc + (long long)oy * y.sy;
    const float bv = bias ? __half2float(bias[c]) : 0.0f;
    for (int ox = blockIdx.x * blockDim.x + threadIdx.x; ox < y.W; ox += gridDim.x * blockDim.x) {
      float acc = 0.0f;
      for (int ky = 0; ky < K; ++ky) {
        const int iy = oy * S - P + ky;
        if (iy < 0 || iy >= x.H) continue;
        const __half *xr = xp + (long long)iy * x.sy;
        for (int kx = 0; kx < K; ++kx) {
          const int ix = ox * S - P + kx;
          if (ix < 0 || ix >= x.W) continue;
          acc += __half2float(xr[(long long)ix * x.sx]) * __half2float(__ldg(w + (ky * K + kx) * y.C + c));
        }
      }
      yr[(long long)ox * y.sx] = dw_epilogue<FN>(acc, bv);
    }
  }
}

// generic direct convolution, weights in the plan layout [Cout][Cin/G][K][K]
__global__ void conv_direct_v4_k(View4 x, const __half *__restrict__ w, const __half *__restrict__ bias,
                                 const __half *res_ptr, View4 res, View4 y, long long n, int K, int S, int P, int G,
                                 int act, int epi, bool cfast) {
  pdl_wait_and_release();
  const int cin_g = x.C / G, cout_g = y.C / G;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const Idx4 o = idx4(i, y, cfast);
    const int g = o.c / cout_g, ic0 = g * cin_g;
    float acc = (epi == 0 && bias) ? __half2float(bias[o.c]) : 0.0f;
    for (int ic = 0; ic < cin_g; ++ic)
      for (int ky = 0; ky < K; ++ky) {
        const int iy = o.y * S - P + ky;
        if (iy < 0 || iy >= x.H) continue;
        for (int kx = 0; kx < K; ++kx) {
          const int ix = o.x * S - P + kx;
          if (ix < 0 || ix >= x.W) continue;
          acc += __half2float(x.ptr[o.b * x.sb + (long long)(ic0 + ic) * x.sc + (long long)iy * x.sy + (long long)ix * x.sx]) *
                 __half2float(w[(((long long)o.c * cin_g + ic) * K + ky) * K + kx]);
        }
      }
    __half v;
    if (epi == 0) {  // conv_general.cl:42-47, codes 1=SiLU 2=HardSwish 3=ReLU 4=HardSigmoid
      float r = acc;
      if (act == 1) r = acc / (1.0f + expf(-acc));
      else if (act == 2) r = acc * fminf(fmaxf(acc + 3.0f, 0.0f), 6.0f) / 6.0f;
      else if (act == 3) r = fmaxf(acc, 0.0f);
      else if (act == 4) r = fminf(fmaxf(acc + 3.0f, 0.0f), 6.0f) / 6.0f;
      v = __float2half_rn(r);
    } else {
      v = epilogue(acc, bias ? __half2float(bias[o.c]) : 0.0f, act, epi == 1 ? kActGemm : kActConv3x3);
    }
    if (res_ptr) v = __float2half_rn(__half2float(v) + __half2float(res_ptr[at(res, o)]));
    y.ptr[at(y, o)] = v;
  }
}

// Stem conv3x3 with Cin <= 4: one thread per output pixel, all Cout channels.
// Weights in shared memory as f32 [Cout][Cin*9]; accumulation order (ci, ky, kx).
constexpr int kStemMaxCout = 64;
__global__ void stem3x3_k(View4 x, const __half *__restrict__ w, const __half *__restrict__ bias, View4 y,
                          long long npix, int Cout, int S, int P, int act) {
  pdl_wait_and_release();
  __shared__ float ws[kStemMaxCout * 36];
  __shared__ float bs[kStemMaxCout];
  const int cin = x.C, kk = cin * 9;
  for (int i = threadIdx.x; i < Cout * kk; i += blockDim.x) ws[i] = __half2float(w[i]);
  for (int i = threadIdx.x; i < Cout; i += blockDim.x) bs[i] = bias ? __half2float(bias[i]) : 0.0f;
  __syncthreads();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < npix; i += (long long)gridDim.x * blockDim.x) {
    const int ox = (int)(i % y.W);
    long long t = i / y.W;
    const int oy = (int)(t % y.H);
    const long long b = t / y.H;
    float in[36];
    for (int ci = 0; ci < cin; ++ci)
      for (int ky = 0; ky < 3; ++ky) {
        const int iy = oy * S - P + ky;
        for (int kx = 0; kx < 3; ++kx) {
          const int ix = ox * S - P + kx;
          const bool ok = iy >= 0 && iy < x.H && ix >= 0 && ix < x.W;
          in[ci * 9 + ky * 3 + kx] =
              ok ? __half2float(x.ptr[b * x.sb + (long long)ci * x.sc + (long long)iy * x.sy + (long long)ix * x.sx]) : 0.0f;
        }
      }
    const long long obase = b * y.sb + (long long)oy * y.sy + (long long)ox * y.sx;
    for (int co = 0; co < Cout; co += 8) {
      __align__(16) __half out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = co + j;
        if (c < Cout) {
          float acc = 0.0f;
          for (int k = 0; k < kk; ++k) acc += in[k] * ws[c * kk + k];
          out[j] = epilogue(acc, bs[c], act, kActConv3x3);
        }
      }
      if (y.sc == 1 && co + 8 <= Cout && ((obase + co) & 7) == 0 && (reinterpret_cast<uintptr_t>(y.ptr) & 15) == 0) {
        *reinterpret_cast<uint4 *>(y.ptr + obase + co) = *reinterpret_cast<const uint4 *>(out);
      } else {
        for (int j = 0; j < 8 && co + j < Cout; ++j) y.ptr[obase + (long long)(co + j) * y.sc] = out[j];
      }
    }
  }
}

// Stem 3x3 (Cin 3 -> Cout 16) on the tensor cores.  K = the 27 taps of one
// output pixel in the reference's (ci, ky, kx) order, zero-padded to 32, forms
// an A row.  Per 8 x 16-pixel tile the CTA stages the planar input patch in
// shared memory, each thread builds its pixel's row in two 32-byte-row
// swizzled K16 slices (the layout TMA writes for the conv kernel: 16-byte chunk
// c of row r at c ^ ((r >> 2) & 1)), one thread issues two MMAs into a
// 16-column TMEM accumulator (fp32), and four warps run the conv epilogue.
struct StemTcParams {
  uint16_t w[16][32];  // [cout][k], k = ci * 9 + ky * 3 + kx, zero beyond 27
  uint4 b8[2];         // fp16 bias
};
constexpr int kStemTW = 16, kStemTH = 8;
constexpr int kStemPR = (kStemTH - 1) * 2 + 3, kStemPC = (kStemTW - 1) * 2 + 3;  // patch for stride <= 2

constexpr int kStemTmaW = 40;  // TMA patch row: 8-aligned start, covers the 33-pixel window

template <int FN, int S, bool TMA>
__global__ void __launch_bounds__(128) stem_tc_k(View4 x, const __grid_constant__ StemTcParams p,
                                                 const __grid_constant__ CUtensorMap pmap, View4 y, int P,
                                                 int tiles_x, int tiles_per_img, long long n_tiles, int vec_out,
                                                 int *status) {
  // TMA: the planar patch of the next tile is fetched into the one patch
  // buffer as soon as this tile's A rows are built, so the copy overlaps the
  // MMA and the epilogue (box {40, rows, 3, 1}, x start rounded down to 8; the
  // buffer starts on a 128-byte boundary, the TMA destination alignment).  One
  // buffer keeps the CTA near 13 KB of shared memory, so 16 CTAs fit an SM and
  // the 148 * 16 grid runs in one wave.
  // One block of shared memory laid out by hand (no alignment padding between
  // arrays): A slices at 0 (1024-aligned, 2 x 4 KB), B slices at 8 KB, the
  // patch at 9 KB (128-aligned), then the barriers and the TMEM address.
  constexpr int kBufHalves = ((3 * kStemPR * kStemTmaW + 63) / 64) * 64;
  constexpr int kOffB = 2 * 128 * 32, kOffPatch = kOffB + 2 * 16 * 32;
  constexpr int kOffBar = kOffPatch + (TMA ? kBufHalves * 2 : 0), kSmemBytes = kOffBar + 24;
  __shared__ __align__(1024) uint8_t stem_sm[kSmemBytes];
  uint8_t(*const a_sm)[128 * 32] = reinterpret_cast<uint8_t(*)[128 * 32]>(stem_sm);
  uint8_t(*const b_sm)[16 * 32] = reinterpret_cast<uint8_t(*)[16 * 32]>(stem_sm + kOffB);
  __half *const patch_t = reinterpret_cast<__half *>(stem_sm + kOffPatch);
  uint64_t &pbar = *reinterpret_cast<uint64_t *>(stem_sm + kOffBar);
  uint64_t &mma_bar = *reinterpret_cast<uint64_t *>(stem_sm + kOffBar + 8);
  uint32_t &tmem_sh = *reinterpret_cast<uint32_t *>(stem_sm + kOffBar + 16);
  __shared__ __half patch[TMA ? 1 : 3][TMA ? 1 : kStemPR][TMA ? 2 : kStemPC + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(smem_u32(&mma_bar), 1);
    mbar_init(smem_u32(&pbar), 1);
    fence_mbar_init();
    if (TMA) tma_prefetch_desc(&pmap);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_sh), 32);  // before the release: a following conv grid never starves us
    tmem_relinquish();
  }
  for (int i = tid; i < 2 * 16 * 2; i += blockDim.x) {  // weights: slice, row, 16-byte chunk
    const int sl = i >> 5, n = (i >> 1) & 15, c = i & 1;
    const uint4 v = *reinterpret_cast<const uint4 *>(&p.w[n][sl * 16 + c * 8]);
    *reinterpret_cast<uint4 *>(&b_sm[sl][n * 32 + ((c ^ ((n >> 2) & 1)) << 4)]) = v;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  pdl_wait_and_release();
  const uint32_t idesc = idesc_f16_f32(128, 16);
  const int ty = tid / kStemTW, tx = tid - ty * kStemTW;  // this thread's pixel in the tile
  constexpr int pr = (kStemTH - 1) * S + 3, pc = (kStemTW - 1) * S + 3;
  constexpr uint32_t kPatchBytes = (uint32_t)(kStemTmaW * pr * 3 * 2);
  static_assert(kBufHalves * 2 % 128 == 0 && kStemTmaW * pr * 3 <= kBufHalves, "patch buffer");
  auto issue_patch = [&](long long t) {  // thread 0
    const long long img = t / tiles_per_img;
    const int rem = (int)(t - img * tiles_per_img);
    const int iy0 = (rem / tiles_x) * kStemTH * S - P, ix0 = (rem % tiles_x) * kStemTW * S - P;
    mbar_expect_tx(smem_u32(&pbar), kPatchBytes);
    tma_load_4d(smem_u32(&patch_t[0]), &pmap, smem_u32(&pbar), ix0 & ~7, iy0, 0, (int)img);
  };
  // thread 0: the iteration whose patch copy is in flight (copy j completes
  // phase j of pbar), or -1
  int in_flight = -1;
  if (TMA && tid == 0 && (long long)blockIdx.x < n_tiles) {
    issue_patch(blockIdx.x);
    in_flight = 0;
  }
  uint32_t phase = 0;
  int k_iter = 0;
  for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x, phase ^= 1u, ++k_iter) {
    const long long img = t / tiles_per_img;
    const int rem = (int)(t - img * tiles_per_img);
    const int oy0 = (rem / tiles_x) * kStemTH, ox0 = (rem % tiles_x) * kStemTW;
    const int iy0 = oy0 * S - P, ix0 = ox0 * S - P;
    const int xoff = TMA ? ix0 - (ix0 & ~7) : 0;  // window start inside the TMA row
    if (TMA) {
      int bad = 0;
      if (tid == 0) {
        if (mbar_wait_poll(smem_u32(&pbar), (uint32_t)k_iter & 1u, 2000000000LL)) {
          in_flight = -1;
        } else {
          bad = 1;
          if (status) atomicCAS(status, 0, (int)kStatusTimeoutFull);
        }
      }
      if (__syncthreads_or(bad)) break;
    } else {  // patch rows rr = warp + 4 i, lanes along x; every load is issued before any store
      constexpr int kRows = (3 * pr + 3) / 4, kCols = (pc + 31) / 32;
      __half v[kRows][kCols];
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int rr = warp + 4 * i;
        const int c = rr / pr, yy = rr - c * pr;
        const int iy = iy0 + yy;
        const bool row_ok = rr < 3 * pr && iy >= 0 && iy < x.H;
        const __half *src = x.ptr + img * x.sb + (long long)c * x.sc + (long long)iy * x.sy;
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          const int ix = ix0 + lane + 32 * j;
          v[i][j] = (row_ok && lane + 32 * j < pc && ix >= 0 && ix < x.W) ? src[(long long)ix * x.sx]
                                                                           : __float2half(0.0f);
        }
      }
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int rr = warp + 4 * i;
        const int c = rr / pr, yy = rr - c * pr;
#pragma unroll
        for (int j = 0; j < kCols; ++j)
          if (rr < 3 * pr && lane + 32 * j < pc) patch[c][yy][lane + 32 * j] = v[i][j];
      }
      __syncthreads();
    }
    {  // this pixel's A row: 27 taps + 5 zeros, packed in pairs
      uint32_t w32[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        uint16_t lo = 0, hi = 0;
        const int k0 = 2 * j, k1 = 2 * j + 1;
        if (TMA) {  // the box lands as [channel][pr rows][40]
          const __half *pt = &patch_t[0];
          if (k0 < 27) lo = __half_as_ushort(pt[((k0 / 9) * pr + ty * S + (k0 % 9) / 3) * kStemTmaW + xoff + tx * S + k0 % 3]);
          if (k1 < 27) hi = __half_as_ushort(pt[((k1 / 9) * pr + ty * S + (k1 % 9) / 3) * kStemTmaW + xoff + tx * S + k1 % 3]);
        } else {
          if (k0 < 27) lo = __half_as_ushort(patch[k0 / 9][ty * S + (k0 % 9) / 3][tx * S + k0 % 3]);
          if (k1 < 27) hi = __half_as_ushort(patch[k1 / 9][ty * S + (k1 % 9) / 3][tx * S + k1 % 3]);
        }
        w32[j] = (uint32_t)lo | ((uint32_t)hi << 16);
      }
      const int sw = (tid >> 2) & 1;
#pragma unroll
      for (int sl = 0; sl < 2; ++sl)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          *reinterpret_cast<uint4 *>(&a_sm[sl][tid * 32 + ((c ^ sw) << 4)]) =
              make_uint4(w32[sl * 8 + c * 4], w32[sl * 8 + c * 4 + 1], w32[sl * 8 + c * 4 + 2], w32[sl * 8 + c * 4 + 3]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      // every thread has read the patch: the next tile's copy may land now
      if (TMA && t + gridDim.x < n_tiles) {
        issue_patch(t + gridDim.x);
        in_flight = k_iter + 1;
      }
      tc_fence_after();
#pragma unroll
      for (int sl = 0; sl < 2; ++sl)
        umma_f16(tmem, smem_desc_kmajor(smem_u32(&a_sm[sl][0]), 32), smem_desc_kmajor(smem_u32(&b_sm[sl][0]), 32),
                 idesc, sl != 0 ? 1u : 0u);
      umma_commit(smem_u32(&mma_bar));
    }
    int bad = 0;
    if (tid == 0 && !mbar_wait_poll(smem_u32(&mma_bar), phase, 2000000000LL)) {  // ~1 s
      bad = 1;
      if (status) atomicCAS(status, 0, (int)kStatusTimeoutAcc);
    }
    if (__syncthreads_or(bad)) break;  // every thread leaves together
    tc_fence_after();
    uint32_t r[16];
    tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16), r);
    tmem_ld_wait();
#pragma unroll
    for (int k = 0; k < 16; ++k) asm volatile("" : "+r"(r[k]));  // uses stay after the wait
    const int oy = oy0 + ty, ox = ox0 + tx;
    const uint32_t(&r0)[8] = *reinterpret_cast<const uint32_t(*)[8]>(&r[0]);
    const uint32_t(&r1)[8] = *reinterpret_cast<const uint32_t(*)[8]>(&r[8]);
    const uint4 o0 = epilogue8<FN>(r0, p.b8[0]), o1 = epilogue8<FN>(r1, p.b8[1]);
    if (oy < y.H && ox < y.W) {
      const long long ob = img * y.sb + (long long)oy * y.sy + (long long)ox * y.sx;
      if (vec_out) {
        *reinterpret_cast<uint4 *>(y.ptr + ob) = o0;
        *reinterpret_cast<uint4 *>(y.ptr + ob + 8) = o1;
      } else {
        const __half *h0 = reinterpret_cast<const __half *>(&o0), *h1 = reinterpret_cast<const __half *>(&o1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          y.ptr[ob + (long long)j * y.sc] = h0[j];
          y.ptr[ob + (long long)(j + 8) * y.sc] = h1[j];
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // patch, A tile and accumulator are reused by the next tile
  }
  if (TMA && tid == 0 && in_flight >= 0)  // only after an early exit: let the last copy land (bounded)
    mbar_wait_poll(smem_u32(&pbar), (uint32_t)in_flight & 1u, 400000000LL);
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

template <int FN>
cudaError_t launch_stem_tc_fn(View4 x, const StemTcParams &p, View4 y, int batch, int S, int P, int vec_out, int *status,
                              cudaStream_t st) {
  const int tiles_x = (y.W + kStemTW - 1) / kStemTW, tiles_y = (y.H + kStemTH - 1) / kStemTH;
  const long long n_tiles = (long long)batch * tiles_x * tiles_y;
  const long long grid = std::min<long long>(n_tiles, 148LL * 16);
  // TMA patches need a planar input whose rows and planes are 16-byte aligned
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  bool tma = x.sx == 1 && x.sy % 8 == 0 && x.sc % 8 == 0 && x.sb % 8 == 0 && x.C == 3 &&
             (reinterpret_cast<uintptr_t>(x.ptr) & 15) == 0;
  if (tma) {
    const int pr = (kStemTH - 1) * S + 3;
    const uint64_t dims[4] = {(uint64_t)x.W, (uint64_t)x.H, 3, (uint64_t)batch};
    const uint64_t strides[3] = {(uint64_t)x.sy * 2, (uint64_t)x.sc * 2, (uint64_t)x.sb * 2};
    const uint32_t box[4] = {(uint32_t)kStemTmaW, (uint32_t)pr, 3, 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    std::string err;
    tma = encode_tiled_f16(&map, 4, x.ptr, dims, strides, box, es, CU_TENSOR_MAP_SWIZZLE_NONE, &err);
  }
  const dim3 g((unsigned)grid), b(128);
  // 16 CTAs of ~14 KB shared memory per SM (one wave) need the largest carveout
  static std::atomic<bool> carve[4][kAttrMaxDevices];
  auto kern = S == 2 ? (tma ? stem_tc_k<FN, 2, true> : stem_tc_k<FN, 2, false>)
                     : (tma ? stem_tc_k<FN, 1, true> : stem_tc_k<FN, 1, false>);
  const cudaError_t ce = ensure_smem_carveout(kern, 100, carve[(S == 2 ? 2 : 0) + (tma ? 1 : 0)]);
  if (ce != cudaSuccess) return ce;
  return launch_kernel(kern, g, b, 0, st, x, p, map, y, P, tiles_x, tiles_x * tiles_y, n_tiles, vec_out, status);
}

// ------------------------------------------------------------------ conversions
// include/infvino/Half.hpp:14-24: truncate the mantissa, flush exp <= 0 to +-0,
// exp >= 31 to +-inf.
__global__ void f32_to_f16_trunc_k(const float *__restrict__ x, __half *__restrict__ y, long long n) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const uint32_t u = __float_as_uint(x[i]);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const int e = (int)((u >> 23) & 0xff) - 112;
    const uint32_t mant = u & 0x7fffffu;
    uint16_t h;
    if (e <= 0) h = (uint16_t)sign;
    else if (e >= 31) h = (uint16_t)(sign | 0x7c00u);
    else h = (uint16_t)(sign | ((uint32_t)e << 10) | (mant >> 13));
    y[i] = __ushort_as_half(h);
  }
}

__global__ void f16_to_f32_k(const __half *__restrict__ x, float *__restrict__ y, long long n) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = __half2float(x[i]);
}

// ------------------------------------------------------------------ NHWC fast paths
// 8 channels (16 bytes) per thread; valid when every view is channels-last with
// channel / pixel strides that keep 16-byte alignment.
inline bool vec8_ok(const View4 &v) {
  return v.sc == 1 && (v.C % 8) == 0 && (v.sx % 8) == 0 && (v.sy % 8) == 0 && (v.sb % 8) == 0 &&
         (reinterpret_cast<uintptr_t>(v.ptr) & 15) == 0;
}

struct Pix {
  int b, y, x, c;
};
__device__ __forceinline__ Pix pix8(unsigned long long i, const View4 &o) {
  Pix p;
  const unsigned C8 = (unsigned)o.C >> 3;
  p.c = (int)(i % C8) * 8;
  unsigned long long t = i / C8;
  p.x = (int)(t % (unsigned)o.W);
  t /= (unsigned)o.W;
  p.y = (int)(t % (unsigned)o.H);
  p.b = (int)(t / (unsigned)o.H);
  return p;
}
__device__ __forceinline__ long long at8(const View4 &v, int b, int y, int x, int c) {
  return (long long)b * v.sb + (long long)y * v.sy + (long long)x * v.sx + c;
}

__global__ void copy_nhwc8_k(View4 x, View4 y, long long n8) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const Pix p = pix8((unsigned long long)i, y);
    *reinterpret_cast<uint4 *>(y.ptr + at8(y, p.b, p.y, p.x, p.c)) =
        *reinterpret_cast<const uint4 *>(x.ptr + at8(x, p.b, p.y, p.x, p.c));
  }
}

__global__ void resize_nhwc8_k(View4 x, View4 y, long long n8, int S) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const Pix p = pix8((unsigned long long)i, y);
    *reinterpret_cast<uint4 *>(y.ptr + at8(y, p.b, p.y, p.x, p.c)) =
        *reinterpret_cast<const uint4 *>(x.ptr + at8(x, p.b, p.y / S, p.x / S, p.c));
  }
}

// Nearest upsample by S, channels-last: one thread per input vector of 8
// channels (read once, written to its S x S output pixels); blockIdx.y is the
// input row (image * H + y), so only the column / channel split divides.
__global__ void resize_up_nhwc8_k(View4 x, View4 y, int S, unsigned row8, unsigned C8) {
  pdl_wait_and_release();
  const unsigned r = blockIdx.y;
  const int b = (int)(r / (unsigned)x.H), iy = (int)(r - (unsigned)b * (unsigned)x.H);
  for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < row8; j += gridDim.x * blockDim.x) {
    const unsigned ix = j / C8;
    const int c = (int)(j - ix * C8) * 8;
    const uint4 v = *reinterpret_cast<const uint4 *>(x.ptr + at8(x, b, iy, (int)ix, c));
    for (int dy = 0; dy < S; ++dy)
      for (int dx = 0; dx < S; ++dx)
        *reinterpret_cast<uint4 *>(y.ptr + at8(y, b, iy * S + dy, (int)ix * S + dx, c)) = v;
  }
}

// Chained KxK stride-1 max pools (K = 2P + 1, pad P, out-of-image taps
// skipped), one block per (8-channel group, image) with the plane in shared
// memory: level l pools level l-1's result, like the separate pool nodes, as a
// row pass then a column pass (max is exact, so the split changes no value),
// on packed halves.  The block has a thread per pixel (up to 1024), and each
// pass reads its 2P neighbours with independent loads, so a level costs two
// shared-memory round trips and two barriers.
constexpr int kPoolChainMax = 3;
constexpr int kPoolChainMaxP = 3;
struct PoolChainOut {
  View4 y[kPoolChainMax];
};
// max of eight packed halves (exact: the result is one of the inputs)
__device__ __forceinline__ uint4 hmax8(uint4 a, uint4 b) {
  uint4 r;
  const __half2 *pa = reinterpret_cast<const __half2 *>(&a), *pb = reinterpret_cast<const __half2 *>(&b);
  __half2 *pr = reinterpret_cast<__half2 *>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) pr[j] = __hmax2(pa[j], pb[j]);
  return r;
}

__global__ void __launch_bounds__(1024) maxpool_chain_nhwc8_k(View4 x, PoolChainOut outs, int levels, int P) {
  pdl_wait_and_release();
  extern __shared__ uint4 pool_sm[];
  const int H = x.H, W = x.W, HW = H * W;
  const int b = blockIdx.y, c = blockIdx.x * 8;
  uint4 *A = pool_sm, *T = pool_sm + HW;
  for (int p = threadIdx.x; p < HW; p += blockDim.x) {
    const int yy = p / W, xx = p - yy * W;
    A[p] = *reinterpret_cast<const uint4 *>(x.ptr + at8(x, b, yy, xx, c));
  }
  __syncthreads();
  for (int l = 0; l < levels; ++l) {
    for (int p = threadIdx.x; p < HW; p += blockDim.x) {  // row pass A -> T
      const int yy = p / W, xx = p - yy * W;
      uint4 m = A[p];
#pragma unroll
      for (int d = 1; d <= kPoolChainMaxP; ++d) {
        if (d > P) break;
        if (xx - d >= 0) m = hmax8(m, A[p - d]);
        if (xx + d < W) m = hmax8(m, A[p + d]);
      }
      T[p] = m;
    }
    __syncthreads();
    const View4 &y = outs.y[l == 0 ? 0 : l == 1 ? 1 : 2];
    for (int p = threadIdx.x; p < HW; p += blockDim.x) {  // column pass T -> A, and out
      const int yy = p / W, xx = p - yy * W;
      uint4 m = T[p];
#pragma unroll
      for (int d = 1; d <= kPoolChainMaxP; ++d) {
        if (d > P) break;
        if (yy - d >= 0) m = hmax8(m, T[p - d * W]);
        if (yy + d < H) m = hmax8(m, T[p + d * W]);
      }
      A[p] = m;
      *reinterpret_cast<uint4 *>(y.ptr + at8(y, b, yy, xx, c)) = m;
    }
    __syncthreads();
  }
}

__global__ void maxpool_nhwc8_k(View4 x, View4 y, long long n8, int K, int S, int P) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const Pix p = pix8((unsigned long long)i, y);
    float m[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) m[j] = -3.4e38f;
    for (int kh = 0; kh < K; ++kh) {
      const int yy = p.y * S - P + kh;
      if (yy < 0 || yy >= x.H) continue;
      for (int kw = 0; kw < K; ++kw) {
        const int xx = p.x * S - P + kw;
        if (xx < 0 || xx >= x.W) continue;
        const uint4 v = *reinterpret_cast<const uint4 *>(x.ptr + at8(x, p.b, yy, xx, p.c));
        const __half *h = reinterpret_cast<const __half *>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) m[j] = fmaxf(m[j], __half2float(h[j]));
      }
    }
    __align__(16) __half o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __float2half_rn(m[j]);
    *reinterpret_cast<uint4 *>(y.ptr + at8(y, p.b, p.y, p.x, p.c)) = *reinterpret_cast<const uint4 *>(o);
  }
}

// binary op; `b` may broadcast over pixels (bpix = 0: per-image channel vector)
__global__ void ew_binary_nhwc8_k(View4 a, View4 b, View4 y, long long n8, int op, int bpix, int bscalar) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const Pix p = pix8((unsigned long long)i, y);
    const uint4 av = *reinterpret_cast<const uint4 *>(a.ptr + at8(a, p.b, p.y, p.x, p.c));
    const __half *ah = reinterpret_cast<const __half *>(&av);
    __align__(16) __half bh[8];
    if (bscalar) {
#pragma unroll
      for (int j = 0; j < 8; ++j) bh[j] = b.ptr[(long long)p.b * b.sb];
    } else {
      const long long bo = bpix ? at8(b, p.b, p.y, p.x, p.c) : (long long)p.b * b.sb + p.c;
      *reinterpret_cast<uint4 *>(bh) = *reinterpret_cast<const uint4 *>(b.ptr + bo);
    }
    __align__(16) __half o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __float2half_rn(binop(__half2float(ah[j]), __half2float(bh[j]), op));
    *reinterpret_cast<uint4 *>(y.ptr + at8(y, p.b, p.y, p.x, p.c)) = *reinterpret_cast<const uint4 *>(o);
  }
}

// Binary op into a channels-last output whose operands need not be
// channels-last (a planar operand, as where YOLO11's attention adds the planar
// product to the channels-last `pe` conv): a thread writes eight channels of
// one pixel, threads run over pixels fastest, so a planar operand's eight
// scalar loads are each coalesced across the warp; a channels-last operand is
// one 16-byte load.  32-bit indices through multiply-high divisions.
__device__ __forceinline__ void ew_load8(const View4 &v, bool vec, int b, int y, int x, int c, __half (&h)[8]) {
  if (vec) {
    *reinterpret_cast<uint4 *>(h) = *reinterpret_cast<const uint4 *>(v.ptr + at8(v, b, y, x, c));
  } else {
    const __half *p = v.ptr + (long long)b * v.sb + (long long)y * v.sy + (long long)x * v.sx;
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = p[(long long)(c + j) * v.sc];
  }
}
__global__ void ew_binary_mixed8_k(View4 a, View4 b, View4 y, int n8, int op, int a_vec, int b_vec, DwDiv d_w,
                                   DwDiv d_hw, DwDiv d_c8) {
  pdl_wait_and_release();
  const uint32_t HW = (uint32_t)(y.H * y.W), C8 = (uint32_t)(y.C / 8);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
    const uint32_t rest = dw_div((uint32_t)i, d_hw), p = (uint32_t)i - rest * HW;
    const uint32_t img = dw_div(rest, d_c8), c = (rest - img * C8) * 8u;
    const uint32_t yy = dw_div(p, d_w), xx = p - yy * (uint32_t)y.W;
    __align__(16) __half ah[8], bh[8], o[8];
    ew_load8(a, a_vec != 0, (int)img, (int)yy, (int)xx, (int)c, ah);
    ew_load8(b, b_vec != 0, (int)img, (int)yy, (int)xx, (int)c, bh);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __float2half_rn(binop(__half2float(ah[j]), __half2float(bh[j]), op));
    *reinterpret_cast<uint4 *>(y.ptr + at8(y, (int)img, (int)yy, (int)xx, (int)c)) = *reinterpret_cast<const uint4 *>(o);
  }
}

__global__ void ew_unary_nhwc8_k(View4 x, View4 y, long long n8, int op) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const Pix p = pix8((unsigned long long)i, y);
    const uint4 v = *reinterpret_cast<const uint4 *>(x.ptr + at8(x, p.b, p.y, p.x, p.c));
    const __half *h = reinterpret_cast<const __half *>(&v);
    __align__(16) __half o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __float2half_rn(unop(__half2float(h[j]), op));
    *reinterpret_cast<uint4 *>(y.ptr + at8(y, p.b, p.y, p.x, p.c)) = *reinterpret_cast<const uint4 *>(o);
  }
}

// planar "row" copies: concat / slice / permute move contiguous runs; each row
// is (dst offset, src pointer + offset, length), elements copied 8 at a time
// when the run and both ends are 16-byte aligned.
__global__ void concat_rows_k(ConcatArgs g, __half *__restrict__ y, long long outer, long long per_img_outer,
                              long long inner) {
  pdl_wait_and_release();
  const long long rows = outer * g.nsrc;
  for (long long r = blockIdx.y; r < rows; r += gridDim.y) {
    const int s = (int)(r % g.nsrc);
    const long long o = r / g.nsrc;
    int base = 0;
    for (int k = 0; k < s; ++k) base += g.s[k].c;
    const long long len = (long long)g.s[s].c * inner;
    const long long oo = g.s[s].shared ? (o % per_img_outer) : o;
    const __half *src = g.s[s].ptr + oo * len;
    __half *dst = y + (o * g.sum + base) * inner;
    const bool v8 = (len % 8) == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
    if (v8) {
      for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < len / 8; i += (long long)gridDim.x * blockDim.x)
        reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(src)[i];
    } else {
      for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < len; i += (long long)gridDim.x * blockDim.x)
        dst[i] = src[i];
    }
  }
}

// ---- row-vectorised planar kernels (decode tail): 8 elements per thread
__host__ __device__ __forceinline__ bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// slice_axis as rows: `outer` rows of len*inner contiguous elements
__global__ void slice_rows8_k(const __half *__restrict__ x, __half *__restrict__ y, long long outer, int axdim,
                              long long inner, int start, int len) {
  pdl_wait_and_release();
  const long long row = (long long)len * inner / 8;  // vectors per row
  const long long n = outer * row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long o = i / row, v = i - o * row;
    reinterpret_cast<uint4 *>(y + o * len * inner)[v] =
        reinterpret_cast<const uint4 *>(x + (o * axdim + start) * inner)[v];
  }
}

// permute_0213 mode 0 moves whole I-rows: [D1][D2][I] -> [D2][D1][I]
__global__ void permute0_rows8_k(const __half *__restrict__ x, __half *__restrict__ y, long long n8, int D1, int D2,
                                 long long I) {
  pdl_wait_and_release();
  const long long I8 = I / 8;
  const long long per = (long long)D1 * D2 * I;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const long long v = i % I8;
    long long t = i / I8;
    const int d2 = (int)(t % D2);
    t /= D2;
    const int d1 = (int)(t % D1);
    const long long img = t / D1;
    reinterpret_cast<uint4 *>(y + img * per + ((long long)d2 * D1 + d1) * I)[v] =
        reinterpret_cast<const uint4 *>(x + img * per + ((long long)d1 * D2 + d2) * I)[v];
  }
}

// broadcast binary op when the innermost output dim is contiguous (stride 1)
// or broadcast (stride 0) for both operands and a multiple of 8
__global__ void ew_bcast_rows8_k(const __half *__restrict__ a, const __half *__restrict__ b, __half *__restrict__ y,
                                 BcastArgs g, long long n8, int op) {
  pdl_wait_and_release();
  const int r = g.rank - 1;
  const long long last8 = g.dims[r] / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const long long v = i % last8;
    long long rem = i / last8, ai = v * 8 * g.as[r], bi = v * 8 * g.bs[r];
    for (int d = r - 1; d >= 0; --d) {
      const long long coord = rem % g.dims[d];
      rem /= g.dims[d];
      ai += coord * g.as[d];
      bi += coord * g.bs[d];
    }
    __align__(16) __half av[8], bv[8], o[8];
    if (g.as[r] == 1) {
      *reinterpret_cast<uint4 *>(av) = *reinterpret_cast<const uint4 *>(a + ai);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) av[j] = a[ai];
    }
    if (g.bs[r] == 1) {
      *reinterpret_cast<uint4 *>(bv) = *reinterpret_cast<const uint4 *>(b + bi);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) bv[j] = b[bi];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __float2half_rn(binop(__half2float(av[j]), __half2float(bv[j]), op));
    reinterpret_cast<uint4 *>(y)[i] = *reinterpret_cast<const uint4 *>(o);
  }
}

// 1x1 convolution on planar [Cin][N] rows with a handful of output channels
// (the DFL projection 16 -> 1): one thread per pixel, gemm-family epilogue,
// fp32 accumulation over ci in order.
constexpr int kPlanarMaxCout = 8;
constexpr int kPlanarMaxCin = 64;
__global__ void conv1x1_planar_k(const __half *__restrict__ x, const __half *__restrict__ w,
                                 const __half *__restrict__ bias, __half *__restrict__ y, long long npix, long long N,
                                 int Cin, int Cout, int act) {
  pdl_wait_and_release();
  __shared__ float ws[kPlanarMaxCout * kPlanarMaxCin];
  for (int i = threadIdx.x; i < Cin * Cout; i += blockDim.x) ws[i] = __half2float(w[i]);
  __syncthreads();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < npix; i += (long long)gridDim.x * blockDim.x) {
    const long long img = i / N, n = i - img * N;
    const __half *xp = x + img * Cin * N + n;
    for (int co = 0; co < Cout; ++co) {
      float acc = 0.0f;
      for (int ci = 0; ci < Cin; ++ci) acc += __half2float(xp[(long long)ci * N]) * ws[co * Cin + ci];
      y[img * Cout * N + (long long)co * N + n] = epilogue(acc, bias ? __half2float(bias[co]) : 0.0f, act, kActGemm);
    }
  }
}

// Distribution-focal-loss head in one pass: permute_0213 (mode 0) of the box
// tensor, softmax_axis over the D2 bins, then the 1x1 projection bins -> Cout.
// x [B][D1*D2][I] holds side j's bins in rows j*D2 .. +D2; y [B][Cout][D1][I].
// The arithmetic is softmax_axis_k's followed by conv1x1_planar_k's (softmax
// rounded to half, f32 accumulation in bin order, conv epilogue), without the
// two intermediate tensors.
template <int D2>
__global__ void dfl_fused_k(const __half *__restrict__ x, const __half *__restrict__ w,
                            const __half *__restrict__ bias, __half *__restrict__ y, long long n, int D1, long long I,
                            int Cout, int act) {
  pdl_wait_and_release();
  __shared__ float ws[kPlanarMaxCout * D2];
  for (int i = threadIdx.x; i < Cout * D2; i += blockDim.x) ws[i] = __half2float(w[i]);
  __syncthreads();
  const long long per = (long long)D1 * I;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long img = i / per, r = i - img * per;
    const long long j = r / I, a = r - j * I;
    const __half *xp = x + (img * D1 + j) * D2 * I + a;
    float v[D2];
#pragma unroll
    for (int k = 0; k < D2; ++k) v[k] = __half2float(xp[(long long)k * I]);
    float m = -3.4e38f;
#pragma unroll
    for (int k = 0; k < D2; ++k) m = fmaxf(m, v[k]);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < D2; ++k) {
      v[k] = expf(v[k] - m);  // the same values softmax_axis_k computes twice
      s += v[k];
    }
    float pr[D2];
#pragma unroll
    for (int k = 0; k < D2; ++k) pr[k] = __half2float(__float2half_rn(v[k] / s));
    for (int co = 0; co < Cout; ++co) {
      float acc = 0.0f;
#pragma unroll
      for (int k = 0; k < D2; ++k) acc += pr[k] * ws[co * D2 + k];
      y[(img * Cout + co) * per + r] = epilogue(acc, bias ? __half2float(bias[co]) : 0.0f, act, kActGemm);
    }
  }
}

// Fused tail program (see TailProgram): one thread per (image, V consecutive
// anchors) runs the whole op list; control flow is the same for every thread.
template <int V>
__device__ __forceinline__ void tail_fetch(const TailProgram &P, const TailOperand &o, const float *my, long long img,
                                           long long an0, float (&v)[V]) {
  if (o.kind == kTailSlot) {
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = my[o.idx * (int)blockDim.x * V + j];
  } else if (o.kind == kTailLeafRow) {
    const TailLeaf &L = P.leaves[o.idx];
    const __half *src = L.ptr + img * L.img_stride + (long long)o.row * L.row_stride + an0;
    if (V == 4) {
      const uint2 u = *reinterpret_cast<const uint2 *>(src);
      const __half2 *h = reinterpret_cast<const __half2 *>(&u);
      const float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]);
      v[0] = f0.x;
      v[1 % V] = f0.y;
      v[2 % V] = f1.x;
      v[3 % V] = f1.y;
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] = __half2float(src[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = __int_as_float(o.idx);
  }
}

template <int V>
__global__ void __launch_bounds__(128) tail_vm_k(const __grid_constant__ TailProgram P, long long n) {
  pdl_wait_and_release();
  extern __shared__ float tail_slots[];
  float *my = tail_slots + threadIdx.x * V;  // slot s at my[s * blockDim.x * V + j]
  const long long AV = P.A / V;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long img = i / AV, an0 = (i - img * AV) * V;
    const int k_end = P.comp_begin[blockIdx.y + 1];
    for (int k = P.comp_begin[blockIdx.y]; k < k_end; ++k) {
      const TailOp &op = P.ops[k];
      float r[V];
      if (op.code == kTailDfl) {  // softmax_axis_k over 16 bins, then conv1x1_planar_k's arithmetic
        const TailLeaf &L = P.leaves[op.a.idx];
        const TailDfl &D = P.dfl[op.arg];
        const __half *xp = L.ptr + img * L.img_stride + (long long)op.a.row * L.row_stride + an0;
#pragma unroll
        for (int j = 0; j < V; ++j) {
          float e[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) e[q] = __half2float(xp[(long long)q * L.row_stride + j]);
          float m = -3.4e38f;
#pragma unroll
          for (int q = 0; q < 16; ++q) m = fmaxf(m, e[q]);
          float s = 0.0f;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            e[q] = expf(e[q] - m);
            s += e[q];
          }
          float acc = 0.0f;
#pragma unroll
          for (int q = 0; q < 16; ++q) acc += __half2float(__float2half_rn(e[q] / s)) * D.w[q];
          r[j] = __half2float(epilogue(acc, D.bias, D.act, kActGemm));
        }
      } else {
        float a[V];
        tail_fetch<V>(P, op.a, my, img, an0, a);
        if (op.code == kTailBin) {
          float b[V];
          tail_fetch<V>(P, op.b, my, img, an0, b);
#pragma unroll
          for (int j = 0; j < V; ++j) r[j] = __half2float(__float2half_rn(binop(a[j], b[j], op.arg)));
        } else if (op.code == kTailUn) {
#pragma unroll
          for (int j = 0; j < V; ++j) r[j] = __half2float(__float2half_rn(unop(a[j], op.arg)));
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j) r[j] = a[j];
        }
      }
      if (op.dst >= 0) {
#pragma unroll
        for (int j = 0; j < V; ++j) my[op.dst * (int)blockDim.x * V + j] = r[j];
      }
      if (op.store_row >= 0) {
        __half *dst = P.out + img * P.out_img + (long long)op.store_row * P.A + an0;
        if (V == 4) {
          uint2 u;
          __half2 *h = reinterpret_cast<__half2 *>(&u);
          h[0] = __floats2half2_rn(r[0], r[1 % V]);
          h[1] = __floats2half2_rn(r[2 % V], r[3 % V]);
          *reinterpret_cast<uint2 *>(dst) = u;
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j) dst[j] = __float2half_rn(r[j]);
        }
      }
    }
  }
}

inline bool cfast_of(const View4 &y) { return y.sc == 1; }
inline long long numel4(const View4 &v, int batch) { return (long long)batch * v.C * v.H * v.W; }

}  // namespace

// ------------------------------------------------------------------ launchers
cudaError_t launch_ew_binary_flat(const __half *a, const __half *b, __half *y, long long n, int op, int b_scalar,
                                  long long per_img, int batch, long long a_bs, long long b_bs, cudaStream_t st) {
  (void)batch;
  if (per_img % 8 == 0 && a_bs % 8 == 0 && (b_scalar || b_bs % 8 == 0) && al16(a) && al16(y) && (b_scalar || al16(b)) &&
      n / 8 < (1LL << 31) && per_img >= 8) {
    const long long n8 = n / 8;
    const uint32_t per8 = (uint32_t)(per_img / 8);
    launch_kernel(ew_binary_flat8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, a, b, y, n8, op, b_scalar, per8, a_bs,
                  b_bs, dw_make_div(per8));
    return cudaGetLastError();
  }
  launch_kernel(ew_binary_flat_k, dim3(grid_for(n)), dim3(kThreads), 0, st, a, b, y, n, op, b_scalar, per_img, a_bs, b_bs);
  return cudaGetLastError();
}
cudaError_t launch_ew_binary_v4(View4 a, View4 b, View4 y, int batch, int op, cudaStream_t st) {
  if (vec8_ok(y) && vec8_ok(a)) {
    const bool bpix = b.sx != 0 || b.sy != 0;
    const bool bscalar = !bpix && b.sc == 0;
    if ((bpix && vec8_ok(b)) || (!bpix && !bscalar && (b.sb % 8) == 0 && (reinterpret_cast<uintptr_t>(b.ptr) & 15) == 0) ||
        bscalar) {
      const long long n8 = numel4(y, batch) / 8;
      launch_kernel(ew_binary_nhwc8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, a, b, y, n8, op, bpix ? 1 : 0, bscalar ? 1 : 0);
      return cudaGetLastError();
    }
  }
  if (vec8_ok(y) && y.C >= 8 && y.H >= 1 && y.W >= 1 && batch >= 1 &&
      numel4(y, batch) / 8 < (1LL << 31)) {  // channels-last output, mixed operands
    const long long n8 = numel4(y, batch) / 8;
    launch_kernel(ew_binary_mixed8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, a, b, y, (int)n8, op,
                  vec8_ok(a) ? 1 : 0, vec8_ok(b) ? 1 : 0, dw_make_div((uint32_t)y.W),
                  dw_make_div((uint32_t)(y.H * y.W)), dw_make_div((uint32_t)(y.C / 8)));
    return cudaGetLastError();
  }
  const long long n = numel4(y, batch);
  launch_kernel(ew_binary_v4_k, dim3(grid_for(n)), dim3(kThreads), 0, st, a, b, y, n, op, cfast_of(y));
  return cudaGetLastError();
}
cudaError_t launch_ew_binary_bcast(const __half *a, const __half *b, __half *y, const BcastArgs &g, int op,
                                   cudaStream_t st) {
  long long n = 1;
  for (int r = 0; r < g.rank; ++r) n *= g.dims[r];
  {
    const int r = g.rank - 1;
    bool rows = r >= 0 && g.dims[r] % 8 == 0 && (g.as[r] == 0 || g.as[r] == 1) && (g.bs[r] == 0 || g.bs[r] == 1) &&
                al16(y) && (g.as[r] == 0 || al16(a)) && (g.bs[r] == 0 || al16(b));
    for (int d = 0; d < r && rows; ++d)
      rows = (g.as[r] == 0 || g.as[d] % 8 == 0) && (g.bs[r] == 0 || g.bs[d] % 8 == 0);
    if (rows) {
      launch_kernel(ew_bcast_rows8_k, dim3(grid_for(n / 8)), dim3(kThreads), 0, st, a, b, y, g, n / 8, op);
      return cudaGetLastError();
    }
  }
  launch_kernel(ew_binary_bcast_k, dim3(grid_for(n)), dim3(kThreads), 0, st, a, b, y, g, n, op);
  return cudaGetLastError();
}
cudaError_t launch_ew_unary_flat(const __half *x, __half *y, long long n, int op, cudaStream_t st) {
  launch_kernel(ew_unary_flat_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, y, n, op);
  return cudaGetLastError();
}
cudaError_t launch_ew_unary_v4(View4 x, View4 y, int batch, int op, cudaStream_t st) {
  if (vec8_ok(x) && vec8_ok(y)) {
    const long long n8 = numel4(y, batch) / 8;
    launch_kernel(ew_unary_nhwc8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, x, y, n8, op);
    return cudaGetLastError();
  }
  const long long n = numel4(y, batch);
  launch_kernel(ew_unary_v4_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, y, n, op, cfast_of(y));
  return cudaGetLastError();
}
cudaError_t launch_copy_v4(View4 x, View4 y, int batch, cudaStream_t st) {
  if (vec8_ok(x) && vec8_ok(y)) {
    const long long n8 = numel4(y, batch) / 8;
    launch_kernel(copy_nhwc8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, x, y, n8);
    return cudaGetLastError();
  }
  const long long n = numel4(y, batch);
  launch_kernel(copy_v4_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, y, n, cfast_of(y));
  return cudaGetLastError();
}
cudaError_t launch_slice_axis(const __half *x, __half *y, long long outer, int axdim, long long inner, int start,
                              int len, cudaStream_t st) {
  if (((long long)len * inner) % 8 == 0 && ((long long)axdim * inner) % 8 == 0 && ((long long)start * inner) % 8 == 0 &&
      al16(x) && al16(y)) {
    const long long n8 = outer * len * inner / 8;
    launch_kernel(slice_rows8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, x, y, outer, axdim, inner, start, len);
    return cudaGetLastError();
  }
  launch_kernel(slice_axis_k, dim3(grid_for(outer * len * inner)), dim3(kThreads), 0, st, x, y, outer, axdim, inner, start, len);
  return cudaGetLastError();
}
cudaError_t launch_concat_planar(const ConcatSrc *src, int nsrc, __half *y, long long outer, long long per_img_outer,
                                 long long inner, cudaStream_t st) {
  ConcatArgs g{};
  g.nsrc = 0;
  g.sum = 0;
  for (int i = 0; i < nsrc; ++i) {
    if (src[i].c <= 0) continue;
    g.s[g.nsrc++] = src[i];
    g.sum += src[i].c;
  }
  if (g.nsrc == 0) return cudaSuccess;
  long long maxlen = 0;
  for (int i = 0; i < g.nsrc; ++i) maxlen = std::max(maxlen, (long long)g.s[i].c * inner);
  const long long rows = outer * g.nsrc;
  dim3 grid((unsigned)std::max<long long>(1, std::min<long long>((maxlen / 8 + kThreads - 1) / kThreads, 64)),
            (unsigned)std::min<long long>(rows, 65535));
  launch_kernel(concat_rows_k, dim3(grid), dim3(kThreads), 0, st, g, y, outer, per_img_outer, inner);
  return cudaGetLastError();
}
cudaError_t launch_maxpool_v4(View4 x, View4 y, int batch, int K, int S, int P, cudaStream_t st) {
  if (vec8_ok(x) && vec8_ok(y)) {
    const long long n8 = numel4(y, batch) / 8;
    launch_kernel(maxpool_nhwc8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, x, y, n8, K, S, P);
    return cudaGetLastError();
  }
  const long long n = numel4(y, batch);
  launch_kernel(maxpool_v4_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, y, n, K, S, P, cfast_of(y));
  return cudaGetLastError();
}
cudaError_t launch_maxpool_chain_v4(View4 x, const View4 *ys, int levels, int batch, int K, int P,
                                    cudaStream_t st) {
  if (levels < 1 || levels > kPoolChainMax) return cudaErrorInvalidValue;
  bool fused = vec8_ok(x) && 2LL * x.H * x.W * 16 <= 48 * 1024 && batch <= 65535 && K == 2 * P + 1 && P >= 0 &&
               P <= kPoolChainMaxP;
  for (int l = 0; l < levels; ++l) fused = fused && vec8_ok(ys[l]) && ys[l].H == x.H && ys[l].W == x.W && ys[l].C == x.C;
  if (!fused) {  // one pool per level
    View4 src = x;
    for (int l = 0; l < levels; ++l) {
      const cudaError_t e = launch_maxpool_v4(src, ys[l], batch, K, 1, P, st);
      if (e != cudaSuccess) return e;
      src = ys[l];
    }
    return cudaSuccess;
  }
  PoolChainOut outs{};
  for (int l = 0; l < levels; ++l) outs.y[l] = ys[l];
  const size_t smem = 2ull * (size_t)x.H * x.W * 16;
  const int threads = (int)std::max<long long>(32, std::min<long long>(1024, ((long long)x.H * x.W + 31) / 32 * 32));
  launch_kernel(maxpool_chain_nhwc8_k, dim3((unsigned)(x.C / 8), (unsigned)batch), dim3((unsigned)threads), smem, st, x, outs,
                levels, P);
  return cudaGetLastError();
}
cudaError_t launch_resize_nn_v4(View4 x, View4 y, int batch, int S, cudaStream_t st) {
  if (vec8_ok(x) && vec8_ok(y) && y.H == x.H * S && y.W == x.W * S && y.C == x.C &&
      (long long)batch * x.H <= 65535 && (long long)x.W * (x.C / 8) < (1LL << 31)) {
    const unsigned C8 = (unsigned)(x.C / 8), row8 = (unsigned)x.W * C8;
    const unsigned gx = (unsigned)std::min<long long>((row8 + 255) / 256, 64);
    launch_kernel(resize_up_nhwc8_k, dim3(gx, (unsigned)(batch * x.H)), dim3(256), 0, st, x, y, S, row8, C8);
    return cudaGetLastError();
  }
  if (vec8_ok(x) && vec8_ok(y)) {
    const long long n8 = numel4(y, batch) / 8;
    launch_kernel(resize_nhwc8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, x, y, n8, S);
    return cudaGetLastError();
  }
  const long long n = numel4(y, batch);
  launch_kernel(resize_nn_v4_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, y, n, S, cfast_of(y));
  return cudaGetLastError();
}
cudaError_t launch_softmax_axis(const __half *x, __half *y, long long outer, int axdim, long long inner,
                                cudaStream_t st) {
  if (inner == 1 && axdim >= 32 && axdim <= kSoftmaxRowMax) {
    const long long blocks = std::min<long long>((outer + 7) / 8, 148LL * 8);
    launch_kernel(softmax_rows_k, dim3((unsigned)blocks), dim3(256), 0, st, x, y, outer, axdim);
    return cudaGetLastError();
  }
  launch_kernel(softmax_axis_k, dim3(grid_for(outer * inner)), dim3(kThreads), 0, st, x, y, outer, axdim, inner);
  return cudaGetLastError();
}
cudaError_t launch_permute_0213(const __half *x, __half *y, int batch, int D1, int D2, long long I, int mode,
                                cudaStream_t st) {
  if (mode == 0 && I % 8 == 0 && al16(x) && al16(y)) {
    const long long n8 = (long long)batch * D1 * D2 * I / 8;
    launch_kernel(permute0_rows8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, x, y, n8, D1, D2, I);
    return cudaGetLastError();
  }
  const long long n = (long long)batch * D1 * D2 * I;
  launch_kernel(permute_0213_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, y, n, D1, D2, I, mode);
  return cudaGetLastError();
}
cudaError_t launch_gap_v4(View4 x, __half *y, int batch, cudaStream_t st) {
  if (vec8_ok(x) && (reinterpret_cast<uintptr_t>(y) & 15) == 0 && (long long)batch * (x.C / 8) < (1LL << 31)) {
    const int nq = x.C / 8;
    launch_kernel(gap_nhwc8_k, dim3((unsigned)(batch * nq)), dim3(128), 0, st, x, y, nq);
    return cudaGetLastError();
  }
  dim3 grid(batch, (x.C + 31) / 32);
  launch_kernel(gap_v4_k, dim3(grid), dim3(256), 0, st, x, y);
  return cudaGetLastError();
}
cudaError_t launch_bmm_t(const __half *A, const __half *B, __half *Y, int batch, int B1, int M, int K, int N,
                         long long a_bs, long long b_bs, int ta, int tb, cudaStream_t st) {
  const int tiles_m = (M + kBmmT - 1) / kBmmT, tiles_n = (N + kBmmT - 1) / kBmmT;
  const long long blocks = (long long)batch * B1 * tiles_m * tiles_n;
  if (blocks >= (1LL << 31)) return cudaErrorInvalidValue;
  // 16-byte chunks: aligned bases and batch offsets, rows of a multiple of 8 halves
  const int a_row = ta ? M : K, b_row = tb ? K : N;
  const int vec = (al16(A) && al16(B) && al16(Y) && a_bs % 8 == 0 && b_bs % 8 == 0 && ((long long)M * K) % 8 == 0 &&
                   ((long long)K * N) % 8 == 0 && ((long long)M * N) % 8 == 0 && a_row % 8 == 0 && b_row % 8 == 0)
                      ? 1
                      : 0;
  const dim3 g((unsigned)blocks), b(256);
  if (ta && tb) launch_kernel(bmm_tiled_k<true, true>, g, b, 0, st, A, B, Y, B1, M, K, N, a_bs, b_bs, tiles_m, tiles_n, vec);
  else if (ta) launch_kernel(bmm_tiled_k<true, false>, g, b, 0, st, A, B, Y, B1, M, K, N, a_bs, b_bs, tiles_m, tiles_n, vec);
  else if (tb) launch_kernel(bmm_tiled_k<false, true>, g, b, 0, st, A, B, Y, B1, M, K, N, a_bs, b_bs, tiles_m, tiles_n, vec);
  else launch_kernel(bmm_tiled_k<false, false>, g, b, 0, st, A, B, Y, B1, M, K, N, a_bs, b_bs, tiles_m, tiles_n, vec);
  return cudaGetLastError();
}
cudaError_t launch_bmm(const __half *A, const __half *B, __half *Y, int batch, int B1, int M, int K, int N,
                       long long a_bs, long long b_bs, cudaStream_t st) {
  if ((long long)M * N >= 64 * 64) return launch_bmm_t(A, B, Y, batch, B1, M, K, N, a_bs, b_bs, 0, 0, st);
  const long long n = (long long)batch * B1 * M * N;
  launch_kernel(bmm_k, dim3(grid_for(n)), dim3(kThreads), 0, st, A, B, Y, n, B1, M, K, N, a_bs, b_bs);
  return cudaGetLastError();
}
cudaError_t launch_bias_add(const __half *x, const __half *b, __half *y, long long per_img, int HW, int batch,
                            cudaStream_t st) {
  const long long n = per_img * batch;
  launch_kernel(bias_add_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, b, y, n, per_img, HW);
  return cudaGetLastError();
}
cudaError_t launch_depthwise_v4(View4 x, const __half *w, const __half *bias, View4 y, int batch, int K, int S, int P,
                                int act, cudaStream_t st) {
  const bool vec = x.sc == 1 && y.sc == 1 && (y.C % 8) == 0 && (x.sx % 8) == 0 && (x.sy % 8) == 0 &&
                   (x.sb % 8) == 0 && (y.sx % 8) == 0 && (y.sy % 8) == 0 && (y.sb % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(x.ptr) & 15) == 0 && (reinterpret_cast<uintptr_t>(y.ptr) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  const long long rows_nhwc = (long long)batch * y.H, rows_planar = rows_nhwc * y.C;
  const int fn = resolve_act(act, kActDepthwise);
  const bool known = fn == kFnNone || fn == kFnSilu || fn == kFnRelu || fn == kFnHswishB || fn == kFnHsigmoid;
  auto make_div = [](uint32_t dv) {
    DwDiv d{0u, 0u};
    uint32_t sh = 0;
    while ((1ull << sh) < dv) ++sh;
    d.s = sh;
    d.m = (uint32_t)(((1ull << (31 + sh)) / dv) + 1ull);
    return d;
  };
  const int strips = (y.W + 3) / 4;  // planar strips of four
  const int nstrips = (y.W + kDwNhwcStrip - 1) / kDwNhwcStrip;
  const long long strip_items = rows_nhwc * nstrips * (y.C / 8);
  // strips when they still fill the GPU twice over (at small batch the
  // one-pixel-per-thread rows kernel below has the shorter critical path)
  if (vec && known && (K == 3 || K == 5) && (S == 1 || S == 2) && strip_items < (1LL << 31) &&
      strip_items >= 148LL * 512) {
    const int C8 = y.C / 8;
    const DwDiv di = make_div((uint32_t)(nstrips * C8)), dc = make_div((uint32_t)C8), dh = make_div((uint32_t)y.H);
    const unsigned blocks = (unsigned)std::min<long long>((strip_items + 255) / 256, 148LL * 64);
#define IVB_DW_STRIP(F, KK, SS) \
  launch_kernel(depthwise_nhwc8_strip_k<F, KK, SS>, dim3(blocks), dim3(256), 0, st, x, w, bias, y, strip_items, P, C8, nstrips, di, dc, dh)
#define IVB_DW_STRIP_KS(F)                                   \
  do {                                                       \
    if (K == 3 && S == 1) IVB_DW_STRIP(F, 3, 1);             \
    else if (K == 3) IVB_DW_STRIP(F, 3, 2);                  \
    else if (S == 1) IVB_DW_STRIP(F, 5, 1);                  \
    else IVB_DW_STRIP(F, 5, 2);                              \
  } while (0)
    switch (fn) {
      case kFnSilu: IVB_DW_STRIP_KS(kFnSilu); break;
      case kFnRelu: IVB_DW_STRIP_KS(kFnRelu); break;
      case kFnHswishB: IVB_DW_STRIP_KS(kFnHswishB); break;
      case kFnHsigmoid: IVB_DW_STRIP_KS(kFnHsigmoid); break;
      default: IVB_DW_STRIP_KS(kFnNone); break;
    }
#undef IVB_DW_STRIP_KS
#undef IVB_DW_STRIP
  } else if (!vec && known && (K == 3 || K == 5) && (S == 1 || S == 2) && x.H * x.W >= 1 && y.H * y.W >= 1 &&
             x.H * x.W <= kDwPlaneMax &&
             (long long)batch * y.C < (1LL << 31) && (long long)batch * y.C >= 148LL * kDwPlanesPerBlock) {
    // small planes staged whole in shared memory (while they fill the GPU)
    const int planes = batch * y.C;
    const DwDiv dhw = make_div((uint32_t)(x.H * x.W)), dw = make_div((uint32_t)x.W), dwo = make_div((uint32_t)y.W),
                dcc = make_div((uint32_t)y.C);
    const unsigned blocks = (unsigned)((planes + kDwPlanesPerBlock - 1) / kDwPlanesPerBlock);
    // packed planes: every block's 16 planes are one aligned run of halves
    const int dense = (x.sx == 1 && x.sy == x.W && x.sc == (long long)x.H * x.W && y.C % kDwPlanesPerBlock == 0 &&
                       x.sb % 8 == 0 && (reinterpret_cast<uintptr_t>(x.ptr) & 15) == 0)
                          ? 1
                          : 0;
#define IVB_DW_PLANE(F, KK, SS)                                                                                  \
  launch_kernel(depthwise_planar_plane_k<F, KK, SS>, dim3(blocks), dim3(256), 0, st, x, w, bias, y, planes, P, dense, \
                dhw, dw, dwo, dcc)
#define IVB_DW_PLANE_KS(F)                                   \
  do {                                                       \
    if (K == 3 && S == 1) IVB_DW_PLANE(F, 3, 1);             \
    else if (K == 3) IVB_DW_PLANE(F, 3, 2);                  \
    else if (S == 1) IVB_DW_PLANE(F, 5, 1);                  \
    else IVB_DW_PLANE(F, 5, 2);                              \
  } while (0)
    switch (fn) {
      case kFnSilu: IVB_DW_PLANE_KS(kFnSilu); break;
      case kFnRelu: IVB_DW_PLANE_KS(kFnRelu); break;
      case kFnHswishB: IVB_DW_PLANE_KS(kFnHswishB); break;
      case kFnHsigmoid: IVB_DW_PLANE_KS(kFnHsigmoid); break;
      default: IVB_DW_PLANE_KS(kFnNone); break;
    }
#undef IVB_DW_PLANE_KS
#undef IVB_DW_PLANE
  } else if (!vec && known && (K == 3 || K == 5) && (S == 1 || S == 2) && rows_planar * strips < (1LL << 31) &&
             rows_planar * strips >= 148LL * 256) {
    // planar strips of four outputs (while they fill the GPU)
    const long long items = rows_planar * strips;
    const DwDiv ds = make_div((uint32_t)strips), dho = make_div((uint32_t)y.H), dcc = make_div((uint32_t)y.C);
    const unsigned blocks = (unsigned)std::min<long long>((items + 255) / 256, 148LL * 64);
#define IVB_DW_PSTRIP(F, KK, SS) \
  launch_kernel(depthwise_planar_strip_k<F, KK, SS>, dim3(blocks), dim3(256), 0, st, x, w, bias, y, items, P, strips, ds, dho, dcc)
#define IVB_DW_PSTRIP_KS(F)                                  \
  do {                                                       \
    if (K == 3 && S == 1) IVB_DW_PSTRIP(F, 3, 1);            \
    else if (K == 3) IVB_DW_PSTRIP(F, 3, 2);                 \
    else if (S == 1) IVB_DW_PSTRIP(F, 5, 1);                 \
    else IVB_DW_PSTRIP(F, 5, 2);                             \
  } while (0)
    switch (fn) {
      case kFnSilu: IVB_DW_PSTRIP_KS(kFnSilu); break;
      case kFnRelu: IVB_DW_PSTRIP_KS(kFnRelu); break;
      case kFnHswishB: IVB_DW_PSTRIP_KS(kFnHswishB); break;
      case kFnHsigmoid: IVB_DW_PSTRIP_KS(kFnHsigmoid); break;
      default: IVB_DW_PSTRIP_KS(kFnNone); break;
    }
#undef IVB_DW_PSTRIP_KS
#undef IVB_DW_PSTRIP
  } else if (!vec && known && rows_planar * y.W < (1LL << 31)) {
    const long long n = rows_planar * y.W;
    const DwDiv dhw = make_div((uint32_t)(y.H * y.W)), dwo = make_div((uint32_t)y.W), dcc = make_div((uint32_t)y.C);
    const unsigned blocks = (unsigned)std::min<long long>((n + 255) / 256, 148LL * 64);
#define IVB_DW_PFLAT(F) launch_kernel(depthwise_planar_flat_k<F>, dim3(blocks), dim3(256), 0, st, x, w, bias, y, n, K, S, P, dhw, dwo, dcc)
    switch (fn) {
      case kFnSilu: IVB_DW_PFLAT(kFnSilu); break;
      case kFnRelu: IVB_DW_PFLAT(kFnRelu); break;
      case kFnHswishB: IVB_DW_PFLAT(kFnHswishB); break;
      case kFnHsigmoid: IVB_DW_PFLAT(kFnHsigmoid); break;
      default: IVB_DW_PFLAT(kFnNone); break;
    }
#undef IVB_DW_PFLAT
  } else if (vec && known && rows_nhwc < (1LL << 31) && (long long)y.W * (y.C / 8) < (1LL << 30)) {
    // one block row per output row; blocks of 256 threads over its (ox, 8-channel) positions
    const int per_row = y.W * (y.C / 8);
    DwDiv d{0u, 0u};
    {
      const uint32_t dv = (uint32_t)(y.C / 8);
      uint32_t sh = 0;
      while ((1ull << sh) < dv) ++sh;
      d.s = sh;
      d.m = (uint32_t)(((1ull << (31 + sh)) / dv) + 1ull);
    }
    const dim3 grid((unsigned)((per_row + 255) / 256), (unsigned)std::min<long long>(rows_nhwc, 65535));
#define IVB_DW_NHWC(F) launch_kernel(depthwise_nhwc8_rows_k<F>, grid, dim3(256), 0, st, x, w, bias, y, (int)rows_nhwc, K, S, P, d)
    switch (fn) {
      case kFnSilu: IVB_DW_NHWC(kFnSilu); break;
      case kFnRelu: IVB_DW_NHWC(kFnRelu); break;
      case kFnHswishB: IVB_DW_NHWC(kFnHswishB); break;
      case kFnHsigmoid: IVB_DW_NHWC(kFnHsigmoid); break;
      default: IVB_DW_NHWC(kFnNone); break;
    }
#undef IVB_DW_NHWC
  } else if (!vec && known && rows_planar < (1LL << 31)) {
    const dim3 grid((unsigned)((y.W + 255) / 256), (unsigned)std::min<long long>(rows_planar, 65535));
    const int threads = y.W >= 256 ? 256 : ((y.W + 31) / 32) * 32;
#define IVB_DW_PLANAR(F) launch_kernel(depthwise_planar_rows_k<F>, grid, dim3(threads), 0, st, x, w, bias, y, (int)rows_planar, K, S, P)
    switch (fn) {
      case kFnSilu: IVB_DW_PLANAR(kFnSilu); break;
      case kFnRelu: IVB_DW_PLANAR(kFnRelu); break;
      case kFnHswishB: IVB_DW_PLANAR(kFnHswishB); break;
      case kFnHsigmoid: IVB_DW_PLANAR(kFnHsigmoid); break;
      default: IVB_DW_PLANAR(kFnNone); break;
    }
#undef IVB_DW_PLANAR
  } else if (vec) {
    const long long n8 = numel4(y, batch) / 8;
    launch_kernel(depthwise_nhwc8_k, dim3(grid_for(n8)), dim3(kThreads), 0, st, x, w, bias, y, n8, K, S, P, act);
  } else {
    const long long n = numel4(y, batch);
    launch_kernel(depthwise_v4_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, w, bias, y, n, K, S, P, act, cfast_of(y));
  }
  return cudaGetLastError();
}
cudaError_t launch_conv_direct_v4(View4 x, const __half *w, const __half *bias, const __half *res_ptr, View4 res,
                                  View4 y, int batch, int Cout, int K, int S, int P, int G, int act, int epi,
                                  cudaStream_t st) {
  (void)Cout;
  const long long n = numel4(y, batch);
  launch_kernel(conv_direct_v4_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, w, bias, res_ptr, res, y, n, K, S, P, G, act, epi,
                                                     cfast_of(y));
  return cudaGetLastError();
}
bool stem_params(int cin, int cout, const uint16_t *w_host, const uint16_t *b_host, std::vector<float> *blob) {
  if (!(cin == 3 && cout == 16)) return false;
  StemTcParams p;
  std::memset(&p, 0, sizeof(p));
  for (int c = 0; c < cout; ++c) {
    for (int k = 0; k < cin * 9; ++k) p.w[c][k] = w_host[(size_t)c * cin * 9 + k];  // [cout][ci][ky][kx]
    if (b_host) reinterpret_cast<uint16_t *>(&p.b8[c / 8])[c % 8] = b_host[c];
  }
  blob->assign((sizeof(p) + sizeof(float) - 1) / sizeof(float), 0.0f);
  std::memcpy(blob->data(), &p, sizeof(p));
  return true;
}

cudaError_t launch_stem3x3_v4(View4 x, const __half *w, const __half *bias, const float *blob, View4 y, int batch,
                              int Cout, int S, int P, int act, int *status, cudaStream_t st) {
  if (Cout > kStemMaxCout || x.C > 4) return cudaErrorInvalidValue;
  const long long npix = (long long)batch * y.H * y.W;
  const int vec_out = (y.sc == 1 && y.sx % 8 == 0 && y.sy % 8 == 0 && y.sb % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(y.ptr) & 15) == 0) ? 1 : 0;
  if (x.C == 3 && Cout == 16 && blob && S >= 1 && S <= 2 && P == 1) {
    StemTcParams p;
    std::memcpy(&p, blob, sizeof(p));
    switch (resolve_act(act, kActConv3x3)) {
      case kFnSilu: return launch_stem_tc_fn<kFnSilu>(x, p, y, batch, S, P, vec_out, status, st);
      case kFnHswishA: return launch_stem_tc_fn<kFnHswishA>(x, p, y, batch, S, P, vec_out, status, st);
      default: return launch_stem_tc_fn<kFnNone>(x, p, y, batch, S, P, vec_out, status, st);
    }
  }
  launch_kernel(stem3x3_k, dim3(grid_for(npix, 128)), dim3(128), 0, st, x, w, bias, y, npix, Cout, S, P, act);
  return cudaGetLastError();
}
cudaError_t launch_conv1x1_planar(const __half *x, const __half *w, const __half *bias, __half *y, int batch,
                                  long long N, int Cin, int Cout, int act, cudaStream_t st) {
  if (Cin > kPlanarMaxCin || Cout > kPlanarMaxCout) return cudaErrorInvalidValue;
  const long long npix = (long long)batch * N;
  launch_kernel(conv1x1_planar_k, dim3(grid_for(npix)), dim3(kThreads), 0, st, x, w, bias, y, npix, N, Cin, Cout, act);
  return cudaGetLastError();
}

cudaError_t launch_tail_program(const TailProgram &prog, int batch, cudaStream_t st) {
  if (prog.n_ops <= 0 || prog.n_ops > kTailMaxOps || prog.n_slots > kTailMaxSlots || prog.A < 1 ||
      prog.n_comp < 1 || prog.n_comp > kTailMaxComp)
    return cudaErrorInvalidValue;
  // four anchors per thread (8-byte loads / stores) when every row start is 8-byte aligned
  bool vec = prog.A % 4 == 0 && (reinterpret_cast<uintptr_t>(prog.out) & 7) == 0 && prog.out_img % 4 == 0;
  for (int i = 0; i < prog.n_leaves; ++i)
    vec = vec && (reinterpret_cast<uintptr_t>(prog.leaves[i].ptr) & 7) == 0 && prog.leaves[i].img_stride % 4 == 0 &&
          prog.leaves[i].row_stride % 4 == 0;
  const int threads = 128;
  const int V = vec ? 4 : 1;
  const size_t smem = (size_t)(prog.n_slots > 0 ? prog.n_slots : 1) * threads * V * sizeof(float);
  const long long n = (long long)batch * (prog.A / V);
  if (vec) {
    static std::atomic<bool> attr_set[kAttrMaxDevices];
    const cudaError_t e = ensure_dynamic_smem(tail_vm_k<4>, 96 * 1024, attr_set);
    if (e != cudaSuccess) return e;
    launch_kernel(tail_vm_k<4>, dim3(dim3(grid_for(n, threads), prog.n_comp)), dim3(threads), smem, st, prog, n);
  } else {
    launch_kernel(tail_vm_k<1>, dim3(dim3(grid_for(n, threads), prog.n_comp)), dim3(threads), smem, st, prog, n);
  }
  return cudaGetLastError();
}

bool dfl_fused_supported(int D2, int Cout) { return D2 == 16 && Cout >= 1 && Cout <= kPlanarMaxCout; }

cudaError_t launch_dfl_fused(const __half *x, const __half *w, const __half *bias, __half *y, int batch, int D1, int D2,
                             long long I, int Cout, int act, cudaStream_t st) {
  if (!dfl_fused_supported(D2, Cout)) return cudaErrorInvalidValue;
  const long long n = (long long)batch * D1 * I;
  launch_kernel(dfl_fused_k<16>, dim3(grid_for(n)), dim3(kThreads), 0, st, x, w, bias, y, n, D1, I, Cout, act);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_f16_trunc(const float *x, __half *y, long long n, cudaStream_t st) {
  launch_kernel(f32_to_f16_trunc_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, y, n);
  return cudaGetLastError();
}
cudaError_t launch_f16_to_f32(const __half *x, float *y, long long n, cudaStream_t st) {
  launch_kernel(f16_to_f32_k, dim3(grid_for(n)), dim3(kThreads), 0, st, x, y, n);
  return cudaGetLastError();
}

}  // namespace ivb
