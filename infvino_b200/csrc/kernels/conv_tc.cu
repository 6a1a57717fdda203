// tcgen05 implicit-GEMM convolution for sm_100a.
//
// GEMM view: D[M = output pixels][N = Cout] = A[M][K] * B[N][K]^T with
//   K = sum over sources s of taps * ceil(C_s / BK) * BK  (zero-padded chunks).
// A tiles come straight from NHWC activations through TMA (the 3x3 halo shift is
// a TMA coordinate offset, padding is TMA out-of-bounds zero fill, stride 2 is a
// TMA element stride), B is the repacked K-major weight matrix.  Accumulation is
// fp32 in TMEM; the epilogue applies the reference's rounding sequence
// (half(acc) + bias -> act -> + residual, each rounded to fp16) and writes any
// strided 4-D view (NHWC or planar NCHW).
//
// Persistent, warp-specialised CTA (one per SM):
//   warp 0      : TMA producer (one elected lane), ring of `stages` A (+B) slots
//   warp 1      : TMEM allocator + MMA issuer (one lane), two accumulator buffers
//   warps 2..17 : epilogue; warp w reads TMEM lanes 32*(w%4) .. +31 (one output
//                 row each) and, with the other three warps of its lane quarter,
//                 splits the accumulator columns in 8-column chunks
// Every wait is bounded; a timeout records a status code, raises a CTA abort
// flag and all roles drain and exit (TMEM is always released).
#include <cstdio>

#include "common.cuh"
#include "conv_tc.cuh"

namespace ivb {

namespace {

struct TileCoord {
  int m, n;          // m tile, n tile
  int b, oy0, ox0;   // 3x3: image and output origin
  long long p0;      // 1x1: first pixel
};

__device__ __forceinline__ TileCoord decode_tile(const ConvTcArgs &a, int t) {
  TileCoord c;
  c.m = t / a.n_tiles;
  c.n = t - c.m * a.n_tiles;
  if (a.ksize == 1) {
    c.p0 = (long long)c.m * 128;
    c.b = c.oy0 = c.ox0 = 0;
  } else {
    c.b = c.m / a.tiles_per_img;
    const int rem = c.m - c.b * a.tiles_per_img;
    const int ty = rem / a.tiles_x;
    c.oy0 = ty * a.TH;
    c.ox0 = (rem - ty * a.tiles_x) * a.TW;
    c.p0 = 0;
  }
  return c;
}

// k-block -> (source, tap, chunk)
__device__ __forceinline__ void decode_kb(const ConvTcArgs &a, int kb, int &src, int &tap, int &chunk) {
  src = 0;
  int base = 0;
#pragma unroll 1
  for (int s = 0; s < a.nsrc; ++s) {
    const int n = a.taps * a.src_chunks[s];
    if (kb < base + n) {
      src = s;
      break;
    }
    base += n;
  }
  const int r = kb - base;
  const int nc = a.src_chunks[src];
  tap = r / nc;
  chunk = r - tap * nc;
}

__device__ __forceinline__ const CUtensorMap *mapA_ptr(const ConvTcArgs &a, int s) {
  switch (s) {
    case 0: return &a.mapA[0];
    case 1: return &a.mapA[1];
    case 2: return &a.mapA[2];
    default: return &a.mapA[3];
  }
}

// Epilogue role: warp w reads TMEM lane quarter (w % 4), i.e. tile rows
// 32*(w%4) .. +31 (one output pixel per thread), and with the other warps of
// its quarter splits the accumulator columns in 8-column chunks.
template <int FN>
__device__ __forceinline__ void epilogue_role(const ConvTcArgs &a, int warp, int lane, uint32_t tmem_base,
                                              uint64_t *accf_bar, uint64_t *acce_bar, volatile int *abort_sh) {
  constexpr int kGroups = kConvEpiWarps / 4;  // warps per lane quarter
  const int q = warp & 3;
  const int grp = (warp - 2) >> 2;
  const int row = q * 32 + lane;
  const int num_tiles = a.m_tiles * a.n_tiles;
  uint32_t tcount = 0;
  for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tcount) {
    const uint32_t buf = tcount & 1u;
    if (!mbar_wait_bounded(smem_u32(&accf_bar[buf]), (tcount >> 1) & 1u, abort_sh, a.status, kStatusTimeoutAcc))
      break;
    tc_fence_after();
    const TileCoord tc = decode_tile(a, t);
    bool valid;
    long long obase, rbase;
    if (a.ksize == 1) {
      const long long p = tc.p0 + row;
      valid = p < a.m_total;
      const long long hw = (long long)a.Ho * a.Wo;
      const long long bimg = valid ? p / hw : 0;
      const long long r2 = valid ? p - bimg * hw : 0;
      const long long oy = r2 / a.Wo, ox = r2 - oy * a.Wo;
      obase = bimg * a.o_sb + oy * a.o_sy + ox * a.o_sx;
      rbase = bimg * a.r_sb + oy * a.r_sy + ox * a.r_sx;
    } else {
      const int ty = row / a.TW, tx = row - ty * a.TW;
      const int oy = tc.oy0 + ty, ox = tc.ox0 + tx;
      valid = row < a.tile_rows && oy < a.Ho && ox < a.Wo;
      obase = (long long)tc.b * a.o_sb + (long long)oy * a.o_sy + (long long)ox * a.o_sx;
      rbase = (long long)tc.b * a.r_sb + (long long)oy * a.r_sy + (long long)ox * a.r_sx;
    }
    const int n0 = tc.n * a.BN;
    const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * (uint32_t)a.BN;
    for (int c0 = grp * 8; c0 < a.BN; c0 += 8 * kGroups) {
      uint32_t r[8];
      tmem_ld8(taddr + (uint32_t)c0, r);
      tmem_ld_wait();
      const int ch0 = n0 + c0;
      if (!valid || ch0 >= a.cout) continue;
      const bool full = ch0 + 8 <= a.cout;
      // the bias is padded to the N tile, so 8 values are always readable
      const uint4 bias8 = a.bias != nullptr ? *reinterpret_cast<const uint4 *>(a.bias + ch0) : make_uint4(0, 0, 0, 0);
      uint4 packed = epilogue8<FN>(r, bias8);
      __half *v = reinterpret_cast<__half *>(&packed);
      if (a.res != nullptr) {
        if (a.res_vec && full) {
          const uint4 rv = *reinterpret_cast<const uint4 *>(a.res + rbase + ch0);
          __half2 *h2 = reinterpret_cast<__half2 *>(&packed);
          const __half2 *r2 = reinterpret_cast<const __half2 *>(&rv);
#pragma unroll
          for (int k = 0; k < 4; ++k) h2[k] = __hadd2(h2[k], r2[k]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (ch0 + j < a.cout)
              v[j] = __float2half_rn(__half2float(v[j]) + __half2float(a.res[rbase + (long long)(ch0 + j) * a.r_sc]));
        }
      }
      if (a.out_vec && full) {
        *reinterpret_cast<uint4 *>(a.out + obase + ch0) = packed;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (ch0 + j < a.cout) a.out[obase + (long long)(ch0 + j) * a.o_sc] = v[j];
      }
    }
    tc_fence_before();
    mbar_arrive(smem_u32(&acce_bar[buf]));
  }
}

}  // namespace

__global__ void __launch_bounds__(kConvThreads, 1) conv_tc_kernel(const __grid_constant__ ConvTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kConvMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kConvMaxStages];
  __shared__ __align__(8) uint64_t accf_bar[2];
  __shared__ __align__(8) uint64_t acce_bar[2];
  __shared__ __align__(8) uint64_t bres_bar;
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // 1024-byte aligned operand area (128B-swizzle atoms repeat every 1024 B)
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  const uint32_t a_tile = 128u * (uint32_t)a.BK * 2u;                       // bytes
  const uint32_t b_tile = (((uint32_t)a.BN * (uint32_t)a.BK * 2u) + 1023u) & ~1023u;
  const uint32_t bres_bytes = a.resident_b ? b_tile * (uint32_t)a.num_kb : 0u;
  const uint32_t stage_bytes = a_tile + (a.resident_b ? 0u : b_tile);
  const uint32_t bres_base = base;
  const uint32_t ring_base = base + bres_bytes;
  const uint32_t row_bytes = (uint32_t)a.BK * 2u;
  const int stages = a.stages;
  const int num_tiles = a.m_tiles * a.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(smem_u32(&accf_bar[j]), 1);
      mbar_init(smem_u32(&acce_bar[j]), 32 * kConvEpiWarps);
    }
    mbar_init(smem_u32(&bres_bar), 1);
    mbar_init(smem_u32(&done_bar), 1);
    abort_sh = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < a.nsrc; ++s) tma_prefetch_desc(mapA_ptr(a, s));
    tma_prefetch_desc(&a.mapB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_base_sh), (uint32_t)a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      // bytes one A box delivers: 128 pixel rows (1x1) or TH*TW rows (3x3)
      const uint32_t a_tx = (uint32_t)(a.ksize == 1 ? 128 : a.tile_rows) * (uint32_t)a.BK * 2u;
      const uint32_t b_tx = (uint32_t)a.BN * (uint32_t)a.BK * 2u;
      if (a.resident_b) {
        mbar_expect_tx(smem_u32(&bres_bar), b_tx * (uint32_t)a.num_kb);
        for (int kb = 0; kb < a.num_kb; ++kb)
          tma_load_2d(bres_base + (uint32_t)kb * b_tile, &a.mapB, smem_u32(&bres_bar), kb * a.BK, 0);
      }
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile(a, t);
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const uint32_t s = it % (uint32_t)stages;
          const uint32_t use = it / (uint32_t)stages;
          if (use > 0 && !mbar_wait_bounded(smem_u32(&empty_bar[s]), (use - 1) & 1u, &abort_sh, a.status,
                                             kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full_bar[s]);
          const uint32_t sa = ring_base + s * stage_bytes;
          mbar_expect_tx(fb, a_tx + (a.resident_b ? 0u : b_tx));
          int src, tap, chunk;
          decode_kb(a, kb, src, tap, chunk);
          if (a.ksize == 1) {
            tma_load_2d(sa, mapA_ptr(a, src), fb, chunk * a.BK, (int)tc.p0);
          } else {
            const int ky = tap / 3, kx = tap - ky * 3;
            tma_load_4d(sa, mapA_ptr(a, src), fb, chunk * a.BK, tc.ox0 * a.stride - a.pad + kx,
                        tc.oy0 * a.stride - a.pad + ky, tc.b);
          }
          if (!a.resident_b) tma_load_2d(sa + a_tile, &a.mapB, fb, kb * a.BK, tc.n * a.BN);
        }
      }
      // drain: wait (bounded, regardless of the abort flag) until the latest load
      // issued into every ring slot has landed, so no TMA write outlives the CTA
      volatile int no_abort = 0;
      const uint32_t issued = it;
      const uint32_t first = issued > (uint32_t)stages ? issued - (uint32_t)stages : 0u;
      for (uint32_t j = first; j < issued; ++j) {
        const uint32_t s = j % (uint32_t)stages;
        mbar_wait_bounded(smem_u32(&full_bar[s]), (j / (uint32_t)stages) & 1u, &no_abort, a.status,
                          kStatusTimeoutDrain, 400000000LL);
      }
      if (a.resident_b)
        mbar_wait_bounded(smem_u32(&bres_bar), 0, &no_abort, a.status, kStatusTimeoutDrain, 400000000LL);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_f16_f32(128, a.BN);
      bool ok = true;
      if (a.resident_b)
        ok = mbar_wait_bounded(smem_u32(&bres_bar), 0, &abort_sh, a.status, kStatusTimeoutFull);
      uint32_t it = 0, tcount = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tcount) {
        const uint32_t buf = tcount & 1u;
        const uint32_t use = tcount >> 1;
        if (use > 0 && !mbar_wait_bounded(smem_u32(&acce_bar[buf]), (use - 1) & 1u, &abort_sh, a.status,
                                           kStatusTimeoutAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * (uint32_t)a.BN;
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const uint32_t s = it % (uint32_t)stages;
          if (!mbar_wait_bounded(smem_u32(&full_bar[s]), (it / (uint32_t)stages) & 1u, &abort_sh, a.status,
                                 kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = ring_base + s * stage_bytes;
          const uint32_t sb = a.resident_b ? bres_base + (uint32_t)kb * b_tile : sa + a_tile;
          for (int k = 0; k < a.BK / 16; ++k) {
            const uint64_t ad = smem_desc_kmajor(sa + (uint32_t)k * 32u, row_bytes);
            const uint64_t bd = smem_desc_kmajor(sb + (uint32_t)k * 32u, row_bytes);
            umma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&empty_bar[s]));  // slot free once these MMAs retire
        }
        if (!ok) break;
        umma_commit(smem_u32(&accf_bar[buf]));   // accumulator ready
      }
      // every MMA issued by this thread must retire before TMEM is released
      volatile int no_abort = 0;
      umma_commit(smem_u32(&done_bar));
      mbar_wait_bounded(smem_u32(&done_bar), 0, &no_abort, a.status, kStatusTimeoutDrain, 400000000LL);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    switch (a.act_fn) {
      case kFnSilu: epilogue_role<kFnSilu>(a, warp, lane, tmem_base, accf_bar, acce_bar, &abort_sh); break;
      case kFnRelu: epilogue_role<kFnRelu>(a, warp, lane, tmem_base, accf_bar, acce_bar, &abort_sh); break;
      case kFnHswishA: epilogue_role<kFnHswishA>(a, warp, lane, tmem_base, accf_bar, acce_bar, &abort_sh); break;
      case kFnHsigmoid: epilogue_role<kFnHsigmoid>(a, warp, lane, tmem_base, accf_bar, acce_bar, &abort_sh); break;
      case kFnSigmoid: epilogue_role<kFnSigmoid>(a, warp, lane, tmem_base, accf_bar, acce_bar, &abort_sh); break;
      default: epilogue_role<kFnNone>(a, warp, lane, tmem_base, accf_bar, acce_bar, &abort_sh); break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)a.tmem_cols);
  }
}

cudaError_t launch_conv_tc(const ConvTcArgs &args, int grid, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - 1024);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  conv_tc_kernel<<<grid, kConvThreads, args.smem_bytes, stream>>>(args);
  return cudaGetLastError();
}

}  // namespace ivb
