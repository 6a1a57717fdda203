// Parameter block of the tcgen05 implicit-GEMM convolution (1x1 / 3x3, stride
// 1 or 2, up to four concatenated NHWC sources), shared by host and device.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

namespace ivb {

constexpr int kConvMaxSrc = 4;
constexpr int kConvMaxStages = 12;
constexpr int kConvEpiWarps = 16;   // four groups of four warps (one per TMEM lane quarter)
constexpr int kConvMaxTeams = 4;    // epilogue teams (tiles in the epilogue at once)
constexpr int kConvMaxBufs = 8;     // TMEM accumulator buffers (one or two per team)
constexpr int kConvThreads = 64 + 32 * kConvEpiWarps;  // warp0 TMA, warp1 MMA, then epilogue

// Division by a launch-invariant divisor as a multiply-high:
//   q = (n * m) >> (31 + s),  s = ceil(log2 d),  m = floor(2^(31+s) / d) + 1,
// exact for 0 <= n < 2^31 and 1 <= d < 2^31 (n * (m - 2^(31+s)/d) < 2^(31+s)/d).
struct FastDiv {
  uint32_t m;
  uint32_t s;
};
FastDiv make_fastdiv(uint32_t d);  // host (conv_tc.cu)

struct alignas(64) ConvTcArgs {
  CUtensorMap mapA[kConvMaxSrc];  // 1x1: 2-D (C, pixels); 3x3: 4-D (C, W, H, B)
  CUtensorMap mapB;               // packed weights, 2-D (Kp, Np), K-major
  int ksize;                      // 1 or 3
  int stride, pad;
  int nsrc;
  int src_chunks[kConvMaxSrc];    // BK-chunks per source
  int taps;                       // ksize * ksize
  int BK;                         // 16 / 32 / 64 halves (one swizzle span)
  int BN;                         // N tile, multiple of 16, <= 256
  int n_tiles;                    // Np / BN
  int num_kb;                     // K blocks per tile
  int stages;
  int kb_per_stage;               // k-blocks per pipeline stage (divides num_kb)
  int resident_b;                 // 1: all of B stays in smem
  // M tiling: a tile is mb M blocks of 128 output pixels, accumulated side by
  // side in TMEM (columns j*BN .. of the tile's buffer for block j)
  long long m_total;              // pixels (B*Ho*Wo)
  int m_tiles;
  int mb;                         // M blocks per tile (3x3 with one box per tap: only 16-wide tiles)
  int Ho, Wo, TH, TW, tiles_x, tiles_per_img;
  int tile_rows;                  // rows of an M block that hold pixels (TH*TW or 128)
  // 3x3 halo mode (halo = the stride, 1 or 2; 0 = one box per tap): the input
  // window of a TW = 8*mb x TH = 16 output tile is loaded once per channel
  // chunk and feeds all nine taps, a tap being a descriptor start offset of
  // whole rows, and M block j the eight columns 8j .. 8j+7 (an offset of 8j
  // rows).  Stride 1: one (TW+2) x 18 box.  Stride 2: four phase boxes (even /
  // odd rows x columns, TMA element stride 2) of (TW+1) x 17 pixels; tap
  // (ky, kx) reads phase (ky & 1, kx & 1) from row (ky >> 1) * hx + (kx >> 1).
  // num_kb then counts channel chunks, and the weights stay resident.
  int halo;
  int hx, hy;                     // one halo / phase box in pixels
  int halo_bytes;                 // smem bytes of one box (1024-aligned)
  // epilogue
  const __half *bias;             // [Np] or null
  int cout;
  int act, act_kind;
  int act_fn;                     // resolve_act(act, act_kind)
  __half *out;
  long long o_sb, o_sc, o_sy, o_sx;
  int out_vec;                    // NHWC-contiguous channels, 16B aligned
  int out_dense;                  // 1x1: dense channels-last output (pixel p at p * o_sx)
  int epi_fast;                   // out_vec, no residual, no padded N columns: the plain epilogue
  const __half *res;
  long long r_sb, r_sc, r_sy, r_sx;
  int res_vec;
  int tmem_cols;
  int nteams;                     // epilogue teams: 1, 2 or 4
  int nbuf;                       // accumulator buffers: nteams or 2 * nteams
  int smem_bytes;
  int *status;
  // bounded waits: the limit of every working wait in SM clocks (drains keep
  // their own), and a test probe: when nonzero the MMA warp first waits on a
  // barrier that nothing arrives on, so the wait runs out and the kernel takes
  // its abort path and reports kStatusTimeoutProbe
  long long wait_limit;
  int wait_probe;
  // derived by conv_tc_finalize(): divisors of the per-tile index arithmetic
  FastDiv fd_ntiles, fd_tiles_per_img, fd_tiles_x, fd_tw, fd_hw, fd_wo;
};

// Fills the derived fields and checks the 32-bit index ranges the kernel uses;
// returns false (with a message) when a size is out of range.
bool conv_tc_finalize(ConvTcArgs &args, const char **why);

// Host-side launcher (conv_tc.cu).
cudaError_t launch_conv_tc(const ConvTcArgs &args, int grid, cudaStream_t stream);

}  // namespace ivb
