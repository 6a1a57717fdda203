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
//   warp 0      : TMA producer (one lane), ring of `stages` A (+B) slots
//   warp 1      : TMEM allocator + MMA issuer, `nbuf` (1 to 8) accumulator
//                 buffers used round robin, each mb M blocks of 128 pixels x
//                 BN columns
//   warps 2..17 : epilogue in `nteams` (1, 2 or 4) teams, team k drains the
//                 CTA's tiles k, k + nteams, ... (one or two buffers per team),
//                 so nteams tiles are in the epilogue at once; warp w reads
//                 TMEM lanes 32*(w%4) .. +31 (one output row each), and the
//                 team's warps of a lane quarter split the columns in
//                 8-column chunks
// The MMA warp runs its loop on all 32 lanes (waits on every lane, results
// combined with __all_sync so control flow stays uniform) and issues MMAs and
// commits from one elected lane.
// Every wait is bounded; a timeout records a status code, raises a CTA abort
// flag and all roles drain and exit (TMEM is always released).
#include <cstdio>

#include "common.cuh"
#include "conv_tc.cuh"

namespace ivb {

// Optional per-CTA cycle counters (compiled only with -DIVB_CONV_TRACE, for a
// diagnostic build of the library): where each role spends its time.
#ifdef IVB_CONV_TRACE
constexpr int kTraceSlots = 8;  // wait-empty, wait-full, wait-acc-empty, wait-acc-full, epi-work, total, tiles, kblocks
__device__ unsigned long long g_conv_trace[256 * kTraceSlots];
#define CONV_TRACE_ADD(slot, v)                                                                   \
  do {                                                                                            \
    if ((threadIdx.x & 31) == 0)                                                                  \
      atomicAdd(&g_conv_trace[(blockIdx.x & 255) * kTraceSlots + (slot)], (unsigned long long)(v)); \
  } while (0)
#define CONV_TRACE_T0() const long long trace_t0_ = clock64()
#define CONV_TRACE_SINCE(slot) CONV_TRACE_ADD(slot, clock64() - trace_t0_)
#else
#define CONV_TRACE_ADD(slot, v) ((void)0)
#define CONV_TRACE_T0() ((void)0)
#define CONV_TRACE_SINCE(slot) ((void)0)
#endif

namespace {

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, FastDiv f) {
  return (uint32_t)(((uint64_t)n * f.m) >> (31u + f.s));
}

// Epilogue role: warp w reads TMEM lane quarter (w % 4), i.e. tile rows
// 32*(w%4) .. +31 (one output pixel per thread), and with the other warps of
// its quarter splits the accumulator columns in 8-column chunks.  Every field
// of the parameter block is read once, before the tile loop: inside the loop
// the global stores and the barrier asm would otherwise force reloads.
// FAST (the common case, `epi_fast`): vector stores of whole 8-channel chunks,
// no residual, no padded N columns, so the chunk loop carries no per-chunk
// tests; with a dense channels-last 1x1 output a pixel's offset is p * o_sx.
template <int FN, bool FAST>
__device__ __forceinline__ void epilogue_role(const ConvTcArgs &a, int warp, int lane, uint32_t tmem_base,
                                              uint64_t *accf_bar, uint64_t *acce_bar, volatile int *abort_sh,
                                              volatile int *epi_go, const uint4 *bias_sh) {
  // The 16 warps form `nteams` teams; team k drains the CTA's tiles k,
  // k + nteams, ... so that nteams tiles are in the epilogue at once.  Tile i
  // of the CTA sits in accumulator buffer i % nbuf; with nbuf = 2 * nteams a
  // team alternates between two buffers, so the MMA warp fills its next tile
  // while it drains the current one.  Inside a team the (4 / nteams) warps of
  // a lane quarter split the columns in 8-column chunks.
  const int nteams = a.nteams;
  const uint32_t nbuf = (uint32_t)a.nbuf;
  const int q = warp & 3;
  const int grp = (warp - 2) >> 2;                 // 0..3: groups of four consecutive warps
  const int team = grp & (nteams - 1);
  const int sub = grp / nteams;                    // position among the team's warps of this quarter
  const int kq = 4 / nteams;                       // team warps per lane quarter
  const int team_threads = 32 * kConvEpiWarps / nteams;
  const bool team_lead = warp == 2 + 4 * team;     // its lane 0 waits for the accumulator
  const int row = q * 32 + lane;
  const bool leader = (warp == 2 && lane == 0);    // tracer
  (void)leader;
  const int ksize = a.ksize, BN = a.BN, n_tiles = a.n_tiles, cout = a.cout, mb = a.mb;
  const int num_tiles = a.m_tiles * n_tiles;
  const uint32_t m_total = (uint32_t)a.m_total;
  const int Ho = a.Ho, Wo = a.Wo, TH = a.TH, TW = a.TW, tiles_x = a.tiles_x, tiles_per_img = a.tiles_per_img;
  const FastDiv fd_nt = a.fd_ntiles, fd_tpi = a.fd_tiles_per_img, fd_tx = a.fd_tiles_x, fd_hw = a.fd_hw,
                fd_wo = a.fd_wo;
  const uint32_t hw = (uint32_t)(Ho * Wo);
  const __half *__restrict__ bias = a.bias;
  __half *__restrict__ out = a.out;
  const __half *__restrict__ res = a.res;
  const long long o_sb = a.o_sb, o_sc = a.o_sc, o_sy = a.o_sy, o_sx = a.o_sx;
  const long long r_sb = a.r_sb, r_sc = a.r_sc, r_sy = a.r_sy, r_sx = a.r_sx;
  const bool out_vec = a.out_vec != 0, res_vec = a.res_vec != 0, has_res = res != nullptr;
  const bool out_dense = a.out_dense != 0;
  const bool bias_in_smem = (n_tiles == 1 || a.resident_b != 0) && bias != nullptr;  // one N tile per CTA
  int *status = a.status;
  const long long wait_limit = a.wait_limit;
  // 3x3: this thread's pixel inside the tile is fixed
  // (halo tiles: M block j holds columns 8j .. 8j+7, so the row splits by 8)
  const int tw_row = a.halo ? 8 : TW;
  const int tyr = ksize == 1 ? 0 : a.halo ? row >> 3 : (int)fdiv((uint32_t)row, a.fd_tw);
  const int txr = ksize == 1 ? 0 : row - tyr * tw_row;
  const bool row_in_tile = row < a.tile_rows;
  // M block j of a 3x3 tile: eight columns further (halo windows) or eight
  // rows further (one box per tap: 16-pixel-wide tiles of 8 * mb rows)
  const int jx = a.halo ? 8 : 0, jy = a.halo ? 0 : 8;

  // bias of chunk cc (tile-relative column) of the current N tile; the bias is
  // padded to the N tile, so 8 values are always readable
  int n0 = 0;
  auto load_bias8 = [&](int cc) -> uint4 {
    if (bias_in_smem) return bias_sh[cc >> 3];
    if (bias != nullptr) return *reinterpret_cast<const uint4 *>(bias + n0 + cc);
    return make_uint4(0, 0, 0, 0);
  };
  volatile int *go = epi_go + 2 * team;
  uint32_t jt = 0;                                 // the team's tile count
  for (int t = blockIdx.x + team * gridDim.x; t < num_tiles; t += nteams * gridDim.x, ++jt) {
    const uint32_t ti = (uint32_t)team + jt * (uint32_t)nteams;  // the CTA's tile index
    const uint32_t buf = ti % nbuf, use = ti / nbuf;
    // One thread per team waits for the accumulator; the team's other warps
    // block in a hardware barrier (no issue slots).  The go flag is
    // double-buffered so a late reader never sees the next tile's value.
    if (team_lead) {
      if (lane == 0) {
        CONV_TRACE_T0();
        go[jt & 1u] = mbar_wait_bounded(smem_u32(&accf_bar[buf]), use & 1u, abort_sh, status, kStatusTimeoutAcc,
                                        wait_limit)
                          ? 1
                          : 0;
        CONV_TRACE_SINCE(3);
      }
      __syncwarp();  // reconverge before the warp-aligned barrier
    }
    named_bar_sync(1 + team, team_threads);
    if (!go[jt & 1u]) break;
    tc_fence_after();
#ifdef IVB_CONV_TRACE
    const long long work_t0 = clock64();
#endif
    const int mt = (int)fdiv((uint32_t)t, fd_nt);
    const int nt = t - mt * n_tiles;
    n0 = nt * BN;
    for (int j = 0; j < mb; ++j) {
      bool valid;
      long long obase, rbase;
      if (ksize == 1) {
        const uint32_t p = ((uint32_t)mt * (uint32_t)mb + (uint32_t)j) * 128u + (uint32_t)row;
        valid = p < m_total;
        if (FAST && out_dense) {
          obase = valid ? (long long)p * o_sx : 0;
          rbase = 0;
        } else {
          const uint32_t bimg = valid ? fdiv(p, fd_hw) : 0u;
          const uint32_t r2 = valid ? p - bimg * hw : 0u;
          const uint32_t oy = fdiv(r2, fd_wo), ox = r2 - oy * (uint32_t)Wo;
          obase = (long long)bimg * o_sb + (long long)oy * o_sy + (long long)ox * o_sx;
          rbase = (long long)bimg * r_sb + (long long)oy * r_sy + (long long)ox * r_sx;
        }
      } else {
        const int b = (int)fdiv((uint32_t)mt, fd_tpi);
        const int rem = mt - b * tiles_per_img;
        const int ty = (int)fdiv((uint32_t)rem, fd_tx);
        const int oy = ty * TH + tyr + jy * j, ox = (rem - ty * tiles_x) * TW + txr + jx * j;
        valid = row_in_tile && oy < Ho && ox < Wo;
        obase = (long long)b * o_sb + (long long)oy * o_sy + (long long)ox * o_sx;
        rbase = (long long)b * r_sb + (long long)oy * r_sy + (long long)ox * r_sx;
      }
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (buf * (uint32_t)mb + (uint32_t)j) * (uint32_t)BN;
      if (FAST) {
        __half *const orow = out + obase + n0;
        for (int c0 = sub * 8; c0 < BN; c0 += 16 * kq) {
          const int c1 = c0 + 8 * kq;
          const bool two = c1 < BN;  // warp-uniform
          uint32_t r[2][8];
          tmem_ld8(taddr + (uint32_t)c0, r[0]);
          if (two) tmem_ld8(taddr + (uint32_t)c1, r[1]);
          tmem_ld_wait();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int k = 0; k < 8; ++k) asm volatile("" : "+r"(r[h][k]));  // uses stay after the wait
          }
          const uint4 p0 = epilogue8<FN>(r[0], load_bias8(c0));
          if (valid) *reinterpret_cast<uint4 *>(orow + c0) = p0;
          if (two) {
            const uint4 p1 = epilogue8<FN>(r[1], load_bias8(c1));
            if (valid) *reinterpret_cast<uint4 *>(orow + c1) = p1;
          }
        }
        continue;
      }
      // two chunks per TMEM wait: c0 and c0 + 8 * kq
      for (int c0 = sub * 8; c0 < BN; c0 += 16 * kq) {
        const int c1 = c0 + 8 * kq;
        const bool two = c1 < BN;
        uint32_t r[2][8];
        tmem_ld8(taddr + (uint32_t)c0, r[0]);
        if (two) tmem_ld8(taddr + (uint32_t)c1, r[1]);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int k = 0; k < 8; ++k) asm volatile("" : "+r"(r[h][k]));  // uses stay after the wait
        }
        // one epilogue call per chunk (one call over both chunks measured slower)
        const int nch = (n0 + c0 < cout ? 1 : 0) + (two && n0 + c1 < cout ? 1 : 0);  // warp-uniform
        if (nch == 0) continue;
        uint4 packed[2];
        packed[0] = epilogue8<FN>(r[0], load_bias8(c0));
        if (nch == 2) packed[1] = epilogue8<FN>(r[1], load_bias8(c1));
        if (!valid) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h >= nch) break;
          const int ch0 = n0 + (h == 0 ? c0 : c1);
          const bool full = ch0 + 8 <= cout;
          __half *v = reinterpret_cast<__half *>(&packed[h]);
          if (has_res) {
            if (res_vec && full) {
              const uint4 rv = *reinterpret_cast<const uint4 *>(res + rbase + ch0);
              __half2 *h2 = reinterpret_cast<__half2 *>(&packed[h]);
              const __half2 *rr = reinterpret_cast<const __half2 *>(&rv);
#pragma unroll
              for (int k = 0; k < 4; ++k) h2[k] = __hadd2(h2[k], rr[k]);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                if (ch0 + e < cout)
                  v[e] = __float2half_rn(__half2float(v[e]) + __half2float(res[rbase + (long long)(ch0 + e) * r_sc]));
            }
          }
          if (out_vec && full) {
            *reinterpret_cast<uint4 *>(out + obase + ch0) = packed[h];
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (ch0 + e < cout) out[obase + (long long)(ch0 + e) * o_sc] = v[e];
          }
        }
      }
    }
    tc_fence_before();
    // one arrival per warp: single-thread arrivals on one mbarrier serialise
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&acce_bar[buf]));
#ifdef IVB_CONV_TRACE
    if (leader) {
      CONV_TRACE_ADD(4, clock64() - work_t0);
      CONV_TRACE_ADD(6, 1);
    }
#endif
  }
}

__device__ __forceinline__ const CUtensorMap *mapA_ptr(const ConvTcArgs &a, int s) {
  switch (s) {
    case 0: return &a.mapA[0];
    case 1: return &a.mapA[1];
    case 2: return &a.mapA[2];
    default: return &a.mapA[3];
  }
}

// MMAs of one k-block (ksteps k-steps of 16): halo tiles run the nine taps (each a
// start offset into the window and its weight block), M block after M block
// so that one accumulator takes its MMAs back to back.  Issued by one lane;
// tap offsets come from three strides (in 16-byte descriptor units): the
// window row `hx_u`, the pixel row `ru`, and (stride 2) the phase box
// `phase_u`; tap t's weights start t * b_tap further.
__device__ __forceinline__ void issue_kblock(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                             uint32_t b_hi, uint32_t idesc, int ksteps, bool halo, bool s2,
                                             uint32_t hx_u, uint32_t ru, uint32_t phase_u, uint32_t b_tap, int mb,
                                             uint32_t mblk_step, int BN, bool first) {
  for (int j = 0; j < mb; ++j) {
    const uint32_t d = d_tmem + (uint32_t)(j * BN), aj = a_lo + (uint32_t)j * mblk_step;
    if (halo) {
#pragma unroll
      for (int tap = 0; tap < 9; ++tap) {
        const int ky = tap / 3, kx = tap % 3;
        const uint32_t ao = s2 ? (uint32_t)((ky & 1) * 2 + (kx & 1)) * phase_u + (uint32_t)(ky >> 1) * hx_u +
                                     (uint32_t)(kx >> 1) * ru
                               : (uint32_t)ky * hx_u + (uint32_t)kx * ru;
        const uint32_t bo = (uint32_t)tap * b_tap;
#pragma unroll 1
        for (int k = 0; k < ksteps; ++k)
          umma_f16_lh(d, aj + ao + 2u * k, a_hi, b_lo + bo + 2u * k, b_hi, idesc,
                      (!first || tap != 0 || k != 0) ? 1u : 0u);
      }
    } else {
#pragma unroll 1
      for (int k = 0; k < ksteps; ++k)
        umma_f16_lh(d, aj + 2u * k, a_hi, b_lo + 2u * k, b_hi, idesc, (!first || k != 0) ? 1u : 0u);
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(kConvThreads, 1) conv_tc_kernel(const __grid_constant__ ConvTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kConvMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kConvMaxStages];
  __shared__ __align__(8) uint64_t accf_bar[kConvMaxBufs];
  __shared__ __align__(8) uint64_t acce_bar[kConvMaxBufs];
  __shared__ __align__(8) uint64_t bres_bar;
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ __align__(8) uint64_t probe_bar;  // nothing arrives on it (test probe)
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  __shared__ volatile int epi_go[2 * kConvMaxTeams];
  __shared__ uint4 bias_sh[256 / 8];  // the bias of the CTA's N tile (one N tile, or resident weights)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // parameters every role uses, read once
  const int BK = a.BK, BN = a.BN, num_kb = a.num_kb, stages = a.stages, n_tiles = a.n_tiles, mb = a.mb;
  const bool resident_b = a.resident_b != 0;
  const int num_tiles = a.m_tiles * n_tiles;
  int *const status = a.status;
  const long long wait_limit = a.wait_limit;
  // Resident weights with several N tiles: tile t is N tile t % n_tiles, and a
  // grid that is a multiple of n_tiles gives each CTA one N tile for all its
  // tiles, whose weights it keeps (checked before anything is set up).
  if (resident_b && n_tiles > 1 && gridDim.x % (unsigned)n_tiles != 0u) {
    if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadConfig);
    return;
  }
  const int nt_cta = (int)(blockIdx.x % (unsigned)n_tiles);
  // 1024-byte aligned operand area (128B-swizzle atoms repeat every 1024 B)
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  const bool halo = a.halo != 0;
  const int nphase = a.halo == 2 ? 4 : 1;  // stride-2 halo: four phase boxes
  const uint32_t a_tile = halo ? (uint32_t)(a.halo_bytes * nphase) : 128u * (uint32_t)(mb * BK) * 2u;  // bytes
  const uint32_t b_tile = (((uint32_t)BN * (uint32_t)BK * 2u) + 1023u) & ~1023u;
  const int b_blocks = halo ? num_kb * 9 : num_kb;  // resident weight blocks
  const uint32_t bres_bytes = resident_b ? b_tile * (uint32_t)b_blocks : 0u;
  const int kbs = a.kb_per_stage;                      // k-blocks per stage
  // B in the ring: one block per k-block, or (halo) the chunk's nine tap blocks
  const uint32_t b_stage = resident_b ? 0u : (halo ? 9u : 1u) * b_tile;
  const uint32_t kb_bytes = a_tile + b_stage;
  const uint32_t stage_bytes = (uint32_t)kbs * kb_bytes;
  const uint32_t bres_base = base;
  const uint32_t ring_base = base + bres_bytes;
  const uint32_t row_bytes = (uint32_t)BK * 2u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int j = 0; j < kConvMaxBufs; ++j) {
      mbar_init(smem_u32(&accf_bar[j]), 1);
      mbar_init(smem_u32(&acce_bar[j]), kConvEpiWarps / a.nteams);  // one arrival per team warp
    }
    mbar_init(smem_u32(&bres_bar), 1);
    mbar_init(smem_u32(&done_bar), 1);
    mbar_init(smem_u32(&probe_bar), 1);
    abort_sh = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < a.nsrc; ++s) tma_prefetch_desc(mapA_ptr(a, s));
    tma_prefetch_desc(&a.mapB);
    // the resident weights are constants (written once at load), so their
    // copy starts before the previous grid has finished; the thread that
    // initialised the barrier issues it
    if (resident_b) {
      mbar_expect_tx(smem_u32(&bres_bar), (uint32_t)BN * (uint32_t)BK * 2u * (uint32_t)b_blocks);
      for (int kb = 0; kb < b_blocks; ++kb)
        tma_load_2d(bres_base + (uint32_t)kb * b_tile, &a.mapB, smem_u32(&bres_bar), kb * BK, nt_cta * BN);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_base_sh), (uint32_t)a.tmem_cols);
    tmem_relinquish();
  }
  if (warp >= 2 && (n_tiles == 1 || resident_b) && a.bias != nullptr) {  // (a constant too)
    // the bias of this CTA's N tile, padded to BN (a multiple of 16), 16 B per thread
    const int i = threadIdx.x - 64;
    if (i < BN / 8) bias_sh[i] = reinterpret_cast<const uint4 *>(a.bias + nt_cta * BN)[i];
  }
  // everything above touched only shared memory, TMEM, the parameter block and
  // the constant weights and bias; activations are read after the previous grid
  pdl_wait_and_release();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
#ifdef IVB_CONV_TRACE
  const long long kernel_t0 = clock64();
#endif

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      // (one lane: a whole-warp loop here needs more registers than the
      // 576-thread CTA leaves, and one TMA box per k-block is no issue limit)
      const int ksize = a.ksize, stride = a.stride, pad = a.pad, nsrc = a.nsrc, taps = a.taps;
      const int TH = a.TH, TW = a.TW, tiles_x = a.tiles_x, tiles_per_img = a.tiles_per_img;
      const FastDiv fd_nt = a.fd_ntiles, fd_tpi = a.fd_tiles_per_img, fd_tx = a.fd_tiles_x;
      int sc[kConvMaxSrc];
#pragma unroll
      for (int i = 0; i < kConvMaxSrc; ++i) sc[i] = a.src_chunks[i];
      // bytes the A boxes of one k-block deliver: mb * 128 pixel rows (1x1),
      // TH*TW rows (3x3) or the hx*hy halo (per phase)
      const uint32_t a_tx =
          (uint32_t)(halo ? a.hx * a.hy * nphase : ksize == 1 ? 128 * mb : a.tile_rows) * (uint32_t)BK * 2u;
      const uint32_t phase_bytes = (uint32_t)a.halo_bytes;
      const uint32_t b_tx = (uint32_t)BN * (uint32_t)BK * 2u;
      const uint32_t tx_bytes = a_tx + (resident_b ? 0u : b_tx * (halo ? 9u : 1u));
      uint32_t stage = 0, wrap = 0, issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int mt = (int)fdiv((uint32_t)t, fd_nt);
        const int nt = t - mt * n_tiles;
        int p0 = 0, b = 0, iy0 = 0, ix0 = 0;
        if (ksize == 1) {
          p0 = mt * 128 * mb;
        } else {
          b = (int)fdiv((uint32_t)mt, fd_tpi);
          const int rem = mt - b * tiles_per_img;
          const int ty = (int)fdiv((uint32_t)rem, fd_tx);
          iy0 = ty * TH * stride - pad;
          ix0 = (rem - ty * tiles_x) * TW * stride - pad;
        }
        // k-block walk: chunk fastest, then tap (ky, kx), then source
        int src = 0, nc = sc[0], chunk = 0, tap = 0, ky = 0, kx = 0;
        for (int kb = 0; kb < num_kb;) {
          CONV_TRACE_T0();
          if (wrap > 0 && !mbar_wait_bounded(smem_u32(&empty_bar[stage]), (wrap - 1u) & 1u, &abort_sh, status,
                                             kStatusTimeoutEmpty, wait_limit)) {
            ok = false;
            break;
          }
          CONV_TRACE_SINCE(0);
          CONV_TRACE_ADD(7, 1);
          const uint32_t fb = smem_u32(&full_bar[stage]);
          mbar_expect_tx(fb, tx_bytes * (uint32_t)kbs);
          for (int g = 0; g < kbs; ++g, ++kb) {
            const uint32_t sa = ring_base + stage * stage_bytes + (uint32_t)g * kb_bytes;
            if (ksize == 1) {  // mb boxes of 128 pixel rows
              for (int j = 0; j < mb; ++j)
                tma_load_2d(sa + (uint32_t)j * 128u * row_bytes, mapA_ptr(a, src), fb, chunk * BK, p0 + 128 * j);
            } else if (halo) {  // the whole window once per chunk; kb counts chunks
              tma_load_4d(sa, mapA_ptr(a, src), fb, kb * BK, ix0, iy0, b);
              if (nphase == 4) {  // odd columns, odd rows, both odd
                tma_load_4d(sa + phase_bytes, mapA_ptr(a, src), fb, kb * BK, ix0 + 1, iy0, b);
                tma_load_4d(sa + 2u * phase_bytes, mapA_ptr(a, src), fb, kb * BK, ix0, iy0 + 1, b);
                tma_load_4d(sa + 3u * phase_bytes, mapA_ptr(a, src), fb, kb * BK, ix0 + 1, iy0 + 1, b);
              }
            } else {
              tma_load_4d(sa, mapA_ptr(a, src), fb, chunk * BK, ix0 + kx, iy0 + ky, b);
            }
            if (!resident_b) {
              if (halo) {  // weights of this chunk for all nine taps (K block tap * chunks + chunk)
                for (int tp = 0; tp < 9; ++tp)
                  tma_load_2d(sa + a_tile + (uint32_t)tp * b_tile, &a.mapB, fb, (tp * num_kb + kb) * BK, nt * BN);
              } else {
                tma_load_2d(sa + a_tile, &a.mapB, fb, kb * BK, nt * BN);
              }
            }
            if (++chunk == nc) {
              chunk = 0;
              if (++kx == ksize) {
                kx = 0;
                ++ky;
              }
              if (++tap == taps) {
                tap = ky = kx = 0;
                if (++src < nsrc) nc = src == 1 ? sc[1] : src == 2 ? sc[2] : sc[3];
              }
            }
          }
          ++issued;
          if (++stage == (uint32_t)stages) {
            stage = 0;
            ++wrap;
          }
        }
      }
      // drain: wait (bounded, regardless of the abort flag) until the latest load
      // issued into every ring slot has landed, so no TMA write outlives the CTA
      volatile int no_abort = 0;
      const uint32_t first = issued > (uint32_t)stages ? issued - (uint32_t)stages : 0u;
      for (uint32_t j = first; j < issued; ++j) {
        const uint32_t s = j % (uint32_t)stages;
        mbar_wait_bounded(smem_u32(&full_bar[s]), (j / (uint32_t)stages) & 1u, &no_abort, status,
                          kStatusTimeoutDrain, 400000000LL);
      }
      if (resident_b)
        mbar_wait_bounded(smem_u32(&bres_bar), 0, &no_abort, status, kStatusTimeoutDrain, 400000000LL);
    }
  } else if (warp == 1) {
    {
      // ------------------------------------------------------------ MMA issuer
      // One lane issues every MMA, so the scalar work between two MMAs is
      // pure latency: descriptors are built once and advanced by 32-bit adds on
      // their low word (start address >> 4), and the tap / k-step loops are
      // unrolled with their offsets fixed before the tile loop.
      const bool leader = elect_one();
      const uint32_t idesc = idesc_f16_f32(128, BN);
      const int ksteps = BK / 16;
      const int hx = a.hx;
      const uint32_t halo_sbo = (uint32_t)hx * row_bytes;  // one image row of the halo per 8-row group
      const uint64_t a_desc0 =
          halo ? smem_desc_kmajor_at(ring_base, row_bytes, halo_sbo, 0u) : smem_desc_kmajor(ring_base, row_bytes);
      const uint64_t b_desc0 = smem_desc_kmajor(resident_b ? bres_base : ring_base + a_tile, row_bytes);
      const uint32_t a_lo0 = (uint32_t)a_desc0, a_hi = (uint32_t)(a_desc0 >> 32);
      const uint32_t b_lo0 = (uint32_t)b_desc0, b_hi = (uint32_t)(b_desc0 >> 32);
      const uint32_t stage_step = stage_bytes >> 4, kb_step = kb_bytes >> 4, b_step = b_tile >> 4;
      // M block j of a tile: 8 rows further into the halo (its 8 columns), or
      // the next 128 pixel rows of a 1x1 A tile
      const uint32_t mblk_step = (halo ? 8u : 128u) * row_bytes >> 4;
      // halo: tap (dy, dx) starts dy*hx + dx rows into the halo, and its weights
      // are resident block tap * num_kb + chunk (streamed: the chunk's nine)
      // (stride 2: phase (ky & 1, kx & 1), row (ky >> 1) * hx + (kx >> 1))
      const bool s2 = a.halo == 2;
      const uint32_t ru = row_bytes >> 4, hx_u = (uint32_t)hx * ru, phase_u = (uint32_t)a.halo_bytes >> 4;
      const uint32_t b_tap = (uint32_t)(resident_b ? num_kb : 1) * b_step;
      bool ok = true;
      if (a.wait_probe)  // test probe: this wait runs out, and the CTA takes its abort path
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(smem_u32(&probe_bar), 0, &abort_sh, status, kStatusTimeoutProbe, wait_limit));
      if (resident_b && ok)
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(smem_u32(&bres_bar), 0, &abort_sh, status, kStatusTimeoutFull, wait_limit));
      const uint32_t nbuf = (uint32_t)a.nbuf;
      uint32_t stage = 0, wrap = 0, buf = 0, use = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        CONV_TRACE_T0();
        if (use > 0 && !__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&acce_bar[buf]), (use - 1) & 1u,
                                                                  &abort_sh, status, kStatusTimeoutAccEmpty,
                                                                  wait_limit))) {
          ok = false;
          break;
        }
        CONV_TRACE_SINCE(2);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * (uint32_t)(mb * BN);
        for (int kb = 0; kb < num_kb;) {
          CONV_TRACE_T0();
          if (!__all_sync(0xffffffffu,
                          mbar_wait_bounded(smem_u32(&full_bar[stage]), wrap & 1u, &abort_sh, status, kStatusTimeoutFull,
                                            wait_limit))) {
            ok = false;
            break;
          }
          CONV_TRACE_SINCE(1);
          tc_fence_after();
          if (leader) {  // one divergent region per stage; the loops inside are exact
            for (int g = 0; g < kbs; ++g) {
              const uint32_t a_lo = a_lo0 + stage * stage_step + (uint32_t)g * kb_step;
              const uint32_t b_lo = resident_b ? b_lo0 + (uint32_t)(kb + g) * b_step : a_lo + (a_tile >> 4);
              const bool first = kb + g == 0;
              issue_kblock(d_tmem, a_lo, a_hi, b_lo, b_hi, idesc, ksteps, halo, s2, hx_u, ru, phase_u, b_tap, mb,
                           mblk_step, BN, first);
            }
          }
          kb += kbs;
          if (leader) umma_commit(smem_u32(&empty_bar[stage]));  // slot free once these MMAs retire
          __syncwarp();
          if (++stage == (uint32_t)stages) {
            stage = 0;
            ++wrap;
          }
        }
        if (!ok) break;
        if (leader) umma_commit(smem_u32(&accf_bar[buf]));  // accumulator ready
        if (++buf == nbuf) {
          buf = 0;
          ++use;
        }
      }
      // every MMA issued by this warp must retire before TMEM is released
      volatile int no_abort = 0;
      __syncwarp();
      if (leader) umma_commit(smem_u32(&done_bar));
      __syncwarp();
      mbar_wait_bounded(smem_u32(&done_bar), 0, &no_abort, status, kStatusTimeoutDrain, 400000000LL);
    }
  } else {
    // -------------------------------------------------------------- epilogue
#define IVB_EPI(F)                                                                                    \
  (a.epi_fast ? epilogue_role<F, true>(a, warp, lane, tmem_base, accf_bar, acce_bar, &abort_sh, epi_go, bias_sh) \
              : epilogue_role<F, false>(a, warp, lane, tmem_base, accf_bar, acce_bar, &abort_sh, epi_go, bias_sh))
    switch (a.act_fn) {
      case kFnSilu: IVB_EPI(kFnSilu); break;
      case kFnRelu: IVB_EPI(kFnRelu); break;
      case kFnHswishA: IVB_EPI(kFnHswishA); break;
      case kFnHsigmoid: IVB_EPI(kFnHsigmoid); break;
      case kFnSigmoid: IVB_EPI(kFnSigmoid); break;
      default: IVB_EPI(kFnNone); break;
    }
#undef IVB_EPI
  }

  tc_fence_before();
  __syncthreads();
#ifdef IVB_CONV_TRACE
  if (threadIdx.x == 0) CONV_TRACE_ADD(5, clock64() - kernel_t0);
#endif
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)a.tmem_cols);
  }
}

#ifdef IVB_CONV_TRACE
extern "C" int ivb_conv_trace_read(unsigned long long *dst, int n, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(dst, g_conv_trace, sizeof(unsigned long long) * (size_t)n);
  if (e == cudaSuccess && clear) {
    static unsigned long long zeros[256 * kTraceSlots] = {};
    e = cudaMemcpyToSymbol(g_conv_trace, zeros, sizeof(zeros));
  }
  return (int)e;
}
#endif

FastDiv make_fastdiv(uint32_t d) {
  FastDiv f{0u, 0u};
  if (d == 0) return f;
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  f.s = s;
  f.m = (uint32_t)(((1ull << (31 + s)) / d) + 1ull);
  return f;
}

bool conv_tc_finalize(ConvTcArgs &a, const char **why) {
  const long long lim = (1ll << 31) - 1;
  if (a.mb < 1 || a.mb > 8 || a.m_total > lim - 128LL * a.mb || (long long)a.m_tiles * a.n_tiles > lim || (long long)a.Ho * a.Wo > lim) {
    if (why) *why = "conv output too large for 32-bit tile indexing";
    return false;
  }
  if (a.kb_per_stage < 1 || a.num_kb % a.kb_per_stage != 0) {
    if (why) *why = "conv k-blocks per stage must divide the k-block count";
    return false;
  }
  if (a.mb < 1 || (a.mb > 1 && a.ksize == 3 && !a.halo && (a.TW != 16 || a.TH != 8 * a.mb))) {
    if (why) *why = "conv M blocks per tile out of range";
    return false;
  }
  if (a.BN > 256 || (a.nteams != 1 && a.nteams != 2 && a.nteams != 4) ||
      (a.nbuf != a.nteams && a.nbuf != 2 * a.nteams) || a.nbuf > kConvMaxBufs || a.nbuf * a.mb * a.BN > a.tmem_cols ||
      a.tmem_cols > 512) {
    if (why) *why = "conv N tile / accumulator buffers out of range";
    return false;
  }
  a.fd_ntiles = make_fastdiv((uint32_t)a.n_tiles);
  a.fd_tiles_per_img = make_fastdiv((uint32_t)a.tiles_per_img);
  a.fd_tiles_x = make_fastdiv((uint32_t)a.tiles_x);
  a.fd_tw = make_fastdiv((uint32_t)a.TW);
  a.fd_hw = make_fastdiv((uint32_t)(a.Ho * a.Wo));
  a.fd_wo = make_fastdiv((uint32_t)a.Wo);
  return true;
}

cudaError_t launch_conv_tc(const ConvTcArgs &args, int grid, cudaStream_t stream) {
  static std::atomic<bool> attr_set[kAttrMaxDevices];
  const cudaError_t e = ensure_dynamic_smem(conv_tc_kernel, 232448 - 1024, attr_set);
  if (e != cudaSuccess) return e;
  return launch_kernel(conv_tc_kernel, dim3(grid), dim3(kConvThreads), (size_t)args.smem_bytes, stream, args);
}

}  // namespace ivb
