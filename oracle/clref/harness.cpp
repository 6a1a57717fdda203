// NDRange runner for reference OpenCL kernels compiled on the CPU through
// ocl_shim.h - TEST INFRASTRUCTURE ONLY (builds oracle/_ref/libclref.so).
//
// Work-items of a work-group run on host threads when the kernel uses
// barrier(); otherwise they run one after another.  Exported wrappers take
// plain pointers (fp16 buffers as uint16 bit patterns) so that Python can call
// them with ctypes.
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "ocl_shim.h"

namespace {

struct WorkItem {
  size_t gid[3], lid[3], grp[3], gsz[3], lsz[3], ngrp[3];
};
thread_local WorkItem wi;

class GroupBarrier {
 public:
  explicit GroupBarrier(int n) : n_(n) {}
  void wait() {
    std::unique_lock<std::mutex> lk(m_);
    const long gen = gen_;
    if (++waiting_ == n_) {
      waiting_ = 0;
      ++gen_;
      cv_.notify_all();
    } else {
      cv_.wait(lk, [&] { return gen_ != gen; });
    }
  }

 private:
  std::mutex m_;
  std::condition_variable cv_;
  int n_, waiting_ = 0;
  long gen_ = 0;
};
GroupBarrier *g_bar = nullptr;

void ndrange(int dim, const size_t *gws, const size_t *lws, bool threaded, const std::function<void()> &fn) {
  size_t g[3] = {1, 1, 1}, l[3] = {1, 1, 1}, ng[3];
  for (int d = 0; d < dim; ++d) {
    g[d] = gws[d];
    l[d] = lws ? lws[d] : 1;
  }
  for (int d = 0; d < 3; ++d) ng[d] = (g[d] + l[d] - 1) / l[d];
  const size_t L = l[0] * l[1] * l[2];
  for (size_t gz = 0; gz < ng[2]; ++gz)
    for (size_t gy = 0; gy < ng[1]; ++gy)
      for (size_t gx = 0; gx < ng[0]; ++gx) {
        auto setup = [&](size_t lin) {
          const size_t lx = lin % l[0], ly = (lin / l[0]) % l[1], lz = lin / (l[0] * l[1]);
          const size_t grp[3] = {gx, gy, gz}, lid[3] = {lx, ly, lz};
          for (int d = 0; d < 3; ++d) {
            wi.lid[d] = lid[d];
            wi.grp[d] = grp[d];
            wi.gid[d] = grp[d] * l[d] + lid[d];
            wi.gsz[d] = g[d];
            wi.lsz[d] = l[d];
            wi.ngrp[d] = ng[d];
          }
        };
        if (!threaded) {
          for (size_t lin = 0; lin < L; ++lin) {
            setup(lin);
            fn();
          }
        } else {
          GroupBarrier bar((int)L);
          g_bar = &bar;
          std::vector<std::thread> th;
          th.reserve(L);
          for (size_t lin = 0; lin < L; ++lin)
            th.emplace_back([&, lin] {
              setup(lin);
              fn();
            });
          for (auto &t : th) t.join();
          g_bar = nullptr;
        }
      }
}

}  // namespace

extern "C" {
size_t get_global_id(uint d) { return d < 3 ? wi.gid[d] : 0; }
size_t get_local_id(uint d) { return d < 3 ? wi.lid[d] : 0; }
size_t get_group_id(uint d) { return d < 3 ? wi.grp[d] : 0; }
size_t get_global_size(uint d) { return d < 3 ? wi.gsz[d] : 1; }
size_t get_local_size(uint d) { return d < 3 ? wi.lsz[d] : 1; }
size_t get_num_groups(uint d) { return d < 3 ? wi.ngrp[d] : 1; }
void barrier(int) {
  if (g_bar) g_bar->wait();
}
}  // extern "C"

// ---- sub-groups: consecutive linear local ids, g_sub_group lanes each
namespace {
int g_sub_group = 16;
size_t linear_local_id() { return wi.lid[0] + wi.lid[1] * wi.lsz[0] + wi.lid[2] * wi.lsz[0] * wi.lsz[1]; }
half g_bcast_slot[1024];
}  // namespace
uint get_sub_group_local_id() { return (uint)(linear_local_id() % (size_t)g_sub_group); }
uint get_sub_group_id() { return (uint)(linear_local_id() / (size_t)g_sub_group); }
half sub_group_broadcast(half v, uint lane) {
  const size_t lin = linear_local_id();
  g_bcast_slot[lin] = v;
  barrier(0);
  const half r = g_bcast_slot[lin / (size_t)g_sub_group * (size_t)g_sub_group + lane];
  barrier(0);
  return r;
}
ushort2 intel_sub_group_block_read_us2(const ushort *p) {
  const uint lane = get_sub_group_local_id();
  ushort2 r;
  r[0] = p[lane];
  r[1] = p[lane + (uint)g_sub_group];
  return r;
}

extern "C" {

// ---- kernels compiled from the reference sources (kernels/ops.cl)
void ew_binary(const half *, const half *, half *, const int, const int, const int);
void ew_binary_bcast(const half *, const half *, half *, const int, const int, const int, const int *);
void ew_binary_ch(const half *, const half *, half *, const int, const int, const int, const int);
void ew_unary(const half *, half *, const int, const int);
void copy_c(const half *, half *, const int, const int, const int, const int);
void slice_axis(const half *, half *, const int, const int, const int, const int, const int);
void concat4(const half *, const int, const half *, const int, const half *, const int, const half *, const int,
             half *, const int, const int);
void maxpool(const half *, half *, const int, const int, const int, const int, const int, const int, const int,
             const int);
void resize_nn(const half *, half *, const int, const int, const int, const int);
void softmax_axis(const half *, half *, const int, const int, const int);
void softmax_axis_r(const half *, half *, const int, const int, const int);
void permute_0213(const half *, half *, const int, const int, const int, const int);
void gap_r(const half *, half *, const int, const int);
void bmm(const half *, const half *, half *, const int, const int, const int, const int, const int);
void bias_add(const half *, const half *, half *, const int);
// kernels/conv_general.cl
void conv_general(const half *, const half *, const half *, half *, const int, const int, const int, const int,
                  const int, const int, const int, const int, const int, const int, const int);
#define DW_DECL(k, s, a) \
  void dw_k##k##_s##s##_a##a(const half *, const half *, const half *, half *, const int, const int, const int, \
                             const int, const int);
DW_DECL(3, 1, 0) DW_DECL(3, 1, 2) DW_DECL(3, 2, 2) DW_DECL(3, 1, 3) DW_DECL(3, 2, 3) DW_DECL(5, 1, 3)
DW_DECL(5, 2, 3) DW_DECL(3, 1, 1) DW_DECL(5, 1, 4)

// kernels/gemm.cl (gemm_f16, default tiles BM=128 BN=64 BK=16 TM=8 TN=4 DBUF=1,
// SG=0), EPI=1 with activation a and RES r; the CAT4 builds take the staged B
// rows from four sources.  One build per (a, r[, CAT4]), kernel renamed.
#define GEMM_DECL(a, r)                                                                                \
  void gemm_a##a##_r##r(const half *, const half *, half *, const int, const int, const int, const half *, \
                        const half *);
#define GEMMCAT_DECL(a, r)                                                                                   \
  void gemmcat_a##a##_r##r(const half *, const half *, half *, const int, const int, const int, const half *,   \
                           const half *, const half *, const half *, const half *, const int, const int, const int, \
                           const int, const int, const int, const int);
GEMM_DECL(0, 0) GEMM_DECL(1, 0) GEMM_DECL(2, 0) GEMM_DECL(3, 0) GEMM_DECL(4, 0) GEMM_DECL(5, 0)
GEMM_DECL(0, 1) GEMM_DECL(1, 1) GEMM_DECL(3, 1)
GEMMCAT_DECL(0, 0) GEMMCAT_DECL(1, 0) GEMMCAT_DECL(1, 1)
// kernels/conv_ov.cl (conv3x3_ov), SG=16 OSV=32, the executor's default blocks
// (stride 1: OBW=8 OBH=2; stride 2: OBW=5 OBH=4), activation a, RES r.
#define OV_DECL(s, a, r)                                                                                      \
  void ov_s##s##_a##a##_r##r(const half *, const half *, const half *, const half *, half *, const int, const int, \
                             const int, const int, const int, const int);
OV_DECL(1, 0, 0) OV_DECL(1, 1, 0) OV_DECL(1, 3, 0) OV_DECL(1, 1, 1) OV_DECL(2, 0, 0) OV_DECL(2, 1, 0)
OV_DECL(2, 3, 0) OV_DECL(2, 1, 1)

// ---- ctypes entry points (fp16 buffers as void*)
#define H(p) static_cast<const half *>(p)
#define HM(p) static_cast<half *>(p)

void clref_ew_binary(const void *a, const void *b, void *y, int n, int op, int bs) {
  const size_t g[1] = {(size_t)n};
  ndrange(1, g, nullptr, false, [&] { ew_binary(H(a), H(b), HM(y), n, op, bs); });
}
void clref_ew_binary_bcast(const void *a, const void *b, void *y, int n, int op, int rank, const int *dims) {
  const size_t g[1] = {(size_t)n};
  ndrange(1, g, nullptr, false, [&] { ew_binary_bcast(H(a), H(b), HM(y), n, op, rank, dims); });
}
void clref_ew_binary_ch(const void *a, const void *b, void *y, int HW, int C, int op, int a_ch) {
  const size_t g[2] = {(size_t)HW, (size_t)C};
  ndrange(2, g, nullptr, false, [&] { ew_binary_ch(H(a), H(b), HM(y), HW, C, op, a_ch); });
}
void clref_ew_unary(const void *x, void *y, int n, int op) {
  const size_t g[1] = {(size_t)n};
  ndrange(1, g, nullptr, false, [&] { ew_unary(H(x), HM(y), n, op); });
}
void clref_copy_c(const void *x, void *y, int HW, int c0, int cnt, int dst) {
  const size_t g[1] = {(size_t)cnt * HW};
  ndrange(1, g, nullptr, false, [&] { copy_c(H(x), HM(y), HW, c0, cnt, dst); });
}
void clref_slice_axis(const void *x, void *y, int outer, int axdim, int inner, int start, int len) {
  const size_t g[1] = {(size_t)outer * len * inner};
  ndrange(1, g, nullptr, false, [&] { slice_axis(H(x), HM(y), outer, axdim, inner, start, len); });
}
void clref_concat4(const void *a, int ca, const void *b, int cb, const void *c, int cc, const void *d, int cd, void *y,
                   int outer, int inner) {
  const size_t g[3] = {(size_t)inner, (size_t)(ca + cb + cc + cd), (size_t)outer};
  ndrange(3, g, nullptr, false, [&] { concat4(H(a), ca, H(b), cb, H(c), cc, H(d), cd, HM(y), outer, inner); });
}
void clref_maxpool(const void *x, void *y, int C, int H, int W, int Ho, int Wo, int K, int S, int P) {
  const size_t g[1] = {(size_t)C * Ho * Wo};
  ndrange(1, g, nullptr, false, [&] { maxpool(H(x), HM(y), C, H, W, Ho, Wo, K, S, P); });
}
void clref_resize_nn(const void *x, void *y, int C, int H, int W, int S) {
  const size_t g[1] = {(size_t)C * H * S * W * S};
  ndrange(1, g, nullptr, false, [&] { resize_nn(H(x), HM(y), C, H, W, S); });
}
void clref_softmax_axis(const void *x, void *y, int outer, int axdim, int inner) {
  const size_t g[1] = {(size_t)outer * inner};
  ndrange(1, g, nullptr, false, [&] { softmax_axis(H(x), HM(y), outer, axdim, inner); });
}
void clref_softmax_axis_r(const void *x, void *y, int outer, int axdim, int inner) {
  const size_t g[2] = {(size_t)outer * 128, (size_t)inner}, l[2] = {128, 1};
  ndrange(2, g, l, true, [&] { softmax_axis_r(H(x), HM(y), outer, axdim, inner); });
}
void clref_permute_0213(const void *x, void *y, int D1, int D2, int I, int mode) {
  const size_t g[1] = {(size_t)D1 * D2 * I};
  ndrange(1, g, nullptr, false, [&] { permute_0213(H(x), HM(y), D1, D2, I, mode); });
}
void clref_gap_r(const void *x, void *y, int C, int HW) {
  const size_t g[1] = {(size_t)C * 128}, l[1] = {128};
  ndrange(1, g, l, true, [&] { gap_r(H(x), HM(y), C, HW); });
}
void clref_bmm(const void *A, const void *B, void *Y, int B0, int B1, int M, int K, int N) {
  const size_t g[1] = {(size_t)B0 * B1 * M * N};
  ndrange(1, g, nullptr, false, [&] { bmm(H(A), H(B), HM(Y), B0, B1, M, K, N); });
}
void clref_bias_add(const void *x, const void *b, void *y, int n, int HW) {
  const size_t g[1] = {(size_t)n};
  ndrange(1, g, nullptr, false, [&] { bias_add(H(x), H(b), HM(y), HW); });
}
void clref_conv_general(const void *x, const void *w, const void *b, void *y, int Cin, int H, int W, int Cout, int Ho,
                        int Wo, int K, int S, int P, int G, int act) {
  const size_t g[1] = {(size_t)Cout * Ho * Wo};
  ndrange(1, g, nullptr, false,
          [&] { conv_general(H(x), H(w), H(b), HM(y), Cin, H, W, Cout, Ho, Wo, K, S, P, G, act); });
}
// depthwise_f16 specialisations (compile-time DW_K / DW_S / DW_ACT, DW_P = DW_K / 2)
int clref_depthwise(const void *x, const void *w, const void *b, void *y, int C, int H, int W, int Ho, int Wo, int K,
                    int S, int act) {
  void (*fn)(const half *, const half *, const half *, half *, const int, const int, const int, const int,
             const int) = nullptr;
#define DW_PICK(k, s, a) \
  if (K == k && S == s && act == a) fn = dw_k##k##_s##s##_a##a;
  DW_PICK(3, 1, 0) DW_PICK(3, 1, 2) DW_PICK(3, 2, 2) DW_PICK(3, 1, 3) DW_PICK(3, 2, 3) DW_PICK(5, 1, 3)
  DW_PICK(5, 2, 3) DW_PICK(3, 1, 1) DW_PICK(5, 1, 4)
  if (!fn) return 1;
  const size_t g[1] = {(size_t)C * Ho * Wo};
  ndrange(1, g, nullptr, false, [&] { fn(H(x), H(w), H(b), HM(y), C, H, W, Ho, Wo); });
  return 0;
}

// C[M][N] = act(half(A[M][K] B[K][N]) + bias) (+ res), A = weights [Cout][Cin],
// B = activations [Cin][HW].  cat: B rows from b0..b3 (channel counts ca, cb,
// cc, rest; row offsets o0..o3 inside each source).  Returns 1 for a variant
// that is not built.
int clref_gemm(const void *A, const void *B, void *C, int M, int N, int K, const void *bias, const void *res, int act,
               int cat, const void *b1, const void *b2, const void *b3, int ca, int cb, int cc, int o0, int o1, int o2,
               int o3) {
  constexpr int kBM = 128, kBN = 64, kTM = 8, kTN = 4;
  const size_t l[2] = {kBN / kTN, kBM / kTM};
  const size_t g[2] = {(size_t)((N + kBN - 1) / kBN) * l[0], (size_t)((M + kBM - 1) / kBM) * l[1]};
  const bool r = res != nullptr;
  if (!cat) {
    void (*fn)(const half *, const half *, half *, const int, const int, const int, const half *, const half *) = nullptr;
#define GEMM_PICK(aa, rr) \
  if (act == aa && r == (rr != 0)) fn = gemm_a##aa##_r##rr;
    GEMM_PICK(0, 0) GEMM_PICK(1, 0) GEMM_PICK(2, 0) GEMM_PICK(3, 0) GEMM_PICK(4, 0) GEMM_PICK(5, 0)
    GEMM_PICK(0, 1) GEMM_PICK(1, 1) GEMM_PICK(3, 1)
    if (!fn) return 1;
    ndrange(2, g, l, true, [&] { fn(H(A), H(B), HM(C), M, N, K, H(bias), H(res)); });
    return 0;
  }
  void (*fc)(const half *, const half *, half *, const int, const int, const int, const half *, const half *,
             const half *, const half *, const half *, const int, const int, const int, const int, const int,
             const int, const int) = nullptr;
#define GEMMCAT_PICK(aa, rr) \
  if (act == aa && r == (rr != 0)) fc = gemmcat_a##aa##_r##rr;
  GEMMCAT_PICK(0, 0) GEMMCAT_PICK(1, 0) GEMMCAT_PICK(1, 1)
  if (!fc) return 1;
  ndrange(2, g, l, true, [&] {
    fc(H(A), H(B), HM(C), M, N, K, H(bias), H(res), H(b1), H(b2), H(b3), ca, cb, cc, o0, o1, o2, o3);
  });
  return 0;
}

// conv3x3_ov over [Cin][H][W] with pad 1; weights in the reference's [Cout][Cin][3][3]
// order, swizzled here into the kernel's OSV layout [ceil(Cout/32)][Cin][9][32]
// (zero rows past Cout).
int clref_conv3x3_ov(const void *x, const void *w, const void *bias, const void *res, void *y, int Cin, int H, int W,
                     int Cout, int Ho, int Wo, int stride, int act) {
  void (*fn)(const half *, const half *, const half *, const half *, half *, const int, const int, const int,
             const int, const int, const int) = nullptr;
  const bool r = res != nullptr;
#define OV_PICK(ss, aa, rr) \
  if (stride == ss && act == aa && r == (rr != 0)) fn = ov_s##ss##_a##aa##_r##rr;
  OV_PICK(1, 0, 0) OV_PICK(1, 1, 0) OV_PICK(1, 3, 0) OV_PICK(1, 1, 1) OV_PICK(2, 0, 0) OV_PICK(2, 1, 0)
  OV_PICK(2, 3, 0) OV_PICK(2, 1, 1)
  if (!fn) return 1;
  const int groups = (Cout + 31) / 32;
  std::vector<half> osv((size_t)groups * Cin * 9 * 32, (half)0);
  const half *wh = H(w);
  for (int co = 0; co < Cout; ++co)
    for (int ci = 0; ci < Cin; ++ci)
      for (int t = 0; t < 9; ++t)
        osv[(((size_t)(co / 32) * Cin + ci) * 9 + t) * 32 + co % 32] = wh[((size_t)co * Cin + ci) * 9 + t];
  const int obw = stride == 2 ? 5 : 8, obh = stride == 2 ? 4 : 2;
  const size_t l[3] = {1, 1, 16};
  const size_t g[3] = {(size_t)((Wo + obw - 1) / obw), (size_t)((Ho + obh - 1) / obh),
                       (size_t)((((Cout + 1) / 2) + 15) / 16) * 16};
  g_sub_group = 16;
  ndrange(3, g, l, true, [&] { fn(H(x), osv.data(), H(bias), H(res), HM(y), Cin, H, W, Cout, Ho, Wo); });
  return 0;
}
}  // extern "C"
