// CPU oracle for the plan executor - TEST INFRASTRUCTURE ONLY.
//
// This file restates, on the CPU, the arithmetic of the reference's plan-driven
// executor (infvino `PlanModel`, src/PlanModel.cpp) so that the CUDA path can be
// checked against it.  It is used by tests/, by `__graft_entry__.smoke()` and by
// bench.py's CPU-baseline leg, never by the product path.
//
// What it follows (citations are paths inside the reference project):
//   * plan grammar ................ src/PlanModel.cpp:447-538 (`PlanModel::parse`)
//   * per-op attribute semantics .. src/PlanModel.cpp:3127-4178 (`run`) and
//                                   src/PlanModel.cpp:2681-3088 (`smallLaunch`)
//   * conv3x3 epilogue ............ kernels/conv_ov.cl:121-131, 255-297
//   * conv1x1 epilogue ............ kernels/gemm.cl:137-153, 644-652;
//                                   kernels/conv1x1.cl:52-68, 159-198 (N == 1)
//   * depthwise ................... kernels/conv_general.cl:71-116 (`depthwise_f16`)
//   * generic conv ................ kernels/conv_general.cl:7-49 (`conv_general`;
//                                   act codes 2 = HardSwish, 3 = ReLU there)
//   * small ops ................... kernels/ops.cl (ew_binary[_bcast], ew_unary,
//                                   copy_c, slice_axis, concat4, maxpool,
//                                   resize_nn, softmax_axis, permute_0213,
//                                   gap_r (GAP_WGS=128 tree), bmm, bias_add)
//   * f32 <-> f16 host conversion . include/infvino/Half.hpp:14-49 (truncating)
//
// Rounding points (all node outputs are fp16, round-to-nearest-even):
//   conv / gemm epilogue: v = half(half(acc) + bias); v = act(v) in f32 -> half;
//   residual add in half.  Elementwise, softmax and gap compute in f32 and round
//   once.  Accumulation is fp32 (the build's contract; the reference kernels
//   accumulate most convolutions in fp16, which this oracle does not emulate).
//   Because f32 carries 24 >= 2*11+2 significand bits, computing a half+half in
//   f32 and rounding to half equals the correctly rounded half addition.
//
// The load-time fusions of the reference (concat->conv1x1 "CAT4", conv->add
// "RES") change no numerics, so the oracle runs the plan unfused.
//
// Batch: every plan tensor declares batch 1 in dim 0.  The oracle runs the plan
// for B images by running each node once per image with per-image offsets for
// activations (initializers are shared).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace ivref {

// ---------------------------------------------------------------- fp16 helpers
static inline float h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t f;
  if (exp == 0) {
    if (mant == 0) {
      f = sign;
    } else {  // subnormal half -> normal float
      int e = 113;
      while (!(mant & 0x400u)) { mant <<= 1; --e; }
      mant &= 0x3ffu;
      f = sign | ((uint32_t)e << 23) | (mant << 13);
    }
  } else if (exp == 31) {
    f = sign | 0x7f800000u | (mant << 13);
  } else {
    f = sign | ((exp + 112u) << 23) | (mant << 13);
  }
  float out;
  std::memcpy(&out, &f, 4);
  return out;
}

// IEEE round-to-nearest-even float -> half (subnormals, inf and NaN handled).
static inline uint16_t f2h(float v) {
  uint32_t x;
  std::memcpy(&x, &v, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
  if (ax < 0x38800000u) {                                     // half subnormal or zero
    if (ax < 0x33000000u) return (uint16_t)sign;              // < 2^-25: rounds to 0
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;  // value = m * 2^(e-150); half ulp = 2^-24
    uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1u);
    if (rem > halfway || (rem == halfway && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
  }
  uint32_t r = ax - 0x38000000u;  // rebias exponent 127 -> 15 (in the shifted field)
  const uint32_t rem = r & 0x1fffu;
  r >>= 13;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
  return (uint16_t)(sign | r);
}

// The reference host conversion: mantissa truncation, exp <= 0 flushed to +-0,
// exp >= 31 to +-inf (include/infvino/Half.hpp:14-24).
static inline uint16_t f2h_trunc(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  const uint32_t mant = x & 0x7fffffu;
  if (exp <= 0) return (uint16_t)sign;
  if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | ((uint32_t)exp << 10) | (mant >> 13));
}

static inline uint16_t hadd(uint16_t a, uint16_t b) { return f2h(h2f(a) + h2f(b)); }

// conv3x3_ov / gemm / gemv epilogue activations (kernels/conv_ov.cl:121-131,
// kernels/gemm.cl:137-153, kernels/conv1x1.cl:52-68).  conv3x3 implements only
// 1 and 3 (others pass through); the 1x1 family implements 1..5.
static inline uint16_t act_gemm(uint16_t v, int act) {
  const float f = h2f(v);
  switch (act) {
    case 1: return f2h(f / (1.0f + std::exp(-f)));
    case 2: return f2h(std::fmax(f, 0.0f));
    case 3: return f2h(f * std::fmin(std::fmax(f + 3.0f, 0.0f), 6.0f) / 6.0f);
    case 4: return f2h(std::fmin(std::fmax(f + 3.0f, 0.0f), 6.0f) / 6.0f);
    case 5: return f2h(1.0f / (1.0f + std::exp(-f)));
    default: return v;
  }
}
static inline uint16_t act_conv3x3(uint16_t v, int act) {
  return (act == 1 || act == 3) ? act_gemm(v, act) : v;
}
// depthwise_f16 `dw_activate` (kernels/conv_general.cl:71-83): HardSwish is
// written f * (clamp / 6) there.
static inline uint16_t act_dw(uint16_t v, int act) {
  const float f = h2f(v);
  switch (act) {
    case 1: return f2h(f / (1.0f + std::exp(-f)));
    case 2: return f2h(std::fmax(f, 0.0f));
    case 3: return f2h(f * (std::fmin(std::fmax(f + 3.0f, 0.0f), 6.0f) / 6.0f));
    case 4: return f2h(std::fmin(std::fmax(f + 3.0f, 0.0f), 6.0f) / 6.0f);
    default: return v;
  }
}
// conv_general (kernels/conv_general.cl:42-46): activation on the f32
// accumulator, codes 1=SiLU 2=HardSwish 3=ReLU 4=HardSigmoid.
static inline float act_general(float a, int act) {
  if (act == 1) return a / (1.0f + std::exp(-a));
  if (act == 2) return a * std::fmin(std::fmax(a + 3.0f, 0.0f), 6.0f) / 6.0f;
  if (act == 3) return std::fmax(a, 0.0f);
  if (act == 4) return std::fmin(std::fmax(a + 3.0f, 0.0f), 6.0f) / 6.0f;
  return a;
}
static inline float binop(float a, float b, int op) {
  if (op == 0) return a + b;
  if (op == 1) return a - b;
  if (op == 2) return a * b;
  return a / b;
}
// ew_unary (kernels/ops.cl:49-62): 0=sigmoid 1=silu 2=relu 3=hswish 4=hsigmoid.
static inline float unop(float v, int op) {
  if (op == 0) return 1.0f / (1.0f + std::exp(-v));
  if (op == 1) return v / (1.0f + std::exp(-v));
  if (op == 2) return std::fmax(v, 0.0f);
  if (op == 3) return v * std::fmin(std::fmax(v + 3.0f, 0.0f), 6.0f) / 6.0f;
  if (op == 4) return std::fmin(std::fmax(v + 3.0f, 0.0f), 6.0f) / 6.0f;
  return v;
}

// ---------------------------------------------------------------- plan model
struct Tensor {
  std::vector<int64_t> dims;
  bool is_init = false;   // initializer: shared across images
  bool is_input = false;
  std::string alias_of;   // reshape/flatten views share storage
  std::vector<uint16_t> data;  // B * numel for activations, numel for inits
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
};

struct Node {
  std::string op;
  std::vector<std::string> ins, outs;
  std::map<std::string, std::string> attr;
  int ai(const char *k, int def) const {
    auto it = attr.find(k);
    return it == attr.end() ? def : std::atoi(it->second.c_str());
  }
};

static std::vector<std::string> split_csv(const std::string &s) {
  std::vector<std::string> out;
  if (s == "-") return out;
  std::stringstream ss(s);
  std::string tok;
  while (std::getline(ss, tok, ',')) out.push_back(tok);
  return out;
}

struct Model {
  std::string plan_dir;
  std::string input;
  std::vector<std::string> outputs;
  std::map<std::string, Tensor> T;
  std::vector<Node> nodes;
  int batch = 0;
  // 0 = fp32 accumulation in natural K order (the build's contract), 1 = fp32 in
  // reversed order (noise-floor probe), 2 = depthwise only: the reference's fp16
  // accumulator (depthwise_f16's mad chain), used to pin against its kernel
  int acc_order = 0;

  Tensor &ref(const std::string &n) {
    auto it = T.find(n);
    if (it == T.end()) throw std::runtime_error("oracle: missing tensor " + n);
    return it->second;
  }
  // storage root (reshape views resolve to their source)
  Tensor &root(const std::string &n) {
    Tensor *t = &ref(n);
    int guard = 0;
    while (!t->alias_of.empty() && guard++ < 1000) t = &ref(t->alias_of);
    return *t;
  }
  // pointer to image b of tensor n (inits: shared)
  uint16_t *ptr(const std::string &n, int b) {
    Tensor &t = ref(n);
    Tensor &r = root(n);
    if (r.is_init) return r.data.data();
    return r.data.data() + (size_t)b * (size_t)t.numel();
  }

  void parse(const std::string &path) {
    std::ifstream f(path);
    if (!f) throw std::runtime_error("oracle: cannot open plan " + path);
    auto slash = path.find_last_of('/');
    plan_dir = slash == std::string::npos ? "." : path.substr(0, slash);
    std::string line;
    while (std::getline(f, line)) {
      if (line.empty() || line[0] == '#') continue;
      std::istringstream ls(line);
      std::string kind;
      ls >> kind;
      if (kind == "input" || kind == "tensor") {
        std::string name;
        ls >> name;
        Tensor t;
        int64_t v;
        while (ls >> v) t.dims.push_back(v);
        t.is_input = kind == "input";
        T[name] = t;
        if (kind == "input" && input.empty()) input = name;
      } else if (kind == "init") {
        std::string name, file;
        ls >> name >> file;
        Tensor t;
        int64_t v;
        while (ls >> v) t.dims.push_back(v);
        t.is_init = true;
        t.data.resize((size_t)t.numel());
        const std::string p = (!file.empty() && file[0] == '/') ? file : plan_dir + "/" + file;
        std::ifstream bf(p, std::ios::binary);
        if (!bf) throw std::runtime_error("oracle: cannot open init " + p);
        bf.read(reinterpret_cast<char *>(t.data.data()), (std::streamsize)(t.data.size() * 2));
        if (!bf) throw std::runtime_error("oracle: short init file " + p);
        T[name] = std::move(t);
      } else if (kind == "node") {
        Node n;
        std::string ins, outs;
        ls >> n.op >> ins >> outs;
        n.ins = split_csv(ins);
        n.outs = split_csv(outs);
        std::string kv;
        while (ls >> kv) {
          auto p = kv.find('=');
          if (p != std::string::npos) n.attr[kv.substr(0, p)] = kv.substr(p + 1);
        }
        nodes.push_back(std::move(n));
      } else if (kind == "output") {
        std::string name;
        ls >> name;
        if (!name.empty()) outputs.push_back(name);
      }
    }
    if (input.empty()) throw std::runtime_error("oracle: plan has no 'input' line");
    if (outputs.empty()) throw std::runtime_error("oracle: plan has no 'output' line");
    for (auto &n : nodes)
      if ((n.op == "reshape" || n.op == "flatten") && !n.ins.empty() && !n.outs.empty())
        ref(n.outs[0]).alias_of = n.ins[0];
  }

  void alloc(int B) {
    batch = B;
    for (auto &kv : T) {
      Tensor &t = kv.second;
      if (t.is_init || !t.alias_of.empty()) continue;
      t.data.assign((size_t)B * (size_t)t.numel(), 0);
    }
  }

  void run(const uint16_t *in, int B);
  void run_node(const Node &n, int b);
};

// ---------------------------------------------------------------- kernels
// The reference's fp16 accumulation step `acc = mad(a, b, acc)` with half
// operands (kernels/gemm.cl:538, kernels/conv_ov.cl:234): the product of two
// halves is exact in f32, the sum is rounded to f32 and then to half.
static inline uint16_t hmad(float a, float b, uint16_t acc) { return f2h(a * b + h2f(acc)); }

static void conv3x3(const uint16_t *x, const uint16_t *w, const uint16_t *bias, const uint16_t *res,
                    uint16_t *y, int Cin, int H, int W, int Cout, int Ho, int Wo, int S, int P, int act,
                    int order) {
  // fp32 accumulation; one output row per (co, oy); order (ci, ky, kx) or
  // reversed.  order 2: the reference conv3x3_ov's fp16 accumulator, one mad
  // per (ci, ky, kx) in that order, taps outside the image contributing
  // mad(w, 0, acc) (kernels/conv_ov.cl:190-239).
#pragma omp parallel for collapse(2) schedule(static)
  for (int co = 0; co < Cout; ++co)
    for (int oy = 0; oy < Ho; ++oy) {
      std::vector<float> acc((size_t)Wo, 0.0f);
      std::vector<uint16_t> hacc((size_t)Wo, 0);
      for (int t = 0; t < Cin * 9; ++t) {
        const int tt = (order == 1) ? (Cin * 9 - 1 - t) : t;
        const int ci = tt / 9, ky = (tt % 9) / 3, kx = tt % 3;
        const int iy = oy * S - P + ky;
        const float wv = h2f(w[((size_t)co * Cin + ci) * 9 + ky * 3 + kx]);
        if (order == 2) {
          for (int ox = 0; ox < Wo; ++ox) {
            const int ix = ox * S - P + kx;
            const bool in = iy >= 0 && iy < H && ix >= 0 && ix < W;
            hacc[ox] = hmad(wv, in ? h2f(x[((size_t)ci * H + iy) * W + ix]) : 0.0f, hacc[ox]);
          }
          continue;
        }
        if (iy < 0 || iy >= H) continue;
        const uint16_t *xr = x + ((size_t)ci * H + iy) * W;
        for (int ox = 0; ox < Wo; ++ox) {
          const int ix = ox * S - P + kx;
          if (ix < 0 || ix >= W) continue;
          acc[ox] += h2f(xr[ix]) * wv;
        }
      }
      const uint16_t b = bias ? bias[co] : 0;
      for (int ox = 0; ox < Wo; ++ox) {
        const size_t o = ((size_t)co * Ho + oy) * Wo + ox;
        uint16_t v = act_conv3x3(hadd(order == 2 ? hacc[ox] : f2h(acc[ox]), b), act);
        if (res) v = hadd(v, res[o]);
        y[o] = v;
      }
    }
}

static void conv1x1(const uint16_t *w, const uint16_t *x, const uint16_t *bias, const uint16_t *res,
                    uint16_t *y, int Cout, int Cin, int64_t N, int act, int order) {
  // order 2 with N > 1: the reference gemm_f16's fp16 accumulator, one mad per
  // input channel in order (kernels/gemm.cl:528-540, 585-602); N == 1 goes to the
  // reference's fp32 GEMV (kernels/conv1x1.cl:172-198), kept in fp32 here.
  const bool half_acc = order == 2 && N > 1;
#pragma omp parallel for schedule(static)
  for (int co = 0; co < Cout; ++co) {
    std::vector<float> acc((size_t)N, 0.0f);
    std::vector<uint16_t> hacc(half_acc ? (size_t)N : 0, 0);
    for (int t = 0; t < Cin; ++t) {
      const int ci = (order == 1) ? (Cin - 1 - t) : t;
      const float wv = h2f(w[(size_t)co * Cin + ci]);
      const uint16_t *xr = x + (size_t)ci * N;
      if (half_acc)
        for (int64_t n = 0; n < N; ++n) hacc[(size_t)n] = hmad(wv, h2f(xr[n]), hacc[(size_t)n]);
      else
        for (int64_t n = 0; n < N; ++n) acc[(size_t)n] += h2f(xr[n]) * wv;
    }
    const uint16_t b = bias ? bias[co] : 0;
    for (int64_t n = 0; n < N; ++n) {
      const size_t o = (size_t)co * N + n;
      uint16_t v = act_gemm(hadd(half_acc ? hacc[(size_t)n] : f2h(acc[(size_t)n]), b), act);
      if (res) v = hadd(v, res[o]);
      y[o] = v;
    }
  }
}

static void depthwise(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y, int C, int H,
                      int W, int Ho, int Wo, int K, int S, int P, int act, int order) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int c = 0; c < C; ++c)
    for (int oy = 0; oy < Ho; ++oy)
      for (int ox = 0; ox < Wo; ++ox) {
        float acc = 0.0f;
        uint16_t hacc = 0;  // order == 2: the reference's fp16 accumulator, mad(x, w, acc) per tap
        for (int t = 0; t < K * K; ++t) {
          const int tt = (order == 1) ? (K * K - 1 - t) : t;
          const int ky = tt / K, kx = tt % K;
          const int iy = oy * S - P + ky, ix = ox * S - P + kx;
          if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
          const float xv = h2f(x[((size_t)c * H + iy) * W + ix]), wv = h2f(w[(size_t)c * K * K + tt]);
          if (order == 2) hacc = f2h(xv * wv + h2f(hacc));
          else acc += xv * wv;
        }
        const uint16_t b = bias ? bias[c] : 0;
        const uint16_t a16 = (order == 2) ? hacc : f2h(acc);
        y[((size_t)c * Ho + oy) * Wo + ox] = act_dw(hadd(a16, b), act);
      }
}

static void conv_general(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y, int Cin,
                         int H, int W, int Cout, int Ho, int Wo, int K, int S, int P, int G, int act) {
  const int cin_g = Cin / G, cout_g = Cout / G;
#pragma omp parallel for collapse(2) schedule(static)
  for (int oc = 0; oc < Cout; ++oc)
    for (int oy = 0; oy < Ho; ++oy)
      for (int ox = 0; ox < Wo; ++ox) {
        const int g = oc / cout_g, ic0 = g * cin_g;
        float acc = bias ? h2f(bias[oc]) : 0.0f;
        for (int ic = 0; ic < cin_g; ++ic)
          for (int ky = 0; ky < K; ++ky) {
            const int iy = oy * S - P + ky;
            if (iy < 0 || iy >= H) continue;
            for (int kx = 0; kx < K; ++kx) {
              const int ix = ox * S - P + kx;
              if (ix < 0 || ix >= W) continue;
              acc += h2f(x[((size_t)(ic0 + ic) * H + iy) * W + ix]) *
                     h2f(w[(((size_t)oc * cin_g + ic) * K + ky) * K + kx]);
            }
          }
        y[((size_t)oc * Ho + oy) * Wo + ox] = f2h(act_general(acc, act));
      }
}

// ---------------------------------------------------------------- dispatch
void Model::run_node(const Node &n, int b) {
  auto in = [&](size_t i) -> uint16_t * {
    if (i >= n.ins.size() || n.ins[i] == "-") return nullptr;
    return ptr(n.ins[i], b);
  };
  auto indims = [&](size_t i) -> const std::vector<int64_t> & { return ref(n.ins[i]).dims; };
  const std::string &op = n.op;
  uint16_t *y = ptr(n.outs[0], b);
  const int64_t nout = ref(n.outs[0]).numel();

  if (op == "reshape" || op == "flatten") return;  // zero-copy view
  if (op == "conv3x3") {  // src/PlanModel.cpp:3688-3700
    const auto &id = indims(0);
    const size_t base = id.size() >= 3 ? id.size() - 3 : 0;
    const int Cin = (int)id[base], H = (int)id[base + 1], W = (int)id[base + 2];
    const auto &od = ref(n.outs[0]).dims;
    const int Cout = (int)od[od.size() >= 3 ? od.size() - 3 : 0];
    conv3x3(in(0), in(1), in(2), in(3), y, Cin, H, W, Cout, n.ai("Hout", 0), n.ai("Wout", 0),
            n.ai("stride", 1), n.ai("pad", 1), n.ai("act", 0), acc_order);
    return;
  }
  if (op == "conv1x1") {  // src/PlanModel.cpp:3394-3413
    const auto &wd = indims(0);
    const int Cout = (int)wd[0], Cin = (int)wd[1];
    const int64_t N = Cin > 0 ? ref(n.ins[1]).numel() / Cin : 0;
    if (n.ins.size() > 4 && n.ins[4] != "-") throw std::runtime_error("oracle: conv1x1 scale input");
    conv1x1(in(0), in(1), in(2), in(3), y, Cout, Cin, N, n.ai("act", 0), acc_order);
    return;
  }
  if (op == "conv_general") {  // src/PlanModel.cpp:3556-3686
    const int K = n.ai("K", 3), S = n.ai("S", 1), P = n.ai("P", 1), G = n.ai("G", 1), act = n.ai("act", 0);
    const auto &id = indims(0);
    const size_t base = id.size() >= 3 ? id.size() - 3 : 0;
    const int Cin = (int)id[base], H = (int)id[base + 1], W = (int)id[base + 2];
    const auto &od = ref(n.outs[0]).dims;
    const int Cout = (int)od[od.size() >= 3 ? od.size() - 3 : 0];
    const int Ho = n.ai("Hout", 0), Wo = n.ai("Wout", 0);
    if (G == Cin && (K == 3 || K == 5) && Cin == Cout)
      depthwise(in(0), in(1), in(2), y, Cin, H, W, Ho, Wo, K, S, P, act, acc_order);
    else
      conv_general(in(0), in(1), in(2), y, Cin, H, W, Cout, Ho, Wo, K, S, P, G, act);
    return;
  }
  if (op == "ew_binary") {  // ops.cl:10-47, 311-373; PlanModel.cpp:2703-2830
    const int opc = n.ai("op", 0);
    const uint16_t *a = in(0), *bb = in(1);
    const bool has_bd = n.attr.count("bdims") && n.ai("b_scalar", 0) != 1;
    if (!has_bd) {
      const int bs = n.ai("b_scalar", 0);
      for (int64_t i = 0; i < nout; ++i)
        y[i] = f2h(binop(h2f(a[i]), h2f(bs ? bb[0] : bb[i]), opc));
      return;
    }
    std::vector<int> v;
    {
      std::stringstream ss(n.attr.at("bdims"));
      std::string tk;
      while (std::getline(ss, tk, ',')) v.push_back(std::atoi(tk.c_str()));
    }
    const int rank = (int)v.size() / 3;
    for (int64_t i = 0; i < nout; ++i) {
      int64_t rem = i, ai = 0, bi = 0;
      for (int r = rank - 1; r >= 0; --r) {
        const int64_t coord = rem % v[r];
        rem /= v[r];
        ai += coord * v[rank + r];
        bi += coord * v[2 * rank + r];
      }
      y[i] = f2h(binop(h2f(a[ai]), h2f(bb[bi]), opc));
    }
    return;
  }
  if (op == "ew_unary") {
    const uint16_t *x = in(0);
    const int opc = n.ai("op", 0);
    for (int64_t i = 0; i < nout; ++i) y[i] = f2h(unop(h2f(x[i]), opc));
    return;
  }
  if (op == "bias_add") {  // ops.cl:268-273
    const uint16_t *x = in(0), *bb = in(1);
    const int HW = n.ai("HW", 1);
    for (int64_t i = 0; i < nout; ++i) y[i] = f2h(h2f(x[i]) + h2f(bb[i / HW]));
    return;
  }
  if (op == "copy_c") {  // ops.cl:65-71
    const uint16_t *x = in(0);
    const int HW = n.ai("HW", 1), c0 = n.ai("c0", 0), cnt = n.ai("cnt", 0), dst = n.ai("dst_off", 0);
    for (int64_t i = 0; i < (int64_t)cnt * HW; ++i) {
      const int64_t c = i / HW, r = i % HW;
      y[dst + i] = x[(c0 + c) * HW + r];
    }
    return;
  }
  if (op == "slice_axis") {  // ops.cl:74-84
    const uint16_t *x = in(0);
    const int outer = n.ai("outer", 1), axdim = n.ai("axdim", 0), inner = n.ai("inner", 1),
              start = n.ai("start", 0), len = n.ai("len", 0);
    const int64_t total = (int64_t)outer * len * inner;
    for (int64_t i = 0; i < total; ++i) {
      const int64_t o = i / ((int64_t)len * inner), rem = i % ((int64_t)len * inner);
      y[i] = x[(o * axdim + start) * inner + rem];
    }
    return;
  }
  if (op == "concat4") {  // ops.cl:93-118
    const int c[4] = {n.ai("ca", 0), n.ai("cb", 0), n.ai("cc", 0), n.ai("cd", 0)};
    const int outer = n.ai("outer", 1), inner = n.ai("inner", 1);
    const int sum = c[0] + c[1] + c[2] + c[3];
    const uint16_t *src[4] = {c[0] ? in(0) : nullptr, c[1] ? in(1) : nullptr, c[2] ? in(2) : nullptr,
                              c[3] ? in(3) : nullptr};
    for (int o = 0; o < outer; ++o) {
      int ax0 = 0;
      for (int s = 0; s < 4; ++s) {
        for (int ax = 0; ax < c[s]; ++ax)
          std::memcpy(y + ((size_t)o * sum + ax0 + ax) * inner, src[s] + ((size_t)o * c[s] + ax) * inner,
                      (size_t)inner * 2);
        ax0 += c[s];
      }
    }
    return;
  }
  if (op == "maxpool") {  // ops.cl:148-165
    const uint16_t *x = in(0);
    const int C = n.ai("C", 0), H = n.ai("H", 0), W = n.ai("W", 0), Ho = n.ai("Hout", 0), Wo = n.ai("Wout", 0),
              K = n.ai("K", 5), S = n.ai("S", 1), P = n.ai("P", 2);
    for (int c = 0; c < C; ++c)
      for (int oh = 0; oh < Ho; ++oh)
        for (int ow = 0; ow < Wo; ++ow) {
          float m = -3.4e38f;
          for (int kh = 0; kh < K; ++kh)
            for (int kw = 0; kw < K; ++kw) {
              const int yy = oh * S - P + kh, xx = ow * S - P + kw;
              if (yy >= 0 && yy < H && xx >= 0 && xx < W) m = std::fmax(m, h2f(x[((size_t)c * H + yy) * W + xx]));
            }
          y[((size_t)c * Ho + oh) * Wo + ow] = f2h(m);
        }
    return;
  }
  if (op == "resize_nn") {  // ops.cl:168-178
    const uint16_t *x = in(0);
    const int C = n.ai("C", 0), H = n.ai("H", 0), W = n.ai("W", 0), S = n.ai("S", 2);
    const int Ho = H * S, Wo = W * S;
    for (int c = 0; c < C; ++c)
      for (int oh = 0; oh < Ho; ++oh)
        for (int ow = 0; ow < Wo; ++ow)
          y[((size_t)c * Ho + oh) * Wo + ow] = x[((size_t)c * H + oh / S) * W + ow / S];
    return;
  }
  if (op == "softmax_axis") {  // ops.cl:181-196 (serial default)
    const uint16_t *x = in(0);
    const int outer = n.ai("outer", 1), axdim = n.ai("axdim", 0), inner = n.ai("inner", 1);
    for (int o = 0; o < outer; ++o)
      for (int r = 0; r < inner; ++r) {
        float m = -3.4e38f;
        for (int a = 0; a < axdim; ++a) m = std::fmax(m, h2f(x[((size_t)o * axdim + a) * inner + r]));
        float s = 0.0f;
        for (int a = 0; a < axdim; ++a) s += std::exp(h2f(x[((size_t)o * axdim + a) * inner + r]) - m);
        for (int a = 0; a < axdim; ++a) {
          const size_t idx = ((size_t)o * axdim + a) * inner + r;
          y[idx] = f2h(std::exp(h2f(x[idx]) - m) / s);
        }
      }
    return;
  }
  if (op == "permute_0213") {  // ops.cl:199-221
    const uint16_t *x = in(0);
    const int D1 = n.ai("D1", 1), D2 = n.ai("D2", 1), I = n.ai("I", 1), mode = n.ai("mode", 0);
    const int64_t total = (int64_t)D1 * D2 * I;
    for (int64_t i = 0; i < total; ++i) {
      const int64_t d1 = i / ((int64_t)D2 * I), rem = i % ((int64_t)D2 * I);
      const int64_t d2 = rem / I, r = rem % I;
      if (mode == 0) y[(d2 * D1 + d1) * I + r] = x[i];
      else y[(d1 * I + r) * D2 + d2] = x[i];
    }
    return;
  }
  if (op == "gap") {  // ops.cl:245-265 (gap_r, GAP_WGS = 128 lane-strided sums + tree)
    const uint16_t *x = in(0);
    const int C = n.ai("C", 0), HW = n.ai("HW", 1);
    for (int c = 0; c < C; ++c) {
      float s[128];
      for (int l = 0; l < 128; ++l) {
        float acc = 0.0f;
        for (int i = l; i < HW; i += 128) acc += h2f(x[(size_t)c * HW + i]);
        s[l] = acc;
      }
      for (int off = 64; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l) s[l] += s[l + off];
      y[c] = f2h(s[0] / (float)HW);
    }
    return;
  }
  if (op == "bmm") {  // ops.cl:276-292
    const auto &ad = indims(0), &bd = indims(1);
    const int B0 = (int)ad[0], B1 = (int)ad[1], M = (int)ad[2], K = (int)ad[3], N = (int)bd[3];
    const uint16_t *A = in(0), *Bm = in(1);
    for (int bb = 0; bb < B0 * B1; ++bb)
      for (int m = 0; m < M; ++m)
        for (int nn = 0; nn < N; ++nn) {
          float acc = 0.0f;
          for (int k = 0; k < K; ++k)
            acc += h2f(A[((size_t)bb * M + m) * K + k]) * h2f(Bm[((size_t)bb * K + k) * N + nn]);
          y[((size_t)bb * M + m) * N + nn] = f2h(acc);
        }
    return;
  }
  throw std::runtime_error("oracle: unknown op: " + op);
}

void Model::run(const uint16_t *in, int B) {
  if (B != batch) alloc(B);
  Tensor &ti = ref(input);
  std::memcpy(ti.data.data(), in, (size_t)B * (size_t)ti.numel() * 2);
  for (const auto &n : nodes)
    for (int b = 0; b < B; ++b) run_node(n, b);
}

}  // namespace ivref

// ---------------------------------------------------------------- C ABI
namespace {
thread_local std::string g_err;
}

extern "C" {

const char *ivref_last_error(void) { return g_err.c_str(); }

int ivref_create(const char *plan_path, void **out) {
  try {
    auto m = std::make_unique<ivref::Model>();
    m->parse(plan_path);
    *out = m.release();
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

void ivref_destroy(void *h) { delete static_cast<ivref::Model *>(h); }

int ivref_set_acc_order(void *h, int order) {
  static_cast<ivref::Model *>(h)->acc_order = order;
  return 0;
}

int ivref_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

int64_t ivref_input_numel(void *h) {
  auto *m = static_cast<ivref::Model *>(h);
  return m->ref(m->input).numel();
}

int ivref_output_count(void *h) { return (int)static_cast<ivref::Model *>(h)->outputs.size(); }

const char *ivref_output_name(void *h, int i) { return static_cast<ivref::Model *>(h)->outputs.at((size_t)i).c_str(); }

// per-image element count of a tensor; -1 if unknown
int64_t ivref_tensor_numel(void *h, const char *name) {
  auto *m = static_cast<ivref::Model *>(h);
  auto it = m->T.find(name);
  return it == m->T.end() ? -1 : it->second.numel();
}

int ivref_tensor_dims(void *h, const char *name, int64_t *dims, int max_rank) {
  auto *m = static_cast<ivref::Model *>(h);
  auto it = m->T.find(name);
  if (it == m->T.end()) return -1;
  const auto &d = it->second.dims;
  for (int i = 0; i < (int)d.size() && i < max_rank; ++i) dims[i] = d[(size_t)i];
  return (int)d.size();
}

int ivref_run(void *h, const uint16_t *input_f16, int batch) {
  try {
    static_cast<ivref::Model *>(h)->run(input_f16, batch);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// copies batch * numel fp16 values of a tensor (activations) or numel (inits)
int ivref_read_tensor(void *h, const char *name, uint16_t *dst) {
  auto *m = static_cast<ivref::Model *>(h);
  try {
    ivref::Tensor &t = m->ref(name);
    ivref::Tensor &r = m->root(name);
    const size_t n = (size_t)t.numel() * (r.is_init ? 1 : (size_t)m->batch);
    if (r.data.size() < n) throw std::runtime_error("oracle: tensor not computed: " + std::string(name));
    std::memcpy(dst, r.data.data(), n * 2);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// The reference's final ordering of the kept detections (src/Decoders.cpp:58-62):
// std::sort by descending score, an unstable sort, applied to the NMS keep list
// in its order.  Equal scores come out in the order std::sort (libstdc++'s
// introsort here) leaves them, which depends only on the sequence of
// comparisons, so sorting (score, position) pairs with a score-only comparator
// gives the permutation the reference applies to its Detection objects.
// perm[k] = position (in the input sequence) of the k-th detection afterwards.
void ivref_std_sort_desc(const float *scores, int n, int *perm) {
  std::vector<std::pair<float, int>> v((size_t)n);
  for (int i = 0; i < n; ++i) v[(size_t)i] = {scores[i], i};
  std::sort(v.begin(), v.end(),
            [](const std::pair<float, int> &a, const std::pair<float, int> &b) { return a.first > b.first; });
  for (int i = 0; i < n; ++i) perm[i] = v[(size_t)i].second;
}

void ivref_f32_to_f16_trunc(const float *in, uint16_t *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = ivref::f2h_trunc(in[i]);
}
void ivref_f32_to_f16_rne(const float *in, uint16_t *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = ivref::f2h(in[i]);
}
void ivref_f16_to_f32(const uint16_t *in, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = ivref::h2f(in[i]);
}

}  // extern "C"
