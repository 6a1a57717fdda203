#include "tail_jit.h"

#include <cuda.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <cstdint>
#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <sstream>
#include <vector>

namespace ivb {

namespace {

// ---------------------------------------------------------------- NVRTC (dlopen'd)
struct Nvrtc {
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
  std::string err;
};

const Nvrtc &nvrtc() {
  static Nvrtc n;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = nullptr;
    for (const char *name : {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"}) {
      h = dlopen(name, RTLD_NOW | RTLD_LOCAL);
      if (h) break;
    }
    if (!h) {
      n.err = "libnvrtc not found";
      return;
    }
    n.create = reinterpret_cast<decltype(n.create)>(dlsym(h, "nvrtcCreateProgram"));
    n.compile = reinterpret_cast<decltype(n.compile)>(dlsym(h, "nvrtcCompileProgram"));
    n.log_size = reinterpret_cast<decltype(n.log_size)>(dlsym(h, "nvrtcGetProgramLogSize"));
    n.log = reinterpret_cast<decltype(n.log)>(dlsym(h, "nvrtcGetProgramLog"));
    n.cubin_size = reinterpret_cast<decltype(n.cubin_size)>(dlsym(h, "nvrtcGetCUBINSize"));
    n.cubin = reinterpret_cast<decltype(n.cubin)>(dlsym(h, "nvrtcGetCUBIN"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "nvrtcDestroyProgram"));
    if (!n.create || !n.compile || !n.log_size || !n.log || !n.cubin_size || !n.cubin || !n.destroy)
      n.err = "libnvrtc lacks an entry point";
  });
  return n;
}

// Compiles `src` for sm_100a; the cubin on success, else empty with *log set.
// Cubins are kept per source text for the life of the process (every engine
// of one model generates the same source).
std::vector<char> compile_cubin_uncached(const std::string &src, std::string *log);
std::vector<char> compile_cubin(const std::string &src, std::string *log) {
  static std::mutex mu;
  static std::map<std::string, std::vector<char>> cache;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(src);
    if (it != cache.end()) return it->second;
  }
  std::vector<char> c = compile_cubin_uncached(src, log);
  if (!c.empty()) {
    std::lock_guard<std::mutex> g(mu);
    cache.emplace(src, c);
  }
  return c;
}
std::vector<char> compile_cubin_uncached(const std::string &src, std::string *log) {
  const Nvrtc &n = nvrtc();
  if (!n.err.empty()) {
    *log = n.err;
    return {};
  }
  nvrtcProgram prog = nullptr;
  if (n.create(&prog, src.c_str(), "ivb_tail.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) {
    *log = "nvrtcCreateProgram failed";
    return {};
  }
  const char *opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-fmad=true"};
  const nvrtcResult rc = n.compile(prog, 3, opts);
  std::vector<char> out;
  if (rc != NVRTC_SUCCESS) {
    size_t ls = 0;
    n.log_size(prog, &ls);
    std::string l(ls, '\0');
    if (ls) n.log(prog, &l[0]);
    *log = "nvrtc: " + l;
  } else {
    size_t cs = 0;
    n.cubin_size(prog, &cs);
    out.resize(cs);
    if (cs) n.cubin(prog, out.data());
  }
  n.destroy(&prog);
  return out;
}

// ---------------------------------------------------------------- driver entry points
struct Driver {
  CUresult (*load)(CUmodule *, const void *) = nullptr;
  CUresult (*get_fn)(CUfunction *, CUmodule, const char *) = nullptr;
  CUresult (*unload)(CUmodule) = nullptr;
  CUresult (*launch)(const CUlaunchConfig *, CUfunction, void **, void **) = nullptr;
  std::string err;
};

const Driver &driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char *name) -> void * {
      void *p = nullptr;
      cudaDriverEntryPointQueryResult q{};
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess)
        return nullptr;
      return p;
    };
    d.load = reinterpret_cast<decltype(d.load)>(get("cuModuleLoadData"));
    d.get_fn = reinterpret_cast<decltype(d.get_fn)>(get("cuModuleGetFunction"));
    d.unload = reinterpret_cast<decltype(d.unload)>(get("cuModuleUnload"));
    d.launch = reinterpret_cast<decltype(d.launch)>(get("cuLaunchKernelEx"));
    if (!d.load || !d.get_fn || !d.unload || !d.launch) d.err = "driver module entry points unavailable";
  });
  return d;
}

// ---------------------------------------------------------------- code generation
std::string flit(float f) {  // exact float literal
  uint32_t u;
  std::memcpy(&u, &f, 4);
  std::ostringstream os;
  os << "__int_as_float(0x" << std::hex << u << std::dec << ")";
  return os.str();
}

// fp16 <-> f32 by cvt, so the generated source needs no header
const char *kPreamble = R"(
typedef unsigned short h16;
__device__ __forceinline__ float h2f(h16 h) { float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
__device__ __forceinline__ h16 f2h(float f) { h16 h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f)); return h; }
__device__ __forceinline__ float rh(float f) { return h2f(f2h(f)); }
// a / b with rb = RN(1 / b) (__frcp_rn) shared by several quotients: Markstein's
// method (P. Markstein, IBM J. Res. Dev. 34(1), 1990): q = RN(a rb), the exact
// residual r = a - b q by one FMA, then RN(q + r rb) is the correctly rounded
// a / b while q and r stay in the normal range.  Used where a in [0, 1] and
// b in [1, 16] (the DFL softmax): a quotient below the normal range rounds to
// fp16 zero either way.
__device__ __forceinline__ float div_rcp(float a, float b, float rb) {
  const float q = a * rb;
  return fmaf(fmaf(-q, b, a), rb, q);
}
struct TailArgs { const h16 *leaf[8]; h16 *out; int batch; int blk0[33]; };
)";

std::string unop_expr(int op, const std::string &v) {
  switch (op) {
    case 0: return "__frcp_rn(1.0f + expf(-" + v + "))";  // 1 / x correctly rounded, as the division
    case 1: return v + " / (1.0f + expf(-" + v + "))";
    case 2: return "fmaxf(" + v + ", 0.0f)";
    case 3: return v + " * fminf(fmaxf(" + v + " + 3.0f, 0.0f), 6.0f) / 6.0f";
    case 4: return "fminf(fmaxf(" + v + " + 3.0f, 0.0f), 6.0f) / 6.0f";
    default: return v;
  }
}

// act_f32(f, act, kActGemm)
std::string gemm_act_expr(int act, const std::string &f) {
  switch (act) {
    case 1: return f + " / (1.0f + expf(-" + f + "))";
    case 2: return "fmaxf(" + f + ", 0.0f)";
    case 3: return f + " * fminf(fmaxf(" + f + " + 3.0f, 0.0f), 6.0f) / 6.0f";
    case 4: return "fminf(fmaxf(" + f + " + 3.0f, 0.0f), 6.0f) / 6.0f";
    case 5: return "__frcp_rn(1.0f + expf(-" + f + "))";
    default: return f;
  }
}

}  // namespace

std::vector<TailJitGroup> tail_jit_groups(const TailProgram &P, const TailJitLayout &L) {
  // chains with a DFL op run alone at one anchor per thread (softmax over 16
  // bins per side: most of the tail's arithmetic); the light chains are packed
  // into a few groups (longest first onto the least loaded) at L.V anchors
  std::vector<TailJitGroup> groups;
  std::vector<std::pair<int, int>> light;  // (ops, chain)
  for (int c = 0; c < P.n_comp; ++c) {
    bool dfl = false;
    for (int k = P.comp_begin[c]; k < P.comp_begin[c + 1]; ++k) dfl = dfl || P.ops[k].code == kTailDfl;
    if (dfl) {
      TailJitGroup g;
      g.V = 1;
      g.chains.push_back(c);
      groups.push_back(g);
    } else {
      light.push_back({P.comp_begin[c + 1] - P.comp_begin[c], c});
    }
  }
  const int nl = std::min<int>((int)light.size(), kTailJitLightGroups);
  if (nl > 0) {
    std::sort(light.begin(), light.end(), [](const std::pair<int, int> &x, const std::pair<int, int> &y) {
      return x.first != y.first ? x.first > y.first : x.second < y.second;
    });
    std::vector<TailJitGroup> lg((size_t)nl);
    std::vector<int> load((size_t)nl, 0);
    for (const auto &ch : light) {
      const size_t g = (size_t)(std::min_element(load.begin(), load.end()) - load.begin());
      lg[g].chains.push_back(ch.second);
      load[g] += ch.first;
    }
    for (auto &g : lg) {
      g.V = L.V;
      std::sort(g.chains.begin(), g.chains.end());  // program order inside a group
      groups.push_back(g);
    }
  }
  return groups;
}

std::string tail_jit_source(const TailProgram &P, const TailJitLayout &L) {
  const std::vector<TailJitGroup> groups = tail_jit_groups(P, L);
  std::ostringstream os;
  os << kPreamble;
  os << "extern \"C\" __global__ void __launch_bounds__(128) ivb_tail(const TailArgs a) {\n"
     << "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
     << "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n"
     << "  int g = 0;\n"
     << "  while (g + 1 < " << groups.size() << " && (int)blockIdx.x >= a.blk0[g + 1]) ++g;\n"
     << "  const long long i = (long long)((int)blockIdx.x - a.blk0[g]) * 128 + threadIdx.x;\n"
     << "  switch (g) {\n";
  for (size_t gi = 0; gi < groups.size(); ++gi) {
    const int V = groups[gi].V;
    const long long AV = L.A / V;
    os << "  case " << gi << ": {\n"
       << "  if (i >= (long long)a.batch * " << AV << "LL) return;\n"
       << "  const long long img = i / " << AV << "LL, an0 = (i - img * " << AV << "LL) * " << V << ";\n";
    auto row_ptr = [&](int li, long long row) {
      std::ostringstream p;
      p << "(a.leaf[" << li << "] + img * " << L.leaf_img[li] << "LL + " << row * L.leaf_row[li] << "LL + an0)";
      return p.str();
    };
    // V halves of a row into floats d[0..V)
    auto load = [&](const std::string &dst, const std::string &ptr) {
      if (V == 4)
        os << "  { const uint2 u = *reinterpret_cast<const uint2 *>(" << ptr << "); " << dst << "[0] = h2f(u.x & 0xffff); "
           << dst << "[1] = h2f(u.x >> 16); " << dst << "[2] = h2f(u.y & 0xffff); " << dst << "[3] = h2f(u.y >> 16); }\n";
      else if (V == 2)
        os << "  { const unsigned u = *reinterpret_cast<const unsigned *>(" << ptr << "); " << dst
           << "[0] = h2f(u & 0xffff); " << dst << "[1] = h2f(u >> 16); }\n";
      else
        os << "  " << dst << "[0] = h2f(*(" << ptr << "));\n";
    };
    std::map<std::pair<int, int>, std::string> leaf_var;
    auto elem = [](const std::string &v) { return v[0] == '#' ? v.substr(1) : v + "[j]"; };
    for (int c : groups[gi].chains) {
      std::vector<std::string> slot_var(kTailMaxSlots + 1);  // slots are per chain
      auto operand = [&](const TailOperand &o) -> std::string {  // a V-array, or an immediate
        if (o.kind == kTailImm) {
          float f;
          std::memcpy(&f, &o.idx, 4);
          return "#" + flit(f);
        }
        if (o.kind == kTailSlot) return slot_var[(size_t)o.idx];
        const auto key = std::make_pair(o.idx, o.row);
        auto it = leaf_var.find(key);
        if (it != leaf_var.end()) return it->second;
        const std::string name = "l" + std::to_string(o.idx) + "_" + std::to_string(o.row);
        os << "  float " << name << "[" << V << "];\n";
        load(name, row_ptr(o.idx, o.row));
        leaf_var[key] = name;
        return name;
      };
      for (int k = P.comp_begin[c]; k < P.comp_begin[c + 1]; ++k) {
        const TailOp &op = P.ops[k];
        const std::string r = "v" + std::to_string(k);
        os << "  float " << r << "[" << V << "];\n";
        if (op.code == kTailDfl) {
          // softmax over the 16 bins of rows a.row .. a.row+15, then the 1x1
          // projection and the gemm-family epilogue (tail_vm_k's DFL arithmetic)
          const TailDfl &D = P.dfl[op.arg];
          os << "  {\n    float e[16][" << V << "];\n";
          for (int q = 0; q < 16; ++q) load("e[" + std::to_string(q) + "]", row_ptr(op.a.idx, (long long)op.a.row + q));
          os << "#pragma unroll\n    for (int j = 0; j < " << V << "; ++j) {\n"
             << "      float m = -3.4e38f;\n"
             << "#pragma unroll\n      for (int q = 0; q < 16; ++q) m = fmaxf(m, e[q][j]);\n"
             << "      float s = 0.0f;\n"
             << "#pragma unroll\n      for (int q = 0; q < 16; ++q) { e[q][j] = expf(e[q][j] - m); s += e[q][j]; }\n"
             << "      const float rs = __frcp_rn(s);  // e / s below: e in [0, 1], s in [1, 16]\n"
             << "      float acc = 0.0f;\n";
          for (int q = 0; q < 16; ++q)
            os << "      acc = fmaf(rh(div_rcp(e[" << q << "][j], s, rs)), " << flit(D.w[q]) << ", acc);\n";
          os << "      const float v = rh(acc) + " << flit(D.bias) << ";\n"
             << "      const float f = rh(v);\n"
             << "      " << r << "[j] = rh(" << gemm_act_expr(D.act, "f") << ");\n"
             << "    }\n  }\n";
        } else {
          const std::string a = operand(op.a);
          std::string expr;
          if (op.code == kTailBin) {
            const std::string b = operand(op.b);
            static const char *sym[] = {" + ", " - ", " * ", " / "};
            expr = "rh(" + elem(a) + sym[op.arg >= 0 && op.arg <= 3 ? op.arg : 3] + elem(b) + ")";
          } else if (op.code == kTailUn) {
            expr = "rh(" + unop_expr(op.arg, elem(a)) + ")";
          } else {
            expr = elem(a);
          }
          os << "#pragma unroll\n  for (int j = 0; j < " << V << "; ++j) " << r << "[j] = " << expr << ";\n";
        }
        if (op.dst >= 0) slot_var[(size_t)op.dst] = r;
        if (op.store_row >= 0) {
          std::ostringstream p;
          p << "(a.out + img * " << L.out_img << "LL + " << (long long)op.store_row * L.A << "LL + an0)";
          if (V == 4)
            os << "  *reinterpret_cast<uint2 *>" << p.str() << " = make_uint2((unsigned)f2h(" << r
               << "[0]) | ((unsigned)f2h(" << r << "[1]) << 16), (unsigned)f2h(" << r << "[2]) | ((unsigned)f2h(" << r
               << "[3]) << 16));\n";
          else if (V == 2)
            os << "  *reinterpret_cast<unsigned *>" << p.str() << " = (unsigned)f2h(" << r << "[0]) | ((unsigned)f2h("
               << r << "[1]) << 16);\n";
          else
            os << "  *" << p.str() << " = f2h(" << r << "[0]);\n";
        }
      }
    }
    os << "  } break;\n";
  }
  os << "  }\n}\n";
  return os.str();
}

TailJit::~TailJit() {
  if (module_ && driver().unload) driver().unload(static_cast<CUmodule>(module_));
}

bool TailJit::build(const TailProgram &prog, const TailJitLayout &lay, bool load, std::string *err) {
  if (tail_jit_groups(prog, lay).size() > (size_t)kTailJitMaxGroups) {
    *err = "too many chain groups";
    return false;
  }
  std::string log;
  const std::vector<char> cubin = compile_cubin(tail_jit_source(prog, lay), &log);
  if (cubin.empty()) {
    *err = log.empty() ? "empty cubin" : log;
    return false;
  }
  if (!load) return true;
  const Driver &d = driver();
  if (!d.err.empty()) {
    *err = d.err;
    return false;
  }
  CUmodule mod = nullptr;
  CUfunction fn = nullptr;
  CUresult r = d.load(&mod, cubin.data());
  if (r == CUDA_SUCCESS) r = d.get_fn(&fn, mod, "ivb_tail");
  if (r != CUDA_SUCCESS) {
    if (mod) d.unload(mod);
    *err = "loading the tail cubin failed with code " + std::to_string((int)r);
    return false;
  }
  module_ = mod;
  fn_ = fn;
  lay_ = lay;
  n_leaves_ = prog.n_leaves;
  group_v_.clear();
  for (const TailJitGroup &g : tail_jit_groups(prog, lay)) group_v_.push_back(g.V);
  return true;
}

cudaError_t TailJit::launch(const TailProgram &prog, int batch, bool pdl, cudaStream_t st) const {
  if (!fn_) return cudaErrorInvalidResourceHandle;
  struct Args {
    const __half *leaf[8];
    __half *out;
    int batch;
    int blk0[kTailJitMaxGroups + 1];
  } args{};
  for (int i = 0; i < n_leaves_ && i < 8; ++i) args.leaf[i] = prog.leaves[i].ptr;
  args.out = prog.out;
  args.batch = batch;
  long long blocks = 0;
  for (size_t g = 0; g < group_v_.size(); ++g) {
    args.blk0[g] = (int)blocks;
    blocks += ((long long)batch * (lay_.A / group_v_[g]) + 127) / 128;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  }
  for (size_t g = group_v_.size(); g <= (size_t)kTailJitMaxGroups; ++g) args.blk0[g] = (int)blocks;
  if (blocks < 1) return cudaErrorInvalidValue;
  CUlaunchAttribute attr{};
  attr.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr.value.programmaticStreamSerializationAllowed = 1;
  CUlaunchConfig cfg{};
  cfg.gridDimX = (unsigned)blocks;
  cfg.gridDimY = cfg.gridDimZ = 1;
  cfg.blockDimX = 128;
  cfg.blockDimY = cfg.blockDimZ = 1;
  cfg.sharedMemBytes = 0;
  cfg.hStream = reinterpret_cast<CUstream>(st);
  cfg.attrs = pdl ? &attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  void *params[] = {&args};
  const CUresult r = driver().launch(&cfg, static_cast<CUfunction>(fn_), params, nullptr);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorLaunchFailure;
}

}  // namespace ivb
