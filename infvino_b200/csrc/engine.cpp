// CudaPlanModel engine implementation.
//
// Correspondence with the reference executor (src/PlanModel.cpp):
//   parse ............................ Plan (plan.cpp), same grammar and errors
//   fuseConcatConv1x1 / fuseResidualAdd  Plan::fuse_* (numerically transparent)
//   allocateActivations + ActPool ..... Engine::allocate (liveness intervals over
//                                       node indices, views share their root's
//                                       interval, largest-first gap placement in
//                                       ONE device arena, self-check for overlap)
//   planBlockedLayout / LayoutSolver .. Engine::plan_layouts (NHWC vs planar)
//   run() dispatch + capture/replay ... Engine::lower + CUDA graph per batch size
#include "engine.h"
#include "host_cast.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <functional>
#include <cstring>
#include <numeric>
#include <set>
#include <sstream>
#include <stdexcept>

#include "kernels/common.cuh"
#include "kernels/conv_tc.cuh"
#include "tail_jit.h"
#include "tma.h"

namespace ivb {

namespace {

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

std::vector<int64_t> parse_ints(const std::string &s) {
  std::vector<int64_t> v;
  std::stringstream ss(s);
  std::string tok;
  while (std::getline(ss, tok, ',')) v.push_back(std::atoll(tok.c_str()));
  return v;
}

uint16_t f32_to_f16_rne_host(float f) {  // host packing of padded weights only (exact values)
  const __half h = __float2half_rn(f);
  uint16_t u;
  std::memcpy(&u, &h, 2);
  return u;
}

float f16_to_f32_host(uint16_t u) {  // exact widening of an init value (host)
  __half_raw r;
  r.x = u;
  return __half2float(__half(r));
}

}  // namespace

// ============================================================================ setup
Engine::Engine(const std::string &plan_path, int device, int max_batch, unsigned flags)
    : device_(device), max_batch_(max_batch), flags_(flags), dry_((flags & kFlagDryRun) != 0) {
  if (max_batch < 1) throw std::runtime_error("CudaPlanModel: max_batch must be >= 1");
  plan_ = std::make_unique<Plan>(plan_path);
  if (!dry_) {
    check(cudaSetDevice(device_), "cudaSetDevice");
    cudaDeviceProp prop{};
    check(cudaGetDeviceProperties(&prop, device_), "cudaGetDeviceProperties");
    if (prop.major != 10)
      throw std::runtime_error("CudaPlanModel: device " + std::to_string(device_) + " (" + prop.name +
                               ") is not an sm_100 GPU");
    num_sms_ = prop.multiProcessorCount;
    check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    own_stream_ = true;
  }
  plan_layouts();
  build_tensors();
  if (!(flags_ & kFlagNoFusion)) plan_tails();
  lifetimes();
  alloc_aux();
  upload_weights();
  lower();
  plan_streams();
  allocate();
}

Engine::~Engine() {
  if (dry_) return;
  cudaSetDevice(device_);
  for (auto &kv : graphs_) cudaGraphExecDestroy(kv.second);
  if (stream_) cudaStreamSynchronize(stream_);
  for (void *p : dev_allocs_) cudaFree(p);
  if (arena_) cudaFree(arena_);
  if (status_) cudaFree(status_);
  if (in_f32_) cudaFree(in_f32_);
  if (out_f32_) cudaFree(out_f32_);
  if (in_f16_host_) cudaFreeHost(in_f16_host_);
  if (out_host_) cudaFreeHost(out_host_);
  if (lbt_.xtab) cudaFree(lbt_.xtab);
  if (lbt_.ytab) cudaFree(lbt_.ytab);
  if (frames_dev_) cudaFree(frames_dev_);
  if (nms_boxes_) cudaFree(nms_boxes_);
  if (nms_counts_) cudaFree(nms_counts_);
  if (nms_dets_) cudaFree(nms_dets_);
  if (nms_lbox_) cudaFree(nms_lbox_);
  if (nms_host_) cudaFreeHost(nms_host_);
  if (nms_kept_) cudaFree(nms_kept_);
  if (nms_pairs_) cudaFree(nms_pairs_);
  if (nms_chosen_) cudaFree(nms_chosen_);
  if (nms_pairs_host_) cudaFreeHost(nms_pairs_host_);
  for (cudaEvent_t e : chunk_events_) cudaEventDestroy(e);
  if (copy_in_) cudaStreamDestroy(copy_in_);
  if (copy_out_) cudaStreamDestroy(copy_out_);
  if (scratch_) cudaFree(scratch_);
  for (cudaEvent_t e : step_events_)
    if (e) cudaEventDestroy(e);
  if (fork_event_) cudaEventDestroy(fork_event_);
  for (int t = 1; t < kMaxStreams; ++t) {
    if (join_events_[t]) cudaEventDestroy(join_events_[t]);
    if (side_[t]) cudaStreamDestroy(side_[t]);
  }
  if (own_stream_ && stream_) cudaStreamDestroy(stream_);
}

void Engine::check(cudaError_t e, const char *what) const {
  if (e != cudaSuccess) throw std::runtime_error(std::string("CudaPlanModel: ") + what + ": " + cudaGetErrorString(e));
}

int Engine::tid(const std::string &name) const {
  auto it = tid_.find(name);
  if (it == tid_.end()) throw std::runtime_error("PlanModel: missing tensor: " + name);
  return it->second;
}

const std::vector<int64_t> &Engine::input_dims() const { return plan_->ref(plan_->input()).dims; }
int64_t Engine::input_numel() const { return plan_->ref(plan_->input()).numel(); }
const std::vector<int64_t> &Engine::output_dims(int i) const { return plan_->ref(output_name(i)).dims; }
int64_t Engine::output_numel(int i) const { return plan_->ref(output_name(i)).numel(); }
int64_t Engine::tensor_numel(const std::string &name) const {
  return plan_->has(name) ? plan_->ref(name).numel() : 0;
}

// ============================================================================ layouts
namespace {

bool is_act4(const PlanTensor &t) { return !t.is_init && t.dims.size() == 4 && t.dims[0] == 1; }

// ew_binary broadcast of a [1,C,1,1] operand over a [1,C,H,W] output (SE scale).
bool per_channel_bcast(const Plan &p, const PlanNode &n, int *scale_slot) {
  if (n.ins.size() < 2) return false;
  const PlanTensor &o = p.ref(n.outs[0]);
  if (o.dims.size() != 4) return false;
  for (int k = 0; k < 2; ++k) {
    const PlanTensor &s = p.ref(n.ins[(size_t)k]);
    const PlanTensor &v = p.ref(n.ins[(size_t)(1 - k)]);
    if (v.dims != o.dims) continue;
    std::vector<int64_t> al(4, 1);
    for (size_t i = 0; i < s.dims.size() && i < 4; ++i) al[4 - s.dims.size() + i] = s.dims[i];
    if (s.dims.size() <= 4 && al[0] == 1 && al[1] == o.dims[1] && al[2] == 1 && al[3] == 1) {
      if (scale_slot) *scale_slot = k;
      return true;
    }
  }
  return false;
}

bool elementwise_same(const PlanNode &n) { return !n.has("bdims") || n.ai("b_scalar", 0) == 1; }

}  // namespace

void Engine::plan_layouts() {
  Plan &p = *plan_;
  const auto &nodes = p.nodes();
  // consumers per tensor
  std::map<std::string, std::vector<std::pair<int, int>>> cons;
  std::map<std::string, int> prod;
  for (size_t i = 0; i < nodes.size(); ++i) {
    for (size_t s = 0; s < nodes[i].ins.size(); ++s)
      if (nodes[i].ins[s] != "-") cons[nodes[i].ins[s]].push_back({(int)i, (int)s});
    for (const auto &o : nodes[i].outs) prod[o] = (int)i;
  }
  auto consumer_ok = [&](const PlanNode &n, int slot) -> bool {
    const std::string &op = n.op;
    if (op == "conv3x3") return slot == 0 || slot == 3;
    if (op == "conv1x1") return slot == 1 || slot == 3;
    if (op == "conv_general") return slot == 0;
    if (op == "maxpool" || op == "resize_nn" || op == "gap" || op == "ew_unary" || op == "copy_c") return slot == 0;
    if (op == "concat4") return n.ai("outer", 1) == 1 && p.ref(n.outs[0]).dims.size() == 4;
    if (op == "ew_binary") return elementwise_same(n) || per_channel_bcast(p, n, nullptr);
    return false;
  };
  auto producer_ok = [&](const PlanNode &n) -> bool {
    const std::string &op = n.op;
    if (op == "conv3x3" || op == "conv_general" || op == "maxpool" || op == "resize_nn" || op == "ew_unary" ||
        op == "copy_c")
      return true;
    if (op == "conv1x1") return p.ref(n.outs[0]).dims.size() == 4;
    if (op == "concat4") return n.ai("outer", 1) == 1;
    if (op == "ew_binary") return elementwise_same(n) || per_channel_bcast(p, n, nullptr);
    return false;
  };
  for (auto &kv : p.tensors()) {
    const PlanTensor &t = kv.second;
    if (!is_act4(t) || t.is_input || t.is_output) continue;
    if (t.dims[2] * t.dims[3] <= 1) continue;
    auto pit = prod.find(t.name);
    if (pit == prod.end() || !producer_ok(nodes[(size_t)pit->second])) continue;
    bool ok = true;
    auto cit = cons.find(t.name);
    if (cit != cons.end())
      for (const auto &c : cit->second)
        if (!consumer_ok(nodes[(size_t)c.first], c.second)) ok = false;
    if (ok) nhwc_names_.insert(t.name);
  }
  // copy_c: channels-last output only as a view of a channels-last parent at an
  // aligned channel offset (16-byte TMA base alignment), else it stays planar.
  for (const auto &n : nodes) {
    if (n.op != "copy_c") continue;
    const bool parent = nhwc_names_.count(n.ins[0]) != 0;
    if (!parent || n.ai("c0", 0) % 8 != 0 || n.ai("dst_off", 0) != 0) nhwc_names_.erase(n.outs[0]);
  }
  // load-time fusions
  if (!(flags_ & kFlagNoFusion)) {
    std::vector<std::string> allowed;
    for (const auto &n : nodes) {
      if (n.op != "concat4" || !nhwc_names_.count(n.outs[0])) continue;
      bool ok = true;
      for (size_t s = 0; s < n.ins.size() && s < 4; ++s)
        if (n.ins[s] != "-" && !nhwc_names_.count(n.ins[s])) ok = false;
      if (ok) allowed.push_back(n.outs[0]);
    }
    p.fuse_concat_conv1x1(allowed);
    p.fuse_residual_add();
    std::vector<std::string> merged;
    p.fuse_sibling_convs(nhwc_names_, &merged);
    nhwc_names_.insert(merged.begin(), merged.end());
  }
  stats_.fusions_concat = p.fusions_concat;
  stats_.fusions_res = p.fusions_res;
}

// ============================================================================ tensors
void Engine::build_tensors() {
  Plan &p = *plan_;
  const auto &nodes = p.nodes();
  std::set<std::string> used;
  used.insert(p.input());
  for (const auto &o : p.outputs()) used.insert(o);
  for (const auto &n : nodes) {
    for (const auto &i : n.ins)
      if (i != "-") used.insert(i);
    for (const auto &o : n.outs)
      if (o != "-") used.insert(o);
  }
  for (const auto &name : used) {
    const PlanTensor &pt = p.ref(name);
    TensorRt t;
    t.name = name;
    t.dims = pt.dims;
    t.numel = pt.numel();
    t.is_init = pt.is_init;
    t.is_input = pt.is_input;
    t.is_output = pt.is_output;
    if (!t.is_init && !t.dims.empty() && t.dims[0] != 1)
      throw std::runtime_error("CudaPlanModel: activation '" + name + "' must have batch dimension 1 in the plan");
    if (t.dims.size() == 4) {
      t.C = (int)t.dims[1];
      t.H = (int)t.dims[2];
      t.W = (int)t.dims[3];
    }
    tid_[name] = (int)T_.size();
    T_.push_back(t);
  }
  auto set_dense = [](TensorRt &t) {
    t.nhwc = false;
    t.dense = true;
    t.Cs = t.C;
    if (t.dims.size() == 4) {
      t.sx = 1;
      t.sy = t.W;
      t.sc = (int64_t)t.H * t.W;
    }
    t.sb = t.is_init ? 0 : t.numel;
    t.bytes_per_img = t.numel * 2;
  };
  auto set_nhwc = [](TensorRt &t) {
    t.nhwc = true;
    t.dense = false;
    t.Cs = (int)round_up(t.C, 8);
    t.sc = 1;
    t.sx = t.Cs;
    t.sy = (int64_t)t.W * t.Cs;
    t.sb = (int64_t)t.H * t.W * t.Cs;
    t.bytes_per_img = t.sb * 2;
  };
  // defaults: every tensor owns dense storage
  for (size_t i = 0; i < T_.size(); ++i) {
    set_dense(T_[i]);
    T_[i].root = (int)i;
  }
  // channels-last roots and views, in node order (parents first)
  for (const auto &n : nodes) {
    const std::string &on = n.outs[0];
    TensorRt &o = T_[(size_t)tid(on)];
    if (n.op == "reshape" || n.op == "flatten") {
      const TensorRt &in = T_[(size_t)tid(n.ins[0])];
      if (!in.dense) throw std::runtime_error("CudaPlanModel: reshape of a non-planar tensor: " + n.ins[0]);
      o.root = in.root;
      o.elem_off = in.elem_off;
      continue;
    }
    if (!nhwc_names_.count(on)) continue;
    if (n.op == "copy_c") {
      const TensorRt &in = T_[(size_t)tid(n.ins[0])];
      o.nhwc = true;
      o.dense = false;
      o.root = in.root;
      o.elem_off = in.elem_off + n.ai("c0", 0);
      o.Cs = in.Cs;
      o.sc = 1;
      o.sx = in.sx;
      o.sy = in.sy;
      o.sb = in.sb;
      o.bytes_per_img = 0;
      continue;
    }
    set_nhwc(o);
  }
  // Concat in place: when every source of a planar concat4 is a convolution
  // output that nothing else reads (directly or through reshapes), the
  // convolutions write their slices of the concat output through strided views
  // and the concat launches nothing.  The head's anchor-axis concats
  // (box/kpt/cls over the three scales) are of this kind.
  if (!(flags_ & kFlagNoFusion)) {
    std::map<int, std::vector<int>> readers;  // storage root -> reading nodes (views excluded)
    std::map<int, std::string> producer;      // storage root -> producing op
    for (size_t ni = 0; ni < nodes.size(); ++ni) {
      const auto &n = nodes[ni];
      if (n.op == "reshape" || n.op == "flatten") continue;
      for (const auto &in : n.ins)
        if (in != "-") readers[T_[(size_t)tid(in)].root].push_back((int)ni);
      producer[T_[(size_t)tid(n.outs[0])].root] = n.op;
    }
    for (int ni = (int)nodes.size() - 1; ni >= 0; --ni) {
      const auto &n = nodes[(size_t)ni];
      if (n.op != "concat4") continue;
      const int y = tid(n.outs[0]);
      const TensorRt &Y = T_[(size_t)y];
      if (Y.nhwc || !Y.dense || Y.root != y) continue;
      const int cnt[4] = {n.ai("ca", 0), n.ai("cb", 0), n.ai("cc", 0), n.ai("cd", 0)};
      const int64_t outer = n.ai("outer", 1), inner = n.ai("inner", 1);
      const int64_t S = (int64_t)cnt[0] + cnt[1] + cnt[2] + cnt[3];
      bool ok = true;
      int roots[4] = {-1, -1, -1, -1};
      for (int k = 0; k < 4 && ok; ++k) {
        if (cnt[k] <= 0) continue;
        if ((size_t)k >= n.ins.size() || n.ins[(size_t)k] == "-") { ok = false; break; }
        const int r = T_[(size_t)tid(n.ins[(size_t)k])].root;
        const TensorRt &R = T_[(size_t)r];
        const std::string &pop = producer.count(r) ? producer[r] : std::string();
        const bool conv = pop == "conv1x1" || pop == "conv3x3" || pop == "conv1x1_cat4";
        const auto &rd = readers[r];
        ok = conv && R.root == r && R.dense && !R.nhwc && !R.is_init && !R.is_input && !R.is_output &&
             R.dims.size() == 4 && rd.size() == 1 && rd[0] == ni &&
             ((outer == R.C && (int64_t)cnt[k] * inner == (int64_t)R.H * R.W) ||
              (outer == 1 && (int64_t)cnt[k] * inner == R.numel));
        for (int j = 0; j < k && ok; ++j) ok = roots[j] != r;
        roots[k] = r;
      }
      if (!ok) continue;
      int64_t off = 0;
      for (int k = 0; k < 4; ++k) {
        if (cnt[k] <= 0) continue;
        TensorRt &R = T_[(size_t)roots[k]];
        R.root = y;
        R.elem_off = Y.elem_off + off * inner;
        R.dense = false;
        R.sx = 1;
        R.sy = R.W;
        R.sc = outer == 1 ? (int64_t)R.H * R.W : S * inner;
        R.sb = Y.sb;
        R.bytes_per_img = 0;
        for (auto &v : T_)  // reshapes of the source follow it
          if (&v != &R && v.root == roots[k]) {
            v.root = y;
            v.elem_off = R.elem_off;
            v.dense = false;
          }
        off += cnt[k];
      }
      elided_nodes_.insert(ni);
    }
  }
  for (auto &t : T_) {
    if (t.root != tid(t.name)) ++stats_.views;
    else if (!t.is_init) ++stats_.roots;
    if (t.nhwc) ++stats_.nhwc_tensors;
  }
}

// ============================================================================ allocation
void Engine::lifetimes() {
  const auto &nodes = plan_->nodes();
  const int N = (int)nodes.size();
  auto touch = [&](const std::string &name, int i) {
    if (name == "-") return;
    TensorRt &t = T_[(size_t)tid(name)];
    if (t.is_init) return;
    TensorRt &r = T_[(size_t)t.root];
    if (r.birth < 0 || i < r.birth) r.birth = i;
    if (i > r.death) r.death = i;
  };
  touch(plan_->input(), 0);
  for (int i = 0; i < N; ++i) {
    for (const auto &in : nodes[(size_t)i].ins) touch(in, i);
    for (const auto &o : nodes[(size_t)i].outs) touch(o, i);
  }
  for (const auto &u : tail_uses_) touch(T_[(size_t)u.first].name, u.second);  // fused tails read late
  for (const auto &o : plan_->outputs()) T_[(size_t)T_[(size_t)tid(o)].root].death = N;
  T_[(size_t)T_[(size_t)tid(plan_->input())].root].death = N;  // the input outlives the run
}

void Engine::alloc_aux() {
  if (dry_) return;
  check(cudaMalloc(&status_, sizeof(int)), "cudaMalloc(status)");
  check(cudaMemset(status_, 0, sizeof(int)), "cudaMemset(status)");
  check(cudaMalloc(&in_f32_, (size_t)input_numel() * max_batch_ * sizeof(float)), "cudaMalloc(input f32)");
}

// Arena placement.  Two roots may share bytes only when every step touching
// one of them is ordered before every step touching the other, by a
// dependency or by the order of one stream (plan_streams); the graph input is
// touched before the first step and the outputs after the last.  With one
// stream this is the node-order liveness of the serial executor.
void Engine::allocate() {
  const int S = (int)steps_.size();
  const int kSource = -1, kSink = S;
  std::vector<std::vector<int>> acc(T_.size());
  for (int j = 0; j < S; ++j) {
    for (int r : step_reads_[(size_t)j]) acc[(size_t)r].push_back(j);
    for (int r : step_writes_[(size_t)j]) acc[(size_t)r].push_back(j);
  }
  // The graph input keeps its own bytes for the whole run (touched before the
  // first step and after the last), as the reference's input buffer does
  // (only `tensor` lines enter its pool, src/PlanModel.cpp:505-510): run()
  // repeated after one setInput() reads the same input every time.
  acc[(size_t)T_[(size_t)tid(plan_->input())].root].push_back(kSource);
  acc[(size_t)T_[(size_t)tid(plan_->input())].root].push_back(kSink);
  for (const auto &o : plan_->outputs()) acc[(size_t)T_[(size_t)tid(o)].root].push_back(kSink);
  for (size_t i = 0; i < T_.size(); ++i)  // values passed inside a fused step only
    if ((int)i == T_[i].root && !T_[i].is_init) T_[i].materialized = !acc[i].empty() || (flags_ & kFlagNoPool);
  auto reaches = [&](int a, int b) -> bool {  // a finishes before b starts
    if (a == kSource) return b != kSource;
    if (b == kSink) return a != kSink;
    if (a == kSink || b == kSource || a == b) return false;
    return (reach_[(size_t)a][(size_t)b >> 6] >> (b & 63)) & 1ull;
  };
  auto before = [&](int x, int y) -> bool {
    for (int a : acc[(size_t)x])
      for (int b : acc[(size_t)y])
        if (!reaches(a, b)) return false;
    return true;
  };
  const bool no_pool = (flags_ & kFlagNoPool) != 0;  // diagnostics: no reuse, every tensor stays readable
  auto conflict = [&](int x, int y) { return no_pool || !(before(x, y) || before(y, x)); };

  std::vector<int> roots;
  for (size_t i = 0; i < T_.size(); ++i)
    if ((int)i == T_[i].root && !T_[i].is_init && T_[i].birth >= 0) roots.push_back((int)i);
  auto bytes_of = [&](int r) { return round_up(T_[(size_t)r].bytes_per_img * max_batch_, 256); };
  std::sort(roots.begin(), roots.end(), [&](int a, int b) {
    if (bytes_of(a) != bytes_of(b)) return bytes_of(a) > bytes_of(b);
    return T_[(size_t)a].birth < T_[(size_t)b].birth;
  });
  std::vector<int> placed;
  int64_t top = 0;
  for (int r : roots) {
    const int64_t sz = bytes_of(r);
    stats_.requested_bytes += sz;
    std::vector<std::pair<int64_t, int64_t>> busy;
    for (int q : placed)
      if (conflict(r, q)) busy.push_back({T_[(size_t)q].arena_off, T_[(size_t)q].arena_off + bytes_of(q)});
    std::sort(busy.begin(), busy.end());
    int64_t cur = 0;
    for (const auto &iv : busy) {
      if (cur + sz <= iv.first) break;
      cur = std::max(cur, round_up(iv.second, 256));
    }
    T_[(size_t)r].arena_off = cur;
    top = std::max(top, cur + sz);
    placed.push_back(r);
  }
  arena_bytes_ = std::max<int64_t>(top, 256);
  stats_.arena_bytes = arena_bytes_;
  // self-check: roots whose accesses are not ordered never share bytes
  for (size_t i = 0; i < placed.size(); ++i)
    for (size_t j = i + 1; j < placed.size(); ++j) {
      if (!conflict(placed[i], placed[j])) continue;
      const int64_t a0 = T_[(size_t)placed[i]].arena_off, a1 = a0 + bytes_of(placed[i]);
      const int64_t b0 = T_[(size_t)placed[j]].arena_off, b1 = b0 + bytes_of(placed[j]);
      if (a0 < b1 && b0 < a1) ++stats_.overlap_errors;
    }
  if (stats_.overlap_errors) throw std::runtime_error("CudaPlanModel: activation allocator produced overlaps");
  if (!dry_) {
    check(cudaMalloc(&arena_, (size_t)arena_bytes_), "cudaMalloc(arena)");
    check(cudaMemset(arena_, 0, (size_t)arena_bytes_), "cudaMemset(arena)");
  }
  uint8_t *base = dry_ ? nullptr : arena_;
  for (auto &t : T_) {
    if (t.is_init) continue;
    const TensorRt &r = T_[(size_t)t.root];
    if (r.arena_off < 0) continue;
    t.dptr = reinterpret_cast<__half *>(base + r.arena_off) + t.elem_off;
  }
}

void Engine::upload_weights() {
  int64_t total = 0;
  for (auto &t : T_)
    if (t.is_init) total += round_up(t.numel * 2, 256);
  stats_.weight_bytes = total;
  if (dry_ || total == 0) return;
  void *w = nullptr;
  check(cudaMalloc(&w, (size_t)total), "cudaMalloc(weights)");
  dev_allocs_.push_back(w);
  int64_t off = 0;
  for (auto &t : T_) {
    if (!t.is_init) continue;
    const PlanTensor &pt = plan_->ref(t.name);
    t.dptr = reinterpret_cast<__half *>(static_cast<uint8_t *>(w) + off);
    check(cudaMemcpy(t.dptr, pt.host.data(), (size_t)t.numel * 2, cudaMemcpyHostToDevice), "upload init");
    off += round_up(t.numel * 2, 256);
  }
}

View4 Engine::view(int i) const {
  const TensorRt &t = T_[(size_t)i];
  View4 v{};
  v.ptr = t.dptr;
  if (t.dims.size() == 4) {
    v.C = t.C;
    v.H = t.H;
    v.W = t.W;
    v.sc = t.sc;
    v.sy = t.sy;
    v.sx = t.sx;
  } else if (t.dims.size() == 2) {  // [1, K] -> K channels of a 1x1 image
    v.C = (int)t.dims[1];
    v.H = v.W = 1;
    v.sc = 1;
    v.sy = v.sx = v.C;
  } else if (t.dims.size() >= 3) {  // [1, C, rest...] -> C x 1 x rest (planar)
    v.C = (int)t.dims[1];
    int64_t rest = 1;
    for (size_t k = 2; k < t.dims.size(); ++k) rest *= t.dims[k];
    v.H = 1;
    v.W = (int)rest;
    v.sc = rest;
    v.sy = rest;
    v.sx = 1;
  } else {
    v.C = (int)t.numel;
    v.H = v.W = 1;
    v.sc = 1;
    v.sy = v.sx = v.C;
  }
  v.sb = t.is_init ? 0 : t.sb;
  return v;
}

__half *Engine::input_device_ptr() const { return T_[(size_t)tid(plan_->input())].dptr; }

// ============================================================================ lowering
namespace {

struct ConvCfg {
  int ksize = 1, stride = 1, pad = 0;
  int nsrc = 1;
  int src[kConvMaxSrc] = {-1, -1, -1, -1};
  int srcC[kConvMaxSrc] = {0, 0, 0, 0};
  int chunks[kConvMaxSrc] = {0, 0, 0, 0};
  int cin_total = 0;
  int cout = 0, Np = 0, BN = 0, BK = 0, n_tiles = 1, num_kb = 0, taps = 1;
  int Ho = 0, Wo = 0, TH = 0, TW = 0;
  int act = 0, act_kind = kActGemm;
  int out = -1, res = -1;
  int halo = 0, kern_kb = 0;  // 3x3 halo mode (= the stride) and the k-blocks the kernel walks
  __half *wp = nullptr;    // packed [Np][Kp]
  __half *bias = nullptr;  // [Np] padded
};

// Per-launch tile geometry of a tensor-core conv.  A tile is `mb` M blocks of
// 128 output pixels (mb accumulators of BN columns side by side in TMEM):
// 1x1 takes mb * 128 consecutive pixels, 3x3 halo a 16-row x 8*mb-column
// window.  Larger tiles spread the per-tile pipeline handshakes over more
// pixels; smaller ones give more tiles to spread over the SMs.
struct ConvGeom {
  int mb = 1, TW = 0, TH = 0, hx = 0, hy = 0, halo_bytes = 0;
  int a_tile = 0, resident_b = 0, kb_per_stage = 1, stages = 0, smem = 0;
};

constexpr int kConvSmemCap = 232448 - 2048 /*static smem + barriers*/ - 1024 /*1 KB alignment*/;

bool conv_geom(const ConvCfg &c, int mb, ConvGeom *g) {
  ConvGeom r;
  r.mb = mb;
  if (c.ksize == 3 && !c.halo) {
    if (c.Wo % 16 == 0) {  // M block j: rows 8j .. 8j+7 of a 16-wide tile
      r.TW = 16;
      r.TH = 8 * mb;
    } else {
      if (mb != 1) return false;
      r.TW = std::min(c.Wo, 128);
      r.TH = std::max(1, 128 / r.TW);
    }
  } else if (c.halo) {
    r.TW = 8 * mb;
    r.TH = 16;
    r.hx = c.stride == 1 ? r.TW + 2 : r.TW + 1;  // stride 2: one phase (every other column)
    r.hy = c.stride == 1 ? 16 + 2 : 16 + 1;
    if (r.hx * c.stride > 256) return false;      // TMA box extent
    r.halo_bytes = (int)round_up((int64_t)r.hx * r.hy * c.BK * 2, 1024);
  }
  r.a_tile = c.halo ? r.halo_bytes * (c.halo == 2 ? 4 : 1) : 128 * mb * c.BK * 2;
  const int b_tile = (int)round_up((int64_t)c.BN * c.BK * 2, 1024);
  const int bres = b_tile * c.num_kb;
  // weights resident when they fit beside two stages; otherwise they travel
  // with the A tiles (halo: each stage carries its chunk's nine tap blocks).
  // A halo conv split into several N tiles keeps one N tile's weights per CTA
  // (the launch grid is then a multiple of n_tiles), and only that way.
  const bool split = c.n_tiles > 1 && c.halo;
  r.resident_b = ((split || (c.n_tiles == 1 && bres <= 96 * 1024)) && kConvSmemCap - bres >= 2 * r.a_tile) ? 1 : 0;
  if (split && !r.resident_b) return false;
  const int kb_bytes = r.a_tile + (r.resident_b ? 0 : (c.halo ? 9 : 1) * b_tile);
  const int ring = kConvSmemCap - (r.resident_b ? bres : 0);
  // k-blocks per pipeline stage: one full/empty handshake costs a few hundred
  // cycles, far more than a 16-channel k-block's MMA, so small k-blocks travel
  // in groups (a divisor of the k-block count, <= 48 KB, >= 3 stages)
  r.kb_per_stage = 1;
  for (int gk = c.kern_kb; gk >= 2; --gk)
    if (c.kern_kb % gk == 0 && gk * kb_bytes <= 48 * 1024 && ring / (gk * kb_bytes) >= 3) {
      r.kb_per_stage = gk;
      break;
    }
  const int stage_bytes = r.kb_per_stage * kb_bytes;
  r.stages = std::min(kConvMaxStages, ring / stage_bytes);
  if (r.stages < 2) return false;
  r.smem = (r.resident_b ? bres : 0) + r.stages * stage_bytes + 1024;
  r.smem = std::max(r.smem, 120 * 1024);  // one CTA per SM (TMEM never contended)
  *g = r;
  return true;
}

// Launch grid of a conv: one CTA per SM at most; with resident weights over
// several N tiles, a multiple of n_tiles (each CTA keeps one N tile).
int conv_grid(const ConvTcArgs &a, int sms) {
  int g = std::max(1, std::min(a.m_tiles * a.n_tiles, sms));
  if (a.resident_b && a.n_tiles > 1) g = std::max(a.n_tiles, g / a.n_tiles * a.n_tiles);
  return g;
}

// M tiles of one launch at batch B with geometry g.
long long conv_m_tiles(const ConvCfg &c, const ConvGeom &g, int B) {
  if (c.ksize == 1) return ((long long)B * c.Ho * c.Wo + 128LL * g.mb - 1) / (128LL * g.mb);
  return (long long)B * ((c.Wo + g.TW - 1) / g.TW) * ((c.Ho + g.TH - 1) / g.TH);
}

// Epilogue teams (tiles in the epilogue at once) for a launch of `tiles`
// tiles: with few tiles per CTA each tile wants all 16 epilogue warps, with
// many, tiles overlap in the epilogue.
int conv_nteams(const ConvCfg &c, long long tiles, int sms) {
  const long long per_cta = (tiles + sms - 1) / sms;
  const int most = c.BN <= 128 ? 4 : 2;
  return per_cta >= 8 ? most : per_cta >= 2 ? std::min(2, most) : 1;
}

// Tile geometries of a launch at batch B, cheapest first by the cost
// ceil(tiles / SMs) * (kTileCost + mb): the per-tile handshakes counted as
// kTileCost M blocks of work, among the tile sizes that fit shared memory and
// leave TMEM for the accumulator buffers.  Two buffers per team let the MMA
// warp fill a team's next tile while the team drains the current one; one
// buffer per team is charged kSingleBufCost.
constexpr double kTileCost = 2.0;
constexpr double kSingleBufCost = 1.25;
constexpr double kOtherTeamsCost = 1.5;
constexpr int kConvTuneCands = 16;  // geometries timed by the load-time tuning
struct ConvCand {
  ConvGeom g;
  int nteams = 1, nbuf = 1;
  double cost = 0.0;
  int mode = 0;  // index of the conv's layout (ConvCfg variant)
};
std::vector<ConvCand> conv_candidates(const ConvCfg &c, int B, int sms) {
  std::vector<ConvCand> out;
  const int max_mb = (c.ksize == 3 && !c.halo && c.Wo % 16 != 0) ? 1 : 8;
  for (int mb = 1; mb <= max_mb; ++mb) {
    ConvGeom g;
    if (!conv_geom(c, mb, &g)) continue;
    if (mb > 1 && g.stages < 3) continue;  // keep loads of two tiles ahead in flight
    const long long tiles = conv_m_tiles(c, g, B) * c.n_tiles;
    const int nt_model = conv_nteams(c, tiles, sms);
    const double base = (double)((tiles + sms - 1) / sms) * (kTileCost + mb);
    // the tile-count rule's team count first; the other counts are kept as
    // candidates for the load-time tuning (charged kOtherTeamsCost)
    const int counts[4] = {nt_model, nt_model == 4 ? 2 : 4, nt_model == 1 ? 2 : 1, nt_model == 2 ? 1 : 2};
    for (int ci = 0; ci < 4; ++ci) {
      const int nt = counts[ci];
      if (ci == 3 && (nt == counts[1] || nt == counts[2])) continue;  // {model, the other two} once each
      if (nt * mb * c.BN > 512 || (nt == 4 && c.BN > 128)) continue;
      const double cb = base * (nt == nt_model ? 1.0 : kOtherTeamsCost);
      if (2 * nt * mb * c.BN <= 512 && tiles > (long long)sms * nt) out.push_back({g, nt, 2 * nt, cb});
      out.push_back({g, nt, nt, cb * kSingleBufCost});
    }
  }
  if (out.empty()) throw std::runtime_error("CudaPlanModel: conv tile does not fit shared memory");
  std::stable_sort(out.begin(), out.end(), [](const ConvCand &x, const ConvCand &y) { return x.cost < y.cost; });
  return out;
}

int pick_bk(int c) {
  const int c16 = (int)round_up(c, 16);
  if (c16 >= 64) return 64;
  if (c16 >= 32) return 32;
  return 16;
}

int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

}  // namespace

// ============================================================================ fused planar tails
// A region of reshape / slice_axis / concat4 / ew_binary / ew_unary nodes (and
// the DFL chain permute_0213 -> softmax_axis -> conv1x1) ending in a plan
// output, whose tensors all keep the anchor axis A innermost, becomes one
// TailProgram: the node DAG expanded per output row (rows, slices, concats and
// broadcasts resolved on the host, scalar inits folded to constants, every
// (tensor, row) value computed once), executed per anchor column on the device.
void Engine::plan_tails() {
  Plan &p = *plan_;
  const auto &nodes = p.nodes();
  std::map<std::string, int> producer;
  std::map<std::string, std::vector<int>> consumers;
  for (size_t ni = 0; ni < nodes.size(); ++ni) {
    for (const auto &in : nodes[ni].ins)
      if (in != "-") consumers[in].push_back((int)ni);
    producer[nodes[ni].outs[0]] = (int)ni;
  }
  auto sole_consumer = [&](const std::string &t) -> int {
    auto it = consumers.find(t);
    return (it != consumers.end() && it->second.size() == 1) ? it->second[0] : -1;
  };
  // DFL chain ending at conv node c: returns the permute's input tensor, or "".
  auto dfl_source = [&](int c) -> std::string {
    const PlanNode &cv = nodes[(size_t)c];
    if (cv.op != "conv1x1" || cv.ins.size() < 2 || (cv.ins.size() > 3 && cv.ins[3] != "-")) return "";
    auto ps = producer.find(cv.ins[1]);
    if (ps == producer.end()) return "";
    const PlanNode &sm = nodes[(size_t)ps->second];
    if (sm.op != "softmax_axis" || sole_consumer(cv.ins[1]) != c) return "";
    auto pp = producer.find(sm.ins[0]);
    if (pp == producer.end()) return "";
    const PlanNode &pm = nodes[(size_t)pp->second];
    if (pm.op != "permute_0213" || pm.ai("mode", 0) != 0 || sole_consumer(sm.ins[0]) != ps->second) return "";
    const int D1 = pm.ai("D1", 1), D2 = pm.ai("D2", 1);
    const int64_t I = pm.ai("I", 1);
    if (D2 != 16 || sm.ai("outer", 1) != 1 || sm.ai("axdim", 0) != D2 || sm.ai("inner", 1) != (int64_t)D1 * I)
      return "";
    const TensorRt &w = T_[(size_t)tid(cv.ins[0])];
    if (!w.is_init || w.dims.empty() || w.numel != w.dims[0] * D2 || w.dims[0] > 8) return "";
    return pm.ins[0];
  };

  for (const auto &oname : p.outputs()) {
    auto po = producer.find(oname);
    if (po == producer.end()) continue;
    const TensorRt &O = T_[(size_t)tid(oname)];
    if (O.nhwc || !O.dense || O.dims.empty()) continue;
    const int64_t A = O.dims.back();
    if (A < 1 || O.numel % A != 0) continue;
    auto planar_a = [&](const std::string &t) {
      const TensorRt &x = T_[(size_t)tid(t)];
      return !x.nhwc && !x.dims.empty() && x.dims.back() == A && x.numel % A == 0;
    };
    auto candidate = [&](int ni) -> bool {
      const PlanNode &n = nodes[(size_t)ni];
      if (!planar_a(n.outs[0])) return false;
      if (n.op == "reshape" || n.op == "flatten" || n.op == "ew_unary") return true;
      if (n.op == "slice_axis") return n.ai("inner", 1) == A;
      if (n.op == "concat4") return n.ai("inner", 1) == A;
      if (n.op == "ew_binary") return true;
      if (n.op == "conv1x1") return !dfl_source(ni).empty();
      return false;
    };
    if (!candidate(po->second)) continue;
    std::set<int> region{po->second};
    auto data_inputs = [&](int ni) {
      const PlanNode &n = nodes[(size_t)ni];
      std::vector<std::string> v;
      if (n.op == "conv1x1") return v;  // the DFL chain is taken whole
      const size_t k = n.op == "concat4" ? std::min<size_t>(4, n.ins.size()) : n.op == "ew_binary" ? 2 : 1;
      for (size_t i = 0; i < k && i < n.ins.size(); ++i)
        if (n.ins[i] != "-") v.push_back(n.ins[i]);
      return v;
    };
    for (bool changed = true; changed;) {
      changed = false;
      for (int ni : std::vector<int>(region.begin(), region.end()))
        for (const auto &x : data_inputs(ni)) {
          const TensorRt &t = T_[(size_t)tid(x)];
          auto pr = producer.find(x);
          if (t.is_init || t.is_input || t.is_output || pr == producer.end() || region.count(pr->second)) continue;
          bool inside = true;
          for (int c : consumers[x]) inside = inside && region.count(c);
          if (inside && candidate(pr->second)) {
            region.insert(pr->second);
            changed = true;
          }
        }
    }
    // ---- expand per output row
    // values in creation (post-) order; loads and constants become operands
    enum { vLoad, vConst, vBin, vUn, vDfl };
    struct Val {
      int code, a, b, arg;
    };
    std::vector<Val> ops;
    std::vector<std::pair<int, int>> events;  // (value, -1) created; (value, row) stored to output row
    std::vector<std::pair<int, bool>> leaf_ids;  // (tensor, shared across images)
    std::map<std::string, int> leaf_of;
    std::vector<TailDfl> dfls;
    std::map<std::pair<int, int>, int> dfl_of;  // (conv node, cout row) -> table entry
    std::map<std::pair<std::string, int64_t>, int> memo;
    std::set<int> dfl_chain;                    // softmax / permute nodes folded into DFL ops
    bool ok = true;
    auto fail = [&]() {
      ok = false;
      return -1;
    };
    auto leaf = [&](const std::string &x, bool shared) -> int {
      auto it = leaf_of.find(x);
      if (it != leaf_of.end()) return it->second;
      const TensorRt &t = T_[(size_t)tid(x)];
      if ((int)leaf_ids.size() >= kTailMaxLeaves || (!shared && !t.dense)) return fail();
      leaf_ids.push_back({tid(x), shared});
      return leaf_of[x] = (int)leaf_ids.size() - 1;
    };
    auto push = [&](int code, int a, int b, int arg) {
      ops.push_back(Val{code, a, b, arg});
      events.push_back({(int)ops.size() - 1, -1});
      return (int)ops.size() - 1;
    };
    auto cst = [&](float f) {
      int bits;
      std::memcpy(&bits, &f, 4);
      return push(vConst, -1, -1, bits);
    };
    auto init_value = [&](const std::string &x, int64_t flat) -> float {
      const PlanTensor &pt = p.ref(x);
      return flat < (int64_t)pt.host.size() ? f16_to_f32_host(pt.host[(size_t)flat]) : 0.0f;
    };
    std::function<int(const std::string &, int64_t)> emit = [&](const std::string &x, int64_t row) -> int {
      if (!ok) return -1;
      auto key = std::make_pair(x, row);
      auto it = memo.find(key);
      if (it != memo.end()) return it->second;
      const TensorRt &t = T_[(size_t)tid(x)];
      int v = -1;
      auto pr = producer.find(x);
      if (t.is_init) {
        if (t.numel == 1) v = cst(init_value(x, 0));
        else if (t.numel % A == 0 && row < t.numel / A) v = push(vLoad, leaf(x, true), -1, (int)row);
        else v = fail();
      } else if (pr == producer.end() || !region.count(pr->second)) {
        if (!planar_a(x) || row >= t.numel / A) v = fail();
        else v = push(vLoad, leaf(x, false), -1, (int)row);
      } else {
        const PlanNode &n = nodes[(size_t)pr->second];
        if (n.op == "reshape" || n.op == "flatten") {
          v = emit(n.ins[0], row);
        } else if (n.op == "slice_axis") {
          const int64_t len = n.ai("len", 0), axdim = n.ai("axdim", 0), start = n.ai("start", 0);
          v = len > 0 ? emit(n.ins[0], (row / len) * axdim + start + row % len) : fail();
        } else if (n.op == "concat4") {
          const int64_t cnt[4] = {n.ai("ca", 0), n.ai("cb", 0), n.ai("cc", 0), n.ai("cd", 0)};
          const int64_t S = cnt[0] + cnt[1] + cnt[2] + cnt[3];
          const int64_t o = row / S;
          int64_t j = row % S;
          int k = 0;
          while (k < 4 && j >= cnt[k]) j -= cnt[k++];
          v = (k < 4 && (size_t)k < n.ins.size()) ? emit(n.ins[(size_t)k], o * cnt[k] + j) : fail();
        } else if (n.op == "ew_unary") {
          const int a = emit(n.ins[0], row);
          v = ok ? push(vUn, a, -1, n.ai("op", 0)) : -1;
        } else if (n.op == "ew_binary") {
          int opv[2] = {-1, -1};
          const bool bsc = n.ai("b_scalar", 0) != 0;
          for (int w = 0; w < 2 && ok; ++w) {
            const std::string &xi = n.ins[(size_t)w];
            const TensorRt &ti = T_[(size_t)tid(xi)];
            if (!n.attr.count("bdims")) {
              if (w == 1 && bsc) opv[w] = ti.is_init ? cst(init_value(xi, 0)) : fail();
              else opv[w] = emit(xi, row);
              continue;
            }
            const std::vector<int64_t> bd = parse_ints(n.attr.at("bdims"));
            const int R = (int)bd.size() / 3;
            if (R < 2 || bd[(size_t)R - 1] != A) {
              opv[w] = fail();
              continue;
            }
            const int64_t *st = &bd[(size_t)(R * (1 + w))];
            int64_t rem = row, flat = 0;
            for (int d = R - 2; d >= 1; --d) {
              flat += (rem % bd[(size_t)d]) * st[d];
              rem /= bd[(size_t)d];
            }
            if (st[R - 1] == 1 && flat % A == 0) opv[w] = emit(xi, flat / A);
            else if (st[R - 1] == 0 && ti.is_init) opv[w] = cst(init_value(xi, flat));
            else opv[w] = fail();
          }
          v = ok ? push(vBin, opv[0], opv[1], n.ai("op", 0)) : -1;
        } else if (n.op == "conv1x1") {
          const std::string src = dfl_source(pr->second);
          const PlanNode &pm = nodes[(size_t)producer[nodes[(size_t)producer[n.ins[1]]].ins[0]]];
          const int D1 = pm.ai("D1", 1);
          dfl_chain.insert(producer[n.ins[1]]);
          dfl_chain.insert(producer[nodes[(size_t)producer[n.ins[1]]].ins[0]]);
          const int co = (int)(row / D1), j = (int)(row % D1);
          auto key2 = std::make_pair(pr->second, co);
          if (!dfl_of.count(key2)) {
            if ((int)dfls.size() >= kTailMaxDfl) {
              v = fail();
            } else {
              TailDfl D{};
              for (int q = 0; q < 16; ++q) D.w[q] = init_value(n.ins[0], (int64_t)co * 16 + q);
              D.bias = (n.ins.size() > 2 && n.ins[2] != "-") ? init_value(n.ins[2], co) : 0.0f;
              D.act = n.ai("act", 0);
              dfls.push_back(D);
              dfl_of[key2] = (int)dfls.size() - 1;
            }
          }
          if (ok && T_[(size_t)tid(src)].numel / A < (int64_t)(j + 1) * 16) v = fail();
          if (ok) v = push(vDfl, leaf(src, false), j * 16, dfl_of[key2]);
        } else {
          v = fail();
        }
      }
      if (ok) memo[key] = v;
      return v;
    };
    for (int64_t r = 0; r < O.numel / A && ok; ++r) {
      const int v = emit(oname, r);
      if (ok) events.push_back({v, (int)r});
    }
    if (!ok || region.size() + dfl_chain.size() < 3) continue;
    // ---- ops: computed values (loads / constants fold into operands), stores
    // attached to the op that produced the value just before, else a copy op
    struct Pending {
      TailOp op;
      int val;  // value computed by this op (-1 for copies)
      int ra, rb;  // slot operands read: value ids, or -1
    };
    std::vector<Pending> seq;
    std::vector<int> op_of(ops.size(), -1);
    auto operand = [&](int v, int &reads) -> TailOperand {
      reads = -1;
      const Val &x = ops[(size_t)v];
      if (x.code == vLoad) return TailOperand{kTailLeafRow, x.a, x.arg};
      if (x.code == vConst) return TailOperand{kTailImm, x.arg, 0};
      reads = v;
      return TailOperand{kTailSlot, -1, 0};
    };
    for (const auto &ev : events) {
      const int v = ev.first;
      const Val &x = ops[(size_t)v];
      if (ev.second < 0) {  // creation
        if (x.code == vLoad || x.code == vConst) continue;
        Pending pd{};
        pd.op.dst = -1;
        pd.op.store_row = -1;
        pd.op.arg = x.arg;
        pd.val = v;
        pd.ra = pd.rb = -1;
        if (x.code == vDfl) {
          pd.op.code = kTailDfl;
          pd.op.a = TailOperand{kTailLeafRow, x.a, x.b};
          pd.op.b = TailOperand{kTailImm, 0, 0};
        } else {
          pd.op.code = x.code == vBin ? kTailBin : kTailUn;
          pd.op.a = operand(x.a, pd.ra);
          pd.op.b = x.code == vBin ? operand(x.b, pd.rb) : TailOperand{kTailImm, 0, 0};
        }
        op_of[(size_t)v] = (int)seq.size();
        seq.push_back(pd);
      } else {  // store of value v to output row ev.second
        if (!seq.empty() && seq.back().val == v && seq.back().op.store_row < 0) {
          seq.back().op.store_row = ev.second;
          continue;
        }
        Pending pd{};
        pd.op.code = kTailCopy;
        pd.op.dst = -1;
        pd.op.store_row = ev.second;
        pd.op.a = operand(v, pd.ra);
        pd.op.b = TailOperand{kTailImm, 0, 0};
        pd.val = -1;
        pd.rb = -1;
        seq.push_back(pd);
      }
    }
    if (seq.size() > (size_t)kTailMaxOps) continue;
    // ---- independent chains (ops linked through slot operands) run on
    // different threads (blockIdx.y); order inside a chain is kept
    std::vector<int> uf(seq.size());
    std::iota(uf.begin(), uf.end(), 0);
    std::function<int(int)> find = [&](int x) { return uf[(size_t)x] == x ? x : uf[(size_t)x] = find(uf[(size_t)x]); };
    for (size_t i = 0; i < seq.size(); ++i)
      for (int r : {seq[i].ra, seq[i].rb})
        if (r >= 0) uf[(size_t)find((int)i)] = find(op_of[(size_t)r]);
    std::map<int, std::vector<int>> chains;  // root -> op indices (in order)
    std::vector<int> chain_order;
    for (size_t i = 0; i < seq.size(); ++i) {
      const int r = find((int)i);
      if (!chains.count(r)) chain_order.push_back(r);
      chains[r].push_back((int)i);
    }
    if ((int)chain_order.size() > kTailMaxComp) continue;
    std::vector<Pending> ordered;
    std::vector<int> comp_begin;
    for (int r : chain_order) {
      comp_begin.push_back((int)ordered.size());
      for (int i : chains[r]) ordered.push_back(seq[(size_t)i]);
    }
    comp_begin.push_back((int)ordered.size());
    seq.swap(ordered);
    // ---- slots by last use within each chain (an op may write the slot its
    // last operand frees)
    std::vector<int> last(ops.size(), -1), slot(ops.size(), -1);
    for (size_t i = 0; i < seq.size(); ++i) {
      if (seq[i].ra >= 0) last[(size_t)seq[i].ra] = (int)i;
      if (seq[i].rb >= 0) last[(size_t)seq[i].rb] = (int)i;
    }
    std::vector<int> free_slots;
    int n_slots = 0, chain_slots = 0;
    TailProgram prog;
    prog.n_comp = (int)chain_order.size();
    for (size_t c = 0; c < comp_begin.size(); ++c) prog.comp_begin[c] = comp_begin[c];
    std::set<int> chain_start(comp_begin.begin(), comp_begin.end() - 1);
    for (size_t i = 0; i < seq.size(); ++i) {
      if (chain_start.count((int)i)) {  // a new chain starts with every slot free
        free_slots.clear();
        chain_slots = 0;
      }
      Pending &pd = seq[i];
      if (pd.ra >= 0) pd.op.a.idx = slot[(size_t)pd.ra];
      if (pd.rb >= 0) pd.op.b.idx = slot[(size_t)pd.rb];
      if (pd.ra >= 0 && last[(size_t)pd.ra] == (int)i) free_slots.push_back(slot[(size_t)pd.ra]);
      if (pd.rb >= 0 && pd.rb != pd.ra && last[(size_t)pd.rb] == (int)i) free_slots.push_back(slot[(size_t)pd.rb]);
      if (pd.val >= 0 && last[(size_t)pd.val] >= 0) {
        int sl;
        if (!free_slots.empty()) {
          auto m = std::min_element(free_slots.begin(), free_slots.end());
          sl = *m;
          free_slots.erase(m);
        } else {
          sl = chain_slots++;
          n_slots = std::max(n_slots, chain_slots);
        }
        slot[(size_t)pd.val] = pd.op.dst = sl;
      }
      prog.ops[prog.n_ops++] = pd.op;
    }
    if (n_slots > kTailMaxSlots) continue;
    prog.n_slots = n_slots;
    prog.n_leaves = (int)leaf_ids.size();
    prog.n_dfl = (int)dfls.size();
    for (size_t i = 0; i < dfls.size(); ++i) prog.dfl[i] = dfls[i];
    prog.A = A;
    const int out_id = tid(oname);
    Step st;
    st.node = po->second;
    st.name = "tail:" + oname;
    st.family = "decode_tail";
    st.info = "ops=" + std::to_string(prog.n_ops) + " chains=" + std::to_string(prog.n_comp) +
              " slots=" + std::to_string(prog.n_slots) + " leaves=" + std::to_string(prog.n_leaves) +
              " dfl=" + std::to_string(prog.n_dfl);
    for (const auto &lf : leaf_ids) {
      const TensorRt &t = T_[(size_t)lf.first];
      if (t.is_init) st.bytes_fixed += (double)t.numel * 2.0;
      else st.bytes_img += (double)t.numel * 2.0;
      if (!t.is_init) tail_uses_.push_back({lf.first, po->second});  // read where the tail runs
    }
    st.bytes_img += (double)O.numel * 2.0;
    auto shared_prog = std::make_shared<TailProgram>(prog);
    auto leaves_v = std::make_shared<std::vector<std::pair<int, bool>>>(leaf_ids);
    // The program compiled at load time into straight-line code (NVRTC); the
    // interpreting kernel runs when that is unavailable or a pointer is not
    // aligned to the vector width.
    std::shared_ptr<TailJit> jit;
    int jit_v = 1;
    if (!(flags_ & kFlagNoJit)) {  // dry runs compile without loading
      TailJitLayout lay;
      lay.A = A;
      lay.out_img = T_[(size_t)out_id].sb;
      bool al4 = A % 4 == 0 && lay.out_img % 4 == 0, al2 = A % 2 == 0 && lay.out_img % 2 == 0;
      for (size_t i = 0; i < leaf_ids.size(); ++i) {
        lay.leaf_img[i] = leaf_ids[i].second ? 0 : T_[(size_t)leaf_ids[i].first].sb;
        lay.leaf_row[i] = A;
        al4 = al4 && lay.leaf_img[i] % 4 == 0;
        al2 = al2 && lay.leaf_img[i] % 2 == 0;
      }
      lay.V = al4 ? 4 : al2 ? 2 : 1;
      jit = std::make_shared<TailJit>();
      std::string err;
      if (jit->build(prog, lay, !dry_, &err)) {
        jit_v = lay.V;
        st.info += " jit=V" + std::to_string(lay.V);
        if (dry_) jit.reset();
      } else {
        jit.reset();
        const size_t nl = err.find('\n');
        st.info += " jit=off(" + err.substr(0, std::min<size_t>(nl, 80)) + ")";
      }
    }
    st.launch = [this, shared_prog, leaves_v, out_id, A, jit, jit_v](int B, cudaStream_t s) -> cudaError_t {
      TailProgram &pr = *shared_prog;  // device pointers are known once the arena is placed
      bool aligned = true;
      for (size_t i = 0; i < leaves_v->size(); ++i) {
        const TensorRt &t = T_[(size_t)(*leaves_v)[i].first];
        pr.leaves[i] = TailLeaf{t.dptr, (*leaves_v)[i].second ? 0 : t.sb, A};
        aligned = aligned && (reinterpret_cast<uintptr_t>(t.dptr) & (uintptr_t)(2 * jit_v - 1)) == 0;
      }
      pr.out = T_[(size_t)out_id].dptr;
      pr.out_img = T_[(size_t)out_id].sb;
      aligned = aligned && (reinterpret_cast<uintptr_t>(pr.out) & (uintptr_t)(2 * jit_v - 1)) == 0;
      if (jit && aligned) return jit->launch(pr, B, g_launch_pdl, s);
      return launch_tail_program(pr, B, s);
    };
    for (int ni : region) elided_nodes_.insert(ni);
    for (int ni : dfl_chain) elided_nodes_.insert(ni);
    elided_nodes_.erase(po->second);
    st.nodes.assign(region.begin(), region.end());
    st.nodes.insert(st.nodes.end(), dfl_chain.begin(), dfl_chain.end());
    if (std::find(st.nodes.begin(), st.nodes.end(), po->second) == st.nodes.end()) st.nodes.push_back(po->second);
    tail_steps_[po->second] = std::move(st);
  }
}

void Engine::lower() {
  Plan &p = *plan_;
  const auto &nodes = p.nodes();
  const bool no_tc = (flags_ & kFlagNoTensorCores) != 0;
  int *status = status_;
  const int sms = num_sms_;

  auto act_bytes = [&](int t) -> double { return T_[(size_t)t].is_init ? 0.0 : (double)T_[(size_t)t].numel * 2.0; };
  auto init_bytes = [&](int t) -> double { return T_[(size_t)t].is_init ? (double)T_[(size_t)t].numel * 2.0 : 0.0; };
  auto opt = [&](const PlanNode &n, size_t i) -> int {
    return (i < n.ins.size() && n.ins[i] != "-") ? tid(n.ins[i]) : -1;
  };
  auto tc_ok = [&](int t) -> bool {  // activation usable as a K-major TMA source
    const TensorRt &x = T_[(size_t)t];
    if (x.is_init) return false;
    const View4 v = view(t);
    if (v.H * v.W == 1) return v.C == 1 || (v.sc == 1 && v.sb % 8 == 0 && (x.elem_off * 2) % 16 == 0);
    if (v.sc != 1) return false;
    if (v.sx % 8 != 0 || v.sy % 8 != 0 || v.sb % 8 != 0) return false;
    return (x.elem_off * 2) % 16 == 0;
  };

  // storage root -> reading nodes (views excluded), for the fused-chain match
  std::map<int, std::vector<int>> readers;
  for (size_t ni = 0; ni < nodes.size(); ++ni) {
    if (nodes[ni].op == "reshape" || nodes[ni].op == "flatten") continue;
    for (const auto &in : nodes[ni].ins)
      if (in != "-") readers[T_[(size_t)tid(in)].root].push_back((int)ni);
  }
  auto sole_reader = [&](int t) -> int {
    const TensorRt &x = T_[(size_t)t];
    if (x.is_output || x.root != t) return -1;
    const auto it = readers.find(t);
    return (it != readers.end() && it->second.size() == 1) ? it->second[0] : -1;
  };

  for (size_t ni = 0; ni < nodes.size(); ++ni) {
    const PlanNode &n = nodes[ni];
    const std::string &op = n.op;
    if (op == "reshape" || op == "flatten") continue;
    if (elided_nodes_.count((int)ni)) continue;  // folded into an earlier step
    if (tail_steps_.count((int)ni)) {             // fused planar tail ending here
      steps_.push_back(tail_steps_[(int)ni]);
      continue;
    }
    const int out = tid(n.outs[0]);
    Step st;
    st.node = (int)ni;
    st.nodes = {(int)ni};
    st.name = op + ":" + n.outs[0];
    st.family = op;

    // ---------------------------------------------------------------- convolutions
    const bool is_conv = op == "conv3x3" || op == "conv1x1" || op == "conv1x1_cat4";
    if (is_conv) {
      ConvCfg c;
      int w = -1, bias = -1;
      if (op == "conv3x3") {
        c.ksize = 3;
        c.stride = n.ai("stride", 1);
        c.pad = n.ai("pad", 1);
        c.src[0] = tid(n.ins[0]);
        w = tid(n.ins[1]);
        bias = opt(n, 2);
        c.res = opt(n, 3);
        c.act_kind = kActConv3x3;
      } else if (op == "conv1x1") {
        w = tid(n.ins[0]);
        c.src[0] = tid(n.ins[1]);
        bias = opt(n, 2);
        c.res = opt(n, 3);
        if (opt(n, 4) >= 0) throw std::runtime_error("CudaPlanModel: conv1x1 scale input is not supported");
      } else {
        w = tid(n.ins[0]);
        c.nsrc = 0;
        const int cnt[4] = {n.ai("cat_ca", 0), n.ai("cat_cb", 0), n.ai("cat_cc", 0), n.ai("cat_cd", 0)};
        for (int s = 0; s < 4; ++s)
          if (cnt[s] > 0) c.src[c.nsrc++] = tid(n.ins[(size_t)(1 + s)]);
        bias = opt(n, 5);
        c.res = opt(n, 6);
      }
      c.act = n.ai("act", 0);
      c.out = out;
      const TensorRt &wt = T_[(size_t)w];
      const TensorRt &ot = T_[(size_t)out];
      c.cout = (int)wt.dims[0];
      for (int s = 0; s < c.nsrc; ++s) {
        c.srcC[s] = view(c.src[s]).C;
        c.cin_total += c.srcC[s];
      }
      if (c.nsrc == 1 && c.ksize == 1) c.cin_total = (int)wt.dims[1];
      const View4 ov = view(out);
      c.Ho = ov.H;
      c.Wo = ov.W;
      if (c.ksize == 3) {
        c.Ho = n.ai("Hout", ov.H);
        c.Wo = n.ai("Wout", ov.W);
      }
      c.taps = c.ksize * c.ksize;
      // FLOPs / bytes (algorithmic, per image) for the roofline
      // (merged sibling convolutions: the members' channels, not the padding)
      st.flops_img = 2.0 * n.ai("alg_cout", c.cout) * c.cin_total * c.taps * (double)c.Ho * c.Wo;
      for (int s = 0; s < c.nsrc; ++s) st.bytes_img += act_bytes(c.src[s]);
      st.bytes_img += act_bytes(out) + (c.res >= 0 ? act_bytes(c.res) : 0.0);
      st.bytes_fixed = init_bytes(w) + (bias >= 0 ? init_bytes(bias) : 0.0);
      const View4 xv0 = view(c.src[0]);
      // consistency with the reference's derivation of the GEMM sizes
      if (c.ksize == 1) {
        const int64_t xn = T_[(size_t)c.src[0]].numel;
        if (c.nsrc == 1 && (int64_t)xv0.C * xv0.H * xv0.W != xn)
          throw std::runtime_error("CudaPlanModel: conv1x1 input view mismatch for " + n.outs[0]);
        if (c.nsrc == 1 && xv0.C != c.cin_total)
          throw std::runtime_error("CudaPlanModel: conv1x1 Cin mismatch for " + n.outs[0]);
      }
      bool use_tc = !no_tc;
      for (int s = 0; s < c.nsrc; ++s) use_tc = use_tc && tc_ok(c.src[s]);
      if (c.ksize == 3 && xv0.C <= 4) use_tc = false;  // stem: dedicated kernel
      if (c.ksize == 1 && c.nsrc == 1 && (xv0.H != ov.H || xv0.W != ov.W)) use_tc = false;
      if (!use_tc) {
        if (c.nsrc != 1) throw std::runtime_error("CudaPlanModel: concatenated sources need channels-last input");
        const int x = c.src[0];
        const int res = c.res;
        const int K = c.ksize, S = c.stride, P = c.pad, act = c.act;
        const __half *wptr = T_[(size_t)w].dptr;
        const __half *bptr = bias >= 0 ? T_[(size_t)bias].dptr : nullptr;
        if (c.ksize == 3 && xv0.C <= 4 && res < 0) {
          st.family = "stem3x3";
          const int cout = c.cout;
          auto blob = std::make_shared<std::vector<float>>();
          if (!stem_params(xv0.C, cout, p.ref(T_[(size_t)w].name).host.data(),
                           bias >= 0 ? p.ref(T_[(size_t)bias].name).host.data() : nullptr, blob.get()))
            blob.reset();
          st.launch = [this, x, out, wptr, bptr, blob, cout, S, P, act, status](int B, cudaStream_t s) {
            return launch_stem3x3_v4(view(x), wptr, bptr, blob ? blob->data() : nullptr, view(out), B, cout, S, P,
                                     act, status, s);
          };
        } else if (c.ksize == 1 && res < 0 && T_[(size_t)x].dense && T_[(size_t)out].dense && c.cout <= 8 &&
                   c.cin_total <= 64) {
          st.family = "conv1x1_planar";
          const int cin = c.cin_total, cout = c.cout;
          const long long N = T_[(size_t)x].numel / cin;
          st.launch = [this, x, out, wptr, bptr, cin, cout, N, act](int B, cudaStream_t s) {
            return launch_conv1x1_planar(T_[(size_t)x].dptr, wptr, bptr, T_[(size_t)out].dptr, B, N, cin, cout, act, s);
          };
        } else {
          st.family = "conv_direct";
          const int epi = (c.ksize == 3) ? 2 : 1;
          const int cout = c.cout;
          st.launch = [this, x, out, res, wptr, bptr, cout, K, S, P, act, epi](int B, cudaStream_t s) {
            View4 xv = view(x), ov = view(out);
            if (K == 1 && (xv.H != ov.H || xv.W != ov.W)) {  // 1x1 over [C, N] planar rows
              xv.W = xv.H * xv.W;
              xv.H = 1;
            }
            const View4 rv = res >= 0 ? view(res) : View4{};
            return launch_conv_direct_v4(xv, wptr, bptr, res >= 0 ? view(res).ptr : nullptr, rv, ov, B, cout, K, S,
                                         P, 1, act, epi, s);
          };
        }
        steps_.push_back(std::move(st));
        continue;
      }
      // ---- tensor-core path: tile choice
      c.BK = 64;
      for (int s = 0; s < c.nsrc; ++s) c.BK = std::min(c.BK, pick_bk(c.srcC[s]));
      for (int s = 0; s < c.nsrc; ++s) c.chunks[s] = (int)((c.srcC[s] + c.BK - 1) / c.BK);
      c.num_kb = 0;
      for (int s = 0; s < c.nsrc; ++s) c.num_kb += c.taps * c.chunks[s];
      const int np16 = (int)round_up(c.cout, 16);
      if (np16 <= 256) {
        c.BN = np16;
        c.n_tiles = 1;
      } else {
        c.BN = 128;
        c.n_tiles = (int)((np16 + 127) / 128);
      }
      c.Np = c.BN * c.n_tiles;
      // 3x3 stride 1 / 2 with resident weights: one halo window per channel
      // chunk feeds all nine taps (conv_geom decides whether it fits)
      c.kern_kb = c.num_kb;
      if (c.ksize == 3 && (c.stride == 1 || c.stride == 2) && c.pad == 1 && c.nsrc == 1 && c.n_tiles == 1 &&
          !(flags_ & kFlagNoHalo)) {
        c.halo = c.stride;
        c.kern_kb = c.chunks[0];
        ConvGeom g1;
        if (!conv_geom(c, 1, &g1)) {
          // weights too large to stay resident beside two stages, or to travel
          // with each stage: split N in two or four so that each CTA keeps one
          // N tile's weights resident, else one box per tap
          bool ok = false;
          if (c.n_tiles == 1)
            for (int sp = 2; sp <= 4 && !ok; sp *= 2) {
              ConvCfg t = c;
              t.BN = (int)round_up((np16 + sp - 1) / sp, 16);
              t.n_tiles = sp;
              t.Np = t.BN * sp;
              if (conv_geom(t, 1, &g1)) {
                c = t;
                ok = true;
              }
            }
          if (!ok) {
            c.halo = 0;
            c.kern_kb = c.num_kb;
          }
        }
      }
      {
        ConvGeom g1;
        if (!conv_geom(c, 1, &g1)) throw std::runtime_error("CudaPlanModel: conv tile does not fit shared memory");
      }
      // Layouts the load-time tuning chooses between (the first is the
      // untuned pick).  All of them accumulate every output in the same K
      // order, so the choice changes no bit, and all read the same packed
      // weights (the largest N padding among them):
      // - a halo conv split over N tiles also keeps the one-box-per-tap
      //   layout, faster where halo tiles cover the image poorly; with one
      //   channel chunk only, where the two walks share the K order (halo
      //   tiles go chunk by chunk, boxes per tap tap by tap);
      // - the N tile split in two or four, for launches with few M tiles
      //   (batch 1, the SE blocks' one-pixel convs), where more CTAs each
      //   stream less of the weights.
      std::vector<ConvCfg> modes{c};
      if (c.halo && c.n_tiles > 1 && c.chunks[0] == 1) {
        ConvCfg t = c;
        t.halo = 0;
        t.kern_kb = t.num_kb;
        t.BN = np16;
        t.n_tiles = 1;
        t.Np = np16;
        ConvGeom gt;
        if (conv_geom(t, 1, &gt)) modes.push_back(t);
      }
      // (convs over at most 16 pixels, such as the SE blocks' fully connected
      // layers, also try 8 and 16 N tiles: with one M tile per image batch
      // they have few tiles, and narrower ones spread over more SMs)
      if (c.n_tiles == 1 && np16 >= 64)
        for (int sp = 2; sp <= (c.Ho * c.Wo <= 16 ? 16 : 4); sp *= 2) {
          ConvCfg t = c;
          t.BN = (int)round_up((np16 + sp - 1) / sp, 16);
          t.n_tiles = (np16 + t.BN - 1) / t.BN;
          t.Np = t.BN * t.n_tiles;
          ConvGeom gt;
          if (t.n_tiles > 1 && conv_geom(t, 1, &gt)) modes.push_back(t);
        }
      int np_alloc = 0;
      for (const ConvCfg &m : modes) np_alloc = std::max(np_alloc, m.Np);
      // ---- weight repack: Wp[Np][Kp], K order (source, tap, chunk, channel)
      const int Kp = c.num_kb * c.BK;
      std::vector<uint16_t> wp((size_t)np_alloc * Kp, 0), bp((size_t)np_alloc, 0);
      const PlanTensor &pw = p.ref(wt.name);
      const int wcin = (int)(pw.numel() / (c.cout * c.taps));
      {
        int kb = 0, cbase = 0;
        for (int s = 0; s < c.nsrc; ++s) {
          for (int tap = 0; tap < c.taps; ++tap)
            for (int ch = 0; ch < c.chunks[s]; ++ch, ++kb)
              for (int j = 0; j < c.BK; ++j) {
                const int cl = ch * c.BK + j;
                if (cl >= c.srcC[s]) continue;
                const int ci = cbase + cl;
                if (ci >= wcin) throw std::runtime_error("CudaPlanModel: weight/input channel mismatch: " + wt.name);
                for (int nn = 0; nn < c.cout; ++nn)
                  wp[(size_t)nn * Kp + (size_t)kb * c.BK + j] = pw.host[((size_t)nn * wcin + ci) * c.taps + tap];
              }
          cbase += c.srcC[s];
        }
        if (cbase != wcin) throw std::runtime_error("CudaPlanModel: weight/input channel mismatch: " + wt.name);
      }
      if (bias >= 0) {
        const PlanTensor &pb = p.ref(T_[(size_t)bias].name);
        for (int nn = 0; nn < c.cout && nn < (int)pb.host.size(); ++nn) bp[(size_t)nn] = pb.host[(size_t)nn];
      }
      (void)f32_to_f16_rne_host;
      if (!dry_) {
        void *dw = nullptr, *db = nullptr;
        check(cudaMalloc(&dw, wp.size() * 2), "cudaMalloc(packed weights)");
        check(cudaMalloc(&db, bp.size() * 2), "cudaMalloc(packed bias)");
        dev_allocs_.push_back(dw);
        dev_allocs_.push_back(db);
        check(cudaMemcpy(dw, wp.data(), wp.size() * 2, cudaMemcpyHostToDevice), "upload packed weights");
        check(cudaMemcpy(db, bp.data(), bp.size() * 2, cudaMemcpyHostToDevice), "upload packed bias");
        for (ConvCfg &m : modes) {
          m.wp = static_cast<__half *>(dw);
          m.bias = bias >= 0 ? static_cast<__half *>(db) : nullptr;
        }
        c = modes[0];
      }
      st.family = c.ksize == 3 ? "conv3x3_tc" : "conv1x1_tc";
      // Launch parameters of one batch size and tile geometry.
      auto build = std::make_shared<std::function<ConvTcArgs(int, const ConvCand &)>>(
          [this, modes, status](int B, const ConvCand &cand) -> ConvTcArgs {
        const ConvCfg &c = modes[(size_t)cand.mode];
        const ConvGeom &g = cand.g;
        const int nteams = cand.nteams, nbuf = cand.nbuf;
        ConvTcArgs a;
        std::memset(&a, 0, sizeof(a));
        std::string err;
        const int Kp = c.num_kb * c.BK;
        for (int sidx = 0; sidx < c.nsrc; ++sidx) {
          const View4 v = view(c.src[sidx]);
          bool ok;
          if (c.ksize == 1) {
            const int64_t pix = (v.H * v.W == 1) ? v.sb : v.sx;
            const uint64_t dims[2] = {(uint64_t)v.C, (uint64_t)B * v.H * v.W};
            const uint64_t strides[1] = {(uint64_t)pix * 2};
            const uint32_t box[2] = {(uint32_t)c.BK, 128};
            const uint32_t es[2] = {1, 1};
            ok = encode_tiled_f16(&a.mapA[sidx], 2, v.ptr, dims, strides, box, es,
                                  swizzle_for_row_bytes(c.BK * 2), &err);
          } else {
            const uint64_t dims[4] = {(uint64_t)v.C, (uint64_t)v.W, (uint64_t)v.H, (uint64_t)B};
            const uint64_t strides[3] = {(uint64_t)v.sx * 2, (uint64_t)v.sy * 2, (uint64_t)v.sb * 2};
            const uint32_t box[4] = {(uint32_t)c.BK, (uint32_t)((c.halo ? g.hx : g.TW) * c.stride),
                                     (uint32_t)((c.halo ? g.hy : g.TH) * c.stride), 1};
            const uint32_t es[4] = {1, (uint32_t)c.stride, (uint32_t)c.stride, 1};
            ok = encode_tiled_f16(&a.mapA[sidx], 4, v.ptr, dims, strides, box, es,
                                  swizzle_for_row_bytes(c.BK * 2), &err);
          }
          if (!ok) throw std::runtime_error("CudaPlanModel: tensor map (activation) " + err);
        }
        {
          const uint64_t dims[2] = {(uint64_t)Kp, (uint64_t)c.Np};
          const uint64_t strides[1] = {(uint64_t)Kp * 2};
          const uint32_t box[2] = {(uint32_t)c.BK, (uint32_t)c.BN};
          const uint32_t es[2] = {1, 1};
          if (!encode_tiled_f16(&a.mapB, 2, c.wp, dims, strides, box, es, swizzle_for_row_bytes(c.BK * 2), &err))
            throw std::runtime_error("CudaPlanModel: tensor map (weights) " + err);
        }
        a.ksize = c.ksize;
        a.stride = c.stride;
        a.pad = c.pad;
        a.nsrc = c.nsrc;
        for (int sidx = 0; sidx < c.nsrc; ++sidx) a.src_chunks[sidx] = c.chunks[sidx];
        a.taps = c.taps;
        a.BK = c.BK;
        a.BN = c.BN;
        a.n_tiles = c.n_tiles;
        a.num_kb = c.kern_kb;
        a.halo = c.halo;
        a.mb = g.mb;
        a.hx = g.hx;
        a.hy = g.hy;
        a.halo_bytes = g.halo_bytes;
        a.stages = g.stages;
        a.kb_per_stage = g.kb_per_stage;
        a.resident_b = g.resident_b;
        a.Ho = c.Ho;
        a.Wo = c.Wo;
        a.m_total = (long long)B * c.Ho * c.Wo;
        const long long m_tiles = conv_m_tiles(c, g, B);
        if (m_tiles * c.n_tiles > INT32_MAX) throw std::runtime_error("CudaPlanModel: conv output too large");
        a.m_tiles = (int)m_tiles;
        if (c.ksize == 1) {
          a.tile_rows = 128;
          a.TH = a.TW = 1;
          a.tiles_x = a.tiles_per_img = 1;
        } else {
          a.TH = g.TH;
          a.TW = g.TW;
          a.tiles_x = (c.Wo + g.TW - 1) / g.TW;
          const int tiles_y = (c.Ho + g.TH - 1) / g.TH;
          a.tiles_per_img = a.tiles_x * tiles_y;
          a.tile_rows = c.halo ? 128 : g.TH * g.TW;  // rows of one M block that hold pixels
        }
        a.bias = c.bias;
        a.cout = c.cout;
        a.act = c.act;
        a.act_kind = c.act_kind;
        a.act_fn = resolve_act(c.act, c.act_kind);
        const View4 ov = view(c.out);
        a.out = ov.ptr;
        a.o_sb = ov.sb;
        a.o_sc = ov.sc;
        a.o_sy = ov.sy;
        a.o_sx = ov.sx;
        if (c.ksize == 1 && (ov.H != c.Ho || ov.W != c.Wo)) throw std::runtime_error("conv1x1 output view mismatch");
        a.out_vec = (ov.sc == 1 && ov.sx % 8 == 0 && ov.sy % 8 == 0 && ov.sb % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(ov.ptr) & 15) == 0)
                        ? 1
                        : 0;
        a.out_dense = (c.ksize == 1 && ov.sc == 1 && ov.sy == (long long)ov.W * ov.sx &&
                       ov.sb == (long long)ov.H * ov.sy)
                          ? 1
                          : 0;
        a.epi_fast = (a.out_vec && c.res < 0 && c.BN * c.n_tiles == c.cout) ? 1 : 0;
        if (c.res >= 0) {
          const View4 rv = view(c.res);
          a.res = rv.ptr;
          a.r_sb = rv.sb;
          a.r_sc = rv.sc;
          a.r_sy = rv.sy;
          a.r_sx = rv.sx;
          a.res_vec = (rv.sc == 1 && rv.sx % 8 == 0 && rv.sy % 8 == 0 && rv.sb % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(rv.ptr) & 15) == 0)
                          ? 1
                          : 0;
        }
        a.nteams = nteams;
        a.nbuf = nbuf;
        a.tmem_cols = pow2_at_least(nbuf * g.mb * c.BN);
        a.smem_bytes = g.smem;
        a.status = status;
        a.wait_limit = kConvWaitLimitDefault;
        a.wait_probe = 0;
        const char *why = nullptr;
        if (!conv_tc_finalize(a, &why)) throw std::runtime_error(std::string("CudaPlanModel: ") + why);
        return a;
      });
      auto cache = std::make_shared<std::map<int, ConvTcArgs>>();
      st.geometry = std::make_shared<std::map<int, std::string>>();
      auto geometry = st.geometry;
      auto record = [c, geometry](int B, const ConvTcArgs &a, const char *how) {
        std::ostringstream gs;
        gs << "mb=" << a.mb << " tile=" << (c.ksize == 1 ? 128 * a.mb : a.TH * a.TW) << " halo=" << a.halo
           << " hx=" << a.hx << " stages=" << a.stages << " kbs=" << a.kb_per_stage << " teams=" << a.nteams
           << " nbuf=" << a.nbuf << " tiles=" << a.m_tiles * a.n_tiles << " smem=" << a.smem_bytes << " " << how;
        (*geometry)[B] = gs.str();
      };
      auto wait = wait_;
      st.launch = [c, cache, build, record, sms, wait](int B, cudaStream_t s) -> cudaError_t {
        auto it = cache->find(B);
        if (it == cache->end()) {  // untuned: the cost model's pick
          const ConvTcArgs a = (*build)(B, conv_candidates(c, B, sms).front());
          record(B, a, "model");
          it = cache->emplace(B, a).first;
        }
        const ConvTcArgs &a = it->second;
        const int grid = conv_grid(a, sms);
        if (wait->probe || wait->limit != kConvWaitLimitDefault) {  // test settings of the bounded waits
          ConvTcArgs b = a;
          b.wait_limit = wait->limit;
          b.wait_probe = wait->probe;
          return launch_conv_tc(b, grid, s);
        }
        return launch_conv_tc(a, grid, s);
      };
      // Load-time tuning: the first run of a batch size times the cost model's
      // best few tile geometries of this conv (each geometry accumulates every
      // output in the same order, so the choice changes no result) and keeps
      // the fastest.
      st.tune = [modes, cache, build, record, sms](int B, cudaStream_t s) {
        // the best few of every layout by the cost model (which compares
        // geometries of one layout only)
        std::vector<ConvCand> cands;
        for (size_t mi = 0; mi < modes.size(); ++mi) {
          std::vector<ConvCand> cm = conv_candidates(modes[mi], B, sms);
          const size_t keep = mi > 0 ? 3 : modes.size() == 1 ? (size_t)kConvTuneCands : (size_t)kConvTuneCands - 4;
          for (size_t k = 0; k < cm.size() && k < keep; ++k) {
            cm[k].mode = (int)mi;
            cands.push_back(cm[k]);
          }
        }
        if (cands.size() < 2) return;
        float best_ms = 0.0f;
        ConvTcArgs best{};
        bool have = false;
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) return;
        for (size_t k = 0; k < cands.size(); ++k) {
          ConvTcArgs a;
          try {
            a = (*build)(B, cands[k]);
          } catch (const std::exception &) {
            continue;
          }
          const int grid = conv_grid(a, sms);
          if (launch_conv_tc(a, grid, s) != cudaSuccess) continue;  // warm-up
          cudaEventRecord(e0, s);
          bool ok = true;
          for (int r = 0; r < 6 && ok; ++r) ok = launch_conv_tc(a, grid, s) == cudaSuccess;
          cudaEventRecord(e1, s);
          if (!ok || cudaEventSynchronize(e1) != cudaSuccess) continue;
          float ms = 0.0f;
          cudaEventElapsedTime(&ms, e0, e1);
          if (!have || ms < best_ms) {
            best_ms = ms;
            best = a;
            have = true;
          }
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        if (have) {
          (*cache)[B] = best;
          record(B, best, "tuned");
        }
      };
      steps_.push_back(std::move(st));
      continue;
    }

    // ---------------------------------------------------------------- depthwise / generic conv
    if (op == "conv_general") {
      const int x = tid(n.ins[0]), w = tid(n.ins[1]), bias = opt(n, 2);
      const int K = n.ai("K", 3), S = n.ai("S", 1), P = n.ai("P", 1), G = n.ai("G", 1), act = n.ai("act", 0);
      const View4 xv = view(x), ov = view(out);
      st.flops_img = 2.0 * ov.C * (xv.C / G) * K * K * (double)ov.H * ov.W;
      st.bytes_img = act_bytes(x) + act_bytes(out);
      st.bytes_fixed = init_bytes(w) + (bias >= 0 ? init_bytes(bias) : 0.0);
      const __half *bptr = bias >= 0 ? T_[(size_t)bias].dptr : nullptr;
      if (G == xv.C && (K == 3 || K == 5) && xv.C == ov.C) {
        st.family = "depthwise";
        // repack [C][1][K][K] -> [K*K][C]
        const PlanTensor &pw = p.ref(T_[(size_t)w].name);
        const int C = xv.C;
        std::vector<uint16_t> r((size_t)K * K * C);
        for (int ch = 0; ch < C; ++ch)
          for (int t = 0; t < K * K; ++t) r[(size_t)t * C + ch] = pw.host[(size_t)ch * K * K + t];
        __half *dw = nullptr;
        if (!dry_) {
          void *d = nullptr;
          check(cudaMalloc(&d, r.size() * 2), "cudaMalloc(depthwise weights)");
          dev_allocs_.push_back(d);
          check(cudaMemcpy(d, r.data(), r.size() * 2, cudaMemcpyHostToDevice), "upload depthwise weights");
          dw = static_cast<__half *>(d);
        }
        st.launch = [this, x, out, dw, bptr, K, S, P, act](int B, cudaStream_t s) {
          return launch_depthwise_v4(view(x), dw, bptr, view(out), B, K, S, P, act, s);
        };
      } else {
        st.family = "conv_direct";
        const __half *wptr = T_[(size_t)w].dptr;
        st.launch = [this, x, out, wptr, bptr, K, S, P, G, act](int B, cudaStream_t s) {
          const View4 ov = view(out);
          return launch_conv_direct_v4(view(x), wptr, bptr, nullptr, View4{}, ov, B, ov.C, K, S, P, G, act, 0, s);
        };
      }
      steps_.push_back(std::move(st));
      continue;
    }

    // ------------------------------------------- DFL head: permute -> softmax -> 1x1
    if (op == "permute_0213" && n.ai("mode", 0) == 0 && !(flags_ & kFlagNoFusion)) {
      const int D1 = n.ai("D1", 1), D2 = n.ai("D2", 1);
      const int64_t I = n.ai("I", 1);
      const int x = tid(n.ins[0]);
      const int sm_node = sole_reader(out);
      const PlanNode *sm = sm_node >= 0 ? &nodes[(size_t)sm_node] : nullptr;
      const bool sm_ok = sm && sm->op == "softmax_axis" && sm->ai("outer", 1) == 1 && sm->ai("axdim", 0) == D2 &&
                         sm->ai("inner", 1) == (int64_t)D1 * I && sm->ins[0] == n.outs[0];
      const int cv_node = sm_ok ? sole_reader(tid(sm->outs[0])) : -1;
      const PlanNode *cv = cv_node >= 0 ? &nodes[(size_t)cv_node] : nullptr;
      bool cv_ok = cv && cv->op == "conv1x1" && cv->ins.size() >= 2 && cv->ins[1] == sm->outs[0] &&
                   (cv->ins.size() < 4 || cv->ins[3] == "-");
      int cout = 0;
      if (cv_ok) {
        const TensorRt &wt = T_[(size_t)tid(cv->ins[0])];
        cout = wt.dims.empty() ? 0 : (int)wt.dims[0];
        cv_ok = wt.is_init && wt.numel == (int64_t)cout * D2 && dfl_fused_supported(D2, cout) && T_[(size_t)x].dense &&
                T_[(size_t)tid(cv->outs[0])].dense && T_[(size_t)tid(cv->outs[0])].numel == (int64_t)cout * D1 * I;
      }
      if (cv_ok) {
        const int y = tid(cv->outs[0]);
        const __half *wptr = T_[(size_t)tid(cv->ins[0])].dptr;
        const int bt = (cv->ins.size() > 2 && cv->ins[2] != "-") ? tid(cv->ins[2]) : -1;
        const __half *bptr = bt >= 0 ? T_[(size_t)bt].dptr : nullptr;
        const int act = cv->ai("act", 0);
        st.name = "dfl:" + cv->outs[0];
        st.family = "dfl_fused";
        st.flops_img = 2.0 * cout * D2 * D1 * (double)I;
        st.bytes_img = act_bytes(x) + act_bytes(y);
        st.bytes_fixed = init_bytes(tid(cv->ins[0])) + (bt >= 0 ? init_bytes(bt) : 0.0);
        st.launch = [this, x, y, wptr, bptr, D1, D2, I, cout, act](int B, cudaStream_t s) {
          return launch_dfl_fused(T_[(size_t)x].dptr, wptr, bptr, T_[(size_t)y].dptr, B, D1, D2, I, cout, act, s);
        };
        elided_nodes_.insert(sm_node);
        elided_nodes_.insert(cv_node);
        st.nodes.push_back(sm_node);
        st.nodes.push_back(cv_node);
        steps_.push_back(std::move(st));
        continue;
      }
    }

    // ------------------------- transposing permute that only feeds a bmm operand
    // permute_0213 mode 1 swaps the last two axes of [B1][D2][I]; when its one
    // reader is a bmm taking it as A ([B1][M=I][K=D2]) or B ([B1][K=I][N=D2]),
    // the bmm reads the source transposed instead (the values are the same)
    if (op == "permute_0213" && n.ai("mode", 0) == 1 && !(flags_ & kFlagNoFusion)) {
      const int x = tid(n.ins[0]);
      const int bj = sole_reader(out);
      const PlanNode *bm = bj >= 0 ? &nodes[(size_t)bj] : nullptr;
      const auto &od = T_[(size_t)out].dims;
      bool fold = bm && bm->op == "bmm" && T_[(size_t)x].dense && T_[(size_t)x].root == x && !T_[(size_t)x].is_init &&
                  T_[(size_t)x].numel == T_[(size_t)out].numel && od.size() == 4 && od[1] == n.ai("D1", 1) &&
                  od[2] == n.ai("I", 1) && od[3] == n.ai("D2", 1);
      if (fold) {
        const bool as_a = bm->ins[0] == n.outs[0], as_b = bm->ins.size() > 1 && bm->ins[1] == n.outs[0];
        fold = as_a != as_b;
      }
      if (fold) {
        folded_transpose_[out] = {x, (int)ni};
        continue;
      }
    }

    // ---------------------------------------------------------------- small ops
    for (const auto &in : n.ins)
      if (in != "-") st.bytes_img += act_bytes(tid(in)), st.bytes_fixed += init_bytes(tid(in));
    st.bytes_img += act_bytes(out);
    const TensorRt &ot = T_[(size_t)out];
    if (op == "ew_binary") {
      const int a = tid(n.ins[0]), b = tid(n.ins[1]), opc = n.ai("op", 0);
      const bool same = elementwise_same(n);
      const int bsc = n.ai("b_scalar", 0);
      const bool all_dense = ot.dense && T_[(size_t)a].dense && T_[(size_t)b].dense;
      if (same && all_dense) {
        const int64_t per = ot.numel;
        st.launch = [this, a, b, out, per, opc, bsc](int B, cudaStream_t s) {
          const TensorRt &ta = T_[(size_t)a], &tb = T_[(size_t)b];
          return launch_ew_binary_flat(ta.dptr, tb.dptr, T_[(size_t)out].dptr, per * B, opc, bsc, per, B,
                                       ta.is_init ? 0 : ta.numel, tb.is_init ? 0 : tb.numel, s);
        };
      } else if (same || per_channel_bcast(p, n, nullptr)) {
        int scale_slot = -1;
        const bool pc = !same && per_channel_bcast(p, n, &scale_slot);
        st.launch = [this, a, b, out, opc, bsc, pc, scale_slot](int B, cudaStream_t s) {
          const View4 ov = view(out);
          auto operand = [&](int t, bool bcast) {
            View4 v = view(t);
            if (bcast) {  // [1,C,1,1] (or scalar) broadcast over H, W
              const TensorRt &tt = T_[(size_t)t];
              v.C = ov.C;
              v.H = ov.H;
              v.W = ov.W;
              v.sc = tt.numel == 1 ? 0 : 1;
              v.sy = v.sx = 0;
              v.sb = tt.is_init ? 0 : tt.numel;
            }
            return v;
          };
          const View4 av = operand(a, pc && scale_slot == 0);
          const View4 bv = operand(b, (pc && scale_slot == 1) || bsc == 1);
          return launch_ew_binary_v4(av, bv, ov, B, opc, s);
        };
      } else {
        // rank-generic broadcast on planar operands; dim 0 is the batch
        const std::vector<int64_t> bd = parse_ints(n.attr.at("bdims"));
        const int rank = (int)bd.size() / 3;
        if (rank < 1 || rank > kMaxRank) throw std::runtime_error("CudaPlanModel: bad bdims for " + n.outs[0]);
        st.launch = [this, a, b, out, opc, bd, rank](int B, cudaStream_t s) {
          BcastArgs g{};
          g.rank = rank;
          for (int r = 0; r < rank; ++r) {
            g.dims[r] = bd[(size_t)r];
            g.as[r] = bd[(size_t)(rank + r)];
            g.bs[r] = bd[(size_t)(2 * rank + r)];
          }
          const TensorRt &ta = T_[(size_t)a], &tb = T_[(size_t)b];
          g.dims[0] = B;
          g.as[0] = (ta.is_init || ta.dims.size() != (size_t)rank) ? 0 : ta.numel;
          g.bs[0] = (tb.is_init || tb.dims.size() != (size_t)rank) ? 0 : tb.numel;
          return launch_ew_binary_bcast(ta.dptr, tb.dptr, T_[(size_t)out].dptr, g, opc, s);
        };
      }
    } else if (op == "ew_unary") {
      const int x = tid(n.ins[0]), opc = n.ai("op", 0);
      if (ot.dense && T_[(size_t)x].dense) {
        st.launch = [this, x, out, opc](int B, cudaStream_t s) {
          return launch_ew_unary_flat(T_[(size_t)x].dptr, T_[(size_t)out].dptr, T_[(size_t)out].numel * B, opc, s);
        };
      } else {
        st.launch = [this, x, out, opc](int B, cudaStream_t s) {
          return launch_ew_unary_v4(view(x), view(out), B, opc, s);
        };
      }
    } else if (op == "copy_c") {
      if (ot.root != out) continue;  // zero-copy channel view
      const int x = tid(n.ins[0]);
      const int c0 = n.ai("c0", 0), cnt = n.ai("cnt", 0), HW = n.ai("HW", 1);
      if (n.ai("dst_off", 0) != 0) throw std::runtime_error("CudaPlanModel: copy_c with dst_off is not supported");
      st.launch = [this, x, out, c0, cnt, HW](int B, cudaStream_t s) {
        View4 xv = view(x);
        const View4 ov = view(out);
        if (T_[(size_t)x].dims.size() != 4) {  // generic [1, C, HW...] planar source
          xv.C = (int)(T_[(size_t)x].numel / HW);
          xv.H = 1;
          xv.W = HW;
          xv.sc = HW;
          xv.sy = HW;
          xv.sx = 1;
        }
        xv.ptr += (int64_t)c0 * xv.sc;
        xv.C = cnt;
        View4 o2 = ov;
        if (T_[(size_t)out].dims.size() != 4) {
          o2.C = cnt;
          o2.H = 1;
          o2.W = HW;
          o2.sc = HW;
          o2.sy = HW;
          o2.sx = 1;
        }
        xv.H = o2.H;
        xv.W = o2.W;
        return launch_copy_v4(xv, o2, B, s);
      };
    } else if (op == "slice_axis") {
      const int x = tid(n.ins[0]);
      const int64_t outer = n.ai("outer", 1), inner = n.ai("inner", 1);
      const int axdim = n.ai("axdim", 0), start = n.ai("start", 0), len = n.ai("len", 0);
      st.launch = [this, x, out, outer, inner, axdim, start, len](int B, cudaStream_t s) {
        return launch_slice_axis(T_[(size_t)x].dptr, T_[(size_t)out].dptr, outer * B, axdim, inner, start, len, s);
      };
    } else if (op == "concat4") {
      const int cnt[4] = {n.ai("ca", 0), n.ai("cb", 0), n.ai("cc", 0), n.ai("cd", 0)};
      const int64_t outer = n.ai("outer", 1), inner = n.ai("inner", 1);
      int srcs[4] = {-1, -1, -1, -1};
      for (int s = 0; s < 4; ++s)
        if (cnt[s] > 0) srcs[s] = tid(n.ins[(size_t)s]);
      if (ot.nhwc) {
        st.launch = [this, srcs, cnt, out](int B, cudaStream_t s) {
          int c0 = 0;
          for (int k = 0; k < 4; ++k) {
            if (cnt[k] <= 0) continue;
            View4 ov = view(out);
            ov.ptr += (int64_t)c0 * ov.sc;
            ov.C = cnt[k];
            const cudaError_t e = launch_copy_v4(view(srcs[k]), ov, B, s);
            if (e != cudaSuccess) return e;
            c0 += cnt[k];
          }
          return cudaSuccess;
        };
      } else {
        for (int s = 0; s < 4; ++s)
          if (srcs[s] >= 0 && !T_[(size_t)srcs[s]].dense && !T_[(size_t)srcs[s]].is_init)
            throw std::runtime_error("CudaPlanModel: planar concat of a channels-last source: " + n.outs[0]);
        st.launch = [this, srcs, cnt, out, outer, inner](int B, cudaStream_t s) {
          ConcatSrc cs[4];
          for (int k = 0; k < 4; ++k) {
            cs[k].ptr = srcs[k] >= 0 ? T_[(size_t)srcs[k]].dptr : nullptr;
            cs[k].c = cnt[k];
            cs[k].shared = (srcs[k] >= 0 && T_[(size_t)srcs[k]].is_init) ? 1 : 0;
          }
          return launch_concat_planar(cs, 4, T_[(size_t)out].dptr, outer * B, outer, inner, s);
        };
      }
    } else if (op == "maxpool") {
      const int x = tid(n.ins[0]);
      const int K = n.ai("K", 5), S = n.ai("S", 1), P = n.ai("P", 2);
      // SPPF: the next plan nodes pool this pool's output again (same size,
      // stride 1): up to three levels run as one step
      std::vector<int> chain{out};
      if (S == 1 && !(flags_ & kFlagNoFusion)) {
        for (size_t nj = ni + 1; nj < nodes.size() && chain.size() < 3; ++nj) {
          const PlanNode &m = nodes[nj];
          if (m.op != "maxpool" || m.ai("K", 5) != K || m.ai("S", 1) != 1 || m.ai("P", 2) != P ||
              tid(m.ins[0]) != chain.back())
            break;
          chain.push_back(tid(m.outs[0]));
          elided_nodes_.insert((int)nj);
        }
      }
      // the fused kernel reads x from global memory while it writes the later
      // levels, so x must stay live (unaliased) until the last pooled node
      if (chain.size() > 1 && T_[(size_t)T_[(size_t)x].root].death < (int)(ni + chain.size() - 1)) {
        for (size_t l = 1; l < chain.size(); ++l) elided_nodes_.erase((int)(ni + l));
        chain.resize(1);
      }
      if (chain.size() > 1) {
        st.family = "maxpool_chain";
        for (size_t l = 1; l < chain.size(); ++l) st.nodes.push_back((int)(ni + l));
        for (size_t l = 1; l < chain.size(); ++l) st.bytes_img += act_bytes(chain[l]);
        st.launch = [this, x, chain, K, P](int B, cudaStream_t s) {
          View4 ys[3];
          for (size_t l = 0; l < chain.size(); ++l) ys[l] = view(chain[l]);
          return launch_maxpool_chain_v4(view(x), ys, (int)chain.size(), B, K, P, s);
        };
      } else {
        st.launch = [this, x, out, K, S, P](int B, cudaStream_t s) {
          return launch_maxpool_v4(view(x), view(out), B, K, S, P, s);
        };
      }
    } else if (op == "resize_nn") {
      const int x = tid(n.ins[0]);
      const int S = n.ai("S", 2);
      st.launch = [this, x, out, S](int B, cudaStream_t s) { return launch_resize_nn_v4(view(x), view(out), B, S, s); };
    } else if (op == "softmax_axis") {
      const int x = tid(n.ins[0]);
      const int64_t outer = n.ai("outer", 1), inner = n.ai("inner", 1);
      const int axdim = n.ai("axdim", 0);
      st.launch = [this, x, out, outer, inner, axdim](int B, cudaStream_t s) {
        return launch_softmax_axis(T_[(size_t)x].dptr, T_[(size_t)out].dptr, outer * B, axdim, inner, s);
      };
    } else if (op == "permute_0213") {
      const int x = tid(n.ins[0]);
      const int D1 = n.ai("D1", 1), D2 = n.ai("D2", 1), mode = n.ai("mode", 0);
      const int64_t I = n.ai("I", 1);
      st.launch = [this, x, out, D1, D2, I, mode](int B, cudaStream_t s) {
        return launch_permute_0213(T_[(size_t)x].dptr, T_[(size_t)out].dptr, B, D1, D2, I, mode, s);
      };
    } else if (op == "gap") {
      const int x = tid(n.ins[0]);
      st.launch = [this, x, out](int B, cudaStream_t s) { return launch_gap_v4(view(x), T_[(size_t)out].dptr, B, s); };
    } else if (op == "bmm") {
      int a = tid(n.ins[0]), b = tid(n.ins[1]);
      const auto &ad = T_[(size_t)a].dims, &bd = T_[(size_t)b].dims;
      if (ad.size() != 4 || bd.size() != 4) throw std::runtime_error("CudaPlanModel: bmm expects 4-D operands");
      const int B1 = (int)ad[1], M = (int)ad[2], K = (int)ad[3], Nn = (int)bd[3];
      st.flops_img = 2.0 * B1 * M * K * Nn;
      // operands produced by a folded transposing permute: read its source
      int ta_flag = 0, tb_flag = 0;
      auto fa = folded_transpose_.find(a), fb = folded_transpose_.find(b);
      if (fa != folded_transpose_.end()) {
        a = fa->second.first;
        ta_flag = 1;
        st.nodes.insert(st.nodes.begin(), fa->second.second);
      }
      if (fb != folded_transpose_.end()) {
        b = fb->second.first;
        tb_flag = 1;
        st.nodes.insert(st.nodes.begin(), fb->second.second);
      }
      if (ta_flag || tb_flag) {
        st.bytes_img = act_bytes(a) + act_bytes(b) + act_bytes(out);
        st.family = "bmm";
      }
      st.launch = [this, a, b, out, B1, M, K, Nn, ta_flag, tb_flag](int B, cudaStream_t s) {
        const TensorRt &ta = T_[(size_t)a], &tb = T_[(size_t)b];
        if (ta_flag || tb_flag)
          return launch_bmm_t(ta.dptr, tb.dptr, T_[(size_t)out].dptr, B, B1, M, K, Nn, ta.is_init ? 0 : ta.numel,
                              tb.is_init ? 0 : tb.numel, ta_flag, tb_flag, s);
        return launch_bmm(ta.dptr, tb.dptr, T_[(size_t)out].dptr, B, B1, M, K, Nn, ta.is_init ? 0 : ta.numel,
                          tb.is_init ? 0 : tb.numel, s);
      };
    } else if (op == "bias_add") {
      const int x = tid(n.ins[0]), b = tid(n.ins[1]);
      const int HW = n.ai("HW", 1);
      st.launch = [this, x, b, out, HW](int B, cudaStream_t s) {
        return launch_bias_add(T_[(size_t)x].dptr, T_[(size_t)b].dptr, T_[(size_t)out].dptr, T_[(size_t)out].numel,
                               HW, B, s);
      };
    } else {
      throw std::runtime_error("PlanModel: unknown op: " + op);
    }
    // small ops read/write their operands densely unless they are views
    for (const auto &in : n.ins) {
      if (in == "-") continue;
      const TensorRt &t = T_[(size_t)tid(in)];
      if (!t.dense && !t.nhwc && !t.is_init)
        throw std::runtime_error("CudaPlanModel: internal layout error at " + n.outs[0]);
    }
    steps_.push_back(std::move(st));
  }
  stats_.steps = (int)steps_.size();
}

// ============================================================================ execution
void Engine::set_stream(cudaStream_t s) {
  if (own_stream_ && stream_ && s != stream_) {
    cudaStreamSynchronize(stream_);
    cudaStreamDestroy(stream_);
    own_stream_ = false;
  }
  stream_ = s;
  for (auto &kv : graphs_) cudaGraphExecDestroy(kv.second);
  graphs_.clear();
}

void Engine::upload_input_f16(const void *src, int batch, bool on_device) {
  require_device();
  if (batch < 1 || batch > max_batch_) throw std::runtime_error("CudaPlanModel: batch out of range");
  check(cudaSetDevice(device_), "cudaSetDevice");
  check(cudaMemcpyAsync(input_device_ptr(), src, (size_t)input_numel() * batch * 2,
                        on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream_),
        "input copy");
}

void Engine::upload_input_f32(const float *src, int batch, bool on_device) {
  require_device();
  pdl_scope();
  if (batch < 1 || batch > max_batch_) throw std::runtime_error("CudaPlanModel: batch out of range");
  check(cudaSetDevice(device_), "cudaSetDevice");
  const int64_t n = input_numel() * batch;
  const float *d = src;
  if (!on_device) {
    check(cudaMemcpyAsync(in_f32_, src, (size_t)n * 4, cudaMemcpyHostToDevice, stream_), "input copy");
    d = in_f32_;
  }
  check(launch_f32_to_f16_trunc(d, input_device_ptr(), n, stream_), "input conversion");
}

// Step dependencies come from the plan nodes each step carries out: two steps
// touching one storage root, at least one of them writing it, keep their
// order.  Steps go to streams greedily: a step continues the stream of its
// latest predecessor when that stream still ends with it, else takes a stream
// whose last step is already ordered before it, else the least recently used
// stream.  A step waits (graph edge) for the latest step it depends on in
// each other stream.  reach_ is the closure of dependencies and stream order:
// the allocator lets two roots share bytes only along it.
void Engine::plan_streams() {
  const auto &nodes = plan_->nodes();
  const int S = (int)steps_.size();
  step_reads_.assign((size_t)S, {});
  step_writes_.assign((size_t)S, {});
  auto root_of = [&](const std::string &name) -> int {
    if (name == "-") return -1;
    const TensorRt &t = T_[(size_t)tid(name)];
    return t.is_init ? -1 : t.root;
  };
  std::vector<std::set<int>> rds((size_t)S), wrs((size_t)S);
  std::map<int, int> writers;  // root -> steps writing it
  for (int j = 0; j < S; ++j) {
    for (int ni : steps_[(size_t)j].nodes) {
      const PlanNode &n = nodes[(size_t)ni];
      for (const auto &in : n.ins)
        if (root_of(in) >= 0) rds[(size_t)j].insert(root_of(in));
      for (const auto &o : n.outs)
        if (root_of(o) >= 0) wrs[(size_t)j].insert(root_of(o));
    }
    for (int r : wrs[(size_t)j]) ++writers[r];
  }
  for (int j = 0; j < S; ++j) {
    const Step &stp = steps_[(size_t)j];
    if (stp.family == "decode_tail" || stp.family == "dfl_fused" || (stp.family == "bmm" && stp.nodes.size() > 1)) {
      // computed in registers: the values the fused nodes pass to each other
      // (written by this step alone, other than its last node's output) never
      // reach memory and are no accesses; tensors other steps write (the
      // in-place concats the region reads) stay reads
      const int last_node = *std::max_element(stp.nodes.begin(), stp.nodes.end());
      std::set<int> out;
      for (const auto &o : nodes[(size_t)last_node].outs)
        if (root_of(o) >= 0) out.insert(root_of(o));
      for (int r : wrs[(size_t)j]) {
        if (out.count(r)) continue;  // the step's own output
        if (writers[r] > 1)
          rds[(size_t)j].insert(r);  // another step writes it: a read here
        else
          rds[(size_t)j].erase(r);   // a value inside the fused region
      }
      wrs[(size_t)j] = out;
    }
    step_reads_[(size_t)j].assign(rds[(size_t)j].begin(), rds[(size_t)j].end());
    step_writes_[(size_t)j].assign(wrs[(size_t)j].begin(), wrs[(size_t)j].end());
  }
  auto meets = [](const std::vector<int> &a, const std::vector<int> &b) {
    size_t i = 0, k = 0;
    while (i < a.size() && k < b.size()) {
      if (a[i] == b[k]) return true;
      if (a[i] < b[k]) ++i;
      else ++k;
    }
    return false;
  };
  std::vector<std::vector<int>> preds((size_t)S);
  for (int j = 0; j < S; ++j)
    for (int i = 0; i < j; ++i)
      if (meets(step_writes_[(size_t)i], step_reads_[(size_t)j]) ||
          meets(step_writes_[(size_t)i], step_writes_[(size_t)j]) ||
          meets(step_reads_[(size_t)i], step_writes_[(size_t)j]))
        preds[(size_t)j].push_back(i);

  const int K = (flags_ & kFlagSerial) ? 1 : kMaxStreams;
  const size_t words = ((size_t)S + 63) / 64;
  std::vector<std::vector<uint64_t>> anc((size_t)S, std::vector<uint64_t>(words, 0));  // ancestors of j
  auto is_anc = [&](int a, int j) { return (anc[(size_t)j][(size_t)a >> 6] >> (a & 63)) & 1ull; };
  auto add_anc = [&](int j, int a) {
    anc[(size_t)j][(size_t)a >> 6] |= 1ull << (a & 63);
    for (size_t w = 0; w < words; ++w) anc[(size_t)j][w] |= anc[(size_t)a][w];
  };
  stream_of_.assign((size_t)S, 0);
  waits_.assign((size_t)S, {});
  signals_.assign((size_t)S, 0);
  std::vector<int> last((size_t)K, -1), used_at((size_t)K, -1);
  for (int j = 0; j < S; ++j) {
    for (int p : preds[(size_t)j]) add_anc(j, p);
    int st = -1;
    for (auto it = preds[(size_t)j].rbegin(); it != preds[(size_t)j].rend() && st < 0; ++it)
      if (last[(size_t)stream_of_[(size_t)*it]] == *it) st = stream_of_[(size_t)*it];
    if (st < 0)
      for (int t = 0; t < K && st < 0; ++t)
        if (last[(size_t)t] < 0 || is_anc(last[(size_t)t], j)) st = t;
    if (st < 0) {
      st = 0;
      for (int t = 1; t < K; ++t)
        if (used_at[(size_t)t] < used_at[(size_t)st]) st = t;
    }
    stream_of_[(size_t)j] = st;
    if (last[(size_t)st] >= 0) add_anc(j, last[(size_t)st]);  // stream order
    // waits: the latest predecessor in each other stream, unless already implied
    std::vector<int> latest((size_t)K, -1);
    for (int p : preds[(size_t)j])
      if (stream_of_[(size_t)p] != st) latest[(size_t)stream_of_[(size_t)p]] = std::max(latest[(size_t)stream_of_[(size_t)p]], p);
    for (int t = 0; t < K; ++t) {
      const int p = latest[(size_t)t];
      if (p < 0) continue;
      if (last[(size_t)st] >= 0 && (last[(size_t)st] == p || is_anc(p, last[(size_t)st]))) continue;
      waits_[(size_t)j].push_back(p);
      signals_[(size_t)p] = 1;
    }
    last[(size_t)st] = j;
    used_at[(size_t)st] = j;
  }
  n_streams_ = 1;
  for (int j = 0; j < S; ++j) n_streams_ = std::max(n_streams_, stream_of_[(size_t)j] + 1);
  reach_.assign((size_t)S, std::vector<uint64_t>(words, 0));
  for (int j = 0; j < S; ++j)
    for (int a = 0; a < j; ++a)
      if (is_anc(a, j)) reach_[(size_t)a][(size_t)j >> 6] |= 1ull << (j & 63);
}

// One eager pass over the network in plan order; a step with a tuning hook
// times its candidates where it runs (its inputs are the values the plan
// gives it there, and repeating it only rewrites its own output, which no
// live tensor aliases), every other step just runs.  The activation pool
// lets later tensors reuse the input's storage, so the input is saved before
// the pass and put back after it: the caller's run reads what it uploaded.
void Engine::tune(int batch) {
  if (dry_ || (flags_ & kFlagNoTune) || tuned_.count(batch)) return;
  tuned_.insert(batch);
  const size_t in_bytes = (size_t)input_numel() * batch * 2;
  void *saved = nullptr;
  if (cudaMalloc(&saved, in_bytes) != cudaSuccess) {  // no room: the cost model's geometry stays
    cudaGetLastError();
    return;
  }
  check(cudaMemcpyAsync(saved, input_device_ptr(), in_bytes, cudaMemcpyDeviceToDevice, stream_), "input save");
  for (auto &s : steps_) {
    if (s.tune) s.tune(batch, stream_);
    const cudaError_t e = s.launch(batch, stream_);  // (tuned steps: the kept geometry once more)
    if (e != cudaSuccess) {
      cudaStreamSynchronize(stream_);
      cudaFree(saved);
      throw std::runtime_error("CudaPlanModel: launch failed at " + s.name + ": " + cudaGetErrorString(e));
    }
  }
  check(cudaMemcpyAsync(input_device_ptr(), saved, in_bytes, cudaMemcpyDeviceToDevice, stream_), "input restore");
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  cudaFree(saved);
  check(cudaGetLastError(), "tuning");
}

void Engine::capture(int batch) {
  pdl_scope();
  tune(batch);
  if (n_streams_ > 1 && !side_[1]) {  // side streams and the events that order them, once
    for (int t = 1; t < n_streams_; ++t) {
      check(cudaStreamCreateWithFlags(&side_[t], cudaStreamNonBlocking), "cudaStreamCreate");
      check(cudaEventCreateWithFlags(&join_events_[t], cudaEventDisableTiming), "cudaEventCreate");
    }
    check(cudaEventCreateWithFlags(&fork_event_, cudaEventDisableTiming), "cudaEventCreate");
    step_events_.assign(steps_.size(), nullptr);
    for (size_t j = 0; j < steps_.size(); ++j)
      if (signals_[j]) check(cudaEventCreateWithFlags(&step_events_[j], cudaEventDisableTiming), "cudaEventCreate");
  }
  cudaGraph_t g = nullptr;
  check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  cudaError_t le = cudaSuccess;
  std::string where;
  try {
    if (n_streams_ > 1) {  // fork: the side streams start after everything queued before the run
      le = cudaEventRecord(fork_event_, stream_);
      for (int t = 1; t < n_streams_ && le == cudaSuccess; ++t) le = cudaStreamWaitEvent(side_[t], fork_event_, 0);
    }
    for (size_t j = 0; j < steps_.size() && le == cudaSuccess; ++j) {
      cudaStream_t st = stream_of_[j] == 0 ? stream_ : side_[stream_of_[j]];
      for (int p : waits_[j])
        if (le == cudaSuccess) le = cudaStreamWaitEvent(st, step_events_[(size_t)p], 0);
      if (le == cudaSuccess) le = steps_[j].launch(batch, st);
      if (le == cudaSuccess && signals_[j]) le = cudaEventRecord(step_events_[j], st);
      if (le != cudaSuccess) where = steps_[j].name;
    }
    for (int t = 1; t < n_streams_ && le == cudaSuccess; ++t) {  // join
      le = cudaEventRecord(join_events_[t], side_[t]);
      if (le == cudaSuccess) le = cudaStreamWaitEvent(stream_, join_events_[t], 0);
    }
  } catch (...) {
    cudaStreamEndCapture(stream_, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  const cudaError_t ee = cudaStreamEndCapture(stream_, &g);
  if (le != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    throw std::runtime_error("CudaPlanModel: launch failed during capture at " + where + ": " + cudaGetErrorString(le));
  }
  check(ee, "cudaStreamEndCapture");
  cudaGraphExec_t ex = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  check(ie, "cudaGraphInstantiate");
  graphs_[batch] = ex;
}

void Engine::run(int batch) {
  require_device();
  pdl_scope();
  if (batch < 1 || batch > max_batch_) throw std::runtime_error("CudaPlanModel: batch out of range");
  check(cudaSetDevice(device_), "cudaSetDevice");
  last_f32_batch_ = 0;  // the output tensors hold this run's images
  if (flags_ & kFlagNoGraph) {
    tune(batch);
    for (auto &s : steps_) {
      const cudaError_t e = s.launch(batch, stream_);
      if (e != cudaSuccess) throw std::runtime_error("CudaPlanModel: launch failed at " + s.name + ": " + cudaGetErrorString(e));
    }
    return;
  }
  auto it = graphs_.find(batch);
  if (it == graphs_.end()) {
    capture(batch);
    it = graphs_.find(batch);
  }
  check(cudaGraphLaunch(it->second, stream_), "cudaGraphLaunch");
}

void Engine::run_profiled(int batch, std::vector<float> *step_ms) {
  require_device();
  pdl_scope();
  check(cudaSetDevice(device_), "cudaSetDevice");
  tune(batch);
  std::vector<cudaEvent_t> ev(steps_.size() + 1);
  for (auto &e : ev) check(cudaEventCreate(&e), "cudaEventCreate");
  check(cudaEventRecord(ev[0], stream_), "cudaEventRecord");
  for (size_t i = 0; i < steps_.size(); ++i) {
    const cudaError_t e = steps_[i].launch(batch, stream_);
    if (e != cudaSuccess) throw std::runtime_error("CudaPlanModel: launch failed at " + steps_[i].name);
    check(cudaEventRecord(ev[i + 1], stream_), "cudaEventRecord");
  }
  check(cudaEventSynchronize(ev.back()), "cudaEventSynchronize");
  step_ms->assign(steps_.size(), 0.0f);
  for (size_t i = 0; i < steps_.size(); ++i) check(cudaEventElapsedTime(&(*step_ms)[i], ev[i], ev[i + 1]), "elapsed");
  for (auto &e : ev) cudaEventDestroy(e);
}

void Engine::download_output_f16(int i, void *dst, int batch, bool on_device) {
  require_device();
  check(cudaSetDevice(device_), "cudaSetDevice");
  const TensorRt &t = T_[(size_t)tid(output_name(i))];
  if (!t.dense) throw std::runtime_error("CudaPlanModel: output is not planar");
  check(cudaMemcpyAsync(dst, t.dptr, (size_t)t.numel * batch * 2,
                        on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, stream_),
        "output copy");
}

void Engine::download_output_f32(int i, float *dst, int batch, bool on_device) {
  require_device();
  pdl_scope();
  check(cudaSetDevice(device_), "cudaSetDevice");
  const TensorRt &t = T_[(size_t)tid(output_name(i))];
  if (!t.dense) throw std::runtime_error("CudaPlanModel: output is not planar");
  const int64_t n = t.numel * batch;
  if (on_device) {
    check(launch_f16_to_f32(t.dptr, dst, n, stream_), "output conversion");
    return;
  }
  // convert on the device into the f32 staging buffer, then one copy
  if (scratch_elems_ < n) {
    if (scratch_) cudaFree(scratch_);
    check(cudaMalloc(&scratch_, (size_t)n * 4), "cudaMalloc(scratch)");
    scratch_elems_ = n * 2;  // counted in halves
  }
  float *tmp = reinterpret_cast<float *>(scratch_);
  check(launch_f16_to_f32(t.dptr, tmp, n, stream_), "output conversion");
  check(cudaMemcpyAsync(dst, tmp, (size_t)n * 4, cudaMemcpyDeviceToHost, stream_), "output copy");
}

namespace {
// Host memory the copy engines can read directly (page-locked or registered);
// for pageable memory the driver would stage every copy through its own small
// bounce buffers.
bool copy_ready(const void *p) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost;
}
}  // namespace

void Engine::infer_f32_host(const float *src, int batch, float *const *outs) {
  require_device();
  pdl_scope();
  if (batch < 1 || batch > max_batch_) throw std::runtime_error("CudaPlanModel: batch out of range");
  check(cudaSetDevice(device_), "cudaSetDevice");
  bool staged = !copy_ready(src);
  for (int i = 0; i < output_count() && !staged; ++i) staged = !copy_ready(outs[i]);
  if (staged && batch > 2) {  // pageable caller memory (a std::vector, a cv::Mat)
    infer_f32_host_staged(src, batch, outs);
    return;
  }
  // The host->device copy of the input bounds the call.  Large batches cast
  // the f32 input to fp16 on the host (the reference's truncation, on the
  // worker pool) into one of two pinned chunk buffers, so the copy carries
  // half the bytes; chunks of 16 images keep the network runs ahead of the
  // copies, and the last chunks shrink (8, 4) so that what follows the final
  // copy (its run and its results' copy back) is short.
  constexpr int kChunk = 16;
  if (batch < 2 * kChunk || staged) {  // too small to overlap (or one or two pageable images): one pass
    upload_input_f32(src, batch, false);
    run(batch);
    for (int i = 0; i < output_count(); ++i) download_output_f32(i, outs[i], batch, false);
    synchronize();
    return;
  }
  const int n_out = output_count();
  std::vector<int64_t> out_numel(n_out), out_off(n_out + 1, 0);
  for (int i = 0; i < n_out; ++i) {
    out_numel[i] = T_[(size_t)tid(output_name(i))].numel;
    if (!T_[(size_t)tid(output_name(i))].dense) throw std::runtime_error("CudaPlanModel: output is not planar");
    out_off[i + 1] = out_off[i] + out_numel[i] * max_batch_;
  }
  const int64_t in_numel = input_numel();
  if (!out_f32_) {
    check(cudaMalloc(&out_f32_, (size_t)out_off[n_out] * sizeof(float)), "cudaMalloc(output f32 staging)");
    check(cudaStreamCreateWithFlags(&copy_in_, cudaStreamNonBlocking), "cudaStreamCreate");
    check(cudaStreamCreateWithFlags(&copy_out_, cudaStreamNonBlocking), "cudaStreamCreate");
    check(cudaHostAlloc(reinterpret_cast<void **>(&in_f16_host_), (size_t)(2 * kChunk * in_numel) * sizeof(uint16_t),
                        cudaHostAllocDefault),
          "cudaHostAlloc(input fp16 chunks)");
  }
  // Split: images [0, n16) are cast on the host and cross as fp16, images
  // [n16, batch) cross as f32 first (no host work, so the link starts at once)
  // and are cast on the device.  A host cast moves 8 bytes of host memory per
  // element (f32 read, fp16 write with streaming stores, fp16 read by the
  // copy) against 4 for an f32 copy, so on a host whose memory bandwidth the
  // copy engines already share, casting everything on the host is slower
  // than casting nothing; five eighths of the batch (a multiple of 4, so that
  // chunks take sizes 16, 8, 4, 2 or 1, each with its graph captured once)
  // was the fastest split measured alone on one GPU (b=64: 5.9 ms against
  // 6.1 ms for half and 6.8 ms for all).  Where several processes share the
  // host (one per GPU) its memory bandwidth per process shrinks and less host
  // casting pays, so the split is tuned per batch size on the first calls:
  // the first (graph captures) runs at 5/8, the next ten try 0, 2, 4, 5 and 6
  // eighths twice each (wall time of the whole call), then the fastest stays.
  // Every split gives the same bits (host and device casts are the same
  // truncation).
  SplitTune &tune = split_tune_[batch];
  static constexpr int kSplitEighths[5] = {0, 2, 4, 5, 6};
  int eighths = 5;
  const int round = tune.calls - 1;
  if (tune.best >= 0)
    eighths = kSplitEighths[tune.best];
  else if (round >= 0 && round < 10)
    eighths = kSplitEighths[round % 5];
  const int n16 = batch * eighths / 8 / 4 * 4;
  const auto call_t0 = std::chrono::steady_clock::now();
  // the fp16 images [0, n16) travel into the front of the f32 staging (2 bytes
  // per element), the f32 images [n16, batch) into their own place (4 bytes)
  uint16_t *in_f16_dev = reinterpret_cast<uint16_t *>(in_f32_);
  struct Chunk {
    int b0, nb;
    bool host;  // cast on the host
  };
  std::vector<Chunk> chunks;
  for (int b0 = n16; b0 < batch;) {
    const int rem = batch - b0;
    const int nb = rem >= kChunk ? kChunk : rem >= 8 ? 8 : rem >= 4 ? 4 : rem >= 2 ? 2 : 1;
    chunks.push_back({b0, nb, false});
    b0 += nb;
  }
  for (int b0 = 0; b0 < n16;) {  // the last copies shrink (8, 4) so that what follows them is short
    const int rem = n16 - b0;
    const int nb = rem >= 2 * kChunk ? kChunk : rem >= kChunk ? kChunk / 2 : 4;
    chunks.push_back({b0, nb, true});
    b0 += nb;
  }
  const int n_chunks = (int)chunks.size();
  while ((int)chunk_events_.size() < 3 * n_chunks + 1) {  // per chunk: copied in, computed; one spare
    cudaEvent_t e;
    check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    chunk_events_.push_back(e);
  }
  // the copy streams start after whatever the compute stream already holds
  check(cudaEventRecord(chunk_events_[3 * n_chunks], stream_), "cudaEventRecord");
  check(cudaStreamWaitEvent(copy_in_, chunk_events_[3 * n_chunks], 0), "cudaStreamWaitEvent");
  // compute and results of one chunk, once its input has arrived
  auto finish = [&](int c) {
    const Chunk &k = chunks[(size_t)c];
    check(cudaStreamWaitEvent(stream_, chunk_events_[3 * c], 0), "cudaStreamWaitEvent");
    if (k.host)
      check(cudaMemcpyAsync(input_device_ptr(), in_f16_dev + k.b0 * in_numel,
                            (size_t)(k.nb * in_numel) * sizeof(uint16_t), cudaMemcpyDeviceToDevice, stream_),
            "input staging copy");
    else
      check(launch_f32_to_f16_trunc(in_f32_ + k.b0 * in_numel, input_device_ptr(), k.nb * in_numel, stream_),
            "input conversion");
    run(k.nb);  // images 0 .. nb-1 of the arena
    for (int i = 0; i < n_out; ++i)
      check(launch_f16_to_f32(T_[(size_t)tid(output_name(i))].dptr, out_f32_ + out_off[i] + k.b0 * out_numel[i],
                              k.nb * out_numel[i], stream_),
            "output conversion");
    check(cudaEventRecord(chunk_events_[3 * c + 1], stream_), "cudaEventRecord");
    check(cudaStreamWaitEvent(copy_out_, chunk_events_[3 * c + 1], 0), "cudaStreamWaitEvent");
    for (int i = 0; i < n_out; ++i)
      check(cudaMemcpyAsync(outs[i] + k.b0 * out_numel[i], out_f32_ + out_off[i] + k.b0 * out_numel[i],
                            (size_t)(k.nb * out_numel[i]) * sizeof(float), cudaMemcpyDeviceToHost, copy_out_),
            "output copy");
  };
  // f32 chunks: every copy queued at once
  for (int c = 0; c < n_chunks; ++c) {
    const Chunk &k = chunks[(size_t)c];
    if (k.host) continue;
    check(cudaMemcpyAsync(in_f32_ + k.b0 * in_numel, src + k.b0 * in_numel, (size_t)(k.nb * in_numel) * sizeof(float),
                          cudaMemcpyHostToDevice, copy_in_),
          "input copy");
    check(cudaEventRecord(chunk_events_[3 * c], copy_in_), "cudaEventRecord");
  }
  for (int c = 0; c < n_chunks; ++c)
    if (!chunks[(size_t)c].host) finish(c);
  // fp16 chunks: cast on the host into one of two pinned buffers, then copied
  for (int c = 0, j = 0; c < n_chunks; ++c) {
    const Chunk &k = chunks[(size_t)c];
    if (!k.host) continue;
    uint16_t *pinned = in_f16_host_ + (size_t)(j & 1) * kChunk * in_numel;
    // the copy that last read this pinned buffer (two fp16 chunks back) must be done
    if (j >= 2) check(cudaEventSynchronize(chunk_events_[3 * (c - 2)]), "cudaEventSynchronize");
    f32_to_f16_trunc_host(src + k.b0 * in_numel, pinned, (size_t)(k.nb * in_numel));
    check(cudaMemcpyAsync(in_f16_dev + k.b0 * in_numel, pinned, (size_t)(k.nb * in_numel) * sizeof(uint16_t),
                          cudaMemcpyHostToDevice, copy_in_),
          "input copy");
    check(cudaEventRecord(chunk_events_[3 * c], copy_in_), "cudaEventRecord");
    finish(c);
    ++j;
  }
  check(cudaEventRecord(chunk_events_[3 * n_chunks], copy_out_), "cudaEventRecord");
  check(cudaStreamWaitEvent(stream_, chunk_events_[3 * n_chunks], 0), "cudaStreamWaitEvent");
  synchronize();
  last_f32_batch_ = batch;  // the whole batch's outputs are in the f32 staging
  if (tune.best < 0) {
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - call_t0).count();
    if (round >= 0 && round < 10) {
      const int k = round % 5;
      tune.ms[k] = tune.ms[k] > 0.0 ? std::min(tune.ms[k], ms) : ms;
    }
    if (++tune.calls > 10) {
      int b = 3;  // 5/8 unless another split measured faster
      for (int k = 0; k < 5; ++k)
        if (tune.ms[k] > 0.0 && tune.ms[k] < tune.ms[b]) b = k;
      tune.best = b;
    }
  }
}

void Engine::infer_f32_host_staged(const float *src, int batch, float *const *outs) {
  // Every image is cast on the host (the reference's truncation, on the
  // worker pool) straight from the caller's memory into one of two pinned
  // fp16 chunk buffers, so the copy engines read pinned memory at half the
  // bytes; results come back into two pinned f32 chunk buffers and the pool
  // copies them out.  The host casts chunk c while the device runs chunk c-1,
  // and copies chunk c-1 out while the device runs chunk c.
  constexpr int kChunk = 16;
  const int n_out = output_count();
  std::vector<int64_t> out_numel(n_out), out_off(n_out + 1, 0), host_off(n_out + 1, 0);
  for (int i = 0; i < n_out; ++i) {
    const TensorRt &t = T_[(size_t)tid(output_name(i))];
    if (!t.dense) throw std::runtime_error("CudaPlanModel: output is not planar");
    out_numel[i] = t.numel;
    out_off[i + 1] = out_off[i] + out_numel[i] * max_batch_;
    host_off[i + 1] = host_off[i] + out_numel[i] * kChunk;
  }
  const int64_t in_numel = input_numel();
  if (!out_f32_) {
    check(cudaMalloc(&out_f32_, (size_t)out_off[n_out] * sizeof(float)), "cudaMalloc(output f32 staging)");
    check(cudaStreamCreateWithFlags(&copy_in_, cudaStreamNonBlocking), "cudaStreamCreate");
    check(cudaStreamCreateWithFlags(&copy_out_, cudaStreamNonBlocking), "cudaStreamCreate");
    check(cudaHostAlloc(reinterpret_cast<void **>(&in_f16_host_), (size_t)(2 * kChunk * in_numel) * sizeof(uint16_t),
                        cudaHostAllocDefault),
          "cudaHostAlloc(input fp16 chunks)");
  }
  if (!out_host_) {
    check(cudaHostAlloc(reinterpret_cast<void **>(&out_host_), (size_t)(2 * host_off[n_out]) * sizeof(float),
                        cudaHostAllocDefault),
          "cudaHostAlloc(output f32 chunks)");
  }
  std::vector<std::pair<int, int>> chunks;  // (first image, images); sizes 16, 8, 4, 2, 1 (one graph each)
  for (int b0 = 0; b0 < batch;) {
    const int rem = batch - b0;
    const int nb = rem >= kChunk ? kChunk : rem >= 8 ? 8 : rem >= 4 ? 4 : rem >= 2 ? 2 : 1;
    chunks.emplace_back(b0, nb);
    b0 += nb;
  }
  const int n_chunks = (int)chunks.size();
  while ((int)chunk_events_.size() < 3 * n_chunks + 1) {  // per chunk: copied in, computed, copied out
    cudaEvent_t e;
    check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    chunk_events_.push_back(e);
  }
  uint16_t *in_f16_dev = reinterpret_cast<uint16_t *>(in_f32_);
  check(cudaEventRecord(chunk_events_[3 * n_chunks], stream_), "cudaEventRecord");
  check(cudaStreamWaitEvent(copy_in_, chunk_events_[3 * n_chunks], 0), "cudaStreamWaitEvent");
  auto drain = [&](int c) {  // chunk c's results from pinned staging into the caller's buffers
    const int b0 = chunks[(size_t)c].first, nb = chunks[(size_t)c].second;
    const float *staged = out_host_ + (size_t)(c & 1) * host_off[n_out];
    check(cudaEventSynchronize(chunk_events_[3 * c + 2]), "cudaEventSynchronize");
    for (int i = 0; i < n_out; ++i) {
      const float *from = staged + host_off[i];
      float *to = outs[i] + (size_t)b0 * out_numel[i];
      host_parallel_for((size_t)(nb * out_numel[i]), 1 << 16, [&](size_t b, size_t e) {
        std::memcpy(to + b, from + b, (e - b) * sizeof(float));
      });
    }
  };
  for (int c = 0; c < n_chunks; ++c) {
    const int b0 = chunks[(size_t)c].first, nb = chunks[(size_t)c].second;
    uint16_t *pinned = in_f16_host_ + (size_t)(c & 1) * kChunk * in_numel;
    // the copy that last read this pinned buffer (two chunks back) must be done
    if (c >= 2) check(cudaEventSynchronize(chunk_events_[3 * (c - 2)]), "cudaEventSynchronize");
    f32_to_f16_trunc_host(src + (size_t)b0 * in_numel, pinned, (size_t)(nb * in_numel));
    check(cudaMemcpyAsync(in_f16_dev + (size_t)b0 * in_numel, pinned, (size_t)(nb * in_numel) * sizeof(uint16_t),
                          cudaMemcpyHostToDevice, copy_in_),
          "input copy");
    check(cudaEventRecord(chunk_events_[3 * c], copy_in_), "cudaEventRecord");
    check(cudaStreamWaitEvent(stream_, chunk_events_[3 * c], 0), "cudaStreamWaitEvent");
    check(cudaMemcpyAsync(input_device_ptr(), in_f16_dev + (size_t)b0 * in_numel,
                          (size_t)(nb * in_numel) * sizeof(uint16_t), cudaMemcpyDeviceToDevice, stream_),
          "input staging copy");
    run(nb);
    for (int i = 0; i < n_out; ++i)
      check(launch_f16_to_f32(T_[(size_t)tid(output_name(i))].dptr, out_f32_ + out_off[i] + (size_t)b0 * out_numel[i],
                              nb * out_numel[i], stream_),
            "output conversion");
    check(cudaEventRecord(chunk_events_[3 * c + 1], stream_), "cudaEventRecord");
    // the pinned output buffer this chunk uses was drained (chunk c-2) in the
    // previous iteration, before this copy is enqueued
    check(cudaStreamWaitEvent(copy_out_, chunk_events_[3 * c + 1], 0), "cudaStreamWaitEvent");
    float *staged = out_host_ + (size_t)(c & 1) * host_off[n_out];
    for (int i = 0; i < n_out; ++i)
      check(cudaMemcpyAsync(staged + host_off[i], out_f32_ + out_off[i] + (size_t)b0 * out_numel[i],
                            (size_t)(nb * out_numel[i]) * sizeof(float), cudaMemcpyDeviceToHost, copy_out_),
            "output copy");
    check(cudaEventRecord(chunk_events_[3 * c + 2], copy_out_), "cudaEventRecord");
    if (c >= 1) drain(c - 1);
  }
  drain(n_chunks - 1);
  check(cudaEventRecord(chunk_events_[3 * n_chunks], copy_out_), "cudaEventRecord");
  check(cudaStreamWaitEvent(stream_, chunk_events_[3 * n_chunks], 0), "cudaStreamWaitEvent");
  synchronize();
  last_f32_batch_ = batch;  // the whole batch's outputs are in the f32 staging
}

// ---- device preprocessing (src/Preprocess.cpp:13-77 on the device)

namespace {
// OpenCV's INTER_LINEAR source coordinates for one axis (the published
// algorithm of cv::resize for 8-bit images): scale = 1 / (dst / src) in
// double; f = float((d + 0.5) * scale - 0.5), s = floor(f), weight f - s; on
// the x axis a coordinate left of the image or at / past its last column is
// clamped with weight 0, on the y axis only the row index is clamped; weights
// in 11-bit fixed point, rounded to nearest even.  x entries carry byte
// offsets of the two taps (3 bytes per pixel), y entries row indices.
void linear_coords(int src, int dst, bool x_axis, std::vector<int4> &tab) {
  tab.resize((size_t)dst);
  const double scale = 1.0 / ((double)dst / (double)src);
  for (int d = 0; d < dst; ++d) {
    float f = (float)((d + 0.5) * scale - 0.5);
    int s = (int)std::floor(f);
    f -= (float)s;
    if (x_axis) {
      if (s < 0) {
        f = 0.f;
        s = 0;
      }
      if (s >= src - 1) {
        f = 0.f;
        s = src - 1;
      }
    }
    const int w1 = (int)std::nearbyint(f * 2048.0f);
    const int w0 = (int)std::nearbyint((1.0f - f) * 2048.0f);
    const int s0 = std::min(std::max(s, 0), src - 1), s1 = std::min(std::max(s + 1, 0), src - 1);
    tab[(size_t)d] = x_axis ? make_int4(3 * s0, 3 * s1, w0, w1) : make_int4(s0, s1, w0, w1);
  }
}
}  // namespace

void Engine::letterbox_tables(int h, int w, int letterbox) {
  if (lbt_.h == h && lbt_.w == w && lbt_.letterbox == letterbox) return;
  const auto &d = input_dims();
  const int in_h = (int)d[2], in_w = (int)d[3];
  LetterboxTables t;
  t.h = h;
  t.w = w;
  t.letterbox = letterbox;
  if (letterbox) {  // Preprocess.cpp:20-27
    t.scale = std::min((float)in_w / (float)w, (float)in_h / (float)h);
    t.rw = (int)std::round((float)w * t.scale);
    t.rh = (int)std::round((float)h * t.scale);
    t.pad_left = (in_w - t.rw) / 2;
    t.pad_top = (in_h - t.rh) / 2;
  } else {
    t.rw = in_w;
    t.rh = in_h;
  }
  if (t.rw < 1 || t.rh < 1) throw std::runtime_error("Preprocessor: the frame letterboxes to an empty image");
  std::vector<int4> xt, yt;
  linear_coords(w, t.rw, true, xt);
  linear_coords(h, t.rh, false, yt);
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");  // earlier launches may still read the old tables
  if (lbt_.xtab) check(cudaFree(lbt_.xtab), "cudaFree(letterbox tables)");
  if (lbt_.ytab) check(cudaFree(lbt_.ytab), "cudaFree(letterbox tables)");
  lbt_.xtab = lbt_.ytab = nullptr;
  check(cudaMalloc(&t.xtab, xt.size() * sizeof(int4)), "cudaMalloc(letterbox tables)");
  check(cudaMalloc(&t.ytab, yt.size() * sizeof(int4)), "cudaMalloc(letterbox tables)");
  check(cudaMemcpy(t.xtab, xt.data(), xt.size() * sizeof(int4), cudaMemcpyHostToDevice), "letterbox tables copy");
  check(cudaMemcpy(t.ytab, yt.data(), yt.size() * sizeof(int4), cudaMemcpyHostToDevice), "letterbox tables copy");
  lbt_ = t;
}

void Engine::launch_letterbox(const uint8_t *dframes, int64_t img_bytes, int64_t row_stride, int first, int n,
                              const PreprocessCfg &cfg, cudaStream_t st) {
  const auto &d = input_dims();
  LetterboxArgs a{};
  a.src = dframes;
  a.img_stride = img_bytes;
  a.row_stride = row_stride;
  a.xtab = lbt_.xtab;
  a.ytab = lbt_.ytab;
  a.in_h = (int)d[2];
  a.in_w = (int)d[3];
  a.dst = input_device_ptr() + (int64_t)first * input_numel();
  a.dst_img_stride = input_numel();
  a.rw = lbt_.rw;
  a.rh = lbt_.rh;
  a.pad_left = lbt_.pad_left;
  a.pad_top = lbt_.pad_top;
  a.to_rgb = cfg.to_rgb;
  a.normalize = cfg.normalize;
  a.has_mean_std = (cfg.n_mean > 0 || cfg.n_std > 0) ? 1 : 0;
  for (int c = 0; c < 3; ++c) {  // Preprocess.cpp:64-74
    a.mean[c] = c < cfg.n_mean ? cfg.mean[c] : 0.f;
    float sd = c < cfg.n_std ? cfg.std[c] : 1.f;
    a.std[c] = sd == 0.f ? 1.f : sd;
  }
  a.vec_store = (a.in_w % 4 == 0 && (reinterpret_cast<uintptr_t>(a.dst) & 7) == 0) ? 1 : 0;
  check(launch_letterbox_bgr(a, n, st), "letterbox preprocessing");
}

void Engine::upload_input_bgr_u8(const uint8_t *frames, int batch, int h, int w, int64_t row_stride, bool on_device,
                                 const PreprocessCfg &cfg, float *letterbox_out) {
  require_device();
  pdl_scope();
  if (batch < 1 || batch > max_batch_) throw std::runtime_error("CudaPlanModel: batch out of range");
  const auto &d = input_dims();
  if (d.size() != 4 || d[1] != 3) throw std::runtime_error("Preprocessor: the plan's input is not [1, 3, H, W]");
  if (h < 1 || w < 1 || row_stride < 3 * (int64_t)w) throw std::runtime_error("Preprocessor: bad frame geometry");
  check(cudaSetDevice(device_), "cudaSetDevice");
  letterbox_tables(h, w, cfg.letterbox);
  const int64_t img_bytes = row_stride * h;
  const uint8_t *src = frames;
  if (!on_device) {
    const int64_t need = img_bytes * batch;
    if (need > frames_cap_) {
      check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
      if (frames_dev_) check(cudaFree(frames_dev_), "cudaFree(frame staging)");
      frames_dev_ = nullptr;
      check(cudaMalloc(&frames_dev_, (size_t)need), "cudaMalloc(frame staging)");
      frames_cap_ = need;
    }
    check(cudaMemcpyAsync(frames_dev_, frames, (size_t)(img_bytes * batch), cudaMemcpyHostToDevice, stream_),
          "frame copy");
    src = frames_dev_;
  }
  launch_letterbox(src, img_bytes, row_stride, 0, batch, cfg, stream_);
  if (letterbox_out)
    for (int b = 0; b < batch; ++b) {
      letterbox_out[3 * b] = cfg.letterbox ? lbt_.scale : 1.f;
      letterbox_out[3 * b + 1] = (float)lbt_.pad_left;
      letterbox_out[3 * b + 2] = (float)lbt_.pad_top;
    }
}

void Engine::infer_bgr_u8_host(const uint8_t *frames, int batch, int h, int w, int64_t row_stride,
                               const PreprocessCfg &cfg, float *const *outs, float *letterbox_out) {
  require_device();
  pdl_scope();
  if (batch < 1 || batch > max_batch_) throw std::runtime_error("CudaPlanModel: batch out of range");
  check(cudaSetDevice(device_), "cudaSetDevice");
  constexpr int kChunk = 16;
  bool out_pinned = true;
  for (int i = 0; i < output_count(); ++i) out_pinned = out_pinned && copy_ready(outs[i]);
  if (batch < 2 * kChunk) {  // one pass
    upload_input_bgr_u8(frames, batch, h, w, row_stride, false, cfg, letterbox_out);
    run(batch);
    for (int i = 0; i < output_count(); ++i) download_output_f32(i, outs[i], batch, false);
    synchronize();
    return;
  }
  const auto &d = input_dims();
  if (d.size() != 4 || d[1] != 3) throw std::runtime_error("Preprocessor: the plan's input is not [1, 3, H, W]");
  if (h < 1 || w < 1 || row_stride < 3 * (int64_t)w) throw std::runtime_error("Preprocessor: bad frame geometry");
  letterbox_tables(h, w, cfg.letterbox);
  const int n_out = output_count();
  std::vector<int64_t> out_numel(n_out), out_off(n_out + 1, 0), host_off(n_out + 1, 0);
  for (int i = 0; i < n_out; ++i) {
    const TensorRt &t = T_[(size_t)tid(output_name(i))];
    if (!t.dense) throw std::runtime_error("CudaPlanModel: output is not planar");
    out_numel[i] = t.numel;
    out_off[i + 1] = out_off[i] + out_numel[i] * max_batch_;
    host_off[i + 1] = host_off[i] + out_numel[i] * kChunk;
  }
  if (!out_f32_) {
    check(cudaMalloc(&out_f32_, (size_t)out_off[n_out] * sizeof(float)), "cudaMalloc(output f32 staging)");
    check(cudaStreamCreateWithFlags(&copy_in_, cudaStreamNonBlocking), "cudaStreamCreate");
    check(cudaStreamCreateWithFlags(&copy_out_, cudaStreamNonBlocking), "cudaStreamCreate");
    check(cudaHostAlloc(reinterpret_cast<void **>(&in_f16_host_), (size_t)(2 * kChunk * input_numel()) * sizeof(uint16_t),
                        cudaHostAllocDefault),
          "cudaHostAlloc(input fp16 chunks)");
  }
  if (!out_pinned && !out_host_)
    check(cudaHostAlloc(reinterpret_cast<void **>(&out_host_), (size_t)(2 * host_off[n_out]) * sizeof(float),
                        cudaHostAllocDefault),
          "cudaHostAlloc(output f32 chunks)");
  const int64_t img_bytes = row_stride * h;
  if (img_bytes * batch > frames_cap_) {
    check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    if (frames_dev_) check(cudaFree(frames_dev_), "cudaFree(frame staging)");
    frames_dev_ = nullptr;
    check(cudaMalloc(&frames_dev_, (size_t)(img_bytes * batch)), "cudaMalloc(frame staging)");
    frames_cap_ = img_bytes * batch;
  }
  std::vector<std::pair<int, int>> chunks;
  for (int b0 = 0; b0 < batch;) {
    const int rem = batch - b0;
    const int nb = rem >= kChunk ? kChunk : rem >= 8 ? 8 : rem >= 4 ? 4 : rem >= 2 ? 2 : 1;
    chunks.emplace_back(b0, nb);
    b0 += nb;
  }
  const int n_chunks = (int)chunks.size();
  while ((int)chunk_events_.size() < 3 * n_chunks + 1) {
    cudaEvent_t e;
    check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    chunk_events_.push_back(e);
  }
  check(cudaEventRecord(chunk_events_[3 * n_chunks], stream_), "cudaEventRecord");
  check(cudaStreamWaitEvent(copy_in_, chunk_events_[3 * n_chunks], 0), "cudaStreamWaitEvent");
  // every chunk's frames queued at once (each into its own staging range)
  for (int c = 0; c < n_chunks; ++c) {
    const int b0 = chunks[(size_t)c].first, nb = chunks[(size_t)c].second;
    check(cudaMemcpyAsync(frames_dev_ + b0 * img_bytes, frames + b0 * img_bytes, (size_t)(nb * img_bytes),
                          cudaMemcpyHostToDevice, copy_in_),
          "frame copy");
    check(cudaEventRecord(chunk_events_[3 * c], copy_in_), "cudaEventRecord");
  }
  auto drain = [&](int c) {
    const int b0 = chunks[(size_t)c].first, nb = chunks[(size_t)c].second;
    const float *staged = out_host_ + (size_t)(c & 1) * host_off[n_out];
    check(cudaEventSynchronize(chunk_events_[3 * c + 2]), "cudaEventSynchronize");
    for (int i = 0; i < n_out; ++i) {
      const float *from = staged + host_off[i];
      float *to = outs[i] + (size_t)b0 * out_numel[i];
      host_parallel_for((size_t)(nb * out_numel[i]), 1 << 16,
                        [&](size_t b, size_t e) { std::memcpy(to + b, from + b, (e - b) * sizeof(float)); });
    }
  };
  for (int c = 0; c < n_chunks; ++c) {
    const int b0 = chunks[(size_t)c].first, nb = chunks[(size_t)c].second;
    check(cudaStreamWaitEvent(stream_, chunk_events_[3 * c], 0), "cudaStreamWaitEvent");
    launch_letterbox(frames_dev_ + b0 * img_bytes, img_bytes, row_stride, 0, nb, cfg, stream_);
    run(nb);
    for (int i = 0; i < n_out; ++i)
      check(launch_f16_to_f32(T_[(size_t)tid(output_name(i))].dptr, out_f32_ + out_off[i] + (size_t)b0 * out_numel[i],
                              nb * out_numel[i], stream_),
            "output conversion");
    check(cudaEventRecord(chunk_events_[3 * c + 1], stream_), "cudaEventRecord");
    check(cudaStreamWaitEvent(copy_out_, chunk_events_[3 * c + 1], 0), "cudaStreamWaitEvent");
    for (int i = 0; i < n_out; ++i) {
      float *dst = out_pinned ? outs[i] + (size_t)b0 * out_numel[i]
                              : out_host_ + (size_t)(c & 1) * host_off[n_out] + host_off[i];
      check(cudaMemcpyAsync(dst, out_f32_ + out_off[i] + (size_t)b0 * out_numel[i],
                            (size_t)(nb * out_numel[i]) * sizeof(float), cudaMemcpyDeviceToHost, copy_out_),
            "output copy");
    }
    check(cudaEventRecord(chunk_events_[3 * c + 2], copy_out_), "cudaEventRecord");
    if (!out_pinned && c >= 1) drain(c - 1);
  }
  if (!out_pinned) drain(n_chunks - 1);
  check(cudaEventRecord(chunk_events_[3 * n_chunks], copy_out_), "cudaEventRecord");
  check(cudaStreamWaitEvent(stream_, chunk_events_[3 * n_chunks], 0), "cudaStreamWaitEvent");
  synchronize();
  last_f32_batch_ = batch;
  if (letterbox_out)
    for (int b = 0; b < batch; ++b) {
      letterbox_out[3 * b] = cfg.letterbox ? lbt_.scale : 1.f;
      letterbox_out[3 * b + 1] = (float)lbt_.pad_left;
      letterbox_out[3 * b + 2] = (float)lbt_.pad_top;
    }
}

void Engine::decode_pose(int batch, float conf, float iou, int max_det, int nk, int kdims, const float *letterbox,
                         int *counts, float *dets) {
  require_device();
  pdl_scope();
  if (batch < 1 || batch > max_batch_) throw std::runtime_error("CudaPlanModel: batch out of range");
  if (output_count() < 1) throw std::runtime_error("PoseDecoder: unexpected output shape");
  const TensorRt &t = T_[(size_t)tid(output_name(0))];
  // channel-major [1, C, A] (the reference also accepts anchor-major; the
  // pose plans emit channel-major)
  if (t.dims.size() != 3 || !t.dense || t.dims[1] > t.dims[2])
    throw std::runtime_error("PoseDecoder: unexpected output shape");
  const int C = (int)t.dims[1], A = (int)t.dims[2];
  if (kdims <= 0) kdims = 3;
  if (nk <= 0) nk = (C - 5) / kdims;
  if (nk < 0 || 5 + nk * kdims > C) throw std::runtime_error("PoseDecoder: keypoints do not fit the output channels");
  if (A > kPoseNmsMaxAnchors) throw std::runtime_error("PoseDecoder: more anchors than the device decoder sorts");
  if (max_det < 1) throw std::runtime_error("PoseDecoder: max_det must be positive");
  check(cudaSetDevice(device_), "cudaSetDevice");
  int P = 4;  // (the boxes follow 4 * P bytes of keys in shared memory, 16-byte aligned)
  while (P < A) P <<= 1;
  const int S = 6 + 2 * nk;
  if (!nms_boxes_) {
    const size_t cap = (size_t)max_batch_ * kPoseNmsMaxAnchors;
    check(cudaMalloc(&nms_boxes_, cap * sizeof(float4)), "cudaMalloc(nms boxes)");
    check(cudaMalloc(&nms_kept_, cap * sizeof(int)), "cudaMalloc(nms kept)");
    check(cudaMalloc(&nms_pairs_, cap * sizeof(int2)), "cudaMalloc(nms keep lists)");
    check(cudaMalloc(&nms_counts_, (size_t)max_batch_ * 2 * sizeof(int)), "cudaMalloc(nms counts)");
    check(cudaMalloc(&nms_lbox_, (size_t)max_batch_ * 3 * sizeof(float)), "cudaMalloc(nms letterbox)");
    check(cudaHostAlloc(reinterpret_cast<void **>(&nms_pairs_host_), cap * sizeof(int2), cudaHostAllocDefault),
          "cudaHostAlloc(nms keep lists)");
  }
  const int64_t need = (int64_t)batch * max_det * S;  // floats of the result rows
  const int64_t idx = (int64_t)batch * (max_det + 2);  // ints: chosen anchors, then chosen and kept counts
  if (need > nms_dets_cap_ || idx > nms_idx_cap_) {
    if (nms_dets_) check(cudaFree(nms_dets_), "cudaFree(nms dets)");
    if (nms_chosen_) check(cudaFree(nms_chosen_), "cudaFree(nms chosen)");
    nms_dets_ = nullptr;
    nms_chosen_ = nullptr;
    check(cudaMalloc(&nms_dets_, (size_t)need * sizeof(float)), "cudaMalloc(nms dets)");
    check(cudaMalloc(&nms_chosen_, (size_t)idx * sizeof(int)), "cudaMalloc(nms chosen)");
    nms_dets_cap_ = need;
    nms_idx_cap_ = idx;
  }
  if (need + idx > nms_host_cap_) {
    if (nms_host_) check(cudaFreeHost(nms_host_), "cudaFreeHost(nms staging)");
    nms_host_ = nullptr;
    check(cudaHostAlloc(reinterpret_cast<void **>(&nms_host_), (size_t)(need + idx) * sizeof(float),
                        cudaHostAllocDefault),
          "cudaHostAlloc(nms staging)");
    nms_host_cap_ = need + idx;
  }
  if (letterbox)
    check(cudaMemcpyAsync(nms_lbox_, letterbox, (size_t)batch * 3 * sizeof(float), cudaMemcpyHostToDevice, stream_),
          "letterbox copy");
  // 1. candidates, stable score order, greedy suppression: each image's keep list
  // after a chunked ClBackend::infer the output tensor holds only the last
  // chunk; the f32 staging holds the whole batch (exact copies of the fp16 values)
  const bool from_f32 = last_f32_batch_ >= batch;
  PoseNmsArgs a{};
  a.out = from_f32 ? (const void *)out_f32_ : (const void *)t.dptr;
  a.out_f32 = from_f32 ? 1 : 0;
  a.img_stride = t.numel;
  a.A = A;
  a.P = P;
  a.nk = nk;
  a.kdims = kdims;
  a.conf = conf;
  a.iou = iou;
  a.letterbox = letterbox ? nms_lbox_ : nullptr;
  a.boxes = nms_boxes_;
  // boxes and the kept list in shared memory where they fit, else in scratch
  a.kept = nms_kept_;
  a.boxes_in_smem = pose_nms_smem_bytes(P, A, true, 0) <= (size_t)kPoseNmsSmemMax ? 1 : 0;
  a.kept_idx_smem = pose_nms_smem_bytes(P, A, a.boxes_in_smem != 0, A) <= (size_t)kPoseNmsSmemMax ? 1 : 0;
  a.counts = nms_counts_;
  a.pairs = nms_pairs_;
  check(launch_pose_nms(a, batch, stream_), "pose decode + NMS");
  int *host_idx = reinterpret_cast<int *>(nms_host_ + need);  // chosen anchors [batch][max_det], counts
  int *host_chosen = host_idx + (size_t)batch * max_det, *host_kept = host_chosen + batch;
  check(cudaMemcpyAsync(host_kept, nms_counts_, (size_t)batch * sizeof(int), cudaMemcpyDeviceToHost, stream_),
        "keep counts copy");
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  int longest = 0;
  for (int b = 0; b < batch; ++b) longest = std::max(longest, host_kept[b]);
  if (longest > 0)
    check(cudaMemcpy2DAsync(nms_pairs_host_, (size_t)longest * sizeof(int2), nms_pairs_, (size_t)P * sizeof(int2),
                            (size_t)longest * sizeof(int2), (size_t)batch, cudaMemcpyDeviceToHost, stream_),
          "keep lists copy");
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  // 2. the reference's last step (src/Decoders.cpp:58-63): the keep list, in
  // keep order, sorted by descending score with std::sort - not a stable
  // sort, so equal scores end up where std::sort leaves them, which depends on
  // the whole list - then cut at max_det.  std::sort's moves depend only on its
  // comparisons, so (score, anchor) pairs under a score-only comparator take
  // the permutation the reference's Detection objects take.
  std::vector<std::pair<float, int>> v;
  for (int b = 0; b < batch; ++b) {
    const int2 *pl = nms_pairs_host_ + (size_t)b * longest;
    v.resize((size_t)host_kept[b]);
    for (int k = 0; k < host_kept[b]; ++k) {
      float sc;
      std::memcpy(&sc, &pl[k].y, sizeof(float));
      v[(size_t)k] = {sc, pl[k].x};
    }
    std::sort(v.begin(), v.end(),
              [](const std::pair<float, int> &x, const std::pair<float, int> &y) { return x.first > y.first; });
    const int c = std::min(host_kept[b], max_det);
    host_chosen[b] = c;
    for (int k = 0; k < c; ++k) host_idx[(size_t)b * max_det + k] = v[(size_t)k].second;
  }
  // 3. the chosen detections' rows, through pinned staging to the caller
  check(cudaMemcpyAsync(nms_chosen_, host_idx, (size_t)batch * (max_det + 1) * sizeof(int), cudaMemcpyHostToDevice,
                        stream_),
        "chosen detections copy");
  PoseGatherArgs g{};
  g.out = a.out;
  g.out_f32 = a.out_f32;
  g.img_stride = t.numel;
  g.A = A;
  g.nk = nk;
  g.kdims = kdims;
  g.max_det = max_det;
  g.letterbox = a.letterbox;
  g.anchors = nms_chosen_;
  g.counts = nms_chosen_ + (size_t)batch * max_det;
  g.dets = nms_dets_;
  check(launch_pose_gather(g, batch, stream_), "pose detections gather");
  check(cudaMemcpyAsync(nms_host_, nms_dets_, (size_t)need * sizeof(float), cudaMemcpyDeviceToHost, stream_),
        "detections copy");
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  for (int b = 0; b < batch; ++b) {
    counts[b] = host_chosen[b];
    std::memcpy(dets + (size_t)b * max_det * S, nms_host_ + (size_t)b * max_det * S,
                (size_t)host_chosen[b] * S * sizeof(float));
  }
}

bool Engine::read_tensor_f16(const std::string &name, void *host_dst, int batch) {
  require_device();
  pdl_scope();
  check(cudaSetDevice(device_), "cudaSetDevice");
  auto it = tid_.find(name);
  if (it == tid_.end()) return false;
  const TensorRt &t = T_[(size_t)it->second];
  if (t.dptr == nullptr) return false;
  const int64_t n = t.numel * (t.is_init ? 1 : batch);
  if (t.dense) {
    check(cudaMemcpyAsync(host_dst, t.dptr, (size_t)n * 2, cudaMemcpyDeviceToHost, stream_), "tensor copy");
  } else {
    if (scratch_elems_ < n) {
      if (scratch_) cudaFree(scratch_);
      check(cudaMalloc(&scratch_, (size_t)n * 4), "cudaMalloc(scratch)");
      scratch_elems_ = n * 2;
    }
    View4 src = view(it->second);
    View4 dst = src;
    dst.ptr = scratch_;
    dst.sx = 1;
    dst.sy = dst.W;
    dst.sc = (int64_t)dst.H * dst.W;
    dst.sb = (int64_t)dst.C * dst.H * dst.W;
    check(launch_copy_v4(src, dst, batch, stream_), "tensor relayout");
    check(cudaMemcpyAsync(host_dst, scratch_, (size_t)n * 2, cudaMemcpyDeviceToHost, stream_), "tensor copy");
  }
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  return true;
}

int Engine::read_tensor_f16_staged(const std::string &name, void *host_dst, int batch, void *scratch,
                                   int64_t scratch_bytes, int64_t *need_bytes) {
  require_device();
  pdl_scope();
  check(cudaSetDevice(device_), "cudaSetDevice");
  auto it = tid_.find(name);
  if (it == tid_.end()) return 1;
  const TensorRt &t = T_[(size_t)it->second];
  if (t.dptr == nullptr) return 1;
  const int64_t n = t.numel * (t.is_init ? 1 : batch);
  if (need_bytes) *need_bytes = t.dense ? 0 : n * 2;
  if (t.dense) {
    check(cudaMemcpyAsync(host_dst, t.dptr, (size_t)n * 2, cudaMemcpyDeviceToHost, stream_), "tensor copy");
  } else {
    if (n * 2 > scratch_bytes) return 2;
    // the relayout writes every one of the n elements before the copy reads them
    View4 src = view(it->second);
    View4 dst = src;
    dst.ptr = static_cast<__half *>(scratch);
    dst.sx = 1;
    dst.sy = dst.W;
    dst.sc = (int64_t)dst.H * dst.W;
    dst.sb = (int64_t)dst.C * dst.H * dst.W;
    check(launch_copy_v4(src, dst, batch, stream_), "tensor relayout");
    check(cudaMemcpyAsync(host_dst, scratch, (size_t)n * 2, cudaMemcpyDeviceToHost, stream_), "tensor copy");
  }
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  return 0;
}

int Engine::graph_kernel_count(int batch) {
  require_device();
  pdl_scope();
  if (batch < 1 || batch > max_batch_) throw std::runtime_error("CudaPlanModel: batch out of range");
  check(cudaSetDevice(device_), "cudaSetDevice");
  tune(batch);
  cudaGraph_t g = nullptr;
  check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  for (auto &s : steps_) s.launch(batch, stream_);
  check(cudaStreamEndCapture(stream_, &g), "cudaStreamEndCapture");
  size_t n = 0;
  check(cudaGraphGetNodes(g, nullptr, &n), "cudaGraphGetNodes");
  std::vector<cudaGraphNode_t> nodes(n);
  check(cudaGraphGetNodes(g, nodes.data(), &n), "cudaGraphGetNodes");
  int kernels = 0;
  for (auto nd : nodes) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
  }
  cudaGraphDestroy(g);
  return kernels;
}

void Engine::set_conv_wait(long long limit_cycles, int probe) {
  require_device();
  if (limit_cycles < 1) throw std::runtime_error("CudaPlanModel: conv wait limit must be positive");
  wait_->limit = limit_cycles;
  wait_->probe = probe ? 1 : 0;
  // captured graphs hold the launch parameters of their capture: capture again
  check(cudaSetDevice(device_), "cudaSetDevice");
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  for (auto &g : graphs_) cudaGraphExecDestroy(g.second);
  graphs_.clear();
}

void Engine::require_device() const {
  if (dry_) throw std::runtime_error("CudaPlanModel: a dry run handle has no device state (IVC_FLAG_DRY_RUN)");
}

void Engine::pdl_scope() const { g_launch_pdl = (flags_ & kFlagNoPdl) == 0; }

void Engine::synchronize() { check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize"); }

int Engine::device_status() {
  int v = 0;
  check(cudaSetDevice(device_), "cudaSetDevice");
  check(cudaMemcpyAsync(&v, status_, sizeof(int), cudaMemcpyDeviceToHost, stream_), "status read");
  check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  if (v) check(cudaMemsetAsync(status_, 0, sizeof(int), stream_), "status reset");
  return v;
}

std::string Engine::describe() const {
  std::ostringstream os;
  for (const auto &t : T_) {
    os << "tensor " << t.name << (t.is_init ? " init" : "") << (t.nhwc ? " nhwc" : " planar") << " root="
       << T_[(size_t)t.root].name << " off=" << t.elem_off;
    if ((int)(&t - &T_[0]) == t.root && !t.is_init)
      os << " arena=" << t.arena_off << " life=[" << t.birth << "," << t.death << "] bytes/img=" << t.bytes_per_img
         << (t.materialized ? "" : " unmaterialized");
    os << "\n";
  }
  for (const auto &s : steps_) {
    os << "step " << s.family << " " << s.name;
    const size_t j = (size_t)(&s - &steps_[0]);
    if (n_streams_ > 1 && j < stream_of_.size()) os << " [stream " << stream_of_[j] << "]";
    if (!s.info.empty()) os << " [" << s.info << "]";
    if (s.geometry)
      for (const auto &g : *s.geometry) os << " [B=" << g.first << " " << g.second << "]";
    os << "\n";
  }
  return os.str();
}

}  // namespace ivb
