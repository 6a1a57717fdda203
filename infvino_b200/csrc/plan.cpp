// Plan parsing and load-time rewrites.  Behaviour (grammar, error messages,
// rewrite conditions) follows the reference executor's `PlanModel::parse`,
// `fuseConcatConv1x1` and `fuseResidualAdd` (src/PlanModel.cpp:447-740).
#include "plan.h"

#include <algorithm>
#include <cstdlib>
#include <fstream>
#include <set>
#include <sstream>
#include <stdexcept>

namespace ivb {

int PlanNode::ai(const char *k, int def) const {
  auto it = attr.find(k);
  return it == attr.end() ? def : std::atoi(it->second.c_str());
}

std::vector<std::string> split_csv(const std::string &s) {
  std::vector<std::string> out;
  if (s == "-") return out;  // a lone "-" means "no tensors"
  std::stringstream ss(s);
  std::string tok;
  while (std::getline(ss, tok, ',')) out.push_back(tok);
  return out;
}

PlanTensor &Plan::ref(const std::string &name) {
  auto it = T_.find(name);
  if (it == T_.end()) throw std::runtime_error("PlanModel: missing tensor: " + name);
  return it->second;
}
const PlanTensor &Plan::ref(const std::string &name) const {
  auto it = T_.find(name);
  if (it == T_.end()) throw std::runtime_error("PlanModel: missing tensor: " + name);
  return it->second;
}

Plan::Plan(const std::string &path) : path_(path) {
  std::ifstream f(path);
  if (!f) throw std::runtime_error("PlanModel: cannot open plan " + path);
  const auto slash = path.find_last_of('/');
  dir_ = slash == std::string::npos ? "." : path.substr(0, slash);
  std::string line;
  int lineno = 0;
  while (std::getline(f, line)) {
    ++lineno;
    if (line.empty() || line[0] == '#') continue;
    std::istringstream ls(line);
    std::string kind;
    ls >> kind;
    if (kind == "input" || kind == "tensor" || kind == "init") {
      PlanTensor t;
      ls >> t.name;
      if (kind == "init") ls >> t.file;
      std::string tok;
      while (ls >> tok) {
        char *end = nullptr;
        const long long v = std::strtoll(tok.c_str(), &end, 10);
        if (!end || *end != '\0' || v < 0)
          throw std::runtime_error("PlanModel: bad dimension '" + tok + "' at line " + std::to_string(lineno));
        t.dims.push_back(v);
      }
      if (t.name.empty()) throw std::runtime_error("PlanModel: missing name at line " + std::to_string(lineno));
      if (kind == "input") {
        t.is_input = true;
        if (input_.empty()) input_ = t.name;
      }
      if (kind == "init") {
        t.is_init = true;
        const std::string p = (!t.file.empty() && t.file[0] == '/') ? t.file : dir_ + "/" + t.file;
        std::ifstream bf(p, std::ios::binary);
        if (!bf) throw std::runtime_error("PlanModel: cannot open init " + p);
        t.host.resize((size_t)t.numel());
        bf.read(reinterpret_cast<char *>(t.host.data()), (std::streamsize)(t.host.size() * 2));
        if (bf.gcount() != (std::streamsize)(t.host.size() * 2))
          throw std::runtime_error("PlanModel: init file too short: " + p);
        t.file = p;
      }
      T_[t.name] = std::move(t);
    } else if (kind == "node") {
      PlanNode n;
      std::string ins, outs;
      ls >> n.op >> ins >> outs;
      if (n.op.empty() || outs.empty())
        throw std::runtime_error("PlanModel: malformed node at line " + std::to_string(lineno));
      n.ins = split_csv(ins);
      n.outs = split_csv(outs);
      std::string kv;
      while (ls >> kv) {
        const auto p = kv.find('=');
        if (p != std::string::npos) n.attr[kv.substr(0, p)] = kv.substr(p + 1);
      }
      nodes_.push_back(std::move(n));
    } else if (kind == "output") {
      std::string name;
      ls >> name;
      if (!name.empty()) outputs_.push_back(name);
    } else {
      throw std::runtime_error("PlanModel: unknown line kind '" + kind + "' at line " + std::to_string(lineno));
    }
  }
  if (input_.empty()) throw std::runtime_error("PlanModel: plan has no 'input' line");
  if (outputs_.empty()) throw std::runtime_error("PlanModel: plan has no 'output' line");
  for (const auto &o : outputs_) {
    auto it = T_.find(o);
    if (it == T_.end()) throw std::runtime_error("PlanModel: output tensor not declared: " + o);
    it->second.is_output = true;
  }
  for (const auto &n : nodes_) {
    for (const auto &i : n.ins)
      if (i != "-" && !T_.count(i)) throw std::runtime_error("PlanModel: missing tensor: " + i);
    for (const auto &o : n.outs)
      if (o != "-" && !T_.count(o)) throw std::runtime_error("PlanModel: missing tensor: " + o);
  }
}

int Plan::fuse_concat_conv1x1(const std::vector<std::string> &allowed) {
  const std::set<std::string> ok_cat(allowed.begin(), allowed.end());
  std::map<std::string, size_t> producer;
  std::map<std::string, int> uses;
  for (size_t i = 0; i < nodes_.size(); ++i) {
    for (const auto &o : nodes_[i].outs) producer[o] = i;
    for (const auto &in : nodes_[i].ins)
      if (in != "-") ++uses[in];
  }
  std::vector<char> drop(nodes_.size(), 0);
  int fused = 0;
  for (auto &n : nodes_) {
    if (n.op != "conv1x1" || n.ins.size() < 2 || n.ins[1] == "-") continue;
    const std::string x = n.ins[1];
    auto pit = producer.find(x);
    if (pit == producer.end()) continue;
    const PlanNode &cat = nodes_[pit->second];
    if (cat.op != "concat4" || uses[x] != 1 || cat.ai("outer", 1) != 1 || !ok_cat.count(x)) continue;
    if (T_.at(x).is_output) continue;
    const int cnt[4] = {cat.ai("ca", 0), cat.ai("cb", 0), cat.ai("cc", 0), cat.ai("cd", 0)};
    if (cnt[0] <= 0) continue;
    bool ok = true;
    std::string src[4];
    for (int j = 0; j < 4; ++j) {
      src[j] = (j < (int)cat.ins.size()) ? cat.ins[j] : "-";
      if (cnt[j] > 0 && (src[j] == "-" || !T_.count(src[j]))) ok = false;
      if (cnt[j] <= 0) src[j] = "-";
    }
    if (!ok) continue;
    PlanNode f;
    f.op = "conv1x1_cat4";
    f.attr = n.attr;
    f.attr["cat_ca"] = std::to_string(cnt[0]);
    f.attr["cat_cb"] = std::to_string(cnt[1]);
    f.attr["cat_cc"] = std::to_string(cnt[2]);
    f.attr["cat_cd"] = std::to_string(cnt[3]);
    // [w, src0..src3, bias, res]
    f.ins = {n.ins[0], src[0], src[1], src[2], src[3], n.ins.size() > 2 ? n.ins[2] : "-",
             n.ins.size() > 3 ? n.ins[3] : "-"};
    f.outs = n.outs;
    n = f;
    drop[pit->second] = 1;
    ++fused;
  }
  if (fused) {
    std::vector<PlanNode> kept;
    for (size_t i = 0; i < nodes_.size(); ++i)
      if (!drop[i]) kept.push_back(std::move(nodes_[i]));
    nodes_ = std::move(kept);
  }
  fusions_concat += fused;
  return fused;
}

int Plan::fuse_residual_add() {
  std::map<std::string, size_t> producer;
  std::map<std::string, int> uses;
  for (size_t i = 0; i < nodes_.size(); ++i) {
    for (const auto &o : nodes_[i].outs) producer[o] = i;
    for (const auto &in : nodes_[i].ins)
      if (in != "-") ++uses[in];
  }
  auto res_slot = [](const std::string &op) -> int {
    if (op == "conv1x1_cat4") return 6;
    if (op == "conv1x1" || op == "conv3x3") return 3;
    return -1;
  };
  std::vector<char> drop(nodes_.size(), 0);
  int fused = 0;
  for (size_t i = 0; i < nodes_.size(); ++i) {
    PlanNode &e = nodes_[i];
    if (e.op != "ew_binary" || e.ai("op", 0) != 0 || e.ins.size() < 2) continue;
    if (e.has("bdims") && e.ai("b_scalar", 0) != 1) continue;  // no broadcast
    if (e.ai("b_scalar", 0) == 1) continue;                     // scalar operand: not a residual
    for (int k = 0; k < 2; ++k) {
      const std::string pname = e.ins[k], rname = e.ins[1 - k];
      auto pit = producer.find(pname);
      if (pit == producer.end() || drop[pit->second]) continue;
      PlanNode &c = nodes_[pit->second];
      const int rs = res_slot(c.op);
      if (rs < 0 || uses[pname] != 1 || T_.at(pname).is_output) continue;
      if (c.outs.size() != 1 || c.outs[0] != pname) continue;
      if (rname == "-" || !T_.count(rname)) continue;
      if (T_.at(rname).numel() != T_.at(pname).numel()) continue;
      if ((int)c.ins.size() > rs && c.ins[rs] != "-") continue;  // already has a residual
      auto rit = producer.find(rname);
      if (rit == producer.end() || rit->second >= pit->second) continue;  // residual must exist first
      if ((int)c.ins.size() <= rs) c.ins.resize((size_t)rs + 1, "-");
      c.ins[(size_t)rs] = rname;
      c.outs[0] = e.outs[0];
      producer.erase(pname);
      producer[e.outs[0]] = pit->second;
      drop[i] = 1;
      ++fused;
      break;
    }
  }
  if (fused) {
    std::vector<PlanNode> kept;
    for (size_t i = 0; i < nodes_.size(); ++i)
      if (!drop[i]) kept.push_back(std::move(nodes_[i]));
    nodes_ = std::move(kept);
  }
  fusions_res += fused;
  return fused;
}

int Plan::fuse_sibling_convs(const std::set<std::string> &channels_last, std::vector<std::string> *merged_outputs) {
  std::map<std::string, int> uses;
  for (const auto &n : nodes_)
    for (const auto &in : n.ins)
      if (in != "-") ++uses[in];
  auto opt_in = [](const PlanNode &n, size_t k) { return n.ins.size() > k ? n.ins[k] : std::string("-"); };
  // members keyed by everything that must agree: op, input, geometry,
  // activation and the weight shape past the output-channel axis
  std::map<std::string, std::vector<size_t>> groups;
  for (size_t i = 0; i < nodes_.size(); ++i) {
    const PlanNode &n = nodes_[i];
    const bool c3 = n.op == "conv3x3", c1 = n.op == "conv1x1";
    if (!(c3 || c1) || n.outs.size() != 1) continue;
    const std::string x = c3 ? opt_in(n, 0) : opt_in(n, 1), w = c3 ? opt_in(n, 1) : opt_in(n, 0), b = opt_in(n, 2);
    if (x == "-" || w == "-" || opt_in(n, 3) != "-" || opt_in(n, 4) != "-") continue;  // no residual / scale
    const PlanTensor &wt = T_.at(w), &ot = T_.at(n.outs[0]);
    if (!wt.is_init || wt.dims.size() < 2 || (int64_t)wt.host.size() != wt.numel()) continue;
    if (b != "-" && (!T_.at(b).is_init || T_.at(b).numel() != wt.dims[0] ||
                     (int64_t)T_.at(b).host.size() != wt.dims[0]))
      continue;
    if (ot.is_output || ot.dims.size() != 4 || ot.dims[1] != wt.dims[0] || !channels_last.count(n.outs[0]) ||
        !channels_last.count(x))
      continue;
    std::string key = n.op + "|" + x + "|" + (b == "-" ? "nb" : "b");
    for (const char *k : {"stride", "pad", "Hout", "Wout", "act"}) key += "|" + std::to_string(n.ai(k, -1));
    for (size_t d = 1; d < wt.dims.size(); ++d) key += "|" + std::to_string(wt.dims[d]);
    for (size_t d = 2; d < 4; ++d) key += "|" + std::to_string(ot.dims[d]);
    groups[key].push_back(i);
  }
  std::vector<char> drop(nodes_.size(), 0);
  std::map<size_t, std::vector<PlanNode>> replace;  // first member -> merged node + views
  int fused = 0;
  for (const auto &g : groups) {
    const std::vector<size_t> &mem = g.second;
    if (mem.size() < 2) continue;
    const PlanNode &first = nodes_[mem[0]];
    const bool c3 = first.op == "conv3x3";
    const std::string wname = c3 ? first.ins[1] : first.ins[0], bname = opt_in(first, 2);
    const PlanTensor &w0 = T_.at(wname);
    const int64_t per = w0.numel() / w0.dims[0];  // weights per output channel
    int64_t ctot = 0, calg = 0;
    std::vector<int64_t> off;
    for (size_t j : mem) {
      const int64_t co = T_.at(c3 ? nodes_[j].ins[1] : nodes_[j].ins[0]).dims[0];
      off.push_back(ctot);
      ctot += (co + 7) / 8 * 8;  // channel views start on 16-byte boundaries
      calg += co;
    }
    const std::string tag = "siblings:" + first.outs[0];
    if (T_.count(tag) || T_.count(tag + ".weight") || T_.count(tag + ".bias")) continue;
    PlanTensor mw;
    mw.name = tag + ".weight";
    mw.dims = w0.dims;
    mw.dims[0] = ctot;
    mw.is_init = true;
    mw.host.assign((size_t)(ctot * per), 0);
    PlanTensor mb;
    mb.name = tag + ".bias";
    mb.dims = {ctot};
    mb.is_init = true;
    mb.host.assign((size_t)ctot, 0);
    PlanTensor mo = T_.at(first.outs[0]);
    mo.name = tag;
    mo.dims[1] = ctot;
    mo.file.clear();
    PlanNode m = first;
    m.ins = c3 ? std::vector<std::string>{first.ins[0], mw.name, bname == "-" ? "-" : mb.name, "-"}
               : std::vector<std::string>{mw.name, first.ins[1], bname == "-" ? "-" : mb.name, "-"};
    m.outs = {tag};
    m.attr["alg_cout"] = std::to_string(calg);
    std::vector<PlanNode> seq{m};
    for (size_t k = 0; k < mem.size(); ++k) {
      const PlanNode &n = nodes_[mem[k]];
      const PlanTensor &wt = T_.at(c3 ? n.ins[1] : n.ins[0]);
      std::copy(wt.host.begin(), wt.host.end(), mw.host.begin() + off[k] * per);
      if (bname != "-") {
        const PlanTensor &bt = T_.at(n.ins[2]);
        std::copy(bt.host.begin(), bt.host.end(), mb.host.begin() + off[k]);
      }
      const PlanTensor &ot = T_.at(n.outs[0]);
      PlanNode v;
      v.op = "copy_c";
      v.ins = {tag};
      v.outs = n.outs;
      v.attr["c0"] = std::to_string(off[k]);
      v.attr["cnt"] = std::to_string(ot.dims[1]);
      v.attr["HW"] = std::to_string(ot.dims[2] * ot.dims[3]);
      v.attr["dst_off"] = "0";
      seq.push_back(v);
      drop[mem[k]] = 1;
    }
    T_[mw.name] = std::move(mw);
    if (bname != "-") T_[mb.name] = std::move(mb);
    T_[tag] = std::move(mo);
    replace[mem[0]] = std::move(seq);
    if (merged_outputs) merged_outputs->push_back(tag);
    ++fused;
  }
  if (fused) {
    std::vector<PlanNode> kept;
    for (size_t i = 0; i < nodes_.size(); ++i) {
      auto it = replace.find(i);
      if (it != replace.end())
        for (auto &n : it->second) kept.push_back(std::move(n));
      else if (!drop[i])
        kept.push_back(std::move(nodes_[i]));
    }
    nodes_ = std::move(kept);
  }
  fusions_sibling += fused;
  return fused;
}

}  // namespace ivb
