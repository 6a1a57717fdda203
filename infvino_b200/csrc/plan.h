// Execution-plan model: text grammar, tensor table, node list and the load-time
// rewrites of the reference executor.
#pragma once

#include <cstdint>
#include <map>
#include <set>
#include <string>
#include <vector>

namespace ivb {

struct PlanTensor {
  std::string name;
  std::vector<int64_t> dims;
  bool is_init = false;
  bool is_input = false;
  bool is_output = false;
  std::string file;                // init: .bin path (resolved)
  std::vector<uint16_t> host;      // init: fp16 payload
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
};

struct PlanNode {
  std::string op;
  std::vector<std::string> ins, outs;
  std::map<std::string, std::string> attr;
  int ai(const char *k, int def) const;
  bool has(const char *k) const { return attr.count(k) != 0; }
};

// Parsed plan.  Grammar (include/infvino/PlanModel.hpp:6-12 in the reference):
//   input  <name> <d0> ...            init <name> <file.bin> <d0> ...
//   tensor <name> <d0> ...            node <op> <in_csv|-> <out_csv> [k=v ...]
//   output <name>                     # comment
class Plan {
 public:
  // Parses the plan and loads every initializer (fp16 little-endian, path
  // relative to the plan's directory).  Throws std::runtime_error with the
  // reference's messages on malformed input.
  explicit Plan(const std::string &path);

  // Load-time rewrites (numerically transparent):
  //  * concat4(outer=1) -> conv1x1 becomes conv1x1_cat4 with four sources
  //    (reference src/PlanModel.cpp:575-665);
  //  * conv -> ew_binary add becomes the conv's residual input (reference
  //    src/PlanModel.cpp:667-740; here conv3x3 qualifies too, since its
  //    epilogue applies the residual after the activation in fp16 just like the
  //    standalone add).
  // `allow_cat` filters which concat outputs may be fused (layout constraint).
  int fuse_concat_conv1x1(const std::vector<std::string> &allowed_concat_outputs);
  int fuse_residual_add();
  //  * sibling convolutions (same op, input, geometry and activation, no
  //    residual) become one convolution over the members' output channels side
  //    by side, each member padded to a multiple of 8 channels with zero weight
  //    rows, and every member output a channel view of it (copy_c at its
  //    offset, zero-copy for channels-last tensors).  Members and input must be
  //    in `channels_last`; the merged outputs are appended to `merged_outputs`.
  //    The merged node carries `alg_cout` (the members' channel total) for the
  //    algorithmic FLOP count.
  int fuse_sibling_convs(const std::set<std::string> &channels_last, std::vector<std::string> *merged_outputs);

  const std::string &path() const { return path_; }
  const std::string &dir() const { return dir_; }
  const std::string &input() const { return input_; }
  const std::vector<std::string> &outputs() const { return outputs_; }
  std::vector<PlanNode> &nodes() { return nodes_; }
  const std::vector<PlanNode> &nodes() const { return nodes_; }
  std::map<std::string, PlanTensor> &tensors() { return T_; }
  const std::map<std::string, PlanTensor> &tensors() const { return T_; }
  PlanTensor &ref(const std::string &name);
  const PlanTensor &ref(const std::string &name) const;
  bool has(const std::string &name) const { return T_.count(name) != 0; }

  int fusions_concat = 0, fusions_res = 0, fusions_sibling = 0;

 private:
  std::string path_, dir_, input_;
  std::vector<std::string> outputs_;
  std::map<std::string, PlanTensor> T_;
  std::vector<PlanNode> nodes_;
};

std::vector<std::string> split_csv(const std::string &s);

}  // namespace ivb
