// Exercises include/infvino_b200_backend.hpp the way a reference-side caller
// would (InferenceEngine / infvino_numtest style): construct, query shapes,
// infer twice (A then B), dump the last outputs as raw f32.
//   backend_driver <plan> <input_a.f32> <input_b.f32> <out.f32>
//   backend_driver --empty-plan     (checks the empty-plan error message)
#include <cstdio>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#ifdef WITH_REFERENCE_TENSOR
#include "infvino/Tensor.hpp"  // the reference's own Tensor type
using TensorT = infvino::Tensor;
#else
struct TensorT {
  std::vector<int64_t> shape;
  std::vector<float> data;
};
#endif
#include "infvino_b200_backend.hpp"

struct ModelInfo {
  std::string plan;
};

static std::vector<float> read_f32(const char *path) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  std::vector<float> v((size_t)f.tellg() / 4);
  f.seekg(0);
  f.read(reinterpret_cast<char *>(v.data()), (std::streamsize)(v.size() * 4));
  return v;
}

int main(int argc, char **argv) {
  using Backend = infvino_b200::CudaBackendT<TensorT, ModelInfo>;
  if (argc == 2 && std::string(argv[1]) == "--empty-plan") {
    try {
      Backend b(ModelInfo{""});
    } catch (const std::runtime_error &e) {
      std::cout << e.what() << "\n";
      return std::string(e.what()).find("ModelInfo.plan is empty") != std::string::npos ? 0 : 1;
    }
    return 1;
  }
  if (argc != 5) return 2;
  Backend b(ModelInfo{argv[1]});
  size_t n = 1;
  for (auto d : b.inputDims()) n *= (size_t)d;
  const auto a = read_f32(argv[2]), bb = read_f32(argv[3]);
  b.infer(a.data(), n);
  auto outs = b.infer(bb.data(), n);
  try {
    b.infer(a.data(), n - 1);
    return 3;
  } catch (const std::runtime_error &e) {
    if (std::string(e.what()).find("input numel mismatch") == std::string::npos) return 4;
  }
  std::ofstream o(argv[4], std::ios::binary);
  for (auto &t : outs) o.write(reinterpret_cast<const char *>(t.data.data()), (std::streamsize)(t.data.size() * 4));
  std::cout << "ok " << outs.size() << " outputs, last infer " << b.lastInferMs() << " ms\n";
  return 0;
}
