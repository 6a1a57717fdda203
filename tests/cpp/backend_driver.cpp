// Exercises include/infvino_b200_backend.hpp the way a reference-side caller
// would (InferenceEngine / infvino_numtest style): construct, query shapes,
// infer twice (A then B), dump the last outputs as raw f32.
//   backend_driver <plan> <input_a.f32> <input_b.f32> <out.f32>
//   backend_driver --empty-plan     (checks the empty-plan error message)
//   backend_driver --pose <plan> <input.f32> <dets.f32>
//                                   (infer one image, decodePose on the device,
//                                    dump anchor, score, box, keypoints per detection)
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
  if (argc == 5 && std::string(argv[1]) == "--pose") {
    Backend b(ModelInfo{argv[2]});
    size_t n = 1;
    for (auto d : b.inputDims()) n *= (size_t)d;
    const auto x = read_f32(argv[3]);
    b.infer(x.data(), n);
    const auto dets = b.decodePose();
    std::ofstream o(argv[4], std::ios::binary);
    for (const auto &d : dets[0]) {
      const float head[6] = {(float)d.anchor, d.score, d.x, d.y, d.w, d.h};
      o.write(reinterpret_cast<const char *>(head), sizeof(head));
      o.write(reinterpret_cast<const char *>(d.keypoints.data()), (std::streamsize)(d.keypoints.size() * 4));
    }
    std::cout << "ok " << dets[0].size() << " detections\n";
    return 0;
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
