// Exercises include/infvino_b200_backend.hpp the way a reference-side caller
// would (InferenceEngine / infvino_numtest style): construct, query shapes,
// infer twice (A then B), dump the last outputs as raw f32.
//   backend_driver <plan> <input_a.f32> <input_b.f32> <out.f32>
//   backend_driver --empty-plan     (checks the empty-plan error message)
//   backend_driver --pose <plan> <input.f32> <dets.f32>
//                                   (infer one image, decodePose on the device,
//                                    dump anchor, score, box, keypoints per detection)
//   backend_driver --planmodel <plan> <input.f32> <out.f16>
//                                   (PlanModel: setInput, run twice with profiling,
//                                    readOutput / readTensor, profile(), pool stats)
//   backend_driver --device <plan>  (DeviceInfo of the backend)
// Built with -DWITH_REFERENCE_TYPES against the reference's headers, the
// backend is instantiated with infvino::Tensor, infvino::ModelInfo and
// infvino::DeviceInfo.
#include <cstdio>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "infvino_b200_backend.hpp"

#ifdef WITH_REFERENCE_TYPES
// the reference's own Tensor, ModelInfo and DeviceInfo types (their OpenCV /
// OpenCL includes resolve to declarations-only stand-ins in the test)
#include "infvino/Device.hpp"
#include "infvino/ModelInfo.hpp"
#include "infvino/Tensor.hpp"
using TensorT = infvino::Tensor;
using ModelInfo = infvino::ModelInfo;
using DeviceInfoT = infvino::DeviceInfo;
static ModelInfo model_info(const std::string &plan) {
  ModelInfo m;
  m.plan = plan;
  return m;
}
#else
struct TensorT {
  std::vector<int64_t> shape;
  std::vector<float> data;
};
struct ModelInfo {
  std::string plan;
};
using DeviceInfoT = infvino_b200::DeviceInfo;
static ModelInfo model_info(const std::string &plan) { return ModelInfo{plan}; }
#endif

static std::vector<float> read_f32(const char *path) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  std::vector<float> v((size_t)f.tellg() / 4);
  f.seekg(0);
  f.read(reinterpret_cast<char *>(v.data()), (std::streamsize)(v.size() * 4));
  return v;
}

// PlanModel the way the reference's tools drive it (infvino_numtest /
// kernel_run: setInput once, run, readOutput / readTensor, profile)
static int drive_plan_model(const char *plan, const char *input_f32, const char *out_f16) {
  infvino_b200::PlanModel pm(plan, "", -1, 0, /*profiling=*/true);
  const auto x = read_f32(input_f32);
  if (x.size() != pm.inputNumel()) return 10;
  std::vector<uint16_t> x16(x.size());
  ivc_f32_to_f16(x.data(), x16.data(), x.size());
  pm.setInput(x16.data());
  pm.run();
  pm.run();  // the input persists across runs
  std::vector<uint16_t> y(pm.outputNumel(0));
  pm.readOutput(0, y.data());
  std::vector<uint16_t> t(pm.tensorNumel(pm.outputName(0)));
  if (!pm.readTensor(pm.outputName(0), t.data()) || t != y) return 11;
  if (pm.readTensor("no such tensor", t.data())) return 12;
  const auto prof = pm.profile();
  if (prof.nodes.empty() || prof.busy_ms <= 0.0 || prof.nodes[0].calls != 2) return 13;
  if (pm.poolAllocatedBytes() == 0 || pm.poolAllocatedBytes() > pm.poolRequestedBytes()) return 14;
  std::ofstream o(out_f16, std::ios::binary);
  o.write(reinterpret_cast<const char *>(y.data()), (std::streamsize)(y.size() * 2));
  std::cout << "ok planmodel " << prof.nodes.size() << " steps, busy " << prof.busy_ms << " ms, last run "
            << pm.lastRunMs() << " ms\n";
  return 0;
}

int main(int argc, char **argv) {
  using Backend = infvino_b200::CudaBackendT<TensorT, ModelInfo, DeviceInfoT>;
  if (argc == 5 && std::string(argv[1]) == "--planmodel") return drive_plan_model(argv[2], argv[3], argv[4]);
  if (argc == 3 && std::string(argv[1]) == "--device") {
    Backend b(model_info(argv[2]));
    const DeviceInfoT &d = b.device();  // what InferenceEngine::device() forwards
    std::cout << "resolved " << d.resolved << " | " << d.full_name << " | eu " << d.eu << " | clock " << d.clock_mhz
              << " | available " << d.available.size() << "\n";
    return (d.eu > 0 && !d.full_name.empty() && !d.available.empty()) ? 0 : 20;
  }
  if (argc == 2 && std::string(argv[1]) == "--empty-plan") {
    try {
      Backend b(model_info(""));
    } catch (const std::runtime_error &e) {
      std::cout << e.what() << "\n";
      return std::string(e.what()).find("ModelInfo.plan is empty") != std::string::npos ? 0 : 1;
    }
    return 1;
  }
  if (argc == 5 && std::string(argv[1]) == "--pose") {
    Backend b(model_info(argv[2]));
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
  Backend b(model_info(argv[1]));
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
