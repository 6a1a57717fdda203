// Header-only C++ drop-in for infvino's ClBackend, layered on the C ABI in
// infvino_b200.h.  Same public surface as the reference class
// (include/infvino/ClBackend.hpp:29-53):
//
//   explicit ClBackend(const ModelInfo &, bool profiling = false);
//   const std::vector<int64_t> &inputDims() const;
//   const std::vector<std::vector<int64_t>> &outputShapes() const;
//   std::vector<Tensor> infer(const float *input_f32, size_t numel);
//   const DeviceInfo &device() const;
//   double lastInferMs() const;
//
// It is a template over the caller's tensor / model-info types so that this
// header needs none of the reference's headers: inside the reference tree,
//
//   using CudaBackend = infvino_b200::CudaBackendT<infvino::Tensor, infvino::ModelInfo>;
//
// `Tensor` needs `shape` (std::vector<int64_t>) and `data` (std::vector<float>)
// members; `ModelInfo` needs a `plan` string.  Errors are std::runtime_error with
// the reference's messages (src/ClBackend.cpp:15-18, :35-39); infer() is
// serialised by a mutex like ClBackend::infer (src/ClBackend.cpp:33).
#ifndef INFVINO_B200_BACKEND_HPP_
#define INFVINO_B200_BACKEND_HPP_

#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "infvino_b200.h"

namespace infvino_b200 {

struct DeviceInfo {
  std::string backend = "cuda";
  int ordinal = 0;
};

// One pose detection of decodePose(): the reference's Detection for a pose
// model (include/infvino/Types.hpp:38-45: box, score, class 0, keypoints)
// without OpenCV types, plus the anchor it came from.
struct PoseDetection {
  int anchor = 0;
  float score = 0.f;
  float x = 0.f, y = 0.f, w = 0.f, h = 0.f;  // box in image coordinates
  std::vector<float> keypoints;             // x, y per keypoint
};

template <class TensorT, class ModelInfoT>
class CudaBackendT {
 public:
  explicit CudaBackendT(const ModelInfoT &info, bool profiling = false, int device_ordinal = 0, int max_batch = 1)
      : profiling_(profiling) {
    if (info.plan.empty())
      throw std::runtime_error(
          "ClBackend: ModelInfo.plan is empty. Generate it first with "
          "scripts/onnx2plan.py --onnx <model.onnx> --out-dir models");
    // profiling runs launch eagerly so that per-launch events can be taken
    const unsigned flags = profiling ? IVC_FLAG_NO_GRAPH : 0u;
    if (ivc_create(info.plan.c_str(), device_ordinal, max_batch, flags, &m_) != IVC_OK)
      throw std::runtime_error(ivc_last_error(nullptr));
    int rank = 0;
    int64_t d[16];
    ivc_input_dims(m_, d, 16, &rank);
    input_dims_.assign(d, d + rank);
    for (int i = 0; i < ivc_output_count(m_); ++i) {
      ivc_output_dims(m_, i, d, 16, &rank);
      output_shapes_.emplace_back(d, d + rank);
    }
    device_.ordinal = device_ordinal;
  }
  ~CudaBackendT() { ivc_destroy(m_); }
  CudaBackendT(const CudaBackendT &) = delete;
  CudaBackendT &operator=(const CudaBackendT &) = delete;

  const std::vector<int64_t> &inputDims() const { return input_dims_; }
  const std::vector<std::vector<int64_t>> &outputShapes() const { return output_shapes_; }
  const DeviceInfo &device() const { return device_; }
  double lastInferMs() const { return ivc_last_infer_ms(m_); }

  // One image (numel == prod(inputDims())), or `batch` images back to back.
  std::vector<TensorT> infer(const float *input_f32, size_t numel, int batch = 1) {
    std::lock_guard<std::mutex> lock(mutex_);
    std::vector<TensorT> outs(output_shapes_.size());
    std::vector<float *> ptrs;
    for (size_t i = 0; i < outs.size(); ++i) {
      outs[i].shape = output_shapes_[i];
      if (batch != 1) outs[i].shape[0] = batch;
      outs[i].data.resize((size_t)ivc_output_numel(m_, (int)i) * (size_t)batch);
      ptrs.push_back(outs[i].data.data());
    }
    if (ivc_infer_f32(m_, input_f32, numel, batch, ptrs.data()) != IVC_OK) throw std::runtime_error(ivc_last_error(m_));
    return outs;
  }

  // Pose decode + greedy NMS of the last infer() on the device, in place of
  // PoseDecoder::decode with nmsPerClass (src/Decoders.cpp:127-179, :33-65):
  // per image, the detections in descending score.  `letterbox` (host):
  // [batch][scale, pad_left, pad_top], or null for scale 1 and no padding.
  std::vector<std::vector<PoseDetection>> decodePose(int batch = 1, float conf = 0.25f, float iou = 0.7f,
                                                     int max_det = 300, int nk = 17, int kdims = 3,
                                                     const float *letterbox = nullptr) {
    std::lock_guard<std::mutex> lock(mutex_);
    const size_t S = 6 + 2 * (size_t)nk;
    std::vector<int> counts((size_t)batch);
    std::vector<float> dets((size_t)batch * (size_t)max_det * S);
    if (ivc_decode_pose(m_, batch, conf, iou, max_det, nk, kdims, letterbox, counts.data(), dets.data()) != IVC_OK)
      throw std::runtime_error(ivc_last_error(m_));
    std::vector<std::vector<PoseDetection>> out((size_t)batch);
    for (int b = 0; b < batch; ++b)
      for (int k = 0; k < counts[(size_t)b]; ++k) {
        const float *r = &dets[((size_t)b * (size_t)max_det + (size_t)k) * S];
        PoseDetection d;
        d.anchor = (int)r[0];
        d.score = r[1];
        d.x = r[2];
        d.y = r[3];
        d.w = r[4];
        d.h = r[5];
        d.keypoints.assign(r + 6, r + S);
        out[(size_t)b].push_back(std::move(d));
      }
    return out;
  }

  ivc_model *handle() const { return m_; }

 private:
  ivc_model *m_ = nullptr;
  bool profiling_ = false;
  std::vector<int64_t> input_dims_;
  std::vector<std::vector<int64_t>> output_shapes_;
  DeviceInfo device_;
  std::mutex mutex_;
};

}  // namespace infvino_b200

#endif  // INFVINO_B200_BACKEND_HPP_
