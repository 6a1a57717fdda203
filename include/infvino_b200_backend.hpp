// Header-only C++ drop-ins for infvino's ClBackend and PlanModel, layered on
// the C ABI in infvino_b200.h.
//
// CudaBackendT: the public surface of the reference's ClBackend
// (include/infvino/ClBackend.hpp:29-53):
//
//   explicit ClBackend(const ModelInfo &, bool profiling = false);
//   const std::vector<int64_t> &inputDims() const;
//   const std::vector<std::vector<int64_t>> &outputShapes() const;
//   std::vector<Tensor> infer(const float *input_f32, size_t numel);
//   const DeviceInfo &device() const;
//   double lastInferMs() const;
//
// It is a template over the caller's tensor / model-info / device-info types
// so that this header needs none of the reference's headers; inside the
// reference tree,
//
//   using CudaBackend = infvino_b200::CudaBackendT<infvino::Tensor, infvino::ModelInfo, infvino::DeviceInfo>;
//
// and InferenceEngine::device() (include/infvino/InferenceEngine.hpp:60)
// forwards backend_->device() unchanged.  `Tensor` needs `shape`
// (std::vector<int64_t>) and `data` (std::vector<float>); `ModelInfo` needs a
// `plan` string (and, when present, `device` is recorded as the request);
// DeviceInfo fields the type has (resolved, full_name, eu, clock_mhz,
// available, requested, opencl_version, fell_back_to_cpu) are filled from
// the CUDA device.  Errors are std::runtime_error with the reference's
// messages (src/ClBackend.cpp:15-18, :35-39); infer() is serialised by a
// mutex like ClBackend::infer (src/ClBackend.cpp:33).
//
// PlanModel: the executor surface the reference's tools bind
// (include/infvino/PlanModel.hpp:57-234): setInput / run / readOutput /
// readTensor / tensorNumel / input and output facts / pool statistics /
// lastRunMs / opProfile / profile() / clearProfile.
#ifndef INFVINO_B200_BACKEND_HPP_
#define INFVINO_B200_BACKEND_HPP_

#include <chrono>
#include <cstdint>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

#include "infvino_b200.h"

namespace infvino_b200 {

// The reference's DeviceInfo fields (include/infvino/Device.hpp:16-26), for
// callers that do not bring their own type, plus the CUDA ordinal.
struct DeviceInfo {
  std::vector<std::string> available;
  std::string requested;
  std::string resolved;
  std::string full_name;
  bool fell_back_to_cpu = false;
  std::string opencl_version;  // here: the CUDA runtime version
  unsigned eu = 0;             // multiprocessors
  unsigned clock_mhz = 0;
  int ordinal = 0;
};

namespace detail {
#define IVB_HAS_MEMBER(m)                                                                            \
  template <class T, class = void>                                                                   \
  struct has_##m : std::false_type {};                                                               \
  template <class T>                                                                                 \
  struct has_##m<T, std::void_t<decltype(std::declval<T &>().m)>> : std::true_type {};
IVB_HAS_MEMBER(available)
IVB_HAS_MEMBER(requested)
IVB_HAS_MEMBER(resolved)
IVB_HAS_MEMBER(full_name)
IVB_HAS_MEMBER(fell_back_to_cpu)
IVB_HAS_MEMBER(opencl_version)
IVB_HAS_MEMBER(eu)
IVB_HAS_MEMBER(clock_mhz)
IVB_HAS_MEMBER(ordinal)
IVB_HAS_MEMBER(device)
#undef IVB_HAS_MEMBER

// describeDevice (include/infvino/Device.hpp:30) for a CUDA device.
template <class DeviceInfoT>
DeviceInfoT describe_device(int ordinal, const std::string &requested) {
  DeviceInfoT d{};
  ivc_device_props p{};
  const bool ok = ivc_device_properties(ordinal, &p) == IVC_OK;
  const std::string name = ok ? std::string(p.name) : std::string("CUDA device ") + std::to_string(ordinal);
  if constexpr (has_available<DeviceInfoT>::value)
    for (int i = 0; i < p.device_count; ++i) {
      ivc_device_props q{};
      d.available.push_back(ivc_device_properties(i, &q) == IVC_OK ? std::string(q.name) : std::string("CUDA"));
    }
  if constexpr (has_requested<DeviceInfoT>::value) d.requested = requested;
  if constexpr (has_resolved<DeviceInfoT>::value) d.resolved = "CUDA:" + std::to_string(ordinal);
  if constexpr (has_full_name<DeviceInfoT>::value)
    d.full_name = name + (ok ? " (sm_" + std::to_string(p.cc_major) + std::to_string(p.cc_minor) + ")" : "");
  if constexpr (has_fell_back_to_cpu<DeviceInfoT>::value) d.fell_back_to_cpu = false;
  if constexpr (has_opencl_version<DeviceInfoT>::value)
    d.opencl_version = "CUDA " + std::to_string(p.runtime_version / 1000) + "." +
                       std::to_string(p.runtime_version % 1000 / 10);
  if constexpr (has_eu<DeviceInfoT>::value) d.eu = (unsigned)p.multiprocessors;
  if constexpr (has_clock_mhz<DeviceInfoT>::value) d.clock_mhz = (unsigned)p.clock_mhz;
  if constexpr (has_ordinal<DeviceInfoT>::value) d.ordinal = ordinal;
  return d;
}

template <class ModelInfoT>
std::string requested_device(const ModelInfoT &info) {
  if constexpr (has_device<ModelInfoT>::value)
    return std::string(info.device);
  else
    return "AUTO";
}
}  // namespace detail

// One pose detection of decodePose(): the reference's Detection for a pose
// model (include/infvino/Types.hpp:38-45: box, score, class 0, keypoints)
// without OpenCV types, plus the anchor it came from.
struct PoseDetection {
  int anchor = 0;
  float score = 0.f;
  float x = 0.f, y = 0.f, w = 0.f, h = 0.f;  // box in image coordinates
  std::vector<float> keypoints;             // x, y per keypoint
};

template <class TensorT, class ModelInfoT, class DeviceInfoT = DeviceInfo>
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
    device_ = detail::describe_device<DeviceInfoT>(device_ordinal, detail::requested_device(info));
  }
  ~CudaBackendT() { ivc_destroy(m_); }
  CudaBackendT(const CudaBackendT &) = delete;
  CudaBackendT &operator=(const CudaBackendT &) = delete;

  const std::vector<int64_t> &inputDims() const { return input_dims_; }
  const std::vector<std::vector<int64_t>> &outputShapes() const { return output_shapes_; }
  const DeviceInfoT &device() const { return device_; }
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

  // Preprocessor + infer in one call, the preprocessing on the device:
  // `batch` 8-bit BGR frames (height x width x 3, rows row_stride bytes
  // apart) in host memory -> outputs; `letterbox` (host, [batch][scale,
  // pad_left, pad_top]) receives the LetterboxInfo values.  cfg null: the
  // ultralytics defaults (letterbox, BGR -> RGB, /255).
  std::vector<TensorT> inferFrames(const uint8_t *frames, int batch, int height, int width, size_t row_stride,
                                   const ivc_preprocess *cfg = nullptr, float *letterbox = nullptr) {
    std::lock_guard<std::mutex> lock(mutex_);
    std::vector<TensorT> outs(output_shapes_.size());
    std::vector<float *> ptrs;
    for (size_t i = 0; i < outs.size(); ++i) {
      outs[i].shape = output_shapes_[i];
      if (batch != 1) outs[i].shape[0] = batch;
      outs[i].data.resize((size_t)ivc_output_numel(m_, (int)i) * (size_t)batch);
      ptrs.push_back(outs[i].data.data());
    }
    if (ivc_infer_bgr_u8(m_, frames, batch, height, width, row_stride, cfg, ptrs.data(), letterbox) != IVC_OK)
      throw std::runtime_error(ivc_last_error(m_));
    return outs;
  }

  // Pose decode + greedy NMS of the last infer() on the device, in place of
  // PoseDecoder::decode with nmsPerClass (src/Decoders.cpp:127-179, :33-65):
  // per image, the detections in the reference's order.  `letterbox` (host):
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
  DeviceInfoT device_;
  std::mutex mutex_;
};

// The executor itself (include/infvino/PlanModel.hpp:57-234), batch 1 as in
// the reference.  The OpenCL kernel directory and platform of the reference's
// constructor have no meaning here and are ignored.  With `profiling` every
// run() launches step by step with CUDA events around each launch, and
// opProfile() / profile() accumulate the times (one row per launch step; a
// fused step carries several plan nodes).
class PlanModel {
 public:
  struct PlanProfile {  // PlanModel.hpp:204-224
    struct NodeRow {
      int index = 0;
      std::string op;         // kernel family of the step
      std::string tag;        // the step (plan op and output tensor)
      std::string signature;  // the step's name (the tuning key of the reference has no counterpart)
      double ms = 0.0;
      int calls = 0;
    };
    std::vector<NodeRow> nodes;
    int plan_nodes = 0, dispatched_nodes = 0, skipped_nodes = 0, dispatches = 0;
    int reorder_calls = 0;
    double reorder_ms = 0.0;
    int fusions_res = 0, fusions_concat = 0;
    int fsv16_tensors = 0;  // channels-last (NHWC) tensors here
    size_t pool_requested = 0, pool_allocated = 0, pool_buffers = 0;
    double wall_ms = 0.0, busy_ms = 0.0, enqueue_ms = 0.0, sync_ms = 0.0;
  };

  explicit PlanModel(const std::string &plan_path, const std::string &kernel_dir = std::string(), int platform = -1,
                     int device_index = 0, bool profiling = false)
      : plan_path_(plan_path), profiling_(profiling) {
    (void)kernel_dir;
    (void)platform;
    if (ivc_create(plan_path.c_str(), device_index, 1, 0u, &m_) != IVC_OK)
      throw std::runtime_error(ivc_last_error(nullptr));
    const char *name = nullptr;
    ivc_input_name(m_, &name);
    input_name_ = name ? name : "";
    int rank = 0;
    int64_t d[16];
    ivc_input_dims(m_, d, 16, &rank);
    input_dims_.assign(d, d + rank);
    for (int i = 0; i < ivc_output_count(m_); ++i) {
      const char *on = nullptr;
      ivc_output_name(m_, i, &on);
      output_names_.emplace_back(on ? on : "");
      ivc_output_dims(m_, i, d, 16, &rank);
      output_dims_.emplace_back(d, d + rank);
    }
  }
  ~PlanModel() { ivc_destroy(m_); }
  PlanModel(const PlanModel &) = delete;
  PlanModel &operator=(const PlanModel &) = delete;

  const std::string &planPath() const { return plan_path_; }
  const std::string &inputName() const { return input_name_; }
  const std::vector<int64_t> &inputDims() const { return input_dims_; }
  size_t inputNumel() const { return (size_t)ivc_input_numel(m_); }
  size_t outputCount() const { return output_names_.size(); }
  const std::string &outputName(size_t i) const { return output_names_.at(i); }
  const std::vector<int64_t> &outputDims(size_t i) const { return output_dims_.at(i); }
  size_t outputNumel(size_t i) const { return (size_t)ivc_output_numel(m_, (int)i); }

  void setInput(const void *fp16_host) { ok(ivc_set_input_f16(m_, static_cast<const uint16_t *>(fp16_host), 1)); }

  void run() {
    const auto t0 = std::chrono::steady_clock::now();
    if (profiling_) {
      const int n = ivc_step_count(m_);
      std::vector<float> ms((size_t)n);
      ok(ivc_profile(m_, 1, ms.data(), n));
      for (int i = 0; i < n; ++i) {
        const char *name = nullptr, *family = nullptr;
        ivc_step_info(m_, i, &name, &family, nullptr, nullptr, nullptr);
        auto &acc = tprof_[name ? name : ""];
        acc.first += ms[(size_t)i];
        acc.second += 1;
      }
    } else {
      ok(ivc_run(m_, 1));
    }
    last_run_ms_ = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    wall_ms_ += last_run_ms_;
    ++runs_;
  }

  void readOutput(size_t i, void *fp16_host) { ok(ivc_read_output_f16(m_, (int)i, static_cast<uint16_t *>(fp16_host), 1)); }
  bool readTensor(const std::string &name, void *fp16_host) const {
    return ivc_read_tensor_f16(m_, name.c_str(), static_cast<uint16_t *>(fp16_host), 1) == IVC_OK;
  }
  size_t tensorNumel(const std::string &name) const { return (size_t)ivc_tensor_numel(m_, name.c_str()); }

  size_t poolRequestedBytes() const { return (size_t)stats().requested; }
  size_t poolAllocatedBytes() const { return (size_t)stats().arena; }
  size_t poolBufferCount() const { return (size_t)stats().roots; }

  double lastRunMs() const { return last_run_ms_; }
  const std::map<std::string, std::pair<double, int>> &opProfile() const { return tprof_; }
  double hostEnqueueMs() const { return 0.0; }
  double hostWaitMs() const { return 0.0; }

  PlanProfile profile() const {
    PlanProfile p;
    const int n = ivc_step_count(m_);
    for (int i = 0; i < n; ++i) {
      const char *name = nullptr, *family = nullptr;
      ivc_step_info(m_, i, &name, &family, nullptr, nullptr, nullptr);
      PlanProfile::NodeRow r;
      r.index = i;
      r.op = family ? family : "";
      r.tag = r.signature = name ? name : "";
      auto it = tprof_.find(r.tag);
      if (it != tprof_.end()) {
        r.ms = it->second.first;
        r.calls = it->second.second;
      }
      p.busy_ms += r.ms;
      p.dispatches += r.calls;
      p.nodes.push_back(std::move(r));
    }
    p.dispatched_nodes = n;
    const Stats s = stats();
    p.plan_nodes = n;
    p.fusions_res = s.fusions_res;
    p.fusions_concat = s.fusions_concat;
    p.fsv16_tensors = s.nhwc;
    p.pool_requested = (size_t)s.requested;
    p.pool_allocated = (size_t)s.arena;
    p.pool_buffers = (size_t)s.roots;
    p.wall_ms = wall_ms_;
    return p;
  }
  void clearProfile() {
    tprof_.clear();
    wall_ms_ = 0.0;
    runs_ = 0;
  }

  ivc_model *handle() const { return m_; }

 private:
  struct Stats {
    int64_t requested = 0, arena = 0, weights = 0;
    int roots = 0, views = 0, nhwc = 0, fusions_concat = 0, fusions_res = 0;
  };
  Stats stats() const {
    Stats s;
    ivc_pool_stats(m_, &s.requested, &s.arena, &s.weights, &s.roots, &s.views, &s.nhwc, &s.fusions_concat,
                   &s.fusions_res);
    return s;
  }
  void ok(int status) const {
    if (status != IVC_OK) throw std::runtime_error(ivc_last_error(m_));
  }

  ivc_model *m_ = nullptr;
  std::string plan_path_, input_name_;
  std::vector<int64_t> input_dims_;
  std::vector<std::string> output_names_;
  std::vector<std::vector<int64_t>> output_dims_;
  bool profiling_ = false;
  double last_run_ms_ = 0.0, wall_ms_ = 0.0;
  int runs_ = 0;
  std::map<std::string, std::pair<double, int>> tprof_;
};

}  // namespace infvino_b200

#endif  // INFVINO_B200_BACKEND_HPP_
