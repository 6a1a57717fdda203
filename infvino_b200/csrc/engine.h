// CudaPlanModel engine: one plan, one device, batch 1..max_batch.
//
// Load: parse -> layout planning (NHWC for convolution-region 4-D tensors,
// planar NCHW elsewhere) -> load-time fusions -> liveness arena allocation ->
// lowering of every node to a kernel launch with all weights repacked and
// resident.  Run: the lowered launch list is captured once per batch size into
// a CUDA graph and replayed.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "kernels/ops.cuh"
#include "plan.h"

namespace ivb {

enum EngineFlags : unsigned {
  kFlagNoGraph = 1u << 0,     // eager launches instead of CUDA graph replay
  kFlagNoFusion = 1u << 1,    // skip the concat->conv1x1 and residual rewrites
  kFlagDryRun = 1u << 2,      // host-only: plan, layout, allocation; no device work
  kFlagNoTensorCores = 1u << 3,  // route convolutions to the CUDA-core direct kernel
  kFlagNoPool = 1u << 4,      // every tensor keeps its own storage (reference INFVINO_NO_POOL)
  kFlagNoHalo = 1u << 5,      // 3x3 convs with per-tap boxes instead of the halo tile
  kFlagNoPdl = 1u << 6,       // launches without programmatic dependent launch
  kFlagNoJit = 1u << 7,       // fused tail on the interpreting kernel instead of load-time compiled code
  kFlagNoTune = 1u << 8,      // convolution tile geometry from the cost model, no timing at load
  kFlagSerial = 1u << 9,      // every step on one stream (no concurrent branches in the graph)
};

struct TensorRt {
  std::string name;
  std::vector<int64_t> dims;
  int64_t numel = 0;            // per image
  bool is_init = false, is_input = false, is_output = false;
  bool nhwc = false;            // channels-last storage (4-D only)
  bool dense = true;            // contiguous per image in plan (row-major) order
  int root = -1;                // storage owner (self when it owns storage)
  int64_t elem_off = 0;         // element offset inside the root's storage
  int C = 0, H = 0, W = 0;      // 4-D view geometry (rank-4 tensors)
  int Cs = 0;                   // NHWC channel stride of the storage
  int64_t sb = 0, sc = 0, sy = 0, sx = 0;  // per-image element strides
  int64_t bytes_per_img = 0;    // roots only
  int64_t arena_off = -1;       // roots only, bytes
  int birth = -1, death = -1;   // roots only, node indices
  bool materialized = true;     // roots only: some step reads or writes it in memory
  __half *dptr = nullptr;       // element (image 0, offset) on the device
};

struct Step {
  std::string name;             // node op + output tensor
  std::string family;           // kernel family (profiling key)
  int node = -1;
  double flops_img = 0.0;       // algorithmic FLOPs per image (2 * MACs)
  double bytes_img = 0.0;       // algorithmic activation bytes per image (inputs + outputs, once)
  double bytes_fixed = 0.0;     // weights / constants, read once per launch
  std::function<cudaError_t(int, cudaStream_t)> launch;
  // launch geometry per batch size, recorded at the first launch (tensor-core convs)
  std::shared_ptr<std::map<int, std::string>> geometry;
  std::string info;  // load-time facts about the step (describe())
  // optional load-time tuning, run once per batch size before the first launch
  std::function<void(int, cudaStream_t)> tune;
  std::vector<int> nodes;  // plan nodes this step carries out (its own and the ones fused into it)
};

// Preprocessor settings (include/infvino/Preprocess.hpp:40-48 PreprocessConfig;
// the input size is the plan's input).
struct PreprocessCfg {
  int letterbox = 1;   // letterbox (aspect kept, 114 border) or plain resize
  int to_rgb = 1;      // BGR -> RGB
  int normalize = 1;   // x 1/255
  int n_mean = 0, n_std = 0;
  float mean[3] = {0.f, 0.f, 0.f}, std[3] = {1.f, 1.f, 1.f};
};

struct EngineStats {
  int64_t requested_bytes = 0;  // sum of per-tensor storage at max_batch
  int64_t arena_bytes = 0;      // liveness-packed arena
  int64_t weight_bytes = 0;
  int roots = 0, views = 0, nhwc_tensors = 0, steps = 0;
  int fusions_concat = 0, fusions_res = 0;
  int overlap_errors = 0;       // allocator self-check (must be 0)
};

class Engine {
 public:
  Engine(const std::string &plan_path, int device, int max_batch, unsigned flags);
  ~Engine();
  Engine(const Engine &) = delete;
  Engine &operator=(const Engine &) = delete;

  // ---- plan facts
  const std::string &input_name() const { return plan_->input(); }
  const std::vector<int64_t> &input_dims() const;
  int64_t input_numel() const;
  int output_count() const { return (int)plan_->outputs().size(); }
  const std::string &output_name(int i) const { return plan_->outputs().at((size_t)i); }
  const std::vector<int64_t> &output_dims(int i) const;
  int64_t output_numel(int i) const;
  int64_t tensor_numel(const std::string &name) const;
  int max_batch() const { return max_batch_; }
  int device() const { return device_; }
  const EngineStats &stats() const { return stats_; }
  const std::vector<Step> &steps() const { return steps_; }
  std::string describe() const;  // one line per tensor / step (diagnostics)

  // ---- execution (asynchronous on the engine stream unless stated)
  void set_stream(cudaStream_t s);
  cudaStream_t stream() const { return stream_; }
  void upload_input_f16(const void *src, int batch, bool src_on_device);
  void upload_input_f32(const float *src, int batch, bool src_on_device);  // reference truncating cast
  void run(int batch);
  void run_profiled(int batch, std::vector<float> *step_ms);  // eager, events around each step
  void download_output_f16(int i, void *dst, int batch, bool dst_on_device);
  void download_output_f32(int i, float *dst, int batch, bool dst_on_device);
  // ClBackend::infer for host buffers: chunks of the batch are copied in,
  // converted, run and copied out on separate streams so that the host copies
  // of one chunk overlap the network on another (same results as one batch).
  void infer_f32_host(const float *src, int batch, float *const *outs);
  // Device preprocessing of `batch` 8-bit BGR frames (HWC, rows `row_stride`
  // bytes apart, frames h * row_stride bytes apart) into the network input:
  // Preprocessor::operator() + the truncating cast, on the device.  Frames in
  // host (pinned or pageable) or device memory.  letterbox_out: [batch][scale,
  // pad_left, pad_top] (host) or null.  Asynchronous on the engine stream.
  void upload_input_bgr_u8(const uint8_t *frames, int batch, int h, int w, int64_t row_stride, bool on_device,
                           const PreprocessCfg &cfg, float *letterbox_out);
  // End to end from 8-bit frames in host memory: chunks of frames copied in,
  // preprocessed, run and their f32 outputs copied out, overlapped.  Synchronous.
  void infer_bgr_u8_host(const uint8_t *frames, int batch, int h, int w, int64_t row_stride, const PreprocessCfg &cfg,
                         float *const *outs, float *letterbox_out);
  // infer_f32_host for pageable caller memory: every image cast on the host
  // into pinned chunks, results staged through pinned chunks (same results).
  void infer_f32_host_staged(const float *src, int batch, float *const *outs);
  // Plan-order (NCHW) copy of any tensor for `batch` images into host memory.
  bool read_tensor_f16(const std::string &name, void *host_dst, int batch);
  // read_tensor_f16 staged through caller-provided device scratch (allocates
  // nothing).  Returns 0 (copied), 1 (unknown tensor) or 2 (scratch too small;
  // *need_bytes says how much the relayout needs).
  int read_tensor_f16_staged(const std::string &name, void *host_dst, int batch, void *scratch,
                             int64_t scratch_bytes, int64_t *need_bytes);
  void synchronize();
  int device_status();  // kernel status word (0 = ok), resets it
  // Pose decode + NMS of output 0 of the last run on the device (reference
  // PoseDecoder::decode + nmsPerClass): per image, counts[b] detections of
  // 6 + 2 * nk floats each (anchor, score, x, y, w, h, keypoint x/y pairs) at
  // dets + b * max_det * (6 + 2 * nk), in host memory.  `letterbox` (host,
  // [batch][scale, pad_left, pad_top]) may be null.  nk <= 0: inferred from
  // the output's channels as (C - 5) / kdims.  Synchronous.
  void decode_pose(int batch, float conf, float iou, int max_det, int nk, int kdims, const float *letterbox,
                   int *counts, float *dets);
  int graph_kernel_count(int batch);  // kernel nodes in the CUDA graph of `batch`
  void require_device() const;  // throws for a dry run handle (no device state)
  // Test settings of the convolutions' bounded waits: the limit of every
  // working wait in SM clocks, and a probe that makes the first wait of every
  // conv CTA run out (the kernel then reports a timeout status).  Takes effect
  // from the next run (captured graphs are dropped).
  void set_conv_wait(long long limit_cycles, int probe);
  __half *input_device_ptr() const;
  float *input_f32_staging() const { return in_f32_; }

 private:
  void plan_layouts();
  void build_tensors();
  void lifetimes();       // node-order birth / death of every root (fusion checks)
  void alloc_aux();       // status word and f32 input staging
  void allocate();        // arena placement over the step DAG, then device pointers
  void upload_weights();
  void lower();
  void plan_streams();    // step dependencies, stream assignment, reachability
  void check(cudaError_t e, const char *what) const;
  int tid(const std::string &name) const;
  View4 view(int t) const;                 // image-0 view with per-image strides
  void capture(int batch);

  std::unique_ptr<Plan> plan_;
  int device_ = 0;
  int max_batch_ = 1;
  unsigned flags_ = 0;
  bool dry_ = false;
  int num_sms_ = 148;

  std::vector<TensorRt> T_;
  std::map<std::string, int> tid_;
  std::set<std::string> nhwc_names_;
  std::map<int, std::pair<int, int>> folded_transpose_;  // permute output -> (its source, the permute node)
  std::set<int> elided_nodes_;       // concat4 nodes whose sources write in place
  std::map<int, Step> tail_steps_;   // fused planar tails, keyed by the node whose place they take
  std::vector<std::pair<int, int>> tail_uses_;  // (tensor, node) reads of fused tails, for liveness
  void plan_tails();
  void pdl_scope() const;  // launches on this thread follow kFlagNoPdl
  void tune(int batch);    // per-step load-time tuning for this batch size (once)
  std::set<int> tuned_;
  std::vector<Step> steps_;
  // concurrency: steps run on up to kMaxStreams streams inside the captured
  // graph; a step waits for the latest step it depends on in every other stream
  static constexpr int kMaxStreams = 4;
  std::vector<std::vector<int>> step_reads_, step_writes_;  // roots
  std::vector<int> stream_of_;                              // per step
  std::vector<std::vector<int>> waits_;                     // per step: steps on other streams
  std::vector<char> signals_;                               // per step: another stream waits for it
  std::vector<std::vector<uint64_t>> reach_;                // step i reaches step j (bitset rows)
  int n_streams_ = 1;
  cudaStream_t side_[kMaxStreams] = {};
  std::vector<cudaEvent_t> step_events_;
  cudaEvent_t fork_event_ = nullptr, join_events_[kMaxStreams] = {};
  EngineStats stats_;

  cudaStream_t stream_ = nullptr;
  bool own_stream_ = false;
  uint8_t *arena_ = nullptr;
  int64_t arena_bytes_ = 0;
  std::vector<void *> dev_allocs_;  // weights and packed weights
  int *status_ = nullptr;           // device status word
  float *in_f32_ = nullptr;         // device staging for f32 input
  float *out_f32_ = nullptr;        // device staging for f32 outputs (pipelined infer)
  uint16_t *in_f16_host_ = nullptr; // pinned fp16 input, two chunks (pipelined infer)
  struct SplitTune {                // host/device cast split of infer_f32, per batch size
    int calls = 0;                  // calls so far
    int best = -1;                  // index of the chosen split, once tuned
    double ms[5] = {0, 0, 0, 0, 0}; // fastest call per candidate split
  };
  std::map<int, SplitTune> split_tune_;
  float *out_host_ = nullptr;       // pinned f32 outputs, two chunks (pageable callers)
  int last_f32_batch_ = 0;          // images of the last chunked infer whose outputs are all in out_f32_
  // device preprocessing: OpenCV coordinate tables of the last frame size, frame staging
  struct LetterboxTables {
    int h = 0, w = 0, letterbox = -1;
    int rw = 0, rh = 0, pad_left = 0, pad_top = 0;
    float scale = 1.f;
    int4 *xtab = nullptr, *ytab = nullptr;
  };
  LetterboxTables lbt_;
  uint8_t *frames_dev_ = nullptr;
  int64_t frames_cap_ = 0;          // bytes
  void letterbox_tables(int h, int w, int letterbox);
  void launch_letterbox(const uint8_t *dframes, int64_t img_bytes, int64_t row_stride, int first, int n,
                        const PreprocessCfg &cfg, cudaStream_t st);
  // pose decode + NMS: box scratch, results and letterboxes (allocated at the first call)
  float4 *nms_boxes_ = nullptr;
  int *nms_counts_ = nullptr, *nms_kept_ = nullptr;
  int2 *nms_pairs_ = nullptr;       // keep lists (anchor, score) per image
  int2 *nms_pairs_host_ = nullptr;  // their pinned staging
  int *nms_chosen_ = nullptr;       // chosen anchors [batch][max_det], then their counts
  int64_t nms_idx_cap_ = 0;         // ints in nms_chosen_
  float *nms_dets_ = nullptr, *nms_lbox_ = nullptr;
  int64_t nms_dets_cap_ = 0;        // floats in nms_dets_
  float *nms_host_ = nullptr;       // pinned staging of results and counts
  int64_t nms_host_cap_ = 0;        // floats in nms_host_
  cudaStream_t copy_in_ = nullptr, copy_out_ = nullptr;
  std::vector<cudaEvent_t> chunk_events_;
  __half *scratch_ = nullptr;       // read_tensor staging
  int64_t scratch_elems_ = 0;
  std::map<int, cudaGraphExec_t> graphs_;
  struct ConvWait {
    long long limit = 4000000000LL;  // kConvWaitLimitDefault
    int probe = 0;
  };
  std::shared_ptr<ConvWait> wait_ = std::make_shared<ConvWait>();  // read by the conv launch closures
};

}  // namespace ivb
