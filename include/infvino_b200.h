/*
 * infvino_b200 - C ABI of the B200 plan executor (drop-in for infvino's
 * OpenCL `PlanModel` / `ClBackend`).
 *
 * Plain C types only: handles are opaque pointers, tensors are raw pointers plus
 * element counts, CUDA streams are passed as `void *` (a cudaStream_t).  Every
 * call returns an ivc_status; the message of the last failure on a handle is
 * available from ivc_last_error().  Calls on one handle are serialised
 * internally (as `ClBackend::infer` is, src/ClBackend.cpp:33 in the reference).
 *
 * Batching: plans declare batch 1 (dim 0 of every activation).  A handle is
 * created for `max_batch` images; each call names the batch it processes and
 * every buffer holds `batch * numel` elements, image-major.
 *
 * Reference interfaces each entry point replaces (paths inside the reference):
 *   ivc_create ............ PlanModel::PlanModel  include/infvino/PlanModel.hpp:57-59
 *                            ClBackend::ClBackend  include/infvino/ClBackend.hpp:32
 *   ivc_input_* / output_*  PlanModel::inputName/inputDims/inputNumel/outputCount/
 *                            outputName/outputDims/outputNumel  PlanModel.hpp:64-73
 *   ivc_tensor_numel ....... PlanModel::tensorNumel  PlanModel.hpp:85-86
 *   ivc_infer_f32 .......... ClBackend::infer(const float*, size_t)  ClBackend.hpp:38-39
 *   ivc_set_input_f16 ...... PlanModel::setInput(const void*)  PlanModel.hpp:75-76
 *   ivc_run ................ PlanModel::run()  PlanModel.hpp:77-78
 *   ivc_run_async .......... PlanModel::run() without the final finish (PlanModel.cpp:4175)
 *   ivc_read_output_f16 .... PlanModel::readOutput(size_t, void*)  PlanModel.hpp:79-80
 *   ivc_read_tensor_f16 .... PlanModel::readTensor(name, void*)  PlanModel.hpp:82-84
 *   ivc_last_infer_ms ...... ClBackend::lastInferMs / PlanModel::lastRunMs
 *                            ClBackend.hpp:41, PlanModel.hpp:190-191
 *   ivc_profile / ivc_step_* PlanModel::profile() / PlanProfile  PlanModel.hpp:204-224
 *   ivc_pool_stats ......... PlanModel::poolRequestedBytes/poolAllocatedBytes/
 *                            poolBufferCount  PlanModel.hpp:94-97
 *   ivc_infer_f16_device ... (new) zero-copy device-pointer inference on a caller stream
 *   ivc_set_input_bgr_u8 / ivc_infer_bgr_u8
 *                            Preprocessor::operator() src/Preprocess.cpp:13-77 (+ ClBackend::infer), on the device
 *   ivc_decode_pose ........ PoseDecoder::decode + nmsPerClass + nms, on the device
 *                            src/Decoders.cpp:33-65,127-179, src/Nms.cpp:10-55
 *   ivc_destroy ............ PlanModel::~PlanModel / ClBackend destructor
 */
#ifndef INFVINO_B200_H_
#define INFVINO_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ivc_model ivc_model;

typedef enum ivc_status {
  IVC_OK = 0,
  IVC_ERR_ARGUMENT = 1,   /* bad pointer / index / batch */
  IVC_ERR_PLAN = 2,       /* plan parse, missing init, unknown op (reference: std::runtime_error) */
  IVC_ERR_CUDA = 3,       /* CUDA runtime / device failure */
  IVC_ERR_NUMEL = 4,      /* input element count does not match the plan */
  IVC_ERR_KERNEL = 5,     /* a kernel reported a bounded-wait timeout (status word) */
  IVC_ERR_NOT_FOUND = 6   /* unknown tensor name */
} ivc_status;

/* creation flags */
#define IVC_FLAG_NO_GRAPH 0x1u        /* eager launches instead of CUDA graph replay */
#define IVC_FLAG_NO_FUSION 0x2u       /* skip concat->conv1x1 / residual load-time rewrites */
#define IVC_FLAG_DRY_RUN 0x4u         /* host only: parse, layout, allocate; no GPU is touched */
#define IVC_FLAG_NO_TENSOR_CORES 0x8u /* convolutions on the CUDA-core direct kernel (diagnostic) */
#define IVC_FLAG_NO_POOL 0x10u        /* no activation memory reuse, every tensor stays readable
                                         (reference INFVINO_NO_POOL, src/PlanModel.cpp:887) */
#define IVC_FLAG_NO_HALO 0x20u        /* diagnostic: 3x3 stride-1 convolutions load one box per tap
                                         instead of one halo box per channel chunk */
#define IVC_FLAG_NO_PDL 0x40u         /* diagnostic: kernels launched without programmatic dependent
                                         launch (each waits for the previous grid to finish) */
#define IVC_FLAG_NO_JIT 0x80u         /* diagnostic: the fused decode tail runs on the interpreting
                                         kernel instead of its load-time compiled (NVRTC) form */
#define IVC_FLAG_NO_TUNE 0x100u       /* convolution tile geometry from the cost model alone (no timing
                                         of candidate geometries at the first run of a batch size) */
#define IVC_FLAG_SERIAL 0x200u        /* every step on one stream: the captured graph has no concurrent
                                         branches (and activations may share more memory) */

/* Loads `plan_path` (+ its init_*.bin files) onto CUDA device `device_ordinal`. */
int ivc_create(const char *plan_path, int device_ordinal, int max_batch, unsigned flags, ivc_model **out);
void ivc_destroy(ivc_model *m);
/* Message of the last failed call on `m`; with m == NULL, of the last failed ivc_create. */
const char *ivc_last_error(const ivc_model *m);

int ivc_input_name(const ivc_model *m, const char **name);
int ivc_input_dims(const ivc_model *m, int64_t *dims, int max_rank, int *rank);
int64_t ivc_input_numel(const ivc_model *m);
int ivc_output_count(const ivc_model *m);
int ivc_output_name(const ivc_model *m, int i, const char **name);
int ivc_output_dims(const ivc_model *m, int i, int64_t *dims, int max_rank, int *rank);
int64_t ivc_output_numel(const ivc_model *m, int i);
/* per-image element count of any declared tensor, 0 if unknown */
int64_t ivc_tensor_numel(const ivc_model *m, const char *name);
int ivc_max_batch(const ivc_model *m);

/* ClBackend::infer: `input` holds batch*input_numel f32 values (host memory,
 * pinned or pageable); converted to fp16 with the reference's truncating cast,
 * run, and every output written as f32 to outputs[i] (batch*output_numel(i)
 * values, host memory).  Synchronous.  Batches of 32 or more are pipelined in
 * chunks, and half of their images are cast on the host by a process-wide
 * pool of worker threads (one per CPU of the process's affinity mask, up to
 * 16, created at the first such call), so that fewer bytes cross PCIe; the
 * first call also pins two chunk buffers. */
int ivc_infer_f32(ivc_model *m, const float *input, size_t numel, int batch, float *const *outputs);

/* PlanModel-style split calls (fp16 host buffers, synchronous). */
int ivc_set_input_f16(ivc_model *m, const uint16_t *input_f16, int batch);
int ivc_run(ivc_model *m, int batch);
/* PlanModel::run without the host wait: enqueues the network for the input set
 * last, on `stream` (NULL = the handle's stream). */
int ivc_run_async(ivc_model *m, int batch, void *stream);
int ivc_read_output_f16(ivc_model *m, int i, uint16_t *dst, int batch);
/* Copies tensor `name` for `batch` images in plan (NCHW) order; IVC_ERR_NOT_FOUND if unknown. */
int ivc_read_tensor_f16(ivc_model *m, const char *name, uint16_t *dst, int batch);

/* Image preprocessing on the device (replaces the host-side
 * Preprocessor::operator(), src/Preprocess.cpp:13-77, and the truncating cast
 * of ClBackend::infer).  Settings as infvino::PreprocessConfig
 * (include/infvino/Preprocess.hpp:40-48); the input size is the plan's input. */
typedef struct ivc_preprocess {
  int letterbox;        /* 1: keep the aspect ratio and pad with 114 (the default); 0: plain resize */
  int to_rgb;           /* 1: BGR -> RGB (the default) */
  int normalize;        /* 1: x 1/255 (the default) */
  int n_mean, n_std;    /* entries of mean / std in use (0: none), applied after /255 */
  float mean[3], std[3];
} ivc_preprocess;

/* `batch` 8-bit BGR frames (height x width x 3, rows `row_stride` bytes apart,
 * frames height * row_stride bytes apart) in host memory (pinned or pageable),
 * or in device memory when frames_on_device is nonzero, become the network
 * input: letterbox + cv::resize INTER_LINEAR (OpenCV's 8-bit arithmetic,
 * bit-exact) + 114 border + blobFromImage + mean / std + the reference's
 * truncating f32 -> f16 cast, in one kernel.  cfg NULL: the defaults above.
 * letterbox (host, [batch][scale, pad_left, pad_top]) or NULL receives what
 * Preprocessor reports in LetterboxInfo.  Synchronous. */
int ivc_set_input_bgr_u8(ivc_model *m, const uint8_t *frames, int batch, int height, int width, size_t row_stride,
                         int frames_on_device, const ivc_preprocess *cfg, float *letterbox);
/* End to end from 8-bit BGR frames in host memory to f32 outputs in host
 * memory (Preprocessor + ClBackend::infer in one call): large batches are
 * pipelined in chunks (frames copied in, preprocessed, run, results copied
 * out, overlapped).  Synchronous. */
int ivc_infer_bgr_u8(ivc_model *m, const uint8_t *frames, int batch, int height, int width, size_t row_stride,
                     const ivc_preprocess *cfg, float *const *outputs, float *letterbox);

/* Pose decode + greedy NMS of output 0 of the last run, on the device, for
 * `batch` images (replaces the host-side PoseDecoder::decode with
 * nmsPerClass, src/Decoders.cpp:127-179 and :33-65, and nms / iou,
 * src/Nms.cpp:10-55).  Candidates are anchors whose score is not below
 * `conf`; boxes and keypoints are mapped through the letterbox
 * (include/infvino/Preprocess.hpp:24-35; `letterbox` is [batch][scale,
 * pad_left, pad_top] in host memory, or NULL for scale 1 and no padding);
 * greedy suppression at IoU above `iou` in descending score (ties by anchor
 * index, the reference's stable sort); the keep list is then re-sorted by
 * score with std::sort and cut at `max_det`, as the reference does, so equal
 * scores come out in the order that (unstable) sort leaves them.  Results in
 * host memory:
 * counts[b] detections for image b, detection k at
 * dets[(b * max_det + k) * (6 + 2 * nk)]: anchor index, score, x, y, w, h,
 * then x, y of each keypoint.  nk <= 0 infers the keypoint count from the
 * output's channels as (C - 5) / kdims (kdims <= 0: 3).  The output must be
 * channel-major [1, 5 + nk * kdims, A] with A <= 16384.  Synchronous. */
int ivc_decode_pose(ivc_model *m, int batch, float conf, float iou, int max_det, int nk, int kdims,
                    const float *letterbox, int *counts, float *dets);
/* ivc_read_tensor_f16 without any allocation (no counterpart in the reference).
 * The NHWC -> NCHW relayout is staged through a static 4 MiB device buffer per
 * device instead of a scratch buffer grown with cudaMalloc; a tensor that needs
 * more than 4 MiB for `batch` images fails with IVC_ERR_ARGUMENT.  For callers
 * that must not allocate or free device memory after set-up: a process whose
 * device memory is owned by another allocator, or a diagnostic read inside a
 * latency-critical loop (cudaFree synchronises the whole device).  Make the
 * first call on each device before any stream capture (it resolves the
 * buffer's address, which may load the module).  Overlapping calls on one
 * device (from any handle) share the buffer and race. */
int ivc_read_tensor_f16_noalloc(ivc_model *m, const char *name, uint16_t *dst, int batch);

/* Zero-copy: device fp16 input / outputs, enqueued on `stream` (cudaStream_t,
 * NULL = the handle's stream) without host synchronisation. */
int ivc_infer_f16_device(ivc_model *m, const void *d_input, int batch, void *const *d_outputs, void *stream);
/* Device f32 input (truncating cast on the device) -> device f32 outputs, asynchronous. */
int ivc_infer_f32_device(ivc_model *m, const float *d_input, int batch, float *const *d_outputs, void *stream);
/* Binds the handle to a caller stream (NULL restores a private stream). */
int ivc_set_stream(ivc_model *m, void *stream);
int ivc_synchronize(ivc_model *m);
double ivc_last_infer_ms(const ivc_model *m);

/* Profiling: eager run with CUDA events around every kernel launch. */
int ivc_step_count(const ivc_model *m);
int ivc_step_info(const ivc_model *m, int i, const char **name, const char **family, double *flops_per_image,
                  double *act_bytes_per_image, double *fixed_bytes);
int ivc_profile(ivc_model *m, int batch, float *step_ms, int n);
/* Number of kernel launches one ivc_run(batch) performs (kernel nodes of its CUDA graph). */
int ivc_launch_count(ivc_model *m, int batch, int *count);

/* Diagnostic (no counterpart in the reference): settings of the convolution
 * kernels' bounded waits.  `limit_cycles` is the limit of every working wait
 * in SM clocks (the default is about 2 s); with `probe` nonzero each conv CTA
 * first waits on a barrier that nothing arrives on, so that wait runs out, the
 * kernel drains its copies and MMAs, releases TMEM and reports its status, and
 * the next synchronising call returns IVC_ERR_KERNEL.  Lets a test exercise the
 * timeout path without any GPU fault; the handle stays usable.  Takes effect
 * from the next run (captured graphs are captured again). */
int ivc_debug_conv_wait(ivc_model *m, long long limit_cycles, int probe);

/* Activation pool statistics (bytes at max_batch). */
int ivc_pool_stats(const ivc_model *m, int64_t *requested_bytes, int64_t *arena_bytes, int64_t *weight_bytes,
                   int *roots, int *views, int *nhwc_tensors, int *fusions_concat, int *fusions_res);
/* Human-readable dump of tensors (layout, arena offset, lifetime) and launches. */
int ivc_describe(const ivc_model *m, char *buf, size_t cap);

/* Properties of CUDA device `device_ordinal`, for the reference's DeviceInfo
 * (include/infvino/Device.hpp:16-26, describeDevice): name, multiprocessor
 * count (DeviceInfo::eu), clock (DeviceInfo::clock_mhz), compute capability,
 * memory, and the number of devices (DeviceInfo::available). */
typedef struct ivc_device_props {
  char name[256];
  int multiprocessors;
  int clock_mhz;
  int cc_major, cc_minor;
  int64_t total_mem_bytes;
  int device_count;
  int runtime_version;  /* CUDA runtime, e.g. 12090 */
} ivc_device_props;
int ivc_device_properties(int device_ordinal, ivc_device_props *out);

/* Host conversions with the reference's semantics (include/infvino/Half.hpp:14-49). */
void ivc_f32_to_f16(const float *in, uint16_t *out, size_t n);
void ivc_f16_to_f32(const uint16_t *in, float *out, size_t n);

#ifdef __cplusplus
}
#endif

#endif /* INFVINO_B200_H_ */
