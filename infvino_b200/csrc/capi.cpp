// C ABI over the engine (include/infvino_b200.h).  Exceptions never cross the
// boundary: every entry point maps them to an ivc_status and keeps the message.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/infvino_b200.h"
#include "engine.h"
#include "host_cast.h"

struct ivc_model {
  std::unique_ptr<ivb::Engine> eng;
  mutable std::mutex mu;
  std::string err;
  double last_ms = 0.0;
  std::string describe_cache;
};

namespace {

std::string g_create_err;
std::mutex g_create_mu;

int fail(ivc_model *m, int code, const std::string &msg) {
  if (m) m->err = msg;
  return code;
}

int classify(const std::string &msg) {
  if (msg.find("numel mismatch") != std::string::npos) return IVC_ERR_NUMEL;
  if (msg.find("PlanModel:") == 0) return IVC_ERR_PLAN;
  if (msg.find("CudaPlanModel: cuda") != std::string::npos) return IVC_ERR_CUDA;
  return msg.find("CudaPlanModel:") == 0 && msg.find(": ") != std::string::npos &&
                 (msg.find("cuda") != std::string::npos || msg.find("launch") != std::string::npos)
             ? IVC_ERR_CUDA
             : IVC_ERR_PLAN;
}

template <class F>
int guarded(ivc_model *m, F &&f) {
  if (!m || !m->eng) return IVC_ERR_ARGUMENT;
  std::lock_guard<std::mutex> lk(m->mu);
  try {
    return f();
  } catch (const std::exception &e) {
    return fail(m, classify(e.what()), e.what());
  }
}

int status_check(ivc_model *m) {
  const int s = m->eng->device_status();
  if (s != 0) return fail(m, IVC_ERR_KERNEL, "CudaPlanModel: kernel bounded wait timed out (status " + std::to_string(s) + ")");
  return IVC_OK;
}

// include/infvino/Half.hpp:14-24 (truncating) and :26-47 (exact widening)
inline float h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu, mant = h & 0x3ffu, f;
  if (e == 0) {
    if (mant == 0) {
      f = sign;
    } else {
      int ee = 113;
      while (!(mant & 0x400u)) {
        mant <<= 1;
        --ee;
      }
      f = sign | ((uint32_t)ee << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (e == 31) {
    f = sign | 0x7f800000u | (mant << 13);
  } else {
    f = sign | ((e + 112u) << 23) | (mant << 13);
  }
  float out;
  std::memcpy(&out, &f, 4);
  return out;
}

template <class F>
void parallel_for(size_t n, F &&f) {
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t nt = n < (1u << 20) ? 1 : std::min<size_t>(hw, 16);
  if (nt <= 1) {
    f(0, n);
    return;
  }
  std::vector<std::thread> th;
  const size_t chunk = (n + nt - 1) / nt;
  for (size_t t = 0; t < nt; ++t) {
    const size_t b = t * chunk, e = std::min(n, b + chunk);
    if (b < e) th.emplace_back([&f, b, e] { f(b, e); });
  }
  for (auto &x : th) x.join();
}

}  // namespace

extern "C" {

int ivc_create(const char *plan_path, int device_ordinal, int max_batch, unsigned flags, ivc_model **out) {
  if (!out) return IVC_ERR_ARGUMENT;
  *out = nullptr;
  if (!plan_path || !*plan_path) {
    std::lock_guard<std::mutex> lk(g_create_mu);
    g_create_err = "ClBackend: ModelInfo.plan is empty";
    return IVC_ERR_ARGUMENT;
  }
  try {
    auto m = std::make_unique<ivc_model>();
    m->eng = std::make_unique<ivb::Engine>(plan_path, device_ordinal, max_batch, flags);
    *out = m.release();
    return IVC_OK;
  } catch (const std::exception &e) {
    std::lock_guard<std::mutex> lk(g_create_mu);
    g_create_err = e.what();
    return classify(e.what());
  }
}

void ivc_destroy(ivc_model *m) { delete m; }

const char *ivc_last_error(const ivc_model *m) {
  if (!m) {
    std::lock_guard<std::mutex> lk(g_create_mu);
    return g_create_err.c_str();
  }
  return m->err.c_str();
}

int ivc_input_name(const ivc_model *m, const char **name) {
  if (!m || !name) return IVC_ERR_ARGUMENT;
  *name = m->eng->input_name().c_str();
  return IVC_OK;
}

int ivc_input_dims(const ivc_model *m, int64_t *dims, int max_rank, int *rank) {
  if (!m) return IVC_ERR_ARGUMENT;
  const auto &d = m->eng->input_dims();
  if (rank) *rank = (int)d.size();
  for (int i = 0; dims && i < (int)d.size() && i < max_rank; ++i) dims[i] = d[(size_t)i];
  return IVC_OK;
}

int64_t ivc_input_numel(const ivc_model *m) { return m ? m->eng->input_numel() : 0; }
int ivc_output_count(const ivc_model *m) { return m ? m->eng->output_count() : 0; }

int ivc_output_name(const ivc_model *m, int i, const char **name) {
  if (!m || !name || i < 0 || i >= m->eng->output_count()) return IVC_ERR_ARGUMENT;
  *name = m->eng->output_name(i).c_str();
  return IVC_OK;
}

int ivc_output_dims(const ivc_model *m, int i, int64_t *dims, int max_rank, int *rank) {
  if (!m || i < 0 || i >= m->eng->output_count()) return IVC_ERR_ARGUMENT;
  const auto &d = m->eng->output_dims(i);
  if (rank) *rank = (int)d.size();
  for (int k = 0; dims && k < (int)d.size() && k < max_rank; ++k) dims[k] = d[(size_t)k];
  return IVC_OK;
}

int64_t ivc_output_numel(const ivc_model *m, int i) {
  if (!m || i < 0 || i >= m->eng->output_count()) return 0;
  return m->eng->output_numel(i);
}

int64_t ivc_tensor_numel(const ivc_model *m, const char *name) {
  if (!m || !name) return 0;
  return m->eng->tensor_numel(name);
}

int ivc_max_batch(const ivc_model *m) { return m ? m->eng->max_batch() : 0; }

int ivc_infer_f32(ivc_model *m, const float *input, size_t numel, int batch, float *const *outputs) {
  return guarded(m, [&]() -> int {
    if (!input || !outputs || batch < 1 || batch > m->eng->max_batch())
      return fail(m, IVC_ERR_ARGUMENT, "ivc_infer_f32: bad arguments");
    const size_t expect = (size_t)m->eng->input_numel() * (size_t)batch;
    if (numel != expect)
      return fail(m, IVC_ERR_NUMEL,
                  "ClBackend: input numel mismatch: got " + std::to_string(numel) + ", expected " + std::to_string(expect));
    for (int i = 0; i < m->eng->output_count(); ++i)
      if (!outputs[i]) return fail(m, IVC_ERR_ARGUMENT, "ivc_infer_f32: null output buffer");
    const auto t0 = std::chrono::steady_clock::now();
    m->eng->infer_f32_host(input, batch, outputs);
    m->last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return status_check(m);
  });
}

int ivc_set_input_f16(ivc_model *m, const uint16_t *input_f16, int batch) {
  return guarded(m, [&]() -> int {
    if (!input_f16 || batch < 1 || batch > m->eng->max_batch()) return fail(m, IVC_ERR_ARGUMENT, "bad arguments");
    m->eng->upload_input_f16(input_f16, batch, false);
    m->eng->synchronize();
    return IVC_OK;
  });
}

int ivc_run(ivc_model *m, int batch) {
  return guarded(m, [&]() -> int {
    if (batch < 1 || batch > m->eng->max_batch()) return fail(m, IVC_ERR_ARGUMENT, "bad batch");
    const auto t0 = std::chrono::steady_clock::now();
    m->eng->run(batch);
    m->eng->synchronize();
    m->last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return status_check(m);
  });
}

int ivc_run_async(ivc_model *m, int batch, void *stream) {
  return guarded(m, [&]() -> int {
    if (batch < 1 || batch > m->eng->max_batch()) return fail(m, IVC_ERR_ARGUMENT, "bad batch");
    if (stream && stream != (void *)m->eng->stream()) m->eng->set_stream((cudaStream_t)stream);
    m->eng->run(batch);
    return IVC_OK;
  });
}

int ivc_read_output_f16(ivc_model *m, int i, uint16_t *dst, int batch) {
  return guarded(m, [&]() -> int {
    if (!dst || i < 0 || i >= m->eng->output_count() || batch < 1 || batch > m->eng->max_batch())
      return fail(m, IVC_ERR_ARGUMENT, "bad arguments");
    m->eng->download_output_f16(i, dst, batch, false);
    m->eng->synchronize();
    return IVC_OK;
  });
}

int ivc_read_tensor_f16(ivc_model *m, const char *name, uint16_t *dst, int batch) {
  return guarded(m, [&]() -> int {
    if (!name || !dst || batch < 1 || batch > m->eng->max_batch()) return fail(m, IVC_ERR_ARGUMENT, "bad arguments");
    if (!m->eng->read_tensor_f16(name, dst, batch))
      return fail(m, IVC_ERR_NOT_FOUND, std::string("PlanModel: no tensor ") + name);
    return IVC_OK;
  });
}

namespace {
ivb::PreprocessCfg preprocess_cfg(const ivc_preprocess *c) {
  ivb::PreprocessCfg p;
  if (!c) return p;
  p.letterbox = c->letterbox ? 1 : 0;
  p.to_rgb = c->to_rgb ? 1 : 0;
  p.normalize = c->normalize ? 1 : 0;
  p.n_mean = std::min(std::max(c->n_mean, 0), 3);
  p.n_std = std::min(std::max(c->n_std, 0), 3);
  for (int i = 0; i < 3; ++i) {
    p.mean[i] = c->mean[i];
    p.std[i] = c->std[i];
  }
  return p;
}
}  // namespace

int ivc_set_input_bgr_u8(ivc_model *m, const uint8_t *frames, int batch, int height, int width, size_t row_stride,
                         int frames_on_device, const ivc_preprocess *cfg, float *letterbox) {
  return guarded(m, [&]() -> int {
    if (!frames || batch < 1 || batch > m->eng->max_batch() || height < 1 || width < 1 ||
        row_stride < (size_t)width * 3)
      return fail(m, IVC_ERR_ARGUMENT, "ivc_set_input_bgr_u8: bad arguments");
    m->eng->upload_input_bgr_u8(frames, batch, height, width, (int64_t)row_stride, frames_on_device != 0,
                                preprocess_cfg(cfg), letterbox);
    m->eng->synchronize();
    return IVC_OK;
  });
}

int ivc_infer_bgr_u8(ivc_model *m, const uint8_t *frames, int batch, int height, int width, size_t row_stride,
                     const ivc_preprocess *cfg, float *const *outputs, float *letterbox) {
  return guarded(m, [&]() -> int {
    if (!frames || !outputs || batch < 1 || batch > m->eng->max_batch() || height < 1 || width < 1 ||
        row_stride < (size_t)width * 3)
      return fail(m, IVC_ERR_ARGUMENT, "ivc_infer_bgr_u8: bad arguments");
    for (int i = 0; i < m->eng->output_count(); ++i)
      if (!outputs[i]) return fail(m, IVC_ERR_ARGUMENT, "ivc_infer_bgr_u8: null output buffer");
    const auto t0 = std::chrono::steady_clock::now();
    m->eng->infer_bgr_u8_host(frames, batch, height, width, (int64_t)row_stride, preprocess_cfg(cfg), outputs,
                              letterbox);
    m->last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return status_check(m);
  });
}

int ivc_decode_pose(ivc_model *m, int batch, float conf, float iou, int max_det, int nk, int kdims,
                    const float *letterbox, int *counts, float *dets) {
  return guarded(m, [&]() -> int {
    if (!counts || !dets || batch < 1 || batch > m->eng->max_batch() || max_det < 1)
      return fail(m, IVC_ERR_ARGUMENT, "ivc_decode_pose: bad arguments");
    m->eng->decode_pose(batch, conf, iou, max_det, nk, kdims, letterbox, counts, dets);
    return status_check(m);
  });
}

// ---- ivc_read_tensor_f16_noalloc: the relayout of ivc_read_tensor_f16 staged
// through one static device buffer per device instead of a cudaMalloc'd one.
// Overlapping calls on the same device (any handles) share the buffer and race.
namespace {
constexpr int64_t kNoAllocScratchBytes = 4ll << 20;  // 4 MiB per device
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_addr[kNoAllocMaxDevices] = {};
}  // namespace
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

int ivc_read_tensor_f16_noalloc(ivc_model *m, const char *name, uint16_t *dst, int batch) {
  return guarded(m, [&]() -> int {
    if (!name || !dst || batch < 1 || batch > m->eng->max_batch()) return fail(m, IVC_ERR_ARGUMENT, "bad arguments");
    m->eng->require_device();  // a dry run handle fails here, before any CUDA call
    const int dev = m->eng->device();
    if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(m, IVC_ERR_ARGUMENT, "read_tensor_f16_noalloc: device ordinal out of range");
    void *scratch = nullptr;
    {
      // device address of the static buffer, resolved once per device (the first
      // call may load the module, so it belongs before any stream capture)
      std::lock_guard<std::mutex> lk(g_noalloc_mu);
      if (g_noalloc_addr[dev] == nullptr) {
        cudaError_t e = cudaSetDevice(dev);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&g_noalloc_addr[dev], g_noalloc_scratch);
        if (e != cudaSuccess) {
          g_noalloc_addr[dev] = nullptr;
          return fail(m, IVC_ERR_CUDA,
                      std::string("CudaPlanModel: cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(e));
        }
      }
      scratch = g_noalloc_addr[dev];
    }
    int64_t need = 0;
    const int r = m->eng->read_tensor_f16_staged(name, dst, batch, scratch, kNoAllocScratchBytes, &need);
    if (r == 1) return fail(m, IVC_ERR_NOT_FOUND, std::string("PlanModel: no tensor ") + name);
    if (r == 2)
      return fail(m, IVC_ERR_ARGUMENT,
                  std::string("read_tensor_f16_noalloc: tensor ") + name + " needs " + std::to_string(need) +
                      " bytes of relayout scratch for " + std::to_string(batch) +
                      " image(s); the static scratch holds " + std::to_string(kNoAllocScratchBytes) + " bytes");
    return IVC_OK;
  });
}

int ivc_infer_f16_device(ivc_model *m, const void *d_input, int batch, void *const *d_outputs, void *stream) {
  return guarded(m, [&]() -> int {
    if (!d_input || !d_outputs || batch < 1 || batch > m->eng->max_batch())
      return fail(m, IVC_ERR_ARGUMENT, "bad arguments");
    cudaStream_t prev = m->eng->stream();
    if (stream && stream != (void *)prev) m->eng->set_stream((cudaStream_t)stream);
    m->eng->upload_input_f16(d_input, batch, true);
    m->eng->run(batch);
    for (int i = 0; i < m->eng->output_count(); ++i)
      if (d_outputs[i]) m->eng->download_output_f16(i, d_outputs[i], batch, true);
    return IVC_OK;
  });
}

int ivc_infer_f32_device(ivc_model *m, const float *d_input, int batch, float *const *d_outputs, void *stream) {
  return guarded(m, [&]() -> int {
    if (!d_input || !d_outputs || batch < 1 || batch > m->eng->max_batch())
      return fail(m, IVC_ERR_ARGUMENT, "bad arguments");
    cudaStream_t prev = m->eng->stream();
    if (stream && stream != (void *)prev) m->eng->set_stream((cudaStream_t)stream);
    m->eng->upload_input_f32(d_input, batch, true);
    m->eng->run(batch);
    for (int i = 0; i < m->eng->output_count(); ++i)
      if (d_outputs[i]) m->eng->download_output_f32(i, d_outputs[i], batch, true);
    return IVC_OK;
  });
}

int ivc_set_stream(ivc_model *m, void *stream) {
  return guarded(m, [&]() -> int {
    if (!stream) {
      cudaStream_t s = nullptr;
      if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
        return fail(m, IVC_ERR_CUDA, "cudaStreamCreate failed");
      m->eng->set_stream(s);
      return IVC_OK;
    }
    m->eng->set_stream((cudaStream_t)stream);
    return IVC_OK;
  });
}

int ivc_synchronize(ivc_model *m) {
  return guarded(m, [&]() -> int {
    m->eng->synchronize();
    return status_check(m);
  });
}

double ivc_last_infer_ms(const ivc_model *m) { return m ? m->last_ms : 0.0; }

int ivc_step_count(const ivc_model *m) { return m ? (int)m->eng->steps().size() : 0; }

int ivc_step_info(const ivc_model *m, int i, const char **name, const char **family, double *flops, double *act_bytes,
                  double *fixed_bytes) {
  if (!m || i < 0 || i >= (int)m->eng->steps().size()) return IVC_ERR_ARGUMENT;
  const ivb::Step &s = m->eng->steps()[(size_t)i];
  if (name) *name = s.name.c_str();
  if (family) *family = s.family.c_str();
  if (flops) *flops = s.flops_img;
  if (act_bytes) *act_bytes = s.bytes_img;
  if (fixed_bytes) *fixed_bytes = s.bytes_fixed;
  return IVC_OK;
}

int ivc_profile(ivc_model *m, int batch, float *step_ms, int n) {
  return guarded(m, [&]() -> int {
    if (!step_ms || n < (int)m->eng->steps().size() || batch < 1 || batch > m->eng->max_batch())
      return fail(m, IVC_ERR_ARGUMENT, "bad arguments");
    std::vector<float> ms;
    m->eng->run_profiled(batch, &ms);
    std::memcpy(step_ms, ms.data(), ms.size() * sizeof(float));
    return status_check(m);
  });
}

int ivc_launch_count(ivc_model *m, int batch, int *count) {
  return guarded(m, [&]() -> int {
    if (!count) return fail(m, IVC_ERR_ARGUMENT, "bad arguments");
    *count = m->eng->graph_kernel_count(batch);
    return IVC_OK;
  });
}

int ivc_debug_conv_wait(ivc_model *m, long long limit_cycles, int probe) {
  return guarded(m, [&]() -> int {
    if (limit_cycles < 1) return fail(m, IVC_ERR_ARGUMENT, "ivc_debug_conv_wait: limit must be positive");
    m->eng->set_conv_wait(limit_cycles, probe);
    return IVC_OK;
  });
}

int ivc_pool_stats(const ivc_model *m, int64_t *requested, int64_t *arena, int64_t *weights, int *roots, int *views,
                   int *nhwc, int *fc, int *fr) {
  if (!m) return IVC_ERR_ARGUMENT;
  const ivb::EngineStats &s = m->eng->stats();
  if (requested) *requested = s.requested_bytes;
  if (arena) *arena = s.arena_bytes;
  if (weights) *weights = s.weight_bytes;
  if (roots) *roots = s.roots;
  if (views) *views = s.views;
  if (nhwc) *nhwc = s.nhwc_tensors;
  if (fc) *fc = s.fusions_concat;
  if (fr) *fr = s.fusions_res;
  return IVC_OK;
}

int ivc_describe(const ivc_model *m, char *buf, size_t cap) {
  if (!m) return IVC_ERR_ARGUMENT;
  const std::string d = m->eng->describe();
  if (buf && cap) {
    const size_t n = d.size() < cap - 1 ? d.size() : cap - 1;
    std::memcpy(buf, d.data(), n);
    buf[n] = '\0';
  }
  return (int)d.size();
}

int ivc_device_properties(int device_ordinal, ivc_device_props *out) {
  if (!out) return IVC_ERR_ARGUMENT;
  std::memset(out, 0, sizeof(*out));
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    (void)cudaGetLastError();
    return IVC_ERR_CUDA;
  }
  out->device_count = n;
  if (device_ordinal < 0 || device_ordinal >= n) return IVC_ERR_ARGUMENT;
  cudaDeviceProp p{};
  if (cudaGetDeviceProperties(&p, device_ordinal) != cudaSuccess) {
    (void)cudaGetLastError();
    return IVC_ERR_CUDA;
  }
  std::snprintf(out->name, sizeof(out->name), "%s", p.name);
  out->multiprocessors = p.multiProcessorCount;
  int khz = 0;
  if (cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device_ordinal) != cudaSuccess) (void)cudaGetLastError();
  out->clock_mhz = khz / 1000;
  out->cc_major = p.major;
  out->cc_minor = p.minor;
  out->total_mem_bytes = (int64_t)p.totalGlobalMem;
  cudaRuntimeGetVersion(&out->runtime_version);
  return IVC_OK;
}

void ivc_f32_to_f16(const float *in, uint16_t *out, size_t n) { ivb::f32_to_f16_trunc_host(in, out, n); }

void ivc_f16_to_f32(const uint16_t *in, float *out, size_t n) {
  parallel_for(n, [&](size_t b, size_t e) {
    for (size_t i = b; i < e; ++i) out[i] = h2f(in[i]);
  });
}

}  // extern "C"
