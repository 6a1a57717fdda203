// C entry point over the reference's own pose decoder and NMS
// (src/Decoders.cpp `PoseDecoder::decode`, `nmsPerClass`; src/Nms.cpp `iou`,
// `nms`), compiled from the reference sources by `make -C oracle ref` into
// oracle/_ref/libref_decode.so.  TEST INFRASTRUCTURE ONLY: it produces golden
// vectors (tests/golden/make_decode_golden.py) that pin oracle/decode.py.
#include <cstring>
#include <vector>

#include "infvino/Decoders.hpp"

extern "C" {

// out: [C][A] channel-major f32 (the executor's output 0 of one image).  Writes
// up to `cap` detections of 5 + 2 * nk floats each (score, x, y, w, h, then the
// keypoints' x, y) in the decoder's order; returns the detection count (which
// may exceed cap) or -1 on an exception.
int ref_pose_decode(const float *out, int C, int A, float conf, float iou, int max_det, int nk, int kdims,
                    float scale, int pad_left, int pad_top, float *dets, int cap) {
  try {
    infvino::ModelInfo info;
    info.task = infvino::Task::Pose;
    info.kpt_shape = {nk, kdims};
    info.conf = conf;
    info.iou = iou;
    info.max_det = max_det;
    infvino::LetterboxInfo lb;
    lb.scale = scale;
    lb.pad_left = pad_left;
    lb.pad_top = pad_top;
    std::vector<infvino::Tensor> outputs;
    outputs.emplace_back(std::vector<int64_t>{1, C, A}, std::vector<float>(out, out + (size_t)C * A));
    const infvino::InferResult r = infvino::PoseDecoder(info).decode(outputs, info, lb);
    const int S = 5 + 2 * nk;
    int k = 0;
    for (const auto &d : r.detections) {
      if (k < cap) {
        float *p = dets + (size_t)k * S;
        p[0] = d.score;
        p[1] = d.box.x;
        p[2] = d.box.y;
        p[3] = d.box.width;
        p[4] = d.box.height;
        for (int j = 0; j < nk && j < (int)d.keypoints.size(); ++j) {
          p[5 + 2 * j] = d.keypoints[(size_t)j].x;
          p[6 + 2 * j] = d.keypoints[(size_t)j].y;
        }
      }
      ++k;
    }
    return k;
  } catch (...) {
    return -1;
  }
}

}  // extern "C"
