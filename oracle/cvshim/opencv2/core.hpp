// Minimal stand-ins for the few OpenCV core types the reference's decoder
// headers name (cv::Rect2f, cv::Point2f, cv::Size, cv::Matx33f, cv::Mat), so
// that src/Decoders.cpp and src/Nms.cpp compile here without OpenCV.  TEST
// INFRASTRUCTURE ONLY: used by `make -C oracle ref` for oracle/_ref/.
// Field names and aggregate construction follow OpenCV's public types; nothing
// else of OpenCV is provided.
#pragma once

namespace cv {

struct Point2f {
  float x = 0.f, y = 0.f;
};

struct Rect2f {
  float x = 0.f, y = 0.f, width = 0.f, height = 0.f;
};

struct Size {
  int width = 0, height = 0;
};

struct Matx33f {
  float val[9] = {};
  static Matx33f eye() {
    Matx33f m;
    m.val[0] = m.val[4] = m.val[8] = 1.f;
    return m;
  }
};

class Mat;  // named by Preprocessor's declarations only

}  // namespace cv
