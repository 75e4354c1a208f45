// Output-length predictor for KV-capacity admission (host C++).
//
// Behaviour of the reference's ForeLen model (core/optimization/gollek-plugin-wait-scheduler/src/
// main/cpp/forelen/gollek_forelen.c:26-161): a 1 -> H -> 1 ReLU MLP on log(1 + prompt_tokens)/10,
// output clamped to [min_out, max_out], trained online by SGD on (prompt, actual output) pairs
// with gradients accumulated and applied in batches, plus a running mean-absolute-error.
// Differences by design: the predictor is an object (one per scheduler, not process-global state),
// the input normalisation, clamp range and learning rate are constructor parameters, and biases
// are trained too.
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <vector>

class LengthPredictor {
 public:
  LengthPredictor(int hidden, float min_out, float max_out, float lr, int batch)
      : h_(hidden), min_out_(min_out), max_out_(max_out), lr_(lr), batch_(batch), w1_(hidden), b1_(hidden),
        w2_(hidden), gw1_(hidden, 0.f), gb1_(hidden, 0.f), gw2_(hidden, 0.f) {
    // deterministic spread of ReLU kinks over the normalised input range [0, 1]
    for (int i = 0; i < h_; ++i) {
      w1_[i] = 1.0f;
      b1_[i] = -(float)i / (float)h_;
      w2_[i] = 0.0f;
    }
    b2_ = 0.5f * (min_out + max_out);
  }

  float predict(float prompt_tokens) const {
    std::vector<float> hid(h_);
    return std::clamp(forward(norm(prompt_tokens), hid), min_out_, max_out_);
  }

  void observe(float prompt_tokens, float actual) {
    std::vector<float> hid(h_);
    const float x = norm(prompt_tokens);
    const float raw = forward(x, hid);
    const float pred = std::clamp(raw, min_out_, max_out_);
    abs_err_sum_ += std::fabs(pred - actual);
    ++n_obs_;
    const float err = (raw - actual) / (max_out_ - min_out_);  // scale-free gradient
    for (int i = 0; i < h_; ++i) {
      gw2_[i] += err * hid[i];
      if (hid[i] > 0.f) {
        const float dh = err * w2_[i];
        gw1_[i] += dh * x;
        gb1_[i] += dh;
      }
    }
    gb2_ += err;
    if (++pending_ >= batch_) flush();
  }

  void flush() {
    if (pending_ == 0) return;
    const float s = lr_ / (float)pending_;
    const float range = max_out_ - min_out_;
    for (int i = 0; i < h_; ++i) {
      w2_[i] -= s * gw2_[i] * range;
      w1_[i] -= s * gw1_[i];
      b1_[i] -= s * gb1_[i];
      gw1_[i] = gb1_[i] = gw2_[i] = 0.f;
    }
    b2_ -= s * gb2_ * range;
    gb2_ = 0.f;
    pending_ = 0;
  }

  float mae() const { return n_obs_ ? abs_err_sum_ / (float)n_obs_ : 0.f; }
  int64_t observations() const { return n_obs_; }

 private:
  static float norm(float p) { return std::log1p(std::max(0.f, p)) / 10.f; }
  float forward(float x, std::vector<float>& hid) const {
    float y = b2_;
    for (int i = 0; i < h_; ++i) {
      hid[i] = std::max(0.f, w1_[i] * x + b1_[i]);
      y += w2_[i] * hid[i];
    }
    return y;
  }
  int h_;
  float min_out_, max_out_, lr_;
  int batch_;
  std::vector<float> w1_, b1_, w2_, gw1_, gb1_, gw2_;
  float b2_ = 0.f, gb2_ = 0.f;
  int pending_ = 0;
  double abs_err_sum_ = 0.0;
  int64_t n_obs_ = 0;
};

void register_forelen(pybind11::module& m) {
  namespace py = pybind11;
  py::class_<LengthPredictor>(m, "LengthPredictor")
      .def(py::init<int, float, float, float, int>(), py::arg("hidden") = 64, py::arg("min_out") = 1.f,
           py::arg("max_out") = 4096.f, py::arg("lr") = 0.05f, py::arg("batch") = 8)
      .def("predict", &LengthPredictor::predict)
      .def("observe", &LengthPredictor::observe)
      .def("flush", &LengthPredictor::flush)
      .def("mae", &LengthPredictor::mae)
      .def("observations", &LengthPredictor::observations);
}
