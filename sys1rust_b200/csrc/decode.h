// Host-side decode of the forward's outputs into answers: the arithmetic of the reference's
// `decode_answers` (runtime/crates/laya-core/src/decode.rs:318-413) and its action head
// (`ActHead::probs`, decode.rs:232-253; `act_features`, :257-267), without the JSON formatting.
//
// Per row r with k = marker_count[r] options and temperature t:
//   p = softmax(logits[r, :k] / t) in double precision (decode.rs:330-332);
//   confidence = 1 - H(p) / ln k, clamped to [0, 1] (1 when k < 2; decode.rs:88-94);
//   choice: argmax (first maximum) and p[argmax]; score: sum_i i p_i and max p; noul: p[1] and
//   max(p[1], 1 - p[1]), which is both confidences (decode.rs:336-411);
//   act_probability = class 0 of the action head: Linear(d + 4, H) -> exact GELU ->
//   Linear(H, n_act) -> softmax in single precision, fed the pooled row and four features of the
//   full masked logits row: top-1 and top-1 - top-2 probabilities, normalised entropy over
//   ln max(k, 2), and max(k, 2) / 255 (decode.rs:257-267).
#pragma once
#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

namespace s1c {
namespace dec {

inline std::vector<float> softmax_f32(const float* z, int n) {
  float m = -INFINITY;
  for (int i = 0; i < n; ++i) m = std::max(m, z[i]);
  std::vector<float> e(n);
  float s = 0.f;
  for (int i = 0; i < n; ++i) {
    e[i] = std::exp(z[i] - m);
    s += e[i];
  }
  for (int i = 0; i < n; ++i) e[i] /= s;
  return e;
}

inline std::vector<double> softmax_f64(const std::vector<double>& z) {
  double m = -INFINITY;
  for (double x : z) m = std::max(m, x);
  std::vector<double> e(z.size());
  double s = 0.0;
  for (size_t i = 0; i < z.size(); ++i) {
    e[i] = std::exp(z[i] - m);
    s += e[i];
  }
  for (double& x : e) x /= s;
  return e;
}

inline double confidence_from_probs(const std::vector<double>& p, int k) {
  if (k < 2) return 1.0;
  double ent = 0.0;
  for (int i = 0; i < k; ++i) ent += -p[i] * std::log(std::min(std::max(p[i], 1e-12), 1.0));
  return std::min(std::max(1.0 - ent / std::log((double)k), 0.0), 1.0);
}

// Exact (erf) GELU evaluated in double and rounded to float.
inline float gelu_exact(float x) {
  const double xf = x;
  return (float)(0.5 * xf * (1.0 + std::erf(xf / std::sqrt(2.0))));
}

inline void act_features(const float* row, int kmax, int marker_count, float out[4]) {
  const std::vector<float> p = softmax_f32(row, kmax);
  const float k = (float)std::max(marker_count, 2);
  float ent = 0.f;
  for (float x : p) ent += x * std::log(std::max(x, 1e-9f));
  ent = -ent / std::log(k);
  std::vector<float> sorted = p;
  std::sort(sorted.begin(), sorted.end(), [](float a, float b) { return a > b; });
  const float top1 = sorted.empty() ? 0.f : sorted[0];
  const float top2 = sorted.size() > 1 ? sorted[1] : 0.f;
  out[0] = top1;
  out[1] = top1 - top2;
  out[2] = ent;
  out[3] = k / 255.0f;
}

inline std::vector<float> act_probs(const s1c_act_head& h, const float* pooled, const float feats[4]) {
  const int d = h.d_in - 4;
  std::vector<float> hid((size_t)h.hidden);
  for (int j = 0; j < h.hidden; ++j) {
    const float* row = h.w0 + (size_t)j * h.d_in;
    float acc = h.b0[j];
    for (int i = 0; i < d; ++i) acc += row[i] * pooled[i];
    for (int i = 0; i < 4; ++i) acc += row[d + i] * feats[i];
    hid[(size_t)j] = gelu_exact(acc);
  }
  std::vector<float> out((size_t)h.n_act);
  for (int j = 0; j < h.n_act; ++j) {
    const float* row = h.w2 + (size_t)j * h.hidden;
    float acc = 0.f;
    for (int i = 0; i < h.hidden; ++i) acc += row[i] * hid[(size_t)i];
    out[(size_t)j] = h.b2[j] + acc;
  }
  return softmax_f32(out.data(), h.n_act);
}

}  // namespace dec
}  // namespace s1c
