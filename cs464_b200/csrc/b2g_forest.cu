// b2g_forest.cu — host-side scoring of the learned ranker: a tree ensemble stored as plain arrays.
//
// The selector ranks ~9k configs per new shape with a gradient-boosted tree ensemble. The model ships as arrays
// (feature index, threshold, children, missing-value direction and value per node; one root per tree) instead of a
// pickled library object, so any version of the training library — or none — can use it. Prediction per row:
// base + sum over trees (in tree order) of the value of the leaf reached by going left when x[feature] <= threshold
// (or, for a missing value, when the node says so). Summation order and arithmetic (double) are those of the
// training library's own predictor, so scores and rankings are reproduced exactly. Rows are split over threads.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <thread>
#include <vector>

#include "b2g.h"

namespace {

void predict_rows(const int32_t* feature, const double* threshold, const int32_t* left, const int32_t* right,
                  const uint8_t* missing_left, const double* value, const int32_t* roots, int32_t n_trees,
                  double base, const double* X, int32_t n_features, double* out, int64_t r0, int64_t r1) {
  for (int64_t r = r0; r < r1; ++r) {
    const double* x = X + r * n_features;
    double acc = base;
    for (int32_t t = 0; t < n_trees; ++t) {
      int32_t node = roots[t];
      while (feature[node] >= 0) {
        const double v = x[feature[node]];
        const bool go_left = std::isnan(v) ? missing_left[node] != 0 : v <= threshold[node];
        node = go_left ? left[node] : right[node];
      }
      acc += value[node];
    }
    out[r] = acc;
  }
}

}  // namespace

extern "C" int32_t b2g_forest_predict(const int32_t* feature, const double* threshold, const int32_t* left,
                                      const int32_t* right, const uint8_t* missing_left, const double* value,
                                      const int32_t* roots, int32_t n_trees, double base, const double* X,
                                      int64_t n_rows, int32_t n_features, double* out, int32_t threads) {
  if (!feature || !threshold || !left || !right || !missing_left || !value || !roots || !X || !out)
    return B2G_ERR_INVALID_ARG;
  if (n_trees < 0 || n_rows < 0 || n_features < 1) return B2G_ERR_INVALID_ARG;
  int64_t nt = std::max<int32_t>(1, threads);
  nt = std::min<int64_t>(nt, std::max<int64_t>(1, n_rows / 256));
  if (nt <= 1) {
    predict_rows(feature, threshold, left, right, missing_left, value, roots, n_trees, base, X, n_features, out, 0,
                 n_rows);
    return B2G_OK;
  }
  std::vector<std::thread> pool;
  const int64_t per = (n_rows + nt - 1) / nt;
  for (int64_t i = 0; i < nt; ++i) {
    const int64_t r0 = i * per, r1 = std::min(n_rows, r0 + per);
    if (r0 >= r1) break;
    pool.emplace_back(predict_rows, feature, threshold, left, right, missing_left, value, roots, n_trees, base, X,
                      n_features, out, r0, r1);
  }
  for (auto& th : pool) th.join();
  return B2G_OK;
}
