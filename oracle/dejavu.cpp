// dejavu.cpp -- CPU restatement of klearu's Deja Vu sparse FFN path.
//
// TEST INFRASTRUCTURE ONLY: the parity checker of the engine's predictor and
// sparse-MLP kernels (klearu_b200/csrc/dejavu.cu).  Nothing in the product
// path links or calls it.  Compiled into liboracle.so with -ffp-contract=off.
//
// Reference files (paths inside QuilibriumNetwork/klearu):
//   SparsityPredictor::predict      crates/klearu-dejavu/src/predictor/mlp_predictor.rs:102-123
//   SparsityPredictor::select_top_k crates/klearu-dejavu/src/predictor/mlp_predictor.rs:126-132
//   sparse_mlp::forward_sparse      crates/klearu-llm/src/sparse/sparse_mlp.rs:4-37
//   SparseMlp::forward (down bias)  crates/klearu-dejavu/src/mlp.rs:23-58
//
// Summation order: every dot product is a sequential f32 left fold from 0,
// as the reference's `iter().map(w * x).sum()` is.  The llm crate's
// Linear::forward_sparse (model/linear.rs:107-113) uses klearu-accel's
// dense_dot_dense_simd, whose AVX2 kernel sums in 8 lanes; the oracle keeps
// the scalar order of dense_dot_dense_scalar (simd/mod.rs), so that path is
// matched within floating-point tolerance, not bit for bit.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

namespace {

float dot_seq(const float* a, const float* b, int n) {
  float s = 0.0f;
  for (int i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}

}  // namespace

extern "C" {

// predict (mlp_predictor.rs:102-123) for T inputs x[T][in]: scores[T][out].
// w1 [hid][in], w2 [out][hid] row-major f32.
void orc_pred_predict(const float* w1, const float* b1, const float* w2, const float* b2, int in, int hid, int out,
                      const float* x, int T, float* scores) {
  std::vector<float> h(hid);
  for (int t = 0; t < T; ++t) {
    const float* xt = x + (size_t)t * in;
    for (int i = 0; i < hid; ++i) {
      const float v = dot_seq(w1 + (size_t)i * in, xt, in) + b1[i];
      h[i] = std::fmax(v, 0.0f);  // f32::max: a NaN operand yields the other one
    }
    for (int i = 0; i < out; ++i) {
      const float logit = dot_seq(w2 + (size_t)i * hid, h.data(), hid) + b2[i];
      scores[(size_t)t * out + i] = 1.0f / (1.0f + std::exp(-logit));
    }
  }
}

// select_top_k (mlp_predictor.rs:126-132): a stable sort by score descending
// (equal scores keep index order), the first min(k, n) indices.  Returns the
// number written.
int orc_pred_topk(const float* scores, int n, int k, uint32_t* idx) {
  std::vector<int> order(n);
  for (int i = 0; i < n; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return scores[a] > scores[b]; });
  const int m = std::min(k, n);
  for (int i = 0; i < m; ++i) idx[i] = (uint32_t)order[i];
  return m;
}

// forward_sparse (sparse_mlp.rs:4-37) for one token: gate/up [inter][hid],
// down [hid][inter] row-major; sel[k] the selected intermediate neurons in
// the order they are summed; bias (nullable) as in SparseMlp::forward
// (mlp.rs:50-53).  out[hid].
void orc_sparse_mlp(const float* gate, const float* up, const float* down, const float* bias, int hid, int inter,
                    const float* x, const uint32_t* sel, int k, float* out) {
  std::vector<float> a(k);
  for (int i = 0; i < k; ++i) {
    const float g = dot_seq(gate + (size_t)sel[i] * hid, x, hid);
    const float u = dot_seq(up + (size_t)sel[i] * hid, x, hid);
    a[i] = (g / (1.0f + std::exp(-g))) * u;
  }
  for (int j = 0; j < hid; ++j) {
    float s = 0.0f;
    const float* row = down + (size_t)j * inter;
    for (int i = 0; i < k; ++i) s += row[sel[i]] * a[i];
    out[j] = bias ? s + bias[j] : s;
  }
}

}  // extern "C"
