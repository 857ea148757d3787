#include "cpu_attention.hpp"

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <thread>
#include <vector>

namespace mgfa::host {

namespace {

template <class Fn>
void parallel_rows(int64_t rows, int threads, Fn fn) {
  int n = threads > 0 ? threads : int(std::max(1u, std::thread::hardware_concurrency()));
  n = int(std::min<int64_t>(n, std::max<int64_t>(1, rows / 16)));
  if (n <= 1) {
    fn(int64_t(0), rows);
    return;
  }
  std::vector<std::thread> pool;
  const int64_t per = (rows + n - 1) / n;
  for (int t = 0; t < n; ++t) {
    const int64_t b = t * per, e = std::min(rows, b + per);
    if (b < e) pool.emplace_back(fn, b, e);
  }
  for (auto& th : pool) th.join();
}

}  // namespace

// Rows go kRows at a time with the row index innermost, so the compiler can put
// rows in SIMD lanes; every sum still runs in the reference's order (over d for
// a score, over j for the row sum and each accumulator element), so the results
// are the reference's bit for bit.
void cpu_attention_partial(const float* q, int64_t seq_q, const float* k, const float* v,
                           int64_t seq_k, int64_t dim, float scale, float* acc, float* m,
                           float* l, int threads) {
  constexpr int kRows = 8;
  parallel_rows(seq_q, threads, [=](int64_t r0, int64_t r1) {
    std::vector<float> qt(size_t(dim) * kRows), at(size_t(dim) * kRows);  // [d][row]
    std::vector<float> s(size_t(std::max<int64_t>(seq_k, 1)) * kRows);    // [j][row]
    for (int64_t i0 = r0; i0 < r1; i0 += kRows) {
      const int nr = int(std::min<int64_t>(kRows, r1 - i0));
      std::fill(qt.begin(), qt.end(), 0.f);
      for (int r = 0; r < nr; ++r)
        for (int64_t d = 0; d < dim; ++d) qt[size_t(d) * kRows + r] = q[(i0 + r) * dim + d];
      float mx[kRows], sum[kRows];
      for (int r = 0; r < kRows; ++r) mx[r] = -FLT_MAX, sum[r] = 0.f;
      for (int64_t j = 0; j < seq_k; ++j) {
        const float* kj = k + j * dim;
        float dot[kRows] = {};
        for (int64_t d = 0; d < dim; ++d)
          for (int r = 0; r < kRows; ++r) dot[r] += qt[size_t(d) * kRows + r] * kj[d];
        for (int r = 0; r < kRows; ++r) {
          const float sc = dot[r] * scale;
          s[size_t(j) * kRows + r] = sc;
          mx[r] = std::max(mx[r], sc);
        }
      }
      std::fill(at.begin(), at.end(), 0.f);
      for (int64_t j = 0; j < seq_k; ++j) {
        float w[kRows];
        for (int r = 0; r < kRows; ++r) {
          w[r] = std::exp(s[size_t(j) * kRows + r] - mx[r]);
          sum[r] += w[r];
        }
        const float* vj = v + j * dim;
        for (int64_t d = 0; d < dim; ++d)
          for (int r = 0; r < kRows; ++r) at[size_t(d) * kRows + r] += w[r] * vj[d];
      }
      for (int r = 0; r < nr; ++r) {
        float* ai = acc + (i0 + r) * dim;
        for (int64_t d = 0; d < dim; ++d) ai[d] = at[size_t(d) * kRows + r];
        m[i0 + r] = mx[r];
        l[i0 + r] = sum[r];
      }
    }
  });
}

void cpu_merge_online_softmax(float* m, float* l, float* acc, const float* m_new,
                              const float* l_new, const float* acc_new, int64_t seq_q,
                              int64_t dim) {
  for (int64_t i = 0; i < seq_q; ++i) {
    const float mm = std::max(m[i], m_new[i]);
    const float a = std::exp(m[i] - mm), b = std::exp(m_new[i] - mm);
    float* ai = acc + i * dim;
    const float* ni = acc_new + i * dim;
    for (int64_t d = 0; d < dim; ++d) ai[d] = a * ai[d] + b * ni[d];
    l[i] = a * l[i] + b * l_new[i];
    m[i] = mm;
  }
}

void cpu_normalize(float* acc, const float* l, int64_t seq_q, int64_t dim) {
  for (int64_t i = 0; i < seq_q; ++i)
    for (int64_t d = 0; d < dim; ++d) acc[i * dim + d] /= l[i];
}

}  // namespace mgfa::host
