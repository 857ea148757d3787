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

void cpu_attention_partial(const float* q, int64_t seq_q, const float* k, const float* v,
                           int64_t seq_k, int64_t dim, float scale, float* acc, float* m,
                           float* l, int threads) {
  parallel_rows(seq_q, threads, [=](int64_t r0, int64_t r1) {
    std::vector<float> s(size_t(std::max<int64_t>(seq_k, 1)));
    for (int64_t i = r0; i < r1; ++i) {
      const float* qi = q + i * dim;
      float mx = -FLT_MAX;
      for (int64_t j = 0; j < seq_k; ++j) {
        const float* kj = k + j * dim;
        float dot = 0.f;
        for (int64_t d = 0; d < dim; ++d) dot += qi[d] * kj[d];
        s[size_t(j)] = dot * scale;
        mx = std::max(mx, s[size_t(j)]);
      }
      float* ai = acc + i * dim;
      std::fill(ai, ai + dim, 0.f);
      float sum = 0.f;
      for (int64_t j = 0; j < seq_k; ++j) {
        const float w = std::exp(s[size_t(j)] - mx);
        sum += w;
        const float* vj = v + j * dim;
        for (int64_t d = 0; d < dim; ++d) ai[d] += w * vj[d];
      }
      m[i] = mx;
      l[i] = sum;
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
