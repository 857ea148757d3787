// Host (CPU) attention of the legacy CPU-compute ring: the reference's
// ring/attention/ring_attention_staged.cu:40-105 (cpu_attention_partial and the
// CPU online-softmax merge) and the final normalisation (:255-260), as a
// multi-threaded C++ library. fp32, row-major [rows, dim] buffers.
#pragma once

#include <cstdint>

namespace mgfa::host {

// Unnormalised partial attention of q [seq_q, dim] against k, v [seq_k, dim]:
//   s_ij = scale * <q_i, k_j>, m_i = max_j s_ij, l_i = sum_j exp(s_ij - m_i),
//   acc_i = sum_j exp(s_ij - m_i) * v_j.
// Rows are split over `threads` worker threads (0 = hardware concurrency).
void cpu_attention_partial(const float* q, int64_t seq_q, const float* k, const float* v,
                           int64_t seq_k, int64_t dim, float scale, float* acc, float* m,
                           float* l, int threads = 0);

// Folds (m_new, l_new, acc_new) into the running (m, l, acc):
//   m' = max(m, m_new), a = exp(m - m'), b = exp(m_new - m'),
//   acc = a * acc + b * acc_new, l = a * l + b * l_new, m = m'.
// A running state starts at m = -FLT_MAX, l = 0, acc = 0.
void cpu_merge_online_softmax(float* m, float* l, float* acc, const float* m_new,
                              const float* l_new, const float* acc_new, int64_t seq_q,
                              int64_t dim);

// acc_i /= l_i.
void cpu_normalize(float* acc, const float* l, int64_t seq_q, int64_t dim);

}  // namespace mgfa::host
