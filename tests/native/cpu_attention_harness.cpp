// Differential-test harness for the host (CPU) attention library
// (csrc/host/cpu_attention.cpp) against the reference prototype's own
// cpu_attention_partial and merge_online_softmax: the reference's source file
// (REF_FILE, ring/attention/ring_attention_staged.cu, host code only) is
// included with its main renamed, so its two functions are called as written.
// Runs a two-step ring-style accumulation (partial on KV shard 0, merge the
// partial on shard 1, normalise) on seeded random and on the reference's
// legacy inputs, and prints the largest absolute and relative differences:
//   cpu_attention_harness <seq_q> <seq_k> <dim> <seed>
//   -> "max_abs <a> max_rel <r> legacy_max_abs <a> legacy_max_rel <r>"
#define main reference_ring_attention_staged_main
#include REF_FILE
#undef main

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "host/cpu_attention.hpp"

namespace {

struct Diff {
  double abs = 0, rel = 0;
};

Diff run(int sq, int sk, int dim, const std::vector<float>& q, const std::vector<float>& k0,
         const std::vector<float>& k1) {
  // reference: K = V as in its ring (the caller passes the same buffer twice)
  std::vector<float> ra(size_t(sq) * dim), rm(sq), rl(sq), pa(size_t(sq) * dim), pm(sq), pl(sq);
  cpu_attention_partial(q.data(), sq, k0.data(), k0.data(), sk, dim, ra.data(), rm.data(),
                        rl.data());
  cpu_attention_partial(q.data(), sq, k1.data(), k1.data(), sk, dim, pa.data(), pm.data(),
                        pl.data());
  merge_online_softmax(rm.data(), rl.data(), ra.data(), pm.data(), pl.data(), pa.data(), sq, dim);
  for (int i = 0; i < sq; ++i)
    for (int d = 0; d < dim; ++d) ra[size_t(i) * dim + d] /= rl[i];
  // this repository: same steps, scale 1 (the reference's scores are unscaled)
  std::vector<float> oa(size_t(sq) * dim), om(sq), ol(sq), qa(size_t(sq) * dim), qm(sq), ql(sq);
  mgfa::host::cpu_attention_partial(q.data(), sq, k0.data(), k0.data(), sk, dim, 1.f, oa.data(),
                                    om.data(), ol.data(), 2);
  mgfa::host::cpu_attention_partial(q.data(), sq, k1.data(), k1.data(), sk, dim, 1.f, qa.data(),
                                    qm.data(), ql.data(), 3);
  mgfa::host::cpu_merge_online_softmax(om.data(), ol.data(), oa.data(), qm.data(), ql.data(),
                                       qa.data(), sq, dim);
  mgfa::host::cpu_normalize(oa.data(), ol.data(), sq, dim);
  Diff df;
  for (size_t i = 0; i < ra.size(); ++i) {
    const double a = std::fabs(double(ra[i]) - double(oa[i]));
    df.abs = std::max(df.abs, a);
    df.rel = std::max(df.rel, a / std::max({std::fabs(double(ra[i])), std::fabs(double(oa[i])), 1e-12}));
  }
  return df;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 5) return 2;
  const int sq = std::atoi(argv[1]), sk = std::atoi(argv[2]), dim = std::atoi(argv[3]);
  std::mt19937 gen(unsigned(std::atoi(argv[4])));
  std::normal_distribution<float> nd(0.f, 1.f);
  std::vector<float> q(size_t(sq) * dim), k0(size_t(sk) * dim), k1(size_t(sk) * dim);
  for (auto& x : q) x = nd(gen) * 0.3f;
  for (auto& x : k0) x = nd(gen);
  for (auto& x : k1) x = nd(gen);
  const Diff r = run(sq, sk, dim, q, k0, k1);
  // the reference's own legacy inputs: Q = (rank*500 + (i % dim)*0.01)*0.001, KV = owner*1000 + i
  for (int i = 0; i < sq * dim; ++i) q[size_t(i)] = (1 * 500.0f + float(i % dim) * 0.01f) * 0.001f;
  for (int i = 0; i < sk * dim; ++i) k0[size_t(i)] = 0 * 1000.0f + float(i);
  for (int i = 0; i < sk * dim; ++i) k1[size_t(i)] = 1 * 1000.0f + float(i);
  const Diff l = run(sq, sk, dim, q, k0, k1);
  std::printf("max_abs %.3g max_rel %.3g legacy_max_abs %.3g legacy_max_rel %.3g\n", r.abs, r.rel,
              l.abs, l.rel);
  return 0;
}
