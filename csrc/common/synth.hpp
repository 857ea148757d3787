// Deterministic synthetic inputs shared by the benchmarks, the checker and the
// Python layer.
//
// * Legacy inputs reproduce the reference prototype's formulas bit for bit
//   (evaluated in fp32 on the host):
//     KV[i] = rank * 1000 + i                (ring/attention/bench/*_bench.cu, h_init)
//     Q[i]  = (rank * 500 + (i % 64) * 0.01) * 0.001
//                                            (same files; verify_full.c:69-90)
// * Seeded normal inputs: element e of tensor `stream` is a standard normal drawn
//   from a counter-based generator, so any rank can produce any slice of the
//   global tensor without generating the rest. Counter -> 64 random bits uses the
//   SplitMix64 finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom
//   number generators", OOPSLA 2014); two 24-bit uniforms -> one normal uses the
//   Box-Muller transform (Box & Muller, 1958), cosine branch, in double.
#pragma once

#include <cmath>
#include <cstdint>

namespace mgfa::synth {

inline float legacy_kv(int rank, int64_t i) { return float(rank) * 1000.0f + float(i); }

inline float legacy_q(int rank, int64_t i, int dim) {
  return (float(rank) * 500.0f + float(i % dim) * 0.01f) * 0.001f;
}

inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Standard normal for (seed, stream, element).
inline double randn(uint64_t seed, uint64_t stream, uint64_t element) {
  const uint64_t key = splitmix64(seed * 0x100000001B3ull + stream);
  const uint64_t bits = splitmix64(key ^ (element * 0xD1B54A32D192ED03ull));
  // two uniforms in (0, 1]
  const double u1 = (double((bits >> 40) & 0xFFFFFF) + 1.0) / 16777216.0;
  const double u2 = double((bits >> 16) & 0xFFFFFF) / 16777216.0;
  const double two_pi = 6.283185307179586476925286766559;
  return std::sqrt(-2.0 * std::log(u1)) * std::cos(two_pi * u2);
}

// Uniform in [0, 1) for (seed, stream, element).
inline double uniform(uint64_t seed, uint64_t stream, uint64_t element) {
  const uint64_t key = splitmix64(seed * 0x100000001B3ull + stream + 0x5bd1e995ull);
  const uint64_t bits = splitmix64(key ^ (element * 0xD1B54A32D192ED03ull));
  return double(bits >> 11) * (1.0 / 9007199254740992.0);
}

// Tensor ids of the seeded streams.
enum Stream : uint64_t { kQ = 0, kK = 1, kV = 2, kdO = 3, kPayload = 4 };

}  // namespace mgfa::synth
