// Host-only self-test of the native tools' process-group layer (dist_env.cpp):
// rendezvous through the TCPStore, barriers, all-gather, MAX reductions and the
// blocking host send/recv around the ring. Launched like the benchmarks
// (`torchrun --nproc-per-node N --no-python build/bin/dist_selftest`); needs no
// GPU. Prints "dist selftest ok rank=<r> world=<P>" on success, exits 1 otherwise.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "dist_env.hpp"

using mgfa::bench::Dist;

static int fail(int r, const std::string& what) {
  std::fprintf(stderr, "[Rank %d] dist selftest failed: %s\n", r, what.c_str());
  return 1;
}

int main() {
  try {
    Dist d = Dist::from_env(120, /*need_gpu=*/false);
    const int r = d.rank(), P = d.world();
    for (int i = 0; i < 3; ++i) d.barrier();
    // all-gather of per-rank strings
    const auto all = d.all_gather("rank" + std::to_string(r));
    if (int(all.size()) != P) return fail(r, "all_gather size");
    for (int i = 0; i < P; ++i)
      if (all[size_t(i)] != "rank" + std::to_string(i)) return fail(r, "all_gather content");
    // MAX over ranks
    const auto mx = d.max({double(r), -double(r), 7.5});
    if (mx[0] != P - 1 || mx[1] != 0.0 || mx[2] != 7.5) return fail(r, "max");
    // host send/recv around the ring, P - 1 steps: the shard of owner
    // (r - s - 1) mod P arrives at step s
    if (P > 1) {
      const int right = (r + 1) % P, left = (r - 1 + P) % P;
      std::vector<int> cur(1000, r), nxt(1000, -1);
      for (int s = 0; s < P - 1; ++s) {
        d.host_sendrecv(cur.data(), cur.size() * sizeof(int), right, nxt.data(), left);
        const int owner = ((r - s - 1) % P + P) % P;
        for (int x : nxt)
          if (x != owner) return fail(r, "sendrecv data at step " + std::to_string(s));
        cur.swap(nxt);
      }
    }
    d.barrier();
    std::printf("dist selftest ok rank=%d world=%d\n", r, P);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "dist selftest: %s\n", e.what());
    return 1;
  }
}
