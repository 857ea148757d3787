// Peer-access report (the reference's ring/check_peer.cu): one line per ordered
// GPU pair, "GPU i -> GPU j: YES|NO" from cudaDeviceCanAccessPeer, in the
// reference's order and format. --attrs adds the runtime's P2P attributes of
// each pair (performance rank, native atomics, CUDA-array access).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

int main(int argc, char** argv) {
  const bool attrs = argc > 1 && std::strcmp(argv[1], "--attrs") == 0;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) count = 0;
  for (int i = 0; i < count; i++)
    for (int j = 0; j < count; j++) {
      if (i == j) continue;
      int can = 0;
      cudaDeviceCanAccessPeer(&can, i, j);
      std::printf("GPU %d -> GPU %d: %s\n", i, j, can ? "YES" : "NO");
      if (attrs && can) {
        int rank = 0, atomics = 0, arrays = 0;
        cudaDeviceGetP2PAttribute(&rank, cudaDevP2PAttrPerformanceRank, i, j);
        cudaDeviceGetP2PAttribute(&atomics, cudaDevP2PAttrNativeAtomicSupported, i, j);
        cudaDeviceGetP2PAttribute(&arrays, cudaDevP2PAttrCudaArrayAccessSupported, i, j);
        std::printf("  performance rank %d, native atomics %s, CUDA arrays %s\n", rank,
                    atomics ? "yes" : "no", arrays ? "yes" : "no");
      }
    }
  return 0;
}
