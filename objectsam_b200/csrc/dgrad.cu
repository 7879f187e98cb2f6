// Weight re-layout for the input-gradient convs (osam_conv_dgrad, abi.cu): the dgrad of a KRSC conv is a
// forward conv over dz whose "output channels" are the forward conv's inputs, so each sub-conv takes
// Wsub[c][r'][s'][k] = W[k][rmap[r']][smap[s']][c] — the filter flipped (stride 1) or split into the taps
// of one output-parity class (stride 2) — as its KRSC weights.
#include "conv_internal.h"

namespace osam {

struct DgradMap {
  int r[8], s[8];
};

__global__ void k_dgrad_weights(const __half* __restrict__ w, __half* __restrict__ dst, int K, int R, int S, int C,
                                int Rs, int Ss, const DgradMap m) {
  const long long n = (long long)C * Rs * Ss * K;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % K);
    long long t = i / K;
    const int s2 = (int)(t % Ss);
    t /= Ss;
    const int r2 = (int)(t % Rs);
    const int c = (int)(t / Rs);
    dst[i] = w[(((long long)k * R + m.r[r2]) * S + m.s[s2]) * C + c];
  }
}

cudaError_t launch_dgrad_weights(const __half* w, __half* dst, int K, int R, int S, int C, int Rs, int Ss,
                                 const int* rmap, const int* smap, cudaStream_t st) {
  DgradMap m{};
  for (int i = 0; i < Rs && i < 8; i++) m.r[i] = rmap[i];
  for (int i = 0; i < Ss && i < 8; i++) m.s[i] = smap[i];
  const long long n = (long long)C * Rs * Ss * K;
  int grid = (int)((n + 255) / 256);
  if (grid > 4096) grid = 4096;
  k_dgrad_weights<<<grid, 256, 0, st>>>(w, dst, K, R, S, C, Rs, Ss, m);
  return cudaGetLastError();
}

__global__ void k_dgrad_weights_batched(const DgradJob* __restrict__ jobs) {
  const DgradJob& j = jobs[blockIdx.y];
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < j.n; i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % j.K);
    long long t = i / j.K;
    const int s2 = (int)(t % j.Ss);
    t /= j.Ss;
    const int r2 = (int)(t % j.Rs);
    const int c = (int)(t / j.Rs);
    j.dst[i] = j.w[(((long long)k * j.R + j.r[r2]) * j.S + j.s[s2]) * j.C + c];
  }
}

cudaError_t launch_dgrad_weights_batched(const DgradJob* jobs, int njobs, cudaStream_t st) {
  if (njobs <= 0) return cudaSuccess;
  k_dgrad_weights_batched<<<dim3(64, njobs), 256, 0, st>>>(jobs);
  return cudaGetLastError();
}

}  // namespace osam
