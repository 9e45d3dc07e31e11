// Conv-state roll after the prefill in_proj.
//
// The prefill causal depthwise conv (K = 4) + SiLU itself runs in the epilogue of the in_proj GEMM
// (kEpiPrefillInProj), which reads the cached history from conv_state and writes the raw inputs at times
// T - 3 .. T - 1 of every sequence to conv_tail.  This kernel then rolls the state: new row j holds the
// input at time T - 3 + j (9B/kernels/layer_reader.cpp:184-197; HF torch_causal_conv1d_update keeps the
// last K - 1 inputs), taken from the old state when T < 3.
#include "gemm.cuh"
#include "kernels.cuh"

namespace gdn {

__global__ void conv_state_roll_tail_kernel(const float* __restrict__ tail, float* __restrict__ conv_state, int B,
                                            int T, int C) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= static_cast<int64_t>(B) * C) return;
  const int c = static_cast<int>(gid % C), b = static_cast<int>(gid / C);
  float* cs = conv_state + static_cast<int64_t>(b) * 3 * C + c;
  const float* tl = tail + static_cast<int64_t>(b) * 3 * C + c;
  float nv[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) nv[j] = T - 3 + j >= 0 ? tl[static_cast<int64_t>(j) * C] : cs[static_cast<int64_t>(T + j) * C];
#pragma unroll
  for (int j = 0; j < 3; ++j) cs[static_cast<int64_t>(j) * C] = nv[j];
}

cudaError_t conv_state_roll_tail(const float* tail, float* conv_state, int B, int T, int C, cudaStream_t stream) {
  if (B <= 0 || T <= 0 || C <= 0) return cudaErrorInvalidValue;
  const int64_t m = static_cast<int64_t>(B) * C;
  count_launch();
  conv_state_roll_tail_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, stream>>>(tail, conv_state, B, T, C);
  return cudaGetLastError();
}

}  // namespace gdn
