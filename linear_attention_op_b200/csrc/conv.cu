// Prefill causal depthwise conv (K = 4) + SiLU with a rolling conv state.
//
// out[t, c] = SiLU(sum_j w[c, j] * x[t - 3 + j, c]) where x[-3..-1] come from conv_state (row i holds the
// input at time i - 3).  9B/kernels/layer_compute.cpp:74-103 (x_s @ diag(w_tap)), layer_reader.cpp:103-124
// (shifts), :184-197 (roll: new row j holds the input at time T - 3 + j; HF torch_causal_conv1d_update).
// HBM-bound: each thread owns one channel quad (float4) of a 16-token segment and issues all 19 row loads
// (3-token history included) before computing, so a warp has 19 x 512 contiguous bytes in flight.
#include "gemm.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace gdn {

constexpr int kConvSeg = 16;  // tokens per thread: all 19 input rows are loaded before any output is formed

__global__ void __launch_bounds__(128) conv_prefill_kernel(const float* __restrict__ in, int64_t in_ld,
                                                           float* __restrict__ out, int64_t out_ld,
                                                           const float* __restrict__ conv_w,
                                                           const float* __restrict__ conv_state, int B, int T,
                                                           int C) {
  const int quads = C / 4;
  const int segs = (T + kConvSeg - 1) / kConvSeg;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= static_cast<int64_t>(B) * segs * quads) return;
  const int cq = static_cast<int>(gid % quads);
  const int seg = static_cast<int>((gid / quads) % segs);
  const int b = static_cast<int>(gid / (static_cast<int64_t>(quads) * segs));
  const int c = cq * 4;
  const int t0 = seg * kConvSeg;
  const float4 w0 = reinterpret_cast<const float4*>(conv_w + static_cast<int64_t>(c) * 4)[0];
  const float4 w1 = reinterpret_cast<const float4*>(conv_w + static_cast<int64_t>(c + 1) * 4)[0];
  const float4 w2 = reinterpret_cast<const float4*>(conv_w + static_cast<int64_t>(c + 2) * 4)[0];
  const float4 w3 = reinterpret_cast<const float4*>(conv_w + static_cast<int64_t>(c + 3) * 4)[0];
  float4 x[kConvSeg + 3];
#pragma unroll
  for (int i = 0; i < kConvSeg + 3; ++i) {
    const int t = t0 - 3 + i;
    if (t >= T) {
      x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if (t >= 0) {
      x[i] = __ldcs(reinterpret_cast<const float4*>(in + (static_cast<int64_t>(b) * T + t) * in_ld + c));
    } else {
      x[i] = *reinterpret_cast<const float4*>(conv_state + (static_cast<int64_t>(b) * 3 + (t + 3)) * C + c);
    }
  }
#pragma unroll
  for (int i = 0; i < kConvSeg; ++i) {
    const int t = t0 + i;
    if (t < T) {
      const float4 &h0 = x[i], &h1 = x[i + 1], &h2 = x[i + 2], &xv = x[i + 3];
      float4 y;
      y.x = silu_f(w0.x * h0.x + w0.y * h1.x + w0.z * h2.x + w0.w * xv.x);
      y.y = silu_f(w1.x * h0.y + w1.y * h1.y + w1.z * h2.y + w1.w * xv.y);
      y.z = silu_f(w2.x * h0.z + w2.y * h1.z + w2.z * h2.z + w2.w * xv.z);
      y.w = silu_f(w3.x * h0.w + w3.y * h1.w + w3.z * h2.w + w3.w * xv.w);
      __stcs(reinterpret_cast<float4*>(out + (static_cast<int64_t>(b) * T + t) * out_ld + c), y);
    }
  }
}

// Runs after conv_prefill_kernel (stream order), so the old history is no longer needed by anyone.
__global__ void conv_state_roll_kernel(const float* __restrict__ in, int64_t in_ld, float* __restrict__ conv_state,
                                       int B, int T, int C) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= static_cast<int64_t>(B) * C) return;
  const int c = static_cast<int>(gid % C), b = static_cast<int>(gid / C);
  float* cs = conv_state + static_cast<int64_t>(b) * 3 * C + c;
  float nv[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = T - 3 + j;
    nv[j] = t >= 0 ? in[(static_cast<int64_t>(b) * T + t) * in_ld + c] : cs[static_cast<int64_t>(T + j) * C];
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) cs[static_cast<int64_t>(j) * C] = nv[j];
}

cudaError_t conv_prefill(const float* in, int64_t in_ld, float* out, int64_t out_ld, const float* conv_w,
                         float* conv_state, int B, int T, int C, cudaStream_t stream) {
  if (B <= 0 || T <= 0 || C <= 0 || (C & 3) || (in_ld & 3) || (out_ld & 3)) return cudaErrorInvalidValue;
  const int segs = (T + kConvSeg - 1) / kConvSeg;
  const int64_t n = static_cast<int64_t>(B) * segs * (C / 4);
  count_launch();
  conv_prefill_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, stream>>>(in, in_ld, out, out_ld, conv_w,
                                                                                 conv_state, B, T, C);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t m = static_cast<int64_t>(B) * C;
  count_launch();
  conv_state_roll_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, stream>>>(in, in_ld, conv_state, B, T, C);
  return cudaGetLastError();
}

}  // namespace gdn
