// Row RMSNorm of the decoder layer around the GDN mixer (Hugging Face Qwen3_5RMSNorm: the row normalised
// in fp32, times (1 + w), cast to the input dtype), optionally after a residual add (Qwen3_5DecoderLayer:
// hidden = residual + mixer output, in the input dtype).  The row is held in registers (16-byte loads),
// so each row is read once and written once: an HBM-bound pass.
//
// The reference stacks GDN mixers only (0.8B/gdn_l1.py:295-325); its optimisation notes name the decoder
// surroundings (input RMSNorm, residual, MLP) as the next step (0.8B/OPTIMIZATION.md:258-259).
#include <cuda_bf16.h>

#include "gemm.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace gdn {

namespace {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return u;
}

// x [rows, h] bf16; add (optional) [rows, h] bf16: then s = bf16(x + add) is normalised and written to
// sum_out; out [rows, h] = bf16(s * rsqrt(mean(s^2) + eps) * (1 + w)).  One 256-thread CTA per row, VPT
// 16-byte vectors per thread held in registers, so even a decode step's 64 rows spread over 64 SMs; the
// sum of squares is reduced over the warp, then over the 8 warps in shared memory.  Launched with
// programmatic dependent launch: it waits for the previous kernel, then lets the next one (a
// weight-streaming GEMM) start its weight prefetch.
template <int VPT>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const uint16_t* __restrict__ x, const uint16_t* add,
                                                           uint16_t* sum_out, const float* __restrict__ w, float eps,
                                                           uint16_t* out, int rows, int h) {
  __shared__ float red[8];
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (row >= rows) return;
  const int nv = h / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * h);
  const uint4* ar = add ? reinterpret_cast<const uint4*>(add + static_cast<int64_t>(row) * h) : nullptr;
  uint4* sr = sum_out ? reinterpret_cast<uint4*>(sum_out + static_cast<int64_t>(row) * h) : nullptr;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = tid + 256 * i;
    if (c < nv) {
      unpack8(xr[c], v[i]);
      if (ar) {
        float a[8];
        unpack8(ar[c], a);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += a[j];
        const uint4 s = pack8(v[i]);  // the residual sum in the activations' dtype
        if (sr) sr[c] = s;
        unpack8(s, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(h) + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * h);
  const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = tid + 256 * i;
    if (c < nv) {
      const float4 wa = __ldg(w4 + 2 * c), wb = __ldg(w4 + 2 * c + 1);
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * r * (1.0f + wv[j]);
      orow[c] = pack8(o);
    }
  }
}

template <int VPT>
cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* add, uint16_t* sum_out, const float* w, float eps,
                           uint16_t* out, int rows, int h, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, rmsnorm_rows_kernel<VPT>, x, add, sum_out, w, eps, out, rows, h);
}

}  // namespace

cudaError_t rmsnorm_rows(const void* x, const void* add, void* sum_out, const float* w, float eps, void* out, int rows,
                         int h, cudaStream_t stream) {
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (rows <= 0 || h <= 0 || (h & 7) || h > 8192 || !x || !w || !out || !al(x) || !al(out) || !al(w) ||
      (add && !al(add)) || (sum_out && (!add || !al(sum_out))))
    return cudaErrorInvalidValue;
  const auto* xx = static_cast<const uint16_t*>(x);
  const auto* aa = static_cast<const uint16_t*>(add);
  auto* so = static_cast<uint16_t*>(sum_out);
  auto* oo = static_cast<uint16_t*>(out);
  const int vpt = (h / 8 + 255) / 256;
  if (vpt <= 1) return launch_rmsnorm<1>(xx, aa, so, w, eps, oo, rows, h, stream);
  if (vpt <= 2) return launch_rmsnorm<2>(xx, aa, so, w, eps, oo, rows, h, stream);
  return launch_rmsnorm<4>(xx, aa, so, w, eps, oo, rows, h, stream);
}

}  // namespace gdn
