// Token-by-token gated delta rule (decode, and the recurrence-only op).
//
// Math per (sequence b, v-head h, token t), fp32 (9B/reference.py:28-34; 9B/kernels/gdn_compute.cpp:51-122):
//   q^ = q rsqrt(|q|^2 + 1e-6) * scale,  k^ = k rsqrt(|k|^2 + 1e-6)        (GQA: k-head = h / (Hv/Hk))
//   S' = exp(g) S;   u = beta (v - S'^T k^);   S <- S' + k^ u^T;   o = S^T q^ = S'^T q^ + (q^.k^) u
// One CTA of 256 threads owns the 128 x 128 fp32 state of one (b, h).  Thread t holds rows
// 16*(t/32) .. +15 of the column quad 4*(t%32) .. +3 in registers, so every warp moves 512 contiguous
// bytes per row and the state is read once and written once per call.  S^T k and S^T q come out of one
// pass (partials per row group reduced through shared memory); the output is either raw o or the gated
// RMSNorm y = RMSNorm(o) * w * SiLU(z) in bf16 (9B/kernels/layer_compute.cpp:287-395).
#include <cuda_bf16.h>

#include "gemm.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace gdn {

constexpr int kRecThreads = 256;

__global__ void __launch_bounds__(kRecThreads, 2) recurrence_kernel(RecurrenceArgs a) {
  const int b = blockIdx.x / a.Hv, h = blockIdx.x % a.Hv;
  const int kh = h / (a.Hv / a.Hk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c0 = lane * 4;    // first of this thread's 4 columns
  const int r0 = warp * 16;   // first of this thread's 16 rows

  __shared__ __align__(16) float s_q[kHeadDim], s_k[kHeadDim], s_v[kHeadDim], s_z[kHeadDim];
  __shared__ __align__(16) float s_u[kHeadDim], s_o[kHeadDim];  // s_u is read as float4
  __shared__ float4 s_rk[8][32], s_rq[8][32];  // per row-group partials of S'^T k and S'^T q
  __shared__ float s_red[4][4];
  __shared__ float s_scal[2];

  griddep_launch_dependents();  // the successor (out_proj) only reads y after waiting for this kernel
  float* S = a.state + (static_cast<int64_t>(b) * a.Hv + h) * kHeadDim * kHeadDim;
  float4 st[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    st[i] = __ldcs(reinterpret_cast<const float4*>(S + (r0 + i) * kHeadDim + c0));
  // The state is not written by the kernel this one may overlap (the in_proj GEMM of the same call, which
  // itself started only after the previous call had finished); the token inputs are.
  griddep_wait();

#pragma unroll 1
  for (int t = 0; t < a.T; ++t) {
    const int64_t row = static_cast<int64_t>(b) * a.T + t;
    // ---- load the token's vectors and reduce |q|^2, |k|^2, q.k (warps 0..3, one element per thread)
    if (tid < kHeadDim) {
      const float qv = a.q[row * a.q_tok + kh * a.q_head + tid];
      const float kv = a.k[row * a.k_tok + kh * a.k_head + tid];
      s_q[tid] = qv;
      s_k[tid] = kv;
      s_v[tid] = a.v[row * a.v_tok + h * a.v_head + tid];
      if (a.z) s_z[tid] = a.z[row * a.z_tok + h * a.z_head + tid];
      float sq = qv * qv, sk = kv * kv, sqk = qv * kv;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, off);
        sk += __shfl_xor_sync(0xffffffffu, sk, off);
        sqk += __shfl_xor_sync(0xffffffffu, sqk, off);
      }
      if (lane == 0) {
        s_red[warp][0] = sq;
        s_red[warp][1] = sk;
        s_red[warp][2] = sqk;
      }
    } else if (tid == kHeadDim) {
      s_scal[0] = expf(a.g[row * a.g_tok + h * a.g_head]);
      s_scal[1] = a.beta[row * a.b_tok + h * a.b_head];
    }
    __syncthreads();
    const float sq = s_red[0][0] + s_red[1][0] + s_red[2][0] + s_red[3][0];
    const float sk = s_red[0][1] + s_red[1][1] + s_red[2][1] + s_red[3][1];
    const float sqk = s_red[0][2] + s_red[1][2] + s_red[2][2] + s_red[3][2];
    const float rq = a.l2norm ? rsqrtf(sq + 1e-6f) * a.scale : a.scale;
    const float rk = a.l2norm ? rsqrtf(sk + 1e-6f) : 1.0f;
    const float qk = sqk * rq * rk;
    const float d = s_scal[0], beta = s_scal[1];

    // ---- decay and the two projections over this thread's 16 rows
    float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = pk;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float kr = s_k[r0 + i] * rk, qr = s_q[r0 + i] * rq;
      float4& s = st[i];
      s.x *= d;
      s.y *= d;
      s.z *= d;
      s.w *= d;
      pk.x += kr * s.x; pk.y += kr * s.y; pk.z += kr * s.z; pk.w += kr * s.w;
      pq.x += qr * s.x; pq.y += qr * s.y; pq.z += qr * s.z; pq.w += qr * s.w;
    }
    s_rk[warp][lane] = pk;
    s_rq[warp][lane] = pq;
    __syncthreads();
    if (tid < kHeadDim) {
      const int quad = tid >> 2, comp = tid & 3;
      float ks = 0.f, qs = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        ks += reinterpret_cast<const float*>(&s_rk[w][quad])[comp];
        qs += reinterpret_cast<const float*>(&s_rq[w][quad])[comp];
      }
      const float u = beta * (s_v[tid] - ks);
      const float o = qs + qk * u;
      s_u[tid] = u;
      s_o[tid] = o;
      float so = o * o;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) so += __shfl_xor_sync(0xffffffffu, so, off);
      if (lane == 0) s_red[warp][3] = so;
    }
    __syncthreads();
    // ---- rank-1 update of the state
    const float4 u4 = *reinterpret_cast<const float4*>(&s_u[c0]);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float kr = s_k[r0 + i] * rk;
      st[i].x += kr * u4.x;
      st[i].y += kr * u4.y;
      st[i].z += kr * u4.z;
      st[i].w += kr * u4.w;
    }
    // ---- output
    if (tid < kHeadDim) {
      const float o = s_o[tid];
      if (a.z) {
        const float ms = (s_red[0][3] + s_red[1][3] + s_red[2][3] + s_red[3][3]) * (1.0f / kHeadDim);
        const float y = o * rsqrtf(ms + a.eps) * a.norm_w[tid] * silu_f(s_z[tid]);
        static_cast<__nv_bfloat16*>(a.y)[row * a.y_tok + h * a.y_head + tid] = __float2bfloat16_rn(y);
      } else {
        a.o[row * a.o_tok + h * a.o_head + tid] = o;
      }
    }
    __syncthreads();  // shared vectors are rewritten by the next token
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) __stcs(reinterpret_cast<float4*>(S + (r0 + i) * kHeadDim + c0), st[i]);
}

cudaError_t recurrence_forward(const RecurrenceArgs& a, cudaStream_t stream, bool pdl) {
  if (a.B <= 0 || a.T <= 0 || a.Hk <= 0 || a.Hv <= 0 || a.Hv % a.Hk) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.B * a.Hv));
  cfg.blockDim = dim3(kRecThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, recurrence_kernel, a);
}


// ---------------------------------------------------------------------------------------------
// Layer decode step with the causal conv fused
// ---------------------------------------------------------------------------------------------
// One CTA per (sequence b, v-head h), as recurrence_kernel, with the causal conv (K = 4) + SiLU of its
// q, k and v channels and the conv-state roll (9B/kernels/layer_reader.cpp:184-197; HF
// torch_causal_conv1d_update).  The v-heads of one GQA group share the q/k channels of their k-head, so
// they run as one thread-block cluster: every CTA reads the q/k history, arrives on the cluster barrier,
// and only cluster rank 0 rolls the q/k state after the barrier, once every sibling has read it.  Before
// waiting for the in_proj GEMM each CTA loads its recurrent state, the conv history and the conv weights
// (cp.async into shared memory), all of which that kernel leaves untouched.
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

constexpr int kStepCh = 3 * kHeadDim;  // q, k, v channels of one CTA

__global__ void __launch_bounds__(kRecThreads, 2) decode_step_kernel(RecurrenceArgs a) {
  const int b = blockIdx.x / a.Hv, h = blockIdx.x % a.Hv;
  const int ratio = a.Hv / a.Hk, kh = h / ratio;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c0 = lane * 4, r0 = warp * 16;

  __shared__ __align__(16) float4 s_w[kStepCh];  // conv taps of each channel
  __shared__ float s_hist[3][kStepCh];           // conv history, oldest first
  __shared__ __align__(16) float s_q[kHeadDim], s_k[kHeadDim], s_v[kHeadDim], s_z[kHeadDim];
  __shared__ __align__(16) float s_u[kHeadDim], s_o[kHeadDim];
  __shared__ float4 s_rk[8][32], s_rq[8][32];
  __shared__ float s_red[4][4];
  __shared__ float s_scal[2];

  griddep_launch_dependents();  // the successor (out_proj) reads y only after waiting for this kernel
  // CTA-local channel idx -> conv channel: q (0..127), k (128..255), v (256..383)
  auto channel = [&](int idx) {
    if (idx < kHeadDim) return kh * kHeadDim + idx;
    if (idx < 2 * kHeadDim) return a.k_conv + kh * kHeadDim + idx - kHeadDim;
    return a.v_conv + h * kHeadDim + idx - 2 * kHeadDim;
  };
  const int64_t row = b;  // T = 1: token row = sequence
  float* cs = a.conv_state + row * 3 * a.conv_dim;
  for (int idx = tid; idx < kStepCh; idx += kRecThreads) {
    const int c = channel(idx);
    cp_async16(&s_w[idx], a.conv_w + static_cast<int64_t>(c) * 4);
#pragma unroll
    for (int i = 0; i < 3; ++i) cp_async4(&s_hist[i][idx], cs + static_cast<int64_t>(i) * a.conv_dim + c);
  }
  float* S = a.state + (static_cast<int64_t>(b) * a.Hv + h) * kHeadDim * kHeadDim;
  float4 st[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    st[i] = __ldcs(reinterpret_cast<const float4*>(S + (r0 + i) * kHeadDim + c0));
  griddep_wait();  // the in_proj outputs are ready

  // ---- raw inputs of this thread's channels (tid, and tid + 256 for tid < 128), z, gates: issued while
  //      the state and history loads are still in flight
  auto raw = [&](int idx) {
    if (idx < kHeadDim) return a.q[row * a.q_tok + kh * a.q_head + idx];
    if (idx < 2 * kHeadDim) return a.k[row * a.k_tok + kh * a.k_head + idx - kHeadDim];
    return a.v[row * a.v_tok + h * a.v_head + idx - 2 * kHeadDim];
  };
  const float x0 = raw(tid);
  const float x1 = tid < kStepCh - kRecThreads ? raw(tid + kRecThreads) : 0.f;
  if (tid >= kHeadDim) {  // threads 128..255 have one conv channel, 0..127 two
    s_z[tid - kHeadDim] = a.z[row * a.z_tok + h * a.z_head + tid - kHeadDim];
    if (tid == kHeadDim) {
      const float ga = a.g[row * a.g_tok + h * a.g_head], gb = a.beta[row * a.b_tok + h * a.b_head];
      if (a.a_log) {  // raw projections: g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
        // (9B/kernels/layer_compute.cpp:160-166,176-177)
        s_scal[0] = expf(-expf(a.a_log[h]) * softplus_f(ga + a.dt_bias[h]));
        s_scal[1] = sigmoid_f(gb);
      } else {
        s_scal[0] = expf(ga);
        s_scal[1] = gb;
      }
    }
  }
  cp_async_wait_all();              // each thread reads back only the history it copied
  if (ratio > 1) cluster_arrive();  // this CTA has read the shared q/k history

  // ---- conv + SiLU; the v state (own) rolls now, the q/k state (rank 0) at the end, after the whole
  //      cluster has read the old history
  auto conv = [&](int idx, float x) {
    const float4 w = s_w[idx];
    const float y = silu_fast(w.x * s_hist[0][idx] + w.y * s_hist[1][idx] + w.z * s_hist[2][idx] + w.w * x);
    if (idx < kHeadDim) s_q[idx] = y;
    else if (idx < 2 * kHeadDim) s_k[idx - kHeadDim] = y;
    else s_v[idx - 2 * kHeadDim] = y;
  };
  auto roll = [&](int idx, float x) {
    const int c = channel(idx);
    cs[c] = s_hist[1][idx];
    cs[a.conv_dim + c] = s_hist[2][idx];
    cs[2 * static_cast<int64_t>(a.conv_dim) + c] = x;
  };
  conv(tid, x0);
  if (tid < kStepCh - kRecThreads) {
    conv(tid + kRecThreads, x1);
    roll(tid + kRecThreads, x1);  // v channels 128..255 of this head
  }
  __syncthreads();
  // ---- |q|^2, |k|^2, q.k (warps 0..3)
  if (tid < kHeadDim) {
    const float qv = s_q[tid], kv = s_k[tid];
    float sq = qv * qv, sk = kv * kv, sqk = qv * kv;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, off);
      sk += __shfl_xor_sync(0xffffffffu, sk, off);
      sqk += __shfl_xor_sync(0xffffffffu, sqk, off);
    }
    if (lane == 0) {
      s_red[warp][0] = sq;
      s_red[warp][1] = sk;
      s_red[warp][2] = sqk;
    }
  }
  __syncthreads();
  const float sq = s_red[0][0] + s_red[1][0] + s_red[2][0] + s_red[3][0];
  const float sk = s_red[0][1] + s_red[1][1] + s_red[2][1] + s_red[3][1];
  const float sqk = s_red[0][2] + s_red[1][2] + s_red[2][2] + s_red[3][2];
  const float rq = rsqrtf(sq + 1e-6f) * a.scale, rk = rsqrtf(sk + 1e-6f);
  const float qk = sqk * rq * rk;
  const float d = s_scal[0], beta = s_scal[1];

  // ---- decay and the two projections over this thread's 16 rows
  float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = pk;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float kr = s_k[r0 + i] * rk, qr = s_q[r0 + i] * rq;
    float4& s = st[i];
    s.x *= d;
    s.y *= d;
    s.z *= d;
    s.w *= d;
    pk.x += kr * s.x; pk.y += kr * s.y; pk.z += kr * s.z; pk.w += kr * s.w;
    pq.x += qr * s.x; pq.y += qr * s.y; pq.z += qr * s.z; pq.w += qr * s.w;
  }
  s_rk[warp][lane] = pk;
  s_rq[warp][lane] = pq;
  __syncthreads();
  if (tid < kHeadDim) {
    const int quad = tid >> 2, comp = tid & 3;
    float ks = 0.f, qs = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      ks += reinterpret_cast<const float*>(&s_rk[w][quad])[comp];
      qs += reinterpret_cast<const float*>(&s_rq[w][quad])[comp];
    }
    const float u = beta * (s_v[tid] - ks);
    const float o = qs + qk * u;
    s_u[tid] = u;
    s_o[tid] = o;
    float so = o * o;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) so += __shfl_xor_sync(0xffffffffu, so, off);
    if (lane == 0) s_red[warp][3] = so;
  }
  __syncthreads();
  // ---- rank-1 update of the state
  const float4 u4 = *reinterpret_cast<const float4*>(&s_u[c0]);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float kr = s_k[r0 + i] * rk;
    st[i].x += kr * u4.x;
    st[i].y += kr * u4.y;
    st[i].z += kr * u4.z;
    st[i].w += kr * u4.w;
  }
  // ---- gated RMSNorm output
  if (tid < kHeadDim) {
    const float ms = (s_red[0][3] + s_red[1][3] + s_red[2][3] + s_red[3][3]) * (1.0f / kHeadDim);
    const float y = s_o[tid] * rsqrtf(ms + a.eps) * a.norm_w[tid] * silu_f(s_z[tid]);
    static_cast<__nv_bfloat16*>(a.y)[row * a.y_tok + h * a.y_head + tid] = __float2bfloat16_rn(y);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) __stcs(reinterpret_cast<float4*>(S + (r0 + i) * kHeadDim + c0), st[i]);
  // q and k channels, last: by now every sibling has long read the old history
  if (ratio > 1) cluster_wait();
  if (ratio == 1 || cluster_ctarank() == 0) roll(tid, x0);
}

cudaError_t decode_step_forward(const RecurrenceArgs& a, cudaStream_t stream) {
  if (a.B <= 0 || a.T != 1 || a.Hk <= 0 || a.Hv <= 0 || a.Hv % a.Hk || a.Hv / a.Hk > 8 || !a.z || !a.y ||
      !a.conv_w || !a.conv_state || a.conv_dim <= 0 || !a.l2norm)
    return cudaErrorInvalidValue;
  const int ratio = a.Hv / a.Hk;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.B * a.Hv));
  cfg.blockDim = dim3(kRecThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (ratio > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(ratio);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  count_launch();
  return cudaLaunchKernelEx(&cfg, decode_step_kernel, a);
}

}  // namespace gdn
