// Chunked (WY/UT) prefill of the gated delta rule, fused with l2norm, gating and the gated RMSNorm.
//
// The reference runs prefill token by token (9B/README.md:150-151,157: "chunked prefill not done yet"); the
// chunked form is pinned by HF torch_chunk_gated_delta_rule (modeling_qwen3_5.py:234-311) and by the
// sequential rule (9B/reference.py:28-34).  One CTA owns one (sequence, v-head) and walks its chunks of
// C = 64 tokens in order, carrying the fp32 128 x 128 state in shared memory.  Per chunk, with
// in-chunk cumulative log decay G_i and everything in fp32:
//   M_ij = beta_i (k_i.k_j) e^(G_i-G_j) (j < i),  A_ij = (q_i.k_j) e^(G_i-G_j) (j <= i)
//   T    = (I + M)^-1                     blocked: 16x16 diagonal inverses, then off-diagonal blocks
//   R    = beta v - (beta e^G k) S;   Vn = T R          (= U - W S of the WY form)
//   O    = (e^G q) S + A Vn  ->  y = RMSNorm(O) * w * SiLU(z)  (bf16)
//   S   <- e^(G_C) S + (e^(G_C - G) k)^T Vn
#include <cuda_bf16.h>

#include "gemm.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace gdn {

constexpr int kC = 64;        // chunk
constexpr int kD = 128;       // head dim
constexpr int kLdT = 132;     // padded row stride of token-major [64][128] tiles
constexpr int kLdC = 68;      // padded row stride of [64][64] tiles
constexpr int kChunkThreads = 256;

struct ChunkSmem {
  float q[kC * kLdT];   // q^ * scale
  float k[kC * kLdT];   // k^
  float v[kC * kLdT];   // v -> R -> Vn
  float s[kD * kD];     // state
  float m[kC * kLdC];   // M (strictly lower)
  float t[kC * kLdC];   // T = (I + M)^-1
  float a[kC * kLdC];   // A (lower incl. diagonal)
  float x[3 * 16 * 16]; // block-inverse temporaries
  float G[kC], beta[kC], eG[kC], eCG[kC];
};

__global__ void __launch_bounds__(kChunkThreads, 1) chunk_prefill_kernel(ChunkArgs p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>(smem_raw);
  const int b = blockIdx.x / p.Hv, h = blockIdx.x % p.Hv;
  const int kh = h / (p.Hv / p.Hk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kd = p.Hk * kD;
  const float scale = rsqrtf(static_cast<float>(kD));
  const float neg_a = -expf(p.a_log[h]), dtb = p.dt_bias[h];

  float* Sg = p.state + (static_cast<int64_t>(b) * p.Hv + h) * kD * kD;
  for (int i = tid; i < kD * kD / 4; i += kChunkThreads)
    reinterpret_cast<float4*>(sm.s)[i] = reinterpret_cast<const float4*>(Sg)[i];

  const int nchunks = (p.T + kC - 1) / kC;
  // 64 x 128 output tiles: rows tr + 16 i, columns 8 tc + j
  const int tr = tid >> 4, tc = tid & 15;

#pragma unroll 1
  for (int ch = 0; ch < nchunks; ++ch) {
    const int t0 = ch * kC;
    const int L = min(kC, p.T - t0);
    // ---------------- load q, k (l2-normalised), v; gating scalars ----------------
    for (int tt = warp; tt < kC; tt += 8) {
      float4 qv = make_float4(0.f, 0.f, 0.f, 0.f), kv = qv, vv = qv;
      if (tt < L) {
        const int64_t row = static_cast<int64_t>(b) * p.T + t0 + tt;
        const float* base = p.qkv + row * p.qkv_ld;
        qv = reinterpret_cast<const float4*>(base + kh * kD)[lane];
        kv = reinterpret_cast<const float4*>(base + kd + kh * kD)[lane];
        vv = reinterpret_cast<const float4*>(base + 2 * kd + h * kD)[lane];
      }
      float sq = qv.x * qv.x + qv.y * qv.y + qv.z * qv.z + qv.w * qv.w;
      float sk = kv.x * kv.x + kv.y * kv.y + kv.z * kv.z + kv.w * kv.w;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, off);
        sk += __shfl_xor_sync(0xffffffffu, sk, off);
      }
      const float rq = rsqrtf(sq + 1e-6f) * scale, rk = rsqrtf(sk + 1e-6f);
      *reinterpret_cast<float4*>(&sm.q[tt * kLdT + 4 * lane]) = make_float4(qv.x * rq, qv.y * rq, qv.z * rq, qv.w * rq);
      *reinterpret_cast<float4*>(&sm.k[tt * kLdT + 4 * lane]) = make_float4(kv.x * rk, kv.y * rk, kv.z * rk, kv.w * rk);
      *reinterpret_cast<float4*>(&sm.v[tt * kLdT + 4 * lane]) = vv;
    }
    if (warp == 0) {
      // g and beta for tokens lane and lane + 32, then an inclusive scan of g over the chunk.
      float g2[2], b2[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int tt = lane + 32 * i;
        g2[i] = 0.f;
        b2[i] = 0.f;
        if (tt < L) {
          const float* pr = p.proj + (static_cast<int64_t>(b) * p.T + t0 + tt) * p.proj_ld;
          g2[i] = neg_a * softplus_f(pr[p.a_off + h] + dtb);
          b2[i] = sigmoid_f(pr[p.b_off + h]);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float n = __shfl_up_sync(0xffffffffu, g2[i], off);
          if (lane >= off) g2[i] += n;
        }
      }
      g2[1] += __shfl_sync(0xffffffffu, g2[0], 31);
      const float gC = __shfl_sync(0xffffffffu, g2[1], 31);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int tt = lane + 32 * i;
        sm.G[tt] = g2[i];
        sm.beta[tt] = b2[i];
        sm.eG[tt] = expf(g2[i]);
        sm.eCG[tt] = expf(gC - g2[i]);
      }
    }
    __syncthreads();

    // ---------------- M and A (64 x 64, inner dim 128) ----------------
    {
      const int ti = tid >> 4, tj = tid & 15;  // rows ti + 16 i, cols tj + 16 j
      float am[4][4] = {}, aa[4][4] = {};
#pragma unroll 2
      for (int kk = 0; kk < kD; kk += 4) {
        float4 kr[4], qr[4], kc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          kr[i] = *reinterpret_cast<const float4*>(&sm.k[(ti + 16 * i) * kLdT + kk]);
          qr[i] = *reinterpret_cast<const float4*>(&sm.q[(ti + 16 * i) * kLdT + kk]);
          kc[i] = *reinterpret_cast<const float4*>(&sm.k[(tj + 16 * i) * kLdT + kk]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            am[i][j] += kr[i].x * kc[j].x + kr[i].y * kc[j].y + kr[i].z * kc[j].z + kr[i].w * kc[j].w;
            aa[i][j] += qr[i].x * kc[j].x + qr[i].y * kc[j].y + qr[i].z * kc[j].z + qr[i].w * kc[j].w;
          }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = ti + 16 * i, c = tj + 16 * j;
          const float dec = c <= r ? expf(sm.G[r] - sm.G[c]) : 0.f;
          sm.m[r * kLdC + c] = c < r ? sm.beta[r] * am[i][j] * dec : 0.f;
          sm.a[r * kLdC + c] = aa[i][j] * dec;
        }
    }
    __syncthreads();

    // ---------------- T = (I + M)^-1, blocked 4 x 4 of 16 x 16 ----------------
    if (warp < 4) {
      // Diagonal block `warp` by forward substitution; lanes 0..15 own columns.
      const int o = warp * 16;
      const int j = lane & 15;
      if (lane < 16) {
        for (int i = 0; i < 16; ++i) sm.t[(o + i) * kLdC + o + j] = (i == j) ? 1.f : 0.f;
      }
      __syncwarp();
      for (int i = 1; i < 16; ++i) {
        float acc = 0.f;
        if (lane < 16 && j < i) {
          for (int mm = j; mm < i; ++mm) acc += sm.m[(o + i) * kLdC + o + mm] * sm.t[(o + mm) * kLdC + o + j];
        }
        __syncwarp();
        if (lane < 16 && j < i) sm.t[(o + i) * kLdC + o + j] = -acc;
        __syncwarp();
      }
    } else {
      // Zero the strictly-upper off-diagonal blocks of T.
      for (int idx = tid - 128; idx < 6 * 256; idx += 128) {
        const int blk = idx >> 8, e = idx & 255;
        const int pairs[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};
        const int ra = pairs[blk][0], cb = pairs[blk][1];
        sm.t[(ra * 16 + (e >> 4)) * kLdC + cb * 16 + (e & 15)] = 0.f;
      }
    }
    __syncthreads();
    for (int d = 1; d < 4; ++d) {
      const int nb = 4 - d;
      // X_ab = sum_{c=b}^{a-1} M_ac T_cb   (a = b + d)
      for (int idx = tid; idx < nb * 256; idx += kChunkThreads) {
        const int bb = idx >> 8, e = idx & 255, i = e >> 4, j = e & 15;
        const int aa = bb + d;
        float acc = 0.f;
        for (int c = bb; c < aa; ++c)
          for (int mm = 0; mm < 16; ++mm)
            acc += sm.m[(aa * 16 + i) * kLdC + c * 16 + mm] * sm.t[(c * 16 + mm) * kLdC + bb * 16 + j];
        sm.x[idx] = acc;
      }
      __syncthreads();
      // T_ab = -T_aa X_ab
      for (int idx = tid; idx < nb * 256; idx += kChunkThreads) {
        const int bb = idx >> 8, e = idx & 255, i = e >> 4, j = e & 15;
        const int aa = bb + d;
        float acc = 0.f;
        for (int mm = 0; mm <= i; ++mm) acc += sm.t[(aa * 16 + i) * kLdC + aa * 16 + mm] * sm.x[bb * 256 + mm * 16 + j];
        sm.t[(aa * 16 + i) * kLdC + bb * 16 + j] = -acc;
      }
      __syncthreads();
    }

    // ---------------- R = beta v - (beta e^G k) S   (in place over v) ----------------
    {
      float acc[4][8] = {};
#pragma unroll 2
      for (int kk = 0; kk < kD; ++kk) {
        const float4 s0 = *reinterpret_cast<const float4*>(&sm.s[kk * kD + 8 * tc]);
        const float4 s1 = *reinterpret_cast<const float4*>(&sm.s[kk * kD + 8 * tc + 4]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float kv = sm.k[(tr + 16 * i) * kLdT + kk];
          acc[i][0] += kv * s0.x; acc[i][1] += kv * s0.y; acc[i][2] += kv * s0.z; acc[i][3] += kv * s0.w;
          acc[i][4] += kv * s1.x; acc[i][5] += kv * s1.y; acc[i][6] += kv * s1.z; acc[i][7] += kv * s1.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = tr + 16 * i;
        const float bt = sm.beta[r], bg = bt * sm.eG[r];
        float* vr = &sm.v[r * kLdT + 8 * tc];
#pragma unroll
        for (int j = 0; j < 8; ++j) vr[j] = bt * vr[j] - bg * acc[i][j];
      }
    }
    __syncthreads();
    // ---------------- Vn = T R ----------------
    {
      float acc[4][8] = {};
#pragma unroll 2
      for (int mm = 0; mm < kC; ++mm) {
        const float4 r0 = *reinterpret_cast<const float4*>(&sm.v[mm * kLdT + 8 * tc]);
        const float4 r1 = *reinterpret_cast<const float4*>(&sm.v[mm * kLdT + 8 * tc + 4]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float tv = sm.t[(tr + 16 * i) * kLdC + mm];
          acc[i][0] += tv * r0.x; acc[i][1] += tv * r0.y; acc[i][2] += tv * r0.z; acc[i][3] += tv * r0.w;
          acc[i][4] += tv * r1.x; acc[i][5] += tv * r1.y; acc[i][6] += tv * r1.z; acc[i][7] += tv * r1.w;
        }
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float* vr = &sm.v[(tr + 16 * i) * kLdT + 8 * tc];
#pragma unroll
        for (int j = 0; j < 8; ++j) vr[j] = acc[i][j];
      }
    }
    __syncthreads();
    // ---------------- O = (e^G q) S + A Vn -> gated RMSNorm -> y ----------------
    {
      float acc[4][8] = {}, acc2[4][8] = {};
#pragma unroll 2
      for (int kk = 0; kk < kD; ++kk) {
        const float4 s0 = *reinterpret_cast<const float4*>(&sm.s[kk * kD + 8 * tc]);
        const float4 s1 = *reinterpret_cast<const float4*>(&sm.s[kk * kD + 8 * tc + 4]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float qv = sm.q[(tr + 16 * i) * kLdT + kk];
          acc[i][0] += qv * s0.x; acc[i][1] += qv * s0.y; acc[i][2] += qv * s0.z; acc[i][3] += qv * s0.w;
          acc[i][4] += qv * s1.x; acc[i][5] += qv * s1.y; acc[i][6] += qv * s1.z; acc[i][7] += qv * s1.w;
        }
      }
#pragma unroll 2
      for (int mm = 0; mm < kC; ++mm) {
        const float4 r0 = *reinterpret_cast<const float4*>(&sm.v[mm * kLdT + 8 * tc]);
        const float4 r1 = *reinterpret_cast<const float4*>(&sm.v[mm * kLdT + 8 * tc + 4]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float av = sm.a[(tr + 16 * i) * kLdC + mm];
          acc2[i][0] += av * r0.x; acc2[i][1] += av * r0.y; acc2[i][2] += av * r0.z; acc2[i][3] += av * r0.w;
          acc2[i][4] += av * r1.x; acc2[i][5] += av * r1.y; acc2[i][6] += av * r1.z; acc2[i][7] += av * r1.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = tr + 16 * i;
        float o[8], ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] = sm.eG[r] * acc[i][j] + acc2[i][j];
          ss += o[j] * o[j];
        }
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (r < L) {
          const float rstd = rsqrtf(ss * (1.0f / kD) + p.eps);
          const int64_t row = static_cast<int64_t>(b) * p.T + t0 + r;
          const float* zr = p.proj + row * p.proj_ld + p.z_off + h * kD + 8 * tc;
          __nv_bfloat16* yr = static_cast<__nv_bfloat16*>(p.y) + row * (static_cast<int64_t>(p.Hv) * kD) + h * kD + 8 * tc;
          uint32_t pk[4];
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const float y0 = o[j] * rstd * p.norm_w[8 * tc + j] * silu_f(zr[j]);
            const float y1 = o[j + 1] * rstd * p.norm_w[8 * tc + j + 1] * silu_f(zr[j + 1]);
            __nv_bfloat162 hh = __floats2bfloat162_rn(y0, y1);
            pk[j / 2] = *reinterpret_cast<uint32_t*>(&hh);
          }
          *reinterpret_cast<uint4*>(yr) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
    __syncthreads();
    // ---------------- S <- e^(G_C) S + (e^(G_C - G) k)^T Vn ----------------
    {
      const float eC = sm.eG[kC - 1];
      float acc[8][8] = {};
#pragma unroll 2
      for (int tt = 0; tt < kC; ++tt) {
        const float w = sm.eCG[tt];
        const float4 v0 = *reinterpret_cast<const float4*>(&sm.v[tt * kLdT + 8 * tc]);
        const float4 v1 = *reinterpret_cast<const float4*>(&sm.v[tt * kLdT + 8 * tc + 4]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float kv = sm.k[tt * kLdT + tr + 16 * i] * w;
          acc[i][0] += kv * v0.x; acc[i][1] += kv * v0.y; acc[i][2] += kv * v0.z; acc[i][3] += kv * v0.w;
          acc[i][4] += kv * v1.x; acc[i][5] += kv * v1.y; acc[i][6] += kv * v1.z; acc[i][7] += kv * v1.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float* sr = &sm.s[(tr + 16 * i) * kD + 8 * tc];
#pragma unroll
        for (int j = 0; j < 8; ++j) sr[j] = eC * sr[j] + acc[i][j];
      }
    }
    __syncthreads();
  }
  for (int i = tid; i < kD * kD / 4; i += kChunkThreads)
    reinterpret_cast<float4*>(Sg)[i] = reinterpret_cast<const float4*>(sm.s)[i];
}

cudaError_t chunk_prefill(const ChunkArgs& a, cudaStream_t stream) {
  if (a.B <= 0 || a.T <= 0 || a.Hk <= 0 || a.Hv <= 0 || a.Hv % a.Hk) return cudaErrorInvalidValue;
  if ((a.qkv_ld & 3) || (a.proj_ld & 3) || (a.z_off & 7)) return cudaErrorInvalidValue;
  const int smem = static_cast<int>(sizeof(ChunkSmem));
  cudaError_t e = cudaFuncSetAttribute(chunk_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  count_launch();
  chunk_prefill_kernel<<<a.B * a.Hv, kChunkThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace gdn
