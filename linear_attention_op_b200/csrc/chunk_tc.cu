// Chunked (WY/UT) prefill of the gated delta rule on the tcgen05 tensor cores, fused with l2norm, gating
// and the gated RMSNorm.
//
// The reference runs prefill token by token (9B/README.md:150-151,157: chunked prefill "not done yet"); the
// chunked form is pinned by HF torch_chunk_gated_delta_rule (modeling_qwen3_5.py:234-311) and by the
// sequential rule (9B/reference.py:28-34).  Per chunk of C = 64 tokens, with in-chunk cumulative log decay
// G_t, normalised k^, scaled q^ and fp32 state S[d][v]:
//   M[t][s] = beta_t (k^_t . k^_s) e^(G_t - G_s)  (s < t),   A[t][s] = (q^_t . k^_s) e^(G_t - G_s)  (s <= t)
//   T  = (I + M)^-1
//   R  = beta (V - e^G (K^ S))           Vn = T R                     (= U - W S of the WY form)
//   O  = e^G (Q^ S) + A Vn  -> y = RMSNorm(O) * w * SiLU(z)
//   S <- e^(G_C) S + (e^(G_C - G) K^)^T Vn
//
// Two kernels:
//   chunk_prep   one CTA per (sequence, k-head, chunk), fully parallel: [K; Q] K^T on the tensor cores,
//                then per v-head of the GQA group M, A and the fp32 blocked inverse T; T (hi/lo) and A are
//                written as ready-to-copy 128B-swizzled bf16 tile images.
//   chunk_state  one CTA per (sequence, v-head), sequential over chunks; the state stays in registers as
//                S^T (thread v holds a row) and feeds three tcgen05 MMA groups per chunk:
//                  MMA1  [ (K^S)^T | (e^G Q^ S)^T ] = S^T [K^ ; e^G Q^]^T      (128 x 128, K = 128)
//                  MMA2  Vn^T = R^T T^T                                        (128 x 64,  K = 64)
//                  MMA3  dS^T = Vn^T Kd ;  O^T += Vn^T A^T                     (128 x 128 / 128 x 64)
// Precision: every operand is split into bf16 hi + lo and the products that feed the state use three
// passes (hi*hi + hi*lo + lo*hi, about 16 mantissa bits); the output-only products use hi*hi.  All tiles are
// K-major with 128-byte swizzle (64 bf16 per row), the layout the GEMM uses.
#include <cuda.h>
#include <cuda_bf16.h>

#include "gemm.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace gdn {

namespace {

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kThreads = 256;
// Per (sequence, v-head, chunk): T hi, T lo, A hi ([64 x 64] bf16 tiles) and the gates (beta, e^G,
// e^(G_C - G), 64 floats each, plus 64 unused).
constexpr int kTImageBytes = 3 * 8192 + 1024;
constexpr int kTGateOff = 3 * 8192;
// Per (sequence, k-head, chunk), independent of the gates: [k^ ; q^] hi (2 atoms of [128][64]) and k^ lo
// (2 atoms of [64][64]).  MMA1 reads them K-major (over d); MMA3 reads the same k^ rows MN-major (K = t).
constexpr int kKImageBytes = 32768 + 16384;
constexpr int kKOffKQ = 0, kKOffKL = 32768;

// Byte offset of bf16 element (r, k), k < 64, in a K-major tile with 128-byte swizzle (1024-aligned base).
__device__ __forceinline__ uint32_t sw_off(int r, int k) {
  return static_cast<uint32_t>(r * 128 + (((k >> 3) ^ (r & 7)) << 4) + ((k & 7) << 1));
}

__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

// Pack 8 floats into hi and lo uint4 (8 bf16 each): hi = bf16(x), lo = bf16(x - hi), two lanes at a time.
__device__ __forceinline__ void pack8(const float* x, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 hh = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    const float2 hf = __bfloat1622float2(hh);
    const __nv_bfloat162 ll = __floats2bfloat162_rn(x[2 * i] - hf.x, x[2 * i + 1] - hf.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&hh);
    l[i] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Contiguous global -> shared copy by the TMA engine (no tensor map, no multicast), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// D (+)= A * B^T over katoms 64-wide K atoms; A and B are K-major SW128 tiles given by the shared address of
// their first atom and the byte distance between atoms.
__device__ __forceinline__ void mma_atoms(uint32_t d, uint32_t a, uint32_t a_stride, uint32_t b, uint32_t b_stride,
                                          int katoms, uint32_t idesc, bool accumulate) {
  for (int at = 0; at < katoms; ++at) {
    const uint64_t da = sdesc_k_sw128(a + at * a_stride), db = sdesc_k_sw128(b + at * b_stride);
#pragma unroll
    for (int k = 0; k < 4; ++k) umma_f16(d, da + 2 * k, db + 2 * k, idesc, (accumulate || at || k) ? 1u : 0u);
  }
}

// Raw gate inputs (a, b columns of the in_proj output) of v-head h for the chunk's tokens lane, lane + 32.
struct GateRaw {
  float a[2], b[2];
};
__device__ __forceinline__ GateRaw gates_load(const float* proj, int64_t proj_ld, int64_t a_off, int64_t b_off,
                                              int64_t row0, int L, int h, int lane) {
  GateRaw r;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int t = lane + 32 * i;
    r.a[i] = r.b[i] = 0.f;
    if (t < L) {
      const float* pr = proj + (row0 + t) * proj_ld;
      r.a[i] = pr[a_off + h];
      r.b[i] = pr[b_off + h];
    }
  }
  return r;
}

// Per-chunk gating scalars of one v-head from its raw inputs: G (inclusive cumsum of g), beta, e^G,
// e^(G_C - G).  Warp-level.
__device__ __forceinline__ void chunk_gates(const GateRaw& raw, int L, float neg_a, float dtb, int lane, float* G,
                                            float* beta, float* eG, float* eCG) {
  float g2[2], b2[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int t = lane + 32 * i;
    g2[i] = t < L ? neg_a * softplus_f(raw.a[i] + dtb) : 0.f;
    b2[i] = t < L ? sigmoid_f(raw.b[i]) : 0.f;
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
    const int t = lane + 32 * i;
    G[t] = g2[i];
    beta[t] = b2[i];
    if (eG) eG[t] = expf(g2[i]);
    if (eCG) eCG[t] = expf(gC - g2[i]);
  }
}

// ------------------------------------------------------------------------------------------------------
// chunk_prep
// ------------------------------------------------------------------------------------------------------
constexpr int kLdF = 68;  // padded fp32 row stride of the 64 x 64 work matrices

struct PrepSmem {
  uint8_t kq_h[2 * 16384];  // [K; Q] hi: 2 atoms of [128 rows][64]
  uint8_t kq_l[2 * 16384];  // [K; Q] lo
  float m[kC * kLdF];
  float t[kC * kLdF];
  float G[kC], beta[kC], eG[kC], eCG[kC];
  uint64_t bar;
  uint32_t tmem;
};

__global__ void __launch_bounds__(kThreads, 2) chunk_prep_kernel(ChunkArgs p, uint8_t* kimg, uint8_t* timg,
                                                                  int nchunks) {
  extern __shared__ uint8_t smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ch = blockIdx.x % nchunks;
  const int kh = (blockIdx.x / nchunks) % p.Hk;
  const int b = blockIdx.x / (nchunks * p.Hk);
  const int t0 = ch * kC, L = min(kC, p.T - t0);
  const int64_t row0 = static_cast<int64_t>(b) * p.T + t0;
  const int kd = p.Hk * kD;
  const int ratio = p.Hv / p.Hk;
  const float scale = rsqrtf(static_cast<float>(kD));

  if (tid == 0) {
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem, 64);
    tmem_relinquish();
  }
  // The first v-head of each warp group (heads kh*ratio + 0 and + 1): its gate inputs are requested now,
  // so their latency hides behind the q/k loads and the MMA.
  const int grp0 = warp >> 2;
  GateRaw gate_raw = {};
  if ((warp & 3) == 0 && grp0 < ratio)
    gate_raw = gates_load(p.proj, p.proj_ld, p.a_off, p.b_off, row0, L, kh * ratio + grp0, lane);
  // ---- q^ and k^ rows, split into bf16 hi/lo: rows 0..63 = k, rows 64..127 = q (all 8 tokens of a warp in
  //      flight at once)
  {
    const int tb = warp;
    float4 qv[8], kv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int t = tb + 8 * u;
      qv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      kv[u] = qv[u];
      if (t < L) {
        const float* base = p.qkv + (row0 + t) * p.qkv_ld;
        qv[u] = reinterpret_cast<const float4*>(base + kh * kD)[lane];
        kv[u] = reinterpret_cast<const float4*>(base + kd + kh * kD)[lane];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int t = tb + 8 * u;
      float sq = qv[u].x * qv[u].x + qv[u].y * qv[u].y + qv[u].z * qv[u].z + qv[u].w * qv[u].w;
      float sk = kv[u].x * kv[u].x + kv[u].y * kv[u].y + kv[u].z * kv[u].z + kv[u].w * kv[u].w;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, off);
        sk += __shfl_xor_sync(0xffffffffu, sk, off);
      }
      const float rq = rsqrtf(sq + 1e-6f) * scale, rk = rsqrtf(sk + 1e-6f);
      const float kvals[4] = {kv[u].x * rk, kv[u].y * rk, kv[u].z * rk, kv[u].w * rk};
      const float qvals[4] = {qv[u].x * rq, qv[u].y * rq, qv[u].z * rq, qv[u].w * rq};
      const int d0 = 4 * lane, atom = d0 >> 6, kk = d0 & 63;
      uint32_t hk[2], lk[2], hq[2], lq[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        __nv_bfloat16 a0, a1, c0, c1;
        split_bf16(kvals[2 * i], a0, c0);
        split_bf16(kvals[2 * i + 1], a1, c1);
        __nv_bfloat162 hh(a0, a1), ll(c0, c1);
        hk[i] = *reinterpret_cast<uint32_t*>(&hh);
        lk[i] = *reinterpret_cast<uint32_t*>(&ll);
        split_bf16(qvals[2 * i], a0, c0);
        split_bf16(qvals[2 * i + 1], a1, c1);
        __nv_bfloat162 hq2(a0, a1), lq2(c0, c1);
        hq[i] = *reinterpret_cast<uint32_t*>(&hq2);
        lq[i] = *reinterpret_cast<uint32_t*>(&lq2);
      }
      *reinterpret_cast<uint2*>(sm.kq_h + atom * 16384 + sw_off(t, kk)) = make_uint2(hk[0], hk[1]);
      *reinterpret_cast<uint2*>(sm.kq_l + atom * 16384 + sw_off(t, kk)) = make_uint2(lk[0], lk[1]);
      *reinterpret_cast<uint2*>(sm.kq_h + atom * 16384 + sw_off(64 + t, kk)) = make_uint2(hq[0], hq[1]);
      *reinterpret_cast<uint2*>(sm.kq_l + atom * 16384 + sw_off(64 + t, kk)) = make_uint2(lq[0], lq[1]);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  if (tid == 0) {
    constexpr uint32_t id = idesc_dense(1, 128, 64);
    const uint32_t kqh = smem_u32(sm.kq_h), kql = smem_u32(sm.kq_l);
    mma_atoms(tmem, kqh, 16384, kqh, 16384, 2, id, false);  // [K;Q]h K_h^T
    mma_atoms(tmem, kqh, 16384, kql, 16384, 2, id, true);   // [K;Q]h K_l^T
    mma_atoms(tmem, kql, 16384, kqh, 16384, 2, id, true);   // [K;Q]l K_h^T
    umma_commit(&sm.bar);
  }
  __syncwarp();
  const bool ok = mbar_wait(&sm.bar, 0, kErrWaitAccum);
  tc_fence_after();
  // Row r of the accumulator: r < 64 -> (k_r . k_s), r >= 64 -> (q_(r-64) . k_s).  Warp w reads the rows of
  // its TMEM lane quarter (w % 4), all 64 columns: the two warp groups (warps 0-3, 4-7) each hold the whole
  // accumulator and work on different v-heads of the GQA group concurrently.
  const int q4 = warp & 3, grp = warp >> 2, gtid = tid & 127;
  const int r = q4 * 32 + lane;
  const int t_row = r & 63;
  const bool is_k = r < 64;
  const int tr = gtid >> 1, th = gtid & 1;  // T image writer: (row, 32-column half)

  // ---- the gate-independent operand image of this (sequence, k-head, chunk)
  {
    uint8_t* ki = kimg + ((static_cast<int64_t>(b) * p.Hk + kh) * nchunks + ch) * kKImageBytes;
    const uint4* kq = reinterpret_cast<const uint4*>(sm.kq_h);
#pragma unroll
    for (int i = 0; i < 8; ++i) reinterpret_cast<uint4*>(ki + kKOffKQ)[tid + i * kThreads] = kq[tid + i * kThreads];
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // k lo: rows 0..63 of both atoms of [K; Q] lo
      const int idx = tid + i * kThreads, atom = idx >> 9, e = idx & 511;
      reinterpret_cast<uint4*>(ki + kKOffKL + atom * 8192)[e] = reinterpret_cast<const uint4*>(sm.kq_l + atom * 16384)[e];
    }
  }

  __syncthreads();  // the [K; Q] tiles are free: group 1 works in that space from here on
  float* gm = grp ? reinterpret_cast<float*>(sm.kq_h) : sm.m;          // M, then read-only
  float* gt = grp ? gm + kC * kLdF : sm.t;                             // T
  float* gG = grp ? gt + kC * kLdF : sm.G;
  float* gB = gG + kC;                                                 // beta
  float* gE = gB + kC;                                                 // e^G
  float* gC = gE + kC;                                                 // e^(G_C - G)
  if (!grp) {
    gB = sm.beta;
    gE = sm.eG;
    gC = sm.eCG;
  }
  auto group_sync = [&]() { asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory"); };

  for (int j = grp; j < ratio && ok; j += 2) {
    const int h = kh * ratio + j;
    if (q4 == 0) {
      if (j != grp) gate_raw = gates_load(p.proj, p.proj_ld, p.a_off, p.b_off, row0, L, h, lane);
      chunk_gates(gate_raw, L, -expf(p.a_log[h]), p.dt_bias[h], lane, gG, gB, gE, gC);
    }
    // this warp's TMEM quarter of the [K; Q] K^T accumulator (re-read per head, so no registers stay
    // allocated to it through the inverse)
    float acc[64];
    {  // both halves in flight, one wait
      uint32_t r0[32], r1[32];
      tmem_ld32_async(tmem + (static_cast<uint32_t>(q4 * 32) << 16), r0);
      tmem_ld32_async(tmem + (static_cast<uint32_t>(q4 * 32) << 16) + 32, r1);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        acc[i] = __uint_as_float(r0[i]);
        acc[32 + i] = __uint_as_float(r1[i]);
      }
    }
    group_sync();
    uint8_t* img = timg + ((static_cast<int64_t>(b) * p.Hv + h) * nchunks + ch) * kTImageBytes;
    if (gtid < kC) {
      float* gi = reinterpret_cast<float*>(img + kTGateOff);
      gi[gtid] = gB[gtid];
      gi[kC + gtid] = gE[gtid];
      gi[2 * kC + gtid] = gC[gtid];
    }
    // Warps q4 = 0 and 2 hold rows 0..31, whose columns 32..63 are above the diagonal: M's there are never
    // read (the inverse reads only entries below the diagonal; W later lives in that quarter) and A's are
    // zeros, written without computing their exps.
    const float Gt = gG[t_row];
    const bool hi_rows = q4 & 1;
    if (is_k) {
      const float bt = gB[t_row];
      float* mrow = gm + t_row * kLdF;
#pragma unroll
      for (int s = 0; s < 32; ++s) mrow[s] = s < t_row ? bt * acc[s] * __expf(Gt - gG[s]) : 0.f;
      if (hi_rows) {
#pragma unroll
        for (int s = 32; s < kC; ++s) mrow[s] = s < t_row ? bt * acc[s] * __expf(Gt - gG[s]) : 0.f;
      }
    } else {
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        float av[8];
        if (c8 < 4 || hi_rows) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int s = 8 * c8 + i;
            av[i] = s <= t_row ? acc[s] * __expf(Gt - gG[s]) : 0.f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) av[i] = 0.f;
        }
        uint4 hi, lo;
        pack8(av, hi, lo);
        *reinterpret_cast<uint4*>(img + 16384 + sw_off(t_row, 8 * c8)) = hi;  // A tile (hi only)
      }
    }
    group_sync();
    // ---- T = (I + M)^-1 with M strictly lower triangular, by 16 x 16 blocks (T_ij = block (i, j)):
    //   1. diagonal blocks T_bb = (I + M_bb)^-1 by forward substitution, one column per thread:
    //      T[i][c] = delta(i, c) - sum_{m < i} M[i][m] T[m][c] (exact zeros above the diagonal);
    //   2. T_10 = -T_11 M_10 T_00 and T_32 = -T_33 M_32 T_22, one column per thread;
    //   3. the lower-left 32 x 32 quarter: W = M_[23][01] T_[01][01], then T_[23][01] = -T_[23][23] W.
    //   Blocks (0, 1) and (2, 3) are zeroed for step 3; the other entries above the diagonal are never
    //   written (the image writer masks them).  W lives in the unused upper-right quarter of M.
    if (gtid < kC) {
      const int o = 16 * (gtid >> 4), c = gtid & 15;
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float* mrow = gm + (o + i) * kLdF + o;
        float a0 = (i == c) ? 1.f : 0.f, a1 = 0.f;
#pragma unroll
        for (int m = 0; m + 1 < i; m += 2) {
          const float2 mm = *reinterpret_cast<const float2*>(mrow + m);
          a0 -= mm.x * x[m];
          a1 -= mm.y * x[m + 1];
        }
        if (i & 1) a0 -= mrow[i - 1] * x[i - 1];
        x[i] = a0 + a1;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) gt[(o + i) * kLdF + o + c] = x[i];
    } else {
      const int z = gtid - kC, blk = z >> 5, row = (z & 31) >> 1, half = z & 1;
      float4* dst = reinterpret_cast<float4*>(gt + (32 * blk + row) * kLdF + 32 * blk + 16 + 8 * half);
      dst[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      dst[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    group_sync();
    if (gtid < 32) {
      const int o = 32 * (gtid >> 4), c = gtid & 15;
      float tcol[16], w[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) tcol[m] = gt[(o + m) * kLdF + o + c];
#pragma unroll
      for (int r = 0; r < 16; ++r) {  // w = M_(o+16, o) T_(o, o)[:, c]
        const float4* mrow = reinterpret_cast<const float4*>(gm + (o + 16 + r) * kLdF + o);
        float acc = 0.f;
#pragma unroll
        for (int m4 = 0; m4 < 4; ++m4) {
          const float4 mm = mrow[m4];
          acc += mm.x * tcol[4 * m4] + mm.y * tcol[4 * m4 + 1] + mm.z * tcol[4 * m4 + 2] + mm.w * tcol[4 * m4 + 3];
        }
        w[r] = acc;
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) {  // T_(o+16, o)[:, c] = -T_(o+16, o+16) w
        const float* trow = gt + (o + 16 + r) * kLdF + o + 16;
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m <= r; ++m) acc += trow[m] * w[m];
        gt[(o + 16 + r) * kLdF + o + c] = -acc;
      }
    }
    group_sync();
    const int c32 = gtid & 31, r8 = 8 * (gtid >> 5);
    {
      float tcol[32], acc[8];
#pragma unroll
      for (int m = 0; m < 32; ++m) tcol[m] = gt[m * kLdF + c32];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float4* mrow = reinterpret_cast<const float4*>(gm + (32 + r8 + r) * kLdF);
        float a = 0.f;
#pragma unroll
        for (int m4 = 0; m4 < 8; ++m4) {
          const float4 mm = mrow[m4];
          a += mm.x * tcol[4 * m4] + mm.y * tcol[4 * m4 + 1] + mm.z * tcol[4 * m4 + 2] + mm.w * tcol[4 * m4 + 3];
        }
        acc[r] = a;
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) gm[(r8 + r) * kLdF + 32 + c32] = acc[r];
    }
    group_sync();
    {
      float wcol[32];
#pragma unroll
      for (int m = 0; m < 32; ++m) wcol[m] = gm[m * kLdF + 32 + c32];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float4* trow = reinterpret_cast<const float4*>(gt + (32 + r8 + r) * kLdF + 32);
        float a = 0.f;
#pragma unroll
        for (int m4 = 0; m4 < 8; ++m4) {
          const float4 tt = trow[m4];
          a += tt.x * wcol[4 * m4] + tt.y * wcol[4 * m4 + 1] + tt.z * wcol[4 * m4 + 2] + tt.w * wcol[4 * m4 + 3];
        }
        gt[(32 + r8 + r) * kLdF + c32] = -a;
      }
    }
    group_sync();
    // ---- T image: hi at +0, lo at +8192; thread (row, 32-column half); entries above the diagonal are 0
    {
      float tv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) tv[i] = 32 * th + i <= tr ? gt[tr * kLdF + 32 * th + i] : 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint4 hi, lo;
        pack8(tv + 8 * c8, hi, lo);
        *reinterpret_cast<uint4*>(img + sw_off(tr, 32 * th + 8 * c8)) = hi;
        *reinterpret_cast<uint4*>(img + 8192 + sw_off(tr, 32 * th + 8 * c8)) = lo;
      }
    }
    group_sync();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 64);
}

// ------------------------------------------------------------------------------------------------------
// chunk_state
// ------------------------------------------------------------------------------------------------------
struct StateSmem {
  uint8_t st_h[32768];   // S^T hi: 2 atoms of [128 v][64 d]
  uint8_t st_l[32768];   // S^T lo
  uint8_t kimg[kKImageBytes];  // this chunk's k-head operand image (bulk-copied)
  uint8_t tmat[3 * 8192];      // this chunk's T hi, T lo, A hi (bulk-copied)
  // The next chunk's v rows [64 t][128 v] fp32 (bulk-copied, one 512-byte row per token); from phase R on
  // R^T hi | lo [128 v][64 t], later (e^(G_C - G) Vn)^T hi | lo.
  uint8_t rv[32768];
  uint8_t vn_h[16384];     // Vn^T hi
  float zrows[kC * kD];    // this chunk's z rows [64 t][128 v] fp32 (bulk-copied)
  float gates[2][4 * kC];  // double-buffered beta | e^G | e^(G_C - G)
  float red[4][kC];
  float rstd[kC];
  uint64_t bar_kq, bar_t, bar_v, bar_z, bar_g[2], bar_mma[3];
  uint32_t tmem;
  int abort;
};

constexpr uint32_t kColP1 = 0, kColVn = 128, kColDs = 256, kColAv = 384;

// One halving step of a warp transpose-reduction: entries [0, N) and [N, 2N) are exchanged with lane ^ N;
// afterwards a[i] (i < N) holds the pair sum for index i + N * ((lane & N) != 0) of the previous level.
template <int N>
__device__ __forceinline__ void butterfly_step(float (&a)[32], int lane) {
  const bool up = (lane & N) != 0;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float send = up ? a[i] : a[i + N];
    const float keep = up ? a[i + N] : a[i];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, N);
  }
}

__device__ __forceinline__ void tmem_ld32(uint32_t addr, float* out) {
  uint32_t r[32];
  tmem_ld32_async(addr, r);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(r[i]);
}

// Write 32 consecutive k values (k0 .. k0+31, k0 a multiple of 32) of row r into a hi/lo tile pair.
__device__ __forceinline__ void write_row32(uint8_t* hi_tile, uint8_t* lo_tile, int r, int k0, const float* x) {
#pragma unroll
  for (int c8 = 0; c8 < 4; ++c8) {
    uint4 hi, lo;
    pack8(x + 8 * c8, hi, lo);
    *reinterpret_cast<uint4*>(hi_tile + sw_off(r, k0 + 8 * c8)) = hi;
    if (lo_tile) *reinterpret_cast<uint4*>(lo_tile + sw_off(r, k0 + 8 * c8)) = lo;
  }
}

// Shared-memory descriptor of an MN-major operand with 128-byte swizzle: 64 elements (128 B) contiguous
// along MN, consecutive K rows 128 B apart in 8-row groups 1024 B apart (SBO), 64-element MN blocks `lbo`
// bytes apart (LBO); base 1024-byte aligned.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// D (+)= A * B with A [128 x 64] K-major (one SW128 atom) and B = k^ rows [64 t][128 d] read MN-major
// (the [t][d] atoms of the K image, `lbo` bytes apart): 4 UMMAs of K = 16 tokens.
__device__ __forceinline__ void mma_a_kmajor_b_mn(uint32_t d, uint32_t a, uint32_t b, uint32_t lbo, uint32_t idesc,
                                                  bool accumulate) {
  const uint64_t da = sdesc_k_sw128(a);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    umma_f16(d, da + 2 * k, sdesc_mn_sw128(b + k * 2048, lbo), idesc, (accumulate || k) ? 1u : 0u);
}

__global__ void __launch_bounds__(kThreads, 1)
    chunk_state_kernel(const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_z,
                       const __grid_constant__ CUtensorMap tm_y, ChunkArgs p, const uint8_t* kimg, const uint8_t* timg,
                       int nchunks) {
  extern __shared__ uint8_t smem_raw[];
  StateSmem& sm = *reinterpret_cast<StateSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x / p.Hv, h = blockIdx.x % p.Hv;
  const int kh = h / (p.Hv / p.Hk);
  const int kd = p.Hk * kD;
  const int q4 = warp & 3, half = warp >> 2;
  const int v = q4 * 32 + lane;  // accumulator row (TMEM lane) this thread reads
  const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
  const uint8_t* kimg_h = kimg + (static_cast<int64_t>(b) * p.Hk + kh) * nchunks * kKImageBytes;
  const uint8_t* timg_h = timg + (static_cast<int64_t>(b) * p.Hv + h) * nchunks * kTImageBytes;
  uint8_t* rv_h = sm.rv;
  uint8_t* rv_l = sm.rv + 16384;
  const float* vrows = reinterpret_cast<const float*>(sm.rv);

  // Bulk copies of chunk c's data, each issued as soon as the buffer it overwrites is free.  Thread 0
  // counts the copies it armed per barrier, so that after an error it can wait out the ones still in flight
  // before the CTA exits.
  int n_kq = 0, n_t = 0, n_v = 0, n_z = 0, n_g[2] = {0, 0}, n_mma[3] = {0, 0, 0};
  auto load_k_t = [&](int c) {  // thread 0: K image (MMA1, MMA3) and T, A (MMA2, MMA3)
    ++n_kq;
    mbar_arrive_expect_tx(&sm.bar_kq, kKImageBytes);
    bulk_load(sm.kimg, kimg_h + static_cast<int64_t>(c) * kKImageBytes, kKImageBytes, &sm.bar_kq);
    ++n_t;
    mbar_arrive_expect_tx(&sm.bar_t, 3 * 8192);
    bulk_load(sm.tmat, timg_h + static_cast<int64_t>(c) * kTImageBytes, 3 * 8192, &sm.bar_t);
  };
  auto load_gates = [&](int c) {  // thread 0
    ++n_g[c & 1];
    mbar_arrive_expect_tx(&sm.bar_g[c & 1], 3 * kC * 4);
    bulk_load(sm.gates[c & 1], timg_h + static_cast<int64_t>(c) * kTImageBytes + kTGateOff, 3 * kC * 4,
              &sm.bar_g[c & 1]);
  };
  // Thread 0: this head's 128 columns of chunk c's 64 token rows (one TMA box; rows past the last token
  // read as zeros, rows of the next sequence are masked by the reader).
  auto load_rows = [&](int c, const CUtensorMap* map, int col, void* dst, uint64_t* bar, int& cnt) {
    ++cnt;
    mbar_arrive_expect_tx(bar, kC * kD * 4);
    tma_load_2d(dst, map, bar, col, b * p.T + c * kC, policy_evict_first());
  };
  const int v_col = 2 * kd + h * kD, z_col = static_cast<int>(p.z_off) + h * kD;

  if (tid == 0) {
    mbar_init(&sm.bar_kq, 1);
    mbar_init(&sm.bar_t, 1);
    mbar_init(&sm.bar_v, 1);
    mbar_init(&sm.bar_z, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&sm.bar_g[i], 1);
    for (int i = 0; i < 3; ++i) mbar_init(&sm.bar_mma[i], 1);
    fence_mbar_init();
    sm.abort = 0;
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_z);
    tma_prefetch_desc(&tm_y);
    load_k_t(0);
    load_rows(0, &tm_v, v_col, sm.rv, &sm.bar_v, n_v);
    load_rows(0, &tm_z, z_col, sm.zrows, &sm.bar_z, n_z);
    load_gates(0);
    if (nchunks > 1) load_gates(1);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem, 512);
    tmem_relinquish();
  }
  // ---- initial state: thread (v, half) holds S^T[v][64 half .. +63] = S[d][v]
  float* Sg = p.state + (static_cast<int64_t>(b) * p.Hv + h) * kD * kD;
  float S[64];
#pragma unroll
  for (int j = 0; j < 64; ++j) S[j] = Sg[(64 * half + j) * kD + v];
#pragma unroll
  for (int c32 = 0; c32 < 2; ++c32)
    write_row32(sm.st_h + half * 16384, sm.st_l + half * 16384, v, 32 * c32, S + 32 * c32);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  const float w_norm = p.norm_w[v];

  // MMA1 of chunk c: [(K^S)^T | (Q^S)^T] = S^T [K^; Q^]^T (thread 0)
  auto issue_mma1 = [&](int c) {
    if (!mbar_wait(&sm.bar_kq, c & 1, kErrWaitTmaFull)) sm.abort = 1;
    tc_fence_after();
    const uint32_t sth = smem_u32(sm.st_h), stl = smem_u32(sm.st_l), kq = smem_u32(sm.kimg + kKOffKQ);
    const uint32_t kl = smem_u32(sm.kimg + kKOffKL);
    mma_atoms(tmem + kColP1, sth, 16384, kq, 16384, 2, idesc_dense(1, 128, 128), false);
    mma_atoms(tmem + kColP1, stl, 16384, kq, 16384, 2, idesc_dense(1, 128, 128), true);
    mma_atoms(tmem + kColP1, sth, 16384, kl, 8192, 2, idesc_dense(1, 128, 64), true);
    umma_commit(&sm.bar_mma[0]);
    ++n_mma[0];
  };

  // MMA1 of chunk c + 1 is issued as soon as chunk c's state update is in shared memory, so that it runs
  // (and its K image finishes arriving) while chunk c's output, RMSNorm and y store are computed.
  if (tid == 0) issue_mma1(0);
  for (int ch = 0; ch < nchunks; ++ch) {
    const int t0 = ch * kC, L = min(kC, p.T - t0);
    const int64_t row0 = static_cast<int64_t>(b) * p.T + t0;
    const uint32_t par = ch & 1;
    const float* gt = sm.gates[ch & 1];
    const float* g_beta = gt;
    const float* g_eG = gt + kC;
    const float* g_eCG = gt + 2 * kC;
    if (tid == 0 && ch + 1 < nchunks) {
      // The next chunk's K image, T / A image, v rows and z rows can only be copied into shared memory once
      // this chunk has finished with their buffers; bring them into L2 now so that those copies are short.
      prefetch_l2(kimg_h + static_cast<int64_t>(ch + 1) * kKImageBytes, kKImageBytes);
      prefetch_l2(timg_h + static_cast<int64_t>(ch + 1) * kTImageBytes, 3 * 8192);
      prefetch_l2_2d(&tm_v, v_col, b * p.T + (ch + 1) * kC);
      prefetch_l2_2d(&tm_z, z_col, b * p.T + (ch + 1) * kC);
    }
    __syncwarp();
    // V of phase R from the prefetched rows (then the buffer becomes R^T)
    if (!mbar_wait(&sm.bar_v, par, kErrWaitTmaFull)) sm.abort = 1;
    float vt[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int t = 32 * half + j;
      vt[j] = t < L ? vrows[t * kD + v] : 0.f;
    }
    if (!mbar_wait(&sm.bar_g[ch & 1], (ch >> 1) & 1, kErrWaitTmaFull)) sm.abort = 1;
    if (!mbar_wait(&sm.bar_mma[0], par, kErrWaitAccum)) sm.abort = 1;
    tc_fence_after();
    __syncthreads();  // every thread has its V: the rows may be overwritten by R^T
    // ---------------- phase R: R^T[v][t] = beta_t (V[t][v] - e^G_t (K^S)^T[v][t]) ----------------
    {
      float ks[32];
      tmem_ld32(tmem + lane_base + kColP1 + 32 * half, ks);
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 bt = reinterpret_cast<const float4*>(g_beta + 32 * half)[j4];
        const float4 eg = reinterpret_cast<const float4*>(g_eG + 32 * half)[j4];
        ks[4 * j4] = bt.x * (vt[4 * j4] - eg.x * ks[4 * j4]);
        ks[4 * j4 + 1] = bt.y * (vt[4 * j4 + 1] - eg.y * ks[4 * j4 + 1]);
        ks[4 * j4 + 2] = bt.z * (vt[4 * j4 + 2] - eg.z * ks[4 * j4 + 2]);
        ks[4 * j4 + 3] = bt.w * (vt[4 * j4 + 3] - eg.w * ks[4 * j4 + 3]);
      }
      write_row32(rv_h, rv_l, v, 32 * half, ks);
    }
    if (tid == 0) bulk_wait_read();  // the previous chunk's y tile has left vn_h (rewritten in phase V)
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (sm.abort) break;
    // ---------------- MMA2: Vn^T = R^T T^T ----------------
    if (tid == 0) {
      if (!mbar_wait(&sm.bar_t, par, kErrWaitTmaFull)) sm.abort = 1;
      tc_fence_after();
      const uint32_t rh = smem_u32(rv_h), rl = smem_u32(rv_l), th = smem_u32(sm.tmat), tl = smem_u32(sm.tmat + 8192);
      constexpr uint32_t id = idesc_dense(1, 128, 64);
      mma_atoms(tmem + kColVn, rh, 0, th, 0, 1, id, false);
      mma_atoms(tmem + kColVn, rl, 0, th, 0, 1, id, true);
      mma_atoms(tmem + kColVn, rh, 0, tl, 0, 1, id, true);
      umma_commit(&sm.bar_mma[1]);
      ++n_mma[1];
    }
    __syncwarp();
    if (!mbar_wait(&sm.bar_mma[1], par, kErrWaitAccum)) sm.abort = 1;
    tc_fence_after();
    // ---------------- phase V: Vn^T hi (for A Vn) and (e^(G_C - G) Vn)^T hi/lo (for the state) ----------------
    {
      float vn[32];
      tmem_ld32(tmem + lane_base + kColVn + 32 * half, vn);
      write_row32(sm.vn_h, nullptr, v, 32 * half, vn);
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 e = reinterpret_cast<const float4*>(g_eCG + 32 * half)[j4];
        vn[4 * j4] *= e.x;
        vn[4 * j4 + 1] *= e.y;
        vn[4 * j4 + 2] *= e.z;
        vn[4 * j4 + 3] *= e.w;
      }
      write_row32(rv_h, rv_l, v, 32 * half, vn);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (sm.abort) break;
    // ---------------- MMA3: dS^T = (e^(G_C-G) Vn)^T K^ ; (A Vn)^T = Vn^T A^T ----------------
    if (tid == 0) {
      const uint32_t rh = smem_u32(rv_h), rl = smem_u32(rv_l);
      const uint32_t kq = smem_u32(sm.kimg + kKOffKQ), kl = smem_u32(sm.kimg + kKOffKL);
      constexpr uint32_t id_mn = idesc_dense(1, 128, 128) | (1u << 16);  // B MN-major
      constexpr uint32_t id64 = idesc_dense(1, 128, 64);
      mma_a_kmajor_b_mn(tmem + kColDs, rh, kq, 16384, id_mn, false);
      mma_a_kmajor_b_mn(tmem + kColDs, rl, kq, 16384, id_mn, true);
      mma_a_kmajor_b_mn(tmem + kColDs, rh, kl, 8192, id_mn, true);
      mma_atoms(tmem + kColAv, smem_u32(sm.vn_h), 0, smem_u32(sm.tmat + 16384), 0, 1, id64, false);
      umma_commit(&sm.bar_mma[2]);
      ++n_mma[2];
    }
    __syncwarp();
    if (!mbar_wait(&sm.bar_z, par, kErrWaitTmaFull)) sm.abort = 1;
    float zt[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) zt[j] = sm.zrows[(32 * half + j) * kD + v];
    if (!mbar_wait(&sm.bar_mma[2], par, kErrWaitAccum)) sm.abort = 1;
    tc_fence_after();
    // K image, T, A and the R buffer have been consumed: the next chunk's copies start now
    if (ch + 1 < nchunks) {  // (also after an error: the exit waits for every armed copy)
      if (tid == 0) {
        load_k_t(ch + 1);
        load_rows(ch + 1, &tm_v, v_col, sm.rv, &sm.bar_v, n_v);
      }
    }
    // ---------------- output: O^T[v][t] = e^G_t (Q^S)^T + (A Vn)^T -> RMSNorm over v -> y ----------------
    float o[32];
    {
      float av[32];
      {  // both loads in flight, one wait
        uint32_t ro[32], ra[32];
        tmem_ld32_async(tmem + lane_base + kColP1 + 64 + 32 * half, ro);
        tmem_ld32_async(tmem + lane_base + kColAv + 32 * half, ra);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          o[j] = __uint_as_float(ro[j]);
          av[j] = __uint_as_float(ra[j]);
        }
      }
      float a[32];
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 eg = reinterpret_cast<const float4*>(g_eG + 32 * half)[j4];
        o[4 * j4] = eg.x * o[4 * j4] + av[4 * j4];
        o[4 * j4 + 1] = eg.y * o[4 * j4 + 1] + av[4 * j4 + 1];
        o[4 * j4 + 2] = eg.z * o[4 * j4 + 2] + av[4 * j4 + 2];
        o[4 * j4 + 3] = eg.w * o[4 * j4 + 3] + av[4 * j4 + 3];
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) a[j] = o[j] * o[j];
      // Butterfly: after the 5 steps lane l holds the warp's sum for t index 32 half + l.
      butterfly_step<16>(a, lane);
      butterfly_step<8>(a, lane);
      butterfly_step<4>(a, lane);
      butterfly_step<2>(a, lane);
      butterfly_step<1>(a, lane);
      sm.red[q4][32 * half + lane] = a[0];
    }
    // ---------------- state: S^T <- e^(G_C) S^T + dS^T ----------------
    {
      const float eC = g_eG[kC - 1];
#pragma unroll
      for (int c32 = 0; c32 < 2; ++c32) {
        float ds[32];
        tmem_ld32(tmem + lane_base + kColDs + 64 * half + 32 * c32, ds);
#pragma unroll
        for (int j = 0; j < 32; ++j) S[32 * c32 + j] = eC * S[32 * c32 + j] + ds[j];
      }
#pragma unroll
      for (int c32 = 0; c32 < 2; ++c32)
        write_row32(sm.st_h + half * 16384, sm.st_l + half * 16384, v, 32 * c32, S + 32 * c32);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();  // red[] complete; every thread has its z; S^T is written
    tc_fence_after();
    if (tid < kC)
      sm.rstd[tid] = rsqrtf((sm.red[0][tid] + sm.red[1][tid] + sm.red[2][tid] + sm.red[3][tid]) * (1.0f / kD) + p.eps);
    if (tid == 0 && ch + 1 < nchunks) load_rows(ch + 1, &tm_z, z_col, sm.zrows, &sm.bar_z, n_z);
    __syncthreads();
    // The next chunk's MMA1 reads only S^T (written before the barrier above) and its K image, and
    // overwrites (K^S)^T | (Q^S)^T, which this chunk's output took from TMEM before that barrier: it runs
    // (and its K image finishes arriving) while this chunk's y is computed and stored.
    if (tid == 0 && ch + 1 < nchunks && !sm.abort) issue_mma1(ch + 1);
    // y = O rstd w SiLU(z): a full chunk is staged as a [64 t][128 v] bf16 tile in vn_h (free since MMA3) and
    // leaves by one TMA store; a partial last chunk is stored directly (the box would spill into the next
    // sequence's rows).
    {
      __nv_bfloat16* ys = reinterpret_cast<__nv_bfloat16*>(sm.vn_h) + v;
      __nv_bfloat16* yb = static_cast<__nv_bfloat16*>(p.y) + static_cast<int64_t>(h) * kD + v;
      const int64_t y_ld = static_cast<int64_t>(p.Hv) * kD;
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 rs = reinterpret_cast<const float4*>(sm.rstd + 32 * half)[j4];
        const float r4[4] = {rs.x, rs.y, rs.z, rs.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = 4 * j4 + u, t = 32 * half + j;
          const __nv_bfloat16 yv = __float2bfloat16_rn(o[j] * r4[u] * w_norm * silu_fast(zt[j]));
          if (L == kC) ys[t * kD] = yv;
          else if (t < L) yb[(row0 + t) * y_ld] = yv;
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      if (L == kC) {
        tma_store_2d(&tm_y, sm.vn_h, h * kD, static_cast<int>(row0));
        bulk_commit();
      }
      if (ch + 2 < nchunks) load_gates(ch + 2);  // this chunk's gate buffer is free again
    }
    if (sm.abort) break;
  }
#pragma unroll
  for (int j = 0; j < 64; ++j) Sg[(64 * half + j) * kD + v] = S[j];
  // After an error the loop may end with bulk copies still in flight into this CTA's shared memory, and MMAs
  // still writing TMEM: wait (bounded) for the last phase of every barrier with an issued copy or commit
  // before the CTA exits.  Phase k of a
  // barrier has parity k & 1; waiting on an already completed phase returns at once.
  if (tid == 0) bulk_wait_all();  // the last y tiles have left shared memory
  if (tid == 0 && sm.abort) {
    if (n_kq) mbar_wait(&sm.bar_kq, (n_kq - 1) & 1, kErrWaitTmaFull);
    if (n_t) mbar_wait(&sm.bar_t, (n_t - 1) & 1, kErrWaitTmaFull);
    if (n_v) mbar_wait(&sm.bar_v, (n_v - 1) & 1, kErrWaitTmaFull);
    if (n_z) mbar_wait(&sm.bar_z, (n_z - 1) & 1, kErrWaitTmaFull);
    for (int i = 0; i < 2; ++i)
      if (n_g[i]) mbar_wait(&sm.bar_g[i], (n_g[i] - 1) & 1, kErrWaitTmaFull);
    // and for the last MMA group committed on each barrier, before TMEM is freed
    for (int i = 0; i < 3; ++i)
      if (n_mma[i]) mbar_wait(&sm.bar_mma[i], (n_mma[i] - 1) & 1, kErrWaitAccum);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace

size_t chunk_prefill_scratch_bytes(int B, int T, int Hk, int Hv) {
  const int64_t nchunks = (T + kC - 1) / kC;
  return static_cast<size_t>(B) * nchunks * (static_cast<size_t>(Hk) * kKImageBytes + static_cast<size_t>(Hv) * kTImageBytes);
}

static cudaError_t check_chunk_args(const ChunkArgs& a, const void* scratch) {
  if (a.B <= 0 || a.T <= 0 || a.Hk <= 0 || a.Hv <= 0 || a.Hv % a.Hk) return cudaErrorInvalidValue;
  if ((a.qkv_ld & 3) || (a.proj_ld & 3) || (a.z_off & 3) || (reinterpret_cast<uintptr_t>(scratch) & 15) ||
      (reinterpret_cast<uintptr_t>(a.qkv) & 15) || (reinterpret_cast<uintptr_t>(a.proj) & 15))
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

// Scratch layout: all k-head images, then all v-head images.
static void split_scratch(const ChunkArgs& a, const void* scratch, uint8_t** kimg, uint8_t** timg) {
  const int64_t nchunks = (a.T + kC - 1) / kC;
  *kimg = static_cast<uint8_t*>(const_cast<void*>(scratch));
  *timg = *kimg + static_cast<int64_t>(a.B) * a.Hk * nchunks * kKImageBytes;
}

cudaError_t chunk_prep(const ChunkArgs& a, void* scratch, cudaStream_t stream) {
  cudaError_t e = check_chunk_args(a, scratch);
  if (e != cudaSuccess) return e;
  const int nchunks = (a.T + kC - 1) / kC;
  const int smem = static_cast<int>(sizeof(PrepSmem)) + 1024;
  e = cudaFuncSetAttribute(chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  uint8_t *kimg, *timg;
  split_scratch(a, scratch, &kimg, &timg);
  count_launch();
  chunk_prep_kernel<<<a.B * a.Hk * nchunks, kThreads, smem, stream>>>(a, kimg, timg, nchunks);
  return cudaGetLastError();
}

cudaError_t chunk_state(const ChunkArgs& a, const void* scratch, cudaStream_t stream) {
  cudaError_t e = check_chunk_args(a, scratch);
  if (e != cudaSuccess) return e;
  const int nchunks = (a.T + kC - 1) / kC;
  const int smem = static_cast<int>(sizeof(StateSmem)) + 1024;
  e = cudaFuncSetAttribute(chunk_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  uint8_t *kimg, *timg;
  split_scratch(a, scratch, &kimg, &timg);
  CUtensorMap tm_v, tm_z, tm_y;
  const int64_t n = static_cast<int64_t>(a.B) * a.T;
  const int kd = a.Hk * kD;
  e = make_tmap_plain(&tm_v, a.qkv, 4, n, 2 * kd + static_cast<int64_t>(a.Hv) * kD, a.qkv_ld, kD, kC);
  if (e != cudaSuccess) return e;
  e = make_tmap_plain(&tm_z, a.proj, 4, n, a.z_off + static_cast<int64_t>(a.Hv) * kD, a.proj_ld, kD, kC);
  if (e != cudaSuccess) return e;
  e = make_tmap_plain(&tm_y, a.y, 2, n, static_cast<int64_t>(a.Hv) * kD, static_cast<int64_t>(a.Hv) * kD, kD, kC);
  if (e != cudaSuccess) return e;
  count_launch();
  chunk_state_kernel<<<a.B * a.Hv, kThreads, smem, stream>>>(tm_v, tm_z, tm_y, a, kimg, timg, nchunks);
  return cudaGetLastError();
}

}  // namespace gdn
