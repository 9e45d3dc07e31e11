// Internal interface of the non-GEMM kernels (recurrence, conv, chunked prefill).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr int kHeadDim = 128;  // dk = dv = 128 (the Qwen3.5 GDN head size; the only one supported)

// Strided views of the per-token inputs of the recurrence.  Element (row, head, i) of a vector input lives
// at ptr[row * tok + head * head_stride + i]; row = b * T + t (sequence-major).
struct RecurrenceArgs {
  const float* q = nullptr;
  int64_t q_tok = 0, q_head = 0;  // indexed by k-head
  const float* k = nullptr;
  int64_t k_tok = 0, k_head = 0;  // indexed by k-head
  const float* v = nullptr;
  int64_t v_tok = 0, v_head = 0;
  const float* g = nullptr;  // log decay
  int64_t g_tok = 0, g_head = 0;
  const float* beta = nullptr;
  int64_t b_tok = 0, b_head = 0;
  // Layer decode only: when a_log is set, g and beta above point at the raw a and b projections, and
  // g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) are formed in the kernel.
  const float* a_log = nullptr;    // [Hv]
  const float* dt_bias = nullptr;  // [Hv]
  // Gated RMSNorm epilogue (when z != nullptr): y = RMSNorm(o) * norm_w * SiLU(z) -> bf16
  const float* z = nullptr;
  int64_t z_tok = 0, z_head = 0;
  const float* norm_w = nullptr;  // [128]
  float eps = 1e-6f;
  void* y = nullptr;  // bf16
  int64_t y_tok = 0, y_head = 0;
  // Raw output (when z == nullptr): o fp32
  float* o = nullptr;
  int64_t o_tok = 0, o_head = 0;
  float* state = nullptr;  // [B, Hv, 128, 128] fp32, in place
  int B = 0, T = 0, Hk = 0, Hv = 0;
  float scale = 0.0f;  // q scale (dk^-0.5 by default)
  int l2norm = 1;
  // Layer decode only (decode_step_forward): q, k, v above are the raw in_proj outputs of the conv
  // channels; channel index (into conv_w / conv_state) of q element (kh, i) is kh * 128 + i, of k element
  // k_conv + kh * 128 + i, of v element v_conv + h * 128 + i.
  const float* conv_w = nullptr;  // [conv_dim, 4]
  float* conv_state = nullptr;    // [B, 3, conv_dim], rolled in place
  int conv_dim = 0;
  int k_conv = 0, v_conv = 0;
};

// Token-by-token gated delta rule, one CTA per (sequence, v-head), state kept in registers.
// pdl: may start while the previous kernel (the in_proj GEMM) runs; it loads the state first.
cudaError_t recurrence_forward(const RecurrenceArgs& a, cudaStream_t stream, bool pdl = false);

// Layer decode step (T = 1): causal conv + SiLU of q, k, v with the conv-state roll, then the gated delta
// rule and the gated RMSNorm.  One CTA per (sequence, v-head); the v-heads of a GQA group (at most 8) form
// a thread-block cluster so that exactly one of them rolls the shared q/k conv state after all have read
// it.  Launched with programmatic dependent launch after the in_proj GEMM.
cudaError_t decode_step_forward(const RecurrenceArgs& a, cudaStream_t stream);

// Conv-state roll after the prefill in_proj (whose epilogue ran the conv): conv_state [B, 3, C] row j
// becomes the input at time T - 3 + j, read from tail [B, 3, C] (the raw inputs at T - 3 .. T - 1) or,
// for times before 0, from the old state.
cudaError_t conv_state_roll_tail(const float* tail, float* conv_state, int B, int T, int C, cudaStream_t stream);

// Chunked prefill of the whole recurrence + gated RMSNorm over the layer's in_proj output.
struct ChunkArgs {
  const float* qkv = nullptr;  // post-conv q | k | v, [B*T, qkv_ld]
  int64_t qkv_ld = 0;
  const float* proj = nullptr;  // in_proj output rows [B*T, proj_ld]: z at z_off, a at a_off, b at b_off
  int64_t proj_ld = 0;
  int64_t z_off = 0, a_off = 0, b_off = 0;  // column offsets of z, a and b inside a proj row
  const float* a_log = nullptr;
  const float* dt_bias = nullptr;
  const float* norm_w = nullptr;
  float eps = 1e-6f;
  float* state = nullptr;  // [B, Hv, 128, 128]
  void* y = nullptr;       // bf16 [B*T, Hv*128]
  int B = 0, T = 0, Hk = 0, Hv = 0;
};
// Scratch (bytes) the chunked prefill needs for B sequences of T tokens: per (sequence, k-head, chunk) the
// bf16 operand tiles of k^ and q^ (80 KB), per (sequence, v-head, chunk) the tiles of T and A and the gates
// (25 KB).
size_t chunk_prefill_scratch_bytes(int B, int T, int Hk, int Hv);
// chunk_prep writes the tile images into scratch; chunk_state (stream-ordered after it) consumes them.
cudaError_t chunk_prep(const ChunkArgs& a, void* scratch, cudaStream_t stream);
cudaError_t chunk_state(const ChunkArgs& a, const void* scratch, cudaStream_t stream);

// Decoder-layer RMSNorm (Qwen3_5RMSNorm: fp32 normalisation, times (1 + w), bf16 out) of `rows` rows of h
// bf16; with `add`, the rows are first summed with it (bf16 residual add) and, with `sum_out`, that sum is
// stored too.  Pointers 16-byte aligned, h a multiple of 8 and at most 8192.  Programmatic dependent launch.
cudaError_t rmsnorm_rows(const void* x, const void* add, void* sum_out, const float* w, float eps, void* out, int rows,
                         int h, cudaStream_t stream);

// NVLink all-reduce (sum) of bf16 [n] partials: src[p] is rank p's first slot (own included, mapped into this
// process; the second follows slot_bytes later), flags[p] rank p's flag page: arrive[kP2PMaxRanks] u64
// counters at [0], reduced[kP2PMaxRanks][kP2PMaxCtas] at [kP2PReducedOff].  epoch and cta_done[2] are this
// rank's device-side control words; call e = epoch + 1 uses slot e % 2.
constexpr int kP2PMaxRanks = 8;
constexpr int kP2PMaxCtas = 256;    // all-reduce grid cap
constexpr int kP2PReducedOff = 64;  // u64 index of reduced[rank][cta] in a flag page
constexpr int kP2PFlagPageBytes = (kP2PReducedOff + kP2PMaxRanks * kP2PMaxCtas) * 8;
struct P2PAllReduceArgs {
  const void* src[kP2PMaxRanks] = {};
  unsigned long long* flags[kP2PMaxRanks] = {};
  unsigned long long* epoch = nullptr;
  unsigned int* cta_done = nullptr;
  void* out = nullptr;
  int64_t n = 0;  // bf16 elements, a multiple of 8
  int64_t slot_bytes = 0;
  int rank = 0, world = 1;
};
cudaError_t allreduce_p2p(const P2PAllReduceArgs& a, cudaStream_t stream);
// One thread waits (bounded, as the all-reduce waits for a peer) until *flag >= value.
cudaError_t peer_wait_selftest(const unsigned long long* flag, unsigned long long value, cudaStream_t stream);

}  // namespace gdn
