// Internal interface of the tcgen05 GEMM (C = A * B^T, bf16 operands, fp32 accumulation in TMEM).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

// What the epilogue does with the fp32 accumulator tile.
enum GemmEpi : int {
  kEpiStoreF32 = 0,      // out[m * ld + n] = acc
  kEpiStoreBF16 = 1,     // out[m * ld + n] = bf16(acc)
  kEpiStoreF32T = 2,     // out[n * ld + m] = acc          (A = weights, B = activations)
  kEpiStoreBF16T = 3,    // out[n * ld + m] = bf16(acc)
  kEpiPrefillInProj = 5, // row-major fp32 store of the prefill in_proj (rows = tokens of seq_len-token
                         // sequences); columns [0, conv_rows) get the causal conv (K = 4) + SiLU, the
                         // raw last 3 inputs of each sequence go to conv_tail (persistent kernel only)
  kEpiSwiGLUT = 6,       // decode MLP gate/up (A = weights with gate and up rows interleaved: row 2j gate_j,
                         // row 2j + 1 up_j): out[n * ld + j] = bf16(SiLU(acc[2j][n]) * acc[2j + 1][n])
  kEpiSwiGLU = 7,        // prefill MLP gate/up (B = the interleaved weights): out[m * ld + j] =
                         // bf16(SiLU(acc[m][2j]) * acc[m][2j + 1]) (persistent kernel only)
};

struct GemmEpiArgs {
  void* out = nullptr;
  int64_t ld = 0;  // leading dimension of `out`, in elements
  // kEpiPrefillInProj
  int conv_rows = 0;
  // kEpiPrefillInProj only
  const float* conv_w = nullptr;  // [conv_rows, 4]
  const float* conv_state = nullptr;  // [M / seq_len, 3, conv_rows], read (the roll runs after the GEMM)
  int seq_len = 0;
  float* conv_tail = nullptr;     // [M / seq_len, 3, conv_rows]: raw inputs at times seq_len - 3 .. - 1
  // Operands stored pre-tiled by tile_weights_bf16 (then A / B must equal these pointers; lda / ldb unused).
  const void* a_tiled = nullptr;
  const void* b_tiled = nullptr;
  // gemm_bf16_tn and gemm_f8_tn: when set, the output goes to out + ((*slot_epoch + 1) % 2) * slot_bytes (the
  // double-buffered slot of the NVLink all-reduce; the epoch is read after the previous kernel finished).
  const unsigned long long* slot_epoch = nullptr;
  int64_t slot_bytes = 0;
  // gemm_f8_tn only: acc[m][n] is multiplied by row_scale[m] * col_scale[n] (the operands' e4m3 scales)
  const float* row_scale = nullptr;
  const float* col_scale = nullptr;
  // with row_scale and no col_scale (weight-only fp8): acc * acc_scale * row_scale[m]
  float acc_scale = 1.0f;
  // kEpiStoreBF16T (gemm_bf16_tn) and kEpiStoreBF16 (gemm_bf16_persistent): when set, the stored value is
  // bf16(acc + residual) with residual bf16 in the output's layout, row stride res_ld (may alias `out`:
  // every element is read and then written by the same thread).
  const void* residual = nullptr;
  int64_t res_ld = 0;
};

// A: [M, K] bf16 row-major with row stride lda (elements); B: [N, K] bf16 row-major with row stride ldb
// (or pre-tiled, see GemmEpiArgs).  ksplit > 1 splits K over a cluster of ksplit CTAs whose partial tiles
// are summed through distributed shared memory (no global workspace).  ksplit = 0 picks a value.
// pdl: launch with programmatic stream serialization (the kernel may start while the previous kernel in
// the stream is still running; it prefetches the weight operand -- A for the transposed epilogues, B
// otherwise -- and waits for the previous kernel before touching anything else).
// trigger: let the next programmatically serialized kernel start as soon as every CTA of this one runs.
// Only a kernel whose successor reads nothing that an earlier, still running kernel may write can set it;
// the last kernel of a layer call never does, so consecutive calls stay ordered.
cudaError_t gemm_bf16_tn(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, int epi,
                         const GemmEpiArgs& args, int ksplit, cudaStream_t stream, bool pdl = false,
                         bool trigger = false);

// Persistent variant for the large prefill projections: one CTA per SM, 128 x 256 tiles, two TMEM
// accumulators so a tile's epilogue overlaps the next tile's MMAs.  A [M, K] bf16 row-major (row stride
// lda); B_tiled = weights [N, K] pre-tiled by tile_weights_bf16.  epi: kEpiStoreF32, kEpiStoreBF16,
// kEpiPrefillInProj or kEpiSwiGLU (N even; out is [M, N / 2]).
cudaError_t gemm_bf16_persistent(const void* A, int64_t lda, const void* B_tiled, int M, int N, int K, int epi,
                                 const GemmEpiArgs& args, cudaStream_t stream, bool pdl = false);

// Plain (unswizzled) 2D tensor map over a matrix [rows, cols] of elem_bytes-byte elements (4: fp32, 2: bf16)
// with row stride ld elements and boxes of box_cols x box_rows (box_cols * elem_bytes a multiple of 16).
// `map` points at a CUtensorMap.
cudaError_t make_tmap_plain(void* map, const void* ptr, int elem_bytes, int64_t rows, int64_t cols, int64_t ld,
                            int box_cols, int box_rows);

// Weights kept in the GEMM's streaming layout: [ceil(rows/128), rounded up to even][cols/64] blocks of
// 16 KB, each block the 128B-swizzled shared-memory image of a 128 x 64 bf16 tile, so that a K-slice of
// an M-tile is one contiguous run of HBM.
size_t tiled_weight_bytes(int rows, int cols);
cudaError_t tile_weights_bf16(const void* src, int64_t ld, int rows, int cols, void* dst, cudaStream_t stream);

// fp8 (e4m3) decode projections.  Every scale is a power of two (the smallest 2^e with max|row| / 2^e <=
// 448), so e4m3 value * scale is exact in bf16 and fp32.
//   quantize_tiled_weights_fp8: row-wise quantisation of a matrix pre-tiled by tile_weights_bf16 (rows x
//     cols, cols % 128 == 0): w8 (tiled_weight_bytes(rows, cols) / 2 bytes) receives the e4m3 weights in the
//     same streaming layout with 128-element K blocks, scale[rows] the scales, and the bf16 tiles are
//     overwritten with the dequantised weights, so bf16 GEMMs over them use the same weights.
//   quantize_rows_fp8: row-wise quantisation of bf16 activations x [rows, cols] (row stride ld) into
//     xq [rows, cols] bytes and xs[rows]; launched with programmatic dependent launch.
//   gemm_f8_tn: gemm_bf16_tn's weight-streaming path with A = w8 (pre-tiled e4m3, ep.a_tiled == A) and
//     B = xq [N, K] (row stride ldb bytes), ep.row_scale / ep.col_scale set; epi kEpiStoreBF16T or
//     kEpiStoreF32T.
//   row_amax (optional): use these row maxima instead of the tiled rows' own (the rows of a column shard
//     then get the scales of the whole rows, so every shard quantises as the unsharded matrix does).
cudaError_t quantize_tiled_weights_fp8(void* w_tiled, int rows, int cols, void* w8, float* scale,
                                       cudaStream_t stream, const float* row_amax = nullptr);
// out[r] = max |src[r][:]| of a row-major bf16 matrix (row stride ld elements, cols % 8 == 0).
cudaError_t row_amax_bf16(const void* src, int64_t ld, int rows, int cols, float* out, cudaStream_t stream);
cudaError_t quantize_rows_fp8(const void* x, int64_t ld, int rows, int cols, void* xq, float* xs,
                              cudaStream_t stream);
cudaError_t gemm_f8_tn(const void* A_tiled, const void* B, int64_t ldb, int M, int N, int K, int epi,
                       const GemmEpiArgs& args, cudaStream_t stream, bool pdl = false, bool trigger = false);
// Weight-only fp8: A8_tiled = e4m3 weights in the fp8 streaming layout (quantize_tiled_weights_fp8), B = bf16
// activations [N, K] (row stride ldb elements), K % 128 == 0, ep.row_scale = the weights' row scales and
// ep.col_scale null; the e4m3 stages are widened to bf16 in shared memory and multiplied on the bf16 tensor
// cores.  epi kEpiStoreBF16T (optionally with ep.residual) or kEpiStoreF32T.
cudaError_t gemm_w8_tn(const void* A8_tiled, const void* B, int64_t ldb, int M, int N, int K, int epi,
                       const GemmEpiArgs& args, cudaStream_t stream, bool pdl = false, bool trigger = false);

// Number of kernel launches issued by this library since load (for the benchmark's launch count).
uint64_t launch_count();
void count_launch();

}  // namespace gdn
