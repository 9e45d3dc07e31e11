/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) Qwen3.5 Gated DeltaNet layer.
 *
 * The ABI keeps the per-layer op API of the reference (chz05/linear_attention_op): weights in; hidden
 * states plus the recurrent and conv state in and out.  It is plain C: opaque handles, plain pointers and
 * sizes, status codes, no exceptions across the boundary, no torch types.  All tensor pointers passed to
 * the compute entry points are CUDA device pointers; `stream` is a cudaStream_t (NULL = legacy stream);
 * work is stream-ordered and asynchronous.  Handles are thread-compatible: use one handle per stream.
 *
 * Layouts (row-major, "rows" are sequence-major tokens b*T + t, as in the reference
 * wormhole_n150/qwen3.5_9B/kernels/layer_reader.cpp:108-110):
 *   x, out      bf16 [B, T, hidden]
 *   rec_state   fp32 [B, Hv_local, 128, 128], S[k_index][v_index]      (9B/reference.py:26-34)
 *   conv_state  fp32 [B, 3, conv_dim_local], row j = pre-conv input at time T-3+j
 *               (the reference's 3-row history, 9B/kernels/layer_reader.cpp:184-197)
 *   conv_dim_local = 2 * Hk_local * 128 + Hv_local * 128, channel order [q | k | v] of this rank's heads.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_ABI_VERSION 1

#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

typedef enum gdn_status {
  GDN_OK = 0,
  GDN_ERR_INVALID_ARGUMENT = 1, /* bad size, shape or alignment */
  GDN_ERR_NULL_POINTER = 2,
  GDN_ERR_UNSUPPORTED = 3,      /* geometry this build does not implement (e.g. head dim != 128) */
  GDN_ERR_CUDA = 4,             /* a CUDA runtime call failed */
  GDN_ERR_NCCL = 5,             /* NCCL missing or a NCCL call failed */
  GDN_ERR_TIMEOUT = 6,          /* a kernel's bounded wait expired (see gdn_device_error) */
  GDN_ERR_OUT_OF_MEMORY = 7
} gdn_status;

/* Layer geometry (global, before head sharding).  Mirrors the HF Qwen3_5TextConfig fields the
 * reference reads (0.8B/test_gdn_l1.py:11-14) and the asserts of 9B/gdn_layer.py:61-64. */
typedef struct gdn_dims {
  int32_t hidden;      /* hidden size; multiple of 64 */
  int32_t num_k_heads; /* Hk */
  int32_t num_v_heads; /* Hv, a multiple of Hk (GQA: v-head h reads k-head h / (Hv/Hk)) */
  int32_t head_k_dim;  /* must be 128 */
  int32_t head_v_dim;  /* must be 128 */
  int32_t conv_kernel; /* must be 4 */
  float eps;           /* RMSNorm epsilon (1e-6) */
  int32_t chunk;       /* prefill chunk; 0 or 64 */
} gdn_dims;

/* One layer's weights in Hugging Face Qwen3_5GatedDeltaNet layout (global, unsharded).  Pointers may be
 * host or device memory; gdn_layer_create copies this rank's head shard into layer-owned device buffers
 * (the reference copies and re-lays out the HF weights in its constructor, 9B/gdn_layer.py:90-127). */
typedef struct gdn_weights {
  const uint16_t* w_qkv;  /* bf16 [2*Hk*128 + Hv*128, hidden]  in_proj_qkv.weight */
  const uint16_t* w_z;    /* bf16 [Hv*128, hidden]             in_proj_z.weight   */
  const uint16_t* w_a;    /* bf16 [Hv, hidden]                 in_proj_a.weight   */
  const uint16_t* w_b;    /* bf16 [Hv, hidden]                 in_proj_b.weight   */
  const float* conv_w;    /* fp32 [2*Hk*128 + Hv*128, 4]       conv1d.weight[:, 0, :] */
  const float* a_log;     /* fp32 [Hv]                         A_log              */
  const float* dt_bias;   /* fp32 [Hv]                         dt_bias            */
  const float* norm_w;    /* fp32 [128]                        norm.weight        */
  const uint16_t* w_out;  /* bf16 [hidden, Hv*128]             out_proj.weight    */
} gdn_weights;

/* Sizes of this rank's shard, for allocating the state buffers. */
typedef struct gdn_layer_info {
  int32_t hidden;
  int32_t num_k_heads_local;
  int32_t num_v_heads_local;
  int32_t conv_dim_local;
  int32_t tp_rank;
  int32_t tp_size;
  int64_t rec_state_floats_per_seq;  /* Hv_local * 128 * 128 */
  int64_t conv_state_floats_per_seq; /* 3 * conv_dim_local */
  int64_t workspace_bytes;           /* currently reserved workspace */
} gdn_layer_info;

typedef struct gdn_layer gdn_layer; /* opaque */
typedef struct gdn_comm gdn_comm;   /* opaque: a NCCL communicator over the tensor-parallel group */

/* Build a layer handle for tensor-parallel rank `tp_rank` of `tp_size` (1 = single GPU), on the current
 * CUDA device.  Rank r owns k-heads [r*Hk/G, (r+1)*Hk/G) and v-heads [r*Hv/G, (r+1)*Hv/G): in_proj rows
 * of those heads, out_proj columns of those v-heads.  Hv/Hk above 8 returns GDN_ERR_UNSUPPORTED (the
 * Qwen3.5 layers use 1 and 2).  Replaces Qwen35GatedDeltaNetTT.__init__
 * (9B/gdn_layer.py:55-78) and Qwen35_08B_GDNStackL1's per-layer _Layer (0.8B/gdn_l1.py:91-130). */
GDN_API gdn_status gdn_layer_create(const gdn_dims* dims, const gdn_weights* weights, int32_t tp_rank, int32_t tp_size,
                            gdn_layer** out_layer);

GDN_API gdn_status gdn_layer_destroy(gdn_layer* layer);

GDN_API gdn_status gdn_layer_get_info(const gdn_layer* layer, gdn_layer_info* info);

/* Pre-allocate the workspace for calls of up to `max_tokens` = B*T rows in at most 64 sequences, so that
 * later forwards allocate nothing (required before capturing forwards into a CUDA graph).  The reference
 * sizes its device buffers for max_rows rows in its constructor (9B/gdn_layer.py:55-66). */
GDN_API gdn_status gdn_layer_reserve(gdn_layer* layer, int64_t max_tokens);

/* gdn_layer_reserve for calls of up to `max_tokens` rows in at most `max_batch` sequences (a prefill call of
 * B sequences needs room for B * ceil(T / 64) chunks, at most max_tokens / 64 + max_batch).  With a row limit
 * (gdn_layer_set_max_rows, set first), max_tokens >= max_rows reserves for calls of any length. */
GDN_API gdn_status gdn_layer_reserve_batch(gdn_layer* layer, int64_t max_tokens, int32_t max_batch);

/* Row limit for prefill calls: a call of B * T > max_rows rows runs as consecutive pieces of tc tokens of
 * every sequence (tc = max_rows / B, rounded down to a multiple of 64 when at least 64), each continuing
 * from the state the previous piece left, so the workspace stays bounded by max_rows rows whatever the
 * input length; max_rows below the batch is rejected at the call.  0 (the default) = no limit.  Pieces of
 * more than one sequence are gathered into contiguous rows of the workspace and scattered back.  With
 * tp_size > 1 every rank must set the same limit (each piece is one all-reduce).  The reference's
 * constructor argument max_rows and its __call__ loop (9B/gdn_layer.py:55-66, 282-292). */
GDN_API gdn_status gdn_layer_set_max_rows(gdn_layer* layer, int64_t max_rows);

/* `layer` drops its own workspace and from now on uses `owner`'s (reference counted; it grows to the largest
 * call any sharer makes), so that the layers of a stack hold one workspace between them instead of one each
 * (a 24-layer stack prefilling 128 x 4096 tokens needs ~40 GB of intermediates once, not 24 times).  Sharers
 * must issue their calls on one stream.  The reference's stack owns one constants tensor and one set of
 * work buffers for all its layers (0.8B/gdn_l1.py:186-190, 214-221); this is the device-memory counterpart
 * (there is no separate reference call). */
GDN_API gdn_status gdn_layer_share_workspace(gdn_layer* layer, gdn_layer* owner);

/* Weight formats (the reference's weight_dtype argument: ttnn.bfloat16 / bfloat8_b, 9B/gdn_layer.py:55,90-119,
 * 0.8B/gdn_l1.py:155). */
enum {
  GDN_WEIGHTS_BF16 = 0,             /* as created */
  GDN_WEIGHTS_FP8_E4M3 = 1,         /* e4m3 weights AND e4m3 decode activations (per-token scales) */
  GDN_WEIGHTS_FP8_WEIGHT_ONLY = 2   /* e4m3 weights, bf16 activations: the reference's bfloat8_b semantics */
};

/* Switch a layer's projection weights to `format` (once; the bf16 originals are not kept).  Both fp8 formats
 * quantise every output row of the fused in_proj and of out_proj to e4m3 with the smallest power-of-two
 * scale that keeps the WHOLE row within +-448 (out_proj rows are split across tensor-parallel ranks by
 * columns; their scales come from the full rows, so every shard quantises exactly as one GPU would).
 * Prefill calls use the dequantised weights (exact in bf16) with bf16 activations.  Decode calls (T == 1)
 * stream the e4m3 weights (half the bytes):
 *   GDN_WEIGHTS_FP8_WEIGHT_ONLY  activations stay bf16; each e4m3 weight stage is widened to bf16 in shared
 *                                memory for the bf16 tensor cores (the reference quantises weights only:
 *                                weight_dtype=bfloat8_b, 9B/gdn_layer.py:55,90-119, 0.8B/test_gdn_l1.py:24-52);
 *                                any tp_size;
 *   GDN_WEIGHTS_FP8_E4M3         activations are quantised per token to e4m3 too and the projections run as
 *                                e4m3 x e4m3 tensor-core GEMMs; tp_size 1 only.
 * gdn_layer_decode_static is unavailable for fp8 layers. */
GDN_API gdn_status gdn_layer_set_weight_format(gdn_layer* layer, int32_t format);

/* One layer call that continues from (rec_state, conv_state) and updates both in place:
 *   T == 1  decode step (one token per sequence);  T > 1  chunked prefill of T tokens per sequence.
 * out receives the layer output (bf16 [B, T, hidden]); with tp_size > 1 every rank receives the full,
 * all-reduced output (one all-reduce per call over `comm`: the NVLink peer-memory kernel for decode outputs
 * up to 8 MiB, NCCL above).  With comm == NULL the call skips the
 * all-reduce and out holds this rank's partial sum (for callers that reduce themselves).
 * Replaces Qwen35GatedDeltaNetTT.__call__ / _forward_rows (9B/gdn_layer.py:244-292) and
 * Qwen35_08B_GDNStackL1.forward_device (0.8B/gdn_l1.py:295-307).  x may alias nothing else.  The device
 * the layer was created on must be current (GDN_ERR_INVALID_ARGUMENT otherwise, before any launch). */
GDN_API gdn_status gdn_layer_forward(gdn_layer* layer, const uint16_t* x, int32_t batch, int32_t seq_len, float* rec_state,
                             float* conv_state, uint16_t* out, gdn_comm* comm, void* stream);

/* Optional stage timing: each forward records events[i] (cudaEvent_t, created by the caller) on its stream:
 * 0 start, 1 after in_proj, 2 after the prefill conv, 3 after the chunk preparation (2 and 3 coincide with
 * 1 for decode), 4 after the recurrence (decode kernel or chunked state pass), 5 after out_proj, 6 after
 * the all-reduce.  count 0 disables, at most 7.  The reference
 * measures the same per-op split with its device profiler (9B/README.md:137-145). */
GDN_API gdn_status gdn_layer_set_stage_events(gdn_layer* layer, void* const* events, int32_t count);

/* One decode step (seq_len 1) that allocates no device memory, for callers that cannot call cudaMalloc
 * during a call: code running inside a memory budget owned by another runtime, or code issuing calls while
 * a stream is being captured (an allocation there breaks the capture).  No counterpart in the reference.
 * Same math, inputs and outputs as gdn_layer_forward with seq_len = 1 and comm = NULL (with tp_size > 1, out
 * holds this rank's partial sum).  The step's intermediates live in a static device array of 8 MiB that
 * every GPU loading this library keeps until exit; a batch whose intermediates do not fit
 * (batch * (4 * proj_ld + 2 * Hv_local * 128) bytes, about 145 sequences for the 9B geometry) is rejected
 * with GDN_ERR_INVALID_ARGUMENT.  The first call on each device looks up the array's device address; make
 * that first call before any stream capture.  The address is looked up again after the device's context
 * was reset (cudaDeviceReset), so the first call after a reset is a first call too.  All calls share the one
 * array: calls whose GPU work overlaps (different streams, or different layers on concurrent streams) race
 * on it.  The device the layer was created on must be current. */
GDN_API gdn_status gdn_layer_decode_static(gdn_layer* layer, const uint16_t* x, int32_t batch, float* rec_state,
                                           float* conv_state, uint16_t* out, void* stream);

/* ---- The decoder layer around the mixer --------------------------------------------------------------
 * A Qwen3.5 decoder layer of the linear-attention type (Hugging Face Qwen3_5DecoderLayer.forward):
 *   h = x + mixer(RMSNorm(x) * (1 + w_in));   out = h + down(SiLU(gate(n)) * up(n)),  n = RMSNorm(h) * (1 + w_post)
 * The reference stacks GDN mixers only (0.8B/gdn_l1.py:295-325) and names these surroundings -- input
 * RMSNorm, residual, MLP -- as its next step (0.8B/OPTIMIZATION.md:258-259). */
typedef struct gdn_mlp_weights {
  const float* input_norm_w;  /* fp32 [hidden]                 input_layernorm.weight (applied as 1 + w) */
  const float* post_norm_w;   /* fp32 [hidden]                 post_attention_layernorm.weight           */
  const uint16_t* w_gate;     /* bf16 [intermediate, hidden]   mlp.gate_proj.weight                      */
  const uint16_t* w_up;       /* bf16 [intermediate, hidden]   mlp.up_proj.weight                        */
  const uint16_t* w_down;     /* bf16 [hidden, intermediate]   mlp.down_proj.weight                      */
  int32_t intermediate;       /* a multiple of 64 * tp_size */
  float eps;                  /* rms_norm_eps */
} gdn_mlp_weights;

typedef struct gdn_decoder gdn_decoder; /* opaque */

/* A decoder layer around `mixer` (which stays owned by the caller and must outlive it), on the mixer's
 * device and tensor-parallel shard: the MLP is split by intermediate columns (gate/up rows, down columns),
 * giving a partial output that one more all-reduce sums.  Pointers may be host or device memory. */
GDN_API gdn_status gdn_decoder_create(gdn_layer* mixer, const gdn_mlp_weights* weights, gdn_decoder** out_decoder);
GDN_API gdn_status gdn_decoder_destroy(gdn_decoder* decoder);
/* Pre-allocate the decoder's own workspace for calls of up to max_tokens rows (the mixer's is reserved with
 * gdn_layer_reserve / gdn_layer_reserve_batch). */
GDN_API gdn_status gdn_decoder_reserve(gdn_decoder* decoder, int64_t max_tokens);
/* One decoder-layer call, continuing the mixer's state like gdn_layer_forward (T == 1 decode, T > 1
 * prefill).  out bf16 [B, T, hidden] must not alias x.  With tp_size > 1, comm is required (the post-mixer
 * norm needs the full mixer output) and every rank receives the full output: two all-reduces per call. */
GDN_API gdn_status gdn_decoder_forward(gdn_decoder* decoder, const uint16_t* x, int32_t batch, int32_t seq_len,
                                       float* rec_state, float* conv_state, uint16_t* out, gdn_comm* comm, void* stream);

/* Recurrence only (no projections, conv or norm), token by token, state updated in place:
 *   q, k fp32 [B, T, Hk, 128]; v fp32 [B, T, Hv, 128]; g (log decay), beta fp32 [B, T, Hv];
 *   state fp32 [B, Hv, 128, 128]; o fp32 [B, T, Hv, 128].
 * scale <= 0 means 128^-0.5.  Replaces GatedDeltaRuleL1.__call__ / forward_packed
 * (9B/gated_delta_l1.py:247-272) with the math of 9B/reference.py:11-35. */
GDN_API gdn_status gdn_recurrence_forward(const float* q, const float* k, const float* v, const float* g, const float* beta,
                                  int32_t batch, int32_t seq_len, int32_t num_k_heads, int32_t num_v_heads,
                                  int32_t use_qk_l2norm, float scale, float* state, float* o, void* stream);

/* The tcgen05 GEMM building block of the layer's projections: C = A * B^T with A bf16 [m, k] (row stride
 * lda) and B bf16 [n, k] (row stride ldb), fp32 accumulation.  out_kind: 0 = fp32 C[m][n], 1 = bf16 C[m][n],
 * 2 = fp32 C[n][m] (transposed), 3 = bf16 C[n][m]; ldo is the output row stride.  ksplit 0 = automatic,
 * 1..8 = K split over a thread-block cluster.  The reference's projections are ttnn.linear calls
 * (9B/gdn_layer.py:255-259,272-276). */
GDN_API gdn_status gdn_gemm_bf16(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int32_t m, int32_t n,
                                 int32_t k, int32_t out_kind, void* out, int64_t ldo, int32_t ksplit, void* stream);

/* Tensor-parallel communicator (NCCL, loaded at run time).  Rank 0 calls gdn_comm_get_unique_id and
 * shares the 128 bytes with the other ranks out of band; every rank then calls gdn_comm_create with its
 * own CUDA device current. */
GDN_API gdn_status gdn_comm_get_unique_id(void* id_out, size_t id_bytes);
GDN_API gdn_status gdn_comm_create(const void* id, size_t id_bytes, int32_t rank, int32_t world, gdn_comm** out_comm);
GDN_API gdn_status gdn_comm_destroy(gdn_comm* comm);
/* In-place all-gather over the communicator on `stream`: rank r's bytes_per_rank bytes at
 * buf + r * bytes_per_rank are copied to the same offset on every rank (ncclAllGather).  Used to give every
 * rank of a tensor-parallel layer the whole input when each rank copied only its share from the host. */
GDN_API gdn_status gdn_comm_allgather(gdn_comm* comm, void* buf, size_t bytes_per_rank, void* stream);

/* Synchronises the current device and returns (and clears) the device error word that bounded waits
 * inside the kernels set; 0 = no error.  After a peer-wait code (0x105: an NVLink all-reduce gave up
 * waiting for another rank) the ranks' call epochs of that communicator may disagree: destroy the
 * communicator on every rank and create a new one before the next tensor-parallel call. */
GDN_API gdn_status gdn_device_error(int32_t* code_out);

/* Failure-detection self-test: one thread waits, with the all-reduce's bounded peer wait, until the u64 at
 * the device address `flag` reaches `value`.  A flag that nothing sets makes the wait expire (after 2 s);
 * the kernel then records GDN's peer-wait error code (0x105) in the device error word and returns, and the
 * context stays usable.  Lets a test exercise the timeout path without a second rank or any GPU fault. */
GDN_API gdn_status gdn_selftest_peer_wait(const uint64_t* flag, uint64_t value, void* stream);

/* Human-readable description of the last error on the calling thread ("" if none). */
GDN_API const char* gdn_last_error_string(void);

/* Number of CUDA kernels this library has launched since it was loaded. */
GDN_API uint64_t gdn_kernel_launch_count(void);

/* ABI version (GDN_ABI_VERSION) of the loaded library. */
GDN_API int32_t gdn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
