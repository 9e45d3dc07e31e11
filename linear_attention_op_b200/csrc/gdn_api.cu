// C-ABI implementation: layer handles (head-sharded weight copies, workspace), the decode and prefill
// pipelines, the recurrence-only op, and the NCCL communicator (loaded with dlopen so the library has no
// link-time NCCL dependency).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "../../include/gdn_b200.h"
#include "gemm.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

using namespace gdn;

// ------------------------------------------------------------------------------------------------
// Errors
// ------------------------------------------------------------------------------------------------
static thread_local std::string t_last_error;

static gdn_status fail(gdn_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return st;
}

#define GDN_CUDA(call)                                                                                   \
  do {                                                                                                   \
    cudaError_t _e = (call);                                                                             \
    if (_e != cudaSuccess) {                                                                             \
      if (_e == cudaErrorMemoryAllocation)                                                               \
        return fail(GDN_ERR_OUT_OF_MEMORY, "%s: %s (%s:%d)", #call, cudaGetErrorString(_e), __FILE__,    \
                    __LINE__);                                                                           \
      return fail(GDN_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(_e), __FILE__, __LINE__);   \
    }                                                                                                    \
  } while (0)

// ------------------------------------------------------------------------------------------------
// NCCL (dlopen)
// ------------------------------------------------------------------------------------------------
struct NcclApi {
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*getErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

static const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy torch already loaded, if any
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.getUniqueId = reinterpret_cast<decltype(api.getUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.commInitRank = reinterpret_cast<decltype(api.commInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.commDestroy = reinterpret_cast<decltype(api.commDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.allReduce = reinterpret_cast<decltype(api.allReduce)>(dlsym(h, "ncclAllReduce"));
    api.allGather = reinterpret_cast<decltype(api.allGather)>(dlsym(h, "ncclAllGather"));
    api.getErrorString = reinterpret_cast<decltype(api.getErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.getUniqueId && api.commInitRank && api.commDestroy && api.allReduce && api.allGather &&
             api.getErrorString;
  });
  return api;
}

// The communicator: NCCL for prefill, and for decode outputs up to kP2PSlotBytes a one-shot NVLink
// all-reduce over buffers that every rank maps from every other rank with CUDA IPC.
// Mapped layout: flag page (arrive[8] u64 | ... | epoch u64 at [16] | cta_done u32[2] at [17] | ... |
// reduced[rank][cta] u64 from [kP2PReducedOff]) | slot 0 at +kP2PSlotOffset | slot 1.
constexpr size_t kP2PSlotBytes = size_t(8) << 20;
constexpr size_t kP2PSlotOffset = 32768;
static_assert(kP2PFlagPageBytes <= static_cast<int>(kP2PSlotOffset), "flag page overlaps slot 0");
struct gdn_comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  bool p2p = false;
  char* sym = nullptr;                       // this rank's mapped page (cudaMalloc)
  char* peer[kP2PMaxRanks] = {};             // every rank's page in this process (own = sym)
};

// Maps every rank's page into every process (collective over the NCCL communicator).  On any failure the
// communicator keeps NCCL only.
static void p2p_setup(gdn_comm* c) {
  const NcclApi& api = nccl();
  if (c->world < 2 || c->world > kP2PMaxRanks) return;
  // The scratch for the two collectives below comes first: once it exists every rank takes part in both,
  // even after a local failure (a rank that failed contributes a zero handle and votes no), so no rank
  // waits for good.
  cudaStream_t s = nullptr;
  char* hbuf = nullptr;
  const size_t hbytes = sizeof(cudaIpcMemHandle_t) * (c->world + 1);
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&hbuf, hbytes + 16) != cudaSuccess) {
    if (s) cudaStreamDestroy(s);
    cudaGetLastError();
    return;
  }
  int* flag = reinterpret_cast<int*>(hbuf + hbytes);
  bool ok = cudaMalloc(&c->sym, kP2PSlotOffset + 2 * kP2PSlotBytes) == cudaSuccess &&
            cudaMemset(c->sym, 0, kP2PSlotOffset) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  cudaIpcMemHandle_t mine;
  ok = ok && cudaIpcGetMemHandle(&mine, c->sym) == cudaSuccess;
  if (!ok) memset(&mine, 0, sizeof(mine));
  cudaMemcpy(hbuf + sizeof(cudaIpcMemHandle_t) * c->world, &mine, sizeof(mine), cudaMemcpyHostToDevice);
  cudaIpcMemHandle_t all[kP2PMaxRanks];
  const bool gathered =
      api.allGather(hbuf + sizeof(cudaIpcMemHandle_t) * c->world, hbuf, sizeof(cudaIpcMemHandle_t), ncclChar, c->comm,
                    s) == ncclSuccess &&
      cudaStreamSynchronize(s) == cudaSuccess &&
      cudaMemcpy(all, hbuf, sizeof(cudaIpcMemHandle_t) * c->world, cudaMemcpyDeviceToHost) == cudaSuccess;
  ok = ok && gathered;
  const cudaIpcMemHandle_t zero{};
  for (int p = 0; ok && p < c->world; ++p) ok = memcmp(&all[p], &zero, sizeof(zero)) != 0;
  for (int p = 0; ok && p < c->world; ++p) {
    if (p == c->rank) {
      c->peer[p] = c->sym;
      continue;
    }
    void* ptr = nullptr;
    ok = cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    c->peer[p] = static_cast<char*>(ptr);
  }
  // Agree on the outcome: a rank that failed must not leave the others on the P2P path.
  int vote = ok ? 1 : 0;
  cudaMemcpy(flag, &vote, sizeof(int), cudaMemcpyHostToDevice);
  if (api.allReduce(flag, flag, 1, ncclInt32, ncclMin, c->comm, s) == ncclSuccess &&
      cudaStreamSynchronize(s) == cudaSuccess && cudaMemcpy(&vote, flag, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess)
    c->p2p = vote == 1;
  cudaFree(hbuf);
  cudaStreamDestroy(s);
  cudaGetLastError();
}

static void p2p_teardown(gdn_comm* c) {
  cudaDeviceSynchronize();
  for (int p = 0; p < kP2PMaxRanks; ++p)
    if (c->peer[p] && c->peer[p] != c->sym) cudaIpcCloseMemHandle(c->peer[p]);
  if (c->sym) cudaFree(c->sym);
  cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// Layer
// ------------------------------------------------------------------------------------------------
// Device workspace for the intermediates of a call.  Layers that issue their calls on one stream (the
// layers of a stack) may share one (gdn_layer_share_workspace): it is reference counted and grows to the
// largest call any of them makes, so a stack of L layers holds one prefill workspace instead of L.
struct WsBlock {
  void* ptr = nullptr;
  size_t bytes = 0;
  int refs = 1;
};

struct gdn_layer {
  gdn_dims dims{};
  int tp_rank = 0, tp_size = 1;
  int device = 0;
  int hk = 0, hv = 0;              // local heads
  int kd = 0, vd = 0, conv_dim = 0; // local channel counts
  int rows = 0;                     // fused in_proj rows: conv_dim + vd + 2 hv
  int proj_ld = 0;                  // row stride of the in_proj output buffer: rows rounded up to 8
  __nv_bfloat16* w_in = nullptr;    // [rows, hidden] = [q | k | v | z | a | b], pre-tiled (tiled_weight_bytes)
  __nv_bfloat16* w_out = nullptr;   // [hidden, vd], pre-tiled
  float* conv_w = nullptr;          // [conv_dim, 4]
  float* a_log = nullptr;           // [hv]
  float* dt_bias = nullptr;         // [hv]
  float* norm_w = nullptr;          // [128]
  // fp8 weights (gdn_layer_set_weight_format): e4m3 copies of w_in / w_out in the streaming layout with
  // 128-element K blocks and their per-row power-of-two scales; w_in / w_out then hold the dequantised
  // values, which the bf16 (prefill) GEMMs use.
  uint8_t* w_in8 = nullptr;
  uint8_t* w_out8 = nullptr;
  float* s_in = nullptr;            // [rows]
  float* s_out = nullptr;           // [hidden]
  int wformat = GDN_WEIGHTS_BF16;   // gdn_layer_set_weight_format
  float* out_amax = nullptr;        // tp_size > 1: max |W_out| over each WHOLE output row (all ranks' columns)
  WsBlock* ws = nullptr;            // never null after gdn_layer_create
  cudaEvent_t stage_events[7] = {};  // optional stage timing (gdn_layer_set_stage_events)
  int n_stage_events = 0;
  int64_t max_rows = 0;             // prefill row limit per launch sequence (gdn_layer_set_max_rows); 0 = none
};

static size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// Workspace layout for n token rows in `chunks` (sequence, chunk) pairs (chunks >= B for prefill):
//   proj fp32 [n, proj_ld] (conv channels already convolved) | y bf16 [n, vd] |
//   conv tail fp32 [chunks, 3, conv_dim] | chunk tile images | (fp8 decode) e4m3 x [n, hidden], x scales
//   [n], e4m3 y [n, vd], y scales [n]
struct WsLayout {
  size_t y, tail, chunk, q8, total;
};
static size_t q8_bytes(const gdn_layer* L, int64_t n) {
  return align256(n * L->dims.hidden) + align256(n * 4) + align256(n * L->vd) + align256(n * 4);
}
static WsLayout ws_layout(const gdn_layer* L, int64_t n, int64_t chunks, bool f8 = false) {
  WsLayout o;
  o.y = align256(n * L->proj_ld * 4);
  o.tail = o.y + align256(n * L->vd * 2);
  o.chunk = o.tail + align256(static_cast<size_t>(chunks) * 3 * L->conv_dim * 4);
  o.q8 = o.chunk + align256(chunk_prefill_scratch_bytes(1, 64, L->hk, L->hv) * static_cast<size_t>(chunks));
  o.total = o.q8 + (f8 ? q8_bytes(L, n) : 0);
  return o;
}
// Row-limited prefill (gdn_layer_set_max_rows): the token range [t0, t0 + tc) of every sequence is one piece
// of B * tc rows.  Pieces of more than one sequence are gathered into contiguous staging rows (x, then out)
// placed after the piece's own workspace layout.
struct PiecePlan {
  int tc = 0;            // tokens per sequence per piece
  int64_t rows = 0;      // B * tc
  int64_t chunks = 0;    // B * ceil(tc / 64)
  size_t stage = 0;      // offset of the staging rows in the workspace (0: no staging, B == 1)
  size_t total = 0;      // workspace bytes the split call needs
};
static PiecePlan piece_plan(const gdn_layer* L, int B) {
  PiecePlan p;
  p.tc = static_cast<int>(std::min<int64_t>(L->max_rows / B, INT32_MAX));
  if (p.tc >= 64) p.tc &= ~63;  // pieces end where a single call's chunks would end
  p.rows = static_cast<int64_t>(B) * p.tc;
  p.chunks = static_cast<int64_t>(B) * ((p.tc + 63) / 64);
  const size_t base = ws_layout(L, p.rows, p.chunks, L->wformat == GDN_WEIGHTS_FP8_E4M3).total;
  const size_t xrows = align256(static_cast<size_t>(p.rows) * L->dims.hidden * 2);
  p.stage = B > 1 ? base : 0;
  p.total = base + (B > 1 ? 2 * xrows : 0);
  return p;
}
static gdn_status ensure_bytes(gdn_layer* L, size_t need, int64_t n, cudaStream_t stream) {
  WsBlock* w = L->ws;
  if (need <= w->bytes) return GDN_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
    return fail(GDN_ERR_INVALID_ARGUMENT,
                "workspace for %lld rows is not reserved; call gdn_layer_reserve before stream capture",
                static_cast<long long>(n));
  if (w->ptr) GDN_CUDA(cudaFree(w->ptr));  // synchronises: no sharer's call still uses the old block
  w->ptr = nullptr;
  w->bytes = 0;
  GDN_CUDA(cudaMalloc(&w->ptr, need));
  w->bytes = need;
  return GDN_OK;
}
static gdn_status ensure_workspace(gdn_layer* L, int64_t n, int64_t chunks, cudaStream_t stream, bool f8 = false) {
  return ensure_bytes(L, ws_layout(L, n, chunks, f8).total, n, stream);
}

static void release_ws(WsBlock* w) {
  if (w && --w->refs == 0) {
    if (w->ptr) cudaFree(w->ptr);
    delete w;
  }
}

static void free_layer(gdn_layer* L) {
  if (!L) return;
  for (void* p : {static_cast<void*>(L->w_in), static_cast<void*>(L->w_out), static_cast<void*>(L->conv_w),
                  static_cast<void*>(L->a_log), static_cast<void*>(L->dt_bias), static_cast<void*>(L->norm_w),
                  static_cast<void*>(L->w_in8), static_cast<void*>(L->w_out8), static_cast<void*>(L->s_in),
                  static_cast<void*>(L->s_out), static_cast<void*>(L->out_amax)})
    if (p) cudaFree(p);
  release_ws(L->ws);
  delete L;
}

// Copy `nrows` rows of `cols` elements (elem bytes each) from a (host or device) matrix with row stride
// src_ld into a dense destination.
static cudaError_t copy_rows(void* dst, const void* src, int64_t src_ld, int64_t row0, int64_t nrows, int64_t cols,
                             size_t elem) {
  return cudaMemcpy2D(dst, cols * elem, static_cast<const char*>(src) + row0 * src_ld * elem, src_ld * elem,
                      cols * elem, nrows, cudaMemcpyDefault);
}

extern "C" gdn_status gdn_layer_create(const gdn_dims* dims, const gdn_weights* w, int32_t tp_rank, int32_t tp_size,
                                       gdn_layer** out_layer) {
  if (!dims || !w || !out_layer) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_create: null argument");
  *out_layer = nullptr;
  const gdn_dims d = *dims;
  if (!w->w_qkv || !w->w_z || !w->w_a || !w->w_b || !w->conv_w || !w->a_log || !w->dt_bias || !w->norm_w ||
      !w->w_out)
    return fail(GDN_ERR_NULL_POINTER, "gdn_layer_create: a weight pointer is null");
  if (d.head_k_dim != kHeadDim || d.head_v_dim != kHeadDim)
    return fail(GDN_ERR_UNSUPPORTED, "head dims %d/%d unsupported (only 128)", d.head_k_dim, d.head_v_dim);
  if (d.conv_kernel != 4) return fail(GDN_ERR_UNSUPPORTED, "conv kernel %d unsupported (only 4)", d.conv_kernel);
  if (d.chunk != 0 && d.chunk != 64) return fail(GDN_ERR_UNSUPPORTED, "chunk %d unsupported (only 64)", d.chunk);
  if (d.hidden <= 0 || d.hidden % 64)
    return fail(GDN_ERR_INVALID_ARGUMENT, "hidden %d must be a positive multiple of 64", d.hidden);
  if (d.num_k_heads <= 0 || d.num_v_heads <= 0 || d.num_v_heads % d.num_k_heads)
    return fail(GDN_ERR_INVALID_ARGUMENT, "num_v_heads %d must be a multiple of num_k_heads %d", d.num_v_heads,
                d.num_k_heads);
  if (d.num_v_heads / d.num_k_heads > 8)
    return fail(GDN_ERR_UNSUPPORTED, "%d v-heads per k-head unsupported (at most 8: one thread-block cluster)",
                d.num_v_heads / d.num_k_heads);
  if (!(d.eps > 0.f)) return fail(GDN_ERR_INVALID_ARGUMENT, "eps must be > 0");
  if (tp_size <= 0 || tp_rank < 0 || tp_rank >= tp_size)
    return fail(GDN_ERR_INVALID_ARGUMENT, "tp_rank %d / tp_size %d", tp_rank, tp_size);
  if (d.num_k_heads % tp_size || d.num_v_heads % tp_size)
    return fail(GDN_ERR_INVALID_ARGUMENT, "tp_size %d must divide num_k_heads %d and num_v_heads %d", tp_size,
                d.num_k_heads, d.num_v_heads);

  gdn_layer* L = new (std::nothrow) gdn_layer();
  if (!L) return fail(GDN_ERR_OUT_OF_MEMORY, "host allocation failed");
  L->ws = new (std::nothrow) WsBlock();
  if (!L->ws) {
    delete L;
    return fail(GDN_ERR_OUT_OF_MEMORY, "host allocation failed");
  }
  L->dims = d;
  L->tp_rank = tp_rank;
  L->tp_size = tp_size;
  cudaGetDevice(&L->device);
  L->hk = d.num_k_heads / tp_size;
  L->hv = d.num_v_heads / tp_size;
  L->kd = L->hk * kHeadDim;
  L->vd = L->hv * kHeadDim;
  L->conv_dim = 2 * L->kd + L->vd;
  L->rows = L->conv_dim + L->vd + 2 * L->hv;
  L->proj_ld = (L->rows + 7) & ~7;
  const int64_t h = d.hidden;
  const int64_t kd_g = static_cast<int64_t>(d.num_k_heads) * kHeadDim;
  const int64_t k0 = static_cast<int64_t>(tp_rank) * L->kd;  // first local q/k channel (global index)
  const int64_t v0 = static_cast<int64_t>(tp_rank) * L->vd;  // first local v/z channel
  const int64_t hv0 = static_cast<int64_t>(tp_rank) * L->hv; // first local v-head

  __nv_bfloat16* w_in_rm = nullptr;   // row-major staging copies, tiled into L->w_in / L->w_out below
  __nv_bfloat16* w_out_rm = nullptr;
  auto run = [&]() -> gdn_status {
    GDN_CUDA(cudaMalloc(&w_in_rm, static_cast<size_t>(L->rows) * h * 2));
    GDN_CUDA(cudaMalloc(&w_out_rm, static_cast<size_t>(h) * L->vd * 2));
    GDN_CUDA(cudaMalloc(&L->w_in, tiled_weight_bytes(L->rows, static_cast<int>(h))));
    GDN_CUDA(cudaMalloc(&L->w_out, tiled_weight_bytes(static_cast<int>(h), L->vd)));
    GDN_CUDA(cudaMalloc(&L->conv_w, static_cast<size_t>(L->conv_dim) * 4 * 4));
    GDN_CUDA(cudaMalloc(&L->a_log, L->hv * 4));
    GDN_CUDA(cudaMalloc(&L->dt_bias, L->hv * 4));
    GDN_CUDA(cudaMalloc(&L->norm_w, kHeadDim * 4));
    char* win = reinterpret_cast<char*>(w_in_rm);
    int64_t r = 0;
    // q, k, v rows of in_proj_qkv, then z, a, b
    GDN_CUDA(copy_rows(win + r * h * 2, w->w_qkv, h, k0, L->kd, h, 2)); r += L->kd;
    GDN_CUDA(copy_rows(win + r * h * 2, w->w_qkv, h, kd_g + k0, L->kd, h, 2)); r += L->kd;
    GDN_CUDA(copy_rows(win + r * h * 2, w->w_qkv, h, 2 * kd_g + v0, L->vd, h, 2)); r += L->vd;
    GDN_CUDA(copy_rows(win + r * h * 2, w->w_z, h, v0, L->vd, h, 2)); r += L->vd;
    GDN_CUDA(copy_rows(win + r * h * 2, w->w_a, h, hv0, L->hv, h, 2)); r += L->hv;
    GDN_CUDA(copy_rows(win + r * h * 2, w->w_b, h, hv0, L->hv, h, 2)); r += L->hv;
    // conv taps of the same channels
    char* cw = reinterpret_cast<char*>(L->conv_w);
    GDN_CUDA(copy_rows(cw, w->conv_w, 4, k0, L->kd, 4, 4));
    GDN_CUDA(copy_rows(cw + static_cast<int64_t>(L->kd) * 16, w->conv_w, 4, kd_g + k0, L->kd, 4, 4));
    GDN_CUDA(copy_rows(cw + static_cast<int64_t>(2 * L->kd) * 16, w->conv_w, 4, 2 * kd_g + v0, L->vd, 4, 4));
    GDN_CUDA(cudaMemcpy(L->a_log, w->a_log + hv0, L->hv * 4, cudaMemcpyDefault));
    GDN_CUDA(cudaMemcpy(L->dt_bias, w->dt_bias + hv0, L->hv * 4, cudaMemcpyDefault));
    GDN_CUDA(cudaMemcpy(L->norm_w, w->norm_w, kHeadDim * 4, cudaMemcpyDefault));
    // out_proj columns of the local v-heads: [hidden, vd] slice of [hidden, Hv*128]
    const int64_t vd_g = static_cast<int64_t>(d.num_v_heads) * kHeadDim;
    GDN_CUDA(cudaMemcpy2D(w_out_rm, L->vd * 2, reinterpret_cast<const char*>(w->w_out) + v0 * 2, vd_g * 2,
                          L->vd * 2, h, cudaMemcpyDefault));
    GDN_CUDA(tile_weights_bf16(w_in_rm, h, L->rows, static_cast<int>(h), L->w_in, nullptr));
    GDN_CUDA(tile_weights_bf16(w_out_rm, L->vd, static_cast<int>(h), L->vd, L->w_out, nullptr));
    if (tp_size > 1) {
      // The maxima of out_proj's whole rows, for fp8 weights that every shard quantises alike (its rows are
      // split by columns across the ranks); the full matrix passes through w_in_rm's space when it fits.
      GDN_CUDA(cudaMalloc(&L->out_amax, static_cast<size_t>(h) * 4));
      void* full = nullptr;
      const size_t fbytes = static_cast<size_t>(h) * vd_g * 2;
      GDN_CUDA(cudaMalloc(&full, fbytes));
      cudaError_t e = cudaMemcpy(full, w->w_out, fbytes, cudaMemcpyDefault);
      if (e == cudaSuccess) e = row_amax_bf16(full, vd_g, static_cast<int>(h), static_cast<int>(vd_g), L->out_amax, nullptr);
      if (e == cudaSuccess) e = cudaDeviceSynchronize();
      cudaFree(full);
      GDN_CUDA(e);
    }
    GDN_CUDA(cudaDeviceSynchronize());
    return GDN_OK;
  };
  const gdn_status st = run();
  if (w_in_rm) cudaFree(w_in_rm);
  if (w_out_rm) cudaFree(w_out_rm);
  if (st != GDN_OK) {
    free_layer(L);
    return st;
  }
  *out_layer = L;
  return GDN_OK;
}

extern "C" gdn_status gdn_layer_destroy(gdn_layer* layer) {
  if (!layer) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_destroy: null layer");
  free_layer(layer);
  return GDN_OK;
}

extern "C" gdn_status gdn_layer_get_info(const gdn_layer* L, gdn_layer_info* info) {
  if (!L || !info) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_get_info: null argument");
  info->hidden = L->dims.hidden;
  info->num_k_heads_local = L->hk;
  info->num_v_heads_local = L->hv;
  info->conv_dim_local = L->conv_dim;
  info->tp_rank = L->tp_rank;
  info->tp_size = L->tp_size;
  info->rec_state_floats_per_seq = static_cast<int64_t>(L->hv) * kHeadDim * kHeadDim;
  info->conv_state_floats_per_seq = 3LL * L->conv_dim;
  info->workspace_bytes = static_cast<int64_t>(L->ws->bytes);
  return GDN_OK;
}

extern "C" gdn_status gdn_layer_reserve_batch(gdn_layer* L, int64_t max_tokens, int32_t max_batch) {
  if (!L) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_reserve_batch: null layer");
  if (max_tokens <= 0 || max_batch <= 0)
    return fail(GDN_ERR_INVALID_ARGUMENT, "max_tokens %lld and max_batch %d must be > 0",
                static_cast<long long>(max_tokens), max_batch);
  // A prefill call of B sequences of T tokens has B * ceil(T / 64) <= B * T / 64 + B chunks.  With a row
  // limit, a reservation of at least max_rows rows covers calls of any length: longer calls run in pieces
  // of at most max_rows rows plus their staging rows.
  int64_t rows = max_tokens;
  size_t stage = 0;
  if (L->max_rows > 0 && rows >= L->max_rows) {
    rows = L->max_rows;
    if (max_batch > 1) stage = 2 * align256(static_cast<size_t>(rows) * L->dims.hidden * 2);
  }
  return ensure_bytes(L, ws_layout(L, rows, rows / 64 + max_batch, L->wformat == GDN_WEIGHTS_FP8_E4M3).total + stage, max_tokens,
                      nullptr);
}

extern "C" gdn_status gdn_layer_reserve(gdn_layer* L, int64_t max_tokens) {
  if (!L) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_reserve: null layer");
  return gdn_layer_reserve_batch(L, max_tokens, 64);
}

extern "C" gdn_status gdn_layer_set_max_rows(gdn_layer* L, int64_t max_rows) {
  if (!L) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_set_max_rows: null layer");
  if (max_rows < 0) return fail(GDN_ERR_INVALID_ARGUMENT, "max_rows %lld must be >= 0", static_cast<long long>(max_rows));
  L->max_rows = max_rows;
  return GDN_OK;
}

extern "C" gdn_status gdn_layer_set_weight_format(gdn_layer* L, int32_t format) {
  if (!L) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_set_weight_format: null layer");
  if (format == L->wformat) return GDN_OK;
  if (format == GDN_WEIGHTS_BF16)
    return fail(GDN_ERR_UNSUPPORTED, "the weights are fp8 already (the bf16 originals are not kept)");
  if (format != GDN_WEIGHTS_FP8_E4M3 && format != GDN_WEIGHTS_FP8_WEIGHT_ONLY)
    return fail(GDN_ERR_INVALID_ARGUMENT, "unknown weight format %d", format);
  if (L->w_in8) return fail(GDN_ERR_UNSUPPORTED, "the weights are fp8 in another mode already");
  if (L->tp_size > 1 && format == GDN_WEIGHTS_FP8_E4M3)
    return fail(GDN_ERR_UNSUPPORTED,
                "fp8 weights with fp8 activations need tp_size 1 (the per-token activation scales of out_proj's "
                "input would differ per shard); GDN_WEIGHTS_FP8_WEIGHT_ONLY works at any tp_size");
  const int h = L->dims.hidden;
  if (h % 128 || L->vd % 128)
    return fail(GDN_ERR_UNSUPPORTED, "fp8 weights need hidden and value width multiples of 128");
  // The layer switches only once everything succeeded; before that a failure leaves it bf16.  (A failure
  // after the first in-place quantisation would leave w_in dequantised: that is reported as a CUDA error.)
  uint8_t *w_in8 = nullptr, *w_out8 = nullptr;
  float *s_in = nullptr, *s_out = nullptr;
  cudaError_t e = cudaMalloc(&w_in8, tiled_weight_bytes(L->rows, h) / 2);
  if (e == cudaSuccess) e = cudaMalloc(&w_out8, tiled_weight_bytes(h, L->vd) / 2);
  if (e == cudaSuccess) e = cudaMalloc(&s_in, static_cast<size_t>(L->rows) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s_out, static_cast<size_t>(h) * 4);
  if (e == cudaSuccess) e = quantize_tiled_weights_fp8(L->w_in, L->rows, h, w_in8, s_in, nullptr);
  if (e == cudaSuccess) e = quantize_tiled_weights_fp8(L->w_out, h, L->vd, w_out8, s_out, nullptr, L->out_amax);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    for (void* p : {static_cast<void*>(w_in8), static_cast<void*>(w_out8), static_cast<void*>(s_in),
                    static_cast<void*>(s_out)})
      if (p) cudaFree(p);
    return fail(e == cudaErrorMemoryAllocation ? GDN_ERR_OUT_OF_MEMORY : GDN_ERR_CUDA,
                "gdn_layer_set_weight_format: %s", cudaGetErrorString(e));
  }
  L->w_in8 = w_in8;
  L->w_out8 = w_out8;
  L->s_in = s_in;
  L->s_out = s_out;
  L->wformat = format;
  return GDN_OK;
}

extern "C" gdn_status gdn_layer_share_workspace(gdn_layer* L, gdn_layer* owner) {
  if (!L || !owner) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_share_workspace: null layer");
  if (L->device != owner->device)
    return fail(GDN_ERR_INVALID_ARGUMENT, "layers live on devices %d and %d", L->device, owner->device);
  if (L->ws == owner->ws) return GDN_OK;
  release_ws(L->ws);
  L->ws = owner->ws;
  ++L->ws->refs;
  return GDN_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static cudaError_t stage_mark(const gdn_layer* L, int i, cudaStream_t s) {
  return i < L->n_stage_events && L->stage_events[i] ? cudaEventRecord(L->stage_events[i], s) : cudaSuccess;
}

extern "C" gdn_status gdn_layer_set_stage_events(gdn_layer* L, void* const* events, int32_t count) {
  if (!L) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_set_stage_events: null layer");
  if (count < 0 || count > 7 || (count > 0 && !events))
    return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_layer_set_stage_events: count %d", count);
  for (int i = 0; i < 7; ++i) L->stage_events[i] = i < count ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  L->n_stage_events = count;
  return GDN_OK;
}

// One decode step (T = 1): in_proj (weights as the 128-row operand, raw fp32 projections) -> gates, conv +
// conv-state roll + gated delta rule + gated RMSNorm (decode_step_kernel, which loads the state and the
// conv history while the GEMM runs) -> out_proj, chained by programmatic dependent launch.
// proj [B, proj_ld] fp32 and y [B, vd] bf16 are scratch.
// q8: with fp8 weights, the workspace region for the e4m3 activations and their scales (q8_bytes); the
// projections then run as quantize_rows_fp8 + gemm_f8_tn.
static gdn_status decode_chain(gdn_layer* L, const uint16_t* x, int B, float* rec_state, float* conv_state,
                               float* proj, __nv_bfloat16* y, uint16_t* out, cudaStream_t stream, bool marks,
                               const unsigned long long* slot_epoch = nullptr, int64_t slot_bytes = 0,
                               void* q8 = nullptr) {
  const int h = L->dims.hidden;
  const int z_off = L->conv_dim, a_off = L->conv_dim + L->vd, b_off = a_off + L->hv;
  GemmEpiArgs ep;
  ep.a_tiled = L->w_in;
  ep.out = proj;
  ep.ld = L->proj_ld;
  uint8_t* xq = static_cast<uint8_t*>(q8);
  float* xs = q8 ? reinterpret_cast<float*>(xq + align256(static_cast<size_t>(B) * h)) : nullptr;
  uint8_t* yq = q8 ? reinterpret_cast<uint8_t*>(xs) + align256(static_cast<size_t>(B) * 4) : nullptr;
  float* ys = q8 ? reinterpret_cast<float*>(yq + align256(static_cast<size_t>(B) * L->vd)) : nullptr;
  const bool w8 = L->wformat == GDN_WEIGHTS_FP8_WEIGHT_ONLY;
  if (q8) {
    GDN_CUDA(quantize_rows_fp8(x, h, B, h, xq, xs, stream));
    ep.a_tiled = L->w_in8;
    ep.row_scale = L->s_in;
    ep.col_scale = xs;
    GDN_CUDA(gemm_f8_tn(L->w_in8, xq, h, L->rows, B, h, kEpiStoreF32T, ep, stream, true, true));
  } else if (w8) {
    ep.a_tiled = L->w_in8;
    ep.row_scale = L->s_in;
    GDN_CUDA(gemm_w8_tn(L->w_in8, x, h, L->rows, B, h, kEpiStoreF32T, ep, stream, true, true));
  } else {
    GDN_CUDA(gemm_bf16_tn(L->w_in, h, x, h, L->rows, B, h, kEpiStoreF32T, ep, 0, stream, true, true));
  }
  if (marks) {
    GDN_CUDA(stage_mark(L, 1, stream));
    GDN_CUDA(stage_mark(L, 2, stream));
    GDN_CUDA(stage_mark(L, 3, stream));
  }
  RecurrenceArgs ra;
  ra.q = proj; ra.q_tok = L->proj_ld; ra.q_head = kHeadDim;
  ra.k = proj + L->kd; ra.k_tok = L->proj_ld; ra.k_head = kHeadDim;
  ra.v = proj + 2 * L->kd; ra.v_tok = L->proj_ld; ra.v_head = kHeadDim;
  ra.z = proj + z_off; ra.z_tok = L->proj_ld; ra.z_head = kHeadDim;
  ra.g = proj + a_off; ra.g_tok = L->proj_ld; ra.g_head = 1;
  ra.beta = proj + b_off; ra.b_tok = L->proj_ld; ra.b_head = 1;
  ra.a_log = L->a_log;
  ra.dt_bias = L->dt_bias;
  ra.norm_w = L->norm_w;
  ra.eps = L->dims.eps;
  ra.y = y; ra.y_tok = L->vd; ra.y_head = kHeadDim;
  ra.state = rec_state;
  ra.B = B; ra.T = 1; ra.Hk = L->hk; ra.Hv = L->hv;
  ra.scale = 1.0f / sqrtf(static_cast<float>(kHeadDim));
  ra.l2norm = 1;
  ra.conv_w = L->conv_w;
  ra.conv_state = conv_state;
  ra.conv_dim = L->conv_dim;
  ra.k_conv = L->kd;
  ra.v_conv = 2 * L->kd;
  GDN_CUDA(decode_step_forward(ra, stream));
  if (marks) GDN_CUDA(stage_mark(L, 4, stream));
  // Without an all-reduce after it, out_proj lets its successor (the next step's in_proj) launch at once:
  // that kernel touches nothing but its weights before its own dependent wait, which returns only after
  // out_proj (and so everything before it) has completed, and SMs left idle by out_proj's CTAs start its
  // weight ring.
  const bool out_trigger = slot_epoch == nullptr;
  GemmEpiArgs eo;
  eo.out = out;
  eo.ld = h;
  eo.a_tiled = L->w_out;
  eo.slot_epoch = slot_epoch;
  eo.slot_bytes = slot_bytes;
  if (q8) {
    GDN_CUDA(quantize_rows_fp8(y, L->vd, B, L->vd, yq, ys, stream));
    eo.a_tiled = L->w_out8;
    eo.row_scale = L->s_out;
    eo.col_scale = ys;
    GDN_CUDA(gemm_f8_tn(L->w_out8, yq, L->vd, h, B, L->vd, kEpiStoreBF16T, eo, stream, true, out_trigger));
  } else if (w8) {
    eo.a_tiled = L->w_out8;
    eo.row_scale = L->s_out;
    GDN_CUDA(gemm_w8_tn(L->w_out8, y, L->vd, h, B, L->vd, kEpiStoreBF16T, eo, stream, true, out_trigger));
  } else {
    GDN_CUDA(gemm_bf16_tn(L->w_out, L->vd, y, L->vd, h, B, L->vd, kEpiStoreBF16T, eo, 0, stream, true, out_trigger));
  }
  if (marks) GDN_CUDA(stage_mark(L, 5, stream));
  return GDN_OK;
}

// The layer's buffers (weights, workspace, static scratch) belong to the device it was created on; a call
// made with another device current would hand them to kernels running elsewhere.
static gdn_status check_device(const gdn_layer* L, const char* fn) {
  int dev = -1;
  GDN_CUDA(cudaGetDevice(&dev));
  if (dev != L->device)
    return fail(GDN_ERR_INVALID_ARGUMENT, "%s: the layer lives on device %d but device %d is current", fn, L->device,
                dev);
  return GDN_OK;
}

// Decode outputs up to the slot size go through the NVLink all-reduce: the GEMM that produced the partial
// wrote it into this rank's slot for this call (GemmEpiArgs.slot_epoch).
static bool p2p_eligible(const gdn_comm* comm, int tp_size, int T, int64_t out_elems) {
  return T == 1 && tp_size > 1 && comm && comm->p2p && out_elems % 8 == 0 &&
         static_cast<size_t>(out_elems) * 2 <= kP2PSlotBytes;
}
static unsigned long long* p2p_epoch_word(gdn_comm* comm) {
  return comm ? reinterpret_cast<unsigned long long*>(comm->sym) + 2 * kP2PMaxRanks : nullptr;
}

// Sum of the ranks' bf16 partials into `out` on every rank: the NVLink kernel (partials in the slots) or
// ncclAllReduce in place (partial in `out`).
static gdn_status allreduce_out(gdn_comm* comm, uint16_t* out, int64_t out_elems, bool p2p, cudaStream_t stream) {
  if (p2p) {
    P2PAllReduceArgs ar;
    for (int p = 0; p < comm->world; ++p) {
      ar.src[p] = comm->peer[p] + kP2PSlotOffset;
      ar.flags[p] = reinterpret_cast<unsigned long long*>(comm->peer[p]);
    }
    ar.epoch = p2p_epoch_word(comm);
    ar.cta_done = reinterpret_cast<unsigned int*>(ar.epoch + 1);
    ar.out = out;
    ar.n = out_elems;
    ar.slot_bytes = static_cast<int64_t>(kP2PSlotBytes);
    ar.rank = comm->rank;
    ar.world = comm->world;
    GDN_CUDA(allreduce_p2p(ar, stream));
    return GDN_OK;
  }
  const NcclApi& api = nccl();
  if (!api.ok) return fail(GDN_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclResult_t r = api.allReduce(out, out, static_cast<size_t>(out_elems), ncclBfloat16, ncclSum, comm->comm, stream);
  if (r != ncclSuccess) return fail(GDN_ERR_NCCL, "ncclAllReduce: %s", api.getErrorString(r));
  return GDN_OK;
}

// One layer call over B * T contiguous rows, no row limit.
static gdn_status forward_rows(gdn_layer* L, const uint16_t* x, int B, int T, float* rec_state, float* conv_state,
                               uint16_t* out, gdn_comm* comm, cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(B) * T;
  const int64_t chunks = T > 1 ? static_cast<int64_t>(B) * ((T + 63) / 64) : 0;
  const bool f8 = T == 1 && L->wformat == GDN_WEIGHTS_FP8_E4M3;
  gdn_status st = ensure_workspace(L, n, chunks, stream, f8);
  if (st != GDN_OK) return st;
  const int h = L->dims.hidden;
  char* ws = static_cast<char*>(L->ws->ptr);
  const WsLayout lay = ws_layout(L, n, chunks, f8);
  float* proj = reinterpret_cast<float*>(ws);
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(ws + lay.y);
  float* conv_tail = reinterpret_cast<float*>(ws + lay.tail);
  void* chunk_scratch = ws + lay.chunk;
  const int z_off = L->conv_dim, a_off = L->conv_dim + L->vd, b_off = a_off + L->hv;

  // Tensor parallel: decode outputs are reduced by the NVLink all-reduce, so out_proj writes this rank's
  // partial into the communicator's mapped slot for this call; prefill outputs by NCCL in place.
  const int64_t out_elems = n * h;
  const bool p2p = p2p_eligible(comm, L->tp_size, T, out_elems);
  unsigned long long* p2p_epoch = p2p_epoch_word(comm);

  GDN_CUDA(stage_mark(L, 0, stream));
  if (T == 1) {
    gdn_status ds =
        p2p ? decode_chain(L, x, B, rec_state, conv_state, proj, y,
                           reinterpret_cast<uint16_t*>(comm->sym + kP2PSlotOffset), stream, true, p2p_epoch,
                           static_cast<int64_t>(kP2PSlotBytes), f8 ? ws + lay.q8 : nullptr)
            : decode_chain(L, x, B, rec_state, conv_state, proj, y, out, stream, true, nullptr, 0,
                           f8 ? ws + lay.q8 : nullptr);
    if (ds != GDN_OK) return ds;
  } else {
    // ---- prefill: in_proj with the causal conv + SiLU fused into its epilogue -> conv-state roll ->
    //      chunked recurrence + gated RMSNorm -> out_proj
    GemmEpiArgs ep;
    ep.out = proj;
    ep.ld = L->proj_ld;
    ep.conv_rows = L->conv_dim;
    ep.conv_w = L->conv_w;
    ep.conv_state = conv_state;
    ep.seq_len = T;
    ep.conv_tail = conv_tail;
    GDN_CUDA(gemm_bf16_persistent(x, h, L->w_in, static_cast<int>(n), L->rows, h, kEpiPrefillInProj, ep, stream, true));
    GDN_CUDA(stage_mark(L, 1, stream));
    GDN_CUDA(conv_state_roll_tail(conv_tail, conv_state, B, T, L->conv_dim, stream));
    GDN_CUDA(stage_mark(L, 2, stream));
    ChunkArgs ca;
    ca.qkv = proj; ca.qkv_ld = L->proj_ld;
    ca.proj = proj; ca.proj_ld = L->proj_ld;
    ca.z_off = z_off; ca.a_off = a_off; ca.b_off = b_off;
    ca.a_log = L->a_log; ca.dt_bias = L->dt_bias; ca.norm_w = L->norm_w; ca.eps = L->dims.eps;
    ca.state = rec_state; ca.y = y;
    ca.B = B; ca.T = T; ca.Hk = L->hk; ca.Hv = L->hv;
    GDN_CUDA(chunk_prep(ca, chunk_scratch, stream));
    GDN_CUDA(stage_mark(L, 3, stream));
    GDN_CUDA(chunk_state(ca, chunk_scratch, stream));
    GDN_CUDA(stage_mark(L, 4, stream));
    GemmEpiArgs eo;
    eo.out = out;
    eo.ld = h;
    eo.b_tiled = L->w_out;
    GDN_CUDA(gemm_bf16_persistent(y, L->vd, L->w_out, static_cast<int>(n), h, L->vd, kEpiStoreBF16, eo, stream, true));
    GDN_CUDA(stage_mark(L, 5, stream));
  }
  if (L->tp_size > 1 && comm) {
    const gdn_status ar = allreduce_out(comm, out, out_elems, p2p, stream);
    if (ar != GDN_OK) return ar;
  }
  GDN_CUDA(stage_mark(L, 6, stream));
  return GDN_OK;
}

extern "C" gdn_status gdn_layer_forward(gdn_layer* L, const uint16_t* x, int32_t B, int32_t T, float* rec_state,
                                        float* conv_state, uint16_t* out, gdn_comm* comm, void* stream_ptr) {
  if (!L || !x || !rec_state || !conv_state || !out) return fail(GDN_ERR_NULL_POINTER, "gdn_layer_forward: null argument");
  if (B <= 0 || T <= 0) return fail(GDN_ERR_INVALID_ARGUMENT, "batch %d and seq_len %d must be > 0", B, T);
  if (!aligned16(x) || !aligned16(out) || !aligned16(rec_state) || !aligned16(conv_state))
    return fail(GDN_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  if (L->tp_size > 1 && comm) {
    if (comm->world != L->tp_size || comm->rank != L->tp_rank)
      return fail(GDN_ERR_INVALID_ARGUMENT, "communicator rank %d/%d does not match layer rank %d/%d", comm->rank,
                  comm->world, L->tp_rank, L->tp_size);
  }
  gdn_status st = check_device(L, "gdn_layer_forward");
  if (st != GDN_OK) return st;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int64_t n = static_cast<int64_t>(B) * T;
  if (T == 1 || L->max_rows <= 0 || n <= L->max_rows)
    return forward_rows(L, x, B, T, rec_state, conv_state, out, comm, stream);

  // Row limit: tokens [t0, t0 + tc) of all B sequences per piece, the state carried from piece to piece
  // (the reference's __call__ loop over max_rows // batch tokens, 9B/gdn_layer.py:282-292).
  if (L->max_rows < B)
    return fail(GDN_ERR_INVALID_ARGUMENT, "max_rows %lld is below the batch %d", static_cast<long long>(L->max_rows),
                B);
  const PiecePlan p = piece_plan(L, B);
  st = ensure_bytes(L, p.total, p.rows, stream);
  if (st != GDN_OK) return st;
  const int64_t h = L->dims.hidden;
  char* ws = static_cast<char*>(L->ws->ptr);
  uint16_t* xs = p.stage ? reinterpret_cast<uint16_t*>(ws + p.stage) : nullptr;
  uint16_t* os = p.stage ? reinterpret_cast<uint16_t*>(ws + p.stage + align256(static_cast<size_t>(p.rows) * h * 2))
                         : nullptr;
  for (int t0 = 0; t0 < T; t0 += p.tc) {
    const int tl = std::min(p.tc, T - t0);
    const size_t row_bytes = static_cast<size_t>(tl) * h * 2, seq_pitch = static_cast<size_t>(T) * h * 2;
    if (p.stage) {
      GDN_CUDA(cudaMemcpy2DAsync(xs, row_bytes, x + t0 * h, seq_pitch, row_bytes, B, cudaMemcpyDeviceToDevice, stream));
      st = forward_rows(L, xs, B, tl, rec_state, conv_state, os, comm, stream);
      if (st != GDN_OK) return st;
      GDN_CUDA(cudaMemcpy2DAsync(out + t0 * h, seq_pitch, os, row_bytes, row_bytes, B, cudaMemcpyDeviceToDevice, stream));
    } else {
      st = forward_rows(L, x + t0 * h, 1, tl, rec_state, conv_state, out + t0 * h, comm, stream);
      if (st != GDN_OK) return st;
    }
  }
  return GDN_OK;
}

// ------------------------------------------------------------------------------------------------
// Decoder layer around the mixer (gdn_decoder_*): input RMSNorm -> GDN mixer -> residual -> post RMSNorm
// -> SwiGLU MLP -> residual, the linear-attention layer type of HF Qwen3_5DecoderLayer.forward.
// ------------------------------------------------------------------------------------------------
struct gdn_decoder {
  gdn_layer* mixer = nullptr;        // not owned
  int hidden = 0, inter = 0, inter_local = 0;
  float eps = 1e-6f;
  float* norm_in = nullptr;          // [hidden], applied as (1 + w)
  float* norm_post = nullptr;        // [hidden]
  __nv_bfloat16* w_gu = nullptr;     // [2 * inter_local, hidden], row 2j = gate_j, 2j + 1 = up_j; pre-tiled
  __nv_bfloat16* w_down = nullptr;   // [hidden, inter_local] (this rank's columns), pre-tiled
  WsBlock* ws = nullptr;             // xn / hn [n, hidden] | mixer output [n, hidden] | act [n, inter_local]
};

static void free_decoder(gdn_decoder* D) {
  if (!D) return;
  for (void* p : {static_cast<void*>(D->norm_in), static_cast<void*>(D->norm_post), static_cast<void*>(D->w_gu),
                  static_cast<void*>(D->w_down)})
    if (p) cudaFree(p);
  release_ws(D->ws);
  delete D;
}

extern "C" gdn_status gdn_decoder_create(gdn_layer* mixer, const gdn_mlp_weights* w, gdn_decoder** out) {
  if (!mixer || !w || !out) return fail(GDN_ERR_NULL_POINTER, "gdn_decoder_create: null argument");
  *out = nullptr;
  if (!w->input_norm_w || !w->post_norm_w || !w->w_gate || !w->w_up || !w->w_down)
    return fail(GDN_ERR_NULL_POINTER, "gdn_decoder_create: a weight pointer is null");
  const int G = mixer->tp_size, r = mixer->tp_rank, h = mixer->dims.hidden, I = w->intermediate;
  if (I <= 0 || I % G) return fail(GDN_ERR_INVALID_ARGUMENT, "intermediate %d must be a positive multiple of tp_size %d", I, G);
  if ((I / G) % 64) return fail(GDN_ERR_UNSUPPORTED, "intermediate per rank %d must be a multiple of 64", I / G);
  if (h > 8192) return fail(GDN_ERR_UNSUPPORTED, "hidden %d above 8192", h);
  if (!(w->eps > 0.f)) return fail(GDN_ERR_INVALID_ARGUMENT, "eps must be > 0");
  gdn_status st = check_device(mixer, "gdn_decoder_create");
  if (st != GDN_OK) return st;
  gdn_decoder* D = new (std::nothrow) gdn_decoder();
  if (!D) return fail(GDN_ERR_OUT_OF_MEMORY, "host allocation failed");
  D->ws = new (std::nothrow) WsBlock();
  if (!D->ws) {
    delete D;
    return fail(GDN_ERR_OUT_OF_MEMORY, "host allocation failed");
  }
  D->mixer = mixer;
  D->hidden = h;
  D->inter = I;
  D->inter_local = I / G;
  D->eps = w->eps;
  const int64_t il = D->inter_local, i0 = static_cast<int64_t>(r) * il;
  __nv_bfloat16 *gu_rm = nullptr, *down_rm = nullptr;
  auto run = [&]() -> gdn_status {
    GDN_CUDA(cudaMalloc(&D->norm_in, h * 4));
    GDN_CUDA(cudaMalloc(&D->norm_post, h * 4));
    GDN_CUDA(cudaMemcpy(D->norm_in, w->input_norm_w, h * 4, cudaMemcpyDefault));
    GDN_CUDA(cudaMemcpy(D->norm_post, w->post_norm_w, h * 4, cudaMemcpyDefault));
    GDN_CUDA(cudaMalloc(&gu_rm, 2 * il * h * 2));
    GDN_CUDA(cudaMalloc(&down_rm, static_cast<size_t>(h) * il * 2));
    // gate rows of this rank's columns to the even rows, up rows to the odd rows
    GDN_CUDA(cudaMemcpy2D(gu_rm, 2 * h * 2, w->w_gate + i0 * h, h * 2, h * 2, il, cudaMemcpyDefault));
    GDN_CUDA(cudaMemcpy2D(reinterpret_cast<char*>(gu_rm) + h * 2, 2 * h * 2, w->w_up + i0 * h, h * 2, h * 2, il,
                          cudaMemcpyDefault));
    GDN_CUDA(cudaMemcpy2D(down_rm, il * 2, w->w_down + i0, static_cast<size_t>(I) * 2, il * 2, h, cudaMemcpyDefault));
    GDN_CUDA(cudaMalloc(&D->w_gu, tiled_weight_bytes(static_cast<int>(2 * il), h)));
    GDN_CUDA(cudaMalloc(&D->w_down, tiled_weight_bytes(h, static_cast<int>(il))));
    GDN_CUDA(tile_weights_bf16(gu_rm, h, static_cast<int>(2 * il), h, D->w_gu, nullptr));
    GDN_CUDA(tile_weights_bf16(down_rm, il, h, static_cast<int>(il), D->w_down, nullptr));
    GDN_CUDA(cudaDeviceSynchronize());
    return GDN_OK;
  };
  st = run();
  if (gu_rm) cudaFree(gu_rm);
  if (down_rm) cudaFree(down_rm);
  if (st != GDN_OK) {
    free_decoder(D);
    return st;
  }
  *out = D;
  return GDN_OK;
}

extern "C" gdn_status gdn_decoder_destroy(gdn_decoder* D) {
  if (!D) return fail(GDN_ERR_NULL_POINTER, "gdn_decoder_destroy: null decoder");
  free_decoder(D);
  return GDN_OK;
}

static size_t decoder_ws_bytes(const gdn_decoder* D, int64_t n) {
  return 2 * align256(static_cast<size_t>(n) * D->hidden * 2) + align256(static_cast<size_t>(n) * D->inter_local * 2);
}

extern "C" gdn_status gdn_decoder_reserve(gdn_decoder* D, int64_t max_tokens) {
  if (!D) return fail(GDN_ERR_NULL_POINTER, "gdn_decoder_reserve: null decoder");
  if (max_tokens <= 0) return fail(GDN_ERR_INVALID_ARGUMENT, "max_tokens must be > 0");
  WsBlock* w = D->ws;
  const size_t need = decoder_ws_bytes(D, max_tokens);
  if (need <= w->bytes) return GDN_OK;
  if (w->ptr) GDN_CUDA(cudaFree(w->ptr));
  w->ptr = nullptr;
  w->bytes = 0;
  GDN_CUDA(cudaMalloc(&w->ptr, need));
  w->bytes = need;
  return GDN_OK;
}

extern "C" gdn_status gdn_decoder_forward(gdn_decoder* D, const uint16_t* x, int32_t B, int32_t T, float* rec_state,
                                          float* conv_state, uint16_t* out, gdn_comm* comm, void* stream_ptr) {
  if (!D || !x || !rec_state || !conv_state || !out) return fail(GDN_ERR_NULL_POINTER, "gdn_decoder_forward: null argument");
  if (B <= 0 || T <= 0) return fail(GDN_ERR_INVALID_ARGUMENT, "batch %d and seq_len %d must be > 0", B, T);
  if (!aligned16(x) || !aligned16(out)) return fail(GDN_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  if (x == out) return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_decoder_forward: out must not alias x");
  gdn_layer* L = D->mixer;
  if (L->tp_size > 1 && !comm)
    return fail(GDN_ERR_INVALID_ARGUMENT,
                "a tensor-parallel decoder layer needs its communicator (the post-mixer norm reads the full sum)");
  gdn_status st = check_device(L, "gdn_decoder_forward");
  if (st != GDN_OK) return st;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int64_t n = static_cast<int64_t>(B) * T;
  const int h = D->hidden;
  const int il = D->inter_local;
  const size_t need = decoder_ws_bytes(D, n);
  if (need > D->ws->bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
      return fail(GDN_ERR_INVALID_ARGUMENT, "decoder workspace for %lld rows is not reserved (gdn_decoder_reserve)",
                  static_cast<long long>(n));
    st = gdn_decoder_reserve(D, n);
    if (st != GDN_OK) return st;
  }
  char* ws = static_cast<char*>(D->ws->ptr);
  const size_t rows_bytes = align256(static_cast<size_t>(n) * h * 2);
  uint16_t* xn = reinterpret_cast<uint16_t*>(ws);
  uint16_t* mixed = reinterpret_cast<uint16_t*>(ws + rows_bytes);
  __nv_bfloat16* act = reinterpret_cast<__nv_bfloat16*>(ws + 2 * rows_bytes);
  // input RMSNorm -> mixer (its own all-reduce) -> h = x + mixer output (into out) and its post RMSNorm
  GDN_CUDA(rmsnorm_rows(x, nullptr, nullptr, D->norm_in, D->eps, xn, static_cast<int>(n), h, stream));
  st = gdn_layer_forward(L, xn, B, T, rec_state, conv_state, mixed, comm, stream);
  if (st != GDN_OK) return st;
  GDN_CUDA(rmsnorm_rows(x, mixed, out, D->norm_post, D->eps, xn, static_cast<int>(n), h, stream));
  // SwiGLU MLP; the residual h (in out) is added by rank 0's down-projection epilogue, before the sum
  const bool p2p = p2p_eligible(comm, L->tp_size, T, n * h);
  GemmEpiArgs eg;
  eg.out = act;
  eg.ld = il;
  GemmEpiArgs ed;
  ed.ld = h;
  ed.residual = L->tp_rank == 0 ? out : nullptr;
  ed.res_ld = h;
  if (T == 1) {
    eg.a_tiled = D->w_gu;
    GDN_CUDA(gemm_bf16_tn(D->w_gu, h, xn, h, 2 * il, B, h, kEpiSwiGLUT, eg, 0, stream, true));
    ed.a_tiled = D->w_down;
    ed.out = p2p ? static_cast<void*>(comm->sym + kP2PSlotOffset) : static_cast<void*>(out);
    ed.slot_epoch = p2p ? p2p_epoch_word(comm) : nullptr;
    ed.slot_bytes = p2p ? static_cast<int64_t>(kP2PSlotBytes) : 0;
    GDN_CUDA(gemm_bf16_tn(D->w_down, il, act, il, h, B, il, kEpiStoreBF16T, ed, 0, stream, true));
  } else {
    eg.b_tiled = D->w_gu;
    GDN_CUDA(gemm_bf16_persistent(xn, h, D->w_gu, static_cast<int>(n), 2 * il, h, kEpiSwiGLU, eg, stream, true));
    ed.out = out;
    ed.b_tiled = D->w_down;
    GDN_CUDA(gemm_bf16_persistent(act, il, D->w_down, static_cast<int>(n), h, il, kEpiStoreBF16, ed, stream, true));
  }
  if (L->tp_size > 1) return allreduce_out(comm, out, n * h, p2p, stream);
  return GDN_OK;
}

// ------------------------------------------------------------------------------------------------
// Decode step with static scratch (gdn_layer_decode_static)
//
// For callers that must not allocate device memory during a call: code running inside a memory budget
// owned by someone else (a serving runtime's pool, an embedded host without allocator access), or code
// that issues calls while a stream is being captured, where a cudaMalloc would break the capture.  The
// step's two intermediates -- the fused in_proj output (fp32 [B, proj_ld]) and the gated-RMSNorm output
// (bf16 [B, vd]) -- live in the file-scope array below instead of the layer workspace.  Every GPU that
// loads this library holds the array until the process exits.
// ------------------------------------------------------------------------------------------------
static constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

static constexpr int kMaxDevices = 64;
struct ScratchAddr {
  void* ptr = nullptr;
  unsigned long long ctx_id = 0;  // the context the address belongs to (0: not looked up)
};
static ScratchAddr g_scratch_addr[kMaxDevices];
static std::mutex g_scratch_mu;

// Unique id of the current CUDA context (cuCtxGetId, reached through the runtime's driver entry points so
// the library needs no link-time libcuda).  A context reset (cudaDeviceReset) makes a new context with a
// new id, so an address cached for the old one is looked up again instead of being reused.
typedef int (*CtxGetCurrentFn)(void** ctx);
typedef int (*CtxGetIdFn)(void* ctx, unsigned long long* id);
static gdn_status current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_current || !get_id) return fail(GDN_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId are unavailable");
  void* ctx = nullptr;
  if (get_current(&ctx) != 0 || !ctx || get_id(ctx, id) != 0)
    return fail(GDN_ERR_CUDA, "no current CUDA context");
  return GDN_OK;
}

// Device address of g_decode_scratch on the current device: looked up once per device and context, with
// that device current (the host-side symbol is only a stand-in and must never be handed to a kernel).
static gdn_status static_scratch(void** out) {
  int dev = 0;
  GDN_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(GDN_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  GDN_CUDA(cudaSetDevice(dev));  // binds the device's primary context to this thread before reading its id
  unsigned long long ctx = 0;
  gdn_status st = current_context_id(&ctx);
  if (st != GDN_OK) return st;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchAddr& a = g_scratch_addr[dev];
  if (!a.ptr || a.ctx_id != ctx) {
    void* p = nullptr;
    GDN_CUDA(cudaGetSymbolAddress(&p, g_decode_scratch));
    if (!p) return fail(GDN_ERR_CUDA, "cudaGetSymbolAddress returned null for the static scratch");
    a.ptr = p;
    a.ctx_id = ctx;
  }
  *out = a.ptr;
  return GDN_OK;
}

extern "C" gdn_status gdn_layer_decode_static(gdn_layer* L, const uint16_t* x, int32_t B, float* rec_state,
                                              float* conv_state, uint16_t* out, void* stream_ptr) {
  if (!L || !x || !rec_state || !conv_state || !out)
    return fail(GDN_ERR_NULL_POINTER, "gdn_layer_decode_static: null argument");
  if (B <= 0) return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_layer_decode_static: batch %d must be > 0", B);
  if (L->w_in8)
    return fail(GDN_ERR_UNSUPPORTED, "gdn_layer_decode_static: not available for fp8 weights (use gdn_layer_forward)");
  if (!aligned16(x) || !aligned16(out) || !aligned16(rec_state) || !aligned16(conv_state))
    return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_layer_decode_static: tensors must be 16-byte aligned");
  const size_t proj_bytes = align256(static_cast<size_t>(B) * L->proj_ld * 4);
  const size_t need = proj_bytes + align256(static_cast<size_t>(B) * L->vd * 2);
  if (need > kStaticScratchBytes)
    return fail(GDN_ERR_INVALID_ARGUMENT,
                "gdn_layer_decode_static: batch %d needs %zu bytes of scratch, the static array holds %zu "
                "(at most %zu sequences for this layer)",
                B, need, kStaticScratchBytes,
                kStaticScratchBytes / (static_cast<size_t>(L->proj_ld) * 4 + static_cast<size_t>(L->vd) * 2));
  gdn_status st = check_device(L, "gdn_layer_decode_static");
  if (st != GDN_OK) return st;
  void* base = nullptr;
  st = static_scratch(&base);
  if (st != GDN_OK) return st;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int h = L->dims.hidden;
  float* proj = static_cast<float*>(base);
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(base) + proj_bytes);
  return decode_chain(L, x, B, rec_state, conv_state, proj, y, out, stream, false);
}

extern "C" gdn_status gdn_recurrence_forward(const float* q, const float* k, const float* v, const float* g,
                                             const float* beta, int32_t B, int32_t T, int32_t Hk, int32_t Hv,
                                             int32_t use_qk_l2norm, float scale, float* state, float* o,
                                             void* stream) {
  if (!q || !k || !v || !g || !beta || !state || !o) return fail(GDN_ERR_NULL_POINTER, "gdn_recurrence_forward: null argument");
  if (B <= 0 || T <= 0 || Hk <= 0 || Hv <= 0 || Hv % Hk)
    return fail(GDN_ERR_INVALID_ARGUMENT, "bad shape B=%d T=%d Hk=%d Hv=%d", B, T, Hk, Hv);
  if (!aligned16(state)) return fail(GDN_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
  RecurrenceArgs ra;
  ra.q = q; ra.q_tok = static_cast<int64_t>(Hk) * kHeadDim; ra.q_head = kHeadDim;
  ra.k = k; ra.k_tok = static_cast<int64_t>(Hk) * kHeadDim; ra.k_head = kHeadDim;
  ra.v = v; ra.v_tok = static_cast<int64_t>(Hv) * kHeadDim; ra.v_head = kHeadDim;
  ra.g = g; ra.g_tok = Hv; ra.g_head = 1;
  ra.beta = beta; ra.b_tok = Hv; ra.b_head = 1;
  ra.o = o; ra.o_tok = static_cast<int64_t>(Hv) * kHeadDim; ra.o_head = kHeadDim;
  ra.state = state;
  ra.B = B; ra.T = T; ra.Hk = Hk; ra.Hv = Hv;
  ra.scale = scale > 0.f ? scale : 1.0f / sqrtf(static_cast<float>(kHeadDim));
  ra.l2norm = use_qk_l2norm ? 1 : 0;
  GDN_CUDA(recurrence_forward(ra, static_cast<cudaStream_t>(stream)));
  return GDN_OK;
}

extern "C" gdn_status gdn_gemm_bf16(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int32_t m,
                                    int32_t n, int32_t k, int32_t out_kind, void* out, int64_t ldo, int32_t ksplit,
                                    void* stream) {
  if (!a || !b || !out) return fail(GDN_ERR_NULL_POINTER, "gdn_gemm_bf16: null argument");
  if (m <= 0 || n <= 0 || k <= 0 || (k & 7) || lda < k || ldb < k)
    return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_gemm_bf16: bad shape m=%d n=%d k=%d lda=%lld ldb=%lld", m, n, k,
                static_cast<long long>(lda), static_cast<long long>(ldb));
  if (out_kind < 0 || out_kind > 3) return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_gemm_bf16: out_kind %d", out_kind);
  if (ksplit < 0 || ksplit > 8) return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_gemm_bf16: ksplit %d", ksplit);
  const bool transposed = out_kind >= 2;
  if (ldo < (transposed ? m : n)) return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_gemm_bf16: ldo too small");
  GemmEpiArgs ep;
  ep.out = out;
  ep.ld = ldo;
  GDN_CUDA(gemm_bf16_tn(a, lda, b, ldb, m, n, k, out_kind, ep, ksplit, static_cast<cudaStream_t>(stream)));
  return GDN_OK;
}

// ------------------------------------------------------------------------------------------------
// Communicator
// ------------------------------------------------------------------------------------------------
extern "C" gdn_status gdn_comm_get_unique_id(void* id_out, size_t id_bytes) {
  if (!id_out) return fail(GDN_ERR_NULL_POINTER, "gdn_comm_get_unique_id: null output");
  if (id_bytes < sizeof(ncclUniqueId)) return fail(GDN_ERR_INVALID_ARGUMENT, "id buffer needs %zu bytes", sizeof(ncclUniqueId));
  const NcclApi& api = nccl();
  if (!api.ok) return fail(GDN_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  ncclResult_t r = api.getUniqueId(&id);
  if (r != ncclSuccess) return fail(GDN_ERR_NCCL, "ncclGetUniqueId: %s", api.getErrorString(r));
  memcpy(id_out, &id, sizeof(id));
  return GDN_OK;
}

extern "C" gdn_status gdn_comm_create(const void* id, size_t id_bytes, int32_t rank, int32_t world, gdn_comm** out) {
  if (!id || !out) return fail(GDN_ERR_NULL_POINTER, "gdn_comm_create: null argument");
  *out = nullptr;
  if (id_bytes < sizeof(ncclUniqueId)) return fail(GDN_ERR_INVALID_ARGUMENT, "id needs %zu bytes", sizeof(ncclUniqueId));
  if (world <= 0 || rank < 0 || rank >= world) return fail(GDN_ERR_INVALID_ARGUMENT, "rank %d / world %d", rank, world);
  const NcclApi& api = nccl();
  if (!api.ok) return fail(GDN_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  gdn_comm* c = new (std::nothrow) gdn_comm();
  if (!c) return fail(GDN_ERR_OUT_OF_MEMORY, "host allocation failed");
  ncclResult_t r = api.commInitRank(&c->comm, world, uid, rank);
  if (r != ncclSuccess) {
    delete c;
    return fail(GDN_ERR_NCCL, "ncclCommInitRank: %s", api.getErrorString(r));
  }
  c->rank = rank;
  c->world = world;
  p2p_setup(c);
  *out = c;
  return GDN_OK;
}

extern "C" gdn_status gdn_comm_destroy(gdn_comm* c) {
  if (!c) return fail(GDN_ERR_NULL_POINTER, "gdn_comm_destroy: null communicator");
  const NcclApi& api = nccl();
  p2p_teardown(c);
  if (api.ok && c->comm) api.commDestroy(c->comm);
  delete c;
  return GDN_OK;
}

extern "C" gdn_status gdn_comm_allgather(gdn_comm* c, void* buf, size_t bytes_per_rank, void* stream) {
  if (!c || !buf) return fail(GDN_ERR_NULL_POINTER, "gdn_comm_allgather: null argument");
  if (bytes_per_rank == 0) return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_comm_allgather: zero bytes");
  const NcclApi& api = nccl();
  if (!api.ok) return fail(GDN_ERR_NCCL, "libnccl.so.2 could not be loaded");
  char* b = static_cast<char*>(buf);
  // in place: this rank's share already sits at its offset
  ncclResult_t r = api.allGather(b + static_cast<size_t>(c->rank) * bytes_per_rank, b, bytes_per_rank, ncclChar,
                                 c->comm, static_cast<cudaStream_t>(stream));
  if (r != ncclSuccess) return fail(GDN_ERR_NCCL, "ncclAllGather: %s", api.getErrorString(r));
  return GDN_OK;
}

// ------------------------------------------------------------------------------------------------
// Misc
// ------------------------------------------------------------------------------------------------
extern "C" gdn_status gdn_device_error(int32_t* code_out) {
  if (!code_out) return fail(GDN_ERR_NULL_POINTER, "gdn_device_error: null output");
  GDN_CUDA(cudaDeviceSynchronize());
  int v = 0;
  GDN_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  const int zero = 0;
  GDN_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  *code_out = v;
  if (v != 0) return fail(GDN_ERR_TIMEOUT, "device error word 0x%x (a bounded wait expired)", v);
  return GDN_OK;
}

extern "C" gdn_status gdn_selftest_peer_wait(const uint64_t* flag, uint64_t value, void* stream) {
  if (!flag) return fail(GDN_ERR_NULL_POINTER, "gdn_selftest_peer_wait: null flag");
  GDN_CUDA(peer_wait_selftest(reinterpret_cast<const unsigned long long*>(flag), value,
                              static_cast<cudaStream_t>(stream)));
  return GDN_OK;
}

extern "C" const char* gdn_last_error_string(void) { return t_last_error.c_str(); }

extern "C" uint64_t gdn_kernel_launch_count(void) { return launch_count(); }

extern "C" int32_t gdn_abi_version(void) { return GDN_ABI_VERSION; }
