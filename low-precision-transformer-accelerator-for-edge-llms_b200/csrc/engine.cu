// engine.cu -- host runtime behind include/tl_api.h.
//
// Replaces the FPGA control plane on the hot path:
//  * prefill_decode_controller.sv:39-198 -> tl_generate / tl_generate_batch:
//    bad-descriptor check, prefill, LM head, token emission, decode loop,
//    prefill-only launch (max_new_tokens == 0), decode-mode continuation.
//  * layer_controller.sv:25-195 -> enqueue_decode_step / enqueue_prefill:
//    the per-layer kernel sequence (norm+QKV, RoPE+KV append+attention,
//    O+residual, norm+gate/up+SiLU*up, down+residual), 22 layers, LM head.
//    The decode step is captured once per batch size into a CUDA graph and
//    replayed with all per-step state (token, position, stop flags) held on
//    the device.
//  * stop_condition_unit.sv:19-37 -> step_finalize kernel (EOS, max tokens)
//    plus the host abort flag sampled between graph replays.
// Device memory layout:
//  * weight arena: per layer W^T int8 [out][in] for QKV (fused rows q|k|v),
//    O, gate/up (interleaved rows gate_j, up_j), down; float64 per-channel
//    scales; float32 norm gains; float32 embedding [V][D]; LM head W^T [V][D].
//  * KV cache: int8 [slot][layer][kv_head][max_pos][64] for K and for V
//    (kv_cache_manager.sv:43-47 layout per slot), float32 scales
//    [slot][layer][kv_head].
// Tensor-parallel prefill (tl_tp_create): rank r of `world` holds kv heads
// [r Hkv/world, (r+1) Hkv/world) with their query heads, the matching
// columns of Q/K/V and the matching columns of gate/up; O, down, RMSNorm,
// embedding and LM head are replicated. The per-sequence activation maxima
// that set the O and down input scales are combined with an NCCL all-reduce
// max; each rank then quantizes its column block of the attention output
// (SiLU*up) with that scale and writes the INT8 bytes into the full-width
// input matrix of every rank -- its own and its peers', through CUDA-IPC
// mapped memory over NVLink -- and the O (down) GEMM runs on the whole
// input everywhere. Every rank thus computes exactly the one-GPU O / down
// products: the result is bit-identical, and the exchange moves INT8
// activations (1 byte per element, once) instead of INT32 partial sums.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tl_api.h"
#include "kernels.cuh"

using namespace tl;

namespace {

thread_local std::string g_last_error;

#define TL_CU(call)                                                                     \
  do {                                                                                  \
    cudaError_t _e = (call);                                                            \
    if (_e != cudaSuccess) {                                                            \
      g_last_error = std::string(#call) + ": " + cudaGetErrorString(_e);                \
      return TL_ERR_CUDA;                                                               \
    }                                                                                   \
  } while (0)

#define TL_TRY(call)                      \
  do {                                    \
    tl_status _s = (call);                \
    if (_s != TL_OK) return _s;           \
  } while (0)

template <typename T>
tl_status dmalloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) return TL_OK;
  TL_CU(cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)));
  return TL_OK;
}

struct Layer {
  int8_t* wqkv = nullptr;
  double* sqkv = nullptr;
  int8_t* wo = nullptr;
  double* so = nullptr;
  int8_t* wgu = nullptr;
  double* sgu = nullptr;
  int8_t* wd = nullptr;
  double* sd = nullptr;
  float* g1 = nullptr;
  float* g2 = nullptr;
};

struct DecodeBufs {
  int rows = 0;
  float *x = nullptr, *qkv = nullptr, *att = nullptr, *hid = nullptr;
  int *tokens = nullptr, *pos = nullptr, *slots = nullptr, *active = nullptr;
  int *count = nullptr, *stop = nullptr, *out_ids = nullptr, *run = nullptr;
  int32_t* argmax = nullptr;
  unsigned long long* am_partial = nullptr;
  unsigned long long* am_key = nullptr;  // [B] fused LM-head argmax keys (zero between steps)
  unsigned int* am_counter = nullptr;
  float* logits = nullptr;  // [rows][V]
  int8_t* xq = nullptr;     // [rows][max(D, F)] int8 activations (tensor-core path)
  int8_t* xq_lm = nullptr;  // [rows][D] the LM head's int8 input, written by every row group
  float* amax = nullptr;    // [rows] per-row absmax of the activation in xq
  // [rows] per-row max |x| folded in by the producer's epilogue (attention
  // output, SiLU*up) with atomics; zeroed by the RMSNorm kernel before it
  float* amax_prod = nullptr;
  float* attn_part = nullptr;         // decode attention split partials
  unsigned int* attn_cnt = nullptr;   // [rows][Hkv] merge tickets
  // persistent single-sequence step (decode1.cu)
  D1Layer* d1_layers = nullptr;       // device copy of the layer pointers
  float* d1_part = nullptr;
  unsigned int* d1_sync = nullptr;
};

// Batches of at least this many rows use the tcgen05 GEMM; smaller ones the
// dp4a GEMV with the fused RMSNorm/quantize prologue.
constexpr int kTcMinRows = 16;

struct PrefillBufs {
  size_t rows = 0;
  int n_seq_cap = 0;
  int* ids = nullptr;
  float *x = nullptr, *h = nullptr, *qkv = nullptr, *att = nullptr, *hid = nullptr;
  float* inv = nullptr;       // [rows] per-row 1/rms of the two-pass prefill norm
  int8_t* xq = nullptr;
  float* amax = nullptr;     // [L][4][n_seq] + [n_seq] (final norm)
  float* kvamax = nullptr;   // [L][n_seq][2][Hkv]
  // this layer's K / V as fp16 rows [(seq * Hkv + h) * S + t][64] (the INT8
  // cache values, exact): the attention's TMA operand rows
  uint16_t *kh = nullptr, *vh = nullptr;
};

// NCCL entry points, resolved at run time from libnccl.so.2 (the copy a host
// framework already loaded, if any), so the library has no link-time NCCL
// dependency and single-GPU use never touches it.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};
const NcclApi& nccl_api() {
  static const NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return a;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.all_gather && a.comm_destroy && a.error_string;
    return a;
  }();
  return api;
}

#define TL_NCCL(call)                                                                    \
  do {                                                                                   \
    const ncclResult_t _r = (call);                                                      \
    if (_r != ncclSuccess) {                                                             \
      g_last_error = std::string(#call) + ": " + nccl_api().error_string(_r);            \
      return TL_ERR_NCCL;                                                                \
    }                                                                                    \
  } while (0)

}  // namespace

struct tl_engine {
  tl_config cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  // The batched decode step runs its rows as independent groups, group i > 0
  // on side[i - 1] (parallel branches of the step graph). Every kernel of the
  // step is latency-bound at 64 rows, so two groups of 32 rows in lockstep
  // keep twice the CTAs in flight, and the second group's weight tiles
  // mostly come from L2 behind the first's (1.047 vs 1.124 ms per 64-row
  // step; 3 and 4 groups: 1.161 and 1.336 ms; group 1 started one to seven
  // kernels behind group 0: 1.07-1.11 ms). TL_DECODE_GROUPS=n overrides.
  static constexpr int kMaxGroups = 4;
  cudaStream_t side[kMaxGroups - 1] = {};
  cudaEvent_t ev_fork = nullptr, ev_join[kMaxGroups - 1] = {};
  int decode_groups = 2;
  // Batched decode steps of at least this many rows run on the tcgen05 GEMMs,
  // which stream every weight once per step whatever the row count below a
  // 32-token tile; batch 1 runs decode1_kernel (or, without it, the dp4a
  // GEMV path). Measured on B200 at context 512..1023, per step on the GEMV
  // path / on the tensor cores: 2 rows 1.397 / 0.941 ms, 4 rows 2.046 /
  // 0.927 ms, 8 rows 3.34 / 0.913 ms. TL_DECODE_TC_MIN_ROWS=n overrides
  // (2..16; 16 keeps every batch below 16 rows on the GEMV path).
  int decode_tc_min_rows = 2;
  int D = 0, F = 0, H = 0, Hkv = 0, Dq = 0, Dkv = 0, Nqkv = 0, V = 0, L = 0, P = 0, B = 0;
  std::vector<Layer> layers;
  float *embed = nullptr, *gfinal = nullptr, *cosT = nullptr, *sinT = nullptr;
  int8_t* wlm = nullptr;
  double* slm = nullptr;
  bool loaded = false;
  int8_t *kc = nullptr, *vc = nullptr;
  float *ks = nullptr, *vs = nullptr;
  DecodeBufs dec;
  PrefillBufs pf;
  std::map<int, cudaGraphExec_t> graphs;
  std::atomic<int> abort_req{0};
  std::vector<int> slot_pos;       // host mirror: tokens held per slot
  std::vector<int> slot_pending;   // emitted token not yet fed (-1 = none)
  int* h_pinned = nullptr;         // pinned staging
  size_t h_pinned_ints = 0;
  bool use_pdl = true;
  // tensor parallelism (prefill only): H, Hkv, Dq, Dkv, Nqkv and F above are
  // this rank's shares; cfg keeps the model's global sizes
  int tp_rank = 0, tp_world = 1;
  int Dq_full = 0, F_full = 0;      // the model's O / down input widths
  // O / down input widths this rank holds: the full widths when O and down
  // are replicated (single GPU, TL_TP_ALLGATHER), this rank's row blocks
  // Dq / F when they are row-split (TL_TP_ALLREDUCE)
  int Dq_in = 0, F_in = 0;
  int tp_exchange = TL_TP_ALLREDUCE;
  int32_t* tp_acc = nullptr;        // [tp_rows][D] partial INT32 accumulators (TL_TP_ALLREDUCE)
  ncclComm_t comm = nullptr;
  // INT8 exchange buffers of the tensor-parallel prefill: two [tp_rows][max(Dq_full, F_full)]
  // matrices (exchange k uses k % 2) and `world` flag words per rank, in one
  // allocation mapped by every peer (tp_peer[q]: rank q's base; tp_peer[rank] = tp_base)
  unsigned char* tp_base = nullptr;
  unsigned char* tp_peer[4] = {nullptr, nullptr, nullptr, nullptr};
  unsigned int* tp_done = nullptr;  // CTA ticket of the scatter kernel
  size_t tp_rows = 0, tp_buf_bytes = 0;
  unsigned int tp_epoch = 0;
  bool use_decode1 = false;         // batch-1 steps run as one persistent kernel
  float* logits_all = nullptr;      // [logits_all_rows][V]: tl_forward_logits
  size_t logits_all_rows = 0;
};

namespace {

tl_status check_cfg(const tl_config* c) {
  if (!c) return TL_ERR_INVALID_ARGUMENT;
  if (c->head_dim != 64) return TL_ERR_INVALID_ARGUMENT;
  if (c->num_heads <= 0 || c->num_kv_heads <= 0 || c->num_heads % c->num_kv_heads) return TL_ERR_INVALID_ARGUMENT;
  const int G = c->num_heads / c->num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return TL_ERR_INVALID_ARGUMENT;
  if (c->hidden_size % 64 || c->intermediate_size % 16 || c->hidden_size != c->num_heads * 64)
    return TL_ERR_INVALID_ARGUMENT;
  if (c->num_layers <= 0 || c->vocab_size <= 0 || c->max_positions <= 0 || c->max_batch <= 0)
    return TL_ERR_INVALID_ARGUMENT;
  NormPlan plan;
  if (!norm_plan(c->hidden_size, &plan)) return TL_ERR_INVALID_ARGUMENT;  // RMSNorm reduction tree
  return TL_OK;
}

// The pinned staging buffer is written by the host and read by async copies
// on the engine stream; every user waits for the stream first so no earlier
// copy can still be reading it.
tl_status ensure_pinned(tl_engine* e, size_t ints) {
  TL_CU(cudaStreamSynchronize(e->stream));
  if (e->h_pinned_ints >= ints) return TL_OK;
  if (e->h_pinned) cudaFreeHost(e->h_pinned);
  e->h_pinned = nullptr;
  TL_CU(cudaMallocHost(reinterpret_cast<void**>(&e->h_pinned), ints * sizeof(int)));
  e->h_pinned_ints = ints;
  return TL_OK;
}

tl_status alloc_decode(tl_engine* e) {
  DecodeBufs& d = e->dec;
  const int B = e->B;
  d.rows = B;
  TL_TRY(dmalloc(&d.x, static_cast<size_t>(B) * e->D));
  TL_TRY(dmalloc(&d.qkv, static_cast<size_t>(B) * e->Nqkv));
  TL_TRY(dmalloc(&d.att, static_cast<size_t>(B) * e->Dq));
  TL_TRY(dmalloc(&d.hid, static_cast<size_t>(B) * e->F));
  TL_TRY(dmalloc(&d.tokens, B));
  TL_TRY(dmalloc(&d.pos, B));
  TL_TRY(dmalloc(&d.slots, B));
  TL_TRY(dmalloc(&d.active, B));
  TL_TRY(dmalloc(&d.count, B));
  TL_TRY(dmalloc(&d.stop, B));
  TL_TRY(dmalloc(&d.out_ids, static_cast<size_t>(B) * e->P));
  TL_TRY(dmalloc(&d.run, 4));
  TL_TRY(dmalloc(&d.argmax, B));
  TL_TRY(dmalloc(&d.am_key, B));
  TL_CU(cudaMemset(d.am_key, 0, B * sizeof(unsigned long long)));
  TL_TRY(dmalloc(&d.am_partial, gemv_argmax_partials(B, e->V)));
  TL_TRY(dmalloc(&d.am_counter, gemv_argmax_row_blocks(B) + 1));
  TL_TRY(dmalloc(&d.logits, static_cast<size_t>(B) * e->V));
  TL_TRY(dmalloc(&d.xq, static_cast<size_t>(B) * std::max(e->D, e->F)));
  TL_TRY(dmalloc(&d.xq_lm, static_cast<size_t>(B) * e->D));
  TL_TRY(dmalloc(&d.amax, B));
  TL_TRY(dmalloc(&d.amax_prod, B));
  TL_TRY(dmalloc(&d.attn_part, tl_engine::kMaxGroups * attn_part_floats(B, e->Hkv, e->P)));  // a region per row group
  TL_TRY(dmalloc(&d.attn_cnt, static_cast<size_t>(B) * e->Hkv));
  TL_CU(cudaMemset(d.attn_cnt, 0, static_cast<size_t>(B) * e->Hkv * sizeof(unsigned int)));
  if (e->use_decode1) {
    TL_TRY(dmalloc(&d.d1_layers, e->L));
    TL_TRY(dmalloc(&d.d1_part, decode1_part_floats(e->Hkv, e->P)));
    TL_TRY(dmalloc(&d.d1_sync, decode1_sync_words(e->L, e->Hkv)));  // barrier counter + attention tickets
    std::vector<D1Layer> h(e->L);
    for (int l = 0; l < e->L; ++l) {
      const Layer& ly = e->layers[l];
      h[l] = {ly.wqkv, ly.sqkv, ly.wo, ly.so, ly.wgu, ly.sgu, ly.wd, ly.sd, ly.g1, ly.g2};
    }
    TL_CU(cudaMemcpy(d.d1_layers, h.data(), h.size() * sizeof(D1Layer), cudaMemcpyHostToDevice));
  }
  TL_CU(cudaMemset(d.am_counter, 0, (gemv_argmax_row_blocks(B) + 1) * sizeof(unsigned int)));
  TL_CU(cudaMemset(d.active, 0, B * sizeof(int)));
  TL_CU(cudaMemset(d.stop, 0, B * sizeof(int)));
  TL_CU(cudaMemset(d.pos, 0, B * sizeof(int)));
  std::vector<int> slots(B);
  for (int i = 0; i < B; ++i) slots[i] = i;
  TL_CU(cudaMemcpy(d.slots, slots.data(), B * sizeof(int), cudaMemcpyHostToDevice));
  return TL_OK;
}

tl_status ensure_prefill(tl_engine* e, size_t rows, int n_seq) {
  PrefillBufs& p = e->pf;
  if (p.rows >= rows && p.n_seq_cap >= n_seq) return TL_OK;
  rows = std::max(rows, p.rows);
  n_seq = std::max(n_seq, p.n_seq_cap);
  cudaFree(p.ids); cudaFree(p.x); cudaFree(p.h); cudaFree(p.qkv); cudaFree(p.att);
  cudaFree(p.hid); cudaFree(p.xq); cudaFree(p.amax); cudaFree(p.kvamax); cudaFree(p.inv);
  cudaFree(p.kh); cudaFree(p.vh);
  p = PrefillBufs{};
  TL_TRY(dmalloc(&p.ids, rows));
  TL_TRY(dmalloc(&p.x, rows * e->D));
  TL_TRY(dmalloc(&p.h, rows * e->D));
  TL_TRY(dmalloc(&p.inv, rows));
  TL_TRY(dmalloc(&p.qkv, rows * e->Nqkv));
  TL_TRY(dmalloc(&p.att, rows * e->Dq));
  TL_TRY(dmalloc(&p.hid, rows * e->F));
  TL_TRY(dmalloc(&p.xq, rows * std::max(e->F, e->D)));
  TL_TRY(dmalloc(&p.amax, static_cast<size_t>(e->L) * 4 * n_seq + n_seq));
  TL_TRY(dmalloc(&p.kvamax, static_cast<size_t>(e->L) * n_seq * 2 * e->Hkv));
  TL_TRY(dmalloc(&p.kh, rows * e->Dkv));
  TL_TRY(dmalloc(&p.vh, rows * e->Dkv));
  p.rows = rows;
  p.n_seq_cap = n_seq;
  return TL_OK;
}

void invalidate_graphs(tl_engine* e) {
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
  e->graphs.clear();
}

// One tcgen05 GEMM: out = epi(X[M][K] . W^T[N][K]); plan (tensor maps, tile,
// split-K) made on the host, so this is also safe inside stream capture.
tl_status tc_gemm(tl_engine* e, const int8_t* w, int N, const int8_t* x, int M, int K, const TcArgs& args,
                  bool pdl, cudaStream_t s = nullptr) {
  TcPlan p;
  TL_CU(tc_make_plan(&p, w, N, x, M, K, device_sm_count(), args.epi));
  TL_CU(launch_gemm_tc(p, args, s ? s : e->stream, pdl));
  return TL_OK;
}

// Optional per-layer capture (tl_decoder_layer, tl_decode_layer): host destinations plus the
// device scratch the extra INT32 / float projections write into. The capture
// re-runs a projection with the raw INT32 (or float) epilogue on the same INT8
// operands; integer MMAs are exact, so these are the accumulators the fused
// epilogues consumed.
struct LayerCap {
  const tl_layer_capture* h = nullptr;
  int32_t* i32 = nullptr;      // [R][max(Nqkv, 2F, D)]
  float* f32 = nullptr;        // [R][2F]
  float* scores = nullptr;     // [H][S][S] (when h->scores or h->probs)
  float* probs = nullptr;
  std::vector<int32_t> tmp_i;  // host staging for the interleaved gate/up rows
  std::vector<float> tmp_f;
};

tl_status d2h(tl_engine* e, void* dst, const void* src, size_t bytes) {
  if (!dst || !bytes) return TL_OK;
  TL_CU(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, e->stream));
  return TL_OK;
}
// columns [c0, c0 + w) of a device matrix [rows][ld] of 4-byte elements
tl_status d2h_cols(tl_engine* e, void* dst, const void* src, int rows, int ld, int c0, int w) {
  if (!dst) return TL_OK;
  TL_CU(cudaMemcpy2DAsync(dst, static_cast<size_t>(w) * 4, static_cast<const char*>(src) + static_cast<size_t>(c0) * 4,
                          static_cast<size_t>(ld) * 4, static_cast<size_t>(w) * 4, rows, cudaMemcpyDeviceToHost,
                          e->stream));
  return TL_OK;
}

// Raw INT32 (EPI_I32) or dequantized (EPI_F32) product of an INT8 input
// already in xq, for the capture.
tl_status capture_gemm(tl_engine* e, const int8_t* xq, const int8_t* w, const double* ws, int N, int K, int R, int S,
                       const float* in_absmax, int epi, void* out) {
  if (R >= kTcMinRows) {
    TcPlan plan;
    TL_CU(tc_make_plan(&plan, w, N, xq, R, K, device_sm_count(), epi));
    TcArgs a;
    a.epi = epi; a.w_scale = ws; a.in_absmax = in_absmax; a.rows_per_group = S;
    if (epi == EPI_I32) a.out_i32 = static_cast<int32_t*>(out);
    else a.out_f32 = static_cast<float*>(out);
    TL_CU(launch_gemm_tc(plan, a, e->stream, false));
    return TL_OK;
  }
  GemvArgs g;
  g.x_q = xq; g.in_absmax = in_absmax; g.rows_per_group = S;
  g.w = w; g.w_scale = ws; g.M = R; g.N = N; g.K = K;
  if (epi == EPI_I32) g.out_i32 = static_cast<int32_t*>(out);
  else g.out_f32 = static_cast<float*>(out);
  TL_CU(launch_gemv(PRO_Q8, epi, g, e->stream, false));
  return TL_OK;
}

// interleaved rows [R][2F] (column 2j = gate j, 2j+1 = up j) -> two host [R][F]
template <typename T>
tl_status split_gate_up(tl_engine* e, const T* dev, int R, int F, std::vector<T>& tmp, T* gate, T* up) {
  if (!gate && !up) return TL_OK;
  tmp.resize(static_cast<size_t>(R) * 2 * F);
  TL_CU(cudaMemcpyAsync(tmp.data(), dev, tmp.size() * sizeof(T), cudaMemcpyDeviceToHost, e->stream));
  TL_CU(cudaStreamSynchronize(e->stream));
  for (size_t r = 0; r < static_cast<size_t>(R); ++r)
    for (size_t j = 0; j < static_cast<size_t>(F); ++j) {
      if (gate) gate[r * F + j] = tmp[(r * F + j) * 2];
      if (up) up[r * F + j] = tmp[(r * F + j) * 2 + 1];
    }
  return TL_OK;
}

// Rows [r0, r0 + M) of the batched decode step, enqueued on stream `s`; the
// per-row buffers are addressed from row r0, the attention split partials
// live in the group's own region `attn_part`, and the attention split count
// is sized for `split_rows` rows (the whole step, when groups run
// concurrently). `pdl_entry` = false launches the group's first kernel
// without programmatic serialization (it follows an event, not a kernel).
struct RowGroup {
  int r0 = 0, M = 0;
  cudaStream_t s = nullptr;
  float* attn_part = nullptr;
  int split_rows = 0;
  bool pdl_entry = true;
};

// Layer l of the batched decode step on the tensor cores (M >=
// decode_tc_min_rows rows): per row RMSNorm + INT8 quantization kernels feed
// tcgen05 GEMMs whose epilogues dequantize, add the residual or apply
// SiLU*up. The attention kernel and the SiLU*up epilogue fold each row's max
// |output| into
// d.amax_prod with atomics, so the quantization of their outputs is
// elementwise over the whole block; each RMSNorm kernel re-arms d.amax_prod
// (its last reader, the GEMM two kernels back, has completed by then).
// `cap` (tl_decode_layer) copies the intermediate tensors of the M rows out
// as they are produced; it is never set inside stream capture.
tl_status enqueue_decode_layer_tc(tl_engine* e, int l, const RowGroup& g, LayerCap* cap) {
  DecodeBufs& d = e->dec;
  cudaStream_t s = g.s;
  const int M = g.M;
  const size_t r0 = static_cast<size_t>(g.r0);
  const bool pdl = e->use_pdl && !cap;
  const float eps = e->cfg.rms_norm_eps;
  const tl_layer_capture* hc = cap ? cap->h : nullptr;
  const size_t rowsD = static_cast<size_t>(M) * e->D * sizeof(float);
  const Layer& ly = e->layers[l];
  float* x = d.x + r0 * e->D;
  float* qkv = d.qkv + r0 * e->Nqkv;
  float* att = d.att + r0 * e->Dq;
  float* hid = d.hid + r0 * e->F;
  int8_t* xq = d.xq + r0 * std::max(e->D, e->F);
  float* amax = d.amax + r0;
  float* amax_prod = d.amax_prod + r0;
  if (hc && hc->attn_input) {
    TL_CU(launch_rmsnorm_rows(x, ly.g1, eps, cap->f32, nullptr, M, e->D, 1, s));
    TL_TRY(d2h(e, hc->attn_input, cap->f32, rowsD));
  }
  TL_CU(launch_norm_quant_rows(x, ly.g1, eps, M, e->D, xq, amax, s, pdl && (l > 0 || g.pdl_entry), amax_prod));
  TcArgs q;
  q.epi = EPI_F32; q.w_scale = ly.sqkv; q.in_absmax = amax; q.rows_per_group = 1; q.out_f32 = qkv;
  TL_TRY(tc_gemm(e, ly.wqkv, e->Nqkv, xq, M, e->D, q, pdl, s));
  if (hc) {
    TL_TRY(d2h(e, hc->qkv_input_q, xq, static_cast<size_t>(M) * e->D));
    TL_TRY(d2h(e, hc->qkv_input_absmax, amax, M * sizeof(float)));
    TL_TRY(d2h_cols(e, hc->q_proj, qkv, M, e->Nqkv, 0, e->Dq));
    TL_TRY(d2h_cols(e, hc->k_proj, qkv, M, e->Nqkv, e->Dq, e->Dkv));
    TL_TRY(d2h_cols(e, hc->v_proj, qkv, M, e->Nqkv, e->Dq + e->Dkv, e->Dkv));
    if (hc->q_acc || hc->k_acc || hc->v_acc) {
      TL_TRY(capture_gemm(e, xq, ly.wqkv, ly.sqkv, e->Nqkv, e->D, M, 1, amax, EPI_I32, cap->i32));
      TL_TRY(d2h_cols(e, hc->q_acc, cap->i32, M, e->Nqkv, 0, e->Dq));
      TL_TRY(d2h_cols(e, hc->k_acc, cap->i32, M, e->Nqkv, e->Dq, e->Dkv));
      TL_TRY(d2h_cols(e, hc->v_acc, cap->i32, M, e->Nqkv, e->Dq + e->Dkv, e->Dkv));
    }
  }
  AttnDecodeArgs at;
  at.qkv = qkv; at.ld = e->Nqkv; at.pos = d.pos + r0; at.slot = d.slots + r0; at.active = d.active + r0;
  at.kc = e->kc; at.vc = e->vc; at.ks = e->ks; at.vs = e->vs;
  at.layer = l; at.L = e->L; at.H = e->H; at.Hkv = e->Hkv; at.P = e->P; at.M = M;
  at.cos = e->cosT; at.sin = e->sinT; at.out = att;
  at.part = g.attn_part; at.counters = d.attn_cnt + r0 * e->Hkv; at.out_absmax = amax_prod;
  at.split_rows = g.split_rows;
  TL_CU(launch_attn_decode(at, s, pdl));
  TL_CU(launch_quant_known_rows(att, amax_prod, M, e->Dq, xq, s, pdl));
  if (hc) {
    TL_TRY(d2h(e, hc->attended, att, static_cast<size_t>(M) * e->Dq * sizeof(float)));
    TL_TRY(d2h(e, hc->o_input_q, xq, static_cast<size_t>(M) * e->Dq));
    TL_TRY(d2h(e, hc->o_input_absmax, amax_prod, M * sizeof(float)));
    if (hc->o_acc) {
      TL_TRY(capture_gemm(e, xq, ly.wo, ly.so, e->D, e->Dq, M, 1, amax_prod, EPI_I32, cap->i32));
      TL_TRY(d2h(e, hc->o_acc, cap->i32, static_cast<size_t>(M) * e->D * 4));
    }
    if (hc->o_proj) {
      TL_TRY(capture_gemm(e, xq, ly.wo, ly.so, e->D, e->Dq, M, 1, amax_prod, EPI_F32, cap->i32));
      TL_TRY(d2h(e, hc->o_proj, cap->i32, static_cast<size_t>(M) * e->D * 4));
    }
  }
  TcArgs o;
  o.epi = EPI_RESID; o.w_scale = ly.so; o.in_absmax = amax_prod; o.rows_per_group = 1; o.out_f32 = x;
  o.resid = x;
  TL_TRY(tc_gemm(e, ly.wo, e->D, xq, M, e->Dq, o, pdl, s));
  if (hc) TL_TRY(d2h(e, hc->x_after_attn, x, rowsD));
  if (hc && hc->ffn_input) {
    TL_CU(launch_rmsnorm_rows(x, ly.g2, eps, cap->f32, nullptr, M, e->D, 1, s));
    TL_TRY(d2h(e, hc->ffn_input, cap->f32, rowsD));
  }
  TL_CU(launch_norm_quant_rows(x, ly.g2, eps, M, e->D, xq, amax, s, pdl, amax_prod));
  TcArgs gu;
  gu.epi = EPI_SILU; gu.w_scale = ly.sgu; gu.in_absmax = amax; gu.rows_per_group = 1; gu.out_f32 = hid;
  gu.out_absmax = amax_prod;
  TL_TRY(tc_gemm(e, ly.wgu, 2 * e->F, xq, M, e->D, gu, pdl, s));
  if (hc) {
    TL_TRY(d2h(e, hc->gate_up_input_q, xq, static_cast<size_t>(M) * e->D));
    TL_TRY(d2h(e, hc->gate_up_input_absmax, amax, M * sizeof(float)));
    if (hc->gate_acc || hc->up_acc) {
      TL_TRY(capture_gemm(e, xq, ly.wgu, ly.sgu, 2 * e->F, e->D, M, 1, amax, EPI_I32, cap->i32));
      TL_TRY(split_gate_up(e, cap->i32, M, e->F, cap->tmp_i, hc->gate_acc, hc->up_acc));
    }
    if (hc->gate_proj || hc->up_proj) {
      TL_TRY(capture_gemm(e, xq, ly.wgu, ly.sgu, 2 * e->F, e->D, M, 1, amax, EPI_F32, cap->f32));
      TL_TRY(split_gate_up(e, static_cast<const float*>(cap->f32), M, e->F, cap->tmp_f, hc->gate_proj,
                           hc->up_proj));
    }
  }
  TL_CU(launch_quant_known_rows(hid, amax_prod, M, e->F, xq, s, pdl));
  if (hc) {
    TL_TRY(d2h(e, hc->hidden, hid, static_cast<size_t>(M) * e->F * sizeof(float)));
    TL_TRY(d2h(e, hc->down_input_q, xq, static_cast<size_t>(M) * e->F));
    TL_TRY(d2h(e, hc->down_input_absmax, amax_prod, M * sizeof(float)));
    if (hc->down_acc) {
      TL_TRY(capture_gemm(e, xq, ly.wd, ly.sd, e->D, e->F, M, 1, amax_prod, EPI_I32, cap->i32));
      TL_TRY(d2h(e, hc->down_acc, cap->i32, static_cast<size_t>(M) * e->D * 4));
    }
    if (hc->down_proj) {
      TL_TRY(capture_gemm(e, xq, ly.wd, ly.sd, e->D, e->F, M, 1, amax_prod, EPI_F32, cap->i32));
      TL_TRY(d2h(e, hc->down_proj, cap->i32, static_cast<size_t>(M) * e->D * 4));
    }
  }
  TcArgs dn;
  dn.epi = EPI_RESID; dn.w_scale = ly.sd; dn.in_absmax = amax_prod; dn.rows_per_group = 1; dn.out_f32 = x;
  dn.resid = x;
  TL_TRY(tc_gemm(e, ly.wd, e->D, xq, M, e->F, dn, pdl, s));
  return TL_OK;
}

// Row groups of a batched decode step of M rows: up to decode_groups
// concurrent groups of about equal size, each of at least kMinGroupRows rows
// (one group on the engine stream when M is smaller). Smaller groups leave
// the 32-token GEMM tiles half empty: at 32 rows one group measured 0.989 ms
// per step against 1.036 ms for two of 16; at 48 rows two groups of 24
// measured 1.009 against 1.088 ms for one.
constexpr int kMinGroupRows = 24;
int decode_row_groups(const tl_engine* e, int M, RowGroup* g) {
  const size_t region = attn_part_floats(e->B, e->Hkv, e->P);
  const int ng = std::max(1, std::min(e->decode_groups, M / kMinGroupRows));
  int r = 0;
  for (int i = 0; i < ng; ++i) {
    const int rows = (M - r) / (ng - i);
    g[i].r0 = r; g[i].M = rows; g[i].s = i == 0 ? e->stream : e->side[i - 1];
    g[i].attn_part = e->dec.attn_part + i * region; g[i].split_rows = M; g[i].pdl_entry = i == 0;
    r += rows;
  }
  return ng;
}

// Batched decode step on the tensor cores (M >= decode_tc_min_rows): embedding
// on the engine stream, then each row group's layers and final RMSNorm on its
// own stream, joined before one LM head (fused argmax) over all rows and the
// finalize (one 64-row LM head launch: 250 CTAs, against 2 x 250 for two
// 32-row ones).
tl_status enqueue_decode_step_tc(tl_engine* e, int M, bool finalize) {
  DecodeBufs& d = e->dec;
  cudaStream_t s = e->stream;
  const bool pdl = e->use_pdl;
  const float eps = e->cfg.rms_norm_eps;
  TL_CU(launch_embed(e->embed, d.tokens, d.x, M, e->D, e->V, s, pdl));
  RowGroup grp[tl_engine::kMaxGroups];
  const int ng = decode_row_groups(e, M, grp);
  if (ng > 1) {
    TL_CU(cudaEventRecord(e->ev_fork, s));
    for (int i = 1; i < ng; ++i) TL_CU(cudaStreamWaitEvent(grp[i].s, e->ev_fork, 0));
  }
  for (int l = 0; l < e->L; ++l)
    for (int i = 0; i < ng; ++i) TL_TRY(enqueue_decode_layer_tc(e, l, grp[i], nullptr));
  for (int i = 0; i < ng; ++i) {
    const RowGroup& g = grp[i];
    const size_t r0 = static_cast<size_t>(g.r0);
    TL_CU(launch_norm_quant_rows(d.x + r0 * e->D, e->gfinal, eps, g.M, e->D, d.xq_lm + r0 * e->D, d.amax + r0, g.s,
                                 pdl));
  }
  for (int i = 1; i < ng; ++i) {
    TL_CU(cudaEventRecord(e->ev_join[i - 1], grp[i].s));
    TL_CU(cudaStreamWaitEvent(s, e->ev_join[i - 1], 0));
  }
  // LM head with the greedy argmax fused into the epilogue (packed keys in
  // d.am_key, consumed and re-armed by step_finalize / keys_to_tokens); the
  // logits themselves are not written. After the join its predecessor is an
  // event, so it launches without programmatic serialization.
  TcArgs lm;
  lm.epi = EPI_F32; lm.w_scale = e->slm; lm.in_absmax = d.amax; lm.rows_per_group = 1; lm.out_f32 = nullptr;
  lm.am_key = d.am_key;
  TL_TRY(tc_gemm(e, e->wlm, e->V, d.xq_lm, M, e->D, lm, pdl && ng == 1, s));
  if (!finalize) TL_CU(launch_keys_to_tokens(d.am_key, d.argmax, M, s));
  if (finalize) {
    StepArgs st;
    st.M = M; st.am_key = d.am_key; st.tokens = d.tokens; st.pos = d.pos; st.active = d.active;
    st.count = d.count; st.stop = d.stop; st.out_ids = d.out_ids; st.out_stride = e->P;
    st.run = d.run; st.P = e->P;
    TL_CU(launch_step_finalize(st, s, pdl));
  }
  return TL_OK;
}

// ------------------------------------------------------------- decode step
// One decode step for rows 0..M-1 (row m uses KV slot dec.slots[m]). All
// inputs (token, position, active) come from device memory, so the sequence
// is graph-capturable.
// The batch-1 step as one persistent kernel (decode1.cu) plus finalize.
tl_status enqueue_decode_step_d1(tl_engine* e, bool finalize) {
  DecodeBufs& d = e->dec;
  cudaStream_t s = e->stream;
  D1Args a;
  a.layers = d.d1_layers; a.L = e->L; a.D = e->D; a.F = e->F; a.H = e->H; a.Hkv = e->Hkv; a.V = e->V;
  a.P = e->P; a.Nqkv = e->Nqkv; a.Dq = e->Dq; a.eps = e->cfg.rms_norm_eps;
  if (!norm_plan(e->D, &a.plan)) return TL_ERR_INVALID_ARGUMENT;
  a.embed = e->embed; a.gfinal = e->gfinal; a.wlm = e->wlm; a.slm = e->slm;
  a.kc = e->kc; a.vc = e->vc; a.ks = e->ks; a.vs = e->vs; a.cos = e->cosT; a.sin = e->sinT;
  a.x = d.x; a.qkv = d.qkv; a.att = d.att; a.hid = d.hid;
  a.token = d.tokens; a.pos = d.pos; a.slot = d.slots; a.active = d.active;
  a.part = d.d1_part; a.sync = d.d1_sync; a.am_key = d.am_key;
  TL_CU(cudaMemsetAsync(d.d1_sync, 0, decode1_sync_words(e->L, e->Hkv) * sizeof(unsigned int), s));
  TL_CU(launch_decode1(a, device_sm_count(), s));
  if (finalize) {
    StepArgs st;
    st.M = 1; st.am_key = d.am_key; st.tokens = d.tokens; st.pos = d.pos; st.active = d.active;
    st.count = d.count; st.stop = d.stop; st.out_ids = d.out_ids; st.out_stride = e->P;
    st.run = d.run; st.P = e->P;
    TL_CU(launch_step_finalize(st, s, false));
  } else {
    TL_CU(launch_keys_to_tokens(d.am_key, d.argmax, 1, s));
  }
  return TL_OK;
}

// Step-scoped debug capture (tl_decode_debug): the fixed tensor set of the
// hardware's debug contract for one layer of a batch-1 decode step, taken by
// extra copies and by kernels that apply the same rules to the same inputs
// (the GEMV's fused RMSNorm/quantize prologue does not materialize its INT8
// row, so it is recomputed by the row kernel with the identical rule).
struct DebugCap {
  tl_debug_record* h = nullptr;
  int layer = 0, slot = 0, pos = 0;
  float* f32 = nullptr;     // [max(D, F)] scratch
  int8_t* i8 = nullptr;     // [max(D, F)]
  float* am = nullptr;      // [5] input absmax: qkv, o, gate/up, down, LM head
  float* sc = nullptr;      // [H][pos + 1]
  float* pr = nullptr;
};

// Layer l of the per-kernel decode step for rows 0..M-1 (M <
// decode_tc_min_rows, batch 1 without decode1_kernel, or teacher-forced
// logits): dp4a GEMVs with the RMSNorm/quantize prologue and the dequant /
// residual / SiLU*up epilogues, decode attention in between.
tl_status enqueue_decode_layer_gemv(tl_engine* e, int l, int M, DebugCap* dbg) {
  DecodeBufs& d = e->dec;
  cudaStream_t s = e->stream;
  const bool pdl = e->use_pdl && !dbg;
  const Layer& ly = e->layers[l];
  const float eps = e->cfg.rms_norm_eps;
  tl_debug_record* h = dbg && dbg->layer == l ? dbg->h : nullptr;
  if (h) {
    TL_TRY(d2h(e, h->layer_input, d.x, e->D * sizeof(float)));
    TL_CU(launch_norm_quant_rows(d.x, ly.g1, eps, 1, e->D, dbg->i8, dbg->am, s, false));
    TL_TRY(d2h(e, h->qkv_input_q, dbg->i8, e->D));
  }
  GemvArgs q;
  q.x_f32 = d.x; q.gamma = ly.g1; q.eps = eps;
  q.w = ly.wqkv; q.w_scale = ly.sqkv; q.M = M; q.N = e->Nqkv; q.K = e->D; q.out_f32 = d.qkv;
  TL_CU(launch_gemv(PRO_NORM, EPI_F32, q, s, pdl));
  if (h) {
    TL_TRY(d2h(e, h->q_proj, d.qkv, e->Dq * sizeof(float)));
    TL_TRY(d2h(e, h->k_proj, d.qkv + e->Dq, e->Dkv * sizeof(float)));
    TL_TRY(d2h(e, h->v_proj, d.qkv + e->Dq + e->Dkv, e->Dkv * sizeof(float)));
  }
  AttnDecodeArgs at;
  at.qkv = d.qkv; at.ld = e->Nqkv; at.pos = d.pos; at.slot = d.slots; at.active = d.active;
  at.kc = e->kc; at.vc = e->vc; at.ks = e->ks; at.vs = e->vs;
  at.layer = l; at.L = e->L; at.H = e->H; at.Hkv = e->Hkv; at.P = e->P; at.M = M;
  at.cos = e->cosT; at.sin = e->sinT; at.out = d.att;
  at.part = d.attn_part; at.counters = d.attn_cnt;
  TL_CU(launch_attn_decode(at, s, pdl));
  if (h) {
    const size_t base = (static_cast<size_t>(dbg->slot) * e->L + l) * e->Hkv;
    const size_t row = static_cast<size_t>(dbg->pos) * 64;
    if (h->k_row)
      TL_CU(cudaMemcpy2DAsync(h->k_row, 64, e->kc + base * e->P * 64 + row, static_cast<size_t>(e->P) * 64, 64,
                              e->Hkv, cudaMemcpyDeviceToHost, s));
    if (h->v_row)
      TL_CU(cudaMemcpy2DAsync(h->v_row, 64, e->vc + base * e->P * 64 + row, static_cast<size_t>(e->P) * 64, 64,
                              e->Hkv, cudaMemcpyDeviceToHost, s));
    TL_TRY(d2h(e, h->k_scale, e->ks + base, e->Hkv * sizeof(float)));
    TL_TRY(d2h(e, h->v_scale, e->vs + base, e->Hkv * sizeof(float)));
    if (h->scores || h->probs) {
      TL_CU(launch_attn_scores_debug(d.qkv, e->Nqkv, 1, dbg->pos + 1, dbg->pos, true, e->H, e->Hkv, e->kc, e->ks,
                                     e->cosT, e->sinT, dbg->slot, l, e->L, e->P, dbg->sc, dbg->pr, s));
      const size_t wb = static_cast<size_t>(e->H) * (dbg->pos + 1) * sizeof(float);
      TL_TRY(d2h(e, h->scores, dbg->sc, wb));
      TL_TRY(d2h(e, h->probs, dbg->pr, wb));
    }
    TL_TRY(d2h(e, h->attended, d.att, e->Dq * sizeof(float)));
    TL_CU(launch_absmax_rows(d.att, 1, e->Dq, 1, dbg->am + 1, s));
  }
  GemvArgs o;
  o.x_f32 = d.att; o.w = ly.wo; o.w_scale = ly.so; o.M = M; o.N = e->D; o.K = e->Dq;
  o.out_f32 = d.x; o.resid = d.x;
  TL_CU(launch_gemv(PRO_F32, EPI_RESID, o, s, pdl));
  if (h) TL_CU(launch_norm_quant_rows(d.x, ly.g2, eps, 1, e->D, dbg->i8, dbg->am + 2, s, false));
  GemvArgs gu;
  gu.x_f32 = d.x; gu.gamma = ly.g2; gu.eps = eps;
  gu.w = ly.wgu; gu.w_scale = ly.sgu; gu.M = M; gu.N = 2 * e->F; gu.K = e->D; gu.out_f32 = d.hid;
  TL_CU(launch_gemv(PRO_NORM, EPI_SILU, gu, s, pdl));
  if (h) TL_CU(launch_absmax_rows(d.hid, 1, e->F, 1, dbg->am + 3, s));
  GemvArgs dn;
  dn.x_f32 = d.hid; dn.w = ly.wd; dn.w_scale = ly.sd; dn.M = M; dn.N = e->D; dn.K = e->F;
  dn.out_f32 = d.x; dn.resid = d.x;
  TL_CU(launch_gemv(PRO_F32, EPI_RESID, dn, s, pdl));
  if (h) TL_TRY(d2h(e, h->layer_output, d.x, e->D * sizeof(float)));
  return TL_OK;
}

tl_status enqueue_decode_step(tl_engine* e, int M, float* logits, bool finalize, DebugCap* dbg = nullptr) {
  if (M >= e->decode_tc_min_rows && !logits) return enqueue_decode_step_tc(e, M, finalize);
  if (M == 1 && !logits && e->use_decode1) return enqueue_decode_step_d1(e, finalize);
  DecodeBufs& d = e->dec;
  cudaStream_t s = e->stream;
  const bool pdl = e->use_pdl && !dbg;
  TL_CU(launch_embed(e->embed, d.tokens, d.x, M, e->D, e->V, s, pdl));
  for (int l = 0; l < e->L; ++l) TL_TRY(enqueue_decode_layer_gemv(e, l, M, dbg));
  if (dbg) {
    TL_CU(launch_rmsnorm_rows(d.x, e->gfinal, e->cfg.rms_norm_eps, dbg->f32, dbg->am + 4, 1, e->D, 1, s));
    TL_TRY(d2h(e, dbg->h->final_hidden, dbg->f32, e->D * sizeof(float)));
  }
  GemvArgs lm;
  lm.x_f32 = d.x; lm.gamma = e->gfinal; lm.eps = e->cfg.rms_norm_eps;
  lm.w = e->wlm; lm.w_scale = e->slm; lm.M = M; lm.N = e->V; lm.K = e->D;
  lm.logits = logits; lm.am_partial = d.am_partial; lm.am_counter = d.am_counter; lm.am_token = d.argmax;
  TL_CU(launch_gemv(PRO_NORM, EPI_ARGMAX, lm, s, pdl));
  if (finalize) {
    StepArgs st;
    st.M = M; st.argmax = d.argmax; st.tokens = d.tokens; st.pos = d.pos; st.active = d.active;
    st.count = d.count; st.stop = d.stop; st.out_ids = d.out_ids; st.out_stride = e->P;
    st.run = d.run; st.P = e->P;
    TL_CU(launch_step_finalize(st, s, pdl));
  }
  return TL_OK;
}

tl_status get_graph(tl_engine* e, int M, cudaGraphExec_t* out) {
  auto it = e->graphs.find(M);
  if (it != e->graphs.end()) {
    *out = it->second;
    return TL_OK;
  }
  cudaGraph_t g = nullptr;
  TL_CU(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  tl_status st = enqueue_decode_step(e, M, nullptr, true);
  cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (st != TL_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  TL_CU(ce);
  cudaGraphExec_t ex = nullptr;
  cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  TL_CU(ie);
  e->graphs[M] = ex;
  *out = ex;
  return TL_OK;
}

// ------------------------------------------------------------------ prefill
// One prefill projection from the INT8 matrix xq [R][K] (rows grouped by
// sequence of S tokens): tcgen05 for R >= kTcMinRows rows, else the dp4a
// GEMV.
tl_status prefill_gemm(tl_engine* e, const int8_t* xq, const int8_t* w, const double* ws, int N, int K, int R, int S,
                       const float* in_absmax, int epi, float* out, const float* resid, float* out_absmax,
                       int32_t* out_i32 = nullptr) {
  if (R >= kTcMinRows) {
    TcPlan plan;
    TL_CU(tc_make_plan(&plan, w, N, xq, R, K, device_sm_count(), epi));
    TcArgs a;
    a.epi = epi; a.w_scale = ws; a.in_absmax = in_absmax; a.rows_per_group = S; a.out_f32 = out;
    a.resid = resid; a.out_absmax = out_absmax; a.out_i32 = out_i32;
    TL_CU(launch_gemm_tc(plan, a, e->stream, false));
    return TL_OK;
  }
  GemvArgs g;
  g.x_q = xq; g.in_absmax = in_absmax; g.rows_per_group = S;
  g.w = w; g.w_scale = ws; g.M = R; g.N = N; g.K = K; g.out_f32 = out; g.resid = resid; g.out_absmax = out_absmax;
  g.out_i32 = out_i32;
  TL_CU(launch_gemv(PRO_Q8, epi, g, e->stream, false));
  return TL_OK;
}

// Tensor parallel: max over ranks of per-sequence activation maxima (in place)
tl_status tp_allreduce_max(tl_engine* e, float* v, int n) {
  TL_NCCL(nccl_api().all_reduce(v, v, static_cast<size_t>(n), ncclFloat32, ncclMax, e->comm, e->stream));
  return TL_OK;
}

// Tensor parallel, row-split O / down (TL_TP_ALLREDUCE): this rank's INT8
// input block xq [R][K_local] (quantized with the group-wide scale) times its
// row block of W (device W^T [D][K_local]) gives partial INT32 accumulators;
// an NCCL all-reduce sums them over the ranks (integer addition: exact and
// order-free) and the dequant + residual epilogue runs on the full sums, so
// every rank holds the one-GPU result bit for bit.
tl_status tp_rowsplit_resid(tl_engine* e, const int8_t* xq, const int8_t* w, const double* ws, int K_local, int R, int S,
                            const float* in_absmax, float* x) {
  if (static_cast<size_t>(R) > e->tp_rows) return TL_ERR_OUT_OF_RANGE;
  TL_TRY(prefill_gemm(e, xq, w, ws, e->D, K_local, R, S, in_absmax, EPI_I32, nullptr, nullptr, nullptr, e->tp_acc));
  TL_NCCL(nccl_api().all_reduce(e->tp_acc, e->tp_acc, static_cast<size_t>(R) * e->D, ncclInt32, ncclSum, e->comm,
                                e->stream));
  TL_CU(launch_dequant_resid(e->tp_acc, in_absmax, S, 0, ws, x, R, e->D, e->stream));
  return TL_OK;
}

// Tensor parallel: this rank's column block x [R][Kl] (columns rank * Kl ..)
// quantized with the group-wide per-sequence scale and written into the
// full-width INT8 input [R][Kf] of every rank, then a bounded wait until
// every peer's block has arrived here. Returns the local full-width input.
tl_status tp_exchange(tl_engine* e, const float* x, int Kl, int Kf, int R, int S, const float* absmax,
                      const int8_t** full) {
  if (static_cast<size_t>(R) > e->tp_rows) return TL_ERR_OUT_OF_RANGE;
  const unsigned int epoch = ++e->tp_epoch;
  const size_t buf = (epoch & 1u) * e->tp_buf_bytes;   // exchange k uses buffer k % 2
  const size_t flag_off = 2 * e->tp_buf_bytes;
  TpScatter t;
  t.ndst = 0;
  t.dst[t.ndst] = reinterpret_cast<int8_t*>(e->tp_base + buf);
  t.flag[t.ndst++] = nullptr;
  for (int q = 0; q < e->tp_world; ++q) {
    if (q == e->tp_rank) continue;
    t.dst[t.ndst] = reinterpret_cast<int8_t*>(e->tp_peer[q] + buf);
    t.flag[t.ndst++] = reinterpret_cast<unsigned int*>(e->tp_peer[q] + flag_off) + e->tp_rank;
  }
  TL_CU(launch_quantize_scatter(x, absmax, S, R, Kl, Kf, e->tp_rank * Kl, t, e->tp_done, epoch, e->stream));
  TL_CU(launch_tp_wait(reinterpret_cast<const unsigned int*>(e->tp_base + flag_off), e->tp_world, e->tp_rank, epoch,
                       e->stream));
  *full = reinterpret_cast<const int8_t*>(e->tp_base + buf);
  return TL_OK;
}

// Layer l of a batched prefill: rows of n_seq sequences of S tokens each, in
// place on pf.x; K/V into slots slot_base..slot_base+n_seq-1. `cap` (one
// sequence only) copies the intermediate tensors out as they are produced.
tl_status enqueue_prefill_layer(tl_engine* e, int l, int n_seq, int S, int slot_base, LayerCap* cap) {
  PrefillBufs& p = e->pf;
  cudaStream_t s = e->stream;
  const bool tp = e->tp_world > 1;
  const int R = n_seq * S;
  const float eps = e->cfg.rms_norm_eps;
  const tl_layer_capture* hc = cap ? cap->h : nullptr;
  const size_t rowsD = static_cast<size_t>(R) * e->D * sizeof(float);
  const Layer& ly = e->layers[l];
  float* am = p.amax + static_cast<size_t>(l) * 4 * n_seq;
  float* kva = p.kvamax + static_cast<size_t>(l) * n_seq * 2 * e->Hkv;
  // attention block
  if (hc && hc->attn_input) {
    TL_CU(launch_rmsnorm_rows(p.x, ly.g1, eps, p.h, nullptr, R, e->D, S, s));
    TL_TRY(d2h(e, hc->attn_input, p.h, rowsD));
  }
  TL_CU(launch_norm_quant_prefill(p.x, ly.g1, eps, R, e->D, S, p.inv, am, p.h, p.xq, s));
  TL_TRY(prefill_gemm(e, p.xq, ly.wqkv, ly.sqkv, e->Nqkv, e->D, R, S, am, EPI_F32, p.qkv, nullptr, nullptr));
  if (hc) {
    TL_TRY(d2h(e, hc->qkv_input_q, p.xq, static_cast<size_t>(R) * e->D));
    TL_TRY(d2h(e, hc->qkv_input_absmax, am, sizeof(float)));
    TL_TRY(d2h_cols(e, hc->q_proj, p.qkv, R, e->Nqkv, 0, e->Dq));
    TL_TRY(d2h_cols(e, hc->k_proj, p.qkv, R, e->Nqkv, e->Dq, e->Dkv));
    TL_TRY(d2h_cols(e, hc->v_proj, p.qkv, R, e->Nqkv, e->Dq + e->Dkv, e->Dkv));
    if (hc->q_acc || hc->k_acc || hc->v_acc) {
      TL_TRY(capture_gemm(e, p.xq, ly.wqkv, ly.sqkv, e->Nqkv, e->D, R, S, am, EPI_I32, cap->i32));
      TL_TRY(d2h_cols(e, hc->q_acc, cap->i32, R, e->Nqkv, 0, e->Dq));
      TL_TRY(d2h_cols(e, hc->k_acc, cap->i32, R, e->Nqkv, e->Dq, e->Dkv));
      TL_TRY(d2h_cols(e, hc->v_acc, cap->i32, R, e->Nqkv, e->Dq + e->Dkv, e->Dkv));
    }
  }
  // RoPE of q in place, RoPE(k) and v maxima per (sequence, kv head), then the INT8 cache
  TL_CU(launch_rope_stats_prefill(p.qkv, e->Nqkv, R, S, e->H, e->Hkv, e->cosT, e->sinT, kva, s));
  TL_CU(launch_kv_write_prefill(p.qkv, e->Nqkv, R, S, e->H, e->Hkv, e->cosT, e->sinT, kva, e->kc, e->vc, e->ks,
                                e->vs, slot_base, l, e->L, e->P, s, p.kh, p.vh));
  if (cap && cap->scores) {
    TL_CU(launch_attn_scores_debug(p.qkv, e->Nqkv, S, S, 0, false, e->H, e->Hkv, e->kc, e->ks, e->cosT, e->sinT,
                                   slot_base, l, e->L, e->P, cap->scores, cap->probs, s));
    const size_t sb = static_cast<size_t>(e->H) * S * S * sizeof(float);
    TL_TRY(d2h(e, hc->scores, cap->scores, sb));
    TL_TRY(d2h(e, hc->probs, cap->probs, sb));
  }
  {
    // two-stream tcgen05 attention over the fp16 rows; the INT8-cache kernel
    // when it is disabled or the output is not 16-byte aligned
    cudaError_t ae = launch_attn_prefill_kvh(p.qkv, e->Nqkv, R, S, e->H, e->Hkv, p.kh, p.vh, e->ks, e->vs, slot_base,
                                             l, e->L, p.att, am + n_seq, s);
    if (ae == cudaErrorNotSupported)
      ae = launch_attn_prefill(p.qkv, e->Nqkv, R, S, e->H, e->Hkv, e->kc, e->vc, e->ks, e->vs, slot_base, l, e->L,
                               e->P, p.att, am + n_seq, s);
    TL_CU(ae);
  }
  const int8_t* xin = p.xq;
  const bool rowsplit = tp && e->tp_exchange == TL_TP_ALLREDUCE;
  if (tp) TL_TRY(tp_allreduce_max(e, am + n_seq, n_seq));
  if (tp && !rowsplit) {
    TL_TRY(tp_exchange(e, p.att, e->Dq, e->Dq_full, R, S, am + n_seq, &xin));
  } else {
    TL_CU(launch_quantize_rows(p.att, am + n_seq, R, e->Dq, S, p.xq, s));
  }
  if (hc) {
    TL_TRY(d2h(e, hc->attended, p.att, static_cast<size_t>(R) * e->Dq * sizeof(float)));
    TL_TRY(d2h(e, hc->o_input_q, p.xq, static_cast<size_t>(R) * e->Dq));
    TL_TRY(d2h(e, hc->o_input_absmax, am + n_seq, sizeof(float)));
    if (hc->o_acc) {
      TL_TRY(capture_gemm(e, p.xq, ly.wo, ly.so, e->D, e->Dq, R, S, am + n_seq, EPI_I32, cap->i32));
      TL_TRY(d2h(e, hc->o_acc, cap->i32, static_cast<size_t>(R) * e->D * 4));
    }
    if (hc->o_proj) {
      TL_TRY(capture_gemm(e, p.xq, ly.wo, ly.so, e->D, e->Dq, R, S, am + n_seq, EPI_F32, cap->i32));
      TL_TRY(d2h(e, hc->o_proj, cap->i32, static_cast<size_t>(R) * e->D * 4));
    }
  }
  if (rowsplit) TL_TRY(tp_rowsplit_resid(e, xin, ly.wo, ly.so, e->Dq, R, S, am + n_seq, p.x));
  else TL_TRY(prefill_gemm(e, xin, ly.wo, ly.so, e->D, e->Dq_full, R, S, am + n_seq, EPI_RESID, p.x, p.x, nullptr));
  if (hc) TL_TRY(d2h(e, hc->x_after_attn, p.x, rowsD));
  // feed-forward block
  if (hc && hc->ffn_input) {
    TL_CU(launch_rmsnorm_rows(p.x, ly.g2, eps, p.h, nullptr, R, e->D, S, s));
    TL_TRY(d2h(e, hc->ffn_input, p.h, rowsD));
  }
  TL_CU(launch_norm_quant_prefill(p.x, ly.g2, eps, R, e->D, S, p.inv, am + 2 * n_seq, p.h, p.xq, s));
  TL_TRY(prefill_gemm(e, p.xq, ly.wgu, ly.sgu, 2 * e->F, e->D, R, S, am + 2 * n_seq, EPI_SILU, p.hid, nullptr,
                      am + 3 * n_seq));
  if (hc) {
    TL_TRY(d2h(e, hc->gate_up_input_q, p.xq, static_cast<size_t>(R) * e->D));
    TL_TRY(d2h(e, hc->gate_up_input_absmax, am + 2 * n_seq, sizeof(float)));
    if (hc->gate_acc || hc->up_acc) {
      TL_TRY(capture_gemm(e, p.xq, ly.wgu, ly.sgu, 2 * e->F, e->D, R, S, am + 2 * n_seq, EPI_I32, cap->i32));
      TL_TRY(split_gate_up(e, cap->i32, R, e->F, cap->tmp_i, hc->gate_acc, hc->up_acc));
    }
    if (hc->gate_proj || hc->up_proj) {
      TL_TRY(capture_gemm(e, p.xq, ly.wgu, ly.sgu, 2 * e->F, e->D, R, S, am + 2 * n_seq, EPI_F32, cap->f32));
      TL_TRY(split_gate_up(e, static_cast<const float*>(cap->f32), R, e->F, cap->tmp_f, hc->gate_proj, hc->up_proj));
    }
  }
  xin = p.xq;
  if (tp) TL_TRY(tp_allreduce_max(e, am + 3 * n_seq, n_seq));
  if (tp && !rowsplit) {
    TL_TRY(tp_exchange(e, p.hid, e->F, e->F_full, R, S, am + 3 * n_seq, &xin));
  } else {
    TL_CU(launch_quantize_rows(p.hid, am + 3 * n_seq, R, e->F, S, p.xq, s));
  }
  if (hc) {
    TL_TRY(d2h(e, hc->hidden, p.hid, static_cast<size_t>(R) * e->F * sizeof(float)));
    TL_TRY(d2h(e, hc->down_input_q, p.xq, static_cast<size_t>(R) * e->F));
    TL_TRY(d2h(e, hc->down_input_absmax, am + 3 * n_seq, sizeof(float)));
    if (hc->down_acc) {
      TL_TRY(capture_gemm(e, p.xq, ly.wd, ly.sd, e->D, e->F, R, S, am + 3 * n_seq, EPI_I32, cap->i32));
      TL_TRY(d2h(e, hc->down_acc, cap->i32, static_cast<size_t>(R) * e->D * 4));
    }
    if (hc->down_proj) {
      TL_TRY(capture_gemm(e, p.xq, ly.wd, ly.sd, e->D, e->F, R, S, am + 3 * n_seq, EPI_F32, cap->i32));
      TL_TRY(d2h(e, hc->down_proj, cap->i32, static_cast<size_t>(R) * e->D * 4));
    }
  }
  if (rowsplit) TL_TRY(tp_rowsplit_resid(e, xin, ly.wd, ly.sd, e->F, R, S, am + 3 * n_seq, p.x));
  else TL_TRY(prefill_gemm(e, xin, ly.wd, ly.sd, e->D, e->F_full, R, S, am + 3 * n_seq, EPI_RESID, p.x, p.x, nullptr));
  return TL_OK;
}

// n_seq sequences of S tokens each, token ids already in pf.ids; slots
// slot_base..slot_base+n_seq-1. Leaves the first greedy token of each
// sequence in dec.argmax[0..n_seq) when `head` is set.
tl_status enqueue_prefill(tl_engine* e, int n_seq, int S, int slot_base, bool head, float* logits) {
  PrefillBufs& p = e->pf;
  cudaStream_t s = e->stream;
  const int R = n_seq * S;
  const float eps = e->cfg.rms_norm_eps;
  TL_CU(cudaMemsetAsync(p.amax, 0, (static_cast<size_t>(e->L) * 4 * n_seq + n_seq) * sizeof(float), s));
  TL_CU(cudaMemsetAsync(p.kvamax, 0, static_cast<size_t>(e->L) * n_seq * 2 * e->Hkv * sizeof(float), s));
  TL_CU(launch_embed(e->embed, p.ids, p.x, R, e->D, e->V, s, false));
  for (int l = 0; l < e->L; ++l) TL_TRY(enqueue_prefill_layer(e, l, n_seq, S, slot_base, nullptr));
  if (!head) return TL_OK;
  float* amf = p.amax + static_cast<size_t>(e->L) * 4 * n_seq;
  TL_CU(launch_rmsnorm_rows(p.x, e->gfinal, eps, p.h, amf, R, e->D, S, s));
  GemvArgs lm;
  lm.x_f32 = p.h; lm.x_row_offset = S - 1; lm.x_row_step = S;
  lm.in_absmax = amf; lm.rows_per_group = 1;
  lm.w = e->wlm; lm.w_scale = e->slm; lm.M = n_seq; lm.N = e->V; lm.K = e->D;
  lm.logits = logits; lm.am_partial = e->dec.am_partial; lm.am_counter = e->dec.am_counter;
  lm.am_token = e->dec.argmax;
  TL_CU(launch_gemv(PRO_F32_GIVEN, EPI_ARGMAX, lm, s, false));
  return TL_OK;
}

void fill_status(tl_run_status* st, int count, int last, int stop, int err, int pos) {
  if (!st) return;
  st->generated_count = static_cast<uint32_t>(count);
  st->last_token = static_cast<uint32_t>(last);
  st->current_layer = 0;
  st->current_block = 0;
  st->stop_reason = stop;
  st->error_code = err;
  st->position = static_cast<uint32_t>(pos);
  const bool error = err != TL_OK;
  const bool stop_valid = stop != TL_STOP_NONE;
  st->status_word = (1u << 1) | (error ? (1u << 2) : 0u) | (stop_valid ? (1u << 3) : 0u) |
                    ((static_cast<uint32_t>(stop) & 7u) << 4) |
                    ((static_cast<uint32_t>(err) & 0xFu) << 8);
}

// Runs decode steps for rows 0..M-1 until every row stopped (or abort).
// Rows must be set up (tokens, pos, active, count, stop, run params).
tl_status run_decode_loop(tl_engine* e, int M, int budget, bool* aborted) {
  *aborted = false;
  cudaGraphExec_t g = nullptr;
  TL_TRY(get_graph(e, M, &g));
  TL_TRY(ensure_pinned(e, 2 * M + 8));
  int done = 0;
  while (done < budget) {
    if (e->abort_req.load()) {
      *aborted = true;
      break;
    }
    const int chunk = std::min(8, budget - done);
    for (int i = 0; i < chunk; ++i) TL_CU(cudaGraphLaunch(g, e->stream));
    done += chunk;
    TL_CU(cudaMemcpyAsync(e->h_pinned, e->dec.active, M * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    TL_CU(cudaStreamSynchronize(e->stream));
    bool any = false;
    for (int m = 0; m < M; ++m) any |= e->h_pinned[m] != 0;
    if (!any) break;
  }
  unsigned int code = 0;
  TL_CU(tc_read_error(&code));
  if (code) {
    g_last_error = "device wait expired (code " + std::to_string(code) + ", detail " +
                   std::to_string(decode1_last_detail()) + ")";
    return TL_ERR_TIMEOUT;
  }
  return TL_OK;
}

tl_status setup_rows_after_prefill(tl_engine* e, int n_seq, int S, uint32_t max_new, uint32_t eos,
                                   uint32_t out_cap) {
  DecodeBufs& d = e->dec;
  TL_TRY(ensure_pinned(e, 8 * static_cast<size_t>(n_seq) + 8));
  int* h = e->h_pinned;
  for (int m = 0; m < n_seq; ++m) {
    h[m] = S - 1;          // finalize advances it to S
    h[n_seq + m] = 1;      // active
  }
  TL_CU(cudaMemcpyAsync(d.pos, h, n_seq * sizeof(int), cudaMemcpyHostToDevice, e->stream));
  TL_CU(cudaMemcpyAsync(d.active, h + n_seq, n_seq * sizeof(int), cudaMemcpyHostToDevice, e->stream));
  TL_CU(cudaMemsetAsync(d.count, 0, n_seq * sizeof(int), e->stream));
  TL_CU(cudaMemsetAsync(d.stop, 0, n_seq * sizeof(int), e->stream));
  int run[4] = {static_cast<int>(max_new), static_cast<int>(eos), static_cast<int>(std::min<uint32_t>(out_cap, e->P)), 0};
  std::memcpy(h + 2 * n_seq, run, sizeof(run));
  TL_CU(cudaMemcpyAsync(d.run, h + 2 * n_seq, sizeof(run), cudaMemcpyHostToDevice, e->stream));
  StepArgs st;
  st.M = n_seq; st.argmax = d.argmax; st.tokens = d.tokens; st.pos = d.pos; st.active = d.active;
  st.count = d.count; st.stop = d.stop; st.out_ids = d.out_ids; st.out_stride = e->P; st.run = d.run;
  st.P = e->P;
  TL_CU(launch_step_finalize(st, e->stream, false));
  return TL_OK;
}

tl_status collect_rows(tl_engine* e, int n_seq, uint32_t* out_ids, uint32_t out_cap, tl_run_status* st,
                       bool aborted) {
  DecodeBufs& d = e->dec;
  TL_TRY(ensure_pinned(e, 4 * static_cast<size_t>(n_seq)));
  int* h = e->h_pinned;
  TL_CU(cudaMemcpyAsync(h, d.count, n_seq * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  TL_CU(cudaMemcpyAsync(h + n_seq, d.stop, n_seq * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  TL_CU(cudaMemcpyAsync(h + 2 * n_seq, d.pos, n_seq * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  TL_CU(cudaStreamSynchronize(e->stream));
  std::vector<int> cnt(h, h + n_seq), stp(h + n_seq, h + 2 * n_seq), pos(h + 2 * n_seq, h + 3 * n_seq);
  for (int m = 0; m < n_seq; ++m) {
    const int c = std::min<int>(cnt[m], static_cast<int>(out_cap));
    if (c > 0)
      TL_CU(cudaMemcpy2D(out_ids + static_cast<size_t>(m) * out_cap, out_cap * sizeof(uint32_t),
                         d.out_ids + static_cast<size_t>(m) * e->P, e->P * sizeof(int), c * sizeof(int), 1,
                         cudaMemcpyDeviceToHost));
    int stop = stp[m], err = TL_OK;
    if (stop == 0 && aborted) stop = TL_STOP_HOST_ABORT;
    if (stop == 4) err = TL_ERR_OUT_OF_RANGE;
    const int last = c > 0 ? static_cast<int>(out_ids[static_cast<size_t>(m) * out_cap + c - 1]) : 0;
    fill_status(st ? st + m : nullptr, c, last, stop, err, pos[m]);
    e->slot_pos[m] = pos[m];
    e->slot_pending[m] = c > 0 ? last : -1;
  }
  return TL_OK;
}

}  // namespace

// ============================================================== public API
extern "C" {

const char* tl_status_string(int32_t s) {
  switch (s) {
    case TL_OK: return "ok";
    case TL_ERR_BAD_DESCRIPTOR: return "bad descriptor";
    case TL_ERR_UNSUPPORTED_MODE: return "unsupported mode";
    case TL_ERR_INTERNAL: return "internal error";
    case TL_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TL_ERR_OUT_OF_RANGE: return "out of range";
    case TL_ERR_CUDA: return g_last_error.empty() ? "cuda error" : g_last_error.c_str();
    case TL_ERR_NCCL: return g_last_error.empty() ? "nccl error" : g_last_error.c_str();
    case TL_ERR_TIMEOUT: return g_last_error.empty() ? "timeout" : g_last_error.c_str();
    case TL_ERR_NOT_LOADED: return "weights not loaded";
    case TL_ERR_UNIMPLEMENTED: return "unimplemented";
    default: return "error";
  }
}

int32_t tl_version(void) { return 0x00010000; }

namespace {
// Tensor-parallel exchange memory: one allocation per rank holding the two
// INT8 exchange matrices and the flag words, exported with a CUDA-IPC handle;
// the handles are all-gathered over the group's NCCL communicator and every
// peer's allocation is mapped here (peer access over NVLink).
tl_status tp_setup_exchange(tl_engine* e, size_t rows) {
  if (e->tp_world > 4) return TL_ERR_INVALID_ARGUMENT;
  e->tp_rows = rows;
  const size_t width = static_cast<size_t>(std::max(e->Dq_full, e->F_full));
  e->tp_buf_bytes = (rows * width + 255) / 256 * 256;
  const size_t bytes = 2 * e->tp_buf_bytes + 64 * sizeof(unsigned int);
  TL_CU(cudaMalloc(&e->tp_base, bytes));
  TL_CU(cudaMemset(e->tp_base + 2 * e->tp_buf_bytes, 0, 64 * sizeof(unsigned int)));
  TL_TRY(dmalloc(&e->tp_done, 1));
  TL_CU(cudaMemset(e->tp_done, 0, sizeof(unsigned int)));
  cudaIpcMemHandle_t mine;
  TL_CU(cudaIpcGetMemHandle(&mine, e->tp_base));
  constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
  unsigned char* dev = nullptr;
  TL_CU(cudaMalloc(&dev, kH * (e->tp_world + 1)));
  std::vector<unsigned char> all(kH * e->tp_world);
  tl_status st = TL_OK;
  cudaError_t ce = cudaMemcpy(dev + kH * e->tp_world, &mine, kH, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) {
    const ncclResult_t r =
        nccl_api().all_gather(dev + kH * e->tp_world, dev, kH, ncclUint8, e->comm, e->stream);
    if (r != ncclSuccess) {
      g_last_error = std::string("ncclAllGather: ") + nccl_api().error_string(r);
      st = TL_ERR_NCCL;
    }
  }
  if (st == TL_OK && ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
  if (st == TL_OK && ce == cudaSuccess) ce = cudaMemcpy(all.data(), dev, all.size(), cudaMemcpyDeviceToHost);
  cudaFree(dev);
  if (st != TL_OK) return st;
  TL_CU(ce);
  for (int q = 0; q < e->tp_world; ++q) {
    if (q == e->tp_rank) {
      e->tp_peer[q] = e->tp_base;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, all.data() + kH * q, kH);
    void* ptr = nullptr;
    TL_CU(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    e->tp_peer[q] = static_cast<unsigned char*>(ptr);
  }
  return TL_OK;
}

// Engine for rank `rank` of a tensor-parallel group of `world` GPUs (world 1:
// the whole model on one GPU). `id` is the NCCL group id (world > 1 only).
tl_status create_engine(const tl_config* cfg, int32_t device, int rank, int world, const ncclUniqueId* id,
                        int exchange, tl_engine** out) {
  if (!out) return TL_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  TL_TRY(check_cfg(cfg));
  if (world < 1 || rank < 0 || rank >= world || cfg->num_kv_heads % world ||
      cfg->intermediate_size % (16 * world))
    return TL_ERR_INVALID_ARGUMENT;
  TL_CU(cudaSetDevice(device));
  tl_engine* e = new tl_engine();
  e->cfg = *cfg;
  e->device = device;
  e->tp_rank = rank;
  e->tp_world = world;
  e->D = cfg->hidden_size; e->F = cfg->intermediate_size / world; e->H = cfg->num_heads / world;
  e->Hkv = cfg->num_kv_heads / world;
  e->Dq = e->H * 64; e->Dkv = e->Hkv * 64; e->Nqkv = e->Dq + 2 * e->Dkv; e->V = cfg->vocab_size;
  e->Dq_full = cfg->num_heads * 64; e->F_full = cfg->intermediate_size;
  e->tp_exchange = exchange;
  const bool rowsplit = world > 1 && exchange == TL_TP_ALLREDUCE;
  e->Dq_in = rowsplit ? e->Dq : e->Dq_full;
  e->F_in = rowsplit ? e->F : e->F_full;
  e->L = cfg->num_layers; e->P = cfg->max_positions; e->B = cfg->max_batch;
  auto fail = [&](tl_status s) { tl_destroy(e); return s; };
  if (world > 1) {
    if (!id || !nccl_api().ok) {
      g_last_error = "libnccl.so.2 not loadable";
      return fail(TL_ERR_NCCL);
    }
    const ncclResult_t r = nccl_api().comm_init_rank(&e->comm, world, *id, rank);
    if (r != ncclSuccess) {
      g_last_error = std::string("ncclCommInitRank: ") + nccl_api().error_string(r);
      e->comm = nullptr;
      return fail(TL_ERR_NCCL);
    }
  }
  cudaError_t ce = prepare_kernels(std::max(e->F, e->D));
  if (ce == cudaSuccess) ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
  for (int i = 0; i < tl_engine::kMaxGroups - 1 && ce == cudaSuccess; ++i) {
    ce = cudaStreamCreateWithFlags(&e->side[i], cudaStreamNonBlocking);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&e->ev_join[i], cudaEventDisableTiming);
  }
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming);
  if (ce != cudaSuccess) { g_last_error = cudaGetErrorString(ce); return fail(TL_ERR_CUDA); }
  if (const char* v = std::getenv("TL_DECODE_GROUPS"))
    e->decode_groups = std::max(1, std::min(tl_engine::kMaxGroups, std::atoi(v)));
  if (const char* v = std::getenv("TL_DECODE_TC_MIN_ROWS"))
    e->decode_tc_min_rows = std::max(2, std::min(kTcMinRows, std::atoi(v)));
  e->layers.resize(e->L);
  for (auto& ly : e->layers) {
    tl_status s;
    if ((s = dmalloc(&ly.wqkv, static_cast<size_t>(e->Nqkv) * e->D)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.sqkv, e->Nqkv)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.wo, static_cast<size_t>(e->D) * e->Dq_in)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.so, e->D)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.wgu, static_cast<size_t>(2) * e->F * e->D)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.sgu, 2 * e->F)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.wd, static_cast<size_t>(e->D) * e->F_in)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.sd, e->D)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.g1, e->D)) != TL_OK) return fail(s);
    if ((s = dmalloc(&ly.g2, e->D)) != TL_OK) return fail(s);
  }
  tl_status s;
  if ((s = dmalloc(&e->embed, static_cast<size_t>(e->V) * e->D)) != TL_OK) return fail(s);
  if ((s = dmalloc(&e->gfinal, e->D)) != TL_OK) return fail(s);
  if ((s = dmalloc(&e->wlm, static_cast<size_t>(e->V) * e->D)) != TL_OK) return fail(s);
  if ((s = dmalloc(&e->slm, e->V)) != TL_OK) return fail(s);
  if ((s = dmalloc(&e->cosT, static_cast<size_t>(e->P) * 64)) != TL_OK) return fail(s);
  if ((s = dmalloc(&e->sinT, static_cast<size_t>(e->P) * 64)) != TL_OK) return fail(s);
  const size_t kv = static_cast<size_t>(e->B) * e->L * e->Hkv * e->P * 64;
  if ((s = dmalloc(&e->kc, kv)) != TL_OK) return fail(s);
  if ((s = dmalloc(&e->vc, kv)) != TL_OK) return fail(s);
  if ((s = dmalloc(&e->ks, static_cast<size_t>(e->B) * e->L * e->Hkv)) != TL_OK) return fail(s);
  if ((s = dmalloc(&e->vs, static_cast<size_t>(e->B) * e->L * e->Hkv)) != TL_OK) return fail(s);
  // TL_DISABLE_DECODE1=1 keeps batch-1 steps on the multi-kernel GEMV path
  // (a comparison aid, off by default).
  const char* no_d1 = std::getenv("TL_DISABLE_DECODE1");
  e->use_decode1 = world == 1 && !(no_d1 && no_d1[0] == '1') &&
                   decode1_supported(e->D, e->F, e->Dq, e->H, e->Hkv, e->P) &&
                   decode1_prepare(e->D, e->F, e->Dq) == cudaSuccess;
  if ((s = alloc_decode(e)) != TL_OK) return fail(s);
  const size_t pf_rows = cfg->max_prefill_tokens > 0 ? cfg->max_prefill_tokens : e->P;
  if ((s = ensure_prefill(e, pf_rows, e->B)) != TL_OK) return fail(s);
  e->slot_pos.assign(e->B, 0);
  e->slot_pending.assign(e->B, -1);
  // TL_DISABLE_PDL=1 launches every kernel without programmatic dependent
  // launch (plain stream order); a debugging aid, off by default.
  if (const char* v = std::getenv("TL_DISABLE_PDL")) e->use_pdl = !(v[0] == '1');
  if (rowsplit) {
    e->tp_rows = pf_rows;
    if ((s = dmalloc(&e->tp_acc, pf_rows * e->D)) != TL_OK) return fail(s);
  } else if (world > 1 && (s = tp_setup_exchange(e, pf_rows)) != TL_OK) {
    return fail(s);
  }
  *out = e;
  return TL_OK;
}
}  // namespace

tl_status tl_create(const tl_config* cfg, int32_t device, tl_engine** out) {
  return create_engine(cfg, device, 0, 1, nullptr, TL_TP_ALLREDUCE, out);
}

tl_status tl_tp_unique_id(uint8_t* id_out) {
  if (!id_out) return TL_ERR_INVALID_ARGUMENT;
  if (!nccl_api().ok) {
    g_last_error = "libnccl.so.2 not loadable";
    return TL_ERR_NCCL;
  }
  ncclUniqueId id;
  TL_NCCL(nccl_api().get_unique_id(&id));
  static_assert(sizeof(ncclUniqueId) == TL_TP_ID_BYTES, "NCCL unique id size");
  std::memcpy(id_out, &id, sizeof(id));
  return TL_OK;
}

tl_status tl_tp_create(const tl_config* cfg, int32_t device, int32_t rank, int32_t world, const uint8_t* id,
                       tl_engine** out) {
  return tl_tp_create_ex(cfg, device, rank, world, id, TL_TP_DEFAULT, out);
}

tl_status tl_tp_create_ex(const tl_config* cfg, int32_t device, int32_t rank, int32_t world, const uint8_t* id,
                          int32_t exchange, tl_engine** out) {
  if (!id || world < 2) return TL_ERR_INVALID_ARGUMENT;
  if (exchange != TL_TP_ALLREDUCE && exchange != TL_TP_ALLGATHER) return TL_ERR_INVALID_ARGUMENT;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  return create_engine(cfg, device, rank, world, &uid, exchange, out);
}

tl_status tl_destroy(tl_engine* e) {
  if (!e) return TL_OK;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  invalidate_graphs(e);
  for (int q = 0; q < 4; ++q)
    if (e->tp_peer[q] && e->tp_peer[q] != e->tp_base) cudaIpcCloseMemHandle(e->tp_peer[q]);
  cudaFree(e->tp_base);
  cudaFree(e->tp_done);
  cudaFree(e->tp_acc);
  if (e->comm) nccl_api().comm_destroy(e->comm);
  e->comm = nullptr;
  for (auto& ly : e->layers) {
    cudaFree(ly.wqkv); cudaFree(ly.sqkv); cudaFree(ly.wo); cudaFree(ly.so); cudaFree(ly.wgu);
    cudaFree(ly.sgu); cudaFree(ly.wd); cudaFree(ly.sd); cudaFree(ly.g1); cudaFree(ly.g2);
  }
  cudaFree(e->embed); cudaFree(e->gfinal); cudaFree(e->wlm); cudaFree(e->slm);
  cudaFree(e->cosT); cudaFree(e->sinT); cudaFree(e->kc); cudaFree(e->vc); cudaFree(e->ks); cudaFree(e->vs);
  DecodeBufs& d = e->dec;
  cudaFree(d.x); cudaFree(d.qkv); cudaFree(d.att); cudaFree(d.hid); cudaFree(d.tokens); cudaFree(d.pos);
  cudaFree(d.slots); cudaFree(d.active); cudaFree(d.count); cudaFree(d.stop); cudaFree(d.out_ids);
  cudaFree(d.run); cudaFree(d.argmax); cudaFree(d.am_key); cudaFree(d.am_partial); cudaFree(d.am_counter); cudaFree(d.logits);
  cudaFree(d.xq); cudaFree(d.xq_lm); cudaFree(d.amax); cudaFree(d.amax_prod); cudaFree(d.attn_part); cudaFree(d.attn_cnt);
  cudaFree(d.d1_layers); cudaFree(d.d1_part); cudaFree(d.d1_sync);
  PrefillBufs& p = e->pf;
  cudaFree(p.ids); cudaFree(p.x); cudaFree(p.h); cudaFree(p.qkv); cudaFree(p.att); cudaFree(p.hid);
  cudaFree(p.xq); cudaFree(p.amax); cudaFree(p.kvamax); cudaFree(p.inv); cudaFree(p.kh); cudaFree(p.vh);
  cudaFree(e->logits_all);
  if (e->h_pinned) cudaFreeHost(e->h_pinned);
  if (e->stream) cudaStreamDestroy(e->stream);
  for (int i = 0; i < tl_engine::kMaxGroups - 1; ++i) {
    if (e->side[i]) cudaStreamDestroy(e->side[i]);
    if (e->ev_join[i]) cudaEventDestroy(e->ev_join[i]);
  }
  if (e->ev_fork) cudaEventDestroy(e->ev_fork);
  delete e;
  return TL_OK;
}

static tl_status upload_transposed(tl_engine* e, int8_t* tmp, const int8_t* host_kn, int K, int N,
                                   int8_t* dst_nk) {
  TL_CU(cudaMemcpyAsync(tmp, host_kn, static_cast<size_t>(K) * N, cudaMemcpyHostToDevice, e->stream));
  TL_CU(launch_transpose_i8(tmp, dst_nk, K, N, e->stream));
  return TL_OK;
}

namespace {
// Host-side slice of one layer for tensor-parallel rank r: the columns of
// Q/K/V and gate/up it produces; O and down stay whole (replicated).
struct LayerSlice {
  std::vector<int8_t> q, k, v, gate, up;
  std::vector<double> sq, sk, sv, sg, su;
  tl_layer_view view{};
};
void slice_cols(const int8_t* src, int rows, int src_cols, int col0, int cols, std::vector<int8_t>& dst) {
  dst.resize(static_cast<size_t>(rows) * cols);
  for (int i = 0; i < rows; ++i)
    std::memcpy(dst.data() + static_cast<size_t>(i) * cols, src + static_cast<size_t>(i) * src_cols + col0, cols);
}
void slice_layer(const tl_engine* e, const tl_layer_view& lv, LayerSlice& out) {
  const int r = e->tp_rank, D = e->D;
  const int Dqg = e->cfg.num_heads * 64, Dkvg = e->cfg.num_kv_heads * 64, Fg = e->cfg.intermediate_size;
  slice_cols(lv.q.w, D, Dqg, r * e->Dq, e->Dq, out.q);
  slice_cols(lv.k.w, D, Dkvg, r * e->Dkv, e->Dkv, out.k);
  slice_cols(lv.v.w, D, Dkvg, r * e->Dkv, e->Dkv, out.v);
  slice_cols(lv.gate.w, D, Fg, r * e->F, e->F, out.gate);
  slice_cols(lv.up.w, D, Fg, r * e->F, e->F, out.up);
  out.sq.assign(lv.q.scale + r * e->Dq, lv.q.scale + (r + 1) * e->Dq);
  out.sk.assign(lv.k.scale + r * e->Dkv, lv.k.scale + (r + 1) * e->Dkv);
  out.sv.assign(lv.v.scale + r * e->Dkv, lv.v.scale + (r + 1) * e->Dkv);
  out.sg.assign(lv.gate.scale + r * e->F, lv.gate.scale + (r + 1) * e->F);
  out.su.assign(lv.up.scale + r * e->F, lv.up.scale + (r + 1) * e->F);
  out.view = lv;
  out.view.q = {out.q.data(), out.sq.data()};
  out.view.k = {out.k.data(), out.sk.data()};
  out.view.v = {out.v.data(), out.sv.data()};
  out.view.gate = {out.gate.data(), out.sg.data()};
  out.view.up = {out.up.data(), out.su.data()};
}
}  // namespace

tl_status tl_load_weights(tl_engine* e, const tl_weights_view* w) {
  if (!e || !w || !w->embed || !w->final_norm || !w->lm_head.w || !w->lm_head.scale || !w->layers)
    return TL_ERR_INVALID_ARGUMENT;
  TL_CU(cudaSetDevice(e->device));
  const int D = e->D, F = e->F, Dq = e->Dq, Dkv = e->Dkv, V = e->V;
  const size_t tmp_bytes = std::max<size_t>(std::max<size_t>(static_cast<size_t>(V) * D, 2 * static_cast<size_t>(F) * D),
                                             static_cast<size_t>(std::max(e->Dq_full, e->F_full)) * D);
  int8_t* tmp = nullptr;
  TL_TRY(dmalloc(&tmp, tmp_bytes));
  auto body = [&]() -> tl_status {
    LayerSlice slice;
    for (int l = 0; l < e->L; ++l) {
      const tl_layer_view& full = w->layers[l];
      const tl_linear_view* all[7] = {&full.q, &full.k, &full.v, &full.o, &full.gate, &full.up, &full.down};
      for (auto* p : all)
        if (!p->w || !p->scale) return TL_ERR_INVALID_ARGUMENT;
      if (!full.input_norm || !full.post_norm) return TL_ERR_INVALID_ARGUMENT;
      if (e->tp_world > 1) {
        TL_CU(cudaStreamSynchronize(e->stream));  // the previous layer's slices are still being read
        slice_layer(e, full, slice);
      }
      const tl_layer_view& lv = e->tp_world > 1 ? slice.view : full;
      Layer& ly = e->layers[l];
      TL_TRY(upload_transposed(e, tmp, lv.q.w, D, Dq, ly.wqkv));
      TL_TRY(upload_transposed(e, tmp, lv.k.w, D, Dkv, ly.wqkv + static_cast<size_t>(Dq) * D));
      TL_TRY(upload_transposed(e, tmp, lv.v.w, D, Dkv, ly.wqkv + static_cast<size_t>(Dq + Dkv) * D));
      TL_CU(cudaMemcpyAsync(ly.sqkv, lv.q.scale, Dq * sizeof(double), cudaMemcpyHostToDevice, e->stream));
      TL_CU(cudaMemcpyAsync(ly.sqkv + Dq, lv.k.scale, Dkv * sizeof(double), cudaMemcpyHostToDevice, e->stream));
      TL_CU(cudaMemcpyAsync(ly.sqkv + Dq + Dkv, lv.v.scale, Dkv * sizeof(double), cudaMemcpyHostToDevice, e->stream));
      // O and down: the whole matrix, or this rank's row block (input
      // features) when they are row-split -- contiguous rows of W[in][out]
      const size_t o_row0 = e->Dq_in == e->Dq_full ? 0 : static_cast<size_t>(e->tp_rank) * e->Dq_in;
      TL_TRY(upload_transposed(e, tmp, lv.o.w + o_row0 * D, e->Dq_in, D, ly.wo));
      TL_CU(cudaMemcpyAsync(ly.so, lv.o.scale, D * sizeof(double), cudaMemcpyHostToDevice, e->stream));
      TL_CU(cudaMemcpyAsync(tmp, lv.gate.w, static_cast<size_t>(D) * F, cudaMemcpyHostToDevice, e->stream));
      TL_CU(cudaMemcpyAsync(tmp + static_cast<size_t>(D) * F, lv.up.w, static_cast<size_t>(D) * F,
                            cudaMemcpyHostToDevice, e->stream));
      TL_CU(launch_interleave_gate_up(tmp, tmp + static_cast<size_t>(D) * F, ly.wgu, D, F, e->stream));
      std::vector<double> sgu(2 * static_cast<size_t>(F));
      for (int j = 0; j < F; ++j) {
        sgu[2 * j] = lv.gate.scale[j];
        sgu[2 * j + 1] = lv.up.scale[j];
      }
      TL_CU(cudaMemcpyAsync(ly.sgu, sgu.data(), sgu.size() * sizeof(double), cudaMemcpyHostToDevice, e->stream));
      TL_CU(cudaStreamSynchronize(e->stream));  // sgu is a host temporary
      const size_t d_row0 = e->F_in == e->F_full ? 0 : static_cast<size_t>(e->tp_rank) * e->F_in;
      TL_TRY(upload_transposed(e, tmp, lv.down.w + d_row0 * D, e->F_in, D, ly.wd));
      TL_CU(cudaMemcpyAsync(ly.sd, lv.down.scale, D * sizeof(double), cudaMemcpyHostToDevice, e->stream));
      TL_CU(cudaMemcpyAsync(ly.g1, lv.input_norm, D * sizeof(float), cudaMemcpyHostToDevice, e->stream));
      TL_CU(cudaMemcpyAsync(ly.g2, lv.post_norm, D * sizeof(float), cudaMemcpyHostToDevice, e->stream));
    }
    TL_CU(cudaMemcpyAsync(e->embed, w->embed, static_cast<size_t>(V) * D * sizeof(float), cudaMemcpyHostToDevice, e->stream));
    TL_CU(cudaMemcpyAsync(e->gfinal, w->final_norm, D * sizeof(float), cudaMemcpyHostToDevice, e->stream));
    TL_TRY(upload_transposed(e, tmp, w->lm_head.w, D, V, e->wlm));
    TL_CU(cudaMemcpyAsync(e->slm, w->lm_head.scale, V * sizeof(double), cudaMemcpyHostToDevice, e->stream));
    std::vector<float> c(static_cast<size_t>(e->P) * 64), sn(static_cast<size_t>(e->P) * 64);
    if (w->rope_cos && w->rope_sin) {
      std::memcpy(c.data(), w->rope_cos, c.size() * sizeof(float));
      std::memcpy(sn.data(), w->rope_sin, sn.size() * sizeof(float));
    } else {
      for (int p = 0; p < e->P; ++p)
        for (int i = 0; i < 32; ++i) {
          const double f = 1.0 / std::pow(static_cast<double>(e->cfg.rope_theta), (2.0 * i) / 64.0);
          const double a = p * f;
          c[p * 64 + i] = c[p * 64 + i + 32] = static_cast<float>(std::cos(a));
          sn[p * 64 + i] = sn[p * 64 + i + 32] = static_cast<float>(std::sin(a));
        }
    }
    TL_CU(cudaMemcpyAsync(e->cosT, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice, e->stream));
    TL_CU(cudaMemcpyAsync(e->sinT, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice, e->stream));
    TL_CU(cudaStreamSynchronize(e->stream));
    return TL_OK;
  };
  tl_status st = body();
  cudaStreamSynchronize(e->stream);
  cudaFree(tmp);
  if (st == TL_OK) e->loaded = true;
  return st;
}

tl_status tl_init_random_weights(tl_engine* e, uint64_t seed) {
  if (!e) return TL_ERR_INVALID_ARGUMENT;
  TL_CU(cudaSetDevice(e->device));
  cudaStream_t s = e->stream;
  const double wscale = 0.02 / 73.3;  // int8 uniform[-127,127] has std ~73.3
  uint64_t k = seed * 1000003ull;
  // Each matrix is drawn as the global model's [out][in] matrix with the
  // element hash of its flat index; a tensor-parallel rank draws exactly its
  // slice, so every rank holds a piece of the same model as one GPU would.
  const long long D = e->D, r = e->tp_rank;
  const long long Dqg = static_cast<long long>(e->cfg.num_heads) * 64;
  const long long Dkvg = static_cast<long long>(e->cfg.num_kv_heads) * 64;
  const long long Fg = e->cfg.intermediate_size;
  for (auto& ly : e->layers) {
    const uint64_t kqkv = ++k;
    TL_CU(launch_random_i8_block(ly.wqkv, e->Dq, e->D, r * e->Dq, 0, D, kqkv, s));
    TL_CU(launch_random_i8_block(ly.wqkv + static_cast<size_t>(e->Dq) * e->D, e->Dkv, e->D, Dqg + r * e->Dkv, 0, D,
                                 kqkv, s));
    TL_CU(launch_random_i8_block(ly.wqkv + static_cast<size_t>(e->Dq + e->Dkv) * e->D, e->Dkv, e->D,
                                 Dqg + Dkvg + r * e->Dkv, 0, D, kqkv, s));
    TL_CU(launch_random_i8_block(ly.wo, e->D, e->Dq_in, 0, e->Dq_in == e->Dq_full ? 0 : r * e->Dq_in, Dqg, ++k, s));
    TL_CU(launch_random_i8_block(ly.wgu, 2 * e->F, e->D, 2 * r * e->F, 0, D, ++k, s));
    TL_CU(launch_random_i8_block(ly.wd, e->D, e->F_in, 0, e->F_in == e->F_full ? 0 : r * e->F_in, Fg, ++k, s));
    TL_CU(launch_fill_f64(ly.sqkv, e->Nqkv, wscale, s));
    TL_CU(launch_fill_f64(ly.so, e->D, wscale, s));
    TL_CU(launch_fill_f64(ly.sgu, 2 * e->F, wscale, s));
    TL_CU(launch_fill_f64(ly.sd, e->D, wscale, s));
    TL_CU(launch_fill_f32(ly.g1, e->D, 1.0f, s));
    TL_CU(launch_fill_f32(ly.g2, e->D, 1.0f, s));
  }
  TL_CU(launch_random_normal_f32(e->embed, static_cast<size_t>(e->V) * e->D, 0.02f, ++k, s));
  TL_CU(launch_fill_f32(e->gfinal, e->D, 1.0f, s));
  TL_CU(launch_random_i8(e->wlm, static_cast<size_t>(e->V) * e->D, ++k, s));
  TL_CU(launch_fill_f64(e->slm, e->V, wscale, s));
  std::vector<float> c(static_cast<size_t>(e->P) * 64), sn(static_cast<size_t>(e->P) * 64);
  for (int p = 0; p < e->P; ++p)
    for (int i = 0; i < 32; ++i) {
      const double f = 1.0 / std::pow(static_cast<double>(e->cfg.rope_theta), (2.0 * i) / 64.0);
      c[p * 64 + i] = c[p * 64 + i + 32] = static_cast<float>(std::cos(p * f));
      sn[p * 64 + i] = sn[p * 64 + i + 32] = static_cast<float>(std::sin(p * f));
    }
  TL_CU(cudaMemcpyAsync(e->cosT, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice, s));
  TL_CU(cudaMemcpyAsync(e->sinT, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice, s));
  TL_CU(cudaStreamSynchronize(s));
  e->loaded = true;
  return TL_OK;
}

static tl_status prefill_common(tl_engine* e, uint32_t n_seq, const uint32_t* prompts, uint32_t S,
                                bool head, float* logits) {
  if (S == 0) return TL_ERR_BAD_DESCRIPTOR;
  if (S > static_cast<uint32_t>(e->P)) return TL_ERR_OUT_OF_RANGE;
  if (n_seq == 0 || n_seq > static_cast<uint32_t>(e->B)) return TL_ERR_OUT_OF_RANGE;
  const size_t R = static_cast<size_t>(n_seq) * S;
  TL_TRY(ensure_prefill(e, R, static_cast<int>(n_seq)));
  TL_TRY(ensure_pinned(e, R));
  for (size_t i = 0; i < R; ++i) e->h_pinned[i] = static_cast<int>(prompts[i]);
  TL_CU(cudaMemcpyAsync(e->pf.ids, e->h_pinned, R * sizeof(int), cudaMemcpyHostToDevice, e->stream));
  TL_TRY(enqueue_prefill(e, static_cast<int>(n_seq), static_cast<int>(S), 0, head, logits));
  return TL_OK;
}

tl_status tl_generate_batch(tl_engine* e, uint32_t n_seqs, const uint32_t* prompts, uint32_t n_prompt,
                            uint32_t max_new, uint32_t eos, uint32_t* out_ids, uint32_t out_cap,
                            tl_run_status* st) {
  if (e && e->tp_world > 1 && max_new != 0) return TL_ERR_UNIMPLEMENTED;  // prefill-only under TP
  if (!e || !prompts || (!out_ids && out_cap)) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  TL_CU(cudaSetDevice(e->device));
  e->abort_req.store(0);
  if (n_prompt == 0) {
    for (uint32_t m = 0; st && m < n_seqs; ++m) fill_status(st + m, 0, 0, TL_STOP_NONE, TL_ERR_BAD_DESCRIPTOR, 0);
    return TL_ERR_BAD_DESCRIPTOR;
  }
  TL_TRY(prefill_common(e, n_seqs, prompts, n_prompt, max_new != 0, nullptr));
  const int M = static_cast<int>(n_seqs);
  if (max_new == 0) {  // prefill-only launch
    TL_CU(cudaStreamSynchronize(e->stream));
    for (int m = 0; m < M; ++m) {
      e->slot_pos[m] = static_cast<int>(n_prompt);
      e->slot_pending[m] = -1;
      fill_status(st ? st + m : nullptr, 0, 0, TL_STOP_NONE, TL_OK, static_cast<int>(n_prompt));
    }
    return TL_OK;
  }
  TL_TRY(setup_rows_after_prefill(e, M, static_cast<int>(n_prompt), max_new, eos, out_cap));
  bool aborted = false;
  const int budget = static_cast<int>(std::min<uint32_t>(max_new ? max_new : out_cap, out_cap));
  if (e->abort_req.load()) aborted = true;
  else TL_TRY(run_decode_loop(e, M, std::max(0, budget - 1), &aborted));
  return collect_rows(e, M, out_ids, out_cap, st, aborted);
}

tl_status tl_generate(tl_engine* e, const uint32_t* prompt, uint32_t n, uint32_t max_new, uint32_t eos,
                      uint32_t mode, uint32_t* out_ids, uint32_t out_cap, tl_run_status* st) {
  if (e && e->tp_world > 1 && (max_new != 0 || mode != TL_MODE_PREFILL)) return TL_ERR_UNIMPLEMENTED;
  if (!e) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (mode == TL_MODE_PREFILL) {
    if (n == 0) {
      fill_status(st, 0, 0, TL_STOP_NONE, TL_ERR_BAD_DESCRIPTOR, 0);
      return TL_ERR_BAD_DESCRIPTOR;
    }
    if (!prompt) return TL_ERR_INVALID_ARGUMENT;
    if (n > static_cast<uint32_t>(e->P)) {
      fill_status(st, 0, 0, TL_STOP_INTERNAL_ERR, TL_ERR_OUT_OF_RANGE, 0);
      return TL_ERR_OUT_OF_RANGE;
    }
    return tl_generate_batch(e, 1, prompt, n, max_new, eos, out_ids, out_cap, st);
  }
  if (mode != TL_MODE_DECODE) {
    fill_status(st, 0, 0, TL_STOP_NONE, TL_ERR_UNSUPPORTED_MODE, 0);
    return TL_ERR_UNSUPPORTED_MODE;
  }
  // decode-mode continuation of slot 0: feed prompt tokens (or the pending
  // token) one decode step at a time, then generate.
  TL_CU(cudaSetDevice(e->device));
  e->abort_req.store(0);
  std::vector<uint32_t> feed(prompt, prompt + n);
  if (feed.empty()) {
    if (e->slot_pending[0] < 0) {
      fill_status(st, 0, 0, TL_STOP_NONE, TL_ERR_BAD_DESCRIPTOR, e->slot_pos[0]);
      return TL_ERR_BAD_DESCRIPTOR;
    }
    feed.push_back(static_cast<uint32_t>(e->slot_pending[0]));
  }
  int pos = e->slot_pos[0];
  if (pos + static_cast<int>(feed.size()) > e->P) {
    fill_status(st, 0, 0, TL_STOP_INTERNAL_ERR, TL_ERR_OUT_OF_RANGE, pos);
    return TL_ERR_OUT_OF_RANGE;
  }
  DecodeBufs& d = e->dec;
  const uint32_t cap = std::min<uint32_t>(out_cap, static_cast<uint32_t>(e->P));
  int run[4] = {static_cast<int>(max_new), static_cast<int>(eos), static_cast<int>(cap), 0};
  TL_TRY(ensure_pinned(e, 16));
  // feed all but the last token without emitting (teacher forcing)
  for (size_t i = 0; i < feed.size(); ++i) {
    int* h = e->h_pinned;
    h[0] = static_cast<int>(feed[i]);
    h[1] = pos;
    h[2] = 1;
    TL_CU(cudaMemcpyAsync(d.tokens, h, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    TL_CU(cudaMemcpyAsync(d.pos, h + 1, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    TL_CU(cudaMemcpyAsync(d.active, h + 2, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    const bool last = i + 1 == feed.size();
    if (!last) {
      TL_TRY(enqueue_decode_step(e, 1, nullptr, false));
      TL_CU(cudaStreamSynchronize(e->stream));
      ++pos;
    } else {
      // the last fed token's step emits the first new token through finalize
      h[3] = 0;
      TL_CU(cudaMemsetAsync(d.count, 0, sizeof(int), e->stream));
      TL_CU(cudaMemsetAsync(d.stop, 0, sizeof(int), e->stream));
      std::memcpy(h + 4, run, sizeof(run));
      TL_CU(cudaMemcpyAsync(d.run, h + 4, sizeof(run), cudaMemcpyHostToDevice, e->stream));
      TL_CU(cudaStreamSynchronize(e->stream));
    }
  }
  bool aborted = false;
  const int budget = static_cast<int>(max_new ? std::min(max_new, cap) : cap);
  TL_TRY(run_decode_loop(e, 1, budget, &aborted));
  return collect_rows(e, 1, out_ids, out_cap, st, aborted);
}

tl_status tl_abort(tl_engine* e) {
  if (!e) return TL_ERR_INVALID_ARGUMENT;
  e->abort_req.store(1);
  return TL_OK;
}

tl_status tl_prefill_logits(tl_engine* e, uint32_t slot, const uint32_t* ids, uint32_t n, float* logits_out) {
  if (!e || !ids || !logits_out) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (slot != 0) return TL_ERR_UNIMPLEMENTED;
  TL_CU(cudaSetDevice(e->device));
  if (!e->dec.logits) TL_TRY(dmalloc(&e->dec.logits, static_cast<size_t>(e->B) * e->V));
  TL_TRY(prefill_common(e, 1, ids, n, true, e->dec.logits));
  TL_CU(cudaMemcpyAsync(logits_out, e->dec.logits, e->V * sizeof(float), cudaMemcpyDeviceToHost, e->stream));
  TL_CU(cudaStreamSynchronize(e->stream));
  e->slot_pos[0] = static_cast<int>(n);
  e->slot_pending[0] = -1;
  return TL_OK;
}

tl_status tl_forward_logits(tl_engine* e, const uint32_t* ids, uint32_t n, float* logits_out, float* hidden_out) {
  if (!e || !ids) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (e->tp_world > 1) return TL_ERR_UNIMPLEMENTED;
  TL_CU(cudaSetDevice(e->device));
  TL_TRY(prefill_common(e, 1, ids, n, false, nullptr));
  if (logits_out && e->logits_all_rows < n) {
    cudaFree(e->logits_all);
    e->logits_all = nullptr;
    e->logits_all_rows = 0;
    TL_TRY(dmalloc(&e->logits_all, static_cast<size_t>(n) * e->V));
    e->logits_all_rows = n;
  }
  // final RMSNorm of every row, one INT8 scale over all rows (the absmax slot
  // after the layers' four, zeroed by the prefill), LM head on every row
  PrefillBufs& p = e->pf;
  const int R = static_cast<int>(n);
  float* amf = p.amax + static_cast<size_t>(e->L) * 4;
  TL_CU(launch_rmsnorm_rows(p.x, e->gfinal, e->cfg.rms_norm_eps, p.h, amf, R, e->D, R, e->stream));
  if (hidden_out) TL_TRY(d2h(e, hidden_out, p.h, static_cast<size_t>(n) * e->D * sizeof(float)));
  if (logits_out) {
    TL_CU(launch_quantize_rows(p.h, amf, R, e->D, R, p.xq, e->stream));
    TL_TRY(prefill_gemm(e, p.xq, e->wlm, e->slm, e->V, e->D, R, R, amf, EPI_F32, e->logits_all, nullptr, nullptr));
    TL_CU(cudaMemcpyAsync(logits_out, e->logits_all, static_cast<size_t>(n) * e->V * sizeof(float),
                          cudaMemcpyDeviceToHost, e->stream));
  }
  TL_CU(cudaStreamSynchronize(e->stream));
  TL_TRY(tl_device_error());
  e->slot_pos[0] = static_cast<int>(n);
  e->slot_pending[0] = -1;
  return TL_OK;
}

tl_status tl_decoder_layer(tl_engine* e, uint32_t slot, uint32_t layer, const float* x, uint32_t n, float* out,
                           const tl_layer_capture* cap) {
  if (!e || !x) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (e->tp_world > 1) return TL_ERR_UNIMPLEMENTED;
  if (n == 0) return TL_ERR_BAD_DESCRIPTOR;
  if (slot >= static_cast<uint32_t>(e->B) || layer >= static_cast<uint32_t>(e->L) || n > static_cast<uint32_t>(e->P))
    return TL_ERR_OUT_OF_RANGE;
  TL_CU(cudaSetDevice(e->device));
  TL_TRY(ensure_prefill(e, n, 1));
  PrefillBufs& p = e->pf;
  const int S = static_cast<int>(n);
  const size_t rowsD = static_cast<size_t>(n) * e->D * sizeof(float);
  LayerCap lc;
  lc.h = cap;
  auto body = [&]() -> tl_status {
    if (cap) {
      const size_t wide = std::max<size_t>(std::max<size_t>(e->Nqkv, 2 * static_cast<size_t>(e->F)), e->D);
      TL_TRY(dmalloc(&lc.i32, static_cast<size_t>(n) * wide));
      if (cap->gate_proj || cap->up_proj) TL_TRY(dmalloc(&lc.f32, static_cast<size_t>(n) * 2 * e->F));
      if (cap->scores || cap->probs) {
        TL_TRY(dmalloc(&lc.scores, static_cast<size_t>(e->H) * n * n));
        TL_TRY(dmalloc(&lc.probs, static_cast<size_t>(e->H) * n * n));
      }
    }
    cudaStream_t s = e->stream;
    float* am = p.amax + static_cast<size_t>(layer) * 4;
    float* kva = p.kvamax + static_cast<size_t>(layer) * 2 * e->Hkv;
    TL_CU(cudaMemsetAsync(am, 0, 4 * sizeof(float), s));
    TL_CU(cudaMemsetAsync(kva, 0, 2 * e->Hkv * sizeof(float), s));
    TL_CU(cudaMemcpyAsync(p.x, x, rowsD, cudaMemcpyHostToDevice, s));
    TL_TRY(enqueue_prefill_layer(e, static_cast<int>(layer), 1, S, static_cast<int>(slot), cap ? &lc : nullptr));
    if (out) TL_CU(cudaMemcpyAsync(out, p.x, rowsD, cudaMemcpyDeviceToHost, s));
    TL_CU(cudaStreamSynchronize(s));
    return tl_device_error();
  };
  const tl_status st = body();
  cudaStreamSynchronize(e->stream);
  cudaFree(lc.i32);
  cudaFree(lc.f32);
  cudaFree(lc.scores);
  cudaFree(lc.probs);
  return st;
}

tl_status tl_decode_layer(tl_engine* e, uint32_t layer, uint32_t n, const uint32_t* slots,
                          const uint32_t* positions, const float* x, float* out, const tl_layer_capture* cap) {
  if (!e || !x || !slots || !positions) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (e->tp_world > 1) return TL_ERR_UNIMPLEMENTED;
  if (cap && (cap->scores || cap->probs)) return TL_ERR_UNIMPLEMENTED;
  if (n < static_cast<uint32_t>(kTcMinRows)) return TL_ERR_UNIMPLEMENTED;
  if (n > static_cast<uint32_t>(e->B) || layer >= static_cast<uint32_t>(e->L)) return TL_ERR_OUT_OF_RANGE;
  std::vector<char> seen(e->B, 0);
  for (uint32_t r = 0; r < n; ++r) {
    if (slots[r] >= static_cast<uint32_t>(e->B) || positions[r] >= static_cast<uint32_t>(e->P))
      return TL_ERR_OUT_OF_RANGE;
    if (seen[slots[r]]++) return TL_ERR_INVALID_ARGUMENT;
  }
  TL_CU(cudaSetDevice(e->device));
  TL_TRY(ensure_pinned(e, 3 * static_cast<size_t>(n) + static_cast<size_t>(e->B)));
  DecodeBufs& d = e->dec;
  const int M = static_cast<int>(n);
  const size_t rowsD = static_cast<size_t>(n) * e->D * sizeof(float);
  LayerCap lc;
  lc.h = cap;
  auto body = [&]() -> tl_status {
    if (cap) {
      const size_t wide = std::max<size_t>(std::max<size_t>(e->Nqkv, 2 * static_cast<size_t>(e->F)), e->D);
      TL_TRY(dmalloc(&lc.i32, static_cast<size_t>(n) * wide));
      TL_TRY(dmalloc(&lc.f32, static_cast<size_t>(n) * 2 * e->F));
    }
    cudaStream_t s = e->stream;
    int* h = e->h_pinned;
    for (int r = 0; r < M; ++r) {
      h[r] = static_cast<int>(slots[r]);
      h[M + r] = static_cast<int>(positions[r]);
      h[2 * M + r] = 1;
    }
    TL_CU(cudaMemcpyAsync(d.slots, h, M * sizeof(int), cudaMemcpyHostToDevice, s));
    TL_CU(cudaMemcpyAsync(d.pos, h + M, M * sizeof(int), cudaMemcpyHostToDevice, s));
    TL_CU(cudaMemcpyAsync(d.active, h + 2 * M, M * sizeof(int), cudaMemcpyHostToDevice, s));
    TL_CU(cudaMemcpyAsync(d.x, x, rowsD, cudaMemcpyHostToDevice, s));
    RowGroup g;
    g.M = M; g.s = s; g.attn_part = d.attn_part; g.split_rows = M;
    TL_TRY(enqueue_decode_layer_tc(e, static_cast<int>(layer), g, cap ? &lc : nullptr));
    if (out) TL_CU(cudaMemcpyAsync(out, d.x, rowsD, cudaMemcpyDeviceToHost, s));
    TL_CU(cudaStreamSynchronize(s));
    return tl_device_error();
  };
  const tl_status st = body();
  // the decode graphs read row m's cache from slot m
  int* h = e->h_pinned + 3 * static_cast<size_t>(n);
  for (int r = 0; r < e->B; ++r) h[r] = r;
  cudaMemcpyAsync(d.slots, h, e->B * sizeof(int), cudaMemcpyHostToDevice, e->stream);
  cudaStreamSynchronize(e->stream);
  cudaFree(lc.i32);
  cudaFree(lc.f32);
  return st;
}

tl_status tl_decode_logits(tl_engine* e, uint32_t slot, uint32_t token, float* logits_out) {
  if (e && e->tp_world > 1) return TL_ERR_UNIMPLEMENTED;  // decode shards by sequence, not by head
  if (!e || !logits_out) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (slot >= static_cast<uint32_t>(e->B)) return TL_ERR_OUT_OF_RANGE;
  TL_CU(cudaSetDevice(e->device));
  const int pos = e->slot_pos[slot];
  if (pos >= e->P) return TL_ERR_OUT_OF_RANGE;
  if (!e->dec.logits) TL_TRY(dmalloc(&e->dec.logits, static_cast<size_t>(e->B) * e->V));
  TL_TRY(ensure_pinned(e, 8));
  int* h = e->h_pinned;
  h[0] = static_cast<int>(token); h[1] = pos; h[2] = 1; h[3] = static_cast<int>(slot);
  DecodeBufs& d = e->dec;
  TL_CU(cudaMemcpyAsync(d.tokens, h, sizeof(int), cudaMemcpyHostToDevice, e->stream));
  TL_CU(cudaMemcpyAsync(d.pos, h + 1, sizeof(int), cudaMemcpyHostToDevice, e->stream));
  TL_CU(cudaMemcpyAsync(d.active, h + 2, sizeof(int), cudaMemcpyHostToDevice, e->stream));
  TL_CU(cudaMemcpyAsync(d.slots, h + 3, sizeof(int), cudaMemcpyHostToDevice, e->stream));
  tl_status st = enqueue_decode_step(e, 1, d.logits, false);
  h[4] = 0;
  TL_CU(cudaMemcpyAsync(d.slots, h + 4, sizeof(int), cudaMemcpyHostToDevice, e->stream));
  TL_TRY(st);
  TL_CU(cudaMemcpyAsync(logits_out, d.logits, e->V * sizeof(float), cudaMemcpyDeviceToHost, e->stream));
  TL_CU(cudaStreamSynchronize(e->stream));
  e->slot_pos[slot] = pos + 1;
  e->slot_pending[slot] = -1;
  return TL_OK;
}

tl_status tl_decode_debug(tl_engine* e, uint32_t slot, uint32_t token, uint32_t layer, tl_debug_record* rec,
                          float* logits_out) {
  if (e && e->tp_world > 1) return TL_ERR_UNIMPLEMENTED;
  if (!e || !rec) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (slot >= static_cast<uint32_t>(e->B) || layer >= static_cast<uint32_t>(e->L)) return TL_ERR_OUT_OF_RANGE;
  TL_CU(cudaSetDevice(e->device));
  const int pos = e->slot_pos[slot];
  if (pos >= e->P) return TL_ERR_OUT_OF_RANGE;
  if (!e->dec.logits) TL_TRY(dmalloc(&e->dec.logits, static_cast<size_t>(e->B) * e->V));
  TL_TRY(ensure_pinned(e, 8));
  DebugCap dc;
  dc.h = rec;
  dc.layer = static_cast<int>(layer);
  dc.slot = static_cast<int>(slot);
  dc.pos = pos;
  DecodeBufs& d = e->dec;
  cudaStream_t s = e->stream;
  auto body = [&]() -> tl_status {
    TL_TRY(dmalloc(&dc.f32, std::max(e->D, e->F)));
    TL_TRY(dmalloc(&dc.i8, std::max(e->D, e->F)));
    TL_TRY(dmalloc(&dc.am, 5));
    TL_TRY(dmalloc(&dc.sc, static_cast<size_t>(e->H) * (pos + 1)));
    TL_TRY(dmalloc(&dc.pr, static_cast<size_t>(e->H) * (pos + 1)));
    TL_CU(cudaMemsetAsync(dc.am, 0, 5 * sizeof(float), s));
    int* h = e->h_pinned;
    h[0] = static_cast<int>(token); h[1] = pos; h[2] = 1; h[3] = static_cast<int>(slot);
    TL_CU(cudaMemcpyAsync(d.tokens, h, sizeof(int), cudaMemcpyHostToDevice, s));
    TL_CU(cudaMemcpyAsync(d.pos, h + 1, sizeof(int), cudaMemcpyHostToDevice, s));
    TL_CU(cudaMemcpyAsync(d.active, h + 2, sizeof(int), cudaMemcpyHostToDevice, s));
    TL_CU(cudaMemcpyAsync(d.slots, h + 3, sizeof(int), cudaMemcpyHostToDevice, s));
    TL_TRY(enqueue_decode_step(e, 1, d.logits, false, &dc));
    TL_TRY(d2h(e, rec->input_absmax, dc.am, 5 * sizeof(float)));
    std::vector<float> lg(e->V);
    TL_CU(cudaMemcpyAsync(lg.data(), d.logits, e->V * sizeof(float), cudaMemcpyDeviceToHost, s));
    int32_t tok = 0;
    TL_CU(cudaMemcpyAsync(&tok, d.argmax, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    TL_CU(cudaStreamSynchronize(s));
    TL_TRY(tl_device_error());
    // top-16 slice: highest logit first, lower id first on equal logits
    std::vector<int> ids(e->V);
    for (int i = 0; i < e->V; ++i) ids[i] = i;
    const int k = std::min(16, e->V);
    std::partial_sort(ids.begin(), ids.begin() + k, ids.end(),
                      [&](int a, int b) { return lg[a] > lg[b] || (lg[a] == lg[b] && a < b); });
    for (int i = 0; i < 16; ++i) {
      rec->top_ids[i] = i < k ? static_cast<uint32_t>(ids[i]) : 0u;
      rec->top_logits[i] = i < k ? lg[ids[i]] : 0.0f;
    }
    rec->position = static_cast<uint32_t>(pos);
    rec->chosen_token = static_cast<uint32_t>(tok);
    if (logits_out) std::memcpy(logits_out, lg.data(), lg.size() * sizeof(float));
    return TL_OK;
  };
  const tl_status st = body();
  int* h = e->h_pinned;
  h[4] = 0;
  cudaMemcpyAsync(d.slots, h + 4, sizeof(int), cudaMemcpyHostToDevice, s);
  cudaStreamSynchronize(s);
  cudaFree(dc.f32); cudaFree(dc.i8); cudaFree(dc.am); cudaFree(dc.sc); cudaFree(dc.pr);
  if (st != TL_OK) return st;
  e->slot_pos[slot] = pos + 1;
  e->slot_pending[slot] = -1;
  return TL_OK;
}

tl_status tl_read_kv(tl_engine* e, uint32_t slot, uint32_t layer, uint32_t n_pos, int8_t* k_out,
                     int8_t* v_out, float* ks_out, float* vs_out) {
  if (!e || !k_out || !v_out || !ks_out || !vs_out) return TL_ERR_INVALID_ARGUMENT;
  if (slot >= static_cast<uint32_t>(e->B) || layer >= static_cast<uint32_t>(e->L) || n_pos > static_cast<uint32_t>(e->P))
    return TL_ERR_OUT_OF_RANGE;
  TL_CU(cudaSetDevice(e->device));
  TL_CU(cudaStreamSynchronize(e->stream));
  for (int h = 0; h < e->Hkv; ++h) {
    const size_t sidx = (static_cast<size_t>(slot) * e->L + layer) * e->Hkv + h;
    TL_CU(cudaMemcpy(k_out + static_cast<size_t>(h) * n_pos * 64, e->kc + sidx * e->P * 64,
                     static_cast<size_t>(n_pos) * 64, cudaMemcpyDeviceToHost));
    TL_CU(cudaMemcpy(v_out + static_cast<size_t>(h) * n_pos * 64, e->vc + sidx * e->P * 64,
                     static_cast<size_t>(n_pos) * 64, cudaMemcpyDeviceToHost));
    TL_CU(cudaMemcpy(ks_out + h, e->ks + sidx, sizeof(float), cudaMemcpyDeviceToHost));
    TL_CU(cudaMemcpy(vs_out + h, e->vs + sidx, sizeof(float), cudaMemcpyDeviceToHost));
  }
  return TL_OK;
}

tl_status tl_get_position(tl_engine* e, uint32_t slot, uint32_t* pos) {
  if (!e || !pos || slot >= static_cast<uint32_t>(e->B)) return TL_ERR_INVALID_ARGUMENT;
  *pos = static_cast<uint32_t>(e->slot_pos[slot]);
  return TL_OK;
}

tl_status tl_prefill_batch_device(tl_engine* e, uint32_t n_seqs, const uint32_t* prompts, uint32_t n_prompt) {
  if (!e || !prompts) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  TL_CU(cudaSetDevice(e->device));
  TL_TRY(prefill_common(e, n_seqs, prompts, n_prompt, true, nullptr));
  // rows ready for device-resident decode: no stop limit except capacity
  TL_TRY(setup_rows_after_prefill(e, static_cast<int>(n_seqs), static_cast<int>(n_prompt), 0, 0xFFFFFFFFu,
                                  static_cast<uint32_t>(e->P)));
  for (uint32_t m = 0; m < n_seqs; ++m) e->slot_pos[m] = static_cast<int>(n_prompt) + 1;
  return TL_OK;
}

tl_status tl_decode_steps_device(tl_engine* e, uint32_t n_seqs, uint32_t steps) {
  if (e && e->tp_world > 1) return TL_ERR_UNIMPLEMENTED;  // decode shards by sequence, not by head
  if (!e) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (n_seqs == 0 || n_seqs > static_cast<uint32_t>(e->B)) return TL_ERR_OUT_OF_RANGE;
  TL_CU(cudaSetDevice(e->device));
  cudaGraphExec_t g = nullptr;
  TL_TRY(get_graph(e, static_cast<int>(n_seqs), &g));
  for (uint32_t i = 0; i < steps; ++i) TL_CU(cudaGraphLaunch(g, e->stream));
  return TL_OK;
}

tl_status tl_decode_rewind(tl_engine* e, uint32_t n_seqs, uint32_t position) {
  if (e && e->tp_world > 1) return TL_ERR_UNIMPLEMENTED;  // decode shards by sequence, not by head
  if (!e) return TL_ERR_INVALID_ARGUMENT;
  if (n_seqs == 0 || n_seqs > static_cast<uint32_t>(e->B) || position >= static_cast<uint32_t>(e->P))
    return TL_ERR_OUT_OF_RANGE;
  TL_CU(cudaSetDevice(e->device));
  DecodeBufs& d = e->dec;
  TL_CU(launch_rows_rewind(d.pos, d.active, d.count, d.stop, static_cast<int>(n_seqs),
                           static_cast<int>(position), e->stream));
  return TL_OK;
}

tl_status tl_synchronize(tl_engine* e) {
  if (!e) return TL_ERR_INVALID_ARGUMENT;
  TL_CU(cudaSetDevice(e->device));
  TL_CU(cudaStreamSynchronize(e->stream));
  TL_CU(cudaGetLastError());
  unsigned int code = 0;
  TL_CU(tc_read_error(&code));
  if (code) {
    g_last_error = "device wait expired (code " + std::to_string(code) + ", detail " +
                   std::to_string(decode1_last_detail()) + ")";
    return TL_ERR_TIMEOUT;
  }
  return TL_OK;
}

tl_status tl_profile_decode_kernels(tl_engine* e, uint32_t n_seqs, uint32_t iters, float* avg_ms_out) {
  if (e && e->tp_world > 1) return TL_ERR_UNIMPLEMENTED;  // decode shards by sequence, not by head
  if (!e || !avg_ms_out || iters == 0) return TL_ERR_INVALID_ARGUMENT;
  if (!e->loaded) return TL_ERR_NOT_LOADED;
  if (n_seqs == 0 || n_seqs > static_cast<uint32_t>(e->B)) return TL_ERR_OUT_OF_RANGE;
  TL_CU(cudaSetDevice(e->device));
  const int M = static_cast<int>(n_seqs);
  const bool tc = M >= e->decode_tc_min_rows;
  DecodeBufs& d = e->dec;
  cudaStream_t s = e->stream;
  // each kind is launched as the step launches it: once per row group, the
  // groups concurrently on their streams (one group below 48 rows)
  RowGroup grp[tl_engine::kMaxGroups];
  int ng = 1;
  if (tc) {
    ng = decode_row_groups(e, M, grp);
  } else {
    grp[0].M = M; grp[0].s = s; grp[0].attn_part = d.attn_part; grp[0].split_rows = M;
  }
  const size_t flush_bytes = 256ull << 20;
  void* flush = nullptr;
  TL_CU(cudaMallocAsync(&flush, flush_bytes, s));
  std::vector<cudaEvent_t> ev(2 * iters);
  for (auto& x : ev) TL_CU(cudaEventCreate(&x));
  tl_status result = TL_OK;
  const float eps = e->cfg.rms_norm_eps;
  const size_t xq_ld = static_cast<size_t>(std::max(e->D, e->F));
  for (int kind = 0; kind < 8 && result == TL_OK; ++kind) {
    if (!tc && kind >= 6) {
      avg_ms_out[kind] = 0.0f;
      continue;
    }
    for (uint32_t it = 0; it < iters; ++it) {
      const int l = static_cast<int>(it % e->L);
      const Layer& ly = e->layers[l];
      // kinds 0-4, 6, 7: one event pair around all iters back-to-back launches
      // (layers cycled, so weights come from HBM); the LM head (one matrix) is
      // timed per launch with an L2 flush outside each interval
      const bool per_launch = kind == 5;
      if (per_launch) TL_CU(cudaMemsetAsync(flush, it & 0xff, flush_bytes, s));
      if (per_launch || it == 0) TL_CU(cudaEventRecord(ev[2 * it], s));
      // the groups fork once per timed interval, around all iters back-to-back
      // launches of each group; the LM head runs once over all rows, as in the step
      const int ngk = kind == 5 ? 1 : ng;
      RowGroup all;
      all.M = M; all.s = s; all.attn_part = d.attn_part; all.split_rows = M;
      const bool fork = it == 0, join = it + 1 == iters;
      if (ngk > 1 && fork) {
        TL_CU(cudaEventRecord(e->ev_fork, s));
        for (int i = 1; i < ngk; ++i) TL_CU(cudaStreamWaitEvent(grp[i].s, e->ev_fork, 0));
      }
      for (int gi = 0; gi < ngk && result == TL_OK; ++gi) {
        const RowGroup& rg = kind == 5 ? all : grp[gi];
        const size_t r0 = static_cast<size_t>(rg.r0);
        const int Mg = rg.M;
        cudaStream_t gs = rg.s;
        float* x = d.x + r0 * e->D;
        float* qkv = d.qkv + r0 * e->Nqkv;
        float* att = d.att + r0 * e->Dq;
        float* hid = d.hid + r0 * e->F;
        int8_t* xq = d.xq + r0 * xq_ld;
        float* amax = d.amax + r0;
        cudaError_t ce = cudaSuccess;
        tl_status ts = TL_OK;
        GemvArgs g;
        g.M = Mg;
        g.eps = eps;
        TcArgs t;
        t.in_absmax = amax;
        t.rows_per_group = 1;
        switch (kind) {
          case 0:
            if (tc) {
              t.epi = EPI_F32; t.w_scale = ly.sqkv; t.out_f32 = qkv;
              ts = tc_gemm(e, ly.wqkv, e->Nqkv, xq, Mg, e->D, t, false, gs);
            } else {
              g.x_f32 = x; g.gamma = ly.g1; g.w = ly.wqkv; g.w_scale = ly.sqkv; g.N = e->Nqkv; g.K = e->D;
              g.out_f32 = qkv;
              ce = launch_gemv(PRO_NORM, EPI_F32, g, gs, false);
            }
            break;
          case 1: {
            AttnDecodeArgs at;
            at.qkv = qkv; at.ld = e->Nqkv; at.pos = d.pos + r0; at.slot = d.slots + r0;
            at.kc = e->kc; at.vc = e->vc; at.ks = e->ks; at.vs = e->vs; at.layer = l; at.L = e->L;
            at.H = e->H; at.Hkv = e->Hkv; at.P = e->P; at.M = Mg; at.cos = e->cosT; at.sin = e->sinT;
            at.out = att;
            at.part = rg.attn_part; at.counters = d.attn_cnt + r0 * e->Hkv; at.split_rows = rg.split_rows;
            at.active = d.stop + r0;  // stop[] is 0 for running rows: read side only, no KV append
            ce = launch_attn_decode(at, gs, false);
            break;
          }
          case 2:
            if (tc) {
              t.epi = EPI_RESID; t.w_scale = ly.so; t.out_f32 = hid; t.resid = hid;
              ts = tc_gemm(e, ly.wo, e->D, xq, Mg, e->Dq, t, false, gs);
            } else {
              g.x_f32 = att; g.w = ly.wo; g.w_scale = ly.so; g.N = e->D; g.K = e->Dq; g.out_f32 = hid;
              g.resid = hid;
              ce = launch_gemv(PRO_F32, EPI_RESID, g, gs, false);
            }
            break;
          case 3:
            if (tc) {
              t.epi = EPI_SILU; t.w_scale = ly.sgu; t.out_f32 = hid;
              ts = tc_gemm(e, ly.wgu, 2 * e->F, xq, Mg, e->D, t, false, gs);
            } else {
              g.x_f32 = x; g.gamma = ly.g2; g.w = ly.wgu; g.w_scale = ly.sgu; g.N = 2 * e->F; g.K = e->D;
              g.out_f32 = hid;
              ce = launch_gemv(PRO_NORM, EPI_SILU, g, gs, false);
            }
            break;
          case 4:
            if (tc) {
              t.epi = EPI_RESID; t.w_scale = ly.sd; t.out_f32 = att; t.resid = att;
              ts = tc_gemm(e, ly.wd, e->D, xq, Mg, e->F, t, false, gs);
            } else {
              g.x_f32 = hid; g.w = ly.wd; g.w_scale = ly.sd; g.N = e->D; g.K = e->F; g.out_f32 = att;
              g.resid = att;
              ce = launch_gemv(PRO_F32, EPI_RESID, g, gs, false);
            }
            break;
          case 5:
            if (tc) {
              t.epi = EPI_F32; t.w_scale = e->slm; t.out_f32 = nullptr; t.am_key = d.am_key + r0;
              ts = tc_gemm(e, e->wlm, e->V, xq, Mg, e->D, t, false, gs);
            } else {
              g.x_f32 = x; g.gamma = e->gfinal; g.w = e->wlm; g.w_scale = e->slm; g.N = e->V; g.K = e->D;
              g.am_partial = d.am_partial; g.am_counter = d.am_counter; g.am_token = d.argmax;
              ce = launch_gemv(PRO_NORM, EPI_ARGMAX, g, gs, false);
            }
            break;
          case 6:
            ce = launch_norm_quant_rows(x, ly.g1, eps, Mg, e->D, xq, amax, gs, false);
            break;
          case 7:
            ce = tc ? launch_quant_known_rows(hid, amax, Mg, e->F, xq, gs, false)
                    : launch_quant_rows(hid, Mg, e->F, xq, amax, gs, false);
            break;
        }
        if (ce != cudaSuccess) {
          g_last_error = cudaGetErrorString(ce);
          result = TL_ERR_CUDA;
        } else if (ts != TL_OK) {
          result = ts;
        }
      }
      for (int i = 1; i < ngk && (join || result != TL_OK); ++i) {
        TL_CU(cudaEventRecord(e->ev_join[i - 1], grp[i].s));
        TL_CU(cudaStreamWaitEvent(s, e->ev_join[i - 1], 0));
      }
      if (result != TL_OK) break;
      if (per_launch || join) TL_CU(cudaEventRecord(ev[2 * it + 1], s));
    }
    if (result != TL_OK) break;
    TL_CU(cudaStreamSynchronize(s));
    double tot = 0.0;
    if (kind == 5) {
      for (uint32_t it = 0; it < iters; ++it) {
        float ms = 0.f;
        TL_CU(cudaEventElapsedTime(&ms, ev[2 * it], ev[2 * it + 1]));
        tot += ms;
      }
    } else {
      float ms = 0.f;
      TL_CU(cudaEventElapsedTime(&ms, ev[0], ev[2 * (iters - 1) + 1]));
      tot = ms;
    }
    avg_ms_out[kind] = static_cast<float>(tot / iters);
  }
  for (auto& x : ev) cudaEventDestroy(x);
  cudaStreamSynchronize(s);
  for (int i = 1; i < ng; ++i) cudaStreamSynchronize(grp[i].s);
  cudaFreeAsync(flush, s);
  // the LM-head timing accumulated argmax keys: re-arm them for the next step
  if (tc) cudaMemsetAsync(d.am_key, 0, static_cast<size_t>(e->B) * sizeof(unsigned long long), s);
  cudaStreamSynchronize(s);
  return result;
}

int32_t tl_decode_step_kernel_count(tl_engine* e) { return tl_decode_step_kernel_count_rows(e, 1); }

int32_t tl_decode_step_kernel_count_rows(tl_engine* e, uint32_t n_seqs) {
  if (!e) return 0;
  // embed, per row group 9 per layer + final norm, LM head with fused
  // argmax, finalize
  if (static_cast<int>(n_seqs) >= e->decode_tc_min_rows) {
    RowGroup g[tl_engine::kMaxGroups];
    return 1 + decode_row_groups(e, static_cast<int>(n_seqs), g) * (9 * e->L + 1) + 2;
  }
  if (n_seqs == 1 && e->use_decode1) return 2;  // persistent step + finalize
  return 1 + 5 * e->L + 2;
}

int32_t tl_decode_row_groups(tl_engine* e, uint32_t n_seqs) {
  if (!e) return 0;
  if (static_cast<int>(n_seqs) < e->decode_tc_min_rows) return 1;
  RowGroup g[tl_engine::kMaxGroups];
  return decode_row_groups(e, static_cast<int>(n_seqs), g);
}

void* tl_engine_stream(tl_engine* e) { return e ? static_cast<void*>(e->stream) : nullptr; }

}  // extern "C"
