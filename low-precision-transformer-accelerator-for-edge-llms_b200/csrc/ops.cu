// ops.cu -- operator-level C ABI (caller-owned device buffers + stream).
// Each entry point maps one reference operator onto the sm_100a kernels; see
// include/tl_api.h for the reference lines each one replaces.
#include <algorithm>
#include <string>

#include "../../include/tl_api.h"
#include "kernels.cuh"

using namespace tl;

namespace {

tl_status cu(cudaError_t e) { return e == cudaSuccess ? TL_OK : TL_ERR_CUDA; }

#define TL_OPS_TRY(expr)          \
  do {                            \
    tl_status _s = (expr);        \
    if (_s != TL_OK) return _s;   \
  } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

tl_status check_gemm(const void* a, const void* w, int M, int N, int K) {
  if (!a || !w) return TL_ERR_INVALID_ARGUMENT;
  if (M <= 0 || N <= 0 || K <= 0 || K % 16) return TL_ERR_INVALID_ARGUMENT;
  if (!aligned16(a) || !aligned16(w)) return TL_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TL_ERR_CUDA;
  return cu(prepare_kernels(K));
}

}  // namespace

extern "C" {

tl_status tl_device_error(void) {
  unsigned int code = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return TL_ERR_CUDA;
  if (tc_read_error(&code) != cudaSuccess) return TL_ERR_CUDA;
  return code ? TL_ERR_TIMEOUT : TL_OK;
}

tl_status tl_transpose_i8(const int8_t* w_kn, int8_t* w_nk, int32_t K, int32_t N, void* stream) {
  if (!w_kn || !w_nk || K <= 0 || N <= 0) return TL_ERR_INVALID_ARGUMENT;
  return cu(launch_transpose_i8(w_kn, w_nk, K, N, static_cast<cudaStream_t>(stream)));
}

tl_status tl_quantize_int8(const float* x, int32_t rows, int32_t cols, int32_t rows_per_group,
                           int8_t* out_q, float* out_absmax, void* stream) {
  if (!x || !out_q || !out_absmax || rows <= 0 || cols <= 0 || rows_per_group <= 0)
    return TL_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int groups = (rows + rows_per_group - 1) / rows_per_group;
  TL_OPS_TRY(cu(cudaMemsetAsync(out_absmax, 0, groups * sizeof(float), s)));
  TL_OPS_TRY(cu(launch_absmax_rows(x, rows, cols, rows_per_group, out_absmax, s)));
  return cu(launch_quantize_rows(x, out_absmax, rows, cols, rows_per_group, out_q, s));
}

// Batches of >= 16 rows go to the tcgen05 GEMM, smaller ones to the GEMV.
static constexpr int kOpsTcMinRows = 16;

static tl_status tc_op(const int8_t* a, const int8_t* w_nk, int M, int N, int K, const TcArgs& args, cudaStream_t s) {
  TcPlan p;
  TL_OPS_TRY(cu(tc_make_plan(&p, w_nk, N, a, M, K, device_sm_count(), args.epi)));
  return cu(launch_gemm_tc(p, args, s, false));
}

tl_status tl_gemm_i8(const int8_t* a, const int8_t* w_nk, int32_t* c, int32_t M, int32_t N, int32_t K,
                     void* stream) {
  if (!c) return TL_ERR_INVALID_ARGUMENT;
  TL_OPS_TRY(check_gemm(a, w_nk, M, N, K));
  if (M >= kOpsTcMinRows) {
    TcArgs t;
    t.epi = EPI_I32;
    t.out_i32 = c;
    return tc_op(a, w_nk, M, N, K, t, static_cast<cudaStream_t>(stream));
  }
  GemvArgs g;
  g.x_q = a; g.w = w_nk; g.M = M; g.N = N; g.K = K; g.out_i32 = c;
  return cu(launch_gemv(PRO_Q8, EPI_I32, g, static_cast<cudaStream_t>(stream), false));
}

tl_status tl_gemm_i8_requant(const int8_t* a, const int8_t* w_nk, const uint32_t* scale_q16,
                             int32_t per_column, int32_t nonnegative_only, int8_t* out, int32_t M,
                             int32_t N, int32_t K, void* stream) {
  if (!out || !scale_q16) return TL_ERR_INVALID_ARGUMENT;
  TL_OPS_TRY(check_gemm(a, w_nk, M, N, K));
  if (M >= kOpsTcMinRows) {
    TcArgs t;
    t.epi = EPI_REQ;
    t.out_i8 = out;
    t.req_scale = scale_q16;
    t.req_per_col = per_column ? 1 : 0;
    t.req_nonneg = nonnegative_only ? 1 : 0;
    return tc_op(a, w_nk, M, N, K, t, static_cast<cudaStream_t>(stream));
  }
  GemvArgs g;
  g.x_q = a; g.w = w_nk; g.M = M; g.N = N; g.K = K; g.out_i8 = out;
  g.req_scale = scale_q16; g.req_per_col = per_column ? 1 : 0; g.req_nonneg = nonnegative_only ? 1 : 0;
  return cu(launch_gemv(PRO_Q8, EPI_REQ, g, static_cast<cudaStream_t>(stream), false));
}

tl_status tl_quantized_linear(const float* x, const int8_t* w_nk, const double* w_scale, float* out,
                              int32_t* acc_out, int32_t M, int32_t N, int32_t K, void* stream) {
  if (!out || !w_scale) return TL_ERR_INVALID_ARGUMENT;
  TL_OPS_TRY(check_gemm(x, w_nk, M, N, K));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int8_t* xq = nullptr;
  float* amax = nullptr;
  TL_OPS_TRY(cu(cudaMallocAsync(reinterpret_cast<void**>(&xq), static_cast<size_t>(M) * K, s)));
  tl_status st = cu(cudaMallocAsync(reinterpret_cast<void**>(&amax), sizeof(float), s));
  if (st == TL_OK) st = tl_quantize_int8(x, M, K, M, xq, amax, stream);
  if (st == TL_OK && M >= kOpsTcMinRows) {
    TcArgs t;
    t.epi = EPI_F32; t.w_scale = w_scale; t.in_absmax = amax; t.rows_per_group = M; t.out_f32 = out;
    st = tc_op(xq, w_nk, M, N, K, t, s);
    if (st == TL_OK && acc_out) {
      TcArgs t2;
      t2.epi = EPI_I32;
      t2.out_i32 = acc_out;
      st = tc_op(xq, w_nk, M, N, K, t2, s);
    }
    cudaFreeAsync(xq, s);
    cudaFreeAsync(amax, s);
    return st;
  }
  if (st == TL_OK) {
    GemvArgs g;
    g.x_q = xq; g.in_absmax = amax; g.rows_per_group = M;
    g.w = w_nk; g.w_scale = w_scale; g.M = M; g.N = N; g.K = K; g.out_f32 = out;
    st = cu(launch_gemv(PRO_Q8, EPI_F32, g, s, false));
  }
  if (st == TL_OK && acc_out) {
    GemvArgs g;
    g.x_q = xq; g.w = w_nk; g.M = M; g.N = N; g.K = K; g.out_i32 = acc_out;
    st = cu(launch_gemv(PRO_Q8, EPI_I32, g, s, false));
  }
  if (xq) cudaFreeAsync(xq, s);
  if (amax) cudaFreeAsync(amax, s);
  return st;
}

tl_status tl_rmsnorm(const float* x, const float* gamma, float eps, float* out, int32_t rows, int32_t cols,
                     void* stream) {
  if (!x || !gamma || !out || rows <= 0 || cols <= 0 || cols % 4) return TL_ERR_INVALID_ARGUMENT;
  NormPlan plan;
  if (!norm_plan(cols, &plan)) return TL_ERR_INVALID_ARGUMENT;
  TL_OPS_TRY(cu(prepare_kernels(cols)));
  return cu(launch_rmsnorm_rows(x, gamma, eps, out, nullptr, rows, cols, 1, static_cast<cudaStream_t>(stream)));
}

tl_status tl_lmhead_argmax(const float* x, const float* gamma, float eps, const int8_t* w_nk,
                           const double* w_scale, int32_t rows, int32_t vocab, int32_t hidden,
                           int32_t* token_out, float* logits_out, void* stream) {
  if (!gamma || !w_scale || !token_out) return TL_ERR_INVALID_ARGUMENT;
  NormPlan plan;
  if (!norm_plan(hidden, &plan)) return TL_ERR_INVALID_ARGUMENT;
  TL_OPS_TRY(check_gemm(x, w_nk, rows, vocab, hidden));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned long long* partial = nullptr;
  unsigned int* counter = nullptr;
  const size_t n_part = gemv_argmax_partials(rows, vocab);
  const int n_cnt = gemv_argmax_row_blocks(rows);
  TL_OPS_TRY(cu(cudaMallocAsync(reinterpret_cast<void**>(&partial), n_part * sizeof(unsigned long long), s)));
  tl_status st = cu(cudaMallocAsync(reinterpret_cast<void**>(&counter), n_cnt * sizeof(unsigned int), s));
  if (st == TL_OK) st = cu(cudaMemsetAsync(counter, 0, n_cnt * sizeof(unsigned int), s));
  if (st == TL_OK) {
    GemvArgs g;
    g.x_f32 = x; g.gamma = gamma; g.eps = eps; g.w = w_nk; g.w_scale = w_scale;
    g.M = rows; g.N = vocab; g.K = hidden; g.logits = logits_out;
    g.am_partial = partial; g.am_counter = counter; g.am_token = token_out;
    st = cu(launch_gemv(PRO_NORM, EPI_ARGMAX, g, s, false));
  }
  if (partial) cudaFreeAsync(partial, s);
  if (counter) cudaFreeAsync(counter, s);
  return st;
}

tl_status tl_attn_decode(const float* qkv, const int32_t* pos, const int32_t* slot, int8_t* kc, int8_t* vc,
                         const float* ks, const float* vs, const float* rope_cos, const float* rope_sin,
                         int32_t layer, int32_t num_layers, int32_t heads, int32_t kv_heads,
                         int32_t max_positions, int32_t rows, float* out, void* stream) {
  if (!qkv || !pos || !slot || !kc || !vc || !ks || !vs || !rope_cos || !rope_sin || !out)
    return TL_ERR_INVALID_ARGUMENT;
  if (rows <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > 8 ||
      layer < 0 || layer >= num_layers || max_positions <= 0)
    return TL_ERR_INVALID_ARGUMENT;
  TL_OPS_TRY(cu(attn_prepare()));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* part = nullptr;
  unsigned int* cnt = nullptr;
  const size_t nparts = attn_part_floats(rows, kv_heads, max_positions);
  TL_OPS_TRY(cu(cudaMallocAsync(reinterpret_cast<void**>(&part), nparts * sizeof(float), s)));
  tl_status st = cu(cudaMallocAsync(reinterpret_cast<void**>(&cnt), static_cast<size_t>(rows) * kv_heads * 4, s));
  if (st == TL_OK) st = cu(cudaMemsetAsync(cnt, 0, static_cast<size_t>(rows) * kv_heads * 4, s));
  if (st == TL_OK) {
    AttnDecodeArgs a;
    a.qkv = qkv; a.ld = (heads + 2 * kv_heads) * 64; a.pos = pos; a.slot = slot; a.active = nullptr;
    a.kc = kc; a.vc = vc; a.ks = ks; a.vs = vs; a.layer = layer; a.L = num_layers; a.H = heads;
    a.Hkv = kv_heads; a.P = max_positions; a.M = rows; a.cos = rope_cos; a.sin = rope_sin; a.out = out;
    a.part = part; a.counters = cnt;
    st = cu(launch_attn_decode(a, s, false));
  }
  if (part) cudaFreeAsync(part, s);
  if (cnt) cudaFreeAsync(cnt, s);
  return st;
}

tl_status tl_attn_prefill(const float* qkv, int32_t seq_len, int32_t n_seqs, const int8_t* kc, const int8_t* vc,
                          const float* ks, const float* vs, int32_t slot_base, int32_t layer, int32_t num_layers,
                          int32_t heads, int32_t kv_heads, int32_t max_positions, float* out,
                          float* out_absmax, void* stream) {
  if (!qkv || !kc || !vc || !ks || !vs || !out) return TL_ERR_INVALID_ARGUMENT;
  if (seq_len <= 0 || n_seqs <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || slot_base < 0 ||
      layer < 0 || layer >= num_layers || max_positions <= 0)
    return TL_ERR_INVALID_ARGUMENT;
  if (seq_len > max_positions) return TL_ERR_OUT_OF_RANGE;
  if (reinterpret_cast<uintptr_t>(qkv) & 7u || reinterpret_cast<uintptr_t>(out) & 7u ||
      reinterpret_cast<uintptr_t>(kc) & 15u || reinterpret_cast<uintptr_t>(vc) & 15u)
    return TL_ERR_INVALID_ARGUMENT;
  TL_OPS_TRY(cu(attn_prepare()));
  return cu(launch_attn_prefill(qkv, (heads + 2 * kv_heads) * 64, seq_len * n_seqs, seq_len, heads, kv_heads, kc,
                                vc, ks, vs, slot_base, layer, num_layers, max_positions, out, out_absmax,
                                static_cast<cudaStream_t>(stream)));
}

tl_status tl_contract_rmsnorm(const int8_t* x_q, int32_t rows, int32_t cols, uint32_t in_scale_q16,
                              const int32_t* gamma_q16, float eps, uint32_t out_scale_q16, int8_t* y_q,
                              int32_t* y_q16, void* stream) {
  if (!x_q || !gamma_q16 || !y_q || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARGUMENT;
  return cu(launch_contract_rmsnorm(x_q, rows, cols, in_scale_q16, gamma_q16, eps, out_scale_q16, y_q, y_q16,
                                    static_cast<cudaStream_t>(stream)));
}

tl_status tl_contract_silu(const int8_t* x_q, int64_t n, uint32_t in_scale_q16, uint32_t out_scale_q16, int8_t* y_q,
                           int32_t* y_q16, void* stream) {
  if (!x_q || !y_q || n <= 0) return TL_ERR_INVALID_ARGUMENT;
  return cu(launch_contract_silu(x_q, n, in_scale_q16, out_scale_q16, y_q, y_q16, static_cast<cudaStream_t>(stream)));
}

tl_status tl_contract_softmax(const int32_t* scores, int32_t rows, int32_t cols, uint32_t score_scale_q16,
                              int8_t* prob_q, int32_t* prob_q16, void* stream) {
  if (!scores || !prob_q || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARGUMENT;
  if (cols > 128) return TL_ERR_OUT_OF_RANGE;
  return cu(launch_contract_softmax(scores, rows, cols, score_scale_q16, prob_q, prob_q16,
                                    static_cast<cudaStream_t>(stream)));
}

tl_status tl_contract_rope(const int8_t* x_q, const int32_t* cos_q16, const int32_t* sin_q16, int32_t rows,
                           int8_t* out, void* stream) {
  if (!x_q || !cos_q16 || !sin_q16 || !out || rows <= 0) return TL_ERR_INVALID_ARGUMENT;
  return cu(launch_contract_rope(x_q, cos_q16, sin_q16, rows, out, static_cast<cudaStream_t>(stream)));
}

tl_status tl_residual_add_i32(const int32_t* residual_q16, const int32_t* update_q16, int32_t* out, int64_t n,
                              void* stream) {
  if (!residual_q16 || !update_q16 || !out || n <= 0) return TL_ERR_INVALID_ARGUMENT;
  return cu(launch_residual_add_i32(residual_q16, update_q16, out, n, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
