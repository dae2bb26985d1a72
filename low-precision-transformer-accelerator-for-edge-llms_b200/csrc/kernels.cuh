// kernels.cuh -- launch interface of the sm_100a kernels (internal to the
// library; the public boundary is include/tl_api.h).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace tl {

// Activation prologue of the fused GEMV/GEMM (how the int8 operand is made).
enum Prologue : int {
  PRO_Q8 = 0,        // int8 rows given + per-group absmax (scale = absmax/127)
  PRO_F32 = 1,       // float rows; per-row absmax computed in the kernel
  PRO_NORM = 2,      // float rows; RMSNorm(gamma) then per-row absmax
  PRO_F32_GIVEN = 3  // float rows; per-group absmax given
};

// Epilogue: what is done with each INT32 accumulator.
enum Epilogue : int {
  EPI_I32 = 0,     // raw accumulator
  EPI_F32 = 1,     // float32(acc) * float32(s_x * s_w[n])
  EPI_RESID = 2,   // resid + dequant (may alias the output)
  EPI_SILU = 3,    // rows (2j, 2j+1) = (gate_j, up_j): silu(gate) * up
  EPI_REQ = 4,     // Q16.16 requantize to int8 (requantize_unit.sv)
  EPI_ARGMAX = 5   // dequant, optional logits, argmax over N per row
};

struct GemvArgs {
  const float* x_f32 = nullptr;
  const int8_t* x_q = nullptr;
  const float* gamma = nullptr;
  float eps = 1e-5f;
  const float* in_absmax = nullptr;  // [groups]
  int rows_per_group = 1;
  const int8_t* w = nullptr;         // [N][K]
  const double* w_scale = nullptr;   // [N]
  int M = 0, N = 0, K = 0;
  int32_t* out_i32 = nullptr;
  float* out_f32 = nullptr;
  const float* resid = nullptr;
  int8_t* out_i8 = nullptr;
  const uint32_t* req_scale = nullptr;
  int req_per_col = 0, req_nonneg = 0;
  float* out_absmax = nullptr;       // optional atomic max of |out| per group
  float* logits = nullptr;           // EPI_ARGMAX optional [M][N]
  unsigned long long* am_partial = nullptr;  // [gridDim.x][M]
  unsigned int* am_counter = nullptr;        // [gridDim.y]
  int32_t* am_token = nullptr;               // [M]
  int x_row_offset = 0;              // float rows: source row of m is offset + m * step
  int x_row_step = 1;                // (prefill LM head: last row of each sequence)
  NormPlan norm{8, 1};               // filled by launch_gemv from K
};

// Raises the dynamic shared-memory limit of every kernel variant for rows of
// up to max_k elements. Called once per process/device before any launch (in
// particular before stream capture, where attribute changes are not wanted).
cudaError_t prepare_kernels(int max_k);

// Upper bound on the GEMV grid (gridDim.x): the argmax epilogue keeps one
// candidate per CTA and row, so its scratch is sized by this bound.
constexpr int kGemvMaxGrid = 1024;

// Picks the tile shape and launches; `pdl` enables programmatic dependent
// launch (the kernel prefetches weights before waiting on its predecessor).
cudaError_t launch_gemv(int pro, int epi, const GemvArgs& a, cudaStream_t s, bool pdl);
// Scratch the argmax epilogue needs for a given shape.
size_t gemv_argmax_partials(int M, int N);
int gemv_argmax_row_blocks(int M);

// ---- tcgen05 INT8 GEMM (gemm_tcgen05.cu): out[m][n] = epi(sum_k X[m][k] W[n][k])
struct TcArgs {
  int M = 0, N = 0, K = 0;             // filled from the plan
  int k_splits = 1, stages = 2;        // filled from the plan
  int epi = EPI_F32;
  const double* w_scale = nullptr;     // [N]
  const float* in_absmax = nullptr;    // [groups]: scale of X row m is absmax[m / rows_per_group]/127
  int rows_per_group = 1;
  float* out_f32 = nullptr;
  const float* resid = nullptr;
  int32_t* out_i32 = nullptr;
  int8_t* out_i8 = nullptr;
  const uint32_t* req_scale = nullptr;
  int req_per_col = 0, req_nonneg = 0;
  float* out_absmax = nullptr;         // per-token max |output| (float epilogues)
  unsigned long long* am_key = nullptr;  // EPI_F32: per-token argmax key (atomic max), zero on entry
};
struct TcPlan {
  CUtensorMap tm_w;                    // W^T [N][K], 128-row boxes
  CUtensorMap tm_x;                    // X [M][K], bn-row boxes
  int bn = 64, k_splits = 1, stages = 2, M = 0, N = 0, K = 0;
};
// Encodes the two operand tensor maps and picks tile/split/stage counts.
cudaError_t tc_make_plan(TcPlan* p, const int8_t* w_nk, int N, const int8_t* x, int M, int K, int num_sms, int epi);
// Tensor map of a [rows][64] fp16 matrix in SW128 boxes of box_rows rows.
cudaError_t tc_encode_f16_rows64(CUtensorMap* tm, const void* base, long long rows, int box_rows);
cudaError_t launch_gemm_tc(const TcPlan& p, const TcArgs& a, cudaStream_t s, bool pdl);
cudaError_t prepare_tc();
int tc_max_stages(int bn, int ks = 1);
int tc_pick_bn(int M);
// Reads (and clears) the device error word of the tensor-core kernels: 0 ok,
// else the code of the bounded wait that expired.
cudaError_t tc_read_error(unsigned int* code);
int device_sm_count();

// ---- persistent single-sequence decode step (decode1.cu)
struct D1Layer {
  const int8_t* wqkv;
  const double* sqkv;
  const int8_t* wo;
  const double* so;
  const int8_t* wgu;
  const double* sgu;
  const int8_t* wd;
  const double* sd;
  const float* g1;
  const float* g2;
};
struct D1Args {
  const D1Layer* layers = nullptr;     // device array [L]
  int L = 0, D = 0, F = 0, H = 0, Hkv = 0, V = 0, P = 0, Nqkv = 0, Dq = 0;
  float eps = 1e-5f;
  NormPlan plan{8, 1};
  const float* embed = nullptr;
  const float* gfinal = nullptr;
  const int8_t* wlm = nullptr;
  const double* slm = nullptr;
  int8_t* kc = nullptr;
  int8_t* vc = nullptr;
  const float* ks = nullptr;
  const float* vs = nullptr;
  const float* cos = nullptr;
  const float* sin = nullptr;
  float* x = nullptr;                  // [D] residual stream (row 0)
  float* qkv = nullptr;
  float* att = nullptr;
  float* hid = nullptr;
  const int* token = nullptr;
  const int* pos = nullptr;
  const int* slot = nullptr;
  const int* active = nullptr;
  float* part = nullptr;               // decode1_part_floats(Hkv, P)
  unsigned int* sync = nullptr;        // decode1_sync_words(L, Hkv): barrier counter + attention tickets, zeroed before every launch
  unsigned long long* am_key = nullptr;  // [1], zero
};
bool decode1_supported(int D, int F, int Dq, int H, int Hkv, int P);
size_t decode1_smem(int D, int F, int Dq);
size_t decode1_part_floats(int Hkv, int P);
// words of D1Args::sync (grid-barrier counter + attention tickets), zeroed before every launch
size_t decode1_sync_words(int L, int Hkv);
cudaError_t decode1_prepare(int D, int F, int Dq);
cudaError_t launch_decode1(const D1Args& a, int grid, cudaStream_t s);
// Reads and clears the persistent step's error word; a nonzero code encodes
// (wait kind) * 1e6 + CTA * 1e3 + warp; decode1_last_detail() gives the ring
// chunk or barrier target of that wait.
cudaError_t decode1_read_error(unsigned int* code);
unsigned int decode1_last_detail();

struct AttnDecodeArgs {
  const float* qkv = nullptr;   // [M][ld]; q at 0, k at H*64, v at H*64 + Hkv*64
  int ld = 0;
  const int* pos = nullptr;     // [M]
  const int* slot = nullptr;    // [M]
  const int* active = nullptr;  // [M] (null = all rows active)
  int8_t* kc = nullptr;
  int8_t* vc = nullptr;
  const float* ks = nullptr;    // [slots][L][Hkv]
  const float* vs = nullptr;
  int layer = 0, L = 0, H = 0, Hkv = 0, P = 0, M = 0;
  const float* cos = nullptr;   // [P][64]
  const float* sin = nullptr;
  float* out = nullptr;         // [M][H*64]
  float* part = nullptr;        // split partials, attn_part_floats(M, Hkv, P)
  unsigned int* counters = nullptr;  // [M][Hkv], zero on entry and on exit
  int splits = 0;               // set by the launcher
  float* out_absmax = nullptr;  // [M] optional: atomic max of |out| per row (zero on entry)
  int split_rows = 0;           // rows the context split count is sized for (0: M)
};
constexpr int kAttnPartStride = 8 * 66;  // per split: 8 heads x (max, sum, 64 values)
cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t s, bool pdl);
int attn_splits(int M, int Hkv, int P);
size_t attn_part_floats(int M, int Hkv, int P);
cudaError_t attn_prepare();
cudaError_t attn_read_error(unsigned int* code);

// ---- prefill helpers (rows of n_seq sequences of seq_len tokens each)
cudaError_t launch_embed(const float* table, const int* ids, float* x, int rows, int D,
                         int vocab, cudaStream_t s, bool pdl);
cudaError_t launch_rmsnorm_rows(const float* x, const float* gamma, float eps, float* out,
                                float* absmax_groups, int rows, int D, int rows_per_group,
                                cudaStream_t s);
cudaError_t launch_quantize_rows(const float* x, const float* absmax_groups, int rows, int K,
                                 int rows_per_group, int8_t* out, cudaStream_t s);
// Prefill RMSNorm + per-sequence INT8 quantization of x into out_q: for
// D = 2048 two passes (row 1/rms into inv_buf [rows] and the sequence absmax,
// then recompute + quantize; h_buf unused), else rmsnorm into h_buf then
// quantize. absmax_groups must be zero on entry.
cudaError_t launch_norm_quant_prefill(const float* x, const float* gamma, float eps, int rows, int D,
                                      int rows_per_group, float* inv_buf, float* absmax_groups, float* h_buf,
                                      int8_t* out_q, cudaStream_t s);
cudaError_t launch_absmax_rows(const float* x, int rows, int K, int rows_per_group, float* absmax,
                               cudaStream_t s);
// Prefill RoPE and K / V cache fill (rows grouped by sequence of seq_len,
// positions 0..seq_len-1): rope_stats rotates q in place and folds max
// |RoPE(k)| and max |v| per (sequence, kv head) into kv_absmax (zero on
// entry, [seq][2][Hkv]); kv_write recomputes RoPE(k) and stores K and V
// quantized with those scales (and the scales). With kh / vh, kv_write also
// stores the same INT8 K / V values as fp16 bits (exact) in rows
// [(seq * Hkv + h) * seq_len + t][64], the operand rows of
// launch_attn_prefill_kvh.
cudaError_t launch_rope_stats_prefill(float* qkv, int ld, int rows, int seq_len, int H, int Hkv, const float* cos,
                                      const float* sin, float* kv_absmax, cudaStream_t s);
cudaError_t launch_kv_write_prefill(const float* qkv, int ld, int rows, int seq_len, int H, int Hkv, const float* cos,
                                    const float* sin, const float* kv_absmax, int8_t* kc, int8_t* vc, float* ks,
                                    float* vs, int slot_base, int layer, int L, int P, cudaStream_t s,
                                    uint16_t* kh = nullptr, uint16_t* vh = nullptr);
// Causal attention of a prefilled batch: q from qkv (rotated), K/V from cache.
cudaError_t launch_attn_prefill(const float* qkv, int ld, int rows, int seq_len, int H, int Hkv,
                                const int8_t* kc, const int8_t* vc, const float* ks,
                                const float* vs, int slot_base, int layer, int L, int P,
                                float* out, float* out_absmax, cudaStream_t s);
// The same attention reading K / V from the fp16 rows kv_write stored (kh,
// vh) through TMA; cudaErrorNotSupported when it is disabled
// (TL_DISABLE_PP_ATTN_PREFILL=1 or TL_DISABLE_TC_ATTN_PREFILL=1) or the
// output rows are not 16-byte aligned.
cudaError_t launch_attn_prefill_kvh(const float* qkv, int ld, int rows, int seq_len, int H, int Hkv,
                                    const uint16_t* kh, const uint16_t* vh, const float* ks, const float* vs,
                                    int slot_base, int layer, int L, float* out, float* out_absmax, cudaStream_t s);

// Debug capture: scores / probabilities [H][n_q][n_keys] of query rows at
// positions pos0.. of one sequence against its cache (slot `slot`); q rows in
// qkv, already rotated unless `rotate`. See kernels.cu.
cudaError_t launch_attn_scores_debug(const float* qkv, int ld, int n_q, int n_keys, int pos0, bool rotate, int H,
                                     int Hkv, const int8_t* kc, const float* ks, const float* cosT, const float* sinT,
                                     int slot, int layer, int L, int P, float* scores, float* probs, cudaStream_t s);

// ---- per-row (one sequence per row) activation prep for the batched path
// out_q[r] = quantize(rmsnorm(x[r]) ), out_absmax[r] = max|rmsnorm(x[r])|;
// zero_rows[r] = 0 when given (re-arms an atomic-max buffer for a later
// producer, after this kernel's dependency wait)
cudaError_t launch_norm_quant_rows(const float* x, const float* gamma, float eps, int rows, int D,
                                   int8_t* out_q, float* out_absmax, cudaStream_t s, bool pdl,
                                   float* zero_rows = nullptr);
// out_q[r] = quantize(x[r]) with the row's own absmax
cudaError_t launch_quant_rows(const float* x, int rows, int K, int8_t* out_q, float* out_absmax,
                              cudaStream_t s, bool pdl);
// out_q[r] = quantize(x[r]) with a precomputed absmax[r] (K % 4 == 0)
cudaError_t launch_quant_known_rows(const float* x, const float* absmax, int rows, int K, int8_t* out_q,
                                    cudaStream_t s, bool pdl);
// out[r] = argmax over logits[r][0..V) (lowest index on ties)
cudaError_t launch_row_argmax(const float* logits, int rows, int V, int32_t* out, cudaStream_t s, bool pdl);

// ---- misc
cudaError_t launch_transpose_i8(const int8_t* src_kn, int8_t* dst_nk, int K, int N,
                                cudaStream_t s);
// gate [K][F] and up [K][F] (reference layout) -> interleaved W^T [2F][K]
cudaError_t launch_interleave_gate_up(const int8_t* gate_kn, const int8_t* up_kn, int8_t* dst,
                                      int K, int F, cudaStream_t s);
cudaError_t launch_random_i8(int8_t* dst, size_t n, uint64_t seed, cudaStream_t s);
cudaError_t launch_random_normal_f32(float* dst, size_t n, float std, uint64_t seed,
                                     cudaStream_t s);
cudaError_t launch_fill_f32(float* dst, size_t n, float v, cudaStream_t s);
cudaError_t launch_fill_f64(double* dst, size_t n, double v, cudaStream_t s);

// Decode-step bookkeeping on the device (after the LM-head argmax).
struct StepArgs {
  int M = 0;
  const int32_t* argmax = nullptr;  // [M] token ids, or
  unsigned long long* am_key = nullptr;  // [M] packed argmax keys (read, then zeroed)
  int* tokens = nullptr;            // [M] next input token
  int* pos = nullptr;               // [M]
  int* active = nullptr;            // [M]
  int* count = nullptr;             // [M] emitted tokens
  int* stop = nullptr;              // [M] stop reason (0 = running)
  int* out_ids = nullptr;           // [M][out_stride]
  int out_stride = 0;
  const int* run = nullptr;         // device {max_new (0 = no limit), eos, out_cap}
  int P = 0;
};
cudaError_t launch_step_finalize(const StepArgs& a, cudaStream_t s, bool pdl);
cudaError_t launch_keys_to_tokens(unsigned long long* key, int32_t* token, int M, cudaStream_t s);
// Tensor-parallel exchange (kernels.cu): quantize this rank's column block
// and write it into every rank's full-width INT8 matrix (dst[0] local, the
// rest CUDA-IPC mapped peers); the last CTA publishes `epoch` into each
// peer's flag slot for this rank. tp_wait blocks the stream (bounded) until
// every peer's epoch has arrived in this rank's flags.
struct TpScatter {
  int8_t* dst[4];
  unsigned int* flag[4];
  int ndst;
};
cudaError_t launch_quantize_scatter(const float* x, const float* absmax, int rows_per_group, int rows, int Kl, int Kf,
                                    int col0, const TpScatter& t, unsigned int* done, unsigned int epoch,
                                    cudaStream_t s);
cudaError_t launch_tp_wait(const unsigned int* flags, int world, int rank, unsigned int epoch, cudaStream_t s);
// out[m][n] += float32(acc[m][n]) * float32(s_x(row0 + m) * w_scale[n]),
// the EPI_RESID arithmetic, after the row-split tensor-parallel all-reduce
// (acc and out point at row row0; s_x from in_absmax[(row0 + m) / rows_per_group]).
cudaError_t launch_dequant_resid(const int32_t* acc, const float* in_absmax, int rows_per_group, int row0,
                                 const double* w_scale, float* out, int rows, int N, cudaStream_t s);
cudaError_t tp_read_error(unsigned int* code);
// random int8 sub-block [rows][cols] of a global [*][src_cols] matrix whose
// element (i, j) is hash(seed, i * src_cols + j), at (src_row0, src_col0)
cudaError_t launch_random_i8_block(int8_t* dst, int rows, int cols, long long src_row0, long long src_col0,
                                   long long src_cols, uint64_t seed, cudaStream_t s);
// rows 0..M-1: pos = position, active = 1, count = 0, stop = 0
cudaError_t launch_rows_rewind(int* pos, int* active, int* count, int* stop, int M, int position,
                               cudaStream_t s);

// ---- contract mode: the hardware's Q16.16 wrappers (kernels.cu)
cudaError_t launch_contract_rmsnorm(const int8_t* xq, int rows, int D, uint32_t in_scale, const int32_t* gamma_q16,
                                    float eps, uint32_t out_scale, int8_t* yq, int32_t* y16, cudaStream_t s);
cudaError_t launch_contract_silu(const int8_t* xq, long long n, uint32_t in_scale, uint32_t out_scale, int8_t* yq,
                                 int32_t* y16, cudaStream_t s);
cudaError_t launch_contract_softmax(const int32_t* scores, int rows, int cols, uint32_t scale, int8_t* pq, int32_t* p16,
                                    cudaStream_t s);
cudaError_t launch_contract_rope(const int8_t* x, const int32_t* cs, const int32_t* sn, int rows, int8_t* out,
                                 cudaStream_t s);
cudaError_t launch_residual_add_i32(const int32_t* a, const int32_t* b, int32_t* out, long long n, cudaStream_t s);

}  // namespace tl
