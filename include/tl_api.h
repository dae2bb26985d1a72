/*
 * tl_api.h -- C ABI of the B200 TinyLlama INT8 engine.
 *
 * Plain C: integer status codes, host/device pointers and sizes; no C++ or
 * torch types. Two layers of entry points:
 *
 *  1. Runtime contract (host buffers). Replaces the FPGA's launch/status
 *     register interface and its three controllers:
 *       rtl/control/prefill_decode_controller.sv:39-198  (prefill -> LM head ->
 *           token -> decode loop, bad-descriptor check, prefill-only launch)
 *       rtl/control/layer_controller.sv:25-195           (per-layer block order)
 *       rtl/control/stop_condition_unit.sv:19-37         (abort > EOS > max)
 *     and the Python driver model/tinyllama_gemm_int8.py:629-685 (run_generate).
 *
 *  2. Operator entry points (caller-owned device buffers plus a CUDA stream),
 *     one per reference operator, for parity checks and for callers that drive
 *     their own loop:
 *       quantize_int8      model/tinyllama_gemm_int8.py:36-42
 *       quantized_linear   model/tinyllama_gemm_int8.py:59-88
 *       shared GEMM        rtl/compute/shared_gemm_engine.sv:127-168
 *       requantize         rtl/compute/requantize_unit.sv:39-93
 *       rms_norm           model/tinyllama.py:45-50
 *       LM head + argmax   rtl/compute/argmax_reduction.sv:47-131,
 *                          model/tinyllama_gemm_int8.py:463-467,671
 *
 * Weight layout at this boundary is the reference's: W[in][out] row-major so
 * that y = x @ W (model/tinyllama.py:106-110, :339-364). Device-side operator
 * entry points take the engine's device layout instead, W^T[out][in] (each
 * output channel's inputs contiguous, the K-major operand of the tensor
 * cores); tl_transpose_i8 converts.
 *
 * Threading: calls on one engine are serialized by the caller (the RTL
 * accepts START only when idle). tl_abort() is the one thread-safe call; the
 * runtime samples it between decode steps.
 */
#ifndef TL_API_H
#define TL_API_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TL_API __attribute__((visibility("default")))
#else
#define TL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 0..7 mirror error_code_e (rtl/common/tinyllama_pkg.sv:260-269);
 * 16.. are engine conditions with no RTL counterpart. */
typedef enum tl_status {
  TL_OK = 0,
  TL_ERR_BAD_DESCRIPTOR = 1,   /* empty prompt in prefill mode (prefill_decode_controller.sv:85-88) */
  TL_ERR_HBM_READ = 2,
  TL_ERR_HBM_WRITE = 3,
  TL_ERR_SCALE_METADATA = 4,
  TL_ERR_DEBUG_OVERFLOW = 5,
  TL_ERR_UNSUPPORTED_MODE = 6,
  TL_ERR_INTERNAL = 7,
  TL_ERR_INVALID_ARGUMENT = 16, /* null pointer, bad shape or alignment */
  TL_ERR_OUT_OF_RANGE = 17,     /* position would exceed max_positions, batch > max_batch */
  TL_ERR_CUDA = 18,
  TL_ERR_NCCL = 19,
  TL_ERR_TIMEOUT = 20,
  TL_ERR_NOT_LOADED = 21,       /* weights not loaded */
  TL_ERR_UNIMPLEMENTED = 22
} tl_status;

/* stop_reason_e (rtl/common/tinyllama_pkg.sv:252-258). */
typedef enum tl_stop_reason {
  TL_STOP_NONE = 0,
  TL_STOP_EOS = 1,
  TL_STOP_MAX_TOKENS = 2,
  TL_STOP_HOST_ABORT = 3,
  TL_STOP_INTERNAL_ERR = 4
} tl_stop_reason;

/* Launch modes (runtime_mode_e, rtl/common/tinyllama_pkg.sv:177-180). */
enum { TL_MODE_PREFILL = 0, TL_MODE_DECODE = 1 };

typedef struct tl_config {
  int32_t hidden_size;        /* 2048 */
  int32_t intermediate_size;  /* 5632 */
  int32_t num_layers;         /* 22 */
  int32_t num_heads;          /* 32 */
  int32_t num_kv_heads;       /* 4 */
  int32_t head_dim;           /* 64 (only 64 is supported) */
  int32_t vocab_size;         /* 32000 */
  int32_t max_positions;      /* 2048 */
  float rms_norm_eps;         /* 1e-5 */
  float rope_theta;           /* 10000 */
  int32_t max_batch;          /* sequences held at once (KV slots) */
  int32_t max_prefill_tokens; /* rows of one batched prefill (sum of prompt lengths) */
} tl_config;

/* One projection: int8 W[in][out] row-major plus one float64 scale per output
 * channel (a per-tensor scale is passed broadcast). */
typedef struct tl_linear_view {
  const int8_t* w;
  const double* scale;
} tl_linear_view;

typedef struct tl_layer_view {
  tl_linear_view q, k, v, o, gate, up, down;
  const float* input_norm;    /* [hidden] */
  const float* post_norm;     /* [hidden] */
} tl_layer_view;

/* Host view of a whole quantized model (TinyLlamaWeights key schema,
 * model/tinyllama.py:240-267). rope_cos/rope_sin are the float32 tables of
 * model/tinyllama.py:59-66, [max_positions][head_dim]. */
typedef struct tl_weights_view {
  const float* embed;         /* [vocab][hidden] */
  const float* final_norm;    /* [hidden] */
  tl_linear_view lm_head;     /* W[hidden][vocab] */
  const tl_layer_view* layers;/* [num_layers] */
  const float* rope_cos;
  const float* rope_sin;
} tl_weights_view;

/* Host-visible run status (STATUS register and status beat,
 * rtl/common/tinyllama_pkg.sv:128-133, 159-166). */
typedef struct tl_run_status {
  uint32_t status_word;      /* bit0 busy, bit1 done, bit2 error, bit3 stop_valid,
                                bits[6:4] stop_reason, bits[11:8] error_code */
  uint32_t generated_count;
  uint32_t last_token;
  uint32_t current_layer;
  uint32_t current_block;
  int32_t stop_reason;       /* tl_stop_reason */
  int32_t error_code;        /* tl_status */
  uint32_t position;         /* tokens held in this sequence's KV cache */
} tl_run_status;

typedef struct tl_engine tl_engine;

/* ---------------------------------------------------------------- runtime */
TL_API const char* tl_status_string(int32_t status);
TL_API int32_t tl_version(void);

TL_API tl_status tl_create(const tl_config* cfg, int32_t device, tl_engine** out);
TL_API tl_status tl_destroy(tl_engine* eng);

/* Tensor-parallel prefill over `world` GPUs, one process (or thread) and one
 * engine per GPU. The reference's prefill is the recompute forward_mixed
 * (model/tinyllama_gemm_int8.py:432-467); its TP-2/4 split is by KV head:
 * rank r holds kv heads [r Hkv/world, (r+1) Hkv/world) and their query
 * heads and the matching columns of Q/K/V and gate/up; RMSNorm, embedding
 * and LM head are replicated. The O and down inputs are quantized with
 * group-wide per-sequence scales (NCCL all-reduce max). Two exchanges:
 *  TL_TP_ALLREDUCE  O and down are row-split (rank r holds the input rows of
 *                   its heads / its FFN columns); each rank's partial INT32
 *                   accumulators are summed by an NCCL all-reduce over
 *                   NVLink before the dequant + residual epilogue;
 *  TL_TP_ALLGATHER  O and down are replicated; each rank's INT8 input block
 *                   is written into every rank's full-width input by peer
 *                   stores over NVLink (CUDA-IPC mappings set up here).
 * Integer sums are exact and order-free, so with either exchange the logits
 * are bit-identical to one GPU's. world (<= 4) must divide num_kv_heads and
 * intermediate_size / 16; a prefill call may hold at most
 * max_prefill_tokens rows.
 * tl_tp_unique_id: rank 0 draws the group id; the host hands the same
 * TL_TP_ID_BYTES bytes to every rank's tl_tp_create (all ranks must call it
 * concurrently: it blocks until the group is complete). tl_load_weights on
 * a TP engine takes the FULL model view and keeps this rank's slice;
 * tl_init_random_weights draws exactly the slice of the single-GPU model of
 * the same seed. Prefill calls (tl_prefill_logits, tl_prefill_batch_device,
 * tl_generate / tl_generate_batch with max_new_tokens == 0) are collective:
 * every rank makes the same calls in the same order. Decode entry points
 * return TL_ERR_UNIMPLEMENTED on a TP engine (decode scales by sequence).
 * tl_read_kv returns this rank's kv heads. NCCL (libnccl.so.2) is loaded at
 * run time; TL_ERR_NCCL when it is missing or a collective fails;
 * TL_ERR_TIMEOUT (tl_synchronize) when a peer's activations do not arrive. */
#define TL_TP_ID_BYTES 128
enum { TL_TP_ALLREDUCE = 0, TL_TP_ALLGATHER = 1 };
/* The default is the faster exchange measured on B200 pairs: at TP-2 on the
 * 8 x 2048 prefill the INT8 all-gather moves 16 + 46 MB per layer and rank
 * against 2 x 134 MB of INT32 partial sums for the all-reduce. */
#define TL_TP_DEFAULT TL_TP_ALLGATHER
TL_API tl_status tl_tp_unique_id(uint8_t* id_out);
/* tl_tp_create_ex with exchange TL_TP_DEFAULT. */
TL_API tl_status tl_tp_create(const tl_config* cfg, int32_t device, int32_t rank, int32_t world, const uint8_t* id,
                              tl_engine** out);
TL_API tl_status tl_tp_create_ex(const tl_config* cfg, int32_t device, int32_t rank, int32_t world, const uint8_t* id,
                                 int32_t exchange, tl_engine** out);
/* Copies (and lays out) the host weights into the engine's device arena. */
TL_API tl_status tl_load_weights(tl_engine* eng, const tl_weights_view* w);
/* Random INT8 weights drawn on the device (benchmarks of the full model
 * without a host archive): int8 uniform in [-127,127], per-channel scale
 * 0.02/73.3 (the uniform int8 std), so each matrix has std ~0.02.
 * Norm gains 1, embeddings N(0, 0.02) via a counter-based hash. */
TL_API tl_status tl_init_random_weights(tl_engine* eng, uint64_t seed);

/* Greedy generation for one sequence held in KV slot 0.
 * mode TL_MODE_PREFILL: resets the slot, prefills prompt[0..n), then decodes.
 *   n == 0 -> TL_ERR_BAD_DESCRIPTOR; max_new_tokens == 0 -> prefill only.
 * mode TL_MODE_DECODE: continues the slot's cache; feeds prompt[0..n) as
 *   decode steps, or the pending last token when n == 0; max_new_tokens == 0
 *   means no limit other than out_cap and max_positions.
 * Tokens are written to out_ids[0..generated_count). */
TL_API tl_status tl_generate(tl_engine* eng, const uint32_t* prompt, uint32_t n_prompt,
                      uint32_t max_new_tokens, uint32_t eos_id, uint32_t mode,
                      uint32_t* out_ids, uint32_t out_cap, tl_run_status* st);

/* Batched generation of n_seqs independent sequences (slots 0..n_seqs), all
 * prompts of equal length n_prompt (prompts is [n_seqs][n_prompt]). Each
 * sequence stops on its own (EOS / max / abort); out_ids is [n_seqs][out_cap],
 * st is [n_seqs]. */
TL_API tl_status tl_generate_batch(tl_engine* eng, uint32_t n_seqs, const uint32_t* prompts,
                            uint32_t n_prompt, uint32_t max_new_tokens, uint32_t eos_id,
                            uint32_t* out_ids, uint32_t out_cap, tl_run_status* st);

/* Host abort request (CONTROL.ABORT_REQ): thread-safe, sampled between steps. */
TL_API tl_status tl_abort(tl_engine* eng);

/* Teacher-forced access for parity checks.
 * tl_prefill_logits: prefill slot `slot` with ids[0..n) and return the last
 *   row's float32 logits [vocab] (host).
 * tl_decode_logits: feed one token to slot `slot` at its current position and
 *   return the float32 logits [vocab] (host). */
TL_API tl_status tl_prefill_logits(tl_engine* eng, uint32_t slot, const uint32_t* ids, uint32_t n,
                            float* logits_out);
TL_API tl_status tl_decode_logits(tl_engine* eng, uint32_t slot, uint32_t token, float* logits_out);

/* Debug capture of one decode step (docs/design_decisions.txt B8, the
 * layer-/step-scoped capture of rtl/compute/debug_capture_mux.sv): the
 * fixed tensor set of layer `layer` plus the step's final hidden state,
 * top-16 logits and chosen token, read back after the step completes. Every
 * pointer is an optional HOST destination (NULL skips it); the scalar fields
 * are always written. Dq = heads*64, Dkv = kv_heads*64, n = position + 1. */
typedef struct tl_debug_record {
  uint32_t position;          /* position of the fed token (its K/V row) */
  uint32_t chosen_token;      /* greedy argmax (lowest id on ties) */
  uint32_t top_ids[16];       /* the 16 largest logits, highest first (lower id first on ties) */
  float top_logits[16];
  float input_absmax[5];      /* max |x| of the INT8 inputs of q/k/v, o, gate/up, down and the
                                 LM head (each quantization scale is absmax / 127) */
  float* layer_input;         /* [hidden]    layer input activation */
  int8_t* qkv_input_q;        /* [hidden]    quantized input of the q/k/v projections */
  float* q_proj;              /* [Dq]        q, k, v before RoPE */
  float* k_proj;              /* [Dkv] */
  float* v_proj;              /* [Dkv] */
  float* scores;              /* [heads][n]  attention-score window */
  float* probs;               /* [heads][n]  post-softmax window */
  int8_t* k_row;              /* [kv_heads][64] updated K-cache row */
  int8_t* v_row;              /* [kv_heads][64] updated V-cache row */
  float* k_scale;             /* [kv_heads]  their scales */
  float* v_scale;             /* [kv_heads] */
  float* attended;            /* [Dq]        attention output */
  float* layer_output;        /* [hidden]    layer output activation */
  float* final_hidden;        /* [hidden]    final RMSNorm output */
} tl_debug_record;

/* tl_decode_logits with the debug capture of layer `layer`: feeds `token`
 * to slot `slot` at its current position (advancing it) on the per-kernel
 * decode path, fills `rec`, and (if logits_out is not NULL) the float32
 * logits [vocab]. The performance path (graph-captured steps) is untouched.
 * TL_ERR_UNIMPLEMENTED on a tensor-parallel engine. */
TL_API tl_status tl_decode_debug(tl_engine* eng, uint32_t slot, uint32_t token, uint32_t layer, tl_debug_record* rec,
                                 float* logits_out);
/* Copies one (slot, layer) of the INT8 KV cache to host: k/v [kv_heads][n_pos][head_dim],
 * scales [kv_heads]. */
TL_API tl_status tl_read_kv(tl_engine* eng, uint32_t slot, uint32_t layer, uint32_t n_pos,
                     int8_t* k_out, int8_t* v_out, float* k_scale_out, float* v_scale_out);
TL_API tl_status tl_get_position(tl_engine* eng, uint32_t slot, uint32_t* pos);

/* Logits of EVERY prompt row, as forward_mixed returns them
 * (model/tinyllama_gemm_int8.py:437-467 with quantize_lm_head: final RMSNorm
 * of all n rows, one per-tensor INT8 scale over those rows, INT8 LM head on
 * each row). Prefills slot 0 with ids[0..n) like tl_prefill_logits;
 * logits_out (may be NULL) is host float32 [n][vocab]; hidden_out (may be
 * NULL) receives the final RMSNorm output [n][hidden], the input of the LM
 * head (:463). */
TL_API tl_status tl_forward_logits(tl_engine* eng, const uint32_t* ids, uint32_t n, float* logits_out,
                                   float* hidden_out);

/* Per-layer capture of tl_decoder_layer: every pointer is an optional HOST
 * destination (NULL skips it). Names follow the debug dictionaries of
 * mixed_precision_decoder_layer (model/tinyllama_gemm_int8.py:136-281):
 * *_input_q / *_acc are the `input_q` / `accum_int32` of each
 * quantized_linear, *_input_absmax the max |x| whose /127 is `input_scale`.
 * S = rows of the call, Dq = heads*64, Dkv = kv_heads*64, F = intermediate. */
typedef struct tl_layer_capture {
  float* attn_input;          /* [S][hidden]  RMSNorm(x, input_norm)      attn_input_fp */
  int8_t* qkv_input_q;        /* [S][hidden]  INT8 input of q/k/v_proj */
  float* qkv_input_absmax;    /* [1] */
  int32_t* q_acc;             /* [S][Dq] */
  int32_t* k_acc;             /* [S][Dkv] */
  int32_t* v_acc;             /* [S][Dkv] */
  float* q_proj;              /* [S][Dq]  dequantized, before RoPE        q_proj_fp */
  float* k_proj;              /* [S][Dkv]                                k_proj_fp */
  float* v_proj;              /* [S][Dkv]                                v_proj_fp */
  float* scores;              /* [heads][S][S] Q.K^T/8, -1e9 above the diagonal  scores_fp */
  float* probs;               /* [heads][S][S] softmax(scores)            weights_fp */
  float* attended;            /* [S][Dq]  attention output                attended_fp */
  int8_t* o_input_q;          /* [S][Dq] */
  float* o_input_absmax;      /* [1] */
  int32_t* o_acc;             /* [S][hidden] */
  float* o_proj;              /* [S][hidden] dequantized o_proj output     attn out_fp */
  float* x_after_attn;        /* [S][hidden]                              x_after_attn_fp */
  float* ffn_input;           /* [S][hidden]  RMSNorm(x_after_attn, post_norm)  ffn_input_fp */
  int8_t* gate_up_input_q;    /* [S][hidden] */
  float* gate_up_input_absmax;/* [1] */
  int32_t* gate_acc;          /* [S][F] */
  int32_t* up_acc;            /* [S][F] */
  float* gate_proj;           /* [S][F]                                   gate_proj_fp */
  float* up_proj;             /* [S][F]                                   up_proj_fp */
  float* hidden;              /* [S][F]   silu(gate) * up                 hidden_fp */
  int8_t* down_input_q;       /* [S][F] */
  float* down_input_absmax;   /* [1] */
  int32_t* down_acc;          /* [S][hidden] */
  float* down_proj;           /* [S][hidden] dequantized down_proj output  ffn out_fp */
} tl_layer_capture;

/* One decoder layer on caller-given activations (teacher forcing):
 * mixed_precision_decoder_layer (model/tinyllama_gemm_int8.py:256-281) on the
 * n rows of host float32 x [n][hidden] as one sequence at positions 0..n-1,
 * run by the engine's prefill kernels for layer `layer`. K/V of those rows
 * are calibrated and written into KV slot `slot` of that layer (INT8, the
 * engine's cache). out (host [n][hidden], may be NULL) receives the layer
 * output; cap (may be NULL) the intermediate tensors. The slot's position
 * is not changed. TL_ERR_UNIMPLEMENTED on a tensor-parallel engine. */
TL_API tl_status tl_decoder_layer(tl_engine* eng, uint32_t slot, uint32_t layer, const float* x, uint32_t n,
                                  float* out, const tl_layer_capture* cap);

/* One decoder layer of a batched DECODE step on caller-given activations
 * (teacher forcing of the decode path, the KV-cached counterpart of
 * mixed_precision_decoder_layer, model/tinyllama_gemm_int8.py:256-281): row r
 * of host float32 x [n][hidden] is the new token at position positions[r] of
 * the sequence held in KV slot slots[r], whose cache already holds positions
 * 0..positions[r]-1 of this layer and their scales (a prefill of that slot).
 * Runs the engine's batched decode kernels for layer `layer` (tcgen05 GEMMs,
 * decode attention): the row's K/V is quantized with the frozen scales and
 * appended at positions[r]; attention reads positions 0..positions[r].
 * Each row is quantized on its own, so the *_input_absmax capture fields
 * receive n floats; scores/probs must be NULL. n must be in
 * [16, max_batch] (the tensor-core decode path) and the slots distinct.
 * The batched decode rows' device state (positions, active flags) is left
 * undefined: tl_generate_batch / tl_prefill_batch_device set it up again.
 * TL_ERR_UNIMPLEMENTED on a tensor-parallel engine. */
TL_API tl_status tl_decode_layer(tl_engine* eng, uint32_t layer, uint32_t n, const uint32_t* slots,
                                 const uint32_t* positions, const float* x, float* out, const tl_layer_capture* cap);

/* Device-resident decode step for benchmarks: runs `steps` captured decode
 * steps of the first n_seqs slots (greedy feedback on the device) and
 * returns without copying tokens to the host. */
TL_API tl_status tl_decode_steps_device(tl_engine* eng, uint32_t n_seqs, uint32_t steps);
TL_API tl_status tl_prefill_batch_device(tl_engine* eng, uint32_t n_seqs, const uint32_t* prompts,
                                  uint32_t n_prompt);
/* Rewinds rows 0..n_seqs-1 to `position` (KV rows at and beyond it will be
 * overwritten), re-arms them (active, zero emitted count, no stop) and keeps
 * each row's current input token. Lets a benchmark replay the same decode
 * span from one prefilled prompt state. Enqueued on the engine stream. */
TL_API tl_status tl_decode_rewind(tl_engine* eng, uint32_t n_seqs, uint32_t position);
TL_API tl_status tl_synchronize(tl_engine* eng);
/* Times each decode-step kernel kind in isolation with CUDA events on the
 * engine stream: [0] QKV projection, [1] attention (+RoPE), [2] O projection +
 * residual, [3] gate/up + SiLU*up, [4] down + residual, [5] LM head + argmax,
 * [6] RMSNorm+quantize rows, [7] quantize rows. For n_seqs = 1 the
 * projections are the dp4a GEMVs with the RMSNorm/quantize prologue fused
 * ([6], [7] = 0); for n_seqs >= 2 they are the tcgen05 GEMMs, launched as
 * the decode step launches them: once per row group (two concurrent groups
 * of n_seqs / 2 rows on two streams for n_seqs >= 48, each group's launches
 * back to back on its stream; the LM head once over all rows), so a time
 * covers all n_seqs rows. Each kind runs
 * `iters` back-to-back launches (no programmatic dependent launch) between
 * one event pair, layers cycled so weights come from HBM as in a real step;
 * the average includes each launch's start-up. The LM head (one matrix) is
 * timed per launch, each after an L2 flush outside the timed interval.
 * avg_ms_out receives 8 averages. The rows must have been prefilled
 * (tl_prefill_batch_device). */
TL_API tl_status tl_profile_decode_kernels(tl_engine* eng, uint32_t n_seqs, uint32_t iters,
                                           float* avg_ms_out);
/* Number of kernels one decode step of n_seqs rows launches. */
TL_API int32_t tl_decode_step_kernel_count_rows(tl_engine* eng, uint32_t n_seqs);
/* Number of concurrent row groups (streams) a decode step of n_seqs rows
 * runs: 2 for n_seqs >= 48 (groups of at least 24 rows; TL_DECODE_GROUPS=n
 * sets the most, up to 4), else 1; 0 for a NULL engine. */
TL_API int32_t tl_decode_row_groups(tl_engine* eng, uint32_t n_seqs);
/* Number of kernels one decode step launches (for launch accounting). */
TL_API int32_t tl_decode_step_kernel_count(tl_engine* eng);
TL_API void* tl_engine_stream(tl_engine* eng);

/* ------------------------------------------------------------- operators */
/* All operator entry points: device pointers, `stream` is a cudaStream_t
 * (NULL = legacy default stream). Shapes must satisfy K % 16 == 0 and
 * 16-byte aligned int8 rows. */

/* Waits for the device and reports TL_ERR_TIMEOUT if a tensor-core kernel
 * gave up on a bounded pipeline wait since the last call (then clears it). */
TL_API tl_status tl_device_error(void);

/* int8 W[K][N] -> W^T[N][K] (device to device). */
TL_API tl_status tl_transpose_i8(const int8_t* w_kn, int8_t* w_nk, int32_t K, int32_t N, void* stream);

/* quantize_int8 over groups of rows: rows [g*rows_per_group, (g+1)*rows_per_group)
 * share one scale. out_absmax[g] receives max|x| of the group (float32);
 * the scale is absmax/127 in float64 (1.0 when absmax == 0). */
TL_API tl_status tl_quantize_int8(const float* x, int32_t rows, int32_t cols, int32_t rows_per_group,
                           int8_t* out_q, float* out_absmax, void* stream);

/* shared GEMM: C[M][N] = A[M][K] (int8) x B (int8, given as W^T[N][K]) in int32. */
TL_API tl_status tl_gemm_i8(const int8_t* a, const int8_t* w_nk, int32_t* c, int32_t M, int32_t N,
                     int32_t K, void* stream);

/* shared GEMM + requantize_unit: out = clamp(RNE((acc * scale_q16) >> 16)).
 * scale_q16 has N entries when per_column != 0, else 1 entry. */
TL_API tl_status tl_gemm_i8_requant(const int8_t* a, const int8_t* w_nk, const uint32_t* scale_q16,
                             int32_t per_column, int32_t nonnegative_only, int8_t* out,
                             int32_t M, int32_t N, int32_t K, void* stream);

/* quantized_linear: quantize x per tensor (all M rows), int8 GEMM, dequantize
 * with float32(s_x * w_scale[n]). out[M][N] float32. acc_out (optional) int32. */
TL_API tl_status tl_quantized_linear(const float* x, const int8_t* w_nk, const double* w_scale,
                              float* out, int32_t* acc_out, int32_t M, int32_t N, int32_t K,
                              void* stream);

/* rms_norm, bit-exact with NumPy's float32 reduction order. */
TL_API tl_status tl_rmsnorm(const float* x, const float* gamma, float eps, float* out, int32_t rows,
                     int32_t cols, void* stream);

/* Final RMSNorm + per-row INT8 quantization + LM-head GEMV + argmax for `rows`
 * rows: token_out[r] = argmax (lowest id on ties); logits_out optional
 * [rows][vocab]. Each call allocates (and frees) its own reduction scratch. */
TL_API tl_status tl_lmhead_argmax(const float* x, const float* gamma, float eps, const int8_t* w_nk,
                           const double* w_scale, int32_t rows, int32_t vocab, int32_t hidden,
                           int32_t* token_out, float* logits_out, void* stream);

/* Decode attention for `rows` sequences at one layer over the INT8 KV cache
 * (device buffers): qkv [rows][(H + 2*Hkv)*64] float32 pre-RoPE q|k|v of the
 * new token, pos[rows] its position, slot[rows] its KV slot; kc/vc int8
 * [slots][L][Hkv][P][64], ks/vs float [slots][L][Hkv]; cos/sin [P][64].
 * Appends the new K (after RoPE) and V rows (quantized with the cached
 * scales) and writes out [rows][H*64]. Allocates its split scratch per call.
 * Follows model/tinyllama_gemm_int8.py:154-163 with the cache layout of
 * rtl/memory/kv_cache_manager.sv:43-47 and rtl/compute/gqa_router.sv:25-31. */
TL_API tl_status tl_attn_decode(const float* qkv, const int32_t* pos, const int32_t* slot, int8_t* kc,
                                int8_t* vc, const float* ks, const float* vs, const float* rope_cos,
                                const float* rope_sin, int32_t layer, int32_t num_layers, int32_t heads,
                                int32_t kv_heads, int32_t max_positions, int32_t rows, float* out,
                                void* stream);

/* Causal prefill attention of n_seqs sequences of seq_len tokens each over the
 * INT8 KV cache. Replaces the attention core of mixed_precision_self_attention
 * (model/tinyllama_gemm_int8.py:154-163: scores = Q.K^T / sqrt(64), causal
 * mask of model/tinyllama.py:90-91, softmax of :100-103, weighted sum of V)
 * with the cache rows of slot slot_base + i standing in for K and V.
 * qkv: fp32 [n_seqs * seq_len][(heads + 2 * kv_heads) * 64], Q already rotated
 * (RoPE); K/V are read from kc/vc ([slot][layer][kv_head][max_positions][64]
 * int8, scales ks/vs [slot][layer][kv_head]). out: fp32 [rows][heads * 64].
 * out_absmax (optional, one float per sequence, zero-initialised by the
 * caller) receives max |out| over the sequence (atomic max). */
TL_API tl_status tl_attn_prefill(const float* qkv, int32_t seq_len, int32_t n_seqs, const int8_t* kc,
                                 const int8_t* vc, const float* ks, const float* vs, int32_t slot_base,
                                 int32_t layer, int32_t num_layers, int32_t heads, int32_t kv_heads,
                                 int32_t max_positions, float* out, float* out_absmax, void* stream);

/* ---------------------------------------------------- contract mode (Q16.16)
 * The hardware's fixed-point path around its nonlinear blocks, as operators
 * on caller-owned device buffers: INT8 activations times a Q16.16 input
 * scale give Q16.16 core values, the block's float32 function runs on their
 * dequantized values (NumPy order, as the reference's float blocks), the
 * result goes back to Q16.16 (round half to even, saturated) and to INT8 by
 * integer division by the Q16.16 output scale (half to even on the
 * remainder, clamped to +-127). y_q16 / prob_q16 (optional) receive the
 * Q16.16 core outputs.
 *   tl_contract_rmsnorm  rtl/nonlinear/rmsnorm_wrapper.sv,
 *                        model/export_fpga_vectors.py:1705-1728 (per row of cols)
 *   tl_contract_silu     rtl/nonlinear/silu_wrapper.sv, :1896-1910
 *   tl_contract_softmax  rtl/nonlinear/softmax_wrapper.sv:23, :1808-1829, :874-888:
 *                        INT32 scores x Q16.16 scale (saturating), float32
 *                        softmax per row (cols <= 128), INT8 probabilities
 *                        p * 127 >> 16 in [0, 127] (the 1/127 probability scale)
 *   tl_contract_rope     rtl/compute/rope_unit.sv:73-127, :684-732: INT8 rows
 *                        [rows][64] with per-row Q16.16 cos/sin tables [rows][64]
 *   tl_residual_add_i32  rtl/compute/residual_add.sv:92-96: unsaturated INT32
 *                        add (modulo 2^32) of Q16.16 residual and update */
TL_API tl_status tl_contract_rmsnorm(const int8_t* x_q, int32_t rows, int32_t cols, uint32_t in_scale_q16,
                                     const int32_t* gamma_q16, float eps, uint32_t out_scale_q16, int8_t* y_q,
                                     int32_t* y_q16, void* stream);
TL_API tl_status tl_contract_silu(const int8_t* x_q, int64_t n, uint32_t in_scale_q16, uint32_t out_scale_q16,
                                  int8_t* y_q, int32_t* y_q16, void* stream);
TL_API tl_status tl_contract_softmax(const int32_t* scores, int32_t rows, int32_t cols, uint32_t score_scale_q16,
                                     int8_t* prob_q, int32_t* prob_q16, void* stream);
TL_API tl_status tl_contract_rope(const int8_t* x_q, const int32_t* cos_q16, const int32_t* sin_q16, int32_t rows,
                                  int8_t* out, void* stream);
TL_API tl_status tl_residual_add_i32(const int32_t* residual_q16, const int32_t* update_q16, int32_t* out, int64_t n,
                                     void* stream);

/* tl_lmhead_argmax for callers that must not have a library allocate GPU
 * memory -- a serving runtime that reserves the whole device at start-up and
 * accounts for every byte, or a framework whose own caching allocator has to
 * own all device memory. No counterpart in the reference (its argmax reduces
 * in FPGA registers). Same arguments and results as tl_lmhead_argmax, but the
 * cross-CTA reduction scratch is one fixed array inside the library (64 KiB +
 * 256 B, held on every GPU that loads the library until the process exits)
 * and the call makes no cudaMalloc/cudaFree. Limit: rows <=
 * TL_LMHEAD_NOALLOC_MAX_ROWS, larger batches get TL_ERR_OUT_OF_RANGE. The
 * first call on a device looks up the array's device address (make that
 * first call before any stream capture). All calls share the one array: two
 * calls that overlap on the GPU (other streams, other host threads) race, so
 * the caller serializes them. */
#define TL_LMHEAD_NOALLOC_MAX_ROWS 8
TL_API tl_status tl_lmhead_argmax_noalloc(const float* x, const float* gamma, float eps, const int8_t* w_nk,
                                          const double* w_scale, int32_t rows, int32_t vocab,
                                          int32_t hidden, int32_t* token_out, float* logits_out,
                                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TL_API_H */
