// noalloc.cu -- an LM-head + argmax entry point that allocates no device memory.
//
// tl_lmhead_argmax reduces the per-CTA argmax candidates of its LM-head GEMV
// through scratch memory that it allocates and frees on every call. Some
// callers cannot let a library do that: a serving runtime that reserves the
// whole GPU at start-up and accounts for every byte (an allocation from
// inside a library either fails against that budget or escapes its
// accounting), or an embedding framework whose own caching allocator must own
// all device memory. For them this file keeps the reduction scratch in one
// fixed array compiled into the library and launches the same kernel
// (gemv_kernel, RMSNorm prologue + argmax epilogue) with pointers into it.
//
// The array is file-scope device memory: every GPU on which the library is
// loaded holds it (64 KiB + 256 B) until the process exits. Host code must
// not use the array's name as a device address; its address on each device
// is looked up once with cudaGetSymbolAddress, with that device current.
#include <mutex>

#include "../../include/tl_api.h"
#include "kernels.cuh"

using namespace tl;

namespace {

constexpr int kMaxRows = TL_LMHEAD_NOALLOC_MAX_ROWS;  // rows of one call
constexpr int kMaxCtas = kGemvMaxGrid;               // bound on the GEMV grid (one CTA per SM)
constexpr int kCandidates = kMaxCtas * kMaxRows;     // per-CTA, per-row argmax keys
constexpr int kTicketWords = 32;                     // 256 bytes: the kernel's completion ticket
// One row block (8 rows) means one ticket word; the candidates cover every
// CTA the GEMV launcher may start for every row of a call.
static_assert(kMaxRows <= 8, "the argmax kernel keeps one ticket per 8-row block");
static_assert(kCandidates >= kGemvMaxGrid * kMaxRows, "candidate scratch smaller than the GEMV grid bound");

// [0, kCandidates): packed (logit, token) keys; then the ticket counter.
static __device__ __align__(256) unsigned long long g_lmhead_scratch[kCandidates + kTicketWords];

std::mutex g_setup_mutex;
void* g_scratch_ptr[64] = {nullptr};

// Device address of g_lmhead_scratch on the current device, looked up once.
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_lmhead_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

tl_status cu(cudaError_t e) { return e == cudaSuccess ? TL_OK : TL_ERR_CUDA; }

}  // namespace

extern "C" {

tl_status tl_lmhead_argmax_noalloc(const float* x, const float* gamma, float eps, const int8_t* w_nk,
                                   const double* w_scale, int32_t rows, int32_t vocab, int32_t hidden,
                                   int32_t* token_out, float* logits_out, void* stream) {
  if (!x || !gamma || !w_nk || !w_scale || !token_out) return TL_ERR_INVALID_ARGUMENT;
  if (rows > kMaxRows) return TL_ERR_OUT_OF_RANGE;  // beyond the fixed scratch
  if (rows <= 0 || vocab <= 0 || hidden <= 0 || hidden % 16) return TL_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(w_nk) & 15u))
    return TL_ERR_INVALID_ARGUMENT;
  NormPlan plan;
  if (!norm_plan(hidden, &plan)) return TL_ERR_INVALID_ARGUMENT;
  if (gemv_argmax_partials(rows, vocab) > static_cast<size_t>(kCandidates)) return TL_ERR_OUT_OF_RANGE;
  if (prepare_kernels(hidden) != cudaSuccess) return TL_ERR_CUDA;
  void* base = nullptr;
  if (scratch_address(&base) != cudaSuccess) return TL_ERR_CUDA;
  unsigned long long* candidates = static_cast<unsigned long long*>(base);
  unsigned int* ticket = reinterpret_cast<unsigned int*>(candidates + kCandidates);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The ticket must start at zero (the kernel leaves it at zero, but an
  // earlier failed launch may not have); the candidates are fully rewritten.
  tl_status st = cu(cudaMemsetAsync(ticket, 0, kTicketWords * sizeof(unsigned long long), s));
  if (st != TL_OK) return st;
  GemvArgs g;
  g.x_f32 = x; g.gamma = gamma; g.eps = eps; g.w = w_nk; g.w_scale = w_scale;
  g.M = rows; g.N = vocab; g.K = hidden; g.logits = logits_out;
  g.am_partial = candidates; g.am_counter = ticket; g.am_token = token_out;
  return cu(launch_gemv(PRO_NORM, EPI_ARGMAX, g, s, false));
}

}  // extern "C"
