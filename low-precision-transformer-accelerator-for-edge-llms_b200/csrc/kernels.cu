// kernels.cu -- sm_100a CUDA-core kernels of the TinyLlama INT8 hot path.
//
//  * gemv_kernel: the decode-path INT8 GEMV (M <= 8 rows per CTA row block),
//    128-bit streaming weight loads, dp4a, warp-shuffle reduction, with a
//    fused activation prologue (RMSNorm + per-row INT8 quantization) and fused
//    epilogues (dequant, residual add, SiLU*up, Q16.16 requant, LM-head
//    argmax). Reference units: shared_gemm_engine.sv:127-168,
//    requantize_unit.sv:39-93, residual_add.sv:92-96, elementwise_mul.sv:112-119,
//    argmax_reduction.sv:47-131; numerics of quantized_linear
//    (model/tinyllama_gemm_int8.py:59-88).
//  (decode attention on tensor cores lives in attention.cu)
//  * prefill helpers: RMSNorm rows, quantize rows, RoPE + KV calibration, KV
//    write, causal attention.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdio>

#include "common.cuh"
#include "kernels.cuh"

namespace tl {

// ============================================================ row helpers
struct RowScratch {
  float part[1024 * 8];
  float leaf[1024];
  float red[32];
};
// Only the used prefix of RowScratch is allocated: n_leaves*8 + n_leaves + 32
// floats (rs_floats()).
static inline size_t rs_floats(const NormPlan& p) { return static_cast<size_t>(p.n_leaves) * 9 + 32; }

struct RowScratchView {
  float* part;
  float* leaf;
  float* red;
};
TL_DEV RowScratchView rs_view(float* base, NormPlan p) {
  return {base, base + p.n_leaves * 8, base + p.n_leaves * 9};
}

// In-place RMSNorm of buf[0..K) by the whole block:
// buf = (buf * (1/sqrt(mean(buf^2) + eps))) * gamma  (model/tinyllama.py:45-50),
// mean of squares in NumPy's float32 reduction order.
TL_DEV void block_rmsnorm(float* buf, int K, const float* gamma, float eps, NormPlan plan,
                          RowScratchView rs) {
  const float tot = block_sumsq_numpy(buf, plan, rs.part, rs.leaf);
  const float mean = __fdiv_rn(tot, static_cast<float>(K));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  for (int i = threadIdx.x; i < K; i += blockDim.x) buf[i] = __fmul_rn(__fmul_rn(buf[i], inv), gamma[i]);
  __syncthreads();
}

TL_DEV float block_absmax(const float* buf, int K, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float m = 0.0f;
  for (int i = tid; i < K; i += blockDim.x) m = fmaxf(m, fabsf(buf[i]));
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  float v = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.0f;
  v = warp_max(v);
  __syncthreads();
  return v;
}

// ================================================================ the GEMV
// Persistent over output-row groups: each warp owns kGemvRW weight rows at a
// time and walks (row group, K chunk) work items with the next item's 16-byte
// weight loads in flight while the current one is reduced. The first item's
// loads are issued before griddepcontrol.wait, so under programmatic
// dependent launch they overlap the previous kernel's tail. The activation
// prologue (RMSNorm, per-row INT8 quantization) runs once per CTA.
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvRW = 2;   // weight rows per warp item
constexpr int kGemvU = 4;    // 16-byte chunks per lane per row per item
static int g_num_sms[64] = {0};


TL_DEV float silu_mul(float g, float u) {
  // model/tinyllama.py:159-161: x / (1 + exp(-clip(x, -60, 60))), then * up
  float c = fminf(fmaxf(g, -60.0f), 60.0f);
  float den = __fadd_rn(1.0f, expf(-c));
  return __fmul_rn(__fdiv_rn(g, den), u);
}

__host__ __device__ constexpr int align16(int x) { return (x + 15) & ~15; }
__host__ __device__ constexpr int gemv_off_sx(int MR, int K) { return MR * K; }
__host__ __device__ constexpr int gemv_off_am(int MR, int K) { return gemv_off_sx(MR, K) + align16(8 * MR); }
__host__ __device__ constexpr int gemv_off_f(int MR, int K) {
  return gemv_off_am(MR, K) + align16(8 * kGemvWarps * MR);
}

template <int MR>
struct GemvItem {
  int4 w[kGemvU][kGemvRW];
};

template <int PRO, int EPI, int MR>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int K = a.K, N = a.N, M = a.M;
  // 16-byte aligned carve-up: xs [MR][K] | sx64 [MR] | am [warps][MR] | fbuf [K] | norm scratch
  int8_t* xs = reinterpret_cast<int8_t*>(smem);
  double* sx64 = reinterpret_cast<double*>(smem + gemv_off_sx(MR, K));
  unsigned long long* am = reinterpret_cast<unsigned long long*>(smem + gemv_off_am(MR, K));
  float* fbuf = reinterpret_cast<float*>(smem + gemv_off_f(MR, K));
  RowScratchView rs = rs_view(fbuf + K, a.norm);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.y * MR;
  const int mr = min(MR, M - m0);
  const int K16 = K >> 4;
  const int nch = (K16 + 32 * kGemvU - 1) / (32 * kGemvU);
  const int groups = (N + kGemvRW - 1) / kGemvRW;
  const int gstride = gridDim.x * kGemvWarps;

  auto load_item = [&](GemvItem<MR>& it, int g, int c) {
#pragma unroll
    for (int i = 0; i < kGemvRW; ++i) {
      const int n = g * kGemvRW + i;
      const int4* wp = reinterpret_cast<const int4*>(a.w + static_cast<size_t>(n < N ? n : 0) * K);
#pragma unroll
      for (int u = 0; u < kGemvU; ++u) {
        const int col = c * 32 * kGemvU + lane + 32 * u;
        it.w[u][i] = (n < N && col < K16) ? ld_stream_v4(wp + col) : make_int4(0, 0, 0, 0);
      }
    }
  };

  // ---- 1. first work item's weights in flight before anything else
  int g = blockIdx.x * kGemvWarps + warp;
  int c = 0;
  GemvItem<MR> cur, nxt;
  if (g < groups) load_item(cur, g, 0);

  // ---- 2. activation prologue (depends on the previous kernel)
  pdl_wait();
  if (PRO == PRO_Q8) {
    for (int r = 0; r < MR; ++r) {
      int4* dst = reinterpret_cast<int4*>(xs + r * K);
      if (r < mr) {
        const int4* src = reinterpret_cast<const int4*>(a.x_q + static_cast<size_t>(m0 + r) * K);
        for (int q = tid; q < K16; q += kGemvThreads) dst[q] = src[q];
      } else {
        for (int q = tid; q < K16; q += kGemvThreads) dst[q] = make_int4(0, 0, 0, 0);
      }
      if (tid == 0)
        sx64[r] = quant_scale64((r < mr && a.in_absmax) ? a.in_absmax[(m0 + r) / a.rows_per_group] : 0.0f);
    }
  } else {
    for (int r = 0; r < MR; ++r) {
      if (r >= mr) {
        int4* dst = reinterpret_cast<int4*>(xs + r * K);
        for (int q = tid; q < K16; q += kGemvThreads) dst[q] = make_int4(0, 0, 0, 0);
        if (tid == 0) sx64[r] = 1.0;
        continue;
      }
      const float4* src = reinterpret_cast<const float4*>(
          a.x_f32 + (static_cast<size_t>(a.x_row_offset) + static_cast<size_t>(m0 + r) * a.x_row_step) * K);
      for (int q = tid; q < (K >> 2); q += kGemvThreads) reinterpret_cast<float4*>(fbuf)[q] = src[q];
      __syncthreads();
      if (PRO == PRO_NORM) block_rmsnorm(fbuf, K, a.gamma, a.eps, a.norm, rs);
      float amax;
      if (PRO == PRO_F32_GIVEN) amax = a.in_absmax[(m0 + r) / a.rows_per_group];
      else amax = block_absmax(fbuf, K, rs.red);
      const double s64 = quant_scale64(amax);
      const float sf = static_cast<float>(s64);
      int8_t* dst = xs + r * K;
      for (int i = tid; i < K; i += kGemvThreads) dst[i] = static_cast<int8_t>(quantize_one(fbuf[i], sf));
      if (tid == 0) sx64[r] = s64;
      __syncthreads();
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  // ---- 3. work items: dot products + epilogue per completed row group
  int acc[kGemvRW][MR];
#pragma unroll
  for (int i = 0; i < kGemvRW; ++i)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[i][m] = 0;
  unsigned long long best[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) best[m] = 0ull;

  auto compute = [&](const GemvItem<MR>& it, int cc) {
#pragma unroll
    for (int u = 0; u < kGemvU; ++u) {
      const int col = cc * 32 * kGemvU + lane + 32 * u;
      if (col < K16) {
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const int4 xv = reinterpret_cast<const int4*>(xs + m * K)[col];
#pragma unroll
          for (int i = 0; i < kGemvRW; ++i) {
            int t = acc[i][m];
            t = dp4a(it.w[u][i].x, xv.x, t);
            t = dp4a(it.w[u][i].y, xv.y, t);
            t = dp4a(it.w[u][i].z, xv.z, t);
            t = dp4a(it.w[u][i].w, xv.w, t);
            acc[i][m] = t;
          }
        }
      }
    }
  };

  auto epilogue = [&](int gg) {
#pragma unroll
    for (int i = 0; i < kGemvRW; ++i)
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[i][m] = warp_sum_i(acc[i][m]);
    if (lane == 0) {
      const int n0 = gg * kGemvRW;
      if (EPI == EPI_ARGMAX) {
#pragma unroll
        for (int i = 0; i < kGemvRW; ++i) {
          const int n = n0 + i;
          if (n >= N) continue;
          const double sw = a.w_scale[n];
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            if (m >= mr) continue;
            const float y = dequant(acc[i][m], sx64[m], sw);
            if (a.logits) a.logits[static_cast<size_t>(m0 + m) * N + n] = y;
            const unsigned long long k = argmax_key(y, n);
            best[m] = k > best[m] ? k : best[m];
          }
        }
      } else if (EPI == EPI_SILU) {
        if (n0 < N) {
          const int j = n0 >> 1, Nh = N >> 1;
          const double sg = a.w_scale[n0], su = a.w_scale[n0 + 1];
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            if (m >= mr) continue;
            const float gv = dequant(acc[0][m], sx64[m], sg);
            const float uv = dequant(acc[1][m], sx64[m], su);
            const float hv = silu_mul(gv, uv);
            a.out_f32[static_cast<size_t>(m0 + m) * Nh + j] = hv;
            if (a.out_absmax) atomic_max_nonneg(a.out_absmax + (m0 + m) / a.rows_per_group, fabsf(hv));
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < kGemvRW; ++i) {
          const int n = n0 + i;
          if (n >= N) continue;
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            if (m >= mr) continue;
            const size_t o = static_cast<size_t>(m0 + m) * N + n;
            if (EPI == EPI_I32) {
              a.out_i32[o] = acc[i][m];
            } else if (EPI == EPI_REQ) {
              const uint32_t sc = a.req_scale[a.req_per_col ? n : 0];
              a.out_i8[o] = static_cast<int8_t>(requant_q16(acc[i][m], sc, a.req_nonneg != 0));
            } else {
              const float y = dequant(acc[i][m], sx64[m], a.w_scale[n]);
              const float v = (EPI == EPI_RESID) ? __fadd_rn(a.resid[o], y) : y;
              a.out_f32[o] = v;
              if (EPI == EPI_F32 && a.out_absmax)
                atomic_max_nonneg(a.out_absmax + (m0 + m) / a.rows_per_group, fabsf(v));
            }
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kGemvRW; ++i)
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[i][m] = 0;
  };

  // ping-pong between two register buffers, prefetching one item ahead
  while (g < groups) {
    {
      int gn = g, cn = c + 1;
      if (cn == nch) { cn = 0; gn = g + gstride; }
      if (gn < groups) load_item(nxt, gn, cn);
      compute(cur, c);
      if (c == nch - 1) epilogue(g);
      g = gn;
      c = cn;
    }
    if (g >= groups) break;
    {
      int gn = g, cn = c + 1;
      if (cn == nch) { cn = 0; gn = g + gstride; }
      if (gn < groups) load_item(cur, gn, cn);
      compute(nxt, c);
      if (c == nch - 1) epilogue(g);
      g = gn;
      c = cn;
    }
  }

  if (EPI == EPI_ARGMAX) {
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < MR; ++m) am[warp * MR + m] = best[m];
    }
    __syncthreads();
    if (tid < mr) {
      unsigned long long b = 0ull;
      for (int w = 0; w < kGemvWarps; ++w) b = am[w * MR + tid] > b ? am[w * MR + tid] : b;
      a.am_partial[static_cast<size_t>(blockIdx.x) * M + m0 + tid] = b;
    }
    __threadfence();
    __syncthreads();
    __shared__ int is_last;
    if (tid == 0) {
      unsigned int prev = atomicAdd(a.am_counter + blockIdx.y, 1u);
      is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      if (tid < mr) {
        unsigned long long b = 0ull;
        for (unsigned int bx = 0; bx < gridDim.x; ++bx) {
          const unsigned long long v = *reinterpret_cast<volatile unsigned long long*>(
              a.am_partial + static_cast<size_t>(bx) * M + m0 + tid);
          b = v > b ? v : b;
        }
        a.am_token[m0 + tid] = argmax_key_index(b);
      }
      if (tid == 0) a.am_counter[blockIdx.y] = 0u;
    }
  }
}

static size_t gemv_smem_bytes(int MR, int K, const NormPlan& plan) {
  return static_cast<size_t>(gemv_off_f(MR, K)) + 4 * static_cast<size_t>(K) + 4 * rs_floats(plan) + 64;
}
static NormPlan plan_or_min(int K) {
  NormPlan p{8, 1};
  if (!norm_plan(K, &p)) p = NormPlan{8, 1};
  return p;
}

static int gemv_grid_x(int N, int MR) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = (dev >= 0 && dev < 64 && g_num_sms[dev] > 0) ? g_num_sms[dev] : 148;
  const int groups = (N + kGemvRW - 1) / kGemvRW;
  const int need = (groups + kGemvWarps - 1) / kGemvWarps;
  // One CTA per SM (8 warps, two work items in flight each) saturates HBM and
  // leaves room on every SM for the next kernel's CTA to start streaming its
  // weights early under programmatic dependent launch.
  (void)MR;
  return std::max(1, std::min(std::min(need, sms), kGemvMaxGrid));
}

size_t gemv_argmax_partials(int M, int N) {
  (void)N;
  return static_cast<size_t>(kGemvMaxGrid) * M;
}
int gemv_argmax_row_blocks(int M) { return (M + 7) / 8; }

template <int PRO, int EPI, int MR>
static cudaError_t launch_gemv_t(const GemvArgs& a0, cudaStream_t s, bool pdl) {
  GemvArgs a = a0;
  if (PRO == PRO_NORM) {
    if (!norm_plan(a.K, &a.norm)) return cudaErrorInvalidValue;
  } else {
    a.norm = plan_or_min(a.K);
  }
  const size_t smem = gemv_smem_bytes(MR, a.K, a.norm);
  auto kfn = gemv_kernel<PRO, EPI, MR>;
  dim3 grid(gemv_grid_x(a.N, MR), (a.M + MR - 1) / MR);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kfn, a);
}

template <int PRO, int EPI, int MR>
static cudaError_t prepare_gemv_t(int max_k) {
  return cudaFuncSetAttribute(gemv_kernel<PRO, EPI, MR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(gemv_smem_bytes(MR, max_k, NormPlan{128, 64})));
}

template <int PRO, int EPI>
static cudaError_t launch_gemv_mr(const GemvArgs& a, cudaStream_t s, bool pdl) {
  if (a.M <= 1) return launch_gemv_t<PRO, EPI, 1>(a, s, pdl);
  if (a.M <= 2) return launch_gemv_t<PRO, EPI, 2>(a, s, pdl);
  if (a.M <= 4) return launch_gemv_t<PRO, EPI, 4>(a, s, pdl);
  return launch_gemv_t<PRO, EPI, 8>(a, s, pdl);
}

template <int PRO, int EPI>
static cudaError_t prepare_gemv_mr(int max_k) {
  cudaError_t e;
  if ((e = prepare_gemv_t<PRO, EPI, 1>(max_k)) != cudaSuccess) return e;
  if ((e = prepare_gemv_t<PRO, EPI, 2>(max_k)) != cudaSuccess) return e;
  if ((e = prepare_gemv_t<PRO, EPI, 4>(max_k)) != cudaSuccess) return e;
  return prepare_gemv_t<PRO, EPI, 8>(max_k);
}

#define TL_GEMV_VARIANTS(X)        \
  X(PRO_Q8, EPI_I32)               \
  X(PRO_Q8, EPI_F32)               \
  X(PRO_Q8, EPI_RESID)             \
  X(PRO_Q8, EPI_SILU)              \
  X(PRO_Q8, EPI_REQ)               \
  X(PRO_NORM, EPI_F32)             \
  X(PRO_NORM, EPI_SILU)            \
  X(PRO_NORM, EPI_ARGMAX)          \
  X(PRO_F32, EPI_RESID)            \
  X(PRO_F32, EPI_F32)              \
  X(PRO_F32_GIVEN, EPI_ARGMAX)

cudaError_t launch_gemv(int pro, int epi, const GemvArgs& a, cudaStream_t s, bool pdl) {
  if (a.K % 16 != 0 || a.K <= 0 || a.N <= 0 || a.M <= 0) return cudaErrorInvalidValue;
  if (epi == EPI_SILU && (a.N % 2 != 0)) return cudaErrorInvalidValue;
#define TL_GEMV_CASE(P, E) \
  if (pro == P && epi == E) return launch_gemv_mr<P, E>(a, s, pdl);
  TL_GEMV_VARIANTS(TL_GEMV_CASE)
#undef TL_GEMV_CASE
  return cudaErrorInvalidValue;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (g_num_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    g_num_sms[dev] = n;
  }
  return g_num_sms[dev];
}

static size_t rmsnorm_rows_smem(int D);
__global__ void rmsnorm_rows_kernel(const float*, const float*, float, float*, float*, int, int, NormPlan);

cudaError_t prepare_kernels(int max_k) {
  static int prepared_k[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (max_k <= prepared_k[dev]) return cudaSuccess;
  if (g_num_sms[dev] == 0) {
    e = cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
#define TL_GEMV_PREP(P, E) \
  if ((e = prepare_gemv_mr<P, E>(max_k)) != cudaSuccess) return e;
  TL_GEMV_VARIANTS(TL_GEMV_PREP)
#undef TL_GEMV_PREP
  e = cudaFuncSetAttribute(rmsnorm_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(rmsnorm_rows_smem(max_k)));
  if (e != cudaSuccess) return e;
  if ((e = prepare_tc()) != cudaSuccess) return e;
  if ((e = attn_prepare()) != cudaSuccess) return e;
  prepared_k[dev] = max_k;
  return cudaSuccess;
}

// ================================================================= prefill
__global__ void embed_kernel(const float* table, const int* ids, float* x, int D, int vocab) {
  pdl_wait();
  const int r = blockIdx.x;
  int id = ids[r];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  const float4* src = reinterpret_cast<const float4*>(table + static_cast<size_t>(id) * D);
  float4* dst = reinterpret_cast<float4*>(x + static_cast<size_t>(r) * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = src[i];
  pdl_launch_dependents();
}

cudaError_t launch_embed(const float* table, const int* ids, float* x, int rows, int D, int vocab,
                         cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_kernel, table, ids, x, D, vocab);
}

static size_t rmsnorm_rows_smem(int D) {
  return 4 * static_cast<size_t>(D) + 4 * rs_floats(NormPlan{128, 64}) + 16;
}

__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* x, const float* gamma, float eps,
                                                           float* out, float* absmax, int D,
                                                           int rows_per_group, NormPlan plan) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* buf = reinterpret_cast<float*>(smem);
  RowScratchView rs = rs_view(buf + D, plan);
  const int r = blockIdx.x;
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) reinterpret_cast<float4*>(buf)[i] = src[i];
  __syncthreads();
  block_rmsnorm(buf, D, gamma, eps, plan, rs);
  float4* dst = reinterpret_cast<float4*>(out + static_cast<size_t>(r) * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = reinterpret_cast<float4*>(buf)[i];
  if (absmax) {
    const float m = block_absmax(buf, D, rs.red);
    if (threadIdx.x == 0) atomic_max_nonneg(absmax + r / rows_per_group, m);
  }
}

cudaError_t launch_rmsnorm_rows(const float* x, const float* gamma, float eps, float* out,
                                float* absmax_groups, int rows, int D, int rows_per_group,
                                cudaStream_t s) {
  NormPlan plan;
  if (!norm_plan(D, &plan) || D % 4) return cudaErrorInvalidValue;
  rmsnorm_rows_kernel<<<rows, 256, rmsnorm_rows_smem(D), s>>>(x, gamma, eps, out, absmax_groups, D,
                                                                rows_per_group, plan);
  return cudaGetLastError();
}

static cudaLaunchConfig_t row_cfg(int rows, int threads, size_t smem, cudaStream_t s, bool pdl,
                                   cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

__global__ void __launch_bounds__(256) norm_quant_rows_kernel(const float* x, const float* gamma, float eps,
                                                              int D, NormPlan plan, int8_t* out_q,
                                                              float* out_absmax, float* zero_rows) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* buf = reinterpret_cast<float*>(smem);
  RowScratchView rs = rs_view(buf + D, plan);
  const int r = blockIdx.x;
  pdl_wait();
  if (threadIdx.x == 0 && zero_rows) zero_rows[r] = 0.0f;
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) reinterpret_cast<float4*>(buf)[i] = src[i];
  __syncthreads();
  block_rmsnorm(buf, D, gamma, eps, plan, rs);
  const float amax = block_absmax(buf, D, rs.red);
  pdl_launch_dependents();
  const float sf = static_cast<float>(quant_scale64(amax));
  int8_t* dst = out_q + static_cast<size_t>(r) * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) dst[i] = static_cast<int8_t>(quantize_one(buf[i], sf));
  if (threadIdx.x == 0) out_absmax[r] = amax;
}

// RMSNorm + INT8 quantization, one 128-thread CTA per row, for rows whose
// NumPy reduction tree has 16 leaves of 128 elements (D = 2048). Thread t
// owns accumulator j = t & 7 of leaf l = t >> 3 and sums its 16 squares
// x[128 l + j + 8 k], k = 0..15, in order (block_sumsq_numpy's inner loop);
// the leaf's accumulators fold ((r0 + r1) + (r2 + r3)) + ((r4 + r5) +
// (r6 + r7)) by XOR shuffles 1, 2, 4 among its eight lanes, the four leaves
// of a warp pair up by shuffles 8 and 16, and the four warp sums combine as
// (w0 + w1) + (w2 + w3) -- the same additions as the tree (float addition is
// commutative, so which partner adds is immaterial). All row elements stay
// in registers: one memory round trip, two CTA barriers.
// Loads thread t's 16 elements of a D = 2048 row (layout above), returns
// the row's 1 / rms in every thread and leaves v[k] = x * inv * gamma with
// gamma's elements `gm` (loaded by the caller, ahead of any dependency wait).
// `red` is four floats of shared scratch; one CTA barrier.
TL_DEV float d2048_norm_regs(const float* xrow, const float (&gm)[16], float eps, float (&v)[16], float* red) {
  constexpr int D = 2048;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* xr = xrow + (t >> 3) * 128 + (t & 7);
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = xr[8 * k];
  float acc = __fmul_rn(v[0], v[0]);
#pragma unroll
  for (int k = 1; k < 16; ++k) acc = __fadd_rn(acc, __fmul_rn(v[k], v[k]));
#pragma unroll
  for (int st = 1; st < 32; st *= 2) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, st));
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  const float tot = __fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3]));
  const float mean = __fdiv_rn(tot, static_cast<float>(D));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = __fmul_rn(__fmul_rn(v[k], inv), gm[k]);
  return inv;
}

// Maximum of |v[k]| over the CTA's 128 threads (one CTA barrier).
TL_DEV float d2048_absmax(const float (&v)[16], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float m = 0.0f;
#pragma unroll
  for (int k = 0; k < 16; ++k) m = fmaxf(m, fabsf(v[k]));
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  return fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
}

TL_DEV uint32_t quant_pack4(float4 v, float sf) {
  return (static_cast<uint32_t>(quantize_one(v.x, sf)) & 0xffu) |
         ((static_cast<uint32_t>(quantize_one(v.y, sf)) & 0xffu) << 8) |
         ((static_cast<uint32_t>(quantize_one(v.z, sf)) & 0xffu) << 16) |
         ((static_cast<uint32_t>(quantize_one(v.w, sf)) & 0xffu) << 24);
}
// the same four results from quantize_one_inv (inv = quant_inv(sf)): for
// the throughput-bound prefill passes; in the latency-bound decode row
// kernels the one serial reciprocal costs more than the divisions it saves
// (64-row step 1.070-1.087 vs 1.053-1.057 ms)
TL_DEV uint32_t quant_pack4_inv(float4 v, float sf, float inv) {
  return (static_cast<uint32_t>(quantize_one_inv(v.x, sf, inv)) & 0xffu) |
         ((static_cast<uint32_t>(quantize_one_inv(v.y, sf, inv)) & 0xffu) << 8) |
         ((static_cast<uint32_t>(quantize_one_inv(v.z, sf, inv)) & 0xffu) << 16) |
         ((static_cast<uint32_t>(quantize_one_inv(v.w, sf, inv)) & 0xffu) << 24);
}

__global__ void __launch_bounds__(128) norm_quant_rows_d2048_kernel(const float* x, const float* gamma,
                                                                     float eps, int8_t* out_q,
                                                                     float* out_absmax, float* zero_rows) {
  constexpr int D = 2048;
  __shared__ float red[2][4];
  const int r = blockIdx.x, t = threadIdx.x;
  const int base = (t >> 3) * 128 + (t & 7);
  float gm[16], v[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) gm[k] = gamma[base + 8 * k];
  // Only gamma (constant) is read before the wait, so the dependent GEMM may
  // launch now and stream its weights while this kernel waits and runs.
  pdl_launch_dependents();
  pdl_wait();
  if (t == 0 && zero_rows) zero_rows[r] = 0.0f;
  d2048_norm_regs(x + static_cast<size_t>(r) * D, gm, eps, v, red[0]);
  const float m = d2048_absmax(v, red[1]);
  const float sf = static_cast<float>(quant_scale64(m));
  int8_t* dst = out_q + static_cast<size_t>(r) * D + base;
#pragma unroll
  for (int k = 0; k < 16; ++k) dst[8 * k] = static_cast<int8_t>(quantize_one(v[k], sf));
  if (t == 0) out_absmax[r] = m;
}

// Prefill RMSNorm + per-sequence INT8 quantization of D = 2048 rows in two
// passes that never store the float normalized rows. Pass 1 evaluates each
// row's 1 / rms (the tree above) and folds max |x * inv * gamma| into its
// sequence's absmax; pass 2 recomputes the same two roundings from the same
// x, inv and gamma (so the values are bit-identical) and quantizes them with
// the sequence scale. Bytes: 8 KB read per row, then 8 KB read + 2 KB written.
__global__ void __launch_bounds__(128) norm_stats_rows_d2048_kernel(const float* x, const float* gamma,
                                                                     float eps, float* inv_out, float* absmax,
                                                                     int rows_per_group) {
  constexpr int D = 2048;
  __shared__ float red[2][4];
  const int r = blockIdx.x, t = threadIdx.x;
  const int base = (t >> 3) * 128 + (t & 7);
  float gm[16], v[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) gm[k] = gamma[base + 8 * k];
  const float inv = d2048_norm_regs(x + static_cast<size_t>(r) * D, gm, eps, v, red[0]);
  const float m = d2048_absmax(v, red[1]);
  if (t == 0) {
    inv_out[r] = inv;
    atomic_max_nonneg(absmax + r / rows_per_group, m);
  }
}

__global__ void __launch_bounds__(128) norm_quant_apply_d2048_kernel(const float* x, const float* gamma,
                                                                      const float* inv, const float* absmax,
                                                                      int rows_per_group, int8_t* out_q) {
  constexpr int D = 2048;
  const int r = blockIdx.x, t = threadIdx.x;
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * D);
  float4 v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = src[t + 128 * i];
  const float iv = inv[r];
  const float sf = static_cast<float>(quant_scale64(absmax[r / rows_per_group])), rsf = quant_inv(sf);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  uint32_t* dst = reinterpret_cast<uint32_t*>(out_q + static_cast<size_t>(r) * D);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 g = g4[t + 128 * i];
    float4 y;
    y.x = __fmul_rn(__fmul_rn(v[i].x, iv), g.x);
    y.y = __fmul_rn(__fmul_rn(v[i].y, iv), g.y);
    y.z = __fmul_rn(__fmul_rn(v[i].z, iv), g.z);
    y.w = __fmul_rn(__fmul_rn(v[i].w, iv), g.w);
    dst[t + 128 * i] = quant_pack4_inv(y, sf, rsf);
  }
}

cudaError_t launch_norm_quant_prefill(const float* x, const float* gamma, float eps, int rows, int D,
                                      int rows_per_group, float* inv_buf, float* absmax_groups, float* h_buf,
                                      int8_t* out_q, cudaStream_t s) {
  NormPlan plan;
  if (!norm_plan(D, &plan) || D % 4) return cudaErrorInvalidValue;
  if (D == 2048 && plan.n_leaves == 16 && plan.leaf_len == 128) {
    norm_stats_rows_d2048_kernel<<<rows, 128, 0, s>>>(x, gamma, eps, inv_buf, absmax_groups, rows_per_group);
    norm_quant_apply_d2048_kernel<<<rows, 128, 0, s>>>(x, gamma, inv_buf, absmax_groups, rows_per_group, out_q);
    return cudaGetLastError();
  }
  cudaError_t e = launch_rmsnorm_rows(x, gamma, eps, h_buf, absmax_groups, rows, D, rows_per_group, s);
  if (e != cudaSuccess) return e;
  return launch_quantize_rows(h_buf, absmax_groups, rows, D, rows_per_group, out_q, s);
}

// Per-row INT8 quantization (quantize_int8 of model/tinyllama_gemm_int8.py:36-42
// applied to one row): one 256-thread CTA per row, the row held in registers
// (up to 8 float4 per thread, K <= 8192), one CTA barrier for max |x|.
constexpr int kQuantThreads = 256;
constexpr int kQuantVec = 8;
__global__ void __launch_bounds__(kQuantThreads) quant_rows_reg_kernel(const float* x, int K, int8_t* out_q,
                                                                       float* out_absmax) {
  __shared__ float red[kQuantThreads / 32];
  const int r = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int n4 = K >> 2;
  pdl_launch_dependents();  // nothing is read before the wait
  pdl_wait();
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * K);
  float4 v[kQuantVec];
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < kQuantVec; ++i) {
    const int c = t + i * kQuantThreads;
    v[i] = c < n4 ? src[c] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
#pragma unroll
  for (int i = 0; i < kQuantVec; ++i)
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < kQuantThreads / 32; ++w) m = fmaxf(m, red[w]);
  const float sf = static_cast<float>(quant_scale64(m));
  uint32_t* dst = reinterpret_cast<uint32_t*>(out_q + static_cast<size_t>(r) * K);
#pragma unroll
  for (int i = 0; i < kQuantVec; ++i) {
    const int c = t + i * kQuantThreads;
    if (c < n4) dst[c] = quant_pack4(v[i], sf);
  }
  if (t == 0) out_absmax[r] = m;
}

cudaError_t launch_norm_quant_rows(const float* x, const float* gamma, float eps, int rows, int D,
                                   int8_t* out_q, float* out_absmax, cudaStream_t s, bool pdl,
                                   float* zero_rows) {
  NormPlan plan;
  if (!norm_plan(D, &plan) || D % 4) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  if (D == 2048 && plan.n_leaves == 16 && plan.leaf_len == 128) {
    cudaLaunchConfig_t cfg = row_cfg(rows, 128, 0, s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, norm_quant_rows_d2048_kernel, x, gamma, eps, out_q, out_absmax, zero_rows);
  }
  cudaLaunchConfig_t cfg = row_cfg(rows, 256, rmsnorm_rows_smem(D), s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, norm_quant_rows_kernel, x, gamma, eps, D, plan, out_q, out_absmax, zero_rows);
}

__global__ void __launch_bounds__(256) quant_rows_kernel(const float* x, int K, int8_t* out_q, float* out_absmax) {
  __shared__ float red[32];
  const int r = blockIdx.x;
  pdl_wait();
  const float* src = x + static_cast<size_t>(r) * K;
  float m = 0.0f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(src[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float v = (threadIdx.x & 31) < static_cast<int>(blockDim.x >> 5) ? red[threadIdx.x & 31] : 0.0f;
  v = warp_max(v);
  pdl_launch_dependents();
  const float sf = static_cast<float>(quant_scale64(v));
  int8_t* dst = out_q + static_cast<size_t>(r) * K;
  for (int i = threadIdx.x; i < K; i += blockDim.x) dst[i] = static_cast<int8_t>(quantize_one(src[i], sf));
  if (threadIdx.x == 0) out_absmax[r] = v;
}

cudaError_t launch_quant_rows(const float* x, int rows, int K, int8_t* out_q, float* out_absmax,
                              cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  if (K % 4 == 0 && K <= 4 * kQuantVec * kQuantThreads) {
    cudaLaunchConfig_t cfg = row_cfg(rows, kQuantThreads, 0, s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, quant_rows_reg_kernel, x, K, out_q, out_absmax);
  }
  cudaLaunchConfig_t cfg = row_cfg(rows, 256, 0, s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, quant_rows_kernel, x, K, out_q, out_absmax);
}

// INT8 quantization of rows whose max |x| is already known (the producer
// folded it into absmax[row] with atomics): elementwise, one float4 per
// thread over the whole [rows][K] block, so the grid covers the SMs instead
// of one CTA per row. Same scale and rounding as quant_rows_reg_kernel.
constexpr int kQuantKnownThreads = 256;
__global__ void __launch_bounds__(kQuantKnownThreads) quant_known_rows_kernel(const float* x, const float* absmax,
                                                                            int rows, int K, int8_t* out_q) {
  const int n4 = K >> 2;
  const long long i = static_cast<long long>(blockIdx.x) * kQuantKnownThreads + threadIdx.x;
  pdl_launch_dependents();  // nothing is read before the wait
  pdl_wait();
  if (i >= static_cast<long long>(rows) * n4) return;
  const int r = static_cast<int>(i / n4);
  const float4 v = reinterpret_cast<const float4*>(x)[i];
  const float sf = static_cast<float>(quant_scale64(absmax[r]));
  reinterpret_cast<uint32_t*>(out_q)[i] = quant_pack4(v, sf);
}

cudaError_t launch_quant_known_rows(const float* x, const float* absmax, int rows, int K, int8_t* out_q,
                                    cudaStream_t s, bool pdl) {
  if (K % 4 || rows <= 0) return cudaErrorInvalidValue;
  const long long n4 = static_cast<long long>(rows) * (K / 4);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg =
      row_cfg(static_cast<int>((n4 + kQuantKnownThreads - 1) / kQuantKnownThreads), kQuantKnownThreads, 0, s, pdl,
              attr);
  return cudaLaunchKernelEx(&cfg, quant_known_rows_kernel, x, absmax, rows, K, out_q);
}

__global__ void __launch_bounds__(512) row_argmax_kernel(const float* logits, int V, int32_t* out) {
  __shared__ unsigned long long red[32];
  const int r = blockIdx.x;
  pdl_wait();
  const float* src = logits + static_cast<size_t>(r) * V;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const unsigned long long k = argmax_key(src[i], i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long b = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
      b = other > b ? other : b;
    }
    if (threadIdx.x == 0) out[r] = argmax_key_index(b);
  }
}

cudaError_t launch_row_argmax(const float* logits, int rows, int V, int32_t* out, cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = row_cfg(rows, 512, 0, s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, row_argmax_kernel, logits, V, out);
}

__global__ void absmax_rows_kernel(const float* x, int K, int rows_per_group, float* absmax) {
  const int r = blockIdx.x;
  const float* src = x + static_cast<size_t>(r) * K;
  float m = 0.0f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(src[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomic_max_nonneg(absmax + r / rows_per_group, m);
}

cudaError_t launch_absmax_rows(const float* x, int rows, int K, int rows_per_group, float* absmax,
                               cudaStream_t s) {
  absmax_rows_kernel<<<rows, 256, 0, s>>>(x, K, rows_per_group, absmax);
  return cudaGetLastError();
}

__global__ void quantize_rows_kernel(const float* x, const float* absmax, int K, int rows_per_group,
                                     int8_t* out) {
  const int r = blockIdx.x;
  const float sf = static_cast<float>(quant_scale64(absmax[r / rows_per_group]));
  const float* src = x + static_cast<size_t>(r) * K;
  int8_t* dst = out + static_cast<size_t>(r) * K;
  for (int i = threadIdx.x; i < K; i += blockDim.x) dst[i] = static_cast<int8_t>(quantize_one(src[i], sf));
}

// Same, for rows of K % 4 == 0 and K <= 8192: every load of the row is
// issued before the first store (16-byte loads, 4-byte stores).
__global__ void __launch_bounds__(kQuantThreads) quantize_rows_vec_kernel(const float* x, const float* absmax,
                                                                          int K, int rows_per_group,
                                                                          int8_t* out) {
  const int r = blockIdx.x, t = threadIdx.x, n4 = K >> 2;
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * K);
  float4 v[kQuantVec];
#pragma unroll
  for (int i = 0; i < kQuantVec; ++i) {
    const int c = t + i * kQuantThreads;
    v[i] = c < n4 ? src[c] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  const float sf = static_cast<float>(quant_scale64(absmax[r / rows_per_group])), inv = quant_inv(sf);
  uint32_t* dst = reinterpret_cast<uint32_t*>(out + static_cast<size_t>(r) * K);
#pragma unroll
  for (int i = 0; i < kQuantVec; ++i) {
    const int c = t + i * kQuantThreads;
    if (c < n4) dst[c] = quant_pack4_inv(v[i], sf, inv);
  }
}

cudaError_t launch_quantize_rows(const float* x, const float* absmax_groups, int rows, int K,
                                 int rows_per_group, int8_t* out, cudaStream_t s) {
  if (K % 4 == 0 && K <= 4 * kQuantVec * kQuantThreads)
    quantize_rows_vec_kernel<<<rows, kQuantThreads, 0, s>>>(x, absmax_groups, K, rows_per_group, out);
  else
    quantize_rows_kernel<<<rows, 256, 0, s>>>(x, absmax_groups, K, rows_per_group, out);
  return cudaGetLastError();
}

// Debug capture of one sequence's attention (not on the generation path):
// query row i (position pos0 + i) against keys 0..n_keys-1 of the cache:
// scores[h][i][j] = (q_i . K_j) * 1/8 with K_j the dequantized cache row
// float32(k_q) * float32(s_K) (model/tinyllama_gemm_int8.py:156-159), -1e9
// where j > pos0 + i (the causal fill of :159), and probs = the max-shifted
// softmax of each row (model/tinyllama.py:100-103). With `rotate` the q rows
// are pre-RoPE (decode) and are rotated here at their position with the
// same float32 roundings as the attention kernels; otherwise they already
// are (prefill). Products are summed in double, so these match the
// reference's float64 scores to well below float32 resolution. One CTA per
// (query row, head).
__global__ void __launch_bounds__(256) attn_scores_debug_kernel(const float* qkv, int ld, int n_keys, int pos0,
                                                                int rotate, int H, int Hkv, const int8_t* kc,
                                                                const float* ks, const float* cosT, const float* sinT,
                                                                int slot, int layer, int L, int P, float* scores,
                                                                float* probs) {
  __shared__ double red[8];
  __shared__ float q[64];
  const int i = blockIdx.x, h = blockIdx.y, t = threadIdx.x, n_q = gridDim.x;
  const int kvh = h / (H / Hkv);
  const int pos = pos0 + i;
  if (t < 32) {
    const float* qr = qkv + static_cast<size_t>(i) * ld + h * 64;
    float a = qr[t], b = qr[t + 32];
    if (rotate) {
      const float* cs = cosT + static_cast<size_t>(pos) * 64;
      const float* sn = sinT + static_cast<size_t>(pos) * 64;
      const float r0 = __fadd_rn(__fmul_rn(a, cs[t]), __fmul_rn(-b, sn[t]));
      const float r1 = __fadd_rn(__fmul_rn(b, cs[t + 32]), __fmul_rn(a, sn[t + 32]));
      a = r0;
      b = r1;
    }
    q[t] = a;
    q[t + 32] = b;
  }
  __syncthreads();
  const size_t base = ((static_cast<size_t>(slot) * L + layer) * Hkv + kvh);
  const int8_t* krows = kc + base * P * 64;
  const float sk = ks[base];
  float* srow = scores + (static_cast<size_t>(h) * n_q + i) * n_keys;
  float* prow = probs + (static_cast<size_t>(h) * n_q + i) * n_keys;
  double m = -1e300;
  for (int j = t; j < n_keys; j += blockDim.x) {
    double sc = -1e9;
    if (j <= pos) {
      double acc = 0.0;
      for (int d = 0; d < 64; ++d)
        acc += static_cast<double>(q[d]) * static_cast<double>(__fmul_rn(static_cast<float>(krows[j * 64 + d]), sk));
      sc = acc * 0.125;
    }
    srow[j] = static_cast<float>(sc);
    m = fmax(m, sc);
  }
  for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((t & 31) == 0) red[t >> 5] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmax(m, red[w]);
  __syncthreads();
  double sum = 0.0;
  for (int j = t; j < n_keys; j += blockDim.x) sum += exp(static_cast<double>(srow[j]) - m);
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((t & 31) == 0) red[t >> 5] = sum;
  __syncthreads();
  sum = 0.0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) sum += red[w];
  for (int j = t; j < n_keys; j += blockDim.x) prow[j] = static_cast<float>(exp(static_cast<double>(srow[j]) - m) / sum);
}

cudaError_t launch_attn_scores_debug(const float* qkv, int ld, int n_q, int n_keys, int pos0, bool rotate, int H,
                                     int Hkv, const int8_t* kc, const float* ks, const float* cosT, const float* sinT,
                                     int slot, int layer, int L, int P, float* scores, float* probs, cudaStream_t s) {
  if (n_q <= 0 || n_keys <= 0 || H <= 0 || Hkv <= 0 || H % Hkv || pos0 < 0 || pos0 + n_q > P || n_keys > P)
    return cudaErrorInvalidValue;
  attn_scores_debug_kernel<<<dim3(n_q, H), 256, 0, s>>>(qkv, ld, n_keys, pos0, rotate ? 1 : 0, H, Hkv, kc, ks, cosT,
                                                        sinT, slot, layer, L, P, scores, probs);
  return cudaGetLastError();
}

// Prefill RoPE and K / V cache fill. rope_stats_prefill_kernel rotates each
// row's q heads in place and folds max |RoPE(k)| and max |v| per (sequence,
// kv head) into kv_absmax without writing k; kv_write_prefill_kernel
// recomputes the same rotated k and writes K and V quantized with those
// scales. Rotations use the float32 roundings of the decode path. One warp
// per row: for q, lanes 0-15 / 16-31 take two heads at a time with float2
// accesses to dims (2j, 2j + 1) and (2j + 32, 2j + 33); for k and v, lane l
// owns dims (l, l + 32) of every head.
TL_DEV void rope_pair(float a0, float a1, const float* cs, const float* sn, int d, float& r0, float& r1) {
  r0 = __fadd_rn(__fmul_rn(a0, cs[d]), __fmul_rn(-a1, sn[d]));
  r1 = __fadd_rn(__fmul_rn(a1, cs[d + 32]), __fmul_rn(a0, sn[d + 32]));
}
constexpr int kKvRowsPerWarp = 8;
constexpr int kRopeMaxH = 32;  // q heads whose loads a warp keeps in flight at once
__global__ void __launch_bounds__(256) rope_stats_prefill_kernel(float* qkv, int ld, int rows, int seq_len, int H,
                                                                 int Hkv, const float* cos, const float* sin,
                                                                 float* kv_absmax) {
  const int lane = threadIdx.x & 31;
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int r0 = w * kKvRowsPerWarp;
  float mk[8], mv[8];  // running maxima over this warp's rows of one sequence
  int cur = -1;
  auto flush = [&]() {
    if (cur < 0) return;
    for (int h = 0; h < Hkv; ++h) {
      const float a = warp_max(mk[h]), b = warp_max(mv[h]);
      if (lane == 0) {
        atomic_max_nonneg(kv_absmax + (cur * 2 + 0) * Hkv + h, a);
        atomic_max_nonneg(kv_absmax + (cur * 2 + 1) * Hkv + h, b);
      }
    }
  };
  const int j = lane & 15, hsub = lane >> 4;
  for (int r = r0; r < min(r0 + kKvRowsPerWarp, rows); ++r) {
    const int seq = r / seq_len, t = r % seq_len;
    if (seq != cur) {
      flush();
      cur = seq;
      for (int h = 0; h < 8; ++h) mk[h] = mv[h] = 0.0f;
    }
    float* row = qkv + static_cast<size_t>(r) * ld;
    const float* cs = cos + static_cast<size_t>(t) * 64;
    const float* sn = sin + static_cast<size_t>(t) * 64;
    const float2 c0 = *reinterpret_cast<const float2*>(cs + 2 * j), c1 = *reinterpret_cast<const float2*>(cs + 2 * j + 32);
    const float2 s0 = *reinterpret_cast<const float2*>(sn + 2 * j), s1 = *reinterpret_cast<const float2*>(sn + 2 * j + 32);
    // every load of the row (up to kRopeMaxH q heads at a time, k and v) is
    // issued before the first store, so the row costs one memory round trip,
    // not one per head pair
    const float* kv = row + H * 64;
    float ka[8], kb[8], va[8], vb[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      if (h < Hkv) {
        ka[h] = kv[h * 64 + lane];
        kb[h] = kv[h * 64 + lane + 32];
        va[h] = kv[(Hkv + h) * 64 + lane];
        vb[h] = kv[(Hkv + h) * 64 + lane + 32];
      }
    }
    for (int hb = 0; hb < H; hb += kRopeMaxH) {
      float2 xa[kRopeMaxH / 2], xb[kRopeMaxH / 2];
#pragma unroll
      for (int i = 0; i < kRopeMaxH / 2; ++i) {
        const int h = hb + hsub + 2 * i;
        if (h < H) {
          xa[i] = *reinterpret_cast<const float2*>(row + h * 64 + 2 * j);
          xb[i] = *reinterpret_cast<const float2*>(row + h * 64 + 2 * j + 32);
        }
      }
#pragma unroll
      for (int i = 0; i < kRopeMaxH / 2; ++i) {
        const int h = hb + hsub + 2 * i;
        if (h >= H) continue;
        const float2 x = xa[i], y = xb[i];
        *reinterpret_cast<float2*>(row + h * 64 + 2 * j) =
            make_float2(__fadd_rn(__fmul_rn(x.x, c0.x), __fmul_rn(-y.x, s0.x)),
                        __fadd_rn(__fmul_rn(x.y, c0.y), __fmul_rn(-y.y, s0.y)));
        *reinterpret_cast<float2*>(row + h * 64 + 2 * j + 32) =
            make_float2(__fadd_rn(__fmul_rn(y.x, c1.x), __fmul_rn(x.x, s1.x)),
                        __fadd_rn(__fmul_rn(y.y, c1.y), __fmul_rn(x.y, s1.y)));
      }
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      if (h < Hkv) {
        float k0, k1;
        rope_pair(ka[h], kb[h], cs, sn, lane, k0, k1);
        mk[h] = fmaxf(mk[h], fmaxf(fabsf(k0), fabsf(k1)));
        mv[h] = fmaxf(mv[h], fmaxf(fabsf(va[h]), fabsf(vb[h])));
      }
    }
  }
  flush();
}

cudaError_t launch_rope_stats_prefill(float* qkv, int ld, int rows, int seq_len, int H, int Hkv, const float* cos,
                                      const float* sin, float* kv_absmax, cudaStream_t s) {
  if (Hkv > 8 || (ld & 1)) return cudaErrorInvalidValue;
  const int warps = (rows + kKvRowsPerWarp - 1) / kKvRowsPerWarp;
  rope_stats_prefill_kernel<<<(warps + 7) / 8, 256, 0, s>>>(qkv, ld, rows, seq_len, H, Hkv, cos, sin, kv_absmax);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256) kv_write_prefill_kernel(const float* qkv, int ld, int rows, int seq_len, int H,
                                                               int Hkv, const float* cos, const float* sin,
                                                               const float* kv_absmax, int8_t* kc, int8_t* vc,
                                                               float* ks, float* vs, int slot_base, int layer, int L,
                                                               int P, uint16_t* kh, uint16_t* vh) {
  const int lane = threadIdx.x & 31;
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= rows) return;
  const int seq = r / seq_len, t = r % seq_len;
  const float* row = qkv + static_cast<size_t>(r) * ld + H * 64;
  const float* cs = cos + static_cast<size_t>(t) * 64;
  const float* sn = sin + static_cast<size_t>(t) * 64;
  // all of the row's k / v values and scales are loaded before the first
  // store (the stores could alias them as far as the compiler knows)
  float a0[16], a1[16], amax[16];
#pragma unroll
  for (int hh = 0; hh < 16; ++hh) {
    if (hh < 2 * Hkv) {
      const int kind = hh / Hkv, h = hh % Hkv;
      a0[hh] = row[hh * 64 + lane];
      a1[hh] = row[hh * 64 + lane + 32];
      amax[hh] = kv_absmax[(seq * 2 + kind) * Hkv + h];
    }
  }
#pragma unroll
  for (int hh = 0; hh < 16; ++hh) {
    if (hh >= 2 * Hkv) break;
    const int kind = hh / Hkv, h = hh % Hkv;  // 0 = K, 1 = V
    const float sf = static_cast<float>(quant_scale64(amax[hh]));
    float b0 = a0[hh], b1 = a1[hh];
    if (kind == 0) rope_pair(b0, b1, cs, sn, lane, b0, b1);
    const size_t sidx = (static_cast<size_t>(slot_base + seq) * L + layer) * Hkv + h;
    int8_t* dst = (kind == 0 ? kc : vc) + (sidx * P + t) * 64;
    const int q0 = quantize_one(b0, sf), q1 = quantize_one(b1, sf);
    dst[lane] = static_cast<int8_t>(q0);
    dst[lane + 32] = static_cast<int8_t>(q1);
    if (kh) {
      uint16_t* hd = (kind == 0 ? kh : vh) + (static_cast<size_t>(seq * Hkv + h) * seq_len + t) * 64;
      hd[lane] = __half_as_ushort(__int2half_rn(q0));
      hd[lane + 32] = __half_as_ushort(__int2half_rn(q1));
    }
    if (t == 0 && lane == 0) (kind == 0 ? ks : vs)[sidx] = sf;
  }
}

cudaError_t launch_kv_write_prefill(const float* qkv, int ld, int rows, int seq_len, int H, int Hkv, const float* cos,
                                    const float* sin, const float* kv_absmax, int8_t* kc, int8_t* vc, float* ks,
                                    float* vs, int slot_base, int layer, int L, int P, cudaStream_t s,
                                    uint16_t* kh, uint16_t* vh) {
  if (Hkv > 8 || (!kh) != (!vh)) return cudaErrorInvalidValue;
  kv_write_prefill_kernel<<<(rows + 7) / 8, 256, 0, s>>>(qkv, ld, rows, seq_len, H, Hkv, cos, sin, kv_absmax, kc, vc,
                                                          ks, vs, slot_base, layer, L, P, kh, vh);
  return cudaGetLastError();
}

// ==================================================================== misc
// dst[n * dst_ld + k] = src[k * N + n]
__global__ void transpose_i8_kernel(const int8_t* src, int8_t* dst, int K, int N, int dst_ld) {
  __shared__ int8_t tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int j = ty; j < 32; j += 8) {
    const int k = k0 + j, n = n0 + tx;
    tile[j][tx] = (k < K && n < N) ? src[static_cast<size_t>(k) * N + n] : 0;
  }
  __syncthreads();
  for (int j = ty; j < 32; j += 8) {
    const int n = n0 + j, k = k0 + tx;
    if (n < N && k < K) dst[static_cast<size_t>(n) * dst_ld + k] = tile[tx][j];
  }
}

cudaError_t launch_transpose_i8(const int8_t* src_kn, int8_t* dst_nk, int K, int N, cudaStream_t s) {
  dim3 grid((N + 31) / 32, (K + 31) / 32);
  transpose_i8_kernel<<<grid, dim3(32, 8), 0, s>>>(src_kn, dst_nk, K, N, K);
  return cudaGetLastError();
}

cudaError_t launch_interleave_gate_up(const int8_t* gate_kn, const int8_t* up_kn, int8_t* dst,
                                      int K, int F, cudaStream_t s) {
  dim3 grid((F + 31) / 32, (K + 31) / 32);
  transpose_i8_kernel<<<grid, dim3(32, 8), 0, s>>>(gate_kn, dst, K, F, 2 * K);
  transpose_i8_kernel<<<grid, dim3(32, 8), 0, s>>>(up_kn, dst + K, K, F, 2 * K);
  return cudaGetLastError();
}

TL_DEV uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__global__ void random_i8_kernel(int8_t* dst, size_t n, uint64_t seed) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = splitmix64(seed ^ (i * 0xD1B54A32D192ED03ull));
    dst[i] = static_cast<int8_t>(static_cast<int>(h % 255ull) - 127);
  }
}

__global__ void random_normal_kernel(float* dst, size_t n, float std, uint64_t seed) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = splitmix64(seed ^ (i * 0xD1B54A32D192ED03ull));
    const float u1 = (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
    dst[i] = std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
  }
}

__global__ void fill_f32_kernel(float* dst, size_t n, float v) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = v;
}
__global__ void fill_f64_kernel(double* dst, size_t n, double v) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = v;
}

cudaError_t launch_random_i8(int8_t* dst, size_t n, uint64_t seed, cudaStream_t s) {
  random_i8_kernel<<<148 * 8, 256, 0, s>>>(dst, n, seed);
  return cudaGetLastError();
}
__global__ void random_i8_block_kernel(int8_t* dst, int rows, int cols, long long r0, long long c0,
                                       long long src_cols, uint64_t seed) {
  const size_t n = static_cast<size_t>(rows) * cols;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const long long r = static_cast<long long>(i / cols), c = static_cast<long long>(i % cols);
    const uint64_t g = static_cast<uint64_t>((r0 + r) * src_cols + c0 + c);
    const uint64_t h = splitmix64(seed ^ (g * 0xD1B54A32D192ED03ull));
    dst[i] = static_cast<int8_t>(static_cast<int>(h % 255ull) - 127);
  }
}
cudaError_t launch_random_i8_block(int8_t* dst, int rows, int cols, long long src_row0, long long src_col0,
                                   long long src_cols, uint64_t seed, cudaStream_t s) {
  random_i8_block_kernel<<<148 * 8, 256, 0, s>>>(dst, rows, cols, src_row0, src_col0, src_cols, seed);
  return cudaGetLastError();
}
cudaError_t launch_random_normal_f32(float* dst, size_t n, float std, uint64_t seed, cudaStream_t s) {
  random_normal_kernel<<<148 * 8, 256, 0, s>>>(dst, n, std, seed);
  return cudaGetLastError();
}
cudaError_t launch_fill_f32(float* dst, size_t n, float v, cudaStream_t s) {
  fill_f32_kernel<<<148 * 4, 256, 0, s>>>(dst, n, v);
  return cudaGetLastError();
}
cudaError_t launch_fill_f64(double* dst, size_t n, double v, cudaStream_t s) {
  fill_f64_kernel<<<148 * 4, 256, 0, s>>>(dst, n, v);
  return cudaGetLastError();
}

// Decode-step bookkeeping: emit the argmax token, apply the stop rules of
// stop_condition_unit.sv:19-37 (EOS before MAX_TOKENS; abort is host-side),
// advance the position.
__global__ void step_finalize_kernel(StepArgs a) {
  pdl_wait();
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= a.M) return;
  int tok = 0;
  if (a.am_key) {  // packed (logit, id) key of the LM-head GEMM; re-armed for the next step
    tok = argmax_key_index(a.am_key[m]);
    a.am_key[m] = 0ull;
  } else {
    tok = a.argmax[m];
  }
  if (a.stop[m] != 0 || !a.active[m]) return;
  const int max_new = a.run[0], eos = a.run[1], out_cap = a.run[2];
  const int c = a.count[m];
  if (c < out_cap) a.out_ids[static_cast<size_t>(m) * a.out_stride + c] = tok;
  a.count[m] = c + 1;
  a.pos[m] += 1;  // the token just processed now sits in the cache
  a.tokens[m] = tok;
  int stop = 0;
  if (tok == eos) stop = 1;
  else if ((max_new != 0 && c + 1 >= max_new) || c + 1 >= out_cap) stop = 2;
  else if (a.pos[m] >= a.P) stop = 4;  // next feed would exceed the cache
  if (stop) {
    a.stop[m] = stop;
    a.active[m] = 0;
  }
}

cudaError_t launch_step_finalize(const StepArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.M + 127) / 128);
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, step_finalize_kernel, a);
}

// ============================================== tensor-parallel exchange
// Per-sequence INT8 quantization of this rank's column block [col0, col0 +
// Kl) of a float matrix [rows][Kl], written into the full-width INT8 matrix
// [rows][Kf] of every rank of the group -- its own and, through CUDA-IPC
// mapped pointers over NVLink, its peers': the all-gather of the quantized
// activations fused into the quantization. Every CTA fences at system
// scope before taking a ticket; the last one publishes `epoch` into each
// peer's flag slot for this rank with a system-scope release, so a peer
// that acquires the epoch also sees every byte.
__device__ unsigned int g_tp_error = 0;

TL_DEV void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
TL_DEV unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) quantize_scatter_kernel(const float* x, const float* absmax, int rpg, int Kl,
                                                               int Kf, int col0, TpScatter t, unsigned int* done,
                                                               unsigned int epoch) {
  const int r = blockIdx.x;
  const float sf = static_cast<float>(quant_scale64(absmax[r / rpg])), inv = quant_inv(sf);
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * Kl);
  const size_t off = static_cast<size_t>(r) * Kf + col0;
  for (int c = threadIdx.x; c < Kl / 4; c += blockDim.x) {
    const uint32_t q = quant_pack4_inv(src[c], sf, inv);
    for (int d = 0; d < t.ndst; ++d) reinterpret_cast<uint32_t*>(t.dst[d] + off)[c] = q;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      __threadfence_system();
      *done = 0u;
      for (int d = 1; d < t.ndst; ++d) st_release_sys(t.flag[d], epoch);
    }
  }
}

cudaError_t launch_quantize_scatter(const float* x, const float* absmax, int rows_per_group, int rows, int Kl, int Kf,
                                    int col0, const TpScatter& t, unsigned int* done, unsigned int epoch,
                                    cudaStream_t s) {
  if (Kl % 4 || Kf % 4 || col0 % 4 || t.ndst < 1 || t.ndst > 4) return cudaErrorInvalidValue;
  quantize_scatter_kernel<<<rows, 256, 0, s>>>(x, absmax, rows_per_group, Kl, Kf, col0, t, done, epoch);
  return cudaGetLastError();
}

// Waits (one thread, ~2 s bound) until every peer q != rank has published
// `epoch` into flags[q]; on expiry records 1 + q in the tensor-parallel
// error word and returns, so the host reports TL_ERR_TIMEOUT.
__global__ void tp_wait_kernel(const unsigned int* flags, int world, int rank, unsigned int epoch) {
  if (threadIdx.x != 0) return;
  const long long t0 = clock64();
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    while (static_cast<int>(ld_acquire_sys(flags + q) - epoch) < 0) {
      if (clock64() - t0 > 4000000000ll) {
        atomicCAS(&g_tp_error, 0u, 1u + static_cast<unsigned int>(q));
        return;
      }
    }
  }
}

cudaError_t launch_tp_wait(const unsigned int* flags, int world, int rank, unsigned int epoch, cudaStream_t s) {
  tp_wait_kernel<<<1, 32, 0, s>>>(flags, world, rank, epoch);
  return cudaGetLastError();
}

// Tensor-parallel prefill, row-split O / down: after the INT32 all-reduce
// of the ranks' partial accumulators, out = resid + float32(acc) *
// float32(s_x * s_w[n]) -- the single-GPU EPI_RESID epilogue's exact
// arithmetic (dequant of model/tinyllama_gemm_int8.py:45-46, then the
// residual add of :266,270), so the result is bit-identical to one GPU's.
// Four elements per thread (N % 4 == 0).
__global__ void __launch_bounds__(256) dequant_resid_kernel(const int32_t* __restrict__ acc,
                                                            const float* __restrict__ in_absmax, int rows_per_group,
                                                            int row0, const double* __restrict__ w_scale, float* out,
                                                            size_t n4, int N) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t e0 = i * 4;
    const int m = row0 + static_cast<int>(e0 / N), n = static_cast<int>(e0 % N);
    const double sx = quant_scale64(in_absmax[m / rows_per_group]);
    const int4 a = reinterpret_cast<const int4*>(acc)[i];
    float4 r = reinterpret_cast<const float4*>(out)[i];
    r.x = __fadd_rn(r.x, dequant(a.x, sx, w_scale[n]));
    r.y = __fadd_rn(r.y, dequant(a.y, sx, w_scale[n + 1]));
    r.z = __fadd_rn(r.z, dequant(a.z, sx, w_scale[n + 2]));
    r.w = __fadd_rn(r.w, dequant(a.w, sx, w_scale[n + 3]));
    reinterpret_cast<float4*>(out)[i] = r;
  }
}

cudaError_t launch_dequant_resid(const int32_t* acc, const float* in_absmax, int rows_per_group, int row0,
                                 const double* w_scale, float* out, int rows, int N, cudaStream_t s) {
  if (N % 4 || rows <= 0) return cudaErrorInvalidValue;
  const size_t n4 = static_cast<size_t>(rows) * N / 4;
  const int grid = static_cast<int>(std::min<size_t>((n4 + 255) / 256, static_cast<size_t>(device_sm_count()) * 8));
  dequant_resid_kernel<<<grid, 256, 0, s>>>(acc, in_absmax, rows_per_group, row0, w_scale, out, n4, N);
  return cudaGetLastError();
}

cudaError_t tp_read_error(unsigned int* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_tp_error, sizeof(unsigned int));
  if (e != cudaSuccess || !*code) return e;
  unsigned int zero = 0;
  return cudaMemcpyToSymbol(g_tp_error, &zero, sizeof(unsigned int));
}

// token id of each row's packed argmax key; the key is re-armed (zeroed)
__global__ void keys_to_tokens_kernel(unsigned long long* key, int32_t* token, int M) {
  pdl_wait();
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  token[m] = argmax_key_index(key[m]);
  key[m] = 0ull;
}

cudaError_t launch_keys_to_tokens(unsigned long long* key, int32_t* token, int M, cudaStream_t s) {
  keys_to_tokens_kernel<<<(M + 127) / 128, 128, 0, s>>>(key, token, M);
  return cudaGetLastError();
}

__global__ void rows_rewind_kernel(int* pos, int* active, int* count, int* stop, int M, int position) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  pos[m] = position;
  active[m] = 1;
  count[m] = 0;
  stop[m] = 0;
}

cudaError_t launch_rows_rewind(int* pos, int* active, int* count, int* stop, int M, int position,
                               cudaStream_t s) {
  rows_rewind_kernel<<<(M + 127) / 128, 128, 0, s>>>(pos, active, count, stop, M, position);
  return cudaGetLastError();
}

// ============================================== contract mode (Q16.16 wrappers)
// The hardware's fixed-point wrappers around its nonlinear blocks
// (rtl/nonlinear/*_wrapper.sv, model/export_fpga_vectors.py:874-927,
// 1522-1990): INT8 in, Q16.16 core values, INT8 out by a Q16.16 scale.
TL_DEV float q16_to_float(int32_t raw) {  // float32(raw / 65536), the division in double
  return static_cast<float>(static_cast<double>(raw) / 65536.0);
}
TL_DEV int32_t float_to_q16(float v) {     // round half to even of v * 65536, saturated
  const long long r = __double2ll_rn(static_cast<double>(v) * 65536.0);
  return static_cast<int32_t>(r > 2147483647ll ? 2147483647ll : (r < -2147483648ll ? -2147483648ll : r));
}
TL_DEV int32_t mul_i32_wrap(int32_t a, int32_t b) {  // int32 product modulo 2^32 (NumPy int32)
  return static_cast<int32_t>(static_cast<uint32_t>(a) * static_cast<uint32_t>(b));
}
// Q16.16 value / Q16.16 scale, half to even on the remainder, clamped
TL_DEV int8_t quant_fixed_q16(int32_t v, uint32_t scale, bool nonneg) {
  const unsigned long long den = scale ? scale : 1u;
  const unsigned long long mag = v < 0 ? static_cast<unsigned long long>(-static_cast<long long>(v))
                                       : static_cast<unsigned long long>(v);
  unsigned long long q = mag / den;
  const unsigned long long r = mag - q * den;
  if (2 * r > den || (2 * r == den && (q & 1))) ++q;
  long long sgn = v < 0 ? -static_cast<long long>(q) : static_cast<long long>(q);
  const long long lo = nonneg ? 0 : -127;
  sgn = sgn < lo ? lo : (sgn > 127 ? 127 : sgn);
  return static_cast<int8_t>(sgn);
}
// |t| >> 16 rounded half to even, sign restored (the RTL's Q16.16 rounding)
TL_DEV long long round_shift16(long long t) {
  const unsigned long long mag = t < 0 ? static_cast<unsigned long long>(-t) : static_cast<unsigned long long>(t);
  unsigned long long q = mag >> 16;
  const unsigned long long rem = mag & 0xffffu;
  if (rem > 0x8000u || (rem == 0x8000u && (q & 1))) ++q;
  return t < 0 ? -static_cast<long long>(q) : static_cast<long long>(q);
}

// RMSNorm wrapper: one CTA per row; the float32 RMSNorm in NumPy's order.
__global__ void __launch_bounds__(256) contract_rmsnorm_kernel(const int8_t* xq, int D, uint32_t in_scale,
                                                               const int32_t* gamma_q16, float eps, uint32_t out_scale,
                                                               NormPlan plan, int8_t* yq, int32_t* y16) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* buf = reinterpret_cast<float*>(smem);
  float* g = buf + D;
  RowScratchView rs = rs_view(g + D, plan);
  const size_t r = blockIdx.x;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    buf[i] = q16_to_float(mul_i32_wrap(xq[r * D + i], static_cast<int32_t>(in_scale)));
    g[i] = q16_to_float(gamma_q16[i]);
  }
  __syncthreads();
  block_rmsnorm(buf, D, g, eps, plan, rs);
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const int32_t v = float_to_q16(buf[i]);
    if (y16) y16[r * D + i] = v;
    yq[r * D + i] = quant_fixed_q16(v, out_scale, false);
  }
}

cudaError_t launch_contract_rmsnorm(const int8_t* xq, int rows, int D, uint32_t in_scale, const int32_t* gamma_q16,
                                    float eps, uint32_t out_scale, int8_t* yq, int32_t* y16, cudaStream_t s) {
  NormPlan plan;
  if (rows <= 0 || !norm_plan(D, &plan)) return cudaErrorInvalidValue;
  const size_t smem = 8 * static_cast<size_t>(D) + 4 * rs_floats(plan) + 16;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(contract_rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  contract_rmsnorm_kernel<<<rows, 256, smem, s>>>(xq, D, in_scale, gamma_q16, eps, out_scale, plan, yq, y16);
  return cudaGetLastError();
}

// SiLU wrapper, elementwise.
__global__ void contract_silu_kernel(const int8_t* xq, long long n, uint32_t in_scale, uint32_t out_scale, int8_t* yq,
                                     int32_t* y16) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float x = q16_to_float(mul_i32_wrap(xq[i], static_cast<int32_t>(in_scale)));
    const float c = fminf(fmaxf(x, -60.0f), 60.0f);
    const float y = __fdiv_rn(x, __fadd_rn(1.0f, expf(-c)));
    const int32_t v = float_to_q16(y);
    if (y16) y16[i] = v;
    yq[i] = quant_fixed_q16(v, out_scale, false);
  }
}

cudaError_t launch_contract_silu(const int8_t* xq, long long n, uint32_t in_scale, uint32_t out_scale, int8_t* yq,
                                 int32_t* y16, cudaStream_t s) {
  if (n <= 0) return cudaErrorInvalidValue;
  const int grid = static_cast<int>(std::min<long long>((n + 255) / 256, device_sm_count() * 8ll));
  contract_silu_kernel<<<grid, 256, 0, s>>>(xq, n, in_scale, out_scale, yq, y16);
  return cudaGetLastError();
}

// Softmax wrapper: one warp per row of <= 128 scores. Scores times the
// Q16.16 scale saturate to int32; the float32 softmax sums in NumPy's order
// (8 strided accumulators, then ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then
// the tail); probabilities to Q16.16, then p * 127 >> 16 (the 1/127 scale).
__global__ void __launch_bounds__(128) contract_softmax_kernel(const int32_t* scores, int rows, int cols,
                                                               uint32_t scale, int8_t* pq, int32_t* p16) {
  __shared__ float e_sm[4][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 4 + warp;
  if (r >= rows) return;
  float x[4];
  float m = -INFINITY;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int c = lane + 32 * u;
    x[u] = -INFINITY;
    if (c < cols) {
      long long t = static_cast<long long>(scores[static_cast<size_t>(r) * cols + c]) * static_cast<long long>(scale);
      t = t > 2147483647ll ? 2147483647ll : (t < -2147483648ll ? -2147483648ll : t);
      x[u] = q16_to_float(static_cast<int32_t>(t));
      m = fmaxf(m, x[u]);
    }
  }
  m = warp_max(m);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int c = lane + 32 * u;
    if (c < cols) e_sm[warp][c] = expf(__fsub_rn(x[u], m));
  }
  __syncwarp();
  float sum = 0.0f;
  if (lane == 0) {
    const float* e = e_sm[warp];
    if (cols < 8) {
      for (int c = 0; c < cols; ++c) sum = __fadd_rn(sum, e[c]);
    } else {
      float acc[8];
      for (int j = 0; j < 8; ++j) acc[j] = e[j];
      const int full = cols - cols % 8;
      for (int b = 8; b < full; b += 8)
        for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], e[b + j]);
      sum = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])),
                      __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7])));
      for (int c = full; c < cols; ++c) sum = __fadd_rn(sum, e[c]);
    }
  }
  sum = __shfl_sync(0xffffffffu, sum, 0);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int c = lane + 32 * u;
    if (c >= cols) continue;
    const int32_t v = float_to_q16(__fdiv_rn(e_sm[warp][c], sum));
    const long long q = round_shift16(static_cast<long long>(v) * 127);
    const size_t o = static_cast<size_t>(r) * cols + c;
    if (p16) p16[o] = v;
    pq[o] = static_cast<int8_t>(q < 0 ? 0 : (q > 127 ? 127 : q));
  }
}

cudaError_t launch_contract_softmax(const int32_t* scores, int rows, int cols, uint32_t scale, int8_t* pq, int32_t* p16,
                                    cudaStream_t s) {
  if (rows <= 0 || cols <= 0 || cols > 128) return cudaErrorInvalidValue;
  contract_softmax_kernel<<<(rows + 3) / 4, 128, 0, s>>>(scores, rows, cols, scale, pq, p16);
  return cudaGetLastError();
}

// Q16.16 RoPE of INT8 rows [rows][64] with per-row tables: lower half
// x*cos - x[d+32]*sin, upper half x*cos + x[d-32]*sin, rounded to INT8
// (rtl/compute/rope_unit.sv:73-127, model/export_fpga_vectors.py:684-732).
__global__ void contract_rope_kernel(const int8_t* x, const int32_t* cs, const int32_t* sn, long long n, int8_t* out) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i >> 6;
    const int d = static_cast<int>(i & 63);
    const long long xv = x[i], pv = x[(row << 6) + (d < 32 ? d + 32 : d - 32)];
    const long long t = d < 32 ? xv * cs[i] - pv * sn[i] : xv * cs[i] + pv * sn[i];
    const long long q = round_shift16(t);
    out[i] = static_cast<int8_t>(q < -127 ? -127 : (q > 127 ? 127 : q));
  }
}

cudaError_t launch_contract_rope(const int8_t* x, const int32_t* cs, const int32_t* sn, int rows, int8_t* out,
                                 cudaStream_t s) {
  if (rows <= 0) return cudaErrorInvalidValue;
  const long long n = static_cast<long long>(rows) * 64;
  const int grid = static_cast<int>(std::min<long long>((n + 255) / 256, device_sm_count() * 8ll));
  contract_rope_kernel<<<grid, 256, 0, s>>>(x, cs, sn, n, out);
  return cudaGetLastError();
}

// Unsaturated INT32 residual add (rtl/compute/residual_add.sv:92-96): modulo 2^32.
__global__ void residual_add_i32_kernel(const int32_t* a, const int32_t* b, int32_t* out, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = static_cast<int32_t>(static_cast<uint32_t>(a[i]) + static_cast<uint32_t>(b[i]));
}

cudaError_t launch_residual_add_i32(const int32_t* a, const int32_t* b, int32_t* out, long long n, cudaStream_t s) {
  if (n <= 0) return cudaErrorInvalidValue;
  const int grid = static_cast<int>(std::min<long long>((n + 255) / 256, device_sm_count() * 8ll));
  residual_add_i32_kernel<<<grid, 256, 0, s>>>(a, b, out, n);
  return cudaGetLastError();
}

}  // namespace tl
