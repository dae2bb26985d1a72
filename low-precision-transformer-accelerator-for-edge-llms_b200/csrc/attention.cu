// attention.cu -- GQA decode attention over the INT8 KV cache on tensor cores.
//
// Reference semantics: scores = (q . k) / sqrt(64) with k the dequantized
// cache row, causal over positions 0..p, softmax, weighted sum of the
// dequantized V rows (model/tinyllama_gemm_int8.py:154-163 with the KV cache
// of docs/design_decisions.txt A7); GQA maps q head g to kv head g / 8
// (rtl/compute/gqa_router.sv:25-31); the new position's K (after RoPE) and V
// are quantized with the frozen per-(layer, kv head) scales and appended in
// place (rtl/memory/kv_cache_manager.sv:43-47 layout).
//
// Mapping: a fixed number of CTAs per (kv head, sequence), each looping over
// its share of TS-position context chunks, four warps. Each warp runs flash-attention tiles of 16 positions with
// mma.sync m16n8k16 fp16: A = the group's query rows (8 heads, padded to 16)
// for Q.K^T and the probabilities for P.V; B = INT8 K / V rows converted to
// fp16, which is exact for |v| <= 127. To keep fp32-level accuracy the fp32
// Q and P operands are split into fp16 hi + lo halves (two MMAs each, ~22
// mantissa bits). Each query row is first scaled by a power of two that puts
// its largest element in [2^13, 2^14) and the probabilities by 2^14, so the
// lo halves stay in fp16's normal range; the scales are exact and undone on
// the fp32 accumulators. (INT8 re-quantization of the attention output makes
// float error visible as rounding flips, so attention has to be as accurate
// as fp32 arithmetic.) Warps merge in shared memory; splits merge via a
// per-(sequence, kv head) partial buffer, the last CTA to arrive (atomic
// ticket) producing the output. CTAs with no chunk exit at once.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.cuh"

namespace tl {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kKStride = 80;   // bytes per cached K row in smem (conflict-free B loads)
constexpr int kVStride = 72;   // bytes per cached V row in smem

// two floats -> packed fp16x2, first argument in the low half
TL_DEV uint32_t pack2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// fp32 pair -> fp16 (hi) and fp16 of the exact remainder (lo)
TL_DEV void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const float r0 = x0 - __half2float(h0), r1 = x1 - __half2float(h1);
  __half2 hv;
  hv.x = h0;
  hv.y = h1;
  hi = *reinterpret_cast<uint32_t*>(&hv);
  lo = pack2(r0, r1);
}
// power of two that maps max|row| into [2^13, 2^14)
TL_DEV float pow2_scale(float amax) {
  if (!(amax > 0.0f)) return 1.0f;
  int e;
  frexpf(amax, &e);
  return ldexpf(1.0f, 14 - e);
}
constexpr float kPScale = 16384.0f;  // probabilities in [0, 1] -> [0, 2^14]
TL_DEV uint32_t pack_i8(int8_t a, int8_t b) {
  return pack2(static_cast<float>(a), static_cast<float>(b));
}

// D += A . B, m16n8k16, fp16 in, fp32 accumulate. a1/a3 (rows 8..15) are 0.
TL_DEV void mma16816(float* d, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

template <int TS>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_mma_kernel(AttnDecodeArgs a) {
  __shared__ __align__(16) int8_t k_sm[TS * kKStride];
  __shared__ __align__(16) int8_t v_sm[TS * kVStride];
  __shared__ float q_sm[8][64];
  __shared__ float q_scale[8];
  __shared__ float comb[kAttnWarps][8][66];
  __shared__ int last_cta;

  const int h = blockIdx.x, m = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.H / a.Hkv;
  const int Dq = a.H * 64;
  pdl_wait();
  const int p = a.pos[m];
  const bool valid_row = p >= 0 && p < a.P;
  if (!valid_row) {
    if (sp == 0)
      for (int i = tid; i < G * 64; i += kAttnThreads) a.out[static_cast<size_t>(m) * Dq + h * G * 64 + i] = 0.0f;
    return;
  }
  const int T = p + 1;
  const int nz = gridDim.z;
  const int n_chunks = (T + TS - 1) / TS;
  if (sp >= n_chunks) return;  // no work for this CTA (not counted in the merge)
  const int n_act = min(nz, n_chunks);
  const int slot = a.slot[m];
  const bool act = a.active ? (a.active[m] != 0) : true;
  const size_t sidx = (static_cast<size_t>(slot) * a.L + a.layer) * a.Hkv + h;
  const float sK = a.ks[sidx], sV = a.vs[sidx];
  int8_t* kbase = a.kc + sidx * static_cast<size_t>(a.P) * 64;
  int8_t* vbase = a.vc + sidx * static_cast<size_t>(a.P) * 64;
  const float* row = a.qkv + static_cast<size_t>(m) * a.ld;
  const float* cs = a.cos + static_cast<size_t>(p) * 64;
  const float* sn = a.sin + static_cast<size_t>(p) * 64;

  // ---- rotated queries of the group (rows >= G stay zero), power-of-two scaled
  for (int g = warp; g < 8; g += kAttnWarps) {
    float r0 = 0.0f, r1 = 0.0f;
    if (g < G) {
      const float* qr = row + (h * G + g) * 64;
      const float q0 = qr[lane], q1 = qr[lane + 32];
      r0 = __fadd_rn(__fmul_rn(q0, cs[lane]), __fmul_rn(-q1, sn[lane]));
      r1 = __fadd_rn(__fmul_rn(q1, cs[lane + 32]), __fmul_rn(q0, sn[lane + 32]));
    }
    const float qs = pow2_scale(warp_max(fmaxf(fabsf(r0), fabsf(r1))));
    q_sm[g][lane] = r0 * qs;
    q_sm[g][lane + 32] = r1 * qs;
    if (lane == 0) q_scale[g] = qs;
  }
  __syncthreads();

  // ---- Q fragments (hi/lo) for the four 16-wide k steps over head_dim
  const int g = lane >> 2, q4 = lane & 3;
  uint32_t qa_hi[4][2], qa_lo[4][2];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int c = ks * 16 + q4 * 2;
    split2(q_sm[g][c], q_sm[g][c + 1], qa_hi[ks][0], qa_lo[ks][0]);
    split2(q_sm[g][c + 8], q_sm[g][c + 9], qa_hi[ks][1], qa_lo[ks][1]);
  }
  // undo the exact power-of-two query scale of this thread's row g
  const float score_scale = sK * 0.125f / q_scale[g];
  float m_run = -INFINITY, l_part = 0.0f;
  float o[8][4];
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.0f;

  // This CTA owns chunks sp, sp + nz, ... of TS positions; the online
  // softmax state of each warp carries across them.
  for (int chunk = sp; chunk < n_chunks; chunk += nz) {
    const int t_begin = chunk * TS;
    const int n = min(TS, T - t_begin);
    __syncthreads();  // previous chunk fully consumed
    for (int i = tid; i < TS * 4; i += kAttnThreads) {
      const int r = i >> 2, c = i & 3;
      int4 v = make_int4(0, 0, 0, 0);
      if (r < n) v = reinterpret_cast<const int4*>(kbase + static_cast<size_t>(t_begin + r) * 64)[c];
      *reinterpret_cast<int4*>(k_sm + r * kKStride + c * 16) = v;
    }
    for (int i = tid; i < TS * 8; i += kAttnThreads) {
      const int r = i >> 3, c = i & 7;
      uint2 v = make_uint2(0u, 0u);
      if (r < n) v = reinterpret_cast<const uint2*>(vbase + static_cast<size_t>(t_begin + r) * 64)[c];
      *reinterpret_cast<uint2*>(v_sm + r * kVStride + c * 8) = v;
    }
    __syncthreads();
    // the new position's K (RoPE) and V: quantize, append, and use
    if (warp == 0 && p >= t_begin && p < t_begin + n) {
      const float* kr = row + Dq + h * 64;
      const float* vr = row + Dq + a.Hkv * 64 + h * 64;
      const float k0 = kr[lane], k1 = kr[lane + 32];
      const float r0 = __fadd_rn(__fmul_rn(k0, cs[lane]), __fmul_rn(-k1, sn[lane]));
      const float r1 = __fadd_rn(__fmul_rn(k1, cs[lane + 32]), __fmul_rn(k0, sn[lane + 32]));
      const int8_t qk0 = static_cast<int8_t>(quantize_one(r0, sK)), qk1 = static_cast<int8_t>(quantize_one(r1, sK));
      const int8_t qv0 = static_cast<int8_t>(quantize_one(vr[lane], sV));
      const int8_t qv1 = static_cast<int8_t>(quantize_one(vr[lane + 32], sV));
      const int rl = p - t_begin;
      k_sm[rl * kKStride + lane] = qk0;
      k_sm[rl * kKStride + lane + 32] = qk1;
      v_sm[rl * kVStride + lane] = qv0;
      v_sm[rl * kVStride + lane + 32] = qv1;
      if (act) {
        kbase[static_cast<size_t>(p) * 64 + lane] = qk0;
        kbase[static_cast<size_t>(p) * 64 + lane + 32] = qk1;
        vbase[static_cast<size_t>(p) * 64 + lane] = qv0;
        vbase[static_cast<size_t>(p) * 64 + lane + 32] = qv1;
      }
    }
    __syncthreads();

    for (int t0 = warp * 16; t0 < n; t0 += kAttnWarps * 16) {
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
        const int8_t* kr = k_sm + (t0 + nt * 8 + g) * kKStride + q4 * 2;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t b0 = pack_i8(kr[ks * 16], kr[ks * 16 + 1]);
          const uint32_t b1 = pack_i8(kr[ks * 16 + 8], kr[ks * 16 + 9]);
          mma16816(s[nt], qa_hi[ks][0], qa_hi[ks][1], b0, b1);
          mma16816(s[nt], qa_lo[ks][0], qa_lo[ks][1], b0, b1);
        }
      }
      float v4[4];
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int tl = t0 + nt * 8 + q4 * 2 + j;
          const float val = tl < n ? s[nt][j] * score_scale : -INFINITY;
          v4[nt * 2 + j] = val;
          mx = fmaxf(mx, val);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const float corr = expf(m_run - m_new);
      float pv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) pv[j] = expf(v4[j] - m_new);
      l_part = l_part * corr + (pv[0] + pv[1] + pv[2] + pv[3]);
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        o[dt][0] *= corr;
        o[dt][1] *= corr;
      }
      m_run = m_new;
      uint32_t pa_hi0, pa_lo0, pa_hi2, pa_lo2;
      split2(pv[0] * kPScale, pv[1] * kPScale, pa_hi0, pa_lo0);
      split2(pv[2] * kPScale, pv[3] * kPScale, pa_hi2, pa_lo2);
      const int8_t* vr = v_sm + (t0 + q4 * 2) * kVStride + g;
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        const int8_t* vc = vr + dt * 8;
        const uint32_t b0 = pack_i8(vc[0], vc[kVStride]);
        const uint32_t b1 = pack_i8(vc[8 * kVStride], vc[9 * kVStride]);
        mma16816(o[dt], pa_hi0, pa_hi2, b0, b1);
        mma16816(o[dt], pa_lo0, pa_lo2, b0, b1);
      }
    }
  }
  pdl_launch_dependents();

  // ---- merge the four warps of this CTA
  float l_row = l_part;
  l_row += __shfl_xor_sync(0xffffffffu, l_row, 1);
  l_row += __shfl_xor_sync(0xffffffffu, l_row, 2);
  if (q4 == 0) {
    comb[warp][g][0] = m_run;
    comb[warp][g][1] = l_row;
  }
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {
    comb[warp][g][2 + dt * 8 + q4 * 2] = o[dt][0] * (1.0f / kPScale);
    comb[warp][g][2 + dt * 8 + q4 * 2 + 1] = o[dt][1] * (1.0f / kPScale);
  }
  __syncthreads();
  float* part = a.part + (static_cast<size_t>(m) * a.Hkv + h) * a.splits * kAttnPartStride +
                static_cast<size_t>(sp) * kAttnPartStride;
  for (int i = tid; i < G * 64; i += kAttnThreads) {
    const int gg = i >> 6, d = i & 63;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, comb[w][gg][0]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = comb[w][gg][0] == -INFINITY ? 0.0f : expf(comb[w][gg][0] - M);
      L += comb[w][gg][1] * f;
      O += comb[w][gg][2 + d] * f;
    }
    part[gg * 66 + 2 + d] = O;
    if (d == 0) {
      part[gg * 66] = M;
      part[gg * 66 + 1] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(a.counters + static_cast<size_t>(m) * a.Hkv + h, 1u);
    last_cta = prev == static_cast<unsigned>(n_act - 1);
  }
  __syncthreads();
  if (!last_cta) return;
  __threadfence();
  // ---- merge the splits (only the last CTA of this (sequence, kv head))
  const float* pall = a.part + (static_cast<size_t>(m) * a.Hkv + h) * a.splits * kAttnPartStride;
  for (int i = tid; i < G * 64; i += kAttnThreads) {
    const int gg = i >> 6, d = i & 63;
    float M = -INFINITY;
    for (int s2 = 0; s2 < n_act; ++s2)
      M = fmaxf(M, *reinterpret_cast<const volatile float*>(pall + s2 * kAttnPartStride + gg * 66));
    float L = 0.0f, O = 0.0f;
    for (int s2 = 0; s2 < n_act; ++s2) {
      const volatile float* ps = pall + s2 * kAttnPartStride + gg * 66;
      const float f = expf(ps[0] - M);
      L += ps[1] * f;
      O += ps[2 + d] * f;
    }
    a.out[static_cast<size_t>(m) * Dq + (h * G + gg) * 64 + d] = O / L * sV;
  }
  if (tid == 0) a.counters[static_cast<size_t>(m) * a.Hkv + h] = 0u;
}

}  // namespace

// Chunk length and CTAs per (row, kv head): batched decode has many rows, so
// few CTAs per row; a single sequence spreads its context over more CTAs.
int attn_split_len(int M) { return M >= 16 ? 128 : 64; }
int attn_splits(int M, int P) {
  const int ts = attn_split_len(M);
  const int most = (P + ts - 1) / ts;
  return std::min(most, M >= 16 ? 4 : 16);
}

cudaError_t launch_attn_decode(const AttnDecodeArgs& a0, cudaStream_t s, bool pdl) {
  AttnDecodeArgs a = a0;
  const int G = a.H / a.Hkv;
  if (G < 1 || G > 8 || a.H % a.Hkv || !a.part || !a.counters) return cudaErrorInvalidValue;
  const int ts = attn_split_len(a.M);
  a.splits = attn_splits(a.M, a.P);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.Hkv, a.M, a.splits);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (ts == 128) return cudaLaunchKernelEx(&cfg, attn_decode_mma_kernel<128>, a);
  return cudaLaunchKernelEx(&cfg, attn_decode_mma_kernel<64>, a);
}

size_t attn_part_floats(int M, int Hkv, int P) {
  return static_cast<size_t>(M) * Hkv * attn_splits(M, P) * kAttnPartStride;
}

}  // namespace tl
