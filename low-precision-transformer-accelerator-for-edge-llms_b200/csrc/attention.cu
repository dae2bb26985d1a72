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
TL_DEV uint32_t smem_u32_attn(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
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

// ------------------------------------------------------------------ prefill
// Causal prefill attention, flash-attention style on mma.sync m16n8k16 fp16
// with the same hi/lo operand split as decode. CTA = (64-query tile, q head,
// sequence), four warps of 16 query rows; key/value tiles of 64 positions
// are read from the INT8 cache, converted once to fp16 in shared memory
// (exact) and fed to the MMAs with ldmatrix (K as the col-major B of Q.K^T,
// V transposed for P.V). The next tile's INT8 bytes are loaded into
// registers while the current tile is computed.
constexpr int kPfQTile = 64;
constexpr int kPfKTile = 64;
constexpr int kPfStride = 72;  // halves per smem row: 144 B, conflict-free ldmatrix

// four int8 in a word -> two half2 (bytes 0,1 and bytes 2,3), exact:
// 0x6400 | (b + 128) is the fp16 value 1024 + b + 128.
TL_DEV void i8x4_to_h2x2(uint32_t w, uint32_t& h01, uint32_t& h23) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t a = __byte_perm(u, 0x64646464u, 0x5140);
  const uint32_t b = __byte_perm(u, 0x64646464u, 0x5342);
  const __half2 bias = __float2half2_rn(1152.0f);
  __half2 ha = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
  __half2 hb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
  h01 = *reinterpret_cast<uint32_t*>(&ha);
  h23 = *reinterpret_cast<uint32_t*>(&hb);
}

TL_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
TL_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D += A . B with all four A registers (rows 0..15 in use)
TL_DEV void mma16816_full(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(128) attn_prefill_mma_kernel(
    const float* __restrict__ qkv, int ld, int seq_len, int H, int Hkv, const int8_t* __restrict__ kc,
    const int8_t* __restrict__ vc, const float* __restrict__ ks, const float* __restrict__ vs, int slot_base,
    int layer, int L, int P, float* __restrict__ out, float* __restrict__ out_absmax) {
  __shared__ __align__(16) __half k_sm[kPfKTile * kPfStride];
  __shared__ __align__(16) __half v_sm[kPfKTile * kPfStride];

  const int n_qt = gridDim.x;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);  // longest rows first
  const int head = blockIdx.y, seq = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q4 = lane & 3;
  const int h = head / (H / Hkv);
  const int Dq = H * 64;
  const size_t sidx = (static_cast<size_t>(slot_base + seq) * L + layer) * Hkv + h;
  const float sK = ks[sidx], sV = vs[sidx];
  const int8_t* kbase = kc + sidx * static_cast<size_t>(P) * 64;
  const int8_t* vbase = vc + sidx * static_cast<size_t>(P) * 64;

  // ---- this warp's 16 query rows: fp32 -> power-of-two scaled hi/lo fragments
  const int r0 = qt * kPfQTile + warp * 16 + g;  // rows r0 and r0 + 8
  float qv[2][16];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int t = r0 + hr * 8;
    const float* q = qkv + static_cast<size_t>(seq * seq_len + (t < seq_len ? t : 0)) * ld + head * 64;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float2 x0 = *reinterpret_cast<const float2*>(q + kk * 16 + q4 * 2);
      const float2 x1 = *reinterpret_cast<const float2*>(q + kk * 16 + 8 + q4 * 2);
      const bool ok = t < seq_len;
      qv[hr][kk * 4 + 0] = ok ? x0.x : 0.0f;
      qv[hr][kk * 4 + 1] = ok ? x0.y : 0.0f;
      qv[hr][kk * 4 + 2] = ok ? x1.x : 0.0f;
      qv[hr][kk * 4 + 3] = ok ? x1.y : 0.0f;
    }
  }
  float qscale[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(qv[hr][i]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    qscale[hr] = pow2_scale(mx);
  }
  uint32_t qa_hi[4][4], qa_lo[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    // a0: row g, k 0..1 | a1: row g+8, k 0..1 | a2: row g, k 8..9 | a3: row g+8, k 8..9
    split2(qv[0][kk * 4 + 0] * qscale[0], qv[0][kk * 4 + 1] * qscale[0], qa_hi[kk][0], qa_lo[kk][0]);
    split2(qv[1][kk * 4 + 0] * qscale[1], qv[1][kk * 4 + 1] * qscale[1], qa_hi[kk][1], qa_lo[kk][1]);
    split2(qv[0][kk * 4 + 2] * qscale[0], qv[0][kk * 4 + 3] * qscale[0], qa_hi[kk][2], qa_lo[kk][2]);
    split2(qv[1][kk * 4 + 2] * qscale[1], qv[1][kk * 4 + 3] * qscale[1], qa_hi[kk][3], qa_lo[kk][3]);
  }
  const float sc0 = sK * 0.125f / qscale[0], sc1 = sK * 0.125f / qscale[1];

  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
  float o[8][4];
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.0f;

  // ---- key/value tiles 0..qt (the causal frontier of this query tile)
  const int n_kt = qt + 1;
  // staging: thread tid moves 16 bytes of K rows and 16 bytes of V rows, twice
  int4 kreg[2], vreg[2];
  auto load_tile = [&](int kt) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = tid + i * 128;         // 16-byte chunk 0..255
      const int row = c >> 2, col = c & 3;  // key row in tile, chunk in row
      const int t = kt * kPfKTile + row;
      if (t < seq_len) {
        kreg[i] = __ldg(reinterpret_cast<const int4*>(kbase + static_cast<size_t>(t) * 64) + col);
        vreg[i] = __ldg(reinterpret_cast<const int4*>(vbase + static_cast<size_t>(t) * 64) + col);
      } else {
        kreg[i] = make_int4(0, 0, 0, 0);
        vreg[i] = make_int4(0, 0, 0, 0);
      }
    }
  };
  auto store_tile = [&]() {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = tid + i * 128;
      const int row = c >> 2, col = c & 3;
      uint4 a, b;
      i8x4_to_h2x2(static_cast<uint32_t>(kreg[i].x), a.x, a.y);
      i8x4_to_h2x2(static_cast<uint32_t>(kreg[i].y), a.z, a.w);
      i8x4_to_h2x2(static_cast<uint32_t>(kreg[i].z), b.x, b.y);
      i8x4_to_h2x2(static_cast<uint32_t>(kreg[i].w), b.z, b.w);
      uint4* kd = reinterpret_cast<uint4*>(k_sm + row * kPfStride + col * 16);
      kd[0] = a;
      kd[1] = b;
      i8x4_to_h2x2(static_cast<uint32_t>(vreg[i].x), a.x, a.y);
      i8x4_to_h2x2(static_cast<uint32_t>(vreg[i].y), a.z, a.w);
      i8x4_to_h2x2(static_cast<uint32_t>(vreg[i].z), b.x, b.y);
      i8x4_to_h2x2(static_cast<uint32_t>(vreg[i].w), b.z, b.w);
      uint4* vd = reinterpret_cast<uint4*>(v_sm + row * kPfStride + col * 16);
      vd[0] = a;
      vd[1] = b;
    }
  };

  const uint32_t k_base = smem_u32_attn(k_sm), v_base = smem_u32_attn(v_sm);
  // ldmatrix lane addresses (bytes): K, non-transposed: key = nt*8 + (lane&7),
  // dim = kk*16 + (lane>>3)*8 (matrices: kk lo, kk hi, kk+1 lo, kk+1 hi).
  const uint32_t k_lane = static_cast<uint32_t>(((lane & 7) * kPfStride + (lane >> 3) * 8) * 2);
  // V, transposed: key = kk*16 + ((lane>>3)&1)*8 + (lane&7), dim = (dt + (lane>>4))*8.
  const uint32_t v_lane = static_cast<uint32_t>(((((lane >> 3) & 1) * 8 + (lane & 7)) * kPfStride + (lane >> 4) * 8) * 2);

  load_tile(0);
  for (int kt = 0; kt < n_kt; ++kt) {
    __syncthreads();  // previous tile fully consumed
    store_tile();
    __syncthreads();
    if (kt + 1 < n_kt) load_tile(kt + 1);

    // S = Q . K^T for 16 rows x 64 keys
    float sacc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 4; kk += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(k_base + k_lane + static_cast<uint32_t>((nt * 8 * kPfStride + kk * 16) * 2), b0, b1, b2, b3);
        mma16816_full(sacc[nt], qa_hi[kk], b0, b1);
        mma16816_full(sacc[nt], qa_lo[kk], b0, b1);
        mma16816_full(sacc[nt], qa_hi[kk + 1], b2, b3);
        mma16816_full(sacc[nt], qa_lo[kk + 1], b2, b3);
      }
    }
    // scale, causal mask (diagonal tile only), online softmax
    const bool diag = kt == qt;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int hr = j >> 1;
        const int key = kt * kPfKTile + nt * 8 + q4 * 2 + (j & 1);
        const int qrow = r0 + hr * 8;
        float v = sacc[nt][j] * (hr ? sc1 : sc0);
        if (diag && key > qrow) v = -INFINITY;
        sacc[nt][j] = v;
        mx[hr] = fmaxf(mx[hr], v);
      }
    float corr[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
      const float m_new = fmaxf(m_run[hr], mx[hr]);  // finite: key 0 of a tile <= every row's position
      corr[hr] = expf(m_run[hr] - m_new);
      m_run[hr] = m_new;
      l_run[hr] *= corr[hr];
    }
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      o[dt][0] *= corr[0];
      o[dt][1] *= corr[0];
      o[dt][2] *= corr[1];
      o[dt][3] *= corr[1];
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int hr = j >> 1;
        const float e = expf(sacc[nt][j] - m_run[hr]);
        sacc[nt][j] = e;
        l_run[hr] += e;
      }
    // O += P . V, P split into hi/lo fp16 (scaled by 2^14)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t ph[4], pl[4];
      split2(sacc[2 * kk][0] * kPScale, sacc[2 * kk][1] * kPScale, ph[0], pl[0]);
      split2(sacc[2 * kk][2] * kPScale, sacc[2 * kk][3] * kPScale, ph[1], pl[1]);
      split2(sacc[2 * kk + 1][0] * kPScale, sacc[2 * kk + 1][1] * kPScale, ph[2], pl[2]);
      split2(sacc[2 * kk + 1][2] * kPScale, sacc[2 * kk + 1][3] * kPScale, ph[3], pl[3]);
#pragma unroll
      for (int dt = 0; dt < 8; dt += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(v_base + v_lane + static_cast<uint32_t>((kk * 16 * kPfStride + dt * 8) * 2), b0, b1, b2, b3);
        mma16816_full(o[dt], ph, b0, b1);
        mma16816_full(o[dt], pl, b0, b1);
        mma16816_full(o[dt + 1], ph, b2, b3);
        mma16816_full(o[dt + 1], pl, b2, b3);
      }
    }
  }

  // ---- normalise and store; per-sequence |out| maximum for the next quantize
  float local_max = 0.0f;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = l_run[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int t = r0 + hr * 8;
    if (t >= seq_len) continue;
    const float inv = sV / (l * kPScale);
    float* orow = out + static_cast<size_t>(seq * seq_len + t) * Dq + head * 64;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      const float2 y = make_float2(o[dt][hr * 2] * inv, o[dt][hr * 2 + 1] * inv);
      *reinterpret_cast<float2*>(orow + dt * 8 + q4 * 2) = y;
      local_max = fmaxf(local_max, fmaxf(fabsf(y.x), fabsf(y.y)));
    }
  }
  if (out_absmax) {
    local_max = warp_max(local_max);
    if (lane == 0) atomic_max_nonneg(out_absmax + seq, local_max);
  }
}

}  // namespace

cudaError_t launch_attn_prefill(const float* qkv, int ld, int rows, int seq_len, int H, int Hkv,
                                const int8_t* kc, const int8_t* vc, const float* ks,
                                const float* vs, int slot_base, int layer, int L, int P,
                                float* out, float* out_absmax, cudaStream_t s) {
  if (seq_len <= 0 || rows % seq_len || H % Hkv || (ld & 1)) return cudaErrorInvalidValue;
  const int nseq = rows / seq_len;
  dim3 grid((seq_len + kPfQTile - 1) / kPfQTile, H, nseq);
  attn_prefill_mma_kernel<<<grid, 128, 0, s>>>(qkv, ld, seq_len, H, Hkv, kc, vc, ks, vs, slot_base, layer,
                                               L, P, out, out_absmax);
  return cudaGetLastError();
}

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
