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
// Decode maps one CTA to (kv head, row, context split) with eight warps that
// stream 32-position chunks through bulk async copies; prefill maps one CTA
// to (64-query tile, q head, sequence). Both run flash-attention tiles on
// mma.sync m16n8k16 fp16 with fp32 accumulation: INT8 K / V values convert
// to fp16 exactly (|v| <= 127), and to keep fp32-level accuracy the fp32 Q
// and P operands are split into fp16 hi + lo halves (~22 mantissa bits).
// Each query row is first scaled by a power of two that puts its largest
// element in [2^13, 2^14) and the probabilities by 2^14, so the lo halves
// stay in fp16's normal range; the scales are exact and undone on the fp32
// accumulators. (INT8 re-quantization of the attention output makes float
// error visible as rounding flips, so attention has to be as accurate as
// fp32 arithmetic.) Decode splits merge via a per-(row, kv head) partial
// buffer, the last CTA to arrive (atomic ticket) producing the output.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace tl {

namespace {

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

// D += A . B, m16n8k32, s8 in, s32 accumulate
TL_DEV void mma16832_s8(int* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 2^x on the special-function unit (flushes subnormal results to zero)
TL_DEV float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// signed 8-bit digit of x in [-128, 127]: x = digit + 256 * rest
TL_DEV int low_digit(int x) { return ((x + 128) & 255) - 128; }
TL_DEV uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | ((static_cast<uint32_t>(d) & 0xffu) << 24);
}
constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------------------- decode
// One CTA per (kv head, row, split) with eight warps. The split's context is
// cut into 32-position chunks; warp w takes chunks w, w+8, ... and streams
// them through its own two ring slots (K 2 KB + V 2 KB each) with bulk async
// copies (cp.async.bulk, completion on a per-slot mbarrier), so every warp
// has its next chunk in flight while it computes the current one and no
// CTA-wide barrier sits in the loop. The position being decoded is not in
// the cache yet: its warp quantizes the rotated K and the V of this step,
// writes them to its slot and (for running rows) to the cache.
//
// Q.K^T runs on the INT8 MMA (m16n8k32, s32 accumulate) straight from the
// cache bytes: each rotated query row is scaled by a power of two into
// [2^21, 2^22), rounded to an integer (error <= 2^-22 of the row maximum)
// and split into three signed 8-bit digits, x = d0 + 256 d1 + 65536 d2.
// Rows 0..7 of the first MMA carry d2 of the group's eight heads and rows
// 8..15 carry d1; the second MMA carries d0 in rows 0..7. The exact INT32
// digit dot products are combined in fp32. P.V uses fp16 (m16n8k16): P hi
// halves in rows 0..7, lo halves in rows 8..15, INT8 V converted to fp16
// exactly. The softmax runs in base 2 (scores pre-multiplied by log2 e,
// ex2.approx). Head-dim and value-dim indices are permuted consistently on
// both operands so that every B fragment comes from one 16-byte (K) or
// 8-byte (V) shared load: thread (g, q4) reads K row g at bytes
// [16 q4, 16 q4 + 16) and V rows at bytes [8 g, 8 g + 8); output column n of
// value tile dt is dimension 8 n + dt.
constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecChunk = 32;                     // positions per chunk
constexpr int kDecHalf = kDecChunk * 64;          // bytes of K (or V) per chunk
constexpr int kDecSlot = 2 * kDecHalf;            // K then V
constexpr int kDecRing = kDecWarps * 2 * kDecSlot;  // two slots per warp
constexpr size_t kDecSmem = kDecRing + 8 * 64 * 4 + 8 * 4 + 2 * kDecWarps * 8 + 16;
constexpr long long kDecWaitCycles = 4000000000ll;  // ~2 s at 1.9 GHz

__device__ unsigned int g_attn_error = 0;

TL_DEV void dec_mbar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32_attn(bar)));
}
TL_DEV void dec_mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32_attn(bar)) : "memory");
}
TL_DEV void dec_mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32_attn(bar)), "r"(bytes)
               : "memory");
}
// Bounded wait on a slot's phase: false (and g_attn_error set) on expiry.
TL_DEV bool dec_mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32_attn(bar);
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kDecWaitCycles) {
      atomicCAS(&g_attn_error, 0u, 4u);
      return false;
    }
  }
}
TL_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32_attn(dst)), "l"(src), "r"(bytes), "r"(smem_u32_attn(bar))
      : "memory");
}

// chunks [0, n_chunks) split into `nz` contiguous ranges of `per` chunks
TL_DEV void dec_ranges(int n_chunks, int nz, int& per, int& n_act) {
  per = (n_chunks + nz - 1) / nz;
  n_act = (n_chunks + per - 1) / per;
}

__global__ void __launch_bounds__(kDecThreads, 2) attn_decode_kernel(AttnDecodeArgs a) {
  extern __shared__ __align__(128) unsigned char dsm[];
  unsigned char* ring = dsm;
  float* q_sm = reinterpret_cast<float*>(dsm + kDecRing);   // [8][64]
  float* q_scale = q_sm + 8 * 64;                           // [8]
  uint64_t* bars = reinterpret_cast<uint64_t*>(q_scale + 8);  // [warps][2]
  int* last_cta = reinterpret_cast<int*>(bars + 2 * kDecWarps);
  float* comb = reinterpret_cast<float*>(ring);  // [warps][8][66], after the chunk loop

  const int h = blockIdx.x, m = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q4 = lane & 3;
  const int G = a.H / a.Hkv;
  const int Dq = a.H * 64;
  // Before the dependency wait this kernel reads only state from earlier
  // steps (positions, slots, frozen KV scales, cache rows < p): the QKV GEMM
  // releases its dependents after its own wait, when every kernel before it
  // has completed. The cache chunks stream in while that GEMM finishes.
  const int p = a.pos[m];
  if (p < 0 || p >= a.P) {
    pdl_wait();
    if (sp == 0)
      for (int i = tid; i < G * 64; i += kDecThreads) a.out[static_cast<size_t>(m) * Dq + h * G * 64 + i] = 0.0f;
    return;
  }
  const int T = p + 1;
  const int n_chunks = (T + kDecChunk - 1) / kDecChunk;
  int per, n_act;
  dec_ranges(n_chunks, static_cast<int>(gridDim.z), per, n_act);
  if (sp >= n_act) return;  // no chunk for this CTA (not counted in the merge)
  const int c_begin = sp * per, c_end = min(c_begin + per, n_chunks);
  const int slot = a.slot[m];
  const bool act = a.active ? (a.active[m] != 0) : true;
  const size_t sidx = (static_cast<size_t>(slot) * a.L + a.layer) * a.Hkv + h;
  const float sK = a.ks[sidx], sV = a.vs[sidx];
  int8_t* kbase = a.kc + sidx * static_cast<size_t>(a.P) * 64;
  int8_t* vbase = a.vc + sidx * static_cast<size_t>(a.P) * 64;
  const float* row = a.qkv + static_cast<size_t>(m) * a.ld;
  const float* cs = a.cos + static_cast<size_t>(p) * 64;
  const float* sn = a.sin + static_cast<size_t>(p) * 64;

  if (tid == 0) {
    for (int i = 0; i < 2 * kDecWarps; ++i) dec_mbar_init(bars + i);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // ---- this warp's chunks and their bulk copies
  uint64_t* wbar = bars + 2 * warp;
  unsigned char* wslot = ring + warp * 2 * kDecSlot;
  const int first = c_begin + warp;
  const int nmine = first < c_end ? (c_end - first + kDecWarps - 1) / kDecWarps : 0;
  // Copies positions [t0, t0 + rows) of K and V, rows excluding position p
  // (written by the warp itself); a copy of nothing still completes the phase.
  auto issue = [&](int c, int s) {
    const int t0 = c * kDecChunk;
    const int rows = min(kDecChunk, T - t0) - ((p >= t0 && p < t0 + kDecChunk) ? 1 : 0);
    uint64_t* bar = wbar + s;
    unsigned char* dst = wslot + s * kDecSlot;
    if (rows > 0) {
      const uint32_t bytes = static_cast<uint32_t>(rows) * 64u;
      dec_mbar_expect_tx(bar, 2 * bytes);
      bulk_g2s(dst, kbase + static_cast<size_t>(t0) * 64, bytes, bar);
      bulk_g2s(dst + kDecHalf, vbase + static_cast<size_t>(t0) * 64, bytes, bar);
    } else {
      dec_mbar_arrive(bar);
    }
  };
  if (lane == 0)
    for (int i = 0; i < min(2, nmine); ++i) issue(first + i * kDecWarps, i);
  pdl_wait();
  // ---- rotated queries of the group, one head per warp, power-of-two scaled
  {
    const int gg = warp;
    float r0 = 0.0f, r1 = 0.0f;
    if (gg < G) {
      const float* qr = row + (h * G + gg) * 64;
      const float q0 = qr[lane], q1 = qr[lane + 32];
      r0 = __fadd_rn(__fmul_rn(q0, cs[lane]), __fmul_rn(-q1, sn[lane]));
      r1 = __fadd_rn(__fmul_rn(q1, cs[lane + 32]), __fmul_rn(q0, sn[lane + 32]));
    }
    // power of two taking max |q| into [2^21, 2^22): 22-bit integer queries
    const float qs = pow2_scale(warp_max(fmaxf(fabsf(r0), fabsf(r1)))) * 256.0f;
    q_sm[gg * 64 + lane] = rintf(r0 * qs);
    q_sm[gg * 64 + lane + 32] = rintf(r1 * qs);
    if (lane == 0) q_scale[gg] = qs;
  }
  __syncthreads();

  // ---- Q digit fragments. k-step ks (32 of the 64 head dims) of thread q4:
  // k 4 q4 + {0..3} <-> dims 16 q4 + 8 ks + {0..3}, k 16 + 4 q4 + {0..3} <->
  // dims 16 q4 + 8 ks + {4..7}. qa2: rows 0..7 d2, rows 8..15 d1; qa0: d0.
  uint32_t qa2[2][4], qa0[2][4];
#pragma unroll
  for (int ks = 0; ks < 2; ++ks)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const float* qr = q_sm + g * 64 + q4 * 16 + ks * 8 + half * 4;
      int d0[4], d1[4], d2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int x = static_cast<int>(qr[j]);
        d0[j] = low_digit(x);
        const int x1 = (x - d0[j]) >> 8;
        d1[j] = low_digit(x1);
        d2[j] = (x1 - d1[j]) >> 8;
      }
      qa2[ks][half * 2] = pack_s8x4(d2[0], d2[1], d2[2], d2[3]);
      qa2[ks][half * 2 + 1] = pack_s8x4(d1[0], d1[1], d1[2], d1[3]);
      qa0[ks][half * 2] = pack_s8x4(d0[0], d0[1], d0[2], d0[3]);
      qa0[ks][half * 2 + 1] = 0u;
    }
  // scores in base 2: dot * sK / 8 * log2(e), the query scale undone exactly
  const float score_scale = sK * 0.125f * kLog2e / q_scale[g];
  float m_run = -INFINITY, l_part = 0.0f;
  float o[8][4];
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.0f;

  bool ok = true;
  for (int i = 0; i < nmine && ok; ++i) {
    const int c = first + i * kDecWarps, s = i & 1;
    const int t0 = c * kDecChunk;
    const int n = min(kDecChunk, T - t0);
    ok = dec_mbar_wait(wbar + s, (i >> 1) & 1);
    if (!ok) break;
    unsigned char* ksm = wslot + s * kDecSlot;
    unsigned char* vsm = ksm + kDecHalf;
    if (p >= t0 && p < t0 + kDecChunk) {
      // the new position: RoPE(K), quantize K and V with the frozen scales
      const float* kr = row + Dq + h * 64;
      const float* vr = row + Dq + a.Hkv * 64 + h * 64;
      const float k0 = kr[lane], k1 = kr[lane + 32];
      const float r0 = __fadd_rn(__fmul_rn(k0, cs[lane]), __fmul_rn(-k1, sn[lane]));
      const float r1 = __fadd_rn(__fmul_rn(k1, cs[lane + 32]), __fmul_rn(k0, sn[lane + 32]));
      const int8_t qk0 = static_cast<int8_t>(quantize_one(r0, sK)), qk1 = static_cast<int8_t>(quantize_one(r1, sK));
      const int8_t qv0 = static_cast<int8_t>(quantize_one(vr[lane], sV));
      const int8_t qv1 = static_cast<int8_t>(quantize_one(vr[lane + 32], sV));
      const int rl = p - t0;
      ksm[rl * 64 + lane] = static_cast<unsigned char>(qk0);
      ksm[rl * 64 + lane + 32] = static_cast<unsigned char>(qk1);
      vsm[rl * 64 + lane] = static_cast<unsigned char>(qv0);
      vsm[rl * 64 + lane + 32] = static_cast<unsigned char>(qv1);
      if (act) {
        kbase[static_cast<size_t>(p) * 64 + lane] = qk0;
        kbase[static_cast<size_t>(p) * 64 + lane + 32] = qk1;
        vbase[static_cast<size_t>(p) * 64 + lane] = qv0;
        vbase[static_cast<size_t>(p) * 64 + lane + 32] = qv1;
      }
      __syncwarp();
    }
    // S = Q.K^T: 4 key tiles of 8
    float sc[4][2];
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      int a21[4] = {0, 0, 0, 0}, a0[4] = {0, 0, 0, 0};
      const uint4 kw = *reinterpret_cast<const uint4*>(ksm + (nt * 8 + g) * 64 + q4 * 16);
      mma16832_s8(a21, qa2[0], kw.x, kw.y);
      mma16832_s8(a0, qa0[0], kw.x, kw.y);
      mma16832_s8(a21, qa2[1], kw.z, kw.w);
      mma16832_s8(a0, qa0[1], kw.z, kw.w);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kl = nt * 8 + q4 * 2 + j;
        const float dot = fmaf(static_cast<float>(a21[j]), 65536.0f,
                               fmaf(static_cast<float>(a21[j + 2]), 256.0f, static_cast<float>(a0[j])));
        const float v = kl < n ? dot * score_scale : -INFINITY;
        sc[nt][j] = v;
        mx = fmaxf(mx, v);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);  // finite: position t0 < T is always valid
    const float corr = ex2f(m_run - m_new);
    m_run = m_new;
    float psum = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        sc[nt][j] = ex2f(sc[nt][j] - m_new);
        psum += sc[nt][j];
      }
    l_part = l_part * corr + psum;
    if (__any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        o[dt][0] *= corr;
        o[dt][1] *= corr;
        o[dt][2] *= corr;
        o[dt][3] *= corr;
      }
    }
    // O += P.V over two 16-key steps
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t pa[4];
      split2(sc[2 * kk][0] * kPScale, sc[2 * kk][1] * kPScale, pa[0], pa[1]);
      split2(sc[2 * kk + 1][0] * kPScale, sc[2 * kk + 1][1] * kPScale, pa[2], pa[3]);
      const int ra = kk * 16 + q4 * 2;  // keys ra, ra+1 (b0) and ra+8, ra+9 (b1)
      const uint2 A0 = *reinterpret_cast<const uint2*>(vsm + ra * 64 + g * 8);
      const uint2 A1 = *reinterpret_cast<const uint2*>(vsm + (ra + 1) * 64 + g * 8);
      const uint2 B0 = *reinterpret_cast<const uint2*>(vsm + (ra + 8) * 64 + g * 8);
      const uint2 B1 = *reinterpret_cast<const uint2*>(vsm + (ra + 9) * 64 + g * 8);
      uint32_t bl[8], bh[8];
      i8x4_to_h2x2(__byte_perm(A0.x, A1.x, 0x5140), bl[0], bl[1]);
      i8x4_to_h2x2(__byte_perm(A0.x, A1.x, 0x7362), bl[2], bl[3]);
      i8x4_to_h2x2(__byte_perm(A0.y, A1.y, 0x5140), bl[4], bl[5]);
      i8x4_to_h2x2(__byte_perm(A0.y, A1.y, 0x7362), bl[6], bl[7]);
      i8x4_to_h2x2(__byte_perm(B0.x, B1.x, 0x5140), bh[0], bh[1]);
      i8x4_to_h2x2(__byte_perm(B0.x, B1.x, 0x7362), bh[2], bh[3]);
      i8x4_to_h2x2(__byte_perm(B0.y, B1.y, 0x5140), bh[4], bh[5]);
      i8x4_to_h2x2(__byte_perm(B0.y, B1.y, 0x7362), bh[6], bh[7]);
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) mma16816_full(o[dt], pa, bl[dt], bh[dt]);
    }
    __syncwarp();  // every lane is done with this slot
    if (lane == 0 && i + 2 < nmine) issue(c + 2 * kDecWarps, s);
  }
  if (!ok && lane == 0) {
    // give copies still in flight a bounded chance to land before the slot
    // memory is reused for the merge
    for (int s = 0; s < 2; ++s) (void)dec_mbar_wait(wbar + s, 0u), (void)dec_mbar_wait(wbar + s, 1u);
  }
  pdl_launch_dependents();
  __syncthreads();  // all chunks consumed: the ring becomes the merge buffer

  // ---- merge the warps of this CTA: comb[w][head][0] = max, [1] = sum, [2 + dim] = O
  {
    float l_row = l_part;
    l_row += __shfl_xor_sync(0xffffffffu, l_row, 1);
    l_row += __shfl_xor_sync(0xffffffffu, l_row, 2);
    float* cw = comb + (warp * 8 + g) * 66;
    if (q4 == 0) {
      cw[0] = m_run;
      cw[1] = l_row;
    }
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      cw[2 + (q4 * 2) * 8 + dt] = (o[dt][0] + o[dt][2]) * (1.0f / kPScale);
      cw[2 + (q4 * 2 + 1) * 8 + dt] = (o[dt][1] + o[dt][3]) * (1.0f / kPScale);
    }
  }
  __syncthreads();
  if (n_act == 1) {
    float omax = 0.0f;  // max |output| of this thread, for the row's absmax
    for (int i = tid; i < G * 64; i += kDecThreads) {
      const int gg = i >> 6, d = i & 63;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, comb[(w * 8 + gg) * 66]);
      float L = 0.0f, O = 0.0f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) {
        const float* cw = comb + (w * 8 + gg) * 66;
        const float f = cw[0] == -INFINITY ? 0.0f : ex2f(cw[0] - M);
        L += cw[1] * f;
        O += cw[2 + d] * f;
      }
      const float y = O / L * sV;
      a.out[static_cast<size_t>(m) * Dq + (h * G + gg) * 64 + d] = y;
      omax = fmaxf(omax, fabsf(y));
    }
    if (a.out_absmax) {
      omax = warp_max(omax);
      if (lane == 0) atomic_max_nonneg(a.out_absmax + m, omax);
    }
    return;
  }
  float* part = a.part + (static_cast<size_t>(m) * a.Hkv + h) * a.splits * kAttnPartStride +
                static_cast<size_t>(sp) * kAttnPartStride;
  for (int i = tid; i < G * 64; i += kDecThreads) {
    const int gg = i >> 6, d = i & 63;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, comb[(w * 8 + gg) * 66]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float* cw = comb + (w * 8 + gg) * 66;
      const float f = cw[0] == -INFINITY ? 0.0f : ex2f(cw[0] - M);
      L += cw[1] * f;
      O += cw[2 + d] * f;
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
    *last_cta = prev == static_cast<unsigned>(n_act - 1);
  }
  __syncthreads();
  if (!*last_cta) return;
  __threadfence();
  // ---- merge the splits (only the last CTA of this (row, kv head))
  const float* pall = a.part + (static_cast<size_t>(m) * a.Hkv + h) * a.splits * kAttnPartStride;
  float omax = 0.0f;
  for (int i = tid; i < G * 64; i += kDecThreads) {
    const int gg = i >> 6, d = i & 63;
    float M = -INFINITY;
    for (int s2 = 0; s2 < n_act; ++s2)
      M = fmaxf(M, *reinterpret_cast<const volatile float*>(pall + s2 * kAttnPartStride + gg * 66));
    float L = 0.0f, O = 0.0f;
    for (int s2 = 0; s2 < n_act; ++s2) {
      const volatile float* ps = pall + s2 * kAttnPartStride + gg * 66;
      const float f = ex2f(ps[0] - M);
      L += ps[1] * f;
      O += ps[2 + d] * f;
    }
    const float y = O / L * sV;
    a.out[static_cast<size_t>(m) * Dq + (h * G + gg) * 64 + d] = y;
    omax = fmaxf(omax, fabsf(y));
  }
  if (a.out_absmax) {
    omax = warp_max(omax);
    if (lane == 0) atomic_max_nonneg(a.out_absmax + m, omax);
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

// ------------------------------------------------- prefill on tcgen05
// The same causal attention with the products on the 5th-generation tensor
// cores, as a persistent grid: one CTA per SM walks work items = (128-query
// tile, q head, sequence), longest rows first. With S = kApfSplit key slices
// per row, 32 (4 S + 1 + 3 + 4) threads:
//   warps 0 .. 4S-1  softmax: warps w, w + 4, .. share query rows 32 (w % 4)
//              .. + 31 (the TMEM lanes their warp rank may read); warp w
//              takes key slice w / 4 of each 128-key tile (128 / S keys) and
//              output dims (64 / S) (w / 4) ..;
//   warp 4S    issues the MMAs (one thread);
//   warps 4S+1 .. 4S+3  convert each tile's INT8 K rows (contiguous in the
//              cache; every 16-byte load of a lane is issued before the
//              first conversion) to fp16, the K-major B operand of
//              S = Q.K^T, in two buffers (two tiles ahead of the MMAs);
//   warps 4S+4 .. 4S+7  the same for V into its natural [key][dim] layout,
//              the MN-major B operand of O = P.V (one buffer: V_j waits for
//              PV_{j-1}, its loads do not); they also prepare each item's
//              query rows (fp16 hi/lo operands), the next item's while the
//              current one finishes.
// Per key tile j: S_j = Q_hi.K^T + Q_lo.K^T (kind::f16, fp32 accumulate)
// into TMEM columns 128 (j % 2) ..; each softmax thread reads its slice of
// S_j once, the slices of a row exchange their maxima through shared
// memory, and write P_j * 2^14 as fp16 hi + lo halves into shared-memory
// buffer j % 2 (the A operand of P.V); P_j.V_j lands in TMEM columns
// 256 + 64 (j % 2) and is folded into the fp32 registers of O two tiles
// later, so no softmax step waits for the P.V it has just fed; the MMA
// thread issues QK_{j+2} before PV_j (the softmax is the critical path).
// Numerics are those of the mma.sync kernel above (exact fp16 K / V, hi/lo
// Q and P, fp32 accumulation, base-2 online softmax).
constexpr int kApfRows = 128;
constexpr int kApfKeys = 128;
constexpr int kApfSplit = 2;                       // key slices per row
constexpr int kApfSoftWarps = 4 * kApfSplit;
constexpr int kApfSliceKeys = kApfKeys / kApfSplit;  // 64
constexpr int kApfSliceDims = 64 / kApfSplit;        // 32
constexpr int kApfConvK = 3, kApfConvV = 4;        // converter warps per operand
constexpr int kApfThreads = 32 * (kApfSoftWarps + 1 + kApfConvK + kApfConvV);
constexpr int kApfWarpMma = kApfSoftWarps, kApfWarpConvK = kApfSoftWarps + 1;
constexpr int kApfOffQHi = 0;          // [128 rows][64 dims] fp16, SW128 K-major (16 KB)
constexpr int kApfOffQLo = 16384;
constexpr int kApfOffK = 32768;        // [2 bufs][128 keys][64 dims] fp16, SW128 K-major
constexpr int kApfOffV = 65536;        // [128 keys][64 dims] fp16, SW128 MN-major
constexpr int kApfOffP = 81920;        // [2 bufs][hi | lo][2 key blocks][128 rows][64 keys] fp16, SW128
constexpr int kApfPBuf = 65536;
constexpr int kApfOffXch = 212992;     // floats: [2 tiles][S][128] row maxima, [S][128] l, [128] scale
constexpr int kApfOffBar = kApfOffXch + (3 * kApfSplit * 128 + 128) * 4;
constexpr size_t kApfSmem = kApfOffBar + 256 + 1024;
constexpr uint32_t kApfTmemCols = 512;  // S x 2 (256) + O tile x 2 (128), rounded up

__device__ unsigned int g_apf_error = 0;

// TL_DISABLE_TC_ATTN_PREFILL=1 keeps prefill attention on the mma.sync
// kernel (A/B comparisons).
bool use_apf_tc() {
  static const bool disabled = [] {
    const char* v = std::getenv("TL_DISABLE_TC_ATTN_PREFILL");
    return v && v[0] == '1';
  }();
  return !disabled;
}
TL_DEV bool apf_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  return mbar_wait_err(bar, parity, code, &g_apf_error);
}
// MN-major SW128 operand whose MN extent is one 128-byte swizzle row: both
// offsets = 1024 B (the 8-row group stride along K; the MN-direction
// stride is never used).
TL_DEV uint64_t smem_desc_sw128_mn(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (64ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}
// fp32 pair -> fp16 hi (x rounded to 11 significant bits in the integer
// domain: half an ulp added to the magnitude bits, the 13 low mantissa bits
// cleared; exactly representable in fp16) and fp16 lo (the exact fp32
// remainder, |lo| <= ulp / 2, rounded): two packed conversions per pair,
// ~22 bits kept, like split2.
TL_DEV float round11(float x) { return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u); }
TL_DEV void split2_fast(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const float h0 = round11(x0), h1 = round11(x1);
  hi = pack2(h0, h1);
  lo = pack2(x0 - h0, x1 - h1);
}
// A converter thread's share of one 128-row INT8 tile (64-byte rows): the
// 16-byte chunks t, t + T, .. (T = threads converting this operand, at most
// six each); rows >= `rows` read as zero (the cache's last position).
constexpr int kApfConvMax = 6;
struct ApfChunks {
  uint4 w[kApfConvMax];
};
TL_DEV void apf_load_rows(const unsigned char* src, int t, int T, int rows, ApfChunks& c) {
#pragma unroll
  for (int i = 0; i < kApfConvMax; ++i) {
    const int unit = t + T * i, r = unit >> 2;
    c.w[i] = (unit < 512 && r < rows) ? __ldg(reinterpret_cast<const uint4*>(src + unit * 16)) : make_uint4(0u, 0u, 0u, 0u);
  }
}
// ... converted to fp16 rows SW128: each 16-byte chunk (16 values) becomes
// two swizzled 16-byte chunks.
TL_DEV void apf_store_rows(unsigned char* dst, int t, int T, const ApfChunks& c) {
#pragma unroll
  for (int i = 0; i < kApfConvMax; ++i) {
    const int unit = t + T * i, r = unit >> 2, k = unit & 3;
    if (unit >= 512) break;
    uint4 a, e;
    i8x4_to_h2x2(c.w[i].x, a.x, a.y);
    i8x4_to_h2x2(c.w[i].y, a.z, a.w);
    i8x4_to_h2x2(c.w[i].z, e.x, e.y);
    i8x4_to_h2x2(c.w[i].w, e.z, e.w);
    *reinterpret_cast<uint4*>(dst + sw128_offset(r, 2 * k)) = a;
    *reinterpret_cast<uint4*>(dst + sw128_offset(r, 2 * k + 1)) = e;
  }
}

// Work item `it` of the persistent grid, longest query rows first: query
// tile qt (rows 128 qt ..), q head, sequence, its kv head and cache index.
struct ApfItem {
  int qt, head, seq;
  size_t sidx;
};
TL_DEV ApfItem apf_item(int it, int n_qt, int H, int Hkv, int nseq, int slot_base, int L, int layer) {
  const int per = H * nseq;
  ApfItem w;
  w.qt = n_qt - 1 - it / per;
  const int rem = it % per;
  w.head = rem % H;
  w.seq = rem / H;
  w.sidx = (static_cast<size_t>(slot_base + w.seq) * L + layer) * Hkv + w.head / (H / Hkv);
  return w;
}

// Query row `row` of item w -> power-of-two scaled fp16 hi/lo operand rows
// and the row's score scale (without the K scale) in xsc; the sixteen
// 16-byte loads are in flight before the first use.
TL_DEV void apf_prep_q_row(unsigned char* sm, float* xsc, const float* qkv, int ld, int seq_len, const ApfItem& w,
                           int row) {
  const int t = w.qt * kApfRows + row;
  const float4* q4 = reinterpret_cast<const float4*>(
      qkv + static_cast<size_t>(w.seq * seq_len + (t < seq_len ? t : 0)) * ld + w.head * 64);
  float4 x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = t < seq_len ? __ldg(q4 + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x[i].x), fabsf(x[i].y)), fmaxf(fabsf(x[i].z), fabsf(x[i].w))));
  const float qs = pow2_scale(mx);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 hi, lo;
    split2_fast(x[2 * c].x * qs, x[2 * c].y * qs, hi.x, lo.x);
    split2_fast(x[2 * c].z * qs, x[2 * c].w * qs, hi.y, lo.y);
    split2_fast(x[2 * c + 1].x * qs, x[2 * c + 1].y * qs, hi.z, lo.z);
    split2_fast(x[2 * c + 1].z * qs, x[2 * c + 1].w * qs, hi.w, lo.w);
    const uint32_t off = sw128_offset(row, c);
    *reinterpret_cast<uint4*>(sm + kApfOffQHi + off) = hi;
    *reinterpret_cast<uint4*>(sm + kApfOffQLo + off) = lo;
  }
  // (the K scale is applied by the softmax threads: sc2 = xsc * sK, the same
  // single rounding of sK * log2 e as sK * 0.125 * log2 e / qs)
  xsc[row] = 0.125f * kLog2e / qs;
}

__global__ void __launch_bounds__(kApfThreads, 1) attn_prefill_tc_kernel(
    const float* __restrict__ qkv, int ld, int seq_len, int nseq, int H, int Hkv, const int8_t* __restrict__ kc,
    const int8_t* __restrict__ vc, const float* __restrict__ ks, const float* __restrict__ vs, int slot_base,
    int layer, int L, int P, float* __restrict__ out, float* __restrict__ out_absmax) {
  extern __shared__ __align__(1024) unsigned char apf_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(apf_raw) + 1023) & ~uintptr_t(1023));
  float* xmax = reinterpret_cast<float*>(sm + kApfOffXch);   // [2 tiles][S][128]
  float* xl = xmax + 2 * kApfSplit * 128;                      // [S][128] final l
  float* xsc = xl + kApfSplit * 128;                           // [128] row score scales
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kApfOffBar);
  uint64_t* k_full = bar + 0;       // [2] fp16 K operand of tile g written to buffer g % 2
  uint64_t* k_free = bar + 2;       // [2] S MMAs reading buffer g % 2 completed
  uint64_t* v_full = bar + 6;       // fp16 V operand written
  uint64_t* v_free = bar + 7;       // P.V MMAs reading it completed
  uint64_t* s_full = bar + 8;       // [2] S_g in TMEM
  uint64_t* s_free = bar + 10;      // [2] the softmax warps have read S_g
  uint64_t* p_full = bar + 12;      // [2] P_g written to buffer g % 2
  uint64_t* o_full = bar + 14;      // [2] P_g.V_g in TMEM; P buffer g % 2 no longer read
  uint64_t* xbar = bar + 16;        // [4] the softmax warps of rows 32 q .. exchanged values
  uint64_t* q_full = bar + 20;      // an item's Q operands and row scales written (V converter warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 21);

  // Tiles are numbered g = 0, 1, .. across this CTA's items (every role
  // walks the same items in the same order); all buffer indices and mbarrier
  // phases follow g, so an item's first tiles wait on the previous item's
  // last ones exactly as within an item.
  const int n_qt = (seq_len + kApfRows - 1) / kApfRows;
  const int items = n_qt * H * nseq;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Dq = H * 64;

  if (tid == 0) {
    for (int i = 0; i < 8; ++i) mbar_init(bar + i, 1);
    for (int i = 0; i < 2; ++i) mbar_init(k_full + i, kApfConvK);
    mbar_init(v_full, kApfConvV);
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(s_free + i, kApfSoftWarps);
      mbar_init(p_full + i, kApfSoftWarps);
      mbar_init(o_full + i, 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(xbar + i, 32 * kApfSplit);
    mbar_init(q_full, kApfConvV);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kApfWarpMma) tmem_alloc(tmem_slot, kApfTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kApfWarpMma) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(kApfRows, kApfKeys);
      constexpr uint32_t id_o = idesc_f16(kApfRows, 64) | (1u << 16);  // B (V) MN-major
      // descriptor start fields advance in 16-byte units: +2 per 32-byte K
      // step, +1024 per 16 KB key block, +128 per 2 KB (16 MN-major V rows)
      const uint64_t dqh = smem_desc_sw128(smem_u32(sm + kApfOffQHi));
      const uint64_t dql = smem_desc_sw128(smem_u32(sm + kApfOffQLo));
      const uint64_t dk0 = smem_desc_sw128(smem_u32(sm + kApfOffK));
      const uint64_t dv = smem_desc_sw128_mn(smem_u32(sm + kApfOffV));
      const uint64_t dp = smem_desc_sw128(smem_u32(sm + kApfOffP));
      auto issue_qk = [&](int g) -> bool {
        const int b = g & 1, u = g >> 1;
        if (!apf_wait(k_full + b, u & 1, 22u)) return false;
        if (u > 0 && !apf_wait(s_free + b, (u - 1) & 1, 23u)) return false;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * kApfKeys);
        const uint64_t dk = dk0 + static_cast<uint64_t>(b * 1024);  // + 16 KB
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_f16(d, dqh + 2 * kk, dk + 2 * kk, id_s, kk > 0 ? 1u : 0u);
          mma_f16(d, dql + 2 * kk, dk + 2 * kk, id_s, 1u);
        }
        mma_commit(s_full + b);
        mma_commit(k_free + b);
        return true;
      };
      auto issue_pv = [&](int g) -> bool {
        const int b = g & 1, u = g >> 1;
        if (!apf_wait(p_full + b, u & 1, 24u)) return false;
        if (!apf_wait(v_full, g & 1, 25u)) return false;
        tc_fence_after();
        const uint32_t d = tmem + 256u + static_cast<uint32_t>(64 * b);
        const uint64_t pbuf = dp + static_cast<uint64_t>(b * (kApfPBuf >> 4));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t dph = pbuf + (kk >> 2) * 1024 + (kk & 3) * 2;
          mma_f16(d, dph, dv + kk * 128, id_o, kk > 0 ? 1u : 0u);
          mma_f16(d, dph + 2048, dv + kk * 128, id_o, 1u);  // lo halves: +32 KB
        }
        mma_commit(o_full + b);
        mma_commit(v_free);
        return true;
      };
      bool ok = true;
      int g0 = 0, itc = 0;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++itc) {
        const ApfItem w = apf_item(it, n_qt, H, Hkv, nseq, slot_base, L, layer);
        const int n_kt = w.qt + 1;  // key tiles 0..qt cover positions 0..128 qt + 127
        ok = apf_wait(q_full, itc & 1, 20u);
        if (ok) ok = issue_qk(g0);
        if (ok && n_kt > 1) ok = issue_qk(g0 + 1);
        for (int j = 0; j < n_kt && ok; ++j) {
          if (j + 2 < n_kt) ok = issue_qk(g0 + j + 2);
          if (ok) ok = issue_pv(g0 + j);
        }
        g0 += n_kt;
      }
    }
  } else if (warp >= kApfWarpConvK) {
    // K (S operand): tile g into buffer g % 2 once QK_{g-2} completed.
    // V (P.V operand): tile g once PV_{g-1} completed; the V warps also
    // prepare each item's Q rows (one per thread), the next item's once the
    // softmax warps have read the current item's last S (so the current Q
    // and row scales are no longer needed). Each tile's loads go first.
    const bool is_v = warp >= kApfWarpConvK + kApfConvK;
    const int T = 32 * (is_v ? kApfConvV : kApfConvK);
    const int ct = tid - 32 * (is_v ? kApfWarpConvK + kApfConvK : kApfWarpConvK);
    int g = 0;
    bool ok = true;
    if (is_v && static_cast<int>(blockIdx.x) < items) {
      apf_prep_q_row(sm, xsc, qkv, ld, seq_len, apf_item(blockIdx.x, n_qt, H, Hkv, nseq, slot_base, L, layer), ct);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const ApfItem w = apf_item(it, n_qt, H, Hkv, nseq, slot_base, L, layer);
      const int n_kt = w.qt + 1;
      const unsigned char* rows =
          reinterpret_cast<const unsigned char*>(is_v ? vc : kc) + w.sidx * static_cast<size_t>(P) * 64;
      for (int j = 0; j < n_kt && ok; ++j, ++g) {
        const int b = g & 1, u = g >> 1;
        const int kv0 = j * kApfKeys;
        ApfChunks c;
        apf_load_rows(rows + static_cast<size_t>(kv0) * 64, ct, T, min(kApfKeys, P - kv0), c);
        if (is_v) {
          if (g > 0 && !(ok = apf_wait(v_free, (g - 1) & 1, 27u))) break;
          apf_store_rows(sm + kApfOffV, ct, T, c);
        } else {
          if (u > 0 && !(ok = apf_wait(k_free + b, (u - 1) & 1, 26u))) break;
          apf_store_rows(sm + kApfOffK + b * 16384, ct, T, c);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(is_v ? v_full : k_full + b);
      }
      const int next = it + static_cast<int>(gridDim.x);
      if (is_v && ok && next < items) {
        const int gl = g - 1;  // this item's last tile
        if (!(ok = apf_wait(s_free + (gl & 1), (gl >> 1) & 1, 21u))) break;
        apf_prep_q_row(sm, xsc, qkv, ld, seq_len, apf_item(next, n_qt, H, Hkv, nseq, slot_base, L, layer), ct);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);
      }
    }
  } else {
    // softmax warps: row r, key slice ks_ (keys kApfSliceKeys ks_ ..), dims kApfSliceDims ks_ ..
    const int qq = warp & 3, ks_ = warp >> 2;
    const int r = qq * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(qq * 32) << 16);
    uint32_t xph = 0;  // phases of xbar[qq] completed so far
    float o[kApfSliceDims];
    auto fold = [&](int gg, float scale) -> bool {
      // o += scale * (P_gg . V_gg) for this slice's dims
      if (!apf_wait(o_full + (gg & 1), (gg >> 1) & 1, 30u)) return false;
      tc_fence_after();
#pragma unroll
      for (int hh = 0; hh < kApfSliceDims / 16; ++hh) {
        int w16[16];
        tmem_ld16(lane_base + 256u + static_cast<uint32_t>(64 * (gg & 1) + kApfSliceDims * ks_ + 16 * hh), w16);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[16 * hh + i] = fmaf(__int_as_float(w16[i]), scale, o[16 * hh + i]);
      }
      return true;
    };
    bool ok = true;
    int g0 = 0, itc = 0;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++itc) {
      const ApfItem w = apf_item(it, n_qt, H, Hkv, nseq, slot_base, L, layer);
      const int qt = w.qt, n_kt = qt + 1;
      const int t = qt * kApfRows + r;
      const float sk = __ldg(ks + w.sidx);
      if (!(ok = apf_wait(q_full, itc & 1, 28u))) break;  // the row scales in xsc
      const float sc2 = xsc[r] * sk;
      float m2 = -INFINITY, l = 0.0f;  // running max (log2 units), running sum of p * 2^14 (this slice)
      float c_prev = 1.0f;             // correction of the previous tile (m_{j-2} -> m_{j-1})
#pragma unroll
      for (int i = 0; i < kApfSliceDims; ++i) o[i] = 0.0f;
      for (int j = 0; j < n_kt && ok; ++j) {
        const int g = g0 + j, b = g & 1, u = g >> 1;
        if (!(ok = apf_wait(s_full + b, u & 1, 29u))) break;
        tc_fence_after();
        const bool diag = j == qt;
        const int lim = t - j * kApfKeys - kApfSliceKeys * ks_;  // keys k > lim of this slice are masked
        const uint32_t sb = lane_base + static_cast<uint32_t>(b * kApfKeys + kApfSliceKeys * ks_);
        // row maximum of the raw scores (the scale is positive), 32 columns at
        // a time in 8-way trees, then across the row's slices through shared
        // memory (double-buffered by tile parity: a warp writes buffer b again
        // only after every partner's arrival for tile g + 1, which follows its
        // read of tile g)
        float mraw = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < kApfSliceKeys / 32; ++cc) {
          uint32_t v[32];
          tmem_ld32(sb + 32 * cc, v);
          if (diag) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (32 * cc + i > lim) v[i] = __float_as_uint(-INFINITY);
          }
          float mq[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            mq[i] = fmaxf(fmaxf(__uint_as_float(v[i]), __uint_as_float(v[i + 8])),
                          fmaxf(__uint_as_float(v[i + 16]), __uint_as_float(v[i + 24])));
          mraw = fmaxf(mraw, fmaxf(fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])),
                                   fmaxf(fmaxf(mq[4], mq[5]), fmaxf(mq[6], mq[7]))));
        }
        xmax[(b * kApfSplit + ks_) * 128 + r] = mraw;
        mbar_arrive(xbar + qq);
        if (!(ok = apf_wait(xbar + qq, xph & 1, 32u))) break;
        ++xph;
        mraw = xmax[(b * kApfSplit) * 128 + r];
#pragma unroll
        for (int k = 1; k < kApfSplit; ++k) mraw = fmaxf(mraw, xmax[(b * kApfSplit + k) * 128 + r]);
        const float m_new = fmaxf(m2, mraw * sc2);
        const float corr = ex2f(m2 - m_new);
        m2 = m_new;
        // o holds tiles <= j - 3 at max m_{j-1}; P_{j-2}.V_{j-2} is at m_{j-2}.
        // Its completion also frees P buffer b for P_j (for j < 2 the previous
        // item's final folds have waited for P_{g-2}.V_{g-2} already).
#pragma unroll
        for (int i = 0; i < kApfSliceDims; ++i) o[i] *= corr;
        if (j >= 2 && !(ok = fold(g - 2, c_prev * corr))) break;
        c_prev = corr;
        // p * 2^14 = 2^(s * sc2 - m + 14) (masked scores are -inf: p = 0) as
        // fp16 hi + lo into this slice's chunks of P buffer b; l sums the p in
        // an 8-way tree
        const float off14 = 14.0f - m_new;
        float lq[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) lq[i] = 0.0f;
        unsigned char* pb = sm + kApfOffP + b * kApfPBuf;
#pragma unroll
        for (int cc = 0; cc < kApfSliceKeys / 32; ++cc) {
          uint32_t v[32];
          tmem_ld32(sb + 32 * cc, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const bool live = !diag || 32 * cc + i <= lim;
            const float p = live ? ex2f(fmaf(__uint_as_float(v[i]), sc2, off14)) : 0.0f;
            v[i] = __float_as_uint(p);
            lq[i & 7] += p;
          }
#pragma unroll
          for (int gq = 0; gq < 4; ++gq) {
            uint4 hi, lo;
            split2_fast(__uint_as_float(v[8 * gq + 0]), __uint_as_float(v[8 * gq + 1]), hi.x, lo.x);
            split2_fast(__uint_as_float(v[8 * gq + 2]), __uint_as_float(v[8 * gq + 3]), hi.y, lo.y);
            split2_fast(__uint_as_float(v[8 * gq + 4]), __uint_as_float(v[8 * gq + 5]), hi.z, lo.z);
            split2_fast(__uint_as_float(v[8 * gq + 6]), __uint_as_float(v[8 * gq + 7]), hi.w, lo.w);
            const int key = kApfSliceKeys * ks_ + 32 * cc + 8 * gq;
            const uint32_t off = static_cast<uint32_t>((key >> 6) * 16384) + sw128_offset(r, (key & 63) >> 3);
            *reinterpret_cast<uint4*>(pb + off) = hi;
            *reinterpret_cast<uint4*>(pb + 32768 + off) = lo;
          }
        }
        l = fmaf(l, corr, ((lq[0] + lq[1]) + (lq[2] + lq[3])) + ((lq[4] + lq[5]) + (lq[6] + lq[7])));
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(s_free + b);
          mbar_arrive(p_full + b);
        }
      }
      if (!ok) break;
      // the last two tiles' P.V: P_{J-1}.V_{J-1} at m_{J-1} (scaled by the last
      // correction), P_J.V_J at the final maximum
      const int gJ = g0 + n_kt - 1;
      if (n_kt >= 2 && !(ok = fold(gJ - 1, c_prev))) break;
      if (!(ok = fold(gJ, 1.0f))) break;
      // the row's l is the sum of its slices' (same running maximum)
      xl[ks_ * 128 + r] = l;
      mbar_arrive(xbar + qq);
      if (!(ok = apf_wait(xbar + qq, xph & 1, 33u))) break;
      ++xph;
      float lt = xl[r];
#pragma unroll
      for (int k = 1; k < kApfSplit; ++k) lt += xl[k * 128 + r];
      float local_max = 0.0f;
      if (t < seq_len) {
        const float inv = vs[w.sidx] / lt;
        float* orow = out + static_cast<size_t>(w.seq * seq_len + t) * Dq + w.head * 64 + kApfSliceDims * ks_;
#pragma unroll
        for (int d = 0; d < kApfSliceDims; d += 4) {
          const float4 y = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
          *reinterpret_cast<float4*>(orow + d) = y;
          local_max = fmaxf(local_max, fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w))));
        }
      }
      if (out_absmax) {
        local_max = warp_max(local_max);
        if (lane == 0) atomic_max_nonneg(out_absmax + w.seq, local_max);
      }
      g0 += n_kt;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kApfWarpMma) tmem_free(tmem, kApfTmemCols);
}


// ---------------------------------------------- prefill, two q-tile streams
// Causal prefill attention with K / V as fp16 rows in global memory (written
// once per layer by the cache-write kernel: the INT8 values, exact) and two
// independent work streams per CTA that share the SM's tensor core. Stream s
// of CTA b takes the CTA's work items b + (2k + s) * gridDim.x (longest query
// tiles first). Per stream: one load warp (lane 0 issues the TMA loads of the
// 64-key K and V tiles, each double-buffered and released separately: K once
// its S is computed, V once its P.V is), one MMA warp (lane 0 issues
// S = (Q_hi + Q_lo) . K^T and O = (P_hi + P_lo) . V) and four softmax warps,
// one thread per query row (so no row maximum is exchanged between threads).
// S is double-buffered in TMEM: S_{g+2} is issued as soon as P_g.V_g has
// completed, while the softmax threads work on S_{g+1}. P is written back
// into the TMEM columns of its S (hi and lo halves of each 16-key group side
// by side) and read from there as the A operand of P.V. P_g.V_g accumulates
// fresh in O buffer g % 2 and is folded into the softmax thread's registers
// two tiles later with the online-softmax correction (as in
// attn_prefill_tc_kernel). Numerics are those of attn_prefill_tc_kernel:
// fp16 hi + lo halves of the power-of-two scaled query and of the
// probabilities (~22 significant bits), fp32 accumulation, base-2 softmax.
//
// TMEM per stream s (columns 256 s ..): S / P buffers [0, 64) and [64, 128),
// O buffers [128, 192) and [192, 256). Shared memory per stream (64 KB): Q hi,
// Q lo (16 KB each, SW128 K-major), K tiles x 2, V tiles x 2 (8 KB each, TMA
// SW128 boxes of 64 rows).
constexpr int kPpRows = 128, kPpKeys = 64;
constexpr int kPpWarps = 12;  // per stream: load, MMA; then 4 + 4 softmax warps (warps 4-7, 8-11)
constexpr int kPpThreads = 32 * kPpWarps;
constexpr int kPpStreamBytes = 65536;
constexpr int kPpTile = kPpKeys * 128;  // bytes of one K or V tile
constexpr int kPpOffQHi = 0, kPpOffQLo = 16384, kPpOffK = 32768, kPpOffV = 32768 + 2 * kPpTile;
constexpr int kPpOffBar = 2 * kPpStreamBytes;
constexpr int kPpBarsPerStream = 16;
constexpr size_t kPpSmem = kPpOffBar + 2 * kPpBarsPerStream * 8 + 16 + 1024;

// TL_DISABLE_PP_ATTN_PREFILL=1 keeps prefill attention on attn_prefill_tc_kernel (A/B).
bool use_apf_pp() {
  static const bool disabled = [] {
    const char* v = std::getenv("TL_DISABLE_PP_ATTN_PREFILL");
    return v && v[0] == '1';
  }();
  return !disabled;
}

struct PpBars {
  uint64_t *q_full, *k_full, *k_free, *v_full, *v_free, *s_full, *p_full, *o_full, *o_free;
};
TL_DEV PpBars pp_bars(unsigned char* sm, int s) {
  uint64_t* b = reinterpret_cast<uint64_t*>(sm + kPpOffBar) + s * kPpBarsPerStream;
  return PpBars{b, b + 1, b + 3, b + 5, b + 7, b + 9, b + 11, b + 12, b + 14};
}
// Query row `row` of item w, power-of-two scaled, into the stream's fp16 hi /
// lo operand rows; returns the row's score scale without the K scale.
TL_DEV float pp_prep_q_row(unsigned char* qs, const float* qkv, int ld, int seq_len, const ApfItem& w, int row) {
  const int t = w.qt * kPpRows + row;
  const float4* q4 = reinterpret_cast<const float4*>(
      qkv + static_cast<size_t>(w.seq * seq_len + (t < seq_len ? t : 0)) * ld + w.head * 64);
  float4 x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = t < seq_len ? __ldg(q4 + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x[i].x), fabsf(x[i].y)), fmaxf(fabsf(x[i].z), fabsf(x[i].w))));
  const float qsc = pow2_scale(mx);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 hi, lo;
    split2_fast(x[2 * c].x * qsc, x[2 * c].y * qsc, hi.x, lo.x);
    split2_fast(x[2 * c].z * qsc, x[2 * c].w * qsc, hi.y, lo.y);
    split2_fast(x[2 * c + 1].x * qsc, x[2 * c + 1].y * qsc, hi.z, lo.z);
    split2_fast(x[2 * c + 1].z * qsc, x[2 * c + 1].w * qsc, hi.w, lo.w);
    const uint32_t off = sw128_offset(row, c);
    *reinterpret_cast<uint4*>(qs + kPpOffQHi + off) = hi;
    *reinterpret_cast<uint4*>(qs + kPpOffQLo + off) = lo;
  }
  return 0.125f * kLog2e / qsc;
}

// Row maximum of the tile's 64 raw scores in TMEM (keys > lim masked when
// MASK: the tiles on the diagonal), 16 columns per load with the next load
// in flight.
template <bool MASK>
TL_DEV float pp_row_max(uint32_t base, int lim) {
  int a[16], b[16];
  float m = -INFINITY;
  tmem_ld16_nw(base, a);
  tmem_ld_wait16(a);
#pragma unroll
  for (int h = 0; h < kPpKeys / 16; ++h) {
    if (h + 1 < kPpKeys / 16) tmem_ld16_nw(base + 16u * (h + 1), b);
    float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float x = (MASK && 16 * h + i > lim) ? -INFINITY : __int_as_float(a[i]);
      mq[i & 3] = fmaxf(mq[i & 3], x);
    }
    m = fmaxf(m, fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])));
    if (h + 1 < kPpKeys / 16) {
      tmem_ld_wait16(b);
#pragma unroll
      for (int i = 0; i < 16; ++i) a[i] = b[i];
    }
  }
  return m;
}
// p * 2^14 = 2^(s * sc2 + off14) of the tile's 64 scores (masked keys: 0),
// written back over the S columns just read as fp16 hi + lo (keys 16 h ..
// + 15: 8 hi words at column 16 h, 8 lo words at 16 h + 8); returns the sum
// of the p (8-way tree). Loads pipelined one ahead as in pp_row_max.
template <bool MASK>
TL_DEV float pp_exp_store(uint32_t base, int lim, float sc2, float off14) {
  int a[16], b[16];
  float lq[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) lq[i] = 0.0f;
  tmem_ld16_nw(base, a);
  tmem_ld_wait16(a);
#pragma unroll
  for (int h = 0; h < kPpKeys / 16; ++h) {
    if (h + 1 < kPpKeys / 16) tmem_ld16_nw(base + 16u * (h + 1), b);
    float p[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      p[i] = (MASK && 16 * h + i > lim) ? 0.0f : ex2f(fmaf(__int_as_float(a[i]), sc2, off14));
      lq[i & 7] += p[i];
    }
    uint32_t hi[8], lo[8];
#pragma unroll
    for (int q2 = 0; q2 < 8; ++q2) split2_fast(p[2 * q2], p[2 * q2 + 1], hi[q2], lo[q2]);
    tmem_st8(base + 16u * h, hi);
    tmem_st8(base + 16u * h + 8u, lo);
    if (h + 1 < kPpKeys / 16) {
      tmem_ld_wait16(b);
#pragma unroll
      for (int i = 0; i < 16; ++i) a[i] = b[i];
    }
  }
  return ((lq[0] + lq[1]) + (lq[2] + lq[3])) + ((lq[4] + lq[5]) + (lq[6] + lq[7]));
}

__global__ void __launch_bounds__(kPpThreads, 1) attn_prefill_pp_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, const float* __restrict__ qkv,
    int ld, int seq_len, int nseq, int H, int Hkv, const float* __restrict__ ks, const float* __restrict__ vs,
    int slot_base, int layer, int L, float* __restrict__ out, float* __restrict__ out_absmax) {
  extern __shared__ __align__(1024) unsigned char pp_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(pp_raw) + 1023) & ~uintptr_t(1023));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kPpOffBar + 2 * kPpBarsPerStream * 8);
  const int n_qt = (seq_len + kPpRows - 1) / kPpRows;
  const int items = n_qt * H * nseq;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Dq = H * 64, G = H / Hkv;

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      const PpBars b = pp_bars(sm, s);
      mbar_init(b.q_full, 4);
      mbar_init(b.p_full, 4);
      for (int i = 0; i < 2; ++i) {
        mbar_init(b.k_full + i, 1);
        mbar_init(b.k_free + i, 1);
        mbar_init(b.v_full + i, 1);
        mbar_init(b.v_free + i, 1);
        mbar_init(b.s_full + i, 1);
        mbar_init(b.o_full + i, 1);
        mbar_init(b.o_free + i, 4);
      }
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_k)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_v)) : "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int s = warp < 4 ? (warp >> 1) : (warp >> 3);  // this warp's stream
  unsigned char* ss = sm + s * kPpStreamBytes;
  const PpBars bb = pp_bars(sm, s);
  const uint32_t tm_s = tmem + 256u * static_cast<uint32_t>(s);
  const int stride = static_cast<int>(gridDim.x);
  // k-th work item of this stream (>= items: none); key tiles of query tile qt
  auto item_of = [&](int k) { return static_cast<int>(blockIdx.x) + (2 * k + s) * stride; };
  auto tiles_of = [&](int qt) { return 2 * qt + 2; };

  if (warp < 4 && (warp & 1) == 0) {
    // ---- load warp: K tile g + 2 once S_g is computed, V tile g + 2 once P_g.V_g is
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int k = 0; ok && item_of(k) < items; ++k) {
        const ApfItem w = apf_item(item_of(k), n_qt, H, Hkv, nseq, slot_base, L, layer);
        const int row0 = (w.seq * Hkv + w.head / G) * seq_len;
        const int n_kt = tiles_of(w.qt);
        for (int j = 0; j < n_kt && ok; ++j, ++g) {
          const int b = g & 1;
          const uint32_t ph = ((g - 2) >> 1) & 1;
          if (g >= 2 && !(ok = apf_wait(bb.k_free + b, ph, 40u))) break;
          mbar_arrive_expect_tx(bb.k_full + b, static_cast<uint32_t>(kPpTile));
          tma_load_2d(ss + kPpOffK + b * kPpTile, &tm_k, 0, row0 + j * kPpKeys, bb.k_full + b);
          if (g >= 2 && !(ok = apf_wait(bb.v_free + b, ph, 39u))) break;
          mbar_arrive_expect_tx(bb.v_full + b, static_cast<uint32_t>(kPpTile));
          tma_load_2d(ss + kPpOffV + b * kPpTile, &tm_v, 0, row0 + j * kPpKeys, bb.v_full + b);
        }
      }
      // after a failed wait anywhere, the copies issued last get a bounded
      // chance to land before the CTA exits
      if (*reinterpret_cast<volatile unsigned int*>(&g_apf_error) != 0u)
        for (int i = g >= 2 ? g - 2 : 0; i < g; ++i) {
          (void)apf_wait(bb.k_full + (i & 1), (i >> 1) & 1, 41u);
          (void)apf_wait(bb.v_full + (i & 1), (i >> 1) & 1, 41u);
        }
    }
  } else if (warp < 4) {
    // ---- MMA warp
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(kPpRows, kPpKeys);
      constexpr uint32_t id_o = idesc_f16(kPpRows, 64) | (1u << 16);  // B (V) MN-major
      const uint64_t dqh = smem_desc_sw128(smem_u32(ss + kPpOffQHi));
      const uint64_t dql = smem_desc_sw128(smem_u32(ss + kPpOffQLo));
      const uint64_t dk0 = smem_desc_sw128(smem_u32(ss + kPpOffK));
      const uint64_t dv0 = smem_desc_sw128_mn(smem_u32(ss + kPpOffV));
      // S_gg into S buffer gg % 2, once K tile gg is in and P_{gg-2}.V_{gg-2}
      // (the buffer's previous P) has completed
      auto issue_qk = [&](int gg) -> bool {
        const int b = gg & 1;
        if (!apf_wait(bb.k_full + b, (gg >> 1) & 1, 43u)) return false;
        if (gg >= 2 && !apf_wait(bb.o_full + b, ((gg - 2) >> 1) & 1, 44u)) return false;
        tc_fence_after();
        const uint32_t d = tm_s + 64u * static_cast<uint32_t>(b);
        const uint64_t dk = dk0 + static_cast<uint64_t>(b * (kPpTile >> 4));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_f16(d, dqh + 2 * kk, dk + 2 * kk, id_s, kk > 0 ? 1u : 0u);
          mma_f16(d, dql + 2 * kk, dk + 2 * kk, id_s, 1u);
        }
        mma_commit(bb.s_full + b);
        mma_commit(bb.k_free + b);
        return true;
      };
      int g = 0;
      bool ok = true;
      for (int k = 0; ok && item_of(k) < items; ++k) {
        const ApfItem w = apf_item(item_of(k), n_qt, H, Hkv, nseq, slot_base, L, layer);
        const int n_kt = tiles_of(w.qt);
        if (!(ok = apf_wait(bb.q_full, k & 1, 42u))) break;
        ok = issue_qk(g) && issue_qk(g + 1);
        for (int j = 0; j < n_kt && ok; ++j) {
          const int gg = g + j, b = gg & 1;
          if (!(ok = apf_wait(bb.p_full, gg & 1, 45u))) break;
          if (!(ok = apf_wait(bb.v_full + b, (gg >> 1) & 1, 38u))) break;
          if (gg >= 2 && !(ok = apf_wait(bb.o_free + b, ((gg - 2) >> 1) & 1, 46u))) break;
          tc_fence_after();
          const uint32_t sp = tm_s + 64u * static_cast<uint32_t>(b);
          const uint32_t d_o = tm_s + 128u + 64u * static_cast<uint32_t>(b);
          const uint64_t dv = dv0 + static_cast<uint64_t>(b * (kPpTile >> 4));
#pragma unroll
          for (int kk = 0; kk < kPpKeys / 16; ++kk) {
            // keys 16 kk .. + 15: P hi at columns 16 kk .. + 7, lo at 16 kk + 8 .. + 15
            const uint32_t a = sp + 16u * static_cast<uint32_t>(kk);
            mma_f16_ts(d_o, a, dv + kk * 128, id_o, kk > 0 ? 1u : 0u);
            mma_f16_ts(d_o, a + 8u, dv + kk * 128, id_o, 1u);
          }
          mma_commit(bb.o_full + b);
          mma_commit(bb.v_free + b);
          if (j + 2 < n_kt) ok = issue_qk(gg + 2);
        }
        g += n_kt;
      }
    }
  } else {
    // ---- softmax warps: thread = query row r of the stream's tile
    const int qq = warp & 3;
    const int r = qq * 32 + lane;
    const uint32_t lane_base = tm_s + (static_cast<uint32_t>(qq * 32) << 16);
    float o[64];
    // o += scale * (P_gg . V_gg), then O buffer gg % 2 may be overwritten
    auto fold = [&](int gg, float scale) -> bool {
      if (!apf_wait(bb.o_full + (gg & 1), (gg >> 1) & 1, 47u)) return false;
      tc_fence_after();
      const uint32_t ob = lane_base + 128u + 64u * static_cast<uint32_t>(gg & 1);
#pragma unroll
      for (int hh = 0; hh < 4; hh += 2) {
        int w0[16], w1[16];
        tmem_ld16_nw(ob + 16u * hh, w0);
        tmem_ld16_nw(ob + 16u * (hh + 1), w1);
        tmem_ld_wait16(w0);
        tmem_ld_wait16(w1);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[16 * hh + i] = fmaf(__int_as_float(w0[i]), scale, o[16 * hh + i]);
          o[16 * hh + 16 + i] = fmaf(__int_as_float(w1[i]), scale, o[16 * hh + 16 + i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bb.o_free + (gg & 1));
      return true;
    };
    int g = 0;
    bool ok = true;
    for (int k = 0; ok && item_of(k) < items; ++k) {
      const ApfItem w = apf_item(item_of(k), n_qt, H, Hkv, nseq, slot_base, L, layer);
      const int qt = w.qt, n_kt = tiles_of(qt);
      const int t = qt * kPpRows + r;
      // this item's query rows (every S MMA of the previous item has completed:
      // its last S was awaited below)
      const float xs = pp_prep_q_row(ss, qkv, ld, seq_len, w, r);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bb.q_full);
      const float sc2 = xs * __ldg(ks + w.sidx);
      float m2 = -INFINITY, l = 0.0f;  // running max (log2 units), running sum of p * 2^14
      float c_prev = 1.0f;             // correction of the previous tile (m_{j-2} -> m_{j-1})
#pragma unroll
      for (int i = 0; i < 64; ++i) o[i] = 0.0f;
      for (int j = 0; j < n_kt && ok; ++j) {
        const int gg = g + j, b = gg & 1;
        if (!(ok = apf_wait(bb.s_full + b, (gg >> 1) & 1, 48u))) break;
        tc_fence_after();
        const uint32_t sb = lane_base + 64u * static_cast<uint32_t>(b);
        const bool diag = j >= 2 * qt;       // key tiles that reach past row 128 qt
        const int lim = t - j * kPpKeys;      // keys k > lim of the tile are masked
        const float mraw = diag ? pp_row_max<true>(sb, lim) : pp_row_max<false>(sb, lim);
        const float m_new = fmaxf(m2, mraw * sc2);  // a fully masked tile keeps m2
        const float corr = ex2f(m2 - m_new);
        m2 = m_new;
        // o holds tiles <= j - 3 at max m_{j-1}; P_{j-2}.V_{j-2} is at m_{j-2}
        if (__any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll
          for (int i = 0; i < 64; ++i) o[i] *= corr;
        }
        if (j >= 2 && !(ok = fold(gg - 2, c_prev * corr))) break;
        c_prev = corr;
        const float off14 = 14.0f - m_new;
        const float psum = diag ? pp_exp_store<true>(sb, lim, sc2, off14) : pp_exp_store<false>(sb, lim, sc2, off14);
        l = fmaf(l, corr, psum);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bb.p_full);
      }
      if (!ok) break;
      // the last two tiles' P.V: P_{J-1}.V_{J-1} at m_{J-1} (scaled by the
      // last correction), P_J.V_J at the final maximum
      const int gJ = g + n_kt - 1;
      if (!(ok = fold(gJ - 1, c_prev))) break;
      if (!(ok = fold(gJ, 1.0f))) break;
      float local_max = 0.0f;
      if (t < seq_len) {
        const float inv = vs[w.sidx] / l;
        float4* orow = reinterpret_cast<float4*>(out + static_cast<size_t>(w.seq * seq_len + t) * Dq + w.head * 64);
#pragma unroll
        for (int d = 0; d < 64; d += 4) {
          const float4 y = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
          orow[d / 4] = y;
          local_max = fmaxf(local_max, fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w))));
        }
      }
      if (out_absmax) {
        local_max = warp_max(local_max);
        if (lane == 0) atomic_max_nonneg(out_absmax + w.seq, local_max);
      }
      g += n_kt;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_free(tmem, 512);
}

}  // namespace

cudaError_t launch_attn_prefill(const float* qkv, int ld, int rows, int seq_len, int H, int Hkv,
                                const int8_t* kc, const int8_t* vc, const float* ks,
                                const float* vs, int slot_base, int layer, int L, int P,
                                float* out, float* out_absmax, cudaStream_t s) {
  if (seq_len <= 0 || rows % seq_len || H % Hkv || (ld & 1)) return cudaErrorInvalidValue;
  const int nseq = rows / seq_len;
  if (use_apf_tc() && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    // (its float4 output stores need 16-byte aligned rows; Dq is a multiple of 64)
    // persistent: one CTA per SM walking the (query tile, head, sequence) items
    const int items = ((seq_len + kApfRows - 1) / kApfRows) * H * nseq;
    attn_prefill_tc_kernel<<<std::min(items, device_sm_count()), kApfThreads, kApfSmem, s>>>(
        qkv, ld, seq_len, nseq, H, Hkv, kc, vc, ks, vs, slot_base, layer, L, P, out, out_absmax);
    return cudaGetLastError();
  }
  dim3 grid((seq_len + kPfQTile - 1) / kPfQTile, H, nseq);
  attn_prefill_mma_kernel<<<grid, 128, 0, s>>>(qkv, ld, seq_len, H, Hkv, kc, vc, ks, vs, slot_base, layer,
                                               L, P, out, out_absmax);
  return cudaGetLastError();
}

cudaError_t launch_attn_prefill_kvh(const float* qkv, int ld, int rows, int seq_len, int H, int Hkv,
                                    const uint16_t* kh, const uint16_t* vh, const float* ks, const float* vs,
                                    int slot_base, int layer, int L, float* out, float* out_absmax, cudaStream_t s) {
  // (TL_DISABLE_TC_ATTN_PREFILL=1 selects the mma.sync kernel for every prefill)
  if (!use_apf_pp() || !use_apf_tc() || (reinterpret_cast<uintptr_t>(out) & 15u)) return cudaErrorNotSupported;
  // (the query rows are read as float4: 16-byte aligned rows)
  if (seq_len <= 0 || rows % seq_len || H % Hkv || (ld & 3) || (reinterpret_cast<uintptr_t>(qkv) & 15u) || !kh || !vh)
    return cudaErrorInvalidValue;
  const int nseq = rows / seq_len;
  CUtensorMap tk, tv;
  const long long krows = static_cast<long long>(nseq) * Hkv * seq_len;
  cudaError_t e = tc_encode_f16_rows64(&tk, kh, krows, kPpKeys);
  if (e != cudaSuccess) return e;
  if ((e = tc_encode_f16_rows64(&tv, vh, krows, kPpKeys)) != cudaSuccess) return e;
  const int items = ((seq_len + kPpRows - 1) / kPpRows) * H * nseq;
  const int grid = std::min(device_sm_count(), (items + 1) / 2);
  attn_prefill_pp_kernel<<<grid, kPpThreads, kPpSmem, s>>>(tk, tv, qkv, ld, seq_len, nseq, H, Hkv, ks, vs, slot_base,
                                                           layer, L, out, out_absmax);
  return cudaGetLastError();
}

// CTAs per (row, kv head): at most two resident CTAs per SM in one wave
// (no split once the (row, kv head) pairs alone fill the GPU), each split
// keeping at least two 32-position chunks of the longest context. The
// engine's partial buffer is sized for the largest count over 1..M rows
// (attn_part_floats).
int attn_splits(int M, int Hkv, int P) {
  const int pairs = std::max(1, M * Hkv);
  const int want = (2 * device_sm_count()) / pairs;
  const int cap = std::max(1, (P + 2 * kDecChunk - 1) / (2 * kDecChunk));
  return std::max(1, std::min(want, cap));
}

cudaError_t attn_prepare() {
  cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kDecSmem));
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kApfSmem));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(attn_prefill_pp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kPpSmem));
}

cudaError_t attn_read_error(unsigned int* code) {
  for (const void* sym : {static_cast<const void*>(&g_attn_error), static_cast<const void*>(&g_apf_error)}) {
    cudaError_t e = cudaMemcpyFromSymbol(code, sym, sizeof(unsigned int));
    if (e != cudaSuccess) return e;
    if (*code) {
      unsigned int zero = 0;
      return cudaMemcpyToSymbol(sym, &zero, sizeof(unsigned int));
    }
  }
  return cudaSuccess;
}

cudaError_t launch_attn_decode(const AttnDecodeArgs& a0, cudaStream_t s, bool pdl) {
  AttnDecodeArgs a = a0;
  const int G = a.H / a.Hkv;
  if (G < 1 || G > 8 || a.H % a.Hkv || !a.part || !a.counters) return cudaErrorInvalidValue;
  // (a larger split_rows never raises the count: part holds attn_part_floats(M, ...))
  a.splits = attn_splits(std::max(a.M, a.split_rows), a.Hkv, a.P);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.Hkv, a.M, a.splits);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = kDecSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel, a);
}

size_t attn_part_floats(int M, int Hkv, int P) {
  size_t most = 0;
  for (int m = 1; m <= M; ++m)
    most = std::max(most, static_cast<size_t>(m) * Hkv * attn_splits(m, Hkv, P) * kAttnPartStride);
  return most;
}

}  // namespace tl
