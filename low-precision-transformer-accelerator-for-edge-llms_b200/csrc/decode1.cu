// decode1.cu -- the whole single-sequence decode step in one persistent kernel.
//
// Batch-1 decode streams 1.04 GB of INT8 weights per token and does almost
// no arithmetic, so its time is set by how continuously HBM is kept busy.
// As separate kernels (5 per layer) every launch pays its own ramp, tail and
// dependency wait, which is several times the weight streaming of the
// smaller projections. Here one CTA per SM (cooperative launch, all CTAs
// resident) runs the entire step:
//
//  * Every weight matrix is split by output rows into one fixed slice per
//    CTA. Warp 12 (one lane) streams the CTA's slices -- layer by layer, in
//    the order they are consumed -- through a ring of shared-memory slots
//    with bulk async copies (cp.async.bulk, completion on a per-slot
//    mbarrier). Weights never depend on activations, so the stream runs
//    ahead across the phase barriers below; it only waits for free slots.
//  * Warps 0..11 take the ring's chunks round-robin and compute each row's
//    INT8 dot product with dp4a against the quantized activation held in
//    shared memory, followed by the same epilogues (and the same rounding)
//    as the multi-kernel GEMV path: dequantize, residual add, SiLU*up,
//    argmax key.
//  * Phases that need a whole activation row -- RMSNorm + quantize before
//    QKV and gate/up, quantize of the attention output and of SiLU*up --
//    are recomputed redundantly by every CTA from the row in L2 (8-22 KB),
//    which costs less than another barrier. Each CTA owns a fixed slice of
//    the residual stream x (the rows it produces in O and down), so only
//    five grid-wide barriers per layer remain: after QKV, after attention,
//    after O, after gate/up and after down.
//  * Attention of the one row: (kv head, 64-position chunk) work items
//    spread over CTAs, fp32 on CUDA cores, each writing its partial softmax
//    state; after the barrier every CTA merges the partials while it
//    quantizes the O projection's input. The new position's K/V are RoPE'd,
//    quantized with the frozen scales and appended in place.
//
// Data other CTAs wrote during this launch is read with ld.global.cg (L2),
// never through the non-coherent L1. Every wait (slot barriers, grid
// barriers) is bounded: on expiry an error word is set, later waits are
// skipped, and the host reports TL_ERR_TIMEOUT.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace tl {

__device__ unsigned int g_d1_error = 0;
// where the first expired wait happened: code, CTA, warp, ring chunk / barrier target
__device__ unsigned int g_d1_where[4] = {0, 0, 0, 0};

namespace {

constexpr int kD1Consumers = 12;                 // warps 0..11 compute, warp 12 streams
constexpr int kD1Threads = (kD1Consumers + 1) * 32;
constexpr int kD1ConsThreads = kD1Consumers * 32;
constexpr int kD1Slot = 8192;                    // bytes per ring slot
// Chunk i goes to warp i % kD1Consumers and slot i % kD1Slots. With the
// slot count a multiple of the warp count, the previous chunk of every slot
// belongs to the same warp, which has already waited for it: a waiter is
// never two phases ahead of a slot's barrier, where mbarrier parity waits
// would alias.
constexpr int kD1Slots = 2 * kD1Consumers;       // 192 KB ring, two slots per warp
static_assert(kD1Slots % kD1Consumers == 0, "slot reuse must stay within one warp");
constexpr int kD1AttnChunk = 32;                 // positions per attention work item (<= 32: one per lane)
// partial record per (kv head, query head, chunk): max, sum, 2 pad, 64 values
// (272 bytes: the values start 16-byte aligned for vector loads)
constexpr int kD1Rec = 68;
constexpr int kD1RecO = 4;
constexpr int kD1XOwn = 64;  // residual rows owned per CTA (D <= 64 * CTAs)
constexpr long long kD1Wait = 4000000000ll;      // ~2 s at 1.9 GHz
// a.sync layout: word 0 the grid-barrier counter; from kD1Tickets one
// attention ticket per (layer, kv head). All zero at launch.
constexpr int kD1Tickets = 256;

TL_DEV uint32_t d1_smem(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
TL_DEV bool d1_failed() { return *reinterpret_cast<volatile unsigned int*>(&g_d1_error) != 0u; }
TL_DEV void d1_fail(unsigned code, unsigned what = 0) {
  if (atomicCAS(&g_d1_error, 0u, code) == 0u) {
    g_d1_where[0] = code;
    g_d1_where[1] = blockIdx.x;
    g_d1_where[2] = threadIdx.x >> 5;
    g_d1_where[3] = what;
  }
}

// named barrier of the consumer warps (the streaming warp never joins)
TL_DEV void bar_cons() { asm volatile("bar.sync 1, %0;" ::"n"(kD1ConsThreads) : "memory"); }

TL_DEV void d1_mbar_init(uint64_t* b) { asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(d1_smem(b))); }
TL_DEV void d1_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(d1_smem(b)) : "memory");
}
TL_DEV void d1_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(d1_smem(b)), "r"(bytes) : "memory");
}
TL_DEV bool d1_wait(uint64_t* b, uint32_t parity, unsigned code, unsigned what = 0) {
  if (d1_failed()) return false;
  const uint32_t a = d1_smem(b);
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kD1Wait) {
      d1_fail(code, what);
      return false;
    }
  }
}
TL_DEV void d1_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(d1_smem(dst)), "l"(src), "r"(bytes), "r"(d1_smem(bar))
               : "memory");
}
TL_DEV unsigned int ld_relaxed_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
TL_DEV unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the consumer warps of every CTA: a monotonic arrival
// counter (zeroed before the launch). Each CTA adds its arrival with a
// fire-and-forget release reduction, then polls the counter with relaxed
// loads until it reaches (barriers so far) x (CTAs), and issues one acquire
// fence. Release is cumulative over the writes the CTA's threads ordered
// before it with the CTA barrier; the fence orders the other CTAs' writes
// before every read after the closing CTA barrier. (Measured on B200 with
// 148 CTAs: ~1.25 us per barrier, below an arrival counter plus a published
// generation word, a hierarchical counter tree, or polled per-CTA flags.)
TL_DEV void d1_grid_sync(unsigned int* counter, unsigned int& gen) {
  bar_cons();
  const unsigned int next = gen + 1;
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
    if (!d1_failed()) {
      const unsigned int target = next * gridDim.x;
      const long long t0 = clock64();
      while (ld_relaxed_u32(counter) < target) {
        if (clock64() - t0 > kD1Wait) {
          d1_fail(5u, gen);
          break;
        }
      }
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
    }
  }
  gen = next;
  bar_cons();
}

// The same barrier in two halves, so that loads that do not depend on the
// other CTAs' writes can be in flight while it completes.
TL_DEV void d1_grid_arrive(unsigned int* counter) {
  bar_cons();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
}
TL_DEV void d1_grid_wait(unsigned int* counter, unsigned int& gen) {
  const unsigned int next = gen + 1;
  if (threadIdx.x == 0 && !d1_failed()) {
    const unsigned int target = next * gridDim.x;
    const long long t0 = clock64();
    while (ld_relaxed_u32(counter) < target) {
      if (clock64() - t0 > kD1Wait) {
        d1_fail(5u, gen);
        break;
      }
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  gen = next;
  bar_cons();
}

TL_DEV float silu_mul_d1(float g, float u) {
  const float c = fminf(fmaxf(g, -60.0f), 60.0f);
  const float den = __fadd_rn(1.0f, expf(-c));
  return __fmul_rn(__fdiv_rn(g, den), u);
}


// ---------------------------------------------------------------- consumers
// The consumer warps' view of shared memory.
struct D1Smem {
  unsigned char* ring;
  float* xf;         // [max(D, F, Dq)] row being normalized / quantized; attention scratch
  int8_t* xq;        // [max(D, F, Dq)] quantized activation
  float* red;        // [64] reduction scratch
  float* rs;         // RMSNorm tree scratch (n_leaves * 9 + 32)
  double* sx;        // [1] activation scale of xq
  unsigned long long* key;  // [1] LM-head argmax of this CTA
  int* flag;         // [1]
  float* x_own;      // [kD1XOwn] this CTA's slice of the residual stream
  uint64_t* full;    // [kD1Slots]
  uint64_t* empty;   // [kD1Slots]
};

// Sum of squares in NumPy's pairwise order over the consumer warps (the
// tree of block_sumsq_numpy: leaves of L elements with 8 interleaved
// accumulators each, folded, then combined level by level).
TL_DEV float cons_sumsq(const float* v, NormPlan plan, float* part, float* leaf) {
  const int tid = threadIdx.x;
  const int L = plan.leaf_len, nl = plan.n_leaves;
  for (int idx = tid; idx < nl * 8; idx += kD1ConsThreads) {
    const int l = idx >> 3, j = idx & 7;
    const float* x = v + l * L;
    float r = __fmul_rn(x[j], x[j]);
    for (int i = 8 + j; i < L; i += 8) r = __fadd_rn(r, __fmul_rn(x[i], x[i]));
    part[idx] = r;
  }
  bar_cons();
  if (nl <= 32) {
    // one warp: lane l folds leaf l, then the leaves combine pairwise by XOR
    // shuffles (adjacent blocks of 1, 2, 4, ... leaves: the same additions)
    if (tid < 32) {
      float t = 0.0f;
      if (tid < nl) {
        const float* q = part + tid * 8;
        t = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3])),
                      __fadd_rn(__fadd_rn(q[4], q[5]), __fadd_rn(q[6], q[7])));
      }
      for (int st = 1; st < nl; st *= 2) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, st));
      if (tid == 0) leaf[0] = t;
    }
    bar_cons();
    return leaf[0];
  }
  for (int l = tid; l < nl; l += kD1ConsThreads) {
    const float* q = part + l * 8;
    leaf[l] = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3])),
                        __fadd_rn(__fadd_rn(q[4], q[5]), __fadd_rn(q[6], q[7])));
  }
  bar_cons();
  for (int st = 1; st < nl; st *= 2) {
    for (int l = tid * 2 * st; l < nl; l += kD1ConsThreads * 2 * st) leaf[l] = __fadd_rn(leaf[l], leaf[l + st]);
    bar_cons();
  }
  return leaf[0];
}


// xf[0..K) <- src (written by other CTAs: L2 reads), optionally RMSNorm'd
// with gamma; then xq <- quantize_int8 of it and sm.sx <- its scale.
constexpr int kD1RowVec = 4;  // float4 per consumer thread: rows of up to 4 * 4 * 384 = 6144

// named barrier of consumer warps 0..3 (the RMSNorm fast path)
TL_DEV void bar_norm4() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

// RMSNorm + INT8 quantization of a 2048-wide row (NumPy tree: 16 leaves of
// 128) by consumer warps 0..3 alone: thread t owns accumulator t & 7 of leaf
// t >> 3 and its 16 elements x[128 (t >> 3) + (t & 7) + 8 k] in registers;
// the leaf folds ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) by XOR shuffles 1, 2,
// 4, leaves pair up by shuffles 8 and 16, the four warp sums combine as
// (w0+w1)+(w2+w3) -- block_sumsq_numpy's additions. Then normalize, max,
// quantize into xq; the other warps only meet the closing barrier.
TL_DEV void cons_norm_quant_d2048(const D1Smem& sm, const float* src, const float* gamma, float eps) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (warp < 4) {
    const int base = (tid >> 3) * 128 + (tid & 7);
    float v[16], gm[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      v[k] = __ldcg(src + base + 8 * k);
      gm[k] = __ldg(gamma + base + 8 * k);
    }
    float acc = __fmul_rn(v[0], v[0]);
#pragma unroll
    for (int k = 1; k < 16; ++k) acc = __fadd_rn(acc, __fmul_rn(v[k], v[k]));
#pragma unroll
    for (int st = 1; st < 32; st *= 2) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, st));
    if (lane == 0) sm.red[32 + warp] = acc;
    bar_norm4();
    const float tot = __fadd_rn(__fadd_rn(sm.red[32], sm.red[33]), __fadd_rn(sm.red[34], sm.red[35]));
    const float mean = __fdiv_rn(tot, 2048.0f);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      v[k] = __fmul_rn(__fmul_rn(v[k], inv), gm[k]);
      m = fmaxf(m, fabsf(v[k]));
    }
    m = warp_max(m);
    if (lane == 0) sm.red[36 + warp] = m;
    bar_norm4();
    m = fmaxf(fmaxf(sm.red[36], sm.red[37]), fmaxf(sm.red[38], sm.red[39]));
    const double s64 = quant_scale64(m);
    const float sf = static_cast<float>(s64);
#pragma unroll
    for (int k = 0; k < 16; ++k) sm.xq[base + 8 * k] = static_cast<int8_t>(quantize_one(v[k], sf));
    if (tid == 0) *sm.sx = s64;
  }
  bar_cons();
}
TL_DEV void cons_quant_regs(const D1Smem& sm, float4* v, int K);

// xf[0..K) <- src (written by other CTAs: L2 reads), optionally RMSNorm'd
// with gamma; then xq <- quantize_int8 of it and sm.sx <- its scale. Every
// thread issues all its loads (row and gain) before using any; the row stays
// in registers, xf only feeds the ordered sum of squares.
TL_DEV void cons_load_quant(const D1Smem& sm, const float* src, int K, const float* gamma, float eps,
                            NormPlan plan) {
  const int tid = threadIdx.x;
  const int n4 = K >> 2;
  float4 v[kD1RowVec], gm[kD1RowVec];
#pragma unroll
  for (int u = 0; u < kD1RowVec; ++u) {
    const int q = tid + u * kD1ConsThreads;
    v[u] = q < n4 ? __ldcg(reinterpret_cast<const float4*>(src) + q) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    gm[u] = (gamma && q < n4) ? __ldg(reinterpret_cast<const float4*>(gamma) + q) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  if (gamma) {
#pragma unroll
    for (int u = 0; u < kD1RowVec; ++u) {
      const int q = tid + u * kD1ConsThreads;
      if (q < n4) reinterpret_cast<float4*>(sm.xf)[q] = v[u];
    }
    bar_cons();
    const float tot = cons_sumsq(sm.xf, plan, sm.rs, sm.rs + plan.n_leaves * 8);
    const float mean = __fdiv_rn(tot, static_cast<float>(K));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
    for (int u = 0; u < kD1RowVec; ++u) {
      v[u].x = __fmul_rn(__fmul_rn(v[u].x, inv), gm[u].x);
      v[u].y = __fmul_rn(__fmul_rn(v[u].y, inv), gm[u].y);
      v[u].z = __fmul_rn(__fmul_rn(v[u].z, inv), gm[u].z);
      v[u].w = __fmul_rn(__fmul_rn(v[u].w, inv), gm[u].w);
    }
  }
  cons_quant_regs(sm, v, K);
}

// max |v| over the row held in the consumer threads' registers, then
// xq <- quantize_int8 and sm.sx <- its float64 scale.
TL_DEV void cons_quant_regs(const D1Smem& sm, float4* v, int K) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n4 = K >> 2;
  float m = 0.0f;
#pragma unroll
  for (int u = 0; u < kD1RowVec; ++u)
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
  m = warp_max(m);
  if (lane == 0) sm.red[warp] = m;
  bar_cons();
  float amax = 0.0f;
  for (int w = 0; w < kD1Consumers; ++w) amax = fmaxf(amax, sm.red[w]);
  const double s64 = quant_scale64(amax);
  const float sf = static_cast<float>(s64);
#pragma unroll
  for (int u = 0; u < kD1RowVec; ++u) {
    const int q = tid + u * kD1ConsThreads;
    if (q < n4)
      reinterpret_cast<uint32_t*>(sm.xq)[q] = (static_cast<uint32_t>(quantize_one(v[u].x, sf)) & 0xffu) |
                                              ((static_cast<uint32_t>(quantize_one(v[u].y, sf)) & 0xffu) << 8) |
                                              ((static_cast<uint32_t>(quantize_one(v[u].z, sf)) & 0xffu) << 16) |
                                              ((static_cast<uint32_t>(quantize_one(v[u].w, sf)) & 0xffu) << 24);
  }
  if (tid == 0) *sm.sx = s64;
  bar_cons();
}

// Dot product of one weight row (K bytes in shared memory) with xq, by the
// whole warp; returned in every lane.
TL_DEV int warp_dot(const int8_t* w, const int8_t* xq, int K) {
  const int lane = threadIdx.x & 31;
  const int4* wr = reinterpret_cast<const int4*>(w);
  const int4* xr = reinterpret_cast<const int4*>(xq);
  int acc = 0;
  const int n16 = K >> 4;
#pragma unroll 4
  for (int q = lane; q < n16; q += 32) {
    const int4 a = wr[q], b = xr[q];
    acc = dp4a(a.x, b.x, acc);
    acc = dp4a(a.y, b.y, acc);
    acc = dp4a(a.z, b.z, acc);
    acc = dp4a(a.w, b.w, acc);
  }
  return warp_sum_i(acc);
}

enum D1Mat : int { D1_QKV = 0, D1_O = 1, D1_GU = 2, D1_DOWN = 3, D1_LM = 4 };

// rows per ring chunk for K-byte rows (gate/up chunks hold whole row pairs)
TL_DEV int d1_rows_per_chunk(int K, bool pairs) {
  int r = kD1Slot / K;
  if (r > 32) r = 32;  // one row scale per lane
  if (pairs) r &= ~1;
  return r < 1 ? 1 : r;
}

// This CTA's slice [r0, r1) of an N-row matrix (gate/up: row pairs).
TL_DEV void d1_slice(int N, bool pairs, int& r0, int& r1) {
  const int units = pairs ? N / 2 : N;
  const long long b = blockIdx.x, g = gridDim.x;
  int u0 = static_cast<int>(b * units / g), u1 = static_cast<int>((b + 1) * units / g);
  r0 = pairs ? 2 * u0 : u0;
  r1 = pairs ? 2 * u1 : u1;
}

}  // namespace


namespace {

// Rows [r, r + nr) of matrix `mat` sit in the ring slot; warp computes them.
// Rows [r, r + nr) of matrix `mat` sit in the ring slot; the warp computes
// them. `wsc` (lane i) is the weight scale of row r + i, loaded before the
// chunk was awaited. x rows live in this CTA's shared copy (x_own, index
// n - x0) and are written through to global memory for the other CTAs.
TL_DEV void d1_rows(const D1Args& a, int mat, const int8_t* w, int r, int nr, double wsc, int x0,
                    const D1Smem& sm) {
  const int lane = threadIdx.x & 31;
  const double sx = *sm.sx;
  if (mat == D1_GU) {
    for (int i = 0; i < nr; i += 2) {
      const int accg = warp_dot(w + static_cast<size_t>(i) * a.D, sm.xq, a.D);
      const int accu = warp_dot(w + static_cast<size_t>(i + 1) * a.D, sm.xq, a.D);
      const double sg = __shfl_sync(0xffffffffu, wsc, i), su = __shfl_sync(0xffffffffu, wsc, i + 1);
      if (lane == 0) {
        const int n = r + i;
        a.hid[n >> 1] = silu_mul_d1(dequant(accg, sx, sg), dequant(accu, sx, su));
      }
    }
    return;
  }
  const int K = mat == D1_O ? a.Dq : (mat == D1_DOWN ? a.F : a.D);
  unsigned long long best = 0ull;
  for (int i = 0; i < nr; ++i) {
    const int acc = warp_dot(w + static_cast<size_t>(i) * K, sm.xq, K);
    const double sw = __shfl_sync(0xffffffffu, wsc, i);
    if (lane == 0) {
      const int n = r + i;
      const float y = dequant(acc, sx, sw);
      if (mat == D1_QKV) {
        a.qkv[n] = y;
      } else if (mat == D1_O || mat == D1_DOWN) {
        const float v = __fadd_rn(sm.x_own[n - x0], y);
        sm.x_own[n - x0] = v;
        a.x[n] = v;
      } else {
        const unsigned long long k = argmax_key(y, n);
        best = k > best ? k : best;
      }
    }
  }
  if (mat == D1_LM && lane == 0 && best) atomicMax(sm.key, best);
}

// Attention of the single row for work item (kv head h, chunk c): the partial
// softmax state (max, sum, unnormalized P.V over the chunk's positions) of
// the kv head's query heads, written to a.part. Every load of the item is
// issued up front: warps take the rotated queries and the cached K/V rows
// while the last consumer warp RoPEs, quantizes and appends the new
// position's K/V (written to the cache for running rows).
// This thread's 16-byte piece of the item's cached K and V rows (row
// tid / 4, piece tid % 4; positions other than the new one), loaded from HBM.
struct D1KvPiece {
  int4 k, v;
};
TL_DEV float4 d1_merge_qd(const D1Args& a, int layer, int qd, int nch);
TL_DEV D1KvPiece d1_load_kv_piece(const D1Args& a, int layer, int h, int c) {
  D1KvPiece r{make_int4(0, 0, 0, 0), make_int4(0, 0, 0, 0)};
  const int tid = threadIdx.x;
  if (tid >= kD1AttnChunk * 4) return r;
  const int p = a.pos[0];
  const int t0 = c * kD1AttnChunk;
  const int n = min(kD1AttnChunk, p + 1 - t0);
  const int row = tid >> 2, cc = tid & 3;
  if (row < n && t0 + row != p) {
    const size_t sidx = (static_cast<size_t>(a.slot[0]) * a.L + layer) * a.Hkv + h;
    const size_t off = (sidx * a.P + t0 + row) * 64;
    r.k = __ldcg(reinterpret_cast<const int4*>(a.kc + off) + cc);
    r.v = __ldcg(reinterpret_cast<const int4*>(a.vc + off) + cc);
  }
  return r;
}

TL_DEV void d1_attention_item(const D1Args& a, int layer, int h, int c, int nch, const D1Smem& sm,
                              const D1KvPiece& pre) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.H / a.Hkv;
  const int p = a.pos[0];
  const int T = p + 1;
  const int t0 = c * kD1AttnChunk;
  const int n = min(kD1AttnChunk, T - t0);
  const int slot = a.slot[0];
  const size_t sidx = (static_cast<size_t>(slot) * a.L + layer) * a.Hkv + h;
  const float sK = a.ks[sidx], sV = a.vs[sidx];
  int8_t* kbase = a.kc + sidx * static_cast<size_t>(a.P) * 64;
  int8_t* vbase = a.vc + sidx * static_cast<size_t>(a.P) * 64;
  const float* cs = a.cos + static_cast<size_t>(p) * 64;
  const float* sn = a.sin + static_cast<size_t>(p) * 64;
  // scratch in xf: q [8][64], scores [8][64], K [64][64] bytes, V [64][64] bytes
  float* q = sm.xf;
  float* sc = q + 8 * 64;
  int8_t* kb = reinterpret_cast<int8_t*>(sc + 8 * 64);
  int8_t* vb = kb + kD1AttnChunk * 64;
  if (tid < G * 32) {
    const int g = tid >> 5, d = tid & 31;
    const float* qr = a.qkv + (h * G + g) * 64;
    const float q0 = __ldcg(qr + d), q1 = __ldcg(qr + d + 32);
    const float c0 = __ldg(cs + d), c1 = __ldg(cs + d + 32), s0 = __ldg(sn + d), s1 = __ldg(sn + d + 32);
    q[g * 64 + d] = __fadd_rn(__fmul_rn(q0, c0), __fmul_rn(-q1, s0));
    q[g * 64 + d + 32] = __fadd_rn(__fmul_rn(q1, c1), __fmul_rn(q0, s1));
  }
  if (tid < kD1AttnChunk * 4) {
    const int r = tid >> 2, cc = tid & 3;
    if (t0 + r != p) {  // the new row is written by the append warp below
      reinterpret_cast<int4*>(kb + r * 64)[cc] = pre.k;
      reinterpret_cast<int4*>(vb + r * 64)[cc] = pre.v;
    }
  }
  if (warp == kD1Consumers - 1 && p >= t0 && p < t0 + n) {
    const bool act = a.active ? (a.active[0] != 0) : true;
    const float* kr = a.qkv + a.Dq + h * 64;
    const float* vr = a.qkv + a.Dq + a.Hkv * 64 + h * 64;
    const float k0 = __ldcg(kr + lane), k1 = __ldcg(kr + lane + 32);
    const float v0 = __ldcg(vr + lane), v1 = __ldcg(vr + lane + 32);
    const float c0 = __ldg(cs + lane), c1 = __ldg(cs + lane + 32), s0 = __ldg(sn + lane), s1 = __ldg(sn + lane + 32);
    const float r0 = __fadd_rn(__fmul_rn(k0, c0), __fmul_rn(-k1, s0));
    const float r1 = __fadd_rn(__fmul_rn(k1, c1), __fmul_rn(k0, s1));
    const int8_t qk0 = static_cast<int8_t>(quantize_one(r0, sK)), qk1 = static_cast<int8_t>(quantize_one(r1, sK));
    const int8_t qv0 = static_cast<int8_t>(quantize_one(v0, sV)), qv1 = static_cast<int8_t>(quantize_one(v1, sV));
    const int rl = p - t0;
    kb[rl * 64 + lane] = qk0;
    kb[rl * 64 + lane + 32] = qk1;
    vb[rl * 64 + lane] = qv0;
    vb[rl * 64 + lane + 32] = qv1;
    if (act) {
      kbase[static_cast<size_t>(p) * 64 + lane] = qk0;
      kbase[static_cast<size_t>(p) * 64 + lane + 32] = qk1;
      vbase[static_cast<size_t>(p) * 64 + lane] = qv0;
      vbase[static_cast<size_t>(p) * 64 + lane + 32] = qv1;
    }
  }
  bar_cons();
  // scores (fp32): s[g][t] = (q_g . k_t) * sK / 8
  const float ss = sK * 0.125f;
  for (int i = tid; i < G * kD1AttnChunk; i += kD1ConsThreads) {
    const int g = i / kD1AttnChunk, t = i % kD1AttnChunk;
    float s = -INFINITY;
    if (t < n) {
      const float* qg = q + g * 64;
      const int8_t* kt = kb + t * 64;
      float acc = 0.0f;
#pragma unroll 16
      for (int d = 0; d < 64; ++d) acc = fmaf(qg[d], static_cast<float>(kt[d]), acc);
      s = acc * ss;
    }
    sc[g * 64 + t] = s;
  }
  bar_cons();
  // per head: max and exp, one warp per head
  float* pm = sm.red;  // [8] max, [8..16) sum
  if (warp < G) {
    const int g = warp;
    const float s0 = lane < kD1AttnChunk ? sc[g * 64 + lane] : -INFINITY;
    const float m = warp_max(s0);
    const float e0 = expf(s0 - m);
    if (lane < kD1AttnChunk) sc[g * 64 + lane] = e0;
    const float l = warp_sum(e0);
    if (lane == 0) {
      pm[g] = m;
      pm[8 + g] = l;
    }
  }
  bar_cons();
  // o[g][d] = sum_t e[g][t] * v[t][d] (V as its int8 value; sV applied at the merge)
  const int maxch = (a.P + kD1AttnChunk - 1) / kD1AttnChunk;
  for (int i = tid; i < G * 64; i += kD1ConsThreads) {
    const int g = i >> 6, d = i & 63;
    float acc = 0.0f;
    for (int t = 0; t < n; ++t) acc = fmaf(sc[g * 64 + t], static_cast<float>(vb[t * 64 + d]), acc);
    float* pr = a.part + ((static_cast<size_t>(h) * 8 + g) * maxch + c) * kD1Rec;
    pr[kD1RecO + d] = acc;
    if (d == 0) {
      pr[0] = pm[g];
      pr[1] = pm[8 + g];
    }
  }
  bar_cons();  // the scratch in xf is reused by the next item
  // The item that finishes kv head h last merges the head's chunks into
  // a.att once (instead of every CTA merging every head after the barrier).
  // Ticket: the CTA barrier orders this CTA's partial stores before thread
  // 0's fence and atomic; the winner fences again before reading the others'.
  if (tid == 0) {
    __threadfence();
    const unsigned int t = atomicAdd(a.sync + kD1Tickets + layer * a.Hkv + h, 1u);
    *sm.flag = t == static_cast<unsigned int>(nch - 1);
    if (*sm.flag) __threadfence();
  }
  bar_cons();
  if (*sm.flag) {
    const int qd0 = h * G * 16;  // 16 four-dim groups per query head
    for (int i = tid; i < G * 16; i += kD1ConsThreads)
      reinterpret_cast<float4*>(a.att)[qd0 + i] = d1_merge_qd(a, layer, qd0 + i, nch);
  }
  bar_cons();  // sm.flag is reused by the next item
}

// Attention output dims 4 qd .. 4 qd + 3 merged from the chunk partials of
// their query head: the chunks' (max, sum, P.V) are combined in chunk order,
// eight chunks per load round, as att = (sum_c o_c e_c) / (sum_c l_c e_c) *
// sV with e_c = exp(m_c - running max). Partials written by other CTAs are
// read from L2.
TL_DEV float4 d1_merge_qd(const D1Args& a, int layer, int qd, int nch) {
  const int G = a.H / a.Hkv;
  const int maxch = (a.P + kD1AttnChunk - 1) / kD1AttnChunk;
  const int gq = (qd * 4) >> 6, d = (qd * 4) & 63;
  const int h = gq / G, g = gq % G;
  const float* rec = a.part + (static_cast<size_t>(h) * 8 + g) * maxch * kD1Rec;
  float M = -INFINITY, L = 0.0f;
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int c0 = 0; c0 < nch; c0 += 8) {
    float mv[8], lv[8];
    float4 ov[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float* r = rec + static_cast<size_t>(c0 + j) * kD1Rec;
      const bool ok = c0 + j < nch;
      mv[j] = ok ? __ldcg(r) : -INFINITY;
      lv[j] = ok ? __ldcg(r + 1) : 0.0f;
      ov[j] = ok ? __ldcg(reinterpret_cast<const float4*>(r + kD1RecO + d)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float bm = M;
#pragma unroll
    for (int j = 0; j < 8; ++j) bm = fmaxf(bm, mv[j]);
    const float keep = expf(M - bm);  // 0 on the first batch (M = -inf)
    L *= keep;
    o.x *= keep;
    o.y *= keep;
    o.z *= keep;
    o.w *= keep;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (c0 + j >= nch) continue;
      const float f = expf(mv[j] - bm);
      L += lv[j] * f;
      o.x += ov[j].x * f;
      o.y += ov[j].y * f;
      o.z += ov[j].z * f;
      o.w += ov[j].w * f;
    }
    M = bm;
  }
  const float sV = a.vs[(static_cast<size_t>(a.slot[0]) * a.L + layer) * a.Hkv + h];
  return make_float4(o.x / L * sV, o.y / L * sV, o.z / L * sV, o.w / L * sV);
}

__global__ void __launch_bounds__(kD1Threads, 1) decode1_kernel(D1Args a) {
  extern __shared__ __align__(128) unsigned char d1_raw[];
  const int K_max = max(max(a.D, a.F), a.Dq);
  D1Smem sm;
  sm.ring = d1_raw;
  sm.full = reinterpret_cast<uint64_t*>(d1_raw + kD1Slots * kD1Slot);
  sm.empty = sm.full + kD1Slots;
  sm.sx = reinterpret_cast<double*>(sm.empty + kD1Slots);
  sm.key = reinterpret_cast<unsigned long long*>(sm.sx + 1);
  sm.flag = reinterpret_cast<int*>(sm.key + 1);
  sm.red = reinterpret_cast<float*>(sm.flag + 4);
  sm.rs = sm.red + 64;
  sm.xf = sm.rs + (a.plan.n_leaves * 9 + 32 + 3) / 4 * 4;
  sm.xq = reinterpret_cast<int8_t*>(sm.xf + max(K_max, 2 * 8 * 64 + 2 * kD1AttnChunk * 16));
  sm.x_own = reinterpret_cast<float*>(sm.xq + K_max);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kD1Slots; ++s) {
      d1_mbar_init(sm.full + s);
      d1_mbar_init(sm.empty + s);
    }
    *sm.key = 0ull;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // ------------------------------------------------------ weight streamer
  if (warp == kD1Consumers) {
    if (lane != 0) return;
    uint32_t i = 0;
    auto stream_matrix = [&](const int8_t* w, int N, int K, bool pairs) {
      int r0, r1;
      d1_slice(N, pairs, r0, r1);
      const int rpc = d1_rows_per_chunk(K, pairs);
      for (int r = r0; r < r1; r += rpc, ++i) {
        const int nr = min(rpc, r1 - r);
        const int s = static_cast<int>(i % kD1Slots);
        if (i >= kD1Slots && !d1_wait(sm.empty + s, ((i / kD1Slots) - 1) & 1, 6u, i)) return false;
        if (d1_failed()) return false;
        const uint32_t bytes = static_cast<uint32_t>(nr) * static_cast<uint32_t>(K);
        d1_expect_tx(sm.full + s, bytes);
        d1_bulk(sm.ring + s * kD1Slot, w + static_cast<size_t>(r) * K, bytes, sm.full + s);
      }
      return true;
    };
    bool ok = true;
    for (int l = 0; l < a.L && ok; ++l) {
      const D1Layer& ly = a.layers[l];
      ok = stream_matrix(ly.wqkv, a.Nqkv, a.D, false) && stream_matrix(ly.wo, a.D, a.Dq, false) &&
           stream_matrix(ly.wgu, 2 * a.F, a.D, true) && stream_matrix(ly.wd, a.D, a.F, false);
    }
    if (ok) stream_matrix(a.wlm, a.V, a.D, false);
    // copies still in flight must land before the CTA can exit
    const uint32_t issued = i;
    for (uint32_t j = issued > kD1Slots ? issued - kD1Slots : 0; j < issued; ++j)
      (void)d1_wait(sm.full + j % kD1Slots, (j / kD1Slots) & 1, 7u, j);
    return;
  }

  // ------------------------------------------------------ consumer warps
  uint32_t i = 0;        // ring chunk counter (same sequence as the streamer)
  unsigned int target = 0;  // grid barrier generation
  int x0, x1;  // residual rows owned by this CTA (its rows of O and down)
  d1_slice(a.D, false, x0, x1);
  auto consume_matrix = [&](const double* scales, int mat, int N, int K, bool pairs) {
    int r0, r1;
    d1_slice(N, pairs, r0, r1);
    const int rpc = d1_rows_per_chunk(K, pairs);
    for (int r = r0; r < r1; r += rpc, ++i) {
      if (static_cast<int>(i % kD1Consumers) != warp) continue;
      const int nr = min(rpc, r1 - r);
      const int s = static_cast<int>(i % kD1Slots);
      const double wsc = lane < nr ? __ldg(scales + r + lane) : 0.0;  // overlaps the slot wait
      if (d1_wait(sm.full + s, (i / kD1Slots) & 1, 8u, i))
        d1_rows(a, mat, reinterpret_cast<const int8_t*>(sm.ring + s * kD1Slot), r, nr, wsc, x0, sm);
      __syncwarp();
      if (lane == 0) d1_arrive(sm.empty + s);
    }
  };

  // embedding row into this CTA's slice of the residual stream
  {
    int id = a.token[0];
    id = id < 0 ? 0 : (id >= a.V ? a.V - 1 : id);
    for (int n = x0 + tid; n < x1; n += kD1ConsThreads) {
      const float v = a.embed[static_cast<size_t>(id) * a.D + n];
      sm.x_own[n - x0] = v;
      a.x[n] = v;
    }
  }
  d1_grid_sync(a.sync, target);

  const bool fast_norm = a.D == 2048 && a.plan.n_leaves == 16 && a.plan.leaf_len == 128;
  const int T = a.pos[0] + 1;
  const int nch = (T + kD1AttnChunk - 1) / kD1AttnChunk;
  const int items = a.Hkv * nch;
  for (int l = 0; l < a.L; ++l) {
    const D1Layer& ly = a.layers[l];
    if (fast_norm) cons_norm_quant_d2048(sm, a.x, ly.g1, a.eps);
    else cons_load_quant(sm, a.x, a.D, ly.g1, a.eps, a.plan);
    consume_matrix(ly.sqkv, D1_QKV, a.Nqkv, a.D, false);
    d1_grid_arrive(a.sync);
    // the cached K/V rows of this CTA's first item stream in during the barrier
    D1KvPiece pre{make_int4(0, 0, 0, 0), make_int4(0, 0, 0, 0)};
    if (static_cast<int>(blockIdx.x) < items) pre = d1_load_kv_piece(a, l, blockIdx.x / nch, blockIdx.x % nch);
    d1_grid_wait(a.sync, target);
    for (int w = blockIdx.x; w < items; w += gridDim.x) {
      if (w != static_cast<int>(blockIdx.x)) pre = d1_load_kv_piece(a, l, w / nch, w % nch);
      d1_attention_item(a, l, w / nch, w % nch, nch, sm, pre);
    }
    d1_grid_sync(a.sync, target);
    cons_load_quant(sm, a.att, a.Dq, nullptr, a.eps, a.plan);  // merged by the heads' last items
    consume_matrix(ly.so, D1_O, a.D, a.Dq, false);
    d1_grid_sync(a.sync, target);
    if (fast_norm) cons_norm_quant_d2048(sm, a.x, ly.g2, a.eps);
    else cons_load_quant(sm, a.x, a.D, ly.g2, a.eps, a.plan);
    consume_matrix(ly.sgu, D1_GU, 2 * a.F, a.D, true);
    d1_grid_sync(a.sync, target);
    cons_load_quant(sm, a.hid, a.F, nullptr, a.eps, a.plan);
    consume_matrix(ly.sd, D1_DOWN, a.D, a.F, false);
    d1_grid_sync(a.sync, target);
  }
  if (fast_norm) cons_norm_quant_d2048(sm, a.x, a.gfinal, a.eps);
  else cons_load_quant(sm, a.x, a.D, a.gfinal, a.eps, a.plan);
  consume_matrix(a.slm, D1_LM, a.V, a.D, false);
  bar_cons();
  if (tid == 0 && *sm.key) atomicMax(a.am_key, *sm.key);
}

}  // namespace

unsigned int g_d1_last_what = 0;

size_t decode1_smem(int D, int F, int Dq) {
  NormPlan plan;
  if (!norm_plan(D, &plan)) return 0;
  const int K_max = std::max(std::max(D, F), Dq);
  const size_t rs = (plan.n_leaves * 9 + 32 + 3) / 4 * 4;
  const size_t xf = std::max(K_max, 2 * 8 * 64 + 2 * kD1AttnChunk * 16);
  return static_cast<size_t>(kD1Slots) * kD1Slot + 2 * kD1Slots * 8 + 8 + 8 + 16 + 64 * 4 + rs * 4 + xf * 4 +
         static_cast<size_t>(K_max) + kD1XOwn * 4 + 64;
}

bool decode1_supported(int D, int F, int Dq, int H, int Hkv, int P) {
  (void)P;
  const int row_max = kD1RowVec * 4 * kD1ConsThreads;  // row phases hold the row in registers
  const int K_max = std::max(std::max(D, F), Dq);
  return device_sm_count() <= 256 && K_max <= kD1Slot && K_max <= row_max && H / Hkv <= 8 && D % 16 == 0 &&
         F % 16 == 0 && (D + device_sm_count() - 1) / device_sm_count() <= kD1XOwn && Dq % 16 == 0 &&
         decode1_smem(D, F, Dq) <= 227 * 1024;
}

size_t decode1_sync_words(int L, int Hkv) { return static_cast<size_t>(kD1Tickets) + static_cast<size_t>(L) * Hkv; }

size_t decode1_part_floats(int Hkv, int P) {
  return static_cast<size_t>(Hkv) * 8 * ((P + kD1AttnChunk - 1) / kD1AttnChunk) * kD1Rec;
}

cudaError_t decode1_prepare(int D, int F, int Dq) {
  return cudaFuncSetAttribute(decode1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(decode1_smem(D, F, Dq)));
}

cudaError_t launch_decode1(const D1Args& a, int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kD1Threads);
  cfg.dynamicSmemBytes = decode1_smem(a.D, a.F, a.Dq);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode1_kernel, a);
}

cudaError_t decode1_read_error(unsigned int* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_d1_error, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  if (*code) {
    unsigned int where[4];
    e = cudaMemcpyFromSymbol(where, g_d1_where, sizeof(where));
    if (e != cudaSuccess) return e;
    // code: 5 grid barrier, 6 slot free (streamer), 7 last copies, 8 slot full (consumer)
    *code = 1000000u * where[0] + 1000u * (where[1] % 1000u) + (where[2] % 1000u);
    g_d1_last_what = where[3];
    unsigned int zero[4] = {0, 0, 0, 0};
    e = cudaMemcpyToSymbol(g_d1_where, zero, sizeof(zero));
    if (e != cudaSuccess) return e;
    return cudaMemcpyToSymbol(g_d1_error, zero, sizeof(unsigned int));
  }
  return cudaSuccess;
}

unsigned int decode1_last_detail() { return g_d1_last_what; }

}  // namespace tl
