// gemm_tcgen05.cu -- INT8 x INT8 -> INT32 GEMM on the 5th-generation tensor
// cores (tcgen05.mma kind::i8), TMA-fed shared memory, TMEM accumulators.
//
// The reference reuses one shared INT8 GEMM engine for every projection
// (rtl/compute/shared_gemm_engine.sv:127-168; numerics of quantized_linear,
// model/tinyllama_gemm_int8.py:59-88). Here it is one kernel with the
// engine's fused epilogues (dequantize, residual add, SiLU*up, Q16.16
// requantize of rtl/compute/requantize_unit.sv:39-93, raw INT32).
//
// Orientation ("swap AB"): the weight tile is the MMA's A operand (128 output
// channels per CTA, K-major W^T[N][K]) and the token tile is B (BN tokens,
// K-major X[M][K]); the accumulator D[n][m] lives in TMEM as 128 lanes x BN
// columns. Decode batches of 16..64 tokens then still fill the 128-row MMA,
// and the epilogue thread that owns TMEM lane n writes out[m][n] for
// consecutive n across a warp (coalesced).
//
// Pipeline per CTA (128 threads): warp 0 lane 0 issues TMA loads into a ring
// of `stages` (A 16 KB + B BN*128 B, 128-byte swizzle); warp 1 lane 0 issues
// four 128xBNx32 MMAs per stage and commits each stage back to its producer
// barrier; warps 2 and 3 meanwhile fetch the weight and activation scales
// into shared memory; all four warps then drain TMEM with tcgen05.ld. The
// kernel is instantiated per tile width, epilogue and split count, so the
// epilogue is straight-line code. With k_splits > 1 the CTAs of one tile
// (a cluster of 1 x 1 x k_splits) each reduce a K range; the INT32 partials
// are exchanged with bulk async copies between the CTAs' shared memories as
// soon as each CTA's MMAs are done (no cluster-wide barrier) and summed
// locally (integer addition: exact, order-free), each CTA running
// the epilogue for 128 / k_splits of the tile's channels.
//
// No TMA multicast is used anywhere. Every mbarrier wait is bounded (about a
// second of clock cycles); on expiry the kernel records an error code in
// g_tc_error and skips ahead so that TMEM is still freed and the host sees
// TL_ERR_TIMEOUT instead of a hung GPU.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace tl {

__device__ unsigned int g_tc_error = 0;

namespace {

constexpr int kTcThreads = 128;
constexpr int kTileN = 128;      // weight rows per CTA (MMA M)
constexpr int kTileK = 128;      // bytes of K per stage (one 128-byte swizzle row)
constexpr int kABytes = kTileN * kTileK;
// Split-K receive area of one CTA, outside the operand ring: KS slices of
// 128 / KS accumulator rows, each row BN + 4 int32 (the padding keeps 16-byte
// accesses to consecutive rows bank-conflict free).
__host__ __device__ constexpr uint32_t tc_recv_bytes(int bn, int ks) {
  return ks > 1 ? static_cast<uint32_t>(kTileN * (bn + 4) * 4) : 0u;
}

// Bounded wait on the GEMM's error word.
TL_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  return mbar_wait_err(bar, parity, code, &g_tc_error);
}

TL_DEV float silu_mul_tc(float g, float u) {
  float c = fminf(fmaxf(g, -60.0f), 60.0f);
  float den = __fadd_rn(1.0f, expf(-c));
  return __fmul_rn(__fdiv_rn(g, den), u);
}

// Per-channel constants of output channel n that the epilogue needs,
// loaded before the accumulator is ready.
struct ChanConst {
  double sw = 0.0;    // weight scale (float epilogues)
  uint32_t rq = 0u;   // Q16.16 requantize multiplier (EPI_REQ)
};
template <int EPI>
TL_DEV ChanConst chan_const(const TcArgs& a, int n) {
  ChanConst c;
  if (n >= a.N) return c;
  if (EPI == EPI_REQ) c.rq = a.req_scale[a.req_per_col ? n : 0];
  else if (EPI != EPI_I32) c.sw = a.w_scale[n];
  return c;
}

// Writes the output element(s) of accumulator `acc` at (token m, channel n);
// `y` is the dequantized value (float epilogues), `partner` the value of
// channel n ^ 1 (SiLU pairs rows 2j, 2j+1 into output column j). Returns
// |value written| for the optional per-token absmax (0 when nothing written).
template <int EPI>
TL_DEV float tc_store(const TcArgs& a, int n, int m, int acc, float y, float partner, float resid,
                      const ChanConst& c) {
  const size_t o = static_cast<size_t>(m) * a.N + n;
  if (EPI == EPI_I32) {
    a.out_i32[o] = acc;
    return 0.0f;
  } else if (EPI == EPI_REQ) {
    a.out_i8[o] = static_cast<int8_t>(requant_q16(acc, c.rq, a.req_nonneg != 0));
    return 0.0f;
  } else if (EPI == EPI_SILU) {
    if (n & 1) return 0.0f;
    const float h = silu_mul_tc(y, partner);
    a.out_f32[static_cast<size_t>(m) * (a.N >> 1) + (n >> 1)] = h;
    return fabsf(h);
  } else if (EPI == EPI_RESID) {
    const float r = __fadd_rn(resid, y);
    a.out_f32[o] = r;
    return fabsf(r);
  } else {
    if (a.out_f32) a.out_f32[o] = y;
    return fabsf(y);
  }
}

// Per-token maximum over the 32 lanes of a warp of 16 packed argmax keys
// (one per token of a 16-token group, lane = output channel): four
// exchange-and-keep-half steps (16 -> 8 -> 4 -> 2 -> 1 keys per lane) and a
// final pair exchange. Returns the warp maximum of token
// 8 b4 + 4 b3 + 2 b2 + b1 (bits of the lane index), held by both lanes of
// each even/odd pair: 16 64-bit shuffles instead of 16 full reductions.
template <typename T>
TL_DEV T warp_max16(const T* k, int lane, int& token) {
  T a8[8], a4[4], a2[2];
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const T keep = b4 ? k[i + 8] : k[i], send = b4 ? k[i] : k[i + 8];
    const T r = __shfl_xor_sync(0xffffffffu, send, 16);
    a8[i] = keep > r ? keep : r;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T keep = b3 ? a8[i + 4] : a8[i], send = b3 ? a8[i] : a8[i + 4];
    const T r = __shfl_xor_sync(0xffffffffu, send, 8);
    a4[i] = keep > r ? keep : r;
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const T keep = b2 ? a4[i + 2] : a4[i], send = b2 ? a4[i] : a4[i + 2];
    const T r = __shfl_xor_sync(0xffffffffu, send, 4);
    a2[i] = keep > r ? keep : r;
  }
  const T keep = b1 ? a2[1] : a2[0], send = b1 ? a2[0] : a2[1];
  const T r = __shfl_xor_sync(0xffffffffu, send, 2);
  T m = keep > r ? keep : r;
  const T o = __shfl_xor_sync(0xffffffffu, m, 1);
  m = m > o ? m : o;
  token = (b4 ? 8 : 0) + (b3 ? 4 : 0) + (b2 ? 2 : 0) + (b1 ? 1 : 0);
  return m;
}

// Split-K reduction slice of one thread: KS CTAs of a cluster each reduce
// R = 128 / KS accumulator rows (output channels) over all peers. Thread t
// takes row t % R and a run of BN / KS consecutive tokens; for SiLU it takes
// the row pair (2p, 2p+1), p = t % (R / 2), and a run of BN / (2 KS) tokens,
// so both halves of each output live in the same thread. Either way a thread
// issues exactly BN / 4 sixteen-byte DSMEM loads, all before the first add.
template <int BN, int KS, int EPI>
struct SplitSlice {
  static constexpr int R = 128 / KS;
  static constexpr bool kPair = EPI == EPI_SILU;
  static constexpr int kRowsPer = kPair ? 2 : 1;
  static constexpr int kLanesPerRun = kPair ? R / 2 : R;   // threads sharing a token run
  static constexpr int kTok = BN * kLanesPerRun / 128;     // tokens per thread
  static constexpr int kQuads = kTok / 4;                  // int4 per (row, peer)
  static_assert(kTok % 4 == 0 && kQuads >= 1, "split slice must be whole int4s");
};

template <int BN, int EPI, int KS>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, TcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ double sx_sm[BN];
  __shared__ double sw_sm[kTileN];
  __shared__ unsigned int amax_sm[BN];
  __shared__ unsigned long long key_sm[EPI == EPI_F32 ? BN : 1];
  __shared__ int issued_sm;  // k-blocks whose TMA loads this CTA issued
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kBBytes = BN * kTileK;
  constexpr int kStage = kABytes + kBBytes;
  constexpr int kTmemCols = BN < 32 ? 32 : BN;
  constexpr bool kFloatEpi = EPI != EPI_I32 && EPI != EPI_REQ;
  const int stages = a.stages;
  int* recv_area = reinterpret_cast<int*>(smem + stages * kStage);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * kStage + tc_recv_bytes(BN, KS));
  uint64_t* empty = full + stages;
  uint64_t* done = empty + stages;
  uint64_t* recv_bar = done + 1;  // split-K: peers' partial slices have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTileN, m0 = blockIdx.y * BN;
  const int nkb = (a.K + kTileK - 1) / kTileK;
  const int kb0 = static_cast<int>(static_cast<long long>(blockIdx.z) * nkb / KS);
  const int kb1 = static_cast<int>(static_cast<long long>(blockIdx.z + 1) * nkb / KS);
  const bool has_amax = kFloatEpi && a.out_absmax != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(done, 1);
    mbar_init(recv_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x)) : "memory");
  }
  for (int j = threadIdx.x; j < BN; j += kTcThreads) amax_sm[j] = 0u;
  if constexpr (EPI == EPI_F32)
    for (int j = threadIdx.x; j < BN; j += kTcThreads) key_sm[j] = 0ull;
  const bool has_key = EPI == EPI_F32 && a.am_key != nullptr;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // split-K: this CTA's receive barrier is initialised; peers wait for this
  // arrive before their first copy into this CTA
  if constexpr (KS > 1) cluster_arrive_relaxed();

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // Weights do not depend on the previous kernel: the first `pre` weight
    // tiles are requested before griddepcontrol.wait, so under programmatic
    // dependent launch they stream while the producer of X is finishing.
    const int pre = min(stages, kb1 - kb0);
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(full + i, kStage);
      tma_load_2d(smem + i * kStage, &tm_w, (kb0 + i) * kTileK, n0, full + i);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(smem + i * kStage + kABytes, &tm_x, (kb0 + i) * kTileK, m0, full + i);
    int issued = pre;
    for (int kb = kb0 + pre, i = pre; kb < kb1 && ok; ++kb, ++i) {
      const int s = i % stages, round = i / stages;
      ok = mbar_wait(empty + s, (round - 1) & 1, 1u);
      if (!ok) break;
      mbar_arrive_expect_tx(full + s, kStage);
      tma_load_2d(smem + s * kStage, &tm_w, kb * kTileK, n0, full + s);
      tma_load_2d(smem + s * kStage + kABytes, &tm_x, kb * kTileK, m0, full + s);
      issued = i + 1;
    }
    issued_sm = issued;
  } else if (warp == 1 && lane == 0) {
    pdl_wait();
    constexpr uint32_t idesc = idesc_i8(kTileN, BN);
    for (int kb = kb0, i = 0; kb < kb1 && ok; ++kb, ++i) {
      const int s = i % stages, round = i / stages;
      ok = mbar_wait(full + s, round & 1, 2u);
      if (!ok) break;
      tc_fence_after();
      const uint64_t ad = smem_desc_sw128(smem_u32(smem + s * kStage));
      const uint64_t bd = smem_desc_sw128(smem_u32(smem + s * kStage + kABytes));
#pragma unroll
      for (int kk = 0; kk < kTileK / 32; ++kk)
        mma_i8(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      mma_commit(empty + s);
    }
    mma_commit(done);  // arrives once every MMA issued above has completed
  } else if (warp >= 2) {
    // Warps 2 and 3 fetch the epilogue's constants while the MMAs run: the
    // weight scales of this CTA's 128 channels, then (once the producer of X
    // has finished) the per-token activation scales absmax / 127 in float64.
    const int t = threadIdx.x - 64;
    if (kFloatEpi)
      for (int j = t; j < kTileN; j += 64) sw_sm[j] = n0 + j < a.N ? a.w_scale[n0 + j] : 0.0;
    pdl_wait();
    if (kFloatEpi)
      for (int j = t; j < BN; j += 64) {
        const int m = m0 + j;
        sx_sm[j] = (m < a.M && a.in_absmax) ? quant_scale64(a.in_absmax[m / a.rows_per_group]) : 1.0;
      }
  }
  // every thread reads the previous kernel's outputs (residuals) below
  pdl_wait();
  __syncwarp();
  // all threads: accumulator ready (uniform across the CTA); also publishes
  // sw_sm / sx_sm / amax_sm
  const bool ready = __syncthreads_and(mbar_wait(done, 0, 3u) ? 1 : 0) != 0;
  tc_fence_after();
  pdl_launch_dependents();

  const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  if constexpr (KS == 1) {
    const int nl = warp * 32 + lane;
    const int n = n0 + nl;
    const bool n_ok = n < a.N;
    ChanConst cc;
    if (EPI == EPI_REQ) cc = chan_const<EPI>(a, n);
    else cc.sw = sw_sm[nl];
    // residuals of the first 16 tokens; each chunk prefetches the next
    float rcur[16], rnext[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      rcur[j] = 0.0f;
      rnext[j] = 0.0f;
    }
    if (EPI == EPI_RESID && n_ok) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (m0 + j < a.M) rcur[j] = a.resid[static_cast<size_t>(m0 + j) * a.N + n];
    }
    if (ready && kb1 > kb0) {
#pragma unroll 1
      for (int c = 0; c < BN / 16; ++c) {
        const int mc = m0 + c * 16;
        if (EPI == EPI_RESID && n_ok && c + 1 < BN / 16) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            rnext[j] = (mc + 16 + j < a.M) ? a.resid[static_cast<size_t>(mc + 16 + j) * a.N + n] : 0.0f;
        }
        int v[16];
        tmem_ld16(lane_base + c * 16, v);
        unsigned long long key[16];
        // when the 16 tokens share one absmax group (prefill: one sequence),
        // the chunk's maximum is reduced in registers and across the warp
        // and lands with one shared atomic per warp instead of one per element
        const bool one_group = has_amax && mc / a.rows_per_group == (mc + 15) / a.rows_per_group;
        float chunk_max = 0.0f;
        uint32_t mag_bits[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = mc + j;
          const float y = kFloatEpi ? dequant(v[j], sx_sm[c * 16 + j], cc.sw) : 0.0f;
          const float partner = EPI == EPI_SILU ? __shfl_xor_sync(0xffffffffu, y, 1) : 0.0f;
          key[j] = 0ull;
          mag_bits[j] = 0u;
          if (n_ok && m < a.M) {
            const float mag = tc_store<EPI>(a, n, m, v[j], y, partner, rcur[j], cc);
            if (one_group) chunk_max = fmaxf(chunk_max, mag);
            mag_bits[j] = __float_as_uint(mag);  // non-negative: bit order is value order
            if (EPI == EPI_F32) key[j] = argmax_key(y, n);
          }
        }
        if (one_group) {
          chunk_max = warp_max(chunk_max);
          if (lane == 0) atomicMax(amax_sm + c * 16, __float_as_uint(chunk_max));
        } else if (has_amax) {
          // one row max per token: reduced across the warp's 32 channels
          // first (transposed butterfly), then one shared atomic per token
          // and warp instead of 32
          int tok;
          const uint32_t mm = warp_max16(mag_bits, lane, tok);
          if ((lane & 1) == 0 && mm) atomicMax(amax_sm + c * 16 + tok, mm);
        }
        if (EPI == EPI_F32 && has_key) {
          int tok;
          const unsigned long long km = warp_max16(key, lane, tok);
          if ((lane & 1) == 0 && km) atomicMax(key_sm + c * 16 + tok, km);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) rcur[j] = rnext[j];
      }
    }
  } else {
    // Split-K across the CTAs of one cluster (cluster dims 1 x 1 x KS): each
    // CTA parks its INT32 partial tile [128 n][BN m] (row stride BN + 4 ints)
    // in its own operand ring (idle once its MMAs are done). CTA `rank` owns
    // rows [rank*R, (rank+1)*R): right away, with no cluster-wide barrier,
    // every CTA pushes the rows each peer owns into that peer's receive area
    // (separate from the peer's ring, so the peer may still be computing)
    // with bulk async copies (shared::cta -> shared::cluster), whose
    // completion lands on the receiver's mbarrier; each CTA then sums its
    // rows over the KS slices from its own shared memory and runs the
    // epilogue for them. Integer addition: exact and order-free.
    using SL = SplitSlice<BN, KS, EPI>;
    constexpr int PS = BN + 4;
    constexpr uint32_t kSliceBytes = SL::R * PS * 4;
    int* part = reinterpret_cast<int*>(smem);
    static_assert(2 * kStage >= kTileN * PS * 4, "two ring stages must hold the parked partial tile");
    int* recv = recv_area;  // [KS][R][PS], slot p from CTA p
    const int nl = warp * 32 + lane;
    const int rank = static_cast<int>(cluster_rank());
    // this thread's slice and the residuals / constants it needs (issued now,
    // consumed after the reduction)
    const int sub = threadIdx.x % SL::kLanesPerRun;
    const int run = threadIdx.x / SL::kLanesPerRun;
    const int rl = sub * SL::kRowsPer;                 // first row of the slice within the owned rows
    const int r0 = rank * SL::R + rl;                  // ... within the tile
    const int t0 = run * SL::kTok;                     // first token (in the tile)
    float rres[SL::kRowsPer][SL::kTok];
    ChanConst cc[SL::kRowsPer];
#pragma unroll
    for (int h = 0; h < SL::kRowsPer; ++h) {
      const int n = n0 + r0 + h;
      if (EPI == EPI_REQ) cc[h] = chan_const<EPI>(a, n);
      else cc[h].sw = sw_sm[r0 + h];
#pragma unroll
      for (int j = 0; j < SL::kTok; ++j) {
        const int m = m0 + t0 + j;
        rres[h][j] = (EPI == EPI_RESID && n < a.N && m < a.M) ? a.resid[static_cast<size_t>(m) * a.N + n] : 0.0f;
      }
    }
    if (ready) {
#pragma unroll
      for (int c = 0; c < BN / 16; ++c) {
        int v[16];
        tmem_ld16(lane_base + c * 16, v);
        int4* dst = reinterpret_cast<int4*>(part + nl * PS + c * 16);
        dst[0] = make_int4(v[0], v[1], v[2], v[3]);
        dst[1] = make_int4(v[4], v[5], v[6], v[7]);
        dst[2] = make_int4(v[8], v[9], v[10], v[11]);
        dst[3] = make_int4(v[12], v[13], v[14], v[15]);
      }
    }
    // the bulk copies read `part` through the async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();  // this CTA's partial is parked
    cluster_wait();   // every peer has started (pairs with the arrive above)
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(recv_bar, (KS - 1) * kSliceBytes);
      const uint32_t bar_local = smem_u32(recv_bar);
      const uint32_t dst_local = smem_u32(recv + rank * SL::R * PS);
#pragma unroll
      for (int p = 0; p < KS; ++p) {
        if (p == rank) continue;
        uint32_t dst, bar;
        asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(dst_local), "r"(static_cast<uint32_t>(p)));
        asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(bar) : "r"(bar_local), "r"(static_cast<uint32_t>(p)));
        asm volatile(
            "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
            ::"r"(dst), "r"(smem_u32(part + p * SL::R * PS)), "r"(kSliceBytes), "r"(bar)
            : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    bool got = mbar_wait(recv_bar, 0, 4u);
    // a timed-out receive (error already recorded): give late pushes from
    // peers one more bounded wait to land before this CTA moves on to exit
    if (!got && threadIdx.x == 0) mbar_wait(recv_bar, 0, 4u);
    if (ready && got) {
#pragma unroll
      for (int q = 0; q < SL::kQuads; ++q) {
        int acc[SL::kRowsPer][4];
#pragma unroll
        for (int h = 0; h < SL::kRowsPer; ++h) {
          const int4 own = *reinterpret_cast<const int4*>(part + (r0 + h) * PS + t0 + 4 * q);
          acc[h][0] = own.x;
          acc[h][1] = own.y;
          acc[h][2] = own.z;
          acc[h][3] = own.w;
#pragma unroll
          for (int p = 0; p < KS; ++p) {
            if (p == rank) continue;
            const int4 v = *reinterpret_cast<const int4*>(recv + (p * SL::R + rl + h) * PS + t0 + 4 * q);
            acc[h][0] += v.x;
            acc[h][1] += v.y;
            acc[h][2] += v.z;
            acc[h][3] += v.w;
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int tt = t0 + 4 * q + j;
          const int m = m0 + tt;
          if (m >= a.M) continue;
          if (SL::kPair) {
            const int n = n0 + r0;  // even channel of the pair
            if (n + 1 < a.N) {
              const float g = dequant(acc[0][j], sx_sm[tt], cc[0].sw);
              const float u = dequant(acc[SL::kRowsPer - 1][j], sx_sm[tt], cc[SL::kRowsPer - 1].sw);
              const float mag = tc_store<EPI>(a, n, m, acc[0][j], g, u, 0.0f, cc[0]);
              if (has_amax) atomicMax(amax_sm + tt, __float_as_uint(mag));
            }
          } else {
            const int n = n0 + r0;
            if (n < a.N) {
              const float y = kFloatEpi ? dequant(acc[0][j], sx_sm[tt], cc[0].sw) : 0.0f;
              const float mag = tc_store<EPI>(a, n, m, acc[0][j], y, 0.0f, rres[0][4 * q + j], cc[0]);
              if (has_amax) atomicMax(amax_sm + tt, __float_as_uint(mag));
              if (EPI == EPI_F32 && has_key) atomicMax(key_sm + tt, argmax_key(y, n));
            }
          }
        }
      }
    }
    // this CTA's outgoing copies must have read `part` before it exits
    if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  // After a failed wait anywhere (the error word is set) this CTA's own TMA
  // loads may still be in flight into its ring (the producer or the MMA
  // warp stopped early): wait, bounded, for the last phase issued on every
  // stage so that no copy lands in shared memory after the CTA has exited.
  // In a CTA without failure these phases have all completed already.
  if (threadIdx.x == 0 && *reinterpret_cast<volatile unsigned int*>(&g_tc_error) != 0u) {
    const int n = issued_sm;
    for (int i = max(0, n - stages); i < n; ++i) mbar_wait(full + i % stages, (i / stages) & 1, 5u);
  }
  tc_fence_before();
  __syncthreads();
  if (has_amax && ready) {
    for (int j = threadIdx.x; j < BN; j += kTcThreads) {
      const int m = m0 + j;
      if (m < a.M && amax_sm[j]) atomic_max_nonneg(a.out_absmax + m / a.rows_per_group, __uint_as_float(amax_sm[j]));
    }
  }
  if constexpr (EPI == EPI_F32) {
    if (has_key && ready)
      for (int j = threadIdx.x; j < BN; j += kTcThreads)
        if (m0 + j < a.M && key_sm[j]) atomicMax(a.am_key + m0 + j, key_sm[j]);
  }
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------ persistent wide-tile GEMM
// Prefill-sized problems (M > 128 tokens, no split-K) run on a persistent
// kernel: one CTA per SM walks the 128-channel x 256-token tiles
// t = blockIdx.x, blockIdx.x + gridDim.x, ... (channel tile fastest, so the
// CTAs in flight share token tiles in L2). Roles: warp 0 lane 0 streams A/B
// k-blocks through a 4-stage ring (48 KB a stage) across tile boundaries;
// warp 1 lane 0 issues the MMAs of tile i into TMEM accumulator i % 2 (two
// 256-column buffers, all 512 columns); warps 2.. drain accumulator i % 2
// while tile i + 1 accumulates in the other, so the epilogue runs under the
// main loop instead of after it. Epilogue warp w reads TMEM lanes
// 32 (w % 4) .. + 31 (the lanes its warp rank may access) and token chunks
// [16 p / P, 16 (p + 1) / P) of 16 tokens, p = (w - 2) / 4, with P epilogue
// warps per lane quarter. Handshakes: acc_full[b] (MMA commit -> epilogue),
// acc_empty[b] (one arrival per epilogue warp -> MMA).
// Epilogue warps per epilogue kind: 16 (four per TMEM lane quarter, four
// 16-token chunks each) keep the SiLU*up and float epilogues ahead of the
// MMAs (prefill 8 x 2048: 39.6 vs 40.9 ms with 12); the residual epilogue
// keeps 12, where 16 would spill its prefetched residual registers.
template <int EPI>
__host__ __device__ constexpr int tcp_epi_warps() { return EPI == EPI_RESID ? 12 : 16; }
template <int EPI>
__host__ __device__ constexpr int tcp_threads() { return 32 * (2 + tcp_epi_warps<EPI>()); }
constexpr int kPBN = 256;
constexpr int kPStages = 4;
constexpr int kPStage = kABytes + kPBN * kTileK;

template <int EPI>
__global__ void __launch_bounds__(tcp_threads<EPI>(), 1)
    gemm_tcp_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, TcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr bool kFloatEpi = EPI != EPI_I32 && EPI != EPI_REQ;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPStages * kPStage);
  uint64_t* empty = full + kPStages;
  uint64_t* acc_full = empty + kPStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (a.N + kTileN - 1) / kTileN;
  const int tiles = n_tiles * ((a.M + kPBN - 1) / kPBN);
  const int nkb = (a.K + kTileK - 1) / kTileK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, tcp_epi_warps<EPI>());
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x)) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kPBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int n0 = (t % n_tiles) * kTileN, m0 = (t / n_tiles) * kPBN;
        int kb = 0;
        if (t == static_cast<int>(blockIdx.x)) {
          // weights do not depend on the previous kernel: the first ring's
          // worth is requested before the grid-dependency wait
          const int pre = min(kPStages, nkb);
          for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(full + i, kPStage);
            tma_load_2d(smem + i * kPStage, &tm_w, i * kTileK, n0, full + i);
          }
          pdl_wait();
          for (int i = 0; i < pre; ++i)
            tma_load_2d(smem + i * kPStage + kABytes, &tm_x, i * kTileK, m0, full + i);
          kb = it = pre;
        }
        for (; kb < nkb; ++kb, ++it) {
          const int s = it % kPStages, round = it / kPStages;
          if (round > 0 && !(ok = mbar_wait(empty + s, (round - 1) & 1, 11u))) break;
          mbar_arrive_expect_tx(full + s, kPStage);
          tma_load_2d(smem + s * kPStage, &tm_w, kb * kTileK, n0, full + s);
          tma_load_2d(smem + s * kPStage + kABytes, &tm_x, kb * kTileK, m0, full + s);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kTileN, kPBN);
      bool ok = true;
      int it = 0, i = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const int b = i & 1, u = i >> 1;
        if (u > 0 && !(ok = mbar_wait(acc_empty + b, (u - 1) & 1, 12u))) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * kPBN);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kPStages, round = it / kPStages;
          if (!(ok = mbar_wait(full + s, round & 1, 13u))) break;
          tc_fence_after();
          const uint64_t ad = smem_desc_sw128(smem_u32(smem + s * kPStage));
          const uint64_t bd = smem_desc_sw128(smem_u32(smem + s * kPStage + kABytes));
#pragma unroll
          for (int kk = 0; kk < kTileK / 32; ++kk)
            mma_i8(d, ad + 2 * kk, bd + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(empty + s);
        }
        mma_commit(acc_full + b);  // arrives once this tile's MMAs have completed
      }
    }
  } else {
    // epilogue warps
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;
    constexpr int kParts = tcp_epi_warps<EPI>() / 4;  // epilogue warps per TMEM lane quarter
    const int c0 = part * 16 / kParts, c1 = (part + 1) * 16 / kParts;  // this warp's 16-token chunks
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c0 * 16);
    const bool has_amax = kFloatEpi && a.out_absmax != nullptr;
    pdl_wait();  // token scales and residuals come from the previous kernel
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int b = i & 1, u = i >> 1;
      const int n0 = (t % n_tiles) * kTileN, m0 = (t / n_tiles) * kPBN + c0 * 16;
      const int n = n0 + q * 32 + lane;
      const bool n_ok = n < a.N;
      double sw = 0.0;
      uint32_t rq = 0u;
      if (EPI == EPI_REQ) {
        if (n_ok) rq = a.req_scale[a.req_per_col ? n : 0];
      } else if (kFloatEpi) {
        if (n_ok) sw = a.w_scale[n];
      }
      if (t + static_cast<int>(gridDim.x) >= tiles) pdl_launch_dependents();
      float rcur[16], rnext[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) rcur[j] = rnext[j] = 0.0f;
      if (EPI == EPI_RESID && n_ok) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (m0 + j < a.M) rcur[j] = a.resid[static_cast<size_t>(m0 + j) * a.N + n];
      }
      const bool ready = mbar_wait(acc_full + b, u & 1, 14u);
      tc_fence_after();
      if (!ready) break;
      // chunks of 16 tokens this warp holds; a warp with none still releases
      // the buffer (after the acc_full wait, so no arrival runs a phase ahead)
      const int nch = a.M > m0 ? min(c1 - c0, (a.M - m0 + 15) / 16) : 0;
      if (nch == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + b);
        continue;
      }
      // dequantization scale float32(sx * sw) of the current absmax group
      int cur_g = -1;
      float cur_s = 0.0f;
      // running |output| maximum of group run_g (flushed when it changes)
      int run_g = -1;
      float run_max = 0.0f;
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const int mc = m0 + c * 16;
        if (EPI == EPI_RESID && n_ok && c + 1 < nch) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            rnext[j] = (mc + 16 + j < a.M) ? a.resid[static_cast<size_t>(mc + 16 + j) * a.N + n] : 0.0f;
        }
        int v[16];
        tmem_ld16(lane_base + static_cast<uint32_t>(b * kPBN + c * 16), v);
        if (c == nch - 1) {
          // this warp's last read of accumulator b for this tile
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty + b);
        }
        const int mlast = min(mc + 15, a.M - 1);
        const int g0 = mc / a.rows_per_group, g1 = mlast / a.rows_per_group;
        const bool one_group = g0 == g1;
        float s[16];
        if (kFloatEpi) {
          if (one_group) {
            if (g0 != cur_g) {
              cur_g = g0;
              const double sx = a.in_absmax ? quant_scale64(a.in_absmax[g0]) : 1.0;
              cur_s = static_cast<float>(sx * sw);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) s[j] = cur_s;
          } else {
            const int mj = mc + (lane & 15);
            const double mine = (a.in_absmax && mj < a.M) ? quant_scale64(a.in_absmax[mj / a.rows_per_group]) : 1.0;
#pragma unroll
            for (int j = 0; j < 16; ++j) s[j] = static_cast<float>(__shfl_sync(0xffffffffu, mine, j) * sw);
          }
        }
        float mag[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) mag[j] = 0.0f;
        if (EPI == EPI_SILU) {
          // channel pairs (2p gate, 2p + 1 up) sit in adjacent lanes: the
          // even lane finishes tokens 0..7 of the chunk, the odd lane 8..15
          const bool odd = lane & 1;
          float y[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) y[j] = __fmul_rn(__int2float_rn(v[j]), s[j]);
          const int tok0 = odd ? 8 : 0;
          const size_t ldo = static_cast<size_t>(a.N >> 1);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float r = __shfl_xor_sync(0xffffffffu, odd ? y[j] : y[8 + j], 1);
            const float g = odd ? r : y[j];
            const float up = odd ? y[8 + j] : r;
            const int m = mc + tok0 + j;
            if (n_ok && m < a.M) {
              const float hv = silu_mul_tc(g, up);
              a.out_f32[static_cast<size_t>(m) * ldo + (n >> 1)] = hv;
              mag[j] = fabsf(hv);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = mc + j;
            if (!n_ok || m >= a.M) continue;
            const size_t o = static_cast<size_t>(m) * a.N + n;
            if (EPI == EPI_I32) {
              a.out_i32[o] = v[j];
            } else if (EPI == EPI_REQ) {
              a.out_i8[o] = static_cast<int8_t>(requant_q16(v[j], rq, a.req_nonneg != 0));
            } else {
              const float y = __fmul_rn(__int2float_rn(v[j]), s[j]);
              if (EPI == EPI_RESID) {
                const float r = __fadd_rn(rcur[j], y);
                a.out_f32[o] = r;
                mag[j] = fabsf(r);
              } else {
                if (a.out_f32) a.out_f32[o] = y;
                mag[j] = fabsf(y);
              }
            }
          }
        }
        if (has_amax) {
          if (one_group) {
            float cm = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) cm = fmaxf(cm, mag[j]);
            if (g0 != run_g) {
              if (run_g >= 0) {
                const float wm = warp_max(run_max);
                if (lane == 0 && wm > 0.0f) atomic_max_nonneg(a.out_absmax + run_g, wm);
              }
              run_g = g0;
              run_max = 0.0f;
            }
            run_max = fmaxf(run_max, cm);
          } else {
            // rows of this chunk span several groups: one warp maximum per
            // token (SiLU: mag[j] of an even lane is token j, of an odd lane
            // token 8 + j)
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float wm;
              int m;
              if (EPI == EPI_SILU) {
                const bool mine = (j < 8) == ((lane & 1) == 0);
                wm = warp_max(mine ? mag[j & 7] : 0.0f);
                m = mc + j;
              } else {
                wm = warp_max(mag[j]);
                m = mc + j;
              }
              if (lane == 0 && m < a.M && wm > 0.0f) atomic_max_nonneg(a.out_absmax + m / a.rows_per_group, wm);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) rcur[j] = rnext[j];
      }
      if (has_amax && run_g >= 0) {
        const float wm = warp_max(run_max);
        if (lane == 0 && wm > 0.0f) atomic_max_nonneg(a.out_absmax + run_g, wm);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kPBN));
  }
}

size_t tcp_smem() { return static_cast<size_t>(kPStages) * kPStage + 1024 + 8 * (2 * kPStages + 4) + 16; }

template <int EPI>
cudaError_t launch_tcp_e(const TcPlan& p, const TcArgs& a, cudaStream_t s, bool pdl) {
  const int tiles = ((a.N + kTileN - 1) / kTileN) * ((a.M + kPBN - 1) / kPBN);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(tiles, device_sm_count()));
  cfg.blockDim = dim3(tcp_threads<EPI>());
  cfg.dynamicSmemBytes = tcp_smem();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemm_tcp_kernel<EPI>, p.tm_w, p.tm_x, a);
}

cudaError_t launch_tcp(const TcPlan& p, const TcArgs& a, cudaStream_t s, bool pdl) {
  switch (a.epi) {
    case EPI_I32: return launch_tcp_e<EPI_I32>(p, a, s, pdl);
    case EPI_F32: return launch_tcp_e<EPI_F32>(p, a, s, pdl);
    case EPI_RESID: return launch_tcp_e<EPI_RESID>(p, a, s, pdl);
    case EPI_SILU: return launch_tcp_e<EPI_SILU>(p, a, s, pdl);
    case EPI_REQ: return launch_tcp_e<EPI_REQ>(p, a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prepare_tcp() {
  const int smem = static_cast<int>(tcp_smem());
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(gemm_tcp_kernel<EPI_I32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem))) return e;
  if ((e = cudaFuncSetAttribute(gemm_tcp_kernel<EPI_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem))) return e;
  if ((e = cudaFuncSetAttribute(gemm_tcp_kernel<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem))) return e;
  if ((e = cudaFuncSetAttribute(gemm_tcp_kernel<EPI_SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem))) return e;
  return cudaFuncSetAttribute(gemm_tcp_kernel<EPI_REQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

// The persistent kernel takes wide-tile problems without split-K and
// without the fused argmax; TL_DISABLE_PERSISTENT_GEMM=1 keeps them on the
// one-tile-per-CTA kernel (A/B comparisons).
bool use_tcp(const TcPlan& p, const TcArgs& a) {
  static const bool disabled = [] {
    const char* v = std::getenv("TL_DISABLE_PERSISTENT_GEMM");
    return v && v[0] == '1';
  }();
  return !disabled && p.bn == kPBN && p.k_splits == 1 && a.am_key == nullptr;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

cudaError_t get_encode() {
  if (g_encode) return cudaSuccess;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess) return e;
  if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return cudaSuccess;
}

template <int BN>
size_t tc_smem(int stages, int ks) {
  return static_cast<size_t>(stages) * (kABytes + BN * kTileK) + tc_recv_bytes(BN, ks) + 1024 +
         16 * (2 * stages + 3);
}

template <int BN, int EPI, int KS>
cudaError_t launch_tc_k(const TcPlan& p, const TcArgs& a, cudaStream_t s, bool pdl) {
  const size_t smem = tc_smem<BN>(a.stages, KS);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + kTileN - 1) / kTileN, (a.M + BN - 1) / BN, KS);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = 1;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = KS;
  ++na;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, EPI, KS>, p.tm_w, p.tm_x, a);
}

// Split counts a tile width supports: every thread's split-K slice must be
// whole 16-byte runs (BN / KS tokens, BN / (2 KS) for the SiLU row pairs).
constexpr bool tc_split_ok(int bn, int epi, int ks) {
  return ks == 1 || (bn <= 64 && (epi == EPI_SILU ? bn / (2 * ks) >= 4 : bn / ks >= 4));
}

template <int BN, int EPI>
cudaError_t launch_tc_e(const TcPlan& p, const TcArgs& a, cudaStream_t s, bool pdl) {
  switch (a.k_splits) {
    case 1: return launch_tc_k<BN, EPI, 1>(p, a, s, pdl);
    case 2: if constexpr (tc_split_ok(BN, EPI, 2)) return launch_tc_k<BN, EPI, 2>(p, a, s, pdl); break;
    case 4: if constexpr (tc_split_ok(BN, EPI, 4)) return launch_tc_k<BN, EPI, 4>(p, a, s, pdl); break;
    case 8: if constexpr (tc_split_ok(BN, EPI, 8)) return launch_tc_k<BN, EPI, 8>(p, a, s, pdl); break;
    default: break;
  }
  return cudaErrorInvalidValue;
}

template <int BN>
cudaError_t launch_tc_t(const TcPlan& p, const TcArgs& a, cudaStream_t s, bool pdl) {
  switch (a.epi) {
    case EPI_I32: return launch_tc_e<BN, EPI_I32>(p, a, s, pdl);
    case EPI_F32: return launch_tc_e<BN, EPI_F32>(p, a, s, pdl);
    case EPI_RESID: return launch_tc_e<BN, EPI_RESID>(p, a, s, pdl);
    case EPI_SILU: return launch_tc_e<BN, EPI_SILU>(p, a, s, pdl);
    case EPI_REQ: return launch_tc_e<BN, EPI_REQ>(p, a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int BN, int EPI, int KS>
cudaError_t prepare_tc_k() {
  if constexpr (!tc_split_ok(BN, EPI, KS)) {
    return cudaSuccess;
  } else {
    return cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(tc_smem<BN>(tc_max_stages(BN, KS), KS)));
  }
}

template <int BN, int EPI>
cudaError_t prepare_tc_e() {
  cudaError_t e;
  if ((e = prepare_tc_k<BN, EPI, 1>()) != cudaSuccess) return e;
  if ((e = prepare_tc_k<BN, EPI, 2>()) != cudaSuccess) return e;
  if ((e = prepare_tc_k<BN, EPI, 4>()) != cudaSuccess) return e;
  return prepare_tc_k<BN, EPI, 8>();
}

template <int BN>
cudaError_t prepare_tc_t() {
  cudaError_t e;
  if ((e = prepare_tc_e<BN, EPI_I32>()) != cudaSuccess) return e;
  if ((e = prepare_tc_e<BN, EPI_F32>()) != cudaSuccess) return e;
  if ((e = prepare_tc_e<BN, EPI_RESID>()) != cudaSuccess) return e;
  if ((e = prepare_tc_e<BN, EPI_SILU>()) != cudaSuccess) return e;
  return prepare_tc_e<BN, EPI_REQ>();
}

}  // namespace

// Ring depth: at most 4 stages (<= 96 KB for 64-token tiles), so two CTAs
// fit on an SM and the next kernel's CTAs can start under programmatic
// dependent launch. Wide prefill tiles keep the ring at <= 100 KB as well:
// with two CTAs per SM one CTA's epilogue runs under the other's main loop.
// Split-K CTAs also hold the receive area: ring + area stay <= 108 KB, still
// two CTAs per SM.
int tc_max_stages(int bn, int ks) {
  const int stage = kABytes + bn * kTileK;
  const int budget = ks > 1 ? 108 * 1024 - static_cast<int>(tc_recv_bytes(bn, ks)) : 100 * 1024;
  return std::max(2, std::min(4, budget / stage));
}

int tc_pick_bn(int M) {
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

cudaError_t tc_encode_operand(CUtensorMap* tm, const int8_t* base, int rows, int K, int box_rows) {
  cudaError_t e = get_encode();
  if (e != cudaSuccess) return e;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || K % 16 || rows <= 0 || box_rows > 256) return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// fp16 rows of 64 values (128 bytes) -> boxes of box_rows rows with the
// 128-byte swizzle: a box lands in shared memory as a K-major (or, read the
// other way, MN-major) SW128 operand tile, byte (row r, 16-byte chunk c) at
// r * 128 + ((c ^ (r & 7)) << 4). Rows past `rows` read as zero.
cudaError_t tc_encode_f16_rows64(CUtensorMap* tm, const void* base, long long rows, int box_rows) {
  cudaError_t e = get_encode();
  if (e != cudaSuccess) return e;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || rows <= 0 || box_rows < 8 || box_rows > 256 || box_rows % 8)
    return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {128};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t tc_make_plan(TcPlan* p, const int8_t* w_nk, int N, const int8_t* x, int M, int K, int num_sms, int epi) {
  p->bn = tc_pick_bn(M);
  cudaError_t e = tc_encode_operand(&p->tm_w, w_nk, N, K, kTileN);
  if (e != cudaSuccess) return e;
  e = tc_encode_operand(&p->tm_x, x, M, K, p->bn);
  if (e != cudaSuccess) return e;
  const int nkb = (K + kTileK - 1) / kTileK;
  const int tiles = ((N + kTileN - 1) / kTileN) * ((M + p->bn - 1) / p->bn);
  const int want = num_sms > 0 ? num_sms : 148;
  int ks = 1;
  // split K over a cluster of 2/4/8 CTAs until the grid covers the SMs;
  // only for tiles of <= 64 tokens (the partial tile must fit the ring)
  while (p->bn <= 64 && ks < 8 && tiles * ks < want && 2 * ks <= nkb && tc_split_ok(p->bn, epi, 2 * ks)) ks *= 2;
  p->k_splits = ks;
  const int per = (nkb + ks - 1) / ks;
  // (two stages always hold the parked split-K partial tile [128][bn + 4])
  p->stages = std::max(2, std::min(tc_max_stages(p->bn, ks), per));
  p->M = M;
  p->N = N;
  p->K = K;
  return cudaSuccess;
}

cudaError_t launch_gemm_tc(const TcPlan& p, const TcArgs& a0, cudaStream_t s, bool pdl) {
  TcArgs a = a0;
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.k_splits = p.k_splits;
  a.stages = p.stages;
  if (a.epi == EPI_SILU && (a.N % 2)) return cudaErrorInvalidValue;
  if (use_tcp(p, a)) return launch_tcp(p, a, s, pdl);
  switch (p.bn) {
    case 32: return launch_tc_t<32>(p, a, s, pdl);
    case 64: return launch_tc_t<64>(p, a, s, pdl);
    case 128: return launch_tc_t<128>(p, a, s, pdl);
    case 256: return launch_tc_t<256>(p, a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prepare_tc() {
  cudaError_t e;
  if ((e = prepare_tc_t<32>()) != cudaSuccess) return e;
  if ((e = prepare_tc_t<64>()) != cudaSuccess) return e;
  if ((e = prepare_tc_t<128>()) != cudaSuccess) return e;
  if ((e = prepare_tc_t<256>()) != cudaSuccess) return e;
  return prepare_tcp();
}

// Reads and clears the bounded-wait error words of the tcgen05 GEMM, the
// attention kernels, the persistent decode step and the tensor-parallel
// exchange (0 = none expired).
cudaError_t tc_read_error(unsigned int* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_tc_error, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  if (*code) {
    unsigned int zero = 0;
    return cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(unsigned int));
  }
  e = attn_read_error(code);
  if (e != cudaSuccess || *code) return e;
  e = decode1_read_error(code);
  if (e != cudaSuccess || *code) return e;
  return tp_read_error(code);
}

}  // namespace tl
