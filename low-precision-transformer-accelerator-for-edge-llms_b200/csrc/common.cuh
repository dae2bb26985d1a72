// common.cuh -- shared device helpers for the sm_100a kernels.
//
// Rounding discipline: every float operation whose result feeds an INT8
// quantization threshold is written with an explicit round-to-nearest
// intrinsic (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn) so that nvcc cannot
// contract it into an FMA; that keeps those values bit-identical to NumPy's
// float32 arithmetic in the reference golden model.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define TL_DEV __device__ __forceinline__

namespace tl {

constexpr int kHeadDim = 64;
constexpr int kWarp = 32;

// ---------------------------------------------------------------- PTX bits
TL_DEV int4 ld_stream_v4(const void* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

TL_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
TL_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

TL_DEV int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

TL_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
TL_DEV int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
TL_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Non-negative floats order like their bit patterns, so atomicMax on the
// bits is a float max for |x| values.
TL_DEV void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

// Packed argmax key: order-preserving bits of the float value above the
// complement of the index, so the 64-bit maximum is the largest value and,
// among equal values, the lowest index (np.argmax, argmax_reduction.sv:47-58).
TL_DEV unsigned long long argmax_key(float v, int idx) {
  unsigned int b = __float_as_uint(v);
  unsigned int ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<unsigned int>(idx));
}
TL_DEV int argmax_key_index(unsigned long long k) {
  return static_cast<int>(0xFFFFFFFFu - static_cast<unsigned int>(k & 0xFFFFFFFFull));
}

// ------------------------------------------------------------ quantization
// quantize_int8 (model/tinyllama_gemm_int8.py:36-42): scale = absmax/127 in
// float64 (1.0 when absmax == 0); q = clip(rint(x / float32(scale))).
TL_DEV double quant_scale64(float absmax) {
  return absmax == 0.0f ? 1.0 : static_cast<double>(absmax) / 127.0;
}
TL_DEV int quantize_one(float x, float scale_f32) {
  float q = rintf(__fdiv_rn(x, scale_f32));
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return static_cast<int>(q);
}
// quantize_one without a division per element: inv = __fdiv_rn(1, scale)
// (correctly rounded) is computed once per group. a = x * inv lies within
// 2^-23 |x / scale| <= 1.6e-5 of x / scale for |x / scale| < 128, and
// fl(x / scale) within 7.7e-6 of it, so rint(a) = rint(fl(x / scale)) unless
// a is within 1e-4 of a half-integer, where the division decides; |a| >= 128
// rounds past 127 either way. The result equals quantize_one for every x.
TL_DEV int quantize_one_inv(float x, float scale_f32, float inv) {
  const float a = __fmul_rn(x, inv);
  if (fabsf(a) >= 128.0f) return a < 0.0f ? -127 : 127;
  float q = rintf(a);
  if (fabsf(a - q) > 0.4999f) q = rintf(__fdiv_rn(x, scale_f32));
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return static_cast<int>(q);
}
TL_DEV float quant_inv(float scale_f32) { return __fdiv_rn(1.0f, scale_f32); }
// dequantize_int32 (model/tinyllama_gemm_int8.py:45-46) with a float64
// product of the two scales rounded to float32 once.
TL_DEV float dequant(int acc, double sx, double sw) {
  return __fmul_rn(__int2float_rn(acc), static_cast<float>(sx * sw));
}

// requantize_scalar (rtl/compute/requantize_unit.sv:39-93).
TL_DEV int requant_q16(int acc, uint32_t scale_q16, bool nonneg) {
  long long prod = static_cast<long long>(acc) * static_cast<long long>(scale_q16);
  unsigned long long mag = prod < 0 ? static_cast<unsigned long long>(-prod)
                                    : static_cast<unsigned long long>(prod);
  unsigned long long q = mag >> 16;
  unsigned long long rem = mag & 0xFFFFull;
  if (rem > 0x8000ull || (rem == 0x8000ull && (q & 1ull))) q += 1;
  long long s = prod < 0 ? -static_cast<long long>(q) : static_cast<long long>(q);
  long long lo = nonneg ? 0 : -127;
  if (s > 127) s = 127;
  if (s < lo) s = lo;
  return static_cast<int>(s);
}

// ------------------------------------------- NumPy float32 pairwise summation
// NumPy reduces a contiguous float32 row as: runs longer than 128 split at
// n/2 rounded down to a multiple of 8; a run of 8..128 keeps eight running
// sums over stride 8, folded ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then adds
// the n%8 tail in order. When every split is exact (n = 2^a * L, L <= 128,
// L % 8 == 0 -- true for TinyLlama's hidden size 2048 = 16 x 128) the tree
// is balanced: 2^a leaves of L elements, combined level by level
// left + right. norm_plan() checks that shape on the host; the device side
// (block_sumsq_numpy) evaluates exactly that tree.
struct NormPlan {
  int leaf_len;   // L
  int n_leaves;   // 2^a
};

inline bool norm_plan(int n, NormPlan* p) {
  int len = n;
  int leaves = 1;
  while (len > 128) {
    int h = len / 2;
    h -= h % 8;
    if (h * 2 != len) return false;
    len = h;
    leaves *= 2;
  }
  if (len < 8 || len % 8 != 0) return false;
  p->leaf_len = len;
  p->n_leaves = leaves;
  return leaves <= 1024;
}

// Sum of v[i]^2 over v[0..n) in NumPy's order; all threads of the block call
// it; `part` is shared scratch of n_leaves*8 floats, `leaf` of n_leaves.
// Returns the total in every thread.
TL_DEV float block_sumsq_numpy(const float* v, NormPlan plan, float* part, float* leaf) {
  const int tid = threadIdx.x, bs = blockDim.x;
  const int L = plan.leaf_len, nl = plan.n_leaves;
  for (int idx = tid; idx < nl * 8; idx += bs) {
    const int l = idx >> 3, j = idx & 7;
    const float* x = v + l * L;
    float r = __fmul_rn(x[j], x[j]);
    for (int i = 8 + j; i < L; i += 8) r = __fadd_rn(r, __fmul_rn(x[i], x[i]));
    part[idx] = r;
  }
  __syncthreads();
  for (int l = tid; l < nl; l += bs) {
    const float* q = part + l * 8;
    leaf[l] = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3])),
                        __fadd_rn(__fadd_rn(q[4], q[5]), __fadd_rn(q[6], q[7])));
  }
  __syncthreads();
  for (int st = 1; st < nl; st *= 2) {
    for (int l = tid * 2 * st; l < nl; l += bs * 2 * st) leaf[l] = __fadd_rn(leaf[l], leaf[l + st]);
    __syncthreads();
  }
  return leaf[0];
}

}  // namespace tl
