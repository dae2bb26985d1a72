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
// the n%8 tail in order; a run shorter than 8 is a plain ordered sum.
// pw_plan() lists the leaf runs in order (depth-first), pw_fold() adds leaf
// sums back up the same binary tree.
constexpr int kPwMaxLeaves = 128;

struct PwPlan {
  int n_leaves;
  int start[kPwMaxLeaves];
  int len[kPwMaxLeaves];
};

TL_DEV void pw_plan_rec(PwPlan& p, int start, int n) {
  if (n <= 128) {
    p.start[p.n_leaves] = start;
    p.len[p.n_leaves] = n;
    p.n_leaves++;
    return;
  }
  int h = n / 2;
  h -= h % 8;
  pw_plan_rec(p, start, h);
  pw_plan_rec(p, start + h, n - h);
}

// Leaf sum of v[0..n) for n <= 128, sequential per lane group: lane j (0..7)
// of an 8-lane group accumulates r[j]; lane 0 folds. Returns the value in
// lane 0 of the group (others hold partials).
TL_DEV float pw_leaf_group8(const float* v, int n, int j /*0..7*/, unsigned mask) {
  if (n < 8) {
    float acc = 0.0f;
    if (j == 0)
      for (int i = 0; i < n; ++i) acc = __fadd_rn(acc, v[i]);
    return acc;
  }
  int full = n - (n % 8);
  float r = v[j];
  for (int i = 8 + j; i < full; i += 8) r = __fadd_rn(r, v[i]);
  // fold ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) inside the 8-lane group
  float r1 = __shfl_down_sync(mask, r, 1, 8);
  float s01 = __fadd_rn(r, r1);                 // valid in even lanes
  float s23 = __shfl_down_sync(mask, s01, 2, 8);
  float s0123 = __fadd_rn(s01, s23);            // valid in lanes 0 and 4
  float s4567 = __shfl_down_sync(mask, s0123, 4, 8);
  float res = __fadd_rn(s0123, s4567);          // valid in lane 0
  if (j == 0)
    for (int i = full; i < n; ++i) res = __fadd_rn(res, v[i]);
  return res;
}

TL_DEV float pw_fold_rec(const float* leaf_sum, int& idx, int n) {
  if (n <= 128) return leaf_sum[idx++];
  int h = n / 2;
  h -= h % 8;
  float a = pw_fold_rec(leaf_sum, idx, h);
  float b = pw_fold_rec(leaf_sum, idx, n - h);
  return __fadd_rn(a, b);
}

}  // namespace tl
