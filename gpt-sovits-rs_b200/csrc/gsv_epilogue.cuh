// gsv_epilogue.cuh -- the fused epilogue shared by every tap-GEMM kernel.
#pragma once
#include <cuda_bf16.h>

#include "gsv_internal.h"

namespace gsv {

template <typename T>
__device__ __forceinline__ float ld_act(const void* p, size_t i);
template <>
__device__ __forceinline__ float ld_act<float>(const void* p, size_t i) {
  return static_cast<const float*>(p)[i];
}
template <>
__device__ __forceinline__ float ld_act<__nv_bfloat16>(const void* p, size_t i) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

template <typename T>
__device__ __forceinline__ void st_act(void* p, size_t i, float v);
template <>
__device__ __forceinline__ void st_act<float>(void* p, size_t i, float v) {
  static_cast<float*>(p)[i] = v;
}
template <>
__device__ __forceinline__ void st_act<__nv_bfloat16>(void* p, size_t i, float v) {
  static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// LeakyReLU of the reference (src/models/sovits_decoder.rs:46-53: sign-bit
// test, -0.0 takes the slope branch).  For a slope in [0, 1], max(v, v * slope)
// is the same function bit for bit (v * slope keeps v's sign, so -0.0 maps to
// -0.0 and a NaN stays a NaN) in two instructions instead of three.
__device__ __forceinline__ float lrelu(float v, float slope) {
  return fmaxf(v, v * slope);
}

// Epilogue value of one output element at flat index e (already in range):
// v = (acc + bias + bias_bc + residuals) / div, or 0 on a masked row.
template <typename T>
__device__ __forceinline__ float epi_value(const TapConv& op, int b, int t, int c, size_t idx,
                                           float acc) {
  if (op.len != nullptr && t >= op.len[b]) return 0.0f;
  float v = acc + op.bias[c];
  if (op.bias_bc != nullptr) v += op.bias_bc[(size_t)b * op.Cout + c];
  for (int r = 0; r < op.nres; ++r) v = ld_act<T>(op.res[r], idx) + v;
  if (op.div != 1.0f) v = v / op.div;
  return v;
}

template <typename T>
__device__ __forceinline__ void epi_store(const TapConv& op, size_t idx, float v) {
  if (op.out_raw != nullptr) st_act<T>(op.out_raw, idx, v);
  if (op.out_act != nullptr) st_act<T>(op.out_act, idx, lrelu(v, op.slope));
}

// Full per-element epilogue for GEMM element (q, n) of utterance b.
template <typename T>
__device__ __forceinline__ void epi_element(const TapConv& op, int b, int q, int n, float acc) {
  const long long e = (long long)q * op.N + n - op.crop;
  if (e < 0 || e >= (long long)op.Lout * op.Cout) return;
  const int t = (int)(e / op.Cout);
  const int c = (int)(e - (long long)t * op.Cout);
  const size_t idx = ((size_t)b * op.Lout + t) * op.Cout + c;
  epi_store<T>(op, idx, epi_value<T>(op, b, t, c, idx, acc));
}

// First output row touched by GEMM rows [q0, ...) of an op (for masked-tile skipping).
__host__ __device__ inline long long first_out_row(const TapConv& op, int q0) {
  long long e = (long long)q0 * op.N - op.crop;
  if (e < 0) e = 0;
  return e / op.Cout;
}

}  // namespace gsv
