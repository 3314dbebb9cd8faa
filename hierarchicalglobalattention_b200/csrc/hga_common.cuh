// Shared device/host helpers for the HGA B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/hga_b200.h"

namespace hga {

// Finite mask fill of the reference (ExistingModelFineTuning/KvRouter/vectorized.py:38).
constexpr float kNeg = -1.0e4f;

template <typename T> struct Num;
template <> struct Num<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
  // value after a store in this dtype (identity for fp32)
  static __device__ __forceinline__ float round(float x) { return x; }
};
template <> struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <> struct Num<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
};

// Score exactly as the reference forms it: einsum output in the input dtype, then "* scale"
// evaluated in fp32 and stored in the input dtype (vectorized.py:307, 369).
template <typename T>
__device__ __forceinline__ float ref_score(float dot, float scale) {
  return Num<T>::round(__fmul_rn(Num<T>::round(dot), scale));
}

// Order-preserving map float -> uint32 (larger float => larger key).
__device__ __forceinline__ uint32_t ord_f32(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unord_f32(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}
// Ranking key: higher score first, then lower index first.
__device__ __forceinline__ unsigned long long rank_key(float s, uint32_t idx) {
  return ((unsigned long long)ord_f32(s) << 32) | (unsigned long long)(0xffffffffu - idx);
}
__device__ __forceinline__ uint32_t rank_idx(unsigned long long k) {
  return 0xffffffffu - (uint32_t)(k & 0xffffffffull);
}
__device__ __forceinline__ float rank_score(unsigned long long k) { return unord_f32((uint32_t)(k >> 32)); }

// The query chunks one prefill launch processes: chunks [chunk0, chunk0 + count) of a sequence of
// S tokens.  q and the per-chunk outputs hold only those chunks (rows, tiles) — sq query rows per
// batch entry, local chunk i = chunk chunk0 + i — while keys, summaries and all routing rules use
// the absolute chunk index.  A whole-sequence launch is {0, N, S}.
struct QRange {
  int chunk0;
  int count;
  int64_t sq;
};

// Windows of query chunk n (vectorized.py:242-253; chunk_placement_policy.py:27-38).
__host__ __device__ __forceinline__ void windows(int n, int keep_first, int keep_last, int& f_hi, int& l_lo) {
  int kf = keep_first > 0 ? keep_first : 0;
  int kl = keep_last > 0 ? keep_last : 0;
  f_hi = kf > 0 ? (n < kf ? n : kf) : 0;
  if (kl > 0) {
    int a = n - kl;
    if (a < kf) a = kf;
    l_lo = a < n ? a : n;
  } else {
    l_lo = n;
  }
}

// Device error word of one translation unit's kernels (a file-scope variable, so each .cu file
// that uses the macro gets its own word) and its host-side reader: 0, or the first error code.
#define HGA_DEVICE_ERROR_WORD(word, reader)                              \
  static __device__ int word = 0;                                        \
  int reader(bool clear) {                                               \
    int v = 0;                                                           \
    if (cudaMemcpyFromSymbol(&v, word, sizeof(int)) != cudaSuccess)      \
      return -1;                                                         \
    if (clear && v) {                                                    \
      int z = 0;                                                         \
      cudaMemcpyToSymbol(word, &z, sizeof(int));                         \
    }                                                                    \
    return v;                                                            \
  }

// Codes of the decode kernels' bounds checks: a position or list entry whose rows lie past a
// buffer's capacity.  The kernel skips those rows (its output for the (b, h) is then zero).
constexpr int kErrBoundsRouteDecode = 0x101;
constexpr int kErrBoundsAttendDecode = 0x102;
constexpr int kErrBoundsAppend = 0x103;

}  // namespace hga
