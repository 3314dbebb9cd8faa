// Selection helpers shared by the portable router kernels (prefill and decode).
#pragma once

#include "hga_common.cuh"

namespace hga {

// ---- block / warp selection helpers ----------------------------------------------------------
// Select the k largest of keys[0..n) (ordered-float keys, 0 = absent) with ties resolved by lower
// index; sets flag[i] = 1 for the selected, 0 otherwise.  Whole block participates.
__device__ __forceinline__ void block_select(const uint32_t* keys, int n, int k, unsigned char* flag, int* sred) {
  const int tid = threadIdx.x;
  // count real
  int local = 0;
  for (int i = tid; i < n; i += blockDim.x) local += keys[i] != 0u;
  int nreal = __syncthreads_count(0);  // barrier only
  (void)nreal;
  if (tid == 0) sred[0] = 0;
  __syncthreads();
  atomicAdd(&sred[0], local);
  __syncthreads();
  nreal = sred[0];
  __syncthreads();
  if (nreal <= k) {
    for (int i = tid; i < n; i += blockDim.x) flag[i] = keys[i] != 0u;
    __syncthreads();
    return;
  }
  uint32_t T = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = T | (1u << bit);
    int cnt = 0;
    for (int i = tid; i < n; i += blockDim.x) cnt += keys[i] >= cand;
    if (tid == 0) sred[1] = 0;
    __syncthreads();
    atomicAdd(&sred[1], cnt);
    __syncthreads();
    if (sred[1] >= k) T = cand;
    __syncthreads();
  }
  // strictly greater ones
  int g = 0;
  for (int i = tid; i < n; i += blockDim.x) {
    flag[i] = keys[i] > T;
    g += keys[i] > T;
  }
  if (tid == 0) sred[2] = 0;
  __syncthreads();
  atomicAdd(&sred[2], g);
  __syncthreads();
  int need = k - sred[2];
  // fill ties in index order (warp 0 scans)
  if (tid < 32) {
    for (int base = 0; base < n && need > 0; base += 32) {
      const int i = base + tid;
      const bool eq = i < n && keys[i] == T;
      const unsigned bal = __ballot_sync(0xffffffffu, eq);
      const int before = __popc(bal & ((1u << tid) - 1u));
      if (eq && before < need) flag[i] = 1;
      need -= __popc(bal);
    }
  }
  __syncthreads();
}

// Warp-scoped version over a row of n <= 32*kMaxPerLane keys held in smem.
__device__ __forceinline__ void warp_select(const uint32_t* keys, int n, int k, unsigned char* flag) {
  const int lane = threadIdx.x & 31;
  int nreal = 0;
  for (int i = lane; i < n; i += 32) nreal += keys[i] != 0u;
  for (int o = 16; o; o >>= 1) nreal += __shfl_xor_sync(0xffffffffu, nreal, o);
  if (nreal <= k) {
    for (int i = lane; i < n; i += 32) flag[i] = keys[i] != 0u;
    __syncwarp();
    return;
  }
  uint32_t T = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = T | (1u << bit);
    int cnt = 0;
    for (int i = lane; i < n; i += 32) cnt += keys[i] >= cand;
    for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (cnt >= k) T = cand;
  }
  int g = 0;
  for (int i = lane; i < n; i += 32) {
    flag[i] = keys[i] > T;
    g += keys[i] > T;
  }
  for (int o = 16; o; o >>= 1) g += __shfl_xor_sync(0xffffffffu, g, o);
  int need = k - g;
  for (int base = 0; base < n && need > 0; base += 32) {
    const int i = base + lane;
    const bool eq = i < n && keys[i] == T;
    const unsigned bal = __ballot_sync(0xffffffffu, eq);
    const int before = __popc(bal & ((1u << lane) - 1u));
    if (eq && before < need) flag[i] = 1;
    need -= __popc(bal);
  }
  __syncwarp();
}

// Warp-wide top-k of keys[0..n), n <= 512 (ordered-float keys, 0 = absent), ties resolved by lower
// index — the same selection as warp_select.  Each lane sorts its 16 (key, index) pairs with a
// bitonic network, then k rounds of warp max-reductions pop the largest remaining pair from its
// owner lane: O(k) reductions instead of 32 radix passes over the keys.
__device__ __forceinline__ void cas_desc64(unsigned long long& a, unsigned long long& b) {
  const unsigned long long hi = a > b ? a : b, lo = a > b ? b : a;
  a = hi;
  b = lo;
}
__device__ __forceinline__ void warp_topk_small(const uint32_t* keys, int n, int k, unsigned char* flag) {
  const int lane = threadIdx.x & 31;
  unsigned long long v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int i = lane + 32 * m;
    const uint32_t key = i < n ? keys[i] : 0u;
    v[m] = key ? ((unsigned long long)key << 32) | (0xffffffffu - (uint32_t)i) : 0ull;
  }
#pragma unroll
  for (int size = 2; size <= 16; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          if ((i & size) == 0) cas_desc64(v[i], v[j]);
          else cas_desc64(v[j], v[i]);
        }
      }
  unsigned long long last = 0ull;
  for (int it = 0; it < k; ++it) {
    const uint32_t hi = __reduce_max_sync(0xffffffffu, (uint32_t)(v[0] >> 32));
    if (hi == 0u) break;
    const uint32_t lo = __reduce_max_sync(0xffffffffu, (uint32_t)(v[0] >> 32) == hi ? (uint32_t)v[0] : 0u);
    last = ((unsigned long long)hi << 32) | lo;
    if (v[0] == last) {  // the owner pops its head (pairs are unique)
#pragma unroll
      for (int m = 0; m < 15; ++m) v[m] = v[m + 1];
      v[15] = 0ull;
    }
  }
  for (int i = lane; i < n; i += 32) {
    const unsigned long long c = keys[i] ? ((unsigned long long)keys[i] << 32) | (0xffffffffu - (uint32_t)i) : 0ull;
    flag[i] = c != 0ull && c >= last;
  }
  __syncwarp();
}

// Insert key into a descending list of length k (list[k-1] is the current threshold).
__device__ __forceinline__ void list_insert(unsigned long long* list, int k, unsigned long long key) {
  if (key <= list[k - 1]) return;
  int j = k - 1;
  while (j > 0 && list[j - 1] < key) {
    list[j] = list[j - 1];
    --j;
  }
  list[j] = key;
}

}  // namespace hga
