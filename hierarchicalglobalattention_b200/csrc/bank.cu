// VRAM token bank of the RAM tier: a per-(sequence, KV head) cache in HBM of 16-token groups of the
// cold token record (pinned host memory), refilled by one gather launch per decode step.
//
// Counterpart of the reference's bounded LRU token bank (ExistingModelFineTuning/KvRouter/
// ram_kv_cache_store.py:266-317 _ensure_bank / _load_missing, gathers :547-607, KV-head union
// dedup gather_chunk_tokens_kvh :397-438), re-laid out for the decode kernels:
//   * granularity: one routing group (16 token rows of K and V) per slot, per (sequence, KV head),
//     instead of a whole chunk for the whole batch; the attention reads only opened groups, so a
//     group bank moves only what is attended;
//   * the groups the query heads of one KV head open are de-duplicated before any host read;
//   * the slot maps live in device memory (gid -> slot, slot -> gid, last-use stamp) and the
//     replacement policy is exact LRU by stamp, ties to the lower slot index;
//   * a miss is copied by the gather kernel itself, reading the pinned record over the host link
//     (16-byte loads, a warp per group, all of a lane's loads in flight before its stores).
// One CTA per (sequence, KV head).  It also rewrites the heads' open lists as bank slots, so the
// decode attention kernel reads opened groups from HBM unchanged (cold buffer = the bank).
#include "hga_common.cuh"

namespace hga {

constexpr int kBankThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kBankThreads) bank_gather_kernel(
    hga_params p, const int32_t* __restrict__ open_gid, int Kg, const T* rec_k, const T* rec_v, int64_t rec_cap,
    T* __restrict__ bank_k, T* __restrict__ bank_v, int n_slots, int32_t* __restrict__ slot_gid,
    int32_t* __restrict__ gid_slot, int64_t gid_cap, int32_t* __restrict__ slot_stamp, int stamp,
    int32_t* __restrict__ open_slot, unsigned long long* __restrict__ counters) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int bk = blockIdx.x;  // b * KVH + kvh
  const int H = p.nhead, KVH = p.kv_heads, rep = H / KVH, gs = p.group_size, Dh = p.head_dim;
  const int b = bk / KVH, kvh = bk % KVH;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwords = (int)((gid_cap + 31) / 32);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem);             // [nwords]
  int* uniq = reinterpret_cast<int*>(bitmap + nwords);               // [rep * Kg]
  int* miss = uniq + rep * Kg;                                       // [rep * Kg]
  int* victim = miss + rep * Kg;                                     // [rep * Kg]
  int* misc = victim + rep * Kg;                                     // [0] unique, [1] misses, [2] hits, [3..] scan
  int32_t* sg = slot_gid + (size_t)bk * n_slots;
  int32_t* gsl = gid_slot + (size_t)bk * gid_cap;
  int32_t* sst = slot_stamp + (size_t)bk * n_slots;

  for (int i = tid; i < nwords; i += kBankThreads) bitmap[i] = 0u;
  if (tid < 3) misc[tid] = 0;
  __syncthreads();
  // (1) the union of the KV head's query heads' opened groups
  const size_t lst0 = ((size_t)b * H + (size_t)kvh * rep) * Kg;
  for (int e = tid; e < rep * Kg; e += kBankThreads) {
    const int g = open_gid[lst0 + e];
    if (g >= 0 && g < gid_cap) atomicOr(&bitmap[g >> 5], 1u << (g & 31));
  }
  __syncthreads();
  // (2) compaction in ascending group order: warp 0 scans the bitmap word by word
  if (warp == 0) {
    int base = 0;
    for (int w0 = 0; w0 < nwords; w0 += 32) {
      const int w = w0 + lane;
      const uint32_t bits = w < nwords ? bitmap[w] : 0u;
      const int c = __popc(bits);
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      int pos = base + inc - c;
      uint32_t x = bits;
      while (x) {
        const int bit = __ffs(x) - 1;
        x &= x - 1;
        uniq[pos++] = (w << 5) + bit;
      }
      base += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) misc[0] = base;
  }
  __syncthreads();
  const int nu = misc[0];
  // (3) hits are stamped (so they cannot be evicted below); misses are listed in group order
  for (int i = tid; i < nu; i += kBankThreads) {
    const int g = uniq[i];
    const int s = gsl[g];
    if (s >= 0) sst[s] = stamp;
  }
  __syncthreads();
  if (warp == 0) {
    int base = 0;
    for (int i0 = 0; i0 < nu; i0 += 32) {
      const int i = i0 + lane;
      const bool m = i < nu && gsl[uniq[i]] < 0;
      const unsigned bal = __ballot_sync(0xffffffffu, m);
      if (m) miss[base + __popc(bal & ((1u << lane) - 1u))] = uniq[i];
      base += __popc(bal);
    }
    if (lane == 0) { misc[1] = base; misc[2] = nu - base; }
  }
  __syncthreads();
  const int nm = misc[1];
  if (nm > 0) {
    // (4) victims: the nm least recently used slots (stamp < T, then stamp == T by slot index),
    // never one stamped by this step; T found by bisection on the stamp counts
    int* cnt = misc + 3;
    int lo = -1, hi = stamp - 1;  // smallest T with count(stamp <= T) >= nm lies in [lo, hi]
    while (lo < hi) {
      const int mid = lo + ((hi - lo) >> 1);
      int c = 0;
      for (int s = tid; s < n_slots; s += kBankThreads) c += sst[s] <= mid;
      c = __reduce_add_sync(0xffffffffu, c);
      __syncthreads();
      if (tid == 0) cnt[0] = 0;
      __syncthreads();
      if (lane == 0) atomicAdd(cnt, c);
      __syncthreads();
      if (cnt[0] >= nm) hi = mid; else lo = mid + 1;
      __syncthreads();
    }
    const int t_lru = lo;  // the stamp threshold
    if (warp == 0) {
      int below = 0;  // slots with stamp < t_lru first (all of them are needed), then stamp == t_lru
      for (int pass = 0; pass < 2; ++pass) {
        for (int s0 = 0; s0 < n_slots && below < nm; s0 += 32) {
          const int s = s0 + lane;
          const bool take = s < n_slots && (pass == 0 ? sst[s] < t_lru : sst[s] == t_lru);
          const unsigned bal = __ballot_sync(0xffffffffu, take);
          const int r = below + __popc(bal & ((1u << lane) - 1u));
          if (take && r < nm) victim[r] = s;
          below += __popc(bal);
        }
      }
    }
    __syncthreads();
    // (5) map updates (one thread per miss), then the copies (one warp per miss)
    for (int i = tid; i < nm; i += kBankThreads) {
      const int s = victim[i], g = miss[i];
      const int old = sg[s];
      if (old >= 0 && old < gid_cap) gsl[old] = -1;
      sg[s] = g;
      gsl[g] = s;
      sst[s] = stamp;
    }
    const int pieces = gs * Dh * (int)sizeof(T) / 16;  // 16-byte pieces of one group's K (or V)
    const size_t rec_base = (size_t)bk * rec_cap * Dh;
    const size_t bank_base = (size_t)bk * n_slots * gs * Dh;
    for (int i = warp; i < nm; i += kBankThreads / 32) {
      const int g = miss[i], s = victim[i];
      if ((int64_t)(g + 1) * gs > rec_cap) continue;
      const uint4* sk = reinterpret_cast<const uint4*>(rec_k + rec_base + (size_t)g * gs * Dh);
      const uint4* sv = reinterpret_cast<const uint4*>(rec_v + rec_base + (size_t)g * gs * Dh);
      uint4* dk = reinterpret_cast<uint4*>(bank_k + bank_base + (size_t)s * gs * Dh);
      uint4* dv = reinterpret_cast<uint4*>(bank_v + bank_base + (size_t)s * gs * Dh);
      for (int c0 = 0; c0 < pieces; c0 += 32 * 8) {
        uint4 xk[8], xv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < pieces) { xk[u] = sk[c]; xv[u] = sv[c]; }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < pieces) { dk[c] = xk[u]; dv[c] = xv[u]; }
        }
      }
    }
  }
  __syncthreads();
  // (6) the heads' open lists as bank slots
  for (int e = tid; e < rep * Kg; e += kBankThreads) {
    const int g = open_gid[lst0 + e];
    open_slot[lst0 + e] = (g >= 0 && g < gid_cap) ? gsl[g] : -1;
  }
  if (tid == 0 && counters) {
    atomicAdd(&counters[0], (unsigned long long)misc[2]);
    atomicAdd(&counters[1], (unsigned long long)nm);
  }
}

size_t bank_gather_smem(const hga_params& p, int Kg, int64_t gid_cap) {
  const int rep = p.nhead / p.kv_heads;
  return (size_t)((gid_cap + 31) / 32) * 4 + (size_t)3 * rep * Kg * 4 + 64;
}

cudaError_t launch_bank_gather(const hga_params& p, const int32_t* open_gid, int Kg, const void* rec_k,
                               const void* rec_v, int64_t rec_cap, void* bank_k, void* bank_v, int n_slots,
                               int32_t* slot_gid, int32_t* gid_slot, int64_t gid_cap, int32_t* slot_stamp, int stamp,
                               int32_t* open_slot, unsigned long long* counters, cudaStream_t st) {
  const size_t smem = bank_gather_smem(p, Kg, gid_cap);
  if (smem > 200 * 1024) return cudaErrorInvalidConfiguration;
#define HGA_BG(TT)                                                                                           \
  {                                                                                                          \
    auto kern = bank_gather_kernel<TT>;                                                                      \
    if (smem > 48 * 1024) {                                                                                  \
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
      if (e != cudaSuccess) return e;                                                                        \
    }                                                                                                        \
    kern<<<p.batch * p.kv_heads, kBankThreads, smem, st>>>(p, open_gid, Kg, (const TT*)rec_k, (const TT*)rec_v, \
                                                           rec_cap, (TT*)bank_k, (TT*)bank_v, n_slots, slot_gid, \
                                                           gid_slot, gid_cap, slot_stamp, stamp, open_slot, counters); \
    return cudaGetLastError();                                                                               \
  }
  switch (p.dtype) {
    case HGA_DTYPE_F32: HGA_BG(float)
    case HGA_DTYPE_BF16: HGA_BG(__nv_bfloat16)
    case HGA_DTYPE_F16: HGA_BG(__half)
  }
#undef HGA_BG
  return cudaErrorInvalidValue;
}

}  // namespace hga
