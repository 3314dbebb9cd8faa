// Two-level prefill router on the tensor cores (bf16, head_dim 128, chunk 64, group 16).
//
// Same selection rules, tie order and outputs as the portable router (route_prefill.cu, which
// states the reference lines it follows); the scoring contractions run on tcgen05 and the
// per-row selections run one thread per query row on TMEM-resident scores:
//   CTA = (query chunk n, pair of query heads sharing a KV head, batch b); M = 128 rows.
//   level 1: the routed pool [f_hi, l_lo) streams through smem in 128-chunk tiles (TMA);
//            S = Q.CK^T lands in TMEM (double-buffered); each row thread keeps its running
//            top-Kc requests in registers (16-bit score key | 16-bit pool index) and finally
//            max-pools them into smem (atomicMax) with the first requesting row (atomicMin).
//   select : one warp per head picks Kc pooled chunks (radix select), forces the previous chunk.
//   level 2: the chosen chunks' group summaries (<= 128 rows per head) are gathered into a
//            256-row SW128 tile; one N=256 MMA scores both heads; each row thread selects its
//            Kg_request groups by a 16-bit radix select; one warp per head picks Kg pooled groups.
#include "tc_common.cuh"

namespace hga {
namespace rtc {

using namespace tc;

struct Args {
  int S, H, KVH, N, Kc, Kg, Kgr, keep_first, keep_last, q_layout;
  int chunk0, nl, sq;  // query chunks [chunk0, chunk0 + nl); q and the lists hold only those
  int NP;  // per-head length of the pooled / t0 / flag arrays: max(N, Kc * M) (reused by level 2)
  int64_t sum_cap;
  float scale;
  const __nv_bfloat16* group_k;
  int32_t *sel_chunk, *sel_t0, *open_gid, *open_t0;
  float *dbg_l1, *dbg_l2;
};

__device__ __forceinline__ uint32_t ord16(float s) {  // order-preserving key of a bf16 value, 0 reserved
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(s));
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}

// Round-to-nearest-even of a finite fp32 value to bf16 precision, on its bit pattern (the
// definition of IEEE rounding at 8 mantissa bits; scores are never NaN).  Integer ops only: the
// scoring loop runs it twice per score, and conversion instructions were the loop's bottleneck.
__device__ __forceinline__ uint32_t round_bf16_bits(uint32_t b) {
  return (b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u;
}
// bits of T(T(acc) * scale): the reference's rounding points for a score (bf16 einsum output,
// then "* scale" evaluated in fp32 and stored in bf16)
__device__ __forceinline__ uint32_t bf16_score_bits(uint32_t acc_bits, float scale) {
  return round_bf16_bits(__float_as_uint(__fmul_rn(__uint_as_float(round_bf16_bits(acc_bits)), scale)));
}
// ord16 of a value already rounded to bf16 (its high 16 bits)
__device__ __forceinline__ uint32_t ord16_bits(uint32_t rounded) {
  const uint32_t b = rounded >> 16;
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}

// two fp32 values rounded to bf16 (round-to-nearest-even) in one word: lo in bits 0-15
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// (lo, hi) * scale, one paired fp32 multiply (round-to-nearest, like two scalar multiplies)
__device__ __forceinline__ void mul2_scale(float lo, float hi, float scale, float& o0, float& o1) {
  uint64_t x, sc, y;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(lo), "f"(hi));
  asm("mov.b64 %0, {%1, %1};" : "=l"(sc) : "f"(scale));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(y) : "l"(x), "l"(sc));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o0), "=f"(o1) : "l"(y));
}

__device__ __forceinline__ float bf16_score(uint32_t acc_bits, float scale) {
  return Num<__nv_bfloat16>::round(__fmul_rn(Num<__nv_bfloat16>::round(__uint_as_float(acc_bits)), scale));
}

// Smem layout (bytes from the 1024-aligned base).  pooled/t0 arrays are sized by N at launch.
struct L {
  static constexpr int kQ = 0, kTile = 32768, kTileBytes = 65536;  // 2 x 32 KB stages, reused as the L2 tile
  static constexpr int kFixed = kTile + kTileBytes;
};
struct Misc {
  uint64_t bars[10];
  uint32_t tmem;
  int abort;
  int ksel[2];
  int sel[2][32];
  int selt0[2][32];
  uint32_t gpool[2][128];
  uint32_t gt0[2][128];
};

// ---- sorting networks on register arrays (descending; fully unrolled, no serial chains) -----
__device__ __forceinline__ void cas_desc(uint32_t& a, uint32_t& b) {
  const uint32_t hi = max(a, b), lo = min(a, b);
  a = hi;
  b = lo;
}
// bitonic sort of v[0..N) into descending order (N a power of two)
template <int N>
__device__ __forceinline__ void sort_desc(uint32_t* v) {
#pragma unroll
  for (int size = 2; size <= N; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          if ((i & size) == 0) cas_desc(v[i], v[j]);
          else cas_desc(v[j], v[i]);
        }
      }
}
// a bitonic v[0..N) into descending order
template <int N>
__device__ __forceinline__ void clean_desc(uint32_t* v) {
#pragma unroll
  for (int stride = N >> 1; stride > 0; stride >>= 1)
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const int j = i ^ stride;
      if (j > i) cas_desc(v[i], v[j]);
    }
}
// lst (descending, KL) := the KL largest of lst and the 32 keys in b (b is clobbered)
template <int KL>
__device__ __forceinline__ void merge_batch(uint32_t* lst, uint32_t* b) {
  if constexpr (KL == 16) {
    sort_desc<16>(b);
    sort_desc<16>(b + 16);
#pragma unroll
    for (int i = 0; i < 16; ++i) b[i] = max(b[i], b[31 - i]);  // top 16 of the batch, bitonic
    clean_desc<16>(b);
#pragma unroll
    for (int i = 0; i < 16; ++i) lst[i] = max(lst[i], b[15 - i]);
    clean_desc<16>(lst);
  } else {
    sort_desc<32>(b);
#pragma unroll
    for (int i = 0; i < 32; ++i) lst[i] = max(lst[i], b[31 - i]);
    clean_desc<32>(lst);
  }
}

// Warp-wide top-k for n <= 512 unique 32-bit keys: every lane sorts its 16 keys (a sorting network),
// then k rounds of one warp max-reduction pop the largest remaining key from its owner lane.  Flags
// the k largest and returns the smallest flagged key (0 if fewer than k keys are non-zero: then
// every non-zero key is flagged).
__device__ uint32_t warp_topk_small(const uint32_t* keys, int n, int k, unsigned char* flag) {
  const int lane = threadIdx.x & 31;
  uint32_t v[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) v[m] = (lane + 32 * m < n) ? keys[lane + 32 * m] : 0u;
  sort_desc<16>(v);
  for (int i = lane; i < n; i += 32) flag[i] = 0;
  __syncwarp();
  uint32_t last = 0u;
  for (int it = 0; it < k; ++it) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, v[0]);
    if (best == 0u) break;
    last = best;
    if (v[0] == best) {  // the owner pops its head (keys are unique: exactly one lane)
#pragma unroll
      for (int m = 0; m < 15; ++m) v[m] = v[m + 1];
      v[15] = 0u;
    }
  }
  __syncwarp();
  for (int i = lane; i < n; i += 32) flag[i] = keys[i] != 0u && keys[i] >= last;
  __syncwarp();
  return last;
}

// Chunk choice of one head for pools of at most 512 chunks, all in registers: lane l holds the
// pooled keys of chunks l + 32m (score << 16 | 0xffff - c, 0 = not requested), the k largest are
// chosen by k rounds of warp max-reductions over per-lane sorted copies, then chunk `pr` (the
// previous chunk, -1 if outside the pool) is forced in, replacing the lowest-ranked choice when k
// are chosen.  Returns the lane's chosen chunks as a bit mask over m.
__device__ uint32_t warp_choose_small(const uint32_t* pooled, int npool, int k, int pr) {
  const int lane = threadIdx.x & 31;
  uint32_t v[16], w[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int c = lane + 32 * m;
    const uint32_t raw = c < npool ? pooled[c] : 0u;
    v[m] = raw ? ((raw << 16) | (0xffffu - (uint32_t)c)) : 0u;
    w[m] = v[m];
  }
  sort_desc<16>(w);
  uint32_t last = 0u;
  for (int it = 0; it < k; ++it) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, w[0]);
    if (best == 0u) break;
    last = best;
    if (w[0] == best) {  // keys are unique: exactly one lane pops
#pragma unroll
      for (int m = 0; m < 15; ++m) w[m] = w[m + 1];
      w[15] = 0u;
    }
  }
  uint32_t mask = 0u;
#pragma unroll
  for (int m = 0; m < 16; ++m) mask |= (v[m] != 0u && v[m] >= last ? 1u : 0u) << m;
  if (pr >= 0) {
    const bool mine = (pr & 31) == lane;
    const bool pr_sel = __shfl_sync(0xffffffffu, (mask >> (pr >> 5)) & 1u, pr & 31) != 0u;
    if (!pr_sel) {
      const int nsel = __reduce_add_sync(0xffffffffu, __popc(mask));
      if (nsel >= k) {  // drop the lowest-ranked choice: the k-th key, `last`
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (v[m] == last) mask &= ~(1u << m);
      }
      if (mine) mask |= 1u << (pr >> 5);
    }
  }
  return mask;
}

// Warp-wide radix select over keys[0..n) (unique 32-bit keys, 0 = absent): flags the k largest.
// Keys are cached in registers (up to 64 per lane, n <= 2048); larger n streams from smem.
__device__ void warp_select_u32(const uint32_t* keys, int n, int k, unsigned char* flag) {
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
  if (n <= 32 * 64) {
    uint32_t kr[64];
#pragma unroll
    for (int m = 0; m < 64; ++m) kr[m] = (lane + 32 * m < n) ? keys[lane + 32 * m] : 0u;
    const int mmax = (n + 31) / 32;
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t cand = T | (1u << bit);
      int c4[4] = {0, 0, 0, 0};  // four partial counts: short dependence chains
#pragma unroll
      for (int m = 0; m < 64; ++m)
        if (m < mmax) c4[m & 3] += kr[m] >= cand;
      const int cnt = __reduce_add_sync(0xffffffffu, c4[0] + c4[1] + c4[2] + c4[3]);
      if (cnt >= k) T = cand;
    }
  } else {
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t cand = T | (1u << bit);
      int cnt = 0;
      for (int i = lane; i < n; i += 32) cnt += keys[i] >= cand;
      cnt = __reduce_add_sync(0xffffffffu, cnt);
      if (cnt >= k) T = cand;
    }
  }
  for (int i = lane; i < n; i += 32) flag[i] = keys[i] >= T;  // keys are unique: exactly k
  __syncwarp();
}

// Threads per CTA: TMA warp, MMA warp, then the row warps.  With KL = 16 two row warps share each
// TMEM lane quarter (each scores half of every 128-chunk tile; the lists merge at the end), which
// doubles the row warps per SM of the latency-bound scoring loop; KL = 32 lists leave room for one.
template <int KL>
__host__ __device__ constexpr int threads_for() { return KL <= 16 ? 320 : 192; }

template <int KL>
__global__ void __launch_bounds__(threads_for<KL>(), 2)
    route_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_ck, const Args a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int ln = blockIdx.x, hp = blockIdx.y, b = blockIdx.z;
  const int n = a.chunk0 + ln;
  const int h0 = 2 * hp;
  const int kvh = h0 / (a.H / a.KVH);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int C = 64, M = 4;
  constexpr int NT = threads_for<KL>(), kRowWarps = NT / 32 - 2, kHalves = kRowWarps / 4;
  const int row0 = n * C;
  const int nvalid = (a.S - row0) < C ? (a.S - row0) : C;
  const int N = a.N, NP = a.NP;
  uint32_t* pooled = reinterpret_cast<uint32_t*>(smem + L::kFixed);      // [2][NP]
  uint32_t* t0c = pooled + 2 * NP;                                        // [2][NP]
  unsigned char* flags = reinterpret_cast<unsigned char*>(t0c + 2 * NP);  // [2][NP]
  Misc* ms = reinterpret_cast<Misc*>(flags + ((2 * NP + 15) & ~15));
  volatile int* abort_flag = &ms->abort;
  uint64_t* q_full = ms->bars + 0;
  uint64_t* ck_full = ms->bars + 1;   // [2]
  uint64_t* ck_empty = ms->bars + 3;  // [2]
  uint64_t* s_full = ms->bars + 5;    // [2]
  uint64_t* s_free = ms->bars + 7;    // [2]
  uint64_t* s2_full = ms->bars + 9;

  int f_hi, l_lo;
  windows(n, a.keep_first, a.keep_last, f_hi, l_lo);
  const int pool_lo = f_hi, npool = l_lo > f_hi ? l_lo - f_hi : 0;
  const size_t out0 = (((size_t)b * a.H + h0) * a.nl + ln);
  const size_t out1 = out0 + a.nl;  // head h0+1
  for (int i = tid; i < 2 * a.Kc; i += NT) {
    const size_t o = (i < a.Kc ? out0 : out1) * a.Kc + (i % a.Kc);
    a.sel_chunk[o] = -1;
    a.sel_t0[o] = -1;
  }
  for (int i = tid; i < 2 * a.Kg; i += NT) {
    const size_t o = (i < a.Kg ? out0 : out1) * a.Kg + (i % a.Kg);
    a.open_gid[o] = -1;
    a.open_t0[o] = -1;
  }
  if (a.Kc == 0 || npool == 0) return;
  const int ntile = (npool + 127) / 128;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(ck_full + i, 1);
      mbar_init(ck_empty + i, 1);
      mbar_init(s_full + i, 1);
      mbar_init(s_free + i, 32 * kRowWarps);
    }
    mbar_init(s2_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    ms->abort = 0;
  }
  for (int i = tid; i < 2 * npool; i += NT) {
    pooled[(i / npool) * NP + i % npool] = 0u;
    t0c[(i / npool) * NP + i % npool] = 0xffffffffu;
  }
  for (int i = tid; i < 2 * 128; i += NT) {
    ms->gpool[i / 128][i % 128] = 0u;
    ms->gt0[i / 128][i % 128] = 0xffffffffu;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&ms->tmem)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = ms->tmem;
  unsigned char* q_s = smem + L::kQ;
  unsigned char* tile_s = smem + L::kTile;

  // ================================ level 1 ===================================================
  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, 32768);
      for (int hh = 0; hh < 2; ++hh)
        for (int kb = 0; kb < 2; ++kb) {
          unsigned char* dst = q_s + kb * 16384 + hh * 8192;
          if (a.q_layout == 1) tma_load_3d(dst, &tm_q, kb * 64, h0 + hh, b * a.sq + ln * C, q_full);
          else tma_load_2d(dst, &tm_q, kb * 64, (b * a.H + h0 + hh) * a.sq + ln * C, q_full);
        }
      const int64_t ckrow = ((int64_t)b * a.KVH + kvh) * a.sum_cap + pool_lo;
      for (int i = 0; i < ntile; ++i) {
        const int st = i & 1;
        if (i >= 2 && !mbar_wait(ck_empty + st, ((i >> 1) - 1) & 1, abort_flag, 11)) break;
        mbar_expect_tx(ck_full + st, 32768);
        for (int kb = 0; kb < 2; ++kb)
          tma_load_2d(tile_s + st * 32768 + kb * 16384, &tm_ck, kb * 64, (int)(ckrow + 128 * i), ck_full + st);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(false);
      const uint32_t q_addr = smem_u32(q_s);
      bool ok = mbar_wait(q_full, 0, abort_flag, 12);
      for (int i = 0; ok && i < ntile; ++i) {
        const int st = i & 1;
        if (!mbar_wait(ck_full + st, (i >> 1) & 1, abort_flag, 13)) break;
        if (i >= 2 && !mbar_wait(s_free + st, ((i >> 1) - 1) & 1, abort_flag, 14)) break;
        fence_after();
        const uint32_t k_addr = smem_u32(tile_s + st * 32768);
        for (int kb = 0; kb < 2; ++kb)
          for (int kk = 0; kk < 4; ++kk)
            mma_ss(tmem + st * 128, sdesc(q_addr + kb * 16384 + kk * 32, 16, 1024),
                   sdesc(k_addr + kb * 16384 + kk * 32, 16, 1024), idesc, (kb | kk) != 0);
        mma_commit(s_full + st);
        mma_commit(ck_empty + st);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // which share of every tile's columns this warp scores
    const int row = quarter * 32 + lane;
    const int hs = row >> 6, t = row & 63;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const bool rvalid = t < nvalid;
    uint32_t lst[KL];  // running top-KL request keys of this row, descending
#pragma unroll
    for (int j = 0; j < KL; ++j) lst[j] = 0u;
    const size_t dbg_row = ((hs ? out1 : out0) * C + t) * (size_t)N + pool_lo;
    for (int i = 0; i < ntile; ++i) {
      const int st = i & 1;
      // tcgen05.ld is warp-collective: keep the branch around it warp-uniform
      if (!__all_sync(0xffffffffu, mbar_wait(s_full + st, (i >> 1) & 1, abort_flag, 15))) break;
      fence_after();
      const uint32_t sa = tmem + lane_addr + st * 128;
      const int cmax = (npool - 128 * i) < 128 ? (npool - 128 * i) : 128;
      for (int c4 = half * (4 / kHalves); c4 < (half + 1) * (4 / kHalves); ++c4) {
        uint32_t r[32];
        HGA_LD32(sa + 32 * c4, r);
        tmem_wait_ld();
        // keys of the 32 columns, two at a time: both reference roundings (bf16 einsum output, then
        // "* scale" in fp32 stored as bf16) as paired conversions and a paired multiply, then the
        // order-preserving 16-bit key of each half (sign set: all bits flipped; else the sign
        // bit set), then the pool index below it (equal scores: the lower index ranks higher)
        const uint32_t thr = lst[KL - 1];
        const int nv = rvalid ? min(32, cmax - 32 * c4) : 0;  // valid columns of this batch
        const uint32_t cbase = 0xffffu - (uint32_t)(128 * i + 32 * c4);
        bool above = false;
#pragma unroll
        for (int cc = 0; cc < 32; cc += 2) {
          const uint32_t w = cvt_bf16x2(__uint_as_float(r[cc]), __uint_as_float(r[cc + 1]));
          float s0, s1;
          mul2_scale(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u), a.scale, s0, s1);
          const uint32_t w2 = cvt_bf16x2(s0, s1);
          const uint32_t o = w2 ^ (((w2 >> 15) & 0x00010001u) * 0x7fffu + 0x80008000u);
          const uint32_t k0 = cc < nv ? ((o << 16) | (cbase - cc)) : 0u;
          const uint32_t k1 = cc + 1 < nv ? ((o & 0xffff0000u) | (cbase - cc - 1)) : 0u;
          if (a.dbg_l1) {
            const size_t cr = dbg_row + 128 * i + 32 * c4 + cc;
            if (cc < nv) a.dbg_l1[cr] = __uint_as_float(w2 << 16);
            if (cc + 1 < nv) a.dbg_l1[cr + 1] = __uint_as_float(w2 & 0xffff0000u);
          }
          r[cc] = k0;
          r[cc + 1] = k1;
          above |= (k0 > thr) | (k1 > thr);
        }
        // the batch's keys join the row's list through sorting networks (no per-key insertion);
        // skipped when no row of the warp has a key above its current threshold
        if (__any_sync(0xffffffffu, above)) merge_batch<KL>(lst, r);
      }
      fence_before();
      mbar_arrive(s_free + st);
    }
    if (kHalves == 2) {
      // the second half's lists join the first half's (staged in the consumed tile stages)
      uint32_t* mbuf = reinterpret_cast<uint32_t*>(tile_s);
      if (half == 1) {
#pragma unroll
        for (int j = 0; j < KL; ++j) mbuf[j * 128 + row] = lst[j];
      }
      asm volatile("bar.sync 1, %0;" ::"r"(32 * kRowWarps) : "memory");
      if (half == 0) {
        // both lists are sorted descending: the top KL of their union is the bitonic max of one
        // against the other reversed, sorted by one clean
#pragma unroll
        for (int j = 0; j < KL; ++j) lst[j] = max(lst[j], mbuf[(KL - 1 - j) * 128 + row]);
        clean_desc<KL>(lst);
      }
    }
    // requests = top k1 of the row's list -> pooled max score and first requesting row per chunk
    const int k1 = a.Kc < npool ? a.Kc : npool;
    if (rvalid && half == 0) {
#pragma unroll
      for (int j = 0; j < KL; ++j) {
        if (j < k1 && lst[j] != 0u) {
          const int c = 0xffff - (int)(lst[j] & 0xffffu);
          atomicMax(&pooled[hs * NP + c], lst[j] >> 16);
          atomicMin(&t0c[hs * NP + c], (uint32_t)t);
        }
      }
    }
  }
  __syncthreads();

  // ================================ chunk choice (one warp per head) ==========================
  if (warp == 2 || warp == 3) {
    const int hs = warp - 2;
    uint32_t* keys = pooled + hs * NP;
    unsigned char* fl = flags + hs * NP;
    const int prev = n - 1;
    const bool prev_in = n > 0 && prev >= pool_lo && prev < l_lo;
    if (npool <= 512) {
      // registers only: choose, force the previous chunk, write the chosen list in chunk order
      const uint32_t mask = warp_choose_small(keys, npool, a.Kc, prev_in ? prev - pool_lo : -1);
      int k = 0;
      const size_t o = (hs ? out1 : out0) * a.Kc;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const int c = lane + 32 * m;
        const bool s = (mask >> m) & 1u;
        const unsigned bal = __ballot_sync(0xffffffffu, s);
        if (s) {
          const int slot = k + __popc(bal & ((1u << lane) - 1u));
          const int t0 = (prev_in && c == prev - pool_lo) ? 0 : (int)t0c[hs * NP + c];
          ms->sel[hs][slot] = pool_lo + c;
          ms->selt0[hs][slot] = t0;
          a.sel_chunk[o + slot] = pool_lo + c;
          a.sel_t0[o + slot] = t0;
        }
        k += __popc(bal);
      }
      if (lane == 0) ms->ksel[hs] = k;
    } else {
    for (int c = lane; c < npool; c += 32) keys[c] = keys[c] ? ((keys[c] << 16) | (0xffffu - c)) : 0u;
    __syncwarp();
    warp_select_u32(keys, npool, a.Kc, fl);
    if (prev_in) {
      const int pr = prev - pool_lo;
      int nsel = 0;
      for (int c = lane; c < npool; c += 32) nsel += fl[c];
      for (int o = 16; o; o >>= 1) nsel += __shfl_xor_sync(0xffffffffu, nsel, o);
      if (!fl[pr]) {
        if (nsel >= a.Kc) {  // drop the lowest-ranked chosen chunk (lowest score, then highest index)
          uint32_t mn = 0xffffffffu;
          for (int c = lane; c < npool; c += 32)
            if (fl[c]) mn = min(mn, keys[c]);
          for (int o = 16; o; o >>= 1) mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
          for (int c = lane; c < npool; c += 32)
            if (fl[c] && keys[c] == mn) fl[c] = 0;
        }
        __syncwarp();
        if (lane == 0) fl[pr] = 1;
      }
      __syncwarp();
      if (lane == 0) t0c[hs * NP + pr] = 0;
      __syncwarp();
    }
    int k = 0;
    const size_t o = (hs ? out1 : out0) * a.Kc;
    for (int base = 0; base < npool; base += 32) {
      const int c = base + lane;
      const bool s = c < npool && fl[c];
      const unsigned bal = __ballot_sync(0xffffffffu, s);
      if (s) {
        const int slot = k + __popc(bal & ((1u << lane) - 1u));
        const int t0 = (int)t0c[hs * NP + c];
        ms->sel[hs][slot] = pool_lo + c;
        ms->selt0[hs][slot] = t0;
        a.sel_chunk[o + slot] = pool_lo + c;
        a.sel_t0[o + slot] = t0;
      }
      k += __popc(bal);
    }
    if (lane == 0) ms->ksel[hs] = k;
    }
  }
  __syncthreads();
  const bool do_l2 = a.Kg > 0 && a.Kgr > 0 && !ms->abort;

  // ================================ level 2 ===================================================
  if (do_l2) {
    // gather the chosen chunks' group summaries: head hs -> rows [hs*128, hs*128 + 4*ksel)
    const __nv_bfloat16* gk = a.group_k + ((size_t)b * a.KVH + kvh) * a.sum_cap * M * 128;
    // every thread issues its 16-byte loads in two batches before storing, so the gather costs
    // two memory round trips instead of one per piece
    constexpr int kPieces = 256 * 16, kBatch = (kPieces / NT + 2) / 2;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint4 vals[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int pc = tid + (half * kBatch + k) * NT;
        vals[k] = make_uint4(0, 0, 0, 0);
        if (pc < kPieces) {
          const int rrow = pc >> 4, c16 = pc & 15;
          const int hs = rrow >> 7, j = rrow & 127;
          if (j < 4 * ms->ksel[hs]) {
            const int chunk = ms->sel[hs][j >> 2];
            vals[k] = __ldg(reinterpret_cast<const uint4*>(gk + ((size_t)chunk * M + (j & 3)) * 128 + c16 * 8));
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int pc = tid + (half * kBatch + k) * NT;
        if (pc < kPieces) {
          const int rrow = pc >> 4, c16 = pc & 15;
          const int kb = c16 >> 3, cc = c16 & 7;
          *reinterpret_cast<uint4*>(tile_s + kb * 32768 + rrow * 128 + ((cc ^ (rrow & 7)) << 4)) = vals[k];
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    fence_before();
    __syncthreads();
    fence_after();
    if (warp == 1 && lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);
      const uint32_t q_addr = smem_u32(q_s), g_addr = smem_u32(tile_s);
      for (int kb = 0; kb < 2; ++kb)
        for (int kk = 0; kk < 4; ++kk)
          mma_ss(tmem, sdesc(q_addr + kb * 16384 + kk * 32, 16, 1024), sdesc(g_addr + kb * 32768 + kk * 32, 16, 1024),
                 idesc, (kb | kk) != 0);
      mma_commit(s2_full);
    }
    // With eight row warps and at most 32 requests per row, two threads score a row: warps w and
    // w + 4 take its candidates [0, 32) and [32, 64), each sorts its 32 keys, and the first thread
    // of the row merges the partner's sorted keys (passed through the freed level-2 tile) into the
    // row's top-32 set.
    constexpr int KT = 4 * KL;  // candidate columns per head (Kc * M <= 4 * KL)
    constexpr int KTP = KT + 8;
    uint16_t* pm = reinterpret_cast<uint16_t*>(q_s);  // pooling matrix [2][64][KTP], see below
    const bool split = kRowWarps == 8 && KT == 64 && (a.Kgr <= 32 || a.Kgr >= a.Kc * M);
    if (split && warp >= 2) {
      const int quarter = warp & 3, part = (warp - 2) >> 2;
      const int row = quarter * 32 + lane;
      const int hs = row >> 6, t = row & 63;
      const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
      const int th = 4 * ms->ksel[hs];
      const bool ok = __all_sync(0xffffffffu, mbar_wait(s2_full, 0, abort_flag, 16));
      fence_after();
      uint32_t r[32];
      if (ok) {
        HGA_LD32(tmem + lane_addr + hs * 128 + part * 32, r);
        tmem_wait_ld();
      }
      const bool rvalid = ok && t < nvalid;
      const size_t dbg_row = ((hs ? out1 : out0) * C + t) * (size_t)(a.Kc * M);
      int nreal = 0;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int j = part * 32 + jj;
        uint32_t key = 0u;
        if (rvalid && j < th) {
          if (t >= ms->selt0[hs][j >> 2]) {
            const uint32_t sb = bf16_score_bits(r[jj], a.scale);
            key = ord16_bits(sb);
            if (a.dbg_l2) a.dbg_l2[dbg_row + j] = __uint_as_float(sb);
          } else if (a.dbg_l2) {
            a.dbg_l2[dbg_row + j] = kNeg;
          }
        }
        r[jj] = key ? ((key << 16) | (0xffffu - j)) : 0u;  // unique: equal scores -> lower j first
        nreal += key != 0u;
      }
      sort_desc<32>(r);
      uint32_t* xk = reinterpret_cast<uint32_t*>(tile_s);  // [128 rows][33]: the second part's keys, count
      if (part == 1) {
#pragma unroll
        for (int i = 0; i < 32; ++i) xk[row * 33 + i] = r[i];
        xk[row * 33 + 32] = (uint32_t)nreal;
      }
      asm volatile("bar.sync 3, 256;" ::: "memory");
      if (part == 0) {
        nreal += (int)xk[row * 33 + 32];
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = max(r[i], xk[row * 33 + 31 - i]);  // the top-32 set
        const bool active = rvalid && nreal > 0;
        // every requested key is in the top-32 set: all non-zero keys when at most Kgr are
        // valid (or Kgr covers every candidate), else the Kgr highest
        const bool all = a.Kgr >= a.Kc * M || nreal <= a.Kgr;
        if (active && !all && a.Kgr < 32) clean_desc<32>(r);
        uint4* prow = reinterpret_cast<uint4*>(pm + (size_t)(hs * 64 + t) * KTP);
#pragma unroll
        for (int c = 0; c < KT / 8; ++c) prow[c] = make_uint4(0, 0, 0, 0);
        if (active) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (r[i] && (all || i < a.Kgr)) pm[(size_t)(hs * 64 + t) * KTP + (0xffff - (int)(r[i] & 0xffffu))] =
                (uint16_t)(r[i] >> 16);
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        for (int i = row; i < 2 * KT; i += 128) {
          const int hh = i / KT, j = i % KT;
          const uint16_t* src = pm + (size_t)hh * 64 * KTP + j;  // column j: consecutive lanes, consecutive j
          uint32_t mx = 0u, first = 0xffffffffu;
#pragma unroll 16
          for (int t2 = 63; t2 >= 0; --t2) {
            const uint32_t v = src[(size_t)t2 * KTP];
            mx = max(mx, v);
            first = v ? (uint32_t)t2 : first;
          }
          ms->gpool[hh][j] = mx;
          ms->gt0[hh][j] = mx ? first : 0xffffffffu;
        }
      }
    } else if (!split && warp >= 2 && warp < 6) {
      const int quarter = warp & 3;
      const int row = quarter * 32 + lane;
      const int hs = row >> 6, t = row & 63;
      const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
      const int th = 4 * ms->ksel[hs];
      const bool ok = __all_sync(0xffffffffu, mbar_wait(s2_full, 0, abort_flag, 16));
      fence_after();
      uint32_t r[KT];
      if (ok) {
        const uint32_t sa = tmem + lane_addr + hs * 128;
#pragma unroll
        for (int c0 = 0; c0 < KT; c0 += 32) HGA_LD32(sa + c0, (r + c0));
        tmem_wait_ld();
      }
      const bool rvalid = ok && t < nvalid;
      const size_t dbg_row = ((hs ? out1 : out0) * C + t) * (size_t)(a.Kc * M);
      int nreal = 0;
#pragma unroll
      for (int j = 0; j < KT; ++j) {
        uint32_t key = 0u;
        if (rvalid && j < th) {
          if (t >= ms->selt0[hs][j >> 2]) {
            const uint32_t sb = bf16_score_bits(r[j], a.scale);
            key = ord16_bits(sb);
            if (a.dbg_l2) a.dbg_l2[dbg_row + j] = __uint_as_float(sb);
          } else if (a.dbg_l2) {
            a.dbg_l2[dbg_row + j] = kNeg;
          }
        }
        r[j] = key ? ((key << 16) | (0xffffu - j)) : 0u;  // unique: equal scores -> lower j first
        nreal += key != 0u;
      }
      // Requests = the row's Kgr highest keys, equal scores broken by the lower candidate index
      // (unique 32-bit keys: score << 16 | 0xffff - j).  With 64 candidates and Kgr <= 32 the
      // threshold comes from sorting networks (two sorted halves, a max-merge to the top-32 set,
      // one bitonic clean); otherwise from a radix select on the 16-bit score.
      const bool active = rvalid && nreal > 0;
      const bool all = a.Kgr >= a.Kc * M || nreal <= a.Kgr;
      // pm rows are padded by 16 bytes so that 16-byte stores of 32 rows spread over all banks (an
      // unpadded row of 64 u16 puts every row at the same banks)
      auto put = [&](uint32_t k32) {  // record a requested key in the pooling matrix
        const int j = 0xffff - (int)(k32 & 0xffffu);
        pm[(size_t)(hs * 64 + t) * KTP + j] = (uint16_t)(k32 >> 16);
      };
      const bool sorted_path = KT == 64 && a.Kgr <= 32 && active && !all;
      uint32_t T = 0u;    // radix path: requested iff score > T, or == T for the first `need` (lowest j)
      int need = 0;
      if constexpr (KT == 64) {
        if (sorted_path) {
          sort_desc<32>(r);
          sort_desc<32>(r + 32);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = max(r[i], r[KT - 1 - i]);
          // r[0..31]: the set of the 32 highest keys (a bitonic sequence); sorted only when fewer
          // than 32 of them are requested
          if (a.Kgr < 32) clean_desc<32>(r);
        }
      }
      if (!sorted_path && active && !all) {
        for (int bit = 15; bit >= 0; --bit) {
          const uint32_t cand = (T | (1u << bit)) << 16;
          int c4[4] = {0, 0, 0, 0};  // four partial counts: short dependence chains
#pragma unroll
          for (int j = 0; j < KT; ++j) c4[j & 3] += r[j] >= cand;
          if (c4[0] + c4[1] + c4[2] + c4[3] >= a.Kgr) T |= 1u << bit;
        }
        need = a.Kgr;
#pragma unroll
        for (int j = 0; j < KT; ++j) need -= (r[j] >> 16) > T;
      }
      // Pooling (max requesting score and first requesting row per candidate): each row thread
      // stores its requested scores into a [head][row][candidate] u16 matrix in the freed Q area,
      // then one thread per (head, candidate) reduces the candidate's column over the 64 rows.
      // every row thread writes its whole row (zeros where nothing is requested); the matrix
      // reuses the Q area, which the level-2 MMA (waited for above) no longer reads
      uint4* prow = reinterpret_cast<uint4*>(pm + (size_t)(hs * 64 + t) * KTP);
      if (sorted_path) {
#pragma unroll
        for (int c = 0; c < KT / 8; ++c) prow[c] = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < a.Kgr && r[i]) put(r[i]);
      } else {
        // the row's requested scores (0 elsewhere), packed in pairs, as whole 16-byte pieces
#pragma unroll
        for (int c = 0; c < KT / 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint32_t sc[2] = {r[8 * c + 2 * e] >> 16, r[8 * c + 2 * e + 1] >> 16};
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              bool req = false;
              if (active && sc[h2]) {
                if (all || sc[h2] > T) req = true;
                else if (sc[h2] == T && need > 0) { req = true; --need; }  // ascending j: lowest index first
              }
              sc[h2] = req ? sc[h2] : 0u;
            }
            w[e] = sc[0] | (sc[1] << 16);
          }
          prow[c] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      asm volatile("bar.sync 2, 128;" ::: "memory");
      for (int i = row; i < 2 * KT; i += 128) {
        const int hh = i / KT, j = i % KT;
        const uint16_t* src = pm + (size_t)hh * 64 * KTP + j;  // column j: consecutive lanes, consecutive j
        uint32_t mx = 0u, first = 0xffffffffu;
#pragma unroll 16
        for (int t2 = 63; t2 >= 0; --t2) {
          const uint32_t v = src[(size_t)t2 * KTP];
          mx = max(mx, v);
          first = v ? (uint32_t)t2 : first;
        }
        ms->gpool[hh][j] = mx;
        ms->gt0[hh][j] = mx ? first : 0xffffffffu;
      }
    }
    __syncthreads();
    if (warp == 2 || warp == 3) {
      const int hs = warp - 2;
      const int th = 4 * ms->ksel[hs];
      unsigned char* fl = flags + hs * NP;
      uint32_t* keys = pooled + hs * NP;  // reused as 32-bit unique keys of the groups
      for (int j = lane; j < th; j += 32) {
        const uint32_t g = ms->gpool[hs][j];
        keys[j] = (ms->gt0[hs][j] != 0xffffffffu) ? ((g << 16) | (0xffffu - j)) : 0u;
      }
      __syncwarp();
      if (a.Kg >= a.Kc * M) {
        for (int j = lane; j < th; j += 32) fl[j] = keys[j] != 0u;
        __syncwarp();
      } else {
        warp_select_u32(keys, th, a.Kg, fl);
      }
      int k = 0;
      const size_t o = (hs ? out1 : out0) * a.Kg;
      for (int base = 0; base < th; base += 32) {
        const int j = base + lane;
        const bool s = j < th && fl[j];
        const unsigned bal = __ballot_sync(0xffffffffu, s);
        if (s) {
          const int slot = k + __popc(bal & ((1u << lane) - 1u));
          a.open_gid[o + slot] = ms->sel[hs][j >> 2] * M + (j & 3);
          a.open_t0[o + slot] = (int)ms->gt0[hs][j];
        }
        k += __popc(bal);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

}  // namespace rtc

bool route_tc_supported(const hga_params& p, int64_t S) {
  const int64_t N = (S + 63) / 64;
  const int Kc = p.topk_chunks > 0 ? (int)(p.topk_chunks < N ? p.topk_chunks : N) : 0;
  return p.dtype == HGA_DTYPE_BF16 && p.head_dim == 128 && p.chunk_size == 64 && p.group_size == 16 &&
         (p.nhead / p.kv_heads) % 2 == 0 && Kc <= 32 && N < 65536 && S * p.batch < (1ll << 31);
}

cudaError_t launch_route_tc(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout, const void* ck, const void* gk,
                            int64_t sum_cap, int32_t* sel_chunk, int32_t* sel_t0, int32_t* open_gid, int32_t* open_t0,
                            float* dbg1, float* dbg2, cudaStream_t st) {
  using namespace tc;
  const int N = (int)((S + 63) / 64);
  const int Kc = p.topk_chunks > 0 ? (p.topk_chunks < N ? p.topk_chunks : N) : 0;
  const int Tg = Kc * 4;
  int Kg = p.topk_groups > 0 ? (p.topk_groups < Tg ? p.topk_groups : Tg) : 0;
  const int Kgr = p.topk_groups > 0 ? ((p.topk_groups / 2) < Tg ? p.topk_groups / 2 : Tg) : 0;
  if (Kgr == 0) Kg = 0;
  if (((uintptr_t)q | (uintptr_t)ck | (uintptr_t)gk) & 15) return cudaErrorMisalignedAddress;
  if ((int64_t)p.batch * p.kv_heads * sum_cap >= (1ll << 31)) return cudaErrorInvalidConfiguration;
  CUtensorMap mq, mck;
  const cuuint64_t dck[2] = {128, (cuuint64_t)p.batch * p.kv_heads * sum_cap}, sck[1] = {256};
  const cuuint32_t bck[2] = {64, 128};
  if (!make_map(&mck, ck, 2, dck, sck, bck)) return cudaErrorInvalidValue;
  if (q_layout == 1) {
    const cuuint64_t dq[3] = {128, (cuuint64_t)p.nhead, (cuuint64_t)(p.batch * qr.sq)};
    const cuuint64_t sq[2] = {256, (cuuint64_t)p.nhead * 256};
    const cuuint32_t bq[3] = {64, 1, 64};
    if (!make_map(&mq, q, 3, dq, sq, bq)) return cudaErrorInvalidValue;
  } else {
    const cuuint64_t dq[2] = {128, (cuuint64_t)p.batch * p.nhead * qr.sq};
    const cuuint64_t sq[1] = {256};
    const cuuint32_t bq[2] = {64, 64};
    if (!make_map(&mq, q, 2, dq, sq, bq)) return cudaErrorInvalidValue;
  }
  rtc::Args a;
  a.chunk0 = qr.chunk0; a.nl = qr.count; a.sq = (int)qr.sq;
  a.S = (int)S; a.H = p.nhead; a.KVH = p.kv_heads; a.N = N; a.Kc = Kc; a.Kg = Kg; a.Kgr = Kgr;
  const int NP = N > Tg ? N : Tg;
  a.NP = NP;
  a.keep_first = p.keep_first; a.keep_last = p.keep_last; a.q_layout = q_layout; a.sum_cap = sum_cap;
  a.scale = p.scale; a.group_k = (const __nv_bfloat16*)gk;
  a.sel_chunk = sel_chunk; a.sel_t0 = sel_t0; a.open_gid = open_gid; a.open_t0 = open_t0;
  a.dbg_l1 = dbg1; a.dbg_l2 = dbg2;
  const int smem = rtc::L::kFixed + 2 * NP * 4 * 2 + ((2 * NP + 15) & ~15) + (int)sizeof(rtc::Misc) + 1024;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  dim3 grid(qr.count, p.nhead / 2, p.batch);
  cudaError_t e;
  if (Kc <= 16) {
    e = cudaFuncSetAttribute(rtc::route_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    rtc::route_tc_kernel<16><<<grid, rtc::threads_for<16>(), smem, st>>>(mq, mck, a);
  } else {
    e = cudaFuncSetAttribute(rtc::route_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    rtc::route_tc_kernel<32><<<grid, rtc::threads_for<32>(), smem, st>>>(mq, mck, a);
  }
  return cudaGetLastError();
}

HGA_DEFINE_ERROR_READER(route_tc_error_status)

}  // namespace hga
