// Summary builder: mixed-RoPE chunk / group key summaries and scaled group value sums.
//
// Reference arithmetic (ExistingModelFineTuning/KvRouter/vectorized.py:168-183, 265-287 and
// chunk_router.py:693-735), reproduced rounding point by rounding point:
//   raw_sum   = T( T(sum_t k_raw)  * scale )          sum accumulated in fp32
//   tokenwise = T( T(sum_t k_rope) * scale )
//   endpoint  = T( rotate(fp32(raw_sum), cos[a], sin[a]) )  a = anchor = start + (len-1)//2
//   summary_d = (d mod Dh/2) < cutoff ? tokenwise_d : endpoint_d
//   group_v   = T( T(sum_t v) * group_kv_scale )
// The fp32 accumulation order is the one torch's CPU reduction uses for these shapes:
// sequential inside blocks of 16 rows, block partials added in order.  For bf16/fp16 inputs the
// fp32 sums are exact for any order in practice.
//
// One CTA per (batch, kv-head, chunk); thread d owns head-dim column d, so every token row is a
// coalesced Dh-wide load, and the summary's rotate-half partner is exchanged through smem.
#include "hga_common.cuh"

namespace hga {

template <typename T, typename R>
__global__ void __launch_bounds__(256) summaries_kernel(
    hga_params p, int64_t S, int64_t pos0, const T* __restrict__ k_raw, const T* __restrict__ k_rope,
    const T* __restrict__ v, int64_t kv_cap, const R* __restrict__ cos_t, const R* __restrict__ sin_t,
    int64_t rot_row0, T* __restrict__ chunk_k, T* __restrict__ group_k, T* __restrict__ group_v,
    int64_t sum_cap, int64_t out_chunk0, int N, int round_tab) {
  extern __shared__ float sm_sum[];  // [2][Dh]: raw sums for the rotation partner exchange
  const int Dh = p.head_dim, C = p.chunk_size, gs = p.group_size, M = C / gs, half = Dh / 2;
  const int d = threadIdx.x;
  const int c = blockIdx.x % N;
  const int bk = blockIdx.x / N;  // b * KVH + kvh
  const int64_t row0 = (int64_t)c * C;
  int len = (int)((S - row0) < C ? (S - row0) : C);
  const size_t base = (size_t)bk * kv_cap * Dh;
  const bool active = d < Dh;

  float craw = 0.f, crope = 0.f;  // chunk totals (sum of 16-row block partials, in order)
  float braw = 0.f, brope = 0.f;  // current 16-row block partial
  float graw = 0.f, grope = 0.f, gv = 0.f;
  for (int m = 0; m < M; ++m) {
    graw = grope = gv = 0.f;
    float g16raw = 0.f, g16rope = 0.f, g16v = 0.f;  // group-local 16-row block partials
    for (int u = 0; u < gs; ++u) {
      const int t = m * gs + u;
      float xr = 0.f, xo = 0.f, xv = 0.f;
      if (active && t < len) {
        const size_t off = base + (size_t)(row0 + t) * Dh + d;
        xr = Num<T>::to_f(k_raw[off]);
        xo = Num<T>::to_f(k_rope[off]);
        xv = Num<T>::to_f(v[off]);
      }
      braw = __fadd_rn(braw, xr);
      brope = __fadd_rn(brope, xo);
      g16raw = __fadd_rn(g16raw, xr);
      g16rope = __fadd_rn(g16rope, xo);
      g16v = __fadd_rn(g16v, xv);
      if (((t + 1) & 15) == 0) {
        craw = __fadd_rn(craw, braw);
        crope = __fadd_rn(crope, brope);
        braw = brope = 0.f;
      }
      if (((u + 1) & 15) == 0 || u == gs - 1) {
        graw = __fadd_rn(graw, g16raw);
        grope = __fadd_rn(grope, g16rope);
        gv = __fadd_rn(gv, g16v);
        g16raw = g16rope = g16v = 0.f;
      }
    }
    // group summary m
    const float sc = p.group_kv_scale;
    const float rs = Num<T>::round(__fmul_rn(Num<T>::round(graw), sc));
    const float tw = Num<T>::round(__fmul_rn(Num<T>::round(grope), sc));
    const float vs = Num<T>::round(__fmul_rn(Num<T>::round(gv), sc));
    int glen = len - m * gs;
    glen = glen < 0 ? 0 : (glen > gs ? gs : glen);
    int64_t anchor = row0 + m * gs + ((glen < 1 ? 1 : glen) - 1) / 2;
    if (anchor > S - 1) anchor = S - 1;
    __syncthreads();
    if (active) sm_sum[d] = rs;
    __syncthreads();
    if (active) {
      const int64_t rr = (pos0 + anchor - rot_row0) * Dh + d;
      float cs = Num<R>::to_f(cos_t[rr]), sn = Num<R>::to_f(sin_t[rr]);
      if (round_tab) { cs = Num<T>::round(cs); sn = Num<T>::round(sn); }
      float ep;
      if (d < half) ep = __fsub_rn(__fmul_rn(rs, cs), __fmul_rn(sm_sum[d + half], sn));
      else          ep = __fadd_rn(__fmul_rn(rs, cs), __fmul_rn(sm_sum[d - half], sn));
      const int pair = d < half ? d : d - half;
      const float out = pair < p.cutoff_pair ? tw : Num<T>::round(ep);
      const size_t go = (((size_t)bk * sum_cap + out_chunk0 + c) * M + m) * Dh + d;
      group_k[go] = Num<T>::from_f(out);
      if (group_v) group_v[go] = Num<T>::from_f(vs);
    }
  }
  if (C & 15) {  // trailing partial 16-row block (only when C is not a multiple of 16)
    craw = __fadd_rn(craw, braw);
    crope = __fadd_rn(crope, brope);
  }
  // chunk summary (scale 1.0)
  const float rs = Num<T>::round(craw);
  const float tw = Num<T>::round(crope);
  int64_t anchor = row0 + ((len < 1 ? 1 : len) - 1) / 2;
  if (anchor > S - 1) anchor = S - 1;
  __syncthreads();
  if (active) sm_sum[d] = rs;
  __syncthreads();
  if (active) {
    const int64_t rr = (pos0 + anchor - rot_row0) * Dh + d;
    float cs = Num<R>::to_f(cos_t[rr]), sn = Num<R>::to_f(sin_t[rr]);
      if (round_tab) { cs = Num<T>::round(cs); sn = Num<T>::round(sn); }
    float ep;
    if (d < half) ep = __fsub_rn(__fmul_rn(rs, cs), __fmul_rn(sm_sum[d + half], sn));
    else          ep = __fadd_rn(__fmul_rn(rs, cs), __fmul_rn(sm_sum[d - half], sn));
    const int pair = d < half ? d : d - half;
    const float out = pair < p.cutoff_pair ? tw : Num<T>::round(ep);
    chunk_k[((size_t)bk * sum_cap + out_chunk0 + c) * Dh + d] = Num<T>::from_f(out);
  }
}

template <typename T, typename R>
static cudaError_t launch_summaries_t(const hga_params& p, int64_t S, int64_t pos0, const void* k_raw,
                                      const void* k_rope, const void* v, int64_t kv_cap, const void* cos,
                                      const void* sin, int64_t rot_row0, void* ck, void* gk, void* gv,
                                      int64_t sum_cap, int64_t out_chunk0, int round_tab, cudaStream_t st) {
  const int N = (int)((S + p.chunk_size - 1) / p.chunk_size);
  const int threads = ((p.head_dim + 31) / 32) * 32;
  const dim3 grid((unsigned)(N * p.batch * p.kv_heads));
  summaries_kernel<T, R><<<grid, threads, 2 * p.head_dim * sizeof(float), st>>>(
      p, S, pos0, (const T*)k_raw, (const T*)k_rope, (const T*)v, kv_cap, (const R*)cos, (const R*)sin,
      rot_row0, (T*)ck, (T*)gk, (T*)gv, sum_cap, out_chunk0, N, round_tab);
  return cudaGetLastError();
}

cudaError_t launch_summaries(const hga_params& p, int64_t S, int64_t pos0, const void* k_raw,
                             const void* k_rope, const void* v, int64_t kv_cap, const void* cos,
                             const void* sin, int rot_mode, int64_t rot_row0, void* ck, void* gk,
                             void* gv, int64_t sum_cap, int64_t out_chunk0, cudaStream_t st) {
  const int round_tab = rot_mode == HGA_ROT_F32_ROUNDED;
#define HGA_SUM(T)                                                                                    \
  return rot_mode != HGA_ROT_MODEL                                                                     \
             ? launch_summaries_t<T, float>(p, S, pos0, k_raw, k_rope, v, kv_cap, cos, sin, rot_row0, \
                                            ck, gk, gv, sum_cap, out_chunk0, round_tab, st)           \
             : launch_summaries_t<T, T>(p, S, pos0, k_raw, k_rope, v, kv_cap, cos, sin, rot_row0, ck, \
                                        gk, gv, sum_cap, out_chunk0, 0, st);
  switch (p.dtype) {
    case HGA_DTYPE_F32: HGA_SUM(float)
    case HGA_DTYPE_BF16: HGA_SUM(__nv_bfloat16)
    case HGA_DTYPE_F16: HGA_SUM(__half)
  }
#undef HGA_SUM
  return cudaErrorInvalidValue;
}

}  // namespace hga

namespace hga {

// Both summary sets of a fresh prefill from one read of K/V: set A (the chunk-parallel routing
// summaries of all N chunks, endpoint rotation from table A) and set B (the store seed of the first
// nB closed chunks, endpoint rotation from table B, group V sums included).  The sums are the same
// for both sets; only the endpoint rotation (table, rounding of the table entries) and the
// destination differ.
//
// Thread = (chunk, 16-row block, 8 contiguous head-dim columns): it reads each of its 16 token rows
// as one 16-byte piece per tensor and sums them sequentially in fp32 (the order of torch's CPU
// reduction, as in summaries_kernel).  The block partials meet in shared memory, where the group
// and chunk totals are formed by adding the partials in block order, then the summaries are
// rotated and written (16-byte stores).  bf16 / fp16, head_dim 64 or 128, chunk and group sizes
// multiples of 16, chunk_size <= 128.
template <typename T, int DH>
__global__ void __launch_bounds__(256, 4) summaries_dual_kernel(
    hga_params p, int64_t S, int64_t pos0, const T* __restrict__ k_raw, const T* __restrict__ k_rope,
    const T* __restrict__ v, int64_t kv_cap, int N, int cpb,
    const float* __restrict__ cosA, const float* __restrict__ sinA, int64_t rowA0, int roundA, T* ckA, T* gkA,
    int64_t capA, int64_t outA0,
    const float* __restrict__ cosB, const float* __restrict__ sinB, int64_t rowB0, int nB, T* ckB, T* gkB, T* gvB,
    int64_t capB, int64_t outB0) {
  constexpr int CG = DH / 8, HALF = DH / 2;
  extern __shared__ float sm[];
  const int C = p.chunk_size, gs = p.group_size, M = C / gs, NBLK = C / 16, BPG = gs / 16;
  // smem: block partials [cpb][NBLK][3][DH] (raw, rope, v), then rotation scratch [cpb][M + 1][DH]
  float* part = sm;
  float* rot = sm + (size_t)cpb * NBLK * 3 * DH;
  const int tid = threadIdx.x;
  const int cg = tid % CG, blk = (tid / CG) % NBLK, ci = tid / (CG * NBLK);
  const int bk = blockIdx.y;
  const int c = blockIdx.x * cpb + ci;
  const bool mine = ci < cpb;
  const int64_t row0 = (int64_t)c * C;
  const int len = (mine && c < N) ? (int)((S - row0) < C ? (S - row0) : C) : 0;
  const size_t base = (size_t)bk * kv_cap * DH + (size_t)cg * 8;

  // ---- phase 1: the 16-row block partials of this thread's 8 columns -------------------------
  if (mine) {
    float sr[8], so[8], sv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) sr[e] = so[e] = sv[e] = 0.f;
    const int t0 = blk * 16;
    // four rows' loads (12 x 16 bytes) in flight before they are added, in row order (few
    // registers: four CTAs per SM hold the whole grid in one wave); rows past the sequence load
    // the chunk's first row (in bounds) and are not added
#pragma unroll
    for (int u0 = 0; u0 < 16; u0 += 4) {
      if (t0 + u0 >= len) break;
      uint4 ur[4], uo[4], uv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + u0 + u;
        const size_t off = base + (size_t)(row0 + (t < len ? t : 0)) * DH;
        ur[u] = __ldg(reinterpret_cast<const uint4*>(k_raw + off));
        uo[u] = __ldg(reinterpret_cast<const uint4*>(k_rope + off));
        uv[u] = __ldg(reinterpret_cast<const uint4*>(v + off));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (t0 + u0 + u >= len) break;
        const T* hr = reinterpret_cast<const T*>(&ur[u]);
        const T* ho = reinterpret_cast<const T*>(&uo[u]);
        const T* hv = reinterpret_cast<const T*>(&uv[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          sr[e] = __fadd_rn(sr[e], Num<T>::to_f(hr[e]));
          so[e] = __fadd_rn(so[e], Num<T>::to_f(ho[e]));
          sv[e] = __fadd_rn(sv[e], Num<T>::to_f(hv[e]));
        }
      }
    }
    float* pp = part + ((size_t)(ci * NBLK + blk) * 3) * DH + cg * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) { pp[e] = sr[e]; pp[DH + e] = so[e]; pp[2 * DH + e] = sv[e]; }
  }
  __syncthreads();

  // ---- phase 2: group and chunk sums (block partials added in order), rounded raw sums -------
  // slot j < M: group j (thread blk == j, when j < NBLK); slot M: the chunk (thread blk == M % NBLK
  // for the raw chunk sum, computed by the thread of block 0 when M == NBLK)
  const int slot = blk < M ? blk : -1;
  const int cslot = (M < NBLK) ? M : 0;  // which block thread also owns the chunk sums
  float g_rs[8], g_tw[8], g_vs[8], c_rs[8], c_tw[8];
  if (mine) {
    if (slot >= 0) {
      float gr[8], go[8], gv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) gr[e] = go[e] = gv[e] = 0.f;
      for (int q = 0; q < BPG; ++q) {
        const float* pp = part + ((size_t)(ci * NBLK + slot * BPG + q) * 3) * DH + cg * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          gr[e] = __fadd_rn(gr[e], pp[e]);
          go[e] = __fadd_rn(go[e], pp[DH + e]);
          gv[e] = __fadd_rn(gv[e], pp[2 * DH + e]);
        }
      }
      const float sc = p.group_kv_scale;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        g_rs[e] = Num<T>::round(__fmul_rn(Num<T>::round(gr[e]), sc));
        g_tw[e] = Num<T>::round(__fmul_rn(Num<T>::round(go[e]), sc));
        g_vs[e] = Num<T>::round(__fmul_rn(Num<T>::round(gv[e]), sc));
        rot[((size_t)ci * (M + 1) + slot) * DH + cg * 8 + e] = g_rs[e];
      }
    }
    if (blk == cslot) {
      float cr[8], co[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) cr[e] = co[e] = 0.f;
      for (int q = 0; q < NBLK; ++q) {
        const float* pp = part + ((size_t)(ci * NBLK + q) * 3) * DH + cg * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) { cr[e] = __fadd_rn(cr[e], pp[e]); co[e] = __fadd_rn(co[e], pp[DH + e]); }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c_rs[e] = Num<T>::round(cr[e]);
        c_tw[e] = Num<T>::round(co[e]);
        rot[((size_t)ci * (M + 1) + M) * DH + cg * 8 + e] = c_rs[e];
      }
    }
  }
  __syncthreads();

  // ---- phase 3: endpoint rotations and stores -----------------------------------------------
  auto emit = [&](int sl, const float* rs, const float* tw, const float* cs_t, const float* sn_t, int64_t trow,
                  int rnd, T* dst) {
    const int d0 = cg * 8;
    const float4* cp = reinterpret_cast<const float4*>(cs_t + trow * DH + d0);
    const float4* sp = reinterpret_cast<const float4*>(sn_t + trow * DH + d0);
    const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
    float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const float* partner = rot + ((size_t)ci * (M + 1) + sl) * DH;
    uint4 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (rnd) { cs[e] = Num<T>::round(cs[e]); sn[e] = Num<T>::round(sn[e]); }
      const int d = d0 + e;
      const float ep = d < HALF ? __fsub_rn(__fmul_rn(rs[e], cs[e]), __fmul_rn(partner[d + HALF], sn[e]))
                                : __fadd_rn(__fmul_rn(rs[e], cs[e]), __fmul_rn(partner[d - HALF], sn[e]));
      h[e] = Num<T>::from_f((d % HALF) < p.cutoff_pair ? tw[e] : Num<T>::round(ep));
    }
    *reinterpret_cast<uint4*>(dst + d0) = u;
  };
  if (len > 0) {
    if (slot >= 0) {
      const int m = slot;
      int glen = len - m * gs;
      glen = glen < 0 ? 0 : (glen > gs ? gs : glen);
      int64_t anchor = row0 + m * gs + ((glen < 1 ? 1 : glen) - 1) / 2;
      if (anchor > S - 1) anchor = S - 1;
      emit(m, g_rs, g_tw, cosA, sinA, pos0 + anchor - rowA0, roundA,
           gkA + (((size_t)bk * capA + outA0 + c) * M + m) * DH);
      if (c < nB) {
        const size_t o = (((size_t)bk * capB + outB0 + c) * M + m) * DH;
        emit(m, g_rs, g_tw, cosB, sinB, pos0 + row0 + m * gs + (gs - 1) / 2 - rowB0, 0, gkB + o);
        if (gvB) {
          uint4 u;
          T* h = reinterpret_cast<T*>(&u);
#pragma unroll
          for (int e = 0; e < 8; ++e) h[e] = Num<T>::from_f(g_vs[e]);
          *reinterpret_cast<uint4*>(gvB + o + cg * 8) = u;
        }
      }
    }
    if (blk == cslot) {
      int64_t anchor = row0 + ((len < 1 ? 1 : len) - 1) / 2;
      if (anchor > S - 1) anchor = S - 1;
      emit(M, c_rs, c_tw, cosA, sinA, pos0 + anchor - rowA0, roundA, ckA + ((size_t)bk * capA + outA0 + c) * DH);
      if (c < nB)
        emit(M, c_rs, c_tw, cosB, sinB, pos0 + row0 + (C - 1) / 2 - rowB0, 0,
             ckB + ((size_t)bk * capB + outB0 + c) * DH);
    }
  }
}

bool summaries_dual_supported(const hga_params& p) {
  return (p.dtype == HGA_DTYPE_BF16 || p.dtype == HGA_DTYPE_F16) && (p.head_dim == 64 || p.head_dim == 128) &&
         p.chunk_size % 16 == 0 && p.group_size % 16 == 0 && p.chunk_size <= 128;
}

cudaError_t launch_summaries_dual(const hga_params& p, int64_t S, int64_t pos0, const void* k_raw,
                                  const void* k_rope, const void* v, int64_t kv_cap, const float* cosA,
                                  const float* sinA, int64_t rowA0, int roundA, void* ckA, void* gkA,
                                  int64_t capA, int64_t outA0, const float* cosB, const float* sinB,
                                  int64_t rowB0, int nB, void* ckB, void* gkB, void* gvB, int64_t capB,
                                  int64_t outB0, cudaStream_t st) {
  const int N = (int)((S + p.chunk_size - 1) / p.chunk_size);
  const int per_chunk = (p.head_dim / 8) * (p.chunk_size / 16);  // threads per chunk
  const int cpb = 256 / per_chunk;                                 // chunks per CTA
  const int M = p.chunk_size / p.group_size;
  const size_t smem = ((size_t)cpb * (p.chunk_size / 16) * 3 + (size_t)cpb * (M + 1)) * p.head_dim * sizeof(float);
  const dim3 grid((unsigned)((N + cpb - 1) / cpb), (unsigned)(p.batch * p.kv_heads));
#define HGA_SD(TT, DHV)                                                                                      \
  summaries_dual_kernel<TT, DHV><<<grid, 256, smem, st>>>(p, S, pos0, (const TT*)k_raw, (const TT*)k_rope,   \
                                                          (const TT*)v, kv_cap, N, cpb, cosA, sinA, rowA0,   \
                                                          roundA, (TT*)ckA, (TT*)gkA, capA, outA0, cosB, sinB, \
                                                          rowB0, nB, (TT*)ckB, (TT*)gkB, (TT*)gvB, capB, outB0)
  if (p.dtype == HGA_DTYPE_BF16) {
    if (p.head_dim == 128) HGA_SD(__nv_bfloat16, 128); else HGA_SD(__nv_bfloat16, 64);
  } else {
    if (p.head_dim == 128) HGA_SD(__half, 128); else HGA_SD(__half, 64);
  }
#undef HGA_SD
  return cudaGetLastError();
}

}  // namespace hga
