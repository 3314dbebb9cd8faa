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
