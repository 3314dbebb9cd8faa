// Fused projection epilogue: q/k RMSNorm + RoPE + head-major K/V layout in one pass.
//
// Input: the fused QKV projection output, one row per token: [q heads | k heads | v heads] x Dh.
// Output: q_rope [B,S,H,Dh] (token-major, what the router and attention read through q_layout 1),
// and k_raw / k_rope / v rows [B,KVH,cap,Dh] (the KV-store layout).
// Reference arithmetic (one rounding per torch op):
//   norm_mode 0 (HierarchicalGlobalAttentionRouted.py:56-67, :151-152):
//       y = T( (fp32(w) * x) * rsqrt(mean(x^2) + eps) )
//   norm_mode 1 (HF Qwen3MoeRMSNorm, used by qwen_routed_attention.py:171-172):
//       y = T( w * T( x * rsqrt(mean(x^2) + eps) ) )
//   rope_mode 0 (HierarchicalGlobalAttentionRouted.py:156-157): fp32 math on fp32 cos/sin, one rounding
//   rope_mode 1 (HF apply_rotary_pos_emb, qwen_routed_attention.py:176): model-dtype math,
//       y = T( T(x*cos) + T(rot(x)*sin) ) with cos/sin in the model dtype.
// rsqrt is evaluated as a correctly rounded 1/sqrt (what torch's CPU kernel computes).
// One warp per (token, projected head row); the row is staged in smem for the rotate-half partner.
#include "hga_common.cuh"

#include <type_traits>

namespace hga {

constexpr int kProWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kProWarps * 32) prologue_kernel(
    hga_params p, int64_t S, const T* __restrict__ qkv, int64_t row_stride, const T* __restrict__ qw,
    const T* __restrict__ kw, float eps, int norm_mode, const void* __restrict__ cos_t,
    const void* __restrict__ sin_t, int rope_mode, int64_t rot_row0, int64_t pos0, T* __restrict__ q_out,
    T* __restrict__ kraw_out, T* __restrict__ krope_out, T* __restrict__ v_out, int64_t kv_cap, int64_t kv_row0) {
  extern __shared__ float prow[];
  const int H = p.nhead, KVH = p.kv_heads, Dh = p.head_dim, half = Dh / 2;
  const int rows_per_tok = H + 2 * KVH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* buf = prow + warp * Dh;
  const int64_t gw = (int64_t)blockIdx.x * kProWarps + warp;
  const int64_t total = (int64_t)p.batch * S * rows_per_tok;
  if (gw >= total) return;
  const int r = (int)(gw % rows_per_tok);
  const int64_t bt = gw / rows_per_tok;  // b * S + t
  const int64_t t = bt % S;
  const int b = (int)(bt / S);
  const T* src = qkv + bt * row_stride + (int64_t)r * Dh;
  const bool is_q = r < H, is_k = r >= H && r < H + KVH;
  const int kvh = is_q ? 0 : (is_k ? r - H : r - H - KVH);
  // load + optional RMSNorm
  const T* w = is_q ? qw : (is_k ? kw : nullptr);
  float ss = 0.f;
  for (int d = lane; d < Dh; d += 32) {
    const float x = Num<T>::to_f(src[d]);
    buf[d] = x;
    ss = __fadd_rn(ss, __fmul_rn(x, x));
  }
  if (!is_q && !is_k) {  // v: layout transform only
    T* dst = v_out + (((int64_t)b * KVH + kvh) * kv_cap + kv_row0 + t) * Dh;
    for (int d = lane; d < Dh; d += 32) dst[d] = src[d];
    return;
  }
  if (w) {
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float mean = __fdiv_rn(ss, (float)Dh);
    const float rs = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (int d = lane; d < Dh; d += 32) {
      const float x = buf[d];
      const float wf = Num<T>::to_f(w[d]);
      float y;
      if (norm_mode == 0) y = Num<T>::round(__fmul_rn(__fmul_rn(wf, x), rs));
      else y = Num<T>::round(__fmul_rn(wf, Num<T>::round(__fmul_rn(x, rs))));
      buf[d] = y;
    }
  }
  __syncwarp();
  // RoPE
  const int64_t rr = (pos0 + t - rot_row0) * Dh;
  T* dst_rope;
  if (is_q) dst_rope = q_out + (bt * H + r) * Dh;
  else dst_rope = krope_out + (((int64_t)b * KVH + kvh) * kv_cap + kv_row0 + t) * Dh;
  T* dst_raw = is_k ? kraw_out + (((int64_t)b * KVH + kvh) * kv_cap + kv_row0 + t) * Dh : nullptr;
  for (int d = lane; d < Dh; d += 32) {
    const float x = buf[d];
    const float xp = d < half ? -buf[d + half] : buf[d - half];
    float y;
    if (rope_mode == 0) {
      const float cs = ((const float*)cos_t)[rr + d], sn = ((const float*)sin_t)[rr + d];
      y = __fadd_rn(__fmul_rn(x, cs), __fmul_rn(xp, sn));
    } else {
      const float cs = Num<T>::to_f(((const T*)cos_t)[rr + d]), sn = Num<T>::to_f(((const T*)sin_t)[rr + d]);
      y = __fadd_rn(Num<T>::round(__fmul_rn(x, cs)), Num<T>::round(__fmul_rn(xp, sn)));
    }
    dst_rope[d] = Num<T>::from_f(y);
    if (dst_raw) dst_raw[d] = Num<T>::from_f(x);
  }
}

// Vectorised variant for head_dim = 32 * EPL: lane l holds elements [EPL*l, EPL*l + EPL) of the
// row (one 8- or 16-byte load), the rotate-half partner lives in lane l ^ (16) and is fetched with a
// shuffle, so nothing is staged in shared memory and every access is a whole-row line.  Same
// arithmetic and rounding points as prologue_kernel; the sum of squares is reduced in another order.
template <int BYTES> struct VecT;
template <> struct VecT<4> { using type = uint32_t; };
template <> struct VecT<8> { using type = uint2; };
template <> struct VecT<16> { using type = uint4; };
// EPL contiguous elements as one aligned vector access (the row layouts keep it aligned)
template <typename T, int EPL>
__device__ __forceinline__ void ld_vec(const T* src, T* v) {
  using V = typename VecT<sizeof(T) * EPL>::type;
  const V x = *reinterpret_cast<const V*>(src);
  memcpy(v, &x, sizeof(V));
}
template <typename T, int EPL>
__device__ __forceinline__ void st_vec(T* dst, const T* v) {
  using V = typename VecT<sizeof(T) * EPL>::type;
  V x;
  memcpy(&x, v, sizeof(V));
  *reinterpret_cast<V*>(dst) = x;
}

template <typename T, int EPL>
__global__ void __launch_bounds__(kProWarps * 32) prologue_vec_kernel(
    hga_params p, int64_t S, const T* __restrict__ qkv, int64_t row_stride, const T* __restrict__ qw,
    const T* __restrict__ kw, float eps, int norm_mode, const void* __restrict__ cos_t,
    const void* __restrict__ sin_t, int rope_mode, int64_t rot_row0, int64_t pos0, T* __restrict__ q_out,
    T* __restrict__ kraw_out, T* __restrict__ krope_out, T* __restrict__ v_out, int64_t kv_cap, int64_t kv_row0) {
  constexpr int Dh = 32 * EPL;
  const int H = p.nhead, KVH = p.kv_heads;
  const int rows_per_tok = H + 2 * KVH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * kProWarps + warp;
  const int64_t total = (int64_t)p.batch * S * rows_per_tok;
  if (gw >= total) return;
  const int r = (int)(gw % rows_per_tok);
  const int64_t bt = gw / rows_per_tok;  // b * S + t
  const int64_t t = bt % S;
  const int b = (int)(bt / S);
  const bool is_q = r < H, is_k = r >= H && r < H + KVH;
  const int kvh = is_q ? 0 : (is_k ? r - H : r - H - KVH);
  const int d0 = lane * EPL;
  T xin[EPL];
  ld_vec<T, EPL>(qkv + bt * row_stride + (int64_t)r * Dh + d0, xin);
  if (!is_q && !is_k) {  // v: layout transform only
    st_vec<T, EPL>(v_out + (((int64_t)b * KVH + kvh) * kv_cap + kv_row0 + t) * Dh + d0, xin);
    return;
  }
  float x[EPL];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    x[e] = Num<T>::to_f(xin[e]);
    ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
  }
  const T* w = is_q ? qw : kw;
  if (w) {
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float mean = __fdiv_rn(ss, (float)Dh);
    const float rs = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float wf = Num<T>::to_f(w[d0 + e]);
      x[e] = norm_mode == 0 ? Num<T>::round(__fmul_rn(__fmul_rn(wf, x[e]), rs))
                            : Num<T>::round(__fmul_rn(wf, Num<T>::round(__fmul_rn(x[e], rs))));
    }
  }
  // RoPE: the partner of element d is d +- Dh/2, held by lane ^ 16 at the same position
  const int64_t rr = (pos0 + t - rot_row0) * Dh + d0;
  T* dst_rope = is_q ? q_out + (bt * H + r) * Dh + d0
                     : krope_out + (((int64_t)b * KVH + kvh) * kv_cap + kv_row0 + t) * Dh + d0;
  T* dst_raw = is_k ? kraw_out + (((int64_t)b * KVH + kvh) * kv_cap + kv_row0 + t) * Dh + d0 : nullptr;
  T yo[EPL], xo[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const float xp = lane < 16 ? -other : other;
    float y;
    if (rope_mode == 0) {
      const float cs = ((const float*)cos_t)[rr + e], sn = ((const float*)sin_t)[rr + e];
      y = __fadd_rn(__fmul_rn(x[e], cs), __fmul_rn(xp, sn));
    } else {
      const float cs = Num<T>::to_f(((const T*)cos_t)[rr + e]), sn = Num<T>::to_f(((const T*)sin_t)[rr + e]);
      y = __fadd_rn(Num<T>::round(__fmul_rn(x[e], cs)), Num<T>::round(__fmul_rn(xp, sn)));
    }
    yo[e] = Num<T>::from_f(y);
    xo[e] = Num<T>::from_f(x[e]);
  }
  st_vec<T, EPL>(dst_rope, yo);
  if (dst_raw) st_vec<T, EPL>(dst_raw, xo);
}

// One warp per token (batch b, position t): the token's H query rows and KVH key rows get the
// same arithmetic as prologue_vec_kernel (lane = EPL contiguous elements, RoPE partner by
// shuffle), but the rotary table entries of the position are read once per token (they depend on
// the position and the column only) instead of once per head row, four rows' loads are issued
// before any of them is used, and the row index needs no 64-bit division.  V rows are copied.
// bf16 pairs on sm_100: two fp32 products / sums in one instruction (each rounded like its scalar
// form), two roundings to bf16 in one conversion
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2(uint64_t v) {  // round both to bf16, lo in bits 0-15
  float lo, hi;
  upk2(v, lo, hi);
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint64_t unbf2(uint32_t w) {  // bf16 pair back to fp32
  return pk2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

template <typename T, int EPL>
__global__ void __launch_bounds__(kProWarps * 32, 4) prologue_tok_kernel(
    hga_params p, int64_t S, const T* __restrict__ qkv, int64_t row_stride, const T* __restrict__ qw,
    const T* __restrict__ kw, float eps, int norm_mode, const void* __restrict__ cos_t,
    const void* __restrict__ sin_t, int rope_mode, int64_t rot_row0, int64_t pos0, T* __restrict__ q_out,
    T* __restrict__ kraw_out, T* __restrict__ krope_out, T* __restrict__ v_out, int64_t kv_cap, int64_t kv_row0) {
  constexpr int Dh = 32 * EPL;
  constexpr int UNR = 4;
  const int H = p.nhead, KVH = p.kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bt = (int64_t)blockIdx.x * kProWarps + warp;  // b * S + t
  if (bt >= (int64_t)p.batch * S) return;
  const int b = (int)(bt / S);
  const int64_t t = bt - (int64_t)b * S;
  const int d0 = lane * EPL;
  const T* src = qkv + bt * row_stride + d0;
  // the position's rotary entries of this lane's columns
  float cs[EPL], sn[EPL];
  const int64_t rr = (pos0 + t - rot_row0) * Dh + d0;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    if (rope_mode == 0) {
      cs[e] = ((const float*)cos_t)[rr + e];
      sn[e] = ((const float*)sin_t)[rr + e];
    } else {
      cs[e] = Num<T>::to_f(((const T*)cos_t)[rr + e]);
      sn[e] = Num<T>::to_f(((const T*)sin_t)[rr + e]);
    }
  }
  float wq[EPL], wk[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    wq[e] = qw ? Num<T>::to_f(qw[d0 + e]) : 1.f;
    wk[e] = kw ? Num<T>::to_f(kw[d0 + e]) : 1.f;
  }
  const int nqk = H + KVH;
  for (int r0 = 0; r0 < nqk; r0 += UNR) {
    T xin[UNR][EPL];
#pragma unroll
    for (int u = 0; u < UNR; ++u)
      if (r0 + u < nqk) ld_vec<T, EPL>(src + (int64_t)(r0 + u) * Dh, xin[u]);
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int r = r0 + u;
      if (r >= nqk) break;  // warp-uniform
      const bool is_q = r < H;
      const int kvh = is_q ? 0 : r - H;
      float x[EPL];
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        x[e] = Num<T>::to_f(xin[u][e]);
        ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
      }
      if (is_q ? qw != nullptr : kw != nullptr) {
        for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        // ss / Dh: Dh is a power of two, so the product with its exact reciprocal is the same
        // correctly rounded quotient
        const float mean = __fmul_rn(ss, 1.f / (float)Dh);
        const float rs = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, eps)));
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          const uint64_t r2 = pk2(rs, rs);
#pragma unroll
          for (int e = 0; e < EPL; e += 2) {
            const uint64_t wv = is_q ? pk2(wq[e], wq[e + 1]) : pk2(wk[e], wk[e + 1]);
            const uint64_t xv = pk2(x[e], x[e + 1]);
            const uint64_t y = norm_mode == 0 ? mul2(mul2(wv, xv), r2) : mul2(wv, unbf2(bf2(mul2(xv, r2))));
            upk2(unbf2(bf2(y)), x[e], x[e + 1]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const float wf = is_q ? wq[e] : wk[e];
            x[e] = norm_mode == 0 ? Num<T>::round(__fmul_rn(__fmul_rn(wf, x[e]), rs))
                                  : Num<T>::round(__fmul_rn(wf, Num<T>::round(__fmul_rn(x[e], rs))));
          }
        }
      }
      T yo[EPL], xo[EPL];
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        // pairs: x is bf16-exact here, so its packed form is the k_raw row and the shuffled partner
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
          uint32_t xb;
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(xb) : "f"(x[e + 1]), "f"(x[e]));
          const uint32_t ob = __shfl_xor_sync(0xffffffffu, xb, 16);
          float o0, o1;
          upk2(unbf2(ob), o0, o1);
          const uint64_t xv = pk2(x[e], x[e + 1]);
          const uint64_t xp = lane < 16 ? pk2(-o0, -o1) : pk2(o0, o1);
          const uint64_t cv = pk2(cs[e], cs[e + 1]), sv = pk2(sn[e], sn[e + 1]);
          const uint32_t yb = rope_mode == 0 ? bf2(add2(mul2(xv, cv), mul2(xp, sv)))
                                             : bf2(add2(unbf2(bf2(mul2(xv, cv))), unbf2(bf2(mul2(xp, sv)))));
          memcpy(&yo[e], &yb, 4);
          memcpy(&xo[e], &xb, 4);
        }
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
          const float xp = lane < 16 ? -other : other;
          float y;
          if (rope_mode == 0) y = __fadd_rn(__fmul_rn(x[e], cs[e]), __fmul_rn(xp, sn[e]));
          else y = __fadd_rn(Num<T>::round(__fmul_rn(x[e], cs[e])), Num<T>::round(__fmul_rn(xp, sn[e])));
          yo[e] = Num<T>::from_f(y);
          xo[e] = Num<T>::from_f(x[e]);
        }
      }
      if (is_q) {
        st_vec<T, EPL>(q_out + (bt * H + r) * Dh + d0, yo);
      } else {
        const int64_t kr = (((int64_t)b * KVH + kvh) * kv_cap + kv_row0 + t) * Dh + d0;
        st_vec<T, EPL>(krope_out + kr, yo);
        st_vec<T, EPL>(kraw_out + kr, xo);
      }
    }
  }
  // V rows: layout transform only, all loads first
  T vin[8][EPL];
  for (int v0 = 0; v0 < KVH; v0 += 8) {
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (v0 + u < KVH) ld_vec<T, EPL>(src + (int64_t)(nqk + v0 + u) * Dh, vin[u]);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (v0 + u < KVH)
        st_vec<T, EPL>(v_out + (((int64_t)b * KVH + v0 + u) * kv_cap + kv_row0 + t) * Dh + d0, vin[u]);
  }
}

cudaError_t launch_prologue(const hga_params& p, int64_t S, const void* qkv, int64_t row_stride, const void* qw,
                            const void* kw, float eps, int norm_mode, const void* cos, const void* sin,
                            int rope_mode, int64_t rot_row0, int64_t pos0, void* q_out, void* kraw_out,
                            void* krope_out, void* v_out, int64_t kv_cap, int64_t kv_row0, cudaStream_t st) {
  const int64_t rows = (int64_t)p.batch * S * (p.nhead + 2 * p.kv_heads);
  const int64_t blocks = (rows + kProWarps - 1) / kProWarps;
  const size_t smem = (size_t)kProWarps * p.head_dim * sizeof(float);
  const int64_t tok_blocks = ((int64_t)p.batch * S + kProWarps - 1) / kProWarps;
#define HGA_PRO_VEC(T, EPL)                                                                                     \
  prologue_tok_kernel<T, EPL><<<(unsigned)tok_blocks, kProWarps * 32, 0, st>>>(                                \
      p, S, (const T*)qkv, row_stride, (const T*)qw, (const T*)kw, eps, norm_mode, cos, sin, rope_mode, rot_row0, \
      pos0, (T*)q_out, (T*)kraw_out, (T*)krope_out, (T*)v_out, kv_cap, kv_row0);                                \
  return cudaGetLastError();
  if (p.head_dim == 128 || p.head_dim == 64) {
    switch (p.dtype) {
      case HGA_DTYPE_F32:
        if (p.head_dim == 128) { HGA_PRO_VEC(float, 4) } else { HGA_PRO_VEC(float, 2) }
      case HGA_DTYPE_BF16:
        if (p.head_dim == 128) { HGA_PRO_VEC(__nv_bfloat16, 4) } else { HGA_PRO_VEC(__nv_bfloat16, 2) }
      case HGA_DTYPE_F16:
        if (p.head_dim == 128) { HGA_PRO_VEC(__half, 4) } else { HGA_PRO_VEC(__half, 2) }
    }
  }
#undef HGA_PRO_VEC
#define HGA_PRO(T)                                                                                              \
  prologue_kernel<T><<<(unsigned)blocks, kProWarps * 32, smem, st>>>(                                          \
      p, S, (const T*)qkv, row_stride, (const T*)qw, (const T*)kw, eps, norm_mode, cos, sin, rope_mode, rot_row0, \
      pos0, (T*)q_out, (T*)kraw_out, (T*)krope_out, (T*)v_out, kv_cap, kv_row0);                                \
  return cudaGetLastError();
  switch (p.dtype) {
    case HGA_DTYPE_F32: HGA_PRO(float)
    case HGA_DTYPE_BF16: HGA_PRO(__nv_bfloat16)
    case HGA_DTYPE_F16: HGA_PRO(__half)
  }
#undef HGA_PRO
  return cudaErrorInvalidValue;
}

}  // namespace hga
