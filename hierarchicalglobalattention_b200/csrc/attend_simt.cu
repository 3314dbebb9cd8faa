// Portable working-set attention (SIMT, any dtype / head_dim <= 256 / chunk_size <= 128).
//
// Query row t of query chunk n attends, with an fp32 online softmax, to the key segments that
// the reference concatenates in vectorized.py:404-490 and scores in RoutedKV.attend
// (chunk_router.py:149-158):
//   current chunk  [n*C, n*C+len)    row t sees local key u iff u <= t (causal)
//   last window    [l_lo*C, n*C)     all rows
//   first window   [0, f_hi*C)       all rows
//   opened group g [g*gs, g*gs+gs)   rows t >= t0[g]
// Every key carries a "first visible row" threshold, so one comparison masks all segments.
// One CTA per (query chunk, head, batch): key/value tiles of 32 tokens are staged in smem once and
// shared by the 4 warps, each warp owning every 4th query row (row state lives in smem).
#include "hga_common.cuh"

namespace hga {

constexpr int kAttThreads = 128;
constexpr int kKeyTile = 32;

template <typename T>
__global__ void __launch_bounds__(kAttThreads) attend_simt_kernel(
    hga_params p, int64_t S, QRange qr, const T* __restrict__ q, int q_layout, const T* __restrict__ k_rope,
    const T* __restrict__ v, int64_t kv_cap, const int32_t* __restrict__ open_gid,
    const int32_t* __restrict__ open_t0, int Kg, int N, T* __restrict__ out, int out_layout) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int ln = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int n = qr.chunk0 + ln;
  const int H = p.nhead, KVH = p.kv_heads, Dh = p.head_dim, C = p.chunk_size, gs = p.group_size;
  const int kvh = h / (H / KVH);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ld = Dh + 1;
  const int nseg_max = 3 + Kg;
  // smem carve-up
  float* qs = (float*)smem;                       // [C][ld]
  float* ks = qs + C * ld;                        // [kKeyTile][ld]
  float* vs = ks + kKeyTile * ld;                 // [kKeyTile][ld]
  float* os = vs + kKeyTile * ld;                 // [C][Dh]
  float* ms = os + C * Dh;                        // [C]
  float* ls = ms + C;                             // [C]
  int* seg_start = (int*)(ls + C);                // [nseg_max]
  int* seg_tmin = seg_start + nseg_max;           // [nseg_max] (-1 => causal)
  int* seg_off = seg_tmin + nseg_max;             // [nseg_max + 1] prefix offsets
  int* kpos = seg_off + nseg_max + 1;             // [kKeyTile]
  int* ktmin = kpos + kKeyTile;                   // [kKeyTile]
  int* nseg_s = ktmin + kKeyTile;
  float* pw = (float*)(nseg_s + 4) + warp * kKeyTile;  // per-warp probabilities of the tile

  const int64_t row0 = (int64_t)n * C;
  const int nvalid = (int)((S - row0) < C ? (S - row0) : C);
  int f_hi, l_lo;
  windows(n, p.keep_first, p.keep_last, f_hi, l_lo);
  if (tid == 0) {
    int ns = 0, off = 0;
    seg_start[ns] = (int)row0; seg_tmin[ns] = -1; seg_off[ns] = off; off += nvalid; ++ns;
    if (n > l_lo) { seg_start[ns] = l_lo * C; seg_tmin[ns] = 0; seg_off[ns] = off; off += (n - l_lo) * C; ++ns; }
    if (f_hi > 0) { seg_start[ns] = 0; seg_tmin[ns] = 0; seg_off[ns] = off; off += f_hi * C; ++ns; }
    const size_t tile = ((size_t)b * H + h) * qr.count + ln;
    for (int j = 0; j < Kg; ++j) {
      const int g = open_gid[tile * Kg + j];
      const int t0 = open_t0[tile * Kg + j];
      if (g < 0 || t0 < 0 || t0 >= nvalid) continue;
      seg_start[ns] = g * gs; seg_tmin[ns] = t0; seg_off[ns] = off; off += gs; ++ns;
    }
    seg_off[ns] = off;
    *nseg_s = ns;
  }
  for (int i = tid; i < C * Dh; i += blockDim.x) {
    const int t = i / Dh, d = i % Dh;
    float x = 0.f;
    if (t < nvalid) {
      const int64_t tt = (int64_t)ln * C + t;  // local q row
      const T* src = q_layout == 0 ? q + (((int64_t)b * H + h) * qr.sq + tt) * Dh
                                   : q + (((int64_t)b * qr.sq + tt) * H + h) * Dh;
      x = Num<T>::to_f(src[d]);
    }
    qs[t * ld + d] = x;
    os[i] = 0.f;
  }
  for (int t = tid; t < C; t += blockDim.x) { ms[t] = -INFINITY; ls[t] = 0.f; }
  __syncthreads();
  const int nseg = *nseg_s;
  const int nkeys = seg_off[nseg];
  const size_t kvbase = (size_t)(b * KVH + kvh) * kv_cap * Dh;
  const float scale = p.scale;

  for (int k0 = 0; k0 < nkeys; k0 += kKeyTile) {
    if (tid < kKeyTile) {
      const int k = k0 + tid;
      int pos = 0, tmin = 0x7fffffff;
      if (k < nkeys) {
        int lo = 0, hi = nseg - 1;  // last seg with seg_off <= k
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (seg_off[mid] <= k) lo = mid; else hi = mid - 1;
        }
        const int u = k - seg_off[lo];
        pos = seg_start[lo] + u;
        tmin = seg_tmin[lo] < 0 ? u : seg_tmin[lo];
      }
      kpos[tid] = pos;
      ktmin[tid] = tmin;
    }
    __syncthreads();
    for (int i = tid; i < kKeyTile * Dh; i += blockDim.x) {
      const int r = i / Dh, d = i % Dh;
      const size_t off = kvbase + (size_t)kpos[r] * Dh + d;
      ks[r * ld + d] = Num<T>::to_f(k_rope[off]);
      vs[r * ld + d] = Num<T>::to_f(v[off]);
    }
    __syncthreads();
    for (int t = warp; t < nvalid; t += kAttThreads / 32) {
      const bool vis = t >= ktmin[lane];
      float s = -INFINITY;
      if (vis) {
        float acc = 0.f;
        const float* qa = qs + t * ld;
        const float* kb = ks + lane * ld;
        for (int d = 0; d < Dh; ++d) acc = fmaf(qa[d], kb[d], acc);
        s = acc * scale;
      }
      float mx = s;
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = ms[t];
      const float m_new = fmaxf(m_old, mx);
      if (m_new == -INFINITY) continue;  // nothing visible yet in this tile
      const float alpha = __expf(m_old - m_new);
      const float pj = vis ? __expf(s - m_new) : 0.f;
      float psum = pj;
      for (int o = 16; o; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      pw[lane] = pj;
      __syncwarp();
      for (int d = lane; d < Dh; d += 32) {
        float acc = os[t * Dh + d] * alpha;
        for (int j = 0; j < kKeyTile; ++j) acc = fmaf(pw[j], vs[j * ld + d], acc);
        os[t * Dh + d] = acc;
      }
      __syncwarp();
      if (lane == 0) { ms[t] = m_new; ls[t] = ls[t] * alpha + psum; }
      __syncwarp();
    }
    __syncthreads();
  }
  for (int i = tid; i < nvalid * Dh; i += blockDim.x) {
    const int t = i / Dh, d = i % Dh;
    const float val = os[i] / ls[t];
    const int64_t tt = (int64_t)ln * C + t;  // local output row
    T* dst = out_layout == 0 ? out + (((int64_t)b * H + h) * qr.sq + tt) * Dh
                             : out + (((int64_t)b * qr.sq + tt) * H + h) * Dh;
    dst[d] = Num<T>::from_f(val);
  }
}

static size_t attend_simt_smem(const hga_params& p, int Kg) {
  const int ld = p.head_dim + 1, C = p.chunk_size, Dh = p.head_dim;
  size_t f = (size_t)C * ld + 2 * kKeyTile * ld + (size_t)C * Dh + 2 * C;
  size_t ints = 3 * (size_t)(3 + Kg) + 1 + 2 * kKeyTile + 4;
  return f * 4 + ints * 4 + (kAttThreads / 32) * kKeyTile * 4 + 16;
}

template <typename T>
static cudaError_t launch_attend_simt_t(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout,
                                        const void* k_rope, const void* v, int64_t kv_cap,
                                        const int32_t* open_gid, const int32_t* open_t0, int Kg, void* out,
                                        int out_layout, cudaStream_t st) {
  const int N = (int)((S + p.chunk_size - 1) / p.chunk_size);
  const size_t smem = attend_simt_smem(p, Kg);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  auto kern = attend_simt_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(qr.count, p.nhead, p.batch);
  kern<<<grid, kAttThreads, smem, st>>>(p, S, qr, (const T*)q, q_layout, (const T*)k_rope, (const T*)v, kv_cap, open_gid,
                                        open_t0, Kg, N, (T*)out, out_layout);
  return cudaGetLastError();
}

cudaError_t launch_attend_simt(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout, const void* k_rope,
                               const void* v, int64_t kv_cap, const int32_t* open_gid, const int32_t* open_t0,
                               int Kg, void* out, int out_layout, cudaStream_t st) {
  switch (p.dtype) {
    case HGA_DTYPE_F32:
      return launch_attend_simt_t<float>(p, S, qr, q, q_layout, k_rope, v, kv_cap, open_gid, open_t0, Kg, out,
                                         out_layout, st);
    case HGA_DTYPE_BF16:
      return launch_attend_simt_t<__nv_bfloat16>(p, S, qr, q, q_layout, k_rope, v, kv_cap, open_gid, open_t0, Kg,
                                                 out, out_layout, st);
    case HGA_DTYPE_F16:
      return launch_attend_simt_t<__half>(p, S, qr, q, q_layout, k_rope, v, kv_cap, open_gid, open_t0, Kg, out,
                                          out_layout, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace hga
