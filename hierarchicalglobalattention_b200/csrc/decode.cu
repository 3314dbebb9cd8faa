// Incremental (single active chunk) routing + attention: ChunkRouter.decode_block
// (ExistingModelFineTuning/KvRouter/chunk_router.py:188-407) on device, for a batch whose
// sequences may sit at different positions (seq_pos[b] = absolute position of the block's first
// new token; the block of L tokens stays inside one chunk).
//
// Routing (chunk_router.py:210-277), per (b, query head h):
//   pool      = closed chunks [f_hi, l_lo) between the keep_first / keep_last windows
//   sc[t][c]  = T(T(q_t . chunk_k[c]) * scale)
//   chunks    = top-Kc of pooled[c] = max_t sc[t][c]            Kc = min(topk_chunks, |pool|)
//   requests  = each row's own top-Kc;  t0(chunk) = first requesting row
//   prev      = chunk n_closed-1 forced in (replacing the lowest pooled score) when in the pool,
//               visible to every row
//   groups    = top-Kg of max_t scg[t][j] over the chosen chunks' groups (not masked)
//   requests  = each row's top-Kg_request groups; t0(group) = max(first requesting row, parent t0)
// Attention (chunk_router.py:336-401 + RoutedKV.attend flat branch :159-162): fp32 online softmax
// over first window, last window, opened groups (rows >= t0) and the active chunk (key u visible to
// row t iff u <= c0 + t, c0 = seq_pos % C).
#include "select.cuh"

namespace hga {

HGA_DEVICE_ERROR_WORD(g_decode_error, decode_error_status)

constexpr int kDecThreads = 256;
constexpr int kDecTile = 64;

template <typename T>
__global__ void __launch_bounds__(kDecThreads) route_decode_kernel(
    hga_params p, int L, const T* __restrict__ q, const int32_t* __restrict__ seq_pos, const T* __restrict__ chunk_k,
    const T* __restrict__ group_k, int64_t sum_cap, int Kcmax, int Kgmax, int32_t* __restrict__ mid_chunk,
    int32_t* __restrict__ mid_t0, int32_t* __restrict__ open_gid, int32_t* __restrict__ open_t0, int nmid_max) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int h = blockIdx.x, b = blockIdx.y;
  const int H = p.nhead, KVH = p.kv_heads, Dh = p.head_dim, C = p.chunk_size, M = C / p.group_size;
  const int kvh = h / (H / KVH);
  const int tid = threadIdx.x;
  const int pos = seq_pos[b];
  const int n_closed = pos / C;
  int f_hi, l_lo;
  windows(n_closed, p.keep_first, p.keep_last, f_hi, l_lo);
  const int n_mid = l_lo > f_hi ? l_lo - f_hi : 0;
  const size_t bh = (size_t)b * H + h;
  for (int i = tid; i < Kcmax; i += blockDim.x) { mid_chunk[bh * Kcmax + i] = -1; mid_t0[bh * Kcmax + i] = -1; }
  for (int i = tid; i < Kgmax; i += blockDim.x) { open_gid[bh * Kgmax + i] = -1; open_t0[bh * Kgmax + i] = -1; }
  if (n_mid == 0 || p.topk_chunks <= 0) return;
  if ((int64_t)l_lo > sum_cap || n_mid > nmid_max) {
    if (tid == 0) atomicCAS(&g_decode_error, 0, kErrBoundsRouteDecode);
    return;
  }
  const int Kc = p.topk_chunks < n_mid ? p.topk_chunks : n_mid;
  const int G = Kc * M;
  const int Kg = p.topk_groups > 0 ? (p.topk_groups < G ? p.topk_groups : G) : 0;
  const int Kgr = p.topk_groups > 0 ? ((p.topk_groups / 2) < G ? p.topk_groups / 2 : G) : 0;
  const int nsub = (kDecThreads / L) < 8 ? (kDecThreads / L < 1 ? 1 : kDecThreads / L) : 8;

  // smem carve-up (float / u32 / u64 / int regions)
  const int ld = Dh + 1;
  float* qs = (float*)smem;                               // [L][ld]
  float* ks = qs + L * ld;                                // [kDecTile or G][ld]
  const int krows = kDecTile > G ? kDecTile : G;
  float* sc = ks + krows * ld;                            // [L][max(kDecTile, G)]
  const int scw = kDecTile > G ? kDecTile : G;
  uint32_t* pooled = (uint32_t*)(sc + L * scw);           // [nmid_max]
  int* t0c = (int*)(pooled + nmid_max);                   // [nmid_max]
  unsigned char* flag = (unsigned char*)(t0c + nmid_max); // [max(nmid_max, G)] (reused for groups)
  const int nflag = nmid_max > G ? nmid_max : G;
  unsigned long long* lists = (unsigned long long*)(((uintptr_t)(flag + nflag + 256) + 15) & ~(uintptr_t)15);
  // per-row request lists [L][nsub][Kc]; after level 1, reused as group request keys [L][G] u32
  const size_t list_words = (size_t)L * nsub * Kc > ((size_t)L * G + 1) / 2 ? (size_t)L * nsub * Kc
                                                                              : ((size_t)L * G + 1) / 2;
  int* red = (int*)(lists + list_words + 16);             // [16]
  int* sel = red + 16;                                    // [Kc]
  int* selt0 = sel + Kc;                                  // [Kc]
  uint32_t* gkeys = (uint32_t*)lists;                     // [L][G]   (after level 1)
  uint32_t* gpool = (uint32_t*)(selt0 + Kc);              // [G]
  int* greq0 = (int*)(gpool + G);                         // [G] first requesting row

  for (int i = tid; i < L * Dh; i += blockDim.x) {
    const int t = i / Dh, d = i % Dh;
    qs[t * ld + d] = Num<T>::to_f(q[((bh * L) + t) * Dh + d]);
  }
  for (int i = tid; i < n_mid; i += blockDim.x) { pooled[i] = 0u; t0c[i] = 0x7fffffff; }
  for (int i = tid; i < L * nsub * Kc; i += blockDim.x) lists[i] = 0ull;
  __syncthreads();
  // ---- level 1 ----------------------------------------------------------------------------
  const T* ckb = chunk_k + ((size_t)b * KVH + kvh) * sum_cap * Dh;
  for (int c0 = 0; c0 < n_mid; c0 += kDecTile) {
    const int nt = (n_mid - c0) < kDecTile ? (n_mid - c0) : kDecTile;
    for (int i = tid; i < nt * Dh; i += blockDim.x) {
      const int r = i / Dh, d = i % Dh;
      ks[r * ld + d] = Num<T>::to_f(ckb[(size_t)(f_hi + c0 + r) * Dh + d]);
    }
    __syncthreads();
    for (int i = tid; i < L * nt; i += blockDim.x) {
      const int t = i / nt, r = i % nt;
      float acc = 0.f;
      for (int d = 0; d < Dh; ++d) acc = fmaf(qs[t * ld + d], ks[r * ld + d], acc);
      const float s = ref_score<T>(acc, p.scale);
      sc[t * scw + r] = s;
      atomicMax(&pooled[c0 + r], ord_f32(s));
    }
    __syncthreads();
    for (int w = tid; w < L * nsub; w += blockDim.x) {
      const int t = w / nsub, sub = w % nsub;
      unsigned long long* lst = lists + (size_t)w * Kc;
      for (int r = sub; r < nt; r += nsub) list_insert(lst, Kc, rank_key(sc[t * scw + r], (uint32_t)(c0 + r)));
    }
    __syncthreads();
  }
  // per-row requests -> first requesting row
  for (int t = tid; t < L; t += blockDim.x) {
    unsigned long long* base = lists + (size_t)t * nsub * Kc;
    int ptr[8];
    for (int s = 0; s < nsub; ++s) ptr[s] = 0;
    for (int r = 0; r < Kc; ++r) {
      int best = -1;
      unsigned long long bk = 0ull;
      for (int s = 0; s < nsub; ++s)
        if (ptr[s] < Kc) {
          const unsigned long long kk = base[s * Kc + ptr[s]];
          if (kk > bk) { bk = kk; best = s; }
        }
      if (best < 0) break;
      ptr[best]++;
      atomicMin(&t0c[rank_idx(bk)], t);
    }
  }
  __syncthreads();
  block_select(pooled, n_mid, Kc, flag, red);
  const int prev = n_closed - 1;
  if (tid == 0) {
    if (prev >= f_hi && prev < l_lo) {
      const int pr = prev - f_hi;
      if (!flag[pr]) {  // drop the lowest pooled chosen chunk (highest index among equals)
        int worst = -1;
        for (int i = 0; i < n_mid; ++i)
          if (flag[i] && (worst < 0 || pooled[i] <= pooled[worst])) worst = i;
        if (worst >= 0) flag[worst] = 0;
        flag[pr] = 1;
      }
      t0c[pr] = 0;
    }
    int k = 0;
    for (int i = 0; i < n_mid; ++i)
      if (flag[i]) { sel[k] = f_hi + i; selt0[k] = t0c[i] < L ? t0c[i] : L; ++k; }
    red[8] = k;
  }
  __syncthreads();
  const int ksel = red[8];
  for (int i = tid; i < ksel; i += blockDim.x) {
    mid_chunk[bh * Kcmax + i] = sel[i];
    mid_t0[bh * Kcmax + i] = selt0[i] < L ? selt0[i] : -1;
  }
  if (Kg <= 0) return;
  // ---- level 2 (candidates are not masked; visibility needs the parent) ----------------------
  const int Gs = ksel * M;
  const T* gkb = group_k + ((size_t)b * KVH + kvh) * sum_cap * M * Dh;
  for (int i = tid; i < Gs * Dh; i += blockDim.x) {
    const int j = i / Dh, d = i % Dh;
    ks[j * ld + d] = Num<T>::to_f(gkb[((size_t)sel[j / M] * M + (j % M)) * Dh + d]);
  }
  for (int j = tid; j < Gs; j += blockDim.x) { gpool[j] = 0u; greq0[j] = 0x7fffffff; }
  __syncthreads();
  for (int i = tid; i < L * Gs; i += blockDim.x) {
    const int t = i / Gs, j = i % Gs;
    float acc = 0.f;
    for (int d = 0; d < Dh; ++d) acc = fmaf(qs[t * ld + d], ks[j * ld + d], acc);
    const float s = ref_score<T>(acc, p.scale);
    gkeys[t * Gs + j] = ord_f32(s);
    atomicMax(&gpool[j], ord_f32(s));
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  if (Kgr > 0) {
    for (int t = warp; t < L; t += blockDim.x / 32) {
      unsigned char* fl = flag + 0;  // per-warp scratch would be cleaner; rows are serialized per warp
      (void)fl;
      // per-row request set: top-Kgr keys (all when Kgr >= Gs)
      // reuse sc rows as flags storage
      unsigned char* rf = (unsigned char*)(sc + t * scw);
      warp_select(gkeys + t * Gs, Gs, Kgr, rf);
      for (int j = lane; j < Gs; j += 32)
        if (rf[j]) atomicMin(&greq0[j], t);
    }
  }
  __syncthreads();
  block_select(gpool, Gs, Kg, flag, red);
  if (tid == 0) {
    int k = 0;
    for (int j = 0; j < Gs; ++j) {
      if (!flag[j] || greq0[j] == 0x7fffffff) continue;
      const int tp = selt0[j / M];
      const int t0 = greq0[j] > tp ? greq0[j] : tp;
      if (t0 >= L) continue;
      open_gid[bh * Kgmax + k] = sel[j / M] * M + (j % M);
      open_t0[bh * Kgmax + k] = t0;
      ++k;
    }
  }
}

// Key source of the decode attention: closed-chunk rows come from `cold` (the complete token
// record: HBM for the VRAM tier, mapped pinned host memory for the RAM tier) unless they belong to
// a window or to the active chunk, which always come from `hot` (HBM).
//   hot_mode 0: hot rows are addressed like cold rows (hot == cold, the VRAM tier)
//   hot_mode 1: hot is a slot buffer: first-window chunk c -> slot c, last-window chunk c ->
//               slot kf + c % kl, active chunk -> slot kf + kl
__device__ __forceinline__ int64_t hot_row(int chunk, int u, int C, int mode, int kf, int kl, bool active) {
  if (mode == 0) return (int64_t)chunk * C + u;
  const int slot = active ? kf + kl : (chunk < kf ? chunk : kf + chunk % (kl > 0 ? kl : 1));
  return (int64_t)slot * C + u;
}

// Dual Chunk Attention (DCA = true; the Qwen3 wrapper's dca_chunk > 0 attention,
// ExistingModelFineTuning/Qwen3LongContext/qwen_routed_attention.py:247-283): q holds the
// un-roped queries and every query row is roped three ways in fp32 from the tables dca_cos /
// dca_sin [dca_ceil + 1][Dh] (rows = remapped positions): intra at qp = (pos + t) % dca_chunk,
// successor at min(qp + dca_chunk, dca_ceil), inter at dca_ceil.  A key scores against the intra
// query when it lies in the query's DCA chunk, the successor one in the chunk just before, else
// the inter one.  Key positions come from the key layout (windows and the active chunk) and, for
// opened groups, from open_pos (the routing's group ids; it differs from open_gid when the cold
// rows are addressed by bank slot).  The reference fills masked scores with -1e4 instead of
// excluding them; every row sees at least its own token, so those terms are exp(<= -1e4 + O(score))
// = 0 in fp32 and exclusion is the same softmax.
struct DcaArgs {
  const float* cos;
  const float* sin;
  int chunk, ceil;
  const int32_t* open_pos;
};

template <typename T, bool DCA>
__global__ void __launch_bounds__(128) attend_decode_kernel(
    hga_params p, int Lfull, int Lt, const T* __restrict__ q, const int32_t* __restrict__ seq_pos,
    const T* __restrict__ hot_k, const T* __restrict__ hot_v, int64_t hot_cap, int hot_mode, const T* cold_k,
    const T* cold_v, int64_t cold_cap, const int32_t* __restrict__ open_gid, const int32_t* __restrict__ open_t0, int Kg,
    T* __restrict__ out, DcaArgs dca) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int h = blockIdx.x, b = blockIdx.y;
  // rows [row0, row0 + L) of the block (a row tile per blockIdx.z when the block's rows do not fit
  // one CTA's shared memory)
  const int row0 = blockIdx.z * Lt, L = min(Lt, Lfull - row0);
  const int H = p.nhead, KVH = p.kv_heads, Dh = p.head_dim, C = p.chunk_size, gs = p.group_size;
  const int kvh = h / (H / KVH);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = 4;
  const int pos = seq_pos[b];
  const int n_closed = pos / C, c0 = pos % C;
  const int kf = p.keep_first > 0 ? p.keep_first : 0, kl = p.keep_last > 0 ? p.keep_last : 0;
  int f_hi, l_lo;
  windows(n_closed, kf, kl, f_hi, l_lo);
  const size_t bh = (size_t)b * H + h;
  const size_t qoff = (bh * Lfull + row0) * Dh;
  const bool hot_oob = hot_mode == 0 ? (int64_t)(n_closed + 1) * C > hot_cap : (int64_t)(kf + kl + 1) * C > hot_cap;
  if (hot_oob || (hot_mode == 0 && (int64_t)n_closed * C > cold_cap)) {
    if (tid == 0) atomicCAS(&g_decode_error, 0, kErrBoundsAttendDecode);
    for (int i = tid; i < L * Dh; i += blockDim.x) out[qoff + i] = Num<T>::from_f(0.f);
    return;
  }
  // key segments: (source 0 hot / 1 cold, chunk, first row, length, tmin, causal offset)
  const int ld = Dh + 1;
  constexpr int NQ = DCA ? 3 : 1;
  float* qs = (float*)smem;                 // [NQ][L][ld] (DCA: intra, successor, inter ropings)
  float* ks = qs + NQ * L * ld;             // [32][ld]
  float* vs = ks + 32 * ld;                 // [32][ld]
  float* os = vs + 32 * ld;                 // [nw][L][Dh] per-warp partial outputs
  float* ms = os + nw * L * Dh;             // [nw][L]
  float* ls = ms + nw * L;                  // [nw][L]
  float* pw = ls + nw * L;                  // [nw][32]
  int* kinfo = (int*)(pw + nw * 32);        // [32][4]: source, row, tmin, absolute position
  const int nfirst = f_hi * C, nlast = (n_closed - l_lo) * C, nact = c0 + row0 + L;
  int nopen = 0;
  for (int j = 0; j < Kg; ++j) nopen += (open_gid[bh * Kg + j] >= 0 && open_t0[bh * Kg + j] >= 0);
  const int nkeys = nfirst + nlast + nopen * gs + nact;
  if constexpr (DCA) {
    // x * cos + rotate_half(x) * sin, each product and the sum rounded to fp32 like the reference
    const int half = Dh / 2;
    for (int i = tid; i < L * Dh; i += blockDim.x) {
      const int t = i / Dh, d = i % Dh;
      const float x = Num<T>::to_f(q[qoff + i]);
      const float y = Num<T>::to_f(q[qoff + t * Dh + (d < half ? d + half : d - half)]);
      const float r = d < half ? -y : y;
      const int qp = (pos + row0 + t) % dca.chunk;
      const int rows[3] = {qp, min(qp + dca.chunk, dca.ceil), dca.ceil};
#pragma unroll
      for (int v = 0; v < 3; ++v) {
        const float c = dca.cos[(size_t)rows[v] * Dh + d], sn = dca.sin[(size_t)rows[v] * Dh + d];
        qs[(v * L + t) * ld + d] = __fadd_rn(__fmul_rn(x, c), __fmul_rn(r, sn));
      }
    }
  } else {
    for (int i = tid; i < L * Dh; i += blockDim.x) qs[(i / Dh) * ld + i % Dh] = Num<T>::to_f(q[qoff + i]);
  }
  for (int i = tid; i < nw * L * Dh; i += blockDim.x) os[i] = 0.f;
  for (int i = tid; i < nw * L; i += blockDim.x) { ms[i] = -INFINITY; ls[i] = 0.f; }
  __syncthreads();
  const size_t hot_base = ((size_t)b * KVH + kvh) * hot_cap;
  const size_t cold_base = ((size_t)b * KVH + kvh) * cold_cap;
  for (int k0 = 0; k0 < nkeys; k0 += 32) {
    if (tid < 32) {
      const int k = k0 + tid;
      int src = 0, tmin = 1 << 30, kpos = 0;
      int64_t row = 0;
      if (k < nkeys) {
        if (k < nfirst) {
          row = hot_row(k / C, k % C, C, hot_mode, kf, kl, false); tmin = 0; kpos = k;
        } else if (k < nfirst + nlast) {
          const int kk = k - nfirst;
          row = hot_row(l_lo + kk / C, kk % C, C, hot_mode, kf, kl, false); tmin = 0; kpos = l_lo * C + kk;
        } else if (k < nfirst + nlast + nopen * gs) {
          const int kk = k - nfirst - nlast;
          // the opened entries are a prefix of the list
          const int j = kk / gs;
          row = (int64_t)open_gid[bh * Kg + j] * gs + kk % gs; tmin = open_t0[bh * Kg + j]; src = 1;
          if constexpr (DCA) kpos = dca.open_pos[bh * Kg + j] * gs + kk % gs;
          if (row >= cold_cap) {  // a list entry past the record: skipped (never visible)
            atomicCAS(&g_decode_error, 0, kErrBoundsAttendDecode);
            row = 0; tmin = 1 << 30;
          }
        } else {
          const int u = k - nfirst - nlast - nopen * gs;
          row = hot_row(n_closed, u, C, hot_mode, kf, kl, true); tmin = u - c0; kpos = n_closed * C + u;
        }
      }
      kinfo[tid * 4 + 0] = src;
      kinfo[tid * 4 + 1] = (int)row;
      kinfo[tid * 4 + 2] = tmin;
      kinfo[tid * 4 + 3] = kpos;
    }
    __syncthreads();
    for (int i = tid; i < 32 * Dh; i += blockDim.x) {
      const int r = i / Dh, d = i % Dh;
      const size_t off = (kinfo[r * 4] ? cold_base : hot_base) + (size_t)kinfo[r * 4 + 1];
      const T* kp = kinfo[r * 4] ? cold_k : hot_k;
      const T* vp = kinfo[r * 4] ? cold_v : hot_v;
      const bool ok = k0 + r < nkeys;
      ks[r * ld + d] = ok ? Num<T>::to_f(kp[off * Dh + d]) : 0.f;
      vs[r * ld + d] = ok ? Num<T>::to_f(vp[off * Dh + d]) : 0.f;
    }
    __syncthreads();
    // each warp takes a subset of the tile's 32 keys (split-K inside the CTA) for every row
    for (int t = 0; t < L; ++t) {
      const int key = lane;  // lane j scores key j; warp w only keeps keys j % nw == w
      const bool mine = (key % nw) == warp;
      const bool vis = mine && (k0 + key < nkeys) && row0 + t >= kinfo[key * 4 + 2];
      float s = -INFINITY;
      if (vis) {
        int qv = 0;
        if constexpr (DCA) {
          const int cq = (pos + row0 + t) / dca.chunk, ck = kinfo[key * 4 + 3] / dca.chunk;
          qv = ck == cq ? 0 : (ck == cq - 1 ? 1 : 2);
        }
        const float* qrow = qs + (qv * L + t) * ld;
        float acc = 0.f;
        for (int d = 0; d < Dh; ++d) acc = fmaf(qrow[d], ks[key * ld + d], acc);
        s = acc * p.scale;
      }
      float mx = s;
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = ms[warp * L + t];
      const float m_new = fmaxf(m_old, mx);
      if (m_new == -INFINITY) continue;
      const float alpha = __expf(m_old - m_new);
      const float pj = vis ? __expf(s - m_new) : 0.f;
      float psum = pj;
      for (int o = 16; o; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      pw[warp * 32 + lane] = pj;
      __syncwarp();
      float* orow = os + (warp * L + t) * Dh;
      for (int d = lane; d < Dh; d += 32) {
        float acc = orow[d] * alpha;
        for (int j = warp; j < 32; j += nw) acc = fmaf(pw[warp * 32 + j], vs[j * ld + d], acc);
        orow[d] = acc;
      }
      __syncwarp();
      if (lane == 0) { ms[warp * L + t] = m_new; ls[warp * L + t] = ls[warp * L + t] * alpha + psum; }
      __syncwarp();
    }
    __syncthreads();
  }
  // merge the warps' partial softmax states
  for (int i = tid; i < L * Dh; i += blockDim.x) {
    const int t = i / Dh, d = i % Dh;
    float m = -INFINITY;
    for (int w = 0; w < nw; ++w) m = fmaxf(m, ms[w * L + t]);
    float l = 0.f, o = 0.f;
    for (int w = 0; w < nw; ++w) {
      if (ms[w * L + t] == -INFINITY) continue;
      const float f = __expf(ms[w * L + t] - m);
      l += ls[w * L + t] * f;
      o += os[(w * L + t) * Dh + d] * f;
    }
    out[qoff + i] = Num<T>::from_f(l > 0.f ? o / l : 0.f);
  }
}

// Append L new rows per sequence (k_rope / v, and k_raw of the active chunk) at seq_pos[b].
template <typename T>
__global__ void append_kernel(hga_params p, int L, const int32_t* __restrict__ seq_pos, const T* __restrict__ k_rope,
                              const T* __restrict__ v, const T* __restrict__ k_raw, T* hot_k, T* hot_v, int64_t hot_cap,
                              int hot_mode, T* cold_k, T* cold_v, int64_t cold_cap, T* act_raw) {
  const int Dh = p.head_dim, C = p.chunk_size, KVH = p.kv_heads;
  const int kf = p.keep_first > 0 ? p.keep_first : 0, kl = p.keep_last > 0 ? p.keep_last : 0;
  const int64_t total = (int64_t)p.batch * KVH * L * Dh;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % Dh);
    const int64_t r = i / Dh;
    const int l = (int)(r % L);
    const int bk = (int)(r / L);
    const int b = bk / KVH;
    const int pos = seq_pos[b] + l;
    const int n = pos / C, u = pos % C;
    const T kr = k_rope[i], vv = v[i];
    const int64_t hr = hot_row(n, u, C, hot_mode, kf, kl, true);
    if (hr >= hot_cap || (hot_mode != 0 && cold_k && pos >= cold_cap)) {
      atomicCAS(&g_decode_error, 0, kErrBoundsAppend);
      continue;
    }
    hot_k[((int64_t)bk * hot_cap + hr) * Dh + d] = kr;
    hot_v[((int64_t)bk * hot_cap + hr) * Dh + d] = vv;
    if (hot_mode != 0 && cold_k) {
      cold_k[((int64_t)bk * cold_cap + pos) * Dh + d] = kr;
      cold_v[((int64_t)bk * cold_cap + pos) * Dh + d] = vv;
    }
    if (act_raw) act_raw[((int64_t)bk * C + u) * Dh + d] = k_raw[i];
  }
}

size_t route_decode_smem(const hga_params& p, int L, int nmid_max, int Kc, int G) {
  const int Dh = p.head_dim, ld = Dh + 1;
  const int krows = kDecTile > G ? kDecTile : G, scw = kDecTile > G ? kDecTile : G;
  int nsub = kDecThreads / L;
  nsub = nsub < 1 ? 1 : (nsub > 8 ? 8 : nsub);
  size_t f = (size_t)L * ld + (size_t)krows * ld + (size_t)L * scw;
  size_t bytes = f * 4 + (size_t)nmid_max * 8 + (size_t)(nmid_max > G ? nmid_max : G) + 256 + 32;
  size_t lists = (size_t)L * nsub * (Kc > 0 ? Kc : 1) * 8;
  const size_t gk = (size_t)L * G * 4;
  bytes += (lists > gk ? lists : gk) + 16 * 8 + 64 + 2 * (size_t)(Kc + 1) * 4 + (size_t)G * 8 + 64;
  return bytes;
}

#define HGA_DISPATCH(dt, FN, ...)                                        \
  switch (dt) {                                                          \
    case HGA_DTYPE_F32: return FN<float>(__VA_ARGS__);                   \
    case HGA_DTYPE_BF16: return FN<__nv_bfloat16>(__VA_ARGS__);          \
    case HGA_DTYPE_F16: return FN<__half>(__VA_ARGS__);                  \
  }                                                                      \
  return cudaErrorInvalidValue;

template <typename T>
static cudaError_t launch_route_decode_t(const hga_params& p, int L, const void* q, const int32_t* seq_pos,
                                         const void* ck, const void* gk, int64_t sum_cap, int nmid_max, int Kcmax,
                                         int Kgmax, int32_t* mc, int32_t* mt, int32_t* og, int32_t* ot,
                                         cudaStream_t st) {
  const int M = p.chunk_size / p.group_size;
  const size_t smem = route_decode_smem(p, L, nmid_max, Kcmax, Kcmax * M);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  auto kern = route_decode_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.nhead, p.batch);
  kern<<<grid, kDecThreads, smem, st>>>(p, L, (const T*)q, seq_pos, (const T*)ck, (const T*)gk, sum_cap, Kcmax, Kgmax,
                                        mc, mt, og, ot, nmid_max);
  return cudaGetLastError();
}

cudaError_t launch_route_decode(const hga_params& p, int L, const void* q, const int32_t* seq_pos, const void* ck,
                                const void* gk, int64_t sum_cap, int nmid_max, int Kcmax, int Kgmax, int32_t* mc,
                                int32_t* mt, int32_t* og, int32_t* ot, cudaStream_t st) {
  HGA_DISPATCH(p.dtype, launch_route_decode_t, p, L, q, seq_pos, ck, gk, sum_cap, nmid_max, Kcmax, Kgmax, mc, mt, og,
               ot, st)
}

template <typename T>
static cudaError_t launch_attend_decode_t(const hga_params& p, int L, const void* q, const int32_t* seq_pos,
                                          const void* hk, const void* hv, int64_t hot_cap, int hot_mode, const void* ckk,
                                          const void* cvv, int64_t cold_cap, const int32_t* og, const int32_t* ot,
                                          int Kg, void* out, const DcaArgs* dca, cudaStream_t st) {
  const int ld = p.head_dim + 1, nw = 4, nq = dca ? 3 : 1;
  auto smem_of = [&](int lt) {
    return ((size_t)nq * lt * ld + 64 * ld + (size_t)nw * lt * p.head_dim + 2 * nw * lt + nw * 32) * 4 + 32 * 4 * 4 +
           64;
  };
  int Lt = L;  // rows per CTA: the whole block unless its rows need more than 227 KB
  while (Lt > 1 && smem_of(Lt) > 227 * 1024) Lt = (Lt + 1) / 2;
  const size_t smem = smem_of(Lt);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  auto kern = dca ? attend_decode_kernel<T, true> : attend_decode_kernel<T, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.nhead, p.batch, (L + Lt - 1) / Lt);
  kern<<<grid, 128, smem, st>>>(p, L, Lt, (const T*)q, seq_pos, (const T*)hk, (const T*)hv, hot_cap, hot_mode,
                                (const T*)ckk, (const T*)cvv, cold_cap, og, ot, Kg, (T*)out,
                                dca ? *dca : DcaArgs{nullptr, nullptr, 1, 0, nullptr});
  return cudaGetLastError();
}

cudaError_t launch_attend_decode(const hga_params& p, int L, const void* q, const int32_t* seq_pos, const void* hk,
                                 const void* hv, int64_t hot_cap, int hot_mode, const void* ckk, const void* cvv,
                                 int64_t cold_cap, const int32_t* og, const int32_t* ot, int Kg, void* out,
                                 cudaStream_t st) {
  HGA_DISPATCH(p.dtype, launch_attend_decode_t, p, L, q, seq_pos, hk, hv, hot_cap, hot_mode, ckk, cvv, cold_cap, og,
               ot, Kg, out, nullptr, st)
}

cudaError_t launch_attend_decode_dca(const hga_params& p, int L, const void* q, const int32_t* seq_pos, const void* hk,
                                     const void* hv, int64_t hot_cap, int hot_mode, const void* ckk, const void* cvv,
                                     int64_t cold_cap, const int32_t* og, const int32_t* ot, const int32_t* open_pos,
                                     int Kg, const float* dca_cos, const float* dca_sin, int dca_chunk, int dca_ceil,
                                     void* out, cudaStream_t st) {
  const DcaArgs a{dca_cos, dca_sin, dca_chunk, dca_ceil, open_pos ? open_pos : og};
  HGA_DISPATCH(p.dtype, launch_attend_decode_t, p, L, q, seq_pos, hk, hv, hot_cap, hot_mode, ckk, cvv, cold_cap, og,
               ot, Kg, out, &a, st)
}

template <typename T>
static cudaError_t launch_append_t(const hga_params& p, int L, const int32_t* seq_pos, const void* kr, const void* v,
                                   const void* kraw, void* hk, void* hv, int64_t hot_cap, int hot_mode, void* ck,
                                   void* cv, int64_t cold_cap, void* act_raw, cudaStream_t st) {
  const int64_t total = (int64_t)p.batch * p.kv_heads * L * p.head_dim;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  append_kernel<T><<<blocks, 256, 0, st>>>(p, L, seq_pos, (const T*)kr, (const T*)v, (const T*)kraw, (T*)hk, (T*)hv,
                                           hot_cap, hot_mode, (T*)ck, (T*)cv, cold_cap, (T*)act_raw);
  return cudaGetLastError();
}

cudaError_t launch_append(const hga_params& p, int L, const int32_t* seq_pos, const void* kr, const void* v,
                          const void* kraw, void* hk, void* hv, int64_t hot_cap, int hot_mode, void* ck, void* cv,
                          int64_t cold_cap, void* act_raw, cudaStream_t st) {
  HGA_DISPATCH(p.dtype, launch_append_t, p, L, seq_pos, kr, v, kraw, hk, hv, hot_cap, hot_mode, ck, cv, cold_cap,
               act_raw, st)
}

}  // namespace hga
