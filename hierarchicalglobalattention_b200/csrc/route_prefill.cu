// Two-level router of the chunk-parallel prefill (ExistingModelFineTuning/KvRouter/vectorized.py:296-384).
//
// One CTA per (query chunk n, query head h, batch b).  The reference materialises the whole
// [B,H,N,C,N] score tensor; here a query chunk streams its routed pool [f_hi, l_lo) through shared
// memory in tiles and keeps, per query row, only its running top-Kc requests.
//
//   level 1:  s[t][c] = T(T(q_t . chunk_k[c]) * scale) over pool chunks c (vectorized.py:307-309)
//             R_t     = top-min(Kc, |pool|) of row t                      (_route_topk_requests)
//             pooled  = amax over rows t with c in R_t                    (_max_route_scores_from_requests)
//             chosen  = top-Kc of pooled (all requested when they fit)    (_topk_scores_indices)
//             prev    = chunk n-1 forced in when it lies in the pool      (vectorized.py:314-328)
//             t0[c]   = first row requesting c (0 for the forced prev)    (cumsum visibility, :330-337)
//   level 2:  candidates = groups of chosen chunks, real for row t iff t >= t0[chunk]
//             the same request / pool / select scheme with Kg_request = topk_groups // 2 and
//             Kg = topk_groups (vectorized.py:365-384); group t0 = first requesting row.
// Selections break ties by higher score, then lower index; the reference's order among equal
// scores is torch.topk's, which is implementation-defined.
#include "select.cuh"

namespace hga {

constexpr int kRouteThreads = 256;
constexpr int kTile = 64;  // pool chunks scored per smem tile

struct RouteSmem {
  // all offsets in bytes from the dynamic smem base
  int qs, ks, sc, lists, gkeys, gflag, pooled, t0c, selflag, sel, selt0, gt0, gpool, red;
  int total;
};

__host__ __device__ inline int align16(int x) { return (x + 15) & ~15; }

// q / key tiles are kept in the input dtype (row pitch Dh + 2 elements); level-1 scratch (score
// tile + per-row request lists) and level-2 scratch (per-row keys + flags) share one region.
__host__ __device__ inline RouteSmem route_smem_layout(int C, int Dh, int N, int Kc, int Tg, int nsub, int esz) {
  RouteSmem L;
  int o = 0;
  const int ldq = Dh + 2;
  L.qs = o;      o = align16(o + C * ldq * esz);
  const int krows = kTile > Tg ? kTile : Tg;
  L.ks = o;      o = align16(o + krows * ldq * esz);
  const int u0 = o;
  L.sc = o;      o = align16(o + C * (kTile + 1) * 4);
  L.lists = o;   o = align16(o + C * nsub * Kc * 8);
  const int u1 = o;
  o = u0;
  L.gkeys = o;   o = align16(o + C * Tg * 4);
  L.gflag = o;   o = align16(o + C * Tg);
  o = o > u1 ? o : u1;
  L.pooled = o;  o = align16(o + N * 4);
  L.t0c = o;     o = align16(o + N * 4);
  L.selflag = o; o = align16(o + N);
  L.sel = o;     o = align16(o + (Kc + 1) * 4);
  L.selt0 = o;   o = align16(o + (Kc + 1) * 4);
  L.gt0 = o;     o = align16(o + Tg * 4);
  L.gpool = o;   o = align16(o + Tg * 4);
  L.red = o;     o = align16(o + 16 * 4);
  L.total = o;
  return L;
}

template <typename T>
__device__ __forceinline__ const T* q_row_ptr(const T* q, int q_layout, int b, int h, int64_t t, int H,
                                              int64_t S, int Dh) {
  return q_layout == 0 ? q + (((int64_t)b * H + h) * S + t) * Dh : q + (((int64_t)b * S + t) * H + h) * Dh;
}

template <typename T>
__global__ void __launch_bounds__(kRouteThreads) route_prefill_kernel(
    hga_params p, int64_t S, QRange qr, const T* __restrict__ q, int q_layout, const T* __restrict__ chunk_k,
    const T* __restrict__ group_k, int64_t sum_cap, int N, int Kc, int Kg, int Kgr, int nsub,
    int32_t* __restrict__ sel_chunk, int32_t* __restrict__ sel_t0, int32_t* __restrict__ open_gid,
    int32_t* __restrict__ open_t0, float* __restrict__ dbg_l1, float* __restrict__ dbg_l2) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int ln = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int n = qr.chunk0 + ln;
  const int H = p.nhead, KVH = p.kv_heads, Dh = p.head_dim, C = p.chunk_size, M = C / p.group_size;
  const int kvh = h / (H / KVH);
  const int tid = threadIdx.x;
  const int Tg = Kc * M;
  const RouteSmem L = route_smem_layout(C, Dh, N, Kc, Tg, nsub, (int)sizeof(T));
  T* qs = (T*)(smem + L.qs);
  T* ks = (T*)(smem + L.ks);
  float* sc = (float*)(smem + L.sc);
  unsigned long long* lists = (unsigned long long*)(smem + L.lists);
  uint32_t* pooled = (uint32_t*)(smem + L.pooled);
  int* t0c = (int*)(smem + L.t0c);
  unsigned char* selflag = smem + L.selflag;
  int* sel = (int*)(smem + L.sel);
  int* selt0 = (int*)(smem + L.selt0);
  uint32_t* gkeys = (uint32_t*)(smem + L.gkeys);
  unsigned char* gflag = smem + L.gflag;
  int* gt0 = (int*)(smem + L.gt0);
  uint32_t* gpool = (uint32_t*)(smem + L.gpool);
  int* red = (int*)(smem + L.red);
  const int ldq = Dh + 2;

  const size_t tile_out = (((size_t)b * H + h) * qr.count + ln);
  // default outputs: empty lists
  for (int i = tid; i < Kc; i += blockDim.x) {
    sel_chunk[tile_out * Kc + i] = -1;
    sel_t0[tile_out * Kc + i] = -1;
  }
  for (int i = tid; i < Kg; i += blockDim.x) {
    open_gid[tile_out * Kg + i] = -1;
    open_t0[tile_out * Kg + i] = -1;
  }
  if (Kc == 0) return;
  int f_hi, l_lo;
  windows(n, p.keep_first, p.keep_last, f_hi, l_lo);
  const int pool_lo = f_hi, pool_hi = l_lo;  // pool = [f_hi, l_lo), all < n
  const int npool = pool_hi > pool_lo ? pool_hi - pool_lo : 0;
  if (npool == 0) return;
  const int64_t row0 = (int64_t)n * C;
  const int nvalid = (int)((S - row0) < C ? (S - row0) : C);

  // q tile -> smem (fp32)
  for (int i = tid; i < C * Dh; i += blockDim.x) {
    const int t = i / Dh, d = i % Dh;
    T x = Num<T>::from_f(0.f);
    if (t < nvalid) x = q_row_ptr(q, q_layout, b, h, (int64_t)ln * C + t, H, qr.sq, Dh)[d];
    qs[t * ldq + d] = x;
  }
  for (int i = tid; i < npool; i += blockDim.x) {
    pooled[i] = 0u;
    t0c[i] = 0x7fffffff;
  }
  const int k1 = Kc < npool ? Kc : npool;  // requests per row
  for (int i = tid; i < C * nsub * Kc; i += blockDim.x) lists[i] = 0ull;
  __syncthreads();

  // ---- level 1: stream the pool through smem tiles ---------------------------------------
  const T* ck_base = chunk_k + (size_t)(b * KVH + kvh) * sum_cap * Dh;
  for (int c0 = 0; c0 < npool; c0 += kTile) {
    const int nt = (npool - c0) < kTile ? (npool - c0) : kTile;
    for (int i = tid; i < nt * Dh; i += blockDim.x) {
      const int r = i / Dh, d = i % Dh;
      ks[r * ldq + d] = ck_base[(size_t)(pool_lo + c0 + r) * Dh + d];
    }
    __syncthreads();
    for (int i = tid; i < C * nt; i += blockDim.x) {
      const int t = i / nt, r = i % nt;
      float acc = 0.f;
      const T* qa = qs + t * ldq;
      const T* kb = ks + r * ldq;
      for (int d = 0; d < Dh; ++d) acc = fmaf(Num<T>::to_f(qa[d]), Num<T>::to_f(kb[d]), acc);
      const float s = ref_score<T>(acc, p.scale);
      sc[t * (kTile + 1) + r] = s;
      if (dbg_l1 && t < nvalid) dbg_l1[(tile_out * C + t) * N + pool_lo + c0 + r] = s;
    }
    __syncthreads();
    // row-thread (t, sub) inserts its share of the tile into its sub-list
    for (int w = tid; w < C * nsub; w += blockDim.x) {
      const int t = w / nsub, sub = w % nsub;
      if (t >= nvalid) continue;
      unsigned long long* lst = lists + (size_t)w * Kc;
      for (int r = sub; r < nt; r += nsub) {
        const unsigned long long key = rank_key(sc[t * (kTile + 1) + r], (uint32_t)(c0 + r));
        list_insert(lst, k1, key);
      }
    }
    __syncthreads();
  }
  // merge sub-lists per row and register requests (pooled amax, first requesting row)
  for (int t = tid; t < nvalid; t += blockDim.x) {
    unsigned long long* base = lists + (size_t)t * nsub * Kc;
    int ptr[8];
    for (int s = 0; s < nsub; ++s) ptr[s] = 0;
    for (int r = 0; r < k1; ++r) {
      int best = -1;
      unsigned long long bk = 0ull;
      for (int s = 0; s < nsub; ++s) {
        if (ptr[s] < k1) {
          const unsigned long long kk = base[s * Kc + ptr[s]];
          if (kk > bk) { bk = kk; best = s; }
        }
      }
      if (best < 0) break;
      ptr[best]++;
      const int c = (int)rank_idx(bk);
      atomicMax(&pooled[c], ord_f32(rank_score(bk)));
      atomicMin(&t0c[c], t);
    }
  }
  __syncthreads();
  // choose Kc of the requested chunks by pooled score
  block_select(pooled, npool, Kc, selflag, red);
  // force-include the previous chunk when it lies in the pool
  const int prev = n - 1;
  const bool prev_in = n > 0 && prev >= pool_lo && prev < pool_hi;
  if (tid == 0) {
    int nsel = 0;
    for (int i = 0; i < npool; ++i) nsel += selflag[i];
    if (prev_in) {
      const int pr = prev - pool_lo;
      if (!selflag[pr]) {
        if (nsel >= Kc) {
          // drop the lowest-ranked chosen chunk (lowest pooled, then highest index)
          int worst = -1;
          for (int i = 0; i < npool; ++i)
            if (selflag[i] && (worst < 0 || pooled[i] <= pooled[worst])) worst = i;
          selflag[worst] = 0;
        }
        selflag[pr] = 1;
      }
      t0c[pr] = 0;
    }
    int k = 0;
    for (int i = 0; i < npool; ++i)
      if (selflag[i]) {
        sel[k] = pool_lo + i;
        selt0[k] = t0c[i];
        ++k;
      }
    red[8] = k;
  }
  __syncthreads();
  const int ksel = red[8];
  for (int i = tid; i < ksel; i += blockDim.x) {
    sel_chunk[tile_out * Kc + i] = sel[i];
    sel_t0[tile_out * Kc + i] = selt0[i];
  }
  if (Kg == 0 || Kgr == 0) return;

  // ---- level 2: groups of the chosen chunks ---------------------------------------------
  const int tsel = ksel * M;
  const T* gk_base = group_k + (size_t)(b * KVH + kvh) * sum_cap * M * Dh;
  for (int i = tid; i < tsel * Dh; i += blockDim.x) {
    const int j = i / Dh, d = i % Dh;
    const int k = j / M, g = j % M;
    ks[j * ldq + d] = gk_base[((size_t)sel[k] * M + g) * Dh + d];
  }
  for (int j = tid; j < Tg; j += blockDim.x) {
    gt0[j] = 0x7fffffff;
    gpool[j] = 0u;
  }
  __syncthreads();
  for (int i = tid; i < C * tsel; i += blockDim.x) {
    const int t = i / tsel, j = i % tsel;
    const bool real = t < nvalid && t >= selt0[j / M];
    float s = kNeg;
    if (real) {
      float acc = 0.f;
      const T* qa = qs + t * ldq;
      const T* kb = ks + j * ldq;
      for (int d = 0; d < Dh; ++d) acc = fmaf(Num<T>::to_f(qa[d]), Num<T>::to_f(kb[d]), acc);
      s = ref_score<T>(acc, p.scale);
    }
    gkeys[t * Tg + j] = real ? ord_f32(s) : 0u;
    if (dbg_l2 && t < nvalid) dbg_l2[(tile_out * C + t) * Tg + j] = s;
  }
  __syncthreads();
  // per-row requests (one warp per row)
  const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  const bool all_req = Kgr >= Tg;
  for (int t = warp; t < nvalid; t += nwarps) {
    unsigned char* fl = gflag + t * Tg;
    if (all_req) {
      for (int j = lane; j < tsel; j += 32) fl[j] = gkeys[t * Tg + j] != 0u;
      __syncwarp();
    } else {
      warp_select(gkeys + t * Tg, tsel, Kgr, fl);
    }
    for (int j = lane; j < tsel; j += 32)
      if (fl[j]) {
        atomicMin(&gt0[j], t);
        atomicMax(&gpool[j], gkeys[t * Tg + j]);
      }
  }
  __syncthreads();
  // choose Kg requested groups by pooled score
  if (Kg >= Tg) {
    for (int j = tid; j < tsel; j += blockDim.x) gflag[j] = gt0[j] != 0x7fffffff;
    __syncthreads();
  } else {
    block_select(gpool, tsel, Kg, gflag, red);
  }
  if (tid == 0) {
    int k = 0;
    for (int j = 0; j < tsel; ++j)
      if (gflag[j] && gt0[j] != 0x7fffffff) {
        open_gid[tile_out * Kg + k] = sel[j / M] * M + (j % M);
        open_t0[tile_out * Kg + k] = gt0[j];
        ++k;
      }
  }
}

template <typename T>
static cudaError_t launch_route_t(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout,
                                  const void* ck, const void* gk, int64_t sum_cap, int32_t* sel_chunk,
                                  int32_t* sel_t0, int32_t* open_gid, int32_t* open_t0, float* dbg1,
                                  float* dbg2, cudaStream_t st, int* smem_bytes_out) {
  const int C = p.chunk_size, M = C / p.group_size;
  const int N = (int)((S + C - 1) / C);
  const int Kc = p.topk_chunks > 0 ? (p.topk_chunks < N ? p.topk_chunks : N) : 0;
  const int Tg = Kc * M;
  int Kg = p.topk_groups > 0 ? (p.topk_groups < Tg ? p.topk_groups : Tg) : 0;
  int Kgr = p.topk_groups > 0 ? ((p.topk_groups / 2) < Tg ? (p.topk_groups / 2) : Tg) : 0;
  if (Kgr == 0) Kg = 0;
  int nsub = kRouteThreads / C;
  if (nsub < 1) nsub = 1;
  if (nsub > 8) nsub = 8;
  while (nsub > 1 && nsub * (Kc > 0 ? Kc : 1) > 64) nsub >>= 1;
  const RouteSmem L = route_smem_layout(C, p.head_dim, N, Kc > 0 ? Kc : 1, Tg, nsub, (int)sizeof(T));
  *smem_bytes_out = L.total;
  if (L.total > 227 * 1024) return cudaErrorInvalidConfiguration;
  auto kern = route_prefill_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
  if (e != cudaSuccess) return e;
  dim3 grid(qr.count, p.nhead, p.batch);
  kern<<<grid, kRouteThreads, L.total, st>>>(p, S, qr, (const T*)q, q_layout, (const T*)ck, (const T*)gk, sum_cap, N,
                                             Kc, Kg, Kgr, nsub, sel_chunk, sel_t0, open_gid, open_t0, dbg1,
                                             dbg2);
  return cudaGetLastError();
}

cudaError_t launch_route_prefill(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout, const void* ck,
                                 const void* gk, int64_t sum_cap, int32_t* sel_chunk, int32_t* sel_t0,
                                 int32_t* open_gid, int32_t* open_t0, float* dbg1, float* dbg2,
                                 cudaStream_t st, int* smem_bytes_out) {
  switch (p.dtype) {
    case HGA_DTYPE_F32:
      return launch_route_t<float>(p, S, qr, q, q_layout, ck, gk, sum_cap, sel_chunk, sel_t0, open_gid, open_t0,
                                   dbg1, dbg2, st, smem_bytes_out);
    case HGA_DTYPE_BF16:
      return launch_route_t<__nv_bfloat16>(p, S, qr, q, q_layout, ck, gk, sum_cap, sel_chunk, sel_t0, open_gid,
                                           open_t0, dbg1, dbg2, st, smem_bytes_out);
    case HGA_DTYPE_F16:
      return launch_route_t<__half>(p, S, qr, q, q_layout, ck, gk, sum_cap, sel_chunk, sel_t0, open_gid, open_t0,
                                    dbg1, dbg2, st, smem_bytes_out);
  }
  return cudaErrorInvalidValue;
}

}  // namespace hga
