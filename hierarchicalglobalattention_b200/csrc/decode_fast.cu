// Decode fast paths: the routing of one new token (L = 1) and the attention of short blocks
// (L <= 8) with 16-token groups and head_dim 64 / 128.  Same results as decode.cu's portable
// kernels (ChunkRouter._route_decision, chunk_router.py:210-277, and the flat branch of
// RoutedKV.attend, :159-162); they differ in how the work is laid out:
//
//  * routing, L = 1: with one row the pooled score of a chunk IS the row's score, so the block's
//    top-Kc and the row's requests are the same set (every chosen chunk is visible from row 0),
//    and the visible groups are the row's top-Kg_request among the chosen chunks' groups (a
//    subset of the pooled top-Kg).  One CTA serves the query heads of one KV head that share
//    it (up to 8): one thread scores one summary row for all of them with 16-byte loads, and the
//    heads' selections run in separate warps.
//  * attention: one warp streams one 16-token unit at a time (a window group, an opened group or
//    a group of the active chunk).  The unit's K rows are read as whole lines (consecutive lanes,
//    consecutive 16-byte pieces) and staged in shared memory, a lane pair then scores one key
//    (each lane half of head_dim), every lane holds head_dim/32 columns of all 16 values (also read
//    as whole lines), and the warp keeps an
//    fp32 online-softmax state per query row; the 8 warps' states are merged at the end.  Opened
//    groups are read from the cold record, which for the RAM tier is pinned host memory.
#include "select.cuh"

namespace hga {

HGA_DEVICE_ERROR_WORD(g_decode_fast_error, decode_fast_error_status)

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = Num<T>::to_f(h[i]);
  }
}

// Ascending compaction of flag[0..n) by warp 0: writes idx[k] = i of the k-th set flag, returns k.
__device__ __forceinline__ int warp_compact(const unsigned char* flag, int n, int* idx) {
  const int lane = threadIdx.x & 31;
  int k = 0;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const bool f = i < n && flag[i];
    const unsigned bal = __ballot_sync(0xffffffffu, f);
    if (f) idx[k + __popc(bal & ((1u << lane) - 1u))] = i;
    k += __popc(bal);
  }
  return k;
}

// q_h . row for HB query heads at once (the row is read once, its 16-byte pieces all in flight);
// every head's sum runs in column order with fp32 FMAs, like dot_row.
template <typename T, int DH, int HB>
__device__ __forceinline__ void dot_rows(const float* qs, const T* row, float* acc) {
  constexpr int PER = 16 / (int)sizeof(T);
  constexpr int NV = DH / PER;
  const uint4* r = reinterpret_cast<const uint4*>(row);
#pragma unroll
  for (int j = 0; j < HB; ++j) acc[j] = 0.f;
#pragma unroll 16
  for (int v = 0; v < NV; ++v) {
    const uint4 u = __ldg(r + v);
    float f[PER];
    unpack16<T>(u, f);
#pragma unroll
    for (int e = 0; e < PER; ++e)
#pragma unroll
      for (int j = 0; j < HB; ++j) acc[j] = fmaf(qs[j * DH + v * PER + e], f[e], acc[j]);
  }
}

// One CTA routes HB query heads that share one KV head (h0 .. h0+HB-1 of batch row b): thread i
// scores pool chunk i (and later candidate group i) for all HB heads from one read of the summary
// row, then warp j selects head j's chunks and groups, the HB selections running side by side.
template <typename T, int DH, int HB>
__global__ void __launch_bounds__(256, 2) route_decode1_kernel(
    hga_params p, const T* __restrict__ q, const int32_t* __restrict__ seq_pos, const T* __restrict__ chunk_k,
    const T* __restrict__ group_k, int64_t sum_cap, int Kcmax, int Kgmax, int32_t* __restrict__ mid_chunk,
    int32_t* __restrict__ mid_t0, int32_t* __restrict__ open_gid, int32_t* __restrict__ open_t0, int nkey_max,
    int nmid_max) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int h0 = blockIdx.x * HB, b = blockIdx.y;
  const int H = p.nhead, KVH = p.kv_heads, C = p.chunk_size, M = C / p.group_size;
  const int kvh = h0 / (H / KVH);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_closed = seq_pos[b] / C;
  int f_hi, l_lo;
  windows(n_closed, p.keep_first, p.keep_last, f_hi, l_lo);
  const int n_mid = l_lo > f_hi ? l_lo - f_hi : 0;
  const size_t bh0 = (size_t)b * H + h0;
  for (int i = tid; i < HB * Kcmax; i += blockDim.x) { mid_chunk[bh0 * Kcmax + i] = -1; mid_t0[bh0 * Kcmax + i] = -1; }
  for (int i = tid; i < HB * Kgmax; i += blockDim.x) { open_gid[bh0 * Kgmax + i] = -1; open_t0[bh0 * Kgmax + i] = -1; }
  if (n_mid == 0 || p.topk_chunks <= 0) return;
  const int Kc = p.topk_chunks < n_mid ? p.topk_chunks : n_mid;
  // a pool larger than the caller's nmid_max is reported and left unrouted, as by the portable
  // kernel (the smem key arrays may be larger than nmid_max: they also hold Kcmax * M groups)
  if ((int64_t)l_lo > sum_cap || n_mid > nmid_max || n_mid > nkey_max || Kc > Kcmax) {
    if (tid == 0) atomicCAS(&g_decode_fast_error, 0, kErrBoundsRouteDecode);
    return;
  }
  const int G = Kc * M;
  const int Kg = p.topk_groups > 0 ? (p.topk_groups < G ? p.topk_groups : G) : 0;
  const int Kgr = p.topk_groups > 0 ? ((p.topk_groups / 2) < G ? p.topk_groups / 2 : G) : 0;

  float* qs = (float*)smem;                                   // [HB][DH]
  uint32_t* keys = (uint32_t*)(qs + HB * DH);                 // [HB][nkey_max]
  int* sred = (int*)(keys + (size_t)HB * nkey_max);           // [16]
  int* idx = sred + 16;                                       // [HB][nkey_max]
  unsigned char* flag = (unsigned char*)(idx + (size_t)HB * nkey_max);   // [HB][nkey_max]

  for (int i = tid; i < HB * DH; i += blockDim.x) qs[i] = Num<T>::to_f(q[bh0 * DH + i]);
  __syncthreads();
  // ---- level 1: one thread per pool chunk, all HB heads ------------------------------------------
  const T* ckb = chunk_k + ((size_t)b * KVH + kvh) * sum_cap * DH;
  for (int i = tid; i < n_mid; i += blockDim.x) {
    float acc[HB];
    dot_rows<T, DH, HB>(qs, ckb + (size_t)(f_hi + i) * DH, acc);
#pragma unroll
    for (int j = 0; j < HB; ++j) keys[(size_t)j * nkey_max + i] = ord_f32(ref_score<T>(acc[j], p.scale));
  }
  __syncthreads();
  // selection: warp j owns head j (shuffle reductions, no block barriers)
  if (warp < HB) {
    const size_t bh = bh0 + warp;
    uint32_t* kw = keys + (size_t)warp * nkey_max;
    unsigned char* fw = flag + (size_t)warp * nkey_max;
    int* iw = idx + (size_t)warp * nkey_max;
    if (n_mid <= 512) warp_topk_small(kw, n_mid, Kc, fw);
    else warp_select(kw, n_mid, Kc, fw);
    // the previous chunk replaces the lowest chosen one (ties: the highest index) when in the pool
    const int prev = n_closed - 1;
    if (prev >= f_hi && prev < l_lo && !fw[prev - f_hi]) {
      unsigned long long worst = ~0ull;
      for (int i = lane; i < n_mid; i += 32)
        if (fw[i]) {
          const unsigned long long c = ((unsigned long long)kw[i] << 32) | (0xffffffffu - (uint32_t)i);
          worst = c < worst ? c : worst;
        }
      for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, worst, o);
        worst = other < worst ? other : worst;
      }
      if (lane == 0) {
        fw[0xffffffffu - (uint32_t)(worst & 0xffffffffull)] = 0;
        fw[prev - f_hi] = 1;
      }
      __syncwarp();
    }
    const int k = warp_compact(fw, n_mid, iw);
    __syncwarp();
    for (int i = lane; i < k; i += 32) {
      iw[i] += f_hi;
      mid_chunk[bh * Kcmax + i] = iw[i];
      mid_t0[bh * Kcmax + i] = 0;
    }
    if (lane == 0) sred[warp] = k;
  }
  __syncthreads();
  if (Kg <= 0 || Kgr <= 0) return;
  // ---- level 2: one thread per (head, candidate group of its chosen chunks) ---------------------
  const T* gkb = group_k + ((size_t)b * KVH + kvh) * sum_cap * M * DH;
  for (int t = tid; t < HB * G; t += blockDim.x) {
    const int j = t / G, g = t - j * G;
    if (g < sred[j] * M) {
      float acc[1];
      dot_rows<T, DH, 1>(qs + j * DH, gkb + ((size_t)idx[(size_t)j * nkey_max + g / M] * M + (g % M)) * DH, acc);
      keys[(size_t)j * nkey_max + g] = ord_f32(ref_score<T>(acc[0], p.scale));
    }
  }
  __syncthreads();
  if (warp < HB) {
    const size_t bh = bh0 + warp;
    uint32_t* kw = keys + (size_t)warp * nkey_max;
    unsigned char* fw = flag + (size_t)warp * nkey_max;
    const int* iw = idx + (size_t)warp * nkey_max;
    const int Gs = sred[warp] * M;
    if (Gs <= 512) warp_topk_small(kw, Gs, Kgr < Gs ? Kgr : Gs, fw);
    else warp_select(kw, Gs, Kgr < Gs ? Kgr : Gs, fw);
    int k = 0;
    for (int base = 0; base < Gs; base += 32) {
      const int j = base + lane;
      const bool f = j < Gs && fw[j];
      const unsigned bal = __ballot_sync(0xffffffffu, f);
      if (f) {
        const int at = k + __popc(bal & ((1u << lane) - 1u));
        open_gid[bh * Kgmax + at] = iw[j / M] * M + (j % M);
        open_t0[bh * Kgmax + at] = 0;
      }
      k += __popc(bal);
    }
  }
}

size_t route_decode1_smem(int Dh, int nkey_max, int hb) {
  return (size_t)hb * Dh * 4 + (size_t)hb * nkey_max * 4 + 64 + (size_t)hb * nkey_max * 4 + (size_t)hb * nkey_max +
         16;
}

// Heads per CTA: the largest of 8, 4, 2 that divides the query heads of one KV head and still
// leaves at least 128 CTAs, else 1 (small batches route with the most CTAs).  A summary row read
// once serves more heads, so with enough CTAs to cover most SMs fewer, fuller CTAs win: at 32K
// tokens, 32 query / 4 KV heads, B=16 routes in 25 us with 4 heads per CTA (128 CTAs) against 31
// us with 2 (256 CTAs), B=32 in 32 us with 8 against 34 us with 4.
static int route_decode1_heads(const hga_params& p) {
  const int rep = p.nhead / p.kv_heads;
  for (int hb = 8; hb > 1; hb >>= 1)
    if (rep % hb == 0 && (int64_t)p.batch * (p.nhead / hb) >= 128) return hb;
  return 1;
}

template <typename T, int DH, int HB>
static cudaError_t launch_route_decode1_h(const hga_params& p, const void* q, const int32_t* seq_pos, const void* ck,
                                          const void* gk, int64_t sum_cap, int nkey, int nmid_max, int Kcmax,
                                          int Kgmax, int32_t* mc, int32_t* mt, int32_t* og, int32_t* ot, cudaStream_t st) {
  const size_t smem = route_decode1_smem(DH, nkey, HB);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  auto kern = route_decode1_kernel<T, DH, HB>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(p.nhead / HB, p.batch);
  kern<<<grid, 256, smem, st>>>(p, (const T*)q, seq_pos, (const T*)ck, (const T*)gk, sum_cap, Kcmax, Kgmax, mc, mt,
                                og, ot, nkey, nmid_max);
  return cudaGetLastError();
}

template <typename T, int DH>
static cudaError_t launch_route_decode1_t(const hga_params& p, const void* q, const int32_t* seq_pos, const void* ck,
                                          const void* gk, int64_t sum_cap, int nmid_max, int Kcmax, int Kgmax,
                                          int32_t* mc, int32_t* mt, int32_t* og, int32_t* ot, cudaStream_t st) {
  const int M = p.chunk_size / p.group_size;
  const int nkey = nmid_max > Kcmax * M ? nmid_max : Kcmax * M;
  switch (route_decode1_heads(p)) {
    case 8: return launch_route_decode1_h<T, DH, 8>(p, q, seq_pos, ck, gk, sum_cap, nkey, nmid_max, Kcmax, Kgmax, mc, mt, og, ot, st);
    case 4: return launch_route_decode1_h<T, DH, 4>(p, q, seq_pos, ck, gk, sum_cap, nkey, nmid_max, Kcmax, Kgmax, mc, mt, og, ot, st);
    case 2: return launch_route_decode1_h<T, DH, 2>(p, q, seq_pos, ck, gk, sum_cap, nkey, nmid_max, Kcmax, Kgmax, mc, mt, og, ot, st);
    default: return launch_route_decode1_h<T, DH, 1>(p, q, seq_pos, ck, gk, sum_cap, nkey, nmid_max, Kcmax, Kgmax, mc, mt, og, ot, st);
  }
}

bool route_decode1_supported(const hga_params& p, int L) {
  return L == 1 && (p.head_dim == 64 || p.head_dim == 128);
}

cudaError_t launch_route_decode1(const hga_params& p, const void* q, const int32_t* seq_pos, const void* ck,
                                 const void* gk, int64_t sum_cap, int nmid_max, int Kcmax, int Kgmax, int32_t* mc,
                                 int32_t* mt, int32_t* og, int32_t* ot, cudaStream_t st) {
#define HGA_R1(TT)                                                                                          \
  return p.head_dim == 128                                                                                  \
             ? launch_route_decode1_t<TT, 128>(p, q, seq_pos, ck, gk, sum_cap, nmid_max, Kcmax, Kgmax, mc, mt, og, \
                                               ot, st)                                                      \
             : launch_route_decode1_t<TT, 64>(p, q, seq_pos, ck, gk, sum_cap, nmid_max, Kcmax, Kgmax, mc, mt, og,  \
                                              ot, st);
  switch (p.dtype) {
    case HGA_DTYPE_F32: HGA_R1(float)
    case HGA_DTYPE_BF16: HGA_R1(__nv_bfloat16)
    case HGA_DTYPE_F16: HGA_R1(__half)
  }
#undef HGA_R1
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------------------------------------
// attention of a short decode block
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ int64_t slot_row(int chunk, int u, int C, int mode, int kf, int kl, bool active) {
  if (mode == 0) return (int64_t)chunk * C + u;
  const int slot = active ? kf + kl : (chunk < kf ? chunk : kf + chunk % (kl > 0 ? kl : 1));
  return (int64_t)slot * C + u;
}

template <int DH> struct VCols;                 // head_dim/32 16-bit values of one key row
template <> struct VCols<128> { using type = uint2; };
template <> struct VCols<64> { using type = uint32_t; };

constexpr int kAttWarps = 8;
constexpr int kUnit = 16;  // tokens per unit (the routing group)

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <typename T, int DH, int LM>
__global__ void __launch_bounds__(kAttWarps * 32, (LM == 1 ? 2 : 1)) attend_decode_fast_kernel(
    hga_params p, int L, const T* __restrict__ q, const int32_t* __restrict__ seq_pos, const T* hot_k, const T* hot_v,
    int64_t hot_cap, int hot_mode, const T* cold_k, const T* cold_v, int64_t cold_cap,
    const int32_t* __restrict__ open_gid, const int32_t* __restrict__ open_t0, int Kg, int cold_direct,
    T* __restrict__ out) {
  static_assert(sizeof(T) == 2, "16-bit K/V only");
  constexpr int HALF = DH / 2;
  constexpr int KLD = HALF / 8;   // 16-byte loads per lane for its half key row
  constexpr int VD = DH / 32;     // value columns per lane
  using VT = typename VCols<DH>::type;
  constexpr int CPK = DH * 2 / 16;        // 16-byte pieces per key row
  constexpr int RS = DH * 2 + 32;         // staged row stride (bytes): conflict-free lane-pair reads
  constexpr int HO = HALF * 2 + 16;       // offset of a staged row's second half
  extern __shared__ __align__(16) unsigned char smem[];
  float* qs = (float*)smem;                               // [LM][DH]
  float* so = qs + LM * DH;                               // [warps][LM][DH]
  float* sm = so + kAttWarps * LM * DH;                   // [warps][LM]
  float* sl = sm + kAttWarps * LM;                        // [warps][LM]
  unsigned char* kst = (unsigned char*)(sl + kAttWarps * LM) + (size_t)(threadIdx.x >> 5) * kUnit * RS;
  // per warp: the V rows of the unit in flight [16][DH], then the CTA's copy of the open lists
  unsigned char* vst = (unsigned char*)(sl + kAttWarps * LM) + (size_t)kAttWarps * kUnit * RS +
                       (size_t)(threadIdx.x >> 5) * kUnit * DH * 2;
  int32_t* lgid = (int32_t*)((unsigned char*)(sl + kAttWarps * LM) + (size_t)kAttWarps * kUnit * (RS + DH * 2));
  int32_t* lt0 = lgid + Kg;

  const int h = blockIdx.x, b = blockIdx.y;
  const int H = p.nhead, KVH = p.kv_heads, C = p.chunk_size, M = C / kUnit;
  const int kvh = h / (H / KVH);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = seq_pos[b];
  const int n_closed = pos / C, c0 = pos % C;
  const int kf = p.keep_first > 0 ? p.keep_first : 0, kl = p.keep_last > 0 ? p.keep_last : 0;
  int f_hi, l_lo;
  windows(n_closed, kf, kl, f_hi, l_lo);
  const size_t bh = (size_t)b * H + h;
  const bool hot_oob = hot_mode == 0 ? (int64_t)(n_closed + 1) * C > hot_cap : (int64_t)(kf + kl + 1) * C > hot_cap;
  if (hot_oob || (hot_mode == 0 && (int64_t)n_closed * C > cold_cap)) {
    if (tid == 0) atomicCAS(&g_decode_fast_error, 0, kErrBoundsAttendDecode);
    for (int i = tid; i < L * DH; i += blockDim.x) out[bh * L * DH + i] = Num<T>::from_f(0.f);
    return;
  }

  // the opened entries are a prefix of the list (entries that no row sees are not written)
  for (int j = tid; j < Kg; j += blockDim.x) {
    lgid[j] = open_gid[bh * Kg + j];
    lt0[j] = open_t0[bh * Kg + j];
  }
  __syncthreads();
  int nopen = 0;
  for (int base = 0; base < Kg; base += 32) {
    const int j = base + lane;
    const bool ok = j < Kg && lgid[j] >= 0 && lt0[j] >= 0;
    nopen += __popc(__ballot_sync(0xffffffffu, ok));
  }
  const int nfirst_u = f_hi * M, nlast_u = (n_closed - l_lo) * M;
  const int nact = c0 + L, nact_u = (nact + kUnit - 1) / kUnit;
  const int U = nfirst_u + nlast_u + nopen + nact_u;

  const float sl2 = p.scale * 1.4426950408889634f;
  for (int i = tid; i < L * DH; i += blockDim.x) qs[i] = Num<T>::to_f(q[bh * L * DH + i]) * sl2;
  __syncthreads();

  float o[LM][VD], m[LM], l[LM];
#pragma unroll
  for (int t = 0; t < LM; ++t) {
    m[t] = -INFINITY;
    l[t] = 0.f;
#pragma unroll
    for (int d = 0; d < VD; ++d) o[t][d] = 0.f;
  }
  const size_t hot_base = ((size_t)b * KVH + kvh) * hot_cap;
  const size_t cold_base = ((size_t)b * KVH + kvh) * cold_cap;
  const int key = lane >> 1, half = lane & 1;

  // unit u -> its first row, K/V base, first visible row t0 and active-chunk offset (ok = false:
  // an opened group past the record, reported and skipped); direct = read with plain loads when it
  // is scored (opened groups in host memory: asynchronous copies from there are much slower)
  auto unit_at = [&](int u, int64_t& row, const T*& kb, const T*& vb, int& t0, int& act0, bool& direct) -> bool {
    t0 = 0;
    act0 = -1;
    direct = false;
    kb = hot_k; vb = hot_v;
    if (u < nfirst_u) {
      row = hot_base + slot_row(u / M, (u % M) * kUnit, C, hot_mode, kf, kl, false);
    } else if (u < nfirst_u + nlast_u) {
      const int uu = u - nfirst_u;
      row = hot_base + slot_row(l_lo + uu / M, (uu % M) * kUnit, C, hot_mode, kf, kl, false);
    } else if (u < nfirst_u + nlast_u + nopen) {
      const int j = u - nfirst_u - nlast_u;
      const int gid = lgid[j];
      if ((int64_t)(gid + 1) * kUnit > cold_cap) return false;
      row = cold_base + (int64_t)gid * kUnit;
      t0 = lt0[j];
      kb = cold_k; vb = cold_v;
      direct = cold_direct != 0;
    } else {
      act0 = (u - nfirst_u - nlast_u - nopen) * kUnit;
      row = hot_base + slot_row(n_closed, act0, C, hot_mode, kf, kl, true);
    }
    return true;
  };
  // K rows land in the lane-pair staging layout, V rows contiguously; one commit group per unit
  auto issue = [&](int64_t row, const T* kb, const T* vb) {
    const uint4* kp = reinterpret_cast<const uint4*>(kb + row * DH);
    const uint4* vp = reinterpret_cast<const uint4*>(vb + row * DH);
#pragma unroll
    for (int i = 0; i < KLD; ++i) {
      const int c = i * 32 + lane;
      const int w = (c % CPK) * 16;
      cp_async16(kst + (c / CPK) * RS + w + (w >= HALF * 2 ? 16 : 0), kp + c);
      cp_async16(vst + c * 16, vp + c);
    }
    cp_async_commit();
  };

  // one unit in flight per warp while the previous one is scored: its K/V copies are issued as
  // soon as the staged rows of the current unit have been read into registers
  int64_t row_c;
  const T *kb_c, *vb_c;
  int t0_c = 0, act0_c = -1;
  bool ok_c = false, direct_c = false;
  if (warp < U) {
    ok_c = unit_at(warp, row_c, kb_c, vb_c, t0_c, act0_c, direct_c);
    if (ok_c && !direct_c) issue(row_c, kb_c, vb_c);
    else if (!ok_c && lane == 0) atomicCAS(&g_decode_fast_error, 0, kErrBoundsAttendDecode);
  }
  for (int u = warp; u < U; u += kAttWarps) {
    uint4 kr[KLD];
    VT vr[kUnit];
    if (ok_c && direct_c) {
      // whole lines per instruction (consecutive lanes, consecutive 16-byte pieces), K staged in
      // shared memory for the lane pairs (no copy is in flight: none was issued for this unit)
      const uint4* kp = reinterpret_cast<const uint4*>(kb_c + row_c * DH);
#pragma unroll
      for (int i = 0; i < KLD; ++i) kr[i] = kp[i * 32 + lane];
      const T* vp = vb_c + row_c * DH + lane * VD;
#pragma unroll
      for (int j = 0; j < kUnit; ++j) vr[j] = *reinterpret_cast<const VT*>(vp + (size_t)j * DH);
#pragma unroll
      for (int i = 0; i < KLD; ++i) {
        const int c = i * 32 + lane;
        const int w = (c % CPK) * 16;
        *reinterpret_cast<uint4*>(kst + (c / CPK) * RS + w + (w >= HALF * 2 ? 16 : 0)) = kr[i];
      }
      __syncwarp();
      const uint4* kmine = reinterpret_cast<const uint4*>(kst + key * RS + half * HO);
#pragma unroll
      for (int i = 0; i < KLD; ++i) kr[i] = kmine[i];
      __syncwarp();
    } else if (ok_c) {
      cp_async_wait_all();
      __syncwarp();
      const uint4* kmine = reinterpret_cast<const uint4*>(kst + key * RS + half * HO);
#pragma unroll
      for (int i = 0; i < KLD; ++i) kr[i] = kmine[i];
#pragma unroll
      for (int j = 0; j < kUnit; ++j) vr[j] = *reinterpret_cast<const VT*>(vst + j * DH * 2 + lane * VD * 2);
      __syncwarp();
    }
    const bool ok = ok_c;
    const int t0 = t0_c, act0 = act0_c;
    const int un = u + kAttWarps;
    if (un < U) {
      ok_c = unit_at(un, row_c, kb_c, vb_c, t0_c, act0_c, direct_c);
      if (ok_c && !direct_c) issue(row_c, kb_c, vb_c);
      else if (!ok_c && lane == 0) atomicCAS(&g_decode_fast_error, 0, kErrBoundsAttendDecode);
    }
    if (!ok) continue;  // warp-uniform

#pragma unroll
    for (int t = 0; t < LM; ++t) {
      if (t >= L) break;
      const float* qt = qs + t * DH + half * HALF;
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < KLD; ++i) {
        float f[8];
        unpack16<T>(kr[i], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) dot = fmaf(qt[i * 8 + e], f[e], dot);
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      const bool vis = act0 < 0 ? (t >= t0) : (act0 + key <= c0 + t);
      const float s = vis ? dot : -INFINITY;
      float mx = s;
#pragma unroll
      for (int off = 16; off >= 2; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m[t], mx);
      if (m_new == -INFINITY) continue;  // warp-uniform: nothing visible yet for this row
      const float alpha = exp2f(m[t] - m_new);
      const float pe = vis ? exp2f(s - m_new) : 0.f;
      float ps = half ? 0.f : pe;
#pragma unroll
      for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[t] = l[t] * alpha + ps;
      m[t] = m_new;
#pragma unroll
      for (int d = 0; d < VD; ++d) o[t][d] *= alpha;
#pragma unroll
      for (int j = 0; j < kUnit; ++j) {
        const float pj = __shfl_sync(0xffffffffu, pe, 2 * j);
        const T* hv = reinterpret_cast<const T*>(&vr[j]);
#pragma unroll
        for (int d = 0; d < VD; ++d) o[t][d] = fmaf(pj, Num<T>::to_f(hv[d]), o[t][d]);
      }
    }
  }
  // merge the warps' states
#pragma unroll
  for (int t = 0; t < LM; ++t) {
    if (t >= L) break;
#pragma unroll
    for (int d = 0; d < VD; ++d) so[(warp * LM + t) * DH + lane * VD + d] = o[t][d];
    if (lane == 0) { sm[warp * LM + t] = m[t]; sl[warp * LM + t] = l[t]; }
  }
  __syncthreads();
  for (int i = tid; i < L * DH; i += blockDim.x) {
    const int t = i / DH, d = i % DH;
    float mm = -INFINITY;
    for (int w = 0; w < kAttWarps; ++w) mm = fmaxf(mm, sm[w * LM + t]);
    float ll = 0.f, oo = 0.f;
    if (mm != -INFINITY) {
      for (int w = 0; w < kAttWarps; ++w) {
        const float mw = sm[w * LM + t];
        if (mw == -INFINITY) continue;
        const float f = exp2f(mw - mm);
        ll += sl[w * LM + t] * f;
        oo += so[(w * LM + t) * DH + d] * f;
      }
    }
    out[bh * L * DH + i] = Num<T>::from_f(ll > 0.f ? oo / ll : 0.f);
  }
}

bool attend_decode_fast_supported(const hga_params& p, int L) {
  return (p.dtype == HGA_DTYPE_BF16 || p.dtype == HGA_DTYPE_F16) && p.group_size == kUnit &&
         (p.head_dim == 64 || p.head_dim == 128) && L >= 1 && L <= 8;
}

template <typename T, int DH, int LM>
static cudaError_t launch_att_fast(const hga_params& p, int L, const void* q, const int32_t* seq_pos, const void* hk,
                                   const void* hv, int64_t hot_cap, int hot_mode, const void* ckk, const void* cvv,
                                   int64_t cold_cap, const int32_t* og, const int32_t* ot, int Kg, void* out,
                                   cudaStream_t st) {
  const size_t smem = ((size_t)LM * DH + (size_t)kAttWarps * LM * DH + 2 * kAttWarps * LM) * 4 +
                      (size_t)kAttWarps * kUnit * (DH * 2 + 32 + DH * 2) + (size_t)2 * Kg * 4;
  auto kern = attend_decode_fast_kernel<T, DH, LM>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  // opened groups in host memory (the RAM tier's record read in place) are loaded directly
  cudaPointerAttributes pa;
  int cold_direct = 0;
  if (cudaPointerGetAttributes(&pa, ckk) == cudaSuccess) cold_direct = pa.type == cudaMemoryTypeHost;
  else (void)cudaGetLastError();
  dim3 grid(p.nhead, p.batch);
  kern<<<grid, kAttWarps * 32, smem, st>>>(p, L, (const T*)q, seq_pos, (const T*)hk, (const T*)hv, hot_cap, hot_mode,
                                           (const T*)ckk, (const T*)cvv, cold_cap, og, ot, Kg, cold_direct, (T*)out);
  return cudaGetLastError();
}

template <typename T, int DH>
static cudaError_t launch_att_fast_l(const hga_params& p, int L, const void* q, const int32_t* seq_pos, const void* hk,
                                     const void* hv, int64_t hot_cap, int hot_mode, const void* ckk, const void* cvv,
                                     int64_t cold_cap, const int32_t* og, const int32_t* ot, int Kg, void* out,
                                     cudaStream_t st) {
  if (L == 1)
    return launch_att_fast<T, DH, 1>(p, L, q, seq_pos, hk, hv, hot_cap, hot_mode, ckk, cvv, cold_cap, og, ot, Kg, out, st);
  if (L <= 2)
    return launch_att_fast<T, DH, 2>(p, L, q, seq_pos, hk, hv, hot_cap, hot_mode, ckk, cvv, cold_cap, og, ot, Kg, out, st);
  if (L <= 4)
    return launch_att_fast<T, DH, 4>(p, L, q, seq_pos, hk, hv, hot_cap, hot_mode, ckk, cvv, cold_cap, og, ot, Kg, out, st);
  return launch_att_fast<T, DH, 8>(p, L, q, seq_pos, hk, hv, hot_cap, hot_mode, ckk, cvv, cold_cap, og, ot, Kg, out, st);
}

cudaError_t launch_attend_decode_fast(const hga_params& p, int L, const void* q, const int32_t* seq_pos,
                                      const void* hk, const void* hv, int64_t hot_cap, int hot_mode, const void* ckk,
                                      const void* cvv, int64_t cold_cap, const int32_t* og, const int32_t* ot, int Kg,
                                      void* out, cudaStream_t st) {
#define HGA_AF(TT)                                                                                              \
  return p.head_dim == 128 ? launch_att_fast_l<TT, 128>(p, L, q, seq_pos, hk, hv, hot_cap, hot_mode, ckk, cvv,  \
                                                         cold_cap, og, ot, Kg, out, st)                         \
                           : launch_att_fast_l<TT, 64>(p, L, q, seq_pos, hk, hv, hot_cap, hot_mode, ckk, cvv,   \
                                                        cold_cap, og, ot, Kg, out, st);
  switch (p.dtype) {
    case HGA_DTYPE_BF16: HGA_AF(__nv_bfloat16)
    case HGA_DTYPE_F16: HGA_AF(__half)
    default: break;
  }
#undef HGA_AF
  return cudaErrorInvalidValue;
}

}  // namespace hga
