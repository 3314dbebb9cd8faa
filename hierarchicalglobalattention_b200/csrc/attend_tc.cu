// Working-set attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Shape: bf16, head_dim 128, chunk 64, group 16.  One CTA per (query chunk n, pair of query heads
// sharing a KV head, batch b): the MMA M dimension is 128 = 2 heads x 64 query rows.  The key
// set of the CTA is the union of both heads' working sets, walked as 16-token "units"
// (one routing group each):
//   current chunk (4 units, causal), keep_last window, keep_first window (both heads see all of
//   them), then the union of the two heads' opened groups (each head sees its own ones from its
//   first-visible row t0 on).
// For every row a unit's visible keys form a prefix (causal: keys j <= t - 16u; otherwise all or
// none), so masking is one count per (row, unit).
// Per 64-key tile (4 units):
//   TMA warp      : K and V of the tile into a 2-stage SW128 smem ring: one 64-row box per
//                   64-column half when the 4 units are consecutive rows (current chunk,
//                   windows), else one 16-row box per unit and half, one lane per box; K and V of
//                   a stage have separate full/empty barriers (K is free once Q.K^T has read it)
//   MMA warp      : S = Q.K^T  (M128 N64, A/B from smem, D in TMEM)
//                   O += P.V   (A = P from its own TMEM columns, B = V from smem as MN-major)
//                   Q.K^T of tile i+1 overwrites S as soon as the softmax warps have read tile i
//                   into registers; P.V(i) reads P, which the softmax writes only after P.V(i-1)
//   4 softmax warps: one thread per query row (TMEM lane), exp2 domain.  Tile 0 (the causal
//                   current chunk) sets the row max; later tiles are exponentiated against it and
//                   take a max pass (and a lazy O rescale) only when a p could exceed 2^8.  Units
//                   that no row of a warp sees are neither loaded from TMEM nor exponentiated.
//                   TMEM loads/stores are warp-collective, so these decisions are per warp.
// Set-up: the shared units (current chunk, windows) need no routing and are written first, so
// their tiles load and score while warps 2-3 build the opened part of the unit table from the
// two heads' lists; the producer and MMA warps wait for the table only past the shared tiles.
// ~105 KB smem and 256 TMEM columns per CTA, so two CTAs share an SM and hide each other's
// serial phases.  Every mbarrier wait is bounded; on timeout the CTA records an error code
// (hga_device_status), lets its copies and MMAs in flight land (bounded), releases its TMEM and
// leaves.
#include "tc_common.cuh"

namespace hga {
namespace tc {

constexpr int kThreads = 192;  // warp0 TMA, warp1 MMA, warps2-5 unit table (2-3), softmax, epilogue
constexpr int kUnitsPerTile = 4;
constexpr int kMaxUnits = 328;  // current 4 + windows <= 64 + opened union <= 256, rounded up to whole tiles
constexpr int kMaxKg = 128;
constexpr uint32_t kTmemCols = 256;
// TMEM columns: S (fp32 scores of one tile), P (its probabilities as packed bf16 pairs, the A
// operand of P.V), O (fp32 accumulator).  P has its own columns, so Q.K^T of the next tile can
// overwrite S as soon as the softmax warps have read it into registers.
constexpr uint32_t kColS = 0, kColP = 64, kColO = 128;

struct Unit {
  int pos;    // first token row of the unit inside the (b, kvh) row block
  int tmin0;  // first visible query row for head 0 (>= 64: never)
  int tmin1;  // same for head 1
  int causal; // 1: key j of the unit is visible to row t iff t >= tmin + j
};

struct SmemLayout {
  static constexpr int kQ = 0;              // 2 x 16 KB (dh halves), rows 0..127
  static constexpr int kStage = 32768;      // 2 stages x (K 2x8KB + V 2x8KB)
  static constexpr int kStageBytes = 32768;
  static constexpr int kUnits = kStage + 2 * kStageBytes;
  static constexpr int kLists = kUnits + kMaxUnits * 16;  // [4][kMaxKg] ints: gid0, t00, gid1, t01
  static constexpr int kBars = kLists + 4 * kMaxKg * 4;
  static constexpr int kMisc = kBars + 16 * 8;  // 16 mbarriers
  static constexpr int kTotal = kMisc + 64;
};

struct Args {
  int S, H, KVH, N, Kg, keep_first, keep_last, out_layout, q_layout;
  int chunk0, nl, sq;  // query chunks [chunk0, chunk0 + nl); q / out hold sq rows per batch entry
  int64_t kv_cap;
  float scale_log2;
  const int32_t* open_gid;
  const int32_t* open_t0;
  __nv_bfloat16* out;
  unsigned long long wait_ns;  // limit of every bounded wait
  int fault;                   // test-only: 1 = the CTA of the last query chunk, heads 0-1, batch 0, does not load K of its tile 1
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// sm_100 paired fp32 arithmetic (one instruction for two lanes of work, same rounding as the
// scalar forms) and the three-input max
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unf2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Row max of one S tile (r: the row's 64 scores, 4 units of 16) over the keys the row sees.
// CAUSAL (the current chunk's tile): key j of unit u is visible iff j < cnt[u]; otherwise a unit
// is seen whole (cnt 16) or not at all (cnt 0).  Dead units (no row of the warp sees them) are
// skipped.  Three-input max in a tree of depth 3 per unit.
template <bool CAUSAL>
__device__ __forceinline__ float tile_max(const uint32_t (&r)[64], const int (&cnt)[kUnitsPerTile], unsigned live) {
  float mx = -INFINITY;
#pragma unroll
  for (int u = 0; u < kUnitsPerTile; ++u) {
    if (!(live >> u & 1)) continue;
    float x[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      x[j] = __uint_as_float(r[u * 16 + j]);
      if constexpr (CAUSAL) x[j] = j < cnt[u] ? x[j] : -INFINITY;
    }
    const float a = max3(x[0], x[1], x[2]), b = max3(x[3], x[4], x[5]), c = max3(x[6], x[7], x[8]);
    const float d = max3(x[9], x[10], x[11]), e = max3(x[12], x[13], x[14]);
    const float mu = fmaxf(max3(a, b, c), max3(d, e, x[15]));
    mx = fmaxf(mx, (CAUSAL || cnt[u] > 0) ? mu : -INFINITY);
  }
  return mx;
}

// P = 2^(s * scale_log2 - m) of one S tile as packed bf16 pairs (pk, 32 words = the 64 keys) and
// its row sum added to ps (two paired fp32 partial sums).  Invisible keys get exactly 0.
template <bool CAUSAL>
__device__ __forceinline__ void tile_exp(const uint32_t (&r)[64], const int (&cnt)[kUnitsPerTile], unsigned live,
                                         uint64_t sl2x2, uint64_t nmx2, uint32_t (&pk)[32], uint64_t& ps) {
#pragma unroll
  for (int u = 0; u < kUnitsPerTile; ++u) {
    if (!(live >> u & 1)) {
#pragma unroll
      for (int w = 0; w < 8; ++w) pk[u * 8 + w] = 0u;
      continue;
    }
    uint64_t s2 = f2(0.f, 0.f);
    uint32_t w8[8];
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      float x0 = __uint_as_float(r[u * 16 + j]), x1 = __uint_as_float(r[u * 16 + j + 1]);
      if constexpr (CAUSAL) {
        // prefix-visible keys: an invisible key's exponent is -inf, which ex2 maps to exactly 0
        x0 = j < cnt[u] ? x0 : -INFINITY;
        x1 = j + 1 < cnt[u] ? x1 : -INFINITY;
      }
      float y0, y1;
      unf2(fma2(f2(x0, x1), sl2x2, nmx2), y0, y1);
      const float p0 = ex2(y0), p1 = ex2(y1);
      s2 = add2(s2, f2(p0, p1));
      w8[j >> 1] = pack_bf16(p0, p1);
    }
    if constexpr (CAUSAL) {
#pragma unroll
      for (int w = 0; w < 8; ++w) pk[u * 8 + w] = w8[w];
      ps = add2(ps, s2);
    } else {
      // whole-or-nothing units: every key was computed; rows that see none of them get zeros
      const bool v = cnt[u] > 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) pk[u * 8 + w] = v ? w8[w] : 0u;
      ps = v ? add2(ps, s2) : ps;
    }
  }
}

__global__ void __launch_bounds__(kThreads, 2)
    attend_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_k64,
                     const __grid_constant__ CUtensorMap tm_v64, const Args a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int ln = blockIdx.x, hp = blockIdx.y, b = blockIdx.z;
  const int n = a.chunk0 + ln;
  const int h0 = 2 * hp, h1 = h0 + 1;
  const int kvh = h0 / (a.H / a.KVH);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int C = 64, gs = 16;
  const int row0 = n * C;       // absolute first row (keys, causality)
  const int lrow0 = ln * C;     // first row in q / out
  const int nvalid = (a.S - row0) < C ? (a.S - row0) : C;

  Unit* units = reinterpret_cast<Unit*>(smem + SmemLayout::kUnits);
  int* lists = reinterpret_cast<int*>(smem + SmemLayout::kLists);
  int* gidA = lists;
  int* t0A = lists + kMaxKg;
  int* gidB = lists + 2 * kMaxKg;
  int* t0B = lists + 3 * kMaxKg;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::kBars);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]  K and V of a stage have their own barriers: a stage's K is
  uint64_t* k_empty = bars + 3;   // [2]  released when Q.K^T is done, its V only after P.V, so the
  uint64_t* v_full = bars + 5;    // [2]  next K load overlaps the softmax of the current tile
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // Q.K^T of a tile is in S
  uint64_t* s_free = bars + 10;   // the softmax warps have read S (128 arrivals)
  uint64_t* p_full = bars + 11;   // P of a tile is in TMEM (128 arrivals)
  uint64_t* table_ready = bars + 12;  // the opened units are in the table (one arrival)
  uint64_t* pv_done = bars + 13;  // one completion per P.V (its waits are never more than one phase behind)
  uint64_t* o_done = bars + 14;   // single completion after the last P.V (the epilogue's wait)
  uint64_t* drain = bars + 15;    // the MMA issuer's last commit: every MMA it issued has completed
  int* misc = reinterpret_cast<int*>(smem + SmemLayout::kMisc);
  volatile int* abort_flag = misc + 0;
  int* n_units_s = misc + 1;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(misc + 2);
  int* la_s = misc + 3;
  int* lb_s = misc + 4;

  // ---- set-up: barriers, TMEM, unit table -------------------------------------------------
  int f_hi, l_lo;
  windows(n, a.keep_first, a.keep_last, f_hi, l_lo);
  const int n_shared = 4 + 4 * (n - l_lo) + 4 * f_hi;
  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(k_full + i, 1);
      mbar_init(k_empty + i, 1);
      mbar_init(v_full + i, 1);
      mbar_init(v_empty + i, 1);
      mbar_init(i ? s_free : s_full, i ? 128 : 1);
    }
    mbar_init(p_full, 128);
    mbar_init(table_ready, 1);
    mbar_init(pv_done, 1);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_flag = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base_s)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // the shared units (current chunk and windows) need no routing: written now, so their tiles
  // load while the softmax warps build the rest of the table from the open lists
  for (int u = tid; u < n_shared; u += kThreads) {
    Unit e;
    if (u < 4) {
      e.pos = row0 + u * gs; e.tmin0 = e.tmin1 = u * gs; e.causal = 1;
    } else if (u < 4 + 4 * (n - l_lo)) {
      e.pos = l_lo * C + (u - 4) * gs; e.tmin0 = e.tmin1 = 0; e.causal = 0;
    } else {
      e.pos = (u - 4 - 4 * (n - l_lo)) * gs; e.tmin0 = e.tmin1 = 0; e.causal = 0;
    }
    units[u] = e;
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_base_s;
  const int ns_tiles = n_shared / kUnitsPerTile;  // n_shared is a multiple of 4
  // number of tiles, read once the table is complete (the producer and the MMA issuer wait for it
  // only when they pass the shared tiles)
  auto table_tiles = [&]() { return (*n_units_s + kUnitsPerTile - 1) / kUnitsPerTile; };
  unsigned char* q_s = smem + SmemLayout::kQ;
  if (warp >= 2) {
    // stage both heads' open lists in smem (coalesced); visible entries are a prefix of each list
    const int st_tid = tid - 64;
    const size_t tile0 = (((size_t)b * a.H + h0) * a.nl + ln) * a.Kg;
    const size_t tile1 = (((size_t)b * a.H + h1) * a.nl + ln) * a.Kg;
    for (int i = st_tid; i < a.Kg; i += 128) {
      gidA[i] = a.open_gid[tile0 + i];
      t0A[i] = a.open_t0[tile0 + i];
      gidB[i] = a.open_gid[tile1 + i];
      t0B[i] = a.open_t0[tile1 + i];
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (warp == 2) {
      int la = 0, lb = 0;
      for (int base = 0; base < a.Kg; base += 32) {
        const int j = base + lane;
        const bool va = j < a.Kg && gidA[j] >= 0 && t0A[j] < nvalid;
        const bool vb = j < a.Kg && gidB[j] >= 0 && t0B[j] < nvalid;
        la += __popc(__ballot_sync(0xffffffffu, va));
        lb += __popc(__ballot_sync(0xffffffffu, vb));
      }
      if (lane == 0) { *la_s = la; *lb_s = lb; }
    }
    if (warp <= 3) {
      asm volatile("bar.sync 2, 64;" ::: "memory");
      const int la = *la_s, lb = *lb_s;
    // opened groups in three runs: both heads (in head 0's order), head 0 only, head 1 only.  A
    // warp's rows belong to one head, so a run of single-head units leaves the other head's warps
    // whole tiles with nothing visible, which they skip.
    if (warp == 2) {
      int both = 0;
      for (int pass = 0; pass < 2; ++pass) {
        int written = 0;
        for (int base = 0; base < la; base += 32) {
          const int j = base + lane;
          int g = 0, t1 = 1 << 20;
          if (j < la) {
            g = gidA[j];
            int lo = 0, hi = lb - 1;
            while (lo <= hi) {
              const int mid = (lo + hi) >> 1;
              const int x = gidB[mid];
              if (x == g) { t1 = t0B[mid]; break; }
              if (x < g) lo = mid + 1; else hi = mid - 1;
            }
          }
          const bool take = j < la && ((t1 < (1 << 20)) == (pass == 0));
          const unsigned bal = __ballot_sync(0xffffffffu, take);
          if (take) {
            const int slot = n_shared + (pass ? both : 0) + written + __popc(bal & ((1u << lane) - 1u));
            Unit e; e.pos = g * gs; e.tmin0 = t0A[j]; e.tmin1 = t1; e.causal = 0;
            units[slot] = e;
          }
          written += __popc(bal);
        }
        if (pass == 0) both = written;
      }
    }
    if (warp == 3) {
      int written = 0;
      for (int base = 0; base < lb; base += 32) {
        const int j = base + lane;
        bool keep = false;
        int g = 0;
        if (j < lb) {
          g = gidB[j];
          keep = true;
          int lo = 0, hi = la - 1;
          while (lo <= hi) {
            const int mid = (lo + hi) >> 1;
            const int x = gidA[mid];
            if (x == g) { keep = false; break; }
            if (x < g) lo = mid + 1; else hi = mid - 1;
          }
        }
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (keep) {
          const int slot = n_shared + la + written + __popc(bal & ((1u << lane) - 1u));
          Unit e; e.pos = g * gs; e.tmin0 = 1 << 20; e.tmin1 = t0B[j]; e.causal = 0;
          units[slot] = e;
        }
        written += __popc(bal);
      }
      if (lane == 0) *n_units_s = n_shared + la + written;
    }
      asm volatile("bar.sync 2, 64;" ::: "memory");  // warp 2's units are written
      if (warp == 3) {
        // pad the last tile with never-visible copies of unit 0 (finite data, zero probability)
        const int nu = *n_units_s, nt = (nu + kUnitsPerTile - 1) / kUnitsPerTile;
        for (int u = nu + lane; u < nt * kUnitsPerTile; u += 32) {
          Unit e = units[0]; e.tmin0 = e.tmin1 = 1 << 20; e.causal = 0;
          units[u] = e;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(table_ready);
      }
    }
  }
  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------------
    // The whole warp runs the loop: lane 0 arms the barriers, lanes 0-7 issue a tile's eight 2 KB
    // boxes (four units x two 64-column halves, one box each), so they are in flight together
    if (lane == 0) {
      mbar_expect_tx(q_full, 32768);
      for (int hh = 0; hh < 2; ++hh)
        for (int kb = 0; kb < 2; ++kb) {
          unsigned char* dst = q_s + kb * 16384 + hh * 8192;
          if (a.q_layout == 1) tma_load_3d(dst, &tm_q, kb * 64, h0 + hh, b * a.sq + lrow0, q_full);
          else tma_load_2d(dst, &tm_q, kb * 64, (b * a.H + h0 + hh) * a.sq + lrow0, q_full);
        }
    }
    const int64_t kvrow = ((int64_t)b * a.KVH + kvh) * a.kv_cap;
    // K of tile i+1 is issued before V of tile i: Q.K^T(i-1), which frees K's stage, completes
    // before P.V(i-2), which frees V's
    int armed_k0 = 0, armed_k1 = 0, armed_v0 = 0, armed_v1 = 0;  // loads issued per kind and stage: the drain's phases
    const bool skip_k1 = a.fault == 1 && blockIdx.x == gridDim.x - 1 && blockIdx.y == 0 && blockIdx.z == 0 && ns_tiles > 2;
    auto load = [&](int i, bool is_v) -> bool {
      const int st = i & 1;
      if (skip_k1 && !is_v && i == 1) return true;  // test-only fault: tile 1's K never arrives
      uint64_t* empty = is_v ? v_empty : k_empty;
      uint64_t* full = is_v ? v_full : k_full;
      if (i >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait(empty + st, ((i >> 1) - 1) & 1, abort_flag, is_v ? 9 : 1, a.wait_ns)))
        return false;
      unsigned char* dst = smem + SmemLayout::kStage + st * SmemLayout::kStageBytes + (is_v ? 16384 : 0);
      if (lane == 0) mbar_expect_tx(full + st, 16384);
      // a tile of four consecutive units (the current chunk, the windows) is one 64-row box per
      // half; the smem image is the same as four 16-row boxes (the swizzle follows the address)
      const Unit* tu = units + i * kUnitsPerTile;
      const bool contiguous = tu[1].pos == tu[0].pos + 16 && tu[2].pos == tu[0].pos + 32 && tu[3].pos == tu[0].pos + 48;
      if (contiguous) {
        if (lane < 2) tma_load_2d(dst + lane * 8192, is_v ? &tm_v64 : &tm_k64, lane * 64, (int)(kvrow + tu[0].pos), full + st);
      } else if (lane < 2 * kUnitsPerTile) {
        const int u = lane >> 1, hf = lane & 1;
        tma_load_2d(dst + hf * 8192 + u * 2048, is_v ? &tm_v : &tm_k, hf * 64, (int)(kvrow + tu[u].pos), full + st);
      }
      if (is_v) (st ? armed_v1 : armed_v0) += 1;
      else (st ? armed_k1 : armed_k0) += 1;
      return true;
    };
    int nt = -1;  // tiles of the whole table, known once it is complete
    auto has_tile = [&](int i) -> bool {  // false past the last tile, or when the wait for the table gave up
      if (i < ns_tiles) return true;
      if (nt < 0) {
        if (!__all_sync(0xffffffffu, mbar_wait(table_ready, 0, abort_flag, 11, a.wait_ns))) return false;
        nt = table_tiles();
      }
      return i < nt;
    };
    bool go = load(0, false);  // tile 0 (the current chunk) always exists
    for (int i = 0; go; ++i) {
      const bool more = has_tile(i + 1);
      if (more) go = load(i + 1, false);
      if (go) go = load(i, true);
      if (!more) break;
    }
    // drain: a CTA that gives up must not release its shared memory under loads still in flight
    if (lane == 0)
      for (int st = 0; st < 2; ++st) {
        const int nk = st ? armed_k1 : armed_k0, nv = st ? armed_v1 : armed_v0;
        if (nk > 0) mbar_drain(k_full + st, (nk - 1) & 1);
        if (nv > 0) mbar_drain(v_full + st, (nv - 1) & 1);
      }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer ---------------------------------------------
    if (lane == 0) {
      // S: M=128, N=64, B K-major.  O: M=128, N=128, B (V) MN-major.
      const uint32_t id_qk = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
      const uint32_t id_pv = idesc_bf16(true);
      const uint32_t q_addr = smem_u32(q_s);
      bool ok = mbar_wait(q_full, 0, abort_flag, 2, a.wait_ns);
      fence_after();
      int nt = -1;  // tiles of the whole table, known once it is complete
      for (int i = 0; ok; ++i) {
        bool si = i < ns_tiles;
        if (!si) {
          if (nt < 0) {
            if (!mbar_wait(table_ready, 0, abort_flag, 11, a.wait_ns)) break;
            nt = table_tiles();
          }
          si = i < nt;
        }
        if (si) {
          const int st = i & 1;
          if (!mbar_wait(k_full + st, (i >> 1) & 1, abort_flag, 3, a.wait_ns)) break;
          // S is free once the softmax warps have read the previous tile's scores
          if (i >= 1 && !mbar_wait(s_free, (i - 1) & 1, abort_flag, 4, a.wait_ns)) break;
          fence_after();
          const uint32_t k_addr = smem_u32(smem + SmemLayout::kStage + st * SmemLayout::kStageBytes);
          const uint32_t d = tmem + kColS;
          for (int kb = 0; kb < 2; ++kb)
            for (int kk = 0; kk < 4; ++kk)
              mma_ss(d, sdesc(q_addr + kb * 16384 + kk * 32, 16, 1024), sdesc(k_addr + kb * 8192 + kk * 32, 16, 1024),
                     id_qk, (kb | kk) != 0);
          mma_commit(s_full);
          mma_commit(k_empty + st);
        }
        if (i >= 1) {
          const int j = i - 1, st = j & 1;
          if (!mbar_wait(p_full, j & 1, abort_flag, 5, a.wait_ns)) break;
          if (!mbar_wait(v_full + st, (j >> 1) & 1, abort_flag, 10, a.wait_ns)) break;
          fence_after();
          const uint32_t v_addr = smem_u32(smem + SmemLayout::kStage + st * SmemLayout::kStageBytes + 16384);
          const uint32_t p_col = tmem + kColP;
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + kColO, p_col + kk * 8, sdesc(v_addr + kk * 2048, 8192, 1024), id_pv,
                   (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(pv_done);
          mma_commit(v_empty + st);
          if (!si) mma_commit(o_done);  // P.V of the last tile
        }
        if (!si) break;
      }
      // drain: wait until every MMA this thread issued has completed (it reads smem and TMEM that
      // are released below), also when the loop was left on a timeout
      mma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // ------------------------------- softmax / epilogue -------------------------------------
    // tcgen05.ld / st are warp-collective (.sync.aligned): every branch around them is warp-uniform
    const int quarter = warp & 3;          // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;   // 0..127
    const int head_sel = row >> 6;         // 0 -> h0, 1 -> h1
    const int t = row & 63;
    const bool rvalid = t < nvalid;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const float sl2 = a.scale_log2;
    float m_run = -INFINITY;  // running max in the scaled log2 domain
    float l_run = 0.f;
    // the table (built by warps 2 and 3) gives the tile count
    bool ok = __all_sync(0xffffffffu, mbar_wait(table_ready, 0, abort_flag, 11, a.wait_ns));
    const int ntiles = ok ? table_tiles() : 0;
    for (int i = 0; i < ntiles && ok; ++i) {
      // visibility of the tile's units for this row: a visible prefix of cnt[u] keys (the causal
      // current-chunk tile, i == 0) or all / none of them; `live` marks the units some row of this
      // warp sees (the others are neither loaded nor exponentiated)
      int cnt[kUnitsPerTile];
      unsigned live = 0;
#pragma unroll
      for (int u = 0; u < kUnitsPerTile; ++u) {
        const Unit e = units[i * kUnitsPerTile + u];
        const int tmin = head_sel ? e.tmin1 : e.tmin0;
        int c = e.causal ? t - tmin + 1 : (t >= tmin ? 16 : 0);
        c = c < 0 ? 0 : (c > 16 ? 16 : c);
        cnt[u] = rvalid ? c : 0;
        if (__any_sync(0xffffffffu, cnt[u] > 0)) live |= 1u << u;
      }
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, i & 1, abort_flag, 6, a.wait_ns));
      if (!ok) break;
      fence_after();
      const uint32_t s_addr = tmem + lane_addr + kColS;
      uint32_t r[64];
#pragma unroll
      for (int u = 0; u < kUnitsPerTile; ++u)
        if (live >> u & 1) HGA_LD16(s_addr + u * 16, (r + u * 16));
      if (live) tmem_wait_ld();
      // the scores are in registers: the next tile's Q.K^T may overwrite S
      fence_before();
      mbar_arrive(s_free);
      bool pv_waited = i == 0;  // P.V(i-1) has completed (P's columns and O may be written)
      // Tile 0 (the causal current chunk, where every valid row sees at least its own key) sets
      // the running max.  Later tiles are exponentiated against the running max directly; only
      // when a p could exceed 2^8 (the row's tile sum is above 2^8, or not finite) does the warp
      // take the max pass and, if the max grew by more than 2^8, rescale O (lazy rescaling).
      uint32_t pk[32];
      uint64_t ps = f2(0.f, 0.f);                            // paired partial row sums
      const uint64_t sl2x2 = f2(sl2, sl2);
      bool redo = i == 0;
      if (i > 0) {
        const float nm = m_run == -INFINITY ? 0.f : -m_run;
        tile_exp<false>(r, cnt, live, sl2x2, f2(nm, nm), pk, ps);
        float q0, q1;
        unf2(ps, q0, q1);
        redo = __any_sync(0xffffffffu, !(q0 + q1 <= 256.f));
      }
      if (redo) {
        const float mx = i == 0 ? tile_max<true>(r, cnt, live) : tile_max<false>(r, cnt, live);
        const float m_tile = mx * sl2;
        float alpha = 1.f;
        bool rescale_o = false;
        if (m_tile > m_run + 8.f) {
          if (m_run != -INFINITY) {
            alpha = ex2(m_run - m_tile);
            l_run *= alpha;
            rescale_o = true;
          }
          m_run = m_tile;
        }
        if (__any_sync(0xffffffffu, rescale_o)) {
          // O holds the sum over tiles < i: wait for the last P.V, then rescale (alpha = 1 elsewhere)
          ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (i - 1) & 1, abort_flag, 7, a.wait_ns));
          if (!ok) break;
          pv_waited = true;
          fence_after();
          const uint32_t o_addr = tmem + lane_addr + kColO;
#pragma unroll 1
          for (int c0 = 0; c0 < 128; c0 += 16) {
            uint32_t o[16];
            HGA_LD16(o_addr + c0, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            HGA_ST16(o_addr + c0, o);
          }
          tmem_wait_st();
        }
        const float nm = m_run == -INFINITY ? 0.f : -m_run;  // no visible key yet: every p is 0
        ps = f2(0.f, 0.f);
        if (i == 0) tile_exp<true>(r, cnt, live, sl2x2, f2(nm, nm), pk, ps);
        else tile_exp<false>(r, cnt, live, sl2x2, f2(nm, nm), pk, ps);
      }
      float ps0, ps1;
      unf2(ps, ps0, ps1);
      l_run += ps0 + ps1;
      if (!pv_waited) {  // P.V(i-1) still reads P's columns
        ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (i - 1) & 1, abort_flag, 4, a.wait_ns));
        if (!ok) break;
        fence_after();
      }
      HGA_ST32(tmem + lane_addr + kColP, pk);
      tmem_wait_st();
      fence_before();
      mbar_arrive(p_full);
    }
    // epilogue
    if (ok && ntiles > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_done, 0, abort_flag, 8, a.wait_ns));
    if (ok) {
      fence_after();
      const int h = head_sel ? h1 : h0;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const uint32_t o_addr = tmem + lane_addr + kColO;
      __nv_bfloat16* dst = nullptr;
      if (rvalid) {
        const int64_t tt = lrow0 + t;
        dst = a.out_layout == 1 ? a.out + (((int64_t)b * a.sq + tt) * a.H + h) * 128
                                : a.out + (((int64_t)b * a.H + h) * a.sq + tt) * 128;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < 128; c0 += 16) {
        uint32_t o[16];
        HGA_LD16(o_addr + c0, o);
        tmem_wait_ld();
        if (dst) {
          uint32_t w[8];
#pragma unroll
          for (int c = 0; c < 8; ++c)
            w[c] = pack_bf16(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv);
          uint4* d4 = reinterpret_cast<uint4*>(dst + c0);
          d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
          d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

}  // namespace tc

// test-only failure injection (hga_debug_fault): read by the next launch
static int g_test_fault = 0;
static long long g_test_wait_ns = 0;
void attend_tc_set_test_fault(int mode, long long wait_ns) {
  g_test_fault = mode;
  g_test_wait_ns = wait_ns;
}

bool attend_tc_supported(const hga_params& p) {
  return p.dtype == HGA_DTYPE_BF16 && p.head_dim == 128 && p.chunk_size == 64 && p.group_size == 16 &&
         (p.nhead / p.kv_heads) % 2 == 0 && p.keep_last <= 1 << 20 && p.keep_first <= 1 << 20;
}

cudaError_t launch_attend_tc(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout, const void* k_rope,
                             const void* v, int64_t kv_cap, const int32_t* open_gid, const int32_t* open_t0, int Kg,
                             void* out, int out_layout, cudaStream_t st) {
  using namespace tc;
  const int N = (int)((S + 63) / 64);
  // windows wider than the unit table hold go through the portable kernel
  const int kl = p.keep_last < N ? p.keep_last : N, kf = p.keep_first < N ? p.keep_first : N;
  if (kl + kf > 16 || Kg > kMaxKg) return cudaErrorNotSupported;
  if ((int64_t)p.batch * p.kv_heads * kv_cap >= (1ll << 31)) return cudaErrorNotSupported;
  if (((uintptr_t)q | (uintptr_t)k_rope | (uintptr_t)v | (uintptr_t)out) & 15) return cudaErrorMisalignedAddress;
  CUtensorMap mq, mk, mv;
  const cuuint64_t rows_kv = (cuuint64_t)p.batch * p.kv_heads * kv_cap;
  const cuuint64_t dkv[2] = {128, rows_kv}, skv[1] = {256};
  const cuuint32_t bkv[2] = {64, 16};
  if (!make_map(&mk, k_rope, 2, dkv, skv, bkv) || !make_map(&mv, v, 2, dkv, skv, bkv)) return cudaErrorInvalidValue;
  CUtensorMap mk64, mv64;
  const cuuint32_t bkv64[2] = {64, 64};
  if (!make_map(&mk64, k_rope, 2, dkv, skv, bkv64) || !make_map(&mv64, v, 2, dkv, skv, bkv64)) return cudaErrorInvalidValue;
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
  Args a;
  a.chunk0 = qr.chunk0; a.nl = qr.count; a.sq = (int)qr.sq;
  a.S = (int)S; a.H = p.nhead; a.KVH = p.kv_heads; a.N = N; a.Kg = Kg;
  a.keep_first = p.keep_first; a.keep_last = p.keep_last; a.out_layout = out_layout; a.q_layout = q_layout;
  a.kv_cap = kv_cap;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.open_gid = open_gid; a.open_t0 = open_t0;
  a.out = (__nv_bfloat16*)out;
  a.wait_ns = g_test_wait_ns > 0 ? (unsigned long long)g_test_wait_ns : kWaitLimitNs;
  a.fault = g_test_fault;
  g_test_fault = 0;  // the fault and its wait limit hold for one launch
  g_test_wait_ns = 0;
  const int smem = SmemLayout::kTotal + 1024;
  cudaError_t e = cudaFuncSetAttribute(attend_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(qr.count, p.nhead / 2, p.batch);
  attend_tc_kernel<<<grid, kThreads, smem, st>>>(mq, mk, mv, mk64, mv64, a);
  return cudaGetLastError();
}

HGA_DEFINE_ERROR_READER(tc_error_status)

}  // namespace hga
