// extern "C" entry points of libhga_b200.so: argument validation, dispatch, error reporting.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "hga_common.cuh"

namespace hga {
cudaError_t launch_summaries(const hga_params& p, int64_t S, int64_t pos0, const void* k_raw, const void* k_rope,
                             const void* v, int64_t kv_cap, const void* cos, const void* sin, int rot_dtype,
                             int64_t rot_row0, void* ck, void* gk, void* gv, int64_t sum_cap, int64_t out_chunk0,
                             cudaStream_t st);
bool summaries_dual_supported(const hga_params& p);
cudaError_t launch_summaries_dual(const hga_params& p, int64_t S, int64_t pos0, const void* k_raw,
                                  const void* k_rope, const void* v, int64_t kv_cap, const float* cosA,
                                  const float* sinA, int64_t rowA0, int roundA, void* ckA, void* gkA,
                                  int64_t capA, int64_t outA0, const float* cosB, const float* sinB,
                                  int64_t rowB0, int nB, void* ckB, void* gkB, void* gvB, int64_t capB,
                                  int64_t outB0, cudaStream_t st);
cudaError_t launch_bank_gather(const hga_params& p, const int32_t* open_gid, int Kg, const void* rec_k,
                               const void* rec_v, int64_t rec_cap, void* bank_k, void* bank_v, int n_slots,
                               int32_t* slot_gid, int32_t* gid_slot, int64_t gid_cap, int32_t* slot_stamp, int stamp,
                               int32_t* open_slot, unsigned long long* counters, cudaStream_t st);
cudaError_t launch_route_prefill(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout, const void* ck,
                                 const void* gk, int64_t sum_cap, int32_t* sel_chunk, int32_t* sel_t0,
                                 int32_t* open_gid, int32_t* open_t0, float* dbg1, float* dbg2, cudaStream_t st,
                                 int* smem_bytes_out);
cudaError_t launch_attend_simt(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout, const void* k_rope,
                               const void* v, int64_t kv_cap, const int32_t* open_gid, const int32_t* open_t0,
                               int Kg, void* out, int out_layout, cudaStream_t st);
cudaError_t launch_prologue(const hga_params& p, int64_t S, const void* qkv, int64_t row_stride, const void* qw,
                            const void* kw, float eps, int norm_mode, const void* cos, const void* sin,
                            int rope_mode, int64_t rot_row0, int64_t pos0, void* q_out, void* kraw_out,
                            void* krope_out, void* v_out, int64_t kv_cap, int64_t kv_row0, cudaStream_t st);
bool attend_tc_supported(const hga_params& p);
cudaError_t launch_attend_tc(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout, const void* k_rope,
                             const void* v, int64_t kv_cap, const int32_t* open_gid, const int32_t* open_t0,
                             int Kg, void* out, int out_layout, cudaStream_t st);
int tc_error_status(bool clear);
void attend_tc_set_test_fault(int mode, long long wait_ns);
int route_tc_error_status(bool clear);
bool route_tc_supported(const hga_params& p, int64_t S);
cudaError_t launch_route_tc(const hga_params& p, int64_t S, const QRange& qr, const void* q, int q_layout, const void* ck, const void* gk,
                            int64_t sum_cap, int32_t* sel_chunk, int32_t* sel_t0, int32_t* open_gid, int32_t* open_t0,
                            float* dbg1, float* dbg2, cudaStream_t st);
cudaError_t launch_route_decode(const hga_params& p, int L, const void* q, const int32_t* seq_pos, const void* ck,
                                const void* gk, int64_t sum_cap, int nmid_max, int Kcmax, int Kgmax, int32_t* mc,
                                int32_t* mt, int32_t* og, int32_t* ot, cudaStream_t st);
cudaError_t launch_attend_decode(const hga_params& p, int L, const void* q, const int32_t* seq_pos, const void* hk,
                                 const void* hv, int64_t hot_cap, int hot_mode, const void* ckk, const void* cvv,
                                 int64_t cold_cap, const int32_t* og, const int32_t* ot, int Kg, void* out,
                                 cudaStream_t st);
cudaError_t launch_attend_decode_dca(const hga_params& p, int L, const void* q, const int32_t* seq_pos, const void* hk,
                                     const void* hv, int64_t hot_cap, int hot_mode, const void* ckk, const void* cvv,
                                     int64_t cold_cap, const int32_t* og, const int32_t* ot, const int32_t* open_pos,
                                     int Kg, const float* dca_cos, const float* dca_sin, int dca_chunk, int dca_ceil,
                                     void* out, cudaStream_t st);
cudaError_t launch_shard_unpack(const void* recv, int64_t rank_stride, int64_t part_offset, int world, int pieces,
                                const int32_t* dst_block, int64_t bk, int64_t rows, int64_t row_bytes, void* dst,
                                cudaStream_t st);
int decode_error_status(bool clear);
int decode_fast_error_status(bool clear);
bool route_decode1_supported(const hga_params& p, int L);
cudaError_t launch_route_decode1(const hga_params& p, const void* q, const int32_t* seq_pos, const void* ck,
                                 const void* gk, int64_t sum_cap, int nmid_max, int Kcmax, int Kgmax, int32_t* mc,
                                 int32_t* mt, int32_t* og, int32_t* ot, cudaStream_t st);
bool attend_decode_fast_supported(const hga_params& p, int L);
cudaError_t launch_attend_decode_fast(const hga_params& p, int L, const void* q, const int32_t* seq_pos,
                                      const void* hk, const void* hv, int64_t hot_cap, int hot_mode, const void* ckk,
                                      const void* cvv, int64_t cold_cap, const int32_t* og, const int32_t* ot, int Kg,
                                      void* out, cudaStream_t st);
cudaError_t launch_append(const hga_params& p, int L, const int32_t* seq_pos, const void* kr, const void* v,
                          const void* kraw, void* hk, void* hv, int64_t hot_cap, int hot_mode, void* ck, void* cv,
                          int64_t cold_cap, void* act_raw, cudaStream_t st);
}  // namespace hga

static thread_local char g_err[512];

static int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return HGA_OK;
  if (e == cudaErrorInvalidConfiguration)
    return fail(HGA_E_UNSUPPORTED, "%s: shape needs more shared memory than one CTA can hold", what);
  return fail(HGA_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static int check_params(const hga_params* p) {
  if (!p) return fail(HGA_E_INVALID, "params is NULL");
  if (p->batch <= 0 || p->nhead <= 0 || p->kv_heads <= 0 || p->head_dim <= 0)
    return fail(HGA_E_INVALID, "batch/nhead/kv_heads/head_dim must be positive");
  if (p->nhead % p->kv_heads) return fail(HGA_E_INVALID, "nhead %% kv_heads != 0");
  if (p->head_dim % 2 || p->head_dim > 256) return fail(HGA_E_UNSUPPORTED, "head_dim must be even and <= 256");
  if (p->chunk_size <= 0 || p->group_size <= 0 || p->chunk_size % p->group_size)
    return fail(HGA_E_INVALID, "chunk_size must be a positive multiple of group_size");
  if (p->chunk_size > 128) return fail(HGA_E_UNSUPPORTED, "chunk_size > 128 is not supported");
  if (p->dtype < HGA_DTYPE_F32 || p->dtype > HGA_DTYPE_F16) return fail(HGA_E_INVALID, "unknown dtype %d", p->dtype);
  return HGA_OK;
}

static int route_sizes(const hga_params* p, int64_t S, int* Kc, int* Kg) {
  const int C = p->chunk_size, M = C / p->group_size;
  const int64_t N = (S + C - 1) / C;
  *Kc = p->topk_chunks > 0 ? (int)(p->topk_chunks < N ? p->topk_chunks : N) : 0;
  const int Tg = *Kc * M;
  int kg = p->topk_groups > 0 ? (p->topk_groups < Tg ? p->topk_groups : Tg) : 0;
  const int kgr = p->topk_groups > 0 ? ((p->topk_groups / 2) < Tg ? p->topk_groups / 2 : Tg) : 0;
  if (kgr == 0) kg = 0;
  *Kg = kg;
  return 0;
}

extern "C" {

int hga_route_prefill_impl(const hga_params* p, int64_t seq_len, const void* q, int32_t q_layout, const void* chunk_k,
                           const void* group_k, int64_t sum_cap, int32_t* sel_chunk, int32_t* sel_t0,
                           int32_t* open_gid, int32_t* open_t0, float* dbg_l1, float* dbg_l2, int32_t impl,
                           cudaStream_t stream);

int hga_route_prefill_range(const hga_params* p, int64_t seq_len, int64_t chunk_lo, int64_t chunk_hi, const void* q,
                            int32_t q_layout, const void* chunk_k, const void* group_k, int64_t sum_cap,
                            int32_t* sel_chunk, int32_t* sel_t0, int32_t* open_gid, int32_t* open_t0, float* dbg_l1,
                            float* dbg_l2, int32_t impl, cudaStream_t stream);
int hga_attend_prefill_range(const hga_params* p, int64_t seq_len, int64_t chunk_lo, int64_t chunk_hi, const void* q,
                             int32_t q_layout, const void* k_rope, const void* v, int64_t kv_cap,
                             const int32_t* open_gid, const int32_t* open_t0, void* out, int32_t out_layout,
                             int32_t impl, cudaStream_t stream);

const char* hga_version(void) { return "hga_b200 0.1 (sm_100a)"; }
const char* hga_last_error(void) { return g_err; }

int hga_summaries(const hga_params* p, int64_t seq_len, int64_t pos0, const void* k_raw, const void* k_rope,
                  const void* v, int64_t kv_cap, const void* cos, const void* sin, int32_t rot_mode,
                  int64_t rot_row0, void* chunk_k, void* group_k, void* group_v, int64_t sum_cap,
                  int64_t out_chunk0, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (seq_len <= 0) return HGA_OK;
  if (!k_raw || !k_rope || !v || !cos || !sin || !chunk_k || !group_k)
    return fail(HGA_E_INVALID, "hga_summaries: NULL tensor");
  if (kv_cap < seq_len) return fail(HGA_E_INVALID, "hga_summaries: kv_cap < seq_len");
  if (pos0 % p->chunk_size) return fail(HGA_E_INVALID, "hga_summaries: pos0 must be chunk aligned");
  if (pos0 < rot_row0) return fail(HGA_E_INVALID, "hga_summaries: rotary table starts after pos0");
  const int64_t N = (seq_len + p->chunk_size - 1) / p->chunk_size;
  if (out_chunk0 < 0 || out_chunk0 + N > sum_cap) return fail(HGA_E_INVALID, "hga_summaries: summary capacity too small");
  if (rot_mode < HGA_ROT_F32 || rot_mode > HGA_ROT_F32_ROUNDED)
    return fail(HGA_E_INVALID, "hga_summaries: unknown rot_mode %d", rot_mode);
  return cuda_status(hga::launch_summaries(*p, seq_len, pos0, k_raw, k_rope, v, kv_cap, cos, sin, rot_mode, rot_row0,
                                           chunk_k, group_k, group_v, sum_cap, out_chunk0, stream),
                     "hga_summaries");
}

int hga_summaries_dual(const hga_params* p, int64_t seq_len, int64_t pos0, const void* k_raw, const void* k_rope,
                       const void* v, int64_t kv_cap, const float* cos_a, const float* sin_a, int64_t rot_row0_a,
                       int32_t round_a, void* chunk_a, void* group_a, int64_t sum_cap_a, int64_t out_a0,
                       const float* cos_b, const float* sin_b, int64_t rot_row0_b, int64_t n_b, void* chunk_b,
                       void* group_b, void* group_vb, int64_t sum_cap_b, int64_t out_b0, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (seq_len <= 0) return HGA_OK;
  if (!hga::summaries_dual_supported(*p))
    return fail(HGA_E_UNSUPPORTED, "hga_summaries_dual: needs bf16/fp16, head_dim 64/128, chunk/group multiples of 16");
  if (!k_raw || !k_rope || !v || !cos_a || !sin_a || !chunk_a || !group_a)
    return fail(HGA_E_INVALID, "hga_summaries_dual: NULL tensor");
  if (kv_cap < seq_len) return fail(HGA_E_INVALID, "hga_summaries_dual: kv_cap < seq_len");
  if (pos0 % p->chunk_size) return fail(HGA_E_INVALID, "hga_summaries_dual: pos0 must be chunk aligned");
  const int64_t N = (seq_len + p->chunk_size - 1) / p->chunk_size;
  if (pos0 < rot_row0_a || out_a0 < 0 || out_a0 + N > sum_cap_a)
    return fail(HGA_E_INVALID, "hga_summaries_dual: set A table or capacity out of range");
  if (n_b < 0 || n_b > seq_len / p->chunk_size) return fail(HGA_E_INVALID, "hga_summaries_dual: n_b beyond the closed chunks");
  if (n_b > 0 && (!cos_b || !sin_b || !chunk_b || !group_b || pos0 < rot_row0_b || out_b0 < 0 || out_b0 + n_b > sum_cap_b))
    return fail(HGA_E_INVALID, "hga_summaries_dual: set B tensors, table or capacity out of range");
  if ((((uintptr_t)k_raw | (uintptr_t)k_rope | (uintptr_t)v | (uintptr_t)chunk_a | (uintptr_t)group_a |
        (uintptr_t)chunk_b | (uintptr_t)group_b | (uintptr_t)group_vb | (uintptr_t)cos_a | (uintptr_t)sin_a |
        (uintptr_t)cos_b | (uintptr_t)sin_b) & 15))
    return fail(HGA_E_INVALID, "hga_summaries_dual: pointers must be 16-byte aligned");
  return cuda_status(hga::launch_summaries_dual(*p, seq_len, pos0, k_raw, k_rope, v, kv_cap, cos_a, sin_a, rot_row0_a,
                                                round_a, chunk_a, group_a, sum_cap_a, out_a0, cos_b, sin_b,
                                                rot_row0_b, (int)n_b, chunk_b, group_b, group_vb, sum_cap_b, out_b0,
                                                stream),
                     "hga_summaries_dual");
}

int hga_route_prefill(const hga_params* p, int64_t seq_len, const void* q, int32_t q_layout, const void* chunk_k,
                      const void* group_k, int64_t sum_cap, int32_t* sel_chunk, int32_t* sel_t0, int32_t* open_gid,
                      int32_t* open_t0, float* dbg_l1, float* dbg_l2, cudaStream_t stream) {
  return hga_route_prefill_impl(p, seq_len, q, q_layout, chunk_k, group_k, sum_cap, sel_chunk, sel_t0, open_gid,
                                open_t0, dbg_l1, dbg_l2, 0, stream);
}

int hga_route_prefill_impl(const hga_params* p, int64_t seq_len, const void* q, int32_t q_layout, const void* chunk_k,
                           const void* group_k, int64_t sum_cap, int32_t* sel_chunk, int32_t* sel_t0,
                           int32_t* open_gid, int32_t* open_t0, float* dbg_l1, float* dbg_l2, int32_t impl,
                           cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (seq_len <= 0) return HGA_OK;
  const int64_t N = (seq_len + p->chunk_size - 1) / p->chunk_size;
  return hga_route_prefill_range(p, seq_len, 0, N, q, q_layout, chunk_k, group_k, sum_cap, sel_chunk, sel_t0,
                                 open_gid, open_t0, dbg_l1, dbg_l2, impl, stream);
}

int hga_route_prefill_range(const hga_params* p, int64_t seq_len, int64_t chunk_lo, int64_t chunk_hi, const void* q,
                            int32_t q_layout, const void* chunk_k, const void* group_k, int64_t sum_cap,
                            int32_t* sel_chunk, int32_t* sel_t0, int32_t* open_gid, int32_t* open_t0, float* dbg_l1,
                            float* dbg_l2, int32_t impl, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (seq_len <= 0) return HGA_OK;
  int Kc, Kg;
  route_sizes(p, seq_len, &Kc, &Kg);
  if (!q || !chunk_k || !group_k) return fail(HGA_E_INVALID, "hga_route_prefill: NULL tensor");
  if ((Kc && (!sel_chunk || !sel_t0)) || (Kg && (!open_gid || !open_t0)))
    return fail(HGA_E_INVALID, "hga_route_prefill: NULL output list");
  if (q_layout != 0 && q_layout != 1) return fail(HGA_E_INVALID, "q_layout must be 0 or 1");
  const int64_t N = (seq_len + p->chunk_size - 1) / p->chunk_size;
  if (chunk_lo < 0 || chunk_hi > N || chunk_lo >= chunk_hi)
    return fail(HGA_E_INVALID, "hga_route_prefill: query chunk range outside [0, N) or empty");
  if (sum_cap < N) return fail(HGA_E_INVALID, "hga_route_prefill: sum_cap < number of chunks");
  if ((int64_t)Kc * (p->chunk_size / p->group_size) > 256)
    return fail(HGA_E_UNSUPPORTED, "hga_route_prefill: topk_chunks * groups_per_chunk > 256");
  const int64_t row_hi = chunk_hi * p->chunk_size < seq_len ? chunk_hi * p->chunk_size : seq_len;
  const hga::QRange qr{(int)chunk_lo, (int)(chunk_hi - chunk_lo), row_hi - chunk_lo * p->chunk_size};
  const bool tc_ok = hga::route_tc_supported(*p, seq_len);
  if (impl == 2 && !tc_ok)
    return fail(HGA_E_UNSUPPORTED, "tensor-core router needs bf16, head_dim 128, chunk 64, group 16, topk_chunks <= 32");
  if ((impl == 0 && tc_ok) || impl == 2) {
    const cudaError_t e = hga::launch_route_tc(*p, seq_len, qr, q, q_layout, chunk_k, group_k, sum_cap, sel_chunk,
                                               sel_t0, open_gid, open_t0, dbg_l1, dbg_l2, stream);
    if (!(impl == 0 && (e == cudaErrorMisalignedAddress || e == cudaErrorInvalidConfiguration)))
      return cuda_status(e, "hga_route_prefill(tcgen05)");
    (void)cudaGetLastError();
  }
  if (impl != 0 && impl != 1) return fail(HGA_E_INVALID, "impl must be 0, 1 or 2");
  int smem = 0;
  return cuda_status(hga::launch_route_prefill(*p, seq_len, qr, q, q_layout, chunk_k, group_k, sum_cap, sel_chunk,
                                               sel_t0, open_gid, open_t0, dbg_l1, dbg_l2, stream, &smem),
                     "hga_route_prefill");
}

int hga_attend_prefill(const hga_params* p, int64_t seq_len, const void* q, int32_t q_layout, const void* k_rope,
                       const void* v, int64_t kv_cap, const int32_t* open_gid, const int32_t* open_t0, void* out,
                       int32_t out_layout, int32_t impl, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (seq_len <= 0) return HGA_OK;
  const int64_t N = (seq_len + p->chunk_size - 1) / p->chunk_size;
  return hga_attend_prefill_range(p, seq_len, 0, N, q, q_layout, k_rope, v, kv_cap, open_gid, open_t0, out,
                                  out_layout, impl, stream);
}

int hga_attend_prefill_range(const hga_params* p, int64_t seq_len, int64_t chunk_lo, int64_t chunk_hi, const void* q,
                             int32_t q_layout, const void* k_rope, const void* v, int64_t kv_cap,
                             const int32_t* open_gid, const int32_t* open_t0, void* out, int32_t out_layout,
                             int32_t impl, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (seq_len <= 0) return HGA_OK;
  int Kc, Kg;
  route_sizes(p, seq_len, &Kc, &Kg);
  if (!q || !k_rope || !v || !out) return fail(HGA_E_INVALID, "hga_attend_prefill: NULL tensor");
  if (Kg && (!open_gid || !open_t0)) return fail(HGA_E_INVALID, "hga_attend_prefill: NULL open lists");
  if (kv_cap < seq_len) return fail(HGA_E_INVALID, "hga_attend_prefill: kv_cap < seq_len");
  if (q_layout != 0 && q_layout != 1) return fail(HGA_E_INVALID, "q_layout must be 0 or 1");
  if (out_layout != 0 && out_layout != 1) return fail(HGA_E_INVALID, "out_layout must be 0 or 1");
  const int64_t N = (seq_len + p->chunk_size - 1) / p->chunk_size;
  if (chunk_lo < 0 || chunk_hi > N || chunk_lo >= chunk_hi)
    return fail(HGA_E_INVALID, "hga_attend_prefill: query chunk range outside [0, N) or empty");
  const int64_t row_hi = chunk_hi * p->chunk_size < seq_len ? chunk_hi * p->chunk_size : seq_len;
  const hga::QRange qr{(int)chunk_lo, (int)(chunk_hi - chunk_lo), row_hi - chunk_lo * p->chunk_size};
  const bool tc_ok = hga::attend_tc_supported(*p);
  if (impl == 2 && !tc_ok)
    return fail(HGA_E_UNSUPPORTED, "tensor-core attention needs bf16, head_dim 128, chunk 64, group 16");
  if ((impl == 0 && tc_ok) || impl == 2) {
    const cudaError_t e = hga::launch_attend_tc(*p, seq_len, qr, q, q_layout, k_rope, v, kv_cap, open_gid, open_t0,
                                                Kg, out, out_layout, stream);
    // windows wider than the tensor-core kernel's unit table (or misaligned pointers) go to the
    // portable kernel when the caller let us choose
    if (!(impl == 0 && (e == cudaErrorNotSupported || e == cudaErrorMisalignedAddress)))
      return cuda_status(e, "hga_attend_prefill(tcgen05)");
    (void)cudaGetLastError();
  }
  if (impl != 0 && impl != 1) return fail(HGA_E_INVALID, "impl must be 0, 1 or 2");
  return cuda_status(hga::launch_attend_simt(*p, seq_len, qr, q, q_layout, k_rope, v, kv_cap, open_gid, open_t0, Kg,
                                             out, out_layout, stream),
                     "hga_attend_prefill");
}

static void decode_sizes(const hga_params* p, int nmid_max, int* Kc, int* Kg) {
  const int M = p->chunk_size / p->group_size;
  *Kc = p->topk_chunks > 0 ? (p->topk_chunks < nmid_max ? p->topk_chunks : nmid_max) : 0;
  const int G = *Kc * M;
  *Kg = p->topk_groups > 0 ? (p->topk_groups < G ? p->topk_groups : G) : 0;
}

int hga_route_decode(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos, const void* chunk_k,
                     const void* group_k, int64_t sum_cap, int32_t nmid_max, int32_t* mid_chunk, int32_t* mid_t0,
                     int32_t* open_gid, int32_t* open_t0, cudaStream_t stream) {
  return hga_route_decode_impl(p, L, q, seq_pos, chunk_k, group_k, sum_cap, nmid_max, mid_chunk, mid_t0, open_gid,
                               open_t0, 0, stream);
}

int hga_route_decode_impl(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos, const void* chunk_k,
                          const void* group_k, int64_t sum_cap, int32_t nmid_max, int32_t* mid_chunk, int32_t* mid_t0,
                          int32_t* open_gid, int32_t* open_t0, int32_t impl, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (L <= 0 || L > p->chunk_size) return fail(HGA_E_INVALID, "hga_route_decode: 1 <= L <= chunk_size");
  if (!q || !seq_pos || !chunk_k || !group_k) return fail(HGA_E_INVALID, "hga_route_decode: NULL tensor");
  if (nmid_max < 0 || nmid_max > sum_cap) return fail(HGA_E_INVALID, "hga_route_decode: nmid_max outside [0, sum_cap]");
  if (impl < 0 || impl > 2) return fail(HGA_E_INVALID, "hga_route_decode: impl must be 0, 1 or 2");
  int Kc, Kg;
  decode_sizes(p, nmid_max, &Kc, &Kg);
  if ((Kc && (!mid_chunk || !mid_t0)) || (Kg && (!open_gid || !open_t0)))
    return fail(HGA_E_INVALID, "hga_route_decode: NULL output list");
  if (Kc * (p->chunk_size / p->group_size) > 256) return fail(HGA_E_UNSUPPORTED, "hga_route_decode: topk_chunks * M > 256");
  const bool fast = hga::route_decode1_supported(*p, L);
  if (impl == 2 && !fast) return fail(HGA_E_UNSUPPORTED, "hga_route_decode: the L = 1 kernel needs L == 1, head_dim 64 or 128");
  if (fast && impl != 1)
    return cuda_status(hga::launch_route_decode1(*p, q, seq_pos, chunk_k, group_k, sum_cap, nmid_max > 0 ? nmid_max : 1,
                                                 Kc, Kg, mid_chunk, mid_t0, open_gid, open_t0, stream),
                       "hga_route_decode");
  return cuda_status(hga::launch_route_decode(*p, L, q, seq_pos, chunk_k, group_k, sum_cap, nmid_max > 0 ? nmid_max : 1,
                                              Kc, Kg, mid_chunk, mid_t0, open_gid, open_t0, stream),
                     "hga_route_decode");
}

int hga_attend_decode(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos, const void* hot_k,
                      const void* hot_v, int64_t hot_cap, int32_t hot_mode, const void* cold_k, const void* cold_v,
                      int64_t cold_cap, const int32_t* open_gid, const int32_t* open_t0, int32_t Kg, void* out,
                      cudaStream_t stream) {
  return hga_attend_decode_impl(p, L, q, seq_pos, hot_k, hot_v, hot_cap, hot_mode, cold_k, cold_v, cold_cap, open_gid,
                                open_t0, Kg, out, 0, stream);
}

int hga_attend_decode_impl(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos, const void* hot_k,
                           const void* hot_v, int64_t hot_cap, int32_t hot_mode, const void* cold_k, const void* cold_v,
                           int64_t cold_cap, const int32_t* open_gid, const int32_t* open_t0, int32_t Kg, void* out,
                           int32_t impl, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (L <= 0 || L > p->chunk_size) return fail(HGA_E_INVALID, "hga_attend_decode: 1 <= L <= chunk_size");
  if (!q || !seq_pos || !hot_k || !hot_v || !out) return fail(HGA_E_INVALID, "hga_attend_decode: NULL tensor");
  if (Kg > 0 && (!open_gid || !open_t0 || !cold_k || !cold_v)) return fail(HGA_E_INVALID, "hga_attend_decode: NULL open lists / cold record");
  if (hot_mode != 0 && hot_mode != 1) return fail(HGA_E_INVALID, "hga_attend_decode: hot_mode must be 0 or 1");
  if (impl < 0 || impl > 2) return fail(HGA_E_INVALID, "hga_attend_decode: impl must be 0, 1 or 2");
  const bool fast = hga::attend_decode_fast_supported(*p, L);
  if (impl == 2 && !fast)
    return fail(HGA_E_UNSUPPORTED, "hga_attend_decode: the fast kernel needs bf16/fp16, group_size 16, head_dim 64/128, L <= 8");
  const void* ck = cold_k ? cold_k : hot_k;
  const void* cv = cold_v ? cold_v : hot_v;
  if (fast && impl != 1)
    return cuda_status(hga::launch_attend_decode_fast(*p, L, q, seq_pos, hot_k, hot_v, hot_cap, hot_mode, ck, cv,
                                                      cold_cap, open_gid, open_t0, Kg, out, stream),
                       "hga_attend_decode");
  return cuda_status(hga::launch_attend_decode(*p, L, q, seq_pos, hot_k, hot_v, hot_cap, hot_mode, ck, cv, cold_cap,
                                               open_gid, open_t0, Kg, out, stream),
                     "hga_attend_decode");
}

int hga_attend_decode_dca(const hga_params* p, int32_t L, const void* q, const int32_t* seq_pos, const void* hot_k,
                          const void* hot_v, int64_t hot_cap, int32_t hot_mode, const void* cold_k, const void* cold_v,
                          int64_t cold_cap, const int32_t* open_gid, const int32_t* open_t0, const int32_t* open_pos,
                          int32_t Kg, const float* dca_cos, const float* dca_sin, int32_t dca_chunk, int32_t dca_ceil,
                          void* out, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (L <= 0 || L > p->chunk_size) return fail(HGA_E_INVALID, "hga_attend_decode_dca: 1 <= L <= chunk_size");
  if (!q || !seq_pos || !hot_k || !hot_v || !out || !dca_cos || !dca_sin)
    return fail(HGA_E_INVALID, "hga_attend_decode_dca: NULL tensor");
  if (Kg > 0 && (!open_gid || !open_t0 || !cold_k || !cold_v))
    return fail(HGA_E_INVALID, "hga_attend_decode_dca: NULL open lists / cold record");
  if (hot_mode != 0 && hot_mode != 1) return fail(HGA_E_INVALID, "hga_attend_decode_dca: hot_mode must be 0 or 1");
  if (dca_chunk <= 0 || dca_ceil < dca_chunk)
    return fail(HGA_E_INVALID, "hga_attend_decode_dca: need dca_chunk > 0 and dca_ceil >= dca_chunk");
  if (p->head_dim % 2) return fail(HGA_E_INVALID, "hga_attend_decode_dca: head_dim must be even");
  const void* ck = cold_k ? cold_k : hot_k;
  const void* cv = cold_v ? cold_v : hot_v;
  return cuda_status(hga::launch_attend_decode_dca(*p, L, q, seq_pos, hot_k, hot_v, hot_cap, hot_mode, ck, cv, cold_cap,
                                                   open_gid, open_t0, open_pos, Kg, dca_cos, dca_sin, dca_chunk,
                                                   dca_ceil, out, stream),
                     "hga_attend_decode_dca");
}

int hga_gather_h2d(const hga_params* p, const int32_t* open_gid, int32_t Kg, const void* rec_k, const void* rec_v,
                   int64_t rec_cap, void* bank_k, void* bank_v, int32_t n_slots, int32_t* slot_gid, int32_t* gid_slot,
                   int64_t gid_cap, int32_t* slot_stamp, int32_t stamp, int32_t* open_slot,
                   unsigned long long* counters, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (Kg <= 0) return HGA_OK;
  if (!open_gid || !rec_k || !rec_v || !bank_k || !bank_v || !slot_gid || !gid_slot || !slot_stamp || !open_slot)
    return fail(HGA_E_INVALID, "hga_gather_h2d: NULL pointer");
  const int rep = p->nhead / p->kv_heads;
  if (n_slots < rep * Kg) return fail(HGA_E_INVALID, "hga_gather_h2d: n_slots %d < (H/KVH) * Kg = %d", n_slots, rep * Kg);
  if (gid_cap <= 0 || gid_cap > (1 << 20) || rec_cap < 0) return fail(HGA_E_INVALID, "hga_gather_h2d: gid_cap out of range");
  if (stamp < 0) return fail(HGA_E_INVALID, "hga_gather_h2d: stamp must be >= 0");
  if ((p->group_size * p->head_dim * (p->dtype == HGA_DTYPE_F32 ? 4 : 2)) % 16 ||
      (((uintptr_t)rec_k | (uintptr_t)rec_v | (uintptr_t)bank_k | (uintptr_t)bank_v) & 15))
    return fail(HGA_E_INVALID, "hga_gather_h2d: groups and buffers must be 16-byte aligned");
  return cuda_status(hga::launch_bank_gather(*p, open_gid, Kg, rec_k, rec_v, rec_cap, bank_k, bank_v, n_slots, slot_gid,
                                             gid_slot, gid_cap, slot_stamp, stamp, open_slot, counters, stream),
                     "hga_gather_h2d");
}

int hga_append_tokens(const hga_params* p, int32_t L, const int32_t* seq_pos, const void* k_rope, const void* v,
                      const void* k_raw, void* hot_k, void* hot_v, int64_t hot_cap, int32_t hot_mode, void* cold_k,
                      void* cold_v, int64_t cold_cap, void* active_raw, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (L <= 0 || L > p->chunk_size) return fail(HGA_E_INVALID, "hga_append_tokens: 1 <= L <= chunk_size");
  if (!seq_pos || !k_rope || !v || !hot_k || !hot_v) return fail(HGA_E_INVALID, "hga_append_tokens: NULL tensor");
  if (active_raw && !k_raw) return fail(HGA_E_INVALID, "hga_append_tokens: k_raw needed for active_raw");
  if (hot_mode != 0 && hot_mode != 1) return fail(HGA_E_INVALID, "hga_append_tokens: hot_mode must be 0 or 1");
  return cuda_status(hga::launch_append(*p, L, seq_pos, k_rope, v, k_raw, hot_k, hot_v, hot_cap, hot_mode, cold_k,
                                        cold_v, cold_cap, active_raw, stream),
                     "hga_append_tokens");
}

int hga_shard_unpack(const void* recv, int64_t rank_stride, int64_t part_offset, int32_t world, int32_t pieces,
                     const int32_t* dst_block, int64_t bk, int64_t rows, int64_t row_bytes, void* dst,
                     cudaStream_t stream) {
  if (!recv || !dst || !dst_block) return fail(HGA_E_INVALID, "hga_shard_unpack: NULL pointer");
  if (world < 1 || pieces < 1 || (int64_t)world * pieces > 128)
    return fail(HGA_E_INVALID, "hga_shard_unpack: world * pieces must be in [1, 128]");
  if (bk < 0 || rows < 0 || row_bytes <= 0 || row_bytes % 16 || rank_stride % 16 || part_offset % 16 ||
      ((uintptr_t)recv | (uintptr_t)dst) & 15)
    return fail(HGA_E_INVALID, "hga_shard_unpack: rows, strides and pointers must be 16-byte aligned");
  for (int i = 0; i < world * pieces; ++i)
    if (dst_block[i] < 0 || dst_block[i] >= world * pieces)
      return fail(HGA_E_INVALID, "hga_shard_unpack: destination block %d out of range", dst_block[i]);
  return cuda_status(hga::launch_shard_unpack(recv, rank_stride, part_offset, world, pieces, dst_block, bk, rows,
                                              row_bytes, dst, stream),
                     "hga_shard_unpack");
}

int hga_debug_fault(int32_t mode, int64_t wait_limit_ns) {
  if (mode < 0 || mode > 1 || wait_limit_ns < 0) return fail(HGA_E_INVALID, "hga_debug_fault: mode 0/1, wait_limit_ns >= 0");
  hga::attend_tc_set_test_fault(mode, (long long)wait_limit_ns);
  return HGA_OK;
}

int hga_device_status(int32_t* code, int32_t clear) {
  const int words[4] = {hga::tc_error_status(clear != 0), hga::route_tc_error_status(clear != 0),
                        hga::decode_error_status(clear != 0), hga::decode_fast_error_status(clear != 0)};
  int first = 0;
  for (int w : words) {
    if (w < 0) return fail(HGA_E_CUDA, "hga_device_status: cannot read the device error word");
    if (!first) first = w;
  }
  if (code) *code = first;
  return HGA_OK;
}

int hga_qkv_prologue(const hga_params* p, int64_t seq_len, const void* qkv, int64_t row_stride, const void* q_norm_w,
                     const void* k_norm_w, float eps, int32_t norm_mode, const void* cos, const void* sin,
                     int32_t rope_mode, int64_t rot_row0, int64_t pos0, void* q_rope, void* k_raw, void* k_rope,
                     void* v, int64_t kv_cap, int64_t kv_row0, cudaStream_t stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (seq_len <= 0) return HGA_OK;
  if (!qkv || !cos || !sin || !q_rope || !k_raw || !k_rope || !v) return fail(HGA_E_INVALID, "hga_qkv_prologue: NULL tensor");
  if (row_stride < (int64_t)(p->nhead + 2 * p->kv_heads) * p->head_dim)
    return fail(HGA_E_INVALID, "hga_qkv_prologue: row_stride smaller than (H + 2*KVH) * Dh");
  if (kv_row0 < 0 || kv_row0 + seq_len > kv_cap) return fail(HGA_E_INVALID, "hga_qkv_prologue: kv capacity too small");
  if (pos0 < rot_row0) return fail(HGA_E_INVALID, "hga_qkv_prologue: rotary table starts after pos0");
  if ((norm_mode != 0 && norm_mode != 1) || (rope_mode != 0 && rope_mode != 1))
    return fail(HGA_E_INVALID, "hga_qkv_prologue: norm_mode / rope_mode must be 0 or 1");
  return cuda_status(hga::launch_prologue(*p, seq_len, qkv, row_stride, q_norm_w, k_norm_w, eps, norm_mode, cos, sin,
                                          rope_mode, rot_row0, pos0, q_rope, k_raw, k_rope, v, kv_cap, kv_row0, stream),
                     "hga_qkv_prologue");
}

}  // extern "C"
