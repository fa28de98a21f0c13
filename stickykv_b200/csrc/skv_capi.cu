// extern "C" entry points: argument validation, workspace carving, dispatch.
#include <stdio.h>
#include <string.h>

#include "skv_common.cuh"

namespace skv {

static thread_local char g_last_cuda_error[256] = "no error";
void set_cuda_error(cudaError_t e) {
  snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e),
           cudaGetErrorString(e));
}

// defined in the kernel files
int append_dispatch(const skv_layer_desc* L, int seq_len, int tier_pages, const void* k_new,
                    const void* v_new, int64_t sb, int64_t sh, int64_t st, int n_new, cudaStream_t stream);
size_t decode_generic_ws_size(const skv_layer_desc* L, int T);
int decode_generic(const skv_layer_desc* L, int T, int tier_pages, const void* q, int64_t q_sb,
                   int64_t q_sh, void* out, int64_t o_sb, int64_t o_sh, float scaling, float* scores,
                   int scores_cap, void* ws, cudaStream_t stream);
bool decode_mma_supported(const skv_layer_desc* L);
bool decode_mma_length_ok(int T);
size_t decode_mma_ws_size(const skv_layer_desc* L, int T);
int decode_mma(const skv_layer_desc* L, int T, int tier_pages, const void* q, int64_t q_sb,
               int64_t q_sh, void* out, int64_t o_sb, int64_t o_sh, float scaling, float* scores,
               int scores_cap, void* ws, cudaStream_t stream, const void* k_new = nullptr,
               const void* v_new = nullptr, int64_t kn_sb = 0, int64_t kn_sh = 0);
int evict_dispatch(EvictParams& p, cudaStream_t stream);
int pack_pages_dispatch(const skv_layer_desc* L, const void* k, const void* v, int first_pos,
                        int n_pages, uint8_t* out, cudaStream_t stream);
int materialize_dispatch(const skv_layer_desc* L, int T_len, int tier_pages, void* k_out, void* v_out,
                         cudaStream_t stream);
size_t prefill_ws_size(const skv_layer_desc* L, int T);
int prefill_dispatch(const skv_layer_desc* L, int T, const void* q, const void* k, const void* v,
                     void* out, float scaling, float* scores, int scores_cap, void* ws,
                     cudaStream_t stream);

static int elt_size(int dt) { return dt == SKV_F32 ? 4 : (dt == SKV_F16 || dt == SKV_BF16) ? 2 : 0; }
static bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

static int check_layer(const skv_layer_desc* L) {
  if (!L) return SKV_ERR_INVALID_ARG;
  if (L->batch <= 0 || L->num_kv_heads <= 0 || L->num_q_heads <= 0 || L->head_dim <= 0)
    return SKV_ERR_INVALID_ARG;
  if (L->num_q_heads % L->num_kv_heads) return SKV_ERR_INVALID_ARG;
  if (L->head_dim != 16 && L->head_dim != 32 && L->head_dim != 64 && L->head_dim != 128)
    return SKV_ERR_UNSUPPORTED;
  if (elt_size(L->kv_dtype) == 0) return SKV_ERR_UNSUPPORTED;
  if (L->window_size <= 0 || L->num_sink < 0) return SKV_ERR_INVALID_ARG;
  if (L->sink_pad != (L->num_sink + 7) / 8 * 8) return SKV_ERR_INVALID_ARG;
  if (L->fp_capacity <= 0 || !L->k_fp || !L->v_fp) return SKV_ERR_INVALID_ARG;
  if (!aligned(L->k_fp, 16) || !aligned(L->v_fp, 16)) return SKV_ERR_MISALIGNED;
  // rope rows are read as 8- and 16-byte vectors
  if ((L->rope_cos && !aligned(L->rope_cos, 16)) || (L->rope_sin && !aligned(L->rope_sin, 16)))
    return SKV_ERR_MISALIGNED;
  if (L->tier_page_capacity < 0) return SKV_ERR_INVALID_ARG;
  if (L->tier_page_capacity > 0) {
    if (L->window_size % kPageTokens) return SKV_ERR_UNSUPPORTED;
    if (L->head_dim % kQGroup) return SKV_ERR_UNSUPPORTED;
    if (!L->tier_pages || !L->tier_table || !L->rope_cos || !L->rope_sin) return SKV_ERR_INVALID_ARG;
    if (!aligned(L->tier_pages, 16)) return SKV_ERR_MISALIGNED;
  }
  return SKV_OK;
}

static Geometry geometry(const skv_layer_desc* L, int T, int tier_pages) {
  return Geometry{L->num_sink, L->sink_pad, L->window_size, T, tier_pages * kPageTokens};
}

// fp slots a cache of T tokens occupies
static int fp_slots_used(const skv_layer_desc* L, int T, int tier_pages) {
  if (T <= 0) return 0;
  const Geometry g = geometry(L, T, tier_pages);
  return g.fp_slot(T - 1) + 1;
}

static int check_counts(const skv_layer_desc* L, int T, int tier_pages) {
  if (T < 0 || tier_pages < 0) return SKV_ERR_INVALID_ARG;
  if (tier_pages > 0 && L->tier_page_capacity == 0) return SKV_ERR_INVALID_ARG;
  if (tier_pages > L->tier_page_capacity) return SKV_ERR_CAPACITY;
  if (tier_pages > 0 && T < L->num_sink + tier_pages * kPageTokens) return SKV_ERR_INVALID_ARG;
  if (fp_slots_used(L, T, tier_pages) > L->fp_capacity) return SKV_ERR_CAPACITY;
  return SKV_OK;
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_abi_version(void) { return SKV_ABI_VERSION; }

const char* skv_status_string(int s) {
  switch (s) {
    case SKV_OK: return "ok";
    case SKV_ERR_INVALID_ARG: return "invalid argument";
    case SKV_ERR_UNSUPPORTED: return "unsupported geometry or dtype";
    case SKV_ERR_MISALIGNED: return "misaligned pointer or stride";
    case SKV_ERR_CAPACITY: return "buffer capacity exceeded";
    case SKV_ERR_CUDA: return "CUDA launch error";
    case SKV_ERR_WORKSPACE: return "workspace too small";
  }
  return "unknown status";
}

const char* skv_last_cuda_error(void) { return g_last_cuda_error; }

int32_t skv_page_bytes(int32_t head_dim) {
  return (head_dim > 0 && head_dim % kQGroup == 0) ? page_bytes(head_dim) : 0;
}

int32_t skv_struct_size(int32_t which) {
  switch (which) {
    case 0: return (int32_t)sizeof(skv_layer_desc);
    case 1: return (int32_t)sizeof(skv_evict_plan);
    case 2: return (int32_t)sizeof(skv_evict_args);
  }
  return 0;
}

int skv_evict_plan_compute(int32_t T, int32_t W, int32_t s, int32_t ws, int32_t top_k, int32_t Lw,
                           int32_t tier, skv_evict_plan* plan) {
  if (!plan || T < 0 || W < 0 || s < 0 || ws <= 0 || top_k < 0 || Lw < 0) return SKV_ERR_INVALID_ARG;
  const int post = T > s ? T - s : 0;
  if (W > (post + ws - 1) / ws) return SKV_ERR_INVALID_ARG;  // scores cover no future windows
  memset(plan, 0, sizeof(*plan));
  const int local = Lw < W ? Lw : W;
  const int E = W - local;
  int k = top_k < E ? top_k : E;
  if (top_k == 0 || E == 0) k = 0;
  if (local == 0 && E > 0 && E * ws > post) return SKV_ERR_INVALID_ARG;
  int tok = 0;
  for (int w = E; w < W; ++w) {
    int n = T - s - w * ws;
    tok += n < 0 ? 0 : (n > ws ? ws : n);
  }
  const int s_eff = T < s ? T : s;
  plan->local_windows = local;
  plan->evictable_windows = E;
  plan->kept_evictable = k;
  plan->retained_windows = k + local;
  plan->seq_len_new = s_eff + k * ws + tok;
  plan->tier_pages_new = tier ? k * ws / kPageTokens : 0;
  const int s_pad = (s + 7) / 8 * 8;
  const int tier_tok = plan->tier_pages_new * kPageTokens;
  plan->fp_len_new = plan->seq_len_new <= s ? plan->seq_len_new : s_pad + (plan->seq_len_new - s - tier_tok);
  return SKV_OK;
}

int skv_append(const skv_layer_desc* L, int32_t seq_len, int32_t tier_pages, const void* k_new,
               const void* v_new, int64_t sb, int64_t sh, int64_t st, int32_t n_new, void* stream) {
  int rc = check_layer(L);
  if (rc) return rc;
  if (n_new <= 0 || !k_new || !v_new) return SKV_ERR_INVALID_ARG;
  if ((rc = check_counts(L, seq_len + n_new, tier_pages))) return rc;
  const int es = elt_size(L->kv_dtype);
  if (!aligned(k_new, 16) || !aligned(v_new, 16)) return SKV_ERR_MISALIGNED;
  if ((sb * es) % 16 || (sh * es) % 16 || (st * es) % 16 || (L->head_dim * es) % 16) return SKV_ERR_MISALIGNED;
  return append_dispatch(L, seq_len, tier_pages, k_new, v_new, sb, sh, st, n_new, (cudaStream_t)stream);
}

size_t skv_decode_workspace_size(const skv_layer_desc* L, int32_t T) {
  if (check_layer(L)) return 0;
  size_t a = decode_generic_ws_size(L, T);
  if (decode_mma_supported(L)) {
    const size_t b = decode_mma_ws_size(L, T);
    if (b > a) a = b;
  }
  return a;
}

// The tensor-core decode takes fp16/bf16 at head_dim 64/128 and any GQA
// ratio; the portable decode takes every dtype and head_dim at GQA 1 to 8.
static bool decode_kernel_exists(const skv_layer_desc* L, int32_t T) {
  if (decode_mma_supported(L) && decode_mma_length_ok(T)) return true;
  const int G = L->num_q_heads / L->num_kv_heads;
  return G >= 1 && G <= 8;
}

}  // extern "C"

namespace skv {
// Every check of a decode call except those of its workspace (shared with
// the allocation-free entry point, which has no workspace argument).
int decode_precheck(const skv_layer_desc* L, int32_t T, int32_t tier_pages, const void* q, void* out,
                    float* scores, int32_t scores_cap) {
  int rc = check_layer(L);
  if (rc) return rc;
  if (T > 0 && !decode_kernel_exists(L, T)) return SKV_ERR_UNSUPPORTED;
  if (T <= 0 || !q || !out) return SKV_ERR_INVALID_ARG;
  if ((rc = check_counts(L, T, tier_pages))) return rc;
  const Geometry g = geometry(L, T, tier_pages);
  if (scores && scores_cap < g.num_windows()) return SKV_ERR_CAPACITY;
  if (tier_pages > 0 && L->rope_positions < L->num_sink + tier_pages * kPageTokens) return SKV_ERR_CAPACITY;
  return SKV_OK;
}
}  // namespace skv

extern "C" {

static int check_decode(const skv_layer_desc* L, int32_t T, int32_t tier_pages, const void* q, void* out,
                        float* scores, int32_t scores_cap, void* ws, size_t ws_bytes) {
  const int rc = decode_precheck(L, T, tier_pages, q, out, scores, scores_cap);
  if (rc) return rc;
  if (!ws || ws_bytes < skv_decode_workspace_size(L, T)) return SKV_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return SKV_ERR_MISALIGNED;
  return SKV_OK;
}

int skv_decode_attention(const skv_layer_desc* L, int32_t T, int32_t tier_pages, const void* q,
                         int64_t q_sb, int64_t q_sh, void* out, int64_t o_sb, int64_t o_sh,
                         float scaling, float* scores, int32_t scores_cap, void* ws, size_t ws_bytes,
                         void* stream) {
  const int rc = check_decode(L, T, tier_pages, q, out, scores, scores_cap, ws, ws_bytes);
  if (rc) return rc;
  const cudaStream_t s = (cudaStream_t)stream;
  if (decode_mma_supported(L) && decode_mma_length_ok(T))
    return decode_mma(L, T, tier_pages, q, q_sb, q_sh, out, o_sb, o_sh, scaling, scores, scores_cap, ws, s);
  return decode_generic(L, T, tier_pages, q, q_sb, q_sh, out, o_sb, o_sh, scaling, scores, scores_cap, ws, s);
}

int skv_decode_attention_append(const skv_layer_desc* L, int32_t T, int32_t tier_pages, const void* k_new,
                                const void* v_new, int64_t sb, int64_t sh, const void* q, int64_t q_sb,
                                int64_t q_sh, void* out, int64_t o_sb, int64_t o_sh, float scaling,
                                float* scores, int32_t scores_cap, void* ws, size_t ws_bytes, void* stream) {
  // every check of both halves runs before anything is launched
  int rc = check_decode(L, T, tier_pages, q, out, scores, scores_cap, ws, ws_bytes);
  if (rc) return rc;
  if (!k_new || !v_new || T - 1 < 0) return SKV_ERR_INVALID_ARG;
  if (tier_pages > 0 && T - 1 < L->num_sink + tier_pages * kPageTokens) return SKV_ERR_INVALID_ARG;
  const int es = elt_size(L->kv_dtype);
  if (!aligned(k_new, 16) || !aligned(v_new, 16)) return SKV_ERR_MISALIGNED;
  if ((sb * es) % 16 || (sh * es) % 16 || (L->head_dim * es) % 16) return SKV_ERR_MISALIGNED;
  const cudaStream_t s = (cudaStream_t)stream;
  if (decode_mma_supported(L) && decode_mma_length_ok(T))
    return decode_mma(L, T, tier_pages, q, q_sb, q_sh, out, o_sb, o_sh, scaling, scores, scores_cap, ws, s,
                      k_new, v_new, sb, sh);
  if ((rc = append_dispatch(L, T - 1, tier_pages, k_new, v_new, sb, sh, 0, 1, s))) return rc;
  return decode_generic(L, T, tier_pages, q, q_sb, q_sh, out, o_sb, o_sh, scaling, scores, scores_cap, ws, s);
}

size_t skv_evict_workspace_size(const skv_layer_desc* L, int32_t W) {
  if (!L || W < 0) return 0;
  return align_up((size_t)L->batch * (W > 0 ? W : 1) * 4, 256) * 3;  // retained, entrant, keys
}

static int evict_impl(const skv_layer_desc* src, const skv_layer_desc* dst, const skv_evict_args* a,
                      const void* k_new, const void* v_new, int64_t sb, int64_t sh, void* ws,
                      size_t ws_bytes, void* stream) {
  int rc = check_layer(src);
  if (rc) return rc;
  if ((rc = check_layer(dst))) return rc;
  if (!a || !a->scores_src || !a->scores_dst || !a->ids_src || !a->ids_dst) return SKV_ERR_INVALID_ARG;
  if (a->scores_src == a->scores_dst || a->ids_src == a->ids_dst) return SKV_ERR_INVALID_ARG;
  if (src->k_fp == dst->k_fp || src->v_fp == dst->v_fp) return SKV_ERR_INVALID_ARG;
  if (src->batch != dst->batch || src->num_kv_heads != dst->num_kv_heads ||
      src->num_q_heads != dst->num_q_heads || src->head_dim != dst->head_dim ||
      src->kv_dtype != dst->kv_dtype || src->window_size != dst->window_size ||
      src->num_sink != dst->num_sink ||
      src->tier_page_capacity != dst->tier_page_capacity || src->tier_pages != dst->tier_pages)
    return SKV_ERR_INVALID_ARG;
  if (!src->rope_cos || !src->rope_sin) return SKV_ERR_INVALID_ARG;
  const int tier = src->tier_page_capacity > 0;
  if (tier && src->tier_table == dst->tier_table) return SKV_ERR_INVALID_ARG;
  if ((rc = check_counts(src, a->seq_len, a->tier_pages))) return rc;
  if (a->num_windows > a->scores_capacity) return SKV_ERR_CAPACITY;
  if (src->rope_positions < a->seq_len) return SKV_ERR_CAPACITY;
  skv_evict_plan plan;
  if ((rc = skv_evict_plan_compute(a->seq_len, a->num_windows, src->num_sink, src->window_size,
                                   a->top_k_windows, a->local_windows, tier, &plan)))
    return rc;
  if (tier) {
    if (a->tier_pages % (src->window_size / kPageTokens)) return SKV_ERR_INVALID_ARG;
    if (plan.tier_pages_new > src->tier_page_capacity) return SKV_ERR_CAPACITY;
  }
  if ((rc = check_counts(dst, plan.seq_len_new, plan.tier_pages_new))) return rc;
  if (!ws || ws_bytes < skv_evict_workspace_size(src, a->num_windows)) return SKV_ERR_WORKSPACE;

  EvictParams p{};
  p.B = src->batch; p.Hq = src->num_q_heads; p.Hkv = src->num_kv_heads; p.D = src->head_dim;
  p.s = src->num_sink; p.s_pad = src->sink_pad; p.ws = src->window_size;
  p.ppw = tier ? src->window_size / kPageTokens : 1;
  p.T_old = a->seq_len; p.n_tier_old_tok = a->tier_pages * kPageTokens; p.W = a->num_windows;
  p.E = plan.evictable_windows; p.kprime = plan.kept_evictable; p.local_w = plan.local_windows;
  p.R = plan.retained_windows; p.T_new = plan.seq_len_new; p.n_tier_new_tok = plan.tier_pages_new * kPageTokens;
  p.tier = tier; p.scores_cap = a->scores_capacity; p.page_cap = src->tier_page_capacity;
  p.fp_cap_src = src->fp_capacity; p.fp_cap_dst = dst->fp_capacity; p.dtype = src->kv_dtype;
  p.scores_src = a->scores_src; p.scores_dst = a->scores_dst; p.ids_src = a->ids_src; p.ids_dst = a->ids_dst;
  const size_t third = skv_evict_workspace_size(src, a->num_windows) / 3;
  p.retained = (int32_t*)ws;
  p.entrant = (int32_t*)((char*)ws + third);
  p.keys = (uint32_t*)((char*)ws + 2 * third);
  p.retained_out = a->retained_out;
  p.next_window_id = a->next_window_id;
  p.table_src = src->tier_table; p.table_dst = dst->tier_table; p.pages = src->tier_pages;
  p.k_src = src->k_fp; p.v_src = src->v_fp; p.k_dst = dst->k_fp; p.v_dst = dst->v_fp;
  p.cos = src->rope_cos; p.sin = src->rope_sin;
  p.k_new = k_new; p.v_new = v_new; p.new_sb = sb; p.new_sh = sh;
  return evict_dispatch(p, (cudaStream_t)stream);
}

int skv_evict(const skv_layer_desc* src, const skv_layer_desc* dst, const skv_evict_args* a,
              void* ws, size_t ws_bytes, void* stream) {
  return evict_impl(src, dst, a, nullptr, nullptr, 0, 0, ws, ws_bytes, stream);
}

int skv_evict_append(const skv_layer_desc* src, const skv_layer_desc* dst, const skv_evict_args* a,
                     const void* k_new, const void* v_new, int64_t sb, int64_t sh, void* ws,
                     size_t ws_bytes, void* stream) {
  int rc = check_layer(src);
  if (rc) return rc;
  if (!a || !k_new || !v_new || a->seq_len < 1) return SKV_ERR_INVALID_ARG;
  const int es = elt_size(src->kv_dtype);
  if (!aligned(k_new, 16) || !aligned(v_new, 16)) return SKV_ERR_MISALIGNED;
  if ((sb * es) % 16 || (sh * es) % 16 || (src->head_dim * es) % 16) return SKV_ERR_MISALIGNED;
  if (a->local_windows < 1) {  // the token need not stay fp: append it, then evict
    if ((rc = skv_append(src, a->seq_len - 1, a->tier_pages, k_new, v_new, sb, sh, src->head_dim, 1, stream)))
      return rc;
    return skv_evict(src, dst, a, ws, ws_bytes, stream);
  }
  return evict_impl(src, dst, a, k_new, v_new, sb, sh, ws, ws_bytes, stream);
}

size_t skv_prefill_workspace_size(const skv_layer_desc* L, int32_t T) {
  if (check_layer(L) || T <= 0) return 0;
  return prefill_ws_size(L, T);
}

int skv_prefill_attention(const skv_layer_desc* L, int32_t T, const void* q, const void* k,
                          const void* v, void* out, float scaling, float* scores, int32_t scores_cap,
                          void* ws, size_t ws_bytes, void* stream) {
  int rc = check_layer(L);
  if (rc) return rc;
  if (T <= 0 || !q || !k || !v || !out) return SKV_ERR_INVALID_ARG;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16)) return SKV_ERR_MISALIGNED;
  const Geometry g = geometry(L, T, 0);
  if (scores && scores_cap < g.num_windows()) return SKV_ERR_CAPACITY;
  if (!ws || ws_bytes < skv_prefill_workspace_size(L, T)) return SKV_ERR_WORKSPACE;
  return prefill_dispatch(L, T, q, k, v, out, scaling, scores, scores_cap, ws, (cudaStream_t)stream);
}

int skv_materialize(const skv_layer_desc* L, int32_t seq_len, int32_t tier_pages, void* k_out, void* v_out,
                    void* stream) {
  int rc = check_layer(L);
  if (rc) return rc;
  if (seq_len <= 0 || !k_out || !v_out) return SKV_ERR_INVALID_ARG;
  if ((rc = check_counts(L, seq_len, tier_pages))) return rc;
  if (tier_pages > 0 && L->rope_positions < L->num_sink + tier_pages * kPageTokens) return SKV_ERR_CAPACITY;
  return materialize_dispatch(L, seq_len, tier_pages, k_out, v_out, (cudaStream_t)stream);
}

int skv_pack_pages(const skv_layer_desc* L, const void* k, const void* v, int32_t first_pos,
                   int32_t n_pages, uint8_t* out, void* stream) {
  if (!L || !k || !v || !out || n_pages <= 0 || first_pos < 0) return SKV_ERR_INVALID_ARG;
  if (L->head_dim % kQGroup || elt_size(L->kv_dtype) == 0) return SKV_ERR_UNSUPPORTED;
  if (!L->rope_cos || !L->rope_sin) return SKV_ERR_INVALID_ARG;
  if (L->rope_positions < first_pos + n_pages * kPageTokens) return SKV_ERR_CAPACITY;
  return pack_pages_dispatch(L, k, v, first_pos, n_pages, out, (cudaStream_t)stream);
}

}  // extern "C"
