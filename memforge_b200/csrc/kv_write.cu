// KV writes into the paged pool: reshape_and_cache (slot-mapping scatter), the
// speculative commit of a window's confirmed rows, and the all-layer
// copy-on-write block copy; and the materialising read (gather_kv).
//
// Both are byte-moving kernels bounded by HBM: every thread moves one 16-byte
// vector (8 bf16 / 4 fp32 elements) when the row is 16-byte aligned, so each
// warp issues fully coalesced 512-byte transactions along head_dim.

#include "mf_internal.h"

namespace mf {

template <typename S, typename P>
MF_DEVINL void copy_row_vec(const S* __restrict__ src, P* __restrict__ dst, int nvec_elems);

template <typename S, typename P>
__global__ void reshape_and_cache_kernel(const S* __restrict__ key, const S* __restrict__ value,
                                         int64_t k_stride_tok, int64_t k_stride_head,
                                         int64_t v_stride_tok, int64_t v_stride_head,
                                         P* __restrict__ key_pool, P* __restrict__ value_pool,
                                         int64_t sb, int64_t ss, int64_t sh, int64_t num_slots,
                                         int32_t block_size, const void* __restrict__ slots,
                                         int slots64, int num_tokens, int num_heads,
                                         int head_dim, int vec, int32_t* err) {
  // The attention kernel that usually follows may be scheduled now: it waits
  // for this kernel's completion before it reads anything.
  grid_launch_dependents();
  // One work item = (token, head, vector of `vec` elements along head_dim).
  const int vecs_per_row = head_dim / vec;
  const int64_t total = (int64_t)num_tokens * num_heads * vecs_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int v = (int)(i % vecs_per_row);
    const int64_t th = i / vecs_per_row;
    const int h = (int)(th % num_heads);
    const int t = (int)(th / num_heads);
    const int64_t slot = slots64 ? reinterpret_cast<const int64_t*>(slots)[t]
                                 : (int64_t)reinterpret_cast<const int32_t*>(slots)[t];
    if (slot < 0) {
      if (slot != -1 && v == 0 && h == 0) set_err(err, MF_ERR_SLOT);
      continue;
    }
    if (slot >= num_slots) {
      if (v == 0 && h == 0) set_err(err, MF_ERR_SLOT);
      continue;
    }
    const int64_t dst_off = (slot / block_size) * sb + (slot % block_size) * ss + h * sh + (int64_t)v * vec;
    const S* ks = key + t * k_stride_tok + h * k_stride_head + (int64_t)v * vec;
    const S* vs = value + t * v_stride_tok + h * v_stride_head + (int64_t)v * vec;
    copy_row_vec<S, P>(ks, key_pool + dst_off, vec);
    copy_row_vec<S, P>(vs, value_pool + dst_off, vec);
  }
}

template <typename S, typename P>
MF_DEVINL void copy_row_vec(const S* __restrict__ src, P* __restrict__ dst, int n) {
  if constexpr (sizeof(S) == sizeof(P) && std::is_same<S, P>::value) {
    if (n * sizeof(S) == 16) {
      *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
    } else {
      for (int j = 0; j < n; ++j) dst[j] = src[j];
    }
  } else {
    // Widening is not supported; narrowing f32 -> f16/bf16 rounds like torch.
    for (int j = 0; j < n; ++j) dst[j] = from_f32<P>(Elt<S>::to_f32(src[j]));
  }
}

// Speculative commit, all layers in one launch: row j of sequence b's window
// goes to pool position
// ctx[b] + j, through b's block table, for j < num_confirmed[b]; the other rows
// (rejected drafts) are not written, so their slots keep what they held.  The
// slot arithmetic of PagedKVPool.slot_indices (memforge_ml/runtime/
// kv_pool.py:92-130) runs on the device.  A confirmed count of 0 or less is a
// no-op (scatter_accepted_kv returns early); a count above the window, a
// confirmed position past the table row or a block id outside the pool sets an
// error bit and skips every row of that sequence in every layer, as the
// reference's IndexError stops the write before it starts.
template <typename S, typename P>
__global__ void commit_window_kernel(const S* __restrict__ wk, const S* __restrict__ wv,
                                     int64_t k_stride_layer, int64_t k_stride_row,
                                     int64_t k_stride_head, int64_t v_stride_layer,
                                     int64_t v_stride_row, int64_t v_stride_head,
                                     P* __restrict__ key_pool, P* __restrict__ value_pool,
                                     int64_t sl, int64_t sb, int64_t ss, int64_t sh,
                                     int num_layers, int32_t num_blocks, int32_t block_size,
                                     const int32_t* __restrict__ tables, int32_t table_stride,
                                     const int32_t* __restrict__ ctx_lens,
                                     const int32_t* __restrict__ num_confirmed, int num_seqs,
                                     int window, int num_heads, int head_dim, int vec,
                                     int32_t* err) {
  const int vecs_per_row = head_dim / vec;
  const int64_t per_layer = (int64_t)num_seqs * window * num_heads * vecs_per_row;
  const int64_t total = per_layer * num_layers;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int layer = (int)(i / per_layer);
    const int64_t li = i - (int64_t)layer * per_layer;
    const int v = (int)(li % vecs_per_row);
    const int64_t rh = li / vecs_per_row;
    const int h = (int)(rh % num_heads);
    const int64_t r = rh / num_heads;  // window row, sequence-major
    const int b = (int)(r / window), j = (int)(r % window);
    // One error report per sequence.  The whole confirmed prefix is validated
    // before any of its rows is written, so a sequence the reference would
    // reject (IndexError from slot_indices before the first layer's write)
    // leaves the pool untouched in every layer.
    const bool lead = v == 0 && h == 0 && layer == 0 && j == 0;
    const int n = __ldg(num_confirmed + b);
    const int c = __ldg(ctx_lens + b);
    if (n <= 0 || j >= n) continue;  // nothing confirmed: a no-op, as in the reference
    if (n > window || c < 0) {
      if (lead) set_err(err, MF_ERR_LENGTH);
      continue;
    }
    const int64_t first_page = (int64_t)c / block_size;
    const int64_t last_page = ((int64_t)c + n - 1) / block_size;
    if (last_page >= table_stride) {
      if (lead) set_err(err, MF_ERR_TABLE);
      continue;
    }
    bool ids_ok = true;
    for (int64_t p = first_page; p <= last_page; ++p) {
      const int id = __ldg(tables + (int64_t)b * table_stride + p);
      ids_ok = ids_ok && id >= 0 && id < num_blocks;
    }
    if (!ids_ok) {
      if (lead) set_err(err, MF_ERR_BLOCK_ID);
      continue;
    }
    const int64_t pos = (int64_t)c + j;
    const int64_t page = pos / block_size;
    const int blk = __ldg(tables + (int64_t)b * table_stride + page);
    const int64_t dst_off = layer * sl + (int64_t)blk * sb + (pos % block_size) * ss + h * sh +
                            (int64_t)v * vec;
    copy_row_vec<S, P>(
        wk + layer * k_stride_layer + r * k_stride_row + h * k_stride_head + (int64_t)v * vec,
        key_pool + dst_off, vec);
    copy_row_vec<S, P>(
        wv + layer * v_stride_layer + r * v_stride_row + h * v_stride_head + (int64_t)v * vec,
        value_pool + dst_off, vec);
  }
}

// Materialising read (paged_gather.gather_kv / PagedKVPool.gather_flat,
// memforge_ml/kernels/paged_gather.py:58-89): output row t holds pool slot
// flat_index[t] for every kv head, written head-major (element (h, t, d) at
// out + h*o_sh + t*o_st + d), the (1, H, T, D) layout the reference returns.
// One work item = (token, head, vector of `vec` elements): a warp reads one
// slot's heads contiguously and writes each head's row as whole 16-byte
// vectors.  A slot outside the pool sets MF_ERR_SLOT and yields zeros.
template <typename T>
__global__ void gather_kv_kernel(const T* __restrict__ kp, const T* __restrict__ vp, int64_t sb,
                                 int64_t ss, int64_t sh, int64_t num_slots, int32_t block_size,
                                 const void* __restrict__ index, int index64, int num_tokens,
                                 int num_heads, int head_dim, int vec, T* __restrict__ ko,
                                 T* __restrict__ vo, int64_t o_sh, int64_t o_st, int32_t* err) {
  const int vecs_per_row = head_dim / vec;
  const int64_t total = (int64_t)num_tokens * num_heads * vecs_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int v = (int)(i % vecs_per_row);
    const int64_t th = i / vecs_per_row;
    const int h = (int)(th % num_heads);
    const int t = (int)(th / num_heads);
    const int64_t slot = index64 ? reinterpret_cast<const int64_t*>(index)[t]
                                 : (int64_t)reinterpret_cast<const int32_t*>(index)[t];
    T* kd = ko + h * o_sh + (int64_t)t * o_st + (int64_t)v * vec;
    T* vd = vo + h * o_sh + (int64_t)t * o_st + (int64_t)v * vec;
    if (slot < 0 || slot >= num_slots) {
      if (v == 0 && h == 0) set_err(err, MF_ERR_SLOT);
      for (int j = 0; j < vec; ++j) {
        kd[j] = from_f32<T>(0.f);
        vd[j] = from_f32<T>(0.f);
      }
      continue;
    }
    const int64_t src = (slot / block_size) * sb + (slot % block_size) * ss + h * sh + (int64_t)v * vec;
    copy_row_vec<T, T>(kp + src, kd, vec);
    copy_row_vec<T, T>(vp + src, vd, vec);
  }
}

__global__ void copy_blocks_kernel(uint8_t* __restrict__ kp, uint8_t* __restrict__ vp,
                                   int num_layers, int num_blocks, int64_t block_bytes,
                                   const int32_t* __restrict__ pairs, int num_pairs,
                                   int32_t* err) {
  // grid.y = pair, grid.z = layer; threads stride the block's bytes in 16B units.
  const int pair = blockIdx.y;
  const int layer = blockIdx.z;
  const int src = pairs[2 * pair];
  const int dst = pairs[2 * pair + 1];
  if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && layer == 0) set_err(err, MF_ERR_BLOCK_ID);
    return;
  }
  if (src == dst) return;
  const int64_t layer_off = (int64_t)layer * num_blocks * block_bytes;
  const int64_t n16 = block_bytes / 16;
  const uint4* ks = reinterpret_cast<const uint4*>(kp + layer_off + (int64_t)src * block_bytes);
  const uint4* vs = reinterpret_cast<const uint4*>(vp + layer_off + (int64_t)src * block_bytes);
  uint4* kd = reinterpret_cast<uint4*>(kp + layer_off + (int64_t)dst * block_bytes);
  uint4* vd = reinterpret_cast<uint4*>(vp + layer_off + (int64_t)dst * block_bytes);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16;
       i += (int64_t)gridDim.x * blockDim.x) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

}  // namespace mf

using namespace mf;

namespace {

template <typename S, typename P>
int launch_rac(const void* key, const void* value, int64_t kst, int64_t ksh, int64_t vst,
               int64_t vsh, void* kp, void* vp, int64_t sb, int64_t ss, int64_t sh,
               int64_t num_slots, int32_t bs, const void* slots, int slots64, int T, int H,
               int D, int32_t* err, cudaStream_t stream) {
  // 16-byte vectors when every row start is 16-byte aligned, else scalar.
  int vec = 1;
  const int v16 = 16 / (int)sizeof(P);
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (std::is_same<S, P>::value && D % v16 == 0 && al(key) && al(value) && al(kp) && al(vp) &&
      (kst * sizeof(S)) % 16 == 0 && (ksh * sizeof(S)) % 16 == 0 &&
      (vst * sizeof(S)) % 16 == 0 && (vsh * sizeof(S)) % 16 == 0 &&
      (sb * sizeof(P)) % 16 == 0 && (ss * sizeof(P)) % 16 == 0 && (sh * sizeof(P)) % 16 == 0) {
    vec = v16;
  }
  const int64_t items = (int64_t)T * H * (D / vec);
  if (items == 0) return MF_OK;
  const int threads = 256;
  int64_t blocks = (items + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  reshape_and_cache_kernel<S, P><<<(unsigned)blocks, threads, 0, stream>>>(
      static_cast<const S*>(key), static_cast<const S*>(value), kst, ksh, vst, vsh,
      static_cast<P*>(kp), static_cast<P*>(vp), sb, ss, sh, num_slots, bs, slots, slots64, T, H,
      D, vec, err);
  return check_launch("reshape_and_cache");
}

template <typename T>
int launch_gather(const void* kp, const void* vp, int64_t sb, int64_t ss, int64_t sh,
                  int64_t num_slots, int32_t bs, const void* index, int index64, int T_, int H,
                  int D, void* ko, void* vo, int64_t o_sh, int64_t o_st, int32_t* err,
                  cudaStream_t stream) {
  int vec = 1;
  const int v16 = 16 / (int)sizeof(T);
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  auto al16 = [](int64_t stride) { return (stride * (int64_t)sizeof(T)) % 16 == 0; };
  if (D % v16 == 0 && al(kp) && al(vp) && al(ko) && al(vo) && al16(sb) && al16(ss) &&
      al16(sh) && al16(o_sh) && al16(o_st)) {
    vec = v16;
  }
  const int64_t items = (int64_t)T_ * H * (D / vec);
  const int threads = 256;
  int64_t blocks = (items + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  gather_kv_kernel<T><<<(unsigned)blocks, threads, 0, stream>>>(
      static_cast<const T*>(kp), static_cast<const T*>(vp), sb, ss, sh, num_slots, bs, index,
      index64, T_, H, D, vec, static_cast<T*>(ko), static_cast<T*>(vo), o_sh, o_st, err);
  return check_launch("gather_kv");
}

template <typename S, typename P>
int launch_commit(const void* wk, const void* wv, int64_t ksl, int64_t kst, int64_t ksh,
                  int64_t vsl, int64_t vst, int64_t vsh, void* kp, void* vp, int64_t sl,
                  int64_t sb, int64_t ss, int64_t sh, int L, int32_t nb, int32_t bs,
                  const int32_t* tables, int32_t table_stride, const int32_t* ctx,
                  const int32_t* conf, int B, int W, int H, int D, int32_t* err,
                  cudaStream_t stream) {
  int vec = 1;
  const int v16 = 16 / (int)sizeof(P);
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  auto al16 = [](int64_t stride, size_t elt) { return (stride * (int64_t)elt) % 16 == 0; };
  if (std::is_same<S, P>::value && D % v16 == 0 && al(wk) && al(wv) && al(kp) && al(vp) &&
      al16(ksl, sizeof(S)) && al16(kst, sizeof(S)) && al16(ksh, sizeof(S)) &&
      al16(vsl, sizeof(S)) && al16(vst, sizeof(S)) && al16(vsh, sizeof(S)) &&
      al16(sl, sizeof(P)) && al16(sb, sizeof(P)) && al16(ss, sizeof(P)) && al16(sh, sizeof(P))) {
    vec = v16;
  }
  const int64_t items = (int64_t)L * B * W * H * (D / vec);
  const int threads = 256;
  int64_t blocks = (items + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  commit_window_kernel<S, P><<<(unsigned)blocks, threads, 0, stream>>>(
      static_cast<const S*>(wk), static_cast<const S*>(wv), ksl, kst, ksh, vsl, vst, vsh,
      static_cast<P*>(kp), static_cast<P*>(vp), sl, sb, ss, sh, L, nb, bs, tables, table_stride,
      ctx, conf, B, W, H, D, vec, err);
  return check_launch("commit_window");
}

}  // namespace

extern "C" int mf_reshape_and_cache(const void* key, const void* value, mf_dtype src_dtype,
                                    int64_t k_stride_tok, int64_t k_stride_head,
                                    int64_t v_stride_tok, int64_t v_stride_head, void* key_pool,
                                    void* value_pool, mf_dtype pool_dtype,
                                    int64_t pool_stride_block, int64_t pool_stride_slot,
                                    int64_t pool_stride_head, int32_t num_blocks,
                                    int32_t block_size, const void* slot_mapping,
                                    int32_t slot_mapping_is_int64, int32_t num_tokens,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t* err_flag,
                                    mf_stream_t stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks <= 0)
    return fail(MF_EINVAL, "reshape_and_cache: non-positive size");
  if (num_tokens == 0) return MF_OK;
  if (!key || !value || !key_pool || !value_pool || !slot_mapping)
    return fail(MF_EINVAL, "reshape_and_cache: null pointer");
  const int64_t num_slots = (int64_t)num_blocks * block_size;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
#define MF_RAC(S, P)                                                                          \
  return launch_rac<S, P>(key, value, k_stride_tok, k_stride_head, v_stride_tok,              \
                          v_stride_head, key_pool, value_pool, pool_stride_block,             \
                          pool_stride_slot, pool_stride_head, num_slots, block_size,          \
                          slot_mapping, slot_mapping_is_int64, num_tokens, num_kv_heads,      \
                          head_dim, err_flag, s)
  if (src_dtype == pool_dtype) {
    if (pool_dtype == MF_F32) MF_RAC(float, float);
    if (pool_dtype == MF_F16) MF_RAC(__half, __half);
    if (pool_dtype == MF_BF16) MF_RAC(__nv_bfloat16, __nv_bfloat16);
  } else if (src_dtype == MF_F32) {
    if (pool_dtype == MF_F16) MF_RAC(float, __half);
    if (pool_dtype == MF_BF16) MF_RAC(float, __nv_bfloat16);
  }
#undef MF_RAC
  return fail(MF_EUNSUPPORTED, "reshape_and_cache: unsupported (src, pool) dtype pair");
}

extern "C" int mf_copy_blocks(void* key_pool, void* value_pool, int32_t num_layers,
                              int32_t num_blocks, int64_t block_elems, int32_t elem_bytes,
                              const int32_t* src_dst_pairs, int32_t num_pairs, int32_t* err_flag,
                              mf_stream_t stream) {
  if (num_pairs == 0) return MF_OK;
  if (!key_pool || !value_pool || !src_dst_pairs || num_pairs < 0 || num_layers <= 0 ||
      num_blocks <= 0 || block_elems <= 0 || elem_bytes <= 0)
    return fail(MF_EINVAL, "copy_blocks: bad argument");
  const int64_t block_bytes = block_elems * elem_bytes;
  if (block_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(key_pool) & 15) ||
      (reinterpret_cast<uintptr_t>(value_pool) & 15))
    return fail(MF_EINVAL, "copy_blocks: blocks must be 16-byte multiples, pools 16-byte aligned");
  if (num_pairs > 65535 || num_layers > 65535)
    return fail(MF_EINVAL, "copy_blocks: at most 65535 pairs and layers per call");
  const int64_t n16 = block_bytes / 16;
  int gx = (int)((n16 + 255) / 256);
  if (gx > 64) gx = 64;
  dim3 grid(gx, num_pairs, num_layers);
  copy_blocks_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(key_pool), static_cast<uint8_t*>(value_pool), num_layers, num_blocks,
      block_bytes, src_dst_pairs, num_pairs, err_flag);
  return check_launch("copy_blocks");
}

extern "C" int mf_commit_window(const void* win_k, const void* win_v, mf_dtype src_dtype,
                                int64_t k_stride_layer, int64_t k_stride_row,
                                int64_t k_stride_head, int64_t v_stride_layer,
                                int64_t v_stride_row, int64_t v_stride_head, void* key_pool,
                                void* value_pool, mf_dtype pool_dtype, int64_t pool_stride_layer,
                                int64_t pool_stride_block, int64_t pool_stride_slot,
                                int64_t pool_stride_head, int32_t num_layers, int32_t num_blocks,
                                int32_t block_size, const int32_t* block_tables,
                                int32_t table_stride, const int32_t* ctx_lens,
                                const int32_t* num_confirmed, int32_t num_seqs, int32_t window,
                                int32_t num_kv_heads, int32_t head_dim, int32_t* err_flag,
                                mf_stream_t stream) {
  if (num_seqs < 0 || num_layers <= 0 || window <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_size <= 0 || num_blocks <= 0 || table_stride < 0)
    return fail(MF_EINVAL, "commit_window: non-positive size");
  if (num_seqs == 0) return MF_OK;
  if (!win_k || !win_v || !key_pool || !value_pool || !block_tables || !ctx_lens ||
      !num_confirmed)
    return fail(MF_EINVAL, "commit_window: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
#define MF_COMMIT(S, P)                                                                        \
  return launch_commit<S, P>(win_k, win_v, k_stride_layer, k_stride_row, k_stride_head,        \
                             v_stride_layer, v_stride_row, v_stride_head, key_pool, value_pool, \
                             pool_stride_layer, pool_stride_block, pool_stride_slot,            \
                             pool_stride_head, num_layers, num_blocks, block_size,              \
                             block_tables, table_stride, ctx_lens, num_confirmed, num_seqs,     \
                             window, num_kv_heads, head_dim, err_flag, s)
  if (src_dtype == pool_dtype) {
    if (pool_dtype == MF_F32) MF_COMMIT(float, float);
    if (pool_dtype == MF_F16) MF_COMMIT(__half, __half);
    if (pool_dtype == MF_BF16) MF_COMMIT(__nv_bfloat16, __nv_bfloat16);
  } else if (src_dtype == MF_F32) {
    if (pool_dtype == MF_F16) MF_COMMIT(float, __half);
    if (pool_dtype == MF_BF16) MF_COMMIT(float, __nv_bfloat16);
  }
#undef MF_COMMIT
  return fail(MF_EUNSUPPORTED, "commit_window: unsupported (src, pool) dtype pair");
}

extern "C" int mf_gather_kv(const void* key_pool, const void* value_pool, mf_dtype dtype,
                            int64_t pool_stride_block, int64_t pool_stride_slot,
                            int64_t pool_stride_head, int32_t num_blocks, int32_t block_size,
                            const void* flat_index, int32_t index_is_int64, int32_t num_tokens,
                            int32_t num_kv_heads, int32_t head_dim, void* key_out,
                            void* value_out, int64_t out_stride_head, int64_t out_stride_tok,
                            int32_t* err_flag, mf_stream_t stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks <= 0)
    return fail(MF_EINVAL, "gather_kv: non-positive size");
  if (num_tokens == 0) return MF_OK;
  if (!key_pool || !value_pool || !flat_index || !key_out || !value_out)
    return fail(MF_EINVAL, "gather_kv: null pointer");
  const int64_t num_slots = (int64_t)num_blocks * block_size;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
#define MF_GATHER(T)                                                                          \
  return launch_gather<T>(key_pool, value_pool, pool_stride_block, pool_stride_slot,          \
                          pool_stride_head, num_slots, block_size, flat_index, index_is_int64, \
                          num_tokens, num_kv_heads, head_dim, key_out, value_out,              \
                          out_stride_head, out_stride_tok, err_flag, s)
  if (dtype == MF_F32) MF_GATHER(float);
  if (dtype == MF_F16) MF_GATHER(__half);
  if (dtype == MF_BF16) MF_GATHER(__nv_bfloat16);
#undef MF_GATHER
  return fail(MF_EUNSUPPORTED, "gather_kv: unsupported dtype");
}
