// C ABI entry points: argument validation, kernel selection and error reporting.

#include <mutex>
#include <string>
#include <vector>

#include "mf_attn.h"

namespace mf {

static thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MF_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return MF_OK;
}

int current_sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n;
  }
  return cache[dev];
}

static int sm_count_of(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  return n;
}

// sizeof(mf_attention_args) before the peer-output fields were added.
constexpr uint32_t kArgsSizeNoPeers =
    (uint32_t)((offsetof(mf_attention_args, num_out_peers) + alignof(mf_attention_args) - 1) /
               alignof(mf_attention_args) * alignof(mf_attention_args));

static int to_params(const mf_attention_args* a, int32_t* err, AttnParams& p) {
  if (!a) return fail(MF_EINVAL, "paged attention: null args");
  // The size up to `dtype` (callers built before the peer-output fields) is
  // accepted and means no peer output.
  const bool full = a->struct_size == sizeof(mf_attention_args);
  if (!full && a->struct_size != kArgsSizeNoPeers)
    return fail(MF_EINVAL, "paged attention: mf_attention_args size mismatch (ABI version)");
  p.n_peers = 0;
  p.out_head_offset = 0;
  if (full && a->num_out_peers != 0) {
    if (a->num_out_peers < 0 || a->num_out_peers > MF_MAX_OUT_PEERS)
      return fail(MF_EINVAL, "paged attention: num_out_peers outside [0, MF_MAX_OUT_PEERS]");
    if (a->out_head_offset < 0)
      return fail(MF_EINVAL, "paged attention: negative out_head_offset");
    for (int i = 0; i < a->num_out_peers; ++i) {
      if (!a->out_peers[i]) return fail(MF_EINVAL, "paged attention: null out_peers entry");
      p.out_peers[i] = a->out_peers[i];
    }
    p.n_peers = a->num_out_peers;
    p.out_head_offset = a->out_head_offset;
  }
  if (a->num_seqs < 0 || a->total_q < 0 || a->max_q_len < 0)
    return fail(MF_EINVAL, "paged attention: negative size");
  if (a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->head_dim <= 0)
    return fail(MF_EINVAL, "paged attention: non-positive head count or head_dim");
  if (a->num_q_heads % a->num_kv_heads != 0)
    return fail(MF_EINVAL, "paged attention: query heads not a multiple of kv heads");
  if (a->block_size <= 0 || a->num_blocks <= 0)
    return fail(MF_EINVAL, "paged attention: non-positive block_size or num_blocks");
  if (a->dtype != MF_F32 && a->dtype != MF_F16 && a->dtype != MF_BF16)
    return fail(MF_EINVAL, "paged attention: unknown dtype");
  if (!a->cu_seqlens_q && a->q_per_seq <= 0)
    return fail(MF_EINVAL, "paged attention: q_per_seq must be positive without cu_seqlens_q");
  if ((a->win_k == nullptr) != (a->win_v == nullptr))
    return fail(MF_EINVAL, "paged attention: win_k and win_v go together");
  if (a->num_seqs > 0 && (!a->q || (!a->out && p.n_peers == 0) || !a->k_pool || !a->v_pool ||
                          !a->block_tables || !a->kv_lens))
    return fail(MF_EINVAL, "paged attention: null pointer");
  p.q = a->q;
  p.q_sr = a->q_stride_row;
  p.q_sh = a->q_stride_head;
  p.out = a->out;
  p.o_sr = a->out_stride_row;
  p.o_sh = a->out_stride_head;
  p.kp = a->k_pool;
  p.vp = a->v_pool;
  p.sb = a->pool_stride_block;
  p.ss = a->pool_stride_slot;
  p.sh = a->pool_stride_head;
  p.num_blocks = a->num_blocks;
  p.block_size = a->block_size;
  p.tables = a->block_tables;
  p.table_stride = a->table_stride;
  p.cu_q = a->cu_seqlens_q;
  p.q_per_seq = a->q_per_seq;
  p.kv_lens = a->kv_lens;
  p.row_map = a->row_map;
  p.wk = a->win_k;
  p.wv = a->win_v;
  p.w_sr = a->win_stride_row;
  p.w_sh = a->win_stride_head;
  p.num_seqs = a->num_seqs;
  p.total_q = a->total_q;
  p.max_q_len = a->cu_seqlens_q ? a->max_q_len : a->q_per_seq;
  p.hq = a->num_q_heads;
  p.hkv = a->num_kv_heads;
  p.d = a->head_dim;
  p.scale = a->scale;
  p.causal = a->causal;
  p.err = err;
  return MF_OK;
}

// Query runs of more than 8 rows per kv head (prefill, speculative verify) go to
// the tcgen05 kernel when it serves the call, the runs of up to 8 rows of the
// same call to the decode kernel (each skips the other's sequences on the
// device, so the split needs no host knowledge of the lengths); when every run
// fits the decode kernel's other consumers or the tcgen05 kernel does not
// serve the layout, the decode kernel alone; the generic kernel for anything
// neither serves.
Dispatch plan_dispatch(const AttnParams& p, mf_dtype dtype, int sm_count) {
  Dispatch d;
  const bool window = p.wk != nullptr;
  const int G = p.hq / p.hkv;
  if ((int64_t)G * p.max_q_len > 8 && prefill_tc_unsupported(p, dtype) == nullptr) {
    if (G > 8 || !p.cu_q) {
      // No run is short enough for the decode kernel: G > 8, or every run has
      // the same q_per_seq rows (no cu_seqlens_q), all of them long.
      d.mode = Dispatch::PREFILL;
      d.rows_cap = 0;
      return d;
    }
    d.short_p = p;
    d.short_p.max_q_len = 8 / G;
    d.decode = plan_attn_tc(d.short_p, dtype, sm_count, window, true);
    if (d.decode.ok && d.decode.SW) {
      d.mode = Dispatch::MIXED;
      d.rows_cap = d.decode.rows_cap;
      return d;
    }
  }
  d.decode = plan_attn_tc(p, dtype, sm_count, window);
  if (d.decode.ok) {
    d.mode = Dispatch::DECODE;
    return d;
  }
  d.mode = Dispatch::GENERIC;
  return d;
}

}  // namespace mf

using namespace mf;

extern "C" int mf_abi_version(void) { return MF_ABI_VERSION; }

extern "C" const char* mf_last_error(void) { return g_last_error.c_str(); }

extern "C" int mf_device_info(int device, int* num_sms, int* is_sm100) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return fail(MF_ECUDA, std::string("device info: ") + cudaGetErrorString(e));
  if (num_sms) *num_sms = prop.multiProcessorCount;
  if (is_sm100) *is_sm100 = (prop.major == 10 && prop.minor == 0) ? 1 : 0;
  return MF_OK;
}

extern "C" size_t mf_paged_attention_workspace_size(const mf_attention_args* args, int device) {
  AttnParams p{};
  if (to_params(args, nullptr, p) != MF_OK) return 0;
  const Dispatch d = plan_dispatch(p, args->dtype, sm_count_of(device));
  return (d.mode == Dispatch::DECODE || d.mode == Dispatch::MIXED) ? d.decode.ws_bytes : 0;
}

extern "C" int mf_paged_attention(const mf_attention_args* args, void* workspace,
                                  size_t workspace_bytes, int32_t* err_flag, mf_stream_t stream) {
  AttnParams p{};
  int rc = to_params(args, err_flag, p);
  if (rc != MF_OK) return rc;
  if (p.num_seqs == 0 || p.total_q == 0) return MF_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const Dispatch d = plan_dispatch(p, args->dtype, current_sm_count());
  if (p.n_peers > 0 && d.mode != Dispatch::DECODE)
    return fail(MF_EUNSUPPORTED, "paged attention: peer output (num_out_peers) is served for "
                                 "decode batches only");
  if (d.mode == Dispatch::GENERIC) return launch_attn_generic(p, args->dtype, s);
  if (d.mode == Dispatch::PREFILL) return launch_attn_prefill_tc(p, args->dtype, 0, s);
  if (!workspace || workspace_bytes < d.decode.ws_bytes)
    return fail(MF_EWORKSPACE, "paged attention: workspace missing or smaller than "
                               "mf_paged_attention_workspace_size()");
  if (d.mode == Dispatch::DECODE) return launch_attn_tc(p, args->dtype, d.decode, workspace, s);
  rc = launch_attn_prefill_tc(p, args->dtype, d.rows_cap, s);
  if (rc != MF_OK) return rc;
  return launch_attn_tc(d.short_p, args->dtype, d.decode, workspace, s);
}

extern "C" int mf_paged_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                               const void* key_flat, const void* value_flat,
                               int64_t flat_stride_slot, int64_t flat_stride_head,
                               int32_t num_slots, const int32_t* block_tables,
                               int32_t table_stride, const int32_t* ctx_lens, int32_t batch,
                               int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               int32_t block_size, float scale, mf_dtype dtype, void* out,
                               void* workspace, size_t workspace_bytes, int32_t* err_flag,
                               mf_stream_t stream) {
  if (block_size <= 0 || num_slots % block_size != 0)
    return fail(MF_EINVAL, "paged decode: num_slots is not a multiple of block_size");
  mf_attention_args a{};
  a.struct_size = sizeof(a);
  a.q = q;
  a.q_stride_row = q_stride_b;
  a.q_stride_head = q_stride_h;
  a.out = out;
  a.out_stride_row = (int64_t)num_q_heads * head_dim;
  a.out_stride_head = head_dim;
  a.k_pool = key_flat;
  a.v_pool = value_flat;
  a.pool_stride_block = flat_stride_slot * block_size;
  a.pool_stride_slot = flat_stride_slot;
  a.pool_stride_head = flat_stride_head;
  a.num_blocks = num_slots / block_size;
  a.block_size = block_size;
  a.block_tables = block_tables;
  a.table_stride = table_stride;
  a.cu_seqlens_q = nullptr;
  a.q_per_seq = 1;
  a.kv_lens = ctx_lens;
  a.num_seqs = batch;
  a.total_q = batch;
  a.max_q_len = 1;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.scale = scale;
  a.causal = 1;
  a.dtype = dtype;
  return mf_paged_attention(&a, workspace, workspace_bytes, err_flag, stream);
}
