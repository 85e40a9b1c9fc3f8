/*
 * memforge_sm100.h — C ABI of the B200 (sm_100a) paged-attention library.
 *
 * This library replaces the KV-scatter and paged-attention hot path of
 * MemForge (reference paths below are relative to the MemForge source tree).
 * Every entry point:
 *   - takes plain device pointers, element strides and sizes (no framework types);
 *   - is stream-ordered on `stream` (NULL = the legacy default stream) and never
 *     synchronises the device or allocates device memory;
 *   - returns 0 on success or a negative MF_E* code; `mf_last_error()` then
 *     gives a message (per calling thread);
 *   - optionally reports device-side violations (a bad block id, a slot past the
 *     pool, a bounded wait that gave up) by OR-ing MF_ERR_* bits into `*err_flag`
 *     (a device int32 the caller zeroes and reads back when it wants to check).
 *     Such a launch never traps: the offending access is skipped or clamped.
 *
 * Pool addressing (one layer): element (slot s, kv head h, dim d) lives at
 *   base + (s / block_size) * stride_block + (s % block_size) * stride_slot
 *        + h * stride_head + d
 * which covers MemForge's pool layer `(blocks, block_size, kv_heads, head_dim)`
 * (memforge_ml/runtime/kv_pool.py:66) and the standalone operator's cache
 * `(blocks, heads, block_size, head_dim)` (memforge_ml/models/paged_attention.py:34-43).
 */
#ifndef MEMFORGE_SM100_H
#define MEMFORGE_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MF_ABI_VERSION 1

#if defined(__GNUC__)
#define MF_API __attribute__((visibility("default")))
#else
#define MF_API
#endif

/* Same object as cudaStream_t. */
typedef struct CUstream_st* mf_stream_t;

typedef enum { MF_F32 = 0, MF_F16 = 1, MF_BF16 = 2 } mf_dtype;

enum {
  MF_OK = 0,
  MF_EINVAL = -1,        /* bad argument: null pointer, shape, stride, dtype */
  MF_EBOUNDS = -2,       /* host-visible bound violation */
  MF_ETIMEOUT = -3,      /* reserved: a bounded wait gave up (also MF_ERR_TIMEOUT) */
  MF_ECUDA = -4,         /* CUDA runtime error while launching */
  MF_EUNSUPPORTED = -5,  /* no kernel in this build handles the shape */
  MF_EWORKSPACE = -6     /* workspace missing or too small */
};

/* Bits OR-ed into *err_flag by kernels. */
#define MF_ERR_BLOCK_ID 0x1  /* block table entry outside [0, num_blocks) */
#define MF_ERR_SLOT 0x2      /* slot_mapping entry outside [-1, num_blocks*block_size) */
#define MF_ERR_TABLE 0x4     /* a context needs more blocks than the table row holds */
#define MF_ERR_LENGTH 0x8    /* kv_len < q_len, or a confirmed count above the window */
#define MF_ERR_TIMEOUT 0x10  /* a bounded pipeline wait gave up */

MF_API int mf_abi_version(void);
MF_API const char* mf_last_error(void);

/* Number of multiprocessors and whether the device is sm_100 (1) or not (0). */
MF_API int mf_device_info(int device, int* num_sms, int* is_sm100);

/*
 * reshape_and_cache — scatter new K/V rows into the paged pool.
 *
 * Replaces paged_gather.scatter_kv (memforge_ml/kernels/paged_gather.py:92-117)
 * and PagedKVPool.write_flat / write (memforge_ml/runtime/kv_pool.py:134-149,
 * 181-192): token t, head h of `key`/`value` (element (t, h, d) at
 * key + t*k_stride_tok + h*k_stride_head + d) lands at pool slot
 * slot_mapping[t].  A slot of -1 skips the token (padding).  When src_dtype
 * differs from pool_dtype the values are rounded to the pool dtype exactly as
 * torch's `.to()` does (round to nearest even; NaN -> the canonical NaN).
 * Supported (src, pool): (f32,f32) (f16,f16) (bf16,bf16) (f32,bf16) (f32,f16).
 * Two tokens naming one slot race (the reference rejects that case,
 * memforge_ml/runtime/varlen_cache.py:186-190).
 */
MF_API int mf_reshape_and_cache(const void* key, const void* value, mf_dtype src_dtype,
                         int64_t k_stride_tok, int64_t k_stride_head,
                         int64_t v_stride_tok, int64_t v_stride_head,
                         void* key_pool, void* value_pool, mf_dtype pool_dtype,
                         int64_t pool_stride_block, int64_t pool_stride_slot,
                         int64_t pool_stride_head, int32_t num_blocks, int32_t block_size,
                         const void* slot_mapping, int32_t slot_mapping_is_int64,
                         int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                         int32_t* err_flag, mf_stream_t stream);

/*
 * gather_kv — materialise a contiguous copy of some pool slots.
 *
 * Replaces paged_gather.gather_kv (memforge_ml/kernels/paged_gather.py:58-89)
 * and PagedKVPool.gather / gather_flat (memforge_ml/runtime/kv_pool.py:151-179):
 * for token t, head h, element (h, t, d) of key_out/value_out (at
 * out + h*out_stride_head + t*out_stride_tok + d) is pool slot flat_index[t]'s
 * element (h, d), i.e. the (1, heads, tokens, head_dim) layout the reference
 * returns.  An index outside [0, num_blocks*block_size) sets MF_ERR_SLOT and
 * yields zeros (the reference's index_select raises).  Bit-exact copy.
 */
MF_API int mf_gather_kv(const void* key_pool, const void* value_pool, mf_dtype dtype,
                        int64_t pool_stride_block, int64_t pool_stride_slot,
                        int64_t pool_stride_head, int32_t num_blocks, int32_t block_size,
                        const void* flat_index, int32_t index_is_int64, int32_t num_tokens,
                        int32_t num_kv_heads, int32_t head_dim, void* key_out,
                        void* value_out, int64_t out_stride_head, int64_t out_stride_tok,
                        int32_t* err_flag, mf_stream_t stream);

/*
 * Paged attention over block tables: decode, speculative verify and varlen
 * chunked prefill in one contract.
 *
 * Sequence s owns query rows [q_start(s), q_start(s) + q_len(s)) where
 * q_start/q_len come from cu_seqlens_q[s..s+1] (or s*q_per_seq / q_per_seq when
 * cu_seqlens_q is NULL).  kv_lens[s] is the number of keys visible to its LAST
 * query row.  With causal != 0, row i (0-based within the sequence) attends to
 * key positions 0 .. kv_lens[s] - q_len(s) + i; with causal == 0 every row
 * attends to 0 .. kv_lens[s] - 1.  Key position p of sequence s is pool slot
 * block_tables[s*table_stride + p/block_size]*block_size + p%block_size, except
 * that, when win_k/win_v are given, positions kv_lens[s]-q_len(s)+j come from
 * window row q_start(s)+j instead (the speculative-verify side buffer, so that
 * rejected drafts never touch the pool).
 *
 * This is the semantics of paged_attention_varlen / _materialised
 * (memforge_ml/kernels/varlen_attention.py:78-235, 291-395) with every
 * sequence's rows at consecutive positions, of paged_attention_blockwise
 * (memforge_ml/kernels/block_attention.py:51-145) for one row, and of the
 * Triton paged_decode_attention (memforge_ml/kernels/triton_paged_decode.py:
 * 129-176) with q_per_seq = 1.  fp32 accumulation; the output has `dtype`.
 * GQA: query head hq reads kv head hq / (num_q_heads / num_kv_heads).
 * row_map (optional) sends logical row r to packed row row_map[r] for q, out
 * and the window (arbitrary packing orders, varlen_attention.py:60-75).
 */
#define MF_MAX_OUT_PEERS 8

typedef struct {
  uint32_t struct_size; /* sizeof(mf_attention_args); the size up to `dtype` is
                           accepted too (no peer output) */
  const void* q;        /* [rows][num_q_heads][head_dim] */
  int64_t q_stride_row, q_stride_head;
  void* out;            /* same indexing as q */
  int64_t out_stride_row, out_stride_head;
  const void* k_pool;   /* one layer of the pool */
  const void* v_pool;
  int64_t pool_stride_block, pool_stride_slot, pool_stride_head;
  int32_t num_blocks, block_size;
  const int32_t* block_tables; /* [num_seqs][table_stride] */
  int32_t table_stride;
  const int32_t* cu_seqlens_q; /* [num_seqs + 1] or NULL */
  int32_t q_per_seq;           /* used when cu_seqlens_q is NULL */
  const int32_t* kv_lens;      /* [num_seqs] */
  const int32_t* row_map;      /* [total_q] or NULL */
  const void* win_k;           /* [rows][num_kv_heads][head_dim] or NULL */
  const void* win_v;
  int64_t win_stride_row, win_stride_head;
  int32_t num_seqs, total_q, max_q_len;
  int32_t num_q_heads, num_kv_heads, head_dim;
  float scale;
  int32_t causal;
  mf_dtype dtype;
  /* Head-sharded output over peer memory (optional; read only when struct_size
   * is the full size of this struct, and ignored when num_out_peers == 0).
   * When a KV pool is split by kv head across GPUs (one process per GPU, the
   * partition memforge_b200.kv_shard implements), each GPU computes
   * num_q_heads heads of a wider output [rows][total heads][head_dim].  With
   * num_out_peers = N > 0 the decode kernel writes every output row of its
   * heads, at head index out_head_offset + local head, straight into all N
   * buffers out_peers[0..N-1] (this GPU's own and the peers' copies of that
   * output, mapped into this process, e.g. through CUDA IPC), with the
   * out_stride_* strides; `out` is not written.  This replaces the all-gather
   * after the attention with stores over NVLink.  The peers may read the output
   * once mf_peer_barrier has completed on every GPU.  Decode batches only (every
   * run of up to 8 rows per kv head): other batches return MF_EUNSUPPORTED. */
  int32_t num_out_peers;
  int32_t out_head_offset;
  void* out_peers[MF_MAX_OUT_PEERS];
} mf_attention_args;

/* Device workspace `mf_paged_attention` needs for these arguments on `device`
 * (0 when none).  The caller allocates it once, ZERO-FILLED, and may reuse it
 * for any later call with an equal or smaller requirement on the same stream:
 * its front holds split-K arrival counters, which every launch leaves zero
 * again; the rest holds partial results that each launch overwrites before
 * reading.  Concurrent launches must not share one. */
MF_API size_t mf_paged_attention_workspace_size(const mf_attention_args* args, int device);

MF_API int mf_paged_attention(const mf_attention_args* args, void* workspace,
                       size_t workspace_bytes, int32_t* err_flag, mf_stream_t stream);

/*
 * Triton-signature decode (memforge_ml/kernels/triton_paged_decode.py:129-176):
 * q [B][Hq][D] (row stride q_stride_b, head stride q_stride_h), the layer's pool
 * viewed flat [slots][Hkv][D] with strides (flat_stride_slot, flat_stride_head),
 * block_tables int32 [B][table_stride], ctx_lens int32 [B] counting the new token,
 * out [B][Hq][D] (contiguous).  A thin form of mf_paged_attention with
 * q_per_seq = 1 over a pool of block_size-token blocks.
 */
MF_API int mf_paged_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                    const void* key_flat, const void* value_flat,
                    int64_t flat_stride_slot, int64_t flat_stride_head, int32_t num_slots,
                    const int32_t* block_tables, int32_t table_stride,
                    const int32_t* ctx_lens, int32_t batch, int32_t num_q_heads,
                    int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                    float scale, mf_dtype dtype, void* out, void* workspace,
                    size_t workspace_bytes, int32_t* err_flag, mf_stream_t stream);

/*
 * mf_paged_decode_noalloc — mf_paged_decode without a caller workspace.
 *
 * No counterpart in the reference: MemForge always allocates with torch.  This
 * entry point is for callers that cannot allocate device memory — a host whose
 * device memory belongs to another allocator, or a plugin that is handed only
 * its input and output buffers.  It allocates nothing: split-K scratch comes
 * from a fixed array of MF_NOALLOC_SCRATCH_BYTES inside the library, which every
 * GPU that loads the library keeps until the process exits.
 *   - The first call on a device resolves the array's device address (make
 *     that first call before any stream capture on that device).
 *   - Batches whose split-K plan needs more than MF_NOALLOC_SCRATCH_BYTES are
 *     rejected with MF_EWORKSPACE (use mf_paged_decode with a workspace then).
 *   - All calls share the array: two calls that can run at the same time on the
 *     GPU (different streams, or different host threads) race and corrupt each
 *     other's results.  Calls on one stream are safe.
 * Arguments and semantics are those of mf_paged_decode.
 */
#define MF_NOALLOC_SCRATCH_BYTES (16u << 20)

/*
 * mf_peer_barrier — completes a head-sharded step (see num_out_peers above).
 *
 * No single counterpart in the reference: it takes the place of the NCCL
 * all-gather of head slices that follows sharded attention.  flags[p] is
 * process-mapped memory of GPU p holding `world` int32 counters (zero-filled
 * once).  Stream-ordered after this GPU's attention launch, it publishes `epoch`
 * into every GPU's counter for this rank (system-scope release stores over
 * NVLink) and waits until this GPU's counters from all ranks reach `epoch`
 * (acquire loads).  `epoch` must increase by one per step, starting at 1.  The
 * wait is bounded (2 s): on expiry it sets MF_ERR_TIMEOUT in err_flag and
 * returns, leaving the context usable.
 */
MF_API int mf_peer_barrier(int32_t* const* flags, int32_t world, int32_t rank, uint32_t epoch,
                           int32_t* err_flag, mf_stream_t stream);

/*
 * CUDA IPC for the peer buffers of a head-sharded step (no counterpart in the
 * reference, which is single-GPU).  mf_ipc_export gives the 64-byte IPC handle
 * of the allocation holding device address `ptr` and ptr's offset in it;
 * mf_ipc_open, in another process of the same node with its own device
 * current, maps that allocation (enabling peer access) and returns the address
 * of the exported byte; mf_ipc_close unmaps it.  One allocation can be opened
 * once per process.
 */
#define MF_IPC_HANDLE_BYTES 64
MF_API int mf_ipc_export(const void* ptr, void* handle, uint64_t* offset);
MF_API int mf_ipc_open(const void* handle, uint64_t offset, void** ptr);
MF_API int mf_ipc_close(void* ptr, uint64_t offset);

MF_API int mf_paged_decode_noalloc(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                   const void* key_flat, const void* value_flat,
                                   int64_t flat_stride_slot, int64_t flat_stride_head,
                                   int32_t num_slots, const int32_t* block_tables,
                                   int32_t table_stride, const int32_t* ctx_lens, int32_t batch,
                                   int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                   int32_t block_size, float scale, mf_dtype dtype, void* out,
                                   int32_t* err_flag, mf_stream_t stream);

/*
 * commit_window — write the confirmed prefix of each speculative window into
 * the pool, for every layer, in one launch.
 *
 * Replaces scatter_accepted_kv (memforge_ml/runtime/batched_speculative.py:
 * 780-811), which the batched engine calls per sequence and writes per layer,
 * with its slot arithmetic (PagedKVPool.slot_indices,
 * memforge_ml/runtime/kv_pool.py:92-130): in layer l, window row j of sequence
 * b (element (l, b*window + j, h, d) at win_k + l*k_stride_layer +
 * (b*window + j)*k_stride_row + h*k_stride_head + d) lands at pool position
 * ctx_lens[b] + j, i.e. slot block_tables[b*table_stride + pos/block_size]*
 * block_size + pos%block_size of layer l (pool_stride_layer apart), for
 * j < num_confirmed[b] (the last confirmed token plus the accepted drafts).
 * Rows j >= num_confirmed[b] are not written, so the rejected slots keep their
 * contents, as in the reference.  num_confirmed[b] <= 0 is a no-op (the
 * reference returns early).  Each sequence's confirmed prefix is validated
 * before any of it is written: num_confirmed above `window` sets
 * MF_ERR_LENGTH, a confirmed position past the table row MF_ERR_TABLE, a block
 * id outside the pool MF_ERR_BLOCK_ID, and then none of that sequence's rows is
 * written in any layer (where the reference raises IndexError before writing).
 * Dtype pairs and rounding as mf_reshape_and_cache.  All integer inputs live
 * on the device, so the call is CUDA-graph safe.
 */
MF_API int mf_commit_window(const void* win_k, const void* win_v, mf_dtype src_dtype,
                     int64_t k_stride_layer, int64_t k_stride_row, int64_t k_stride_head,
                     int64_t v_stride_layer, int64_t v_stride_row, int64_t v_stride_head,
                     void* key_pool, void* value_pool, mf_dtype pool_dtype,
                     int64_t pool_stride_layer, int64_t pool_stride_block,
                     int64_t pool_stride_slot, int64_t pool_stride_head,
                     int32_t num_layers, int32_t num_blocks, int32_t block_size,
                     const int32_t* block_tables, int32_t table_stride,
                     const int32_t* ctx_lens, const int32_t* num_confirmed,
                     int32_t num_seqs, int32_t window, int32_t num_kv_heads,
                     int32_t head_dim, int32_t* err_flag, mf_stream_t stream);

/*
 * accept_commit — a speculative round's acceptance decision and the commit of
 * its confirmed prefix, fused into one launch.
 *
 * Replaces, per round, the reference's RejectionSampler.verify_tokens
 * (memforge_ml/speculative/rejection_sampler.py:28-84, reached through
 * resolve_round, memforge_ml/runtime/batched_speculative.py:731-777) followed
 * by scatter_accepted_kv (:780-811).  For sequence b with K = num_drafts draft
 * tokens x_0..x_{K-1}:
 *   - greedy mode (target_probs == NULL): draft i is accepted while
 *     x_i == target_tokens[b][i] (the target's argmax at candidate slot i);
 *     next_token[b] = target_tokens[b][a];
 *   - sampling mode: draft i is accepted while uniforms[b][i] <=
 *     min(1, p_i / (q_i + 1e-9)), p_i = target_probs[b][i][x_i],
 *     q_i = draft_probs[b][i][x_i]; next_token[b] is drawn at
 *     resample_uniform[b] (inverse CDF, vocabulary order) from
 *     max(0, p_a - q_a) renormalised (p_a when that is all zero) if a < K, or
 *     from p_K (the bonus) if every draft was accepted;
 *   a = the number of leading accepted drafts, written to num_accepted[b].
 * When win_k is given, window rows 0..a of sequence b (the last confirmed token
 * plus the accepted drafts; element (l, b*(K+1)+j, h, d) at
 * win_k + l*win_stride_layer + (b*(K+1)+j)*win_stride_row + h*win_stride_head + d)
 * are written at positions ctx_lens[b]+j of every layer, exactly as
 * mf_commit_window with num_confirmed = a + 1 (same validation and error bits;
 * window and pool share the element type, elem_bytes 2 or 4).  Rejected slots
 * keep their contents.  All inputs live on the device: a round (verify
 * attention, the target's softmax, this call) can be one CUDA graph.
 * Probabilities are fp32 [seq][slot][vocab] with the given strides (vocab
 * contiguous); token ids int32.
 */
typedef struct {
  uint32_t struct_size;        /* sizeof(mf_accept_args) */
  int32_t num_seqs, num_drafts;
  const int32_t* draft_tokens; /* [num_seqs][draft_tokens_stride] */
  int64_t draft_tokens_stride;
  const int32_t* target_tokens; /* greedy: [num_seqs][target_tokens_stride], K+1 used */
  int64_t target_tokens_stride;
  const float* target_probs;   /* sampling: [num_seqs][K+1][vocab] or NULL (greedy) */
  int64_t tp_stride_seq, tp_stride_slot;
  const float* draft_probs;    /* sampling: [num_seqs][K][vocab] */
  int64_t dp_stride_seq, dp_stride_slot;
  int32_t vocab;
  const float* uniforms;       /* sampling: [num_seqs][uniforms_stride], K used */
  int64_t uniforms_stride;
  const float* resample_uniform; /* sampling: [num_seqs] */
  int32_t* num_accepted;       /* out: [num_seqs] */
  int32_t* next_token;         /* out: [num_seqs] or NULL */
  /* commit (optional: win_k == NULL decides only) */
  const void* win_k;
  const void* win_v;
  int64_t win_stride_layer, win_stride_row, win_stride_head;
  void* key_pool;
  void* value_pool;
  int64_t pool_stride_layer, pool_stride_block, pool_stride_slot, pool_stride_head;
  int32_t num_layers, num_blocks, block_size;
  const int32_t* block_tables; /* [num_seqs][table_stride] */
  int32_t table_stride;
  const int32_t* ctx_lens;     /* [num_seqs] */
  int32_t num_kv_heads, head_dim, elem_bytes;
  int32_t* err_flag;
} mf_accept_args;

MF_API int mf_accept_commit(const mf_accept_args* args, mf_stream_t stream);

/*
 * Copy-on-write block copy across all layers: for each pair i, block
 * src[i] -> dst[i] in every layer of both pools (prefix_sharing.copy_block,
 * memforge_ml/runtime/prefix_sharing.py:28-42).  Pools are contiguous
 * [num_layers][num_blocks][block_elems] of `elem_bytes`-byte elements.
 */
MF_API int mf_copy_blocks(void* key_pool, void* value_pool, int32_t num_layers,
                   int32_t num_blocks, int64_t block_elems, int32_t elem_bytes,
                   const int32_t* src_dst_pairs, int32_t num_pairs, int32_t* err_flag,
                   mf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MEMFORGE_SM100_H */
