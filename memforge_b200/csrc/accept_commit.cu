// Fused speculative accept + commit: the acceptance decision of a verify round
// and the write of its confirmed prefix into the pool, in one launch.
//
// The reference decides per sequence on the host (RejectionSampler.verify_tokens,
// memforge_ml/speculative/rejection_sampler.py:28-84, through resolve_round,
// memforge_ml/runtime/batched_speculative.py:731-777) and then writes the
// confirmed rows layer by layer (scatter_accepted_kv, :780-811).  Here one grid
// does both, so a round needs no host round trip between the target's
// probabilities and the pool update:
//
//  * grid (B, 1 + C).  Every CTA of sequence b first computes a, the number of
//    leading accepted drafts (K <= 64 comparisons, done redundantly per CTA so
//    that no CTA waits on another).
//  * CTA (b, 0) writes num_accepted[b] = a and next_token[b], the token that
//    follows the accepted drafts: in greedy mode the target's own choice at
//    slot a; in sampling mode a draw from max(0, p_a - q_a) (renormalised; p_a
//    when that is all zero) after a rejection, or from p_K (the bonus) when all
//    K drafts were accepted, by inverse CDF at resample_uniform[b].  The sum is
//    reduced in a fixed order (a contiguous chunk per thread, then a scan of
//    the chunk sums), so the draw is deterministic.
//  * CTAs (b, 1..C) write window rows 0..a of sequence b (a + 1 rows: the last
//    confirmed token plus the accepted drafts) at positions ctx[b] .. ctx[b]+a,
//    every layer, with mf_commit_window's validation (a sequence whose prefix
//    leaves its table or names a block outside the pool writes nothing).

#include "mf_internal.h"

namespace mf {
namespace {

constexpr int AC_THREADS = 256;
constexpr int AC_MAX_DRAFTS = 64;

struct AcceptParams {
  mf_accept_args a;
  int window;
};

// Leading accepted drafts of sequence b (identical in every CTA of b).
MF_DEVINL int accepted_count(const mf_accept_args& a, int b) {
  const int K = a.num_drafts;
  int n = 0;
  for (int i = 0; i < K; ++i) {
    const int x = a.draft_tokens[(int64_t)b * a.draft_tokens_stride + i];
    bool ok;
    if (a.target_probs == nullptr) {
      ok = x == a.target_tokens[(int64_t)b * a.target_tokens_stride + i];
    } else {
      if (x < 0 || x >= a.vocab) {
        ok = false;
      } else {
        const double p = a.target_probs[(int64_t)b * a.tp_stride_seq + (int64_t)i * a.tp_stride_slot + x];
        const double q = a.draft_probs[(int64_t)b * a.dp_stride_seq + (int64_t)i * a.dp_stride_slot + x];
        // min(1, p / (q + 1e-9)), in double as the reference's Python floats
        const double ratio = fmin(1.0, p / (q + 1e-9));
        ok = (double)a.uniforms[(int64_t)b * a.uniforms_stride + i] <= ratio;
      }
    }
    if (!ok) break;
    ++n;
  }
  return n;
}

// Weight of token v for the draw after `acc` accepted drafts.
MF_DEVINL float draw_weight(const mf_accept_args& a, int b, int acc, int v, bool diff) {
  const float p = a.target_probs[(int64_t)b * a.tp_stride_seq + (int64_t)acc * a.tp_stride_slot + v];
  if (!diff) return fmaxf(p, 0.f);
  const float q = a.draft_probs[(int64_t)b * a.dp_stride_seq + (int64_t)acc * a.dp_stride_slot + v];
  return fmaxf(p - q, 0.f);
}

// Block-wide inverse-CDF draw over the vocabulary (sampling mode), thread 0's
// result is returned in every thread.  Deterministic reduction order.
MF_DEVINL int draw_token(const mf_accept_args& a, int b, int acc, bool diff, float u,
                         float* scan) {
  const int V = a.vocab, T = blockDim.x, t = threadIdx.x;
  const int per = (V + T - 1) / T;
  const int lo = min(V, t * per), hi = min(V, lo + per);
  float local = 0.f;
  for (int v = lo; v < hi; ++v) local += draw_weight(a, b, acc, v, diff);
  scan[t] = local;
  __syncthreads();
  if (t == 0) {
    float run = 0.f;
    for (int i = 0; i < T; ++i) {
      const float x = scan[i];
      scan[i] = run;  // exclusive prefix
      run += x;
    }
    scan[T] = run;
  }
  __syncthreads();
  const float total = scan[T];
  __shared__ int chosen;
  if (t == 0) chosen = V - 1;
  __syncthreads();
  if (total > 0.f) {
    const float target = u * total;
    const float start = scan[t];
    // The one non-empty chunk with start <= target < its end (scan[T] = total).
    if (hi > lo && start <= target && target < scan[t + 1]) {
      float run = start;
      int pick = hi - 1;
      for (int v = lo; v < hi; ++v) {
        run += draw_weight(a, b, acc, v, diff);
        if (run > target) {
          pick = v;
          break;
        }
      }
      atomicMin(&chosen, pick);
    }
  }
  __syncthreads();
  int tok = chosen;
  if (!(total > 0.f)) tok = -1;  // caller falls back
  __syncthreads();
  return tok;
}

MF_DEVINL void copy16(const void* src, void* dst, int bytes) {
  if (bytes == 16) {
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
  } else {
    const char* s = static_cast<const char*>(src);
    char* d = static_cast<char*>(dst);
    for (int j = 0; j < bytes; ++j) d[j] = s[j];
  }
}

__global__ void __launch_bounds__(AC_THREADS) accept_commit_kernel(AcceptParams P, int commit_ctas,
                                                                   int vec_bytes) {
  const mf_accept_args& a = P.a;
  const int b = blockIdx.x;
  const int part = blockIdx.y;
  const int acc = accepted_count(a, b);
  if (part == 0) {
    __shared__ float scan[AC_THREADS + 1];
    int next;
    if (a.target_probs == nullptr) {
      next = a.target_tokens[(int64_t)b * a.target_tokens_stride + acc];
    } else {
      const float u = a.resample_uniform[b];
      const bool rejected = acc < a.num_drafts;
      next = draw_token(a, b, acc, rejected, u, scan);
      if (next < 0 && rejected) next = draw_token(a, b, acc, false, u, scan);
      if (next < 0) next = min(a.vocab - 1, (int)(u * a.vocab));  // all-zero: uniform
    }
    if (threadIdx.x == 0) {
      a.num_accepted[b] = acc;
      if (a.next_token) a.next_token[b] = next;
    }
    return;
  }
  if (a.win_k == nullptr) return;  // decision only
  // Commit rows 0..acc of sequence b, layers part-1, part-1+C, ...
  const int n = acc + 1;
  const int c = a.ctx_lens[b];
  const int bs = a.block_size;
  if (c < 0) {
    if (part == 1 && threadIdx.x == 0) set_err(a.err_flag, MF_ERR_LENGTH);
    return;
  }
  const int64_t first_page = (int64_t)c / bs, last_page = ((int64_t)c + n - 1) / bs;
  if (last_page >= a.table_stride) {
    if (part == 1 && threadIdx.x == 0) set_err(a.err_flag, MF_ERR_TABLE);
    return;
  }
  for (int64_t p = first_page; p <= last_page; ++p) {
    const int id = a.block_tables[(int64_t)b * a.table_stride + p];
    if (id < 0 || id >= a.num_blocks) {
      if (part == 1 && threadIdx.x == 0) set_err(a.err_flag, MF_ERR_BLOCK_ID);
      return;
    }
  }
  const int elt = a.elem_bytes;
  const int vecs = a.head_dim * elt / vec_bytes;
  const int64_t per_layer = (int64_t)n * a.num_kv_heads * vecs;
  for (int layer = part - 1; layer < a.num_layers; layer += commit_ctas) {
    for (int64_t i = threadIdx.x; i < per_layer; i += blockDim.x) {
      const int v = (int)(i % vecs);
      const int64_t jh = i / vecs;
      const int h = (int)(jh % a.num_kv_heads);
      const int j = (int)(jh / a.num_kv_heads);
      const int64_t pos = (int64_t)c + j;
      const int blk = a.block_tables[(int64_t)b * a.table_stride + pos / bs];
      const int64_t row = (int64_t)b * P.window + j;
      const int64_t src = ((int64_t)layer * a.win_stride_layer + row * a.win_stride_row +
                           (int64_t)h * a.win_stride_head) * elt + (int64_t)v * vec_bytes;
      const int64_t dst = ((int64_t)layer * a.pool_stride_layer + (int64_t)blk * a.pool_stride_block +
                           (pos % bs) * a.pool_stride_slot + (int64_t)h * a.pool_stride_head) * elt +
                          (int64_t)v * vec_bytes;
      copy16(static_cast<const char*>(a.win_k) + src, static_cast<char*>(a.key_pool) + dst,
             vec_bytes);
      copy16(static_cast<const char*>(a.win_v) + src, static_cast<char*>(a.value_pool) + dst,
             vec_bytes);
    }
  }
}

}  // namespace
}  // namespace mf

using namespace mf;

extern "C" int mf_accept_commit(const mf_accept_args* args, mf_stream_t stream) {
  if (!args) return fail(MF_EINVAL, "accept_commit: null args");
  const mf_accept_args& a = *args;
  if (a.struct_size != sizeof(mf_accept_args))
    return fail(MF_EINVAL, "accept_commit: struct_size does not match this library");
  if (a.num_seqs < 0 || a.num_drafts < 0 || a.num_drafts > AC_MAX_DRAFTS)
    return fail(MF_EINVAL, "accept_commit: num_drafts outside [0, 64] or negative num_seqs");
  if (a.num_seqs == 0) return MF_OK;
  if (!a.draft_tokens || !a.num_accepted)
    return fail(MF_EINVAL, "accept_commit: null draft_tokens or num_accepted");
  if (a.target_probs == nullptr) {
    if (!a.target_tokens) return fail(MF_EINVAL, "accept_commit: greedy mode needs target_tokens");
  } else {
    if (!a.draft_probs || !a.uniforms || !a.resample_uniform || a.vocab <= 0)
      return fail(MF_EINVAL,
                  "accept_commit: sampling mode needs draft_probs, uniforms, resample_uniform "
                  "and vocab");
  }
  int commit_ctas = 0, vec_bytes = 1;
  if (a.win_k != nullptr) {
    if (!a.win_v || !a.key_pool || !a.value_pool || !a.block_tables || !a.ctx_lens)
      return fail(MF_EINVAL, "accept_commit: commit needs window, pool, tables and lengths");
    if (a.num_layers <= 0 || a.num_kv_heads <= 0 || a.head_dim <= 0 || a.block_size <= 0 ||
        a.num_blocks <= 0 || a.table_stride < 0 ||
        !(a.elem_bytes == 2 || a.elem_bytes == 4))
      return fail(MF_EINVAL, "accept_commit: bad pool geometry");
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    auto al16 = [&](int64_t s) { return (s * a.elem_bytes) % 16 == 0; };
    vec_bytes = (a.head_dim * a.elem_bytes) % 16 == 0 && al(a.win_k) && al(a.win_v) &&
                        al(a.key_pool) && al(a.value_pool) && al16(a.win_stride_layer) &&
                        al16(a.win_stride_row) && al16(a.win_stride_head) &&
                        al16(a.pool_stride_layer) && al16(a.pool_stride_block) &&
                        al16(a.pool_stride_slot) && al16(a.pool_stride_head)
                    ? 16
                    : a.elem_bytes;
    commit_ctas = a.num_layers < 8 ? a.num_layers : 8;
  }
  if (a.num_seqs > 65535 * 16) return fail(MF_EINVAL, "accept_commit: too many sequences");
  AcceptParams P{a, a.num_drafts + 1};
  dim3 grid((unsigned)a.num_seqs, (unsigned)(1 + commit_ctas));
  accept_commit_kernel<<<grid, AC_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      P, commit_ctas, vec_bytes);
  return check_launch("accept_commit");
}
