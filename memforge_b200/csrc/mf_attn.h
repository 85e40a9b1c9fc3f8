// Parameters shared by the paged-attention kernels (device side view of
// mf_attention_args plus derived values).
#pragma once

#include "mf_internal.h"

namespace mf {

struct AttnParams {
  const void* q;
  int64_t q_sr, q_sh;
  void* out;
  int64_t o_sr, o_sh;
  const void* kp;
  const void* vp;
  int64_t sb, ss, sh;
  int32_t num_blocks, block_size;
  const int32_t* tables;
  int32_t table_stride;
  const int32_t* cu_q;
  int32_t q_per_seq;
  const int32_t* kv_lens;
  const int32_t* row_map;
  const void* wk;
  const void* wv;
  int64_t w_sr, w_sh;
  int32_t num_seqs, total_q, max_q_len;
  int32_t hq, hkv, d;
  float scale;
  int32_t causal;
  int32_t* err;
  // Head-sharded output: when n_peers > 0, output rows go to every out_peers[i]
  // at head out_head_offset + local head (and not to `out`).
  int32_t n_peers;
  int32_t out_head_offset;
  void* out_peers[MF_MAX_OUT_PEERS];
};

// Output targets of a call (the peers' buffers, or `out`) and the address of
// element `off` of target t.
MF_DEVINL int out_targets(const AttnParams& p) { return p.n_peers > 0 ? p.n_peers : 1; }
template <typename T>
MF_DEVINL T* out_at(const AttnParams& p, int t, int64_t off) {
  return p.n_peers > 0
             ? static_cast<T*>(p.out_peers[t]) + off + (int64_t)p.out_head_offset * p.o_sh
             : static_cast<T*>(p.out) + off;
}

// Query extent of sequence s.
MF_DEVINL void seq_rows(const AttnParams& p, int s, int& q_start, int& q_len) {
  if (p.cu_q) {
    q_start = p.cu_q[s];
    q_len = p.cu_q[s + 1] - q_start;
  } else {
    q_start = s * p.q_per_seq;
    q_len = p.q_per_seq;
  }
}

MF_DEVINL int map_row(const AttnParams& p, int r) { return p.row_map ? p.row_map[r] : r; }

// Bytes at the front of a decode workspace that hold arrival counters (they
// must be zero when a launch starts; every launch leaves the ones it used zero).
constexpr size_t kSemRegionBytes = size_t(1) << 20;

// Host launchers.
int launch_attn_generic(const AttnParams& p, mf_dtype dtype, cudaStream_t stream);

struct TcPlan {
  bool ok = false;
  const char* why = "";
  bool SW = false;  // swapped-operand decode consumer (<= 8 rows per kv head)
  bool skip_long = false;
  int rows_cap = 0;
  int MT = 1, HG = 1, NHG = 1, PPS = 1, NS = 2, ctas = 0;
  size_t smem = 0;
  size_t part_floats = 0;   // floats per partial slot
  size_t ws_bytes = 0;
};

TcPlan plan_attn_tc(const AttnParams& p, mf_dtype dtype, int sm_count, bool window,
                    bool skip_long = false);

// tcgen05 prefill kernel: nullptr when it serves these arguments, else why not.
const char* prefill_tc_unsupported(const AttnParams& p, mf_dtype dtype);
// Serves every sequence whose query run has more than rows_cap rows per kv head.
int launch_attn_prefill_tc(const AttnParams& p, mf_dtype dtype, int rows_cap,
                           cudaStream_t stream);

// How one mf_paged_attention call is split across kernels.
struct Dispatch {
  // DECODE: decode kernel alone.  MIXED: tcgen05 kernel for runs of more than
  // rows_cap rows per kv head, decode kernel for the rest.  PREFILL: tcgen05
  // kernel alone (every run is long).  GENERIC: CUDA-core kernel.
  enum Mode { DECODE, MIXED, PREFILL, GENERIC } mode = GENERIC;
  TcPlan decode;       // DECODE / MIXED: the decode kernel's plan
  AttnParams short_p;  // MIXED: the decode kernel's view (short runs only)
  int rows_cap = 0;    // MIXED / PREFILL: longest run the decode kernel keeps
};
Dispatch plan_dispatch(const AttnParams& p, mf_dtype dtype, int sm_count);
int launch_attn_tc(const AttnParams& p, mf_dtype dtype, const TcPlan& plan, void* ws,
                   cudaStream_t stream);

}  // namespace mf
