// Paged decode / speculative-verify attention for bf16 / fp16 pools on sm_100a.
//
// HBM-bound design (4, 5):
//  * Work = the concatenated list of KV pages (16-token blocks) of all
//    sequences, for each group of HG kv heads.  It is cut into equal
//    contiguous ranges, one per "virtual CTA" (stream-K), so every SM streams
//    the same number of bytes whatever the context lengths are (small batches
//    use fewer ranges, MIN_PAGES pages at least, to bound the merge fan-in).  A range that
//    covers a whole sequence writes the output directly; a sequence split
//    across ranges leaves fp32 partials (running max, sum, unnormalised
//    accumulator) in the workspace and the last range to finish merges them
//    with the log-sum-exp identity (a per-sequence arrival counter; no waiting).
//  * One warp (the producer) walks the block tables and issues one 4-D TMA
//    tile load per page per K/V: box (64 dims, 16 tokens, D/64, HG kv heads) of
//    the pool viewed as [slots][kv_heads][D], 128-byte swizzled, into a ring
//    of shared-memory stages guarded by mbarriers.  The box puts the 16 tokens
//    of one (head, 64-dim half) in consecutive 128-byte rows, so the swizzle
//    spreads every 8-token ldmatrix phase over all banks.  No multicast.
//  * Eight consumer warps each own one (kv head, 16-row m-tile, half of D):
//    rows are (query position, query head) pairs of the GQA group, so a page is
//    read from HBM once for all query heads sharing its kv head.  Both halves
//    compute the full Q K^T (mma.sync m16n8k16, fp32 accumulate); each keeps
//    the P V accumulator for its half of head_dim, which keeps the streaming
//    loop within the register budget of a 288-thread CTA.  Online softmax in
//    the log2 domain with quad shuffles.
//  * When fewer than 8 (head, m-tile, half) units exist, the CTA runs
//    PPS = 8/units independent virtual CTAs side by side, one page each per stage.
//  * Every mbarrier wait is bounded; on expiry the CTA sets MF_ERR_TIMEOUT,
//    drains its own TMA loads and returns.
//
// Workspace: [0, SEM_REGION) arrival counters, always all-zero between launches
// (each launch resets the ones it used); partial slots after it.

#include "mf_attn.h"

namespace mf {

namespace tc {

constexpr int CONSUMER_WARPS = 8;
constexpr int THREADS = (CONSUMER_WARPS + 1) * 32;
constexpr int PAGE = 16;
constexpr int DS = 2;  // consumer warps per (head, m-tile): halves of head_dim for P V
constexpr uint64_t WAIT_LIMIT = 2000000000ull;  // 2 s of wall time per wait
constexpr int MAX_SEQS = 4096;
constexpr int MAX_WINDOW_SEQS = 1024;
constexpr size_t SEM_REGION = kSemRegionBytes;
constexpr int MIN_PAGES = 4;  // fewest pages a virtual CTA is given

struct Params {
  AttnParams a;
  int G, HG, NHG, MT, PPS, NS;
  int rows_cap;   // longest query run (rows = q_len * G) this launch serves
  int skip_long;  // 1: longer runs belong to another kernel of the same call
  int window;
  float scale_log2;
  float* part;      // partial slots
  int32_t* sems;    // arrival counters
  int part_floats;  // floats per partial slot
};

struct Smem {
  uint32_t page_bytes, stage_bytes, bar_off, prefix_off, qstart_off, flag_off, total;
};

__host__ __device__ inline Smem smem_layout(int D, int HG, int PPS, int NS, int B, int window) {
  Smem s;
  s.page_bytes = (uint32_t)(HG * PAGE * D * 2);
  s.stage_bytes = 2u * PPS * s.page_bytes;
  s.bar_off = NS * s.stage_bytes;
  s.prefix_off = s.bar_off + 2 * NS * 8;
  s.qstart_off = s.prefix_off + (uint32_t)(B + 1) * 4;
  s.flag_off = s.qstart_off + (window ? (uint32_t)B * 4 : 0u);
  s.total = s.flag_off + 16;
  return s;
}

// Swizzled shared-memory address of 16-byte chunk `chunk` (0..D/8-1) of token
// `tok` of local kv head `hl` in a page tile written by the 128B-swizzle TMA
// box (64, 16, D/64, HG): 128-byte row R = (hl * D/64 + chunk/8) * 16 + tok.
template <int D>
MF_DEVINL uint32_t tile_addr(uint32_t base, int tok, int hl, int chunk) {
  const int half = chunk >> 3, cc = chunk & 7;
  const int R = ((hl * (D / 64) + half) << 4) + tok;
  return base + (uint32_t)(R * 128) + (uint32_t)((cc ^ (R & 7)) << 4);
}

// Page geometry of sequence i (identical in the prologue and the consumers).
struct SeqGeo {
  int q_start, q_len, kv_len, pool_len, pool_pages, pages;
};

MF_DEVINL SeqGeo seq_geo(const Params& P, int i) {
  SeqGeo g;
  seq_rows(P.a, i, g.q_start, g.q_len);
  g.kv_len = P.a.kv_lens[i];
  const bool bad = g.q_len < 0 || g.kv_len < g.q_len || (g.q_len > 0 && g.kv_len <= 0) ||
                   g.q_len * P.G > P.rows_cap || (P.window && g.q_len > PAGE);
  if (bad || g.q_len == 0) {
    g.pool_len = 0;
    g.pool_pages = 0;
    g.pages = 0;
    return g;
  }
  g.pool_len = P.window ? g.kv_len - g.q_len : g.kv_len;
  g.pool_pages = (g.pool_len + PAGE - 1) / PAGE;
  if (g.pool_pages > P.a.table_stride) g.pool_pages = P.a.table_stride;  // flagged in prologue
  g.pages = g.pool_pages + (P.window ? 1 : 0);
  return g;
}

// The virtual page list [0, total) cut over the virtual CTAs: range vc is
// [bound(vc), bound(vc+1)).  The first `rem` ranges hold base+1 pages, the
// next nv-rem hold base (>= 1), and virtual CTAs from nv on hold none, so
// every range below nv is non-empty and a page's owner is closed-form.
struct Split {
  int64_t total, nv, base, rem;
  MF_DEVINL int64_t bound(int64_t vc) const {
    return vc >= nv ? total : vc * base + (vc < rem ? vc : rem);
  }
  MF_DEVINL int owner(int64_t page) const {
    const int64_t big = (base + 1) * rem;
    return (int)(page < big ? page / (base + 1) : rem + (page - big) / base);
  }
  MF_DEVINL int len(int64_t vc) const { return (int)(bound(vc + 1) - bound(vc)); }
};

MF_DEVINL Split make_split(int64_t total, int64_t nv_max) {
  Split s;
  s.total = total;
  s.nv = (total + MIN_PAGES - 1) / MIN_PAGES;
  if (s.nv > nv_max) s.nv = nv_max;
  if (s.nv < 1) s.nv = 1;
  s.base = total / s.nv;
  s.rem = total - s.base * s.nv;
  return s;
}

// Sequence index i with prefix[i] <= off < prefix[i+1] (prefix nondecreasing).
MF_DEVINL int find_seq(const int* prefix, int B, int off) {
  int lo = 0, hi = B;  // invariant: prefix[lo] <= off < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= off) lo = mid; else hi = mid;
  }
  return lo;
}

// Position in the virtual page list, advanced one page at a time from shared
// memory only (no global loads).
struct Cursor {
  int hg, i, k, pages;
};

MF_DEVINL Cursor cursor_at(const int* prefix, int B, int64_t T1, int64_t v) {
  Cursor c;
  c.hg = (int)(v / T1);
  const int off = (int)(v - (int64_t)c.hg * T1);
  c.i = find_seq(prefix, B, off);
  c.k = off - prefix[c.i];
  c.pages = prefix[c.i + 1] - prefix[c.i];
  return c;
}

// Only called while the next page is inside the range, so a non-empty
// sequence always follows.
MF_DEVINL void cursor_next(Cursor& c, const int* prefix, int B) {
  if (++c.k < c.pages) return;
  c.k = 0;
  do {
    if (++c.i == B) {
      c.i = 0;
      ++c.hg;
    }
    c.pages = prefix[c.i + 1] - prefix[c.i];
  } while (c.pages == 0);
}


// State every consumer warp needs from the kernel prologue.
struct Ctx {
  const Params& P;
  Smem L;
  uint32_t base;
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort_flag;
  const int* prefix;
  int B;
  int64_t T1;
  Split S;
  int warp, lane, max_len;
};

// Partial slot layout, per virtual CTA and slot: acc[unit][RU rows][DU cols],
// then m[unit][RU], then l[unit][RU] (unit_rows = units * RU).
template <int RU, int DU>
struct PartLayout {
  const Params& P;
  int unit_rows;
  MF_DEVINL float* slot(int64_t vcx, int sl) const {
    return P.part + (vcx * 2 + sl) * (int64_t)P.part_floats;
  }
  MF_DEVINL float* acc(float* s, int unit, int rr) const {
    return s + (int64_t)(unit * RU + rr) * DU;
  }
  MF_DEVINL float* m(float* s, int unit) const { return s + (int64_t)unit_rows * DU + unit * RU; }
  MF_DEVINL float* l(float* s, int unit) const { return m(s, unit) + unit_rows; }
};

// Merge every covering range's partial for one (sequence, head, unit) with the
// log-sum-exp identity and write the output rows [row0, row0+RU) (columns
// [col0, col0+DU) of the head).  Run by the warp whose arrival completed the
// set.  Latency-bound: each round trip loads RB ranges at once, their (m, l)
// (lane l: range l / RU, row l % RU) together with their accumulator rows as
// float4 (lane l: columns 4 (l % (DU/4)) .. +3 of rows i*RPL + l / (DU/4)),
// and skips rows past the unit's query rows.  HALF: the unit has at most RU/2
// query rows, so a round trip carries twice the ranges.  The arrival that
// chose this warp (arrive_last) was an acquire, so no fence is needed here.
template <typename T, int RU, int DU, bool HALF>
MF_DEVINL void merge_rows(const Ctx& C, const PartLayout<RU, DU>& PL, int hg, int si, int hl,
                          int unit, int row0, int col0) {
  constexpr int VPR = DU / 4;                 // float4 per accumulator row
  constexpr int RPL = 32 / VPR;               // rows one warp-wide float4 load covers
  constexpr int NR = (HALF ? RU / 2 : RU) / RPL;  // float4 per lane per range
  constexpr int RB = RU == 8 ? (HALF ? 4 : 2) : (HALF ? 2 : 1);  // ranges per round trip
  static_assert(RB * RU <= 32 && NR >= 1, "merge tiling");
  const Params& P = C.P;
  const int lane = C.lane;
  // Geometry without global loads (the prefix sums are in shared memory).
  int q_start, q_len;
  seq_rows(P.a, si, q_start, q_len);
  const int pages = C.prefix[si + 1] - C.prefix[si];
  const int head = hg * P.HG + hl;
  const int64_t vstart = (int64_t)hg * C.T1 + C.prefix[si];
  const int vc0 = C.S.owner(vstart);
  const int vc1 = C.S.owner(vstart + pages - 1);
  const int rows = min(RU, q_len * P.G - row0);  // rows of this unit that exist
  const int lr = lane / VPR, lc = (lane % VPR) * 4;
  float Mrun[RU], Lrun = 0.f;  // Lrun: row lane % RU
  float4 acc[NR];
#pragma unroll
  for (int r = 0; r < RU; ++r) Mrun[r] = -INFINITY;
#pragma unroll
  for (int i = 0; i < NR; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c = vc0; c <= vc1; c += RB) {
    const int n = min(RB, vc1 - c + 1);
    float* slots[RB];
#pragma unroll
    for (int j = 0; j < RB; ++j) {
      const int cj = j < n ? c + j : c;
      slots[j] = PL.slot(cj, C.S.bound(cj) >= vstart ? 0 : 1);
    }
    // One round trip: (m, l) and accumulator rows of all n ranges.
    const int my_r = lane % RU, my_j = lane / RU;
    float mk = -INFINITY, lk = 0.f;
#pragma unroll
    for (int j = 0; j < RB; ++j)
      if (j == my_j && j < n) {
        mk = __ldcg(PL.m(slots[j], unit) + my_r);
        lk = __ldcg(PL.l(slots[j], unit) + my_r);
      }
    float4 v[RB][NR];
#pragma unroll
    for (int j = 0; j < RB; ++j)
#pragma unroll
      for (int i = 0; i < NR; ++i)
        v[j][i] = (j < n && i * RPL < rows)
                      ? __ldcg(reinterpret_cast<const float4*>(PL.acc(slots[j], unit, i * RPL + lr) + lc))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    float mx = mk;
#pragma unroll
    for (int o = RU; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // New running max of every row, and the factor for what was accumulated so far.
    float scale_old[RU], mu_mine = 0.f, so_mine = 0.f;
#pragma unroll
    for (int r = 0; r < RU; ++r) {
      const float mn = fmaxf(Mrun[r], __shfl_sync(0xffffffffu, mx, r));
      const float mu = mn == -INFINITY ? 0.f : mn;
      scale_old[r] = Mrun[r] == -INFINITY ? 0.f : fast_exp2(Mrun[r] - mu);
      Mrun[r] = mn;
      if (r == my_r) {
        mu_mine = mu;
        so_mine = scale_old[r];
      }
    }
    const float w = (mk == -INFINITY) ? 0.f : fast_exp2(mk - mu_mine);
    float lw = w * lk;
#pragma unroll
    for (int o = RU; o < 32; o <<= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
    Lrun = Lrun * so_mine + lw;  // lanes with equal lane % RU agree
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      float so = scale_old[i * RPL];
#pragma unroll
      for (int t = 1; t < RPL; ++t)
        if (lr == t) so = scale_old[i * RPL + t];
      float4& a = acc[i];
      a.x *= so;
      a.y *= so;
      a.z *= so;
      a.w *= so;
#pragma unroll
      for (int j = 0; j < RB; ++j) {
        const float wj = __shfl_sync(0xffffffffu, w, j * RU + i * RPL + lr);
        if (j < n) {
          a.x += wj * v[j][i].x;
          a.y += wj * v[j][i].y;
          a.z += wj * v[j][i].z;
          a.w += wj * v[j][i].w;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    const int r = i * RPL + lr;
    const float Lr = __shfl_sync(0xffffffffu, Lrun, r);
    if (r >= rows) continue;
    const int qi = (row0 + r) / P.G, gg = (row0 + r) % P.G;
    const float inv = Lr > 0.f ? 1.f / Lr : 0.f;
    const int64_t off = (int64_t)map_row(P.a, q_start + qi) * P.a.o_sr +
                        (int64_t)(head * P.G + gg) * P.a.o_sh + col0 + lc;
    const T v0 = from_f32<T>(acc[i].x * inv), v1 = from_f32<T>(acc[i].y * inv);
    const T v2 = from_f32<T>(acc[i].z * inv), v3 = from_f32<T>(acc[i].w * inv);
    for (int t = 0; t < out_targets(P.a); ++t) {
      T* orow = out_at<T>(P.a, t, off);
      orow[0] = v0;
      orow[1] = v1;
      orow[2] = v2;
      orow[3] = v3;
    }
  }
}

// Out of line: the streaming loop keeps its registers; picks the HALF form
// when the unit has at most RU/2 query rows.
template <typename T, int RU, int DU>
__device__ __noinline__ void merge_unit(const Ctx& C, const PartLayout<RU, DU>& PL, int hg,
                                        int si, int hl, int unit, int row0, int col0) {
  int q_start, q_len;
  seq_rows(C.P.a, si, q_start, q_len);
  if (q_len * C.P.G - row0 <= RU / 2)
    merge_rows<T, RU, DU, true>(C, PL, hg, si, hl, unit, row0, col0);
  else
    merge_rows<T, RU, DU, false>(C, PL, hg, si, hl, unit, row0, col0);
}

// Arrival bookkeeping after a partial was written: true when this warp's
// arrival completed the set of ranges covering the sequence.  The warp barrier
// orders every lane's partial stores before lane 0's acquire-release add, which
// publishes them (release) and, for the last arrival, makes the other ranges'
// partials visible to the merge that follows (acquire, then the warp barrier).
MF_DEVINL bool arrive_last(const Ctx& C, int32_t* sem, int hg, int si, int pages) {
  __syncwarp();
  const int64_t vstart = (int64_t)hg * C.T1 + C.prefix[si];
  // Ranges covering the sequence: [vc0, vc1], all non-empty.
  const int covering = C.S.owner(vstart + pages - 1) - C.S.owner(vstart) + 1;
  int old = 0;
  if (C.lane == 0) old = atom_add_acq_rel_gpu(sem, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  __syncwarp();
  return old == covering - 1;
}

// Wait for a stage; false (after flagging) when the wait gave up or another
// warp aborted.
MF_DEVINL bool wait_full(const Ctx& C, int stage, uint32_t phase) {
  if (!mbar_wait_bounded(&C.full[stage], phase, WAIT_LIMIT)) {
    if (C.lane == 0) set_err(C.P.a.err, MF_ERR_TIMEOUT);
    *C.abort_flag = 1;
  }
  return !__any_sync(0xffffffffu, *C.abort_flag != 0);
}

MF_DEVINL void release(const Ctx& C, int stage) {
  __syncwarp();
  if (C.lane == 0) mbar_arrive(&C.empty[stage]);
}

MF_DEVINL uint32_t movm_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// -------------------------------------------------------------------------
// Consumer for up to 8 query rows per kv head (decode): one warp per kv head.
// S^T = K Q^T (M = 16 tokens, N = 8 rows, K = head_dim), P^T turned into the B
// operand with movmatrix, O^T = V^T P^T (M = head_dim in 16-row tiles).
// -------------------------------------------------------------------------
template <typename T, int D>
MF_DEVINL void consume_swapped(const Ctx& C) {
  const Params& P = C.P;
  using M = Mma<T>;
  constexpr int RU = 8;
  const int lane = C.lane;
  const int units = P.HG;
  const int hl = C.warp % units;          // local kv head
  const int ps = C.warp / units;          // virtual CTA within this CTA
  const int g4 = lane >> 2, c4 = lane & 3;
  const int64_t vc = (int64_t)blockIdx.x * P.PPS + ps;
  const int64_t lo = C.S.bound(vc);
  const int len = C.S.len(vc);
  const T* qbase = static_cast<const T*>(P.a.q);
  const float sl2 = P.scale_log2;
  const int NS = P.NS, G = P.G, causal = P.a.causal, window = P.window;
  const uint32_t stage_bytes = C.L.stage_bytes, page_bytes = C.L.page_bytes;
  const uint32_t v_off = P.PPS * page_bytes;
  const PartLayout<RU, D> PL{P, units * RU};

  int hg = 0, si = 0, k = 0, k0 = 0;
  SeqGeo geo{};
  bool first_piece = true;
  int n_merge = 0, mhg0 = 0, msi0 = 0, mhg1 = 0, msi1 = 0;
  uint32_t qb[D / 16][2];   // Q^T as the B operand: (k = dims, n = row g4)
  float o[D / 16][4];       // O^T: (dims g4 / g4+8 of each 16-dim tile, rows 2c4, 2c4+1)
  float mrow[2], lrow[2];   // rows 2c4, 2c4+1

  int stage = 0;
  uint32_t phase = 0;
  for (int it = 0; it < C.max_len; ++it, stage = (stage + 1 == NS) ? 0 : stage + 1,
           phase ^= (stage == 0) ? 1u : 0u) {
    if (it >= len) {
      release(C, stage);
      continue;
    }
    if (it == 0 || k == geo.pages) {
      const Cursor c = cursor_at(C.prefix, C.B, C.T1, lo + it);
      hg = c.hg;
      si = c.i;
      k = c.k;
      k0 = k;
      geo = seq_geo(P, si);
      const int head = hg * P.HG + hl;
      const int qi = g4 / P.G, gg = g4 % P.G;
      const bool valid = qi < geo.q_len;
      const T* qrow = qbase + (valid ? (int64_t)map_row(P.a, geo.q_start + qi) * P.a.q_sr +
                                           (int64_t)(head * P.G + gg) * P.a.q_sh
                                     : 0);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        qb[ks][0] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * c4) : 0u;
        qb[ks][1] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * c4) : 0u;
      }
#pragma unroll
      for (int n = 0; n < D / 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      mrow[0] = mrow[1] = -INFINITY;
      lrow[0] = lrow[1] = 0.f;
    }
    if (!wait_full(C, stage, phase)) return;

    const uint32_t sK = C.base + stage * stage_bytes + ps * page_bytes;
    const uint32_t sV = sK + v_off;
    const bool is_win = window && k == geo.pool_pages;
    const int kbase = is_win ? geo.pool_len : k * PAGE;
    const int valid = is_win ? geo.q_len : min(PAGE, geo.pool_len - k * PAGE);
    const int win_start = geo.kv_len - geo.q_len;
    const bool need_mask = valid < PAGE || (causal && kbase + PAGE - 1 > win_start);

    // S^T: two accumulators (even / odd k-steps) halve the dependent chain.
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a[4];
      const int tok = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int chunk = ks * 2 + (lane >> 4);
      ldsm_x4(a[0], a[1], a[2], a[3], tile_addr<D>(sK, tok, hl, chunk));
      M::run((ks & 1) ? s1 : s0, a, qb[ks][0], qb[ks][1]);
    }
    float sc[4];  // (tok g4, row 2c4), (tok g4, row 2c4+1), (tok g4+8, row 2c4), (tok g4+8, row 2c4+1)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float v = (s0[e] + s1[e]) * sl2;
      if (need_mask) {
        const int tok = g4 + 8 * (e >> 1);
        const int r = 2 * c4 + (e & 1);
        const int lim = causal ? win_start + r / G : geo.kv_len - 1;
        if (tok >= valid || kbase + tok > lim) v = -INFINITY;
      }
      sc[e] = v;
    }
    uint32_t pb[2];  // P^T for tokens 0-7 / 8-15 as B fragments
    float alpha[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float mx = fmaxf(sc[j], sc[2 + j]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mnew = fmaxf(mrow[j], mx);
      const float mu = (mnew == -INFINITY) ? 0.f : mnew;
      alpha[j] = fast_exp2(mrow[j] - mu);
      mrow[j] = mnew;
      sc[j] = fast_exp2(sc[j] - mu);
      sc[2 + j] = fast_exp2(sc[2 + j] - mu);
      lrow[j] = lrow[j] * alpha[j] + (sc[j] + sc[2 + j]);
    }
    pb[0] = movm_trans(M::pack(sc[0], sc[1]));  // -> (row g4, tokens 2c4..2c4+1)
    pb[1] = movm_trans(M::pack(sc[2], sc[3]));  // -> (row g4, tokens 8+2c4..)
    // The running max rarely moves after the first pages: rescale only when
    // some row's max changed (alpha != 1) anywhere in the warp.
    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
      for (int n = 0; n < D / 16; ++n) {
        o[n][0] *= alpha[0];
        o[n][1] *= alpha[1];
        o[n][2] *= alpha[0];
        o[n][3] *= alpha[1];
      }
    }
    // O^T += V^T P^T, one 16-dim tile per mma
#pragma unroll
    for (int n = 0; n < D / 16; ++n) {
      uint32_t a[4];
      const int tok = (lane & 7) + ((lane >> 4) << 3);
      const int chunk = n * 2 + ((lane >> 3) & 1);
      ldsm_x4_trans(a[0], a[1], a[2], a[3], tile_addr<D>(sV, tok, hl, chunk));
      if (valid < PAGE) {
        // Unwritten slots may hold anything (NaN included): zero them.
        const int t_lo = 2 * c4, t_hi = 8 + 2 * c4;
        const uint32_t mlo = (t_lo < valid ? 0xffffu : 0u) | (t_lo + 1 < valid ? 0xffff0000u : 0u);
        const uint32_t mhi = (t_hi < valid ? 0xffffu : 0u) | (t_hi + 1 < valid ? 0xffff0000u : 0u);
        a[0] &= mlo;
        a[1] &= mlo;
        a[2] &= mhi;
        a[3] &= mhi;
      }
      M::run(o[n], a, pb[0], pb[1]);
    }
    ++k;
    release(C, stage);
    if (k != geo.pages && it != len - 1) continue;

    // ------------------------------------------------------ finish a piece
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      lrow[j] += __shfl_xor_sync(0xffffffffu, lrow[j], 4);
      lrow[j] += __shfl_xor_sync(0xffffffffu, lrow[j], 8);
      lrow[j] += __shfl_xor_sync(0xffffffffu, lrow[j], 16);
    }
    const int head = hg * P.HG + hl;
    if (k0 == 0 && k == geo.pages) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = 2 * c4 + j;
        const int qi = r / P.G, gg = r % P.G;
        if (qi >= geo.q_len) continue;
        const float inv = lrow[j] > 0.f ? 1.f / lrow[j] : 0.f;
        const int64_t off = (int64_t)map_row(P.a, geo.q_start + qi) * P.a.o_sr +
                            (int64_t)(head * P.G + gg) * P.a.o_sh;
        for (int t = 0; t < out_targets(P.a); ++t) {
          T* orow = out_at<T>(P.a, t, off);
#pragma unroll
          for (int n = 0; n < D / 16; ++n) {
            orow[n * 16 + g4] = from_f32<T>(o[n][j] * inv);
            orow[n * 16 + 8 + g4] = from_f32<T>(o[n][2 + j] * inv);
          }
        }
      }
      first_piece = false;
      continue;
    }
    float* sl = PL.slot(vc, first_piece ? 0 : 1);
    first_piece = false;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (2 * c4 + j >= geo.q_len * G) continue;  // no such query row
      float* pa = PL.acc(sl, hl, 2 * c4 + j);
#pragma unroll
      for (int n = 0; n < D / 16; ++n) {
        pa[n * 16 + g4] = o[n][j];
        pa[n * 16 + 8 + g4] = o[n][2 + j];
      }
      if (g4 == 0) {
        PL.m(sl, hl)[2 * c4 + j] = mrow[j];
        PL.l(sl, hl)[2 * c4 + j] = lrow[j];
      }
    }
    int32_t* sem = P.sems + (((int64_t)hg * C.B + si) * P.HG + hl);
    if (!arrive_last(C, sem, hg, si, geo.pages)) continue;
    if (n_merge == 0) {
      mhg0 = hg;
      msi0 = si;
    } else {
      mhg1 = hg;
      msi1 = si;
    }
    ++n_merge;
  }
  for (int m = 0; m < n_merge; ++m) {
    const int mhg = m == 0 ? mhg0 : mhg1;
    const int msi = m == 0 ? msi0 : msi1;
    merge_unit<T, RU, D>(C, PL, mhg, msi, hl, hl, 0, 0);
    if (lane == 0) P.sems[((int64_t)mhg * C.B + msi) * P.HG + hl] = 0;
  }
}

// -------------------------------------------------------------------------
// Consumer for 9..64 query rows per kv head (speculative verify): warps own
// (kv head, 16-row m-tile, half of head_dim); S = Q K^T in full, O[:, half] +=
// P V.
// -------------------------------------------------------------------------
template <typename T, int D>
MF_DEVINL void consume_split(const Ctx& C) {
  const Params& P = C.P;
  using M = Mma<T>;
  constexpr int DH = D / 2;
  constexpr int RU = 16;
  const int lane = C.lane;
  const int units = P.HG * P.MT * DS;
  const int u = C.warp % units;
  const int ps = C.warp / units;
  const int dh = u % DS;
  const int pair = u / DS;
  const int mt = pair % P.MT;
  const int hl = pair / P.MT;
  const int unit = u;  // == (hl * MT + mt) * DS + dh
  const int g4 = lane >> 2, c4 = lane & 3;
  const int64_t vc = (int64_t)blockIdx.x * P.PPS + ps;
  const int64_t lo = C.S.bound(vc);
  const int len = C.S.len(vc);
  const T* qbase = static_cast<const T*>(P.a.q);
  const float sl2 = P.scale_log2;
  const PartLayout<RU, DH> PL{P, units * RU};

  int hg = 0, si = 0, k = 0, k0 = 0;
  SeqGeo geo{};
  bool first_piece = true;
  int n_merge = 0, mhg0 = 0, msi0 = 0, mhg1 = 0, msi1 = 0;
  uint32_t qf[D / 16][4];
  float o[DH / 8][4];
  float mrow[2], lrow[2];

  const int NS = P.NS;
  int stage = 0;
  uint32_t phase = 0;
  for (int it = 0; it < C.max_len; ++it, stage = (stage + 1 == NS) ? 0 : stage + 1,
           phase ^= (stage == 0) ? 1u : 0u) {
    if (it >= len) {
      release(C, stage);
      continue;
    }
    if (it == 0 || k == geo.pages) {
      const Cursor c = cursor_at(C.prefix, C.B, C.T1, lo + it);
      hg = c.hg;
      si = c.i;
      k = c.k;
      k0 = k;
      geo = seq_geo(P, si);
      const int head = hg * P.HG + hl;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int r = mt * 16 + g4 + 8 * h2;
        const int qi = r / P.G, gg = r % P.G;
        const bool valid = qi < geo.q_len;
        const T* qrow = qbase + (valid ? (int64_t)map_row(P.a, geo.q_start + qi) * P.a.q_sr +
                                             (int64_t)(head * P.G + gg) * P.a.q_sh
                                       : 0);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          uint32_t lo32 = 0, hi32 = 0;
          if (valid) {
            lo32 = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * c4);
            hi32 = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * c4);
          }
          qf[ks][h2] = lo32;      // rows g / g+8, k 0..7 of the step
          qf[ks][2 + h2] = hi32;  // rows g / g+8, k 8..15
        }
      }
#pragma unroll
      for (int n = 0; n < DH / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      mrow[0] = mrow[1] = -INFINITY;
      lrow[0] = lrow[1] = 0.f;
    }
    if (!wait_full(C, stage, phase)) return;

    const uint32_t sK = C.base + stage * C.L.stage_bytes + ps * C.L.page_bytes;
    const uint32_t sV = sK + P.PPS * C.L.page_bytes;
    const bool is_win = P.window && k == geo.pool_pages;
    const int kbase = is_win ? geo.pool_len : k * PAGE;
    const int valid = is_win ? geo.q_len : min(PAGE, geo.pool_len - k * PAGE);
    const int win_start = geo.kv_len - geo.q_len;
    const bool need_mask = valid < PAGE || (P.a.causal && kbase + PAGE - 1 > win_start);

    float sc[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t b0, b1, b2, b3;
      const int tok = (lane & 7) + ((lane >> 4) << 3);
      const int chunk = ks * 2 + ((lane >> 3) & 1);
      ldsm_x4(b0, b1, b2, b3, tile_addr<D>(sK, tok, hl, chunk));
      M::run(sc[0], qf[ks], b0, b1);
      M::run(sc[1], qf[ks], b2, b3);
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float s = sc[n][e] * sl2;
        if (need_mask) {
          const int tok = n * 8 + 2 * c4 + (e & 1);
          const int r = mt * 16 + g4 + 8 * (e >> 1);
          const int lim = P.a.causal ? win_start + r / P.G : geo.kv_len - 1;
          if (tok >= valid || kbase + tok > lim) s = -INFINITY;
        }
        sc[n][e] = s;
        mx[e >> 1] = fmaxf(mx[e >> 1], s);
      }
    }
    uint32_t pa[4];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      mx[h2] = fmaxf(mx[h2], __shfl_xor_sync(0xffffffffu, mx[h2], 1));
      mx[h2] = fmaxf(mx[h2], __shfl_xor_sync(0xffffffffu, mx[h2], 2));
      const float mnew = fmaxf(mrow[h2], mx[h2]);
      const float mu = (mnew == -INFINITY) ? 0.f : mnew;
      const float alpha = fast_exp2(mrow[h2] - mu);
      mrow[h2] = mnew;
      const float p0 = fast_exp2(sc[0][2 * h2] - mu), p1 = fast_exp2(sc[0][2 * h2 + 1] - mu);
      const float p2 = fast_exp2(sc[1][2 * h2] - mu), p3 = fast_exp2(sc[1][2 * h2 + 1] - mu);
      lrow[h2] = lrow[h2] * alpha + (p0 + p1 + p2 + p3);
#pragma unroll
      for (int n = 0; n < DH / 8; ++n) {
        o[n][2 * h2] *= alpha;
        o[n][2 * h2 + 1] *= alpha;
      }
      pa[h2] = M::pack(p0, p1);
      pa[2 + h2] = M::pack(p2, p3);
    }
#pragma unroll
    for (int np = 0; np < DH / 16; ++np) {
      uint32_t b0, b1, b2, b3;
      const int tok = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int chunk = dh * (DH / 8) + np * 2 + (lane >> 4);
      ldsm_x4_trans(b0, b1, b2, b3, tile_addr<D>(sV, tok, hl, chunk));
      if (valid < PAGE) {
        const int t_lo = 2 * c4, t_hi = 8 + 2 * c4;
        const uint32_t mlo = (t_lo < valid ? 0xffffu : 0u) | (t_lo + 1 < valid ? 0xffff0000u : 0u);
        const uint32_t mhi = (t_hi < valid ? 0xffffu : 0u) | (t_hi + 1 < valid ? 0xffff0000u : 0u);
        b0 &= mlo;
        b1 &= mhi;
        b2 &= mlo;
        b3 &= mhi;
      }
      M::run(o[2 * np], pa, b0, b1);
      M::run(o[2 * np + 1], pa, b2, b3);
    }
    ++k;
    release(C, stage);
    if (k != geo.pages && it != len - 1) continue;

#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      lrow[h2] += __shfl_xor_sync(0xffffffffu, lrow[h2], 1);
      lrow[h2] += __shfl_xor_sync(0xffffffffu, lrow[h2], 2);
    }
    const int head = hg * P.HG + hl;
    if (k0 == 0 && k == geo.pages) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int r = mt * 16 + g4 + 8 * h2;
        const int qi = r / P.G, gg = r % P.G;
        if (qi >= geo.q_len) continue;
        const float inv = lrow[h2] > 0.f ? 1.f / lrow[h2] : 0.f;
        const int64_t off = (int64_t)map_row(P.a, geo.q_start + qi) * P.a.o_sr +
                            (int64_t)(head * P.G + gg) * P.a.o_sh + dh * DH;
        for (int t = 0; t < out_targets(P.a); ++t) {
          T* orow = out_at<T>(P.a, t, off);
#pragma unroll
          for (int n = 0; n < DH / 8; ++n) {
            *reinterpret_cast<uint32_t*>(orow + n * 8 + 2 * c4) =
                M::pack(o[n][2 * h2] * inv, o[n][2 * h2 + 1] * inv);
          }
        }
      }
      first_piece = false;
      continue;
    }
    float* sl = PL.slot(vc, first_piece ? 0 : 1);
    first_piece = false;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int rr = g4 + 8 * h2;
      if (mt * 16 + rr >= geo.q_len * P.G) continue;  // no such query row
      float* pacc = PL.acc(sl, unit, rr);
#pragma unroll
      for (int n = 0; n < DH / 8; ++n)
        *reinterpret_cast<float2*>(pacc + n * 8 + 2 * c4) =
            make_float2(o[n][2 * h2], o[n][2 * h2 + 1]);
      if (c4 == 0) {
        PL.m(sl, unit)[rr] = mrow[h2];
        PL.l(sl, unit)[rr] = lrow[h2];
      }
    }
    int32_t* sem = P.sems + ((int64_t)hg * C.B + si) * units + unit;
    if (!arrive_last(C, sem, hg, si, geo.pages)) continue;
    if (n_merge == 0) {
      mhg0 = hg;
      msi0 = si;
    } else {
      mhg1 = hg;
      msi1 = si;
    }
    ++n_merge;
  }
  for (int m = 0; m < n_merge; ++m) {
    const int mhg = m == 0 ? mhg0 : mhg1;
    const int msi = m == 0 ? msi0 : msi1;
    merge_unit<T, RU, DH>(C, PL, mhg, msi, hl, unit, mt * 16, dh * DH);
    if (lane == 0) P.sems[((int64_t)mhg * C.B + msi) * units + unit] = 0;
  }
}

template <typename T, int D, bool SW>
__global__ void __launch_bounds__(THREADS, 1) decode_kernel(
    const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
    const __grid_constant__ CUtensorMap twk, const __grid_constant__ CUtensorMap twv,
    const __grid_constant__ Params P) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);
  const int B = P.a.num_seqs;
  const Smem L = smem_layout(D, P.HG, P.PPS, P.NS, B, P.window);
  uint64_t* full = reinterpret_cast<uint64_t*>(gbase + L.bar_off);
  uint64_t* empty = full + P.NS;
  int* prefix = reinterpret_cast<int*>(gbase + L.prefix_off);
  int* qstart = reinterpret_cast<int*>(gbase + L.qstart_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L.flag_off);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int units = SW ? P.HG : P.HG * P.MT * DS;  // consumer warps per page
  const int active_warps = units * P.PPS;          // consumer warps with work

  // ---------------------------------------------------------------- prologue
  if (tid == 0) {
    for (int s = 0; s < P.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (uint32_t)active_warps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Everything above overlaps the previous kernel (programmatic launch);
  // nothing in global memory is read before this point.
  grid_dependency_wait();
  for (int i = tid; i < B; i += blockDim.x) {
    const SeqGeo g = seq_geo(P, i);
    const bool other = P.skip_long && g.q_len * P.G > P.rows_cap;
    if (g.q_len > 0 && g.pages == 0 && !other) set_err(P.a.err, MF_ERR_LENGTH);
    if (g.pages > 0 && (g.pool_len + PAGE - 1) / PAGE > P.a.table_stride)
      set_err(P.a.err, MF_ERR_TABLE);
    prefix[i + 1] = g.pages;
    if (P.window) qstart[i] = g.q_start;
  }
  __syncthreads();
  if (warp == 0) {
    int run = 0;
    if (lane == 0) prefix[0] = 0;
    for (int c0 = 0; c0 < B; c0 += 32) {
      const int i = c0 + lane;
      int v = (i < B) ? prefix[i + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      if (i < B) prefix[i + 1] = run + v;
      run += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();

  const int64_t T1 = prefix[B];
  if (T1 == 0) return;
  const Split S = make_split(T1 * P.NHG, (int64_t)gridDim.x * P.PPS);
  // Longest virtual-CTA range of this CTA (the first one: lengths do not grow
  // with vc): every consumer loops this many stages.
  const int max_len = S.len((int64_t)blockIdx.x * P.PPS);
  if (max_len == 0) return;

  if (warp == CONSUMER_WARPS) {
    // ============================================================ producer
    const uint64_t pol = l2_evict_first_policy();
    if (lane == 0) {
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
      if (P.window) {
        prefetch_tmap(&twk);
        prefetch_tmap(&twv);
      }
    }
    // Lane j < PPS feeds virtual CTA j; block ids are loaded two pages ahead.
    const bool feeder = lane < P.PPS;
    const int64_t vc = (int64_t)blockIdx.x * P.PPS + lane;
    const int64_t lo = feeder ? S.bound(vc) : 0;
    const int len = feeder ? S.len(vc) : 0;
    auto block_of = [&](const Cursor& c) -> int {
      if (P.window && c.k == c.pages - 1) return 0;  // window page: no table entry
      return __ldg(P.a.tables + (int64_t)c.i * P.a.table_stride + c.k);
    };
    Cursor cur{0, 0, 0, 1}, ahead{0, 0, 0, 1};
    int blk0 = 0, blk1 = 0;
    if (len > 0) {
      cur = cursor_at(prefix, B, T1, lo);
      ahead = cur;
      blk0 = block_of(cur);
      if (len > 1) {
        cursor_next(ahead, prefix, B);
        blk1 = block_of(ahead);
      }
    }
    int armed = 0;
    for (int it = 0; it < max_len; ++it) {
      const int stage = it % P.NS;
      if (it >= P.NS) {
        if (lane == 0 && !mbar_wait_bounded(&empty[stage], ((it / P.NS) - 1) & 1, WAIT_LIMIT)) {
          set_err(P.a.err, MF_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        __syncwarp();
        if (*abort_flag) break;
      }
      // Pages this stage carries.
      const int n = __popc(__ballot_sync(0xffffffffu, feeder && it < len));
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], (uint32_t)n * 2u * L.page_bytes);
      __syncwarp();
      if (feeder && it < len) {
        uint8_t* sk = gbase + stage * L.stage_bytes + lane * L.page_bytes;
        uint8_t* sv = sk + P.PPS * L.page_bytes;
        if (P.window && cur.k == cur.pages - 1) {
          const int row = qstart[cur.i];
          tma_load_4d(sk, &twk, &full[stage], 0, row, 0, cur.hg * P.HG, pol);
          tma_load_4d(sv, &twv, &full[stage], 0, row, 0, cur.hg * P.HG, pol);
        } else {
          int blk = blk0;
          if (blk < 0 || blk >= P.a.num_blocks) {
            set_err(P.a.err, MF_ERR_BLOCK_ID);
            blk = 0;
          }
          tma_load_4d(sk, &tmk, &full[stage], 0, blk * PAGE, 0, cur.hg * P.HG, pol);
          tma_load_4d(sv, &tmv, &full[stage], 0, blk * PAGE, 0, cur.hg * P.HG, pol);
        }
        int blk2 = 0;
        if (it + 2 < len) {
          cursor_next(ahead, prefix, B);
          blk2 = block_of(ahead);
        }
        if (it + 1 < len) cursor_next(cur, prefix, B);
        blk0 = blk1;
        blk1 = blk2;
      }
      armed = it + 1;
    }
    // Drain: no TMA write may still target this CTA's shared memory at exit.
    if (lane == 0) {
      for (int it = max(0, armed - P.NS); it < armed; ++it) {
        if (!mbar_wait_bounded(&full[it % P.NS], (it / P.NS) & 1, WAIT_LIMIT))
          set_err(P.a.err, MF_ERR_TIMEOUT);
      }
    }
    return;
  }

  // ============================================================== consumers
  if (warp >= active_warps) return;
  Ctx C{P, L, base, full, empty, abort_flag, prefix, B, T1, S, warp, lane, max_len};
  if constexpr (SW)
    consume_swapped<T, D>(C);
  else
    consume_split<T, D>(C);
}

}  // namespace tc

TcPlan plan_attn_tc(const AttnParams& p, mf_dtype dtype, int sm_count, bool window,
                    bool skip_long) {
  TcPlan pl;
  pl.skip_long = skip_long;
  auto no = [&](const char* why) {
    pl.ok = false;
    pl.why = why;
    return pl;
  };
  if (dtype != MF_BF16 && dtype != MF_F16) return no("dtype is not bf16/f16");
  if (p.d != 64 && p.d != 128) return no("head_dim is not 64 or 128");
  if (p.block_size != tc::PAGE) return no("block_size is not 16");
  if (p.sb != (int64_t)tc::PAGE * p.ss) return no("pool blocks are not slot-contiguous");
  if ((p.ss * 2) % 16 || (p.sh * 2) % 16) return no("pool strides not 16-byte multiples");
  if ((reinterpret_cast<uintptr_t>(p.kp) | reinterpret_cast<uintptr_t>(p.vp)) & 15)
    return no("pool base not 16-byte aligned");
  if (p.num_seqs > tc::MAX_SEQS) return no("more than 4096 sequences");
  if ((p.q_sr | p.q_sh | p.o_sr | p.o_sh) & 1) return no("odd q/out strides");
  if ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.out)) & 3)
    return no("q/out not 4-byte aligned");
  if ((int64_t)p.num_blocks * tc::PAGE > 0x7fffffffLL) return no("pool slots exceed int32");
  const int G = p.hq / p.hkv;
  const int rows = G * p.max_q_len;
  if (rows > 64 || rows <= 0) return no("more than 64 rows per kv head");
  if (window) {
    if (p.max_q_len > tc::PAGE) return no("window longer than one page");
    if (p.num_seqs > tc::MAX_WINDOW_SEQS) return no("window batch above 1024 sequences");
    if ((p.w_sr * 2) % 16 || (p.w_sh * 2) % 16) return no("window strides not 16-byte multiples");
    if ((reinterpret_cast<uintptr_t>(p.wk) | reinterpret_cast<uintptr_t>(p.wv)) & 15)
      return no("window base not 16-byte aligned");
    if (p.row_map) return no("window with row_map");
  }
  pl.SW = rows <= 8;
  pl.MT = (rows + 15) / 16;
  pl.rows_cap = pl.SW ? 8 : pl.MT * 16;
  const int per_head = pl.SW ? 1 : pl.MT * tc::DS;  // consumer warps per kv head
  const int cap = tc::CONSUMER_WARPS / per_head;
  pl.HG = 1;
  for (int hg = cap; hg >= 1; --hg)
    if (p.hkv % hg == 0) {
      pl.HG = hg;
      break;
    }
  pl.NHG = p.hkv / pl.HG;
  pl.PPS = tc::CONSUMER_WARPS / (pl.HG * per_head);
  if (pl.PPS < 1) pl.PPS = 1;
  const size_t sem_bytes = (size_t)p.num_seqs * p.hkv * per_head * sizeof(int32_t);
  if (sem_bytes > tc::SEM_REGION) return no("too many (sequence, head) counters");
  const int budget = 227 * 1024 - 1024;  // opt-in maximum minus alignment slack
  auto layout = [&](int ns) {
    return tc::smem_layout(p.d, pl.HG, pl.PPS, ns, p.num_seqs, window ? 1 : 0);
  };
  int ns = 8;
  while (ns > 2 && layout(ns).total > (uint32_t)budget) --ns;
  if (layout(ns).total > (uint32_t)budget) return no("shared memory budget");
  pl.NS = ns;
  pl.smem = layout(ns).total + 1024;
  pl.ctas = sm_count;
  // partial slot: per unit RU rows x DU columns of fp32 plus m and l per row
  const int ru = pl.SW ? 8 : 16, du = pl.SW ? p.d : p.d / 2;
  const int unit_rows = pl.HG * per_head * ru;
  pl.part_floats = (size_t)unit_rows * (du + 2);
  pl.part_floats = (pl.part_floats + 63) & ~(size_t)63;
  pl.ws_bytes = tc::SEM_REGION + (size_t)pl.ctas * pl.PPS * 2 * pl.part_floats * sizeof(float);
  pl.ok = true;
  return pl;
}

static CUresult encode_4d(CUtensorMap* map, const void* base, int D, int64_t stride_head_bytes,
                          int64_t stride_tok_bytes, int heads, int64_t tokens, int HG,
                          CUtensorMapDataType dt);

template <typename T, int D>
static int launch_tc_t(const AttnParams& p, const TcPlan& pl, void* ws, cudaStream_t stream,
                       CUtensorMapDataType dt) {
  CUtensorMap mk, mv, mwk, mwv;
  const int64_t slots = (int64_t)p.num_blocks * tc::PAGE;
  CUresult r1 = encode_4d(&mk, p.kp, D, p.sh * 2, p.ss * 2, p.hkv, slots, pl.HG, dt);
  CUresult r2 = encode_4d(&mv, p.vp, D, p.sh * 2, p.ss * 2, p.hkv, slots, pl.HG, dt);
  if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS)
    return fail(MF_ECUDA, "paged attention: tensor map encoding failed for the pool");
  const bool window = p.wk != nullptr;
  if (window) {
    CUresult r3 = encode_4d(&mwk, p.wk, D, p.w_sh * 2, p.w_sr * 2, p.hkv, p.total_q, pl.HG, dt);
    CUresult r4 = encode_4d(&mwv, p.wv, D, p.w_sh * 2, p.w_sr * 2, p.hkv, p.total_q, pl.HG, dt);
    if (r3 != CUDA_SUCCESS || r4 != CUDA_SUCCESS)
      return fail(MF_ECUDA, "paged attention: tensor map encoding failed for the window");
  } else {
    mwk = mk;
    mwv = mv;
  }
  tc::Params P;
  P.a = p;
  P.G = p.hq / p.hkv;
  P.HG = pl.HG;
  P.NHG = pl.NHG;
  P.MT = pl.MT;
  P.PPS = pl.PPS;
  P.NS = pl.NS;
  P.rows_cap = pl.rows_cap;
  P.skip_long = pl.skip_long ? 1 : 0;
  P.window = window ? 1 : 0;
  P.scale_log2 = p.scale * 1.4426950408889634f;
  P.sems = static_cast<int32_t*>(ws);
  P.part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + tc::SEM_REGION);
  P.part_floats = (int)pl.part_floats;
  auto kern = pl.SW ? tc::decode_kernel<T, D, true> : tc::decode_kernel<T, D, false>;
  static thread_local int configured_dev[2] = {-1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev[pl.SW] != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess)
      return fail(MF_ECUDA, std::string("paged attention: ") + cudaGetErrorString(e));
    configured_dev[pl.SW] = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.ctas);
  cfg.blockDim = dim3(tc::THREADS);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&cfg, kern, mk, mv, mwk, mwv, P);
  if (le != cudaSuccess)
    return fail(MF_ECUDA, std::string("paged attention (tcgen05 decode): ") + cudaGetErrorString(le));
  return check_launch("paged attention (tensor-core decode)");
}

int launch_attn_tc(const AttnParams& p, mf_dtype dtype, const TcPlan& pl, void* ws,
                   cudaStream_t stream) {
  if (dtype == MF_BF16) {
    if (p.d == 128)
      return launch_tc_t<__nv_bfloat16, 128>(p, pl, ws, stream, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
    return launch_tc_t<__nv_bfloat16, 64>(p, pl, ws, stream, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  }
  if (p.d == 128)
    return launch_tc_t<__half, 128>(p, pl, ws, stream, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  return launch_tc_t<__half, 64>(p, pl, ws, stream, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
}

// ------------------------------------------------------------ tensor maps

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

// Tensor [tokens][heads][D] described as 4 dims, innermost first:
// (64 elements, tokens, D/64 halves, heads) with strides (., tok, 128 B, head),
// box (64, 16, D/64, HG): one page of HG heads lands in shared memory as
// [HG][D/64][16 tokens][128 bytes], 128-byte swizzled.
static CUresult encode_4d(CUtensorMap* map, const void* base, int D, int64_t stride_head_bytes,
                          int64_t stride_tok_bytes, int heads, int64_t tokens, int HG,
                          CUtensorMapDataType dt) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return CUDA_ERROR_NOT_SUPPORTED;
  cuuint64_t dims[4] = {64, (cuuint64_t)tokens, (cuuint64_t)(D / 64), (cuuint64_t)heads};
  cuuint64_t strides[3] = {(cuuint64_t)stride_tok_bytes, 128, (cuuint64_t)stride_head_bytes};
  cuuint32_t box[4] = {64, (cuuint32_t)tc::PAGE, (cuuint32_t)(D / 64), (cuuint32_t)HG};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace mf
