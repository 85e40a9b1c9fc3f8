// Paged decode / speculative-verify attention for bf16 / fp16 pools on sm_100a.
//
// HBM-bound design (4, 5):
//  * Work = the concatenated list of KV pages (16-token blocks) of all
//    sequences, for each group of HG kv heads.  It is cut into equal
//    contiguous ranges, one per "virtual CTA" (stream-K), so every SM streams
//    the same number of bytes whatever the context lengths are.  A range that
//    covers a whole sequence writes the output directly; a sequence split
//    across ranges leaves fp32 partials (running max, sum, unnormalised
//    accumulator) in the workspace and the last range to finish merges them
//    with the log-sum-exp identity (a per-sequence arrival counter; no waiting).
//  * One warp (the producer) walks the block table and issues one 4-D TMA
//    tile load per page per K/V: box (64 dims, D/64, HG kv heads, 16 tokens)
//    of the pool viewed as [slots][kv_heads][D], 128-byte swizzled, into a
//    ring of shared-memory stages guarded by mbarriers.  No multicast.
//  * Eight consumer warps each own one (kv head, 16-row m-tile): the rows are
//    (query position, query head) pairs of the GQA group, so a page is read
//    from HBM once for all query heads that share its kv head.  Scores and the
//    PV product use mma.sync m16n8k16 with fp32 accumulation; the online
//    softmax runs in registers in the log2 domain with quad shuffles.
//  * When fewer than 8 (head, m-tile) pairs exist, the CTA runs PPS = 8/(HG*MT)
//    independent virtual CTAs side by side, one page of each per stage.
//  * Every mbarrier wait is bounded; on expiry the CTA sets MF_ERR_TIMEOUT,
//    drains its own TMA loads and returns.

#include "mf_attn.h"

namespace mf {

namespace tc {

constexpr int CONSUMER_WARPS = 8;
constexpr int THREADS = (CONSUMER_WARPS + 1) * 32;
constexpr int PAGE = 16;
constexpr uint64_t WAIT_LIMIT = 2000000000ull;  // 2 s of wall time per wait
constexpr int MAX_SEQS = 4096;

struct Params {
  AttnParams a;
  int G, HG, NHG, MT, PPS, NS;
  int window;
  float scale_log2;
  float* part;       // partial slots
  int32_t* sems;     // arrival counters
  int part_floats;   // floats per partial slot
};

struct Smem {
  // layout offsets (bytes from the 1024-aligned base)
  uint32_t stage_bytes, page_bytes, bar_off, prefix_off, flag_off;
};

__host__ __device__ inline Smem smem_layout(int D, int HG, int PPS, int NS, int B) {
  Smem s;
  s.page_bytes = (uint32_t)(HG * PAGE * D * 2);
  s.stage_bytes = 2u * PPS * s.page_bytes;
  s.bar_off = NS * s.stage_bytes;
  s.prefix_off = s.bar_off + 2 * NS * 8;
  s.flag_off = s.prefix_off + (uint32_t)(B + 1) * 4;
  return s;
}

// Swizzled shared-memory address of the 16-byte chunk `chunk` (0..D/8-1) of
// token `tok`, local kv head `hl`, in a page tile written by a 128B-swizzle TMA.
template <int D>
MF_DEVINL uint32_t tile_addr(uint32_t base, int tok, int hl, int chunk, int HG) {
  const int half = chunk >> 3, cc = chunk & 7;
  const int R = (tok * HG + hl) * (D / 64) + half;
  return base + (uint32_t)(R * 128) + (uint32_t)((cc ^ (R & 7)) << 4);
}

// Page geometry of sequence i (identical in producer and consumers).
struct SeqGeo {
  int q_start, q_len, kv_len, pool_len, pool_pages, pages;
};

MF_DEVINL SeqGeo seq_geo(const Params& P, int i) {
  SeqGeo g;
  seq_rows(P.a, i, g.q_start, g.q_len);
  g.kv_len = P.a.kv_lens[i];
  const bool bad = g.q_len < 0 || g.kv_len < g.q_len || (g.q_len > 0 && g.kv_len <= 0) ||
                   g.q_len * P.G > P.MT * 16 || (P.window && g.q_len > PAGE);
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

// Virtual-CTA boundaries: range of vc is [bound(vc), bound(vc+1)).
MF_DEVINL int64_t bound(int64_t vc, int64_t total, int64_t NV) { return vc * total / NV; }

MF_DEVINL int owner(int64_t page, int64_t total, int64_t NV) {
  int64_t vc = page * NV / total;
  while (vc + 1 < NV && bound(vc + 1, total, NV) <= page) ++vc;
  while (vc > 0 && bound(vc, total, NV) > page) --vc;
  return (int)vc;
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

template <typename T, int D>
__global__ void __launch_bounds__(THREADS, 1) decode_kernel(
    const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
    const __grid_constant__ CUtensorMap twk, const __grid_constant__ CUtensorMap twv,
    const Params P) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);
  const int B = P.a.num_seqs;
  const Smem L = smem_layout(D, P.HG, P.PPS, P.NS, B);
  uint64_t* full = reinterpret_cast<uint64_t*>(gbase + L.bar_off);
  uint64_t* empty = full + P.NS;
  int* prefix = reinterpret_cast<int*>(gbase + L.prefix_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L.flag_off);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int units = P.HG * P.MT;           // (head, m-tile) pairs per page
  const int active_warps = units * P.PPS;  // consumer warps with work

  // ---------------------------------------------------------------- prologue
  if (tid == 0) {
    for (int s = 0; s < P.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (uint32_t)active_warps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = tid; i < B; i += blockDim.x) {
    const SeqGeo g = seq_geo(P, i);
    int q_start, q_len;
    seq_rows(P.a, i, q_start, q_len);
    if (q_len > 0 && g.pages == 0) set_err(P.a.err, MF_ERR_LENGTH);
    if (g.pages > 0) {
      const int need = (g.pool_len + PAGE - 1) / PAGE;
      if (need > P.a.table_stride) set_err(P.a.err, MF_ERR_TABLE);
    }
    prefix[i + 1] = g.pages;
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
  const int64_t TP = T1 * P.NHG;
  const int64_t NV = (int64_t)gridDim.x * P.PPS;
  if (TP == 0) return;
  // Longest virtual-CTA range of this CTA: every consumer loops this many stages.
  int max_len = 0;
  for (int j = 0; j < P.PPS; ++j) {
    const int64_t vc = (int64_t)blockIdx.x * P.PPS + j;
    max_len = max(max_len, (int)(bound(vc + 1, TP, NV) - bound(vc, TP, NV)));
  }
  if (max_len == 0) return;

  if (warp == CONSUMER_WARPS) {
    // ============================================================ producer
    const uint64_t pol = l2_evict_first_policy();
    if (lane == 0) {
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
      if (P.window) { prefetch_tmap(&twk); prefetch_tmap(&twv); }
    }
    // Lane j < PPS feeds virtual CTA j; block ids are fetched two pages ahead.
    const bool feeder = lane < P.PPS;
    const int64_t vc = (int64_t)blockIdx.x * P.PPS + lane;
    const int64_t lo = feeder ? bound(vc, TP, NV) : 0;
    const int len = feeder ? (int)(bound(vc + 1, TP, NV) - lo) : 0;
    auto page_src = [&](int it, int& hg, int& i, int& k, int& is_win) {
      const int64_t v = lo + it;
      hg = (int)(v / T1);
      const int off = (int)(v - (int64_t)hg * T1);
      i = find_seq(prefix, B, off);
      k = off - prefix[i];
      const SeqGeo g = seq_geo(P, i);
      is_win = (P.window && k == g.pool_pages) ? 1 : 0;
      return g;
    };
    auto fetch_block = [&](int it) -> int {
      if (!feeder || it >= len) return 0;
      int hg, i, k, w;
      page_src(it, hg, i, k, w);
      if (w) return 0;
      return __ldg(P.a.tables + (int64_t)i * P.a.table_stride + k);
    };
    int blk0 = fetch_block(0), blk1 = fetch_block(1);
    int armed = 0;
    bool ok = true;
    for (int it = 0; it < max_len; ++it) {
      const int stage = it % P.NS;
      if (it >= P.NS) {
        if (lane == 0 && !mbar_wait_bounded(&empty[stage], ((it / P.NS) - 1) & 1, WAIT_LIMIT)) {
          set_err(P.a.err, MF_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        __syncwarp();
        if (*abort_flag) { ok = false; break; }
      }
      const int blk2 = fetch_block(it + 2);
      // Pages this stage carries.
      int n = 0;
      for (int j = 0; j < P.PPS; ++j) {
        const int64_t vcj = (int64_t)blockIdx.x * P.PPS + j;
        if (it < (int)(bound(vcj + 1, TP, NV) - bound(vcj, TP, NV))) ++n;
      }
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], (uint32_t)n * 2u * L.page_bytes);
      __syncwarp();
      if (feeder && it < len) {
        int hg, i, k, w;
        const SeqGeo g = page_src(it, hg, i, k, w);
        uint8_t* sk = gbase + stage * L.stage_bytes + lane * L.page_bytes;
        uint8_t* sv = sk + P.PPS * L.page_bytes;
        if (w) {
          tma_load_4d(sk, &twk, &full[stage], 0, 0, hg * P.HG, map_row(P.a, g.q_start), pol);
          tma_load_4d(sv, &twv, &full[stage], 0, 0, hg * P.HG, map_row(P.a, g.q_start), pol);
        } else {
          int blk = blk0;
          if (blk < 0 || blk >= P.a.num_blocks) {
            set_err(P.a.err, MF_ERR_BLOCK_ID);
            blk = 0;
          }
          tma_load_4d(sk, &tmk, &full[stage], 0, 0, hg * P.HG, blk * PAGE, pol);
          tma_load_4d(sv, &tmv, &full[stage], 0, 0, hg * P.HG, blk * PAGE, pol);
        }
      }
      blk0 = blk1;
      blk1 = blk2;
      armed = it + 1;
    }
    (void)ok;
    // Drain: no TMA write may still target this CTA's shared memory at exit.
    if (lane == 0) {
      const int first = max(0, armed - P.NS);
      for (int it = first; it < armed; ++it) {
        if (!mbar_wait_bounded(&full[it % P.NS], (it / P.NS) & 1, WAIT_LIMIT))
          set_err(P.a.err, MF_ERR_TIMEOUT);
      }
    }
    return;
  }

  // ============================================================== consumers
  if (warp >= active_warps) return;
  using M = Mma<T>;
  const int pair = warp % units;
  const int ps = warp / units;       // virtual CTA within this CTA
  const int hl = pair / P.MT;        // local kv head
  const int mt = pair % P.MT;        // m-tile
  const int g4 = lane >> 2, c4 = lane & 3;
  const int64_t vc = (int64_t)blockIdx.x * P.PPS + ps;
  const int64_t lo = bound(vc, TP, NV);
  const int len = (int)(bound(vc + 1, TP, NV) - lo);
  const T* qbase = static_cast<const T*>(P.a.q);
  T* obase = static_cast<T*>(P.a.out);
  const float sl2 = P.scale_log2;

  // Piece state.
  int hg = 0, si = 0, k = 0, k0 = 0;
  SeqGeo geo{};
  bool first_piece = true;
  uint32_t qf[D / 16][4];
  float o[D / 8][4];
  float mrow[2], lrow[2];

  auto start_piece = [&](int64_t v) {
    hg = (int)(v / T1);
    const int off = (int)(v - (int64_t)hg * T1);
    si = find_seq(prefix, B, off);
    k = off - prefix[si];
    k0 = k;
    geo = seq_geo(P, si);
    const int head = hg * P.HG + hl;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int r = mt * 16 + g4 + 8 * h2;
      const int qi = r / P.G, gg = r % P.G;
      const bool valid = qi < geo.q_len;
      const T* qrow = valid ? qbase + (int64_t)map_row(P.a, geo.q_start + qi) * P.a.q_sr +
                                  (int64_t)(head * P.G + gg) * P.a.q_sh
                            : nullptr;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t lo32 = 0, hi32 = 0;
        if (valid) {
          lo32 = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * c4);
          hi32 = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * c4);
        }
        qf[ks][h2] = lo32;       // a0a1 (row g) / a2a3 (row g+8)
        qf[ks][2 + h2] = hi32;   // a4a5 / a6a7
      }
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    mrow[0] = mrow[1] = -INFINITY;
    lrow[0] = lrow[1] = 0.f;
  };

  auto finish_piece = [&]() {
    // quad-reduce the per-thread partial row sums
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      lrow[h2] += __shfl_xor_sync(0xffffffffu, lrow[h2], 1);
      lrow[h2] += __shfl_xor_sync(0xffffffffu, lrow[h2], 2);
    }
    const int head = hg * P.HG + hl;
    const bool whole = (k0 == 0 && k == geo.pages);
    const int64_t vs = (int64_t)hg * B + si;
    const int64_t vstart = (int64_t)hg * T1 + prefix[si];
    const int64_t vend = vstart + geo.pages;
    if (whole) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int r = mt * 16 + g4 + 8 * h2;
        const int qi = r / P.G, gg = r % P.G;
        if (qi >= geo.q_len) continue;
        const float inv = lrow[h2] > 0.f ? 1.f / lrow[h2] : 0.f;
        T* orow = obase + (int64_t)map_row(P.a, geo.q_start + qi) * P.a.o_sr +
                  (int64_t)(head * P.G + gg) * P.a.o_sh;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          *reinterpret_cast<uint32_t*>(orow + n * 8 + 2 * c4) =
              M::pack(o[n][2 * h2] * inv, o[n][2 * h2 + 1] * inv);
        }
      }
      first_piece = false;
      return;
    }
    // Partial: slot 0 when this piece starts the virtual CTA's range.
    const int slot = first_piece ? 0 : 1;
    first_piece = false;
    float* part = P.part + ((vc * 2 + slot) * (int64_t)P.part_floats);
    const int rows_total = P.HG * P.MT * 16;
    float* pacc = part + (int64_t)((hl * P.MT + mt) * 16) * D;
    float* pm = part + (int64_t)rows_total * D + (hl * P.MT + mt) * 16;
    float* pl = pm + rows_total;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int rr = g4 + 8 * h2;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        *reinterpret_cast<float2*>(pacc + rr * D + n * 8 + 2 * c4) =
            make_float2(o[n][2 * h2], o[n][2 * h2 + 1]);
      }
      if (c4 == 0) {
        pm[rr] = mrow[h2];
        pl[rr] = lrow[h2];
      }
    }
    __threadfence();
    __syncwarp();
    int32_t* sem = P.sems + (vs * P.HG + hl) * P.MT + mt;
    const int vc0 = owner(vstart, TP, NV);
    const int vc1 = owner(vend - 1, TP, NV);
    int old = 0;
    if (lane == 0) old = atomicAdd(sem, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != vc1 - vc0) return;
    // Last arrival for this (sequence, head, m-tile): merge every range's partial.
    __threadfence();
    for (int rr = 0; rr < 16; ++rr) {
      const int r = mt * 16 + rr;
      const int qi = r / P.G, gg = r % P.G;
      if (qi >= geo.q_len) continue;
      float Mx = -INFINITY;
      for (int c = vc0; c <= vc1; ++c) {
        const int sl = (bound(c, TP, NV) >= vstart) ? 0 : 1;
        const float* pp = P.part + (int64_t)(c * 2 + sl) * P.part_floats +
                          (int64_t)rows_total * D + (hl * P.MT + mt) * 16;
        Mx = fmaxf(Mx, __ldcg(pp + rr));
      }
      const float Mu = (Mx == -INFINITY) ? 0.f : Mx;
      float Ls = 0.f;
      float acc[D / 32];
#pragma unroll
      for (int e = 0; e < D / 32; ++e) acc[e] = 0.f;
      for (int c = vc0; c <= vc1; ++c) {
        const int sl = (bound(c, TP, NV) >= vstart) ? 0 : 1;
        const float* pp = P.part + (int64_t)(c * 2 + sl) * P.part_floats;
        const float* ppm = pp + (int64_t)rows_total * D + (hl * P.MT + mt) * 16;
        const float mk = __ldcg(ppm + rr);
        const float w = (mk == -INFINITY) ? 0.f : fast_exp2(mk - Mu);
        Ls += w * __ldcg(ppm + rows_total + rr);
        const float* pa = pp + (int64_t)((hl * P.MT + mt) * 16 + rr) * D;
#pragma unroll
        for (int e = 0; e < D / 32; ++e) acc[e] += w * __ldcg(pa + lane + 32 * e);
      }
      const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
      T* orow = obase + (int64_t)map_row(P.a, geo.q_start + qi) * P.a.o_sr +
                (int64_t)(head * P.G + gg) * P.a.o_sh;
#pragma unroll
      for (int e = 0; e < D / 32; ++e) orow[lane + 32 * e] = from_f32<T>(acc[e] * inv);
    }
    if (lane == 0) *sem = 0;  // leave the counter zeroed for the next launch
  };

  bool have_piece = false;
  for (int it = 0; it < max_len; ++it) {
    const int stage = it % P.NS;
    if (it < len) {
      if (!have_piece) {
        start_piece(lo + it);
        have_piece = true;
      }
      bool ok = true;
      if (!mbar_wait_bounded(&full[stage], (it / P.NS) & 1, WAIT_LIMIT)) {
        if (lane == 0) set_err(P.a.err, MF_ERR_TIMEOUT);
        ok = false;
      }
      if (!__all_sync(0xffffffffu, ok) || *abort_flag) {
        *abort_flag = 1;
        return;
      }
      const uint32_t sK = base + stage * L.stage_bytes + ps * L.page_bytes;
      const uint32_t sV = sK + P.PPS * L.page_bytes;
      const bool is_win = P.window && k == geo.pool_pages;
      const int kbase = is_win ? geo.pool_len : k * PAGE;
      const int valid = is_win ? geo.q_len : min(PAGE, geo.pool_len - k * PAGE);
      const int win_start = geo.kv_len - geo.q_len;
      const bool need_mask = valid < PAGE || (P.a.causal && kbase + PAGE - 1 > win_start);

      // S = Q K^T for 16 rows x 16 tokens
      float sc[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t b0, b1, b2, b3;
        const int tok = (lane & 7) + ((lane >> 4) << 3);
        const int chunk = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, tile_addr<D>(sK, tok, hl, chunk, P.HG));
        M::run(sc[0], qf[ks], b0, b1);
        M::run(sc[1], qf[ks], b2, b3);
      }
      // online softmax (log2 domain)
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
        for (int n = 0; n < D / 8; ++n) {
          o[n][2 * h2] *= alpha;
          o[n][2 * h2 + 1] *= alpha;
        }
        pa[h2] = M::pack(p0, p1);      // (row g / g+8, tokens 2c..2c+1)
        pa[2 + h2] = M::pack(p2, p3);  // (row g / g+8, tokens 8+2c..)
      }
      // O += P V
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int tok = (lane & 7) + (((lane >> 3) & 1) << 3);
        const int chunk = np * 2 + (lane >> 4);
        ldsm_x4_trans(b0, b1, b2, b3, tile_addr<D>(sV, tok, hl, chunk, P.HG));
        if (valid < PAGE) {
          // Unwritten slots may hold anything (NaN included): zero them so
          // that p = 0 really contributes nothing.
          const int t_lo = 2 * c4, t_hi = 8 + 2 * c4;
          const uint32_t mlo = (t_lo < valid ? 0xffffu : 0u) | (t_lo + 1 < valid ? 0xffff0000u : 0u);
          const uint32_t mhi = (t_hi < valid ? 0xffffu : 0u) | (t_hi + 1 < valid ? 0xffff0000u : 0u);
          b0 &= mlo; b1 &= mhi; b2 &= mlo; b3 &= mhi;
        }
        M::run(o[2 * np], pa, b0, b1);
        M::run(o[2 * np + 1], pa, b2, b3);
      }
      ++k;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      // A piece ends with its sequence or with this virtual CTA's range.
      if (k == geo.pages || it == len - 1) {
        finish_piece();
        have_piece = false;
      }
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }
  }
}

}  // namespace tc

TcPlan plan_attn_tc(const AttnParams& p, mf_dtype dtype, int sm_count, bool window) {
  TcPlan pl;
  auto no = [&](const char* why) { pl.ok = false; pl.why = why; return pl; };
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
    if ((p.w_sr * 2) % 16 || (p.w_sh * 2) % 16) return no("window strides not 16-byte multiples");
    if ((reinterpret_cast<uintptr_t>(p.wk) | reinterpret_cast<uintptr_t>(p.wv)) & 15)
      return no("window base not 16-byte aligned");
    if (p.row_map) return no("window with row_map");
  }
  pl.MT = (rows + 15) / 16;
  const int cap = 8 / pl.MT;
  pl.HG = 1;
  for (int hg = cap; hg >= 1; --hg)
    if (p.hkv % hg == 0) { pl.HG = hg; break; }
  pl.NHG = p.hkv / pl.HG;
  pl.PPS = 8 / (pl.HG * pl.MT);
  if (pl.PPS < 1) pl.PPS = 1;
  const int budget = 227 * 1024 - 1024;  // opt-in maximum minus alignment slack
  auto layout = [&](int ns) { return tc::smem_layout(p.d, pl.HG, pl.PPS, ns, p.num_seqs); };
  int ns = 8;
  while (ns > 2 && layout(ns).flag_off + 16 > (uint32_t)budget) --ns;
  if (layout(ns).flag_off + 16 > (uint32_t)budget) return no("shared memory budget");
  pl.NS = ns;
  pl.smem = layout(ns).flag_off + 16 + 1024;
  pl.ctas = sm_count;
  const int rows_total = pl.HG * pl.MT * 16;
  pl.part_floats = (size_t)rows_total * (p.d + 2);
  pl.part_floats = (pl.part_floats + 63) & ~(size_t)63;
  const size_t part_bytes = (size_t)pl.ctas * pl.PPS * 2 * pl.part_floats * sizeof(float);
  const size_t sem_bytes = (size_t)p.num_seqs * pl.NHG * pl.HG * pl.MT * sizeof(int32_t);
  pl.ws_bytes = part_bytes + ((sem_bytes + 255) & ~(size_t)255);
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
  P.window = window ? 1 : 0;
  P.scale_log2 = p.scale * 1.4426950408889634f;
  P.part = static_cast<float*>(ws);
  const size_t part_bytes = (size_t)pl.ctas * pl.PPS * 2 * pl.part_floats * sizeof(float);
  P.sems = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + part_bytes);
  P.part_floats = (int)pl.part_floats;
  auto kern = tc::decode_kernel<T, D>;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev || configured_smem < pl.smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return fail(MF_ECUDA, std::string("paged attention: ") + cudaGetErrorString(e));
    configured_dev = dev;
    configured_smem = 227 * 1024;
  }
  kern<<<pl.ctas, tc::THREADS, pl.smem, stream>>>(mk, mv, mwk, mwv, P);
  return check_launch("paged attention (tensor-core decode)");
}

int launch_attn_tc(const AttnParams& p, mf_dtype dtype, const TcPlan& pl, void* ws,
                   cudaStream_t stream) {
  if (dtype == MF_BF16) {
    if (p.d == 128) return launch_tc_t<__nv_bfloat16, 128>(p, pl, ws, stream, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
    return launch_tc_t<__nv_bfloat16, 64>(p, pl, ws, stream, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  }
  if (p.d == 128) return launch_tc_t<__half, 128>(p, pl, ws, stream, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
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

// [tokens][heads][D] with D split into 64-element (128-byte) rows so that the
// 128-byte swizzle applies; box = (64, D/64, HG, 16 tokens).
static CUresult encode_4d(CUtensorMap* map, const void* base, int D, int64_t stride_head_bytes,
                          int64_t stride_tok_bytes, int heads, int64_t tokens, int HG,
                          CUtensorMapDataType dt) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return CUDA_ERROR_NOT_SUPPORTED;
  cuuint64_t dims[4] = {64, (cuuint64_t)(D / 64), (cuuint64_t)heads, (cuuint64_t)tokens};
  cuuint64_t strides[3] = {128, (cuuint64_t)stride_head_bytes, (cuuint64_t)stride_tok_bytes};
  cuuint32_t box[4] = {64, (cuuint32_t)(D / 64), (cuuint32_t)HG, (cuuint32_t)tc::PAGE};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace mf
