// Paged chunked-prefill attention on the sm_100a tensor cores (tcgen05 + TMEM).
//
// Persistent: one CTA per SM walks a list of work items, each one 128-row
// query tile of one sequence for one kv head.  The 128 rows are (query
// position, query head of the GQA group) pairs, so each K/V tile is loaded once
// for every query head sharing the kv head.
//
//   warps 0..4*WPQ-1  softmax and epilogue: warp w reads TMEM lanes 32 (w % 4) ..
//              (tile rows) and columns [CW (w / 4), CW (w / 4 + 1)) of S, P and O;
//              the WPQ warps of one lane quarter combine their partial row maxima
//              (and, at the end, row sums) through shared memory
//   next 2     TMA producer warps: Q (two buffers) and K, and V; per 128-key
//              tile 8 pages x 2 halves (4-D tiled loads from the pool, 128-byte
//              swizzled), one box per lane, into two-stage K and V rings
//   next warp  S issuer (one thread): S = Q K^T into one of two TMEM S buffers
//   last warp  P V issuer (one thread): O += P V with P read from one of two
//              TMEM P buffers
//
// tcgen05.mma issue returns only as the tensor pipe takes the instruction, so
// one thread issuing everything would leave the pipe idle whenever it waits
// (for a P, a K tile, a free buffer).  Two issuers, one per product, let each
// keep the pipe busy while the other waits.
//
// TMEM (512 columns): S_a S_b (128 fp32 each), P_a P_b (64 columns of packed
// 16-bit pairs each), O (128 fp32).  P does not alias S, so an S buffer is free
// again as soon as the softmax warps have loaded it: the S of a tile can be
// computed while the softmax of the previous tile runs.
//
// Each lane quarter has two softmax warps that take alternate key tiles, so one
// warp's TMEM load, row max and P store overlap the other's exponentials.  An
// item's epilogue (combining the two warps' row sums, normalising O, storing)
// is deferred past each warp's first tile of the next item, so the tensor pipe
// is not idle while O is read out.
//
// The online softmax keeps a per-row reference max (log2 units) and only
// rescales O (a TMEM read-modify-write) when a tile's max exceeds it by more
// than 2^8, so the exponentials stay <= 256 and the correction is rare after the
// first tiles.  Masking: key k is visible to row r iff k < kv_len and k <=
// kv_len - q_len + position(r) (causal) — the varlen rule of
// memforge_ml/kernels/varlen_attention.py:193-201.  Pages past the block table
// load as zeros (out-of-range TMA coordinates) and unwritten slots of the last
// page are zeroed in shared memory before the P V product.
//
// Every mbarrier wait is bounded; on expiry the CTA raises MF_ERR_TIMEOUT, drains
// its TMA loads and MMAs, frees its TMEM and returns.

#include "mf_attn.h"

namespace mf {
namespace pf {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int WPQ = 2;                  // softmax warps per TMEM lane quarter (tile parities)
constexpr int SM_WARPS = 4 * WPQ;       // softmax warps
constexpr int TILE_WARPS = 4;           // softmax warps working on one tile (one per quarter)
constexpr int CW = BN;                  // score columns per softmax warp (all of its tiles)
constexpr int TMA_WARP = SM_WARPS, V_WARP = SM_WARPS + 1, MMA_WARP = SM_WARPS + 2,
              PV_WARP = SM_WARPS + 3;
constexpr int THREADS = (SM_WARPS + 4) * 32;

static_assert(CW == 32 || CW == 64 || CW == 128, "softmax column split");
constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int KS = 2;  // K and V ring stages
constexpr int MAX_SEQS = 4096;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint64_t WAIT_LIMIT = 2000000000ull;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

constexpr uint32_t TILE_BYTES = BN * D * 2;   // 32 KB: [half][128 rows][128 B]
constexpr uint32_t HALF_BYTES = BN * 128;     // 16 KB
constexpr uint32_t OFF_Q = 0;                 // two Q buffers
constexpr uint32_t OFF_K = OFF_Q + 2 * TILE_BYTES;
constexpr uint32_t OFF_V = OFF_K + KS * TILE_BYTES;
constexpr uint32_t OFF_BAR = OFF_V + KS * TILE_BYTES;

// mbarrier indices
// S_DONE[b] (the S of tile g completed, b = g & 1) also frees K ring stage
// g % KS, and PV_DONE[b] (the P V of tile g completed) also frees P buffer b and
// V ring stage g % KS: with two stages the indices coincide, so one commit
// serves both waiters.
static_assert(KS == 2, "ring stages double as S / P buffer indices");
constexpr int B_QFULL = 0, B_QEMPTY = 2, B_KFULL = 4, B_VFULL = B_KFULL + KS,
              B_SDONE = B_VFULL + KS, B_SFREE = B_SDONE + 2, B_PFULL = B_SFREE + 2,
              B_PVDONE = B_PFULL + 2,
              B_OFULL = B_PVDONE + 2, B_OFREE = B_OFULL + 1, B_IDLE = B_OFREE + 1,
              B_HAND = B_IDLE + 1, B_EXL = B_HAND + 8, NBAR = B_EXL + 4;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;  // TMEM base, abort flag
// Row statistics passed between the two softmax warps of a lane quarter:
// m[2 parities][BM] (the reference max after a tile), then l[2 items][2
// parities][BM] and ms[2 items][2 parities][BM] (an item's partial row sums and
// the reference max they are scaled to).
constexpr uint32_t OFF_XCH = OFF_MISC + 16;
// Work-list tables: prefix int[num_seqs + 1] (query tiles before the k-th
// sequence in longest-first order), order uint16[num_seqs] (that sequence), and
// NBK bucket counters of the counting sort.
constexpr uint32_t OFF_PREFIX = OFF_XCH + 10 * BM * 4;
constexpr int NBK = 256;

// TMEM column offsets
constexpr uint32_t COL_S = 0, COL_P = 256, COL_O = 384;

__host__ __device__ constexpr uint32_t off_order(int num_seqs) {
  return OFF_PREFIX + (((uint32_t)(num_seqs + 1) * 4u + 15u) & ~15u);
}
__host__ __device__ constexpr uint32_t off_counts(int num_seqs) {
  return off_order(num_seqs) + (((uint32_t)num_seqs * 2u + 15u) & ~15u);
}
__host__ __device__ constexpr uint32_t smem_bytes(int num_seqs) {
  return off_counts(num_seqs) + NBK * 4u;
}
static_assert(smem_bytes(MAX_SEQS) + 1024 <= 227u * 1024u, "shared memory budget");

// Sort key of a sequence: about 8 buckets per doubling of kv_len, longest first
// (bucket 0); sequences without work last.
MF_DEVINL int length_bucket(int kv_len, int tiles) {
  if (tiles == 0 || kv_len <= 0) return NBK - 1;
  const int e = 31 - __clz(kv_len);
  const int mant = e >= 3 ? (kv_len >> (e - 3)) & 7 : (kv_len << (3 - e)) & 7;
  return NBK - 2 - min(8 * e + mant, NBK - 2);
}

// Verify items (a window: one query tile per sequence in practice) sort by
// their exact key-tile count, so the snake deal pairs long and short items
// as closely as the counts allow; other items by length_bucket.
template <typename PP>
MF_DEVINL int sort_bucket(const PP& P, int kv_len, int q_len, int tiles) {
  if (!P.window || tiles == 0 || kv_len <= 0) return length_bucket(kv_len, tiles);
  const int nt = (kv_len - q_len + BN - 1) / BN + 1;
  return NBK - 2 - min(nt, NBK - 2);
}

// Work item handled by this CTA in its k-th step: items are dealt to the CTAs
// in a snake order (0..G-1, then G-1..0, ...), so that with the longest items
// first the CTAs that get the longest of one pass get the shortest of the next.
MF_DEVINL int snake_item(int k) {
  const int G = gridDim.x, c = blockIdx.x;
  return k * G + ((k & 1) ? G - 1 - c : c);
}

struct Params {
  AttnParams a;
  int G;
  int rows_cap;      // sequences with q_len * G <= rows_cap belong to the decode kernel
  float scale_log2;
  uint32_t in_fmt;   // 0 = f16, 1 = bf16
  int window;        // 1: the last q_len keys of each sequence come from the window buffers
};

// Geometry of one work item (identical in every role).
struct Item {
  int s, h, q_start, q_len, kv_len, win_start, pos0, nt;
  int pool_len;  // keys read from the pool (the rest, with a window, from the window buffers)
};

// Query positions per tile: the tile's rows are (position, query head) pairs,
// floor(128 / G) positions x G heads (the rows past that are padding).
__host__ __device__ constexpr int positions_per_tile(int G) { return BM / G; }

MF_DEVINL int find_tile_seq(const int* prefix, int B, int t) {
  int lo = 0, hi = B;  // prefix[lo] <= t < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

// Items run longest first: sequences by decreasing kv_len, and within a
// sequence the last query tiles (which see the most keys) first.
MF_DEVINL Item item_at(const Params& P, const int* prefix, const uint16_t* order, int B,
                       int it) {
  Item I;
  const int hkv = P.a.hkv;
  const int t = it / hkv;
  I.h = it % hkv;
  const int k = find_tile_seq(prefix, B, t);
  I.s = order[k];
  const int qt = prefix[k + 1] - 1 - t;
  seq_rows(P.a, I.s, I.q_start, I.q_len);
  I.kv_len = __ldg(P.a.kv_lens + I.s);
  I.win_start = I.kv_len - I.q_len;
  const int ppt = positions_per_tile(P.G);
  I.pos0 = qt * ppt;
  const int pos_last = min(I.q_len - 1, I.pos0 + ppt - 1);
  if (P.window) {
    // Pool tiles for positions < kv_len - q_len, then one tile holding the
    // window (q_len <= 16 keys) in its first rows.
    I.pool_len = I.win_start;
    I.nt = (I.pool_len + BN - 1) / BN + 1;
  } else {
    I.pool_len = I.kv_len;
    const int key_end = I.win_start + pos_last + 1;  // keys this tile can see
    I.nt = (key_end + BN - 1) / BN;
  }
  return I;
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1) prefill_kernel(
    const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
    const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmwk,
    const __grid_constant__ CUtensorMap tmwv, const __grid_constant__ Params P) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);
  uint64_t* bar = reinterpret_cast<uint64_t*>(gbase + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_MISC + 4);
  int* prefix = reinterpret_cast<int*>(gbase + OFF_PREFIX);
  uint16_t* order = reinterpret_cast<uint16_t*>(gbase + off_order(P.a.num_seqs));
  int* counts = reinterpret_cast<int*>(gbase + off_counts(P.a.num_seqs));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = P.a.num_seqs;
  const int G = P.G;

  // ------------------------------------------------------------- set-up
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[B_QFULL + i], 1);
      mbar_init(&bar[B_QEMPTY + i], 1);
      mbar_init(&bar[B_SDONE + i], 1);
      mbar_init(&bar[B_SFREE + i], TILE_WARPS);
      mbar_init(&bar[B_PFULL + i], TILE_WARPS);
      mbar_init(&bar[B_PVDONE + i], 1);
    }
    for (int st = 0; st < KS; ++st) {
      mbar_init(&bar[B_KFULL + st], 1);
      mbar_init(&bar[B_VFULL + st], 1);
    }
    mbar_init(&bar[B_OFULL], 1);
    mbar_init(&bar[B_OFREE], SM_WARPS);  // every softmax warp reads its half of O
    mbar_init(&bar[B_IDLE], 2);  // one commit per issuer
    for (int i = 0; i < 8; ++i) mbar_init(&bar[B_HAND + i], 1);
    for (int q = 0; q < 4; ++q) mbar_init(&bar[B_EXL + q], WPQ);
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = tid; i < NBK; i += THREADS) counts[i] = 0;
  // Everything above overlaps the previous kernel (programmatic launch);
  // nothing in global memory is read before this point.
  grid_dependency_wait();
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  // Query tiles per sequence (only runs longer than rows_cap rows are served
  // here) and a counting sort of the sequences by kv_len, longest first.  Every
  // CTA builds the same list, so the sort is stable (ties keep index order).
  for (int i = tid; i < B; i += THREADS) {
    int qs, ql;
    seq_rows(P.a, i, qs, ql);
    int tiles = 0;
    const int kvl = P.a.kv_lens[i];
    if (ql > 0 && ql * G > P.rows_cap) {
      if (kvl < ql) {
        set_err(P.a.err, MF_ERR_LENGTH);
      } else if (((P.window ? kvl - ql : kvl) + PAGE - 1) / PAGE > P.a.table_stride) {
        set_err(P.a.err, MF_ERR_TABLE);
      } else {
        const int ppt = positions_per_tile(G);
        tiles = (ql + ppt - 1) / ppt;
      }
    }
    atomicAdd(&counts[sort_bucket(P, kvl, ql, tiles)], 1);
    prefix[i + 1] = tiles;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the bucket counts
    int run = 0;
    for (int c0 = 0; c0 < NBK; c0 += 32) {
      int v = counts[c0 + lane];
      const int own = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      counts[c0 + lane] = run + v - own;
      run += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  if (warp == 0) {  // place the sequences 32 at a time, in index order
    for (int c0 = 0; c0 < B; c0 += 32) {
      const int i = c0 + lane;
      int qs_, ql_ = 0;
      if (i < B) seq_rows(P.a, i, qs_, ql_);
      const int b = i < B ? sort_bucket(P, P.a.kv_lens[i], ql_, prefix[i + 1]) : -1;
      const unsigned same = __match_any_sync(0xffffffffu, b);
      const int slot = b >= 0 ? counts[b] + __popc(same & ((1u << lane) - 1u)) : 0;
      __syncwarp();
      if (b >= 0) {
        order[slot] = (uint16_t)i;
        if (lane == __ffs(same) - 1) counts[b] += __popc(same);
      }
      __syncwarp();
    }
  }
  __syncthreads();
  // Tiles per sequence in sorted order (all read before any is overwritten),
  // then their prefix sums.
  {
    constexpr int NR = (MAX_SEQS + THREADS - 1) / THREADS;
    int tv[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const int k = r * THREADS + tid;
      tv[r] = k < B ? prefix[order[k] + 1] : 0;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const int k = r * THREADS + tid;
      if (k < B) prefix[k + 1] = tv[r];
    }
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
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int items = prefix[B] * P.a.hkv;

  if (warp == TMA_WARP || warp == V_WARP) {
    // ======================================================= TMA producers
    // One warp loads Q and K, another V: the K ring frees at S completion and
    // the V ring only at P V completion, so K loads never queue behind V.  A
    // 128-key tile is 8 pages x 2 halves = 16 boxes: lane l < 16 loads the block
    // id of page l / 2 (one tile ahead) and issues the box of (page l / 2, half
    // l % 2), so a tile goes out as one warp instruction; lane 0 does the ring
    // waits and the transaction count, and broadcasts every decision.
    const bool is_v = warp == V_WARP;
    const uint32_t q_bytes = (uint32_t)(positions_per_tile(G) * G) * D * 2;  // both halves
    const CUtensorMap* wmap = is_v ? &tmwv : &tmwk;
    const uint64_t pol_once = l2_evict_first_policy();
    const uint64_t pol_keep = l2_evict_last_policy();
    if (lane == 0) {
      if (!is_v) {
        prefetch_tmap(&tmq);
        prefetch_tmap(&tmk);
      } else {
        prefetch_tmap(&tmv);
      }
      if (P.window) prefetch_tmap(wmap);
    }
    const CUtensorMap* tmap = is_v ? &tmv : &tmk;
    const uint32_t ring = is_v ? OFF_V : OFF_K;
    uint64_t* fullb = &bar[is_v ? B_VFULL : B_KFULL];
    uint64_t* emptyb = &bar[is_v ? B_PVDONE : B_SDONE];  // ring stage g % KS frees
    const int nb = P.a.num_blocks;
    const bool boxer = lane < 2 * (BN / PAGE);
    const int my_pg = lane >> 1, my_half = lane & 1;
    uint32_t g = 0;      // tiles started (all items)
    uint32_t armed = 0;  // tiles whose loads were issued
    int ic = 0;          // items whose Q load was issued
    bool run = true;
    for (int k = 0; run && snake_item(k) < items; ++k) {
      run = __shfl_sync(0xffffffffu, *abort_flag == 0, 0);
      if (!run) break;
      const Item I = item_at(P, prefix, order, B, snake_item(k));
      if (!is_v) {
        const int qb = ic & 1;
        bool fine = true;
        if (lane == 0) {
          if (ic >= 2 &&
              !mbar_wait_bounded(&bar[B_QEMPTY + qb], ((ic >> 1) - 1) & 1, WAIT_LIMIT)) {
            set_err(P.a.err, MF_ERR_TIMEOUT);
            *abort_flag = 1;
            fine = false;
          } else {
            mbar_arrive_expect_tx(&bar[B_QFULL + qb], q_bytes);
            for (int half = 0; half < 2; ++half)
              tma_load_4d(gbase + OFF_Q + qb * TILE_BYTES + half * HALF_BYTES, &tmq,
                          &bar[B_QFULL + qb], 0, I.h * G, half, I.q_start + I.pos0, pol_once);
          }
        }
        run = __shfl_sync(0xffffffffu, fine, 0);
        if (!run) break;
        ++ic;
      }
      const int pool_pages = (I.pool_len + PAGE - 1) / PAGE;
      const int32_t* table = P.a.tables + (int64_t)I.s * P.a.table_stride;
      // Block id of this lane's page, loaded one tile ahead.  Out-of-table
      // pages use an out-of-range coordinate: TMA fills zeros.
      int nxt = (boxer && my_pg < pool_pages) ? __ldg(table + my_pg) : -1;
      for (int j = 0; j < I.nt; ++j, ++g) {
        const int L = j * (BN / PAGE) + my_pg;
        int tok = nb * PAGE;
        if (boxer && L < pool_pages) {
          if (nxt >= 0 && nxt < nb) tok = nxt * PAGE;
          else set_err(P.a.err, MF_ERR_BLOCK_ID);
        }
        if (j + 1 < I.nt)
          nxt = (boxer && L + BN / PAGE < pool_pages) ? __ldg(table + L + BN / PAGE) : -1;
        const int st = g % KS;
        // With a window, the last tile is the window: 16 rows of each half.
        const bool win_tile = P.window && j == I.nt - 1;
        bool fine = true;
        if (lane == 0) {
          if (g >= KS && !mbar_wait_bounded(&emptyb[st], ((g / KS) - 1) & 1, WAIT_LIMIT)) {
            set_err(P.a.err, MF_ERR_TIMEOUT);
            *abort_flag = 1;
            fine = false;
          } else if (*abort_flag) {
            fine = false;
          } else {
            mbar_arrive_expect_tx(&fullb[st], win_tile ? 2u * PAGE * 128u : TILE_BYTES);
          }
        }
        run = __shfl_sync(0xffffffffu, fine, 0);  // also orders expect_tx before the loads
        if (!run) break;
        armed = g + 1;
        uint8_t* dst = gbase + ring + st * TILE_BYTES + my_half * HALF_BYTES;
        if (win_tile) {
          if (lane < 2)
            tma_load_4d(dst, wmap, &fullb[st], 0, I.q_start, my_half, I.h, pol_once);
        } else if (boxer) {
          tma_load_4d(dst + my_pg * PAGE * 128, tmap, &fullb[st], 0, tok, my_half, I.h, pol_keep);
        }
      }
    }
    // Drain every armed load before the CTA can exit (the ring holds the last
    // KS tiles and the last two Q tiles in flight at most).
    if (lane == 0) {
      for (uint32_t k = armed > (uint32_t)KS ? armed - KS : 0u; k < armed; ++k)
        if (!mbar_wait_bounded(&fullb[k % KS], (k / KS) & 1, WAIT_LIMIT))
          set_err(P.a.err, MF_ERR_TIMEOUT);
      if (!is_v)
        for (int i = ic > 2 ? ic - 2 : 0; i < ic; ++i)
          if (!mbar_wait_bounded(&bar[B_QFULL + (i & 1)], (i >> 1) & 1, WAIT_LIMIT))
            set_err(P.a.err, MF_ERR_TIMEOUT);
    }
  } else if (warp == MMA_WARP || warp == PV_WARP) {
    // ========================================================= MMA issuers
    if (lane == 0) {
      const bool is_pv = warp == PV_WARP;
      const uint32_t idesc_s = idesc_f16(BM, BN, P.in_fmt, false);
      const uint32_t idesc_o = idesc_f16(BM, D, P.in_fmt, true);
      const uint32_t tO = tmem + COL_O;
      bool ok = true;
      uint32_t g = 0;
      int ic = 0;
      for (int k = 0; ok && snake_item(k) < items; ++k, ++ic) {
        const Item I = item_at(P, prefix, order, B, snake_item(k));
        const int qb = ic & 1;
        if (!is_pv) ok = mbar_wait_bounded(&bar[B_QFULL + qb], (ic >> 1) & 1, WAIT_LIMIT);
        const uint32_t qbase = base + OFF_Q + qb * TILE_BYTES;
        for (int j = 0; ok && j < I.nt; ++j, ++g) {
          const int b2 = g & 1, st = g % KS;
          if (!is_pv) {
            // S_g = Q K_g^T once the softmax has loaded the S of tile g - 2.
            if (g >= 2)
              ok = ok && mbar_wait_bounded(&bar[B_SFREE + b2], ((g >> 1) - 1) & 1, WAIT_LIMIT);
            ok = ok && mbar_wait_bounded(&bar[B_KFULL + st], (g / KS) & 1, WAIT_LIMIT);
            if (!ok || *abort_flag) break;
            tc_fence_after();
            const uint32_t kb = base + OFF_K + st * TILE_BYTES;
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
              const uint32_t off = (ks >> 2) * HALF_BYTES + (ks & 3) * 32;
              umma_ss(tmem + COL_S + b2 * 128, sdesc_sw128(qbase + off, 16, 1024),
                      sdesc_sw128(kb + off, 16, 1024), idesc_s, ks > 0);
            }
            umma_commit(&bar[B_SDONE + b2]);
            if (j == I.nt - 1) umma_commit(&bar[B_QEMPTY + qb]);
          } else {
            // O += P_g V_g; the first P V of an item overwrites O, after the
            // previous epilogue has read it.
            ok = ok && mbar_wait_bounded(&bar[B_PFULL + b2], (g >> 1) & 1, WAIT_LIMIT);
            ok = ok && mbar_wait_bounded(&bar[B_VFULL + st], (g / KS) & 1, WAIT_LIMIT);
            if (j == 0 && ic > 0)
              ok = ok && mbar_wait_bounded(&bar[B_OFREE], (ic - 1) & 1, WAIT_LIMIT);
            if (!ok || *abort_flag) break;
            tc_fence_after();
            const uint32_t vb = base + OFF_V + st * TILE_BYTES;
#pragma unroll
            for (int ks = 0; ks < BN / 16; ++ks)
              // P columns ks*8 .. (16 keys packed 2 per column); V rows ks*16 ..
              umma_ts(tO, tmem + COL_P + b2 * 64 + ks * 8,
                      sdesc_sw128(vb + ks * 16 * 128, HALF_BYTES, 1024), idesc_o,
                      (j == 0 && ks == 0) ? 0u : 1u);
            umma_commit(&bar[B_PVDONE + b2]);
            if (j == I.nt - 1) umma_commit(&bar[B_OFULL]);
          }
        }
      }
      if (!ok) {
        set_err(P.a.err, MF_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // Every MMA either thread issued has completed before TMEM can be freed.
      umma_commit(&bar[B_IDLE]);
      if (!mbar_wait_bounded(&bar[B_IDLE], 0, WAIT_LIMIT)) set_err(P.a.err, MF_ERR_TIMEOUT);
    }
  } else {
    // ====================================== softmax (warps 0 .. SM_WARPS-1)
    // Two warps per TMEM lane quarter: the warp of parity par = warp / 4 takes
    // the tiles whose global index g has g % 2 == par (S buffer par, P buffer
    // par), so one warp's TMEM load, row max and P store overlap the other's
    // exponentials.  The online softmax is sequential only in its reference
    // max: a warp finishes its tile's row max, then takes the previous tile's
    // reference max from the other warp (mbox, B_HAND), decides its own,
    // publishes it, and only then computes the exponentials.  Each warp keeps
    // its own row sums, scaled to the reference max it last saw; at an item's
    // end the two partial sums are combined (l / ms boxes, B_EXL) and each
    // warp normalises and stores half of O's columns.
    const int quarter = warp & 3, par = warp >> 2;
    const int row = quarter * 32 + lane;  // TMEM lane == tile row
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tO = tmem + COL_O + lane_off;
    float* mbox = reinterpret_cast<float*>(gbase + OFF_XCH);  // [2][BM]
    float* lbox = mbox + 2 * BM;                               // [2 items][2][BM]
    float* msbox = lbox + 4 * BM;                              // [2 items][2][BM]
    const float sl2 = P.scale_log2;
    bool ok = true;
    // An item's epilogue runs after this warp's first tile of the next item
    // (or at the next item's end when it has none): by then the item's last
    // P V has completed and the other warp has finished the item too, so
    // neither the O wait nor the row-sum exchange stalls, and the next item's
    // first tiles run meanwhile.  Its first P V waits for O to be read.
    bool pend = false;
    int pend_ic = 0;
    bool pend_valid = false;
    T* pend_row = nullptr;
    float pend_l = 0.f, pend_m = -INFINITY;
    auto epilogue = [&]() -> bool {
      float* lb = lbox + (pend_ic & 1) * 2 * BM;
      float* mb = msbox + (pend_ic & 1) * 2 * BM;
      lb[par * BM + row] = pend_l;
      mb[par * BM + row] = pend_m;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_EXL + quarter]);
      bool done = mbar_wait_bounded(&bar[B_EXL + quarter], pend_ic & 1, WAIT_LIMIT);
      const float l_oth = lb[(par ^ 1) * BM + row], m_oth = mb[(par ^ 1) * BM + row];
      const float m_fin = fmaxf(pend_m, m_oth);
      float l_tot = 0.f;
      if (pend_m != -INFINITY) l_tot += pend_l * fast_exp2(pend_m - m_fin);
      if (m_oth != -INFINITY) l_tot += l_oth * fast_exp2(m_oth - m_fin);
      done = done && !*abort_flag && mbar_wait_bounded(&bar[B_OFULL], pend_ic & 1, WAIT_LIMIT);
      done = __all_sync(0xffffffffu, done);
      if (!done) return false;
      tc_fence_after();
      uint32_t o[64];
      tmem_ld32(tO + par * 64, o);
      tmem_ld32(tO + par * 64 + 32, o + 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_OFREE]);  // O may be overwritten
      if (pend_valid) {
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
#pragma unroll
        for (int e = 0; e < 64; e += 8) {
          uint4 v;
          v.x = Mma<T>::pack(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
          v.y = Mma<T>::pack(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
          v.z = Mma<T>::pack(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
          v.w = Mma<T>::pack(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
          *reinterpret_cast<uint4*>(pend_row + e) = v;
        }
      }
      pend = false;
      return true;
    };
    uint32_t g = 0;
    int ic = 0;
    for (int k = 0; ok && snake_item(k) < items; ++k, ++ic) {
      const Item I = item_at(P, prefix, order, B, snake_item(k));
      const int pos = I.pos0 + row / G;  // query position of this row within the sequence
      const int gg = row % G;
      const bool row_valid = row < positions_per_tile(G) * G && pos < I.q_len;
      // Last visible key: causal over the context; with a window, every pool key
      // and, in the window tile, window keys 0..pos.
      const int limit = P.window ? I.pool_len - 1 : min(I.win_start + pos, I.kv_len - 1);
      float m_seen = -INFINITY;  // reference max l_own is scaled to
      float l_own = 0.f;
      for (int j = 0; j < I.nt; ++j, ++g) {
        if ((int)(g & 1) != par) continue;  // the other warp's tile
        if (!mbar_wait_bounded(&bar[B_SDONE + par], (g >> 1) & 1, WAIT_LIMIT)) ok = false;
        // Warp-uniform decision: tcgen05.ld/st below are warp-collective.
        if (__any_sync(0xffffffffu, !ok || *abort_flag != 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[CW];
#pragma unroll
        for (int c = 0; c < CW / 32; ++c)
          tmem_ld32(tmem + COL_S + par * 128 + lane_off + c * 32,
                    reinterpret_cast<uint32_t*>(sv + c * 32));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_SFREE + par]);  // S buffer may be overwritten

        // Row max of the raw scores over the visible columns (c <= limit).
        const bool win_tile = P.window && j == I.nt - 1;
        const int lim = win_tile ? pos : limit - j * BN;
        if (__any_sync(0xffffffffu, lim < CW - 1)) {
#pragma unroll
          for (int c = 0; c < CW; ++c)
            if (c > lim) sv[c] = -INFINITY;
        }
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = sv[e];
#pragma unroll
        for (int c = 8; c < CW; c += 2) mx[(c >> 1) & 7] = fmax3f(mx[(c >> 1) & 7], sv[c], sv[c + 1]);
        const float mraw = fmax3f(fmax3f(mx[0], mx[1], mx[2]), fmax3f(mx[3], mx[4], mx[5]),
                                  fmaxf(mx[6], mx[7]));
        // The previous tile's reference max (the other warp's), unless this
        // tile starts an item.
        float m_prev = -INFINITY;
        if (g > 0) {
          if (!mbar_wait_bounded(&bar[B_HAND + quarter * 2 + (par ^ 1)], ((g - 1) >> 1) & 1,
                                 WAIT_LIMIT))
            ok = false;
          if (j > 0) m_prev = mbox[(par ^ 1) * BM + row];
        }
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        // l_own follows every rescale the other warp decided.
        if (m_prev != m_seen && m_seen != -INFINITY) l_own *= fast_exp2(m_seen - m_prev);
        // Lazy rescale: a row keeps its reference max unless this tile exceeds
        // it by more than 2^8 (log2 units).
        const float tmax = mraw * sl2;
        float m_ref = m_prev, f = 1.f;
        if (mraw != -INFINITY && (m_ref == -INFINITY || tmax > m_ref + RESCALE_THRESHOLD)) {
          if (m_ref != -INFINITY) f = fast_exp2(m_ref - tmax);
          m_ref = tmax;
        }
        l_own *= f;
        m_seen = m_ref;
        mbox[par * BM + row] = m_ref;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_HAND + quarter * 2 + par]);
        // The P buffer is free once the P V product of two tiles ago completed.
        if (g >= 2 && !mbar_wait_bounded(&bar[B_PVDONE + par], ((g >> 1) - 1) & 1, WAIT_LIMIT))
          ok = false;
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // P = 2^(s * scale_log2 - m_ref), packed to 16-bit pairs and stored 32
        // columns at a time (the scores of a stored chunk are dead, so their
        // registers hold the next chunk's P); scaling and row sums as packed
        // fp32 pairs, the exponentials on the SFU.
        const float nmu = (m_ref == -INFINITY) ? 0.f : -m_ref;
        const uint64_t sl2x2 = f32x2(sl2, sl2), nmux2 = f32x2(nmu, nmu);
        uint64_t ps2[2] = {f32x2(0.f, 0.f), f32x2(0.f, 0.f)};
        const uint32_t tp = tmem + COL_P + par * 64 + lane_off;
#pragma unroll
        for (int ch = 0; ch < CW / 32; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            float x0, x1;
            const int col = ch * 32 + 2 * c;
            f32x2_split(f32x2_fma(f32x2(sv[col], sv[col + 1]), sl2x2, nmux2), x0, x1);
            const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
            ps2[c & 1] = f32x2_add(ps2[c & 1], f32x2(p0, p1));
            pk[c] = Mma<T>::pack(p0, p1);
          }
          tmem_st16(tp + ch * 16, pk);
        }
        float ps_lo, ps_hi;
        f32x2_split(f32x2_add(ps2[0], ps2[1]), ps_lo, ps_hi);
        l_own += ps_lo + ps_hi;
        tmem_wait_st();
        if (j > 0 && __any_sync(0xffffffffu, f != 1.f)) {
          // O must include P_{g-1} V_{g-1} before it is rescaled, and the
          // rescale must land before this tile's P V (ordered by P-full below).
          // A pending epilogue goes first: P_{g-1} V_{g-1} may be this item's
          // first P V, which waits for the previous item's O to be read.
          if (pend && !epilogue()) ok = false;
          if (!mbar_wait_bounded(&bar[B_PVDONE + ((g - 1) & 1)], ((g - 1) >> 1) & 1, WAIT_LIMIT))
            ok = false;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < CW / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tmem_st32(tO + c * 32, o);
          }
          tmem_wait_st();
        }
        const int kbase = j * BN;
        // Keys of this tile past the last one loaded: past the pool in the last
        // pool tile, past q_len in the window tile (whose other rows were never
        // written by this tile's loads).
        const int loaded = win_tile ? I.q_len : I.pool_len - kbase;
        if (quarter == 0 && loaded < BN) {
          // Zero the V rows of those keys (whole 128-byte rows of both halves)
          // so p = 0 adds nothing even where a slot holds NaN.  This warp's
          // P-full arrival orders it before P V.
          const int st = g % KS;
          if (!mbar_wait_bounded(&bar[B_VFULL + st], (g / KS) & 1, WAIT_LIMIT)) ok = false;
          const uint32_t vb = base + OFF_V + st * TILE_BYTES;
          const int first = max(0, loaded);
          for (int idx = lane; idx < (BN - first) * 16; idx += 32) {
            const int r = first + idx / 16, c16 = idx % 16;
            const uint32_t a = vb + (c16 >> 3) * HALF_BYTES + r * 128 + (c16 & 7) * 16;
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
          }
          fence_proxy_async_smem();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[B_PFULL + par]);
        if (pend && !epilogue()) {
          ok = false;
          break;
        }
      }
      // Uniform: the epilogue below is warp-collective.
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      if (pend && !epilogue()) {  // no tile of this item was this warp's
        ok = false;
        break;
      }
      pend = true;
      pend_ic = ic;
      pend_valid = row_valid;
      pend_row = static_cast<T*>(P.a.out) + (int64_t)(I.q_start + (row_valid ? pos : 0)) * P.a.o_sr +
                 (int64_t)(I.h * G + gg) * P.a.o_sh + par * 64;
      pend_l = l_own;
      pend_m = m_seen;
    }
    if (ok && pend && !epilogue()) ok = false;
    if (!ok) {
      if (lane == 0) set_err(P.a.err, MF_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  // ---------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace pf

// ----------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn() {
  static EncodeTiledFn2 fn = []() -> EncodeTiledFn2 {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn2>(ptr);
  }();
  return fn;
}

// 4-D view (64 elements, dim1, 2 halves of 64, dim3) with byte strides
// (s1, 128, s3) and box (64, b1, 1, b3), 128-byte swizzle.
static CUresult encode_pf(CUtensorMap* m, const void* base, uint64_t n1, uint64_t s1,
                          uint64_t n3, uint64_t s3, uint32_t b1, uint32_t b3,
                          CUtensorMapDataType dt) {
  EncodeTiledFn2 fn = encode_fn();
  if (!fn) return CUDA_ERROR_NOT_SUPPORTED;
  cuuint64_t dims[4] = {64, n1, 2, n3};
  cuuint64_t strides[3] = {s1, 128, s3};
  cuuint32_t box[4] = {64, b1, 1, b3};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

const char* prefill_tc_unsupported(const AttnParams& p, mf_dtype dtype) {
  if (dtype != MF_BF16 && dtype != MF_F16) return "dtype is not bf16/f16";
  if (p.d != pf::D) return "head_dim is not 128";
  if (p.block_size != pf::PAGE) return "block_size is not 16";
  if (p.sb != (int64_t)pf::PAGE * p.ss) return "pool blocks are not slot-contiguous";
  if ((p.ss * 2) % 16 || (p.sh * 2) % 16) return "pool strides not 16-byte multiples";
  if ((reinterpret_cast<uintptr_t>(p.kp) | reinterpret_cast<uintptr_t>(p.vp) |
       reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.out)) & 15)
    return "q/out/pool not 16-byte aligned";
  if ((p.q_sr * 2) % 16 || (p.q_sh * 2) % 16 || (p.o_sr * 2) % 16 || (p.o_sh * 2) % 16)
    return "q/out strides not 16-byte multiples";
  const int G = p.hq / p.hkv;
  if (G < 1 || G > 16) return "GQA group above 16";
  if (p.row_map) return "row_map";
  if (p.wk) {
    if (p.max_q_len > pf::PAGE) return "window longer than 16 rows";
    if ((p.w_sr * 2) % 16 || (p.w_sh * 2) % 16) return "window strides not 16-byte multiples";
    if ((reinterpret_cast<uintptr_t>(p.wk) | reinterpret_cast<uintptr_t>(p.wv)) & 15)
      return "window not 16-byte aligned";
  }
  if (p.num_seqs > pf::MAX_SEQS) return "more than 4096 sequences";
  if (!p.causal) return "non-causal";
  if ((int64_t)p.num_blocks * pf::PAGE > 0x7fffffffLL) return "pool slots exceed int32";
  return nullptr;
}

int launch_attn_prefill_tc(const AttnParams& p, mf_dtype dtype, int rows_cap,
                           cudaStream_t stream) {
  const CUtensorMapDataType dt =
      dtype == MF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int G = p.hq / p.hkv;
  CUtensorMap mq, mk, mv, mwk, mwv;
  const uint64_t slots = (uint64_t)p.num_blocks * pf::PAGE;
  const int ppt = pf::positions_per_tile(G);
  // q: (64, heads, halves, rows), box (64, G heads, 1, floor(128/G) positions)
  CUresult r0 = encode_pf(&mq, p.q, (uint64_t)p.hq, (uint64_t)p.q_sh * 2, (uint64_t)p.total_q,
                          (uint64_t)p.q_sr * 2, (uint32_t)G, (uint32_t)ppt, dt);
  // pool: (64, slots, halves, kv heads), box (64, 16 tokens, 1, 1 head)
  CUresult r1 = encode_pf(&mk, p.kp, slots, (uint64_t)p.ss * 2, (uint64_t)p.hkv,
                          (uint64_t)p.sh * 2, pf::PAGE, 1, dt);
  CUresult r2 = encode_pf(&mv, p.vp, slots, (uint64_t)p.ss * 2, (uint64_t)p.hkv,
                          (uint64_t)p.sh * 2, pf::PAGE, 1, dt);
  // window: (64, rows, halves, kv heads), box (64, 16 rows, 1, 1 head)
  CUresult r3 = CUDA_SUCCESS, r4 = CUDA_SUCCESS;
  if (p.wk) {
    r3 = encode_pf(&mwk, p.wk, (uint64_t)p.total_q, (uint64_t)p.w_sr * 2, (uint64_t)p.hkv,
                   (uint64_t)p.w_sh * 2, pf::PAGE, 1, dt);
    r4 = encode_pf(&mwv, p.wv, (uint64_t)p.total_q, (uint64_t)p.w_sr * 2, (uint64_t)p.hkv,
                   (uint64_t)p.w_sh * 2, pf::PAGE, 1, dt);
  } else {
    mwk = mk;
    mwv = mv;
  }
  if (r0 != CUDA_SUCCESS || r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS || r3 != CUDA_SUCCESS ||
      r4 != CUDA_SUCCESS)
    return fail(MF_ECUDA, "prefill: tensor map encoding failed");
  pf::Params P;
  P.a = p;
  P.G = G;
  P.rows_cap = rows_cap;
  P.scale_log2 = p.scale * 1.4426950408889634f;
  P.in_fmt = dtype == MF_BF16 ? 1u : 0u;
  P.window = p.wk ? 1 : 0;
  // Persistent grid: one CTA per SM, or fewer when there are fewer items
  // (num_seqs x query tiles of the longest run x kv heads bounds the count).
  const int64_t q_tiles = ((int64_t)p.max_q_len + ppt - 1) / ppt;
  const int64_t items_max = (int64_t)p.num_seqs * q_tiles * p.hkv;
  if (items_max == 0) return MF_OK;
  const int64_t grid = std::min<int64_t>(items_max, current_sm_count());
  auto kern = dtype == MF_BF16 ? pf::prefill_kernel<__nv_bfloat16> : pf::prefill_kernel<__half>;
  const size_t smem = pf::smem_bytes(p.num_seqs) + 1024;
  static thread_local int configured_dev[2] = {-1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  const int which = dtype == MF_BF16 ? 1 : 0;
  if (configured_dev[which] != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(pf::smem_bytes(pf::MAX_SEQS) + 1024));
    if (e != cudaSuccess) return fail(MF_ECUDA, std::string("prefill: ") + cudaGetErrorString(e));
    configured_dev[which] = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(pf::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, mwk, mwv, P);
  if (le != cudaSuccess)
    return fail(MF_ECUDA, std::string("prefill: ") + cudaGetErrorString(le));
  return check_launch("paged attention (tcgen05 prefill)");
}

}  // namespace mf
