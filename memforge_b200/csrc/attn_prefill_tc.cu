// Paged chunked-prefill attention on the sm_100a tensor cores (tcgen05 + TMEM).
//
// One CTA computes one 128-row query tile of one sequence for one kv head.
// The 128 rows are (query position, query head of the GQA group) pairs, so
// each K/V tile is loaded once for every query head sharing the kv head.
//
//   warps 0-3  softmax / correction / epilogue: thread t owns TMEM lane t (row t)
//   warp 4     TMA producer: Q once, then per 128-key tile 8 pages x 2 halves of
//              K and of V (4-D tiled loads from the pool, 128-byte swizzled)
//   warp 5     MMA issuer (one thread): S = Q K^T into TMEM (two S buffers), and
//              O += P V with P read back from TMEM as the A operand
//
// The online softmax keeps a per-row reference max and only rescales O (a TMEM
// read-modify-write) when a tile's max exceeds it by more than 2^8, so the
// exponentials stay <= 256 and the correction is rare after the first tiles.
// Masking: key k is visible to row r iff k < kv_len and k <= kv_len - q_len +
// position(r) (causal) — the varlen rule of memforge_ml/kernels/
// varlen_attention.py:193-201.  Pages past the block table load as zeros
// (out-of-range TMA coordinates) and unwritten slots of the last page are
// zeroed in shared memory before the P V product.
//
// Every mbarrier wait is bounded; on expiry the CTA raises MF_ERR_TIMEOUT, drains
// its TMA loads and MMAs, frees its TMEM and returns.

#include "mf_attn.h"

namespace mf {
namespace pf {

constexpr int THREADS = 192;
constexpr int BM = 128;
constexpr int BN = 128;
constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int STAGES = 2;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint64_t WAIT_LIMIT = 2000000000ull;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

constexpr uint32_t TILE_BYTES = BN * D * 2;   // 32 KB: [half][128 rows][128 B]
constexpr uint32_t HALF_BYTES = BN * 128;     // 16 KB
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + TILE_BYTES;
constexpr uint32_t OFF_V = OFF_K + STAGES * TILE_BYTES;
constexpr uint32_t OFF_BAR = OFF_V + STAGES * TILE_BYTES;
// barriers: q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2],
// s_free[2], p_full[2], o_done, mma_idle
constexpr int NBAR = 1 + 4 * STAGES + 6 + 2;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 64;

struct Params {
  AttnParams a;
  int G;
  int rows_cap;      // sequences with q_len * G <= rows_cap belong to the decode kernel
  int q_tiles;       // grid.x = num_seqs * q_tiles
  float scale_log2;
  uint32_t in_fmt;   // 0 = f16, 1 = bf16
};

struct Bars {
  uint64_t* base;
  MF_DEVINL uint64_t* q_full() const { return base; }
  MF_DEVINL uint64_t* k_full(int s) const { return base + 1 + s; }
  MF_DEVINL uint64_t* k_empty(int s) const { return base + 1 + STAGES + s; }
  MF_DEVINL uint64_t* v_full(int s) const { return base + 1 + 2 * STAGES + s; }
  MF_DEVINL uint64_t* v_empty(int s) const { return base + 1 + 3 * STAGES + s; }
  MF_DEVINL uint64_t* s_full(int b) const { return base + 1 + 4 * STAGES + b; }
  MF_DEVINL uint64_t* s_free(int b) const { return base + 3 + 4 * STAGES + b; }
  MF_DEVINL uint64_t* p_full(int b) const { return base + 5 + 4 * STAGES + b; }
  MF_DEVINL uint64_t* o_done() const { return base + 7 + 4 * STAGES; }
  MF_DEVINL uint64_t* mma_idle() const { return base + 8 + 4 * STAGES; }
};

template <typename T>
__global__ void __launch_bounds__(THREADS, 1) prefill_kernel(
    const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
    const __grid_constant__ CUtensorMap tmv, const __grid_constant__ Params P) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);
  Bars bars{reinterpret_cast<uint64_t*>(gbase + OFF_BAR)};
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_MISC + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s = blockIdx.x / P.q_tiles;
  const int qt = blockIdx.x % P.q_tiles;
  const int h = blockIdx.y;  // kv head
  const int G = P.G;
  const int ppt = BM / G;    // query positions per tile

  int q_start, q_len;
  seq_rows(P.a, s, q_start, q_len);
  const int kv_len = P.a.kv_lens[s];
  // Whole-CTA early exits (uniform): short sequences belong to the decode kernel.
  if (q_len <= 0 || q_len * G <= P.rows_cap || qt * ppt >= q_len) return;
  if (kv_len < q_len) {
    if (tid == 0 && qt == 0 && h == 0) set_err(P.a.err, MF_ERR_LENGTH);
    return;
  }
  const int win_start = kv_len - q_len;
  const int pos0 = qt * ppt;
  const int pos_last = min(q_len - 1, pos0 + ppt - 1);
  const int key_end = win_start + pos_last + 1;            // keys this tile can see
  const int ntiles = (key_end + BN - 1) / BN;
  const int pool_pages = (kv_len + PAGE - 1) / PAGE;
  if (pool_pages > P.a.table_stride) {
    if (tid == 0) set_err(P.a.err, MF_ERR_TABLE);
    return;
  }

  // ------------------------------------------------------------- set-up
  if (tid == 0) {
    mbar_init(bars.q_full(), 1);
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(bars.k_full(st), 1);
      mbar_init(bars.k_empty(st), 1);
      mbar_init(bars.v_full(st), 1);
      mbar_init(bars.v_empty(st), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bars.s_full(b), 1);
      mbar_init(bars.s_free(b), 1);
      mbar_init(bars.p_full(b), 4);
    }
    mbar_init(bars.o_done(), 1);
    mbar_init(bars.mma_idle(), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};  // S / P buffers (columns)
  const uint32_t tO = tmem + 256;             // O accumulator (128 fp32 columns)

  if (warp == 4) {
    // ======================================================== TMA producer
    if (lane == 0) {
      const uint64_t pol_once = l2_evict_first_policy();
      const uint64_t pol_keep = l2_evict_last_policy();
      prefetch_tmap(&tmq);
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
      mbar_arrive_expect_tx(bars.q_full(), TILE_BYTES);
      for (int half = 0; half < 2; ++half)
        tma_load_4d(gbase + OFF_Q + half * HALF_BYTES, &tmq, bars.q_full(), 0, h * G, half,
                    q_start + pos0, pol_once);
      const int nb = P.a.num_blocks;
      const int32_t* table = P.a.tables + (int64_t)s * P.a.table_stride;
      int armed = 0, armed_k = 0;  // tiles whose V (K) loads were issued
      for (int j = 0; j < ntiles && !*abort_flag; ++j) {
        const int st = j % STAGES;
        const uint32_t ph = ((j / STAGES) - 1) & 1;
        for (int kv = 0; kv < 2; ++kv) {
          uint64_t* empty = kv ? bars.v_empty(st) : bars.k_empty(st);
          uint64_t* full = kv ? bars.v_full(st) : bars.k_full(st);
          if (j >= STAGES && !mbar_wait_bounded(empty, ph, WAIT_LIMIT)) {
            set_err(P.a.err, MF_ERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(full, TILE_BYTES);
          uint8_t* dst = gbase + (kv ? OFF_V : OFF_K) + st * TILE_BYTES;
          for (int pg = 0; pg < BN / PAGE; ++pg) {
            const int L = j * (BN / PAGE) + pg;
            int tok = nb * PAGE;  // out of range: TMA fills zeros
            if (L < pool_pages) {
              const int blk = __ldg(table + L);
              if (blk >= 0 && blk < nb) tok = blk * PAGE;
              else set_err(P.a.err, MF_ERR_BLOCK_ID);
            }
            for (int half = 0; half < 2; ++half)
              tma_load_4d(dst + half * HALF_BYTES + pg * PAGE * 128, kv ? &tmv : &tmk, full, 0,
                          tok, half, h, pol_keep);
          }
          if (kv == 0) armed_k = j + 1;
          else armed = j + 1;
        }
        if (*abort_flag) break;
      }
      // Drain every armed load before the CTA can exit.
      for (int j = max(0, armed_k - STAGES); j < armed_k; ++j)
        if (!mbar_wait_bounded(bars.k_full(j % STAGES), (j / STAGES) & 1, WAIT_LIMIT))
          set_err(P.a.err, MF_ERR_TIMEOUT);
      for (int j = max(0, armed - STAGES); j < armed; ++j)
        if (!mbar_wait_bounded(bars.v_full(j % STAGES), (j / STAGES) & 1, WAIT_LIMIT))
          set_err(P.a.err, MF_ERR_TIMEOUT);
      mbar_wait_bounded(bars.q_full(), 0, WAIT_LIMIT);
    }
  } else if (warp == 5) {
    // ========================================================= MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = idesc_f16(BM, BN, P.in_fmt, false);
      const uint32_t idesc_o = idesc_f16(BM, D, P.in_fmt, true);
      bool ok = mbar_wait_bounded(bars.q_full(), 0, WAIT_LIMIT);
      tc_fence_after();
      for (int j = 0; ok && j < ntiles + 1; ++j) {
        // S_j = Q K_j^T  (issued one tile ahead of P_{j-1} V_{j-1})
        if (j < ntiles) {
          const int st = j % STAGES, b = j & 1;
          if (j >= 2) ok = ok && mbar_wait_bounded(bars.s_free(b), ((j >> 1) - 1) & 1, WAIT_LIMIT);
          ok = ok && mbar_wait_bounded(bars.k_full(st), (j / STAGES) & 1, WAIT_LIMIT);
          if (!ok || *abort_flag) break;
          tc_fence_after();
          const uint32_t qb = base + OFF_Q, kb = base + OFF_K + st * TILE_BYTES;
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * HALF_BYTES + (ks & 3) * 32;
            umma_ss(tS[b], sdesc_sw128(qb + off, 16, 1024), sdesc_sw128(kb + off, 16, 1024),
                    idesc_s, ks > 0);
          }
          umma_commit(bars.k_empty(st));
          umma_commit(bars.s_full(b));
        }
        // O += P_{j-1} V_{j-1}
        if (j >= 1) {
          const int jj = j - 1, st = jj % STAGES, b = jj & 1;
          ok = ok && mbar_wait_bounded(bars.p_full(b), (jj >> 1) & 1, WAIT_LIMIT);
          ok = ok && mbar_wait_bounded(bars.v_full(st), (jj / STAGES) & 1, WAIT_LIMIT);
          if (!ok || *abort_flag) break;
          tc_fence_after();
          const uint32_t vb = base + OFF_V + st * TILE_BYTES;
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks) {
            // P columns ks*8 .. (16 bf16 keys packed 2 per column); V rows ks*16 ..
            umma_ts(tO, tS[b] + ks * 8, sdesc_sw128(vb + ks * 16 * 128, HALF_BYTES, 1024),
                    idesc_o, (jj > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(bars.v_empty(st));
          umma_commit(bars.s_free(b));
          umma_commit(bars.o_done());
        }
      }
      if (!ok) {
        set_err(P.a.err, MF_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // Every MMA issued above has completed before TMEM can be freed.
      umma_commit(bars.mma_idle());
      if (!mbar_wait_bounded(bars.mma_idle(), 0, WAIT_LIMIT)) set_err(P.a.err, MF_ERR_TIMEOUT);
    }
  } else {
    // ================================================ softmax (warps 0-3)
    const int row = tid;  // TMEM lane == tile row
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const int pos = pos0 + row / G;  // query position of this row within the sequence
    const int g = row % G;
    const int limit = win_start + pos;  // last visible key (causal)
    const float sl2 = P.scale_log2;
    float m_ref = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int b = j & 1;
      if (!mbar_wait_bounded(bars.s_full(b), (j >> 1) & 1, WAIT_LIMIT)) {
        ok = false;
      }
      // Warp-uniform decision: tcgen05.ld/st below are warp-collective.
      if (__any_sync(0xffffffffu, !ok || *abort_flag != 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS[b] + lane_off + c * 32,
                                                  reinterpret_cast<uint32_t*>(sv + c * 32));
      tmem_wait_ld();
      const int kbase = j * BN;
      const bool full_tile = kbase + BN - 1 <= win_start + pos0 && kbase + BN <= kv_len;
      float tmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        float x = sv[c] * sl2;
        if (!full_tile && (kbase + c > limit || kbase + c >= kv_len)) x = -INFINITY;
        sv[c] = x;
        tmax = fmaxf(tmax, x);
      }
      // Lazy rescale: a row keeps its reference max unless this tile exceeds it
      // by more than 2^8.  The O correction is a warp-collective TMEM
      // read-modify-write, done when any row of the warp needs it (the other
      // rows multiply by 1).
      float f = 1.f;
      if (tmax != -INFINITY && (m_ref == -INFINITY || tmax > m_ref + RESCALE_THRESHOLD)) {
        if (m_ref != -INFINITY) f = fast_exp2(m_ref - tmax);
        m_ref = tmax;
      }
      l_sum *= f;
      if (j > 0 && __any_sync(0xffffffffu, f != 1.f)) {
        // O must include P_{j-1} V_{j-1} before it is rescaled.
        if (!mbar_wait_bounded(bars.o_done(), (j - 1) & 1, WAIT_LIMIT)) ok = false;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + lane_off + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(tO + lane_off + c * 32, o);
        }
      }
      const float mu = (m_ref == -INFINITY) ? 0.f : m_ref;
      uint32_t pk[BN / 2];
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < BN / 2; ++c) {
        const float p0 = fast_exp2(sv[2 * c] - mu), p1 = fast_exp2(sv[2 * c + 1] - mu);
        psum += p0 + p1;
        pk[c] = Mma<T>::pack(p0, p1);
      }
      l_sum += psum;
      // P overwrites the first 64 columns of this S buffer (own lane only).
      tmem_st32(tS[b] + lane_off, pk);
      tmem_st32(tS[b] + lane_off + 32, pk + 32);
      tmem_wait_st();
      if (warp == 0 && kbase + BN > kv_len) {
        // Last tile: zero the V rows of keys past the context (whole 128-byte
        // rows of both halves) so p = 0 adds nothing even where an unwritten
        // slot holds NaN.  Warp 0's p_full arrival orders it before P V.
        const int st = j % STAGES;
        if (!mbar_wait_bounded(bars.v_full(st), (j / STAGES) & 1, WAIT_LIMIT)) ok = false;
        const uint32_t vb = base + OFF_V + st * TILE_BYTES;
        const int first = max(0, kv_len - kbase);
        for (int idx = lane; idx < (BN - first) * 16; idx += 32) {
          const int r = first + idx / 16, c16 = idx % 16;
          const uint32_t a = vb + (c16 >> 3) * HALF_BYTES + r * 128 + (c16 & 7) * 16;
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.p_full(b));
    }
    // ---------------------------------------------------------- epilogue
    bool done = ok && !*abort_flag && mbar_wait_bounded(bars.o_done(), (ntiles - 1) & 1, WAIT_LIMIT);
    done = __all_sync(0xffffffffu, done);
    if (done) {
      tc_fence_after();
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      const bool valid = pos < q_len;
      T* orow = static_cast<T*>(P.a.out) + (int64_t)(q_start + pos) * P.a.o_sr +
                (int64_t)(h * G + g) * P.a.o_sh;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + lane_off + c * 32, o);
        tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 v;
            v.x = Mma<T>::pack(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
            v.y = Mma<T>::pack(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            v.z = Mma<T>::pack(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
            v.w = Mma<T>::pack(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + e) = v;
          }
        }
      }
    } else {
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
  if (G > 8 || pf::BM % G) return "GQA group does not divide 128";
  if (p.wk || p.row_map) return "window / row_map";
  if (!p.causal) return "non-causal";
  if ((int64_t)p.num_blocks * pf::PAGE > 0x7fffffffLL) return "pool slots exceed int32";
  return nullptr;
}

int launch_attn_prefill_tc(const AttnParams& p, mf_dtype dtype, int rows_cap,
                           cudaStream_t stream) {
  const CUtensorMapDataType dt =
      dtype == MF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int G = p.hq / p.hkv;
  CUtensorMap mq, mk, mv;
  const uint64_t slots = (uint64_t)p.num_blocks * pf::PAGE;
  // q: (64, heads, halves, rows), box (64, G heads, 1, 128/G positions)
  CUresult r0 = encode_pf(&mq, p.q, (uint64_t)p.hq, (uint64_t)p.q_sh * 2, (uint64_t)p.total_q,
                          (uint64_t)p.q_sr * 2, (uint32_t)G, (uint32_t)(pf::BM / G), dt);
  // pool: (64, slots, halves, kv heads), box (64, 16 tokens, 1, 1 head)
  CUresult r1 = encode_pf(&mk, p.kp, slots, (uint64_t)p.ss * 2, (uint64_t)p.hkv,
                          (uint64_t)p.sh * 2, pf::PAGE, 1, dt);
  CUresult r2 = encode_pf(&mv, p.vp, slots, (uint64_t)p.ss * 2, (uint64_t)p.hkv,
                          (uint64_t)p.sh * 2, pf::PAGE, 1, dt);
  if (r0 != CUDA_SUCCESS || r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS)
    return fail(MF_ECUDA, "prefill: tensor map encoding failed");
  pf::Params P;
  P.a = p;
  P.G = G;
  P.rows_cap = rows_cap;
  P.q_tiles = (p.max_q_len * G + pf::BM - 1) / pf::BM;
  P.scale_log2 = p.scale * 1.4426950408889634f;
  P.in_fmt = dtype == MF_BF16 ? 1u : 0u;
  const int64_t gx = (int64_t)p.num_seqs * P.q_tiles;
  if (gx == 0) return MF_OK;
  if (gx > 0x7fffffff || p.hkv > 65535) return fail(MF_EINVAL, "prefill: grid too large");
  auto kern = dtype == MF_BF16 ? pf::prefill_kernel<__nv_bfloat16> : pf::prefill_kernel<__half>;
  const size_t smem = pf::SMEM_BYTES + 1024;
  static thread_local int configured_dev[2] = {-1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  const int which = dtype == MF_BF16 ? 1 : 0;
  if (configured_dev[which] != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return fail(MF_ECUDA, std::string("prefill: ") + cudaGetErrorString(e));
    configured_dev[which] = dev;
  }
  kern<<<dim3((unsigned)gx, p.hkv), pf::THREADS, smem, stream>>>(mq, mk, mv, P);
  return check_launch("paged attention (tcgen05 prefill)");
}

}  // namespace mf
