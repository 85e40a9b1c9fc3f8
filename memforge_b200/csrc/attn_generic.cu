// Generic paged attention on CUDA cores, fp32 arithmetic throughout.
//
// Serves every shape the tensor-core decode kernel does not: fp32 pools (there
// is no fp32 tensor-core path that keeps 1e-5 parity), head_dim other than
// 64/128, block sizes other than 16, arbitrary pool strides (the standalone
// operator's (blocks, heads, block_size, dim) cache) and long query runs until
// the prefill kernel takes them.  It is a GPU kernel, not a CPU fallback.
//
// One CTA = (sequence, kv head, tile of up to 32 query rows).  Rows are the
// (query position, query head in the GQA group) pairs of that kv head; the
// CTA stages 32 keys at a time in shared memory as fp32 and every warp runs the
// online softmax (block_attention.py:30-40 identity) for the rows it owns,
// lanes over keys for the scores and lanes over head_dim for the accumulator.

#include "mf_attn.h"

namespace mf {

constexpr int GEN_WARPS = 4;
constexpr int GEN_ROWS = 32;   // query rows per CTA
constexpr int GEN_TILE = 32;   // keys per shared-memory tile
constexpr int GEN_RPW = GEN_ROWS / GEN_WARPS;

template <typename T, int DMAX>
__global__ void __launch_bounds__(GEN_WARPS * 32)
    attn_generic_kernel(AttnParams p, int row_tiles) {
  constexpr int CPL = DMAX / 32;  // accumulator columns per lane
  const int D = p.d;
  const int G = p.hq / p.hkv;
  const int s = blockIdx.x / row_tiles;
  const int rt = blockIdx.x % row_tiles;
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  int q_start, q_len;
  seq_rows(p, s, q_start, q_len);
  const int nrows = q_len * G;
  const int r0 = rt * GEN_ROWS;
  if (r0 >= nrows) return;
  const int r1 = min(nrows, r0 + GEN_ROWS);
  const int kv_len = p.kv_lens[s];
  const T* q = static_cast<const T*>(p.q);
  T* out = static_cast<T*>(p.out);

  if (kv_len < q_len || kv_len <= 0) {
    // No visible key for some row: the reference raises (varlen_attention.py:
    // 228-232); here the rows are zeroed and the error word says why.
    if (tid == 0) set_err(p.err, MF_ERR_LENGTH);
    for (int idx = tid; idx < (r1 - r0) * D; idx += blockDim.x) {
      const int r = r0 + idx / D, d = idx % D;
      const int prow = map_row(p, q_start + r / G);
      out[prow * p.o_sr + (int64_t)(h * G + r % G) * p.o_sh + d] = from_f32<T>(0.f);
    }
    return;
  }
  const int win_start = kv_len - q_len;
  const int last_i = (r1 - 1) / G;
  const int key_end = (p.causal ? win_start + last_i : kv_len - 1) + 1;

  extern __shared__ float gsm[];
  float* sq = gsm;                             // [GEN_ROWS][D]
  float* sk = sq + GEN_ROWS * D;               // [GEN_TILE][D+1]
  float* sv = sk + GEN_TILE * (D + 1);         // [GEN_TILE][D+1]
  int64_t* sbase = reinterpret_cast<int64_t*>(sv + GEN_TILE * (D + 1));  // [GEN_TILE]

  for (int idx = tid; idx < (r1 - r0) * D; idx += blockDim.x) {
    const int r = r0 + idx / D, d = idx % D;
    const int prow = map_row(p, q_start + r / G);
    sq[(r - r0) * D + d] = Elt<T>::to_f32(q[prow * p.q_sr + (int64_t)(h * G + r % G) * p.q_sh + d]);
  }

  float m[GEN_RPW], l[GEN_RPW], acc[GEN_RPW][CPL];
#pragma unroll
  for (int k = 0; k < GEN_RPW; ++k) {
    m[k] = -INFINITY;
    l[k] = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[k][c] = 0.f;
  }

  const T* kp = static_cast<const T*>(p.kp);
  const T* vp = static_cast<const T*>(p.vp);
  const T* wk = static_cast<const T*>(p.wk);
  const T* wv = static_cast<const T*>(p.wv);
  const float scale = p.scale;

  for (int t0 = 0; t0 < key_end; t0 += GEN_TILE) {
    // Resolve each key of the tile to an element offset: >= 0 pool offset,
    // -2 - row for a window row, -1 for nothing (past the range / bad id).
    if (tid < GEN_TILE) {
      const int kpos = t0 + tid;
      int64_t off = -1;
      if (kpos < key_end) {
        if (wk && kpos >= win_start) {
          off = -2 - (int64_t)map_row(p, q_start + (kpos - win_start));
        } else {
          const int lb = kpos / p.block_size;
          if (lb >= p.table_stride) {
            set_err(p.err, MF_ERR_TABLE);
          } else {
            const int blk = p.tables[(int64_t)s * p.table_stride + lb];
            if (blk < 0 || blk >= p.num_blocks) {
              set_err(p.err, MF_ERR_BLOCK_ID);
            } else {
              off = (int64_t)blk * p.sb + (int64_t)(kpos % p.block_size) * p.ss + (int64_t)h * p.sh;
            }
          }
        }
      }
      sbase[tid] = off;
    }
    __syncthreads();
    for (int idx = tid; idx < GEN_TILE * D; idx += blockDim.x) {
      const int j = idx / D, d = idx % D;
      const int64_t off = sbase[j];
      float kv = 0.f, vv = 0.f;
      if (off >= 0) {
        kv = Elt<T>::to_f32(kp[off + d]);
        vv = Elt<T>::to_f32(vp[off + d]);
      } else if (off <= -2) {
        const int64_t row = -2 - off;
        kv = Elt<T>::to_f32(wk[row * p.w_sr + (int64_t)h * p.w_sh + d]);
        vv = Elt<T>::to_f32(wv[row * p.w_sr + (int64_t)h * p.w_sh + d]);
      }
      sk[j * (D + 1) + d] = kv;
      sv[j * (D + 1) + d] = vv;
    }
    __syncthreads();

#pragma unroll
    for (int k = 0; k < GEN_RPW; ++k) {
      const int rr = warp + GEN_WARPS * k;
      const int r = r0 + rr;
      if (r >= r1) continue;
      const int i = r / G;
      const int limit = p.causal ? win_start + i : kv_len - 1;
      const int kpos = t0 + lane;
      float sc = -INFINITY;
      if (kpos <= limit) {
        float dot = 0.f;
        const float* qr = sq + rr * D;
        const float* kr = sk + lane * (D + 1);
        for (int d = 0; d < D; ++d) dot = fmaf(qr[d], kr[d], dot);
        sc = dot * scale;
      }
      float tmax = sc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float m_new = fmaxf(m[k], tmax);
      if (m_new == -INFINITY) continue;  // nothing visible yet (cannot happen past tile 0)
      const float alpha = (m[k] == -INFINITY) ? 0.f : expf(m[k] - m_new);
      const float pj = (kpos <= limit) ? expf(sc - m_new) : 0.f;
      float psum = pj;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      l[k] = l[k] * alpha + psum;
#pragma unroll
      for (int c = 0; c < CPL; ++c) acc[k][c] *= alpha;
      const int nvis = min(GEN_TILE, limit - t0 + 1);
      for (int j = 0; j < nvis; ++j) {
        const float pb = __shfl_sync(0xffffffffu, pj, j);
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          const int d = lane + 32 * c;
          if (d < D) acc[k][c] = fmaf(pb, sv[j * (D + 1) + d], acc[k][c]);
        }
      }
      m[k] = m_new;
    }
    __syncthreads();
  }

#pragma unroll
  for (int k = 0; k < GEN_RPW; ++k) {
    const int r = r0 + warp + GEN_WARPS * k;
    if (r >= r1) continue;
    const int prow = map_row(p, q_start + r / G);
    const float inv = l[k] > 0.f ? 1.f / l[k] : 0.f;
    T* o = out + prow * p.o_sr + (int64_t)(h * G + r % G) * p.o_sh;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      const int d = lane + 32 * c;
      if (d < D) o[d] = from_f32<T>(acc[k][c] * inv);
    }
  }
}

template <typename T, int DMAX>
static int launch_gen(const AttnParams& p, cudaStream_t stream) {
  const int G = p.hq / p.hkv;
  const int row_tiles = (p.max_q_len * G + GEN_ROWS - 1) / GEN_ROWS;
  const int64_t gx = (int64_t)p.num_seqs * row_tiles;
  if (gx == 0) return MF_OK;
  if (gx > 0x7fffffff) return fail(MF_EINVAL, "generic attention: grid too large");
  const size_t smem = (size_t)(GEN_ROWS * p.d + 2 * GEN_TILE * (p.d + 1)) * sizeof(float) +
                      GEN_TILE * sizeof(int64_t);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(attn_generic_kernel<T, DMAX>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(MF_ECUDA, std::string("generic attention: ") + cudaGetErrorString(e));
  }
  attn_generic_kernel<T, DMAX><<<dim3((unsigned)gx, p.hkv), GEN_WARPS * 32, smem, stream>>>(p, row_tiles);
  return check_launch("paged attention (generic)");
}

template <typename T>
static int launch_gen_d(const AttnParams& p, cudaStream_t stream) {
  if (p.d <= 64) return launch_gen<T, 64>(p, stream);
  if (p.d <= 128) return launch_gen<T, 128>(p, stream);
  if (p.d <= 256) return launch_gen<T, 256>(p, stream);
  return fail(MF_EUNSUPPORTED, "paged attention: head_dim above 256");
}

int launch_attn_generic(const AttnParams& p, mf_dtype dtype, cudaStream_t stream) {
  switch (dtype) {
    case MF_F32: return launch_gen_d<float>(p, stream);
    case MF_F16: return launch_gen_d<__half>(p, stream);
    case MF_BF16: return launch_gen_d<__nv_bfloat16>(p, stream);
  }
  return fail(MF_EINVAL, "paged attention: unknown dtype");
}

}  // namespace mf
