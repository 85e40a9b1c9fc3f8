// mf_paged_decode_noalloc: the Triton-signature paged decode for callers that
// cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits — a host whose
// device memory is owned by another allocator it must not bypass (a caching
// pool that would otherwise see foreign allocations), a call made from inside
// a region that forbids allocation, or a plugin whose host application hands
// it only the input and output buffers.  mf_paged_decode needs a split-K
// workspace from its caller; this variant uses a fixed device array that lives
// in the library instead, so the caller supplies nothing but inputs and outputs.
//
// The array is a file-scope __device__ object of MF_NOALLOC_SCRATCH_BYTES; every
// GPU that loads the library holds it until the process exits.  Host code may
// not use the array's name as a device address: the first call on each device
// asks the runtime for its device address (cudaGetSymbolAddress, with that
// device current) and caches it.  Calls whose split-K plan needs more scratch
// than the array holds are rejected with MF_EWORKSPACE.

#include <mutex>
#include <vector>

#include "mf_attn.h"

namespace {

constexpr size_t kScratchBytes = MF_NOALLOC_SCRATCH_BYTES;

// Arrival counters at the front (they must start at zero), partial slots after.
__device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
std::vector<void*> g_addr;  // per device, nullptr until resolved

// Device address of the scratch array on the current device (resolved once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return mf::fail(MF_ECUDA, std::string("noalloc decode: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_mu);
  if ((int)g_addr.size() <= dev) g_addr.resize(dev + 1, nullptr);
  if (!g_addr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return mf::fail(MF_ECUDA, std::string("noalloc decode: cannot resolve the scratch array: ") +
                                    cudaGetErrorString(e));
    g_addr[dev] = ptr;
  }
  *out = g_addr[dev];
  return MF_OK;
}

}  // namespace

extern "C" int mf_paged_decode_noalloc(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                       const void* key_flat, const void* value_flat,
                                       int64_t flat_stride_slot, int64_t flat_stride_head,
                                       int32_t num_slots, const int32_t* block_tables,
                                       int32_t table_stride, const int32_t* ctx_lens,
                                       int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                       int32_t head_dim, int32_t block_size, float scale,
                                       mf_dtype dtype, void* out, int32_t* err_flag,
                                       mf_stream_t stream) {
  using namespace mf;
  if (block_size <= 0 || num_slots % block_size != 0)
    return fail(MF_EINVAL, "noalloc decode: num_slots is not a multiple of block_size");
  if (batch == 0) return MF_OK;
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
  const size_t need = mf_paged_attention_workspace_size(&a, [] {
    int d = 0;
    cudaGetDevice(&d);
    return d;
  }());
  if (need > kScratchBytes)
    return fail(MF_EWORKSPACE, "noalloc decode: this batch needs " + std::to_string(need) +
                                   " bytes of split-K scratch, more than the library's fixed " +
                                   std::to_string(kScratchBytes) +
                                   " bytes; use mf_paged_decode with a caller workspace");
  void* scratch = nullptr;
  if (need > 0) {
    int rc = scratch_address(&scratch);
    if (rc != MF_OK) return rc;
    // The arrival counters must start at zero; a launch that gave up early
    // (bounded wait expired) could have left some behind, so clear the ones
    // this call can use.  Stream-ordered, no allocation.
    // At most 8 counters per (sequence, kv head) whatever the plan.
    size_t counters = (size_t)batch * num_kv_heads * 8 * sizeof(int32_t);
    if (counters > kSemRegionBytes) counters = kSemRegionBytes;
    cudaError_t e = cudaMemsetAsync(scratch, 0, counters, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess)
      return fail(MF_ECUDA, std::string("noalloc decode: ") + cudaGetErrorString(e));
  }
  return mf_paged_attention(&a, scratch, kScratchBytes, err_flag, stream);
}
