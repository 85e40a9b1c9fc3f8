// mf_peer_barrier: the completion step of a head-sharded attention call whose
// output rows were stored straight into every GPU's output buffer (the
// num_out_peers fields of mf_attention_args), in place of an all-gather.
//
// One warp per GPU.  Lane p publishes `epoch` into GPU p's counter for this
// rank with a system-scope release store (after a system-scope fence, so the
// attention kernel's peer stores that precede it on the stream are visible
// first); lane q != rank then polls this GPU's counter from rank q with
// system-scope acquire loads until it reaches `epoch`.  The poll is bounded
// (2 s of %globaltimer): on expiry it sets MF_ERR_TIMEOUT and returns.  Each
// GPU runs its own barrier kernel, so the kernels that wait on one another are
// always on different GPUs.

#include <cstring>

#include "mf_attn.h"

namespace {

constexpr uint64_t kWaitLimitNs = 2000000000ull;

struct PeerFlagPtrs {
  int32_t* f[MF_MAX_OUT_PEERS];
};

__global__ void peer_barrier_kernel(PeerFlagPtrs flags, int world, int rank, uint32_t epoch,
                                    int32_t* err) {
  const int t = threadIdx.x;
  __threadfence_system();
  if (t < world) {
    int32_t* dst = flags.f[t] + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
  }
  if (t < world && t != rank) {
    const int32_t* src = flags.f[rank] + t;
    uint64_t t0 = 0;
    for (int spin = 0;; ++spin) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(src) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      const uint64_t now = mf::global_ns();
      if (spin == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        mf::set_err(err, MF_ERR_TIMEOUT);
        break;
      }
    }
  }
}

}  // namespace

extern "C" int mf_peer_barrier(int32_t* const* flags, int32_t world, int32_t rank,
                               uint32_t epoch, int32_t* err_flag, mf_stream_t stream) {
  using namespace mf;
  if (world < 1 || world > MF_MAX_OUT_PEERS)
    return fail(MF_EINVAL, "peer barrier: world outside [1, MF_MAX_OUT_PEERS]");
  if (rank < 0 || rank >= world) return fail(MF_EINVAL, "peer barrier: rank outside [0, world)");
  if (!flags) return fail(MF_EINVAL, "peer barrier: null flags");
  PeerFlagPtrs p{};
  for (int i = 0; i < world; ++i) {
    if (!flags[i]) return fail(MF_EINVAL, "peer barrier: null flags entry");
    p.f[i] = flags[i];
  }
  if (world == 1) return MF_OK;
  peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p, world, rank, epoch,
                                                                            err_flag);
  return check_launch("peer barrier");
}

// ------------------------------------------------------------------ CUDA IPC
// The peer buffers of a head-sharded step are shared between the processes of
// one node with CUDA IPC.  A handle names a whole cudaMalloc allocation, so the
// exporter sends its allocation base's handle and the offset of the buffer in
// it; the importer maps the allocation into ITS OWN device's address space
// (the current device, with peer access enabled on first use) and adds the
// offset.

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = []() -> GetAddressRangeFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<GetAddressRangeFn>(ptr);
  }();
  return fn;
}

extern "C" int mf_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  using namespace mf;
  if (!ptr || !handle || !offset) return fail(MF_EINVAL, "ipc export: null argument");
  GetAddressRangeFn range = address_range_fn();
  if (!range) return fail(MF_ECUDA, "ipc export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(MF_EINVAL, "ipc export: pointer is not device memory");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(MF_ECUDA, std::string("ipc export: ") + cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  *offset = (uint64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MF_OK;
}

extern "C" int mf_ipc_open(const void* handle, uint64_t offset, void** ptr) {
  using namespace mf;
  if (!handle || !ptr) return fail(MF_EINVAL, "ipc open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(MF_ECUDA, std::string("ipc open: ") + cudaGetErrorString(e));
  *ptr = static_cast<char*>(base) + offset;
  return MF_OK;
}

extern "C" int mf_ipc_close(void* ptr, uint64_t offset) {
  using namespace mf;
  if (!ptr) return fail(MF_EINVAL, "ipc close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return fail(MF_ECUDA, std::string("ipc close: ") + cudaGetErrorString(e));
  return MF_OK;
}
