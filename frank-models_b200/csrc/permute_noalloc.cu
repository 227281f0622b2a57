// frank_permute_noalloc: the expert permutation with its scratch memory in
// a fixed, library-owned device array instead of a caller workspace.
//
// Who needs it: callers that cannot allocate device memory at the point of
// the call -- a host framework that owns the whole device memory pool and
// hands plugins only their input/output buffers, an FFI binding from a
// language runtime that has no way to size and keep a CUDA workspace alive,
// or a latency-critical loop where an allocation (and the synchronisation
// it can imply) is not allowed.  They pass ids and the output buffers only.
//
// The scratch is FRANK_PERMUTE_NOALLOC_SCRATCH_BYTES (1 MiB) in a
// file-scope __device__ array: every GPU that loads this library holds it
// until the process exits.  Requests whose scratch need
// (frank_permute_workspace_size) exceeds it are rejected with FRANK_EINVAL.
//
// Host code cannot use the array's name as a device address (in host code it
// names a host-side stand-in).  The device address is looked up once per
// device with cudaGetSymbolAddress, with that device current, on the first
// call made on the device; that first call should therefore come before
// any stream capture.  The looked-up address is cached per device ordinal
// for the life of the process, which assumes one context per device: after
// cudaDeviceReset (or anything else that destroys and recreates the
// device's primary context) the module is reloaded, the array may move, and
// this entry point must not be called again in that process.
//
// All calls share the one array, which keeps whatever the last call left in
// it: calls that overlap on the GPU (different streams, or different host
// threads on the same device) race on it and must be serialised by the
// caller.  Nothing in it needs to start at zero -- every scratch word the
// permutation reads is written earlier in the same call.
#include <mutex>
#include <vector>

#include "common.cuh"

namespace frank {
size_t permute_workspace_size(int64_t, int64_t);
int launch_permute(const int32_t*, int64_t, int64_t, int32_t*, int32_t*, int32_t*, int32_t*, void*, size_t,
                   cudaStream_t, const float* = nullptr, float* = nullptr);
}  // namespace frank

namespace {

constexpr size_t kScratchBytes = FRANK_PERMUTE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_permute_scratch[kScratchBytes];

std::mutex g_mu;
std::vector<void*> g_addr;  // per device ordinal

// Device address of g_permute_scratch on the current device.
int scratch_address(void** out) {
  int dev = 0;
  FRANK_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_addr.size() <= dev) g_addr.resize(dev + 1, nullptr);
  if (!g_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_permute_scratch);
    if (e != cudaSuccess || p == nullptr) {
      frank::set_error("permute_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                       cudaGetErrorString(e));
      return FRANK_ECUDA;
    }
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return FRANK_OK;
}

}  // namespace

extern "C" int frank_permute_noalloc(const int32_t* ids, int64_t n_slots, int64_t E, int32_t* sorted_slots,
                                     int32_t* offsets, int32_t* slot_pos, int32_t* err_flag, void* stream) {
  if (n_slots < 0 || n_slots >= 0x7fffffffLL) {
    frank::set_error("permute_noalloc: n_slots=%lld out of range", (long long)n_slots);
    return FRANK_EINVAL;
  }
  if (E < 1 || E > 1024) {
    frank::set_error("permute_noalloc: E=%lld outside [1, 1024]", (long long)E);
    return FRANK_EINVAL;
  }
  const size_t need = frank::permute_workspace_size(n_slots, E);
  if (need > kScratchBytes) {
    frank::set_error(
        "permute_noalloc: n_slots=%lld with E=%lld needs %zu bytes of scratch, more than the fixed %zu; "
        "use frank_permute with a caller workspace",
        (long long)n_slots, (long long)E, need, kScratchBytes);
    return FRANK_EINVAL;
  }
  void* scratch = nullptr;
  FRANK_TRY(scratch_address(&scratch));
  return frank::launch_permute(ids, n_slots, E, sorted_slots, offsets, slot_pos, err_flag, scratch, kScratchBytes,
                               frank::as_stream(stream));
}
