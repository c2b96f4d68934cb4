// Split-key decode without any allocation: the scratch lives in a fixed
// device array compiled into the library.
//
// Some callers of the decode hook cannot allocate device memory.  A plugin
// running inside an inference engine such as vLLM receives the engine's own
// tensors (query rows, the paged KV cache, the slot table) and a stream, but
// the engine has already handed all remaining HBM to its KV-cache pool and
// owns every allocation; an extra cudaMalloc during a decode step can fail,
// or stall the step behind an implicit device synchronisation.  Hosts that
// bind the C ABI from another language may also have no handle to a CUDA
// allocator at all.  cs_cope_attn_decode_noalloc serves them: it runs the same
// kernels as cs_cope_attn_decode, with the workspace carved out of
// kScratchBytes of static device memory that every GPU loading this library
// holds until the process exits.
#include <mutex>

#include "common.cuh"

namespace cs {
int validate_attn_params(const cs_attn_params* p);
int64_t decode_workspace_bytes(const cs_attn_params* p);
int launch_decode(const cs_attn_params* p, void* workspace, cudaStream_t stream);
}  // namespace cs

namespace {

constexpr int64_t kScratchBytes = 16ll << 20;  // 16 MiB, the documented maximum
constexpr int kMaxDevices = 64;

// Device scratch shared by every call on a device.  In host code this name
// is only a stand-in for the device symbol: its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char cs_decode_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch[kMaxDevices] = {};

// Device address of the scratch array on the current device, resolved once
// per device (with that device current) and cached for the life of the
// process; a device reset, which re-creates the context and the array, makes
// the cached address stale (documented at the entry point's declaration).
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CS_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, cs_decode_scratch) != cudaSuccess || ptr == nullptr) {
      (void)cudaGetLastError();
      return CS_ERR_CUDA;
    }
    g_scratch[dev] = ptr;
  }
  *out = g_scratch[dev];
  return CS_OK;
}

}  // namespace

extern "C" int cs_cope_attn_decode_noalloc(const cs_attn_params* p, void* stream) {
  const int rc0 = cs::validate_attn_params(p);
  if (rc0 != CS_OK) return rc0;
  // 0 bytes: no rows, or a mode the decode kernels do not handle
  const int64_t need = cs::decode_workspace_bytes(p);
  if (need == 0) return p->nq == 0 ? CS_OK : CS_ERR_UNSUPPORTED;
  if (need > kScratchBytes) return CS_ERR_TOO_LARGE;
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != CS_OK) return rc;
  return cs::launch_decode(p, scratch, cs::as_stream(stream));
}
