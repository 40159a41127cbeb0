// Allocation-free chamfer forward (tpo_chamfer_fwd_noalloc).
//
// Some callers cannot call cudaMalloc: code running inside a host memory pool
// or a custom allocator that must not be re-entered, real-time/inference
// services that forbid device allocation after start-up, and foreign-language
// hosts whose only handle on the GPU is buffers they were given.  For them this
// entry point runs the same chamfer forward as tpo_chamfer_fwd but keeps its
// per-point keys in a fixed device array owned by this library instead of a
// caller-provided workspace.
//
// The array is a file-scope __device__ variable, so every GPU that loads this
// library holds it (kNoAllocScratchBytes) until the process exits.  Its host-
// side name is only a stand-in: host code must obtain the device address with
// cudaGetSymbolAddress, once per device, with that device current.  All calls
// share the array and it keeps the previous call's contents; each call resets
// the part it uses before use.  Calls that overlap on the GPU (different
// streams, or different host threads on the same device) race on the array.
#include <mutex>

#include "tpo_internal.h"

namespace tpo {

// Limit: B*(N+M) <= 2,097,152 points for f32/f16 (8-byte keys, e.g. two
// 1M-point clouds), 1,048,576 for f64 (16-byte keys): 16 MiB of keys.  The array
// holds 512 bytes more because the two key regions each start on a 256-byte
// boundary (up to 248 bytes of padding each for 8-byte keys), so every problem
// within the point limit fits whatever the split between N and M.
constexpr size_t kNoAllocKeyBytes = size_t(16) << 20;
constexpr size_t kNoAllocScratchBytes = kNoAllocKeyBytes + 512;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once).
int scratch_for_current_device(void** out) {
  int dev = -1;
  int s = cuda_status(cudaGetDevice(&dev));
  if (s) return s;
  if (dev < 0 || dev >= kMaxDevices) return TPO_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    s = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (s) return s;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TPO_OK;
}
}  // namespace

}  // namespace tpo

using namespace tpo;

extern "C" TPO_API int tpo_chamfer_fwd_noalloc(int dtype, int flags, const void* xyz1,
                                               const void* xyz2, int64_t B, int64_t N, int64_t M,
                                               void* dist1, void* dist2, int32_t* idx1,
                                               int32_t* idx2, void* stream) {
  if (dtype != TPO_F32 && dtype != TPO_F16 && dtype != TPO_F64)
    return set_error(TPO_ERR_INVALID_ARGUMENT, "chamfer_fwd_noalloc: dtype must be f32, f16 or f64");
  if (B < 0 || N < 0 || M < 0) return set_error(TPO_ERR_INVALID_ARGUMENT, "chamfer_fwd_noalloc: negative size");
  // the point limit, checked without overflow: each factor is bounded first
  const int64_t max_points = (int64_t)(kNoAllocKeyBytes / (size_t)tpo_chamfer_key_bytes(dtype));
  if (B > max_points || N > max_points || M > max_points || B * (N + M) > max_points)
    return set_error(TPO_ERR_WORKSPACE,
                     "chamfer_fwd_noalloc: problem too large for the library's 16 MiB scratch "
                     "(B*(N+M) must be <= 2,097,152 points for f32/f16, 1,048,576 for f64); "
                     "use tpo_chamfer_fwd with a caller-provided workspace");
  if ((B * N > 0 && (!xyz1 || !dist1 || !idx1)) || (B * M > 0 && (!xyz2 || !dist2 || !idx2)))
    return set_error(TPO_ERR_INVALID_ARGUMENT, "chamfer_fwd_noalloc: null pointer");
  void* scratch = nullptr;
  int s = scratch_for_current_device(&scratch);
  if (s) return s;
  // Same work as tpo_chamfer_fwd with the library-owned array as its workspace
  // (that entry point resets the key region before use).
  return tpo_chamfer_fwd(dtype, flags, xyz1, xyz2, B, N, M, dist1, dist2, idx1, idx2, scratch,
                         kNoAllocScratchBytes, stream);
}
