// smb_moe_forward_noalloc: the whole MoE layer call without any device allocation.
//
// Some callers cannot allocate device memory when they call the layer: a host
// application whose own allocator owns the HBM (a serving engine that reserves the
// expert page pool and the KV cache up front and hands out nothing else), code on a
// latency-critical path where cudaMalloc and its implicit device synchronisation are not
// allowed, or a foreign-language binding that has no device allocator at hand.  This
// entry point takes only the inputs and outputs of smb_moe_forward and runs the same
// kernels on a scratch buffer the library owns: a file-scope static __device__ array of
// kScratchBytes (64 MiB), which every GPU that loads this code keeps until the process
// exits.  Problems whose workspace (smb_moe_workspace_bytes) exceeds it are rejected
// with SMB_ERR_SCRATCH_LIMIT.
//
// The device address of the array is looked up once per device, on the first call made
// with that device current (cudaGetSymbolAddress; in host code the array's name is only a
// host-side stand-in and must never be handed to a kernel).  Make that first call on each
// device before any stream capture.
//
// All calls on a device share the one array and it keeps the last call's contents.
// Nothing in it has to start at zero: every scratch element a kernel reads is written
// earlier in the same call, and the first kernel resets the status word.  Calls that
// overlap on the GPU (different streams, or different host threads without ordering)
// race on the array; callers must order them.
#include <mutex>

#include "../../include/ae_b200.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = static_cast<size_t>(64) << 20;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxScratchDevices = 64;

struct ScratchSlot {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};

ScratchSlot g_scratch_slots[kMaxScratchDevices];

// Device address of g_scratch on the current device (set up once per device).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SMB_ERR_CUDA;
  if (dev < 0 || dev >= kMaxScratchDevices) return SMB_ERR_CUDA;
  ScratchSlot& s = g_scratch_slots[dev];
  std::call_once(s.once, [&s] {
    void* p = nullptr;
    s.err = cudaGetSymbolAddress(&p, g_scratch);
    s.ptr = (s.err == cudaSuccess) ? p : nullptr;
  });
  if (s.err != cudaSuccess || s.ptr == nullptr) return SMB_ERR_CUDA;
  *out = s.ptr;
  return SMB_OK;
}

}  // namespace

extern "C" int smb_moe_forward_noalloc(const void* x, const void* router_logits, int logits_dtype,
                                       const void* pool, int64_t num_pages, const int64_t* page_of_expert,
                                       int dtype, int T, int E, int k, int H, int I, int renormalize, void* out,
                                       float* topk_weights, int32_t* topk_ids, smb_stream_t stream) {
  const size_t need = smb_moe_workspace_bytes(T, E, k, H, I, dtype);
  if (need == 0) {
    // invalid sizes or dtype: let the regular validation name the problem
    return smb_moe_forward(x, router_logits, logits_dtype, pool, num_pages, page_of_expert, dtype, T, E, k, H, I,
                           renormalize, out, topk_weights, topk_ids, nullptr, 0, stream);
  }
  if (need > kScratchBytes) return SMB_ERR_SCRATCH_LIMIT;
  void* ws = nullptr;
  const int rc = scratch_address(&ws);
  if (rc != SMB_OK) return rc;
  return smb_moe_forward(x, router_logits, logits_dtype, pool, num_pages, page_of_expert, dtype, T, E, k, H, I,
                         renormalize, out, topk_weights, topk_ids, ws, kScratchBytes, stream);
}
