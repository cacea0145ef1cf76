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
// host-side stand-in and must never be handed to a kernel); a lookup that fails is tried
// again on the next call.  Make that first call on each device before any stream capture.
//
// All calls on a device share the one array and it keeps the last call's contents.
// Apart from the CTA tickets in its control block, nothing in it has to start at zero:
// every other scratch element a kernel reads is written earlier in the same call, and the
// first kernel resets the status word.  The tickets start at zero with the array (static
// device memory is zero-initialised when the module loads) and every launch that takes
// one leaves it at zero again.  Calls that
// overlap on the GPU (different streams, or different host threads without ordering)
// race on the array; callers must order them.  The kernels report a bad page id, a bad
// expert id or a device wait that ran out in the array's status word, which
// smb_moe_noalloc_read_status returns.
#include <mutex>

#include "../../include/ae_b200.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = static_cast<size_t>(64) << 20;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxScratchDevices = 64;

// Device address of g_scratch per device, filled by the first successful lookup on that
// device.  A failed lookup (for instance a first call made during a stream capture, or a
// transient error) is not kept: the next call on that device tries again.
struct ScratchSlot {
  std::mutex mu;
  void* ptr = nullptr;
};

ScratchSlot g_scratch_slots[kMaxScratchDevices];

// Device address of g_scratch on the current device.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return smb::record_cuda_error(err);
  if (dev < 0 || dev >= kMaxScratchDevices) return smb::record_cuda_error(cudaErrorInvalidDevice);
  ScratchSlot& s = g_scratch_slots[dev];
  std::lock_guard<std::mutex> lock(s.mu);
  if (s.ptr == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_scratch);
    if (err != cudaSuccess) return smb::record_cuda_error(err);
    if (p == nullptr) return smb::record_cuda_error(cudaErrorInvalidSymbol);
    s.ptr = p;
  }
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

// The status word the kernels of the last smb_moe_forward_noalloc call on the current
// device wrote (it sits at offset 0 of the scratch, as in every workspace).  A call that
// returned 0 has only been queued: a page id outside [0, num_pages), a given expert id
// out of range or a device wait that ran out shows here, not in the return code.
extern "C" int smb_moe_noalloc_read_status(smb_stream_t stream) {
  void* ws = nullptr;
  const int rc = scratch_address(&ws);
  if (rc != SMB_OK) return rc;
  return smb::read_status_word(static_cast<const int*>(ws), reinterpret_cast<cudaStream_t>(stream));
}
