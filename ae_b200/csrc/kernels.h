// Internal host-side declarations shared between the kernel files and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "layout.h"

namespace smb {

enum FfnMode { kGateUp = 1, kDown = 2 };

struct FfnArgs {
  const int32_t* expert_off;      // [E+1]
  const int64_t* page_of_expert;  // [E]  page of each expert inside the pool
  int* status;                    // device status word
  void* out;                      // kGateUp: A2 [rows, I] storage dtype; kDown: fp32 [S, Tk, H]
  long long num_pages;            // P
  int E, H, I, Tk, splits;
};

cudaError_t launch_ffn_gemm(int mode, bool bf16, int grid, cudaStream_t stream, bool pdl, const CUtensorMap& a,
                            const CUtensorMap& b64, const CUtensorMap& b32, const CUtensorMap& b16,
                            const FfnArgs& args);
int ffn_units(int mode, int E, int H, int I, int splits);

struct RouteArgs {
  const void* logits;      // [T, E] or nullptr (routing given)
  int logits_dtype;        // SMB_DTYPE_*
  const float* in_w;       // [T, k] given routing weights (logits == nullptr)
  const int32_t* in_ids;   // [T, k] given expert ids
  const void* x;           // [T, H] token rows
  int T, E, k, H, renormalize;
  float* out_w;            // optional [T, k]
  int32_t* out_ids;        // optional [T, k]
  int32_t* expert_off;     // workspace
  int32_t* perm;
  int32_t* inv;
  float* ws_w;
  int32_t* ws_ids;
  void* xp;
  int* status;
  int rows_per_cta;
};

cudaError_t launch_topk(const void* logits, int logits_dtype, int T, int E, int k, int renorm, float* out_w,
                        int32_t* out_ids, cudaStream_t stream);
cudaError_t launch_route(const RouteArgs& a, int elem_bytes, int grid, cudaStream_t stream, bool pdl);
size_t route_smem_bytes(int T, int E, int k);

struct CombineArgs {
  const float* part;    // [S, Tk, H]
  const int32_t* inv;   // [Tk]
  const float* w;       // [Tk]
  void* out;            // [T, H] storage dtype
  int T, k, H, splits;
};

cudaError_t launch_combine(const CombineArgs& a, bool bf16, cudaStream_t stream, bool pdl);

cudaError_t launch_align(const int32_t* ids, int numel, int E, int block, int32_t* sorted_ids, int32_t* expert_ids,
                         int32_t* num_post_pad, int max_blocks, cudaStream_t stream);

}  // namespace smb
