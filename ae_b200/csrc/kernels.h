// Internal host-side declarations shared between the kernel files and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "layout.h"

namespace smb {

// Raise a kernel's dynamic shared-memory limit on the current device unless an earlier
// call already raised it at least as far (the attribute lasts for the process).  One
// `seen` table per kernel; concurrent first calls may both set it, which is harmless.
inline cudaError_t ensure_dyn_smem(const void* fn, int bytes, std::atomic<int>* seen, int seen_len) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev >= 0 && dev < seen_len && seen[dev].load(std::memory_order_relaxed) >= bytes) return cudaSuccess;
  err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess && dev >= 0 && dev < seen_len) {
    int cur = seen[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !seen[dev].compare_exchange_weak(cur, bytes)) {
    }
  }
  return err;
}

// Expert-parallel exchange over peer memory.  Rank r's arena (same layout on every rank,
// mapped by its peers through CUDA IPC) holds a control block (epoch, CTA tickets), the
// flags its peers set, and the receive / return chunks.  chunk[d] is where this kernel
// puts the rows meant for rank d; with the NCCL transport it points into the local send
// buffer instead, and no flag is set or waited for.
struct EpLink {
  void* chunk[kMaxRanks];  // per destination: base of this rank's chunk in its buffer
  int* flag[kMaxRanks];    // per destination: the flag slot this rank sets there (p2p)
  int* ctrl;               // local control block: [0] epoch of the last finished call, [1..3] tickets
  const int* wait_flags;   // local flags to wait for (one per peer), p2p receive sides
  int nranks;
  int p2p;                 // 1: peer memory with flags, 0: NCCL moves the buffers
};

struct FfnArgs {
  int32_t* expert_off;            // [E+1]
  const int64_t* page_of_expert;  // [E]  page of each expert inside the pool
  int* status;                    // device status word
  int* done;                      // [E*S*ntc] finished gate/up tiles per (expert, down split, token tile)
  int* sched;                     // [2] next unit to hand out, CTAs done gathering (all zeroed by the router)
  int ntc;                        // token-tile bound per expert (counter stride)
  const void* x;                  // token rows: the layer input [T, H], or the exchange layout
  int x_chunk;                    // 0: row t of x; C > 0: payload row t of [G][C+1][H]
  int32_t* inv;                   // [Tk] expert-major position of each flat slot
  int k;                          // top-k (slot f belongs to token f / k)
  void* xp;                       // [rows, H] gathered token rows, expert-major
  void* a2;                       // [rows, I] activations, expert-major
  float* part;                    // [S, Tk, H] split-K partials of the down projection
  long long num_pages;            // P
  int E, H, I, Tk, splits;
  int phase_mask;                 // 1: gate/up, 2: down, 3: both in one launch
  // streamed expert pages: page p's weights are usable once page_ready[p] >= page_epoch
  // (raised by the copy stream after the page's host-to-device copy); nullptr: resident
  const int* page_ready;
  int page_epoch;
  StageClock* clk;                // stage clock of the call's chain (stage 2), or nullptr
  // Expert side of the exchange (ep_C > 0): the down units of an output tile (256 rows of
  // H x one token tile) count themselves in tile_done; fix-up units (64 rows of H of one
  // such tile each, claimed after every down unit) wait for the tile's S splits, sum their
  // rows' partials in split order and write the sums, in the storage dtype, to row f % C
  // of chunk f / C of `link` (f = perm[p], the slot of position p).  Over peer memory the
  // grid's last CTA then raises each source's return flag.
  int* tile_done;                 // [E*m2*ntc] finished down units per (expert, row tile, token tile)
  int32_t* perm;                  // [Tk] slot of each expert-major position
  int ep_C;                       // C, or 0: partials only (the combine kernel reduces them)
  EpLink link;
  // Receive routing inside the kernel (recv_G > 0, expert side of the exchange): x is the
  // received [G][C+1][H] (x_chunk = C), whose header rows hold each source's counts per
  // local expert.  Every CTA derives the expert offsets and the positions of the slots it
  // gathers from them, after waiting (bounded) for recv_flags[0..G) >= *recv_epoch + 1 when
  // the rows come over peer memory (recv_flags non-null).  No router runs before such a
  // launch: the grid's last CTA leaves the ndone counters at `sched` at zero for the next
  // call (the workspace starts zeroed, smb_moe_workspace_init).
  int recv_G;
  const int* recv_flags;
  const int* recv_epoch;
  int ndone;
  int* exit_ticket;               // CTA ticket of the launch, 0 between launches
};

cudaError_t launch_ffn_gemm(bool bf16, int grid, cudaStream_t stream, bool pdl, const CUtensorMap& w13,
                            const CUtensorMap& w2, const CUtensorMap& xp, const CUtensorMap& a2, const FfnArgs& args);

// Prefill-sized calls on CTA pairs (ffn_pair.cu): phase 1 = gate/up with SiLU*mul into a2
// (w = the [P*3I, H] weight map, tok = xp), phase 2 = down split-K partials (w = the
// [P*3H, I] map, tok = a2).  `pairs` pairs; ffn_pair_capacity = pairs resident at once.
cudaError_t launch_ffn_pair(bool bf16, int phase, int pairs, cudaStream_t stream, bool pdl, const CUtensorMap& w,
                            const CUtensorMap& tok, const FfnArgs& args);
int ffn_pair_capacity(bool bf16);

struct RouteArgs {
  const void* logits;      // [T, E] or nullptr (routing given)
  int logits_dtype;        // SMB_DTYPE_*
  const float* in_w;       // [T, k] given routing weights (logits == nullptr)
  const int32_t* in_ids;   // [T, k] given expert ids
  const void* x;           // [T, H] token rows
  int T, E, k, H, renormalize;  // E, k: all experts / slots per token, shared ones included
  int k_routed;            // top-k slots per token (k - n_shared)
  int n_shared;            // pseudo-experts E-n_shared..E-1 every token takes (a shared expert)
  const float* shared_w;   // [T] weight of the shared slots, or nullptr for 1
  float* out_w;            // optional [T, k]
  int32_t* out_ids;        // optional [T, k]
  int32_t* expert_off;     // workspace
  int32_t* perm;
  int32_t* inv;
  float* ws_w;
  int32_t* ws_ids;
  int* status;
  int* done;               // [done_count] counters of the FFN kernel (see WsLayout::done), zeroed here
  int done_count;
  int rows_per_cta;
  // expert-parallel exchange layout: G chunks of (1 header row + C payload rows) x H; a
  // header row holds the chunk's per-local-expert counts as int32 in its first bytes
  void* ep_send;           // dispatch: gather rows into link.chunk[d] (non-null marks dispatch mode)
  int ep_G, ep_C, ep_Eloc;
  EpLink link;
  StageClock* clk;         // stage clock of the call's chain, or nullptr
  int stage;               // stage-clock stage (0: routing / dispatch)
};

// Expert-parallel dispatch: a CTA's token rows (slots [g0, g0 + rows_per_cta) span at
// most (rows_per_cta + k - 2) / k + 1 tokens) are copied into shared memory at the start of
// the kernel, while the CTA routes, if they fit in this many bytes; larger spans copy
// straight from global memory after the routing.
constexpr int kDispatchStageBytes = 64 * 1024;
__host__ __device__ inline int dispatch_stage_bytes(int rows_per_cta, int k, int row_bytes) {
  const int span = (rows_per_cta + k - 2) / k + 1;
  const long long b = static_cast<long long>(span) * row_bytes;
  return b <= kDispatchStageBytes ? static_cast<int>(b) : 0;
}

// Router gate fused with the routing (gate_route_kernel): logits = x W^T of
// ReplicatedLinear(H, E, bias=False) (specmoe/models/mixtral.py:85-92,111).
struct GateArgs {
  const void* x;        // [T, H] storage dtype
  const void* weight;   // [E, H] storage dtype
  float* logits;        // [T, E] workspace copy (values rounded to the storage dtype)
  void* logits_out;     // optional [T, E] storage dtype
  int* ticket;          // CTA ticket, 0 between launches
  int T, E, H;
  int route;            // 1: the last CTA routes all tokens with RouteArgs
};

cudaError_t launch_gate_route(const RouteArgs& a, const GateArgs& g, int dtype, int grid, cudaStream_t stream,
                              bool pdl);

cudaError_t launch_topk(const void* logits, int logits_dtype, int T, int E, int k, int renorm, float* out_w,
                        int32_t* out_ids, cudaStream_t stream);
cudaError_t launch_route(const RouteArgs& a, int elem_bytes, int grid, cudaStream_t stream, bool pdl);
// The router over many CTAs for large calls (no gate, no exchange): tpc tokens per CTA,
// hist [grid * E] int32 scratch, ticket and gen two int32 words that stay between calls
// (ticket back at 0 after each launch, gen counting launches).
constexpr int kMultiRouteMinSlots = 2048;
size_t route_multi_smem_bytes(int tpc, int E, int k);
cudaError_t launch_route_multi(const RouteArgs& a, int tpc, int grid, int* hist, int* ticket, int* gen,
                               cudaStream_t stream, bool pdl);
size_t route_smem_bytes(int T, int E, int k);

struct CombineArgs {
  const float* part;    // [S, Tk, H]
  const int32_t* inv;   // [Tk]
  const float* w;       // [Tk]
  void* out;            // [T, H] storage dtype
  int T, k, H, splits;
  StageClock* clk;      // stage clock of the call's chain (stage 3), or nullptr
};

cudaError_t launch_combine(const CombineArgs& a, bool bf16, cudaStream_t stream, bool pdl);

// ep_C > 0: rows are the returned expert outputs in the exchange layout [G][C][H];
// slot f reads row (ids[f] / ep_Eloc) * ep_C + inv[f] - expert_off[(ids[f] / ep_Eloc) * ep_Eloc]
cudaError_t launch_combine_rows(const void* rows, long long nrows, const int32_t* inv, const float* w, void* out,
                                int T, int k, int H, bool bf16, cudaStream_t stream, bool pdl, const EpLink* link,
                                int* status, StageClock* clk);

// Host helpers of the C ABI shared with the other entry-point files: record a CUDA error
// for smb_last_cuda_error (returns SMB_ERR_CUDA), and read a device status word as an
// SMB_* code (synchronous on `stream`).
int record_cuda_error(cudaError_t err);
int read_status_word(const int* status, cudaStream_t stream);

cudaError_t launch_align(const int32_t* ids, int numel, int E, int block, int32_t* sorted_ids, int32_t* expert_ids,
                         int32_t* num_post_pad, int max_blocks, cudaStream_t stream);

}  // namespace smb
