/*
 * ae_b200 — C ABI of the B200 (sm_100a) MoE verify layer.
 *
 * The layer replaces the GPU expert path of SpecMoE (zzhbrr/ae):
 *   FusedMoE.forward           specmoe/layers/FusedMoE.py:508-532
 *   -> UnquantizedFusedMoEMethod.forward_cuda   specmoe/layers/FusedMoE.py:155-196
 *      -> sglang select_experts                 (call at FusedMoE.py:174-185)
 *      -> stack_fused_moe                       specmoe/layers/fused_moe_kernel.py:253-349
 *           moe_align_block_size (:16-85), fused_moe_kernel GEMM1 (:332-335),
 *           silu_and_mul (:337), fused_moe_kernel GEMM2 x routing weight (:339-342),
 *           torch.sum over top-k into hidden_states (:344-349)
 *
 * The reference has no FFI for this path (it is Python + Triton); these entry points
 * are what a binding of that Python surface calls.  Conventions:
 *   - every pointer is a device pointer unless stated; the caller owns every buffer,
 *     including the workspace (size from smb_moe_workspace_bytes); no layer call
 *     allocates device memory (the one allocating entry point is smb_ep_ipc_alloc, a
 *     set-up call of the peer-memory exchange);
 *   - calls are asynchronous and ordered on `stream` (a cudaStream_t); distinct streams
 *     may call concurrently with distinct workspaces;
 *   - return 0 (SMB_OK) or a negative SMB_ERR_* code; nothing aborts the process;
 *   - weights: `pool` is the expert page pool [num_pages, 3*I*H] in the page layout of
 *     FusedMoE.weight_loader (specmoe/layers/FusedMoE.py:485-505): page = [w1 (I x H) |
 *     w3 (I x H) | w2 (H x I)], row-major; `page_of_expert` is the int64 [E] indirection
 *     (`expert_cache_indices`, FusedMoE.py:508; `indicies`, fused_moe_kernel.py:256);
 *   - storage dtype SMB_DTYPE_F16 or SMB_DTYPE_BF16 for x / pool / out; router logits may
 *     also be SMB_DTYPE_F32; routing weights are fp32 and expert ids int32 (as
 *     select_experts returns them);
 *   - shape limits: H % 128 == 0, I % 64 == 0, 1 <= E <= 256, 1 <= k <= min(E, 8),
 *     T*k <= 16384, 16-byte aligned x / pool / out, 256-byte aligned workspace.
 */
#ifndef AE_B200_H_
#define AE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SMB_API __attribute__((visibility("default")))
#else
#define SMB_API
#endif

typedef struct CUstream_st* smb_stream_t; /* same handle as cudaStream_t */

enum smb_dtype { SMB_DTYPE_F16 = 0, SMB_DTYPE_BF16 = 1, SMB_DTYPE_F32 = 2 };

enum smb_status {
  SMB_OK = 0,
  SMB_ERR_SHAPE = -1,         /* a size outside the limits above */
  SMB_ERR_DTYPE = -2,         /* unsupported dtype code */
  SMB_ERR_ALIGN = -3,         /* pointer alignment (TMA needs 16 B; workspace 256 B) */
  SMB_ERR_WORKSPACE = -4,     /* workspace smaller than smb_moe_workspace_bytes */
  SMB_ERR_CUDA = -5,          /* a CUDA runtime call failed (smb_last_cuda_error) */
  SMB_ERR_TMA = -6,           /* tensor-map encoding failed or is unavailable */
  SMB_ERR_ARCH = -7,          /* current device is not compute capability 10.0 */
  SMB_ERR_NULL = -8,          /* a required pointer is NULL */
  SMB_ERR_DEVICE_TIMEOUT = -9,/* device status: a pipeline wait exceeded its budget */
  SMB_ERR_BAD_PAGE = -10,     /* device status: page_of_expert[e] outside [0, num_pages) */
  SMB_ERR_BAD_EXPERT = -11,   /* device status: a given expert id outside [0, E) */
  SMB_ERR_SCRATCH_LIMIT = -12 /* smb_moe_forward_noalloc: problem needs more than its 64 MiB scratch */
};

/* Library version (major*100 + minor). */
SMB_API int smb_version(void);

/* Static description of an error code. */
SMB_API const char* smb_strerror(int code);

/* Text of the last CUDA error seen by this thread inside the library. */
SMB_API const char* smb_last_cuda_error(void);

/* Bytes of workspace one layer call needs (0 for invalid sizes).  Depends on the
 * current device's SM count (split-K factor), so query it on the device you run on. */
SMB_API size_t smb_moe_workspace_bytes(int T, int E, int k, int H, int I, int dtype);

/* Split-K factor the down projection uses for these sizes (Tk = T*k) on the current
 * device. */
SMB_API int smb_moe_splits(int E, int H, int I, int Tk);


/* Router: softmax over E in fp32, top-k (ties to the lower expert index), optional
 * renormalisation; then the expert-major permutation (positions in the workspace).  Replaces select_experts (FusedMoE.py:174-185) + moe_align_block_size
 * (fused_moe_kernel.py:329).  topk_weights [T,k] fp32 / topk_ids [T,k] int32 are optional
 * outputs (NULL to skip). */
SMB_API int smb_moe_route(const void* router_logits, int logits_dtype, const void* x, int dtype, int T, int E, int k,
                  int H, int I, int renormalize, float* topk_weights, int32_t* topk_ids, void* ws,
                  size_t ws_bytes, smb_stream_t stream);

/* Routing only, sglang select_experts semantics (FusedMoE.py:174-185): topk_weights
 * [T,k] fp32, topk_ids [T,k] int32. */
SMB_API int smb_moe_topk(const void* router_logits, int logits_dtype, int T, int E, int k, int renormalize,
                 float* topk_weights, int32_t* topk_ids, smb_stream_t stream);

/* Permutation from a routing computed elsewhere (stack_fused_moe's
 * topk_weights / topk_ids arguments, fused_moe_kernel.py:257-259).  An id of -1 marks a
 * slot with no expert: it is left out of the permutation and contributes nothing to the
 * output (the padding rows of the expert-parallel exchange use it). */
SMB_API int smb_moe_permute(const float* topk_weights, const int32_t* topk_ids, const void* x, int dtype, int T, int E,
                    int k, int H, int I, void* ws, size_t ws_bytes, smb_stream_t stream);

/* Expert FFN on the permuted rows: tcgen05 gate/up GEMM with SiLU*mul epilogue, then the
 * split-K down GEMM.  Replaces fused_moe_kernel GEMM1 + silu_and_mul + GEMM2
 * (fused_moe_kernel.py:332-342).  Needs smb_moe_route or smb_moe_permute first, with the
 * same x [T,H]: token rows are read from x through the permutation, so x must be
 * unchanged between the two calls. */
SMB_API int smb_moe_ffn(const void* x, const void* pool, int64_t num_pages, const int64_t* page_of_expert,
                        int dtype, int T, int E, int k, int H, int I, void* ws, size_t ws_bytes,
                        smb_stream_t stream);

/* The two halves of smb_moe_ffn, for callers that interleave other work or time them
 * separately: the gate/up GEMM with the SiLU*mul epilogue (fused_moe_kernel.py:332-337)
 * and the split-K down GEMM (fused_moe_kernel.py:339-342). */
SMB_API int smb_moe_gate_up(const void* x, const void* pool, int64_t num_pages, const int64_t* page_of_expert,
                            int dtype, int T, int E, int k, int H, int I, void* ws, size_t ws_bytes,
                            smb_stream_t stream);
SMB_API int smb_moe_down(const void* pool, int64_t num_pages, const int64_t* page_of_expert, int dtype, int T,
                         int E, int k, int H, int I, void* ws, size_t ws_bytes, smb_stream_t stream);

/* Routing-weighted combine into out [T,H] (may alias x).  Replaces the routed-weight
 * multiply (fused_moe_kernel.py:197-201) and torch.sum over top-k (:344-349). */
SMB_API int smb_moe_combine(void* out, int dtype, int T, int E, int k, int H, int I, const void* ws, size_t ws_bytes,
                    smb_stream_t stream);

/* Routing-weighted combine of per-slot rows: out[t] = sum_j w[t,j] * rows[p(t,j)], where
 * rows [T*k, H] (storage dtype) are in the expert-major order of the smb_moe_route /
 * smb_moe_permute call that used `ws` (its routing weights and positions are read from
 * `ws`).  The expert-parallel path combines the expert outputs returned by the
 * all-to-all with it; replaces the routed-weight multiply and torch.sum over top-k
 * (fused_moe_kernel.py:197-201, 344-349) on the token's home rank. */
SMB_API int smb_moe_combine_rows(const void* rows, void* out, int dtype, int T, int E, int k, int H, int I,
                                 const void* ws, size_t ws_bytes, smb_stream_t stream);

/* Expert parallelism over G ranks (E/G experts per rank).  Exchange layout: G chunks, one
 * per peer rank, each of one header row plus C payload rows of H elements (storage
 * dtype); a header row carries the chunk's per-local-expert row counts as int32 in its
 * first (E/G)*4 bytes.  With C >= T*k (the worst case) nothing can overflow and the
 * all-to-alls move fixed sizes, so no count has to reach the host.  The reference has
 * no expert-parallel path (its ep flags are parsed but unused,
 * specmoe/utils/server_args.py:148,202); these replace the TP all-reduce placement of
 * specmoe/models/mixtral.py:113-114 for expert-sharded deployments.
 *
 * Source side, before the exchange: routing (as smb_moe_route) and the gather of token
 * rows into send [G][C+1][H] (destination-major, headers filled). */
SMB_API int smb_moe_ep_dispatch(const void* router_logits, int logits_dtype, const void* x, int dtype, int T, int E,
                                int k, int H, int I, int renormalize, int G, int C, void* send,
                                float* topk_weights, int32_t* topk_ids, void* ws, size_t ws_bytes,
                                smb_stream_t stream);

/* Workspace of the expert side of a G-rank exchange with C slots per (source, rank)
 * pair: the layout of smb_moe_workspace_bytes(G*C, E_loc, 1, H, I, dtype) with the
 * down split-K factor chosen for the ~C slots that hold a token (a source sends each rank
 * C/G rows on average), not for all G*C. */
SMB_API size_t smb_moe_ep_workspace_bytes(int G, int C, int E_loc, int H, int I, int dtype);

/* Expert side: the received chunks recv [G][C+1][H] through this rank's E_loc experts
 * (pool / page_of_expert hold the local pages); out_rows [G][C][H] gets each payload
 * row's expert output (rows past a chunk's counts are not written).  The FFN kernel
 * writes the rows itself (the down units that complete an output tile sum its split-K
 * partials).  ws is sized by smb_moe_ep_workspace_bytes(G, C, E_loc, H, I, dtype). */
SMB_API int smb_moe_ep_experts(const void* recv, int G, int C, const void* pool, int64_t num_pages,
                               const int64_t* page_of_expert, int dtype, int E_loc, int H, int I, void* out_rows,
                               void* ws, size_t ws_bytes, smb_stream_t stream);

/* Source side, after the exchange: out[t] = sum_j w[t,j] * back[row of slot (t,j)], back
 * [G][C][H] holding the returned expert outputs; ws is the workspace of the matching
 * smb_moe_ep_dispatch call. */
SMB_API int smb_moe_ep_combine(const void* back, void* out, int dtype, int T, int E, int k, int H, int I, int G,
                               int C, const void* ws, size_t ws_bytes, smb_stream_t stream);

/* Expert parallelism over peer memory (NVLink), without a collective library.  Every rank
 * owns an exchange arena of smb_ep_arena_bytes(G, C, H, dtype) bytes (the same layout on
 * all ranks) that its peers map through CUDA IPC: smb_ep_ipc_alloc on each rank, the
 * 64-byte handles exchanged by the host (e.g. torch.distributed), smb_ep_ipc_open of
 * every peer's handle.  `arenas` is then a host array of G device pointers, arenas[r]
 * being rank r's arena as seen from this process (this rank's own at index `rank`).
 * A layer call is the three calls below, in this order, on every rank (a rank without
 * tokens passes T = 0 and still makes them):
 *   dispatch: routing, then the rows for rank d are written into d's arena and a flag
 *     raised there when they have all landed;
 *   experts: waits (bounded) for the G flags, runs the local experts, writes each row's
 *     output into its source's arena and raises a flag there;
 *   combine: waits (bounded) for the G return flags, weighted sum into out [T,H].
 * The experts call is one kernel (the FFN kernel routes the received rows itself from the
 * chunks' header counts and its last CTA raises the return flags), so a layer call is
 * three kernels per rank.  The experts workspace must start zeroed (smb_moe_workspace_init)
 * and serve only experts calls: with no router before it, that kernel leaves its counters
 * at zero for the next call.
 * Flags carry an epoch kept in the arena (the count of finished calls), so calls can be
 * replayed from a CUDA graph.  A wait that runs out (2 s) records SMB_ERR_DEVICE_TIMEOUT in
 * the workspace status (smb_moe_read_status) and the call continues without the missing
 * rows.  G <= 8.  The reference has no expert-parallel path (see smb_moe_ep_dispatch). */
SMB_API size_t smb_ep_arena_bytes(int G, int C, int H, int dtype);
SMB_API int smb_ep_ipc_alloc(size_t bytes, void** dev_ptr, void* ipc_handle /* 64 bytes out */);
SMB_API int smb_ep_ipc_open(const void* ipc_handle, void** peer_ptr);
SMB_API int smb_ep_ipc_close(void* peer_ptr);
SMB_API int smb_ep_ipc_free(void* dev_ptr);
/* Zero this rank's arena control block and flags (epoch 0, tickets 0, no flag raised), on
 * `stream`.  Recovery after a call in which some rank's wait ran out (SMB_ERR_DEVICE_TIMEOUT,
 * e.g. a rank that skipped the call): the ranks' epochs no longer agree, so every rank
 * finishes its queued work, the ranks meet (host barrier), each resets its own arena, and
 * they meet again before the next call.  No kernel of the exchange may be running on any
 * rank meanwhile.  The reference has no expert-parallel path; its transfer engine bounds
 * its waits and reports failures the same way (specmoe/backend/htod_transfer_engine.py:347-370). */
SMB_API int smb_ep_arena_reset(void* arena, int G, int C, int H, int dtype, smb_stream_t stream);
SMB_API int smb_moe_ep_dispatch_p2p(const void* router_logits, int logits_dtype, const void* x, int dtype, int T,
                                    int E, int k, int H, int I, int renormalize, int G, int rank, int C,
                                    void* const* arenas, float* topk_weights, int32_t* topk_ids, void* ws,
                                    size_t ws_bytes, smb_stream_t stream);
SMB_API int smb_moe_ep_experts_p2p(int G, int rank, int C, void* const* arenas, const void* pool, int64_t num_pages,
                                   const int64_t* page_of_expert, int dtype, int E_loc, int H, int I, void* ws,
                                   size_t ws_bytes, smb_stream_t stream);
SMB_API int smb_moe_ep_combine_p2p(void* out, int dtype, int T, int E, int k, int H, int I, int G, int rank, int C,
                                   void* const* arenas, const void* ws, size_t ws_bytes, smb_stream_t stream);

/* Whole layer: route + ffn + combine (FusedMoE.forward, FusedMoE.py:508-532, without
 * the tensor-parallel all-reduce).  out may alias x (the reference writes in place). */
SMB_API int smb_moe_forward(const void* x, const void* router_logits, int logits_dtype, const void* pool,
                    int64_t num_pages, const int64_t* page_of_expert, int dtype, int T, int E, int k, int H, int I,
                    int renormalize, void* out, float* topk_weights, int32_t* topk_ids, void* ws,
                    size_t ws_bytes, smb_stream_t stream);

/* Whole layer from a given routing (stack_fused_moe, fused_moe_kernel.py:253-349). */
SMB_API int smb_moe_forward_routed(const void* x, const float* topk_weights, const int32_t* topk_ids, const void* pool,
                           int64_t num_pages, const int64_t* page_of_expert, int dtype, int T, int E, int k, int H,
                           int I, void* out, void* ws, size_t ws_bytes, smb_stream_t stream);

/* Layer with a shared expert (a Qwen2-MoE-style block: routed top-k experts plus one
 * expert every token takes, scaled by shared_weight[t], e.g. sigmoid of a shared gate;
 * NULL = 1).  The reference has no shared expert; this extends smb_moe_forward for the
 * fine-grained configurations.  The shared expert of intermediate size I_s is passed as
 * n_shared = ceil(I_s / I) pseudo-experts of intermediate I (SwiGLU is separable along
 * the intermediate dimension): page q holds rows [q*I, (q+1)*I) of its w1 and w3 and the
 * same columns of w2, zero-padded past I_s; their pages are page_of_expert[E ..
 * E+n_shared-1].  The pseudo-experts share the grouped GEMM launch with the routed ones.
 * router_logits [T, E] cover the routed experts; topk_weights / topk_ids [T, k] as in
 * smb_moe_route; ws sized by smb_moe_workspace_bytes(T, E+n_shared, k+n_shared, H, I, dtype);
 * k + n_shared <= 8. */
SMB_API int smb_moe_forward_shared(const void* x, const void* router_logits, int logits_dtype,
                                   const float* shared_weight, const void* pool, int64_t num_pages,
                                   const int64_t* page_of_expert, int dtype, int T, int E, int k, int n_shared,
                                   int H, int I, int renormalize, void* out, float* topk_weights, int32_t* topk_ids,
                                   void* ws, size_t ws_bytes, smb_stream_t stream);

/* Expert pages streamed from host memory while the layer runs (the reference keeps the
 * experts in page-locked host memory and copies them into its GPU page pool per layer:
 * HtoDTransferEngine / StreamPriorityEngine.decode_load_weight,
 * specmoe/backend/htod_transfer_engine.py:260-341, specmoe/engine.py:143-154,549-588).
 * smb_moe_page_copy queues, on copy_stream, the copy of one page (bytes from page-locked
 * host_src to page_dst, one cudaMemcpyAsync) followed by a write of `epoch` to the device
 * int page_ready (cuStreamWriteValue32, no kernel involved).  smb_moe_forward_streamed is
 * smb_moe_forward whose FFN kernel starts at once and waits (bounded) per unit for
 * page_ready[page] >= page_epoch before it loads that page's weights, so experts are
 * computed while later pages are still crossing PCIe.  page_ready holds one int per page of
 * the pool (num_pages), starts at 0; use a larger epoch for every new round of copies. */
SMB_API int smb_moe_page_copy(void* page_dst, const void* host_src, size_t bytes, int* page_ready, int epoch,
                              smb_stream_t copy_stream);
SMB_API int smb_moe_forward_streamed(const void* x, const void* router_logits, int logits_dtype, const void* pool,
                                     int64_t num_pages, const int64_t* page_of_expert, const int* page_ready,
                                     int page_epoch, int dtype, int T, int E, int k, int H, int I, int renormalize,
                                     void* out, float* topk_weights, int32_t* topk_ids, void* ws, size_t ws_bytes,
                                     smb_stream_t stream);

/* Zero the whole workspace (its control block, timers and counters).  Call once after
 * allocating a workspace, before its first smb_moe_forward_gated or expert-parallel experts
 * call: the gated launch counts its CTAs in a ticket kept in the control block, the experts
 * call relies on zeroed counters, and every call leaves them at zero again. */
SMB_API int smb_moe_workspace_init(void* ws, size_t ws_bytes, smb_stream_t stream);

/* Router gate only: router_logits [T,E] = x [T,H] gate_weight[E,H]^T, fp32 accumulation,
 * rounded to the storage dtype.  Replaces MixtralMoE.gate, a ReplicatedLinear(H, E,
 * bias=False) in the storage dtype (specmoe/models/mixtral.py:85-92, called at :111). */
SMB_API int smb_moe_gate(const void* x, const void* gate_weight, int dtype, int T, int E, int H, void* router_logits,
                         smb_stream_t stream);

/* Whole MixtralMoE block without the tensor-parallel all-reduce
 * (specmoe/models/mixtral.py:106-115): the gate of smb_moe_gate and the routing run in
 * one launch (router_logits, topk_weights, topk_ids: optional outputs, may be NULL),
 * then the FFN and the combine as smb_moe_forward.  The workspace must have been
 * initialised once with smb_moe_workspace_init. */
SMB_API int smb_moe_forward_gated(const void* x, const void* gate_weight, const void* pool, int64_t num_pages,
                                  const int64_t* page_of_expert, int dtype, int T, int E, int k, int H, int I,
                                  int renormalize, void* out, void* router_logits, float* topk_weights,
                                  int32_t* topk_ids, void* ws, size_t ws_bytes, smb_stream_t stream);

/* smb_moe_forward without any device allocation, for callers that cannot allocate
 * device memory at call time (a host whose allocator owns the HBM, a latency-critical
 * path where cudaMalloc's implicit synchronisation is not allowed, a binding without a
 * device allocator).  No counterpart in the reference: SpecMoE always allocates its
 * intermediate caches with torch.empty per call.  The caller passes inputs and outputs
 * only; the workspace is a library-owned static device array of 64 MiB per GPU (held
 * until the process exits).  Sizes whose smb_moe_workspace_bytes exceed 64 MiB return
 * SMB_ERR_SCRATCH_LIMIT (Mixtral-8x7B shapes fit for every T <= 448 on a
 * 148-SM B200; the split-K factor, and with it the need, depends on T).  The first call
 * on each device looks up the array's device address; make it before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race. */
SMB_API int smb_moe_forward_noalloc(const void* x, const void* router_logits, int logits_dtype, const void* pool,
                                    int64_t num_pages, const int64_t* page_of_expert, int dtype, int T, int E,
                                    int k, int H, int I, int renormalize, void* out, float* topk_weights,
                                    int32_t* topk_ids, smb_stream_t stream);

/* Device status of the last smb_moe_forward_noalloc call on the current device, read
 * synchronously on `stream` from the library's scratch (0, SMB_ERR_DEVICE_TIMEOUT,
 * SMB_ERR_BAD_PAGE or SMB_ERR_BAD_EXPERT): the companion of smb_moe_read_status for
 * callers that hold no workspace.  A noalloc call that returned 0 has only been queued;
 * problems the kernels find (a page id outside [0, num_pages) is skipped, not faulted)
 * show here.  No counterpart in the reference. */
SMB_API int smb_moe_noalloc_read_status(smb_stream_t stream);

/* Block-padded layout of moe_align_block_size (fused_moe_kernel.py:16-85):
 * sorted_ids [numel + E*(block_size-1)] (pad value numel), expert_ids
 * [cdiv(numel + E*(block_size-1), block_size)] (-1 past the last used block),
 * num_tokens_post_pad [1]. */
SMB_API int smb_moe_align_block_size(const int32_t* topk_ids, int numel, int E, int block_size, int32_t* sorted_ids,
                             int32_t* expert_ids, int32_t* num_tokens_post_pad, smb_stream_t stream);

/* Synchronously read the device status word of the last layer call that used `ws`
 * (0, SMB_ERR_DEVICE_TIMEOUT, SMB_ERR_BAD_PAGE or SMB_ERR_BAD_EXPERT). */
SMB_API int smb_moe_read_status(const void* ws, size_t ws_bytes, int T, int E, int k, int H, int I, int dtype,
                        smb_stream_t stream);

/* Device-side timers accumulated in a workspace's control block by the kernels that
 * used it (nanoseconds of the GPU's global timer), for profiling without a profiler, in
 * CUDA-graph replays too.  The reference has no counterpart (its Triton launches are
 * timed from the host, specmoe/optimizer/performance_simulator/operators/gpu_fused_moe.py:84-116).
 *   ffn_ns / ffn_launches: per FFN kernel launch, from the first CTA past its wait on the
 *     router to the last CTA done, summed;
 *   recv_wait_ns / recv_waits: expert side of the peer-memory exchange, time the FFN kernel
 *     waited for the sources' flags;
 *   combine_wait_ns / combine_waits: source side, time the final combine waited for the
 *     returned rows;
 *   stage_ns[i] / stage_calls[i]: per stage of a layer call, from the stage's first kernel
 *     block passing its wait on the previous kernel to the next stage's; stages 0 routing
 *     (expert-parallel: dispatch), 1 unused (reserved), 2 FFN (expert-parallel: with the
 *     wait for the sources' rows, their routing and the returned rows written), 3 combine,
 *     4 source-side final combine; the last stage
 *     of a call ends when the next call starts; stage_busy_ns[i]: the part of it until the
 *     stage's kernel finished (recorded by its last CTA where the kernel keeps a CTA
 *     ticket: the gated or single-CTA routing, the dispatch over peer memory, the FFN, the
 *     final combine over peer memory).  Over peer memory the whole chain keeps
 *     its stage clock in the rank's exchange arena: pass the arena (its own, at least 256
 *     bytes) as `ws` to read it.
 * Reads synchronously on `stream`; reset != 0 then zeroes the timers (stream-ordered). */
typedef struct smb_timers {
  uint64_t ffn_ns;
  uint64_t recv_wait_ns;
  uint64_t combine_wait_ns;
  uint32_t ffn_launches;
  uint32_t recv_waits;
  uint32_t combine_waits;
  uint32_t reserved;
  uint64_t stage_ns[5];
  uint32_t stage_calls[5];
  uint32_t reserved2;
  uint64_t stage_busy_ns[5];
} smb_timers_t;
SMB_API int smb_moe_read_timers(const void* ws, size_t ws_bytes, int reset, smb_timers_t* out, smb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* AE_B200_H_ */
