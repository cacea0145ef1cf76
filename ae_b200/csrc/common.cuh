// Device helpers for sm_100a: mbarriers with bounded waits, TMA tile loads, tcgen05
// (TMEM alloc / MMA / commit / load), programmatic dependent launch.  Written from the
// PTX ISA; every wait in this file gives up after a wall-clock budget and reports it.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "layout.h"

namespace smb {

// Wait budget for one mbarrier wait: 2 s of %globaltimer.  Normal waits last
// microseconds; hitting the budget means a protocol error, and the kernel then
// unwinds instead of hanging the GPU.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// System-scope flag access for the peer-memory exchange (flags live in another GPU's
// memory or are written from one).
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Raise n flags (typically in other GPUs' memory) to v as one release: one release fence,
// then relaxed system-scope stores that are all in flight together.  A release store per
// flag would wait, each, for the previous flag's store to reach its GPU.
__device__ __forceinline__ void raise_flags_sys(int* const* flags, int n, int v) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int i = 0; i < n; ++i) asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(flags[i]), "r"(v) : "memory");
}

// Wait, bounded, until flags[0..n) are all >= epoch (called by one thread; n <= kMaxRanks).
// Each round reads every flag with relaxed system-scope loads that are in flight together
// (one round trip, not n), and once all have reached the epoch one acquire fence orders
// the caller's later reads after the writes the flags publish.
__device__ __forceinline__ bool wait_flags_sys(const int* flags, int n, int epoch) {
  const uint64_t t0 = global_timer_ns();
  while (true) {
    int v[kMaxRanks];
#pragma unroll
    for (int s = 0; s < kMaxRanks; ++s) {
      v[s] = epoch;
      if (s < n) asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v[s]) : "l"(flags + s) : "memory");
    }
    bool all = true;
#pragma unroll
    for (int s = 0; s < kMaxRanks; ++s) all = all && v[s] >= epoch;
    if (all) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      return true;
    }
    if (global_timer_ns() - t0 > kWaitBudgetNs) return false;
    __nanosleep(100);
  }
}

// Called by every thread of every CTA once its global / peer stores are issued: true in
// the CTA that finished last; that CTA leaves the ticket at 0 for the next launch.  After
// the CTA barrier one thread takes the ticket with an acquire-release atomic at system
// scope: its release half is cumulative over the stores of the CTA it has synchronised
// with, and in the last CTA its acquire half (it reads every earlier CTA's increment) orders
// all CTAs' stores before what that thread writes next, so the flags it then raises with
// st.release.sys publish every CTA's stores system-wide.  Only thread 0 of the last CTA may
// raise flags.  No CTA waits for another.
__device__ __forceinline__ bool last_cta_of_grid(int* ticket, int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const int n = static_cast<int>(gridDim.x * gridDim.y * gridDim.z);
    int old;
    asm volatile("atom.acq_rel.sys.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(ticket) : "memory");
    *s_flag = old == n - 1 ? 1 : 0;
    if (*s_flag) *ticket = 0;
  }
  __syncthreads();
  return *s_flag != 0;
}

// last_cta_of_grid at GPU scope: for a grid whose last CTA only updates this GPU's own
// memory (read by later kernels on the same GPU), no system-scope fence is needed.
__device__ __forceinline__ bool last_cta_of_grid_gpu(int* ticket, int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int n = static_cast<int>(gridDim.x * gridDim.y * gridDim.z);
    *s_flag = atomicAdd(ticket, 1) == n - 1 ? 1 : 0;
    if (*s_flag) {
      __threadfence();
      *ticket = 0;
    }
  }
  __syncthreads();
  return *s_flag != 0;
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// Timer block of the workspace whose status word is `status` (the control block starts
// at the status word).
__device__ __forceinline__ DevTimers* timers_of(int* status) {
  return reinterpret_cast<DevTimers*>(reinterpret_cast<uint8_t*>(status) + kTimerOffset);
}

// Add one timed wait (ns since t0) to a (sum, count) pair of the timer block.
__device__ __forceinline__ void add_wait_time(unsigned long long* sum, unsigned int* count, uint64_t t0) {
  atomicAdd(sum, static_cast<unsigned long long>(global_timer_ns() - t0));
  atomicAdd(count, 1u);
}

// Stage clock of the control block whose first byte is `ctrl`.
__device__ __forceinline__ StageClock* stage_clock_of(void* ctrl) {
  return reinterpret_cast<StageClock*>(reinterpret_cast<uint8_t*>(ctrl) + kStageOffset);
}

// Called by one thread of block 0, after the kernel's wait on its predecessor.
__device__ __forceinline__ void stage_mark(StageClock* c, int stage) {
  if (c == nullptr) return;
  const unsigned long long t = global_timer_ns();
  const unsigned long long last = c->last;
  const unsigned int prev = c->last_stage;
  if (last != 0 && t > last && prev < static_cast<unsigned int>(kStages)) {
    c->ns[prev] += t - last;
    c->n[prev] += 1u;
  }
  c->last = t;
  c->last_stage = static_cast<unsigned int>(stage);
}

// Called by one thread once the stage's kernel has done its work (the last CTA of the
// grid): adds the time since the stage's stamp to its busy time.
__device__ __forceinline__ void stage_busy(StageClock* c, int stage) {
  if (c == nullptr || c->last_stage != static_cast<unsigned int>(stage) || c->last == 0) return;
  const unsigned long long t = global_timer_ns();
  if (t > c->last) c->busy[stage] += t - c->last;
}

// Kernel-duration timer of a grid: every CTA calls begin once (after its dependency
// wait) and end once (after its last store); the CTA that ends last adds the span from
// the earliest begin to its end.  One thread per CTA calls them.
__device__ __forceinline__ void grid_timer_begin(DevTimers* tm) {
  atomicMax(&tm->ffn_neg_t0, ~0ull - static_cast<unsigned long long>(global_timer_ns()));
}
// True in the CTA that ended last.
__device__ __forceinline__ bool grid_timer_end(DevTimers* tm) {
  __threadfence();
  const unsigned int n = gridDim.x * gridDim.y * gridDim.z;
  if (atomicAdd(&tm->ffn_exit, 1u) == n - 1) {
    const unsigned long long t1 = global_timer_ns();
    const unsigned long long t0 = ~0ull - atomicExch(&tm->ffn_neg_t0, 0ull);
    atomicAdd(&tm->ffn_ns, t1 > t0 ? t1 - t0 : 0ull);
    atomicAdd(&tm->ffn_launches, 1u);
    atomicExch(&tm->ffn_exit, 0u);
    return true;
  }
  return false;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and records
// kDevTimeout) when the budget runs out or when *abort was raised by another role.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status,
                                          volatile int* abort_flag) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitBudgetNs) {
        record_status(status, kDevTimeout);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2D tiled bulk tensor load global -> shared, completion counted on `bar` in bytes.
// c0 is the innermost (contiguous) coordinate in elements; callers keep c0 * elem
// size a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// L2 prefetch of one 2D tile (no shared-memory destination, no completion); the tensor
// map bounds-checks the coordinates, so a guessed tile can never fault.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

// ---------------------------------------------------------------- clusters (CTA pairs)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_index_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_shared_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// All threads of both CTAs: everything before (shared-memory initialisation, remote
// arrivals) is visible to the peer after.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive once on an mbarrier of a CTA of the cluster (address from map_shared_rank).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2D tiled TMA load into this CTA's shared memory whose completion (bytes) is counted on
// the pair leader's mbarrier (cluster address), for a cta_group::2 MMA.  c0 * elem size is
// a multiple of 16 bytes (callers pass multiples of 64 elements).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t leader_bar,
                                                 int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------- PDL
__device__ __forceinline__ void pdl_wait_prior_grids() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// TMEM of a CTA pair (cta_group::2): both CTAs' allocator warps (same warp index, same
// shared-memory slot) allocate and free; the allocation covers the same columns in both.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair MMA, issued by the leader CTA only: M = 256 rows, the first 128 from the leader's
// shared memory and the next 128 from the peer's at the same offset; the N columns of B
// split the same way (first N/2 in the leader, the rest in the peer); each CTA's TMEM at
// d_tmem receives its own 128 rows x N.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on an mbarrier (cluster address: this CTA's or the peer's) when every pair
// MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16/f16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread (thread i <- lane base+i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand stored with the 128-byte
// swizzle that TMA (CU_TENSOR_MAP_SWIZZLE_128B) writes: rows of 128 B (64 bf16), 8-row
// groups 1024 B apart.  Fields: start address >> 4 [0,14), leading byte offset >> 4
// [16,30) (not used by swizzled K-major layouts, set to 1), stride byte offset >> 4
// [32,46) = 1024 B, descriptor version 1 [46,48), layout type [61,64) = 2 (128B swizzle).
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor, kind::f16: D fp32 [4,6)=1, A/B format [7,10)/[10,13)
// (0 = f16, 1 = bf16), both K-major (bits 15/16 = 0), N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Two 16-column loads (32 lanes x 32 bit each) issued back to back and waited for once,
// in one asm statement so that no read of the destinations can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, uint32_t tb, float (&va)[16], float (&vb)[16]) {
  uint32_t a[16], b[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]),
        "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]),
        "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]),
        "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15])
      : "r"(ta), "r"(tb)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    va[i] = __uint_as_float(a[i]);
    vb[i] = __uint_as_float(b[i]);
  }
}

// silu(g) = g / (1 + e^-g) with the hardware exponential and an approximate divide: the
// result is rounded to the 16-bit storage type right after, far coarser than their error.
// For g -> -inf the divisor overflows to inf and the quotient is 0, the limit.
__device__ __forceinline__ float silu_f32(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}

}  // namespace smb
