// Expert FFN of the MoE layer as one persistent, weight-streaming kernel on the
// 5th-generation tensor cores: phase 1 = gate/up GEMM with the SiLU*mul epilogue,
// phase 2 = down GEMM (split-K), in one launch.
//
// Reference arithmetic: the Triton fused_moe_kernel (specmoe/layers/fused_moe_kernel.py:88-210)
// launched twice by stack_fused_moe (:332-342) with silu_and_mul in between (:337).
//
// Shape of the work.  In the verify regime an expert sees 1..~100 tokens, so the layer
// streams the touched experts' weights once from HBM (swap-AB: weight rows fill the
// 128-row MMA M operand, the expert's tokens fill N = 16..256).  A unit of work is 256
// weight rows x a K range, issued as two M=128 tcgen05 MMAs per 16-wide K step that share
// one token tile:
//   phase 1 unit (expert, 128 features): rows of w1 (gate) and the same rows of w3 (up)
//     from the page viewed as [P*3I, H] -> two fp32 accumulators whose lane r holds gate
//     and up of feature r, so the epilogue forms silu(gate) * up in registers and stores
//     the activation rows of A2 [Tk, I] (expert-major token order, storage dtype);
//   phase 2 unit (expert, 256 hidden rows, K split): rows 2H.. of the page viewed as
//     [P*3H, I] (the reference's w2_off) against the expert's A2 rows -> fp32 partials
//     part[split][p][h].
// A phase-2 unit of expert e and split s needs the phase-1 units of e whose features lie
// in the split's K range: phase-1 epilogues count their finished units per (expert,
// split) (release), the token loaders of phase 2 wait for the count (acquire, bounded).
// On the expert side of an exchange, phase-3 (fix-up) units follow: 64 rows of H of one
// output tile each, summed over the S splits by the loader warps once the tile's down
// units have counted in, and written to the sources' chunks.  Units are claimed in order
// (all phase-1 units first, fix-ups last) and the grid is at most one CTA per SM, so the
// waits end.
//
// Data movement.  Each SM's TMA engine delivers about 50 GB/s; 148 SMs together
// saturate HBM only if TMA moves nothing but weights.  So weights come by TMA in 16 KB
// boxes (128 rows x 64 K, 128-byte swizzle, evict-first) and the small, L2-resident token
// tiles come by cp.async from six loader warps, written in the same swizzled layout
// (tiles of 128+ rows, prefill-sized batches, by TMA in 64-row boxes instead).  The
// gate/up token rows are first gathered into expert-major order by all CTAs in the
// prologue (a grid counter tells the loaders when it is complete), the down rows are A2.
// With streamed expert pages the producer also waits (bounded) for a unit's page to have
// arrived from host memory before loading it.
//
// Roles (384 threads, one CTA per SM):
//   warp 0      TMA producer (one thread): weight boxes, 32 KB per stage
//   warp 1      MMA issuer (one thread)
//   warps 2..7  token-tile loaders (192 threads, cp.async); warp 2 also owns TMEM.  Six
//               warps, because at 64 tokens per expert two loader warps moved only ~6 B
//               per cycle (the MMA waited on token tiles 4x longer than on weights and
//               the weight ring stayed full); measured T = 256: 536 -> 472 us per layer,
//               ten warps no better
//   warps 8..11 epilogue (128 threads = 128 TMEM lanes)
// TMEM: 512 columns = two 256-column buffers (double-buffered accumulators when the
// token tile is at most 128 wide, one buffer otherwise).
//
// Every wait is bounded (common.cuh); a timed-out wait records a status, unwinds and
// releases tensor memory.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace smb {

namespace {

#ifndef SMB_LOADER_WARPS
#define SMB_LOADER_WARPS 6
#endif
constexpr int kLoaderWarps = SMB_LOADER_WARPS;  // token-tile loader warps (2, 6 or 10)
static_assert((2 + kLoaderWarps) % 4 == 0, "epilogue warps must start at a multiple of 4 (TMEM lane quarters)");
constexpr int kEpiWarp0 = 2 + kLoaderWarps;      // first of the four epilogue warps
constexpr int kThreads = 32 * (kEpiWarp0 + 4);
constexpr int kBK = 64;                        // K elements per stage = one 128 B swizzle row
constexpr int kBoxRows = 128;                  // rows per weight box = MMA M
constexpr int kBoxBytes = kBoxRows * kBK * 2;  // 16 KB
constexpr int kATileBytes = 2 * kBoxBytes;     // 256 weight rows per stage
constexpr int kMaxN = 256;
constexpr int kTmemCols = 512;
constexpr int kMaxStages = 8;
constexpr int kLoaderThreads = 32 * kLoaderWarps;
constexpr int kQueue = 8;                      // unit-id queue between the producer and the other roles
constexpr int kQueueReaders = 2 + kLoaderWarps;  // MMA thread, each loader-warp leader, epilogue leader
constexpr int kDynSmem = 227 * 1024 - 5120;  // static shared block (~3.5 KB) + this <= 227 KB
constexpr int kEpiStage = 4 * 2048;            // epilogue staging, 2 KB per epilogue warp, at the end
constexpr int kPrefetchBlocks = 16;
#ifndef SMB_TMA_B_MIN
#define SMB_TMA_B_MIN 128
#endif
// Token tiles of experts with at least this many tokens in the pass come by TMA (64-row
// boxes) instead of cp.async: at 128+ tokens per expert the loader warps' cp.async stream
// fell behind the MMA.  Narrower experts of the same launch keep cp.async.
constexpr int kTmaBMin = SMB_TMA_B_MIN;            // K blocks of the first unit warmed in L2 (512 KB)
// Fix-up units per output tile of the exchange: 32 of its 256 rows of H each, so the sums
// of the last tiles spread over many CTAs instead of one epilogue.
#ifndef SMB_FIX_CHUNKS
#define SMB_FIX_CHUNKS 8
#endif
constexpr int kFixChunks = SMB_FIX_CHUNKS;
static_assert(256 % (4 * kFixChunks) == 0, "fix-up chunks hold whole float4 columns");
constexpr int kFixRows = 256 / kFixChunks;
// the loader warps and the epilogue warps share a fix-up unit
constexpr int kFixThreads = 32 * kLoaderWarps + 128;

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 16-byte copy global -> shared (zero-filled when !valid), with an L2 eviction policy:
// token rows are re-read by every weight tile of their expert, so they are kept in L2
// ahead of the streamed weights.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool valid, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0), "l"(pol)
               : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed; the
// arrival counts towards the phase (the barrier is initialised with one per loader).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 16-byte store with an L2 eviction policy (both addresses 16-byte aligned).
__device__ __forceinline__ void st_evict_last_v4(void* p, const uint4& v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w), "l"(pol)
               : "memory");
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct Unit {
  int phase;  // 1 gate/up, 2 down, 3 fix-up of an output tile of the exchange
  int te;     // index into the touched-expert list
  int mt;     // 128-feature tile (phase 1) or 256-row tile of w2 (phase 2)
  int nt;     // token tile of the expert (ncap tokens each)
  int ks;     // split index (phase 2), 64-row chunk of the tile (phase 3)
  int kb0;    // first 64-wide K block
  int kb1;    // one past the last K block
};

struct Geometry {
  int n1, n2, n3, total;  // phase-1, phase-2 and phase-3 units, all
  int m1, m2;         // tiles per expert
  int kb1_total, kb2_total;
  int splits;         // down split-K factor S
  const int* ntp;     // [touched + 1] prefix of token tiles over the touched experts (shared memory)
  int ntouched;
};

// Touched expert whose token tiles hold global token tile q: the last te with ntp[te] <= q.
__device__ __forceinline__ int expert_of_tile(const Geometry& g, int q) {
  int lo = 0, hi = g.ntouched;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (g.ntp[mid] <= q) lo = mid; else hi = mid;
  }
  return lo;
}

// Unit order: all gate/up units, expert by expert, then feature tile and token tile; then
// all down units, expert by expert, then split, row tile and token tile; then the fix-up
// units, expert by expert, then row tile, token tile and chunk.
// Units that stream the same weight rows for different token tiles are adjacent, so they
// are claimed at about the same time and the later ones read the rows from L2.
__device__ __forceinline__ Unit decode(int u, const Geometry& g) {
  Unit r;
  if (u < g.n1) {
    r.phase = 1;
    r.te = expert_of_tile(g, u / g.m1);
    const int nte = g.ntp[r.te + 1] - g.ntp[r.te];
    const int v = u - g.ntp[r.te] * g.m1;
    r.mt = v / nte;
    r.nt = v - r.mt * nte;
    r.ks = 0;
    r.kb0 = 0;
    r.kb1 = g.kb1_total;
  } else if (u >= g.n1 + g.n2) {
    const int per_tile = g.m2 * kFixChunks;
    const int v0 = u - g.n1 - g.n2;
    r.phase = 3;
    r.te = expert_of_tile(g, v0 / per_tile);
    const int nte = g.ntp[r.te + 1] - g.ntp[r.te];
    const int v = v0 - g.ntp[r.te] * per_tile;
    r.mt = v / (nte * kFixChunks);
    const int q = v - r.mt * nte * kFixChunks;
    r.nt = q / kFixChunks;
    r.ks = q - r.nt * kFixChunks;
    r.kb0 = 0;
    r.kb1 = 0;
  } else {
    // expert-major like the gate/up units, then split: an expert's first down units read
    // only its first features, whose gate/up units finish first
    const int per_tile = g.m2 * g.splits;
    const int v0 = u - g.n1;
    r.phase = 2;
    r.te = expert_of_tile(g, v0 / per_tile);
    const int nte = g.ntp[r.te + 1] - g.ntp[r.te];
    const int v = v0 - g.ntp[r.te] * per_tile;
    r.ks = v / (g.m2 * nte);
    const int q = v - r.ks * g.m2 * nte;
    r.mt = q / nte;
    r.nt = q - r.mt * nte;
    r.kb0 = static_cast<int>((static_cast<long long>(g.kb2_total) * r.ks) / g.splits);
    r.kb1 = static_cast<int>((static_cast<long long>(g.kb2_total) * (r.ks + 1)) / g.splits);
  }
  return r;
}

// K blocks [kb0, kb1) of split ks of the down projection (64-wide blocks of I).
__device__ __forceinline__ int split_kb0(const Geometry& g, int ks) {
  return static_cast<int>((static_cast<long long>(g.kb2_total) * ks) / g.splits);
}
// Gate/up feature tiles (128 features = 2 K blocks of the down projection each) a down
// unit of split ks waits for: those whose features overlap the split's K range.
__device__ __forceinline__ int split_need(const Geometry& g, int ks) {
  const int b0 = split_kb0(g, ks), b1 = split_kb0(g, ks + 1);
  return min(g.m1, (b1 + 1) / 2) - b0 / 2;
}

// Bounded wait by one thread until *p >= need (acquire at GPU scope); false after the
// wait budget or when another role aborted.
__device__ __forceinline__ bool wait_count(const int* p, int need, int* status, volatile int* abort_flag) {
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (ld_acquire(p) >= need) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitBudgetNs) {
      record_status(status, kDevTimeout);
      *abort_flag = 1;
      return false;
    }
    if (++spins > 8) __nanosleep(64);
  }
}

// Expert side of the exchange: the receive routing, by every CTA from the G x E_loc header
// counts of the received chunks.  Payload row i of source s belongs to the local expert
// whose run of s's counts holds i; positions are expert-major, and inside an expert ordered
// by source, then row (the order the generic permutation gives), so row (s, i) of expert e
// sits at off[e] + (rows of e from sources before s) + (i - first row of e in chunk s).
// Counts are clamped to the chunk's C rows.  Writes expert_off (every CTA the same values)
// and inv / perm of the slots this CTA gathers.  `rs`: 4 * kMaxExperts + 1 ints of shared
// memory (G * E_loc = E <= kMaxExperts).
template <typename T>
__device__ __forceinline__ void receive_routing(const FfnArgs& args, int* rs, int* s_ready) {
  const int G = args.recv_G, C = args.x_chunk, El = args.E;
  int* s_cnt = rs;
  int* s_start = rs + kMaxExperts;
  int* s_base = rs + 2 * kMaxExperts;
  int* s_off = rs + 3 * kMaxExperts;
  if (threadIdx.x == 0) {
    int ready = 1;
    // this call's status (errors are recorded only after a wait budget, long after this)
    if (blockIdx.x == 0) args.status[0] = 0;
    if (args.recv_flags != nullptr) {
      const uint64_t tw = global_timer_ns();
      ready = wait_flags_sys(args.recv_flags, G, *args.recv_epoch + 1) ? 1 : 0;
      if (!ready) record_status(args.status, kDevTimeout);
      if (blockIdx.x == 0) {
        DevTimers* tm = timers_of(args.status);
        add_wait_time(&tm->recv_wait_ns, &tm->recv_waits, tw);
      }
    }
    *s_ready = ready;
  }
  __syncthreads();
  const size_t row_bytes = static_cast<size_t>(args.H) * sizeof(T);
  for (int src = threadIdx.x; src < G; src += blockDim.x) {
    const int32_t* hdr = reinterpret_cast<const int32_t*>(static_cast<const uint8_t*>(args.x) +
                                                          static_cast<size_t>(src) * (C + 1) * row_bytes);
    int run = 0;
    for (int e = 0; e < El; ++e) {
      int c = *s_ready ? __ldcg(hdr + e) : 0;  // written by the source (another GPU over peer memory)
      c = max(0, min(c, C - run));
      s_cnt[src * El + e] = c;
      s_start[src * El + e] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < El; e += blockDim.x) {
    int acc = 0;
    for (int src = 0; src < G; ++src) {
      s_base[src * El + e] = acc;
      acc += s_cnt[src * El + e];
    }
    s_off[e] = acc;  // rows of expert e, for now
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int pos = 0;
    for (int e = 0; e < El; ++e) {
      const int c = s_off[e];
      s_off[e] = pos;
      args.expert_off[e] = pos;
      pos += c;
    }
    s_off[El] = pos;
    args.expert_off[El] = pos;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * El; i += blockDim.x) s_base[i] += s_off[i % El];
  __syncthreads();
  // the slots this CTA gathers (the same split as the gather below)
  const int Tk = args.Tk;
  const int per = (Tk + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int f0 = min(Tk, static_cast<int>(blockIdx.x) * per), f1 = min(Tk, f0 + per);
  for (int f = f0 + threadIdx.x; f < f1; f += blockDim.x) {
    const int src = f / C, i = f - (f / C) * C;
    int p = -1;
    for (int e = 0; e < El; ++e) {
      const int q = src * El + e;
      if (i >= s_start[q] && i < s_start[q] + s_cnt[q]) {
        p = s_base[q] + (i - s_start[q]);
        break;
      }
    }
    args.inv[f] = p;
    if (p >= 0) args.perm[p] = f;
  }
  __syncthreads();
}

// Fix-up of one chunk (kFixRows rows of H) of an output tile of the exchange: rows
// [p0, p0 + nlen) of the expert-major positions; every split's partial of an element loaded
// at once, summed in split order, and the row written in the storage dtype into its
// source's chunk.  Threads first, first + stride, ... take the elements.
template <typename T>
__device__ __forceinline__ void fixup_rows(const FfnArgs& args, int splits, int mt, int ks, int p0, int nlen,
                                           int first, int stride) {
  const int H = args.H;
  const int h0 = mt * 256 + ks * kFixRows;
  const int nh4 = max(0, min(kFixRows, H - h0)) / 4;  // float4 per row of the chunk
  const size_t sstride = static_cast<size_t>(args.Tk) * H;
  for (int idx = first; idx < nlen * nh4; idx += stride) {
    const int r = idx / nh4, c4 = idx - r * nh4;
    const int p = p0 + r;
    const int h = h0 + c4 * 4;
    const float* src = args.part + static_cast<size_t>(p) * H + h;
    // every split's load in flight at once, then the sum in split order
    float4 v[kMaxSplits];
#pragma unroll
    for (int j = 0; j < kMaxSplits; ++j) {
      if (j < splits) v[j] = __ldcg(reinterpret_cast<const float4*>(src + j * sstride));
    }
    const int f = args.perm[p];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < kMaxSplits; ++j) {
      if (j < splits) {
        acc.x += v[j].x;
        acc.y += v[j].y;
        acc.z += v[j].z;
        acc.w += v[j].w;
      }
    }
    if (f < 0 || f >= args.Tk) continue;
    const int src_rank = f / args.ep_C;
    const int i = f - src_rank * args.ep_C;
    union {
      T h[4];
      uint2 u;
    } pk;
    pk.h[0] = from_f32<T>(acc.x);
    pk.h[1] = from_f32<T>(acc.y);
    pk.h[2] = from_f32<T>(acc.z);
    pk.h[3] = from_f32<T>(acc.w);
    *reinterpret_cast<uint2*>(reinterpret_cast<T*>(args.link.chunk[src_rank]) + static_cast<size_t>(i) * H + h) =
        pk.u;
  }
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    ffn_gemm_kernel(const __grid_constant__ CUtensorMap tm_w13, const __grid_constant__ CUtensorMap tm_w2,
                    const __grid_constant__ CUtensorMap tm_xp, const __grid_constant__ CUtensorMap tm_a2,
                    const FfnArgs args) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t dyn_smem[];
  __shared__ uint64_t fullA_bar[kMaxStages], fullB_bar[kMaxStages], empty_bar[kMaxStages];
  __shared__ uint64_t tfull_bar[2], tempty_bar[2], drain_bar, fix_bar;
  __shared__ uint64_t qfull_bar[kQueue], qempty_bar[kQueue];
  __shared__ int s_queue[kQueue];
  __shared__ uint32_t s_tmem;
  __shared__ int s_touched[kMaxExperts];
  __shared__ int s_page[kMaxExperts];
  __shared__ int s_ntp[kMaxExperts + 1];
  __shared__ int s_ntouched, s_ncap, s_stages;
  __shared__ int s_abort, s_epi_ok, s_epi_unit, s_issued, s_consumed, s_last_cta, s_recv_ready;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t raw_base = smem_u32(dyn_smem);
  const uint32_t ring_base = (raw_base + 1023u) & ~1023u;

  const int E = args.E, H = args.H, I = args.I;
  const bool do1 = (args.phase_mask & 1) != 0;
  const bool do2 = (args.phase_mask & 2) != 0;
  const bool chained = do1 && do2;  // phase 2 waits on this launch's phase 1

  if (threadIdx.x == 0) {
    s_abort = 0;
    s_issued = 0;
    s_consumed = 0;
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&fullA_bar[s], 1);
      mbar_init(&fullB_bar[s], kLoaderThreads);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 128);
    }
    for (int q = 0; q < kQueue; ++q) {
      mbar_init(&qfull_bar[q], 1);
      mbar_init(&qempty_bar[q], kQueueReaders);
    }
    mbar_init(&drain_bar, 1);
    mbar_init(&fix_bar, kLoaderWarps + 1);
    fence_mbarrier_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tmap(&tm_w13);
    prefetch_tmap(&tm_w2);
  }
  if (warp == 2) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }

  // While the router (launched just before) may still run, warm L2 with the first K
  // blocks of the gate/up unit this CTA's index would get if every expert is touched and
  // has one token tile (units are claimed roughly in CTA order, and any CTA reuses what
  // another fetched).  A guess only: the prefetch is bounds-checked by the tensor map and
  // never waited on.  page_of_expert was written before the router started, so it is final.
  if (threadIdx.x == 0 && do1 && args.page_ready == nullptr) {
    const int m1 = (I + 127) / 128;
    const int e = static_cast<int>(blockIdx.x) / m1;
    if (e < E) {
      const long long pg = args.page_of_expert[e];
      if (pg >= 0 && pg < args.num_pages) {
        const int r0 = static_cast<int>(pg) * 3 * I + (static_cast<int>(blockIdx.x) % m1) * 128;
        const int kbs = min(H / kBK, kPrefetchBlocks);
        for (int kb = 0; kb < kbs; ++kb) {
          tma_prefetch_l2_2d(&tm_w13, kb * kBK, r0);
          tma_prefetch_l2_2d(&tm_w13, kb * kBK, r0 + I);
        }
      }
    }
  }

  // Everything above touched only this CTA's own shared and tensor memory (and L2
  // hints); the routing results and the token rows come from the router.
  pdl_wait_prior_grids();
  if (threadIdx.x == 0) grid_timer_begin(timers_of(args.status));
  if (threadIdx.x == 0 && blockIdx.x == 0) stage_mark(args.clk, 2);
  if (args.recv_G > 0) {
    // scratch in the epilogue staging area (first used by the epilogue after its first
    // accumulator, long after this)
    receive_routing<T>(args, reinterpret_cast<int*>(dyn_smem + (kDynSmem - kEpiStage)), &s_recv_ready);
  }

  if (threadIdx.x == 0) {
    int nt = 0, maxn = 0;
    for (int e = 0; e < E; ++e) {
      const int n = args.expert_off[e + 1] - args.expert_off[e];
      if (n > 0) {
        const long long pg = args.page_of_expert[e];
        if (pg < 0 || pg >= args.num_pages) {
          record_status(args.status, kDevBadPage);
          continue;
        }
        s_touched[nt] = e;
        s_page[nt] = static_cast<int>(pg);
        ++nt;
        maxn = max(maxn, n);
      }
    }
    int ncap = (maxn + 15) & ~15;
    ncap = max(16, min(kMaxN, ncap));
    if (ncap >= kTmaBMin) ncap = min(kMaxN, (ncap + 63) & ~63);  // whole 64-row TMA boxes
    // token tiles per touched expert (ncap tokens each), prefix-summed; never more than
    // the counters' bound args.ntc (an expert with more than 256 tokens has ncap = 256)
    s_ntp[0] = 0;
    for (int t = 0; t < nt; ++t) {
      const int e = s_touched[t];
      const int n = args.expert_off[e + 1] - args.expert_off[e];
      s_ntp[t + 1] = s_ntp[t] + min(args.ntc, (n + ncap - 1) / ncap);
    }
    const int stage_bytes = kATileBytes + ncap * 128;
    s_ntouched = nt;
    s_ncap = ncap;
    s_stages = min(kMaxStages, (kDynSmem - 1024 - kEpiStage) / stage_bytes);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();

  // Gather: token rows into xp in expert-major order, each CTA a contiguous share of
  // the flat slots (slot f -> position inv[f], token f / k; in the expert-parallel
  // exchange layout token t is payload row t of chunk t / C).  The CTA then counts
  // itself in (release); token loaders wait for all CTAs before the first gate/up tile,
  // while the weight stream has already started.  Skipped when only the down phase runs.
  if (do1) {
    const int Tk = args.Tk;
    const int per = (Tk + gridDim.x - 1) / gridDim.x;
    const int f0 = min(Tk, static_cast<int>(blockIdx.x) * per), f1 = min(Tk, f0 + per);
    const int vec = H * static_cast<int>(sizeof(T)) / 16;
    const uint4* xs = reinterpret_cast<const uint4*>(args.x);
    uint4* xd = reinterpret_cast<uint4*>(args.xp);
    const int nvec = (f1 - f0) * vec;
    for (int i = threadIdx.x; i < nvec; i += kThreads) {
      const int f = f0 + i / vec;
      const int p = args.inv[f];
      if (p < 0 || p >= Tk) continue;
      const int t = f / args.k;
      const int srow = args.x_chunk == 0 ? t : (t / args.x_chunk) * (args.x_chunk + 1) + 1 + (t % args.x_chunk);
      xd[static_cast<size_t>(p) * vec + (i % vec)] = __ldg(xs + static_cast<size_t>(srow) * vec + (i % vec));
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(args.sched + 1, 1);
  }

  const uint32_t tmem = s_tmem;
  const int ncap = s_ncap;
  const int nstages = s_stages;
  const int stage_bytes = kATileBytes + ncap * 128;
  const int nbuf = ncap <= 128 ? 2 : 1;
  const bool tma_b = ncap >= kTmaBMin;
  const uint32_t acc1_off = nbuf == 2 ? 128u : 256u;

  Geometry g;
  g.m1 = (I + 127) / 128;
  g.m2 = (H + 255) / 256;
  g.kb1_total = H / kBK;
  g.kb2_total = I / kBK;
  g.splits = args.splits;
  g.ntp = s_ntp;
  g.ntouched = s_ntouched;
  const int tiles = s_ntp[s_ntouched];
  g.n1 = do1 ? tiles * g.m1 : 0;
  g.n2 = do2 ? tiles * g.m2 * g.splits : 0;
  g.n3 = do2 && args.ep_C > 0 ? tiles * g.m2 * kFixChunks : 0;
  g.total = g.n1 + g.n2 + g.n3;

  // Units are handed out dynamically: the producer claims the next unit id from a
  // global counter (zeroed by the router) and publishes it through a small queue in
  // shared memory; the other roles read the same ids in the same order.  Claims run in
  // increasing order, so every gate/up unit is claimed before any down unit.
  auto next_unit = [&](int& qi, uint32_t& qph) -> int {
    if (!mbar_wait(&qfull_bar[qi], qph, args.status, &s_abort)) return -1;
    const int u = *reinterpret_cast<volatile int*>(&s_queue[qi]);
    mbar_arrive(&qempty_bar[qi]);
    if (++qi == kQueue) {
      qi = 0;
      qph ^= 1u;
    }
    return u;
  };
  // tokens [n0, n0 + nlen) of touched expert te in the unit's token tile
  auto tile_tokens = [&](const Unit& un, int& row0, int& n0, int& nlen) {
    const int e = s_touched[un.te];
    row0 = args.expert_off[e];
    n0 = un.nt * ncap;
    nlen = min(ncap, args.expert_off[e + 1] - row0 - n0);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (weights)
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      int qi = 0;
      uint32_t qph = 0;
      int issued = 0;
      uint32_t fix_phase = 0;
      bool ok = true;
      while (ok) {
        if (!mbar_wait(&qempty_bar[qi], qph ^ 1u, args.status, &s_abort)) break;
        int u = atomicAdd(args.sched, 1);
        if (u >= g.total) u = -1;
        s_queue[qi] = u;
        mbar_arrive(&qfull_bar[qi]);
        if (++qi == kQueue) {
          qi = 0;
          qph ^= 1u;
        }
        if (u < 0) break;
        const Unit un = decode(u, g);
        if (un.phase == 3) {
          // no weights: claim nothing more until the loader and epilogue warps have done
          // this fix-up, so that fix-ups spread over the CTAs instead of queueing up in one
          if (!mbar_wait(&fix_bar, fix_phase, args.status, &s_abort)) break;
          fix_phase ^= 1u;
          continue;
        }
        const int page = s_page[un.te];
        if (args.page_ready != nullptr) {
          // streamed pages: the weights of this unit's page must have arrived
          const uint64_t t0 = global_timer_ns();
          while (ld_acquire_sys(args.page_ready + page) < args.page_epoch) {
            if (*reinterpret_cast<volatile int*>(&s_abort)) {
              ok = false;
              break;
            }
            if (global_timer_ns() - t0 > kWaitBudgetNs) {
              record_status(args.status, kDevTimeout);
              s_abort = 1;
              ok = false;
              break;
            }
            __nanosleep(200);
          }
          if (!ok) break;
          // the page was written by the copy engine; the TMA reads it through the async proxy
          asm volatile("fence.proxy.async;" ::: "memory");
        }
        const CUtensorMap* map = un.phase == 1 ? &tm_w13 : &tm_w2;
        // rows of the two 128-row boxes
        const int r0 = un.phase == 1 ? page * 3 * I + un.mt * 128 : page * 3 * H + 2 * H + un.mt * 256;
        const int r1 = un.phase == 1 ? r0 + I : r0 + 128;
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, args.status, &s_abort)) {
            ok = false;
            break;
          }
          uint8_t* sA = dyn_smem + (ring_base - raw_base) + stage * stage_bytes;
          mbar_arrive_expect_tx(&fullA_bar[stage], kATileBytes);
          tma_load_2d(sA, map, &fullA_bar[stage], kb * kBK, r0, pol_w);
          tma_load_2d(sA + kBoxBytes, map, &fullA_bar[stage], kb * kBK, r1, pol_w);
          ++issued;
          if (++stage == nstages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      s_issued = issued;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int qi = 0;
      uint32_t qph = 0;
      int pass = 0;
      int consumed = 0;
      bool ok = true;
      while (ok) {
        const int u = next_unit(qi, qph);
        if (u < 0) break;
        const Unit un = decode(u, g);
        if (un.phase == 3) continue;  // no MMA
        int row0, n0, nlen;
        tile_tokens(un, row0, n0, nlen);
        const int nb = (nlen + 15) & ~15;
        const uint32_t idesc = idesc_f16(kBF16, 128, nb);
        const int buf = pass % nbuf;
        if (!mbar_wait(&tempty_bar[buf], ((pass / nbuf) & 1) ^ 1u, args.status, &s_abort)) break;
        tc_fence_after();
        const uint32_t acc0 = tmem + static_cast<uint32_t>(buf * 256);
        const uint32_t acc1 = acc0 + acc1_off;
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&fullA_bar[stage], phase, args.status, &s_abort) ||
              !mbar_wait(&fullB_bar[stage], phase, args.status, &s_abort)) {
            ok = false;
            break;
          }
          // the token tile was written by cp.async (generic proxy); the MMA reads it
          // through the async proxy
          fence_proxy_async_smem();
          tc_fence_after();
          const uint32_t a_addr = ring_base + stage * stage_bytes;
          const uint64_t ad0 = desc_kmajor_sw128(a_addr);
          const uint64_t ad1 = desc_kmajor_sw128(a_addr + kBoxBytes);
          const uint64_t bd = desc_kmajor_sw128(a_addr + kATileBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // +32 bytes along K inside the swizzle row = +2 in the encoded start address
            const uint32_t acc = (kb > un.kb0 || kk > 0) ? 1u : 0u;
            umma_f16(acc0, ad0 + 2 * kk, bd + 2 * kk, idesc, acc);
            umma_f16(acc1, ad1 + 2 * kk, bd + 2 * kk, idesc, acc);
          }
          umma_commit(&empty_bar[stage]);
          ++consumed;
          if (++stage == nstages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[buf]);
        ++pass;
      }
      s_consumed = consumed;
    }
  } else if (warp >= 2 && warp < kEpiWarp0) {
    // ------------------------------------------------------------ token-tile loaders
    // Lane 0 of each loader warp does every wait and broadcasts the outcome, so a wait
    // that gives up ends the whole warp together.
    // Gate/up token rows come from xp (gathered in this kernel's prologue, see above),
    // down rows from A2; both in expert-major order, rows row0 + n0 + r.
    const int bt = threadIdx.x - 64;
    const T* xp = reinterpret_cast<const T*>(args.xp);
    const T* a2 = reinterpret_cast<const T*>(args.a2);
    const uint64_t pol_rows = policy_evict_last();
    bool gathered = false;
    const unsigned full = 0xffffffffu;
    int stage = 0;
    uint32_t phase = 0;
    int qi = 0;
    uint32_t qph = 0;
    bool ok = true;
    while (ok) {
      int u = 0;
      if (lane == 0) u = next_unit(qi, qph);
      u = __shfl_sync(full, u, 0);
      if (u < 0) break;
      const Unit un = decode(u, g);
      const int e = s_touched[un.te];
      int row0, n0, nlen;
      tile_tokens(un, row0, n0, nlen);
      if (un.phase == 3) {
        // fix-up: once all S down units of the output tile have stored their partials,
        // sum this chunk's rows in split order and write them to the sources' chunks
        int ready = 1;
        if (lane == 0) {
          ready = wait_count(args.tile_done + (e * g.m2 + un.mt) * args.ntc + un.nt, g.splits, args.status,
                             &s_abort) ? 1 : 0;
        }
        ready = __shfl_sync(full, ready, 0);
        __syncwarp();
        if (!ready) break;
        fixup_rows<T>(args, g.splits, un.mt, un.ks, row0 + n0, nlen, bt, kFixThreads);
        __syncwarp();
        if (lane == 0) mbar_arrive(&fix_bar);
        continue;
      }
      const int K = un.phase == 1 ? H : I;
      const int nb = (nlen + 15) & ~15;
      int ready = 1;
      if (lane == 0) {
        if (un.phase == 2 && chained) {
          // A2 rows of this token tile are complete once the gate/up tiles covering the
          // split's K range have counted in
          ready = wait_count(args.done + (e * g.splits + un.ks) * args.ntc + un.nt, split_need(g, un.ks),
                             args.status, &s_abort) ? 1 : 0;
        } else if (un.phase == 1 && !gathered) {
          // every CTA's share of xp must be written before the first gate/up tile
          ready = wait_count(args.sched + 1, static_cast<int>(gridDim.x), args.status, &s_abort) ? 1 : 0;
        }
        // rows written by generic stores; a TMA token load reads them through the async proxy
        if (ready && tma_b) asm volatile("fence.proxy.async;" ::: "memory");
      }
      ready = __shfl_sync(full, ready, 0);
      if (!ready) break;
      if (un.phase == 1) gathered = true;
      const T* src = un.phase == 1 ? xp : a2;
      for (int kb = un.kb0; kb < un.kb1; ++kb) {
        int got = 0;
        if (lane == 0) got = mbar_wait(&empty_bar[stage], phase ^ 1u, args.status, &s_abort) ? 1 : 0;
        got = __shfl_sync(full, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        const uint32_t sB = ring_base + stage * stage_bytes + kATileBytes;
        // per unit: a wide expert's tile by TMA, a narrow one (a few tokens) by cp.async of
        // just its rows; both give the barrier the same 192 arrivals
        if (tma_b && nb >= kTmaBMin) {
          // one thread loads ceil(nb / 64) boxes of 64 rows (same swizzled layout); the
          // other loader threads only arrive.  Rows past the expert's tokens belong to
          // the next expert (or are zero past the buffer) and are never stored.
          if (bt == 0) {
            const int boxes = (nb + 63) / 64;
            mbar_arrive_expect_tx(&fullB_bar[stage], static_cast<uint32_t>(boxes) * 64u * 128u);
            const CUtensorMap* mb = un.phase == 1 ? &tm_xp : &tm_a2;
            for (int j = 0; j < boxes; ++j) {
              tma_load_2d(dyn_smem + (sB - raw_base) + j * 64 * 128, mb, &fullB_bar[stage], kb * kBK,
                          row0 + n0 + j * 64, pol_rows);
            }
          } else {
            mbar_arrive(&fullB_bar[stage]);
          }
        } else {
          // nb rows x 8 chunks of 16 B, written with the 128-byte swizzle (chunk ^ row%8)
          for (int c = bt; c < nb * 8; c += kLoaderThreads) {
            const int r = c >> 3;
            const int q = c & 7;
            const bool valid = r < nlen;
            const T* p = valid ? src + static_cast<size_t>(row0 + n0 + r) * K + kb * kBK + q * 8 : src;
            cp_async_16(sB + r * 128 + ((q ^ (r & 7)) << 4), p, valid, pol_rows);
          }
          cp_async_arrive_noinc(&fullB_bar[stage]);
        }
        if (++stage == nstages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    cp_async_wait_all();
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;          // TMEM lane quarter this warp may read
    const int et = threadIdx.x - 32 * kEpiWarp0;  // 0..127
    // A2 rows are read back by the down units and the partials by the combine moments
    // later; keep them in L2 while the weight stream (evict-first) passes through
    const uint64_t pol_keep = policy_evict_last();
    int qi = 0;
    uint32_t qph = 0;
    int pass = 0;
    bool ok = true;
    while (ok) {
      // the leader reads the queue; the id is broadcast so all 128 threads agree
      if (et == 0) s_epi_unit = next_unit(qi, qph);
      named_bar_sync(1, 128);
      const int u = s_epi_unit;
      named_bar_sync(1, 128);
      if (u < 0) break;
      const Unit un = decode(u, g);
      if (un.phase == 3) {
        // the epilogue warps' share of the fix-up (the loader warps take the rest)
        int row0, n0, nlen;
        tile_tokens(un, row0, n0, nlen);
        if (et == 0) {
          s_epi_ok = wait_count(args.tile_done + (s_touched[un.te] * g.m2 + un.mt) * args.ntc + un.nt, g.splits,
                                args.status, &s_abort) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        ok = s_epi_ok != 0;
        named_bar_sync(1, 128);
        if (!ok) break;
        fixup_rows<T>(args, g.splits, un.mt, un.ks, row0 + n0, nlen, kLoaderThreads + et, kFixThreads);
        named_bar_sync(1, 128);
        if (et == 0) mbar_arrive(&fix_bar);
        continue;
      }
      const int e = s_touched[un.te];
      int row0, n0, nlen;
      tile_tokens(un, row0, n0, nlen);
      const int buf = pass % nbuf;
      if (et == 0) s_epi_ok = mbar_wait(&tfull_bar[buf], (pass / nbuf) & 1, args.status, &s_abort) ? 1 : 0;
      named_bar_sync(1, 128);
      ok = s_epi_ok != 0;
      named_bar_sync(1, 128);
      if (!ok) break;
      tc_fence_after();
      const uint32_t lane_base =
          tmem + (static_cast<uint32_t>(sub * 32) << 16) + static_cast<uint32_t>(buf * 256);
      // Each warp stages its 32 rows x 16 tokens in shared memory and writes 16-byte
      // vectors along the row (8 activations or 4 partials per store) instead of one
      // element per thread per token.
      uint8_t* stg = dyn_smem + (kDynSmem - kEpiStage) + sub * 2048;
      for (int c0 = 0; c0 < nlen; c0 += 16) {
        float va[16], vb[16];
        tmem_ld16x2(lane_base + static_cast<uint32_t>(c0), lane_base + acc1_off + static_cast<uint32_t>(c0), va, vb);
        const int nt = min(16, nlen - c0);
        if (un.phase == 1) {
          T* st = reinterpret_cast<T*>(stg);
#pragma unroll
          for (int i = 0; i < 16; ++i) st[i * 32 + lane] = from_f32<T>(silu_f32(va[i]) * vb[i]);
          __syncwarp();
#pragma unroll
          for (int j = lane; j < 64; j += 32) {  // 16 tokens x 4 chunks of 8 features
            const int i = j >> 2, q = j & 3;
            const int p = row0 + n0 + c0 + i;
            const int f = un.mt * 128 + sub * 32 + q * 8;
            if (i < nt && p >= 0 && p < args.Tk && f < I) {
              st_evict_last_v4(reinterpret_cast<T*>(args.a2) + static_cast<size_t>(p) * I + f,
                               *reinterpret_cast<const uint4*>(st + i * 32 + q * 8), pol_keep);
            }
          }
          __syncwarp();
        } else {
          float* st = reinterpret_cast<float*>(stg);
          auto put_rows = [&](const float (&v)[16], int half) {
#pragma unroll
            for (int i = 0; i < 16; ++i) st[i * 32 + lane] = v[i];
            __syncwarp();
#pragma unroll
            for (int j = lane; j < 128; j += 32) {  // 16 tokens x 8 chunks of 4 rows
              const int i = j >> 3, q = j & 7;
              const int p = row0 + n0 + c0 + i;
              const int h = un.mt * 256 + half * 128 + sub * 32 + q * 4;
              if (i < nt && p >= 0 && p < args.Tk && h < H) {
                st_evict_last_v4(args.part + (static_cast<size_t>(un.ks) * args.Tk + p) * H + h,
                                 *reinterpret_cast<const uint4*>(st + i * 32 + q * 4), pol_keep);
              }
            }
            __syncwarp();
          };
          put_rows(va, 0);
          put_rows(vb, 1);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[buf]);
      ++pass;
      if (un.phase == 2 && args.ep_C > 0) {
        // expert side of the exchange: publish this unit's partials (release at GPU
        // scope) and count it for its output tile; the tile's fix-up units sum them
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) atomicAdd(args.tile_done + (e * g.m2 + un.mt) * args.ntc + un.nt, 1);
      } else if (un.phase == 1 && chained) {
        // publish: this tile's A2 columns are written (release at GPU scope); count it
        // for every down split whose K range overlaps its 128 features
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) {
          const int f0 = un.mt * 2, f1 = min(un.mt * 2 + 2, g.kb2_total);
          for (int ks = 0; ks < g.splits; ++ks) {
            if (f0 < split_kb0(g, ks + 1) && f1 > split_kb0(g, ks))
              atomicAdd(args.done + (e * g.splits + ks) * args.ntc + un.nt, 1);
          }
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (s_abort) {
    // Unwind after a failed wait: let our own weight fills and MMAs land before the
    // shared and tensor memory they target is released.
    if (threadIdx.x == 0) {
      for (int i = s_consumed; i < s_issued; ++i) {
        mbar_wait(&fullA_bar[i % nstages], static_cast<uint32_t>((i / nstages) & 1), nullptr, nullptr);
      }
    }
    if (threadIdx.x == 32) {
      umma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, nullptr);
    }
    __syncthreads();
  }
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  const bool ret_p2p = args.ep_C > 0 && args.link.p2p;
  if (ret_p2p || args.recv_G > 0) {
    // the last CTA (system scope when it raises flags) zeroes the counters for the next
    // call when no router runs before it, and over peer memory raises each source's return
    // flag once every CTA's returned rows are stored (also after a failed wait, so that no
    // peer stalls)
    const bool last = ret_p2p ? last_cta_of_grid(args.link.ctrl + 2, &s_last_cta)
                              : last_cta_of_grid_gpu(args.exit_ticket, &s_last_cta);
    if (last) {
      if (args.recv_G > 0) {
        for (int i = threadIdx.x; i < args.ndone; i += blockDim.x) args.sched[i] = 0;
        __threadfence();
      }
      __syncthreads();
      if (ret_p2p && threadIdx.x == 0) {
        const int epoch = args.link.ctrl[0] + 1;
        raise_flags_sys(args.link.flag, args.link.nranks, epoch);
      }
    }
  }
  if (threadIdx.x == 0 && grid_timer_end(timers_of(args.status))) stage_busy(args.clk, 2);
}

// ---------------------------------------------------------------- host side

cudaError_t launch_ffn_gemm(bool bf16, int grid, cudaStream_t stream, bool pdl, const CUtensorMap& w13,
                            const CUtensorMap& w2, const CUtensorMap& xp, const CUtensorMap& a2, const FfnArgs& args) {
  static std::atomic<int> seen_bf16[64], seen_f16[64];
  const void* fn = bf16 ? reinterpret_cast<const void*>(&ffn_gemm_kernel<__nv_bfloat16>)
                        : reinterpret_cast<const void*>(&ffn_gemm_kernel<__half>);
  cudaError_t err = ensure_dyn_smem(fn, kDynSmem, bf16 ? seen_bf16 : seen_f16, 64);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kDynSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<CUtensorMap*>(&w13), const_cast<CUtensorMap*>(&w2), const_cast<CUtensorMap*>(&xp),
                    const_cast<CUtensorMap*>(&a2), const_cast<FfnArgs*>(&args)};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

}  // namespace smb
