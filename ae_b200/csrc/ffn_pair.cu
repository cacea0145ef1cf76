// Expert FFN for prefill-sized calls (hundreds of tokens per expert) on CTA pairs: the
// 5th-generation tensor cores' 2-SM MMA (tcgen05.mma.cta_group::2), M = 256 weight rows
// across the pair and N up to 256 tokens, so each SM holds half the token tile.
//
// Reference arithmetic: the Triton fused_moe_kernel (specmoe/layers/fused_moe_kernel.py:88-210)
// launched twice by stack_fused_moe (:332-342) with silu_and_mul in between (:337); the
// reference sends prefill through the same call (specmoe/backend/execution_engine.py:947,
// large-token tile configs at fused_moe_kernel.py:290-306).
//
// Why a second kernel.  At a few tokens per expert the layer streams weights and the
// verify kernel (ffn_gemm.cu) runs at the HBM roofline; at 256+ tokens per expert the
// tensor pipe bounds it, and what limits the verify kernel there is operand traffic per
// SM: each SM reads 256 weight rows and the whole token tile per K step for its 256 x N
// outputs.  Here a pair of SMs computes 2 x 256 x N outputs per K step; each SM reads its
// own 256 weight rows (gate and up of 128 features, or two 128-row blocks of w2) and only
// half of the token tile: 48 KB per 64-wide K step for 8.4 MFLOP per SM, 25 % fewer bytes
// per flop.  Two launches: gate/up (phase 1, SiLU*mul in the epilogue, activations in
// storage dtype) then down (phase 2, split-K fp32 partials for the combine kernel; 32 KB
// per K step for 4.2 MFLOP per SM, double-buffered accumulators).
//
// Per pair and unit (CTA rank r = 0 leader, 1 peer):
//   phase 1: features [f0 + 128 r, +128) of w1 (gate) and w3 (up), tokens [n0, n0 + nb):
//     accumulators gate [128 lanes x nb] at TMEM column 0 and up at column 256 in each
//     CTA; lane l of CTA r holds feature f0 + 128 r + l, so SiLU*mul is local;
//   phase 2: rows [h0 + 128 r, +128) of w2 over the split's K range: one accumulator per
//     unit (row h0 + 128 r + l), two TMEM buffers, so the next unit's MMAs run while the
//     epilogue drains the last; 256-row units also make twice as many units as 512-row
//     ones, which the down launch needs to spread over the pairs in small waves (with
//     512-row units 24 % of the SM time sat in the last partial wave).
// Shared memory per stage and CTA: the unit's 128-row weight boxes and nb/2 token rows (two
// 64-row boxes), all by TMA; both CTAs' bytes complete on the leader's full barrier, the
// leader's MMA thread commits to both CTAs' empty barriers and TMEM-full barriers, and
// both epilogues release the accumulators on the leader's TMEM-empty barrier.
// Units are spread over the pairs statically (unit = pair + i * pairs), so both CTAs of
// a pair walk the same list without talking.  The gate/up accumulators are single-
// buffered (512 columns for two N = 256 accumulators).
//
// Every wait is bounded; after a failed wait the CTA stops, waits a bounded time for its
// copies in flight, meets its peer and frees its TMEM.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace smb {

namespace {

constexpr int kPThreads = 192;                // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kPBK = 64;
constexpr int kPBox = 128 * kPBK * 2;         // 16 KB: 128 rows x 64 K
constexpr int kPEpiStage = 4 * 2048;
constexpr int kPRing = 192 * 1024;            // stage ring per CTA
constexpr int kPDynSmem = kPRing + 1024 + kPEpiStage;
constexpr int kPTmemCols = 512;
constexpr int kPMaxStages = 6;

// Per launch: gate/up units hold two accumulators (gate, up: 2 x 256 columns = all of TMEM,
// one buffer); down units one accumulator of 256 rows (128 per CTA), double-buffered, so
// the MMA of the next unit overlaps the epilogue of the last and twice as many units
// spread the down launch over the pairs in smaller waves.
template <int kPhase>
struct PairShape {
  static constexpr int kAccs = kPhase == 1 ? 2 : 1;        // weight boxes / accumulators per unit
  static constexpr int kBufs = kPhase == 1 ? 1 : 2;        // TMEM buffers
  static constexpr int kStageBytes = (kAccs + 1) * kPBox;  // weight boxes + 128 token rows
  static constexpr int kStages = kPRing / kStageBytes;     // 4 / 6
  static_assert(kStages <= kPMaxStages, "stage barriers");
};

__device__ __forceinline__ void pair_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_evict_last_v4p(void* p, const uint4& v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w), "l"(pol)
               : "memory");
}

struct PairUnit {
  int te, mt, nt, ks, kb0, kb1;
};

}  // namespace

template <typename T, int kPhase>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    ffn_pair_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_tok,
                    const FfnArgs args) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  using St = PairShape<kPhase>;
  constexpr int kStages = St::kStages;
  constexpr int kStageBytes = St::kStageBytes;
  extern __shared__ uint8_t dyn_smem[];
  __shared__ uint64_t full_bar[kPMaxStages], empty_bar[kPMaxStages], tfull_bar[2], tempty_bar[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_touched[kMaxExperts];
  __shared__ int s_page[kMaxExperts];
  __shared__ int s_ntp[kMaxExperts + 1];
  __shared__ int s_ntouched, s_abort, s_epi_ok;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_index_x());
  const int pairs = static_cast<int>(cluster_count_x());
  const uint32_t raw_base = smem_u32(dyn_smem);
  const uint32_t ring_base = (raw_base + 1023u) & ~1023u;
  uint8_t* ring = dyn_smem + (ring_base - raw_base);
  const int E = args.E, H = args.H, I = args.I;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < St::kBufs; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2);  // one arrival from each CTA's epilogue
    }
    fence_mbarrier_init();
  }
  if (threadIdx.x == 32) prefetch_tmap(&tm_w), prefetch_tmap(&tm_tok);
  if (warp == 1) {
    tmem_alloc_pair(&s_tmem, kPTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // both CTAs' barriers exist before any remote arrival, commit or TMA completion
  cluster_sync_all();
  tc_fence_after();

  pdl_wait_prior_grids();
  // the FFN timer spans both launches: started by the gate/up grid, ended by the down grid
  if (threadIdx.x == 0 && kPhase == 1) grid_timer_begin(timers_of(args.status));
  if (threadIdx.x == 0 && blockIdx.x == 0 && kPhase == 1) stage_mark(args.clk, 2);
  if (threadIdx.x == 0) {
    int nt = 0;
    s_ntp[0] = 0;
    for (int e = 0; e < E; ++e) {
      const int n = args.expert_off[e + 1] - args.expert_off[e];
      if (n <= 0) continue;
      const long long pg = args.page_of_expert[e];
      if (pg < 0 || pg >= args.num_pages) {
        record_status(args.status, kDevBadPage);
        continue;
      }
      s_touched[nt] = e;
      s_page[nt] = static_cast<int>(pg);
      s_ntp[nt + 1] = s_ntp[nt] + min(args.ntc, (n + 255) / 256);
      ++nt;
    }
    s_ntouched = nt;
  }
  __syncthreads();
  pdl_launch_dependents();

  // phase 1: every CTA gathers its share of the token rows into xp (expert-major), then
  // counts itself in; the TMA producers wait for all CTAs before the first token tile
  if (kPhase == 1) {
    const int Tk = args.Tk;
    const int per = (Tk + gridDim.x - 1) / gridDim.x;
    const int f0 = min(Tk, static_cast<int>(blockIdx.x) * per), f1 = min(Tk, f0 + per);
    const int vec = H * static_cast<int>(sizeof(T)) / 16;
    const uint4* xs = reinterpret_cast<const uint4*>(args.x);
    uint4* xd = reinterpret_cast<uint4*>(args.xp);
    const int nvec = (f1 - f0) * vec;
    for (int i = threadIdx.x; i < nvec; i += kPThreads) {
      const int f = f0 + i / vec;
      const int p = args.inv[f];
      if (p < 0 || p >= Tk) continue;
      xd[static_cast<size_t>(p) * vec + (i % vec)] = __ldg(xs + static_cast<size_t>(f / args.k) * vec + (i % vec));
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(args.sched + 1, 1);
  }

  const int ntouched = s_ntouched;
  const int tiles = s_ntp[ntouched];
  // phase 1: 256 features per pair unit; phase 2: 256 rows of w2 per pair unit, split-K
  const int mt_n = kPhase == 1 ? (I + 255) / 256 : (H + 255) / 256;
  const int S = kPhase == 1 ? 1 : args.splits;
  const int kbt = (kPhase == 1 ? H : I) / kPBK;
  const int total = tiles * mt_n * S;

  auto decode = [&](int u) -> PairUnit {
    PairUnit r;
    const int per_tile = mt_n * S;
    const int q = u / per_tile;  // global token tile index (expert-major)
    int lo = 0, hi = ntouched;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_ntp[mid] <= q) lo = mid; else hi = mid;
    }
    r.te = lo;
    const int nte = s_ntp[lo + 1] - s_ntp[lo];
    const int v = u - s_ntp[lo] * per_tile;
    // order inside an expert: split, row/feature tile, token tile (token tiles of the same
    // weight rows run on neighbouring pairs at about the same time and share them in L2)
    r.ks = v / (mt_n * nte);
    const int w = v - r.ks * mt_n * nte;
    r.mt = w / nte;
    r.nt = w - r.mt * nte;
    r.kb0 = static_cast<int>((static_cast<long long>(kbt) * r.ks) / S);
    r.kb1 = static_cast<int>((static_cast<long long>(kbt) * (r.ks + 1)) / S);
    return r;
  };
  auto tokens_of = [&](const PairUnit& un, int& row0, int& n0, int& nlen) {
    const int e = s_touched[un.te];
    row0 = args.expert_off[e];
    n0 = un.nt * 256;
    nlen = min(256, args.expert_off[e + 1] - row0 - n0);
  };

  int issued = 0, consumed = 0;
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_t = policy_evict_last();
      int stage = 0;
      uint32_t ph = 0;
      bool ok = true;
      if (kPhase == 1) {
        // every CTA's share of xp must be written before the first token tile
        const uint64_t t0 = global_timer_ns();
        while (ld_acquire_gpu(args.sched + 1) < static_cast<int>(gridDim.x)) {
          if (global_timer_ns() - t0 > kWaitBudgetNs) {
            record_status(args.status, kDevTimeout);
            s_abort = 1;
            ok = false;
            break;
          }
          __nanosleep(64);
        }
        // xp was written by generic stores; the TMA reads it through the async proxy
        asm volatile("fence.proxy.async;" ::: "memory");
      }
      for (int u = pair; ok && u < total; u += pairs) {
        const PairUnit un = decode(u);
        int row0, n0, nlen;
        tokens_of(un, row0, n0, nlen);
        const int nb = (nlen + 31) & ~31;
        const int page = s_page[un.te];
        const int rA0 = kPhase == 1 ? page * 3 * I + un.mt * 256 + static_cast<int>(rank) * 128
                                    : page * 3 * H + 2 * H + un.mt * 256 + static_cast<int>(rank) * 128;
        const int rA1 = rA0 + I;  // up rows (gate/up units only)
        const int rB = row0 + n0 + static_cast<int>(rank) * (nb / 2);
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], ph ^ 1u, args.status, &s_abort)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + stage * kStageBytes;
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2u * kStageBytes);
          const uint32_t bar = map_shared_rank(smem_u32(&full_bar[stage]), 0);
          tma_load_2d_pair(st, &tm_w, bar, kb * kPBK, rA0, pol_w);
          if (St::kAccs == 2) tma_load_2d_pair(st + kPBox, &tm_w, bar, kb * kPBK, rA1, pol_w);
          uint8_t* sb = st + St::kAccs * kPBox;
          tma_load_2d_pair(sb, &tm_tok, bar, kb * kPBK, rB, pol_t);
          tma_load_2d_pair(sb + kPBox / 2, &tm_tok, bar, kb * kPBK, rB + 64, pol_t);
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      // tail: every stage's last release (a commit the leader's MMA thread aims at this
      // CTA's empty barrier) has arrived before this CTA may go
      for (int i = 0; ok && i < kStages; ++i) {
        if (!mbar_wait(&empty_bar[stage], ph ^ 1u, args.status, &s_abort)) break;
        if (++stage == kStages) {
          stage = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      const uint32_t tmem = s_tmem;
      int stage = 0;
      uint32_t ph = 0;
      int ul = 0;
      bool ok = true;

      for (int u = pair; ok && u < total; u += pairs, ++ul) {
        const PairUnit un = decode(u);
        int row0, n0, nlen;
        tokens_of(un, row0, n0, nlen);
        const int nb = (nlen + 31) & ~31;
        const uint32_t idesc = idesc_f16(kBF16, 256, nb);
        const int buf = ul % St::kBufs;
        if (!mbar_wait(&tempty_bar[buf], ((ul / St::kBufs) & 1) ^ 1u, args.status, &s_abort)) break;
        tc_fence_after();
        const uint32_t acc0 = tmem + static_cast<uint32_t>(buf * 256);
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], ph, args.status, &s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = ring_base + stage * kStageBytes;
          const uint64_t ad0 = desc_kmajor_sw128(a);
          const uint64_t ad1 = desc_kmajor_sw128(a + kPBox);
          const uint64_t bd = desc_kmajor_sw128(a + St::kAccs * kPBox);
#pragma unroll
          for (int kk = 0; kk < kPBK / 16; ++kk) {
            const uint32_t acc = (kb > un.kb0 || kk > 0) ? 1u : 0u;
            umma_f16_pair(acc0, ad0 + 2 * kk, bd + 2 * kk, idesc, acc);
            if (St::kAccs == 2) umma_f16_pair(tmem + 256u, ad1 + 2 * kk, bd + 2 * kk, idesc, acc);
          }
          // the stage is free in both CTAs once these MMAs have read it
          umma_commit_pair(smem_u32(&empty_bar[stage]));
          umma_commit_pair(map_shared_rank(smem_u32(&empty_bar[stage]), 1));
          ++consumed;
          if (++stage == kStages) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&tfull_bar[buf]));
        umma_commit_pair(map_shared_rank(smem_u32(&tfull_bar[buf]), 1));
      }
      // tail: both epilogues' last releases of every buffer (one of them remote) have arrived
      for (int j = ul - St::kBufs; ok && j < ul; ++j) {
        if (j >= 0) mbar_wait(&tempty_bar[j % St::kBufs], (j / St::kBufs) & 1, args.status, &s_abort);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;            // TMEM lanes this warp may read
    const int et = threadIdx.x - 64;         // 0..127
    const uint64_t pol_keep = policy_evict_last();

    uint8_t* stg = dyn_smem + (kPDynSmem - kPEpiStage) + quarter * 2048;
    int ul = 0;
    for (int u = pair; u < total; u += pairs, ++ul) {
      const PairUnit un = decode(u);
      int row0, n0, nlen;
      tokens_of(un, row0, n0, nlen);
      const int buf = ul % St::kBufs;
      if (et == 0) s_epi_ok = mbar_wait(&tfull_bar[buf], (ul / St::kBufs) & 1, args.status, &s_abort) ? 1 : 0;
      pair_bar_sync(1, 128);
      const bool ok = s_epi_ok != 0;
      pair_bar_sync(1, 128);
      if (!ok) break;
      tc_fence_after();
      const uint32_t lane_base = s_tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * 256);
      for (int c0 = 0; c0 < nlen; c0 += 16) {
        float va[16], vb[16];
        if (kPhase == 1) {
          tmem_ld16x2(lane_base + static_cast<uint32_t>(c0), lane_base + 256u + static_cast<uint32_t>(c0), va, vb);
        } else {
          tmem_ld16(lane_base + static_cast<uint32_t>(c0), va);
        }
        const int nt = min(16, nlen - c0);
        if (kPhase == 1) {
          // activations of 32 features x 16 tokens through shared memory, 16-byte stores
          T* st = reinterpret_cast<T*>(stg);
#pragma unroll
          for (int i = 0; i < 16; ++i) st[i * 32 + lane] = from_f32<T>(silu_f32(va[i]) * vb[i]);
          __syncwarp();
#pragma unroll
          for (int j = lane; j < 64; j += 32) {
            const int i = j >> 2, q = j & 3;
            const int p = row0 + n0 + c0 + i;
            const int f = un.mt * 256 + static_cast<int>(rank) * 128 + quarter * 32 + q * 8;
            if (i < nt && p < args.Tk && f < I) {
              st_evict_last_v4p(reinterpret_cast<T*>(args.a2) + static_cast<size_t>(p) * I + f,
                                *reinterpret_cast<const uint4*>(st + i * 32 + q * 8), pol_keep);
            }
          }
          __syncwarp();
        } else {
          float* st = reinterpret_cast<float*>(stg);
          auto put_rows = [&](const float (&v)[16], int hbase) {
#pragma unroll
            for (int i = 0; i < 16; ++i) st[i * 32 + lane] = v[i];
            __syncwarp();
#pragma unroll
            for (int j = lane; j < 128; j += 32) {
              const int i = j >> 3, q = j & 7;
              const int p = row0 + n0 + c0 + i;
              const int h = hbase + quarter * 32 + q * 4;
              if (i < nt && p < args.Tk && h < H) {
                st_evict_last_v4p(args.part + (static_cast<size_t>(un.ks) * args.Tk + p) * H + h,
                                  *reinterpret_cast<const uint4*>(st + i * 32 + q * 4), pol_keep);
              }
            }
            __syncwarp();
          };
          put_rows(va, un.mt * 256 + static_cast<int>(rank) * 128);
        }
      }
      // this CTA's half of the accumulators is drained: tell the leader's MMA thread
      tc_fence_before();
      pair_bar_sync(1, 128);
      if (et == 0) mbar_arrive_cluster(map_shared_rank(smem_u32(&tempty_bar[buf]), 0));
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (s_abort) {
    // after a failed wait: give this CTA's copies in flight (bounded) time to land; the
    // leader also drains the stages it saw issued
    if (threadIdx.x == 0) {
      const uint64_t t0 = global_timer_ns();
      while (global_timer_ns() - t0 < 200000ull) __nanosleep(1000);
    }
    __syncthreads();
  }
  // neither CTA's shared memory or TMEM may go while the peer can still reach it
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(s_tmem, kPTmemCols);
  if (threadIdx.x == 0 && kPhase == 2 && grid_timer_end(timers_of(args.status))) stage_busy(args.clk, 2);
  (void)issued;
  (void)consumed;
}

// ---------------------------------------------------------------- host side

template <typename T, int kPhase>
static cudaError_t launch_pair(int pairs, cudaStream_t stream, bool pdl, const CUtensorMap& w, const CUtensorMap& tok,
                               const FfnArgs& args) {
  static std::atomic<int> seen[64];
  const void* fn = reinterpret_cast<const void*>(&ffn_pair_kernel<T, kPhase>);
  cudaError_t err = ensure_dyn_smem(fn, kPDynSmem, seen, 64);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPDynSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<CUtensorMap*>(&w), const_cast<CUtensorMap*>(&tok), const_cast<FfnArgs*>(&args)};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

// CTA pairs that can be resident at once (the phase-1 grid counter needs all of them).
int ffn_pair_capacity(bool bf16) {
  static std::atomic<int> cap[2][64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::atomic<int>& slot = cap[bf16 ? 1 : 0][dev];
  int c = slot.load();
  if (c > 0) return c;
  const void* fn = bf16 ? reinterpret_cast<const void*>(&ffn_pair_kernel<__nv_bfloat16, 1>)
                        : reinterpret_cast<const void*>(&ffn_pair_kernel<__half, 1>);
  static std::atomic<int> seen[2][64];
  if (ensure_dyn_smem(fn, kPDynSmem, seen[bf16 ? 1 : 0], 64) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPDynSmem;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) return 0;
  slot.store(n);
  return n;
}

cudaError_t launch_ffn_pair(bool bf16, int phase, int pairs, cudaStream_t stream, bool pdl, const CUtensorMap& w,
                            const CUtensorMap& tok, const FfnArgs& args) {
  if (bf16) {
    return phase == 1 ? launch_pair<__nv_bfloat16, 1>(pairs, stream, pdl, w, tok, args)
                      : launch_pair<__nv_bfloat16, 2>(pairs, stream, pdl, w, tok, args);
  }
  return phase == 1 ? launch_pair<__half, 1>(pairs, stream, pdl, w, tok, args)
                    : launch_pair<__half, 2>(pairs, stream, pdl, w, tok, args);
}

}  // namespace smb
