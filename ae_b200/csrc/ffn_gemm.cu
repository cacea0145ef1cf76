// Expert FFN as two grouped, weight-streaming GEMMs on the 5th-generation tensor cores.
//
// Reference arithmetic: the Triton fused_moe_kernel (specmoe/layers/fused_moe_kernel.py:88-210)
// launched twice by stack_fused_moe (:332-342) with silu_and_mul in between (:337).
//
// Swap-AB: in the verify regime an expert sees 1..~100 tokens, so the weight rows fill
// the 128-row MMA M operand and the expert's tokens fill N (16..256).  Both operands
// are K-major bf16/f16 tiles staged by TMA with the 128-byte swizzle; the fp32
// accumulator lives in tensor memory.  One CTA per SM (persistent), warp-specialised:
//   warp 0      TMA producer (one thread)        weights evict-first, tokens evict-last
//   warp 1      MMA issuer (one thread)          tcgen05.mma, commits free the smem stage
//   warp 2      TMEM allocator
//   warps 4..7  epilogue (128 threads = 128 TMEM lanes)
//
// Mode kGateUp  (GEMM1): unit = (expert, 64 intermediate features).  The A tile stacks
//   64 rows of w1 (gate) over the matching 64 rows of w3 (up) from the page viewed as
//   [P*3I, H]; the epilogue forms silu(gate) * up in fp32 and stores the activation
//   row-block of A2 [Tk, I] (expert-major token order) in the storage dtype.
// Mode kDown    (GEMM2): unit = (expert, 128 hidden rows of w2, K split).  A tile = 128
//   rows of w2 from the page viewed as [P*3H, I] at row 2H (the w2_off of the reference),
//   B = the expert's rows of A2; fp32 partial sums go to part[split][p][h].
//
// Shape limits (checked by the host): H % 128 == 0, I % 64 == 0.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace smb {

namespace {

constexpr int kThreads = 256;
constexpr int kBK = 64;                      // K elements per stage = one 128 B swizzle row
constexpr int kATileBytes = 128 * kBK * 2;   // 128 weight rows
constexpr int kMaxN = 256;                   // tokens per MMA (N) and TMEM columns
constexpr int kTmemCols = 256;
constexpr int kMaxStages = 16;
constexpr int kXchgFloats = 16 * 64;         // GEMM1 epilogue gate/up exchange
constexpr int kDynSmem = 227 * 1024 - 3072;  // leaves room for the static shared block

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

struct Unit {
  int te;   // index into the touched-expert list
  int mt;   // row tile of the weight matrix
  int kb0;  // first 64-wide K block
  int kb1;  // one past the last K block
  int ks;   // split index (GEMM2)
};

template <int MODE>
__device__ __forceinline__ Unit decode_unit(int u, int m_tiles, int splits, int kb_total) {
  Unit r;
  if (MODE == kGateUp) {
    r.te = u / m_tiles;
    r.mt = u % m_tiles;
    r.ks = 0;
    r.kb0 = 0;
    r.kb1 = kb_total;
  } else {
    r.ks = u % splits;
    const int q = u / splits;
    r.te = q / m_tiles;
    r.mt = q % m_tiles;
    r.kb0 = static_cast<int>((static_cast<long long>(kb_total) * r.ks) / splits);
    r.kb1 = static_cast<int>((static_cast<long long>(kb_total) * (r.ks + 1)) / splits);
  }
  return r;
}

}  // namespace

template <int MODE, typename T>
__global__ void __launch_bounds__(kThreads, 1)
    ffn_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_b64,
                    const __grid_constant__ CUtensorMap tm_b32, const __grid_constant__ CUtensorMap tm_b16,
                    const FfnArgs args) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t dyn_smem[];
  __shared__ uint64_t full_bar[kMaxStages];
  __shared__ uint64_t empty_bar[kMaxStages];
  __shared__ uint64_t tfull_bar, tempty_bar, drain_bar;
  __shared__ uint32_t s_tmem;
  __shared__ int s_touched[kMaxExperts];
  __shared__ int s_page[kMaxExperts];
  __shared__ int s_ntouched, s_ncap, s_stages;
  __shared__ int s_abort, s_epi_ok, s_issued, s_consumed;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t raw_base = smem_u32(dyn_smem);
  const uint32_t ring_base = (raw_base + 1023u) & ~1023u;
  uint8_t* ring_gen = dyn_smem + (ring_base - raw_base);

  const int E = args.E, H = args.H, I = args.I;
  const int kb_total = (MODE == kGateUp) ? H / kBK : I / kBK;
  const int m_tiles = (MODE == kGateUp) ? I / 64 : H / 128;
  const int splits = (MODE == kGateUp) ? 1 : args.splits;

  if (threadIdx.x == 0) {
    s_abort = 0;
    s_issued = 0;
    s_consumed = 0;
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&tfull_bar, 1);
    mbar_init(&tempty_bar, 128);
    mbar_init(&drain_bar, 1);
    fence_mbarrier_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_b64);
    prefetch_tmap(&tm_b32);
    prefetch_tmap(&tm_b16);
  }
  if (warp == 2) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }

  // Everything above touched only this CTA's own shared and tensor memory; the
  // routing results and token rows come from the previous kernels in the stream.
  pdl_wait_prior_grids();

  if (threadIdx.x == 0) {
    int nt = 0, maxn = 0;
    for (int e = 0; e < E; ++e) {
      const int n = args.expert_off[e + 1] - args.expert_off[e];
      if (n > 0) {
        long long pg = args.page_of_expert[e];
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
    const int stage_bytes = kATileBytes + ncap * 128;
    const int ring = kDynSmem - 1024 - static_cast<int>(sizeof(float)) * kXchgFloats;
    s_ntouched = nt;
    s_ncap = ncap;
    s_stages = min(kMaxStages, ring / stage_bytes);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();

  const uint32_t tmem = s_tmem;
  const int ncap = s_ncap;
  const int nstages = s_stages;
  const int stage_bytes = kATileBytes + ncap * 128;
  const int total_units = s_ntouched * m_tiles * splits;
  float* xchg = reinterpret_cast<float*>(ring_gen + nstages * stage_bytes);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < total_units; u += gridDim.x) {
        const Unit un = decode_unit<MODE>(u, m_tiles, splits, kb_total);
        const int e = s_touched[un.te];
        const int page = s_page[un.te];
        const int row0 = args.expert_off[e];
        const int n_e = args.expert_off[e + 1] - row0;
        const int wrow = (MODE == kGateUp) ? page * 3 * I + un.mt * 64 : page * 3 * H + 2 * H + un.mt * 128;
        for (int n0 = 0; ok && n0 < n_e; n0 += ncap) {
          const int nlen = min(ncap, n_e - n0);
          const int nb = (nlen + 15) & ~15;
          for (int kb = un.kb0; kb < un.kb1; ++kb) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1u, args.status, &s_abort)) {
              ok = false;
              break;
            }
            uint8_t* sA = ring_gen + stage * stage_bytes;
            uint8_t* sB = sA + kATileBytes;
            mbar_arrive_expect_tx(&full_bar[stage], kATileBytes + nb * 128);
            if (MODE == kGateUp) {
              tma_load_2d(sA, &tm_w, &full_bar[stage], kb * kBK, wrow, pol_w);
              tma_load_2d(sA + kATileBytes / 2, &tm_w, &full_bar[stage], kb * kBK, wrow + I, pol_w);
            } else {
              tma_load_2d(sA, &tm_w, &full_bar[stage], kb * kBK, wrow, pol_w);
            }
            int r = 0;
            const int brow = row0 + n0;
            for (; r + 64 <= nb; r += 64) tma_load_2d(sB + r * 128, &tm_b64, &full_bar[stage], kb * kBK, brow + r, pol_b);
            if (r + 32 <= nb) {
              tma_load_2d(sB + r * 128, &tm_b32, &full_bar[stage], kb * kBK, brow + r, pol_b);
              r += 32;
            }
            if (r + 16 <= nb) {
              tma_load_2d(sB + r * 128, &tm_b16, &full_bar[stage], kb * kBK, brow + r, pol_b);
              r += 16;
            }
            ++issued;
            if (++stage == nstages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      s_issued = issued;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, tphase = 0;
      int consumed = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < total_units; u += gridDim.x) {
        const Unit un = decode_unit<MODE>(u, m_tiles, splits, kb_total);
        const int e = s_touched[un.te];
        const int n_e = args.expert_off[e + 1] - args.expert_off[e];
        for (int n0 = 0; ok && n0 < n_e; n0 += ncap) {
          const int nlen = min(ncap, n_e - n0);
          const int nb = (nlen + 15) & ~15;
          const uint32_t idesc = idesc_f16(kBF16, 128, nb);
          if (!mbar_wait(&tempty_bar, tphase ^ 1u, args.status, &s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int kb = un.kb0; kb < un.kb1; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase, args.status, &s_abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = ring_base + stage * stage_bytes;
            const uint64_t ad = desc_kmajor_sw128(a_addr);
            const uint64_t bd = desc_kmajor_sw128(a_addr + kATileBytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              // +32 bytes along K inside the swizzle row = +2 in the encoded start address
              umma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kb > un.kb0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&empty_bar[stage]);
            ++consumed;
            if (++stage == nstages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(&tfull_bar);
          tphase ^= 1u;
        }
      }
      s_consumed = consumed;
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;          // TMEM lane quarter this warp may read
    const int row = sub * 32 + lane;   // accumulator row = TMEM lane
    const int et = threadIdx.x - 128;  // 0..127
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(sub * 32) << 16);
    uint32_t tphase = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
      const Unit un = decode_unit<MODE>(u, m_tiles, splits, kb_total);
      const int e = s_touched[un.te];
      const int row0 = args.expert_off[e];
      const int n_e = args.expert_off[e + 1] - row0;
      bool ok = true;
      for (int n0 = 0; n0 < n_e; n0 += ncap) {
        const int nlen = min(ncap, n_e - n0);
        if (et == 0) s_epi_ok = mbar_wait(&tfull_bar, tphase, args.status, &s_abort) ? 1 : 0;
        named_bar_sync(1, 128);
        ok = s_epi_ok != 0;
        named_bar_sync(1, 128);
        if (!ok) break;
        tc_fence_after();
        for (int c0 = 0; c0 < nlen; c0 += 16) {
          float v[16];
          tmem_ld16(lane_addr + static_cast<uint32_t>(c0), v);
          if (MODE == kGateUp) {
            if (sub >= 2) {
#pragma unroll
              for (int i = 0; i < 16; ++i) xchg[i * 64 + (row - 64)] = v[i];
            }
            named_bar_sync(1, 128);
            if (sub < 2) {
              T* a2 = reinterpret_cast<T*>(args.out);
              const size_t col = static_cast<size_t>(un.mt) * 64 + row;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if (c0 + i < nlen) {
                  const float up = xchg[i * 64 + row];
                  a2[static_cast<size_t>(row0 + n0 + c0 + i) * I + col] = from_f32<T>(silu_f32(v[i]) * up);
                }
              }
            }
            named_bar_sync(1, 128);
          } else {
            float* part = reinterpret_cast<float*>(args.out);
            const size_t h = static_cast<size_t>(un.mt) * 128 + row;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              if (c0 + i < nlen) {
                part[(static_cast<size_t>(un.ks) * args.Tk + row0 + n0 + c0 + i) * H + h] = v[i];
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar);
        tphase ^= 1u;
      }
      if (!ok) break;
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (s_abort) {
    // Unwind after a failed wait: let our own TMA fills and MMAs land before the
    // shared and tensor memory they target is released.
    if (threadIdx.x == 0) {
      for (int i = s_consumed; i < s_issued; ++i) {
        mbar_wait(&full_bar[i % nstages], static_cast<uint32_t>((i / nstages) & 1), nullptr, nullptr);
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
}

// ---------------------------------------------------------------- host side

static cudaError_t launch_one(const void* fn, int grid, cudaStream_t stream, bool pdl, const CUtensorMap& a,
                              const CUtensorMap& b64, const CUtensorMap& b32, const CUtensorMap& b16,
                              const FfnArgs& args) {
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
  void* params[] = {const_cast<CUtensorMap*>(&a), const_cast<CUtensorMap*>(&b64), const_cast<CUtensorMap*>(&b32),
                    const_cast<CUtensorMap*>(&b16), const_cast<FfnArgs*>(&args)};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

template <int MODE, typename T>
static cudaError_t launch_mode(int grid, cudaStream_t stream, bool pdl, const CUtensorMap& a, const CUtensorMap& b64,
                               const CUtensorMap& b32, const CUtensorMap& b16, const FfnArgs& args) {
  const void* fn = reinterpret_cast<const void*>(&ffn_gemm_kernel<MODE, T>);
  cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem);
  if (err != cudaSuccess) return err;
  return launch_one(fn, grid, stream, pdl, a, b64, b32, b16, args);
}

cudaError_t launch_ffn_gemm(int mode, bool bf16, int grid, cudaStream_t stream, bool pdl, const CUtensorMap& a,
                            const CUtensorMap& b64, const CUtensorMap& b32, const CUtensorMap& b16,
                            const FfnArgs& args) {
  if (mode == kGateUp) {
    return bf16 ? launch_mode<kGateUp, __nv_bfloat16>(grid, stream, pdl, a, b64, b32, b16, args)
                : launch_mode<kGateUp, __half>(grid, stream, pdl, a, b64, b32, b16, args);
  }
  return bf16 ? launch_mode<kDown, __nv_bfloat16>(grid, stream, pdl, a, b64, b32, b16, args)
              : launch_mode<kDown, __half>(grid, stream, pdl, a, b64, b32, b16, args);
}

int ffn_units(int mode, int E, int H, int I, int splits) {
  return mode == kGateUp ? E * (I / 64) : E * (H / 128) * splits;
}

}  // namespace smb
