// Weighted combine back to token order, and the block-padded permutation.
//
// combine: out[t, h] = sum_j w[t, j] * sum_s part[s][inv[t*k+j]][h], summed in that fixed
// order in fp32 and rounded once to the storage dtype.  The reference applies the
// routing weight in the down-projection epilogue (specmoe/layers/fused_moe_kernel.py:197-201)
// and sums the k slots with torch.sum into hidden_states (:344-347); here the weight is
// applied while the split-K partials are reduced, which keeps the result deterministic.
//
// align: the moe_align_block_size contract (specmoe/layers/fused_moe_kernel.py:16-85):
// flat ids sorted by expert (ascending flat index inside an expert), each expert padded
// to a multiple of block_size with the value numel, expert id per block, padded total.
#include "common.cuh"
#include "kernels.h"

namespace smb {

namespace {

constexpr int kCombineThreads = 256;

// out[t, 4 columns] in the storage dtype from the fp32 sum.
template <typename TO>
__device__ __forceinline__ void store4(const CombineArgs& a, int t, int h4, const float4& acc) {
  TO* out = reinterpret_cast<TO*>(a.out) + static_cast<size_t>(t) * a.H;
  union {
    TO h[4];
    uint2 u;
  } pack;
  pack.h[0] = from_f32<TO>(acc.x);
  pack.h[1] = from_f32<TO>(acc.y);
  pack.h[2] = from_f32<TO>(acc.z);
  pack.h[3] = from_f32<TO>(acc.w);
  *reinterpret_cast<uint2*>(out + static_cast<size_t>(h4) * 4) = pack.u;
}

// k <= 2 and S <= kCombineSplits (the usual top-2 layers): both slots' positions and weights
// first, then every split partial of both slots at once, so a thread waits for two memory
// round trips instead of two per slot; the sums run in the same order as combine_one's.
// (A bound of 4 splits keeps the registers low enough for several CTAs per SM.)
constexpr int kCombineSplits = 4;
template <typename TO>
__device__ __forceinline__ void combine_two(const CombineArgs& a, int t, int h4) {
  const size_t Tk = static_cast<size_t>(a.T) * a.k;
  const size_t split_stride = Tk * a.H / 4;  // float4 elements between splits
  int p[2];
  float wj[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    p[j] = -1;
    wj[j] = 0.f;
    if (j < a.k) {
      const size_t f = static_cast<size_t>(t) * a.k + j;
      const int pj = a.inv[f];
      if (pj >= 0 && static_cast<size_t>(pj) < Tk) {  // else only after a failed or skipped route
        p[j] = pj;
        wj[j] = a.w[f];
      }
    }
  }
  float4 v[2][kCombineSplits];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float4* src = reinterpret_cast<const float4*>(a.part + static_cast<size_t>(p[j] < 0 ? 0 : p[j]) * a.H) + h4;
#pragma unroll
    for (int sp = 0; sp < kCombineSplits; ++sp) {
      if (p[j] >= 0 && sp < a.splits) v[j][sp] = __ldg(src + sp * split_stride);
    }
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    if (p[j] < 0) continue;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int sp = 0; sp < kCombineSplits; ++sp) {
      if (sp < a.splits) {
        s.x += v[j][sp].x;
        s.y += v[j][sp].y;
        s.z += v[j][sp].z;
        s.w += v[j][sp].w;
      }
    }
    acc.x += wj[j] * s.x;
    acc.y += wj[j] * s.y;
    acc.z += wj[j] * s.z;
    acc.w += wj[j] * s.w;
  }
  store4<TO>(a, t, h4, acc);
}

template <typename TO>
__device__ __forceinline__ void combine_one(const CombineArgs& a, int t, int h4) {
  const size_t Tk = static_cast<size_t>(a.T) * a.k;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < a.k; ++j) {
    const size_t f = static_cast<size_t>(t) * a.k + j;
    const int p = a.inv[f];
    if (p < 0 || static_cast<size_t>(p) >= Tk) continue;  // only after a failed or skipped route
    const float wj = a.w[f];
    const float4* src = reinterpret_cast<const float4*>(a.part + static_cast<size_t>(p) * a.H) + h4;
    const size_t split_stride = Tk * a.H / 4;  // float4 elements between splits
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    int sp = 0;
    // the splits in a fixed order, four independent loads in flight
    for (; sp + 4 <= a.splits; sp += 4) {
      float4 v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = __ldg(src + (sp + q) * split_stride);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        s.x += v[q].x;
        s.y += v[q].y;
        s.z += v[q].z;
        s.w += v[q].w;
      }
    }
    for (; sp < a.splits; ++sp) {
      const float4 v = __ldg(src + sp * split_stride);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    acc.x += wj * s.x;
    acc.y += wj * s.y;
    acc.z += wj * s.z;
    acc.w += wj * s.w;
  }
  store4<TO>(a, t, h4, acc);
}

template <typename TO>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const CombineArgs a) {
  pdl_wait_prior_grids();
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) stage_mark(a.clk, 3);
  pdl_launch_dependents();
  const int t = blockIdx.y;
  const int h4 = blockIdx.x * kCombineThreads + threadIdx.x;
  if (h4 * 4 < a.H) {
    if (a.k <= 2 && a.splits <= kCombineSplits) {
      combine_two<TO>(a, t, h4);
    } else {
      combine_one<TO>(a, t, h4);
    }
  }
}

// Weighted combine of per-slot rows: out[t, h] = sum_j w[t, j] * rows[inv[t*k+j]][h], in
// that order in fp32, rows in the storage dtype: the expert outputs of the expert-parallel
// path returned by the exchange, where the dispatch recorded in inv each slot's row of the
// returned rows [G][C] (rank d = expert / E_loc, row within d's chunk), or per-slot rows in
// expert-major order, where inv holds the slot's position.
//
// A CTA takes a contiguous range of tokens.  The row and weight of each of its slots are
// read before the wait for the returned rows (they depend only on this rank's own
// routing), then each thread loads all k rows' parts of up to kCombineVec 16-byte columns of
// a token at once, so a token costs one memory round trip.  Over peer memory thread 0 first
// waits (bounded) for every expert rank's return flag; the grid's last CTA advances the
// epoch (GPU scope: only this rank's kernels read it).
constexpr int kCombineVec = 4;        // 16-byte columns per thread per pass (H <= 8192 in one)
constexpr int kCombineSlots = 256;    // slots of a CTA's token range (the launch keeps it below)

template <typename TO>
__global__ void __launch_bounds__(kCombineThreads) combine_rows_kernel(const void* rows_v, const int32_t* inv,
                                                                        const float* w, void* out_v, int T, int k,
                                                                        int H, long long nrows, const EpLink link,
                                                                        int* status, StageClock* clk) {
  __shared__ long long s_row[kCombineSlots];
  __shared__ float s_w[kCombineSlots];
  __shared__ int s_ok, s_last;
  pdl_wait_prior_grids();
  if (blockIdx.x == 0 && threadIdx.x == 0) stage_mark(clk, 4);
  pdl_launch_dependents();
  const int per = (T + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int t0 = min(T, static_cast<int>(blockIdx.x) * per);
  const int t1 = min(T, t0 + per);
  const int nslot = min(kCombineSlots, (t1 - t0) * k);
  for (int q = threadIdx.x; q < nslot; q += kCombineThreads) {
    const size_t f = static_cast<size_t>(t0) * k + q;
    const int r = inv[f];
    const bool ok = r >= 0 && r < nrows;  // else only after a failed or skipped route
    s_row[q] = ok ? r : -1;
    s_w[q] = ok ? w[f] : 0.f;
  }
  if (threadIdx.x == 0) {
    s_ok = 1;
    if (link.p2p) {
      // the returned rows are complete once every expert rank raised its flag to this epoch
      const uint64_t tw = global_timer_ns();
      s_ok = wait_flags_sys(link.wait_flags, link.nranks, link.ctrl[0] + 1) ? 1 : 0;
      if (blockIdx.x == 0 && status != nullptr) {
        if (!s_ok) record_status(status, kDevTimeout);
        DevTimers* tm = timers_of(status);
        add_wait_time(&tm->combine_wait_ns, &tm->combine_waits, tw);
      }
    }
  }
  __syncthreads();
  const TO* rows = reinterpret_cast<const TO*>(rows_v);
  TO* out = reinterpret_cast<TO*>(out_v);
  const int nv = H / 8;  // 16-byte columns of a row
  for (int t = t0; t < t1; ++t) {
    const int qb = (t - t0) * k;
    for (int c0 = 0; c0 < nv; c0 += kCombineVec * kCombineThreads) {
      uint4 v[kCombineVec][kMaxTopK];
#pragma unroll
      for (int u = 0; u < kCombineVec; ++u) {
        const int c = c0 + u * kCombineThreads + static_cast<int>(threadIdx.x);
#pragma unroll
        for (int j = 0; j < kMaxTopK; ++j) {
          // L2 loads: over peer memory the rows were written by other GPUs while this grid ran
          if (j < k && c < nv && qb + j < nslot && s_row[qb + j] >= 0)
            v[u][j] = __ldcg(reinterpret_cast<const uint4*>(rows + s_row[qb + j] * H) + c);
        }
      }
#pragma unroll
      for (int u = 0; u < kCombineVec; ++u) {
        const int c = c0 + u * kCombineThreads + static_cast<int>(threadIdx.x);
        if (c >= nv) continue;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxTopK; ++j) {
          if (j < k && qb + j < nslot && s_row[qb + j] >= 0) {
            const TO* e = reinterpret_cast<const TO*>(&v[u][j]);
            const float wj = s_w[qb + j];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += wj * to_f32<TO>(e[i]);
          }
        }
        union {
          TO h[8];
          uint4 u4;
        } pack;
#pragma unroll
        for (int i = 0; i < 8; ++i) pack.h[i] = from_f32<TO>(acc[i]);
        reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H)[c] = pack.u4;
      }
    }
  }
  if (link.p2p) {
    // every CTA has read its rows: this call is finished on this rank, advance the epoch
    if (last_cta_of_grid_gpu(link.ctrl + 3, &s_last) && threadIdx.x == 0) {
      link.ctrl[0] = link.ctrl[0] + 1;
      stage_busy(clk, 4);
    }
  }
}

constexpr int kAlignThreads = 1024;

__global__ void __launch_bounds__(kAlignThreads) align_kernel(const int32_t* ids, int numel, int E, int block,
                                                                int32_t* sorted_ids, int32_t* expert_ids,
                                                                int32_t* num_post_pad, int max_blocks) {
  extern __shared__ int32_t sm[];
  int32_t* s_cnt = sm;          // [E]
  int32_t* s_off = sm + E;      // [E+1]
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += kAlignThreads) s_cnt[e] = 0;
  __syncthreads();
  for (int f = tid; f < numel; f += kAlignThreads) {
    const int e = ids[f];
    if (e >= 0 && e < E) atomicAdd(&s_cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = acc;
      acc += (s_cnt[e] + block - 1) / block * block;
    }
    s_off[E] = acc;
  }
  const int max_padded = numel + E * (block - 1);
  for (int i = tid; i < max_padded; i += kAlignThreads) sorted_ids[i] = numel;
  for (int b = tid; b < max_blocks; b += kAlignThreads) expert_ids[b] = -1;
  __syncthreads();
  for (int e = tid; e < E; e += kAlignThreads) {
    for (int b = s_off[e] / block; b < s_off[e + 1] / block; ++b) expert_ids[b] = e;
    s_cnt[e] = s_off[e];  // running write position
  }
  if (tid == 0) num_post_pad[0] = s_off[E];
  __syncthreads();
  if (tid < 32) {
    const int lane = tid;
    for (int base = 0; base < numel; base += 32) {
      const int f = base + lane;
      int e = (f < numel) ? ids[f] : -1;
      const bool act = e >= 0 && e < E;
      const int key = act ? e : E + lane;
      const unsigned peers = __match_any_sync(0xffffffffu, key);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      const int bpos = act ? s_cnt[e] : 0;
      if (act) sorted_ids[bpos + rank] = f;
      __syncwarp();
      if (act && lane == __ffs(peers) - 1) s_cnt[e] = bpos + __popc(peers);
      __syncwarp();
    }
  }
}

}  // namespace

cudaError_t launch_combine(const CombineArgs& a, bool bf16, cudaStream_t stream, bool pdl) {
  const void* fn = bf16 ? reinterpret_cast<const void*>(&combine_kernel<__nv_bfloat16>)
                        : reinterpret_cast<const void*>(&combine_kernel<__half>);
  cudaLaunchConfig_t cfg = {};
  const int h4 = a.H / 4;
  cfg.gridDim = dim3((h4 + kCombineThreads - 1) / kCombineThreads, a.T);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<CombineArgs*>(&a)};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

cudaError_t launch_combine_rows(const void* rows, long long nrows, const int32_t* inv, const float* w, void* out,
                                int T, int k, int H, bool bf16, cudaStream_t stream, bool pdl, const EpLink* link,
                                int* status, StageClock* clk) {
  EpLink lk{};
  if (link != nullptr) lk = *link;
  const void* fn = bf16 ? reinterpret_cast<const void*>(&combine_rows_kernel<__nv_bfloat16>)
                        : reinterpret_cast<const void*>(&combine_rows_kernel<__half>);
  cudaLaunchConfig_t cfg = {};
  // at most one CTA per SM while a CTA's slots fit its table; T = 0: flags only
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int grid = T < sms ? T : sms;
  const int per_max = kCombineSlots / (k > 0 ? k : 1);  // tokens whose slots fit one CTA's table
  const int need = (T + per_max - 1) / per_max;
  if (grid < need) grid = need;
  if (grid < 1) grid = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<void**>(&rows), const_cast<int32_t**>(&inv), const_cast<float**>(&w), &out, &T,
                    &k, &H, &nrows, &lk, &status, &clk};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

cudaError_t launch_align(const int32_t* ids, int numel, int E, int block, int32_t* sorted_ids, int32_t* expert_ids,
                         int32_t* num_post_pad, int max_blocks, cudaStream_t stream) {
  const size_t smem = sizeof(int32_t) * (2 * static_cast<size_t>(E) + 1);
  align_kernel<<<1, kAlignThreads, smem, stream>>>(ids, numel, E, block, sorted_ids, expert_ids, num_post_pad,
                                                  max_blocks);
  return cudaGetLastError();
}

}  // namespace smb
