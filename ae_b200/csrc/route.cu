// Router + permutation, one launch.
//
// Reference semantics:
//  * routing = sglang select_experts as called at specmoe/layers/FusedMoE.py:174-185
//    (softmax over E in fp32, top-k, optional renormalisation; weights fp32, ids int32);
//  * permutation = the moe_align_block_size contract of
//    specmoe/layers/fused_moe_kernel.py:19-55 without the block padding: flat slots
//    f = t*k + j bucketed by expert, ascending f inside an expert.
//
// One CTA routes every token (a group of lanes per token, logits in registers,
// shuffle argmax with ties to the lower expert) and computes the expert-major positions
// (per-warp histograms, a scan, then match_any ranks inside 32-slot chunks).  The FFN
// kernel reads token rows through the permutation, so nothing is copied here, except
// for the expert-parallel dispatch: then every CTA recomputes the (cheap) routing and
// copies its share of the token rows into the destination chunks of the exchange (a
// local send buffer for NCCL, or the destinations' receive buffers over peer memory,
// followed by a flag per destination).  Calls of 2048+ slots without a gate or an exchange
// use route_multi_kernel instead: many CTAs route their own tokens and meet once on a table
// of per-CTA counts, giving the same permutation.
#include <cfloat>
#include <climits>

#include "../../include/ae_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace smb {

namespace {

constexpr int kRouteThreads = 512;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr unsigned kFull = 0xffffffffu;

// Dynamic shared memory of route_body: ids, positions and weights of the Tk slots, the
// per-warp histograms and the expert offsets.
__host__ __device__ inline size_t route_body_smem(int T, int E, int k) {
  const size_t Tk = static_cast<size_t>(T) * k;
  return sizeof(int32_t) * (3 * Tk + static_cast<size_t>(kRouteWarps) * E + E + 1);
}

// L2 loads (ld.global.cg): in the gated launch the logits were written by other CTAs of
// the same grid, so the SM's L1 must not serve them.
template <typename TL>
__device__ __forceinline__ float logit_at(const void* base, size_t idx) {
  return to_f32<TL>(__ldcg(reinterpret_cast<const TL*>(base) + idx));
}

// Top-k of one token's logits by a group of G lanes (G a power of two, G * 8 >= E):
// lane q of the group holds experts q, q+G, q+2G, ... (at most 8).  Reductions are
// xor-shuffles inside the group, so every lane of the group ends with all k (id, w).
// Ties go to the lower expert index.  The probabilities follow select_experts:
// p = exp(x - max) * (1 / sum), then (renormalise) p_j / sum of the k selected p.
template <typename TL, int G>
__device__ __forceinline__ void route_token_group(const void* logits, int t, int E, int k, int renorm, int q,
                                                  int (&ids)[kMaxTopK], float (&ws)[kMaxTopK]) {
  constexpr int kPer = 8;
  float v[kPer];
  const size_t row = static_cast<size_t>(t) * E;
  float m = -INFINITY;
#pragma unroll
  for (int r = 0; r < kPer; ++r) {
    const int e = q + G * r;
    v[r] = (e < E) ? logit_at<TL>(logits, row + e) : -INFINITY;
    m = fmaxf(m, v[r]);
  }
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
  float s = 0.f;
#pragma unroll
  for (int r = 0; r < kPer; ++r) {
    if (q + G * r < E) s += expf(v[r] - m);
  }
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  const float inv_s = 1.0f / s;

  unsigned taken = 0;
  float sel_sum = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    ids[j] = -1;
    ws[j] = 0.f;
    if (j < k) {
      float bv = -INFINITY;
      int be = INT_MAX;
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int e = q + G * r;
        if (e < E && !((taken >> r) & 1u) && (be == INT_MAX || v[r] > bv)) {
          bv = v[r];
          be = e;
        }
      }
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, o);
        const int oe = __shfl_xor_sync(kFull, be, o);
        if (ov > bv || (ov == bv && oe < be)) {
          bv = ov;
          be = oe;
        }
      }
      if (be != INT_MAX && q == (be % G)) taken |= 1u << (be / G);
      const float p = expf(bv - m) * inv_s;
      sel_sum += p;
      ids[j] = be;
      ws[j] = p;
    }
  }
  if (renorm) {
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) ws[j] = ws[j] / sel_sum;
  }
}

// Route tokens [t_begin, t_end) with groups of G lanes over nthreads threads; hands
// (token t, choice j, expert id, weight) to the callback.
template <typename TL, int G, typename Sink>
__device__ __forceinline__ void route_range(const void* logits, int t_begin, int t_end, int E, int k, int renorm,
                                            int tid, int nthreads, Sink sink) {
  const int q = tid & (G - 1);
  const int groups = nthreads / G;
  // every lane of a warp runs the same number of iterations (shuffles stay converged)
  for (int base = t_begin; base < t_end; base += groups) {
    const int t = base + tid / G;
    const int tc = t < t_end ? t : t_end - 1;
    int ids[kMaxTopK];
    float ws[kMaxTopK];
    route_token_group<TL, G>(logits, tc, E, k, renorm, q, ids, ws);
    if (t < t_end) {
#pragma unroll
      for (int j = 0; j < kMaxTopK; ++j) {
        if (j < k && (j % G) == q) sink(t, j, ids[j], ws[j]);
      }
    }
  }
}

template <typename TL, typename Sink>
__device__ __forceinline__ void route_dispatch(const void* logits, int t_begin, int t_end, int E, int k,
                                               int renorm, int tid, int nthreads, Sink sink) {
  if (E <= 8) {
    route_range<TL, 1>(logits, t_begin, t_end, E, k, renorm, tid, nthreads, sink);
  } else if (E <= 16) {
    route_range<TL, 2>(logits, t_begin, t_end, E, k, renorm, tid, nthreads, sink);
  } else if (E <= 32) {
    route_range<TL, 4>(logits, t_begin, t_end, E, k, renorm, tid, nthreads, sink);
  } else if (E <= 64) {
    route_range<TL, 8>(logits, t_begin, t_end, E, k, renorm, tid, nthreads, sink);
  } else if (E <= 128) {
    route_range<TL, 16>(logits, t_begin, t_end, E, k, renorm, tid, nthreads, sink);
  } else {
    route_range<TL, 32>(logits, t_begin, t_end, E, k, renorm, tid, nthreads, sink);
  }
}

// Routing + permutation of every flat slot by one CTA's worth of threads.  `cta` is the
// index of the calling CTA among `ncta` that run the body redundantly (each writes the
// outputs of its own flat range; CTA 0 also the offsets, headers and counters).  `stage`:
// shared memory for the token rows of this CTA's flat range in the expert-parallel dispatch
// (copied in while the CTA routes), or nullptr.
template <typename TL>
__device__ __forceinline__ void route_body(const RouteArgs& a, int vec_per_row, int cta, int32_t* sm,
                                           uint4* stage = nullptr) {
  const int Tk = a.T * a.k;
  const int E = a.E;
  int32_t* s_ids = sm;                                   // [Tk]
  int32_t* s_pos = s_ids + Tk;                           // [Tk]
  float* s_w = reinterpret_cast<float*>(s_pos + Tk);     // [Tk]
  int32_t* s_cnt = reinterpret_cast<int32_t*>(s_w + Tk); // [warps][E]
  int32_t* s_off = s_cnt + kRouteWarps * E;              // [E+1]
  __shared__ int s_bad;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    s_bad = 0;
    if (cta == 0 && a.status != nullptr) a.status[0] = 0;
  }
  const int g0 = min(Tk, cta * a.rows_per_cta);
  const int g1 = min(Tk, g0 + a.rows_per_cta);
  if (stage != nullptr && g1 > g0) {
    // the rows this CTA sends do not depend on the routing: start their copy now
    const int t_first = g0 / a.k, t_last = (g1 - 1) / a.k;
    const int n = (t_last - t_first + 1) * vec_per_row;
    const uint4* xsrc = reinterpret_cast<const uint4*>(a.x) + static_cast<size_t>(t_first) * vec_per_row;
    for (int i = tid; i < n; i += kRouteThreads) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(stage + i)), "l"(xsrc + i)
                   : "memory");
    }
  }
  __syncthreads();

  // 1. routing of every token (or the given routing)
  if (a.logits != nullptr) {
    // softmax / top-k over the routed experts, then the shared slots: every token also
    // takes the n_shared pseudo-experts E_routed.. (pieces of one shared expert along its
    // intermediate dimension) with the shared weight
    const int Er = E - a.n_shared;
    route_dispatch<TL>(a.logits, 0, a.T, Er, a.k_routed, a.renormalize, tid, kRouteThreads,
                       [&](int t, int j, int id, float w) {
                         const int f = t * a.k + j;
                         s_ids[f] = id;
                         s_w[f] = w;
                       });
    for (int i = tid; i < a.T * a.n_shared; i += kRouteThreads) {
      const int t = i / a.n_shared, q = i - (i / a.n_shared) * a.n_shared;
      const int f = t * a.k + a.k_routed + q;
      s_ids[f] = Er + q;
      s_w[f] = a.shared_w != nullptr ? a.shared_w[t] : 1.0f;
    }
  } else {
    // given routing [T, k_routed] (+ the shared slots, as above)
    const int Er = E - a.n_shared;
    for (int f = tid; f < Tk; f += kRouteThreads) {
      const int t = f / a.k, j = f - (f / a.k) * a.k;
      if (j < a.k_routed) {
        int id = a.in_ids[t * a.k_routed + j];
        if (id != -1 && (id < 0 || id >= Er)) {
          s_bad = 1;
          id = 0;
        }
        s_ids[f] = id;  // -1: the slot has no expert (padding of the expert-parallel exchange)
        s_w[f] = a.in_w[t * a.k_routed + j];
      } else {
        s_ids[f] = Er + (j - a.k_routed);
        s_w[f] = a.shared_w != nullptr ? a.shared_w[t] : 1.0f;
      }
    }
  }
  for (int i = tid; i < kRouteWarps * E; i += kRouteThreads) s_cnt[i] = 0;
  __syncthreads();
  if (tid == 0 && s_bad && cta == 0) record_status(a.status, kDevBadExpertId);

  // 2. per-warp histograms over contiguous flat segments
  const int seg = (Tk + kRouteWarps - 1) / kRouteWarps;
  const int f0 = min(Tk, warp * seg);
  const int f1 = min(Tk, f0 + seg);
  for (int f = f0 + lane; f < f1; f += 32) {
    if (s_ids[f] >= 0) atomicAdd(&s_cnt[warp * E + s_ids[f]], 1);
  }
  __syncthreads();

  // 3. scan: per expert over warps, then over experts
  for (int e = tid; e < E; e += kRouteThreads) {
    int run = 0;
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = s_cnt[w * E + e];
      s_cnt[w * E + e] = run;
      run += c;
    }
    s_off[e] = run;  // total for now
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive scan of E totals by one warp, 8 experts per lane at most
    int vals[kMaxExperts / 32];
    int local = 0;
#pragma unroll
    for (int r = 0; r < kMaxExperts / 32; ++r) {
      const int e = lane * (kMaxExperts / 32) + r;
      vals[r] = (e < E) ? s_off[e] : 0;
      local += vals[r];
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += y;
    }
    int run = incl - local;
    __syncwarp();
#pragma unroll
    for (int r = 0; r < kMaxExperts / 32; ++r) {
      const int e = lane * (kMaxExperts / 32) + r;
      if (e < E) s_off[e] = run;
      run += vals[r];
    }
    if (lane == 31) s_off[E] = incl;
  }
  __syncthreads();
  for (int i = tid; i < kRouteWarps * E; i += kRouteThreads) s_cnt[i] += s_off[i % E];
  __syncthreads();

  // 4. positions, in ascending flat order inside each expert
  for (int base = f0; base < f1; base += 32) {
    const int f = base + lane;
    const bool act = f < f1 && s_ids[f] >= 0;
    const int e = act ? s_ids[f] : E + lane;  // distinct keys for idle lanes and empty slots
    if (f < f1 && !act) s_pos[f] = -1;
    const unsigned peers = __match_any_sync(kFull, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const int leader = __ffs(peers) - 1;
    const int bpos = act ? s_cnt[warp * E + e] : 0;
    if (act) s_pos[f] = bpos + rank;
    __syncwarp();
    if (act && lane == leader) s_cnt[warp * E + e] = bpos + __popc(peers);
    __syncwarp();
  }
  __syncthreads();

  // 5. outputs for this CTA's flat range
  if (cta == 0) {
    for (int e = tid; e <= E; e += kRouteThreads) a.expert_off[e] = s_off[e];
    if (a.ep_send != nullptr) {
      // header row of each destination chunk: counts of that destination's experts
      for (int e = tid; e < E; e += kRouteThreads) {
        const int d = e / a.ep_Eloc;
        int32_t* hdr = reinterpret_cast<int32_t*>(a.link.chunk[d]);
        hdr[e - d * a.ep_Eloc] = s_off[e + 1] - s_off[e];
      }
    }
    if (a.done != nullptr) {
      for (int i = tid; i < a.done_count; i += kRouteThreads) a.done[i] = 0;
    }
  }
  for (int f = g0 + tid; f < g1; f += kRouteThreads) {
    const int p = s_pos[f];
    if (p >= 0) a.perm[p] = f;
    // dispatch: the slot's row in the returned rows [G][C] (what the final combine reads)
    // instead of its position
    a.inv[f] = (a.ep_send == nullptr || p < 0)
                   ? p
                   : (s_ids[f] / a.ep_Eloc) * a.ep_C + (p - s_off[(s_ids[f] / a.ep_Eloc) * a.ep_Eloc]);
    a.ws_w[f] = s_w[f];
    a.ws_ids[f] = s_ids[f];
    const int t = f / a.k, j = f - (f / a.k) * a.k;
    if (j < a.k_routed) {  // the caller's routing outputs [T, k_routed] leave out the shared slots
      if (a.out_w != nullptr) a.out_w[t * a.k_routed + j] = s_w[f];
      if (a.out_ids != nullptr) a.out_ids[t * a.k_routed + j] = s_ids[f];
    }
  }
  // expert-parallel dispatch: token rows of this CTA's flat range into the exchange
  // layout, all threads on all rows, four independent 16-byte loads in flight per thread
  if (a.ep_send == nullptr) return;  // the FFN reads token rows through the permutation
  const uint4* xsrc = reinterpret_cast<const uint4*>(a.x);
  const size_t row_bytes_out = static_cast<size_t>(vec_per_row) * 16;
  // destination row of flat slot f at expert-major position p: payload row
  // p - (first position of the destination's experts) of the destination's chunk
  auto dst_row = [&](int f, int p) -> uint4* {
    const int d = s_ids[f] / a.ep_Eloc;
    return reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.link.chunk[d]) +
                                    static_cast<size_t>(1 + p - s_off[d * a.ep_Eloc]) * row_bytes_out);
  };
  const int nvec = (g1 - g0) * vec_per_row;
  if (stage != nullptr) {
    // rows from shared memory (copied in during the routing); the stores go out together
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int t_first = g0 / a.k;
    for (int f = g0; f < g1; ++f) {
      if (s_pos[f] < 0) continue;
      uint4* dst = dst_row(f, s_pos[f]);
      const uint4* src = stage + (f / a.k - t_first) * vec_per_row;
      for (int c = tid; c < vec_per_row; c += kRouteThreads) dst[c] = src[c];
    }
  }
  for (int base = tid; stage == nullptr && base < nvec; base += 4 * kRouteThreads) {
    uint4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = base + j * kRouteThreads;
      if (i < nvec) {
        const int f = g0 + i / vec_per_row;
        if (s_pos[f] >= 0) v[j] = __ldg(xsrc + static_cast<size_t>(f / a.k) * vec_per_row + (i % vec_per_row));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = base + j * kRouteThreads;
      if (i < nvec) {
        const int f = g0 + i / vec_per_row;
        if (s_pos[f] >= 0) dst_row(f, s_pos[f])[i % vec_per_row] = v[j];
      }
    }
  }
  // over peer memory: once every CTA's rows (and CTA 0's headers) have landed, tell each
  // destination that this rank's chunk for the current call is complete
  if (a.link.p2p) {
    __shared__ int s_last;
    if (last_cta_of_grid(a.link.ctrl + 1, &s_last) && tid == 0) {
      const int epoch = a.link.ctrl[0] + 1;
      raise_flags_sys(a.link.flag, a.link.nranks, epoch);
      stage_busy(a.clk, a.stage);
    }
  }
}

template <typename TL>
__global__ void __launch_bounds__(kRouteThreads) route_kernel(const RouteArgs a, int vec_per_row) {
  extern __shared__ int32_t sm[];
  pdl_wait_prior_grids();
  if (blockIdx.x == 0 && threadIdx.x == 0) stage_mark(a.clk, a.stage);
  pdl_launch_dependents();
  uint4* stage = nullptr;
  if (a.ep_send != nullptr && dispatch_stage_bytes(a.rows_per_cta, a.k, vec_per_row * 16) > 0) {
    const size_t off = (route_body_smem(a.T, a.E, a.k) + 15) & ~static_cast<size_t>(15);
    stage = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm) + off);
  }
  route_body<TL>(a, vec_per_row, static_cast<int>(blockIdx.x), sm, stage);
  if (gridDim.x == 1) {
    __syncthreads();
    if (threadIdx.x == 0) stage_busy(a.clk, a.stage);
  }
}

// ---------------------------------------------------------------------------- gate

// The 16 / sizeof(TX) elements of a 16-byte vector as fp32.
template <typename TX>
__device__ __forceinline__ void unpack16(const uint4& va, float (&f)[16 / sizeof(TX)]) {
  const TX* v = reinterpret_cast<const TX*>(&va);
#pragma unroll
  for (int i = 0; i < static_cast<int>(16 / sizeof(TX)); ++i) f[i] = to_f32<TX>(v[i]);
}

constexpr int kGateTok = 2;   // tokens per CTA pass
constexpr int kGateExp = 8;   // experts per pass

// Router gate: logits[t, e] = sum_h x[t, h] * W[e, h] (ReplicatedLinear(H, E, bias=False),
// specmoe/models/mixtral.py:85-92,111), fp32 accumulation, rounded once to the storage
// dtype like the reference's half-precision linear output.  A CTA takes a contiguous
// range of tokens, 2 tokens x 8 experts per pass; its 512 threads split H into 16-byte
// vectors (each converted to fp32 once), each warp reduces its 16 values with a
// 16-shuffle transpose-reduction, and 16 threads add the 16 warp sums in warp order, so
// the result does not depend on timing.  With g.route set, every CTA then
// takes a ticket and the last one to finish routes all tokens (route_body), reading the
// logits the others wrote; it leaves the ticket at 0 for the next call.
template <typename TX>
__global__ void __launch_bounds__(kRouteThreads) gate_route_kernel(const RouteArgs a, const GateArgs g,
                                                                   int vec_per_row) {
  extern __shared__ int32_t sm[];
  __shared__ float s_red[kRouteWarps][kGateTok * kGateExp];
  __shared__ int s_last;
  pdl_wait_prior_grids();
  if (blockIdx.x == 0 && threadIdx.x == 0 && g.route) stage_mark(a.clk, a.stage);
  pdl_launch_dependents();
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int vpr = g.H * static_cast<int>(sizeof(TX)) / 16;
  const uint4* xv = reinterpret_cast<const uint4*>(g.x);
  const uint4* wv = reinterpret_cast<const uint4*>(g.weight);
  // this CTA's tokens: a contiguous range, at most kGateTok per pass
  const int per_cta = (g.T + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int t_begin = min(g.T, static_cast<int>(blockIdx.x) * per_cta);
  const int t_end = min(g.T, t_begin + per_cta);
  constexpr int kEl = 16 / static_cast<int>(sizeof(TX));
  for (int t0 = t_begin; t0 < t_end; t0 += kGateTok) {
    const int nt = min(kGateTok, t_end - t0);
    for (int e0 = 0; e0 < g.E; e0 += kGateExp) {
      float v[kGateTok * kGateExp];
#pragma unroll
      for (int i = 0; i < kGateTok * kGateExp; ++i) v[i] = 0.f;
      for (int c = tid; c < vpr; c += kRouteThreads) {
        float xf[kGateTok][kEl];
#pragma unroll
        for (int j = 0; j < kGateTok; ++j) {
          uint4 xr = make_uint4(0u, 0u, 0u, 0u);
          if (j < nt) xr = __ldg(xv + static_cast<size_t>(t0 + j) * vpr + c);
          unpack16<TX>(xr, xf[j]);
        }
#pragma unroll
        for (int e = 0; e < kGateExp; ++e) {
          if (e0 + e < g.E) {
            float wf[kEl];
            unpack16<TX>(__ldg(wv + static_cast<size_t>(e0 + e) * vpr + c), wf);
#pragma unroll
            for (int j = 0; j < kGateTok; ++j) {
              float acc = v[j * kGateExp + e];
#pragma unroll
              for (int i = 0; i < kEl; ++i) acc = fmaf(xf[j][i], wf[i], acc);
              v[j * kGateExp + e] = acc;
            }
          }
        }
      }
      // transpose-reduction of the NV = 16 values over the warp: after the step of width
      // o, a lane holds o partial sums, of the half of the indices selected by its bit o;
      // then lanes that differ only in bit 4 add their sums, and lane l holds value l % 16
      constexpr int kNV = kGateTok * kGateExp;
      static_assert(kNV == 16, "reduction below is written for 16 values");
#pragma unroll
      for (int o = kNV / 2; o >= 1; o >>= 1) {
        const bool hi = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < o; ++i) {
          const float send = hi ? v[i] : v[i + o];
          const float keep = hi ? v[i + o] : v[i];
          v[i] = keep + __shfl_xor_sync(kFull, send, o);
        }
      }
      v[0] += __shfl_xor_sync(kFull, v[0], 16);
      if (lane < kNV) s_red[warp][lane] = v[0];
      __syncthreads();
      if (tid < kGateTok * kGateExp) {
        const int j = tid / kGateExp, e = tid % kGateExp;
        float s = 0.f;
        for (int w = 0; w < kRouteWarps; ++w) s += s_red[w][tid];
        if (j < nt && e0 + e < g.E) {
          const TX r = from_f32<TX>(s);
          const size_t o = static_cast<size_t>(t0 + j) * g.E + e0 + e;
          if (g.logits != nullptr) g.logits[o] = to_f32<TX>(r);
          if (g.logits_out != nullptr) reinterpret_cast<TX*>(g.logits_out)[o] = r;
        }
      }
      __syncthreads();
    }
  }
  if (!g.route) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(g.ticket, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) *g.ticket = 0;
  route_body<float>(a, vec_per_row, 0, sm);
}

// Routing only (select_experts): one warp per token.
template <typename TL>
__global__ void __launch_bounds__(256) topk_kernel(const void* logits, int T, int E, int k, int renorm,
                                                   float* out_w, int32_t* out_ids) {
  pdl_wait_prior_grids();
  pdl_launch_dependents();
  // this CTA's tokens: a contiguous range sized for 256 lanes in groups of 32 (covers E <= 256)
  const int per_cta = blockDim.x / 32;
  const int t0 = blockIdx.x * per_cta;
  const int t1 = min(T, t0 + per_cta);
  if (t0 >= T) return;
  route_dispatch<TL>(logits, t0, t1, E, k, renorm, threadIdx.x, blockDim.x, [&](int t, int j, int id, float w) {
    const int f = t * k + j;
    out_w[f] = w;
    out_ids[f] = id;
  });
}


// ---------------------------------------------------------------- multi-CTA router

// Large calls (no gate, no exchange, Tk >= kMultiRouteMinSlots): the router over many
// CTAs instead of one.  CTA c routes the contiguous tokens [c*tpc, (c+1)*tpc) and counts its
// slots per expert into a table in the workspace; the CTA that takes the last ticket turns
// the ncta x E counts into every CTA's first position per expert (expert-major, CTAs in flat
// order) and the expert offsets, zeroes the FFN's counters and bumps a generation word,
// while the others wait (bounded) for that bump.  Every CTA of the grid is resident at once
// (at most one per SM; the FFN launched behind it starts only after all of them have
// started), so the wait ends.  Then each CTA places its slots the way the one-CTA router
// does (per-warp segments, match_any ranks), so the permutation is the same.
template <typename TL>
__global__ void __launch_bounds__(kRouteThreads) route_multi_kernel(const RouteArgs a, int tpc, int* hist,
                                                                     int* ticket, int* gen) {
  extern __shared__ int32_t sm[];
  __shared__ int s_gen0, s_bad, s_last;
  pdl_wait_prior_grids();
  if (blockIdx.x == 0 && threadIdx.x == 0) stage_mark(a.clk, a.stage);
  pdl_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = a.E, k = a.k;
  const int cta = static_cast<int>(blockIdx.x);
  const int t0 = min(a.T, cta * tpc), t1 = min(a.T, t0 + tpc);
  const int fb = t0 * k, n = (t1 - t0) * k;  // this CTA's flat slots [fb, fb + n)
  const int nmax = tpc * k;
  int32_t* s_ids = sm;                                    // [nmax]
  int32_t* s_pos = s_ids + nmax;                          // [nmax]
  float* s_w = reinterpret_cast<float*>(s_pos + nmax);    // [nmax]
  int32_t* s_cnt = reinterpret_cast<int32_t*>(s_w + nmax);  // [warps][E]
  int32_t* s_base = s_cnt + kRouteWarps * E;              // [E]
  if (tid == 0) {
    s_gen0 = *reinterpret_cast<volatile int*>(gen);
    s_bad = 0;
    // this call's status (the other CTAs record only after the table below, which comes
    // after every CTA, this one included, has taken its ticket)
    if (cta == 0 && a.status != nullptr) a.status[0] = 0;
  }
  __syncthreads();

  // 1. routing of this CTA's tokens (or the given routing), then the shared slots
  const int Er = E - a.n_shared;
  if (a.logits != nullptr) {
    route_dispatch<TL>(a.logits, t0, t1, Er, a.k_routed, a.renormalize, tid, kRouteThreads,
                       [&](int t, int j, int id, float w) {
                         const int q = (t - t0) * k + j;
                         s_ids[q] = id;
                         s_w[q] = w;
                       });
    for (int i = tid; i < (t1 - t0) * a.n_shared; i += kRouteThreads) {
      const int tt = i / a.n_shared, qq = i - (i / a.n_shared) * a.n_shared;
      const int q = tt * k + a.k_routed + qq;
      s_ids[q] = Er + qq;
      s_w[q] = a.shared_w != nullptr ? a.shared_w[t0 + tt] : 1.0f;
    }
  } else {
    for (int q = tid; q < n; q += kRouteThreads) {
      const int f = fb + q;
      const int t = f / k, j = f - (f / k) * k;
      if (j < a.k_routed) {
        int id = a.in_ids[t * a.k_routed + j];
        if (id != -1 && (id < 0 || id >= Er)) {
          s_bad = 1;
          id = 0;
        }
        s_ids[q] = id;
        s_w[q] = a.in_w[t * a.k_routed + j];
      } else {
        s_ids[q] = Er + (j - a.k_routed);
        s_w[q] = a.shared_w != nullptr ? a.shared_w[t] : 1.0f;
      }
    }
  }
  for (int i = tid; i < kRouteWarps * E; i += kRouteThreads) s_cnt[i] = 0;
  __syncthreads();

  // 2. per-warp histograms over contiguous segments of this CTA's slots; per expert the
  // warps' offsets inside the CTA, and the CTA's count into the table
  const int seg = (n + kRouteWarps - 1) / kRouteWarps;
  const int q0 = min(n, warp * seg), q1 = min(n, q0 + seg);
  for (int q = q0 + lane; q < q1; q += 32) {
    if (s_ids[q] >= 0) atomicAdd(&s_cnt[warp * E + s_ids[q]], 1);
  }
  __syncthreads();
  for (int e = tid; e < E; e += kRouteThreads) {
    int run = 0;
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = s_cnt[w * E + e];
      s_cnt[w * E + e] = run;
      run += c;
    }
    hist[cta * E + e] = run;
  }
  __syncthreads();

  // 3. the last CTA to take a ticket builds the table of first positions
  if (tid == 0) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(ticket) : "memory");
    s_last = old == static_cast<int>(gridDim.x) - 1 ? 1 : 0;
  }
  __syncthreads();
  if (s_last) {
    const int G = static_cast<int>(gridDim.x);
    for (int e = tid; e < E; e += kRouteThreads) {
      int tot = 0;
      for (int c = 0; c < G; ++c) tot += __ldcg(hist + c * E + e);
      s_base[e] = tot;
    }
    __syncthreads();
    if (tid == 0) {
      int pos = 0;
      for (int e = 0; e < E; ++e) {
        const int c = s_base[e];
        s_base[e] = pos;
        a.expert_off[e] = pos;
        pos += c;
      }
      a.expert_off[E] = pos;
    }
    __syncthreads();
    for (int e = tid; e < E; e += kRouteThreads) {
      int run = s_base[e];
      for (int c = 0; c < G; ++c) {
        const int v = __ldcg(hist + c * E + e);
        hist[c * E + e] = run;
        run += v;
      }
    }
    if (a.done != nullptr) {
      for (int i = tid; i < a.done_count; i += kRouteThreads) a.done[i] = 0;
    }
    __syncthreads();
    if (tid == 0) {
      *ticket = 0;
      __threadfence();
      atomicExch(gen, s_gen0 + 1);  // after the fence: publishes the table
    }
  } else if (tid == 0) {
    const uint64_t t_start = global_timer_ns();
    while (*reinterpret_cast<volatile int*>(gen) == s_gen0) {
      if (global_timer_ns() - t_start > kWaitBudgetNs) {
        record_status(a.status, kDevTimeout);
        break;
      }
      __nanosleep(64);
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  __syncthreads();
  for (int e = tid; e < E; e += kRouteThreads) s_base[e] = __ldcg(hist + cta * E + e);
  __syncthreads();
  if (tid == 0 && s_bad) record_status(a.status, kDevBadExpertId);

  // 4. positions: the CTA's first position of the expert + the warp's offset + the rank
  for (int i = tid; i < kRouteWarps * E; i += kRouteThreads) s_cnt[i] += s_base[i % E];
  __syncthreads();
  for (int base = q0; base < q1; base += 32) {
    const int q = base + lane;
    const bool act = q < q1 && s_ids[q] >= 0;
    const int e = act ? s_ids[q] : E + lane;
    if (q < q1 && !act) s_pos[q] = -1;
    const unsigned peers = __match_any_sync(kFull, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const int leader = __ffs(peers) - 1;
    const int bpos = act ? s_cnt[warp * E + e] : 0;
    if (act) s_pos[q] = bpos + rank;
    __syncwarp();
    if (act && lane == leader) s_cnt[warp * E + e] = bpos + __popc(peers);
    __syncwarp();
  }
  __syncthreads();

  // 5. outputs of this CTA's slots
  for (int q = tid; q < n; q += kRouteThreads) {
    const int f = fb + q;
    const int p = s_pos[q];
    if (p >= 0) a.perm[p] = f;
    a.inv[f] = p;
    a.ws_w[f] = s_w[q];
    a.ws_ids[f] = s_ids[q];
    const int t = f / k, j = f - (f / k) * k;
    if (j < a.k_routed) {
      if (a.out_w != nullptr) a.out_w[t * a.k_routed + j] = s_w[q];
      if (a.out_ids != nullptr) a.out_ids[t * a.k_routed + j] = s_ids[q];
    }
  }
}

}  // namespace

cudaError_t launch_topk(const void* logits, int logits_dtype, int T, int E, int k, int renorm, float* out_w,
                        int32_t* out_ids, cudaStream_t stream) {
  const int grid = (T + 7) / 8;
  switch (logits_dtype) {
    case SMB_DTYPE_F16: topk_kernel<__half><<<grid, 256, 0, stream>>>(logits, T, E, k, renorm, out_w, out_ids); break;
    case SMB_DTYPE_BF16:
      topk_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(logits, T, E, k, renorm, out_w, out_ids);
      break;
    default: topk_kernel<float><<<grid, 256, 0, stream>>>(logits, T, E, k, renorm, out_w, out_ids); break;
  }
  return cudaGetLastError();
}

size_t route_smem_bytes(int T, int E, int k) { return route_body_smem(T, E, k); }

cudaError_t launch_route(const RouteArgs& a, int elem_bytes, int grid, cudaStream_t stream, bool pdl) {
  static std::atomic<int> seen[3][64];
  const void* fn = nullptr;
  int which = 0;
  switch (a.logits == nullptr ? SMB_DTYPE_F32 : a.logits_dtype) {
    case SMB_DTYPE_F16: fn = reinterpret_cast<const void*>(&route_kernel<__half>); which = 0; break;
    case SMB_DTYPE_BF16: fn = reinterpret_cast<const void*>(&route_kernel<__nv_bfloat16>); which = 1; break;
    default: fn = reinterpret_cast<const void*>(&route_kernel<float>); which = 2; break;
  }
  int vec_per_row = static_cast<int>(static_cast<size_t>(a.H) * elem_bytes / 16);
  size_t smem = route_smem_bytes(a.T, a.E, a.k);
  if (a.ep_send != nullptr) {
    const int st = dispatch_stage_bytes(a.rows_per_cta, a.k, vec_per_row * 16);
    if (st > 0) smem = ((smem + 15) & ~static_cast<size_t>(15)) + st;
  }
  cudaError_t err = smem > 40 * 1024 ? ensure_dyn_smem(fn, static_cast<int>(smem), seen[which], 64) : cudaSuccess;
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRouteThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<RouteArgs*>(&a), &vec_per_row};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

cudaError_t launch_gate_route(const RouteArgs& a, const GateArgs& g, int dtype, int grid, cudaStream_t stream,
                              bool pdl) {
  static std::atomic<int> seen[2][64];
  const bool bf16 = dtype == SMB_DTYPE_BF16;
  const void* fn = bf16 ? reinterpret_cast<const void*>(&gate_route_kernel<__nv_bfloat16>)
                        : reinterpret_cast<const void*>(&gate_route_kernel<__half>);
  const size_t smem = g.route ? route_smem_bytes(a.T, a.E, a.k) : 0;
  cudaError_t err = smem > 40 * 1024 ? ensure_dyn_smem(fn, static_cast<int>(smem), seen[bf16 ? 1 : 0], 64)
                                     : cudaSuccess;
  if (err != cudaSuccess) return err;
  int vec_per_row = static_cast<int>(static_cast<size_t>(a.H) * 2 / 16);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRouteThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<RouteArgs*>(&a), const_cast<GateArgs*>(&g), &vec_per_row};
  return cudaLaunchKernelExC(&cfg, fn, params);
}


size_t route_multi_smem_bytes(int tpc, int E, int k) {
  const size_t nmax = static_cast<size_t>(tpc) * k;
  return sizeof(int32_t) * (3 * nmax + static_cast<size_t>(kRouteWarps) * E + E);
}

cudaError_t launch_route_multi(const RouteArgs& a, int tpc, int grid, int* hist, int* ticket, int* gen,
                               cudaStream_t stream, bool pdl) {
  static std::atomic<int> seen[3][64];
  const void* fn = nullptr;
  int which = 0;
  switch (a.logits == nullptr ? SMB_DTYPE_F32 : a.logits_dtype) {
    case SMB_DTYPE_F16: fn = reinterpret_cast<const void*>(&route_multi_kernel<__half>); which = 0; break;
    case SMB_DTYPE_BF16: fn = reinterpret_cast<const void*>(&route_multi_kernel<__nv_bfloat16>); which = 1; break;
    default: fn = reinterpret_cast<const void*>(&route_multi_kernel<float>); which = 2; break;
  }
  const size_t smem = route_multi_smem_bytes(tpc, a.E, a.k);
  cudaError_t err = smem > 40 * 1024 ? ensure_dyn_smem(fn, static_cast<int>(smem), seen[which], 64) : cudaSuccess;
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRouteThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<RouteArgs*>(&a), &tpc, &hist, &ticket, &gen};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

}  // namespace smb
