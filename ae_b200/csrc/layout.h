// Workspace layout and launch-shape choices shared by the host launchers.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <queue>
#include <vector>

namespace smb {

constexpr int kMaxExperts = 256;   // router keeps up to 8 logits per lane
constexpr int kMaxTopK = 8;
constexpr int kMaxFlat = 16384;    // T*k limit of the single-pass permutation
constexpr size_t kAlign = 256;
constexpr size_t kWsHeaderBytes = 256;  // status block at offset 0, zeroed by smb_moe_workspace_init

// Status codes written to the device status word (first error wins).
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeout = 1,      // an mbarrier wait ran past its budget
  kDevBadPage = 2,      // page_of_expert[e] outside [0, P)
  kDevBadExpertId = 3,  // a given expert id outside [0, E)
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Device-side timers kept in a workspace's control block at byte kTimerOffset (zeroed by
// smb_moe_workspace_init, read and optionally cleared by smb_moe_read_timers).  The FFN
// kernel adds, per launch, the time from the first CTA past its dependency wait to the
// last CTA done; the expert-parallel receive router and final combine add the time
// their flag waits took.  Nanoseconds of %globaltimer.
constexpr size_t kTimerOffset = 64;
struct DevTimers {
  unsigned long long ffn_neg_t0;       // ~0 - earliest CTA start of the running FFN launch (0 = none)
  unsigned int ffn_exit;               // CTAs of the running FFN launch that have finished
  unsigned int ffn_launches;           // FFN launches timed
  unsigned long long ffn_ns;           // their summed duration
  unsigned long long recv_wait_ns;     // expert side: time spent waiting for the sources' flags
  unsigned int recv_waits;
  unsigned int combine_waits;
  unsigned long long combine_wait_ns;  // source side: time the final combine waited for the returns
};
static_assert(sizeof(DevTimers) == 48, "timer block layout");
static_assert(kTimerOffset + sizeof(DevTimers) <= 256, "timer block inside the control block");

// How the FFN kernel cuts a layer call into units of work (host-chosen, a pure function
// of the sizes and the SM count, so that workspace sizing and launches agree):
//   splits  S: split-K factor of the down projection;
//   ks1:       split-K factor of the gate/up projection, > 1 only when there are fewer
//              gate/up units than SMs (one expert on a rank of an expert-parallel layer);
//              slices before the last store fp32 partials that the last slice adds
//   ntc:       bound on token tiles per expert (an expert with more than 256 tokens is
//              cut into tiles of 256, each its own unit)
struct FfnPlan {
  int splits = 1;
  int ks1 = 1;
};

inline int token_tile_cap(size_t Tk) { return Tk > 256 ? static_cast<int>((Tk + 255) / 256) : 1; }

// Device scratch for one layer call.  Every buffer is owned by the caller (one
// contiguous allocation); the library only carves it.
struct WsLayout {
  size_t status;      // int32 [64]    [0] device status word, [1] CTA ticket of the gated router,
                      //               timers from byte kTimerOffset; always at offset 0 so a buffer
                      //               reused for other shapes keeps it
  size_t expert_off;  // int32 [E+1]   exclusive prefix of tokens per expert
  size_t done;        // int32 [ndone] [0] FFN work counter, [1] CTAs done gathering xp, then
                      //               [E*S*ntc] finished gate/up tiles per (expert, down split,
                      //               token tile), then [E*m1*ntc] gate/up K slices stored per
                      //               (expert, feature tile, token tile) when ks1 > 1
  size_t xp;          // elem  [rows, H] token rows in expert-major order (gathered by the FFN kernel)
  size_t perm;        // int32 [Tk]    perm[p] = flat slot f = t*k + j at position p
  size_t inv;         // int32 [Tk]    inv[f] = p
  size_t w;           // fp32  [Tk]    routing weight of flat slot f
  size_t ids;         // int32 [Tk]    expert of flat slot f
  size_t logits;      // fp32  [T, E]  router logits of the gated launch (rounded to the storage dtype)
  size_t a2;          // elem  [rows, I] silu(x W1^T) * (x W3^T) in expert-major order
  size_t part;        // fp32  [S, Tk, H] split-K partials of the down projection
  size_t gu;          // fp32  [ks1-1, rows, 2I] gate/up partials of the K slices before the last
  size_t total;
  int rows;           // padded row count of xp / a2
  int splits;         // S
  int ks1;            // gate/up K slices
  int ntc;            // token-tile bound per expert
  int ndone;          // int32 counters in `done`
};

inline WsLayout make_ws_layout(int T, int E, int k, int H, int I, int elem_bytes, FfnPlan plan) {
  WsLayout L{};
  const size_t Tk = static_cast<size_t>(T) * static_cast<size_t>(k);
  L.rows = static_cast<int>(align_up(Tk, 64) + 64);
  L.splits = plan.splits;
  L.ks1 = plan.ks1;
  L.ntc = token_tile_cap(Tk);
  const size_t m1 = (static_cast<size_t>(I) + 127) / 128;
  L.ndone = static_cast<int>(2 + static_cast<size_t>(E) * plan.splits * L.ntc +
                             (plan.ks1 > 1 ? static_cast<size_t>(E) * m1 * L.ntc : 0));
  size_t o = 0;
  L.status = o;     o = align_up(o + sizeof(int32_t) * 64, kAlign);
  L.expert_off = o; o = align_up(o + sizeof(int32_t) * (E + 1), kAlign);
  L.done = o;       o = align_up(o + sizeof(int32_t) * static_cast<size_t>(L.ndone), kAlign);
  L.perm = o;       o = align_up(o + sizeof(int32_t) * Tk, kAlign);
  L.inv = o;        o = align_up(o + sizeof(int32_t) * Tk, kAlign);
  L.w = o;          o = align_up(o + sizeof(float) * Tk, kAlign);
  L.ids = o;        o = align_up(o + sizeof(int32_t) * Tk, kAlign);
  L.logits = o;     o = align_up(o + sizeof(float) * static_cast<size_t>(T) * E, kAlign);
  L.xp = o;         o = align_up(o + static_cast<size_t>(elem_bytes) * L.rows * H, kAlign);
  L.a2 = o;         o = align_up(o + static_cast<size_t>(elem_bytes) * L.rows * I, kAlign);
  L.part = o;       o = align_up(o + sizeof(float) * static_cast<size_t>(plan.splits) * Tk * H, kAlign);
  L.gu = o;         o = align_up(o + sizeof(float) * static_cast<size_t>(plan.ks1 - 1) * L.rows * 2 * I, kAlign);
  L.total = o;
  return L;
}

// Exchange arena of the peer-memory expert-parallel transport (one per rank, the same
// layout on every rank; peers write into it through CUDA IPC mappings):
//   ctrl  int32 [64]      [0] epoch = number of finished layer calls, [1..3] CTA tickets of
//                         the dispatch, expert-combine and final-combine kernels
//   flags int32 [2 x 8]   [s] source s finished writing its chunk of this rank's recv for
//                         epoch e (value e); [8 + d] expert rank d finished writing its
//                         chunk of this rank's back
//   recv  [G][C+1][H]     chunk s = header row (counts per local expert) + C payload rows
//                         from source s
//   back  [G][C][H]       chunk d = expert outputs returned by expert rank d
struct EpArena {
  size_t ctrl, flags, recv, back, total;
};
inline EpArena make_ep_arena(int G, int C, int H, int elem_bytes) {
  EpArena A{};
  A.ctrl = 0;
  A.flags = 256;
  A.recv = 1024;
  A.back = A.recv + align_up(static_cast<size_t>(G) * (C + 1) * H * elem_bytes, kAlign);
  A.total = A.back + align_up(static_cast<size_t>(G) * C * H * elem_bytes, kAlign);
  return A;
}
constexpr int kEpReturnFlags = 8;  // offset of the return flags in the flag block

// Unit plan of the FFN kernel, chosen by simulating its dynamic unit queue on `num_sms`
// SMs.  Gate/up K slices: when the touched experts give fewer gate/up units (256 weight
// rows each) than SMs, every unit is cut into ks1 in {2, 4} K slices so that the first
// wave fills the GPU.  Down split-K factor S: more splits make smaller down units (256 rows
// x I/S), so the run ends with less idle time, but add fp32 partials (S x Tk x H x 4 B)
// that the epilogue writes and the combine reads back.  The simulation hands units to the
// earliest free SM in claim order (all gate/up units, then down units expert by expert,
// split by split), each streaming its weights at 44 GB/s per SM, and a down unit starts no
// earlier than the gate/up units that cover its K range (its token rows).  Cost =
// simulated makespan + 2 x the partials' write+read time at 6.5 TB/s (the factor fitted
// to graph-replay sweeps).  Measured optima it reproduces: Mixtral-8x7B T=256 -> S=2,
// Mixtral-8x22B T=512 -> S=3.  Touched experts are estimated as min(E, Tk).
inline FfnPlan choose_plan(int E, int H, int I, int Tk, int num_sms) {
  const double rate = 44e9, hbm = 6.5e12, part_factor = 2.0;
  const int kb2 = I / 64;
  const int et = E < Tk ? E : (Tk > 0 ? Tk : 1);
  const int sms = num_sms > 0 ? num_sms : 1;
  const int m1 = (I + 127) / 128;
  const int m2 = (H + 255) / 256;
  const int smax = kb2 < 16 ? kb2 : 16;
  FfnPlan plan;
  plan.ks1 = 1;
  while (static_cast<long long>(et) * m1 * plan.ks1 < sms && plan.ks1 < 4 && (H / 64) % (plan.ks1 * 2) == 0) {
    plan.ks1 *= 2;
  }
  const int ks1 = plan.ks1;
  typedef std::priority_queue<double, std::vector<double>, std::greater<double>> Heap;
  // phase 1 is the same for every S: simulate it once; a feature tile is ready when its
  // last K slice is
  Heap base;
  for (int i = 0; i < sms; ++i) base.push(0.0);
  std::vector<double> done1(static_cast<size_t>(et) * m1, 0.0);
  const double d1 = 256.0 * H * 2 / rate / ks1;
  for (size_t u = 0; u < done1.size() * ks1; ++u) {
    const double t = base.top();
    base.pop();
    const size_t tile = u / ks1;
    done1[tile] = done1[tile] > t + d1 ? done1[tile] : t + d1;
    base.push(t + d1);
  }
  int best = 1;
  double best_t = 1e30;
  for (int s = 1; s <= smax; ++s) {
    Heap q = base;
    for (int e = 0; e < et; ++e) {
      for (int ks = 0; ks < s; ++ks) {
        const int k0 = ks * kb2 / s, k1 = (ks + 1) * kb2 / s;
        double dep = 0.0;
        for (int mt = k0 / 2; mt < m1 && 2 * mt < k1; ++mt) {
          const double v = done1[static_cast<size_t>(e) * m1 + mt];
          dep = v > dep ? v : dep;
        }
        const double d = 256.0 * (k1 - k0) * 64 * 2 / rate;
        for (int j = 0; j < m2; ++j) {
          const double t = q.top();
          q.pop();
          q.push((t > dep ? t : dep) + d);
        }
      }
    }
    double make = 0.0;
    while (!q.empty()) {
      make = q.top() > make ? q.top() : make;
      q.pop();
    }
    const double cost = make + part_factor * 2.0 * s * static_cast<double>(Tk) * H * 4 / hbm;
    if (cost < best_t * 0.999) {
      best_t = cost;
      best = s;
    }
  }
  plan.splits = best;
  return plan;
}

// Down split-K factor alone (the plan's S).
inline int choose_splits(int E, int H, int I, int Tk, int num_sms) { return choose_plan(E, H, I, Tk, num_sms).splits; }

}  // namespace smb
