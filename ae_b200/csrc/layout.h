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
constexpr int kMaxSplits = 16;
constexpr int kMaxRanks = 8;       // ranks of the expert-parallel exchange     // down split-K factor S (the fix-up sums S partials in registers)
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
// last CTA done; on the expert side of the exchange the FFN kernel, on the source side
// the final combine, add the time their flag waits took.  Nanoseconds of %globaltimer.
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

// Stage clock of a chain of kernels (one layer call), after the timers in the same control
// block (a workspace's, or an exchange arena's for the peer-memory expert-parallel layer):
// block 0 of each kernel, once past its wait on the previous kernel, charges the time
// since the previous kernel's stamp to that kernel's stage and stamps itself.  Kernels of
// a chain run one after another, so plain loads and stores suffice.  Stages: 0 routing
// (or the expert-parallel dispatch), 1 unused (reserved), 2 FFN (on the expert side of the
// exchange with the receive routing), 3 combine, 4 source-side final combine.  The last stage of a
// call is charged when the next call starts.
constexpr int kStages = 5;
constexpr size_t kStageOffset = kTimerOffset + sizeof(DevTimers);
struct StageClock {
  unsigned long long last;        // %globaltimer of the last stamp (0: none yet)
  unsigned int last_stage;        // the stage that stamped it
  unsigned int pad;
  unsigned long long ns[kStages];  // summed time from a stage's stamp to the next stamp
  unsigned int n[kStages];
  unsigned long long busy[kStages];  // summed time from a stage's stamp to its kernel's last CTA done
};
static_assert(kStageOffset + sizeof(StageClock) <= 256, "stage clock inside the control block");

// Token tiles: an expert with more than 256 tokens in a call is cut into tiles of 256,
// each its own unit of the FFN kernel; ntc bounds the tiles of any expert (counter stride).
inline int token_tile_cap(size_t Tk) { return Tk > 256 ? static_cast<int>((Tk + 255) / 256) : 1; }

// Device scratch for one layer call.  Every buffer is owned by the caller (one
// contiguous allocation); the library only carves it.
struct WsLayout {
  size_t status;      // int32 [64]    [0] device status word, [1] CTA ticket of the gated router,
                      //               [2] FFN exit ticket, [3] / [4] ticket and generation of the
                      //               multi-CTA router,
                      //               timers from byte kTimerOffset; always at offset 0 so a buffer
                      //               reused for other shapes keeps it
  size_t expert_off;  // int32 [E+1]   exclusive prefix of tokens per expert
  size_t done;        // int32 [ndone] [0] FFN work counter, [1] CTAs done gathering xp, then
                      //               [E*S*ntc] finished gate/up tiles per (expert, down split,
                      //               token tile), then [E*m2*ntc] finished down units per
                      //               (expert, row tile, token tile)
  size_t xp;          // elem  [rows, H] token rows in expert-major order (gathered by the FFN kernel)
  size_t perm;        // int32 [Tk]    perm[p] = flat slot f = t*k + j at position p
  size_t inv;         // int32 [Tk]    inv[f] = p
  size_t w;           // fp32  [Tk]    routing weight of flat slot f
  size_t ids;         // int32 [Tk]    expert of flat slot f
  size_t logits;      // fp32  [T, E]  router logits of the gated launch (rounded to the storage dtype)
  size_t a2;          // elem  [rows, I] silu(x W1^T) * (x W3^T) in expert-major order
  size_t part;        // fp32  [S, Tk, H] split-K partials of the down projection
  size_t total;
  int rows;           // padded row count of xp / a2
  int splits;         // S
  int ntc;            // token-tile bound per expert
  int ndone;          // int32 counters in `done`
};

inline WsLayout make_ws_layout(int T, int E, int k, int H, int I, int elem_bytes, int splits) {
  WsLayout L{};
  const size_t Tk = static_cast<size_t>(T) * static_cast<size_t>(k);
  L.rows = static_cast<int>(align_up(Tk, 64) + 64);
  L.splits = splits;
  L.ntc = token_tile_cap(Tk);
  const size_t m2 = (static_cast<size_t>(H) + 255) / 256;
  L.ndone = static_cast<int>(2 + static_cast<size_t>(E) * (splits + m2) * L.ntc);
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
  L.part = o;       o = align_up(o + sizeof(float) * static_cast<size_t>(splits) * Tk * H, kAlign);
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

// Split-K factor of the down projection, chosen by simulating the FFN kernel's dynamic
// unit queue on `num_sms` SMs.  More splits make smaller down units (256 rows x I/S), so
// the run ends with less idle time, but add fp32 partials (S x rows x H x 4 B) that the
// epilogue writes and the combine reads back.  The simulation hands units to the
// earliest free SM in claim order (all gate/up units, then down units expert by expert,
// split by split), each streaming its weights at 44 GB/s per SM, and a down unit starts
// no earlier than the gate/up units that cover its K range (its token rows).  Cost =
// simulated makespan + 2 x the partials' write+read time at 6.5 TB/s (the factor fitted
// to graph-replay sweeps).  `valid_tk` is the number of slots expected to hold a token
// (default Tk): the expert side of an expert-parallel layer reserves G x C slots of
// which about C are used.  Touched experts are estimated as min(E, valid_tk).  Measured
// optima it reproduces: Mixtral-8x7B T=256 -> 2, Mixtral-8x22B T=512 -> 3, one
// Mixtral-8x7B expert of an 8-rank layer (512 slots, ~64 used) -> 9.
inline int choose_splits(int E, int H, int I, int Tk, int num_sms, int valid_tk = -1) {
  const double rate = 44e9, hbm = 6.5e12, part_factor = 2.0;
  const int kb2 = I / 64;
  const int vt = valid_tk >= 0 && valid_tk < Tk ? valid_tk : Tk;
  const int et = E < vt ? E : (vt > 0 ? vt : 1);
  const int sms = num_sms > 0 ? num_sms : 1;
  const int m1 = (I + 127) / 128;
  const int m2 = (H + 255) / 256;
  const int smax = kb2 < kMaxSplits ? kb2 : kMaxSplits;
  typedef std::priority_queue<double, std::vector<double>, std::greater<double>> Heap;
  // phase 1 is the same for every S: simulate it once
  Heap base;
  for (int i = 0; i < sms; ++i) base.push(0.0);
  std::vector<double> done1(static_cast<size_t>(et) * m1);
  const double d1 = 256.0 * H * 2 / rate;
  for (size_t u = 0; u < done1.size(); ++u) {
    const double t = base.top();
    base.pop();
    done1[u] = t + d1;
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
    const double cost = make + part_factor * 2.0 * s * static_cast<double>(vt) * H * 4 / hbm;
    if (cost < best_t * 0.999) {
      best_t = cost;
      best = s;
    }
  }
  return best;
}

}  // namespace smb
