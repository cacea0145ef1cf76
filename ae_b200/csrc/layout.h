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

// Device scratch for one layer call.  Every buffer is owned by the caller (one
// contiguous allocation); the library only carves it.
struct WsLayout {
  size_t status;      // int32 [64]    [0] device status word, [1] CTA ticket of the gated router;
                      //               always at offset 0 so a buffer reused for other shapes keeps it
  size_t expert_off;  // int32 [E+1]   exclusive prefix of tokens per expert
  size_t done;        // int32 [E*S+2] finished gate/up units per (expert, down split), then the FFN work
                      //               counter and the count of CTAs done gathering xp
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
};

inline WsLayout make_ws_layout(int T, int E, int k, int H, int I, int elem_bytes, int splits) {
  WsLayout L{};
  const size_t Tk = static_cast<size_t>(T) * static_cast<size_t>(k);
  L.rows = static_cast<int>(align_up(Tk, 64) + 64);
  L.splits = splits;
  size_t o = 0;
  L.status = o;     o = align_up(o + sizeof(int32_t) * 64, kAlign);
  L.expert_off = o; o = align_up(o + sizeof(int32_t) * (E + 1), kAlign);
  L.done = o;       o = align_up(o + sizeof(int32_t) * (static_cast<size_t>(E) * splits + 2), kAlign);
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
// the run ends with less idle time, but add fp32 partials (S x Tk x H x 4 B) that the
// epilogue writes and the combine reads back.  The simulation hands units to the
// earliest free SM in claim order (all gate/up units, then down units expert by expert,
// split by split), each streaming its weights at 44 GB/s per SM, and a down unit starts
// no earlier than the gate/up units that cover its K range (its token rows).  Cost =
// simulated makespan + 2 x the partials' write+read time at 6.5 TB/s (the factor fitted
// to graph-replay sweeps).  Measured optima it reproduces: Mixtral-8x7B T=256 -> 2,
// Mixtral-8x22B T=512 -> 3.  Touched experts are estimated as min(E, Tk).
inline int choose_splits(int E, int H, int I, int Tk, int num_sms) {
  const double rate = 44e9, hbm = 6.5e12, part_factor = 2.0;
  const int kb2 = I / 64;
  const int et = E < Tk ? E : (Tk > 0 ? Tk : 1);
  const int sms = num_sms > 0 ? num_sms : 1;
  const int m1 = (I + 127) / 128;
  const int m2 = (H + 255) / 256;
  const int smax = kb2 < 16 ? kb2 : 16;
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
    const double cost = make + part_factor * 2.0 * s * static_cast<double>(Tk) * H * 4 / hbm;
    if (cost < best_t * 0.999) {
      best_t = cost;
      best = s;
    }
  }
  return best;
}

}  // namespace smb
