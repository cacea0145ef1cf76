// Workspace layout and launch-shape choices shared by the host launchers.
#pragma once

#include <cstddef>
#include <cstdint>

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

// Split-K factor of the down projection.  The FFN kernel hands out units dynamically,
// gate/up units first, so the run ends with a tail of about half a down unit (256 rows x
// I/S) during which SMs fall idle one by one.  More splits shorten that tail but add fp32
// partials that the kernel writes and the combine reads back.  Pick S in
// [1, min(16, I/64)] minimising tail + partial traffic, at a per-SM streaming rate of
// 45 GB/s and an HBM rate of 6.5 TB/s.
inline int choose_splits(int E, int H, int I, int Tk, int num_sms) {
  (void)E;
  (void)num_sms;
  const double per_sm = 45e9, hbm = 6.5e12;
  const int kb2 = I / 64;
  const int smax = kb2 < 16 ? kb2 : 16;
  int best = 1;
  double best_t = 1e30;
  for (int s = 1; s <= smax; ++s) {
    const double unit = 256.0 * ((kb2 + s - 1) / s) * 64 * 2;
    const double t = 0.5 * unit / per_sm + 2.0 * s * static_cast<double>(Tk) * H * 4 / hbm;
    if (t < best_t * 0.999) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

}  // namespace smb
