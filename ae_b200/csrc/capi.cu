// C ABI entry points: argument checks, workspace carving, TMA descriptor encoding and
// the launch sequence route -> gate/up GEMM -> down GEMM -> combine.  Consecutive
// launches use programmatic dependent launch so each kernel's prologue overlaps the
// previous kernel's tail; every kernel waits for its predecessor before it touches
// global memory.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/ae_b200.h"
#include "kernels.h"

using namespace smb;

namespace {

thread_local char g_last_cuda_error[256] = "";

int cuda_fail(cudaError_t err) {
  std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(err),
                cudaGetErrorString(err));
  return SMB_ERR_CUDA;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

typedef CUresult (*StreamWriteValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

// cuStreamWriteValue32: a stream-ordered 32-bit write done by the GPU's front end, so a
// copy stream can raise a flag that a running kernel polls without needing an SM.
StreamWriteValue32Fn write_value_fn() {
  static StreamWriteValue32Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<StreamWriteValue32Fn>(p);
    }
  });
  return fn;
}

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

struct DeviceInfo {
  int sms = 0;
  bool sm100 = false;
};

constexpr int kMaxDevices = 64;

// Per-device facts, filled once per device.
int device_info(DeviceInfo* out) {
  static DeviceInfo table[kMaxDevices];
  static std::once_flag flags[kMaxDevices];
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err);
  if (dev < 0 || dev >= kMaxDevices) return SMB_ERR_CUDA;
  int rc = SMB_OK;
  std::call_once(flags[dev], [&] {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      rc = SMB_ERR_CUDA;
      return;
    }
    table[dev].sms = sms;
    table[dev].sm100 = (major == 10 && minor == 0);
  });
  if (rc != SMB_OK) return rc;
  if (table[dev].sms == 0) return SMB_ERR_CUDA;
  *out = table[dev];
  return SMB_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SMB_DISABLE_PDL");
    return !(v != nullptr && v[0] == '1');
  }();
  return on;
}

int elem_bytes_of(int dtype) { return (dtype == SMB_DTYPE_F16 || dtype == SMB_DTYPE_BF16) ? 2 : 0; }

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_shape(int T, int E, int k, int H, int I, int dtype) {
  if (elem_bytes_of(dtype) == 0) return SMB_ERR_DTYPE;
  if (T < 0 || E < 1 || E > kMaxExperts || k < 1 || k > kMaxTopK || k > E) return SMB_ERR_SHAPE;
  if (H < 128 || H % 128 != 0 || I < 64 || I % 64 != 0) return SMB_ERR_SHAPE;
  if (static_cast<long long>(T) * k > kMaxFlat) return SMB_ERR_SHAPE;
  return SMB_OK;
}

// choose_splits simulates the unit queue (a few ms for the largest shapes), so its
// answer is kept per shape.
int cached_splits(int E, int H, int I, int Tk, int valid, int sms) {
  struct Entry {
    int E, H, I, Tk, valid, sms, s;
  };
  constexpr int kSlots = 128;
  static Entry table[kSlots];
  static int used = 0, next = 0;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i) {
      const Entry& t = table[i];
      if (t.E == E && t.H == H && t.I == I && t.Tk == Tk && t.valid == valid && t.sms == sms) return t.s;
    }
  }
  const int s = choose_splits(E, H, I, Tk, sms, valid);
  std::lock_guard<std::mutex> lock(mu);
  const int slot = used < kSlots ? used++ : (next++ % kSlots);
  table[slot] = Entry{E, H, I, Tk, valid, sms, s};
  return s;
}

// Down split-K factor for these sizes on the current device; `valid` = slots expected to
// hold a token (-1: all Tk).  SMB_SPLIT_K overrides it (experiments; workspaces must then
// be sized in the same environment).
int splits_for(int E, int H, int I, int Tk, int valid, int* out) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != SMB_OK) return rc;
  int s = cached_splits(E, H, I, Tk, valid, di.sms);
  const char* env = std::getenv("SMB_SPLIT_K");
  if (env != nullptr) {
    int v = std::atoi(env);
    if (v >= 1 && v <= I / 64 && v <= kMaxSplits) s = v;
  }
  *out = s;
  return SMB_OK;
}

// Carve the workspace; checks size and alignment.
// `valid`: slots expected to hold a token (-1: all), the expert side of the exchange.
int carve(const void* ws, size_t ws_bytes, int T, int E, int k, int H, int I, int dtype, WsLayout* L,
          int valid = -1) {
  int rc = check_shape(T, E, k, H, I, dtype);
  if (rc != SMB_OK) return rc;
  int s = 1;
  rc = splits_for(E, H, I, T * k, valid, &s);
  if (rc != SMB_OK) return rc;
  *L = make_ws_layout(T, E, k, H, I, elem_bytes_of(dtype), s);
  if (ws == nullptr) return SMB_ERR_NULL;
  if (!aligned(ws, kAlign)) return SMB_ERR_ALIGN;
  if (ws_bytes < L->total) return SMB_ERR_WORKSPACE;
  return SMB_OK;
}

template <typename P>
P* at(const void* ws, size_t off) {
  return reinterpret_cast<P*>(reinterpret_cast<uintptr_t>(ws) + off);
}

// Stage clock of the control block at `ctrl` (a workspace, or an exchange arena).
StageClock* clock_at(const void* ctrl) { return at<StageClock>(ctrl, kStageOffset); }

// Small cache of encoded tensor maps: a layer is called with the same pool and
// workspace over and over, and encoding costs microseconds of host time per map.
struct TmapKey {
  const void* base;
  int dtype;
  uint64_t rows, cols;
  uint32_t box_rows;
  bool operator==(const TmapKey& o) const {
    return base == o.base && dtype == o.dtype && rows == o.rows && cols == o.cols && box_rows == o.box_rows;
  }
};
constexpr int kTmapCacheSize = 64;
struct TmapCache {
  std::mutex mu;
  TmapKey keys[kTmapCacheSize];
  CUtensorMap maps[kTmapCacheSize];
  int used = 0;
  int next = 0;
};
TmapCache g_tmaps;

int encode_2d_uncached(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
                       uint32_t box_rows);

// 2D row-major [rows, cols] tensor of 16-bit elements, box [box_rows, 64], 128B swizzle.
int encode_2d(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  const TmapKey key{base, dtype, rows, cols, box_rows};
  {
    std::lock_guard<std::mutex> lock(g_tmaps.mu);
    for (int i = 0; i < g_tmaps.used; ++i) {
      if (g_tmaps.keys[i] == key) {
        *map = g_tmaps.maps[i];
        return SMB_OK;
      }
    }
  }
  const int rc = encode_2d_uncached(map, base, dtype, rows, cols, box_rows);
  if (rc != SMB_OK) return rc;
  std::lock_guard<std::mutex> lock(g_tmaps.mu);
  const int slot = g_tmaps.used < kTmapCacheSize ? g_tmaps.used++ : (g_tmaps.next++ % kTmapCacheSize);
  g_tmaps.keys[slot] = key;
  g_tmaps.maps[slot] = *map;
  return SMB_OK;
}

int encode_2d_uncached(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
                       uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return SMB_ERR_TMA;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == SMB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SMB_OK : SMB_ERR_TMA;
}

// The router gathers token rows only into the expert-parallel send buffer; then the
// copy is spread over CTAs (2 rows each, at most one CTA per SM): over peer memory each
// CTA waits at its release for its own stores to reach the other GPUs, so fewer rows per
// CTA shorten both its stores and that wait.  Otherwise one CTA routes and permutes.
int route_grid(int Tk, int sms, bool gathers) {
  if (!gathers) return 1;
  int g = (Tk + 1) / 2;
  if (g < 1) g = 1;
  if (g > sms) g = sms;
  return g;
}

// Gate CTAs: every CTA takes ceil(T / SMs) consecutive tokens, no CTA is left empty.
int gate_grid(int T, int sms) {
  const int per = (T + sms - 1) / sms;
  return (T + per - 1) / per;
}

struct EpLayout {
  void* send = nullptr;        // dispatch mode marker (rows go to link.chunk[d])
  int G = 0, C = 0, Eloc = 1;
  EpLink link{};
};

// Pointers of the peer-memory transport for rank `rank` of G, from the arenas of all
// ranks (arenas[rank] is this rank's own).
struct EpPeers {
  uint8_t* arena[kMaxRanks];
  EpArena A;
  int G, rank;
  size_t row_bytes;
};

int ep_peers(void* const* arenas, int G, int rank, int C, int H, int dtype, EpPeers* P) {
  if (G < 1 || G > kMaxRanks || rank < 0 || rank >= G || C < 1) return SMB_ERR_SHAPE;
  if (arenas == nullptr) return SMB_ERR_NULL;
  P->A = make_ep_arena(G, C, H, elem_bytes_of(dtype));
  P->G = G;
  P->rank = rank;
  P->row_bytes = static_cast<size_t>(H) * elem_bytes_of(dtype);
  for (int r = 0; r < G; ++r) {
    if (arenas[r] == nullptr) return SMB_ERR_NULL;
    if (!aligned(arenas[r], kAlign)) return SMB_ERR_ALIGN;
    P->arena[r] = static_cast<uint8_t*>(arenas[r]);
  }
  return SMB_OK;
}
int* ep_ctrl(const EpPeers& P, int r) { return reinterpret_cast<int*>(P.arena[r] + P.A.ctrl); }
int* ep_flags(const EpPeers& P, int r) { return reinterpret_cast<int*>(P.arena[r] + P.A.flags); }

// Router gate inputs of the gated launch (x is the token matrix passed to do_route).
struct GateIn {
  const void* weight = nullptr;  // [E, H] storage dtype
  void* logits_out = nullptr;    // optional [T, E] storage dtype
};

// Shared expert as n pseudo-experts (the last n of E) that every token takes.
struct SharedIn {
  int n = 0;
  const float* w = nullptr;  // [T] or nullptr (weight 1)
};

// E and k count the shared pseudo-experts / slots too.
int do_route(const void* logits, int logits_dtype, const float* in_w, const int32_t* in_ids, const void* x,
             int dtype, int T, int E, int k, int H, int I, int renorm, float* out_w, int32_t* out_ids, void* ws,
             size_t ws_bytes, cudaStream_t stream, const EpLayout& ep = EpLayout(), const GateIn* gate = nullptr,
             const SharedIn& shared = SharedIn()) {
  WsLayout L;
  // the expert side of the exchange: about C of its G x C slots hold a token
  int rc = carve(ws, ws_bytes, T, E, k, H, I, dtype, &L);
  if (rc != SMB_OK) return rc;
  if (logits != nullptr && logits_dtype != SMB_DTYPE_F16 && logits_dtype != SMB_DTYPE_BF16 &&
      logits_dtype != SMB_DTYPE_F32)
    return SMB_ERR_DTYPE;
  // over peer memory a rank without tokens still sends its (empty) chunks and flags
  if (T == 0 && !ep.link.p2p) return SMB_OK;
  if (x == nullptr && T > 0) return SMB_ERR_NULL;
  if (T > 0 && gate == nullptr && logits == nullptr && (in_w == nullptr || in_ids == nullptr))
    return SMB_ERR_NULL;
  if (gate != nullptr && (gate->weight == nullptr || ep.send != nullptr)) return SMB_ERR_NULL;
  if (!aligned(x, 16)) return SMB_ERR_ALIGN;
  if (gate != nullptr && !aligned(gate->weight, 16)) return SMB_ERR_ALIGN;
  DeviceInfo di;
  rc = device_info(&di);
  if (rc != SMB_OK) return rc;
  if (!di.sm100) return SMB_ERR_ARCH;
  RouteArgs a{};
  a.logits = logits;
  a.logits_dtype = logits_dtype;
  a.in_w = in_w;
  a.in_ids = in_ids;
  a.x = x;
  a.T = T;
  a.E = E;
  a.k = k;
  a.k_routed = k - shared.n;
  a.n_shared = shared.n;
  a.shared_w = shared.w;
  a.H = H;
  a.renormalize = renorm ? 1 : 0;
  a.out_w = out_w;
  a.out_ids = out_ids;
  a.expert_off = at<int32_t>(ws, L.expert_off);
  a.perm = at<int32_t>(ws, L.perm);
  a.inv = at<int32_t>(ws, L.inv);
  a.ws_w = at<float>(ws, L.w);
  a.ws_ids = at<int32_t>(ws, L.ids);
  a.status = at<int>(ws, L.status);
  a.done = at<int>(ws, L.done);
  a.done_count = L.ndone;
  a.ep_send = ep.send;
  a.ep_G = ep.G;
  a.ep_C = ep.C;
  a.ep_Eloc = ep.Eloc;
  a.link = ep.link;
  // over peer memory the whole exchange chain stamps the arena's clock
  a.clk = ep.link.p2p ? clock_at(ep.link.ctrl) : clock_at(ws);
  a.stage = 0;
  const int Tk = T * k;
  if (gate != nullptr) {
    // gate + routing in one launch: the gate's CTAs each take ceil(T / SMs) tokens, the
    // last CTA to finish routes every token from the logits in the workspace
    GateArgs g{};
    g.x = x;
    g.weight = gate->weight;
    g.logits = at<float>(ws, L.logits);
    g.logits_out = gate->logits_out;
    g.ticket = at<int>(ws, L.status) + 1;
    g.T = T;
    g.E = E - shared.n;
    g.H = H;
    g.route = 1;
    a.logits = g.logits;
    a.logits_dtype = SMB_DTYPE_F32;
    a.rows_per_cta = Tk;
    cudaError_t err = launch_gate_route(a, g, dtype, gate_grid(T, di.sms), stream, pdl_enabled());
    return err == cudaSuccess ? SMB_OK : cuda_fail(err);
  }
  if (ep.send == nullptr && Tk >= kMultiRouteMinSlots) {
    // large call: many CTAs route their own tokens and meet once on a table of counts (in
    // the workspace's logits area, unused without the gate); ticket and generation words
    // in the control block
    int tpc = (T + di.sms - 1) / di.sms;
    if (tpc < 32) tpc = 32;
    const int grid = (T + tpc - 1) / tpc;
    a.rows_per_cta = tpc * k;
    int* ctrl = at<int>(ws, L.status);
    cudaError_t err = launch_route_multi(a, tpc, grid, at<int>(ws, L.logits), ctrl + 3, ctrl + 4, stream,
                                         pdl_enabled());
    return err == cudaSuccess ? SMB_OK : cuda_fail(err);
  }
  const int grid = route_grid(Tk, di.sms, ep.send != nullptr);
  a.rows_per_cta = (Tk + grid - 1) / grid;
  cudaError_t err = launch_route(a, elem_bytes_of(dtype), grid, stream, pdl_enabled());
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

// Prefill-sized calls (at least 256 routed slots per expert on average, both phases, no
// streamed pages or exchange output) go to the CTA-pair kernels: there the tensor pipe,
// not HBM, bounds the layer.  SMB_PAIR=0 / 1 forces the choice (experiments).
bool use_pair_path(int Tk, int E, int phases, bool special) {
  if (phases != 3 || special) return false;
  static const int forced = [] {
    const char* v = std::getenv("SMB_PAIR");
    return v == nullptr ? -1 : (v[0] == '1' ? 1 : 0);
  }();
  if (forced >= 0) return forced == 1;
  return static_cast<long long>(Tk) >= 256LL * E;
}

// phase bit 1: gate/up GEMM (+SiLU*mul), bit 2: down GEMM (split-K partials); both bits
// run both phases in one persistent launch.
int do_ffn(const void* x, int x_chunk, const void* pool, int64_t num_pages, const int64_t* page_of_expert, int dtype,
           int T, int E, int k, int H, int I, void* ws, size_t ws_bytes, cudaStream_t stream, int phases,
           bool counters_zeroed, const int* page_ready = nullptr, int page_epoch = 0, StageClock* clk = nullptr,
           const EpLink* out_link = nullptr, int recv_G = 0, const int* recv_flags = nullptr,
           const int* recv_epoch = nullptr) {
  WsLayout L;
  int rc = carve(ws, ws_bytes, T, E, k, H, I, dtype, &L, x_chunk > 0 ? x_chunk : -1);
  if (rc != SMB_OK) return rc;
  if (T == 0) return SMB_OK;
  if (pool == nullptr || page_of_expert == nullptr) return SMB_ERR_NULL;
  if ((phases & 1) && x == nullptr) return SMB_ERR_NULL;
  if (!aligned(pool, 16) || !aligned(x, 16)) return SMB_ERR_ALIGN;
  if (num_pages < 1) return SMB_ERR_SHAPE;
  const long long rows1 = static_cast<long long>(num_pages) * 3 * I;
  const long long rows2 = static_cast<long long>(num_pages) * 3 * H;
  if (rows1 >= (1LL << 31) || rows2 >= (1LL << 31)) return SMB_ERR_SHAPE;
  DeviceInfo di;
  rc = device_info(&di);
  if (rc != SMB_OK) return rc;
  if (!di.sm100) return SMB_ERR_ARCH;
  const bool bf16 = dtype == SMB_DTYPE_BF16;

  CUtensorMap w13, w2, txp, ta2;
  if ((rc = encode_2d(&w13, pool, dtype, rows1, H, 128)) != SMB_OK) return rc;
  // token-row tiles for wide experts: the workspace's xp [rows, H] and a2 [rows, I]
  if ((rc = encode_2d(&txp, at<void>(ws, L.xp), dtype, L.rows, H, 64)) != SMB_OK) return rc;
  if ((rc = encode_2d(&ta2, at<void>(ws, L.a2), dtype, L.rows, I, 64)) != SMB_OK) return rc;
  if ((rc = encode_2d(&w2, pool, dtype, rows2, I, 128)) != SMB_OK) return rc;

  FfnArgs args{};
  args.expert_off = at<int32_t>(ws, L.expert_off);
  args.page_of_expert = page_of_expert;
  args.status = at<int>(ws, L.status);
  args.sched = at<int>(ws, L.done);
  args.done = args.sched + 2;
  args.ntc = L.ntc;
  args.x = x;
  args.x_chunk = x_chunk;
  args.inv = at<int32_t>(ws, L.inv);
  args.k = k;
  args.xp = at<void>(ws, L.xp);
  args.a2 = at<void>(ws, L.a2);
  args.part = at<float>(ws, L.part);
  args.num_pages = num_pages;
  args.E = E;
  args.H = H;
  args.I = I;
  args.Tk = T * k;
  args.page_ready = page_ready;
  args.page_epoch = page_epoch;
  args.splits = L.splits;
  args.phase_mask = phases;
  args.clk = clk != nullptr ? clk : clock_at(ws);
  args.tile_done = args.done + static_cast<size_t>(E) * L.splits * L.ntc;
  args.perm = at<int32_t>(ws, L.perm);
  args.ndone = L.ndone;
  args.exit_ticket = at<int>(ws, L.status) + 2;
  if (recv_G > 0) {
    // expert side of the exchange: the kernel routes the received rows itself
    args.recv_G = recv_G;
    args.recv_flags = recv_flags;
    args.recv_epoch = recv_epoch;
    counters_zeroed = true;  // left at zero by the previous launch on this workspace
  }
  if (out_link != nullptr) {
    // expert side of the exchange: the FFN writes the returned rows itself
    args.ep_C = x_chunk;
    args.link = *out_link;
  }
  if (!counters_zeroed) {
    // standalone call: the router zeroed the counters for the first FFN launch only
    cudaError_t err = cudaMemsetAsync(args.sched, 0, sizeof(int) * static_cast<size_t>(L.ndone), stream);
    if (err != cudaSuccess) return cuda_fail(err);
  }
  if (use_pair_path(T * k, E, phases, page_ready != nullptr || out_link != nullptr)) {
    // prefill-sized: gate/up then down on CTA pairs (2-SM MMA), all pairs resident
    const int pairs = ffn_pair_capacity(bf16);
    if (pairs < 1) return cuda_fail(cudaErrorLaunchOutOfResources);
    cudaError_t err = launch_ffn_pair(bf16, 1, pairs, stream, pdl_enabled(), w13, txp, args);
    if (err == cudaSuccess) err = launch_ffn_pair(bf16, 2, pairs, stream, pdl_enabled(), w2, ta2, args);
    return err == cudaSuccess ? SMB_OK : cuda_fail(err);
  }
  cudaError_t err = launch_ffn_gemm(bf16, di.sms, stream, pdl_enabled(), w13, w2, txp, ta2, args);
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int do_combine(void* out, int dtype, int T, int E, int k, int H, int I, const void* ws, size_t ws_bytes,
               cudaStream_t stream) {
  WsLayout L;
  int rc = carve(ws, ws_bytes, T, E, k, H, I, dtype, &L);
  if (rc != SMB_OK) return rc;
  if (T == 0) return SMB_OK;
  if (out == nullptr) return SMB_ERR_NULL;
  if (!aligned(out, 16)) return SMB_ERR_ALIGN;
  CombineArgs a{};
  a.part = at<const float>(ws, L.part);
  a.inv = at<const int32_t>(ws, L.inv);
  a.w = at<const float>(ws, L.w);
  a.out = out;
  a.T = T;
  a.k = k;
  a.H = H;
  a.splits = L.splits;
  a.clk = clock_at(ws);
  cudaError_t err = launch_combine(a, dtype == SMB_DTYPE_BF16, stream, pdl_enabled());
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

}  // namespace

namespace smb {
int record_cuda_error(cudaError_t err) { return cuda_fail(err); }
// Device status word at `status` as an SMB_* code (synchronous on `stream`).
int read_status_word(const int* status, cudaStream_t stream) {
  int h = 0;
  cudaError_t err = cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
  if (err != cudaSuccess) return cuda_fail(err);
  switch (h) {
    case kDevOk: return SMB_OK;
    case kDevTimeout: return SMB_ERR_DEVICE_TIMEOUT;
    case kDevBadPage: return SMB_ERR_BAD_PAGE;
    case kDevBadExpertId: return SMB_ERR_BAD_EXPERT;
    default: return SMB_ERR_CUDA;
  }
}
}  // namespace smb

extern "C" {

int smb_version(void) { return 100; }

const char* smb_strerror(int code) {
  switch (code) {
    case SMB_OK: return "ok";
    case SMB_ERR_SHAPE: return "unsupported size (need H%128==0, I%64==0, 1<=E<=256, 1<=k<=min(E,8), T*k<=16384)";
    case SMB_ERR_DTYPE: return "unsupported dtype (storage f16/bf16; logits f16/bf16/f32)";
    case SMB_ERR_ALIGN: return "misaligned pointer (tensors 16 B, workspace 256 B)";
    case SMB_ERR_WORKSPACE: return "workspace smaller than smb_moe_workspace_bytes";
    case SMB_ERR_CUDA: return "CUDA runtime error (see smb_last_cuda_error)";
    case SMB_ERR_TMA: return "tensor-map encoding failed";
    case SMB_ERR_ARCH: return "current device is not sm_100 (B200)";
    case SMB_ERR_NULL: return "required pointer is NULL";
    case SMB_ERR_DEVICE_TIMEOUT: return "device pipeline wait exceeded its budget";
    case SMB_ERR_BAD_PAGE: return "page_of_expert entry outside [0, num_pages)";
    case SMB_ERR_BAD_EXPERT: return "expert id outside [0, E)";
    case SMB_ERR_SCRATCH_LIMIT: return "workspace need exceeds the 64 MiB static scratch of smb_moe_forward_noalloc";
    default: return "unknown error";
  }
}

const char* smb_last_cuda_error(void) { return g_last_cuda_error; }

size_t smb_moe_workspace_bytes(int T, int E, int k, int H, int I, int dtype) {
  if (check_shape(T, E, k, H, I, dtype) != SMB_OK) return 0;
  int s = 1;
  if (splits_for(E, H, I, T * k, -1, &s) != SMB_OK) return 0;
  return make_ws_layout(T, E, k, H, I, elem_bytes_of(dtype), s).total;
}

size_t smb_moe_ep_workspace_bytes(int G, int C, int E_loc, int H, int I, int dtype) {
  if (G < 1 || G > kMaxRanks || C < 1) return 0;
  const int T = G * C;
  if (check_shape(T, E_loc, 1, H, I, dtype) != SMB_OK) return 0;
  int s = 1;
  if (splits_for(E_loc, H, I, T, C, &s) != SMB_OK) return 0;
  return make_ws_layout(T, E_loc, 1, H, I, elem_bytes_of(dtype), s).total;
}

int smb_moe_splits(int E, int H, int I, int Tk) {
  if (E < 1 || H < 128 || H % 128 != 0 || I < 64 || I % 64 != 0 || Tk < 0) return SMB_ERR_SHAPE;
  int s = 1;
  int rc = splits_for(E, H, I, Tk, -1, &s);
  return rc == SMB_OK ? s : rc;
}

int smb_moe_route(const void* router_logits, int logits_dtype, const void* x, int dtype, int T, int E, int k,
                  int H, int I, int renormalize, float* topk_weights, int32_t* topk_ids, void* ws,
                  size_t ws_bytes, smb_stream_t stream) {
  if (router_logits == nullptr && T > 0) return SMB_ERR_NULL;
  return do_route(router_logits, logits_dtype, nullptr, nullptr, x, dtype, T, E, k, H, I, renormalize,
                  topk_weights, topk_ids, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int smb_moe_permute(const float* topk_weights, const int32_t* topk_ids, const void* x, int dtype, int T, int E,
                    int k, int H, int I, void* ws, size_t ws_bytes, smb_stream_t stream) {
  if ((topk_weights == nullptr || topk_ids == nullptr) && T > 0) return SMB_ERR_NULL;
  return do_route(nullptr, SMB_DTYPE_F32, topk_weights, topk_ids, x, dtype, T, E, k, H, I, 0, nullptr, nullptr,
                  ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int smb_moe_ffn(const void* x, const void* pool, int64_t num_pages, const int64_t* page_of_expert, int dtype, int T,
                int E, int k, int H, int I, void* ws, size_t ws_bytes, smb_stream_t stream) {
  return do_ffn(x, 0, pool, num_pages, page_of_expert, dtype, T, E, k, H, I, ws, ws_bytes,
                reinterpret_cast<cudaStream_t>(stream), 3, false);
}

int smb_moe_gate_up(const void* x, const void* pool, int64_t num_pages, const int64_t* page_of_expert, int dtype,
                    int T, int E, int k, int H, int I, void* ws, size_t ws_bytes, smb_stream_t stream) {
  return do_ffn(x, 0, pool, num_pages, page_of_expert, dtype, T, E, k, H, I, ws, ws_bytes,
                reinterpret_cast<cudaStream_t>(stream), 1, false);
}

int smb_moe_down(const void* pool, int64_t num_pages, const int64_t* page_of_expert, int dtype, int T, int E,
                 int k, int H, int I, void* ws, size_t ws_bytes, smb_stream_t stream) {
  return do_ffn(nullptr, 0, pool, num_pages, page_of_expert, dtype, T, E, k, H, I, ws, ws_bytes,
                reinterpret_cast<cudaStream_t>(stream), 2, false);
}

int smb_moe_combine(void* out, int dtype, int T, int E, int k, int H, int I, const void* ws, size_t ws_bytes,
                    smb_stream_t stream) {
  return do_combine(out, dtype, T, E, k, H, I, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int smb_moe_combine_rows(const void* rows, void* out, int dtype, int T, int E, int k, int H, int I, const void* ws,
                         size_t ws_bytes, smb_stream_t stream) {
  WsLayout L;
  int rc = carve(ws, ws_bytes, T, E, k, H, I, dtype, &L);
  if (rc != SMB_OK) return rc;
  if (T == 0) return SMB_OK;
  if (rows == nullptr || out == nullptr) return SMB_ERR_NULL;
  if (!aligned(rows, 16) || !aligned(out, 16)) return SMB_ERR_ALIGN;
  cudaError_t err = launch_combine_rows(rows, static_cast<long long>(T) * k, at<const int32_t>(ws, L.inv),
                                        at<const float>(ws, L.w), out, T, k, H, dtype == SMB_DTYPE_BF16,
                                        reinterpret_cast<cudaStream_t>(stream), pdl_enabled(), nullptr, nullptr,
                                        clock_at(ws));
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_moe_ep_dispatch(const void* router_logits, int logits_dtype, const void* x, int dtype, int T, int E, int k,
                        int H, int I, int renormalize, int G, int C, void* send, float* topk_weights,
                        int32_t* topk_ids, void* ws, size_t ws_bytes, smb_stream_t stream) {
  if (G < 1 || E % G != 0 || C < T * k || (E / G) * 4 > H * 2) return SMB_ERR_SHAPE;
  if (send == nullptr || (router_logits == nullptr && T > 0)) return SMB_ERR_NULL;
  if (!aligned(send, 16)) return SMB_ERR_ALIGN;
  if (G > kMaxRanks) return SMB_ERR_SHAPE;
  EpLayout ep;
  ep.send = send;
  ep.G = G;
  ep.C = C;
  ep.Eloc = E / G;
  ep.link.nranks = G;
  for (int d = 0; d < G; ++d) {
    ep.link.chunk[d] = static_cast<uint8_t*>(send) + static_cast<size_t>(d) * (C + 1) * H * elem_bytes_of(dtype);
  }
  if (T == 0) {
    // no tokens: the peers must still read zero counts in this rank's header rows
    if (elem_bytes_of(dtype) == 0) return SMB_ERR_DTYPE;
    const size_t row = static_cast<size_t>(H) * elem_bytes_of(dtype);
    cudaError_t err = cudaMemset2DAsync(send, (C + 1) * row, 0, row, G, reinterpret_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? SMB_OK : cuda_fail(err);
  }
  return do_route(router_logits, logits_dtype, nullptr, nullptr, x, dtype, T, E, k, H, I, renormalize, topk_weights,
                  topk_ids, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream), ep);
}

int smb_moe_ep_experts(const void* recv, int G, int C, const void* pool, int64_t num_pages,
                       const int64_t* page_of_expert, int dtype, int E_loc, int H, int I, void* out_rows, void* ws,
                       size_t ws_bytes, smb_stream_t stream) {
  if (G < 1 || C < 1 || E_loc < 1 || E_loc * 4 > H * 2) return SMB_ERR_SHAPE;
  if (recv == nullptr || out_rows == nullptr) return SMB_ERR_NULL;
  if (!aligned(recv, 16) || !aligned(out_rows, 16)) return SMB_ERR_ALIGN;
  const int T = G * C;  // payload rows, one slot each (k = 1)
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (G > kMaxRanks) return SMB_ERR_SHAPE;
  EpLink link{};
  link.nranks = G;
  for (int src = 0; src < G; ++src) {
    link.chunk[src] = static_cast<uint8_t*>(out_rows) + static_cast<size_t>(src) * C * H * elem_bytes_of(dtype);
  }
  // one launch: receive routing from the chunk headers, the FFN, the returned rows
  return do_ffn(recv, C, pool, num_pages, page_of_expert, dtype, T, E_loc, 1, H, I, ws, ws_bytes, s, 3, true, nullptr,
                0, nullptr, &link, G);
}

size_t smb_ep_arena_bytes(int G, int C, int H, int dtype) {
  if (G < 1 || G > kMaxRanks || C < 1 || H < 128 || elem_bytes_of(dtype) == 0) return 0;
  return make_ep_arena(G, C, H, elem_bytes_of(dtype)).total;
}

int smb_ep_ipc_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
  if (dev_ptr == nullptr || ipc_handle == nullptr) return SMB_ERR_NULL;
  if (bytes == 0) return SMB_ERR_SHAPE;
  void* p = nullptr;
  cudaError_t err = cudaMalloc(&p, bytes);
  if (err != cudaSuccess) return cuda_fail(err);
  err = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, p);
  if (err != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(err);
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return SMB_OK;
}

int smb_ep_ipc_open(const void* ipc_handle, void** peer_ptr) {
  if (ipc_handle == nullptr || peer_ptr == nullptr) return SMB_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t err = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_ep_ipc_close(void* peer_ptr) {
  if (peer_ptr == nullptr) return SMB_ERR_NULL;
  cudaError_t err = cudaIpcCloseMemHandle(peer_ptr);
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_ep_ipc_free(void* dev_ptr) {
  if (dev_ptr == nullptr) return SMB_ERR_NULL;
  cudaError_t err = cudaFree(dev_ptr);
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_ep_arena_reset(void* arena, int G, int C, int H, int dtype, smb_stream_t stream) {
  if (arena == nullptr) return SMB_ERR_NULL;
  if (G < 1 || G > kMaxRanks || C < 1 || H < 128 || elem_bytes_of(dtype) == 0) return SMB_ERR_SHAPE;
  if (!aligned(arena, kAlign)) return SMB_ERR_ALIGN;
  const EpArena A = make_ep_arena(G, C, H, elem_bytes_of(dtype));
  // control block (epoch, CTA tickets) and the flag block, everything before the chunks
  cudaError_t err = cudaMemsetAsync(arena, 0, A.recv, reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_moe_ep_dispatch_p2p(const void* router_logits, int logits_dtype, const void* x, int dtype, int T, int E,
                            int k, int H, int I, int renormalize, int G, int rank, int C, void* const* arenas,
                            float* topk_weights, int32_t* topk_ids, void* ws, size_t ws_bytes, smb_stream_t stream) {
  if (G < 1 || E % G != 0 || C < T * k || (E / G) * 4 > H * 2) return SMB_ERR_SHAPE;
  if (router_logits == nullptr && T > 0) return SMB_ERR_NULL;
  EpPeers P;
  int rc = ep_peers(arenas, G, rank, C, H, dtype, &P);
  if (rc != SMB_OK) return rc;
  EpLayout ep;
  ep.send = P.arena[rank];  // dispatch mode; the rows go to the destinations' receive chunks
  ep.G = G;
  ep.C = C;
  ep.Eloc = E / G;
  ep.link.nranks = G;
  ep.link.p2p = 1;
  ep.link.ctrl = ep_ctrl(P, rank);
  for (int d = 0; d < G; ++d) {
    ep.link.chunk[d] = P.arena[d] + P.A.recv + static_cast<size_t>(rank) * (C + 1) * P.row_bytes;
    ep.link.flag[d] = ep_flags(P, d) + rank;
  }
  return do_route(router_logits, logits_dtype, nullptr, nullptr, x, dtype, T, E, k, H, I, renormalize, topk_weights,
                  topk_ids, ws, ws_bytes, reinterpret_cast<cudaStream_t>(stream), ep);
}

int smb_moe_ep_experts_p2p(int G, int rank, int C, void* const* arenas, const void* pool, int64_t num_pages,
                           const int64_t* page_of_expert, int dtype, int E_loc, int H, int I, void* ws,
                           size_t ws_bytes, smb_stream_t stream) {
  if (E_loc < 1 || E_loc * 4 > H * 2) return SMB_ERR_SHAPE;
  EpPeers P;
  int rc = ep_peers(arenas, G, rank, C, H, dtype, &P);
  if (rc != SMB_OK) return rc;
  const int T = G * C;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const void* recv = P.arena[rank] + P.A.recv;
  EpLink link{};
  link.nranks = G;
  link.p2p = 1;
  link.ctrl = ep_ctrl(P, rank);
  for (int src = 0; src < G; ++src) {
    link.chunk[src] = P.arena[src] + P.A.back + static_cast<size_t>(rank) * C * P.row_bytes;
    link.flag[src] = ep_flags(P, src) + kEpReturnFlags + rank;
  }
  // one launch: waits for the sources' flags (one per source), routes the received rows
  // from the chunk headers, runs the FFN, writes every row's output into its source's arena
  // and raises the return flags
  return do_ffn(recv, C, pool, num_pages, page_of_expert, dtype, T, E_loc, 1, H, I, ws, ws_bytes, s, 3, true, nullptr,
                0, clock_at(ep_ctrl(P, rank)), &link, G, ep_flags(P, rank), ep_ctrl(P, rank));
}

int smb_moe_ep_combine_p2p(void* out, int dtype, int T, int E, int k, int H, int I, int G, int rank, int C,
                           void* const* arenas, const void* ws, size_t ws_bytes, smb_stream_t stream) {
  if (G < 1 || E % G != 0 || C < T * k) return SMB_ERR_SHAPE;
  EpPeers P;
  int rc = ep_peers(arenas, G, rank, C, H, dtype, &P);
  if (rc != SMB_OK) return rc;
  WsLayout L;
  rc = carve(ws, ws_bytes, T, E, k, H, I, dtype, &L);
  if (rc != SMB_OK) return rc;
  if (out == nullptr && T > 0) return SMB_ERR_NULL;
  if (T > 0 && !aligned(out, 16)) return SMB_ERR_ALIGN;
  EpLink link{};
  link.nranks = G;
  link.p2p = 1;
  link.ctrl = ep_ctrl(P, rank);
  link.wait_flags = ep_flags(P, rank) + kEpReturnFlags;  // one flag per expert rank
  // T = 0 still takes part: it waits for the returns and advances this rank's epoch
  // the dispatch recorded each slot's row of the returned rows [G][C] in inv
  cudaError_t err = launch_combine_rows(P.arena[rank] + P.A.back, static_cast<long long>(G) * C,
                                        at<const int32_t>(ws, L.inv), at<const float>(ws, L.w), out, T, k, H,
                                        dtype == SMB_DTYPE_BF16, reinterpret_cast<cudaStream_t>(stream),
                                        pdl_enabled(), &link, at<int>(ws, L.status), clock_at(ep_ctrl(P, rank)));
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_moe_ep_combine(const void* back, void* out, int dtype, int T, int E, int k, int H, int I, int G, int C,
                       const void* ws, size_t ws_bytes, smb_stream_t stream) {
  if (G < 1 || E % G != 0 || C < T * k) return SMB_ERR_SHAPE;
  WsLayout L;
  int rc = carve(ws, ws_bytes, T, E, k, H, I, dtype, &L);
  if (rc != SMB_OK) return rc;
  if (T == 0) return SMB_OK;
  if (back == nullptr || out == nullptr) return SMB_ERR_NULL;
  if (!aligned(back, 16) || !aligned(out, 16)) return SMB_ERR_ALIGN;
  // the dispatch recorded each slot's row of the returned rows [G][C] in inv
  cudaError_t err = launch_combine_rows(back, static_cast<long long>(G) * C, at<const int32_t>(ws, L.inv),
                                        at<const float>(ws, L.w), out, T, k, H, dtype == SMB_DTYPE_BF16,
                                        reinterpret_cast<cudaStream_t>(stream), pdl_enabled(), nullptr, nullptr,
                                        clock_at(ws));
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_moe_forward(const void* x, const void* router_logits, int logits_dtype, const void* pool,
                    int64_t num_pages, const int64_t* page_of_expert, int dtype, int T, int E, int k, int H, int I,
                    int renormalize, void* out, float* topk_weights, int32_t* topk_ids, void* ws,
                    size_t ws_bytes, smb_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = smb_moe_route(router_logits, logits_dtype, x, dtype, T, E, k, H, I, renormalize, topk_weights,
                         topk_ids, ws, ws_bytes, stream);
  if (rc != SMB_OK) return rc;
  rc = do_ffn(x, 0, pool, num_pages, page_of_expert, dtype, T, E, k, H, I, ws, ws_bytes, s, 3, true);
  if (rc != SMB_OK) return rc;
  return do_combine(out, dtype, T, E, k, H, I, ws, ws_bytes, s);
}

int smb_moe_forward_routed(const void* x, const float* topk_weights, const int32_t* topk_ids, const void* pool,
                           int64_t num_pages, const int64_t* page_of_expert, int dtype, int T, int E, int k, int H,
                           int I, void* out, void* ws, size_t ws_bytes, smb_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = smb_moe_permute(topk_weights, topk_ids, x, dtype, T, E, k, H, I, ws, ws_bytes, stream);
  if (rc != SMB_OK) return rc;
  rc = do_ffn(x, 0, pool, num_pages, page_of_expert, dtype, T, E, k, H, I, ws, ws_bytes, s, 3, true);
  if (rc != SMB_OK) return rc;
  return do_combine(out, dtype, T, E, k, H, I, ws, ws_bytes, s);
}

int smb_moe_forward_shared(const void* x, const void* router_logits, int logits_dtype, const float* shared_weight,
                           const void* pool, int64_t num_pages, const int64_t* page_of_expert, int dtype, int T,
                           int E, int k, int n_shared, int H, int I, int renormalize, void* out,
                           float* topk_weights, int32_t* topk_ids, void* ws, size_t ws_bytes, smb_stream_t stream) {
  if (n_shared < 0 || k < 1 || k > E) return SMB_ERR_SHAPE;
  if (router_logits == nullptr && T > 0) return SMB_ERR_NULL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SharedIn sh;
  sh.n = n_shared;
  sh.w = shared_weight;
  const int Et = E + n_shared, kt = k + n_shared;
  int rc = do_route(router_logits, logits_dtype, nullptr, nullptr, x, dtype, T, Et, kt, H, I, renormalize,
                    topk_weights, topk_ids, ws, ws_bytes, s, EpLayout(), nullptr, sh);
  if (rc != SMB_OK) return rc;
  rc = do_ffn(x, 0, pool, num_pages, page_of_expert, dtype, T, Et, kt, H, I, ws, ws_bytes, s, 3, true);
  if (rc != SMB_OK) return rc;
  return do_combine(out, dtype, T, Et, kt, H, I, ws, ws_bytes, s);
}

int smb_moe_page_copy(void* page_dst, const void* host_src, size_t bytes, int* page_ready, int epoch,
                      smb_stream_t copy_stream) {
  if (page_dst == nullptr || host_src == nullptr || page_ready == nullptr) return SMB_ERR_NULL;
  if (bytes == 0) return SMB_ERR_SHAPE;
  if (!aligned(page_ready, 4)) return SMB_ERR_ALIGN;
  StreamWriteValue32Fn wv = write_value_fn();
  if (wv == nullptr) return SMB_ERR_CUDA;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(copy_stream);
  cudaError_t err = cudaMemcpyAsync(page_dst, host_src, bytes, cudaMemcpyHostToDevice, s);
  if (err != cudaSuccess) return cuda_fail(err);
  const CUresult r = wv(reinterpret_cast<CUstream>(s), reinterpret_cast<CUdeviceptr>(page_ready),
                        static_cast<cuuint32_t>(epoch), 0);
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuStreamWriteValue32 failed (%d)", static_cast<int>(r));
    return SMB_ERR_CUDA;
  }
  return SMB_OK;
}

int smb_moe_forward_streamed(const void* x, const void* router_logits, int logits_dtype, const void* pool,
                             int64_t num_pages, const int64_t* page_of_expert, const int* page_ready, int page_epoch,
                             int dtype, int T, int E, int k, int H, int I, int renormalize, void* out,
                             float* topk_weights, int32_t* topk_ids, void* ws, size_t ws_bytes, smb_stream_t stream) {
  if (page_ready == nullptr && T > 0) return SMB_ERR_NULL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = smb_moe_route(router_logits, logits_dtype, x, dtype, T, E, k, H, I, renormalize, topk_weights,
                         topk_ids, ws, ws_bytes, stream);
  if (rc != SMB_OK) return rc;
  rc = do_ffn(x, 0, pool, num_pages, page_of_expert, dtype, T, E, k, H, I, ws, ws_bytes, s, 3, true, page_ready,
              page_epoch);
  if (rc != SMB_OK) return rc;
  return do_combine(out, dtype, T, E, k, H, I, ws, ws_bytes, s);
}

int smb_moe_workspace_init(void* ws, size_t ws_bytes, smb_stream_t stream) {
  if (ws == nullptr) return SMB_ERR_NULL;
  if (!aligned(ws, kAlign)) return SMB_ERR_ALIGN;
  if (ws_bytes < kWsHeaderBytes) return SMB_ERR_WORKSPACE;
  cudaError_t err = cudaMemsetAsync(ws, 0, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_moe_gate(const void* x, const void* gate_weight, int dtype, int T, int E, int H, void* router_logits,
                 smb_stream_t stream) {
  if (elem_bytes_of(dtype) == 0) return SMB_ERR_DTYPE;
  if (T < 0 || E < 1 || E > kMaxExperts || H < 128 || H % 128 != 0) return SMB_ERR_SHAPE;
  if (T == 0) return SMB_OK;
  if (x == nullptr || gate_weight == nullptr || router_logits == nullptr) return SMB_ERR_NULL;
  if (!aligned(x, 16) || !aligned(gate_weight, 16)) return SMB_ERR_ALIGN;
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != SMB_OK) return rc;
  if (!di.sm100) return SMB_ERR_ARCH;
  RouteArgs a{};
  a.T = T;
  a.E = E;
  a.k = 1;
  a.k_routed = 1;
  a.H = H;
  GateArgs g{};
  g.x = x;
  g.weight = gate_weight;
  g.logits_out = router_logits;
  g.T = T;
  g.E = E;
  g.H = H;
  g.route = 0;
  g.logits = nullptr;  // logits only: no workspace copy, no routing
  cudaError_t err =
      launch_gate_route(a, g, dtype, gate_grid(T, di.sms), reinterpret_cast<cudaStream_t>(stream), pdl_enabled());
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_moe_forward_gated(const void* x, const void* gate_weight, const void* pool, int64_t num_pages,
                          const int64_t* page_of_expert, int dtype, int T, int E, int k, int H, int I,
                          int renormalize, void* out, void* router_logits, float* topk_weights, int32_t* topk_ids,
                          void* ws, size_t ws_bytes, smb_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  GateIn gate;
  gate.weight = gate_weight;
  gate.logits_out = router_logits;
  if (gate_weight == nullptr && T > 0) return SMB_ERR_NULL;
  int rc = do_route(nullptr, SMB_DTYPE_F32, nullptr, nullptr, x, dtype, T, E, k, H, I, renormalize, topk_weights,
                    topk_ids, ws, ws_bytes, s, EpLayout(), &gate);
  if (rc != SMB_OK) return rc;
  rc = do_ffn(x, 0, pool, num_pages, page_of_expert, dtype, T, E, k, H, I, ws, ws_bytes, s, 3, true);
  if (rc != SMB_OK) return rc;
  return do_combine(out, dtype, T, E, k, H, I, ws, ws_bytes, s);
}

int smb_moe_align_block_size(const int32_t* topk_ids, int numel, int E, int block_size, int32_t* sorted_ids,
                             int32_t* expert_ids, int32_t* num_tokens_post_pad, smb_stream_t stream) {
  if (numel < 0 || E < 1 || E > 4096 || block_size < 1) return SMB_ERR_SHAPE;
  if (sorted_ids == nullptr || expert_ids == nullptr || num_tokens_post_pad == nullptr) return SMB_ERR_NULL;
  if (numel > 0 && topk_ids == nullptr) return SMB_ERR_NULL;
  const long long max_padded = static_cast<long long>(numel) + static_cast<long long>(E) * (block_size - 1);
  if (max_padded >= (1LL << 31)) return SMB_ERR_SHAPE;
  const int max_blocks = static_cast<int>((max_padded + block_size - 1) / block_size);
  cudaError_t err = launch_align(topk_ids, numel, E, block_size, sorted_ids, expert_ids, num_tokens_post_pad,
                                 max_blocks, reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_moe_topk(const void* router_logits, int logits_dtype, int T, int E, int k, int renormalize,
                 float* topk_weights, int32_t* topk_ids, smb_stream_t stream) {
  if (T < 0 || E < 1 || E > kMaxExperts || k < 1 || k > kMaxTopK || k > E) return SMB_ERR_SHAPE;
  if (logits_dtype != SMB_DTYPE_F16 && logits_dtype != SMB_DTYPE_BF16 && logits_dtype != SMB_DTYPE_F32)
    return SMB_ERR_DTYPE;
  if (T == 0) return SMB_OK;
  if (router_logits == nullptr || topk_weights == nullptr || topk_ids == nullptr) return SMB_ERR_NULL;
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != SMB_OK) return rc;
  if (!di.sm100) return SMB_ERR_ARCH;
  cudaError_t err = launch_topk(router_logits, logits_dtype, T, E, k, renormalize ? 1 : 0, topk_weights, topk_ids,
                                reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? SMB_OK : cuda_fail(err);
}

int smb_moe_read_timers(const void* ws, size_t ws_bytes, int reset, smb_timers_t* out, smb_stream_t stream) {
  if (ws == nullptr || out == nullptr) return SMB_ERR_NULL;
  if (!aligned(ws, kAlign)) return SMB_ERR_ALIGN;
  if (ws_bytes < kWsHeaderBytes) return SMB_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  struct {
    DevTimers t;
    StageClock c;
  } h{};
  static_assert(kStageOffset == kTimerOffset + sizeof(DevTimers), "timers then stage clock");
  const void* src = at<const void>(ws, kTimerOffset);
  cudaError_t err = cudaMemcpyAsync(&h, src, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err == cudaSuccess && reset) err = cudaMemsetAsync(const_cast<void*>(src), 0, sizeof(h), s);
  if (err != cudaSuccess) return cuda_fail(err);
  for (int i = 0; i < kStages; ++i) {
    out->stage_ns[i] = h.c.ns[i];
    out->stage_calls[i] = h.c.n[i];
    out->stage_busy_ns[i] = h.c.busy[i];
  }
  DevTimers& t = h.t;
  out->ffn_ns = t.ffn_ns;
  out->recv_wait_ns = t.recv_wait_ns;
  out->combine_wait_ns = t.combine_wait_ns;
  out->ffn_launches = t.ffn_launches;
  out->recv_waits = t.recv_waits;
  out->combine_waits = t.combine_waits;
  out->reserved = 0;
  return SMB_OK;
}

int smb_moe_read_status(const void* ws, size_t ws_bytes, int T, int E, int k, int H, int I, int dtype,
                        smb_stream_t stream) {
  WsLayout L;
  int rc = carve(ws, ws_bytes, T, E, k, H, I, dtype, &L);
  if (rc != SMB_OK) return rc;
  return read_status_word(at<const int>(ws, L.status), reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
