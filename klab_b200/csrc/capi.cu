// C ABI entry points of libklab_b200.so (declared in include/klab_b200.h):
// argument validation, launch planning for the streaming projection kernel,
// options and the per-device status word.
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

#include "gemv_launch.cuh"
#include "klab_kernels.h"

namespace klab {

// Device status word: kernels that give up a bounded wait record a code here.
__device__ int g_status_word;

namespace {

constexpr size_t kXSmemMin = 16 * 1024;       // smallest x staging budget considered
#ifndef KLAB_PREFER_X16
#define KLAB_PREFER_X16 KLAB_MIXED_BF16      // stage 16-bit x unconverted for 16-bit weights
#endif
// Split-K workspace layout: [tickets: kTicketCap u32][partials]. The ticket region
// has a fixed size so that launches of different shapes sharing one workspace
// never see another launch's partials where they expect zeroed tickets.
constexpr size_t kTicketCap = 16384;
constexpr size_t kMaxSmem = 227 * 1024;

std::atomic<int> g_opt_pdl{1};
std::atomic<int> g_opt_split{-1};
std::atomic<int> g_opt_generic{0};
std::atomic<int> g_opt_ctas_per_sm{0};  // 0: as many as fit
// Prologue of the projection kernel: items copied into shared memory (low 4 bits)
// and items prefetched into L2 (next 4 bits) before griddepcontrol.wait; -1: tuned.
std::atomic<int> g_opt_prologue{-1};
// Largest token tile of the CUDA-core kernel (1, 2, 4 or 8). Default 4: two
// 4-token tiles with 16 warps beat one 8-token tile with 8 warps (config 3 M=8:
// 63.3 -> 50.8 us; config 2 M=16 on CUDA cores: 111.7 -> 97.9 us).
std::atomic<int> g_opt_max_tile{4};
// Tensor-core routes: 0 off (CUDA cores only); 1 (default) the fastest measured on B200:
// the warp-level tensor-core token tiles (tile_mma.cu: one weight decode per token tile)
// for INT8 per-row at 2 <= M <= 8 and E2M1/FP16-per-32 at 2 <= M <= 16 with BF16 or FP16
// x, INT8 per-row at M > 8 on tcgen05, M = 1 on the CUDA cores; 2 INT8 per-row and BF16
// weights at M >= 2 on tcgen05 (BF16 M-tiles then differ from M = 1 in the last bits; the
// CUDA-core M-tiles are bit-identical to M = 1); 3 the token tiles for INT8 per-row and
// E2M1 at every M <= 16 (a token's result then does not depend on M), INT8 per-row at
// M > 16 on tcgen05.
std::atomic<int> g_opt_tensor{1};

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int* status = nullptr;
};

std::mutex g_mutex;
DeviceInfo g_devices[64];
std::map<std::tuple<int, int, int, int, int, size_t>, int> g_occupancy;

int current_device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return KLAB_E_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceInfo& info = g_devices[dev];
  if (!info.ready) {
    err = cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return err;
    // The host-side name of a __device__ variable is not its device address;
    // ask the runtime for this device's address once.
    err = cudaGetSymbolAddress(reinterpret_cast<void**>(&info.status), g_status_word);
    if (err != cudaSuccess) return err;
    info.ready = true;
  }
  *out = &info;
  return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int* device_status_address() {
  DeviceInfo* info = nullptr;
  return current_device_info(&info) == 0 ? info->status : nullptr;
}

namespace {

int dtype_bytes(int dt) { return dt == KLAB_DT_F32 ? 4 : 2; }

int vals_of(int wfmt) {
  switch (wfmt) {
    case W_F32:
    case W_LF32:
    case W_FP28: return 4;
    case W_I8_ROW:
    case W_I8_G64: return 16;
    case W_FP4_G32H:
    case W_FP4_G16E: return 32;
    default: return 8;
  }
}

size_t warp_region_bytes(int wfmt) {
  switch (wfmt) {
    case W_BF16: return Layout<W_BF16>::WARP_BYTES;
    case W_F16: return Layout<W_F16>::WARP_BYTES;
    case W_F32:
    case W_LF32:
    case W_FP28: return Layout<W_F32>::WARP_BYTES;
    case W_CBF16: return Layout<W_CBF16>::WARP_BYTES;
    case W_I8_ROW: return Layout<W_I8_ROW>::WARP_BYTES;
    case W_I8_G64: return Layout<W_I8_G64>::WARP_BYTES;
    case W_FP4_G32H: return Layout<W_FP4_G32H>::WARP_BYTES;
    default: return Layout<W_FP4_G16E>::WARP_BYTES;
  }
}

size_t bar_region_bytes(int wfmt, int warps) {
  const int bars = kDepth + (wfmt == W_CBF16 ? kMetaRing : 0);
  return ((static_cast<size_t>(warps) * bars * 8 + 127) / 128) * 128;
}

int tile_for(int m) { return m == 1 ? 1 : m == 2 ? 2 : m <= 4 ? 4 : 8; }

cudaError_t run_family(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ) {
  switch (wfmt) {
    case W_BF16:
    case W_F16:
    case W_F32: return gemv_run_half(wfmt, p, s, stream, occ);
    case W_CBF16: return gemv_run_cbf16(wfmt, p, s, stream, occ);
    case W_I8_ROW:
    case W_I8_G64: return gemv_run_int8(wfmt, p, s, stream, occ);
    case W_FP4_G32H: return gemv_run_fp4a(wfmt, p, s, stream, occ);
    case W_FP4_G16E: return gemv_run_fp4b(wfmt, p, s, stream, occ);
    case W_LF32:
    case W_FP28: return gemv_run_lossless(wfmt, p, s, stream, occ);
    default: return cudaErrorNotSupported;
  }
}

int occupancy(int wfmt, const LaunchShape& s) {
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, wfmt, s.xfmt * 16 + s.xmode, s.mt, 0, s.smem);
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end()) return it->second;
  }
  int occ = 0;
  GemvParams dummy = {};
  if (run_family(wfmt, dummy, s, nullptr, &occ) != cudaSuccess) occ = 0;
  std::lock_guard<std::mutex> lock(g_mutex);
  g_occupancy[key] = occ;
  return occ;
}

bool tma_eligible(int wfmt, const void* w, const void* aux, int k) {
  switch (wfmt) {
    case W_BF16:
    case W_F16: return aligned16(w) && k % 8 == 0;
    case W_F32: return aligned16(w) && k % 4 == 0;
    case W_I8_ROW: return aligned16(w) && k % 16 == 0;
    case W_CBF16:
    case W_I8_G64:
    case W_FP4_G32H:
    case W_FP4_G16E: return aligned16(w) && aligned16(aux) && k % 256 == 0;
    default: return false;
  }
}

bool x_compatible(int wfmt, int xdt) {
  switch (wfmt) {
    case W_BF16:
    case W_CBF16: return xdt == KLAB_DT_BF16;
    case W_F16: return xdt == KLAB_DT_F16;
    case W_F32:
    case W_LF32:
    case W_FP28: return xdt == KLAB_DT_F32;
    default: return xdt == KLAB_DT_BF16 || xdt == KLAB_DT_F16 || xdt == KLAB_DT_F32;
  }
}

int shape_ok(int wfmt, int k) {
  switch (wfmt) {
    case W_CBF16:
    case W_I8_G64:
    case W_LF32:
    case W_FP28: return k % 64 == 0;
    case W_FP4_G32H: return k % 32 == 0;
    case W_FP4_G16E: return k % 16 == 0;
    default: return 1;
  }
}

// A launch planned once (klab_plan_create) and replayed with new pointers.
struct PlannedLaunch {
  int wfmt = 0;
  GemvParams p{};
  LaunchShape s{};
  size_t ws_need = 0;  // split-K workspace the launch needs (0: no split)
};

size_t workspace_need(int tiles, int mt, int n, int chunks) {
  return kTicketCap * 4 + static_cast<size_t>(tiles) * mt * n * chunks * 4;
}

int run_gemv_multi(int wfmt, int xdt, const void* x, int ldx, int nseg, const void* const* w,
                   const void* const* aux, const float* gscale, void* const* out, const int* ldo, const int* nrows,
                   int out_dt, int m, int k, void* ws, size_t ws_bytes, void* stream,
                   const klab_gather_t* gather = nullptr, const void* const* aux2 = nullptr,
                   PlannedLaunch* plan_out = nullptr, const Prologue* pro = nullptr) {
  if (!x || !w || !out || !ldo || !nrows || nseg < 1 || nseg > kMaxSegs) return KLAB_E_INVALID;
  if (m <= 0 || k <= 0 || ldx < k) return KLAB_E_INVALID;
  if (wfmt < W_BF16 || wfmt > W_FP28) return KLAB_E_UNSUPPORTED;
  if (!x_compatible(wfmt, xdt)) return KLAB_E_UNSUPPORTED;
  if (wfmt == W_LF32 && !aux2) return KLAB_E_INVALID;
  if (out_dt != KLAB_DT_BF16 && out_dt != KLAB_DT_F32) return KLAB_E_UNSUPPORTED;
  const bool needs_aux = wfmt >= W_CBF16;
  if (wfmt == W_FP4_G16E && !gscale) return KLAB_E_INVALID;
  if (!shape_ok(wfmt, k)) return KLAB_E_SHAPE;
  long long total = 0;
  for (int i = 0; i < nseg; ++i) {
    if (!w[i] || !out[i] || nrows[i] <= 0 || ldo[i] < nrows[i]) return KLAB_E_INVALID;
    if (needs_aux && (!aux || !aux[i])) return KLAB_E_INVALID;
    if (wfmt == W_LF32 && !aux2[i]) return KLAB_E_INVALID;
    total += nrows[i];
  }
  if (total >= (1ll << 31)) return KLAB_E_SHAPE;
  const int n = static_cast<int>(total);

  DeviceInfo* info = nullptr;
  int rc = current_device_info(&info);
  if (rc) return rc;

  const int vals = vals_of(wfmt);
  const int kc = 256 * vals;
  const int chunks = (k + kc - 1) / kc;
  const int seg_cols = 32 * vals;
  const long long kpad = ((static_cast<long long>(k) + seg_cols - 1) / seg_cols) * seg_cols;
  const int xb = dtype_bytes(xdt);
  const bool x_global_ok =
      aligned16(x) && (static_cast<long long>(ldx) * xb) % 16 == 0 && k % vals == 0;

  if (gather && gather->npeers > 0) {
    if (gather->npeers > kMaxPeers || gather->rank < 0 || gather->rank >= gather->npeers || !gather->epoch)
      return KLAB_E_INVALID;
    if (gather->seg >= nseg || (gather->seg >= 0 && out_dt != KLAB_DT_BF16)) return KLAB_E_UNSUPPORTED;
    if (gather->signal_slot >= 0 && !gather->done) return KLAB_E_INVALID;
    for (int q = 0; q < gather->npeers; ++q) {
      if (gather->seg >= 0 && !gather->peer_out[q]) return KLAB_E_INVALID;
      if (gather->signal_slot >= 0 && !gather->peer_flags[q]) return KLAB_E_INVALID;
    }
  }
  const bool gathered_x = gather && gather->npeers > 0 && gather->wait_flags;
  // A fused elementwise op computes x while staging it: BF16 x and weights, K % 8 == 0.
  if (pro && (xdt != KLAB_DT_BF16 || (wfmt != W_BF16 && wfmt != W_CBF16) || k % 8 || gather))
    return KLAB_E_UNSUPPORTED;
  const int tensor = g_opt_tensor.load();
  // INT8 per-row and E2M1/FP16-per-32 weights: warp-level tensor-core token tiles.
  const int tile_max = tensor == 3 ? 16 : (wfmt == W_I8_ROW ? 8 : 16), tile_min = tensor == 3 ? 1 : 2;
  if ((tensor == 1 || tensor == 3) && !plan_out && !pro && m >= tile_min && m <= tile_max && nseg == 1 && !gather &&
      (xdt == KLAB_DT_BF16 || xdt == KLAB_DT_F16) && (wfmt == W_I8_ROW || wfmt == W_FP4_G32H)) {
    const int rc_tm = tile_mma_launch(wfmt == W_I8_ROW ? 0 : 1, xdt == KLAB_DT_F16, x, ldx, w[0], aux[0], out[0],
                                      ldo[0], out_dt == KLAB_DT_F32, m, nrows[0], k, ws, ws_bytes, info->sms,
                                      info->status, g_opt_pdl.load() != 0, static_cast<cudaStream_t>(stream));
    if (rc_tm != KLAB_E_ALIGN && rc_tm != KLAB_E_UNSUPPORTED) return rc_tm;  // else the CUDA cores
  }
  // Token tiles of INT8 (and, optionally, BF16) weights on tcgen05.
  if (!plan_out && !pro && m >= 2 && nseg == 1 && !gather && xdt == KLAB_DT_BF16 &&
      ((wfmt == W_I8_ROW && (tensor == 2 || (tensor == 1 && m > 8) || (tensor == 3 && m > 16))) ||
       (wfmt == W_BF16 && tensor == 2))) {
    const int rc_tc = tc_gemm_launch(wfmt == W_I8_ROW ? 1 : 0, x, ldx, w[0], wfmt == W_I8_ROW ?
                                     static_cast<const float*>(aux[0]) : nullptr, out[0], ldo[0],
                                     out_dt == KLAB_DT_F32, m, nrows[0], k, info->status,
                                     static_cast<cudaStream_t>(stream));
    if (rc_tc != KLAB_E_ALIGN) return rc_tc;  // misaligned operands fall through to the CUDA cores
  }
  int mt = tile_for(m);
  while (mt > g_opt_max_tile.load()) mt /= 2;
  int xmode = XM_SMEM;
  // 16-bit x is staged unconverted; the x budget is what the rings leave of the
  // CTA's shared memory, so wide token tiles keep x on chip instead of
  // re-reading it from L1 for every item.
  const bool x16 = KLAB_PREFER_X16 && xdt != KLAB_DT_F32;
  for (;;) {
    const int w_ = warps_for(wfmt, mt);
    const size_t rings = bar_region_bytes(wfmt, w_) + static_cast<size_t>(w_) * warp_region_bytes(wfmt);
    const size_t cap = rings + kXSmemMin < kMaxSmem ? kMaxSmem - rings : kXSmemMin;
    if (x16 && static_cast<size_t>(mt) * kpad * 2 <= cap) {
      xmode = XM_SMEM16;
      break;
    }
    if (!x16 && static_cast<size_t>(mt) * kpad * 4 <= cap) {
      xmode = XM_SMEM;
      break;
    }
    // Gathered x must be staged (its global reads bypass L1); never read it in place.
    if (x_global_ok && !gathered_x && !pro) {
      xmode = XM_GLOBAL;
      break;
    }
    if (mt == 1) return KLAB_E_SHAPE;
    mt /= 2;
  }
  const int tiles = (m + mt - 1) / mt;
  if (tiles > 65535) return KLAB_E_SHAPE;

  LaunchShape s = {};
  s.xfmt = xdt;
  s.xmode = xmode;
  s.mt = mt;
  s.pdl = g_opt_pdl.load() != 0;
  const int warps = warps_for(wfmt, mt);
  s.smem = bar_region_bytes(wfmt, warps) + warps * warp_region_bytes(wfmt) +
           (xmode == XM_SMEM ? static_cast<size_t>(mt) * kpad * 4
                             : xmode == XM_SMEM16 ? static_cast<size_t>(mt) * kpad * 2 : 0);
  if (s.smem > kMaxSmem) return KLAB_E_SHAPE;
  int occ = occupancy(wfmt, s);
  if (occ <= 0) return KLAB_E_UNSUPPORTED;
  const int cap = g_opt_ctas_per_sm.load();
  if (cap > 0 && cap < occ) occ = cap;
  const int gmax = occ * info->sms / tiles > 0 ? occ * info->sms / tiles : 1;

  GemvParams p = {};
  if (pro) p.pro = *pro;
  p.x = x;
  p.gscale = gscale;
  p.nseg = nseg;
  p.gather.seg = -1;
  p.gather.signal_slot = -1;
  p.gather.wait_slot = -1;
  if (gather && gather->npeers > 0) {
    p.gather.npeers = gather->npeers;
    p.gather.rank = gather->rank;
    p.gather.seg = gather->seg;
    for (int q = 0; q < gather->npeers; ++q) {
      p.gather.peer_out[q] = gather->peer_out[q];
      p.gather.peer_flags[q] = gather->peer_flags[q];
    }
    p.gather.signal_slot = gather->signal_slot;
    p.gather.wait_flags = gather->wait_flags;
    p.gather.wait_slot = gather->wait_slot;
    p.gather.epoch = gather->epoch;
    p.gather.done = gather->done;
  }
  bool tma = g_opt_generic.load() == 0;
  int row0 = 0;
  for (int i = 0; i < nseg; ++i) {
    p.seg[i].w = w[i];
    p.seg[i].aux = needs_aux ? aux[i] : nullptr;
    p.seg[i].aux2 = aux2 ? aux2[i] : nullptr;
    p.seg[i].out = out[i];
    p.seg[i].ldo = ldo[i];
    p.seg[i].row0 = row0;
    row0 += nrows[i];
    tma = tma && tma_eligible(wfmt, w[i], needs_aux ? aux[i] : nullptr, k);
  }
  p.status = info->status;
  p.m = m;
  p.n = n;
  p.k = k;
  p.ldx = ldx;
  p.out_f32 = out_dt == KLAB_DT_F32;
  p.chunks = chunks;
  p.use_tma = tma;
  {
    const int pro = g_opt_prologue.load();
    p.pro_smem = pro < 0 ? kProSmem : (pro & 15);
    p.pro_l2 = pro < 0 ? kProL2 : (pro >> 4);
  }

  const size_t need = workspace_need(tiles, mt, n, chunks);
  const bool can_split = ws && ws_bytes >= need && chunks >= 2 && aligned16(ws) &&
                         static_cast<size_t>(tiles) * n <= kTicketCap;
  const int opt = g_opt_split.load();
  const bool split = can_split && (opt == 1 || (opt == -1 && chunks >= 3 &&
                                                static_cast<long long>(n) * 2 < static_cast<long long>(gmax) * warps));
  int grid_x;
  if (split) {
    const long long items = static_cast<long long>(n) * chunks;
    const long long want = (items + warps - 1) / warps;
    grid_x = static_cast<int>(want < gmax ? want : gmax);
    p.split = 1;
    p.tickets = static_cast<unsigned*>(ws);
    p.ws = reinterpret_cast<float*>(static_cast<char*>(ws) + kTicketCap * 4);
  } else {
    grid_x = n < gmax ? n : gmax;
    p.split = 0;
  }
  s.grid = dim3(grid_x, tiles, 1);
  if (plan_out) {
    plan_out->wfmt = wfmt;
    plan_out->p = p;
    plan_out->s = s;
    plan_out->ws_need = split ? need : 0;
    return 0;
  }
  return run_family(wfmt, p, s, static_cast<cudaStream_t>(stream), nullptr);
}

int run_gemv(int wfmt, int xdt, const void* x, int ldx, const void* w, const void* aux, const float* gscale,
             void* out, int ldo, int out_dt, int m, int n, int k, void* ws, size_t ws_bytes, void* stream) {
  if (!x || !w || !out) return KLAB_E_INVALID;
  if (m <= 0 || n <= 0 || k <= 0 || ldx < k || ldo < n) return KLAB_E_INVALID;
  if (wfmt >= W_CBF16 && wfmt <= W_FP28 && !aux) return KLAB_E_INVALID;
  if (wfmt == W_LF32) return KLAB_E_UNSUPPORTED;  // needs the exponent stream: klab_lossless_f32_linear
  const void* ws_[1] = {w};
  const void* as_[1] = {aux};
  void* os_[1] = {out};
  const int ldo_[1] = {ldo};
  const int n_[1] = {n};
  return run_gemv_multi(wfmt, xdt, x, ldx, 1, ws_, as_, gscale, os_, ldo_, n_, out_dt, m, k, ws, ws_bytes, stream);
}

// Byte ranges [a, a + na) and [b, b + nb) share at least one byte.
bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + nb && pb < pa + na;
}

}  // namespace
}  // namespace klab

using namespace klab;

extern "C" {

int klab_gemv(int wfmt, int xdtype, const void* x, int ldx, const void* w, const void* aux, const float* gscale,
              void* out, int ldo, int out_dtype, int m, int n, int k, void* workspace, size_t workspace_bytes,
              void* stream) {
  return run_gemv(wfmt, xdtype, x, ldx, w, aux, gscale, out, ldo, out_dtype, m, n, k, workspace, workspace_bytes,
                  stream);
}

int klab_raw_linear(const void* x, const void* w, void* out, int out_dtype, int m, int n, int k, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return run_gemv(W_BF16, KLAB_DT_BF16, x, k, w, nullptr, nullptr, out, n, out_dtype, m, n, k, workspace,
                  workspace_bytes, stream);
}

int klab_add_rmsnorm_linear(const void* res, const void* y, const void* norm_weight, float eps, const void* w,
                            void* out, void* x_out, int m, int n, int k, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (!res || !y || !norm_weight || !w || !out || m <= 0 || n <= 0 || k <= 0 || !(eps > 0.0f)) return KLAB_E_INVALID;
  if (k % 8) return KLAB_E_SHAPE;
  // Every CTA re-reads res and y while it stages x, and column 0 of the grid writes x_out: an x_out
  // (or out) that overlaps what the launch reads would feed updated values to later CTAs.
  const size_t act = size_t(m) * size_t(k) * 2, outb = size_t(m) * size_t(n) * 2;
  if (x_out && (overlaps(x_out, act, res, act) || overlaps(x_out, act, y, act) ||
                overlaps(x_out, act, norm_weight, size_t(k) * 2) || overlaps(x_out, act, out, outb)))
    return KLAB_E_INVALID;
  if (overlaps(out, outb, res, act) || overlaps(out, outb, y, act) || overlaps(out, outb, norm_weight, size_t(k) * 2))
    return KLAB_E_INVALID;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(res) | reinterpret_cast<uintptr_t>(y) |
                        reinterpret_cast<uintptr_t>(norm_weight) | reinterpret_cast<uintptr_t>(x_out);
  if (mis & 3) return KLAB_E_ALIGN;
  Prologue pr = {};
  pr.op = PRO_ADD_RMSNORM;
  pr.ld = k;
  pr.eps = eps;
  pr.a = res;
  pr.b = y;
  pr.w = norm_weight;
  pr.x_out = x_out;
  pr.x_out_ld = k;
  const void* ws_[1] = {w};
  const void* as_[1] = {nullptr};
  void* os_[1] = {out};
  const int ldo_[1] = {n}, n_[1] = {n};
  return run_gemv_multi(W_BF16, KLAB_DT_BF16, res, k, 1, ws_, as_, nullptr, os_, ldo_, n_, KLAB_DT_BF16, m, k,
                        workspace, workspace_bytes, stream, nullptr, nullptr, nullptr, &pr);
}

int klab_silu_mul_linear(const void* gu, const void* w, void* out, int m, int n, int inter, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (!gu || !w || !out || m <= 0 || n <= 0 || inter <= 0) return KLAB_E_INVALID;
  if (inter % 8) return KLAB_E_SHAPE;
  if (overlaps(out, size_t(m) * size_t(n) * 2, gu, size_t(m) * size_t(inter) * 4)) return KLAB_E_INVALID;
  if (reinterpret_cast<uintptr_t>(gu) & 3) return KLAB_E_ALIGN;
  Prologue pr = {};
  pr.op = PRO_SILU_MUL;
  pr.ld = 2 * inter;
  pr.a = gu;
  const void* ws_[1] = {w};
  const void* as_[1] = {nullptr};
  void* os_[1] = {out};
  const int ldo_[1] = {n}, n_[1] = {n};
  return run_gemv_multi(W_BF16, KLAB_DT_BF16, gu, 2 * inter, 1, ws_, as_, nullptr, os_, ldo_, n_, KLAB_DT_BF16, m, inter,
                        workspace, workspace_bytes, stream, nullptr, nullptr, nullptr, &pr);
}

int klab_coded_linear(const void* x, const void* payload, const uint32_t* metadata, void* out, int out_dtype, int m,
                      int n, int k, void* workspace, size_t workspace_bytes, void* stream) {
  if (payload && (reinterpret_cast<uintptr_t>(payload) & 31u)) return KLAB_E_ALIGN;
  return run_gemv(W_CBF16, KLAB_DT_BF16, x, k, payload, metadata, nullptr, out, n, out_dtype, m, n, k, workspace,
                  workspace_bytes, stream);
}

int klab_half_linear(const void* x, const void* w, int dtype, float* out, int m, int n, int k, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (dtype != KLAB_DT_BF16 && dtype != KLAB_DT_F16) return KLAB_E_UNSUPPORTED;
  return run_gemv(dtype == KLAB_DT_BF16 ? W_BF16 : W_F16, dtype, x, k, w, nullptr, nullptr, out, n, KLAB_DT_F32, m,
                  n, k, workspace, workspace_bytes, stream);
}

int klab_f32_linear(const float* x, const float* w, float* out, int m, int n, int k, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return run_gemv(W_F32, KLAB_DT_F32, x, k, w, nullptr, nullptr, out, n, KLAB_DT_F32, m, n, k, workspace,
                  workspace_bytes, stream);
}

int klab_int8_linear(const void* x, int xdtype, const int8_t* codes, const float* scales, int group, void* out,
                     int out_dtype, int m, int n, int k, void* workspace, size_t workspace_bytes, void* stream) {
  if (group != 0 && group != 64) return KLAB_E_UNSUPPORTED;
  return run_gemv(group ? W_I8_G64 : W_I8_ROW, xdtype, x, k, codes, scales, nullptr, out, n, out_dtype, m, n, k,
                  workspace, workspace_bytes, stream);
}

int klab_fp4_linear(const void* x, int xdtype, const uint8_t* packed, const void* scales, int scale_kind,
                    const float* gscale, void* out, int out_dtype, int m, int n, int k, void* workspace,
                    size_t workspace_bytes, void* stream) {
  int wfmt;
  if (scale_kind == KLAB_FP4_E4M3_G16)
    wfmt = W_FP4_G16E;
  else if (scale_kind == KLAB_FP4_F16_G32)
    wfmt = W_FP4_G32H;
  else
    return KLAB_E_UNSUPPORTED;
  return run_gemv(wfmt, xdtype, x, k, packed, scales, gscale, out, n, out_dtype, m, n, k, workspace,
                  workspace_bytes, stream);
}

int klab_lossless_f32_linear(const float* x, const uint8_t* mantissa, const uint8_t* exponents,
                             const int32_t* metadata, float* out, int m, int n, int k, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (!x || !mantissa || !exponents || !metadata || !out || m <= 0 || n <= 0 || k <= 0) return KLAB_E_INVALID;
  if (reinterpret_cast<uintptr_t>(mantissa) & 3u) return KLAB_E_ALIGN;
  const void* w_[1] = {mantissa};
  const void* a_[1] = {metadata};
  const void* e_[1] = {exponents};
  void* o_[1] = {out};
  const int ldo_[1] = {n};
  const int n_[1] = {n};
  return run_gemv_multi(W_LF32, KLAB_DT_F32, x, k, 1, w_, a_, nullptr, o_, ldo_, n_, KLAB_DT_F32, m, k, workspace,
                        workspace_bytes, stream, nullptr, e_);
}

int klab_fp28_linear(const float* x, const int32_t* payload, const int32_t* metadata, float* out, int m, int n,
                     int k, void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !payload || !metadata || !out) return KLAB_E_INVALID;
  if (reinterpret_cast<uintptr_t>(payload) & 3u) return KLAB_E_ALIGN;
  return run_gemv(W_FP28, KLAB_DT_F32, x, k, payload, metadata, nullptr, out, n, KLAB_DT_F32, m, n, k, workspace,
                  workspace_bytes, stream);
}

int klab_lossless_f32_unpack(const uint8_t* mantissa, const uint8_t* exponents, const int32_t* metadata, float* out,
                             long long count, void* stream) {
  if (!mantissa || !exponents || !metadata || !out || count <= 0) return KLAB_E_INVALID;
  if (count % 64) return KLAB_E_SHAPE;
  if ((reinterpret_cast<uintptr_t>(mantissa) & 3u) || (reinterpret_cast<uintptr_t>(out) & 15u)) return KLAB_E_ALIGN;
  return launch_lossless_unpack(mantissa, exponents, nullptr, reinterpret_cast<const unsigned*>(metadata), out,
                                count, static_cast<cudaStream_t>(stream));
}

int klab_fp28_unpack(const int32_t* payload, const int32_t* metadata, float* out, long long count, void* stream) {
  if (!payload || !metadata || !out || count <= 0) return KLAB_E_INVALID;
  if (count % 64) return KLAB_E_SHAPE;
  if (reinterpret_cast<uintptr_t>(out) & 15u) return KLAB_E_ALIGN;
  return launch_lossless_unpack(nullptr, nullptr, payload, reinterpret_cast<const unsigned*>(metadata), out, count,
                                static_cast<cudaStream_t>(stream));
}

int klab_gemv_multi(int wfmt, int xdtype, const void* x, int ldx, int nseg, const void* const* w,
                    const void* const* aux, const float* gscale, void* const* out, const int* ldo, const int* n,
                    int out_dtype, int m, int k, void* workspace, size_t workspace_bytes, void* stream) {
  return run_gemv_multi(wfmt, xdtype, x, ldx, nseg, w, aux, gscale, out, ldo, n, out_dtype, m, k, workspace,
                        workspace_bytes, stream);
}

int klab_gemv_multi_gather(int wfmt, int xdtype, const void* x, int ldx, int nseg, const void* const* w,
                           const void* const* aux, const float* gscale, void* const* out, const int* ldo,
                           const int* n, int out_dtype, int m, int k, const klab_gather_t* gather, void* workspace,
                           size_t workspace_bytes, void* stream) {
  return run_gemv_multi(wfmt, xdtype, x, ldx, nseg, w, aux, gscale, out, ldo, n, out_dtype, m, k, workspace,
                        workspace_bytes, stream, gather);
}

// ---------------------------------------------------------------- prepared plans

struct Plan {
  PlannedLaunch launch;
  int device = -1;
  int m = 0, n = 0, k = 0, xdtype = 0, out_dtype = 0;
  void* ws = nullptr;
};

int klab_plan_create(int wfmt, int xdtype, int out_dtype, int m, int n, int k, void** plan_out) {
  if (!plan_out) return KLAB_E_INVALID;
  *plan_out = nullptr;
  if (wfmt < W_BF16 || wfmt > W_FP28 || m <= 0 || n <= 0 || k <= 0) return KLAB_E_INVALID;
  // Plan with stand-in addresses that satisfy every alignment the kernels use;
  // launches check that the real pointers do too.
  void* const fake = reinterpret_cast<void*>(static_cast<uintptr_t>(1) << 20);
  const void* w_[1] = {fake};
  const void* a_[1] = {fake};
  const void* e_[1] = {fake};
  void* o_[1] = {fake};
  const int ldo_[1] = {n};
  const int n_[1] = {n};
  const size_t ws_bytes = klab_gemv_workspace_bytes(wfmt, m, n, k);
  Plan* plan = new Plan();
  int rc = run_gemv_multi(wfmt, xdtype, fake, k, 1, w_, a_, static_cast<const float*>(fake), o_, ldo_, n_,
                          out_dtype, m, k, ws_bytes ? fake : nullptr, ws_bytes, nullptr, nullptr,
                          wfmt == W_LF32 ? e_ : nullptr, &plan->launch);
  if (rc == 0) rc = cudaGetDevice(&plan->device);
  if (rc == 0 && plan->launch.ws_need) {
    rc = cudaMalloc(&plan->ws, plan->launch.ws_need);
    if (rc == 0) rc = cudaMemset(plan->ws, 0, plan->launch.ws_need);
  }
  if (rc) {
    if (plan->ws) cudaFree(plan->ws);
    delete plan;
    return rc;
  }
  plan->m = m;
  plan->n = n;
  plan->k = k;
  plan->xdtype = xdtype;
  plan->out_dtype = out_dtype;
  if (plan->ws) {
    plan->launch.p.tickets = static_cast<unsigned*>(plan->ws);
    plan->launch.p.ws = reinterpret_cast<float*>(static_cast<char*>(plan->ws) + kTicketCap * 4);
  }
  *plan_out = plan;
  return 0;
}

int klab_plan_launch(void* plan_ptr, const void* x, const void* w, const void* aux, const void* aux2,
                     const float* gscale, void* out, void* stream) {
  Plan* plan = static_cast<Plan*>(plan_ptr);
  if (!plan || !x || !w || !out) return KLAB_E_INVALID;
  const int wfmt = plan->launch.wfmt;
  if (wfmt >= W_CBF16 && !aux) return KLAB_E_INVALID;
  if ((wfmt == W_LF32 && !aux2) || (wfmt == W_FP4_G16E && !gscale)) return KLAB_E_INVALID;
  if (!aligned16(x) || !aligned16(w) || (aux && !aligned16(aux)) || (aux2 && !aligned16(aux2))) return KLAB_E_ALIGN;
  if (wfmt == W_CBF16 && (reinterpret_cast<uintptr_t>(w) & 31u)) return KLAB_E_ALIGN;
  GemvParams p = plan->launch.p;
  p.x = x;
  p.gscale = gscale;
  p.seg[0].w = w;
  p.seg[0].aux = wfmt >= W_CBF16 ? aux : nullptr;
  p.seg[0].aux2 = aux2;
  p.seg[0].out = out;
  return run_family(wfmt, p, plan->launch.s, static_cast<cudaStream_t>(stream), nullptr);
}

int klab_plan_info(void* plan_ptr, char* buffer, size_t bytes) {
  Plan* plan = static_cast<Plan*>(plan_ptr);
  if (!plan || !buffer || bytes == 0) return KLAB_E_INVALID;
  const LaunchShape& s = plan->launch.s;
  const char* xmodes[] = {"smem_fp32", "global", "smem_16bit"};
  const int warps = warps_for(plan->launch.wfmt, s.mt);
  const int len = std::snprintf(
      buffer, bytes,
      "{\"wfmt\": %d, \"xdtype\": %d, \"out_dtype\": %d, \"shape_mnk\": [%d, %d, %d], \"tile\": %d, "
      "\"x_staging\": \"%s\", \"grid\": [%u, %u, 1], \"block\": [%d, 1, 1], \"dynamic_shared_bytes\": %zu, "
      "\"split_k\": %s, \"workspace_bytes\": %zu, \"bulk_copy\": %s, \"pdl\": %s, \"device\": %d, "
      "\"kernel\": \"stream_gemv_kernel<%d,%d,%d,%d>\"}",
      plan->launch.wfmt, plan->xdtype, plan->out_dtype, plan->m, plan->n, plan->k, s.mt, xmodes[s.xmode],
      s.grid.x, s.grid.y, warps * 32, s.smem, plan->launch.p.split ? "true" : "false", plan->launch.ws_need,
      plan->launch.p.use_tma ? "true" : "false", s.pdl ? "true" : "false", plan->device, plan->launch.wfmt,
      s.xfmt, s.xmode, s.mt);
  return (len < 0 || static_cast<size_t>(len) >= bytes) ? KLAB_E_SHAPE : 0;
}

int klab_plan_destroy(void* plan_ptr) {
  Plan* plan = static_cast<Plan*>(plan_ptr);
  if (!plan) return KLAB_E_INVALID;
  if (plan->ws) cudaFree(plan->ws);
  delete plan;
  return 0;
}

size_t klab_gemv_workspace_bytes(int wfmt, int m, int n, int k) {
  if (wfmt < W_BF16 || wfmt > W_FP28 || m <= 0 || n <= 0 || k <= 0) return 0;
  const int kc = 256 * vals_of(wfmt);
  const int chunks = (k + kc - 1) / kc;
  // The warp-level tensor-core token tiles keep phase partials of row groups split between CTAs.
  size_t best = (m <= 16 && (wfmt == W_I8_ROW || wfmt == W_FP4_G32H))
                    ? tile_mma_workspace(wfmt == W_I8_ROW ? 0 : 1, m, n, k) : 0;
  if (chunks < 2 || static_cast<size_t>(n) > kTicketCap) return best;
  // Largest need over the tile choices the planner can make for this M.
  for (int mt = tile_for(m); mt >= 1; mt /= 2) {
    const size_t need = workspace_need((m + mt - 1) / mt, mt, n, chunks);
    if (need > best) best = need;
  }
  return best;
}

int klab_cbf16_unpack(const void* payload, const uint32_t* metadata, uint16_t* out, int n, int k, void* stream) {
  if (!payload || !metadata || !out || n <= 0 || k <= 0) return KLAB_E_INVALID;
  return launch_cbf16_unpack(payload, metadata, out, n, k, static_cast<cudaStream_t>(stream));
}

int klab_int8_dequantize(const int8_t* codes, const float* scales, int group, float* out, int n, int k,
                         void* stream) {
  if (!codes || !scales || !out || n <= 0 || k <= 0) return KLAB_E_INVALID;
  if (group != 0 && group != 64) return KLAB_E_UNSUPPORTED;
  if (group == 64 && k % 64) return KLAB_E_SHAPE;
  return launch_int8_dequant(codes, scales, group, out, n, k, static_cast<cudaStream_t>(stream));
}

int klab_add_rmsnorm(const void* res, const void* y, const void* weight, void* x_out, void* xn_out, int m, int d,
                     float eps, void* stream) {
  if (!res || !y || !weight || !x_out || !xn_out || m <= 0 || d <= 0 || !(eps > 0.0f)) return KLAB_E_INVALID;
  if (d % 2 || static_cast<long long>(m) * d >= (1LL << 31)) return KLAB_E_SHAPE;
  return launch_add_rmsnorm(res, y, weight, x_out, xn_out, m, d, eps, static_cast<cudaStream_t>(stream));
}

int klab_silu_mul(const void* gu, void* out, int m, int inter, void* stream) {
  if (!gu || !out || m <= 0 || inter <= 0) return KLAB_E_INVALID;
  if (inter % 2 || static_cast<long long>(m) * inter * 2 >= (1LL << 31)) return KLAB_E_SHAPE;
  return launch_silu_mul(gu, out, m, inter, static_cast<cudaStream_t>(stream));
}

int klab_residual_rmsnorm(const float* x, const float* residual, const float* weight, float* out, int m, int k,
                          float eps, void* stream) {
  if (!x || !residual || !weight || !out || m <= 0 || k <= 0 || !(eps > 0.0f)) return KLAB_E_INVALID;
  if (k > 8192 || static_cast<long long>(m) * k >= (1LL << 31) || m > 0x7fffffff) return KLAB_E_SHAPE;
  return launch_residual_rmsnorm(x, residual, weight, out, m, k, eps, static_cast<cudaStream_t>(stream));
}

int klab_fp4_dequantize(const uint8_t* packed, const void* scales, int scale_kind, const float* gscale, float* out,
                        int n, int k, void* stream) {
  if (!packed || !scales || !out || n <= 0 || k <= 0) return KLAB_E_INVALID;
  if (scale_kind == KLAB_FP4_E4M3_G16) {
    if (!gscale) return KLAB_E_INVALID;
    if (k % 16) return KLAB_E_SHAPE;
  } else if (scale_kind == KLAB_FP4_F16_G32) {
    if (k % 32) return KLAB_E_SHAPE;
  } else {
    return KLAB_E_UNSUPPORTED;
  }
  return launch_fp4_dequant(packed, scales, scale_kind, gscale, out, n, k, static_cast<cudaStream_t>(stream));
}

int klab_l2_prefetch(const void* p, long long bytes, int blocks, int threads, int stride, int kind, unsigned* sink,
                     void* stream) {
  if (!p || bytes < 0 || blocks <= 0 || threads <= 0 || threads > 1024 || stride <= 0) return KLAB_E_INVALID;
  if (kind != KLAB_L2_HINT && kind != KLAB_L2_HINT_LAST && kind != KLAB_L2_LOAD && kind != KLAB_L2_BULK)
    return KLAB_E_UNSUPPORTED;
  if (kind == KLAB_L2_LOAD && !sink) return KLAB_E_INVALID;
  return launch_l2_prefetch(p, bytes, blocks, stride, threads, kind, sink, static_cast<cudaStream_t>(stream));
}

int klab_set_option(int option, int value) {
  switch (option) {
    case KLAB_OPT_PDL: g_opt_pdl.store(value ? 1 : 0); return 0;
    case KLAB_OPT_SPLIT:
      if (value < -1 || value > 1) return KLAB_E_INVALID;
      g_opt_split.store(value);
      return 0;
    case KLAB_OPT_GENERIC: g_opt_generic.store(value ? 1 : 0); return 0;
    case KLAB_OPT_CTAS_PER_SM:
      if (value < 0 || value > 32) return KLAB_E_INVALID;
      g_opt_ctas_per_sm.store(value);
      return 0;
    case KLAB_OPT_TENSOR:
      if (value < 0 || value > 3) return KLAB_E_INVALID;
      g_opt_tensor.store(value);
      return 0;
    case KLAB_OPT_PROLOGUE:
      if (value != -1 && (value < 0 || (value & 15) > 3 || (value >> 4) > 3)) return KLAB_E_INVALID;
      g_opt_prologue.store(value);
      return 0;
    case KLAB_OPT_MAX_TILE:
      if (value != 1 && value != 2 && value != 4 && value != 8) return KLAB_E_INVALID;
      g_opt_max_tile.store(value);
      return 0;
    default: return KLAB_E_INVALID;
  }
}

int klab_get_option(int option) {
  switch (option) {
    case KLAB_OPT_PDL: return g_opt_pdl.load();
    case KLAB_OPT_SPLIT: return g_opt_split.load();
    case KLAB_OPT_TENSOR: return g_opt_tensor.load();
    case KLAB_OPT_GENERIC: return g_opt_generic.load();
    case KLAB_OPT_CTAS_PER_SM: return g_opt_ctas_per_sm.load();
    case KLAB_OPT_PROLOGUE: return g_opt_prologue.load();
    case KLAB_OPT_MAX_TILE: return g_opt_max_tile.load();
    default: return KLAB_E_INVALID;
  }
}

int klab_device_status(int clear) {
  DeviceInfo* info = nullptr;
  int rc = current_device_info(&info);
  if (rc) return rc;
  int value = 0;
  cudaError_t err = cudaMemcpy(&value, info->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return err;
  if (clear && value) {
    const int zero = 0;
    err = cudaMemcpy(info->status, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (err != cudaSuccess) return err;
  }
  return value;
}

const char* klab_error_string(int code) {
  switch (code) {
    case 0: return "success";
    case KLAB_E_DRIVER: return "Cannot load CUDA driver or required symbols";
    case KLAB_E_NO_CONTEXT: return "No current CUDA context; initialize PyTorch CUDA first";
    case KLAB_E_INVALID: return "Invalid null argument or launch dimensions";
    case KLAB_E_SHAPE: return "Shape not supported by this weight format";
    case KLAB_E_ALIGN: return "Pointer or stride alignment not supported";
    case KLAB_E_UNSUPPORTED: return "Unsupported dtype or format combination";
    case KLAB_E_DEVICE: return "A kernel recorded a device-side error (bounded wait expired)";
    case KLAB_E_SCRATCH: return "Shape needs more split-K scratch than the library's static 4 MiB array";
    default:
      if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
      return "Unknown klab error";
  }
}

int klab_version(void) { return 1; }

}  // extern "C"
