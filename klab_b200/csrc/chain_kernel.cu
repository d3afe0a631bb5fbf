// Persistent projection chain: one launch runs every projection of a token step.
//
// The chain (BF16 weights, one token) is a list of stages; stage s > 0 reads the
// gathered output of stage s-1. One CTA per SM (cooperative launch), 16 warps,
// each with a private ring of kChainDepth bulk-copy slots (one slot = one row x
// 4 KiB chunk of weights = one "item").
//
// Work: every CTA takes an equal share of a stage's rows in at most two
// contiguous parts (the gathered segment first when a stage lists it first with
// other rows, so it is produced first everywhere), and a CTA's items (its rows x
// S chunks) go to its warps as contiguous runs of equal length (no atomics
// across CTAs). A warp's lane 0 issues its next item as soon
// as a slot is consumed, running on into the next stage's run, so the weight
// stream of stage s+1 is in flight while the stage-s data dependency is still
// being resolved (weights never depend on activations). Rows inside one run are
// folded in registers. A row cut by a warp-run boundary lies inside one CTA: its
// contributors put their chunk partials in a shared-memory slot and add their
// chunk count to the slot's counter; the one that completes the count folds the
// partials in chunk order at once and clears the counter. No warp waits on
// another CTA except through the gathered inputs, which are the true data
// dependencies.
//
// Data exchange: the outputs that later stages read (the gathered segment of a
// stage) are written as 32-bit words (tag << 16 | bf16) into every rank's copy
// of the gather buffer, over NVLink for the peers; the tag identifies the step
// and stage. A CTA stages x for stage s by polling those words until every one
// carries stage s-1's tag (bounded by time). No grid barrier, no counters and no
// system-scope fence sit between stages: each 32-bit store is single-copy
// atomic, so a word with the right tag holds the right value. A CTA that holds
// no unit of a stage skips staging that stage's x (it may already be
// overwritten by later stages, whose producers only wait for CTAs that hold
// units).
//
// Arithmetic order is the one of stream_gemv_kernel (a function of K only):
// chunk partials by the same per-lane tree and warp butterfly, row total folded
// over chunks in order, one RNE to BF16.
// The chain's outputs are therefore bit-identical to one launch per stage.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "klab_kernels.h"
#include "stream_gemv.cuh"

namespace klab {
namespace {

#ifndef KLAB_CHAIN_WARPS
#define KLAB_CHAIN_WARPS 16
#endif
#ifndef KLAB_CHAIN_DEPTH
#define KLAB_CHAIN_DEPTH 3
#endif
constexpr int kChainWarps = KLAB_CHAIN_WARPS;  // warps per CTA
constexpr int kChainDepth = KLAB_CHAIN_DEPTH;  // ring slots per warp
constexpr int kChainKC = Layout<W_BF16>::KC;  // 2048 columns per item
constexpr int kChainSlot = kWeightSlot;       // 4096 bytes per item
constexpr int kChainMaxK = 16384;             // x staging capacity (BF16 values)
constexpr int kChainMaxS = kChainMaxK / kChainKC;
constexpr int kChainBarBytes = 512;           // mbarriers
constexpr int kChainSmem = kChainBarBytes + kChainWarps * kChainDepth * kChainSlot + kChainMaxK * 2;
constexpr int kChainMaxStages = 4096;
constexpr unsigned long long kChainWaitNs = 2000000000ull;  // polling limit per stage (2 s)

struct ChainSeg {
  const char* w;  // BF16 [rows, k]
  void* out;      // BF16 outputs (plain segments)
  int row0;       // first stage row of this segment
  int pad;
};

struct ChainStage {
  const void* x;         // plain BF16 [k] (x_stage < 0) or tagged words [k]
  int k, chunks, n, nseg;
  int gather_seg;        // segment written as tagged words to every rank (-1: none)
  int x_stage;           // stage whose gathered output x is (-1: plain input)
  ChainSeg seg[kMaxSegs];
  unsigned* peer_out[kMaxPeers];  // rank q's tagged buffer, at gather_seg's first row
};

struct ChainParams {
  const ChainStage* stages;
  int nstages;
  int npeers, rank;
  unsigned* epoch;                 // completed steps (this rank)
  unsigned* exits;                 // CTAs finished with the step, zero between steps
  int* status;
  const unsigned* final_in;        // tagged output of stage final_stage
  unsigned short* final_out;       // its BF16 values
  int final_n;
  int final_stage;
  unsigned long long* trace;       // optional: [nstages][grid][kTraceSlots] global-timer ns
};

// Trace slots per (stage, CTA): entered, every warp done with the previous
// stage, x staged, then per warp: its first item of the stage landed, its run
// computed, and done.
constexpr int kTraceCta = 3;
constexpr int kTraceWarp = 3;
constexpr int kTraceSlots = kTraceCta + kTraceWarp * kChainWarps;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void trace_mark(const ChainParams& p, int s, int slot) {
  if (p.trace) p.trace[(static_cast<long long>(s) * gridDim.x + blockIdx.x) * kTraceSlots + slot] = global_ns();
}

__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Tag of stage s's outputs in step `epoch` (never 0, the value of a fresh buffer).
__device__ __forceinline__ unsigned stage_tag(unsigned epoch, int nstages, int s) {
  return 1u + (epoch * static_cast<unsigned>(nstages) + static_cast<unsigned>(s)) % 65535u;
}

__device__ __forceinline__ int seg_of(const ChainStage& st, int row) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < kMaxSegs; ++i)
    if (i < st.nseg && row >= st.seg[i].row0) s = i;
  return s;
}

// Rows of segment i of a stage.
__device__ __forceinline__ int seg_rows(const ChainStage& st, int i) {
  return (i + 1 < st.nseg ? st.seg[i + 1].row0 : st.n) - st.seg[i].row0;
}

// CTA b's share of a stage, in two contiguous parts so that a CTA touches few weight pages
// (a warp's first access to a page whose translation is not cached stalls it ~1 us): part 1
// is the gathered segment when it is segment 0 of a stage with other segments (CTA b takes
// rows [n1 b / G, n1 (b + 1) / G) of it first, so those rows are produced first everywhere),
// part 2 the stage's other rows (rows [n1 + n2 b / G, n1 + n2 (b + 1) / G)). "Local rows"
// number the share in that order.
__device__ __forceinline__ int first_part_rows(const ChainStage& st) {
  return (st.gather_seg == 0 && st.nseg > 1) ? seg_rows(st, 0) : 0;
}

// 32-bit arithmetic throughout: rows x CTAs and items x 16 stay below 2^31 (checked at plan
// creation), and these run on the issue path of every row.
__device__ __forceinline__ int share_rows(const ChainStage& st, unsigned b, unsigned G) {
  const unsigned n1 = static_cast<unsigned>(first_part_rows(st)), n2 = static_cast<unsigned>(st.n) - n1;
  return static_cast<int>(n1 * (b + 1) / G - n1 * b / G + n2 * (b + 1) / G - n2 * b / G);
}

// CTA b's share as (first part: rows lo1 .. lo1 + c1 - 1; then rows from base2), computed once
// per stage; row(lr) is the stage row of local row lr.
struct Share {
  int lo1, c1, base2;
  __device__ __forceinline__ void set(const ChainStage& st, unsigned b, unsigned G) {
    const unsigned n1 = static_cast<unsigned>(first_part_rows(st)), n2 = static_cast<unsigned>(st.n) - n1;
    lo1 = static_cast<int>(n1 * b / G);
    c1 = static_cast<int>(n1 * (b + 1) / G) - lo1;
    base2 = static_cast<int>(n1 + n2 * b / G);
  }
  __device__ __forceinline__ int row(int lr) const { return lr < c1 ? lo1 + lr : base2 + (lr - c1); }
};

// This warp's contiguous run [begin, end) of its CTA's local items (local row x S + chunk).
__device__ __forceinline__ void warp_range(const ChainStage& st, unsigned gw, unsigned nw, long long* begin,
                                           long long* end) {
  const unsigned T = static_cast<unsigned>(share_rows(st, gw / kChainWarps, nw / kChainWarps) * st.chunks);
  const unsigned w = gw % kChainWarps;
  *begin = T * w / kChainWarps;
  *end = T * (w + 1) / kChainWarps;
}

// Shared-memory slot of a row cut by warp-run boundaries: the first warp whose run begins
// inside the row (local item index L of its first chunk, T items in the CTA), in 1..15.
// Distinct cut rows have distinct first boundaries.
__device__ __forceinline__ int cut_slot(long long L, long long T) {
  const unsigned l = static_cast<unsigned>(L), t = static_cast<unsigned>(T);
  return static_cast<int>((kChainWarps * (l + 1) + t - 1) / t);
}

// Issue side of one warp's item sequence over all stages (lane 0 only).
struct IssueCursor {
  int stage, lr, c, row;  // local row, chunk, and the local row's stage row
  Share share;            // this CTA's share of `stage`
  long long left;         // items left in this stage's run
  __device__ __forceinline__ void enter(const ChainParams& p, unsigned gw, unsigned nw, int s) {
    for (stage = s; stage < p.nstages; ++stage) {
      long long b, e;
      warp_range(p.stages[stage], gw, nw, &b, &e);
      if (e > b) {
        const int S = p.stages[stage].chunks;
        lr = static_cast<int>(b / S);
        c = static_cast<int>(b - static_cast<long long>(lr) * S);
        share.set(p.stages[stage], gw / kChainWarps, nw / kChainWarps);
        row = share.row(lr);
        left = e - b;
        return;
      }
    }
  }
  __device__ __forceinline__ bool valid(const ChainParams& p) const { return stage < p.nstages; }
  // Issue the current item into `slot`, then advance.
  __device__ __forceinline__ void issue(const ChainParams& p, unsigned gw, unsigned nw, unsigned slot,
                                        unsigned bar) {
    const ChainStage& st = p.stages[stage];
    const int s = seg_of(st, row);
    const int L = min(kChainKC, st.k - c * kChainKC);
    const char* src = st.seg[s].w + (static_cast<long long>(row - st.seg[s].row0) * st.k + c * kChainKC) * 2;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, L * 2);
    bulk_g2s(slot, src, L * 2, bar);
    if (--left == 0) {
      enter(p, gw, nw, stage + 1);
    } else if (++c == st.chunks) {
      c = 0;
      row = share.row(++lr);
    }
  }
};

__device__ __forceinline__ void chain_finalize(const ChainParams& p, const ChainStage& st, int row, float v,
                                               unsigned tag) {
  const int s = seg_of(st, row);
  const int local = row - st.seg[s].row0;
  const unsigned short b = f32_to_bf16_rn(v);
  if (s == st.gather_seg) {
    const unsigned word = (tag << 16) | b;
    for (int q = 0; q < p.npeers; ++q) st_relaxed_sys(st.peer_out[q] + local, word);
  } else {
    static_cast<unsigned short*>(st.seg[s].out)[local] = b;
  }
}

// Stage x into shared memory as BF16 (natural order, zero-padded to whole
// 256-column segments). Tagged inputs are polled until every word carries
// `tag`; returns false when the time limit passed first.
__device__ bool stage_chain_x(const ChainStage& st, bool tagged, unsigned tag, unsigned char* xs, int* broken) {
  const int k = st.k;
  const int segs = (k + 255) / 256;
  bool ok = true;
  if (!tagged) {
    const uint4* src = static_cast<const uint4*>(st.x);
    for (int u = threadIdx.x; u < segs * 32; u += blockDim.x) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (u * 8 < k) v = __ldcg(src + u);
      reinterpret_cast<uint4*>(xs)[u] = v;
    }
    return true;
  }
  // Four tagged words (16 bytes) -> four BF16 values (8 bytes) per vector.
  // All of a thread's vectors are loaded at once; only stale ones are re-read.
  const char* src = static_cast<const char*>(st.x);
  constexpr int kPer = (kChainMaxK / 4 + kChainWarps * 32 - 1) / (kChainWarps * 32);  // vectors per thread
  const int nvec = segs * 64;
  uint4 v[kPer];
  bool fresh[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int u = threadIdx.x + j * blockDim.x;
    fresh[j] = true;
    v[j] = make_uint4(0u, 0u, 0u, 0u);
    if (u < nvec && u * 4 < k) v[j] = ld_volatile_v4(src + 16ll * u);
  }
  const unsigned long long t0 = global_ns();
  for (;;) {
    bool all = true;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int u = threadIdx.x + j * blockDim.x;
      if (u < nvec && u * 4 < k) {
        fresh[j] = (v[j].x >> 16) == tag && (v[j].y >> 16) == tag && (v[j].z >> 16) == tag && (v[j].w >> 16) == tag;
        all = all && fresh[j];
      }
    }
    if (all) break;
    if (*reinterpret_cast<volatile int*>(broken) || global_ns() - t0 > kChainWaitNs) {
      ok = false;
      *reinterpret_cast<volatile int*>(broken) = 1;
      break;
    }
    __nanosleep(32);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int u = threadIdx.x + j * blockDim.x;
      if (!fresh[j]) v[j] = ld_volatile_v4(src + 16ll * u);
    }
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int u = threadIdx.x + j * blockDim.x;
    if (u < nvec)
      reinterpret_cast<uint2*>(xs)[u] =
          make_uint2((v[j].x & 0xffffu) | (v[j].y << 16), (v[j].z & 0xffffu) | (v[j].w << 16));
  }
  return ok;
}

__global__ void __launch_bounds__(kChainWarps * 32, 1) chain_kernel(const ChainParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_broken;
  __shared__ float s_part[kChainWarps][kChainMaxS];   // cut rows' chunk partials, by slot
  __shared__ int s_count[kChainWarps];                 // chunks stored per slot (0 between stages)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned gw = blockIdx.x * kChainWarps + warp, nw = gridDim.x * kChainWarps;
  const unsigned pbar0 = smem_addr(smem) + warp * kChainDepth * 8;
  const unsigned slot0 = smem_addr(smem) + kChainBarBytes + warp * kChainDepth * kChainSlot;
  unsigned char* xs = smem + kChainBarBytes + kChainWarps * kChainDepth * kChainSlot;
  const unsigned xs_lane0 = smem_addr(xs) + lane * 16;
  if (threadIdx.x == 0) s_broken = 0;
  if (threadIdx.x < kChainWarps) s_count[threadIdx.x] = 0;

  // Ring prologue: the first kChainDepth items of this warp's sequence.
  IssueCursor iss{};
  long long issued = 0;  // lane 0: items issued so far
  if (lane == 0) {
    for (int i = 0; i < kChainDepth; ++i) mbar_init(pbar0 + 8 * i, 1);
    fence_mbar_init();
    iss.enter(p, gw, nw, 0);
    for (int i = 0; i < kChainDepth && iss.valid(p); ++i) {
      iss.issue(p, gw, nw, slot0 + i * kChainSlot, pbar0 + i * 8);
      ++issued;
    }
  }
  __syncwarp();

  const unsigned epoch = *p.epoch + 1u;  // this step
  const void* staged_x = nullptr;        // input now in xs (the same in every thread)
  int staged_from = -2;
  bool ok = true;
  long long g = 0;        // ring position of the next item to consume
  long long failed = -1;  // ring position of a copy that never completed

  for (int s = 0; s < p.nstages; ++s) {
    const ChainStage& st = p.stages[s];
    const int S = st.chunks, k = st.k;
    long long wbegin, wend;
    warp_range(st, gw, nw, &wbegin, &wend);
    const int nitems = static_cast<int>(wend - wbegin);
    if (threadIdx.x == 0) trace_mark(p, s, 0);
    // Barrier (every warp is done with the previous x); stage x if any warp
    // of this CTA has items in this stage.
    const bool need = __syncthreads_or(nitems > 0 ? 1 : 0);
    if (threadIdx.x == 0) trace_mark(p, s, 1);
    // Stage x unless this CTA holds no item of the stage or x is already there
    // (the same input as the previous staging).
    if (need && (st.x != staged_x || st.x_stage != staged_from)) {
      const bool tagged = st.x_stage >= 0;
      if (!stage_chain_x(st, tagged, tagged ? stage_tag(epoch, p.nstages, st.x_stage) : 0u, xs, &s_broken))
        record_status(p.status, kStatusFlagTimeout);
      staged_x = st.x;
      staged_from = st.x_stage;
      __syncthreads();
    }
    if (threadIdx.x == 0) trace_mark(p, s, 2);
    const unsigned tag = stage_tag(epoch, p.nstages, s);

    int lr = 0, c = 0, row = 0;   // local row, chunk, stage row
    if (nitems > 0) {
      lr = static_cast<int>(wbegin / S);
      c = static_cast<int>(wbegin - static_cast<long long>(lr) * S);
    }
    const long long cta_items = static_cast<long long>(share_rows(st, blockIdx.x, gridDim.x)) * S;
    Share share;
    share.set(st, blockIdx.x, gridDim.x);
    float rowsum = 0.0f;
    bool whole = true;
    int cut = 0, mine = 0;  // a cut row: its shared-memory slot, chunks this warp stored
    for (int q = 0; q < nitems; ++q, ++g) {
      const int L = min(kChainKC, k - c * kChainKC);
      const unsigned slot = slot0 + static_cast<unsigned>(g % kChainDepth) * kChainSlot;
      const unsigned bar = pbar0 + static_cast<unsigned>(g % kChainDepth) * 8;
      float P[1] = {0.0f};
      if (ok) {
        const bool landed = mbar_wait(bar, static_cast<unsigned>((g / kChainDepth) & 1));
        ok = __all_sync(0xffffffffu, landed);
        if (!ok) failed = g;
        if (q == 0 && lane == 0) trace_mark(p, s, kTraceCta + kTraceWarp * warp);
      }
      if (ok) {
        const unsigned xs_lane = xs_lane0 + c * kSegs * 512;
        if (L == kChainKC)
          compute_item<W_BF16, X_BF16, XM_SMEM16, 1, true>(slot, 0, 0, lane, L, xs_lane, 0, nullptr, 0, 1, P);
        else
          compute_item<W_BF16, X_BF16, XM_SMEM16, 1, false>(slot, 0, 0, lane, L, xs_lane, 0, nullptr, 0, 1, P);
        __syncwarp();  // every lane is done with the slot before it is refilled
        if (lane == 0 && iss.valid(p)) {
          iss.issue(p, gw, nw, slot, bar);
          ++issued;
        }
      }
      if (c == 0 || q == 0) {
        row = share.row(lr);
        whole = static_cast<long long>(lr) * S >= wbegin && static_cast<long long>(lr) * S + S <= wend;
        if (!whole) {
          cut = cut_slot(static_cast<long long>(lr) * S, cta_items);
          mine = 0;
        }
      }
      if (whole) {
        rowsum = (c == 0) ? P[0] : add_rn(rowsum, P[0]);
        if (c == S - 1 && lane == 0) chain_finalize(p, st, row, rowsum, tag);
      } else {
        ++mine;
        if (lane == 0) {
          s_part[cut][c] = P[0];
          if (c == S - 1 || q == nitems - 1) {   // this warp's last chunk of the row
            __threadfence_block();
            if (atomicAdd(&s_count[cut], mine) + mine == S) {   // every chunk is in: fold in chunk order
              __threadfence_block();
              const volatile float* part = s_part[cut];
              float total = part[0];
              for (int cc = 1; cc < S; ++cc) total = add_rn(total, part[cc]);
              chain_finalize(p, st, row, total, tag);
              s_count[cut] = 0;
            }
          }
        }
      }
      if (++c == S) {
        c = 0;
        ++lr;
      }
    }
    if (lane == 0) trace_mark(p, s, kTraceCta + kTraceWarp * warp + 1);
    if (lane == 0) trace_mark(p, s, kTraceCta + kTraceWarp * warp + 2);
  }

  // CTA 0 publishes the step's output once every rank's last-stage words are in.
  if (blockIdx.x == 0) {
    const unsigned tag = stage_tag(epoch, p.nstages, p.final_stage);
    const unsigned long long t0 = global_ns();
    for (int j = threadIdx.x; j < p.final_n; j += blockDim.x) {
      unsigned v = 0;
      for (;;) {
        asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p.final_in + j) : "memory");
        if ((v >> 16) == tag) break;
        if (*reinterpret_cast<volatile int*>(&s_broken) || global_ns() - t0 > kChainWaitNs) {
          *reinterpret_cast<volatile int*>(&s_broken) = 1;
          record_status(p.status, kStatusFlagTimeout);
          break;
        }
        __nanosleep(32);
      }
      p.final_out[j] = static_cast<unsigned short>(v & 0xffffu);
    }
  }

  if (!ok) {
    record_status(p.status, kStatusMbarTimeout);
    // Drain copies still in flight (bounded) before shared memory is released.
    if (lane == 0)
      for (long long i = failed; i < issued; ++i)
        mbar_wait(pbar0 + static_cast<unsigned>(i % kChainDepth) * 8, static_cast<unsigned>((i / kChainDepth) & 1));
  }

  // The last CTA to finish advances the step (every CTA read it at its start).
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(p.exits, 1u) == gridDim.x - 1) {
    *p.exits = 0u;
    *p.epoch = epoch;
  }
}

struct ChainPlan {
  ChainParams params{};
  ChainStage* d_stages = nullptr;
  void* d_ws = nullptr;
  int grid = 0;
};

}  // namespace
}  // namespace klab

using klab::ChainPlan;

extern "C" {

KLAB_API int klab_chain_create(const klab_chain_stage_t* stages, int nstages, const klab_chain_sync_t* sync,
                               void** plan_out) {
  using namespace klab;
  if (!stages || !sync || !plan_out || nstages <= 0 || nstages > kChainMaxStages) return KLAB_E_INVALID;
  if (sync->npeers < 1 || sync->npeers > kMaxPeers || sync->rank < 0 || sync->rank >= sync->npeers ||
      !sync->epoch || !sync->final_out)
    return KLAB_E_INVALID;
  if (!sync->final_in || (reinterpret_cast<uintptr_t>(sync->final_in) & 3)) return KLAB_E_INVALID;
  std::vector<ChainStage> host(nstages);
  for (int s = 0; s < nstages; ++s) {
    const klab_chain_stage_t& in = stages[s];
    ChainStage& st = host[s];
    std::memset(&st, 0, sizeof(st));
    if (!in.x || in.k <= 0 || in.k > kChainMaxK || in.k % 8 || in.nseg < 1 || in.nseg > kMaxSegs)
      return KLAB_E_SHAPE;
    if (reinterpret_cast<uintptr_t>(in.x) & 15) return KLAB_E_ALIGN;
    if (in.gather_seg < -1 || in.gather_seg >= in.nseg) return KLAB_E_INVALID;
    // x is the plain step input or the gathered output of an earlier stage.
    if (in.x_stage >= s || in.x_stage < -1) return KLAB_E_INVALID;
    if (in.x_stage >= 0) {
      const klab_chain_stage_t& src = stages[in.x_stage];
      if (src.gather_seg < 0) return KLAB_E_INVALID;
      if (in.k != src.n[src.gather_seg] * sync->npeers) return KLAB_E_SHAPE;
    }
    st.x = in.x;
    st.x_stage = in.x_stage;
    st.k = in.k;
    st.chunks = (in.k + kChainKC - 1) / kChainKC;
    st.nseg = in.nseg;
    st.gather_seg = in.gather_seg;
    int rows = 0;
    for (int i = 0; i < in.nseg; ++i) {
      if (!in.w[i] || in.n[i] <= 0 || (i != in.gather_seg && !in.out[i])) return KLAB_E_INVALID;
      if (reinterpret_cast<uintptr_t>(in.w[i]) & 15) return KLAB_E_ALIGN;
      st.seg[i].w = static_cast<const char*>(in.w[i]);
      st.seg[i].out = in.out[i];
      st.seg[i].row0 = rows;
      rows += in.n[i];
    }
    for (int q = 0; q < sync->npeers && in.gather_seg >= 0; ++q) {
      if (!in.peer_out[q] || (reinterpret_cast<uintptr_t>(in.peer_out[q]) & 3)) return KLAB_E_INVALID;
      st.peer_out[q] = static_cast<unsigned*>(in.peer_out[q]);
    }
    st.n = rows;
  }

  int dev = 0, sms = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kChainSmem);
  if (err != cudaSuccess) return err;
  int per_sm = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain_kernel, kChainWarps * 32, kChainSmem);
  if (err != cudaSuccess) return err;
  if (per_sm < 1) return KLAB_E_UNSUPPORTED;
  // Every CTA holds rows of every stage (its share of each segment, share_rows),
  // so no CTA can still be reading a gather buffer when a later stage rewrites it
  // (the rewriting stage's input is only complete once every CTA has passed the
  // reading stages).
  int final_stage = -1;
  for (int s = 0; s < nstages; ++s) {
    if (static_cast<long long>(host[s].n) * sms >= (1LL << 31) ||
        static_cast<long long>(host[s].n) * host[s].chunks * kChainWarps >= (1LL << 31))
      return KLAB_E_SHAPE;   // the kernel's 32-bit share arithmetic
    const long long n1 = (host[s].gather_seg == 0 && host[s].nseg > 1) ? host[s].seg[1].row0 : 0;
    const long long n2 = host[s].n - n1;
    for (int b = 0; b < sms; ++b)
      if (n1 * (b + 1) / sms - n1 * b / sms + n2 * (b + 1) / sms - n2 * b / sms < 1) return KLAB_E_SHAPE;
    if (host[s].gather_seg >= 0) final_stage = s;
  }
  if (final_stage < 0) return KLAB_E_INVALID;

  ChainPlan* plan = new ChainPlan();
  plan->grid = sms;
  const size_t stage_bytes = sizeof(ChainStage) * nstages;
  // The CTA exit count (zero between steps).
  const size_t total = 256;
  err = cudaMalloc(reinterpret_cast<void**>(&plan->d_stages), stage_bytes);
  if (err == cudaSuccess) err = cudaMemcpy(plan->d_stages, host.data(), stage_bytes, cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = cudaMalloc(&plan->d_ws, total);
  if (err == cudaSuccess) err = cudaMemset(plan->d_ws, 0, total);
  if (err != cudaSuccess) {
    cudaFree(plan->d_stages);
    cudaFree(plan->d_ws);
    delete plan;
    return err;
  }
  ChainParams& p = plan->params;
  char* base = static_cast<char*>(plan->d_ws);
  p.stages = plan->d_stages;
  p.nstages = nstages;
  p.npeers = sync->npeers;
  p.rank = sync->rank;
  p.epoch = sync->epoch;
  p.exits = reinterpret_cast<unsigned*>(base);
  p.status = device_status_address();
  p.final_in = sync->final_in;
  p.final_out = static_cast<unsigned short*>(sync->final_out);
  p.final_stage = final_stage;
  p.final_n = stages[final_stage].n[stages[final_stage].gather_seg] * sync->npeers;
  *plan_out = plan;
  return 0;
}

KLAB_API int klab_chain_info(void* plan_ptr, int* grid, int* trace_slots) {
  using namespace klab;
  ChainPlan* plan = static_cast<ChainPlan*>(plan_ptr);
  if (!plan) return KLAB_E_INVALID;
  if (grid) *grid = plan->grid;
  if (trace_slots) *trace_slots = kTraceSlots;
  return 0;
}

KLAB_API int klab_chain_trace(void* plan_ptr, unsigned long long* buffer, size_t bytes) {
  using namespace klab;
  ChainPlan* plan = static_cast<ChainPlan*>(plan_ptr);
  if (!plan) return KLAB_E_INVALID;
  if (buffer && bytes < static_cast<size_t>(plan->params.nstages) * plan->grid * kTraceSlots * 8)
    return KLAB_E_SHAPE;
  plan->params.trace = buffer;
  return 0;
}

KLAB_API int klab_chain_launch(void* plan_ptr, void* stream) {
  using namespace klab;
  ChainPlan* plan = static_cast<ChainPlan*>(plan_ptr);
  if (!plan) return KLAB_E_INVALID;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  cfg.blockDim = dim3(kChainWarps * 32);
  cfg.dynamicSmemBytes = kChainSmem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, chain_kernel, plan->params);
}

KLAB_API int klab_chain_destroy(void* plan_ptr) {
  ChainPlan* plan = static_cast<ChainPlan*>(plan_ptr);
  if (!plan) return KLAB_E_INVALID;
  cudaFree(plan->d_stages);
  cudaFree(plan->d_ws);
  delete plan;
  return 0;
}

}  // extern "C"
