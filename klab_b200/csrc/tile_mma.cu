// Token tiles of INT8 per-row and E2M1 (FP16 scale per 32) weights on the warp-level
// tensor cores: y[M, N] = x[M, K] . W[N, K]^T for M = 1..16, BF16 or FP16 x.
//
// The CUDA-core projection spends one FMA per weight and token plus the weight decode;
// here a warp multiplies a 16-row group of weights with up to 16 tokens per mma.sync,
// so the weight bytes are read and decoded once per tile and the math is a few tensor
// instructions per 512 weights. On B200, mma.sync issues at most one m16n8k16 per 8
// cycles per SM sub-partition with a 20-cycle latency (measured): the MMA rate covers
// the weight stream up to M = 16, but with two warps per scheduler this kernel is
// bound by dependency latency and by x staging and the fold around the stream.
//
// Operands are FP16 with FP32 accumulation on mma.m16n8k16 for both formats:
//   x of token t in a K phase is staged in FP16: BF16 x is scaled by 2^s, s from the
//   phase's largest exponent (exact when the phase's nonzero values span at most 32
//   binades; smaller values are rounded to FP16's subnormal grid, below 2^-39 of the
//   phase's largest); FP16 x is taken as is. The scaling is undone on the phase total.
// INT8 per row (benchmark config 2): the codes are exact in FP16 (1024 + code + 128,
//   minus 1152). A unit's 32-K steps chain in four FP32 accumulators (two per step
//   parity) that are added in a fixed order at the end of the unit; phases are added in
//   K order, then one multiply by the row's scale and one rounding to the output type.
// E2M1 with an FP16 scale per 32 K (benchmark config 3): codes become FP16 with
//   cvt.rn.f16x2.e2m1x2. Each 32-K group is two mma.m16n8k16 into FP32 (the tensor
//   core's order), scaled by the group's FP16 scale with one fma.rn; a unit's groups
//   chain in K order, phases are added in K order.
//
// Work: K is cut into phases (INT8 1024, E2M1 2048 columns) and N into 16-row groups; a
// unit is (row group, phase), 16 rows x 1 KiB of weights, streamed as two items of 16
// rows x 512 bytes through the ring of the warp that owns the unit: one 1-D bulk copy
// (cp.async.bulk, this CTA only) per row into rows of 528 bytes, so ldmatrix reads are
// conflict-free. Each CTA (one per SM) takes an equal run of units in row-group order.
// It stages x for a window of phases (as many as fit in 64 KiB), deals the window's units
// round-robin to its warps, and each warp accumulates a unit in registers and writes its
// phase partial to the workspace. After its run the CTA adds each of its row groups'
// phase partials in phase order; a row group whose phases are split between two CTAs
// (only the ends of a run) is added by the CTA that completes its ticket, in the same
// order. The arithmetic depends only on K: results do not change with M, the row shard,
// the grid or the partition.
//
// Fragment layout (PTX ISA, mma.m16n8k16): thread (g = lane / 4, c = lane % 4) holds A
// rows g and g + 8 and B column (token) g. The K slots a thread owns are free to map to
// any K columns as long as A and B agree. INT8 maps thread c's slots of a 32-K step to
// columns 4c..4c+3 (first MMA) and 16+4c..16+4c+3 (second MMA); E2M1 maps them to
// columns 8c..8c+7 of the group: in both cases the bytes ldmatrix hands the thread.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "klab_kernels.h"

namespace klab {

namespace {

constexpr int kTmWarps = 8;
constexpr int kTmThreads = 32 * kTmWarps;
constexpr int kTmRows = 16;                      // rows per group (MMA M)
constexpr int kTmRowBytes = 512;                 // weight bytes per row per item
constexpr int kTmPitch = kTmRowBytes + 16;       // shared-memory row pitch (ldmatrix conflict-free)
constexpr int kTmItem = kTmRows * kTmPitch;      // 8448 bytes
constexpr int kTmScaleRow = 64;                  // E2M1: 32 FP16 scales per row and item
constexpr int kTmScaleItem = kTmRows * kTmScaleRow;
constexpr int kTmXMax = 64 * 1024;               // x staging of a window of phases (FP16)
constexpr int kTmUpt = kTmXMax / (kTmThreads * 16);   // 16-byte x chunks per thread and window
constexpr int kTmKsI8 = 1024, kTmKsF4 = 2048;    // K columns per phase (1 KiB of weights per row)
constexpr int kTmBoxes = 2;                      // items per unit
constexpr int kTmMaxWin = 32;                    // phases per window at most
constexpr int kTmDepth = 2;                      // items in flight per warp
constexpr int kTmEarly = 1;                      // items a warp issues before x is staged

enum TmKind : int { TM_I8_ROW = 0, TM_FP4_G32H = 1 };

struct alignas(64) TmParams {
  const unsigned char* w;   // W bytes [N, row_bytes]
  const unsigned char* s;   // E2M1: FP16 scales [N, K / 32]
  long long row_bytes;
  const void* x;
  const float* row_scale;   // INT8: [N]
  void* out;
  float* part;              // phase partials [group][phase][M][16]
  unsigned* tickets;        // [group]: row groups split between CTAs
  int* status;
  int ldx, ldo, out_f32, x_f16;
  int m, n, k, phases;
  int window;               // phases staged at once
  int units, per_cta, extra;   // units = groups * phases; CTA b runs per_cta (+1 if b < extra)
  int div_m;                // ceil(2^16 / m): chunk index -> (group, token) without a divide
};

template <int KIND>
struct TmLayout {
  static constexpr int W = kTmWarps * kTmDepth * kTmItem;
  static constexpr int S = KIND == TM_FP4_G32H ? kTmWarps * kTmDepth * kTmScaleItem : 0;
  static constexpr int X = kTmXMax;
  static constexpr int BARS = kTmWarps * kTmDepth * 8;
  static constexpr int TOTAL = W + S + X + BARS + kTmMaxWin * 16 * 4 + 16 + 128;   // + exponents, flags, align
};

// ------------------------------------------------------------------ device helpers

__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// D = A . B + C in FP32, A and B FP16 (A [16 x 16], B [16 x 8]).
__device__ __forceinline__ void mma_f16(float (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3,
                                        unsigned b0, unsigned b1, const float (&c)[4]) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%10, %11, %12, %13};"
               : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
                 "f"(c[3]));
}

// Four INT8 codes -> two FP16x2 words (bytes 0, 1 and bytes 2, 3), exact: the FP16 bit
// pattern 0x6400 | (code + 128) is 1024 + code + 128.
__device__ __forceinline__ void i8x4_to_f16x4(unsigned w, unsigned& lo, unsigned& hi) {
  const unsigned b = w ^ 0x80808080u;
  const unsigned bias = 0x64806480u;   // FP16 1152 in both halves
  const unsigned l = __byte_perm(b, 0x64646464u, 0x4140), h = __byte_perm(b, 0x64646464u, 0x4342);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(l), "r"(bias));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(h), "r"(bias));
}

// Predicated loads through L2 (zero where !valid). Written as one PTX block each so that a
// run of them issues back to back: the stage and the fold wait one round trip, not one per load.
__device__ __forceinline__ void ldcg_v4_pred(const void* src, bool valid, unsigned (&w)[4]) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.b32 q, %5, 0;\n mov.b32 %0, 0;\n mov.b32 %1, 0;\n mov.b32 %2, 0;\n"
      " mov.b32 %3, 0;\n @q ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];\n}\n"
      : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
      : "l"(src), "r"(static_cast<int>(valid)));
}
__device__ __forceinline__ void ldcg_v2_pred(const void* src, bool valid, unsigned& w0, unsigned& w1) {
  asm volatile("{\n .reg .pred q;\n setp.ne.b32 q, %3, 0;\n mov.b32 %0, 0;\n mov.b32 %1, 0;\n"
               " @q ld.global.cg.v2.u32 {%0, %1}, [%2];\n}\n"
               : "=r"(w0), "=r"(w1)
               : "l"(src), "r"(static_cast<int>(valid)));
}
__device__ __forceinline__ unsigned ldcg_u16_pred(const void* src, bool valid) {
  unsigned short h;
  asm volatile("{\n .reg .pred q;\n setp.ne.b32 q, %2, 0;\n mov.b16 %0, 0;\n @q ld.global.cg.u16 %0, [%1];\n}\n"
               : "=h"(h)
               : "l"(src), "r"(static_cast<int>(valid)));
  return h;
}
__device__ __forceinline__ float ldcg_pred(const float* src, bool valid) {
  float v;
  asm volatile("{\n .reg .pred q;\n setp.ne.b32 q, %2, 0;\n mov.b32 %0, 0;\n @q ld.global.cg.f32 %0, [%1];\n}\n"
               : "=f"(v)
               : "l"(src), "r"(static_cast<int>(valid)));
  return v;
}

// Largest exponent field of the eight 16-bit values of a chunk (BF16: bits 7-14; FP16: 10-14).
__device__ __forceinline__ int chunk_exp(const unsigned (&w)[4], bool f16) {
  const int sh = f16 ? 10 : 7;
  const unsigned mask = f16 ? 0x001f001fu : 0x00ff00ffu;
  const unsigned m = __vmaxu2(__vmaxu2((w[0] >> sh) & mask, (w[1] >> sh) & mask),
                              __vmaxu2((w[2] >> sh) & mask, (w[3] >> sh) & mask));
  return static_cast<int>(max(m & 0xffffu, m >> 16));
}

// The exponent es a (phase, token)'s BF16 x is scaled by: x * 2^(142 - es) is staged in FP16.
// es = the phase's largest exponent field, clamped so that 2^(142 - es) and 2^(es - 142) are
// normal FP32 powers of two (a phase below 2^-112 is scaled by 2^127; Inf / NaN stay so).
__device__ __forceinline__ int x_scale_exp(int emax) { return min(max(emax, 15), 254); }

// ------------------------------------------------------------------ kernel

// A CTA's run of units [u0, u1) in row-group order. Phase ph's units are the row groups
// lo(ph)..hi(ph); only the run's first and last row groups can miss phases.
struct TmRun {
  int u0, u1;
  int P, rg_lo, rg_hi, W;
  __device__ __forceinline__ int lo(int ph) const { return rg_lo + (rg_lo * P + ph < u0 ? 1 : 0); }
  __device__ __forceinline__ int hi(int ph) const { return rg_hi - (rg_hi * P + ph >= u1 ? 1 : 0); }
  __device__ __forceinline__ int count(int ph) const { return max(0, hi(ph) - lo(ph) + 1); }
  __device__ __forceinline__ int windows() const { return (P + W - 1) / W; }
  __device__ __forceinline__ int total(int win) const {   // units of a window
    int t = 0;
    for (int ph = win * W; ph < min(P, (win + 1) * W); ++ph) t += count(ph);
    return t;
  }
  __device__ __forceinline__ void unit(int win, int j, int& ph, int& rg) const {   // j-th unit of a window
    for (ph = win * W;; ++ph) {
      const int c = count(ph);
      if (j < c) break;
      j -= c;
    }
    rg = lo(ph) + j;
  }
  __device__ __forceinline__ bool whole(int rg) const { return rg * P >= u0 && rg * P + P <= u1; }
};

// A warp's position in its item sequence: window, unit index in the window (the warp's
// units are warp, warp + 8, ...), box of the unit.
struct TmPos {
  int win, j, box;
};

// Grid (CTAs); block kTmThreads. NB token blocks of 8.
template <int KIND, int NB>
__global__ void __launch_bounds__(kTmThreads, 1) tile_mma_kernel(const __grid_constant__ TmParams p) {
  using L = TmLayout<KIND>;
  constexpr int D = kTmDepth;
  constexpr int KS = KIND == TM_I8_ROW ? kTmKsI8 : kTmKsF4;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const unsigned wring = smem_addr(smem);
  const unsigned sring = wring + L::W;
  unsigned char* xs = smem + L::W + L::S;
  const unsigned bars = smem_addr(xs + L::X);
  int* tok_exp = reinterpret_cast<int*>(xs + L::X + L::BARS);   // [window phase][16]
  int* fold_flag = tok_exp + kTmMaxWin * 16;                     // [2] split groups to fold

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int P = p.phases;
  TmRun run;
  run.u0 = p.per_cta * blockIdx.x + min(static_cast<int>(blockIdx.x), p.extra);
  run.u1 = run.u0 + p.per_cta + (static_cast<int>(blockIdx.x) < p.extra ? 1 : 0);
  if (run.u1 <= run.u0) return;   // uniform per CTA
  run.P = P;
  run.rg_lo = run.u0 / P;
  run.rg_hi = (run.u1 - 1) / P;
  run.W = p.window;
  const int nwin = run.windows();

  // Item sequence of this warp: (window, unit, box); false past the end.
  auto settle = [&](TmPos& q) {
    while (q.win < nwin && q.j >= run.total(q.win)) {
      ++q.win;
      q.j = warp;
    }
    return q.win < nwin;
  };
  auto advance = [&](TmPos& q) {
    if (++q.box == kTmBoxes) {
      q.box = 0;
      q.j += kTmWarps;
    }
    return settle(q);
  };

  const unsigned wslot0 = wring + warp * D * kTmItem;
  const unsigned sslot0 = sring + warp * D * kTmScaleItem;
  const unsigned bar0 = bars + warp * D * 8;
  // Whole warp: item i = half q.box of unit (q.win, q.j): 16 rows x 512 bytes (and, E2M1, 16 x
  // 64 scale bytes), one 1-D bulk copy per row. Bytes past the row's end and rows past N are
  // not copied: x is zero there (INT8: stale codes times zero add nothing), E2M1 skips the
  // 256-column quarters past K, and rows past N are never stored.
  auto issue = [&](int i, const TmPos& q) {
    int ph, rg;
    run.unit(q.win, q.j, ph, rg);
    const long long col = static_cast<long long>(ph) * 1024 + q.box * kTmRowBytes;   // byte column
    const int rows = min(kTmRows, p.n - rg * kTmRows);
    const int bytes = static_cast<int>(max(0LL, min(static_cast<long long>(kTmRowBytes), p.row_bytes - col)));
    int sbytes = 0;
    const long long scol = col / 8, srow_bytes = p.row_bytes / 8;   // E2M1: 2 scale bytes per 16 weight bytes
    if constexpr (KIND == TM_FP4_G32H)
      sbytes = static_cast<int>(max(0LL, min(static_cast<long long>(kTmScaleRow), srow_bytes - scol)));
    const unsigned bar = bar0 + (i % D) * 8;
    if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<unsigned>(rows * (bytes + sbytes)));
    __syncwarp();
    const long long row0 = static_cast<long long>(rg) * kTmRows;
    if (lane < rows && bytes > 0)
      bulk_g2s(wslot0 + (i % D) * kTmItem + lane * kTmPitch, p.w + (row0 + lane) * p.row_bytes + col, bytes, bar);
    if constexpr (KIND == TM_FP4_G32H) {
      const int r = lane - 16;
      if (r >= 0 && r < rows && sbytes > 0)
        bulk_g2s(sslot0 + (i % D) * kTmScaleItem + r * kTmScaleRow, p.s + (row0 + r) * srow_bytes + scol, sbytes,
                 bar);
    }
  };

  TmPos iss{0, warp, 0};
  bool more = settle(iss);
  int issued = 0;
  if (lane == 0) {
    for (int i = 0; i < D; ++i) mbar_init(bar0 + 8 * i, 1);
    fence_mbar_init();
  }
  // The first access to a page whose translation is not cached stalls the issuing warp
  // for a page walk (about 0.7 us, 1.8 us when the page tables are out of L2). Touch the
  // pages of x, the partials, the tickets, the output and the row scales now, from lanes
  // with nothing else to do, so that the walks overlap the weight stream. (A prefetch
  // of x before the grid dependency wait only warms translations and L2.)
  if (warp == kTmWarps - 1 && lane >= 27) {
    const long long r0 = static_cast<long long>(run.rg_lo) * kTmRows;
    const void* addr = lane == 27   ? p.x
                       : lane == 28 ? static_cast<const void*>(p.part + static_cast<long long>(run.rg_lo) * P * p.m * kTmRows)
                       : lane == 29 ? static_cast<const void*>(p.tickets + run.rg_lo)
                       : lane == 30 ? static_cast<const void*>(static_cast<const char*>(p.out) + r0 * (p.out_f32 ? 4 : 2))
                       : KIND == TM_I8_ROW ? static_cast<const void*>(p.row_scale + r0)
                                           : static_cast<const void*>(p.s + r0 * (p.row_bytes / 8));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(addr));
  }
  __syncwarp();
  // Weights do not depend on the previous grid: start streaming before the wait, but only
  // kTmEarly items, so that the x loads of the first window do not queue behind a full ring
  // of weight requests from every SM; the rest of the ring is issued once x is staged.
  for (; issued < kTmEarly && more; ++issued) {
    issue(issued, iss);
    more = advance(iss);
  }

  grid_dependency_wait();

  const bool f16 = p.x_f16 != 0;
  const int mt = p.m;   // tokens (<= NB * 8)
  const bool xvec = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 && (p.ldx & 7) == 0;
  const unsigned xs_base = smem_addr(xs);

  // Stage x of window win as FP16 chunks [32-K group][t][c] (groups counted from the
  // window's first column; chunk c = the eight columns thread c owns: INT8 4c..4c+3 and
  // 16+4c..16+4c+3, E2M1 8c..8c+7). Every load of the window is issued before any is
  // used (one round trip to L2), each (phase, token)'s largest exponent is gathered in
  // shared memory, then the chunks are scaled and converted from registers.
  auto stage = [&](int win) {
    const int ph0 = win * run.W, nph = min(P, ph0 + run.W) - ph0;
    const int kw = ph0 * KS;                      // first column of the window
    const int units = nph * (KS / 32) * mt * 4;   // <= kTmThreads * kTmUpt (the window's size rule)
    unsigned raw[kTmUpt][4];
    int key[kTmUpt];                              // (phase in window) * 16 + token, -1 past the window
    const unsigned short* xb = static_cast<const unsigned short*>(p.x);
#pragma unroll
    for (int q = 0; q < kTmUpt; ++q) {
      const int u = threadIdx.x + q * kTmThreads;   // chunk (G, t, cc) sits at (G * mt + t) * 4 + cc = u
      const int gt = u >> 2, cc = u & 3;
      const int G = (gt * p.div_m) >> 16;           // 32-K group in the window (exact: gt < 2^10, m <= 16)
      const int t = gt - G * mt;
      key[q] = u < units ? (G / (KS / 32)) * 16 + t : -1;
      const int col0 = kw + 32 * G + (KIND == TM_I8_ROW ? 4 : 8) * cc;
      const unsigned short* row = xb + static_cast<long long>(t) * p.ldx;
      if (xvec) {   // chunks never straddle K (INT8: K % 16 == 0, E2M1: K % 256 == 0)
        if constexpr (KIND == TM_I8_ROW) {
          ldcg_v2_pred(row + col0, key[q] >= 0 && col0 < p.k, raw[q][0], raw[q][1]);
          ldcg_v2_pred(row + col0 + 16, key[q] >= 0 && col0 + 16 < p.k, raw[q][2], raw[q][3]);
        } else {
          ldcg_v4_pred(row + col0, key[q] >= 0 && col0 < p.k, raw[q]);
        }
      } else {      // x not 16-byte aligned (or its row stride not a multiple of 8): 16-bit loads
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const int col = KIND == TM_I8_ROW ? col0 + (v & 3) + 16 * (v >> 2) : col0 + v;
          const unsigned h = ldcg_u16_pred(row + col, key[q] >= 0 && col < p.k);
          raw[q][v >> 1] = (v & 1) ? (raw[q][v >> 1] | (h << 16)) : h;
        }
      }
    }
    if (threadIdx.x < nph * 16) tok_exp[threadIdx.x] = 0;
    __syncthreads();
    if (!f16) {   // FP16 x is staged as it is
#pragma unroll
      for (int q = 0; q < kTmUpt; ++q) {
        const int e = chunk_exp(raw[q], false);
        const int k0 = __shfl_sync(0xffffffffu, key[q], 0);
        if (__all_sync(0xffffffffu, key[q] == k0)) {   // one (phase, token) for the warp (M = 1)
          const int em = __reduce_max_sync(0xffffffffu, e);
          if (lane == 0 && k0 >= 0) atomicMax(tok_exp + k0, em);
        } else if (key[q] >= 0) {
          atomicMax(tok_exp + key[q], e);
        }
      }
    }
    __syncthreads();
    uint4* dst = reinterpret_cast<uint4*>(xs);
#pragma unroll
    for (int q = 0; q < kTmUpt; ++q) {
      if (key[q] < 0) break;   // keys rise with q
      unsigned w4[4] = {raw[q][0], raw[q][1], raw[q][2], raw[q][3]};
      if (!f16) {   // BF16 -> FP16 scaled by 2^(142 - es): the largest lands in [2^15, 2^16)
        const float scale = __int_as_float((269 - x_scale_exp(tok_exp[key[q]])) << 23);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float f0 = mul_rn(__uint_as_float(w4[v] << 16), scale);
          const float f1 = mul_rn(__uint_as_float(w4[v] & 0xffff0000u), scale);
          asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(w4[v]) : "f"(f1), "f"(f0));
        }
      }
      dst[threadIdx.x + q * kTmThreads] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
    __syncthreads();
  };

  // Final value of (row, token t) from its K total v (INT8: times the row scale).
  auto store = [&](int row, int t, float v) {
    const long long o = static_cast<long long>(t) * p.ldo + row;
    if constexpr (KIND == TM_I8_ROW) v = mul_rn(v, __ldg(p.row_scale + row));
    if (p.out_f32)
      static_cast<float*>(p.out)[o] = v;
    else
      static_cast<unsigned short*>(p.out)[o] = f32_to_bf16_rn(v);
  };

  float* part = p.part;
  bool ok = true;
  int drain_from = -1;   // first item not waited for after a timeout
  int i = 0;             // items consumed by this warp
  for (int win = 0; win < nwin; ++win) {
    __syncthreads();     // every warp is done with the previous window's x
    stage(win);
    if (win == 0) {
      grid_launch_dependents();
      for (; issued < D && more; ++issued) {   // the rest of the ring
        issue(issued, iss);
        more = advance(iss);
      }
    }
    const int tot = run.total(win);
    for (int j = warp; j < tot; j += kTmWarps) {
      int ph, rg;
      run.unit(win, j, ph, rg);
      const int pw = ph - win * run.W;
      float acc[4][NB][4];   // INT8: [step parity x MMA half][token block][C register]
      float facc[NB][4];     // E2M1: group-scaled FP32 chain over the unit
#pragma unroll
      for (int b = 0; b < NB; ++b)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          facc[b][q] = 0.0f;
#pragma unroll
          for (int h = 0; h < 4; ++h) acc[h][b][q] = 0.0f;
        }
      for (int box = 0; box < kTmBoxes; ++box, ++i) {
        const unsigned slot = wslot0 + (i % D) * kTmItem;
        const bool landed = ok && mbar_wait(bar0 + (i % D) * 8, (i / D) & 1);
        if (!__all_sync(0xffffffffu, landed)) {   // a timed-out warp stops waiting and issuing
          if (ok) drain_from = i;
          ok = false;
        }
        if (ok) {
          if constexpr (KIND == TM_I8_ROW) {
            // Straight-line and software-pipelined: step st + 1's fragments are read before
            // step st's MMAs. Token columns past M read token M - 1's x; their sums are never
            // stored, and no branch splits the block.
            unsigned a[2][4];
            uint4 xq[2][NB];
            auto load_step = [&](int st, unsigned (&aa)[4], uint4 (&xx)[NB]) {
              ldsm_x4(slot + (lane & 15) * kTmPitch + (2 * st + (lane >> 4)) * 16, aa);
              const int G = pw * (KS / 32) + box * 16 + st;   // 32-K group in the window
#pragma unroll
              for (int b = 0; b < NB; ++b) xx[b] = lds128(xs_base + (((G * mt + min(8 * b + g, mt - 1)) * 4 + c) << 4));
            };
            load_step(0, a[0], xq[0]);
#pragma unroll
            for (int st = 0; st < 16; ++st) {   // the item's sixteen 32-K steps
              const int cur = st & 1;
              if (st + 1 < 16) load_step(st + 1, a[cur ^ 1], xq[cur ^ 1]);
              // a[0] / a[1]: rows g / g + 8, columns 4c..4c+3; a[2] / a[3]: columns 16+4c..
              unsigned w0l, w0h, w1l, w1h, w2l, w2h, w3l, w3h;
              i8x4_to_f16x4(a[cur][0], w0l, w0h);
              i8x4_to_f16x4(a[cur][1], w1l, w1h);
              i8x4_to_f16x4(a[cur][2], w2l, w2h);
              i8x4_to_f16x4(a[cur][3], w3l, w3h);
#pragma unroll
              for (int b = 0; b < NB; ++b) {
                mma_f16(acc[2 * cur][b], w0l, w1l, w0h, w1h, xq[cur][b].x, xq[cur][b].y, acc[2 * cur][b]);
                mma_f16(acc[2 * cur + 1][b], w2l, w3l, w2h, w3h, xq[cur][b].z, xq[cur][b].w, acc[2 * cur + 1][b]);
              }
            }
          } else {
            const unsigned sslot = sslot0 + (i % D) * kTmScaleItem;
            const int g0 = (ph * KS + box * 1024) / 32;   // first 32-K group of the item in K
            // Per quarter (8 groups): the four A loads, then every group's first MMA, then
            // every second MMA (each group still chains its two halves in the tensor core's
            // order), then the FP32 chain over the groups in K order. Token columns past M
            // read token M - 1's x (never stored); no branch splits the quarter.
#pragma unroll 1
            for (int pq = 0; pq < 4; ++pq) {   // quarters of the item: 8 groups each
              if ((g0 + 8 * pq) * 32 >= p.k) break;   // past K (uniform): scales there are not copied
              unsigned a[4][4];   // pair pr: rows g / g + 8 of groups 2pr, 2pr + 1, columns 8c .. 8c + 7
#pragma unroll
              for (int pr = 0; pr < 4; ++pr)
                ldsm_x4(slot + (lane & 15) * kTmPitch + (8 * pq + 2 * pr + (lane >> 4)) * 16, a[pr]);
              const uint4 sg = lds128(sslot + g * kTmScaleRow + 16 * pq);        // row g, 8 groups' FP16 scales
              const uint4 sg8 = lds128(sslot + (g + 8) * kTmScaleRow + 16 * pq);
              uint4 xv[8][NB];
#pragma unroll
              for (int gl = 0; gl < 8; ++gl) {
                const int G = pw * (KS / 32) + box * 32 + 8 * pq + gl;   // group within the window
#pragma unroll
                for (int b = 0; b < NB; ++b)
                  xv[gl][b] = lds128(xs_base + (((G * mt + min(8 * b + g, mt - 1)) * 4 + c) << 4));
              }
              unsigned wa[8][4];   // group gl: second-MMA A words (columns 8c+4..8c+7, rows g / g + 8)
              float d[8][NB][4];
#pragma unroll
              for (int gl = 0; gl < 8; ++gl) {
                // Byte v of a row word holds columns 8c + 2v, 8c + 2v + 1.
                const unsigned ra = a[gl >> 1][2 * (gl & 1)], rb = a[gl >> 1][2 * (gl & 1) + 1];   // row g, row g + 8
                const unsigned a00 = e2m1x2_to_f16x2(ra & 0xffu), a01 = e2m1x2_to_f16x2((ra >> 8) & 0xffu);
                const unsigned a10 = e2m1x2_to_f16x2(rb & 0xffu), a11 = e2m1x2_to_f16x2((rb >> 8) & 0xffu);
                wa[gl][0] = e2m1x2_to_f16x2((ra >> 16) & 0xffu), wa[gl][1] = e2m1x2_to_f16x2((rb >> 16) & 0xffu);
                wa[gl][2] = e2m1x2_to_f16x2(ra >> 24), wa[gl][3] = e2m1x2_to_f16x2(rb >> 24);
                const float zero[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int b = 0; b < NB; ++b) mma_f16(d[gl][b], a00, a10, a01, a11, xv[gl][b].x, xv[gl][b].y, zero);
              }
#pragma unroll
              for (int gl = 0; gl < 8; ++gl)
#pragma unroll
                for (int b = 0; b < NB; ++b)
                  mma_f16(d[gl][b], wa[gl][0], wa[gl][1], wa[gl][2], wa[gl][3], xv[gl][b].z, xv[gl][b].w, d[gl][b]);
              const unsigned srow[4] = {sg.x, sg.y, sg.z, sg.w}, srow8[4] = {sg8.x, sg8.y, sg8.z, sg8.w};
#pragma unroll
              for (int gl = 0; gl < 8; ++gl) {
                const unsigned hs = (gl & 1) ? (srow[gl >> 1] >> 16) : (srow[gl >> 1] & 0xffffu);
                const unsigned hs8 = (gl & 1) ? (srow8[gl >> 1] >> 16) : (srow8[gl >> 1] & 0xffffu);
                const float s0 = f16_to_f32(static_cast<unsigned short>(hs));
                const float s8 = f16_to_f32(static_cast<unsigned short>(hs8));
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                  facc[b][0] = fma_rn(d[gl][b][0], s0, facc[b][0]);
                  facc[b][1] = fma_rn(d[gl][b][1], s0, facc[b][1]);
                  facc[b][2] = fma_rn(d[gl][b][2], s8, facc[b][2]);
                  facc[b][3] = fma_rn(d[gl][b][3], s8, facc[b][3]);
                }
              }
            }
          }
        }
        __syncwarp();
        // Refill the slot with the item D ahead (the warp's cursor is uniform).
        if (more && ok) {
          issue(issued, iss);
          more = advance(iss);
          ++issued;
        }
      }
      // The unit's phase partial, the phase's x scaling undone (a power of two: exact), into
      // the workspace. C register q: row g + 8 * (q >> 1), token 8b + 2c + (q & 1).
#pragma unroll
      for (int b = 0; b < NB; ++b)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int r = g + 8 * (q >> 1), t = 8 * b + 2 * c + (q & 1);
          if (t >= p.m) continue;
          float v = KIND == TM_I8_ROW ? add_rn(add_rn(acc[0][b][q], acc[1][b][q]), add_rn(acc[2][b][q], acc[3][b][q]))
                                      : facc[b][q];
          if (!f16) v = mul_rn(v, __int_as_float((x_scale_exp(tok_exp[pw * 16 + t]) - 15) << 23));
          part[((static_cast<long long>(rg) * P + ph) * p.m + t) * kTmRows + r] = v;
        }
    }
  }

  // ---- this CTA's row groups: add the phase partials in phase order. A group split with a
  // neighbouring CTA (the run's ends) is added by the CTA that completes its ticket.
  __syncthreads();   // every phase partial of this CTA is written
  if (threadIdx.x == 0) {   // tickets are counted even after a timeout, so they always return to zero
    fold_flag[0] = fold_flag[1] = -1;
    const int ends[2] = {run.rg_lo, run.rg_hi};
    __threadfence();
    for (int e = 0; e < 2; ++e) {
      const int rg = ends[e];
      if (e == 1 && run.rg_hi == run.rg_lo) break;
      if (run.whole(rg)) continue;
      unsigned mine = 0;
      for (int ph = 0; ph < P; ++ph) mine += (run.lo(ph) <= rg && rg <= run.hi(ph)) ? 1u : 0u;
      if (atomicAdd(p.tickets + rg, mine) + mine == static_cast<unsigned>(P)) fold_flag[e] = rg;
    }
    __threadfence();
  }
  __syncthreads();
  const int first = run.whole(run.rg_lo) ? run.rg_lo : run.rg_lo + 1;
  const int last = run.whole(run.rg_hi) ? run.rg_hi : run.rg_hi - 1;
  auto fold_group = [&](int rg, int idx) {   // element idx = t * 16 + r of row group rg
    const int t = idx / kTmRows, r = idx % kTmRows, row = rg * kTmRows + r;
    if (row >= p.n) return;
    const float* src = part + static_cast<long long>(rg) * P * p.m * kTmRows + t * kTmRows + r;
    const long long step = static_cast<long long>(p.m) * kTmRows;
    float v = 0.0f;
    for (int ph0 = 0; ph0 < P; ph0 += 8) {   // eight phases' loads in flight, added in phase order
      float buf[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) buf[q] = ldcg_pred(src + (ph0 + q) * step, ph0 + q < P);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (ph0 + q < P) v = ph0 + q == 0 ? buf[q] : add_rn(v, buf[q]);
    }
    store(row, t, v);
  };
  {
    const int per = p.m * kTmRows;
    for (int e = threadIdx.x; e < (last - first + 1) * per; e += kTmThreads) fold_group(first + e / per, e % per);
    for (int e = 0; e < 2; ++e) {
      const int rg = fold_flag[e];
      if (rg < 0) continue;
      for (int idx = threadIdx.x; idx < per; idx += kTmThreads) fold_group(rg, idx);
      if (threadIdx.x == 0) p.tickets[rg] = 0u;
    }
  }

  if (!ok) {
    record_status(p.status, kStatusMbarTimeout);
    if (lane == 0 && drain_from >= 0)   // drain this warp's copies still in flight (bounded)
      for (int it = drain_from; it < issued; ++it) mbar_wait(bar0 + (it % D) * 8, (it / D) & 1);
  }
}

template <int KIND, int NB>
cudaError_t tm_launch(const TmParams& p, int ctas, cudaStream_t stream, bool pdl) {
  auto kernel = tile_mma_kernel<KIND, NB>;
  constexpr int smem = TmLayout<KIND>::TOTAL;
  const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kTmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace

size_t tile_mma_workspace(int kind, int m, int n, int k) {
  const int ks = kind == TM_I8_ROW ? kTmKsI8 : kTmKsF4;
  const long long phases = (k + ks - 1) / ks;
  const long long groups = (n + kTmRows - 1) / kTmRows;
  return kTileMmaTicketBytes + static_cast<size_t>(groups * phases) * m * kTmRows * sizeof(float);
}

int tile_mma_launch(int kind, int x_f16, const void* x, int ldx, const void* w, const void* scales, void* out,
                    int ldo, int out_f32, int m, int n, int k, void* ws, size_t ws_bytes, int sms, int* status,
                    bool pdl, cudaStream_t stream) {
  if (!x || !w || !scales || !out || m <= 0 || n <= 0 || k <= 0) return KLAB_E_INVALID;
  if (m > 16) return KLAB_E_UNSUPPORTED;
  // Bulk copies: 16-byte aligned bases and row strides; x read as 16-bit values.
  const long long row_bytes = kind == TM_I8_ROW ? k : k / 2;
  if ((reinterpret_cast<uintptr_t>(w) & 15) || row_bytes % 16 || (reinterpret_cast<uintptr_t>(x) & 1))
    return KLAB_E_ALIGN;
  if (kind == TM_FP4_G32H && (k % 256 || (reinterpret_cast<uintptr_t>(scales) & 15))) return KLAB_E_ALIGN;
  const int ks = kind == TM_I8_ROW ? kTmKsI8 : kTmKsF4;
  const long long phases = (k + ks - 1) / ks;
  const long long ngroups = (n + kTmRows - 1) / kTmRows;
  const long long units = ngroups * phases;
  // The phase partials live in the workspace: without it the CUDA cores take the launch.
  if (!ws || ws_bytes < tile_mma_workspace(kind, m, n, k) || (reinterpret_cast<uintptr_t>(ws) & 15) ||
      static_cast<size_t>(ngroups) * 4 > kTileMmaTicketBytes || units > (1LL << 30))
    return KLAB_E_UNSUPPORTED;
  TmParams p;
  std::memset(&p, 0, sizeof(p));
  p.tickets = static_cast<unsigned*>(ws);
  p.part = reinterpret_cast<float*>(static_cast<char*>(ws) + kTileMmaTicketBytes);
  const int ctas = units < sms ? static_cast<int>(units) : sms;
  long long window = kTmXMax / (static_cast<long long>(m) * ks * 2);
  window = window < 1 ? 1 : window > kTmMaxWin ? kTmMaxWin : window;
  if (window > phases) window = phases;
  p.w = static_cast<const unsigned char*>(w);
  p.s = static_cast<const unsigned char*>(scales);
  p.row_bytes = row_bytes;
  p.x = x;
  p.row_scale = kind == TM_I8_ROW ? static_cast<const float*>(scales) : nullptr;
  p.out = out;
  p.status = status;
  p.ldx = ldx;
  p.ldo = ldo;
  p.out_f32 = out_f32;
  p.x_f16 = x_f16;
  p.m = m;
  p.n = n;
  p.k = k;
  p.phases = static_cast<int>(phases);
  p.window = static_cast<int>(window);
  p.units = static_cast<int>(units);
  p.per_cta = static_cast<int>(units / ctas);
  p.extra = static_cast<int>(units % ctas);
  p.div_m = (65536 + m - 1) / m;
  const bool two = m > 8;
  if (kind == TM_I8_ROW)
    return two ? tm_launch<TM_I8_ROW, 2>(p, ctas, stream, pdl) : tm_launch<TM_I8_ROW, 1>(p, ctas, stream, pdl);
  return two ? tm_launch<TM_FP4_G32H, 2>(p, ctas, stream, pdl) : tm_launch<TM_FP4_G32H, 1>(p, ctas, stream, pdl);
}

}  // namespace klab
