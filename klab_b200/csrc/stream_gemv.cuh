// Weight-streaming projection y[M,N] = x[M,K] . W[N,K]^T for M <= 8 per token tile.
//
// One template serves every weight format of the reference's projection path:
//   W_BF16    BF16 weights (compressed_kernels.cu raw, half_kernels.cu bf16)
//   W_F16     FP16 weights (half_kernels.cu f16)
//   W_F32     FP32 weights (kernels.cu gemv_*, projection_kernels.cu)
//   W_CBF16   lossless BF16 codec v1 (compressed_kernels.cu:38-106, docs/bf16-format.md)
//   W_I8_ROW  int8 + one fp32 scale per row (benchmark config 2)
//   W_I8_G64  int8 + fp32 scale per 64 (int8_kernels.cu, int8_weights.py:23-35)
//   W_FP4_G32H E2M1 + fp16 scale per 32 (benchmark config 3)
//   W_FP4_G16E E2M1 + E4M3 scale per 16 + fp32 global (fp4_kernels.cu, fp4.py:33-60)
//   W_LF32    lossless FP32 v1 (lossless_kernels.cu, lossless_weights.py)
//   W_FP28    lossless FP32 as 28-bit codes (adaptive_kernels.cu fp28, packed_fp32.py)
// The two lossless FP32 formats are decoded to their exact FP32 bits while a warp
// fills its slot (cooperative fill, no bulk copy) and then use W_F32's arithmetic,
// so their results are bit-identical to the FP32 projection of the same weights.
//
// Data movement (B200): every warp owns a private ring of DEPTH shared-memory
// slots filled by 1-D bulk copies (cp.async.bulk into this CTA only) with mbarrier
// completion; a slot holds one "item" = one row x one K-chunk of 4 KiB of weight
// bytes plus that chunk's scales. Weights never depend on the previous kernel, so
// the first copies are issued before griddepcontrol.wait (programmatic dependent
// launch): under PDL they overlap the previous kernel's tail.
//
// Arithmetic order (a function of K and the format only, never of N, M, the
// grid, the shard or whether the weights are coded):
//   * chunk c covers columns [c*KC, min(K, (c+1)*KC)), KC = 256*VALS;
//   * segment j (0..7) of a chunk, lane l: values v = 0..VALS-1 at column
//     c*KC + 32*VALS*j + VALS*l + v;
//   * unscaled formats: per lane eight FP32 sums s0..s7, value v feeding s[v % 8]
//     with fma.rn, running over the chunk's segments in order; lane partial =
//     ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7));
//   * scaled formats: per lane and scale group the same eight sums start at
//     zero, g = their tree, then acc = fma.rn(g, scale, acc) in segment order;
//     lane partial = acc;
//   * chunk partial = butterfly warp sum of lane partials;
//   * row total = ((P0 + P1) + P2) + ... over chunks in order;
//   * per-row scale (W_I8_ROW) or global scale (W_FP4_G16E): one fp32 multiply;
//   * BF16 output: a single cvt.rn.bf16.f32.
// Consequences: raw and coded BF16 are bit-identical; every token of an M-tile
// is bit-identical to the same token computed alone; a column shard (any row
// subset) is bit-identical to the 1-GPU result; split-K across CTAs (below) gives
// the same bits as one warp doing the whole row.
#pragma once
#include "common.cuh"
#include "decode_ops.cuh"
#include "lossless_f32.cuh"

namespace klab {

enum WFmt : int {
  W_BF16 = 0,
  W_F16 = 1,
  W_F32 = 2,
  W_CBF16 = 3,
  W_I8_ROW = 4,
  W_I8_G64 = 5,
  W_FP4_G32H = 6,
  W_FP4_G16E = 7,
  W_LF32 = 8,      // lossless FP32 v1 (3-byte mantissa + exponent stream), decoded into the slot
  W_FP28 = 9,      // lossless FP32 in 28-bit codes, decoded into the slot
};
enum XFmt : int { X_BF16 = 0, X_F16 = 1, X_F32 = 2 };
// Where x lives while the tile is computed.
enum XMode : int { XM_SMEM = 0, XM_GLOBAL = 1, XM_SMEM16 = 2 };

#ifndef KLAB_WARPS
#define KLAB_WARPS 16      // warps per CTA for single-token tiles
#endif
#ifndef KLAB_WARPS_MT
#define KLAB_WARPS_MT 16   // warps per CTA for 2- and 4-token tiles
#endif
#ifndef KLAB_WARPS_MT8
#define KLAB_WARPS_MT8 8   // warps per CTA for 8-token tiles (their x takes the shared memory)
#endif
#ifndef KLAB_DEPTH
#define KLAB_DEPTH 2
#endif
#ifndef KLAB_SEG_UNROLL
#define KLAB_SEG_UNROLL 8
#endif
// Warps per CTA for a token tile of MT.
// INT8 single-token tiles run as two 12-warp CTAs per SM: their item math is
// the heaviest per byte, and 24 resident warps hide its latency better than 16
// (config 2, M=1: 14.4 -> 13.3 us); the other formats keep one 16-warp CTA.
#ifndef KLAB_WARPS_I8
#define KLAB_WARPS_I8 12
#endif
__host__ __device__ constexpr bool int8_format(int f) { return f == W_I8_ROW || f == W_I8_G64; }
__host__ __device__ constexpr int warps_for(int f, int mt) {
  return mt == 1 ? (int8_format(f) ? KLAB_WARPS_I8 : KLAB_WARPS) : mt == 8 ? KLAB_WARPS_MT8 : KLAB_WARPS_MT;
}
__host__ __device__ constexpr int min_blocks_for(int f, int mt) { return mt == 1 && int8_format(f) ? 2 : 1; }
constexpr int kDepth = KLAB_DEPTH;    // ring slots per warp
constexpr int kSegUnroll = KLAB_SEG_UNROLL;
constexpr int kSegs = 8;              // segments per chunk
constexpr int kWeightSlot = 4096;     // weight bytes per full chunk
constexpr int kMetaRing = 2 * kDepth;  // coded: metadata entries per warp
constexpr int kMetaEntry = 128;       // 32 blocks * 4 bytes
// Default prologue (before griddepcontrol.wait), per warp: items copied into the
// ring and the following items prefetched into L2. x is staged right after the
// wait and its loads queue behind this SM's bulk copies, so copies into shared
// memory delay x; L2 prefetches only load the weights into L2.
#ifndef KLAB_PRO_SMEM
#define KLAB_PRO_SMEM 1
#endif
#ifndef KLAB_PRO_L2
#define KLAB_PRO_L2 0
#endif
constexpr int kProSmem = KLAB_PRO_SMEM;
constexpr int kProL2 = KLAB_PRO_L2;

template <int F>
struct WTraits;
template <>
struct WTraits<W_BF16> {
  static constexpr int VALS = 8, NUM = 2, DEN = 1, SCALE_BYTES = 0;
};
template <>
struct WTraits<W_F16> {
  static constexpr int VALS = 8, NUM = 2, DEN = 1, SCALE_BYTES = 0;
};
template <>
struct WTraits<W_F32> {
  static constexpr int VALS = 4, NUM = 4, DEN = 1, SCALE_BYTES = 0;
};
template <>
struct WTraits<W_CBF16> {
  static constexpr int VALS = 8, NUM = 2, DEN = 1, SCALE_BYTES = 0;
};
template <>
struct WTraits<W_I8_ROW> {
  static constexpr int VALS = 16, NUM = 1, DEN = 1, SCALE_BYTES = 0;
};
template <>
struct WTraits<W_I8_G64> {
  static constexpr int VALS = 16, NUM = 1, DEN = 1, SCALE_BYTES = 256;
};
template <>
struct WTraits<W_FP4_G32H> {
  static constexpr int VALS = 32, NUM = 1, DEN = 2, SCALE_BYTES = 512;
};
template <>
struct WTraits<W_FP4_G16E> {
  static constexpr int VALS = 32, NUM = 1, DEN = 2, SCALE_BYTES = 512;
};
template <>
struct WTraits<W_LF32> {
  static constexpr int VALS = 4, NUM = 4, DEN = 1, SCALE_BYTES = 0;
};
template <>
struct WTraits<W_FP28> {
  static constexpr int VALS = 4, NUM = 4, DEN = 1, SCALE_BYTES = 0;
};

template <int F>
struct Layout {
  static constexpr int VALS = WTraits<F>::VALS;
  static constexpr int KC = 32 * kSegs * VALS;
  static constexpr int SLOT = kWeightSlot + WTraits<F>::SCALE_BYTES;
  static constexpr int META = (F == W_CBF16) ? kMetaRing * kMetaEntry : 0;
  static constexpr int WARP_BYTES = kDepth * SLOT + META;
  static constexpr int BARS = kDepth + ((F == W_CBF16) ? kMetaRing : 0);
};

// One weight matrix of a launch. Several matrices that share x and K (the
// projections that read the same activations) can run in one launch; their rows
// are concatenated: segment s owns launch rows [row0, next row0).
constexpr int kMaxSegs = 8;
struct Segment {
  const void* w;    // weights, codes or coded payload
  const void* aux;  // coded metadata (u32) / scales
  const void* aux2; // W_LF32: exponent stream
  void* out;        // out[t * ldo + local row]
  int ldo;
  int row0;         // first launch row of this segment
};

// Output gather over NVLink peer memory, fused into the projection. The
// gathered segment's output rows are also stored into every peer's copy of the
// full-width output buffer; when the whole grid is done, the last CTA raises this
// rank's flag in `signal_slot` of every peer with the current epoch. A launch
// whose x is a gathered buffer first waits (bounded) until every rank's flag in
// `wait_slot` of the local flag array reaches the epoch. Flags are monotonic.
constexpr int kMaxPeers = 8;
struct Gather {
  int npeers;                     // ranks taking part (0: no gather)
  int rank;
  int seg;                        // segment whose output is pushed (-1: none)
  void* peer_out[kMaxPeers];      // rank r's copy of that segment's output buffer
  unsigned* peer_flags[kMaxPeers];  // rank r's flag array [slots][npeers]
  int signal_slot;                // slot raised after this launch (-1: none)
  const unsigned* wait_flags;     // local flag array (nullptr: no wait)
  int wait_slot;
  const unsigned* epoch;          // current step's epoch (device word)
  unsigned* done;                 // CTA completion counter, zero between launches
};

// Elementwise op fused into the x staging (BF16 x, BF16 weights): x is not read
// from `x` but computed per token from the op's inputs, with the arithmetic of
// the standalone kernels (decode_ops.cuh), so the projection equals the
// standalone op followed by the plain projection, bit for bit.
enum ProOp : int { PRO_NONE = 0, PRO_ADD_RMSNORM = 1, PRO_SILU_MUL = 2 };
struct Prologue {
  int op;
  int ld;              // row stride of a / b in elements (BF16)
  float eps;
  const void* a;       // ADD_RMSNORM: residual [M, K]; SILU_MUL: [gate | up] [M, 2K]
  const void* b;       // ADD_RMSNORM: y [M, K]
  const void* w;       // ADD_RMSNORM: norm weight [K]
  void* x_out;         // ADD_RMSNORM: RNE(residual + y) [M, K] (written by the grid's column 0)
  int x_out_ld;
};

struct GemvParams {
  Gather gather;
  Prologue pro;
  const void* x;        // [M, ldx] activations (X format)
  const float* gscale;  // W_FP4_G16E global scale (device scalar)
  Segment seg[kMaxSegs];
  int nseg;
  float* ws;            // split mode: partials [tiles*MT][N][S]
  unsigned* tickets;    // split mode: [tiles][N], zero between launches
  int* status;          // device status word
  int m, n, k;          // n: total rows over all segments
  int ldx;
  int out_f32;
  int split;      // 0: rows dealt to CTAs; 1: items dealt to CTAs (split-K)
  int use_tma;    // 1: bulk copies; 0: cooperative loads (any alignment)
  int chunks;     // S = ceil(K / KC)
  int pro_smem;   // prologue: items copied into the ring before griddepcontrol.wait
  int pro_l2;     // prologue: following items prefetched into L2 (uncoded formats)
};

// Segment of a launch row and the row's index inside that segment.
struct RowRef {
  const char* w;
  const char* aux;
  const char* aux2;
  int local;
  int seg;
};

__device__ __forceinline__ RowRef resolve_row(const GemvParams& p, int row) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < kMaxSegs; ++i)
    if (i < p.nseg && row >= p.seg[i].row0) s = i;
  return RowRef{static_cast<const char*>(p.seg[s].w), static_cast<const char*>(p.seg[s].aux),
                static_cast<const char*>(p.seg[s].aux2), row - p.seg[s].row0, s};
}

// ------------------------------------------------------------------ x staging

// x lives in shared memory in a lane-interleaved layout. For token t, global
// segment g (32*VALS columns) and 16-byte vector i of a lane's VALS values,
// lane l's vector is 16-byte unit ((t*G + g)*NV + i)*32 + l. A warp's
// ld.shared.v4 of vector i of one segment touches 512 consecutive bytes: no
// bank conflicts. XM_SMEM stores FP32 (NV = VALS/4); XM_SMEM16 stores the
// 16-bit input values unchanged (NV = VALS/8, BF16/FP16 x only). Columns >= K
// and tokens >= M are zero.
// x is read with L2-only loads (ld.global.cg): peers may have written it over
// NVLink, so no line of it may come from this SM's L1.
template <int X>
__device__ __forceinline__ float x_value(const void* x, long long idx) {
  if constexpr (X == X_BF16) {
    return __uint_as_float(static_cast<unsigned>(__ldcg(static_cast<const unsigned short*>(x) + idx)) << 16);
  } else if constexpr (X == X_F16) {
    return f16_to_f32(__ldcg(static_cast<const unsigned short*>(x) + idx));
  } else {
    return __ldcg(static_cast<const float*>(x) + idx);
  }
}

template <int F, int XM>
struct XLayout {
  static constexpr int VALS = WTraits<F>::VALS;
  static constexpr int EB = (XM == XM_SMEM16) ? 2 : 4;  // bytes per staged value
  static constexpr int NV = VALS * EB / 16;             // 16-byte vectors per lane per segment
  static constexpr int SEG_BYTES = NV * 512;            // one segment of one token
};

// FP16 activations for integer and E2M1 weights. Their weight values are exact in
// FP16 (|int8| <= 127, E2M1 magnitudes 0..6), so with x in FP16 every product is
// one fma.rn.f32.f16 on unconverted 16-bit operands: exact product, one rounding,
// the same value sequence and accumulators as the FP32 path, so the same bits.
// BF16 x is staged as FP16 after multiplying token t by 2^s_t (exact), chosen
// per token from the exponents of its nonzero values; the row total is multiplied
// by 2^-s_t (exact) before any weight scale. The scaling commutes with every
// rounding when the token's values satisfy (bf16 exponent fields, nonzero values)
//   emin >= 39       products, group sums and group-scaled sums stay normal in
//                    FP32 (group scales are FP16 or E4M3, >= 2^-24),
//   emax <= 200      no FP32 overflow in either scaling,
//   emax - emin <= 32  every scaled value is exact in FP16 (largest < 2^16,
//                    lowest set bit >= 2^-24), with s_t = 142 - emax;
// otherwise the tile keeps BF16 staging and the FP32 path. FP16 x needs no check.
template <int F, int X, int XM>
struct HalfX {
  static constexpr bool value = XM == XM_SMEM16 && (X == X_BF16 || X == X_F16) &&
                                (F == W_I8_ROW || F == W_FP4_G32H || F == W_FP4_G16E);
};

// Per-CTA state of the FP16 staging (shared memory).
struct XHalfState {
  int emax[8], emin[8];  // per token: bf16 exponent field range of the nonzero values
  float inv[8];          // per token: 2^-s_t
  int on;                // 1: x is staged as FP16
};

// Exponent field range of the nonzero BF16 values in four words (eight values).
__device__ __forceinline__ void bf16_exp_range(const uint4 v, int& emax, int& emin) {
  const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const unsigned b = (w[i] >> (16 * h)) & 0xffffu;
      const int e = static_cast<int>((b >> 7) & 0xffu);
      emax = max(emax, e);
      emin = min(emin, (b & 0x7fffu) ? e : 255);
    }
  }
}

// Eight BF16 values times 2^s (exact by the staging rule) as eight FP16 values.
__device__ __forceinline__ uint4 bf16x8_to_f16x8_scaled(const uint4 v, float scale) {
  const unsigned w[4] = {v.x, v.y, v.z, v.w};
  unsigned o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = mul_rn(__uint_as_float(w[i] << 16), scale);
    const float hi = mul_rn(__uint_as_float(w[i] & 0xffff0000u), scale);
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(o[i]) : "f"(hi), "f"(lo));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// x staging with a fused elementwise op (16-bit staging, K % 8 == 0): each
// 16-byte unit (8 values = 4 pairs) of token t is computed from the op's inputs.
template <int F, int MT>
__device__ void stage_x_prologue(const GemvParams& p, int tile, unsigned char* xs, int segs) {
  constexpr int VALS = WTraits<F>::VALS;
  constexpr int NV = XLayout<F, XM_SMEM16>::NV;
  __shared__ float red[8];
  __shared__ float s_inv[MT];
  const Prologue& pr = p.pro;
  const int kpad = segs * 32 * VALS;
  const int upt = kpad / 8;
  if (pr.op == PRO_ADD_RMSNORM) {
    for (int t = 0; t < MT; ++t) {
      const int token = tile * MT + t;
      if (token >= p.m) break;  // uniform
      const unsigned* res2 = static_cast<const unsigned*>(pr.a) + static_cast<long long>(token) * (pr.ld / 2);
      const unsigned* y2 = static_cast<const unsigned*>(pr.b) + static_cast<long long>(token) * (pr.ld / 2);
      unsigned* x2 = blockIdx.x == 0 && pr.x_out
                         ? static_cast<unsigned*>(pr.x_out) + static_cast<long long>(token) * (pr.x_out_ld / 2)
                         : nullptr;
      const float inv = add_rmsnorm_inv(res2, y2, x2, p.k, pr.eps, red);
      if (threadIdx.x == 0) s_inv[t] = inv;
      __syncthreads();  // red is free again; s_inv[t] is visible
    }
  }
  for (int u = threadIdx.x; u < MT * upt; u += blockDim.x) {
    const int t = u / upt;
    const int col0 = (u - t * upt) * 8;
    const int token = tile * MT + t;
    unsigned v[4] = {0u, 0u, 0u, 0u};
    if (token < p.m && col0 < p.k) {
      const long long row = static_cast<long long>(token) * (pr.ld / 2);
      const int i0 = col0 / 2;
      if (pr.op == PRO_ADD_RMSNORM) {
        const unsigned* res2 = static_cast<const unsigned*>(pr.a) + row;
        const unsigned* y2 = static_cast<const unsigned*>(pr.b) + row;
        const unsigned* w2 = static_cast<const unsigned*>(pr.w);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          v[e] = add_rmsnorm_pair(__ldg(res2 + i0 + e), __ldg(y2 + i0 + e), __ldg(w2 + i0 + e), s_inv[t]);
      } else {
        const unsigned* g2 = static_cast<const unsigned*>(pr.a) + row;
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = silu_mul_pair(__ldg(g2 + i0 + e), __ldg(g2 + p.k / 2 + i0 + e));
      }
    }
    const int g = col0 / (32 * VALS);
    const int r = col0 - g * 32 * VALS;
    const int l = r / VALS;
    const int i = (r - l * VALS) / 8;
    *reinterpret_cast<uint4*>(xs + ((((t * segs + g) * NV + i) * 32 + l) << 4)) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

template <int F, int X, int XM, int MT>
__device__ void stage_x(const GemvParams& p, int tile, unsigned char* xs, int segs, XHalfState* xh) {
  constexpr bool HALF = HalfX<F, X, XM>::value;
  if constexpr (XM == XM_SMEM16 && X == X_BF16 && !HALF) {
    if (p.pro.op != PRO_NONE) {
      stage_x_prologue<F, MT>(p, tile, xs, segs);
      return;
    }
  }
  constexpr int VALS = WTraits<F>::VALS;
  constexpr int EB = XLayout<F, XM>::EB;
  constexpr int PER = 16 / EB;  // values per 16-byte unit
  constexpr int NV = XLayout<F, XM>::NV;
  const int kpad = segs * 32 * VALS;
  const int units = MT * kpad / PER;
  const int upt = kpad / PER;  // units per token
  // Aligned rows: one 16-byte (or 8-byte for 16-bit x staged as FP32) L2 load per
  // unit, a batch of them in flight per thread before the first store. Every CTA
  // reads the same few lines, so per-element loads would multiply the L2 requests
  // on them by the vector width; this staging sits on every launch's critical path.
  constexpr int XBYTES = (X == X_F32) ? 4 : 2;
  constexpr int LBYTES = PER * XBYTES;  // global bytes per unit: 16 or 8
  static_assert(LBYTES == 16 || LBYTES == 8, "16-bit staging takes 16-bit x only");
  if ((p.k % PER) == 0 && (p.ldx % PER) == 0 && (reinterpret_cast<uintptr_t>(p.x) % LBYTES) == 0) {
    constexpr int B = 4;
    for (int u0 = threadIdx.x; u0 < units; u0 += B * blockDim.x) {
      uint4 v[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int u = u0 + b * blockDim.x;
        v[b] = make_uint4(0u, 0u, 0u, 0u);
        if (u < units) {
          const int t = u / upt;
          const int col0 = (u - t * upt) * PER;
          const int token = tile * MT + t;
          if (token < p.m && col0 < p.k) {
            const char* src = static_cast<const char*>(p.x) +
                              (static_cast<long long>(token) * p.ldx + col0) * XBYTES;
            if constexpr (LBYTES == 16) {
              v[b] = __ldcg(reinterpret_cast<const uint4*>(src));
            } else {
              const uint2 h = __ldcg(reinterpret_cast<const uint2*>(src));
              v[b] = make_uint4(h.x, h.y, 0u, 0u);
            }
          }
        }
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int u = u0 + b * blockDim.x;
        if (u >= units) break;
        const int t = u / upt;
        const int col0 = (u - t * upt) * PER;
        const int g = col0 / (32 * VALS);
        const int r = col0 - g * 32 * VALS;
        const int l = r / VALS;
        const int i = (r - l * VALS) / PER;
        unsigned char* dst = xs + ((((t * segs + g) * NV + i) * 32 + l) << 4);
        uint4 s = v[b];
        if constexpr (HALF && X == X_BF16) {
          // Units of one batch step of a warp belong to one token (units per
          // token is a multiple of 32), so the warp reduces before one atomic.
          int emax = 0, emin = 255;
          bf16_exp_range(v[b], emax, emin);
          emax = __reduce_max_sync(0xffffffffu, emax);
          emin = __reduce_min_sync(0xffffffffu, emin);
          if ((threadIdx.x & 31) == 0) {
            atomicMax(&xh->emax[t], emax);
            atomicMin(&xh->emin[t], emin);
          }
        }
        if constexpr (EB == 4 && X != X_F32) {
          // Four 16-bit values widened to FP32.
          const unsigned lo = v[b].x, hi = v[b].y;
          if constexpr (X == X_BF16)
            s = make_uint4(lo << 16, lo & 0xffff0000u, hi << 16, hi & 0xffff0000u);
          else
            s = make_uint4(__float_as_uint(f16lo(lo)), __float_as_uint(f16hi(lo)), __float_as_uint(f16lo(hi)),
                           __float_as_uint(f16hi(hi)));
        }
        *reinterpret_cast<uint4*>(dst) = s;
      }
    }
    if constexpr (HALF && X == X_BF16) {
      __syncthreads();
      bool fast = true;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int emax = xh->emax[t], emin = xh->emin[t];
        fast = fast && (emin == 255 || (emax <= 200 && emin >= 39 && emax - emin <= 32));
      }
      if (fast) {
        for (int u = threadIdx.x; u < units; u += blockDim.x) {
          const int t = u / upt;
          const int col0 = (u - t * upt) * PER;
          const int g = col0 / (32 * VALS);
          const int r = col0 - g * 32 * VALS;
          const int l = r / VALS;
          const int i = (r - l * VALS) / PER;
          uint4* dst = reinterpret_cast<uint4*>(xs + ((((t * segs + g) * NV + i) * 32 + l) << 4));
          const float scale = xh->emin[t] == 255 ? 1.0f : __int_as_float((269 - xh->emax[t]) << 23);  // 2^s_t
          *dst = bf16x8_to_f16x8_scaled(*dst, scale);
        }
      }
      if (threadIdx.x == 0) {
        xh->on = fast ? 1 : 0;
        for (int t = 0; t < MT; ++t)  // 2^-s_t
          xh->inv[t] = (!fast || xh->emin[t] == 255) ? 1.0f : __int_as_float((xh->emax[t] - 15) << 23);
      }
    } else if constexpr (HALF) {
      if (threadIdx.x == 0) {
        xh->on = 1;
        for (int t = 0; t < MT; ++t) xh->inv[t] = 1.0f;
      }
    }
    return;
  }
  if constexpr (HALF) {
    // Unaligned rows keep the staged 16-bit values as they are: FP16 x runs the
    // FP16 path unscaled, BF16 x the FP32 path.
    if (threadIdx.x == 0) {
      xh->on = (X == X_F16) ? 1 : 0;
      for (int t = 0; t < MT; ++t) xh->inv[t] = 1.0f;
    }
  }
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int t = u / (kpad / PER);
    const int col0 = (u - t * (kpad / PER)) * PER;  // first column of this unit
    const int token = tile * MT + t;
    const int g = col0 / (32 * VALS);
    const int r = col0 - g * 32 * VALS;
    const int l = r / VALS;
    const int i = (r - l * VALS) / PER;
    unsigned char* dst = xs + ((((t * segs + g) * NV + i) * 32 + l) << 4);
    if constexpr (EB == 4) {
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = col0 + e;
        v[e] = (token < p.m && col < p.k) ? x_value<X>(p.x, static_cast<long long>(token) * p.ldx + col) : 0.0f;
      }
      *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      unsigned short v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int col = col0 + e;
        v[e] = (token < p.m && col < p.k)
                   ? __ldcg(static_cast<const unsigned short*>(p.x) + static_cast<long long>(token) * p.ldx + col)
                   : static_cast<unsigned short>(0);
      }
      *reinterpret_cast<uint4*>(dst) =
          make_uint4(v[0] | (unsigned(v[1]) << 16), v[2] | (unsigned(v[3]) << 16), v[4] | (unsigned(v[5]) << 16),
                     v[6] | (unsigned(v[7]) << 16));
    }
  }
}

// The lane's VALS activations of one token and segment, widened to FP32.
// XM_SMEM / XM_SMEM16: `addr` is the shared address of the lane's first vector;
// XM_GLOBAL: `src` points at the lane's first value in global memory (16-byte
// aligned, K % VALS == 0 guaranteed by the host).
template <int F, int X, int XM>
__device__ __forceinline__ void load_x(unsigned addr, const void* src, float (&xv)[WTraits<F>::VALS]) {
  constexpr int VALS = WTraits<F>::VALS;
  if constexpr (XM == XM_SMEM) {
#pragma unroll
    for (int i = 0; i < VALS / 4; ++i) {
      uint4 v = lds128(addr + i * 512);
      xv[4 * i + 0] = __uint_as_float(v.x);
      xv[4 * i + 1] = __uint_as_float(v.y);
      xv[4 * i + 2] = __uint_as_float(v.z);
      xv[4 * i + 3] = __uint_as_float(v.w);
    }
  } else {
    constexpr int XB = (X == X_F32) ? 4 : 2;
#pragma unroll
    for (int i = 0; i < VALS * XB / 16; ++i) {
      uint4 v;
      if constexpr (XM == XM_SMEM16)
        v = lds128(addr + i * 512);
      else
        v = ldg128_cached(static_cast<const char*>(src) + 16 * i);
      const unsigned q[4] = {v.x, v.y, v.z, v.w};
      if constexpr (X == X_F32) {
#pragma unroll
        for (int e = 0; e < 4; ++e) xv[4 * i + e] = __uint_as_float(q[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xv[8 * i + 2 * e] = (X == X_BF16) ? bf16lo(q[e]) : f16lo(q[e]);
          xv[8 * i + 2 * e + 1] = (X == X_BF16) ? bf16hi(q[e]) : f16hi(q[e]);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ decode

// Lossless BF16 codec v1 (docs/bf16-format.md): 12-bit code -> FP32 bits.
// `base` is metadata & 0x7f800000 (the block base exponent at FP32 bits 23..30).
__device__ __forceinline__ float cbf16_code(unsigned code, unsigned base) {
  return __uint_as_float(((code & 0x7fu) << 16) | ((code & 0x80u) << 24) |
                         (base + ((code & 0xf00u) << 15)));
}

// Weights of lane `lane`, segment j of the item in `slot` (shared address).
// Fixed-size formats read the lane's 16 bytes at slot + (32*j + lane)*16.
template <int F>
__device__ __forceinline__ void load_w(unsigned slot, unsigned meta_entry, unsigned first_unit,
                                       int j, int lane, float (&w)[WTraits<F>::VALS]) {
  if constexpr (F == W_BF16) {
    uint4 v = lds128(slot + (j * 32 + lane) * 16);
    unsigned q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w[2 * i] = bf16lo(q[i]);
      w[2 * i + 1] = bf16hi(q[i]);
    }
  } else if constexpr (F == W_F16) {
    uint4 v = lds128(slot + (j * 32 + lane) * 16);
    unsigned q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w[2 * i] = f16lo(q[i]);
      w[2 * i + 1] = f16hi(q[i]);
    }
  } else if constexpr (F == W_F32 || F == W_LF32 || F == W_FP28) {
    uint4 v = lds128(slot + (j * 32 + lane) * 16);
    w[0] = __uint_as_float(v.x);
    w[1] = __uint_as_float(v.y);
    w[2] = __uint_as_float(v.z);
    w[3] = __uint_as_float(v.w);
  } else if constexpr (F == W_CBF16) {
    const int block = 4 * j + (lane >> 3);
    const int q8 = lane & 7;
    const unsigned meta = lds32(meta_entry + 4 * block);
    const unsigned off = slot + (((meta & 0x7fffffu) - first_unit) << 5);
    if (meta >> 31) {
      uint4 v = lds128(off + 16 * q8);
      unsigned q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w[2 * i] = bf16lo(q[i]);
        w[2 * i + 1] = bf16hi(q[i]);
      }
    } else {
      const unsigned a = lds32(off + 12 * q8), b = lds32(off + 12 * q8 + 4),
                     c = lds32(off + 12 * q8 + 8);
      const unsigned base = meta & 0x7f800000u;
      w[0] = cbf16_code(a, base);
      w[1] = cbf16_code(a >> 12, base);
      w[2] = cbf16_code((a >> 24) | (b << 8), base);
      w[3] = cbf16_code(b >> 4, base);
      w[4] = cbf16_code(b >> 16, base);
      w[5] = cbf16_code((b >> 28) | (c << 4), base);
      w[6] = cbf16_code(c >> 8, base);
      w[7] = cbf16_code(c >> 20, base);
    }
  } else if constexpr (F == W_I8_ROW || F == W_I8_G64) {
    // Signed int8 -> FP32 exactly: bytes biased by 128 become the low mantissa
    // byte of 2^23 + u, and the bias is subtracted in FP32 (exact).
    uint4 v = lds128(slot + (j * 32 + lane) * 16);
    unsigned q[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int b = 0; b < 4; b += 2) {
        const f2 u{__uint_as_float(__byte_perm(q[i], 0x4b000000u, 0x7540u + b)),
                   __uint_as_float(__byte_perm(q[i], 0x4b000000u, 0x7541u + b))};
        const f2 v = add2(u, f2{-8388736.0f, -8388736.0f});
        w[4 * i + b] = v.x;
        w[4 * i + b + 1] = v.y;
      }
    }
  } else {
    // E2M1 pairs: low nibble = even column (fp4.py:59).
    uint4 v = lds128(slot + (j * 32 + lane) * 16);
    unsigned q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const unsigned h = e2m1x2_to_f16x2((q[i] >> (8 * b)) & 0xffu);
        w[8 * i + 2 * b] = f16lo(h);
        w[8 * i + 2 * b + 1] = f16hi(h);
      }
    }
  }
}

// Two codec-v1 codes, the low one in bits 0-11 and the high one in bits 16-27
// (bits 12-15 and 28-31 ignored) -> two BF16 values, exactly the upper halves of
// cbf16_code's FP32 bits; base2 holds the block's exponent base at BF16 bits 7-14
// of both halves.
__device__ __forceinline__ unsigned cbf16_pair(unsigned p, unsigned base2) {
  return (p & 0x007f007fu) | ((p << 8) & 0x80008000u) | (base2 + ((p >> 1) & 0x07800780u));
}

// The lane's eight 16-bit weights of segment j as four pairs (value 2i in the low
// half of word i): raw 16-bit formats read them, coded BF16 decodes a coded block
// two codes at a time.
template <int F>
__device__ __forceinline__ uint4 load_w16(unsigned slot, unsigned meta_entry, unsigned first_unit, int j, int lane) {
  if constexpr (F == W_CBF16) {
    const int block = 4 * j + (lane >> 3);
    const int q8 = lane & 7;
    const unsigned meta = lds32(meta_entry + 4 * block);
    const unsigned off = slot + (((meta & 0x7fffffu) - first_unit) << 5);
    if (meta >> 31) return lds128(off + 16 * q8);
    const unsigned a = lds32(off + 12 * q8), b = lds32(off + 12 * q8 + 4), c = lds32(off + 12 * q8 + 8);
    const unsigned base2 = ((meta & 0x7f800000u) >> 16) * 0x00010001u;
    const unsigned p01 = __byte_perm(a, a << 4, 0x7610u);
    const unsigned p23 = __byte_perm(__funnelshift_r(a, b, 24), b << 12, 0x7610u);
    const unsigned p45 = __byte_perm(b >> 16, __funnelshift_r(b, c, 12), 0x7610u);
    const unsigned p67 = __byte_perm(c >> 8, c >> 4, 0x7610u);
    return make_uint4(cbf16_pair(p01, base2), cbf16_pair(p23, base2), cbf16_pair(p45, base2),
                      cbf16_pair(p67, base2));
  } else {
    return lds128(slot + (j * 32 + lane) * 16);
  }
}

// ------------------------------------------------------------------ item math

#ifndef KLAB_MIXED_BF16
#define KLAB_MIXED_BF16 1
#endif

// acc = x * w + acc with BF16 (or FP16) x and w taken from the low or high half
// of a 32-bit word: the product is exact in FP32 and the sum is rounded once,
// exactly like widening both to FP32 and using fma.rn.f32.
template <bool HI, bool F16>
__device__ __forceinline__ float fma_half_mixed(unsigned x2, unsigned w2, float acc) {
  float d;
  if constexpr (F16) {
    if constexpr (HI)
      asm("{\n .reg .b16 xl, xh, wl, wh;\n mov.b32 {xl, xh}, %1;\n mov.b32 {wl, wh}, %2;\n"
          " fma.rn.f32.f16 %0, xh, wh, %3;\n}\n" : "=f"(d) : "r"(x2), "r"(w2), "f"(acc));
    else
      asm("{\n .reg .b16 xl, xh, wl, wh;\n mov.b32 {xl, xh}, %1;\n mov.b32 {wl, wh}, %2;\n"
          " fma.rn.f32.f16 %0, xl, wl, %3;\n}\n" : "=f"(d) : "r"(x2), "r"(w2), "f"(acc));
  } else {
    if constexpr (HI)
      asm("{\n .reg .b16 xl, xh, wl, wh;\n mov.b32 {xl, xh}, %1;\n mov.b32 {wl, wh}, %2;\n"
          " fma.rn.f32.bf16 %0, xh, wh, %3;\n}\n" : "=f"(d) : "r"(x2), "r"(w2), "f"(acc));
    else
      asm("{\n .reg .b16 xl, xh, wl, wh;\n mov.b32 {xl, xh}, %1;\n mov.b32 {wl, wh}, %2;\n"
          " fma.rn.f32.bf16 %0, xl, wl, %3;\n}\n" : "=f"(d) : "r"(x2), "r"(w2), "f"(acc));
  }
  return d;
}

// True when a (weight format, x mode) pair multiplies 16-bit operands directly.
template <int F, int XM>
struct MixedPath {
  static constexpr bool value = KLAB_MIXED_BF16 && (F == W_BF16 || F == W_F16 || F == W_CBF16) && XM == XM_SMEM16;
};

// Lane accumulators of one token: eight FP32 sums held as four pairs. Value v
// of a lane's vector goes to sum (v % 8): pair (v / 2) % 4, half v % 2.
struct Acc8 {
  f2 a[4];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = f2{0.0f, 0.0f};
  }
  // ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7))
  __device__ __forceinline__ float tree() const {
    return add_rn(add_rn(add_rn(a[0].x, a[0].y), add_rn(a[1].x, a[1].y)),
                  add_rn(add_rn(a[2].x, a[2].y), add_rn(a[3].x, a[3].y)));
  }
};

// Chunk partial of every token of the tile (the same value in every lane).
// FULL: the chunk has all KC columns (no bounds checks). xs_lane: shared address
// of token 0's first x vector for this lane and chunk (XM_SMEM*); xg: pointer to
// token 0's first value for this lane and chunk (XM_GLOBAL).
template <int F, int X, int XM, int MT, bool FULL>
__device__ __forceinline__ void compute_item(unsigned slot, unsigned meta_entry, unsigned first_unit, int lane,
                                             int L, unsigned xs_lane, int tok_stride, const char* xg,
                                             long long xg_stride, int tvalid, float (&P)[MT]) {
  constexpr int VALS = WTraits<F>::VALS;
  constexpr bool SCALED = (F == W_I8_G64 || F == W_FP4_G32H || F == W_FP4_G16E);
  constexpr bool MIXED = MixedPath<F, XM>::value;
  constexpr int SEG = XLayout<F, XM>::SEG_BYTES;
  constexpr int XB = (X == X_F32) ? 4 : 2;
  Acc8 acc8[MT];
  float acc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    acc8[t].zero();
    acc[t] = 0.0f;
  }
  // Full unrolling of the segment loop pays for one or two tokens; wider tiles
  // would exceed the register budget.
  constexpr int UNROLL = MT <= 2 ? kSegUnroll : (kSegUnroll < 2 ? kSegUnroll : 2);
#pragma unroll(UNROLL)
  for (int j = 0; j < kSegs; ++j) {
    if (!FULL) {
      if (32 * VALS * j >= L) break;
      if ((32 * j + lane) * VALS >= L) continue;
    }
    const unsigned xs_seg = xs_lane + j * SEG;
    const char* xg_seg = xg + static_cast<long long>(32 * VALS * j) * XB;
    if constexpr (MIXED) {
      const uint4 wv = load_w16<F>(slot, meta_entry, first_unit, j, lane);
      const unsigned wq[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const uint4 xv = lds128(xs_seg + t * tok_stride);
        const unsigned xq[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc8[t].a[i].x = fma_half_mixed<false, F == W_F16>(xq[i], wq[i], acc8[t].a[i].x);
          acc8[t].a[i].y = fma_half_mixed<true, F == W_F16>(xq[i], wq[i], acc8[t].a[i].y);
        }
      }
    } else {
      float w[VALS];
      load_w<F>(slot, meta_entry, first_unit, j, lane, w);
      float s0 = 1.0f, s1 = 1.0f;
      if constexpr (F == W_I8_G64) {
        s0 = __uint_as_float(lds32(slot + kWeightSlot + 4 * (8 * j + (lane >> 2))));
      } else if constexpr (F == W_FP4_G32H) {
        s0 = f16_to_f32(lds16(slot + kWeightSlot + 2 * (32 * j + lane)));
      } else if constexpr (F == W_FP4_G16E) {
        const unsigned h = e4m3x2_to_f16x2(lds16(slot + kWeightSlot + 64 * j + 2 * lane));
        s0 = f16lo(h);
        s1 = f16hi(h);
      }
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        float xv[VALS];
        // Global mode: tokens past M (ragged last tile) re-read the last valid
        // token; their sums are never stored.
        load_x<F, X, XM>(xs_seg + t * tok_stride, xg_seg + min(t, tvalid - 1) * xg_stride, xv);
        if constexpr (!SCALED) {
#pragma unroll
          for (int v = 0; v < VALS; v += 2) {
            f2& a = acc8[t].a[(v >> 1) & 3];
            a = fma2(f2{xv[v], xv[v + 1]}, f2{w[v], w[v + 1]}, a);
          }
        } else {
          constexpr int GROUP = (F == W_FP4_G16E) ? 16 : VALS;
#pragma unroll
          for (int g0 = 0; g0 < VALS; g0 += GROUP) {
            Acc8 sub;
            sub.zero();
#pragma unroll
            for (int v = g0; v < g0 + GROUP; v += 2) {
              f2& a = sub.a[(v >> 1) & 3];
              a = fma2(f2{xv[v], xv[v + 1]}, f2{w[v], w[v + 1]}, a);
            }
            acc[t] = fma_rn(sub.tree(), g0 == 0 ? s0 : s1, acc[t]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) P[t] = warp_allsum(SCALED ? acc[t] : acc8[t].tree());
}

// Four signed int8 codes (one word) -> two FP16 pairs, exactly: bytes biased by
// 128 become the low mantissa byte of 1024 + u, and 1152 is subtracted in FP16.
__device__ __forceinline__ void int8x4_to_f16x4(unsigned q, unsigned& h01, unsigned& h23) {
  const unsigned u = q ^ 0x80808080u;
  const unsigned a = __byte_perm(u, 0x64646464u, 0x4140u), b = __byte_perm(u, 0x64646464u, 0x4342u);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(h01) : "r"(a), "r"(0x64806480u));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(h23) : "r"(b), "r"(0x64806480u));
}

// compute_item for HalfX formats with x staged as FP16: the same values, sums and
// order as compute_item, each product a mixed fma.rn.f32.f16 on the raw pairs.
template <int F, int MT, bool FULL>
__device__ __forceinline__ void compute_item_h(unsigned slot, int lane, int L, unsigned xs_lane, int tok_stride,
                                               float (&P)[MT]) {
  constexpr int VALS = WTraits<F>::VALS;
  constexpr bool SCALED = (F == W_FP4_G32H || F == W_FP4_G16E);
  constexpr int SEG = XLayout<F, XM_SMEM16>::SEG_BYTES;
  constexpr int WORDS = VALS / 2;  // FP16 pairs per lane and segment
  Acc8 acc8[MT];
  float acc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    acc8[t].zero();
    acc[t] = 0.0f;
  }
  constexpr int UNROLL = MT <= 2 ? kSegUnroll : (kSegUnroll < 2 ? kSegUnroll : 2);
#pragma unroll(UNROLL)
  for (int j = 0; j < kSegs; ++j) {
    if (!FULL) {
      if (32 * VALS * j >= L) break;
      if ((32 * j + lane) * VALS >= L) continue;
    }
    const unsigned xs_seg = xs_lane + j * SEG;
    const uint4 wv = lds128(slot + (j * 32 + lane) * 16);
    const unsigned q[4] = {wv.x, wv.y, wv.z, wv.w};
    unsigned wh[WORDS];  // pair i: values 2i, 2i + 1
    if constexpr (F == W_I8_ROW) {
#pragma unroll
      for (int i = 0; i < 4; ++i) int8x4_to_f16x4(q[i], wh[2 * i], wh[2 * i + 1]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int b = 0; b < 4; ++b) wh[4 * i + b] = e2m1x2_to_f16x2((q[i] >> (8 * b)) & 0xffu);
    }
    float s0 = 1.0f, s1 = 1.0f;
    if constexpr (F == W_FP4_G32H) {
      s0 = f16_to_f32(lds16(slot + kWeightSlot + 2 * (32 * j + lane)));
    } else if constexpr (F == W_FP4_G16E) {
      const unsigned h = e4m3x2_to_f16x2(lds16(slot + kWeightSlot + 64 * j + 2 * lane));
      s0 = f16lo(h);
      s1 = f16hi(h);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      unsigned xq[WORDS];
#pragma unroll
      for (int i = 0; i < WORDS / 4; ++i) {
        const uint4 v = lds128(xs_seg + t * tok_stride + i * 512);
        xq[4 * i] = v.x;
        xq[4 * i + 1] = v.y;
        xq[4 * i + 2] = v.z;
        xq[4 * i + 3] = v.w;
      }
      if constexpr (!SCALED) {
#pragma unroll
        for (int i = 0; i < WORDS; ++i) {
          f2& a = acc8[t].a[i & 3];
          a.x = fma_half_mixed<false, true>(xq[i], wh[i], a.x);
          a.y = fma_half_mixed<true, true>(xq[i], wh[i], a.y);
        }
      } else {
        constexpr int GW = ((F == W_FP4_G16E) ? 16 : VALS) / 2;  // pairs per scale group
#pragma unroll
        for (int g0 = 0; g0 < WORDS; g0 += GW) {
          Acc8 sub;
          sub.zero();
#pragma unroll
          for (int i = g0; i < g0 + GW; ++i) {
            f2& a = sub.a[i & 3];
            a.x = fma_half_mixed<false, true>(xq[i], wh[i], a.x);
            a.y = fma_half_mixed<true, true>(xq[i], wh[i], a.y);
          }
          acc[t] = fma_rn(sub.tree(), g0 == 0 ? s0 : s1, acc[t]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) P[t] = warp_allsum(SCALED ? acc[t] : acc8[t].tree());
}

// ------------------------------------------------------------------ filling

template <int F>
__device__ __forceinline__ long long w_offset_bytes(long long elem) {
  return elem * WTraits<F>::NUM / WTraits<F>::DEN;
}

// Scale bytes of (row, chunk c) covering L columns; source pointer and byte count.
template <int F>
__device__ __forceinline__ void scale_span(const RowRef& r, int k, int c, int L, const char** src, int* bytes) {
  constexpr int KC = Layout<F>::KC;
  if constexpr (F == W_I8_G64) {
    *src = r.aux + (static_cast<long long>(r.local) * (k / 64) + c * (KC / 64)) * 4;
    *bytes = (L / 64) * 4;
  } else if constexpr (F == W_FP4_G32H) {
    *src = r.aux + (static_cast<long long>(r.local) * (k / 32) + c * (KC / 32)) * 2;
    *bytes = (L / 32) * 2;
  } else if constexpr (F == W_FP4_G16E) {
    *src = r.aux + (static_cast<long long>(r.local) * (k / 16) + c * (KC / 16));
    *bytes = L / 16;
  } else {
    *src = nullptr;
    *bytes = 0;
  }
}

// Cooperative (non-bulk) fill of one slot by the whole warp, any alignment.
// Bytes past the item's data are zero so padded lanes contribute exact zeros.
__device__ __forceinline__ void warp_copy_bytes(char* dst, const char* src, int bytes, int cap,
                                                int lane) {
  if ((reinterpret_cast<uintptr_t>(src) & 3) == 0 && (bytes & 3) == 0) {
    const unsigned* s = reinterpret_cast<const unsigned*>(src);
    unsigned* d = reinterpret_cast<unsigned*>(dst);
    for (int i = lane; i < bytes / 4; i += 32) d[i] = __ldg(s + i);
  } else {
    for (int i = lane; i < bytes; i += 32) dst[i] = static_cast<char>(__ldg(reinterpret_cast<const unsigned char*>(src) + i));
  }
  for (int i = bytes + lane; i < cap; i += 32) dst[i] = 0;
}


// Fill of one slot with the exact FP32 values of a lossless-FP32 item: the
// item's L weights start at flat index local * k + c * KC of the row's matrix;
// lane l decodes weights 4l, 4l + 128, ... into the slot's natural order.
template <int F>
__device__ __forceinline__ void decode_f32_item(float* dst, const RowRef& r, int k, int c, int L, int lane) {
  const long long first = static_cast<long long>(r.local) * k + static_cast<long long>(c) * Layout<F>::KC;
  for (int i = lane * 4; i < L; i += 128) {
    float4 v;
    if constexpr (F == W_LF32)
      v = lf32_load4(reinterpret_cast<const unsigned char*>(r.w), reinterpret_cast<const unsigned char*>(r.aux2),
                     reinterpret_cast<const unsigned*>(r.aux), first + i);
    else
      v = fp28_load4(reinterpret_cast<const unsigned*>(r.w), reinterpret_cast<const unsigned*>(r.aux), first + i);
    *reinterpret_cast<float4*>(dst + i) = v;
  }
}

// ------------------------------------------------------------------ kernel

// (row, chunk) position in a warp's item sequence.
struct Cursor {
  int row, c;
  __device__ __forceinline__ void advance(int chunks, int row_step) {
    if (++c == chunks) {
      c = 0;
      row += row_step;
    }
  }
};

template <int F, int MT>
__device__ __forceinline__ void finalize_token(const GemvParams& p, const RowRef& r, int token, float v,
                                               float row_scale) {
  if constexpr (F == W_I8_ROW) v = mul_rn(v, row_scale);
  if constexpr (F == W_FP4_G16E) v = mul_rn(v, __ldg(p.gscale));
  const Segment& sg = p.seg[r.seg];
  const long long idx = static_cast<long long>(token) * sg.ldo + r.local;
  if (p.out_f32) {
    static_cast<float*>(sg.out)[idx] = v;
  } else {
    const unsigned short b = f32_to_bf16_rn(v);
    static_cast<unsigned short*>(sg.out)[idx] = b;
    if (r.seg == p.gather.seg) {
      // Fused all-gather: the same value into every other rank's copy (NVLink stores).
      for (int q = 0; q < p.gather.npeers; ++q)
        if (q != p.gather.rank) static_cast<unsigned short*>(p.gather.peer_out[q])[idx] = b;
    }
  }
}

// Grid (G, ceil(M / MT)); block warps_for(F, MT)*32. Dynamic shared memory:
// [mbarriers][kWarps warp regions: kDepth slots (+ metadata ring)][x staging].
template <int F, int X, int XM, int MT>
__global__ void __launch_bounds__(warps_for(F, MT) * 32, min_blocks_for(F, MT))
    stream_gemv_kernel(const GemvParams p) {
  constexpr int kWarps = warps_for(F, MT);
  constexpr int KC = Layout<F>::KC;
  constexpr int SLOT = Layout<F>::SLOT;
  constexpr int VALS = WTraits<F>::VALS;
  constexpr bool CODED = (F == W_CBF16);
  constexpr int BAR_REGION = ((kWarps * Layout<F>::BARS * 8 + 127) / 128) * 128;
  constexpr int XB = (X == X_F32) ? 4 : 2;
  extern __shared__ __align__(128) unsigned char smem[];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.y;
  const int S = p.chunks;
  const int n = p.n, k = p.k;
  const unsigned pbar0 = smem_addr(smem) + warp * Layout<F>::BARS * 8;
  const unsigned mbar0 = pbar0 + kDepth * 8;
  const unsigned slot0 = smem_addr(smem) + BAR_REGION + warp * Layout<F>::WARP_BYTES;
  const unsigned meta0 = slot0 + kDepth * SLOT;
  unsigned char* slot0_ptr = smem + BAR_REGION + warp * Layout<F>::WARP_BYTES;
  unsigned char* xs = smem + BAR_REGION + kWarps * Layout<F>::WARP_BYTES;
  const int segs = (k + 32 * VALS - 1) / (32 * VALS);

  // This warp's items, as (row, chunk) cursors that advance without division:
  // aligned mode deals whole rows round-robin (row step kWarps); split mode gives
  // each warp a contiguous run of items (row step 1).
  int nitems = 0, row_step = kWarps;
  Cursor start{0, 0};
  long long wbegin = 0, wend = 0;
  if (!p.split) {
    const int r0 = static_cast<int>(static_cast<long long>(n) * blockIdx.x / gridDim.x);
    const int r1 = static_cast<int>(static_cast<long long>(n) * (blockIdx.x + 1) / gridDim.x);
    const int rows = r1 - r0 - warp > 0 ? (r1 - r0 - warp + kWarps - 1) / kWarps : 0;
    nitems = rows * S;
    start = Cursor{r0 + warp, 0};
  } else {
    const long long T = static_cast<long long>(n) * S;
    const long long i0 = T * blockIdx.x / gridDim.x, i1 = T * (blockIdx.x + 1) / gridDim.x;
    wbegin = i0 + (i1 - i0) * warp / kWarps;
    wend = i0 + (i1 - i0) * (warp + 1) / kWarps;
    nitems = static_cast<int>(wend - wbegin);
    start = Cursor{static_cast<int>(wbegin / S), static_cast<int>(wbegin % S)};
    row_step = 1;
  }
  Cursor cur = start, iss = start, mcur = start;

  // lane 0: bulk copy of the metadata of item `ix` (coded) at cursor m.
  auto issue_meta = [&](int ix, const Cursor& m) {
    const int nb = min(32, k / 64 - 32 * m.c);
    const unsigned bar = mbar0 + (ix % kMetaRing) * 8;
    const RowRef r = resolve_row(p, m.row);
    const char* src = r.aux + (static_cast<long long>(r.local) * (k / 64) + 32 * m.c) * 4;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, nb * 4);
    bulk_g2s(meta0 + (ix % kMetaRing) * kMetaEntry, src, nb * 4, bar);
  };
  // lane 0: bulk copy of item `ix`'s weight bytes (+ scales) at cursor it.
  auto issue_item = [&](int ix, const Cursor& it) {
    const int L = min(KC, k - it.c * KC);
    const unsigned slot = slot0 + (ix % kDepth) * SLOT;
    const unsigned bar = pbar0 + (ix % kDepth) * 8;
    const char* src;
    int bytes;
    const char* ssrc = nullptr;
    int sbytes = 0;
    const RowRef r = resolve_row(p, it.row);
    if constexpr (CODED) {
      const unsigned entry = meta0 + (ix % kMetaRing) * kMetaEntry;
      const int nb = L / 64;
      const unsigned m0 = lds32(entry), ml = lds32(entry + 4 * (nb - 1));
      const unsigned off = (m0 & 0x7fffffu) << 5;
      const unsigned end = ((ml & 0x7fffffu) << 5) + ((ml >> 31) ? 128u : 96u);
      src = r.w + off;
      bytes = static_cast<int>(end - off);
    } else {
      src = r.w + w_offset_bytes<F>(static_cast<long long>(r.local) * k + it.c * KC);
      bytes = static_cast<int>(w_offset_bytes<F>(L));
      scale_span<F>(r, k, it.c, L, &ssrc, &sbytes);
    }
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, bytes + sbytes);
    bulk_g2s(slot, src, bytes, bar);
    if (sbytes) bulk_g2s(slot + kWeightSlot, ssrc, sbytes, bar);
  };
  // lane 0: L2 prefetch of the item at cursor it (uncoded formats).
  auto prefetch_item = [&](const Cursor& it) {
    const int L = min(KC, k - it.c * KC);
    const RowRef r = resolve_row(p, it.row);
    const char* ssrc = nullptr;
    int sbytes = 0;
    bulk_prefetch_l2(r.w + w_offset_bytes<F>(static_cast<long long>(r.local) * k + it.c * KC),
                     static_cast<unsigned>(w_offset_bytes<F>(L)));
    scale_span<F>(r, k, it.c, L, &ssrc, &sbytes);
    if (sbytes) bulk_prefetch_l2(ssrc, static_cast<unsigned>(sbytes));
  };

  bool ok = true;
  int issued_meta = 0, issued = 0;  // lane 0 bookkeeping
  if (p.use_tma) {
    if (lane == 0) {
      for (int i = 0; i < Layout<F>::BARS; ++i) mbar_init(pbar0 + 8 * i, 1);
      fence_mbar_init();
    }
    __syncwarp();
    // Prologue: weights do not depend on the previous grid, so the first items
    // are copied (or prefetched into L2) before griddepcontrol.wait and stream
    // while the previous grid drains.
    const int pro = min(min(p.pro_smem, kDepth), nitems);
    if (lane == 0) {
      if constexpr (CODED) {
        for (; issued_meta < min(kMetaRing, nitems); ++issued_meta) {
          issue_meta(issued_meta, mcur);
          mcur.advance(S, row_step);
        }
        for (; issued < pro; ++issued) {
          if (!mbar_wait(mbar0 + (issued % kMetaRing) * 8, (issued / kMetaRing) & 1)) {
            ok = false;
            break;
          }
          issue_item(issued, iss);
          iss.advance(S, row_step);
        }
      } else {
        for (; issued < pro; ++issued) {
          issue_item(issued, iss);
          iss.advance(S, row_step);
        }
        Cursor pc = iss;
        for (int i = issued; i < min(issued + p.pro_l2, nitems); ++i) {
          prefetch_item(pc);
          pc.advance(S, row_step);
        }
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
  }

  grid_dependency_wait();
  if (p.gather.wait_flags && threadIdx.x < p.gather.npeers) {
    // x was gathered from the peers: wait until every rank's slice has landed.
    const unsigned target = *p.gather.epoch;
    if (!wait_flag_geq(p.gather.wait_flags + p.gather.wait_slot * p.gather.npeers + threadIdx.x, target))
      record_status(p.status, kStatusFlagTimeout);
  }
  __shared__ XHalfState s_xh;
  if (threadIdx.x < 8) {
    s_xh.emax[threadIdx.x] = 0;
    s_xh.emin[threadIdx.x] = 255;
  }
  __syncthreads();
  if constexpr (XM != XM_GLOBAL) stage_x<F, X, XM, MT>(p, tile, xs, segs, &s_xh);
  __syncthreads();
  constexpr bool HALF = HalfX<F, X, XM>::value;
  const bool xhalf = HALF && s_xh.on;
  grid_launch_dependents();
  if (p.use_tma && ok) {
    // Fill the rest of the ring; afterwards each consumed slot is refilled at once.
    if (lane == 0) {
      for (; issued < min(kDepth, nitems); ++issued) {
        if constexpr (CODED) {
          if (!mbar_wait(mbar0 + (issued % kMetaRing) * 8, (issued / kMetaRing) & 1)) {
            ok = false;
            break;
          }
        }
        issue_item(issued, iss);
        iss.advance(S, row_step);
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
  }

  constexpr int SEG = XLayout<F, XM>::SEG_BYTES;
  const int tok_stride = segs * SEG;
  const unsigned xs_lane0 = smem_addr(xs) + lane * 16;
  const char* xg_lane0 =
      static_cast<const char*>(p.x) + (static_cast<long long>(tile * MT) * p.ldx + lane * VALS) * XB;
  const long long xg_stride = static_cast<long long>(p.ldx) * XB;
  const int tvalid = min(MT, p.m - tile * MT);

  float rowsum[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) rowsum[t] = 0.0f;
  float row_scale = 1.0f;
  RowRef rref = resolve_row(p, cur.row);
  bool row_complete = true;
  int contributed = 0;

  int q = 0;
  for (; q < nitems && ok; ++q) {
    const int row = cur.row, c = cur.c;
    const int L = min(KC, k - c * KC);
    if (c == 0 || q == 0) rref = resolve_row(p, row);
    const unsigned slot = slot0 + (q % kDepth) * SLOT;
    const unsigned entry = meta0 + (q % kMetaRing) * kMetaEntry;
    if (p.use_tma) {
      const bool landed = mbar_wait(pbar0 + (q % kDepth) * 8, (q / kDepth) & 1);
      if (!__all_sync(0xffffffffu, landed)) {
        ok = false;
        break;
      }
    } else {
      // Cooperative fill: any alignment, zero padding past the item's data.
      unsigned char* sp = slot0_ptr + (q % kDepth) * SLOT;
      if constexpr (F == W_LF32 || F == W_FP28) {
        decode_f32_item<F>(reinterpret_cast<float*>(sp), rref, k, c, L, lane);
      } else if constexpr (CODED) {
        unsigned* ep = reinterpret_cast<unsigned*>(slot0_ptr + kDepth * SLOT + (q % kMetaRing) * kMetaEntry);
        const int nb = L / 64;
        if (lane < nb)
          ep[lane] = __ldg(reinterpret_cast<const unsigned*>(rref.aux) + static_cast<long long>(rref.local) * (k / 64) +
                           32 * c + lane);
        __syncwarp();
        const unsigned m0 = ep[0], ml = ep[nb - 1];
        const unsigned off = (m0 & 0x7fffffu) << 5;
        const unsigned end = ((ml & 0x7fffffu) << 5) + ((ml >> 31) ? 128u : 96u);
        warp_copy_bytes(reinterpret_cast<char*>(sp), rref.w + off, static_cast<int>(end - off), kWeightSlot, lane);
      } else {
        const char* src = rref.w + w_offset_bytes<F>(static_cast<long long>(rref.local) * k + c * KC);
        warp_copy_bytes(reinterpret_cast<char*>(sp), src, static_cast<int>(w_offset_bytes<F>(L)),
                        kWeightSlot, lane);
        if constexpr (WTraits<F>::SCALE_BYTES > 0) {
          const char* ssrc;
          int sbytes;
          scale_span<F>(rref, k, c, L, &ssrc, &sbytes);
          warp_copy_bytes(reinterpret_cast<char*>(sp) + kWeightSlot, ssrc, sbytes, WTraits<F>::SCALE_BYTES,
                          lane);
        }
      }
      __syncwarp();
    }

    if (c == 0 || q == 0) {
      if constexpr (F == W_I8_ROW) row_scale = __ldg(reinterpret_cast<const float*>(rref.aux) + rref.local);
      if (p.split)
        row_complete = static_cast<long long>(row) * S >= wbegin && static_cast<long long>(row) * S + S <= wend;
    }
    const unsigned first_unit = CODED ? (lds32(entry) & 0x7fffffu) : 0u;
    const unsigned xs_lane = xs_lane0 + c * kSegs * SEG;
    const char* xg = xg_lane0 + static_cast<long long>(c) * KC * XB;
    float P[MT];
    if (HALF && xhalf) {
      if constexpr (HALF) {
        if (L == KC)
          compute_item_h<F, MT, true>(slot, lane, L, xs_lane, tok_stride, P);
        else
          compute_item_h<F, MT, false>(slot, lane, L, xs_lane, tok_stride, P);
      }
    } else if (L == KC) {
      compute_item<F, X, XM, MT, true>(slot, entry, first_unit, lane, L, xs_lane, tok_stride, xg, xg_stride, tvalid,
                                       P);
    } else {
      compute_item<F, X, XM, MT, false>(slot, entry, first_unit, lane, L, xs_lane, tok_stride, xg, xg_stride,
                                        tvalid, P);
    }
    __syncwarp();  // every lane is done with this slot before it is refilled
    if (p.use_tma) {
      // Refill the slot just consumed with item q + kDepth (its metadata was
      // requested two items ago).
      if (lane == 0 && issued < nitems) {
        bool ready = true;
        if constexpr (CODED) ready = mbar_wait(mbar0 + (issued % kMetaRing) * 8, (issued / kMetaRing) & 1);
        if (ready) {
          issue_item(issued, iss);
          iss.advance(S, row_step);
          ++issued;
        } else {
          ok = false;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }

    if (row_complete) {
#pragma unroll
      for (int t = 0; t < MT; ++t) rowsum[t] = (c == 0) ? P[t] : add_rn(rowsum[t], P[t]);
      if (c == S - 1) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const int token = tile * MT + t;
          if (lane == t && token < p.m)
            finalize_token<F, MT>(p, rref, token, xhalf ? mul_rn(rowsum[t], s_xh.inv[t]) : rowsum[t], row_scale);
        }
      }
    } else {
      // Split-K: publish this chunk's partials; the last contributor of the row
      // folds all S partials in chunk order and resets the row's ticket.
#pragma unroll
      for (int t = 0; t < MT; ++t)
        if (lane == t) p.ws[((static_cast<long long>(tile) * MT + t) * n + row) * S + c] = P[t];
      ++contributed;
      if (c == S - 1 || q == nitems - 1) {
        __syncwarp();
        __threadfence();
        unsigned last = 0;
        unsigned* ticket = p.tickets + static_cast<long long>(tile) * n + row;
        if (lane == 0) {
          const unsigned old = atomicAdd(ticket, static_cast<unsigned>(contributed));
          last = (old + contributed == static_cast<unsigned>(S)) ? 1u : 0u;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        contributed = 0;
        if (last) {
          __threadfence();
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const int token = tile * MT + t;
            if (lane == t && token < p.m) {
              const float* src = p.ws + ((static_cast<long long>(tile) * MT + t) * n + row) * S;
              float total = __ldcg(src);
              for (int cc = 1; cc < S; ++cc) total = add_rn(total, __ldcg(src + cc));
              finalize_token<F, MT>(p, rref, token, xhalf ? mul_rn(total, s_xh.inv[t]) : total, row_scale);
            }
          }
          if (lane == 0) *ticket = 0u;
        }
      }
    }
    cur.advance(S, row_step);

    if constexpr (CODED) {
      if (p.use_tma && lane == 0 && issued_meta < nitems && issued_meta == q + kMetaRing) {
        issue_meta(issued_meta, mcur);
        mcur.advance(S, row_step);
        ++issued_meta;
      }
    }
  }

  if (p.gather.signal_slot >= 0) {
    // The CTA's peer stores reach thread 0 through the barrier; one system-scope
    // fence per CTA orders them before its count. The CTA that completes the
    // count fences again (acquiring the others' counts, releasing for the peers)
    // and raises this rank's flag on every rank.
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned total = gridDim.x * gridDim.y;
      fence_acq_rel_sys();
      if (atomicAdd(p.gather.done, 1u) == total - 1) {
        *p.gather.done = 0u;
        fence_acq_rel_sys();
        const unsigned epoch = *p.gather.epoch;
        for (int q = 0; q < p.gather.npeers; ++q)
          st_relaxed_sys(p.gather.peer_flags[q] + p.gather.signal_slot * p.gather.npeers + p.gather.rank, epoch);
      }
    }
  }

  if (!ok) {
    record_status(p.status, kStatusMbarTimeout);
    // Drain this warp's copies still in flight (each wait bounded) so no bulk
    // copy lands in shared memory after the CTA has exited.
    if (lane == 0 && p.use_tma) {
      for (int i = q; i < issued; ++i) mbar_wait(pbar0 + (i % kDepth) * 8, (i / kDepth) & 1);
      if constexpr (CODED)
        for (int i = issued; i < issued_meta; ++i)
          mbar_wait(mbar0 + (i % kMetaRing) * 8, (i / kMetaRing) & 1);
    }
  }
}

}  // namespace klab
