// Weight-streaming projection y[M,N] = x[M,K] . W[N,K]^T for M <= 8 per token tile.
//
// One template serves every weight format of the reference's projection path:
//   W_BF16    BF16 weights (compressed_kernels.cu raw, half_kernels.cu bf16)
//   W_F16     FP16 weights (half_kernels.cu f16)
//   W_F32     FP32 weights (kernels.cu gemv_*, projection_kernels.cu)
//   W_CBF16   lossless BF16 codec v1 (compressed_kernels.cu:38-106, docs/bf16-format.md)
//   W_I8_ROW  int8 + one fp32 scale per row
//   W_I8_G64  int8 + fp32 scale per 64 (int8_kernels.cu, int8_weights.py:23-35)
//   W_FP4_G32H E2M1 + fp16 scale per 32
//   W_FP4_G16E E2M1 + E4M3 scale per 16 + fp32 global (fp4_kernels.cu, fp4.py:33-60)
//
// Data movement (B200): every warp owns a private ring of DEPTH shared-memory
// slots filled by 1-D bulk copies (cp.async.bulk, no multicast) with mbarrier
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
//   * unscaled formats: per lane two FP32 chains (even v, odd v), fma.rn, run over
//     the chunk's segments in order; lane partial = even + odd;
//   * scaled formats: per lane and scale group the same two chains start at zero,
//     g = even + odd, then acc = fma.rn(g, scale, acc) in segment order;
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
};
enum XFmt : int { X_BF16 = 0, X_F16 = 1, X_F32 = 2 };
// Where x lives while the tile is computed.
enum XMode : int { XM_SMEM = 0, XM_GLOBAL = 1 };

#ifndef KLAB_WARPS
#define KLAB_WARPS 8
#endif
#ifndef KLAB_DEPTH
#define KLAB_DEPTH 3
#endif
#ifndef KLAB_SEG_UNROLL
#define KLAB_SEG_UNROLL 1
#endif
constexpr int kWarps = KLAB_WARPS;    // warps per CTA
constexpr int kDepth = KLAB_DEPTH;    // ring slots per warp
constexpr int kSegUnroll = KLAB_SEG_UNROLL;
constexpr int kSegs = 8;              // segments per chunk
constexpr int kWeightSlot = 4096;     // weight bytes per full chunk
constexpr int kMetaRing = 2 * kDepth - 1;  // coded: metadata entries per warp
constexpr int kMetaEntry = 128;       // 32 blocks * 4 bytes

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

template <int F>
struct Layout {
  static constexpr int VALS = WTraits<F>::VALS;
  static constexpr int KC = 32 * kSegs * VALS;
  static constexpr int SLOT = kWeightSlot + WTraits<F>::SCALE_BYTES;
  static constexpr int META = (F == W_CBF16) ? kMetaRing * kMetaEntry : 0;
  static constexpr int WARP_BYTES = kDepth * SLOT + META;
  static constexpr int BARS = kDepth + ((F == W_CBF16) ? kMetaRing : 0);
};

struct GemvParams {
  const void* x;        // [M, ldx] activations (X format)
  const void* w;        // weights, codes or coded payload
  const void* aux;      // coded metadata (u32) / scales
  const float* gscale;  // W_FP4_G16E global scale (device scalar)
  void* out;            // out[t * ldo + row]
  float* ws;            // split mode: partials [tiles*MT][N][S]
  unsigned* tickets;    // split mode: [tiles][N], zero between launches
  int* status;          // device status word
  int m, n, k;
  int ldx, ldo;
  int out_f32;
  int split;      // 0: rows dealt to CTAs; 1: items dealt to CTAs (split-K)
  int use_tma;    // 1: bulk copies; 0: cooperative loads (any alignment)
  int chunks;     // S = ceil(K / KC)
};

// ------------------------------------------------------------------ x staging

// x in shared memory is FP32 in a lane-interleaved layout: for token t, segment
// g (global, 32*VALS columns) and 16-byte vector i of a lane's VALS values, lane
// l's vector sits at ((t*G + g)*NV + i)*32 + l (16-byte units). A warp's
// ld.shared.v4 of vector i of one segment therefore touches 512 consecutive
// bytes: no bank conflicts. Columns >= K are zero.
template <int F>
struct XLayout {
  static constexpr int VALS = WTraits<F>::VALS;
  static constexpr int NV = VALS / 4;  // fp32 vectors per lane per segment
};

template <int X>
__device__ __forceinline__ float x_value(const void* x, long long idx) {
  if constexpr (X == X_BF16) {
    return __uint_as_float(static_cast<unsigned>(static_cast<const unsigned short*>(x)[idx]) << 16);
  } else if constexpr (X == X_F16) {
    return f16_to_f32(static_cast<const unsigned short*>(x)[idx]);
  } else {
    return static_cast<const float*>(x)[idx];
  }
}

template <int F, int X, int MT>
__device__ void stage_x(const GemvParams& p, int tile, float* xs, int kpad) {
  constexpr int VALS = WTraits<F>::VALS;
  constexpr int NV = VALS / 4;
  const int segs = kpad / (32 * VALS);
  const int total = MT * kpad;
  for (int e = threadIdx.x; e < total; e += blockDim.x) {
    const int t = e / kpad;
    const int col = e - t * kpad;
    const int token = tile * MT + t;
    float v = 0.0f;
    if (token < p.m && col < p.k) v = x_value<X>(p.x, static_cast<long long>(token) * p.ldx + col);
    const int g = col / (32 * VALS);
    const int r = col - g * 32 * VALS;
    const int l = r / VALS;
    const int vv = r - l * VALS;
    const int i = vv >> 2;
    xs[((((t * segs + g) * NV + i) * 32 + l) << 2) + (vv & 3)] = v;
  }
}

// The lane's VALS activation values (FP32) of token t at global segment g.
template <int F, int X, int XM>
__device__ __forceinline__ void load_x(const GemvParams& p, const float* xs, int segs, int t,
                                       int token, int g, int lane, int col,
                                       float (&xv)[WTraits<F>::VALS]) {
  constexpr int VALS = WTraits<F>::VALS;
  constexpr int NV = VALS / 4;
  if constexpr (XM == XM_SMEM) {
    const unsigned base = smem_addr(xs) + static_cast<unsigned>((((t * segs + g) * NV) * 32 + lane) * 16);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      uint4 v = lds128(base + i * 512);
      xv[4 * i + 0] = __uint_as_float(v.x);
      xv[4 * i + 1] = __uint_as_float(v.y);
      xv[4 * i + 2] = __uint_as_float(v.z);
      xv[4 * i + 3] = __uint_as_float(v.w);
    }
  } else {
    // Global (L1-cached) reads; the host guarantees 16-byte alignment and
    // K % VALS == 0 for this mode.
    const char* row = static_cast<const char*>(p.x);
    if constexpr (X == X_F32) {
      const float* src = reinterpret_cast<const float*>(row) + static_cast<long long>(token) * p.ldx + col;
#pragma unroll
      for (int i = 0; i < VALS / 4; ++i) {
        uint4 v = ldg128_cached(src + 4 * i);
        xv[4 * i + 0] = __uint_as_float(v.x);
        xv[4 * i + 1] = __uint_as_float(v.y);
        xv[4 * i + 2] = __uint_as_float(v.z);
        xv[4 * i + 3] = __uint_as_float(v.w);
      }
    } else {
      const unsigned short* src =
          reinterpret_cast<const unsigned short*>(row) + static_cast<long long>(token) * p.ldx + col;
#pragma unroll
      for (int i = 0; i < VALS / 8; ++i) {
        uint4 v = ldg128_cached(src + 8 * i);
        unsigned wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if constexpr (X == X_BF16) {
            xv[8 * i + 2 * q] = bf16lo(wv[q]);
            xv[8 * i + 2 * q + 1] = bf16hi(wv[q]);
          } else {
            xv[8 * i + 2 * q] = f16lo(wv[q]);
            xv[8 * i + 2 * q + 1] = f16hi(wv[q]);
          }
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
  } else if constexpr (F == W_F32) {
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
      for (int b = 0; b < 4; ++b) {
        const float f = __uint_as_float(__byte_perm(q[i], 0x4b000000u, 0x7540u + b));
        w[4 * i + b] = add_rn(f, -8388736.0f);
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

// ------------------------------------------------------------------ item math

// Chunk partial for each token of the tile (identical in every lane).
template <int F, int X, int XM, int MT>
__device__ __forceinline__ void compute_item(const GemvParams& p, const float* xs, int segs,
                                             int tile, int c, int L, unsigned slot,
                                             unsigned meta_entry, unsigned first_unit, int lane,
                                             float (&P)[MT]) {
  constexpr int VALS = WTraits<F>::VALS;
  constexpr int KC = Layout<F>::KC;
  constexpr bool SCALED = (F == W_I8_G64 || F == W_FP4_G32H || F == W_FP4_G16E);
  f2 chain[MT];
  float acc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    chain[t] = f2{0.0f, 0.0f};
    acc[t] = 0.0f;
  }
#pragma unroll(kSegUnroll)
  for (int j = 0; j < kSegs; ++j) {
    const int lcol = (32 * j + lane) * VALS;  // chunk-relative column of v = 0
    if (32 * VALS * j >= L) break;
    if (lcol < L) {
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
      const int g = (c * KC + 32 * VALS * j) / (32 * VALS);
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        // Tokens past M (ragged last tile) read row M-1; their sums are never stored.
        const int token = min(tile * MT + t, p.m - 1);
        float xv[VALS];
        load_x<F, X, XM>(p, xs, segs, t, token, g, lane, c * KC + lcol, xv);
        if constexpr (!SCALED) {
#pragma unroll
          for (int v = 0; v < VALS; v += 2)
            chain[t] = fma2(f2{xv[v], xv[v + 1]}, f2{w[v], w[v + 1]}, chain[t]);
        } else if constexpr (F == W_FP4_G16E) {
          f2 ga{0.0f, 0.0f}, gb{0.0f, 0.0f};
#pragma unroll
          for (int v = 0; v < 16; v += 2) ga = fma2(f2{xv[v], xv[v + 1]}, f2{w[v], w[v + 1]}, ga);
#pragma unroll
          for (int v = 16; v < 32; v += 2) gb = fma2(f2{xv[v], xv[v + 1]}, f2{w[v], w[v + 1]}, gb);
          acc[t] = fma_rn(add_rn(ga.x, ga.y), s0, acc[t]);
          acc[t] = fma_rn(add_rn(gb.x, gb.y), s1, acc[t]);
        } else {
          f2 ga{0.0f, 0.0f};
#pragma unroll
          for (int v = 0; v < VALS; v += 2) ga = fma2(f2{xv[v], xv[v + 1]}, f2{w[v], w[v + 1]}, ga);
          acc[t] = fma_rn(add_rn(ga.x, ga.y), s0, acc[t]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const float lane_partial = SCALED ? acc[t] : add_rn(chain[t].x, chain[t].y);
    P[t] = warp_allsum(lane_partial);
  }
}

// ------------------------------------------------------------------ filling

template <int F>
__device__ __forceinline__ long long w_offset_bytes(long long elem) {
  return elem * WTraits<F>::NUM / WTraits<F>::DEN;
}

// Scale bytes of (row, chunk c) covering L columns; source pointer and byte count.
template <int F>
__device__ __forceinline__ void scale_span(const GemvParams& p, int row, int c, int L,
                                           const char** src, int* bytes) {
  constexpr int KC = Layout<F>::KC;
  if constexpr (F == W_I8_G64) {
    *src = static_cast<const char*>(p.aux) + (static_cast<long long>(row) * (p.k / 64) + c * (KC / 64)) * 4;
    *bytes = (L / 64) * 4;
  } else if constexpr (F == W_FP4_G32H) {
    *src = static_cast<const char*>(p.aux) + (static_cast<long long>(row) * (p.k / 32) + c * (KC / 32)) * 2;
    *bytes = (L / 32) * 2;
  } else if constexpr (F == W_FP4_G16E) {
    *src = static_cast<const char*>(p.aux) + (static_cast<long long>(row) * (p.k / 16) + c * (KC / 16));
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


// ------------------------------------------------------------------ kernel

template <int F, int MT>
__device__ __forceinline__ void finalize_token(const GemvParams& p, int row, int token, float v,
                                               float row_scale) {
  if constexpr (F == W_I8_ROW) v = mul_rn(v, row_scale);
  if constexpr (F == W_FP4_G16E) v = mul_rn(v, __ldg(p.gscale));
  const long long idx = static_cast<long long>(token) * p.ldo + row;
  if (p.out_f32) {
    static_cast<float*>(p.out)[idx] = v;
  } else {
    static_cast<unsigned short*>(p.out)[idx] = f32_to_bf16_rn(v);
  }
}

// Grid (G, ceil(M / MT)); block kWarps*32. Dynamic shared memory:
// [mbarriers][kWarps warp regions: kDepth slots (+ metadata ring)][x staging].
template <int F, int X, int XM, int MT>
__global__ void __launch_bounds__(kWarps * 32, 1) stream_gemv_kernel(const GemvParams p) {
  constexpr int KC = Layout<F>::KC;
  constexpr int SLOT = Layout<F>::SLOT;
  constexpr int VALS = WTraits<F>::VALS;
  constexpr bool CODED = (F == W_CBF16);
  constexpr int BAR_REGION = ((kWarps * Layout<F>::BARS * 8 + 127) / 128) * 128;
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
  float* xs = reinterpret_cast<float*>(smem + BAR_REGION + kWarps * Layout<F>::WARP_BYTES);
  const int kpad = ((k + 32 * VALS - 1) / (32 * VALS)) * (32 * VALS);
  const int segs = kpad / (32 * VALS);

  // This warp's items: (row, chunk) pairs in processing order.
  int r0 = 0, nitems = 0;
  long long wbegin = 0, wend = 0;
  if (!p.split) {
    const int g = gridDim.x;
    const int b = blockIdx.x;
    r0 = static_cast<int>(static_cast<long long>(n) * b / g);
    const int r1 = static_cast<int>(static_cast<long long>(n) * (b + 1) / g);
    const int rows = r1 - r0 - warp > 0 ? (r1 - r0 - warp + kWarps - 1) / kWarps : 0;
    nitems = rows * S;
  } else {
    const long long T = static_cast<long long>(n) * S;
    const long long i0 = T * blockIdx.x / gridDim.x, i1 = T * (blockIdx.x + 1) / gridDim.x;
    wbegin = i0 + (i1 - i0) * warp / kWarps;
    wend = i0 + (i1 - i0) * (warp + 1) / kWarps;
    nitems = static_cast<int>(wend - wbegin);
  }
  auto item_rc = [&](int q, int& row, int& c) {
    if (!p.split) {
      row = r0 + warp + kWarps * (q / S);
      c = q - (q / S) * S;
    } else {
      const long long gi = wbegin + q;
      row = static_cast<int>(gi / S);
      c = static_cast<int>(gi - static_cast<long long>(row) * S);
    }
  };

  // lane 0: bulk copy of item q's metadata (coded) into its ring entry.
  auto issue_meta = [&](int q) {
    int row, c;
    item_rc(q, row, c);
    const int nb = min(32, k / 64 - 32 * c);
    const unsigned bar = mbar0 + (q % kMetaRing) * 8;
    const char* src = static_cast<const char*>(p.aux) + (static_cast<long long>(row) * (k / 64) + 32 * c) * 4;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, nb * 4);
    bulk_g2s(meta0 + (q % kMetaRing) * kMetaEntry, src, nb * 4, bar);
  };
  // lane 0: bulk copy of item q's weight bytes (+ scales) into slot q % kDepth.
  auto issue_item = [&](int q) {
    int row, c;
    item_rc(q, row, c);
    const int L = min(KC, k - c * KC);
    const unsigned slot = slot0 + (q % kDepth) * SLOT;
    const unsigned bar = pbar0 + (q % kDepth) * 8;
    const char* src;
    int bytes;
    const char* ssrc;
    int sbytes;
    if constexpr (CODED) {
      const unsigned entry = meta0 + (q % kMetaRing) * kMetaEntry;
      const int nb = L / 64;
      const unsigned m0 = lds32(entry), ml = lds32(entry + 4 * (nb - 1));
      const unsigned off = (m0 & 0x7fffffu) << 5;
      const unsigned end = ((ml & 0x7fffffu) << 5) + ((ml >> 31) ? 128u : 96u);
      src = static_cast<const char*>(p.w) + off;
      bytes = static_cast<int>(end - off);
      ssrc = nullptr;
      sbytes = 0;
    } else {
      src = static_cast<const char*>(p.w) + w_offset_bytes<F>(static_cast<long long>(row) * k + c * KC);
      bytes = static_cast<int>(w_offset_bytes<F>(L));
      scale_span<F>(p, row, c, L, &ssrc, &sbytes);
    }
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, bytes + sbytes);
    bulk_g2s(slot, src, bytes, bar);
    if (sbytes) bulk_g2s(slot + kWeightSlot, ssrc, sbytes, bar);
  };

  bool ok = true;
  int issued_meta = 0, issued = 0;  // lane 0 bookkeeping (items issued so far)
  if (p.use_tma) {
    if (lane == 0) {
      for (int i = 0; i < Layout<F>::BARS; ++i) mbar_init(pbar0 + 8 * i, 1);
      fence_mbar_init();
    }
    __syncwarp();
    // Prologue: weights do not depend on the previous grid, so these copies are
    // in flight before griddepcontrol.wait.
    if (lane == 0) {
      if constexpr (CODED) {
        for (; issued_meta < min(kMetaRing, nitems); ++issued_meta) issue_meta(issued_meta);
        for (; issued < min(kDepth - 1, nitems); ++issued) {
          if (!mbar_wait(mbar0 + (issued % kMetaRing) * 8, (issued / kMetaRing) & 1)) {
            ok = false;
            break;
          }
          issue_item(issued);
        }
      } else {
        for (; issued < min(kDepth - 1, nitems); ++issued) issue_item(issued);
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
  }

  grid_dependency_wait();
  if constexpr (XM == XM_SMEM) stage_x<F, X, MT>(p, tile, xs, kpad);
  __syncthreads();
  grid_launch_dependents();

  float rowsum[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) rowsum[t] = 0.0f;
  float row_scale = 1.0f;
  int contributed = 0;

  int q = 0;
  for (; q < nitems && ok; ++q) {
    int row, c;
    item_rc(q, row, c);
    const int L = min(KC, k - c * KC);
    const unsigned slot = slot0 + (q % kDepth) * SLOT;
    const unsigned entry = meta0 + (q % kMetaRing) * kMetaEntry;
    if (p.use_tma) {
      if (lane == 0 && issued < nitems && issued == q + kDepth - 1) {
        bool ready = true;
        if constexpr (CODED) ready = mbar_wait(mbar0 + (issued % kMetaRing) * 8, (issued / kMetaRing) & 1);
        if (ready) {
          issue_item(issued);
          ++issued;
        } else {
          ok = false;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const bool landed = mbar_wait(pbar0 + (q % kDepth) * 8, (q / kDepth) & 1);
      if (!__all_sync(0xffffffffu, landed)) {
        ok = false;
        break;
      }
    } else {
      // Cooperative fill: any alignment, zero padding past the item's data.
      unsigned char* sp = slot0_ptr + (q % kDepth) * SLOT;
      if constexpr (CODED) {
        unsigned* ep = reinterpret_cast<unsigned*>(slot0_ptr + kDepth * SLOT + (q % kMetaRing) * kMetaEntry);
        const int nb = L / 64;
        if (lane < nb) ep[lane] = __ldg(static_cast<const unsigned*>(p.aux) + static_cast<long long>(row) * (k / 64) + 32 * c + lane);
        __syncwarp();
        const unsigned m0 = ep[0], ml = ep[nb - 1];
        const unsigned off = (m0 & 0x7fffffu) << 5;
        const unsigned end = ((ml & 0x7fffffu) << 5) + ((ml >> 31) ? 128u : 96u);
        warp_copy_bytes(reinterpret_cast<char*>(sp), static_cast<const char*>(p.w) + off,
                        static_cast<int>(end - off), kWeightSlot, lane);
      } else {
        const char* src = static_cast<const char*>(p.w) + w_offset_bytes<F>(static_cast<long long>(row) * k + c * KC);
        warp_copy_bytes(reinterpret_cast<char*>(sp), src, static_cast<int>(w_offset_bytes<F>(L)),
                        kWeightSlot, lane);
        if constexpr (WTraits<F>::SCALE_BYTES > 0) {
          const char* ssrc;
          int sbytes;
          scale_span<F>(p, row, c, L, &ssrc, &sbytes);
          warp_copy_bytes(reinterpret_cast<char*>(sp) + kWeightSlot, ssrc, sbytes,
                          WTraits<F>::SCALE_BYTES, lane);
        }
      }
      __syncwarp();
    }

    if constexpr (F == W_I8_ROW) {
      if (c == 0 || q == 0) row_scale = __ldg(static_cast<const float*>(p.aux) + row);
    }
    const unsigned first_unit = CODED ? (lds32(entry) & 0x7fffffu) : 0u;
    float P[MT];
    compute_item<F, X, XM, MT>(p, xs, segs, tile, c, L, slot, entry, first_unit, lane, P);
    __syncwarp();  // every lane is done with this slot before it is refilled

    const bool complete = !p.split || (static_cast<long long>(row) * S >= wbegin &&
                                       static_cast<long long>(row) * S + S <= wend);
    if (complete) {
#pragma unroll
      for (int t = 0; t < MT; ++t) rowsum[t] = (c == 0) ? P[t] : add_rn(rowsum[t], P[t]);
      if (c == S - 1) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const int token = tile * MT + t;
          if (lane == t && token < p.m) finalize_token<F, MT>(p, row, token, rowsum[t], row_scale);
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
          if constexpr (F == W_I8_ROW) row_scale = __ldg(static_cast<const float*>(p.aux) + row);
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const int token = tile * MT + t;
            if (lane == t && token < p.m) {
              const float* src = p.ws + ((static_cast<long long>(tile) * MT + t) * n + row) * S;
              float total = __ldcg(src);
              for (int cc = 1; cc < S; ++cc) total = add_rn(total, __ldcg(src + cc));
              finalize_token<F, MT>(p, row, token, total, row_scale);
            }
          }
          if (lane == 0) *ticket = 0u;
        }
      }
    }

    if constexpr (CODED) {
      if (p.use_tma && lane == 0 && issued_meta < nitems && issued_meta == q + kMetaRing) {
        issue_meta(issued_meta);
        ++issued_meta;
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
