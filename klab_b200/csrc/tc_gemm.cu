// Tensor-core (tcgen05) projection for token tiles: y[M, N] = x[M, K] . W[N, K]^T
// with BF16 x, for weight formats whose values are exact in BF16: BF16 and INT8
// with one FP32 scale per row (benchmark config 2). Used for M >= 2, where the
// CUDA-core kernel's per-token FMAs make it issue-bound.
//
// CTA = 128 weight rows (the MMA's M) x 16 tokens (its N, zero-padded) x all K.
// Warp roles (320 threads):
//   warp 8      producer: 2-D TMA loads (cp.async.bulk.tensor, no multicast) of
//               the next W tile [128 rows x 128 k] and x tile [16 x 128] per
//               stage, all 128-byte swizzled; BF16 W lands directly in the
//               K-major operand layout the MMA reads from shared memory (two
//               64-column atoms), INT8 W lands raw in a 12-stage byte ring; lane
//               0 streams W and lane 1 streams x, each gated only by its own ring
//               (x has a 6-stage ring released by its own commit);
//   warps 0..7  INT8 only: decode each raw tile to exact BF16 (|code| <= 127 has
//               at most 7 significant bits) straight into tensor memory: warp w
//               owns TMEM lanes 32*(w%4).. (its rows) and half w/4 of the stage's
//               K, one row per thread, 64 codes -> 32 columns (tcgen05.st). The
//               A operand then never occupies shared memory, which holds twice
//               the raw ring instead (INT8 streaming is bound by bytes in
//               flight). Warps 0..3 then run the epilogue: TMEM -> registers
//               (tcgen05.ld), row scale, one RNE to BF16 (or FP32), store;
//   warp 9      allocates TMEM (128 accumulator columns, plus six 64-column A
//               stages for INT8); lane 0 issues eight tcgen05.mma.kind::f16
//               (K = 16 each) per stage, A from shared memory (BF16) or from
//               tensor memory (INT8), MMA k into FP32 accumulator k [128 lanes x
//               16 columns] (eight independent chains), and releases the stage's
//               slots with tcgen05.commit; the epilogue adds the eight
//               accumulators in a fixed tree.
// Every mbarrier wait is bounded; on a timeout the kernel records the status
// word, stops issuing, drains what it issued and frees TMEM.
//
// Arithmetic: products are exact, sums are FP32 in the tensor core's order, so
// results meet the FP64 tolerance of the projection contract but are not
// bit-identical to the CUDA-core kernel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "common.cuh"
#include "klab_kernels.h"

namespace klab {
namespace {

constexpr int kTcRows = 128;   // MMA M
constexpr int kTcTok = 16;     // MMA N
constexpr int kTcAtom = 64;    // K of one 128-byte swizzle row of BF16
constexpr int kTcBK = 128;     // K per stage: two swizzle atoms
#ifndef KLAB_TC_DECODERS
#define KLAB_TC_DECODERS 8
#endif
constexpr int kTcDec = KLAB_TC_DECODERS;  // decoder warps: two per TMEM lane quarter
static_assert(kTcDec == 8 || kTcDec == 16, "INT8 decoders: warp w owns lane quarter w % 4 and K part w / 4");
constexpr int kTcParts = kTcDec / 4;             // K parts of a stage per lane quarter
constexpr int kTcChunks = 8 / kTcParts;          // 16-code chunks per decoder thread and stage
constexpr int kTcDecCols = 8 * kTcChunks;        // TMEM columns a decoder thread writes per stage
constexpr int kTcASub = kTcRows * kTcAtom * 2;   // 16 KiB per atom column
constexpr int kTcBSub = kTcTok * kTcAtom * 2;    // 2 KiB per atom column
constexpr int kTcABytes = 2 * kTcASub;           // 32 KiB: W operand of one stage
constexpr int kTcBBytes = 2 * kTcBSub;           // 4 KiB: x operand of one stage
constexpr int kTcRawBytes = kTcRows * kTcBK;     // 16 KiB: raw INT8 W of one stage
constexpr int kTcX = 6;                          // x stages
constexpr int kTcMaxA = 6, kTcMaxRaw = 12;       // operand (BF16: smem; INT8: TMEM) and raw INT8 stages
constexpr int kTcProducer = kTcDec, kTcMma = kTcDec + 1;  // warp indices
constexpr int kTcThreads = 32 * (kTcDec + 2);
// Shared memory, 1024-aligned: BF16 [6 operand stages][x ring], INT8 [12 raw
// stages][x ring]; then [barriers, TMEM address].
constexpr int kTcSmemData = kTcX * kTcBBytes + 6 * kTcABytes;
static_assert(kTcMaxRaw * kTcRawBytes == 6 * kTcABytes, "both layouts put the x ring at the same offset");
constexpr int kTcBarBytes = 512;
constexpr int kTcSmem = kTcSmemData + kTcBarBytes + 1024;  // + slack to align the base to 1024
constexpr int kTcAcc = kTcBK / 16;                // independent accumulators (one per MMA of a stage)
constexpr int kTcAccCols = kTcAcc * kTcTok;       // 128 accumulator columns
constexpr int kTcACols = kTcBK / 2;               // 64 columns: one INT8 stage's A in TMEM (2 BF16 per column)
// INT8: accumulators + six A stages = 512 columns (the whole TMEM of the SM; one CTA per SM).
constexpr int kTcTmemColsI8 = kTcAccCols + kTcMaxA * kTcACols;
static_assert(kTcTmemColsI8 == 512, "TMEM allocation must be a power of two");

enum TcKind : int { TC_BF16 = 0, TC_I8_ROW = 1 };

struct alignas(64) TcParams {
  CUtensorMap tmap_w;
  CUtensorMap tmap_x;
  const float* scales;  // TC_I8_ROW: per row
  void* out;
  int ldo, out_f32;
  int m, n, k;
  int kind;
  int* status;
};

// 64-bit shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (start address >> 4 in bits 0-13, SBO >> 4 in bits 32-45,
// version 1 in bits 46-47, layout SWIZZLE_128B = 2 in bits 61-63).
__device__ __forceinline__ uint64_t sw128_desc(unsigned smem_byte_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>(1u) << 16;                 // LBO (ignored for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;         // SBO
  d |= static_cast<uint64_t>(1u) << 46;                 // version
  d |= static_cast<uint64_t>(2u) << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, A = B = BF16 (K-major), D = F32, M = 128, N = 16.
constexpr uint32_t kTcIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((kTcTok >> 3) << 17) | ((kTcRows >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(unsigned dst, const CUtensorMap* map, int x, int y, unsigned bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate)
      : "memory");
}

// A from tensor memory (K-major: row m in lane m, K pairs packed per column).
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(unsigned bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ unsigned pack_bf16x2(float lo, float hi) {
  unsigned d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// 16 signed int8 codes (as four words) -> 16 exact BF16 values (eight words).
__device__ __forceinline__ void int8x16_to_bf16(const uint4 q, uint4& lo, uint4& hi) {
  const unsigned w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
  unsigned o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int b = 0; b < 4; b += 2) {
      const f2 u{__uint_as_float(__byte_perm(w[i], 0x4b000000u, 0x7540u + b)),
                 __uint_as_float(__byte_perm(w[i], 0x4b000000u, 0x7541u + b))};
      const f2 v = add2(u, f2{-8388736.0f, -8388736.0f});
      o[2 * i + b / 2] = pack_bf16x2(v.x, v.y);
    }
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row r in a 128-byte-swizzled
// K-major tile.
__device__ __forceinline__ unsigned sw128_offset(int r, int chunk) {
  return static_cast<unsigned>((r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled operand tiles.
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  __shared__ int s_fail;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool int8 = p.kind == TC_I8_ROW;
  const int DA = kTcMaxA;                     // W operand stages (BF16: shared memory; INT8: TMEM)
  const int DR = int8 ? kTcMaxRaw : 0;        // raw INT8 stages
  const unsigned base = smem_addr(smem);
  const unsigned xoff = 6 * kTcABytes, rawoff = 0;  // raw INT8 ring where BF16 keeps its operand ring
  const unsigned bar0 = base + kTcSmemData;
  const uint32_t tmem_cols = int8 ? kTcTmemColsI8 : kTcAccCols;
  // Barriers (8 bytes each): raw_full/empty[12], a_full/empty[6], x_full/empty[6], done; TMEM address.
  const unsigned raw_full = bar0, raw_empty = bar0 + 8 * kTcMaxRaw;
  const unsigned a_full = bar0 + 16 * kTcMaxRaw, a_empty = a_full + 8 * kTcMaxA;
  const unsigned x_full = a_empty + 8 * kTcMaxA, x_empty = x_full + 8 * kTcX;
  const unsigned done_bar = x_empty + 8 * kTcX;
  constexpr int kBars = 2 * kTcMaxRaw + 2 * kTcMaxA + 2 * kTcX + 1;
  static_assert(8 * kBars + 4 <= kTcBarBytes, "barrier region");
  unsigned* tmem_slot = reinterpret_cast<unsigned*>(smem + kTcSmemData + 8 * kBars);

  const int stages = (p.k + kTcBK - 1) / kTcBK;
  const int row0 = blockIdx.x * kTcRows;
  const int tok0 = blockIdx.y * kTcTok;

  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int i = 0; i < kTcMaxRaw; ++i) {
      mbar_init(raw_full + 8 * i, 1);
      mbar_init(raw_empty + 8 * i, kTcDec);
    }
    for (int i = 0; i < kTcMaxA; ++i) {
      mbar_init(a_full + 8 * i, int8 ? kTcDec : 1);  // decoder warps, or the producer's TMA
      mbar_init(a_empty + 8 * i, 1);                  // tcgen05.commit
    }
    for (int i = 0; i < kTcX; ++i) {
      mbar_init(x_full + 8 * i, 1);
      mbar_init(x_empty + 8 * i, 1);                  // tcgen05.commit
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == kTcMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_addr(tmem_slot)), "r"(tmem_cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTcProducer) {
    // ---------------- producer: lane 0 streams W (INT8 into the raw ring, BF16
    // straight into the operand ring), lane 1 streams x into the x ring. Each
    // lane is gated only by its own ring.
    if (lane < 2) {
      const bool w_lane = lane == 0;
      const int depth = w_lane ? (int8 ? DR : DA) : kTcX;
      const unsigned full = w_lane ? (int8 ? raw_full : a_full) : x_full;
      const unsigned empty = w_lane ? (int8 ? raw_empty : a_empty) : x_empty;
      const unsigned data = base + (w_lane ? (int8 ? rawoff : 0u) : xoff);
      const unsigned bytes = w_lane ? (int8 ? kTcRawBytes : kTcABytes) : kTcBBytes;
      int issued = 0;
      bool ok = true;
      for (int s = 0; s < stages; ++s) {
        const int i = s % depth;
        if (!mbar_wait(empty + 8 * i, ((s / depth) & 1) ^ 1) || *reinterpret_cast<volatile int*>(&s_fail)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(full + 8 * i, bytes);
        const unsigned dst = data + i * bytes;
        const int kx = s * kTcBK;
        if (!w_lane) {
          for (int j = 0; j < 2; ++j) tma_load_2d(dst + j * kTcBSub, &p.tmap_x, kx + j * kTcAtom, tok0, full + 8 * i);
        } else if (int8) {
          tma_load_2d(dst, &p.tmap_w, kx, row0, full + 8 * i);
        } else {
          for (int j = 0; j < 2; ++j) tma_load_2d(dst + j * kTcASub, &p.tmap_w, kx + j * kTcAtom, row0, full + 8 * i);
        }
        ++issued;
      }
      if (!ok) {
        atomicExch(&s_fail, 1);
        record_status(p.status, kStatusMbarTimeout);
      }
      // Drain: the last `depth` issued stages are the latest uses of their
      // slots; each has landed (bounded wait) before the CTA may exit.
      for (int s = issued > depth ? issued - depth : 0; s < issued; ++s)
        mbar_wait(full + 8 * (s % depth), (s / depth) & 1);
    }
  } else if (warp == kTcMma) {
    // ---------------- MMA issuer
    if (lane == 0) {
      bool ok = true;
      for (int s = 0; s < stages; ++s) {
        const int a = s % DA, xi = s % kTcX;
        if (!mbar_wait(a_full + 8 * a, (s / DA) & 1) || !mbar_wait(x_full + 8 * xi, (s / kTcX) & 1) ||
            *reinterpret_cast<volatile int*>(&s_fail)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const unsigned abase = base + a * kTcABytes, bbase = base + xoff + xi * kTcBBytes;
        // MMA kk of every stage accumulates into its own TMEM accumulator, so the
        // eight MMAs of a stage are independent (one chain would serialise them).
        // INT8: A stage a sits in TMEM columns kTcAccCols + 64a.., MMA kk reads 8 of them.
        const uint32_t atmem = tmem + kTcAccCols + a * kTcACols;
#pragma unroll
        for (int kk = 0; kk < kTcAcc; ++kk) {
          const unsigned off = 32 * (kk % 4);
          const int j = kk / 4;
          if (int8)
            tc_mma_ts(tmem + kk * kTcTok, atmem + kk * 8, sw128_desc(bbase + j * kTcBSub + off), s > 0 ? 1u : 0u);
          else
            tc_mma(tmem + kk * kTcTok, sw128_desc(abase + j * kTcASub + off), sw128_desc(bbase + j * kTcBSub + off),
                   s > 0 ? 1u : 0u);
        }
        tc_commit(a_empty + 8 * a);
        tc_commit(x_empty + 8 * xi);
      }
      if (!ok) {
        atomicExch(&s_fail, 1);
        record_status(p.status, kStatusMbarTimeout);
      }
      tc_commit(done_bar);  // completes when every MMA issued above has finished
    }
  } else {
    // ---------------- decoders (INT8, warps 0..7) and epilogue (warps 0..3)
    if (int8) {
      for (int s = 0; s < stages; ++s) {
        const int r = s % DR, a = s % DA;
        bool ok = mbar_wait(raw_full + 8 * r, (s / DR) & 1);
        ok = ok && mbar_wait(a_empty + 8 * a, ((s / DA) & 1) ^ 1);
        if (!__all_sync(0xffffffffu, ok) || *reinterpret_cast<volatile int*>(&s_fail)) {
          if (lane == 0) {
            atomicExch(&s_fail, 1);
            record_status(p.status, kStatusMbarTimeout);
          }
          break;
        }
        tc_fence_after();  // the MMAs that read this TMEM stage have completed
        // Thread = one row (TMEM lane 32*(w%4) + lane); warp w decodes K part
        // w/4 of the stage: raw 16-byte chunks of its row (128-byte swizzled:
        // chunk c of row r at (c ^ (r & 7)) * 16, conflict-free), each 16 codes
        // -> 8 BF16 pairs = 8 TMEM columns.
        const int quarter = warp & 3, part = warp >> 2;
        const int row = 32 * quarter + lane;
        const unsigned char* raw = smem + rawoff + r * kTcRawBytes + row * kTcBK;
        unsigned v[32];
#pragma unroll
        for (int j = 0; j < kTcChunks; ++j) {
          const int c = kTcChunks * part + j;
          const uint4 q = *reinterpret_cast<const uint4*>(raw + ((c ^ (row & 7)) << 4));
          uint4 lo, hi;
          int8x16_to_bf16(q, lo, hi);
          v[8 * j] = lo.x; v[8 * j + 1] = lo.y; v[8 * j + 2] = lo.z; v[8 * j + 3] = lo.w;
          v[8 * j + 4] = hi.x; v[8 * j + 5] = hi.y; v[8 * j + 6] = hi.z; v[8 * j + 7] = hi.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(raw_empty + 8 * r);  // the raw slot is read
        const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quarter) << 16) + kTcAccCols + a * kTcACols +
                               kTcDecCols * part;
        if constexpr (kTcDecCols == 32) {
          asm volatile(
              "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
              "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
              ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
                "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
                "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
                "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
              : "memory");
        } else {
          asm volatile(
              "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
              ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
                "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
              : "memory");
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full + 8 * a);
      }
    }
    // Epilogue (warps 0..3 own the TMEM lane quarters): row 32*warp + lane,
    // tokens tok0 .. tok0+15.
    if (warp < 4) {
      const bool fin = mbar_wait(done_bar, 0);
      tc_fence_after();
      // Sum of the eight accumulators: ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)) per
      // token, built pair by pair so at most four accumulators are live.
      auto load_acc = [&](int j, float (&a)[kTcTok]) {
        unsigned v[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(tmem + (static_cast<uint32_t>(32 * warp) << 16) + j * kTcTok));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int t = 0; t < kTcTok; ++t) a[t] = __uint_as_float(v[t]);
      };
      // Sum of accumulators 4h .. 4h+3 as ((a0 + a1) + (a2 + a3)).
      auto quad = [&](int h, float (&q)[kTcTok]) {
        float x0[kTcTok], x1[kTcTok];
        load_acc(4 * h, x0);
        load_acc(4 * h + 1, x1);
#pragma unroll
        for (int t = 0; t < kTcTok; ++t) q[t] = add_rn(x0[t], x1[t]);
        load_acc(4 * h + 2, x0);
        load_acc(4 * h + 3, x1);
#pragma unroll
        for (int t = 0; t < kTcTok; ++t) q[t] = add_rn(q[t], add_rn(x0[t], x1[t]));
      };
      float total[kTcTok], upper[kTcTok];
      quad(0, total);
      quad(1, upper);
#pragma unroll
      for (int t = 0; t < kTcTok; ++t) total[t] = add_rn(total[t], upper[t]);
      const int row = row0 + 32 * warp + lane;
      if (!fin) record_status(p.status, kStatusMbarTimeout);
      if (fin && row < p.n) {
        const float scale = int8 ? __ldg(p.scales + row) : 1.0f;
#pragma unroll
        for (int t = 0; t < kTcTok; ++t) {
          const int token = tok0 + t;
          if (token < p.m) {
            float y = total[t];
            if (int8) y = mul_rn(y, scale);
            const long long idx = static_cast<long long>(token) * p.ldo + row;
            if (p.out_f32)
              static_cast<float*>(p.out)[idx] = y;
            else
              static_cast<unsigned short*>(p.out)[idx] = f32_to_bf16_rn(y);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  }
  return fn;
}

// 2-D map over a row-major [rows, cols] matrix with a box of [box_rows, box_cols].
int make_map(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* ptr, long long rows,
             long long cols, long long row_stride_elems, int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  EncodeTiled fn = encode_fn();
  if (!fn) return KLAB_E_DRIVER;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems) * elem_bytes};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : KLAB_E_ALIGN;
}

}  // namespace

// Host launcher: kind TC_BF16 (w BF16 [n, k]) or TC_I8_ROW (w int8 [n, k] + scales [n]).
int tc_gemm_launch(int kind, const void* x, int ldx, const void* w, const float* scales, void* out, int ldo,
                   int out_f32, int m, int n, int k, int* status, cudaStream_t stream) {
  if (!x || !w || !out || m <= 0 || n <= 0 || k <= 0) return KLAB_E_INVALID;
  if (kind == TC_I8_ROW && !scales) return KLAB_E_INVALID;
  // TMA: 16-byte aligned bases and row strides.
  const int wbytes = kind == TC_I8_ROW ? 1 : 2;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) || (ldx * 2) % 16 ||
      (static_cast<long long>(k) * wbytes) % 16)
    return KLAB_E_ALIGN;
  TcParams p;
  std::memset(&p, 0, sizeof(p));
  int rc = make_map(&p.tmap_w, kind == TC_I8_ROW ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                    wbytes, w, n, k, k, kind == TC_I8_ROW ? kTcBK : kTcAtom, kTcRows,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_map(&p.tmap_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, m, k, ldx, kTcAtom, kTcTok,
                CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  p.scales = scales;
  p.out = out;
  p.ldo = ldo;
  p.out_f32 = out_f32;
  p.m = m;
  p.n = n;
  p.k = k;
  p.kind = kind;
  p.status = status;
  static bool attr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KLAB_E_UNSUPPORTED;
  if (!attr[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  const dim3 grid((n + kTcRows - 1) / kTcRows, (m + kTcTok - 1) / kTcTok);
  if (grid.y > 65535) return KLAB_E_SHAPE;
  tc_gemm_kernel<<<grid, kTcThreads, kTcSmem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace klab
