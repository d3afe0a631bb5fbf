// Decode attention for one token (M = 1) with grouped-query heads and the new
// K/V row appended to the cache in the same launch: out = softmax(q K^T * scale) V
// over the cache's first `len` tokens plus the new one. Replaces the reference's
// decode_attn_v4 / v4d / v5 kernels (research/l2-prefetch/src/decode_attn.cu:
// 258-460, 530-600) behind decode_attn.decode_attention(_dynamic)
// (decode_attn.py:20-107).
//
// Work split (flash-decoding): the token span (len + 1, or the capacity when the
// length is read from device memory) is cut into `splits` tiles of `tile` tokens
// (a multiple of 64, at most 512). CTA (kv head, split) serves every query head
// of its group, so each K/V row crosses HBM once:
//   1. K and V rows are copied with coalesced 16-byte cp.async into XOR-swizzled
//      tiles (chunk i of row r at chunk i ^ (r mod 8)), which keeps the fragment
//      loads below conflict-free; V's copies land while the scores run. The CTA whose tile
//      holds position `len` writes the new K/V row into the cache and its tiles.
//   2. Scores on the tensor cores (mma.sync m16n8k16, BF16 in, FP32 out): the
//      group's query heads (at most 16) are the 16 rows of the A fragment, loaded
//      once from global memory; warp w takes a contiguous run of tokens and reads
//      K fragments with ldmatrix. Tokens past the end are masked to -inf.
//   3. Softmax partials in registers: per-warp row maxima through shared memory,
//      p = exp(s - m), per-warp row sums.
//   4. O = P V on the tensor cores: p is split into hi + lo BF16 halves (so the
//      product keeps close to FP32 accuracy) that feed the A fragments straight
//      from the score accumulators; V fragments come from transposing ldmatrix.
//      The warps' 16 x 64 partials are summed in warp order through shared memory.
//   5. Merge of the splits with weights exp(m_c - max m):
//      - cluster mode (splits <= the cluster limit): the splits of one kv head
//        form a thread-block cluster; each CTA keeps (m, l, o[64]) per head in
//        shared memory and the cluster reads them over distributed shared memory;
//      - ticket mode (longer spans): records go to global scratch and the last
//        CTA of a kv head (atomic ticket) merges them and resets the ticket.
// The two contractions are 16-row matrix products: warp-level mma.sync fits them,
// where a tcgen05 tile (64 or 128 rows) would leave most of its rows empty.
// FP32 arithmetic, the fast exp intrinsic, one RNE to BF16. A device length
// outside [0, capacity) leaves the caches and the output untouched and sets the
// device status word (kStatusBadLength).
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "klab_b200.h"
#include "klab_kernels.h"

namespace klab {
namespace {

constexpr int kHD = 64;             // head dimension
constexpr int kRowBytes = kHD * 2;  // one BF16 K or V row
#ifndef KLAB_ATTN_MIN_TILE
#define KLAB_ATTN_MIN_TILE 128  // smallest tile the planner cuts a span into (a multiple of 64)
#endif
constexpr int kMinTile = KLAB_ATTN_MIN_TILE;
#ifndef KLAB_ATTN_SINGLE_SPAN
#define KLAB_ATTN_SINGLE_SPAN 384  // spans up to this many tokens run as one tile per kv head (no merge)
#endif
#ifndef KLAB_ATTN_CLUSTER
#define KLAB_ATTN_CLUSTER 1  // 1: merge over a thread-block cluster when one covers the span
#endif
#ifndef KLAB_ATTN_SMEM_FLOOR
#define KLAB_ATTN_SMEM_FLOOR 0  // minimum dynamic shared memory per CTA (bytes): limits CTAs per SM
#endif
constexpr int kMaxTile = 512;
constexpr int kMaxGroup = 16;       // query heads per kv head
constexpr int kAttnThreads = 256;
constexpr int kWarps = kAttnThreads / 32;
constexpr int kRecord = kHD + 2;    // (m, l, o[64]) per (head, split)
constexpr int kMaxSpan = 65536;
constexpr int kMaxClusterSplits = 16;  // the largest (non-portable) cluster
constexpr size_t kMaxSmem = 227 * 1024;
constexpr float kNegInf = -__builtin_huge_valf();

struct AttnParams {
  const unsigned short* q;
  const unsigned short* k_new;
  const unsigned short* v_new;
  unsigned short* kc;
  unsigned short* vc;
  unsigned short* out;
  float* scratch;
  unsigned* tickets;
  const int* len_ptr;
  int* status;
  int len_value, max_len, heads, kv_heads, splits, tile;
  int tpw;  // tokens per warp: a multiple of 16; 8 * tpw >= tile
  float scale;
};

struct SmemLayout {
  size_t ks, vs, red, part, wts, ml, stats, tk, total;
};

constexpr int kRedStride = kHD + 8;  // floats per (warp, head row) of the output partials

// Tokens per warp for a tile: 16-token steps of the tensor-core fragments.
__host__ __device__ inline int tokens_per_warp(int tile) { return ((tile + kWarps - 1) / kWarps + 15) & ~15; }

__host__ __device__ inline SmemLayout layout_for(int tile, int group, int splits, bool ticket) {
  const size_t rows = static_cast<size_t>(kWarps) * tokens_per_warp(tile);  // tile rounded up
  SmemLayout s;
  s.ks = 0;
  s.vs = s.ks + rows * kRowBytes;
  s.red = s.vs + rows * kRowBytes;
  s.part = s.red + static_cast<size_t>(kWarps) * 16 * kRedStride * 4;  // per warp: 16 head rows
  s.wts = s.part + static_cast<size_t>(group) * kRecord * 4;
  s.ml = s.wts + (ticket ? 2 * static_cast<size_t>(group) * splits * 4 : 0);
  s.stats = s.ml + 2 * kMaxGroup * 4;
  s.tk = (s.stats + 2 * kWarps * 16 * 4 + 15) / 16 * 16;
  s.total = s.tk + 16;
  return s;
}

__device__ __forceinline__ unsigned cluster_map(unsigned addr, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_cluster_f32(unsigned addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float warp_max(float m) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return m;
}

__device__ __forceinline__ unsigned short rne_bf16(float v) { return f32_to_bf16_rn(v); }

// D += A (16x16, BF16, row) * B (16x8, BF16, col) with FP32 accumulation.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(unsigned addr, unsigned (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Two floats as BF16 (RNE), x0 in the low half.
__device__ __forceinline__ unsigned pack_bf16x2(float x0, float x1) {
  return static_cast<unsigned>(f32_to_bf16_rn(x0)) | (static_cast<unsigned>(f32_to_bf16_rn(x1)) << 16);
}

// p = hi + lo with hi, lo BF16: the pair's hi word and the residuals' lo word.
__device__ __forceinline__ void split_bf16x2(float x0, float x1, unsigned& hi, unsigned& lo) {
  hi = pack_bf16x2(x0, x1);
  lo = pack_bf16x2(__fsub_rn(x0, bf16lo(hi)), __fsub_rn(x1, bf16hi(hi)));
}

// Byte offset of 16-byte chunk `ch` of row `r` in a swizzled 128-byte-row tile.
__device__ __forceinline__ unsigned swz(int r, int ch) {
  return static_cast<unsigned>(r * kRowBytes + ((ch ^ (r & 7)) << 4));
}

template <bool kCluster>
__global__ void __launch_bounds__(kAttnThreads) decode_attn_kernel(const AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  // Programmatic dependent launch: nothing global is read or written before the
  // previous kernel on the stream has completed.
  grid_dependency_wait();
  grid_launch_dependents();
  const int len = p.len_ptr ? *p.len_ptr : p.len_value;  // cached tokens before the new one
  if (len < 0 || len >= p.max_len || len >= p.splits * p.tile) {  // every CTA sees the same value
    if (blockIdx.x == 0 && threadIdx.x == 0) record_status(p.status, kStatusBadLength);
    return;
  }
  const int splits = p.splits, tile = p.tile;
  const int group = p.heads / p.kv_heads;
  const SmemLayout L = layout_for(tile, group, splits, !kCluster);
  unsigned char* ks = smem + L.ks;
  unsigned char* vs = smem + L.vs;
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* part = reinterpret_cast<float*>(smem + L.part);
  float* ml = reinterpret_cast<float*>(smem + L.ml);
  float* wmax = reinterpret_cast<float*>(smem + L.stats);  // [warp][16 head rows]
  float* wsum = wmax + kWarps * 16;                         // [warp][16 head rows]

  const int kvh = blockIdx.x / splits, c = blockIdx.x - kvh * splits;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t base = static_cast<size_t>(kvh) * p.max_len * kHD;  // element offset of this kv head's cache
  const int lo = c * tile;
  const int ncache = min(max(len - lo, 0), tile);                 // cached tokens [lo, lo + ncache)
  const bool owns_new = len >= lo && len < lo + tile;             // the new token is local token ncache
  const int n = ncache + (owns_new ? 1 : 0);

  const int tpw = p.tpw, rows = kWarps * tpw;

  // ---- 1. staging: K and V rows by 16-byte cp.async copies (coalesced, straight
  // into the swizzled tiles, every copy of the tile in flight at once; K and V in
  // separate groups); rows [n, rows) of V are zeroed (p = 0 there, and 0 * garbage
  // could be NaN); the new token's row goes to the cache and the tiles.
  {
    const uint4* ksrc = reinterpret_cast<const uint4*>(p.kc + base + static_cast<size_t>(lo) * kHD);
    const uint4* vsrc = reinterpret_cast<const uint4*>(p.vc + base + static_cast<size_t>(lo) * kHD);
    const int total = ncache * 8;
    const unsigned ks_s = smem_addr(ks), vs_s = smem_addr(vs);
    for (int i = tid; i < total; i += kAttnThreads)  // K first: the scores wait for it alone
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ks_s + swz(i >> 3, i & 7)), "l"(ksrc + i)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int i = tid; i < total; i += kAttnThreads)  // V lands while the scores run
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(vs_s + swz(i >> 3, i & 7)), "l"(vsrc + i)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int i = n * 8 + tid; i < rows * 8; i += kAttnThreads)
      *reinterpret_cast<uint4*>(vs + swz(i >> 3, i & 7)) = make_uint4(0u, 0u, 0u, 0u);
  }
  if (owns_new && tid < 16) {  // append: 8 x 16 bytes of K, 8 of V, to the cache and to the tiles
    const int ch = tid & 7;
    const bool is_v = tid >= 8;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>((is_v ? p.v_new : p.k_new) + kvh * kHD) + ch);
    reinterpret_cast<uint4*>((is_v ? p.vc : p.kc) + base + static_cast<size_t>(len) * kHD)[ch] = v;
    *reinterpret_cast<uint4*>((is_v ? vs : ks) + swz(ncache, ch)) = v;
  }
  // q as the A fragments of the four 16-dimension steps: head rows g and g + 8
  // (zero beyond the group), dimensions 16 kk + 2 t (+ 8).
  const int g = lane >> 2, t4 = lane & 3;
  unsigned qa[4][4];
  {
    const unsigned* q0 = reinterpret_cast<const unsigned*>(p.q + (kvh * group + g) * kHD);
    const unsigned* q1 = reinterpret_cast<const unsigned*>(p.q + (kvh * group + g + 8) * kHD);
    const bool r0 = g < group, r1 = g + 8 < group;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      qa[kk][0] = r0 ? __ldg(q0 + 8 * kk + t4) : 0u;
      qa[kk][1] = r1 ? __ldg(q1 + 8 * kk + t4) : 0u;
      qa[kk][2] = r0 ? __ldg(q0 + 8 * kk + 4 + t4) : 0u;
      qa[kk][3] = r1 ? __ldg(q1 + 8 * kk + 4 + t4) : 0u;
    }
  }
  asm volatile("cp.async.wait_group 1;" ::: "memory");  // this thread's K copies
  __syncthreads();

  // ---- 2. scores S = (Q K^T) * scale on the tensor cores: warp w takes tokens
  // [w * tpw, (w + 1) * tpw) in 8-token tiles; tokens >= n are masked to -inf.
  const int j0w = warp * tpw;
  const bool active = j0w < n;  // warp-uniform
  const int ntile = tpw / 8;
  const unsigned ks0 = smem_addr(ks), vs0 = smem_addr(vs);
  float s[8][4];
  float mx0 = kNegInf, mx1 = kNegInf;
  if (active) {
#pragma unroll
    for (int tt = 0; tt < 8; ++tt) {
      if (tt < ntile) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int row = j0w + 8 * tt + (lane & 7);
#pragma unroll
        for (int kk = 0; kk < 4; kk += 2) {
          unsigned b[4];  // chunks 2kk .. 2kk + 3 of 8 token rows: B fragments of steps kk, kk + 1
          ldsm_x4(ks0 + swz(row, 2 * kk + (lane >> 3)), b);
          mma_bf16_16816(acc, qa[kk], b[0], b[1]);
          mma_bf16_16816(acc, qa[kk + 1], b[2], b[3]);
        }
        const int col = j0w + 8 * tt + 2 * t4;
#pragma unroll
        for (int e = 0; e < 4; ++e) s[tt][e] = col + (e & 1) < n ? __fmul_rn(acc[e], p.scale) : kNegInf;
        mx0 = fmaxf(mx0, fmaxf(s[tt][0], s[tt][1]));
        mx1 = fmaxf(mx1, fmaxf(s[tt][2], s[tt][3]));
      }
    }
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  if (t4 == 0) {
    wmax[warp * 16 + g] = mx0;
    wmax[warp * 16 + g + 8] = mx1;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");  // this thread's V copies
  __syncthreads();

  // ---- 3. p = exp(s - m) in registers; per-warp row sums
  float m0 = kNegInf, m1 = kNegInf;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    m0 = fmaxf(m0, wmax[w * 16 + g]);
    m1 = fmaxf(m1, wmax[w * 16 + g + 8]);
  }
  float l0 = 0.0f, l1 = 0.0f;
  float o[8][4];
#pragma unroll
  for (int nd = 0; nd < 8; ++nd)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[nd][e] = 0.0f;
  if (active) {
#pragma unroll
    for (int tt = 0; tt < 8; ++tt) {
      if (tt < ntile) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float m = e < 2 ? m0 : m1;
          s[tt][e] = s[tt][e] == kNegInf ? 0.0f : __expf(__fsub_rn(s[tt][e], m));
        }
        l0 = __fadd_rn(l0, __fadd_rn(s[tt][0], s[tt][1]));
        l1 = __fadd_rn(l1, __fadd_rn(s[tt][2], s[tt][3]));
      }
    }
    // ---- 4. O = P V on the tensor cores: P (16 heads x 16 tokens) as hi + lo
    // BF16 A fragments straight from the score accumulators; V B fragments by
    // transposing loads of the swizzled tile.
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
      if (2 * kt < ntile) {
        unsigned ahi[4], alo[4];
        split_bf16x2(s[2 * kt][0], s[2 * kt][1], ahi[0], alo[0]);
        split_bf16x2(s[2 * kt][2], s[2 * kt][3], ahi[1], alo[1]);
        split_bf16x2(s[2 * kt + 1][0], s[2 * kt + 1][1], ahi[2], alo[2]);
        split_bf16x2(s[2 * kt + 1][2], s[2 * kt + 1][3], ahi[3], alo[3]);
        const int mi = lane >> 3;
        const int row = j0w + 16 * kt + (lane & 7) + ((mi & 1) << 3);
#pragma unroll
        for (int nd = 0; nd < 8; nd += 2) {
          unsigned b[4];  // dims 8 nd .. 8 nd + 15: B fragments of output tiles nd, nd + 1
          ldsm_x4_trans(vs0 + swz(row, nd + (mi >> 1)), b);
          mma_bf16_16816(o[nd], ahi, b[0], b[1]);
          mma_bf16_16816(o[nd], alo, b[0], b[1]);
          mma_bf16_16816(o[nd + 1], ahi, b[2], b[3]);
          mma_bf16_16816(o[nd + 1], alo, b[2], b[3]);
        }
      }
    }
  }
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 1));
  l0 = __fadd_rn(l0, __shfl_xor_sync(0xffffffffu, l0, 2));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 1));
  l1 = __fadd_rn(l1, __shfl_xor_sync(0xffffffffu, l1, 2));
  if (t4 == 0) {
    wsum[warp * 16 + g] = l0;
    wsum[warp * 16 + g + 8] = l1;
  }
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) {
    float* r0 = red + (warp * 16 + g) * kRedStride + 8 * nd + 2 * t4;
    *reinterpret_cast<float2*>(r0) = make_float2(o[nd][0], o[nd][1]);
    *reinterpret_cast<float2*>(r0 + 8 * kRedStride) = make_float2(o[nd][2], o[nd][3]);
  }
  __syncthreads();
  if (tid < group) {  // m and l per head row, warps summed in order
    float m = kNegInf, l = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      m = fmaxf(m, wmax[w * 16 + tid]);
      l = __fadd_rn(l, wsum[w * 16 + tid]);
    }
    ml[2 * tid] = m;
    ml[2 * tid + 1] = l;
  }
  __syncthreads();
  for (int it = tid; it < group * kHD; it += kAttnThreads) {  // o per (head, dim): warps in order
    const int h = it / kHD, d = it - h * kHD;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) acc = __fadd_rn(acc, red[(w * 16 + h) * kRedStride + d]);
    if (splits == 1) {
      p.out[(kvh * group + h) * kHD + d] = rne_bf16(__fdiv_rn(acc, ml[2 * h + 1]));
    } else {
      float* rec = kCluster ? part + h * kRecord
                            : p.scratch + (static_cast<size_t>(kvh * group + h) * splits + c) * kRecord;
      rec[2 + d] = acc;
      if (d == 0) {
        const bool any = n > 0;
        rec[0] = any ? ml[2 * h] : kNegInf;
        rec[1] = any ? ml[2 * h + 1] : 0.0f;
      }
    }
  }
  if (splits == 1) return;

  // ---- 5. merge
  if constexpr (kCluster) {
    cluster_sync_all();  // every split's record is in its CTA's shared memory
    const unsigned part0 = smem_addr(part);
    for (int it = c * kAttnThreads + tid; it < group * kHD; it += splits * kAttnThreads) {
      const int h = it / kHD, d = it - h * kHD;
      const unsigned off = part0 + static_cast<unsigned>(h * kRecord) * 4u;
      float mk[kMaxClusterSplits], lk[kMaxClusterSplits], ok[kMaxClusterSplits];
#pragma unroll
      for (int k = 0; k < kMaxClusterSplits; ++k) {  // all loads issued before any is used
        if (k < splits) {
          const unsigned a = cluster_map(off, k);
          mk[k] = ld_cluster_f32(a);
          lk[k] = ld_cluster_f32(a + 4);
          ok[k] = ld_cluster_f32(a + 8 + 4 * d);
        }
      }
      float gm = __int_as_float(0xff800000u);
#pragma unroll
      for (int k = 0; k < kMaxClusterSplits; ++k)
        if (k < splits && lk[k] > 0.0f) gm = fmaxf(gm, mk[k]);
      float num = 0.0f, den = 0.0f;
#pragma unroll
      for (int k = 0; k < kMaxClusterSplits; ++k) {
        if (k < splits && lk[k] > 0.0f) {  // empty tiles (l = 0) carry no weight
          const float w = __expf(__fsub_rn(mk[k], gm));
          num = __fmaf_rn(w, ok[k], num);
          den = __fmaf_rn(w, lk[k], den);
        }
      }
      p.out[(kvh * group + h) * kHD + d] = rne_bf16(__fdiv_rn(num, den));
    }
    cluster_sync_all();  // no CTA leaves while another reads its shared memory
  } else {
    unsigned* s_ticket = reinterpret_cast<unsigned*>(smem + L.tk);
    float* wts = reinterpret_cast<float*>(smem + L.wts);
    __threadfence();
    __syncthreads();
    if (tid == 0) *s_ticket = atomicAdd(p.tickets + kvh, 1u);
    __syncthreads();
    if (*s_ticket != static_cast<unsigned>(splits - 1)) return;
    __threadfence();
    const float* recs = p.scratch + static_cast<size_t>(kvh * group) * splits * kRecord;
    for (int i = tid; i < group * splits; i += kAttnThreads) {
      const float2 v = __ldcg(reinterpret_cast<const float2*>(recs + static_cast<size_t>(i) * kRecord));
      wts[2 * i] = v.x;
      wts[2 * i + 1] = v.y;
    }
    __syncthreads();
    for (int h = warp; h < group; h += kWarps) {
      float gm = __int_as_float(0xff800000u);
      for (int k = lane; k < splits; k += 32)
        if (wts[2 * (h * splits + k) + 1] > 0.0f) gm = fmaxf(gm, wts[2 * (h * splits + k)]);
      gm = warp_max(gm);
      float den = 0.0f;
      for (int k = lane; k < splits; k += 32) {
        float* wk = wts + 2 * (h * splits + k);
        const float lk = wk[1];
        const float w = lk > 0.0f ? __expf(__fsub_rn(wk[0], gm)) : 0.0f;
        wk[0] = w;
        den = __fmaf_rn(w, lk, den);
      }
      den = warp_allsum(den);
      if (lane == 0) ml[2 * h + 1] = den;
    }
    __syncthreads();
    // Thread (head, dimension) x split class; classes summed in order through `red`.
    const int items = group * kHD;
    const int classes = items >= kAttnThreads ? 1 : kAttnThreads / items;
    for (int t = tid; t < items * classes; t += kAttnThreads) {
      const int item = t % items, k0 = t / items;
      const int h = item / kHD, d = item - h * kHD;
      const float* ph = recs + static_cast<size_t>(h) * splits * kRecord + 2 + d;
      float a = 0.0f;
#pragma unroll 4
      for (int k = k0; k < splits; k += classes)
        a = __fmaf_rn(wts[2 * (h * splits + k)], __ldcg(ph + static_cast<size_t>(k) * kRecord), a);
      if (classes == 1)
        p.out[(kvh * group + h) * kHD + d] = rne_bf16(__fdiv_rn(a, ml[2 * h + 1]));
      else
        red[t] = a;
    }
    if (classes > 1) {
      __syncthreads();
      for (int item = tid; item < items; item += kAttnThreads) {
        const int h = item / kHD;
        float a = 0.0f;
        for (int t = item; t < items * classes; t += items) a = __fadd_rn(a, red[t]);
        p.out[(kvh * group + h) * kHD + item - h * kHD] = rne_bf16(__fdiv_rn(a, ml[2 * h + 1]));
      }
    }
    if (tid == 0) p.tickets[kvh] = 0u;
  }
}

struct AttnDevice {
  std::atomic<bool> ready;
  int sms;
  int cluster_max;  // largest cluster the cluster mode may use on this device
};
AttnDevice g_attn_dev[64];

// Short spans (<= 384 tokens) run as one tile per kv head with no merge. Longer
// spans: tiles of at least 128 tokens, cluster mode whenever one cluster of
// `splits` CTAs covers the span with tiles of at most 512 tokens; the split count
// aims at about two CTAs per SM. (Measured on B200 at 32/8 heads: 256 tokens as one
// tile 4.7 us vs four 64-token tiles 5.4 us; 384 tokens as one tile 4.9 us vs three
// 128-token tiles 5.2 us, but 512 tokens as one tile 5.5 us vs four 5.2 us; 1024
// tokens as 8 x 128 6.2 us vs 16 x 64 6.8 us.)
struct AttnPlan {
  int splits, tile;
  bool cluster;
};

AttnPlan plan_for(int span, int kv_heads, const AttnDevice& dev) {
  if (span <= KLAB_ATTN_SINGLE_SPAN) return {1, (span + 63) / 64 * 64, true};
  const int want = (2 * dev.sms) / kv_heads > 1 ? (2 * dev.sms) / kv_heads : 1;
  int splits = (span + kMinTile - 1) / kMinTile;
  if (splits > want) splits = want;
  AttnPlan plan{};
  const int csplits = splits < dev.cluster_max ? splits : dev.cluster_max;
  int tile = ((span + csplits - 1) / csplits + kMinTile - 1) / kMinTile * kMinTile;
  if (KLAB_ATTN_CLUSTER && tile <= kMaxTile) {
    plan.tile = tile;
    plan.splits = (span + tile - 1) / tile;
    plan.cluster = true;
    return plan;
  }
  tile = ((span + splits - 1) / splits + kMinTile - 1) / kMinTile * kMinTile;
  plan.tile = tile > kMaxTile ? kMaxTile : tile;
  plan.splits = (span + plan.tile - 1) / plan.tile;
  plan.cluster = false;
  return plan;
}

std::mutex g_attn_mutex;

// Once per device (the caller's device is current): kernel attributes, SM count and
// the largest usable cluster. Guarded so concurrent first calls do it once.
int prepare_device(int dev) {
  AttnDevice& d = g_attn_dev[dev];
  if (d.ready.load(std::memory_order_acquire)) return 0;
  std::lock_guard<std::mutex> lock(g_attn_mutex);
  if (d.ready.load(std::memory_order_relaxed)) return 0;
  cudaError_t err = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(decode_attn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kMaxSmem));
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(decode_attn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kMaxSmem));
  if (err != cudaSuccess) return err;
  d.cluster_max = 8;  // portable cluster size
  if (cudaFuncSetAttribute(decode_attn_kernel<true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
      cudaSuccess) {
    // 16 when a 16-CTA cluster of the largest cluster-mode footprint can be resident.
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kMaxClusterSplits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(kMaxClusterSplits);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = layout_for(kMaxTile, kMaxGroup, kMaxClusterSplits, false).total;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, decode_attn_kernel<true>, &cfg) == cudaSuccess && clusters > 0)
      d.cluster_max = kMaxClusterSplits;
  }
  (void)cudaGetLastError();
  d.ready.store(true, std::memory_order_release);
  return 0;
}

}  // namespace
}  // namespace klab

extern "C" {

KLAB_API int klab_decode_attention(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                                   void* out, float* scratch, long long scratch_floats, unsigned* tickets,
                                   const int* len_ptr, int len, int max_len, int heads, int kv_heads, float scale,
                                   void* stream) {
  using namespace klab;
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !out || !scratch || !tickets) return KLAB_E_INVALID;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > kMaxGroup || max_len <= 0 ||
      max_len > kMaxSpan)
    return KLAB_E_SHAPE;
  if (!len_ptr && (len < 0 || len + 1 > max_len)) return KLAB_E_SHAPE;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_new) |
                        reinterpret_cast<uintptr_t>(v_new) | reinterpret_cast<uintptr_t>(k_cache) |
                        reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(out) |
                        reinterpret_cast<uintptr_t>(scratch);
  if (mis & 15) return KLAB_E_ALIGN;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return KLAB_E_UNSUPPORTED;
  const int prep = prepare_device(dev);
  if (prep) return prep;
  const AttnPlan plan = plan_for(len_ptr ? max_len : len + 1, kv_heads, g_attn_dev[dev]);
  if (static_cast<long long>(heads) * plan.splits * kRecord > scratch_floats) return KLAB_E_INVALID;
  size_t smem = layout_for(plan.tile, heads / kv_heads, plan.splits, !plan.cluster).total;
  if (smem < KLAB_ATTN_SMEM_FLOOR) smem = KLAB_ATTN_SMEM_FLOOR;
  if (smem > kMaxSmem) return KLAB_E_SHAPE;
  AttnParams p{};
  p.q = static_cast<const unsigned short*>(q);
  p.k_new = static_cast<const unsigned short*>(k_new);
  p.v_new = static_cast<const unsigned short*>(v_new);
  p.kc = static_cast<unsigned short*>(k_cache);
  p.vc = static_cast<unsigned short*>(v_cache);
  p.out = static_cast<unsigned short*>(out);
  p.scratch = scratch;
  p.tickets = tickets;
  p.len_ptr = len_ptr;
  p.status = device_status_address();
  p.len_value = len;
  p.max_len = max_len;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.splits = plan.splits;
  p.tile = plan.tile;
  p.tpw = tokens_per_warp(plan.tile);
  p.scale = scale;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  cfg.gridDim = dim3(static_cast<unsigned>(kv_heads * plan.splits));
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  if (klab_get_option(KLAB_OPT_PDL)) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (plan.cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(plan.splits);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return plan.cluster ? cudaLaunchKernelEx(&cfg, decode_attn_kernel<true>, p)
                      : cudaLaunchKernelEx(&cfg, decode_attn_kernel<false>, p);
}

}  // extern "C"
