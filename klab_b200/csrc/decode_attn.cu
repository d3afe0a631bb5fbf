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
//   1. K rows are loaded with coalesced 16-byte loads and stored XOR-swizzled
//      (chunk i of row r at chunk i ^ (r mod 8)); V rows arrive by one 1-D bulk
//      copy, overlapped with the scores. The CTA whose tile holds position `len`
//      writes the new K/V row into the cache and into its tile.
//   2. Scores: thread per token, four heads at a time. The swizzle keeps the K
//      reads conflict-free while every thread reads the same q chunk (broadcast).
//   3. Softmax partial (m, l): warp per head. p is stored [token][head].
//   4. o = sum_j p_j V_j: thread per (8-dimension chunk, token class), four heads
//      at a time (one 16-byte V read and one 16-byte p read per 32 FMAs); token
//      classes are summed in a fixed order (shuffles, then warps in order).
//   5. Merge of the splits with weights exp(m_c - max m):
//      - cluster mode (splits <= the cluster limit): the splits of one kv head
//        form a thread-block cluster; each CTA keeps (m, l, o[64]) per head in
//        shared memory and the cluster reads them over distributed shared memory;
//      - ticket mode (longer spans): records go to global scratch and the last
//        CTA of a kv head (atomic ticket) merges them and resets the ticket.
// FP32 arithmetic, the fast exp intrinsic, one RNE to BF16. A device length
// outside [0, capacity) leaves the caches and the output untouched and sets the
// device status word (kStatusBadLength).
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "klab_b200.h"
#include "klab_kernels.h"

namespace klab {
namespace {

constexpr int kHD = 64;             // head dimension
constexpr int kRowBytes = kHD * 2;  // one BF16 K or V row
#ifndef KLAB_ATTN_MIN_TILE
#define KLAB_ATTN_MIN_TILE 64  // smallest tile the planner cuts the span into (a multiple of 64)
#endif
constexpr int kMinTile = KLAB_ATTN_MIN_TILE;
constexpr int kMaxTile = 512;
constexpr int kMaxGroup = 16;       // query heads per kv head
constexpr int kAttnThreads = 256;
constexpr int kWarps = kAttnThreads / 32;
constexpr int kRecord = kHD + 2;    // (m, l, o[64]) per (head, split)
constexpr int kMaxSpan = 65536;
constexpr int kMaxClusterSplits = 16;  // the largest (non-portable) cluster
constexpr size_t kMaxSmem = 227 * 1024;

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
  float scale;
};

struct SmemLayout {
  size_t ks, vs, qs, sc, red, part, wts, ml, bar, total;
};

__host__ __device__ inline int group4(int group) { return (group + 3) & ~3; }

__host__ __device__ inline SmemLayout layout_for(int tile, int group, int splits, bool ticket) {
  const size_t g4 = group4(group);
  SmemLayout s;
  s.ks = 0;
  s.vs = s.ks + static_cast<size_t>(tile) * kRowBytes;
  s.qs = s.vs + static_cast<size_t>(tile) * kRowBytes;
  s.sc = s.qs + g4 * kHD * 4;
  s.red = s.sc + static_cast<size_t>(tile) * g4 * 4;
  s.part = s.red + static_cast<size_t>(kWarps) * 4 * kHD * 4;  // per warp: 4 heads x 64 dims
  s.wts = s.part + static_cast<size_t>(group) * kRecord * 4;
  s.ml = s.wts + (ticket ? 2 * static_cast<size_t>(group) * splits * 4 : 0);
  s.bar = (s.ml + 2 * kMaxGroup * 4 + 15) / 16 * 16;
  s.total = s.bar + 16;
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
  const int group = p.heads / p.kv_heads, g4 = group4(group);
  const SmemLayout L = layout_for(tile, group, splits, !kCluster);
  unsigned char* ks = smem + L.ks;
  unsigned char* vs = smem + L.vs;
  float* qs = reinterpret_cast<float*>(smem + L.qs);
  float* sc = reinterpret_cast<float*>(smem + L.sc);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* part = reinterpret_cast<float*>(smem + L.part);
  float* ml = reinterpret_cast<float*>(smem + L.ml);
  const unsigned bar = smem_addr(smem + L.bar);

  const int kvh = blockIdx.x / splits, c = blockIdx.x - kvh * splits;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t base = static_cast<size_t>(kvh) * p.max_len * kHD;  // element offset of this kv head's cache
  const int lo = c * tile;
  const int ncache = min(max(len - lo, 0), tile);                 // cached tokens [lo, lo + ncache)
  const bool owns_new = len >= lo && len < lo + tile;             // the new token is local token ncache
  const int n = ncache + (owns_new ? 1 : 0);

  // ---- 1. staging
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    if (ncache > 0) {
      const unsigned bytes = static_cast<unsigned>(ncache) * kRowBytes;
      mbar_arrive_expect_tx(bar, bytes);
      bulk_g2s(smem_addr(vs), p.vc + base + static_cast<size_t>(lo) * kHD, bytes, bar);
    }
  }
  {  // K: eight 16-byte loads in flight per thread, then the swizzled stores
    const uint4* src = reinterpret_cast<const uint4*>(p.kc + base + static_cast<size_t>(lo) * kHD);
    const int total = ncache * 8;
    for (int b = 0; b < total; b += 8 * kAttnThreads) {
      uint4 buf[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = b + u * kAttnThreads + tid;
        if (i < total) buf[u] = __ldg(src + i);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = b + u * kAttnThreads + tid;
        if (i < total) {
          const int r = i >> 3, ch = i & 7;
          *reinterpret_cast<uint4*>(ks + r * kRowBytes + ((ch ^ (r & 7)) << 4)) = buf[u];
        }
      }
    }
  }
  if (owns_new && tid < 16) {  // append: 8 x 16 bytes of K, 8 of V, to the cache and to the tile
    const int ch = tid & 7;
    const bool is_v = tid >= 8;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>((is_v ? p.v_new : p.k_new) + kvh * kHD) + ch);
    reinterpret_cast<uint4*>((is_v ? p.vc : p.kc) + base + static_cast<size_t>(len) * kHD)[ch] = v;
    if (is_v)
      reinterpret_cast<uint4*>(vs + ncache * kRowBytes)[ch] = v;
    else
      *reinterpret_cast<uint4*>(ks + ncache * kRowBytes + ((ch ^ (ncache & 7)) << 4)) = v;
  }
  for (int i = tid; i < g4 * kHD; i += kAttnThreads) {
    const int h = i / kHD;
    qs[i] = h < group ? __fmul_rn(bf16lo(p.q[(kvh * group) * kHD + i]), p.scale) : 0.0f;
  }
  __syncthreads();

  // ---- 2. scores s[j][h] = (q_h * scale) . k_j
  for (int j = tid; j < n; j += kAttnThreads) {
    const unsigned char* krow = ks + j * kRowBytes;
    for (int hb = 0; hb < g4; hb += 4) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int i = 0; i < kHD / 8; ++i) {
        const uint4 kv = *reinterpret_cast<const uint4*>(krow + ((i ^ (j & 7)) << 4));
        const float k8[8] = {bf16lo(kv.x), bf16hi(kv.x), bf16lo(kv.y), bf16hi(kv.y),
                             bf16lo(kv.z), bf16hi(kv.z), bf16lo(kv.w), bf16hi(kv.w)};
#pragma unroll
        for (int hh = 0; hh < 4; ++hh) {
          const float4 q0 = *reinterpret_cast<const float4*>(qs + (hb + hh) * kHD + 8 * i);
          const float4 q1 = *reinterpret_cast<const float4*>(qs + (hb + hh) * kHD + 8 * i + 4);
          float a = acc[hh];
          a = __fmaf_rn(q0.x, k8[0], a);
          a = __fmaf_rn(q0.y, k8[1], a);
          a = __fmaf_rn(q0.z, k8[2], a);
          a = __fmaf_rn(q0.w, k8[3], a);
          a = __fmaf_rn(q1.x, k8[4], a);
          a = __fmaf_rn(q1.y, k8[5], a);
          a = __fmaf_rn(q1.z, k8[6], a);
          a = __fmaf_rn(q1.w, k8[7], a);
          acc[hh] = a;
        }
      }
      *reinterpret_cast<float4*>(sc + j * g4 + hb) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
  }
  __syncthreads();

  // ---- 3. softmax partials; p replaces s (padded heads stay finite: p = 0)
  for (int h = warp; h < g4; h += kWarps) {
    if (h >= group) {
      for (int j = lane; j < n; j += 32) sc[j * g4 + h] = 0.0f;
      continue;
    }
    float m = __int_as_float(0xff800000u);
    for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[j * g4 + h]);
    m = warp_max(m);
    float l = 0.0f;
    for (int j = lane; j < n; j += 32) {
      const float e = __expf(__fsub_rn(sc[j * g4 + h], m));
      sc[j * g4 + h] = e;
      l = __fadd_rn(l, e);
    }
    l = warp_allsum(l);
    if (lane == 0) {
      ml[2 * h] = m;
      ml[2 * h + 1] = l;
    }
  }
  if (ncache > 0 && !mbar_wait(bar, 0)) record_status(p.status, kStatusMbarTimeout);
  __syncthreads();

  // ---- 4. o[h][d] = sum_j p[j][h] v[j][d]; thread (dc = 8-dim chunk, cls = token class)
  const int dc = tid & 7, cls = tid >> 3;
  for (int hb = 0; hb < g4; hb += 4) {
    float acc[4][8];
#pragma unroll
    for (int hh = 0; hh < 4; ++hh)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[hh][e] = 0.0f;
#pragma unroll 2
    for (int j = cls; j < n; j += kAttnThreads / 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(vs + j * kRowBytes + dc * 16);
      const float4 pj = *reinterpret_cast<const float4*>(sc + j * g4 + hb);
      const float v8[8] = {bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y),
                           bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)};
      const float pp[4] = {pj.x, pj.y, pj.z, pj.w};
#pragma unroll
      for (int hh = 0; hh < 4; ++hh)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[hh][e] = __fmaf_rn(pp[hh], v8[e], acc[hh][e]);
    }
    // Token classes of one warp: lanes dc, dc + 8, dc + 16, dc + 24.
#pragma unroll
    for (int hh = 0; hh < 4; ++hh)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float a = acc[hh][e];
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 8));
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 16));
        acc[hh][e] = a;
      }
    if (lane < 8) {
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        float4* dst = reinterpret_cast<float4*>(red + (warp * 4 + hh) * kHD + dc * 8);
        dst[0] = make_float4(acc[hh][0], acc[hh][1], acc[hh][2], acc[hh][3]);
        dst[1] = make_float4(acc[hh][4], acc[hh][5], acc[hh][6], acc[hh][7]);
      }
    }
    __syncthreads();
    {  // thread (hh, d): warps summed in order
      const int hh = tid >> 6, d = tid & 63, h = hb + hh;
      float o = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) o = __fadd_rn(o, red[(w * 4 + hh) * kHD + d]);
      if (h < group) {
        if (splits == 1) {
          p.out[(kvh * group + h) * kHD + d] = rne_bf16(__fdiv_rn(o, ml[2 * h + 1]));
        } else {
          float* rec = kCluster ? part + h * kRecord
                                : p.scratch + (static_cast<size_t>(kvh * group + h) * splits + c) * kRecord;
          rec[2 + d] = o;
          if (d == 0) {
            const bool any = n > 0;
            rec[0] = any ? ml[2 * h] : __int_as_float(0xff800000u);
            rec[1] = any ? ml[2 * h + 1] : 0.0f;
          }
        }
      }
    }
    __syncthreads();
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
    unsigned* s_ticket = reinterpret_cast<unsigned*>(smem + L.bar + 8);
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
  bool ready;
  int sms;
  int cluster_max;  // largest cluster the cluster mode may use on this device
};
AttnDevice g_attn_dev[64];

// Cluster mode whenever one cluster of `splits` CTAs covers the span with tiles
// of at most 512 tokens; the split count aims at about two CTAs per SM.
struct AttnPlan {
  int splits, tile;
  bool cluster;
};

AttnPlan plan_for(int span, int kv_heads, const AttnDevice& dev) {
  const int want = (2 * dev.sms) / kv_heads > 1 ? (2 * dev.sms) / kv_heads : 1;
  int splits = (span + kMinTile - 1) / kMinTile;
  if (splits > want) splits = want;
  AttnPlan plan{};
  const int csplits = splits < dev.cluster_max ? splits : dev.cluster_max;
  int tile = ((span + csplits - 1) / csplits + kMinTile - 1) / kMinTile * kMinTile;
  if (tile <= kMaxTile) {
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

int prepare_device(int dev) {
  AttnDevice& d = g_attn_dev[dev];
  if (d.ready) return 0;
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
  d.ready = true;
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
  const size_t smem = layout_for(plan.tile, heads / kv_heads, plan.splits, !plan.cluster).total;
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
