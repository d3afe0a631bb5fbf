/* klab_b200: C ABI of the B200-native small-batch projection path.
 *
 * Plain pointers, sizes and a CUDA stream handle; no C++ or framework types.
 * All device pointers are caller-owned; every call enqueues asynchronously on
 * `stream` (a cudaStream_t, NULL = legacy default stream) of the current CUDA
 * device and never synchronizes. Return value: 0 on success, a positive
 * cudaError_t, or a negative KLAB_E* code below. Output layout is
 * out[t * ldo + row] for token t and output row `row` (ldo = N for a dense
 * [M, N] result; a larger ldo writes into a column slice of a wider buffer).
 *
 * Numerics (every projection): FP32 accumulation with fma.rn, a fixed
 * reduction order that depends only on K and the weight format, and one final
 * cvt.rn.bf16.f32 for BF16 outputs. Coded (lossless) BF16 weights give
 * bit-identical results to the same weights stored raw; any subset of output
 * rows (a column shard) gives bit-identical values to the full projection.
 *
 * Workspace: projections may split K across thread blocks when N is small.
 * That needs `workspace` of klab_gemv_workspace_bytes(...) bytes (16-byte
 * aligned), zero-filled once before first use and then left alone: its first
 * 64 KiB hold completion tickets that every launch leaves zeroed, the rest is
 * scratch for partial sums. Pass NULL / 0 to disable splitting; results are
 * identical either way. One workspace must not be used by launches that can
 * run concurrently.
 */
#ifndef KLAB_B200_H
#define KLAB_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KLAB_API __attribute__((visibility("default")))
#else
#define KLAB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- codes */

/* Element types of activations and outputs. */
#define KLAB_DT_BF16 0
#define KLAB_DT_F16 1
#define KLAB_DT_F32 2

/* Weight formats (klab_gemv wfmt). */
#define KLAB_W_BF16 0      /* BF16 [N,K] */
#define KLAB_W_F16 1       /* FP16 [N,K] */
#define KLAB_W_F32 2       /* FP32 [N,K] */
#define KLAB_W_CBF16 3     /* lossless BF16 codec v1: payload u8 + metadata u32 [N*ceil(K/64)] */
#define KLAB_W_I8_ROW 4    /* int8 [N,K] + fp32 scale [N] */
#define KLAB_W_I8_G64 5    /* int8 [N,K] + fp32 scale [N,K/64] */
#define KLAB_W_FP4_G32H 6  /* E2M1 [N,K/2] (low nibble = even k) + fp16 scale [N,K/32] */
#define KLAB_W_FP4_G16E 7  /* E2M1 [N,K/2] + E4M3 scale [N,K/16] + fp32 global scale */
#define KLAB_W_LF32 8      /* lossless FP32 v1: 3-byte mantissa + exponent stream (lossless_weights.py) */
#define KLAB_W_FP28 9      /* lossless FP32 as 28-bit codes (packed_fp32.py) */

/* FP4 scale kinds (klab_fp4_linear / klab_fp4_dequantize). */
#define KLAB_FP4_E4M3_G16 0
#define KLAB_FP4_F16_G32 1

/* L2 prefetch kinds (klab_l2_prefetch). */
#define KLAB_L2_HINT 0
#define KLAB_L2_HINT_LAST 1
#define KLAB_L2_LOAD 2
#define KLAB_L2_BULK 3 /* this library's own: cp.async.bulk.prefetch.L2, `stride` = bytes per request */

/* Error codes. -1000..-1002 keep the meaning of the reference driver ABI. */
#define KLAB_E_DRIVER (-1000)      /* CUDA driver or a required symbol not loadable */
#define KLAB_E_NO_CONTEXT (-1001)  /* no current CUDA context */
#define KLAB_E_INVALID (-1002)     /* null argument or zero/negative dimension */
#define KLAB_E_SHAPE (-2001)       /* shape not supported by this format */
#define KLAB_E_ALIGN (-2002)       /* pointer/stride alignment not supported */
#define KLAB_E_UNSUPPORTED (-2003) /* dtype/format combination not supported */
#define KLAB_E_DEVICE (-2004)      /* a kernel recorded a device-side error (bounded wait expired) */
#define KLAB_E_SCRATCH (-2005)     /* the shape needs more than the library's static 4 MiB scratch */

/* Options (klab_set_option). */
#define KLAB_OPT_PDL 0        /* 1 (default): launch with programmatic dependent launch */
#define KLAB_OPT_SPLIT 1      /* -1 (default) automatic, 0 never, 1 always (when workspace allows) */
#define KLAB_OPT_GENERIC 2    /* 1: force the cooperative-load (non bulk-copy) fill path */
#define KLAB_OPT_CTAS_PER_SM 3 /* cap on projection CTAs per SM (0, default: as many as fit) */
#define KLAB_OPT_TENSOR 4      /* tensor-core routes: 0 never (CUDA cores only); 1 (default) warp-level
                                  tensor-core token tiles for INT8 per-row at M = 2..8 and E2M1/FP16-per-32
                                  at M = 2..16 (BF16/FP16 x), INT8 per-row at M > 8 on tcgen05, M = 1 on the
                                  CUDA cores; 2 INT8 per-row and BF16 weights at M >= 2 on tcgen05; 3 the
                                  token tiles at every M <= 16 (results independent of M), tcgen05 above */
#define KLAB_OPT_PROLOGUE 5    /* weight copies issued before the previous launch completes, per warp:
                                  (items into shared memory) + 16 * (items prefetched into L2);
                                  each part 0..3, -1 (default) the tuned choice */
#define KLAB_OPT_MAX_TILE 6    /* largest token tile of the CUDA-core projection kernel: 1, 2, 4 (default) or 8;
                                  results are the same bits for every tile */

/* ---------------------------------------------------------------- projections */

/* Generic projection: out = x[M,K] . W^T for any weight format.
 * Replaces the per-format launches of the reference wrappers:
 *   compressed_bf16.py:421-460 (_coded, raw_linear), mtile_bf16.py:150-188 (_launch),
 *   int8_weights.py:38-67, fp4.py:63-97, half_projection.py:24-50,
 *   kernel_lab.py:197-279 (matmul / warp_matmul / tiled_matmul).
 * aux: coded metadata, or scales (per wfmt); gscale: device pointer (FP4_G16E only). */
KLAB_API int klab_gemv(int wfmt, int xdtype, const void* x, int ldx, const void* w, const void* aux,
              const float* gscale, void* out, int ldo, int out_dtype, int m, int n, int k,
              void* workspace, size_t workspace_bytes, void* stream);

/* Several projections that read the same x[M,K] in one launch: segment i has
 * n[i] output rows, weights w[i] (+ aux[i]) and writes out[i][t * ldo[i] + row].
 * 1 <= nseg <= 8. Every output equals the separate klab_gemv call bit for bit.
 * Fuses what the reference launches one projection at a time, e.g. the QKV /
 * gate-up groups of examples/kv_pair_projection.py:13-36. */
KLAB_API int klab_gemv_multi(int wfmt, int xdtype, const void* x, int ldx, int nseg, const void* const* w,
                             const void* const* aux, const float* gscale, void* const* out, const int* ldo,
                             const int* n, int out_dtype, int m, int k, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Lossless FP32 projections (FP32 x, FP32 out); results are bit-identical to
 * klab_f32_linear on the decoded weights. Replace lossless_weights.fused_linear
 * (lossless_weights.py:78-116, kernels lossless_t* in lossless_kernels.cu:41-65)
 * and packed_fp32.fused_linear (packed_fp32.py:70-88, kernels fp28_t* in
 * adaptive_kernels.cu:78-99). Formats: klab_b200/csrc/lossless_f32.cuh. */
KLAB_API int klab_lossless_f32_linear(const float* x, const uint8_t* mantissa, const uint8_t* exponents,
                                      const int32_t* metadata, float* out, int m, int n, int k, void* workspace,
                                      size_t workspace_bytes, void* stream);
KLAB_API int klab_fp28_linear(const float* x, const int32_t* payload, const int32_t* metadata, float* out, int m,
                              int n, int k, void* workspace, size_t workspace_bytes, void* stream);
/* Decode to FP32 [count] (count % 64 == 0): lossless_unpack / fp28_unpack
 * (lossless_kernels.cu:31-37, adaptive_kernels.cu:70-75). */
KLAB_API int klab_lossless_f32_unpack(const uint8_t* mantissa, const uint8_t* exponents, const int32_t* metadata,
                                      float* out, long long count, void* stream);
KLAB_API int klab_fp28_unpack(const int32_t* payload, const int32_t* metadata, float* out, long long count,
                              void* stream);

/* Prepared projection plans: validate a (format, x dtype, out dtype, M, N, K)
 * case once and freeze its launch (token tile, x staging, grid, split-K, the
 * split-K workspace, owned by the plan); launches then only bind pointers.
 * Replaces the reference's native plan registry (native/prepared.cpp:155-413:
 * make_plan / register_plan / launch / raw / coded), whose kernel name and grid
 * are likewise a pure function of the prepared case. Pointers passed to
 * klab_plan_launch must be 16-byte aligned (coded payload 32-byte); aux is the
 * format's side data (metadata or scales), aux2 the W_LF32 exponent stream.
 * Launches of one plan must not overlap on the GPU (they share its workspace).
 * The plan belongs to the device that was current at klab_plan_create. */
KLAB_API int klab_plan_create(int wfmt, int xdtype, int out_dtype, int m, int n, int k, void** plan);
KLAB_API int klab_plan_launch(void* plan, const void* x, const void* w, const void* aux, const void* aux2,
                              const float* gscale, void* out, void* stream);
/* JSON description of the frozen launch into buffer (NUL-terminated). */
KLAB_API int klab_plan_info(void* plan, char* buffer, size_t bytes);
KLAB_API int klab_plan_destroy(void* plan);

/* Output gather fused into a projection, over NVLink peer memory (no
 * counterpart in the reference, which has no multi-GPU code; it replaces the
 * per-layer NCCL all-gather of the sharded chain). Segment `seg`'s outputs are
 * also stored into each rank's copy of its output buffer (peer_out, mapped with
 * klab_ipc_open); after the grid, this rank's flag (slot signal_slot) is raised
 * to *epoch on every rank. With wait_flags set, the launch first waits
 * (bounded) until all npeers flags of wait_slot reach *epoch before reading x.
 * Flag arrays are [slots][npeers] u32, monotonic, zero at start. `done` is a
 * device word that is zero between launches. */
typedef struct klab_gather {
  int npeers;
  int rank;
  int seg;
  void* peer_out[8];
  unsigned* peer_flags[8];
  int signal_slot;
  const unsigned* wait_flags;
  int wait_slot;
  const unsigned* epoch;
  unsigned* done;
} klab_gather_t;

/* klab_gemv_multi with a fused output gather (gather may be NULL). */
KLAB_API int klab_gemv_multi_gather(int wfmt, int xdtype, const void* x, int ldx, int nseg, const void* const* w,
                                    const void* const* aux, const float* gscale, void* const* out, const int* ldo,
                                    const int* n, int out_dtype, int m, int k, const klab_gather_t* gather,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Peer memory for the fused gather (CUDA IPC, one node): allocate a zero-filled
 * buffer and its 64-byte IPC handle; map a peer's handle; unmap; free. */
KLAB_API int klab_ipc_malloc(size_t bytes, void** ptr, void* handle64);
KLAB_API int klab_ipc_open(const void* handle64, void** ptr);
KLAB_API int klab_ipc_close(void* ptr);
KLAB_API int klab_ipc_free(void* ptr);
/* Start a gathered step: *epoch += 1 on `stream` (one thread). */
KLAB_API int klab_step_begin(unsigned* epoch, void* stream);
/* Wait (bounded, on the device) until all npeers flags of `slot` reach *epoch. */
KLAB_API int klab_wait_flags(const unsigned* flags, int slot, int npeers, const unsigned* epoch, void* stream);

/* Persistent projection chain (no counterpart in the reference, whose chain is
 * one launch per projection, l2prefetch.py:38-60): every projection of a token
 * step in ONE cooperative launch, BF16 weights, one token. Stage s computes
 * the rows of its nseg weights w[i] [n[i], k] from the input x: the plain BF16
 * step input when x_stage = -1, else the local gather buffer of stage x_stage
 * (an earlier stage). A stage's gather segment (gather_seg, -1: none) is
 * written as 32-bit words (tag << 16 | bf16) into every rank's gather buffer
 * (peer_out[q], rank q's buffer at this rank's first row; peer_out[rank] is the
 * local one), over NVLink for the peers; other segments write plain BF16 to
 * out[i]. A stage that rewrites a gather buffer must take its input from a
 * stage after every reader of the buffer's previous content; every stage must
 * have at least as many row x 2048-column items as the GPU has SMs. Gather
 * buffers start zeroed. sync->final_in is the last gathering stage's local
 * buffer; the launch ends after its plain BF16 values are in final_out. epoch
 * (device u32, zero at start) counts completed steps. Outputs are
 * bit-identical to one klab_gemv_multi launch per stage. One GPU: npeers = 1. */
typedef struct klab_chain_stage {
  const void* x;
  int k;
  int nseg;
  const void* w[8];
  void* out[8];
  int n[8];
  int gather_seg;
  void* peer_out[8];
  int x_stage;
} klab_chain_stage_t;

typedef struct klab_chain_sync {
  int npeers;
  int rank;
  unsigned* epoch;
  const unsigned* final_in;
  void* final_out;
} klab_chain_sync_t;

/* Validate the stages once and upload them (call outside graph capture). */
KLAB_API int klab_chain_create(const klab_chain_stage_t* stages, int nstages, const klab_chain_sync_t* sync,
                               void** plan);
/* One token step: a single kernel launch on `stream` (capturable). */
KLAB_API int klab_chain_launch(void* plan, void* stream);
KLAB_API int klab_chain_destroy(void* plan);
/* Launch shape of a plan: CTAs and trace slots per (stage, CTA). */
KLAB_API int klab_chain_info(void* plan, int* grid, int* trace_slots);
/* Optional timeline: later launches write global-timer ns per (stage, CTA):
 * [entered, previous stage done in this CTA, x staged, then each warp's last
 * item] into buffer
 * [nstages][grid][trace_slots] u64 (NULL: off). */
KLAB_API int klab_chain_trace(void* plan, unsigned long long* buffer, size_t bytes);

/* BF16 x, raw BF16 W, BF16 or FP32 out.
 * Replaces compressed_bf16.raw_linear (compressed_bf16.py:450-460, kernels
 * cbf16_raw_{bf16,fp32}_t*_v*, compressed_kernels.cu:156-176) and
 * mtile_bf16.raw_linear (mtile_bf16.py:177-188, mtbf16_raw_*, mtile_kernels.cu:122-144). */
KLAB_API int klab_raw_linear(const void* x, const void* w, void* out, int out_dtype, int m, int n, int k,
                    void* workspace, size_t workspace_bytes, void* stream);

/* BF16 x, lossless-coded BF16 W (payload 32-byte aligned, K % 64 == 0).
 * Replaces compressed_bf16._coded / fused_linear (compressed_bf16.py:421-447,
 * cbf16_coded_*) and mtile_bf16.fused_linear (mtile_bf16.py:161-174, mtbf16_coded_*). */
KLAB_API int klab_coded_linear(const void* x, const void* payload, const uint32_t* metadata, void* out,
                      int out_dtype, int m, int n, int k, void* workspace, size_t workspace_bytes,
                      void* stream);

/* x and W both FP16 or both BF16 (dtype), FP32 out.
 * Replaces half_projection.fused_linear (half_projection.py:24-50, half_warp_*,
 * half_kernels.cu:63-80). */
KLAB_API int klab_half_linear(const void* x, const void* w, int dtype, float* out, int m, int n, int k,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Decode elementwise ops, BF16 rows (two values per 32-bit word, d and inter even).
 * x_out = RNE(res + y); xn_out = RNE(x * rsqrt(mean(x^2, row) + eps) * weight), in the
 * reference kernel's order. Replaces add_rmsnorm_bf16 behind decode_attn.add_rmsnorm
 * (research/l2-prefetch/src/decode_attn.cu:471-511, decode_attn.py:64-71). */
KLAB_API int klab_add_rmsnorm(const void* res, const void* y, const void* weight, void* x_out, void* xn_out, int m,
                              int d, float eps, void* stream);
/* gu[M, 2*inter] = [gate | up] -> out[M, inter] = RNE(silu(gate) * up). Replaces silu_mul_bf16
 * behind decode_attn.silu_mul (decode_attn.cu:513-527, decode_attn.py:74-81). */
KLAB_API int klab_silu_mul(const void* gu, void* out, int m, int inter, void* stream);

/* M=1 decode attention with the new K/V row appended: writes k_new/v_new at row `len` of each kv
 * head's cache and out = softmax(q K^T * scale) V over len + 1 tokens; q [heads*64], k_new/v_new
 * [kv_heads*64], caches [kv_heads, max_len, 64], BF16, 16-byte aligned (out and scratch too);
 * heads / kv_heads <= 16; max_len <= 65536. len_ptr (device int32), when not null, replaces len and
 * the launch shape depends on max_len only (graph replay with a growing length; a device length
 * outside [0, max_len) sets device status 3 and touches nothing). scratch: heads * ceil(max_len /
 * 64) * 66 floats always suffice (scratch_floats is checked); tickets: kv_heads zeroed words, left
 * zero; one stream at a time per scratch/tickets pair. Replaces decode_attn_v4/v4d/v5_bf16 behind
 * decode_attn.decode_attention(_dynamic) (research/l2-prefetch/src/decode_attn.cu:258-460,
 * decode_attn.py:20-107). */
KLAB_API int klab_decode_attention(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                                   void* out, float* scratch, long long scratch_floats, unsigned* tickets,
                                   const int* len_ptr, int len, int max_len, int heads, int kv_heads, float scale,
                                   void* stream);

/* Fused: the projection out[M,N] = xn . W^T (BF16 W [N,K], BF16 out) with xn computed while
 * x is staged, as klab_add_rmsnorm would (x_out, when not null, gets RNE(res + y)); bit-identical
 * to klab_add_rmsnorm followed by klab_raw_linear. K % 8 == 0. x_out and out must not overlap res,
 * y, norm_weight or each other (no in-place residual update: every CTA re-reads res and y while
 * another writes x_out); an overlap returns KLAB_E_INVALID. No counterpart kernel in the
 * reference: it fuses its add_rmsnorm_bf16 into the next projection (the "prologue fusion"
 * named beside kernels.cu:168-222 and decode_attn.cu:473). */
KLAB_API int klab_add_rmsnorm_linear(const void* res, const void* y, const void* norm_weight, float eps,
                                     const void* w, void* out, void* x_out, int m, int n, int k, void* workspace,
                                     size_t workspace_bytes, void* stream);
/* Fused: out[M,N] = silu_mul(gu) . W^T with gu [M, 2*inter], W [N, inter]; bit-identical to
 * klab_silu_mul followed by klab_raw_linear. inter % 8 == 0; out must not overlap gu
 * (KLAB_E_INVALID). No counterpart kernel in the
 * reference (fuses its silu_mul_bf16, decode_attn.cu:513-527, into the down projection). */
KLAB_API int klab_silu_mul_linear(const void* gu, const void* w, void* out, int m, int n, int inter,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* out[M,K] = ((x + residual) * rsqrt(mean((x + residual)^2, row) + eps)) * weight[K],
 * FP32, 1 <= K <= 8192, eps > 0. Replaces KernelLab.residual_rmsnorm and the op
 * kernel_lab::residual_rmsnorm (kernel_lab.py:281-294, 343-353; kernels.cu:168-222). */
KLAB_API int klab_residual_rmsnorm(const float* x, const float* residual, const float* weight, float* out, int m,
                                   int k, float eps, void* stream);

/* FP32 x, FP32 W, FP32 out.
 * Replaces KernelLab.matmul / warp_matmul / tiled_matmul / tiny_matmul
 * (kernel_lab.py:197-294, kernels.cu:13-166, adaptive_kernels.cu:3-41,
 * projection_kernels.cu:17-89). */
KLAB_API int klab_f32_linear(const float* x, const float* w, float* out, int m, int n, int k, void* workspace,
                    size_t workspace_bytes, void* stream);

/* int8 W with fp32 scales: group 64 -> scales [N,K/64] (reference format,
 * int8_weights.py:23-35), group 0 -> scales [N] (per-row). x BF16/FP16/FP32.
 * Replaces int8_weights.fused_linear (int8_weights.py:38-67, int8_a{16,32}_t*,
 * int8_kernels.cu:28-34). */
KLAB_API int klab_int8_linear(const void* x, int xdtype, const int8_t* codes, const float* scales, int group,
                     void* out, int out_dtype, int m, int n, int k, void* workspace,
                     size_t workspace_bytes, void* stream);

/* E2M1 W, two per byte (low nibble = even k). scale_kind KLAB_FP4_E4M3_G16:
 * scales [N,K/16] E4M3 bytes and `gscale` one fp32 (reference format,
 * fp4.py:33-60); KLAB_FP4_F16_G32: scales [N,K/32] fp16, gscale unused.
 * Replaces fp4.fused_linear (fp4.py:63-97, fp4_a{16,32}_t*, fp4_kernels.cu:56-63). */
KLAB_API int klab_fp4_linear(const void* x, int xdtype, const uint8_t* packed, const void* scales,
                    int scale_kind, const float* gscale, void* out, int out_dtype, int m, int n, int k,
                    void* workspace, size_t workspace_bytes, void* stream);

/* klab_raw_linear without any allocation, for callers that cannot allocate
 * device memory (no framework allocator, a host application that owns all
 * device memory, a fixed-footprint process). Split-K scratch comes from a
 * static 4 MiB array inside the library (held by every GPU that loads it);
 * shapes whose scratch need (klab_gemv_workspace_bytes) exceeds 4 MiB return
 * KLAB_E_SCRATCH. The first call on a device looks up the array's address:
 * make it before any CUDA graph capture. Calls share the array: calls whose
 * kernels can overlap on the GPU race and must be serialized by the caller.
 * No counterpart in the reference (its kernels have no workspace). */
KLAB_API int klab_raw_linear_noalloc(const void* x, const void* w, void* out, int out_dtype, int m, int n, int k,
                                     void* stream);

/* Workspace bytes a klab_gemv call of this shape can use for split-K (0 = none);
 * for klab_gemv_multi pass the total row count as n. */
KLAB_API size_t klab_gemv_workspace_bytes(int wfmt, int m, int n, int k);

/* ---------------------------------------------------------------- decode */

/* Lossless BF16 codec v1 -> original uint16 bits [N,K] (any K).
 * Replaces compressed_bf16.unpack_weights (compressed_bf16.py:463-473,
 * cbf16_unpack, compressed_kernels.cu:181-200). */
KLAB_API int klab_cbf16_unpack(const void* payload, const uint32_t* metadata, uint16_t* out, int n, int k,
                      void* stream);

/* int8 -> fp32 [N,K] = code * scale (group 64 or 0 = per row).
 * Replaces Int8Weights.dequantize (int8_weights.py:15-17). */
KLAB_API int klab_int8_dequantize(const int8_t* codes, const float* scales, int group, float* out, int n, int k,
                         void* stream);

/* E2M1 -> fp32 [N,K]; E4M3/16: e2m1 * (scale * gscale) (fp4.py:21-27); F16/32: e2m1 * scale.
 * Replaces FP4Weights.dequantize (fp4.py:21-27). */
KLAB_API int klab_fp4_dequantize(const uint8_t* packed, const void* scales, int scale_kind, const float* gscale,
                        float* out, int n, int k, void* stream);

/* Host-side codec (CPU, preparation time). Pack: writes N*ceil(K/64) metadata
 * words and sets *payload_bytes; writes the payload when `payload` is non-NULL
 * and payload_capacity is large enough (a NULL payload is a size query).
 * Replaces compressed_bf16.pack_bits (compressed_bf16.py:99-151). */
KLAB_API int klab_cbf16_pack_host(const uint16_t* bits, int n, int k, uint32_t* metadata, uint8_t* payload,
                                  size_t payload_capacity, size_t* payload_bytes);
/* Validated decode to [N,K] bits: canonical offsets, raw-block base zero,
 * exponent range and tail padding; KLAB_E_INVALID on malformed input.
 * Replaces the checks and decode of compressed_bf16._decoded_chunks / unpack_bits
 * (compressed_bf16.py:162-243). */
KLAB_API int klab_cbf16_unpack_host(const uint8_t* payload, size_t payload_bytes, const uint32_t* metadata, int n,
                                    int k, uint16_t* out);

/* ---------------------------------------------------------------- L2 prefetch */

/* Side-stream prefetch of [p, p + bytes) into L2 with `blocks` x `threads`
 * threads, one request per `stride` bytes; never writes. sink: a device word
 * (never written in practice). Replaces l2prefetch.prefetch
 * (research/l2-prefetch/src/l2prefetch.py:27-35; kernels l2_hint / l2_hint_last /
 * l2_load, prefetch_kernels.cu:3-25). KLAB_L2_BULK has no counterpart in the reference: each
 * thread hands `stride` bytes (16 B .. 64 KiB) at a time to the bulk-copy engine. */
KLAB_API int klab_l2_prefetch(const void* p, long long bytes, int blocks, int threads, int stride, int kind,
                     unsigned* sink, void* stream);

/* ---------------------------------------------------------------- control */

KLAB_API int klab_set_option(int option, int value);
KLAB_API int klab_get_option(int option);
/* Read the current device's status word (0 = no device-side error; 1 = a bulk copy wait gave up,
 * 2 = a peer flag wait gave up, 3 = a length read from device memory was out of range); clear it
 * when clear != 0. */
KLAB_API int klab_device_status(int clear);
KLAB_API const char* klab_error_string(int code);
KLAB_API int klab_version(void);

/* ---------------------------------------------------------------- driver ABI
 * The reference's C ABI over the CUDA driver (native/driver.cpp:46-90), same
 * signatures, error codes and threading: load an image (PTX, cubin or fatbin)
 * into the current context, look up a kernel, launch it on a stream. */
KLAB_API int lab_load_ptx(const char* image, void** module_out);                                 /* driver.cpp:46-57 */
KLAB_API int lab_get_kernel(void* module, const char* name, void** fn_out);                     /* driver.cpp:59-63 */
KLAB_API int lab_launch(void* fn, unsigned grid_x, unsigned grid_y, unsigned block_x, void* stream,
               void** args);                                                           /* driver.cpp:65-71 */
KLAB_API int lab_unload(void* module);                                                          /* driver.cpp:73-77 */
KLAB_API const char* lab_error_string(int code);                                                /* driver.cpp:79-90 */
/* Extension (no reference counterpart): dynamic shared memory and flags
 * (bit 0: programmatic dependent launch) for bulk-copy ring kernels. */
KLAB_API int lab_launch_ex(void* fn, unsigned grid_x, unsigned grid_y, unsigned block_x, unsigned smem_bytes,
                  unsigned flags, void* stream, void** args);
/* Load an image from a file path (cubins shipped beside the library). */
KLAB_API int lab_load_file(const char* path, void** module_out);

#ifdef __cplusplus
}
#endif

#endif /* KLAB_B200_H */
