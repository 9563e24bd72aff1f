/*
 * prismyra_moe.h -- C ABI of the B200 (sm_100a) routed-expert MoE layer.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream handle (cudaStream_t passed as
 * void*; NULL = the legacy default stream), launches asynchronously on that stream, allocates nothing and
 * returns a status code (PM_OK = 0).  Scratch memory is caller-owned: size it with pm_moe_workspace_bytes and
 * pass it to the calls that need it.  No call synchronises the stream except pm_moe_read_status.
 *
 * Layouts (row-major, bf16 = 16-bit brain float bit pattern, e4m3 = float8 e4m3fn byte):
 *   x          bf16  [T, H]            hidden states of T tokens
 *   router_w   bf16  [E, H]            the router's projection weight (reference: block.gate.weight)
 *   logits     bf16  [T, E]
 *   topk_w     f32   [T, k]            renormalised routing weights;  topk_ids  i32 [T, k]
 *   w1         e4m3  [E, 2I, H]        gate rows 0..I-1, up rows I..2I-1 (reference: experts.gate_up_proj)
 *   w1_s       f32   [E, 2I/128, H/128] per 128x128 block multiplier (reference: gate_up_proj_scale_inv)
 *   w2         e4m3  [E, H, I]          (reference: experts.down_proj);  w2_s f32 [E, H/128, I/128]
 *   out        bf16  [T, H]            routed-expert output (the shared expert is not part of this layer)
 * Shape limits: H % 256 == 0, I % 128 == 0, 1 <= k <= 16, k <= E <= 256.  Pointers 16-byte aligned.
 *
 * The references cited beside each declaration are files of the Prismyra reference (prismyra/...) and of the
 * vLLM release it calls (vllm/...).
 */
#ifndef PRISMYRA_MOE_H
#define PRISMYRA_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *pm_stream_t;

enum pm_status {
    PM_OK = 0,
    PM_ERR_INVALID = 1,   /* a NULL pointer or negative size */
    PM_ERR_SHAPE = 2,     /* dimensions outside the supported set */
    PM_ERR_ALIGN = 3,     /* a pointer is not 16-byte aligned */
    PM_ERR_WORKSPACE = 4, /* workspace too small */
    PM_ERR_CUDA = 5,      /* a CUDA launch or driver call failed */
    PM_ERR_DEVICE = 6,    /* the current device is not sm_100 */
    PM_ERR_TIMEOUT = 7,   /* a kernel gave up on a bounded wait (reported by pm_moe_read_status) */
    PM_ERR_TOO_LARGE = 8  /* beyond the fixed scratch of pm_moe_align_noalloc */
};

enum pm_format { PM_FMT_FP8 = 0, PM_FMT_NVFP4 = 1 };

/* Workspace regions, for callers that want to inspect intermediates (pm_moe_workspace_region). */
enum pm_region {
    PM_WS_STATUS = 0,   /* i32 [4]: [0] = timeout flag, [2] = grid barrier of the few-token front end */
    PM_WS_LOGITS = 1,   /* bf16 [T, E] */
    PM_WS_TOPK_W = 2,   /* f32 [T, k] */
    PM_WS_TOPK_IDS = 3, /* i32 [T, k] */
    PM_WS_COUNTS = 4,   /* i32 [chunks, E] (not written when 512 <= T*k <= 4096: one-launch front end) */
    PM_WS_EXPERT_OFF = 5, /* i32 [E + 1] first slot of each expert, padded total last */
    PM_WS_SORTED = 6,   /* i32 [max_slots] flat index t*k+j per slot, T*k = padding */
    PM_WS_EXPERT_IDS = 7, /* i32 [max_slots / 128] expert of each 128-slot block */
    PM_WS_NUM_POST_PAD = 8, /* i32 [1] slots in use */
    PM_WS_A1 = 9,       /* e4m3 [max_slots, H] activations in slot order (NVFP4: packed e2m1 [max_slots, H/2]) */
    PM_WS_A1_SCALE = 10, /* f32 [max_slots, H/128] (NVFP4: e4m3 [max_slots, H/16]) */
    PM_WS_A2 = 11,      /* e4m3 [max_slots, I] down-projection input (NVFP4: packed e2m1 [max_slots, I/2]) */
    PM_WS_A2_SCALE = 12, /* f32 [max_slots, I/128] (NVFP4: e4m3 [max_slots, I/16]) */
    PM_WS_C3 = 13,      /* bf16 [T*k, H] weighted expert outputs per (token, slot) */
    PM_WS_SLOT_OF = 14, /* i32 [T*k] slot of each flat index (the inverse of PM_WS_SORTED) */
    PM_WS_ROUTER_PART = 15, /* f32 [H/256, T, E] router partial sums per 256-column chunk (small T; else empty) */
    PM_WS_SCHED = 16    /* i32 [1 + 2 * max_slots / 128] few-token GEMMs' work queue and per-block-half counters */
};

/* Version of this ABI; bumped on any incompatible change. */
int pm_moe_abi_version(void);
const char *pm_moe_status_string(int status);

/* Maximum slots after per-expert padding to 128: T*k + E*127, rounded up to 128
 * (vllm/model_executor/layers/fused_moe/moe_align_block_size.py:74 max_num_tokens_padded). */
int pm_moe_max_slots(int T, int E, int k);

/* Bytes of caller-owned scratch the layer needs for T tokens; the reference sizes its per-thread workspace
 * the same way from the token count (prismyra/kernels/nvfp4.py:213-245 FusedExpertsFp4._workspace). */
size_t pm_moe_workspace_bytes(int T, int H, int I, int E, int k, int fmt);
/* Offset and size of one region inside that workspace. */
int pm_moe_workspace_region(int T, int H, int I, int E, int k, int fmt, int region, size_t *offset, size_t *bytes);

/* Router projection + softmax + top-k + renormalise, row-count invariant.  Replaces
 * prismyra/kernels/qwen3_moe.py:169-171 (FusedExperts._route) followed by :196 (vllm fused_topk,
 * renormalize=True; vllm/model_executor/layers/fused_moe/router/fused_topk_router.py:69-113).
 * logits (bf16 [T, E], 16-byte aligned) receives the router's output and is read back by the ranking.  bias
 * (fp32 [E], may be NULL) is added to every logit before the ranking; it has no counterpart in the reference and
 * exists to skew the expert load in benchmarks (a Zipf-shaped bias). */
int pm_moe_router_topk(const void *x, const void *router_w, const float *bias, int T, int H, int E, int k,
                       void *logits, float *topk_w, int32_t *topk_ids, pm_stream_t stream);

/* Softmax + top-k + renormalise from given bf16 logits: prismyra/kernels/qwen3_moe.py:196 (fused_topk); bias as
 * for pm_moe_router_topk. */
int pm_moe_topk(const void *logits, const float *bias, int T, int E, int k, float *topk_w, int32_t *topk_ids,
                pm_stream_t stream);

/* Bytes of device scratch pm_moe_align needs (its per-chunk expert counts); 0 for invalid arguments.  No
 * counterpart in the reference (vLLM allocates this scratch inside moe_align_block_size). */
size_t pm_moe_align_workspace_bytes(int T, int k, int E);

/* Expert alignment: vllm/model_executor/layers/fused_moe/moe_align_block_size.py:11-99 with block 128, the
 * reference's call at vllm/model_executor/layers/fused_moe/fused_moe.py:1536-1585.  Flat indices grouped by
 * expert in ascending order, padded with T*k.  Needs pm_moe_align_workspace_bytes(T, k, E) bytes of workspace
 * for its per-chunk counts.  expert_off and slot_of (the inverse permutation, slot_of[t*k + j] = slot) may be
 * NULL. */
int pm_moe_align(const int32_t *topk_ids, int T, int k, int E, int32_t *sorted_ids, int32_t *expert_ids,
                 int32_t *num_post_pad, int32_t *expert_off, int32_t *slot_of, void *workspace,
                 size_t workspace_bytes, pm_stream_t stream);

/* Per-token, per-128-column e4m3 quantisation of the activations:
 * vllm/model_executor/layers/quantization/utils/fp8_utils.py:110-150 (per_token_group_quant_fp8), applied by
 * vllm/model_executor/layers/fused_moe/fused_moe.py:1780-1786 before the gate_up GEMM.  slot_of == NULL: row t of
 * a_q e4m3 [T, H] / a_s f32 [T, H/128]; otherwise each token's row is written to its k slots
 * (a_q [max_slots, H], a_s [max_slots, H/128]; vLLM reads the same rows through sorted_ids // top_k,
 * fused_moe.py:437-439) and padding slots are left unwritten. */
int pm_moe_quant_fp8(const void *x, int T, int H, int k, const int32_t *slot_of, uint8_t *a_q, float *a_s,
                     pm_stream_t stream);

/* Grouped gate_up GEMM with fused silu*mul and e4m3 re-quantisation:
 * vllm/model_executor/layers/fused_moe/fused_moe.py:1801-1822 (GEMM1), :1825-1827 (silu_and_mul),
 * :1829-1835 (requantisation).  a_q/a_s in slot order; out_q e4m3 [max_slots, I], out_s f32 [max_slots, I/128].
 * err (may be NULL) is set to 1 if the kernel gave up on a bounded wait. */
int pm_moe_gemm1_fp8(const uint8_t *a_q, const float *a_s, const uint8_t *w1, const float *w1_s,
                     const int32_t *expert_ids, const int32_t *num_post_pad, int max_slots, int H, int I, int E,
                     uint8_t *out_q, float *out_s, int32_t *err, pm_stream_t stream);

/* Grouped down GEMM with the routing weight applied in fp32 before the bf16 cast, scattered to the
 * (token, slot) row: vllm/model_executor/layers/fused_moe/fused_moe.py:1840-1861, :538-548. */
int pm_moe_gemm2_fp8(const uint8_t *a_q, const float *a_s, const uint8_t *w2, const float *w2_s,
                     const int32_t *expert_ids, const int32_t *num_post_pad, const int32_t *sorted_ids,
                     const float *topk_w, int max_slots, int T, int k, int H, int I, int E, void *c3, int32_t *err,
                     pm_stream_t stream);

/* out[t] = bf16(sum_j c3[row(t*k + j)]) accumulated in fp32, j ascending: vllm/model_executor/layers/fused_moe/
 * fused_moe.py:1864 (ops.moe_sum).  row_of (i32 [T*k], may be NULL = identity) lets rows come back from
 * expert-parallel ranks in their send order. */
int pm_moe_combine(const void *c3, const int32_t *row_of, int T, int k, int H, void *out, pm_stream_t stream);

/* Row scatter for expert parallelism (no counterpart in the reference, which runs on one device):
 * dst + dst_index[i]*dst_stride <- src + i*src_stride, row_bytes bytes per row (multiples of 16); rows whose
 * dst_index is negative are skipped. */
int pm_moe_scatter_rows(const void *src, int rows, int row_bytes, int src_stride, const int32_t *dst_index,
                        void *dst, int dst_stride, pm_stream_t stream);

/* The whole routed FP8 layer: prismyra/kernels/qwen3_moe.py:184-199 (FusedExperts.forward) minus the shared
 * expert, i.e. logits -> fused_topk -> fused_experts (vllm/model_executor/layers/fused_moe/fused_moe.py:
 * 1664-1869).  Give either router_w (the router runs in-kernel) or logits (bf16 [T, E], router_w ignored). */
int pm_moe_forward_fp8(const void *x, const void *router_w, const void *logits, const uint8_t *w1,
                       const float *w1_s, const uint8_t *w2, const float *w2_s, int T, int H, int I, int E, int k,
                       void *out, void *workspace, size_t workspace_bytes, pm_stream_t stream);

/* pm_moe_quant_fp8 and pm_moe_forward_fp8 with a choice of activation-scale rule (flags; 0 gives exactly those
 * calls).  Every FP8 activation quantisation -- the input's, and the gate_up epilogue's requantisation of
 * silu(gate)*up -- divides a 128-value group by one fp32 scale derived from its maximum magnitude amax, as vLLM's
 * per_token_group_quant_fp8 does (vllm/model_executor/layers/quantization/utils/fp8_utils.py:510-640):
 *   0                        s = max(amax, 1e-10) / 448, correctly rounded: vLLM's compiled CUDA quantiser, the op the
 *                            reference's fused_experts call (prismyra/kernels/qwen3_moe.py:197) runs on a GPU;
 *   PM_FLAG_ACT_SCALE_UE8M0  that s rounded up to a power of two, 2^ceil(log2(s)) (fp8_utils.py:145): vLLM's mode when
 *                            it runs DeepGEMM with E8M0 scales (VLLM_USE_DEEP_GEMM_E8M0, on by default where DeepGEMM
 *                            is installed);
 *   PM_FLAG_ACT_SCALE_RCP    s = max(amax, 1e-10) * fl(1/448): vLLM's Triton quantiser (fp8_utils.py:143-144), one ulp
 *                            away from the quotient for about half of all values.
 * Each value's code is the correctly rounded quotient x / s, clamped to +-448, rounded to e4m3.  bias (fp32 [E], may
 * be NULL) is added to every logit before the ranking, as for pm_moe_router_topk (no counterpart in the reference:
 * a benchmark's expert-load skew). */
#define PM_FLAG_ACT_SCALE_UE8M0 1
#define PM_FLAG_ACT_SCALE_RCP 2
int pm_moe_quant_fp8_ex(const void *x, int T, int H, int k, const int32_t *slot_of, uint8_t *a_q, float *a_s,
                        int flags, pm_stream_t stream);
int pm_moe_forward_fp8_ex(const void *x, const void *router_w, const void *logits, const float *bias,
                          const uint8_t *w1, const float *w1_s, const uint8_t *w2, const float *w2_s, int T, int H,
                          int I, int E, int k, int flags, void *out, void *workspace, size_t workspace_bytes,
                          pm_stream_t stream);

/* The shared expert, `torch.sigmoid(self._gate(x)) * self.shared_expert(x)` (prismyra/kernels/qwen3_moe.py:198):
 * gate = bf16(sigmoid(bf16(x . w_sg))) (w_sg bf16 [H], the shared_expert_gate weight, qwen3_moe.py:172-183), and
 * the MLP down(bf16(silu(gate_proj x)) * up_proj x) on 128x128 block-FP8 weights with the reference's Fp8Linear
 * arithmetic (per_token_group_quant_fp8 + w8a8 block-scaled matmul, qwen3_moe.py:211-230): w13 e4m3 [2*Is, H]
 * (gate_proj rows, then up_proj rows), w13_s f32 [2*Is/128, H/128], w2 e4m3 [H, Is], w2_s f32 [H/128, Is/128].
 * The MLP output is rounded to bf16 before the bf16 product with the gate.  out bf16 [T, H].  H % 256 == 0,
 * Is % 128 == 0.  Every row is computed in a fixed order (row-count invariant, deterministic). */
size_t pm_moe_shared_workspace_bytes(int T, int H, int Is);
int pm_moe_shared_fp8(const void *x, const void *w_sg, const uint8_t *w13, const float *w13_s, const uint8_t *w2,
                      const float *w2_s, int T, int H, int Is, void *out, void *workspace, size_t workspace_bytes,
                      pm_stream_t stream);

/* A dense block-FP8 projection, the reference's Fp8Linear.forward (prismyra/kernels/qwen3_moe.py:211-230: vLLM
 * per_token_group_quant_fp8 of x, then w8a8_triton_block_scaled_mm): out bf16 [T, N] = x [T, K] bf16 times
 * w e4m3 [N, K] with fp32 128x128 block multipliers w_s [N/128, K/128], each 128-deep K block's exact product sum
 * scaled by the activation and weight scales and added in K order in fp32, then rounded to bf16.  Row-count
 * invariant and deterministic.  K % 128 == 0, N % 256 == 0.  Status word at the start of the workspace. */
size_t pm_fp8_linear_workspace_bytes(int T, int K, int N);
int pm_fp8_linear(const void *x, const uint8_t *w, const float *w_s, int T, int K, int N, void *out,
                  void *workspace, size_t workspace_bytes, pm_stream_t stream);

/* The whole FusedExperts.forward (prismyra/kernels/qwen3_moe.py:184-199): routed experts as pm_moe_forward_fp8
 * plus the shared expert as pm_moe_shared_fp8, summed as two bf16 tensors (`routed + shared`, :199: the routed
 * top-k sum is rounded to bf16 first).  Status word at the start of the workspace, as for pm_moe_forward_fp8. */
size_t pm_moe_block_workspace_bytes(int T, int H, int I, int Is, int E, int k);
int pm_moe_block_fp8(const void *x, const void *router_w, const void *logits, const uint8_t *w1, const float *w1_s,
                     const uint8_t *w2, const float *w2_s, const void *w_sg, const uint8_t *sw13,
                     const float *sw13_s, const uint8_t *sw2, const float *sw2_s, int T, int H, int I, int Is, int E,
                     int k, void *out, void *workspace, size_t workspace_bytes, pm_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * NVFP4 (e2m1 values, one e4m3 scale per 16 elements, one fp32 global scale per tensor): the routed path of
 * prismyra/kernels/nvfp4.py:112-312 (FusedExpertsFp4, which calls FlashInfer's cutlass_fused_moe).
 * Packed e2m1: two values per byte, the even column in the low nibble (prismyra/kernels/nvfp4.py:50).
 * Scale layout ("blocked"): a matrix of R rows and K/16 scales per row is [R/128][K/64][512 bytes]; in a block,
 * row r (0..127) stores its four scales of the 64-column chunk as one 32-bit word at byte (r%32)*16 + (r/32)*4.
 * Weights: w1 u8 [E, 2I, H/2] (gate rows then up rows, as in prepare_layer), w1_sf blocked [E][2I/128][H/64][512];
 * w2 u8 [E, H, I/2], w2_sf blocked [E][H/128][I/64][512]; alpha1/alpha2 f32 [E] = 1/(g_w[e] * a_gs)
 * (prismyra/kernels/nvfp4.py:141-142).  Extra shape limit: I % 256 == 0.
 * --------------------------------------------------------------------------------------------------------------- */

/* NVFP4 quantisation of token rows with global scale gs (vllm/model_executor/layers/quantization/utils/
 * nvfp4_emulation_utils.py:172-216; the reference's ops.scaled_fp4_quant call at prismyra/kernels/nvfp4.py:260).
 * slot_of == NULL: row t of a_q [T, H/2] / blocked a_sf; otherwise the token's k slots. */
int pm_moe_quant_nvfp4(const void *x, int T, int H, int k, const int32_t *slot_of, float gs, uint8_t *a_q,
                       uint8_t *a_sf, pm_stream_t stream);

/* NVFP4 grouped gate_up GEMM: alpha1[e] * (A . W1^T) -> bf16 -> silu*mul -> bf16 -> NVFP4 with a2_gs
 * (FlashInfer FC1 + activation + requantisation inside cutlass_fused_moe, prismyra/kernels/nvfp4.py:262-287). */
int pm_moe_gemm1_nvfp4(const uint8_t *a_q, const uint8_t *a_sf, const uint8_t *w1, const uint8_t *w1_sf,
                       const float *alpha1, float a2_gs, const int32_t *expert_ids, const int32_t *num_post_pad,
                       int max_slots, int H, int I, int E, uint8_t *out_q, uint8_t *out_sf, int32_t *err,
                       pm_stream_t stream);

/* NVFP4 grouped down GEMM: bf16(alpha2[e] * (A . W2^T) * routing weight) scattered to c3[t*k + j]
 * (FlashInfer FC2 + finalize, prismyra/kernels/nvfp4.py:262-287). */
int pm_moe_gemm2_nvfp4(const uint8_t *a_q, const uint8_t *a_sf, const uint8_t *w2, const uint8_t *w2_sf,
                       const float *alpha2, const int32_t *expert_ids, const int32_t *num_post_pad,
                       const int32_t *sorted_ids, const float *topk_w, int max_slots, int T, int k, int H, int I,
                       int E, void *c3, int32_t *err, pm_stream_t stream);

/* The whole routed NVFP4 layer: prismyra/kernels/nvfp4.py:147-170 (FusedExpertsFp4.forward) minus the shared
 * expert.  a1_gs / a2_gs are the activation global scales (nvfp4.py:125-126). */
int pm_moe_forward_nvfp4(const void *x, const void *router_w, const void *logits, const uint8_t *w1,
                         const uint8_t *w1_sf, const float *alpha1, float a1_gs, const uint8_t *w2,
                         const uint8_t *w2_sf, const float *alpha2, float a2_gs, int T, int H, int I, int E, int k,
                         void *out, void *workspace, size_t workspace_bytes, pm_stream_t stream);

/* NVFP4 weight preparation on the GPU: prismyra/kernels/nvfp4.py:315-331 (prepare_layer without the optional
 * importance search) for a stack of E expert matrices of R x C, bit for bit.  w: e4m3 [E, R, C] with fp32 block
 * multipliers s [E, R/128, C/128] (the checkpoint's *_scale_inv, restored as in _dequant_fp8, nvfp4.py:97-100).
 * Outputs: packed e2m1 [E, R, C/2] (even column in the low nibble), row-major e4m3 scales [E, R, C/16] and the
 * global scales g [E] = reciprocal(max(amax, 1e-12)) * 2688 (nvfp4.py:321, which torch evaluates that way), with
 * quantize's arithmetic (nvfp4.py:41-51).  R % 128 == 0, C % 128 == 0; w 16-byte and packed 8-byte aligned. */
int pm_nvfp4_prepare(const uint8_t *w, const float *s, int E, int R, int C, uint8_t *packed, uint8_t *scales,
                     float *g, pm_stream_t stream);

/* The same with the importance search: prismyra/kernels/nvfp4.py:57-94 (quantize_search, which prepare_layer uses
 * when it is given importance weights, nvfp4.py:322-325): each 16-group's e4m3 scale is the first of the fractions
 * 1, 0.95, ..., 0.7 of its plain scale whose decoded group has the smallest importance-weighted squared error.
 * importance: fp32 [E, C] per input column of each matrix (16-byte aligned), or NULL for weight 1 everywhere (the
 * reference's choice for an expert that saw no tokens is a row of ones). */
int pm_nvfp4_prepare_search(const uint8_t *w, const float *s, const float *importance, int E, int R, int C,
                            uint8_t *packed, uint8_t *scales, float *g, pm_stream_t stream);

/* Expert alignment that allocates nothing -- no counterpart in the reference.  Same results as pm_moe_align,
 * for callers that cannot hand the library scratch memory on demand: hosts that route every device byte through
 * their own pool and forbid library allocations, and latency-critical loops that cannot afford the implicit
 * device synchronisation of cudaMalloc/cudaFree.  The per-chunk count table lives in a fixed 256 KiB device array
 * inside the library (held on every GPU that loads it until the process exits).  Limits: T*k <= 2^20 and
 * E <= 256, else PM_ERR_TOO_LARGE.  All calls share that array: calls whose kernels overlap on the GPU (e.g. on
 * two streams) race and must be serialised by the caller.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current); make it before any stream capture begins.  The
 * address is kept for the life of the process: it does not survive cudaDeviceReset or the destruction of the
 * device's primary context, after which this entry point must not be called. */
int pm_moe_align_noalloc(const int32_t *topk_ids, int T, int k, int E, int32_t *sorted_ids, int32_t *expert_ids,
                         int32_t *num_post_pad, int32_t *expert_off, pm_stream_t stream);

/* ---- Expert parallelism over peer memory.  No counterpart in the reference, which runs the layer on one
 * device: these move a layer's rows between the ranks of one node by direct NVLink loads and stores.
 * pm_ep_alloc: device memory (zeroed) plus its 64-byte CUDA IPC handle for the other ranks; pm_ep_open maps a
 * peer's handle into this process (pm_ep_close / pm_ep_free undo them).  The other calls take device arrays of G
 * addresses (peer_*, one per rank, this rank's own included) and are stream-ordered, without host synchronisation.
 *   pm_ep_count       store this rank's per-expert pair counts into row `rank` of every rank's count matrix [G][E]
 *   pm_ep_barrier     add 1 to every rank's counter and wait until the own counter reaches target, for at most
 *                     wait_limit_ns nanoseconds (0: the library's 2 s); on timeout *err = 1 and the kernel returns
 *   pm_ep_offsets     from the full count matrix: for each global expert, where this rank's pairs of it start in
 *                     the owner's slot space (experts padded to 128 slots, sources in rank order), and the block
 *                     table and slot count of this rank's own experts; with bounds (int32 [groups + 1], may be
 *                     NULL) also the first slot of each of `groups` equal groups of its experts and the slot count
 *   pm_ep_dispatch_quant  per-token per-128 e4m3 quantisation (as pm_moe_quant_fp8) stored straight into the
 *                     owners' slots, with each slot's (source rank << 24 | pair index) and routing weight; T*k < 2^24;
 *                     only pairs whose expert is local expert [local_lo, local_hi) of its owner; on at most max_sms
 *                     SMs' worth of blocks (0: all), so that it can run beside a GEMM that leaves those SMs free
 *   pm_ep_gemm1_fp8   the gate_up GEMM of pm_moe_gemm1_fp8 over slots [bounds[group], bounds[group + 1]) of this
 *                     rank's slot space, on at most max_sms SMs (0: all)
 *   pm_ep_local_rows  per slot, the address of its source rank's result row for its pair (0 for padding)
 *   pm_ep_gemm2_fp8   the down GEMM of pm_moe_gemm2_fp8 over this rank's slots, each weighted bf16 row stored to
 *                     dst_rows[slot] (another rank's memory over NVLink) instead of a local C3 */
int pm_ep_alloc(size_t bytes, void **ptr, void *ipc_handle);
int pm_ep_open(const void *ipc_handle, void **ptr);
int pm_ep_close(void *ptr);
int pm_ep_free(void *ptr);
int pm_ep_count(const int32_t *ids, int n, int E, int G, int rank, const uint64_t *peer_cm, pm_stream_t stream);
int pm_ep_barrier(const uint64_t *peer_flag, unsigned *own_flag, int G, unsigned target, int32_t *err,
                  uint64_t wait_limit_ns, pm_stream_t stream);
int pm_ep_offsets(const int32_t *cm, int G, int E, int epr, int rank, int32_t *base, int32_t *expert_ids,
                  int32_t *num_post_pad, int cap_slots, int32_t *err, int32_t *bounds, int groups,
                  pm_stream_t stream);
int pm_ep_dispatch_quant(const void *x, int T, int H, int k, const int32_t *topk_ids, const float *topk_w,
                         const int32_t *slot_local, const int32_t *expert_off_local, const int32_t *base, int E,
                         int epr, int rank, int cap_slots, const uint64_t *peer_a1, const uint64_t *peer_a1_scale,
                         const uint64_t *peer_meta, const uint64_t *peer_weight, int32_t *err, int local_lo,
                         int local_hi, int max_sms, pm_stream_t stream);
int pm_ep_gemm1_fp8(const uint8_t *a_q, const float *a_s, const uint8_t *w1, const float *w1_s,
                    const int32_t *expert_ids, const int32_t *bounds, int group, int cap_slots, int H, int I, int E,
                    uint8_t *out_q, float *out_s, int32_t *err, int max_sms, pm_stream_t stream);
int pm_ep_local_rows(const int32_t *meta, const int32_t *num_post_pad, int cap_slots, int H, int G, int n_pairs,
                     const uint64_t *peer_back, uint64_t *dst_rows, int32_t *err, pm_stream_t stream);
int pm_ep_gemm2_fp8(const uint8_t *a_q, const float *a_s, const uint8_t *w2, const float *w2_s,
                    const int32_t *expert_ids, const int32_t *num_post_pad, const float *weight,
                    const uint64_t *dst_rows, int cap_slots, int H, int I, int E, int32_t *err, pm_stream_t stream);

/* Synchronise the stream and report PM_ERR_TIMEOUT if any kernel of the last calls on this workspace gave up
 * on a bounded wait (the flag is cleared by each pm_moe_forward_* call). */
int pm_moe_read_status(const void *workspace, pm_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PRISMYRA_MOE_H */
