// Internal launch interface between the kernel translation units and the C-ABI layer (moe_capi.cu).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

namespace pm {

// Returns a failed cudaError_t from the enclosing function.
#define PM_TRY(expr)                                 \
    do {                                             \
        const cudaError_t pm_err_ = (expr);          \
        if (pm_err_ != cudaSuccess) return pm_err_;  \
    } while (0)

// Launches a kernel of the forward chain with programmatic stream serialisation: it may be scheduled while the
// previous kernel of the stream finishes, and waits for it (pdl_wait) before touching global memory.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}


constexpr int kBlockM = 128;  // rows of one GEMM tile == the alignment block of the expert permutation
// Activation-scale rules of the FP8 quantisations (e4m3_group_scale in ptx.cuh).
constexpr int kScaleDiv = 0, kScaleUe8m0 = 1, kScaleRcp = 2;
constexpr int kMaxExperts = 256;
// T*k range in which the forward runs the top-k, the alignment and the quantisation as one launch (below it the
// three short launches measured faster: at T*k = 256 the one launch's grid barrier costs more than it saves)
constexpr int kFrontMinIndices = 512;
constexpr int kFrontMaxIndices = 4096;
constexpr int kMaxTopK = 16;
// The alignment kernels split the n flat (token, slot) indices into at most kAlignMaxChunks chunks of
// align_chunk(n) indices (one chunk up to 1024 indices, else at least 512, a multiple of 256); the per-chunk count
// table has align_chunks(n) rows.
constexpr int kAlignMaxChunks = 256;
inline int align_chunk(long n) {
    if (n <= 1024) return 1024;
    long c = (n + kAlignMaxChunks - 1) / kAlignMaxChunks;
    if (c < 512) c = 512;
    return (int)((c + 255) / 256 * 256);
}
inline int align_chunks(long n) { return n > 0 ? (int)((n + align_chunk(n) - 1) / align_chunk(n)) : 0; }

inline int cdiv(long a, long b) { return static_cast<int>((a + b - 1) / b); }

// Router projection (bf16, fp32 accumulation in a fixed order per row) fused with softmax / top-k.
// bias (may be null): fp32 [E] added to each logit before the ranking.
// part: fp32 scratch of router_split_bytes(T, H, E) bytes for the split launch shape, or nullptr (fused shape);
// both give the same bits.  Without topk only the projection runs: the bf16 logits (fused shape) or the fp32
// partials (split shape, router_split_bytes > 0) are left for launch_front_small.
size_t router_split_bytes(int T, int H, int E);
int router_chunks(int H);  // the split shape's partials per token
// clear (may be null): four status words the launch zeroes first (the forward's, instead of a memset).
cudaError_t launch_router_topk(const void* x, const void* w, const float* bias, int T, int H, int E, int k,
                               void* logits, float* topk_w, int32_t* topk_ids, int32_t* err, cudaStream_t s,
                               float* part = nullptr, bool topk = true, int32_t* clear = nullptr);
// Softmax / top-k / renormalise from given bf16 logits (+ optional fp32 bias per expert).
cudaError_t launch_topk(const void* logits, const float* bias, int T, int E, int k, float* topk_w, int32_t* topk_ids,
                        cudaStream_t s);
// Top-k from fp32 chunk partials part[c][t][e] (c < chunks, added in ascending order): also writes the bf16 logits.
cudaError_t launch_topk_partials(const float* part, int chunks, void* logits, const float* bias, int T, int E, int k,
                                 float* topk_w, int32_t* topk_ids, cudaStream_t s);
// Stable counting sort of the flat (token, slot) indices by expert, padded per expert to kBlockM.
// slot_of (may be null) receives the inverse permutation: slot_of[flat index] = its slot.
cudaError_t launch_align(const int32_t* ids, int n, int E, int32_t* counts, int32_t* sorted, int32_t* expert_ids,
                         int32_t* num_post_pad, int32_t* expert_off, int32_t* slot_of, cudaStream_t s);
// Quantise every token row of x to e4m3 with one fp32 scale per 128 columns.  With slot_of, each quantised row
// is written to the k slots of its token (a_q [slots, H], a_s [slots, H/128]) instead of to row t.
// scale_rule: how each group's scale is formed (e4m3_group_scale in ptx.cuh; 0 = the correctly rounded quotient).
// zero (may be null): zero_n int32 counters the launch sets to 0 once its predecessor has completed.
cudaError_t launch_quant_fp8(const void* x, int T, int H, int k, const int32_t* slot_of, uint8_t* x_q, float* x_s,
                             cudaStream_t s, int scale_rule = 0, int32_t* zero = nullptr, int zero_n = 0);
// The few-token front end in one launch (T*k <= kFrontMaxIndices, E <= kMaxExperts): the top-k (from the
// router's fp32 partials, which also gives the bf16 logits, from bf16 logits_in, or skipped when both are null and
// topk_w/topk_ids are given), the alignment (launch_align's outputs; counts not written) and the quantisation into
// slots (launch_quant_fp8 with slot_of), with one grid barrier on the counter *bar, which must be zero when the
// launch starts.  A barrier that times out sets *err.
cudaError_t launch_front_small(const float* part, int chunks, const void* logits_in, void* logits_out,
                               const float* bias, int T, int E, int k, float* topk_w, int32_t* topk_ids,
                               int32_t* sorted, int32_t* expert_ids, int32_t* num_post_pad, int32_t* expert_off,
                               int32_t* slot_of, const void* x, int H, uint8_t* x_q, float* x_s, int scale_rule,
                               int32_t* zero, int zero_n, int32_t* bar, int32_t* err, cudaStream_t s);
// out[t] = bf16(sum_j c3[row(t*k + j)]) in fp32, j ascending; row = identity or row_of.
cudaError_t launch_combine(const void* c3, const int32_t* row_of, int T, int k, int H, void* out, cudaStream_t s,
                           const void* add = nullptr);
// Shared-expert gate g[t] = bf16(sigmoid(bf16(x[t] . w_sg))) as fp32, plus the one-expert plan of the shared
// expert's GEMMs (expert_ids[b] = 0 for the ceil(T/128) blocks, *num_post_pad = their slots).
cudaError_t launch_shared_gate(const void* x, const void* w_sg, int T, int H, float* gate, int32_t* expert_ids,
                               int32_t* num_post_pad, int sms, cudaStream_t s);
// The one-expert plan of a dense block-FP8 projection: expert_ids = 0, *num_post_pad, ones[t] = 1.
cudaError_t launch_dense_plan(int T, float* ones, int32_t* expert_ids, int32_t* num_post_pad, int sms,
                              cudaStream_t s);
// dst[dst_index[i]] = src[i] for rows of row_bytes (multiple of 16) with the given byte strides.
cudaError_t launch_scatter_rows(const void* src, int rows, int row_bytes, int src_stride, const int32_t* dst_index,
                                void* dst, int dst_stride, cudaStream_t s);

struct GemmArgs {
    const float* a_scale;     // [rows, K/128]
    const float* b_scale;     // [E, N_total/128, K/128]
    const int32_t* expert_ids;   // [blocks]
    const int32_t* num_post_pad; // [1]
    int n_total;              // rows of one expert's weight matrix (2I for gate_up, H for down)
    int K;                    // reduction length (H for gate_up, I for down)
    int n_tiles;              // tiles along N
    int max_tiles;            // upper bound of tiles (grid sizing)
    int inter;                // I (gate_up: column offset of the up rows; width of the output)
    // gate_up epilogue
    uint8_t* out_q;           // [rows, I] e4m3
    float* out_s;             // [rows, I/128]
    // down epilogue
    const int32_t* sorted_ids;   // [rows] flat index per row (n_valid = padding); nullptr: the row index itself
    const float* topk_w;      // [n_valid]
    __nv_bfloat16* c3;        // [n_valid, H]
    const uint64_t* dst_rows; // [rows] or nullptr: the address each row's [H] bf16 result is stored to (0: none),
                              // instead of c3 -- e.g. another GPU's memory over NVLink
    int n_valid;
    int round_first;          // down epilogue: bf16(bf16(acc) * w) instead of bf16(acc * w) (a bf16 product)
    int scale_rule;           // gate_up epilogue: how requantisation scales are formed (e4m3_group_scale)
    int* err;                 // set to 1 when a wait timed out
    const int32_t* slot_lo;   // optional (null: 0): the launch covers slots [*slot_lo, *num_post_pad) only
};

cudaError_t launch_gemm_fp8(int mode, const CUtensorMap& tm_a, const CUtensorMap& tm_b, const GemmArgs& args,
                            int num_sms, cudaStream_t s);

// Grouped FP8 GEMM for few tokens per expert (moe_gemm_fp8_small.cu): weights as the MMA's 128-row operand,
// the real token sub-blocks of each 128-slot block as its N operand.
struct SmallGemmArgs {
    const float* a_scale;        // [rows, K/128]
    const float* b_scale;        // [E, n_total/128, K/128]
    const int32_t* expert_ids;   // [blocks]
    const int32_t* num_post_pad; // [1]
    const int32_t* sorted_ids;   // [rows] flat index per slot (n_valid = padding; a block's real slots first)
    int n_valid;                 // T * k
    int n_total;                 // rows of one expert's weight matrix (2I for gate_up, H for down)
    int K;                       // reduction length (H for gate_up, I for down)
    int n_tiles;                 // 128-column units along the output (I/128 or H/128)
    int max_units;               // upper bound of units (grid sizing)
    int inter;                   // I
    int stages;                  // set by the launcher
    uint8_t* out_q;              // gate_up: [rows, I] e4m3
    float* out_s;                // gate_up: [rows, I/128]
    const float* topk_w;         // down: [n_valid]
    __nv_bfloat16* c3;           // down: [n_valid, H]
    int scale_rule;              // gate_up: how requantisation scales are formed (e4m3_group_scale)
    int* err;
    int prefetch_units;          // fused, gate_up: units whose weights CTA b (b < this) prefetches before it waits
};
// The small-token path is used when T*k <= kSmallTokensPerExpert * E and the K-block scale table fits.
constexpr int kSmallTokensPerExpert = 32;
bool gemm_fp8_small_fits(int mode, int K);
// tm_tok: the slot-ordered FP8 activations with a {128, 32} box; tm_w: the weights with a {128, 128} box.
cudaError_t launch_gemm_fp8_small(int mode, const CUtensorMap& tm_tok, const CUtensorMap& tm_w,
                                  const SmallGemmArgs& args, int num_sms, cudaStream_t s);
// Both GEMMs in one persistent launch: the gate_up units, then the down units, taken from a work queue; a down
// unit starts once every gate_up unit of its block half has stored its rows.  sched: small_sched_ints(blocks)
// int32 set to 0 before the launch (the quantisation kernel does it).
inline int small_sched_ints(int max_blocks) { return 1 + 2 * max_blocks; }
bool gemm_fp8_small_fused_fits(int H, int I);
cudaError_t launch_gemm_fp8_small_fused(const CUtensorMap& tm_tok1, const CUtensorMap& tm_w1,
                                        const CUtensorMap& tm_tok2, const CUtensorMap& tm_w2,
                                        const SmallGemmArgs& gate_up, const SmallGemmArgs& down, int32_t* sched,
                                        int num_sms, cudaStream_t s);

struct NvGemmArgs {
    const uint8_t* a_sf;          // blocked e4m3 scales of A: [rows/128][K/64][512]
    const uint8_t* b_sf;          // blocked e4m3 scales of B: [E][n_total/128][K/64][512]
    const float* alpha;           // [E] 1 / (weight global scale * activation global scale)
    const int32_t* expert_ids;
    const int32_t* num_post_pad;
    int n_total, K, n_tiles, max_tiles, inter;
    // gate_up epilogue: NVFP4 re-quantisation of silu(gate)*up with the layer's second activation scale
    float gs_out;
    uint8_t* out_q;               // packed e2m1 [rows, I/2]
    uint8_t* out_sf;              // blocked [rows/128][I/64][512]
    // down epilogue
    const int32_t* sorted_ids;
    const float* topk_w;
    __nv_bfloat16* c3;
    int n_valid;
    int* err;
};

// NVFP4 quantisation of token rows (global scale gs), written to each token's k slots when slot_of is given.
cudaError_t launch_quant_nvfp4(const void* x, int T, int H, int k, const int32_t* slot_of, float gs, uint8_t* a_q,
                               uint8_t* a_sf, cudaStream_t s);
cudaError_t launch_gemm_nvfp4(int mode, const CUtensorMap& tm_a, const CUtensorMap& tm_b, const NvGemmArgs& args,
                              int num_sms, cudaStream_t s);
// NVFP4 weight preparation of E FP8 block-scaled matrices of R x C (g doubles as the scratch of the maxima).
// search: each 16-group's scale chosen by the importance search (imp [E, C] per input column, or null: weight 1).
cudaError_t launch_nvfp4_prepare(const uint8_t* w, const float* s, int E, int R, int C, uint8_t* packed,
                                 uint8_t* sf, float* g, int sms, cudaStream_t stream, bool search = false,
                                 const float* imp = nullptr);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda): a 2-D row-major
// tensor of `outer` rows x `inner` elements, rows `row_bytes` apart, 128-byte swizzled boxes.
bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);
inline bool encode_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                              uint32_t box_inner, uint32_t box_outer) {
    return encode_tmap_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, inner, outer, row_bytes, box_inner, box_outer);
}

// Expert parallelism over peer memory (moe_ep.cu); peer_* are device arrays of G addresses (one per rank).
cudaError_t launch_ep_count(const int32_t* ids, int n, int E, int G, int rank, const uint64_t* peer_cm,
                            cudaStream_t s);
cudaError_t launch_ep_barrier(const uint64_t* peer_flag, unsigned* own_flag, int G, unsigned target, int32_t* err,
                              uint64_t limit_ns, cudaStream_t s);
cudaError_t launch_ep_offsets(const int32_t* cm, int G, int E, int epr, int rank, int32_t* base, int32_t* expert_ids,
                              int32_t* npp, int cap_blocks, int32_t* err, int32_t* bounds, int groups,
                              cudaStream_t s);
cudaError_t launch_ep_dispatch_quant(const void* x, int T, int H, int k, const int32_t* ids, const float* topk_w,
                                     const int32_t* slot_local, const int32_t* off_local, const int32_t* base,
                                     int E, int epr, int rank, int cap, const uint64_t* peer_a1,
                                     const uint64_t* peer_a1s, const uint64_t* peer_meta, const uint64_t* peer_wgt,
                                     int32_t* err, int sms, int le_lo, int le_hi, int ctas, cudaStream_t s);
cudaError_t launch_ep_local_rows(const int32_t* meta, const int32_t* npp, int cap, int H, int G, int n_pairs,
                                 const uint64_t* peer_back, uint64_t* dst_rows, int32_t* err, int sms,
                                 cudaStream_t s);

}  // namespace pm
