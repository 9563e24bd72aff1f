// Routing stage of the routed-expert layer: softmax / top-k / renormalise from given logits, and the stable
// expert alignment of the flat (token, slot) indices (the router projection itself is moe_router_tc.cu).
//
// Reference behaviour (restated here, see the oracle for the executable statement):
//   router  prismyra/kernels/qwen3_moe.py:169-171 (_route: bf16 x . W^T, fp32 accumulation, bf16 logits)
//   top-k   prismyra/kernels/qwen3_moe.py:196 -> vLLM fused_topk(renormalize=True): fp32 softmax over the experts,
//           the k largest (equal values: lower expert index first), divided by their sum
//   align   prismyra/kernels/qwen3_moe.py:197 -> vLLM moe_align_block_size: flat indices grouped by expert in
//           ascending order, each expert padded to a multiple of the block with the value T*k
#include <math.h>

#include "moe_internal.h"
#include "ptx.cuh"
#include "quant_dev.cuh"

namespace pm {
namespace {

constexpr int kMaxEPT = kMaxExperts / 32;  // logits held per lane at most (EPT: 4 for E <= 128, else 8)

// One warp ranks one token.  v[i] holds the logit of expert lane + 32 i (or -inf past E).
template <int EPT>
__device__ __forceinline__ void warp_topk(const float (&v)[EPT], int E, int k, float* w_out, int32_t* id_out) {
    const int lane = threadIdx.x & 31;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPT; ++i) mx = fmaxf(mx, v[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float ex[EPT];
#pragma unroll
    for (int i = 0; i < EPT; ++i) ex[i] = (lane + 32 * i < E) ? expf(v[i] - mx) : 0.0f;
    // The exponent sum in ascending expert order over whole 32-expert groups (zeros past E), one fp32 add per
    // term: the row is staged in this warp's shared-memory row and every lane adds it in order from 16-byte
    // broadcast loads.
    __shared__ __align__(16) float rows[8][32 * EPT];
    float* row = rows[(threadIdx.x >> 5) & 7];
#pragma unroll
    for (int i = 0; i < EPT; ++i) row[lane + 32 * i] = ex[i];
    __syncwarp();
    float sum = 0.0f;
    const int n = 32 * min(EPT, (E + 31) / 32);
    for (int e = 0; e < n; e += 4) {
        const float4 q = *reinterpret_cast<const float4*>(row + e);
        sum += q.x;
        sum += q.y;
        sum += q.z;
        sum += q.w;
    }

    // Selection j takes the largest remaining logit, the lowest expert on ties: each lane's best remaining entry
    // as an order-preserving unsigned key (-0 counted as +0, NaN below every number), then a warp max of the keys
    // and a warp min of the experts that hold it.
    uint32_t key[EPT];
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
        const uint32_t b = __float_as_uint(v[i] + 0.0f);
        key[i] = v[i] != v[i] ? 0u : ((b & 0x80000000u) ? ~b : (b | 0x80000000u));
    }
    uint32_t used = 0;
    float my_x = 0.0f;  // lane j < k: the exponent of selection j
    int my_id = 0;
    for (int j = 0; j < k; ++j) {
        uint32_t bk = 0;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((used >> i) & 1u) && (key[i] > bk || bi == 0x7fffffff)) {
                bk = key[i];
                bi = e;
            }
        }
        const uint32_t top = __reduce_max_sync(0xffffffffu, bi != 0x7fffffff ? bk : 0u);
        bi = (int)__reduce_min_sync(0xffffffffu, (bi != 0x7fffffff && bk == top) ? (uint32_t)bi : 0x7fffffffu);
        float mine = 0.0f;
        if ((bi & 31) == lane) {
            const int slot = bi >> 5;
            used |= 1u << slot;
#pragma unroll
            for (int i = 0; i < EPT; ++i)
                if (i == slot) mine = ex[i];
        }
        const float xj = __shfl_sync(0xffffffffu, mine, bi & 31);
        if (lane == j) {
            my_x = xj;
            my_id = bi;
        }
    }
    // p_j = x_j / sum, their sum in selection order, then w_j = p_j / that sum
    const float p = my_x / sum;
    float sel = 0.0f;
    for (int j = 0; j < k; ++j) sel += __shfl_sync(0xffffffffu, p, j);
    if (lane < k) {
        w_out[lane] = p / sel;
        id_out[lane] = my_id;
    }
}

template <int EPT>
__global__ void __launch_bounds__(256) topk_kernel(const __nv_bfloat16* __restrict__ logits,
                                                   const float* __restrict__ bias, int T, int E, int k,
                                                   float* __restrict__ topk_w, int32_t* __restrict__ topk_ids) {
    pdl_wait();
    pdl_trigger();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= T) return;
    float v[EPT];
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < E ? __bfloat162float(logits[(size_t)warp * E + e]) + (bias != nullptr ? bias[e] : 0.0f)
                     : -INFINITY;
    }
    warp_topk(v, E, k, topk_w + (size_t)warp * k, topk_ids + (size_t)warp * k);
}

// Token t's ranking inputs from the router's fp32 chunk partials: logit = bf16(((P_0 + P_1) + P_2) + ...), written
// out, plus the bias.  All of this lane's chunk partials are loaded before any is added (one round trip for up to 8
// chunks), then added in chunk order.
template <int EPT>
__device__ __forceinline__ void logits_from_partials(const float* __restrict__ part, int chunks, int T, int t, int E,
                                                     const float* __restrict__ bias,
                                                     __nv_bfloat16* __restrict__ logits, float (&v)[EPT]) {
    const int lane = threadIdx.x & 31;
    constexpr int kC = 8;
    for (int c0 = 0; c0 < chunks; c0 += kC) {
        float pv[EPT][kC];
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
            const int e = lane + 32 * i;
#pragma unroll
            for (int j = 0; j < kC; ++j)
                pv[i][j] = (e < E && c0 + j < chunks) ? part[((size_t)(c0 + j) * T + t) * E + e] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < EPT; ++i)
#pragma unroll
            for (int j = 0; j < kC; ++j)
                if (c0 + j < chunks) v[i] = (c0 + j == 0) ? pv[i][j] : v[i] + pv[i][j];
    }
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
        const int e = lane + 32 * i;
        if (e < E) {
            const __nv_bfloat16 b = __float2bfloat16_rn(v[i]);
            logits[(size_t)t * E + e] = b;
            v[i] = __bfloat162float(b) + (bias != nullptr ? bias[e] : 0.0f);
        } else {
            v[i] = -INFINITY;
        }
    }
}

// The same from the router's fp32 chunk partials (the logits are written out too).
template <int EPT>
__global__ void __launch_bounds__(256) topk_partials_kernel(const float* __restrict__ part, int chunks,
                                                            __nv_bfloat16* __restrict__ logits,
                                                            const float* __restrict__ bias, int T, int E, int k,
                                                            float* __restrict__ topk_w,
                                                            int32_t* __restrict__ topk_ids) {
    pdl_wait();
    pdl_trigger();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (warp >= T) return;
    float v[EPT];
    logits_from_partials(part, chunks, T, warp, E, bias, logits, v);
    warp_topk(v, E, k, topk_w + (size_t)warp * k, topk_ids + (size_t)warp * k);
}

// ------------------------------------------------------------------------------------------- alignment
// Two launches over chunks of align_chunk(n) flat indices (at most kAlignMaxChunks chunks, so that every CTA of
// the second pass can afford to read the whole count table).
//
// Pass 1: per-chunk expert histogram.
__global__ void __launch_bounds__(256) align_count_kernel(const int32_t* __restrict__ ids, int n, int E, int chunk,
                                                          int32_t* __restrict__ counts) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ int32_t cnt[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const int lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
#pragma unroll 4
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int e = ids[i];
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts[(size_t)blockIdx.x * E + e] = cnt[e];
}

constexpr int kAlignEPT = 4;     // experts per thread in pass 2 (E <= 1024 with 256 threads)
constexpr int kAlignRounds = 16;  // rounds of 256 indices a chunk may have for its ids to be held in registers

// Pass 2: every CTA derives, from the count table, each expert's padded offset (an exclusive scan of the padded
// totals) and the number of its indices in earlier chunks, then scatters its chunk's indices with stable ranks:
// within a round of 256 indices, equal experts are ordered by warp (per-warp counts) and by lane (match mask).
// The block -> expert table and the padding slots (value n) are written warp-cooperatively, experts spread over
// the CTAs; CTA 0 writes the expert offsets and the total.  With a single chunk (counts == nullptr) pass 1 is not
// launched: every CTA counts the (at most one chunk of) indices itself; all CTAs and the scatter: a warp per expert walks the indices in order and places that expert's
// with ballots (stable without any per-round synchronisation).
__global__ void __launch_bounds__(256) align_scatter_kernel(const int32_t* __restrict__ ids, int n, int E, int chunk,
                                                            int nchunks, const int32_t* __restrict__ counts,
                                                            int32_t* __restrict__ sorted,
                                                            int32_t* __restrict__ expert_ids,
                                                            int32_t* __restrict__ num_post_pad,
                                                            int32_t* __restrict__ expert_off,
                                                            int32_t* __restrict__ slot_of) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ int32_t sm[];
    int32_t* base = sm;            // [E]  next slot of each expert for this chunk
    int32_t* pad = sm + E;         // [E]  padded totals, then padded offsets
    int32_t* totv = sm + 2 * E;    // [E]  indices per expert
    int32_t* wcnt = sm + 3 * E;    // [8][E]; single chunk: [E] counts, then the n <= 1024 indices' experts
    int32_t* sids = wcnt + E;
    __shared__ int32_t wsum[8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool single = counts == nullptr;
    const int cta_chunk = single ? 0 : (int)blockIdx.x;
    const int lo = cta_chunk * chunk, hi = (single && blockIdx.x > 0) ? lo : min(n, lo + chunk);
    const int rounds = (min(n, lo + chunk) - lo + 255) / 256;
    const bool held = rounds <= kAlignRounds;

    // this chunk's ids, loaded up front (their latency overlaps the count table reads)
    int idv[kAlignRounds];
#pragma unroll
    for (int r = 0; r < kAlignRounds; ++r) {
        const int i = lo + r * 256 + tid;
        idv[r] = (held && r < rounds && i < min(n, lo + chunk)) ? ids[i] : -1;
    }
    int tot[kAlignEPT], pre[kAlignEPT];
    if (counts == nullptr) {  // single chunk: count here
#pragma unroll
        for (int r = 0; r < 4; ++r) sids[r * 256 + tid] = idv[r];
        for (int e = tid; e < E; e += 256) wcnt[e] = 0;
        __syncthreads();
#pragma unroll
        for (int r = 0; r < kAlignRounds; ++r)
            if (idv[r] >= 0 && idv[r] < E) atomicAdd(&wcnt[idv[r]], 1);
        __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < kAlignEPT; ++q) {
        const int e = tid + 256 * q;
        tot[q] = pre[q] = 0;
        if (e < E) {
            if (single) {
                tot[q] = wcnt[e];
            } else {
                // sixteen loads in flight per batch
                for (int c0 = 0; c0 < nchunks; c0 += 16) {
                    int v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = c0 + j < nchunks ? counts[(size_t)(c0 + j) * E + e] : 0;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        tot[q] += v[j];
                        if (c0 + j < cta_chunk) pre[q] += v[j];
                    }
                }
            }
            pad[e] = (tot[q] + kBlockM - 1) / kBlockM * kBlockM;
            totv[e] = tot[q];
        }
    }
    __syncthreads();
    // exclusive scan of pad[0..E): thread t owns entries [4t, 4t+4)
    int loc[kAlignEPT], run = 0;
#pragma unroll
    for (int j = 0; j < kAlignEPT; ++j) {
        const int e = kAlignEPT * tid + j;
        loc[j] = run;
        run += e < E ? pad[e] : 0;
    }
    int inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    int wpre = 0, total = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        wpre += w < warp ? wsum[w] : 0;
        total += wsum[w];
    }
    const int tpre = wpre + inc - run;  // exclusive prefix of this thread's four entries
#pragma unroll
    for (int j = 0; j < kAlignEPT; ++j) {
        const int e = kAlignEPT * tid + j;
        if (e < E) pad[e] = tpre + loc[j];
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kAlignEPT; ++q) {
        const int e = tid + 256 * q;
        if (e < E) {
            base[e] = pad[e] + pre[q];
            if (blockIdx.x == 0 && expert_off != nullptr) expert_off[e] = pad[e];
        }
    }
    if (blockIdx.x == 0 && tid == 0) {
        *num_post_pad = total;
        if (expert_off != nullptr) expert_off[E] = total;
    }
    // block table and padding slots: one warp per expert, experts spread over the CTAs; the padding run is written
    // with 16-byte stores between its unaligned head and tail (sorted + i is 16-byte aligned iff (i + mis) % 4 == 0)
    const int mis = (int)((reinterpret_cast<uintptr_t>(sorted) >> 2) & 3);
    for (int e = (int)blockIdx.x * 8 + warp; e < E; e += (int)gridDim.x * 8) {
        const int off = pad[e], te = totv[e];
        const int padded = (te + kBlockM - 1) / kBlockM * kBlockM;
        for (int blk = off / kBlockM + lane; blk < (off + padded) / kBlockM; blk += 32) expert_ids[blk] = e;
        const int p0 = off + te, p1 = off + padded;
        const int pa = min(p1, p0 + ((4 - ((p0 + mis) & 3)) & 3));
        const int pb = pa + ((p1 - pa) & ~3);
        if (p0 + lane < pa) sorted[p0 + lane] = n;
        for (int i = pa + 4 * lane; i < pb; i += 128) *reinterpret_cast<int4*>(sorted + i) = make_int4(n, n, n, n);
        if (pb + lane < p1) sorted[pb + lane] = n;
    }
    __syncthreads();

    if (single) {
        // a warp per expert: its indices in ascending order, 32 at a time
        for (int e = (int)blockIdx.x * 8 + warp; e < E; e += (int)gridDim.x * 8) {
            int pos = pad[e];
            for (int i0 = 0; i0 < n; i0 += 32) {
                const int i = i0 + lane;
                const bool hit = i < n && sids[i] == e;
                const uint32_t b = __ballot_sync(0xffffffffu, hit);
                if (hit) {
                    const int p = pos + __popc(b & ((1u << lane) - 1u));
                    sorted[p] = i;
                    if (slot_of != nullptr) slot_of[i] = p;
                }
                pos += __popc(b);
            }
        }
        return;
    }

    // one round of up to 256 indices starting at r0; e_in is this thread's id (or -1 past the chunk)
    auto round = [&](int r0, int e_in) {
        for (int q = tid; q < 8 * E; q += 256) wcnt[q] = 0;
        __syncthreads();
        const int i = r0 + tid;
        const int e = (i < hi) ? e_in : -1 - lane;  // distinct sentinels keep idle lanes apart
        const uint32_t peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const bool valid = (i < hi) && e >= 0 && e < E;
        if (valid && rank == 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        if (valid) {
            int pos = base[e] + rank;
            for (int w = 0; w < warp; ++w) pos += wcnt[w * E + e];
            sorted[pos] = i;
            if (slot_of != nullptr) slot_of[i] = pos;
        }
        __syncthreads();
        for (int q = tid; q < E; q += 256) {
            int s2 = 0;
            for (int w = 0; w < 8; ++w) s2 += wcnt[w * E + q];
            base[q] += s2;
        }
        __syncthreads();
    };
    if (hi <= lo) return;  // a padding-only CTA of a single-chunk call
    if (held) {
#pragma unroll
        for (int r = 0; r < kAlignRounds; ++r)
            if (r < rounds) round(lo + r * 256, idv[r]);
    } else {
        for (int r0 = lo; r0 < hi; r0 += 256) round(r0, r0 + tid < hi ? ids[r0 + tid] : -1);
    }
}

// ------------------------------------------------------------------------------------- fused few-token front end
// For T*k <= kFrontMaxIndices the top-k, the alignment and the quantisation into slots run as one launch with one
// grid barrier.  CTA b owns a contiguous run of tokens: before the barrier it ranks them (a warp per token) and
// converts each warp's first two (token, group) items to e4m3 in registers; after it every CTA loads all T*k
// expert ids, counts them per expert (in total and before its own first flat index i0), scans the padded counts,
// places its own tokens' flat indices (the slot of index i is the expert's padded offset plus its indices before i0
// plus its indices in [i0, i)) and stores its converted rows to their slots.

// Grid barrier on a counter that is zero before the launch (one use per launch).  Bounded: on timeout *err = 1 and
// false for every thread of the CTA.
__device__ __forceinline__ bool front_grid_sync(int32_t* count, int32_t* err) {
    __shared__ int ok_s;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        // the CTA's writes are ordered before this release by the barrier above; the acquire loads below and the
        // barrier after them order the other CTAs' writes before this CTA's later reads
        asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(count) : "memory");
        const uint64_t t0 = globaltimer();
        while (true) {
            int c;
            asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(c) : "l"(count) : "memory");
            if (c >= (int)gridDim.x) break;
            if (globaltimer() - t0 > PM_WAIT_TIMEOUT_NS) {
                atomicExch(err, 1);
                ok = 0;
                break;
            }
        }
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

// part: the router's fp32 chunk partials (logits_out receives the bf16 logits); or logits_in; or neither, with
// topk_w / topk_ids given.
template <int EPT>
__global__ void __launch_bounds__(256) front_small_kernel(
    const float* __restrict__ part, int chunks, const __nv_bfloat16* __restrict__ logits_in,
    __nv_bfloat16* __restrict__ logits_out, const float* __restrict__ bias, int T, int E, int k,
    float* __restrict__ topk_w, int32_t* topk_ids, int32_t* __restrict__ sorted, int32_t* __restrict__ expert_ids,
    int32_t* __restrict__ num_post_pad, int32_t* __restrict__ expert_off, int32_t* __restrict__ slot_of,
    const __nv_bfloat16* __restrict__ x, int H, uint8_t* __restrict__ x_q, float* __restrict__ x_s, int scale_rule,
    int32_t* __restrict__ zero, int zero_n, int32_t* bar, int32_t* err) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = (int)gridDim.x, b = (int)blockIdx.x;
    // this CTA's tokens [t0, t1), their flat indices [i0, i1) and (token, group) items [q0, q1); warp w converts
    // items q0 + 2 w + (lane >> 4) + 16 j
    const int tpc = (T + G - 1) / G;
    const int t0 = min(T, b * tpc), t1 = min(T, t0 + tpc);
    const int i0 = t0 * k, i1 = t1 * k;
    const long q0 = (long)t0 * (H / 128), q1 = (long)t1 * (H / 128);
    QuantItem item = quant_fp8_load(x, H, q0 + 2 * warp + (lane >> 4), q1);  // x is not written by the predecessor
    pdl_wait();
    pdl_trigger();
    if (part != nullptr || logits_in != nullptr) {
        for (int t = t0 + warp; t < t1; t += 8) {
            float v[EPT];
            if (part != nullptr) {
                logits_from_partials(part, chunks, T, t, E, bias, logits_out, v);
            } else {
#pragma unroll
                for (int i = 0; i < EPT; ++i) {
                    const int e = lane + 32 * i;
                    v[i] = e < E ? __bfloat162float(logits_in[(size_t)t * E + e]) + (bias != nullptr ? bias[e] : 0.0f)
                                 : -INFINITY;
                }
            }
            warp_topk(v, E, k, topk_w + (size_t)t * k, topk_ids + (size_t)t * k);
        }
    }
    for (int i = b * 256 + tid; i < zero_n; i += G * 256) zero[i] = 0;
    quant_fp8_finish(item, scale_rule);
    if (!front_grid_sync(bar, err)) return;

    // all n = T*k expert ids, the counts per expert and the padded offsets
    const int n = T * k;
    extern __shared__ int32_t fsm[];
    int32_t* ids = fsm;        // [n] expert of each flat index
    int32_t* tot = fsm + n;    // [E] indices per expert
    int32_t* below = tot + E;  // [E] indices per expert before i0
    int32_t* pad = below + E;  // [E] padded offset of each expert
    int32_t* cslot = pad + E;  // [i1 - i0] slot of each of this CTA's indices
    __shared__ int32_t wsum[8];
    for (int e = tid; e < E; e += 256) tot[e] = below[e] = 0;
    for (int j = tid; j < n; j += 256) ids[j] = __ldcg(topk_ids + j);  // written by other CTAs: not the nc path
    __syncthreads();
    for (int j = tid; j < n; j += 256) {
        const int e = ids[j];
        if (e >= 0 && e < E) {
            atomicAdd(&tot[e], 1);
            if (j < i0) atomicAdd(&below[e], 1);
        }
    }
    __syncthreads();
    // exclusive scan of the padded totals: thread t owns experts [4t, 4t + 4)
    int loc[4], run = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int e = 4 * tid + j;
        const int p = e < E ? (tot[e] + kBlockM - 1) / kBlockM * kBlockM : 0;
        loc[j] = run;
        run += p;
    }
    int inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v2 = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v2;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    int wpre = 0, total = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        wpre += w < warp ? wsum[w] : 0;
        total += wsum[w];
    }
    const int tpre = wpre + inc - run;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int e = 4 * tid + j;
        if (e < E) pad[e] = tpre + loc[j];
    }
    __syncthreads();

    // this CTA's indices, a thread each
    for (int i = i0 + tid; i < i1; i += 256) {
        const int e = ids[i];
        int c = 0;
        for (int j = i0; j < i; ++j) c += ids[j] == e ? 1 : 0;
        const int sl = (e >= 0 && e < E) ? pad[e] + below[e] + c : -1;  // an expert outside [0, E) has no slot
        cslot[i - i0] = sl;
        if (sl >= 0) sorted[sl] = i;
        slot_of[i] = sl;
    }
    // the padding slots and the block table, a warp per expert; the offsets
    for (int e = b * 8 + warp; e < E; e += G * 8) {
        const int off = pad[e], te = tot[e];
        const int padded = (te + kBlockM - 1) / kBlockM * kBlockM;
        for (int blk = off / kBlockM + lane; blk < (off + padded) / kBlockM; blk += 32) expert_ids[blk] = e;
        for (int i = off + te + lane; i < off + padded; i += 32) sorted[i] = n;
    }
    if (b == 0) {
        if (expert_off != nullptr)
            for (int e = tid; e < E; e += 256) expert_off[e] = pad[e];
        if (tid == 0) {
            *num_post_pad = total;
            if (expert_off != nullptr) expert_off[E] = total;
        }
    }
    __syncthreads();

    // this CTA's rows into their k slots
    for (long q = q0 + 2 * warp; q < q1; q += 16) {
        if (q != q0 + 2 * warp) {
            item = quant_fp8_load(x, H, q + (lane >> 4), q1);
            quant_fp8_finish(item, scale_rule);
        }
        if (!item.valid) continue;
        for (int c = 0; c < k; ++c) {
            const int sl = cslot[(int)item.row * k + c - i0];
            if (sl >= 0) store_quant_item(item, H, (size_t)sl, x_q, x_s);
        }
    }
}

}  // namespace

// ids [T*k]; tot, below and pad [E] each; cslot [tokens per CTA * k]
static size_t front_small_smem(int T, int E, int k, int grid) {
    const int tpc = (T + grid - 1) / grid;
    return sizeof(int32_t) * ((size_t)T * k + 3 * (size_t)E + (size_t)tpc * k);
}

cudaError_t launch_front_small(const float* part, int chunks, const void* logits_in, void* logits_out,
                               const float* bias, int T, int E, int k, float* topk_w, int32_t* topk_ids,
                               int32_t* sorted, int32_t* expert_ids, int32_t* num_post_pad, int32_t* expert_off,
                               int32_t* slot_of, const void* x, int H, uint8_t* x_q, float* x_s, int scale_rule,
                               int32_t* zero, int zero_n, int32_t* bar, int32_t* err, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    if ((long)T * k > kFrontMaxIndices || E > kMaxExperts) return cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // a CTA per token up to one per SM (every CTA must be resident for the grid barrier: 256 threads and at most
    // 28 KB of shared memory each)
    const dim3 grid(T < sms ? T : sms);
    const size_t smem = front_small_smem(T, E, k, (int)grid.x);
    if (E <= 128)
        PM_TRY(launch_pdl(front_small_kernel<4>, grid, dim3(256), smem, s, part, chunks,
                          static_cast<const __nv_bfloat16*>(logits_in), static_cast<__nv_bfloat16*>(logits_out), bias,
                          T, E, k, topk_w, topk_ids, sorted, expert_ids, num_post_pad, expert_off, slot_of,
                          static_cast<const __nv_bfloat16*>(x), H, x_q, x_s, scale_rule, zero, zero_n, bar, err));
    else
        PM_TRY(launch_pdl(front_small_kernel<kMaxEPT>, grid, dim3(256), smem, s, part, chunks,
                          static_cast<const __nv_bfloat16*>(logits_in), static_cast<__nv_bfloat16*>(logits_out), bias,
                          T, E, k, topk_w, topk_ids, sorted, expert_ids, num_post_pad, expert_off, slot_of,
                          static_cast<const __nv_bfloat16*>(x), H, x_q, x_s, scale_rule, zero, zero_n, bar, err));
    return cudaGetLastError();
}

cudaError_t launch_topk(const void* logits, const float* bias, int T, int E, int k, float* topk_w, int32_t* topk_ids,
                        cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    const int blocks = cdiv((long)T * 32, 256);
    if (E <= 128)
        PM_TRY(launch_pdl(topk_kernel<4>, dim3(blocks), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(logits),
                          bias, T, E, k, topk_w, topk_ids));
    else
        PM_TRY(launch_pdl(topk_kernel<kMaxEPT>, dim3(blocks), dim3(256), 0, s,
                          static_cast<const __nv_bfloat16*>(logits), bias, T, E, k, topk_w, topk_ids));
    return cudaGetLastError();
}

cudaError_t launch_topk_partials(const float* part, int chunks, void* logits, const float* bias, int T, int E, int k,
                                 float* topk_w, int32_t* topk_ids, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    const int blocks = cdiv((long)T * 32, 256);
    if (E <= 128)
        PM_TRY(launch_pdl(topk_partials_kernel<4>, dim3(blocks), dim3(256), 0, s, part, chunks,
                          static_cast<__nv_bfloat16*>(logits), bias, T, E, k, topk_w, topk_ids));
    else
        PM_TRY(launch_pdl(topk_partials_kernel<kMaxEPT>, dim3(blocks), dim3(256), 0, s, part, chunks,
                          static_cast<__nv_bfloat16*>(logits), bias, T, E, k, topk_w, topk_ids));
    return cudaGetLastError();
}

cudaError_t launch_align(const int32_t* ids, int n, int E, int32_t* counts, int32_t* sorted, int32_t* expert_ids,
                         int32_t* num_post_pad, int32_t* expert_off, int32_t* slot_of, cudaStream_t s) {
    if (E > kAlignEPT * 256) return cudaErrorInvalidValue;
    const int chunk = align_chunk(n);
    const int nchunks = align_chunks(n);
    if (nchunks > 1) {
        PM_TRY(launch_pdl(align_count_kernel, dim3(nchunks), dim3(256), sizeof(int32_t) * E, s, ids, n, E, chunk,
                          counts));
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    // a single chunk is scattered by CTA 0; the extra CTAs only share the padding writes
    const int grid = nchunks > 1 ? nchunks : max(1, min(16, E / 8));
    const size_t smem = sizeof(int32_t) * (3 * (size_t)E + (size_t)(nchunks > 1 ? 8 * E : max(8 * E, E + 1024)));
    PM_TRY(launch_pdl(align_scatter_kernel, dim3(grid), dim3(256), smem, s, ids, n, E, chunk,
                      nchunks, nchunks > 1 ? counts : nullptr, sorted, expert_ids, num_post_pad, expert_off,
                      slot_of));
    return cudaGetLastError();
}

}  // namespace pm
