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

    uint32_t used = 0;
    float sel = 0.0f, my_p = 0.0f;
    int my_id = 0;
    for (int j = 0; j < k; ++j) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((used >> i) & 1u) && (v[i] > bv || bi == 0x7fffffff)) {
                bv = v[i];
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        float mine = 0.0f;
        if ((bi & 31) == lane) {
            const int slot = bi >> 5;
            used |= 1u << slot;
#pragma unroll
            for (int i = 0; i < EPT; ++i)
                if (i == slot) mine = ex[i];
        }
        const float p = __shfl_sync(0xffffffffu, mine, bi & 31) / sum;
        sel += p;
        if (lane == j) {
            my_p = p;
            my_id = bi;
        }
    }
    if (lane < k) {
        w_out[lane] = my_p / sel;
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

// The same from the router's fp32 chunk partials: logit = bf16(((P_0 + P_1) + P_2) + ...), written out, then ranked.
template <int EPT>
__global__ void __launch_bounds__(256) topk_partials_kernel(const float* __restrict__ part, int chunks,
                                                            __nv_bfloat16* __restrict__ logits,
                                                            const float* __restrict__ bias, int T, int E, int k,
                                                            float* __restrict__ topk_w,
                                                            int32_t* __restrict__ topk_ids) {
    pdl_wait();
    pdl_trigger();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= T) return;
    float v[EPT];
    // all of this lane's chunk partials are loaded before any is added (one round trip for up to 8 chunks), then
    // added in chunk order
    constexpr int kC = 8;
    for (int c0 = 0; c0 < chunks; c0 += kC) {
        float pv[EPT][kC];
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
            const int e = lane + 32 * i;
#pragma unroll
            for (int j = 0; j < kC; ++j)
                pv[i][j] = (e < E && c0 + j < chunks) ? part[((size_t)(c0 + j) * T + warp) * E + e] : 0.0f;
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
            logits[(size_t)warp * E + e] = b;
            v[i] = __bfloat162float(b) + (bias != nullptr ? bias[e] : 0.0f);
        } else {
            v[i] = -INFINITY;
        }
    }
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

}  // namespace

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
