// Expert parallelism over peer memory (no counterpart in the reference, which runs the layer on one device).
//
// Every rank holds one region with the same layout, mapped into every other rank's address space (CUDA IPC over
// NVLink).  One layer call, with no host synchronisation and no collective library on the data path:
//   1. count: rank s counts its (token, slot) pairs per global expert and stores that row into row s of every
//      rank's count matrix [G][E] (peer stores); barrier.
//   2. offsets: every rank now holds the whole matrix and derives, for each global expert e, where its own pairs of
//      e start in the owning rank's slot space (experts padded to 128 slots, sources in rank order, a source's pairs
//      in ascending flat order — exactly the single-GPU alignment restricted to the owner's experts), plus the
//      block table and slot count of its own experts.
//   3. dispatch: each token is quantised once (per-128 e4m3, IEEE division, as the single-GPU path) and its row is
//      stored straight into the owner's slot of each of its k pairs, with (source rank, pair, routing weight);
//      barrier.
//   4. the owner runs its local gate_up / down GEMMs on its slots (the existing kernels); the down GEMM's
//      epilogue stores each slot's weighted bf16 row straight into the source rank's result row for that pair
//      (per-slot destination addresses), so the return overlaps the GEMM; barrier; then the ordinary fixed-order
//      combine.
// The rows, their arithmetic and the combine order are those of one GPU, so the result is bit-identical.
//
// Barrier: a one-thread kernel adds 1 to every rank's counter (system-scope atomics after a system fence) and
// waits, bounded by the call's limit (PM_WAIT_TIMEOUT_NS when it gives 0), until its own counter reaches the call's target; on timeout it sets the
// error word and returns.  Only plain peer loads/stores/atomics are used (no multicast).
#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

// ---------------------------------------------------------------------------------------------- count
__global__ void __launch_bounds__(1024) ep_count_kernel(const int32_t* __restrict__ ids, int n, int E, int G,
                                                        int rank, const uint64_t* __restrict__ peer_cm) {
    pdl_wait();
    pdl_trigger();
    __shared__ int cnt[kMaxExperts];
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = ids[i];
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    for (int q = threadIdx.x; q < G * E; q += blockDim.x) {
        const int d = q / E, e = q % E;
        reinterpret_cast<int32_t*>(peer_cm[d])[(size_t)rank * E + e] = cnt[e];
    }
}

// ---------------------------------------------------------------------------------------------- barrier
__global__ void ep_barrier_kernel(const uint64_t* __restrict__ peer_flag, unsigned* own_flag, int G,
                                  unsigned target, int32_t* err, uint64_t limit_ns) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    __threadfence_system();
    for (int d = 0; d < G; ++d) atomicAdd_system(reinterpret_cast<unsigned*>(peer_flag[d]), 1u);
    const uint64_t t0 = globaltimer();
    while (true) {
        const unsigned v = *reinterpret_cast<volatile unsigned*>(own_flag);
        if ((int)(v - target) >= 0) break;  // counters only grow (wrap-safe comparison)
        if (globaltimer() - t0 > limit_ns) {
            if (err != nullptr) atomicExch(err, 1);
            return;
        }
    }
    __threadfence_system();
}

// ---------------------------------------------------------------------------------------------- offsets
// cm [G][E] counts; own bases base[e] for every global expert; block table / slot count of this rank's experts.
// bounds (may be null): with `groups` groups of epr / groups local experts each, bounds[g] = the first slot of group
// g's experts and bounds[groups] = the slot count (a group's tiles can then run while a later group is dispatched).
__global__ void __launch_bounds__(kMaxExperts) ep_offsets_kernel(const int32_t* __restrict__ cm, int G, int E,
                                                                 int epr, int rank, int32_t* __restrict__ base,
                                                                 int32_t* __restrict__ expert_ids,
                                                                 int32_t* __restrict__ npp, int cap_blocks,
                                                                 int32_t* err, int32_t* __restrict__ bounds,
                                                                 int groups) {
    pdl_wait();
    pdl_trigger();
    __shared__ int padded[kMaxExperts];
    const int e = threadIdx.x;
    int tot = 0, pre = 0;
    if (e < E) {
        for (int s = 0; s < G; ++s) {
            const int v = cm[(size_t)s * E + e];
            tot += v;
            if (s < rank) pre += v;
        }
        padded[e] = (tot + kBlockM - 1) / kBlockM * kBlockM;
    }
    __syncthreads();
    if (e >= E) return;
    const int d = e / epr;
    int off = 0;
    for (int e2 = d * epr; e2 < e; ++e2) off += padded[e2];
    base[e] = off + pre;
    if (d == rank) {
        const int el = e - rank * epr;
        for (int b = off / kBlockM; b < (off + padded[e]) / kBlockM; ++b) {
            if (b < cap_blocks) expert_ids[b] = el;
            else atomicExch(err, 1);
        }
        if (bounds != nullptr && el % (epr / groups) == 0) bounds[el / (epr / groups)] = off;
        if (el == epr - 1) {
            *npp = off + padded[e];
            if (bounds != nullptr) bounds[groups] = off + padded[e];
        }
    }
}

// ---------------------------------------------------------------------------------------------- dispatch
// One half-warp per (token, 128-column group), as the single-GPU quantisation; each of the token's k rows goes
// to slot base[e] + (rank of the pair among this rank's pairs of expert e) of the owner of e.
struct PeerPtrs {
    const uint64_t* a1;    // [G] e4m3 [cap, H]
    const uint64_t* a1s;   // [G] f32 [cap, H/128]
    const uint64_t* meta;  // [G] i32 [cap]: source rank << 24 | pair index (-1: padding)
    const uint64_t* wgt;   // [G] f32 [cap]
};

// One (token, 128-column group) item per half-warp: a lane's 8 columns, the group's amax over the half-warp, the
// quantised row stored to the owners' slots of the pairs in [le_lo, le_hi).  ILP items per lane are loaded before
// any is processed (a launch on few SMs keeps that many loads in flight per warp).
template <int ILP>
__device__ __forceinline__ void ep_dispatch_items(const __nv_bfloat16* __restrict__ x, int T, int H, int k,
                                                  const int32_t* __restrict__ ids, const float* __restrict__ topk_w,
                                                  const int32_t* __restrict__ slot_local,
                                                  const int32_t* __restrict__ off_local,
                                                  const int32_t* __restrict__ base, int E, int epr, int rank,
                                                  int cap, const PeerPtrs& peers, int32_t* err, int le_lo, int le_hi) {
    const int lane = threadIdx.x & 31, sub = lane & 15;
    const int G128 = H / 128;
    const long items = (long)T * G128;
    const long pairs = (items + 1) / 2;
    const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
    for (long wp0 = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wp0 < pairs; wp0 += nwarps * ILP) {
        uint4 raw[ILP];
#pragma unroll
        for (int u = 0; u < ILP; ++u) {
            const long item = 2 * (wp0 + u * nwarps) + (lane >> 4);
            raw[u] = make_uint4(0, 0, 0, 0);
            if (wp0 + u * nwarps < pairs && item < items)
                raw[u] = *reinterpret_cast<const uint4*>(x + (item / G128) * H + (int)(item % G128) * 128 + sub * 8);
        }
#pragma unroll
        for (int u = 0; u < ILP; ++u) {
            const long wp = wp0 + u * nwarps;
            const long item = 2 * wp + (lane >> 4);
            const bool valid = wp < pairs && item < items;
            const long t = valid ? item / G128 : 0;
            const int g = valid ? (int)(item % G128) : 0;
            const int col = g * 128 + sub * 8;
            float v[8];
            float amax = 0.0f;
            const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw[u]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[i] = __bfloat162float(b[i]);
                amax = fmaxf(amax, fabsf(v[i]));
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            // (an invalid half-warp item goes through the shuffles below with every destination skipped)
            const float sc = e4m3_group_scale(amax, kScaleDiv);
            uint32_t packed[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float q0 = fminf(fmaxf(__fdiv_rn(v[4 * i + 0], sc), -448.0f), 448.0f);
                const float q1 = fminf(fmaxf(__fdiv_rn(v[4 * i + 1], sc), -448.0f), 448.0f);
                const float q2 = fminf(fmaxf(__fdiv_rn(v[4 * i + 2], sc), -448.0f), 448.0f);
                const float q3 = fminf(fmaxf(__fdiv_rn(v[4 * i + 3], sc), -448.0f), 448.0f);
                packed[i] = (uint32_t)e4m3x2(q0, q1) | ((uint32_t)e4m3x2(q2, q3) << 16);
            }
            // lane j of the half-warp resolves pair j's owner and slot (-1: skipped), all k at once
            int my_d = -1, my_slot = -1;
            float my_w = 0.0f;
            if (valid && sub < k) {
                const long p = t * k + sub;
                const int e = ids[p];
                if (e < 0 || e >= E) {
                    atomicExch(err, 1);
                } else {
                    const int d = e / epr;
                    if (e - d * epr >= le_lo && e - d * epr < le_hi) {  // else another group's pair
                        const int slot = base[e] + (slot_local[p] - off_local[e]);
                        if (slot < 0 || slot >= cap) {
                            atomicExch(err, 1);
                        } else {
                            my_d = d;
                            my_slot = slot;
                            my_w = topk_w[p];
                        }
                    }
                }
            }
            for (int j = 0; j < k; ++j) {
                const long p = t * k + j;
                const int d = __shfl_sync(0xffffffffu, my_d, j, 16);
                const int slot = __shfl_sync(0xffffffffu, my_slot, j, 16);
                const float wj = __shfl_sync(0xffffffffu, my_w, j, 16);
                if (slot < 0) continue;
                uint8_t* a1 = reinterpret_cast<uint8_t*>(peers.a1[d]);
                *reinterpret_cast<uint2*>(a1 + (size_t)slot * H + col) = make_uint2(packed[0], packed[1]);
                if (sub == 0) reinterpret_cast<float*>(peers.a1s[d])[(size_t)slot * G128 + g] = sc;
                if (sub == 0 && g == 0) {
                    reinterpret_cast<int32_t*>(peers.meta[d])[slot] = (rank << 24) | (int)p;
                    reinterpret_cast<float*>(peers.wgt[d])[slot] = wj;
                }
            }
        }
    }
}

template <int ILP>
__global__ void __launch_bounds__(1024) ep_dispatch_quant_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int H, int k, const int32_t* __restrict__ ids,
    const float* __restrict__ topk_w, const int32_t* __restrict__ slot_local, const int32_t* __restrict__ off_local,
    const int32_t* __restrict__ base, int E, int epr, int rank, int cap, PeerPtrs peers, int32_t* err, int le_lo,
    int le_hi) {
    pdl_wait();
    pdl_trigger();
    ep_dispatch_items<ILP>(x, T, H, k, ids, topk_w, slot_local, off_local, base, E, epr, rank, cap, peers, err, le_lo,
                           le_hi);
}

// ---------------------------------------------------------------------------------------------- local rows
// For each filled slot, the address of its source rank's result row for its pair (0 for padding): the local down
// GEMM stores each weighted row there directly, over NVLink when the source is another rank.
__global__ void ep_local_rows_kernel(const int32_t* __restrict__ meta, const int32_t* __restrict__ npp, int cap,
                                     int H, int G, int n_pairs, const uint64_t* __restrict__ peer_back,
                                     uint64_t* __restrict__ dst_rows, int32_t* err) {
    pdl_wait();
    pdl_trigger();
    const int n = *npp;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cap; i += gridDim.x * blockDim.x) {
        uint64_t d = 0;
        const int m = i < n ? meta[i] : -1;
        if (m >= 0) {
            const int s = m >> 24, p = m & 0xFFFFFF;
            if (s < G && p < n_pairs) d = peer_back[s] + (uint64_t)p * H * sizeof(__nv_bfloat16);
            else atomicExch(err, 1);
        }
        dst_rows[i] = d;
    }
}

int grid_for(long work_items, int per_block, int sms) {
    const long want = (work_items + per_block - 1) / per_block;
    const long cap = (long)sms * 8;
    return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

cudaError_t launch_ep_count(const int32_t* ids, int n, int E, int G, int rank, const uint64_t* peer_cm,
                            cudaStream_t s) {
    PM_TRY(launch_pdl(ep_count_kernel, dim3(1), dim3(1024), 0, s, ids, n, E, G, rank, peer_cm));
    return cudaGetLastError();
}

cudaError_t launch_ep_barrier(const uint64_t* peer_flag, unsigned* own_flag, int G, unsigned target, int32_t* err,
                              uint64_t limit_ns, cudaStream_t s) {
    // A plain launch: the barrier publishes its predecessor's peer stores to the other ranks, so it starts only
    // after that kernel has fully completed in stream order.
    ep_barrier_kernel<<<1, 32, 0, s>>>(peer_flag, own_flag, G, target, err,
                                       limit_ns != 0 ? limit_ns : (uint64_t)PM_WAIT_TIMEOUT_NS);
    return cudaGetLastError();
}

cudaError_t launch_ep_offsets(const int32_t* cm, int G, int E, int epr, int rank, int32_t* base, int32_t* expert_ids,
                              int32_t* npp, int cap_blocks, int32_t* err, int32_t* bounds, int groups,
                              cudaStream_t s) {
    if (E > kMaxExperts) return cudaErrorInvalidValue;
    if (bounds != nullptr && (groups < 1 || epr % groups != 0)) return cudaErrorInvalidValue;
    PM_TRY(launch_pdl(ep_offsets_kernel, dim3(1), dim3(kMaxExperts), 0, s, cm, G, E, epr, rank, base, expert_ids,
                      npp, cap_blocks, err, bounds, groups));
    return cudaGetLastError();
}

cudaError_t launch_ep_dispatch_quant(const void* x, int T, int H, int k, const int32_t* ids, const float* topk_w,
                                     const int32_t* slot_local, const int32_t* off_local, const int32_t* base,
                                     int E, int epr, int rank, int cap, const uint64_t* peer_a1, const uint64_t* peer_a1s,
                                     const uint64_t* peer_meta, const uint64_t* peer_wgt, int32_t* err, int sms,
                                     int le_lo, int le_hi, int ctas, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    PeerPtrs p{peer_a1, peer_a1s, peer_meta, peer_wgt};
    const long pairs = ((long)T * (H / 128) + 1) / 2;
    if (ctas > 0)  // a few wide CTAs (one per SM left free beside a GEMM), four items in flight per warp
        PM_TRY(launch_pdl(ep_dispatch_quant_kernel<4>, dim3(ctas), dim3(1024), 0, s,
                          static_cast<const __nv_bfloat16*>(x), T, H, k, ids, topk_w, slot_local, off_local, base, E,
                          epr, rank, cap, p, err, le_lo, le_hi));
    else
        PM_TRY(launch_pdl(ep_dispatch_quant_kernel<1>, dim3(grid_for(pairs, 8, sms * 2)), dim3(256), 0, s,
                          static_cast<const __nv_bfloat16*>(x), T, H, k, ids, topk_w, slot_local, off_local, base, E,
                          epr, rank, cap, p, err, le_lo, le_hi));
    return cudaGetLastError();
}

cudaError_t launch_ep_local_rows(const int32_t* meta, const int32_t* npp, int cap, int H, int G, int n_pairs,
                                 const uint64_t* peer_back, uint64_t* dst_rows, int32_t* err, int sms,
                                 cudaStream_t s) {
    PM_TRY(launch_pdl(ep_local_rows_kernel, dim3(grid_for(cap, 256, sms)), dim3(256), 0, s, meta, npp, cap, H, G,
                      n_pairs, peer_back, dst_rows, err));
    return cudaGetLastError();
}

}  // namespace pm
