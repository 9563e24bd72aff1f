// Router projection on the tensor cores, fused with softmax / top-k / renormalise.
//
// logits[t, e] = bf16(sum_h x[t, h] * W[e, h]) (prismyra/kernels/qwen3_moe.py:169-171, the batch-invariant
// router: bf16 operands, fp32 accumulation, bf16 result), then vLLM fused_topk(renormalize=True) semantics
// (router/fused_topk_router.py:69-113): p = softmax(logits) in fp32, the k largest (equal values: lower expert
// index first), weights = p / sum of the selected p.
//
// The fp32 reduction over h is fixed: the tcgen05 kind::f16 MMAs (M=128 tokens, N=32 experts, K=16 per
// instruction) accumulate each 256-column chunk c of H into a partial P_c in TMEM, and the logit is
// bf16(((P_0 + P_1) + P_2) + ...), chunks in ascending order.  Two launch shapes compute exactly that:
//   fused  one CTA per (128 tokens, 32 experts): P_c alternate between two TMEM accumulators and the epilogue
//          warps add them in order as they complete, then write bf16 logits;
//   split  (few tokens) one CTA per (128 tokens, 32 experts, chunk c), so a short call still spreads over many
//          SMs: each writes its P_c in fp32 and the top-k kernel adds the chunks in the same order, rounds,
//          writes the logits and ranks.
// Either way a row's result never depends on which rows share the call or which shape ran.
#include <atomic>

#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

constexpr int kTM = 128;       // tokens per CTA
constexpr int kTN = 32;        // experts per CTA
constexpr int kTK = 64;        // bf16 columns of H per stage (128-byte rows)
constexpr int kChunkK = 256;   // columns of H per partial P_c
constexpr int kStepsPerChunk = kChunkK / kTK;
// Pipeline depth: deep when the grid fits on the SMs one CTA each (few CTAs, latency-bound streaming),
// shallower when two CTAs per SM are needed to cover the grid in one wave.
constexpr int kTStagesDeep = 10;
constexpr int kTStagesWide = 5;
constexpr int kTXBytes = kTM * kTK * 2;  // 16 KB
constexpr int kTWBytes = kTN * kTK * 2;  // 4 KB
constexpr int kTStageBytes = kTXBytes + kTWBytes;

template <int STAGES>
struct RouterTail {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t pfull[2];   // chunk partial c is in TMEM accumulator c % 2
    uint64_t pempty[2];  // the epilogue has read it
    uint32_t tmem_base;
    int abort;
};

template <int STAGES>
constexpr size_t router_smem() {
    return 1024 + (size_t)STAGES * kTStageBytes + sizeof(RouterTail<STAGES>);
}

// SPLIT: this CTA computes the single chunk blockIdx.z and stores it to part[c][t][e] (fp32); otherwise it
// computes every chunk and stores bf16 logits.
constexpr int kRouterThreads = 192;
constexpr int kClearWords = 4;  // status words a launch given `clear` zeroes  // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 epilogue (lane quarter = warp % 4)

template <int STAGES, bool SPLIT>
__global__ void __launch_bounds__(kRouterThreads, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, int T, int H,
                     int E, __nv_bfloat16* __restrict__ logits, float* __restrict__ part, int* err, int* clear) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    RouterTail<STAGES>* tail = reinterpret_cast<RouterTail<STAGES>*>(smem + (size_t)STAGES * kTStageBytes);
    volatile int* abort = &tail->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kTM, e0 = blockIdx.y * kTN;
    const int c_lo = SPLIT ? (int)blockIdx.z : 0, c_hi = SPLIT ? c_lo + 1 : H / kChunkK;
    constexpr uint32_t kCols = SPLIT ? 32 : 64;

    if (threadIdx.x == 0) {
        for (int st = 0; st < STAGES; ++st) {
            mbar_init(smem_u32(&tail->full[st]), 1);
            mbar_init(smem_u32(&tail->empty[st]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tail->pfull[b]), 1);
            mbar_init(smem_u32(&tail->pempty[b]), 4);
        }
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        prefetch_tensormap(&tm_x);
        prefetch_tensormap(&tm_w);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    pdl_wait();
    pdl_trigger();
    // the forward's status words, zeroed by its first kernel in place of a memset (which would stop the previous
    // forward's last kernel and this one from overlapping): CTA 0 does it at once, long before any wait of this
    // grid could time out and raise them
    if (clear != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) {
#pragma unroll
        for (int i = 0; i < kClearWords; ++i) clear[i] = 0;
    }

    if (warp == 0 && lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        for (int kb = c_lo * kStepsPerChunk; kb < c_hi * kStepsPerChunk; ++kb) {
            if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, abort)) break;
            const uint32_t xd = sbase + stage * kTStageBytes;
            const uint32_t fb = smem_u32(&tail->full[stage]);
            mbar_arrive_expect_tx(fb, kTStageBytes);
            tma_load_2d(xd, &tm_x, fb, kb * kTK, t0);
            tma_load_2d(xd + kTXBytes, &tm_w, fb, kb * kTK, e0);
            if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = idesc_f32acc(1 /*bf16*/, 1 /*bf16*/, kTM, kTN);
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int c = c_lo; c < c_hi && ok; ++c) {
            const uint32_t buf = (uint32_t)(c - c_lo) & 1u, use = (uint32_t)(c - c_lo) >> 1;
            if (!SPLIT && !mbar_wait(smem_u32(&tail->pempty[buf]), (use & 1u) ^ 1u, abort)) break;
            const uint32_t d = tmem + buf * kTN;
            for (int kk = 0; kk < kStepsPerChunk; ++kk) {
                if (!mbar_wait(smem_u32(&tail->full[stage]), phase, abort)) { ok = false; break; }
                tc_fence_after();
                const uint32_t xa = sbase + stage * kTStageBytes;
                const uint64_t da = desc_kmajor_sw128(xa), db = desc_kmajor_sw128(xa + kTXBytes);
#pragma unroll
                for (int j = 0; j < kTK / 16; ++j)  // 16 bf16 (32 bytes) of K per instruction
                    mma_f16(d, da + 2 * j, db + 2 * j, idesc, (kk | j) != 0 ? 1u : 0u);
                mma_commit(smem_u32(&tail->empty[stage]));
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (ok) mma_commit(smem_u32(&tail->pfull[buf]));
        }
    }
    __syncwarp();

    // Epilogue (warps 2-5): TMEM lane row = token t0 + row and its 32 experts; partials are added in chunk order.
    const int row = (warp & 3) * 32 + lane;
    float acc[32];
    bool ok = warp >= 2;
    for (int c = c_lo; c < c_hi && warp >= 2; ++c) {
        const uint32_t buf = (uint32_t)(c - c_lo) & 1u, use = (uint32_t)(c - c_lo) >> 1;
        if (!mbar_wait(smem_u32(&tail->pfull[buf]), use & 1u, abort)) { ok = false; break; }
        tc_fence_after();
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)((warp & 3) * 32) << 16) + buf * kTN, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = c == c_lo ? __uint_as_float(r[i]) : acc[i] + __uint_as_float(r[i]);
        tc_fence_before();
        __syncwarp();
        if (!SPLIT && lane == 0) mbar_arrive(smem_u32(&tail->pempty[buf]));
    }
    const int t = t0 + row;
    if (ok && t < T) {
        if (SPLIT) {
            float* dst = part + ((size_t)c_lo * T + t) * E + e0;
            if (e0 + kTN <= E && (E & 3) == 0) {
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    reinterpret_cast<float4*>(dst)[u] = make_float4(acc[4 * u], acc[4 * u + 1], acc[4 * u + 2],
                                                                    acc[4 * u + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < kTN; ++i)
                    if (e0 + i < E) dst[i] = acc[i];
            }
        } else if (e0 + kTN <= E && (E & 7) == 0) {
            uint4* dst = reinterpret_cast<uint4*>(logits + (size_t)t * E + e0);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                uint4 o;
                __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                for (int i = 0; i < 4; ++i) ob[i] = __floats2bfloat162_rn(acc[8 * u + 2 * i], acc[8 * u + 2 * i + 1]);
                dst[u] = o;
            }
        } else {
#pragma unroll
            for (int i = 0; i < kTN; ++i)
                if (e0 + i < E) logits[(size_t)t * E + e0 + i] = __float2bfloat16_rn(acc[i]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
    }
    if (threadIdx.x == 0 && tail->abort && err != nullptr) atomicExch(err, 1);
}

template <int STAGES, bool SPLIT>
cudaError_t configure_router() {
    return cudaFuncSetAttribute(router_tc_kernel<STAGES, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)router_smem<STAGES>());
}

}  // namespace

int router_chunks(int H) { return H / kChunkK; }

size_t router_split_bytes(int T, int H, int E) {
    // the split shape when the fused grid would occupy few SMs
    if (T <= 0 || (long)cdiv(T, kTM) * cdiv(E, kTN) > 64) return 0;
    return (size_t)(H / kChunkK) * T * E * sizeof(float);
}

cudaError_t launch_router_topk(const void* x, const void* w, const float* bias, int T, int H, int E, int k,
                               void* logits, float* topk_w, int32_t* topk_ids, int32_t* err, cudaStream_t s,
                               float* part, bool topk, int32_t* clear) {
    if (T == 0) return cudaSuccess;
    if (logits == nullptr || H % kChunkK != 0) return cudaErrorInvalidValue;
    CUtensorMap tx, tw;
    if (!encode_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H, (uint64_t)T, (uint64_t)H * 2,
                        kTK, kTM) ||
        !encode_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H, (uint64_t)E, (uint64_t)H * 2, kTK,
                        kTN))
        return cudaErrorInvalidValue;
    static std::atomic<bool> configured[64];  // zero-initialised: false
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (dev < 64 && !configured[dev].load(std::memory_order_acquire)) {
        cudaError_t e = configure_router<kTStagesDeep, false>();
        if (e == cudaSuccess) e = configure_router<kTStagesWide, false>();
        if (e == cudaSuccess) e = configure_router<kStepsPerChunk, true>();
        if (e != cudaSuccess) return e;
        configured[dev].store(true, std::memory_order_release);
    }
    __nv_bfloat16* lg = static_cast<__nv_bfloat16*>(logits);
    const int chunks = H / kChunkK;
    if (part != nullptr && router_split_bytes(T, H, E) > 0) {
        const dim3 grid(cdiv(T, kTM), cdiv(E, kTN), chunks);
        PM_TRY(launch_pdl(router_tc_kernel<kStepsPerChunk, true>, dim3(grid), dim3(kRouterThreads),
                          router_smem<kStepsPerChunk>(), s, tx, tw, T, H, E, lg, part, err, clear));
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess || !topk) return e;
        return launch_topk_partials(part, chunks, lg, bias, T, E, k, topk_w, topk_ids, s);
    }
    const dim3 grid(cdiv(T, kTM), cdiv(E, kTN));
    if ((long)grid.x * grid.y <= sms)
        PM_TRY(launch_pdl(router_tc_kernel<kTStagesDeep, false>, dim3(grid), dim3(kRouterThreads),
                          router_smem<kTStagesDeep>(), s, tx, tw, T, H, E, lg, nullptr, err, clear));
    else
        PM_TRY(launch_pdl(router_tc_kernel<kTStagesWide, false>, dim3(grid), dim3(kRouterThreads),
                          router_smem<kTStagesWide>(), s, tx, tw, T, H, E, lg, nullptr, err, clear));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !topk) return e;
    return launch_topk(logits, bias, T, E, k, topk_w, topk_ids, s);
}

}  // namespace pm
