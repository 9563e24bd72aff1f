// Router projection on the tensor cores, fused with softmax / top-k / renormalise.
//
// logits[t, e] = bf16(sum_h x[t, h] * W[e, h]) (prismyra/kernels/qwen3_moe.py:169-171, the batch-invariant
// router: bf16 operands, fp32 accumulation, bf16 result), then vLLM fused_topk(renormalize=True) semantics
// (router/fused_topk_router.py:69-113): p = softmax(logits) in fp32, the k largest (equal values: lower expert
// index first), weights = p / sum of the selected p.
//
// One CTA = 128 tokens x 32 experts: tcgen05 kind::f16 MMAs (M=128, N=32, K=16 per instruction) accumulate the
// whole H reduction in TMEM, fed by a 4-stage TMA pipeline of 64-column slices; the grid covers the experts in
// 32-wide slices, so even a 128-token call spreads over E/32 SMs.  Every token's logits are reduced in the same
// fixed order whatever the token count, so a row's result never depends on which rows share the call.  The
// epilogue writes bf16 logits; the ranking (softmax / top-k / renormalise) is the warp-per-token top-k kernel.
#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

constexpr int kTM = 128;       // tokens per CTA
constexpr int kTN = 32;        // experts per CTA
constexpr int kTK = 64;        // bf16 columns of H per stage (128-byte rows)
constexpr int kTStages = 4;
constexpr int kTXBytes = kTM * kTK * 2;  // 16 KB
constexpr int kTWBytes = kTN * kTK * 2;  // 4 KB
constexpr int kTStageBytes = kTXBytes + kTWBytes;

struct RouterTail {
    uint64_t full[kTStages];
    uint64_t empty[kTStages];
    uint64_t done;
    uint32_t tmem_base;
    int abort;
};

constexpr size_t kRouterSmem = 1024 + (size_t)kTStages * kTStageBytes + sizeof(RouterTail);

__global__ void __launch_bounds__(128, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, int T, int H,
                     int E, __nv_bfloat16* __restrict__ logits, int* err) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    RouterTail* tail = reinterpret_cast<RouterTail*>(smem + (size_t)kTStages * kTStageBytes);
    volatile int* abort = &tail->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kTM, e0 = blockIdx.y * kTN;
    const int KB = H / kTK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTStages; ++s) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        mbar_init(smem_u32(&tail->done), 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        prefetch_tensormap(&tm_x);
        prefetch_tensormap(&tm_w);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;

    if (warp == 0 && lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        for (int kb = 0; kb < KB; ++kb) {
            if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, abort)) break;
            const uint32_t xd = sbase + stage * kTStageBytes;
            const uint32_t fb = smem_u32(&tail->full[stage]);
            mbar_arrive_expect_tx(fb, kTStageBytes);
            tma_load_2d(xd, &tm_x, fb, kb * kTK, t0);
            tma_load_2d(xd + kTXBytes, &tm_w, fb, kb * kTK, e0);
            if (++stage == kTStages) { stage = 0; phase ^= 1u; }
        }
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = idesc_f32acc(1 /*bf16*/, 1 /*bf16*/, kTM, kTN);
        int stage = 0;
        uint32_t phase = 0;
        for (int kb = 0; kb < KB; ++kb) {
            if (!mbar_wait(smem_u32(&tail->full[stage]), phase, abort)) break;
            tc_fence_after();
            const uint32_t xa = sbase + stage * kTStageBytes;
            const uint64_t da = desc_kmajor_sw128(xa), db = desc_kmajor_sw128(xa + kTXBytes);
#pragma unroll
            for (int j = 0; j < kTK / 16; ++j)  // 16 bf16 (32 bytes) of K per instruction
                mma_f16(tmem, da + 2 * j, db + 2 * j, idesc, (kb | j) != 0 ? 1u : 0u);
            mma_commit(smem_u32(&tail->empty[stage]));
            if (++stage == kTStages) { stage = 0; phase ^= 1u; }
        }
        mma_commit(smem_u32(&tail->done));
    }
    __syncwarp();

    // Epilogue: thread i owns token t0 + i (TMEM lane i) and writes its 32 bf16 logits.
    const bool ok = mbar_wait(smem_u32(&tail->done), 0, abort);
    tc_fence_after();
    const int t = t0 + threadIdx.x;
    if (ok) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), r);
        tmem_ld_wait();
        if (t < T) {
            if (e0 + kTN <= E) {
                uint4* dst = reinterpret_cast<uint4*>(logits + (size_t)t * E + e0);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    uint4 o;
                    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        ob[i] = __floats2bfloat162_rn(__uint_as_float(r[8 * u + 2 * i]),
                                                      __uint_as_float(r[8 * u + 2 * i + 1]));
                    dst[u] = o;
                }
            } else {
#pragma unroll
                for (int i = 0; i < kTN; ++i)
                    if (e0 + i < E) logits[(size_t)t * E + e0 + i] = __float2bfloat16_rn(__uint_as_float(r[i]));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
    if (threadIdx.x == 0 && tail->abort && err != nullptr) atomicExch(err, 1);
}

}  // namespace

cudaError_t launch_router_topk(const void* x, const void* w, const float* bias, int T, int H, int E, int k,
                               void* logits, float* topk_w, int32_t* topk_ids, int32_t* err, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    if (logits == nullptr) return cudaErrorInvalidValue;  // the ranking reads the logits back
    CUtensorMap tx, tw;
    if (!encode_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H, (uint64_t)T, (uint64_t)H * 2,
                        kTK, kTM) ||
        !encode_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H, (uint64_t)E, (uint64_t)H * 2, kTK,
                        kTN))
        return cudaErrorInvalidValue;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kRouterSmem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const dim3 grid(cdiv(T, kTM), cdiv(E, kTN));
    router_tc_kernel<<<grid, 128, kRouterSmem, s>>>(tx, tw, T, H, E, static_cast<__nv_bfloat16*>(logits), err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_topk(logits, bias, T, E, k, topk_w, topk_ids, s);
}

}  // namespace pm
