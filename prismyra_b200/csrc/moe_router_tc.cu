// Router projection on the tensor cores, fused with softmax / top-k / renormalise.
//
// logits[t, e] = bf16(sum_h x[t, h] * W[e, h]) (prismyra/kernels/qwen3_moe.py:169-171, the batch-invariant
// router: bf16 operands, fp32 accumulation, bf16 result), then vLLM fused_topk(renormalize=True) semantics
// (router/fused_topk_router.py:69-113): p = softmax(logits) in fp32, the k largest (equal values: lower expert
// index first), weights = p / sum of the selected p.
//
// One CTA = 128 tokens x all experts: tcgen05 kind::f16 MMAs (M=128, N=E rounded up to 16, K=16 per instruction)
// accumulate the whole H reduction in TMEM, fed by a 4-stage TMA pipeline of 64-column slices.  Every token's
// logits are reduced in the same fixed order whatever the token count, so a row's result never depends on which
// rows share the call.  The epilogue (4 warps, one token per thread) stages the bf16 logits in shared memory and
// ranks each token sequentially.
#include <math.h>

#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

constexpr int kTM = 128;       // tokens per CTA
constexpr int kTK = 64;        // bf16 columns of H per stage (128-byte rows)
constexpr int kTStages = 4;
constexpr int kTXBytes = kTM * kTK * 2;  // 16 KB

struct RouterTail {
    uint64_t full[kTStages];
    uint64_t empty[kTStages];
    uint64_t done;
    uint32_t tmem_base;
    int abort;
};

__host__ __device__ constexpr size_t router_smem(int N) {
    return 1024 + (size_t)kTStages * (kTXBytes + (size_t)N * 128) + sizeof(RouterTail);
}

__global__ void __launch_bounds__(128, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, int T, int H,
                     int E, int N, uint32_t tmem_cols, int k, __nv_bfloat16* __restrict__ logits,
                     float* __restrict__ topk_w, int32_t* __restrict__ topk_ids, int* err) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const int stage_bytes = kTXBytes + N * 128;
    RouterTail* tail = reinterpret_cast<RouterTail*>(smem + (size_t)kTStages * stage_bytes);
    volatile int* abort = &tail->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kTM;
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
        tmem_alloc(smem_u32(&tail->tmem_base), tmem_cols);
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
            const uint32_t xd = sbase + stage * stage_bytes;
            const uint32_t fb = smem_u32(&tail->full[stage]);
            mbar_arrive_expect_tx(fb, stage_bytes);
            tma_load_2d(xd, &tm_x, fb, kb * kTK, t0);
            tma_load_2d(xd + kTXBytes, &tm_w, fb, kb * kTK, 0);
            if (++stage == kTStages) { stage = 0; phase ^= 1u; }
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = idesc_f32acc(1 /*bf16*/, 1 /*bf16*/, kTM, (uint32_t)N);
        int stage = 0;
        uint32_t phase = 0;
        for (int kb = 0; kb < KB; ++kb) {
            if (!mbar_wait(smem_u32(&tail->full[stage]), phase, abort)) break;
            tc_fence_after();
            const uint32_t xa = sbase + stage * stage_bytes;
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

    // Epilogue: every thread owns token t0 + threadIdx.x (TMEM lane threadIdx.x).
    const bool ok = mbar_wait(smem_u32(&tail->done), 0, abort);
    tc_fence_after();
    float* lg = reinterpret_cast<float*>(smem);  // [128][E + 1] floats, reusing the drained pipeline buffers
    const int LS = E + 1;
    const int row = threadIdx.x;
    const int t = t0 + row;
    if (ok) {
        for (int c0 = 0; c0 < N; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int e = c0 + i;
                if (e < E) {
                    const __nv_bfloat16 b = __float2bfloat16_rn(__uint_as_float(r[i]));
                    lg[row * LS + e] = __bfloat162float(b);
                    if (logits != nullptr && t < T) logits[(size_t)t * E + e] = b;
                }
            }
        }
        if (t < T) {
            float* v = lg + row * LS;
            float mx = -INFINITY;
            for (int e = 0; e < E; ++e) mx = fmaxf(mx, v[e]);
            float sum = 0.0f;
            for (int e = 0; e < E; ++e) sum += expf(v[e] - mx);
            float sel = 0.0f;
            float pj[kMaxTopK];
            int ij[kMaxTopK];
            for (int j = 0; j < k; ++j) {
                // the largest untaken logit; a strict '>' keeps the lower index among equal values.  Taken
                // entries are marked NaN, which no comparison selects.
                int best = -1;
                float bv = 0.0f;
                for (int e = 0; e < E; ++e) {
                    const float x = v[e];
                    if (isnan(x)) continue;
                    if (best < 0 || x > bv) {
                        bv = x;
                        best = e;
                    }
                }
                if (best < 0) best = 0;  // fewer than k finite logits (non-finite input): keep the output defined
                const float p = expf(bv - mx) / sum;
                pj[j] = p;
                ij[j] = best;
                sel += p;
                v[best] = __int_as_float(0x7fc00000);
            }
            for (int j = 0; j < k; ++j) {
                topk_w[(size_t)t * k + j] = pj[j] / sel;
                topk_ids[(size_t)t * k + j] = ij[j];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
    if (threadIdx.x == 0 && tail->abort && err != nullptr) atomicExch(err, 1);
}

}  // namespace

cudaError_t launch_router_topk(const void* x, const void* w, int T, int H, int E, int k, void* logits, float* topk_w,
                               int32_t* topk_ids, int32_t* err, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    const int N = (E + 15) / 16 * 16;
    uint32_t cols = 32;
    while (cols < (uint32_t)N) cols <<= 1;
    CUtensorMap tx, tw;
    if (!encode_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H, (uint64_t)T, (uint64_t)H * 2,
                        kTK, kTM) ||
        !encode_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H, (uint64_t)E, (uint64_t)H * 2, kTK,
                        (uint32_t)N))
        return cudaErrorInvalidValue;
    const size_t smem = router_smem(N);
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)router_smem(kMaxExperts));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    router_tc_kernel<<<cdiv(T, kTM), 128, smem, s>>>(tx, tw, T, H, E, N, cols, k,
                                                    static_cast<__nv_bfloat16*>(logits), topk_w, topk_ids, err);
    return cudaGetLastError();
}

}  // namespace pm
