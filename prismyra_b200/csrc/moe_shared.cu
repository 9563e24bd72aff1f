// The shared expert's gate, the reference's `torch.sigmoid(self._gate(x))` (prismyra/kernels/qwen3_moe.py:172-183,
// 198): a bf16 projection of each token onto the one-row gate weight, then a sigmoid of that bf16 value, rounded
// to bf16 again.  One warp per token: lane l accumulates the 8-column chunks l, l+32, ... in ascending order in
// fp32, then a fixed xor-shuffle tree adds the 32 lane sums, so a token's gate never depends on the other rows.
// The same launch writes the one-expert plan the shared expert's grouped GEMMs run on (every 128-row block
// belongs to expert 0).  A dense block-FP8 projection (the reference's Fp8Linear) runs on the same plan with unit
// row weights (dense_plan_kernel).
#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

__global__ void __launch_bounds__(256) shared_gate_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w_sg, int T, int H,
                                                          float* __restrict__ gate, int32_t* __restrict__ expert_ids,
                                                          int32_t* __restrict__ num_post_pad) {
    pdl_wait();
    pdl_trigger();
    const long gtid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int blocks = (T + kBlockM - 1) / kBlockM;
    for (long b = gtid; b < blocks; b += (long)gridDim.x * blockDim.x) expert_ids[b] = 0;
    if (gtid == 0) *num_post_pad = blocks * kBlockM;

    const int lane = threadIdx.x & 31;
    const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
    for (long t = gtid >> 5; t < T; t += nwarps) {
        float acc = 0.0f;
        for (int c = lane * 8; c < H; c += 256) {
            const uint4 xv = *reinterpret_cast<const uint4*>(x + t * H + c);
            const uint4 wv = *reinterpret_cast<const uint4*>(w_sg + c);
            const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
            const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = fmaf(__bfloat162float(xb[i]), __bfloat162float(wb[i]), acc);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            const float logit = __bfloat162float(__float2bfloat16_rn(acc));
            const float sig = __fdiv_rn(1.0f, 1.0f + expf(-logit));
            gate[t] = __bfloat162float(__float2bfloat16_rn(sig));
        }
    }
}

// The one-expert plan of a dense projection run on the grouped GEMMs: expert_ids[b] = 0 for the ceil(T/128)
// blocks, *num_post_pad = their slots, and a row weight of exactly 1 for every token (bf16(acc * 1) = bf16(acc)).
__global__ void __launch_bounds__(256) dense_plan_kernel(int T, float* __restrict__ ones,
                                                         int32_t* __restrict__ expert_ids,
                                                         int32_t* __restrict__ num_post_pad) {
    pdl_wait();
    pdl_trigger();
    const long gtid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const long stride = (long)gridDim.x * blockDim.x;
    const int blocks = (T + kBlockM - 1) / kBlockM;
    for (long b = gtid; b < blocks; b += stride) expert_ids[b] = 0;
    for (long t = gtid; t < T; t += stride) ones[t] = 1.0f;
    if (gtid == 0) *num_post_pad = blocks * kBlockM;
}

}  // namespace

cudaError_t launch_dense_plan(int T, float* ones, int32_t* expert_ids, int32_t* num_post_pad, int sms,
                              cudaStream_t s) {
    const int blocks = (int)std::min<long>(((long)T + 255) / 256 + 1, (long)sms * 4);
    PM_TRY(launch_pdl(dense_plan_kernel, dim3(blocks), dim3(256), 0, s, T, ones, expert_ids, num_post_pad));
    return cudaGetLastError();
}

cudaError_t launch_shared_gate(const void* x, const void* w_sg, int T, int H, float* gate, int32_t* expert_ids,
                               int32_t* num_post_pad, int sms, cudaStream_t s) {
    const long warps = T > 0 ? T : 1;
    const int blocks = (int)std::min<long>((warps + 7) / 8, (long)sms * 16);
    PM_TRY(launch_pdl(shared_gate_kernel, dim3(blocks), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(x),
                      static_cast<const __nv_bfloat16*>(w_sg), T, H, gate, expert_ids, num_post_pad));
    return cudaGetLastError();
}

}  // namespace pm
