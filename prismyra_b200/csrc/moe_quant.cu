// Element-wise stages around the grouped GEMMs: the per-128-column FP8 quantisation of the token activations
// (vLLM per_token_group_quant_fp8, fp8_utils.py:137-147) and the final top-k sum (vLLM moe_sum,
// fused_moe.py:1864).
#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

// One half-warp per (token, 128-column group), two groups per warp: each lane converts 8 columns, the group's amax
// is a half-warp reduction, and every copy of the group is one coalesced 128-byte segment (so small token counts
// still spread over the whole GPU).  s = e4m3_group_scale(amax, scale_rule) (ptx.cuh: by default the correctly
// rounded max(amax, 1e-10) / 448 of vLLM's compiled quantiser); q = e4m3(clamp(x / s, -448, 448)) with an IEEE
// division.  With slot_of the row is written to the
// token's k slots (its expert-ordered copies for the gate_up GEMM; vLLM reads the same rows through
// sorted_ids // top_k); the padding slots are left unwritten -- their GEMM rows are computed and discarded, never
// stored.  Without slot_of the single copy goes to row t.
__global__ void __launch_bounds__(256) quant_fp8_kernel(const __nv_bfloat16* __restrict__ x, int T, int H, int k,
                                                        const int32_t* __restrict__ slot_of,
                                                        uint8_t* __restrict__ x_q, float* __restrict__ x_s,
                                                        int scale_rule, int32_t* __restrict__ zero, int zero_n) {
    pdl_wait();
    pdl_trigger();
    // counters the next kernel starts from zero (its work queue and hand-off counters)
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < zero_n; i += gridDim.x * blockDim.x) zero[i] = 0;
    const int lane = threadIdx.x & 31, sub = lane & 15;
    const int G = H / 128;
    const long items = (long)T * G;
    const long pairs = (items + 1) / 2;
    const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
    const int ncopies = slot_of != nullptr ? k : 1;
    for (long wp = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wp < pairs; wp += nwarps) {
        const long item = 2 * wp + (lane >> 4);
        const bool valid = item < items;
        const long row = valid ? item / G : 0;
        const int col = valid ? (int)(item % G) * 128 + sub * 8 : 0;
        float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        float amax = 0.0f;
        if (valid) {
            const uint4 w = *reinterpret_cast<const uint4*>(x + row * H + col);
            const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[i] = __bfloat162float(b[i]);
                amax = fmaxf(amax, fabsf(v[i]));
            }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (!valid) continue;
        const float sc = e4m3_group_scale(amax, scale_rule);
        uint32_t packed[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float q0 = fminf(fmaxf(__fdiv_rn(v[4 * i + 0], sc), -448.0f), 448.0f);
            const float q1 = fminf(fmaxf(__fdiv_rn(v[4 * i + 1], sc), -448.0f), 448.0f);
            const float q2 = fminf(fmaxf(__fdiv_rn(v[4 * i + 2], sc), -448.0f), 448.0f);
            const float q3 = fminf(fmaxf(__fdiv_rn(v[4 * i + 3], sc), -448.0f), 448.0f);
            packed[i] = (uint32_t)e4m3x2(q0, q1) | ((uint32_t)e4m3x2(q2, q3) << 16);
        }
        for (int c = 0; c < ncopies; ++c) {
            const size_t dst = slot_of != nullptr ? (size_t)slot_of[row * k + c] : (size_t)row;
            *reinterpret_cast<uint2*>(x_q + dst * H + col) = make_uint2(packed[0], packed[1]);
            if (sub == 0) x_s[dst * G + col / 128] = sc;
        }
    }
}

// out[t, c..c+7] = bf16(sum_j c3[row(t*k + j), c..c+7]) with an fp32 running sum, j ascending; row() is the
// identity or the row_of map (rows returned by expert-parallel ranks arrive in their send order).  With add, the
// rounded sum is then added to add[t] and rounded again: `routed + shared` of two bf16 tensors (reference
// prismyra/kernels/qwen3_moe.py:199).
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ c3,
                                                      const int32_t* __restrict__ row_of, int T, int k, int H,
                                                      const __nv_bfloat16* __restrict__ add,
                                                      __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const long total = (long)T * (H / 8);
    for (long q = (long)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (long)gridDim.x * blockDim.x) {
        const long t = q / (H / 8);
        const int c = (int)(q % (H / 8)) * 8;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        for (int j = 0; j < k; ++j) {
            const size_t rrow = row_of != nullptr ? (size_t)row_of[(size_t)t * k + j] : (size_t)t * k + j;
            const uint4 u = *reinterpret_cast<const uint4*>(c3 + rrow * H + c);
            const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(b[i]);
        }
        uint4 o;
        __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
        for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(acc[i]);
        if (add != nullptr) {
            const uint4 u = *reinterpret_cast<const uint4*>(add + (size_t)t * H + c);
            const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
            for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(__bfloat162float(ob[i]) + __bfloat162float(b[i]));
        }
        *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = o;
    }
}

}  // namespace

cudaError_t launch_quant_fp8(const void* x, int T, int H, int k, const int32_t* slot_of, uint8_t* x_q, float* x_s,
                             cudaStream_t s, int scale_rule, int32_t* zero, int zero_n) {
    if (T == 0) return zero_n > 0 ? cudaMemsetAsync(zero, 0, sizeof(int32_t) * (size_t)zero_n, s) : cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long pairs = ((long)T * (H / 128) + 1) / 2;  // one warp per two (token, group) items
    const int blocks = (int)min((pairs + 7) / 8, (long)sms * 16);
    PM_TRY(launch_pdl(quant_fp8_kernel, dim3(blocks), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(x), T, H, k,
                      slot_of, x_q, x_s, scale_rule, zero, zero_n));
    return cudaGetLastError();
}

// dst row dst_index[i] (dst_stride bytes apart) = src row i (src_stride bytes apart), row_bytes bytes each;
// rows with a negative dst_index are skipped.
__global__ void __launch_bounds__(256) scatter_rows_kernel(const uint8_t* __restrict__ src, int rows, int row_bytes,
                                                           int src_stride, const int32_t* __restrict__ dst_index,
                                                           uint8_t* __restrict__ dst, int dst_stride) {
    const int per_row = row_bytes / 16;
    const long total = (long)rows * per_row;
    for (long q = (long)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (long)gridDim.x * blockDim.x) {
        const long r = q / per_row;
        const int c = (int)(q % per_row) * 16;
        const int d = dst_index[r];
        if (d < 0) continue;  // a row with no destination (padding received from an expert-parallel peer)
        const uint4 v = *reinterpret_cast<const uint4*>(src + r * src_stride + c);
        *reinterpret_cast<uint4*>(dst + (size_t)d * dst_stride + c) = v;
    }
}

cudaError_t launch_scatter_rows(const void* src, int rows, int row_bytes, int src_stride, const int32_t* dst_index,
                                void* dst, int dst_stride, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long total = (long)rows * (row_bytes / 16);
    const long want = (total + 255) / 256;
    const int blocks = (int)(want < (long)sms * 16 ? want : (long)sms * 16);
    scatter_rows_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(src), rows, row_bytes, src_stride,
                                               dst_index, static_cast<uint8_t*>(dst), dst_stride);
    return cudaGetLastError();
}

cudaError_t launch_combine(const void* c3, const int32_t* row_of, int T, int k, int H, void* out, cudaStream_t s,
                           const void* add) {
    if (T == 0) return cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long total = (long)T * (H / 8);
    const long want = (total + 255) / 256;
    const int blocks = (int)(want < (long)sms * 16 ? want : (long)sms * 16);
    PM_TRY(launch_pdl(combine_kernel, dim3(blocks), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(c3), row_of, T,
                      k, H, static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out)));
    return cudaGetLastError();
}

}  // namespace pm
