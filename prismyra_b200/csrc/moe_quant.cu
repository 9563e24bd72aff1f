// Element-wise stages around the grouped GEMMs: the per-128-column FP8 quantisation of the token activations
// (vLLM per_token_group_quant_fp8, fp8_utils.py:137-147) and the final top-k sum (vLLM moe_sum,
// fused_moe.py:1864).
#include "moe_internal.h"
#include "ptx.cuh"
#include "quant_dev.cuh"

namespace pm {
namespace {

// Two (token, 128-column group) items per warp (quant_fp8_item, quant_dev.cuh): every copy of a group is one
// coalesced 128-byte segment, so small token counts still spread over the whole GPU.  s = e4m3_group_scale(amax,
// scale_rule) (ptx.cuh: by default the correctly rounded max(amax, 1e-10) / 448 of vLLM's compiled quantiser).
// With slot_of the row is written to the token's k slots (its expert-ordered copies for the gate_up GEMM; vLLM reads
// the same rows through sorted_ids // top_k); the padding slots are left unwritten -- their GEMM rows are computed
// and discarded, never stored.  Without slot_of the single copy goes to row t.
__global__ void __launch_bounds__(256) quant_fp8_kernel(const __nv_bfloat16* __restrict__ x, int T, int H, int k,
                                                        const int32_t* __restrict__ slot_of,
                                                        uint8_t* __restrict__ x_q, float* __restrict__ x_s,
                                                        int scale_rule, int32_t* __restrict__ zero, int zero_n) {
    pdl_wait();
    pdl_trigger();
    // counters the next kernel starts from zero (its work queue and hand-off counters)
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < zero_n; i += gridDim.x * blockDim.x) zero[i] = 0;
    const long pairs = ((long)T * (H / 128) + 1) / 2;
    const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
    for (long wp = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wp < pairs; wp += nwarps) {
        const QuantItem it = quant_fp8_item(x, T, H, scale_rule, wp);
        if (!it.valid) continue;
        if (slot_of == nullptr) {
            store_quant_item(it, H, (size_t)it.row, x_q, x_s);
        } else {
            for (int c = 0; c < k; ++c) store_quant_item(it, H, (size_t)slot_of[it.row * k + c], x_q, x_s);
        }
    }
}

// out[t, c..c+7] = bf16(sum_j c3[row(t*k + j), c..c+7]) with an fp32 running sum, j ascending; row() is the
// identity or the row_of map (rows returned by expert-parallel ranks arrive in their send order).  With add, the
// rounded sum is then added to add[t] and rounded again: `routed + shared` of two bf16 tensors (reference
// prismyra/kernels/qwen3_moe.py:199).
// KT: the top-k as a compile-time constant (all k rows' loads issued before the sum), or 0 for any k.
template <int KT>
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ c3,
                                                      const int32_t* __restrict__ row_of, int T, int k_rt, int H,
                                                      const __nv_bfloat16* __restrict__ add,
                                                      __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int k = KT > 0 ? KT : k_rt;
    const long total = (long)T * (H / 8);
    for (long q = (long)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (long)gridDim.x * blockDim.x) {
        const long t = q / (H / 8);
        const int c = (int)(q % (H / 8)) * 8;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        auto row = [&](int j) {
            return row_of != nullptr ? (size_t)row_of[(size_t)t * k + j] : (size_t)t * k + j;
        };
        if (KT > 0) {
            uint4 u[KT > 0 ? KT : 1];
#pragma unroll
            for (int j = 0; j < KT; ++j) u[j] = *reinterpret_cast<const uint4*>(c3 + row(j) * H + c);
#pragma unroll
            for (int j = 0; j < KT; ++j) {
                const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u[j]);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(b[i]);
            }
        } else {
            for (int j = 0; j < k; ++j) {
                const uint4 u = *reinterpret_cast<const uint4*>(c3 + row(j) * H + c);
                const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(b[i]);
            }
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
    if (k == 8)
        PM_TRY(launch_pdl(combine_kernel<8>, dim3(blocks), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(c3),
                          row_of, T, k, H, static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out)));
    else
        PM_TRY(launch_pdl(combine_kernel<0>, dim3(blocks), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(c3),
                          row_of, T, k, H, static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out)));
    return cudaGetLastError();
}

}  // namespace pm
