// Device-side FP8 quantisation of token rows shared by the quantisation kernel (moe_quant.cu) and the fused
// few-token front end (moe_route.cu).
#pragma once

#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {

// One (token, 128-column group) item per half-warp, quantised in registers: each lane converts 8 columns, the
// group's amax is a half-warp reduction, s = e4m3_group_scale(amax, scale_rule) and q = e4m3(clamp(x / s, -448,
// 448)) with an IEEE division.
struct QuantItem {
    long row;       // token
    int col;        // this lane's first column
    uint4 raw;      // this lane's 8 bf16 inputs
    float sc;       // the group's scale
    uint32_t q[2];  // this lane's 8 e4m3 values
    bool valid;
};

// This half-warp's item of the (token, group) sequence (valid below items): its inputs only (quant_fp8_finish
// converts them).
__device__ __forceinline__ QuantItem quant_fp8_load(const __nv_bfloat16* __restrict__ x, int H, long item,
                                                    long items) {
    const int sub = threadIdx.x & 15;
    const int G = H / 128;
    QuantItem it;
    it.valid = item < items;
    it.row = it.valid ? item / G : 0;
    it.col = it.valid ? (int)(item % G) * 128 + sub * 8 : 0;
    it.raw = it.valid ? *reinterpret_cast<const uint4*>(x + it.row * H + it.col) : make_uint4(0u, 0u, 0u, 0u);
    return it;
}

// Every lane of the warp calls this (the reduction shuffles take all 32).
__device__ __forceinline__ void quant_fp8_finish(QuantItem& it, int scale_rule) {
    float v[8];
    float amax = 0.0f;
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&it.raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[i] = __bfloat162float(b[i]);
        amax = fmaxf(amax, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    it.sc = e4m3_group_scale(amax, scale_rule);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float q0 = fminf(fmaxf(__fdiv_rn(v[4 * i + 0], it.sc), -448.0f), 448.0f);
        const float q1 = fminf(fmaxf(__fdiv_rn(v[4 * i + 1], it.sc), -448.0f), 448.0f);
        const float q2 = fminf(fmaxf(__fdiv_rn(v[4 * i + 2], it.sc), -448.0f), 448.0f);
        const float q3 = fminf(fmaxf(__fdiv_rn(v[4 * i + 3], it.sc), -448.0f), 448.0f);
        it.q[i] = (uint32_t)e4m3x2(q0, q1) | ((uint32_t)e4m3x2(q2, q3) << 16);
    }
}

// Warp pair index wp: items 2 wp and 2 wp + 1 of the T * (H / 128) items, one per half-warp, loaded and converted.
__device__ __forceinline__ QuantItem quant_fp8_item(const __nv_bfloat16* __restrict__ x, int T, int H,
                                                   int scale_rule, long wp) {
    QuantItem it = quant_fp8_load(x, H, 2 * wp + ((threadIdx.x & 31) >> 4), (long)T * (H / 128));
    quant_fp8_finish(it, scale_rule);
    return it;
}

// This lane's part of a valid item into row dst of x_q [rows, H] / x_s [rows, H / 128].
__device__ __forceinline__ void store_quant_item(const QuantItem& it, int H, size_t dst, uint8_t* __restrict__ x_q,
                                                 float* __restrict__ x_s) {
    *reinterpret_cast<uint2*>(x_q + dst * H + it.col) = make_uint2(it.q[0], it.q[1]);
    if ((threadIdx.x & 15) == 0) x_s[dst * (H / 128) + it.col / 128] = it.sc;
}

}  // namespace pm
