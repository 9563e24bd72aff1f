// NVFP4 weight preparation on the GPU: a stack of FP8 (e4m3, 128x128 fp32 block multipliers) expert matrices ->
// packed e2m1 codes, one e4m3 scale per 16 elements and one fp32 global scale per matrix, bit for bit what the
// reference's prepare_layer computes (prismyra/kernels/nvfp4.py:315-331) with _dequant_fp8 (nvfp4.py:97-100) and
// quantize (nvfp4.py:41-51) in fp32 torch arithmetic (for finite weights):
//
//   d     = fp32(q) * s_block                                   one rounding
//   g     = reciprocal(max(amax|d|, 1e-12)) * 2688              torch evaluates `448.0 * 6.0 / t` as
//                                                               t.reciprocal() * 2688: two roundings
//   sf    = e4m3(min((amax16 / 6) * g, 448))                    amax over each 16-element group of a row
//   eff   = fp32(sf) / g
//   x     = eff > 0 ? clamp(d / eff, -6, 6) : 0
//   code  = first j minimising |(|x| - E2M1[j])|, | 8 if x < 0  (torch.argmin keeps the first minimum, so a tie
//                                                               takes the smaller magnitude; computed from d
//                                                               and per-group bounds, see e2m1_bounds)
//
// Launches: a zeroing of the per-matrix maxima, the maxima (byte-wise magnitude maxima of the e4m3 codes, then an
// unsigned max on the bit patterns of non-negative floats -- exact and order-free), the global scales, and the
// quantisation of every 16-element group (one thread per group, 16-byte loads, no division per weight) -- or, with
// the importance search, the same with each group's scale chosen among seven candidates (prep_search_kernel).
#include "moe_internal.h"
#include "ptx.cuh"

#include <cuda_fp16.h>

namespace pm {
namespace {

__device__ __forceinline__ float e4m3_to_f32(uint32_t byte) {
    const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(byte), __NV_E4M3);
    return __half2float(__half(h));
}

// The largest magnitude code of 16 e4m3 bytes: e4m3 is sign-magnitude with magnitudes ordered like their 7-bit
// codes, and fl(|q| * s) grows with |q|, so max_i |fl(q_i * s)| = fl(e4m3(max code) * s) exactly.
__device__ __forceinline__ uint32_t max_magnitude_code(uint4 q) {
    const uint32_t m = __vmaxu4(__vmaxu4(q.x & 0x7f7f7f7fu, q.y & 0x7f7f7f7fu),
                                __vmaxu4(q.z & 0x7f7f7f7fu, q.w & 0x7f7f7f7fu));
    const uint32_t h = __vmaxu4(m, m >> 16);
    return max(h & 0xffu, (h >> 8) & 0xffu);
}

// A grid-stride walk over the 16-byte vectors of a row-major [rows, C] byte matrix that keeps (row, vector within
// the row) up to date by addition: one division per thread instead of two per vector.
struct VecWalk {
    unsigned row, cv;                 // current row and 16-byte vector within it
    unsigned step_rows, step_cv;      // the grid stride, in rows and vectors
    unsigned per_row;                 // vectors per row (C / 16)

    __device__ VecWalk(unsigned start, unsigned stride, unsigned per_row_)
        : row(start / per_row_), cv(start % per_row_), step_rows(stride / per_row_), step_cv(stride % per_row_),
          per_row(per_row_) {}
    __device__ void next() {
        cv += step_cv;
        row += step_rows;
        if (cv >= per_row) {
            cv -= per_row;
            ++row;
        }
    }
};

__global__ void __launch_bounds__(256) prep_amax_kernel(const uint8_t* __restrict__ w, const float* __restrict__ s,
                                                        int R, int C, unsigned* __restrict__ amax_bits) {
    const unsigned m = blockIdx.y;
    const unsigned per_row = C / 16, cb = C / 128;
    const uint8_t* wm = w + (size_t)m * R * C;
    const float* sm = s + (size_t)m * (R / 128) * cb;
    float amax = 0.0f;
    for (VecWalk it(blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x, per_row); it.row < (unsigned)R;
         it.next()) {
        const uint4 q = *reinterpret_cast<const uint4*>(wm + (size_t)it.row * C + it.cv * 16);
        const float sb = sm[(it.row / 128) * cb + it.cv / 8];
        amax = fmaxf(amax, fabsf(__fmul_rn(e4m3_to_f32(max_magnitude_code(q)), sb)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    __shared__ float warp_max[8];
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = warp_max[0];
        for (int i = 1; i < (int)(blockDim.x >> 5); ++i) b = fmaxf(b, warp_max[i]);
        atomicMax(amax_bits + m, __float_as_uint(b));  // non-negative floats order like their bit patterns
    }
}

// In place: the maximum's bit pattern -> g = reciprocal(max(amax, 1e-12)) * 2688.
__global__ void prep_global_kernel(float* __restrict__ g, int E) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= E) return;
    const float amax = fmaxf(__uint_as_float(reinterpret_cast<unsigned*>(g)[m]), 1e-12f);
    g[m] = __fmul_rn(__frcp_rn(amax), 2688.0f);
}

// The e2m1 code needs x = fl(d / eff) only through "fl(|x|) > m_j" for the seven midpoints m_j of the e2m1 grid
// (0.25 ... 5): the count of midpoints below |x| equals the reference's first arg-min of |fl(|x| - grid[j])|, ties
// to the smaller magnitude (checked exhaustively over every fp32 value in [0, 6]).  Round-half-even keeps m_j (an
// even mantissa) for quotients up to m_j + ulp(m_j)/2 =: B_j, so fl(|d| / eff) > m_j exactly when |d| > B_j * eff.
// B_j * eff is exact in double (at most 49 significant bits), and F_j, the smallest float above it, turns the test
// into |d| >= F_j: seven float comparisons per weight and no division (checked against the IEEE quotient on 14.4
// million cases, every neighbour of every F_j included).
__device__ __forceinline__ void e2m1_bounds(float eff, float F[7]) {
    const double kB[7] = {0.25 + 0x1p-26, 0.75 + 0x1p-25, 1.25 + 0x1p-24, 1.75 + 0x1p-24,
                          2.5 + 0x1p-23,  3.5 + 0x1p-23,  5.0 + 0x1p-22};
#pragma unroll
    for (int j = 0; j < 7; ++j) {
        const double t = kB[j] * (double)eff;
        float f = __double2float_ru(t);
        if ((double)f == t) f = __int_as_float(__float_as_int(f) + 1);  // strictly above (f is finite and > 0)
        F[j] = f;
    }
}

// The count of bounds at or below |d| (the bounds ascend) by a three-step branchless binary search.
__device__ __forceinline__ uint32_t e2m1_code(float d, const float F[7], bool live) {
    const float a = fabsf(d);
    const bool b2 = a >= F[3];
    const bool b1 = a >= (b2 ? F[5] : F[1]);
    const bool b0 = a >= (b2 ? (b1 ? F[6] : F[4]) : (b1 ? F[2] : F[0]));
    return (b2 ? 4u : 0u) | (b1 ? 2u : 0u) | (b0 ? 1u : 0u) | (live && d < 0.0f ? 8u : 0u);
}

// One thread per 16-element group of the stacked [E * R, C] matrix (matrix m = row / R).
__global__ void __launch_bounds__(256) prep_quant_kernel(const uint8_t* __restrict__ w, const float* __restrict__ s,
                                                         const float* __restrict__ g, int E, int R, int C,
                                                         uint8_t* __restrict__ packed, uint8_t* __restrict__ sf) {
    const unsigned per_row = C / 16, cb = C / 128, rows = (unsigned)E * R;
    for (VecWalk it(blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x, per_row); it.row < rows;
         it.next()) {
        const size_t i = (size_t)it.row * per_row + it.cv;  // group index = 16-byte vector index
        const uint4 q = *reinterpret_cast<const uint4*>(w + i * 16);
        const float sb = s[(it.row / 128) * cb + it.cv / 8];  // R % 128 == 0: blocks never straddle matrices
        const float amax = fabsf(__fmul_rn(e4m3_to_f32(max_magnitude_code(q)), sb));
        const float gm = g[it.row / (unsigned)R];
        const float scale = fminf(__fmul_rn(__fdiv_rn(amax, 6.0f), gm), 448.0f);
        const __nv_fp8_storage_t sbyte = __nv_cvt_float_to_fp8(scale, __NV_SATFINITE, __NV_E4M3);
        const float eff = __fdiv_rn(e4m3_to_f32(sbyte), gm);
        // eff == 0 (a zero scale): every x is 0, so every code is 0 -- bounds at +inf, no sign
        const bool live = eff > 0.0f;
        float F[7];
        if (live) {
            e2m1_bounds(eff, F);
        } else {
#pragma unroll
            for (int j = 0; j < 7; ++j) F[j] = __int_as_float(0x7f800000);
        }
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
        uint32_t out[2] = {0u, 0u};
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            const __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2(
                static_cast<__nv_fp8x2_storage_t>((words[p / 2] >> (16 * (p % 2))) & 0xffffu), __NV_E4M3);
            const float2 v = __half22float2(__half2(h2));
            const uint32_t c0 = e2m1_code(__fmul_rn(v.x, sb), F, live);
            const uint32_t c1 = e2m1_code(__fmul_rn(v.y, sb), F, live);
            out[p / 4] |= (c0 | (c1 << 4)) << (8 * (p % 4));
        }
        *reinterpret_cast<uint2*>(packed + i * 8) = make_uint2(out[0], out[1]);
        sf[i] = static_cast<uint8_t>(sbyte);
    }
}

// The importance search (prismyra/kernels/nvfp4.py:57-94, quantize_search): each 16-group's scale is the first of
// the SEARCH fractions c of its plain value, sf_c = e4m3(min(((amax16 / 6) * g) * c, 448)), that minimises the
// importance-weighted squared error of the decoded group, err_c = sum_j imp_j * (back_j - d_j)^2 with
// back_j = (E2M1[code_j] * sign_j) * eff_c, every step rounded in fp32 as torch evaluates it (the fraction is an fp32
// scalar; (x)^2 is x * x; amax / 6 a true division) and the 16 products added as torch's last-dimension sum adds
// them on the CPU, where the reference's golden outputs were made: eight strided partial sums p_j + p_{j+8}, added
// in order (checked against torch on 200,000 rows).  torch on a GPU computes amax / 6 as amax * fl(1/6) and adds
// the products by halving steps, so the reference run on a GPU can choose differently where candidates nearly tie;
// this kernel follows the CPU, like the plain preparation above.  imp: [E, C] per input column, or null (every
// column weighs 1).
__device__ __constant__ float kSearchFrac[7] = {1.0f, 0.95f, 0.9f, 0.85f, 0.8f, 0.75f, 0.7f};

// The e2m1 magnitude of a 3-bit code (0, 0.5, 1, 1.5, 2, 3, 4, 6), exactly, without a table lookup.
__device__ __forceinline__ float e2m1_value(uint32_t m) {
    const float pow2 = __int_as_float((int)(((m >> 1) + 126u) << 23));  // 2^((m >> 1) - 1)
    return m < 2u ? 0.5f * (float)m : pow2 * (1.0f + 0.5f * (float)(m & 1u));
}

__device__ __forceinline__ float e4m3_scale(float amax, float gm, float frac, __nv_fp8_storage_t* byte) {
    const float scale = fminf(__fmul_rn(__fmul_rn(__fdiv_rn(amax, 6.0f), gm), frac), 448.0f);
    *byte = __nv_cvt_float_to_fp8(scale, __NV_SATFINITE, __NV_E4M3);
    return __fdiv_rn(e4m3_to_f32(*byte), gm);
}

__global__ void __launch_bounds__(256) prep_search_kernel(const uint8_t* __restrict__ w, const float* __restrict__ s,
                                                          const float* __restrict__ g,
                                                          const float* __restrict__ imp, int E, int R, int C,
                                                          uint8_t* __restrict__ packed, uint8_t* __restrict__ sf) {
    const unsigned per_row = C / 16, cb = C / 128, rows = (unsigned)E * R;
    for (VecWalk it(blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x, per_row); it.row < rows;
         it.next()) {
        const size_t i = (size_t)it.row * per_row + it.cv;
        const uint4 q = *reinterpret_cast<const uint4*>(w + i * 16);
        const float sb = s[(it.row / 128) * cb + it.cv / 8];
        const float amax = fabsf(__fmul_rn(e4m3_to_f32(max_magnitude_code(q)), sb));
        const unsigned m = it.row / (unsigned)R;
        const float gm = g[m];
        float d[16], wt[16];
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            const __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2(
                static_cast<__nv_fp8x2_storage_t>((words[p / 2] >> (16 * (p % 2))) & 0xffffu), __NV_E4M3);
            const float2 v = __half22float2(__half2(h2));
            d[2 * p] = __fmul_rn(v.x, sb);
            d[2 * p + 1] = __fmul_rn(v.y, sb);
        }
        if (imp != nullptr) {
            const float4* ip = reinterpret_cast<const float4*>(imp + (size_t)m * C + (size_t)it.cv * 16);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float4 f = ip[u];
                wt[4 * u] = f.x;
                wt[4 * u + 1] = f.y;
                wt[4 * u + 2] = f.z;
                wt[4 * u + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) wt[j] = 1.0f;
        }
        __nv_fp8_storage_t best_byte = 0;
        float best_eff = 0.0f, best_err = 0.0f;
        for (int c = 0; c < 7; ++c) {
            __nv_fp8_storage_t byte;
            const float eff = e4m3_scale(amax, gm, kSearchFrac[c], &byte);
            const bool live = eff > 0.0f;
            float F[7];
            if (live) {
                e2m1_bounds(eff, F);
            } else {
#pragma unroll
                for (int j = 0; j < 7; ++j) F[j] = __int_as_float(0x7f800000);
            }
            float e[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t code = e2m1_code(d[j], F, live);
                const float sgn = (code & 8u) ? -1.0f : 1.0f;
                const float back = __fmul_rn(__fmul_rn(e2m1_value(code & 7u), sgn), eff);
                const float diff = __fsub_rn(back, d[j]);
                e[j] = __fmul_rn(wt[j], __fmul_rn(diff, diff));
            }
            float err = __fadd_rn(e[0], e[8]);
#pragma unroll
            for (int j = 1; j < 8; ++j) err = __fadd_rn(err, __fadd_rn(e[j], e[j + 8]));
            if (c == 0 || err < best_err) {
                best_err = err;
                best_byte = byte;
                best_eff = eff;
            }
        }
        const bool live = best_eff > 0.0f;
        float F[7];
        if (live) {
            e2m1_bounds(best_eff, F);
        } else {
#pragma unroll
            for (int j = 0; j < 7; ++j) F[j] = __int_as_float(0x7f800000);
        }
        uint32_t out[2] = {0u, 0u};
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            const uint32_t c0 = e2m1_code(d[2 * p], F, live);
            const uint32_t c1 = e2m1_code(d[2 * p + 1], F, live);
            out[p / 4] |= (c0 | (c1 << 4)) << (8 * (p % 4));
        }
        *reinterpret_cast<uint2*>(packed + i * 8) = make_uint2(out[0], out[1]);
        sf[i] = static_cast<uint8_t>(best_byte);
    }
}

}  // namespace

cudaError_t launch_nvfp4_prepare(const uint8_t* w, const float* s, int E, int R, int C, uint8_t* packed,
                                 uint8_t* sf, float* g, int sms, cudaStream_t stream, bool search, const float* imp) {
    cudaError_t e = cudaMemsetAsync(g, 0, sizeof(float) * (size_t)E, stream);
    if (e != cudaSuccess) return e;
    const long groups = (long)R * C / 16;  // per matrix
    const int per_matrix = (int)std::min<long>(std::max(1, (8 * sms + E - 1) / E), (groups + 255) / 256);
    prep_amax_kernel<<<dim3(per_matrix, E), 256, 0, stream>>>(w, s, R, C, reinterpret_cast<unsigned*>(g));
    prep_global_kernel<<<(E + 255) / 256, 256, 0, stream>>>(g, E);
    const long blocks = std::min<long>((long)sms * 8, (groups * E + 255) / 256);
    if (search)
        prep_search_kernel<<<(int)blocks, 256, 0, stream>>>(w, s, g, imp, E, R, C, packed, sf);
    else
        prep_quant_kernel<<<(int)blocks, 256, 0, stream>>>(w, s, g, E, R, C, packed, sf);
    return cudaGetLastError();
}

}  // namespace pm
