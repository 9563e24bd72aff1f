// NVFP4 routed experts on sm_100a: e2m1 operands with one e4m3 scale per 16 elements and one fp32 global scale
// per tensor, applied by the tensor core (tcgen05.mma kind::mxf4nvf4.block_scale, 16-element scale blocks).
//
// Reference path: prismyra/kernels/nvfp4.py:247-312 (FusedExpertsFp4.routed -> FlashInfer cutlass_fused_moe):
//   activations x are quantised with the per-layer scale a1 = 448*6/(1.25*w13_in_amax) (nvfp4.py:125), the
//   gate_up product is multiplied by alpha1[e] = 1/(g1[e]*a1) (nvfp4.py:141), silu(gate)*up is re-quantised with
//   a2 (nvfp4.py:126), the down product is multiplied by alpha2[e] = 1/(g2[e]*a2) and by the routing weight, and
//   the k rows of each token are summed.  Activation quantisation follows vLLM's NVFP4 emulation
//   (quantization/utils/nvfp4_emulation_utils.py:172-216): sf = e4m3(gs * amax/6), x * (gs/sf) rounded to
//   e2m1 (nearest even).  The intermediate is bf16 as in the FP8 path.
//
// Scale-factor layout ("blocked", the one the tensor core reads): a matrix of R rows and K/16 scales per row is
// stored as [R/128][K/64][512 bytes]; inside a 512-byte block, row r (0..127) keeps its four scales (16-element
// groups 4c..4c+3 of the 64-column chunk c) as one 32-bit word at byte (r % 32) * 16 + (r / 32) * 4.
// tcgen05.cp.32x128b.warpx4 moves one block into 4 TMEM columns (replicated over the 4 lane quarters).
#include <cuda_fp4.h>

#include <atomic>

#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

__device__ __forceinline__ uint32_t sf_word_offset(int r_in_block) {
    return (uint32_t)((r_in_block & 31) * 16 + (r_in_block >> 5) * 4);
}

// 16 values -> 8 packed e2m1 bytes (low nibble = even column) and the group's e4m3 scale byte.
// sf = e4m3(clamp(gs * (amax * (1/6)), +-448)); code = e2m1_rne(clamp(v * (gs / sf), +-6)).
__device__ __forceinline__ uint8_t nvfp4_group(const float* v, float gs, uint32_t* packed2) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    float sc = gs * (amax * (1.0f / 6.0f));
    sc = fminf(fmaxf(sc, -448.0f), 448.0f);
    const __nv_fp8_storage_t sfb = __nv_cvt_float_to_fp8(sc, __NV_SATFINITE, __NV_E4M3);
    const float sfv = __half2float(__nv_cvt_fp8_to_halfraw(sfb, __NV_E4M3));
    const float osc = sfv == 0.0f ? 0.0f : __fdiv_rn(gs, sfv);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = fminf(fmaxf(v[2 * i] * osc, -6.0f), 6.0f);
        const float b = fminf(fmaxf(v[2 * i + 1] * osc, -6.0f), 6.0f);
        const uint32_t byte = (uint32_t)__nv_cvt_float2_to_fp4x2(make_float2(a, b), __NV_E2M1, cudaRoundNearest);
        if (i < 4) w0 |= byte << (8 * i);
        else w1 |= byte << (8 * (i - 4));
    }
    packed2[0] = w0;
    packed2[1] = w1;
    return (uint8_t)sfb;
}

// One warp per token: lane L holds 64 consecutive columns per iteration (four 16-groups -> 32 code bytes and one
// scale word).  The quantised row is written to each of the token's k slots (or to row t when slot_of is null).
__global__ void __launch_bounds__(256) quant_nvfp4_kernel(const __nv_bfloat16* __restrict__ x, int T, int H, int k,
                                                          const int32_t* __restrict__ slot_of, float gs,
                                                          uint8_t* __restrict__ a_q, uint8_t* __restrict__ a_sf) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int chunks = H / 64;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < T; row += warps) {
        const __nv_bfloat16* src = x + (size_t)row * H;
        const int ncopies = slot_of != nullptr ? k : 1;
        for (int c0 = 0; c0 < H; c0 += 32 * 64) {
            const int col = c0 + lane * 64;
            if (col >= H) continue;
            float v[64];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint4 w = *reinterpret_cast<const uint4*>(src + col + u * 8);
                const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[u * 8 + i] = __bfloat162float(b[i]);
            }
            uint32_t codes[8];
            uint32_t sfw = 0;
#pragma unroll
            for (int g = 0; g < 4; ++g) sfw |= (uint32_t)nvfp4_group(v + 16 * g, gs, codes + 2 * g) << (8 * g);
            for (int c = 0; c < ncopies; ++c) {
                const int dst = slot_of != nullptr ? slot_of[(size_t)row * k + c] : row;
                uint4* dq = reinterpret_cast<uint4*>(a_q + (size_t)dst * (H / 2) + col / 2);
                dq[0] = make_uint4(codes[0], codes[1], codes[2], codes[3]);
                dq[1] = make_uint4(codes[4], codes[5], codes[6], codes[7]);
                *reinterpret_cast<uint32_t*>(a_sf + ((size_t)(dst >> 7) * chunks + col / 64) * 512 +
                                             sf_word_offset(dst & 127)) = sfw;
            }
        }
    }
}

// ------------------------------------------------------------------------------------------- grouped GEMM
constexpr int kBM = 128, kBN = 256, kBKe = 256;  // K elements per stage (128 packed bytes per row)
constexpr int kA = kBM * 128, kB = kBN * 128, kSFA = 2048, kSFB = 4096;
constexpr int kStageBytes = kA + kB + kSFA + kSFB;  // 54 KB
constexpr int kThreads = 384, kEpiWarp0 = 4, kEpiWarps = 8;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAcc = 0, kTSFA = 256, kTSFB = 272;  // TMEM columns: accumulator, A scales, B scales

template <int MODE> struct NCfg {
    static constexpr int kStages = MODE == 0 ? 4 : 2;
    static constexpr int kRowBytes = 272;
    static constexpr int kStaging = MODE == 0 ? 0 : 8 * 32 * kRowBytes;
};

struct NTail {
    uint64_t full[4];
    uint64_t empty[4];
    uint64_t tfull;
    uint64_t tempty;
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

template <int MODE>
constexpr size_t nv_smem() {
    return 1024 + (size_t)NCfg<MODE>::kStages * kStageBytes + NCfg<MODE>::kStaging + sizeof(NTail);
}

// Block-scaled MMA descriptor: A/B e2m1 (MXF4 format 1), scales e4m3 (bit 23 = 0), K-major, N>>3 at [17,23),
// M>>4 at [24,29); scale-factor ids 0 (the four scales of a row fill one 32-bit TMEM word).
constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

// Descriptor of one 512-byte scale block for tcgen05.cp: no swizzle, 8-row x 16-byte core matrices stacked
// 128 bytes apart (stride byte offset 128, leading byte offset unused).
__device__ __forceinline__ uint64_t desc_sf(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(128u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}

__device__ __forceinline__ void utccp_sf(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void mma_nvfp4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                          uint32_t sfb, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], [%5], p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
                 : "memory");
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                          const NvGemmArgs args) {
    constexpr int kStages = NCfg<MODE>::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    uint8_t* staging = smem + (size_t)kStages * kStageBytes;
    NTail* tail = reinterpret_cast<NTail*>(staging + NCfg<MODE>::kStaging);
    volatile int* abort = &tail->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        mbar_init(smem_u32(&tail->tfull), 1);
        mbar_init(smem_u32(&tail->tempty), kEpiWarps);
        mbar_init(smem_u32(&tail->drain), 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        prefetch_tensormap(&tm_a);
        prefetch_tensormap(&tm_b);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    pdl_wait();
    pdl_trigger();
    const int KB = args.K / kBKe;
    const int kchunks = args.K / 64;
    const int nb_total = args.n_total / 128;
    const int num_tiles = (*args.num_post_pad / kBM) * args.n_tiles;

    if (warp < kEpiWarp0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");
        if (warp == 0 && lane == 0) {
            // ---------------------------------------------------------------- producer: TMA tiles + scale blocks
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int mb = tile / args.n_tiles, nt = tile % args.n_tiles;
                const int e = args.expert_ids[mb];
                const int rb0 = MODE == 0 ? nt : 2 * nt;
                const int rb1 = MODE == 0 ? args.inter / 128 + nt : 2 * nt + 1;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, abort)) { ok = false; break; }
                    const uint32_t st = sbase + stage * kStageBytes;
                    const uint32_t fb = smem_u32(&tail->full[stage]);
                    mbar_arrive_expect_tx(fb, kStageBytes);
                    tma_load_2d(st, &tm_a, fb, kb * 128, mb * kBM);
                    tma_load_2d(st + kA, &tm_b, fb, kb * 128, e * args.n_total + rb0 * 128);
                    tma_load_2d(st + kA + kB / 2, &tm_b, fb, kb * 128, e * args.n_total + rb1 * 128);
                    bulk_load(st + kA + kB, args.a_sf + ((size_t)mb * kchunks + kb * 4) * 512, kSFA, fb);
                    bulk_load(st + kA + kB + kSFA,
                              args.b_sf + ((size_t)(e * nb_total + rb0) * kchunks + kb * 4) * 512, 2048, fb);
                    bulk_load(st + kA + kB + kSFA + 2048,
                              args.b_sf + ((size_t)(e * nb_total + rb1) * kchunks + kb * 4) * 512, 2048, fb);
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                for (int s = 0; s < kStages; ++s) {
                    const uint64_t t0 = globaltimer();
                    while (!mbar_try_wait(smem_u32(&tail->full[s]), phase ^ (s < stage ? 0u : 1u)) &&
                           globaltimer() - t0 < PM_WAIT_TIMEOUT_NS) {
                    }
                }
            }
        } else if (warp == 1 && lane == 0) {
            // ---------------------------------------------------------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0;
            uint32_t local = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
                if (!mbar_wait(smem_u32(&tail->tempty), (local & 1u) ^ 1u, abort)) break;
                tc_fence_after();
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(smem_u32(&tail->full[stage]), phase, abort)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t st = sbase + stage * kStageBytes;
                    const uint32_t sfa = st + kA + kB, sfb = sfa + kSFA;
#pragma unroll
                    for (int c = 0; c < 4; ++c) utccp_sf(tmem + kTSFA + 4 * c, desc_sf(sfa + 512 * c));
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        utccp_sf(tmem + kTSFB + 8 * c, desc_sf(sfb + 512 * c));
                        utccp_sf(tmem + kTSFB + 8 * c + 4, desc_sf(sfb + 2048 + 512 * c));
                    }
                    const uint64_t da = desc_kmajor_sw128(st), db = desc_kmajor_sw128(st + kA);
#pragma unroll
                    for (int c = 0; c < 4; ++c)  // 64 e2m1 (32 bytes) of K per instruction
                        mma_nvfp4(tmem + kAcc, da + 2 * c, db + 2 * c, kIdesc, tmem + kTSFA + 4 * c,
                                  tmem + kTSFB + 8 * c, (kb | c) != 0 ? 1u : 0u);
                    mma_commit(smem_u32(&tail->empty[stage]));
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
                if (ok) mma_commit(smem_u32(&tail->tfull));
            }
            mma_commit(smem_u32(&tail->drain));
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(smem_u32(&tail->drain), 0) && globaltimer() - t0 < PM_WAIT_TIMEOUT_NS) {
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 224;" ::: "memory");
        // -------------------------------------------------------------------- epilogue
        const int q = warp & 3, half = (warp - kEpiWarp0) >> 2, row = q * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
        uint32_t local = 0;
        float acc[128];
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
            const int mb = tile / args.n_tiles, nt = tile % args.n_tiles;
            const int e = args.expert_ids[mb];
            const int grow = mb * kBM + row;
            const float alpha = args.alpha[e];
            if (!mbar_wait(smem_u32(&tail->tfull), local & 1u, abort)) break;
            tc_fence_after();
            {
                uint32_t r[32];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t col = MODE == 0 ? (c < 2 ? 64 * half + 32 * c : 128 + 64 * half + 32 * (c - 2))
                                                   : 128 * half + 32 * c;
                    tmem_ld32(t_lane + kAcc + col, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc[32 * c + i] = __uint_as_float(r[i]) * alpha;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tail->tempty));  // the accumulator may be overwritten now

            if (MODE == 0) {
                // bf16(alpha*gate), bf16(alpha*up) -> silu(gate)*up in bf16 -> NVFP4 with the layer's a2 scale.
                float y[64];
#pragma unroll
                for (int c = 0; c < 64; c += 2) {
                    const float2 g = bf16x2_round(acc[c], acc[c + 1]);
                    const float2 u = bf16x2_round(acc[64 + c], acc[64 + c + 1]);
                    const float2 s2 = silu2(g);
                    const float2 sg = bf16x2_round(s2.x, s2.y);
                    const float2 p2 = __fmul2_rn(sg, u);
                    const float2 yy = bf16x2_round(p2.x, p2.y);
                    y[c] = yy.x;
                    y[c + 1] = yy.y;
                }
                uint32_t codes[8];
                uint32_t sfw = 0;
#pragma unroll
                for (int g = 0; g < 4; ++g)
                    sfw |= (uint32_t)nvfp4_group(y + 16 * g, args.gs_out, codes + 2 * g) << (8 * g);
                const int col = nt * 128 + 64 * half;  // first intermediate column of this thread
                uint4* dq = reinterpret_cast<uint4*>(args.out_q + (size_t)grow * (args.inter / 2) + col / 2);
                dq[0] = make_uint4(codes[0], codes[1], codes[2], codes[3]);
                dq[1] = make_uint4(codes[4], codes[5], codes[6], codes[7]);
                *reinterpret_cast<uint32_t*>(args.out_sf + ((size_t)mb * (args.inter / 64) + col / 64) * 512 +
                                             sf_word_offset(row)) = sfw;
            } else {
                const int flat = args.sorted_ids[grow];
                const float w = flat < args.n_valid ? args.topk_w[flat] : 0.0f;
                constexpr int RB = NCfg<MODE>::kRowBytes;
                uint8_t* wst = staging + (size_t)(warp - kEpiWarp0) * 32 * RB;
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    uint4 o;
                    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        ob[i] = __floats2bfloat162_rn(acc[8 * u + 2 * i] * w, acc[8 * u + 2 * i + 1] * w);
                    *reinterpret_cast<uint4*>(wst + lane * RB + u * 16) = o;
                }
                __syncwarp();
                const int H = args.n_total;
                const int sub = lane >> 4, chunk = lane & 15;
                for (int r = 0; r < 32; r += 2) {
                    const int f = __shfl_sync(0xffffffffu, flat, r + sub);
                    if (f < args.n_valid) {
                        const uint4 v = *reinterpret_cast<const uint4*>(wst + (r + sub) * RB + chunk * 16);
                        *reinterpret_cast<uint4*>(args.c3 + (size_t)f * H + nt * kBN + 128 * half + chunk * 8) = v;
                    }
                }
                __syncwarp();
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && tail->abort && args.err != nullptr) atomicExch(args.err, 1);
}

}  // namespace

cudaError_t launch_quant_nvfp4(const void* x, int T, int H, int k, const int32_t* slot_of, float gs, uint8_t* a_q,
                               uint8_t* a_sf, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int blocks = min(cdiv(T, 8), sms * 8);
    PM_TRY(launch_pdl(quant_nvfp4_kernel, dim3(blocks), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(x), T, H,
                      k, slot_of, gs, a_q, a_sf));
    return cudaGetLastError();
}

cudaError_t launch_gemm_nvfp4(int mode, const CUtensorMap& tm_a, const CUtensorMap& tm_b, const NvGemmArgs& args,
                              int num_sms, cudaStream_t s) {
    static std::atomic<bool> configured[64][2];  // zero-initialised: false
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev][mode].load(std::memory_order_acquire)) {
        cudaError_t e = mode == 0 ? cudaFuncSetAttribute(moe_gemm_nvfp4_kernel<0>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                         (int)nv_smem<0>())
                                  : cudaFuncSetAttribute(moe_gemm_nvfp4_kernel<1>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                         (int)nv_smem<1>());
        if (e != cudaSuccess) return e;
        configured[dev][mode].store(true, std::memory_order_release);
    }
    const int grid = args.max_tiles < num_sms ? (args.max_tiles > 0 ? args.max_tiles : 1) : num_sms;
    if (mode == 0)
        PM_TRY(launch_pdl(moe_gemm_nvfp4_kernel<0>, dim3(grid), dim3(kThreads), nv_smem<0>(), s, tm_a, tm_b, args));
    else
        PM_TRY(launch_pdl(moe_gemm_nvfp4_kernel<1>, dim3(grid), dim3(kThreads), nv_smem<1>(), s, tm_a, tm_b, args));
    return cudaGetLastError();
}

}  // namespace pm
