// Grouped FP8 GEMM for few tokens per expert ("swap-AB"), the branch-readout regime where the layer streams
// every expert's weights for a handful of tokens.
//
// Same arithmetic and outputs as moe_gemm_fp8.cu (vLLM fused_moe_kernel, fused_moe.py:483-548: per 128-wide K
// block, acc += (A_q . B_q) * a_scale[token, kb] * b_scale[n/128, kb], software promotion in fp32), with the
// operands' roles exchanged: the MMA's 128-row operand is a block of the expert's weight rows and its N operand is
// the tokens of one half (64 slots) of a 128-slot block, N = 32 x (32-slot sub-blocks of the half holding real
// tokens; a block's real tokens come first).  With ~8 tokens per expert the MMA and the promotion shrink from 128
// padded rows to 32 columns, and the kernel is bound by streaming the weights.
//
// Unit of work: (64-slot half hp of block mb, 128 output columns nt); all first halves come before all second
// halves, and a half without real tokens is skipped (a block with more than 64 real tokens reads its weights
// twice).
//   mode 0 (gate_up): gate rows nt*128.. and up rows I + nt*128.. of expert e: two MMAs per K step into two TMEM
//          accumulators; epilogue bf16 -> silu(gate)*up -> bf16 -> e4m3 with one scale per token over the unit's
//          128 output columns (exactly one requantisation group), written to the down GEMM's A operand.
//   mode 1 (down): hidden rows nt*128.. of expert e; epilogue multiplies by the token's routing weight in fp32,
//          rounds to bf16 and writes c3[flat index, nt*128 ..].
// Warp roles (384 threads): warp 0 TMA (weight tiles, token tiles, and per unit the block's activation scales as
// one bulk copy), warp 1 TMEM + MMA, warps 4-11 promotion and epilogue: warp w reads TMEM lanes 32*(w%4).. (weight
// rows) and token columns of half (w-4)/4 of the unit.  TMEM holds a ring of K-block accumulators (4 of 128
// columns for gate_up: gate at +0, up at +64; 8 of 64 for down), so the MMA runs several K blocks ahead of the
// promotion and through a unit's epilogue.  Every wait is bounded.
#include <atomic>

#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

constexpr int kThreads = 384;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = 8;
constexpr int kMaxStages = 8;
constexpr int kMaxSlots = 8;
constexpr int kWBytes = 128 * 128;  // one 128-row x 128-byte weight tile
constexpr int kTokBytes = 64 * 128; // up to 64 token rows x 128 bytes
constexpr uint32_t kTmemCols = 512;
constexpr int kUnitCache = 512;     // units per CTA whose (expert, sub-blocks) are staged in shared memory

template <int MODE> struct SCfg {
    static constexpr int kStageBytes = (MODE == 0 ? 2 : 1) * kWBytes + kTokBytes;
    static constexpr int kSlots = MODE == 0 ? 4 : 8;         // TMEM K-block accumulators
    static constexpr uint32_t kSlotCols = MODE == 0 ? 128 : 64;
};

struct SmallTail {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tfull[kMaxSlots];
    uint64_t tempty[kMaxSlots];
    uint64_t safull[2];   // the unit's activation-scale table (by unit parity) has landed
    uint64_t saempty[2];  // the epilogue is done with it
    uint64_t xbar[2][2];  // [column half][unit parity] per-token amax exchange between the four lane quarters
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    float amax_x[2][2][4][32];  // [unit parity][column half][lane quarter][token column]
    int unit_info[kUnitCache];  // this CTA's j-th (possibly empty) unit: expert * 8 + real sub-blocks of the half
};

// Unit u of the (2 x blocks x n_tiles) sequence -> (half, block, column tile).
struct Unit {
    int hp, mb, nt;
};
__device__ __forceinline__ Unit unit_of(int u, int blocks, int n_tiles) {
    const int per = blocks * n_tiles;
    const int hp = u >= per ? 1 : 0, rem = u - hp * per;
    return Unit{hp, rem / n_tiles, rem % n_tiles};
}

// Expert * 8 + real 32-slot sub-blocks (0..2) of half hp of block mb: sub-block j holds real tokens iff its first
// slot does.
__device__ __forceinline__ int half_info(const SmallGemmArgs& a, int mb, int hp) {
    int n = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) n += a.sorted_ids[mb * 128 + hp * 64 + 32 * j] < a.n_valid ? 1 : 0;
    return a.expert_ids[mb] * 8 + n;
}

// The same, staged at kernel start for the CTA's first kUnitCache units.
__device__ __forceinline__ int unit_info(const SmallGemmArgs& a, const int* staged, int j, const Unit& un) {
    return j < kUnitCache ? staged[j] : half_info(a, un.mb, un.hp);
}

// acc[c] += D[c] * (sa[column c] * sw) for 16 columns; D from TMEM, sa from the unit's scale table.
__device__ __forceinline__ void promote16(uint32_t taddr, const float* sa, int sa_stride, float sw, float* acc) {
    uint32_t r[16];
    tmem_ld16(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = fmaf(__uint_as_float(r[i]), sa[i * sa_stride] * sw, acc[i]);
}

struct Ring {
    uint32_t it = 0;  // K blocks promoted so far (TMEM slot ring)
    int local = 0;    // units done so far
};

// Promotion over one unit's K blocks and its epilogue, for NSUB real token sub-blocks in the half (this thread:
// 16*NSUB token columns starting at half * 16*NSUB).  Returns false when a wait gave up.
template <int MODE, int NSUB>
__device__ __forceinline__ bool run_unit(const SmallGemmArgs& a, SmallTail* tail, const float* sa_tab, const Unit& un,
                                         int e, Ring& ring, volatile int* abort, uint32_t tmem_base) {
    constexpr int C = 16 * NSUB;  // token columns of this thread
    constexpr int kSlots = SCfg<MODE>::kSlots;
    constexpr uint32_t kSlotCols = SCfg<MODE>::kSlotCols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = warp & 3, half = (warp - kEpiWarp0) >> 2;
    const int r = q * 32 + lane;  // weight row of the unit (output column nt*128 + r)
    const int KB = a.K / 128;
    const int nb_total = a.n_total / 128;
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    const int col0 = half * C;                  // first token column of this thread within the unit
    const int row0 = un.hp * 64 + col0;         // ... as a slot of block mb
    const uint32_t par = (uint32_t)ring.local & 1u, use = (uint32_t)ring.local >> 1;

    // weight block scales of the unit, lane-distributed (lane l holds K blocks l and l + 32)
    const float* bsg = a.b_scale + ((size_t)e * nb_total + un.nt) * KB;
    const float* bsu = a.b_scale + ((size_t)e * nb_total + (MODE == 0 ? a.inter / 128 : 0) + un.nt) * KB;
    const float g0 = lane < KB ? bsg[lane] : 0.0f, g1 = lane + 32 < KB ? bsg[lane + 32] : 0.0f;
    const float u0 = (MODE == 0 && lane < KB) ? bsu[lane] : 0.0f;
    const float u1 = (MODE == 0 && lane + 32 < KB) ? bsu[lane + 32] : 0.0f;
    // down: flat index and routing weight of each token column (lane l: column col0 + l)
    int fl = 0;
    float wl = 0.0f;
    if (MODE == 1) {
        fl = lane < C ? a.sorted_ids[un.mb * 128 + row0 + lane] : a.n_valid;
        wl = fl < a.n_valid ? a.topk_w[fl] : 0.0f;
    }

    float accg[C], accu[MODE == 0 ? C : 1];
#pragma unroll
    for (int i = 0; i < C; ++i) accg[i] = 0.0f;
#pragma unroll
    for (int i = 0; i < (MODE == 0 ? C : 1); ++i) accu[i] = 0.0f;

    if (!mbar_wait(smem_u32(&tail->safull[par]), use & 1u, abort)) return false;
    const float* sa = sa_tab + (size_t)par * 128 * KB + (size_t)row0 * KB;
    for (int kb = 0; kb < KB; ++kb, ++ring.it) {
        const uint32_t slot = ring.it % kSlots, su = ring.it / kSlots;
        const float swg = __shfl_sync(0xffffffffu, kb < 32 ? g0 : g1, kb & 31);
        const float swu = MODE == 0 ? __shfl_sync(0xffffffffu, kb < 32 ? u0 : u1, kb & 31) : 0.0f;
        if (!mbar_wait(smem_u32(&tail->tfull[slot]), su & 1u, abort)) return false;
        tc_fence_after();
        const uint32_t tb = t_lane + slot * kSlotCols + (uint32_t)col0;
#pragma unroll
        for (int c = 0; c < NSUB; ++c) {
            promote16(tb + 16 * c, sa + (size_t)(16 * c) * KB + kb, KB, swg, accg + 16 * c);
            if (MODE == 0) promote16(tb + 64 + 16 * c, sa + (size_t)(16 * c) * KB + kb, KB, swu, accu + 16 * c);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tail->tempty[slot]));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&tail->saempty[par]));

    if (MODE == 0) {
        // y = bf16(bf16(silu(bf16(gate))) * bf16(up)) per (row, token); per token the amax over the 128 rows: a
        // warp reduction, then the four lane quarters through shared memory (bounded mbarrier wait)
#pragma unroll
        for (int i = 0; i < C; i += 2) {
            const float2 g = bf16x2_round(accg[i], accg[i + 1]);
            const float2 u = bf16x2_round(accu[i], accu[i + 1]);
            const float2 s2 = silu2(g);
            const float2 sg = bf16x2_round(s2.x, s2.y);
            const float2 p2 = __fmul2_rn(sg, u);
            const float2 y = bf16x2_round(p2.x, p2.y);
            accg[i] = y.x;
            accg[i + 1] = y.y;
        }
        float(*ax)[32] = tail->amax_x[par][half];
#pragma unroll
        for (int i = 0; i < C; ++i) {
            float m = fabsf(accg[i]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) ax[q][i] = m;
        }
        const uint32_t xb = smem_u32(&tail->xbar[half][par]);
        mbar_arrive(xb);
        if (!mbar_wait(xb, use & 1u, abort)) return false;
        const int I = a.inter;
#pragma unroll
        for (int i = 0; i < C; ++i) {
            const float amax = fmaxf(fmaxf(ax[0][i], ax[1][i]), fmaxf(ax[2][i], ax[3][i]));
            const float sc = e4m3_group_scale(amax, a.scale_rule);
            // the correctly rounded quotient y / s (quot2 in ptx.cuh), as in the gate_up epilogue of moe_gemm_fp8.cu
            const float rs = __frcp_rn(sc);
            const float qv = quot2(make_float2(accg[i], 0.0f), make_float2(rs, rs), make_float2(-sc, -sc)).x;
            const size_t slot = (size_t)un.mb * 128 + row0 + i;
            a.out_q[slot * I + un.nt * 128 + r] = (uint8_t)__nv_cvt_float_to_fp8(qv, __NV_SATFINITE, __NV_E4M3);
            if (q == 0 && lane == i) a.out_s[slot * (I / 128) + un.nt] = sc;
        }
    } else {
        const int H = a.n_total;
#pragma unroll
        for (int i = 0; i < C; ++i) {
            const int f = __shfl_sync(0xffffffffu, fl, i);
            const float w = __shfl_sync(0xffffffffu, wl, i);
            if (f < a.n_valid) a.c3[(size_t)f * H + un.nt * 128 + r] = __float2bfloat16_rn(accg[i] * w);
        }
    }
    return true;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_fp8_small_kernel(const __grid_constant__ CUtensorMap tm_tok, const __grid_constant__ CUtensorMap tm_w,
                              const SmallGemmArgs args) {
    constexpr int kStageBytes = SCfg<MODE>::kStageBytes;
    constexpr int kSlots = SCfg<MODE>::kSlots;
    constexpr uint32_t kSlotCols = SCfg<MODE>::kSlotCols;
    const int stages = args.stages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const int KB = args.K / 128;
    float* sa_tab = reinterpret_cast<float*>(smem + (size_t)stages * kStageBytes);  // [2][128][KB]
    SmallTail* tail = reinterpret_cast<SmallTail*>(smem + (size_t)stages * kStageBytes + 2 * 128 * KB * 4);
    volatile int* abort = &tail->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        for (int b = 0; b < kSlots; ++b) {
            mbar_init(smem_u32(&tail->tfull[b]), 1);
            mbar_init(smem_u32(&tail->tempty[b]), kEpiWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tail->safull[b]), 1);
            mbar_init(smem_u32(&tail->saempty[b]), kEpiWarps);
            mbar_init(smem_u32(&tail->xbar[0][b]), 128);
            mbar_init(smem_u32(&tail->xbar[1][b]), 128);
        }
        mbar_init(smem_u32(&tail->drain), 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        prefetch_tensormap(&tm_tok);
        prefetch_tensormap(&tm_w);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    pdl_wait();
    const int blocks = *args.num_post_pad / 128;
    const int num_units = 2 * blocks * args.n_tiles;
    // every thread stages a share of this CTA's unit table (one round of loads in parallel)
    for (int j = threadIdx.x; j < kUnitCache; j += kThreads) {
        const long long u = blockIdx.x + (long long)j * gridDim.x;
        if (u < num_units) {
            const Unit un = unit_of((int)u, blocks, args.n_tiles);
            tail->unit_info[j] = half_info(args, un.mb, un.hp);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tail->tmem_base;
    pdl_trigger();  // after this CTA's TMEM allocation (a dependent CTA could otherwise take the columns first)

    if (warp < kEpiWarp0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 40;" ::: "memory");
        if (warp == 0 && lane == 0) {
            // ---------------------------------------------------------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            int sa_issued[2] = {0, 0};  // scale-table copies issued per buffer
            bool ok = true;
            const uint32_t sa_bytes = (uint32_t)(128 * KB * 4);
            int j = 0;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++j) {
                const Unit un = unit_of(u, blocks, args.n_tiles);
                const int info = unit_info(args, tail->unit_info, j, un);
                const int e = info >> 3, nsub = info & 7;
                if (nsub == 0) continue;
                const uint32_t par = (uint32_t)local & 1u, use = (uint32_t)local >> 1;
                ++local;
                // the block's activation scales [128 slots][KB], contiguous in global memory
                if (!mbar_wait(smem_u32(&tail->saempty[par]), (use & 1u) ^ 1u, abort)) { ok = false; break; }
                mbar_arrive_expect_tx(smem_u32(&tail->safull[par]), sa_bytes);
                bulk_copy_g2s(smem_u32(sa_tab) + par * sa_bytes, args.a_scale + (size_t)un.mb * 128 * KB, sa_bytes,
                              smem_u32(&tail->safull[par]));
                ++sa_issued[par];
                const int wrow = e * args.n_total + un.nt * 128;
                const uint32_t bytes = (uint32_t)((MODE == 0 ? 2 : 1) * kWBytes + nsub * 32 * 128);
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, abort)) { ok = false; break; }
                    const uint32_t dst = sbase + stage * kStageBytes;
                    const uint32_t fb = smem_u32(&tail->full[stage]);
                    mbar_arrive_expect_tx(fb, bytes);
                    tma_load_2d(dst, &tm_w, fb, kb * 128, wrow);
                    if (MODE == 0) tma_load_2d(dst + kWBytes, &tm_w, fb, kb * 128, wrow + args.inter);
                    const uint32_t tok = dst + (MODE == 0 ? 2 : 1) * kWBytes;
                    for (int s = 0; s < nsub; ++s)
                        tma_load_2d(tok + s * 4096, &tm_tok, fb, kb * 128, un.mb * 128 + un.hp * 64 + 32 * s);
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // Unwind: let every copy this thread issued land before the CTA exits (bounded).
                for (int s = 0; s < stages; ++s) {
                    const uint64_t t0 = globaltimer();
                    while (!mbar_try_wait(smem_u32(&tail->full[s]), phase ^ (s < stage ? 0u : 1u)) &&
                           globaltimer() - t0 < PM_WAIT_TIMEOUT_NS) {
                    }
                }
                for (int b = 0; b < 2; ++b) {
                    if (sa_issued[b] == 0) continue;
                    // the last copy into buffer b completes phase sa_issued[b] - 1
                    const uint32_t p = (uint32_t)(sa_issued[b] - 1) & 1u;
                    const uint64_t t0 = globaltimer();
                    while (!mbar_try_wait(smem_u32(&tail->safull[b]), p) && globaltimer() - t0 < PM_WAIT_TIMEOUT_NS) {
                    }
                }
            }
        } else if (warp == 1 && lane == 0) {
            // ---------------------------------------------------------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0, it = 0;
            bool ok = true;
            int j = 0;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++j) {
                const int nsub = unit_info(args, tail->unit_info, j, unit_of(u, blocks, args.n_tiles)) & 7;
                if (nsub == 0) continue;
                const uint32_t idesc = idesc_f32acc(0 /*e4m3*/, 0 /*e4m3*/, 128, 32u * (uint32_t)nsub);
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const uint32_t slot = it % kSlots, use = it / kSlots;
                    if (!mbar_wait(smem_u32(&tail->tempty[slot]), (use & 1u) ^ 1u, abort)) { ok = false; break; }
                    if (!mbar_wait(smem_u32(&tail->full[stage]), phase, abort)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t base = sbase + stage * kStageBytes;
                    const uint64_t dwg = desc_kmajor_sw128(base);
                    const uint64_t dwu = desc_kmajor_sw128(base + kWBytes);
                    const uint64_t dt = desc_kmajor_sw128(base + (MODE == 0 ? 2 : 1) * kWBytes);
                    const uint32_t d = tmem_base + slot * kSlotCols;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {  // 32 e4m3 (32 bytes) of K per instruction
                        mma_f8f6f4(d, dwg + 2 * k, dt + 2 * k, idesc, k > 0 ? 1u : 0u);
                        if (MODE == 0) mma_f8f6f4(d + 64, dwu + 2 * k, dt + 2 * k, idesc, k > 0 ? 1u : 0u);
                    }
                    mma_commit(smem_u32(&tail->empty[stage]));
                    mma_commit(smem_u32(&tail->tfull[slot]));
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                }
            }
            mma_commit(smem_u32(&tail->drain));
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(smem_u32(&tail->drain), 0) && globaltimer() - t0 < PM_WAIT_TIMEOUT_NS) {
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 232;" ::: "memory");
        // ------------------------------------------------------------------ promotion + epilogue
        Ring ring;
        int j = 0;
        for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++j) {
            const Unit un = unit_of(u, blocks, args.n_tiles);
            const int info = unit_info(args, tail->unit_info, j, un);
            const int nsub = info & 7;
            if (nsub == 0) continue;
            const bool ok = nsub == 1 ? run_unit<MODE, 1>(args, tail, sa_tab, un, info >> 3, ring, abort, tmem_base)
                                      : run_unit<MODE, 2>(args, tail, sa_tab, un, info >> 3, ring, abort, tmem_base);
            if (!ok) break;
            ++ring.local;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
    if (threadIdx.x == 0 && tail->abort && args.err != nullptr) atomicExch(args.err, 1);
}

template <int MODE>
size_t small_smem(int stages, int KB) {
    return 1024 + (size_t)stages * SCfg<MODE>::kStageBytes + (size_t)2 * 128 * KB * 4 + sizeof(SmallTail);
}

}  // namespace

bool gemm_fp8_small_fits(int mode, int K) {
    const int KB = K / 128;
    if (K % 128 != 0 || KB > 64) return false;
    const size_t limit = 227 * 1024;
    return (mode == 0 ? small_smem<0>(2, KB) : small_smem<1>(2, KB)) <= limit;
}

cudaError_t launch_gemm_fp8_small(int mode, const CUtensorMap& tm_tok, const CUtensorMap& tm_w,
                                  const SmallGemmArgs& args_in, int num_sms, cudaStream_t s) {
    if (!gemm_fp8_small_fits(mode, args_in.K)) return cudaErrorInvalidValue;
    SmallGemmArgs args = args_in;
    const int KB = args.K / 128;
    const size_t limit = 227 * 1024;
    int stages = kMaxStages;
    while (stages > 2 && (mode == 0 ? small_smem<0>(stages, KB) : small_smem<1>(stages, KB)) > limit) --stages;
    args.stages = stages;
    const size_t smem = mode == 0 ? small_smem<0>(stages, KB) : small_smem<1>(stages, KB);
    static std::atomic<bool> configured[64][2];  // zero-initialised: false
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !configured[dev][mode].load(std::memory_order_acquire)) {
        cudaError_t e = mode == 0 ? cudaFuncSetAttribute(moe_gemm_fp8_small_kernel<0>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)limit)
                                  : cudaFuncSetAttribute(moe_gemm_fp8_small_kernel<1>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)limit);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured[dev][mode].store(true, std::memory_order_release);
    }
    const int units = 2 * args.max_units;  // two halves per block and column tile
    const int grid = units < num_sms ? (units > 0 ? units : 1) : num_sms;
    if (mode == 0)
        PM_TRY(launch_pdl(moe_gemm_fp8_small_kernel<0>, dim3(grid), dim3(kThreads), smem, s, tm_tok, tm_w, args));
    else
        PM_TRY(launch_pdl(moe_gemm_fp8_small_kernel<1>, dim3(grid), dim3(kThreads), smem, s, tm_tok, tm_w, args));
    return cudaGetLastError();
}

}  // namespace pm
