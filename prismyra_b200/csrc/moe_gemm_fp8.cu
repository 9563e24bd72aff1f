// Persistent grouped GEMM for the FP8 (e4m3, 128x128 fp32 block scales) routed experts on sm_100a.
//
// Arithmetic (vLLM fused_moe_kernel, fused_moe.py:483-548, the kernel the reference's FusedExperts calls):
//   acc = sum over 128-wide K blocks kb of  (A_q[row, kb] . B_q[n, kb]) * a_scale[row, kb] * b_scale[n/128, kb]
// The block scales are fp32 (not powers of two), so the tensor core cannot apply them: every K block is one
// tcgen05 MMA chain into a fresh TMEM accumulator, and the promotion warps add it into fp32 registers with the
// block's scale ("software promotion").  Two TMEM accumulators alternate so the MMA of block kb+1 runs while
// block kb is being promoted.
//
// Tiles: 128 rows (one alignment block, one expert) x 256 columns x 128 K per pipeline stage.
//   mode 0 (gate_up, K = H): A is the expert-ordered FP8 copy of x written by the quantisation kernel.  The 256
//           columns are 128 gate rows n0.. and the matching 128 up rows I+n0..; the epilogue applies
//           bf16 -> silu(gate)*up -> bf16 and re-quantises to e4m3 with one scale per 128 output columns (exactly one
//           tile), writing the down GEMM's A operand in slot order.
//   mode 1 (down, K = I): the 256 columns are hidden columns n0..n0+255; the epilogue multiplies by the routing
//           weight in fp32, rounds to bf16 and writes the row to c3[flat index] (or to a per-row destination).
//
// Warp roles (384 threads, three warpgroups):
//   warp 0       TMA producer (A and B tiles of each K block into the stage ring);
//   warp 1       TMEM owner and MMA issuer (one elected lane);
//   warps 2-3    scale loaders: for every tile, in chunks of 16 K blocks, the 128 rows' activation scales and the
//                tile's two weight-scale rows go into a double-buffered shared-memory ring, transposed to
//                [K block][row] so that a promotion warp reads its 32 rows' scales of one K block without bank
//                conflicts.  The scales are thus loaded well ahead of use, off the promotion warps' critical path;
//   warps 4-11   promotion and epilogue: warp w reads TMEM lanes 32*(w%4).. and one half of the tile's columns
//                (two 32-column TMEM loads per wait; the accumulator goes back to the MMA once the last loads have
//                landed), adds each K block into 128 fp32 registers per thread, then runs the tile's epilogue.
// Registers are rebalanced with setmaxnreg: 64 for warpgroup 0 (the scale loaders hold a chunk's 32 scales) and
// 216 for the promotion warpgroups (64*128 + 216*256 = 63488 <= 168*384, the launch's total).
// Every wait is bounded (ptx.cuh): on timeout the kernel raises its abort flag, unwinds and reports through err.
#include <atomic>

#include "moe_internal.h"
#include "ptx.cuh"

namespace pm {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 128;
template <int MODE> struct Cfg {
    // gate_up keeps four pipeline stages; down gives one up for the bf16 staging of its output rows.
    static constexpr int kStages = MODE == 0 ? 4 : 3;
    static constexpr int kStageRowBytes = 144;  // 64 bf16 + 16 B pad: conflict-free row-per-thread writes
    static constexpr int kStagingBytes = MODE == 0 ? 0 : 8 * 32 * kStageRowBytes;
};
constexpr int kMaxStages = 4;
constexpr int kABytes = kBM * kBK;          // 16 KB
constexpr int kBBytes = kBN * kBK;          // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 384;
constexpr int kLoadWarp0 = 2;               // scale loader warps 2-3
constexpr int kLoadThreads = 64;
constexpr int kEpiWarp0 = 4;                // first promotion / epilogue warp
constexpr int kEpiWarps = 8;
constexpr int kChunk = 16;                  // K blocks per scale chunk
constexpr uint32_t kTmemCols = 512;         // two 256-column fp32 accumulators
constexpr uint32_t kIdesc = idesc_f32acc(0 /*e4m3*/, 0 /*e4m3*/, kBM, kBN);

struct ScaleSlot {
    float a[kChunk][kBM];   // activation scale of row r for K block c0 + j, at a[j][r]
    float b[2][kChunk];     // the tile's two weight-scale rows (gate / up groups, or the two column halves)
};

struct SmemTail {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t sc_full[2];    // scale slot filled (arrived by the 64 loader threads)
    uint64_t sc_empty[2];   // scale slot read (arrived by the 8 promotion warps)
    uint64_t drain;
    uint64_t xbar[2];       // epilogue amax exchange, one per tile parity
    uint32_t tmem_base;
    int abort;
    float amax_x[2][2][kBM];  // [tile parity][column half][row]
    ScaleSlot sc[2];
};

template <int MODE>
constexpr size_t smem_bytes() {
    return 1024 /*alignment slack*/ + (size_t)Cfg<MODE>::kStages * kStageBytes + Cfg<MODE>::kStagingBytes +
           sizeof(SmemTail);
}
static_assert(smem_bytes<0>() <= 227 * 1024 && smem_bytes<1>() <= 227 * 1024, "shared memory per CTA");

// silu(g) * u on bf16 values with bf16 rounding after each step (vLLM silu_and_mul semantics) is computed pairwise
// in the gate_up epilogue.  The sigmoid comes from the hardware tanh (relative error below 2^-11): the result is
// rounded to bf16 (8 significant bits) right after, so the error changes an output only when it straddles a bf16
// rounding boundary, and then by one bf16 unit before the e4m3 requantisation.

// acc[c] += scale * r[c] for two runs of 32 values (r0 -> acc0, r1 -> acc1) just loaded from TMEM: packed fp32x2
// FMAs when PACKED.
template <bool PACKED>
__device__ __forceinline__ void fma2x32(const uint32_t (&r0)[32], const uint32_t (&r1)[32], float scale, float* acc0,
                                        float* acc1) {
    if (PACKED) {
        const float2 s2 = make_float2(scale, scale);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
            const float2 v0 = __ffma2_rn(make_float2(__uint_as_float(r0[i]), __uint_as_float(r0[i + 1])), s2,
                                         make_float2(acc0[i], acc0[i + 1]));
            const float2 v1 = __ffma2_rn(make_float2(__uint_as_float(r1[i]), __uint_as_float(r1[i + 1])), s2,
                                         make_float2(acc1[i], acc1[i + 1]));
            acc0[i] = v0.x;
            acc0[i + 1] = v0.y;
            acc1[i] = v1.x;
            acc1[i + 1] = v1.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            acc0[i] = fmaf(__uint_as_float(r0[i]), scale, acc0[i]);
            acc1[i] = fmaf(__uint_as_float(r1[i]), scale, acc1[i]);
        }
    }
}

// Down-GEMM epilogue variants (EPI): kEpiPlain stores bf16(acc * w) to c3; kEpiRoundFirst stores
// bf16(bf16(acc) * w), the bf16 product of a rounded result and a bf16 weight; kEpiDstRows stores each row to the
// address args.dst_rows gives for it (0: not stored).
constexpr int kEpiPlain = 0, kEpiRoundFirst = 1, kEpiDstRows = 2;

template <int MODE, int EPI = kEpiPlain>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_fp8_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const GemmArgs args) {
    constexpr int kStages = Cfg<MODE>::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    uint8_t* staging = smem + (size_t)kStages * kStageBytes;
    SmemTail* tail = reinterpret_cast<SmemTail*>(staging + Cfg<MODE>::kStagingBytes);
    volatile int* abort = &tail->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar_full = smem_u32(tail->full), bar_empty = smem_u32(tail->empty);
    const uint32_t bar_tfull = smem_u32(tail->tfull), bar_tempty = smem_u32(tail->tempty);
    const uint32_t bar_scf = smem_u32(tail->sc_full), bar_sce = smem_u32(tail->sc_empty);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar_tfull + 8 * b, 1);
            mbar_init(bar_tempty + 8 * b, kEpiWarps);
            mbar_init(bar_scf + 8 * b, kLoadThreads);
            mbar_init(bar_sce + 8 * b, kEpiWarps);
        }
        mbar_init(smem_u32(&tail->drain), 1);
        mbar_init(smem_u32(&tail->xbar[0]), kEpiWarps * 32);
        mbar_init(smem_u32(&tail->xbar[1]), kEpiWarps * 32);
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
    const uint32_t tmem_base = tail->tmem_base;
    pdl_wait();
    pdl_trigger();

    const int KB = args.K / kBK;
    const int mb0 = args.slot_lo != nullptr ? *args.slot_lo / kBM : 0;  // first block of this launch
    const int num_tiles = (*args.num_post_pad / kBM - mb0) * args.n_tiles;

    if (warp < kEpiWarp0) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 64;" ::: "memory");
      if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            const int mb = mb0 + tile / args.n_tiles, nt = tile % args.n_tiles;
            const int e = args.expert_ids[mb];
            const int row0 = e * args.n_total + (MODE == 0 ? nt * 128 : nt * kBN);
            const int row1 = (MODE == 0) ? e * args.n_total + args.inter + nt * 128 : row0 + 128;
            for (int kb = 0; kb < KB; ++kb) {
                int go = 1;
                if (lane == 0) go = mbar_wait(bar_empty + 8 * stage, phase ^ 1u, abort) ? 1 : 0;
                go = __shfl_sync(0xffffffffu, go, 0);
                if (!go) { ok = false; break; }
                const uint32_t a_dst = sbase + stage * kStageBytes;
                const uint32_t b_dst = a_dst + kABytes;
                const uint32_t fb = bar_full + 8 * stage;
                if (lane == 0) {
                    mbar_arrive_expect_tx(fb, kStageBytes);
                    tma_load_2d(a_dst, &tm_a, fb, kb * kBK, mb * kBM);
                    tma_load_2d(b_dst, &tm_b, fb, kb * kBK, row0);
                    tma_load_2d(b_dst + kBBytes / 2, &tm_b, fb, kb * kBK, row1);
                }
                __syncwarp();
                if (++stage == kStages) { stage = 0; phase ^= 1u; }
            }
        }
        if (!ok && lane == 0) {
            // Unwind: let every load this warp issued land before the CTA exits (bounded).
            for (int s = 0; s < kStages; ++s) {
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(bar_full + 8 * s, phase ^ (s < stage ? 0u : 1u)) &&
                       globaltimer() - t0 < PM_WAIT_TIMEOUT_NS) {
                }
            }
        }
      } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const uint32_t buf = it & 1u, use = it >> 1;
                    if (!mbar_wait(bar_tempty + 8 * buf, (use & 1u) ^ 1u, abort)) { ok = false; break; }
                    if (!mbar_wait(bar_full + 8 * stage, phase, abort)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = sbase + stage * kStageBytes;
                    const uint64_t da = desc_kmajor_sw128(a_addr);
                    const uint64_t db = desc_kmajor_sw128(a_addr + kABytes);
                    const uint32_t d_tmem = tmem_base + buf * kBN;
#pragma unroll
                    for (int k = 0; k < kBK / 32; ++k)  // 32 e4m3 (32 bytes) of K per instruction
                        mma_f8f6f4(d_tmem, da + 2 * k, db + 2 * k, kIdesc, k > 0 ? 1u : 0u);
                    mma_commit(bar_empty + 8 * stage);
                    mma_commit(bar_tfull + 8 * buf);
                    if (++stage == kStages) { stage = 0; phase ^= 1u; }
                }
            }
            // Every MMA this thread issued completes before TMEM is released.
            mma_commit(smem_u32(&tail->drain));
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(smem_u32(&tail->drain), 0) && globaltimer() - t0 < PM_WAIT_TIMEOUT_NS) {
            }
        }
      } else {
        // ------------------------------------------------------------------ scale loaders (warps 2-3)
        // Thread t fills rows t and t+64 of a chunk; threads 0..15 also the two weight-scale rows.
        const int t = threadIdx.x - kLoadWarp0 * 32;
        const int nb_total = args.n_total / 128;
        uint32_t chunk = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            const int mb = mb0 + tile / args.n_tiles, nt = tile % args.n_tiles;
            const int e = args.expert_ids[mb];
            const float* bs = args.b_scale + (size_t)e * nb_total * KB;
            const float* brow0 = bs + (size_t)(MODE == 0 ? nt : nt * 2) * KB;
            const float* brow1 = bs + (size_t)(MODE == 0 ? args.inter / 128 + nt : nt * 2 + 1) * KB;
            const float* as0 = args.a_scale + (size_t)(mb * kBM + t) * KB;
            const float* as1 = as0 + (size_t)64 * KB;
            for (int c0 = 0; c0 < KB; c0 += kChunk, ++chunk) {
                const uint32_t slot = chunk & 1u, use = chunk >> 1;
                const int n = KB - c0 < kChunk ? KB - c0 : kChunk;
                float v0[kChunk], v1[kChunk];
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {  // the loads are issued before the slot is waited for
                    v0[j] = j < n ? as0[c0 + j] : 0.0f;
                    v1[j] = j < n ? as1[c0 + j] : 0.0f;
                }
                float b0 = 0.0f, b1 = 0.0f;
                if (t < n) {
                    b0 = brow0[c0 + t];
                    b1 = brow1[c0 + t];
                }
                if (!mbar_wait(bar_sce + 8 * slot, (use & 1u) ^ 1u, abort)) { ok = false; break; }
                ScaleSlot& S = tail->sc[slot];
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {
                    S.a[j][t] = v0[j];
                    S.a[j][t + 64] = v1[j];
                }
                if (t < kChunk) {
                    S.b[0][t] = b0;
                    S.b[1][t] = b1;
                }
                mbar_arrive(bar_scf + 8 * slot);
            }
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
        // ------------------------------------------------------------------ promotion + epilogue
        const int q = warp & 3;                    // TMEM lane quarter
        const int half = (warp - kEpiWarp0) >> 2;  // column half
        const int row = q * 32 + lane;
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
        // Packed FMAs halve the promotion's issue slots; in the down GEMM they cost spills, so it stays scalar.
        constexpr bool kPackedPromote = MODE == 0;
        uint32_t it = 0, chunk = 0;
        int local = 0;
        float acc[128];
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
            const int mb = mb0 + tile / args.n_tiles, nt = tile % args.n_tiles;
            const int grow = mb * kBM + row;
            // down: the row's flat index (the slot itself when there is no row map), its routing weight and, with a
            // destination table, the address its weighted row is stored to (0: the slot holds no row)
            const int flat = MODE == 1 ? (args.sorted_ids != nullptr ? args.sorted_ids[grow] : grow) : 0;
            const uint64_t drow = (MODE == 1 && EPI == kEpiDstRows) ? args.dst_rows[grow] : 0;
            float w = 0.0f;
#pragma unroll
            for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
            bool ok = true;
            const ScaleSlot* S = nullptr;
            for (int kb = 0; kb < KB; ++kb, ++it) {
                const uint32_t buf = it & 1u, use = it >> 1;
                const int j = kb % kChunk;
                if (j == 0) {
                    if (!mbar_wait(bar_scf + 8 * (chunk & 1u), (chunk >> 1) & 1u, abort)) { ok = false; break; }
                    S = &tail->sc[chunk & 1u];
                }
                const float sa = S->a[j][row];
                const float s0 = sa * S->b[MODE == 0 ? 0 : half][j];
                const float s1 = sa * S->b[MODE == 0 ? 1 : half][j];
                if (j == kChunk - 1 || kb == KB - 1) {  // this chunk's scales have been read
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar_sce + 8 * (chunk & 1u));
                    ++chunk;
                }
                if (MODE == 1 && kb == (KB > 1 ? 1 : 0)) w = flat < args.n_valid ? args.topk_w[flat] : 0.0f;
                if (!mbar_wait(bar_tfull + 8 * buf, use & 1u, abort)) { ok = false; break; }
                tc_fence_after();
                const uint32_t tb = t_lane + buf * kBN;
                // this thread's 128 columns: mode 0 gate columns [64*half, +64) then up columns [128+64*half, +64);
                // mode 1 columns [128*half, +128).  Two 32-column TMEM loads per wait; the accumulator is handed
                // back to the MMA as soon as the last load has landed, before that pair's FMAs.
                const uint32_t c0 = MODE == 0 ? 64 * half : 128 * half;
                const uint32_t c1 = MODE == 0 ? 128 + 64 * half : 128 * half + 64;
                {
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tb + c0, r0);
                    tmem_ld32(tb + c0 + 32, r1);
                    tmem_ld_wait();
                    fma2x32<kPackedPromote>(r0, r1, s0, acc, acc + 32);
                }
                {
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tb + c1, r0);
                    tmem_ld32(tb + c1 + 32, r1);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar_tempty + 8 * buf);
                    fma2x32<kPackedPromote>(r0, r1, MODE == 0 ? s1 : s0, acc + 64, acc + 96);
                }
            }
            if (!ok) break;

            if (MODE == 0) {
                // bf16(gate), bf16(up) -> silu(gate) * up in bf16 -> e4m3 with one scale per 128 columns, a
                // pair of columns per instruction.  The loop is bound by its instruction count, so up, silu(gate)
                // and their product stay packed bf16: the product of two bf16 values is exact in fp32, so one
                // correctly rounded bf16 multiply gives the same bits as the fp32 product rounded to bf16, and the
                // row maximum of |y| is taken on the packed values.
                __nv_bfloat162 amax2 = __float2bfloat162_rn(0.0f);
#pragma unroll
                for (int c = 0; c < 64; c += 2) {
                    const __nv_bfloat162 gb = __floats2bfloat162_rn(acc[c], acc[c + 1]);
                    const __nv_bfloat162 ub = __floats2bfloat162_rn(acc[64 + c], acc[64 + c + 1]);
                    const float2 s2 = silu2(__bfloat1622float2(gb));
                    const __nv_bfloat162 yb = __hmul2(__floats2bfloat162_rn(s2.x, s2.y), ub);
                    amax2 = __hmax2(amax2, __habs2(yb));
                    const float2 y = __bfloat1622float2(yb);
                    acc[c] = y.x;
                    acc[c + 1] = y.y;
                }
                float amax = fmaxf(__low2float(amax2), __high2float(amax2));
                // The other column half of this row lives in another warp: exchange the half maxima through
                // shared memory, synchronised by an mbarrier (a bounded wait, unlike a named barrier).
                tail->amax_x[local & 1][half][row] = amax;
                const uint32_t xb = smem_u32(&tail->xbar[local & 1]);
                mbar_arrive(xb);
                if (!mbar_wait(xb, (uint32_t)(local >> 1) & 1u, abort)) break;
                amax = fmaxf(tail->amax_x[local & 1][0][row], tail->amax_x[local & 1][1][row]);
                const float sc = e4m3_group_scale(amax, args.scale_rule);
                // Codes are the correctly rounded quotients y / s (quot2), as vLLM's quantiser computes them; the
                // saturating conversion clamps to +-448 exactly as clamp-then-round does.
                const float inv = __frcp_rn(sc);
                const float2 inv2 = make_float2(inv, inv), nsc2 = make_float2(-sc, -sc);
                uint32_t packed[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float2 q01 = quot2(make_float2(acc[4 * i + 0], acc[4 * i + 1]), inv2, nsc2);
                    const float2 q23 = quot2(make_float2(acc[4 * i + 2], acc[4 * i + 3]), inv2, nsc2);
                    packed[i] = (uint32_t)e4m3x2(q01.x, q01.y) | ((uint32_t)e4m3x2(q23.x, q23.y) << 16);
                }
                uint4* dst = reinterpret_cast<uint4*>(args.out_q + (size_t)grow * args.inter + nt * 128 + 64 * half);
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    dst[u] = make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
                if (half == 0) args.out_s[(size_t)grow * (args.inter / 128) + nt] = sc;
            } else {
                // Weight, round, and stage this warp's 32 rows in shared memory 64 columns at a time (one row per
                // thread), writing each pass out as coalesced 128-byte row segments, four rows per instruction.
                constexpr int RB = Cfg<MODE>::kStageRowBytes;
                uint8_t* wst = staging + (size_t)(warp - kEpiWarp0) * 32 * RB;
                if constexpr (EPI == kEpiRoundFirst) {
#pragma unroll
                    for (int i = 0; i < 128; ++i) acc[i] = __bfloat162float(__float2bfloat16_rn(acc[i]));
                }
                const int H = args.n_total;
                const int sub = lane >> 3, chunk8 = lane & 7;
#pragma unroll
                for (int p = 0; p < 2; ++p) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        uint4 o;
                        __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            ob[i] = __floats2bfloat162_rn(acc[64 * p + 8 * u + 2 * i] * w,
                                                          acc[64 * p + 8 * u + 2 * i + 1] * w);
                        *reinterpret_cast<uint4*>(wst + lane * RB + u * 16) = o;
                    }
                    __syncwarp();
                    // Columns [nt*256 + 128*half + 64*p, +64) of an H-wide row: 128 bytes = 8 lanes x 16 bytes.
                    const int col = nt * kBN + 128 * half + 64 * p + chunk8 * 8;
#pragma unroll 4
                    for (int r = 0; r < 32; r += 4) {
                        const int f = __shfl_sync(0xffffffffu, flat, r + sub);
                        const uint4 v = *reinterpret_cast<const uint4*>(wst + (r + sub) * RB + chunk8 * 16);
                        if constexpr (EPI == kEpiDstRows) {
                            const uint64_t dr = __shfl_sync(0xffffffffu, drow, r + sub);
                            if (f < args.n_valid && dr != 0)
                                *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dr) + col) = v;
                        } else if (f < args.n_valid) {
                            *reinterpret_cast<uint4*>(args.c3 + (size_t)f * H + col) = v;
                        }
                    }
                    __syncwarp();
                }
            }
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

}  // namespace

cudaError_t launch_gemm_fp8(int mode, const CUtensorMap& tm_a, const CUtensorMap& tm_b, const GemmArgs& args,
                            int num_sms, cudaStream_t s) {
    // variant 0: gate_up; 1..3: down with the plain, round-first or per-row-destination epilogue
    static std::atomic<bool> configured[64][4];  // zero-initialised: false
    const int variant = mode == 0 ? 0 : (args.dst_rows != nullptr ? 3 : (args.round_first ? 2 : 1));
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured[dev][variant].load(std::memory_order_acquire)) {
        cudaError_t e;
        switch (variant) {
            case 0: e = cudaFuncSetAttribute(moe_gemm_fp8_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem_bytes<0>()); break;
            case 1: e = cudaFuncSetAttribute(moe_gemm_fp8_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem_bytes<1>()); break;
            case 2: e = cudaFuncSetAttribute(moe_gemm_fp8_kernel<1, kEpiRoundFirst>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes<1>()); break;
            default: e = cudaFuncSetAttribute(moe_gemm_fp8_kernel<1, kEpiDstRows>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes<1>());
        }
        if (e != cudaSuccess) return e;
        configured[dev][variant].store(true, std::memory_order_release);
    }
    const int grid = args.max_tiles < num_sms ? (args.max_tiles > 0 ? args.max_tiles : 1) : num_sms;
    switch (variant) {
        case 0: PM_TRY(launch_pdl(moe_gemm_fp8_kernel<0>, dim3(grid), dim3(kThreads), smem_bytes<0>(), s, tm_a, tm_b,
                                  args)); break;
        case 1: PM_TRY(launch_pdl(moe_gemm_fp8_kernel<1>, dim3(grid), dim3(kThreads), smem_bytes<1>(), s, tm_a, tm_b,
                                  args)); break;
        case 2: PM_TRY(launch_pdl(moe_gemm_fp8_kernel<1, kEpiRoundFirst>, dim3(grid), dim3(kThreads), smem_bytes<1>(),
                                  s, tm_a, tm_b, args)); break;
        default: PM_TRY(launch_pdl(moe_gemm_fp8_kernel<1, kEpiDstRows>, dim3(grid), dim3(kThreads), smem_bytes<1>(),
                                   s, tm_a, tm_b, args));
    }
    return cudaGetLastError();
}

}  // namespace pm
