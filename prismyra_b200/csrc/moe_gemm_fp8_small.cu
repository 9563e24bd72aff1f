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
// Unit of work: (64-slot half hp of block mb, 128 output columns nt); all first halves come before the second
// halves, which exist only for blocks with more than 64 real tokens (those read their weights twice).  One launch
// runs one GEMM (units round-robin over the CTAs) or, in the forward, both: the gate_up units and then the down
// units from one work queue, a down unit starting once its block half's gate_up rows are all stored -- so the SMs
// that finish the gate_up units early stream down weights instead of idling through the gate_up tail.
//   mode 0 (gate_up): gate rows nt*128.. and up rows I + nt*128.. of expert e: two MMAs per K step into two TMEM
//          accumulators; epilogue bf16 -> silu(gate)*up -> bf16 -> e4m3 with one scale per token over the unit's
//          128 output columns (exactly one requantisation group), written to the down GEMM's A operand.
//   mode 1 (down): hidden rows nt*256.. and nt*256+128.. of expert e, as two tiles and two accumulators like
//          gate_up (a unit twice as large as one tile halves its fixed costs per byte); epilogue multiplies by the
//          token's routing weight in fp32, rounds to bf16 and writes c3[flat index, nt*256 ..].
// Warp roles (384 threads): warp 0 TMA (weight tiles, token tiles, and per unit the block's activation scales as
// one bulk copy), warp 1 TMEM + MMA, warps 4-11 promotion and epilogue: warp w reads TMEM lanes 32*(w%4).. (weight
// rows) and token columns of half (w-4)/4 of the unit.  TMEM is a ring of eight 64-column slots: a K block takes
// one (first tile at +0, second at +32) when the half holds one token sub-block and two when it holds two; the MMA
// thus runs up to eight K blocks ahead of the promotion, through a unit's epilogue.
// An M=128 FP8 MMA with N <= 128 costs ~107 cycles in a chain on one accumulator whatever N is, but ~196 when
// consecutive instructions alternate between two accumulators (~143 over four): the MMA thread issues each
// accumulator's four K steps back to back (gate, then up).  setmaxnreg gives warpgroup 0 64 registers and the
// promotion warpgroups 216 (64*128 + 216*256 = 63488 <= 168*384, the launch's total).  Every wait is bounded.
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

constexpr int kSlots = 8;            // TMEM slots of kSlotCols columns
constexpr uint32_t kSlotCols = 64;
constexpr int kQueue = 4;            // units handed from the producer to the MMA and promotion warps
constexpr int kMaxBlocks = 512;      // 128-slot blocks a launch may have (the few-token regime has far fewer)
// Stage bytes: a unit's two weight tiles (gate and up rows; down: two consecutive 128-row tiles) and up to 64
// token rows.
template <int MODE> __host__ __device__ constexpr int stage_bytes() { return 2 * kWBytes + kTokBytes; }
// TMEM slots one K block of a unit with nsub token sub-blocks takes: its two accumulators share a 64-column slot
// (at +0 and +32) for one sub-block, or take one slot each for two.
__device__ __forceinline__ int slots_per_kblock(int nsub) { return nsub; }
// First weight row of a unit's second tile, relative to its first: the up rows (gate_up), or the next 128 rows.
__device__ __forceinline__ int second_tile_rows(int m, int inter) { return m == 0 ? inter : 128; }

// Per-unit values the promotion warps need, loaded ahead by warp 2: the unit's two weight-scale rows (gate and up;
// down: one) and, for a down unit, the flat index and routing weight of each of the half's 64 slots.
struct UnitRec {
    float bg[64];
    float bu[64];
    int fl[64];
    float wl[64];
};

struct SmallTail {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tfull[kMaxSlots];
    uint64_t tempty[kMaxSlots];
    uint64_t safull[2];   // the unit's activation-scale table (by unit parity) has landed
    uint64_t saempty[2];  // the epilogue is done with it
    uint64_t xbar[2][2];  // [column half][gate_up unit parity] per-token amax exchange between the lane quarters
    uint64_t dbar[2];     // fused: every promotion thread has stored its rows of a gate_up unit (by parity)
    uint64_t qfull[kQueue];
    uint64_t qempty[kQueue];
    uint64_t ufull[2];    // the unit record (by unit parity) is loaded
    uint64_t uempty[2];   // the promotion warps are done with it
    uint64_t drain;
    int2 queue[kQueue];   // (unit index or -1 at the end, expert * 8 + real token sub-blocks)
    uint32_t tmem_base;
    int abort;
    float amax_x[2][2][4][32];  // [gate_up unit parity][column half][lane quarter][token column]
    int n_second;               // blocks whose second half holds tokens, listed in ascending order:
    int second[kMaxBlocks];
    int wcount[kThreads / 32];  // per-warp counts of the listing
    UnitRec urec[2];
};

// A launch's units, in order: per GEMM (gate_up, then down when fused), the first 64-slot halves of all blocks, then
// the second halves of the blocks listed in SmallTail::second (the others hold no token there); block-major, column
// tile minor.
struct Unit {
    int hp, mb, nt;
};
struct UnitSpace {
    int blocks, n_second, nt0, nt1, per0, total;  // per0: units of the first GEMM
    __device__ __forceinline__ Unit resolve(const int* second, int g, int& ph) const {
        ph = g >= per0 ? 1 : 0;
        const int v = ph ? g - per0 : g, nt = ph ? nt1 : nt0;
        if (v < blocks * nt) return Unit{0, v / nt, v % nt};
        const int w = v - blocks * nt;
        return Unit{1, second[w / nt], w % nt};
    }
};

// Expert * 8 + real 32-slot sub-blocks (1 or 2) of half hp of block mb (a half in the unit space holds a token in
// its first slot; its second sub-block holds tokens iff its first slot does).
__device__ __forceinline__ int half_info(const SmallGemmArgs& a, int mb, int hp) {
    return a.expert_ids[mb] * 8 + 1 + (a.sorted_ids[mb * 128 + hp * 64 + 32] < a.n_valid ? 1 : 0);
}

// acc[c] += D[c] * (sa[c] * sw) for 16 columns already loaded from TMEM.
__device__ __forceinline__ void fma16(const uint32_t (&d)[16], const float* sa, float sw, float* acc) {
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = fmaf(__uint_as_float(d[i]), sa[i] * sw, acc[i]);
}

// Halving step of a transposed warp max: W values per lane -> W/2, lanes with `mask` set keeping the upper half.
template <int W>
__device__ __forceinline__ void col_max_halve(float* w, int lane, int mask) {
    const bool hi = (lane & mask) != 0;
#pragma unroll
    for (int j = 0; j < W / 2; ++j) {
        const float send = hi ? w[j] : w[j + W / 2];
        const float keep = hi ? w[j + W / 2] : w[j];
        w[j] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, mask));
    }
}
// The maxima over the warp's 32 lanes of each of C (16 or 32) columns, transposed: lane l returns the maximum of
// column l >> 1 (C = 16; lanes l and l ^ 1 agree) or l (C = 32).  C - 1 + (C == 16) shuffles instead of 5 C.
template <int C>
__device__ __forceinline__ float warp_col_max(const float* v, int lane) {
    float w[C];
#pragma unroll
    for (int i = 0; i < C; ++i) w[i] = v[i];
    if constexpr (C == 32) col_max_halve<32>(w, lane, 16);
    col_max_halve<16>(w, lane, C == 32 ? 8 : 16);
    col_max_halve<8>(w, lane, C == 32 ? 4 : 8);
    col_max_halve<4>(w, lane, C == 32 ? 2 : 4);
    col_max_halve<2>(w, lane, C == 32 ? 1 : 2);
    if constexpr (C == 16) w[0] = fmaxf(w[0], __shfl_xor_sync(0xffffffffu, w[0], 1));
    return w[0];
}

struct Ring {
    uint32_t it = 0;  // TMEM slots consumed so far
    int local = 0;    // units done so far (activation-scale table buffers)
    int n0 = 0;       // gate_up units done so far (row-maximum exchange; fused: the hand-off barrier)
};

// Promotion over one unit's K blocks and its epilogue, for NSUB real token sub-blocks in the half (this thread:
// 16*NSUB token columns starting at half * 16*NSUB).  Returns false when a wait gave up.
template <int MODE, int NSUB>
__device__ __forceinline__ bool run_unit(const SmallGemmArgs& a, SmallTail* tail, const float* sa_tab, int kb_max,
                                         const Unit& un, int e, Ring& ring, volatile int* abort, uint32_t tmem_base) {
    constexpr int C = 16 * NSUB;  // token columns of this thread
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = warp & 3, half = (warp - kEpiWarp0) >> 2;
    const int r = q * 32 + lane;  // weight row of the unit's tiles (gate_up: output column nt*128 + r)
    const int KB = a.K / 128;
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    const int col0 = half * C;                  // first token column of this thread within the unit
    const int row0 = un.hp * 64 + col0;         // ... as a slot of block mb
    const uint32_t par = (uint32_t)ring.local & 1u, use = (uint32_t)ring.local >> 1;
    const uint32_t xpar = (uint32_t)ring.n0 & 1u, xuse = (uint32_t)ring.n0 >> 1;  // gate_up units only

    // the unit record: weight block scales lane-distributed (lane l holds K blocks l and l + 32) and, down, the flat
    // index and routing weight of each token column (lane l: column col0 + l)
    if (!mbar_wait(smem_u32(&tail->ufull[par]), use & 1u, abort)) return false;
    const UnitRec& R = tail->urec[par];
    const float g0 = lane < KB ? R.bg[lane] : 0.0f, g1 = lane + 32 < KB ? R.bg[lane + 32] : 0.0f;
    const float u0 = lane < KB ? R.bu[lane] : 0.0f;
    const float u1 = lane + 32 < KB ? R.bu[lane + 32] : 0.0f;
    int fl = 0;
    float wl = 0.0f;
    if (MODE == 1) {
        fl = lane < C ? R.fl[col0 + lane] : a.n_valid;
        wl = lane < C ? R.wl[col0 + lane] : 0.0f;
    }

    float accg[C], accu[C];  // the unit's first and second tile (gate and up)
#pragma unroll
    for (int i = 0; i < C; ++i) accg[i] = 0.0f;
#pragma unroll
    for (int i = 0; i < C; ++i) accu[i] = 0.0f;

    if (!mbar_wait(smem_u32(&tail->safull[par]), use & 1u, abort)) return false;
    const float* sa = sa_tab + (size_t)par * 128 * kb_max + (size_t)row0 * KB;
    for (int kb = 0; kb < KB; ++kb) {
        // this K block's TMEM slots (the MMA thread walks the same sequence)
        const uint32_t s0 = ring.it % kSlots, p0 = (ring.it / kSlots) & 1u;
        ++ring.it;
        uint32_t s1 = s0, p1 = p0;
        if (NSUB == 2) {
            s1 = ring.it % kSlots;
            p1 = (ring.it / kSlots) & 1u;
            ++ring.it;
        }
        const float swg = __shfl_sync(0xffffffffu, kb < 32 ? g0 : g1, kb & 31);
        const float swu = __shfl_sync(0xffffffffu, kb < 32 ? u0 : u1, kb & 31);
        float sak[C];  // the token columns' activation scales (loaded before the TMEM wait)
#pragma unroll
        for (int i = 0; i < C; ++i) sak[i] = sa[(size_t)i * KB + kb];
        if (!mbar_wait(smem_u32(&tail->tfull[s0]), p0, abort)) return false;
        if (NSUB == 2 && !mbar_wait(smem_u32(&tail->tfull[s1]), p1, abort)) return false;
        tc_fence_after();
        const uint32_t tg = t_lane + s0 * kSlotCols + (uint32_t)col0;
        const uint32_t tu = NSUB == 1 ? tg + 32 : t_lane + s1 * kSlotCols + (uint32_t)col0;
        uint32_t dg[NSUB][16], du[NSUB][16];
#pragma unroll
        for (int c = 0; c < NSUB; ++c) {
            tmem_ld16(tg + 16 * c, dg[c]);
            tmem_ld16(tu + 16 * c, du[c]);
        }
        tmem_ld_wait();
        // the values are in registers: hand the slots back to the MMA before the FMAs
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(smem_u32(&tail->tempty[s0]));
            if (NSUB == 2) mbar_arrive(smem_u32(&tail->tempty[s1]));
        }
#pragma unroll
        for (int c = 0; c < NSUB; ++c) {
            fma16(dg[c], sak + 16 * c, swg, accg + 16 * c);
            fma16(du[c], sak + 16 * c, swu, accu + 16 * c);
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&tail->saempty[par]));

    if (MODE == 0) {
        // y = bf16(bf16(silu(bf16(gate))) * bf16(up)) per (row, token); per token the amax over the 128 rows: a
        // transposed warp maximum (lane l ends with one column's), then the four lane quarters through shared
        // memory (bounded mbarrier wait); each column's scale is formed once, by the lane holding it
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
            accu[i] = fabsf(y.x);
            accu[i + 1] = fabsf(y.y);
        }
        const float m = warp_col_max<C>(accu, lane);
        const int mycol = C == 32 ? lane : lane >> 1;
        float(*ax)[32] = tail->amax_x[xpar][half];
        if (C == 32 || (lane & 1) == 0) ax[q][mycol] = m;
        const uint32_t xb = smem_u32(&tail->xbar[half][xpar]);
        mbar_arrive(xb);
        if (!mbar_wait(xb, xuse & 1u, abort)) return false;
        const int I = a.inter;
        const float amax = fmaxf(fmaxf(ax[0][mycol], ax[1][mycol]), fmaxf(ax[2][mycol], ax[3][mycol]));
        const float sc = e4m3_group_scale(amax, a.scale_rule);
        const float rs = __frcp_rn(sc);
        if (q == 0 && (C == 32 || (lane & 1) == 0))
            a.out_s[((size_t)un.mb * 128 + row0 + mycol) * (I / 128) + un.nt] = sc;
#pragma unroll
        for (int i = 0; i < C; i += 2) {
            // column i's scale from the lane holding it; the correctly rounded quotients y / s (quot2 in ptx.cuh),
            // as in the gate_up epilogue of moe_gemm_fp8.cu
            const int l0 = C == 32 ? i : 2 * i, l1 = C == 32 ? i + 1 : 2 * i + 2;
            const float sc0 = __shfl_sync(0xffffffffu, sc, l0), sc1 = __shfl_sync(0xffffffffu, sc, l1);
            const float rs0 = __shfl_sync(0xffffffffu, rs, l0), rs1 = __shfl_sync(0xffffffffu, rs, l1);
            const float2 qv =
                quot2(make_float2(accg[i], accg[i + 1]), make_float2(rs0, rs1), make_float2(-sc0, -sc1));
            const size_t slot = (size_t)un.mb * 128 + row0 + i;
            a.out_q[slot * I + un.nt * 128 + r] = (uint8_t)__nv_cvt_float_to_fp8(qv.x, __NV_SATFINITE, __NV_E4M3);
            a.out_q[(slot + 1) * I + un.nt * 128 + r] =
                (uint8_t)__nv_cvt_float_to_fp8(qv.y, __NV_SATFINITE, __NV_E4M3);
        }
    } else {
        const int H = a.n_total;
#pragma unroll
        for (int i = 0; i < C; ++i) {
            const int f = __shfl_sync(0xffffffffu, fl, i);
            const float w = __shfl_sync(0xffffffffu, wl, i);
            if (f < a.n_valid) {
                a.c3[(size_t)f * H + un.nt * 256 + r] = __float2bfloat16_rn(accg[i] * w);
                a.c3[(size_t)f * H + un.nt * 256 + 128 + r] = __float2bfloat16_rn(accu[i] * w);
            }
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&tail->uempty[par]));
    return true;
}

// MODE 0: gate_up units of (tm_tok0, tm_w0, a0); 1: down units of the same; 2 (fused): the gate_up units of
// (tm_tok0, tm_w0, a0), then the down units of (tm_tok1, tm_w1, a1), taken from the work queue sched[0]; a down unit
// waits until sched[1 + 2 * block + half] counts every gate_up unit of its block half, whose promotion threads raise
// it after their stores (an mbarrier among them, a fence, an atomic add).  Each CTA takes its gate_up units before
// its down units, so the units a down unit waits for are held by CTAs that never wait themselves, and the grid is
// resident at once (one CTA per SM, at most one per SM): the waits end.
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_fp8_small_kernel(const __grid_constant__ CUtensorMap tm_tok0, const __grid_constant__ CUtensorMap tm_w0,
                              const __grid_constant__ CUtensorMap tm_tok1, const __grid_constant__ CUtensorMap tm_w1,
                              const SmallGemmArgs a0, const SmallGemmArgs a1, int32_t* sched) {
    constexpr int kStageBytes = stage_bytes<MODE>();
    const int stages = a0.stages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const int kb_max = (MODE == 2 && a1.K > a0.K ? a1.K : a0.K) / 128;
    float* sa_tab = reinterpret_cast<float*>(smem + (size_t)stages * kStageBytes);  // [2][128][K/128 of the unit]
    SmallTail* tail = reinterpret_cast<SmallTail*>(smem + (size_t)stages * kStageBytes + 2 * 128 * kb_max * 4);
    volatile int* abort = &tail->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (MODE == 2 && threadIdx.x == 96 && (int)blockIdx.x < a0.prefetch_units) {
        // The weights of this CTA's likely first gate_up unit (unit = CTA index, block b taken to hold expert b, as
        // when every expert has one block), into L2 while the predecessor runs: constant data, so no need to wait
        // for it; a wrong guess only costs the prefetch.
        const int e = (int)blockIdx.x / a0.n_tiles, nt = (int)blockIdx.x % a0.n_tiles;
        const int wrow = e * a0.n_total + nt * 128;
        for (int kb = 0; kb < a0.K / 128; ++kb) {
            tma_prefetch_l2(&tm_w0, kb * 128, wrow);
            tma_prefetch_l2(&tm_w0, kb * 128, wrow + a0.inter);
        }
    }
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
            mbar_init(smem_u32(&tail->dbar[b]), kEpiWarps * 32);
        }
        for (int b = 0; b < kQueue; ++b) {
            mbar_init(smem_u32(&tail->qfull[b]), 1);
            mbar_init(smem_u32(&tail->qempty[b]), 2 + kEpiWarps);  // the MMA thread, warp 2, the promotion warps
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tail->ufull[b]), 1);
            mbar_init(smem_u32(&tail->uempty[b]), kEpiWarps);
        }
        mbar_init(smem_u32(&tail->drain), 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        prefetch_tensormap(&tm_tok0);
        prefetch_tensormap(&tm_w0);
        if (MODE == 2) {
            prefetch_tensormap(&tm_tok1);
            prefetch_tensormap(&tm_w1);
        }
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    pdl_wait();
    const int blocks = min(*a0.num_post_pad / 128, kMaxBlocks);
    // the blocks with tokens in their second half, in ascending order (a ballot compaction per round of 384)
    if (threadIdx.x == 0) tail->n_second = 0;
    __syncthreads();
    for (int b0 = 0; b0 < blocks; b0 += kThreads) {
        const int b = b0 + (int)threadIdx.x;
        const bool has = b < blocks && a0.sorted_ids[b * 128 + 64] < a0.n_valid;
        const uint32_t ball = __ballot_sync(0xffffffffu, has);
        int* wcount = tail->wcount;
        if (lane == 0) wcount[warp] = __popc(ball);
        __syncthreads();
        int before = tail->n_second, total = 0;
        for (int w = 0; w < kThreads / 32; ++w) {
            before += w < warp ? wcount[w] : 0;
            total += wcount[w];
        }
        if (has) tail->second[before + __popc(ball & ((1u << lane) - 1u))] = b;
        __syncthreads();
        if (threadIdx.x == 0) tail->n_second += total;
        __syncthreads();
    }
    UnitSpace sp;
    sp.blocks = blocks;
    sp.n_second = tail->n_second;
    sp.nt0 = a0.n_tiles;
    sp.nt1 = MODE == 2 ? a1.n_tiles : 0;
    sp.per0 = (blocks + sp.n_second) * sp.nt0;
    sp.total = sp.per0 + (blocks + sp.n_second) * sp.nt1;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tail->tmem_base;
    pdl_trigger();  // after this CTA's TMEM allocation (a dependent CTA could otherwise take the columns first)

    if (warp < kEpiWarp0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 64;" ::: "memory");
        if (warp == 0 && lane == 0) {
            // ---------------------------------------------------------------- TMA producer and scheduler
            // One GEMM: units go round-robin over the fewest CTAs that need as many rounds as the whole grid would
            // (each unit runs at a per-SM rate, so a last round only some CTAs have gains nothing from the others,
            // and fewer CTAs contend less for HBM; second halves are not counted).  Fused: a queue.
            const int first_units = blocks * a0.n_tiles;
            const int rounds = first_units > 0 ? (first_units + (int)gridDim.x - 1) / (int)gridDim.x : 1;
            const int stride = first_units > 0 ? (first_units + rounds - 1) / rounds : (int)gridDim.x;
            int next_g = (int)blockIdx.x < stride ? (int)blockIdx.x : sp.total;
            // the fused queue is read one unit ahead: the next index is fetched while this unit's loads go out
            auto grab = [&]() -> int {
                if (MODE == 2) return atomicAdd(sched, 1);
                const int v = next_g;
                next_g += stride;
                return v;
            };
            int stage = 0;
            uint32_t phase = 0;
            int local = 0, nq = 0;
            int sa_issued[2] = {0, 0};  // scale-table copies issued per buffer
            bool ok = true;
            int g = grab();
            int ph = 0;
            Unit un{0, 0, 0};
            int info = 0;
            if (g < sp.total) {
                un = sp.resolve(tail->second, g, ph);
                info = half_info(ph ? a1 : a0, un.mb, un.hp);
            }
            while (ok) {
                if (g >= sp.total) g = -1;
                {
                    const uint32_t qs = (uint32_t)nq % kQueue, qu = (uint32_t)nq / kQueue;
                    ++nq;
                    if (!mbar_wait(smem_u32(&tail->qempty[qs]), (qu & 1u) ^ 1u, abort)) { ok = false; break; }
                    tail->queue[qs] = make_int2(g, info);
                    mbar_arrive(smem_u32(&tail->qfull[qs]));
                }
                if (g < 0) break;
                const int g_next = grab();
                const SmallGemmArgs& A = ph ? a1 : a0;
                const CUtensorMap* tm_tok = ph ? &tm_tok1 : &tm_tok0;
                const CUtensorMap* tm_w = ph ? &tm_w1 : &tm_w0;
                const int m = MODE == 2 ? ph : MODE;
                const int e = info >> 3, nsub = info & 7, KB = A.K / 128;
                const Unit cur = un;
                if (MODE == 2 && ph == 1) {
                    // the gate_up rows of this block half (written by other CTAs' generic stores) before the TMA
                    // and bulk copies read them
                    if (!wait_counter_gpu(sched + 1 + 2 * cur.mb + cur.hp, a0.n_tiles, abort)) { ok = false; break; }
                    fence_proxy_async_global();
                }
                const uint32_t par = (uint32_t)local & 1u, use = (uint32_t)local >> 1;
                ++local;
                // the block's activation scales [128 slots][KB], contiguous in global memory
                const uint32_t sa_bytes = (uint32_t)(128 * KB * 4);
                if (!mbar_wait(smem_u32(&tail->saempty[par]), (use & 1u) ^ 1u, abort)) { ok = false; break; }
                mbar_arrive_expect_tx(smem_u32(&tail->safull[par]), sa_bytes);
                bulk_copy_g2s(smem_u32(sa_tab) + par * (128 * kb_max * 4), A.a_scale + (size_t)cur.mb * 128 * KB,
                              sa_bytes, smem_u32(&tail->safull[par]));
                ++sa_issued[par];
                const int wrow = e * A.n_total + cur.nt * (m == 0 ? 128 : 256);
                const uint32_t bytes = (uint32_t)(2 * kWBytes + nsub * 32 * 128);
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(smem_u32(&tail->empty[stage]), phase ^ 1u, abort)) { ok = false; break; }
                    const uint32_t dst = sbase + stage * kStageBytes;
                    const uint32_t fb = smem_u32(&tail->full[stage]);
                    mbar_arrive_expect_tx(fb, bytes);
                    tma_load_2d(dst, tm_w, fb, kb * 128, wrow);
                    tma_load_2d(dst + kWBytes, tm_w, fb, kb * 128, wrow + second_tile_rows(m, A.inter));
                    const uint32_t tok = dst + 2 * kWBytes;
                    for (int s = 0; s < nsub; ++s)
                        tma_load_2d(tok + s * 4096, tm_tok, fb, kb * 128, cur.mb * 128 + cur.hp * 64 + 32 * s);
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                    if (kb == 0) {  // the next unit, resolved while this one streams
                        g = g_next;
                        if (g < sp.total) {
                            un = sp.resolve(tail->second, g, ph);
                            info = half_info(ph ? a1 : a0, un.mb, un.hp);
                        }
                    }
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
        } else if (warp == 2) {
            // ---------------------------------------------------------------- unit records (warp 2)
            for (int nq = 0, local = 0;; ++nq) {
                const uint32_t qs = (uint32_t)nq % kQueue, qu = (uint32_t)nq / kQueue;
                if (!mbar_wait(smem_u32(&tail->qfull[qs]), qu & 1u, abort)) break;
                const int2 ref = tail->queue[qs];
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tail->qempty[qs]));
                if (ref.x < 0) break;
                int ph = 0;
                const Unit un = sp.resolve(tail->second, ref.x, ph);
                const SmallGemmArgs& A = ph ? a1 : a0;
                const int m = MODE == 2 ? ph : MODE, e = ref.y >> 3;
                const uint32_t par = (uint32_t)local & 1u, use = (uint32_t)local >> 1;
                ++local;
                if (!mbar_wait(smem_u32(&tail->uempty[par]), (use & 1u) ^ 1u, abort)) break;
                UnitRec& R = tail->urec[par];
                const int KB = A.K / 128, nb_total = A.n_total / 128;
                const float* bs = A.b_scale + (size_t)e * nb_total * KB;
                const int r0 = m == 0 ? un.nt : 2 * un.nt;  // the two tiles' 128-row scale blocks
                const int r1 = r0 + second_tile_rows(m, A.inter) / 128;
                for (int j = lane; j < KB; j += 32) {
                    R.bg[j] = bs[(size_t)r0 * KB + j];
                    R.bu[j] = bs[(size_t)r1 * KB + j];
                }
                if (m == 1) {
                    for (int j = lane; j < 64; j += 32) {
                        const int f = A.sorted_ids[un.mb * 128 + un.hp * 64 + j];
                        R.fl[j] = f;
                        R.wl[j] = f < A.n_valid ? A.topk_w[f] : 0.0f;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tail->ufull[par]));
            }
        } else if (warp == 1 && lane == 0) {
            // ---------------------------------------------------------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0, it = 0;
            bool ok = true;
            for (int nq = 0; ok; ++nq) {
                const uint32_t qs = (uint32_t)nq % kQueue, qu = (uint32_t)nq / kQueue;
                if (!mbar_wait(smem_u32(&tail->qfull[qs]), qu & 1u, abort)) break;
                const int2 ref = tail->queue[qs];
                mbar_arrive(smem_u32(&tail->qempty[qs]));
                if (ref.x < 0) break;
                int ph = 0;
                sp.resolve(tail->second, ref.x, ph);
                const int m = MODE == 2 ? ph : MODE;
                const int nsub = ref.y & 7, KB = (ph ? a1.K : a0.K) / 128;
                const uint32_t idesc = idesc_f32acc(0 /*e4m3*/, 0 /*e4m3*/, 128, 32u * (uint32_t)nsub);
                const int spk = slots_per_kblock(nsub);
                for (int kb = 0; kb < KB && ok; ++kb) {
                    uint32_t sl[2] = {0, 0};
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (h >= spk) break;
                        const uint32_t slot = it % kSlots, use = it / kSlots;
                        ++it;
                        if (!mbar_wait(smem_u32(&tail->tempty[slot]), (use & 1u) ^ 1u, abort)) { ok = false; break; }
                        sl[h] = slot;
                    }
                    if (!ok) break;
                    if (!mbar_wait(smem_u32(&tail->full[stage]), phase, abort)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t base = sbase + stage * kStageBytes;
                    const uint64_t dwg = desc_kmajor_sw128(base);
                    const uint64_t dwu = desc_kmajor_sw128(base + kWBytes);
                    const uint64_t dt = desc_kmajor_sw128(base + 2 * kWBytes);
                    const uint32_t dg = tmem_base + sl[0] * kSlotCols;
                    const uint32_t du = spk == 1 ? dg + 32 : tmem_base + sl[1] * kSlotCols;
                    // each accumulator's four K steps back to back: a chain on one accumulator issues at ~107
                    // cycles per MMA, alternating accumulators at every instruction at ~196
#pragma unroll
                    for (int k = 0; k < 4; ++k)  // 32 e4m3 (32 bytes) of K per instruction
                        mma_f8f6f4(dg, dwg + 2 * k, dt + 2 * k, idesc, k > 0 ? 1u : 0u);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f8f6f4(du, dwu + 2 * k, dt + 2 * k, idesc, k > 0 ? 1u : 0u);
                    mma_commit(smem_u32(&tail->empty[stage]));
                    mma_commit(smem_u32(&tail->tfull[sl[0]]));
                    if (spk == 2) mma_commit(smem_u32(&tail->tfull[sl[1]]));
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                }
            }
            mma_commit(smem_u32(&tail->drain));
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(smem_u32(&tail->drain), 0) && globaltimer() - t0 < PM_WAIT_TIMEOUT_NS) {
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
        // ------------------------------------------------------------------ promotion + epilogue
        Ring ring;
        for (int nq = 0;; ++nq) {
            const uint32_t qs = (uint32_t)nq % kQueue, qu = (uint32_t)nq / kQueue;
            if (!mbar_wait(smem_u32(&tail->qfull[qs]), qu & 1u, abort)) break;
            const int2 ref = tail->queue[qs];
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tail->qempty[qs]));
            if (ref.x < 0) break;
            int ph = 0;
            const Unit un = sp.resolve(tail->second, ref.x, ph);
            const int nsub = ref.y & 7, e = ref.y >> 3;
            bool ok;
            if constexpr (MODE == 2) {
                if (ph == 0)
                    ok = nsub == 1 ? run_unit<0, 1>(a0, tail, sa_tab, kb_max, un, e, ring, abort, tmem_base)
                                   : run_unit<0, 2>(a0, tail, sa_tab, kb_max, un, e, ring, abort, tmem_base);
                else
                    ok = nsub == 1 ? run_unit<1, 1>(a1, tail, sa_tab, kb_max, un, e, ring, abort, tmem_base)
                                   : run_unit<1, 2>(a1, tail, sa_tab, kb_max, un, e, ring, abort, tmem_base);
            } else {
                ok = nsub == 1 ? run_unit<MODE, 1>(a0, tail, sa_tab, kb_max, un, e, ring, abort, tmem_base)
                               : run_unit<MODE, 2>(a0, tail, sa_tab, kb_max, un, e, ring, abort, tmem_base);
            }
            if (!ok) break;
            ++ring.local;
            if (MODE == 2 && ph == 0) {
                // this block half's rows of this column tile are stored: count them for the down units
                const uint32_t db = smem_u32(&tail->dbar[ring.n0 & 1]);
                mbar_arrive(db);
                int go = 1;
                if (warp == kEpiWarp0) {
                    if (lane == 0) {
                        go = mbar_wait(db, ((uint32_t)ring.n0 >> 1) & 1u, abort) ? 1 : 0;
                        if (go) {
                            __threadfence();
                            atomicAdd(sched + 1 + 2 * un.mb + un.hp, 1);
                        }
                    }
                    go = __shfl_sync(0xffffffffu, go, 0);
                }
                if (!go) break;
            }
            if ((MODE == 2 ? ph : MODE) == 0) ++ring.n0;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
    if (threadIdx.x == 0 && tail->abort && a0.err != nullptr) atomicExch(a0.err, 1);
}

template <int MODE>
size_t small_smem(int stages, int kb_max) {
    return 1024 + (size_t)stages * stage_bytes<MODE>() + (size_t)2 * 128 * kb_max * 4 + sizeof(SmallTail);
}

template <int MODE>
cudaError_t launch_small(const CUtensorMap& tok0, const CUtensorMap& w0, const CUtensorMap& tok1,
                         const CUtensorMap& w1, SmallGemmArgs a0, const SmallGemmArgs& a1, int32_t* sched, int grid,
                         int kb_max, cudaStream_t s) {
    const size_t limit = 227 * 1024;
    int stages = kMaxStages;
    while (stages > 2 && small_smem<MODE>(stages, kb_max) > limit) --stages;
    a0.stages = stages;
    const size_t smem = small_smem<MODE>(stages, kb_max);
    static std::atomic<bool> configured[64];  // zero-initialised: false
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
        PM_TRY(cudaFuncSetAttribute(moe_gemm_fp8_small_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)limit));
        if (dev < 64) configured[dev].store(true, std::memory_order_release);
    }
    PM_TRY(launch_pdl(moe_gemm_fp8_small_kernel<MODE>, dim3(grid), dim3(kThreads), smem, s, tok0, w0, tok1, w1, a0,
                      a1, sched));
    return cudaGetLastError();
}

}  // namespace

bool gemm_fp8_small_fits(int mode, int K) {
    const int KB = K / 128;
    if (K % 128 != 0 || KB > 64) return false;
    const size_t limit = 227 * 1024;
    return (mode == 0 ? small_smem<0>(2, KB) : small_smem<1>(2, KB)) <= limit;
}

bool gemm_fp8_small_fused_fits(int H, int I) {
    if (H % 128 != 0 || I % 128 != 0 || H / 128 > 64 || I / 128 > 64) return false;
    return small_smem<2>(2, (H > I ? H : I) / 128) <= 227 * 1024;
}

cudaError_t launch_gemm_fp8_small(int mode, const CUtensorMap& tm_tok, const CUtensorMap& tm_w,
                                  const SmallGemmArgs& args, int num_sms, cudaStream_t s) {
    if (!gemm_fp8_small_fits(mode, args.K) || args.max_units / args.n_tiles > kMaxBlocks) return cudaErrorInvalidValue;
    const int units = 2 * args.max_units;  // two halves per block and column tile
    const int grid = units < num_sms ? (units > 0 ? units : 1) : num_sms;
    return mode == 0 ? launch_small<0>(tm_tok, tm_w, tm_tok, tm_w, args, args, nullptr, grid, args.K / 128, s)
                     : launch_small<1>(tm_tok, tm_w, tm_tok, tm_w, args, args, nullptr, grid, args.K / 128, s);
}

cudaError_t launch_gemm_fp8_small_fused(const CUtensorMap& tm_tok1, const CUtensorMap& tm_w1,
                                        const CUtensorMap& tm_tok2, const CUtensorMap& tm_w2,
                                        const SmallGemmArgs& gate_up, const SmallGemmArgs& down, int32_t* sched,
                                        int num_sms, cudaStream_t s) {
    if (!gemm_fp8_small_fused_fits(gate_up.K, down.K) || sched == nullptr ||
        gate_up.max_units / gate_up.n_tiles > kMaxBlocks)
        return cudaErrorInvalidValue;
    const int units = 2 * (gate_up.max_units > down.max_units ? gate_up.max_units : down.max_units);
    const int grid = units < num_sms ? (units > 0 ? units : 1) : num_sms;
    const int kb_max = (gate_up.K > down.K ? gate_up.K : down.K) / 128;
    return launch_small<2>(tm_tok1, tm_w1, tm_tok2, tm_w2, gate_up, down, sched, grid, kb_max, s);
}

}  // namespace pm
