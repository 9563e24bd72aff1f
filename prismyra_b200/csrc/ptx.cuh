// Thin inline-PTX helpers for sm_100a: shared-memory barriers, TMA tile loads and the tcgen05 tensor-core
// instructions (TMEM allocation, MMA issue, commit, TMEM -> register loads).  Every wait here is bounded: a
// wait that does not complete within PM_WAIT_TIMEOUT_NS sets the kernel's abort flag and returns false, so a
// kernel can unwind (free TMEM, return) instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "moe_internal.h"

#ifndef PM_WAIT_TIMEOUT_NS
#define PM_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: a healthy wait in these kernels lasts microseconds
#endif

namespace pm {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and raises *abort) on timeout, or
// immediately once another thread of the CTA has raised *abort.
// Programmatic dependent launch: pdl_wait() returns once the previous kernel of the stream has completed and its
// memory is visible (a no-op when the kernel was launched without the programmatic-serialisation attribute);
// pdl_trigger() lets the next kernel be scheduled (its own pdl_wait still waits for this kernel to complete).
// Every kernel of the forward chain calls both before its first global memory access, so no kernel reads or
// writes global memory while its predecessor runs, and completion stays transitive along the chain.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer() - t0 > PM_WAIT_TIMEOUT_NS) {
            *abort = 1;
            return false;
        }
    }
}

// A counter in global memory that other CTAs of this grid raise (atomically, after a fence): poll it with
// GPU-scope acquire loads until it reaches `target`.  Returns false (and raises *abort) on timeout, or once another
// thread of the CTA has raised *abort.
__device__ __forceinline__ bool wait_counter_gpu(const int* p, int target, volatile int* abort) {
    const uint64_t t0 = globaltimer();
    while (true) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v >= target) return true;
        if (*abort) return false;
        if (globaltimer() - t0 > PM_WAIT_TIMEOUT_NS) {
            *abort = 1;
            return false;
        }
    }
}

// Orders this thread's earlier generic-proxy memory accesses (such as the acquire above) before its later
// async-proxy (TMA, bulk copy) accesses of global memory.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ------------------------------------------------------------------------------------------- TMA
// 2-D tiled bulk tensor load into this CTA's shared memory, completing on an mbarrier (transaction bytes).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// One box of a tensor map into L2 (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_l2(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------------------------------- tcgen05
// TMEM allocation: executed by one full warp; the allocated base address is written to shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte swizzle: rows of
// 128 bytes, 8-row atoms of 1024 bytes laid out contiguously (stride byte offset 1024).  Bits: start address
// >> 4 at [0,14), leading byte offset >> 4 at [16,30) (unused for swizzled K-major; 1), stride byte offset
// >> 4 at [32,46), descriptor version 1 at [46,48), swizzle mode 2 (128B) at [61,64).
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor, kind::f8f6f4 / kind::f16: D format at [4,6) (1 = f32), A format at [7,10),
// B format at [10,13), A/B major at bits 15/16 (0 = K-major), N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_f32acc(uint32_t a_fmt, uint32_t b_fmt, uint32_t M, uint32_t N) {
    return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one CTA, FP8/FP6/FP4 operands with f32 accumulation.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T with 16-bit (bf16 / f16) operands.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive (once) on an mbarrier when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM -> 32 registers per thread (thread i reads lane base+i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// 16 consecutive TMEM columns of this warp's 32 lanes (one per thread).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// Contiguous global -> shared copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) completing on an
// mbarrier's transaction count (the untiled bulk copy, this CTA only).
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :
                 : "r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Named barrier among a subset of the CTA's warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------------------------------- numerics
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// silu of a pair through the identity g * sigmoid(g) = h + h * tanh(h), h = g / 2: one hardware tanh (the PTX
// tanh.approx.f32 instruction, maximum relative error 2^-11) per value instead of an exponential and a reciprocal,
// halving the transcendental-unit work of the gate_up epilogue.  The callers round the result to bf16 (8
// significant bits) right after.
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float2 silu2(float2 g) {
    const float2 h = __fmul2_rn(g, make_float2(0.5f, 0.5f));
    return __ffma2_rn(h, make_float2(tanh_approx(h.x), tanh_approx(h.y)), h);
}

// How an activation group's e4m3 scale is formed from its maximum magnitude amax (vLLM's per_token_group_quant_fp8,
// vllm/model_executor/layers/quantization/utils/fp8_utils.py:510-640):
//   kScaleDiv   the correctly rounded quotient max(amax, 1e-10) / 448 -- what vLLM's compiled CUDA quantiser, the
//               op the reference's fused_experts runs on a GPU, computes (matched bit for bit on B200);
//   kScaleRcp   max(amax, 1e-10) * fl(1/448) -- vLLM's Triton kernel (fp8_utils.py:143-144), 1 ulp apart from the
//               quotient for about half of all values;
//   kScaleUe8m0 the quotient rounded up to a power of two, 2^ceil(log2(s)) (fp8_utils.py:145), vLLM's mode when
//               DeepGEMM runs with E8M0 scales.  The power of two is taken from the float's own bits: s is a positive
//               normal number (at least 1e-10/448), so ceil(log2(s)) is its exponent, plus one unless its
//               significand is exactly 1.
__device__ __forceinline__ float e4m3_group_scale(float amax, int rule) {
    const float a = fmaxf(amax, 1e-10f);
    if (rule == kScaleRcp) return a * (1.0f / 448.0f);
    const float s = __fdiv_rn(a, 448.0f);
    if (rule != kScaleUe8m0) return s;
    const uint32_t u = __float_as_uint(s);
    return __uint_as_float(((u >> 23) + ((u & 0x7FFFFFu) != 0u)) << 23);
}

// The correctly rounded quotients y / s of a pair by one divisor s, given r = RN(1/s) and ns = -s: the reciprocal
// product q0 = RN(y * r) followed by one correction step, q = RN(q0 + RN(y - q0 * s) * r), the residual being exact
// in an FMA (P. Markstein, "Computation of elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990).  Used where every quotient of a group shares its divisor and must equal the IEEE quotient:
// the requantisation reproduces vLLM's compiled quantiser code for code, ties to even on e4m3 midpoints included.
__device__ __forceinline__ float2 quot2(float2 y, float2 r, float2 ns) {
    const float2 q0 = __fmul2_rn(y, r);
    const float2 e = __ffma2_rn(q0, ns, y);
    return __ffma2_rn(e, r, q0);
}

// Two values rounded to bf16 with one packed conversion (cvt.rn.bf16x2.f32) and widened back.
__device__ __forceinline__ float2 bf16x2_round(float a, float b) {
    return __bfloat1622float2(__floats2bfloat162_rn(a, b));
}

// Two fp32 -> two e4m3 bytes (low byte = a), round to nearest even, saturating.
__device__ __forceinline__ uint16_t e4m3x2(float a, float b) {
    return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}

}  // namespace pm
