// lc_sm100.cuh -- device helpers shared by the sm_100a kernels (not installed):
// bounded mbarrier waits, TMA tensor copies, shared-memory loads, packed f32x2
// arithmetic, the activation scale and the f16 scale decode.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "lc_internal.cuh"

// The driver's cuTensorMapEncodeTiled, resolved once (lc_proj.cu).
int lc_tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000 *out);

namespace {

// Power-of-two activation scale: x * 2^e has max|x * 2^e| in [2^13, 2^14), so
// its f16 hi / lo split cannot overflow (f16 max 65504) however large the
// activations grow; outputs are multiplied by 2^-e.  Both steps are exact.
__device__ __forceinline__ void act_scale(float maxabs, float &s, float &inv) {
    int e = 0;
    if (maxabs > 0.f && maxabs < INFINITY) {
        int x;
        frexpf(maxabs, &x);  // maxabs = f * 2^x, f in [0.5, 1)
        e = min(max(14 - x, -100), 100);
    }
    s = ldexpf(1.f, e);
    inv = ldexpf(1.f, -e);
}

// (d, dmin) of a header word -> two floats.  The reference rule for subnormal
// halves (2^-14 * (1 + m/1024)) is the half with its exponent field set to 1,
// applied branch-free to both halves: per half, bit 10 is OR-ed in when the
// exponent is 0 and the mantissa is not (ref = 0x04000400 mask, IEEE = 0).
__device__ __forceinline__ float2 scales2_f32(uint32_t h2, uint32_t ref_mask) {
    const uint32_t man = h2 & 0x03FF03FFu, ex = h2 & 0x7C007C00u;
    const uint32_t m_nz = (man + 0x03FF03FFu) & 0x04000400u;     // bit 10: mantissa != 0
    const uint32_t e_nz = ((ex + 0x7C007C00u) & 0x80008000u) >> 5;  // bit 10: exponent != 0
    const uint32_t fixed = h2 | (m_nz & ~e_nz & ref_mask);
    return __half22float2(lc_u32_as_h2(fixed));
}

// ---------------------------------------------------------------------------
// Bulk asynchronous copies into shared memory (cp.async.bulk, completion on an
// mbarrier).  Every wait is bounded: after kWaitSpins polls the waiter records
// LC_DEV_WAIT_TIMEOUT in the context's status word and gives up.

constexpr uint32_t kWaitSpins = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase of `bar` with the given parity; false if the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_test(bar, parity)) return true;
    for (uint32_t i = 0; i < kWaitSpins; ++i)
        if (mbar_test(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
    return p;
}

// 16-byte shared load into `v` when `pred`, else `v` keeps its value (the
// lanes that skip it generate no shared-memory traffic).
__device__ __forceinline__ void lds128_if(bool pred, uint4 &v, const void *p) {
    asm volatile(
        "{\n .reg .pred q;\n setp.ne.u32 q, %4, 0;\n @q ld.shared.v4.u32 {%0,%1,%2,%3}, [%5];\n}\n"
        : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
        : "r"((uint32_t)pred), "r"(smem_addr(p)));
}

__device__ __forceinline__ uint4 lds128(const void *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_addr(p)));
    return v;
}

// 2D tensor copy global -> shared (TMA, tile mode) of the box at element
// coordinates (x, y) of `tm`, completing on `bar`; evict-first in L2.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;\n" ::"r"(smem_addr(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}

// Lane 0 of the warp arms `bar` for one 16-row unit and issues its copy;
// predicated rather than branched, so the warp stays converged.
__device__ __forceinline__ void tma_unit_lane0(int lane, void *dst, const CUtensorMap *tm, int x, int y,
                                               uint64_t *bar, uint64_t pol, uint32_t bytes) {
    asm volatile(
        "{\n .reg .pred p;\n setp.eq.s32 p, %0, 0;\n"
        " @p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n"
        " @p cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%3], [%4, {%5, %6}], [%1], %7;\n}\n" ::"r"(lane),
        "r"(smem_addr(bar)), "r"(bytes), "r"(smem_addr(dst)), "l"(tm), "r"(x), "r"(y), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *tm) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(tm) : "memory");
}

// Named barrier over the first `nthreads` threads of the CTA (id 1; id 0 is
// __syncthreads).
__device__ __forceinline__ void named_barrier_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;\n" ::"r"(nthreads) : "memory");
}

// Packed f32x2 arithmetic (sm_100): two fp32 lanes per instruction.
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}\n"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mov.b64 rc, {%6, %7};\n fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}\n"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ uint32_t lds32(const void *p) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(smem_addr(p)));
    return v;
}

}  // namespace
