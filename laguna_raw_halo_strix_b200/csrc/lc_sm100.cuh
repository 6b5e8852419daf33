// lc_sm100.cuh -- device helpers shared by the sm_100a kernels (not installed):
// bounded mbarrier waits, TMA tensor copies, shared-memory loads, packed f32x2
// arithmetic, the activation scale, the f16 scale decode, tcgen05 descriptors,
// MMAs and tensor-memory access, programmatic dependent launch.
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
    // maxabs = f * 2^x with f in [0.5, 1): x = E - 126 for the biased exponent E of
    // a normal float; a subnormal (E = 0) gives e above 100 either way.
    int e = 0;
    if (maxabs > 0.f && maxabs < INFINITY) e = min(max(140 - (int)(__float_as_uint(maxabs) >> 23), -100), 100);
    s = __uint_as_float((uint32_t)(e + 127) << 23);
    inv = __uint_as_float((uint32_t)(127 - e) << 23);
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

// ---- tcgen05 ---------------------------------------------------------------

// Shared-memory matrix descriptor, K-major with 128-byte swizzle: rows of
// 128 bytes in groups of 8 (1024 bytes, SBO), 16-byte chunks XOR-swizzled by
// the row within the group; LBO unused (1); version 1; layout type 2.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;               // LBO (16 B; unused for this layout)
    d |= (uint64_t)(1024u >> 4) << 32;     // SBO: 8 rows x 128 B
    d |= (uint64_t)1u << 46;               // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;               // SWIZZLE_128B
    return d;
}

// Shared-memory matrix descriptor, K-major without swizzle, for a K = 16
// operand in core matrices of 8 rows x 16 bytes: the two K groups 128 bytes
// apart (LBO), 8-row groups 256 bytes apart (SBO).
__device__ __forceinline__ uint64_t umma_desc_core16(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)(128u >> 4) << 16;
    d |= (uint64_t)(256u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}

// Instruction descriptor of kind::f16: D f32, A and B f16, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D (TMEM) (+)= A (shared memory) * B (shared memory)^T.
__device__ __forceinline__ void umma_f16_ss(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (TMEM) (+)= A (TMEM: row i in lane i, two f16 per column) * B (shared memory)^T.
__device__ __forceinline__ void umma_f16_ts(uint32_t dtmem, uint32_t atmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(dtmem),
        "r"(atmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this thread's lane -> registers
// (complete after tmem_ld_wait).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// The values of every tcgen05.ld issued so far are in their registers.
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// Ties registers written by tcgen05.ld to a point after tmem_ld_wait(): their
// uses depend on these (ordered) volatile statements, so none moves above the
// wait.
template <int N>
__device__ __forceinline__ void tmem_regs_ready(float (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N; i++) asm volatile("" : "+f"(v[i])::"memory");
}

// Registers -> 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// Every tcgen05.st this thread issued has written the tensor memory.
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}

// Programmatic dependent launch: the dependent grid may start once every CTA
// of this grid has executed launch_dependents (or exited); griddep_wait blocks
// until the prerequisite grid has completed and its writes are visible (a no-op
// in a grid launched without the attribute).
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// Untiled bulk copy global -> shared (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}

// 16-byte asynchronous copy global -> shared by this thread (cp.async through
// L2 only); completes in the thread's current group.
__device__ __forceinline__ void cp_async16_l2(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
// Close the thread's current group of cp.async copies.
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
// Wait until at most N of the thread's groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Named barrier `id` (1..15) over `nthreads` threads (a multiple of 32); the
// id is an immediate in every form issued.
__device__ __forceinline__ void named_barrier_sync_id(int id, int nthreads) {
    switch (id) {
#define LC_NAMED_BAR(N) \
    case N: asm volatile("bar.sync " #N ", %0;\n" ::"r"(nthreads) : "memory"); break;
        LC_NAMED_BAR(1) LC_NAMED_BAR(2) LC_NAMED_BAR(3) LC_NAMED_BAR(4) LC_NAMED_BAR(5)
        LC_NAMED_BAR(6) LC_NAMED_BAR(7) LC_NAMED_BAR(8) LC_NAMED_BAR(9) LC_NAMED_BAR(10)
        LC_NAMED_BAR(11) LC_NAMED_BAR(12) LC_NAMED_BAR(13) LC_NAMED_BAR(14) LC_NAMED_BAR(15)
#undef LC_NAMED_BAR
        default: break;
    }
}

// Same, without an L2 hint (for data many CTAs read).
__device__ __forceinline__ void bulk_load_plain(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

}  // namespace
