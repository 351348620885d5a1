// Blackwell (sm_100a) building blocks: TMA tile loads, mbarriers with bounded
// waits, tensor memory, and tcgen05 TF32 MMAs with shared-memory descriptors.
//
// Encodings follow the PTX ISA for sm_100a: the shared-memory matrix
// descriptor (start >> 4 in bits 0-13, leading byte offset >> 4 in 16-29,
// stride byte offset >> 4 in 32-45, version 1 in 46-47, swizzle mode in
// 61-63) and the instruction descriptor of kind::tf32 (F32 accumulator in bits
// 4-5, TF32 A/B formats in 7-9 and 10-12, K- or MN-major flags in bits 15/16,
// N >> 3 in 17-22, M >> 4 in 24-28).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cpde {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// --- mbarriers -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Waits for the phase with the given parity to complete, giving up after
// `limit` clock cycles. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long limit) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - start > limit) return false;
    return true;
}

// As mbar_wait, but also gives up as soon as *abort becomes nonzero (another
// role of the CTA timed out); a timeout here raises *abort itself.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, long long limit,
                                                   volatile int* abort) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (clock64() - start > limit) {
            *abort = 1;
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// --- TMA ---------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
// A hint that brings the box a later tma_load_2d of the same map and
// coordinates will read into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// --- per-thread asynchronous copies (global -> shared, 4 bytes) -------------------
__device__ __forceinline__ void copy_async4(float* dst, const float* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void copy_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// waits until at most PENDING of this thread's committed groups are in flight
template <int PENDING>
__device__ __forceinline__ void copy_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(PENDING) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// --- tensor memory -------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(columns)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x N consecutive 32-bit columns per warp; thread i gets lane base+i.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld1(uint32_t taddr, float& v) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
    v = __uint_as_float(r);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 8 consecutive 32-bit columns from registers; thread i writes lane base+i.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                 "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// After tmem_wait_ld: marks the registers of v as written here, so that no use
// of them can be scheduled above the wait (the loads' asm statements already
// name them as outputs).
template <int COUNT>
__device__ __forceinline__ void tmem_landed(float (&v)[COUNT]) {
#pragma unroll
    for (int i = 0; i < COUNT; ++i) asm volatile("" : "+f"(v[i]));
}

// Issues the loads of columns [col, col + COUNT) of this thread's lane into v
// (COUNT <= 64); v is valid after tmem_wait_ld() and tmem_landed(v).
template <int COUNT>
__device__ __forceinline__ void tmem_load(uint32_t taddr, float (&v)[COUNT]) {
    int c = 0;
#pragma unroll
    for (; c + 16 <= COUNT; c += 16) {
        float t[16];
        tmem_ld16(taddr + c, t);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[c + i] = t[i];
    }
    if (COUNT - c >= 8) {
        float t[8];
        tmem_ld8(taddr + c, t);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c + i] = t[i];
        c += 8;
    }
    if (COUNT - c >= 4) {
        float t[4];
        tmem_ld4(taddr + c, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[c + i] = t[i];
        c += 4;
    }
#pragma unroll
    for (; c < COUNT; ++c) tmem_ld1(taddr + c, v[c]);
}

// Reads columns [col, col + COUNT) of this thread's lane into v (COUNT <= 64).
template <int COUNT>
__device__ __forceinline__ void tmem_read(uint32_t taddr, float (&v)[COUNT]) {
    tmem_load<COUNT>(taddr, v);
    tmem_wait_ld();
    tmem_landed(v);
}

// --- MMA ---------------------------------------------------------------------
// K-major operand tile written by TMA with 128-byte swizzle: rows of 128 bytes
// (32 fp32 along K), 8-row swizzle atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
    d |= uint64_t(1u) << 16;             // leading byte offset (unused for swizzled K-major)
    d |= uint64_t(1024u >> 4) << 32;     // stride byte offset: next 8-row group
    d |= uint64_t(1u) << 46;             // descriptor version
    d |= uint64_t(2u) << 61;             // 128-byte swizzle
    return d;
}

// MN-major TF32 operand in the 128-byte swizzle with 32-byte atoms (layout
// type 1): rows of 128 bytes hold 32 consecutive M (or N) elements of one K
// index, the 32-byte chunk index of a row xor (row % 4); 4-row groups 512
// bytes apart along K (stride byte offset), 32-element MN blocks `mn_stride`
// bytes apart (leading byte offset).
__device__ __forceinline__ uint64_t desc_mn32_sw128(uint32_t smem_addr, uint32_t mn_stride) {
    uint64_t d = 0;
    d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
    d |= uint64_t((mn_stride >> 4) & 0x3FFFu) << 16;
    d |= uint64_t(512u >> 4) << 32;
    d |= uint64_t(1u) << 46;
    d |= uint64_t(1u) << 61;
    return d;
}

__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    uint32_t mask = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(mask)
        : "memory");
}
// Same with A read from tensor memory (K-major: lane = row, one column per K element).
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    uint32_t mask = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(mask)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// TF32 split: hi keeps the top 10 explicit mantissa bits (round half away),
// lo = x - hi exactly, then rounded the same way for the tensor core.
__device__ __forceinline__ float tf32_round(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

}  // namespace tc
}  // namespace cpde
