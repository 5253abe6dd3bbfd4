// Blackwell (sm_100a) tensor-core primitives: tcgen05 MMA with TMEM accumulators.
//
// Shared-memory operands use the canonical no-swizzle ("interleaved") layout of
// 8 x 16-byte core matrices.  A [rows x cols] fp16 matrix is stored "blocked":
//   byte(r, c) = ((c / 8) * (rows / 8) + r / 8) * 128 + (r % 8) * 16 + (c % 8) * 2
// Read with cols as K (K-major operand): LBO = (rows / 8) * 128, SBO = 128,
// K-step s starts 2 * s * LBO bytes further.  Read with cols as M/N and rows as
// K (MN-major operand): LBO = 128, SBO = (rows / 8) * 128, K-step s starts
// 256 * s bytes further.  Descriptor and instruction-descriptor bit layouts
// follow the PTX ISA (tcgen05 matrix / instruction descriptors).
#pragma once
#include "common.cuh"

namespace odie {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of element (r, c) of a blocked [rows x cols] fp16 matrix.
__host__ __device__ constexpr int blocked(int rows, int r, int c) {
    return ((c >> 3) * (rows >> 3) + (r >> 3)) * 128 + (r & 7) * 16 + (c & 7) * 2;
}

// Shared-memory matrix descriptor, no swizzle, version 1 (Blackwell).
__device__ __forceinline__ uint64_t sdesc(uint32_t address, uint32_t lbo, uint32_t sbo) {
    return uint64_t((address >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
// K-major view of a blocked [rows x cols] matrix (K along cols), K-step s.
__device__ __forceinline__ uint64_t kmajor(uint32_t base, int rows, int s) {
    const uint32_t lbo = uint32_t(rows >> 3) * 128u;
    return sdesc(base + 2u * uint32_t(s) * lbo, lbo, 128u);
}
// MN-major view of a blocked [rows x cols] matrix (M/N along cols, K along rows), K-step s.
__device__ __forceinline__ uint64_t mnmajor(uint32_t base, int rows, int s) {
    return sdesc(base + 256u * uint32_t(s), 128u, uint32_t(rows >> 3) * 128u);
}

// Instruction descriptor of kind::f16: fp16 A and B, fp32 D.
__host__ __device__ constexpr uint32_t idesc(int M, int N, int a_mn_major, int b_mn_major) {
    return (1u << 4) | (uint32_t(a_mn_major) << 15) | (uint32_t(b_mn_major) << 16) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

// D[tmem] (+)= A * B, issued by one thread.
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
    const uint32_t mask = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(accumulate), "r"(mask), "r"(mask), "r"(mask), "r"(mask));
}

// Arrive on an mbarrier once every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_bar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }

// Bounded wait for the phase with the given parity; false when the limit ran out.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, uint32_t limit) {
    const uint32_t address = smem_u32(bar);
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(address), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// TMEM allocation by one full warp; the base address is written to shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst)),
                 "r"(columns)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(base), "r"(columns) : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (32x32b shape, warp-collective).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Load 32 consecutive fp32 columns of this thread's TMEM lane: one load and its wait in one
// statement, so nothing reads the registers before they land (32x32b shape, warp-collective).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive fp32 columns of this thread's TMEM lane (32x32b shape, warp-collective).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

}  // namespace tc
}  // namespace odie
