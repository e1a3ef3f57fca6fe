// umma.cuh -- sm_100a tensor-core (tcgen05) building blocks: tensor-memory
// allocation, shared-memory matrix descriptors, instruction descriptors, MMA
// issue and commit, tensor-memory loads, and TMA tile stores.
//
// Descriptor formats (PTX ISA 8.7, tcgen05 "shared memory descriptor" and
// "instruction descriptor"; the same bit layout as CUTLASS's
// cute/arch/mma_sm100_desc.hpp):
//   shared-memory descriptor (64 bit): start address >> 4 in [0,14), leading
//   byte offset >> 4 in [16,30), stride byte offset >> 4 in [32,46), version 1
//   in [46,48), base offset in [49,52), layout type in [61,64) (2 = 128-byte
//   swizzle).
//   instruction descriptor (32 bit, kind::f16): D format in [4,6) (1 = F32),
//   A format in [7,10) and B format in [10,13) (1 = BF16), A major in bit 15
//   and B major in bit 16 (0 = K-major, 1 = MN-major), N >> 3 in [17,23),
//   M >> 4 in [24,29).
// All operand tiles here use the 128-byte swizzle: rows of 128 bytes, 8-row
// atoms of 1024 bytes (1024-byte aligned), 16-byte chunk j of row r stored at
// chunk j ^ (r % 8) -- the layout a TMA load with CU_TENSOR_MAP_SWIZZLE_128B
// writes.
#pragma once

#include <stdint.h>

#include "ptx.cuh"

namespace need {
namespace umma {

// --------------------------------------------------------------- descriptors
enum Major : uint32_t { K_MAJOR = 0, MN_MAJOR = 1 };

// 128-byte-swizzled operand at shared address `saddr` (bytes).  K-major: rows
// of the M/N dimension, 8-row groups `sbo` bytes apart (lbo unused).  MN-major:
// rows of the K dimension, 8-row groups `sbo` bytes apart, 64-element groups
// of M/N `lbo` bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;  // descriptor version for sm_100
    d |= 2ull << 61;  // 128-byte swizzle
    return d;
}

// bf16 x bf16 -> fp32, M x N, operand majors
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, uint32_t a_major, uint32_t b_major) {
    return (1u << 4)                                   // D: F32
           | (1u << 7) | (1u << 10)                    // A, B: BF16
           | (a_major << 15) | (b_major << 16)         // operand majors
           | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// --------------------------------------------------------------- tensor memory
// Allocates `ncols` columns (a power of two >= 32) for the CTA; one warp calls
// it and the base address lands in shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]; one thread issues it.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}
// The mbarrier receives one arrival when every MMA this thread issued before
// has completed (and its shared-memory operands have been read).
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// 32 consecutive fp32 columns of this thread's lane (warp w reads lanes
// 32w..32w+31: taddr carries the lane in its high half).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// the store counterpart: 32 fp32 columns into this thread's lane
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
        "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]),
        "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]),
        "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// --------------------------------------------------------------- TMA stores
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, const void* src, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tm),
        "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of every committed store have been read
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// every committed store has completed
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, int c0, int c1, int c2,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_addr(dst)),
        "l"(tm), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// byte offset of 16-byte chunk `j` of row `r` in a 128-byte-swizzled tile
__host__ __device__ constexpr uint32_t sw128(uint32_t r, uint32_t j) {
    return (r >> 3) * 1024u + (r & 7u) * 128u + ((j ^ (r & 7u)) << 4);
}

}  // namespace umma
}  // namespace need
