// sm_100a building blocks for the tensor-core (tcgen05) kernels: TMEM allocation,
// shared-memory matrix descriptors, bf16 x bf16 -> f32 MMAs, completion through an
// mbarrier with a bounded wait, and TMEM -> register loads.
//
// Operand layout used everywhere: K-major with the 128-byte swizzle.  For an operand of R
// rows (R a multiple of 8) a "K block" holds 64 bf16 values per row (128 bytes); element
// (r, k) of K block kb lives at byte
//     kb * R * 128 + (r / 8) * 1024 + (r % 8) * 128 + (((k % 64) / 8) ^ (r % 8)) * 16 + (k % 8) * 2
// from a 1024-byte aligned base.  The descriptor of one MMA (K = 16) starts at the K block
// base plus 32 bytes per K step; rows are 128 B apart and 8-row groups 1024 B apart (SBO).
// The fp32 "bf16x3" product a*b ~= ah*bh + ah*bl + al*bh uses the splits
// ah = bf16(a), al = bf16(a - ah) (error ~2^-17 relative per product).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace scx {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of element (r, k) in a K-major SW128 operand of `rows` rows.
__host__ __device__ __forceinline__ uint32_t kmajor_offset(int rows, int r, int k) {
    const int kb = k >> 6, kk = k & 63;
    return static_cast<uint32_t>(kb) * static_cast<uint32_t>(rows) * 128u + static_cast<uint32_t>(r >> 3) * 1024u +
           static_cast<uint32_t>(r & 7) * 128u + static_cast<uint32_t>(((kk >> 3) ^ (r & 7)) << 4) +
           static_cast<uint32_t>((kk & 7) << 1);
}

// Shared-memory matrix descriptor (sm_100 format): start address >> 4 in bits [0,14),
// leading byte offset >> 4 in [16,30) (unused by swizzled K-major layouts, set to 1),
// stride byte offset >> 4 in [32,46), version 1 in [46,48), layout type in [61,64)
// (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor, kind::f16 with bf16 A and B (K-major), f32 accumulator:
// c_format [4,6) = 1 (F32), a_format [7,10) = 1 (BF16), b_format [10,13) = 1 (BF16),
// N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of parity `parity`; gives up after ~2^31 SM cycles (about a second)
// and returns false instead of spinning forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > (1LL << 31)) return false;
    }
    return true;
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
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

// Makes generic-proxy shared-memory writes visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32*(w%4)+lane);
// the load is waited for before returning.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void split2(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(x);
    lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

// 8 floats -> one 16-byte unit of bf16 high parts and one of low parts.
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
    __nv_bfloat16 h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) split2(v[i], h[i], l[i]);
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        hw[i] = static_cast<uint32_t>(__bfloat16_as_ushort(h[2 * i])) |
                (static_cast<uint32_t>(__bfloat16_as_ushort(h[2 * i + 1])) << 16);
        lw[i] = static_cast<uint32_t>(__bfloat16_as_ushort(l[2 * i])) |
                (static_cast<uint32_t>(__bfloat16_as_ushort(l[2 * i + 1])) << 16);
    }
    hi = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    lo = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

}  // namespace tc
}  // namespace scx
