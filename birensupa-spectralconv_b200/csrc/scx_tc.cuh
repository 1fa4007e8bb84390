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

// The thread may sleep in the instruction until the phase completes, for at most about
// 20 us per call (the suspend-time hint, in ns); without the hint it returns after a short
// system-dependent limit and a waiting warp spends issue slots on the retry loop.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
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

// Programmatic dependent launch: wait until the grids this one depends on have completed and
// their writes are visible; allow the next grid in the stream to be scheduled.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

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

// Non-blocking probe of the phase of parity `parity` (no suspension, unlike try_wait).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// 2-D tiled TMA load (no multicast) of the box at (c0 = column, c1 = row) of `tmap` into
// shared memory; completion counted on `bar` in bytes.  c0 * element size must be a
// multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// kind::tf32 variant of mma_bf16 (operands are 32-bit; K = 8 per instruction).
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor, kind::tf32 (K-major A and B), f32 accumulator: a/b format 2 (TF32).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// Byte offset of 32-bit element (r, k) in a K-major SW128 operand of `rows` rows (32
// elements per 128-byte row of a K block).
__host__ __device__ __forceinline__ uint32_t kmajor_offset32(int rows, int r, int k) {
    const int kb = k >> 5, kk = k & 31;
    return static_cast<uint32_t>(kb) * static_cast<uint32_t>(rows) * 128u + static_cast<uint32_t>(r >> 3) * 1024u +
           static_cast<uint32_t>(r & 7) * 128u + static_cast<uint32_t>(((kk >> 2) ^ (r & 7)) << 4) +
           static_cast<uint32_t>((kk & 3) << 2);
}

// x = hi + lo with hi = x with its 13 low mantissa bits cleared (exactly representable in
// tf32, whatever rounding the tensor core applies) and lo = x - hi (exact in fp32).
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    lo = x - hi;
}

// Arms `bar` to expect `bytes` more transaction bytes and arrives once.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> shared (TMA engine, no multicast); completion is counted on `bar`
// in bytes.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier over `n` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Named barrier that also ORs `pred` over the participating threads (uniform result).
__device__ __forceinline__ bool named_any(int id, int n, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}\n"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void split2(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(x);
    lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

// Two floats -> packed bf16 high parts and packed bf16 low parts (x in the low half).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// 4 floats -> 8 bytes of bf16 high parts and 8 bytes of low parts.
__device__ __forceinline__ void split4(const float4& v, uint2& hi, uint2& lo) {
    split_pair(v.x, v.y, hi.x, lo.x);
    split_pair(v.z, v.w, hi.y, lo.y);
}

// 32 consecutive fp32 columns of this thread's TMEM lane, waited for before returning.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 8 floats -> one 16-byte unit of bf16 high parts and one of low parts.
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
    split_pair(v[0], v[1], hi.x, lo.x);
    split_pair(v[2], v[3], hi.y, lo.y);
    split_pair(v[4], v[5], hi.z, lo.z);
    split_pair(v[6], v[7], hi.w, lo.w);
}


// D[tmem] (+)= A[tmem] * B[smem]^T: A (M = 128 rows) is read from tensor memory, one row
// per lane with two bf16 values of consecutive k packed per 32-bit column (the even k in
// the low half), 8 columns per K = 16 step.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Shared-memory descriptor of an MN-major operand with the 128-byte swizzle: element
// (mn, k) of a 16-bit operand lives at
//     (k / 8) * sbo + (mn / 64) * lbo + (k % 8) * 128 + ((((mn % 64) / 8) ^ (k % 8)) * 16) + (mn % 8) * 2
// (lbo = stride of the 64-element MN atoms, sbo = stride of the 8-row K groups).
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction-descriptor bits selecting MN-major A / B operands.
constexpr uint32_t kIdescAMajorMN = 1u << 15;
constexpr uint32_t kIdescBMajorMN = 1u << 16;

// 16 consecutive 32-bit columns of this thread's TMEM lane from registers (not waited for;
// see tmem_wait_st).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Asks the TMA engine to bring `bytes` (a multiple of 16) of global memory into L2.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023);
    return reinterpret_cast<uint8_t*>(a);
}

// Whole CTA: copies a 16-byte aligned table of `bytes` (a multiple of 16) into shared memory.
__device__ __forceinline__ void copy_table(uint8_t* dst, const uint4* src, uint32_t bytes) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (uint32_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = __ldg(src + i);
}


// 8 consecutive 32-bit columns of this thread's TMEM lane from registers (not waited for).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

// 4 consecutive 32-bit columns of this thread's TMEM lane from registers (not waited for).
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane; the registers are valid only after
// tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, float* v) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// 4 / 8 / 16 consecutive fp32 columns of this thread's TMEM lane (valid after tmem_wait_ld).
__device__ __forceinline__ void tmem_ld4_nowait(uint32_t taddr, float* v) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, float* v) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, float* v) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
// N (a multiple of 4, at most 32) consecutive columns through the widest shapes that fit.
template <int N>
__device__ __forceinline__ void tmem_ld_cols_nowait(uint32_t taddr, float* v) {
    static_assert(N % 4 == 0 && N <= 32, "column count");
    if constexpr (N >= 16) {
        tmem_ld16_nowait(taddr, v);
        if constexpr (N > 16) tmem_ld_cols_nowait<N - 16>(taddr + 16, v + 16);
    } else if constexpr (N >= 8) {
        tmem_ld8_nowait(taddr, v);
        if constexpr (N > 8) tmem_ld_cols_nowait<N - 8>(taddr + 8, v + 8);
    } else {
        tmem_ld4_nowait(taddr, v);
    }
}


// 3-D tiled TMA load (no multicast) of the box at (c0, c1, c2) of `tmap` into shared memory;
// completion counted on `bar` in bytes.  c0 * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// GELU(z) = z * Phi(z) = z * (1 + erf(z / sqrt 2)) / 2 without branches.  erfc(x) for x >= 0
// is the rational-times-Gaussian formula 7.1.26 of Abramowitz & Stegun, Handbook of
// Mathematical Functions (1964): erfc(x) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e^(-x^2),
// t = 1 / (1 + p x), with |error| <= 1.5e-7; with the fast reciprocal and exponential the
// GELU's absolute error stays below 1e-6 |z|.  Phi(z) = 1 - erfc(|z| / sqrt 2) / 2 for z >= 0
// and erfc(|z| / sqrt 2) / 2 below.  No data-dependent branch: every lane runs the same
// 17 or so instructions.
__device__ __forceinline__ float gelu_as(float z) {
    const float x = fabsf(z) * 0.70710678118654752f;
    const float t = __fdividef(1.0f, fmaf(0.3275911f, x, 1.0f));
    float p = fmaf(1.061405429f, t, -1.453152027f);
    p = fmaf(p, t, 1.421413741f);
    p = fmaf(p, t, -0.284496736f);
    p = fmaf(p, t, 0.254829592f);
    const float half_erfc = 0.5f * (p * t) * __expf(-x * x);
    return z * (z >= 0.f ? 1.0f - half_erfc : half_erfc);
}

// ---- packed fp32 pairs (sm_100 f32x2 instructions: two fp32 lanes per 64-bit register)
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t r) {
    float2 v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
    return v;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// GELU of two values at once: the formula of gelu_as (Abramowitz & Stegun 7.1.26 for
// erfc(|z| / sqrt 2), t = 1 / (1 + p x)) with the polynomial, the products and the final
// blend in packed f32x2 instructions and the reciprocal and exponential as one approximate
// instruction per value.  The factor 1/2 of Phi's tail is taken into the exponent
// (exp(-x^2) / 2 = 2^(-x^2 log2 e - 1)), and Phi = s + m * tail with m = -1, s = 1 for
// z >= 0 and m = 1, s = 0 below, so both branches round once, as in gelu_as.
__device__ __forceinline__ float2 gelu_pair(float z0, float z1) {
    const uint64_t z = f2_pack(z0, z1);
    const float a0 = fabsf(z0), a1 = fabsf(z1);
    const uint64_t x = f2_mul(f2_pack(a0, a1), f2_pack(0.70710678118654752f, 0.70710678118654752f));
    const uint64_t den = f2_fma(f2_pack(0.3275911f, 0.3275911f), x, f2_pack(1.0f, 1.0f));
    const float2 dn = f2_unpack(den);
    const uint64_t t = f2_pack(rcp_approx(dn.x), rcp_approx(dn.y));
    uint64_t p = f2_fma(f2_pack(1.061405429f, 1.061405429f), t, f2_pack(-1.453152027f, -1.453152027f));
    p = f2_fma(p, t, f2_pack(1.421413741f, 1.421413741f));
    p = f2_fma(p, t, f2_pack(-0.284496736f, -0.284496736f));
    p = f2_fma(p, t, f2_pack(0.254829592f, 0.254829592f));
    const uint64_t pt = f2_mul(p, t);
    const uint64_t xx = f2_mul(x, x);
    // -log2(e) x^2 - 1
    const float2 arg = f2_unpack(f2_fma(xx, f2_pack(-1.4426950408889634f, -1.4426950408889634f), f2_pack(-1.0f, -1.0f)));
    const uint64_t tail = f2_mul(pt, f2_pack(ex2_approx(arg.x), ex2_approx(arg.y)));  // erfc(x) / 2
    // m = +1 below zero, -1 from zero up (1.0f with the inverted sign of z)
    const float m0 = __uint_as_float(0x3f800000u | (~__float_as_uint(z0) & 0x80000000u));
    const float m1 = __uint_as_float(0x3f800000u | (~__float_as_uint(z1) & 0x80000000u));
    const uint64_t m = f2_pack(m0, m1);
    const uint64_t s = f2_fma(m, f2_pack(-0.5f, -0.5f), f2_pack(0.5f, 0.5f));
    const uint64_t phi = f2_fma(m, tail, s);
    return f2_unpack(f2_mul(z, phi));
}

}  // namespace tc
}  // namespace scx

namespace scx {
namespace tc {

// Shared-memory descriptor of a K-major operand with the 32-byte swizzle: rows of 32 bytes
// (8 tf32 values), 8-row groups 256 bytes apart (SBO), the two 16-byte halves of row r swapped
// when (r / 4) is odd (address bit 4 ^= bit 7, so the base is 256-byte aligned).  One tf32 MMA
// (K = 8) covers a whole row.  Layout type 6 = SWIZZLE_32B in the sm_100 descriptor format.
__device__ __forceinline__ uint64_t desc_sw32(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(256u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(6u) << 61;
    return d;
}

// Waits for the phase of parity `parity` with try_wait and no suspend-time hint (the thread
// blocks in the instruction for a short system-dependent time and retries), for short
// hand-offs where a suspended thread would wake late; gives up after ~2^31 SM cycles like
// mbar_wait_bounded.
__device__ __forceinline__ bool mbar_try_wait_nohint(uint64_t* bar, uint32_t parity) {
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
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity) {
    const long long start = clock64();
    while (!mbar_try_wait_nohint(bar, parity)) {
        if (clock64() - start > (1LL << 31)) return false;
    }
    return true;
}

// Byte offset of the 16-byte unit `half` (values 4*half .. 4*half + 3) of row r in a K-major
// SW32 operand (see desc_sw32).
__host__ __device__ __forceinline__ uint32_t sw32_offset(int r, int half) {
    return static_cast<uint32_t>(r >> 3) * 256u + static_cast<uint32_t>(r & 7) * 32u +
           (static_cast<uint32_t>(half ^ ((r >> 2) & 1)) << 4);
}

// 3-D tiled TMA store of a shared-memory box to (c0, c1, c2) of `tmap` (elements outside the
// tensor are not written); completion tracked by the bulk-group of the issuing thread.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace tc
}  // namespace scx
