// FNO projection on the tensor core (fno_ns/model.py:162-166):
//
//   y[b][oc][p] = b2[oc] + sum_j W2[oc][j] GELU(b1[j] + sum_c W1[j][c] h[b][c][p])
//
// One CTA (4 warps) per tile of 128 pixels of one batch item.  The first layer is a GEMM
// D[pixel][j] = sum_c h[c][pixel] W1[j][c] (M = 128 pixels, N = proj_hidden, K = hidden) in
// bf16x3 (hi*hi + hi*lo + lo*hi, fp32 TMEM accumulator):
//   A = the h tile, MN-major in shared memory (pixels are contiguous for a fixed channel in
//       h's [B][C][H*W] layout), split into bf16 hi/lo by the CTA's threads;
//   B = W1, K-major in shared memory, split the same way.
// Lane l of warp w then holds pixel 32w + l: it reads its row of D from TMEM 32 columns at a
// time and finishes bias, GELU and the second layer in registers, taking the hidden units in
// order j = 0, 1, ... like fno_project_kernel.  The wait for the MMAs is bounded (about a
// second); a CTA that gives up stores a code in the device watchdog word and writes nothing.
#include "scx_internal.h"
#include "scx_tc.cuh"

namespace scx {
namespace {

constexpr int kProjThreads = 128;  // 4 warps: one TMEM sub-partition each
constexpr int kTile = 128;         // pixels per CTA (MMA M)
constexpr int kMaxOut = 4;

__device__ __forceinline__ float gelu(float z) { return 0.5f * z * (1.0f + erff(z * 0.70710678118654752f)); }

struct ProjArgs {
    const float* h;
    float* y;
    const float* w1;  // [ph][C]
    const float* b1;  // [ph]
    const float* w2;  // [oc][ph]
    const float* b2;  // [oc]
    int HW, C, ph, oc;
    uint32_t tmem_cols;
    int* watchdog;
};

// Shared memory: W1 hi | W1 lo (K-major SW128, ph rows of 128 bytes each) | h tile hi | lo
// (MN-major SW128: C/8 K-groups of 2 x 1 KB MN atoms) | b1 | w2.
__global__ void __launch_bounds__(kProjThreads) fno_project_tc_kernel(const ProjArgs a) {
    extern __shared__ uint8_t proj_raw[];
    __shared__ uint64_t done;
    __shared__ uint32_t tmem_base;
    uint8_t* base = tc::align1024(proj_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = a.C, ph = a.ph;
    const uint32_t WB = static_cast<uint32_t>(ph) * 128u;       // one W1 part
    const uint32_t AB = static_cast<uint32_t>(C / 8) * 2048u;   // one h part
    uint8_t* w_hi = base;
    uint8_t* w_lo = base + WB;
    uint8_t* a_hi = base + 2 * WB;
    uint8_t* a_lo = a_hi + AB;
    float* b1s = reinterpret_cast<float*>(a_lo + AB);
    float* w2s = b1s + ph;

    if (warp == 0) {
        tc::tmem_alloc(&tmem_base, a.tmem_cols);
        tc::tmem_relinquish();
    }
    if (tid == 0) tc::mbar_init(&done, 1);

    // W1 -> bf16 hi/lo, K-major: 8 consecutive channels of row j per 16-byte unit
    for (int u = tid; u < ph * (C / 8); u += kProjThreads) {
        const int j = u / (C / 8), c0 = (u % (C / 8)) * 8;
        const float4* src = reinterpret_cast<const float4*>(a.w1 + static_cast<size_t>(j) * C + c0);
        const float4 v0 = __ldg(src), v1 = __ldg(src + 1);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint4 hi, lo;
        tc::split8(v, hi, lo);
        const uint32_t off = tc::kmajor_offset(ph, j, c0);
        *reinterpret_cast<uint4*>(w_hi + off) = hi;
        *reinterpret_cast<uint4*>(w_lo + off) = lo;
    }
    // h tile -> bf16 hi/lo, MN-major: 8 consecutive pixels of channel c per 16-byte unit
    const int tiles_per_plane = a.HW / kTile;
    const int b = blockIdx.x / tiles_per_plane;
    const int p0 = (blockIdx.x % tiles_per_plane) * kTile;
    const float* hb = a.h + static_cast<size_t>(b) * C * a.HW + p0;
    for (int u = tid; u < C * (kTile / 8); u += kProjThreads) {
        const int c = u / (kTile / 8), m0 = (u % (kTile / 8)) * 8;
        const float4* src = reinterpret_cast<const float4*>(hb + static_cast<size_t>(c) * a.HW + m0);
        const float4 v0 = __ldg(src), v1 = __ldg(src + 1);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint4 hi, lo;
        tc::split8(v, hi, lo);
        const uint32_t off = static_cast<uint32_t>(c >> 3) * 2048u + static_cast<uint32_t>(m0 >> 6) * 1024u +
                             static_cast<uint32_t>(c & 7) * 128u +
                             (static_cast<uint32_t>(((m0 & 63) >> 3) ^ (c & 7)) << 4);
        *reinterpret_cast<uint4*>(a_hi + off) = hi;
        *reinterpret_cast<uint4*>(a_lo + off) = lo;
    }
    for (int i = tid; i < ph; i += kProjThreads) b1s[i] = __ldg(a.b1 + i);
    for (int i = tid; i < a.oc * ph; i += kProjThreads) w2s[i] = __ldg(a.w2 + i);
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base;

    if (tid == 0) {
        const uint32_t sb = tc::smem_u32(base);
        const uint64_t dW[2] = {tc::desc_sw128(sb), tc::desc_sw128(sb + WB)};
        const uint64_t dA[2] = {tc::desc_mn_sw128(sb + 2 * WB, 1024u, 2048u),
                                tc::desc_mn_sw128(sb + 2 * WB + AB, 1024u, 2048u)};
        const uint32_t id = tc::idesc_bf16(kTile, ph) | tc::kIdescAMajorMN;
        // (h_hi, W_hi), (h_hi, W_lo), (h_lo, W_hi), chained along K
        for (int part = 0; part < 3; ++part) {
            const int ap = part == 2 ? 1 : 0, bp = part == 1 ? 1 : 0;
            for (int ks = 0; ks < C / 16; ++ks) {
                const uint32_t ao = (static_cast<uint32_t>(ks) * 4096u) >> 4, bo = (static_cast<uint32_t>(ks) * 32u) >> 4;
                tc::mma_bf16(tmem, dA[ap] + ao, dW[bp] + bo, id, (part | ks) ? 1u : 0u);
            }
        }
        tc::mma_commit(&done);
    }
    const bool ok = tc::mbar_wait_bounded(&done, 0);
    tc::fence_after_sync();
    if (ok) {
        float out[kMaxOut];
#pragma unroll
        for (int o = 0; o < kMaxOut; ++o) out[o] = 0.f;
        const uint32_t row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        for (int j0 = 0; j0 < ph; j0 += 32) {
            float v[32];
            tc::tmem_ld32_nowait(row + static_cast<uint32_t>(j0), v);
            tc::tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                const float g = gelu(v[k] + b1s[j0 + k]);
#pragma unroll
                for (int o = 0; o < kMaxOut; ++o)
                    if (o < a.oc) out[o] = fmaf(w2s[o * ph + j0 + k], g, out[o]);
            }
        }
        const int p = p0 + warp * 32 + lane;
#pragma unroll
        for (int o = 0; o < kMaxOut; ++o)
            if (o < a.oc) a.y[(static_cast<size_t>(b) * a.oc + o) * a.HW + p] = out[o] + __ldg(a.b2 + o);
    } else if (lane == 0) {
        atomicExch(a.watchdog, 50);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, a.tmem_cols);
    }
}

size_t proj_smem(int C, int ph, int oc) {
    return 2u * static_cast<size_t>(ph) * 128u + 2u * static_cast<size_t>(C / 8) * 2048u +
           static_cast<size_t>(ph + oc * ph) * 4u + 1024u;
}

}  // namespace

bool fno_project_tc_supported(int hidden, int ph, int oc, int HW) {
    return hidden % 16 == 0 && hidden >= 16 && hidden <= 64 && ph % 32 == 0 && ph >= 32 && ph <= 256 && oc >= 1 &&
           oc <= kMaxOut && HW % kTile == 0 && proj_smem(hidden, ph, oc) <= 200u * 1024u;
}

cudaError_t launch_fno_project_tc(const float* h, float* y, const float* w1, const float* b1, const float* w2,
                                  const float* b2, int B, int HW, int hidden, int ph, int oc, cudaStream_t stream) {
    if (!fno_project_tc_supported(hidden, ph, oc, HW) || B <= 0 ||
        ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(w1)) & 15) != 0)
        return cudaErrorInvalidValue;
    ProjArgs a;
    a.h = h;
    a.y = y;
    a.w1 = w1;
    a.b1 = b1;
    a.w2 = w2;
    a.b2 = b2;
    a.HW = HW;
    a.C = hidden;
    a.ph = ph;
    a.oc = oc;
    a.tmem_cols = ph <= 32 ? 32u : (ph <= 64 ? 64u : (ph <= 128 ? 128u : 256u));
    cudaError_t e = device_watchdog(&a.watchdog);
    if (e != cudaSuccess) return e;
    const size_t smem = proj_smem(hidden, ph, oc);
    int per_sm = 1;
    e = prepare_kernel(reinterpret_cast<const void*>(fno_project_tc_kernel), smem, kProjThreads, &per_sm);
    if (e != cudaSuccess) return e;
    const unsigned grid = static_cast<unsigned>(static_cast<long long>(B) * (HW / kTile));
    fno_project_tc_kernel<<<grid, kProjThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace scx
