// FNO projection on the tensor core (fno_ns/model.py:162-166):
//
//   y[b][oc][p] = b2[oc] + sum_j W2[oc][j] GELU(b1[j] + sum_c W1[j][c] h[b][c][p])
//
// One CTA (8 warps) per tile of 128 pixels of one batch item.  The first layer is a GEMM
// D[pixel][j] = sum_c h[c][pixel] W1[j][c] (M = 128 pixels, N = proj_hidden, K = hidden) in
// 3xTF32 (hi*hi + hi*lo + lo*hi with hi = the top 19 bits and lo = the exact remainder, fp32
// TMEM accumulator; about 1e-6 relative per product, where bf16x3's 2e-5 was too coarse for
// 32-term sums feeding the output):
//   A = the h tile, K-major in shared memory (transposed from h's [B][C][H*W] layout while it
//       is split by the CTA's threads);
//   B = W1, K-major in shared memory, split the same way.
// Lane l of warps w and w + 4 then holds pixel 32w + l: each reads half of its row of D from
// TMEM, 16 columns at a time, and finishes bias, GELU and the second layer for its half of the
// hidden units in order; the two halves' sums are added through shared memory.  The wait for the MMAs is bounded (about a
// second); a CTA that gives up stores a code in the device watchdog word and writes nothing.
#include <algorithm>

#include "scx_internal.h"
#include "scx_tc.cuh"

namespace scx {
namespace {

constexpr int kProjThreads = 256;  // 8 warps: two per TMEM sub-partition
constexpr int kTile = 128;         // pixels per CTA (MMA M)
constexpr int kMaxOut = 4;
constexpr int kProjCtasPerSm = 3;  // register budget of the launch bounds; the persistent grid

// W [N][K] (row-major, K = channels) -> tf32 hi/lo (fp32 containers), K-major SW128: 4
// consecutive k of row n per 16-byte unit.
__device__ __forceinline__ void stage_weights(const float* __restrict__ w, int N, int K, uint8_t* w_hi,
                                              uint8_t* w_lo) {
    for (int u = threadIdx.x; u < N * (K / 4); u += blockDim.x) {
        const int n = u / (K / 4), k0 = (u % (K / 4)) * 4;
        const float4 v = __ldg(reinterpret_cast<const float4*>(w + static_cast<size_t>(n) * K + k0));
        float4 hi, lo;
        tc::split_tf32(v.x, hi.x, lo.x);
        tc::split_tf32(v.y, hi.y, lo.y);
        tc::split_tf32(v.z, hi.z, lo.z);
        tc::split_tf32(v.w, hi.w, lo.w);
        const uint32_t off = tc::kmajor_offset32(N, n, k0);
        *reinterpret_cast<float4*>(w_hi + off) = hi;
        *reinterpret_cast<float4*>(w_lo + off) = lo;
    }
}

// The [C][kTile] pixel tile at hb (channel stride HW) -> tf32 hi/lo, K-major SW128 (row =
// pixel, K = channel): each unit reads 4 channels of one pixel (consecutive lanes take
// consecutive pixels, so every load instruction reads 128 contiguous bytes) and writes one
// 16-byte unit.  load_tile / store_tile do the same in two steps for C == kPrefC, so that the
// next tile's loads are in flight while the current tile is finished.
constexpr int kPrefC = 32;
constexpr int kPrefUnits = kTile * (kPrefC / 4) / kProjThreads;  // units per thread

__device__ __forceinline__ void load_tile(const float* __restrict__ hb, int HW, float4 (&v)[kPrefUnits]) {
#pragma unroll
    for (int j = 0; j < kPrefUnits; ++j) {
        const int u = threadIdx.x + j * kProjThreads;
        const int m = u % kTile, c0 = (u / kTile) * 4;
        const float* src = hb + static_cast<size_t>(c0) * HW + m;
        v[j] = make_float4(__ldg(src), __ldg(src + HW), __ldg(src + 2 * static_cast<size_t>(HW)),
                           __ldg(src + 3 * static_cast<size_t>(HW)));
    }
}

__device__ __forceinline__ void store_tile(const float4 (&v)[kPrefUnits], uint8_t* a_hi, uint8_t* a_lo) {
#pragma unroll
    for (int j = 0; j < kPrefUnits; ++j) {
        const int u = threadIdx.x + j * kProjThreads;
        const int m = u % kTile, c0 = (u / kTile) * 4;
        float4 hi, lo;
        tc::split_tf32(v[j].x, hi.x, lo.x);
        tc::split_tf32(v[j].y, hi.y, lo.y);
        tc::split_tf32(v[j].z, hi.z, lo.z);
        tc::split_tf32(v[j].w, hi.w, lo.w);
        const uint32_t off = tc::kmajor_offset32(kTile, m, c0);
        *reinterpret_cast<float4*>(a_hi + off) = hi;
        *reinterpret_cast<float4*>(a_lo + off) = lo;
    }
}
__device__ __forceinline__ void stage_tile(const float* __restrict__ hb, int C, int HW, uint8_t* a_hi,
                                           uint8_t* a_lo) {
    for (int u = threadIdx.x; u < kTile * (C / 4); u += blockDim.x) {
        const int m = u % kTile, c0 = (u / kTile) * 4;
        const float* src = hb + static_cast<size_t>(c0) * HW + m;
        float4 hi, lo;
        tc::split_tf32(__ldg(src), hi.x, lo.x);
        tc::split_tf32(__ldg(src + HW), hi.y, lo.y);
        tc::split_tf32(__ldg(src + 2 * static_cast<size_t>(HW)), hi.z, lo.z);
        tc::split_tf32(__ldg(src + 3 * static_cast<size_t>(HW)), hi.w, lo.w);
        const uint32_t off = tc::kmajor_offset32(kTile, m, c0);
        *reinterpret_cast<float4*>(a_hi + off) = hi;
        *reinterpret_cast<float4*>(a_lo + off) = lo;
    }
}

// D[pixel][n] = sum_c tile[c][pixel] W[n][c] in 3xTF32 ((A_hi, W_hi), (A_hi, W_lo), (A_lo, W_hi)
// chained along K, 8 channels per instruction), issued by the calling thread, completion on
// `done`.
__device__ __forceinline__ void issue_gemm(uint32_t tmem, const uint8_t* w_hi, const uint8_t* w_lo,
                                           const uint8_t* a_hi, const uint8_t* a_lo, int N, int K, uint64_t* done) {
    const uint64_t dW[2] = {tc::desc_sw128(tc::smem_u32(w_hi)), tc::desc_sw128(tc::smem_u32(w_lo))};
    const uint64_t dA[2] = {tc::desc_sw128(tc::smem_u32(a_hi)), tc::desc_sw128(tc::smem_u32(a_lo))};
    const uint32_t id = tc::idesc_tf32(kTile, N);
    for (int part = 0; part < 3; ++part) {
        const int ap = part == 2 ? 1 : 0, bp = part == 1 ? 1 : 0;
        for (int ks = 0; ks < K / 8; ++ks) {
            // K blocks of 32 channels: rows * 128 bytes apart; 32 bytes per K step within one
            const uint32_t ao = (static_cast<uint32_t>(ks >> 2) * kTile * 128u + (ks & 3) * 32u) >> 4;
            const uint32_t bo = (static_cast<uint32_t>(ks >> 2) * static_cast<uint32_t>(N) * 128u + (ks & 3) * 32u) >> 4;
            tc::mma_tf32(tmem, dA[ap] + ao, dW[bp] + bo, id, (part | ks) ? 1u : 0u);
        }
    }
    tc::mma_commit(done);
}

// Bias, GELU and the second layer over hidden units [j_begin, j_end) (multiples of 16) of this
// thread's TMEM lane: out[o] += W2[o][j] GELU(D[j] + b1[j]) in order j = j_begin, ...
template <int OC>
__device__ __forceinline__ void finish_units(uint32_t row, int j_begin, int j_end, const float* b1s,
                                             const float* w2s, int ph, float (&out)[kMaxOut]) {
    for (int j0 = j_begin; j0 < j_end; j0 += 16) {
        float v[16];
        tc::tmem_ld16_nowait(row + static_cast<uint32_t>(j0), v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
            const float4 bb = *reinterpret_cast<const float4*>(b1s + j0 + 4 * k4);
            const float2 g01 = tc::gelu_pair(v[4 * k4 + 0] + bb.x, v[4 * k4 + 1] + bb.y);
            const float2 g23 = tc::gelu_pair(v[4 * k4 + 2] + bb.z, v[4 * k4 + 3] + bb.w);
            const float g0 = g01.x, g1 = g01.y, g2 = g23.x, g3 = g23.y;
#pragma unroll
            for (int o = 0; o < OC; ++o) {
                const float4 ww = *reinterpret_cast<const float4*>(w2s + o * ph + j0 + 4 * k4);
                out[o] = fmaf(ww.x, g0, out[o]);
                out[o] = fmaf(ww.y, g1, out[o]);
                out[o] = fmaf(ww.z, g2, out[o]);
                out[o] = fmaf(ww.w, g3, out[o]);
            }
        }
    }
}

uint32_t tmem_cols_for(int n) { return n <= 32 ? 32u : (n <= 64 ? 64u : (n <= 128 ? 128u : 256u)); }

struct ProjArgs {
    const float* h;
    float* y;
    const float* w1;  // [ph][C]
    const float* b1;  // [ph]
    const float* w2;  // [oc][ph]
    const float* b2;  // [oc]
    int HW, C, ph, oc;
    int ntiles;  // B * HW / kTile
    uint32_t tmem_cols;
    int* watchdog;
};

// Shared memory: W1 hi | W1 lo | h tile hi | h tile lo (all K-major SW128, fp32) | b1 | w2.
// Persistent: CTA i takes the pixel tiles i, i + gridDim.x, ...; the weights are staged once,
// and for hidden == kPrefC the next tile's h loads are in flight during the current tile's MMAs
// and epilogue.
__global__ void __launch_bounds__(kProjThreads, kProjCtasPerSm) fno_project_tc_kernel(const ProjArgs a) {
    extern __shared__ uint8_t proj_raw[];
    __shared__ uint64_t done;
    __shared__ uint32_t tmem_base;
    uint8_t* base = tc::align1024(proj_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = a.C, ph = a.ph;
    const uint32_t WB = static_cast<uint32_t>(ph) * C * 4u;     // one W1 part
    const uint32_t AB = static_cast<uint32_t>(kTile) * C * 4u;  // one h part
    uint8_t* w_hi = base;
    uint8_t* w_lo = base + WB;
    uint8_t* a_hi = base + 2 * WB;
    uint8_t* a_lo = a_hi + AB;
    float* b1s = reinterpret_cast<float*>(a_lo + AB);
    float* w2s = b1s + ph;
    float* part = w2s + a.oc * ph;  // [kMaxOut][kTile]: the second half's partial outputs

    if (warp == 0) {
        tc::tmem_alloc(&tmem_base, a.tmem_cols);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        tc::grid_dep_launch();  // launched as a programmatic dependent: the next kernel may start
        tc::mbar_init(&done, 1);
    }
    stage_weights(a.w1, ph, C, w_hi, w_lo);
    for (int i = tid; i < ph; i += kProjThreads) b1s[i] = __ldg(a.b1 + i);
    for (int i = tid; i < a.oc * ph; i += kProjThreads) w2s[i] = __ldg(a.w2 + i);
    tc::grid_dep_wait();  // h comes from the last layer's kernels
    const int tiles_per_plane = a.HW / kTile;
    auto tile_src = [&](int t) {
        return a.h + static_cast<size_t>(t / tiles_per_plane) * C * a.HW + (t % tiles_per_plane) * kTile;
    };
    const bool pref = C == kPrefC;
    float4 nxt[kPrefUnits];
    if (pref && static_cast<int>(blockIdx.x) < a.ntiles) load_tile(tile_src(blockIdx.x), a.HW, nxt);
    const int sub = warp & 3, half = warp >> 2, m = sub * 32 + lane;
    bool ok = true;
    int it = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, ++it) {
        if (pref)
            store_tile(nxt, a_hi, a_lo);
        else
            stage_tile(tile_src(t), C, a.HW, a_hi, a_lo);
        tc::fence_async_smem();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        const uint32_t tmem = tmem_base;
        if (tid == 0) issue_gemm(tmem, w_hi, w_lo, a_hi, a_lo, ph, C, &done);
        const int tn = t + static_cast<int>(gridDim.x);
        if (pref && tn < a.ntiles) load_tile(tile_src(tn), a.HW, nxt);
        ok = tc::mbar_wait_bounded(&done, it & 1);
        tc::fence_after_sync();
        // warps w and w + 4 read the same TMEM lanes (pixels 32 (w % 4) ..): the first takes the
        // hidden units [0, ph/2), the second [ph/2, ph); the outputs are the first half's sums
        // plus the second's
        float out[kMaxOut];
#pragma unroll
        for (int o = 0; o < kMaxOut; ++o) out[o] = 0.f;
        if (ok) {
            const uint32_t row = tmem + (static_cast<uint32_t>(sub * 32) << 16);
            const int jh = ph / 2;
            switch (a.oc) {
                case 1: finish_units<1>(row, half * jh, (half + 1) * jh, b1s, w2s, ph, out); break;
                case 2: finish_units<2>(row, half * jh, (half + 1) * jh, b1s, w2s, ph, out); break;
                case 3: finish_units<3>(row, half * jh, (half + 1) * jh, b1s, w2s, ph, out); break;
                default: finish_units<4>(row, half * jh, (half + 1) * jh, b1s, w2s, ph, out); break;
            }
            if (half == 1) {
#pragma unroll
                for (int o = 0; o < kMaxOut; ++o) part[o * kTile + m] = out[o];
            }
        }
        __syncthreads();
        if (ok && half == 0) {
            const int b = t / tiles_per_plane, p = (t % tiles_per_plane) * kTile + m;
#pragma unroll
            for (int o = 0; o < kMaxOut; ++o)
                if (o < a.oc)
                    a.y[(static_cast<size_t>(b) * a.oc + o) * a.HW + p] = (out[o] + part[o * kTile + m]) + __ldg(a.b2 + o);
        }
        // this tile's TMEM rows, A operand and partials are no longer read; every thread agrees
        // on whether to go on
        tc::fence_before_sync();
        ok = __syncthreads_and(ok) != 0;
        tc::fence_after_sync();
        if (!ok) break;
    }
    if (!ok && tid == 0) atomicExch(a.watchdog, 50);
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem_base, a.tmem_cols);
    }
}

size_t proj_smem(int C, int ph, int oc) {
    return 2u * static_cast<size_t>(ph) * C * 4u + 2u * static_cast<size_t>(kTile) * C * 4u +
           static_cast<size_t>(ph + oc * ph + kMaxOut * kTile) * 4u + 1024u;
}

}  // namespace

bool fno_project_tc_supported(int hidden, int ph, int oc, int HW) {
    // K-major rows are 32 channels (128 bytes) wide, so hidden is 32 or 64
    return (hidden == 32 || hidden == 64) && ph % 32 == 0 && ph >= 32 && ph <= 256 && oc >= 1 &&
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
    a.tmem_cols = tmem_cols_for(ph);
    a.ntiles = static_cast<int>(static_cast<long long>(B) * (HW / kTile));
    cudaError_t e = device_watchdog(&a.watchdog);
    if (e != cudaSuccess) return e;
    const size_t smem = proj_smem(hidden, ph, oc);
    int per_sm = 1;
    e = prepare_kernel(reinterpret_cast<const void*>(fno_project_tc_kernel), smem, kProjThreads, &per_sm);
    if (e != cudaSuccess) return e;
    // persistent: kProjCtasPerSm CTAs per SM (the launch bounds' register budget; the shared
    // memory of three fits), at most one per tile; CTAs that do not fit at once simply start later
    const unsigned grid = static_cast<unsigned>(std::min<long long>(a.ntiles, static_cast<long long>(kProjCtasPerSm) * num_sms()));
    return launch_chained(fno_project_tc_kernel, dim3(grid), dim3(kProjThreads), smem, stream, a);
}

}  // namespace scx

