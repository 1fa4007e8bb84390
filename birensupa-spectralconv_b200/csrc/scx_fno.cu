// FNO-2d forward (fno_ns/model.py:137-259) as one C-ABI call.
//
// Kernels besides the spectral convolution (scx_dft_*.cu, scx_mix.cu), all launched as
// programmatic dependents of the previous kernel (each CTA waits with griddepcontrol.wait
// before its first read of activations; weights are staged before that):
//   fno_lift_kernel            1x1 conv (T+2 -> hidden) with the grid channels generated
//                              in-kernel (fno_ns/model.py:168-181,193-195) or read from a
//                              channels-last input
//   fno_skip_norm_kernel       with instance norm, planes of up to 8192 pixels (a multiple
//                              of 4): skip GEMM, two-pass instance statistics over a
//                              thread-block cluster per plane group, normalisation and GELU
//                              (fno_ns/model.py:96-99,133-134) in one launch
//   fno_skip_kernel            otherwise, per pixel: z = spectral + W h + b for every output
//                              channel (fno_skip_quad_kernel: four pixels per thread)
//   fno_norm_gelu_kernel       then one CTA per plane: two-pass instance statistics,
//                              normalisation and GELU
//   fno_project_kernel         per pixel: hidden -> proj_hidden (GELU) -> out_channels, the
//                              proj_hidden-wide intermediate never leaves registers
//                              (fno_ns/model.py:162-166); the shapes scx_fno_proj_tc.cu
//                              supports run its tensor-core version instead
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <utility>

#include <cuda.h>

#include "scx.h"
#include "scx_internal.h"
#include "scx_tc.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float gelu_erf(float z) { return scx::tc::gelu_as(z); }

// torch.linspace(0, 1, n)[i] in fp32: start + i*step on the first half, end - (n-1-i)*step on
// the second half, step = 1/(n-1).
__device__ __forceinline__ float linspace01(int i, int n) {
    if (n <= 1) return 0.f;
    const float step = 1.0f / static_cast<float>(n - 1);
    return i < n / 2 ? static_cast<float>(i) * step : 1.0f - static_cast<float>(n - 1 - i) * step;
}

// h[b][c][p] = b[c] + sum_k W[c][k] in[b][k][p]; in = (T frames, grid_x, grid_y).
// HMAX >= hidden (compile-time register budget).  grid = (ceil(HW / 256), B)
template <int HMAX>
__global__ void __launch_bounds__(kThreads) fno_lift_kernel(const float* __restrict__ x, float* __restrict__ h,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ bias, int H, int W, int T,
                                                            int hidden, int layout) {
    scx::tc::grid_dep_launch();  // launched as a programmatic dependent: the next kernel may start
    extern __shared__ float lift_smem[];
    const int cin = T + 2;
    float* ws = lift_smem;  // [cin][HMAX] (transposed: one input channel's weights contiguous)
    for (int i = threadIdx.x; i < cin * HMAX; i += kThreads) {
        const int k = i / HMAX, c = i - k * HMAX;
        ws[i] = c < hidden ? w[c * cin + k] : 0.f;
    }
    __syncthreads();
    scx::tc::grid_dep_wait();  // inputs may come from the previous kernel in the stream
    const int HW = H * W;
    const int b = blockIdx.y;
    const int p = blockIdx.x * kThreads + threadIdx.x;
    if (p >= HW) return;
    float acc[HMAX];
#pragma unroll
    for (int c = 0; c < HMAX; ++c) acc[c] = c < hidden ? __ldg(bias + c) : 0.f;
    const int row = p / W, col = p - row * W;
    for (int k = 0; k < cin; ++k) {
        float v;
        if (layout == 0)
            v = k < T ? __ldg(x + (static_cast<size_t>(b) * T + k) * HW + p)
                      : (k == T ? linspace01(row, H) : linspace01(col, W));
        else
            v = __ldg(x + (static_cast<size_t>(b) * HW + p) * cin + k);
        const float4* wk = reinterpret_cast<const float4*>(ws + k * HMAX);
#pragma unroll
        for (int c4 = 0; c4 < HMAX / 4; ++c4) {
            const float4 wv = wk[c4];
            acc[4 * c4 + 0] = fmaf(wv.x, v, acc[4 * c4 + 0]);
            acc[4 * c4 + 1] = fmaf(wv.y, v, acc[4 * c4 + 1]);
            acc[4 * c4 + 2] = fmaf(wv.z, v, acc[4 * c4 + 2]);
            acc[4 * c4 + 3] = fmaf(wv.w, v, acc[4 * c4 + 3]);
        }
    }
    float* hb = h + static_cast<size_t>(b) * hidden * HW + p;
#pragma unroll
    for (int c = 0; c < HMAX; ++c)
        if (c < hidden) hb[static_cast<size_t>(c) * HW] = acc[c];
}

// Fourier-layer epilogue, part A:
//   z[b][o][p] = s[b][o][p] + bias[o] + sum_i Wskip[o][i] h[b][i][p]
// written over s when instance_norm is on (part B normalises it), else GELU(z) written to
// h_next.  Each thread takes PX pixels kThreads apart (one shared-memory read of a weight row
// feeds PX pixels) and four output channels per pass (independent FMA chains; each channel's
// sum keeps its order over i); the output channels are split into groups of kSkipGroup over
// grid.z, for enough warps per SM.  grid = (ceil(HW / (kThreads * PX)), B, ceil(hidden / kSkipGroup))
constexpr int kSkipGroup = 8;
// Input channels per batch of loads in the four-pixel kernels: eight float4 registers, which
// keeps them at three 256-thread CTAs per SM (one wave for B20 at 64x64)
constexpr int kSkipBatch = 8;

template <int HMAX, int PX>
__global__ void __launch_bounds__(kThreads) fno_skip_kernel(float* __restrict__ s, const float* __restrict__ h,
                                                            float* __restrict__ h_next,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ bias, int HW, int hidden,
                                                            int instance_norm) {
    scx::tc::grid_dep_launch();
    __shared__ __align__(16) float ws[HMAX * HMAX];  // [o][i], zero padded
    for (int i = threadIdx.x; i < HMAX * HMAX; i += kThreads) {
        const int o = i / HMAX, k = i - o * HMAX;
        ws[i] = (o < hidden && k < hidden) ? w[o * hidden + k] : 0.f;
    }
    __syncthreads();
    scx::tc::grid_dep_wait();  // s and h come from earlier kernels in the stream
    const int b = blockIdx.y;
    const int p0 = blockIdx.x * kThreads * PX + threadIdx.x;
    if (p0 >= HW) return;
    int pix[PX];
    bool live[PX];
#pragma unroll
    for (int x = 0; x < PX; ++x) {
        live[x] = p0 + x * kThreads < HW;
        pix[x] = live[x] ? p0 + x * kThreads : p0;  // a pixel past the plane repeats the first one
    }
    const size_t plane0 = static_cast<size_t>(b) * hidden * HW;
    float hv[PX][HMAX];
#pragma unroll
    for (int x = 0; x < PX; ++x)
#pragma unroll
        for (int i = 0; i < HMAX; ++i)
            hv[x][i] = i < hidden ? __ldg(h + plane0 + static_cast<size_t>(i) * HW + pix[x]) : 0.f;
    const int o_end = min(hidden, static_cast<int>(blockIdx.z + 1) * kSkipGroup);
    for (int o0 = blockIdx.z * kSkipGroup; o0 < o_end; o0 += 4) {
        float z[4][PX];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int o = min(o0 + t, hidden - 1);
            const float bo = __ldg(bias + o);
#pragma unroll
            for (int x = 0; x < PX; ++x) z[t][x] = bo + s[plane0 + static_cast<size_t>(o) * HW + pix[x]];
        }
#pragma unroll
        for (int i4 = 0; i4 < HMAX / 4; ++i4) {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float4 wv = reinterpret_cast<const float4*>(ws + min(o0 + t, hidden - 1) * HMAX)[i4];
#pragma unroll
                for (int x = 0; x < PX; ++x) {
                    z[t][x] = fmaf(wv.x, hv[x][4 * i4 + 0], z[t][x]);
                    z[t][x] = fmaf(wv.y, hv[x][4 * i4 + 1], z[t][x]);
                    z[t][x] = fmaf(wv.z, hv[x][4 * i4 + 2], z[t][x]);
                    z[t][x] = fmaf(wv.w, hv[x][4 * i4 + 3], z[t][x]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            if (o0 + t >= o_end) break;
            const size_t row = plane0 + static_cast<size_t>(o0 + t) * HW;
#pragma unroll
            for (int x = 0; x < PX; ++x) {
                if (!live[x]) continue;
                if (instance_norm)
                    s[row + pix[x]] = z[t][x];
                else
                    h_next[row + pix[x]] = gelu_erf(z[t][x]);
            }
        }
    }
}

// The same skip GEMM with four consecutive pixels per thread (float4 loads and stores), for
// planes whose pixel count is a multiple of 4 and hidden a multiple of 16: input channels in
// batches of kSkipBatch loads, each float4 of weights feeding 16 FMAs.  Each output keeps the order bias + s,
// then i = 0, 1, ..., so the results equal fno_skip_kernel's bit for bit.
// grid = (ceil(HW / (4 * kThreads)), B, ceil(hidden / kSkipGroup))
template <int HMAX>
__global__ void __launch_bounds__(kThreads, 3) fno_skip_quad_kernel(float* __restrict__ s, const float* __restrict__ h,
                                                                 float* __restrict__ h_next,
                                                                 const float* __restrict__ w,
                                                                 const float* __restrict__ bias, int HW, int hidden,
                                                                 int instance_norm) {
    scx::tc::grid_dep_launch();
    __shared__ __align__(16) float ws[HMAX * HMAX];  // [o][i], zero padded
    for (int i = threadIdx.x; i < HMAX * HMAX; i += kThreads) {
        const int o = i / HMAX, k = i - o * HMAX;
        ws[i] = (o < hidden && k < hidden) ? w[o * hidden + k] : 0.f;
    }
    __syncthreads();
    scx::tc::grid_dep_wait();  // s and h come from earlier kernels in the stream
    const int HW4 = HW / 4;
    const int q = blockIdx.x * kThreads + threadIdx.x;  // pixel quad
    if (q >= HW4) return;
    const int b = blockIdx.y;
    const int o_begin = blockIdx.z * kSkipGroup, o_end = min(hidden, o_begin + kSkipGroup);
    const size_t plane0 = static_cast<size_t>(b) * hidden * HW;
    const float4* h4 = reinterpret_cast<const float4*>(h + plane0) + q;
    float4* s4 = reinterpret_cast<float4*>(s + plane0) + q;
    float4 z[kSkipGroup];
#pragma unroll
    for (int t = 0; t < kSkipGroup; ++t) {
        const int o = min(o_begin + t, hidden - 1);
        const float bo = __ldg(bias + o);
        const float4 sv = s4[static_cast<size_t>(o) * HW4];
        z[t] = make_float4(bo + sv.x, bo + sv.y, bo + sv.z, bo + sv.w);
    }
    for (int i0 = 0; i0 < hidden; i0 += kSkipBatch) {
        float4 hv[kSkipBatch];
#pragma unroll
        for (int i = 0; i < kSkipBatch; ++i) hv[i] = __ldg(h4 + static_cast<size_t>(i0 + i) * HW4);
#pragma unroll
        for (int t = 0; t < kSkipGroup; ++t) {
            const float4* wr = reinterpret_cast<const float4*>(ws + min(o_begin + t, hidden - 1) * HMAX + i0);
#pragma unroll
            for (int i4 = 0; i4 < kSkipBatch / 4; ++i4) {
                const float4 wv = wr[i4];
                const float wk[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 hk = hv[4 * i4 + k];
                    z[t].x = fmaf(wk[k], hk.x, z[t].x);
                    z[t].y = fmaf(wk[k], hk.y, z[t].y);
                    z[t].z = fmaf(wk[k], hk.z, z[t].z);
                    z[t].w = fmaf(wk[k], hk.w, z[t].w);
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < kSkipGroup; ++t) {
        const int o = o_begin + t;
        if (o >= o_end) break;
        if (instance_norm) {
            s4[static_cast<size_t>(o) * HW4] = z[t];
        } else {
            reinterpret_cast<float4*>(h_next + plane0)[static_cast<size_t>(o) * HW4 + q] =
                make_float4(gelu_erf(z[t].x), gelu_erf(z[t].y), gelu_erf(z[t].z), gelu_erf(z[t].w));
        }
    }
}

// Sum over the CTA in a fixed order (per-warp butterflies, then warp 0 adds the warp sums in
// warp order); every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // red is free (an earlier call's readers are done)
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kThreads / 32; ++k) t += red[k];
    return t;
}

// Fourier-layer epilogue, part B, one CTA per (b, o) plane: instance statistics in two exact
// passes (mean, then the mean of (z - mean)^2, biased like torch's InstanceNorm2d) and
// h_next = GELU((z - mean) / sqrt(var + eps)) (fno_ns/model.py:96-99,133-134).  A plane of at
// most 16 values per thread (4096 pixels) is read once into registers; larger planes are read
// again for each pass.  grid = B * hidden
constexpr int kNormRegs = 16;

__global__ void __launch_bounds__(kThreads) fno_norm_gelu_kernel(const float* __restrict__ z,
                                                                 float* __restrict__ h_next, int HW) {
    __shared__ float red[kThreads / 32];
    scx::tc::grid_dep_launch();
    scx::tc::grid_dep_wait();  // z comes from the skip kernel
    const size_t plane = blockIdx.x;
    const float* zp = z + plane * HW;
    float* hp = h_next + plane * HW;
    const float inv_n = 1.0f / static_cast<float>(HW);
    if ((HW & 3) == 0 && HW <= kNormRegs * kThreads) {
        // the same with 16-byte accesses: element 4 (tid + k kThreads) + e of the plane
        const float4* z4 = reinterpret_cast<const float4*>(zp);
        float4* h4 = reinterpret_cast<float4*>(hp);
        const int HW4 = HW / 4;
        float4 v[kNormRegs / 4];
#pragma unroll
        for (int k = 0; k < kNormRegs / 4; ++k) {
            const int i = threadIdx.x + k * kThreads;
            v[k] = i < HW4 ? __ldg(z4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < kNormRegs / 4; ++k) sum += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        const float mean = block_sum(sum, red) * inv_n;
        float m2 = 0.f;
#pragma unroll
        for (int k = 0; k < kNormRegs / 4; ++k) {
            if (threadIdx.x + k * kThreads >= HW4) continue;
            const float dx = v[k].x - mean, dy = v[k].y - mean, dz = v[k].z - mean, dw = v[k].w - mean;
            m2 = fmaf(dx, dx, m2);
            m2 = fmaf(dy, dy, m2);
            m2 = fmaf(dz, dz, m2);
            m2 = fmaf(dw, dw, m2);
        }
        const float rstd = 1.0f / sqrtf(block_sum(m2, red) * inv_n + 1e-5f);
#pragma unroll
        for (int k = 0; k < kNormRegs / 4; ++k) {
            const int i = threadIdx.x + k * kThreads;
            if (i < HW4)
                h4[i] = make_float4(gelu_erf((v[k].x - mean) * rstd), gelu_erf((v[k].y - mean) * rstd),
                                    gelu_erf((v[k].z - mean) * rstd), gelu_erf((v[k].w - mean) * rstd));
        }
        return;
    }
    if (HW <= kNormRegs * kThreads) {
        float v[kNormRegs];
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) {
            const int i = threadIdx.x + k * kThreads;
            v[k] = i < HW ? __ldg(zp + i) : 0.f;
        }
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) sum += v[k];
        const float mean = block_sum(sum, red) * inv_n;
        float m2 = 0.f;
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) {
            const int i = threadIdx.x + k * kThreads;
            const float d = i < HW ? v[k] - mean : 0.f;
            m2 = fmaf(d, d, m2);
        }
        const float rstd = 1.0f / sqrtf(block_sum(m2, red) * inv_n + 1e-5f);
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) {
            const int i = threadIdx.x + k * kThreads;
            if (i < HW) hp[i] = gelu_erf((v[k] - mean) * rstd);
        }
        return;
    }
    float sum = 0.f;
    for (int i = threadIdx.x; i < HW; i += kThreads) sum += __ldg(zp + i);
    const float mean = block_sum(sum, red) * inv_n;
    float m2 = 0.f;
    for (int i = threadIdx.x; i < HW; i += kThreads) {
        const float d = __ldg(zp + i) - mean;
        m2 = fmaf(d, d, m2);
    }
    const float rstd = 1.0f / sqrtf(block_sum(m2, red) * inv_n + 1e-5f);
    for (int i = threadIdx.x; i < HW; i += kThreads) hp[i] = gelu_erf((__ldg(zp + i) - mean) * rstd);
}

// Per-channel sums of v[t] over this CTA in a fixed order (warp butterflies, then warp sums
// in warp order), written to out[t] by thread t.  The caller synchronises before reading out.
__device__ __forceinline__ void cta_channel_sums(float (&v)[kSkipGroup], float (*red)[kSkipGroup], float* out) {
#pragma unroll
    for (int t = 0; t < kSkipGroup; ++t)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v[t] += __shfl_xor_sync(0xffffffffu, v[t], off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane < kSkipGroup) {
        float mine = v[0];
#pragma unroll
        for (int t = 1; t < kSkipGroup; ++t) mine = lane == t ? v[t] : mine;
        red[warp][lane] = mine;
    }
    __syncthreads();
    if (threadIdx.x < kSkipGroup) {
        float tot = 0.f;
#pragma unroll
        for (int k = 0; k < kThreads / 32; ++k) tot += red[k][threadIdx.x];
        out[threadIdx.x] = tot;
    }
}

// Fourier-layer epilogue with instance norm in one kernel: the skip GEMM of
// fno_skip_quad_kernel (same z, bit for bit), then the instance statistics of each (b, o)
// plane, then h_next = GELU((z - mean) / sqrt(var + eps)) (fno_ns/model.py:96-99,133-134).
// A thread-block cluster of gridDim.x CTAs (at most 8) covers one plane group: each CTA
// reduces its pixels per output channel, and the partial sums are read from the cluster's
// CTAs through distributed shared memory in rank order, so every CTA gets the same mean and
// variance (two exact passes, biased like torch's InstanceNorm2d).  z stays in registers:
// no z write, no second read, one launch per layer fewer.
// grid = (ceil(HW / (4 * kThreads)), B, ceil(hidden / kSkipGroup)), cluster = (gridDim.x, 1, 1)
template <int HMAX>
__global__ void __launch_bounds__(kThreads, 3) fno_skip_norm_kernel(const float* __restrict__ s,
                                                                 const float* __restrict__ h,
                                                                 float* __restrict__ h_next,
                                                                 const float* __restrict__ w,
                                                                 const float* __restrict__ bias, int HW, int hidden) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    scx::tc::grid_dep_launch();
    __shared__ __align__(16) float ws[HMAX * HMAX];  // [o][i], zero padded
    __shared__ float red[kThreads / 32][kSkipGroup];
    __shared__ float part[2][kSkipGroup];  // this CTA's channel sums: z, then (z - mean)^2
    __shared__ float stat[2][kSkipGroup];  // mean, 1 / sqrt(var + eps)
    for (int i = threadIdx.x; i < HMAX * HMAX; i += kThreads) {
        const int o = i / HMAX, k = i - o * HMAX;
        ws[i] = (o < hidden && k < hidden) ? w[o * hidden + k] : 0.f;
    }
    __syncthreads();
    scx::tc::grid_dep_wait();  // s and h come from earlier kernels in the stream
    const int HW4 = HW / 4;
    const int q = blockIdx.x * kThreads + threadIdx.x;  // pixel quad
    const bool live = q < HW4;  // a thread past the plane computes on quad 0 and contributes nothing
    const int qq = live ? q : 0;
    const int b = blockIdx.y;
    const int o_begin = blockIdx.z * kSkipGroup, o_end = min(hidden, o_begin + kSkipGroup);
    const size_t plane0 = static_cast<size_t>(b) * hidden * HW;
    const float4* h4 = reinterpret_cast<const float4*>(h + plane0) + qq;
    const float4* s4 = reinterpret_cast<const float4*>(s + plane0) + qq;
    float4 z[kSkipGroup];
#pragma unroll
    for (int t = 0; t < kSkipGroup; ++t) {
        const int o = min(o_begin + t, hidden - 1);
        const float bo = __ldg(bias + o);
        const float4 sv = __ldg(s4 + static_cast<size_t>(o) * HW4);
        z[t] = make_float4(bo + sv.x, bo + sv.y, bo + sv.z, bo + sv.w);
    }
    for (int i0 = 0; i0 < hidden; i0 += kSkipBatch) {
        float4 hv[kSkipBatch];
#pragma unroll
        for (int i = 0; i < kSkipBatch; ++i) hv[i] = __ldg(h4 + static_cast<size_t>(i0 + i) * HW4);
#pragma unroll
        for (int t = 0; t < kSkipGroup; ++t) {
            const float4* wr = reinterpret_cast<const float4*>(ws + min(o_begin + t, hidden - 1) * HMAX + i0);
#pragma unroll
            for (int i4 = 0; i4 < kSkipBatch / 4; ++i4) {
                const float4 wv = wr[i4];
                const float wk[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 hk = hv[4 * i4 + k];
                    z[t].x = fmaf(wk[k], hk.x, z[t].x);
                    z[t].y = fmaf(wk[k], hk.y, z[t].y);
                    z[t].z = fmaf(wk[k], hk.z, z[t].z);
                    z[t].w = fmaf(wk[k], hk.w, z[t].w);
                }
            }
        }
    }
    const float inv_n = 1.0f / static_cast<float>(HW);
    const unsigned ranks = cluster.num_blocks();
    // pass 1: mean
    float v[kSkipGroup];
#pragma unroll
    for (int t = 0; t < kSkipGroup; ++t) v[t] = live ? (z[t].x + z[t].y) + (z[t].z + z[t].w) : 0.f;
    cta_channel_sums(v, red, part[0]);
    cluster.sync();  // every CTA's part[0] is written and visible cluster-wide
    if (threadIdx.x < kSkipGroup) {
        float tot = 0.f;
        for (unsigned r = 0; r < ranks; ++r) tot += cluster.map_shared_rank(&part[0][0], r)[threadIdx.x];
        stat[0][threadIdx.x] = tot * inv_n;
    }
    __syncthreads();
    // pass 2: biased variance about the mean
#pragma unroll
    for (int t = 0; t < kSkipGroup; ++t) {
        const float mean = stat[0][t];
        const float dx = z[t].x - mean, dy = z[t].y - mean, dz = z[t].z - mean, dw = z[t].w - mean;
        float m2 = 0.f;
        m2 = fmaf(dx, dx, m2);
        m2 = fmaf(dy, dy, m2);
        m2 = fmaf(dz, dz, m2);
        m2 = fmaf(dw, dw, m2);
        v[t] = live ? m2 : 0.f;
    }
    cta_channel_sums(v, red, part[1]);
    cluster.sync();  // every CTA's part[1] is written and visible cluster-wide
    if (threadIdx.x < kSkipGroup) {
        float tot = 0.f;
        for (unsigned r = 0; r < ranks; ++r) tot += cluster.map_shared_rank(&part[1][0], r)[threadIdx.x];
        stat[1][threadIdx.x] = 1.0f / sqrtf(tot * inv_n + 1e-5f);
    }
    // no CTA leaves (and releases its shared memory) while another may still read its part[];
    // also publishes stat[1] within the CTA
    cluster.sync();
    if (!live) return;
    float4* out4 = reinterpret_cast<float4*>(h_next + plane0) + q;
#pragma unroll
    for (int t = 0; t < kSkipGroup; ++t) {
        const int o = o_begin + t;
        if (o >= o_end) break;
        const float mean = stat[0][t], rstd = stat[1][t];
        const float2 g01 = scx::tc::gelu_pair((z[t].x - mean) * rstd, (z[t].y - mean) * rstd);
        const float2 g23 = scx::tc::gelu_pair((z[t].z - mean) * rstd, (z[t].w - mean) * rstd);
        out4[static_cast<size_t>(o) * HW4] = make_float4(g01.x, g01.y, g23.x, g23.y);
    }
}

// Largest cluster the fused skip+norm kernel is launched with (portable cluster size).
constexpr int kMaxNormCluster = 8;

// Fourier-layer epilogue with instance norm, tiled by pixels with every output channel in one
// CTA (hidden == kTileC, HW a multiple of kTilePx, at most kMaxTileCluster tiles per plane):
//   z[o][p] = s[o][p] + (bias[o] + sum_i Wskip[o][i] h[i][p])
//   h_next[o][p] = GELU((z - mean_o) / sqrt(var_o + eps))              (fno_ns/model.py:96-99,133-134)
// One CTA takes kTilePx pixels of one batch item b, one pixel per thread.  The skip GEMM runs on
// the tensor core: D[pixel][o] = sum_i h[i][pixel] W[o][i] for two M = 128 pixel tiles (N = 32,
// K = 32) in 3xTF32 (hi*hi + hi*lo + lo*hi, hi = the top 19 bits, lo = the exact remainder; fp32
// TMEM accumulators), the same scheme as the FNO projection.  One thread brings the weights, the
// bias (bulk copies) and the tile's h rows (four 2-D tensor copies) into shared memory; each
// thread splits its pixel's 32 channels into the K-major operands, and two threads issue the
// MMAs of one pixel tile each.  Each thread then reads its pixel's 32 accumulators from TMEM
// and adds bias and s (read from global memory while the MMAs run).
// Statistics: z goes to shared memory; eight threads per channel sum 32 pixels each (a rotated
// order keeps the float4 reads free of bank conflicts), then three shuffles, first the CTA's
// channel sum, then its sum of squared deviations about the CTA's own mean.  Each CTA writes the
// pair into every CTA of the cluster (distributed shared memory), and after one cluster barrier
// every CTA combines the partials in rank order (the pairwise variance formula of Chan, Golub and
// LeVeque), so all CTAs of a plane group hold the same mean and biased variance.
// grid = (HW / kTilePx, B), cluster = (HW / kTilePx, 1, 1), kTileThreads threads, dynamic smem
// kTileSmem; th: 2-D fp32 map (HW, B * kTileC) of h with box (kTilePx, kTileGroupRows)
constexpr int kTileC = 32;
constexpr int kTilePx = 256;
constexpr int kTileThreads = kTilePx;
constexpr int kTileGroups = 4;  // tensor copies of the h tile
constexpr int kTileGroupRows = kTileC / kTileGroups;
constexpr int kMaxTileCluster = 16;  // non-portable cluster size, opted into at set-up
constexpr uint32_t kTileA = kTilePx * kTileC * 4u;          // one operand part of both pixel tiles
constexpr size_t kTileSmem = 2ull * kTileA + 1024;          // A hi | A lo, + alignment slack
constexpr uint32_t kTileCols = 2 * kTileC;                  // TMEM: D of pixel tiles 0 and 1

__global__ void __launch_bounds__(kTileThreads, 3) fno_skip_norm_tile_kernel(const __grid_constant__ CUtensorMap th,
                                                                          const float* __restrict__ s,
                                                                          float* __restrict__ h_next,
                                                                          const float* __restrict__ w,
                                                                          const float* __restrict__ bias, int HW,
                                                                          int* watchdog) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    scx::tc::grid_dep_launch();
    extern __shared__ uint8_t tile_raw[];
    // A hi | A lo, K-major SW128 (pixel rows of 32 channels; tile t at t * kTileA / 2).  Before
    // the split, the raw weights land in the A hi area and the raw h tile [i][pixel] in the A lo
    // area; after the MMAs, z [o][pixel] reuses A hi and the cluster partials A lo.
    uint8_t* a_hi = scx::tc::align1024(tile_raw);
    uint8_t* a_lo = a_hi + kTileA;
    float* wraw = reinterpret_cast<float*>(a_hi);
    float* hraw = reinterpret_cast<float*>(a_lo);
    float* zs = reinterpret_cast<float*>(a_hi);
    float2* xpart = reinterpret_cast<float2*>(a_lo);  // [kMaxTileCluster][kTileC]
    __shared__ __align__(1024) uint8_t wsw[2][kTileC * kTileC * 4];  // W hi | W lo, K-major SW128
    __shared__ __align__(16) float bs[kTileC];
    __shared__ float stat[2][kTileC];  // the plane's mean and 1 / sqrt(var + eps)
    __shared__ __align__(8) uint64_t bar[2];  // 0: W, bias and h landed; 1: the MMAs are done
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.y, px0 = blockIdx.x * kTilePx;
    if (warp == 0) {
        scx::tc::tmem_alloc(&tmem_base, kTileCols);
        scx::tc::tmem_relinquish();
    }
    if (tid == 32) {
        scx::tc::mbar_init(&bar[0], 1);
        scx::tc::mbar_init(&bar[1], 2);
        scx::tc::fence_async_smem();
        scx::tc::mbar_arrive_expect_tx(&bar[0], kTileC * kTileC * 4u + kTileC * 4u + kTileA);
        // the weights are not written by the kernels chained before this one
        scx::tc::bulk_g2s(wraw, w, kTileC * kTileC * 4u, &bar[0]);
        scx::tc::bulk_g2s(bs, bias, kTileC * 4u, &bar[0]);
        scx::tc::grid_dep_wait();  // h comes from earlier kernels in the stream
        for (int g = 0; g < kTileGroups; ++g)
            scx::tc::tma_load_2d(hraw + g * kTileGroupRows * kTilePx, &th, px0, b * kTileC + g * kTileGroupRows,
                                 &bar[0]);
    }
    scx::tc::fence_before_sync();
    __syncthreads();  // barriers initialised, TMEM allocated
    scx::tc::fence_after_sync();
    const uint32_t tmem = tmem_base;
    bool ok = scx::tc::mbar_wait_bounded(&bar[0], 0);
    {
        // W [o][i] -> hi / lo, K-major SW128 with N = kTileC rows: four channels per thread
        const int e = tid * 4, o = e / kTileC, i0 = e % kTileC;
        const float4 v = *reinterpret_cast<const float4*>(wraw + e);
        float4 hi, lo;
        scx::tc::split_tf32(v.x, hi.x, lo.x);
        scx::tc::split_tf32(v.y, hi.y, lo.y);
        scx::tc::split_tf32(v.z, hi.z, lo.z);
        scx::tc::split_tf32(v.w, hi.w, lo.w);
        const uint32_t off = scx::tc::kmajor_offset32(kTileC, o, i0);
        *reinterpret_cast<float4*>(&wsw[0][off]) = hi;
        *reinterpret_cast<float4*>(&wsw[1][off]) = lo;
    }
    float hv[kTileC];
#pragma unroll
    for (int i = 0; i < kTileC; ++i) hv[i] = hraw[i * kTilePx + tid];
    __syncthreads();  // the raw tiles have been read: A hi and A lo overwrite them
    {
        const int t = tid >> 7, m = tid & 127;
        uint8_t* ah = a_hi + t * (kTileA / 2);
        uint8_t* al = a_lo + t * (kTileA / 2);
#pragma unroll
        for (int c4 = 0; c4 < kTileC / 4; ++c4) {
            float4 hi, lo;
            scx::tc::split_tf32(hv[4 * c4 + 0], hi.x, lo.x);
            scx::tc::split_tf32(hv[4 * c4 + 1], hi.y, lo.y);
            scx::tc::split_tf32(hv[4 * c4 + 2], hi.z, lo.z);
            scx::tc::split_tf32(hv[4 * c4 + 3], hi.w, lo.w);
            const uint32_t off = scx::tc::kmajor_offset32(128, m, 4 * c4);
            *reinterpret_cast<float4*>(ah + off) = hi;
            *reinterpret_cast<float4*>(al + off) = lo;
        }
    }
    scx::tc::fence_async_smem();  // the operands are visible to the tensor core
    scx::tc::fence_before_sync();
    __syncthreads();
    scx::tc::fence_after_sync();
    if ((tid & 31) == 0 && warp < 2) {
        // pixel tile t = warp: (A hi, W hi), (A hi, W lo), (A lo, W hi), 8 channels per MMA
        const int t = warp;
        const uint64_t dA[2] = {scx::tc::desc_sw128(scx::tc::smem_u32(a_hi + t * (kTileA / 2))),
                                scx::tc::desc_sw128(scx::tc::smem_u32(a_lo + t * (kTileA / 2)))};
        const uint64_t dW[2] = {scx::tc::desc_sw128(scx::tc::smem_u32(&wsw[0][0])),
                                scx::tc::desc_sw128(scx::tc::smem_u32(&wsw[1][0]))};
        constexpr uint32_t id = scx::tc::idesc_tf32(128, kTileC);
        const uint32_t d = tmem + static_cast<uint32_t>(t * kTileC);
#pragma unroll
        for (int part = 0; part < 3; ++part) {
            const int ap = part == 2 ? 1 : 0, bp = part == 1 ? 1 : 0;
#pragma unroll
            for (int ks = 0; ks < kTileC / 8; ++ks)
                scx::tc::mma_tf32(d, dA[ap] + 2u * ks, dW[bp] + 2u * ks, id, (part | ks) ? 1u : 0u);
        }
        scx::tc::mma_commit(&bar[1]);
    }
    // s of this pixel while the MMAs run (written by the kernels chained before this one)
    scx::tc::grid_dep_wait();
    float sv[kTileC];
    const float* sp = s + static_cast<size_t>(b) * kTileC * HW + px0 + tid;
#pragma unroll
    for (int o = 0; o < kTileC; ++o) sv[o] = sp[static_cast<size_t>(o) * HW];
    ok = scx::tc::mbar_wait_bounded(&bar[1], 0) && ok;
    if (!ok && lane == 0) atomicExch(watchdog, 30);
    scx::tc::fence_after_sync();
    {
        // D row of pixel tid: tile warp / 4, TMEM lanes 32 (warp % 4) ..
        float d[kTileC];
        scx::tc::tmem_ld32(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + static_cast<uint32_t>((warp >> 2) * kTileC), d);
#pragma unroll
        for (int o = 0; o < kTileC; ++o) zs[o * kTilePx + tid] = sv[o] + (bs[o] + d[o]);
    }
    // once this barrier phase completes, every CTA of the cluster has started and its MMAs have
    // finished reading A lo, so its partials area may be written; it is waited for before the
    // first remote store
    asm volatile("barrier.cluster.arrive.aligned;" ::: "memory");
    scx::tc::fence_before_sync();
    __syncthreads();  // z complete in shared memory
    scx::tc::fence_after_sync();

    // channel co = tid / 8, pixels [32 ck, 32 ck + 32) with ck = tid % 8, as eight float4 in the
    // rotated order (j + ck) % 8
    const int co = tid >> 3, ck = tid & 7;
    const float4* zr = reinterpret_cast<const float4*>(zs + co * kTilePx) + ck * 8;
    float csum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float4 q = zr[(j + ck) & 7];
        csum += (q.x + q.y) + (q.z + q.w);
    }
    csum += __shfl_xor_sync(0xffffffffu, csum, 1);
    csum += __shfl_xor_sync(0xffffffffu, csum, 2);
    csum += __shfl_xor_sync(0xffffffffu, csum, 4);
    const float cmean = csum * (1.0f / kTilePx);
    float cm2 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float4 q = zr[(j + ck) & 7];
        const float dx = q.x - cmean, dy = q.y - cmean, dz = q.z - cmean, dw = q.w - cmean;
        cm2 += fmaf(dx, dx, dy * dy) + fmaf(dz, dz, dw * dw);
    }
    cm2 += __shfl_xor_sync(0xffffffffu, cm2, 1);
    cm2 += __shfl_xor_sync(0xffffffffu, cm2, 2);
    cm2 += __shfl_xor_sync(0xffffffffu, cm2, 4);
    // push (sum, m2) of channel co into slot `rank` of every CTA of the cluster: the eight
    // threads of the channel take the ranks ck and ck + 8
    const unsigned ranks = cluster.num_blocks(), rank = cluster.block_rank();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // all CTAs have started
    const float2 mine = make_float2(csum, cm2);
    for (unsigned r = ck; r < ranks; r += 8) cluster.map_shared_rank(xpart, r)[rank * kTileC + co] = mine;
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (tid < kTileC) {
        float tot = 0.f;
        for (unsigned r = 0; r < ranks; ++r) tot += xpart[r * kTileC + tid].x;
        const float mean = tot / static_cast<float>(HW);
        float m2 = 0.f;
        for (unsigned r = 0; r < ranks; ++r) {
            const float2 p = xpart[r * kTileC + tid];
            const float d = p.x * (1.0f / kTilePx) - mean;
            m2 += fmaf(static_cast<float>(kTilePx) * d, d, p.y);
        }
        stat[0][tid] = mean;
        stat[1][tid] = 1.0f / sqrtf(m2 / static_cast<float>(HW) + 1e-5f);
    }
    __syncthreads();
    float* out = h_next + static_cast<size_t>(b) * kTileC * HW + px0 + tid;
#pragma unroll
    for (int o = 0; o < kTileC; o += 2) {
        const float z0 = zs[o * kTilePx + tid], z1 = zs[(o + 1) * kTilePx + tid];
        const float2 g = scx::tc::gelu_pair((z0 - stat[0][o]) * stat[1][o], (z1 - stat[0][o + 1]) * stat[1][o + 1]);
        out[static_cast<size_t>(o) * HW] = g.x;
        out[static_cast<size_t>(o + 1) * HW] = g.y;
    }
    if (warp == 0) scx::tc::tmem_dealloc(tmem, kTileCols);
}

// y[b][oc][p] = b2[oc] + sum_j W2[oc][j] GELU(b1[j] + sum_c W1[j][c] h[b][c][p])
// Each thread takes PX pixels (kThreads apart, so loads and stores stay coalesced): one
// shared-memory read of a weight row feeds PX pixels.  Four hidden units per pass give four
// independent FMA chains; each unit's sum keeps its order over c and the output sums take the
// units in order j = 0, 1, ...  grid = (ceil(HW / (kThreads * PX)), B)
template <int HMAX, int PX>
__global__ void __launch_bounds__(kThreads) fno_project_kernel(const float* __restrict__ h, float* __restrict__ y,
                                                               const float* __restrict__ w1,
                                                               const float* __restrict__ b1,
                                                               const float* __restrict__ w2,
                                                               const float* __restrict__ b2, int HW, int hidden,
                                                               int ph, int oc_n) {
    scx::tc::grid_dep_launch();
    extern __shared__ __align__(16) float proj_smem[];
    float* w1s = proj_smem;          // [ph][HMAX] zero padded
    float* b1s = w1s + ph * HMAX;    // [ph]
    float* w2s = b1s + ph;           // [oc][ph]
    for (int i = threadIdx.x; i < ph * HMAX; i += kThreads) {
        const int j = i / HMAX, c = i - j * HMAX;
        w1s[i] = c < hidden ? w1[j * hidden + c] : 0.f;
    }
    for (int i = threadIdx.x; i < ph; i += kThreads) b1s[i] = b1[i];
    for (int i = threadIdx.x; i < oc_n * ph; i += kThreads) w2s[i] = w2[i];
    __syncthreads();
    scx::tc::grid_dep_wait();  // h comes from the last layer's kernels
    const int b = blockIdx.y;
    const int p0 = blockIdx.x * kThreads * PX + threadIdx.x;
    if (p0 >= HW) return;
    constexpr int kMaxOut = 4;
    float hv[PX][HMAX];
#pragma unroll
    for (int x = 0; x < PX; ++x) {
        const int p = min(p0 + x * kThreads, HW - 1);  // a pixel past the plane repeats the last one
        const float* hb = h + static_cast<size_t>(b) * hidden * HW + p;
#pragma unroll
        for (int c = 0; c < HMAX; ++c) hv[x][c] = c < hidden ? __ldg(hb + static_cast<size_t>(c) * HW) : 0.f;
    }
    float out[PX][kMaxOut];
#pragma unroll
    for (int x = 0; x < PX; ++x)
#pragma unroll
        for (int o = 0; o < kMaxOut; ++o) out[x][o] = 0.f;
    for (int j0 = 0; j0 < ph; j0 += 4) {
        float acc[4][PX];
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int x = 0; x < PX; ++x) acc[t][x] = b1s[min(j0 + t, ph - 1)];
#pragma unroll
        for (int c4 = 0; c4 < HMAX / 4; ++c4) {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float4 wv = reinterpret_cast<const float4*>(w1s + min(j0 + t, ph - 1) * HMAX)[c4];
#pragma unroll
                for (int x = 0; x < PX; ++x) {
                    acc[t][x] = fmaf(wv.x, hv[x][4 * c4 + 0], acc[t][x]);
                    acc[t][x] = fmaf(wv.y, hv[x][4 * c4 + 1], acc[t][x]);
                    acc[t][x] = fmaf(wv.z, hv[x][4 * c4 + 2], acc[t][x]);
                    acc[t][x] = fmaf(wv.w, hv[x][4 * c4 + 3], acc[t][x]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            if (j0 + t >= ph) break;
#pragma unroll
            for (int x = 0; x < PX; ++x) {
                const float g = gelu_erf(acc[t][x]);
#pragma unroll
                for (int o = 0; o < kMaxOut; ++o)
                    if (o < oc_n) out[x][o] = fmaf(w2s[o * ph + j0 + t], g, out[x][o]);
            }
        }
    }
#pragma unroll
    for (int x = 0; x < PX; ++x) {
        const int p = p0 + x * kThreads;
        if (p >= HW) break;
#pragma unroll
        for (int o = 0; o < kMaxOut; ++o)
            if (o < oc_n) y[(static_cast<size_t>(b) * oc_n + o) * HW + p] = out[x][o] + b2[o];
    }
}

struct FnoLayout {
    size_t act_bytes, spec_in, spec_out, total;
};

bool fno_valid(const scx_fno2d_config* c) {
    if (!c) return false;
    if (c->batch_size <= 0 || c->height <= 0 || c->width <= 0 || c->in_frames <= 0 || c->hidden <= 0) return false;
    if (c->in_frames + 2 > 64 || c->hidden > 64 || c->proj_hidden <= 0 || c->proj_hidden > 1024) return false;
    if (c->out_channels <= 0 || c->out_channels > 4) return false;
    if (c->n_layers <= 0 || c->n_layers > SCX_FNO_MAX_LAYERS) return false;
    if (c->input_layout != 0 && c->input_layout != 1) return false;
    if (c->instance_norm != 0 && c->instance_norm != 1) return false;
    if (c->modes1 <= 0 || c->modes2 <= 0 || c->modes1 > c->height || c->modes2 > c->width / 2 + 1) return false;
    const long long hw = static_cast<long long>(c->height) * c->width;
    const long long act = static_cast<long long>(c->batch_size) * c->hidden * hw;
    return act < (1LL << 31) && c->batch_size <= 65535;
}

FnoLayout fno_layout(const scx_fno2d_config* c) {
    auto a256 = [](size_t n) { return (n + 255) & ~static_cast<size_t>(255); };
    FnoLayout l;
    const size_t hw = static_cast<size_t>(c->height) * c->width;
    l.act_bytes = a256(static_cast<size_t>(c->batch_size) * c->hidden * hw * 4);
    const size_t corner = static_cast<size_t>(c->batch_size) * c->hidden * c->modes1 * c->modes2 * 8;
    l.spec_in = a256(corner);
    l.spec_out = l.spec_in;
    l.total = 3 * l.act_bytes + 2 * l.spec_in + 2 * l.spec_out;
    return l;
}

int hmax_for(int hidden) { return hidden <= 16 ? 16 : (hidden <= 32 ? 32 : 64); }

template <int HMAX>
cudaError_t run_pixel_kernels_lift(const scx_fno2d_config* cfg, const scx_fno2d_params* prm, const float* x,
                                   float* h0, cudaStream_t s) {
    const int HW = cfg->height * cfg->width;
    const dim3 grid((HW + kThreads - 1) / kThreads, cfg->batch_size);
    const size_t smem = static_cast<size_t>(cfg->in_frames + 2) * HMAX * 4;
    return scx::launch_chained(fno_lift_kernel<HMAX>, grid, dim3(kThreads), smem, s, x, h0, prm->lift_w, prm->lift_b,
                               cfg->height, cfg->width, cfg->in_frames, cfg->hidden, cfg->input_layout);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// A [rows][HW] fp32 activation as a 2-D tensor map with box (kTilePx, kTileGroupRows), through the
// runtime's driver entry point (no libcuda link).
bool encode_act_map(CUtensorMap* m, const float* ptr, int HW, int rows) {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(HW), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(HW) * 4};
    const cuuint32_t box[2] = {kTilePx, kTileGroupRows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Whether the pixel-tiled skip+norm kernel can run with clusters of `ctas` CTAs on the current
// device.  Set-up (non-portable cluster size, dynamic shared memory, an occupancy check) runs
// once per device and cluster size.
bool tile_norm_ready(int ctas) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    static std::mutex m;
    static std::map<std::pair<int, int>, bool> seen;
    std::lock_guard<std::mutex> lock(m);
    const auto key = std::make_pair(dev, ctas);
    auto it = seen.find(key);
    if (it != seen.end()) return it->second;
    bool ok = cudaFuncSetAttribute(fno_skip_norm_tile_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                  cudaSuccess &&
              cudaFuncSetAttribute(fno_skip_norm_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kTileSmem)) == cudaSuccess;
    if (ok) {
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(ctas, 1, 1);
        lc.blockDim = dim3(kTileThreads);
        lc.dynamicSmemBytes = kTileSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = ctas;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
        int clusters = 0;
        ok = cudaOccupancyMaxActiveClusters(&clusters, fno_skip_norm_tile_kernel, &lc) == cudaSuccess && clusters > 0;
    }
    cudaGetLastError();  // a refused attribute or query leaves no sticky error behind
    seen[key] = ok;
    return ok;
}

template <int HMAX>
cudaError_t run_layer_epilogue(const scx_fno2d_config* cfg, float* spec, const float* h, float* h_next, const float* w, const float* bias, cudaStream_t s) {
    const int HW = cfg->height * cfg->width;
    cudaError_t e;
    const int tiles = HW / kTilePx;
    if (cfg->instance_norm && cfg->hidden == kTileC && HW % kTilePx == 0 && tiles >= 1 && tiles <= kMaxTileCluster &&
        ((reinterpret_cast<uintptr_t>(spec) | reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(h_next) |
          reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(bias)) & 15) == 0 &&
        tile_norm_ready(tiles)) {
        int* wd = nullptr;
        e = scx::device_watchdog(&wd);
        if (e != cudaSuccess) return e;
        CUtensorMap th;
        if (!encode_act_map(&th, h, HW, cfg->batch_size * cfg->hidden)) return cudaErrorInvalidValue;
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(tiles, cfg->batch_size, 1);
        lc.blockDim = dim3(kTileThreads);
        lc.dynamicSmemBytes = kTileSmem;
        lc.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = tiles;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        lc.attrs = attr;
        lc.numAttrs = 2;
        return cudaLaunchKernelEx(&lc, fno_skip_norm_tile_kernel, th, static_cast<const float*>(spec), h_next, w, bias,
                                  HW, wd);
    }
    const bool quads = HW % 4 == 0 && cfg->hidden % 16 == 0 &&
                       ((reinterpret_cast<uintptr_t>(spec) | reinterpret_cast<uintptr_t>(h) |
                         reinterpret_cast<uintptr_t>(h_next)) & 15) == 0;
    const int cluster = (HW / 4 + kThreads - 1) / kThreads;  // CTAs per plane in the quad layout
    if (quads && cfg->instance_norm && cluster <= kMaxNormCluster) {
        // skip GEMM, statistics and GELU in one launch: a cluster of CTAs per plane group
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(cluster, cfg->batch_size, (cfg->hidden + kSkipGroup - 1) / kSkipGroup);
        lc.blockDim = dim3(kThreads);
        lc.dynamicSmemBytes = 0;
        lc.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = cluster;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        lc.attrs = attr;
        lc.numAttrs = 2;
        return cudaLaunchKernelEx(&lc, fno_skip_norm_kernel<HMAX>, static_cast<const float*>(spec), h, h_next, w,
                                  bias, HW, cfg->hidden);
    }
    if (quads) {
        const dim3 grid((HW / 4 + kThreads - 1) / kThreads, cfg->batch_size, (cfg->hidden + kSkipGroup - 1) / kSkipGroup);
        e = scx::launch_chained(fno_skip_quad_kernel<HMAX>, grid, dim3(kThreads), 0, s, spec, h, h_next, w, bias, HW,
                                cfg->hidden, cfg->instance_norm);
    } else {
        constexpr int PX = HMAX <= 32 ? 2 : 1;  // pixels per thread within the register budget
        const dim3 grid((HW + kThreads * PX - 1) / (kThreads * PX), cfg->batch_size,
                        (cfg->hidden + kSkipGroup - 1) / kSkipGroup);
        e = scx::launch_chained(fno_skip_kernel<HMAX, PX>, grid, dim3(kThreads), 0, s, spec, h, h_next, w, bias, HW,
                                cfg->hidden, cfg->instance_norm);
    }
    if (e != cudaSuccess || !cfg->instance_norm) return e;
    return scx::launch_chained(fno_norm_gelu_kernel, dim3(static_cast<unsigned>(cfg->batch_size * cfg->hidden)),
                               dim3(kThreads), 0, s, spec, h_next, HW);
}

template <int HMAX>
cudaError_t run_project(const scx_fno2d_config* cfg, const scx_fno2d_params* prm, const float* h, float* y,
                        cudaStream_t s) {
    const int HW = cfg->height * cfg->width;
    if (scx::fno_project_tc_supported(cfg->hidden, cfg->proj_hidden, cfg->out_channels, HW) &&
        ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(prm->proj1_w)) & 15) == 0)
        return scx::launch_fno_project_tc(h, y, prm->proj1_w, prm->proj1_b, prm->proj2_w, prm->proj2_b,
                                          cfg->batch_size, HW, cfg->hidden, cfg->proj_hidden, cfg->out_channels, s);
    // FFMA fallback, one pixel per thread: with two, the 128-unit loop runs on too few warps to
    // hide its latency
    constexpr int PX = 1;
    const dim3 grid((HW + kThreads * PX - 1) / (kThreads * PX), cfg->batch_size);
    const size_t smem = static_cast<size_t>(cfg->proj_hidden * HMAX + cfg->proj_hidden +
                                            cfg->out_channels * cfg->proj_hidden) * 4;
    int per_sm = 1;
    cudaError_t e = scx::prepare_kernel(reinterpret_cast<const void*>(fno_project_kernel<HMAX, PX>), smem, kThreads,
                                        &per_sm);
    if (e != cudaSuccess) return e;
    return scx::launch_chained(fno_project_kernel<HMAX, PX>, grid, dim3(kThreads), smem, s, h, y, prm->proj1_w,
                               prm->proj1_b, prm->proj2_w, prm->proj2_b, HW, cfg->hidden, cfg->proj_hidden,
                               cfg->out_channels);
}

}  // namespace

extern "C" size_t scx_fno2d_workspace_size(const scx_fno2d_config* cfg) {
    if (!fno_valid(cfg)) return 0;
    return fno_layout(cfg).total;
}

extern "C" int scx_fno2d_fwd(const scx_fno2d_config* cfg, const scx_fno2d_params* prm, const float* x, float* y,
                             void* workspace, size_t workspace_bytes, scx_stream_t stream) {
    if (!fno_valid(cfg) || !prm || !x || !y || !workspace) return cudaErrorInvalidValue;
    const FnoLayout L = fno_layout(cfg);
    if (workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) % 256) != 0) return cudaErrorInvalidValue;
    if (!prm->lift_w || !prm->lift_b || !prm->proj1_w || !prm->proj1_b || !prm->proj2_w || !prm->proj2_b)
        return cudaErrorInvalidValue;
    for (int l = 0; l < cfg->n_layers; ++l)
        if (!prm->spectral_w1[l] || !prm->spectral_w2[l] || !prm->skip_w[l] || !prm->skip_b[l])
            return cudaErrorInvalidValue;
    const int B = cfg->batch_size, H = cfg->height, W = cfg->width, C = cfg->hidden;
    const int m1 = cfg->modes1, m2 = cfg->modes2;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const scx::Twiddles* tw = nullptr;
    cudaError_t e = scx::get_twiddles(H, W, m1, m2, &tw);
    if (e != cudaSuccess) return e;

    unsigned char* base = static_cast<unsigned char*>(workspace);
    float* act[3] = {reinterpret_cast<float*>(base), reinterpret_cast<float*>(base + L.act_bytes),
                     reinterpret_cast<float*>(base + 2 * L.act_bytes)};
    unsigned char* sp = base + 3 * L.act_bytes;
    float2* X1 = reinterpret_cast<float2*>(sp);
    float2* X2 = reinterpret_cast<float2*>(sp + L.spec_in);
    float2* Y1 = reinterpret_cast<float2*>(sp + 2 * L.spec_in);
    float2* Y2 = reinterpret_cast<float2*>(sp + 2 * L.spec_in + L.spec_out);
    const int hmax = hmax_for(C);

    e = hmax == 16 ? run_pixel_kernels_lift<16>(cfg, prm, x, act[0], s)
                   : (hmax == 32 ? run_pixel_kernels_lift<32>(cfg, prm, x, act[0], s)
                                 : run_pixel_kernels_lift<64>(cfg, prm, x, act[0], s));
    if (e != cudaSuccess) return e;
    // Fourier layers: act[cur] -> spectral conv -> act[spec] (overwritten by z) -> act[nxt]
    const long long NM = static_cast<long long>(m1) * m2;
    int cur = 0;
    for (int l = 0; l < cfg->n_layers; ++l) {
        const int spec = (cur + 1) % 3, nxt = (cur + 2) % 3;
        e = scx::dft_fwd(act[cur], X1, X2, NM, m2, B * C, H, W, m1, m2, *tw, s);
        if (e != cudaSuccess) return e;
        e = scx::launch_mix(X1, X2, reinterpret_cast<const float2*>(prm->spectral_w1[l]),
                            reinterpret_cast<const float2*>(prm->spectral_w2[l]), Y1, Y2, 2, B, C, C,
                            static_cast<int>(NM), s, true);  // weights are not written in the forward
        if (e != cudaSuccess) return e;
        e = scx::dft_inv(Y1, Y2, NM, m2, act[spec], B * C, H, W, m1, m2, *tw, s);
        if (e != cudaSuccess) return e;
        e = hmax == 16 ? run_layer_epilogue<16>(cfg, act[spec], act[cur], act[nxt], prm->skip_w[l], prm->skip_b[l], s)
                       : (hmax == 32 ? run_layer_epilogue<32>(cfg, act[spec], act[cur], act[nxt], prm->skip_w[l],
                                                              prm->skip_b[l], s)
                                     : run_layer_epilogue<64>(cfg, act[spec], act[cur], act[nxt], prm->skip_w[l],
                                                              prm->skip_b[l], s));
        if (e != cudaSuccess) return e;
        cur = nxt;
    }
    return hmax == 16 ? run_project<16>(cfg, prm, act[cur], y, s)
                      : (hmax == 32 ? run_project<32>(cfg, prm, act[cur], y, s)
                                    : run_project<64>(cfg, prm, act[cur], y, s));
}
