// FNO-2d forward (fno_ns/model.py:137-259) as one C-ABI call.
//
// Kernels besides the spectral convolution (scx_dft_*.cu, scx_mix.cu):
//   fno_lift_kernel            1x1 conv (T+2 -> hidden) with the grid channels generated
//                              in-kernel (fno_ns/model.py:168-181,193-195) or read from a
//                              channels-last input
//   fno_skip_kernel            per pixel: z = spectral + W h + b for every output channel,
//                              plus per-warp (mean, M2) partial statistics of each plane
//   fno_norm_gelu_kernel       instance statistics combined exactly (Chan's formula), then
//                              normalisation and GELU (fno_ns/model.py:96-99,133-134)
//   fno_project_kernel         per pixel: hidden -> proj_hidden (GELU) -> out_channels, the
//                              proj_hidden-wide intermediate never leaves registers
//                              (fno_ns/model.py:162-166)
#include <algorithm>
#include <cmath>

#include "scx.h"
#include "scx_internal.h"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float gelu_erf(float z) { return 0.5f * z * (1.0f + erff(z * 0.70710678118654752f)); }

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
    extern __shared__ float lift_smem[];
    const int cin = T + 2;
    float* ws = lift_smem;  // [cin][HMAX] (transposed: one input channel's weights contiguous)
    for (int i = threadIdx.x; i < cin * HMAX; i += kThreads) {
        const int k = i / HMAX, c = i - k * HMAX;
        ws[i] = c < hidden ? w[c * cin + k] : 0.f;
    }
    __syncthreads();
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

// Fourier-layer epilogue, part A (one thread per pixel):
//   z[b][o][p] = s[b][o][p] + bias[o] + sum_i Wskip[o][i] h[b][i][p]    (written over s)
// With instance_norm it also writes, per warp of 32 pixels and channel, the partial
// statistics (mean, M2 = sum (z - mean)^2) to part[b][o][warp]; without it, it writes
// GELU(z) to h_next directly.  grid = (ceil(HW / 256), B)
template <int HMAX>
__global__ void __launch_bounds__(kThreads) fno_skip_kernel(float* __restrict__ s, const float* __restrict__ h,
                                                            float* __restrict__ h_next, float2* __restrict__ part,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ bias, int HW, int hidden,
                                                            int instance_norm) {
    __shared__ __align__(16) float ws[HMAX * HMAX];  // [o][i], zero padded
    for (int i = threadIdx.x; i < HMAX * HMAX; i += kThreads) {
        const int o = i / HMAX, k = i - o * HMAX;
        ws[i] = (o < hidden && k < hidden) ? w[o * hidden + k] : 0.f;
    }
    __syncthreads();
    const int b = blockIdx.y;
    const int p = blockIdx.x * kThreads + threadIdx.x;
    const bool valid = p < HW;
    const int pp = valid ? p : 0;
    float hv[HMAX];
    const float* hb = h + static_cast<size_t>(b) * hidden * HW + pp;
#pragma unroll
    for (int i = 0; i < HMAX; ++i) hv[i] = i < hidden ? __ldg(hb + static_cast<size_t>(i) * HW) : 0.f;
    float* sb = s + static_cast<size_t>(b) * hidden * HW + pp;
    const int lane = threadIdx.x & 31;
    const int nwarps_plane = (HW + 31) / 32;
    const int gwarp = p / 32;  // warp index within the plane
    for (int o = 0; o < hidden; ++o) {
        const float4* wr = reinterpret_cast<const float4*>(ws + o * HMAX);
        float z = __ldg(bias + o) + (valid ? sb[static_cast<size_t>(o) * HW] : 0.f);
#pragma unroll
        for (int i4 = 0; i4 < HMAX / 4; ++i4) {
            const float4 wv = wr[i4];
            z = fmaf(wv.x, hv[4 * i4 + 0], z);
            z = fmaf(wv.y, hv[4 * i4 + 1], z);
            z = fmaf(wv.z, hv[4 * i4 + 2], z);
            z = fmaf(wv.w, hv[4 * i4 + 3], z);
        }
        if (!instance_norm) {
            if (valid) h_next[(static_cast<size_t>(b) * hidden + o) * HW + p] = gelu_erf(z);
            continue;
        }
        if (valid) sb[static_cast<size_t>(o) * HW] = z;
        // warp partials over the valid pixels of this warp (a warp wholly past the plane
        // has none; the condition is uniform across the warp)
        const int wstart = gwarp * 32;
        if (wstart >= HW) continue;
        const int n = min(32, HW - wstart);
        float sum = valid ? z : 0.f;
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        const float mean = sum / static_cast<float>(n);
        const float d = valid ? z - mean : 0.f;
        float m2 = d * d;
        for (int off = 16; off > 0; off >>= 1) m2 += __shfl_xor_sync(0xffffffffu, m2, off);
        if (lane == 0) part[(static_cast<size_t>(b) * hidden + o) * nwarps_plane + gwarp] = make_float2(mean, m2);
    }
}

// Fourier-layer epilogue, part B: combines the warp partials of each (b, o) plane with
// Chan's parallel-variance formula (mean = sum n_w mean_w / N, M2 = sum [M2_w + n_w
// (mean_w - mean)^2]) and writes h_next = GELU((z - mean) / sqrt(M2 / N + eps)).
// grid = (ceil(HW / 256), B); each block recombines the statistics of its batch item.
template <int HMAX>
__global__ void __launch_bounds__(kThreads) fno_norm_gelu_kernel(const float* __restrict__ z,
                                                                 float* __restrict__ h_next,
                                                                 const float2* __restrict__ part, int HW,
                                                                 int hidden) {
    __shared__ float mean_s[HMAX], rstd_s[HMAX];
    const int b = blockIdx.y;
    const int nw = (HW + 31) / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = warp; o < hidden; o += kThreads / 32) {
        const float2* pp = part + (static_cast<size_t>(b) * hidden + o) * nw;
        float sum = 0.f;
        for (int k = lane; k < nw; k += 32) {
            const int n = min(32, HW - k * 32);
            sum += pp[k].x * static_cast<float>(n);
        }
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        const float mean = sum / static_cast<float>(HW);
        float m2 = 0.f;
        for (int k = lane; k < nw; k += 32) {
            const int n = min(32, HW - k * 32);
            const float d = pp[k].x - mean;
            m2 += pp[k].y + static_cast<float>(n) * d * d;
        }
        for (int off = 16; off > 0; off >>= 1) m2 += __shfl_xor_sync(0xffffffffu, m2, off);
        if (lane == 0) {
            mean_s[o] = mean;
            rstd_s[o] = 1.0f / sqrtf(m2 / static_cast<float>(HW) + 1e-5f);
        }
    }
    __syncthreads();
    const int p = blockIdx.x * kThreads + threadIdx.x;
    if (p >= HW) return;
    const size_t base = static_cast<size_t>(b) * hidden * HW + p;
    for (int o = 0; o < hidden; ++o) {
        const size_t i = base + static_cast<size_t>(o) * HW;
        h_next[i] = gelu_erf((z[i] - mean_s[o]) * rstd_s[o]);
    }
}

// y[b][oc][p] = b2[oc] + sum_j W2[oc][j] GELU(b1[j] + sum_c W1[j][c] h[b][c][p])
// grid = (ceil(HW / 256), B)
template <int HMAX>
__global__ void __launch_bounds__(kThreads) fno_project_kernel(const float* __restrict__ h, float* __restrict__ y,
                                                               const float* __restrict__ w1,
                                                               const float* __restrict__ b1,
                                                               const float* __restrict__ w2,
                                                               const float* __restrict__ b2, int HW, int hidden,
                                                               int ph, int oc_n) {
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
    const int b = blockIdx.y;
    const int p = blockIdx.x * kThreads + threadIdx.x;
    if (p >= HW) return;
    constexpr int kMaxOut = 4;
    float hv[HMAX];
    const float* hb = h + static_cast<size_t>(b) * hidden * HW + p;
#pragma unroll
    for (int c = 0; c < HMAX; ++c) hv[c] = c < hidden ? __ldg(hb + static_cast<size_t>(c) * HW) : 0.f;
    float out[kMaxOut];
#pragma unroll
    for (int o = 0; o < kMaxOut; ++o) out[o] = 0.f;
    for (int j = 0; j < ph; ++j) {
        const float4* wr = reinterpret_cast<const float4*>(w1s + j * HMAX);
        float acc = b1s[j];
#pragma unroll
        for (int c4 = 0; c4 < HMAX / 4; ++c4) {
            const float4 wv = wr[c4];
            acc = fmaf(wv.x, hv[4 * c4 + 0], acc);
            acc = fmaf(wv.y, hv[4 * c4 + 1], acc);
            acc = fmaf(wv.z, hv[4 * c4 + 2], acc);
            acc = fmaf(wv.w, hv[4 * c4 + 3], acc);
        }
        const float g = gelu_erf(acc);
#pragma unroll
        for (int o = 0; o < kMaxOut; ++o)
            if (o < oc_n) out[o] = fmaf(w2s[o * ph + j], g, out[o]);
    }
#pragma unroll
    for (int o = 0; o < kMaxOut; ++o)
        if (o < oc_n) y[(static_cast<size_t>(b) * oc_n + o) * HW + p] = out[o] + b2[o];
}

struct FnoLayout {
    size_t act_bytes, spec_in, spec_out, part_bytes, total;
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
    l.part_bytes = a256(static_cast<size_t>(c->batch_size) * c->hidden * ((hw + 31) / 32) * sizeof(float2));
    l.total = 3 * l.act_bytes + 2 * l.spec_in + 2 * l.spec_out + l.part_bytes;
    return l;
}

int hmax_for(int hidden) { return hidden <= 16 ? 16 : (hidden <= 32 ? 32 : 64); }

template <int HMAX>
cudaError_t run_pixel_kernels_lift(const scx_fno2d_config* cfg, const scx_fno2d_params* prm, const float* x,
                                   float* h0, cudaStream_t s) {
    const int HW = cfg->height * cfg->width;
    const dim3 grid((HW + kThreads - 1) / kThreads, cfg->batch_size);
    const size_t smem = static_cast<size_t>(cfg->in_frames + 2) * HMAX * 4;
    fno_lift_kernel<HMAX><<<grid, kThreads, smem, s>>>(x, h0, prm->lift_w, prm->lift_b, cfg->height, cfg->width,
                                                       cfg->in_frames, cfg->hidden, cfg->input_layout);
    return cudaGetLastError();
}

template <int HMAX>
cudaError_t run_layer_epilogue(const scx_fno2d_config* cfg, float* spec, const float* h, float* h_next, float2* part,
                               const float* w, const float* bias, cudaStream_t s) {
    const int HW = cfg->height * cfg->width;
    const dim3 grid((HW + kThreads - 1) / kThreads, cfg->batch_size);
    fno_skip_kernel<HMAX><<<grid, kThreads, 0, s>>>(spec, h, h_next, part, w, bias, HW, cfg->hidden,
                                                    cfg->instance_norm);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !cfg->instance_norm) return e;
    fno_norm_gelu_kernel<HMAX><<<grid, kThreads, 0, s>>>(spec, h_next, part, HW, cfg->hidden);
    return cudaGetLastError();
}

template <int HMAX>
cudaError_t run_project(const scx_fno2d_config* cfg, const scx_fno2d_params* prm, const float* h, float* y,
                        cudaStream_t s) {
    const int HW = cfg->height * cfg->width;
    const dim3 grid((HW + kThreads - 1) / kThreads, cfg->batch_size);
    const size_t smem = static_cast<size_t>(cfg->proj_hidden * HMAX + cfg->proj_hidden +
                                            cfg->out_channels * cfg->proj_hidden) * 4;
    int per_sm = 1;
    cudaError_t e = scx::prepare_kernel(reinterpret_cast<const void*>(fno_project_kernel<HMAX>), smem, kThreads,
                                        &per_sm);
    if (e != cudaSuccess) return e;
    fno_project_kernel<HMAX><<<grid, kThreads, smem, s>>>(h, y, prm->proj1_w, prm->proj1_b, prm->proj2_w,
                                                          prm->proj2_b, HW, cfg->hidden, cfg->proj_hidden,
                                                          cfg->out_channels);
    return cudaGetLastError();
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
    float2* part = reinterpret_cast<float2*>(sp + 2 * L.spec_in + 2 * L.spec_out);
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
                            static_cast<int>(NM), s);
        if (e != cudaSuccess) return e;
        e = scx::dft_inv(Y1, Y2, NM, m2, act[spec], B * C, H, W, m1, m2, *tw, s);
        if (e != cudaSuccess) return e;
        e = hmax == 16 ? run_layer_epilogue<16>(cfg, act[spec], act[cur], act[nxt], part, prm->skip_w[l],
                                                prm->skip_b[l], s)
                       : (hmax == 32 ? run_layer_epilogue<32>(cfg, act[spec], act[cur], act[nxt], part,
                                                              prm->skip_w[l], prm->skip_b[l], s)
                                     : run_layer_epilogue<64>(cfg, act[spec], act[cur], act[nxt], part,
                                                              prm->skip_w[l], prm->skip_b[l], s));
        if (e != cudaSuccess) return e;
        cur = nxt;
    }
    return hmax == 16 ? run_project<16>(cfg, prm, act[cur], y, s)
                      : (hmax == 32 ? run_project<32>(cfg, prm, act[cur], y, s)
                                    : run_project<64>(cfg, prm, act[cur], y, s));
}
