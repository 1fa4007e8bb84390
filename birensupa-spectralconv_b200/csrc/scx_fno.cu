// FNO-2d forward (fno_ns/model.py:137-259) as one C-ABI call.
//
// Kernels besides the spectral convolution (scx_dft_*.cu, scx_mix.cu):
//   fno_lift_kernel            1x1 conv (T+2 -> hidden) with the grid channels generated
//                              in-kernel (fno_ns/model.py:168-181,193-195) or read from a
//                              channels-last input
//   fno_skip_norm_gelu_kernel  per (batch, group of output channels): z = spectral + W h + b
//                              over the whole plane kept in shared memory, then instance
//                              statistics, normalisation and GELU (fno_ns/model.py:96-99,133-134)
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
// grid = (ceil(HW / 256), B)
__global__ void __launch_bounds__(kThreads) fno_lift_kernel(const float* __restrict__ x, float* __restrict__ h,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ bias, int H, int W, int T,
                                                            int hidden, int layout) {
    extern __shared__ float lift_smem[];
    const int cin = T + 2;
    float* ws = lift_smem;              // [hidden][cin]
    float* bs = lift_smem + hidden * cin;  // [hidden]
    for (int i = threadIdx.x; i < hidden * cin; i += kThreads) ws[i] = w[i];
    for (int i = threadIdx.x; i < hidden; i += kThreads) bs[i] = bias[i];
    __syncthreads();
    const int HW = H * W;
    const int b = blockIdx.y;
    const int p = blockIdx.x * kThreads + threadIdx.x;
    if (p >= HW) return;
    const int row = p / W, col = p - row * W;
    float in[64];
    const int nin = min(cin, 64);
    if (layout == 0) {
        const float* xb = x + static_cast<size_t>(b) * T * HW + p;
        for (int k = 0; k < T && k < 62; ++k) in[k] = __ldg(xb + static_cast<size_t>(k) * HW);
        in[T] = linspace01(row, H);
        in[T + 1] = linspace01(col, W);
    } else {
        const float* xp = x + (static_cast<size_t>(b) * HW + p) * cin;
        for (int k = 0; k < nin; ++k) in[k] = __ldg(xp + k);
    }
    float* hb = h + static_cast<size_t>(b) * hidden * HW + p;
    for (int c = 0; c < hidden; ++c) {
        float acc = bs[c];
        const float* wc = ws + c * cin;
        for (int k = 0; k < nin; ++k) acc = fmaf(wc[k], in[k], acc);
        hb[static_cast<size_t>(c) * HW] = acc;
    }
}

// h_next[b][o] = GELU(IN(s[b][o] + sum_i W[o][i] h[b][i] + bias[o])) for OG output
// channels o per block.  grid = (ceil(hidden / OG), B); dynamic smem OG*HW floats + weights.
__global__ void __launch_bounds__(kThreads) fno_skip_norm_gelu_kernel(
    const float* __restrict__ s, const float* __restrict__ h, float* __restrict__ h_next,
    const float* __restrict__ w, const float* __restrict__ bias, int HW, int hidden, int OG, int instance_norm) {
    extern __shared__ float skip_smem[];
    const int b = blockIdx.y;
    const int o0 = blockIdx.x * OG;
    const int og_n = min(OG, hidden - o0);
    float* z = skip_smem;                        // [OG][HW]
    float* wsh = skip_smem + static_cast<size_t>(OG) * HW;  // [OG][hidden]
    float* red = wsh + OG * hidden;              // [2 * kThreads / 32]
    for (int i = threadIdx.x; i < og_n * hidden; i += kThreads) wsh[i] = w[static_cast<size_t>(o0) * hidden + i];
    __syncthreads();
    const float* hb = h + static_cast<size_t>(b) * hidden * HW;
    const float* sb = s + (static_cast<size_t>(b) * hidden + o0) * HW;
    constexpr int kMaxOG = 16;
    for (int p = threadIdx.x; p < HW; p += kThreads) {
        float acc[kMaxOG];
#pragma unroll
        for (int j = 0; j < kMaxOG; ++j) acc[j] = 0.f;
        for (int i = 0; i < hidden; ++i) {
            const float hv = __ldg(hb + static_cast<size_t>(i) * HW + p);
#pragma unroll
            for (int j = 0; j < kMaxOG; ++j)
                if (j < og_n) acc[j] = fmaf(wsh[j * hidden + i], hv, acc[j]);
        }
#pragma unroll
        for (int j = 0; j < kMaxOG; ++j)
            if (j < og_n) z[static_cast<size_t>(j) * HW + p] = acc[j] + bias[o0 + j] + __ldg(sb + static_cast<size_t>(j) * HW + p);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int j = 0; j < og_n; ++j) {
        float* zj = z + static_cast<size_t>(j) * HW;
        float mean = 0.f, rstd = 1.f;
        if (instance_norm) {
            float sum = 0.f;
            for (int p = threadIdx.x; p < HW; p += kThreads) sum += zj[p];
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            if (lane == 0) red[warp] = sum;
            __syncthreads();
            float tot = 0.f;
            for (int k = 0; k < kThreads / 32; ++k) tot += red[k];
            mean = tot / static_cast<float>(HW);
            float sq = 0.f;
            for (int p = threadIdx.x; p < HW; p += kThreads) {
                const float d = zj[p] - mean;
                sq = fmaf(d, d, sq);
            }
            for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
            if (lane == 0) red[kThreads / 32 + warp] = sq;
            __syncthreads();
            float tsq = 0.f;
            for (int k = 0; k < kThreads / 32; ++k) tsq += red[kThreads / 32 + k];
            rstd = 1.0f / sqrtf(tsq / static_cast<float>(HW) + 1e-5f);
        }
        float* out = h_next + (static_cast<size_t>(b) * hidden + o0 + j) * HW;
        for (int p = threadIdx.x; p < HW; p += kThreads) out[p] = gelu_erf((zj[p] - mean) * rstd);
        __syncthreads();  // red[] is reused by the next channel
    }
}

// y[b][oc][p] = b2[oc] + sum_j W2[oc][j] GELU(b1[j] + sum_c W1[j][c] h[b][c][p])
// grid = (ceil(HW / 256), B)
__global__ void __launch_bounds__(kThreads) fno_project_kernel(const float* __restrict__ h, float* __restrict__ y,
                                                               const float* __restrict__ w1,
                                                               const float* __restrict__ b1,
                                                               const float* __restrict__ w2,
                                                               const float* __restrict__ b2, int HW, int hidden,
                                                               int ph, int oc_n) {
    extern __shared__ float proj_smem[];
    float* w1s = proj_smem;               // [ph][hidden]
    float* b1s = w1s + ph * hidden;       // [ph]
    float* w2s = b1s + ph;                // [oc][ph]
    for (int i = threadIdx.x; i < ph * hidden; i += kThreads) w1s[i] = w1[i];
    for (int i = threadIdx.x; i < ph; i += kThreads) b1s[i] = b1[i];
    for (int i = threadIdx.x; i < oc_n * ph; i += kThreads) w2s[i] = w2[i];
    __syncthreads();
    const int b = blockIdx.y;
    const int p = blockIdx.x * kThreads + threadIdx.x;
    if (p >= HW) return;
    constexpr int kMaxHidden = 64;
    constexpr int kMaxOut = 4;
    float hv[kMaxHidden];
    const float* hb = h + static_cast<size_t>(b) * hidden * HW + p;
#pragma unroll
    for (int c = 0; c < kMaxHidden; ++c)
        if (c < hidden) hv[c] = __ldg(hb + static_cast<size_t>(c) * HW);
    float out[kMaxOut];
#pragma unroll
    for (int o = 0; o < kMaxOut; ++o) out[o] = 0.f;
    for (int j = 0; j < ph; ++j) {
        const float* wr = w1s + j * hidden;
        float acc = b1s[j];
#pragma unroll
        for (int c = 0; c < kMaxHidden; ++c)
            if (c < hidden) acc = fmaf(wr[c], hv[c], acc);
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
    // one whole plane per output channel stays in shared memory in the skip/norm kernel
    if (hw * 4 > 160 * 1024) return false;
    const long long act = static_cast<long long>(c->batch_size) * c->hidden * hw;
    return act < (1LL << 31);
}

FnoLayout fno_layout(const scx_fno2d_config* c) {
    FnoLayout l;
    const size_t hw = static_cast<size_t>(c->height) * c->width;
    l.act_bytes = ((static_cast<size_t>(c->batch_size) * c->hidden * hw * 4) + 255) & ~static_cast<size_t>(255);
    const size_t corner = static_cast<size_t>(c->batch_size) * c->hidden * c->modes1 * c->modes2 * 8;
    l.spec_in = (corner + 255) & ~static_cast<size_t>(255);
    l.spec_out = l.spec_in;
    l.total = 3 * l.act_bytes + 2 * l.spec_in + 2 * l.spec_out;
    return l;
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
    const int HW = H * W;
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

    // lift
    const int cin = cfg->in_frames + 2;
    const dim3 pix_grid((HW + kThreads - 1) / kThreads, B);
    const size_t lift_smem = static_cast<size_t>(C * cin + C) * 4;
    fno_lift_kernel<<<pix_grid, kThreads, lift_smem, s>>>(x, act[0], prm->lift_w, prm->lift_b, H, W, cfg->in_frames,
                                                          C, cfg->input_layout);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    // Fourier layers: act[cur] -> spectral -> act[spec]; skip/norm/GELU -> act[nxt]
    int OG = std::min(16, C);
    while (OG > 1 && static_cast<size_t>(OG) * HW * 4 + static_cast<size_t>(OG) * C * 4 > 150 * 1024) OG = (OG + 1) / 2;
    const size_t skip_smem = static_cast<size_t>(OG) * HW * 4 + static_cast<size_t>(OG) * C * 4 + 2 * kThreads / 32 * 4;
    int per_sm = 1;
    e = scx::prepare_kernel(reinterpret_cast<const void*>(fno_skip_norm_gelu_kernel), skip_smem, kThreads, &per_sm);
    if (e != cudaSuccess) return e;
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
        const dim3 g((C + OG - 1) / OG, B);
        fno_skip_norm_gelu_kernel<<<g, kThreads, skip_smem, s>>>(act[spec], act[cur], act[nxt], prm->skip_w[l],
                                                                 prm->skip_b[l], HW, C, OG, cfg->instance_norm);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        cur = nxt;
    }
    // projection
    const size_t proj_smem = static_cast<size_t>(cfg->proj_hidden * C + cfg->proj_hidden +
                                                 cfg->out_channels * cfg->proj_hidden) * 4;
    e = scx::prepare_kernel(reinterpret_cast<const void*>(fno_project_kernel), proj_smem, kThreads, &per_sm);
    if (e != cudaSuccess) return e;
    fno_project_kernel<<<pix_grid, kThreads, proj_smem, s>>>(act[cur], y, prm->proj1_w, prm->proj1_b, prm->proj2_w,
                                                             prm->proj2_b, HW, C, cfg->proj_hidden, cfg->out_channels);
    return cudaGetLastError();
}
