// General-shape truncated DFT kernels on FP32 FFMA (any H, W, m1, m2).
//
// Forward (replaces rfft2_sufft + the two corner gathers,
// spectral_conv/spectral_conv_ext.cpp:314-347 and spectral_conv/spectral_conv_ops.py:385-392):
//   stage 1  R[h][ky]      = sum_w x[h][w] * exp(-2 pi i ky w / W)      ky < m2
//   stage 2  X[slot][ky]   = sum_h exp(-2 pi i kx(slot) h / H) * R[h][ky]
// Only the 2*m1 x m2 retained modes are ever formed; no full spectrum, no permutes.
//
// Inverse (replaces the zeroed out_freq, the corner scatters and irfft2_sufft,
// spectral_conv/spectral_conv_ops.py:386-406 and spectral_conv/spectral_conv_ext.cpp:349-384):
//   stage 4  Z[h][ky] = sum_slot exp(+2 pi i kx(slot) h / H) * Y[slot][ky]
//   stage 5  y[h][w]  = sum_ky c_ky/(HW) * Re(Z[h][ky] * exp(+2 pi i ky w / W))
// Zero padding is implicit and the 1/(HW) scale lives in the twiddles.
#include <algorithm>

#include "scx_internal.h"

namespace scx {
namespace {

constexpr int kThreads = 256;
constexpr int kRpt = 4;    // stage-1 rows per thread

// Cooperative copy of n elements, element i from load(i) to store(i, v): each thread first
// issues up to LB loads into registers and only then stores them, so a batch of loads is in
// flight at once (a plain load-store loop waits a full memory latency per element: the
// compiler cannot move a load above the previous shared-memory store).
template <int LB, typename T, typename LoadF, typename StoreF>
__device__ __forceinline__ void batched_copy(int n, LoadF load, StoreF store) {
    for (int i0 = threadIdx.x; i0 < n; i0 += kThreads * LB) {
        T v[LB];
#pragma unroll
        for (int u = 0; u < LB; ++u) {
            const int i = i0 + u * kThreads;
            if (i < n) v[u] = load(i);
        }
#pragma unroll
        for (int u = 0; u < LB; ++u) {
            const int i = i0 + u * kThreads;
            if (i < n) store(i, v[u]);
        }
    }
}
constexpr int kRt = 32;    // inverse: output rows per tile
constexpr int kSmemBudget = 200 * 1024;

struct FwdArgs {
    const float* x;
    float2* out1;
    float2* out2;
    long long ops;  // output plane stride (float2)
    int ors;        // output row stride (float2)
    int P, H, W, m1, m2;
    int KT, ST, RC, WP;  // ky tile, slot tile, rows per chunk, smem row pitch of x
    const float2* tw_row;
    const float2* tw_col;
};

// grid = (plane blocks [persistent], ky tiles, slot tiles)
template <int NPT>
__global__ void __launch_bounds__(kThreads) dft_fwd_ffma_kernel(const FwdArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x;
    const int ky0 = blockIdx.y * a.KT;
    const int kt = min(a.KT, a.m2 - ky0);
    const int s0 = blockIdx.z * a.ST;
    const int st = min(a.ST, 2 * a.m1 - s0);
    const int W = a.W, H = a.H, RC = a.RC, WP = a.WP, KT = a.KT;

    float2* twr = reinterpret_cast<float2*>(smem);  // [W][kt]
    float2* twc = twr + W * KT;                      // [ST][RC]
    float2* Rs = twc + a.ST * RC;                    // [RC][KT]
    float* xs = reinterpret_cast<float*>(Rs + RC * KT);  // [RC][WP]

    batched_copy<8, float2>(
        W * kt,
        [&](int i) {
            const int w = i / kt, k = i - w * kt;
            return a.tw_row[static_cast<size_t>(w) * a.m2 + ky0 + k];
        },
        [&](int i, float2 v) { twr[i] = v; });
    const int groups = RC / kRpt;
    const int s1_active = groups * kt;
    const int nout = st * kt;

    for (int p = blockIdx.x; p < a.P; p += gridDim.x) {
        float2 acc[NPT];
#pragma unroll
        for (int k = 0; k < NPT; ++k) acc[k] = make_float2(0.f, 0.f);
        const float* xp = a.x + static_cast<size_t>(p) * H * W;
        for (int h0 = 0; h0 < H; h0 += RC) {
            const int rows = min(RC, H - h0);
            __syncthreads();
            const float* src = xp + static_cast<size_t>(h0) * W;
            batched_copy<16, float>(
                rows * W, [&](int i) { return __ldcs(src + i); },
                [&](int i, float v) {
                    const int r = i / W, c = i - r * W;
                    xs[r * WP + c] = v;
                });
            batched_copy<8, float2>(
                st * RC,
                [&](int i) {
                    const int s = i / RC, hh = i - s * RC;
                    return hh < rows ? a.tw_col[static_cast<size_t>(s0 + s) * H + h0 + hh] : make_float2(0.f, 0.f);
                },
                [&](int i, float2 v) { twc[i] = v; });
            __syncthreads();
            if (tid < s1_active) {
                const int g = tid / kt, k = tid - g * kt;
                float re[kRpt], im[kRpt];
#pragma unroll
                for (int j = 0; j < kRpt; ++j) re[j] = im[j] = 0.f;
                const float* xr = xs + g * kRpt * WP;
                for (int w = 0; w < W; ++w) {
                    const float2 t = twr[w * kt + k];
#pragma unroll
                    for (int j = 0; j < kRpt; ++j) {
                        const float v = xr[j * WP + w];
                        re[j] = fmaf(v, t.x, re[j]);
                        im[j] = fmaf(v, t.y, im[j]);
                    }
                }
#pragma unroll
                for (int j = 0; j < kRpt; ++j) {
                    const int r = g * kRpt + j;
                    Rs[r * KT + k] = r < rows ? make_float2(re[j], im[j]) : make_float2(0.f, 0.f);
                }
            }
            __syncthreads();
#pragma unroll
            for (int k = 0; k < NPT; ++k) {
                const int o = tid + k * kThreads;
                if (o < nout) {
                    const int s = o / kt, ky = o - s * kt;
                    const float2* tc = twc + s * RC;
                    float2 v = acc[k];
                    for (int hh = 0; hh < rows; ++hh) {
                        const float2 t = tc[hh];
                        const float2 r = Rs[hh * KT + ky];
                        v.x = fmaf(t.x, r.x, fmaf(-t.y, r.y, v.x));
                        v.y = fmaf(t.x, r.y, fmaf(t.y, r.x, v.y));
                    }
                    acc[k] = v;
                }
            }
        }
#pragma unroll
        for (int k = 0; k < NPT; ++k) {
            const int o = tid + k * kThreads;
            if (o < nout) {
                const int s = o / kt, ky = o - s * kt;
                const int sg = s0 + s;
                float2* dst = (sg < a.m1 ? a.out1 + static_cast<size_t>(p) * a.ops +
                                               static_cast<size_t>(sg) * a.ors
                                         : a.out2 + static_cast<size_t>(p) * a.ops +
                                               static_cast<size_t>(sg - a.m1) * a.ors) +
                              ky0 + ky;
                *dst = acc[k];
            }
        }
    }
}

struct InvArgs {
    const float2* in1;
    const float2* in2;
    long long ips;  // input plane stride (float2)
    int irs;        // input row stride (float2)
    float* y;
    int Q, H, W, m1, m2;
    int KC;  // ky chunk
    const float2* tw_col;  // [H][2m1]
    const float2* tw_row;  // [m2][W]
};

// grid = persistent over (plane, 32-row tile)
template <int WPT>
__global__ void __launch_bounds__(kThreads) dft_inv_ffma_kernel(const InvArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x;
    const int S2 = 2 * a.m1, KC = a.KC, W = a.W, H = a.H;
    float2* Ys = reinterpret_cast<float2*>(smem);  // [S2][KC]
    float2* twci = Ys + S2 * KC;                    // [kRt][S2]
    float2* twri = twci + kRt * S2;                 // [KC][W]
    float2* Zs = twri + KC * W;                     // [kRt][KC]

    const bool single_chunk = KC >= a.m2;
    if (single_chunk)
        batched_copy<8, float2>(a.m2 * W, [&](int i) { return a.tw_row[i]; }, [&](int i, float2 v) { twri[i] = v; });
    const int tpp = (H + kRt - 1) / kRt;
    const int ntiles = a.Q * tpp;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int q = t / tpp;
        const int h0 = (t - q * tpp) * kRt;
        const int rows = min(kRt, H - h0);
        float acc[kRt][WPT];
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int j = 0; j < WPT; ++j) acc[r][j] = 0.f;
        __syncthreads();
        batched_copy<8, float2>(
            kRt * S2,
            [&](int i) {
                const int r = i / S2, s = i - r * S2;
                return r < rows ? a.tw_col[static_cast<size_t>(h0 + r) * S2 + s] : make_float2(0.f, 0.f);
            },
            [&](int i, float2 v) { twci[i] = v; });
        for (int kc0 = 0; kc0 < a.m2; kc0 += KC) {
            const int kc = min(KC, a.m2 - kc0);
            __syncthreads();
            batched_copy<8, float2>(
                S2 * kc,
                [&](int i) {
                    const int s = i / kc, k = i - s * kc;
                    const float2* src = s < a.m1 ? a.in1 + static_cast<size_t>(q) * a.ips + static_cast<size_t>(s) * a.irs
                                                 : a.in2 + static_cast<size_t>(q) * a.ips +
                                                       static_cast<size_t>(s - a.m1) * a.irs;
                    return src[kc0 + k];
                },
                [&](int i, float2 v) {
                    const int s = i / kc, k = i - s * kc;
                    Ys[s * KC + k] = v;
                });
            if (!single_chunk)
                batched_copy<8, float2>(
                    kc * W, [&](int i) { return a.tw_row[static_cast<size_t>(kc0) * W + i]; },
                    [&](int i, float2 v) { twri[i] = v; });
            __syncthreads();
            for (int o = tid; o < kRt * kc; o += kThreads) {
                const int r = o / kc, k = o - r * kc;
                const float2* tc = twci + r * S2;
                float2 z = make_float2(0.f, 0.f);
                for (int s = 0; s < S2; ++s) {
                    const float2 tv = tc[s];
                    const float2 v = Ys[s * KC + k];
                    z.x = fmaf(tv.x, v.x, fmaf(-tv.y, v.y, z.x));
                    z.y = fmaf(tv.x, v.y, fmaf(tv.y, v.x, z.y));
                }
                Zs[r * KC + k] = z;
            }
            __syncthreads();
            for (int k = 0; k < kc; ++k) {
                float2 tw[WPT];
#pragma unroll
                for (int j = 0; j < WPT; ++j) {
                    const int w = tid + j * kThreads;
                    tw[j] = w < W ? twri[k * W + w] : make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int r = 0; r < kRt; ++r) {
                    const float2 z = Zs[r * KC + k];
#pragma unroll
                    for (int j = 0; j < WPT; ++j)
                        acc[r][j] = fmaf(z.x, tw[j].x, fmaf(-z.y, tw[j].y, acc[r][j]));
                }
            }
        }
        float* yp = a.y + (static_cast<size_t>(q) * H + h0) * W;
#pragma unroll
        for (int r = 0; r < kRt; ++r) {
            if (r < rows) {
#pragma unroll
                for (int j = 0; j < WPT; ++j) {
                    const int w = tid + j * kThreads;
                    if (w < W) __stcs(yp + static_cast<size_t>(r) * W + w, acc[r][j]);
                }
            }
        }
    }
}

}  // namespace

cudaError_t launch_dft_fwd(const float* x, float2* out1, float2* out2, long long out_plane_stride,
                           int out_row_stride, int P, int H, int W, int m1, int m2, const Twiddles& tw,
                           cudaStream_t stream) {
    FwdArgs a;
    a.x = x;
    a.out1 = out1;
    a.out2 = out2;
    a.ops = out_plane_stride;
    a.ors = out_row_stride;
    a.P = P;
    a.H = H;
    a.W = W;
    a.m1 = m1;
    a.m2 = m2;
    a.tw_row = tw.row_fwd;
    a.tw_col = tw.col_fwd;
    // ky tile: keep the [W][KT] row twiddles within ~96 KB of shared memory.
    int KT = std::min(m2, std::max(1, (96 * 1024) / (8 * W)));
    KT = std::min(KT, kThreads);
    int ST = std::min(2 * m1, std::max(1, 4096 / KT));
    int RC = std::min(kRpt * (kThreads / KT), ((H + kRpt - 1) / kRpt) * kRpt);
    const int WP = (W % 2 == 0) ? W + 1 : W;
    auto smem_of = [&](int rc, int st) {
        return static_cast<size_t>(W) * KT * 8 + static_cast<size_t>(st) * rc * 8 +
               static_cast<size_t>(rc) * KT * 8 + static_cast<size_t>(rc) * WP * 4;
    };
    while (smem_of(RC, ST) > kSmemBudget && RC > kRpt) RC -= kRpt;
    while (smem_of(RC, ST) > kSmemBudget && ST > 1) ST = (ST + 1) / 2;
    const size_t smem = smem_of(RC, ST);
    if (smem > kSmemBudget) return cudaErrorInvalidValue;
    a.KT = KT;
    a.ST = ST;
    a.RC = RC;
    a.WP = WP;
    const int npt_needed = (ST * KT + kThreads - 1) / kThreads;
    const dim3 block(kThreads);
    auto run = [&](auto kernel) -> cudaError_t {
        int per_sm = 1;
        cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(kernel), smem, kThreads, &per_sm);
        if (e != cudaSuccess) return e;
        const int gx = std::max(1, std::min(P, per_sm * num_sms()));
        const dim3 grid(gx, (m2 + KT - 1) / KT, (2 * m1 + ST - 1) / ST);
        kernel<<<grid, block, smem, stream>>>(a);
        return cudaGetLastError();
    };
    if (npt_needed <= 1) return run(dft_fwd_ffma_kernel<1>);
    if (npt_needed <= 2) return run(dft_fwd_ffma_kernel<2>);
    if (npt_needed <= 4) return run(dft_fwd_ffma_kernel<4>);
    if (npt_needed <= 8) return run(dft_fwd_ffma_kernel<8>);
    return run(dft_fwd_ffma_kernel<16>);
}

cudaError_t launch_dft_inv(const float2* in1, const float2* in2, long long in_plane_stride,
                           int in_row_stride, float* y, int Q, int H, int W, int m1, int m2,
                           const Twiddles& tw, cudaStream_t stream) {
    if (W > 4 * kThreads) return cudaErrorInvalidValue;
    InvArgs a;
    a.in1 = in1;
    a.in2 = in2;
    a.ips = in_plane_stride;
    a.irs = in_row_stride;
    a.y = y;
    a.Q = Q;
    a.H = H;
    a.W = W;
    a.m1 = m1;
    a.m2 = m2;
    a.tw_col = tw.col_inv;
    a.tw_row = tw.row_inv;
    const int S2 = 2 * m1;
    const long long fixed = static_cast<long long>(kRt) * S2 * 8;
    const long long per_k = static_cast<long long>(S2) * 8 + static_cast<long long>(W) * 8 + kRt * 8;
    long long KC = (kSmemBudget - fixed) / per_k;
    if (KC < 1) return cudaErrorInvalidValue;
    KC = std::min<long long>(KC, m2);
    a.KC = static_cast<int>(KC);
    const size_t smem = static_cast<size_t>(fixed + per_k * KC);
    const int wpt = (W + kThreads - 1) / kThreads;
    const int tiles = Q * ((H + kRt - 1) / kRt);
    auto run = [&](auto kernel) -> cudaError_t {
        int per_sm = 1;
        cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(kernel), smem, kThreads, &per_sm);
        if (e != cudaSuccess) return e;
        const int gx = std::max(1, std::min(tiles, per_sm * num_sms()));
        kernel<<<gx, kThreads, smem, stream>>>(a);
        return cudaGetLastError();
    };
    if (wpt <= 1) return run(dft_inv_ffma_kernel<1>);
    if (wpt <= 2) return run(dft_inv_ffma_kernel<2>);
    return run(dft_inv_ffma_kernel<4>);
}

}  // namespace scx
