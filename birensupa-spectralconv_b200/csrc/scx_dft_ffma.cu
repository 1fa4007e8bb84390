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

// Register-tiled forward for the shapes the tensor-core kernels do not take (W <= kTileMaxW,
// m2 <= 32, 2*m1 <= 64).  One CTA per (plane, ky tile); the ky range is split only as far as
// needed for the grid to cover the SMs (a tile computes only its own stage-1 columns, so the
// split adds no work; each tile reads its plane again, from L2).  Rows go in chunks of RC.
//   stage 1  R[h][ky] = sum_w x[h][w] T[w][ky]  thread tile 4 rows x 2 ky, w in steps of 4:
//            x as one 16-byte read per row, two complex twiddles per 16-byte read, 64 FMAs
//            per 8 shared-memory reads
//   stage 2  X[s][ky] += sum_h F[s][h] R[h][ky]  thread tile 2 slots x 2 ky, 16 FMAs per
//            3 reads, accumulated over the chunks in registers
// Per output the sums run over w, then over h, in order, as in dft_fwd_ffma_kernel.
constexpr int kTileMaxW = 320;
constexpr int kTileMaxRC = 128;

struct TileArgs {
    const float* x;
    float2* out1;
    float2* out2;
    long long ops;  // output plane stride (float2)
    int ors;        // output row stride (float2)
    int P, H, W, m1, m2;
    int KPT;        // ky pairs per tile
    int RC;         // rows per chunk (multiple of 4)
    int WP;         // shared-memory row pitch of x (multiple of 4, >= W + 4 columns of zeros)
    const float2* tw_row;  // [W][m2]
    const float2* tw_col;  // [2 m1][H]
};

__global__ void __launch_bounds__(kThreads) dft_fwd_tile_kernel(const TileArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x;
    const int W = a.W, H = a.H, m2 = a.m2, S = 2 * a.m1, WP = a.WP, RC = a.RC, KPT = a.KPT;
    const int K2 = 2 * KPT;       // ky per tile
    const int SP = (S + 1) / 2;   // slot pairs
    const int ky0 = blockIdx.y * K2;
    float2* T = reinterpret_cast<float2*>(smem);          // [WP][K2], zero past W and m2
    float2* F = T + WP * K2;                               // [2 SP][RC], zero past S and the chunk
    float2* R = F + 2 * SP * RC;                           // [RC][K2]
    float* xs = reinterpret_cast<float*>(R + RC * K2);     // [RC][WP], zero past W
    batched_copy<8, float2>(
        WP * K2,
        [&](int i) {
            const int w = i / K2, k = i - w * K2;
            return (w < W && ky0 + k < m2) ? a.tw_row[static_cast<size_t>(w) * m2 + ky0 + k] : make_float2(0.f, 0.f);
        },
        [&](int i, float2 v) { T[i] = v; });
    const int n1 = (RC / 4) * KPT;  // stage-1 threads
    const int kp1 = tid % KPT, r0 = 4 * (tid / KPT);
    const int n2 = SP * KPT;        // stage-2 threads
    const int kp2 = tid % KPT, s0 = 2 * (tid / KPT);
    for (int p = blockIdx.x; p < a.P; p += gridDim.x) {
        float2 acc2[2][2];
#pragma unroll
        for (int i = 0; i < 2; ++i) acc2[i][0] = acc2[i][1] = make_float2(0.f, 0.f);
        const float* xp = a.x + static_cast<size_t>(p) * H * W;
        for (int h0 = 0; h0 < H; h0 += RC) {
            const int rows = min(RC, H - h0);
            __syncthreads();  // the previous chunk's readers are done
            batched_copy<16, float>(
                RC * WP,
                [&](int i) {
                    const int r = i / WP, c = i - r * WP;
                    return (r < rows && c < W) ? __ldcs(xp + static_cast<size_t>(h0 + r) * W + c) : 0.f;
                },
                [&](int i, float v) { xs[i] = v; });
            batched_copy<8, float2>(
                2 * SP * RC,
                [&](int i) {
                    const int sl = i / RC, hh = i - sl * RC;
                    return (sl < S && hh < rows) ? a.tw_col[static_cast<size_t>(sl) * H + h0 + hh] : make_float2(0.f, 0.f);
                },
                [&](int i, float2 v) { F[i] = v; });
            __syncthreads();
            if (tid < n1) {
                float2 acc[4][2];
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
                for (int w = 0; w < WP; w += 4) {
                    float4 xv[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(xs + (r0 + i) * WP + w);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 tv = *reinterpret_cast<const float4*>(T + (w + u) * K2 + 2 * kp1);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float xval = u == 0 ? xv[i].x : (u == 1 ? xv[i].y : (u == 2 ? xv[i].z : xv[i].w));
                            acc[i][0].x = fmaf(xval, tv.x, acc[i][0].x);
                            acc[i][0].y = fmaf(xval, tv.y, acc[i][0].y);
                            acc[i][1].x = fmaf(xval, tv.z, acc[i][1].x);
                            acc[i][1].y = fmaf(xval, tv.w, acc[i][1].y);
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    *reinterpret_cast<float4*>(R + (r0 + i) * K2 + 2 * kp1) =
                        make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
            }
            __syncthreads();
            if (tid < n2) {
                for (int hh = 0; hh < rows; ++hh) {
                    const float4 rv = *reinterpret_cast<const float4*>(R + hh * K2 + 2 * kp2);
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const float2 f = F[(s0 + i) * RC + hh];
                        acc2[i][0].x = fmaf(f.x, rv.x, fmaf(-f.y, rv.y, acc2[i][0].x));
                        acc2[i][0].y = fmaf(f.x, rv.y, fmaf(f.y, rv.x, acc2[i][0].y));
                        acc2[i][1].x = fmaf(f.x, rv.z, fmaf(-f.y, rv.w, acc2[i][1].x));
                        acc2[i][1].y = fmaf(f.x, rv.w, fmaf(f.y, rv.z, acc2[i][1].y));
                    }
                }
            }
        }
        if (tid < n2) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int sl = s0 + i, ky = ky0 + 2 * kp2 + j;
                    if (sl < S && ky < m2) {
                        float2* dst = sl < a.m1 ? a.out1 + static_cast<size_t>(p) * a.ops + static_cast<size_t>(sl) * a.ors
                                                : a.out2 + static_cast<size_t>(p) * a.ops +
                                                      static_cast<size_t>(sl - a.m1) * a.ors;
                        dst[ky] = acc2[i][j];
                    }
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

// grid = persistent over (plane, 32-row tile).  In stage 5 a thread owns a register block of
// RB rows x CB columns: rows RB*rg .. RB*rg + RB - 1 and columns c, c + NC, ..., c + (CB-1) NC
// with NC = ceil(W / CB) and thread = rg * NC + c, so one ky step reads CB twiddles and RB
// spectrum values (broadcast) for RB*CB*2 FMAs; consecutive threads take consecutive columns
// (conflict-free twiddle reads, coalesced stores).  Needs NC * (kRt / RB) <= kThreads.
template <int RB, int CB>
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
    const int NC = (W + CB - 1) / CB;
    const int my_c = tid % NC, my_rg = tid / NC;
    const bool active = my_rg < kRt / RB;  // warp-uniform except in the warp that straddles the end
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int q = t / tpp;
        const int h0 = (t - q * tpp) * kRt;
        const int rows = min(kRt, H - h0);
        float acc[RB][CB];
#pragma unroll
        for (int r = 0; r < RB; ++r)
#pragma unroll
            for (int j = 0; j < CB; ++j) acc[r][j] = 0.f;
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
            if (active) {
                for (int k = 0; k < kc; ++k) {
                    float2 tw[CB];
#pragma unroll
                    for (int j = 0; j < CB; ++j) {
                        const int w = my_c + j * NC;
                        tw[j] = w < W ? twri[k * W + w] : make_float2(0.f, 0.f);
                    }
#pragma unroll
                    for (int r = 0; r < RB; ++r) {
                        const float2 z = Zs[(my_rg * RB + r) * KC + k];
#pragma unroll
                        for (int j = 0; j < CB; ++j)
                            acc[r][j] = fmaf(z.x, tw[j].x, fmaf(-z.y, tw[j].y, acc[r][j]));
                    }
                }
            }
        }
        float* yp = a.y + (static_cast<size_t>(q) * H + h0) * W;
        if (active) {
#pragma unroll
            for (int r = 0; r < RB; ++r) {
                const int row = my_rg * RB + r;
                if (row < rows) {
#pragma unroll
                    for (int j = 0; j < CB; ++j) {
                        const int w = my_c + j * NC;
                        if (w < W) __stcs(yp + static_cast<size_t>(row) * W + w, acc[r][j]);
                    }
                }
            }
        }
    }
}

}  // namespace

cudaError_t launch_dft_fwd(const float* x, float2* out1, float2* out2, long long out_plane_stride,
                           int out_row_stride, int P, int H, int W, int m1, int m2, const Twiddles& tw,
                           cudaStream_t stream) {
    if (W <= kTileMaxW && m2 <= 32 && 2 * m1 <= 64) {
        TileArgs t;
        t.x = x;
        t.out1 = out1;
        t.out2 = out2;
        t.ops = out_plane_stride;
        t.ors = out_row_stride;
        t.P = P;
        t.H = H;
        t.W = W;
        t.m1 = m1;
        t.m2 = m2;
        t.tw_row = tw.row_fwd;
        t.tw_col = tw.col_fwd;
        t.WP = (W + 3) / 4 * 4 + 4;
        const int KP = (m2 + 1) / 2, SP = m1;  // ky pairs, slot pairs (2 m1 slots)
        // ky tiles: as few as give the grid one CTA per SM (or all of them)
        int ntile = 1;
        while (ntile < KP && static_cast<long long>(P) * ntile < num_sms()) ++ntile;
        t.KPT = (KP + ntile - 1) / ntile;
        ntile = (KP + t.KPT - 1) / t.KPT;
        // rows per chunk: enough for every thread in stage 1, within the shared-memory budget
        int RC = std::min({4 * (kThreads / t.KPT), (H + 3) / 4 * 4, kTileMaxRC});
        const int K2 = 2 * t.KPT;
        auto smem_of = [&](int rc) {
            return static_cast<size_t>(t.WP) * K2 * 8 + static_cast<size_t>(2 * SP) * rc * 8 +
                   static_cast<size_t>(rc) * K2 * 8 + static_cast<size_t>(rc) * t.WP * 4;
        };
        // two CTAs per SM when the chunk can shrink to fit (at least 32 rows), else one
        int rc2 = RC;
        while (smem_of(rc2) > static_cast<size_t>(kSmemBudget) / 2 && rc2 > 32) rc2 -= 4;
        if (smem_of(rc2) <= static_cast<size_t>(kSmemBudget) / 2) RC = rc2;
        while (smem_of(RC) > static_cast<size_t>(kSmemBudget) && RC > 4) RC -= 4;
        t.RC = RC;
        const size_t smem = smem_of(RC);
        if (smem <= static_cast<size_t>(kSmemBudget) && SP * t.KPT <= kThreads) {
            int per_sm = 1;
            cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(dft_fwd_tile_kernel), smem, kThreads, &per_sm);
            if (e != cudaSuccess) return e;
            const int gx = std::max(1, std::min(P, (per_sm * num_sms() + ntile - 1) / ntile));
            dft_fwd_tile_kernel<<<dim3(gx, ntile), kThreads, smem, stream>>>(t);
            return cudaGetLastError();
        }
    }
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
    const int tiles = Q * ((H + kRt - 1) / kRt);
    auto run = [&](auto kernel) -> cudaError_t {
        int per_sm = 1;
        cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(kernel), smem, kThreads, &per_sm);
        if (e != cudaSuccess) return e;
        const int gx = std::max(1, std::min(tiles, per_sm * num_sms()));
        kernel<<<gx, kThreads, smem, stream>>>(a);
        return cudaGetLastError();
    };
    // the register block with the most threads busy (at most kThreads) and, among equals, the
    // most FMAs per shared-memory read; wide planes fall back to all 32 rows per thread
    auto threads_for = [&](int rb, int cb) { return ((W + cb - 1) / cb) * (kRt / rb); };
    if (threads_for(4, 2) <= kThreads) return run(dft_inv_ffma_kernel<4, 2>);
    const int t82 = threads_for(8, 2), t84 = threads_for(8, 4);
    if (t82 <= kThreads && (t84 > kThreads || t82 > t84)) return run(dft_inv_ffma_kernel<8, 2>);
    if (t84 <= kThreads) return run(dft_inv_ffma_kernel<8, 4>);
    if (threads_for(16, 4) <= kThreads) return run(dft_inv_ffma_kernel<16, 4>);
    if (threads_for(kRt, 1) <= kThreads) return run(dft_inv_ffma_kernel<kRt, 1>);
    if (threads_for(kRt, 2) <= kThreads) return run(dft_inv_ffma_kernel<kRt, 2>);
    return run(dft_inv_ffma_kernel<kRt, 4>);
}

}  // namespace scx
