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

#include <cooperative_groups.h>

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

// Row-split forward for the shapes the tensor-core kernels do not take (W <= kRowsMaxW,
// m2 <= 32, 2*m1 <= 64).  A thread-block cluster of HB CTAs takes one plane and CTA r of it the
// rows [r*RB, r*RB + RB), in chunks of RC rows, so a plane's work spreads over up to 8 SMs
// (48 planes at 130 x 130 used to run as 48 CTAs).  Per chunk:
//   stage 1  R[h][ky] = sum_w x[h][w] T[w][ky] from the symmetry T[W-w] = conj(T[w]): with
//            u[w] = x[w] + x[W-w] and v[w] = x[w] - x[W-w] for 0 < w < W/2 (u = x, v = 0 at
//            w = 0 and W/2), Re R = sum u Re T and Im R = sum v Im T over w <= W/2, half the
//            FMAs and twiddles of the direct sum.  The chunk is stored as u and v rows.
//            Thread tile RT rows x 2 ky, w in steps of 4 (16-byte reads of u and v per row, two
//            complex twiddles per 16-byte read); the w range is
//            split over WS thread groups so that the small per-chunk tile count still fills the
//            CTA, and their partial sums are added in group order.  RT = 1 (three CTAs per SM)
//            where a chunk's row tiles fit the CTA's threads, RT = 4 (two CTAs per SM, four
//            times the FMAs per shared-memory read) where they do not
//   stage 2  Xp[s][ky] += sum_h F[s][h] R[h][ky]  thread tile 2 slots x 2 ky, kept in shared
//            memory across the chunks (each element owned by one thread)
// Then the cluster adds the CTAs' partial spectra Xp through distributed shared memory, rank
// 0 first, each CTA finishing its share of the outputs.  Every sum runs in a fixed order, so
// results are bitwise reproducible.  Row pitches are padded so that the rows a warp reads at
// once fall in different banks (x: a pitch of an odd number of 16-byte units; F: an odd
// number of 8-byte elements).
constexpr int kRowsMaxW = 320;
constexpr int kRowsMaxCluster = 8;

struct RowsArgs {
    const float* x;
    float2* out1;
    float2* out2;
    long long ops;  // output plane stride (float2)
    int ors;        // output row stride (float2)
    int P, H, W, m1, m2;
    int RB;         // rows per CTA (the last CTA of a plane may hold fewer, or none)
    int RC;         // rows per chunk (a multiple of the stage-1 row tile)
    int WP;         // shared-memory row pitch of u and v (4 times an odd number, >= W/2 + 1, zero past it)
    int WS, WR;     // stage-1 w splits, and the w range of each (a multiple of 4)
    const float2* tw_row;  // [W][m2]
    const float2* tw_col;  // [2 m1][H]
};

template <int RT>
__global__ void __launch_bounds__(kThreads, RT == 1 ? 3 : 2) dft_fwd_rows_kernel(const RowsArgs a) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x;
    const int W = a.W, H = a.H, m2 = a.m2, S = 2 * a.m1, WP = a.WP, RC = a.RC, WS = a.WS, WR = a.WR;
    const int FP = RC + 1;                     // F row pitch (odd)
    const int KP = (m2 + 1) / 2, K2 = 2 * KP;  // ky pairs, ky padded to pairs
    const int SP = (S + 1) / 2, S2 = 2 * SP;   // slot pairs, slots padded to pairs
    const int p = blockIdx.y;
    const int rank = static_cast<int>(cluster.block_rank()), HB = static_cast<int>(cluster.num_blocks());
    const int h0 = rank * a.RB;
    const int my_rows = max(0, min(a.RB, H - h0));
    const int NPW = W / 2 + 1;                          // w = 0 .. W/2
    float2* T = reinterpret_cast<float2*>(smem);       // [WP][K2], zero past NPW and m2
    float2* F = T + WP * K2;                            // [S2][FP], zero past S and the chunk
    float2* Rp = F + S2 * FP;                           // [WS][RC][K2] stage-1 partial sums
    float2* R = WS > 1 ? Rp + WS * RC * K2 : Rp;        // [RC][K2] (the partial sums themselves if WS = 1)
    float2* Xp = R + RC * K2;                           // [S2][K2] this CTA's partial spectrum
    float* xs = reinterpret_cast<float*>(Xp + S2 * K2);  // [RC][WP], zero past W and the chunk
    batched_copy<8, float2>(
        WP * K2,
        [&](int i) {
            const int w = i / K2, k = i - w * K2;
            return (w < NPW && k < m2) ? a.tw_row[static_cast<size_t>(w) * m2 + k] : make_float2(0.f, 0.f);
        },
        [&](int i, float2 v) { T[i] = v; });
    for (int i = tid; i < S2 * K2; i += kThreads) Xp[i] = make_float2(0.f, 0.f);
    float* vs = xs + RC * WP;                           // [RC][WP]: v rows (xs holds the u rows)
    const float* xp = a.x + static_cast<size_t>(p) * H * W;
    const int RG = RC / RT;
    for (int c0 = 0; c0 < my_rows; c0 += RC) {
        const int rows = min(RC, my_rows - c0), hb = h0 + c0;
        __syncthreads();  // the previous chunk's readers are done
        batched_copy<8, float2>(
            RC * WP,
            [&](int i) {
                // both samples loaded unconditionally (a self-partner column loads itself twice), so
                // the batch's loads are all in flight before any is used
                const int r = i / WP, c = i - r * WP;
                if (r >= rows || c >= NPW) return make_float2(0.f, 0.f);
                const float* row = xp + static_cast<size_t>(hb + r) * W;
                const int c1 = c == 0 ? 0 : W - c;
                return make_float2(__ldcs(row + c), __ldcs(row + c1));
            },
            [&](int i, float2 x2) {
                const int c = i % WP;
                const bool self = c == 0 || 2 * c == W;
                xs[i] = self ? x2.x : x2.x + x2.y;
                vs[i] = self ? 0.f : x2.x - x2.y;
            });
        batched_copy<8, float2>(
            S2 * FP,
            [&](int i) {
                const int sl = i / FP, r = i - sl * FP;
                return (sl < S && r < rows) ? a.tw_col[static_cast<size_t>(sl) * H + hb + r] : make_float2(0.f, 0.f);
            },
            [&](int i, float2 v) { F[i] = v; });
        __syncthreads();
        for (int t = tid; t < RG * KP * WS; t += kThreads) {
            const int kp = t % KP, rg = (t / KP) % RG, ws = t / (KP * RG);
            const int r0 = RT * rg, w0 = ws * WR, w1 = min(WP, w0 + WR);
            float2 acc[RT][2];
#pragma unroll
            for (int i = 0; i < RT; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
            for (int w = w0; w < w1; w += 4) {
                float4 uv[RT], vv[RT];
#pragma unroll
                for (int i = 0; i < RT; ++i) {
                    uv[i] = *reinterpret_cast<const float4*>(xs + (r0 + i) * WP + w);
                    vv[i] = *reinterpret_cast<const float4*>(vs + (r0 + i) * WP + w);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 tv = *reinterpret_cast<const float4*>(T + (w + u) * K2 + 2 * kp);
#pragma unroll
                    for (int i = 0; i < RT; ++i) {
                        const float uval = u == 0 ? uv[i].x : (u == 1 ? uv[i].y : (u == 2 ? uv[i].z : uv[i].w));
                        const float vval = u == 0 ? vv[i].x : (u == 1 ? vv[i].y : (u == 2 ? vv[i].z : vv[i].w));
                        acc[i][0].x = fmaf(uval, tv.x, acc[i][0].x);
                        acc[i][0].y = fmaf(vval, tv.y, acc[i][0].y);
                        acc[i][1].x = fmaf(uval, tv.z, acc[i][1].x);
                        acc[i][1].y = fmaf(vval, tv.w, acc[i][1].y);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < RT; ++i)
                *reinterpret_cast<float4*>(Rp + (ws * RC + r0 + i) * K2 + 2 * kp) =
                    make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
        }
        __syncthreads();
        if (WS > 1) {
            for (int i = tid; i < RC * KP; i += kThreads) {
                const int r = i / KP, kp = i - r * KP;
                float4 v = *reinterpret_cast<const float4*>(Rp + r * K2 + 2 * kp);
                for (int ws = 1; ws < WS; ++ws) {
                    const float4 u = *reinterpret_cast<const float4*>(Rp + (ws * RC + r) * K2 + 2 * kp);
                    v.x += u.x;
                    v.y += u.y;
                    v.z += u.z;
                    v.w += u.w;
                }
                *reinterpret_cast<float4*>(R + r * K2 + 2 * kp) = v;
            }
            __syncthreads();
        }
        for (int t = tid; t < SP * KP; t += kThreads) {
            const int kp = t % KP, s0 = 2 * (t / KP);
            float4 acc2[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) acc2[i] = *reinterpret_cast<const float4*>(Xp + (s0 + i) * K2 + 2 * kp);
            for (int r = 0; r < rows; ++r) {
                const float4 rv = *reinterpret_cast<const float4*>(R + r * K2 + 2 * kp);
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float2 f = F[(s0 + i) * FP + r];
                    acc2[i].x = fmaf(f.x, rv.x, fmaf(-f.y, rv.y, acc2[i].x));
                    acc2[i].y = fmaf(f.x, rv.y, fmaf(f.y, rv.x, acc2[i].y));
                    acc2[i].z = fmaf(f.x, rv.z, fmaf(-f.y, rv.w, acc2[i].z));
                    acc2[i].w = fmaf(f.x, rv.w, fmaf(f.y, rv.z, acc2[i].w));
                }
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) *reinterpret_cast<float4*>(Xp + (s0 + i) * K2 + 2 * kp) = acc2[i];
        }
    }
    cluster.sync();  // every CTA's partial spectrum is complete and visible cluster-wide
    const int n = S * m2;
    const int o_begin = static_cast<int>(static_cast<long long>(n) * rank / HB);
    const int o_end = static_cast<int>(static_cast<long long>(n) * (rank + 1) / HB);
    for (int o = o_begin + tid; o < o_end; o += kThreads) {
        const int sl = o / m2, ky = o - sl * m2;
        float2 sum = make_float2(0.f, 0.f);
        for (int q = 0; q < HB; ++q) {
            const float2 v = cluster.map_shared_rank(Xp, q)[sl * K2 + ky];
            sum.x += v.x;
            sum.y += v.y;
        }
        float2* dst = sl < a.m1 ? a.out1 + static_cast<size_t>(p) * a.ops + static_cast<size_t>(sl) * a.ors
                                : a.out2 + static_cast<size_t>(p) * a.ops + static_cast<size_t>(sl - a.m1) * a.ors;
        dst[ky] = sum;
    }
    cluster.sync();  // no CTA leaves while another still reads its partial spectrum
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

// grid = persistent over (plane, 32-row tile).
// Stage 4: thread tile 2 rows x 2 ky over the slots (16 FMAs per three shared-memory reads);
// the twiddle rows have an odd pitch, so a warp's row pairs fall in different banks.
// Stage 5 uses the symmetry of the row twiddles: E[ky][W-w] = conj(E[ky][w]), so with
// A = sum_ky Zr Er and B = sum_ky Zi Ei over one pass, y[w] = A - B and y[W-w] = A + B
// (w = 0 and w = W/2 are their own partners).  A thread owns a register block of RB rows x
// CB column pairs: rows RB*rg .. RB*rg + RB - 1 and pairs c, c + NC, ..., c + (CB-1) NC with
// NC = ceil(NPW / CB), NPW = W/2 + 1, thread = rg * NC + c, so one ky step reads CB twiddles
// and RB spectrum values (broadcast) for 2*RB*CB FMAs covering 2*RB*CB outputs; consecutive
// threads take consecutive columns (conflict-free twiddle reads, coalesced stores).  Needs
// NC * (kRt / RB) <= kThreads.
template <int RB, int CB>
__global__ void __launch_bounds__(kThreads) dft_inv_ffma_kernel(const InvArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x;
    const int S2 = 2 * a.m1, KC = a.KC, W = a.W, H = a.H;
    const int GP = S2 + 1;                // twiddle row pitch (odd)
    constexpr int ZP = kRt + 1;           // Zs row pitch (odd)
    const int KCP = (KC + 1) / 2 * 2;     // spectrum row pitch (pairs)
    const int NPW = W / 2 + 1;            // column pairs
    // Ys, read as 16-byte vectors, first (its size is a multiple of 16 bytes, an even pitch)
    float2* Ys = reinterpret_cast<float2*>(smem);  // [S2][KCP], zero past kc
    float2* twci = Ys + S2 * KCP;                   // [kRt][GP]
    float2* Zs = twci + kRt * GP;                   // [KCP][ZP] (ky-major: a warp's row groups in different banks)
    float2* twri = Zs + KCP * ZP;                   // [KC][NPW]

    const bool single_chunk = KC >= a.m2;
    if (single_chunk)
        batched_copy<8, float2>(
            a.m2 * NPW,
            [&](int i) {
                const int k = i / NPW, w = i - k * NPW;
                return a.tw_row[static_cast<size_t>(k) * W + w];
            },
            [&](int i, float2 v) { twri[i] = v; });
    const int tpp = (H + kRt - 1) / kRt;
    const int ntiles = a.Q * tpp;
    const int NC = (NPW + CB - 1) / CB;
    const int my_c = tid % NC, my_rg = tid / NC;
    const bool active = my_rg < kRt / RB;  // warp-uniform except in the warp that straddles the end
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int q = t / tpp;
        const int h0 = (t - q * tpp) * kRt;
        const int rows = min(kRt, H - h0);
        float accA[RB][CB], accB[RB][CB];
#pragma unroll
        for (int r = 0; r < RB; ++r)
#pragma unroll
            for (int j = 0; j < CB; ++j) accA[r][j] = accB[r][j] = 0.f;
        __syncthreads();
        batched_copy<8, float2>(
            kRt * GP,
            [&](int i) {
                const int r = i / GP, s = i - r * GP;
                return (r < rows && s < S2) ? a.tw_col[static_cast<size_t>(h0 + r) * S2 + s] : make_float2(0.f, 0.f);
            },
            [&](int i, float2 v) { twci[i] = v; });
        for (int kc0 = 0; kc0 < a.m2; kc0 += KC) {
            const int kc = min(KC, a.m2 - kc0);
            const int kpc = (kc + 1) / 2;
            __syncthreads();
            batched_copy<8, float2>(
                S2 * KCP,
                [&](int i) {
                    const int s = i / KCP, k = i - s * KCP;
                    if (k >= kc) return make_float2(0.f, 0.f);
                    const float2* src = s < a.m1 ? a.in1 + static_cast<size_t>(q) * a.ips + static_cast<size_t>(s) * a.irs
                                                 : a.in2 + static_cast<size_t>(q) * a.ips +
                                                       static_cast<size_t>(s - a.m1) * a.irs;
                    return src[kc0 + k];
                },
                [&](int i, float2 v) { Ys[i] = v; });
            if (!single_chunk)
                batched_copy<8, float2>(
                    kc * NPW,
                    [&](int i) {
                        const int k = i / NPW, w = i - k * NPW;
                        return a.tw_row[static_cast<size_t>(kc0 + k) * W + w];
                    },
                    [&](int i, float2 v) { twri[i] = v; });
            __syncthreads();
            for (int o = tid; o < (kRt / 2) * kpc; o += kThreads) {
                const int kp = o % kpc, r0 = 2 * (o / kpc);
                float4 z[2];
                z[0] = z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int s = 0; s < S2; ++s) {
                    const float4 v = *reinterpret_cast<const float4*>(Ys + s * KCP + 2 * kp);
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const float2 g = twci[(r0 + i) * GP + s];
                        z[i].x = fmaf(g.x, v.x, fmaf(-g.y, v.y, z[i].x));
                        z[i].y = fmaf(g.x, v.y, fmaf(g.y, v.x, z[i].y));
                        z[i].z = fmaf(g.x, v.z, fmaf(-g.y, v.w, z[i].z));
                        z[i].w = fmaf(g.x, v.w, fmaf(g.y, v.z, z[i].w));
                    }
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    Zs[(2 * kp) * ZP + r0 + i] = make_float2(z[i].x, z[i].y);
                    Zs[(2 * kp + 1) * ZP + r0 + i] = make_float2(z[i].z, z[i].w);
                }
            }
            __syncthreads();
            if (active) {
                for (int k = 0; k < kc; ++k) {
                    float2 tw[CB];
#pragma unroll
                    for (int j = 0; j < CB; ++j) {
                        const int w = my_c + j * NC;
                        tw[j] = w < NPW ? twri[k * NPW + w] : make_float2(0.f, 0.f);
                    }
#pragma unroll
                    for (int r = 0; r < RB; ++r) {
                        const float2 z = Zs[k * ZP + my_rg * RB + r];
#pragma unroll
                        for (int j = 0; j < CB; ++j) {
                            accA[r][j] = fmaf(z.x, tw[j].x, accA[r][j]);
                            accB[r][j] = fmaf(z.y, tw[j].y, accB[r][j]);
                        }
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
                        if (w < NPW && 2 * w <= W) {
                            __stcs(yp + static_cast<size_t>(row) * W + w, accA[r][j] - accB[r][j]);
                            if (w > 0 && 2 * w < W)
                                __stcs(yp + static_cast<size_t>(row) * W + (W - w), accA[r][j] + accB[r][j]);
                        }
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
    if (W <= kRowsMaxW && m2 <= 32 && 2 * m1 <= 64) {
        RowsArgs t;
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
        t.WP = (W / 2 + 1 + 3) / 4 * 4;
        if ((t.WP / 4) % 2 == 0) t.WP += 4;  // an odd number of 16-byte units per row
        const int KP = (m2 + 1) / 2, K2 = 2 * KP, S2 = 2 * m1;
        // One-row tiles with three CTAs per SM (about three per SM over the whole batch) where a
        // chunk's tiles fit the CTA's threads; else four-row tiles with two CTAs per SM, as many
        // CTAs per plane as fit one such wave.  At least 8 rows per CTA.
        const int hb_cap = std::min(kRowsMaxCluster, (H + 7) / 8);
        int HB = std::max(1, std::min(hb_cap, static_cast<int>((2LL * num_sms() + P - 1) / P)));
        int RT = 1;
        if (((H + HB - 1) / HB) * KP > kThreads) {
            RT = 4;
            HB = std::max(1, std::min(hb_cap, static_cast<int>(2LL * num_sms() / P)));
        }
        t.RB = (H + HB - 1) / HB;
        auto smem_of = [&](int rc, int ws) {
            return (static_cast<size_t>(t.WP) * K2 + static_cast<size_t>(S2) * (rc + 1) +
                    static_cast<size_t>(ws + (ws > 1 ? 1 : 0)) * rc * K2 + static_cast<size_t>(S2) * K2) * 8 +
                   2 * static_cast<size_t>(rc) * t.WP * 4;
        };
        int RC = (t.RB + RT - 1) / RT * RT;
        // w splits: as many as keep the stage-1 tiles within the CTA's threads, 16 columns each at least
        auto splits = [&](int rc) {
            const int tiles = (rc / RT) * KP;
            return std::max(1, std::min({8, kThreads / tiles, t.WP / 16}));
        };
        while (smem_of(RC, splits(RC)) > static_cast<size_t>(kSmemBudget) / (RT == 1 ? 3 : 2) && RC > 4 * RT)
            RC -= RT;
        t.RC = RC;
        t.WS = splits(RC);
        t.WR = (t.WP / 4 + t.WS - 1) / t.WS * 4;
        const size_t smem = smem_of(RC, t.WS);
        if (smem <= static_cast<size_t>(kSmemBudget) / 2) {
            auto launch = [&](auto kernel) -> cudaError_t {
                int per_sm = 1;
                cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(kernel), smem, kThreads, &per_sm);
                if (e != cudaSuccess) return e;
                cudaLaunchConfig_t lc = {};
                lc.gridDim = dim3(HB, P);
                lc.blockDim = dim3(kThreads);
                lc.dynamicSmemBytes = smem;
                lc.stream = stream;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = HB;
                attr[0].val.clusterDim.y = 1;
                attr[0].val.clusterDim.z = 1;
                lc.attrs = attr;
                lc.numAttrs = 1;
                return cudaLaunchKernelEx(&lc, kernel, t);
            };
            return RT == 4 ? launch(dft_fwd_rows_kernel<4>) : launch(dft_fwd_rows_kernel<1>);
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
    const int S2 = 2 * m1, NPW = W / 2 + 1;
    // shared memory: Ys [S2][KCP] + twci [kRt][S2+1] + Zs [KCP][kRt+1] + twri [KC][NPW], KCP = KC
    // rounded up to even
    auto smem_of = [&](long long kc) {
        const long long kcp = (kc + 1) / 2 * 2;
        return static_cast<size_t>(S2 * kcp + kRt * (S2 + 1LL) + kcp * (kRt + 1LL) + kc * NPW) * 8;
    };
    long long KC = std::max<long long>(1, m2);
    while (KC > 1 && smem_of(KC) > static_cast<size_t>(kSmemBudget)) --KC;
    if (smem_of(KC) > static_cast<size_t>(kSmemBudget)) return cudaErrorInvalidValue;
    a.KC = static_cast<int>(KC);
    const size_t smem = smem_of(KC);
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
    auto threads_for = [&](int rb, int cb) { return ((NPW + cb - 1) / cb) * (kRt / rb); };
    if (threads_for(4, 2) <= kThreads) return run(dft_inv_ffma_kernel<4, 2>);
    const int t82 = threads_for(8, 2), t44 = threads_for(4, 4), t84 = threads_for(8, 4);
    if (t82 <= kThreads && t82 >= t44) return run(dft_inv_ffma_kernel<8, 2>);
    if (t44 <= kThreads) return run(dft_inv_ffma_kernel<4, 4>);
    if (t84 <= kThreads) return run(dft_inv_ffma_kernel<8, 4>);
    if (threads_for(16, 4) <= kThreads) return run(dft_inv_ffma_kernel<16, 4>);
    if (threads_for(kRt, 1) <= kThreads) return run(dft_inv_ffma_kernel<kRt, 1>);
    if (threads_for(kRt, 2) <= kThreads) return run(dft_inv_ffma_kernel<kRt, 2>);
    return run(dft_inv_ffma_kernel<kRt, 4>);
}

}  // namespace scx
