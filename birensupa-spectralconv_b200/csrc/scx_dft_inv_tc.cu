// Tensor-core (tcgen05, bf16x3 -> fp32) zero-padded inverse real DFT from the two corner
// spectra: the B200 replacement for the corner scatter + suFFT C2R of spectral_conv2d_supa
// (spectral_conv/spectral_conv_ops.py:400-431, spectral_conv/spectral_conv_ext.cpp:180-245).
//
// For planes y[h][w] (H, W in {64, 128}), corner slots s < 2*m1 <= 32 and ky < m2 <= 32:
//
//   S4  column inverse, 128 TMEM lanes = (plane, c) for G4 planes, c = (re|im, ky):
//         D4[(p,c)][h] = sum_j Yr[(p,c)][j] * G[h][j]
//       j = (cos|sin, slot); G = cos / sin(2 pi kx_s h / H), 0 for a corner-1 slot that
//       corner 2 overwrites (spectral_conv/reference_pytorch.py:44-46);
//       Yr rows (re, ky) = [Y_re | -Y_im], rows (im, ky) = [Y_im | Y_re].
//   E4  D4 rows -> Z operand in shared memory, MN-major (n = h), one thread per (p, c)
//       writing 16-byte vectors
//   S5  row inverse, 128 TMEM lanes = w (W = 128) or (plane, w) for two planes (W = 64,
//       block-diagonal twiddle operand):
//         D5[w][h] = sum_c E[w][c] * Z[h][c],  E = c_ky/(HW) (cos | -sin)(2 pi ky w / W)
//       with c_ky = 1 for ky = 0 and ky = W/2, else 2 (the C2R Hermitian weights).
//   E5  each thread holds one column w of the plane: y[h][w] stores, 128 bytes per warp
//       instruction, no shared-memory staging.
//
// Every product is bf16x3 (hi*hi + hi*lo + lo*hi) chained along K into one fp32
// accumulator.  Warp roles (persistent, one CTA per SM, contiguous balanced plane ranges):
//   warps 0..3   loaders: corner spectra -> Yr operand (MN-major, double-buffered); the first
//                group's loads are issued before the setup barrier, after griddepcontrol.wait
//                (the kernel is launched as a programmatic dependent of the previous one).  They also run E4 for the
//                upper half of h.
//   warps 4..7   E4 for the lower half of h; each warp hands its S5 chain's Z over alone, so
//                the next group's E4 for a chain waits only for that chain's S5
//   warps 8..15  E5 (two per TMEM sub-partition, halves of h)
//   warp 16      lane 0 brings the twiddle tables into shared memory with one bulk copy and
//                issues the S4 MMAs
//   warp 17      lane 0 issues the S5 MMAs.  A tcgen05.mma costs its issuing thread about
//                110 SM cycles, so S4 of the next group runs while S5 chains are issued.
// Every wait is bounded (about a second); a role that gives up stores a code in the
// device watchdog word and leaves its loop.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "scx_internal.h"
#include "scx_tc.cuh"
#include "scx_tc_host.h"

namespace scx {
namespace {

constexpr int kLoadWarps = 4;
constexpr int kE4Warps = 4;
constexpr int kE5Warps = 8;
constexpr int kE4Warp0 = kLoadWarps;             // 4
constexpr int kE5Warp0 = kE4Warp0 + kE4Warps;    // 8
constexpr int kMmaWarp = kE5Warp0 + kE5Warps;    // 16 (S4), 17 (S5)
constexpr int kThreads = (kMmaWarp + 2) * 32;    // 576
constexpr int kBarE5 = 3;                        // named barrier of the E5 warps
struct InvArgs {
    const float2* in1;
    const float2* in2;
    long long ips;  // input plane stride (float2 units)
    int irs;        // input row stride (float2 units)
    int iks;        // input ky stride (float2 units): 2 for a parity sub-problem of a folded plane
    float* y;
    long long yps;  // output plane stride (floats)
    int yrs;        // output row stride (floats)
    int Q, m1, m2;
    const uint4* tab;  // G (hi, lo) then E (hi, lo)
    uint32_t tab_bytes;
    int* watchdog;
    // quadrant launches: the table and the offset of the first output element of quadrant
    // (alpha, beta) = (quad >> 1, quad & 1)
    const uint4* tabq[4];
    long long yoff[4];
};

struct InvBars {
    uint64_t yFull[2], yEmpty[2], d4Full, d4Empty, zFull[4], zEmpty[4], d5Full[2], d5Empty[2], drain[2], tab;
};

// QUAD: one CTA computes one H x W quadrant of a 2H x 2W output plane directly from the full
// corners (up to 64 spectrum rows, so S4's K is (cos|sin) x 64 slots), with the quadrant's
// offset in its twiddle tables; CTAs come in groups of four, one per quadrant.  Yr is then
// single-buffered to fit shared memory.
template <int H, int W, int N1P, bool QUAD>
struct InvCfg {
    static constexpr int KSL = QUAD ? 64 : 32;     // spectrum-row slots per cos / sin block of S4's K
    static constexpr int KG = 2 * KSL;             // S4 K
    static constexpr int NYB = QUAD ? 1 : 2;       // Yr buffers
    static constexpr int R2P = N1P / 2;            // ky rows per re/im block
    static constexpr int G4 = 128 / N1P;           // planes per S4 group
    static constexpr int G5 = 128 / W;             // planes per S5 chain
    static constexpr int NZ = G4 / G5;             // S5 chains per group
    static constexpr int WPC = G5 * N1P / 32;      // D4 warps per chain (per half of h)
    static constexpr int K5 = G5 * N1P;            // S5 K (block-diagonal for W = 64)
    static constexpr int K5P = (K5 + 63) / 64 * 64;                      // K-major rows span 64 K
    static constexpr uint32_t YRB = 128u * KG * 2u;                      // one Yr part, MN-major
    static constexpr uint32_t GB = static_cast<uint32_t>(H) * KG * 2u;   // one G part, K-major
    static constexpr uint32_t EB = 128u * K5P * 2u;                      // one E part, K-major
    static constexpr uint32_t ZB = static_cast<uint32_t>(H) * K5 * 2u;   // one Z part, MN-major
    static constexpr uint32_t ZSBO = static_cast<uint32_t>(H / 64) * 1024u;  // Z K-group stride
    static constexpr uint32_t OFF_YR = 0;                        // NYB buffers x (hi, lo)
    static constexpr uint32_t OFF_G = OFF_YR + 2u * NYB * YRB;   // G hi, G lo
    static constexpr uint32_t OFF_E = OFF_G + 2u * GB;           // E hi, E lo
    static constexpr uint32_t OFF_Z = OFF_E + 2u * EB;           // NZ chains x (hi, lo)
    static constexpr uint32_t SMEM = OFF_Z + 2u * NZ * ZB + 1024u;
    static_assert(SMEM <= 227u * 1024u - 512u, "shared memory budget");
    static constexpr uint32_t COL_D5 = static_cast<uint32_t>(H);  // D4 at 0
    static constexpr uint32_t COLS = 3u * H;
    static constexpr uint32_t TMEM_COLS = COLS <= 256 ? 256u : 512u;
};

template <int H, int W, int N1P, bool QUAD>
__global__ void __launch_bounds__(kThreads, 1) dft_inv_tc_kernel(const InvArgs a) {
    using C = InvCfg<H, W, N1P, QUAD>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ InvBars bars;
    __shared__ uint32_t tmem_base;
    uint8_t* base = tc::align1024(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int Q = a.Q;
    const int ngrp = QUAD ? static_cast<int>(gridDim.x) / 4 : static_cast<int>(gridDim.x);
    const int grp = QUAD ? static_cast<int>(blockIdx.x) / 4 : static_cast<int>(blockIdx.x);
    const int quad = QUAD ? static_cast<int>(blockIdx.x) % 4 : 0;
    const int q0 = static_cast<int>(static_cast<long long>(grp) * Q / ngrp);
    const int q1 = static_cast<int>(static_cast<long long>(grp + 1) * Q / ngrp);
    const int NG = (q1 - q0 + C::G4 - 1) / C::G4;  // S4 groups
    // S5 chains of group t holding a live plane (fewer than NZ only in a partial last group)
    auto nz_live = [&](int t) { return min(C::NZ, (q1 - q0 - t * C::G4 + C::G5 - 1) / C::G5); };

    // loaders: the spectra of one group, 8 consecutive ky per unit, in registers
    constexpr int kKB = C::R2P / 8;                                   // ky blocks per slot
    // loader warps: the first four, and in quadrant mode (twice the spectrum rows) the four E4
    // warps as well, so that a thread's prefetched units stay in registers
    constexpr int kLW = QUAD ? kLoadWarps + kE4Warps : kLoadWarps;
    constexpr int kUnitsPT = C::G4 * C::KSL * kKB / (kLW * 32);  // units per loader thread
    static_assert(C::G4 * C::KSL * kKB % (kLW * 32) == 0, "loader split");
    float2 v[kUnitsPT][8];
    auto load_group = [&](int t) {
        const int m1 = a.m1, m2 = a.m2, S = 2 * m1;
#pragma unroll
        for (int u = 0; u < kUnitsPT; ++u) {
            const int e = tid + u * kLW * 32;
            const int kb = e % kKB, rest = e / kKB;
            const int ss = rest % C::KSL, p = rest / C::KSL;
            const int q = q0 + t * C::G4 + p;
            const bool live = q < q1 && ss < S;
            const float2* src = ss < m1 ? a.in1 + static_cast<long long>(q) * a.ips + static_cast<long long>(ss) * a.irs
                                        : a.in2 + static_cast<long long>(q) * a.ips + static_cast<long long>(ss - m1) * a.irs;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int ky = kb * 8 + i;
                v[u][i] = (live && ky < m2) ? __ldg(src + static_cast<long long>(ky) * a.iks) : make_float2(0.f, 0.f);
            }
        }
    };
    if (tid == 0) tc::grid_dep_launch();  // the next kernel's CTAs may start their prologue
    if (warp < kLW && NG > 0) {
        tc::grid_dep_wait();  // the spectra come from the previous kernel in the stream
        load_group(0);        // in flight during the setup below
    }

    if (warp == 0) {
        tc::tmem_alloc(&tmem_base, C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&bars.yFull[i], kLW);
            tc::mbar_init(&bars.yEmpty[i], 1);
            tc::mbar_init(&bars.d5Full[i], 1);
            tc::mbar_init(&bars.d5Empty[i], 1);
        }
        tc::mbar_init(&bars.d4Full, 1);
        tc::mbar_init(&bars.d4Empty, 2 * kE4Warps);
        for (int j = 0; j < 4; ++j) {
            tc::mbar_init(&bars.zFull[j], 2 * C::WPC);
            tc::mbar_init(&bars.zEmpty[j], 1);
        }
        tc::mbar_init(&bars.drain[0], 1);
        tc::mbar_init(&bars.drain[1], 1);
        tc::mbar_init(&bars.tab, 1);
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base;

    // E4 of group t by one warp for h in [h_lo, h_lo + H/2): D4 lanes 32q.. hold rows (p, c),
    // written as K row kz of the Z operand of the plane's S5 chain.
    auto e4 = [&](int t, int h_lo) -> bool {
        const int q = warp & 3;
        const int l = q * 32 + lane, p = l / N1P, c = l % N1P;
        const int chain = p / C::G5, kz = (p % C::G5) * N1P + c;
        const bool live = chain < nz_live(t);  // warp-uniform
        bool ok = tc::mbar_wait_bounded(&bars.d4Full, t & 1);
        if (ok && live) ok = tc::mbar_wait_bounded(&bars.zEmpty[chain], (t & 1) ^ 1);
        if (!__all_sync(0xffffffffu, ok)) return false;
        tc::fence_after_sync();
        if (live) {
            const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
            uint8_t* z_hi = base + C::OFF_Z + static_cast<uint32_t>(chain) * 2u * C::ZB;
            uint8_t* z_lo = z_hi + C::ZB;
            const uint32_t krow = static_cast<uint32_t>(kz >> 3) * C::ZSBO + static_cast<uint32_t>(kz & 7) * 128u;
#pragma unroll
            for (int hh = 0; hh < H / 2; hh += 32) {
                const int h0 = h_lo + hh;
                float v[32];
                tc::tmem_ld32_nowait(tmem + lane_addr + static_cast<uint32_t>(h0), v);
                tc::tmem_wait_ld();
#pragma unroll
                for (int c8 = 0; c8 < 4; ++c8) {
                    uint4 h4, l4;
                    tc::split8(v + 8 * c8, h4, l4);
                    const int hc = h0 + 8 * c8;  // first h of this 16-byte chunk
                    const uint32_t off = krow + static_cast<uint32_t>(hc >> 6) * 1024u +
                                         (static_cast<uint32_t>(((hc & 63) >> 3) ^ (kz & 7)) << 4);
                    *reinterpret_cast<uint4*>(z_hi + off) = h4;
                    *reinterpret_cast<uint4*>(z_lo + off) = l4;
                }
            }
        }
        tc::fence_before_sync();
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) {
            tc::mbar_arrive(&bars.d4Empty);
            if (live) tc::mbar_arrive(&bars.zFull[chain]);
        }
        return true;
    };

    if (warp < kLW) {
        // ------------------------------------------------------------ loaders (and E4)
        // Unit (p, s, kb) = 8 consecutive ky of slot s of group plane p feeds four 16-byte
        // vectors of Yr (MN-major, rows contiguous): rows (p, re, ky) at K = s [Y_re] and
        // K = 32 + s [-Y_im], rows (p, im, ky) at K = s [Y_im] and K = 32 + s [Y_re].
        uint8_t* yr0 = base + C::OFF_YR;
        bool ok = true;
        for (int t = 0; t < NG && ok; ++t) {
            const int yb = t % C::NYB;
            ok = __all_sync(0xffffffffu, tc::mbar_wait_bounded(&bars.yEmpty[yb], ((t / C::NYB) & 1) ^ 1));
            if (!ok) break;
            uint8_t* yr_hi = yr0 + static_cast<uint32_t>(yb) * 2u * C::YRB;
            uint8_t* yr_lo = yr_hi + C::YRB;
#pragma unroll
            for (int u = 0; u < kUnitsPT; ++u) {
                const int e = tid + u * kLW * 32;
                const int kb = e % kKB, rest = e / kKB;
                const int ss = rest % C::KSL, p = rest / C::KSL;
                uint32_t re_hi[4], re_lo[4], im_hi[4], im_lo[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    tc::split_pair(v[u][2 * i].x, v[u][2 * i + 1].x, re_hi[i], re_lo[i]);
                    tc::split_pair(v[u][2 * i].y, v[u][2 * i + 1].y, im_hi[i], im_lo[i]);
                }
                const int mre = p * N1P + kb * 8, mim = mre + C::R2P;
                auto put = [&](int m, int k, const uint32_t* hi, const uint32_t* lo, uint32_t neg) {
                    const uint32_t off = static_cast<uint32_t>(k >> 3) * 2048u + static_cast<uint32_t>(m >> 6) * 1024u +
                                         static_cast<uint32_t>(k & 7) * 128u +
                                         (static_cast<uint32_t>(((m & 63) >> 3) ^ (k & 7)) << 4);
                    *reinterpret_cast<uint4*>(yr_hi + off) = make_uint4(hi[0] ^ neg, hi[1] ^ neg, hi[2] ^ neg, hi[3] ^ neg);
                    *reinterpret_cast<uint4*>(yr_lo + off) = make_uint4(lo[0] ^ neg, lo[1] ^ neg, lo[2] ^ neg, lo[3] ^ neg);
                };
                put(mre, ss, re_hi, re_lo, 0u);
                put(mre, C::KSL + ss, im_hi, im_lo, 0x80008000u);  // -Y_im: bf16 sign bits
                put(mim, ss, im_hi, im_lo, 0u);
                put(mim, C::KSL + ss, re_hi, re_lo, 0u);
            }
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars.yFull[yb]);
            if (t + 1 < NG) load_group(t + 1);
            ok = e4(t, warp < kLoadWarps ? H / 2 : 0);
        }
        if (!ok && lane == 0) atomicExch(a.watchdog, warp < kLoadWarps ? 30 : 31);
    } else if (warp < kE5Warp0) {
        // ------------------------------------------------------------ E4 (lower half of h)
        bool ok = true;
        for (int t = 0; t < NG && ok; ++t) ok = e4(t, 0);
        if (!ok && lane == 0) atomicExch(a.watchdog, 31);
    } else if (warp < kMmaWarp) {
        // ------------------------------------------------------------ E5
        const int q = warp & 3, sub = (warp - kE5Warp0) >> 2;  // sub-partition, half of h
        const int e5tid = tid - kE5Warp0 * 32;                  // 0..255
        const int l = q * 32 + lane;
        const int g = l / W, w = l % W;
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        constexpr int HH = H / 2;
        bool ok = true;
        int n = 0;  // S5 chains consumed
        for (int t = 0; t < NG && ok; ++t) {
            const int nzl = nz_live(t);
            for (int j = 0; j < nzl; ++j, ++n) {
                const int b = n & 1;
                ok = tc::mbar_wait_bounded(&bars.d5Full[b], (n >> 1) & 1);
                if (tc::named_any(kBarE5, kE5Warps * 32, !ok)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const int qp = q0 + t * C::G4 + j * C::G5 + g;  // warp-uniform plane
                float* dst = a.y + (QUAD ? a.yoff[quad] : 0) + static_cast<long long>(qp) * a.yps +
                             static_cast<long long>(sub * HH) * a.yrs + w;
                const uint32_t src = tmem + lane_addr + C::COL_D5 + static_cast<uint32_t>(b * H + sub * HH);
#pragma unroll
                for (int h0 = 0; h0 < HH; h0 += 32) {
                    float v[32];
                    tc::tmem_ld32_nowait(src + static_cast<uint32_t>(h0), v);
                    tc::tmem_wait_ld();
                    if (qp < q1) {
#pragma unroll
                        for (int k = 0; k < 32; ++k) __stcs(dst + static_cast<long long>(h0 + k) * a.yrs, v[k]);
                    }
                }
                tc::fence_before_sync();
                tc::named_sync(kBarE5, kE5Warps * 32);
                if (e5tid == 0) tc::mbar_arrive(&bars.d5Empty[b]);
            }
        }
        if (!ok && e5tid == 0) atomicExch(a.watchdog, 32);
    } else if (warp >= kMmaWarp && lane == 0) {
        // ------------------------------------------------------------ MMA issuers
        const int role = warp - kMmaWarp;  // 0: S4 (and the table copy), 1: S5
        const uint32_t sb = tc::smem_u32(base);
        if (role == 0) {
            tc::mbar_arrive_expect_tx(&bars.tab, a.tab_bytes);
            tc::bulk_g2s(base + C::OFF_G, QUAD ? a.tabq[quad] : a.tab, a.tab_bytes, &bars.tab);
        }
        bool ok = tc::mbar_wait_bounded(&bars.tab, 0);
        if (role == 0) {
            // S4: parts (Yr_hi, G_hi), (Yr_hi, G_lo), (Yr_lo, G_hi), K = KG each
            constexpr uint32_t id4 = tc::idesc_bf16(128, H) | tc::kIdescAMajorMN;
            const uint64_t dG[2] = {tc::desc_sw128(sb + C::OFF_G), tc::desc_sw128(sb + C::OFF_G + C::GB)};
            for (int t = 0; t < NG && ok; ++t) {
                const int yb = t % C::NYB;
                ok = tc::mbar_wait_bounded(&bars.yFull[yb], (t / C::NYB) & 1) &&
                     tc::mbar_wait_bounded(&bars.d4Empty, (t & 1) ^ 1);
                if (!ok) break;
                tc::fence_after_sync();
                const uint32_t yr = sb + C::OFF_YR + static_cast<uint32_t>(yb) * 2u * C::YRB;
                const uint64_t dY[2] = {tc::desc_mn_sw128(yr, 1024u, 2048u), tc::desc_mn_sw128(yr + C::YRB, 1024u, 2048u)};
#pragma unroll
                for (int part = 0; part < 3; ++part) {
                    const int ap = part == 2 ? 1 : 0, bp = part == 1 ? 1 : 0;
#pragma unroll
                    for (int ks = 0; ks < C::KG / 16; ++ks) {
                        // G is K-major with 64-element K blocks of H rows each
                        const uint32_t ao = (static_cast<uint32_t>(ks) * 4096u) >> 4;
                        const uint32_t bo = (static_cast<uint32_t>(ks >> 2) * H * 128u + (ks & 3) * 32u) >> 4;
                        tc::mma_bf16(tmem, dY[ap] + ao, dG[bp] + bo, id4, (part | ks) ? 1u : 0u);
                    }
                }
                tc::mma_commit(&bars.yEmpty[yb]);
                tc::mma_commit(&bars.d4Full);
            }
        } else {
            // S5 chains of each group once E4 has written its Z
            constexpr uint32_t id5 = tc::idesc_bf16(128, H) | tc::kIdescBMajorMN;
            const uint32_t d5 = tmem + C::COL_D5;
            const uint64_t dE[2] = {tc::desc_sw128(sb + C::OFF_E), tc::desc_sw128(sb + C::OFF_E + C::EB)};
            int n = 0;
            for (int t = 0; t < NG && ok; ++t) {
                const int nzl = nz_live(t);
                for (int j = 0; j < nzl && ok; ++j, ++n) {
                    const int b = n & 1;
                    ok = tc::mbar_wait_bounded(&bars.zFull[j], t & 1) &&
                         tc::mbar_wait_bounded(&bars.d5Empty[b], ((n >> 1) & 1) ^ 1);
                    if (!ok) break;
                    tc::fence_after_sync();
                    const uint32_t zc = sb + C::OFF_Z + static_cast<uint32_t>(j) * 2u * C::ZB;
                    const uint64_t dZ[2] = {tc::desc_mn_sw128(zc, 1024u, C::ZSBO), tc::desc_mn_sw128(zc + C::ZB, 1024u, C::ZSBO)};
                    const uint32_t dd = d5 + static_cast<uint32_t>(b * H);
#pragma unroll
                    for (int part = 0; part < 3; ++part) {
                        const int ap = part == 2 ? 1 : 0, bp = part == 1 ? 1 : 0;
#pragma unroll
                        for (int ks = 0; ks < C::K5 / 16; ++ks) {
                            const uint32_t ao = (static_cast<uint32_t>(ks >> 2) * 128u * 128u + (ks & 3) * 32u) >> 4;
                            const uint32_t bo = (static_cast<uint32_t>(ks) * 2u * C::ZSBO) >> 4;
                            tc::mma_bf16(dd, dE[ap] + ao, dZ[bp] + bo, id5, (part | ks) ? 1u : 0u);
                        }
                    }
                    tc::mma_commit(&bars.d5Full[b]);
                    tc::mma_commit(&bars.zEmpty[j]);
                }
            }
        }
        if (!ok) atomicExch(a.watchdog, 33);
        // every MMA this thread issued has completed before TMEM is released
        tc::mma_commit(&bars.drain[role]);
        tc::mbar_wait_bounded(&bars.drain[role], 0);
    }
    // lanes that skipped a single-lane role rejoin their warp before the CTA barrier
    __syncwarp();
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host side

struct InvTable {
    const uint4* data;
    uint32_t bytes;
};

std::mutex g_mutex;
std::map<std::tuple<int, int, int, int, int, int>, InvTable> g_tables;

// G (H rows x 64, K-major) hi then lo, followed by E (128 rows x K5, K-major) hi then lo.  With
// a sub-problem description they hold the modes of that parity of a folded plane (TcSub).
cudaError_t get_inv_table(int H, int W, int m1, int m2, int N1P, const TcSub* sub, const InvTable** out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    const int sub_code = sub ? 1 + sub->a * 2 + sub->b + 4 * (sub->m1_full + 64 * sub->period_h) : 0;
    const auto key = std::make_tuple(dev, H, W, m1, m2, sub_code);
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_tables.find(key);
    if (it != g_tables.end()) {
        *out = &it->second;
        return cudaSuccess;
    }
    const int S = 2 * m1, R2P = N1P / 2, G5 = 128 / W, K5 = G5 * N1P;
    constexpr int kKg = 64;  // S4 K of the direct kernel: (cos|sin) x 32 slots
    host::KMajor ghi(H, kKg), glo(H, kKg);
    const int Hp = sub ? sub->period_h : H, Wp = sub ? sub->period_w : W;
    for (int s = 0; s < S; ++s) {
        const int kx = sub ? sub_row(*sub, s, m1) : host::slot_row(s, H, m1);
        const int m1f = sub ? sub->m1_full : m1;
        if (s < m1 && kx >= Hp - m1f) continue;  // corner-1 row that corner 2 overwrites
        for (int h = 0; h < H; ++h) {
            const double t = host::ang(kx, h, Hp);
            uint16_t hi, lo;
            host::bf16_split(std::cos(t), hi, lo);
            ghi.set(h, s, hi);
            glo.set(h, s, lo);
            host::bf16_split(std::sin(t), hi, lo);
            ghi.set(h, 32 + s, hi);
            glo.set(h, 32 + s, lo);
        }
    }
    host::KMajor ehi(128, K5), elo(128, K5);
    const double inv_hw = 1.0 / (static_cast<double>(Hp) * static_cast<double>(Wp));
    for (int g = 0; g < G5; ++g)
        for (int w = 0; w < W; ++w)
            for (int ky = 0; ky < m2; ++ky) {
                const int kyf = sub ? 2 * ky + sub->b : ky;  // column of the full spectrum
                const bool single = (kyf == 0) || ((Wp % 2 == 0) && (kyf == Wp / 2));
                const double cw = (single ? 1.0 : 2.0) * inv_hw;
                const double t = host::ang(kyf, w, Wp);
                uint16_t hi, lo;
                host::bf16_split(cw * std::cos(t), hi, lo);
                ehi.set(g * W + w, g * N1P + ky, hi);
                elo.set(g * W + w, g * N1P + ky, lo);
                host::bf16_split(-cw * std::sin(t), hi, lo);
                ehi.set(g * W + w, g * N1P + R2P + ky, hi);
                elo.set(g * W + w, g * N1P + R2P + ky, lo);
            }
    std::vector<uint16_t> buf(ghi.data);
    for (const auto* part : {&glo, &ehi, &elo}) buf.insert(buf.end(), part->data.begin(), part->data.end());
    const size_t bytes = buf.size() * 2;
    void* d = nullptr;
    err = cudaMalloc(&d, bytes);
    if (err != cudaSuccess) return err;
    err = cudaMemcpy(d, buf.data(), bytes, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        cudaFree(d);
        return err;
    }
    InvTable t;
    t.data = static_cast<const uint4*>(d);
    t.bytes = static_cast<uint32_t>(bytes);
    auto res = g_tables.emplace(key, t);
    *out = &res.first->second;
    return cudaSuccess;
}

// Quadrant tables for planes of Hf x Wf = 2H x 2W: G for the rows of quadrant alpha (all 2 m1
// spectrum rows, cos block then sin block, KSL = 64 slots each) and E for the columns of
// quadrant beta, the angles taken at the full-plane position (h + H alpha, w + W beta).
cudaError_t get_inv_table_quad(int Hf, int Wf, int m1, int m2, int quad, const InvTable** out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    const auto key = std::make_tuple(dev, Hf, Wf, m1, m2, -1 - quad);
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_tables.find(key);
    if (it != g_tables.end()) {
        *out = &it->second;
        return cudaSuccess;
    }
    using C = InvCfg<128, 128, 64, true>;
    const int H = Hf / 2, W = Wf / 2, alpha = quad >> 1, beta = quad & 1;
    host::KMajor ghi(H, C::KG), glo(H, C::KG);
    for (int s = 0; s < 2 * m1; ++s) {
        const int kx = host::slot_row(s, Hf, m1);
        if (s < m1 && kx >= Hf - m1) continue;  // corner-1 row that corner 2 overwrites
        for (int h = 0; h < H; ++h) {
            const double t = host::ang(kx, h + H * alpha, Hf);
            uint16_t hi, lo;
            host::bf16_split(std::cos(t), hi, lo);
            ghi.set(h, s, hi);
            glo.set(h, s, lo);
            host::bf16_split(std::sin(t), hi, lo);
            ghi.set(h, C::KSL + s, hi);
            glo.set(h, C::KSL + s, lo);
        }
    }
    host::KMajor ehi(128, C::K5), elo(128, C::K5);
    const double inv_hw = 1.0 / (static_cast<double>(Hf) * static_cast<double>(Wf));
    for (int w = 0; w < W; ++w)
        for (int ky = 0; ky < m2; ++ky) {
            const bool single = (ky == 0) || ((Wf % 2 == 0) && (ky == Wf / 2));
            const double cw = (single ? 1.0 : 2.0) * inv_hw;
            const double t = host::ang(ky, w + W * beta, Wf);
            uint16_t hi, lo;
            host::bf16_split(cw * std::cos(t), hi, lo);
            ehi.set(w, ky, hi);
            elo.set(w, ky, lo);
            host::bf16_split(-cw * std::sin(t), hi, lo);
            ehi.set(w, C::R2P + ky, hi);
            elo.set(w, C::R2P + ky, lo);
        }
    std::vector<uint16_t> buf(ghi.data);
    for (const auto* part : {&glo, &ehi, &elo}) buf.insert(buf.end(), part->data.begin(), part->data.end());
    const size_t bytes = buf.size() * 2;
    void* d = nullptr;
    err = cudaMalloc(&d, bytes);
    if (err != cudaSuccess) return err;
    err = cudaMemcpy(d, buf.data(), bytes, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        cudaFree(d);
        return err;
    }
    InvTable t;
    t.data = static_cast<const uint4*>(d);
    t.bytes = static_cast<uint32_t>(bytes);
    auto res = g_tables.emplace(key, t);
    *out = &res.first->second;
    return cudaSuccess;
}

template <int H, int W, int N1P, bool QUAD>
cudaError_t run_inv(const InvArgs& a, cudaStream_t stream) {
    using C = InvCfg<H, W, N1P, QUAD>;
    if (a.tab_bytes != 2u * C::GB + 2u * C::EB) return cudaErrorInvalidValue;
    auto kernel = dft_inv_tc_kernel<H, W, N1P, QUAD>;
    int per_sm = 1;
    cudaError_t err = prepare_kernel(reinterpret_cast<const void*>(kernel), C::SMEM, kThreads, &per_sm);
    if (err != cudaSuccess) return err;
    // quadrants: groups of four CTAs, at most one per SM, at most one group per S4 group of planes
    const int grid = QUAD ? 4 * std::max(1, std::min(num_sms() / 4, (a.Q + C::G4 - 1) / C::G4))
                          : std::max(1, std::min(a.Q, num_sms()));
    return launch_chained(kernel, dim3(grid), dim3(kThreads), C::SMEM, stream, a);
}

template <int H, int W>
cudaError_t run_inv_n(const InvArgs& a, int N1P, cudaStream_t stream) {
    return N1P == 32 ? run_inv<H, W, 32, false>(a, stream) : run_inv<H, W, 64, false>(a, stream);
}

}  // namespace

bool tc_inv_supported(int H, int W, int m1, int m2) {
    return (H == 64 || H == 128) && (W == 64 || W == 128) && m1 >= 1 && 2 * m1 <= 32 && m2 >= 1 && m2 <= 32 &&
           m2 <= W / 2 + 1;
}

cudaError_t launch_dft_inv_tc(const float2* in1, const float2* in2, long long ips, int irs, float* y, int Q, int H,
                              int W, int m1, int m2, cudaStream_t stream, const TcSub* sub) {
    if (!tc_inv_supported(H, W, m1, m2) || Q <= 0 || (reinterpret_cast<uintptr_t>(y) & 3) != 0)
        return cudaErrorInvalidValue;
    const int N1P = m2 <= 16 ? 32 : 64;
    const InvTable* t = nullptr;
    cudaError_t e = get_inv_table(H, W, m1, m2, N1P, sub, &t);
    if (e != cudaSuccess) return e;
    int* wd = nullptr;
    e = device_watchdog(&wd);
    if (e != cudaSuccess) return e;
    InvArgs a = {};
    a.in1 = in1;
    a.in2 = in2;
    a.ips = ips;
    a.irs = irs;
    a.iks = sub ? 2 : 1;
    a.y = y;
    a.yps = static_cast<long long>(H) * W;
    a.yrs = W;
    a.Q = Q;
    a.m1 = m1;
    a.m2 = m2;
    a.tab = t->data;
    a.tab_bytes = t->bytes;
    a.watchdog = wd;
    if (H == 64 && W == 64) return run_inv_n<64, 64>(a, N1P, stream);
    if (H == 64 && W == 128) return run_inv_n<64, 128>(a, N1P, stream);
    if (H == 128 && W == 64) return run_inv_n<128, 64>(a, N1P, stream);
    return run_inv_n<128, 128>(a, N1P, stream);
}

bool tc_quad_supported(int H, int W, int m1, int m2) {
    return H == 256 && W == 256 && m1 >= 1 && m1 <= 32 && m2 >= 1 && m2 <= 32;
}

cudaError_t launch_dft_inv_tc_quad(const float2* in1, const float2* in2, long long ips, int irs, float* y, int Q,
                                   int H, int W, int m1, int m2, cudaStream_t stream) {
    if (!tc_quad_supported(H, W, m1, m2) || Q <= 0 || (reinterpret_cast<uintptr_t>(y) & 3) != 0)
        return cudaErrorInvalidValue;
    InvArgs a = {};
    for (int q = 0; q < 4; ++q) {
        const InvTable* t = nullptr;
        cudaError_t e = get_inv_table_quad(H, W, m1, m2, q, &t);
        if (e != cudaSuccess) return e;
        a.tabq[q] = t->data;
        a.tab_bytes = t->bytes;
        a.yoff[q] = static_cast<long long>((q >> 1) * (H / 2)) * W + (q & 1) * (W / 2);
    }
    cudaError_t e = device_watchdog(&a.watchdog);
    if (e != cudaSuccess) return e;
    a.in1 = in1;
    a.in2 = in2;
    a.ips = ips;
    a.irs = irs;
    a.iks = 1;
    a.y = y;
    a.yps = static_cast<long long>(H) * W;
    a.yrs = W;
    a.Q = Q;
    a.m1 = m1;
    a.m2 = m2;
    a.tab = a.tabq[0];
    return run_inv<128, 128, 64, true>(a, stream);
}

}  // namespace scx
