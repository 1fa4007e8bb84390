// Tensor-core (tcgen05, bf16x3 -> fp32) truncated forward real DFT, column transform first:
// the B200 replacement for the suFFT R2C + corner gather of spectral_conv2d_supa
// (spectral_conv/spectral_conv_ops.py:372-399, spectral_conv/spectral_conv_ext.cpp:123-178).
//
// For every plane x[h][w] (H, W in {64, 128}) and corner slots s < 2*m1 <= 32 (row
// kx_s = s for corner 1, H - 2*m1 + s for corner 2), ky < m2 <= 32:
//
//   S2  column DFT on the tensor core, A = x^T from TMEM:
//         D2[(g,w)][j] = sum_h x_g[h][w] * F[j][h]       lanes (g,w): G1 = 128/W planes
//       F rows j = 32*grp + 16*cs + i hold cos (cs = 0) / sin (cs = 1) of 2 pi kx_s h / H
//       for slot s = 16*grp + i.  Each plane is read once from HBM by the TMA engine, each
//       thread reads its column (lane = w) from shared memory, splits it into bf16 hi/lo
//       in registers and writes the pairs to TMEM with tcgen05.st.
//   E2  D2 rows -> C/S operand in shared memory (MN-major: each thread writes the 64
//       values of its column as 16-byte vectors), rows m = 64*plane + j, K = w
//   S1  row DFT:   D1[m][n] = sum_w CS[m][w] * TW[n][w]   (M = 128 = 2 planes)
//       TW rows n < R2: cos(2 pi n w / W), rows R2 + n: -sin(2 pi n w / W)
//   E1  X[s][ky] = (Cc + Ss) + i (Cs - Sc) from the cos row (lane i) and the sin row
//       (lane i + 16) of slot s, exchanged with one shuffle; written to the corner arrays.
//
// Every product is bf16x3 (hi*hi + hi*lo + lo*hi) accumulated in fp32 TMEM.  A tcgen05.mma
// issued by one thread costs about 110 SM cycles whatever its N up to 128 (measured on B200),
// while the tensor core finishes an M128 N64 K16 product in about 35 when several threads
// issue, so S2 is split over two issuing warps with accumulators of their own, added by the
// epilogue in a fixed order, and S1 has a third:
//   S2P  x_hi * [F_hi; F_lo]  (N = 128)    S2Q  x_lo * F_hi  (N = 64)
//   S1   CS_hi * [TW_hi; TW_lo] and CS_lo * TW_hi, both into D1, in that order per K step
//
// Warp roles (persistent, one CTA per SM, planes split into contiguous balanced ranges):
//   warp 19      lane 0 initialises the barriers, starts the table and the first ring loads
//                before the setup barrier (the x loads after griddepcontrol.wait: the kernel is
//                launched as a programmatic dependent of the previous one), then streams 32-row chunks of x into a shared-memory
//                ring with 1-D bulk copies (about 100 KB in flight per SM)
//   warps 0..7   converters: ring -> bf16 hi/lo in registers -> the TMEM A operand, stored
//                only while no A-in-TMEM MMA is in flight (stores issued while such MMAs ran
//                corrupted about 1% of the planes on B200, even into other columns)
//   warps 8..15  epilogue: E2 for every column tile, E1 for every 2-plane tile
//   warps 16..18 lane 0 of each issues the S2P, S2Q and S1 MMAs
// All hand-offs are mbarriers; every wait is bounded (about a second): a role that gives up
// stores a code in the device watchdog word and leaves its loop, so the kernel returns.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "scx_internal.h"
#include "scx_tc.cuh"
#include "scx_tc_host.h"

namespace scx {
namespace {

constexpr int kConvWarps = 8;                      // 2 per TMEM sub-partition
constexpr int kEpiWarps = 8;                       // 2 per TMEM sub-partition
constexpr int kMmaWarp = kConvWarps + kEpiWarps;   // 16..18: S2P, S2Q, S1
constexpr int kTmaWarp = kMmaWarp + 3;             // 19
constexpr int kThreads = (kTmaWarp + 1) * 32;      // 640
constexpr int kBarEpi = 1;                         // named barrier of the epilogue warps
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kJF = 64;                            // column-DFT rows per plane (2 groups x 32)
constexpr int kFRows = 2 * kJF;                    // [F_hi; F_lo]
constexpr int kChunkRows = 32;                     // rows of x per ring slot
constexpr int kMaxSlots = 8;

struct FwdArgs {
    const float* x;
    float2* out1;
    float2* out2;
    long long ops;  // output plane stride (float2 units)
    int ors;        // output row stride (float2 units)
    int oks;        // output ky stride (float2 units): 2 for a parity sub-problem of a folded plane
    int P, m1, m2;
    const uint4* tab;  // [F_hi; F_lo] then [TW_hi; TW_lo], both K-major SW128
    uint32_t tab_bytes;
    int* watchdog;
    // folded launches (x holds the full 2H x 2W planes): the table of parity q = 2a + b and the
    // offset of its first output element (a rows, b columns) within out1 / out2
    const uint4* tabq[4];
    long long qoff[4];
};

struct FwdBars {
    uint64_t full[kMaxSlots], empty[kMaxSlots];  // x ring
    uint64_t aFull, aEmpty;                      // A operand (TMEM)
    uint64_t d2Full, d2Empty, csFull, csEmpty, d1Full, d1Empty, tab;
    uint64_t drain[3];
};

// FOLD: the kernel reads full planes of 2H x 2W samples and computes the parity sub-planes
// (the H x W sub-problems of TcSub) in its converters; a ring chunk then holds CHR rows of the
// upper half and the same CHR rows of the lower half of each plane, full width.
template <int H, int W, int R2, bool FOLD>
struct FwdCfg {
    static constexpr int G1 = 128 / W;  // planes per column tile (TMEM lanes = (plane, w))
    static constexpr int CT = 2 / G1;   // column tiles per 2-plane tile
    static constexpr int N1 = 2 * R2;   // S1 columns per TW part (cos block | -sin block)
    static constexpr int CHR = FOLD ? 16 : kChunkRows;  // (sub-)plane rows per ring chunk
    static constexpr int RPW = CHR / 2;                  // rows per converter warp per chunk
    static constexpr int CPC = H / CHR;                  // ring chunks per column tile
    static constexpr uint32_t HALF_CHUNK = static_cast<uint32_t>(CHR) * (FOLD ? 2 * W : W) * 4u;
    static constexpr uint32_t PLANE_CHUNK = FOLD ? 2u * HALF_CHUNK : HALF_CHUNK;
    static constexpr uint32_t SLOT = PLANE_CHUNK * G1;  // 16 KB (32 KB folded)
    static constexpr uint32_t CSB = 128u * W * 2u;      // one CS operand (hi or lo), MN-major
    static constexpr uint32_t OFF_FB = 2u * CSB;        // CS hi | CS lo
    static constexpr uint32_t FB_BYTES = static_cast<uint32_t>(kFRows) * H * 2u;
    static constexpr uint32_t OFF_TW = OFF_FB + FB_BYTES;
    static constexpr uint32_t TW_BYTES = 2u * N1 * W * 2u;
    static constexpr uint32_t OFF_RING = OFF_TW + TW_BYTES;
    static constexpr uint32_t BUDGET = 227u * 1024u - 1024u - 512u;  // minus alignment slack and static smem
    static constexpr int NS = static_cast<int>((BUDGET - OFF_RING) / SLOT) < kMaxSlots
                                  ? static_cast<int>((BUDGET - OFF_RING) / SLOT)
                                  : kMaxSlots;
    static constexpr uint32_t SMEM = OFF_RING + static_cast<uint32_t>(NS) * SLOT + 1024u;
    static_assert(NS >= 3, "x ring too small");
    // TMEM columns: A (H: hi H/2 packed columns | lo H/2) | D2P (kFRows: F_hi part | F_lo part)
    // | D2Q (kJF) | D1 (2*N1: TW_hi part | TW_lo part)
    static constexpr uint32_t COL_D2P = H;
    static constexpr uint32_t COL_D2Q = COL_D2P + kFRows;
    static constexpr uint32_t COL_D1 = COL_D2Q + kJF;
    static constexpr uint32_t COLS = COL_D1 + 2u * N1;
    static constexpr uint32_t TMEM_COLS = COLS <= 256 ? 256u : 512u;
    static_assert(COLS <= 512, "TMEM budget");
};

template <int H, int W, int R2, bool FOLD>
__global__ void __launch_bounds__(kThreads, 1) dft_fwd_tc_kernel(const FwdArgs a) {
    using C = FwdCfg<H, W, R2, FOLD>;
    constexpr int N1 = C::N1;
    extern __shared__ uint8_t smem_raw[];
    __shared__ FwdBars bars;
    __shared__ uint32_t tmem_base;
    uint8_t* base = tc::align1024(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // this CTA's planes [p0, p1): contiguous, sizes differ by at most one.  Folded: CTAs come in
    // groups of four, one per parity q = 2a + b, that take the same planes in the same order,
    // so a plane is read from HBM about once and by the other three from L2.
    const int P = a.P;
    const int ngrp = FOLD ? static_cast<int>(gridDim.x) / 4 : static_cast<int>(gridDim.x);
    const int grp = FOLD ? static_cast<int>(blockIdx.x) / 4 : static_cast<int>(blockIdx.x);
    const int qpar = FOLD ? static_cast<int>(blockIdx.x) % 4 : 0;
    const int p0 = static_cast<int>(static_cast<long long>(grp) * P / ngrp);
    const int p1 = static_cast<int>(static_cast<long long>(grp + 1) * P / ngrp);
    const int NC = (p1 - p0 + C::G1 - 1) / C::G1;  // column tiles
    const int NT = (NC + C::CT - 1) / C::CT;        // 2-plane tiles
    const int NK = NC * C::CPC;                     // ring chunks

    // the producer's loads of chunk k: every live plane of its column tile
    auto issue_chunk = [&](int k) {
        const int c = k / C::CPC, ch = k % C::CPC, slot = k % C::NS;
        const int pa = p0 + c * C::G1, np = min(C::G1, p1 - pa);
        uint8_t* ring = base + C::OFF_RING;
        tc::mbar_arrive_expect_tx(&bars.full[slot], static_cast<uint32_t>(np) * C::PLANE_CHUNK);
        for (int g = 0; g < np; ++g) {
            uint8_t* dst = ring + static_cast<uint32_t>(slot) * C::SLOT + static_cast<uint32_t>(g) * C::PLANE_CHUNK;
            if (FOLD) {  // rows [CHR ch, CHR ch + CHR) of both halves of the 2H x 2W plane
                const float* src = a.x + (static_cast<size_t>(pa + g) * (2 * H) + ch * C::CHR) * (2 * W);
                tc::bulk_g2s(dst, src, C::HALF_CHUNK, &bars.full[slot]);
                tc::bulk_g2s(dst + C::HALF_CHUNK, src + static_cast<size_t>(H) * (2 * W), C::HALF_CHUNK,
                             &bars.full[slot]);
            } else {
                tc::bulk_g2s(dst, a.x + (static_cast<size_t>(pa + g) * H + ch * C::CHR) * W, C::PLANE_CHUNK,
                             &bars.full[slot]);
            }
        }
    };
    const int k_first = min(NK, C::NS);  // chunks issued before the setup barrier
    // Folded launches: L2 prefetch of the chunk PF chunks ahead.  The ring alone keeps NS chunks
    // in flight per CTA; the prefetched chunk is in L2 by the time its slot frees and its bulk
    // copy is issued (256 x 256, B16 C64: 122.7 -> 114.4 us at one ring ahead, 116.2 us at two).
    // Unfolded planes stream each byte once and the prefetches only delayed their first chunks
    // (15.0 -> 16.1 us at 128 x 128), so they have none.
    constexpr int PF = C::NS;
    auto prefetch_chunk = [&](int k) {
        if (!FOLD || k >= NK) return;
        const int c = k / C::CPC, ch = k % C::CPC;
        const int pa = p0 + c * C::G1, np = min(C::G1, p1 - pa);
        for (int g = 0; g < np; ++g) {
            if (FOLD) {
                const float* src = a.x + (static_cast<size_t>(pa + g) * (2 * H) + ch * C::CHR) * (2 * W);
                tc::prefetch_l2(src, C::HALF_CHUNK);
                tc::prefetch_l2(src + static_cast<size_t>(H) * (2 * W), C::HALF_CHUNK);
            } else {
                tc::prefetch_l2(a.x + (static_cast<size_t>(pa + g) * H + ch * C::CHR) * W, C::PLANE_CHUNK);
            }
        }
    };

    if (tid == 0) tc::grid_dep_launch();  // the next kernel's CTAs may start their prologue
    if (warp == 0) {
        tc::tmem_alloc(&tmem_base, C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    if (warp == kTmaWarp && lane == 0) {
        for (int i = 0; i < kMaxSlots; ++i) {
            tc::mbar_init(&bars.full[i], 1);
            tc::mbar_init(&bars.empty[i], kConvWarps);
        }
        tc::mbar_init(&bars.aFull, kConvWarps);
        tc::mbar_init(&bars.aEmpty, 2);
        tc::mbar_init(&bars.d2Full, 2);
        tc::mbar_init(&bars.d2Empty, 1);
        tc::mbar_init(&bars.csFull, 1);
        tc::mbar_init(&bars.csEmpty, 1);
        tc::mbar_init(&bars.d1Full, 1);
        tc::mbar_init(&bars.d1Empty, 1);
        tc::mbar_init(&bars.tab, 1);
        for (int i = 0; i < 3; ++i) tc::mbar_init(&bars.drain[i], 1);
        tc::fence_async_smem();
        tc::mbar_arrive_expect_tx(&bars.tab, a.tab_bytes);
        tc::bulk_g2s(base + C::OFF_FB, FOLD ? a.tabq[qpar] : a.tab, a.tab_bytes, &bars.tab);
        // x may be written by the previous kernel in the stream; the ring starts empty, so the
        // first NS chunks need no slot wait
        tc::grid_dep_wait();
        for (int k = 0; k < k_first; ++k) issue_chunk(k);
        for (int k = k_first; k < k_first + PF; ++k) prefetch_chunk(k);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base;

    if (warp < kConvWarps) {
        // ------------------------------------------------------------ converters
        // Warp (q, hf) owns TMEM lanes 32q.. and rows [RPW hf, RPW hf + RPW) of every ring chunk:
        // it reads its column of those rows from shared memory, splits them into bf16 hi/lo
        // pairs and stores RPW / 2 packed columns of each into the A operand.  Folded, each
        // value is the parity-q combination of the four quadrant samples, computed with the
        // additions and subtractions of the fold kernel (scx_fold.cu) in the same order
        // (a signed sum by fmaf with +-1 rounds exactly as the add or subtract does).
        const int q = warp & 3, hf = warp >> 2;
        const int l = q * 32 + lane, g = l / W, w = l % W;
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        const uint8_t* ring = base + C::OFF_RING;
        bool ok = true;
        for (int c = 0; c < NC && ok; ++c) {
            const bool live = p0 + c * C::G1 + g < p1;  // warp-uniform
            // read and split the whole column tile while the previous tile's MMAs run
            uint32_t hi[C::CPC][C::RPW / 2], lo[C::CPC][C::RPW / 2];
#pragma unroll
            for (int ch = 0; ch < C::CPC; ++ch) {
                const int k = c * C::CPC + ch, slot = k % C::NS, use = k / C::NS;
                if (ok) ok = __all_sync(0xffffffffu, tc::mbar_wait_bounded(&bars.full[slot], use & 1));
                if (ok) {
                    const uint8_t* pc = ring + static_cast<uint32_t>(slot) * C::SLOT + static_cast<uint32_t>(g) * C::PLANE_CHUNK;
                    float v[C::RPW];
                    if constexpr (FOLD) {
                        constexpr int WF = 2 * W;  // full-plane row length
                        const float sa = (qpar & 2) ? -1.f : 1.f, sb = (qpar & 1) ? -1.f : 1.f;
                        const float* top = reinterpret_cast<const float*>(pc) + (C::RPW * hf) * WF + w;
                        const float* bot = reinterpret_cast<const float*>(pc + C::HALF_CHUNK) + (C::RPW * hf) * WF + w;
#pragma unroll
                        for (int j = 0; j < C::RPW; ++j) {
                            const float u = fmaf(sb, top[j * WF + W], top[j * WF]);
                            const float t = fmaf(sb, bot[j * WF + W], bot[j * WF]);
                            v[j] = live ? fmaf(sa, t, u) : 0.f;
                        }
                    } else {
                        const float* src = reinterpret_cast<const float*>(pc) + (C::RPW * hf) * W + w;
#pragma unroll
                        for (int j = 0; j < C::RPW; ++j) v[j] = live ? src[j * W] : 0.f;
                    }
#pragma unroll
                    for (int j = 0; j < C::RPW / 2; ++j) tc::split_pair(v[2 * j], v[2 * j + 1], hi[ch][j], lo[ch][j]);
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&bars.empty[slot]);
                }
            }
            // the S2 MMAs of tile c - 1 (both issuers) have completed
            if (ok) ok = __all_sync(0xffffffffu, tc::mbar_wait_bounded(&bars.aEmpty, (c & 1) ^ 1));
            if (!ok) break;
            tc::fence_after_sync();
#pragma unroll
            for (int ch = 0; ch < C::CPC; ++ch) {
                const uint32_t col = tmem + lane_addr + static_cast<uint32_t>((ch * C::CHR + C::RPW * hf) / 2);
                if constexpr (C::RPW == 16) {
                    tc::tmem_st8(col, hi[ch]);
                    tc::tmem_st8(col + H / 2, lo[ch]);
                } else {
                    tc::tmem_st4(col, hi[ch]);
                    tc::tmem_st4(col + H / 2, lo[ch]);
                }
            }
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars.aFull);
        }
        if (!ok && lane == 0) atomicExch(a.watchdog, 20);
    } else if (warp < kMmaWarp) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3, sub = (warp - kConvWarps) >> 2;  // sub-partition, column half
        const int etid = tid - kConvWarps * 32;                   // 0..255
        const int l = q * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        const int m1 = a.m1, m2 = a.m2, S = 2 * m1;

        // E2: D2 of column tile c -> CS operand rows of its planes (this warp: j in [32 sub, 32 sub + 32)).
        // D2[j] = P[j] + (P[64 + j] + Q[j]): x_hi F_hi, then the two correction products.
        auto e2 = [&](int c) -> bool {
            const int i = c / C::CT, ct = c % C::CT;
            bool ok = tc::mbar_wait_bounded(&bars.d2Full, c & 1);
            if (ok && ct == 0) ok = tc::mbar_wait_bounded(&bars.csEmpty, (i & 1) ^ 1);
            if (tc::named_any(kBarEpi, kEpiThreads, !ok)) return false;
            tc::fence_after_sync();
            const int g = l / W, w = l % W;
            const int pit = ct * C::G1 + g;  // plane within the tile
            uint8_t* cs_hi = base;
            uint8_t* cs_lo = cs_hi + C::CSB;
            const uint32_t row_off = static_cast<uint32_t>(w >> 3) * 2048u + static_cast<uint32_t>(pit) * 1024u +
                                     static_cast<uint32_t>(w & 7) * 128u;
            const uint32_t dp = tmem + lane_addr + C::COL_D2P + 32u * sub;
            const uint32_t dq = tmem + lane_addr + C::COL_D2Q + 32u * sub;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float ph[16], pl[16], pq[16];
                tc::tmem_ld_cols_nowait<16>(dp + 16u * half, ph);
                tc::tmem_ld_cols_nowait<16>(dp + kJF + 16u * half, pl);
                tc::tmem_ld_cols_nowait<16>(dq + 16u * half, pq);
                tc::tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 16; ++k) ph[k] += pl[k] + pq[k];
#pragma unroll
                for (int c8 = 0; c8 < 2; ++c8) {
                    uint4 h4, l4;
                    tc::split8(ph + 8 * c8, h4, l4);
                    const uint32_t off = row_off + (static_cast<uint32_t>((sub * 4 + half * 2 + c8) ^ (w & 7)) << 4);
                    *reinterpret_cast<uint4*>(cs_hi + off) = h4;
                    *reinterpret_cast<uint4*>(cs_lo + off) = l4;
                }
            }
            tc::fence_before_sync();
            tc::fence_async_smem();
            tc::named_sync(kBarEpi, kEpiThreads);
            if (etid == 0) {
                tc::mbar_arrive(&bars.d2Empty);
                if (ct == C::CT - 1 || c == NC - 1) tc::mbar_arrive(&bars.csFull);
            }
            return true;
        };

        // E1: D1 of tile i -> corner spectra.  Lane l holds CS row l: plane l / 64, slot
        // group (l / 32) % 2, cos (lanes 0..15) or sin (lanes 16..31) row of slot 16*group + lane%16.
        // Warp set `sub` finishes ky in [sub*QR, sub*QR + QR): the cos lane the first HQ of
        // them, the sin lane the rest, after one exchange of partial sums.  Each TW product is
        // the TW_hi part plus the TW_lo part.
        auto e1 = [&](int i) -> bool {
            constexpr int QR = R2 / 2, HQ = QR / 2;
            const bool ok = tc::mbar_wait_bounded(&bars.d1Full, i & 1);
            if (tc::named_any(kBarEpi, kEpiThreads, !ok)) return false;
            tc::fence_after_sync();
            const uint32_t d1 = tmem + lane_addr + C::COL_D1 + static_cast<uint32_t>(sub * QR);
            float uc[QR], us[QR];
            {
                float t0[QR], t1[QR];
                tc::tmem_ld_cols_nowait<QR>(d1, uc);
                tc::tmem_ld_cols_nowait<QR>(d1 + N1, t0);
                tc::tmem_ld_cols_nowait<QR>(d1 + R2, us);
                tc::tmem_ld_cols_nowait<QR>(d1 + N1 + R2, t1);
                tc::tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < QR; ++k) {
                    uc[k] += t0[k];
                    us[k] += t1[k];
                }
            }
            tc::fence_before_sync();
            const int pit = l >> 6, grp = (l >> 5) & 1, cs = lane >> 4, si = lane & 15;
            const int s = 16 * grp + si;
            const int p = p0 + 2 * i + pit;
            const bool valid = s < S && p < p1;
            float2* dst = nullptr;
            const long long qo = FOLD ? a.qoff[qpar] : 0;
            if (valid)
                dst = (s < m1 ? a.out1 + qo + static_cast<long long>(p) * a.ops + static_cast<long long>(s) * a.ors
                              : a.out2 + qo + static_cast<long long>(p) * a.ops + static_cast<long long>(s - m1) * a.ors);
#pragma unroll
            for (int k = 0; k < HQ; ++k) {
                const float uc0 = uc[k], us0 = us[k];
                const float uc1 = uc[HQ + k], us1 = us[HQ + k];
                const float ra = __shfl_xor_sync(0xffffffffu, cs ? uc0 : uc1, 16);
                const float rb = __shfl_xor_sync(0xffffffffu, cs ? us0 : us1, 16);
                const float Cc = cs ? ra : uc0, Cs = cs ? rb : us0;
                const float Sc = cs ? uc1 : ra, Ss = cs ? us1 : rb;
                const int ky = sub * QR + (cs ? HQ + k : k);
                if (valid && ky < m2) dst[static_cast<long long>(ky) * a.oks] = make_float2(Cc + Ss, Cs - Sc);
            }
            tc::named_sync(kBarEpi, kEpiThreads);
            if (etid == 0) tc::mbar_arrive(&bars.d1Empty);
            return true;
        };

        bool ok = true;
        for (int c = 0; c < NC && ok; ++c) {
            const int i = c / C::CT, ct = c % C::CT;
            ok = e2(c);
            if (ok && ct == 0 && i > 0) ok = e1(i - 1);
        }
        if (ok && NT > 0) ok = e1(NT - 1);
        if (!ok && etid == 0) atomicExch(a.watchdog, 21);
    } else if (warp < kTmaWarp && lane == 0) {
        // ------------------------------------------------------------ MMA issuers
        const int role = warp - kMmaWarp;  // 0 S2P, 1 S2Q, 2 S1
        const uint32_t sb = tc::smem_u32(base);
        bool ok = tc::mbar_wait_bounded(&bars.tab, 0);
        if (role < 2) {
            // S2: column DFT of every column tile, A = x^T from TMEM (hi or lo half)
            const uint64_t dFB = tc::desc_sw128(sb + C::OFF_FB);
            const uint32_t id = role == 0 ? tc::idesc_bf16(128, kFRows) : tc::idesc_bf16(128, kJF);
            const uint32_t d = tmem + (role == 0 ? C::COL_D2P : C::COL_D2Q);
            const uint32_t a0 = tmem + (role == 0 ? 0u : static_cast<uint32_t>(H / 2));
            for (int c = 0; c < NC && ok; ++c) {
                ok = tc::mbar_wait_bounded(&bars.d2Empty, (c & 1) ^ 1) && tc::mbar_wait_bounded(&bars.aFull, c & 1);
                if (!ok) break;
                tc::fence_after_sync();
#pragma unroll
                for (int ks = 0; ks < H / 16; ++ks) {
                    const uint32_t bo = (static_cast<uint32_t>(ks >> 2) * kFRows * 128u + (ks & 3) * 32u) >> 4;
                    tc::mma_ts(d, a0 + 8u * ks, dFB + bo, id, ks > 0 ? 1u : 0u);
                }
                tc::mma_commit(&bars.aEmpty);
                tc::mma_commit(&bars.d2Full);
            }
        } else {
            // S1: row DFT of every 2-plane tile, A = CS hi / lo from shared memory
            const uint64_t dTW = tc::desc_sw128(sb + C::OFF_TW);
            const uint64_t dCShi = tc::desc_mn_sw128(sb, 1024u, 2048u);
            const uint64_t dCSlo = tc::desc_mn_sw128(sb + C::CSB, 1024u, 2048u);
            constexpr uint32_t idC = tc::idesc_bf16(128, 2 * N1) | tc::kIdescAMajorMN;
            constexpr uint32_t idD = tc::idesc_bf16(128, N1) | tc::kIdescAMajorMN;
            const uint32_t d = tmem + C::COL_D1;
            for (int i = 0; i < NT && ok; ++i) {
                ok = tc::mbar_wait_bounded(&bars.csFull, i & 1) && tc::mbar_wait_bounded(&bars.d1Empty, (i & 1) ^ 1);
                if (!ok) break;
                tc::fence_after_sync();
#pragma unroll
                for (int ks = 0; ks < W / 16; ++ks) {
                    const uint32_t ao = (static_cast<uint32_t>(ks) * 4096u) >> 4;
                    const uint32_t bo = (static_cast<uint32_t>(ks >> 2) * (2u * N1) * 128u + (ks & 3) * 32u) >> 4;
                    tc::mma_bf16(d, dCShi + ao, dTW + bo, idC, ks > 0 ? 1u : 0u);
                    tc::mma_bf16(d, dCSlo + ao, dTW + bo, idD, 1u);
                }
                tc::mma_commit(&bars.csEmpty);
                tc::mma_commit(&bars.d1Full);
            }
        }
        if (!ok) atomicExch(a.watchdog, 22);
        // every MMA this thread issued has completed before TMEM is released
        tc::mma_commit(&bars.drain[role]);
        tc::mbar_wait_bounded(&bars.drain[role], 0);
    } else if (warp == kTmaWarp && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        for (int k = k_first; k < NK; ++k) {
            const int slot = k % C::NS, use = k / C::NS;
            if (!tc::mbar_wait_bounded(&bars.empty[slot], (use & 1) ^ 1)) {
                atomicExch(a.watchdog, 23);
                break;
            }
            issue_chunk(k);
            prefetch_chunk(k + PF);
        }
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

struct FwdTable {
    const uint4* data;
    uint32_t bytes;
};

std::mutex g_mutex;
std::map<std::tuple<int, int, int, int, int, int>, FwdTable> g_tables;

// [F_hi; F_lo] (kFRows x H) followed by [TW_hi; TW_lo] (2*N1 x W), K-major SW128 bf16.  With a
// sub-problem description the rows hold the modes of that parity of the folded plane
// (spectrum row kx, column ky of the full Hp x Wp plane; see TcSub).
cudaError_t get_fwd_table(int H, int W, int m1, int m2, const TcSub* sub, const FwdTable** out) {
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
    const int R2 = host::round_up(m2, 8), N1 = 2 * R2, S = 2 * m1;
    host::KMajor fb(kFRows, H);
    for (int j = 0; j < kJF; ++j) {
        const int grp = j / 32, cs = (j / 16) & 1, s = 16 * grp + (j & 15);
        if (s >= S) continue;
        const int kx = sub ? sub_row(*sub, s, m1) : host::slot_row(s, H, m1);
        const int Hp = sub ? sub->period_h : H;
        for (int h = 0; h < H; ++h) {
            const double t = host::ang(kx, h, Hp);
            uint16_t hi, lo;
            host::bf16_split(cs ? std::sin(t) : std::cos(t), hi, lo);
            fb.set(j, h, hi);
            fb.set(kJF + j, h, lo);
        }
    }
    host::KMajor tw(2 * N1, W);
    for (int n = 0; n < m2; ++n)
        for (int w = 0; w < W; ++w) {
            const double t = sub ? host::ang(2 * n + sub->b, w, sub->period_w) : host::ang(n, w, W);
            uint16_t hi, lo;
            host::bf16_split(std::cos(t), hi, lo);
            tw.set(n, w, hi);
            tw.set(N1 + n, w, lo);
            host::bf16_split(-std::sin(t), hi, lo);
            tw.set(R2 + n, w, hi);
            tw.set(N1 + R2 + n, w, lo);
        }
    std::vector<uint16_t> host_buf(fb.data);
    host_buf.insert(host_buf.end(), tw.data.begin(), tw.data.end());
    const size_t bytes = host_buf.size() * 2;
    void* d = nullptr;
    err = cudaMalloc(&d, bytes);
    if (err != cudaSuccess) return err;
    err = cudaMemcpy(d, host_buf.data(), bytes, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        cudaFree(d);
        return err;
    }
    FwdTable t;
    t.data = static_cast<const uint4*>(d);
    t.bytes = static_cast<uint32_t>(bytes);
    auto res = g_tables.emplace(key, t);
    *out = &res.first->second;
    return cudaSuccess;
}

template <int H, int W, int R2, bool FOLD>
cudaError_t run_fwd(const FwdArgs& a, cudaStream_t stream) {
    using C = FwdCfg<H, W, R2, FOLD>;
    static_assert(C::SMEM <= 227u * 1024u - 512u, "shared memory budget");
    if (a.tab_bytes != C::FB_BYTES + C::TW_BYTES) return cudaErrorInvalidValue;
    auto kernel = dft_fwd_tc_kernel<H, W, R2, FOLD>;
    int per_sm = 1;
    cudaError_t err = prepare_kernel(reinterpret_cast<const void*>(kernel), C::SMEM, kThreads, &per_sm);
    if (err != cudaSuccess) return err;
    int grid;
    if (FOLD) {
        // groups of four CTAs (one per parity), as many groups as fit one per SM, at most one
        // plane-column tile each
        const int groups = std::max(1, std::min(num_sms() / 4, (a.P + C::G1 - 1) / C::G1));
        grid = 4 * groups;
    } else {
        // Every CTA gets the same number of planes, ceil(P / SMs): 640 planes run as 128 CTAs of 5
        // rather than 148 CTAs of 4 or 5.  The busiest CTA streams as many planes either way, but
        // with all ranges equal no CTA finishes its last plane alone after the others (15.7 ->
        // 14.8 us at B20 C32 128x128).
        const int per_cta = (a.P + num_sms() - 1) / num_sms();
        grid = std::max(1, (a.P + per_cta - 1) / per_cta);
    }
    return launch_chained(kernel, dim3(grid), dim3(kThreads), C::SMEM, stream, a);
}

template <int H, int W, bool FOLD>
cudaError_t run_fwd_r2(const FwdArgs& a, int R2, cudaStream_t stream) {
    switch (R2) {
        case 8: return run_fwd<H, W, 8, FOLD>(a, stream);
        case 16: return run_fwd<H, W, 16, FOLD>(a, stream);
        case 24: return run_fwd<H, W, 24, FOLD>(a, stream);
        case 32: return run_fwd<H, W, 32, FOLD>(a, stream);
        default: return cudaErrorInvalidValue;
    }
}

template <bool FOLD>
cudaError_t run_fwd_shape(const FwdArgs& a, int H, int W, int R2, cudaStream_t stream) {
    if (H == 64 && W == 64) return run_fwd_r2<64, 64, FOLD>(a, R2, stream);
    if (H == 64 && W == 128) return run_fwd_r2<64, 128, FOLD>(a, R2, stream);
    if (H == 128 && W == 64) return run_fwd_r2<128, 64, FOLD>(a, R2, stream);
    return run_fwd_r2<128, 128, FOLD>(a, R2, stream);
}

}  // namespace

bool tc_fwd_supported(int H, int W, int m1, int m2) {
    return (H == 64 || H == 128) && (W == 64 || W == 128) && m1 >= 1 && 2 * m1 <= 32 && m2 >= 1 && m2 <= 32 &&
           m1 <= H && m2 <= W / 2 + 1;
}

cudaError_t launch_dft_fwd_tc(const float* x, float2* out1, float2* out2, long long ops, int ors, int P, int H,
                              int W, int m1, int m2, cudaStream_t stream, const TcSub* sub) {
    if (!tc_fwd_supported(H, W, m1, m2) || P <= 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
        return cudaErrorInvalidValue;
    const FwdTable* t = nullptr;
    cudaError_t e = get_fwd_table(H, W, m1, m2, sub, &t);
    if (e != cudaSuccess) return e;
    int* wd = nullptr;
    e = device_watchdog(&wd);
    if (e != cudaSuccess) return e;
    FwdArgs a = {};
    a.x = x;
    a.out1 = out1;
    a.out2 = out2;
    a.ops = ops;
    a.ors = ors;
    a.oks = sub ? 2 : 1;
    a.P = P;
    a.m1 = m1;
    a.m2 = m2;
    a.tab = t->data;
    a.tab_bytes = t->bytes;
    a.watchdog = wd;
    return run_fwd_shape<false>(a, H, W, host::round_up(m2, 8), stream);
}

cudaError_t launch_dft_fwd_tc_folded(const float* x, float2* out1, float2* out2, long long ops, int ors, int P,
                                     int Hf, int Wf, int m1f, int m2f, cudaStream_t stream) {
    if (!tc_split_supported(Hf, Wf, m1f, m2f) || P <= 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
        return cudaErrorInvalidValue;
    const int H = Hf / 2, W = Wf / 2, m1 = m1f / 2, m2 = m2f / 2;
    FwdArgs a = {};
    for (int q = 0; q < 4; ++q) {
        const TcSub sub{Hf, Wf, q >> 1, q & 1, m1f, m2f};
        const FwdTable* t = nullptr;
        cudaError_t e = get_fwd_table(H, W, m1, m2, &sub, &t);
        if (e != cudaSuccess) return e;
        a.tabq[q] = t->data;
        a.tab_bytes = t->bytes;
        a.qoff[q] = static_cast<long long>(sub.a) * ors + sub.b;
    }
    cudaError_t e = device_watchdog(&a.watchdog);
    if (e != cudaSuccess) return e;
    a.x = x;
    a.out1 = out1;
    a.out2 = out2;
    a.ops = ops;
    a.ors = 2 * ors;
    a.oks = 2;
    a.P = P;
    a.m1 = m1;
    a.m2 = m2;
    a.tab = a.tabq[0];
    return run_fwd_shape<true>(a, H, W, host::round_up(m2, 8), stream);
}

}  // namespace scx
