// Dual-corner complex mode mixing: the B200 replacement for spectral_mul_kernel and
// spectral_mul_dual_packed_kernel (spectral_conv_combo/spectral_conv_ext.su:5-92).
//
//   y_c[b][o][k] = sum_i x_c[b][i][k] * w_c[i][o][k]      c in {1, 2}, k over m1*m2 modes
//
// mix_ring_kernel (mode counts that are even, 16-byte aligned operands, at least 8 input
// channels): one CTA owns one corner, a tile of 16 consecutive modes (128-byte rows), a
// block of batch items and a block of output channels.  Input channels stream in chunks of
// 8 through a ring of 3-D TMA loads (x_c[b-block, chunk, tile] and w_c[chunk, o-block,
// tile]) consumed by KS groups of warps in turn (split K, for enough warps per SM at small
// sizes); each thread keeps a BT x OT block of complex accumulators for one mode, and the
// stores of a half-warp cover one 128-byte line of y.  mix_smem_kernel is the same contraction with
// per-thread loads, for the shapes the TMA boxes cannot describe.  Both corners run in one
// launch on the caller's stream (the reference launched them serially on the null stream).
#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>

#include <cuda.h>

#include "scx_internal.h"
#include "scx_tc.cuh"

namespace scx {
namespace {

constexpr int kThreads = 256;
constexpr int kOT = 2;  // output channels per thread
constexpr int kBT = 4;  // batch items per thread

struct MixArgs {
    const float2* x[2];
    const float2* w[2];
    float2* y[2];
    int B, Cin, Cout, NM, TM;
};

__global__ void __launch_bounds__(kThreads) mix_smem_kernel(const MixArgs a) {
    extern __shared__ float2 mix_smem[];
    const int corner = blockIdx.y;
    const int TM = a.TM;
    const int k0 = blockIdx.x * TM;
    const int tm = min(TM, a.NM - k0);
    const int B = a.B, Cin = a.Cin, Cout = a.Cout, NM = a.NM;
    float2* Xs = mix_smem;                                  // [B][Cin][TM]
    float2* Ws = mix_smem + static_cast<size_t>(B) * Cin * TM;  // [Cin][Cout][TM]
    const float2* __restrict__ X = a.x[corner];
    const float2* __restrict__ Wt = a.w[corner];
    float2* __restrict__ Y = a.y[corner];

    // staged in batches of 8 loads per thread before their stores, so that a batch is in flight
    // at once (a load-store loop waits a full memory latency per element)
    constexpr int LB = 8;
    auto stage = [&](const float2* __restrict__ src, float2* dst, int nrow) {
        const int n = nrow * tm;
        for (int i0 = threadIdx.x; i0 < n; i0 += kThreads * LB) {
            float2 v[LB];
#pragma unroll
            for (int u = 0; u < LB; ++u) {
                const int i = i0 + u * kThreads;
                if (i < n) {
                    const int row = i / tm, kk = i - row * tm;
                    v[u] = __ldg(src + static_cast<size_t>(row) * NM + k0 + kk);
                }
            }
#pragma unroll
            for (int u = 0; u < LB; ++u) {
                const int i = i0 + u * kThreads;
                if (i < n) {
                    const int row = i / tm, kk = i - row * tm;
                    dst[row * TM + kk] = v[u];
                }
            }
        }
    };
    stage(X, Xs, B * Cin);
    stage(Wt, Ws, Cin * Cout);
    __syncthreads();

    const int nog = (Cout + kOT - 1) / kOT;
    const int nbg = (B + kBT - 1) / kBT;
    const int ntiles = tm * nog * nbg;
    for (int t = threadIdx.x; t < ntiles; t += kThreads) {
        const int kk = t % tm;
        const int rest = t / tm;
        const int og = rest % nog, bg = rest / nog;
        const int o0 = og * kOT, b0 = bg * kBT;
        float2 acc[kOT][kBT];
#pragma unroll
        for (int p = 0; p < kOT; ++p)
#pragma unroll
            for (int q = 0; q < kBT; ++q) acc[p][q] = make_float2(0.f, 0.f);
        for (int i = 0; i < Cin; ++i) {
            float2 wv[kOT], xv[kBT];
#pragma unroll
            for (int p = 0; p < kOT; ++p)
                wv[p] = (o0 + p < Cout) ? Ws[(i * Cout + o0 + p) * TM + kk] : make_float2(0.f, 0.f);
#pragma unroll
            for (int q = 0; q < kBT; ++q)
                xv[q] = (b0 + q < B) ? Xs[((b0 + q) * Cin + i) * TM + kk] : make_float2(0.f, 0.f);
#pragma unroll
            for (int p = 0; p < kOT; ++p)
#pragma unroll
                for (int q = 0; q < kBT; ++q) {
                    acc[p][q].x = fmaf(xv[q].x, wv[p].x, fmaf(-xv[q].y, wv[p].y, acc[p][q].x));
                    acc[p][q].y = fmaf(xv[q].x, wv[p].y, fmaf(xv[q].y, wv[p].x, acc[p][q].y));
                }
        }
#pragma unroll
        for (int p = 0; p < kOT; ++p)
#pragma unroll
            for (int q = 0; q < kBT; ++q)
                if (o0 + p < Cout && b0 + q < B)
                    Y[(static_cast<size_t>(b0 + q) * Cout + o0 + p) * NM + k0 + kk] = acc[p][q];
    }
}


constexpr int kRingTM = 16;        // modes per tile: every staged row is one 128-byte line
constexpr int kRingIC = 8;         // input channels per ring chunk
constexpr int kRingMaxStages = 4;

struct MixRingArgs {
    float2* y[2];
    int B, Cin, Cout, NM;
    int NCH, NS, n_os;  // channel chunks, ring stages, output-channel blocks
    uint32_t stage_bytes;
    int* watchdog;
    int m2, W;          // CJ = 2: the per-mode output scale c_ky * inv_hw (ky = mode % m2)
    float inv_hw;
    int w_early;        // w is not written by the kernels this one is chained after: the first
                        // stages' w boxes are requested before griddepcontrol.wait
};

// x_c viewed as [B][Cin][2*NM] floats, w_c as [Cin][Cout][2*NM].  Chunk c of the ring holds
// x_c[b-block, 8c.., tile] as [BB][8][16] float2 and w_c[8c.., o-block, tile] as [8][OC][16]
// float2 (TMA boxes (32, 8, BB) and (32, OC, 8), zero-filled past the tensor edges, so a
// partial tile, batch block or channel chunk contributes nothing).  The CTA's KS groups of
// warps take every KS-th chunk (the ring depth is a multiple of KS, so a group refills its
// own slots); within a group, thread (g, mode k) keeps BT batch items x OT output channels,
// and the two half-warps share their batch items, so an x read is one broadcast line.  The
// groups' partial sums are added in group order at the end.
// CJ selects what the staged operands mean (the boxes are the same; the tensor maps decide which
// stored tensor and order they come from): 0 = x and w as stored; 1 = w is the conjugate of the
// staged values (the backward's W^H, read through a transposed map); 2 = x is the conjugate of
// the staged values (X^H) and the result is scaled per mode by c_ky * inv_hw (c_ky = 1 for
// ky = 0 and, W even, ky = W/2, else 2).
template <int BT, int OT, int NBQ, int NOQ, int KS, int CJ>
__global__ void __launch_bounds__(16 * NBQ * NOQ * KS) mix_ring_kernel(const __grid_constant__ CUtensorMap tx0,
                                                                       const __grid_constant__ CUtensorMap tx1,
                                                                       const __grid_constant__ CUtensorMap tw0,
                                                                       const __grid_constant__ CUtensorMap tw1,
                                                                       const MixRingArgs a) {
    constexpr int BB = BT * NBQ, OC = OT * NOQ, IC = kRingIC, GT = 16 * NBQ * NOQ;
    constexpr uint32_t XB = static_cast<uint32_t>(BB) * IC * kRingTM * 8u;
    extern __shared__ uint8_t mix_raw[];
    __shared__ uint64_t full[kRingMaxStages];
    __shared__ int failed;
    uint8_t* base = tc::align1024(mix_raw);
    const int corner = blockIdx.y;
    const int k0 = blockIdx.x * kRingTM;
    const int o_base = (blockIdx.z % a.n_os) * OC, b_base = (blockIdx.z / a.n_os) * BB;
    const CUtensorMap* mx = corner ? &tx1 : &tx0;
    const CUtensorMap* mw = corner ? &tw1 : &tw0;
    const int NS = a.NS, NCH = a.NCH;
    auto issue_x = [&](int c) {
        tc::tma_load_3d(base + static_cast<uint32_t>(c % NS) * a.stage_bytes, mx, 2 * k0, c * IC, b_base, &full[c % NS]);
    };
    auto issue_w = [&](int c) {
        uint64_t* bar = &full[c % NS];
        tc::mbar_arrive_expect_tx(bar, a.stage_bytes);
        tc::tma_load_3d(base + static_cast<uint32_t>(c % NS) * a.stage_bytes + XB, mw, 2 * k0, o_base, c * IC, bar);
    };
    auto issue = [&](int c) {
        issue_w(c);
        issue_x(c);
    };
    if (threadIdx.x == 0) {
        tc::grid_dep_launch();  // the next kernel's CTAs may start their prologue
        for (int i = 0; i < kRingMaxStages; ++i) tc::mbar_init(&full[i], 1);
        tc::fence_async_smem();
        const int first = min(NS, NCH);
        if (a.w_early) {
            // the weights do not depend on the previous kernel: their boxes overlap its tail
            for (int c = 0; c < first; ++c) issue_w(c);
            tc::grid_dep_wait();  // x comes from the previous kernel in the stream
            for (int c = 0; c < first; ++c) issue_x(c);
        } else {
            tc::grid_dep_wait();  // x (and w) may come from the previous kernel in the stream
            for (int c = 0; c < first; ++c) issue(c);
        }
        failed = 0;
    }
    __syncthreads();

    const int kg = threadIdx.x / GT, gt = threadIdx.x % GT;
    const int k = gt & (kRingTM - 1), g = gt >> 4;
    const int oq = g % NOQ, bq = g / NOQ;
    float2 acc[BT][OT];
#pragma unroll
    for (int q = 0; q < BT; ++q)
#pragma unroll
        for (int p = 0; p < OT; ++p) acc[q][p] = make_float2(0.f, 0.f);
    for (int c = kg; c < NCH; c += KS) {
        const int slot = c % NS;
        const bool ok = tc::mbar_wait_bounded(&full[slot], (c / NS) & 1);
        if (tc::named_any(1 + kg, GT, !ok)) {
            if (gt == 0) failed = 1;
            break;
        }
        const float2* xp = reinterpret_cast<const float2*>(base + static_cast<uint32_t>(slot) * a.stage_bytes) +
                           bq * BT * IC * kRingTM + k;
        const float2* wp = reinterpret_cast<const float2*>(base + static_cast<uint32_t>(slot) * a.stage_bytes + XB) +
                           oq * OT * kRingTM + k;
#pragma unroll
        for (int i = 0; i < IC; ++i) {
            float2 xv[BT], wv[OT];
#pragma unroll
            for (int q = 0; q < BT; ++q) {
                xv[q] = xp[(q * IC + i) * kRingTM];
                if (CJ == 2) xv[q].y = -xv[q].y;
            }
#pragma unroll
            for (int p = 0; p < OT; ++p) {
                wv[p] = wp[(i * OC + p) * kRingTM];
                if (CJ == 1) wv[p].y = -wv[p].y;
            }
#pragma unroll
            for (int q = 0; q < BT; ++q)
#pragma unroll
                for (int p = 0; p < OT; ++p) {
                    acc[q][p].x = fmaf(xv[q].x, wv[p].x, fmaf(-xv[q].y, wv[p].y, acc[q][p].x));
                    acc[q][p].y = fmaf(xv[q].x, wv[p].y, fmaf(xv[q].y, wv[p].x, acc[q][p].y));
                }
        }
        tc::named_sync(1 + kg, GT);  // the group is done with the slot before it is refilled
        if (gt == 0 && c + NS < NCH) issue(c + NS);
    }
    __syncthreads();  // every chunk has been consumed: no copy is in flight
    if (failed) {
        if (threadIdx.x == 0) atomicExch(a.watchdog, 40);
        return;
    }
    if (KS > 1) {
        // partial sums of groups 1.. through shared memory, [group][element][thread]
        float2* red = reinterpret_cast<float2*>(base);
        if (kg > 0) {
#pragma unroll
            for (int q = 0; q < BT; ++q)
#pragma unroll
                for (int p = 0; p < OT; ++p) red[((kg - 1) * BT * OT + q * OT + p) * GT + gt] = acc[q][p];
        }
        __syncthreads();
        if (kg > 0) return;
        for (int j = 1; j < KS; ++j)
#pragma unroll
            for (int q = 0; q < BT; ++q)
#pragma unroll
                for (int p = 0; p < OT; ++p) {
                    const float2 v = red[((j - 1) * BT * OT + q * OT + p) * GT + gt];
                    acc[q][p].x += v.x;
                    acc[q][p].y += v.y;
                }
    }
    const int kk = k0 + k;
    if (kk >= a.NM) return;
    if (CJ == 2 && a.W > 0) {
        const int ky = kk % a.m2;
        const float f = (ky == 0 || ((a.W % 2) == 0 && 2 * ky == a.W)) ? a.inv_hw : 2.0f * a.inv_hw;
#pragma unroll
        for (int q = 0; q < BT; ++q)
#pragma unroll
            for (int p = 0; p < OT; ++p) {
                acc[q][p].x *= f;
                acc[q][p].y *= f;
            }
    }
    float2* __restrict__ Y = corner ? a.y[1] : a.y[0];
#pragma unroll
    for (int q = 0; q < BT; ++q)
#pragma unroll
        for (int p = 0; p < OT; ++p) {
            const int b = b_base + bq * BT + q, o = o_base + oq * OT + p;
            if (b < a.B && o < a.Cout) Y[(static_cast<size_t>(b) * a.Cout + o) * a.NM + kk] = acc[q][p];
        }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
EncodeTiledFn encode_tiled() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 3-D fp32 tensor with dims (d0 innermost, d1, d2) and byte strides s1, s2 of dims 1 and 2 (in
// either order: a transposed view of a stored tensor), box (b0, b1, b2).
bool encode3d(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0, uint32_t b1,
              uint32_t b2, uint64_t s1 = 0, uint64_t s2 = 0) {
    EncodeTiledFn fn = encode_tiled();
    if (fn == nullptr) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {s1 ? s1 : d0 * 4, s2 ? s2 : d0 * d1 * 4};
    const cuuint32_t box[3] = {b0, b1, b2};
    const cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct RingCfg {
    int BT, OT, NBQ, NOQ, KS;
};

// the last shape takes one batch item per CTA (B = 1: a matrix-vector product per mode)
const RingCfg kRingCands[] = {{5, 2, 4, 4, 2}, {5, 2, 4, 2, 4}, {4, 4, 4, 4, 2}, {4, 4, 4, 2, 4},
                              {4, 2, 4, 4, 2}, {2, 2, 4, 4, 2}, {1, 2, 2, 4, 2}, {1, 2, 1, 8, 2}};
constexpr int kNumRingCands = static_cast<int>(sizeof(kRingCands) / sizeof(kRingCands[0]));

template <int CJ>
const void* ring_kernel_cj(int ci) {
    switch (ci) {
        case 0: return reinterpret_cast<const void*>(mix_ring_kernel<5, 2, 4, 4, 2, CJ>);
        case 1: return reinterpret_cast<const void*>(mix_ring_kernel<5, 2, 4, 2, 4, CJ>);
        case 2: return reinterpret_cast<const void*>(mix_ring_kernel<4, 4, 4, 4, 2, CJ>);
        case 3: return reinterpret_cast<const void*>(mix_ring_kernel<4, 4, 4, 2, 4, CJ>);
        case 4: return reinterpret_cast<const void*>(mix_ring_kernel<4, 2, 4, 4, 2, CJ>);
        case 5: return reinterpret_cast<const void*>(mix_ring_kernel<2, 2, 4, 4, 2, CJ>);
        case 6: return reinterpret_cast<const void*>(mix_ring_kernel<1, 2, 2, 4, 2, CJ>);
        default: return reinterpret_cast<const void*>(mix_ring_kernel<1, 2, 1, 8, 2, CJ>);
    }
}

const void* ring_kernel(int ci, int cj = 0) {
    return cj == 1 ? ring_kernel_cj<1>(ci) : cj == 2 ? ring_kernel_cj<2>(ci) : ring_kernel_cj<0>(ci);
}

struct RingChoice {
    int ci, ns;
    size_t smem;
};

// The ring shape with the least modelled time: FMA work (padding included) at a rate that
// saturates at 16 resident warps per SM, or the staging traffic from L2 at 64 B per SM cycle,
// whichever is larger, plus a load latency per CTA wave.  `only` >= 0 restricts the choice to
// that shape (a measured variant).  ci < 0 when no shape fits.
cudaError_t choose_ring(int ncorner, int B, int Cin, int Cout, int NM, int only, RingChoice* out) {
    const int NMT = (NM + kRingTM - 1) / kRingTM;
    const int sms = num_sms();
    const int nch = (Cin + kRingIC - 1) / kRingIC;
    const double x_total = static_cast<double>(ncorner) * B * Cin * NM * 8.0;
    const double w_total = static_cast<double>(ncorner) * Cin * Cout * NM * 8.0;
    *out = RingChoice{-1, 0, 0};
    double best_t = 0;
    for (int ci = 0; ci < kNumRingCands; ++ci) {
        if (only >= 0 && ci != only) continue;
        const RingCfg& c = kRingCands[ci];
        const int BB = c.BT * c.NBQ, OC = c.OT * c.NOQ, threads = 16 * c.NBQ * c.NOQ * c.KS;
        if (BB > B || OC > Cout) continue;  // TMA boxes stay inside the tensors
        const long long stage = static_cast<long long>(BB + OC) * kRingIC * kRingTM * 8;
        // ring depth: a multiple of KS, at most 4, every chunk in flight if they fit; a group
        // that takes more than one chunk needs two slots, or each refill waits for its load
        const int ns = std::min(kRingMaxStages, (nch + c.KS - 1) / c.KS * c.KS);
        if (ns < std::min(nch, 2 * c.KS)) continue;
        const long long red = static_cast<long long>(c.KS - 1) * c.BT * c.OT * (threads / c.KS) * 8;
        const size_t smem = static_cast<size_t>(std::max(ns * stage, red) + 1024);
        if (smem > 200 * 1024) continue;
        int per_sm = 1;
        cudaError_t err = prepare_kernel(ring_kernel(ci), smem, threads, &per_sm);
        if (err != cudaSuccess) return err;
        if (per_sm < 1) continue;
        const long long nbs = (B + BB - 1) / BB, nos = (Cout + OC - 1) / OC;
        const long long ctas = static_cast<long long>(ncorner) * NMT * nbs * nos;
        const double resident = std::min<double>(static_cast<double>(ctas) / sms, static_cast<double>(per_sm));
        const double warps = resident * threads / 32.0;
        const double cmacs = static_cast<double>(ncorner) * NMT * kRingTM * nbs * BB * nos * OC * Cin;
        const double fma = 4.0 * cmacs / (sms * 128.0 * std::min(1.0, warps / 16.0));
        const double l2 = (x_total * nos + w_total * nbs) / (sms * 64.0);
        const double waves = std::ceil(static_cast<double>(ctas) / (static_cast<double>(sms) * per_sm));
        const double t = std::max(fma, l2) + 2000.0 * waves;
        if (out->ci < 0 || t < best_t) {
            *out = RingChoice{ci, ns, smem};
            best_t = t;
        }
    }
    return cudaSuccess;
}

// mix_smem_kernel stages one mode's x and w rows (at least) in shared memory.
bool smem_kernel_fits(int B, int Cin, int Cout) {
    return (static_cast<size_t>(B) * Cin + static_cast<size_t>(Cin) * Cout) * sizeof(float2) <= 200 * 1024;
}

// The TMA ring launch; returns cudaErrorNotSupported when the shape or alignment does not fit
// its boxes (the caller then uses mix_smem_kernel).
cudaError_t launch_mix_ring(const float2* x1, const float2* x2, const float2* w1, const float2* w2, float2* y1,
                            float2* y2, int ncorner, int B, int Cin, int Cout, int NM, cudaStream_t stream,
                            int cj = 0, int m2 = 1, int Wd = 1, float inv_hw = 1.f, bool w_early = false) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(x1) | reinterpret_cast<uintptr_t>(w1) |
                         (ncorner == 2 ? (reinterpret_cast<uintptr_t>(x2) | reinterpret_cast<uintptr_t>(w2)) : 0);
    if (NM % 2 != 0 || (al & 15) != 0 || Cin < kRingIC) return cudaErrorNotSupported;
    const int forced = cj == 0 ? mix_variant(ncorner, B, Cin, Cout, NM) : kMixAuto;
    // measured: the per-thread kernel wins (when one mode's operands fit its shared memory)
    if (forced == kMixSmem && smem_kernel_fits(B, Cin, Cout)) return cudaErrorNotSupported;
    // Tile shapes: the measured one when the variant table names one that fits, else the one
    // with the least modelled time; chosen once per shape, variant and device.
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex m;
    static std::map<std::tuple<int, int, int, int, int, int, int>, RingChoice> chosen;
    RingChoice ch{-1, 0, 0};
    const int nch = (Cin + kRingIC - 1) / kRingIC;
    {
        std::lock_guard<std::mutex> lock(m);
        const auto key = std::make_tuple(dev, ncorner, B, Cin, Cout, NM, forced);
        auto it = chosen.find(key);
        if (it != chosen.end()) {
            ch = it->second;
        } else {
            if (forced >= 0) {
                e = choose_ring(ncorner, B, Cin, Cout, NM, forced, &ch);
                if (e != cudaSuccess) return e;
            }
            if (ch.ci < 0) {
                e = choose_ring(ncorner, B, Cin, Cout, NM, -1, &ch);
                if (e != cudaSuccess) return e;
            }
            chosen.emplace(key, ch);
        }
    }
    if (ch.ci < 0) return cudaErrorNotSupported;
    const int best = ch.ci, best_ns = ch.ns;
    const size_t best_smem = ch.smem;
    const RingCfg& cfg = kRingCands[best];
    const int BB = cfg.BT * cfg.NBQ, OC = cfg.OT * cfg.NOQ;
    MixRingArgs a;
    a.y[0] = y1;
    a.y[1] = y2;
    a.B = B;
    a.Cin = Cin;
    a.Cout = Cout;
    a.NM = NM;
    a.NCH = nch;
    a.NS = best_ns;
    a.n_os = (Cout + OC - 1) / OC;
    a.stage_bytes = static_cast<uint32_t>(BB + OC) * kRingIC * kRingTM * 8u;
    a.m2 = m2;
    a.W = Wd;
    a.inv_hw = inv_hw;
    a.w_early = w_early ? 1 : 0;
    const int n_bs = (B + BB - 1) / BB;
    const int threads = 16 * cfg.NBQ * cfg.NOQ * cfg.KS;
    e = device_watchdog(&a.watchdog);
    if (e != cudaSuccess) return e;
    CUtensorMap tx[2], tw[2];
    const float2* xs[2] = {x1, x2};
    const float2* ws[2] = {w1, w2};
    const uint64_t row = 2ull * NM * 4ull;  // bytes between consecutive channels of one mode row
    for (int c = 0; c < 2; ++c) {
        const int src = c < ncorner ? c : 0;  // an unused second corner repeats the first map
        // cj = 2: x is stored [Cin][B] per mode (read transposed); cj = 1: w is stored [Cout][Cin]
        const bool xt = cj == 2, wt = cj == 1;
        if (!encode3d(&tx[c], xs[src], 2ull * NM, Cin, B, 2u * kRingTM, kRingIC, BB, xt ? row * B : 0, xt ? row : 0) ||
            !encode3d(&tw[c], ws[src], 2ull * NM, Cout, Cin, 2u * kRingTM, OC, kRingIC, wt ? row * Cin : 0,
                      wt ? row : 0))
            return cudaErrorNotSupported;
    }
    const dim3 grid(static_cast<unsigned>((NM + kRingTM - 1) / kRingTM), ncorner, a.n_os * n_bs);
    void* args[] = {&tx[0], &tx[1], &tw[0], &tw[1], &a};
    const void* kernel = ring_kernel(best, cj);
    if (cj != 0) {
        int per_sm = 1;
        e = prepare_kernel(kernel, best_smem, threads, &per_sm);
        if (e != cudaSuccess) return e;
    }
    return launch_chained_raw(kernel, grid, dim3(threads), best_smem, stream, args);
}

}  // namespace

cudaError_t launch_mix_ring_ct(const float2* x1, const float2* x2, const float2* w1, const float2* w2, float2* y1,
                               float2* y2, int ncorner, int B, int Cin, int Cout, int NM, int mode, int m2, int W,
                               float inv_hw, cudaStream_t stream) {
    if (mode < 1 || mode > 2) return cudaErrorInvalidValue;
    // mode 1 reads the weights (never written in the chain); mode 2 reads G, which the chain writes
    return launch_mix_ring(x1, x2, w1, w2, y1, y2, ncorner, B, Cin, Cout, NM, stream, mode, m2, W, inv_hw, mode == 1);
}

cudaError_t launch_mix(const float2* x1, const float2* x2, const float2* w1, const float2* w2,
                       float2* y1, float2* y2, int ncorner, int B, int Cin, int Cout, int NM,
                       cudaStream_t stream, bool w_early) {
    // The tensor-core kernel only where the variant table names it: with B <= 16 each weight
    // element feeds 2B real products, and its conversion into tf32 operands costs more than the
    // FFMA work it replaces (B16 C64 m32: 61 us against 45 us for the TMA-ring kernel).
    const int forced = mix_variant(ncorner, B, Cin, Cout, NM);
    if (forced == kMixTc) {
        const cudaError_t ce = launch_mix_tc(x1, x2, w1, w2, y1, y2, ncorner, B, Cin, Cout, NM, stream);
        if (ce != cudaErrorNotSupported) return ce;
    }
    const cudaError_t te = launch_mix_ring(x1, x2, w1, w2, y1, y2, ncorner, B, Cin, Cout, NM, stream, 0, 1, 1, 1.f,
                                           w_early);
    if (te != cudaErrorNotSupported) return te;
    MixArgs a;
    a.x[0] = x1;
    a.x[1] = x2;
    a.w[0] = w1;
    a.w[1] = w2;
    a.y[0] = y1;
    a.y[1] = y2;
    a.B = B;
    a.Cin = Cin;
    a.Cout = Cout;
    a.NM = NM;
    // Largest mode tile (4, 2 or 1) whose staging fits 96 KB and still gives >= 2 CTAs per SM.
    const size_t per_mode = (static_cast<size_t>(B) * Cin + static_cast<size_t>(Cin) * Cout) * sizeof(float2);
    const long long want = 2LL * num_sms();
    int TM = 1;
    for (int t : {4, 2}) {
        const long long ctas = static_cast<long long>(ncorner) * ((NM + t - 1) / t);
        if (per_mode * t <= 96 * 1024 && ctas >= want) {
            TM = t;
            break;
        }
    }
    const size_t smem = per_mode * TM;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;  // B*Cin + Cin*Cout too large for one mode
    a.TM = TM;
    int per_sm = 1;
    cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(mix_smem_kernel), smem, kThreads, &per_sm);
    if (e != cudaSuccess) return e;
    const dim3 grid((NM + TM - 1) / TM, ncorner);
    mix_smem_kernel<<<grid, kThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace scx
