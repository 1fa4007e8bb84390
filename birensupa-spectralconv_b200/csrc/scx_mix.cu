// Dual-corner complex mode mixing: the B200 replacement for spectral_mul_kernel and
// spectral_mul_dual_packed_kernel (spectral_conv_combo/spectral_conv_ext.su:5-92).
//
//   y_c[b][o][k] = sum_i x_c[b][i][k] * w_c[i][o][k]      c in {1, 2}, k over m1*m2 modes
//
// mix_tma_kernel (mode counts that are even, 16-byte aligned operands): one CTA owns one
// corner, a tile of TM consecutive modes and a range of output channels.  One 3-D TMA
// load brings x_c[:, :, tile] (every batch item and input channel) and one brings
// w_c[:, o-range, tile] into shared memory - no per-thread global loads, every weight
// byte read once per CTA - then each thread accumulates a 2 (output channels) x 4 (batch
// items) block of complex outputs per mode.  mix_smem_kernel is the same contraction with
// per-thread loads, for the shapes the TMA boxes cannot describe.  Both corners run in
// one launch on the caller's stream (the reference launched them serially on the null
// stream).
#include <algorithm>
#include <mutex>

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

    for (int idx = threadIdx.x; idx < B * Cin * tm; idx += kThreads) {
        const int row = idx / tm, kk = idx - row * tm;
        Xs[row * TM + kk] = __ldg(X + static_cast<size_t>(row) * NM + k0 + kk);
    }
    for (int idx = threadIdx.x; idx < Cin * Cout * tm; idx += kThreads) {
        const int row = idx / tm, kk = idx - row * tm;
        Ws[row * TM + kk] = __ldg(Wt + static_cast<size_t>(row) * NM + k0 + kk);
    }
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


struct MixTmaArgs {
    float2* y[2];
    int B, Cin, Cout, NM, OC, TM, BB, n_os;  // BB batch items per CTA; n_os output-channel splits
    uint32_t x_bytes, w_bytes, w_off;  // box bytes, byte offset of the weight tile
    int* watchdog;
};

// x_c viewed as [B][Cin][2*NM] floats, w_c as [Cin][Cout][2*NM]; boxes (2*TM, Cin, B) and
// (2*TM, OC, Cin) land in shared memory in exactly the [B][Cin][TM] / [Cin][OC][TM] float2
// order the accumulation loop reads (no swizzle).  Modes past NM read as zero.
template <int TM>
__global__ void __launch_bounds__(kThreads) mix_tma_kernel(const __grid_constant__ CUtensorMap tx0,
                                                           const __grid_constant__ CUtensorMap tx1,
                                                           const __grid_constant__ CUtensorMap tw0,
                                                           const __grid_constant__ CUtensorMap tw1,
                                                           const MixTmaArgs a) {
    extern __shared__ uint8_t mix_raw[];
    __shared__ uint64_t bar;
    __shared__ int tiles_ok;
    uint8_t* base = tc::align1024(mix_raw);
    const int corner = blockIdx.y;
    const int k0 = blockIdx.x * TM;
    const int o_base = (blockIdx.z % a.n_os) * a.OC, b_base = (blockIdx.z / a.n_os) * a.BB;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        tc::fence_async_smem();
        tc::mbar_arrive_expect_tx(&bar, a.x_bytes + a.w_bytes);
        tc::tma_load_3d(base, corner ? &tx1 : &tx0, 2 * k0, 0, b_base, &bar);
        tc::tma_load_3d(base + a.w_off, corner ? &tw1 : &tw0, 2 * k0, o_base, 0, &bar);
        // one thread waits for the tiles while the others park at the barrier
        tiles_ok = tc::mbar_wait_bounded(&bar, 0) ? 1 : 0;
        if (!tiles_ok) atomicExch(a.watchdog, 40);
    }
    __syncthreads();
    if (!tiles_ok) return;
    const float2* Xs = reinterpret_cast<const float2*>(base);            // [BB][Cin][TM]
    const float2* Ws = reinterpret_cast<const float2*>(base + a.w_off);  // [Cin][OCs][TM]
    const int BBs = a.BB, B = min(a.BB, a.B - b_base), Cin = a.Cin, OCs = a.OC, OC = min(a.OC, a.Cout - o_base);
    const int tm = min(TM, a.NM - k0);
    float2* __restrict__ Y = a.y[corner];
    const int nog = (OC + kOT - 1) / kOT;
    const int nbg = (B + kBT - 1) / kBT;
    const int ntiles = tm * nog * nbg;
    const int wstride = OCs * TM;  // float2 between consecutive input channels of a weight column
    for (int t = threadIdx.x; t < ntiles; t += kThreads) {
        const int kk = t % tm;
        const int rest = t / tm;
        const int og = rest % nog, bg = rest / nog;
        const int o0 = og * kOT, b0 = bg * kBT;
        // operand columns; rows past the staged tile are clamped (their products are never stored)
        const float2* wp[kOT];
        const float2* xp[kBT];
#pragma unroll
        for (int p = 0; p < kOT; ++p) wp[p] = Ws + min(o0 + p, OCs - 1) * TM + kk;
#pragma unroll
        for (int q = 0; q < kBT; ++q) xp[q] = Xs + static_cast<size_t>(min(b0 + q, BBs - 1)) * Cin * TM + kk;
        float2 acc[kOT][kBT];
#pragma unroll
        for (int p = 0; p < kOT; ++p)
#pragma unroll
            for (int q = 0; q < kBT; ++q) acc[p][q] = make_float2(0.f, 0.f);
#pragma unroll 4
        for (int i = 0; i < Cin; ++i) {
            float2 wv[kOT], xv[kBT];
#pragma unroll
            for (int p = 0; p < kOT; ++p) wv[p] = wp[p][i * wstride];
#pragma unroll
            for (int q = 0; q < kBT; ++q) xv[q] = xp[q][i * TM];
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
                if (o0 + p < OC && b0 + q < B)
                    Y[(static_cast<size_t>(b_base + b0 + q) * a.Cout + o_base + o0 + p) * a.NM + k0 + kk] = acc[p][q];
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

// 3-D fp32 tensor [d2][d1][d0] (d0 innermost), box (b0, b1, b2).
bool encode3d(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0, uint32_t b1,
              uint32_t b2) {
    EncodeTiledFn fn = encode_tiled();
    if (fn == nullptr) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {d0 * 4, d0 * d1 * 4};
    const cuuint32_t box[3] = {b0, b1, b2};
    const cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The TMA-staged launch; returns cudaErrorNotSupported when the shape or alignment does not
// fit its boxes (the caller then uses mix_smem_kernel).
cudaError_t launch_mix_tma(const float2* x1, const float2* x2, const float2* w1, const float2* w2, float2* y1,
                           float2* y2, int ncorner, int B, int Cin, int Cout, int NM, cudaStream_t stream) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(x1) | reinterpret_cast<uintptr_t>(w1) |
                         (ncorner == 2 ? (reinterpret_cast<uintptr_t>(x2) | reinterpret_cast<uintptr_t>(w2)) : 0);
    if (NM % 2 != 0 || (al & 15) != 0 || B > 256 || Cin > 256) return cudaErrorNotSupported;
    // Mode tile: 4 when there are enough tiles to fill the GPU twice over, else 2; output
    // channels split across CTAs until the GPU is filled and the weight tile stays small.
    const long long want = 2LL * num_sms();
    const int TM = (static_cast<long long>(ncorner) * (NM / 4) >= want) ? 4 : 2;
    const long long tiles = static_cast<long long>(ncorner) * ((NM + TM - 1) / TM);
    int os = 1;
    const int bs = 1;
    while (os < Cout && (tiles * os < want || static_cast<long long>(Cin) * ((Cout + os - 1) / os) * TM * 8 > 64 * 1024))
        os *= 2;
    const int OC = (Cout + os - 1) / os, BB = (B + bs - 1) / bs;
    if (OC > 256 || BB > 256) return cudaErrorNotSupported;
    MixTmaArgs a;
    a.y[0] = y1;
    a.y[1] = y2;
    a.B = B;
    a.Cin = Cin;
    a.Cout = Cout;
    a.NM = NM;
    a.OC = OC;
    a.TM = TM;
    a.BB = BB;
    a.n_os = (Cout + OC - 1) / OC;
    const int n_bs = (B + BB - 1) / BB;
    a.x_bytes = static_cast<uint32_t>(BB) * Cin * TM * 8u;
    a.w_bytes = static_cast<uint32_t>(Cin) * OC * TM * 8u;
    a.w_off = (a.x_bytes + 127u) / 128u * 128u;
    const size_t smem = a.w_off + a.w_bytes + 1024;
    if (smem > 200 * 1024) return cudaErrorNotSupported;
    cudaError_t e = device_watchdog(&a.watchdog);
    if (e != cudaSuccess) return e;
    CUtensorMap tx[2], tw[2];
    const int nc = ncorner;
    const float2* xs[2] = {x1, x2};
    const float2* ws[2] = {w1, w2};
    for (int c = 0; c < 2; ++c) {
        const int src = c < nc ? c : 0;  // an unused second corner repeats the first map
        if (!encode3d(&tx[c], xs[src], 2ull * NM, Cin, B, 2u * TM, Cin, BB) ||
            !encode3d(&tw[c], ws[src], 2ull * NM, Cout, Cin, 2u * TM, OC, Cin))
            return cudaErrorNotSupported;
    }
    int per_sm = 1;
    const dim3 grid((NM + TM - 1) / TM, ncorner, a.n_os * n_bs);
    auto run = [&](auto kernel) -> cudaError_t {
        cudaError_t err = prepare_kernel(reinterpret_cast<const void*>(kernel), smem, kThreads, &per_sm);
        if (err != cudaSuccess) return err;
        kernel<<<grid, kThreads, smem, stream>>>(tx[0], tx[1], tw[0], tw[1], a);
        return cudaGetLastError();
    };
    return TM == 4 ? run(mix_tma_kernel<4>) : run(mix_tma_kernel<2>);
}

}  // namespace

cudaError_t launch_mix(const float2* x1, const float2* x2, const float2* w1, const float2* w2,
                       float2* y1, float2* y2, int ncorner, int B, int Cin, int Cout, int NM,
                       cudaStream_t stream) {
    const cudaError_t te = launch_mix_tma(x1, x2, w1, w2, y1, y2, ncorner, B, Cin, Cout, NM, stream);
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
