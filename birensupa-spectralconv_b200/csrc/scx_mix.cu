// Dual-corner complex mode mixing: the B200 replacement for spectral_mul_kernel and
// spectral_mul_dual_packed_kernel (spectral_conv_combo/spectral_conv_ext.su:5-92).
//
//   y_c[b][o][k] = sum_i x_c[b][i][k] * w_c[i][o][k]      c in {1, 2}, k over m1*m2 modes
//
// One CTA owns one corner and a tile of TM consecutive modes for every batch item and
// output channel.  It stages x_c[:, :, tile] and w_c[:, :, tile] in shared memory with
// loads of TM contiguous modes (one 32-byte sector at TM = 4) - every weight byte is
// read once - and then each thread accumulates a 2 (output channels) x 4 (batch items)
// block of complex outputs per mode from shared memory.  Both corners run in one launch
// on the caller's stream (the reference launched them serially on the null stream).
#include <algorithm>

#include "scx_internal.h"

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

}  // namespace

cudaError_t launch_mix(const float2* x1, const float2* x2, const float2* w1, const float2* w2,
                       float2* y1, float2* y2, int ncorner, int B, int Cin, int Cout, int NM,
                       cudaStream_t stream) {
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
