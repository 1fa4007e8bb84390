// Dual-corner complex mode mixing: the B200 replacement for spectral_mul_kernel and
// spectral_mul_dual_packed_kernel (spectral_conv_combo/spectral_conv_ext.su:5-92).
//
//   y_c[b][o][k] = sum_i x_c[b][i][k] * w_c[i][o][k]      c in {1, 2}, k over m1*m2 modes
//
// Unlike the reference kernel (one thread per output, weights re-read for every batch
// item) a thread here keeps one weight in a register and applies it to a block of
// batch items, and both corners run in one launch on the caller's stream.  Lanes of a
// warp walk consecutive modes, so every weight and spectrum load is a coalesced 256-byte
// row of the reference's [.., m1, m2, 2] layout.
#include <algorithm>

#include "scx_internal.h"

namespace scx {
namespace {

constexpr int kWarps = 8;
constexpr int kBatch = 8;  // batch items per thread

struct MixArgs {
    const float2* x[2];
    const float2* w[2];
    float2* y[2];
    int B, Cin, Cout, NM, nbchunk;
};

// grid = (mode tiles of 32, output-channel tiles of kWarps, ncorner * batch chunks)
__global__ void __launch_bounds__(kWarps * 32) mix_ffma_kernel(const MixArgs a) {
    const int corner = blockIdx.z / a.nbchunk;
    const int b0 = (blockIdx.z - corner * a.nbchunk) * kBatch;
    const float2* __restrict__ X = a.x[corner];
    const float2* __restrict__ Wt = a.w[corner];
    float2* __restrict__ Y = a.y[corner];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int mode = blockIdx.x * 32 + lane;
    const int o = blockIdx.y * kWarps + warp;
    if (mode >= a.NM || o >= a.Cout) return;
    const int nb = min(kBatch, a.B - b0);
    const size_t xs_b = static_cast<size_t>(a.Cin) * a.NM;
    float2 acc[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) acc[j] = make_float2(0.f, 0.f);
    const float2* xp = X + static_cast<size_t>(b0) * xs_b + mode;
    const float2* wp = Wt + static_cast<size_t>(o) * a.NM + mode;
    const size_t ws_i = static_cast<size_t>(a.Cout) * a.NM;
    for (int i = 0; i < a.Cin; ++i) {
        const float2 wv = __ldg(wp + i * ws_i);
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (j < nb) {
                const float2 xv = __ldg(xp + j * xs_b + static_cast<size_t>(i) * a.NM);
                acc[j].x = fmaf(xv.x, wv.x, fmaf(-xv.y, wv.y, acc[j].x));
                acc[j].y = fmaf(xv.x, wv.y, fmaf(xv.y, wv.x, acc[j].y));
            }
        }
    }
    float2* yp = Y + (static_cast<size_t>(b0) * a.Cout + o) * a.NM + mode;
    const size_t ys_b = static_cast<size_t>(a.Cout) * a.NM;
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
        if (j < nb) yp[j * ys_b] = acc[j];
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
    a.nbchunk = (B + kBatch - 1) / kBatch;
    const long long gz = static_cast<long long>(ncorner) * a.nbchunk;
    const long long gy = (Cout + kWarps - 1) / kWarps;
    if (gz > 65535 || gy > 65535) return cudaErrorInvalidValue;
    const dim3 grid((NM + 31) / 32, static_cast<unsigned>(gy), static_cast<unsigned>(gz));
    mix_ffma_kernel<<<grid, kWarps * 32, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace scx
