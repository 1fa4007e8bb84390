// Quadrant unfold for the folded tensor-core path (planes of 2Hs x 2Ws samples):
//
//   unfold: y[p][h + Hs alpha][w + Ws beta] = sum_q (-1)^(a alpha + b beta) zs[q][p][h][w]
//
// with q = 2a + b.  Because exp(-2 pi i k (n + N/2) / N) = (-1)^k exp(-2 pi i k n / N), the
// inverse of each parity class of the spectrum (rows kx = a, columns ky = b mod 2) against the
// full-period twiddles, unfolded, is the full inverse.  (The forward direction, the same 4 x 4
// sign matrix applied to the quadrants, runs inside the tensor-core forward kernel.)  Each
// thread reads four float4 (one per sub-plane) and writes four.
#include <algorithm>

#include "scx_internal.h"

namespace scx {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void butterfly(const float4& v00, const float4& v01, const float4& v10, const float4& v11,
                                          float4* o) {
    // v<alpha><beta>; o[2a + b]
#define SCX_BF(c)                                \
    {                                            \
        const float s0 = v00.c + v01.c;          \
        const float d0 = v00.c - v01.c;          \
        const float s1 = v10.c + v11.c;          \
        const float d1 = v10.c - v11.c;          \
        o[0].c = s0 + s1;                        \
        o[1].c = d0 + d1;                        \
        o[2].c = s0 - s1;                        \
        o[3].c = d0 - d1;                        \
    }
    SCX_BF(x) SCX_BF(y) SCX_BF(z) SCX_BF(w)
#undef SCX_BF
}

// Sub-planes zs[q] -> quadrants of y.
__global__ void __launch_bounds__(kThreads) unfold_kernel(const float4* __restrict__ in, float4* __restrict__ out,
                                                          int P, int Hs, int Ws4) {
    const long long per_plane = static_cast<long long>(Hs) * Ws4;  // float4 per sub-plane
    const long long total = per_plane * P;
    const long long sub_stride = total;                             // float4 between sub-planes
    for (long long i = blockIdx.x * static_cast<long long>(kThreads) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * kThreads) {
        const long long p = i / per_plane;
        const long long r = i - p * per_plane;
        const long long h = r / Ws4, w = r - h * Ws4;
        // full plane: 2Hs rows of 2 Ws4 float4
        const long long row0 = (p * 2 * Hs + h) * (2LL * Ws4), row1 = row0 + static_cast<long long>(Hs) * 2 * Ws4;
        const float4 z0 = __ldg(in + i), z1 = __ldg(in + sub_stride + i), z2 = __ldg(in + 2 * sub_stride + i),
                     z3 = __ldg(in + 3 * sub_stride + i);
        // y quadrant (alpha, beta) = sum_q (-1)^(a alpha + b beta) z_q
        float4 o[4];
        butterfly(z0, z1, z2, z3, o);
        __stcs(out + row0 + w, o[0]);
        __stcs(out + row0 + Ws4 + w, o[1]);
        __stcs(out + row1 + w, o[2]);
        __stcs(out + row1 + Ws4 + w, o[3]);
    }
}

}  // namespace

cudaError_t launch_unfold(const float* zs, float* y, int P, int Hs, int Ws, cudaStream_t stream) {
    if (P <= 0 || Hs <= 0 || Ws % 4 != 0 || ((reinterpret_cast<uintptr_t>(zs) | reinterpret_cast<uintptr_t>(y)) & 15))
        return cudaErrorInvalidValue;
    const long long total = static_cast<long long>(P) * Hs * (Ws / 4);
    const long long blocks = std::min<long long>((total + kThreads - 1) / kThreads, 8LL * num_sms());
    unfold_kernel<<<dim3(static_cast<unsigned>(blocks)), kThreads, 0, stream>>>(
        reinterpret_cast<const float4*>(zs), reinterpret_cast<float4*>(y), P, Hs, Ws / 4);
    return cudaGetLastError();
}

bool tc_split_supported(int H, int W, int m1, int m2) {
    if ((H != 128 && H != 256) || (W != 128 && W != 256)) return false;
    if (m1 % 2 != 0 || m2 % 2 != 0 || 2 * m1 > H) return false;
    const int Hs = H / 2, Ws = W / 2, m1s = m1 / 2, m2s = m2 / 2;
    return m1s >= 1 && m2s >= 1 && tc_fwd_supported(Hs, Ws, m1s, m2s) && tc_inv_supported(Hs, Ws, m1s, m2s);
}

size_t split_scratch_bytes(long long P, int H, int W) {
    return static_cast<size_t>(P) * static_cast<size_t>(H) * static_cast<size_t>(W) * sizeof(float);
}

}  // namespace scx
