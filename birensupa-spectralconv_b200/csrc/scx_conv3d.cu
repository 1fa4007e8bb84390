// SpectralConv3d forward, single low-frequency corner: the device replacement for
// spectral_conv3d_supa (spectral_conv_combo/spectral_conv_ops.py:435-472), which runs rfftn on
// the CPU, the mixing on the device and irfftn on the CPU.  The math is
// spectral_conv_combo/reference_pytorch.py:51-82: rfftn over (D, H, W), keep
// [:m1, :m2, :m3], per-mode channel mixing, zero-padded irfftn.
//
// Separable truncated direct DFTs (FFMA, fp32 accumulation; twiddles from sincospif of the
// exactly reduced phase (j t mod N) / N):
//   forward  W: real row -> m3 bins     H: keep ky < m2     D: keep kx < m1
//   mixing   the dual-corner kernel with one corner over NM = m1 m2 m3 modes
//   inverse  D: m1 -> D samples         H: m2 -> H samples  W: C2R from m3 bins, with the
//            Hermitian weights c_kz (1 for kz = 0 and, W even, kz = W/2; else 2) and 1/(DHW)
// The two complex passes of each direction are one kernel, out[o][t][i] = sum_j in[o][j][i]
// exp(sign 2 pi i j t / N), with the transformed axis between an outer and an inner index.
#include <algorithm>

#include "scx.h"
#include "scx_internal.h"

namespace {

constexpr int kThreads = 256;

inline size_t a256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

unsigned blocks_for(long long n) {
    return static_cast<unsigned>(std::max<long long>(1, std::min<long long>((n + kThreads - 1) / kThreads, 148LL * 32)));
}

// exp(sign * 2 pi i * (j t mod N) / N)
__device__ __forceinline__ float2 twiddle(long long jt, int N, float sign) {
    const int r = static_cast<int>(jt % N);
    float s, c;
    sincospif(2.0f * static_cast<float>(r) / static_cast<float>(N), &s, &c);
    return make_float2(c, sign * s);
}

// out[r][k] = sum_w x[r][w] exp(-2 pi i k w / W), k < m (real rows of length W).
__global__ void __launch_bounds__(kThreads) rdft_rows_kernel(const float* __restrict__ x, float2* __restrict__ out,
                                                             long long rows, int W, int m) {
    const long long total = rows * m;
    for (long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * kThreads) {
        const int k = static_cast<int>(t % m);
        const long long r = t / m;
        const float* xr = x + r * W;
        float re = 0.f, im = 0.f;
        for (int w = 0; w < W; ++w) {
            const float2 e = twiddle(static_cast<long long>(k) * w, W, -1.f);
            const float v = __ldg(xr + w);
            re = fmaf(v, e.x, re);
            im = fmaf(v, e.y, im);
        }
        out[t] = make_float2(re, im);
    }
}

// Frequency of slot u when the slots hold two corners of m rows each (m > 0): rows [0, m)
// are frequencies 0..m-1, rows [m, 2m) the top m frequencies N-m..N-1; m = 0 is the identity.
__device__ __forceinline__ int slot_freq(int u, int m, int N) { return (m > 0 && u >= m) ? N - 2 * m + u : u; }

// out[o][t][i] = sum_{j < nin} in[o][j][i] exp(sign 2 pi i f_j f_t / N), t < nout, with
// f_j = slot_freq(j, jmap, N) and f_t = slot_freq(t, tmap, N).
__global__ void __launch_bounds__(kThreads) axis_dft_kernel(const float2* __restrict__ in, float2* __restrict__ out,
                                                            long long outer, int nin, int nout, int inner, int N,
                                                            float sign, int jmap, int tmap) {
    const long long total = outer * nout * inner;
    for (long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * kThreads) {
        const int i = static_cast<int>(t % inner);
        const long long r = t / inner;
        const int to = static_cast<int>(r % nout);
        const long long o = r / nout;
        const float2* src = in + o * nin * inner + i;
        const int ft = slot_freq(to, tmap, N);
        float re = 0.f, im = 0.f;
        for (int j = 0; j < nin; ++j) {
            const float2 e = twiddle(static_cast<long long>(slot_freq(j, jmap, N)) * ft, N, sign);
            const float2 v = __ldg(src + static_cast<long long>(j) * inner);
            re = fmaf(v.x, e.x, fmaf(-v.y, e.y, re));
            im = fmaf(v.x, e.y, fmaf(v.y, e.x, im));
        }
        out[t] = make_float2(re, im);
    }
}

// y[r][w] = scale * sum_{k < m} c_k Re(v[r][k] exp(+2 pi i k w / W)).
__global__ void __launch_bounds__(kThreads) c2r_rows_kernel(const float2* __restrict__ v, float* __restrict__ y,
                                                            long long rows, int W, int m, float scale) {
    const long long total = rows * W;
    for (long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * kThreads) {
        const int w = static_cast<int>(t % W);
        const long long r = t / W;
        const float2* vr = v + r * m;
        float acc = 0.f;
        for (int k = 0; k < m; ++k) {
            const float2 e = twiddle(static_cast<long long>(k) * w, W, 1.f);
            const float2 a = __ldg(vr + k);
            const float c = (k == 0 || ((W % 2) == 0 && k == W / 2)) ? 1.f : 2.f;
            acc = fmaf(c, fmaf(a.x, e.x, -a.y * e.y), acc);
        }
        y[t] = acc * scale;
    }
}

// Corner c = a + 2 b (a: kx rows high, b: ky rows high) of the slot array all
// [P][2 m1][2 m2][m3] <-> its own array corners[c] [P][m1][m2][m3].
__global__ void __launch_bounds__(kThreads) split_corners_kernel(const float2* __restrict__ all, float2* c0,
                                                                 float2* c1, float2* c2, float2* c3, long long P,
                                                                 int m1, int m2, int m3) {
    const long long total = P * 4 * m1 * m2 * m3;
    for (long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * kThreads) {
        const int kz = static_cast<int>(t % m3);
        long long r = t / m3;
        const int s2 = static_cast<int>(r % (2 * m2));
        r /= 2 * m2;
        const int s1 = static_cast<int>(r % (2 * m1));
        const long long p = r / (2 * m1);
        const int c = (s1 >= m1 ? 1 : 0) + (s2 >= m2 ? 2 : 0);
        float2* dst = c == 0 ? c0 : (c == 1 ? c1 : (c == 2 ? c2 : c3));
        dst[((p * m1 + s1 % m1) * m2 + s2 % m2) * m3 + kz] = __ldg(all + t);
    }
}

// The inverse's slot array from the four mixed corners, where a frequency that several
// corners hold keeps only the last assignment of official_baseline.py:89-96 (corner order
// 0, 1, 2, 3 as above): every other slot holding it is zero.
__global__ void __launch_bounds__(kThreads) merge_corners_kernel(const float2* c0, const float2* c1,
                                                                 const float2* c2, const float2* c3,
                                                                 float2* __restrict__ all, long long P, int m1,
                                                                 int m2, int m3, int D, int H) {
    const long long total = P * 4 * m1 * m2 * m3;
    for (long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * kThreads) {
        const int kz = static_cast<int>(t % m3);
        long long r = t / m3;
        const int s2 = static_cast<int>(r % (2 * m2));
        r /= 2 * m2;
        const int s1 = static_cast<int>(r % (2 * m1));
        const long long p = r / (2 * m1);
        const int a = s1 >= m1 ? 1 : 0, b = s2 >= m2 ? 1 : 0, c = a + 2 * b;
        const int kx = slot_freq(s1, m1, D), ky = slot_freq(s2, m2, H);
        const bool kx_in[2] = {kx < m1, kx >= D - m1};
        const bool ky_in[2] = {ky < m2, ky >= H - m2};
        bool dropped = false;
        for (int c2i = c + 1; c2i < 4; ++c2i) dropped = dropped || (kx_in[c2i & 1] && ky_in[c2i >> 1]);
        const float2* src = c == 0 ? c0 : (c == 1 ? c1 : (c == 2 ? c2 : c3));
        all[t] = dropped ? make_float2(0.f, 0.f) : __ldg(src + ((p * m1 + s1 % m1) * m2 + s2 % m2) * m3 + kz);
    }
}

struct Layout3 {
    size_t t1, t2, xc, yc, u1, u2, total;
};

// Work arrays (complex): forward T1 [B Cin D H][m3], T2 [B Cin D][m2][m3], X [B Cin][m1 m2 m3];
// Y [B Cout][m1 m2 m3]; inverse U1 [B Cout][D][m2 m3], U2 [B Cout D][H][m3].
Layout3 layout3(int B, int Cin, int Cout, int D, int H, int m1, int m2, int m3) {
    Layout3 L;
    const size_t f2 = sizeof(float2);
    L.t1 = a256(static_cast<size_t>(B) * Cin * D * H * m3 * f2);
    L.t2 = a256(static_cast<size_t>(B) * Cin * D * m2 * m3 * f2);
    L.xc = a256(static_cast<size_t>(B) * Cin * m1 * m2 * m3 * f2);
    L.yc = a256(static_cast<size_t>(B) * Cout * m1 * m2 * m3 * f2);
    L.u1 = a256(static_cast<size_t>(B) * Cout * D * m2 * m3 * f2);
    L.u2 = a256(static_cast<size_t>(B) * Cout * D * H * m3 * f2);
    L.total = L.t1 + L.t2 + L.xc + L.yc + L.u1 + L.u2;
    return L;
}

bool valid3(int B, int Cin, int Cout, int D, int H, int W, int m1, int m2, int m3) {
    if (B <= 0 || Cin <= 0 || Cout <= 0 || D <= 0 || H <= 0 || W <= 0 || m1 <= 0 || m2 <= 0 || m3 <= 0)
        return false;
    if (m1 > D || m2 > H || m3 > W / 2 + 1) return false;
    const double big = static_cast<double>(B) * std::max(Cin, Cout) * D * H * W;
    const double nm = static_cast<double>(m1) * m2 * m3;
    return big < 2147483647.0 && static_cast<double>(Cin) * Cout * nm < 2147483647.0 &&
           static_cast<double>(B) * std::max(Cin, Cout) * nm < 2147483647.0;
}

}  // namespace

extern "C" size_t scx_spectral_conv3d_workspace_size(int batch_size, int channels_in, int channels_out, int depth,
                                                     int height, int width, int modes1, int modes2, int modes3) {
    if (!valid3(batch_size, channels_in, channels_out, depth, height, width, modes1, modes2, modes3)) return 0;
    return layout3(batch_size, channels_in, channels_out, depth, height, modes1, modes2, modes3).total;
}

extern "C" int scx_spectral_conv3d_fwd(const float* x, const float* weights, float* y, int batch_size,
                                       int channels_in, int channels_out, int depth, int height, int width,
                                       int modes1, int modes2, int modes3, void* workspace, size_t workspace_bytes,
                                       scx_stream_t stream) {
    if (!x || !weights || !y || !workspace) return cudaErrorInvalidValue;
    const size_t need = scx_spectral_conv3d_workspace_size(batch_size, channels_in, channels_out, depth, height,
                                                           width, modes1, modes2, modes3);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) % 4 != 0 ||
        reinterpret_cast<uintptr_t>(weights) % 8 != 0 || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return cudaErrorInvalidValue;
    const int B = batch_size, Cin = channels_in, Cout = channels_out, D = depth, H = height, W = width;
    const int m1 = modes1, m2 = modes2, m3 = modes3;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Layout3 L = layout3(B, Cin, Cout, D, H, m1, m2, m3);
    unsigned char* base = static_cast<unsigned char*>(workspace);
    float2* T1 = reinterpret_cast<float2*>(base);
    float2* T2 = reinterpret_cast<float2*>(base + L.t1);
    float2* X = reinterpret_cast<float2*>(base + L.t1 + L.t2);
    float2* Y = reinterpret_cast<float2*>(base + L.t1 + L.t2 + L.xc);
    float2* U1 = reinterpret_cast<float2*>(base + L.t1 + L.t2 + L.xc + L.yc);
    float2* U2 = reinterpret_cast<float2*>(base + L.t1 + L.t2 + L.xc + L.yc + L.u1);
    const long long bi = static_cast<long long>(B) * Cin, bo = static_cast<long long>(B) * Cout;
    const int NM = m1 * m2 * m3;

    // forward: W (real -> m3), H (keep m2), D (keep m1)
    long long n = bi * D * H * m3;
    rdft_rows_kernel<<<blocks_for(n), kThreads, 0, s>>>(x, T1, bi * D * H, W, m3);
    n = bi * D * m2 * m3;
    axis_dft_kernel<<<blocks_for(n), kThreads, 0, s>>>(T1, T2, bi * D, H, m2, m3, H, -1.f, 0, 0);
    n = bi * m1 * m2 * m3;
    axis_dft_kernel<<<blocks_for(n), kThreads, 0, s>>>(T2, X, bi, D, m1, m2 * m3, D, -1.f, 0, 0);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // mixing over the corner's modes
    e = scx::launch_mix(X, nullptr, reinterpret_cast<const float2*>(weights), nullptr, Y, nullptr, 1, B, Cin, Cout,
                        NM, s);
    if (e != cudaSuccess) return e;
    // inverse: D (m1 -> D), H (m2 -> H), W (C2R from m3)
    n = bo * D * m2 * m3;
    axis_dft_kernel<<<blocks_for(n), kThreads, 0, s>>>(Y, U1, bo, m1, D, m2 * m3, D, 1.f, 0, 0);
    n = bo * D * H * m3;
    axis_dft_kernel<<<blocks_for(n), kThreads, 0, s>>>(U1, U2, bo * D, m2, H, m3, H, 1.f, 0, 0);
    n = bo * D * H * W;
    c2r_rows_kernel<<<blocks_for(n), kThreads, 0, s>>>(U2, y, bo * D * H, W, m3,
                                                        static_cast<float>(1.0 / (static_cast<double>(D) * H * W)));
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Four-corner SpectralConv3d (official_baseline.py:60-100): corners (low|high kx) x (low|high
// ky), low kz, each with its own weights.  The forward H and D passes keep 2 m2 and 2 m1 slot
// rows (low then high frequencies), the corners are split out for two dual-corner mixings,
// merged back with the baseline's overwrite order, and the inverse runs over the slots.

namespace {

struct Layout4 {
    size_t t1, t2, xall, xc, yc, yall, u1, u2, total;
};

Layout4 layout4(int B, int Cin, int Cout, int D, int H, int m1, int m2, int m3) {
    Layout4 L;
    const size_t f2 = sizeof(float2);
    const size_t nm = static_cast<size_t>(m1) * m2 * m3;
    L.t1 = a256(static_cast<size_t>(B) * Cin * D * H * m3 * f2);
    L.t2 = a256(static_cast<size_t>(B) * Cin * D * 2 * m2 * m3 * f2);
    L.xall = a256(static_cast<size_t>(B) * Cin * 4 * nm * f2);
    L.xc = a256(static_cast<size_t>(B) * Cin * nm * f2);   // per corner
    L.yc = a256(static_cast<size_t>(B) * Cout * nm * f2);  // per corner
    L.yall = a256(static_cast<size_t>(B) * Cout * 4 * nm * f2);
    L.u1 = a256(static_cast<size_t>(B) * Cout * D * 2 * m2 * m3 * f2);
    L.u2 = a256(static_cast<size_t>(B) * Cout * D * H * m3 * f2);
    L.total = L.t1 + L.t2 + L.xall + 4 * L.xc + 4 * L.yc + L.yall + L.u1 + L.u2;
    return L;
}

}  // namespace

extern "C" size_t scx_spectral_conv3d_4c_workspace_size(int batch_size, int channels_in, int channels_out, int depth,
                                                        int height, int width, int modes1, int modes2, int modes3) {
    if (!valid3(batch_size, channels_in, channels_out, depth, height, width, modes1, modes2, modes3)) return 0;
    if (static_cast<double>(batch_size) * std::max(channels_in, channels_out) * 4.0 * modes1 * modes2 * modes3 >=
        2147483647.0)
        return 0;
    return layout4(batch_size, channels_in, channels_out, depth, height, modes1, modes2, modes3).total;
}

extern "C" int scx_spectral_conv3d_4c_fwd(const float* x, const float* w1, const float* w2, const float* w3,
                                          const float* w4, float* y, int batch_size, int channels_in,
                                          int channels_out, int depth, int height, int width, int modes1,
                                          int modes2, int modes3, void* workspace, size_t workspace_bytes,
                                          scx_stream_t stream) {
    if (!x || !w1 || !w2 || !w3 || !w4 || !y || !workspace) return cudaErrorInvalidValue;
    const size_t need = scx_spectral_conv3d_4c_workspace_size(batch_size, channels_in, channels_out, depth, height,
                                                              width, modes1, modes2, modes3);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) % 4 != 0 ||
        (reinterpret_cast<uintptr_t>(w1) | reinterpret_cast<uintptr_t>(w2) | reinterpret_cast<uintptr_t>(w3) |
         reinterpret_cast<uintptr_t>(w4)) % 8 != 0 ||
        reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return cudaErrorInvalidValue;
    const int B = batch_size, Cin = channels_in, Cout = channels_out, D = depth, H = height, W = width;
    const int m1 = modes1, m2 = modes2, m3 = modes3;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Layout4 L = layout4(B, Cin, Cout, D, H, m1, m2, m3);
    unsigned char* p = static_cast<unsigned char*>(workspace);
    auto take = [&](size_t bytes) {
        float2* r = reinterpret_cast<float2*>(p);
        p += bytes;
        return r;
    };
    float2* T1 = take(L.t1);
    float2* T2 = take(L.t2);
    float2* Xall = take(L.xall);
    float2* Xc[4] = {take(L.xc), take(L.xc), take(L.xc), take(L.xc)};
    float2* Yc[4] = {take(L.yc), take(L.yc), take(L.yc), take(L.yc)};
    float2* Yall = take(L.yall);
    float2* U1 = take(L.u1);
    float2* U2 = take(L.u2);
    const long long bi = static_cast<long long>(B) * Cin, bo = static_cast<long long>(B) * Cout;
    const int NM = m1 * m2 * m3;

    // forward: W (real -> m3), H (2 m2 slot rows), D (2 m1 slot rows), split into corners
    long long n = bi * D * H * m3;
    rdft_rows_kernel<<<blocks_for(n), kThreads, 0, s>>>(x, T1, bi * D * H, W, m3);
    n = bi * D * 2 * m2 * m3;
    axis_dft_kernel<<<blocks_for(n), kThreads, 0, s>>>(T1, T2, bi * D, H, 2 * m2, m3, H, -1.f, 0, m2);
    n = bi * 2 * m1 * 2 * m2 * m3;
    axis_dft_kernel<<<blocks_for(n), kThreads, 0, s>>>(T2, Xall, bi, D, 2 * m1, 2 * m2 * m3, D, -1.f, 0, m1);
    split_corners_kernel<<<blocks_for(n), kThreads, 0, s>>>(Xall, Xc[0], Xc[1], Xc[2], Xc[3], bi, m1, m2, m3);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // mixing: corners 0, 1 and 2, 3
    const float2* Wc[4] = {reinterpret_cast<const float2*>(w1), reinterpret_cast<const float2*>(w2),
                           reinterpret_cast<const float2*>(w3), reinterpret_cast<const float2*>(w4)};
    e = scx::launch_mix(Xc[0], Xc[1], Wc[0], Wc[1], Yc[0], Yc[1], 2, B, Cin, Cout, NM, s);
    if (e == cudaSuccess) e = scx::launch_mix(Xc[2], Xc[3], Wc[2], Wc[3], Yc[2], Yc[3], 2, B, Cin, Cout, NM, s);
    if (e != cudaSuccess) return e;
    // inverse: merge with the overwrite order, D (2 m1 slots -> D), H (2 m2 slots -> H), W (C2R)
    n = bo * 2 * m1 * 2 * m2 * m3;
    merge_corners_kernel<<<blocks_for(n), kThreads, 0, s>>>(Yc[0], Yc[1], Yc[2], Yc[3], Yall, bo, m1, m2, m3, D, H);
    n = bo * D * 2 * m2 * m3;
    axis_dft_kernel<<<blocks_for(n), kThreads, 0, s>>>(Yall, U1, bo, 2 * m1, D, 2 * m2 * m3, D, 1.f, m1, 0);
    n = bo * D * H * m3;
    axis_dft_kernel<<<blocks_for(n), kThreads, 0, s>>>(U1, U2, bo * D, 2 * m2, H, m3, H, 1.f, m2, 0);
    n = bo * D * H * W;
    c2r_rows_kernel<<<blocks_for(n), kThreads, 0, s>>>(U2, y, bo * D * H, W, m3,
                                                        static_cast<float>(1.0 / (static_cast<double>(D) * H * W)));
    return cudaGetLastError();
}
