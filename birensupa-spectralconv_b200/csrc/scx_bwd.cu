// SpectralConv2d backward: the gradients torch's autograd gives for the reference forward
// (spectral_conv/reference_pytorch.py:30-47: rfft2, two corner einsums, zero-padded irfft2),
// from the forward's corner spectra.  The reference itself differentiates only the mixing
// (SpectralMulFunction, spectral_conv/spectral_conv_ops.py:260-286); this extends it to the
// whole layer on the device.
//
// With y = sum over retained (kx, ky) of (c_ky / HW) Re(Y e^{+i theta}) (c_ky = 1 for ky = 0
// and, W even, ky = W/2, else 2; the inverse kernels' row weights), Y_c = mix(X_c, W_c) per
// mode and X = sum x e^{-i theta}, torch's conventions (gradient = dL/dRe + i dL/dIm) give
//   G       = fwd(grad_y)                          (the forward DFT kernel, unscaled)
//   grad_Y  = (c_ky / HW) G
//   grad_X  = grad_Y W^H per mode,   grad_W = X^H grad_Y per mode
//   grad_x  = sum Re(grad_X e^{+i theta}) = inv(G W^H)
// The last line holds because c_ky / HW depends only on the mode, so it commutes with the
// channel mixing and cancels the inverse kernel's own row weights.  Corner-1 rows that corner
// 2 overwrites in the forward (2 m1 > H) do not reach y, so their G rows are zeroed first;
// the inverse drops those rows of grad_X, which are then zero anyway.
//
// Kernels: the forward DFT, two dual-corner mixings and the inverse DFT of the forward path.
// The mixings read W^H and X^H straight from the weights and the saved corners (the TMA-ring
// kernel with transposed tensor maps, conjugating in registers; the per-ky scale of grad_W is
// per mode, so it commutes with the mixing and is applied to its result).  Where the ring
// kernel does not apply, conjugate-transpose passes write W^H and (c_ky / HW) X^H first.  With
// overlapping corners a small pass masks the overlap rows.
#include <algorithm>

#include "scx.h"
#include "scx_internal.h"

namespace {

constexpr int kThreads = 256;

inline size_t a256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

// out_c[d1][d0][m] = f(m) conj(in_c[d0][d1][m]) for both corners c = blockIdx.y (complex
// [D0][D1][NM], modes contiguous), f(m) = 1, or c_ky / (H W) for mode m = kx m2 + ky when
// `scaled` (c_ky = 1 for ky = 0 and, W even, ky = W/2, else 2).  Threads walk the output in
// order.
__global__ void __launch_bounds__(kThreads) conj_transpose_kernel(const float2* __restrict__ in1,
                                                                  const float2* __restrict__ in2,
                                                                  float2* __restrict__ out1, float2* __restrict__ out2,
                                                                  int D0, int D1, int NM, int scaled, int m2, int W,
                                                                  float inv_hw) {
    const float2* in = blockIdx.y == 0 ? in1 : in2;
    float2* out = blockIdx.y == 0 ? out1 : out2;
    const long long total = static_cast<long long>(D0) * D1 * NM;
    for (long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * kThreads) {
        const int m = static_cast<int>(t % NM);
        const long long r = t / NM;
        const int d0 = static_cast<int>(r % D0), d1 = static_cast<int>(r / D0);
        const float2 v = __ldg(in + (static_cast<long long>(d0) * D1 + d1) * NM + m);
        float f = 1.f;
        if (scaled) {
            const int ky = m % m2;
            f = (ky == 0 || ((W % 2) == 0 && ky == W / 2)) ? inv_hw : 2.0f * inv_hw;
        }
        out[t] = make_float2(f * v.x, -(f * v.y));
    }
}

// g1[p][s][ky] = 0 for corner-1 slots s in [r0, m1) (spectrum rows that corner 2 overwrites).
__global__ void __launch_bounds__(kThreads) zero_rows_kernel(float2* __restrict__ g1, long long planes, int m1,
                                                             int m2, int r0) {
    const int nrow = m1 - r0;
    const long long total = planes * nrow * m2;
    for (long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * kThreads) {
        const int ky = static_cast<int>(t % m2);
        const long long r = t / m2;
        const int s = r0 + static_cast<int>(r % nrow);
        const long long p = r / nrow;
        g1[(p * m1 + s) * m2 + ky] = make_float2(0.f, 0.f);
    }
}

unsigned blocks_for(long long n) {
    return static_cast<unsigned>(std::min<long long>((n + kThreads - 1) / kThreads, 148LL * 16));
}

struct BwdLayout {
    size_t g, z, wh, xh, scratch, total;
};

BwdLayout bwd_layout(int B, int Cin, int Cout, int H, int W, int m1, int m2) {
    const size_t NM = static_cast<size_t>(m1) * m2;
    BwdLayout L;
    L.g = a256(static_cast<size_t>(B) * Cout * NM * sizeof(float2));    // G per corner
    L.z = a256(static_cast<size_t>(B) * Cin * NM * sizeof(float2));     // G W^H per corner
    L.wh = a256(static_cast<size_t>(Cout) * Cin * NM * sizeof(float2)); // W^H per corner
    L.xh = a256(static_cast<size_t>(Cin) * B * NM * sizeof(float2));    // X^H per corner
    L.scratch = scx::tc_split_supported(H, W, m1, m2)
                    ? a256(scx::split_scratch_bytes(static_cast<long long>(B) * std::max(Cin, Cout), H, W))
                    : 0;
    L.total = 2 * (L.g + L.z + L.wh + L.xh) + L.scratch;
    return L;
}

}  // namespace

extern "C" size_t scx_spectral_conv2d_bwd_workspace_size(int batch_size, int channels_in, int channels_out,
                                                         int height, int width, int modes1, int modes2) {
    // the forward's shape rules
    if (scx_spectral_conv2d_workspace_size(batch_size, channels_in, channels_out, height, width, modes1, modes2) == 0)
        return 0;
    return bwd_layout(batch_size, channels_in, channels_out, height, width, modes1, modes2).total;
}

extern "C" int scx_spectral_conv2d_bwd(const float* grad_y, const float* x_corners, const float* weights1,
                                       const float* weights2, float* grad_x, float* grad_w1, float* grad_w2,
                                       int batch_size, int channels_in, int channels_out, int height, int width,
                                       int modes1, int modes2, void* workspace, size_t workspace_bytes,
                                       scx_stream_t stream) {
    if (!grad_y || !weights1 || !weights2 || !workspace) return cudaErrorInvalidValue;
    if ((grad_w1 == nullptr) != (grad_w2 == nullptr)) return cudaErrorInvalidValue;
    if (grad_w1 && !x_corners) return cudaErrorInvalidValue;
    const size_t need = scx_spectral_conv2d_bwd_workspace_size(batch_size, channels_in, channels_out, height, width,
                                                               modes1, modes2);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    auto misaligned = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) != 0; };
    if (misaligned(grad_y, 4) || misaligned(weights1, 8) || misaligned(weights2, 8) || misaligned(workspace, 256) ||
        (grad_x && misaligned(grad_x, 4)) || (x_corners && misaligned(x_corners, 8)) ||
        (grad_w1 && (misaligned(grad_w1, 8) || misaligned(grad_w2, 8))))
        return cudaErrorInvalidValue;
    const int B = batch_size, Cin = channels_in, Cout = channels_out, H = height, W = width, m1 = modes1,
              m2 = modes2;
    const int NM = m1 * m2;
    const scx::Twiddles* tw = nullptr;
    cudaError_t e = scx::get_twiddles(H, W, m1, m2, &tw);
    if (e != cudaSuccess) return e;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const BwdLayout L = bwd_layout(B, Cin, Cout, H, W, m1, m2);
    unsigned char* base = static_cast<unsigned char*>(workspace);
    float2* G1 = reinterpret_cast<float2*>(base);
    float2* G2 = reinterpret_cast<float2*>(base + L.g);
    float2* Z1 = reinterpret_cast<float2*>(base + 2 * L.g);
    float2* Z2 = reinterpret_cast<float2*>(base + 2 * L.g + L.z);
    float2* WH1 = reinterpret_cast<float2*>(base + 2 * (L.g + L.z));
    float2* WH2 = reinterpret_cast<float2*>(base + 2 * (L.g + L.z) + L.wh);
    float2* XH1 = reinterpret_cast<float2*>(base + 2 * (L.g + L.z + L.wh));
    float2* XH2 = reinterpret_cast<float2*>(base + 2 * (L.g + L.z + L.wh) + L.xh);
    float* scratch = L.scratch ? reinterpret_cast<float*>(base + 2 * (L.g + L.z + L.wh + L.xh)) : nullptr;

    // G = fwd(grad_y), both corners, [B][Cout][m1][m2]
    e = scx::dft_fwd(grad_y, G1, G2, NM, m2, B * Cout, H, W, m1, m2, *tw, s, scratch, L.scratch);
    if (e != cudaSuccess) return e;
    if (2 * m1 > H) {
        const long long n = static_cast<long long>(B) * Cout * (2 * m1 - H) * m2;
        zero_rows_kernel<<<blocks_for(n), kThreads, 0, s>>>(G1, static_cast<long long>(B) * Cout, m1, m2, H - m1);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    // conjugate transposes per mode: W^H [Cout][Cin] ahead of the grad_x chain, (c_ky / HW) X^H
    // [Cin][B] after it
    const float inv_hw = static_cast<float>(1.0 / (static_cast<double>(H) * W));
    // The TMA-ring mixing reads W^H and X^H straight from W and X (transposed tensor maps,
    // conjugated in the kernel, the per-ky scale in its epilogue); where it does not apply the
    // conjugate transposes run as separate passes.
    const float2* W1 = reinterpret_cast<const float2*>(weights1);
    const float2* W2 = reinterpret_cast<const float2*>(weights2);
    if (grad_x) {
        // grad_x = inv(G W^H)
        e = scx::launch_mix_ring_ct(G1, G2, W1, W2, Z1, Z2, 2, B, Cout, Cin, NM, 1, m2, W, inv_hw, s);
        if (e == cudaErrorNotSupported) {
            conj_transpose_kernel<<<dim3(blocks_for(static_cast<long long>(Cin) * Cout * NM), 2), kThreads, 0, s>>>(
                W1, W2, WH1, WH2, Cin, Cout, NM, 0, m2, W, inv_hw);
            e = cudaGetLastError();
            if (e == cudaSuccess) e = scx::launch_mix(G1, G2, WH1, WH2, Z1, Z2, 2, B, Cout, Cin, NM, s);
        }
        if (e == cudaSuccess) e = scx::dft_inv(Z1, Z2, NM, m2, grad_x, B * Cin, H, W, m1, m2, *tw, s, scratch, L.scratch);
        if (e != cudaSuccess) return e;
    }
    if (grad_w1) {
        // grad_W = ((c_ky / HW) X^H) G; X1 then X2 are contiguous at x_corners
        const float2* X1 = reinterpret_cast<const float2*>(x_corners);
        const float2* X2 = X1 + static_cast<size_t>(B) * Cin * NM;
        float2* gw1 = reinterpret_cast<float2*>(grad_w1);
        float2* gw2 = reinterpret_cast<float2*>(grad_w2);
        e = scx::launch_mix_ring_ct(X1, X2, G1, G2, gw1, gw2, 2, Cin, B, Cout, NM, 2, m2, W, inv_hw, s);
        if (e == cudaErrorNotSupported) {
            conj_transpose_kernel<<<dim3(blocks_for(static_cast<long long>(B) * Cin * NM), 2), kThreads, 0, s>>>(
                X1, X2, XH1, XH2, B, Cin, NM, 1, m2, W, inv_hw);
            e = cudaGetLastError();
            if (e == cudaSuccess) e = scx::launch_mix(XH1, XH2, G1, G2, gw1, gw2, 2, Cin, B, Cout, NM, s);
        }
    }
    return e;
}

// ---- backward of the single-corner mixing alone (SpectralMulFunction.backward,
// spectral_conv/spectral_conv_ops.py:272-278):
//   grad_x[b][i][k] = sum_o grad_y[b][o][k] conj(w[i][o][k])   = mix(grad_y, W^H)
//   grad_w[i][o][k] = sum_b conj(x[b][i][k]) grad_y[b][o][k]   = mix(X^H, grad_y)
// with W^H = [Cout][Cin] and X^H = [Cin][B] per mode (conj_transpose_kernel, one corner).

namespace {

struct MulBwdLayout {
    size_t wh, xh, total;
};

MulBwdLayout mul_bwd_layout(int B, int Cin, int Cout, int m1, int m2) {
    const size_t NM = static_cast<size_t>(m1) * m2;
    MulBwdLayout L;
    L.wh = a256(static_cast<size_t>(Cout) * Cin * NM * sizeof(float2));
    L.xh = a256(static_cast<size_t>(Cin) * B * NM * sizeof(float2));
    L.total = L.wh + L.xh;
    return L;
}

bool mul_bwd_valid(int B, int Cin, int Cout, int m1, int m2) {
    if (B <= 0 || Cin <= 0 || Cout <= 0 || m1 <= 0 || m2 <= 0) return false;
    const long long NM = static_cast<long long>(m1) * m2, lim = (1LL << 31) - 1;
    return NM * B * Cin * 2 <= lim && NM * B * Cout * 2 <= lim && NM * Cin * Cout * 2 <= lim;
}

}  // namespace

extern "C" size_t scx_spectral_mul_bwd_workspace_size(int batch_size, int channels_in, int channels_out, int modes1,
                                                      int modes2) {
    if (!mul_bwd_valid(batch_size, channels_in, channels_out, modes1, modes2)) return 0;
    return mul_bwd_layout(batch_size, channels_in, channels_out, modes1, modes2).total;
}

extern "C" int scx_spectral_mul_bwd(const float* x_freq, const float* weights, const float* grad_y, float* grad_x,
                                    float* grad_w, int batch_size, int channels_in, int channels_out, int modes1,
                                    int modes2, void* workspace, size_t workspace_bytes, scx_stream_t stream) {
    if (!grad_y || !workspace || (!grad_x && !grad_w)) return cudaErrorInvalidValue;
    if ((grad_x && !weights) || (grad_w && !x_freq)) return cudaErrorInvalidValue;
    const size_t need = scx_spectral_mul_bwd_workspace_size(batch_size, channels_in, channels_out, modes1, modes2);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    auto misaligned = [](const void* p, uintptr_t a) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) % a) != 0; };
    if (misaligned(x_freq, 8) || misaligned(weights, 8) || misaligned(grad_y, 8) || misaligned(grad_x, 8) ||
        misaligned(grad_w, 8) || misaligned(workspace, 256))
        return cudaErrorInvalidValue;
    const int B = batch_size, Cin = channels_in, Cout = channels_out, NM = modes1 * modes2;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const MulBwdLayout L = mul_bwd_layout(B, Cin, Cout, modes1, modes2);
    unsigned char* base = static_cast<unsigned char*>(workspace);
    float2* WH = reinterpret_cast<float2*>(base);
    float2* XH = reinterpret_cast<float2*>(base + L.wh);
    const float2* G = reinterpret_cast<const float2*>(grad_y);
    cudaError_t e = cudaSuccess;
    // as in scx_spectral_conv2d_bwd: W^H and X^H read in place by the TMA-ring mixing where it
    // applies (no scale: W = 0), else written by conjugate-transpose passes first
    if (grad_x) {
        const float2* Wc = reinterpret_cast<const float2*>(weights);
        float2* gx = reinterpret_cast<float2*>(grad_x);
        e = scx::launch_mix_ring_ct(G, G, Wc, Wc, gx, gx, 1, B, Cout, Cin, NM, 1, modes2, 0, 1.f, s);
        if (e == cudaErrorNotSupported) {
            conj_transpose_kernel<<<dim3(blocks_for(static_cast<long long>(Cin) * Cout * NM), 1), kThreads, 0, s>>>(
                Wc, nullptr, WH, nullptr, Cin, Cout, NM, 0, modes2, 2, 1.f);  // one corner: grid.y = 1
            e = cudaGetLastError();
            if (e == cudaSuccess) e = scx::launch_mix(G, nullptr, WH, nullptr, gx, nullptr, 1, B, Cout, Cin, NM, s);
        }
        if (e != cudaSuccess) return e;
    }
    if (grad_w) {
        const float2* Xc = reinterpret_cast<const float2*>(x_freq);
        float2* gw = reinterpret_cast<float2*>(grad_w);
        e = scx::launch_mix_ring_ct(Xc, Xc, G, G, gw, gw, 1, Cin, B, Cout, NM, 2, modes2, 0, 1.f, s);
        if (e == cudaErrorNotSupported) {
            conj_transpose_kernel<<<dim3(blocks_for(static_cast<long long>(B) * Cin * NM), 1), kThreads, 0, s>>>(
                Xc, nullptr, XH, nullptr, B, Cin, NM, 0, modes2, 2, 1.f);
            e = cudaGetLastError();
            if (e == cudaSuccess) e = scx::launch_mix(XH, nullptr, G, nullptr, gw, nullptr, 1, Cin, B, Cout, NM, s);
        }
    }
    return e;
}
