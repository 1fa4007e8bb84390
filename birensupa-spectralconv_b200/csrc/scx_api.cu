// extern "C" entry points of libscx.so (declared in include/scx.h).
// Argument validation mirrors the TORCH_CHECKs of spectral_conv/spectral_conv_ext.cpp:26-31,
// 123-245 and the launcher checks of spectral_conv_combo/spectral_conv_ext.su:98-101, but
// reports cudaErrorInvalidValue instead of throwing.
#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "scx.h"
#include "scx_internal.h"

namespace {

constexpr long long kMaxElems = (1LL << 31) - 1;

inline cudaStream_t as_stream(scx_stream_t s) { return static_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline bool fits(long long a, long long b, long long c = 1, long long d = 1, long long e = 1) {
    long long v = a;
    for (long long f : {b, c, d, e}) {
        if (f <= 0 || v > kMaxElems / f) return false;
        v *= f;
    }
    return v > 0 && v <= kMaxElems;
}

bool valid_shape(int B, int C, int H, int W, int m1, int m2) {
    if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || m1 <= 0 || m2 <= 0) return false;
    if (m1 > H || m2 > W / 2 + 1) return false;
    return fits(B, C, H, W) && fits(B, C, 2 * m1, m2, 2);
}

bool valid_mix(int B, int Cin, int Cout, int m1, int m2) {
    if (B <= 0 || Cin <= 0 || Cout <= 0 || m1 <= 0 || m2 <= 0) return false;
    return fits(B, Cin, m1, m2, 2) && fits(B, Cout, m1, m2, 2) && fits(Cin, Cout, m1, m2, 2);
}

bool ffma_forced() {
    const char* v = std::getenv("SCX_VARIANT");
    return v != nullptr && std::strcmp(v, "ffma") == 0;
}

}  // namespace

namespace scx {

cudaError_t dft_fwd(const float* x, float2* out1, float2* out2, long long out_plane_stride, int out_row_stride,
                    int P, int H, int W, int m1, int m2, const Twiddles& tw, cudaStream_t stream, float* scratch,
                    size_t scratch_bytes) {
    const int v = dft_variant(H, W, m1, m2);
    if (!ffma_forced() && v != kDftFfma) {
        if (v != kDftFolded && tc_fwd_supported(H, W, m1, m2) && (reinterpret_cast<uintptr_t>(x) & 15) == 0)
            return launch_dft_fwd_tc(x, out1, out2, out_plane_stride, out_row_stride, P, H, W, m1, m2, stream);
        if (tc_split_supported(H, W, m1, m2) && (reinterpret_cast<uintptr_t>(x) & 15) == 0)
            // the four parity sub-problems of every plane in one launch, folded in the kernel
            return launch_dft_fwd_tc_folded(x, out1, out2, out_plane_stride, out_row_stride, P, H, W, m1, m2,
                                            stream);
    }
    return launch_dft_fwd(x, out1, out2, out_plane_stride, out_row_stride, P, H, W, m1, m2, tw, stream);
}

cudaError_t dft_inv(const float2* in1, const float2* in2, long long in_plane_stride, int in_row_stride, float* y,
                    int Q, int H, int W, int m1, int m2, const Twiddles& tw, cudaStream_t stream, float* scratch,
                    size_t scratch_bytes) {
    const int v = dft_variant(H, W, m1, m2);
    if (!ffma_forced() && v != kDftFfma) {
        if (v != kDftFolded && tc_inv_supported(H, W, m1, m2) && (reinterpret_cast<uintptr_t>(y) & 3) == 0)
            return launch_dft_inv_tc(in1, in2, in_plane_stride, in_row_stride, y, Q, H, W, m1, m2, stream);
        if (v != kDftFolded && tc_quad_supported(H, W, m1, m2) && (reinterpret_cast<uintptr_t>(y) & 3) == 0)
            // four output quadrants per plane, straight from the corners (no fold, no scratch)
            return launch_dft_inv_tc_quad(in1, in2, in_plane_stride, in_row_stride, y, Q, H, W, m1, m2, stream);
        if (scratch != nullptr && tc_split_supported(H, W, m1, m2) && scratch_bytes >= split_scratch_bytes(Q, H, W) &&
            ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(scratch)) & 15) == 0) {
            // one tensor-core inverse per parity class of the spectrum into half-size
            // sub-planes, then unfold them into the quadrants of y
            const int Hs = H / 2, Ws = W / 2;
            cudaError_t e = cudaSuccess;
            for (int q = 0; q < 4 && e == cudaSuccess; ++q) {
                const TcSub sub{H, W, q >> 1, q & 1, m1, m2};
                const long long off = static_cast<long long>(sub.a) * in_row_stride + sub.b;
                e = launch_dft_inv_tc(in1 + off, in2 + off, in_plane_stride, 2 * in_row_stride,
                                      scratch + static_cast<size_t>(q) * Q * Hs * Ws, Q, Hs, Ws, m1 / 2, m2 / 2, stream,
                                      &sub);
            }
            if (e == cudaSuccess) e = launch_unfold(scratch, y, Q, Hs, Ws, stream);
            return e;
        }
    }
    return launch_dft_inv(in1, in2, in_plane_stride, in_row_stride, y, Q, H, W, m1, m2, tw, stream);
}

}  // namespace scx

extern "C" {

int scx_version(void) { return 100; }

int scx_watchdog(int reset) {
    int v = 0;
    const cudaError_t e = scx::read_watchdog(&v, reset != 0);
    return e == cudaSuccess ? v : -static_cast<int>(e);
}

const char* scx_status_string(int status) {
    return cudaGetErrorString(static_cast<cudaError_t>(status));
}

int scx_prepare(int H, int W, int modes1, int modes2) {
    if (!valid_shape(1, 1, H, W, modes1, modes2)) return cudaErrorInvalidValue;
    const scx::Twiddles* tw = nullptr;
    return scx::get_twiddles(H, W, modes1, modes2, &tw);
}

int scx_spectral_mul(const float* x_freq, const float* weights, float* y_freq, int batch_size,
                     int channels_in, int channels_out, int modes1, int modes2,
                     scx_stream_t stream) {
    if (!x_freq || !weights || !y_freq) return cudaErrorInvalidValue;
    if (!valid_mix(batch_size, channels_in, channels_out, modes1, modes2)) return cudaErrorInvalidValue;
    if (!aligned(x_freq, 8) || !aligned(weights, 8) || !aligned(y_freq, 8)) return cudaErrorInvalidValue;
    return scx::launch_mix(reinterpret_cast<const float2*>(x_freq), nullptr,
                           reinterpret_cast<const float2*>(weights), nullptr,
                           reinterpret_cast<float2*>(y_freq), nullptr, 1, batch_size, channels_in,
                           channels_out, modes1 * modes2, as_stream(stream));
}

int scx_spectral_mul_dual(const float* x1, const float* x2, const float* w1, const float* w2,
                          float* y1, float* y2, int batch_size, int channels_in,
                          int channels_out, int modes1, int modes2, scx_stream_t stream) {
    if (!x1 || !x2 || !w1 || !w2 || !y1 || !y2) return cudaErrorInvalidValue;
    if (!valid_mix(batch_size, channels_in, channels_out, modes1, modes2)) return cudaErrorInvalidValue;
    for (const void* p : {static_cast<const void*>(x1), static_cast<const void*>(x2),
                          static_cast<const void*>(w1), static_cast<const void*>(w2),
                          static_cast<const void*>(y1), static_cast<const void*>(y2)})
        if (!aligned(p, 8)) return cudaErrorInvalidValue;
    return scx::launch_mix(reinterpret_cast<const float2*>(x1), reinterpret_cast<const float2*>(x2),
                           reinterpret_cast<const float2*>(w1), reinterpret_cast<const float2*>(w2),
                           reinterpret_cast<float2*>(y1), reinterpret_cast<float2*>(y2), 2, batch_size,
                           channels_in, channels_out, modes1 * modes2, as_stream(stream));
}

int scx_rfft2_corners(const float* x, float* x1, float* x2, int batch_size, int channels,
                      int height, int width, int modes1, int modes2, scx_stream_t stream) {
    if (!x || !x1 || !x2) return cudaErrorInvalidValue;
    if (!valid_shape(batch_size, channels, height, width, modes1, modes2)) return cudaErrorInvalidValue;
    if (!aligned(x, 4) || !aligned(x1, 8) || !aligned(x2, 8)) return cudaErrorInvalidValue;
    const scx::Twiddles* tw = nullptr;
    cudaError_t e = scx::get_twiddles(height, width, modes1, modes2, &tw);
    if (e != cudaSuccess) return e;
    return scx::dft_fwd(x, reinterpret_cast<float2*>(x1), reinterpret_cast<float2*>(x2),
                        static_cast<long long>(modes1) * modes2, modes2, batch_size * channels, height, width,
                        modes1, modes2, *tw, as_stream(stream));
}

int scx_irfft2_corners(const float* y1, const float* y2, float* y, int batch_size, int channels,
                       int height, int width, int modes1, int modes2, scx_stream_t stream) {
    if (!y1 || !y2 || !y) return cudaErrorInvalidValue;
    if (!valid_shape(batch_size, channels, height, width, modes1, modes2)) return cudaErrorInvalidValue;
    if (!aligned(y, 4) || !aligned(y1, 8) || !aligned(y2, 8)) return cudaErrorInvalidValue;
    const scx::Twiddles* tw = nullptr;
    cudaError_t e = scx::get_twiddles(height, width, modes1, modes2, &tw);
    if (e != cudaSuccess) return e;
    return scx::dft_inv(reinterpret_cast<const float2*>(y1), reinterpret_cast<const float2*>(y2),
                        static_cast<long long>(modes1) * modes2, modes2, y, batch_size * channels, height, width,
                        modes1, modes2, *tw, as_stream(stream));
}

int scx_rfft2(const float* x, float* x_freq, int batch_size, int channels, int height, int width,
              scx_stream_t stream) {
    if (!x || !x_freq) return cudaErrorInvalidValue;
    const int wf = width / 2 + 1;
    const int m1 = (height + 1) / 2;
    if (!valid_shape(batch_size, channels, height, width, m1, wf)) return cudaErrorInvalidValue;
    if (!aligned(x, 4) || !aligned(x_freq, 8)) return cudaErrorInvalidValue;
    const scx::Twiddles* tw = nullptr;
    cudaError_t e = scx::get_twiddles(height, width, m1, wf, &tw);
    if (e != cudaSuccess) return e;
    // Corner 1 = rows [0, m1), corner 2 = rows [H-m1, H): together every row of the
    // spectrum (the middle row twice, with identical values, when H is odd).
    float2* out = reinterpret_cast<float2*>(x_freq);
    return scx::launch_dft_fwd(x, out, out + static_cast<size_t>(height - m1) * wf,
                               static_cast<long long>(height) * wf, wf, batch_size * channels, height,
                               width, m1, wf, *tw, as_stream(stream));
}

int scx_irfft2(const float* x_freq, float* y, int batch_size, int channels, int height, int width,
               scx_stream_t stream) {
    if (!x_freq || !y) return cudaErrorInvalidValue;
    const int wf = width / 2 + 1;
    const int m1 = (height + 1) / 2;
    if (!valid_shape(batch_size, channels, height, width, m1, wf)) return cudaErrorInvalidValue;
    if (!aligned(y, 4) || !aligned(x_freq, 8)) return cudaErrorInvalidValue;
    const scx::Twiddles* tw = nullptr;
    cudaError_t e = scx::get_twiddles(height, width, m1, wf, &tw);
    if (e != cudaSuccess) return e;
    const float2* in = reinterpret_cast<const float2*>(x_freq);
    return scx::launch_dft_inv(in, in + static_cast<size_t>(height - m1) * wf,
                               static_cast<long long>(height) * wf, wf, y, batch_size * channels, height,
                               width, m1, wf, *tw, as_stream(stream));
}

size_t scx_spectral_conv2d_workspace_size(int batch_size, int channels_in, int channels_out,
                                          int height, int width, int modes1, int modes2) {
    if (!valid_shape(batch_size, channels_in, height, width, modes1, modes2) ||
        !valid_shape(batch_size, channels_out, height, width, modes1, modes2))
        return 0;
    const size_t corner_in = static_cast<size_t>(batch_size) * channels_in * modes1 * modes2;
    const size_t corner_out = static_cast<size_t>(batch_size) * channels_out * modes1 * modes2;
    size_t bytes = 2 * (corner_in + corner_out) * sizeof(float2);
    // folded tensor-core path: one set of planes of the larger side, after the spectra
    if (scx::tc_split_supported(height, width, modes1, modes2))
        bytes += scx::split_scratch_bytes(static_cast<long long>(batch_size) * std::max(channels_in, channels_out),
                                          height, width);
    return bytes;
}

int scx_spectral_conv2d_fwd(const float* x, const float* weights1, const float* weights2, float* y,
                            int batch_size, int channels_in, int channels_out, int height, int width,
                            int modes1, int modes2, void* workspace, size_t workspace_bytes,
                            scx_stream_t stream) {
    if (!x || !weights1 || !weights2 || !y || !workspace) return cudaErrorInvalidValue;
    const size_t need = scx_spectral_conv2d_workspace_size(batch_size, channels_in, channels_out, height,
                                                           width, modes1, modes2);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    if (!valid_mix(batch_size, channels_in, channels_out, modes1, modes2)) return cudaErrorInvalidValue;
    if (!aligned(x, 4) || !aligned(y, 4) || !aligned(weights1, 8) || !aligned(weights2, 8) ||
        !aligned(workspace, 16))
        return cudaErrorInvalidValue;
    const scx::Twiddles* tw = nullptr;
    cudaError_t e = scx::get_twiddles(height, width, modes1, modes2, &tw);
    if (e != cudaSuccess) return e;
    const cudaStream_t s = as_stream(stream);
    const size_t ci = static_cast<size_t>(batch_size) * channels_in * modes1 * modes2;
    const size_t co = static_cast<size_t>(batch_size) * channels_out * modes1 * modes2;
    float2* X1 = static_cast<float2*>(workspace);
    float2* X2 = X1 + ci;
    float2* Y1 = X2 + ci;
    float2* Y2 = Y1 + co;
    const long long NM = static_cast<long long>(modes1) * modes2;
    float* scratch = reinterpret_cast<float*>(Y2 + co);  // present when the folded path applies
    const size_t scratch_bytes = need - 2 * (ci + co) * sizeof(float2);
    e = scx::dft_fwd(x, X1, X2, NM, modes2, batch_size * channels_in, height, width, modes1, modes2, *tw, s,
                     scratch_bytes ? scratch : nullptr, scratch_bytes);
    if (e != cudaSuccess) return e;
    // the weights are not written by the forward DFT it follows
    e = scx::launch_mix(X1, X2, reinterpret_cast<const float2*>(weights1),
                        reinterpret_cast<const float2*>(weights2), Y1, Y2, 2, batch_size, channels_in,
                        channels_out, static_cast<int>(NM), s, true);
    if (e != cudaSuccess) return e;
    return scx::dft_inv(Y1, Y2, NM, modes2, y, batch_size * channels_out, height, width, modes1, modes2, *tw, s,
                        scratch_bytes ? scratch : nullptr, scratch_bytes);
}

}  // extern "C"
