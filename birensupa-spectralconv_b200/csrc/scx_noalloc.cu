// Allocation-free SpectralConv2d forward: scx_spectral_conv2d_fwd_noalloc.
//
// Who needs this: callers that cannot (or must not) call cudaMalloc from inside the
// library.  Typical cases are processes whose memory pool or arena has already reserved
// the GPU's memory up front, where a stray allocation from a library would fail or
// fragment that pool, and latency-critical loops where an allocation's implicit device
// synchronisation is not acceptable.  The regular entry point needs both a caller
// workspace and the library's twiddle cache, and that cache is filled by cudaMalloc on the
// first call for each shape.
//
// This variant keeps every intermediate in one fixed, file-scope device array instead:
// the two corner spectra in, the two corner spectra out, and the four truncated DFT
// twiddle tables (recomputed on the device for every call).  The array is
// SCX_NOALLOC_SCRATCH_BYTES (16 MiB) large and every GPU that loads libscx.so keeps it
// until the process exits.  The caller still passes x, the weights and y.
//
// Rules of use:
// * The first call on a device looks up the array's device address with
//   cudaGetSymbolAddress (with that device current) and caches it per device; make that
//   first call before any stream capture.  The cache does not survive a cudaDeviceReset.
// * The mixing kernel's bounded waits report to the library's watchdog word, which is a
//   static device variable as well (no allocation); after a call whose result matters, read
//   scx_watchdog() once the stream has been synchronised.
// * The truncated DFTs use the FFMA kernels: the tensor-core kernels need operand tables
//   that the library allocates, so this path is slower on the shapes those kernels cover.
// * All calls share the array.  Calls that may overlap on the GPU (different streams,
//   different host threads without ordering) race on it and corrupt each other's results;
//   order them on one stream.
// * Nothing in the array has to start at zero: each call rewrites the twiddles and both
//   spectra before any kernel reads them, so the previous call's leftovers never leak.
// * Shapes whose scratch need exceeds the array are refused with cudaErrorMemoryAllocation
//   before anything is launched.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "scx.h"
#include "scx_internal.h"

namespace {

constexpr size_t kScratchBytes = SCX_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The fixed scratch.  In host code this name is only a stand-in for the symbol, never a
// usable device address: host code must use the pointer cudaGetSymbolAddress returns.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

inline size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

// Device address of the scratch on the current device (looked up once per device).
cudaError_t scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        if (p == nullptr) return cudaErrorInvalidSymbol;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

// Fills the four twiddle tables with the same definitions the host-built cache uses
// (scx_twiddle.cu), in double precision on the device: the angle 2*pi*((k*n) mod N)/N is
// reduced exactly in integers and evaluated with sincospi(2*r/N).
__global__ void fill_twiddles_kernel(float2* row_fwd, float2* col_fwd, float2* col_inv, float2* row_inv, int H,
                                     int W, int m1, int m2) {
    const long long n_row = static_cast<long long>(W) * m2;
    const long long n_col = static_cast<long long>(2 * m1) * H;
    const long long total = 2 * n_row + 2 * n_col;
    const double inv_hw = 1.0 / (static_cast<double>(H) * static_cast<double>(W));
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        double s, c;
        if (i < n_row) {  // row_fwd[w][ky] = (cos, -sin)(2 pi ky w / W)
            const int w = static_cast<int>(i / m2), ky = static_cast<int>(i % m2);
            sincospi(2.0 * static_cast<double>((static_cast<long long>(ky) * w) % W) / W, &s, &c);
            row_fwd[i] = make_float2(static_cast<float>(c), static_cast<float>(-s));
        } else if (i < n_row + n_col) {  // col_fwd[slot][h] = exp(-2 pi i kx h / H)
            const long long j = i - n_row;
            const int slot = static_cast<int>(j / H), h = static_cast<int>(j % H);
            const int kx = slot < m1 ? slot : H - m1 + (slot - m1);
            sincospi(2.0 * static_cast<double>((static_cast<long long>(kx) * h) % H) / H, &s, &c);
            col_fwd[j] = make_float2(static_cast<float>(c), static_cast<float>(-s));
        } else if (i < n_row + 2 * n_col) {  // col_inv[h][slot] = exp(+2 pi i kx h / H), 0 if overwritten
            const long long j = i - n_row - n_col;
            const int h = static_cast<int>(j / (2 * m1)), slot = static_cast<int>(j % (2 * m1));
            const int kx = slot < m1 ? slot : H - m1 + (slot - m1);
            const bool dropped = (slot < m1) && (kx >= H - m1);
            sincospi(2.0 * static_cast<double>((static_cast<long long>(kx) * h) % H) / H, &s, &c);
            col_inv[j] = dropped ? make_float2(0.f, 0.f) : make_float2(static_cast<float>(c), static_cast<float>(s));
        } else {  // row_inv[ky][w] = c_ky/(HW) (cos, sin)(2 pi ky w / W)
            const long long j = i - n_row - 2 * n_col;
            const int ky = static_cast<int>(j / W), w = static_cast<int>(j % W);
            const bool single = (ky == 0) || ((W % 2 == 0) && (ky == W / 2));
            const double scale = (single ? 1.0 : 2.0) * inv_hw;
            sincospi(2.0 * static_cast<double>((static_cast<long long>(ky) * w) % W) / W, &s, &c);
            row_inv[j] = make_float2(static_cast<float>(scale * c), static_cast<float>(scale * s));
        }
    }
}

inline bool is_aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace

extern "C" int scx_spectral_conv2d_fwd_noalloc(const float* x, const float* weights1, const float* weights2,
                                               float* y, int batch_size, int channels_in, int channels_out,
                                               int height, int width, int modes1, int modes2,
                                               scx_stream_t stream) {
    if (!x || !weights1 || !weights2 || !y) return cudaErrorInvalidValue;
    // Same shape rules as scx_spectral_conv2d_fwd (its workspace query validates them).
    const size_t spectra = scx_spectral_conv2d_workspace_size(batch_size, channels_in, channels_out, height,
                                                              width, modes1, modes2);
    if (spectra == 0) return cudaErrorInvalidValue;
    const long long n_weights = static_cast<long long>(channels_in) * channels_out * modes1 * modes2 * 2;
    if (n_weights <= 0 || n_weights >= (1LL << 31)) return cudaErrorInvalidValue;
    if (!is_aligned(x, 4) || !is_aligned(y, 4) || !is_aligned(weights1, 8) || !is_aligned(weights2, 8))
        return cudaErrorInvalidValue;
    const size_t ci = static_cast<size_t>(batch_size) * channels_in * modes1 * modes2;
    const size_t co = static_cast<size_t>(batch_size) * channels_out * modes1 * modes2;
    const size_t n_row = static_cast<size_t>(width) * modes2;
    const size_t n_col = static_cast<size_t>(2 * modes1) * height;
    // layout: X1 | X2 | Y1 | Y2 | row_fwd | col_fwd | col_inv | row_inv, each 256-byte aligned
    size_t off[9];
    off[0] = 0;
    const size_t sizes[8] = {ci * 8, ci * 8, co * 8, co * 8, n_row * 8, n_col * 8, n_col * 8, n_row * 8};
    for (int i = 0; i < 8; ++i) off[i + 1] = off[i] + align256(sizes[i]);
    if (off[8] > kScratchBytes) return cudaErrorMemoryAllocation;  // does not fit the fixed scratch

    void* base = nullptr;
    cudaError_t e = scratch_for_current_device(&base);
    if (e != cudaSuccess) return e;
    unsigned char* b = static_cast<unsigned char*>(base);
    float2* X1 = reinterpret_cast<float2*>(b + off[0]);
    float2* X2 = reinterpret_cast<float2*>(b + off[1]);
    float2* Y1 = reinterpret_cast<float2*>(b + off[2]);
    float2* Y2 = reinterpret_cast<float2*>(b + off[3]);
    scx::Twiddles tw;
    tw.H = height;
    tw.W = width;
    tw.m1 = modes1;
    tw.m2 = modes2;
    tw.row_fwd = reinterpret_cast<const float2*>(b + off[4]);
    tw.col_fwd = reinterpret_cast<const float2*>(b + off[5]);
    tw.col_inv = reinterpret_cast<const float2*>(b + off[6]);
    tw.row_inv = reinterpret_cast<const float2*>(b + off[7]);

    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const long long total = 2LL * static_cast<long long>(n_row + n_col);
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<long long>((total + threads - 1) / threads, 4096));
    fill_twiddles_kernel<<<blocks, threads, 0, s>>>(reinterpret_cast<float2*>(b + off[4]),
                                                    reinterpret_cast<float2*>(b + off[5]),
                                                    reinterpret_cast<float2*>(b + off[6]),
                                                    reinterpret_cast<float2*>(b + off[7]), height, width, modes1,
                                                    modes2);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const long long NM = static_cast<long long>(modes1) * modes2;
    e = scx::launch_dft_fwd(x, X1, X2, NM, modes2, batch_size * channels_in, height, width, modes1, modes2, tw, s);
    if (e != cudaSuccess) return e;
    e = scx::launch_mix(X1, X2, reinterpret_cast<const float2*>(weights1), reinterpret_cast<const float2*>(weights2),
                        Y1, Y2, 2, batch_size, channels_in, channels_out, static_cast<int>(NM), s);
    if (e != cudaSuccess) return e;
    return scx::launch_dft_inv(Y1, Y2, NM, modes2, y, batch_size * channels_out, height, width, modes1, modes2, tw,
                               s);
}
