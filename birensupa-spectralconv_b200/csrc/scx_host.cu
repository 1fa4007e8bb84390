// Host-buffer SpectralConv2d forward: scx_spectral_conv2d_fwd_host.
//
// The reference's host-facing call (spectral_conv2d_supa with a CPU tensor,
// spectral_conv/spectral_conv_ops.py:480-505) uploads the whole batch, runs the forward and
// downloads the result one after the other.  Here the batch is cut into chunks and three
// streams overlap them: the upload of chunk i + 1 (copy stream `up`), the forward of chunk i
// (the caller's stream) and the download of chunk i - 1 (copy stream `down`), so both PCIe
// directions are busy at once.  The first upload and the last download have nothing to
// overlap with, so the first and last chunks are half the size of the others.  One
// cudaMemcpyAsync per chunk and direction; the streams are ordered through events.
#include <algorithm>
#include <mutex>

#include "scx.h"
#include "scx_internal.h"

namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxChunks = 32;
constexpr int kDefaultChunks = 6;

// Per-device copy streams and events.  A call holds `m` until its downloads have completed,
// so the events are never re-recorded while a wait on them is pending.
struct HostPipe {
    std::mutex m;
    bool ready = false;
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t start = nullptr, done = nullptr;
    cudaEvent_t uploaded[kMaxChunks] = {}, computed[kMaxChunks] = {};
};

HostPipe g_pipes[kMaxDevices];

// Creates the device's streams and events on first use (the device is current); called with
// the pipe's mutex held.
cudaError_t init_pipe(HostPipe& p) {
    if (p.ready) return cudaSuccess;
    cudaError_t e = cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.done, cudaEventDisableTiming);
    for (int i = 0; i < kMaxChunks && e == cudaSuccess; ++i) {
        e = cudaEventCreateWithFlags(&p.uploaded[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.computed[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) p.ready = true;
    return e;
}

// Batch offset of chunk boundary i of n: chunk weights 1, 2, ..., 2, 1 (n >= 3), equal
// otherwise; consecutive boundaries may coincide when n is close to B (empty chunks are
// skipped by the caller).
int chunk_start(int B, int n, int i) {
    if (n < 3) return static_cast<int>(static_cast<long long>(B) * i / n);
    const long long total = 2LL * (n - 1);  // 1 + 2 (n - 2) + 1
    const long long cum = i == 0 ? 0 : (i == n ? total : 2LL * i - 1);
    return static_cast<int>((B * cum + total / 2) / total);
}

}  // namespace

extern "C" int scx_spectral_conv2d_fwd_host(const float* x_host, const float* weights1, const float* weights2,
                                            float* y_host, int batch_size, int channels_in, int channels_out,
                                            int height, int width, int modes1, int modes2, float* x_dev,
                                            float* y_dev, void* workspace, size_t workspace_bytes, int chunks,
                                            scx_stream_t stream) {
    if (!x_host || !y_host || !x_dev || !y_dev || !weights1 || !weights2 || !workspace || chunks < 0)
        return cudaErrorInvalidValue;
    // shape, weight and workspace checks of the device call, once for the whole batch
    const size_t need = scx_spectral_conv2d_workspace_size(batch_size, channels_in, channels_out, height, width,
                                                           modes1, modes2);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    HostPipe& p = g_pipes[dev];
    std::lock_guard<std::mutex> lock(p.m);
    e = init_pipe(p);
    if (e != cudaSuccess) return e;

    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int n = std::min(std::min(chunks == 0 ? kDefaultChunks : chunks, batch_size), kMaxChunks);
    const size_t plane = static_cast<size_t>(height) * width;
    const size_t in_per = static_cast<size_t>(channels_in) * plane;    // floats per batch item
    const size_t out_per = static_cast<size_t>(channels_out) * plane;
    // the device buffers may still be in use by earlier work on the caller's stream
    e = cudaEventRecord(p.start, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p.up, p.start, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p.down, p.start, 0);
    for (int i = 0; i < n && e == cudaSuccess; ++i) {
        const int b0 = chunk_start(batch_size, n, i), b1 = chunk_start(batch_size, n, i + 1);
        if (b1 <= b0) continue;
        const size_t nb = static_cast<size_t>(b1 - b0);
        e = cudaMemcpyAsync(x_dev + b0 * in_per, x_host + b0 * in_per, nb * in_per * sizeof(float),
                            cudaMemcpyHostToDevice, p.up);
        if (e == cudaSuccess) e = cudaEventRecord(p.uploaded[i], p.up);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, p.uploaded[i], 0);
        if (e == cudaSuccess)
            e = static_cast<cudaError_t>(scx_spectral_conv2d_fwd(
                x_dev + b0 * in_per, weights1, weights2, y_dev + b0 * out_per, static_cast<int>(nb), channels_in,
                channels_out, height, width, modes1, modes2, workspace, workspace_bytes, stream));
        if (e == cudaSuccess) e = cudaEventRecord(p.computed[i], s);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p.down, p.computed[i], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(y_host + b0 * out_per, y_dev + b0 * out_per, nb * out_per * sizeof(float),
                                cudaMemcpyDeviceToHost, p.down);
    }
    // whatever was enqueued (uploads included, after an error) finishes before the call
    // returns and before later work on the caller's stream (which may reuse the device buffers)
    cudaError_t e2 = cudaEventRecord(p.start, p.up);
    if (e2 == cudaSuccess) e2 = cudaStreamWaitEvent(p.down, p.start, 0);
    if (e2 == cudaSuccess) e2 = cudaEventRecord(p.done, p.down);
    if (e2 == cudaSuccess) e2 = cudaStreamWaitEvent(s, p.done, 0);
    if (e2 == cudaSuccess) e2 = cudaEventSynchronize(p.done);
    return e != cudaSuccess ? e : e2;
}
