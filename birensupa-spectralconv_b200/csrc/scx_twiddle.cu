// Twiddle-table cache: the B200 replacement for the suFFT plan / work-area cache of
// spectral_conv/spectral_conv_ext.cpp:51-121.  Instead of FFT plans, every shape gets
// four small truncated DFT matrices, computed on the host in double precision with the
// angle reduced exactly in integers ((k*n) mod N) and rounded once to fp32.
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "scx_internal.h"

namespace scx {
namespace {

struct Key {
    int dev, H, W, m1, m2;
    bool operator<(const Key& o) const {
        return std::tie(dev, H, W, m1, m2) < std::tie(o.dev, o.H, o.W, o.m1, o.m2);
    }
};

std::mutex g_mutex;
std::map<Key, Twiddles> g_cache;
std::map<int, int> g_sms;

inline double angle(long long k, long long n, long long N) {
    // 2*pi*((k*n) mod N)/N, reduced exactly before the multiply.
    long long r = (k * n) % N;
    return 2.0 * M_PI * static_cast<double>(r) / static_cast<double>(N);
}

// Spectrum row held by corner slot s (s < m1: corner 1, else corner 2).
inline int slot_row(int s, int H, int m1) { return s < m1 ? s : H - m1 + (s - m1); }

}  // namespace

int num_sms() {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_sms.find(dev);
    if (it != g_sms.end()) return it->second;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        n = 148;
    g_sms[dev] = n;
    return n;
}

cudaError_t launch_chained_raw(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                               void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, kernel, args);
}

cudaError_t prepare_kernel(const void* kernel, size_t bytes, int threads, int* blocks_per_sm) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    static std::mutex m;
    static std::map<std::tuple<int, const void*, size_t, int>, int> seen;
    // The shared-memory limit is one value per (device, kernel): only ever raise it, or a
    // later smaller request would lower it under a launch that needs more.
    static std::map<std::pair<int, const void*>, size_t> limit;
    std::lock_guard<std::mutex> lock(m);
    const auto key = std::make_tuple(dev, kernel, bytes, threads);
    auto it = seen.find(key);
    if (it != seen.end()) {
        *blocks_per_sm = it->second;
        return cudaSuccess;
    }
    size_t& cur = limit[std::make_pair(dev, kernel)];
    if (bytes > 48 * 1024 && bytes > cur) {
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
        if (err != cudaSuccess) return err;
        // prefer the largest shared-memory carveout so that occupancy is limited by the
        // kernel's own needs, not by the default L1/shared split
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                   static_cast<int>(cudaSharedmemCarveoutMaxShared));
        if (err != cudaSuccess) return err;
        cur = bytes;
    }
    int n = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, bytes);
    if (err != cudaSuccess) return err;
    if (n < 1) return cudaErrorInvalidConfiguration;
    seen[key] = n;
    *blocks_per_sm = n;
    return cudaSuccess;
}

// The watchdog word: one per device, zero when the module is loaded.  It is a static device
// variable rather than an allocation, so that finding it needs no cudaMalloc and no copy
// (the allocation-free entry point reaches it too).  In host code the name only stands for
// the symbol: the device address comes from cudaGetSymbolAddress.
static __device__ int g_watchdog_word = 0;

cudaError_t device_watchdog(int** out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    static std::mutex m;
    static std::map<int, int*> words;
    std::lock_guard<std::mutex> lock(m);
    auto it = words.find(dev);
    if (it != words.end()) {
        *out = it->second;
        return cudaSuccess;
    }
    void* w = nullptr;
    err = cudaGetSymbolAddress(&w, g_watchdog_word);
    if (err != cudaSuccess) return err;
    if (w == nullptr) return cudaErrorInvalidSymbol;
    words[dev] = static_cast<int*>(w);
    *out = static_cast<int*>(w);
    return cudaSuccess;
}

cudaError_t read_watchdog(int* value, bool reset) {
    int* w = nullptr;
    cudaError_t e = device_watchdog(&w);
    if (e != cudaSuccess) return e;
    e = cudaMemcpy(value, w, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess || !reset) return e;
    const int zero = 0;
    return cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice);
}

cudaError_t get_twiddles(int H, int W, int m1, int m2, const Twiddles** out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    const Key key{dev, H, W, m1, m2};
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_cache.find(key);
    if (it != g_cache.end()) {
        *out = &it->second;
        return cudaSuccess;
    }
    const size_t n_row_fwd = static_cast<size_t>(W) * m2;
    const size_t n_col_fwd = static_cast<size_t>(2 * m1) * H;
    const size_t n_col_inv = static_cast<size_t>(H) * (2 * m1);
    const size_t n_row_inv = static_cast<size_t>(m2) * W;
    std::vector<float2> host(n_row_fwd + n_col_fwd + n_col_inv + n_row_inv);
    float2* row_fwd = host.data();
    float2* col_fwd = row_fwd + n_row_fwd;
    float2* col_inv = col_fwd + n_col_fwd;
    float2* row_inv = col_inv + n_col_inv;

    for (int w = 0; w < W; ++w)
        for (int ky = 0; ky < m2; ++ky) {
            const double a = angle(ky, w, W);
            row_fwd[static_cast<size_t>(w) * m2 + ky] =
                make_float2(static_cast<float>(std::cos(a)), static_cast<float>(-std::sin(a)));
        }
    for (int s = 0; s < 2 * m1; ++s) {
        const int kx = slot_row(s, H, m1);
        for (int h = 0; h < H; ++h) {
            const double a = angle(kx, h, H);
            col_fwd[static_cast<size_t>(s) * H + h] =
                make_float2(static_cast<float>(std::cos(a)), static_cast<float>(-std::sin(a)));
        }
    }
    for (int h = 0; h < H; ++h)
        for (int s = 0; s < 2 * m1; ++s) {
            const int kx = slot_row(s, H, m1);
            // A corner-1 row that corner 2 also covers is overwritten in the reference
            // (spectral_conv/reference_pytorch.py:44-46): it contributes nothing.
            const bool dropped = (s < m1) && (kx >= H - m1);
            const double a = angle(kx, h, H);
            col_inv[static_cast<size_t>(h) * (2 * m1) + s] =
                dropped ? make_float2(0.f, 0.f)
                        : make_float2(static_cast<float>(std::cos(a)), static_cast<float>(std::sin(a)));
        }
    // C2R along W: bin 0 and (W even) bin W/2 count once, every other bin twice; only the
    // real part of Z*exp(+i*theta) survives, which also drops Im of the DC/Nyquist bins.
    const double inv_hw = 1.0 / (static_cast<double>(H) * static_cast<double>(W));
    for (int ky = 0; ky < m2; ++ky) {
        const bool single = (ky == 0) || ((W % 2 == 0) && (ky == W / 2));
        const double c = (single ? 1.0 : 2.0) * inv_hw;
        for (int w = 0; w < W; ++w) {
            const double a = angle(ky, w, W);
            row_inv[static_cast<size_t>(ky) * W + w] =
                make_float2(static_cast<float>(c * std::cos(a)), static_cast<float>(c * std::sin(a)));
        }
    }

    float2* dev_buf = nullptr;
    err = cudaMalloc(&dev_buf, host.size() * sizeof(float2));
    if (err != cudaSuccess) return err;
    err = cudaMemcpy(dev_buf, host.data(), host.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        cudaFree(dev_buf);
        return err;
    }
    Twiddles t;
    t.H = H;
    t.W = W;
    t.m1 = m1;
    t.m2 = m2;
    t.row_fwd = dev_buf;
    t.col_fwd = dev_buf + n_row_fwd;
    t.col_inv = dev_buf + n_row_fwd + n_col_fwd;
    t.row_inv = dev_buf + n_row_fwd + n_col_fwd + n_col_inv;
    auto res = g_cache.emplace(key, t);
    *out = &res.first->second;
    return cudaSuccess;
}

}  // namespace scx
