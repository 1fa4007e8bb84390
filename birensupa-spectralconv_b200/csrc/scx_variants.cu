// Per-shape kernel-variant table: the device-side half of the B200 counterpart of the
// reference's tuning table (_AUTO_TUNE_TABLE, spectral_conv_combo/spectral_conv_ops.py:45-63,
// written by spectral_conv_combo/tune.py:154-261, which the reference never reads back).
// Here a host-side tuner (scx_tune.py) measures the variants that apply to a shape, and the
// winners are set through the entry points below, process-wide for every device; the
// dispatch in scx_api.cu (truncated DFTs) and scx_mix.cu (mixing) consults them.
#include <map>
#include <mutex>
#include <tuple>

#include "scx.h"
#include "scx_internal.h"

namespace scx {
namespace {

std::mutex g_mutex;
std::map<std::tuple<int, int, int, int>, int> g_dft;
std::map<std::tuple<int, int, int, int, int>, int> g_mix;

}  // namespace

int dft_variant(int H, int W, int m1, int m2) {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_dft.find(std::make_tuple(H, W, m1, m2));
    return it == g_dft.end() ? kDftAuto : it->second;
}

int mix_variant(int ncorner, int B, int Cin, int Cout, int NM) {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_mix.find(std::make_tuple(ncorner, B, Cin, Cout, NM));
    return it == g_mix.end() ? kMixAuto : it->second;
}

}  // namespace scx

extern "C" {

int scx_dft_variants(int H, int W, int modes1, int modes2) {
    if (H <= 0 || W <= 0 || modes1 <= 0 || modes2 <= 0 || modes1 > H || modes2 > W / 2 + 1) return 0;
    int mask = 1 << scx::kDftFfma;
    if (scx::tc_fwd_supported(H, W, modes1, modes2) && scx::tc_inv_supported(H, W, modes1, modes2))
        mask |= 1 << scx::kDftTensor;
    if (scx::tc_split_supported(H, W, modes1, modes2)) mask |= 1 << scx::kDftFolded;
    return mask;
}

int scx_set_dft_variant(int H, int W, int modes1, int modes2, int variant) {
    if (variant < scx::kDftAuto || variant > scx::kDftFolded) return cudaErrorInvalidValue;
    if (variant != scx::kDftAuto && !(scx_dft_variants(H, W, modes1, modes2) & (1 << variant)))
        return cudaErrorInvalidValue;
    std::lock_guard<std::mutex> lock(scx::g_mutex);
    const auto key = std::make_tuple(H, W, modes1, modes2);
    if (variant == scx::kDftAuto)
        scx::g_dft.erase(key);
    else
        scx::g_dft[key] = variant;
    return cudaSuccess;
}

int scx_set_mix_variant(int ncorner, int batch_size, int channels_in, int channels_out, int modes, int variant) {
    if (ncorner < 1 || ncorner > 2 || batch_size <= 0 || channels_in <= 0 || channels_out <= 0 || modes <= 0)
        return cudaErrorInvalidValue;
    if (variant < scx::kMixAuto || variant > scx::kMixTc) return cudaErrorInvalidValue;
    std::lock_guard<std::mutex> lock(scx::g_mutex);
    const auto key = std::make_tuple(ncorner, batch_size, channels_in, channels_out, modes);
    if (variant == scx::kMixAuto)
        scx::g_mix.erase(key);
    else
        scx::g_mix[key] = variant;
    return cudaSuccess;
}

int scx_get_variant(int kind, int a, int b, int c, int d, int e) {
    if (kind == 0) return scx::dft_variant(a, b, c, d);
    if (kind == 1) return scx::mix_variant(a, b, c, d, e);
    return -2;
}

void scx_clear_variants(void) {
    std::lock_guard<std::mutex> lock(scx::g_mutex);
    scx::g_dft.clear();
    scx::g_mix.clear();
}

}  // extern "C"
