// Internal declarations shared by the sm_100a kernels and the C-ABI layer.
//
// Data layout in HBM (all fp32, complex values interleaved re/im = float2):
//   x            [P = B*Cin ][H][W]          real input planes
//   corner spec  [B][C][m1][m2] float2        one array per corner, the layout of
//                                             spectral_conv/spectral_conv_ext.cpp:26-31
//   weights      [Cin][Cout][m1][m2] float2   view_as_real of the complex64 Parameter
//   y            [Q = B*Cout][H][W]          real output planes
//
// Corner 1 holds spectrum rows kx in [0, m1), corner 2 rows kx in [H-m1, H), both for
// ky in [0, m2) (spectral_conv/reference_pytorch.py:41-46).  When 2*m1 > H the rows
// overlap and corner 2 wins on the inverse side, exactly as the second slice
// assignment in the reference overwrites the first.
#pragma once

#include <utility>

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace scx {

// Host-built (double precision) twiddle tables for one (H, W, m1, m2) shape, resident on
// one device.  Owned by a process-wide cache; never freed before process exit.
struct Twiddles {
    int H, W, m1, m2;
    const float2* row_fwd;  // [W][m2]    (cos, -sin)(2 pi ky w / W)
    const float2* col_fwd;  // [2*m1][H]  exp(-2 pi i kx(slot) h / H)
    const float2* col_inv;  // [H][2*m1]  exp(+2 pi i kx(slot) h / H); 0 where corner 2 overwrites
    const float2* row_inv;  // [m2][W]    c_ky/(H*W) * (cos, sin)(2 pi ky w / W)
};

// Returns the cached tables for the current device, building them on first use
// (one cudaMalloc + one cudaMemcpy, so the first call must not happen inside stream
// capture).  Thread-safe.
cudaError_t get_twiddles(int H, int W, int m1, int m2, const Twiddles** out);

// Number of SMs of the current device (cached per device).
int num_sms();

// Raises a kernel's dynamic shared-memory limit to at least `bytes` on the current device
// (once per kernel/device/size: later launches, e.g. inside stream capture, make no call)
// and returns how many blocks of `threads` threads fit on one SM.
cudaError_t prepare_kernel(const void* kernel, size_t bytes, int threads, int* blocks_per_sm);

// Launches `kernel` with programmatic stream serialization: its CTAs may start (and run their
// prologue) while the previous kernel in the stream finishes; the kernel must execute
// griddepcontrol.wait in every CTA before it reads what earlier work wrote.
template <typename... Params, typename... Args>
cudaError_t launch_chained(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           Args&&... args) {
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
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same for a kernel known by address, with its arguments as an array of pointers.
cudaError_t launch_chained_raw(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                               void** args);

// ---- kernel launchers (no argument validation here; the C-ABI layer validates) ----

// Truncated forward real DFT of P planes, writing the two corner spectra.
// Output element (plane p, corner row j, ky) lives at
//   out_c + p*out_plane_stride + j*out_row_stride + ky.
cudaError_t launch_dft_fwd(const float* x, float2* out1, float2* out2,
                           long long out_plane_stride, int out_row_stride,
                           int P, int H, int W, int m1, int m2,
                           const Twiddles& tw, cudaStream_t stream);

// Zero-padded inverse real DFT of Q planes from the two corner spectra (corner 2
// overwrites corner 1 where the rows overlap).  Input element (plane q, row j, ky) at
//   in_c + q*in_plane_stride + j*in_row_stride + ky.
cudaError_t launch_dft_inv(const float2* in1, const float2* in2,
                           long long in_plane_stride, int in_row_stride,
                           float* y, int Q, int H, int W, int m1, int m2,
                           const Twiddles& tw, cudaStream_t stream);

// A parity sub-problem of a folded plane.  A plane of Hp x Wp = 2H x 2W samples is folded
// into four H x W planes q = 2a + b, sum over quadrants (alpha, beta) of
// (-1)^(a alpha + b beta) x[h + H alpha][w + W beta]; the spectrum of sub-plane q against
// the period-Hp / period-Wp twiddles is the full spectrum at the rows kx = a (mod 2) and the
// columns ky = b (mod 2).  A sub-problem's m1 slots per corner are the full corner rows
// 2t + a (t < m1_full / 2), and its m2 columns are ky = 2j + b.
struct TcSub {
    int period_h, period_w, a, b, m1_full, m2_full;
};

// Full-spectrum row of sub-problem slot s (m1s slots per corner).
inline int sub_row(const TcSub& sp, int s, int m1s) {
    const int corner = s < m1s ? 0 : 1, r = 2 * (s - corner * m1s) + sp.a;
    return corner == 0 ? r : sp.period_h - sp.m1_full + r;
}

// Tensor-core (tcgen05) truncated DFT kernels for the shapes tc_fwd_supported /
// tc_inv_supported accept.  Their operand tables are built per shape on first use
// (cudaMalloc + synchronous copy, so the first call must not happen inside stream capture).
bool tc_fwd_supported(int H, int W, int m1, int m2);
bool tc_inv_supported(int H, int W, int m1, int m2);
// With `sub`, the kernels run one parity sub-problem of folded planes: H, W, m1, m2 are the
// sub-plane's, and the spectrum columns are read / written with a stride of 2.
cudaError_t launch_dft_fwd_tc(const float* x, float2* out1, float2* out2, long long out_plane_stride,
                              int out_row_stride, int P, int H, int W, int m1, int m2, cudaStream_t stream,
                              const TcSub* sub = nullptr);
cudaError_t launch_dft_inv_tc(const float2* in1, const float2* in2, long long in_plane_stride,
                              int in_row_stride, float* y, int Q, int H, int W, int m1, int m2,
                              cudaStream_t stream, const TcSub* sub = nullptr);

// Folded tensor-core path for 256 x 256 planes (even m1 <= 32, even m2 <= 64).  Forward: one
// launch of the tensor-core kernel in its folded mode (launch_dft_fwd_tc_folded: CTAs in groups
// of four, one per parity sub-problem, each folding the full planes in its converters).
// Inverse: four sub-problem DFTs into `scratch` (P planes of floats, split_scratch_bytes), then
// the unfold.
bool tc_split_supported(int H, int W, int m1, int m2);
// 256 x 256 planes (m1, m2 <= 32) on the inverse side without the fold: one launch whose CTAs,
// in groups of four, each compute one 128 x 128 quadrant of the output from the full corners
// (the quadrant's offset is in its twiddle tables).  No scratch.
bool tc_quad_supported(int H, int W, int m1, int m2);
cudaError_t launch_dft_inv_tc_quad(const float2* in1, const float2* in2, long long in_plane_stride,
                                   int in_row_stride, float* y, int Q, int H, int W, int m1, int m2,
                                   cudaStream_t stream);
cudaError_t launch_dft_fwd_tc_folded(const float* x, float2* out1, float2* out2, long long out_plane_stride,
                                     int out_row_stride, int P, int H, int W, int m1, int m2, cudaStream_t stream);
size_t split_scratch_bytes(long long P, int H, int W);
cudaError_t launch_unfold(const float* zs, float* y, int P, int Hs, int Ws, cudaStream_t stream);

// Per-shape kernel variants chosen by measurement (scx_set_dft_variant / scx_set_mix_variant,
// filled from a tuning table by the host; scx_variants.cu).  kDftAuto and kMixAuto leave the
// choice to the library's fixed rules.  A variant that does not apply to a shape (or to the
// operands' alignment) falls back to those rules, so a table never makes a call fail.
constexpr int kDftAuto = 0, kDftFfma = 1, kDftTensor = 2, kDftFolded = 3;
constexpr int kMixAuto = -1, kMixSmem = 8;  // 0 .. 7: the TMA-ring tile shapes of scx_mix.cu
constexpr int kMixTc = 9;                    // the tcgen05 3xTF32 kernel of scx_mix_tc.cu
int dft_variant(int H, int W, int m1, int m2);
int mix_variant(int ncorner, int B, int Cin, int Cout, int NM);

// Forward / inverse truncated DFT through the fastest kernel for the shape: the
// tensor-core kernels where supported (unless SCX_VARIANT=ffma or the shape's variant says
// otherwise), else the FFMA kernels.  `scratch` (optional) enables the folded path for shapes
// that need it.
cudaError_t dft_fwd(const float* x, float2* out1, float2* out2, long long out_plane_stride, int out_row_stride,
                    int P, int H, int W, int m1, int m2, const Twiddles& tw, cudaStream_t stream,
                    float* scratch = nullptr, size_t scratch_bytes = 0);
cudaError_t dft_inv(const float2* in1, const float2* in2, long long in_plane_stride, int in_row_stride, float* y,
                    int Q, int H, int W, int m1, int m2, const Twiddles& tw, cudaStream_t stream,
                    float* scratch = nullptr, size_t scratch_bytes = 0);

// Device watchdog word of the current device (a static device variable, zero at module load,
// whose address is looked up once per device; no allocation): the tensor-core and TMA-ring
// kernels store a non-zero code there when they give up on a wait.
cudaError_t device_watchdog(int** out);

// FNO projection y = b2 + W2 GELU(b1 + W1 h) on the tensor core (scx_fno_proj_tc.cu): h is
// [B][hidden][HW], y [B][oc][HW].  Supported: hidden 32 or 64, proj_hidden a multiple of 32 up
// to 256, oc <= 4, HW a multiple of 128, 16-byte aligned h and W1.
bool fno_project_tc_supported(int hidden, int ph, int oc, int HW);
cudaError_t launch_fno_project_tc(const float* h, float* y, const float* w1, const float* b1, const float* w2,
                                  const float* b2, int B, int HW, int hidden, int ph, int oc, cudaStream_t stream);
cudaError_t read_watchdog(int* value, bool reset);

// Per-mode complex channel mixing y_c[b,o,k] = sum_i x_c[b,i,k] * w_c[i,o,k] for
// ncorner (1 or 2) corners, k over NM = m1*m2 modes.  The kernel is a programmatic dependent of
// the previous kernel in the stream; `w_early` tells it that w is not written by the kernels it
// is chained after (the layer's weights in a forward), so the TMA-ring kernel may request the
// first w boxes before waiting for them.
cudaError_t launch_mix(const float2* x1, const float2* x2, const float2* w1, const float2* w2,
                       float2* y1, float2* y2, int ncorner, int B, int Cin, int Cout, int NM,
                       cudaStream_t stream, bool w_early = false);

// The mixing with one operand read as the conjugate transpose of a stored tensor, on the
// TMA-ring kernel only (the backward's W^H and X^H without a transpose pass).  B, Cin, Cout are
// the product's: y[b][o] = sum_i x'[b][i] w'[i][o] per mode.  mode 1: w' = conj(w)^T with w stored
// [Cout][Cin] per mode; mode 2: x' = conj(x)^T with x stored [Cin][B] per mode, and, for W > 0,
// y scaled per mode by c_ky * inv_hw (c_ky = 1 for ky = 0 and, W even, ky = W/2, else 2;
// ky = mode % m2).
// Returns cudaErrorNotSupported where the ring kernel does not apply.
cudaError_t launch_mix_ring_ct(const float2* x1, const float2* x2, const float2* w1, const float2* w2, float2* y1,
                               float2* y2, int ncorner, int B, int Cin, int Cout, int NM, int mode, int m2, int W,
                               float inv_hw, cudaStream_t stream);

// The same contraction on the tensor core (3xTF32), used where the variant table selects it
// (variant kMixTc): B <= 16, Cin a multiple of 8, Cout a multiple of 64, an even mode count and
// 16-byte aligned operands.  Returns cudaErrorNotSupported for anything else.
bool mix_tc_supported(int B, int Cin, int Cout, int NM);
cudaError_t launch_mix_tc(const float2* x1, const float2* x2, const float2* w1, const float2* w2, float2* y1,
                          float2* y2, int ncorner, int B, int Cin, int Cout, int NM, cudaStream_t stream);

}  // namespace scx
