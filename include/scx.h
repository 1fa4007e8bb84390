/*
 * scx.h - C ABI of the B200 (sm_100a) SpectralConv2d / FNO-2d forward library (libscx.so).
 *
 * Drop-in device layer for the reference's SUPA extension: every entry point takes plain
 * device pointers, sizes and a CUDA stream, returns a status code and never allocates the
 * caller's buffers.  Status codes are cudaError_t values (0 = success, 1 =
 * cudaErrorInvalidValue for bad arguments); scx_status_string() names them.  No entry
 * point aborts, traps or synchronises the device.
 *
 * Tensor layouts (fp32; complex values interleaved re/im, i.e. view_as_real of complex64):
 *   x        [B][Cin][H][W]             real input
 *   y        [B][Cout][H][W]            real output
 *   weights  [Cin][Cout][m1][m2][2]     one tensor per corner (weights1, weights2)
 *   corner   [B][C][m1][m2][2]          corner 1 = rows kx in [0,m1), corner 2 = rows
 *                                       kx in [H-m1,H), both for ky in [0,m2)
 *   spectrum [B][C][H][W/2+1][2]        full half-spectrum (compatibility entry points)
 * Shape rules are the reference's: 1 <= m1 <= H and 1 <= m2 <= W/2+1; when 2*m1 > H the
 * corner rows overlap and corner 2 overwrites corner 1 (spectral_conv/reference_pytorch.py:41-46).
 *
 * Twiddle tables are built once per (device, H, W, m1, m2) by the library and kept for
 * the life of the process; the first call for a shape performs that set-up (a
 * cudaMalloc and a synchronous copy), so make it outside CUDA-graph capture, e.g. with
 * scx_prepare().  Calls are thread-safe.
 */
#ifndef SCX_H_
#define SCX_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t; NULL selects the legacy default stream. */
typedef void* scx_stream_t;

/* Library version, major*10000 + minor*100 + patch. */
int scx_version(void);

/* Human-readable name of a status code returned by this library. */
const char* scx_status_string(int status);

/* Diagnostic without a reference counterpart: the device watchdog word of the current
 * device (0 = no kernel ever gave up waiting on its own tensor-core pipeline; a positive
 * code names the wait that timed out), optionally resetting it.  Synchronous; negative
 * values are -cudaError_t of the read. */
int scx_watchdog(int reset);

/* Builds (if needed) the twiddle tables for one shape on the current device.
 * Replaces the suFFT plan/work-area warm-up: get_cached_plan / get_workspace
 * (spectral_conv/spectral_conv_ext.cpp:77-121) driven by warmup_spectral_plans
 * (spectral_conv/spectral_conv_ops.py:459-477). */
int scx_prepare(int H, int W, int modes1, int modes2);

/* Single-corner complex mode mixing y[b,o,k] = sum_i x[b,i,k] * w[i,o,k].
 * Replaces launch_spectral_mul (spectral_conv_combo/spectral_conv_ext.su:94-109), same
 * argument order; the stream is honoured instead of the null stream.
 * x_freq [B][Cin][m1][m2][2], weights [Cin][Cout][m1][m2][2], y_freq [B][Cout][m1][m2][2]. */
int scx_spectral_mul(const float* x_freq, const float* weights, float* y_freq, int batch_size,
                     int channels_in, int channels_out, int modes1, int modes2,
                     scx_stream_t stream);

/* Both corners in one launch.  Replaces launch_spectral_mul_dual_packed
 * (spectral_conv_combo/spectral_conv_ext.su:111-127), same argument order; serves the
 * pybind entry points spectral_mul_dual_out (spectral_conv/spectral_conv_ext.cpp:200-245). */
int scx_spectral_mul_dual(const float* x1, const float* x2, const float* w1, const float* w2,
                          float* y1, float* y2, int batch_size, int channels_in,
                          int channels_out, int modes1, int modes2, scx_stream_t stream);

/* Backward of the single-corner mixing: the gradients of SpectralMulFunction
 * (spectral_conv/spectral_conv_ops.py:260-278, whose backward is two torch.einsum calls):
 *   grad_x[b,i,k] = sum_o grad_y[b,o,k] conj(w[i,o,k]),  grad_w[i,o,k] = sum_b conj(x[b,i,k]) grad_y[b,o,k]
 * x_freq [B][Cin][m1][m2][2], weights [Cin][Cout][m1][m2][2], grad_y [B][Cout][m1][m2][2];
 * grad_x like x_freq and grad_w like weights, either NULL to skip it (x_freq may then be NULL
 * when grad_w is, weights when grad_x is).  workspace: device memory of
 * scx_spectral_mul_bwd_workspace_size() bytes, 256-byte aligned (the per-mode conjugate
 * transposes of w and x). */
size_t scx_spectral_mul_bwd_workspace_size(int batch_size, int channels_in, int channels_out,
                                           int modes1, int modes2);
int scx_spectral_mul_bwd(const float* x_freq, const float* weights, const float* grad_y,
                         float* grad_x, float* grad_w, int batch_size, int channels_in,
                         int channels_out, int modes1, int modes2, void* workspace,
                         size_t workspace_bytes, scx_stream_t stream);

/* Truncated forward real DFT writing only the two retained corners.
 * Replaces rfft2_sufft followed by the corner gathers x_freq[:, :, :m1, :m2] and
 * x_freq[:, :, -m1:, :m2] (spectral_conv/spectral_conv_ext.cpp:314-347,
 * spectral_conv/spectral_conv_ops.py:385-392).
 * x [B][C][H][W]; x1, x2 [B][C][m1][m2][2]. */
int scx_rfft2_corners(const float* x, float* x1, float* x2, int batch_size, int channels,
                      int height, int width, int modes1, int modes2, scx_stream_t stream);

/* Zero-padded inverse real DFT from the two corners straight to the real output.
 * Replaces the zeroed out_freq buffer, the two corner scatters and irfft2_sufft
 * (spectral_conv/spectral_conv_ops.py:386-406, spectral_conv/spectral_conv_ext.cpp:349-384).
 * y1, y2 [B][C][m1][m2][2]; y [B][C][H][W]. */
int scx_irfft2_corners(const float* y1, const float* y2, float* y, int batch_size, int channels,
                       int height, int width, int modes1, int modes2, scx_stream_t stream);

/* Full half-spectrum forward 2-D real DFT, x [B][C][H][W] -> x_freq [B][C][H][W/2+1][2].
 * Compatibility path for rfft2_sufft (spectral_conv/spectral_conv_ext.cpp:314-347);
 * not used by the fused forward. */
int scx_rfft2(const float* x, float* x_freq, int batch_size, int channels, int height,
              int width, scx_stream_t stream);

/* Full half-spectrum inverse 2-D real DFT (scale 1/(H*W)), x_freq [B][C][H][W/2+1][2] ->
 * y [B][C][H][W].  Compatibility path for irfft2_sufft
 * (spectral_conv/spectral_conv_ext.cpp:349-384); not used by the fused forward. */
int scx_irfft2(const float* x_freq, float* y, int batch_size, int channels, int height,
               int width, scx_stream_t stream);

/* Bytes of device workspace scx_spectral_conv2d_fwd needs (the two corner spectra in and
 * out); 0 on invalid sizes. */
size_t scx_spectral_conv2d_workspace_size(int batch_size, int channels_in, int channels_out,
                                          int height, int width, int modes1, int modes2);

/* Fused SpectralConv2d forward: truncated rfft2 -> dual-corner mixing -> zero-padded
 * irfft2, y = SpectralConv2d(x) of spectral_conv/reference_pytorch.py:30-47.
 * Replaces spectral_conv2d_fused (spectral_conv/spectral_conv_ops.py:363-417) and its
 * native calls.  workspace: caller-owned device memory of at least
 * scx_spectral_conv2d_workspace_size() bytes, 16-byte aligned. */
int scx_spectral_conv2d_fwd(const float* x, const float* weights1, const float* weights2,
                            float* y, int batch_size, int channels_in, int channels_out,
                            int height, int width, int modes1, int modes2, void* workspace,
                            size_t workspace_bytes, scx_stream_t stream);

/* On return from scx_spectral_conv2d_fwd the workspace starts with the input corner
 * spectra X1 then X2 ([B][Cin][m1][m2] complex, interleaved float pairs, each); the backward
 * below takes them as the forward's saved state. */

/* Bytes of device workspace scx_spectral_conv2d_bwd needs; 0 on invalid sizes. */
size_t scx_spectral_conv2d_bwd_workspace_size(int batch_size, int channels_in, int channels_out,
                                              int height, int width, int modes1, int modes2);

/* SpectralConv2d backward: the gradients torch autograd gives for the forward of
 * spectral_conv/reference_pytorch.py:30-47 (the reference differentiates only the mixing,
 * SpectralMulFunction in spectral_conv/spectral_conv_ops.py:260-286).  grad_y
 * [B][Cout][H][W]; x_corners: X1 then X2 as the forward left them at the head of its
 * workspace (needed only for the weight gradients); weights as for the forward.  Outputs:
 * grad_x [B][Cin][H][W] (NULL to skip), grad_w1 and grad_w2 [Cin][Cout][m1][m2] complex
 * (both NULL to skip; x_corners may then be NULL).  workspace: device memory of
 * scx_spectral_conv2d_bwd_workspace_size() bytes, 256-byte aligned. */
int scx_spectral_conv2d_bwd(const float* grad_y, const float* x_corners, const float* weights1,
                            const float* weights2, float* grad_x, float* grad_w1, float* grad_w2,
                            int batch_size, int channels_in, int channels_out, int height, int width,
                            int modes1, int modes2, void* workspace, size_t workspace_bytes,
                            scx_stream_t stream);

/* Single-corner SpectralConv3d forward (spectral_conv_combo/reference_pytorch.py:51-82):
 * rfftn over (D, H, W), the corner [:m1, :m2, :m3] mixed per mode, zero-padded irfftn.
 * Replaces spectral_conv3d_supa (spectral_conv_combo/spectral_conv_ops.py:435-472).  x
 * [B][Cin][D][H][W], weights [Cin][Cout][m1][m2][m3] complex (interleaved), y
 * [B][Cout][D][H][W]; device pointers.  Needs m1 <= D, m2 <= H, m3 <= W/2 + 1; workspace of
 * scx_spectral_conv3d_workspace_size() bytes, 256-byte aligned. */
size_t scx_spectral_conv3d_workspace_size(int batch_size, int channels_in, int channels_out,
                                          int depth, int height, int width, int modes1,
                                          int modes2, int modes3);
int scx_spectral_conv3d_fwd(const float* x, const float* weights, float* y, int batch_size,
                            int channels_in, int channels_out, int depth, int height, int width,
                            int modes1, int modes2, int modes3, void* workspace,
                            size_t workspace_bytes, scx_stream_t stream);

/* Four-corner SpectralConv3d forward (spectral_conv_combo/official_baseline.py:60-100):
 * corners (low | high kx) x (low | high ky) x low kz with weights w1 (low, low), w2 (high kx),
 * w3 (high ky), w4 (high, high), each [Cin][Cout][m1][m2][m3] complex; where corners overlap
 * (2 m1 > D or 2 m2 > H) the later one wins, as in the baseline's assignments.  Other
 * arguments as scx_spectral_conv3d_fwd. */
size_t scx_spectral_conv3d_4c_workspace_size(int batch_size, int channels_in, int channels_out,
                                             int depth, int height, int width, int modes1,
                                             int modes2, int modes3);
int scx_spectral_conv3d_4c_fwd(const float* x, const float* w1, const float* w2, const float* w3,
                               const float* w4, float* y, int batch_size, int channels_in,
                               int channels_out, int depth, int height, int width, int modes1,
                               int modes2, int modes3, void* workspace, size_t workspace_bytes,
                               scx_stream_t stream);

/* The same forward from host memory to host memory: the host-facing call of
 * spectral_conv2d_supa with a CPU tensor (spectral_conv/spectral_conv_ops.py:480-505, which
 * copies the batch up, runs the forward and copies it down in turn).  x_host
 * [B][Cin][H][W] and y_host [B][Cout][H][W] are host memory, page-locked for the copies to
 * overlap (cudaHostAlloc / cudaHostRegister; pageable memory gives the same result, slower);
 * weights1/weights2 as for scx_spectral_conv2d_fwd.  x_dev and y_dev are caller-owned device
 * buffers of B*Cin*H*W and B*Cout*H*W floats, workspace as for scx_spectral_conv2d_fwd with
 * the whole batch.  The batch is split into `chunks` pieces (0: the library's default, 6;
 * the first and last half-size): the upload of piece i+1, the forward of piece i on `stream`
 * and the download of piece i-1 overlap on two library-owned copy streams.  Returns when
 * y_host holds the result (not graph-capturable); later work on `stream` is ordered after
 * it.  Calls on one device are serialised. */
int scx_spectral_conv2d_fwd_host(const float* x_host, const float* weights1, const float* weights2,
                                 float* y_host, int batch_size, int channels_in, int channels_out,
                                 int height, int width, int modes1, int modes2, float* x_dev,
                                 float* y_dev, void* workspace, size_t workspace_bytes, int chunks,
                                 scx_stream_t stream);

/* ---------------------------------------------------------------------------------
 * FNO-2d forward (fno_ns/model.py:137-259): lift -> n_layers x Fourier layer ->
 * projection, one call.  Replaces FNO2d.forward_supa_chain (fno_ns/model.py:219-259) with
 * FourierLayer.forward_supa (:101-134).  Fourier layer:
 *   h' = GELU(InstanceNorm(SpectralConv2d(h) + Conv1x1(h)))   (instance_norm = 1)
 *   h' = GELU(SpectralConv2d(h) + Conv1x1(h))                  (instance_norm = 0)
 * InstanceNorm2d defaults: no affine, no running stats, eps 1e-5, biased variance.
 * GELU is the exact (erf) form.  Projection: Conv1x1(hidden->proj_hidden), GELU,
 * Conv1x1(proj_hidden->out_channels).
 * --------------------------------------------------------------------------------- */
#define SCX_FNO_MAX_LAYERS 16

typedef struct scx_fno2d_config {
    int batch_size;    /* B */
    int height;        /* H */
    int width;         /* W */
    int in_frames;     /* T: input frames; the lift sees T + 2 channels (frames, grid_x, grid_y) */
    int input_layout;  /* 0: x [B][T][H][W], the grid is generated inside (fno_ns/model.py:168-194)
                          1: x [B][H][W][T+2] channels-last, the frames then the 2 grid channels */
    int hidden;        /* channel width of the Fourier layers */
    int modes1;
    int modes2;
    int n_layers;      /* 1 .. SCX_FNO_MAX_LAYERS */
    int proj_hidden;   /* 128 in fno_ns/model.py:162-166 */
    int out_channels;  /* 1 */
    int instance_norm; /* 1 or 0, see above */
} scx_fno2d_config;

typedef struct scx_fno2d_params {
    const float* lift_w;                              /* [hidden][T+2]              */
    const float* lift_b;                              /* [hidden]                   */
    const float* spectral_w1[SCX_FNO_MAX_LAYERS];     /* [hidden][hidden][m1][m2][2] */
    const float* spectral_w2[SCX_FNO_MAX_LAYERS];     /* [hidden][hidden][m1][m2][2] */
    const float* skip_w[SCX_FNO_MAX_LAYERS];          /* [hidden][hidden] (out, in) */
    const float* skip_b[SCX_FNO_MAX_LAYERS];          /* [hidden]                   */
    const float* proj1_w;                             /* [proj_hidden][hidden]      */
    const float* proj1_b;                             /* [proj_hidden]              */
    const float* proj2_w;                             /* [out_channels][proj_hidden] */
    const float* proj2_b;                             /* [out_channels]             */
} scx_fno2d_params;

/* Device workspace bytes scx_fno2d_fwd needs; 0 for an invalid configuration. */
size_t scx_fno2d_workspace_size(const scx_fno2d_config* cfg);

/* y [B][out_channels][H][W] = FNO2d(x).  All pointers are device pointers except cfg and
 * params (host structs).  The first call for a (H, W, modes) shape builds the twiddle
 * tables (see above). */
int scx_fno2d_fwd(const scx_fno2d_config* cfg, const scx_fno2d_params* params, const float* x,
                  float* y, void* workspace, size_t workspace_bytes, scx_stream_t stream);

/* ---------------------------------------------------------------------------------
 * Per-shape kernel variants.  Replaces the reference's tuning table: _AUTO_TUNE_TABLE
 * (spectral_conv_combo/spectral_conv_ops.py:45-63), written by tune.py's sweep
 * (spectral_conv_combo/tune.py:154-261) and never read back there.  The host-side tuner
 * (scx_tune.py) measures the variants that apply to a shape, persists the winners as JSON and
 * sets them through these calls when the Python package is imported.  The table is
 * process-wide (every device); a variant that does not fit a call (alignment, workspace)
 * falls back to the library's rule, so setting one never makes a call fail.  No CUDA calls.
 * --------------------------------------------------------------------------------- */
/* Truncated-DFT variants: 0 = the library's rule, 1 = FFMA direct DFT, 2 = tensor-core
 * kernels, 3 = the folded tensor-core path (256-point sides).  scx_dft_variants returns the
 * bit mask (1 << variant) of the variants 1..3 that apply to the shape. */
int scx_dft_variants(int H, int W, int modes1, int modes2);
int scx_set_dft_variant(int H, int W, int modes1, int modes2, int variant);
/* Mixing variants for (corners, B, Cin, Cout, modes = m1*m2): -1 = the library's cost model
 * (FFMA kernels), 0..7 = one of the TMA-ring tile shapes, 8 = the per-thread shared-memory kernel,
 * 9 = the tcgen05 3xTF32 kernel (B <= 16, Cin a multiple of 8, Cout a multiple of 64, an even
 * mode count, 16-byte aligned operands; other calls fall back to the library's choice). */
int scx_set_mix_variant(int ncorner, int batch_size, int channels_in, int channels_out, int modes,
                        int variant);
/* kind 0: the DFT variant set for (a, b, c, d) = (H, W, m1, m2); kind 1: the mixing variant for
 * (a, b, c, d, e) = (corners, B, Cin, Cout, modes). */
int scx_get_variant(int kind, int a, int b, int c, int d, int e);
void scx_clear_variants(void);

/* Size of the fixed device scratch used by scx_spectral_conv2d_fwd_noalloc (16 MiB). */
#define SCX_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* Peer-memory plumbing for the multi-GPU output gather (one process per GPU).  No counterpart
 * in the reference, which has no multi-GPU path; it replaces the NCCL point-to-point gather of
 * the output shards to one rank.  The gathering rank exports its output buffer once
 * (scx_ipc_export: an IPC handle of scx_ipc_handle_bytes() bytes for the allocation that
 * contains dev_ptr, plus dev_ptr's byte offset in it).  Every other rank imports the handle
 * (scx_ipc_import, peer access enabled on first use), and each step pushes its shard with
 * scx_copy_async into base + offset + its slice: one device-to-device copy over NVLink, run by
 * the copy engines and ordered on the caller's stream after the kernels that produced it.  The
 * push is complete when that stream reaches it; the gathering rank reads the buffer only after
 * every pusher has synchronised (a host barrier).  scx_ipc_close releases an import. */
int scx_ipc_handle_bytes(void);
int scx_ipc_export(const void* dev_ptr, void* handle_out, unsigned long long* offset_out);
int scx_ipc_import(const void* handle, void** base_out);
int scx_ipc_close(void* base);
int scx_copy_async(void* dst, const void* src, size_t bytes, scx_stream_t stream);

/* Allocation-free variant of scx_spectral_conv2d_fwd.  No counterpart in the reference:
 * it exists for callers that cannot let a library call cudaMalloc (a process whose
 * memory pool already owns the GPU's memory, or a latency-critical loop that cannot
 * absorb an allocation's device synchronisation).  Same arguments and result as
 * scx_spectral_conv2d_fwd minus the workspace: the corner spectra and the twiddle tables
 * live in one library-owned static device array of SCX_NOALLOC_SCRATCH_BYTES, held by
 * every GPU that loads the library until the process exits.  Its scratch need is
 *   sum over {X1,X2,Y1,Y2,four twiddle tables} of the region size rounded up to 256 B,
 * i.e. about 16*B*(Cin+Cout)*m1*m2 + 32*(W*m2 + 2*m1*H) bytes; larger shapes return
 * cudaErrorMemoryAllocation (2) without launching.  The first call on a device looks up
 * the array's address (cudaGetSymbolAddress) with that device current: make it before
 * any stream capture.  The address is cached per device for the life of the process, so it
 * does not survive a cudaDeviceReset of that device.  All calls share the array: calls that
 * overlap on the GPU race, so order them on one stream.  Nothing has to be cleared between
 * calls.  The truncated DFTs run on the FFMA kernels (the tensor-core kernels read operand
 * tables that the library allocates), so expect lower throughput than
 * scx_spectral_conv2d_fwd on the shapes where that one uses the tensor cores.  As with every
 * entry point, a kernel that gave up on a bounded wait leaves y undefined and records a code
 * that scx_watchdog() returns: read it after synchronising when the result matters. */
int scx_spectral_conv2d_fwd_noalloc(const float* x, const float* weights1, const float* weights2,
                                    float* y, int batch_size, int channels_in, int channels_out,
                                    int height, int width, int modes1, int modes2,
                                    scx_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SCX_H_ */
