/*
 * ORACLE - TEST INFRASTRUCTURE ONLY.  Float64 CPU restatement of the reference's
 * SpectralConv2d forward, used by tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg as the checker.  The product path never links or calls this file.
 *
 * It restates spectral_conv/reference_pytorch.py:30-47 with direct DFTs in double
 * precision (no FFT library), following the reference's steps literally:
 *   x_ft  = rfft2(x)                                       (:32)  -> only rows/cols used
 *   out_ft = zeros(B, Cout, H, W//2+1)                      (:33-40)
 *   out_ft[:, :, :m1, :m2]  = einsum(bixy,ioxy->boxy)(x_ft[:, :, :m1, :m2], w1)   (:41-43)
 *   out_ft[:, :, -m1:, :m2] = einsum(...)(x_ft[:, :, -m1:, :m2], w2)             (:44-46)
 *   y = irfft2(out_ft, s=(H, W))                            (:47)
 * The irfft2 is the C2C inverse along H over the whole out_ft followed by the C2R inverse
 * along W, whose Hermitian rule keeps only Re() of each term, counts bins 0 and W/2
 * (W even) once and every other bin twice, and scales by 1/(H*W).
 * Pinned against fixtures produced by the reference itself (tests/golden/).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

typedef struct {
    double re, im;
} cplx;

static double ang(long long k, long long n, long long N) {
    return 2.0 * M_PI * (double)((k * n) % N) / (double)N;
}

/* Forward corners for one plane: X[2*m1][m2], rows 0..m1-1 = kx 0..m1-1 and
 * rows m1..2m1-1 = kx H-m1..H-1. */
static void plane_forward(const float* xp, int H, int W, int m1, int m2, cplx* R, cplx* X) {
    for (int h = 0; h < H; ++h)
        for (int ky = 0; ky < m2; ++ky) {
            double re = 0.0, im = 0.0;
            for (int w = 0; w < W; ++w) {
                const double a = ang(ky, w, W);
                const double v = (double)xp[(size_t)h * W + w];
                re += v * cos(a);
                im -= v * sin(a);
            }
            R[(size_t)h * m2 + ky].re = re;
            R[(size_t)h * m2 + ky].im = im;
        }
    for (int s = 0; s < 2 * m1; ++s) {
        const int kx = s < m1 ? s : H - m1 + (s - m1);
        for (int ky = 0; ky < m2; ++ky) {
            double re = 0.0, im = 0.0;
            for (int h = 0; h < H; ++h) {
                const double a = ang(kx, h, H);
                const double c = cos(a), sn = -sin(a);
                const cplx r = R[(size_t)h * m2 + ky];
                re += c * r.re - sn * r.im;
                im += c * r.im + sn * r.re;
            }
            X[(size_t)s * m2 + ky].re = re;
            X[(size_t)s * m2 + ky].im = im;
        }
    }
}

/* Inverse of one plane from out_ft rows (H x m2, zero elsewhere) to y[H][W]. */
static void plane_inverse(const cplx* out_ft, const unsigned char* nonzero, int H, int W, int m2,
                          cplx* Z, double* y) {
    for (int h = 0; h < H; ++h)
        for (int ky = 0; ky < m2; ++ky) {
            double re = 0.0, im = 0.0;
            for (int kx = 0; kx < H; ++kx) {
                if (!nonzero[kx]) continue;
                const double a = ang(kx, h, H);
                const double c = cos(a), sn = sin(a);
                const cplx v = out_ft[(size_t)kx * m2 + ky];
                re += c * v.re - sn * v.im;
                im += c * v.im + sn * v.re;
            }
            Z[(size_t)h * m2 + ky].re = re;
            Z[(size_t)h * m2 + ky].im = im;
        }
    const double scale = 1.0 / ((double)H * (double)W);
    for (int h = 0; h < H; ++h)
        for (int w = 0; w < W; ++w) {
            double acc = 0.0;
            for (int ky = 0; ky < m2; ++ky) {
                const int single = (ky == 0) || ((W % 2 == 0) && (ky == W / 2));
                const double a = ang(ky, w, W);
                const cplx z = Z[(size_t)h * m2 + ky];
                acc += (single ? 1.0 : 2.0) * (z.re * cos(a) - z.im * sin(a));
            }
            y[(size_t)h * W + w] = acc * scale;
        }
}

/* Corner spectra of every plane: x [P][H][W] -> x1, x2 [P][m1][m2][2] (double). */
int oracle_rfft2_corners(const float* x, double* x1, double* x2, int P, int H, int W, int m1, int m2) {
    if (P <= 0 || H <= 0 || W <= 0 || m1 <= 0 || m2 <= 0 || m1 > H || m2 > W / 2 + 1) return 1;
    cplx* R = (cplx*)malloc(sizeof(cplx) * (size_t)H * m2);
    cplx* X = (cplx*)malloc(sizeof(cplx) * (size_t)2 * m1 * m2);
    if (!R || !X) {
        free(R);
        free(X);
        return 2;
    }
    for (int p = 0; p < P; ++p) {
        plane_forward(x + (size_t)p * H * W, H, W, m1, m2, R, X);
        for (int s = 0; s < 2 * m1; ++s)
            for (int ky = 0; ky < m2; ++ky) {
                double* dst = s < m1 ? x1 + (((size_t)p * m1 + s) * m2 + ky) * 2
                                     : x2 + (((size_t)p * m1 + (s - m1)) * m2 + ky) * 2;
                dst[0] = X[(size_t)s * m2 + ky].re;
                dst[1] = X[(size_t)s * m2 + ky].im;
            }
    }
    free(R);
    free(X);
    return 0;
}

/* y = SpectralConv2d(x) in double.  w1, w2: [Cin][Cout][m1][m2][2] float (view_as_real
 * of the complex64 parameters); y: [B][Cout][H][W] double. */
int oracle_spectral_conv2d(const float* x, const float* w1, const float* w2, double* y, int B, int Cin,
                           int Cout, int H, int W, int m1, int m2) {
    if (B <= 0 || Cin <= 0 || Cout <= 0 || H <= 0 || W <= 0 || m1 <= 0 || m2 <= 0 || m1 > H ||
        m2 > W / 2 + 1)
        return 1;
    const size_t NM = (size_t)m1 * m2;
    cplx* R = (cplx*)malloc(sizeof(cplx) * (size_t)H * m2);
    cplx* X = (cplx*)malloc(sizeof(cplx) * (size_t)B * Cin * 2 * NM);
    cplx* out_ft = (cplx*)malloc(sizeof(cplx) * (size_t)H * m2);
    unsigned char* nonzero = (unsigned char*)malloc((size_t)H);
    cplx* Z = (cplx*)malloc(sizeof(cplx) * (size_t)H * m2);
    if (!R || !X || !out_ft || !nonzero || !Z) {
        free(R);
        free(X);
        free(out_ft);
        free(nonzero);
        free(Z);
        return 2;
    }
    for (int b = 0; b < B; ++b)
        for (int i = 0; i < Cin; ++i)
            plane_forward(x + ((size_t)b * Cin + i) * H * W, H, W, m1, m2, R,
                          X + ((size_t)b * Cin + i) * 2 * NM);
    memset(nonzero, 0, (size_t)H);
    for (int kx = 0; kx < m1; ++kx) nonzero[kx] = 1;
    for (int kx = H - m1; kx < H; ++kx) nonzero[kx] = 1;
    for (int b = 0; b < B; ++b)
        for (int o = 0; o < Cout; ++o) {
            memset(out_ft, 0, sizeof(cplx) * (size_t)H * m2);
            /* corner 1 then corner 2, the second assignment overwriting the first */
            for (int c = 0; c < 2; ++c) {
                const float* w = c == 0 ? w1 : w2;
                for (int j = 0; j < m1; ++j) {
                    const int kx = c == 0 ? j : H - m1 + j;
                    for (int ky = 0; ky < m2; ++ky) {
                        double re = 0.0, im = 0.0;
                        for (int i = 0; i < Cin; ++i) {
                            const cplx xv = X[((size_t)b * Cin + i) * 2 * NM + (size_t)(c * m1 + j) * m2 + ky];
                            const float* wv = w + ((((size_t)i * Cout + o) * m1 + j) * m2 + ky) * 2;
                            re += xv.re * (double)wv[0] - xv.im * (double)wv[1];
                            im += xv.re * (double)wv[1] + xv.im * (double)wv[0];
                        }
                        out_ft[(size_t)kx * m2 + ky].re = re;
                        out_ft[(size_t)kx * m2 + ky].im = im;
                    }
                }
            }
            plane_inverse(out_ft, nonzero, H, W, m2, Z, y + ((size_t)b * Cout + o) * H * W);
        }
    free(R);
    free(X);
    free(out_ft);
    free(nonzero);
    free(Z);
    return 0;
}
