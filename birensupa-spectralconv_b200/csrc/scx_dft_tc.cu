// Tensor-core (tcgen05, bf16x3 -> fp32) truncated DFT kernels for H in {64, 128},
// W in {64, 128}, m2 <= 32 and 4*m1 <= 128 (the 64x64 and 128x128 workloads and the
// FNO-NS layers).  Other shapes use the FFMA kernels of scx_dft_ffma.cu.
//
// Forward, one tile = 128 consecutive rows of x viewed as [P*H][W] (2 planes at H=64,
// 1 plane at H=128):
//   S1  D1[r][n]  = sum_w x[r][w] * TW[n][w]                  (M=128, N=N1, K=W)
//       TW rows n < R2: cos(2 pi n w / W); rows R2+n: -sin(2 pi n w / W)  (n < m2, else 0)
//   E1  D1 (lane = row) -> R^T in shared memory: rows (plane, n), K = h
//   S2  D2[j][c]  = sum_h F[j][h] * R^T[c][h]                 (M=128, N=planes*N1, K=H)
//       F rows j < 2m1: cos(2 pi kx_j h / H); rows 2m1+j: sin(...); rows >= 4m1 zero
//   E2  X[slot][ky] = (D2[cos][re] + D2[sin][im], D2[cos][im] - D2[sin][re])
// Inverse, one tile = the planes whose spectra fill one S4 (2 planes at H=64, 1 at H=128):
//   S4  D4[h][c] = sum_j G[h][j] * Yr^T[c][j]                 (M=128, N=planes*N1, K=4m1)
//       G = [cos | sin](2 pi kx h / H) per slot (0 where corner 2 overwrites corner 1);
//       Yr^T rows (plane, re, ky): [Y_re | -Y_im], rows (plane, im, ky): [Y_im | Y_re]
//   E4  D4 (lane = h) -> Z rows in shared memory, K = (re|im, ky)
//   S5  D5[h][w] = sum_c Z[h][c] * E[w][c]                    (M=128, N=W, K=N1)
//       E = c_ky/(HW) [cos | -sin](2 pi ky w / W)
//   E5  D5 -> y rows
// Every product uses three bf16 MMAs (hi*hi + hi*lo + lo*hi) accumulating in fp32 TMEM.
// One thread issues the MMAs; the CTA waits on an mbarrier (bounded: a stuck wait raises
// the watchdog word and the kernel returns instead of hanging).
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "scx_internal.h"
#include "scx_tc.cuh"

namespace scx {

namespace {

constexpr int kTcThreads = 256;

// ------------------------------------------------------------------ host-side tables

uint16_t bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    return static_cast<uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

float bf16_float(uint16_t b) {
    const uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

struct Operand {  // [hi block | lo block], each rows x kpad bf16 in the K-major SW128 order
    int rows, kpad;
    std::vector<uint16_t> data;
    Operand(int r, int k) : rows(r), kpad(k), data(static_cast<size_t>(2) * r * k, 0) {}
    void put(int r, int k, double v) {
        const uint16_t hi = bf16_bits(static_cast<float>(v));
        const uint16_t lo = bf16_bits(static_cast<float>(v - static_cast<double>(bf16_float(hi))));
        const size_t off = tc::kmajor_offset(rows, r, k) / 2;
        data[off] = hi;
        data[static_cast<size_t>(rows) * kpad + off] = lo;
    }
    size_t bytes() const { return data.size() * 2; }
};

inline double ang(long long k, long long n, long long N) {
    return 2.0 * M_PI * static_cast<double>((k * n) % N) / static_cast<double>(N);
}
inline int slot_row(int s, int H, int m1) { return s < m1 ? s : H - m1 + (s - m1); }
inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

struct TcShape {
    int H, W, m1, m2;
    int R2, N1, np, N2, Kg;  // re block, 2*R2, planes per tile, np*N1, 4*m1 rounded to 16
    int MF;                  // rows of the forward column-DFT operand: 64 if 4*m1 <= 64, else 128
};

TcShape tc_shape(int H, int W, int m1, int m2) {
    TcShape s;
    s.H = H;
    s.W = W;
    s.m1 = m1;
    s.m2 = m2;
    s.R2 = round_up(m2, 8);
    s.N1 = 2 * s.R2;
    s.np = 128 / H;
    s.N2 = s.np * s.N1;
    s.Kg = round_up(4 * m1, 16);
    s.MF = (4 * m1 <= 64) ? 64 : 128;
    return s;
}

constexpr size_t kMaxDynSmem = 227 * 1024 - 256;  // minus the kernel's static shared memory
size_t inv_smem_bytes(const TcShape& s) {
    const int kgp = round_up(s.Kg, 64);
    return static_cast<size_t>(128) * kgp * 4 + static_cast<size_t>(s.W) * 64 * 4 +
           static_cast<size_t>(s.N2) * kgp * 4 + static_cast<size_t>(s.np) * 128 * 128 * 2 * 2 + 1024;
}

struct TcTables {
    const uint4* inv_g;
    const uint4* inv_e;
    uint32_t g_bytes, e_bytes;
};

std::mutex g_tc_mutex;
std::map<std::tuple<int, int, int, int, int>, TcTables> g_tc_cache;

cudaError_t get_tc_tables(const TcShape& s, const TcTables** out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    const auto key = std::make_tuple(dev, s.H, s.W, s.m1, s.m2);
    std::lock_guard<std::mutex> lock(g_tc_mutex);
    auto it = g_tc_cache.find(key);
    if (it != g_tc_cache.end()) {
        *out = &it->second;
        return cudaSuccess;
    }
    const int H = s.H, W = s.W, m1 = s.m1, m2 = s.m2;
    Operand g(128, round_up(s.Kg, 64));  // S4 A operand
    for (int h = 0; h < H; ++h)
        for (int j = 0; j < 2 * m1; ++j) {
            const int kx = slot_row(j, H, m1);
            if (j < m1 && kx >= H - m1) continue;  // overwritten by corner 2
            g.put(h, j, std::cos(ang(kx, h, H)));
            g.put(h, 2 * m1 + j, std::sin(ang(kx, h, H)));
        }
    Operand e(W, 64);  // S5 B operand
    const double inv_hw = 1.0 / (static_cast<double>(H) * static_cast<double>(W));
    for (int ky = 0; ky < m2; ++ky) {
        const bool single = (ky == 0) || ((W % 2 == 0) && (ky == W / 2));
        const double c = (single ? 1.0 : 2.0) * inv_hw;
        for (int w = 0; w < W; ++w) {
            e.put(w, ky, c * std::cos(ang(ky, w, W)));
            e.put(w, s.R2 + ky, -c * std::sin(ang(ky, w, W)));
        }
    }
    const size_t total = g.bytes() + e.bytes();
    uint8_t* dbuf = nullptr;
    err = cudaMalloc(&dbuf, total);
    if (err != cudaSuccess) return err;
    std::vector<uint8_t> host(total);
    size_t off = 0;
    const void* srcs[2] = {g.data.data(), e.data.data()};
    const size_t sizes[2] = {g.bytes(), e.bytes()};
    size_t offs[2];
    for (int i = 0; i < 2; ++i) {
        offs[i] = off;
        std::memcpy(host.data() + off, srcs[i], sizes[i]);
        off += sizes[i];
    }
    err = cudaMemcpy(dbuf, host.data(), total, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        cudaFree(dbuf);
        return err;
    }
    TcTables t;
    t.inv_g = reinterpret_cast<const uint4*>(dbuf + offs[0]);
    t.inv_e = reinterpret_cast<const uint4*>(dbuf + offs[1]);
    t.g_bytes = static_cast<uint32_t>(g.bytes());
    t.e_bytes = static_cast<uint32_t>(e.bytes());
    auto res = g_tc_cache.emplace(key, t);
    *out = &res.first->second;
    return cudaSuccess;
}

inline uint32_t tmem_cols_for(int n) {
    uint32_t c = 32;
    while (c < static_cast<uint32_t>(n)) c <<= 1;
    return c;
}

// ------------------------------------------------------------------ device helpers

// all threads: bounded wait, then agree on success
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t& phase, int* abort_flag, int* watchdog, int code) {
    const bool ok = tc::mbar_wait_bounded(bar, phase);
    phase ^= 1u;
    if (!ok) {
        *abort_flag = 1;
        atomicExch(watchdog, code);
    }
    __syncthreads();
    return *abort_flag == 0;
}

// bf16x3 product of one K step: D (+)= Ahi*Bhi + Ahi*Blo + Alo*Bhi
__device__ __forceinline__ void mma3(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                     uint32_t idesc, bool first) {
    tc::mma_bf16(d, tc::desc_sw128(a_hi), tc::desc_sw128(b_hi), idesc, first ? 0u : 1u);
    tc::mma_bf16(d, tc::desc_sw128(a_hi), tc::desc_sw128(b_lo), idesc, 1u);
    tc::mma_bf16(d, tc::desc_sw128(a_lo), tc::desc_sw128(b_hi), idesc, 1u);
}

// ------------------------------------------------------------------ inverse

struct InvTcArgs {
    const float2* in1;
    const float2* in2;
    long long ips;
    int irs;
    float* y;
    int Q, H, W, m1, m2, R2, N1, np, N4, Kg, ntiles;
    const uint4* g;
    const uint4* e;
    uint32_t g_bytes, e_bytes;
    uint32_t off_e, off_b4, off_a5, b4_half, a5_half, tmem_cols;
    int* watchdog;
};

__global__ void __launch_bounds__(kTcThreads, 1) dft_inv_tc_kernel(const InvTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    uint8_t* base = tc::align1024(smem_raw);
    uint8_t* sG = base;
    uint8_t* sE = base + a.off_e;
    uint8_t* sB4 = base + a.off_b4;
    uint8_t* sA5 = base + a.off_a5;  // np operands of 128 rows x one K block, hi | lo
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int W = a.W, H = a.H, N1 = a.N1, N4 = a.N4, np = a.np;

    tc::copy_table(sG, a.g, a.g_bytes);
    tc::copy_table(sE, a.e, a.e_bytes);
    {  // padded rows / K columns of the spectrum operand stay zero for the whole kernel
        uint4* z = reinterpret_cast<uint4*>(sB4);
        for (uint32_t i = tid; i < 2 * a.b4_half / 16; i += kTcThreads) z[i] = make_uint4(0, 0, 0, 0);
    }
    if (warp == 0) {
        tc::tmem_alloc(&tmem_base, a.tmem_cols);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        tc::mbar_init(&bar, 1);
        abort_flag = 0;
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base;
    const uint32_t d4 = tmem, d5 = tmem + static_cast<uint32_t>(N4);
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t phase = 0;
    const int m1 = a.m1, m2 = a.m2, S = 2 * m1;
    const uint32_t id4 = tc::idesc_bf16(128, N4), id5 = tc::idesc_bf16(128, W);

    for (int tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
        const int q0 = tile * np;
        // spectra -> Yr^T rows (plane, re|im, ky), K = slot | 2m1 + slot
        for (int o = tid; o < np * S * m2; o += kTcThreads) {
            const int pl = o / (S * m2);
            const int rem = o - pl * S * m2;
            const int s = rem / m2, ky = rem - s * m2;
            const int q = q0 + pl;
            float2 yv = make_float2(0.f, 0.f);
            if (q < a.Q)
                yv = s < m1 ? a.in1[q * a.ips + static_cast<long long>(s) * a.irs + ky]
                            : a.in2[q * a.ips + static_cast<long long>(s - m1) * a.irs + ky];
            const int rre = pl * N1 + ky, rim = rre + a.R2;
            const float vals[4] = {yv.x, -yv.y, yv.y, yv.x};
            const int rows[4] = {rre, rre, rim, rim};
            const int cols[4] = {s, S + s, s, S + s};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                __nv_bfloat16 hi, lo;
                tc::split2(vals[t], hi, lo);
                const uint32_t off = tc::kmajor_offset(N4, rows[t], cols[t]);
                *reinterpret_cast<__nv_bfloat16*>(sB4 + off) = hi;
                *reinterpret_cast<__nv_bfloat16*>(sB4 + a.b4_half + off) = lo;
            }
        }
        tc::fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
            const uint32_t A = tc::smem_u32(sG), B = tc::smem_u32(sB4);
            for (int k = 0; k < a.Kg / 16; ++k) {
                const uint32_t ao = tc::kmajor_offset(128, 0, k * 16), bo = tc::kmajor_offset(N4, 0, k * 16);
                mma3(d4, A + ao, A + a.g_bytes / 2 + ao, B + bo, B + a.b4_half + bo, id4, k == 0);
            }
            tc::mma_commit(&bar);
        }
        if (!cta_wait(&bar, phase, &abort_flag, a.watchdog, 3)) break;
        tc::fence_after_sync();
        // E4: D4 (lane = h) -> Z operand rows h of plane pl, K = c (re block | im block)
        {
            const int h = (warp & 3) * 32 + lane;
            const int half = warp >> 2;
            for (int c0 = half * 16; c0 < N4; c0 += 32) {
                float v[16];
                tc::tmem_ld16(d4 + lane_base + static_cast<uint32_t>(c0), v);
                const int pl = c0 / N1, c = c0 - pl * N1;
                uint8_t* dst = sA5 + static_cast<uint32_t>(pl) * 128u * 128u;
#pragma unroll
                for (int g8 = 0; g8 < 2; ++g8) {
                    uint4 hi, lo;
                    tc::split8(v + 8 * g8, hi, lo);
                    const uint32_t off = tc::kmajor_offset(128, h, c + 8 * g8);
                    *reinterpret_cast<uint4*>(dst + off) = hi;
                    *reinterpret_cast<uint4*>(dst + a.a5_half + off) = lo;
                }
            }
        }
        tc::fence_async_smem();
        tc::fence_before_sync();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
            const uint32_t A = tc::smem_u32(sA5), B = tc::smem_u32(sE);
            for (int pl = 0; pl < np; ++pl) {
                const uint32_t ap = A + static_cast<uint32_t>(pl) * 128u * 128u;
                for (int k = 0; k < N1 / 16; ++k) {
                    const uint32_t ao = tc::kmajor_offset(128, 0, k * 16), bo = tc::kmajor_offset(W, 0, k * 16);
                    mma3(d5 + static_cast<uint32_t>(pl * W), ap + ao, ap + a.a5_half + ao, B + bo,
                         B + a.e_bytes / 2 + bo, id5, k == 0);
                }
            }
            tc::mma_commit(&bar);
        }
        if (!cta_wait(&bar, phase, &abort_flag, a.watchdog, 4)) break;
        tc::fence_after_sync();
        // E5: D5 -> y rows
        {
            const int h = (warp & 3) * 32 + lane;
            const int half = warp >> 2;
            if ((warp & 3) * 32 < H) {  // warp-uniform: lanes below H hold rows of the tile
                for (int pl = 0; pl < np; ++pl) {
                    const int q = q0 + pl;
                    for (int c0 = half * 16; c0 < W; c0 += 32) {
                        float v[16];
                        tc::tmem_ld16(d5 + lane_base + static_cast<uint32_t>(pl * W + c0), v);
                        if (q < a.Q && h < H) {
                            float4* dst = reinterpret_cast<float4*>(a.y + (static_cast<long long>(q) * H + h) * W + c0);
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                __stcs(dst + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
                        }
                    }
                }
            }
        }
        tc::fence_before_sync();
        __syncthreads();
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, a.tmem_cols);
    }
}

}  // namespace

bool tc_inv_supported(int H, int W, int m1, int m2) {
    if (!((H == 64 || H == 128) && (W == 64 || W == 128) && m2 >= 1 && m2 <= 32 && m1 >= 1 && 4 * m1 <= 128))
        return false;
    const TcShape s = tc_shape(H, W, m1, m2);
    if (s.N2 > 256) return false;
    if (inv_smem_bytes(s) > kMaxDynSmem) return false;
    // inverse: D4 (N2 columns) and D5 (np*W columns) share one 256-column TMEM allocation
    if (s.N2 + s.np * W > 256) return false;
    return true;
}

cudaError_t launch_dft_inv_tc(const float2* in1, const float2* in2, long long ips, int irs, float* y, int Q,
                              int H, int W, int m1, int m2, cudaStream_t stream) {
    if (!tc_inv_supported(H, W, m1, m2) || (reinterpret_cast<uintptr_t>(y) & 15) != 0) return cudaErrorInvalidValue;
    const TcShape s = tc_shape(H, W, m1, m2);
    if (s.np * W > 256 - s.N2) return cudaErrorInvalidValue;  // D4 + D5 columns
    const TcTables* t = nullptr;
    cudaError_t e = get_tc_tables(s, &t);
    if (e != cudaSuccess) return e;
    InvTcArgs a;
    a.in1 = in1;
    a.in2 = in2;
    a.ips = ips;
    a.irs = irs;
    a.y = y;
    a.Q = Q;
    a.H = H;
    a.W = W;
    a.m1 = m1;
    a.m2 = m2;
    a.R2 = s.R2;
    a.N1 = s.N1;
    a.np = s.np;
    a.N4 = s.N2;
    a.Kg = s.Kg;
    a.ntiles = (Q + s.np - 1) / s.np;
    a.g = t->inv_g;
    a.e = t->inv_e;
    a.g_bytes = t->g_bytes;
    a.e_bytes = t->e_bytes;
    a.off_e = a.g_bytes;
    a.off_b4 = a.off_e + a.e_bytes;
    a.b4_half = static_cast<uint32_t>(s.N2) * static_cast<uint32_t>(round_up(s.Kg, 64)) * 2u;
    a.off_a5 = a.off_b4 + 2 * a.b4_half;
    a.a5_half = static_cast<uint32_t>(s.np) * 128u * 128u;
    const size_t smem = a.off_a5 + 2 * a.a5_half + 1024;
    a.tmem_cols = tmem_cols_for(s.N2 + s.np * W);
    e = device_watchdog(&a.watchdog);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = prepare_kernel(reinterpret_cast<const void*>(dft_inv_tc_kernel), smem, kTcThreads, &per_sm);
    if (e != cudaSuccess) return e;
    per_sm = std::min<int>(per_sm, static_cast<int>(512 / a.tmem_cols));
    const int grid = std::max(1, std::min(a.ntiles, per_sm * num_sms()));
    dft_inv_tc_kernel<<<grid, kTcThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace scx
