// Tensor-core (tcgen05, 3xTF32 -> fp32) dual-corner mode mixing for wide channel counts: the
// B200 replacement for spectral_mul_dual_packed_kernel (spectral_conv_combo/spectral_conv_ext.su:5-92)
// where Cin x Cout makes each mode a real dense contraction (64 output channels per tile).
//
// Per corner c and mode k the complex product y[b][o] = sum_i x[b][i] w[i][o] is one real GEMM
//
//   D[(s, o)][(b, t)] = sum_i W_s[i][o] X_t[b][i]        s, t in {re, im}
//   M = 128 rows: Wr^T and Wi^T of 64 output channels, the two parts of a channel 16 rows apart
//   (a_row); N = 2B: Xr and Xi of each batch item in adjacent rows
//   y_re[b][o] = D[(re,o)][(b,re)] - D[(im,o)][(b,im)],   y_im = D[(im,o)][(b,re)] + D[(re,o)][(b,im)]
//
// in 3xTF32: a*b ~= ah*bh + ah*bl + al*bh with ah = a with its 13 low mantissa bits cleared and
// al = a - ah.  Per mode and chunk of 8 input channels (one K = 8 step) two MMAs:
//   Ah x [Bh; Bl]   (N = 2*NB: columns [0, NB) get Ah*Bh, [NB, 2*NB) get Ah*Bl)
//   Al x Bh         (N = NB, accumulated onto the Ah*Bh columns)
// and the epilogue adds the two column blocks in that order, so results are reproducible.
//
// Operands arrive by TMA in the spectra's own layouts (x_c [B][Cin][modes], w_c [Cin][Cout]
// [modes], 4 modes = one 32-byte swizzled row per (channel, channel) pair) and are rewritten by
// the converter warps as K-major SW32 tf32 hi / lo operands of each mode, three chunks of
// operands in flight.  Tiles are (corner, 64 output channels, 4 modes); CTAs are persistent (one
// per SM) and the TMEM accumulators are double-buffered, so one tile's epilogue overlaps the
// next tile's MMAs.  The hand-offs between converters and MMA issuers wait without suspending
// (a suspended thread wakes late, and these waits are short).
//
// Warp roles (416 threads):
//   warp 0        lane 0: TMA producer (w boxes of the first ring stages before griddepcontrol.wait,
//                 the x boxes after it); the warp allocates and frees TMEM
//   warps 1..4    lane 0 of warp 1 + j issues the MMAs of mode j of every tile
//   warps 5..8    converters: ring stage -> the four modes' hi / lo operands
//   warps 9..12   epilogue: TMEM -> y, the two parts of each output channel combined with
//                 shuffles
// Every wait is bounded; a role that gives up stores a code in the watchdog word and leaves.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include <cuda.h>

#include "scx_internal.h"
#include "scx_tc.cuh"

namespace scx {
namespace {

constexpr int kMT = 4;          // modes per tile: a 32-byte row of 4 complex values
constexpr int kIC = 8;          // input channels per chunk: one tf32 K step
constexpr int kOB = 64;         // output channels per tile (M = 128: Wr and Wi rows)
constexpr int kStages = 4;      // TMA ring stages
constexpr int kOpSlots = 3;     // converted-operand slots (one chunk of four modes each)
constexpr int kIssueWarp = 1, kConvWarp = 1 + kMT, kEpiWarp = kConvWarp + 4;
constexpr int kThreads = (kEpiWarp + 4) * 32;  // 416
constexpr int kBarConv = 1, kBarEpi = 2;

// Row of the A operand (and TMEM lane of D) holding part s (0 = Wr, 1 = Wi) of output channel
// o of the tile: the two parts of one channel sit 16 lanes apart in the same warp, so the
// epilogue combines them with shuffles.
__host__ __device__ __forceinline__ int a_row(int s, int o) { return 32 * (o >> 4) + 16 * s + (o & 15); }

template <int NB>
struct TcMixCfg {
    static constexpr int BMAX = NB / 2;                                     // batch items per tile
    static constexpr uint32_t WBOX = static_cast<uint32_t>(kIC) * kOB * 32u;  // 16 KB
    static constexpr uint32_t XBOX_MAX = static_cast<uint32_t>(kIC) * BMAX * 32u;
    static constexpr uint32_t STAGE = (WBOX + XBOX_MAX + 1023u) / 1024u * 1024u;
    static constexpr uint32_t A_BYTES = 128u * 32u;                         // one of Ah / Al
    static constexpr uint32_t MODE_OP = 2u * A_BYTES + 2u * NB * 32u;       // Ah | Al | [Bh; Bl]
    static constexpr uint32_t OP_SLOT = kMT * MODE_OP;
    static constexpr uint32_t OFF_OP = kStages * STAGE;
    static constexpr uint32_t SMEM = OFF_OP + kOpSlots * OP_SLOT + 1024u;
    static constexpr uint32_t ACC_COLS = kMT * 2 * NB;                      // one accumulator buffer
    static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS <= 256 ? 256u : 512u;
    static_assert(SMEM <= 227u * 1024u - 256u, "shared memory budget");
    static_assert(2 * ACC_COLS <= 512, "TMEM budget");
    static_assert(MODE_OP % 256 == 0 && OFF_OP % 1024 == 0 && OP_SLOT % 256 == 0, "SW32 alignment");
};

struct MixTcArgs {
    float2* y[2];
    int B, Cin, Cout, NM;
    int n_mt, n_ob, ntiles;  // mode tiles and output-channel blocks per corner, tiles in total
    int* watchdog;
};

struct MixTcBars {
    uint64_t stgFull[kStages], stgEmpty[kStages];
    uint64_t opFull[kOpSlots], opEmpty[kOpSlots];
    uint64_t accFull[2], accEmpty[2];
    uint64_t drain[kMT];
};

// The hi / lo split of four values into the 16-byte units of one operand row.
__device__ __forceinline__ void put_split4(uint8_t* hi_base, uint8_t* lo_base, uint32_t off, float e0, float e1,
                                           float e2, float e3) {
    float4 hi, lo;
    tc::split_tf32(e0, hi.x, lo.x);
    tc::split_tf32(e1, hi.y, lo.y);
    tc::split_tf32(e2, hi.z, lo.z);
    tc::split_tf32(e3, hi.w, lo.w);
    *reinterpret_cast<float4*>(hi_base + off) = hi;
    *reinterpret_cast<float4*>(lo_base + off) = lo;
}

template <int NB>
__global__ void __launch_bounds__(kThreads, 1) mix_tc_kernel(const __grid_constant__ CUtensorMap tw0,
                                                             const __grid_constant__ CUtensorMap tw1,
                                                             const __grid_constant__ CUtensorMap tx0,
                                                             const __grid_constant__ CUtensorMap tx1,
                                                             const MixTcArgs a) {
    using C = TcMixCfg<NB>;
    extern __shared__ uint8_t mixtc_raw[];
    __shared__ MixTcBars bars;
    __shared__ uint32_t tmem_base;
    uint8_t* base = tc::align1024(mixtc_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int B = a.B, NCH = a.Cin / kIC;
    const uint32_t xbox = static_cast<uint32_t>(kIC) * B * 32u;
    // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...; tile -> (corner, o block, mode tile)
    const int my_tiles = a.ntiles > static_cast<int>(blockIdx.x)
                             ? (a.ntiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                             : 0;
    const int my_chunks = my_tiles * NCH;
    auto tile_of = [&](int i, int& corner, int& k0, int& o0) {
        const int t = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
        const int per_corner = a.n_mt * a.n_ob;
        corner = t / per_corner;
        const int r = t % per_corner;
        o0 = (r / a.n_mt) * kOB;
        k0 = (r % a.n_mt) * kMT;
    };

    if (tid == 0) tc::grid_dep_launch();
    if (warp == 0) {
        tc::tmem_alloc(&tmem_base, C::TMEM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 32) {
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&bars.stgFull[i], 1);
            tc::mbar_init(&bars.stgEmpty[i], 1);
        }
        for (int i = 0; i < kOpSlots; ++i) {
            tc::mbar_init(&bars.opFull[i], 1);
            tc::mbar_init(&bars.opEmpty[i], kMT);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&bars.accFull[i], kMT);
            tc::mbar_init(&bars.accEmpty[i], 1);
        }
        for (int i = 0; i < kMT; ++i) tc::mbar_init(&bars.drain[i], 1);
        tc::fence_async_smem();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------------------- TMA producer
            auto load_w = [&](int g) {
                int corner, k0, o0;
                tile_of(g / NCH, corner, k0, o0);
                const int s = g % kStages;
                tc::mbar_arrive_expect_tx(&bars.stgFull[s], C::WBOX + xbox);
                tc::tma_load_3d(base + s * C::STAGE, corner ? &tw1 : &tw0, 2 * k0, o0, (g % NCH) * kIC,
                                &bars.stgFull[s]);
            };
            auto load_x = [&](int g) {
                int corner, k0, o0;
                tile_of(g / NCH, corner, k0, o0);
                const int s = g % kStages;
                tc::tma_load_3d(base + s * C::STAGE + C::WBOX, corner ? &tx1 : &tx0, 2 * k0, 0, (g % NCH) * kIC,
                                &bars.stgFull[s]);
            };
            // the weights are not written by the previous kernel in the stream: the first stages'
            // w boxes are requested before waiting for it, the x boxes after
            const int first = min(my_chunks, kStages);
            for (int g = 0; g < first; ++g) load_w(g);
            tc::grid_dep_wait();
            for (int g = 0; g < first; ++g) load_x(g);
            for (int g = first; g < my_chunks; ++g) {
                const int s = g % kStages;
                if (!tc::mbar_wait_spin(&bars.stgEmpty[s], ((g / kStages) & 1) ^ 1)) {
                    atomicExch(a.watchdog, 50);
                    break;
                }
                load_w(g);
                load_x(g);
            }
        }
    } else if (warp < kConvWarp) {
        // ---------------------------------------------------------------- MMA issuers
        if (lane == 0) {
            const int j = warp - kIssueWarp;  // this warp's mode within a tile
            const uint32_t sb = tc::smem_u32(base + C::OFF_OP) + static_cast<uint32_t>(j) * C::MODE_OP;
            constexpr uint32_t id1 = tc::idesc_tf32(128, 2 * NB), id2 = tc::idesc_tf32(128, NB);
            bool ok = true;
            int g = 0;
            for (int i = 0; i < my_tiles && ok; ++i) {
                const int tb = i & 1;
                ok = tc::mbar_wait_bounded(&bars.accEmpty[tb], ((i >> 1) & 1) ^ 1);
                const uint32_t d = tmem + static_cast<uint32_t>(tb) * C::ACC_COLS + static_cast<uint32_t>(j) * 2u * NB;
                for (int c = 0; c < NCH && ok; ++c, ++g) {
                    const int os = g % kOpSlots;
                    ok = tc::mbar_wait_spin(&bars.opFull[os], (g / kOpSlots) & 1);
                    if (!ok) break;
                    tc::fence_after_sync();
                    const uint32_t sa = sb + static_cast<uint32_t>(os) * C::OP_SLOT;
                    tc::mma_tf32(d, tc::desc_sw32(sa), tc::desc_sw32(sa + 2u * C::A_BYTES), id1, c > 0 ? 1u : 0u);
                    tc::mma_tf32(d, tc::desc_sw32(sa + C::A_BYTES), tc::desc_sw32(sa + 2u * C::A_BYTES), id2, 1u);
                    tc::mma_commit(&bars.opEmpty[os]);
                }
                if (ok) tc::mma_commit(&bars.accFull[tb]);
            }
            if (!ok) atomicExch(a.watchdog, 51);
            // every MMA of this thread has completed before TMEM is released
            tc::mma_commit(&bars.drain[j]);
            tc::mbar_wait_bounded(&bars.drain[j], 0);
        }
    } else if (warp < kEpiWarp) {
        // ---------------------------------------------------------------- converters
        // W: thread (o, pair) rewrites rows a_row(0, o) (Wr) and a_row(1, o) (Wi) of modes 2 pair
        // and 2 pair + 1.  X: 2B items (b, pair) spread over the four warps, rows 2b (Xr) and
        // 2b + 1 (Xi) of Bh and NB + 2b, NB + 2b + 1 of Bl.
        const int ct = tid - kConvWarp * 32;
        const int o = ct & 63, wp = ct >> 6;
        const int xi = (ct & 31) * 4 + (ct >> 5);
        bool ok = true;
        for (int g = 0; g < my_chunks; ++g) {
            const int s = g % kStages, os = g % kOpSlots;
            bool w8 = tc::mbar_wait_spin(&bars.stgFull[s], (g / kStages) & 1);
            w8 = w8 && tc::mbar_wait_spin(&bars.opEmpty[os], ((g / kOpSlots) & 1) ^ 1);
            if (tc::named_any(kBarConv, 128, !w8)) {
                ok = false;
                break;
            }
            const uint8_t* stg = base + s * C::STAGE;
            uint8_t* op = base + C::OFF_OP + os * C::OP_SLOT;
            {
                float4 v[kIC];
#pragma unroll
                for (int i = 0; i < kIC; ++i) {
                    const int row = i * kOB + o;
                    v[i] = *reinterpret_cast<const float4*>(stg + row * 32 + ((wp ^ ((row >> 2) & 1)) << 4));
                }
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    uint8_t* mo = op + (2 * wp + m) * C::MODE_OP;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const float4 &u0 = v[4 * h], &u1 = v[4 * h + 1], &u2 = v[4 * h + 2], &u3 = v[4 * h + 3];
                        const uint32_t offr = tc::sw32_offset(a_row(0, o), h), offi = tc::sw32_offset(a_row(1, o), h);
                        if (m == 0) {
                            put_split4(mo, mo + C::A_BYTES, offr, u0.x, u1.x, u2.x, u3.x);
                            put_split4(mo, mo + C::A_BYTES, offi, u0.y, u1.y, u2.y, u3.y);
                        } else {
                            put_split4(mo, mo + C::A_BYTES, offr, u0.z, u1.z, u2.z, u3.z);
                            put_split4(mo, mo + C::A_BYTES, offi, u0.w, u1.w, u2.w, u3.w);
                        }
                    }
                }
            }
            if (xi < 2 * B) {
                const int b = xi % B, xp = xi / B;
                float4 v[kIC];
#pragma unroll
                for (int i = 0; i < kIC; ++i) {
                    const int row = i * B + b;
                    v[i] = *reinterpret_cast<const float4*>(stg + C::WBOX + row * 32 + ((xp ^ ((row >> 2) & 1)) << 4));
                }
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    uint8_t* bo = op + (2 * xp + m) * C::MODE_OP + 2u * C::A_BYTES;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const float4 &u0 = v[4 * h], &u1 = v[4 * h + 1], &u2 = v[4 * h + 2], &u3 = v[4 * h + 3];
                        const int nr = 2 * b, ni = 2 * b + 1;
                        if (m == 0) {
                            put_split4(bo, bo + (NB / 8) * 256, tc::sw32_offset(nr, h), u0.x, u1.x, u2.x, u3.x);
                            put_split4(bo, bo + (NB / 8) * 256, tc::sw32_offset(ni, h), u0.y, u1.y, u2.y, u3.y);
                        } else {
                            put_split4(bo, bo + (NB / 8) * 256, tc::sw32_offset(nr, h), u0.z, u1.z, u2.z, u3.z);
                            put_split4(bo, bo + (NB / 8) * 256, tc::sw32_offset(ni, h), u0.w, u1.w, u2.w, u3.w);
                        }
                    }
                }
            }
            tc::fence_async_smem();  // this thread's operand writes -> the tensor core
            tc::named_sync(kBarConv, 128);
            if (ct == 0) {
                tc::mbar_arrive(&bars.stgEmpty[s]);
                tc::mbar_arrive(&bars.opFull[os]);
            }
        }
        if (!ok && ct == 0) atomicExch(a.watchdog, 52);
    } else {
        // ---------------------------------------------------------------- epilogue
        // Lane l of warp q holds D row 32q + l: part s = l / 16 of output channel 16q + l % 16,
        // columns 2b (times Xr) and 2b + 1 (times Xi), plus the Ah*Bl correction NB columns on.
        // y_re = Wr.Xr - Wi.Xi and y_im = Wi.Xr + Wr.Xi combine the two parts 16 lanes apart:
        // of each batch pair (2t, 2t + 1) the Wr lane finishes 2t and the Wi lane 2t + 1.
        const int et = tid - kEpiWarp * 32;
        const int q = warp & 3, part = (lane >> 4) & 1;
        const int ol = 16 * q + (lane & 15);
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        bool ok = true;
        for (int i = 0; i < my_tiles; ++i) {
            int corner, k0, o0;
            tile_of(i, corner, k0, o0);
            const int tb = i & 1;
            const bool w8 = tc::mbar_wait_bounded(&bars.accFull[tb], (i >> 1) & 1);
            if (tc::named_any(kBarEpi, 128, !w8)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            float2* __restrict__ Y = corner ? a.y[1] : a.y[0];
#pragma unroll 1
            for (int j = 0; j < kMT; ++j) {
                const uint32_t col = tmem + lane_addr + static_cast<uint32_t>(tb) * C::ACC_COLS +
                                     static_cast<uint32_t>(j) * 2u * NB;
                float d[NB];
#pragma unroll
                for (int hh = 0; hh < NB / 16; ++hh) {
                    float e[16];
                    tc::tmem_ld_cols_nowait<16>(col + 16 * hh, d + 16 * hh);
                    tc::tmem_ld_cols_nowait<16>(col + NB + 16 * hh, e);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int n = 0; n < 16; ++n) d[16 * hh + n] += e[n];
                }
                const int k = k0 + j;
                float2* yrow = Y + static_cast<size_t>(o0 + ol) * a.NM + k;
                const size_t bstride = static_cast<size_t>(a.Cout) * a.NM;
#pragma unroll
                for (int t = 0; t < NB / 4; ++t) {
                    const float r1 = __shfl_xor_sync(0xffffffffu, part ? d[4 * t] : d[4 * t + 2], 16);
                    const float r2 = __shfl_xor_sync(0xffffffffu, part ? d[4 * t + 1] : d[4 * t + 3], 16);
                    const float yr = part ? r1 - d[4 * t + 3] : d[4 * t] - r2;
                    const float yi = part ? d[4 * t + 2] + r2 : r1 + d[4 * t + 1];
                    const int b = 2 * t + part;
                    if (b < B && k < a.NM) yrow[static_cast<size_t>(b) * bstride] = make_float2(yr, yi);
                }
            }
            tc::fence_before_sync();
            tc::named_sync(kBarEpi, 128);
            if (et == 0) tc::mbar_arrive(&bars.accEmpty[tb]);
        }
        if (!ok && et == 0) atomicExch(a.watchdog, 53);
    }
    __syncwarp();
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 3-D fp32 map with dims (d0 innermost, d1, d2), byte strides s1, s2 of dims 1 and 2 (any
// order), box (b0, b1, b2), 32-byte swizzle (b0 = 8 floats = one swizzle row).
bool encode_sw32(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
                 uint32_t b0, uint32_t b1, uint32_t b2) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {s1, s2};
    const cuuint32_t box[3] = {b0, b1, b2};
    const cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NB>
cudaError_t run_mix_tc(const float2* const xs[2], const float2* const ws[2], float2* const ys[2], int ncorner, int B,
                       int Cin, int Cout, int NM, cudaStream_t stream) {
    using C = TcMixCfg<NB>;
    const auto kernel = mix_tc_kernel<NB>;
    int per_sm = 1;
    cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(kernel), C::SMEM, kThreads, &per_sm);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    MixTcArgs a;
    a.y[0] = ys[0];
    a.y[1] = ys[1];
    a.B = B;
    a.Cin = Cin;
    a.Cout = Cout;
    a.NM = NM;
    a.n_mt = (NM + kMT - 1) / kMT;
    a.n_ob = Cout / kOB;
    a.ntiles = ncorner * a.n_mt * a.n_ob;
    e = device_watchdog(&a.watchdog);
    if (e != cudaSuccess) return e;
    const uint64_t row = 2ull * NM * 4ull;  // bytes between consecutive channels of one mode row
    CUtensorMap tw[2], tx[2];
    for (int c = 0; c < 2; ++c) {
        const int src = c < ncorner ? c : 0;  // an unused second corner repeats the first maps
        // w_c [Cin][Cout][2 NM]: box (4 modes, 64 o, 8 i) -> shared [i][o][32 B]
        // x_c [B][Cin][2 NM] seen as (modes, b, i): box (4 modes, B, 8 i) -> shared [i][b][32 B]
        if (!encode_sw32(&tw[c], ws[src], 2ull * NM, Cout, Cin, row, row * Cout, 2 * kMT, kOB, kIC) ||
            !encode_sw32(&tx[c], xs[src], 2ull * NM, B, Cin, row * Cin, row, 2 * kMT, B, kIC))
            return cudaErrorNotSupported;
    }
    const int grid = std::max(1, std::min(a.ntiles, num_sms()));
    void* args[] = {&tw[0], &tw[1], &tx[0], &tx[1], &a};
    return launch_chained_raw(reinterpret_cast<const void*>(kernel), dim3(grid), dim3(kThreads), C::SMEM, stream,
                              args);
}

}  // namespace

bool mix_tc_supported(int B, int Cin, int Cout, int NM) {
    return B >= 1 && B <= 16 && Cin >= kIC && Cin % kIC == 0 && Cout >= kOB && Cout % kOB == 0 && NM >= 2 &&
           NM % 2 == 0;
}

cudaError_t launch_mix_tc(const float2* x1, const float2* x2, const float2* w1, const float2* w2, float2* y1,
                          float2* y2, int ncorner, int B, int Cin, int Cout, int NM, cudaStream_t stream) {
    if (!mix_tc_supported(B, Cin, Cout, NM) || ncorner < 1 || ncorner > 2) return cudaErrorNotSupported;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x1) | reinterpret_cast<uintptr_t>(w1) |
                         reinterpret_cast<uintptr_t>(y1) |
                         (ncorner == 2 ? (reinterpret_cast<uintptr_t>(x2) | reinterpret_cast<uintptr_t>(w2) |
                                          reinterpret_cast<uintptr_t>(y2))
                                       : 0);
    if ((al & 15) != 0) return cudaErrorNotSupported;
    const float2* xs[2] = {x1, x2};
    const float2* ws[2] = {w1, w2};
    float2* ys[2] = {y1, y2};
    if (2 * B <= 16) return run_mix_tc<16>(xs, ws, ys, ncorner, B, Cin, Cout, NM, stream);
    return run_mix_tc<32>(xs, ws, ys, ncorner, B, Cin, Cout, NM, stream);
}

}  // namespace scx
