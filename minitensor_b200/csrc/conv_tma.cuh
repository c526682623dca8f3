// conv_tma.cuh -- Conv2D implicit GEMM with every operand tile loaded by TMA (sm_100a).
//
// With NCHW activations a shifted conv window is a run of pixels that starts at an
// arbitrary x, and TMA cannot start a box at an x that is not 16-byte aligned. With the
// channels innermost (NHWC) the shift lands in the x / y coordinates of a 4-D box
// {32 channels, TX pixels, TY rows, 1 image}, which have no alignment rule, and the
// padding comes for free from TMA's zero fill of out-of-range coordinates. So:
//
//   nchw_to_nhwc_kernel   x[N,C,H,W] (any strides) -> xt[N,H,W,Cp], Cp = C rounded to 4
//   reorder_weights_kernel W[Co,C,kh,kw] -> Wt[tap][row][col] K-major per tap
//   conv_fwd_tma_kernel   M = output pixels of TY rows x TX columns of one image (128
//                         TMEM lanes), N = C_out, K = (tap, 32-channel block); A and B are
//                         one TMA box each per stage. Stride 1. Input-grad (stride 1) is
//                         the same kernel on NHWC dy with flipped, transposed weights.
//   (conv_wgrad.cuh)      weight-grad: M = (tap, channel), N = C_out, K = output pixels;
//                         A = four 32-channel chunks of NHWC x (M-major), B = dy straight
//                         from NCHW. Split-K partials, then
//   wgrad_reduce_kernel   dW[co,c,r,s] = sum over splits (in order) of the partials.
//
// Warp roles as in the GEMM kernel: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-5
// epilogue, 6-9 (TF32X3) hi/lo splitter.
#pragma once

#include "mt_common.cuh"

namespace mt {
namespace convt {

// ------------------------------------------------------------------ layout kernels --
// One block per (64 channels x 64 columns) tile of one image row: each thread keeps 16
// loads in flight (coalesced along W), then 16 stores (coalesced along C) from a padded
// shared tile. Channels in [C, Cp) are written as zeros. Grid: x = column tiles,
// y = channel tiles, z strides over the N*H rows.
__global__ void __launch_bounds__(256) nchw_to_nhwc_kernel(const float* __restrict__ x, int64_t s0, int64_t s1,
                                                           int64_t s2, int64_t s3, float* __restrict__ xt, int N,
                                                           int C, int H, int W, int Cp) {
    __shared__ float tile[64][65];
    const int w0 = blockIdx.x * 64, c0 = blockIdx.y * 64;
    const int t = threadIdx.x;
    const int lo = t & 63, hi = t >> 6;   // 64 x 4
    for (int nh = blockIdx.z; nh < N * H; nh += gridDim.z) {
        const int n = nh / H, h = nh - n * H;
        const float* src = x + (int64_t)n * s0 + (int64_t)h * s2;
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int c = c0 + hi + 4 * i, w = w0 + lo;
            v[i] = (c < C && w < W) ? __ldg(src + (int64_t)c * s1 + (int64_t)w * s3) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) tile[hi + 4 * i][lo] = v[i];
        __syncthreads();
        float* row = xt + ((int64_t)n * H + h) * W * Cp;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int w = w0 + hi + 4 * i, c = c0 + lo;
            if (w < W && c < Cp) row[(int64_t)w * Cp + c] = tile[lo][hi + 4 * i];
        }
        __syncthreads();
    }
}

// Fast form for activations whose H x W plane is contiguous (and 16-byte aligned rows of
// channels): one block per (image, 32 channels, 256 pixels) moves 32 KB with 8 float4
// loads and 8 float4 stores per thread. The shared tile [32][256] stores element (c, p)
// at column p ^ (4 * ((c / 4) % 8)): float4 writes along p stay aligned and conflict-free,
// and the transposed reads (8 channel groups x 4 pixels per warp) hit 32 distinct banks.
// Requires HW % 4 == 0; channels in [C, Cp) are written as zeros.
__global__ void __launch_bounds__(256) nchw_to_nhwc_flat_kernel(const float* __restrict__ x, int64_t s0, int64_t s1,
                                                                float* __restrict__ xt, int N, int C, int HW, int Cp) {
    __shared__ __align__(16) float tile[32][256];
    const int p0 = blockIdx.x * 256, c0 = blockIdx.y * 32;
    const int t = threadIdx.x;
    for (int n = blockIdx.z; n < N; n += gridDim.z) {
        const float* src = x + (int64_t)n * s0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = t + 256 * k;
            const int c = i >> 6, q = i & 63;
            const int p = p0 + 4 * q;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c0 + c < C && p < HW) v = __ldg(reinterpret_cast<const float4*>(src + (int64_t)(c0 + c) * s1 + p));
            *reinterpret_cast<float4*>(&tile[c][(4 * q) ^ (4 * ((c >> 2) & 7))]) = v;
        }
        __syncthreads();
        float* dst = xt + (int64_t)n * HW * Cp;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = t + 256 * k;
            const int pl = i >> 3, cg = i & 7;
            const int p = p0 + pl, c = c0 + 4 * cg;
            const int col = pl ^ (4 * cg);
            if (p < HW && c < Cp)
                *reinterpret_cast<float4*>(dst + (int64_t)p * Cp + c) =
                    make_float4(tile[4 * cg][col], tile[4 * cg + 1][col], tile[4 * cg + 2][col], tile[4 * cg + 3][col]);
        }
        __syncthreads();
    }
}

// Wt[tap][row][col] (col padded to colsp with zeros), tap = r * kw + s:
//   forward:    row = co, col = ci, value W[co, ci, r, s]
//   input-grad: row = ci, col = co, value W[co, ci, kh-1-r, kw-1-s] (flipped, transposed)
// split != 0 writes the TF32X3 pair instead, Wt[tap][h][row][col] with h = 0 the tf32
// rounding hi = rna_tf32(v) and h = 1 the remainder lo = v - hi, so that one TMA box
// brings both halves of a weight tile and no kernel has to split weights again.
__global__ void reorder_weights_kernel(const float* __restrict__ w, int64_t s0, int64_t s1, int64_t s2, int64_t s3,
                                       float* __restrict__ wt, int Co, int C, int kh, int kw, int dgrad, int split) {
    const int rows = dgrad ? C : Co, cols = dgrad ? Co : C;
    const int colsp = (cols + 3) & ~3;
    const int64_t total = (int64_t)kh * kw * rows * colsp;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int col = (int)(i % colsp);
        const int64_t t2 = i / colsp;
        const int row = (int)(t2 % rows);
        const int tap = (int)(t2 / rows);
        const int r = tap / kw, s = tap - r * kw;
        float v = 0.f;
        if (col < cols) {
            v = dgrad ? __ldg(w + col * s0 + row * s1 + (kh - 1 - r) * s2 + (kw - 1 - s) * s3)
                      : __ldg(w + row * s0 + col * s1 + r * s2 + s * s3);
        }
        if (split) {
            const int64_t plane = (int64_t)rows * colsp;
            const int64_t o = (int64_t)tap * 2 * plane + (int64_t)row * colsp + col;
            const float hi = tf32_round(v);
            wt[o] = hi;
            wt[o + plane] = v - hi;
        } else {
            wt[i] = v;
        }
    }
}

// ------------------------------------------------------------------ shared config ---
template <int BN, bool X3, int STAGES>
struct Cfg {
    static constexpr int BM = 128, BKE = 32;
    static constexpr uint32_t A_BYTES = BM * BKE * 4;          // 16 KB (a box may fill less)
    static constexpr uint32_t B_BYTES = BN * BKE * 4;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr uint32_t RING_BYTES = STAGE_BYTES * STAGES * (X3 ? 2 : 1);
    static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr int THREADS = (X3 ? 10 : 6) * 32;
    static constexpr uint32_t BAR_BYTES = 8 * (3 * STAGES + 4) + 16;
    static constexpr uint32_t SMEM_BYTES = 1024 + RING_BYTES + BAR_BYTES;
};

struct FwdParams {
    int N, Ho, Wo, Ncol, C, kh, kw, pad;   // Ncol = output channels; C = input channels
    int TX, TY, tiles_y, tiles_x, tiles_n, cblocks, kblocks;
    long long num_tiles;
    uint32_t a_box_bytes;                  // 32 * TX * TY * 4
    float* out;                            // [N, Ncol, Ho, Wo] contiguous
    const float* bias;                     // [Ncol] or null
};

struct WgradParams {
    int N, Ho, Wo, C, Co, kh, kw, pad;
    int M, tiles_m, tiles_n, xblocks, kb_per_img, kb_total, splits;
    long long num_units;
    float* ws;                             // partials [splits][M][Cop], Cop = tiles_n * BN
    int ws_ld;
};

// ------------------------------------------------------------------ common pieces ---
struct Bars {
    uint64_t *full, *empty, *conv, *acc_full, *acc_empty;
    volatile uint32_t* tmem_slot;
    volatile int* abort_flag;
};

template <int STAGES>
__device__ __forceinline__ Bars carve_bars(uint8_t* base) {
    Bars b;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base);
    b.full = bars;
    b.empty = bars + STAGES;
    b.conv = bars + 2 * STAGES;
    b.acc_full = bars + 3 * STAGES;
    b.acc_empty = bars + 3 * STAGES + 2;
    b.tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 3 * STAGES + 4);
    b.abort_flag = reinterpret_cast<volatile int*>(bars + 3 * STAGES + 4) + 1;
    return b;
}

template <int STAGES>
__device__ __forceinline__ void init_bars(const Bars& b) {
    for (int s = 0; s < STAGES; ++s) {
        mbar_init(smem_u32(&b.full[s]), 1);
        mbar_init(smem_u32(&b.empty[s]), 1);
        mbar_init(smem_u32(&b.conv[s]), 128);
    }
    for (int a = 0; a < 2; ++a) {
        mbar_init(smem_u32(&b.acc_full[a]), 1);
        mbar_init(smem_u32(&b.acc_empty[a]), 128);
    }
    *b.abort_flag = 0;
    fence_barrier_init();
}

// TF32X3: split every landed stage into hi (in place) and lo (parallel ring).
template <int STAGES, uint32_t STAGE_BYTES>
__device__ __forceinline__ bool splitter_stage(const Bars& b, uint8_t* ring, uint8_t* ring_lo, int s, uint32_t ph,
                                               int ct) {
    if (!mbar_wait(smem_u32(&b.full[s]), ph, b.abort_flag, kDevTimeoutMisc)) return false;
    float4* hi = reinterpret_cast<float4*>(ring + s * STAGE_BYTES);
    float4* lo = reinterpret_cast<float4*>(ring_lo + s * STAGE_BYTES);
#pragma unroll 4
    for (uint32_t i = ct; i < STAGE_BYTES / 16; i += 128) {
        const float4 x = hi[i];
        const float4 h = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
        hi[i] = h;
        lo[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    }
    fence_proxy_async_smem();
    mbar_arrive(smem_u32(&b.conv[s]));
    return true;
}

// One stage of MMAs (4 k-steps of 8), 1 or 3 products per k-step.
template <bool A_MN, bool X3, uint32_t A_BYTES>
__device__ __forceinline__ void mma_stage(uint32_t d_tmem, uint32_t sa, uint32_t la, uint32_t idesc, bool first) {
    const uint32_t sb = sa + A_BYTES, lb = la + A_BYTES;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint64_t ad = A_MN ? umma_desc(sa + k * 1024, 32 * 128, 512, kLayoutSw128Base32)
                                 : umma_desc(sa + k * 32, 16, 1024, kLayoutSw128);
        const uint64_t bd = umma_desc(sb + k * 32, 16, 1024, kLayoutSw128);
        const uint32_t acc = (!first || k > 0) ? 1u : 0u;
        if (X3) {
            const uint64_t ald = A_MN ? umma_desc(la + k * 1024, 32 * 128, 512, kLayoutSw128Base32)
                                      : umma_desc(la + k * 32, 16, 1024, kLayoutSw128);
            const uint64_t bld = umma_desc(lb + k * 32, 16, 1024, kLayoutSw128);
            umma_tf32(d_tmem, ald, bd, idesc, acc);
            umma_tf32(d_tmem, ad, bld, idesc, 1u);
            umma_tf32(d_tmem, ad, bd, idesc, 1u);
        } else {
            umma_tf32(d_tmem, ad, bd, idesc, acc);
        }
    }
}

// ------------------------------------------------------------------ forward ---------
// Tile t -> (image, first output row, first output column, C_out block); the C_out block
// varies fastest so consecutive CTAs reuse the same activation boxes from L2.
__device__ __forceinline__ void fwd_tile(const FwdParams& p, long long t, int& n, int& y0, int& x0, int& nt) {
    long long r = t;
    nt = (int)(r % p.tiles_n); r /= p.tiles_n;
    const int xt = (int)(r % p.tiles_x); r /= p.tiles_x;
    const int yt = (int)(r % p.tiles_y); r /= p.tiles_y;
    n = (int)r;
    y0 = yt * p.TY;
    x0 = xt * p.TX;
}

template <int BN, bool X3, int STAGES>
__global__ void __launch_bounds__(Cfg<BN, X3, STAGES>::THREADS, 1)
conv_fwd_tma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const FwdParams p) {
    using G = Cfg<BN, X3, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;
    uint8_t* ring_lo = smem + G::STAGE_BYTES * STAGES;
    const Bars bb = carve_bars<STAGES>(smem + G::RING_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long first = blockIdx.x, step = gridDim.x;

    if (threadIdx.x == 0) init_bars<STAGES>(bb);
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)bb.tmem_slot), G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *bb.tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (long long t = first; t < p.num_tiles; t += step) {
                int n, y0, x0, nt;
                fwd_tile(p, t, n, y0, x0, nt);
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    const int tap = kb / p.cblocks, cb = kb - tap * p.cblocks;
                    const int r = tap / p.kw, sx = tap - r * p.kw;
                    if (!mbar_wait(smem_u32(&bb.empty[s]), ph ^ 1, bb.abort_flag, kDevTimeoutEmpty)) goto done;
                    const uint32_t bar = smem_u32(&bb.full[s]);
                    mbar_arrive_expect_tx(bar, p.a_box_bytes + G::B_BYTES);
                    const uint32_t sa = smem_u32(ring + s * G::STAGE_BYTES);
                    tma_load_4d(sa, &tmA, bar, cb * 32, x0 + sx - p.pad, y0 + r - p.pad, n);
                    tma_load_3d(sa + G::A_BYTES, &tmB, bar, cb * 32, nt * BN, tap);
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_tf32(128, BN, 0, 0);
            int s = 0, it = 0;
            uint32_t ph = 0;
            for (long long t = first; t < p.num_tiles; t += step, ++it) {
                const int a = it & 1;
                if (!mbar_wait(smem_u32(&bb.acc_empty[a]), ((it >> 1) & 1) ^ 1, bb.abort_flag, kDevTimeoutAccEmpty))
                    goto done;
                tc_fence_after();
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    const uint32_t wbar = X3 ? smem_u32(&bb.conv[s]) : smem_u32(&bb.full[s]);
                    if (!mbar_wait(wbar, ph, bb.abort_flag, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    mma_stage<false, X3, G::A_BYTES>(tmem_base + a * BN, smem_u32(ring + s * G::STAGE_BYTES),
                                                     smem_u32(ring_lo + s * G::STAGE_BYTES), idesc, kb == 0);
                    umma_commit(smem_u32(&bb.empty[s]));
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                umma_commit(smem_u32(&bb.acc_full[a]));
            }
        }
    } else if (warp < 6) {
        const int q = warp & 3;
        const int HoWo = p.Ho * p.Wo;
        int it = 0;
        for (long long t = first; t < p.num_tiles; t += step, ++it) {
            int n, y0, x0, nt;
            fwd_tile(p, t, n, y0, x0, nt);
            const int a = it & 1;
            if (!mbar_wait(smem_u32(&bb.acc_full[a]), (it >> 1) & 1, bb.abort_flag, kDevTimeoutAccFull)) goto done;
            __syncwarp();
            tc_fence_after();
            const int l = q * 32 + lane;             // TMEM lane = slot (ty, tx) of the tile
            const int ty = l / p.TX, tx = l - ty * p.TX;
            const int oy = y0 + ty, ox = x0 + tx;
            const bool valid = ty < p.TY && oy < p.Ho && ox < p.Wo;
            float* obase = p.out + (int64_t)n * p.Ncol * HoWo + (int64_t)oy * p.Wo + ox;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t rr[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + a * BN + c * 32, rr);
                tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    mbar_arrive(smem_u32(&bb.acc_empty[a]));
                }
                if (valid) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int co = nt * BN + c * 32 + j;
                        if (co < p.Ncol) {
                            float v = __uint_as_float(rr[j]);
                            if (p.bias) v = v + __ldg(p.bias + co);
                            obase[(int64_t)co * HoWo] = v;
                        }
                    }
                }
            }
        }
    } else if (X3) {
        const int ct = threadIdx.x - 6 * 32;
        int s = 0;
        uint32_t ph = 0;
        for (long long t = first; t < p.num_tiles; t += step)
            for (int kb = 0; kb < p.kblocks; ++kb) {
                if (!splitter_stage<STAGES, G::STAGE_BYTES>(bb, ring, ring_lo, s, ph, ct)) goto done;
                if (++s == STAGES) { s = 0; ph ^= 1; }
            }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, G::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ weight-grad -----
// The weight-gradient kernel itself lives in conv_wgrad.cuh; its partials are summed here.
// dW[co, c, r, s] = sum over splits (in order) of ws[split][(r*kw + s) * C + c][co].
// Threads run along C_out (the partials' contiguous dimension) so reads coalesce; the
// split loads are issued eight at a time ahead of the in-order sum.
__global__ void wgrad_reduce_kernel(const float* __restrict__ ws, int splits, int M, int ws_ld, float* __restrict__ dw,
                                    int Co, int C, int taps) {
    const int64_t total = (int64_t)M * Co;           // M = taps * C partial rows
    const int64_t plane = (int64_t)M * ws_ld;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int co = (int)(i % Co);
        const int m = (int)(i / Co);
        const int tap = m / C, c = m - tap * C;
        const float* src = ws + (int64_t)m * ws_ld + co;
        float acc = 0.f;
        if (splits <= 32) {
            // Every partial in flight at once (one L2 round trip), then added in split order.
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = j < splits ? __ldg(src + (int64_t)j * plane) : 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < splits) acc += v[j];
        } else {
            int sp = 0;
            for (; sp + 8 <= splits; sp += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __ldg(src + (int64_t)(sp + j) * plane);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc += v[j];
            }
            for (; sp < splits; ++sp) acc += __ldg(src + (int64_t)sp * plane);
        }
        dw[((int64_t)co * C + c) * taps + tap] = acc;
    }
}

}  // namespace convt
}  // namespace mt
