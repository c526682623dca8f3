// conv_gemm.cuh -- Conv2D as implicit GEMM on tcgen05 (sm_100a), NCHW in place.
//
// The reference lowers conv to im2col + a SIMT GEMM (src/gpu_ops.cpp:2237-2325 forward,
// :2623-2713 weight-grad, :2499-2550 input-grad), materialising a col buffer in HBM.
// Here the col tiles never exist in HBM: four producer warps gather them from the NCHW
// tensors straight into the swizzled shared-memory layout the MMA reads, one pipeline
// stage at a time, and (for TF32X3) split each element into hi/lo on the way.
//
//   kind      GEMM rows (M, TMEM lanes)   cols (N)      reduction (K)        output
//   FWD       output pixels n,oy,ox       C_out         c_in, r, s           y[n,co,oy,ox] (+bias)
//   DGRAD     input pixels n,iy,ix        C_in          c_out, r, s          dx[n,ci,iy,ix]
//   WGRAD     c_in, r, s                  C_out         output pixels        dW[co,ci,r,s]
//
// FWD/DGRAD: the A tile (128 pixels x 32 k) is M-major -- lane i of a producer warp owns
// pixel i, so each warp-wide load reads consecutive pixels (coalesced) and each warp-wide
// store fills one 128-byte smem row (conflict-free). The output is written by the same
// pixel-per-lane mapping, so every store instruction covers 32 consecutive pixels.
// WGRAD: the A tile (128 rows (c,r,s) x 32 pixels) is K-major, lane = pixel again; K is
// split over blocks of 32 output pixels (never straddling an image) into `splits`
// contiguous ranges whose fp32 partials go to a workspace and are summed in split order
// by splitk_reduce_kernel (deterministic).
//
// Warp roles: 0 idle (keeps warp ids aligned), 1 MMA issuer + TMEM owner, 2-5 epilogue,
// 6-9 gather producers.
#pragma once

#include "mt_common.cuh"

namespace mt {
namespace conv {

enum Kind : int { kFwd = 0, kDgrad = 1, kWgrad = 2 };

struct Params {
    // Tensors (element strides, NCHW order). For FWD: src = x, wt = weight, dst = y.
    // DGRAD: src = dy, wt = weight, dst = dx. WGRAD: src = x, wt = dy, dst = workspace or dW.
    const float* x;  int64_t sx[4];      // input activations [N, C, H, W]
    const float* w;  int64_t sw[4];      // weight [Co, C, kh, kw]
    const float* dy; int64_t sdy[4];     // output gradient [N, Co, Ho, Wo]
    float* out;                          // y / dx (contiguous NCHW) or partials [splits][Co][C*kh*kw]
    const float* bias;                   // FWD only, may be null
    int N, C, H, W, Co, kh, kw, stride, pad, Ho, Wo;
    int M, Ncol, K;                      // GEMM extents
    int tiles_m, tiles_n;
    int splits, kb_per_img, kb_total;    // WGRAD split-K over 32-pixel blocks
    long long num_units;                 // tiles_m * tiles_n * splits
};

template <int BN, bool X3, int STAGES>
struct Cfg {
    static constexpr int BM = 128, BKE = 32;
    static constexpr uint32_t A_BYTES = BM * BKE * 4;          // 16 KB
    static constexpr uint32_t B_BYTES = BN * BKE * 4;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr uint32_t RING_BYTES = STAGE_BYTES * STAGES * (X3 ? 2 : 1);
    static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr int THREADS = 10 * 32;
    static constexpr uint32_t BAR_BYTES = 8 * (2 * STAGES + 4) + 16;
    static constexpr uint32_t SMEM_BYTES = 1024 + RING_BYTES + BAR_BYTES;
};

// Unit u -> (m tile, n tile, split).
__device__ __forceinline__ void unit_coords(const Params& p, long long u, int& mt, int& nt, int& sp) {
    sp = (int)(u % p.splits);
    long long r = u / p.splits;
    nt = (int)(r % p.tiles_n);
    mt = (int)(r / p.tiles_n);
}

__device__ __forceinline__ void kb_range(const Params& p, int sp, int& kb0, int& kb1) {
    // Reduction blocks of this split: FWD/DGRAD have one split over ceil(K/32) blocks;
    // WGRAD splits kb_total pixel blocks into `splits` near-equal contiguous ranges.
    const int total = p.kb_total;
    kb0 = (int)((long long)total * sp / p.splits);
    kb1 = (int)((long long)total * (sp + 1) / p.splits);
}

// Swizzled byte offsets inside one operand tile.
// MN-major (layout 1): 32-element chunks of 32 k-rows; granule (32 B) ^= row & 3.
__device__ __forceinline__ uint32_t off_mn(int mn, int k) {
    const int chunk = mn >> 5, e = mn & 31;
    return chunk * (32 * 128) + k * 128 + ((((e >> 3) ^ (k & 3)) << 5) | ((e & 7) << 2));
}
// K-major 128-byte swizzle (layout 2): row of 32 k; granule (16 B) ^= row & 7.
__device__ __forceinline__ uint32_t off_k(int row, int k) {
    return row * 128 + ((((k >> 2) ^ (row & 7)) << 4) | ((k & 3) << 2));
}

// ------------------------------------------------------------------------------------
// Producers. issue() starts the asynchronous copies (cp.async, 4 bytes each, zero-fill for
// padding and tile edges) of the A (128 x 32) and B (BN x 32) tiles of reduction block kb
// straight into their swizzled slots; finish() runs once they have landed: for TF32X3 it
// splits every element this thread copied into hi (in place) and lo (the parallel ring).
// t = producer thread 0..127, lane = t & 31, pw = t >> 5. Element offsets are 32-bit: the
// host checks that every view spans fewer than 2^31 elements.
// ------------------------------------------------------------------------------------
template <int KIND, int BN>
__device__ __forceinline__ void issue(const Params& p, int m0, int n0, int kb, int t, uint32_t a, uint32_t b) {
    const int lane = t & 31, pw = t >> 5;
    const int khkw = p.kh * p.kw;
    if (KIND == kFwd || KIND == kDgrad) {
        // ---- A: pixel m = m0 + t, k-rows k0..k0+31, k = (c, r, s) ----
        const int m = m0 + t;
        const bool mv = m < p.M;
        const int HW = (KIND == kFwd) ? p.Ho * p.Wo : p.H * p.W;
        const int wdim = (KIND == kFwd) ? p.Wo : p.W;
        const int img = mv ? m / HW : 0;
        const int pix = mv ? m - img * HW : 0;
        const int py = pix / wdim, px = pix - py * wdim;
        const int k0 = kb * 32;
        int c = k0 / khkw, rs = k0 - c * khkw;
        int r = rs / p.kw, s = rs - r * p.kw;
        if (KIND == kFwd) {
            const int s1 = (int)p.sx[1], s2 = (int)p.sx[2], s3 = (int)p.sx[3];
            const float* base = p.x + (int64_t)img * p.sx[0];
            const int iy0 = py * p.stride - p.pad, ix0 = px * p.stride - p.pad;
            int off = c * s1 + r * s2 + s * s3;          // x offset of tap (c, r, s), image-relative
            const int pixoff = iy0 * s2 + ix0 * s3;
#pragma unroll 8
            for (int kk = 0; kk < 32; ++kk) {
                const bool v = mv && (k0 + kk < p.K) && (unsigned)(iy0 + r) < (unsigned)p.H &&
                               (unsigned)(ix0 + s) < (unsigned)p.W;
                cp_async4(a + off_mn(t, kk), v ? base + (pixoff + off) : p.x, v);
                off += s3;
                if (++s == p.kw) {
                    s = 0; off += s2 - p.kw * s3;
                    if (++r == p.kh) { r = 0; off += s1 - p.kh * s2; }
                }
            }
        } else {
            // dx[iy,ix] gathers dy[oy,ox] with oy*stride - pad + r == iy.
            const float* base = p.dy + (int64_t)img * p.sdy[0];
            const int s1 = (int)p.sdy[1], s2 = (int)p.sdy[2], s3 = (int)p.sdy[3];
#pragma unroll 8
            for (int kk = 0; kk < 32; ++kk) {
                const int ny = py + p.pad - r, nx = px + p.pad - s;
                bool v = mv && (k0 + kk < p.K) && ny >= 0 && nx >= 0;
                int oy = ny, ox = nx;
                if (p.stride != 1) {
                    v = v && (ny % p.stride == 0) && (nx % p.stride == 0);
                    oy = ny / p.stride;
                    ox = nx / p.stride;
                }
                v = v && oy < p.Ho && ox < p.Wo;
                cp_async4(a + off_mn(t, kk), v ? base + (c * s1 + oy * s2 + ox * s3) : p.dy, v);
                if (++s == p.kw) { s = 0; if (++r == p.kh) { r = 0; ++c; } }
            }
        }
        // ---- B: rows n (C_out for FWD, C_in for DGRAD), k = lane ----
        const int k = k0 + lane;
        const bool kv = k < p.K;
        int koff = 0;            // weight offset of this k (rows add n * nstride)
        if (kv) {
            const int bc = k / khkw, q = k - bc * khkw, br = q / p.kw, bs = q - br * p.kw;
            // FWD: W[co = n, ci = bc, r, s];  DGRAD: W[co = bc, ci = n, r, s]
            koff = (int)((KIND == kFwd ? bc * p.sw[1] : bc * p.sw[0]) + br * p.sw[2] + bs * p.sw[3]);
        }
        const int nstride = (int)((KIND == kFwd) ? p.sw[0] : p.sw[1]);
#pragma unroll 4
        for (int row = pw; row < BN; row += 4) {
            const int n = n0 + row;
            const bool v = kv && n < p.Ncol;
            cp_async4(b + off_k(row, lane), v ? p.w + (koff + n * nstride) : p.w, v);
        }
    } else {
        // ---- WGRAD: reduction block kb = 32 output pixels of one image ----
        const int img = kb / p.kb_per_img;
        const int p0 = (kb - img * p.kb_per_img) * 32;
        const int pix = p0 + lane;
        const bool pv = pix < p.Ho * p.Wo;
        const int oy = pv ? pix / p.Wo : 0, ox = pv ? pix - (pix / p.Wo) * p.Wo : 0;
        // A rows m = (ci, r, s); warp pw covers rows pw*32 .. pw*32+31.
        const int mrow0 = m0 + pw * 32;
        int c = mrow0 / khkw, rs = mrow0 - c * khkw;
        int r = rs / p.kw, s = rs - r * p.kw;
        const int s1 = (int)p.sx[1], s2 = (int)p.sx[2], s3 = (int)p.sx[3];
        const float* xb = p.x + (int64_t)img * p.sx[0];
        const int iy0 = oy * p.stride - p.pad, ix0 = ox * p.stride - p.pad;
        const int pixoff = iy0 * s2 + ix0 * s3;
        int off = c * s1 + r * s2 + s * s3;
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
            const bool v = pv && mrow0 + i < p.M && (unsigned)(iy0 + r) < (unsigned)p.H &&
                           (unsigned)(ix0 + s) < (unsigned)p.W;
            cp_async4(a + off_k(pw * 32 + i, lane), v ? xb + (pixoff + off) : p.x, v);
            off += s3;
            if (++s == p.kw) {
                s = 0; off += s2 - p.kw * s3;
                if (++r == p.kh) { r = 0; off += s1 - p.kh * s2; }
            }
        }
        // B rows = co, k = pixel (dy[img, co, oy, ox]).
        const float* db = p.dy + (int64_t)img * p.sdy[0] + oy * p.sdy[2] + ox * p.sdy[3];
        const int cs = (int)p.sdy[1];
#pragma unroll 4
        for (int row = pw; row < BN; row += 4) {
            const int co = n0 + row;
            const bool v = pv && co < p.Ncol;
            cp_async4(b + off_k(row, lane), v ? db + co * cs : p.dy, v);
        }
    }
}

// 3xTF32: hi = rna_tf32(x) in place, lo = x - hi into the lo ring, for exactly the slots
// this thread's issue() filled.
template <int KIND, int BN>
__device__ __forceinline__ void split_slots(int t, uint8_t* a, uint8_t* al, uint8_t* b, uint8_t* bl) {
    const int lane = t & 31, pw = t >> 5;
    auto split = [](uint8_t* hi, uint8_t* lo, uint32_t off) {
        const float x = *reinterpret_cast<float*>(hi + off);
        const float h = tf32_round(x);
        *reinterpret_cast<float*>(hi + off) = h;
        *reinterpret_cast<float*>(lo + off) = x - h;
    };
    if (KIND == kFwd || KIND == kDgrad) {
#pragma unroll 8
        for (int kk = 0; kk < 32; ++kk) split(a, al, off_mn(t, kk));
    } else {
#pragma unroll 8
        for (int i = 0; i < 32; ++i) split(a, al, off_k(pw * 32 + i, lane));
    }
#pragma unroll 4
    for (int row = pw; row < BN; row += 4) split(b, bl, off_k(row, lane));
}

template <int KIND, int BN, bool X3, int STAGES>
__global__ void __launch_bounds__(Cfg<BN, X3, STAGES>::THREADS, 1) conv_kernel(const Params p) {
    using G = Cfg<BN, X3, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;
    uint8_t* ring_lo = smem + G::STAGE_BYTES * STAGES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::RING_BYTES);
    uint64_t* full = bars;                    // producers filled the stage (count 128)
    uint64_t* empty = bars + STAGES;          // MMA done with the stage
    uint64_t* acc_full = bars + 2 * STAGES;   // [2]
    uint64_t* acc_empty = bars + 2 * STAGES + 2;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 2 * STAGES + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 4) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long first = blockIdx.x, step = gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 128);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&acc_full[a]), 1);
            mbar_init(smem_u32(&acc_empty[a]), 128);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)tmem_slot), G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp >= 6) {
        // ------------------------------ gather producers ---------------------------
        // Each thread keeps up to DEPTH stages of copies in flight: stage i is handed to
        // the MMA issuer (split for 3xTF32, proxy fence, arrive on full) once the copies of
        // stage i + DEPTH - 1 have been issued. DEPTH < STAGES, so the stage whose empty
        // barrier the producer waits on was handed over long before (no cycle).
        constexpr int DEPTH = (STAGES - 1) < 3 ? (STAGES - 1) : 3;
        const int t = threadIdx.x - 6 * 32;
        int s_issue = 0, s_done = 0, inflight = 0;
        uint32_t ph = 0;
        auto hand_over = [&]() {
            uint8_t* a = ring + s_done * G::STAGE_BYTES;
            if (X3) {
                uint8_t* al = ring_lo + s_done * G::STAGE_BYTES;
                split_slots<KIND, BN>(t, a, al, a + G::A_BYTES, al + G::A_BYTES);
            }
            fence_proxy_async_smem();
            mbar_arrive(smem_u32(&full[s_done]));
            if (++s_done == STAGES) s_done = 0;
            --inflight;
        };
        for (long long u = first; u < p.num_units; u += step) {
            int mt, nt, sp, kb0, kb1;
            unit_coords(p, u, mt, nt, sp);
            kb_range(p, sp, kb0, kb1);
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(smem_u32(&empty[s_issue]), ph ^ 1, abort_flag, kDevTimeoutEmpty)) goto done;
                const uint32_t a = smem_u32(ring + s_issue * G::STAGE_BYTES);
                issue<KIND, BN>(p, mt * G::BM, nt * BN, kb, t, a, a + G::A_BYTES);
                cp_async_commit();
                if (++s_issue == STAGES) { s_issue = 0; ph ^= 1; }
                if (++inflight == DEPTH) {
                    cp_async_wait<DEPTH - 1>();
                    hand_over();
                }
            }
        }
        cp_async_wait<0>();
        while (inflight > 0) hand_over();
    } else if (warp == 1) {
        // ------------------------------ MMA issuer --------------------------------
        if (lane == 0) {
            constexpr bool A_MN = (KIND != kWgrad);
            constexpr uint32_t idesc = umma_idesc_tf32(128, BN, A_MN ? 1 : 0, 0);
            int s = 0;
            uint32_t ph = 0;
            int it = 0;
            for (long long u = first; u < p.num_units; u += step, ++it) {
                int mt, nt, sp, kb0, kb1;
                unit_coords(p, u, mt, nt, sp);
                kb_range(p, sp, kb0, kb1);
                const int a = it & 1;
                if (!mbar_wait(smem_u32(&acc_empty[a]), ((it >> 1) & 1) ^ 1, abort_flag, kDevTimeoutAccEmpty))
                    goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + a * BN;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(smem_u32(&full[s]), ph, abort_flag, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(ring + s * G::STAGE_BYTES), sb = sa + G::A_BYTES;
                    const uint32_t la = smem_u32(ring_lo + s * G::STAGE_BYTES), lb = la + G::A_BYTES;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t ad = A_MN ? umma_desc(sa + k * 1024, 32 * 128, 512, kLayoutSw128Base32)
                                                 : umma_desc(sa + k * 32, 16, 1024, kLayoutSw128);
                        const uint64_t bd = umma_desc(sb + k * 32, 16, 1024, kLayoutSw128);
                        const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
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
                    umma_commit(smem_u32(&empty[s]));
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                umma_commit(smem_u32(&acc_full[a]));
            }
        }
    } else if (warp >= 2 && warp < 6) {
        // ------------------------------ epilogue ----------------------------------
        const int q = warp & 3;
        int it = 0;
        for (long long u = first; u < p.num_units; u += step, ++it) {
            int mt, nt, sp, kb0, kb1;
            unit_coords(p, u, mt, nt, sp);
            kb_range(p, sp, kb0, kb1);
            const int a = it & 1;
            if (!mbar_wait(smem_u32(&acc_full[a]), (it >> 1) & 1, abort_flag, kDevTimeoutAccFull)) goto done;
            __syncwarp();
            tc_fence_after();
            const int m = mt * 128 + q * 32 + lane;
            const bool mv = m < p.M;
            const bool empty_k = kb1 <= kb0;   // this split got no blocks: partial is zero
            // Output addressing for this lane's row.
            float* obase;
            int64_t ostride;   // distance between consecutive columns n
            if (KIND == kWgrad) {
                // partial [split][Co][C*kh*kw]: column co at co * M
                obase = p.out + (int64_t)sp * p.Ncol * p.M + m;
                ostride = p.M;
            } else {
                const int HW = (KIND == kFwd) ? p.Ho * p.Wo : p.H * p.W;
                const int img = mv ? m / HW : 0, pix = mv ? m - img * HW : 0;
                obase = p.out + ((int64_t)img * p.Ncol) * HW + pix;
                ostride = HW;
            }
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + a * BN + c * 32, r);
                tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    mbar_arrive(smem_u32(&acc_empty[a]));
                }
                if (mv) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int n = nt * BN + c * 32 + j;
                        if (n < p.Ncol) {
                            float vj = empty_k ? 0.f : __uint_as_float(r[j]);
                            if (KIND == kFwd && p.bias) vj = vj + __ldg(p.bias + n);
                            obase[(int64_t)n * ostride] = vj;
                        }
                    }
                }
            }
        }
    }

done:
    cp_async_wait_all();   // no copy may still target this CTA's shared memory
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, G::TMEM_COLS);
    }
}

// dW[i] = sum over splits s = 0..S-1 (in order) of part[s][i]; i over Co*C*kh*kw.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, float* __restrict__ out, int splits,
                                     int64_t count) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int s = 0; s < splits; ++s) acc += part[(int64_t)s * count + i];
        out[i] = acc;
    }
}

// db[co] = sum over n (ascending) of the spatial sum of dy[n, co, :, :]
// (include/TensorOps.hpp:398-418 order: a per-image partial, then accumulate over n).
// One block per channel; the spatial sum is a tree over the block.
__global__ void bias_grad_kernel(const float* __restrict__ dy, float* __restrict__ db, int N, int Co, int HW,
                                 int64_t s0, int64_t s1) {
    const int co = blockIdx.x;
    __shared__ float red[32];
    float total = 0.f;
    for (int n = 0; n < N; ++n) {
        const float* base = dy + n * s0 + co * s1;
        float part = 0.f;
        for (int i = threadIdx.x; i < HW; i += blockDim.x) part += __ldg(base + i);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (threadIdx.x == 0) total += v;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) db[co] = total;
}

// ------------------------------------------------------------------------------------
// Strict-fp32 SIMT kernels: one thread per output element, products accumulated in the
// loop order of the reference's CPU routines (FFMA instead of separate multiply/add).
// ------------------------------------------------------------------------------------

// include/TensorOps.hpp:235-273: start from bias, then c_in, r, s.
__global__ void direct_fwd_kernel(const Params p) {
    const int64_t total = (int64_t)p.N * p.Co * p.Ho * p.Wo;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int ox = (int)(i % p.Wo);
        int64_t r0 = i / p.Wo;
        const int oy = (int)(r0 % p.Ho); r0 /= p.Ho;
        const int co = (int)(r0 % p.Co);
        const int n = (int)(r0 / p.Co);
        float acc = p.bias ? __ldg(p.bias + co) : 0.f;
        for (int c = 0; c < p.C; ++c)
            for (int r = 0; r < p.kh; ++r) {
                const int iy = oy * p.stride + r - p.pad;
                if (iy < 0 || iy >= p.H) continue;
                for (int s = 0; s < p.kw; ++s) {
                    const int ix = ox * p.stride + s - p.pad;
                    if (ix < 0 || ix >= p.W) continue;
                    acc = __fmaf_rn(__ldg(p.x + n * p.sx[0] + c * p.sx[1] + iy * p.sx[2] + ix * p.sx[3]),
                                    __ldg(p.w + co * p.sw[0] + c * p.sw[1] + r * p.sw[2] + s * p.sw[3]), acc);
                }
            }
        p.out[i] = acc;
    }
}

// include/TensorOps.hpp:319-356 (as a gather): dx[n,c,iy,ix] sums over c_out, r, s.
__global__ void direct_dgrad_kernel(const Params p) {
    const int64_t total = (int64_t)p.N * p.C * p.H * p.W;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int ix = (int)(i % p.W);
        int64_t r0 = i / p.W;
        const int iy = (int)(r0 % p.H); r0 /= p.H;
        const int c = (int)(r0 % p.C);
        const int n = (int)(r0 / p.C);
        float acc = 0.f;
        for (int co = 0; co < p.Co; ++co)
            for (int r = 0; r < p.kh; ++r) {
                const int ny = iy + p.pad - r;
                if (ny < 0 || ny % p.stride) continue;
                const int oy = ny / p.stride;
                if (oy >= p.Ho) continue;
                for (int s = 0; s < p.kw; ++s) {
                    const int nx = ix + p.pad - s;
                    if (nx < 0 || nx % p.stride) continue;
                    const int ox = nx / p.stride;
                    if (ox >= p.Wo) continue;
                    acc = __fmaf_rn(__ldg(p.dy + n * p.sdy[0] + co * p.sdy[1] + oy * p.sdy[2] + ox * p.sdy[3]),
                                    __ldg(p.w + co * p.sw[0] + c * p.sw[1] + r * p.sw[2] + s * p.sw[3]), acc);
                }
            }
        p.out[i] = acc;
    }
}

// include/TensorOps.hpp:358-396: per image a spatial partial sum, accumulated over n.
__global__ void direct_wgrad_kernel(const Params p) {
    const int64_t total = (int64_t)p.Co * p.C * p.kh * p.kw;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int s = (int)(i % p.kw);
        int64_t r0 = i / p.kw;
        const int r = (int)(r0 % p.kh); r0 /= p.kh;
        const int c = (int)(r0 % p.C);
        const int co = (int)(r0 / p.C);
        float gw = 0.f;
        for (int n = 0; n < p.N; ++n) {
            float sum = 0.f;
            for (int oy = 0; oy < p.Ho; ++oy) {
                const int iy = oy * p.stride + r - p.pad;
                if (iy < 0 || iy >= p.H) continue;
                for (int ox = 0; ox < p.Wo; ++ox) {
                    const int ix = ox * p.stride + s - p.pad;
                    if (ix < 0 || ix >= p.W) continue;
                    sum = __fmaf_rn(__ldg(p.x + n * p.sx[0] + c * p.sx[1] + iy * p.sx[2] + ix * p.sx[3]),
                                    __ldg(p.dy + n * p.sdy[0] + co * p.sdy[1] + oy * p.sdy[2] + ox * p.sdy[3]), sum);
                }
            }
            gw += sum;
        }
        p.out[i] = gw;
    }
}

}  // namespace conv
}  // namespace mt
