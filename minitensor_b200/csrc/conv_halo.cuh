// conv_halo.cuh -- stride-1 Conv2D forward (and input-grad, which is the same kernel on
// dy with flipped, transposed weights) with ONE activation load per 32-channel block
// serving every filter tap, and weight stages that carry several taps each.
//
// Pitched halo tile. For an output tile of TY rows x TXv columns, TMA loads the input
// window it needs -- HR = TY + kh - 1 rows of P = TXv + kw - 1 pixels, 32 channels each
// (NHWC, 128 bytes per pixel) -- into shared memory as P*HR consecutive 128-byte rows,
// zero-filling the padding. Number the MMA's 128 M rows by the pitched position
// p = ty * P + tx. The input pixel that tap (r, s) contributes to output p is halo row
// p + r * P + s, so the A operand of every tap is the same buffer read from start row
// o = r * P + s: 128 consecutive rows, a plain K-major SW128 operand whose descriptor
// start moves by o * 128 bytes (the swizzle phase follows the address; see halo_desc).
// Positions with tx >= TXv are computed and discarded; a valid position never reads
// past the rows TMA wrote.
//
// Few, large pipeline stages. Each handoff between roles costs a few hundred cycles (an
// mbarrier wait, an expect-tx, a TMA issue), which is more than the MMA time of one tap
// of a 32-channel block at N = 64 (4 k-steps of 32 cycles). So a weight stage is ONE TMA
// box holding G taps ({32 channels, BN, G}, or {32, BN, 2 (hi/lo), G} for TF32X3 with
// the weights split into hi and lo in global memory by reorder_weights_kernel), and an
// activation halo is one box per 32-channel block: the MMA issuer then waits once per
// G * 4 (* 3) MMAs instead of once per 4.
//
// Resident weights. When C_out fits one N tile and every weight stage fits beside the
// halo ring (TF32 at C_out = 64: 2 x 72 KB), stage cb * tgroups + g holds its taps for
// the whole kernel: loaded once, never released, waited for once.
//
// Warp roles: 0 weight (B) producer, 1 MMA issuer + TMEM owner, 2-5 epilogue, 6 halo (A)
// producer, 7-10 (TF32X3) hi/lo splitter of the halos.
#pragma once

#include "conv_tma.cuh"

namespace mt {
namespace convh {

constexpr int kMaxASlots = 4;
constexpr int kMaxBStages = 8;

struct HaloParams {
    int N, Ho, Wo, Ncol, C, kh, kw, pad;  // Ncol = output channels, C = input channels
    int P, TXv, TY, HR;                   // pitch, valid columns, output rows, halo rows
    int tiles_y, tiles_x, tiles_n, cblocks, taps;
    int G, tgroups;                       // taps per weight stage, stages per channel block
    int b_resident;                       // 1: every weight stage is loaded once and kept
    long long num_tiles;
    int a_slots, b_stages;
    uint32_t halo_bytes;                  // bytes TMA writes per halo (P * HR * 128)
    uint32_t slot_bytes;                  // shared bytes per halo slot (multiple of 1024)
    uint32_t b_bytes;                     // bytes per weight stage (G * (1 or 2) * BN * 128)
    uint32_t a_off, alo_off, b_off, bar_off;   // offsets from the 1024-aligned base
    float* out;                           // [N, Ncol, Ho, Wo] contiguous
    const float* bias;                    // [Ncol] or null
};

// Tile t -> (image, first output row, first output column, C_out block); C_out block
// fastest so CTAs running the same pixels at once share halo reads in L2.
__device__ __forceinline__ void halo_tile(const HaloParams& p, long long t, int& n, int& y0, int& x0, int& nt) {
    long long r = t;
    nt = (int)(r % p.tiles_n); r /= p.tiles_n;
    const int xt = (int)(r % p.tiles_x); r /= p.tiles_x;
    const int yt = (int)(r % p.tiles_y); r /= p.tiles_y;
    n = (int)r;
    y0 = yt * p.TY;
    x0 = xt * p.TXv;
}

// K-major SW128 operand descriptor whose start may sit at any 128-byte row of a
// 1024-aligned swizzled buffer. The base-offset field stays 0: the MMA takes the XOR
// phase of each 128-byte row from the row's shared-memory address (address bits 7-9),
// the same rule TMA used when it wrote the rows, so a moved start needs no correction
// (checked against the oracle by the conv parity tests, where a wrong phase reads the
// zero-filled channel chunks and loses every tap but the first).
__device__ __forceinline__ uint64_t halo_desc(uint32_t start) {
    return umma_desc(start, 16, 1024, kLayoutSw128);
}

// The MMAs of NT taps of a 3x3 filter (whole filter rows starting at row `row0`) over one
// 32-channel block: 4 k-steps per tap, 3 MMAs per k-step in TF32X3. Unrolled so that every
// descriptor offset but the pitch is a constant: a 128 x 64 x 8 MMA takes ~48 cycles, and
// the loop's per-tap arithmetic on the one issuing thread had cost as much again (c4
// forward: 3.84 -> 3.52 us of issue per tile). CG2: the CTA-pair form (M = 256, each
// CTA's halo rows and half of the weight matrix, BMAT = that half's bytes).
__device__ __forceinline__ void umma_tf32_cg(bool cg2, uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if (cg2) umma_tf32_pair(d, a, b, idesc, acc);
    else umma_tf32(d, a, b, idesc, acc);
}
template <int NT, bool X3, uint32_t BMAT, bool CG2 = false>
__device__ __forceinline__ void issue_row_taps(uint32_t d_tmem, uint64_t a0, uint64_t alo0, uint64_t b0,
                                               uint32_t idesc, uint32_t P8, uint32_t row0, bool& first_mma) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const uint64_t ao = (uint64_t)((row0 + t / 3) * P8 + (t % 3) * 8u);   // (r * P + s) * 128 B >> 4
        const uint64_t bo = (uint64_t)(((X3 ? 2u * t : (uint32_t)t) * BMAT) >> 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint64_t ad = a0 + ao + 2 * k, bd = b0 + bo + 2 * k;
            const uint32_t acc = (!first_mma || t > 0 || k > 0) ? 1u : 0u;
            if (X3) {
                umma_tf32_cg(CG2, d_tmem, alo0 + ao + 2 * k, bd, idesc, acc);
                umma_tf32_cg(CG2, d_tmem, ad, bd + (BMAT >> 4), idesc, 1u);
                umma_tf32_cg(CG2, d_tmem, ad, bd, idesc, 1u);
            } else {
                umma_tf32_cg(CG2, d_tmem, ad, bd, idesc, acc);
            }
        }
    }
    first_mma = false;
}

template <bool X3>
struct HaloCfg {
    static constexpr int NUM_WARPS = X3 ? 11 : 7;
    static constexpr int THREADS = NUM_WARPS * 32;
};

// Split `bytes` of shared memory at `hi` into hi (in place) and lo, 128 threads.
__device__ __forceinline__ void split_block(uint8_t* hi_p, uint8_t* lo_p, uint32_t bytes, int ct) {
    float4* hi = reinterpret_cast<float4*>(hi_p);
    float4* lo = reinterpret_cast<float4*>(lo_p);
#pragma unroll 4
    for (uint32_t i = ct; i < bytes / 16; i += 128) {
        const float4 x = hi[i];
        const float4 h = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
        hi[i] = h;
        lo[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    }
}

template <int BN, bool X3>
__global__ void __launch_bounds__(HaloCfg<X3>::THREADS, 1)
conv_fwd_halo_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const HaloParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a_ring = smem + p.a_off;
    uint8_t* alo_ring = smem + p.alo_off;
    uint8_t* b_ring = smem + p.b_off;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
    uint64_t* a_full = bars;                          // [kMaxASlots]
    uint64_t* a_empty = a_full + kMaxASlots;
    uint64_t* a_conv = a_empty + kMaxASlots;
    uint64_t* b_full = a_conv + kMaxASlots;           // [kMaxBStages]
    uint64_t* b_empty = b_full + kMaxBStages;
    uint64_t* acc_full = b_empty + kMaxBStages;       // [2]
    uint64_t* acc_empty = acc_full + 2;               // [2]
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(acc_empty + 2) + 1;
    constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    constexpr uint32_t BMAT = BN * 128;               // one tap's weight matrix (hi or lo)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long first = blockIdx.x, step = gridDim.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxASlots; ++i) {
            mbar_init(smem_u32(&a_full[i]), 1);
            mbar_init(smem_u32(&a_empty[i]), 1);
            mbar_init(smem_u32(&a_conv[i]), 128);
        }
        for (int i = 0; i < kMaxBStages; ++i) {
            mbar_init(smem_u32(&b_full[i]), 1);
            mbar_init(smem_u32(&b_empty[i]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&acc_full[a]), 1);
            mbar_init(smem_u32(&acc_empty[a]), 4);   // one arrival per epilogue warp
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------ weight producer -----------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (long long t = first; t < p.num_tiles; t += step) {
                int n, y0, x0, nt;
                halo_tile(p, t, n, y0, x0, nt);
                if (p.b_resident && t != first) break;   // resident weights: loaded for the first tile only
                for (int cb = 0; cb < p.cblocks; ++cb)
                    for (int g = 0; g < p.tgroups; ++g) {
                        if (!p.b_resident &&
                            !mbar_wait(smem_u32(&b_empty[s]), ph ^ 1, abort_flag, kDevTimeoutEmpty))
                            goto done;
                        const uint32_t bar = smem_u32(&b_full[s]);
                        mbar_arrive_expect_tx(bar, p.b_bytes);
                        const uint32_t dst = smem_u32(b_ring + s * p.b_bytes);
                        const int tap0 = g * p.G;
                        if (X3) tma_load_4d(dst, &tmB, bar, cb * 32, nt * BN, 0, tap0);
                        else tma_load_4d(dst, &tmB, bar, cb * 32, nt * BN, tap0, 0);
                        if (++s == p.b_stages) { s = 0; ph ^= 1; }
                    }
            }
        }
    } else if (warp == 6) {
        // ------------------------------ halo producer -------------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (long long t = first; t < p.num_tiles; t += step) {
                int n, y0, x0, nt;
                halo_tile(p, t, n, y0, x0, nt);
                for (int cb = 0; cb < p.cblocks; ++cb) {
                    if (!mbar_wait(smem_u32(&a_empty[s]), ph ^ 1, abort_flag, kDevTimeoutEmpty)) goto done;
                    const uint32_t bar = smem_u32(&a_full[s]);
                    mbar_arrive_expect_tx(bar, p.halo_bytes);
                    tma_load_4d(smem_u32(a_ring + s * p.slot_bytes), &tmA, bar, cb * 32, x0 - p.pad, y0 - p.pad, n);
                    if (++s == p.a_slots) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ----------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_tf32(128, BN, 0, 0);
            int as = 0, bs = 0, it = 0;
            uint32_t aph = 0, bph = 0;
            for (long long t = first; t < p.num_tiles; t += step, ++it) {
                const int acc_i = it & 1;
                if (!mbar_wait(smem_u32(&acc_empty[acc_i]), ((it >> 1) & 1) ^ 1, abort_flag, kDevTimeoutAccEmpty))
                    goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc_i * BN;
                bool first_mma = true;
                for (int cb = 0; cb < p.cblocks; ++cb) {
                    const uint32_t abar = X3 ? smem_u32(&a_conv[as]) : smem_u32(&a_full[as]);
                    if (!mbar_wait(abar, aph, abort_flag, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(a_ring + as * p.slot_bytes);
                    const uint32_t alo_base = smem_u32(alo_ring + as * p.slot_bytes);
                    // Descriptors at offset 0 of this halo slot; the start address moved by
                    // `off` bytes is the same descriptor plus off >> 4: the 14-bit field holds
                    // addr >> 4 of a shared address below 256 KB, so the sum never carries
                    // out. With N = 64 an MMA takes 48 cycles, less than recomputing two
                    // descriptors and a tap division on the one issuing thread took.
                    const uint64_t a0 = halo_desc(a_base), alo0 = halo_desc(alo_base);
                    int tr = 0, ts = 0;   // (r, s) of the next tap, advanced without division
                    for (int g = 0; g < p.tgroups; ++g) {
                        if (p.b_resident) bs = cb * p.tgroups + g;
                        if ((!p.b_resident || it == 0) &&
                            !mbar_wait(smem_u32(&b_full[bs]), p.b_resident ? 0u : bph, abort_flag, kDevTimeoutFull))
                            goto done;
                        tc_fence_after();
                        const uint64_t b0 = umma_desc(smem_u32(b_ring + bs * p.b_bytes), 16, 1024, kLayoutSw128);
                        if (p.kw == 3 && ts == 0 && (p.G == 9 || p.G == 3)) {
                            // 3x3 filter, a stage of whole filter rows
                            const uint32_t P8 = (uint32_t)p.P * 8u;
                            if (p.G == 9) issue_row_taps<9, X3, BMAT>(d_tmem, a0, alo0, b0, idesc, P8, (uint32_t)tr, first_mma);
                            else issue_row_taps<3, X3, BMAT>(d_tmem, a0, alo0, b0, idesc, P8, (uint32_t)tr, first_mma);
                            tr += p.G / 3;
                        } else
                        for (int gi = 0; gi < p.G; ++gi) {
                            const uint64_t ao = (uint64_t)(((uint32_t)(tr * p.P + ts) * 128u) >> 4);
                            const uint64_t bo = (uint64_t)(((X3 ? 2u * gi : (uint32_t)gi) * BMAT) >> 4);
                            if (++ts == p.kw) { ts = 0; ++tr; }
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const uint64_t ad = a0 + ao + 2 * k, bd = b0 + bo + 2 * k;   // + 32 B per k-step
                                const uint32_t acc = (!first_mma || k > 0) ? 1u : 0u;
                                if (X3) {
                                    umma_tf32(d_tmem, alo0 + ao + 2 * k, bd, idesc, acc);
                                    umma_tf32(d_tmem, ad, bd + (BMAT >> 4), idesc, 1u);
                                    umma_tf32(d_tmem, ad, bd, idesc, 1u);
                                } else {
                                    umma_tf32(d_tmem, ad, bd, idesc, acc);
                                }
                            }
                            first_mma = false;
                        }
                        if (!p.b_resident) {
                            umma_commit(smem_u32(&b_empty[bs]));
                            if (++bs == p.b_stages) { bs = 0; bph ^= 1; }
                        }
                    }
                    umma_commit(smem_u32(&a_empty[as]));
                    if (++as == p.a_slots) { as = 0; aph ^= 1; }
                }
                umma_commit(smem_u32(&acc_full[acc_i]));
            }
        }
    } else if (warp < 6) {
        // ------------------------------ epilogue ------------------------------------
        const int q = warp & 3;
        const int HoWo = p.Ho * p.Wo;
        int it = 0;
        for (long long t = first; t < p.num_tiles; t += step, ++it) {
            int n, y0, x0, nt;
            halo_tile(p, t, n, y0, x0, nt);
            const int acc_i = it & 1;
            if (!mbar_wait_warp(smem_u32(&acc_full[acc_i]), (it >> 1) & 1, abort_flag, kDevTimeoutAccFull)) goto done;
            tc_fence_after();
            const int l = q * 32 + lane;             // TMEM lane = pitched position
            const int ty = l / p.P, tx = l - ty * p.P;
            const int oy = y0 + ty, ox = x0 + tx;
            const bool valid = ty < p.TY && tx < p.TXv && oy < p.Ho && ox < p.Wo;
            float* obase = p.out + (int64_t)n * p.Ncol * HoWo + (int64_t)oy * p.Wo + ox;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t rr[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc_i * BN + c * 32, rr);
                tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc_i]));
                }
                if (valid) {
                    // The chunk's 32 biases are loaded once (vector loads when aligned), and
                    // the output pointer steps one channel plane per element: a bias load, an
                    // add and a 64-bit multiply per element made this epilogue cost more than
                    // the MMAs of its tile.
                    const int co0 = nt * BN + c * 32;
                    float bv[32];
                    if (p.bias && co0 + 32 <= p.Ncol && ((reinterpret_cast<uintptr_t>(p.bias + co0) & 15) == 0)) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float4 t = __ldg(reinterpret_cast<const float4*>(p.bias + co0) + j);
                            bv[4 * j] = t.x; bv[4 * j + 1] = t.y; bv[4 * j + 2] = t.z; bv[4 * j + 3] = t.w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) bv[j] = (p.bias && co0 + j < p.Ncol) ? __ldg(p.bias + co0 + j) : 0.f;
                    }
                    float* o = obase + (int64_t)co0 * HoWo;
                    if (co0 + 32 <= p.Ncol) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) { *o = __uint_as_float(rr[j]) + bv[j]; o += HoWo; }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (co0 + j < p.Ncol) *o = __uint_as_float(rr[j]) + bv[j];
                            o += HoWo;
                        }
                    }
                }
            }
        }
    } else if (X3) {
        // ------------------------------ halo hi/lo splitter -------------------------
        const int ct = threadIdx.x - 7 * 32;
        int as = 0;
        uint32_t aph = 0;
        for (long long t = first; t < p.num_tiles; t += step)
            for (int cb = 0; cb < p.cblocks; ++cb) {
                if (!mbar_wait_warp(smem_u32(&a_full[as]), aph, abort_flag, kDevTimeoutMisc)) goto done;
                split_block(a_ring + as * p.slot_bytes, alo_ring + as * p.slot_bytes, p.slot_bytes, ct);
                fence_proxy_async_smem();
                mbar_arrive(smem_u32(&a_conv[as]));
                if (++as == p.a_slots) { as = 0; aph ^= 1; }
            }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace convh
}  // namespace mt
