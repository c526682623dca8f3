// conv_halo2.cuh -- the CTA-pair form of the pitched-halo forward (conv_halo.cuh).
//
// Why a pair. With C_out = 64 the forward's MMA is 128 x 64 x 8: 48 cycles of work, and the
// one issuing thread per SM was measured as the bound (about 72 cycles per MMA, plus a
// fixed start-up per 32-channel block). Two CTAs on the two SMs of a TPC share one
// tcgen05.mma.cta_group::2 of M = 256: one instruction from the even CTA's issuer does both
// SMs' 128 x BN, so the issue cost per output halves, while each SM reads only its own
// halo rows and HALF of the weight matrix (BN/2 output channels) per MMA.
//
// A pair tile is two horizontally adjacent halo tiles of TY x TXv outputs: CTA rank r takes
// columns x0 + r * TXv (HaloParams.tiles_x counts pairs of tiles here). Roles per CTA:
//   warp 0      weight producer: this CTA's half of every weight stage (rows nt*BN + r*BN/2
//               .. of the reordered weights); completes on the EVEN CTA's b_full, whose
//               producer expects both halves.
//   warp 1      TMEM owner (pair allocation); in the even CTA the MMA issuer, which commits
//               slot releases and accumulator-ready to the barriers of both CTAs.
//   warps 2-5   epilogue of this CTA's 128 pitched positions; a drained accumulator is
//               reported to the even CTA's acc_empty (8 arrivals per tile).
//   warp 6      halo producer for this CTA's tile. TF32: completes on the even CTA's a_full
//               (both halos expected there). TF32X3: on this CTA's own a_full, for:
//   warps 7-10  (TF32X3) hi/lo splitter of this CTA's halo; one arrival per warp on the even
//               CTA's a_conv (8 per block).
// Every wait is bounded; the kernel ends with a cluster barrier so that no CTA leaves while
// its peer may still signal it or read its shared memory. Each output is accumulated by the
// same sequence of MMA k-steps as in the one-CTA kernel, so the results are bitwise equal.
//
// Measured on config 4 it is slower than the one-CTA kernel (TF32 33.1 vs 31.1 us, 3xTF32
// 81.4 vs 77.6 us): the bound is each SM's own MMA work, not the issuing thread, so the
// host runs it only on request (MT_CONV_PAIR=1).
#pragma once

#include "conv_halo.cuh"

namespace mt {
namespace convh {

// On the abort path only: give TMA copies already issued time to land (2 ms bound).
__device__ __forceinline__ void halo_drain_pause() {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) __nanosleep(1000);
}

// Warp-cooperative bounded wait at cluster scope: lane 0 spins, then every lane takes the
// completed phase with one try_wait of its own (the acquire of what the peer published).
__device__ __forceinline__ bool mbar_wait_warp_cl(uint32_t bar, uint32_t parity, volatile int* abort_flag, int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait_cl(bar, parity, abort_flag, code) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) (void)mbar_try_wait_cl(bar, parity);
    return ok != 0;
}

template <int BN, bool X3>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(HaloCfg<X3>::THREADS, 1)
conv_fwd_halo_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const HaloParams p) {
    extern __shared__ uint8_t smem_raw[];
    // Same dynamic-smem base in both CTAs, so every descriptor the even CTA builds is at
    // identical offsets in the pair.
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
    constexpr uint32_t TMEM_COLS = 2 * BN;
    constexpr uint32_t BH = BN / 2;                   // output channels of B held per CTA
    constexpr uint32_t BMATH = BH * 128;              // one tap's weight half (hi or lo)
    static_assert(BN == 64 || BN == 128, "pair halo: BN must be 64 or 128");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const long long first = blockIdx.x >> 1, step = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxASlots; ++i) {
            mbar_init(smem_u32(&a_full[i]), 1);
            mbar_init(smem_u32(&a_empty[i]), 1);
            mbar_init(smem_u32(&a_conv[i]), 8);       // one arrival per splitter warp of both CTAs
        }
        for (int i = 0; i < kMaxBStages; ++i) {
            mbar_init(smem_u32(&b_full[i]), 1);
            mbar_init(smem_u32(&b_empty[i]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&acc_full[a]), 1);
            mbar_init(smem_u32(&acc_empty[a]), 8);    // one arrival per epilogue warp of both CTAs
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32((const void*)tmem_slot), TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();   // barriers of both CTAs initialised, TMEM allocated in both
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------ weight producer -----------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (long long t = first; t < p.num_tiles; t += step) {
                int n, y0, x0p, nt;
                halo_tile(p, t, n, y0, x0p, nt);
                if (p.b_resident && t != first) break;   // resident weights: loaded for the first tile only
                for (int cb = 0; cb < p.cblocks; ++cb)
                    for (int g = 0; g < p.tgroups; ++g) {
                        if (!p.b_resident &&
                            !mbar_wait_cl(smem_u32(&b_empty[s]), ph ^ 1, abort_flag, kDevTimeoutEmpty))
                            goto done;
                        if (leader) mbar_arrive_expect_tx(smem_u32(&b_full[s]), 2 * p.b_bytes);
                        const uint32_t bar = mapa_shared(smem_u32(&b_full[s]), 0);
                        const uint32_t dst = smem_u32(b_ring + s * p.b_bytes);
                        const int tap0 = g * p.G, co0 = nt * BN + (int)(rank * BH);
                        if (X3) tma_load_4d_pair(dst, &tmB, bar, cb * 32, co0, 0, tap0);
                        else tma_load_4d_pair(dst, &tmB, bar, cb * 32, co0, tap0, 0);
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
                int n, y0, x0p, nt;
                halo_tile(p, t, n, y0, x0p, nt);
                const int x0 = 2 * x0p + (int)rank * p.TXv;
                for (int cb = 0; cb < p.cblocks; ++cb) {
                    if (!mbar_wait_cl(smem_u32(&a_empty[s]), ph ^ 1, abort_flag, kDevTimeoutEmpty)) goto done;
                    const uint32_t dst = smem_u32(a_ring + s * p.slot_bytes);
                    if (X3) {
                        const uint32_t bar = smem_u32(&a_full[s]);
                        mbar_arrive_expect_tx(bar, p.halo_bytes);
                        tma_load_4d(dst, &tmA, bar, cb * 32, x0 - p.pad, y0 - p.pad, n);
                    } else {
                        if (leader) mbar_arrive_expect_tx(smem_u32(&a_full[s]), 2 * p.halo_bytes);
                        tma_load_4d_pair(dst, &tmA, mapa_shared(smem_u32(&a_full[s]), 0), cb * 32, x0 - p.pad,
                                         y0 - p.pad, n);
                    }
                    if (++s == p.a_slots) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer (even CTA) -----------------------
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = umma_idesc_tf32(256, BN, 0, 0);
            int as = 0, bs = 0, it = 0;
            uint32_t aph = 0, bph = 0;
            for (long long t = first; t < p.num_tiles; t += step, ++it) {
                const int acc_i = it & 1;
                if (!mbar_wait_cl(smem_u32(&acc_empty[acc_i]), ((it >> 1) & 1) ^ 1, abort_flag, kDevTimeoutAccEmpty))
                    goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc_i * BN;
                bool first_mma = true;
                for (int cb = 0; cb < p.cblocks; ++cb) {
                    const uint32_t abar = X3 ? smem_u32(&a_conv[as]) : smem_u32(&a_full[as]);
                    if (!mbar_wait_cl(abar, aph, abort_flag, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint64_t a0 = halo_desc(smem_u32(a_ring + as * p.slot_bytes));
                    const uint64_t alo0 = halo_desc(smem_u32(alo_ring + as * p.slot_bytes));
                    int tr = 0, ts = 0;
                    for (int g = 0; g < p.tgroups; ++g) {
                        if (p.b_resident) bs = cb * p.tgroups + g;
                        if ((!p.b_resident || it == 0) &&
                            !mbar_wait_cl(smem_u32(&b_full[bs]), p.b_resident ? 0u : bph, abort_flag, kDevTimeoutFull))
                            goto done;
                        tc_fence_after();
                        const uint64_t b0 = umma_desc(smem_u32(b_ring + bs * p.b_bytes), 16, 1024, kLayoutSw128);
                        if (p.kw == 3 && ts == 0 && (p.G == 9 || p.G == 3)) {
                            const uint32_t P8 = (uint32_t)p.P * 8u;
                            if (p.G == 9)
                                issue_row_taps<9, X3, BMATH, true>(d_tmem, a0, alo0, b0, idesc, P8, (uint32_t)tr, first_mma);
                            else
                                issue_row_taps<3, X3, BMATH, true>(d_tmem, a0, alo0, b0, idesc, P8, (uint32_t)tr, first_mma);
                            tr += p.G / 3;
                        } else {
                            for (int gi = 0; gi < p.G; ++gi) {
                                const uint64_t ao = (uint64_t)(((uint32_t)(tr * p.P + ts) * 128u) >> 4);
                                const uint64_t bo = (uint64_t)(((X3 ? 2u * gi : (uint32_t)gi) * BMATH) >> 4);
                                if (++ts == p.kw) { ts = 0; ++tr; }
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const uint64_t ad = a0 + ao + 2 * k, bd = b0 + bo + 2 * k;
                                    const uint32_t acc = (!first_mma || k > 0) ? 1u : 0u;
                                    if (X3) {
                                        umma_tf32_pair(d_tmem, alo0 + ao + 2 * k, bd, idesc, acc);
                                        umma_tf32_pair(d_tmem, ad, bd + (BMATH >> 4), idesc, 1u);
                                        umma_tf32_pair(d_tmem, ad, bd, idesc, 1u);
                                    } else {
                                        umma_tf32_pair(d_tmem, ad, bd, idesc, acc);
                                    }
                                }
                                first_mma = false;
                            }
                        }
                        if (!p.b_resident) {
                            umma_commit_pair(smem_u32(&b_empty[bs]));
                            umma_commit_pair(mapa_shared(smem_u32(&b_empty[bs]), 1));
                            if (++bs == p.b_stages) { bs = 0; bph ^= 1; }
                        }
                    }
                    umma_commit_pair(smem_u32(&a_empty[as]));
                    umma_commit_pair(mapa_shared(smem_u32(&a_empty[as]), 1));
                    if (++as == p.a_slots) { as = 0; aph ^= 1; }
                }
                umma_commit_pair(smem_u32(&acc_full[acc_i]));
                umma_commit_pair(mapa_shared(smem_u32(&acc_full[acc_i]), 1));
            }
        }
    } else if (warp < 6) {
        // ------------------------------ epilogue ------------------------------------
        const int q = warp & 3;
        const int HoWo = p.Ho * p.Wo;
        int it = 0;
        for (long long t = first; t < p.num_tiles; t += step, ++it) {
            int n, y0, x0p, nt;
            halo_tile(p, t, n, y0, x0p, nt);
            const int x0 = 2 * x0p + (int)rank * p.TXv;
            const int acc_i = it & 1;
            if (!mbar_wait_warp_cl(smem_u32(&acc_full[acc_i]), (it >> 1) & 1, abort_flag, kDevTimeoutAccFull)) goto done;
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
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc_i]), 0));
                }
                if (valid) {
                    const int co0 = nt * BN + c * 32;
                    float bv[32];
                    if (p.bias && co0 + 32 <= p.Ncol && ((reinterpret_cast<uintptr_t>(p.bias + co0) & 15) == 0)) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float4 b4 = __ldg(reinterpret_cast<const float4*>(p.bias + co0) + j);
                            bv[4 * j] = b4.x; bv[4 * j + 1] = b4.y; bv[4 * j + 2] = b4.z; bv[4 * j + 3] = b4.w;
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
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&a_conv[as]), 0));
                if (++as == p.a_slots) { as = 0; aph ^= 1; }
            }
    }
done:
    if ((warp == 0 || warp == 6) && lane == 0 && *abort_flag) halo_drain_pause();
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();   // the peer no longer signals us or reads our shared memory / TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

}  // namespace convh
}  // namespace mt
