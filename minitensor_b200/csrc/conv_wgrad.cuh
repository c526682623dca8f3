// conv_wgrad.cuh -- stride-1 Conv2D weight gradient with wide pipeline stages.
//
// GEMM view: dW[m = (tap, c)][n = co] = sum over output pixels p of
//   x[c][p shifted by the tap] * dy[co][p],
// M = taps * C (128-row tiles = four 32-channel chunks, each a (tap, channel block)
// pair), N = C_out, K = output pixels, split over the CTAs (ordered reduction after).
//
// A stage covers RS output rows x XCS runs of 32 output pixels (K = RS * 32 * XCS,
// ordered row, pixel):
//   A: four boxes {32 channels, 32 * XCS pixels, RS rows} of NHWC x, one per chunk, each
//      shifted by its tap (M-major, 128-byte pixel rows; out-of-image pixels zero-filled).
//   B: XCS boxes {32 pixels, BN output channels, RS rows} of dy read straight from NCHW
//      through a map whose dimensions are ordered (W, C_out, H, N), so that each row's
//      32-pixel block lands as BN consecutive 128-byte rows (K-major). Pixels and rows
//      past the output edge are zero-filled, which also cancels any A values there.
// Every handoff between the roles costs a few hundred cycles (an mbarrier wait, an
// expect-tx, a TMA issue per box), so the producer does no division in its loop: the
// four chunk offsets are fixed per tile and the (image, row, run) position advances by
// counting. Wider stages (XCS = 2) halve the handoffs per pixel.
//
// Warp roles as in the GEMM kernel: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-5
// epilogue (raw fp32 partial sums), 6-9 (TF32X3) hi/lo splitter.
#pragma once

#include "conv_tma.cuh"

namespace mt {
namespace convw {

using convt::WgradParams;   // xblocks here counts runs of 32 * XCS pixels per row

template <int BN, bool X3, int STAGES, int XCS, int RS>
struct WCfg {
    static constexpr int KSTEPS = 4 * XCS * RS;                    // 8 pixels per k-step
    static constexpr uint32_t CHUNK_BYTES = 32u * XCS * RS * 128u; // one (tap, cb) chunk: K rows x 128 B
    static constexpr uint32_t A_BYTES = 4 * CHUNK_BYTES;
    static constexpr uint32_t B_BLOCK_BYTES = BN * 128u;           // 32 pixels of one row of dy
    static constexpr uint32_t B_RUN_BYTES = RS * B_BLOCK_BYTES;    // one box: RS rows of a run
    static constexpr uint32_t B_BYTES = XCS * B_RUN_BYTES;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr uint32_t RING_BYTES = STAGE_BYTES * STAGES * (X3 ? 2 : 1);
    static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr int THREADS = (X3 ? 10 : 6) * 32;
    static constexpr uint32_t BAR_BYTES = 8 * (3 * STAGES + 4) + 16;
    static constexpr uint32_t SMEM_BYTES = 1024 + RING_BYTES + BAR_BYTES;
};

__device__ __forceinline__ void unit_coords(const WgradParams& p, long long u, int& mt, int& nt, int& kb0, int& kb1) {
    const int sp = (int)(u % p.splits);
    const long long r = u / p.splits;
    nt = (int)(r % p.tiles_n);
    mt = (int)(r / p.tiles_n);
    kb0 = (int)((long long)p.kb_total * sp / p.splits);
    kb1 = (int)((long long)p.kb_total * (sp + 1) / p.splits);
}

template <int BN, bool X3, int STAGES, int XCS, int RS>
__global__ void __launch_bounds__(WCfg<BN, X3, STAGES, XCS, RS>::THREADS, 1)
conv_wgrad_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const WgradParams p) {
    using G = WCfg<BN, X3, STAGES, XCS, RS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;
    uint8_t* ring_lo = smem + G::STAGE_BYTES * STAGES;
    const convt::Bars bb = convt::carve_bars<STAGES>(smem + G::RING_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long first = blockIdx.x, step = gridDim.x;

    if (threadIdx.x == 0) convt::init_bars<STAGES>(bb);
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
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (long long u = first; u < p.num_units; u += step) {
                int mt, nt, kb0, kb1;
                unit_coords(p, u, mt, nt, kb0, kb1);
                // Chunk q of the tile: rows m0 + 32q = (tap, first channel); fixed per tile.
                int cc0[4], dxq[4], dyq[4];
                uint32_t a_bytes = 0;
                int nchunks = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int m = mt * 128 + q * 32;
                    const bool valid = m < p.M;
                    const int tap = valid ? m / p.C : 0;
                    const int r = tap / p.kw;
                    cc0[q] = valid ? m - tap * p.C : 0;
                    dxq[q] = tap - r * p.kw - p.pad;
                    dyq[q] = r - p.pad;
                    if (valid) { a_bytes += G::CHUNK_BYTES; nchunks = q + 1; }
                }
                if (kb0 >= kb1) continue;
                // Position of k-block kb0: image, first output row (multiple of RS), run
                // of 32*XCS pixels.
                int img = kb0 / p.kb_per_img;
                int rem = kb0 - img * p.kb_per_img;
                int y = (rem / p.xblocks) * RS;
                int xg = rem - (y / RS) * p.xblocks;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(smem_u32(&bb.empty[s]), ph ^ 1, bb.abort_flag, kDevTimeoutEmpty)) goto done;
                    const uint32_t bar = smem_u32(&bb.full[s]);
                    mbar_arrive_expect_tx(bar, a_bytes + G::B_BYTES);
                    const uint32_t sa = smem_u32(ring + s * G::STAGE_BYTES);
                    const int x0 = xg * 32 * XCS;
                    for (int q = 0; q < nchunks; ++q)
                        tma_load_4d(sa + q * G::CHUNK_BYTES, &tmA, bar, cc0[q], x0 + dxq[q], y + dyq[q], img);
#pragma unroll
                    for (int c = 0; c < XCS; ++c)
                        tma_load_4d(sa + G::A_BYTES + c * G::B_RUN_BYTES, &tmB, bar, x0 + 32 * c, nt * BN, y, img);
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                    if (++xg == p.xblocks) {
                        xg = 0;
                        y += RS;
                        if (y >= p.Ho) { y = 0; ++img; }
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer --------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_tf32(128, BN, 1, 0);
            int s = 0, it = 0;
            uint32_t ph = 0;
            for (long long u = first; u < p.num_units; u += step, ++it) {
                int mt, nt, kb0, kb1;
                unit_coords(p, u, mt, nt, kb0, kb1);
                const int a = it & 1;
                if (!mbar_wait(smem_u32(&bb.acc_empty[a]), ((it >> 1) & 1) ^ 1, bb.abort_flag, kDevTimeoutAccEmpty))
                    goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + a * BN;
                for (int kb = kb0; kb < kb1; ++kb) {
                    const uint32_t wbar = X3 ? smem_u32(&bb.conv[s]) : smem_u32(&bb.full[s]);
                    if (!mbar_wait(wbar, ph, bb.abort_flag, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(ring + s * G::STAGE_BYTES), sb = sa + G::A_BYTES;
                    const uint32_t la = smem_u32(ring_lo + s * G::STAGE_BYTES), lb = la + G::A_BYTES;
                    // Descriptors at the stage's base; a start moved by `off` bytes is the same
                    // descriptor plus off >> 4 (the address field is addr >> 4, no carry below
                    // 256 KB), so each MMA adds a constant instead of re-encoding: at N = 64 an
                    // MMA is only 48 cycles of work for the one issuing thread to keep up with.
                    const uint64_t a0 = umma_desc(sa, G::CHUNK_BYTES, 512, kLayoutSw128Base32);
                    const uint64_t b0 = umma_desc(sb, 16, 1024, kLayoutSw128);
                    const uint64_t alo0 = umma_desc(la, G::CHUNK_BYTES, 512, kLayoutSw128Base32);
                    const uint64_t blo0 = umma_desc(lb, 16, 1024, kLayoutSw128);
#pragma unroll
                    for (int k = 0; k < G::KSTEPS; ++k) {
                        // A: 8 pixel rows per k-step (1024 B); chunks G::CHUNK_BYTES apart.
                        // B: k-step k is in row (k / 4) / XCS, run (k / 4) % XCS of the stage,
                        // 8 pixels (32 B) per k-step inside the 32-pixel block.
                        const int blk = k >> 2, rr = blk / XCS, cc = blk - rr * XCS;
                        const uint32_t boff = cc * G::B_RUN_BYTES + rr * G::B_BLOCK_BYTES + (k & 3) * 32;
                        const uint64_t ad = a0 + (uint64_t)((k * 1024) >> 4);
                        const uint64_t bd = b0 + (uint64_t)(boff >> 4);
                        const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
                        if (X3) {
                            umma_tf32(d_tmem, alo0 + (uint64_t)((k * 1024) >> 4), bd, idesc, acc);
                            umma_tf32(d_tmem, ad, blo0 + (uint64_t)(boff >> 4), idesc, 1u);
                            umma_tf32(d_tmem, ad, bd, idesc, 1u);
                        } else {
                            umma_tf32(d_tmem, ad, bd, idesc, acc);
                        }
                    }
                    umma_commit(smem_u32(&bb.empty[s]));
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                umma_commit(smem_u32(&bb.acc_full[a]));
            }
        }
    } else if (warp < 6) {
        // ------------------------------ epilogue ----------------------------------
        const int q = warp & 3;
        int it = 0;
        for (long long u = first; u < p.num_units; u += step, ++it) {
            int mt, nt, kb0, kb1;
            unit_coords(p, u, mt, nt, kb0, kb1);
            const int sp = (int)(u % p.splits);
            const bool no_k = kb1 <= kb0;
            const int a = it & 1;
            if (!mbar_wait(smem_u32(&bb.acc_full[a]), (it >> 1) & 1, bb.abort_flag, kDevTimeoutAccFull)) goto done;
            __syncwarp();
            tc_fence_after();
            const int m = mt * 128 + q * 32 + lane;
            float* row = p.ws + ((int64_t)sp * p.M + m) * p.ws_ld + nt * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t rr[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + a * BN + c * 32, rr);
                tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    mbar_arrive(smem_u32(&bb.acc_empty[a]));
                }
                if (m < p.M) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(row + c * 32 + j) =
                            no_k ? make_float4(0.f, 0.f, 0.f, 0.f)
                                 : make_float4(__uint_as_float(rr[j]), __uint_as_float(rr[j + 1]),
                                               __uint_as_float(rr[j + 2]), __uint_as_float(rr[j + 3]));
                }
            }
        }
    } else if (X3) {
        // ------------------------------ hi/lo splitter ----------------------------
        const int ct = threadIdx.x - 6 * 32;
        int s = 0;
        uint32_t ph = 0;
        for (long long u = first; u < p.num_units; u += step) {
            int mt, nt, kb0, kb1;
            unit_coords(p, u, mt, nt, kb0, kb1);
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!convt::splitter_stage<STAGES, G::STAGE_BYTES>(bb, ring, ring_lo, s, ph, ct)) goto done;
                if (++s == STAGES) { s = 0; ph ^= 1; }
            }
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

}  // namespace convw
}  // namespace mt
