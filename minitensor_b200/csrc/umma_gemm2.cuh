// umma_gemm2.cuh -- the CTA-pair form of the tensor-core GEMM (tcgen05 cta_group::2) used
// for outputs large enough to fill the GPU with 256 x BN tiles.
//
// Why a pair. With one CTA per 128 x 256 tile every SM streams a full 256-column B tile
// through its shared memory for each 128 rows of A: per 8-deep k-step the tensor core
// reads 4 KB of A and 8 KB of B, and TMA writes the same 12 KB, which is more shared-
// memory bandwidth than one SM has. Two CTAs on the two SMs of a TPC form a cluster and
// share one 256 x BN MMA (M = 256): each CTA holds its own 128 rows of A and HALF of the
// B tile (BN/2 columns); the even CTA issues tcgen05.mma.cta_group::2, which reads both
// halves of B across the pair and writes each CTA's 128 x BN accumulator into that CTA's
// TMEM. Per SM the B traffic halves while the MMA work per SM stays 128 x BN.
//
// Roles (both CTAs run all of them except the MMA issuer, which only the even CTA runs):
//   warp 0      TMA producer for this CTA's A rows and B half. TF32: the load completes
//               on the EVEN CTA's `full` barrier (cta_group::2 form of the plain per-CTA
//               load); the even CTA's producer expects both CTAs' bytes. TF32X3: the load
//               completes on this CTA's own `full` barrier, for the local splitter.
//   warp 1      TMEM owner (pair allocation: same columns in both CTAs); in the even CTA
//               also the single-thread MMA issuer. Stage release and accumulator-ready
//               are committed to the barriers of BOTH CTAs (two commits, own + peer).
//   warps 2-5   epilogue of this CTA's 128 rows; a drained accumulator is reported to the
//               even CTA's `acc_empty` (one remote arrival per warp, 8 per tile).
//   warps 6-9   (TF32X3) splitter of this CTA's stage; reports to the even CTA's `conv`
//               barrier (one arrival per warp, 8 per stage).
// Every wait is bounded (mbar_wait*); the kernel ends with a cluster barrier so that no
// CTA leaves while its peer may still signal it or read its shared memory.
#pragma once

#include "umma_gemm.cuh"

namespace mt {
namespace umma2 {

using umma::Params;

constexpr int BM = 256;     // rows of a pair tile (128 per CTA)
constexpr int BMC = 128;    // rows per CTA

template <int BN, int BKE_, bool X3, int STAGES>
struct Cfg {
    static constexpr int BKE = BKE_;
    static constexpr int BH = BN / 2;                          // B columns held per CTA
    static constexpr uint32_t A_BYTES = BMC * BKE * 4;
    static constexpr uint32_t B_BYTES = BH * BKE * 4;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int KSTEPS = BKE / 8;
    static constexpr uint32_t TMEM_COLS = 2 * BN;              // double-buffered accumulator
    static constexpr int NUM_WARPS = X3 ? 10 : 6;
    static constexpr int THREADS = NUM_WARPS * 32;
    static constexpr uint32_t RING_BYTES = STAGE_BYTES * STAGES * (X3 ? 2 : 1);
    static constexpr uint32_t EPI_BYTES = 4 * 8192;                // epilogue staging, 2 x 4 KB per warp
    static constexpr uint32_t BAR_BYTES = 8 * (3 * STAGES + 4) + 16;
    static constexpr uint32_t SMEM_BYTES = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES;
    static constexpr uint32_t CHUNK = 32;
    static constexpr uint32_t MN_CHUNK_BYTES = BKE * 128;
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "pair TMEM allocation must be a power of two");
    static_assert(BH % 32 == 0, "B half must be whole 32-column chunks");
};

// On the abort path only: give TMA copies already issued time to land before the CTA
// leaves (a copy completes in microseconds; 2 ms is a generous bound).
__device__ __forceinline__ void drain_pause() {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) __nanosleep(1000);
}

// One piece of a cluster's work: k-blocks [kb0, kb1) of output tile `tile`. nseg > 1: the
// tile is cut between nseg clusters and this piece is the seg-th in k order.
struct Item {
    long long tile;
    int kb0, kb1, seg, nseg;
};

// The work of cluster c of C, in order: units c, c + C, ... of the sk_dp * S units of the
// tiles below p.sk_dp (unit u = piece u % S of tile u / S; S = 1: whole tiles), then the
// cluster's contiguous range [W c / C, W (c+1) / C) of the W = (num_tiles - sk_dp) * kblocks
// k-blocks of the stream-K tiles, cut at tile boundaries. Every role of the kernel walks
// the same sequence.
struct Sched {
    long long u, x, hi, c, C, W, dp_units;
    int kblocks, S;
    __device__ Sched(const Params& p, int kblocks_, long long cluster, long long clusters)
        : u(cluster), c(cluster), C(clusters), kblocks(kblocks_), S(p.sk_split > 1 ? p.sk_split : 1) {
        dp_units = p.sk_dp * S;
        W = (p.num_tiles - p.sk_dp) * (long long)kblocks;
        x = W * c / C;
        hi = W * (c + 1) / C;
    }
    // The cluster whose range holds stream-K k-block y: the largest c with W c / C <= y.
    __device__ long long owner(long long y) const { return ((y + 1) * C + W - 1) / W - 1; }
    __device__ bool next(const Params& p, Item& it) {
        if (u < dp_units) {
            it.tile = u / S;
            const int sp = (int)(u - it.tile * S);
            it.kb0 = (int)((long long)kblocks * sp / S);
            it.kb1 = (int)((long long)kblocks * (sp + 1) / S);
            it.seg = sp;
            it.nseg = S;
            u += C;
            return true;
        }
        if (x >= hi) return false;
        const long long t = x / kblocks;
        it.tile = p.sk_dp + t;
        it.kb0 = (int)(x - t * kblocks);
        it.kb1 = (int)min((long long)kblocks, (long long)it.kb0 + (hi - x));
        const long long cf = owner(t * kblocks);
        it.nseg = (int)(owner(t * kblocks + kblocks - 1) - cf + 1);
        it.seg = (int)(c - cf);
        x += it.kb1 - it.kb0;
        return true;
    }
};

template <int BN, int BKE, bool A_MN, bool B_MN, bool X3, int STAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg<BN, BKE, X3, STAGES>::THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ umma::DstMaps dm, const Params p) {
    using G = Cfg<BN, BKE, X3, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    // Same dynamic-smem base in both CTAs, so the aligned layout (and every descriptor
    // the even CTA builds) is at identical offsets in the pair.
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;
    uint8_t* ring_lo = smem + G::STAGE_BYTES * STAGES;
    float4* epi_stage = reinterpret_cast<float4*>(smem + G::RING_BYTES);   // [4 warps][2][256]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::RING_BYTES + G::EPI_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* conv = bars + 2 * STAGES;
    uint64_t* acc_full = bars + 3 * STAGES;
    uint64_t* acc_empty = bars + 3 * STAGES + 2;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 3 * STAGES + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * STAGES + 4) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const long long first = blockIdx.x >> 1, step = gridDim.x >> 1;
    const int kblocks = (p.K + G::BKE - 1) / G::BKE;

    // The stream-K split is planned on the host for this many clusters and at least one
    // k-block per cluster, the split pieces for at least one k-block each; any other launch
    // does no work and says so (both CTAs return before touching a barrier, so neither
    // waits for the other).
    if ((p.sk_dp < p.num_tiles &&
         (p.sk_clusters != (int)step || (p.num_tiles - p.sk_dp) * (long long)kblocks < step)) ||
        (p.sk_split > 1 && kblocks < p.sk_split)) {
        if (threadIdx.x == 0) atomicCAS(&g_dev_status, 0, (int)kDevBadLaunch);
        return;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
            mbar_init(smem_u32(&conv[s]), 8);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&acc_full[a]), 1);
            mbar_init(smem_u32(&acc_empty[a]), 8);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32((const void*)tmem_slot), G::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();   // barriers of both CTAs initialised, TMEM allocated in both
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    Item item;
    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (Sched sc(p, kblocks, first, step); sc.next(p, item);) {
                int b, mb, nb;
                umma::tile_coords(p, item.tile, b, mb, nb);
                const int m0 = mb * BM + (int)rank * BMC;
                const int n0 = nb * BN + (int)rank * G::BH;
                const int ab = p.a_batched ? b : 0, bb = p.b_batched ? b : 0;
                for (int kb = item.kb0; kb < item.kb1; ++kb) {
                    if (!mbar_wait_cl(smem_u32(&empty[s]), ph ^ 1, abort_flag, kDevTimeoutEmpty)) goto done;
                    const uint32_t sa = smem_u32(ring + s * G::STAGE_BYTES);
                    const uint32_t sb = sa + G::A_BYTES;
                    const int k0 = kb * G::BKE;
                    uint32_t bar;
                    if (X3) {
                        bar = smem_u32(&full[s]);
                        mbar_arrive_expect_tx(bar, G::STAGE_BYTES);
                    } else {
                        if (leader) mbar_arrive_expect_tx(smem_u32(&full[s]), 2 * G::STAGE_BYTES);
                        bar = mapa_shared(smem_u32(&full[s]), 0);
                    }
                    auto load = [&](uint32_t dst, const CUtensorMap* m, int c0, int c1, int c2) {
                        if (X3) tma_load_3d(dst, m, bar, c0, c1, c2);
                        else tma_load_3d_pair(dst, m, bar, c0, c1, c2);
                    };
                    if (A_MN) {
#pragma unroll
                        for (int c = 0; c < BMC / (int)G::CHUNK; ++c)
                            load(sa + c * G::MN_CHUNK_BYTES, &tmA, m0 + c * G::CHUNK, k0, ab);
                    } else {
                        load(sa, &tmA, k0, m0, ab);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int c = 0; c < G::BH / (int)G::CHUNK; ++c)
                            load(sb + c * G::MN_CHUNK_BYTES, &tmB, n0 + c * G::CHUNK, k0, bb);
                    } else {
                        load(sb, &tmB, k0, n0, bb);
                    }
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer (even CTA) ---------------------
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = umma_idesc_tf32(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
            int s = 0;
            uint32_t ph = 0;
            int it = 0;
            for (Sched sc(p, kblocks, first, step); sc.next(p, item); ++it) {
                const int a = it & 1;
                const uint32_t aph = (it >> 1) & 1;
                if (!mbar_wait_cl(smem_u32(&acc_empty[a]), aph ^ 1, abort_flag, kDevTimeoutAccEmpty)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + a * BN;
                for (int kb = item.kb0; kb < item.kb1; ++kb) {
                    const uint32_t wbar = X3 ? smem_u32(&conv[s]) : smem_u32(&full[s]);
                    if (!mbar_wait_cl(wbar, ph, abort_flag, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(ring + s * G::STAGE_BYTES);
                    const uint32_t sb = sa + G::A_BYTES;
#pragma unroll
                    for (int k = 0; k < G::KSTEPS; ++k) {
                        const uint64_t ad = umma::operand_desc<A_MN, BKE>(sa, k);
                        const uint64_t bd = umma::operand_desc<B_MN, BKE>(sb, k);
                        const uint32_t acc = (kb > item.kb0 || k > 0) ? 1u : 0u;
                        if (X3) {
                            const uint32_t la = smem_u32(ring_lo + s * G::STAGE_BYTES);
                            const uint32_t lb = la + G::A_BYTES;
                            umma_tf32_pair(d_tmem, umma::operand_desc<A_MN, BKE>(la, k), bd, idesc, acc);
                            umma_tf32_pair(d_tmem, ad, umma::operand_desc<B_MN, BKE>(lb, k), idesc, 1u);
                            umma_tf32_pair(d_tmem, ad, bd, idesc, 1u);
                        } else {
                            umma_tf32_pair(d_tmem, ad, bd, idesc, acc);
                        }
                    }
                    umma_commit_pair(smem_u32(&empty[s]));
                    umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                umma_commit_pair(smem_u32(&acc_full[a]));
                umma_commit_pair(mapa_shared(smem_u32(&acc_full[a]), 1));
            }
        }
    } else if (warp < 6) {
        // ------------------------------ epilogue ----------------------------------
        const int q = warp & 3;
        int it = 0, seq = 0;
        for (Sched sc(p, kblocks, first, step); sc.next(p, item); ++it) {
            int b, mb, nb;
            umma::tile_coords(p, item.tile, b, mb, nb);
            const int a = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!mbar_wait_cl(smem_u32(&acc_full[a]), aph, abort_flag, kDevTimeoutAccFull)) goto done;
            __syncwarp();
            tc_fence_after();
            const int m0w = mb * BM + (int)rank * BMC + q * 32;   // this warp's first row
            const int m = m0w + lane;
            const int64_t row_off = (int64_t)b * p.sc_b + (int64_t)m * p.sc_m;
            const float bias_row = (p.epi & 1) && m < p.M ? __ldg(p.bias + m) : 0.f;
            // Epilogue of one finished 32-column chunk c: bias / ReLU, then the stores.
            auto finish = [&](float (&v)[32], int c) {
                const int n0 = nb * BN + c * 32;
                if (p.epi) {   // plain product: no per-element tests in a loop one warp runs alone
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float x = v[j] + bias_row;
                        if (p.epi & 2) x = x + ((n0 + j < p.N) ? __ldg(p.bias + n0 + j) : 0.f);
                        if (p.epi & 4) x = x > 0.f ? x : 0.f;
                        v[j] = x;
                    }
                }
                if (p.tma_multi) {
                    umma::store_block_tma(dm, p.ndst, epi_stage + q * 512, seq, v, lane, n0, m0w, b, p.M, p.N);
                } else if (p.vec_store && n0 + 32 <= p.N && p.ndst > 1) {
                    // several destinations (peers over NVLink): whole-row stores
                    umma::store_block_lines(epi_stage + q * 512, v, lane, p, (int64_t)b * p.sc_b, m0w, n0);
                } else if (p.vec_store && n0 + 32 <= p.N) {
                    // one destination without tensor maps (the TMA epilogue switched
                    // off): straight from registers
                    if (m < p.M) {
                        float* crow = p.dst[0] + row_off;
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(crow + n0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    }
                } else if (m < p.M) {
#pragma unroll
                    for (int d = 0; d < umma::kMaxDst; ++d) {
                        if (d >= p.ndst) break;
                        float* crow = p.dst[d] + row_off;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + j < p.N) crow[n0 + j] = v[j];
                    }
                }
            };
            const bool part = item.nseg > 1;
            const long long skt = item.tile - p.sk_t0;
            // This warp's row of the partial slots of a cut tile (slot stride 256 x BN).
            const long long slot_row = (umma::sk_slot(p, item.tile) * BM + (int)rank * BMC + q * 32 + lane) * (long long)BN;
            const long long slot_stride = (long long)BM * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + a * BN + c * 32, r);
                tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[a]), 0));
                }
                if (part) {
                    // Raw partial sum to this piece's slot (L2; other SMs read it).
                    float4* w = reinterpret_cast<float4*>(p.sk_ws + slot_row + item.seg * slot_stride + c * 32);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        __stcg(w + j, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                  __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
                    continue;
                }
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                finish(v, c);
            }
            if (part) {
                // Count this piece; the last of the tile's pieces to arrive sums all of
                // them in k order (slot 0 first) and writes the tile. No one waits.
                __threadfence();
                __syncwarp();
                int old = 0;
                if (lane == 0) old = atomicAdd(p.sk_cnt + (skt * 2 + (long long)rank) * 4 + q, 1);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == item.nseg - 1) {
                    __threadfence();
#pragma unroll 1
                    for (int c = 0; c < BN / 32; ++c) {
                        float v[32];
                        const float4* r0 = reinterpret_cast<const float4*>(p.sk_ws + slot_row + c * 32);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float4 x = __ldcg(r0 + j);
                            v[4 * j] = x.x; v[4 * j + 1] = x.y; v[4 * j + 2] = x.z; v[4 * j + 3] = x.w;
                        }
                        for (int sg = 1; sg < item.nseg; ++sg) {
                            const float4* rs = reinterpret_cast<const float4*>(p.sk_ws + slot_row + sg * slot_stride + c * 32);
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const float4 x = __ldcg(rs + j);
                                v[4 * j] += x.x; v[4 * j + 1] += x.y; v[4 * j + 2] += x.z; v[4 * j + 3] += x.w;
                            }
                        }
                        finish(v, c);
                    }
                }
            }
        }
    } else if (X3) {
        // ------------------------------ 3xTF32 splitter ---------------------------
        const int ct = threadIdx.x - 6 * 32;
        int s = 0;
        uint32_t ph = 0;
        for (Sched sc(p, kblocks, first, step); sc.next(p, item);) {
            for (int kb = item.kb0; kb < item.kb1; ++kb) {
                if (!mbar_wait(smem_u32(&full[s]), ph, abort_flag, kDevTimeoutMisc)) goto done;
                float4* hi = reinterpret_cast<float4*>(ring + s * G::STAGE_BYTES);
                float4* lo = reinterpret_cast<float4*>(ring_lo + s * G::STAGE_BYTES);
#pragma unroll 4
                for (uint32_t i = ct; i < G::STAGE_BYTES / 16; i += 128) {
                    float4 x = hi[i];
                    float4 h = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
                    hi[i] = h;
                    lo[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&conv[s]), 0));
                if (++s == STAGES) { s = 0; ph ^= 1; }
            }
        }
    }

done:
    if (warp == 0 && lane == 0 && *abort_flag) drain_pause();
    if (warp >= 2 && warp < 6 && lane == 0) bulk_wait_all();   // TMA stores performed, buffers free
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();   // the peer no longer signals us or reads our shared memory / TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, G::TMEM_COLS);
    }
}

}  // namespace umma2
}  // namespace mt
