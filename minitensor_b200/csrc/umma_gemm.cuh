// umma_gemm.cuh -- the tensor-core fp32-input GEMM for sm_100a (tcgen05 + TMA + TMEM).
//
// C[b,m,n] = epi( sum_k A[b,m,k] * B[b,k,n] ) in two precisions:
//   TF32   -- one kind::tf32 MMA per k-step on the raw fp32 tiles.
//   TF32X3 -- the split-precision method of Ootomo & Yokota (2022): x = hi + lo with
//             hi = rna_tf32(x), lo = x - hi; C += Ahi*Bhi + Ahi*Blo + Alo*Bhi, all three
//             products accumulated in the same fp32 TMEM accumulator.
//
// Layout of work. One persistent CTA per SM walks output tiles of 128 x BN, BKE (32 for
// TF32, 16 for TF32X3) k-elements per pipeline stage. Warp roles:
//   warp 0      TMA producer: swizzled tiles into a STAGES-deep shared-memory ring,
//               completion counted on mbarriers (plain per-CTA loads).
//   warp 1      TMEM owner and single-thread MMA issuer (tcgen05.mma.cta_group::1).
//   warps 2-5   epilogue: TMEM -> registers (tcgen05.ld 32x32b) -> bias/ReLU -> global.
//   warps 6-9   (TF32X3 only) converter: splits each landed stage into hi (in place) and
//               lo (a parallel ring), then hands the stage to the MMA issuer.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// Operand layouts come straight from the views: A is K-major (row-major A) or M-major (a
// transposed view), B is K-major (a transposed view, e.g. W^T) or N-major (row-major B).
// The instruction descriptor's major bits select the smem layout, so NN, NT and TN need
// no copies. Ragged M/N/K edges are zero-filled by TMA and clipped in the epilogue.
#pragma once

#include "mt_common.cuh"

namespace mt {
namespace umma {

constexpr int BM = 128;
constexpr int kMaxDst = 8;      // output copies (one per GPU of a sharded GEMM)

struct Params {
    int M, N, K, batch;
    int a_batched, b_batched;   // operand has a batch dimension in its tensor map
    // The epilogue writes every tile to each of the ndst outputs: dst[0] is the local C;
    // for a column-sharded GEMM over several GPUs, dst[1..] are the same shard columns
    // of the other GPUs' C buffers (peer pointers), so the all-gather of C happens in
    // the epilogue, tile by tile, while the next tile's main loop runs.
    float* dst[kMaxDst];
    int ndst;
    int64_t sc_b, sc_m;         // C element strides (n stride is 1), same for every dst
    const float* bias;
    int epi;
    int vec_store;              // rows 16-byte aligned and N % 4 == 0
    int tiles_m, tiles_n;
    long long num_tiles;        // output tiles
    // Split-K: unit u is tile u / splits, k-split u % splits (k-blocks [kb0, kb1)); the
    // epilogue of split s writes raw partial sums at dst[d] + s * split_stride.
    int splits;
    int64_t split_stride;
    long long num_units;        // num_tiles * splits
    // TMA epilogue: each warp hands its 32 x 32 blocks to the TMA engine, one tensor store
    // per destination (maps in DstMaps, C as {N, M, batch}, box {32, 32, 1}, 128-byte
    // swizzle), whole lines instead of a 16-byte piece of 32 rows per store instruction,
    // and SM stores to peer memory top out far below the link rate. Off (0) for split-K
    // partials, rows that are not 16-byte aligned, or with MT_TMA_EPILOGUE=0.
    int tma_multi;
    // Stream-K remainder (CTA-pair kernel only; splits == 1 there). Tiles [0, sk_dp) run
    // whole, round-robin over the clusters. The k-blocks of tiles [sk_dp, num_tiles),
    // taken tile after tile, are cut into one contiguous range per cluster, so that every
    // cluster ends at the same time instead of some running one tile more than others.
    // A tile cut between clusters: every contributing warp writes its raw partial to
    // sk_ws and counts itself in sk_cnt; the last to arrive sums the partials in k order
    // (a fixed order, so the result does not depend on timing) and runs the epilogue.
    // sk_dp == num_tiles turns it off. With sk_split = S > 1 the whole tiles are themselves
    // cut into S near-equal k-ranges handed out round-robin as separate units (the same
    // partial slots and last-arriver sum): a sharded GEMM with few rounds of tiles then
    // finishes tiles twice as often, so its stores to the peers start earlier.
    long long sk_dp;
    int sk_clusters;            // clusters in the launch
    int sk_split;               // S: pieces per whole tile (1 = whole tiles)
    int sk_maxseg;              // partial slots per stream-K tile
    long long sk_t0;            // first tile with slots (0 when S > 1, else sk_dp)
    float* sk_ws;               // partial slots [256 rows][BN] each: S per split whole tile in
                                // [sk_t0, sk_dp), then sk_maxseg per stream-K tile (sk_slot)
    int* sk_cnt;                // [tile - sk_t0][2 CTAs][4 warps] arrivals, zero at launch
};

// First partial slot of a tile cut into pieces (see sk_ws).
__host__ __device__ __forceinline__ long long sk_slot(const Params& p, long long tile) {
    return tile < p.sk_dp ? (tile - p.sk_t0) * p.sk_split
                          : (p.sk_dp - p.sk_t0) * p.sk_split + (tile - p.sk_dp) * p.sk_maxseg;
}

// Tensor maps of the ndst destinations (same view, different base pointers).
struct DstMaps {
    CUtensorMap m[kMaxDst];
};

// k-blocks of split `sp`: a near-equal contiguous share of [0, kblocks).
__device__ __forceinline__ void split_range(const Params& p, int kblocks, int sp, int& kb0, int& kb1) {
    kb0 = (int)((long long)kblocks * sp / p.splits);
    kb1 = (int)((long long)kblocks * (sp + 1) / p.splits);
}

template <int BN, int BKE_, bool X3, int STAGES>
struct Cfg {
    static constexpr int BKE = BKE_;                           // k elements per stage (16 or 32)
    static constexpr int KSWB = BKE * 4;                       // K-major swizzle span, bytes
    static constexpr uint32_t A_BYTES = BM * BKE * 4;
    static constexpr uint32_t B_BYTES = BN * BKE * 4;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int KSTEPS = BKE / 8;                     // tf32 MMA K = 8
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr int NUM_WARPS = X3 ? 10 : 6;
    static constexpr int THREADS = NUM_WARPS * 32;
    static constexpr uint32_t RING_BYTES = STAGE_BYTES * STAGES * (X3 ? 2 : 1);
    static constexpr uint32_t EPI_BYTES = 4 * 8192;                // epilogue staging, 2 x 4 KB per warp
    static constexpr uint32_t BAR_BYTES = 8 * (3 * STAGES + 4) + 16;
    static constexpr uint32_t SMEM_BYTES = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES;
    static constexpr uint32_t CHUNK = 32;                      // MN-major: 32 elements (128 B) per row
    // MN-major: one chunk = BKE k-rows x 128 bytes.
    static constexpr uint32_t MN_CHUNK_BYTES = BKE * 128;
};

// Tile t -> (batch, m block, n block); m blocks are grouped by 8 so that consecutive CTAs
// share B tiles in L2.
__device__ __forceinline__ void tile_coords(const Params& p, long long t, int& b, int& mb, int& nb) {
    constexpr int G = 8;
    if (p.num_tiles < (1ll << 28)) {
        // Every quotient below fits 32 bits (8 * tiles_n <= 8 * num_tiles < 2^31): 32-bit
        // division, several times cheaper than the 64-bit routine, which matters on the
        // epilogue warps of short-K problems where this runs once per tile per role.
        const unsigned per_batch = (unsigned)p.tiles_m * (unsigned)p.tiles_n;
        const unsigned tt = (unsigned)t;
        const unsigned bb = tt / per_batch;
        const unsigned r = tt - bb * per_batch;
        const unsigned gw = (unsigned)G * (unsigned)p.tiles_n;
        const unsigned group = r / gw;
        const int first_m = (int)(group * G);
        const unsigned gsize = (unsigned)min(p.tiles_m - first_m, G);
        const unsigned in_group = r - group * gw;
        const unsigned q = in_group / gsize;
        b = (int)bb;
        mb = first_m + (int)(in_group - q * gsize);
        nb = (int)q;
        return;
    }
    const long long per_batch = (long long)p.tiles_m * p.tiles_n;
    b = (int)(t / per_batch);
    long long r = t % per_batch;
    long long group = r / ((long long)G * p.tiles_n);
    int first_m = (int)(group * G);
    int gsize = min(p.tiles_m - first_m, G);
    long long in_group = r % ((long long)G * p.tiles_n);
    mb = first_m + (int)(in_group % gsize);
    nb = (int)(in_group / gsize);
}

// Stores one warp's 32 x 32 block of C (lane i holds row m0w + i, columns n0 .. n0+31 in
// v) to every destination as whole 128-byte rows: the block passes through a 4 KB shared
// tile (16-byte chunks XOR-swizzled by row, conflict-free both ways) so that each store
// instruction covers 4 complete rows instead of 16 bytes of 32 rows. Over NVLink this turns
// 32 partial-line writes per instruction into 4 full-line ones. Warp-collective; rows at or
// past M are skipped. `base` = offset of row 0 (batch and split already applied).
__device__ __forceinline__ void store_block_lines(float4* stage, const float (&v)[32], int lane, const Params& p,
                                                  int64_t base, int m0w, int n0) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
        stage[lane * 8 + (j ^ (lane & 7))] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int r = 4 * k + (lane >> 3), c = lane & 7;
        const float4 x = stage[r * 8 + (c ^ (r & 7))];
        const int m = m0w + r;
        if (m < p.M) {
            const int64_t off = base + (int64_t)m * p.sc_m + n0 + 4 * c;
#pragma unroll
            for (int d = 0; d < kMaxDst; ++d) {
                if (d >= p.ndst) break;
                *reinterpret_cast<float4*>(p.dst[d] + off) = x;
            }
        }
    }
    __syncwarp();   // the tile is rewritten by the next block
}

// Hands one warp's 32 x 32 block (lane i = row m0w + i, columns n0..n0+31 in v) to the TMA
// engine for every destination: the block goes into a 4 KB shared buffer in the 128-byte
// swizzled layout of the maps (16-byte chunk j of row r at j ^ (r & 7)), then lane 0
// issues one tensor store per destination; TMA clips rows / columns past C's edge, and a
// block wholly past the edge is skipped (no store starts outside C). Two buffers per warp
// alternate; `seq` counts the warp's blocks, and a buffer is rewritten only after the
// stores that read it two blocks earlier are done reading.
__device__ __forceinline__ void store_block_tma(const DstMaps& dm, int ndst, float4* bufs, int& seq,
                                                const float (&v)[32], int lane, int n0, int m0w, int bz, int M, int N) {
    if (m0w >= M || n0 >= N) return;
    float4* buf = bufs + (seq & 1) * 256;
    if (seq >= 2) {
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
        buf[lane * 8 + (j ^ (lane & 7))] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        for (int d = 0; d < ndst; ++d) tma_store_3d(&dm.m[d], smem_u32(buf), n0, m0w, bz);
        bulk_commit();
    }
    ++seq;
}

template <bool MN_MAJOR, int BKE>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kstep) {
    if (MN_MAJOR) {
        // k-step of 8 rows = 1024 bytes; LBO = next 32-element MN chunk, SBO = next
        // 4-row K group.
        return umma_desc(base + kstep * 8 * 128, BKE * 128, 4 * 128, kLayoutSw128Base32);
    } else {
        // k-step of 8 tf32 = 32 bytes inside the swizzled row; SBO = 8 rows.
        return umma_desc(base + kstep * 32, 16, 8 * BKE * 4, BKE == 32 ? kLayoutSw128 : kLayoutSw64);
    }
}

template <int BN, int BKE, bool A_MN, bool B_MN, bool X3, int STAGES>
__global__ void __launch_bounds__(Cfg<BN, BKE, X3, STAGES>::THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ DstMaps dm, const Params p) {
    using G = Cfg<BN, BKE, X3, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;                                      // [STAGES][A|B]
    uint8_t* ring_lo = smem + G::STAGE_BYTES * STAGES;         // X3: [STAGES][Alo|Blo]
    float4* epi_stage = reinterpret_cast<float4*>(smem + G::RING_BYTES);   // [4 warps][2][256]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::RING_BYTES + G::EPI_BYTES);
    uint64_t* full = bars;                                     // TMA landed
    uint64_t* empty = bars + STAGES;                           // MMA done with stage
    uint64_t* conv = bars + 2 * STAGES;                        // X3: split done
    uint64_t* acc_full = bars + 3 * STAGES;                    // [2]
    uint64_t* acc_empty = bars + 3 * STAGES + 2;               // [2]
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 3 * STAGES + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * STAGES + 4) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long first_tile = blockIdx.x, tile_step = gridDim.x;
    const int kblocks = (p.K + G::BKE - 1) / G::BKE;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
            mbar_init(smem_u32(&conv[s]), 128);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&acc_full[a]), 1);
            mbar_init(smem_u32(&acc_empty[a]), 128);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32((const void*)tmem_slot), G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (long long u = first_tile; u < p.num_units; u += tile_step) {
                int b, mb, nb, kb0, kb1;
                tile_coords(p, u / p.splits, b, mb, nb);
                split_range(p, kblocks, (int)(u % p.splits), kb0, kb1);
                const int m0 = mb * BM, n0 = nb * BN;
                const int ab = p.a_batched ? b : 0, bb = p.b_batched ? b : 0;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1, abort_flag, kDevTimeoutEmpty)) goto done;
                    const uint32_t bar = smem_u32(&full[s]);
                    mbar_arrive_expect_tx(bar, G::STAGE_BYTES);
                    const uint32_t sa = smem_u32(ring + s * G::STAGE_BYTES);
                    const uint32_t sb = sa + G::A_BYTES;
                    const int k0 = kb * G::BKE;
                    if (A_MN) {
#pragma unroll
                        for (int c = 0; c < BM / (int)G::CHUNK; ++c)
                            tma_load_3d(sa + c * G::MN_CHUNK_BYTES, &tmA, bar, m0 + c * G::CHUNK, k0, ab);
                    } else {
                        tma_load_3d(sa, &tmA, bar, k0, m0, ab);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int c = 0; c < BN / (int)G::CHUNK; ++c)
                            tma_load_3d(sb + c * G::MN_CHUNK_BYTES, &tmB, bar, n0 + c * G::CHUNK, k0, bb);
                    } else {
                        tma_load_3d(sb, &tmB, bar, k0, n0, bb);
                    }
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer --------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_tf32(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
            int s = 0;
            uint32_t ph = 0;
            int it = 0;
            for (long long u = first_tile; u < p.num_units; u += tile_step, ++it) {
                int kb0, kb1;
                split_range(p, kblocks, (int)(u % p.splits), kb0, kb1);
                const int a = it & 1;
                const uint32_t aph = (it >> 1) & 1;
                if (!mbar_wait(smem_u32(&acc_empty[a]), aph ^ 1, abort_flag, kDevTimeoutAccEmpty)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + a * BN;
                for (int kb = kb0; kb < kb1; ++kb) {
                    uint32_t wbar = X3 ? smem_u32(&conv[s]) : smem_u32(&full[s]);
                    if (!mbar_wait(wbar, ph, abort_flag, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(ring + s * G::STAGE_BYTES);
                    const uint32_t sb = sa + G::A_BYTES;
#pragma unroll
                    for (int k = 0; k < G::KSTEPS; ++k) {
                        const uint64_t ad = operand_desc<A_MN, BKE>(sa, k);
                        const uint64_t bd = operand_desc<B_MN, BKE>(sb, k);
                        const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
                        if (X3) {
                            const uint32_t la = smem_u32(ring_lo + s * G::STAGE_BYTES);
                            const uint32_t lb = la + G::A_BYTES;
                            const uint64_t ald = operand_desc<A_MN, BKE>(la, k);
                            const uint64_t bld = operand_desc<B_MN, BKE>(lb, k);
                            umma_tf32(d_tmem, ald, bd, idesc, acc);   // Alo * Bhi
                            umma_tf32(d_tmem, ad, bld, idesc, 1u);    // Ahi * Blo
                            umma_tf32(d_tmem, ad, bd, idesc, 1u);     // Ahi * Bhi
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
    } else if (warp < 6) {
        // ------------------------------ epilogue ----------------------------------
        const int q = warp & 3;   // TMEM lane quarter this warp may access
        int it = 0, seq = 0;
        for (long long u = first_tile; u < p.num_units; u += tile_step, ++it) {
            int b, mb, nb, kb0, kb1;
            tile_coords(p, u / p.splits, b, mb, nb);
            const int sp = (int)(u % p.splits);
            split_range(p, kblocks, sp, kb0, kb1);
            const bool no_k = kb1 <= kb0;   // this split got no k-blocks: its partial is zero
            const int a = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!mbar_wait(smem_u32(&acc_full[a]), aph, abort_flag, kDevTimeoutAccFull)) goto done;
            __syncwarp();   // tcgen05.ld below is .sync.aligned: reconverge after the spin
            tc_fence_after();
            const int m = mb * BM + q * 32 + lane;
            const int64_t row_off = (int64_t)b * p.sc_b + (int64_t)m * p.sc_m + (int64_t)sp * p.split_stride;
            const float bias_row = (p.epi & 1) && m < p.M ? __ldg(p.bias + m) : 0.f;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + a * BN + c * 32, r);
                tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    mbar_arrive(smem_u32(&acc_empty[a]));
                }
                const int n0 = nb * BN + c * 32;
                float v[32];
                if (p.epi == 0 && !no_k) {
                    // plain product: no per-element tests in a loop that one warp runs alone
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float x = (no_k ? 0.f : __uint_as_float(r[j])) + bias_row;
                        if (p.epi & 2) x = x + ((n0 + j < p.N) ? __ldg(p.bias + n0 + j) : 0.f);
                        if (p.epi & 4) x = x > 0.f ? x : 0.f;
                        v[j] = x;
                    }
                }
                if (p.tma_multi) {
                    store_block_tma(dm, p.ndst, epi_stage + q * 512, seq, v, lane, n0, mb * BM + q * 32, b, p.M, p.N);
                } else if (p.vec_store && n0 + 32 <= p.N && p.ndst > 1) {
                    // several destinations (peers over NVLink): whole-row stores
                    store_block_lines(epi_stage + q * 512, v, lane, p,
                                      (int64_t)b * p.sc_b + (int64_t)sp * p.split_stride, mb * BM + q * 32, n0);
                } else if (p.vec_store && n0 + 32 <= p.N) {
                    // one destination without tensor maps (split-K partials, or the TMA
                    // epilogue switched off): straight from registers
                    if (m < p.M) {
                        float* crow = p.dst[0] + row_off;
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(crow + n0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    }
                } else if (m < p.M) {
#pragma unroll
                    for (int d = 0; d < kMaxDst; ++d) {
                        if (d >= p.ndst) break;
                        float* crow = p.dst[d] + row_off;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + j < p.N) crow[n0 + j] = v[j];
                    }
                }
            }
        }
    } else if (X3) {
        // ------------------------------ 3xTF32 splitter ---------------------------
        const int ct = threadIdx.x - 6 * 32;   // 0..127
        int s = 0;
        uint32_t ph = 0;
        for (long long u = first_tile; u < p.num_units; u += tile_step) {
            int kb0, kb1;
            split_range(p, kblocks, (int)(u % p.splits), kb0, kb1);
            for (int kb = kb0; kb < kb1; ++kb) {
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
                mbar_arrive(smem_u32(&conv[s]));
                if (++s == STAGES) { s = 0; ph ^= 1; }
            }
        }
    }

done:
    if (warp >= 2 && warp < 6 && lane == 0) bulk_wait_all();   // TMA stores performed, buffers free
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, G::TMEM_COLS);
    }
}

// C[m, n] = epi(sum over splits s (in order) of ws[s][m][n]); ws rows have N elements.
__global__ void splitk_epilogue_kernel(const float* __restrict__ ws, int splits, int M, int N, float* C, int64_t sc_m,
                                       const float* __restrict__ bias, int epi) {
    const int64_t total = (int64_t)M * N;
    const int64_t plane = total;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), n = (int)(i - (int64_t)m * N);
        float acc = 0.f;
        for (int s = 0; s < splits; ++s) acc += ws[s * plane + i];
        if (epi & 1) acc = acc + __ldg(bias + m);
        if (epi & 2) acc = acc + __ldg(bias + n);
        if (epi & 4) acc = acc > 0.f ? acc : 0.f;
        C[(int64_t)m * sc_m + n] = acc;
    }
}

}  // namespace umma
}  // namespace mt
