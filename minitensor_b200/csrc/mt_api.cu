// mt_api.cu -- the C ABI of libmtgemm.so (declared in include/mtgemm.h): argument
// checks with the reference's error semantics, view -> problem mapping, kernel
// selection, TMA tensor-map encoding and launches.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "mtgemm.h"
#include "mt_common.cuh"
#include "simt_gemm.cuh"
#include "umma_gemm.cuh"
#include "umma_gemm2.cuh"
#include "conv_gemm.cuh"
#include "conv_tma.cuh"
#include "conv_halo.cuh"
#include "conv_halo2.cuh"
#include "conv_wgrad.cuh"
#include "conv_simt.cuh"

namespace {

using mt::GemmProblem;

thread_local std::string t_err;
thread_local std::string t_path;
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_default_mode{-2};   // -2: not yet read from the environment

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(MT_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

int resolve_mode(int mode) {
    if (mode >= MT_STRICT_FP32 && mode <= MT_TF32X3) return mode;
    int d = g_default_mode.load();
    if (d == -2) {
        d = MT_TF32X3;
        if (const char* e = std::getenv("MT_GEMM_MODE")) {
            if (!strcmp(e, "strict") || !strcmp(e, "fp32")) d = MT_STRICT_FP32;
            else if (!strcmp(e, "tf32")) d = MT_TF32;
            else if (!strcmp(e, "tf32x3") || !strcmp(e, "3xtf32")) d = MT_TF32X3;
        }
        int expect = -2;
        g_default_mode.compare_exchange_strong(expect, d);
        d = g_default_mode.load();
    }
    return d;
}

// ------------------------------- device properties -------------------------------
struct DevInfo {
    int sms = 0;
    int cc = 0;
};

DevInfo dev_info() {
    static std::mutex mu;
    static DevInfo cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    DevInfo& d = cache[dev & 63];
    if (d.sms == 0) {
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        int maj = 0, mnr = 0;
        cudaDeviceGetAttribute(&maj, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&mnr, cudaDevAttrComputeCapabilityMinor, dev);
        d.cc = maj * 10 + mnr;
    }
    return d;
}

// ------------------------------- TMA descriptors ---------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 3-D fp32 map {d0 (contiguous), d1, d2} with byte strides s1, s2 and box {b0, b1, 1}.
bool encode_3d(CUtensorMap* m, const float* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
               uint64_t s2, uint32_t b0, uint32_t b1, int swizzle_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, 1};
    cuuint32_t es[3] = {1, 1, 1};
    // swizzle_bytes: 128 / 64 = 16-byte granules (K-major operands); 32 = the 128-byte
    // span with 32-byte granules that MN-major tf32 operands require.
    CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swizzle_bytes == 32  ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                 : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 4-D fp32 map {d0 (contiguous), d1, d2, d3}, byte strides s[0..2] of d1..d3, box b[4].
bool encode_4d(CUtensorMap* m, const float* base, const uint64_t (&d)[4], const uint64_t (&st)[3],
               const uint32_t (&b)[4], int swizzle_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {d[0], d[1], d[2], d[3]};
    cuuint64_t strides[3] = {st[0], st[1], st[2]};
    cuuint32_t box[4] = {b[0], b[1], b[2], b[3]};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 32  ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                 : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

uint64_t round16(uint64_t x) { return (x + 15) & ~uint64_t(15); }

// ------------------------------- views -> problem --------------------------------
struct View {
    const float* ptr;
    int64_t d[3];   // batch, rows, cols
    int64_t s[3];
};

int to_view(const mt_tensor* t, int want_ndim, const char* name, View& v) {
    if (!t) return fail(MT_EINVAL, "%s: null tensor", name);
    if ((int)t->ndim != want_ndim) return fail(MT_EINVAL, "%s: expected a %d-D tensor, got %u-D", name, want_ndim, t->ndim);
    v.ptr = t->data ? t->data + t->offset : nullptr;
    if (want_ndim == 2) {
        v.d[0] = 1; v.s[0] = 0;
        v.d[1] = (int64_t)t->shape[0]; v.s[1] = (int64_t)t->strides[0];
        v.d[2] = (int64_t)t->shape[1]; v.s[2] = (int64_t)t->strides[1];
    } else {
        for (int i = 0; i < 3; ++i) { v.d[i] = (int64_t)t->shape[i]; v.s[i] = (int64_t)t->strides[i]; }
    }
    if (v.d[1] * v.d[2] * v.d[0] > 0 && !t->data) return fail(MT_EINVAL, "%s: null data pointer", name);
    return MT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ------------------------------- launchers ---------------------------------------
int launch_simt(const GemmProblem& p, cudaStream_t st) {
    using namespace mt;
    int la = kLdGeneric, lb = kLdGeneric;
    const bool okA = aligned16(p.A) && ((p.batch == 1 || p.sa_b % 4 == 0));
    const bool okB = aligned16(p.B) && ((p.batch == 1 || p.sb_b % 4 == 0));
    if (okA && p.sa_k == 1 && p.sa_m % 4 == 0) la = kLdKContigVec;
    else if (okA && p.sa_m == 1 && p.sa_k % 4 == 0) la = kLdMNContigVec;
    if (okB && p.sb_n == 1 && p.sb_k % 4 == 0) lb = kLdMNContigVec;
    else if (okB && p.sb_k == 1 && p.sb_n % 4 == 0) lb = kLdKContigVec;
    dim3 grid((unsigned)((p.N + simt::BN - 1) / simt::BN), (unsigned)((p.M + simt::BM - 1) / simt::BM),
              (unsigned)p.batch);
    // Fewer 128 x 128 tiles than SMs: 64 x 64 tiles, 4x the CTAs (the per-output order and
    // so the bits are the same; strict fp32 cannot split K).
    const bool small = (long long)grid.x * grid.y * grid.z < (long long)dev_info().sms;
    if (small)
        grid = dim3((unsigned)((p.N + simt::small::BN - 1) / simt::small::BN),
                    (unsigned)((p.M + simt::small::BM - 1) / simt::small::BM), (unsigned)p.batch);
    if (grid.y > 65535 || grid.z > 65535) return fail(MT_EUNSUPPORTED, "simt: grid too large (M=%lld batch=%lld)",
                                                      (long long)p.M, (long long)p.batch);
#define MT_SIMT_CASE(LA, LB)                                                                          \
    if (la == LA && lb == LB) {                                                                       \
        if (small) simt::small::gemm_kernel<LA, LB><<<grid, simt::small::THREADS, 0, st>>>(p);        \
        else simt::gemm_kernel<LA, LB><<<grid, simt::THREADS, 0, st>>>(p);                            \
    }
    MT_SIMT_CASE(kLdKContigVec, kLdMNContigVec)
    else MT_SIMT_CASE(kLdKContigVec, kLdKContigVec)
    else MT_SIMT_CASE(kLdKContigVec, kLdGeneric)
    else MT_SIMT_CASE(kLdMNContigVec, kLdMNContigVec)
    else MT_SIMT_CASE(kLdMNContigVec, kLdKContigVec)
    else MT_SIMT_CASE(kLdMNContigVec, kLdGeneric)
    else MT_SIMT_CASE(kLdGeneric, kLdMNContigVec)
    else MT_SIMT_CASE(kLdGeneric, kLdKContigVec)
    else MT_SIMT_CASE(kLdGeneric, kLdGeneric)
#undef MT_SIMT_CASE
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, "simt gemm launch");
    g_launches.fetch_add(1);
    static const char* names[3] = {"K", "MN", "gen"};
    t_path = std::string(small ? "simt_fp32 tile=64 a=" : "simt_fp32 a=") + names[la] + " b=" + names[lb];
    return MT_OK;
}

template <int BN, int BKE, bool AMN, bool BMN, bool X3, int STAGES>
int launch_umma_inst(const CUtensorMap& ta, const CUtensorMap& tb, const mt::umma::DstMaps& dm,
                     const mt::umma::Params& up, int grid, cudaStream_t st) {
    using G = mt::umma::Cfg<BN, BKE, X3, STAGES>;
    auto kern = mt::umma::gemm_kernel<BN, BKE, AMN, BMN, X3, STAGES>;
    static std::atomic<uint64_t> attr_set_mask{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set_mask.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "umma gemm: set smem attribute");
        attr_set_mask.fetch_or(bit);
    }
    kern<<<grid, G::THREADS, G::SMEM_BYTES, st>>>(ta, tb, dm, up);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, "umma gemm launch");
    g_launches.fetch_add(1);
    return MT_OK;
}

// ---- scratch memory ----------------------------------------------------------------
// Every temporary buffer of the library (split-K and stream-K partials, the NHWC copy and
// reordered weights of the stride-1 conv, weight-grad partials) comes from scratch_alloc.
// By default that is a stream-ordered allocation from the library's own pool
// (cudaMallocFromPoolAsync / cudaFreeAsync on the call's stream: capturable, freed in
// stream order).
// A host that manages device memory itself installs its allocator with
// mt_set_scratch_allocator; the library then returns each block right after enqueuing the
// kernels that use it, which is safe for work ordered on one stream.
struct ScratchHook {
    mt_scratch_alloc_fn alloc = nullptr;
    mt_scratch_free_fn free = nullptr;
    void* ctx = nullptr;
};
std::mutex g_scratch_mu;
ScratchHook g_scratch;
std::atomic<uint64_t> g_async_allocs{0}, g_hook_allocs{0};

ScratchHook scratch_hook() {
    std::lock_guard<std::mutex> g(g_scratch_mu);
    return g_scratch;
}

// The library's own stream-ordered pool on the current device, created on first use. It
// keeps freed memory cached (release threshold: no limit) instead of returning it to the
// driver at every synchronisation, as the device's default pool does: re-mapping a
// 100 MB workspace cost ~0.45 ms of host time on the first call after each sync. Other
// users of the default pool are not affected. Null if the pool cannot be made (the
// default pool is used then).
cudaMemPool_t scratch_pool() {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    static bool tried[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> g(mu);
    if (!tried[dev]) {
        tried[dev] = true;
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        if (cudaMemPoolCreate(&pool, &props) == cudaSuccess) {
            uint64_t keep = ~0ull;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
            pools[dev] = pool;
        } else {
            cudaGetLastError();
        }
    }
    return pools[dev];
}

int scratch_alloc(void** p, size_t bytes, cudaStream_t st, const char* who) {
    *p = nullptr;
    if (bytes == 0) return MT_OK;
    const ScratchHook h = scratch_hook();
    if (h.alloc) {
        int dev = 0;
        cudaGetDevice(&dev);
        *p = h.alloc(bytes, dev, h.ctx);
        if (!*p) return fail(MT_ENOMEM, "%s: the scratch allocator returned NULL for %zu bytes", who, bytes);
        g_hook_allocs.fetch_add(1);
        return MT_OK;
    }
    cudaMemPool_t pool = scratch_pool();
    cudaError_t e = pool ? cudaMallocFromPoolAsync(p, bytes, pool, st) : cudaMallocAsync(p, bytes, st);
    if (e != cudaSuccess) return cuda_fail(e, who);
    g_async_allocs.fetch_add(1);
    return MT_OK;
}

void scratch_free(void* p, size_t bytes, cudaStream_t st) {
    if (!p) return;
    const ScratchHook h = scratch_hook();
    if (h.free) {
        int dev = 0;
        cudaGetDevice(&dev);
        h.free(p, bytes, dev, h.ctx);
    } else {
        cudaFreeAsync(p, st);
    }
}

// Stream-K remainder of a pair launch with `clusters` clusters (see umma::Params). When
// the tiles do not divide into whole rounds over the clusters, the last num_tiles %
// clusters tiles are cut into equal k-block ranges, one per cluster, as long as every range
// gets at least 8 k-blocks. *ws_out receives the stream-ordered workspace (partial slots and
// arrival counters, the counters zeroed on the stream) that the caller frees after the launch.
bool streamk_enabled() {
    static int v = [] {
        const char* e = std::getenv("MT_GEMM_STREAMK");
        return (e && e[0] == '0') ? 0 : 1;
    }();
    return v != 0;
}

int pair_streamk_plan(mt::umma::Params& up, int clusters, int kblocks, int bn, bool split_dp, bool x3, cudaStream_t st,
                      void** ws_out, size_t* ws_bytes_out) {
    *ws_out = nullptr;
    *ws_bytes_out = 0;
    up.sk_dp = up.num_tiles;
    up.sk_clusters = clusters;
    up.sk_split = 1;
    up.sk_maxseg = 0;
    up.sk_t0 = up.num_tiles;
    up.sk_ws = nullptr;
    up.sk_cnt = nullptr;
    if (!streamk_enabled() || clusters <= 0) return MT_OK;
    // Whole tiles in two k-halves: only where asked (a sharded GEMM with few rounds) and
    // with at least 8 k-blocks per half.
    const int S = (split_dp && kblocks >= 16) ? 2 : 1;
    const long long units = up.num_tiles * S;
    long long sk_dp = up.num_tiles;
    int maxseg = 0;
    // The remainder goes to stream-K only where that measured faster: 3xTF32 with more than
    // 5% of the last round idle (e.g. 3.46 rounds: +12% on the 8192 x 2048 x 8192 shard). In
    // TF32 the remainder's k-ranges, run at different k at once, share less of A and B in L2
    // (+24% DRAM bytes, tensor pipe 86% -> 78% active on that shape), which costs more than
    // the idle part of the last round; with 13.8 rounds (8192^3 on one GPU) the last round
    // is 1% of the work.
    const long long rounds_up = (units + clusters - 1) / clusters;
    const bool worth_it = x3 && (double)(rounds_up * clusters - units) / (double)units > 0.05;
    if (units > clusters && worth_it) {
        const long long dp = (units / clusters) * clusters / S;   // whole tiles in whole rounds
        const long long rem = up.num_tiles - dp;
        const long long W = rem * (long long)kblocks;
        if (rem > 0 && W >= 8LL * clusters) {
            sk_dp = dp;
            // A range holds at least floor(W / C) k-blocks, so a tile meets at most this many.
            const long long minr = W / clusters;
            maxseg = (int)((kblocks + minr - 1) / minr + 1);
        }
    }
    if (S == 1 && sk_dp == up.num_tiles) return MT_OK;
    const long long t0 = S > 1 ? 0 : sk_dp;
    // S slots for each split whole tile, maxseg for each stream-K tile (umma::sk_slot).
    const long long nslots = (sk_dp - t0) * S + (up.num_tiles - sk_dp) * (long long)maxseg;
    const size_t ws_bytes = (size_t)nslots * mt::umma2::BM * bn * sizeof(float);
    const size_t cnt_bytes = (size_t)(up.num_tiles - t0) * 8 * sizeof(int);
    void* ws = nullptr;
    int rc = scratch_alloc(&ws, ws_bytes + cnt_bytes, st, "stream-K workspace");
    if (rc) return rc;
    int* cnt = reinterpret_cast<int*>(static_cast<char*>(ws) + ws_bytes);
    cudaError_t e = cudaMemsetAsync(cnt, 0, cnt_bytes, st);
    if (e != cudaSuccess) {
        scratch_free(ws, ws_bytes + cnt_bytes, st);
        return cuda_fail(e, "stream-K counters");
    }
    up.sk_dp = sk_dp;
    up.sk_split = S;
    up.sk_maxseg = maxseg;
    up.sk_t0 = t0;
    up.sk_ws = static_cast<float*>(ws);
    up.sk_cnt = cnt;
    *ws_out = ws;
    *ws_bytes_out = ws_bytes + cnt_bytes;
    return MT_OK;
}

// The pair kernel's schedule for mt_last_path: " split=S" and/or " streamk=<tiles>".
thread_local std::string t_sched;

// CTA-pair kernel: grid = 2 x (clusters that fit at once, capped by the tile count), with
// the stream-K remainder planned for exactly that many clusters.
template <int BN, int BKE, bool AMN, bool BMN, bool X3, int STAGES>
int launch_pair_inst(const CUtensorMap& ta, const CUtensorMap& tb, const mt::umma::DstMaps& dm,
                     mt::umma::Params up, int sms, cudaStream_t st) {
    using G = mt::umma2::Cfg<BN, BKE, X3, STAGES>;
    auto kern = mt::umma2::gemm_pair_kernel<BN, BKE, AMN, BMN, X3, STAGES>;
    static std::atomic<uint64_t> attr_set_mask{0};
    static std::atomic<int> max_clusters[64];
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set_mask.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "umma pair gemm: set smem attribute");
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
        cfg.blockDim = dim3(G::THREADS, 1, 1);
        cfg.dynamicSmemBytes = G::SMEM_BYTES;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sms / 2;
        }
        max_clusters[dev & 63].store(std::min(n, sms / 2));
        attr_set_mask.fetch_or(bit);
    }
    const int clusters = (int)std::min<long long>(up.num_tiles, (long long)max_clusters[dev & 63].load());
    void* ws = nullptr;
    size_t ws_bytes = 0;
    // A GEMM that stores into peers (ndst > 1) with fewer than two rounds of tiles splits
    // its whole tiles in two, so that finished tiles (and their stores) come twice as often.
    const bool split_dp = up.ndst > 1 && up.num_tiles < 2LL * clusters;
    int rc = pair_streamk_plan(up, clusters, (up.K + BKE - 1) / BKE, BN, split_dp, X3, st, &ws, &ws_bytes);
    if (rc) return rc;
    t_sched.clear();
    if (up.sk_split > 1) t_sched += " split=" + std::to_string(up.sk_split);
    if (up.sk_dp < up.num_tiles) t_sched += " streamk=" + std::to_string(up.num_tiles - up.sk_dp);
    kern<<<2 * clusters, G::THREADS, G::SMEM_BYTES, st>>>(ta, tb, dm, up);
    cudaError_t e = cudaGetLastError();
    scratch_free(ws, ws_bytes, st);
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, "umma pair gemm launch");
    g_launches.fetch_add(1);
    return MT_OK;
}

// The pair kernel serves outputs with at least one 256 x 256 tile per SM pair; the
// environment variable MT_GEMM_PAIR=0 turns it off (the 128-row kernel then runs).
bool pair_enabled() {
    static int v = [] {
        const char* e = std::getenv("MT_GEMM_PAIR");
        return (e && e[0] == '0') ? 0 : 1;
    }();
    return v != 0;
}

// TMA-store epilogue for several destinations; MT_TMA_EPILOGUE=0 keeps the SM-store one.
bool tma_epilogue_enabled() {
    static int v = [] {
        const char* e = std::getenv("MT_TMA_EPILOGUE");
        return (e && e[0] == '0') ? 0 : 1;
    }();
    return v != 0;
}

// Returns MT_OK when launched, MT_EUNSUPPORTED when the views do not fit the tensor-core
// kernel (the caller then uses the SIMT kernel).
int launch_umma(const GemmProblem& p, bool x3, cudaStream_t st, float* const* extra_dst = nullptr, int nextra = 0) {
    DevInfo di = dev_info();
    if (di.cc != 100) return fail(MT_EUNSUPPORTED, "umma: device is sm_%d, kernel built for sm_100a", di.cc);
    if (p.M > INT32_MAX || p.N > INT32_MAX || p.K > INT32_MAX || p.batch > INT32_MAX)
        return fail(MT_EUNSUPPORTED, "umma: extent beyond 2^31");
    // Output: unit stride along n, 4-byte element rows.
    if (p.sc_n != 1 && !(p.N == 1)) return fail(MT_EUNSUPPORTED, "umma: C needs unit n-stride");
    // Operand A: K-major needs sa_k == 1; M-major needs sa_m == 1. Strides multiple of 16 B.
    auto mult4 = [](int64_t s) { return s % 4 == 0; };
    const bool a_batched = p.batch > 1 && p.sa_b != 0;
    const bool b_batched = p.batch > 1 && p.sb_b != 0;
    if (!aligned16(p.A) || !aligned16(p.B)) return fail(MT_EUNSUPPORTED, "umma: operand not 16-byte aligned");
    if (a_batched && !mult4(p.sa_b)) return fail(MT_EUNSUPPORTED, "umma: A batch stride");
    if (b_batched && !mult4(p.sb_b)) return fail(MT_EUNSUPPORTED, "umma: B batch stride");
    int a_mn = -1, b_mn = -1;
    if ((p.sa_k == 1 || p.K == 1) && (p.M == 1 || mult4(p.sa_m))) a_mn = 0;
    else if ((p.sa_m == 1 || p.M == 1) && (p.K == 1 || mult4(p.sa_k))) a_mn = 1;
    if ((p.sb_n == 1 || p.N == 1) && (p.K == 1 || mult4(p.sb_k))) b_mn = 1;
    else if ((p.sb_k == 1 || p.K == 1) && (p.N == 1 || mult4(p.sb_n))) b_mn = 0;
    if (a_mn < 0 || b_mn < 0) return fail(MT_EUNSUPPORTED, "umma: operand strides not TMA-expressible");

    const int64_t tiles_m1 = (p.M + 127) / 128;
    const bool small = tiles_m1 * ((p.N + 255) / 256) * p.batch < (int64_t)di.sms || p.N <= 128;
    const int bn = small ? 128 : 256;
    // CTA pairs: 256 x 256 tiles, at least one per pair of SMs.
    const int64_t tiles256 = ((p.M + 255) / 256) * ((p.N + 255) / 256) * p.batch;
    const bool pair = pair_enabled() && !small && p.M > 128 && tiles256 >= (int64_t)(di.sms / 2);

    // k elements per stage: 32 (a 128-byte swizzled row); the one-CTA TF32X3 kernel takes
    // 16 to keep 4-6 stages of hi + lo in shared memory, the pair kernel 32 with 3 stages
    // (half the stage hand-offs per MMA; measured +5% on 8192^3 and a higher clock under
    // the power cap).
    const bool x3_wide = pair && x3;
    const uint32_t bke = (x3 && !x3_wide) ? 16 : 32;
    const int kswz = (int)bke * 4;             // K-major swizzle span (bytes)
    const uint32_t chunk = 32;                 // MN-major box width (elements)
    const int64_t tiles_m = pair ? (p.M + 255) / 256 : tiles_m1;
    const uint32_t b_rows = pair ? (uint32_t)bn / 2 : (uint32_t)bn;   // B tile rows one CTA loads

    // Sizes of unit dims get a harmless 16-byte stride.
    auto st_or = [](int64_t extent, int64_t stride_elems, uint64_t fallback_bytes) -> uint64_t {
        return extent > 1 ? (uint64_t)stride_elems * 4 : fallback_bytes;
    };
    CUtensorMap ta, tb;
    bool ok;
    if (a_mn == 0) {   // dims {K, M, batch}
        uint64_t s1 = st_or(p.M, p.sa_m, round16(p.K * 4));
        uint64_t s2 = a_batched ? (uint64_t)p.sa_b * 4 : round16(s1 * p.M);
        ok = encode_3d(&ta, p.A, p.K, p.M, a_batched ? p.batch : 1, s1, s2, bke, 128, kswz);
    } else {           // dims {M, K, batch}
        uint64_t s1 = st_or(p.K, p.sa_k, round16(p.M * 4));
        uint64_t s2 = a_batched ? (uint64_t)p.sa_b * 4 : round16(s1 * p.K);
        ok = encode_3d(&ta, p.A, p.M, p.K, a_batched ? p.batch : 1, s1, s2, chunk, bke, 32);
    }
    if (!ok) return fail(MT_EUNSUPPORTED, "umma: A tensor map rejected");
    if (b_mn == 0) {   // dims {K, N, batch}
        uint64_t s1 = st_or(p.N, p.sb_n, round16(p.K * 4));
        uint64_t s2 = b_batched ? (uint64_t)p.sb_b * 4 : round16(s1 * p.N);
        ok = encode_3d(&tb, p.B, p.K, p.N, b_batched ? p.batch : 1, s1, s2, bke, b_rows, kswz);
    } else {           // dims {N, K, batch}
        uint64_t s1 = st_or(p.K, p.sb_k, round16(p.N * 4));
        uint64_t s2 = b_batched ? (uint64_t)p.sb_b * 4 : round16(s1 * p.K);
        ok = encode_3d(&tb, p.B, p.N, p.K, b_batched ? p.batch : 1, s1, s2, chunk, bke, 32);
    }
    if (!ok) return fail(MT_EUNSUPPORTED, "umma: B tensor map rejected");

    mt::umma::Params up;
    up.M = (int)p.M; up.N = (int)p.N; up.K = (int)p.K; up.batch = (int)p.batch;
    up.a_batched = a_batched; up.b_batched = b_batched;
    up.ndst = 1 + nextra;
    up.dst[0] = p.C;
    bool dst_aligned = aligned16(p.C);
    for (int d = 0; d < nextra; ++d) {
        up.dst[1 + d] = extra_dst[d];
        dst_aligned = dst_aligned && aligned16(extra_dst[d]);
    }
    for (int d = up.ndst; d < mt::umma::kMaxDst; ++d) up.dst[d] = nullptr;
    up.sc_b = p.sc_b; up.sc_m = p.sc_m;
    up.bias = p.bias; up.epi = p.epi;
    up.vec_store = dst_aligned && p.sc_m % 4 == 0 && (p.batch == 1 || p.sc_b % 4 == 0) && p.N % 4 == 0;
    up.tiles_m = (int)tiles_m;
    up.tiles_n = (int)((p.N + bn - 1) / bn);
    up.num_tiles = (long long)up.tiles_m * up.tiles_n * p.batch;
    // Split-K when the output has too few tiles to occupy the GPU (e.g. the Linear
    // backward dX = dY . W^T: 16 tiles, K = 4096): fp32 partials in a stream-ordered
    // workspace, then one pass that sums them in split order and applies the epilogue.
    // (Measured on 512^3: more CTAs beat the extra pass even when a tile's unsplit MMA
    // work is only a few microseconds -- the per-CTA start-up cost dominates there.)
    const int kblocks = (int)((p.K + bke - 1) / bke);
    int splits = 1;
    if (!pair && p.batch == 1 && nextra == 0 && up.num_tiles * 2 <= di.sms && kblocks >= 8)
        splits = (int)std::max<long long>(
            1, std::min<long long>(std::min<long long>(di.sms / up.num_tiles, kblocks / 4), 16));
    up.splits = splits;
    up.num_units = up.num_tiles * splits;
    float* ws = nullptr;
    const size_t splitk_bytes = (size_t)splits * (size_t)p.M * (size_t)p.N * sizeof(float);
    if (splits > 1) {
        const int arc = scratch_alloc(reinterpret_cast<void**>(&ws), splitk_bytes, st, "gemm split-K workspace");
        if (arc) return arc;
        up.dst[0] = ws;
        up.sc_m = p.N;
        up.split_stride = (int64_t)p.M * p.N;
        up.epi = 0;
        up.vec_store = p.N % 4 == 0;
    } else {
        up.split_stride = 0;
    }
    // TMA tensor stores from the epilogue, one map per destination over the same
    // {N, M, batch} view: the local C and, for a sharded GEMM, the peers' copies. Stores
    // straight from registers put each lane on its own row (32 partial lines per
    // instruction); on short-K problems, where the epilogue is the bound, that took 40%
    // longer than the tensor stores (config 3: 33 vs 23 us).
    mt::umma::DstMaps dm;
    memset(&dm, 0, sizeof dm);
    up.tma_multi = 0;
    if (splits == 1 && up.vec_store && tma_epilogue_enabled()) {
        const uint64_t s1 = (uint64_t)p.sc_m * 4;
        const uint64_t s2 = p.batch > 1 ? (uint64_t)p.sc_b * 4 : round16(s1 * (uint64_t)p.M);
        bool ok = true;
        for (int d = 0; d < up.ndst && ok; ++d)
            ok = encode_3d(&dm.m[d], up.dst[d], (uint64_t)p.N, (uint64_t)p.M, (uint64_t)p.batch, s1, s2, 32, 32, 128);
        up.tma_multi = ok ? 1 : 0;
    }
    const int grid = (int)std::min<long long>(up.num_units, (long long)di.sms);

    int rc;
#define MT_UMMA_DISPATCH(BN_, BKE_, X3_, ST_)                                                       \
    if (a_mn == 0 && b_mn == 0) rc = launch_umma_inst<BN_, BKE_, false, false, X3_, ST_>(ta, tb, dm, up, grid, st); \
    else if (a_mn == 0 && b_mn == 1) rc = launch_umma_inst<BN_, BKE_, false, true, X3_, ST_>(ta, tb, dm, up, grid, st); \
    else if (a_mn == 1 && b_mn == 0) rc = launch_umma_inst<BN_, BKE_, true, false, X3_, ST_>(ta, tb, dm, up, grid, st); \
    else rc = launch_umma_inst<BN_, BKE_, true, true, X3_, ST_>(ta, tb, dm, up, grid, st);
#define MT_PAIR_DISPATCH(BN_, BKE_, X3_, ST_)                                                               \
    if (a_mn == 0 && b_mn == 0) rc = launch_pair_inst<BN_, BKE_, false, false, X3_, ST_>(ta, tb, dm, up, di.sms, st); \
    else if (a_mn == 0 && b_mn == 1) rc = launch_pair_inst<BN_, BKE_, false, true, X3_, ST_>(ta, tb, dm, up, di.sms, st); \
    else if (a_mn == 1 && b_mn == 0) rc = launch_pair_inst<BN_, BKE_, true, false, X3_, ST_>(ta, tb, dm, up, di.sms, st); \
    else rc = launch_pair_inst<BN_, BKE_, true, true, X3_, ST_>(ta, tb, dm, up, di.sms, st);
    if (pair) {
        // 256 x 256 tiles only: 256 x 128 pair tiles (N = 128 per MMA) measured at half the
        // rate in both precisions (8192 x 1024 x 8192: 140 vs 260 TFLOP/s in 3xTF32).
        if (!x3) { MT_PAIR_DISPATCH(256, 32, false, 6) }
        else { MT_PAIR_DISPATCH(256, 32, true, 3) }
    } else if (!x3) {
        if (bn == 256) { MT_UMMA_DISPATCH(256, 32, false, 4) }
        else { MT_UMMA_DISPATCH(128, 32, false, 6) }
    } else {
        if (bn == 256) { MT_UMMA_DISPATCH(256, 16, true, 4) }
        else { MT_UMMA_DISPATCH(128, 16, true, 6) }
    }
#undef MT_UMMA_DISPATCH
#undef MT_PAIR_DISPATCH
    if (splits > 1) {
        if (rc == MT_OK) {
            const int blocks = (int)std::min<int64_t>((p.M * p.N + 255) / 256, 8 * di.sms);
            mt::umma::splitk_epilogue_kernel<<<blocks, 256, 0, st>>>(ws, splits, (int)p.M, (int)p.N, p.C, p.sc_m,
                                                                     p.bias, p.epi);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) rc = cuda_fail(e, "split-K epilogue");
            else g_launches.fetch_add(1);
        }
        scratch_free(ws, splitk_bytes, st);
    }
    if (rc == MT_OK) {
        char buf[112];
        snprintf(buf, sizeof buf, "umma%s_%s bn=%d a=%s b=%s%s", pair ? "_pair" : "", x3 ? "tf32x3" : "tf32", bn,
                 a_mn ? "MN" : "K", b_mn ? "MN" : "K",
                 splits > 1 ? (" splitk=" + std::to_string(splits)).c_str() : "");
        t_path = buf;
        if (pair) t_path += t_sched;
        if (up.tma_multi) t_path += " tma_store";
    }
    return rc;
}

int run_gemm(GemmProblem p, int mode, cudaStream_t st) {
    if (p.M == 0 || p.N == 0 || p.batch == 0) { t_path = "empty"; return MT_OK; }
    if ((p.epi & (MT_EPI_BIAS_ROW | MT_EPI_BIAS_COL)) && !p.bias) return fail(MT_EINVAL, "bias epilogue without bias");
    if (p.K == 0) {
        int blocks = (int)std::min<int64_t>((p.batch * p.M * p.N + 255) / 256, 4096);
        mt::simt::fill_epilogue_kernel<<<blocks, 256, 0, st>>>(p);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, "fill launch");
        g_launches.fetch_add(1);
        t_path = "fill_k0";
        return MT_OK;
    }
    mode = resolve_mode(mode);
    // Column-major output: compute C^T = B^T A^T so the kernel always writes rows.
    if (p.sc_n != 1 && p.sc_m == 1 && mode != MT_STRICT_FP32) {
        GemmProblem q = p;
        q.A = p.B; q.sa_b = p.sb_b; q.sa_m = p.sb_n; q.sa_k = p.sb_k;
        q.B = p.A; q.sb_b = p.sa_b; q.sb_k = p.sa_k; q.sb_n = p.sa_m;
        q.sc_m = p.sc_n; q.sc_n = 1;
        q.M = p.N; q.N = p.M;
        q.epi = (p.epi & MT_EPI_RELU) | ((p.epi & MT_EPI_BIAS_ROW) ? MT_EPI_BIAS_COL : 0) |
                ((p.epi & MT_EPI_BIAS_COL) ? MT_EPI_BIAS_ROW : 0);
        p = q;
    }
    if (mode != MT_STRICT_FP32) {
        std::string saved = t_err;
        int rc = launch_umma(p, mode == MT_TF32X3, st);
        if (rc == MT_OK) return MT_OK;
        if (rc != MT_EUNSUPPORTED) return rc;
        t_err = saved;   // not an error: the SIMT kernel serves this view
    }
    return launch_simt(p, st);
}

int gemm_from_views(const View& a, const View& b, const View& c, const float* bias, int epi, int mode,
                    void* stream) {
    GemmProblem p;
    p.A = a.ptr; p.sa_b = a.s[0]; p.sa_m = a.s[1]; p.sa_k = a.s[2];
    p.B = b.ptr; p.sb_b = b.s[0]; p.sb_k = b.s[1]; p.sb_n = b.s[2];
    p.C = const_cast<float*>(c.ptr); p.sc_b = c.s[0]; p.sc_m = c.s[1]; p.sc_n = c.s[2];
    p.M = a.d[1]; p.K = a.d[2]; p.N = b.d[2]; p.batch = c.d[0];
    p.bias = bias; p.epi = epi;
    if (p.batch > 1 && p.sc_b == 0) return fail(MT_EINVAL, "C must not be a broadcast view");
    return run_gemm(p, mode, static_cast<cudaStream_t>(stream));
}

// include/TensorOps.hpp:993-1005 checks: 2-D operands, A.K == B.K; plus C's shape.
int matmul_2d(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream, const char* who) {
    View a, b, c;
    int rc;
    if ((rc = to_view(A, 2, who, a)) || (rc = to_view(B, 2, who, b)) || (rc = to_view(C, 2, who, c))) return rc;
    if (a.d[2] != b.d[1]) return fail(MT_EINVAL, "%s: Dimension mismatch: A columns must match B rows.", who);
    if (c.d[1] != a.d[1] || c.d[2] != b.d[2])
        return fail(MT_EINVAL, "%s: C must be [%lld,%lld]", who, (long long)a.d[1], (long long)b.d[2]);
    return gemm_from_views(a, b, c, nullptr, MT_EPI_NONE, MT_MODE_DEFAULT, stream);
}


// ------------------------------- Conv2D -------------------------------------------
// include/TensorOps.hpp:17-20 safe_out_size.
int64_t out_size(int64_t in, int64_t pad, int64_t k, int64_t stride) {
    if (in + 2 * pad < k) return 0;
    return (in + 2 * pad - k) / stride + 1;
}

bool is_contig(const mt_tensor* t) {
    for (uint32_t i = 0; i < t->ndim; ++i)
        if (t->shape[i] == 0) return true;   // empty: nothing to address
    uint64_t expect = 1;
    for (int i = (int)t->ndim - 1; i >= 0; --i) {
        if (t->shape[i] != 1 && t->strides[i] != expect) return false;
        expect *= t->shape[i];
    }
    return true;
}

// A 4-D (N, C, H, W) view already laid out as the conv kernels' NHWC copy: channel stride
// 1, then W, H, N densely, C a multiple of 4 (no channel padding) and a 16-byte-aligned
// start -- what mt_nchw_to_nhwc writes. The stride-1 tensor-core paths read such an input
// in place instead of transforming it. Strides of size-1 dimensions are not looked at.
bool nhwc_dense(const mt_tensor* t) {
    if (!t || t->ndim != 4 || !t->data) return false;
    const uint64_t N = t->shape[0], C = t->shape[1], H = t->shape[2], W = t->shape[3];
    if (N * C * H * W == 0 || C % 4 != 0) return false;
    if (t->strides[1] != 1) return false;
    if (W > 1 && t->strides[3] != C) return false;
    if (H > 1 && t->strides[2] != W * C) return false;
    if (N > 1 && t->strides[0] != H * W * C) return false;
    return aligned16(t->data + t->offset);
}

uint64_t numel(const mt_tensor* t) {
    if (!t) return 0;
    uint64_t n = 1;
    for (uint32_t i = 0; i < t->ndim; ++i) n *= t->shape[i];
    return t->ndim ? n : 0;
}

int check4(const mt_tensor* t, const char* who, const char* name) {
    if (!t) return fail(MT_EINVAL, "%s: %s is null", who, name);
    if (t->ndim != 4) return fail(MT_EINVAL, "%s: %s must be 4-D (NCHW), got %u-D", who, name, t->ndim);
    if (numel(t) && !t->data) return fail(MT_EINVAL, "%s: %s has no data", who, name);
    return MT_OK;
}

void fill_strides(int64_t (&d)[4], const mt_tensor* t) {
    for (int i = 0; i < 4; ++i) d[i] = (int64_t)t->strides[i];
}

template <int KIND, int BN, bool X3, int STAGES>
int launch_conv_inst(const mt::conv::Params& cp, int grid, cudaStream_t st) {
    using G = mt::conv::Cfg<BN, X3, STAGES>;
    auto kern = mt::conv::conv_kernel<KIND, BN, X3, STAGES>;
    static std::atomic<uint64_t> attr_set_mask{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set_mask.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "conv: set smem attribute");
        attr_set_mask.fetch_or(bit);
    }
    kern<<<grid, G::THREADS, G::SMEM_BYTES, st>>>(cp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, "conv launch");
    g_launches.fetch_add(1);
    return MT_OK;
}

template <int KIND, bool X3>
int launch_conv_bn(const mt::conv::Params& cp, int bn, int grid, cudaStream_t st) {
    // Stages: the ring (x2 for the lo copy) stays within ~192 KB of shared memory.
    switch (bn) {
        case 32:  return launch_conv_inst<KIND, 32, X3, X3 ? 4 : 8>(cp, grid, st);
        case 64:  return launch_conv_inst<KIND, 64, X3, X3 ? 4 : 8>(cp, grid, st);
        case 128: return launch_conv_inst<KIND, 128, X3, X3 ? 3 : 6>(cp, grid, st);
        default:  return launch_conv_inst<KIND, 256, X3, X3 ? 2 : 4>(cp, grid, st);
    }
}

int pick_bn(int ncol) { return ncol <= 32 ? 32 : ncol <= 64 ? 64 : ncol <= 128 ? 128 : 256; }

struct ConvShape {
    int64_t N, C, H, W, Co, kh, kw, Ho, Wo, stride, pad;
};

// Shared shape checks (include/TensorOps.hpp:1076-1110 conv2d and the backward
// dispatchers :1112-1149): x [N,C,H,W], w [Co,C,kh,kw], y/dy [N,Co,Ho,Wo].
int conv_shape(const mt_tensor* x, const mt_tensor* w, const mt_tensor* y, uint64_t stride, uint64_t pad,
               const char* who, ConvShape& s) {
    if (stride == 0) return fail(MT_EINVAL, "%s: stride must be >= 1", who);
    s.N = (int64_t)x->shape[0]; s.C = (int64_t)x->shape[1]; s.H = (int64_t)x->shape[2]; s.W = (int64_t)x->shape[3];
    s.Co = (int64_t)w->shape[0]; s.kh = (int64_t)w->shape[2]; s.kw = (int64_t)w->shape[3];
    s.stride = (int64_t)stride; s.pad = (int64_t)pad;
    if ((int64_t)w->shape[1] != s.C)
        return fail(MT_EINVAL, "%s: weight C_in (%llu) != input C (%lld)", who, (unsigned long long)w->shape[1], (long long)s.C);
    s.Ho = out_size(s.H, s.pad, s.kh, s.stride);
    s.Wo = out_size(s.W, s.pad, s.kw, s.stride);
    if ((int64_t)y->shape[0] != s.N || (int64_t)y->shape[1] != s.Co || (int64_t)y->shape[2] != s.Ho ||
        (int64_t)y->shape[3] != s.Wo)
        return fail(MT_EINVAL, "%s: output must be [%lld,%lld,%lld,%lld]", who, (long long)s.N, (long long)s.Co,
                    (long long)s.Ho, (long long)s.Wo);
    const int64_t big = (int64_t)1 << 31;
    if (s.N * s.C * s.H * s.W >= big || s.N * s.Co * s.Ho * s.Wo >= big || s.C * s.kh * s.kw >= big)
        return fail(MT_EUNSUPPORTED, "%s: tensors beyond 2^31 elements", who);
    return MT_OK;
}

// Largest element offset a view can address; the implicit-GEMM gathers use 32-bit offsets.
bool offsets_fit_32(const mt_tensor* t) {
    uint64_t span = 0;
    for (uint32_t i = 0; i < t->ndim; ++i)
        if (t->shape[i]) span += (t->shape[i] - 1) * t->strides[i];
    return span < (uint64_t(1) << 31);
}

mt::conv::Params conv_params(const ConvShape& s) {
    mt::conv::Params cp;
    memset(&cp, 0, sizeof cp);
    cp.N = (int)s.N; cp.C = (int)s.C; cp.H = (int)s.H; cp.W = (int)s.W; cp.Co = (int)s.Co;
    cp.kh = (int)s.kh; cp.kw = (int)s.kw; cp.stride = (int)s.stride; cp.pad = (int)s.pad;
    cp.Ho = (int)s.Ho; cp.Wo = (int)s.Wo;
    cp.splits = 1;
    return cp;
}

int direct_launch(void (*kern)(const mt::conv::Params), const mt::conv::Params& cp, int64_t total, cudaStream_t st,
                  const char* name) {
    if (total == 0) return MT_OK;
    int blocks = (int)std::min<int64_t>((total + 127) / 128, 1 << 20);
    kern<<<blocks, 128, 0, st>>>(cp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, name);
    g_launches.fetch_add(1);
    return MT_OK;
}

// ---- strict fp32: implicit GEMMs on FFMA (conv_simt.cuh) ------------------------------
// kind: mt::convs::kFwd / kDgrad / kWgrad. `part` (wgrad) = N * C*kh*kw * C_out floats of
// per-image partial sums. Returns MT_EUNSUPPORTED when the grid would exceed its limits
// (the caller then takes the direct kernels).
int conv_strict(int kind, const mt::conv::Params& cp, float* part, cudaStream_t st, const char* who) {
    namespace cs = mt::convs;
    cs::Params q;
    memset(&q, 0, sizeof q);
    q.x = cp.x; q.w = cp.w; q.dy = cp.dy; q.bias = cp.bias;
    for (int i = 0; i < 4; ++i) { q.sx[i] = cp.sx[i]; q.sw[i] = cp.sw[i]; q.sdy[i] = cp.sdy[i]; }
    q.N = cp.N; q.C = cp.C; q.H = cp.H; q.W = cp.W; q.Co = cp.Co; q.kh = cp.kh; q.kw = cp.kw;
    q.Ho = cp.Ho; q.Wo = cp.Wo; q.stride = cp.stride; q.pad = cp.pad;
    const int64_t khw = (int64_t)cp.kh * cp.kw;
    int64_t K;
    int images = 1;
    if (kind == cs::kFwd) {
        q.M = (int64_t)cp.N * cp.Ho * cp.Wo; q.Ncol = cp.Co; K = cp.C * khw;
        q.out = cp.out;
        q.so[0] = (int64_t)cp.Co * cp.Ho * cp.Wo; q.so[1] = (int64_t)cp.Ho * cp.Wo; q.so[2] = cp.Wo; q.so[3] = 1;
    } else if (kind == cs::kDgrad) {
        q.M = (int64_t)cp.N * cp.H * cp.W; q.Ncol = cp.C; K = cp.Co * khw;
        q.out = cp.out;
        q.so[0] = (int64_t)cp.C * cp.H * cp.W; q.so[1] = (int64_t)cp.H * cp.W; q.so[2] = cp.W; q.so[3] = 1;
    } else {
        q.M = cp.C * khw; q.Ncol = cp.Co; K = (int64_t)cp.Ho * cp.Wo;
        q.out = part;
        images = cp.N;
    }
    if (K > INT32_MAX) return fail(MT_EUNSUPPORTED, "%s: reduction too long for the strict kernels", who);
    q.K = (int)K;
    const int bn = q.Ncol <= 64 ? 64 : 128;
    const dim3 grid((unsigned)((q.Ncol + bn - 1) / bn), (unsigned)((q.M + cs::BM - 1) / cs::BM), (unsigned)images);
    if (grid.y > 65535 || grid.z > 65535) return fail(MT_EUNSUPPORTED, "%s: strict grid too large", who);
#define MT_CONVS(KIND)                                                                            \
    if (bn == 64) cs::conv_simt_kernel<KIND, 64><<<grid, cs::THREADS, 0, st>>>(q);               \
    else cs::conv_simt_kernel<KIND, 128><<<grid, cs::THREADS, 0, st>>>(q);
    if (kind == cs::kFwd) { MT_CONVS(cs::kFwd) }
    else if (kind == cs::kDgrad) { MT_CONVS(cs::kDgrad) }
    else { MT_CONVS(cs::kWgrad) }
#undef MT_CONVS
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, who);
    g_launches.fetch_add(1);
    if (kind == cs::kWgrad) {
        const int64_t total = q.M * q.Ncol;
        const int blocks = (int)std::min<int64_t>((total + 255) / 256, 1024);
        cs::wgrad_sum_kernel<<<blocks, 256, 0, st>>>(part, images, (int)q.M, q.Ncol, cp.out);
        e = cudaGetLastError();
        if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, who);
        g_launches.fetch_add(1);
    }
    return MT_OK;
}

size_t strict_wgrad_bytes(const ConvShape& s) { return (size_t)s.N * s.C * s.kh * s.kw * s.Co * sizeof(float); }

// ---- TMA conv path ----------------------------------------------------------------
int launch_simple(cudaError_t e, const char* what) {
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, what);
    g_launches.fetch_add(1);
    return MT_OK;
}

// NCHW view -> NHWC copy with Cp = round_up(C, 4) channels.
int to_nhwc(const float* src, const int64_t (&sv)[4], float* dst, int N, int C, int H, int W, cudaStream_t st) {
    const int Cp = (C + 3) & ~3;
    const int64_t HW = (int64_t)H * W;
    if (sv[3] == 1 && sv[2] == W && HW % 4 == 0 && sv[1] % 4 == 0 && sv[0] % 4 == 0 && aligned16(src) &&
        HW <= INT32_MAX && (HW + 255) / 256 <= INT32_MAX && (Cp + 31) / 32 <= 65535) {
        dim3 grid((unsigned)((HW + 255) / 256), (unsigned)((Cp + 31) / 32), (unsigned)std::min(N, 65535));
        mt::convt::nchw_to_nhwc_flat_kernel<<<grid, 256, 0, st>>>(src, sv[0], sv[1], dst, N, C, (int)HW, Cp);
        return launch_simple(cudaGetLastError(), "nchw_to_nhwc");
    }
    if ((W + 63) / 64 > 65535 || (Cp + 63) / 64 > 65535) return fail(MT_EUNSUPPORTED, "nchw_to_nhwc: extent");
    dim3 grid((W + 63) / 64, (Cp + 63) / 64, (unsigned)std::min(N * H, 65535));
    mt::convt::nchw_to_nhwc_kernel<<<grid, 256, 0, st>>>(src, sv[0], sv[1], sv[2], sv[3], dst, N, C, H, W, Cp);
    return launch_simple(cudaGetLastError(), "nchw_to_nhwc");
}

int reorder_w(const float* w, const int64_t (&sw)[4], float* wt, int Co, int C, int kh, int kw, bool dgrad,
              cudaStream_t st, bool split = false) {
    const int rows = dgrad ? C : Co, cols = dgrad ? Co : C;
    const int64_t total = (int64_t)kh * kw * rows * ((cols + 3) & ~3);
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 1024);
    mt::convt::reorder_weights_kernel<<<blocks, 256, 0, st>>>(w, sw[0], sw[1], sw[2], sw[3], wt, Co, C, kh, kw,
                                                              dgrad ? 1 : 0, split ? 1 : 0);
    return launch_simple(cudaGetLastError(), "reorder_weights");
}

template <typename Kern>
int set_smem(Kern kern, uint32_t bytes, std::atomic<uint64_t>& mask) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(mask.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return cuda_fail(e, "conv: set smem attribute");
        mask.fetch_or(bit);
    }
    return MT_OK;
}

template <int BN, bool X3, int STAGES>
int launch_fwd_tma_inst(const CUtensorMap& ta, const CUtensorMap& tb, const mt::convt::FwdParams& fp, int grid,
                        cudaStream_t st) {
    using G = mt::convt::Cfg<BN, X3, STAGES>;
    auto kern = mt::convt::conv_fwd_tma_kernel<BN, X3, STAGES>;
    static std::atomic<uint64_t> mask{0};
    int rc = set_smem(kern, G::SMEM_BYTES, mask);
    if (rc) return rc;
    kern<<<grid, G::THREADS, G::SMEM_BYTES, st>>>(ta, tb, fp);
    return launch_simple(cudaGetLastError(), "conv fwd tma");
}

// Stages keep the ring (doubled for the lo copy) within ~192 KB of shared memory.
template <bool X3>
int launch_fwd_tma(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const mt::convt::FwdParams& fp, int grid,
                   cudaStream_t st) {
    switch (bn) {
        case 32:  return launch_fwd_tma_inst<32, X3, X3 ? 4 : 8>(ta, tb, fp, grid, st);
        case 64:  return launch_fwd_tma_inst<64, X3, X3 ? 4 : 8>(ta, tb, fp, grid, st);
        case 128: return launch_fwd_tma_inst<128, X3, X3 ? 3 : 6>(ta, tb, fp, grid, st);
        default:  return launch_fwd_tma_inst<256, X3, X3 ? 2 : 4>(ta, tb, fp, grid, st);
    }
}

// ---- weight-grad with wide stages -------------------------------------------------
template <int BN, bool X3, int STAGES, int XCS, int RS>
int launch_wgrad_wide_inst(const CUtensorMap& ta, const CUtensorMap& tb, const mt::convt::WgradParams& wp, int grid,
                           cudaStream_t st) {
    using G = mt::convw::WCfg<BN, X3, STAGES, XCS, RS>;
    auto kern = mt::convw::conv_wgrad_wide_kernel<BN, X3, STAGES, XCS, RS>;
    static std::atomic<uint64_t> mask{0};
    int rc = set_smem(kern, G::SMEM_BYTES, mask);
    if (rc) return rc;
    kern<<<grid, G::THREADS, G::SMEM_BYTES, st>>>(ta, tb, wp);
    return launch_simple(cudaGetLastError(), "conv wgrad wide");
}

// Stage shape: XCS runs of 32 pixels of RS output rows, and ring depth, rings of <= ~192 KB
// (doubled for the TF32X3 lo copies). Measured on c4 (weight-grad alone):
// - TF32 at C_out <= 64: 2 runs x 2 rows, 2 stages (16 MMAs per stage), 36.4 us, against
//   42.0 us with 1 row and 4 stages. Per-stage stamps of the issuer showed ~330 cycles of
//   wait, commit and loop per 8-MMA stage, which the deeper stage amortises.
// - TF32X3: 1 run x 1 row, 4 stages. 2 rows and 2 stages measured 104.8 against 91.9 us.
// Wider C_out tiles keep 1 row: a 2-row stage of 128 channels would need 256 KB.
struct WideShape { int xcs, rs; };
WideShape wgrad_shape(bool x3, int bn) {
    if (x3) return WideShape{1, 1};
    return bn <= 64 ? WideShape{2, 2} : WideShape{2, 1};
}
template <bool X3>
int launch_wgrad_wide(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const mt::convt::WgradParams& wp,
                      int grid, cudaStream_t st) {
    if constexpr (X3) {
        switch (bn) {
            case 32:  return launch_wgrad_wide_inst<32, true, 4, 1, 1>(ta, tb, wp, grid, st);
            case 64:  return launch_wgrad_wide_inst<64, true, 4, 1, 1>(ta, tb, wp, grid, st);
            case 128: return launch_wgrad_wide_inst<128, true, 3, 1, 1>(ta, tb, wp, grid, st);
            default:  return launch_wgrad_wide_inst<256, true, 2, 1, 1>(ta, tb, wp, grid, st);
        }
    } else {
        switch (bn) {
            case 32:  return launch_wgrad_wide_inst<32, false, 2, 2, 2>(ta, tb, wp, grid, st);
            case 64:  return launch_wgrad_wide_inst<64, false, 2, 2, 2>(ta, tb, wp, grid, st);
            case 128: return launch_wgrad_wide_inst<128, false, 3, 2, 1>(ta, tb, wp, grid, st);
            default:  return launch_wgrad_wide_inst<256, false, 2, 2, 1>(ta, tb, wp, grid, st);
        }
    }
}

// ---- pitched-halo forward (one activation box per 32-channel block for all taps) ----
constexpr uint32_t kHaloSmemMax = 227 * 1024;

template <int BN, bool X3>
int launch_halo_inst(const CUtensorMap& ta, const CUtensorMap& tb, const mt::convh::HaloParams& hp, uint32_t smem,
                     int grid, cudaStream_t st) {
    auto kern = mt::convh::conv_fwd_halo_kernel<BN, X3>;
    static std::atomic<uint64_t> mask{0};
    int rc = set_smem(kern, kHaloSmemMax, mask);
    if (rc) return rc;
    kern<<<grid, mt::convh::HaloCfg<X3>::THREADS, smem, st>>>(ta, tb, hp);
    return launch_simple(cudaGetLastError(), "conv fwd halo");
}

// The CTA-pair halo kernel: clusters of 2 on the TPCs, as many as fit at once.
template <int BN, bool X3>
int launch_halo_pair_inst(const CUtensorMap& ta, const CUtensorMap& tb, const mt::convh::HaloParams& hp,
                          uint32_t smem, int sms, cudaStream_t st) {
    auto kern = mt::convh::conv_fwd_halo_pair_kernel<BN, X3>;
    static std::atomic<uint64_t> mask{0};
    static std::atomic<int> max_clusters[64];
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(mask.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHaloSmemMax);
        if (e != cudaSuccess) return cuda_fail(e, "conv halo pair: set smem attribute");
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
        cfg.blockDim = dim3(mt::convh::HaloCfg<X3>::THREADS, 1, 1);
        cfg.dynamicSmemBytes = kHaloSmemMax;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sms / 2;
        }
        max_clusters[dev & 63].store(std::min(n, sms / 2));
        mask.fetch_or(bit);
    }
    const int clusters = (int)std::min<long long>(hp.num_tiles, (long long)max_clusters[dev & 63].load());
    kern<<<2 * clusters, mt::convh::HaloCfg<X3>::THREADS, smem, st>>>(ta, tb, hp);
    return launch_simple(cudaGetLastError(), "conv fwd halo pair");
}

// MT_CONV_PAIR=1 runs the halo forward on CTA pairs (M = 256). Off by default: on config 4
// it measured slower than one CTA per tile (TF32 33.1 vs 31.1 us, 3xTF32 81.4 vs 77.6 us,
// bitwise equal): halving the MMA instructions issued per output did not help, so the
// forward is bound by each SM's own MMA work, not by the issuing thread.
bool conv_pair_enabled() {
    static int v = [] {
        const char* e = std::getenv("MT_CONV_PAIR");
        return (e && e[0] == '1') ? 1 : 0;
    }();
    return v != 0;
}

// The halo kernel serves stride-1 forward-shaped convs whose halo ring fits in shared
// memory; MT_CONV_HALO=0 turns it off (the per-tap TMA kernel then runs).
bool halo_enabled() {
    static int v = [] {
        const char* e = std::getenv("MT_CONV_HALO");
        return (e && e[0] == '0') ? 0 : 1;
    }();
    return v != 0;
}

// Fills the tile geometry and shared-memory layout; false when the halo does not fit.
// The weight stage takes the largest G (a divisor of the tap count) for which two
// stages fit beside two halo slots.
bool plan_halo(int Ho, int Wo, int Cin, int kh, int kw, int Ncol, bool x3, int& bn, mt::convh::HaloParams& hp,
               uint32_t& smem, bool pair = false) {
    if (kh < 1 || kw < 1 || Wo < 1 || Ho < 1) return false;
    const uint64_t mult = x3 ? 2 : 1;
    bn = std::min(pick_bn(Ncol), 128);
    if (pair && bn != 64 && bn != 128) return false;
    const int taps = kh * kw;
    const uint64_t bmat = (uint64_t)(pair ? bn / 2 : bn) * 128;   // a CTA of a pair holds half the columns
    const uint32_t bars = 8u * (3 * mt::convh::kMaxASlots + 2 * mt::convh::kMaxBStages + 4) + 16u;
    const uint64_t budget = kHaloSmemMax - 1024 - bars;
    // Tile shape: TY rows of TXv output columns, pitched P = TXv + kw - 1, TY * P <= 128 MMA
    // rows, among the shapes whose two halo slots and two one-tap weight stages fit. Fewest
    // tiles first (every tile costs the same MMA work), then the smallest halo (less L2 ->
    // shared traffic, and room for a deeper halo ring). E.g. c4's 56 x 56: 8 x 14 tiles
    // (21 KB halos) rather than 2 x 56 (31.7 KB), both 896 tiles of 112 valid rows.
    int TXv = 0, P = 0, TY = 0, HR = 0;
    int64_t nr = 0, best_tiles = -1;
    for (int tx = std::min(Wo, 128 - (kw - 1)); tx >= 1; --tx) {
        const int p = tx + kw - 1;
        const int ty = std::min(Ho, (128 - tx) / p + 1);
        const int hr = ty + kh - 1;
        if (hr > 256) continue;
        const int64_t rows = std::max<int64_t>((int64_t)p * hr, (int64_t)(kh - 1) * p + (kw - 1) + 128);
        const int64_t r8 = (rows + 7) / 8 * 8;
        if (2 * (uint64_t)r8 * 128 * mult + 2 * mult * bmat > budget) continue;
        const int64_t tiles = (int64_t)((Ho + ty - 1) / ty) * ((Wo + tx - 1) / tx);
        if (best_tiles < 0 || tiles < best_tiles || (tiles == best_tiles && r8 < nr)) {
            best_tiles = tiles; TXv = tx; P = p; TY = ty; HR = hr; nr = r8;
        }
    }
    if (best_tiles < 0) return false;
    const uint64_t slot = (uint64_t)nr * 128;
    const int cblocks = (Cin + 31) / 32;
    // Halo slots: 2, or more (up to kMaxASlots) while the weights can stay resident -- a
    // deeper ring hides the TMA latency of the next channel block's halo behind more MMAs.
    int a_slots = 2, G = 0, b_stages = 0;
    uint64_t a_total = 0, bstage = 0;
    for (int want = mt::convh::kMaxASlots; want >= 2; --want) {
        const uint64_t at = want * slot * mult;
        int g0 = 0;
        for (int g = std::min(taps, 256); g >= 1; --g)
            if (taps % g == 0 && at + 2 * (uint64_t)g * mult * bmat <= budget) { g0 = g; break; }
        if (g0 == 0) continue;
        const uint64_t bs = (uint64_t)g0 * mult * bmat;
        const int nb = (int)std::min<uint64_t>(mt::convh::kMaxBStages, (budget - at) / bs);
        const int all = cblocks * (taps / g0);
        const bool resident = Ncol <= bn && all <= mt::convh::kMaxBStages && all <= nb;
        if (resident || want == 2) {
            a_slots = want; G = g0; b_stages = nb; a_total = at; bstage = bs;
            break;
        }
    }
    if (G == 0) return false;
    // Resident weights: one N tile, and every (channel block, tap group) stage fits.
    const int all_stages = cblocks * (taps / G);
    hp.b_resident = (Ncol <= bn && all_stages <= mt::convh::kMaxBStages && all_stages <= b_stages) ? 1 : 0;
    if (hp.b_resident) b_stages = all_stages;
    hp.P = P; hp.TXv = TXv; hp.TY = TY; hp.HR = HR;
    hp.G = G; hp.tgroups = taps / G;
    hp.a_slots = a_slots; hp.b_stages = b_stages;
    hp.halo_bytes = (uint32_t)P * HR * 128u;
    hp.slot_bytes = (uint32_t)slot;
    hp.b_bytes = (uint32_t)bstage;
    hp.a_off = 0;
    hp.alo_off = (uint32_t)(a_slots * slot);                  // used only by TF32X3
    hp.b_off = (uint32_t)a_total;
    hp.bar_off = hp.b_off + (uint32_t)(b_stages * bstage);
    smem = 1024u + hp.bar_off + bars;
    return smem <= kHaloSmemMax;
}

// `wt` holds the reordered weights: [taps][Ncol][Cinp] for TF32, [taps][2][Ncol][Cinp]
// (hi, lo) for TF32X3.
int run_fwd_halo(const float* act, int N, int Hin, int Win, int Cin, const float* wt, int Ncol, int kh, int kw,
                 int pad, float* out, int Ho, int Wo, const float* bias, bool x3, cudaStream_t st, int sms,
                 const mt::convh::HaloParams& plan, int bn, uint32_t smem, std::string& path, bool pair = false) {
    mt::convh::HaloParams hp = plan;
    const int Cinp = (Cin + 3) & ~3;
    hp.N = N; hp.Ho = Ho; hp.Wo = Wo; hp.Ncol = Ncol; hp.C = Cin; hp.kh = kh; hp.kw = kw; hp.pad = pad;
    hp.tiles_y = (Ho + hp.TY - 1) / hp.TY;
    hp.tiles_x = (Wo + hp.TXv - 1) / hp.TXv;
    if (pair) hp.tiles_x = (hp.tiles_x + 1) / 2;   // a pair tile: two tiles side by side
    hp.tiles_n = (Ncol + bn - 1) / bn;
    hp.cblocks = (Cin + 31) / 32;
    hp.taps = kh * kw;
    hp.num_tiles = (long long)N * hp.tiles_y * hp.tiles_x * hp.tiles_n;
    hp.out = out;
    hp.bias = bias;
    CUtensorMap ta, tb;
    const uint64_t rowb = (uint64_t)Cinp * 4;
    if (!encode_4d(&ta, act, {(uint64_t)Cin, (uint64_t)Win, (uint64_t)Hin, (uint64_t)N},
                   {rowb, rowb * Win, rowb * Win * Hin}, {32u, (uint32_t)hp.P, (uint32_t)hp.HR, 1u}, 128))
        return fail(MT_EUNSUPPORTED, "conv halo: activation tensor map rejected");
    const uint64_t taps_all = (uint64_t)(kh * kw);
    const uint32_t bbox = (uint32_t)(pair ? bn / 2 : bn);   // a pair's CTA loads half the columns
    bool ok;
    if (x3)
        ok = encode_4d(&tb, wt, {(uint64_t)Cin, (uint64_t)Ncol, 2, taps_all}, {rowb, rowb * Ncol, rowb * Ncol * 2},
                       {32u, bbox, 2u, (uint32_t)hp.G}, 128);
    else
        ok = encode_4d(&tb, wt, {(uint64_t)Cin, (uint64_t)Ncol, taps_all, 1},
                       {rowb, rowb * Ncol, rowb * Ncol * taps_all}, {32u, bbox, (uint32_t)hp.G, 1u}, 128);
    if (!ok) return fail(MT_EUNSUPPORTED, "conv halo: weight tensor map rejected");
    const int grid = (int)std::min<long long>(hp.num_tiles, sms);
    int rc;
    if (pair) {
        rc = bn == 64 ? (x3 ? launch_halo_pair_inst<64, true>(ta, tb, hp, smem, sms, st)
                            : launch_halo_pair_inst<64, false>(ta, tb, hp, smem, sms, st))
                      : (x3 ? launch_halo_pair_inst<128, true>(ta, tb, hp, smem, sms, st)
                            : launch_halo_pair_inst<128, false>(ta, tb, hp, smem, sms, st));
    } else
    switch (bn) {
        case 32:  rc = x3 ? launch_halo_inst<32, true>(ta, tb, hp, smem, grid, st)
                          : launch_halo_inst<32, false>(ta, tb, hp, smem, grid, st); break;
        case 64:  rc = x3 ? launch_halo_inst<64, true>(ta, tb, hp, smem, grid, st)
                          : launch_halo_inst<64, false>(ta, tb, hp, smem, grid, st); break;
        default:  rc = x3 ? launch_halo_inst<128, true>(ta, tb, hp, smem, grid, st)
                          : launch_halo_inst<128, false>(ta, tb, hp, smem, grid, st); break;
    }
    path = std::string("tma_halo bn=") + std::to_string(bn) + " tile=" + std::to_string(hp.TY) + "x" +
           std::to_string(hp.TXv) + " pitch=" + std::to_string(hp.P) + " taps/stage=" + std::to_string(hp.G) +
           " bstages=" + std::to_string(hp.b_stages) + (hp.b_resident ? " resident" : "") + (pair ? " pair" : "");
    return rc;
}

// Forward-shaped TMA conv: `act` is an NHWC activation [N, Hin, Win, Cin_p] (Cin real
// channels), `wt` the reordered weights [taps][Ncol][Cin_p], output `out` NCHW [N, Ncol, Ho, Wo].
// `w` / `sw`: the weight view [Co, C, kh, kw]; `wt`: scratch for the reordered weights
// (2 * taps * Ncol * Cinp floats); `dgrad` selects the flipped, transposed input-grad form.
int run_fwd_tma(const float* act, int N, int Hin, int Win, int Cin, const float* w, const int64_t (&sw)[4],
                bool dgrad, float* wt, int Ncol, int kh, int kw, int pad, float* out, int Ho, int Wo,
                const float* bias, bool x3, cudaStream_t st, int sms, std::string& path) {
    const int Co = dgrad ? Cin : Ncol, Ci = dgrad ? Ncol : Cin;   // the weight view's own dims
    if (halo_enabled()) {
        mt::convh::HaloParams plan;
        memset(&plan, 0, sizeof plan);
        int bn = 0;
        uint32_t smem = 0;
        // CTA pairs when the pair tiles fill at least one round of the GPU's TPCs.
        bool pair = false;
        if (conv_pair_enabled() && plan_halo(Ho, Wo, Cin, kh, kw, Ncol, x3, bn, plan, smem, true)) {
            const long long ptiles = (long long)N * ((Ho + plan.TY - 1) / plan.TY) *
                                     (((Wo + plan.TXv - 1) / plan.TXv + 1) / 2) * ((Ncol + bn - 1) / bn);
            pair = ptiles >= sms / 2;
        }
        if (!pair) memset(&plan, 0, sizeof plan);
        if (pair || plan_halo(Ho, Wo, Cin, kh, kw, Ncol, x3, bn, plan, smem)) {
            int rc = reorder_w(w, sw, wt, Co, Ci, kh, kw, dgrad, st, x3);
            if (rc) return rc;
            return run_fwd_halo(act, N, Hin, Win, Cin, wt, Ncol, kh, kw, pad, out, Ho, Wo, bias, x3, st, sms, plan,
                                bn, smem, path, pair);
        }
    }
    int rc = reorder_w(w, sw, wt, Co, Ci, kh, kw, dgrad, st, false);
    if (rc) return rc;
    const int Cinp = (Cin + 3) & ~3;
    mt::convt::FwdParams fp;
    memset(&fp, 0, sizeof fp);
    fp.N = N; fp.Ho = Ho; fp.Wo = Wo; fp.Ncol = Ncol; fp.C = Cin; fp.kh = kh; fp.kw = kw; fp.pad = pad;
    fp.TX = std::min(Wo, 128);
    fp.TY = std::max(1, std::min(128 / fp.TX, Ho));
    fp.tiles_y = (Ho + fp.TY - 1) / fp.TY;
    fp.tiles_x = (Wo + fp.TX - 1) / fp.TX;
    const int bn = pick_bn(Ncol);
    fp.tiles_n = (Ncol + bn - 1) / bn;
    fp.cblocks = (Cin + 31) / 32;
    fp.kblocks = kh * kw * fp.cblocks;
    fp.num_tiles = (long long)N * fp.tiles_y * fp.tiles_x * fp.tiles_n;
    fp.a_box_bytes = 32u * fp.TX * fp.TY * 4u;
    fp.out = out;
    fp.bias = bias;
    CUtensorMap ta, tb;
    const uint64_t rowb = (uint64_t)Cinp * 4;
    if (!encode_4d(&ta, act, {(uint64_t)Cin, (uint64_t)Win, (uint64_t)Hin, (uint64_t)N},
                   {rowb, rowb * Win, rowb * Win * Hin}, {32u, (uint32_t)fp.TX, (uint32_t)fp.TY, 1u}, 128))
        return fail(MT_EUNSUPPORTED, "conv tma: activation tensor map rejected");
    if (!encode_3d(&tb, wt, (uint64_t)Cin, (uint64_t)Ncol, (uint64_t)(kh * kw), rowb, rowb * Ncol, 32, bn, 128))
        return fail(MT_EUNSUPPORTED, "conv tma: weight tensor map rejected");
    const int grid = (int)std::min<long long>(fp.num_tiles, sms);
    rc = x3 ? launch_fwd_tma<true>(bn, ta, tb, fp, grid, st) : launch_fwd_tma<false>(bn, ta, tb, fp, grid, st);
    path = std::string("tma bn=") + std::to_string(bn) + " tile=" + std::to_string(fp.TY) + "x" +
           std::to_string(fp.TX);
    return rc;
}

// Floats of the NHWC copy at the head of the forward's scratch (0 when the input is read in
// place), rounded so that the reordered weights after it start 256-byte aligned.
int64_t fwd_xt_floats(int64_t N, int64_t H, int64_t W, int64_t C, bool in_place) {
    return in_place ? 0 : ((N * H * W * ((C + 3) & ~3) + 63) & ~int64_t(63));
}
size_t fwd_tma_scratch(int64_t N, int64_t H, int64_t W, int64_t C, int64_t Co, int64_t taps, bool in_place) {
    const int64_t Cp = (C + 3) & ~3;
    return (size_t)(fwd_xt_floats(N, H, W, C, in_place) + 2 * taps * Co * Cp) * sizeof(float) + 256;   // weights: hi + lo
}

int conv_fwd(const mt_tensor* x, const mt_tensor* w, const mt_tensor* bias, const mt_tensor* y, uint64_t stride,
             uint64_t pad, int mode, cudaStream_t st, const char* who) {
    int rc;
    if ((rc = check4(x, who, "input")) || (rc = check4(w, who, "weight")) || (rc = check4(y, who, "output"))) return rc;
    ConvShape s;
    if ((rc = conv_shape(x, w, y, stride, pad, who, s))) return rc;
    if (!is_contig(y)) return fail(MT_EINVAL, "%s: output must be contiguous", who);
    const float* bp = nullptr;
    if (bias && numel(bias)) {
        if ((int64_t)numel(bias) != s.Co) return fail(MT_EINVAL, "%s: bias must hold C_out elements", who);
        if (!is_contig(bias)) return fail(MT_EINVAL, "%s: bias must be contiguous", who);
        bp = bias->data + bias->offset;
    }
    mt::conv::Params cp = conv_params(s);
    cp.x = x->data + x->offset; fill_strides(cp.sx, x);
    cp.w = w->data + w->offset; fill_strides(cp.sw, w);
    cp.out = y->data + y->offset;
    cp.bias = bp;
    const int64_t total = s.N * s.Co * s.Ho * s.Wo;
    if (total == 0) { t_path = "empty"; return MT_OK; }
    mode = resolve_mode(mode);
    DevInfo di = dev_info();
    if (mode == MT_STRICT_FP32 || di.cc != 100) {
        if (mode != MT_STRICT_FP32) return fail(MT_EUNSUPPORTED, "%s: tensor-core conv needs sm_100a", who);
        if (conv_strict(mt::convs::kFwd, cp, nullptr, st, who) == MT_OK) {
            t_path = "conv_simt_fwd_fp32";
            return MT_OK;
        }
        t_path = "conv_direct_fwd_fp32";
        return direct_launch(mt::conv::direct_fwd_kernel, cp, total, st, who);
    }
    const bool x3 = mode == MT_TF32X3;
    if (s.stride == 1) {
        // TMA path: x -> NHWC (unless x already is) and W -> [tap][co][ci] in a
        // stream-ordered scratch buffer.
        const bool in_place = nhwc_dense(x);
        const size_t bytes = fwd_tma_scratch(s.N, s.H, s.W, s.C, s.Co, s.kh * s.kw, in_place);
        float* scratch = nullptr;
        if ((rc = scratch_alloc(reinterpret_cast<void**>(&scratch), bytes, st, "conv fwd scratch"))) return rc;
        float* xt = in_place ? const_cast<float*>(cp.x) : scratch;
        float* wt = scratch + fwd_xt_floats(s.N, s.H, s.W, s.C, in_place);
        std::string path;
        if (!in_place) rc = to_nhwc(cp.x, cp.sx, xt, (int)s.N, (int)s.C, (int)s.H, (int)s.W, st);
        if (!rc) rc = run_fwd_tma(xt, (int)s.N, (int)s.H, (int)s.W, (int)s.C, cp.w, cp.sw, false, wt, (int)s.Co,
                                  (int)s.kh, (int)s.kw,
                                  (int)s.pad, cp.out, (int)s.Ho, (int)s.Wo, bp, x3, st, di.sms, path);
        scratch_free(scratch, bytes, st);
        if (rc == MT_OK)
            t_path = std::string("conv_umma_fwd_") + (x3 ? "tf32x3 " : "tf32 ") + path + (in_place ? " nhwc_in" : "");
        return rc;
    }
    if (!offsets_fit_32(x) || !offsets_fit_32(w))
        return fail(MT_EUNSUPPORTED, "%s: a view spans 2^31 elements or more", who);
    cp.M = (int)(s.N * s.Ho * s.Wo); cp.Ncol = (int)s.Co; cp.K = (int)(s.C * s.kh * s.kw);
    cp.tiles_m = (cp.M + 127) / 128;
    const int bn = pick_bn(cp.Ncol);
    cp.tiles_n = (cp.Ncol + bn - 1) / bn;
    cp.kb_total = (cp.K + 31) / 32;
    cp.num_units = (long long)cp.tiles_m * cp.tiles_n;
    if (cp.K == 0) return fail(MT_EUNSUPPORTED, "%s: empty reduction", who);
    const int grid = (int)std::min<long long>(cp.num_units, di.sms);
    rc = x3 ? launch_conv_bn<mt::conv::kFwd, true>(cp, bn, grid, st) : launch_conv_bn<mt::conv::kFwd, false>(cp, bn, grid, st);
    if (rc == MT_OK) t_path = std::string("conv_umma_fwd_") + (x3 ? "tf32x3" : "tf32") + " gather bn=" + std::to_string(bn);
    return rc;
}

int conv_dgrad(const mt_tensor* dy, const mt_tensor* w, const mt_tensor* dx, uint64_t stride, uint64_t pad, int mode,
               cudaStream_t st, const char* who) {
    int rc;
    if ((rc = check4(dy, who, "grad_output")) || (rc = check4(w, who, "weight")) || (rc = check4(dx, who, "grad_input")))
        return rc;
    ConvShape s;
    if ((rc = conv_shape(dx, w, dy, stride, pad, who, s))) return rc;
    if (!is_contig(dx)) return fail(MT_EINVAL, "%s: grad_input must be contiguous", who);
    mt::conv::Params cp = conv_params(s);
    cp.dy = dy->data + dy->offset; fill_strides(cp.sdy, dy);
    cp.w = w->data + w->offset; fill_strides(cp.sw, w);
    cp.out = dx->data + dx->offset;
    const int64_t total = s.N * s.C * s.H * s.W;
    if (total == 0) { t_path = "empty"; return MT_OK; }
    mode = resolve_mode(mode);
    DevInfo di = dev_info();
    if (mode == MT_STRICT_FP32 || di.cc != 100) {
        if (mode != MT_STRICT_FP32) return fail(MT_EUNSUPPORTED, "%s: tensor-core conv needs sm_100a", who);
        if (conv_strict(mt::convs::kDgrad, cp, nullptr, st, who) == MT_OK) {
            t_path = "conv_simt_dgrad_fp32";
            return MT_OK;
        }
        t_path = "conv_direct_dgrad_fp32";
        return direct_launch(mt::conv::direct_dgrad_kernel, cp, total, st, who);
    }
    const bool x3 = mode == MT_TF32X3;
    if (s.stride == 1 && s.kh == s.kw && s.Ho > 0 && s.Wo > 0 && s.kh - 1 - s.pad >= 0) {
        // Stride 1: dx = forward conv of NHWC dy with W flipped and transposed, padding
        // kh-1-pad (the dy positions an input pixel receives from). The forward kernels take
        // one padding for both dimensions, as the reference's conv does, so this mapping
        // needs a square filter: kh != kw would need kw-1-pad across. Non-square filters
        // take the gather kernel below, which indexes dy per dimension.
        const bool in_place = nhwc_dense(dy);
        const size_t bytes = fwd_tma_scratch(s.N, s.Ho, s.Wo, s.Co, s.C, s.kh * s.kw, in_place);
        float* scratch = nullptr;
        if ((rc = scratch_alloc(reinterpret_cast<void**>(&scratch), bytes, st, "conv dgrad scratch"))) return rc;
        float* dyt = in_place ? const_cast<float*>(cp.dy) : scratch;
        float* wt = scratch + fwd_xt_floats(s.N, s.Ho, s.Wo, s.Co, in_place);
        std::string path;
        if (!in_place) rc = to_nhwc(cp.dy, cp.sdy, dyt, (int)s.N, (int)s.Co, (int)s.Ho, (int)s.Wo, st);
        if (!rc) rc = run_fwd_tma(dyt, (int)s.N, (int)s.Ho, (int)s.Wo, (int)s.Co, cp.w, cp.sw, true, wt, (int)s.C,
                                  (int)s.kh, (int)s.kw,
                                  (int)(s.kh - 1 - s.pad), cp.out, (int)s.H, (int)s.W, nullptr, x3, st, di.sms, path);
        scratch_free(scratch, bytes, st);
        if (rc == MT_OK)
            t_path = std::string("conv_umma_dgrad_") + (x3 ? "tf32x3 " : "tf32 ") + path + (in_place ? " nhwc_in" : "");
        return rc;
    }
    if (!offsets_fit_32(dy) || !offsets_fit_32(w))
        return fail(MT_EUNSUPPORTED, "%s: a view spans 2^31 elements or more", who);
    cp.M = (int)total / (int)s.C; cp.Ncol = (int)s.C; cp.K = (int)(s.Co * s.kh * s.kw);
    cp.tiles_m = (cp.M + 127) / 128;
    const int bn = pick_bn(cp.Ncol);
    cp.tiles_n = (cp.Ncol + bn - 1) / bn;
    cp.kb_total = (cp.K + 31) / 32;
    cp.num_units = (long long)cp.tiles_m * cp.tiles_n;
    if (cp.K == 0) {   // no output pixels: the gradient is zero
        cudaError_t e = cudaMemsetAsync(cp.out, 0, total * sizeof(float), st);
        return e == cudaSuccess ? MT_OK : cuda_fail(e, who);
    }
    const int grid = (int)std::min<long long>(cp.num_units, di.sms);
    rc = x3 ? launch_conv_bn<mt::conv::kDgrad, true>(cp, bn, grid, st) : launch_conv_bn<mt::conv::kDgrad, false>(cp, bn, grid, st);
    if (rc == MT_OK) t_path = std::string("conv_umma_dgrad_") + (x3 ? "tf32x3" : "tf32") + " bn=" + std::to_string(bn);
    return rc;
}

// Split-K plan of the weight gradient: one wave of (m tile, split) units.
struct WgradPlan {
    int tiles_m, tiles_n, kb_per_img, kb_total, splits;
    size_t ws_bytes;
};

WgradPlan wgrad_plan(const ConvShape& s, int sms) {
    WgradPlan w;
    const int M = (int)(s.C * s.kh * s.kw);
    const int bn = pick_bn((int)s.Co);
    w.tiles_m = (M + 127) / 128;
    w.tiles_n = ((int)s.Co + bn - 1) / bn;
    w.kb_per_img = (int)((s.Ho * s.Wo + 31) / 32);
    w.kb_total = (int)s.N * w.kb_per_img;
    const int tiles = w.tiles_m * w.tiles_n;
    int splits = tiles >= sms ? 1 : sms / tiles;
    splits = std::max(1, std::min(splits, w.kb_total));
    w.splits = splits;
    w.ws_bytes = splits > 1 ? (size_t)splits * (size_t)s.Co * (size_t)M * sizeof(float) : 0;
    return w;
}

// Weight-grad on the TMA path: x -> NHWC (xt), partials [splits][taps*C][Cop].
struct WgradTmaPlan {
    bool ok, x_in_place;
    int bn, xcs, rs, tiles_m, tiles_n, xblocks, kb_per_img, kb_total, splits, M, ws_ld;
    size_t xt_floats, part_floats, bytes;
};

WgradTmaPlan wgrad_tma_plan(const ConvShape& s, const mt_tensor* dy, const mt_tensor* x, int sms, bool x3) {
    WgradTmaPlan w;
    memset(&w, 0, sizeof w);
    const bool dy_ok = dy->strides[3] == 1 && dy->strides[2] % 4 == 0 && dy->strides[1] % 4 == 0 &&
                       dy->strides[0] % 4 == 0 && (((uintptr_t)(dy->data + dy->offset)) & 15) == 0;
    w.ok = s.stride == 1 && s.C % 32 == 0 && dy_ok && s.N * s.Ho * s.Wo > 0;
    if (!w.ok) return w;
    w.M = (int)(s.kh * s.kw * s.C);
    w.bn = pick_bn((int)s.Co);
    w.tiles_m = (w.M + 127) / 128;
    w.tiles_n = ((int)s.Co + w.bn - 1) / w.bn;
    w.ws_ld = w.tiles_n * w.bn;
    const WideShape ws = wgrad_shape(x3, w.bn);
    w.xcs = ws.xcs;
    w.rs = ws.rs;
    w.xblocks = (int)((s.Wo + 32 * w.xcs - 1) / (32 * w.xcs));   // runs of 32 * xcs pixels per row
    w.kb_per_img = (int)((s.Ho + w.rs - 1) / w.rs) * w.xblocks;
    w.kb_total = (int)s.N * w.kb_per_img;
    const int tiles = w.tiles_m * w.tiles_n;
    w.splits = std::max(1, std::min(tiles >= sms ? 1 : sms / tiles, w.kb_total));
    w.x_in_place = nhwc_dense(x);   // read x where it is, no NHWC copy
    w.xt_floats = w.x_in_place ? 0 : (size_t)(s.N * s.H * s.W * ((s.C + 3) & ~3));
    w.xt_floats = (w.xt_floats + 63) & ~size_t(63);
    w.part_floats = (size_t)w.splits * w.M * w.ws_ld;
    w.bytes = (w.xt_floats + w.part_floats) * sizeof(float);
    return w;
}

int conv_wgrad_tma(const ConvShape& s, const WgradTmaPlan& w, const mt::conv::Params& cp, float* dwp, float* scratch,
                   bool x3, cudaStream_t st, int sms, const char* who) {
    float* xt = w.x_in_place ? const_cast<float*>(cp.x) : scratch;
    float* part = scratch + w.xt_floats;
    int rc = w.x_in_place ? MT_OK : to_nhwc(cp.x, cp.sx, xt, (int)s.N, (int)s.C, (int)s.H, (int)s.W, st);
    if (rc) return rc;
    mt::convt::WgradParams wp;
    memset(&wp, 0, sizeof wp);
    wp.N = (int)s.N; wp.Ho = (int)s.Ho; wp.Wo = (int)s.Wo; wp.C = (int)s.C; wp.Co = (int)s.Co;
    wp.kh = (int)s.kh; wp.kw = (int)s.kw; wp.pad = (int)s.pad;
    wp.M = w.M; wp.tiles_m = w.tiles_m; wp.tiles_n = w.tiles_n; wp.xblocks = w.xblocks;
    wp.kb_per_img = w.kb_per_img; wp.kb_total = w.kb_total; wp.splits = w.splits;
    wp.num_units = (long long)w.tiles_m * w.tiles_n * w.splits;
    wp.ws = part;
    wp.ws_ld = w.ws_ld;
    CUtensorMap ta, tb;
    const uint64_t Cp = (uint64_t)((s.C + 3) & ~3), rowb = Cp * 4;
    // A: NHWC x as M-major 32-channel chunks x 32 * xcs pixels (K) of one row.
    if (!encode_4d(&ta, xt, {(uint64_t)s.C, (uint64_t)s.W, (uint64_t)s.H, (uint64_t)s.N},
                   {rowb, rowb * s.W, rowb * s.W * s.H}, {32u, 32u * (uint32_t)w.xcs, (uint32_t)w.rs, 1u}, 32))
        return fail(MT_EUNSUPPORTED, "%s: activation tensor map rejected", who);
    // B: dy straight from NCHW with the map's dimensions ordered (W, C_out, H, N): a box
    // {32 pixels, BN channels, rs rows} lands as rs blocks of BN 128-byte rows (K-major).
    if (!encode_4d(&tb, cp.dy, {(uint64_t)s.Wo, (uint64_t)s.Co, (uint64_t)s.Ho, (uint64_t)s.N},
                   {(uint64_t)cp.sdy[1] * 4, (uint64_t)cp.sdy[2] * 4, (uint64_t)cp.sdy[0] * 4},
                   {32u, (uint32_t)w.bn, (uint32_t)w.rs, 1u}, 128))
        return fail(MT_EUNSUPPORTED, "%s: grad_output tensor map rejected", who);
    const int grid = (int)std::min<long long>(wp.num_units, sms);
    rc = x3 ? launch_wgrad_wide<true>(w.bn, ta, tb, wp, grid, st) : launch_wgrad_wide<false>(w.bn, ta, tb, wp, grid, st);
    if (rc) return rc;
    const int64_t total = s.Co * s.C * s.kh * s.kw;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4 * sms);
    mt::convt::wgrad_reduce_kernel<<<blocks, 256, 0, st>>>(part, w.splits, w.M, w.ws_ld, dwp, (int)s.Co, (int)s.C,
                                                           (int)(s.kh * s.kw));
    return launch_simple(cudaGetLastError(), "wgrad reduce");
}

int conv_wgrad(const mt_tensor* dy, const mt_tensor* x, const mt_tensor* dw, uint64_t stride, uint64_t pad, int mode,
               void* workspace, size_t ws_bytes, cudaStream_t st, const char* who, bool allow_tma = true) {
    int rc;
    if ((rc = check4(dy, who, "grad_output")) || (rc = check4(x, who, "input")) || (rc = check4(dw, who, "grad_weight")))
        return rc;
    ConvShape s;
    if ((rc = conv_shape(x, dw, dy, stride, pad, who, s))) return rc;
    if (!is_contig(dw)) return fail(MT_EINVAL, "%s: grad_weight must be contiguous", who);
    mt::conv::Params cp = conv_params(s);
    cp.x = x->data + x->offset; fill_strides(cp.sx, x);
    cp.dy = dy->data + dy->offset; fill_strides(cp.sdy, dy);
    float* dwp = dw->data + dw->offset;
    const int64_t total = s.Co * s.C * s.kh * s.kw;
    if (total == 0) { t_path = "empty"; return MT_OK; }
    mode = resolve_mode(mode);
    DevInfo di = dev_info();
    if (s.N * s.Ho * s.Wo == 0) {   // empty reduction: the gradient is zero
        cudaError_t e = cudaMemsetAsync(dwp, 0, total * sizeof(float), st);
        t_path = "zero";
        return e == cudaSuccess ? MT_OK : cuda_fail(e, who);
    }
    if (mode == MT_STRICT_FP32 || di.cc != 100) {
        if (mode != MT_STRICT_FP32) return fail(MT_EUNSUPPORTED, "%s: tensor-core conv needs sm_100a", who);
        cp.out = dwp;
        // Per-image partials: in the caller's workspace when it is large enough, else in
        // scratch when the caller gave none; a workspace too small for them (e.g. the
        // fixed array of the no-allocation entry point) takes the direct kernel, which
        // needs none.
        const size_t need = strict_wgrad_bytes(s);
        float* part = nullptr;
        bool owned = false;
        if (workspace && ws_bytes >= need) {
            part = static_cast<float*>(workspace);
        } else if (!workspace) {
            if ((rc = scratch_alloc(reinterpret_cast<void**>(&part), need, st, "conv strict wgrad partials"))) return rc;
            owned = true;
        }
        if (part) {
            rc = conv_strict(mt::convs::kWgrad, cp, part, st, who);
            if (owned) scratch_free(part, need, st);
            if (rc == MT_OK) {
                t_path = "conv_simt_wgrad_fp32";
                return MT_OK;
            }
        }
        t_path = "conv_direct_wgrad_fp32";
        return direct_launch(mt::conv::direct_wgrad_kernel, cp, total, st, who);
    }
    if (!offsets_fit_32(dy) || !offsets_fit_32(x))
        return fail(MT_EUNSUPPORTED, "%s: a view spans 2^31 elements or more", who);
    const bool x3w = mode == MT_TF32X3;
    const WgradTmaPlan tp = allow_tma ? wgrad_tma_plan(s, dy, x, di.sms, x3w) : WgradTmaPlan{};
    if (tp.ok) {
        float* scratch = static_cast<float*>(workspace);
        bool owned = false;
        if (workspace) {
            if (ws_bytes < tp.bytes)
                return fail(MT_EINVAL, "%s: workspace of %zu bytes < %zu needed", who, ws_bytes, tp.bytes);
        } else {
            if ((rc = scratch_alloc(reinterpret_cast<void**>(&scratch), tp.bytes, st, "conv wgrad scratch"))) return rc;
            owned = true;
        }
        rc = conv_wgrad_tma(s, tp, cp, dwp, scratch, x3w, st, di.sms, who);
        if (owned) scratch_free(scratch, tp.bytes, st);
        if (rc == MT_OK)
            t_path = std::string("conv_umma_wgrad_") + (x3w ? "tf32x3" : "tf32") + " tma bn=" + std::to_string(tp.bn) +
                     " splits=" + std::to_string(tp.splits) + (tp.x_in_place ? " nhwc_in" : "");
        return rc;
    }
    WgradPlan wp = wgrad_plan(s, di.sms);
    cp.M = (int)(s.C * s.kh * s.kw); cp.Ncol = (int)s.Co; cp.K = (int)(s.N * s.Ho * s.Wo);
    cp.tiles_m = wp.tiles_m; cp.tiles_n = wp.tiles_n;
    cp.kb_per_img = wp.kb_per_img; cp.kb_total = wp.kb_total; cp.splits = wp.splits;
    cp.num_units = (long long)wp.tiles_m * wp.tiles_n * wp.splits;
    bool owned = false;
    float* part = dwp;
    if (wp.splits > 1) {
        if (workspace) {
            if (ws_bytes < wp.ws_bytes)
                return fail(MT_EINVAL, "%s: workspace of %zu bytes < %zu needed", who, ws_bytes, wp.ws_bytes);
            part = static_cast<float*>(workspace);
        } else {
            if ((rc = scratch_alloc(reinterpret_cast<void**>(&part), wp.ws_bytes, st, "conv wgrad workspace")))
                return rc;
            owned = true;
        }
    }
    cp.out = part;
    const int grid = (int)std::min<long long>(cp.num_units, di.sms);
    const bool x3 = x3w;
    const int bn = pick_bn(cp.Ncol);
    rc = x3 ? launch_conv_bn<mt::conv::kWgrad, true>(cp, bn, grid, st) : launch_conv_bn<mt::conv::kWgrad, false>(cp, bn, grid, st);
    if (rc == MT_OK && wp.splits > 1) {
        const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4 * di.sms);
        mt::conv::splitk_reduce_kernel<<<blocks, 256, 0, st>>>(part, dwp, wp.splits, total);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) rc = cuda_fail(e, "splitk reduce");
        else g_launches.fetch_add(1);
    }
    if (owned) scratch_free(part, wp.ws_bytes, st);
    if (rc == MT_OK)
        t_path = std::string("conv_umma_wgrad_") + (x3 ? "tf32x3" : "tf32") + " gather bn=" + std::to_string(bn) +
                 " splits=" + std::to_string(wp.splits);
    return rc;
}

int conv_bgrad(const mt_tensor* dy, const mt_tensor* db, cudaStream_t st, const char* who) {
    int rc;
    if ((rc = check4(dy, who, "grad_output"))) return rc;
    if (!db || numel(db) != dy->shape[1]) return fail(MT_EINVAL, "%s: grad_bias must hold C_out elements", who);
    if (!is_contig(db) || !db->data) return fail(MT_EINVAL, "%s: grad_bias must be contiguous", who);
    const int N = (int)dy->shape[0], Co = (int)dy->shape[1];
    const int64_t HW = (int64_t)dy->shape[2] * (int64_t)dy->shape[3];
    if (Co == 0) return MT_OK;
    // Spatial dims must be flat (stride W = 1, stride H = W) for the per-channel sweep.
    if (HW > 1 && !(dy->strides[3] == 1 && dy->strides[2] == dy->shape[3]))
        return fail(MT_EUNSUPPORTED, "%s: grad_output needs contiguous spatial dims", who);
    mt::conv::bias_grad_kernel<<<Co, 256, 0, st>>>(dy->data + dy->offset, db->data + db->offset, N, Co, (int)HW,
                                                   (int64_t)dy->strides[0], (int64_t)dy->strides[1]);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, "bias grad launch");
    g_launches.fetch_add(1);
    t_path = "conv_bias_grad";
    return MT_OK;
}


// ------------------------------- multi-GPU ----------------------------------------
namespace peer {
struct Flags {
    int* f[mt::umma::kMaxDst];   // f[d] = rank d's flag array (world ints), peer-mapped
};

// Rank `rank` raises its flag in every rank's array, then waits (bounded) until every
// rank has raised its flag in the local array. Stream order puts this after the GEMM
// kernel whose epilogue wrote into the peers' C buffers; the system-scope fence and
// release/acquire make those writes visible before anyone reads C.
__global__ void barrier_kernel(Flags fl, int rank, int world, int epoch, unsigned long long timeout_ns) {
    const int d = threadIdx.x;
    if (d < world) {
        __threadfence_system();
        asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(fl.f[d] + rank), "r"(epoch) : "memory");
    }
    __syncwarp();
    if (d < world) {
        const int* mine = fl.f[rank] + d;
        const unsigned long long t0 = mt::globaltimer_ns();
        for (;;) {
            int v;
            asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if (v == epoch) break;
            if (mt::globaltimer_ns() - t0 > timeout_ns) {
                atomicCAS(&mt::g_dev_status, 0, mt::kDevTimeoutPeer);
                break;
            }
        }
    }
}
}  // namespace peer

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn addr_range_fn() {
    static GetAddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetAddressRangeFn>(p);
    });
    return fn;
}

}  // namespace

extern "C" {

MT_API int mt_matmul_gpu(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream) {
    return matmul_2d(A, B, C, stream, "matmul_gpu");
}
MT_API int mt_matmul_gpu_strided(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream) {
    return matmul_2d(A, B, C, stream, "matmul_gpu_strided");
}
MT_API int mt_matmul_gpu_v2(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream) {
    return matmul_2d(A, B, C, stream, "matmul_gpu_v2");
}
MT_API int mt_matmul_gpu_bk16(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream) {
    return matmul_2d(A, B, C, stream, "matmul_gpu_bk16");
}

// include/TensorOps.hpp:937-943 checks: 3-D, equal batch, A.K == B.K.
MT_API int mt_bmm_gpu(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream) {
    View a, b, c;
    int rc;
    if ((rc = to_view(A, 3, "bmm", a)) || (rc = to_view(B, 3, "bmm", b)) || (rc = to_view(C, 3, "bmm", c))) return rc;
    if (a.d[0] != b.d[0]) return fail(MT_EINVAL, "bmm: batch dimension mismatch.");
    if (a.d[2] != b.d[1]) return fail(MT_EINVAL, "bmm: inner dimension mismatch (A.K != B.K).");
    if (c.d[0] != a.d[0] || c.d[1] != a.d[1] || c.d[2] != b.d[2]) return fail(MT_EINVAL, "bmm: C shape mismatch");
    if (a.d[0] == 1) { a.s[0] = 0; b.s[0] = 0; c.s[0] = 0; }
    return gemm_from_views(a, b, c, nullptr, MT_EPI_NONE, MT_MODE_DEFAULT, stream);
}

MT_API int mt_linear_fwd_gpu(const mt_tensor* X, const mt_tensor* W, const mt_tensor* bias, const mt_tensor* Y,
                             int relu, void* stream) {
    View x, w, y;
    int rc;
    if ((rc = to_view(X, 2, "linear", x)) || (rc = to_view(W, 2, "linear", w)) || (rc = to_view(Y, 2, "linear", y)))
        return rc;
    if (x.d[2] != w.d[1]) return fail(MT_EINVAL, "linear: x features (%lld) != weight in (%lld)", (long long)x.d[2], (long long)w.d[1]);
    if (y.d[1] != x.d[1] || y.d[2] != w.d[2]) return fail(MT_EINVAL, "linear: Y shape mismatch");
    const float* bp = nullptr;
    if (bias) {
        uint64_t n = 1;
        for (uint32_t i = 0; i < bias->ndim; ++i) n *= bias->shape[i];
        if ((int64_t)n != w.d[2]) return fail(MT_EINVAL, "linear: bias must hold out_features elements");
        // The epilogue reads bias[0..n) densely: every dimension longer than 1 must have the
        // stride of a contiguous layout ([1,out], [out] and [out,1] all qualify).
        uint64_t expect = 1;
        for (int i = (int)bias->ndim - 1; i >= 0; --i) {
            if (bias->shape[i] > 1 && bias->strides[i] != expect)
                return fail(MT_EINVAL, "linear: bias must be contiguous");
            expect *= bias->shape[i];
        }
        if (n > 0 && !bias->data) return fail(MT_EINVAL, "linear: null bias data");
        bp = bias->data + bias->offset;
    }
    int epi = (bp ? MT_EPI_BIAS_COL : 0) | (relu ? MT_EPI_RELU : 0);
    return gemm_from_views(x, w, y, bp, epi, MT_MODE_DEFAULT, stream);
}

MT_API int mt_gemm(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, const float* bias, int epi, int mode,
                   void* stream) {
    if (!A || !B || !C) return fail(MT_EINVAL, "gemm: null tensor");
    int nd = (int)C->ndim;
    if (nd != 2 && nd != 3) return fail(MT_EINVAL, "gemm: 2-D or 3-D views only");
    if (mode < MT_MODE_DEFAULT || mode > MT_TF32X3) return fail(MT_EINVAL, "gemm: bad mode %d", mode);
    if (epi & ~7) return fail(MT_EINVAL, "gemm: bad epilogue flags %d", epi);
    View a, b, c;
    int rc;
    if ((rc = to_view(A, nd, "gemm A", a)) || (rc = to_view(B, nd, "gemm B", b)) || (rc = to_view(C, nd, "gemm C", c)))
        return rc;
    if (a.d[0] != c.d[0] || b.d[0] != c.d[0]) return fail(MT_EINVAL, "gemm: batch mismatch");
    if (a.d[2] != b.d[1]) return fail(MT_EINVAL, "gemm: inner dimension mismatch (A.K != B.K)");
    if (c.d[1] != a.d[1] || c.d[2] != b.d[2]) return fail(MT_EINVAL, "gemm: C shape mismatch");
    if (c.d[0] == 1) { a.s[0] = 0; b.s[0] = 0; c.s[0] = 0; }
    return gemm_from_views(a, b, c, bias, epi, mode, stream);
}


// ---- GEMM on host buffers: copies in, GEMM and copies out overlapped by row panels ----
namespace {

// Device-side layout of mt_matmul_host's workspace: A [M,K], B [K,N], C [M,N], each on a
// 256-byte boundary.
struct HostGemmLayout {
    uint64_t a_off, b_off, c_off, bytes;
};

HostGemmLayout host_gemm_layout(uint64_t M, uint64_t K, uint64_t N) {
    auto up = [](uint64_t x) { return (x + 255) & ~uint64_t(255); };
    HostGemmLayout l;
    l.a_off = 0;
    l.b_off = up(M * K * 4);
    l.c_off = l.b_off + up(K * N * 4);
    l.bytes = l.c_off + M * N * 4;
    return l;
}

// Copy streams of the current device, created on first use and kept for the process.
int host_copy_streams(cudaStream_t& h2d, cudaStream_t& d2h) {
    static std::mutex mu;
    static cudaStream_t streams[64][2] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "matmul_host: cudaGetDevice");
    std::lock_guard<std::mutex> g(mu);
    cudaStream_t* s = streams[dev & 63];
    for (int i = 0; i < 2; ++i)
        if (!s[i] && (e = cudaStreamCreateWithFlags(&s[i], cudaStreamNonBlocking)) != cudaSuccess)
            return cuda_fail(e, "matmul_host: copy stream");
    h2d = s[0];
    d2h = s[1];
    return MT_OK;
}

}  // namespace

MT_API size_t mt_matmul_host_workspace_bytes(uint64_t M, uint64_t K, uint64_t N) {
    return (size_t)host_gemm_layout(M, K, N).bytes;
}

MT_API int mt_matmul_host(const float* A, const float* B, float* C, uint64_t M, uint64_t K, uint64_t N, int mode,
                          int panels, void* workspace, size_t ws_bytes, void* stream) {
    if (mode < MT_MODE_DEFAULT || mode > MT_TF32X3) return fail(MT_EINVAL, "matmul_host: bad mode %d", mode);
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
        return fail(MT_EINVAL, "matmul_host: extent beyond 2^31 (M=%llu K=%llu N=%llu)", (unsigned long long)M,
                    (unsigned long long)K, (unsigned long long)N);
    if (M == 0 || N == 0) { t_path = "empty"; return MT_OK; }
    if (!C || (K > 0 && (!A || !B))) return fail(MT_EINVAL, "matmul_host: null buffer");
    const HostGemmLayout lay = host_gemm_layout(M, K, N);
    if (workspace && ws_bytes < lay.bytes)
        return fail(MT_EINVAL, "matmul_host: workspace of %zu bytes < %llu needed", ws_bytes,
                    (unsigned long long)lay.bytes);
    if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(MT_EINVAL, "matmul_host: workspace must be 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream), h2d = nullptr, d2h = nullptr;
    int rc = host_copy_streams(h2d, d2h);
    if (rc) return rc;

    // Row panels on 256-row boundaries (a CTA pair's tile height), at most 8 by default.
    const int64_t tiles = ((int64_t)M + 255) / 256;
    const int P = (int)std::max<int64_t>(1, std::min<int64_t>(panels > 0 ? panels : 8, tiles));
    auto row = [&](int p) -> int64_t { return p >= P ? (int64_t)M : 256 * (tiles * p / P); };

    char* ws = static_cast<char*>(workspace);
    bool owned = false;
    cudaError_t e;
    if (!ws) {
        if ((e = cudaMallocAsync(reinterpret_cast<void**>(&ws), lay.bytes, st)) != cudaSuccess)
            return cuda_fail(e, "matmul_host: workspace");
        owned = true;
    }
    float* Ad = reinterpret_cast<float*>(ws + lay.a_off);
    float* Bd = reinterpret_cast<float*>(ws + lay.b_off);
    float* Cd = reinterpret_cast<float*>(ws + lay.c_off);

    // Events: start (on st), one per A panel landed (h2d), one per C panel computed (st),
    // and the two copy streams' tails, which st waits for before it returns or frees.
    std::vector<cudaEvent_t> ev(2 * P + 3, nullptr);
    for (auto& x : ev)
        if ((e = cudaEventCreateWithFlags(&x, cudaEventDisableTiming)) != cudaSuccess) {
            rc = cuda_fail(e, "matmul_host: event");
            break;
        }
    cudaEvent_t ev_start = ev[0], ev_h2d_tail = ev[2 * P + 1], ev_d2h_tail = ev[2 * P + 2];
    auto ev_a = [&](int p) { return ev[1 + p]; };
    auto ev_c = [&](int p) { return ev[1 + P + p]; };
    auto ck = [&](cudaError_t err, const char* what) {
        if (err != cudaSuccess && rc == MT_OK) rc = cuda_fail(err, what);
        return rc == MT_OK;
    };
    bool joined = false;
    if (rc == MT_OK && ck(cudaEventRecord(ev_start, st), "matmul_host: record") &&
        ck(cudaStreamWaitEvent(h2d, ev_start, 0), "matmul_host: wait") &&
        ck(cudaStreamWaitEvent(d2h, ev_start, 0), "matmul_host: wait")) {
        joined = true;
        // B whole, then A panel by panel (cudaMemcpyDefault: pinned, pageable or device).
        // (K == 0: nothing to copy in; the GEMM then writes zeros.)
        if (K > 0) ck(cudaMemcpyAsync(Bd, B, K * N * 4, cudaMemcpyDefault, h2d), "matmul_host: copy B");
        for (int p = 0; p < P && rc == MT_OK; ++p) {
            const int64_t r0 = row(p), r1 = row(p + 1);
            if (K == 0 || ck(cudaMemcpyAsync(Ad + r0 * K, A + r0 * K, (r1 - r0) * K * 4, cudaMemcpyDefault, h2d),
                             "matmul_host: copy A panel"))
                ck(cudaEventRecord(ev_a(p), h2d), "matmul_host: record");
        }
        for (int p = 0; p < P && rc == MT_OK; ++p) {
            const int64_t r0 = row(p), r1 = row(p + 1);
            if (!ck(cudaStreamWaitEvent(st, ev_a(p), 0), "matmul_host: wait")) break;
            GemmProblem gp;
            gp.A = Ad + r0 * K; gp.sa_b = 0; gp.sa_m = (int64_t)K; gp.sa_k = 1;
            gp.B = Bd;          gp.sb_b = 0; gp.sb_k = (int64_t)N; gp.sb_n = 1;
            gp.C = Cd + r0 * N; gp.sc_b = 0; gp.sc_m = (int64_t)N; gp.sc_n = 1;
            gp.M = r1 - r0; gp.N = (int64_t)N; gp.K = (int64_t)K; gp.batch = 1;
            gp.bias = nullptr; gp.epi = 0;
            if ((rc = run_gemm(gp, mode, st)) != MT_OK) break;
            ck(cudaEventRecord(ev_c(p), st), "matmul_host: record");
        }
        // Copies out after every GEMM is queued: a copy into pageable host memory returns
        // only when it is done, which must not hold back the queueing of later panels.
        for (int p = 0; p < P && rc == MT_OK; ++p) {
            const int64_t r0 = row(p), r1 = row(p + 1);
            if (ck(cudaStreamWaitEvent(d2h, ev_c(p), 0), "matmul_host: wait"))
                ck(cudaMemcpyAsync(C + r0 * N, Cd + r0 * N, (r1 - r0) * N * 4, cudaMemcpyDefault, d2h),
                   "matmul_host: copy C panel");
        }
    }
    // Join: whatever was queued on the copy streams completes before st moves on, on the
    // error paths too, so the workspace is never released under a copy in flight.
    if (joined) {
        cudaError_t e1 = cudaEventRecord(ev_h2d_tail, h2d);
        cudaError_t e2 = cudaEventRecord(ev_d2h_tail, d2h);
        cudaError_t e3 = e1 == cudaSuccess ? cudaStreamWaitEvent(st, ev_h2d_tail, 0) : e1;
        cudaError_t e4 = e2 == cudaSuccess ? cudaStreamWaitEvent(st, ev_d2h_tail, 0) : e2;
        if (e3 != cudaSuccess || e4 != cudaSuccess) {
            // The copy streams could not be joined to st: wait for them here rather than free
            // or return while they may still touch the workspace.
            cudaStreamSynchronize(h2d);
            cudaStreamSynchronize(d2h);
            ck(e3 != cudaSuccess ? e3 : e4, "matmul_host: join");
        }
    }
    if (owned) cudaFreeAsync(ws, st);
    for (auto x : ev)
        if (x) cudaEventDestroy(x);
    if (rc == MT_OK) t_path = "matmul_host " + std::to_string(P) + " panels, last " + t_path;
    return rc;
}


// ---- Conv2D: mirrors of include/TensorOps.hpp:708-712 and explicit-mode variants ----
MT_API int mt_conv2d_gpu(const mt_tensor* in, const mt_tensor* w, const mt_tensor* bias, const mt_tensor* out,
                         uint64_t stride, uint64_t padding, void* stream) {
    return conv_fwd(in, w, bias, out, stride, padding, MT_MODE_DEFAULT, static_cast<cudaStream_t>(stream), "conv2d_gpu");
}
MT_API int mt_conv2d_gpu_strided(const mt_tensor* in, const mt_tensor* w, const mt_tensor* bias, const mt_tensor* out,
                                 uint64_t stride, uint64_t padding, void* stream) {
    return conv_fwd(in, w, bias, out, stride, padding, MT_MODE_DEFAULT, static_cast<cudaStream_t>(stream),
                    "conv2d_gpu_strided");
}
MT_API int mt_conv2d_backward_input_gpu(const mt_tensor* dY, const mt_tensor* w, const mt_tensor* dX, uint64_t stride,
                                        uint64_t padding, void* stream) {
    return conv_dgrad(dY, w, dX, stride, padding, MT_MODE_DEFAULT, static_cast<cudaStream_t>(stream),
                      "conv2d_backward_input_gpu");
}
MT_API int mt_conv2d_backward_weight_gpu(const mt_tensor* dY, const mt_tensor* x, const mt_tensor* dW, uint64_t stride,
                                         uint64_t padding, void* stream) {
    return conv_wgrad(dY, x, dW, stride, padding, MT_MODE_DEFAULT, nullptr, 0, static_cast<cudaStream_t>(stream),
                      "conv2d_backward_weight_gpu");
}
MT_API int mt_conv2d_backward_bias_gpu(const mt_tensor* dY, const mt_tensor* db, void* stream) {
    return conv_bgrad(dY, db, static_cast<cudaStream_t>(stream), "conv2d_backward_bias_gpu");
}

MT_API int mt_sum_rows_gpu(const mt_tensor* X, const mt_tensor* out, void* stream) {
    if (!X || !out) return fail(MT_EINVAL, "sum_rows_gpu: null tensor");
    if (X->ndim != 2) return fail(MT_EINVAL, "sum_rows_gpu: X must be 2-D, got %u dims", X->ndim);
    const uint64_t M = X->shape[0], N = X->shape[1];
    uint64_t on = 0, os = 0;
    if (out->ndim == 1) { on = out->shape[0]; os = out->strides[0]; }
    else if (out->ndim == 2 && out->shape[0] == 1) { on = out->shape[1]; os = out->strides[1]; }
    else return fail(MT_EINVAL, "sum_rows_gpu: out must be [N] or [1, N]");
    if (on != N) return fail(MT_EINVAL, "sum_rows_gpu: out has %llu elements, X has %llu columns",
                             (unsigned long long)on, (unsigned long long)N);
    if (M > INT32_MAX || N > INT32_MAX) return fail(MT_EINVAL, "sum_rows_gpu: extent beyond 2^31");
    if (N == 0) { t_path = "empty"; return MT_OK; }
    if (!out->data || (M > 0 && !X->data)) return fail(MT_EINVAL, "sum_rows_gpu: null data pointer");
    const unsigned blocks = (unsigned)((N + 31) / 32);
    mt::simt::sum_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        X->data + X->offset, (int64_t)X->strides[0], (int64_t)X->strides[1], (int)M, (int)N, out->data + out->offset,
        (int64_t)os);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, "sum_rows launch");
    g_launches.fetch_add(1);
    t_path = "sum_rows";
    return MT_OK;
}

MT_API int mt_conv2d_fwd(const mt_tensor* x, const mt_tensor* w, const mt_tensor* bias, const mt_tensor* y,
                         uint64_t stride, uint64_t padding, int mode, void* stream) {
    if (mode < MT_MODE_DEFAULT || mode > MT_TF32X3) return fail(MT_EINVAL, "conv2d_fwd: bad mode %d", mode);
    return conv_fwd(x, w, bias, y, stride, padding, mode, static_cast<cudaStream_t>(stream), "conv2d_fwd");
}
MT_API int mt_nchw_to_nhwc(const mt_tensor* x, const mt_tensor* out, void* stream) {
    const char* who = "nchw_to_nhwc";
    int rc;
    if ((rc = check4(x, who, "input")) || (rc = check4(out, who, "output"))) return rc;
    for (int i = 0; i < 4; ++i)
        if (x->shape[i] != out->shape[i]) return fail(MT_EINVAL, "%s: output shape differs from the input's", who);
    if (numel(x) == 0) return MT_OK;
    if (!nhwc_dense(out))
        return fail(MT_EINVAL, "%s: output must be a channels-last dense (N, C, H, W) view, C a multiple of 4, "
                               "16-byte aligned", who);
    if (!offsets_fit_32(x)) return fail(MT_EUNSUPPORTED, "%s: a view spans 2^31 elements or more", who);
    int64_t sv[4];
    fill_strides(sv, x);
    rc = to_nhwc(x->data + x->offset, sv, out->data + out->offset, (int)x->shape[0], (int)x->shape[1],
                 (int)x->shape[2], (int)x->shape[3], static_cast<cudaStream_t>(stream));
    if (rc == MT_OK) t_path = "nchw_to_nhwc";
    return rc;
}
MT_API int mt_conv2d_dgrad(const mt_tensor* dy, const mt_tensor* w, const mt_tensor* dx, uint64_t stride,
                           uint64_t padding, int mode, void* stream) {
    if (mode < MT_MODE_DEFAULT || mode > MT_TF32X3) return fail(MT_EINVAL, "conv2d_dgrad: bad mode %d", mode);
    return conv_dgrad(dy, w, dx, stride, padding, mode, static_cast<cudaStream_t>(stream), "conv2d_dgrad");
}
MT_API int mt_conv2d_wgrad(const mt_tensor* dy, const mt_tensor* x, const mt_tensor* dw, uint64_t stride,
                           uint64_t padding, int mode, void* workspace, size_t ws_bytes, void* stream) {
    if (mode < MT_MODE_DEFAULT || mode > MT_TF32X3) return fail(MT_EINVAL, "conv2d_wgrad: bad mode %d", mode);
    return conv_wgrad(dy, x, dw, stride, padding, mode, workspace, ws_bytes, static_cast<cudaStream_t>(stream),
                      "conv2d_wgrad");
}
// ---- weight gradient without any allocation -----------------------------------------
// For callers that cannot allocate device memory at call time: code running under a
// CUDA-graph capture that forbids allocation nodes, plugin hosts that own every byte of
// device memory and reject cudaMalloc from libraries, or real-time loops where an
// allocation could block. The split-K partials go to this fixed file-scope array
// instead of a workspace. The array exists once per GPU that loads the library and stays
// until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;   // 8 MiB of partials per GPU
static __device__ __align__(256) float g_wgrad_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_current_fn() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    return fn;
}

// Device address of the array on the current device. On the host the array's name is
// only a stand-in symbol, so the address is looked up once per device (with that device
// current) and cached together with the context it belongs to: after a device reset the
// runtime makes a new context and loads the module again, and the next call looks the
// address up afresh.
int noalloc_scratch(float** out) {
    static std::mutex mu;
    static float* cache[64] = {};
    static CUcontext cache_ctx[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "conv2d_wgrad_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(MT_EUNSUPPORTED, "conv2d_wgrad_noalloc: device index %d", dev);
    CtxGetCurrentFn cur = ctx_current_fn();
    auto current = [cur]() {
        CUcontext c = nullptr;
        if (!cur || cur(&c) != CUDA_SUCCESS) c = nullptr;
        return c;
    };
    // A thread whose context the runtime has not set up yet reads null here; the lookup
    // below sets it up, and the context is read again after it.
    CUcontext ctx = current();
    std::lock_guard<std::mutex> g(mu);
    if (!cache[dev] || !ctx || cache_ctx[dev] != ctx) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_wgrad_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "conv2d_wgrad_noalloc: cudaGetSymbolAddress");
        cache[dev] = static_cast<float*>(ptr);
        cache_ctx[dev] = current();
    }
    *out = cache[dev];
    return MT_OK;
}

MT_API int mt_conv2d_wgrad_noalloc(const mt_tensor* dy, const mt_tensor* x, const mt_tensor* dw, uint64_t stride,
                                   uint64_t padding, int mode, void* stream) {
    if (mode < MT_MODE_DEFAULT || mode > MT_TF32X3) return fail(MT_EINVAL, "conv2d_wgrad_noalloc: bad mode %d", mode);
    // This variant always takes the gather kernel (its only scratch is the partials).
    size_t need = 0;
    if (dy && x && dw && dy->ndim == 4 && x->ndim == 4 && dw->ndim == 4) {
        ConvShape s;
        if (!conv_shape(x, dw, dy, stride, padding, "conv2d_wgrad_noalloc", s) &&
            resolve_mode(mode) != MT_STRICT_FP32 && s.N * s.Ho * s.Wo > 0)
            need = wgrad_plan(s, dev_info().sms).ws_bytes;
    }
    if (need > kNoAllocScratchBytes)
        return fail(MT_EINVAL,
                    "conv2d_wgrad_noalloc: this problem needs %zu bytes of split-K partials; the static scratch "
                    "holds %zu (use mt_conv2d_wgrad with a workspace)",
                    need, kNoAllocScratchBytes);
    float* scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // Every split writes its whole partial tile (zeros for an empty split), so nothing
    // left in the array by an earlier call is read.
    return conv_wgrad(dy, x, dw, stride, padding, mode, scratch, kNoAllocScratchBytes,
                      static_cast<cudaStream_t>(stream), "conv2d_wgrad_noalloc", /*allow_tma=*/false);
}

MT_API size_t mt_conv2d_wgrad_workspace_bytes(const mt_tensor* dy, const mt_tensor* x, const mt_tensor* dw,
                                              uint64_t stride, uint64_t padding, int mode) {
    // Shapes only: no pointer is dereferenced, so data may be NULL here.
    if (!dy || !x || !dw || dy->ndim != 4 || x->ndim != 4 || dw->ndim != 4) return 0;
    ConvShape s;
    if (conv_shape(x, dw, dy, stride, padding, "wgrad_ws", s)) return 0;
    if (s.N * s.Ho * s.Wo == 0 || s.Co * s.C * s.kh * s.kw == 0) return 0;
    if (resolve_mode(mode) == MT_STRICT_FP32) return strict_wgrad_bytes(s);
    const WgradTmaPlan tp = wgrad_tma_plan(s, dy, x, dev_info().sms, resolve_mode(mode) == MT_TF32X3);
    return tp.ok ? tp.bytes : wgrad_plan(s, dev_info().sms).ws_bytes;
}


// ---- multi-GPU: peer memory and the GEMM that writes every rank's output -------------

// Longest wait mt_peer_barrier accepts (60 s): every device-side wait has a bound.
constexpr uint64_t kMaxPeerWaitNs = 60ull * 1000 * 1000 * 1000;

MT_API int mt_ipc_get_handle(const void* dptr, void* handle_out, uint64_t* offset_out) {
    if (!dptr || !handle_out || !offset_out) return fail(MT_EINVAL, "ipc_get_handle: null argument");
    GetAddressRangeFn range = addr_range_fn();
    if (!range) return fail(MT_EUNSUPPORTED, "ipc_get_handle: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dptr)) != CUDA_SUCCESS)
        return fail(MT_EINVAL, "ipc_get_handle: not a device allocation");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    memcpy(handle_out, &h, sizeof h);
    *offset_out = reinterpret_cast<uint64_t>(dptr) - static_cast<uint64_t>(base);
    return MT_OK;
}

MT_API int mt_ipc_open(const void* handle, uint64_t offset, void** dptr_out) {
    if (!handle || !dptr_out) return fail(MT_EINVAL, "ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    *dptr_out = static_cast<char*>(base) + offset;
    return MT_OK;
}

MT_API int mt_ipc_close(void* dptr, uint64_t offset) {
    cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(dptr) - offset);
    return e == cudaSuccess ? MT_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

MT_API int mt_gemm_multi(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, float* const* extra_dst,
                         int nextra, const float* bias, int epi, int mode, void* stream) {
    if (nextra < 0 || nextra >= mt::umma::kMaxDst) return fail(MT_EINVAL, "gemm_multi: 0 <= nextra < %d", mt::umma::kMaxDst);
    if (nextra && !extra_dst) return fail(MT_EINVAL, "gemm_multi: extra_dst is null");
    for (int i = 0; i < nextra; ++i)
        if (!extra_dst[i]) return fail(MT_EINVAL, "gemm_multi: extra_dst[%d] is null", i);
    if (mode < MT_MODE_DEFAULT || mode > MT_TF32X3) return fail(MT_EINVAL, "gemm_multi: bad mode %d", mode);
    if (epi & ~7) return fail(MT_EINVAL, "gemm_multi: bad epilogue flags %d", epi);
    if (!A || !B || !C) return fail(MT_EINVAL, "gemm_multi: null tensor");
    const int nd = (int)C->ndim;
    if (nd != 2 && nd != 3) return fail(MT_EINVAL, "gemm_multi: 2-D or 3-D views only");
    View a, b, c;
    int rc;
    if ((rc = to_view(A, nd, "gemm_multi A", a)) || (rc = to_view(B, nd, "gemm_multi B", b)) ||
        (rc = to_view(C, nd, "gemm_multi C", c)))
        return rc;
    if (a.d[0] != c.d[0] || b.d[0] != c.d[0]) return fail(MT_EINVAL, "gemm_multi: batch mismatch");
    if (a.d[2] != b.d[1]) return fail(MT_EINVAL, "gemm_multi: inner dimension mismatch (A.K != B.K)");
    if (c.d[1] != a.d[1] || c.d[2] != b.d[2]) return fail(MT_EINVAL, "gemm_multi: C shape mismatch");
    if (c.s[2] != 1 && c.d[2] > 1) return fail(MT_EINVAL, "gemm_multi: C rows must be contiguous");
    if (c.d[0] == 1) { a.s[0] = 0; b.s[0] = 0; c.s[0] = 0; }
    GemmProblem p;
    p.A = a.ptr; p.sa_b = a.s[0]; p.sa_m = a.s[1]; p.sa_k = a.s[2];
    p.B = b.ptr; p.sb_b = b.s[0]; p.sb_k = b.s[1]; p.sb_n = b.s[2];
    p.C = const_cast<float*>(c.ptr); p.sc_b = c.s[0]; p.sc_m = c.s[1]; p.sc_n = 1;
    p.M = a.d[1]; p.K = a.d[2]; p.N = b.d[2]; p.batch = c.d[0];
    p.bias = bias; p.epi = epi;
    if (p.M == 0 || p.N == 0 || p.batch == 0) return MT_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int m = resolve_mode(mode);
    if (m != MT_STRICT_FP32 && p.K > 0) {
        std::string saved = t_err;
        rc = launch_umma(p, m == MT_TF32X3, st, extra_dst, nextra);
        if (rc == MT_OK) { t_path += " +" + std::to_string(nextra) + " peers"; return MT_OK; }
        if (rc != MT_EUNSUPPORTED) return rc;
        t_err = saved;
    }
    // Local product, then one 2-D copy per peer and batch (stream-ordered, over NVLink).
    if ((rc = run_gemm(p, m, st))) return rc;
    for (int i = 0; i < nextra; ++i) {
        for (int64_t bi = 0; bi < p.batch; ++bi) {
            cudaError_t e = cudaMemcpy2DAsync(extra_dst[i] + bi * p.sc_b, p.sc_m * 4, p.C + bi * p.sc_b, p.sc_m * 4,
                                              p.N * 4, p.M, cudaMemcpyDeviceToDevice, st);
            if (e != cudaSuccess) return cuda_fail(e, "gemm_multi peer copy");
        }
    }
    t_path += " +" + std::to_string(nextra) + " peer copies";
    return MT_OK;
}

MT_API int mt_peer_barrier(int* const* flags, int rank, int world, int epoch, uint64_t timeout_ns, void* stream) {
    // Every device-side wait stays bounded: a longer limit is refused, not clamped.
    if (timeout_ns > kMaxPeerWaitNs)
        return fail(MT_EINVAL, "peer_barrier: timeout_ns %llu above the %llu ns maximum",
                    (unsigned long long)timeout_ns, (unsigned long long)kMaxPeerWaitNs);
    if (world < 1 || world > mt::umma::kMaxDst || rank < 0 || rank >= world || !flags)
        return fail(MT_EINVAL, "peer_barrier: bad rank/world");
    peer::Flags fl;
    for (int d = 0; d < mt::umma::kMaxDst; ++d) fl.f[d] = d < world ? flags[d] : nullptr;
    for (int d = 0; d < world; ++d)
        if (!fl.f[d]) return fail(MT_EINVAL, "peer_barrier: flags[%d] is null", d);
    peer::barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(fl, rank, world, epoch,
                                                                          (unsigned long long)timeout_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && e != cudaErrorStreamCaptureUnsupported) return cuda_fail(e, "peer barrier launch");
    g_launches.fetch_add(1);
    return MT_OK;
}

MT_API int mt_copy_rows_async(void* dst, uint64_t dpitch, const void* src, uint64_t spitch, uint64_t width_bytes,
                              uint64_t rows, void* stream) {
    if (rows == 0 || width_bytes == 0) return MT_OK;
    if (!dst || !src) return fail(MT_EINVAL, "copy_rows_async: null pointer");
    if (dpitch < width_bytes || spitch < width_bytes) return fail(MT_EINVAL, "copy_rows_async: pitch < width");
    cudaError_t e = cudaMemcpy2DAsync(dst, dpitch, src, spitch, width_bytes, rows, cudaMemcpyDeviceToDevice,
                                      static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "copy_rows_async");
    return MT_OK;
}

MT_API int mt_set_scratch_allocator(mt_scratch_alloc_fn alloc, mt_scratch_free_fn free_fn, void* ctx) {
    if ((alloc == nullptr) != (free_fn == nullptr))
        return fail(MT_EINVAL, "set_scratch_allocator: give both functions, or neither");
    std::lock_guard<std::mutex> g(g_scratch_mu);
    g_scratch.alloc = alloc;
    g_scratch.free = free_fn;
    g_scratch.ctx = ctx;
    return MT_OK;
}

MT_API void mt_scratch_counts(uint64_t* stream_ordered, uint64_t* from_allocator) {
    if (stream_ordered) *stream_ordered = g_async_allocs.load();
    if (from_allocator) *from_allocator = g_hook_allocs.load();
}

MT_API int mt_set_default_mode(int mode) {
    int prev = resolve_mode(MT_MODE_DEFAULT);
    if (mode >= MT_STRICT_FP32 && mode <= MT_TF32X3) g_default_mode.store(mode);
    return prev;
}
MT_API int mt_get_default_mode(void) { return resolve_mode(MT_MODE_DEFAULT); }
MT_API const char* mt_last_error(void) { return t_err.c_str(); }
MT_API const char* mt_last_path(void) { return t_path.c_str(); }
MT_API uint64_t mt_launch_count(void) { return g_launches.load(); }

MT_API int mt_device_status(int reset) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return -cuda_fail(e, "device_status sync");
    int v = 0;
    e = cudaMemcpyFromSymbol(&v, mt::g_dev_status, sizeof(int));
    if (e != cudaSuccess) return -cuda_fail(e, "device_status read");
    if (reset) {
        int z = 0;
        cudaMemcpyToSymbol(mt::g_dev_status, &z, sizeof(int));
    }
    return v;
}

MT_API const char* mt_version(void) { return "minitensor_b200 mtgemm 0.1 (sm_100a)"; }

}  // extern "C"
