// simt_gemm.cuh -- FFMA-only fp32 GEMM: the strict-fp32 mode and the path for shapes or
// views the tensor-core kernel cannot take (unaligned views, tiny problems).
//
// C[b,m,n] = epi( sum_k A[b,m,k] * B[b,k,n] ), every operand an arbitrary strided view
// (element strides; batch stride 0 = broadcast operand, as produced by expand()).
// Each output element is accumulated over k in ascending order in one fp32 register,
// the order of the reference's matmul_cpu (include/TensorOps.hpp:150-159), with FFMA.
//
// Tile 128x128x16, 256 threads, 8x8 outputs per thread (two 4x4 quadrants 64 apart so the
// shared-memory reads are conflict-free float4 broadcasts), double-buffered shared tiles
// filled through registers one 128x8 slab at a time (the next tile's slab h is loaded while
// slab h of this one is computed), 128-bit global loads when the contiguous dimension and
// the view alignment allow them. The 16-deep tile halves the barriers per FFMA of the
// 8-deep one; with one CTA per SM (up to 255 registers) it measured 5% (8192^3) to 28%
// (256 x 4096 x 1024) faster, bitwise equal; the TN layout keeps two CTAs per SM, where it
// is 9% faster than with one.
#pragma once

#include "mt_common.cuh"

namespace mt {

struct GemmProblem {
    const float* A; int64_t sa_b, sa_m, sa_k;
    const float* B; int64_t sb_b, sb_k, sb_n;
    float* C;       int64_t sc_b, sc_m, sc_n;
    int64_t M, N, K, batch;
    const float* bias;   // may be null
    int epi;             // MT_EPI_* flags
};

enum : int { kEpiBiasRow = 1, kEpiBiasCol = 2, kEpiRelu = 4 };

// Loader layouts for the A tile (BM x BK) and the B tile (BK x BN).
enum : int { kLdKContigVec = 0, kLdMNContigVec = 1, kLdGeneric = 2 };

namespace simt {
constexpr int BM = 128, BN = 128, BK = 16, THREADS = 256;
constexpr int SLABS = BK / 8;   // 128 x 8 slabs per operand tile

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Each thread fetches 4 elements of the A tile into registers.
template <int LA>
__device__ __forceinline__ void load_a(const GemmProblem& p, const float* A, int64_t m0, int64_t k0, int t,
                                       float (&v)[4]) {
    if (LA == kLdMNContigVec) {
        // 8 k-rows x 32 float4 along m.
        int k = t >> 5, mq = (t & 31) * 4;
        int64_t gk = k0 + k, gm = m0 + mq;
        if (gk < p.K && gm + 3 < p.M) {
            float4 x = ldg4(A + gm + gk * p.sa_k);
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                v[i] = (gk < p.K && gm + i < p.M) ? __ldg(A + (gm + i) + gk * p.sa_k) : 0.f;
        }
    } else {
        // 128 m-rows x 2 groups of 4 consecutive k.
        int m = t >> 1, kq = (t & 1) * 4;
        int64_t gm = m0 + m, gk = k0 + kq;
        if (LA == kLdKContigVec && gm < p.M && gk + 3 < p.K) {
            float4 x = ldg4(A + gm * p.sa_m + gk);
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                v[i] = (gm < p.M && gk + i < p.K) ? __ldg(A + gm * p.sa_m + (gk + i) * p.sa_k) : 0.f;
        }
    }
}

template <int LA>
__device__ __forceinline__ void store_a(float (*As)[BM], int t, const float (&v)[4]) {
    if (LA == kLdMNContigVec) {
        int k = t >> 5, mq = (t & 31) * 4;
        *reinterpret_cast<float4*>(&As[k][mq]) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        int m = t >> 1, kq = (t & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) As[kq + i][m] = v[i];
    }
}

// B loaders: kLdMNContigVec = contiguous along n (row-major B), kLdKContigVec =
// contiguous along k (a transposed view).
template <int LB>
__device__ __forceinline__ void load_b(const GemmProblem& p, const float* B, int64_t k0, int64_t n0, int t,
                                       float (&v)[4]) {
    if (LB == kLdKContigVec) {
        int n = t >> 1, kq = (t & 1) * 4;
        int64_t gn = n0 + n, gk = k0 + kq;
        if (gn < p.N && gk + 3 < p.K) {
            float4 x = ldg4(B + gn * p.sb_n + gk);
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                v[i] = (gn < p.N && gk + i < p.K) ? __ldg(B + gn * p.sb_n + (gk + i) * p.sb_k) : 0.f;
        }
    } else {
        int k = t >> 5, nq = (t & 31) * 4;
        int64_t gk = k0 + k, gn = n0 + nq;
        if (LB == kLdMNContigVec && gk < p.K && gn + 3 < p.N) {
            float4 x = ldg4(B + gk * p.sb_k + gn);
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                v[i] = (gk < p.K && gn + i < p.N) ? __ldg(B + gk * p.sb_k + (gn + i) * p.sb_n) : 0.f;
        }
    }
}

template <int LB>
__device__ __forceinline__ void store_b(float (*Bs)[BN], int t, const float (&v)[4]) {
    if (LB == kLdKContigVec) {
        int n = t >> 1, kq = (t & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) Bs[kq + i][n] = v[i];
    } else {
        int k = t >> 5, nq = (t & 31) * 4;
        *reinterpret_cast<float4*>(&Bs[k][nq]) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

__device__ __forceinline__ float epilogue(float acc, const GemmProblem& p, int64_t m, int64_t n) {
    if (p.epi & kEpiBiasCol) acc = acc + __ldg(p.bias + n);
    if (p.epi & kEpiBiasRow) acc = acc + __ldg(p.bias + m);
    if (p.epi & kEpiRelu) acc = acc > 0.f ? acc : 0.f;
    return acc;
}

template <int LA, int LB>
__global__ void __launch_bounds__(THREADS, (LA == kLdMNContigVec && LB == kLdMNContigVec) ? 2 : 1)
gemm_kernel(GemmProblem p) {
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int t = threadIdx.x;
    const int tx = t & 15, ty = t >> 4;
    const int64_t b = blockIdx.z;
    const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
    const float* A = p.A + b * p.sa_b;
    const float* B = p.B + b * p.sb_b;
    float* C = p.C + b * p.sc_b;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    float ra[4], rb[4];
    const int64_t ktiles = (p.K + BK - 1) / BK;
    if (ktiles > 0) {
#pragma unroll
        for (int h = 0; h < SLABS; ++h) {
            load_a<LA>(p, A, m0, 8 * h, t, ra);
            load_b<LB>(p, B, 8 * h, n0, t, rb);
            store_a<LA>(As[0] + 8 * h, t, ra);
            store_b<LB>(Bs[0] + 8 * h, t, rb);
        }
    }
    __syncthreads();

    for (int64_t kt = 0; kt < ktiles; ++kt) {
        const int cur = (int)(kt & 1);
        const bool more = kt + 1 < ktiles;
#pragma unroll
        for (int h = 0; h < SLABS; ++h) {
            if (more) {
                load_a<LA>(p, A, m0, (kt + 1) * BK + 8 * h, t, ra);
                load_b<LB>(p, B, (kt + 1) * BK + 8 * h, n0, t, rb);
            }
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const int k = 8 * h + kk;
                float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
                float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4 + 64]);
                float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4]);
                float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4 + 64]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
            }
            if (more) {
                store_a<LA>(As[cur ^ 1] + 8 * h, t, ra);
                store_b<LB>(Bs[cur ^ 1] + 8 * h, t, rb);
            }
        }
        __syncthreads();
    }

    const bool vec = (p.sc_n == 1) && ((p.sc_m & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t m = m0 + ty * 4 + (i & 3) + (i >> 2) * 64;
        if (m >= p.M) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t n = n0 + tx * 4 + h * 64;
            float o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = (n + j < p.N) ? epilogue(acc[i][h * 4 + j], p, m, n + j) : 0.f;
            if (vec && n + 3 < p.N) {
                *reinterpret_cast<float4*>(C + m * p.sc_m + n) = make_float4(o[0], o[1], o[2], o[3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (n + j < p.N) C[m * p.sc_m + (n + j) * p.sc_n] = o[j];
            }
        }
    }
}

// Small grids. A strict-fp32 output is one FFMA chain in k order (the reference's order),
// so K cannot be split; an output with fewer 128x128 tiles than the GPU has SMs (512^3:
// 16 CTAs for 148 SMs, each running a 512- to 4096-long chain per output) is instead cut
// into 64x64 tiles: 4x the CTAs, each 128 threads with 8 x 4 outputs (rows ty*4.. and
// ty*4+32.., columns tx*4..), the same per-output order, so the same bits.
namespace small {
constexpr int BM = 64, BN = 64, BK = 16, THREADS = 128;

// Eight elements of the A tile (64 x 16) into v: K-contiguous layouts take row t/2, k
// (t%2)*8 .. +7; the M-contiguous layout takes k-row t/8, rows (t%8)*8 .. +7.
template <int LA>
__device__ __forceinline__ void load_a(const GemmProblem& p, const float* A, int64_t m0, int64_t k0, int t,
                                       float (&v)[8]) {
    if (LA == kLdMNContigVec) {
        const int64_t gk = k0 + (t >> 3), gm = m0 + (t & 7) * 8;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (gk < p.K && gm + 4 * h + 3 < p.M) {
                const float4 x = ldg4(A + gm + 4 * h + gk * p.sa_k);
                v[4 * h] = x.x; v[4 * h + 1] = x.y; v[4 * h + 2] = x.z; v[4 * h + 3] = x.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    v[4 * h + i] = (gk < p.K && gm + 4 * h + i < p.M) ? __ldg(A + (gm + 4 * h + i) + gk * p.sa_k) : 0.f;
            }
        }
    } else {
        const int64_t gm = m0 + (t >> 1), gk = k0 + (t & 1) * 8;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (LA == kLdKContigVec && gm < p.M && gk + 4 * h + 3 < p.K) {
                const float4 x = ldg4(A + gm * p.sa_m + gk + 4 * h);
                v[4 * h] = x.x; v[4 * h + 1] = x.y; v[4 * h + 2] = x.z; v[4 * h + 3] = x.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    v[4 * h + i] = (gm < p.M && gk + 4 * h + i < p.K)
                                       ? __ldg(A + gm * p.sa_m + (gk + 4 * h + i) * p.sa_k) : 0.f;
            }
        }
    }
}

template <int LA>
__device__ __forceinline__ void store_a(float (*As)[BM], int t, const float (&v)[8]) {
    if (LA == kLdMNContigVec) {
        const int k = t >> 3, mq = (t & 7) * 8;
        *reinterpret_cast<float4*>(&As[k][mq]) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(&As[k][mq + 4]) = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        const int m = t >> 1, kq = (t & 1) * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) As[kq + i][m] = v[i];
    }
}

// Eight elements of the B tile (16 x 64): the N-contiguous layout takes k-row t/8, columns
// (t%8)*8 .. +7; K-contiguous layouts take column t/2, k (t%2)*8 .. +7.
template <int LB>
__device__ __forceinline__ void load_b(const GemmProblem& p, const float* B, int64_t k0, int64_t n0, int t,
                                       float (&v)[8]) {
    if (LB == kLdMNContigVec) {
        const int64_t gk = k0 + (t >> 3), gn = n0 + (t & 7) * 8;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (gk < p.K && gn + 4 * h + 3 < p.N) {
                const float4 x = ldg4(B + gk * p.sb_k + gn + 4 * h);
                v[4 * h] = x.x; v[4 * h + 1] = x.y; v[4 * h + 2] = x.z; v[4 * h + 3] = x.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    v[4 * h + i] = (gk < p.K && gn + 4 * h + i < p.N) ? __ldg(B + gk * p.sb_k + gn + 4 * h + i) : 0.f;
            }
        }
    } else {
        const int64_t gn = n0 + (t >> 1), gk = k0 + (t & 1) * 8;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (LB == kLdKContigVec && gn < p.N && gk + 4 * h + 3 < p.K) {
                const float4 x = ldg4(B + gn * p.sb_n + gk + 4 * h);
                v[4 * h] = x.x; v[4 * h + 1] = x.y; v[4 * h + 2] = x.z; v[4 * h + 3] = x.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    v[4 * h + i] = (gn < p.N && gk + 4 * h + i < p.K)
                                       ? __ldg(B + gn * p.sb_n + (gk + 4 * h + i) * p.sb_k) : 0.f;
            }
        }
    }
}

template <int LB>
__device__ __forceinline__ void store_b(float (*Bs)[BN], int t, const float (&v)[8]) {
    if (LB == kLdMNContigVec) {
        const int k = t >> 3, nq = (t & 7) * 8;
        *reinterpret_cast<float4*>(&Bs[k][nq]) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(&Bs[k][nq + 4]) = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        const int n = t >> 1, kq = (t & 1) * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) Bs[kq + i][n] = v[i];
    }
}

template <int LA, int LB>
__global__ void __launch_bounds__(THREADS) gemm_kernel(GemmProblem p) {
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    const int t = threadIdx.x;
    const int tx = t & 15, ty = t >> 4;
    const int64_t b = blockIdx.z;
    const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
    const float* A = p.A + b * p.sa_b;
    const float* B = p.B + b * p.sb_b;
    float* C = p.C + b * p.sc_b;

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    float ra[8], rb[8];
    const int64_t ktiles = (p.K + BK - 1) / BK;
    if (ktiles > 0) {
        load_a<LA>(p, A, m0, 0, t, ra);
        load_b<LB>(p, B, 0, n0, t, rb);
        store_a<LA>(As[0], t, ra);
        store_b<LB>(Bs[0], t, rb);
    }
    __syncthreads();
    for (int64_t kt = 0; kt < ktiles; ++kt) {
        const int cur = (int)(kt & 1);
        const bool more = kt + 1 < ktiles;
        if (more) {
            load_a<LA>(p, A, m0, (kt + 1) * BK, t, ra);
            load_b<LB>(p, B, (kt + 1) * BK, n0, t, rb);
        }
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4 + 32]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
        }
        if (more) {
            store_a<LA>(As[cur ^ 1], t, ra);
            store_b<LB>(Bs[cur ^ 1], t, rb);
        }
        __syncthreads();
    }

    const bool vec = (p.sc_n == 1) && ((p.sc_m & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    const int64_t n = n0 + tx * 4;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t m = m0 + ty * 4 + (i & 3) + (i >> 2) * 32;
        if (m >= p.M) continue;
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = (n + j < p.N) ? simt::epilogue(acc[i][j], p, m, n + j) : 0.f;
        if (vec && n + 3 < p.N) {
            *reinterpret_cast<float4*>(C + m * p.sc_m + n) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (n + j < p.N) C[m * p.sc_m + (n + j) * p.sc_n] = o[j];
        }
    }
}
}  // namespace small

__global__ void fill_epilogue_kernel(GemmProblem p) {
    const int64_t total = p.batch * p.M * p.N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = i / (p.M * p.N), r = i % (p.M * p.N);
        int64_t m = r / p.N, n = r % p.N;
        p.C[b * p.sc_b + m * p.sc_m + n * p.sc_n] = epilogue(0.f, p, m, n);
    }
}

// out[n] = sum over rows m of X[m, n] (the axis-0 sum). One block of 8 warps per 32
// columns: lane = column, warp w sums rows w, w + 8, ... in ascending order, then thread
// (0, lane) adds the 8 partial sums in warp order -- a fixed order, so the result is
// deterministic. X is any 2-D view (strides in elements), out any 1-D view.
__global__ void __launch_bounds__(256) sum_rows_kernel(const float* __restrict__ x, int64_t sm, int64_t sn, int M,
                                                       int N, float* __restrict__ out, int64_t so) {
    __shared__ float part[8][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int n = blockIdx.x * 32 + lane;
    float acc = 0.f;
    if (n < N) {
        const float* col = x + (int64_t)n * sn;
        int m = w;
        for (; m + 56 < M; m += 64) {          // 8 independent loads in flight
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldg(col + (int64_t)(m + 8 * j) * sm);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc += v[j];
        }
        for (; m < M; m += 8) acc += __ldg(col + (int64_t)m * sm);
    }
    part[w][lane] = acc;
    __syncthreads();
    if (w == 0 && n < N) {
        float t = part[0][lane];
#pragma unroll
        for (int j = 1; j < 8; ++j) t += part[j][lane];
        out[(int64_t)n * so] = t;
    }
}

}  // namespace simt
}  // namespace mt
