// conv_simt.cuh -- Conv2D in strict fp32: implicit GEMMs on FFMA, the strict-fp32 mode of
// the conv entry points (the tensor-core kernels serve TF32 and 3xTF32).
//
// No im2col buffer: the loaders gather the operand tiles straight from the NCHW views
// (any strides). Tile 128 x BN x 8 (BN = 64 or 128), 256 threads, 8 x BN/16 outputs per
// thread in quadrants 64 apart (conflict-free float4 reads of shared memory),
// register-staged double buffering -- the structure of the SIMT GEMM (simt_gemm.cuh).
//
// Every output accumulates in the reference CPU routine's order, with FFMA:
//   forward   y = bias, then + over (c_in, r, s) ascending          (include/TensorOps.hpp:235-273)
//             M = N*Ho*Wo pixels, N = C_out, K = C_in*kh*kw
//   input-grad dx = 0, then + over (c_out, r descending, s descending), i.e. output rows
//             and columns ascending (the reference scatters over (c_out, y, x), :319-356)
//             M = N*H*W pixels, N = C_in, K = C_out*kh*kw
//   weight-grad per image n: part_n = sum over (y, x) ascending; dW = 0 + part_0 + part_1 ...
//             in image order (:358-396). One GEMM per image (grid z): M = C_in*kh*kw,
//             N = C_out, K = Ho*Wo, into part[n][C_in*kh*kw][C_out]; wgrad_sum_kernel then
//             adds the images in order (and transposes to [C_out][C_in][kh][kw]).
#pragma once

#include "mt_common.cuh"

namespace mt {
namespace convs {

constexpr int BM = 128, BK = 8, THREADS = 256;
enum : int { kFwd = 0, kDgrad = 1, kWgrad = 2 };

struct Params {
    const float* x; int64_t sx[4];     // input (fwd, wgrad)
    const float* w; int64_t sw[4];     // weights (fwd, dgrad)
    const float* dy; int64_t sdy[4];   // grad_output (dgrad, wgrad)
    const float* bias;                 // fwd, may be null
    float* out; int64_t so[4];         // y (fwd) / dx (dgrad); wgrad: part [N][M][Ncol] dense
    int N, C, H, W, Co, kh, kw, Ho, Wo, stride, pad;
    int64_t M;                         // GEMM rows
    int Ncol, K;                       // GEMM columns, reduction length
};

// The A tile (128 x 8) element for GEMM row m, reduction index k. Thread t loads 4
// consecutive rows m0 + 4 (t & 31) .. +3 of reduction index k0 + (t >> 5); the row-dependent
// parts of the address are computed once per thread (RowInfo).
struct RowInfo {
    int64_t base[4];   // element offset of the row's origin in its tensor
    int a[4], b[4];    // fwd: iy0, ix0; dgrad: iy + pad, ix + pad; wgrad: r, s
    bool ok[4];
};

template <int KIND>
__device__ __forceinline__ void row_info(const Params& p, int64_t m0, int t, RowInfo& ri) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + (t & 31) * 4 + i;
        ri.ok[i] = m < p.M;
        const int64_t mm = ri.ok[i] ? m : 0;
        if (KIND == kFwd) {
            const int64_t hw = (int64_t)p.Ho * p.Wo;
            const int n = (int)(mm / hw);
            const int rem = (int)(mm - (int64_t)n * hw);
            const int oy = rem / p.Wo, ox = rem - oy * p.Wo;
            ri.base[i] = (int64_t)n * p.sx[0];
            ri.a[i] = oy * p.stride - p.pad;
            ri.b[i] = ox * p.stride - p.pad;
        } else if (KIND == kDgrad) {
            const int64_t hw = (int64_t)p.H * p.W;
            const int n = (int)(mm / hw);
            const int rem = (int)(mm - (int64_t)n * hw);
            const int iy = rem / p.W, ix = rem - iy * p.W;
            ri.base[i] = (int64_t)n * p.sdy[0];
            ri.a[i] = iy + p.pad;
            ri.b[i] = ix + p.pad;
        } else {
            // row j = (ci, r, s) of the weight gradient
            const int khw = p.kh * p.kw;
            const int ci = (int)(mm / khw);
            const int rs = (int)(mm - (int64_t)ci * khw);
            const int r = rs / p.kw, s = rs - r * p.kw;
            ri.base[i] = (int64_t)ci * p.sx[1];
            ri.a[i] = r - p.pad;
            ri.b[i] = s - p.pad;
        }
    }
}

template <int KIND>
__device__ __forceinline__ void load_a(const Params& p, const RowInfo& ri, int img, int k0, int t, float (&v)[4]) {
    const int k = k0 + (t >> 5);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = 0.f;
    if (k >= p.K) return;
    if (KIND == kFwd) {
        const int khw = p.kh * p.kw;
        const int ci = k / khw, rs = k - ci * khw;
        const int r = rs / p.kw, s = rs - r * p.kw;
        const int64_t cb = (int64_t)ci * p.sx[1];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int iy = ri.a[i] + r, ix = ri.b[i] + s;
            if (ri.ok[i] && iy >= 0 && iy < p.H && ix >= 0 && ix < p.W)
                v[i] = __ldg(p.x + ri.base[i] + cb + (int64_t)iy * p.sx[2] + (int64_t)ix * p.sx[3]);
        }
    } else if (KIND == kDgrad) {
        const int khw = p.kh * p.kw;
        const int co = k / khw, rs = k - co * khw;
        const int r = p.kh - 1 - rs / p.kw, s = p.kw - 1 - (rs - (rs / p.kw) * p.kw);
        const int64_t cb = (int64_t)co * p.sdy[1];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int ty = ri.a[i] - r, tx = ri.b[i] - s;   // oy * stride, ox * stride
            if (!ri.ok[i] || ty < 0 || tx < 0) continue;
            const int oy = ty / p.stride, ox = tx / p.stride;
            if (oy * p.stride == ty && ox * p.stride == tx && oy < p.Ho && ox < p.Wo)
                v[i] = __ldg(p.dy + ri.base[i] + cb + (int64_t)oy * p.sdy[2] + (int64_t)ox * p.sdy[3]);
        }
    } else {
        const int oy = k / p.Wo, ox = k - oy * p.Wo;
        const int64_t ib = (int64_t)img * p.sx[0];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int iy = oy * p.stride + ri.a[i], ix = ox * p.stride + ri.b[i];
            if (ri.ok[i] && iy >= 0 && iy < p.H && ix >= 0 && ix < p.W)
                v[i] = __ldg(p.x + ib + ri.base[i] + (int64_t)iy * p.sx[2] + (int64_t)ix * p.sx[3]);
        }
    }
}

// The B tile (8 x BN): thread t loads NB = BN / 32 consecutive reduction indices
// k0 + (t % (8 / NB)) * NB .. of column n0 + t / (8 / NB).
template <int KIND, int BN>
__device__ __forceinline__ void load_b(const Params& p, int img, int64_t n0, int k0, int t, float (&v)[BN / 32]) {
    constexpr int NB = BN / 32, GROUPS = BK / NB;
    const int n = (int)n0 + t / GROUPS;
    const int kq = k0 + (t % GROUPS) * NB;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
        const int k = kq + i;
        float x = 0.f;
        if (n < p.Ncol && k < p.K) {
            if (KIND == kFwd) {
                const int khw = p.kh * p.kw;
                const int ci = k / khw, rs = k - ci * khw;
                const int r = rs / p.kw, s = rs - r * p.kw;
                x = __ldg(p.w + (int64_t)n * p.sw[0] + (int64_t)ci * p.sw[1] + (int64_t)r * p.sw[2] + (int64_t)s * p.sw[3]);
            } else if (KIND == kDgrad) {
                const int khw = p.kh * p.kw;
                const int co = k / khw, rs = k - co * khw;
                const int r = p.kh - 1 - rs / p.kw, s = p.kw - 1 - (rs - (rs / p.kw) * p.kw);
                x = __ldg(p.w + (int64_t)co * p.sw[0] + (int64_t)n * p.sw[1] + (int64_t)r * p.sw[2] + (int64_t)s * p.sw[3]);
            } else {
                const int oy = k / p.Wo, ox = k - oy * p.Wo;
                x = __ldg(p.dy + (int64_t)img * p.sdy[0] + (int64_t)n * p.sdy[1] + (int64_t)oy * p.sdy[2] +
                          (int64_t)ox * p.sdy[3]);
            }
        }
        v[i] = x;
    }
}

template <int KIND, int BN>
__global__ void __launch_bounds__(THREADS, 2) conv_simt_kernel(Params p) {
    constexpr int NB = BN / 32, GROUPS = BK / NB, TN = BN / 16;   // TN outputs per thread along n
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int t = threadIdx.x;
    const int tx = t & 15, ty = t >> 4;
    const int img = blockIdx.z;                       // wgrad: the image of this GEMM
    const int64_t m0 = (int64_t)blockIdx.y * BM;
    const int64_t n0 = (int64_t)blockIdx.x * BN;

    RowInfo ri;
    row_info<KIND>(p, m0, t, ri);

    float acc[8][TN];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            // forward: the reference starts each sum from the bias
            const int64_t n = n0 + tx * 4 + (j & 3) + (j >> 2) * 64;
            acc[i][j] = (KIND == kFwd && p.bias && n < p.Ncol) ? __ldg(p.bias + n) : 0.f;
        }

    float ra[4] = {}, rb[NB] = {};
    const int ktiles = (p.K + BK - 1) / BK;
    auto stage = [&](int buf) {
        *reinterpret_cast<float4*>(&As[buf][t >> 5][(t & 31) * 4]) = make_float4(ra[0], ra[1], ra[2], ra[3]);
#pragma unroll
        for (int i = 0; i < NB; ++i) Bs[buf][(t % GROUPS) * NB + i][t / GROUPS] = rb[i];
    };
    if (ktiles > 0) {
        load_a<KIND>(p, ri, img, 0, t, ra);
        load_b<KIND, BN>(p, img, n0, 0, t, rb);
        stage(0);
    }
    __syncthreads();
    for (int kt = 0; kt < ktiles; ++kt) {
        const int cur = kt & 1;
        const bool more = kt + 1 < ktiles;
        if (more) {
            load_a<KIND>(p, ri, img, (kt + 1) * BK, t, ra);
            load_b<KIND, BN>(p, img, n0, (kt + 1) * BK, t, rb);
        }
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4 + 64]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            float bv[TN];
#pragma unroll
            for (int h = 0; h < TN / 4; ++h) {
                const float4 b = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4 + h * 64]);
                bv[4 * h] = b.x; bv[4 * h + 1] = b.y; bv[4 * h + 2] = b.z; bv[4 * h + 3] = b.w;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
        }
        if (more) stage(cur ^ 1);
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t m = m0 + ty * 4 + (i & 3) + (i >> 2) * 64;
        if (m >= p.M) continue;
        if (KIND == kWgrad) {
            float* row = p.out + ((int64_t)img * p.M + m) * p.Ncol;
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const int64_t n = n0 + tx * 4 + (j & 3) + (j >> 2) * 64;
                if (n < p.Ncol) row[n] = acc[i][j];
            }
        } else {
            // m -> (image, row, column) of y (fwd) or dx (dgrad); n = output channel
            const int oh = KIND == kFwd ? p.Ho : p.H, ow = KIND == kFwd ? p.Wo : p.W;
            const int64_t hw = (int64_t)oh * ow;
            const int nn = (int)(m / hw);
            const int rem = (int)(m - (int64_t)nn * hw);
            const int yy = rem / ow, xx = rem - yy * ow;
            float* o = p.out + (int64_t)nn * p.so[0] + (int64_t)yy * p.so[2] + (int64_t)xx * p.so[3];
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const int64_t n = n0 + tx * 4 + (j & 3) + (j >> 2) * 64;
                if (n < p.Ncol) o[n * p.so[1]] = acc[i][j];
            }
        }
    }
}

// dW[co][j] = ((0 + part[0][j][co]) + part[1][j][co]) + ... over the images in order, j =
// (ci, r, s): the reference adds each image's sum into the zeroed gradient in turn.
__global__ void wgrad_sum_kernel(const float* __restrict__ part, int images, int J, int Co, float* __restrict__ dw) {
    const int64_t total = (int64_t)J * Co;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int co = (int)(i / J), j = (int)(i - (int64_t)co * J);
        float s = 0.f;
        for (int n = 0; n < images; ++n) s += part[((int64_t)n * J + j) * Co + co];
        dw[i] = s;
    }
}

}  // namespace convs
}  // namespace mt
