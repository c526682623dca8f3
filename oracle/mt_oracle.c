/*
 * mt_oracle.c -- CPU oracle (test infrastructure only; see mt_oracle.h).
 *
 * Plain-C restatement of the reference CPU routines on the fp32 GEMM path. The loop
 * nests and the order of every fp32 addition follow the cited reference lines so the
 * results are bit-identical to the reference's own CPU build. Build with
 * -O2 -ffp-contract=off (oracle/Makefile).
 */
#include "mt_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* include/TensorOps.hpp:139-160 -- i, j, then k ascending; `sum` starts at 0. */
void orc_matmul(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N) {
    for (int64_t i = 0; i < M; ++i) {
        for (int64_t j = 0; j < N; ++j) {
            float sum = 0.0f;
            for (int64_t k = 0; k < K; ++k) sum += A[i * K + k] * B[k * N + j];
            C[i * N + j] = sum;
        }
    }
}

/* include/TensorOps.hpp:162-189 -- same loop nest with explicit strides. */
void orc_matmul_strided(const float* A, int64_t sa_m, int64_t sa_k,
                        const float* B, int64_t sb_k, int64_t sb_n,
                        float* C, int64_t sc_m, int64_t sc_n,
                        int64_t M, int64_t K, int64_t N) {
    for (int64_t i = 0; i < M; ++i) {
        for (int64_t j = 0; j < N; ++j) {
            float sum = 0.0f;
            for (int64_t k = 0; k < K; ++k) {
                float a = A[i * sa_m + k * sa_k];
                float b = B[k * sb_k + j * sb_n];
                sum += a * b;
            }
            C[i * sc_m + j * sc_n] = sum;
        }
    }
}

typedef struct {
    const float *A, *B;
    float* C;
    int64_t K, N, r0, r1;
} rows_job;

static void* rows_worker(void* p) {
    rows_job* j = (rows_job*)p;
    for (int64_t i = j->r0; i < j->r1; ++i) {
        const float* a = j->A + i * j->K;
        for (int64_t c = 0; c < j->N; ++c) {
            float sum = 0.0f;
            for (int64_t k = 0; k < j->K; ++k) sum += a[k] * j->B[k * j->N + c];
            j->C[i * j->N + c] = sum;
        }
    }
    return NULL;
}

void orc_matmul_rows_mt(const float* A, const float* B, float* C,
                        int64_t M, int64_t K, int64_t N,
                        int64_t r0, int64_t r1, int threads) {
    (void)M;
    if (threads < 1) threads = 1;
    int64_t rows = r1 - r0;
    if (rows <= 0) return;
    if (threads > rows) threads = (int)rows;
    pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    rows_job* jobs = (rows_job*)calloc((size_t)threads, sizeof(rows_job));
    for (int t = 0; t < threads; ++t) {
        jobs[t].A = A; jobs[t].B = B; jobs[t].C = C; jobs[t].K = K; jobs[t].N = N;
        jobs[t].r0 = r0 + rows * t / threads;
        jobs[t].r1 = r0 + rows * (t + 1) / threads;
        pthread_create(&tid[t], NULL, rows_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
}

/* include/TensorOps.hpp:933-991 -- the CPU branch makes both operands contiguous
 * (a value-preserving copy) and calls matmul_cpu on per-batch 2-D slices, so each
 * batch is the matmul_cpu loop over the (possibly broadcast) operands. */
void orc_bmm(const float* A, int64_t sa_b, int64_t sa_m, int64_t sa_k,
             const float* B, int64_t sb_b, int64_t sb_k, int64_t sb_n,
             float* C, int64_t batch, int64_t M, int64_t K, int64_t N) {
    for (int64_t b = 0; b < batch; ++b)
        orc_matmul_strided(A + b * sa_b, sa_m, sa_k, B + b * sb_b, sb_k, sb_n,
                           C + b * M * N, N, 1, M, K, N);
}

/* include/Module.hpp:112-114 -- matmul first, then a separate elementwise add of the
 * [1,out] bias broadcast over rows. */
void orc_linear_fwd(const float* X, const float* W, const float* bias, float* Y,
                    int64_t M, int64_t K, int64_t N) {
    orc_matmul(X, W, Y, M, K, N);
    if (bias)
        for (int64_t i = 0; i < M; ++i)
            for (int64_t j = 0; j < N; ++j) Y[i * N + j] = Y[i * N + j] + bias[j];
}

/* include/TensorOps.hpp:17-20 */
int64_t orc_conv_out_size(int64_t in, int64_t pad, int64_t k, int64_t stride) {
    if (in + 2 * pad < k) return 0;
    return (in + 2 * pad - k) / stride + 1;
}

typedef struct {
    const float *x, *w, *bias;
    float* y;
    int64_t N, C, H, W, Cout, kH, kW, stride, pad, Ho, Wo;
    int64_t n0, n1;   /* batch range (fwd) or c_out range (wgrad) */
} conv_job;

/* include/TensorOps.hpp:235-273 -- per output: start from bias, then c_in, r, s. */
static void conv_fwd_range(const conv_job* j) {
    for (int64_t n = j->n0; n < j->n1; ++n)
        for (int64_t co = 0; co < j->Cout; ++co)
            for (int64_t y = 0; y < j->Ho; ++y)
                for (int64_t x = 0; x < j->Wo; ++x) {
                    float val = j->bias ? j->bias[co] : 0.0f;
                    for (int64_t ci = 0; ci < j->C; ++ci)
                        for (int64_t r = 0; r < j->kH; ++r)
                            for (int64_t s = 0; s < j->kW; ++s) {
                                int64_t iy = y * j->stride + r - j->pad;
                                int64_t ix = x * j->stride + s - j->pad;
                                if (iy >= 0 && iy < j->H && ix >= 0 && ix < j->W) {
                                    int64_t in_idx = n * (j->C * j->H * j->W) + ci * (j->H * j->W) + iy * j->W + ix;
                                    int64_t w_idx = co * (j->C * j->kH * j->kW) + ci * (j->kH * j->kW) + r * j->kW + s;
                                    val += j->x[in_idx] * j->w[w_idx];
                                }
                            }
                    j->y[n * (j->Cout * j->Ho * j->Wo) + co * (j->Ho * j->Wo) + y * j->Wo + x] = val;
                }
}

static void* conv_fwd_worker(void* p) { conv_fwd_range((conv_job*)p); return NULL; }

/* include/TensorOps.hpp:358-396 -- gw zero-filled; for n, c_out, c_in, r, s: a spatial
 * partial `sum` over (y, x) is added into gw. Threads split c_out (disjoint gw rows), so
 * each element still sees the n-ascending order of the reference. */
static void conv_wgrad_range(const conv_job* j) {
    const float* go = j->w;   /* dy stored in the w slot for this job type */
    for (int64_t n = 0; n < j->N; ++n)
        for (int64_t co = j->n0; co < j->n1; ++co)
            for (int64_t ci = 0; ci < j->C; ++ci)
                for (int64_t r = 0; r < j->kH; ++r)
                    for (int64_t s = 0; s < j->kW; ++s) {
                        float sum = 0.0f;
                        for (int64_t y = 0; y < j->Ho; ++y)
                            for (int64_t x = 0; x < j->Wo; ++x) {
                                int64_t iy = y * j->stride + r - j->pad;
                                int64_t ix = x * j->stride + s - j->pad;
                                if (iy >= 0 && iy < j->H && ix >= 0 && ix < j->W) {
                                    int64_t in_idx = n * (j->C * j->H * j->W) + ci * (j->H * j->W) + iy * j->W + ix;
                                    int64_t go_idx = n * (j->Cout * j->Ho * j->Wo) + co * (j->Ho * j->Wo) + y * j->Wo + x;
                                    sum += j->x[in_idx] * go[go_idx];
                                }
                            }
                        int64_t w_idx = co * (j->C * j->kH * j->kW) + ci * (j->kH * j->kW) + r * j->kW + s;
                        j->y[w_idx] += sum;
                    }
}

static void* conv_wgrad_worker(void* p) { conv_wgrad_range((conv_job*)p); return NULL; }

static void run_split(conv_job base, int64_t total, int threads, void* (*fn)(void*)) {
    if (threads < 1) threads = 1;
    if (threads > total) threads = (int)(total > 0 ? total : 1);
    pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    conv_job* jobs = (conv_job*)calloc((size_t)threads, sizeof(conv_job));
    for (int t = 0; t < threads; ++t) {
        jobs[t] = base;
        jobs[t].n0 = total * t / threads;
        jobs[t].n1 = total * (t + 1) / threads;
        pthread_create(&tid[t], NULL, fn, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
}

void orc_conv2d_fwd(const float* x, const float* w, const float* bias, float* y,
                    int64_t N, int64_t C, int64_t H, int64_t W,
                    int64_t Cout, int64_t kH, int64_t kW,
                    int64_t stride, int64_t pad, int threads) {
    conv_job j;
    memset(&j, 0, sizeof j);
    j.x = x; j.w = w; j.bias = bias; j.y = y;
    j.N = N; j.C = C; j.H = H; j.W = W; j.Cout = Cout; j.kH = kH; j.kW = kW;
    j.stride = stride; j.pad = pad;
    j.Ho = orc_conv_out_size(H, pad, kH, stride);
    j.Wo = orc_conv_out_size(W, pad, kW, stride);
    run_split(j, N, threads, conv_fwd_worker);
}

/* include/TensorOps.hpp:319-356 -- gi zero-filled, then scatter-add in the order
 * n, c_out, y, x, c_in, r, s. Images are independent, so threads split n without
 * changing the order of additions into any element. */
static void conv_dgrad_range(const conv_job* j) {
    const float* dy = j->x;   /* dy stored in the x slot for this job type */
    const float* w = j->w;
    float* dx = j->y;
    int64_t C = j->C, H = j->H, W = j->W, Cout = j->Cout, kH = j->kH, kW = j->kW;
    int64_t stride = j->stride, pad = j->pad, Ho = j->Ho, Wo = j->Wo;
    for (int64_t n = j->n0; n < j->n1; ++n)
        for (int64_t co = 0; co < Cout; ++co)
            for (int64_t y = 0; y < Ho; ++y)
                for (int64_t x = 0; x < Wo; ++x) {
                    float g = dy[n * (Cout * Ho * Wo) + co * (Ho * Wo) + y * Wo + x];
                    for (int64_t ci = 0; ci < C; ++ci)
                        for (int64_t r = 0; r < kH; ++r)
                            for (int64_t s = 0; s < kW; ++s) {
                                int64_t iy = y * stride + r - pad;
                                int64_t ix = x * stride + s - pad;
                                if (iy >= 0 && iy < H && ix >= 0 && ix < W) {
                                    int64_t in_idx = n * (C * H * W) + ci * (H * W) + iy * W + ix;
                                    int64_t w_idx = co * (C * kH * kW) + ci * (kH * kW) + r * kW + s;
                                    dx[in_idx] += g * w[w_idx];
                                }
                            }
                }
}

static void* conv_dgrad_worker(void* p) { conv_dgrad_range((conv_job*)p); return NULL; }

void orc_conv2d_bwd_weight(const float* dy, const float* x, float* dw,
                           int64_t N, int64_t C, int64_t H, int64_t W,
                           int64_t Cout, int64_t kH, int64_t kW,
                           int64_t stride, int64_t pad, int threads) {
    conv_job j;
    memset(&j, 0, sizeof j);
    j.x = x; j.w = dy; j.y = dw;
    j.N = N; j.C = C; j.H = H; j.W = W; j.Cout = Cout; j.kH = kH; j.kW = kW;
    j.stride = stride; j.pad = pad;
    j.Ho = orc_conv_out_size(H, pad, kH, stride);
    j.Wo = orc_conv_out_size(W, pad, kW, stride);
    memset(dw, 0, (size_t)(Cout * C * kH * kW) * sizeof(float));
    run_split(j, Cout, threads, conv_wgrad_worker);
}

/* include/TensorOps.hpp:398-418 -- gb zero-filled; per n a spatial partial sum. */
void orc_conv2d_bwd_bias(const float* dy, float* db,
                         int64_t N, int64_t Cout, int64_t Hout, int64_t Wout) {
    for (int64_t c = 0; c < Cout; ++c) db[c] = 0.0f;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t c = 0; c < Cout; ++c) {
            float sum = 0.0f;
            for (int64_t y = 0; y < Hout; ++y)
                for (int64_t x = 0; x < Wout; ++x)
                    sum += dy[n * (Cout * Hout * Wout) + c * (Hout * Wout) + y * Wout + x];
            db[c] += sum;
        }
}

void orc_conv2d_bwd_input(const float* dy, const float* w, float* dx,
                          int64_t N, int64_t C, int64_t H, int64_t W,
                          int64_t Cout, int64_t kH, int64_t kW,
                          int64_t stride, int64_t pad, int threads) {
    conv_job j;
    memset(&j, 0, sizeof j);
    j.x = dy; j.w = w; j.y = dx;
    j.N = N; j.C = C; j.H = H; j.W = W; j.Cout = Cout; j.kH = kH; j.kW = kW;
    j.stride = stride; j.pad = pad;
    j.Ho = orc_conv_out_size(H, pad, kH, stride);
    j.Wo = orc_conv_out_size(W, pad, kW, stride);
    memset(dx, 0, (size_t)(N * C * H * W) * sizeof(float));
    run_split(j, N, threads, conv_dgrad_worker);
}
