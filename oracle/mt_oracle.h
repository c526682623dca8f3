/*
 * mt_oracle.h -- CPU oracle for the fp32 dense-contraction path of miniTensor.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA engine in
 * minitensor_b200/ is compared against. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs may load it. The product never links it.
 *
 * Every function restates one CPU routine of dionkadi/miniTensor in plain C, with the
 * same loop nest and the same fp32 accumulation order, so that for identical inputs it
 * returns bit-identical results to the reference's own CPU path (built with g++ -O2 for
 * x86-64, which does not contract a*b+c into an FMA; this file is built with
 * -ffp-contract=off for the same reason). The citation above each function names the
 * reference routine it follows (paths relative to the reference project root).
 *
 * Parity is pinned two ways (tests/test_oracle.py):
 *   - against the reference's own known-answer tests (test/tensor_test.cpp,
 *     test/engien_test.cpp, test/spatial_test.cpp), and
 *   - bit-exactly against golden vectors produced by the reference's own headers,
 *     compiled here from source (oracle/ref_cpu.cpp -> oracle/_ref/libref_cpu.so,
 *     fixtures in tests/golden/).
 */
#ifndef MT_ORACLE_H
#define MT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* include/TensorOps.hpp:139-160 matmul_cpu: C[M,N] = A[M,K] * B[K,N], row-major. */
void orc_matmul(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N);

/* include/TensorOps.hpp:162-189 matmul_cpu_strided: element strides per operand. */
void orc_matmul_strided(const float* A, int64_t sa_m, int64_t sa_k,
                        const float* B, int64_t sb_k, int64_t sb_n,
                        float* C, int64_t sc_m, int64_t sc_n,
                        int64_t M, int64_t K, int64_t N);

/* matmul_cpu over output rows [r0, r1) only, split over `threads` POSIX threads.
 * Each element is computed by exactly the loop of matmul_cpu, so the result is
 * bit-identical to the single-thread call (used to time/sample 8192^3). */
void orc_matmul_rows_mt(const float* A, const float* B, float* C,
                        int64_t M, int64_t K, int64_t N,
                        int64_t r0, int64_t r1, int threads);

/* include/TensorOps.hpp:933-991 bmm (CPU branch): contiguous() copies, then
 * matmul_cpu per batch. Batch stride 0 is a broadcast (expand) operand. */
void orc_bmm(const float* A, int64_t sa_b, int64_t sa_m, int64_t sa_k,
             const float* B, int64_t sb_b, int64_t sb_k, int64_t sb_n,
             float* C, int64_t batch, int64_t M, int64_t K, int64_t N);

/* include/Module.hpp:112-114 Linear::forward = matmul(x, W) + bias (broadcast add,
 * include/TensorOps.hpp dispatch_binary, one fp32 add per element). W is [in,out]. */
void orc_linear_fwd(const float* X, const float* W, const float* bias, float* Y,
                    int64_t M, int64_t K, int64_t N);

/* include/TensorOps.hpp:17-20 safe_out_size. */
int64_t orc_conv_out_size(int64_t in, int64_t pad, int64_t k, int64_t stride);

/* include/TensorOps.hpp:235-273 conv2d_cpu (NCHW, bias may be NULL). */
void orc_conv2d_fwd(const float* x, const float* w, const float* bias, float* y,
                    int64_t N, int64_t C, int64_t H, int64_t W,
                    int64_t Cout, int64_t kH, int64_t kW,
                    int64_t stride, int64_t pad, int threads);

/* include/TensorOps.hpp:319-356 conv2d_backward_input_cpu. */
void orc_conv2d_bwd_input(const float* dy, const float* w, float* dx,
                          int64_t N, int64_t C, int64_t H, int64_t W,
                          int64_t Cout, int64_t kH, int64_t kW,
                          int64_t stride, int64_t pad, int threads);

/* include/TensorOps.hpp:358-396 conv2d_backward_weight_cpu. */
void orc_conv2d_bwd_weight(const float* dy, const float* x, float* dw,
                           int64_t N, int64_t C, int64_t H, int64_t W,
                           int64_t Cout, int64_t kH, int64_t kW,
                           int64_t stride, int64_t pad, int threads);

/* include/TensorOps.hpp:398-418 conv2d_backward_bias_cpu. */
void orc_conv2d_bwd_bias(const float* dy, float* db,
                         int64_t N, int64_t Cout, int64_t Hout, int64_t Wout);

#ifdef __cplusplus
}
#endif
#endif
