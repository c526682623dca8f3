// ref_gpu.cpp -- extern "C" shim that times the reference's OWN GPU kernels on this GPU
// (the same-hardware baseline; not part of the product, and not a parity oracle).
//
// This file is ours and contains no reference source. It #includes the reference headers
// unmodified and calls the reference's GPU entry points, whose definitions come from the
// reference's src/gpu_ops.cpp compiled unmodified for sm_100a (minitensor_b200.build
// .build_refgpu). Tensors are built the way the reference's own test/benchmark.cpp builds
// them: a CPU Tensor filled on the host, then .to(CUDA) through the reference's
// MemoryPool. Timing: cudaEvents on the legacy default stream (the reference's
// active_stream() when none is set), around `iters` back-to-back calls after `warmup`
// calls, then one device synchronize.
//
// Kernels reached (file:line in the reference):
//   matmul_gpu            -> sgemm_kernel_v2<128,128,16,4,4>  src/gpu_ops.cpp:932-1101, :1103-1144
//   matmul_gpu_strided    -> matmul_kernel_strided            src/gpu_ops.cpp:909-930, :1199-1223
//   conv2d_gpu            -> im2col + batched_sgemm_kernel_v2 src/gpu_ops.cpp:2237-2325
//   conv2d_backward_weight_gpu                                src/gpu_ops.cpp:2623-2713
// Every function returns 0 on success, 1 if the reference threw (message in ref_gpu_error).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <functional>
#include <string>
#include <vector>

#include "Tensor.hpp"
#include "TensorOps.hpp"

namespace {

thread_local std::string g_err;

Tensor<float> to_gpu(const float* src, std::vector<size_t> shape) {
    Tensor<float> cpu(shape, Device{DeviceType::CPU});
    std::memcpy(cpu.data(), src, cpu.total_elements() * sizeof(float));
    return cpu.to(Device{DeviceType::CUDA});
}

Tensor<float> gpu_empty(std::vector<size_t> shape) { return Tensor<float>(shape, Device{DeviceType::CUDA}); }

void to_host(const Tensor<float>& t, float* dst) {
    Tensor<float> h = t.to(Device{DeviceType::CPU});
    std::memcpy(dst, h.data() + h.offset(), h.total_elements() * sizeof(float));
}

// ms per call of fn over `iters` calls, after `warmup` calls.
float time_calls(const std::function<void()>& fn, int warmup, int iters) {
    for (int i = 0; i < warmup; ++i) fn();
    cudaDeviceSynchronize();
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, nullptr);
    for (int i = 0; i < iters; ++i) fn();
    cudaEventRecord(b, nullptr);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA: ") + cudaGetErrorString(e));
    return ms / (float)(iters > 0 ? iters : 1);
}

}  // namespace

extern "C" {

const char* ref_gpu_error(void) { return g_err.c_str(); }

// C = A . B by the reference's matmul_gpu (sgemm_kernel_v2 for M,N >= 64).
int ref_gpu_matmul(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N, int warmup,
                   int iters, float* ms) {
    try {
        Tensor<float> a = to_gpu(A, {(size_t)M, (size_t)K});
        Tensor<float> b = to_gpu(B, {(size_t)K, (size_t)N});
        Tensor<float> c = gpu_empty({(size_t)M, (size_t)N});
        *ms = time_calls([&] { matmul_gpu<float>(a, b, c); }, warmup, iters);
        if (C) to_host(c, C);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return 1; }
}

// The Linear step of configuration 2 as the reference's GPU path runs it: Y = X . W
// (matmul_gpu), dX = dY . W^T and dW = X^T . dY on transposed views (matmul_gpu_strided,
// which MatmulBackward reaches through matmul()'s non-contiguous branch).
int ref_gpu_linear_step(const float* X, const float* W, const float* dY, float* Y, float* dX, float* dW, int64_t M,
                        int64_t K, int64_t N, int warmup, int iters, float* ms) {
    try {
        Tensor<float> x = to_gpu(X, {(size_t)M, (size_t)K});
        Tensor<float> w = to_gpu(W, {(size_t)K, (size_t)N});
        Tensor<float> dy = to_gpu(dY, {(size_t)M, (size_t)N});
        Tensor<float> y = gpu_empty({(size_t)M, (size_t)N});
        Tensor<float> dx = gpu_empty({(size_t)M, (size_t)K});
        Tensor<float> dw = gpu_empty({(size_t)K, (size_t)N});
        Tensor<float> wt = w.transpose(0, 1), xt = x.transpose(0, 1);
        *ms = time_calls([&] {
            matmul_gpu<float>(x, w, y);
            matmul_gpu_strided<float>(dy, wt, dx);
            matmul_gpu_strided<float>(xt, dy, dw);
        }, warmup, iters);
        if (Y) to_host(y, Y);
        if (dX) to_host(dx, dX);
        if (dW) to_host(dw, dW);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return 1; }
}

// The broadcast bmm of configuration 3 as the reference composes it (include/TensorOps.hpp
// :933-991): B0 [1,K,N] expanded to the batch and made contiguous, then one matmul_gpu per
// batch on slices. matmul_gpu ignores the slices' offsets (src/gpu_ops.cpp:1125-1127), so
// every batch reads batch 0: the output is wrong for batch > 0 and is returned only for
// inspection.
int ref_gpu_bmm_bcast(const float* A, const float* B0, float* C, int64_t bt, int64_t M, int64_t K, int64_t N,
                      int warmup, int iters, float* ms) {
    try {
        Tensor<float> a = to_gpu(A, {(size_t)bt, (size_t)M, (size_t)K});
        Tensor<float> b0 = to_gpu(B0, {1, (size_t)K, (size_t)N});
        Tensor<float> c = gpu_empty({(size_t)bt, (size_t)M, (size_t)N});
        *ms = time_calls([&] {
            Tensor<float> bc = b0.expand({(size_t)bt, (size_t)K, (size_t)N}).contiguous();
            for (int64_t i = 0; i < bt; ++i) {
                Tensor<float> ai = a.slice(0, (size_t)i, (size_t)i + 1).reshape({(size_t)M, (size_t)K});
                Tensor<float> bi = bc.slice(0, (size_t)i, (size_t)i + 1).reshape({(size_t)K, (size_t)N});
                Tensor<float> ci = c.slice(0, (size_t)i, (size_t)i + 1).reshape({(size_t)M, (size_t)N});
                matmul_gpu<float>(ai, bi, ci);
            }
        }, warmup, iters);
        if (C) to_host(c, C);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return 1; }
}

// Conv2D forward + weight gradient of configuration 4 by conv2d_gpu and
// conv2d_backward_weight_gpu (stride, padding as given).
int ref_gpu_conv_step(const float* x, const float* w, const float* bias, const float* dy, float* y, float* dw,
                      int64_t N, int64_t C, int64_t H, int64_t Wd, int64_t Co, int64_t k, int64_t stride,
                      int64_t pad, int warmup, int iters, float* ms) {
    try {
        const size_t Ho = (size_t)((H + 2 * pad - k) / stride + 1), Wo = (size_t)((Wd + 2 * pad - k) / stride + 1);
        Tensor<float> tx = to_gpu(x, {(size_t)N, (size_t)C, (size_t)H, (size_t)Wd});
        Tensor<float> tw = to_gpu(w, {(size_t)Co, (size_t)C, (size_t)k, (size_t)k});
        Tensor<float> tb = to_gpu(bias, {(size_t)Co});
        Tensor<float> tdy = to_gpu(dy, {(size_t)N, (size_t)Co, Ho, Wo});
        Tensor<float> ty = gpu_empty({(size_t)N, (size_t)Co, Ho, Wo});
        Tensor<float> tdw = gpu_empty({(size_t)Co, (size_t)C, (size_t)k, (size_t)k});
        *ms = time_calls([&] {
            conv2d_gpu<float>(tx, tw, tb, ty, (size_t)stride, (size_t)pad);
            conv2d_backward_weight_gpu<float>(tdy, tx, tdw, (size_t)stride, (size_t)pad);
        }, warmup, iters);
        if (y) to_host(ty, y);
        if (dw) to_host(tdw, dw);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return 1; }
}

}  // extern "C"
