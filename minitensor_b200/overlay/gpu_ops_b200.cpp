// gpu_ops_b200.cpp -- drop-in definitions of miniTensor's GPU GEMM/conv entry points
// (include/TensorOps.hpp:703-712, T = float) on top of libmtgemm.so.
//
// Build this translation unit with the reference headers on the include path and
// -DUSE_CUDA, link libmtgemm.so, and leave the reference's own definitions of these
// symbols out of the link (src/gpu_ops.cpp defines them at :1103-1223, :2237-2741; the
// other kernels of that file -- elementwise, reductions, BN, pooling, ... -- stay).
// Every function maps the reference's Tensor view to an mt_tensor (storage pointer, view
// offset, shape, strides), launches on the reference's active_stream() and turns a
// status into the reference's error behaviour: std::invalid_argument for argument errors
// (as its dispatchers throw), std::runtime_error after printing the message for CUDA
// failures (as GPU_CHECK does, include/GpuUtils.hpp:10-18).
//
// Also registers the engine in the reference's (otherwise unused) OpRegistry<float>
// under OpType::Matmul and OpType::Conv2D (include/Dispatch.hpp:12-58), and hands the
// engine's scratch allocations to the reference's MemoryPool.
#include <iostream>
#include <stdexcept>
#include <type_traits>

#include "Dispatch.hpp"
#include "GpuUtils.hpp"
#include "MemoryPool.hpp"
#include "Tensor.hpp"
#include "TensorOps.hpp"
#include "mtgemm.h"

namespace {

template <typename T>
mt_tensor to_mt(const Tensor<T>& t) {
    static_assert(std::is_same_v<T, float>, "libmtgemm serves float tensors");
    mt_tensor v{};
    if (t.empty()) return v;
    v.data = const_cast<float*>(t.data());
    v.offset = t.offset();
    v.ndim = static_cast<uint32_t>(t.shape().size());
    if (v.ndim > MT_MAX_DIMS) throw std::runtime_error("Exceeded MAX_DIMS");
    for (uint32_t i = 0; i < v.ndim; ++i) {
        v.shape[i] = t.shape()[i];
        v.strides[i] = t.strides()[i];
    }
    return v;
}

void check(int rc) {
    if (rc == MT_OK) return;
    const char* msg = mt_last_error();
    if (rc == MT_EINVAL) throw std::invalid_argument(msg);
    std::cerr << "libmtgemm error " << rc << ": " << msg << std::endl;
    throw std::runtime_error(msg);
}

void* stream() { return static_cast<void*>(active_stream()); }

}  // namespace

// ---- include/TensorOps.hpp:703-706 --------------------------------------------------
template <typename T>
void matmul_gpu(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C) {
    mt_tensor a = to_mt(A), b = to_mt(B), c = to_mt(C);
    check(mt_matmul_gpu(&a, &b, &c, stream()));
}
template <typename T>
void matmul_gpu_strided(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C) {
    mt_tensor a = to_mt(A), b = to_mt(B), c = to_mt(C);
    check(mt_matmul_gpu_strided(&a, &b, &c, stream()));
}
template <typename T>
void matmul_gpu_v2(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C) {
    mt_tensor a = to_mt(A), b = to_mt(B), c = to_mt(C);
    check(mt_matmul_gpu_v2(&a, &b, &c, stream()));
}
template <typename T>
void matmul_gpu_bk16(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C) {
    mt_tensor a = to_mt(A), b = to_mt(B), c = to_mt(C);
    check(mt_matmul_gpu_bk16(&a, &b, &c, stream()));
}

// ---- include/TensorOps.hpp:708-712 --------------------------------------------------
template <typename T>
void conv2d_gpu(const Tensor<T>& input, const Tensor<T>& weight, const Tensor<T>& bias, Tensor<T>& output,
                size_t stride, size_t padding) {
    mt_tensor x = to_mt(input), w = to_mt(weight), b = to_mt(bias), y = to_mt(output);
    check(mt_conv2d_gpu(&x, &w, bias.empty() ? nullptr : &b, &y, stride, padding, stream()));
}
template <typename T>
void conv2d_gpu_strided(const Tensor<T>& input, const Tensor<T>& weight, const Tensor<T>& bias, Tensor<T>& output,
                        size_t stride, size_t padding) {
    mt_tensor x = to_mt(input), w = to_mt(weight), b = to_mt(bias), y = to_mt(output);
    check(mt_conv2d_gpu_strided(&x, &w, bias.empty() ? nullptr : &b, &y, stride, padding, stream()));
}
template <typename T>
void conv2d_backward_input_gpu(const Tensor<T>& grad_output, const Tensor<T>& weight, Tensor<T>& grad_input,
                               size_t stride, size_t padding) {
    mt_tensor dy = to_mt(grad_output), w = to_mt(weight), dx = to_mt(grad_input);
    check(mt_conv2d_backward_input_gpu(&dy, &w, &dx, stride, padding, stream()));
}
template <typename T>
void conv2d_backward_weight_gpu(const Tensor<T>& grad_output, const Tensor<T>& input, Tensor<T>& grad_weight,
                                size_t stride, size_t padding) {
    mt_tensor dy = to_mt(grad_output), x = to_mt(input), dw = to_mt(grad_weight);
    check(mt_conv2d_backward_weight_gpu(&dy, &x, &dw, stride, padding, stream()));
}
template <typename T>
void conv2d_backward_bias_gpu(const Tensor<T>& grad_output, Tensor<T>& grad_bias) {
    mt_tensor dy = to_mt(grad_output), db = to_mt(grad_bias);
    check(mt_conv2d_backward_bias_gpu(&dy, &db, stream()));
}

// Explicit instantiations for float: the same set src/gpu_ops.cpp provides.
template void matmul_gpu<float>(const Tensor<float>&, const Tensor<float>&, Tensor<float>&);
template void matmul_gpu_strided<float>(const Tensor<float>&, const Tensor<float>&, Tensor<float>&);
template void matmul_gpu_v2<float>(const Tensor<float>&, const Tensor<float>&, Tensor<float>&);
template void matmul_gpu_bk16<float>(const Tensor<float>&, const Tensor<float>&, Tensor<float>&);
template void conv2d_gpu<float>(const Tensor<float>&, const Tensor<float>&, const Tensor<float>&, Tensor<float>&,
                                size_t, size_t);
template void conv2d_gpu_strided<float>(const Tensor<float>&, const Tensor<float>&, const Tensor<float>&,
                                        Tensor<float>&, size_t, size_t);
template void conv2d_backward_input_gpu<float>(const Tensor<float>&, const Tensor<float>&, Tensor<float>&, size_t,
                                               size_t);
template void conv2d_backward_weight_gpu<float>(const Tensor<float>&, const Tensor<float>&, Tensor<float>&, size_t,
                                                size_t);
template void conv2d_backward_bias_gpu<float>(const Tensor<float>&, Tensor<float>&);

// ---- batched / fused entry points the reference has no GPU form of -------------------

// One-launch bmm (replaces the per-batch loop of include/TensorOps.hpp:933-991, whose
// GPU branch drops view offsets): operands stay views, a stride-0 batch is a broadcast.
Tensor<float> mt_bmm(const Tensor<float>& A, const Tensor<float>& B) {
    if (A.device() != B.device()) throw std::invalid_argument("Tensors must be on the same device for bmm.");
    if (A.shape().size() != 3 || B.shape().size() != 3) throw std::invalid_argument("bmm requires 3D tensors.");
    if (A.shape()[0] != B.shape()[0]) throw std::invalid_argument("bmm: batch dimension mismatch.");
    if (A.shape()[2] != B.shape()[1]) throw std::invalid_argument("bmm: inner dimension mismatch (A.K != B.K).");
    Tensor<float> C({A.shape()[0], A.shape()[1], B.shape()[2]}, A.device());
    mt_tensor a = to_mt(A), b = to_mt(B), c = to_mt(C);
    check(mt_bmm_gpu(&a, &b, &c, stream()));
    return C;
}

// Linear forward with the bias add (and optional ReLU) in the GEMM epilogue
// (include/Module.hpp:112-114 does matmul then a separate broadcast add).
Tensor<float> mt_linear_forward(const Tensor<float>& x, const Tensor<float>& W, const Tensor<float>& bias,
                                bool relu) {
    Tensor<float> y({x.shape()[0], W.shape()[1]}, x.device());
    mt_tensor xv = to_mt(x), wv = to_mt(W), bv = to_mt(bias), yv = to_mt(y);
    check(mt_linear_fwd_gpu(&xv, &wv, bias.empty() ? nullptr : &bv, &yv, relu ? 1 : 0, stream()));
    return y;
}

// ---- scratch from the reference's MemoryPool (include/MemoryPool.hpp:45-99) -----------
// The reference's GPU routines take their temporary buffers from MemoryPool::get() and
// return them right after enqueuing their kernels on active_stream(); the engine's scratch
// (split-K / stream-K partials, conv NHWC copies, weight-grad partials) now does the same,
// so a captured step (GraphExecutor) holds no allocation node of this library and reuses
// the pool's cached blocks on every replay.
namespace {
void* pool_alloc(size_t bytes, int device, void*) {
    try {
        return MemoryPool::get().allocate(bytes, Device{DeviceType::CUDA, static_cast<uint8_t>(device)});
    } catch (const std::exception& e) {
        std::cerr << "MemoryPool: " << e.what() << std::endl;
        return nullptr;
    }
}
void pool_free(void* ptr, size_t bytes, int device, void*) {
    MemoryPool::get().free(ptr, bytes, Device{DeviceType::CUDA, static_cast<uint8_t>(device)});
}
struct InstallPool {
    InstallPool() { mt_set_scratch_allocator(pool_alloc, pool_free, nullptr); }
} install_pool;
}  // namespace

// ---- OpRegistry registrations (include/Dispatch.hpp:50-58) ----------------------------
namespace {
AutoRegistrar<float> reg_matmul(OpType::Matmul, BinaryOpFn<float>([](const Tensor<float>& a, const Tensor<float>& b,
                                                                      Tensor<float>& c) { matmul_gpu_strided(a, b, c); }));
// Conv2D through the binary slot: stride 1, padding inferred from the output height
// (H_out = H + 2p - kh + 1), no bias.
AutoRegistrar<float> reg_conv(OpType::Conv2D, BinaryOpFn<float>([](const Tensor<float>& x, const Tensor<float>& w,
                                                                    Tensor<float>& y) {
    const size_t pad = (y.shape()[2] + w.shape()[2] - 1 - x.shape()[2]) / 2;
    conv2d_gpu_strided(x, w, Tensor<float>(), y, 1, pad);
}));
}  // namespace
