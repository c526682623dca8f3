// ref_cpu.cpp -- extern "C" shim over the reference's OWN CPU code (test infrastructure).
//
// This file is ours; it contains no reference source. It #includes the reference
// headers unmodified (include/Tensor.hpp, include/TensorOps.hpp, include/Module.hpp)
// and calls the reference's own CPU routines, so that golden vectors and the timed
// "reference" CPU baseline come from the reference itself. Built by oracle/Makefile
// into oracle/_ref/libref_cpu.so (git-ignored, shipped with built artefacts).
//
// Only tests/ (golden-vector generation and oracle pinning) and bench.py's reference
// arm load the result.
#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <random>
#include <thread>
#include <vector>

#include "Tensor.hpp"
#include "TensorOps.hpp"
#include "Module.hpp"

namespace {

Tensor<float> from_host(const float* src, std::vector<size_t> shape) {
    Tensor<float> t(shape);
    std::memcpy(t.data(), src, t.total_elements() * sizeof(float));
    return t;
}

void to_host(const Tensor<float>& t, float* dst) {
    const float* p = t.data() + t.offset();
    std::memcpy(dst, p, t.total_elements() * sizeof(float));
}

}  // namespace

extern "C" {

// matmul() dispatcher, CPU branch (include/TensorOps.hpp:993-1045 -> matmul_cpu :139-160).
int ref_matmul(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N) {
    try {
        Tensor<float> a = from_host(A, {(size_t)M, (size_t)K});
        Tensor<float> b = from_host(B, {(size_t)K, (size_t)N});
        Tensor<float> c = matmul(a, b);
        to_host(c, C);
        return 0;
    } catch (const std::exception&) { return 1; }
}

// matmul() on transposed views, as MatmulBackward builds them
// (include/Autograd.hpp:131-141 -> matmul_cpu_strided :162-189).
//   ta: use A_store[K,M].transpose(0,1) as A;  tb: use B_store[N,K].transpose(0,1) as B.
int ref_matmul_t(const float* A_store, const float* B_store, float* C,
                 int64_t M, int64_t K, int64_t N, int ta, int tb) {
    try {
        Tensor<float> a = ta ? from_host(A_store, {(size_t)K, (size_t)M}).transpose(0, 1)
                             : from_host(A_store, {(size_t)M, (size_t)K});
        Tensor<float> b = tb ? from_host(B_store, {(size_t)N, (size_t)K}).transpose(0, 1)
                             : from_host(B_store, {(size_t)K, (size_t)N});
        Tensor<float> c = matmul(a, b);
        to_host(c, C);
        return 0;
    } catch (const std::exception&) { return 1; }
}

// matmul() on a row slice of A (a contiguous view with a non-zero offset,
// include/Tensor.hpp:52-74): C = A[r0:r1, :] * B.
int ref_matmul_rowslice(const float* A, const float* B, float* C,
                        int64_t M, int64_t K, int64_t N, int64_t r0, int64_t r1) {
    try {
        Tensor<float> a = from_host(A, {(size_t)M, (size_t)K}).slice(0, (size_t)r0, (size_t)r1);
        Tensor<float> b = from_host(B, {(size_t)K, (size_t)N});
        Tensor<float> c = matmul(a, b);
        to_host(c, C);
        return 0;
    } catch (const std::exception&) { return 1; }
}

// bmm (include/TensorOps.hpp:933-991). The reference's bmm<float> does not compile
// (it reads the private Tensor::impl_ at :962), so this composes the same steps from
// the reference's own pieces: expand -> contiguous -> per-batch 2-D views -> matmul_cpu.
// b_bcast: B holds one [K,N] matrix expanded (stride 0) over the batch.
int ref_bmm(const float* A, const float* B, float* C,
            int64_t batch, int64_t M, int64_t K, int64_t N, int b_bcast) {
    try {
        Tensor<float> a = from_host(A, {(size_t)batch, (size_t)M, (size_t)K});
        Tensor<float> b = b_bcast
            ? from_host(B, {1, (size_t)K, (size_t)N}).expand({(size_t)batch, (size_t)K, (size_t)N})
            : from_host(B, {(size_t)batch, (size_t)K, (size_t)N});
        Tensor<float> ac = a.contiguous();
        Tensor<float> bc = b.contiguous();
        Tensor<float> c({(size_t)batch, (size_t)M, (size_t)N});
        for (int64_t i = 0; i < batch; ++i) {
            Tensor<float> as = ac.slice(0, (size_t)i, (size_t)i + 1).reshape({(size_t)M, (size_t)K});
            Tensor<float> bs = bc.slice(0, (size_t)i, (size_t)i + 1).reshape({(size_t)K, (size_t)N});
            Tensor<float> cs = c.slice(0, (size_t)i, (size_t)i + 1).reshape({(size_t)M, (size_t)N});
            matmul_cpu(as, bs, cs);
        }
        to_host(c, C);
        return 0;
    } catch (const std::exception&) { return 1; }
}

// Linear<float> forward (include/Module.hpp:112-114) and the two backward GEMMs of
// MatmulBackward (include/Autograd.hpp:124-141) with an explicit upstream gradient.
// W is the reference's [in,out] weight. Any of Y, dX, dW may be null.
int ref_linear(const float* X, const float* W, const float* bias, const float* dY,
               float* Y, float* dX, float* dW, int64_t M, int64_t K, int64_t N) {
    try {
        Linear<float> lin((size_t)K, (size_t)N);
        std::memcpy(lin.weight_.data(), W, (size_t)(K * N) * sizeof(float));
        if (bias) std::memcpy(lin.bias_.data(), bias, (size_t)N * sizeof(float));
        else lin.bias_.fill(0.0f);
        Tensor<float> x = from_host(X, {(size_t)M, (size_t)K});
        x.set_requires_grad(true);
        if (Y) to_host(lin.forward(x), Y);
        if (dY && (dX || dW)) {
            Tensor<float> mm = matmul(x, lin.weight_);
            Tensor<float> g = from_host(dY, {(size_t)M, (size_t)N});
            mm.grad_fn()->apply(g);
            if (dX) to_host(x.grad(), dX);
            if (dW) to_host(lin.weight_.grad(), dW);
        }
        return 0;
    } catch (const std::exception&) { return 1; }
}

// conv2d() dispatcher CPU branch (include/TensorOps.hpp:1076-1110 -> conv2d_cpu :235-273).
int ref_conv2d(const float* x, const float* w, const float* bias, float* y,
               int64_t N, int64_t C, int64_t H, int64_t W, int64_t Cout, int64_t kH, int64_t kW,
               int64_t stride, int64_t pad) {
    try {
        Tensor<float> xt = from_host(x, {(size_t)N, (size_t)C, (size_t)H, (size_t)W});
        Tensor<float> wt = from_host(w, {(size_t)Cout, (size_t)C, (size_t)kH, (size_t)kW});
        Tensor<float> bt = bias ? from_host(bias, {(size_t)Cout}) : Tensor<float>();
        Tensor<float> yt = conv2d(xt, wt, bt, (size_t)stride, (size_t)pad);
        to_host(yt, y);
        return 0;
    } catch (const std::exception&) { return 1; }
}

// conv2d_backward_{input,weight,bias} dispatchers (include/TensorOps.hpp:1112-1149).
int ref_conv2d_backward(const float* dy, const float* x, const float* w,
                        float* dx, float* dw, float* db,
                        int64_t N, int64_t C, int64_t H, int64_t W, int64_t Cout,
                        int64_t kH, int64_t kW, int64_t stride, int64_t pad) {
    try {
        size_t Ho = safe_out_size((size_t)H, (size_t)pad, (size_t)kH, (size_t)stride);
        size_t Wo = safe_out_size((size_t)W, (size_t)pad, (size_t)kW, (size_t)stride);
        Tensor<float> go = from_host(dy, {(size_t)N, (size_t)Cout, Ho, Wo});
        if (dx) {
            Tensor<float> wt = from_host(w, {(size_t)Cout, (size_t)C, (size_t)kH, (size_t)kW});
            Tensor<float> gi({(size_t)N, (size_t)C, (size_t)H, (size_t)W});
            conv2d_backward_input(go, wt, gi, (size_t)stride, (size_t)pad);
            to_host(gi, dx);
        }
        if (dw) {
            Tensor<float> xt = from_host(x, {(size_t)N, (size_t)C, (size_t)H, (size_t)W});
            Tensor<float> gw({(size_t)Cout, (size_t)C, (size_t)kH, (size_t)kW});
            conv2d_backward_weight(go, xt, gw, (size_t)stride, (size_t)pad);
            to_host(gw, dw);
        }
        if (db) {
            Tensor<float> gb({(size_t)Cout});
            conv2d_backward_bias(go, gb);
            to_host(gb, db);
        }
        return 0;
    } catch (const std::exception&) { return 1; }
}

// The reference CPU matmul over output rows [r0, r1), one std::thread per block of
// rows. Each thread calls the reference's matmul_cpu on a row slice of A
// (include/Tensor.hpp:52-74 slice keeps the storage and advances the offset), which
// gives per-element results identical to one matmul_cpu call over all rows.
// *seconds (optional) receives the wall time of the threaded matmul_cpu calls alone,
// without the copies of A and B into reference Tensors.
int ref_matmul_rows_mt(const float* A, const float* B, float* C,
                       int64_t M, int64_t K, int64_t N, int64_t r0, int64_t r1, int threads,
                       double* seconds) {
    try {
        Tensor<float> a = from_host(A, {(size_t)M, (size_t)K});
        Tensor<float> b = from_host(B, {(size_t)K, (size_t)N});
        int64_t rows = r1 - r0;
        if (rows <= 0) return 0;
        if (threads < 1) threads = 1;
        if (threads > rows) threads = (int)rows;
        std::vector<Tensor<float>> outs((size_t)threads);
        std::vector<std::thread> pool;
        auto t0 = std::chrono::steady_clock::now();
        for (int t = 0; t < threads; ++t) {
            size_t s = (size_t)(r0 + rows * t / threads), e = (size_t)(r0 + rows * (t + 1) / threads);
            outs[(size_t)t] = Tensor<float>({e - s, (size_t)N});
            pool.emplace_back([&, t, s, e] {
                Tensor<float> as = a.slice(0, s, e);
                matmul_cpu(as, b, outs[(size_t)t]);
            });
        }
        for (auto& th : pool) th.join();
        if (seconds) *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        size_t row = 0;
        for (int t = 0; t < threads; ++t) {
            to_host(outs[(size_t)t], C + row * (size_t)N);
            row += outs[(size_t)t].shape()[0];
        }
        return 0;
    } catch (const std::exception&) { return 1; }
}

// The first n draws of std::normal_distribution<float>(mean, stddev) on std::mt19937(seed),
// filled in order as the reference fills its weights (include/Module.hpp:99-105, :226-232).
// Pins the synthetic-input generator to this C++ standard library.
int ref_normal(uint32_t seed, float mean, float stddev, float* out, int64_t n) {
    std::mt19937 gen(seed);
    std::normal_distribution<float> dist(mean, stddev);
    for (int64_t i = 0; i < n; ++i) out[i] = dist(gen);
    return 0;
}

// The weights of the FIRST Conv2D<float> this process constructs (include/Module.hpp:
// 199-233: its static init_seed starts at 42 and counts up per instance). Built once and
// cached, so every call returns that first instance's weights, which must have the
// requested shape.
int ref_conv2d_first_weight(int64_t out_ch, int64_t in_ch, int64_t k, float* out) {
    try {
        static std::unique_ptr<Conv2D<float>> first;
        static int64_t shape[3];
        if (!first) {
            first = std::make_unique<Conv2D<float>>((size_t)in_ch, (size_t)out_ch, (size_t)k, 1, 0, false);
            shape[0] = out_ch; shape[1] = in_ch; shape[2] = k;
        }
        if (shape[0] != out_ch || shape[1] != in_ch || shape[2] != k) return 2;
        to_host(first->weight_, out);
        return 0;
    } catch (const std::exception&) { return 1; }
}

}  // extern "C"
