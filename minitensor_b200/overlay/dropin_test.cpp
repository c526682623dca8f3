// dropin_test.cpp -- the reference's own code paths on CUDA tensors, served by
// libmtgemm.so through gpu_ops_b200.cpp. Built against the reference headers
// (unmodified) and the reference's src/gpu_ops.cpp minus the symbols the overlay defines;
// prints one line per check and exits non-zero on any failure.
//
// Each check also reads mt_launch_count() to prove the work ran on this library's kernels.
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "Dispatch.hpp"
#include "GraphExecutor.hpp"
#include "Loss.hpp"
#include "Module.hpp"
#include "Optimizer.hpp"
#include "Tensor.hpp"
#include "TensorOps.hpp"
#include "mtgemm.h"

Tensor<float> mt_bmm(const Tensor<float>& A, const Tensor<float>& B);

namespace {

int failures = 0;
const Device kCpu{DeviceType::CPU};
const Device kGpu{DeviceType::CUDA, 0};

void report(const char* name, bool ok, double err) {
    std::printf("%-48s %s  (max err %.3e)\n", name, ok ? "PASS" : "FAIL", err);
    if (!ok) ++failures;
}

Tensor<float> filled(std::vector<size_t> shape, unsigned seed, float lo = -1.f, float hi = 1.f) {
    Tensor<float> t(shape, kCpu);
    std::mt19937 g(seed);
    std::uniform_real_distribution<float> d(lo, hi);
    for (size_t i = 0; i < t.total_elements(); ++i) t.data()[i] = d(g);
    return t;
}

// max |a - b| / (atol + rtol |b|) over elements in logical (row-major) order.
double compare(const Tensor<float>& gpu, const Tensor<float>& cpu, double rtol, double atol, bool* ok) {
    Tensor<float> g = gpu.to(kCpu).contiguous();
    Tensor<float> c = cpu.contiguous();
    double worst = 0;
    *ok = g.total_elements() == c.total_elements();
    for (size_t i = 0; *ok && i < g.total_elements(); ++i) {
        const double a = g.data()[g.offset() + i], b = c.data()[c.offset() + i];
        const double r = std::fabs(a - b) / (atol + rtol * std::fabs(b));
        if (!(r <= 1.0)) *ok = false;
        if (r > worst || std::isnan(r)) worst = std::isnan(r) ? 1e30 : r;
    }
    return worst;
}

}  // namespace

int main() {
    mt_set_default_mode(MT_TF32X3);

    {   // test/tensor_test.cpp:285-317 GpuMatmul known answer, via matmul() -> matmul_gpu.
        Tensor<float> A({2, 3}, kCpu), B({3, 2}, kCpu);
        for (int i = 0; i < 6; ++i) { A.data()[i] = float(i + 1); B.data()[i] = float(i + 7); }
        const uint64_t n0 = mt_launch_count();
        Tensor<float> C = matmul(A.to(kGpu), B.to(kGpu)).to(kCpu);
        const bool ok = C.data()[0] == 58.f && C.data()[1] == 64.f && C.data()[2] == 139.f && C.data()[3] == 154.f &&
                        mt_launch_count() > n0;
        report("matmul known answer (tensor_test.cpp:285)", ok, 0.0);
    }
    {   // test/tensor_test.cpp:490-510 GPUGradients: backward through transposed views.
        Tensor<float> A({2, 3}, kGpu), B({3, 2}, kGpu);
        A.fill(2.0f);
        B.fill(3.0f);
        A.set_requires_grad(true);
        B.set_requires_grad(true);
        Tensor<float> C = matmul(A, B);
        C.backward();
        const float da = A.grad().to(kCpu).data()[0], db = B.grad().to(kCpu).data()[0];
        report("autograd GPUGradients dA=6 dB=4 (tensor_test.cpp:490)", da == 6.f && db == 4.f, 0.0);
    }
    {   // Random contiguous, transposed and row-sliced matmul vs the reference CPU path.
        Tensor<float> A = filled({300, 200}, 1), B = filled({200, 260}, 2);
        bool ok;
        double e = compare(matmul(A.to(kGpu), B.to(kGpu)), matmul(A, B), 1e-4, 1e-4, &ok);
        report("matmul 300x200x260", ok, e);
        Tensor<float> At = filled({200, 300}, 3), Bt = filled({260, 200}, 4);
        e = compare(matmul(At.to(kGpu).transpose(0, 1), Bt.to(kGpu).transpose(0, 1)),
                    matmul(At.transpose(0, 1), Bt.transpose(0, 1)), 1e-4, 1e-4, &ok);
        report("matmul on transposed views (strided)", ok, e);
        Tensor<float> As = filled({64, 128}, 5);
        e = compare(matmul(As.to(kGpu).slice(0, 8, 40), B.to(kGpu).slice(0, 72, 200)),
                    matmul(As.slice(0, 8, 40), B.slice(0, 72, 200)), 1e-4, 1e-4, &ok);
        report("matmul on offset views (slices)", ok, e);
    }
    {   // Linear<float> forward + backward on the GPU vs the same module on the CPU.
        Linear<float> cpu(96, 80);
        Linear<float> gpu(96, 80);
        std::copy(cpu.weight_.data(), cpu.weight_.data() + 96 * 80, gpu.weight_.data());
        Tensor<float> bias = filled({1, 80}, 6, -0.1f, 0.1f);
        std::copy(bias.data(), bias.data() + 80, cpu.bias_.data());
        std::copy(bias.data(), bias.data() + 80, gpu.bias_.data());
        gpu.to(kGpu);
        Tensor<float> x = filled({48, 96}, 7);
        Tensor<float> xg = x.to(kGpu);
        x.set_requires_grad(true);
        xg.set_requires_grad(true);
        Tensor<float> yc = cpu.forward(x), yg = gpu.forward(xg);
        bool ok;
        double e = compare(yg, yc, 1e-4, 1e-4, &ok);
        report("Linear forward", ok, e);
        yc.backward();
        yg.backward();
        e = compare(xg.grad(), x.grad(), 1e-4, 1e-4, &ok);
        report("Linear backward dX (dY . W^T)", ok, e);
        e = compare(gpu.weight_.grad(), cpu.weight_.grad(), 1e-4, 1e-4, &ok);
        report("Linear backward dW (X^T . dY)", ok, e);
    }
    {   // test/spatial_test.cpp:209-230 conv device equivalence (stride 2, pad 1).
        Tensor<float> in({4, 3, 32, 32}, kCpu), w({16, 3, 3, 3}, kCpu), b({16}, kCpu);
        for (size_t i = 0; i < in.total_elements(); ++i) in.data()[i] = 0.1f + i * 0.01f;
        for (size_t i = 0; i < w.total_elements(); ++i) w.data()[i] = -0.5f + i * 0.02f;
        b.fill(0.1f);
        bool ok;
        double e = compare(conv2d(in.to(kGpu), w.to(kGpu), b.to(kGpu), 2, 1), conv2d(in, w, b, 2, 1), 1e-3, 1e-4, &ok);
        report("conv2d device equivalence (spatial_test.cpp:209)", ok, e);
    }
    {   // Conv2D module forward + Conv2DBackward (input, weight, bias grads) GPU vs CPU.
        Tensor<float> x = filled({2, 8, 12, 12}, 8), w = filled({16, 8, 3, 3}, 9, -0.3f, 0.3f),
                      b = filled({16}, 10, -0.1f, 0.1f);
        Tensor<float> xg = x.to(kGpu), wg = w.to(kGpu), bg = b.to(kGpu);
        for (Tensor<float>* t : {&x, &w, &b, &xg, &wg, &bg}) t->set_requires_grad(true);
        Tensor<float> yc = conv2d(x, w, b, 1, 1), yg = conv2d(xg, wg, bg, 1, 1);
        Tensor<float> gc = filled(yc.shape(), 11);
        Tensor<float> gg = gc.to(kGpu);
        yc.grad_fn()->apply(gc);
        yg.grad_fn()->apply(gg);
        bool ok;
        double e = compare(yg, yc, 1e-4, 1e-4, &ok);
        report("conv2d forward (Conv2D layer shape)", ok, e);
        e = compare(xg.grad(), x.grad(), 1e-4, 1e-4, &ok);
        report("conv2d backward input", ok, e);
        e = compare(wg.grad(), w.grad(), 1e-4, 1e-3, &ok);
        report("conv2d backward weight", ok, e);
        e = compare(bg.grad(), b.grad(), 1e-4, 1e-3, &ok);
        report("conv2d backward bias", ok, e);
    }
    {   // Broadcast bmm: one launch, expanded operand read in place.
        Tensor<float> A = filled({6, 40, 24}, 12), B0 = filled({1, 24, 56}, 13);
        Tensor<float> Cg = mt_bmm(A.to(kGpu), B0.to(kGpu).expand({6, 24, 56})).to(kCpu);
        double worst = 0;
        bool ok = true;
        for (size_t bi = 0; bi < 6; ++bi) {
            Tensor<float> a2 = A.slice(0, bi, bi + 1).reshape({40, 24});
            Tensor<float> c2({40, 56}, kCpu);
            matmul_cpu(a2, B0.reshape({24, 56}), c2);
            for (size_t i = 0; i < 40 * 56; ++i) {
                const double r = std::fabs(Cg.data()[bi * 40 * 56 + i] - c2.data()[i]) / (1e-4 + 1e-4 * std::fabs(c2.data()[i]));
                worst = std::max(worst, r);
                ok = ok && r <= 1.0;
            }
        }
        report("bmm with expand (stride-0) operand", ok, worst);
    }
    {   // OpRegistry<float> slot (include/Dispatch.hpp) now holds the engine.
        Tensor<float> A = filled({33, 17}, 14), B = filled({17, 29}, 15);
        Tensor<float> C({33, 29}, kGpu);
        dispatch_binary_op(OpType::Matmul, A.to(kGpu), B.to(kGpu), C);
        bool ok;
        double e = compare(C, matmul(A, B), 1e-4, 1e-4, &ok);
        report("OpRegistry<float> Matmul dispatch", ok, e);
    }
    {   // include/GraphExecutor.hpp: warm-up, capture (Relaxed, on active_stream()) and replay
        // of a whole training step; the captured GEMMs are this library's kernels. Compared
        // step by step with eager training of an identical model. The first layer's forward
        // (32 x 1024 . 1024 x 128: one output tile, a long K) runs split-K, whose partials are
        // scratch; with the overlay's MemoryPool allocator installed, no stream-ordered
        // allocation may happen anywhere in the step, so the captured graph holds none.
        uint64_t async0 = 0, pool0 = 0;
        mt_scratch_counts(&async0, &pool0);
        auto make = [] {
            return std::make_shared<Sequential<float>>(std::initializer_list<std::shared_ptr<Module<float>>>{
                std::make_shared<Linear<float>>(1024, 128), std::make_shared<ReLU<float>>(),
                std::make_shared<Linear<float>>(128, 16)});
        };
        auto eager = make();
        auto graphed = make();
        auto pe = eager->parameters(), pg = graphed->parameters();
        for (size_t i = 0; i < pe.size(); ++i)
            std::copy(pe[i].data(), pe[i].data() + pe[i].total_elements(), pg[i].data());
        eager->to(kGpu);
        graphed->to(kGpu);
        SGD<float> opt_e(eager->parameters(), 0.05f), opt_g(graphed->parameters(), 0.05f);
        GraphExecutor<float> exec(graphed, opt_g,
                                  [](const Tensor<float>& p, const Tensor<float>& t) { return mse_loss(p, t); });
        Tensor<float> x = filled({32, 1024}, 16).to(kGpu), y = filled({32, 16}, 17).to(kGpu);
        bool ok = true;
        double worst = 0;
        for (int step = 0; step < 4; ++step) {
            opt_e.zero_grad();
            Tensor<float> le = mse_loss(eager->forward(x), y);
            le.backward();
            opt_e.step();
            Tensor<float> lg = exec.step(x, y);
            const double a = le.to(kCpu).data()[0], b = lg.to(kCpu).data()[0];
            const double r = std::fabs(a - b) / (1e-5 + 1e-4 * std::fabs(a));
            worst = std::max(worst, r);
            ok = ok && r <= 1.0;
        }
        auto fe = eager->parameters(), fg = graphed->parameters();
        for (size_t i = 0; i < fe.size(); ++i) {
            bool pok;
            worst = std::max(worst, compare(fg[i], fe[i].to(kCpu), 1e-4, 1e-5, &pok));
            ok = ok && pok;
        }
        report("GraphExecutor capture/replay of a training step", ok, worst);
        uint64_t async1 = 0, pool1 = 0;
        mt_scratch_counts(&async1, &pool1);
        std::printf("scratch during the step: %llu from MemoryPool, %llu stream-ordered (total stream-ordered %llu)\n",
                    (unsigned long long)(pool1 - pool0), (unsigned long long)(async1 - async0),
                    (unsigned long long)async1);
        report("step scratch from MemoryPool, no stream-ordered allocation", pool1 > pool0 && async1 == 0, 0.0);
    }
    std::printf("%s: %d failure(s)\n", failures ? "FAILED" : "ALL PASSED", failures);
    return failures ? 1 : 0;
}
